"""Machine configuration: paths and values resolved as CLI > --site-config JSON > environment > default.

Resolution happens before torch is imported by the entry points (cache directories and thread
counts must be in the environment first), as in the reference's ``runtime/site.py``.

``python -m nexttransformer_b200.runtime.site --shell [options]`` prints the resolved settings as
shell ``export`` lines (``launch/env.sh`` evaluates them); the site JSON is read as data, and every
value is shell-quoted, so nothing from it is executed.
"""
import argparse
import json
import os
import shlex
import sys
from pathlib import Path

HOME = Path(os.environ.get("NEXTTRANSFORMER_HOME", Path.home() / ".cache" / "nexttransformer_b200"))
PATHS = {  # name: (environment variable, default)
    "runtime_dir": ("NEXTTRANSFORMER_RUNTIME", HOME),
    "resources": ("NEXTTRANSFORMER_RESOURCES", HOME / "resources"),
    "data_dir": ("NEXTTRANSFORMER_DATA", None),
    "cache_dir": ("NEXTTRANSFORMER_CACHE", HOME / "cache"),
}
VALUES = {
    "micro_batch": ("NEXTTRANSFORMER_MICRO_BATCH", None, int),
    "wandb_mode": ("WANDB_MODE", "disabled", str),
    "omp_threads": ("OMP_NUM_THREADS", "8", str),
    "run_name": ("NEXTTRANSFORMER_RUN_NAME", None, str),
}


def add_runtime_arguments(parser: argparse.ArgumentParser):
    parser.add_argument("--site-config", type=Path, help="JSON file with machine paths/values")
    for name in PATHS:
        parser.add_argument("--" + name.replace("_", "-"), dest=name, type=Path, default=None)
    for name, (_, _, kind) in VALUES.items():
        parser.add_argument("--" + name.replace("_", "-"), dest=name, type=kind, default=None)
    return parser


def resolve(args):
    """Fill every path/value of `args` by precedence; returns the resolved dict."""
    site = {}
    if getattr(args, "site_config", None):
        site = json.loads(Path(args.site_config).read_text())
    out = {}
    for name, (env, default) in PATHS.items():
        v = getattr(args, name, None) or site.get(name) or os.environ.get(env) or default
        out[name] = Path(v) if v is not None else None
    for name, (env, default, kind) in VALUES.items():
        v = getattr(args, name, None)
        if v is None:
            v = site.get(name, os.environ.get(env, default))
        out[name] = kind(v) if v is not None else None
    for k, v in out.items():
        setattr(args, k, v)
    return out


def bootstrap_runtime(argv=None):
    """Export cache locations and thread counts before torch is imported."""
    parser = add_runtime_arguments(argparse.ArgumentParser(add_help=False))
    args, _ = parser.parse_known_args(argv)
    r = resolve(args)
    os.environ.setdefault("OMP_NUM_THREADS", str(r["omp_threads"]))
    if r["cache_dir"] is not None:
        Path(r["cache_dir"]).mkdir(parents=True, exist_ok=True)
    return r


def shell_exports(argv=None):
    """``export VAR=value`` lines of every resolved setting (None values are skipped)."""
    parser = add_runtime_arguments(argparse.ArgumentParser(add_help=False))
    args, _ = parser.parse_known_args(argv)
    r = resolve(args)
    lines = []
    for name, (env, _) in PATHS.items():
        if r[name] is not None:
            lines.append(f"export {env}={shlex.quote(str(r[name]))}")
    for name, (env, _, _) in VALUES.items():
        if r[name] is not None:
            lines.append(f"export {env}={shlex.quote(str(r[name]))}")
    return "\n".join(lines)


if __name__ == "__main__":
    argv = sys.argv[1:]
    if "--shell" not in argv:
        raise SystemExit("usage: python -m nexttransformer_b200.runtime.site --shell [--site-config F] [--runtime-dir D] ...")
    print(shell_exports([a for a in argv if a != "--shell"]))
