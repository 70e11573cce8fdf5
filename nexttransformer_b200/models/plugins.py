"""Plugin methods: one directory per method, discovered from its ``method.json``.

The declaration format is the reference's (``nexttransformer/models/plugins.py:1-27``) so that
a contributed method can be dropped into either tree: ``name``, ``family``, ``title``, ``paper``,
``options`` / ``debug_options`` (JSON scalars or lists), ``shell`` (``layers``, ``mlp_width``,
``window_pattern``) and ``layer_multiple``.  Roots are this package's ``methods/`` directory and
every directory listed in ``NEXTTRANSFORMER_METHOD_PATHS``.

A plugin package may define the hooks ``mixer(config, layer)``, ``ffn(config, layer)``,
``block(block, config, layer)``, ``model`` (a ``LanguageModel`` subclass), ``frozen`` (shell
parameter names the method leaves unused), ``init(model)``, ``stages(config)`` and
``check(config)``.
"""
from functools import lru_cache
import importlib
import importlib.util
import json
import os
from pathlib import Path
import re
import sys
from types import SimpleNamespace

BUILTIN_ROOT = Path(__file__).resolve().parents[1] / "methods"
PLUGIN_FAMILIES = ("looped", "sparse", "linear", "residual", "hybrid", "others")
HOOK_NAMES = ("mixer", "ffn", "block", "model", "frozen", "init", "stages", "check")
SHELL_KEYS = ("layers", "mlp_width", "window_pattern")
_IDENT = re.compile(r"[a-z][a-z0-9_]{1,40}")


def plugin_roots():
    extra = os.environ.get("NEXTTRANSFORMER_METHOD_PATHS", "")
    return [BUILTIN_ROOT] + [Path(p).resolve() for p in extra.split(os.pathsep) if p]


def _json_value(v):
    if isinstance(v, (str, int, float, bool)):
        return True
    return isinstance(v, list) and all(_json_value(x) for x in v)


def _problems(path, spec, taken):
    name = spec.get("name")
    opts = spec.get("options", {})
    mult = spec.get("layer_multiple", 1)
    checks = [
        (isinstance(name, str) and bool(_IDENT.fullmatch(name)), "name: lowercase letters, digits and _"),
        (name == path.parent.name, "name must equal its directory"),
        (name not in taken, "name is already registered"),
        (spec.get("family") in PLUGIN_FAMILIES, "family must be one of " + ", ".join(PLUGIN_FAMILIES)),
        (isinstance(opts, dict) and all(_IDENT.fullmatch(k) and _json_value(v) for k, v in opts.items()),
         "options map lowercase names to JSON scalars or lists"),
        (set(spec.get("debug_options", {})) <= set(opts), "debug_options may only set declared options"),
        (set(spec.get("shell", {})) <= set(SHELL_KEYS), "shell may set only " + ", ".join(SHELL_KEYS)),
        (isinstance(mult, int) and mult > 0, "layer_multiple must be a positive integer"),
        ((path.parent / "__init__.py").is_file(), "the method directory needs an __init__.py"),
    ]
    return [msg for good, msg in checks if not good]


def discover(reserved):
    """name -> declaration (plus ``path``) of every plugin, without importing plugin code."""
    found = {}
    for root in plugin_roots():
        for path in sorted(root.glob("*/method.json")):
            spec = json.loads(path.read_text())
            bad = _problems(path, spec, set(reserved) | set(found))
            if bad:
                raise ValueError(f"plugin {path.parent}: " + "; ".join(bad))
            found[spec["name"]] = {**spec, "path": str(path.parent)}
    return found


@lru_cache(maxsize=None)
def load(name):
    """Import a plugin once and return its hooks."""
    from nexttransformer_b200.models.registry import PLUGINS
    spec = PLUGINS[name]
    where = Path(spec["path"])
    if where.parent == BUILTIN_ROOT:
        module = importlib.import_module(f"nexttransformer_b200.methods.{name}")
    else:
        modname = f"nexttransformer_b200_plugin_{name}"
        found = importlib.util.spec_from_file_location(modname, where / "__init__.py",
                                                       submodule_search_locations=[str(where)])
        module = importlib.util.module_from_spec(found)
        sys.modules[modname] = module
        found.loader.exec_module(module)
    hooks = SimpleNamespace(spec=spec, **{h: getattr(module, h, None) for h in HOOK_NAMES})
    if not (hooks.mixer or hooks.ffn or hooks.block or hooks.model):
        raise ValueError(f"plugin {name} defines none of mixer, ffn, block or model")
    if hooks.model is not None:
        from nexttransformer_b200.models.lm import LanguageModel
        if not (isinstance(hooks.model, type) and issubclass(hooks.model, LanguageModel)):
            raise ValueError(f"plugin {name}: model must subclass LanguageModel")
    return hooks


def stages(config, total_steps=None):
    """[(stage name, updates)] of a plugin method in training order; one "joint" stage by default."""
    from nexttransformer_b200.protocol.spec import Protocol
    steps = total_steps or Protocol().steps
    hook = load(config.method).stages
    out = [tuple(s) for s in hook(config)] if hook else [("joint", steps)]
    names = [s[0] for s in out]
    valid = (len(set(names)) == len(names)
             and all(len(s) == 2 and isinstance(s[0], str) and isinstance(s[1], int) and s[1] > 0 for s in out)
             and sum(s[1] for s in out) == steps)
    if not valid:
        raise ValueError(f"{config.method}: stages must be distinct names with positive steps summing to {steps}")
    return out


def stage_at(config, step):
    start = 0
    for name, count in stages(config):
        if step < start + count:
            return name, start
        start += count
    raise ValueError("update outside the training schedule")


def check_shell(model):
    """Every block keeps the shell's linear layers (the shell initializes them)."""
    from torch import nn
    for i, block in enumerate(model.transformer.h):
        for part, names in (("attn", ("c_q", "c_k", "c_v", "c_proj")), ("mlp", ("c_fc", "c_proj"))):
            mod = getattr(block, part, None)
            if mod is None or not all(isinstance(getattr(mod, n, None), nn.Linear) for n in names):
                raise ValueError(f"{model.config.method}: block {i} needs {part}.{'/'.join(names)} linear layers")


def reset(model):
    """Call reset_parameters on plugin modules (``to_empty`` leaves their tensors unset)."""
    from torch import nn
    for m in model.modules():
        if not isinstance(m, (nn.Linear, nn.LayerNorm)) and callable(getattr(m, "reset_parameters", None)):
            m.reset_parameters()
