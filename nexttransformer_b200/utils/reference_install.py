"""Offline install of the unmodified reference implementation under ``baseline/_ref``.

The reference (NextTransformer: the ``nexttransformer`` and ``nanochat`` packages) is the CPU
oracle of the parity tests and the comparison arm of ``bench.py --impl reference``.  It is never
committed; it is installed from the reference's source tree with pip, offline:

* the source tree is copied to a temporary directory, because the reference is read-only and a
  build writes next to its sources;
* the copy's build backend (hatchling, which the offline wheelhouse does not carry) is switched
  to setuptools with the same two packages and every data file (``method.json``, README files,
  ``core-lengths.json``) included, which is what hatchling's wheel would contain;
* ``pip install --no-index --no-build-isolation --no-deps --target baseline/_ref`` installs the
  packages without touching any source file.

The source tree is taken from ``NT_REFERENCE_SRC`` or else from ``reference_path`` in the
benchmark specification ``BASELINE.json`` at the repository root.
"""
import json
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
TARGET = ROOT / "baseline" / "_ref"
PACKAGES = ("nexttransformer", "nanochat")


def installed(target=TARGET):
    """True when both reference packages are importable from ``target``."""
    return all((Path(target) / p / "__init__.py").is_file() for p in PACKAGES)


def source_tree():
    """The reference source tree to install from, or None when none is known or present."""
    src = os.environ.get("NT_REFERENCE_SRC")
    if not src:
        spec = ROOT / "BASELINE.json"
        if spec.is_file():
            try:
                src = json.loads(spec.read_text()).get("reference_path")
            except (OSError, ValueError):
                src = None
    if src and all((Path(src) / p).is_dir() for p in PACKAGES) and (Path(src) / "pyproject.toml").is_file():
        return Path(src)
    return None


def _setuptools_pyproject(text):
    """Switch a hatchling pyproject to setuptools with the same packages and all package data."""
    lines, out, skip = text.splitlines(), [], False
    for line in lines:
        s = line.strip()
        if s.startswith("[") and s.endswith("]"):
            skip = s in ("[build-system]", "[tool.hatch.build.targets.wheel]")
        if not skip:
            out.append(line)
    head = ['[build-system]', 'requires = ["setuptools"]', 'build-backend = "setuptools.build_meta"', '']
    tail = ['', '[tool.setuptools]', 'include-package-data = true', '',
            '[tool.setuptools.packages.find]', 'include = [' + ", ".join(f'"{p}*"' for p in PACKAGES) + ']', '',
            '[tool.setuptools.package-data]', '"*" = ["*", "**/*"]']
    return "\n".join(head + out + tail) + "\n"


def install(src=None, target=TARGET, wheelhouse="/opt/wheelhouse"):
    """Install the reference from ``src`` into ``target``; returns the target path.

    Raises RuntimeError when no source tree is available or pip fails."""
    src = Path(src) if src else source_tree()
    if src is None:
        raise RuntimeError("no reference source tree (set NT_REFERENCE_SRC or BASELINE.json reference_path)")
    target = Path(target)
    with tempfile.TemporaryDirectory(prefix="nt_ref_") as tmp:
        copy = Path(tmp) / "src"
        copy.mkdir()
        for p in PACKAGES:
            shutil.copytree(src / p, copy / p, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
        for f in ("README.md", "LICENSE"):
            if (src / f).is_file():
                shutil.copy2(src / f, copy / f)
        (copy / "pyproject.toml").write_text(_setuptools_pyproject((src / "pyproject.toml").read_text()))
        if target.exists():
            shutil.rmtree(target)
        target.parent.mkdir(parents=True, exist_ok=True)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", wheelhouse, "--target", str(target), str(copy)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0 or not installed(target):
            raise RuntimeError(f"reference install failed (rc {res.returncode}): {res.stderr.strip()[-400:]}")
    return target


def ensure(target=TARGET):
    """The install path, installing first when it is missing and a source tree is available.

    Returns None when the reference is neither installed nor installable here."""
    import fcntl
    if installed(target):
        return Path(target)
    if source_tree() is None:
        return None
    Path(target).parent.mkdir(parents=True, exist_ok=True)
    # concurrent callers (parallel test workers) install once: the others wait on the lock
    with open(Path(target).parent / ".install.lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if installed(target):
            return Path(target)
        return install(target=target)


if __name__ == "__main__":
    path = install() if "--force" in sys.argv[1:] else ensure()
    print(path if path else "reference unavailable")
