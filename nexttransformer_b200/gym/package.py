"""Candidate packages: a base64 ZIP holding one source-only method plugin and its proposal.

Validation reads the archive without extracting it first: sizes and file counts are bounded,
names must be plain relative paths inside the allowed layout, symlinks and non-UTF-8 content are
refused, ``method.json`` passes the plugin declaration rules and names its own directory, and the
Python sources must compile.  A candidate's id is the sha256 of its canonical content (sorted
names and bytes), so resubmitting the same files gives the same candidate.
"""
import base64
import binascii
import hashlib
import io
import json
import re
import stat
import zipfile
from pathlib import Path, PurePosixPath

from nexttransformer_b200.gym.contract import PACKAGE_CONTRACT, GymError

LIMITS = PACKAGE_CONTRACT["limits"]
_NAME = re.compile(r"[a-z][a-z0-9_]{1,40}")
_FAMILIES = ("looped", "sparse", "linear", "residual", "hybrid", "others")
_FILE = re.compile(r"[A-Za-z0-9_][A-Za-z0-9_.-]{0,63}")


def _refuse(message):
    raise GymError("invalid_package", message)


def read_package(package_b64):
    """{path: bytes} of a package after every structural check."""
    try:
        raw = base64.b64decode(package_b64, validate=True)
    except (binascii.Error, ValueError):
        _refuse("package is not valid base64")
    if len(raw) > LIMITS["compressed_bytes"]:
        _refuse(f"package exceeds {LIMITS['compressed_bytes']} bytes")
    try:
        zf = zipfile.ZipFile(io.BytesIO(raw))
    except zipfile.BadZipFile:
        _refuse("package is not a ZIP archive")
    infos = [i for i in zf.infolist() if not i.is_dir()]
    if len(infos) > LIMITS["files"]:
        _refuse(f"more than {LIMITS['files']} files")
    total, files = 0, {}
    for info in infos:
        mode = info.external_attr >> 16
        if stat.S_ISLNK(mode):
            _refuse(f"{info.filename}: symlinks are not allowed")
        path = PurePosixPath(info.filename)
        if path.is_absolute() or ".." in path.parts or "\\" in info.filename:
            _refuse(f"{info.filename}: only plain relative paths are allowed")
        total += info.file_size
        if total > LIMITS["uncompressed_bytes"]:
            _refuse(f"package expands beyond {LIMITS['uncompressed_bytes']} bytes")
        data = zf.read(info)
        try:
            data.decode("utf-8")
        except UnicodeDecodeError:
            _refuse(f"{info.filename}: only UTF-8 source files are allowed")
        files[str(path)] = data
    return files


def candidate_from_package(package_b64):
    """(candidate id, method name, proposal, files) of a valid package."""
    files = read_package(package_b64)
    if "proposal.json" not in files:
        _refuse("proposal.json is missing")
    methods = {PurePosixPath(p).parts[1] for p in files if PurePosixPath(p).parts[0] == "plugin"
               and len(PurePosixPath(p).parts) == 3}
    if len(methods) != 1:
        _refuse("the package must hold exactly one plugin/<method>/ directory")
    method = methods.pop()
    for p in files:
        parts = PurePosixPath(p).parts
        allowed = p == "proposal.json" or (len(parts) == 3 and parts[0] == "plugin" and parts[1] == method
                                            and _FILE.fullmatch(parts[2])
                                            and (parts[2] == "method.json" or parts[2].endswith(".py")))
        if not allowed:
            _refuse(f"{p}: not part of the package layout")
    base = f"plugin/{method}/"
    for need in ("method.json", "__init__.py"):
        if base + need not in files:
            _refuse(f"{base}{need} is missing")
    try:
        proposal = json.loads(files["proposal.json"])
        spec = json.loads(files[base + "method.json"])
    except json.JSONDecodeError as e:
        _refuse(f"invalid JSON: {e}")
    if not (isinstance(proposal, dict) and isinstance(proposal.get("name"), str)
            and isinstance(proposal.get("summary"), str)):
        _refuse("proposal.json needs a name and a summary")
    if not _NAME.fullmatch(method) or spec.get("name") != method:
        _refuse("method.json name must equal its lowercase directory name")
    if spec.get("family") not in _FAMILIES:
        _refuse("method.json family must be one of " + ", ".join(_FAMILIES))
    for p, data in files.items():
        if p.endswith(".py"):
            try:
                compile(data.decode(), p, "exec")
            except SyntaxError as e:
                _refuse(f"{p}: {e.msg} (line {e.lineno})")
    digest = hashlib.sha256()
    for p in sorted(files):
        digest.update(p.encode() + b"\0" + hashlib.sha256(files[p]).digest())
    return "cand_" + digest.hexdigest()[:24], method, proposal, files


def unpack(files, root):
    """Write a validated package under ``root``; returns the plugin root (for the method path)."""
    root = Path(root)
    for p, data in files.items():
        target = root / p
        target.parent.mkdir(parents=True, exist_ok=True)
        target.write_bytes(data)
    return root / "plugin"


def make_package(files):
    """base64 ZIP of {path: text or bytes} (clients and tests)."""
    buf = io.BytesIO()
    with zipfile.ZipFile(buf, "w", zipfile.ZIP_DEFLATED) as zf:
        for p, data in sorted(files.items()):
            zf.writestr(p, data)
    return base64.b64encode(buf.getvalue()).decode()
