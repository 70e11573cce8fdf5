"""Pinned resources: dataset inventory and manifest checks, the CORE bundle, tokenizer provenance.

Behaviour of the reference's ``runtime/resources.py`` / ``runtime/data.py:18-43`` /
``evaluation/metrics.py:31-39``: the dataset directory must hold exactly the parquet files (names
and sizes) of the pinned Hub revision, the validation shard must match its published sha256, the
CORE bundle must match the pinned archive digest and contain 22 task entries, and a prepared
``native_manifest.json`` ties the tokenizer and the data inventory together.  This machine has no
network: the source manifest and the CORE archive are given as local files; fetching them is left
to the caller (``--source-manifest``, ``--core-archive``).
"""
import hashlib
import json
from pathlib import Path
import zipfile

from nexttransformer_b200.runtime.files import CORE_SHA256, DATA_REPO, DATA_REVISION, atomic_json, sha256

CORE_URL = "https://karpathy-public.s3.us-west-2.amazonaws.com/eval_bundle.zip"
CORE_ENTRIES = 22


def data_inventory(data_dir):
    return [(p.name, p.stat().st_size) for p in sorted(Path(data_dir).glob("*.parquet"))]


def inventory_fingerprint(inventory):
    return hashlib.sha256(json.dumps([list(x) for x in inventory], separators=(",", ":")).encode()).hexdigest()


def tokenizer_fingerprint(resources):
    root = Path(resources) / "tokenizer"
    return hashlib.sha256("".join(sha256(root / n) for n in ("tokenizer.pkl", "token_bytes.pt")).encode()).hexdigest()


def load_source_manifest(path):
    """The Hub file listing of the pinned dataset revision (``{"repo", "revision", "files": [...]}``)."""
    official = json.loads(Path(path).read_text())
    if official.get("revision") != DATA_REVISION or official.get("repo", DATA_REPO) != DATA_REPO:
        raise ValueError("unexpected source dataset revision or repository")
    return official


def verify_dataset(data_dir, official, validation_shard):
    expected = sorted((f["rfilename"], f["size"]) for f in official["files"] if f["rfilename"].endswith(".parquet"))
    if data_inventory(data_dir) != [tuple(x) for x in expected]:
        raise ValueError("dataset files/sizes differ from the pinned manifest")
    record = next(f for f in official["files"] if f["rfilename"] == validation_shard)
    if sha256(Path(data_dir) / validation_shard) != record["lfs"]["sha256"]:
        raise ValueError("validation shard checksum differs from the manifest")
    return expected, record["lfs"]["sha256"]


def prepare_core(resources, archive):
    """Unpack and pin the CORE bundle from a local archive (digest-checked; idempotent)."""
    resources = Path(resources)
    bundle = resources / "eval_bundle"
    pin_path = resources / "core_manifest.json"
    if pin_path.exists():
        return verify_core(resources)
    archive = Path(archive)
    if not archive.is_file():
        raise FileNotFoundError(f"CORE archive missing: {archive} (download {CORE_URL})")
    if sha256(archive) != CORE_SHA256:
        raise ValueError("CORE archive sha256 mismatch; use the pinned bundle")
    with zipfile.ZipFile(archive) as z:
        for m in z.infolist():
            if not (resources / m.filename).resolve().is_relative_to(resources.resolve()):
                raise ValueError("unsafe path in the CORE archive")
        z.extractall(resources)
    import yaml
    tasks = yaml.safe_load((bundle / "core.yaml").read_text())["icl_tasks"]
    if len(tasks) != CORE_ENTRIES:
        raise ValueError(f"expected {CORE_ENTRIES} CORE entries, got {len(tasks)}")
    pin = {"url": CORE_URL, "archive_sha256": sha256(archive), "entries": len(tasks),
           "files": {str(p.relative_to(bundle)): sha256(p) for p in sorted(bundle.rglob("*")) if p.is_file()}}
    atomic_json(pin_path, pin)
    return pin


def verify_core(resources):
    resources = Path(resources)
    pin = json.loads((resources / "core_manifest.json").read_text())
    if pin["archive_sha256"] != CORE_SHA256:
        raise ValueError("CORE archive differs from the experiment protocol")
    if pin["entries"] != CORE_ENTRIES:
        raise ValueError(f"CORE must contain {CORE_ENTRIES} entries")
    for name, digest in pin["files"].items():
        if sha256(resources / "eval_bundle" / name) != digest:
            raise ValueError(f"CORE resource checksum mismatch: {name}")
    return pin


def verify_resources(resources, data_dir=None):
    """Check a prepared resource directory against its ``native_manifest.json``."""
    resources = Path(resources)
    record = json.loads((resources / "native_manifest.json").read_text())
    if record["data_revision"] != DATA_REVISION or record["tokenizer_sha256"] != tokenizer_fingerprint(resources):
        raise ValueError("resource provenance mismatch (tokenizer or data revision)")
    data_dir = Path(data_dir) if data_dir is not None else resources / "base_data_climbmix"
    if inventory_fingerprint(data_inventory(data_dir)) != record["data_inventory_sha256"]:
        raise ValueError("dataset inventory differs from the prepared manifest")
    return record, record["data_inventory_sha256"]
