"""Resource preparation on CPU: a fake two-shard dataset, a pinned-manifest check, an existing CORE
bundle and a tiny tokenizer trained by the C++ merge learner."""
import json

import pytest


def _dataset(tmp_path):
    import pyarrow as pa
    import pyarrow.parquet as pq
    from nexttransformer_b200.runtime.files import DATA_REPO, DATA_REVISION, VALIDATION_SHARD, sha256
    data = tmp_path / "data"
    data.mkdir()
    docs = ["the quick brown fox jumps over the lazy dog %d" % i for i in range(200)]
    pq.write_table(pa.table({"text": docs}), data / "shard_00000.parquet")
    pq.write_table(pa.table({"text": docs[:20]}), data / VALIDATION_SHARD)
    files = [{"rfilename": p.name, "size": p.stat().st_size, "lfs": {"sha256": sha256(p)}}
             for p in sorted(data.glob("*.parquet"))]
    manifest = tmp_path / "manifest.json"
    manifest.write_text(json.dumps({"repo": DATA_REPO, "revision": DATA_REVISION, "files": files}))
    return data, manifest


def _core(tmp_path):
    from nexttransformer_b200.runtime.files import CORE_SHA256, sha256
    core = tmp_path / "core"
    (core / "eval_bundle").mkdir(parents=True)
    (core / "eval_bundle" / "core.yaml").write_text("icl_tasks: []\n")
    pin = {"archive_sha256": CORE_SHA256, "entries": 22,
           "files": {"core.yaml": sha256(core / "eval_bundle" / "core.yaml")}}
    (core / "core_manifest.json").write_text(json.dumps(pin))
    return core


def test_prepare_end_to_end(tmp_path):
    from nexttransformer_b200 import prepare
    from nexttransformer_b200.runtime import resources as res
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    data, manifest = _dataset(tmp_path)
    core = _core(tmp_path)
    out = tmp_path / "resources"
    rec = prepare.main(["--data-dir", str(data), "--resources", str(out), "--source-manifest", str(manifest),
                        "--existing-core-resources", str(core), "--vocab-size", "300", "--max-chars", "5000"])
    tok = BPETokenizer.from_directory(str(out / "tokenizer"))
    assert tok.get_vocab_size() == 300
    assert tok.decode(tok.encode("the lazy dog")) == "the lazy dog"
    assert res.verify_resources(out)[0]["tokenizer_sha256"] == rec["tokenizer_sha256"]
    # a second run reuses the tokenizer and yields the same manifest
    assert prepare.main(["--data-dir", str(data), "--resources", str(out), "--source-manifest", str(manifest),
                         "--existing-core-resources", str(core), "--vocab-size", "300"]) == rec


def test_prepare_rejects_changed_dataset(tmp_path):
    from nexttransformer_b200 import prepare
    data, manifest = _dataset(tmp_path)
    core = _core(tmp_path)
    (data / "shard_00000.parquet").write_bytes(b"corrupted")
    with pytest.raises(ValueError, match="differ"):
        prepare.main(["--data-dir", str(data), "--resources", str(tmp_path / "r"), "--source-manifest",
                      str(manifest), "--existing-core-resources", str(core), "--vocab-size", "300"])


def test_core_digest_mismatch_is_refused(tmp_path):
    from nexttransformer_b200.runtime import resources as res
    core = _core(tmp_path)
    (core / "eval_bundle" / "core.yaml").write_text("tampered\n")
    with pytest.raises(ValueError, match="checksum"):
        res.verify_core(core)


def test_integration_check_on_prepared_resources(tmp_path):
    from nexttransformer_b200 import prepare
    from nexttransformer_b200.checks import integration
    data, manifest = _dataset(tmp_path)
    core = _core(tmp_path)
    out = tmp_path / "resources"
    prepare.main(["--data-dir", str(data), "--resources", str(out), "--source-manifest", str(manifest),
                  "--existing-core-resources", str(core), "--vocab-size", "300", "--max-chars", "5000"])
    bundle = tmp_path / "bundle"
    bundle.mkdir()
    (bundle / "tasks.json").write_text(json.dumps([{"label": "lm", "random_baseline": 0.0,
                                                    "meta": {"task_type": "language_modeling", "num_fewshot": 0}}]))
    items = [{"context": "the quick brown", "continuation": " fox"} for _ in range(12)]
    (bundle / "lm.jsonl").write_text("".join(json.dumps(i) + "\n" for i in items))
    res = integration.main(["--data-dir", str(data), "--resources", str(out), "--output", str(tmp_path / "o.json"),
                            "--device", "cpu", "--sequence-len", "32", "--core", str(bundle),
                            "--core-methods", "dense", "--core-max-per-task", "11"])
    assert res["status"] == "passed" and res["bpb_exact"] and len(res["core_smoke"]) == 1
    assert json.loads((tmp_path / "o.json").read_text())["status"] == "passed"
