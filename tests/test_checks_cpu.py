"""The verification tools on CPU: validate, golden dump, public scanner, change classifier and the
multi-rank distributed check on gloo ranks."""
import json
import os

import pytest
import torch
import torch.multiprocessing as mp

from tests.conftest import free_port


def test_validate_smoke(tmp_path):
    from nexttransformer_b200.checks import validate
    res = validate.main(["--device", "cpu", "--methods", "dense_full", "gdn", "hc", "xsa", "--output",
                         str(tmp_path / "v.json")])
    assert [r["status"] for r in res] == ["passed"] * 4
    assert json.loads((tmp_path / "v.json").read_text())["results"][0]["causal_max_abs"] <= 3e-3


def test_golden_dump_is_reproducible():
    from nexttransformer_b200.checks import golden
    a = golden.dump(["dense_full", "mhc"])
    b = golden.dump(["dense_full", "mhc"])
    assert a == b and set(a) == {"dense_full", "mhc"}


def test_public_scanner():
    from nexttransformer_b200.checks.public import scan_text
    bad = "token ghp_" + "a" * 36 + " at /home/alice/x and mail bob@corp.io via 192.168.1.4"
    hits = scan_text("f.txt", bad)
    assert len(hits) == 4
    assert scan_text("f.txt", "MASTER_ADDR=127.0.0.1 noreply@example.com") == []


def test_change_classifier():
    from nexttransformer_b200.checks.changes import classify
    r = classify(["nexttransformer_b200/csrc/gemm_sm100.cu", "nexttransformer_b200/models/linear.py"])
    assert r["gpu"] and r["tests"] and "gdn" in r["affected"] and "dense" not in r["affected"]
    assert classify(["profiles/gemm.txt"])["tests"] is False
    assert "xsa" in classify(["nexttransformer_b200/methods/xsa/__init__.py"])["affected"]


def _dist_rank(rank, world, port, out, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="")
    try:
        from nexttransformer_b200.checks import distributed
        res = distributed.main(["--methods", "dense_full", "moba", "--micro-batch", "2", "--sequence-len", "12",
                                "--global-batch", "96", "--smoke", "--output", out])
        q.put((rank, [r["status"] for r in res]))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


def test_distributed_check_two_gloo_ranks(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_dist_rank, args=(r, 2, port, str(tmp_path / "d.json"), q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert got == {0: ["passed", "passed"], 1: ["passed", "passed"]}, got
    rec = json.loads((tmp_path / "d.json").read_text())
    assert rec["results"][0]["all_rank_parameters_equal"] and rec["results"][0]["accumulation"] == 2
