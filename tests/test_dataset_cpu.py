"""Shard download and listing (runtime/dataset.py) against a local HTTP server."""
import functools
import http.server
import threading

import pytest

from nexttransformer_b200.runtime import dataset as ds


@pytest.fixture
def server(tmp_path):
    root = tmp_path / "hub"
    root.mkdir()
    for i in (0, 1, 2, 9):
        (root / ds.shard_name(i)).write_bytes(bytes([i]) * (3 * ds.CHUNK // 2))
    handler = functools.partial(http.server.SimpleHTTPRequestHandler, directory=str(root))
    handler.log_message = lambda *a: None
    srv = http.server.ThreadingHTTPServer(("127.0.0.1", 0), handler)
    t = threading.Thread(target=srv.serve_forever, daemon=True)
    t.start()
    yield f"http://127.0.0.1:{srv.server_address[1]}"
    srv.shutdown()


def test_download_train_and_validation(server, tmp_path):
    out = tmp_path / "data"
    status = ds.download(out, num_train=3, workers=3, base_url=server, max_shard=9, sleep=lambda s: None)
    assert status == {0: "downloaded", 1: "downloaded", 2: "downloaded", 9: "downloaded"}
    assert (out / ds.shard_name(9)).read_bytes() == bytes([9]) * (3 * ds.CHUNK // 2)
    assert not list(out.glob("*.tmp"))
    assert ds.split_shards(out, "val") == [str(out / ds.shard_name(9))]
    assert len(ds.split_shards(out, "train")) == 3
    again = ds.download(out, num_train=3, workers=2, base_url=server, max_shard=9)
    assert set(again.values()) == {"present"}


def test_missing_shard_retries_then_fails(server, tmp_path):
    waits = []
    out = tmp_path / "data"
    out.mkdir()
    idx, status = ds.download_shard(5, out, server, attempts=3, backoff=2.0, sleep=waits.append)
    assert idx == 5 and status.startswith("failed")
    assert waits == [2.0, 4.0]
    assert not list(out.iterdir())


def test_partial_transfer_leaves_no_shard(tmp_path):
    calls = []

    def flaky(url):
        calls.append(url)
        yield b"x" * 10
        if len(calls) < 2:
            raise OSError("connection reset")
        yield b"y" * 10

    idx, status = ds.download_shard(0, tmp_path, "http://unused", attempts=3, fetch=flaky, sleep=lambda s: None)
    assert status == "downloaded" and len(calls) == 2
    assert (tmp_path / ds.shard_name(0)).read_bytes() == b"x" * 10 + b"y" * 10


def test_iter_batched_strides_row_groups(tmp_path):
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq
    for i, n in ((0, 4), (1, 2)):
        table = pa.table({"text": [f"s{i}-{j}" for j in range(n)]})
        pq.write_table(table, tmp_path / ds.shard_name(i), row_group_size=1)
    rank0 = [t for batch in ds.iter_batched(tmp_path, "train", start=0, step=2) for t in batch]
    rank1 = [t for batch in ds.iter_batched(tmp_path, "train", start=1, step=2) for t in batch]
    assert rank0 == ["s0-0", "s0-2"] and rank1 == ["s0-1", "s0-3"]
    assert [t for b in ds.iter_batched(tmp_path, "val") for t in b] == ["s1-0", "s1-1"]
