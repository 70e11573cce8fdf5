"""Pretraining shards: listing, batched iteration and on-demand download.

    python -m nexttransformer_b200.runtime.dataset --data-dir D -n 170 -w 8

The dataset is a directory of ``shard_NNNNN.parquet`` files with a ``text`` column (ClimbMix-400B,
shards 0 .. 6542).  The last shard in sorted order is the validation split; a download always
fetches it beside the first ``n`` training shards.  Behaviour follows the reference's
``nanochat/dataset.py:32-160`` (shard names, split rule, retry-with-backoff download to a ``.tmp``
file renamed into place); the implementation is its own: a thread pool of streaming HTTP reads
(downloads wait on the network, not on the interpreter), an injectable fetcher so the logic is
tested against a local server, and a per-shard result record instead of prints.
"""
import argparse
import os
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

BASE_URL = "https://huggingface.co/datasets/karpathy/climbmix-400b-shuffle/resolve/main"
MAX_SHARD = 6542   # the validation shard: shard_06542.parquet
CHUNK = 1 << 20


def shard_name(index):
    return f"shard_{index:05d}.parquet"


def list_shards(data_dir):
    """Sorted full paths of the complete parquet shards in ``data_dir`` (partial ``.tmp`` files skipped)."""
    d = Path(data_dir)
    return [str(p) for p in sorted(d.glob("*.parquet")) if p.is_file()]


def split_shards(data_dir, split):
    """Training shards (all but the last) or the validation shard (the last)."""
    if split not in ("train", "val"):
        raise ValueError("split must be 'train' or 'val'")
    paths = list_shards(data_dir)
    return paths[:-1] if split == "train" else paths[-1:]


def iter_batched(data_dir, split, start=0, step=1):
    """Text lists, one per parquet row group, of a split; ``start`` / ``step`` stride the row groups
    (rank / world size under data parallelism)."""
    import pyarrow.parquet as pq
    for path in split_shards(data_dir, split):
        pf = pq.ParquetFile(path)
        for rg in range(start, pf.num_row_groups, step):
            yield pf.read_row_group(rg).column("text").to_pylist()


def http_fetch(url, timeout=30):
    """Chunks of the body of ``url`` (raises on an HTTP error)."""
    import requests
    response = requests.get(url, stream=True, timeout=timeout)
    response.raise_for_status()
    return response.iter_content(chunk_size=CHUNK)


def download_shard(index, data_dir, base_url=BASE_URL, attempts=5, backoff=2.0, fetch=http_fetch, sleep=time.sleep):
    """Fetch one shard into ``data_dir`` unless present; returns ``(index, status)`` with status
    ``"present"``, ``"downloaded"`` or ``"failed: <last error>"``.  The body is written to
    ``<name>.tmp`` and renamed, so a listing never sees a partial shard; waits between attempts grow
    as ``backoff ** attempt`` seconds."""
    name = shard_name(index)
    path = Path(data_dir) / name
    if path.exists():
        return index, "present"
    tmp = path.with_name(name + ".tmp")
    error = None
    for attempt in range(1, attempts + 1):
        try:
            with open(tmp, "wb") as f:
                for chunk in fetch(f"{base_url}/{name}"):
                    if chunk:
                        f.write(chunk)
            os.replace(tmp, path)
            return index, "downloaded"
        except (OSError, ValueError, RuntimeError) as e:   # requests' errors derive from OSError
            error = e
            tmp.unlink(missing_ok=True)
            if attempt < attempts:
                sleep(backoff ** attempt)
    return index, f"failed: {error}"


def download(data_dir, num_train=-1, workers=4, base_url=BASE_URL, max_shard=MAX_SHARD, **kw):
    """The first ``num_train`` training shards (all with -1) plus the validation shard; returns
    ``{index: status}``."""
    Path(data_dir).mkdir(parents=True, exist_ok=True)
    n = max_shard if num_train < 0 else min(num_train, max_shard)
    ids = list(range(n)) + [max_shard]
    with ThreadPoolExecutor(max_workers=max(1, workers)) as pool:
        results = pool.map(lambda i: download_shard(i, data_dir, base_url, **kw), ids)
    return dict(results)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--data-dir", type=Path, required=True)
    p.add_argument("-n", "--num-files", type=int, default=-1, help="training shards to fetch (-1: all)")
    p.add_argument("-w", "--num-workers", type=int, default=4)
    p.add_argument("--base-url", default=BASE_URL)
    a = p.parse_args(argv)
    status = download(a.data_dir, a.num_files, a.num_workers, a.base_url)
    failed = {i: s for i, s in status.items() if s.startswith("failed")}
    print(f"{len(status) - len(failed)}/{len(status)} shards in {a.data_dir}")
    for i, s in sorted(failed.items()):
        print(f"  {shard_name(i)}: {s}")
    return 1 if failed else 0


if __name__ == "__main__":
    raise SystemExit(main())
