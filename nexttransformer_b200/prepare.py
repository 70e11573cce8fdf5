"""Prepare the pinned resources: ``python -m nexttransformer_b200.prepare --data-dir D --resources R
--source-manifest M.json --core-archive eval_bundle.zip``.

Steps (behaviour of the reference's ``nexttransformer/prepare.py``): verify the dataset against the
pinned Hub manifest (file names and sizes, validation-shard sha256); unpack and pin the CORE bundle;
link both into the resource directory; train the BPE tokenizer once (GPT-4 split pattern, vocabulary
32768, the first 2e9 characters with each document capped at 10,000 characters, merges learned by
the C++ trainer); write ``native_manifest.json`` with every digest.  A file lock serialises
concurrent preparations.
"""
from nexttransformer_b200.runtime.site import add_runtime_arguments, bootstrap_runtime

if __name__ == "__main__":
    bootstrap_runtime()

import argparse
import json
from pathlib import Path

VOCAB = 32768
MAX_CHARS = 2_000_000_000
DOC_CAP = 10_000


def training_texts(data_dir, validation_shard, max_chars=MAX_CHARS, doc_cap=DOC_CAP):
    """Documents of the training shards in order, each capped, until ``max_chars`` are reached."""
    import pyarrow.parquet as pq
    seen = 0
    for path in sorted(Path(data_dir).glob("*.parquet")):
        if path.name == validation_shard:
            continue
        pf = pq.ParquetFile(path)
        for rg in range(pf.num_row_groups):
            for text in pf.read_row_group(rg).column("text").to_pylist():
                text = text[:doc_cap]
                yield text
                seen += len(text)
                if seen >= max_chars:
                    return


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, allow_abbrev=False)
    add_runtime_arguments(p)
    p.add_argument("--source-manifest", type=Path, required=True, help="Hub file listing of the pinned revision")
    p.add_argument("--core-archive", type=Path, help="local eval_bundle.zip (skipped with --existing-core-resources)")
    p.add_argument("--existing-core-resources", type=Path)
    p.add_argument("--max-chars", type=int, default=MAX_CHARS)
    p.add_argument("--vocab-size", type=int, default=VOCAB)
    p.add_argument("--download-shards", type=int, default=None,
                   help="fetch this many training shards (-1: all) and the validation shard before verifying")
    a = p.parse_args(argv)
    from nexttransformer_b200.runtime.site import resolve
    resolve(a)
    if a.data_dir is None:
        p.error("--data-dir is required")
    from filelock import FileLock
    from nexttransformer_b200.models.native.config import UPSTREAM_COMMIT
    from nexttransformer_b200.runtime import resources as res
    from nexttransformer_b200.runtime.files import DATA_REVISION, VALIDATION_SHARD, atomic_json, sha256
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    out = Path(a.resources)
    out.mkdir(parents=True, exist_ok=True)
    with FileLock(str(out / "prepare.lock")):
        if a.download_shards is not None:
            from nexttransformer_b200.runtime.dataset import download
            failed = [i for i, s in download(a.data_dir, a.download_shards).items() if s.startswith("failed")]
            if failed:
                raise SystemExit(f"{len(failed)} shard downloads failed (first: {failed[0]})")
        official = res.load_source_manifest(a.source_manifest)
        expected, val_sha = res.verify_dataset(a.data_dir, official, VALIDATION_SHARD)
        core_root = a.existing_core_resources or out
        if a.existing_core_resources is None:
            if a.core_archive is None:
                p.error("give --core-archive or --existing-core-resources")
            res.prepare_core(out, a.core_archive)
        res.verify_core(core_root)
        for name, target in (("base_data_climbmix", Path(a.data_dir)), ("eval_bundle", core_root / "eval_bundle"),
                             ("core_manifest.json", core_root / "core_manifest.json")):
            link = out / name
            if link.exists() or link.is_symlink():
                if link.resolve() != target.resolve():
                    raise ValueError(f"resource target changed: {link}")
            else:
                link.symlink_to(target.resolve(), target_is_directory=target.is_dir())
        marker = out / "tokenizer_complete.json"
        if not marker.exists():
            if (out / "tokenizer").exists():
                raise ValueError("an incomplete tokenizer exists; inspect it before retraining")
            tok = BPETokenizer.train_from_iterator(training_texts(a.data_dir, VALIDATION_SHARD, a.max_chars),
                                                   a.vocab_size, max_chars=a.max_chars)
            tok.save(str(out / "tokenizer"))
            atomic_json(marker, {"max_chars": a.max_chars, "doc_cap": DOC_CAP, "vocab_size": a.vocab_size,
                                 "upstream_commit": UPSTREAM_COMMIT})
        tok = BPETokenizer.from_directory(str(out / "tokenizer"))
        if tok.get_vocab_size() != a.vocab_size:
            raise ValueError(f"tokenizer must have {a.vocab_size} entries")
        record = {"upstream_commit": UPSTREAM_COMMIT, "data_revision": DATA_REVISION,
                  "source_manifest_sha256": sha256(a.source_manifest),
                  "tokenizer_sha256": res.tokenizer_fingerprint(out),
                  "data_inventory_sha256": res.inventory_fingerprint(expected), "validation_sha256": val_sha,
                  "tokenizer_recipe": json.loads(marker.read_text()),
                  "packing": "BOS best-fit; buffer=1000; tokenizer_batch=128"}
        atomic_json(out / "native_manifest.json", record)
        print(json.dumps(record, indent=2))
        return record


if __name__ == "__main__":
    main()
