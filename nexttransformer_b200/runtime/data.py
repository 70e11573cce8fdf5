"""Training data streams with exact, checkpointable per-rank state.

``BestFitStream`` reads parquet shards (the last shard is the validation split), strides row
groups over ranks, tokenises documents with BOS prepended and packs rows of T + 1 tokens by BOS
best-fit (``_native.BestFitPacker``; the behaviour of the reference's ``nexttransformer/
runtime/data.py:45-119``).  Row generation never depends on micro-batch size.

``SyntheticStream`` yields iid uniform tokens from a counter-keyed generator (benchmarks,
tests); ``stateless_rows`` is the deterministic pattern the distributed checks use.
"""
import copy
import hashlib
import json
from pathlib import Path

import torch

from nexttransformer_b200.runtime.files import VALIDATION_SHARD


class BestFitStream:
    def __init__(self, data_dir, tokenizer, split, rank=0, world=1, sequence_len=2048, buffer_size=1000,
                 tokenizer_batch_size=128, tokenizer_threads=4, validation_shard=VALIDATION_SHARD):
        import nexttransformer_b200._native as native
        paths = sorted(Path(data_dir).glob("*.parquet"))
        if not paths or paths[-1].name != validation_shard:
            raise ValueError("data needs the pinned final validation shard")
        self.paths = paths[:-1] if split == "train" else paths[-1:]
        if split not in ("train", "val") or not self.paths:
            raise ValueError("invalid split or no training shards")
        self.tokenizer, self.split = tokenizer, split
        self.rank, self.world = rank, world
        self.sequence_len, self.buffer_size = sequence_len, buffer_size
        self.tokenizer_batch_size, self.tokenizer_threads = tokenizer_batch_size, tokenizer_threads
        self.cursor = dict(pq_idx=0, rg_idx=rank, document_offset=0, epoch=1)
        self.packer = native.BestFitPacker()
        self.rows = 0
        self._key, self._texts = None, None
        self.identity = hashlib.sha256(json.dumps({
            "files": [(p.name, p.stat().st_size) for p in self.paths], "rank": rank, "world": world,
            "sequence_len": sequence_len, "split": split, "buffer": buffer_size,
            "tokenizer_batch_size": tokenizer_batch_size}, sort_keys=True).encode()).hexdigest()

    def _documents(self):
        import pyarrow.parquet as pq
        c = self.cursor
        while True:
            if c["pq_idx"] >= len(self.paths):
                c.update(pq_idx=0, rg_idx=self.rank, document_offset=0, epoch=c["epoch"] + 1)
            key = (c["pq_idx"], c["rg_idx"], c["epoch"])
            pf = pq.ParquetFile(self.paths[c["pq_idx"]]) if self._key != key else None
            if pf is not None and c["rg_idx"] >= pf.num_row_groups:
                c.update(pq_idx=c["pq_idx"] + 1, rg_idx=self.rank, document_offset=0)
                continue
            if self._key != key:
                self._texts = pf.read_row_group(c["rg_idx"]).column("text").to_pylist()
                self._key = key
            s = c["document_offset"]
            batch = self._texts[s:s + self.tokenizer_batch_size]
            c["document_offset"] += len(batch)
            if c["document_offset"] >= len(self._texts):
                c.update(rg_idx=c["rg_idx"] + self.world, document_offset=0)
            if batch:
                return batch

    def _row(self):
        cap = self.sequence_len + 1
        row = []
        while len(row) < cap:
            while self.packer.size() < self.buffer_size:
                self.packer.add(self.tokenizer.encode(self._documents(), prepend=self.tokenizer.get_bos_token_id(),
                                                      num_threads=self.tokenizer_threads))
            row.extend(self.packer.pick(cap - len(row)))
        self.rows += 1
        return row

    def cpu_batch(self, batch_size, pin=False):
        rows = torch.tensor([self._row() for _ in range(batch_size)], dtype=torch.long)
        x, y = rows[:, :-1].contiguous(), rows[:, 1:].contiguous()
        return (x.pin_memory(), y.pin_memory()) if pin else (x, y)

    def batch(self, batch_size, device):
        x, y = self.cpu_batch(batch_size, pin=torch.device(device).type == "cuda")
        return x.to(device, non_blocking=True), y.to(device, non_blocking=True)

    def batches(self, batch_size, device):
        while True:
            yield self.batch(batch_size, device)

    def state_dict(self):
        return copy.deepcopy(dict(identity=self.identity, cursor=self.cursor, buffer=self.packer.state(),
                                  rows=self.rows))

    def load_state_dict(self, state):
        if state["identity"] != self.identity:
            raise ValueError("data stream configuration changed on resume")
        self.cursor, self.rows = copy.deepcopy(state["cursor"]), state["rows"]
        self.packer.set_state(state["buffer"])
        self._key, self._texts = None, None


class SyntheticStream:
    """iid uniform tokens; row r of rank k is a pure function of (seed, k, r), so resume is exact."""

    def __init__(self, vocab_size, sequence_len, rank=0, world=1, seed=42):
        self.vocab_size, self.sequence_len = vocab_size, sequence_len
        self.rank, self.world, self.seed = rank, world, seed
        self.rows = 0
        self.identity = hashlib.sha256(json.dumps(dict(kind="synthetic", v=vocab_size, t=sequence_len, r=rank, w=world,
                                                       s=seed), sort_keys=True).encode()).hexdigest()

    def _row(self, r):
        g = torch.Generator().manual_seed((self.seed * 1_000_003 + self.rank) * 1_000_033 + r)
        return torch.randint(0, self.vocab_size, (self.sequence_len + 1,), generator=g)

    def cpu_batch(self, batch_size, pin=False):
        rows = torch.stack([self._row(self.rows + i) for i in range(batch_size)])
        self.rows += batch_size
        x, y = rows[:, :-1].contiguous(), rows[:, 1:].contiguous()
        return (x.pin_memory(), y.pin_memory()) if pin else (x, y)

    def batch(self, batch_size, device):
        x, y = self.cpu_batch(batch_size, pin=torch.device(device).type == "cuda")
        return x.to(device, non_blocking=True), y.to(device, non_blocking=True)

    def state_dict(self):
        return dict(identity=self.identity, rows=self.rows)

    def load_state_dict(self, state):
        if state["identity"] != self.identity:
            raise ValueError("synthetic stream configuration changed on resume")
        self.rows = state["rows"]


def stateless_rows(batch, sequence_len, vocab_size, rank, step=0):
    """Token (pos mod (T + 1) + row 17 + 42) mod vocab: the pattern of the distributed checks."""
    pos = torch.arange(sequence_len + 1)
    rows = torch.arange(batch) + rank * batch + step * 7919
    tok = (pos[None, :] % (sequence_len + 1) + rows[:, None] * 17 + 42) % vocab_size
    return tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
