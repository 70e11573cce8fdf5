"""Runtime pieces on CPU: checkpoints (both formats), tokenizer, data streams, KV-cache decoding."""
import json

import pytest
import torch

from nexttransformer_b200.models.config import debug_config
from nexttransformer_b200.models.lm import build_model


def test_formal_checkpoint_roundtrip(tmp_path):
    from nexttransformer_b200.optim.groups import protocol_groups
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW
    from nexttransformer_b200.runtime import checkpoint as ck
    from nexttransformer_b200.runtime.data import SyntheticStream
    c = debug_config("dense")
    m = build_model(c, "cpu", seed=1)
    opt = MuonAdamW(protocol_groups(m))
    s = SyntheticStream(c.vocab_size, c.sequence_len)
    x, y = s.batch(2, torch.device("cpu"))
    m(x, y).backward()
    opt.step()
    d = ck.save_checkpoint(tmp_path, m, opt, s, c, {"k": 1}, {"step": 1}, 0, 1)
    assert json.loads((d / "complete.json").read_text())["step"] == 1
    m2 = build_model(c, "cpu", seed=2)
    opt2 = MuonAdamW(protocol_groups(m2))
    s2 = SyntheticStream(c.vocab_size, c.sequence_len)
    ck.load_checkpoint(d, m2, opt2, s2)
    for (n, a), (_, b) in zip(m.state_dict().items(), m2.state_dict().items()):
        assert torch.equal(a, b), n
    assert s2.rows == s.rows
    (d / "model.pt").write_bytes((d / "model.pt").read_bytes()[:-8] + b"corrupt!")
    with pytest.raises(ValueError, match="checksum"):
        ck.load_checkpoint(d, m2)


def test_nanochat_format(tmp_path):
    from nexttransformer_b200.runtime import checkpoint as ck
    m = build_model(debug_config("dense"), "cpu", seed=1)
    ck.save_nanochat(tmp_path, 7, m.state_dict(), {"x": torch.ones(1)}, {"step": 7})
    assert ck.last_nanochat_step(tmp_path) == 7
    sd, opt, meta = ck.load_nanochat(tmp_path, 7, load_optimizer=True)
    assert meta["step"] == 7 and torch.equal(opt["x"], torch.ones(1))
    m.load_state_dict(sd)


def test_tokenizer_train_roundtrip(tmp_path):
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    texts = ["hello world, hello there! numbers 12345 and more words."] * 20 + ["the quick brown fox"] * 10
    tok = BPETokenizer.train_from_iterator(texts, vocab_size=300)
    assert tok.get_vocab_size() == 300
    ids = tok.encode("hello world, the quick fox", prepend="<|bos|>")
    assert ids[0] == tok.get_bos_token_id()
    assert tok.decode(ids[1:]) == "hello world, the quick fox"
    tok.save(tmp_path)
    tok2 = BPETokenizer.from_directory(tmp_path)
    assert tok2.encode("hello there") == tok.encode("hello there")
    tb = torch.load(tmp_path / "token_bytes.pt")
    assert tb[tok.get_bos_token_id()] == 0 and tb[ord("a")] == 1


def test_bestfit_stream_exact_resume(tmp_path):
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq
    from nexttransformer_b200.runtime.data import BestFitStream
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    words = ["alpha", "beta", "gamma", "delta", "epsilon", "zeta"]
    docs = [" ".join(words[(i + j) % 6] for j in range(3 + i % 11)) for i in range(400)]
    for k, name in enumerate(("shard_00000.parquet", "shard_00001.parquet", "shard_06542.parquet")):
        pq.write_table(pa.table({"text": docs[k * 100:(k + 1) * 100]}), tmp_path / name, row_group_size=20)
    tok = BPETokenizer.train_from_iterator(docs, vocab_size=300)
    a = BestFitStream(tmp_path, tok, "train", sequence_len=16, buffer_size=8, tokenizer_batch_size=4)
    x1, _ = a.batch(3, torch.device("cpu"))
    state = a.state_dict()
    x2, _ = a.batch(3, torch.device("cpu"))
    b = BestFitStream(tmp_path, tok, "train", sequence_len=16, buffer_size=8, tokenizer_batch_size=4)
    b.load_state_dict(state)
    y2, _ = b.batch(3, torch.device("cpu"))
    assert torch.equal(x2, y2)
    assert (x1[:, 0] == tok.get_bos_token_id()).all()


def test_kv_cache_decode_matches_full_forward():
    from nexttransformer_b200.inference import KVCache, decode
    c = debug_config("dense")
    m = build_model(c, "cpu", seed=3)
    with torch.no_grad():
        for b in m.transformer.h:
            b.attn.c_proj.weight.normal_(0, .05)
            b.mlp.c_proj.weight.normal_(0, .05)
        m.smear_lambda.fill_(.7)
    m.eval()
    ids = torch.randint(0, c.vocab_size, (1, 10))
    full = m(ids)[:, -1]
    cache = KVCache(1, 16, c.n_layer, c.n_kv_head, c.head_dim, "cpu", m.cos.dtype)
    decode(m, ids[:, :6], cache)
    for t in range(6, 9):
        decode(m, ids[:, t:t + 1], cache)
    last = decode(m, ids[:, 9:10], cache)
    assert torch.allclose(last, full, atol=1e-4), (last - full).abs().max()


def test_tracking_auth_preflight():
    import subprocess
    from types import SimpleNamespace
    from nexttransformer_b200.runtime.tracking_auth import preflight
    preflight("disabled", runner=None)          # offline modes never start the check
    preflight("online", runner=lambda *a, **k: SimpleNamespace(returncode=0))
    for code in (2, 3, 4, 9):
        with pytest.raises(RuntimeError):
            preflight("online", runner=lambda *a, code=code, **k: SimpleNamespace(returncode=code))

    def slow(*a, **k):
        raise subprocess.TimeoutExpired(a[0], k["timeout"])
    with pytest.raises(RuntimeError, match="timed out"):
        preflight("online", timeout=1, runner=slow)


def test_optimizer_state_keeps_fp32_moments_of_bf16_tables():
    """torch's load_state_dict casts state to the parameter dtype; bf16 tables keep fp32 moments."""
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW
    from nexttransformer_b200.runtime.checkpoint import load_optimizer_state

    def make():
        torch.manual_seed(0)
        table = torch.nn.Parameter(torch.randn(16, 8).to(torch.bfloat16))
        return table, MuonAdamW([dict(kind="adamw", params=[table], lr=1e-2, betas=(0.9, 0.95), eps=1e-10,
                                      weight_decay=0.0)])
    table, opt = make()
    table.grad = torch.randn(16, 8).to(torch.bfloat16)
    opt.step()
    saved = opt.state_dict()
    fresh_table, fresh = make()
    load_optimizer_state(fresh, saved)
    for key in ("exp_avg", "exp_avg_sq"):
        assert fresh.state[fresh_table][key].dtype == torch.float32
        assert torch.equal(fresh.state[fresh_table][key], opt.state[table][key])


def test_prefetch_stream_is_exact(tmp_path):
    """Prefetched batches, row counts and checkpoint states equal the plain stream's, across a
    batch-size change and a resume."""
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq
    from nexttransformer_b200.runtime.data import BestFitStream, SyntheticStream
    from nexttransformer_b200.runtime.prefetch import PrefetchStream
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    words = ["alpha", "beta", "gamma", "delta", "epsilon", "zeta"]
    docs = [" ".join(words[(i + j) % 6] for j in range(3 + i % 11)) for i in range(400)]
    for k, name in enumerate(("shard_00000.parquet", "shard_00001.parquet", "shard_06542.parquet")):
        pq.write_table(pa.table({"text": docs[k * 100:(k + 1) * 100]}), tmp_path / name, row_group_size=20)
    tok = BPETokenizer.train_from_iterator(docs, vocab_size=300)
    cpu = torch.device("cpu")
    for make in (lambda: BestFitStream(tmp_path, tok, "train", sequence_len=16, buffer_size=8, tokenizer_batch_size=4),
                 lambda: SyntheticStream(300, 16, seed=3)):
        plain, pre = make(), PrefetchStream(make(), depth=3)
        for size in (3, 3, 2, 3):
            a, b = plain.batch(size, cpu), pre.batch(size, cpu)
            assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
            assert plain.rows == pre.rows
        assert pre.state_dict() == plain.state_dict()
        state = pre.state_dict()
        nxt = plain.batch(2, cpu)
        resumed = PrefetchStream(make(), depth=2)
        resumed.load_state_dict(state)
        got = resumed.batch(2, cpu)
        assert torch.equal(nxt[0], got[0])
        pre.close()
        resumed.close()
