"""GPT-4-style BPE tokenizer: merges learned by the native trainer, encoding through tiktoken.

Pre-tokenisation splits text with the same regex as the reference (numbers in runs of at most
two digits); the merge table is learned by ``_native.train_bpe`` (C++), then packed into a
``tiktoken.Encoding`` whose pickle (``tokenizer.pkl``) and byte table (``token_bytes.pt``) are
the reference's on-disk tokenizer format (``nanochat/tokenizer.py``).
"""
from collections import Counter
import os
import pickle

import torch

SPECIAL_TOKENS = ["<|bos|>", "<|user_start|>", "<|user_end|>", "<|assistant_start|>", "<|assistant_end|>",
                  "<|python_start|>", "<|python_end|>", "<|output_start|>", "<|output_end|>"]
SPLIT_PATTERN = (r"""'(?i:[sdmt]|ll|ve|re)|[^\r\n\p{L}\p{N}]?+\p{L}+|\p{N}{1,2}| ?[^\s\p{L}\p{N}]++[\r\n]*|"""
                 r"""\s*[\r\n]|\s+(?!\S)|\s+""")


class BPETokenizer:
    def __init__(self, enc, bos_token="<|bos|>"):
        self.enc = enc
        self.bos_token_id = self.encode_special(bos_token)

    # ------------------------------------------------------------------ construction
    @classmethod
    def train_from_iterator(cls, texts, vocab_size, max_chars=None):
        import regex
        import tiktoken
        import nexttransformer_b200._native as native
        n_merges = vocab_size - len(SPECIAL_TOKENS) - 256
        if n_merges < 0:
            raise ValueError("vocab_size must leave room for 256 byte tokens and the special tokens")
        pat = regex.compile(SPLIT_PATTERN)
        counts, seen = Counter(), 0
        for text in texts:
            for piece in pat.findall(text):
                counts[piece] += 1
            seen += len(text)
            if max_chars and seen >= max_chars:
                break
        words = [list(w.encode("utf-8")) for w in counts]
        merges = native.train_bpe(words, list(counts.values()), n_merges, 256)
        token = {i: bytes([i]) for i in range(256)}
        ranks = {token[i]: i for i in range(256)}
        for i, (a, b) in enumerate(merges):
            token[256 + i] = token[a] + token[b]
            ranks[token[256 + i]] = 256 + i
        offset = len(ranks)
        specials = {name: offset + i for i, name in enumerate(SPECIAL_TOKENS)}
        enc = tiktoken.Encoding(name="nt_bpe", pat_str=SPLIT_PATTERN, mergeable_ranks=ranks, special_tokens=specials)
        return cls(enc)

    @classmethod
    def from_directory(cls, path):
        with open(os.path.join(path, "tokenizer.pkl"), "rb") as f:
            return cls(pickle.load(f))

    def save(self, path):
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, "tokenizer.pkl"), "wb") as f:
            pickle.dump(self.enc, f)
        torch.save(self.token_bytes(), os.path.join(path, "token_bytes.pt"))

    # ------------------------------------------------------------------ use
    def get_vocab_size(self):
        return self.enc.n_vocab

    def get_special_tokens(self):
        return self.enc.special_tokens_set

    def encode_special(self, text):
        return self.enc.encode_single_token(text)

    def get_bos_token_id(self):
        return self.bos_token_id

    def encode(self, text, prepend=None, append=None, num_threads=8):
        pre = self.encode_special(prepend) if isinstance(prepend, str) else prepend
        post = self.encode_special(append) if isinstance(append, str) else append
        if isinstance(text, str):
            ids = self.enc.encode_ordinary(text)
            return ([pre] if pre is not None else []) + ids + ([post] if post is not None else [])
        out = self.enc.encode_ordinary_batch(text, num_threads=num_threads)
        return [([pre] if pre is not None else []) + ids + ([post] if post is not None else []) for ids in out]

    __call__ = encode

    def decode(self, ids):
        return self.enc.decode(ids)

    def token_bytes(self):
        """UTF-8 byte length of every token id (0 for special tokens), for bits-per-byte."""
        special = set(self.enc.special_tokens_set)
        out = []
        for i in range(self.enc.n_vocab):
            try:
                b = self.enc.decode_single_token_bytes(i)
            except KeyError:
                b = b""
            out.append(0 if b.decode("utf-8", "replace") in special else len(b))
        return torch.tensor(out, dtype=torch.int32)
