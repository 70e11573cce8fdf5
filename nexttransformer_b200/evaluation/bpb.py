"""Bits per byte: sum of token cross-entropies (nats) / (ln 2 x sum of UTF-8 bytes of the targets).

Targets that are ignored (-1) or special tokens (byte length 0) are excluded; partial sums are
all-reduced over ranks (reference: ``nanochat/loss_eval.py:9-65``).
"""
import math
import time

import torch
import torch.distributed as dist


@torch.no_grad()
def evaluate_bpb(model, batches, steps, token_bytes):
    """batches yields (x, y); token_bytes [V] int tensor on the model device."""
    dev = token_bytes.device
    nats = torch.zeros((), device=dev, dtype=torch.float64)
    nbytes = torch.zeros((), device=dev, dtype=torch.int64)
    was = model.training
    model.eval()
    it = iter(batches)
    for _ in range(steps):
        x, y = next(it)
        loss = model(x, y, loss_reduction="none").view(-1).double()
        yf = y.view(-1)
        valid = yf >= 0
        b = torch.where(valid, token_bytes[yf.clamp_min(0)], torch.zeros_like(yf)).to(torch.int64)
        count = b > 0
        nats += (loss * count).sum()
        nbytes += b.sum()
    model.train(was)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(nats)
        dist.all_reduce(nbytes)
    return float(nats) / (math.log(2) * max(int(nbytes), 1))


@torch.no_grad()
def evaluate_stream_loss(model, config, tokens, micro, rank, world, device, seed=0):
    """Mean token loss on a held-out synthetic stream (research runs without a dataset)."""
    from nexttransformer_b200.runtime.data import SyntheticStream
    stream = SyntheticStream(config.vocab_size, config.sequence_len, rank, world, seed=seed + 10_007)
    rows = max(1, tokens // (world * config.sequence_len))
    t0 = time.time()
    was = model.training
    model.eval()
    total = torch.zeros(2, device=device, dtype=torch.float64)
    done = 0
    while done < rows:
        b = min(micro, rows - done)
        x, y = stream.batch(b, device)
        loss = model(x, y, loss_reduction="none").double()
        total += torch.stack((loss.sum(), torch.tensor(float(loss.numel()), device=device, dtype=torch.float64)))
        done += b
    model.train(was)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(total)
    return dict(val_loss=float(total[0] / total[1]), val_tokens=int(total[1]), seconds=time.time() - t0)
