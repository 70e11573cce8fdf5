"""CORE-style in-context evaluation (DCLM task formats: multiple choice, schema, language modelling).

Prompt rendering and scoring follow the reference's ``nanochat/core_eval.py``: few-shot examples
are joined by blank lines with a continuation delimiter; multiple-choice items compare the mean
loss of each choice's continuation (common prefix excluded), schema items compare contexts with
a shared continuation (common suffix scored), LM items require every continuation token to be
the greedy prediction.  The task score is centred accuracy (acc - random) / (1 - random).
"""
import random

import torch
import torch.distributed as dist


def _fewshot(examples, fmt):
    return "".join(fmt(e) + "\n\n" for e in examples)


def render_mc(item, delim, shots=()):
    pre = _fewshot(shots, lambda e: f"{e['query']}{delim}{e['choices'][e['gold']]}")
    return [f"{pre}{item['query']}{delim}{c}" for c in item["choices"]]


def render_schema(item, delim, shots=()):
    pre = _fewshot(shots, lambda e: f"{e['context_options'][e['gold']]}{delim}{e['continuation']}")
    return [f"{pre}{ctx}{delim}{item['continuation']}" for ctx in item["context_options"]]


def render_lm(item, delim, shots=()):
    pre = _fewshot(shots, lambda e: f"{e['context'].strip()}{delim}{e['continuation']}")
    without = f"{pre}{item['context'].strip()}{delim}".strip()
    return [without, f"{pre}{item['context'].strip()}{delim}{item['continuation']}"]


def common_length(seqs, direction="left"):
    n = min(len(s) for s in seqs)
    idx = range(n) if direction == "left" else range(-1, -n - 1, -1)
    for i, j in enumerate(idx):
        if not all(s[j] == seqs[0][j] for s in seqs):
            return i
    return n


@torch.no_grad()
def score_item(model, tokenizer, item, task_type, delim, shots, device, max_len=None):
    if task_type == "multiple_choice":
        prompts = render_mc(item, delim, shots)
    elif task_type == "schema":
        prompts = render_schema(item, delim, shots)
    else:
        prompts = render_lm(item, delim, shots)
    toks = tokenizer(prompts, prepend=tokenizer.get_bos_token_id())
    if task_type == "multiple_choice":
        s = common_length(toks, "left")
        spans = [(s, len(t)) for t in toks]
    elif task_type == "schema":
        s = common_length(toks, "right")
        spans = [(len(t) - s, len(t)) for t in toks]
    else:
        spans = [(len(toks[0]), len(toks[1]))]
        toks = [toks[1]]
    if max_len:
        cut = [max(0, len(t) - max_len) for t in toks]
        toks = [t[c:] for t, c in zip(toks, cut)]
        spans = [(a - c, b - c) for (a, b), c in zip(spans, cut)]
    L = max(len(t) for t in toks)
    ids = torch.zeros(len(toks), L, dtype=torch.long)
    for i, t in enumerate(toks):
        ids[i, :len(t)] = torch.tensor(t)
    ids = ids.to(device)
    logits = model(ids).float()
    lp = torch.log_softmax(logits[:, :-1], -1)
    tgt = ids[:, 1:]
    losses = -lp.gather(-1, tgt[..., None]).squeeze(-1)
    if task_type == "language_modeling":
        a, b = spans[0]
        return bool((logits[0, a - 1:b - 1].argmax(-1) == ids[0, a:b]).all())
    mean = [losses[i, a - 1:b - 1].mean().item() for i, (a, b) in enumerate(spans)]
    return int(min(range(len(mean)), key=mean.__getitem__)) == item["gold"]


def evaluate_task(model, tokenizer, data, meta, device, rank=0, world=1, max_per_task=-1, max_len=None):
    """Accuracy of one task; examples are sharded over ranks and counts all-reduced."""
    rng = random.Random(1234)
    items = data if max_per_task < 0 else data[:max_per_task]
    correct = torch.zeros(2, device=device)
    for i in range(rank, len(items), world):
        item = items[i]
        k = meta.get("num_fewshot", 0)
        pool = [j for j in range(len(data)) if j != i]
        shots = [data[j] for j in rng.sample(pool, min(k, len(pool)))] if k else []
        ok = score_item(model, tokenizer, item, meta["task_type"], meta.get("continuation_delimiter", " "), shots,
                        device, max_len)
        correct += torch.tensor([float(ok), 1.], device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(correct)
    return float(correct[0] / correct[1].clamp_min(1))


def centered(acc, random_baseline):
    """Centred accuracy: 0 at the random baseline (given in percent), 1 at perfect."""
    r = random_baseline / 100.0
    return (acc - r) / (1 - r)


def evaluate_core(model, tokenizer, tasks, device, rank=0, world=1, max_per_task=-1, max_len=None):
    """tasks: list of dict(label, data, meta{task_type, num_fewshot, continuation_delimiter}, random_baseline)."""
    results, cent = {}, {}
    for t in tasks:
        acc = evaluate_task(model, tokenizer, t["data"], t["meta"], device, rank, world, max_per_task, max_len)
        results[t["label"]] = acc
        cent[t["label"]] = centered(acc, t.get("random_baseline", 0.0))
    return dict(results=results, centered_results=cent, core_metric=sum(cent.values()) / max(len(cent), 1))
