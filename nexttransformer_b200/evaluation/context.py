"""CORE input-length policy: evaluation beyond the training context (``nexttransformer/evaluation/
context.py`` and ``inference_view`` in ``nexttransformer/evaluation/core.py`` of the reference).

By default every CORE prompt is scored whole, which is longer than the 2048-token training context
for three tasks; the model is evaluated through ``inference_view``, a shallow copy that shares the
weights and the trained attention windows but accepts inputs up to its rotary capacity.
``--core-max-tokens N`` instead left-truncates every input to N tokens.  ``check_full_context``
refuses a limit that would cut a scored answer (or, for Inkling REL, a length beyond its learned
table) before a run starts; ``core_context`` / ``validate_submission`` record and check the policy
beside a result, and ``resume_core_limit`` keeps it fixed across resumed segments.
"""
import argparse
from copy import copy

# Token lengths of the pinned CORE-22 bundle under the pinned tokenizer (the reference's
# core-lengths.json): the longest prompt, the longest scored answer, the training context.
CORE_LENGTHS = {"trainingTokens": 2048, "maxPromptTokens": 5835, "longestAnswerTokens": 224,
                "overTrainingContext": {"SQuAD": 6895, "BoolQ": 185, "Language Identification": 1820},
                "taskCount": 22, "questionCount": 91037}


def positive_tokens(value):
    count = int(value)
    if count <= 0:
        raise argparse.ArgumentTypeError("the CORE token limit must be positive")
    return count


def add_core_max_tokens(parser):
    parser.add_argument("--core-max-tokens", type=positive_tokens, metavar="N",
                        help="left-truncate each CORE input to N tokens (default: the full prompt)")


def check_full_context(config, max_tokens):
    minimum = CORE_LENGTHS["longestAnswerTokens"] + 1
    if max_tokens is not None and max_tokens < minimum:
        raise ValueError(f"--core-max-tokens must be at least {minimum} so full CORE keeps every scored answer "
                         "and the token before it")
    extent = dict(getattr(config, "options", ()) or ()).get("rel_extent")
    needed = CORE_LENGTHS["maxPromptTokens"] if max_tokens is None else min(CORE_LENGTHS["maxPromptTokens"],
                                                                              max_tokens)
    if extent is not None and needed > extent:
        raise ValueError(f"CORE needs {needed} tokens but the learned REL table covers {extent}; "
                         f"set --core-max-tokens {extent} for left truncation")


def core_context(training_tokens, max_tokens, measured):
    return {"trainingTokens": training_tokens, "truncation": "none" if max_tokens is None else "left",
            "maxTokens": max_tokens, "maxEvaluatedTokens": measured}


def validate_submission(context):
    """Full leaderboard runs share one tokenizer, the 22 tasks and the training length."""
    keys = {"trainingTokens", "truncation", "maxTokens", "maxEvaluatedTokens"}
    if not isinstance(context, dict) or not keys <= context.keys():
        raise ValueError("CORE context must declare " + ", ".join(sorted(keys)))
    cap = context["maxTokens"]
    if cap is not None and (type(cap) is not int or cap <= CORE_LENGTHS["longestAnswerTokens"]):
        raise ValueError("CORE maxTokens must keep every answer and at least one token before it")
    expected = CORE_LENGTHS["maxPromptTokens"] if cap is None else min(cap, CORE_LENGTHS["maxPromptTokens"])
    if (type(context["trainingTokens"]) is not int or type(context["maxEvaluatedTokens"]) is not int
            or context != core_context(CORE_LENGTHS["trainingTokens"], cap, expected)):
        raise ValueError("CORE context disagrees with its truncation setting or the pinned prompt lengths")


def resume_core_limit(state, requested, training_tokens):
    """Checkpoints written before the policy existed used the training context."""
    previous = state.get("core_max_tokens", training_tokens)
    if requested is not None and requested != previous:
        raise ValueError(f"resume CORE length policy differs from the checkpoint (max tokens: {previous})")
    return previous


class _LongerContext:
    """A model configuration read through, with the sequence length raised to the rotary capacity."""

    def __init__(self, trained, capacity):
        self.trained, self.sequence_len = trained, capacity

    def __getattr__(self, name):
        return getattr(self.trained, name)


def inference_view(model, max_tokens):
    """The model itself when inputs fit its context; else a shallow copy that shares weights and the
    trained windows and accepts inputs up to its rotary capacity."""
    from nexttransformer_b200.models.lm import LanguageModel
    from nexttransformer_b200.models.native.model import NativeExperiment
    if max_tokens is not None and max_tokens <= model.config.sequence_len:
        return model
    if not isinstance(model, (LanguageModel, NativeExperiment)):
        return model
    view = copy(model)
    capacity = model.cos.size(1)
    if isinstance(model, NativeExperiment):
        view.max_seq_len = capacity
    else:
        view.config = _LongerContext(model.config, capacity)
        view._window = model._window       # windows stay those of the training length
    return view


class LengthProbe:
    """Forwards to a model and records the longest input it saw."""

    def __init__(self, model):
        self.model, self.longest = model, 0

    def __call__(self, ids, *args, **kwargs):
        self.longest = max(self.longest, ids.shape[1])
        return self.model(ids, *args, **kwargs)
