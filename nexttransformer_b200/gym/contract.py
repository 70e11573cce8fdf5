"""Operations, parameter schemas and research profiles of the gym API.

One table describes every operation (its description and JSON schema); the HTTP service validates
each call against it and the MCP adapter lists it as its tools, so the two cannot drift.  Operation
names and their parameters follow the reference gym's API (``gym/src/nexttransformer_gym/api.py``)
so agents written for one can call the other; the schemas here are this package's.

A profile is a fixed research configuration: the shell dimensions a candidate is trained at, the
rows per update and the sequence length.  Agents choose a candidate and a profile, never raw
training options.
"""
from copy import deepcopy

from jsonschema import Draft202012Validator

SCHEMA_VERSION = "gym.api.v1"

_ID = {"type": "string", "minLength": 1, "maxLength": 128}
_PAGE = {"cursor": {"type": "string", "default": ""},
         "limit": {"type": "integer", "minimum": 1, "maximum": 100, "default": 50}}
_IDEMPOTENCY = {"idempotency_key": {"type": "string", "minLength": 1, "maxLength": 128}}
_CAND = {"candidate_id": _ID, "profile_id": _ID}


def _op(description, properties=None, required=(), mutation=False):
    props = dict(properties or {})
    if mutation:
        props.update(_IDEMPOTENCY)
    return {"description": description, "mutation": mutation,
            "inputSchema": {"type": "object", "properties": props, "required": list(required),
                            "additionalProperties": False}}


OPERATIONS = {
    "describe_space": _op("Profiles, the candidate package contract and every operation's schema."),
    "get_resources": _op("GPUs of this host: discovered, leased and free, with memory."),
    "submit_candidate": _op(
        "Upload a base64 ZIP with proposal.json and plugin/<method>/{method.json, __init__.py, *.py}: a "
        "source-only method plugin.  Identical content gives the same candidate.",
        {"package_base64": {"type": "string", "minLength": 1}}, ["package_base64"], mutation=True),
    "list_candidates": _op("This session's candidates.", _PAGE),
    "get_candidate": _op("One candidate's metadata and files.", {"candidate_id": _ID}, ["candidate_id"]),
    "inspect_cost": _op("Parameters and traced training FLOPs per token of a candidate at a profile.", _CAND,
                        list(_CAND)),
    "quote_experiment": _op(
        "Cost of training a candidate at a profile for target_update updates; reserves nothing.",
        {**_CAND, "target_update": {"type": "integer", "minimum": 1, "maximum": 100000, "default": 1},
         "gpus": {"type": "integer", "minimum": 0, "maximum": 8, "default": 0}},
        list(_CAND)),
    "run_experiment": _op("Queue a quoted experiment; reserves its FLOPs.", {"quote_id": _ID}, ["quote_id"],
                          mutation=True),
    "get_job": _op("State and progress of a job.", {"job_id": _ID}, ["job_id"]),
    "get_result": _op("Result of a finished job.", {"job_id": _ID}, ["job_id"]),
    "cancel_job": _op("Cancel a queued or running job; unused FLOPs return to the budget.", {"job_id": _ID},
                      ["job_id"], mutation=True),
    "read_events": _op("Session events after a cursor.",
                       {"cursor": {"type": "integer", "minimum": 0, "default": 0},
                        "limit": {"type": "integer", "minimum": 1, "maximum": 100, "default": 50}}),
    "get_budget": _op("Limit, spent, reserved and available research FLOPs."),
    "finalize": _op("Freeze a candidate and profile as the session's submission.", _CAND, list(_CAND),
                    mutation=True),
    "get_submission": _op("The frozen submission.", {"submission_id": _ID}, ["submission_id"]),
}

_VALIDATORS = {name: Draft202012Validator(op["inputSchema"]) for name, op in OPERATIONS.items()}

# Research profiles: shell dimensions of the candidate, rows per update and sequence length.
PROFILES = {
    "debug": dict(width=64, heads=2, layers=2, mlp_width=256, vocab_size=512, sequence_len=64, rows=8,
                  micro_rows=4, description="CPU-sized smoke profile"),
    "small": dict(width=512, heads=4, layers=8, mlp_width=2048, vocab_size=32768, sequence_len=1024, rows=64,
                  micro_rows=16, description="one-GPU research profile"),
    "d12": dict(width=768, heads=6, layers=12, mlp_width=3072, vocab_size=65536, sequence_len=2048, rows=256,
                micro_rows=32, description="GPT-2-small scale on 1-8 GPUs"),
}

PACKAGE_CONTRACT = {
    "format": "zip, base64-encoded",
    "files": ["proposal.json", "plugin/<method>/method.json", "plugin/<method>/__init__.py", "plugin/<method>/*.py"],
    "proposal": {"name": "string", "summary": "string"},
    "limits": {"compressed_bytes": 262144, "uncompressed_bytes": 1048576, "files": 32},
    "method_json": "name (= directory), family (looped, sparse, linear, residual, hybrid, others), optional "
                   "title, paper, options, debug_options, shell, layer_multiple",
    "forbidden": "binaries, symlinks, absolute or parent paths, files outside the list above",
}


class GymError(Exception):
    """An error reported to the caller as ``{"error": {"code", "message"}}``."""

    def __init__(self, code, message, status=400):
        super().__init__(message)
        self.code, self.message, self.status = code, message, status


def validate(operation, params):
    """Parameters with defaults filled in; raises GymError for an unknown operation or bad input."""
    if operation not in OPERATIONS:
        raise GymError("unknown_operation", f"no operation {operation!r}", 404)
    params = dict(params or {})
    errors = sorted(_VALIDATORS[operation].iter_errors(params), key=lambda e: list(e.path))
    if errors:
        raise GymError("invalid_params", "; ".join(e.message for e in errors[:5]))
    for key, spec in OPERATIONS[operation]["inputSchema"]["properties"].items():
        if key not in params and "default" in spec:
            params[key] = spec["default"]
    return params


def describe():
    return {"schema_version": SCHEMA_VERSION, "profiles": deepcopy(PROFILES), "candidate_contract": PACKAGE_CONTRACT,
            "operation_schemas": {k: {"description": v["description"], "inputSchema": v["inputSchema"]}
                                  for k, v in OPERATIONS.items()}}
