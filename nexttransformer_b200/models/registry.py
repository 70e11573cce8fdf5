"""Method registry: built-in families and methods, then plugins in name order.

Method names and their historical order are the reference's (``nexttransformer/models/
registry.py:13-27``): the order keys configuration audits and test ids, so it must not change.
"""
from nexttransformer_b200.models.plugins import discover

BUILTIN_FAMILIES = {
    "baseline": ("dense_full",),
    "looped": ("ut_act", "fixed_recursive", "huginn", "ouro", "deeploop"),
    "sparse": ("dsa", "qsa", "nsa", "seer", "moba"),
    "linear": ("deltanet", "gla", "kda", "retnet", "elu_linear", "elu_norm", "elu_qknorm", "gdn", "kda_no_ve"),
    "residual": ("residual_standard", "hc", "mhc", "attnres"),
    "hybrid": ("gdn_hybrid", "gdn_hybrid_swa", "deltanet_hybrid", "kda_hybrid", "qsa_hybrid", "moba_hybrid"),
    "others": ("dense", "mla_nope", "mha_no_ve"),
    # B200 additions (no reference counterpart as a registered method): Megatron-style MoE decoder.
    "moe": ("moe",),
}
BUILTIN_METHODS = (
    "dense", "ut_act", "fixed_recursive", "huginn", "ouro", "deeploop",
    "dsa", "qsa", "nsa", "seer", "moba", "deltanet", "gla",
    "kda", "retnet", "elu_linear", "elu_norm", "elu_qknorm", "gdn",
    "dense_full", "residual_standard", "hc", "mhc", "attnres",
    "gdn_hybrid", "gdn_hybrid_swa", "deltanet_hybrid",
    "kda_hybrid", "kda_no_ve", "mla_nope", "mha_no_ve", "qsa_hybrid", "moba_hybrid",
    "moe",
)
# Per-layer kinds of hybrid stacks that are not methods on their own.
MIXER_KINDS = ("attention", "swa")

PLUGINS = discover(BUILTIN_METHODS + MIXER_KINDS)
PLUGIN_METHODS = frozenset(PLUGINS)
FAMILIES = {fam: (*names, *sorted(n for n in PLUGINS if PLUGINS[n]["family"] == fam))
            for fam, names in BUILTIN_FAMILIES.items()}
METHODS = BUILTIN_METHODS + tuple(sorted(PLUGINS))
FAMILY = {m: fam for fam, names in FAMILIES.items() for m in names}
if sorted(FAMILY) != sorted(METHODS) or len(set(METHODS)) != len(METHODS):
    raise RuntimeError("method registry is inconsistent")


def members(family):
    """Built-in methods of a family (model rules never apply to plugins)."""
    return frozenset(BUILTIN_FAMILIES[family])
