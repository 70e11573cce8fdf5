"""Model configuration of every registered method.

Field names, defaults, the scoped-field rule and the JSON serialisation are those of the
reference (``nexttransformer/models/config.py:74-252``), so configuration files and model
fingerprints are interchangeable between the two trees.  Fields added here for the B200
configurations (GQA, MoE, NSA stride, custom scale) are "extension" fields: they are omitted
from the serialised form while they hold their defaults, so reference hashes still match.
"""
from dataclasses import asdict, dataclass, fields, replace
import hashlib
import json

from nexttransformer_b200.models.registry import METHODS, PLUGINS, members

LOOPED = members("looped")
SPARSE = members("sparse")
LINEAR = members("linear")
RESIDUAL = members("residual")
HYBRID = members("hybrid")
MOE = members("moe")
MLA = frozenset(("mla_nope",))
MLA_CONFIG = MLA | {"kda_hybrid"}
NO_VE = frozenset(("kda_hybrid", "kda_no_ve", "mla_nope", "mha_no_ve"))
V2_CALIBRATION = HYBRID | NO_VE | frozenset(PLUGINS)
FULL_ATTENTION = frozenset(("dense_full", *RESIDUAL, *MLA, "mha_no_ve"))
SCOPED_FIELDS = {
    "residual_streams": ("hc", "mhc"), "residual_gate_init": ("hc", "mhc"),
    "sinkhorn_iterations": ("mhc",), "attnres_groups": ("attnres",),
    "sliding_window": ("gdn_hybrid_swa",),
    **{f: tuple(sorted(MLA_CONFIG)) for f in ("q_rank", "kv_rank", "qk_nope_dim", "qk_rope_dim", "v_head_dim")},
}
# Extension fields (not in the reference): serialised only when they differ from the default.
EXTENSION_FIELDS = ("kv_heads", "attn_head_dim", "value_embeds", "compression_stride", "moe_experts", "moe_topk", "moe_ffn",
                    "moe_shared", "moe_dense_layers", "moe_bias_rate", "moe_aux_loss_coeff", "moe_z_loss_coeff")
CHUNK_BACKENDS = {"fla_chunk64": 64}
CHUNKED_METHODS = frozenset(("deltanet", "kda", "kda_no_ve", "retnet", "elu_linear", "elu_norm", "elu_qknorm", "gdn",
                             *(HYBRID - {"moba_hybrid"})))
LAYER_MULTIPLE = {"deltanet_hybrid": 2, "gdn_hybrid": 4, "gdn_hybrid_swa": 2, "kda_hybrid": 4,
                  "qsa_hybrid": 4, "moba_hybrid": 1,
                  **{n: spec.get("layer_multiple", 1) for n, spec in PLUGINS.items()}}


def frozen_options(options):
    """Plugin options as sorted (name, value) pairs with lists turned into tuples (hashable)."""
    def freeze(v):
        return tuple(freeze(x) for x in v) if isinstance(v, (list, tuple)) else v
    items = options.items() if isinstance(options, dict) else options
    pairs = tuple(sorted((str(k), freeze(v)) for k, v in items))
    if len({k for k, _ in pairs}) != len(pairs):
        raise ValueError("an option is given twice")
    return pairs


def hybrid_layout(method, layers):
    """Mixer kind of each physical layer of a hybrid stack (0-based).

    deltanet_hybrid: attention at 1-based positions 2 and N/2+1, DeltaNet elsewhere.
    gdn_hybrid: (GDN, GDN, GDN, attention) repeated.  kda_hybrid: (KDA x3, MLA-NoPE) repeated.
    qsa_hybrid: (GDN x3, QSA) repeated.  moba_hybrid: MoBA then three attention layers.
    gdn_hybrid_swa: GDN at even positions, sliding-window attention at odd ones.
    """
    if layers % LAYER_MULTIPLE[method]:
        raise ValueError(f"{method} needs a layer count that is a multiple of {LAYER_MULTIPLE[method]}")
    if method == "deltanet_hybrid":
        if layers < 4:
            raise ValueError("deltanet_hybrid needs at least four layers")
        return tuple("attention" if i in (1, layers // 2) else "deltanet" for i in range(layers))
    unit = {"gdn_hybrid": ("gdn", "gdn", "gdn", "attention"), "kda_hybrid": ("kda", "kda", "kda", "mla_nope"),
            "qsa_hybrid": ("gdn", "gdn", "gdn", "qsa"), "gdn_hybrid_swa": ("gdn", "swa")}
    if method in unit:
        u = unit[method]
        return tuple(u[i % len(u)] for i in range(layers))
    if method == "moba_hybrid":
        if layers < 4:
            raise ValueError("moba_hybrid needs at least one MoBA layer and three attention layers")
        return ("moba",) * (layers - 3) + ("attention",) * 3
    raise ValueError(f"{method} is not a hybrid")


@dataclass(frozen=True)
class ModelConfig:
    method: str = "dense"
    width: int = 1536
    heads: int = 12
    vocab_size: int = 32768
    sequence_len: int = 2048
    mlp_width: int = 6144
    layers: int = 24
    pre_layers: int = 3
    core_layers: int = 9
    post_layers: int = 3
    loops: int = 2
    window_pattern: str = "SSSL"
    max_loops: int = 3
    act_epsilon: float = .01
    ponder_weight: float = .01
    huginn_mean: float = 3.
    huginn_sigma: float = .5
    huginn_backprop_loops: int = 2
    routing_seed: int = 1729
    eval_loops: int = 3
    ouro_entropy_weight: float = .1
    ouro_gate_steps: int = 1024
    ouro_exit_quantile: float = .5
    sparse_topk: int = 256
    block_size: int = 128
    compression_size: int = 4
    local_window: int = 512
    index_heads: int = 4
    index_dim: int = 128
    index_rope_dim: int = 64
    index_loss_weight: float = 1.
    burnin_steps: int = 512
    slots: int = 64
    gate_rank: int = 16
    conv_size: int = 4
    reference_chunk: int = 32
    backend: str = "reference"
    scale: str = "formal"
    residual_streams: int = 4
    residual_gate_init: float = .01
    sinkhorn_iterations: int = 20
    attnres_groups: int = 8
    sliding_window: int = 2048
    q_rank: int = 768
    kv_rank: int = 256
    qk_nope_dim: int = 64
    qk_rope_dim: int = 64
    v_head_dim: int = 128
    options: tuple = ()
    # ---- extension fields (B200 configurations) -------------------------------------------
    kv_heads: int = 0              # 0: multi-head attention (kv heads = heads); else GQA group count
    attn_head_dim: int = 0         # 0: width / heads; else the softmax-attention head dimension (heads x
                                   # attn_head_dim may differ from width: q and output projections resize)
    value_embeds: int = -1         # -1: the method's rule; 0 / 1 force value embeddings off / on
    compression_stride: int = 0    # NSA compression stride; 0 = compression_size (no overlap)
    moe_experts: int = 64
    moe_topk: int = 8
    moe_ffn: int = 1024
    moe_shared: int = 1
    moe_dense_layers: int = 0      # leading layers with a dense FFN instead of experts
    moe_bias_rate: float = 1e-3    # aux-loss-free balancing: router-bias update speed
    moe_aux_loss_coeff: float = 0.0  # Switch-style load-balance loss weight (0: aux-loss-free only)
    moe_z_loss_coeff: float = 0.0    # router z-loss weight

    # ------------------------------------------------------------------ validation
    def __post_init__(self):
        object.__setattr__(self, "options", frozen_options(self.options))
        if self.method not in METHODS:
            raise ValueError(f"unknown method {self.method!r}")
        self._check_plugin_and_scope()
        self._check_shapes()
        self._check_method_rules()

    def _check_plugin_and_scope(self):
        if self.method in PLUGINS:
            declared = PLUGINS[self.method].get("options", {})
            if {k for k, _ in self.options} != set(declared):
                raise ValueError(f"{self.method} options must be exactly: {', '.join(sorted(declared)) or 'none'}")
            if self.layers % LAYER_MULTIPLE[self.method]:
                raise ValueError(f"{self.method} needs a layer count multiple of {LAYER_MULTIPLE[self.method]}")
        elif self.options:
            raise ValueError("options are parameters of plugin methods")
        defaults = {f.name: f.default for f in fields(self)}
        for name, users in SCOPED_FIELDS.items():
            if self.method not in users and getattr(self, name) != defaults[name]:
                raise ValueError(f"{name} is not a parameter of {self.method}")
        moe_fields = ("moe_experts", "moe_topk", "moe_ffn", "moe_shared", "moe_dense_layers", "moe_bias_rate",
                      "moe_aux_loss_coeff", "moe_z_loss_coeff")
        if self.method not in MOE and any(getattr(self, f) != defaults[f] for f in moe_fields):
            raise ValueError("MoE fields belong to the moe method")

    def _check_shapes(self):
        if min(self.residual_streams, self.sinkhorn_iterations, self.attnres_groups) <= 0 \
                or not self.residual_gate_init > 0:
            raise ValueError("residual stream, iteration and group counts and gate scale must be positive")
        if self.width < 24 or (self.width % self.heads and not self.attn_head_dim) or self.head_dim % 2 \
                or self.attn_head_dim < 0:
            raise ValueError("width >= 24 divisible by heads with an even head dimension required")
        if self.kv_heads < 0 or (self.kv_heads and self.heads % self.kv_heads):
            raise ValueError("kv_heads must divide heads")
        if min(self.layers, self.core_layers, self.loops, self.max_loops, self.sequence_len, self.mlp_width,
               self.vocab_size, self.sparse_topk, self.block_size, self.compression_size, self.index_dim,
               self.slots, self.reference_chunk) <= 0:
            raise ValueError("dimensions and counts must be positive")
        if min(self.pre_layers, self.post_layers, self.burnin_steps, self.compression_stride) < 0:
            raise ValueError("negative stage depth or stride")
        if self.sliding_window <= 0:
            raise ValueError("sliding window must contain the current token")
        if self.value_embeds not in (-1, 0, 1):
            raise ValueError("value_embeds is -1 (method rule), 0 or 1")

    def _check_method_rules(self):
        if self.method in FULL_ATTENTION and self.window_pattern != "L":
            raise ValueError(f"{self.method} uses full causal attention in every layer (window_pattern L)")
        if self.method in HYBRID:
            if self.window_pattern != "L":
                raise ValueError(f"{self.method} sets attention windows per layer (window_pattern L)")
            hybrid_layout(self.method, self.layers)
        if self.method in MLA_CONFIG:
            if min(self.q_rank, self.kv_rank, self.qk_nope_dim, self.v_head_dim) <= 0 or self.qk_rope_dim != 0:
                raise ValueError("MLA-NoPE requires positive latent/head dimensions and zero RoPE dimensions")
            if self.scale == "formal" and (self.q_rank, self.kv_rank, self.qk_nope_dim, self.v_head_dim) != \
                    (768, 256, 128, 128):
                raise ValueError("formal MLA-NoPE keeps ranks (768, 256) and head dimensions (128, 128)")
        if self.method == "attnres" and self.attnres_groups > self.layers:
            raise ValueError("AttnRes needs at least one block per group")
        if not 0 < self.act_epsilon < 1 or not 0 < self.ouro_exit_quantile <= 1:
            raise ValueError("invalid halting threshold")
        if self.huginn_mean <= 1 or not 0 < self.huginn_backprop_loops <= self.max_loops:
            raise ValueError("invalid Huginn depth distribution")
        if self.index_rope_dim % 2 or not 0 <= self.index_rope_dim <= self.index_dim:
            raise ValueError("invalid partial RoPE size")
        if self.backend not in ("reference", *CHUNK_BACKENDS):
            raise ValueError("unknown chunk backend")
        if self.backend in CHUNK_BACKENDS and self.method not in CHUNKED_METHODS:
            raise ValueError("chunked backend applies to DeltaNet, KDA, RetNet, ELU+1, GDN and hybrids")
        if self.scale not in ("formal", "debug", "custom"):
            raise ValueError("scale must be formal, debug or custom")
        if self.scale == "formal":
            if (self.width, self.heads, self.vocab_size, self.sequence_len) != (1536, 12, 32768, 2048):
                raise ValueError("formal configurations keep the d24 shell dimensions")
            if not 3 * self.width <= self.mlp_width <= 5 * self.width or self.mlp_width % 128:
                raise ValueError("formal FFN width lies on the 3d..5d, multiple-of-128 grid")
            if self.kv_heads not in (0, self.heads) or self.method in MOE:
                raise ValueError("the formal shell is multi-head attention without experts")
        if self.method in MOE:
            if not 0 < self.moe_topk <= self.moe_experts or self.moe_ffn <= 0 or self.moe_shared < 0 \
                    or self.moe_aux_loss_coeff < 0 or self.moe_z_loss_coeff < 0:
                raise ValueError("invalid MoE shape")
        if self.method in PLUGINS:
            from nexttransformer_b200.models.plugins import load
            check = load(self.method).check
            if check:
                check(self)

    # ------------------------------------------------------------------ derived
    def option(self, name):
        return dict(self.options)[name]

    @property
    def head_dim(self):
        return self.attn_head_dim or self.width // self.heads

    @property
    def n_embd(self):
        return self.width

    @property
    def n_head(self):
        return self.heads

    @property
    def n_kv_head(self):
        return self.kv_heads or self.heads

    @property
    def value_embeddings(self):
        if self.value_embeds >= 0:
            return bool(self.value_embeds)
        return self.method not in NO_VE

    @property
    def layer_mixers(self):
        if self.method not in HYBRID:
            raise ValueError(f"{self.method} is not a per-layer hybrid")
        return hybrid_layout(self.method, self.layers)

    @property
    def has_sparse(self):
        kinds = self.layer_mixers if self.method in HYBRID else (self.method,)
        return any(k in SPARSE for k in kinds)

    @property
    def has_sparse_burnin(self):
        kinds = self.layer_mixers if self.method in HYBRID else (self.method,)
        return any(k in ("dsa", "qsa", "seer") for k in kinds)

    @property
    def n_layer(self):
        if self.method in LOOPED:
            return self.pre_layers + self.core_layers + self.post_layers
        return self.layers

    @property
    def maximum_depth(self):
        if self.method not in LOOPED:
            return self.layers
        n = self.max_loops if self.method in ("ut_act", "huginn", "ouro") else self.loops
        return self.pre_layers + n * self.core_layers + self.post_layers

    @property
    def attnres_group_sizes(self):
        q, r = divmod(self.layers, self.attnres_groups)
        return (q + 1,) * r + (q,) * (self.attnres_groups - r)

    @property
    def attnres_group_starts(self):
        starts = [0]
        for s in self.attnres_group_sizes[:-1]:
            starts.append(starts[-1] + s)
        return tuple(starts)

    # ------------------------------------------------------------------ serialisation
    def serialized(self):
        data = asdict(self)
        for name, users in SCOPED_FIELDS.items():
            if self.method not in users:
                data.pop(name)
        defaults = {f.name: f.default for f in fields(self)}
        for name in EXTENSION_FIELDS:
            if data[name] == defaults[name]:
                data.pop(name)
        if self.method in HYBRID:
            data["layer_mixers"] = list(self.layer_mixers)

        def thaw(v):
            return [thaw(x) for x in v] if isinstance(v, tuple) else v
        if self.options:
            data["options"] = {k: thaw(v) for k, v in self.options}
        else:
            data.pop("options")
        return data

    @property
    def fingerprint(self):
        return hashlib.sha256(json.dumps(self.serialized(), sort_keys=True).encode()).hexdigest()


def config_from_dict(raw):
    """Rebuild a configuration from its JSON form (lists back to tuples; layer layout dropped)."""
    raw = dict(raw)
    raw.pop("layer_mixers", None)
    names = {f.name for f in fields(ModelConfig)}
    for k in list(raw):
        if k not in names:
            raise ValueError(f"unknown configuration field {k!r}")
        if isinstance(raw[k], list):
            raw[k] = tuple(raw[k])
    return ModelConfig(**raw)


_CANDIDATE_CHANGES = {
    "ut_act": dict(core_layers=6), "huginn": dict(core_layers=8, max_loops=4), "ouro": dict(core_layers=4),
    "deeploop": dict(pre_layers=0, post_layers=0, core_layers=12),
    "nsa": dict(block_size=32, compression_size=32), "seer": dict(block_size=64),
    "elu_norm": dict(backend="fla_chunk64"), "elu_qknorm": dict(backend="fla_chunk64"), "gdn": dict(backend="fla_chunk64"),
    "deltanet_hybrid": dict(backend="fla_chunk64", window_pattern="L"),
    "gdn_hybrid": dict(backend="fla_chunk64", window_pattern="L"),
    "gdn_hybrid_swa": dict(backend="fla_chunk64", window_pattern="L"),
    "kda_hybrid": dict(backend="fla_chunk64", window_pattern="L", qk_nope_dim=128, qk_rope_dim=0),
    "qsa_hybrid": dict(backend="fla_chunk64", window_pattern="L"),
    "moba_hybrid": dict(window_pattern="L"), "kda_no_ve": dict(backend="fla_chunk64"),
    "mla_nope": dict(qk_nope_dim=128, qk_rope_dim=0),
}


def candidate_config(method):
    """The registered starting configuration of a method at formal scale."""
    if method in PLUGINS:
        spec = PLUGINS[method]
        shell = {"layers": 24, "mlp_width": 6144, "window_pattern": "L", **spec.get("shell", {})}
        return ModelConfig(method=method, options=spec.get("options", {}), **shell)
    if method in MOE:
        return ModelConfig(method=method, scale="custom", window_pattern="L")
    changes = dict(_CANDIDATE_CHANGES.get(method, {}))
    if method in FULL_ATTENTION:
        changes["window_pattern"] = "L"
    return ModelConfig(method=method, **changes)


def debug_config(method, *, width=48, sequence_len=12):
    """A tiny configuration of `method` for CPU tests (dimensions kept off the chunk length)."""
    c = candidate_config(method)
    plugin = PLUGINS.get(method)
    mult = LAYER_MULTIPLE.get(method, 2 if not plugin else 1)
    if plugin:
        layers = mult * (2 if mult == 1 else 1)
    elif method == "attnres":
        layers = 3
    elif method in ("deltanet_hybrid", "moba_hybrid"):
        layers = 4
    else:
        layers = LAYER_MULTIPLE.get(method, 2)
    extra = {}
    if plugin:
        extra["options"] = dict(c.options, **plugin.get("debug_options", {}))
    if method == "attnres":
        extra["attnres_groups"] = 2
    if method in MLA_CONFIG:
        extra.update(q_rank=20, kv_rank=8, qk_nope_dim=16, qk_rope_dim=0, v_head_dim=16)
    if method == "gdn_hybrid_swa":
        extra["sliding_window"] = 4
    if method in MOE:
        extra.update(moe_experts=4, moe_topk=2, moe_ffn=32, moe_dense_layers=1)
    return replace(c, scale="debug", width=width, heads=2, vocab_size=96 if c.backend in CHUNK_BACKENDS else 64,
                   sequence_len=sequence_len, mlp_width=4 * width, layers=layers,
                   pre_layers=0 if method == "deeploop" else 1, core_layers=1,
                   post_layers=0 if method == "deeploop" else 1, index_dim=8, index_heads=2, index_rope_dim=4,
                   slots=4, block_size=4, compression_size=2, sparse_topk=4, local_window=4, reference_chunk=4,
                   gate_rank=4, **extra)
