"""Architecture and cost estimates of the 2K-sequence scaling expert families (Vanilla MoE, Hybrid
KDA-DSA, Looped), after ``nexttransformer/scaling/moe_recipe.py`` of the reference.

The three families share one feed-forward recipe: a dense first layer (4 d ReLU^2), then per layer
256 routed experts of width d / 4 with top-8 selection plus one always-on shared expert of the same
width.  ``MoERecipe`` validates a cell, counts its parameters (total and active per token) and
estimates the updates its FLOP budget buys; ``load_t3_recipe`` reads a cell of the T3 manifest and
refuses a manifest whose shared feed-forward keys changed.  The counting formulas are the
reference's (the estimates must agree with the published manifest); the code is this module's.
Nothing here needs a GPU or Megatron: on B200 the routed layer is ``models.moe`` (grouped sm_100a
expert GEMMs, peer-memory expert exchange).
"""
from dataclasses import asdict, dataclass, replace
import json
import math
from pathlib import Path

SHARED_FFN_RECIPE = {"firstLayerDense": True, "ffn": "ReLU²", "routedExperts": 256, "selectedExperts": 8,
                     "sharedExperts": 1, "expertWidthDivisor": 4}
FULL_ATTENTION = ("moe", "looped")
EXPERT_FAMILIES = FULL_ATTENTION + ("kda-dsa",)
ATTENTION_NOTE = {"moe": "native full causal MHA; no VE",
                  "looped": "native full causal MHA, shared core executed twice; no VE",
                  "kda-dsa": "three KDA mixers then one DSA mixer; no VE"}
MANIFEST = Path(__file__).resolve().parents[2] / "configs" / "scaling" / "t3.json"


@dataclass(frozen=True)
class MoERecipe:
    layers: int
    width: int
    heads: int
    vocab_size: int = 32768
    sequence_len: int = 2048
    routed_experts: int = 256
    top_k: int = 8
    expert_width: int = None
    seed: int = 42
    global_batch_tokens: int = 1048576
    training_flops: int = 10 ** 20
    cell_id: str = ""
    aux_loss_coeff: float = 0.01
    z_loss_coeff: float = 0.001
    router_init_std: float = 0.02
    family: str = "moe"
    unique_layers: int = None     # layers with their own weights (Looped stores its core once)
    loops: int = 1

    def __post_init__(self):
        if self.expert_width is None:
            object.__setattr__(self, "expert_width", self.width // 4)
        if self.unique_layers is None:
            object.__setattr__(self, "unique_layers", self.layers)
        problems = []
        if self.family not in EXPERT_FAMILIES:
            problems.append(f"not a T3 expert family: {self.family}")
        if self.loops < 1 or not 2 <= self.unique_layers <= self.layers:
            problems.append("unique layers must be between two and the executed depth")
        dims = (self.layers, self.width, self.heads, self.vocab_size, self.sequence_len, self.routed_experts,
                self.expert_width, self.global_batch_tokens, self.training_flops)
        if min(dims) <= 0:
            problems.append("model dimensions and budgets must be positive")
        elif self.layers < 2 or self.width < 24 or self.width % self.heads or self.width % 4:
            problems.append("MoE needs >=2 layers, width>=24 divisible by heads and four")
        elif (self.width // self.heads) % 2 or self.expert_width != self.width // 4:
            problems.append("even head dimension and two-matrix d/4 experts are required")
        if not 1 <= self.top_k <= self.routed_experts:
            problems.append("top-k must fit the expert count")
        if self.sequence_len > 0 and self.global_batch_tokens % self.sequence_len:
            problems.append("batch must contain whole sequences")
        if not all(math.isfinite(c) and c >= 0 for c in (self.aux_loss_coeff, self.z_loss_coeff)):
            problems.append("routing loss coefficients must be finite and nonnegative")
        if not (math.isfinite(self.router_init_std) and self.router_init_std > 0):
            problems.append("router initialization standard deviation must be positive")
        if problems:
            raise ValueError(problems[0])

    # parameters of one expert (up and down matrices of width d/4)
    def _expert(self):
        return 2 * self.width * self.expert_width

    def block_active(self):
        """Parameters one token activates over the executed depth (attention 4 d^2 per layer, the dense
        first FFN 8 d^2, then top-k routed plus the shared expert and the router per later layer)."""
        if self.family not in FULL_ATTENTION:
            raise ValueError(f"{self.family} attention needs its own cost proof")
        d, later = self.width, self.layers - 1
        return 4 * self.layers * d * d + 8 * d * d + later * ((self.top_k + 1) * self._expert() + d * self.routed_experts)

    def describes_capacity(self):
        return self.family in FULL_ATTENTION and self.unique_layers == self.layers

    def counts(self):
        if not self.describes_capacity():
            raise ValueError(f"{self.family} capacity needs its own accounting")
        d, later = self.width, self.layers - 1
        blocks = (4 * self.layers * d * d + 8 * d * d + later * (self.routed_experts + 1) * self._expert()
                  + later * d * self.routed_experts)
        small = 2 * self.layers + 26                       # residual / x0 / smear / backout scalars
        io = 2 * d * (-(-self.vocab_size // 64) * 64)      # embedding + head, vocabulary padded to 64
        return {"block_total": blocks, "block_active": self.block_active(), "embedding_and_head": io,
                "native_small_parameters": small, "model_total": blocks + io + small}

    def estimate(self):
        if self.family not in FULL_ATTENTION:
            return {"flops_per_token_main_term": None, "estimated_updates": None, "estimated_tokens": None,
                    "cost_proof_complete": False}
        d = self.width
        per_token = 6 * self.block_active() + 12 * self.sequence_len * d * self.layers + 6 * d * self.vocab_size
        updates = round(self.training_flops / (per_token * self.global_batch_tokens))
        return {"flops_per_token_main_term": per_token, "estimated_updates": updates,
                "estimated_tokens": updates * self.global_batch_tokens, "cost_proof_complete": False}

    def manifest(self):
        return {"protocol": "nextt-scale-2k-v1", "recipe": asdict(self),
                "counts": self.counts() if self.describes_capacity() else None, "estimate": self.estimate(),
                "attention": ATTENTION_NOTE[self.family],
                "ffn": "first dense 4d; then routed top-k plus one shared d/4; ReLU squared",
                "optimizer": "native Muon + AdamW; AdamW router",
                "routing_status": "pilot coefficients; not frozen for formal training",
                "expert_layer": "models.moe grouped sm_100a GEMMs", "formal_training_ready": False}

    def debug(self, routed_experts=8, top_k=2):
        """A CPU-sized cell of the same family: one block per role."""
        shape = dict(layers=2 + self.loops, unique_layers=3) if self.loops > 1 else dict(layers=3, unique_layers=3)
        return replace(self, width=32, heads=2, vocab_size=64, sequence_len=8, routed_experts=routed_experts,
                       top_k=top_k, expert_width=8, global_batch_tokens=32, cell_id=self.cell_id + "-cpu-debug",
                       **shape)


def load_t3_recipe(cell_id="moe-T3-L20", path=None):
    data = json.loads(Path(path or MANIFEST).read_text())
    cells = [c for c in data["cells"] if c["id"] == cell_id and c["family"] in EXPERT_FAMILIES]
    if not cells:
        raise ValueError(f"unknown T3 expert cell: {cell_id}")
    cell = cells[0]
    rule = next(f["recipe"] for f in data["families"] if f["id"] == cell["family"])
    shared = {k: v for k, v in rule.items() if k in SHARED_FFN_RECIPE}
    if shared != SHARED_FFN_RECIPE or data["valueEmbeddings"] or data["protocol"] != "nextt-scale-2k-v1":
        raise ValueError("the shared T3 expert recipe changed; review the adapter before using it")
    loops = rule.get("loops", 1)
    unique = cell["preLayers"] + cell["coreLayers"] + cell["postLayers"] if loops > 1 else cell["layers"]
    return MoERecipe(layers=cell["layers"], width=cell["width"], heads=cell["heads"], vocab_size=data["vocabSize"],
                     sequence_len=data["sequenceLength"], seed=data["seed"],
                     global_batch_tokens=data["globalBatchTokens"], training_flops=data["trainingFlops"],
                     expert_width=cell["expertWidth"], cell_id=cell_id, family=cell["family"],
                     unique_layers=unique, loops=loops)
