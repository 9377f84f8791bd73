"""Model and engine configuration.

Two model configs are defined here:

* ``full_config()`` -- the GLM-5.3-Flash architecture as the reference serves it: 45 decoder layers (34 KDA
  linear-attention, 11 MLA/DSA sparse-attention; layers 0-2 are KDA with a dense MLP, then the pattern
  (MLA, KDA, KDA, KDA) with MoE), hidden 4096, vocab 154,880, 4 mHC residual streams, 288 routed experts top-8 plus
  one shared expert of width 2048, EXL3 4-bpw routed experts.  Dimensions follow the reference's model notes
  (code/fork/docs/DESIGN.md:77-79, code/fork/docs/ref/tf_weights.py:44-115, code/fork/fp8_gemv.py:68-90).
* ``tiny_config()`` -- the CPU proxy used as the correctness oracle: 4 layers (3 KDA with 4 heads x 64, then one
  MLA/DSA layer with 8 heads, kv_lora 128, qk_nope 64, qk_rope 32, v_head 64, DSA top-k 64), hidden 512, 16 routed
  experts of width 256 + 1 shared, sigmoid top-4, 2 mHC streams, vocab 4096.

DSA selection rule used by this engine: keys are pooled ``kpool`` at a time; a query at position t always sees its
own (possibly partial) pool and the top ``index_topk // kpool - 1`` complete earlier pools.  A query therefore sees
every key while t < ``index_topk`` (``dense_limit``) and at most ``index_topk`` keys after that.
"""

from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field


@dataclass
class ModelConfig:
    name: str
    hidden: int
    vocab: int
    eps: float
    # layer plan
    layer_kinds: list[str]          # per layer: "kda" or "mla"
    mlp_kinds: list[str]            # per layer: "dense" or "moe"
    # MLA / DSA
    heads: int
    q_lora: int
    kv_lora: int
    qk_nope: int
    qk_rope: int
    v_dim: int
    index_heads: int
    index_dim: int
    index_topk: int
    kpool: int
    # KDA
    lin_heads: int
    lin_dim: int
    conv: int
    lower: float
    # MLP / MoE
    dense_width: int
    experts: int
    top_k: int
    moe_width: int
    shared_experts: int
    routed_scale: float
    norm_topk: bool
    limit: float
    # mHC
    streams: int
    hc_iters: int
    hc_eps: float
    # vocabulary / quant
    eos: tuple[int, ...] = ()
    bits: int = 4                    # EXL3 bits per weight of the routed experts
    rope_theta: float = 10000.0
    extra: dict = field(default_factory=dict)

    # ---- derived -----------------------------------------------------------------------------------------
    @property
    def layers(self) -> int:
        return len(self.layer_kinds)

    @property
    def qk_dim(self) -> int:
        return self.qk_nope + self.qk_rope

    @property
    def shared_width(self) -> int:
        return self.moe_width * self.shared_experts

    @property
    def n_mix(self) -> int:
        """mHC mixing logits: S pre + S post + S*S comb."""
        return 2 * self.streams + self.streams * self.streams

    @property
    def kda_proj_width(self) -> int:
        """in_proj rows: [q | k | v | f_a | g_a | b] (3*H*Dh + Dh + Dh + H)."""
        return 3 * self.lin_heads * self.lin_dim + 2 * self.lin_dim + self.lin_heads

    @property
    def dense_limit(self) -> int:
        return self.index_topk

    @property
    def pools_selected(self) -> int:
        return self.index_topk // self.kpool

    def kda_layers(self) -> list[int]:
        return [i for i, k in enumerate(self.layer_kinds) if k == "kda"]

    def mla_layers(self) -> list[int]:
        return [i for i, k in enumerate(self.layer_kinds) if k == "mla"]

    def moe_layers(self) -> list[int]:
        return [i for i, k in enumerate(self.mlp_kinds) if k == "moe"]

    def kv_bytes_per_token(self) -> float:
        """Device bytes per token slot of the paged caches, summed over the MLA/DSA layers: the fp8 latent and its
        fp32 scale, the bf16 rope key, and the token's share of its pool's fp8 index key and fp32 scale. The same on
        every tensor-parallel rank (the latent cache is not split by heads)."""
        per_layer = self.kv_lora + 4 + 2 * max(self.qk_rope, 1) + (self.index_dim + 4) / self.kpool
        return len(self.mla_layers()) * per_layer

    def validate(self, tp: int = 1) -> None:
        assert len(self.layer_kinds) == len(self.mlp_kinds)
        assert all(k in ("kda", "mla") for k in self.layer_kinds)
        assert all(k in ("dense", "moe") for k in self.mlp_kinds)
        assert self.heads % tp == 0 and self.lin_heads % tp == 0, "heads must divide over tp"
        assert self.moe_width % (tp * 128) == 0 or tp == 1, "EXL3 expert width must split in whole 128-blocks"
        assert self.dense_width % tp == 0 and self.vocab % tp == 0
        assert self.hidden % 128 == 0 and self.moe_width % 128 == 0, "EXL3 Hadamard blocks are 128 wide"
        assert self.index_topk % self.kpool == 0

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self), indent=1)

    @classmethod
    def from_json(cls, s: str) -> "ModelConfig":
        d = json.loads(s)
        d["eos"] = tuple(d.get("eos", ()))
        return cls(**d)


def glm53_layer_plan(n_layers: int = 45, first_dense: int = 3, mla_every: int = 4) -> tuple[list[str], list[str]]:
    """Layers 0..first_dense-1: KDA + dense MLP; then (MLA, KDA, KDA, KDA) + MoE repeated, so MLA sits at
    first_dense, first_dense + 4, ... (code/fork/tests/roof/sim_step.py:13)."""
    kinds, mlps = [], []
    for i in range(n_layers):
        if i < first_dense:
            kinds.append("kda")
            mlps.append("dense")
        else:
            kinds.append("mla" if (i - first_dense) % mla_every == 0 else "kda")
            mlps.append("moe")
    return kinds, mlps


def full_config(layers: int = 45) -> ModelConfig:
    kinds, mlps = glm53_layer_plan(layers)
    return ModelConfig(
        name="glm-5.3-flash", hidden=4096, vocab=154880, eps=1e-5,
        layer_kinds=kinds, mlp_kinds=mlps,
        heads=64, q_lora=1536, kv_lora=512, qk_nope=256, qk_rope=0, v_dim=256,
        index_heads=32, index_dim=128, index_topk=2048, kpool=4,
        lin_heads=64, lin_dim=128, conv=4, lower=-5.0,
        dense_width=12288, experts=288, top_k=8, moe_width=2048, shared_experts=1,
        routed_scale=2.5, norm_topk=True, limit=10.0,
        streams=4, hc_iters=20, hc_eps=1e-6,
        eos=(154820, 154827, 154829), bits=4,
    )


def tiny_config() -> ModelConfig:
    """the CPU proxy (3 KDA layers then 1 MLA/DSA layer; layer 0 dense MLP, rest MoE)."""
    kinds = ["kda", "kda", "kda", "mla"]
    mlps = ["dense", "moe", "moe", "moe"]
    return ModelConfig(
        name="glm53-tiny", hidden=512, vocab=4096, eps=1e-5,
        layer_kinds=kinds, mlp_kinds=mlps,
        heads=8, q_lora=256, kv_lora=128, qk_nope=64, qk_rope=32, v_dim=64,
        index_heads=4, index_dim=128, index_topk=64, kpool=4,
        lin_heads=4, lin_dim=64, conv=4, lower=-5.0,
        dense_width=1024, experts=16, top_k=4, moe_width=256, shared_experts=1,
        routed_scale=1.0, norm_topk=True, limit=10.0,
        streams=2, hc_iters=20, hc_eps=1e-6,
        eos=(), bits=4,
    )


def config_by_name(name: str) -> ModelConfig:
    if name in ("full", "glm-5.3-flash", "glm53"):
        return full_config()
    if name in ("tiny", "glm53-tiny"):
        return tiny_config()
    raise KeyError(name)
