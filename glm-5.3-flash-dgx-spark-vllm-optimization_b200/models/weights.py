"""Checkpoint layout, random initialisation, load-time quantisation and tensor-parallel sharding.

Checkpoint layout (HF names, the reference's tensor names: code/fork/docs/ref/tf_weights.py:294-399):

  model.embed_tokens.weight                                  bf16 [V, D]
  model.layers.{i}.input_layernorm.weight / post_attention_layernorm.weight      [D]
  model.layers.{i}.hc_{attn,ffn}_{fn,base,scale}             [n_mix, S*D], [n_mix], [3]
  KDA  model.layers.{i}.self_attn.{q,k,v,f_a,g_a,b}_proj.weight, f_b_proj, g_b_proj, {q,k,v}_conv1d.weight,
       A_log [H], dt_bias [H*Dh], o_norm.weight [Dh], o_proj.weight
  MLA  self_attn.q_a_proj, q_a_layernorm, q_b_proj, kv_a_proj_with_mqa, kv_a_layernorm, kv_b_proj, o_proj;
       self_attn.indexer.{wq_b, wk, k_norm.{weight,bias}, weights_proj, index_kpool_compress_gate,
       index_kpool_compress_ape}
  MoE  mlp.gate.weight [E, D], mlp.gate.e_score_correction_bias [E],
       mlp.experts.{e}.{gate,up,down}_proj.{trellis,suh,svh,mcg}  (EXL3), mlp.shared_experts.{gate,up,down}_proj
  MLP  mlp.{gate,up,down}_proj.weight (dense layers)
  model.norm.weight, lm_head.weight

At load (``prepare``) every dense projection is quantised to fp8 e4m3 with one fp32 scale per output channel (the
reference production does the same: code/fork/docs/prod_exl3_reference.py:1916-2033); the EXL3 experts keep their
trellis; router, norms, mHC mixers, KDA gates and the embedding stay bf16/fp32.  ``prepare`` also shards for
tensor parallelism: heads, MLP/expert widths and vocabulary rows are split; o_proj / down_proj are row-parallel.
"""

from __future__ import annotations

import hashlib
import json
import math
import os
from dataclasses import dataclass, field
from typing import Callable

import torch

from ..config import ModelConfig
from ..ops import exl3 as exl3_ops

P = "model."
FP8_MAX = 448.0


# ---------------------------------------------------------------------------------------------------------------
# prepared (runtime) weight containers
# ---------------------------------------------------------------------------------------------------------------
@dataclass
class Linear8:
    """fp8 e4m3 weight [N, K] (stored as uint8) with an fp32 scale per output row: W = w8 * scale[:, None]."""
    w: torch.Tensor
    s: torch.Tensor

    @property
    def n(self) -> int:
        return self.w.shape[-2]

    @property
    def k(self) -> int:
        return self.w.shape[-1]

    def dequant(self) -> torch.Tensor:
        return self.w.view(torch.float8_e4m3fn).float() * self.s.float()[..., None]

    def to(self, device) -> "Linear8":
        return Linear8(self.w.to(device), self.s.to(device))


@dataclass
class Exl3Stack:
    """EXL3 linears of E experts: trellis int16 [E, K/16, N/16, 64], suh fp16 [E, K], svh fp16 [E, N]."""
    trellis: torch.Tensor
    suh: torch.Tensor
    svh: torch.Tensor

    @property
    def k(self) -> int:
        return self.suh.shape[-1]

    @property
    def n(self) -> int:
        return self.svh.shape[-1]

    def to(self, device) -> "Exl3Stack":
        return Exl3Stack(self.trellis.to(device), self.suh.to(device), self.svh.to(device))


@dataclass
class HCW:
    fn: torch.Tensor          # bf16 [n_mix, S*D]
    base: torch.Tensor        # fp32 [n_mix]
    scale: torch.Tensor       # fp32 [3]


@dataclass
class KDAW:
    in_proj: Linear8          # [q | k | v | f_a | g_a | b] local rows
    f_b: Linear8              # [Hl*Dh, Dh]
    g_b: Linear8
    conv: torch.Tensor        # fp32 [3*Hl*Dh, taps]
    a_log: torch.Tensor       # fp32 [Hl]
    dt_bias: torch.Tensor     # fp32 [Hl*Dh]
    o_norm: torch.Tensor      # bf16 [Dh]
    o_proj: Linear8           # [D, Hl*Dh]
    heads: int


@dataclass
class IndexW:
    proj: torch.Tensor        # bf16 [ID + IH + ID, D]: wk | weights_proj | kpool gate  (fp32 outputs)
    wq_b: Linear8             # [IH*ID, q_lora]
    ln_w: torch.Tensor        # fp32 [ID]
    ln_b: torch.Tensor        # fp32 [ID]
    ape: torch.Tensor         # fp32 [kpool, ID]


@dataclass
class MLAW:
    qkv_a: Linear8            # [q_lora + kv_lora + rope, D]  (replicated)
    q_norm: torch.Tensor      # bf16 [q_lora]
    kv_norm: torch.Tensor     # bf16 [kv_lora]
    q_b: Linear8              # [Hl*qk, q_lora]
    w_uk_t: Linear8           # [Hl, kv_lora, nope]   (absorbed key up-projection, transposed per head)
    w_uv: Linear8             # [Hl, v, kv_lora]
    o_proj: Linear8           # [D, Hl*v]
    index: IndexW
    heads: int
    full: "MLAFull | None" = None   # all heads' query / output projections (row-parallel prefill), when kept


@dataclass
class MLAFull:
    """The head-dependent MLA projections of every head (the same fp8 bits as the tensor-parallel shards): with
    sequence-parallel prefill a rank runs the attention of its own rows over all heads, so the block needs no
    cross-rank reduction and the per-row key gathers are divided by the world size."""
    q_b: Linear8              # [H*qk, q_lora]
    w_uk_t: Linear8           # [H, kv_lora, nope]
    w_uv: Linear8             # [H, v, kv_lora]
    o_proj: Linear8           # [D, H*v]


@dataclass
class MLPW:
    gu: Linear8               # [2*Wl, D]  (gate rows then up rows)
    down: Linear8             # [D, Wl]
    width: int


@dataclass
class MoEW:
    router: torch.Tensor      # bf16 [E, D]
    bias: torch.Tensor        # fp32 [E]
    gate: Exl3Stack           # [E] D -> Wl
    up: Exl3Stack
    down: Exl3Stack           # [E] Wl -> D
    shared: MLPW


@dataclass
class LayerW:
    index: int
    kind: str
    mlp_kind: str
    attn_hc: HCW
    ffn_hc: HCW
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    kda: KDAW | None = None
    mla: MLAW | None = None
    mlp: MLPW | None = None
    moe: MoEW | None = None


@dataclass
class Weights:
    cfg: ModelConfig
    embed: torch.Tensor       # bf16 [V, D] (replicated)
    layers: list[LayerW]
    norm: torch.Tensor        # bf16 [D]
    head: Linear8             # [V/world, D]
    rank: int = 0
    world: int = 1
    meta: dict = field(default_factory=dict)

    @property
    def device(self) -> torch.device:
        return self.embed.device

    def nbytes(self) -> int:
        seen, total = set(), 0

        def add(o):
            nonlocal total
            if isinstance(o, torch.Tensor):
                if o.data_ptr() not in seen:
                    seen.add(o.data_ptr())
                    total += o.numel() * o.element_size()
            elif isinstance(o, (list, tuple)):
                for v in o:
                    add(v)
            elif hasattr(o, "__dataclass_fields__"):
                for k in o.__dataclass_fields__:
                    add(getattr(o, k))
        add(self.embed)
        add(self.layers)
        add(self.norm)
        add(self.head)
        return total


# ---------------------------------------------------------------------------------------------------------------
# quantisation helpers
# ---------------------------------------------------------------------------------------------------------------
def quantize_fp8_rows(w: torch.Tensor) -> Linear8:
    """Per-output-row e4m3 quantisation: scale = amax / 448 (1 when the row is zero)."""
    wf = w.float()
    amax = wf.abs().amax(dim=-1).clamp_min(1e-12)
    s = amax / FP8_MAX
    q = (wf / s[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return Linear8(q.view(torch.uint8).contiguous(), s.float().contiguous())


# ---------------------------------------------------------------------------------------------------------------
# tensor sources: a checkpoint directory, a dict, or a seeded random generator
# ---------------------------------------------------------------------------------------------------------------
class TensorSource:
    def get(self, name: str) -> torch.Tensor:
        raise NotImplementedError

    def experts(self, layer: int, proj: str, n_experts: int) -> Exl3Stack:
        base = f"{P}layers.{layer}.mlp.experts."
        tr = torch.stack([self.get(f"{base}{e}.{proj}.trellis") for e in range(n_experts)])
        su = torch.stack([self.get(f"{base}{e}.{proj}.suh") for e in range(n_experts)])
        sv = torch.stack([self.get(f"{base}{e}.{proj}.svh") for e in range(n_experts)])
        return Exl3Stack(tr, su, sv)


class DictSource(TensorSource):
    def __init__(self, d: dict[str, torch.Tensor]):
        self.d = d

    def get(self, name):
        return self.d[name]


class OverrideSource(TensorSource):
    """A source with some tensors replaced at load (the reference's o_proj transplant of layers 15-45,
    README.md:43, data/ablit_transplant_sha256.csv): ``overrides`` maps a checkpoint name to a tensor or to a
    ``.pt`` / ``.safetensors`` file holding it; ``sha256`` (optional) maps the same names to the expected digest of the
    file bytes, and a mismatch refuses to load.  Shapes must match the base tensor."""

    def __init__(self, base: TensorSource, overrides: dict, sha256: dict | None = None):
        self.base, self.overrides, self.sha256 = base, dict(overrides), dict(sha256 or {})
        for k in ("cfg", "device", "shapes"):
            if hasattr(base, k):
                setattr(self, k, getattr(base, k))

    @staticmethod
    def _digest(path: str) -> str:
        import hashlib
        h = hashlib.sha256()
        with open(path, "rb") as f:
            for blk in iter(lambda: f.read(1 << 20), b""):
                h.update(blk)
        return h.hexdigest()

    def get(self, name):
        if name not in self.overrides:
            return self.base.get(name)
        v = self.overrides[name]
        if isinstance(v, str):
            if name in self.sha256 and self._digest(v) != self.sha256[name].lower():
                raise ValueError(f"override for {name}: sha256 mismatch ({v})")
            if v.endswith(".safetensors"):
                from safetensors.torch import load_file
                d = load_file(v)
                v = d[name] if name in d else next(iter(d.values()))
            else:
                v = torch.load(v, map_location="cpu", weights_only=True)
        ref = self.base.get(name)
        if tuple(v.shape) != tuple(ref.shape):
            raise ValueError(f"override for {name}: shape {tuple(v.shape)} != {tuple(ref.shape)}")
        return v.to(ref.dtype)

    def experts(self, layer, proj, n_experts):
        if not any(k.startswith(f"{P}layers.{layer}.mlp.experts.") for k in self.overrides):
            return self.base.experts(layer, proj, n_experts)
        return TensorSource.experts(self, layer, proj, n_experts)


class SafetensorsSource(TensorSource):
    """Reads a (sharded) safetensors checkpoint directory lazily, tensor by tensor."""

    def __init__(self, path: str):
        from safetensors import safe_open
        self.path = path
        self.index: dict[str, str] = {}
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                wm = json.load(f)["weight_map"]
            self.index = {k: os.path.join(path, v) for k, v in wm.items()}
        else:
            for fn in sorted(os.listdir(path)):
                if fn.endswith(".safetensors"):
                    full = os.path.join(path, fn)
                    with safe_open(full, "pt") as f:
                        for k in f.keys():
                            self.index[k] = full
        self._open: dict[str, object] = {}

    def get(self, name):
        from safetensors import safe_open
        fn = self.index[name]
        h = self._open.get(fn)
        if h is None:
            h = safe_open(fn, "pt")
            self._open[fn] = h
        return h.get_tensor(name)


def _seed_of(seed: int, name: str) -> int:
    return int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little") & ((1 << 62) - 1)


class RandomSource(TensorSource):
    """Deterministic random-init weights of the architecture: every tensor is drawn from a generator seeded by
    (seed, tensor name), so a tensor does not depend on which others were drawn before it.  Distributions keep
    activations O(1) through the stack: linears N(0, 1/fan_in), router logits ~N(0, 1), EXL3 weights with std
    1/sqrt(K) (random trellis words; random-sign suh/svh), norms 1 + N(0, 0.05)."""

    def __init__(self, cfg: ModelConfig, seed: int = 0, device: str | torch.device = "cpu"):
        self.cfg = cfg
        self.seed = seed
        self.device = torch.device(device)
        self.shapes = checkpoint_shapes(cfg)

    def _gen(self, name):
        g = torch.Generator(device=self.device)
        g.manual_seed(_seed_of(self.seed, name))
        return g

    def get(self, name):
        c = self.cfg
        shape, kind = self.shapes[name]
        g = self._gen(name)
        dev = self.device

        def randn(std, dtype=torch.bfloat16):
            return (torch.randn(shape, generator=g, device=dev) * std).to(dtype)

        if kind == "linear":
            return randn(1.0 / math.sqrt(shape[-1]))
        if kind == "embed":
            return randn(1.0)
        if kind == "norm":
            return (1.0 + torch.randn(shape, generator=g, device=dev) * 0.05).to(torch.bfloat16)
        if kind == "zero_f32":
            return torch.zeros(shape, device=dev)
        if kind == "hc_fn":
            return randn(1.0 / math.sqrt(shape[-1]))
        if kind == "hc_base":
            return (torch.randn(shape, generator=g, device=dev) * 0.5).float()
        if kind == "hc_scale":
            return torch.tensor([1.0, 1.0, 1.0], device=dev)
        if kind == "conv":
            return randn(1.0 / math.sqrt(c.conv))
        if kind == "a_log":
            return torch.log(torch.rand(shape, generator=g, device=dev) * 15 + 1).float()
        if kind == "dt_bias":
            return (torch.randn(shape, generator=g, device=dev) * 0.5).float()
        if kind == "router_bias":
            return (torch.randn(shape, generator=g, device=dev) * 0.1).float()
        if kind == "ape":
            return (torch.randn(shape, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        if kind == "ln_bias":
            return (torch.randn(shape, generator=g, device=dev) * 0.05).to(torch.bfloat16)
        if kind.startswith("exl3_"):
            part = kind[5:]
            k, n = shape
            tr, su, sv = exl3_ops.random_linear(k, n, bits=c.bits, generator=g, device=dev)
            return {"trellis": tr, "suh": su, "svh": sv, "mcg": torch.tensor([1], dtype=torch.int32)}[part]
        raise KeyError(kind)

    def experts(self, layer, proj, n_experts):
        """Stacked draw of all experts of one projection (one generator per layer/projection; the per-expert
        ``get`` path is used for files, this path for the full-size random model)."""
        c = self.cfg
        if proj == "down_proj":
            k, n = c.moe_width, c.hidden
        else:
            k, n = c.hidden, c.moe_width
        g = self._gen(f"{P}layers.{layer}.mlp.experts.{proj}.stacked")
        tr, su, sv = exl3_ops.random_linear(k, n, bits=c.bits, generator=g, device=self.device, lead=(n_experts,))
        return Exl3Stack(tr, su, sv)


def to_device(obj, device):
    """A copy of prepared weights (dataclasses, lists, tensors) on another device (e.g. CPU-generated weights
    moved to the GPU so that both sides of a comparison hold identical values)."""
    import copy
    if isinstance(obj, torch.Tensor):
        return obj.to(device)
    if isinstance(obj, list):
        return [to_device(v, device) for v in obj]
    if isinstance(obj, dict):
        return {k: to_device(v, device) for k, v in obj.items()}
    if hasattr(obj, "__dataclass_fields__"):
        o = copy.copy(obj)
        for k in obj.__dataclass_fields__:
            setattr(o, k, to_device(getattr(obj, k), device))
        if hasattr(o, "device"):
            try:
                o.device = torch.device(device)
            except (AttributeError, TypeError):
                pass
        return o
    return obj


def checkpoint_shapes(cfg: ModelConfig) -> dict[str, tuple[tuple[int, ...], str]]:
    """name -> (shape, init kind) for every tensor of the checkpoint (EXL3 experts listed per expert)."""
    c = cfg
    D, S = c.hidden, c.streams
    out: dict[str, tuple[tuple[int, ...], str]] = {}
    out[P + "embed_tokens.weight"] = ((c.vocab, D), "embed")
    out[P + "norm.weight"] = ((D,), "norm")
    out["lm_head.weight"] = ((c.vocab, D), "linear")
    H, Dh = c.lin_heads, c.lin_dim
    for i in range(c.layers):
        L = f"{P}layers.{i}."
        out[L + "input_layernorm.weight"] = ((D,), "norm")
        out[L + "post_attention_layernorm.weight"] = ((D,), "norm")
        for site in ("attn", "ffn"):
            out[L + f"hc_{site}_fn"] = ((c.n_mix, S * D), "hc_fn")
            out[L + f"hc_{site}_base"] = ((c.n_mix,), "hc_base")
            out[L + f"hc_{site}_scale"] = ((3,), "hc_scale")
        a = L + "self_attn."
        if c.layer_kinds[i] == "kda":
            for x in "qkv":
                out[a + f"{x}_proj.weight"] = ((H * Dh, D), "linear")
                out[a + f"{x}_conv1d.weight"] = ((H * Dh, 1, c.conv), "conv")
            out[a + "f_a_proj.weight"] = ((Dh, D), "linear")
            out[a + "g_a_proj.weight"] = ((Dh, D), "linear")
            out[a + "b_proj.weight"] = ((H, D), "linear")
            out[a + "f_b_proj.weight"] = ((H * Dh, Dh), "linear")
            out[a + "g_b_proj.weight"] = ((H * Dh, Dh), "linear")
            out[a + "A_log"] = ((H,), "a_log")
            out[a + "dt_bias"] = ((H * Dh,), "dt_bias")
            out[a + "o_norm.weight"] = ((Dh,), "norm")
            out[a + "o_proj.weight"] = ((D, H * Dh), "linear")
        else:
            out[a + "q_a_proj.weight"] = ((c.q_lora, D), "linear")
            out[a + "q_a_layernorm.weight"] = ((c.q_lora,), "norm")
            out[a + "q_b_proj.weight"] = ((c.heads * c.qk_dim, c.q_lora), "linear")
            out[a + "kv_a_proj_with_mqa.weight"] = ((c.kv_lora + c.qk_rope, D), "linear")
            out[a + "kv_a_layernorm.weight"] = ((c.kv_lora,), "norm")
            out[a + "kv_b_proj.weight"] = ((c.heads * (c.qk_nope + c.v_dim), c.kv_lora), "linear")
            out[a + "o_proj.weight"] = ((D, c.heads * c.v_dim), "linear")
            ix = a + "indexer."
            out[ix + "wq_b.weight"] = ((c.index_heads * c.index_dim, c.q_lora), "linear")
            out[ix + "wk.weight"] = ((c.index_dim, D), "linear")
            out[ix + "k_norm.weight"] = ((c.index_dim,), "norm")
            out[ix + "k_norm.bias"] = ((c.index_dim,), "ln_bias")
            out[ix + "weights_proj.weight"] = ((c.index_heads, D), "linear")
            out[ix + "index_kpool_compress_gate"] = ((c.index_dim, D), "linear")
            out[ix + "index_kpool_compress_ape"] = ((c.kpool, c.index_dim), "ape")
        m = L + "mlp."
        if c.mlp_kinds[i] == "dense":
            out[m + "gate_proj.weight"] = ((c.dense_width, D), "linear")
            out[m + "up_proj.weight"] = ((c.dense_width, D), "linear")
            out[m + "down_proj.weight"] = ((D, c.dense_width), "linear")
        else:
            out[m + "gate.weight"] = ((c.experts, D), "linear")
            out[m + "gate.e_score_correction_bias"] = ((c.experts,), "router_bias")
            for e in range(c.experts):
                for proj, (k, n) in (("gate_proj", (D, c.moe_width)), ("up_proj", (D, c.moe_width)),
                                     ("down_proj", (c.moe_width, D))):
                    for part in ("trellis", "suh", "svh", "mcg"):
                        out[m + f"experts.{e}.{proj}.{part}"] = ((k, n), f"exl3_{part}")
            out[m + "shared_experts.gate_proj.weight"] = ((c.shared_width, D), "linear")
            out[m + "shared_experts.up_proj.weight"] = ((c.shared_width, D), "linear")
            out[m + "shared_experts.down_proj.weight"] = ((D, c.shared_width), "linear")
    return out


def random_checkpoint(cfg: ModelConfig, seed: int = 0) -> dict[str, torch.Tensor]:
    """Every checkpoint tensor, materialised on the CPU (use for small configs)."""
    src = RandomSource(cfg, seed)
    return {name: src.get(name) for name in checkpoint_shapes(cfg)}


def save_checkpoint(tensors: dict[str, torch.Tensor], cfg: ModelConfig, path: str, shard_bytes: int = 2 << 30):
    """Write a sharded safetensors checkpoint + config.json + index (the layout ``SafetensorsSource`` reads)."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    shards: list[dict[str, torch.Tensor]] = [{}]
    size = 0
    for k, v in tensors.items():
        nb = v.numel() * v.element_size()
        if size + nb > shard_bytes and shards[-1]:
            shards.append({})
            size = 0
        shards[-1][k] = v.contiguous()
        size += nb
    wm = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(path, fn))
        for k in sh:
            wm[k] = fn
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"weight_map": wm}, f)
    with open(os.path.join(path, "config.json"), "w") as f:
        f.write(cfg.to_json())


def load_config(path: str) -> ModelConfig:
    with open(os.path.join(path, "config.json")) as f:
        return ModelConfig.from_json(f.read())


# ---------------------------------------------------------------------------------------------------------------
# prepare: quantise + shard into runtime containers
# ---------------------------------------------------------------------------------------------------------------
def _rows(x: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    n = x.shape[dim]
    assert n % world == 0, (x.shape, world)
    step = n // world
    return x.narrow(dim, rank * step, step)


def prepare(src: TensorSource, cfg: ModelConfig, *, rank: int = 0, world: int = 1,
            device: str | torch.device = "cpu", layers: list[int] | None = None,
            progress: Callable[[str], None] | None = None, ep: bool = False, sp_mla: bool = False) -> Weights:
    """Quantise and shard a checkpoint into runtime weights for rank ``rank`` of ``world``.  ``ep``: the routed
    experts are sharded by expert (rank j holds experts [j E/W, (j+1) E/W) at full width, for the expert-parallel
    MoE of parallel/ep.py) instead of by width; everything else stays tensor-parallel.  ``sp_mla``: the MLA
    layers also keep every head's query / output projections (``MLAW.full``) for row-parallel prefill."""
    if ep and world > 1 and cfg.experts % world:
        raise ValueError(f"{cfg.experts} experts do not split over {world} ranks")
    c = cfg
    c.validate(world)
    dev = torch.device(device)
    D = c.hidden

    def g(name, dtype=None):
        t = src.get(name)
        if dtype is not None:
            t = t.to(dtype)
        return t

    def lin(t):
        return quantize_fp8_rows(t.to(dev))

    def lin_rowpar(t):
        """Row-parallel projection: quantise the whole weight (per-row scales over all inputs), then take this
        rank's input columns, so every tensor-parallel degree holds slices of the same fp8 weights and the rank
        partials add up to the unsharded result."""
        q = quantize_fp8_rows(t.to(dev))
        if world == 1:
            return q
        return Linear8(_rows(q.w, rank, world, 1).contiguous(), q.s)

    def f32(t):
        return t.float().to(dev).contiguous()

    def bf(t):
        return t.to(torch.bfloat16).to(dev).contiguous()

    def hc(i, site):
        L = f"{P}layers.{i}."
        return HCW(bf(g(L + f"hc_{site}_fn")), f32(g(L + f"hc_{site}_base")), f32(g(L + f"hc_{site}_scale")))

    def kda(i):
        a = f"{P}layers.{i}.self_attn."
        Hl = c.lin_heads // world
        qkv = [_rows(g(a + f"{x}_proj.weight"), rank, world) for x in "qkv"]
        rows = qkv + [g(a + "f_a_proj.weight"), g(a + "g_a_proj.weight"), _rows(g(a + "b_proj.weight"), rank, world)]
        in_proj = lin(torch.cat([r.to(dev) for r in rows], 0))
        conv = torch.cat([_rows(g(a + f"{x}_conv1d.weight"), rank, world).reshape(-1, c.conv) for x in "qkv"])
        return KDAW(in_proj, lin(_rows(g(a + "f_b_proj.weight"), rank, world)),
                    lin(_rows(g(a + "g_b_proj.weight"), rank, world)), f32(conv),
                    f32(_rows(g(a + "A_log"), rank, world)), f32(_rows(g(a + "dt_bias"), rank, world)),
                    bf(g(a + "o_norm.weight")), lin_rowpar(g(a + "o_proj.weight")), Hl)

    def mla(i):
        a = f"{P}layers.{i}.self_attn."
        Hl = c.heads // world
        qkv_a = lin(torch.cat([g(a + "q_a_proj.weight").to(dev), g(a + "kv_a_proj_with_mqa.weight").to(dev)], 0))
        kvb = _rows(g(a + "kv_b_proj.weight"), rank, world).float().to(dev)
        kvb = kvb.view(Hl, c.qk_nope + c.v_dim, c.kv_lora)
        w_uk_t = quantize_fp8_rows(kvb[:, :c.qk_nope, :].transpose(1, 2).contiguous())   # [Hl, kv_lora, nope]
        w_uv = quantize_fp8_rows(kvb[:, c.qk_nope:, :].contiguous())                      # [Hl, v, kv_lora]
        ix = a + "indexer."
        iproj = torch.cat([g(ix + "wk.weight").to(dev), g(ix + "weights_proj.weight").to(dev),
                           g(ix + "index_kpool_compress_gate").to(dev)], 0)
        index = IndexW(bf(iproj), lin(g(ix + "wq_b.weight")), f32(g(ix + "k_norm.weight")),
                       f32(g(ix + "k_norm.bias")), f32(g(ix + "index_kpool_compress_ape")))
        full = None
        if sp_mla and world > 1:
            kvf = g(a + "kv_b_proj.weight").float().to(dev).view(c.heads, c.qk_nope + c.v_dim, c.kv_lora)
            full = MLAFull(lin(g(a + "q_b_proj.weight")),
                           quantize_fp8_rows(kvf[:, :c.qk_nope, :].transpose(1, 2).contiguous()),
                           quantize_fp8_rows(kvf[:, c.qk_nope:, :].contiguous()), lin(g(a + "o_proj.weight")))
        return MLAW(qkv_a, bf(g(a + "q_a_layernorm.weight")), bf(g(a + "kv_a_layernorm.weight")),
                    lin(_rows(g(a + "q_b_proj.weight"), rank, world)), w_uk_t, w_uv,
                    lin_rowpar(g(a + "o_proj.weight")), index, Hl, full)

    def mlp(prefix, width):
        gate = _rows(g(prefix + "gate_proj.weight"), rank, world).to(dev)
        up = _rows(g(prefix + "up_proj.weight"), rank, world).to(dev)
        return MLPW(lin(torch.cat([gate, up], 0)), lin_rowpar(g(prefix + "down_proj.weight")), width // world)

    def experts(i, proj):
        st = src.experts(i, proj, c.experts)
        tr, su, sv = st.trellis, st.suh, st.svh
        if world > 1 and ep:             # expert-parallel: this rank's experts at full width
            el = c.experts // world
            tr, su, sv = tr[rank * el:(rank + 1) * el], su[rank * el:(rank + 1) * el], sv[rank * el:(rank + 1) * el]
        elif world > 1:
            if proj == "down_proj":      # row-parallel: split k tiles and suh
                tr, su = _rows(tr, rank, world, 1), _rows(su, rank, world, 1)
            else:                        # column-parallel: split n tiles and svh
                tr, sv = _rows(tr, rank, world, 2), _rows(sv, rank, world, 1)
        return Exl3Stack(tr.to(dev).contiguous(), su.to(dev).half().contiguous(), sv.to(dev).half().contiguous())

    def moe(i):
        m = f"{P}layers.{i}.mlp."
        return MoEW(bf(g(m + "gate.weight")), f32(g(m + "gate.e_score_correction_bias")),
                    experts(i, "gate_proj"), experts(i, "up_proj"), experts(i, "down_proj"),
                    mlp(m + "shared_experts.", c.shared_width))

    out_layers = []
    which = range(c.layers) if layers is None else layers
    for i in which:
        if progress:
            progress(f"layer {i}")
        L = f"{P}layers.{i}."
        lw = LayerW(i, c.layer_kinds[i], c.mlp_kinds[i], hc(i, "attn"), hc(i, "ffn"),
                    bf(g(L + "input_layernorm.weight")), bf(g(L + "post_attention_layernorm.weight")))
        if lw.kind == "kda":
            lw.kda = kda(i)
        else:
            lw.mla = mla(i)
        if lw.mlp_kind == "dense":
            lw.mlp = mlp(L + "mlp.", c.dense_width)
        else:
            lw.moe = moe(i)
        out_layers.append(lw)
    head = lin(_rows(g("lm_head.weight"), rank, world))
    return Weights(c, bf(g(P + "embed_tokens.weight")), out_layers, bf(g(P + "norm.weight")), head, rank, world,
                   meta={"ep": bool(ep and world > 1)})
