"""CPU tests: EXL3 codec, configuration, random init, and the fp32 reference model."""

import math

import numpy as np
import pytest
import torch


def _slow_unpack_tile(words16: np.ndarray, bits: int = 4) -> np.ndarray:
    """Independent decoder of one tile: read the circular bitstream bit by bit (MSB first within each
    little-endian 32-bit word), evaluate the mcg codebook in Python integers, place by the fragment map."""
    w32 = [int(words16[2 * i]) & 0xFFFF | ((int(words16[2 * i + 1]) & 0xFFFF) << 16) for i in range(8 * bits)]
    total = 32 * len(w32)

    def bit(b):
        b %= total
        return (w32[b // 32] >> (31 - b % 32)) & 1

    out = np.zeros((16, 16), dtype=np.float16)
    for p in range(256):
        end = (p + 1) * bits
        s = 0
        for b in range(end - 16, end):
            s = (s << 1) | bit(b)
        x = (s * 0xCBAC1FED) & 0xFFFFFFFF
        x = (x & 0x8FFF8FFF) ^ 0x3B603B60
        lo = np.array([x & 0xFFFF], dtype=np.uint16).view(np.float16)[0]
        hi = np.array([x >> 16], dtype=np.uint16).view(np.float16)[0]
        v = np.float16(np.float64(lo) + np.float64(hi))
        lane, j = p // 8, p % 8
        out[2 * (lane % 4) + (j & 1) + 8 * ((j >> 1) & 1), lane // 4 + 8 * (j >> 2)] = v
    return out


def test_exl3_unpack_matches_bitwise_decoder():
    from glm53.ops import exl3
    g = torch.Generator().manual_seed(0)
    tr, _, _ = exl3.random_linear(128, 128, generator=g)
    full = exl3.unpack(tr).numpy()
    for kt, nt in [(0, 0), (3, 5), (7, 7)]:
        ref = _slow_unpack_tile(tr[kt, nt].numpy())
        assert np.array_equal(full[kt * 16:(kt + 1) * 16, nt * 16:(nt + 1) * 16].view(np.uint16), ref.view(np.uint16))


def test_hadamard_orthonormal_and_rotate():
    from glm53.ops import exl3
    h = exl3.hadamard(128)
    assert torch.allclose(h @ h.t(), torch.eye(128, dtype=torch.float64), atol=1e-12)
    x = torch.randn(3, 256, dtype=torch.float64)
    y = exl3.rotate(exl3.rotate(x))
    assert torch.allclose(x, y, atol=1e-12)


def test_exl3_linear_consistent_with_dequantize():
    from glm53.ops import exl3
    g = torch.Generator().manual_seed(2)
    tr, su, sv = exl3.random_linear(256, 128, generator=g)
    x = torch.randn(4, 256)
    ref = (x.double() @ exl3.dequantize(tr, su, sv)).float()
    got = exl3.linear(x, tr, su, sv, f16_input=False)
    assert torch.allclose(got, ref, atol=1e-4, rtol=1e-4)
    w = exl3.dequantize(tr, su, sv)
    assert abs(w.std().item() - 1 / math.sqrt(256)) < 0.01


def test_full_config_layer_plan():
    import glm53
    c = glm53.full_config()
    assert c.layers == 45
    assert c.mla_layers() == list(range(3, 45, 4))
    assert len(c.kda_layers()) == 34 and len(c.moe_layers()) == 42
    assert c.mlp_kinds[:3] == ["dense"] * 3
    assert c.vocab == 154880 and c.n_mix == 24 and c.kda_proj_width == 3 * 64 * 128 + 256 + 64
    for tp in (1, 2, 4, 8):
        c.validate(tp)


def test_random_source_deterministic(tiny_cfg):
    from glm53.models import weights as W
    a = W.RandomSource(tiny_cfg, seed=3)
    b = W.RandomSource(tiny_cfg, seed=3)
    name = "model.layers.1.self_attn.q_proj.weight"
    assert torch.equal(a.get(name), b.get(name))
    assert not torch.equal(a.get(name), W.RandomSource(tiny_cfg, seed=4).get(name))


def test_fp8_row_quantisation():
    from glm53.models.weights import quantize_fp8_rows
    w = torch.randn(64, 128)
    q = quantize_fp8_rows(w)
    err = (q.dequant() - w).abs() / w.abs().amax(1, keepdim=True)
    assert err.max() < 0.07


def test_oracle_tiny_deterministic(tiny_weights):
    from glm53.models.reference import ReferenceModel
    m1, m2 = ReferenceModel(tiny_weights), ReferenceModel(tiny_weights)
    toks = [5, 17, 99, 1024, 7, 7, 3000, 12]
    a = m1.prefill(toks)
    b = m2.prefill(toks)
    assert torch.isfinite(a).all() and torch.equal(a, b)
    assert a.shape == (tiny_weights.cfg.vocab,)


def test_oracle_dsa_sparse_rows(tiny_cfg, tiny_weights):
    """Past index_topk tokens a query sees (P-1) pools + its own partial pool."""
    from glm53.models.reference import ReferenceModel
    m = ReferenceModel(tiny_weights)
    c = tiny_cfg
    toks = torch.randint(0, c.vocab, (c.index_topk + 9,), generator=torch.Generator().manual_seed(0)).tolist()
    m.prefill(toks)
    st = m.state.mla[c.mla_layers()[0]]
    assert len(st.pool) == len(toks) // c.kpool
    from glm53.models.reference import index_select
    t = len(toks) - 1
    qi = torch.randn(c.index_heads, c.index_dim)
    hw = torch.rand(c.index_heads)
    sel = index_select(c, st, qi, hw, t)
    assert len(sel) == (c.pools_selected - 1) * c.kpool + (t % c.kpool) + 1
    assert sel == sorted(sel) and sel[-1] == t


def test_override_source_sha_and_shape(tmp_path, tiny_cfg):
    import hashlib
    import pytest
    import torch
    from glm53.models import weights as W
    base = W.RandomSource(tiny_cfg, seed=0, device="cpu")
    name = next(n for n in base.shapes if n.endswith("self_attn.o_proj.weight"))
    ref = base.get(name)
    new = torch.ones_like(ref)
    path = str(tmp_path / "o.pt")
    torch.save(new, path)
    digest = hashlib.sha256(open(path, "rb").read()).hexdigest()
    src = W.OverrideSource(base, {name: path}, {name: digest})
    assert torch.equal(src.get(name), new)
    other = next(n for n in base.shapes if n != name and not n.endswith(".trellis"))
    assert torch.equal(src.get(other), base.get(other))
    with pytest.raises(ValueError):
        W.OverrideSource(base, {name: path}, {name: "0" * 64}).get(name)
    with pytest.raises(ValueError):
        W.OverrideSource(base, {name: torch.ones(3)}).get(name)


def test_kl_harness_reference_vs_itself(tiny_cfg, tiny_weights):
    """The harness on the CPU oracle against itself: zero KL, full top-1 agreement, finite NLL and intervals."""
    import torch
    from glm53.utils.klh import compare, reference_provider
    run = reference_provider(tiny_weights)
    seqs = [torch.randint(16, tiny_cfg.vocab, (24,), generator=torch.Generator().manual_seed(1)).tolist()]
    res = compare(run, run, seqs, block=4)
    assert res["kl_mean"] < 1e-12 and res["top1_agree"] == 1.0 and res["aa_kl_mean"] < 1e-12
    assert res["positions"] == 23 and res["nll_a"] > 0


def test_host_codec_matches_format_oracle():
    """The C++ host codec (csrc/exl3_codec.cpp): all 65536 codebook states and a whole-matrix tile decode equal
    the Python format oracle bit for bit (runs on the CPU when the extension is built)."""
    import pytest
    import torch
    from glm53.ops import _ext, exl3
    C = _ext.load(build_if_missing=False)
    if C is None:
        pytest.skip("extension not built")
    assert torch.equal(C.exl3_codebook_cpu().view(torch.int16), exl3.codebook().view(torch.int16))
    tr, _, _ = exl3.random_linear(512, 256, generator=torch.Generator().manual_seed(3))
    assert torch.equal(C.exl3_decode_cpu(tr, 4).view(torch.int16), exl3.unpack(tr).view(torch.int16))


def test_kv_bytes_per_token_of_the_full_model():
    """fp8 latent 512 + fp32 scale 4 + the bf16 rope-key column 2 (the full model's MLA has no rope part; the cache
    keeps one placeholder column) + pooled fp8 index key share (128 + 4) / 4, over 11 MLA layers: 6,061 bytes."""
    from glm53.config import full_config
    c = full_config()
    assert len(c.mla_layers()) == 11
    assert c.kv_bytes_per_token() == 11 * (c.kv_lora + 4 + 2 * max(c.qk_rope, 1) + (c.index_dim + 4) / c.kpool) == 6061


def test_scratch_guard_bands_detect_overruns():
    """Guard bands of the bounds-checked build's scratch allocator: intact after in-range writes, named after the
    owner's attribute when a write runs past either end of a buffer, and absent (plain zeros) when disabled."""
    from glm53.utils.canary import GUARD, Scratch

    class Owner:
        pass

    own = Owner()
    sc = Scratch("cpu", enabled=True)
    sc.attach(own)
    own.a = sc.zeros(5, 7, dtype=torch.float32)
    own.b = [sc.zeros(3, dtype=torch.int32), sc.zeros(2, 4, dtype=torch.bfloat16)]
    assert own.a.shape == (5, 7) and own.a.dtype == torch.float32 and not own.a.any()
    assert own.a.data_ptr() % 256 == sc._bands[0][0].data_ptr() % 256     # the band keeps 256-byte alignment
    own.a.fill_(3.0)
    own.b[0].fill_(-1)
    assert sc.check() == [] and len(sc) == 3
    # one element past the end of b[1] and one before the start of a
    raw_b1 = sc._bands[2][0]
    raw_b1[GUARD + own.b[1].numel() * 2] = 0
    raw_a = sc._bands[0][0]
    raw_a[GUARD - 1] = 0
    assert sorted(sc.check()) == ["a", "b[1]"]
    plain = Scratch("cpu", enabled=False)
    t = plain.zeros(4, dtype=torch.float32)
    assert t.shape == (4,) and len(plain) == 0 and plain.check() == []


def _order_key(f):
    import struct
    u = struct.unpack("<I", struct.pack("<f", f))[0]
    return (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)


def _sliced_radix_select(vals, K, nc):
    """Python model of the DSA select's cluster path: slices of the logits, 256-bin radix histograms summed over
    the slices for each of four 8-bit passes, then per-slice counts of keys above / equal to the threshold key give
    each slice its output offset; ties are taken in index order up to the remainder."""
    c = len(vals)
    keys = [_order_key(v) for v in vals]
    bounds = [(c * k // nc, c * (k + 1) // nc) for k in range(nc)]
    prefix, mask, rem = 0, 0, K
    for p in range(4):
        shift = 24 - 8 * p
        hist = [0] * 256
        for j0, j1 in bounds:                       # per-slice histograms, summed in rank order
            for j in range(j0, j1):
                if keys[j] & mask == prefix:
                    hist[(keys[j] >> shift) & 255] += 1
        acc, b = 0, 0
        for bin_ in range(255, 0, -1):              # highest bin whose count from the top reaches rem
            if acc + hist[bin_] >= rem:
                b = bin_
                break
            acc += hist[bin_]
        prefix |= b << shift
        rem -= acc
        mask |= 255 << shift
    counts = [(sum(keys[j] > prefix for j in range(j0, j1)), sum(keys[j] == prefix for j in range(j0, j1)))
              for j0, j1 in bounds]
    out = [None] * K
    for k, (j0, j1) in enumerate(bounds):
        base_sel = base_eq = 0
        for gk, ek in counts[:k]:
            base_sel += gk + max(0, min(ek, rem - base_eq))
            base_eq += ek
        for j in range(j0, j1):
            if keys[j] > prefix or (keys[j] == prefix and base_eq < rem):
                out[base_sel] = j
                base_sel += 1
            base_eq += keys[j] == prefix
    return out


@pytest.mark.parametrize("nc", [1, 3, 8])
def test_sliced_radix_select_matches_sorted_selection(nc):
    """The cluster select's offset rule (counts of lower slices, ties in index order) gives exactly the top-K
    indices of a stable descending sort, listed in index order, for any number of slices."""
    import random
    rng = random.Random(nc)
    for trial in range(20):
        c = rng.randrange(40, 400)
        vals = [round(rng.gauss(0, 1), 1) for _ in range(c)]          # one decimal: many exact ties
        if trial % 4 == 0:
            vals = [0.0] * c                                          # all tied
        K = rng.randrange(1, c)
        ref = sorted(sorted(range(c), key=lambda j: (-vals[j], j))[:K])
        assert _sliced_radix_select(vals, K, nc) == ref
