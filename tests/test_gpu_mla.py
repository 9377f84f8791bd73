"""Sparse MLA attention over the fp8 latent cache: the tcgen05 kernel and the mma.sync kernel against a plain fp32
PyTorch reference of the same op (softmax over each row's selected keys, V = the same latent rows), for every
tensor-parallel head count, decode splits (partials merged by the second kernel), ranges that leave some splits
empty, and prefill-sized row counts (several rows per persistent CTA)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
L = 512


@pytest.fixture(scope="module")
def C():
    from glm53.ops import _ext
    return _ext.require()


def _inputs(seed, R, H, slots=5000, max_sel=2048, qscale=0.5, counts=None, ordered=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q_lat = (torch.randn(R, H, L, device=DEV, generator=g) * qscale).to(torch.bfloat16)
    kv = (torch.randn(slots, L, device=DEV, generator=g) * 40).clamp(-448, 448).to(torch.float8_e4m3fn)
    scale = torch.rand(slots, device=DEV, generator=g) * 0.02 + 0.001
    if ordered:     # scales grow with the slot: later tiles raise the running maximum (online-softmax rescaling)
        scale = torch.linspace(0.001, 0.03, slots, device=DEV)
    sel = torch.stack([torch.randperm(slots, device=DEV, generator=g)[:max_sel] for _ in range(R)]).to(torch.int32)
    if ordered:
        sel = sel.sort(dim=1).values
    if counts is None:
        counts = [max(1, max_sel - 37 * i) for i in range(R)]
    counts = torch.tensor(counts, dtype=torch.int32, device=DEV)
    return q_lat, kv.view(torch.uint8), scale, sel, counts


def _reference(q_lat, kv, scale, sel, counts, sm_scale):
    R, H, _ = q_lat.shape
    kvf = kv.view(torch.float8_e4m3fn).float() * scale[:, None]
    out = torch.empty(R, H, L, device=DEV)
    for r in range(R):
        n = int(counts[r])
        keys = kvf[sel[r, :n].long()]
        s = q_lat[r].float() @ keys.T * sm_scale
        out[r] = torch.softmax(s, -1) @ keys
    return out


def _run(C, args, splits, tensor_cores, sm_scale):
    q_lat = args[0]
    R, H, _ = q_lat.shape
    part_o = torch.empty(R * splits * H * L, device=DEV)
    part_ml = torch.empty(R * splits * H * 2, device=DEV)
    out = torch.full_like(q_lat, float("nan"))
    C.mla_decode(q_lat, None, 0, 0, args[1], args[2], None, args[3], args[4], 0, sm_scale, splits, part_o, part_ml,
                 out, tensor_cores)
    torch.cuda.synchronize()
    return out.float()


@pytest.mark.parametrize("H", [64, 32, 8])
@pytest.mark.parametrize("splits", [1, 4, 16])
def test_mla_tcgen05_matches_fp32_reference(C, H, splits):
    sm = 256 ** -0.5
    args = _inputs(1, R=8, H=H, counts=[2048, 2000, 1111, 129, 128, 100, 7, 1])
    ref = _reference(*args, sm)
    tc = _run(C, args, splits, 1, sm)
    cc = _run(C, args, splits, 0, sm)
    assert torch.isfinite(tc).all()
    e_tc = (tc - ref).abs().max().item()
    e_cc = (cc - ref).abs().max().item()
    print(f"H={H} splits={splits}: max |tc - ref| {e_tc:.3e}, max |mma.sync - ref| {e_cc:.3e}, "
          f"max |ref| {ref.abs().max().item():.3f}")
    torch.testing.assert_close(tc, ref, atol=1e-2, rtol=2e-2)


@pytest.mark.parametrize("qscale", [0.5, 6.0])
def test_mla_tcgen05_peaked_and_rescaled(C, qscale):
    """Large logits (peaked softmax) with keys ordered so that later tiles raise the running maximum."""
    sm = 256 ** -0.5
    args = _inputs(2, R=4, H=64, qscale=qscale, ordered=True, counts=[2048, 1500, 700, 300])
    ref = _reference(*args, sm)
    tc = _run(C, args, 1, 1, sm)
    err = (tc - ref).abs().max().item()
    rel = err / ref.abs().max().item()
    print(f"qscale={qscale}: max err {err:.3e} (relative to max |ref| {rel:.3e})")
    torch.testing.assert_close(tc, ref, atol=2e-2, rtol=3e-2)


def test_mla_tcgen05_many_rows_persistent(C):
    """More rows than SMs: every CTA loops over several rows (queries, key tiles and O^T reused across items)."""
    sm = 256 ** -0.5
    R = 400
    counts = [(37 * i) % 2048 + 1 for i in range(R)]
    args = _inputs(3, R=R, H=16, counts=counts)
    tc = _run(C, args, 1, 1, sm)
    idx = [0, 1, 57, 148, 149, 296, 399]
    sub = tuple(a[idx] if a.dim() and a.shape[0] == R else a for a in args)
    ref = _reference(sub[0], args[1], args[2], sub[3], sub[4], sm)
    torch.testing.assert_close(tc[idx], ref, atol=1e-2, rtol=2e-2)
    assert torch.isfinite(tc).all()
