"""The allocation-free MLA decode entry point (g53_mla_decode_noalloc), called through its exported C symbol.

It serves callers that cannot allocate device memory (the regular entry point needs caller-provided scratch for
the split partials): its output must match the regular entry point's on the same inputs, on two calls in a row
(the second call reuses the shared scratch array left over from the first), and an oversized problem must be
rejected before anything is launched.  This file is collected last on purpose."""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _lib():
    from glm53.ops import _ext
    _ext.require()                                # torch and the extension are loaded (symbol dependencies)
    lib = ctypes.CDLL(_ext.so_path())
    fn = lib.g53_mla_decode_noalloc
    fn.restype = ctypes.c_int
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    fn.argtypes = [vp, vp, i64, i32, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, ctypes.c_float, i32, vp, vp]
    err = lib.g53_mla_decode_noalloc_error
    err.restype = ctypes.c_char_p
    err.argtypes = [i32]
    return fn, err


def _inputs(seed, R=8, H=64, L=512, slots=3000):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q_lat = (torch.randn(R, H, L, device=DEV, generator=g) * 0.5).to(torch.bfloat16)
    kv = (torch.randn(slots, L, device=DEV, generator=g) * 40).clamp(-448, 448).to(torch.float8_e4m3fn)
    kv = kv.view(torch.uint8)
    scale = torch.rand(slots, device=DEV, generator=g) * 0.02 + 0.001
    max_sel = 2048
    counts = torch.tensor([max_sel - 37 * i for i in range(R)], dtype=torch.int32, device=DEV)
    sel = torch.stack([torch.randperm(slots, device=DEV, generator=g)[:max_sel] for _ in range(R)]).to(torch.int32)
    return q_lat, kv, scale, sel, counts


def _regular(q_lat, kv, scale, sel, counts, splits):
    from glm53.ops import _ext
    C = _ext.require()
    R, H, L = q_lat.shape
    part_o = torch.empty(R * splits * H * L, device=DEV)
    part_ml = torch.empty(R * splits * H * 2, device=DEV)
    out = torch.empty_like(q_lat)
    # tensor_cores=0: the CUDA-core flash-decoding kernel, the one the allocation-free entry point runs, so the two
    # results must be bit-identical (same kernel, same split count); only the scratch's home differs
    C.mla_decode(q_lat, None, 0, 0, kv, scale, None, sel, counts, 0, 256 ** -0.5, splits, part_o, part_ml, out,
                 tensor_cores=0)
    return out


def _noalloc(fn, q_lat, kv, scale, sel, counts, splits):
    R, H, L = q_lat.shape
    out = torch.empty_like(q_lat)
    p = lambda t: ctypes.c_void_p(t.data_ptr())      # noqa: E731
    rc = fn(p(q_lat), None, 0, 0, p(kv), p(scale), None, p(sel), p(counts), sel.shape[1], R, H, L, 0,
            256 ** -0.5, splits, p(out), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


def test_noalloc_matches_regular_entry_point_twice():
    fn, err = _lib()
    for call, seed in enumerate((11, 12)):        # two calls in a row, different inputs
        args = _inputs(seed)
        ref = _regular(*args, splits=4)
        rc, out = _noalloc(fn, *args, splits=4)
        assert rc == 0, err(rc).decode()
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert torch.equal(out, ref), f"call {call}: max diff {(out.float() - ref.float()).abs().max().item()}"


def test_noalloc_rejects_oversized_problem():
    fn, err = _lib()
    q_lat, kv, scale, sel, counts = _inputs(3)
    rc, _ = _noalloc(fn, q_lat, kv, scale, sel, counts, splits=16)     # 8*16*64*512 > 2^20 partial floats
    assert rc == 1001
    assert "too large" in err(rc).decode()


def test_noalloc_rejects_bad_arguments_before_launch():
    """Null inputs, a rope kernel without its rope tensors and unsupported (L, rope) pairs are refused on the host
    (cudaErrorInvalidValue = 1) instead of reaching a kernel that would dereference them."""
    fn, err = _lib()
    q_lat, kv, scale, sel, counts = _inputs(5, R=2)
    R, H, L = q_lat.shape
    out = torch.empty_like(q_lat)
    p = lambda t: ctypes.c_void_p(t.data_ptr())      # noqa: E731
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # rope = 32 with no q_pe / kpe_cache
    rc = fn(p(q_lat), None, 0, 0, p(kv), p(scale), None, p(sel), p(counts), sel.shape[1], R, H, 128, 32,
            0.1, 1, p(out), st)
    assert rc == 1, err(rc).decode()
    # an (L, rope) pair with no kernel
    rc = fn(p(q_lat), None, 0, 0, p(kv), p(scale), None, p(sel), p(counts), sel.shape[1], R, H, 256, 0, 0.1, 1,
            p(out), st)
    assert rc == 1
    # a null selection table
    rc = fn(p(q_lat), None, 0, 0, p(kv), p(scale), None, None, p(counts), sel.shape[1], R, H, L, 0, 0.1, 1,
            p(out), st)
    assert rc == 1
    torch.cuda.synchronize()                       # nothing was launched, the context is clean
