"""EXL3 trellis format: decoder, random generator and the rotated-domain linear, in torch (CPU or CUDA).

The format is fixed by the checkpoints (ExLlamaV3 0.0.43 "mcg" codebook; described in the reference at
code/fork/kernels/exl3_format_ref.py:1-31).  A linear with K inputs and N outputs is stored as

    trellis  int16 [K/16, N/16, 16*bits]   one 16x16 tile per (k-tile, n-tile); read as 8*bits little-endian
                                           uint32 words, a circular bitstream, first bit = MSB of word 0
    suh      fp16  [K]                     input sign/scale vector
    svh      fp16  [N]                     output sign/scale vector
    mcg      int32 [1]                     marker of the mcg codebook

Value p (0..255) of a tile is read from the 16-bit state that ends at stream bit (p+1)*bits.  The state s is
multiplied by 0xCBAC1FED (mod 2^32), masked with 0x8FFF8FFF and xor-ed with 0x3B603B60; the two 16-bit halves of
that word, read as fp16 numbers, add up to the weight (the sum is rounded to fp16 a single time).  It lands at tile (row, col) = (2*(l%4) + (j&1) + 8*((j>>1)&1), l//4 + 8*(j>>2)) with l = p//8, j = p%8
(the tensor-core B-fragment order of m16n8k16: lane l holds values j = 0..7).  With H the 128-point orthonormal
Sylvester Hadamard transform applied per 128-block,

    y = ((((x * suh) @ H) @ W_q) @ H) * svh.

This module is this engine's own implementation of those rules (bit extraction by 64-bit windows, codebook
evaluated in integer arithmetic); the CUDA kernels in csrc/exl3_*.cu implement the same rules and are checked
against ``unpack`` here.
"""

from __future__ import annotations

import math
from functools import lru_cache

import torch

MCG_MUL = 0xCBAC1FED
MCG_MASK = 0x8FFF8FFF
MCG_XOR = 0x3B603B60
HBLOCK = 128


@lru_cache(maxsize=1)
def codebook() -> torch.Tensor:
    """Lookup table of all 65,536 states -> fp16 weight value (computed on first use).  Both halves of the masked
    product are widened to float64 before they are added; a double has room for the exact result of adding two
    half-precision numbers, so the only rounding is the final conversion back to fp16."""
    s = torch.arange(65536, dtype=torch.int64)
    x = ((s * MCG_MUL) & 0xFFFFFFFF)
    x = (x & MCG_MASK) ^ MCG_XOR
    lo = (x & 0xFFFF).to(torch.int16)            # two's-complement reinterpretation of the 16 low bits
    hi = ((x >> 16) & 0xFFFF).to(torch.int16)
    lo = lo.view(torch.float16).double()
    hi = hi.view(torch.float16).double()
    return (lo + hi).to(torch.float16)


@lru_cache(maxsize=1)
def tile_index() -> torch.Tensor:
    """Flat position (row*16 + col) inside its 16x16 tile of each stream value p = 0..255."""
    p = torch.arange(256)
    l, j = p // 8, p % 8
    row = 2 * (l % 4) + (j & 1) + 8 * ((j >> 1) & 1)
    col = l // 4 + 8 * (j >> 2)
    return row * 16 + col


def words(trellis: torch.Tensor) -> torch.Tensor:
    """int16 [..., 16*bits] -> int32 [..., 8*bits] words (little-endian pairs), a view when contiguous."""
    t = trellis.contiguous()
    return t.view(torch.int32)


def states(trellis: torch.Tensor, bits: int = 4) -> torch.Tensor:
    """The 16-bit state of each stream value: int64 [..., 256] from trellis int16 [..., 16*bits]."""
    if trellis.dtype == torch.int16:
        if trellis.shape[-1] != 16 * bits:
            raise ValueError(f"trellis must be int16 [..., {16 * bits}], got {tuple(trellis.shape)}")
        w = words(trellis)
    elif trellis.dtype == torch.int32:
        w = trellis
    else:
        raise TypeError(trellis.dtype)
    nw = w.shape[-1]
    if nw != 8 * bits:
        raise ValueError(f"expected {8 * bits} words per tile, got {nw}")
    w64 = w.to(torch.int64) & 0xFFFFFFFF
    dev = w.device
    p = torch.arange(256, device=dev)
    total = 32 * nw
    start = ((p + 1) * bits - 16) % total            # first stream bit of the state (circular)
    w0 = start // 32
    w1 = (w0 + 1) % nw
    off = start % 32
    window = (w64[..., w0] << 32) | w64[..., w1]     # 64 stream bits, first at bit 63
    return (window >> (48 - off)) & 0xFFFF


def unpack(trellis: torch.Tensor, bits: int = 4) -> torch.Tensor:
    """W_q [K, N] fp16 (rotated domain) from trellis [K/16, N/16, 16*bits] (or stacked [..., K/16, N/16, .])."""
    s = states(trellis, bits)
    vals = codebook().to(s.device)[s]                               # [..., kt, nt, 256]
    lead = vals.shape[:-3]
    kt, nt = vals.shape[-3], vals.shape[-2]
    tile = torch.empty_like(vals)
    tile[..., tile_index().to(s.device)] = vals                      # scatter into row-major 16x16
    tile = tile.view(*lead, kt, nt, 16, 16).transpose(-3, -2)        # [..., kt, 16, nt, 16]
    return tile.reshape(*lead, kt * 16, nt * 16)


@lru_cache(maxsize=8)
def hadamard(n: int = HBLOCK, dtype: torch.dtype = torch.float64) -> torch.Tensor:
    """Orthonormal Sylvester Hadamard matrix (H[i, j] = (-1)^popcount(i & j) / sqrt(n))."""
    i = torch.arange(n)
    pc = torch.zeros(n, n, dtype=torch.int64)
    a = i[:, None] & i[None, :]
    while bool(a.any()):
        pc += a & 1
        a = a >> 1
    h = 1.0 - 2.0 * (pc & 1).to(torch.float64)
    return (h / math.sqrt(n)).to(dtype)


def rotate(x: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Apply the orthonormal 128-point Hadamard transform to every block of 128 along ``dim`` (in x's dtype when
    it is fp32/fp64, fp32 otherwise)."""
    dt = x.dtype if x.dtype in (torch.float32, torch.float64) else torch.float32
    h = hadamard(HBLOCK).to(device=x.device, dtype=dt)
    y = x.to(dt).movedim(dim, -1)
    shp = y.shape
    y = (y.reshape(*shp[:-1], shp[-1] // HBLOCK, HBLOCK) @ h).reshape(shp)
    return y.movedim(-1, dim)


def dequantize(trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, bits: int = 4) -> torch.Tensor:
    """W [K, N] fp64 = diag(suh) H W_q H diag(svh)."""
    wq = unpack(trellis, bits).double()
    w = rotate(wq, -2) * suh.double()[..., :, None]
    return rotate(w, -1) * svh.double()[..., None, :]


def linear(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, bits: int = 4,
           f16_input: bool = True) -> torch.Tensor:
    """y = x @ W (fp32) the way the engine computes it: the rotated input is rounded to fp16 (the tensor-core
    operand type), the rotated-domain product accumulates in fp32, then the output transform."""
    xh = rotate(x.float() * suh.float(), -1)
    if f16_input:
        xh = xh.half().float()
    z = xh @ unpack(trellis, bits).float()
    return rotate(z, -1) * svh.float()


def codebook_std() -> float:
    return float(codebook().double().std())


def random_linear(k: int, n: int, *, bits: int = 4, generator: torch.Generator | None = None,
                  device: str | torch.device = "cpu", lead: tuple[int, ...] = (),
                  out_std: float | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Random EXL3 tensors of a [k -> n] linear (optionally stacked over ``lead`` dims): uniform random trellis
    words, random-sign suh/svh whose product sets the weight std to ``out_std`` (default 1/sqrt(k))."""
    if k % HBLOCK or n % HBLOCK:
        raise ValueError("EXL3 dims must be multiples of 128")
    std = (1.0 / math.sqrt(k)) if out_std is None else out_std
    mag = math.sqrt(std / codebook_std())
    shape = (*lead, k // 16, n // 16, 16 * bits)
    tr = torch.randint(-32768, 32768, shape, dtype=torch.int32, generator=generator, device=device).to(torch.int16)

    def signs(m):
        r = torch.randint(0, 2, (*lead, m), generator=generator, device=device)
        return ((r * 2 - 1).to(torch.float32) * mag).to(torch.float16)

    return tr, signs(k), signs(n)
