"""DSA indexer logits: the tcgen05 kernel against the CUDA-core kernel (fp32 dot products of the same bf16 queries
and e4m3 keys), with paged pools, two sequences in one launch and both the prefill (many rows) and the decode
(few rows, pool tiles split over CTAs) grids (GPU only)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(R_seqs, IH, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    ID, kpool, bs, max_blocks, pages = 128, 4, 64, 32, 80
    rows, pos, seq = [], [], []
    for s, (n, p0) in enumerate(R_seqs):
        pos += list(range(p0, p0 + n))
        seq += [s] * n
    R = len(pos)
    bt = torch.stack([torch.randperm(pages, generator=torch.Generator().manual_seed(seed + s))[:max_blocks]
                      for s in range(len(R_seqs))]).to(torch.int32).to(DEV)
    raw = torch.randint(0, 256, (pages * bs // kpool, ID), generator=g, device=DEV, dtype=torch.int32)
    raw[(raw == 0x7F) | (raw == 0xFF)] = 0                      # no e4m3 NaN codes
    pool_cache = raw.to(torch.uint8)
    pool_scale = torch.exp2(torch.randint(-4, 3, (pages * bs // kpool,), generator=g, device=DEV).float())
    iproj = torch.randn(R, ID + IH + ID, generator=g, device=DEV)
    qi = torch.randn(R, IH * ID, generator=g, device=DEV).to(torch.bfloat16)
    positions = torch.tensor(pos, dtype=torch.int32, device=DEV)
    row_seq = torch.tensor(seq, dtype=torch.int32, device=DEV)
    ln_w = torch.ones(ID, device=DEV)
    max_pools = max_blocks * bs // kpool
    return dict(iproj=iproj, qi=qi, ln_w=ln_w, pool_cache=pool_cache, pool_scale=pool_scale, positions=positions,
                block_table=bt, row_seq=row_seq, bs=bs, IH=IH, kpool=kpool, max_pools=max_pools, pos=pos)


@pytest.mark.parametrize("IH", [32, 4])
@pytest.mark.parametrize("shape", ["prefill", "decode"])
def test_dsa_logits_tc_matches_cuda_cores(IH, shape):
    from glm53.ops import kernels as Kk
    C = Kk.C()
    seqs = [(100, 900), (40, 300)] if shape == "prefill" else [(8, 1500)]
    d = _case(seqs, IH, 3 if shape == "prefill" else 4)
    R = len(d["pos"])
    out = []
    for tc in (False, True):
        lg = torch.zeros(R, d["max_pools"], device=DEV)
        C.dsa_logits(d["iproj"], d["qi"], d["ln_w"], d["pool_cache"], d["pool_scale"], d["positions"],
                     d["block_table"], d["row_seq"], d["bs"], d["IH"], d["kpool"], lg, tc)
        out.append(lg)
    torch.cuda.synchronize()
    assert C.gemm_error(out[1]) == 0
    for r, p in enumerate(d["pos"]):
        c = p // d["kpool"]
        torch.testing.assert_close(out[1][r, :c], out[0][r, :c], atol=1e-3, rtol=1e-3)
