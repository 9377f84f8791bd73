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


def _pools_by_launches(launches, streams, IH=4, seed=9):
    """Run dsa_update over a list of launches; each launch is a list of (sequence, first position, rows) runs.
    `streams[s]` gives every position's iproj row of sequence s (a launch may override rows with `garbage`).
    Returns the pool cache and scales."""
    from glm53.ops import kernels as Kk
    C = Kk.C()
    ID, kpool, bs, pages, nseq = 128, 4, 64, 16, 2
    slots_per_seq = pages // nseq * bs
    pool_cache = torch.zeros(pages * bs // kpool, ID, dtype=torch.uint8, device=DEV)
    pool_scale = torch.zeros(pages * bs // kpool, device=DEV)
    ik_rows = torch.zeros(512, ID, dtype=torch.bfloat16, device=DEV)
    ig_rows = torch.zeros(512, ID, device=DEV)
    ring = Kk.DSA_RING
    assert C.dsa_ring_positions() == ring
    owners = [3, 1]                                   # state slots of the two sequences (ring owners)
    ik_ring = torch.zeros(4 * ring, ID, dtype=torch.bfloat16, device=DEV)
    ig_ring = torch.zeros(4 * ring, ID, device=DEV)
    bt = torch.arange(pages, dtype=torch.int32, device=DEV).view(nseq, pages // nseq)
    g = torch.Generator(device=DEV).manual_seed(seed)
    ln_w = 1 + 0.1 * torch.randn(ID, generator=g, device=DEV)
    ln_b = 0.1 * torch.randn(ID, generator=g, device=DEV)
    ape = torch.randn(kpool, ID, generator=g, device=DEV)
    for runs in launches:
        rows, pos, seq, slots, desc = [], [], [], [], []
        for b, (s, p0, n, garbage) in enumerate(runs):
            desc.append((len(rows), n, 0, 0, owners[s]))
            for i in range(n):
                p = p0 + i
                rows.append(garbage[i] if garbage is not None and garbage[i] is not None else streams[s][p])
                pos.append(p)
                seq.append(b)
                slots.append(int(bt[s, p // bs]) * bs + p % bs)
        iproj = torch.stack(rows)
        btl = torch.stack([bt[s] for s, _, _, _ in runs])
        sd = torch.tensor(desc, dtype=torch.int32, device=DEV).t().contiguous()
        C.dsa_update(iproj, ln_w, ln_b, ape, ik_rows, ig_rows, ik_ring, ig_ring, pool_cache, pool_scale,
                     torch.tensor(slots, dtype=torch.int32, device=DEV), torch.tensor(pos, dtype=torch.int32,
                                                                                      device=DEV),
                     btl, torch.tensor(seq, dtype=torch.int32, device=DEV), sd, bs, IH, kpool, 1e-6)
    torch.cuda.synchronize()
    return pool_cache, pool_scale, slots_per_seq


def test_dsa_pools_tail_ring_any_launch_split():
    """Pooled index keys keep no per-token raw keys: a pool's tokens come from the launch's own rows or from the
    sequence's tail ring.  The pools must be bit-identical whether the tokens arrive in one launch, in odd-sized
    chunks (pools straddling launches), or in verify windows whose rejected rows carried other keys and were
    rewritten by the next window -- with two sequences (different ring owners) interleaved in one launch."""
    IH, ID = 4, 128
    g = torch.Generator(device=DEV).manual_seed(1)
    N = 150
    streams = [torch.randn(N, ID + IH + ID, generator=g, device=DEV) for _ in range(2)]
    whole = [[(0, 0, N, None), (1, 0, N, None)]]
    chunks = []
    p = 0
    for n in (37, 1, 5, 64, 43):
        chunks.append([(0, p, n, None), (1, p, n, None)])
        p += n
    # verify windows of 8 rows after a 50-token prefill: window w keeps a rows; rejected rows carry junk keys
    windows = [[(0, 0, 50, None), (1, 0, 50, None)]]
    p = 50
    for keep in (3, 8, 1, 5, 8, 2, 7, 4, 8, 6, 8, 8, 3):
        junk = [None] * keep + [torch.randn(ID + IH + ID, generator=g, device=DEV) for _ in range(8 - keep)]
        windows.append([(0, p, 8, junk), (1, p, 8, junk)])
        p += keep
    final = p
    windows.append([(0, p, N - p, None), (1, p, N - p, None)])
    ref, ref_s, sps = _pools_by_launches(whole, streams)
    for launches in (chunks, windows):
        got, got_s, _ = _pools_by_launches(launches, streams)
        for s in range(2):
            base = s * sps // 4
            npools = N // 4
            assert torch.equal(got[base:base + npools], ref[base:base + npools]), (s, final)
            assert torch.equal(got_s[base:base + npools], ref_s[base:base + npools])


def _ref_selection(lg_row, c, pos, P, kp, bt_row, bs):
    """Top P - 1 complete pools by logit (ties: lower index first), listed in index order and expanded to token
    slots through the page table, then the row's own partial pool."""
    order = sorted(range(c), key=lambda j: (-lg_row[j], j))[:P - 1]
    slots = []
    for j in sorted(order):
        for i in range(kp):
            p = j * kp + i
            slots.append(bt_row[p // bs] * bs + p % bs)
    for p in range(c * kp, pos + 1):
        slots.append(bt_row[p // bs] * bs + p % bs)
    return slots


def test_dsa_select_long_rows_cluster_path():
    """Rows longer than the split threshold are selected by a cluster of CTAs (histograms summed through DSMEM,
    per-slice output offsets); a short row in the same launch by one CTA.  The logits of a decode-sized launch come
    from the tcgen05 kernel when the longest row is long.  Both must give exactly the reference selection, with
    exact ties (repeated pool keys) broken by index."""
    from glm53.ops import kernels as Kk
    C = Kk.C()
    g = torch.Generator(device=DEV).manual_seed(11)
    ID, IH, kp, bs, P = 128, 4, 4, 64, 512
    rows = [(0, 80003), (1, 36001), (2, 12002)]           # (sequence, position): 20000, 9000 and 3000 pools
    pages_per_seq = 1300
    n_pages = pages_per_seq * len(rows)
    bt = torch.randperm(n_pages, generator=torch.Generator().manual_seed(3)).to(torch.int32).view(len(rows), -1)
    bt = bt.contiguous().to(DEV)
    raw = torch.randint(0, 256, (n_pages * bs // kp, ID), generator=g, device=DEV, dtype=torch.int32)
    raw[(raw == 0x7F) | (raw == 0xFF)] = 0
    pool_cache = raw.to(torch.uint8)
    # exact ties: a few pools of each sequence share one key
    for s in range(len(rows)):
        for j in (5, 77, 1234, 2999):
            p = j * kp
            slot = int(bt[s, p // bs]) * bs + p % bs
            pool_cache[slot // kp] = pool_cache[int(bt[s, 0]) * bs // kp]
    pool_scale = torch.ones(n_pages * bs // kp, device=DEV)
    R = len(rows)
    iproj = torch.randn(R, ID + IH + ID, generator=g, device=DEV)
    qi = torch.randn(R, IH * ID, generator=g, device=DEV).to(torch.bfloat16)
    positions = torch.tensor([p for _, p in rows], dtype=torch.int32, device=DEV)
    row_seq = torch.tensor([s for s, _ in rows], dtype=torch.int32, device=DEV)
    ln_w = torch.ones(ID, device=DEV)
    max_pools = 32768
    lg_tc = torch.zeros(R, max_pools, device=DEV)
    C.dsa_logits(iproj, qi, ln_w, pool_cache, pool_scale, positions, bt, row_seq, bs, IH, kp, lg_tc, True)
    lg = torch.zeros(R, max_pools, device=DEV)
    sel = torch.zeros(R, P * kp, dtype=torch.int32, device=DEV)
    cnt = torch.zeros(R, dtype=torch.int32, device=DEV)
    C.dsa_select(iproj, qi, ln_w, pool_cache, pool_scale, positions, bt, row_seq, bs, IH, kp, P, lg, sel, cnt)
    torch.cuda.synchronize()
    assert C.gemm_error(lg) == 0 and C.gemm_error(lg_tc) == 0
    bt_h = bt.cpu().tolist()
    for r, (s, pos) in enumerate(rows):
        c = pos // kp
        assert torch.equal(lg[r, :c], lg_tc[r, :c])          # the tcgen05 kernel of the pair wrote the logits
        exp = _ref_selection(lg[r, :c].cpu().tolist(), c, pos, P, kp, bt_h[s], bs)
        n = int(cnt[r])
        assert n == len(exp)
        assert sel[r, :n].cpu().tolist() == exp, r
