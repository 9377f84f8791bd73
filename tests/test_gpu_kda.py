"""KDA kernels: the chunked prefill form against the recurrent form, multi-sequence batches, and the verify-window
replay (state after `keep` rows), on random inputs (GPU only)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(T, H, Dh, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    HD = H * Dh
    width = 3 * HD + 2 * Dh + H
    ldp = (width + 63) // 64 * 64
    proj = (torch.randn(T, ldp, device=DEV, generator=g) * 0.5).to(torch.bfloat16)
    qkv = (torch.randn(T, 3 * HD, device=DEV, generator=g)).to(torch.bfloat16)
    f = (torch.randn(T, HD, device=DEV, generator=g)).to(torch.bfloat16)
    a_log = torch.log(torch.rand(H, device=DEV, generator=g) * 15 + 1)
    dt_bias = torch.randn(HD, device=DEV, generator=g) * 0.5
    return proj, qkv, f, a_log, dt_bias, 3 * HD + 2 * Dh


def _close(a, b, rel=4e-3, abs_=3e-2):
    """tf32 tensor-core products in the chunked scan against the fp32 recurrent kernel"""
    err = (a - b).float()
    assert err.norm() <= rel * b.float().norm() + 1e-6, (err.norm().item(), b.norm().item())
    assert err.abs().max().item() <= abs_


@pytest.mark.parametrize("Dh", [64, 128])
@pytest.mark.parametrize("T", [64, 200, 1000])
def test_kda_chunk_matches_recurrent(Dh, T):
    from glm53.ops import kernels as Kk
    C = Kk.C()
    H = 4
    proj, qkv, f, a_log, dt_bias, b_off = _inputs(T, H, Dh, T + Dh)
    S = torch.randn(4, H, Dh, Dh, device=DEV) * 0.1
    S[1].zero_()
    S[3].zero_()
    seq = torch.tensor([[0], [T], [0], [1], [0]], dtype=torch.int32, device=DEV)
    o1 = torch.zeros(T, H * Dh, device=DEV)
    C.kda_recurrent(proj, seq, f, qkv, a_log, dt_bias, S, o1, H, Dh, b_off, -5.0)
    seq2 = torch.tensor([[0], [T], [0], [3], [0]], dtype=torch.int32, device=DEV)
    o2 = torch.zeros(T, H * Dh, device=DEV)
    scr = torch.empty(C.kda_chunk_scratch_floats(T, 1, H, Dh), device=DEV)
    C.kda_chunk(proj, seq2, f, qkv, a_log, dt_bias, S, o2, H, Dh, b_off, -5.0, scr)
    _close(o2, o1)
    _close(S[3], S[1])


def test_kda_chunk_many_heads_single_buffer_scan():
    """48 heads x 4 value blocks = 192 scan CTAs, more than the SMs: the scan runs its single-buffer, two-CTAs-per-SM
    form; it must match the recurrent form like the double-buffer one does."""
    from glm53.ops import kernels as Kk
    C = Kk.C()
    H, Dh, T = 48, 128, 200
    proj, qkv, f, a_log, dt_bias, b_off = _inputs(T, H, Dh, 77)
    S = torch.randn(4, H, Dh, Dh, device=DEV) * 0.1
    S[1].zero_()
    S[3].zero_()
    o1 = torch.zeros(T, H * Dh, device=DEV)
    C.kda_recurrent(proj, torch.tensor([[0], [T], [0], [1], [0]], dtype=torch.int32, device=DEV), f, qkv, a_log,
                    dt_bias, S, o1, H, Dh, b_off, -5.0)
    o2 = torch.zeros(T, H * Dh, device=DEV)
    scr = torch.empty(C.kda_chunk_scratch_floats(T, 1, H, Dh), device=DEV)
    C.kda_chunk(proj, torch.tensor([[0], [T], [0], [3], [0]], dtype=torch.int32, device=DEV), f, qkv, a_log, dt_bias,
                S, o2, H, Dh, b_off, -5.0, scr)
    _close(o2, o1)
    _close(S[3], S[1])


def test_kda_chunk_two_sequences_unaligned():
    """Two sequences in one chunked launch, the second starting at a row that is not a multiple of 64."""
    from glm53.ops import kernels as Kk
    C = Kk.C()
    H, Dh = 4, 128
    n0, n1 = 150, 230
    T = n0 + n1
    proj, qkv, f, a_log, dt_bias, b_off = _inputs(T, H, Dh, 5)
    S = torch.randn(8, H, Dh, Dh, device=DEV) * 0.1
    o_ref = torch.zeros(T, H * Dh, device=DEV)
    S_ref = S.clone()
    for row0, n, si, so in [(0, n0, 0, 1), (n0, n1, 2, 3)]:
        sq = torch.tensor([[row0], [n], [si], [so], [0]], dtype=torch.int32, device=DEV)
        C.kda_recurrent(proj, sq, f, qkv, a_log, dt_bias, S_ref, o_ref, H, Dh, b_off, -5.0)
    seq = torch.tensor([[0, n0], [n0, n1], [0, 2], [5, 7], [0, 1]], dtype=torch.int32, device=DEV)
    o = torch.zeros(T, H * Dh, device=DEV)
    scr = torch.empty(C.kda_chunk_scratch_floats(T, 2, H, Dh), device=DEV)
    C.kda_chunk(proj, seq, f, qkv, a_log, dt_bias, S, o, H, Dh, b_off, -5.0, scr)
    _close(o, o_ref)
    _close(S[5], S_ref[1])
    _close(S[7], S_ref[3])


def test_kda_multi_sequence_and_replay():
    from glm53.ops import kernels as Kk
    C = Kk.C()
    H, Dh = 4, 64
    T = 24
    proj, qkv, f, a_log, dt_bias, b_off = _inputs(T, H, Dh, 7)
    S = torch.randn(6, H, Dh, Dh, device=DEV) * 0.1
    # two sequences of 8 and 16 rows in one launch == separate launches
    seq = torch.tensor([[0, 8], [8, 16], [0, 2], [1, 3], [0, 1]], dtype=torch.int32, device=DEV)
    o = torch.zeros(T, H * Dh, device=DEV)
    S_a = S.clone()
    C.kda_recurrent(proj, seq, f, qkv, a_log, dt_bias, S_a, o, H, Dh, b_off, -5.0)
    o_ref = torch.zeros(T, H * Dh, device=DEV)
    S_b = S.clone()
    for row0, n, si, so in [(0, 8, 0, 1), (8, 16, 2, 3)]:
        sq = torch.tensor([[row0], [n], [si], [so], [0]], dtype=torch.int32, device=DEV)
        C.kda_recurrent(proj, sq, f, qkv, a_log, dt_bias, S_b, o_ref, H, Dh, b_off, -5.0)
    torch.testing.assert_close(o, o_ref, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(S_a, S_b, atol=1e-5, rtol=1e-5)
    # replay: keeping 3 rows of the first sequence gives the state a 3-row window produces
    keep = torch.tensor([[0], [3], [0], [4], [0]], dtype=torch.int32, device=DEV)
    C.kda_recurrent(proj, keep, f, qkv, a_log, dt_bias, S_a, None, H, Dh, b_off, -5.0)
    S_c = S.clone()
    o3 = torch.zeros(T, H * Dh, device=DEV)
    C.kda_recurrent(proj[:3], torch.tensor([[0], [3], [0], [4], [0]], dtype=torch.int32, device=DEV), f[:3],
                    qkv[:3], a_log, dt_bias, S_c, o3, H, Dh, b_off, -5.0)
    torch.testing.assert_close(S_a[4], S_c[4], atol=1e-6, rtol=1e-6)


def test_kda_decode_fused_matches_five_kernels():
    """The fused decode-window kernel (f_b, g_b, conv, recurrence, gated norm in one launch) against the five-kernel
    path on a model whose KDA heads have Dh = 128: every window's logits agree closely, and windows that keep fewer
    rows than they verified (commit replay from the stored conv outputs and decay logits) keep agreeing."""
    import dataclasses
    from glm53.config import tiny_config
    from glm53.models import weights as W
    from glm53.models.runtime import Runtime, RuntimeConfig
    from glm53.models.session import Sequence
    cfg = dataclasses.replace(tiny_config(), lin_heads=2, lin_dim=128)
    dev = torch.device("cuda", 0)
    w = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, device=dev)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(16, cfg.vocab, (150,), generator=g).tolist()
    windows = [(torch.randint(16, cfg.vocab, (n,), generator=g).tolist(), keep)
               for n, keep in ((8, 3), (8, 8), (5, 1), (1, 1), (8, 6), (16, 9))]
    outs = []
    for fused in (False, True):
        rt = Runtime(w, RuntimeConfig(max_rows=64, max_seqs=1, kv_slots=64 * 8, block_size=64, max_blocks=8))
        rt.kda_fused = fused
        seq = Sequence(rt)
        lg = [seq.prefill(prompt, chunk=64).float().clone()]
        for toks, keep in windows:
            lg.append(seq.verify(toks).float().clone())
            seq.commit(keep)
        outs.append(lg)
    for a, b in zip(*outs):
        cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
        assert cos > 0.9999, cos
        assert (a - b).abs().max().item() < 5e-2 * max(1.0, a.abs().max().item())


@pytest.mark.parametrize("Dh", [64, 128])
def test_kda_recurrent_chaining_is_bit_exact(Dh):
    """One launch over n rows leaves the same state and outputs, bit for bit, as n launches of one row each (plain
    decoding steps one row at a time, speculative windows and commit replays run several rows per launch)."""
    from glm53.ops import kernels as Kk
    C = Kk.C()
    H, T = 4, 8
    proj, qkv, f, a_log, dt_bias, b_off = _inputs(T, H, Dh, 77)
    S = torch.randn(3, H, Dh, Dh, device=DEV) * 0.1

    def seq(r0, n, s_in, s_out):
        return torch.tensor([[r0], [n], [s_in], [s_out], [0]], dtype=torch.int32, device=DEV)

    o1 = torch.zeros(T, H * Dh, device=DEV)
    C.kda_recurrent(proj, seq(0, T, 0, 1), f, qkv, a_log, dt_bias, S, o1, H, Dh, b_off, -5.0)
    o2 = torch.zeros(T, H * Dh, device=DEV)
    src = 0
    for t in range(T):
        dst = 2 if src == 0 else 0
        C.kda_recurrent(proj, seq(t, 1, src, dst), f, qkv, a_log, dt_bias, S, o2, H, Dh, b_off, -5.0)
        src = dst
    torch.cuda.synchronize()
    assert torch.equal(o1, o2), (o1 - o2).abs().max().item()
    assert torch.equal(S[1], S[src]), (S[1] - S[src]).abs().max().item()
