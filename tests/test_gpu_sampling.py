"""Distribution tests of the speculative-decoding rejection sampler (csrc/sample.cu) on the GPU: with drafts
drawn from the draft distribution q, the tokens the sampler emits must follow the target distribution p, which is
what keeps speculative decoding lossless.  Many independent windows (distinct positions key independent noise)
are sampled in one launch and compared with a chi-square test."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _chi2_pvalue(counts: torch.Tensor, probs: torch.Tensor) -> float:
    from scipy.stats import chi2
    n = counts.sum().item()
    exp = probs.double() * n
    stat = ((counts.double() - exp) ** 2 / exp).sum().item()
    return float(chi2.sf(stat, probs.numel() - 1))


@pytest.mark.parametrize("block", [False, True])
def test_rejection_sampler_emits_target_distribution(block):
    from glm53.ops import kernels as Kk
    V, K, B = 8, 2, 120_000
    g = torch.Generator().manual_seed(3)
    p = torch.softmax(torch.randn(K + 1, V, generator=g) * 1.5, -1)          # target rows 0..K
    q = torch.softmax(torch.randn(K, V, generator=g) * 1.5, -1)              # draft rows 0..K-1
    drafts = torch.stack([torch.multinomial(q[i], B, replacement=True, generator=g) for i in range(K)], 1)
    tp = p.expand(B, K + 1, V).contiguous().to(DEV)
    dp = q.expand(B, K, V).contiguous().to(DEV)
    pos = (torch.arange(B, dtype=torch.int64) * 97).to(DEV)                 # one noise stream per window
    acc = torch.zeros(B, dtype=torch.int32, device=DEV)
    nxt = torch.zeros(B, K + 1, dtype=torch.int32, device=DEV)
    scratch = torch.zeros(B, K + 1, device=DEV)
    Kk.C().rejection_sample(tp, dp, drafts.to(torch.int32).to(DEV), 12345, pos, block, acc, nxt, scratch)
    torch.cuda.synchronize()
    acc, nxt = acc.cpu(), nxt.cpu()
    assert (acc >= 0).all() and (acc <= K).all()
    # accepted positions repeat the drafts
    for i in range(K):
        sel = acc > i
        assert torch.equal(nxt[sel, i], drafts[sel, i].to(torch.int32))
    # the first emitted token follows p[0]
    c0 = torch.bincount(nxt[:, 0].long(), minlength=V)
    assert _chi2_pvalue(c0, p[0]) > 1e-4, (c0, p[0] * B)
    if not block:
        # standard verification: after an accepted first draft, the next emitted token follows p[1]
        sel = acc >= 1
        c1 = torch.bincount(nxt[sel, 1].long(), minlength=V)
        assert _chi2_pvalue(c1, p[1]) > 1e-4, (c1, p[1] * sel.sum())
        # acceptance rate of the first draft = sum_x min(p0, q0)
        rate = (acc >= 1).double().mean().item()
        assert abs(rate - torch.minimum(p[0], q[0]).sum().item()) < 0.01


@pytest.mark.parametrize("block", [False, True])
def test_engine_sampled_speculative_decoding(block):
    """Sampled requests through the engine with the tiny proxy: drafts drawn from the drafter's filtered distribution,
    verified by the CUDA rejection kernel (standard or block). Every request reaches max_tokens, windows accept
    drafts, and the same seeds reproduce the same tokens."""
    from glm53.api.offline import LLM, LLMOptions
    from glm53.engine.llm import SamplingParams
    llm = LLM(LLMOptions(model="tiny", max_seqs=2, max_model_len=512, prefill_chunk=128, page_size=64,
                         checkpoints=0, k_fixed=4))
    llm.engine.cfg.block_verify = block
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(16, 4096, (96,), generator=g).tolist() for _ in range(2)]
    sp = [SamplingParams(max_tokens=24, temperature=1.0, top_p=0.95, seed=7 + i, ignore_eos=True) for i in range(2)]
    a = llm.engine.generate(prompts, sp)
    b = llm.engine.generate(prompts, sp)
    assert [len(o) for o in a] == [24, 24]
    assert a == b
    m = llm.engine.metrics
    assert m["spec_windows"] > 0 and m["spec_drafts"] > 0
