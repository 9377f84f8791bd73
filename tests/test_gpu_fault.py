"""Failure detection without a GPU fault: the fused tensor-parallel reduction waits on a peer's arrival flag with a
bounded spin.  A flag that nothing sets makes the wait run out; the kernel records an error code that the host
reads, and the CUDA context stays usable for the next launch (single GPU, world of 1 emulated)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_bounded_wait_reports_error_and_context_survives():
    from glm53.ops import _ext
    C = _ext.require()
    R, S, D = 2, 2, 256
    X = torch.randn(R, S, D, device=DEV).to(torch.bfloat16)
    gath = torch.zeros(1 * R * D, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)       # nobody will ever raise this flag
    epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
    done = torch.zeros(1, dtype=torch.int32, device=DEV)
    err = torch.zeros(4, dtype=torch.int32, device=DEV)
    post = torch.ones(R, S, device=DEV)
    comb = torch.eye(S, device=DEV).expand(R, S, S).contiguous()
    part = torch.zeros(R, D // 64, 32, device=DEV)
    C.hc_post_pre_tp(X, gath, R * D, 1, flags, epoch, done, err, post, comb, None, None, None, None, None, None,
                     None, part, 1e-5, 1e-6, 20)
    torch.cuda.synchronize()
    assert int(err[0].item()) == 21                             # the wait gave up and said so
    # the context is still usable: a flag that is set lets the same kernel complete without an error
    err.zero_()
    flags.fill_(int(epoch.item()) + 1)
    C.hc_post_pre_tp(X, gath, R * D, 1, flags, epoch, done, err, post, comb, None, None, None, None, None, None,
                     None, part, 1e-5, 1e-6, 20)
    torch.cuda.synchronize()
    assert int(err[0].item()) == 0
    y = torch.randn(64, device=DEV).sum()                       # ordinary work still runs
    assert torch.isfinite(y)
