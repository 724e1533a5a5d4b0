"""GPU: a wait that nothing satisfies gives up with an error status and the context stays usable.

Every pipelined kernel here bounds its mbarrier waits; this drives that path on purpose through
sm_selftest_bounded_wait (a barrier nothing arrives on), checks the recorded code, then runs a
normal kernel on the same context.  No fault, no trap, no unbounded spin: the wait ends after 2 s.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives():
    from sonicmoe import _native as nat
    from sonicmoe import ops

    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    nat.call("sm_selftest_bounded_wait", err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert err.item() == 105
    logits = torch.randn(64, 16, device="cuda").to(torch.bfloat16)
    scores, idx = ops.router_topk(logits, 4)
    torch.cuda.synchronize()
    assert torch.isfinite(scores).all() and idx.shape == (64, 4)
