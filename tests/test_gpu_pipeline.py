"""GPU: the overlapped host-batch runner returns, for every submitted batch, what the public layer
call returns for that batch (copies and forward on three streams)."""
import pytest
import torch

from _util import make_layer_inputs

pytestmark = pytest.mark.gpu


def test_overlapped_host_runner_matches_direct_calls():
    from sonicmoe.functional import moe_TC_softmax_topk_layer
    from sonicmoe.pipeline import OverlappedHostRunner

    T, H, I, E, K = 512, 512, 256, 16, 4
    dev = torch.device("cuda", 0)
    batches = [make_layer_inputs(T, H, I, E, seed=40 + i)[0] for i in range(5)]
    _, rw, w1, w2 = make_layer_inputs(T, H, I, E, seed=40)
    rw, w1v, w2v = rw.to(dev), w1.to(dev).permute(1, 2, 0), w2.to(dev).permute(1, 2, 0)

    def fwd(xd):
        return moe_TC_softmax_topk_layer(xd, rw, w1v, None, w2v, None, K, None, is_inference_mode_enabled=True)[0]

    expect = [fwd(b.to(dev)).cpu() for b in batches]
    runner = OverlappedHostRunner(fwd, (T, H), torch.bfloat16, dev, depth=2)
    hosts = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in batches]
    events = [runner.submit(b.pin_memory(), h) for b, h in zip(batches, hosts)]
    runner.drain()
    for ev, h, e in zip(events, hosts, expect):
        ev.synchronize()
        # the combine adds the K partial rows in bf16 in arbitrary order: equal up to that rounding
        err = (h.float() - e.float()).norm() / e.float().norm()
        assert err < 5e-3, err
