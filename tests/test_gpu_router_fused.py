"""GPU parity of the opt-in fused router (router GEMM + top-k in one tcgen05 kernel, C ABI
sm_router_fused / sm_moe_forward_fused_router).

Its logits are a bf16 rounding of an fp32 tensor-core accumulation, so against torch's F.linear
(cuBLAS) they may differ by one bf16 unit in the last place where the two fp32 sums round to
different sides of a bf16 boundary; that is the asserted bound.  The ranking of the logits it
returns is bit-exact against the oracle (reference semantics of functional/topk.py:143-260), and
the layer output is within the FP8 tolerance of the fake-quantised oracle run on those logits.
"""
import numpy as np
import pytest
import torch

from oracle import layer as olayer
from oracle import routing as oroute
from _util import make_layer_inputs, rel_fro

pytestmark = pytest.mark.gpu

TOL_FP8 = 1e-2


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from sonicmoe import ops as _ops

    return _ops


def _bf16_ulp(v):
    """One unit in the last place of bf16 at |v| (float32 array)."""
    a = np.abs(v).astype(np.float32)
    e = np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126))))
    return np.exp2(e - 7).astype(np.float32)


def _inputs(T, H, E, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    rw = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    return x, rw


def _check_logits(lg_fused, x, rw):
    ref = torch.nn.functional.linear(x.cuda(), rw.cuda()).float().cpu().numpy()
    got = lg_fused.float().cpu().numpy()
    d = np.abs(got - ref)
    bound = _bf16_ulp(np.maximum(np.abs(got), np.abs(ref)))
    assert np.all(d <= bound), f"max |fused - F.linear| {d.max():.3g} beyond one bf16 ulp"
    assert np.mean(d == 0) > 0.9, f"only {np.mean(d == 0):.3f} of the logits equal F.linear's"


ROUTER_CASES = [
    # T, H, E, K
    (4096, 4096, 128, 8),  # headline router shape
    (300, 2048, 128, 8),  # ragged last tile
    (1, 4096, 128, 8),
    (128, 7168, 256, 8),  # E = 256 (config 4's router), H = 7168
    (200, 512, 64, 6),
    (97, 1024, 32, 4),
    (256, 256, 96, 32),  # K = 32
]


@pytest.mark.parametrize("T,H,E,K", ROUTER_CASES)
@pytest.mark.parametrize("mode", ["sot", "tos", "tosn"])
def test_router_fused_vs_oracle(ops, T, H, E, K, mode):
    sot, norm = {"sot": (True, False), "tos": (False, False), "tosn": (False, True)}[mode]
    x, rw = _inputs(T, H, E, seed=T + H + E)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    lg, s, i = ops.router_fused(x.cuda(), rw.cuda(), K, sot, norm, err=err)
    torch.cuda.synchronize()
    assert err.item() == 0
    _check_logits(lg, x, rw)
    s_ref, i_ref = oroute.topk_route(lg.float().cpu().numpy(), K, sot, norm)
    np.testing.assert_array_equal(i.cpu().numpy(), i_ref)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def test_router_fused_full_size_matches_topk_kernel(ops):
    """T = 32768 tokens (the headline batch): the fused ranking equals the standalone top-k kernel's
    on the fused logits, bit for bit, and the logits stay within one bf16 ulp of F.linear."""
    T, H, E, K = 32768, 4096, 128, 8
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    rw = (torch.randn(E, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    lg, s, i = ops.router_fused(x, rw, K)
    s2, i2 = ops.router_topk(lg, K)
    assert torch.equal(i, i2) and torch.equal(s.view(torch.int32), s2.view(torch.int32))
    ref = torch.nn.functional.linear(x, rw).float()
    d = (lg.float() - ref).abs()
    bound = torch.from_numpy(_bf16_ulp(torch.maximum(lg.float().abs(), ref.abs()).cpu().numpy())).cuda()
    assert bool((d <= bound).all())


def test_router_fused_rejects_unsupported_shapes(ops):
    x, rw = _inputs(16, 512, 48, seed=1)  # E % 32 != 0
    with pytest.raises(NotImplementedError, match="fused router"):
        ops.router_fused(x.cuda(), rw.cuda(), 2)
    x, rw = _inputs(16, 96, 64, seed=1)  # H % 64 != 0
    with pytest.raises(NotImplementedError, match="fused router"):
        ops.router_fused(x.cuda(), rw.cuda(), 2)


LAYER_CASES = [
    # T, H, I, E, K, softmax_over_topk, norm, concat
    (512, 512, 256, 32, 4, True, False, False),
    (384, 1024, 384, 64, 8, False, True, True),
    (300, 2048, 256, 128, 8, True, False, False),
]


@pytest.mark.parametrize("T,H,I,E,K,sot,norm,concat", LAYER_CASES)
def test_layer_fused_router_vs_fp8_oracle(T, H, I, E, K, sot, norm, concat):
    from sonicmoe.functional import moe_TC_softmax_topk_layer

    x, rw, w1, w2 = make_layer_inputs(T, H, I, E, seed=5 * T + E)
    o, logits, freq = moe_TC_softmax_topk_layer(
        x.cuda(), rw.cuda(), w1.cuda().permute(1, 2, 0), None, w2.cuda().permute(1, 2, 0), None, K, None,
        is_inference_mode_enabled=True, is_softmax_over_topk=sot, norm_topk_probs=norm, concat_layout=concat,
        fused_router=True,
    )
    torch.cuda.synchronize()
    _check_logits(logits, x, rw)
    lg = logits.float().cpu().numpy()
    o_ref, scores, idx = olayer.fp8_oracle(x.float().numpy(), lg, w1.float().numpy(), w2.float().numpy(), K, sot,
                                           norm, concat)
    np.testing.assert_array_equal(freq.cpu().numpy(), np.bincount(idx.reshape(-1), minlength=E))
    assert rel_fro(o.float().cpu().numpy(), o_ref.numpy()) <= TOL_FP8
