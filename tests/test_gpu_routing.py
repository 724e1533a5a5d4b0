"""GPU parity: router top-k and routing metadata, bit-exact against the oracle (through the C ABI)."""
import numpy as np
import pytest
import torch

from oracle import metadata as ometa
from oracle import routing as oroute

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from sonicmoe import ops as _ops

    return _ops


def _logits(T, E, seed, dtype=torch.bfloat16, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(T, E, generator=g) * scale).to(dtype)


ROUTE_CASES = [
    (4096, 128, 8),  # headline routing shape, bf16 logits have many exact ties
    (1000, 96, 7),
    (333, 64, 4),
    (256, 256, 16),
    (100, 512, 10),
    (77, 8, 2),
    (5, 40, 3),  # E not a multiple of 32
    (64, 2048, 8),
    (1, 128, 8),
]


@pytest.mark.parametrize("T,E,K", ROUTE_CASES)
@pytest.mark.parametrize("mode", ["sot", "tos", "tosn"])
def test_router_topk_bit_exact(ops, T, E, K, mode):
    sot, norm = {"sot": (True, False), "tos": (False, False), "tosn": (False, True)}[mode]
    lg = _logits(T, E, seed=T * 7 + E)
    s_gpu, i_gpu = ops.router_topk(lg.cuda(), K, sot, norm)
    s_ref, i_ref = oroute.topk_route(lg.float().numpy(), K, sot, norm)
    np.testing.assert_array_equal(i_gpu.cpu().numpy(), i_ref)
    np.testing.assert_array_equal(s_gpu.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_router_topk_other_dtypes(ops, dtype):
    lg = _logits(512, 128, seed=3, dtype=dtype, scale=3.0)
    for sot, norm in ((True, False), (False, True)):
        s_gpu, i_gpu = ops.router_topk(lg.cuda(), 8, sot, norm)
        s_ref, i_ref = oroute.topk_route(lg.float().numpy(), 8, sot, norm)
        np.testing.assert_array_equal(i_gpu.cpu().numpy(), i_ref)
        np.testing.assert_array_equal(s_gpu.cpu().numpy(), s_ref)


def test_router_ties_lower_index_first(ops):
    lg = torch.zeros(4, 64, dtype=torch.bfloat16)
    lg[1] = -1.5
    lg[2, 10] = 2.0
    lg[2, 3] = 2.0
    s, i = ops.router_topk(lg.cuda(), 4, True)
    i = i.cpu().numpy()
    np.testing.assert_array_equal(i[0], [0, 1, 2, 3])
    np.testing.assert_array_equal(i[1], [0, 1, 2, 3])
    np.testing.assert_array_equal(i[2], [3, 10, 0, 1])


def _make_topk_indices(T, E, K, seed):
    rs = np.random.RandomState(seed)
    if T == 0:
        return np.zeros((0, K), dtype=np.int32)
    return np.stack([np.sort(rs.permutation(E)[:K]) for _ in range(T)]).astype(np.int32)


META_CASES = [(10, 8, 2), (236, 16, 4), (1024, 128, 8), (8192, 128, 8), (8192, 256, 16), (32768, 128, 8),
              (1000, 96, 7), (50, 384, 3), (2048, 512, 10), (1, 8, 2), (0, 8, 2)]


@pytest.mark.parametrize("T,E,K", META_CASES)
def test_route_metadata_bit_exact(ops, T, E, K):
    idx = _make_topk_indices(T, E, K, seed=T + E)
    got = ops.route_metadata(torch.from_numpy(idx).reshape(T, K).cuda(), E)
    ref = ometa.tc_metadata(idx.reshape(T, K), E)
    for name, g, r in zip(("freq", "off", "gather", "scatter", "rev"), got, ref):
        np.testing.assert_array_equal(g.cpu().numpy(), r, err_msg=name)


def test_route_metadata_golden(ops, golden):
    d = golden("metadata_ref.npz")
    for key, E in (("tc_2048_512_10", 512), ("tc_1000_96_7", 96), ("edge_same", 8), ("edge_single", 8),
                   ("edge_empty", 64)):
        idx = torch.from_numpy(d[key + "_idx"].astype(np.int32)).cuda()
        got = ops.route_metadata(idx, E)
        for n, g in zip(("freq", "off", "gather", "scatter", "rev"), got):
            np.testing.assert_array_equal(g.cpu().numpy(), d[key + "_" + n], err_msg=f"{key} {n}")


def test_route_metadata_deterministic_and_skewed(ops):
    T, E, K = 4096, 64, 4
    idx = np.zeros((T, K), dtype=np.int32)
    idx[:, 1], idx[:, 2], idx[:, 3] = 1, 2, 3  # every token on the same four experts
    t = torch.from_numpy(idx).cuda()
    a = ops.route_metadata(t, E)
    b = ops.route_metadata(t, E)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    ref = ometa.tc_metadata(idx, E)
    for g, r in zip(a, ref):
        np.testing.assert_array_equal(g.cpu().numpy(), r)


def test_route_metadata_bad_expert_sets_error(ops):
    idx = torch.tensor([[0, 9]], dtype=torch.int32).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.route_metadata(idx, 8, err=err)
    assert err.item() == 201


@pytest.mark.parametrize("T,E,avg_k", [(10, 8, 2), (236, 16, 4), (1000, 96, 7), (50, 384, 3), (8192, 128, 8)])
def test_general_route_metadata_bit_exact(ops, T, E, avg_k):
    rs = np.random.RandomState(T)
    toks, exps = [], []
    for t in range(T):
        k = rs.randint(1, min(2 * avg_k, E) + 1)
        toks += [t] * k
        exps += list(rs.permutation(E)[:k])
    tok = np.array(toks, dtype=np.int32)
    ex = np.array(exps, dtype=np.int32)
    got = ops.general_route_metadata(torch.from_numpy(tok).cuda(), torch.from_numpy(ex).cuda(), T, E)
    ref = ometa.general_metadata(tok, ex, T, E)
    for name, g, r in zip(("freq", "off", "gather", "scatter", "rev", "tokoff"), got, ref):
        np.testing.assert_array_equal(g.cpu().numpy(), r, err_msg=name)


def test_route_plan_padded_layout(ops):
    T, E, K = 3000, 32, 4
    idx = _make_topk_indices(T, E, K, seed=5)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    plan = ops.route_plan(torch.from_numpy(idx).cuda(), E, err)
    freq = np.bincount(idx.reshape(-1), minlength=E)
    off_pad, blk_expert, nblk = ometa.padded_layout(freq)
    np.testing.assert_array_equal(plan.off_pad.cpu().numpy(), off_pad)
    assert plan.n_blocks.item() == nblk
    np.testing.assert_array_equal(plan.blk_expert.cpu().numpy()[:nblk], blk_expert)
    assert err.item() == 0
