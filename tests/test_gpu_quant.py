"""GPU parity: e4m3 quantisers, bit-exact against the quantiser spec (oracle/quant.py)."""
import numpy as np
import pytest
import torch

from oracle import metadata as ometa
from oracle import quant as oq
from _util import sf_bytes_of_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from sonicmoe import ops as _ops

    return _ops


def _bf16(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("R,C,scale", [(256, 512, 1.0), (300, 4096, 0.2), (7, 128, 30.0), (130, 768, 1e-3), (64, 7168, 5.0)])
def test_quant_1x128_bit_exact(ops, R, C, scale):
    x = _bf16((R, C), seed=R + C, scale=scale)
    q, sf = ops.quant_1x128(x.cuda())
    q_ref, sf_ref = oq.quant_1x128(x.float().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(sf.cpu().numpy(), oq.act_sf_atoms(sf_ref))


def test_quant_edge_values(ops):
    """Zeros, amax exactly 448*2^k, values that round to the e4m3 subnormals, saturation corner."""
    rows = []
    r = np.zeros(256, np.float32)
    rows.append(r)  # all zero -> scale byte 0, q = 0
    r = np.full(256, 3.0, np.float32)
    r[0] = 448.0 * 4
    rows.append(r)
    r = np.linspace(-1, 1, 256).astype(np.float32) * 1e-2
    r[5] = 448.0
    rows.append(r)  # tiny values under a large amax -> subnormal / zero codes
    r = np.random.RandomState(0).randn(256).astype(np.float32) * 1e4
    rows.append(r)
    x = torch.from_numpy(np.stack(rows)).to(torch.bfloat16)
    q, sf = ops.quant_1x128(x.cuda())
    q_ref, sf_ref = oq.quant_1x128(x.float().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(sf.cpu().numpy(), oq.act_sf_atoms(sf_ref))


@pytest.mark.parametrize("E,N,K,concat", [(4, 256, 256, False), (3, 512, 384, True), (2, 2048, 1024, False), (2, 1536, 2048, True)])
def test_weight_prep_bit_exact(ops, E, N, K, concat):
    w = _bf16((E, N, K), seed=N + K, scale=0.02)
    prep = ops.weight_prep(w.cuda(), concat_glu=concat)
    wf = w.float().numpy()
    src = oq.concat_to_blocked(wf) if concat else wf
    q_ref, sf_ref = oq.quant_128x128(wf)
    if concat:
        q_ref = oq.concat_to_blocked(q_ref)
        I = N // 2
        g_sf, u_sf = sf_ref[:, : I // 128], sf_ref[:, I // 128 :]
        sf_ref = np.stack([g_sf, u_sf], axis=2).reshape(E, N // 128, K // 128)
    q_dir, _ = oq.quant_128x128(src)
    np.testing.assert_array_equal(q_ref, q_dir)  # re-blocking commutes with 128x128 quantisation
    np.testing.assert_array_equal(prep.q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(prep.sf.cpu().numpy(), oq.weight_sf_atoms(sf_ref))


@pytest.mark.parametrize("T,H,E,K", [(256, 512, 8, 2), (1000, 2048, 32, 4), (64, 4096, 128, 8)])
def test_quant_pack_bit_exact(ops, T, H, E, K):
    rs = np.random.RandomState(T)
    idx = np.stack([rs.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    x = _bf16((T, H), seed=T, scale=0.5)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    plan = ops.route_plan(torch.from_numpy(idx).cuda(), E, err)
    xq, xsf = ops.quant_pack(x.cuda(), torch.from_numpy(idx).cuda(), plan)
    q_ref, sf_ref = oq.quant_1x128(x.float().numpy())
    freq, off, _, _, s_rev = ometa.tc_metadata(idx, E)
    off_pad, _, _ = ometa.padded_layout(freq)
    rows = ometa.padded_rows(idx, s_rev, off, off_pad)
    tok = np.repeat(np.arange(T), K)
    xq_h = xq.cpu().numpy()
    np.testing.assert_array_equal(xq_h[rows], q_ref[tok])
    got_sf = sf_bytes_of_rows(xsf.cpu().numpy(), rows, H // 128)
    np.testing.assert_array_equal(got_sf, sf_ref[tok])
