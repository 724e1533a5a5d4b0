"""CPU tests: the oracle against the reference's golden vectors and known-answer cases."""
import numpy as np
import pytest
import torch

from oracle import layer, metadata, quant, routing
from oracle.mathfn import exp_f32, log_f32


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- math functions
def test_exp_log_accuracy():
    x = np.linspace(-87, 0, 100001).astype(np.float32)
    ref = np.exp(x.astype(np.float64))
    assert (np.abs(exp_f32(x) - ref) / ref).max() < 4 * 2.0**-24
    s = np.linspace(1, 8192, 100001).astype(np.float32)
    assert np.abs(log_f32(s) - np.log(s.astype(np.float64))).max() < 2e-6
    assert exp_f32(np.float32(-200.0)) == 0.0
    assert exp_f32(np.float32(0.0)) == 1.0


# ---------------------------------------------------------------- routing
@pytest.mark.parametrize("case", [(256, 128, 8), (64, 96, 7), (32, 64, 4)])
@pytest.mark.parametrize("mode", ["sot", "tos", "tosn"])
def test_routing_matches_reference(golden, case, mode):
    d = golden("routing_ref.npz")
    T, E, K = case
    logits = bf16_to_f32(d[f"logits_{T}_{E}_{K}"])
    sot, norm = {"sot": (True, False), "tos": (False, False), "tosn": (False, True)}[mode]
    s, i = routing.topk_route(logits, K, sot, norm)
    np.testing.assert_array_equal(i, d[f"idx_{mode}_{T}_{E}_{K}"])
    # Softmax over top-k: the bf16 logits lose nothing to the index bits -> fp32 rounding only.
    # Top-k over softmax: the reference kernel drops the low log2(next_pow2(E)) mantissa bits of
    # the log-probabilities (topk.py:213-215) that its torch branch keeps, so the probability
    # differs by up to |logp| * 2^(log2(E) - 23) relative (|logp| < 8 here).
    rtol = 2e-6 if mode == "sot" else 8.0 * 2.0 ** (int(np.ceil(np.log2(E))) - 23)
    np.testing.assert_allclose(s, d[f"scores_{mode}_{T}_{E}_{K}"], rtol=rtol, atol=1e-7)


def test_routing_tie_semantics():
    """Known answers from sonicmoe/functional/topk.py:200-234: equal scores -> lower expert first,
    for positive and for negative values; output is in descending order."""
    logits = np.array(
        [
            [1.0, 2.0, 2.0, 0.5, 2.0, -1.0, 0.0, 0.0],
            [-1.0, -0.5, -0.5, -3.0, -0.5, -2.0, -4.0, -0.5],
            [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],
            [-2.0, -2.0, -2.0, -2.0, -2.0, -2.0, -2.0, -2.0],
        ],
        dtype=np.float32,
    )
    s, i = routing.topk_route(logits, 3, True)
    np.testing.assert_array_equal(i[0], [1, 2, 4])
    np.testing.assert_array_equal(i[1], [1, 2, 4])
    np.testing.assert_array_equal(i[2], [0, 1, 2])
    np.testing.assert_array_equal(i[3], [0, 1, 2])
    np.testing.assert_allclose(s[2], [1 / 3] * 3, rtol=1e-6)


def test_routing_truncation_ties_topk_over_softmax():
    """Top-k over softmax ranks log-probs whose low log2(E) mantissa bits are dropped
    (topk.py:195-215); two logits one float32 ulp apart become a tie won by the lower index."""
    x = np.zeros((1, 8), dtype=np.float32)
    x[0, 5] = np.float32(1.0)
    x[0, 3] = np.nextafter(np.float32(1.0), np.float32(2.0))  # larger, but only in low bits
    s, i = routing.topk_route(x, 2, False)
    np.testing.assert_array_equal(i[0], [3, 5])  # tie after truncation -> lower index first
    x2 = x.copy()
    x2[0, 3], x2[0, 5] = x[0, 5], x[0, 3]
    s2, i2 = routing.topk_route(x2, 2, False)
    np.testing.assert_array_equal(i2[0], [3, 5])


# ---------------------------------------------------------------- metadata
def _check_tc(d, key, E):
    idx = d[key + "_idx"]
    freq, off, gather, scatter, rev = metadata.tc_metadata(idx, E)
    for n, v in zip(("freq", "off", "gather", "scatter", "rev"), (freq, off, gather, scatter, rev)):
        np.testing.assert_array_equal(v, d[key + "_" + n], err_msg=f"{key} {n}")


@pytest.mark.parametrize("shape", [(10, 8, 2), (236, 16, 4), (1024, 128, 8), (1000, 96, 7), (50, 384, 3), (2048, 512, 10)])
def test_tc_metadata_matches_reference(golden, shape):
    d = golden("metadata_ref.npz")
    T, E, K = shape
    _check_tc(d, f"tc_{T}_{E}_{K}", E)


@pytest.mark.parametrize("name,E", [("same", 8), ("single", 8), ("empty", 64)])
def test_tc_metadata_edges(golden, name, E):
    _check_tc(golden("metadata_ref.npz"), f"edge_{name}", E)


@pytest.mark.parametrize("shape", [(10, 8, 2), (236, 16, 4), (1000, 96, 7), (50, 384, 3)])
def test_general_metadata_matches_reference(golden, shape):
    d = golden("metadata_ref.npz")
    T, E, k = shape
    key = f"gen_{T}_{E}_{k}"
    res = metadata.general_metadata(d[key + "_tok"], d[key + "_exp"], T, E)
    for n, v in zip(("freq", "off", "gather", "scatter", "rev", "tokoff"), res):
        np.testing.assert_array_equal(v, d[key + "_" + n], err_msg=f"{key} {n}")


def test_padded_layout():
    freq = np.array([0, 1, 128, 129, 0, 300])
    off_pad, blk_expert, nblk = metadata.padded_layout(freq)
    np.testing.assert_array_equal(off_pad, [0, 0, 128, 256, 512, 512, 896])
    np.testing.assert_array_equal(blk_expert, [1, 2, 3, 3, 5, 5, 5])
    assert nblk == 7


# ---------------------------------------------------------------- quantiser spec
def test_e4m3_matches_torch():
    v = np.concatenate(
        [
            np.linspace(-448, 448, 200001),
            np.random.RandomState(0).randn(100000) * 50,
            np.random.RandomState(1).randn(100000) * 1e-2,
        ]
    ).astype(np.float32)
    mine = quant.e4m3_encode(v)
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(mine, ref)


def test_quant_scale_rules():
    x = np.zeros((4, 128), dtype=np.float32)
    x[0, 0] = 448.0  # amax/448 = 1 -> e = 0
    x[1, 5] = -449.0  # just above -> e = 1
    x[2, :] = 1e-3  # ceil(log2(1e-3/448)) = -18
    q, sf = quant.quant_1x128(x)
    assert sf[:, 0].tolist() == [127, 128, 127 - 18, 0]
    assert q[0, 0] == 0x7E and q[1, 5] == 0xF6  # 448 ; -224.5 -> RNE -> -224 (0xF6)
    np.testing.assert_array_equal(q[3], 0)
    d = quant.dequant_1x128(q, sf)
    assert d[0, 0] == 448.0 and d[1, 5] == -448.0


def test_quant_roundtrip_error():
    rs = np.random.RandomState(3)
    x = rs.randn(64, 512).astype(np.float32)
    q, sf = quant.quant_1x128(x)
    d = quant.dequant_1x128(q, sf)
    assert np.abs(d - x).max() <= np.abs(x).max() * 2.0**-3  # e4m3 has 3 mantissa bits
    w = (rs.randn(2, 256, 384) * 0.02).astype(np.float32)
    wq, ws = quant.quant_128x128(w)
    assert ws.shape == (2, 2, 3)
    wd = quant.dequant_128x128(wq, ws)
    assert layer.rel_fro(wd, w) < 0.05


def test_fast_weight_fake_quant_matches_spec():
    """The torch-conversion fake quantiser used at full sizes equals the spec path bit for bit,
    including zero blocks, subnormal-scale blocks, round-half-even ties and the 448 edge."""
    rs = np.random.RandomState(11)
    w = (rs.randn(3, 256, 384) * 0.02).astype(np.float32)
    w[0, :128, :128] = 0.0
    w[1, 128:, 128:256] = rs.randn(128, 128).astype(np.float32) * 1e-39
    w[2, 0, 0] = 448.0 * 7
    w[2, 1, :8] = np.float32(448.0 * 7) * np.array([0.5, 0.53125, 0.5625, 1 / 64, 1 / 512, 3 / 1024, -1.0, -0.03125],
                                                     dtype=np.float32)
    ref = quant.dequant_128x128(*quant.quant_128x128(w))
    fast = quant.fake_quant_128x128_fast(w)
    assert np.array_equal(ref.view(np.uint32), fast.view(np.uint32))


def test_sf_atoms_layout():
    sf = np.arange(130 * 5, dtype=np.uint8).reshape(130, 5)
    at = quant.act_sf_atoms(sf)
    assert at.shape == (2, 2, 512)
    r, g = 37, 2
    assert at[0, 0, 16 * (r % 32) + 4 * (r // 32) + g] == sf[r, g]
    r, g = 129, 4
    assert at[1, 1, 16 * 1 + 4 * 0 + 0] == sf[r, g]


# ---------------------------------------------------------------- layer restatements
def test_reference_port_matches_reference(golden):
    d = golden("layer_ref.npz")
    T, H, I, E, K = d["shape"].tolist()
    x = torch.from_numpy(bf16_to_f32(d["x"]).reshape(T, H))
    rw = torch.from_numpy(bf16_to_f32(d["router_w"]).reshape(E, H))
    w1 = torch.from_numpy(bf16_to_f32(d["w1"]).reshape(E, 2 * I, H))
    w2 = torch.from_numpy(bf16_to_f32(d["w2"]).reshape(E, H, I))
    o, _, _ = layer.reference_port(x, rw, w1, w2, K)
    np.testing.assert_array_equal(o.numpy(), d["o"])


def test_expert_loop_concat_matches_reference(golden):
    d = golden("layer_ref.npz")
    if "concat_tosn_o" not in d:
        pytest.skip("fixture generated without the benchmark's swiglu")
    T, H, I, E, K = d["shape"].tolist()
    x = bf16_to_f32(d["x"]).reshape(T, H)
    w1 = bf16_to_f32(d["w1"]).reshape(E, 2 * I, H)
    w2 = bf16_to_f32(d["w2"]).reshape(E, H, I)
    o = layer.expert_loop(x, w1, w2, d["concat_tosn_scores"], d["concat_tosn_idx"], concat_layout=True)
    assert layer.rel_fro(o, d["concat_tosn_o"]) < 1e-5


def test_c1_reference_port(golden):
    d = golden("c1_ref.npz")
    T, H, I, E, K = 256, 512, 256, 8, 2
    g = torch.Generator().manual_seed(1111)
    rw = torch.randn(E, H, generator=g) * 0.02
    w1 = torch.randn(E, 2 * I, H, generator=g) * 0.02
    w2 = torch.randn(E, H, I, generator=g) * 0.02
    x = torch.randn(T, H, generator=g)
    assert abs(x.double().sum().item() + w1.double().sum().item() - float(d["input_sum"])) < 1e-6
    o, _, _ = layer.reference_port(x, rw, w1, w2, K)
    np.testing.assert_allclose(o[:8].numpy(), d["rows"], rtol=1e-5, atol=1e-6)
    assert abs(o.double().sum().item() - float(d["sum"])) < 1e-3
    assert abs((o.double() ** 2).sum().item() - float(d["sumsq"])) / float(d["sumsq"]) < 1e-6


def test_fp8_oracle_close_to_dense():
    """The fake-quantised layer stays near the dense layer; the gap is the e4m3 floor."""
    rs = np.random.RandomState(7)
    T, H, I, E, K = 64, 256, 128, 4, 2
    x = torch.from_numpy(rs.randn(T, H).astype(np.float32)).bfloat16().float()
    w1 = torch.from_numpy((rs.randn(E, 2 * I, H) * 0.02).astype(np.float32)).bfloat16().float()
    w2 = torch.from_numpy((rs.randn(E, H, I) * 0.02).astype(np.float32)).bfloat16().float()
    rw = torch.from_numpy((rs.randn(E, H) * 0.02).astype(np.float32)).bfloat16().float()
    logits = (x @ rw.T).bfloat16().float().numpy()
    o8, sc, idx = layer.fp8_oracle(x.numpy(), logits, w1.numpy(), w2.numpy(), K)
    od = layer.expert_loop(x, w1, w2, sc, idx, concat_layout=False)
    err = layer.rel_fro(o8, od)
    assert 0.0 < err < 0.15


def test_fp8_oracle_rows_matches_whole_layer_oracle():
    """The per-token oracle used at full configuration sizes equals the whole-layer oracle on the
    rows it computes (interleaved and concatenated w1)."""
    rs = np.random.RandomState(11)
    T, H, I, E, K = 24, 256, 128, 6, 3
    x = rs.randn(T, H).astype(np.float32)
    logits = rs.randn(T, E).astype(np.float32)
    w1 = (rs.randn(E, 2 * I, H) * 0.02).astype(np.float32)
    w2 = (rs.randn(E, H, I) * 0.02).astype(np.float32)
    for concat in (False, True):
        o, scores, idx = layer.fp8_oracle(x, logits, w1, w2, K, concat_layout=concat)
        rows = np.array([0, 5, 17, 23])
        sub = layer.fp8_oracle_rows(x[rows], scores[rows], idx[rows], lambda e: (w1[e], w2[e]), concat)
        np.testing.assert_allclose(sub.numpy(), o.numpy()[rows], rtol=1e-12, atol=1e-12)


def test_home_rows_layout_invariants():
    """The home-down expert-parallel path writes entry (t, k) of a rank's tokens into row
    s_rev - off[e] + off_pad[e] of that rank's padded layout, encoded as (source rank << 27) | row,
    and its scale byte for k-group g into atom ((row/128)*KG + g/4)*512 + 16*(row%32) +
    4*((row%128)/32) + g%4.  On random routing: the rows are a bijection onto each expert's valid
    rows, stay below max_padded_blocks(T*K, E)*128, survive the encoding, and no two (row, k-group)
    pairs share a scale byte inside the atom buffer."""
    rs = np.random.RandomState(11)
    T, E, K, I, W = 300, 24, 6, 384, 3
    idx = np.stack([rs.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    freq, off, _, _, s_rev = metadata.tc_metadata(idx, E)
    off_pad, _, nblk = metadata.padded_layout(freq)
    rows = metadata.padded_rows(idx, s_rev, off, off_pad)
    max_rows = ((T * K + 127) // 128 + min(T * K, E)) * 128  # sm_max_padded_blocks(T*K, E) * 128
    assert nblk * 128 <= max_rows and rows.max() < max_rows
    assert len(np.unique(rows)) == T * K
    e = idx.reshape(-1)
    assert np.all(rows >= off_pad[e]) and np.all(rows < off_pad[e] + freq[e])
    for s in range(W):
        code = (s << 27) | rows
        assert np.all(code >> 27 == s) and np.all(code & ((1 << 27) - 1) == rows)
    KG = -(-(I // 128) // 4)
    g = np.arange(I // 128)
    r = rows[:, None]
    byte = ((r // 128) * KG + g // 4) * 512 + 16 * (r % 32) + 4 * ((r % 128) // 32) + g % 4
    assert len(np.unique(byte)) == byte.size and byte.max() < (max_rows // 128) * KG * 512


# ---------------------------------------------------------------- backward restatement
def test_router_backward_matches_autograd():
    """oracle.backward.router_backward against torch autograd of the router's forward math
    (softmax over the top-k; top-k of the softmax, optionally renormalised), float64."""
    from oracle import backward as obwd

    rs = np.random.RandomState(5)
    T, E, K = 40, 16, 4
    lg = rs.randn(T, E)
    g = rs.randn(T, K)
    idx = np.argsort(-lg, axis=1)[:, :K]
    for sot, norm in ((True, False), (False, False), (False, True)):
        lt = torch.tensor(lg, requires_grad=True)
        sel = torch.gather(lt, 1, torch.from_numpy(idx))
        if sot:
            s = torch.softmax(sel, dim=1)
        else:
            p = torch.softmax(lt, dim=1)
            s = torch.gather(p, 1, torch.from_numpy(idx))
            if norm:
                s = s / s.sum(1, keepdim=True)
        (s * torch.from_numpy(g)).sum().backward()
        got = obwd.router_backward(lg, s.detach().numpy(), idx, g, sot, norm)
        np.testing.assert_allclose(got, lt.grad.numpy(), rtol=1e-10, atol=1e-12)


def test_backward_general_equals_topk_form():
    """The explicit-entries backward equals the top-k backward on the same routing."""
    from oracle import backward as obwd
    from oracle import quant as oq

    rs = np.random.RandomState(6)
    T, H, I, E, K = 64, 256, 128, 8, 2
    x = (rs.randn(T, H)).astype(np.float32)
    w1 = (rs.randn(E, 2 * I, H) * 0.02).astype(np.float32)
    w2 = (rs.randn(E, H, I) * 0.02).astype(np.float32)
    idx = np.stack([np.sort(rs.permutation(E)[:K]) for _ in range(T)]).astype(np.int32)
    sc = rs.rand(T, K).astype(np.float32)
    dout = (rs.randn(T, H) * 0.1).astype(np.float32)
    # pre-activation of the fake-quantised operands, rows in expert-sorted order
    xd = oq.dequant_1x128(*oq.quant_1x128(x))
    w1d = oq.dequant_128x128(*oq.quant_128x128(w1))
    _, _, _, s_scatter, _ = metadata.tc_metadata(idx, E)
    f = s_scatter.astype(np.int64)
    h = np.einsum("rh,rnh->rn", xd[f // K], w1d[idx.reshape(-1)[f]]).astype(np.float32)
    a = obwd.fp8_backward(x, dout, w1, w2, sc, idx, h)
    b = obwd.fp8_backward_general(x, dout, w1, w2, sc.reshape(-1), np.arange(T * K) // K, idx.reshape(-1), h)
    for u, v in zip(a[:3], b[:3]):
        np.testing.assert_allclose(u, v, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(a[3].reshape(-1), b[3], rtol=1e-12, atol=1e-12)
