"""GPU parity of the FP8 backward (stages of ``sonicmoe.ops.moe_backward`` and the autograd path of
``moe_TC_softmax_topk_layer`` / ``MoE``) against the CPU restatement in ``oracle/backward.py``.

Tolerance: relative Frobenius error <= 1e-2 for every gradient against the float64 oracle that
fake-quantises the same operands (1x128 / 128x128 / column-wise e4m3, bf16 intermediates) -- the
bound the forward uses.
"""
import numpy as np
import pytest
import torch

from oracle import backward as obwd
from oracle import routing as oroute
from _util import make_layer_inputs, rel_fro

pytestmark = pytest.mark.gpu

TOL = 1e-2

CASES = [
    # T, H, I, E, K, softmax_over_topk, norm, concat
    (256, 512, 256, 8, 2, True, False, False),
    (384, 1024, 512, 16, 4, False, True, True),  # Qwen3-style routing + concatenated w1
    (64, 512, 256, 64, 8, False, False, False),  # most experts empty
    (320, 512, 768, 8, 4, True, False, True),  # concat with I = 768 (three 256-column tiles)
]


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from sonicmoe import ops as _ops

    return _ops


def _forward_state(ops, x, rw, w1, w2, K, sot, norm, concat=False):
    """Routing, plan and stored pre-activation of the training forward (as the autograd function runs it)."""
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    logits = torch.nn.functional.linear(x, rw)
    scores, idx = ops.router_topk(logits, K, sot, norm)
    plan = ops.route_plan(idx, w1.shape[0], err)
    xq, xsf = ops.quant_pack(x, idx, plan)
    h = torch.empty(x.shape[0] * K, w1.shape[1], dtype=torch.bfloat16, device="cuda")
    ops.moe_up(xq, xsf, ops.weight_prep(w1, concat_glu=concat), plan, err, preact_out=h)
    return logits, scores, idx, plan, h, err


@pytest.mark.parametrize("T,H,I,E,K,sot,norm,concat", CASES)
def test_moe_backward_stages_vs_oracle(ops, T, H, I, E, K, sot, norm, concat):
    x, rw, w1, w2 = make_layer_inputs(T, H, I, E, seed=11 * T + E)
    xc, rwc, w1c, w2c = x.cuda(), rw.cuda(), w1.cuda(), w2.cuda()
    logits, scores, idx, plan, h, err = _forward_state(ops, xc, rwc, w1c, w2c, K, sot, norm, concat)
    g = torch.Generator().manual_seed(T + 1)
    dout = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16)
    dx, dl, dw1, dw2, ds = ops.moe_backward(dout.cuda(), xc, logits, ops.weight_prep(w1c, concat_glu=concat),
                                            ops.weight_prep(w2c), scores, idx, plan, h, sot, norm, err)
    torch.cuda.synchronize()
    assert err.item() == 0, f"kernel error word {err.item()}"
    s_np, i_np = scores.cpu().numpy(), idx.cpu().numpy()
    s_ref, i_ref = oroute.topk_route(logits.float().cpu().numpy(), K, sot, norm)
    np.testing.assert_array_equal(i_np, i_ref)
    rdx, rdw1, rdw2, rds, rdl = obwd.fp8_backward(
        x.float().numpy(), dout.float().numpy(), w1.float().numpy(), w2.float().numpy(), s_np, i_np,
        h.float().cpu().numpy(), sot, norm, logits=logits.float().cpu().numpy(), concat_layout=concat)
    for name, got, ref in (("ds", ds, rds), ("dlogits", dl, rdl), ("dx", dx, rdx), ("dw2", dw2, rdw2),
                           ("dw1", dw1, rdw1)):
        err_rel = rel_fro(got.float().cpu().numpy(), ref)
        assert err_rel <= TOL, f"{name}: rel. Frobenius {err_rel:.3g}"


def test_router_bwd_matches_oracle(ops):
    T, E, K = 300, 64, 6
    g = torch.Generator().manual_seed(3)
    lg = torch.randn(T, E, generator=g).to(torch.bfloat16)
    ds = torch.randn(T, K, generator=g)
    for sot, norm in ((True, False), (False, False), (False, True)):
        s, i = ops.router_topk(lg.cuda(), K, sot, norm)
        dl = ops.router_bwd(lg.cuda(), s, i, ds.cuda(), sot, norm)
        ref = obwd.router_backward(lg.float().numpy(), s.cpu().numpy(), i.cpu().numpy(), ds.numpy(), sot, norm)
        assert rel_fro(dl.cpu().numpy(), ref) < 1e-5


def test_weight_prep_t_is_the_transpose(ops):
    """The transposed weight holds the forward's e4m3 values read transposed, and its scale atoms the
    same 128x128 block scales: both dequantise to the transposed fake-quantised weight."""
    from oracle import quant as oq

    g = torch.Generator().manual_seed(4)
    w = (torch.randn(3, 256, 384, generator=g) * 0.05).to(torch.bfloat16)
    w_f = ops.weight_prep(w.cuda())
    wt = ops.weight_prep_t(w_f)
    assert torch.equal(wt.q.cpu(), w_f.q.cpu().transpose(1, 2))
    q, sf = oq.quant_128x128(w.float().numpy())
    np.testing.assert_array_equal(wt.q.cpu().numpy(), q.transpose(0, 2, 1))
    # scale of block (k, n) of the transpose = scale of block (n, k): byte (n % 4) of atom (e, k, n / 4)
    atoms = wt.sf.cpu().numpy()  # [E, K/128, ceil(N/512), 512]
    for e in range(3):
        for kb in range(384 // 128):
            for nb in range(256 // 128):
                assert atoms[e, kb, nb // 4, nb % 4] == sf[e, nb, kb]


@pytest.mark.parametrize("concat", [False, True])
def test_weight_prep_with_t_matches_the_two_passes(ops, concat):
    """The one-pass preparation (forward weight + transposed copy) writes exactly what weight_prep
    followed by weight_prep_t writes, in both w1 layouts."""
    g = torch.Generator().manual_seed(6)
    w = (torch.randn(3, 512, 384, generator=g) * 0.05).to(torch.bfloat16).cuda()
    both = ops.weight_prep(w, concat_glu=concat, with_t=True)
    one = ops.weight_prep(w, concat_glu=concat)
    t = ops.weight_prep_t(one)
    assert ops.weight_prep_t(both) is both.t
    for a, b in ((both.q, one.q), (both.sf, one.sf), (both.t.q, t.q), (both.t.sf, t.sf)):
        assert torch.equal(a, b)


@pytest.mark.parametrize("concat", [False, True])
def test_tq_pack_dual_matches_dact_q_and_tq_pack(ops, concat):
    """The dual operand pack of dH writes, from one read, the dX operand bit for bit as the dA'
    epilogue's own e4m3 copy (row groups, re-blocked for a concatenated w1) and the dW1 operand bit
    for bit as tq_pack; the epilogue without its e4m3 copy writes the same bf16 dH, a' and dS."""
    T, H, I, E, K = 300, 512, 256, 8, 4
    x, rw, w1, w2 = make_layer_inputs(T, H, I, E, seed=21)
    xc, rwc, w1c, w2c = x.cuda(), rw.cuda(), w1.cuda(), w2.cuda()
    logits, scores, idx, plan, h, err = _forward_state(ops, xc, rwc, w1c, w2c, K, True, False, concat)
    g = torch.Generator().manual_seed(22)
    dout = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16).cuda()
    doq, dosf = ops.quant_pack(dout, idx, plan)
    w2t = ops.weight_prep_t(ops.weight_prep(w2c))
    dh_q, dh_sf, dh, ap, ds = ops.moe_dact(doq, dosf, w2t, plan, scores.view(-1), h, err, concat_layout=concat)
    n_q, n_sf, dh2, ap2, ds2 = ops.moe_dact(doq, dosf, w2t, plan, scores.view(-1), h, err, concat_layout=concat,
                                            with_q=False)
    assert n_q is None and n_sf is None
    cq, csf, rq, rsf = ops.tq_pack_dual(dh, plan, concat_i=I if concat else 0)
    tq, tsf = ops.tq_pack(dh, plan, True)
    torch.cuda.synchronize()
    assert err.item() == 0
    nb = int(plan.n_blocks.item())
    valid = torch.zeros(plan.max_blocks * 128, dtype=torch.bool)
    fr, op = plan.freq.cpu(), plan.off_pad.cpu()
    for e in range(E):
        valid[int(op[e]):int(op[e]) + int(fr[e])] = True
    valid = valid.cuda()
    assert torch.equal(rq[valid], dh_q[valid])
    # scale bytes of the valid rows: rows r of block b at byte 16 (r % 32) + 4 (r / 32) + (kb % 4)
    rows = torch.nonzero(valid).view(-1).cpu()
    kbs = torch.arange(2 * I // 128)
    byte = (16 * (rows % 32) + 4 * ((rows % 128) // 32))[:, None] + (kbs % 4)[None, :]
    blk, kg = (rows // 128)[:, None].expand(-1, kbs.numel()), (kbs // 4)[None, :].expand(rows.numel(), -1)
    assert torch.equal(rsf.cpu()[blk, kg, byte], dh_sf.cpu()[blk, kg, byte])
    assert torch.equal(cq[:, :nb * 128], tq[:, :nb * 128]) and torch.equal(csf, tsf)
    assert torch.equal(dh2[valid], dh[valid]) and torch.equal(ap2[valid], ap[valid])
    torch.testing.assert_close(ds2, ds, rtol=1e-5, atol=1e-6)  # fp32 atomics: order may differ


@pytest.mark.parametrize("padded", [False, True])
@pytest.mark.parametrize("T,C,E,K", [(300, 512, 8, 2), (200, 384, 64, 8)])
def test_tq_pack_bit_exact(ops, T, C, E, K, padded):
    """The weight-gradient operand: column c of the padded layout's rows (token rows gathered, or the
    padded rows themselves with pad rows read as zero) quantised in 1x128 groups along the rows, bytes
    and scale atoms equal to the oracle quantiser's on the transposed matrix."""
    from oracle import metadata as ometa
    from oracle import quant as oq

    g = torch.Generator().manual_seed(T + C)
    lg = torch.randn(T, E, generator=g).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _, idx = ops.router_topk(lg.cuda(), K)
    plan = ops.route_plan(idx, E, err)
    i_np = idx.cpu().numpy()
    freq, off, _, _, s_rev = ometa.tc_metadata(i_np, E)
    off_pad, _, nblk = ometa.padded_layout(freq)
    prow = ometa.padded_rows(i_np, s_rev, off, off_pad)
    rows = plan.max_blocks * 128
    P = np.zeros((nblk * 128, C), dtype=np.float32)
    if padded:
        src = (torch.randn(rows, C, generator=g) * 3).to(torch.bfloat16)
        P[prow] = src.float().numpy()[prow]
    else:
        src = (torch.randn(T, C, generator=g) * 3).to(torch.bfloat16)
        P[prow] = src.float().numpy()[np.arange(T * K) // K]
    q, sf = ops.tq_pack(src.cuda(), plan, padded)
    torch.cuda.synchronize()
    assert err.item() == 0
    q_ref, e8_ref = oq.quant_1x128(P.T.copy())  # [C, nblk*128], [C, nblk]
    np.testing.assert_array_equal(q.cpu().numpy()[:, :nblk * 128], q_ref)
    atoms = sf.cpu().numpy()
    kg = -(-nblk // 4)
    np.testing.assert_array_equal(atoms[:, :kg], oq.act_sf_atoms(e8_ref))
    assert not atoms[:, kg:].any()


@pytest.mark.parametrize("T,H,I,E,K,sot,norm,concat", CASES[:2])
def test_layer_autograd_vs_oracle(T, H, I, E, K, sot, norm, concat):
    """moe_TC_softmax_topk_layer in training mode: gradients of x (expert path + router F.linear),
    router_w, w1, w2 through the autograd function, against the oracle plus the router GEMM's
    float64 backward."""
    from sonicmoe.functional import moe_TC_softmax_topk_layer

    x, rw, w1, w2 = make_layer_inputs(T, H, I, E, seed=13 * T + E)
    xc = x.cuda().requires_grad_()
    rwc = rw.cuda().requires_grad_()
    w1c = w1.cuda().requires_grad_()
    w2c = w2.cuda().requires_grad_()
    o, logits, freq = moe_TC_softmax_topk_layer(xc, rwc, w1c.permute(1, 2, 0), None, w2c.permute(1, 2, 0), None, K,
                                                None, is_inference_mode_enabled=False, is_softmax_over_topk=sot,
                                                norm_topk_probs=norm, concat_layout=concat)
    g = torch.Generator().manual_seed(T + 2)
    dout = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16)
    (o.float() * dout.cuda().float()).sum().backward()
    torch.cuda.synchronize()
    from sonicmoe import ops

    _, scores, idx, plan, h, _ = _forward_state(ops, x.cuda(), rw.cuda(), w1.cuda(), w2.cuda(), K, sot, norm, concat)
    lg = logits.detach().float().cpu().numpy()
    rdx, rdw1, rdw2, _, rdl = obwd.fp8_backward(
        x.float().numpy(), dout.float().numpy(), w1.float().numpy(), w2.float().numpy(), scores.cpu().numpy(),
        idx.cpu().numpy(), h.float().cpu().numpy(), sot, norm, logits=lg, concat_layout=concat)
    rdx_total = rdx + rdl @ rw.double().numpy()
    rdrw = rdl.T @ x.double().numpy()
    for name, got, ref in (("dx", xc.grad, rdx_total), ("drouter_w", rwc.grad, rdrw), ("dw1", w1c.grad, rdw1),
                           ("dw2", w2c.grad, rdw2)):
        assert got is not None, name
        err_rel = rel_fro(got.float().cpu().numpy(), ref)
        assert err_rel <= TOL, f"{name}: rel. Frobenius {err_rel:.3g}"


def test_training_refusals():
    from sonicmoe.functional import moe_TC_softmax_topk_layer

    x, rw, w1, w2 = make_layer_inputs(64, 512, 256, 8, seed=1)
    w1c = w1.cuda().requires_grad_()
    with pytest.raises(NotImplementedError, match="fused_router"):
        moe_TC_softmax_topk_layer(x.cuda(), rw.cuda(), w1c.permute(1, 2, 0), None, w2.cuda().permute(1, 2, 0), None,
                                  2, None, is_inference_mode_enabled=False, fused_router=True)


def _general_entries(T, E, avg_k, seed):
    rs = np.random.RandomState(seed)
    toks, exps, scs = [], [], []
    for t in range(T):
        k = rs.randint(0, min(2 * avg_k, E) + 1)  # tokens without entries get zero gradients
        e = rs.permutation(E)[:k]
        w = rs.rand(k).astype(np.float32)
        toks += [t] * k
        exps += list(e)
        scs += list(w / max(w.sum(), 1e-6))
    return (np.array(toks, dtype=np.int32), np.array(exps, dtype=np.int32), np.array(scs, dtype=np.float32))


@pytest.mark.parametrize("T,H,I,E,avg_k,concat", [(256, 512, 256, 8, 2, False), (300, 512, 512, 16, 4, True)])
def test_general_routing_autograd_vs_oracle(T, H, I, E, avg_k, concat):
    """moe_general_routing_inputs in training mode: gradients of x, the router scores, w1 and w2
    through the autograd function, against oracle.backward.fp8_backward_general."""
    from sonicmoe import ops
    from sonicmoe.functional import moe_general_routing_inputs

    x, _, w1, w2 = make_layer_inputs(T, H, I, E, seed=T + 5 * E)
    tok, ex, sc = _general_entries(T, E, avg_k, seed=T + 1)
    xc = x.cuda().requires_grad_()
    scc = torch.from_numpy(sc).cuda().requires_grad_()
    w1c = w1.cuda().requires_grad_()
    w2c = w2.cuda().requires_grad_()
    tokc, exc = torch.from_numpy(tok).cuda(), torch.from_numpy(ex).cuda()
    o, freq = moe_general_routing_inputs(xc, scc, tokc, exc, w1c.permute(1, 2, 0), None, w2c.permute(1, 2, 0), None,
                                         E, None, is_inference_mode_enabled=False, concat_layout=concat)
    g = torch.Generator().manual_seed(T + 3)
    dout = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16)
    (o.float() * dout.cuda().float()).sum().backward()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(freq.cpu().numpy(), np.bincount(ex, minlength=E))
    # the stored pre-activation, recomputed through the same stages
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    plan = ops.general_route_plan(tokc, exc, T, E, err)
    xq, xsf = ops.quant_pack_general(x.cuda(), exc, plan)
    h = torch.empty(tok.shape[0], 2 * I, dtype=torch.bfloat16, device="cuda")
    ops.moe_up(xq, xsf, ops.weight_prep(w1.cuda(), concat_glu=concat), plan, err, preact_out=h)
    rdx, rdw1, rdw2, rds = obwd.fp8_backward_general(x.float().numpy(), dout.float().numpy(), w1.float().numpy(),
                                                     w2.float().numpy(), sc, tok, ex, h.float().cpu().numpy(),
                                                     concat_layout=concat)
    for name, got, ref in (("dx", xc.grad, rdx), ("dscores", scc.grad, rds), ("dw1", w1c.grad, rdw1),
                           ("dw2", w2c.grad, rdw2)):
        assert got is not None, name
        err_rel = rel_fro(got.float().cpu().numpy(), ref)
        assert err_rel <= TOL, f"{name}: rel. Frobenius {err_rel:.3g}"
    counts = np.bincount(tok, minlength=T)
    assert torch.all(xc.grad[torch.from_numpy(counts == 0).cuda()] == 0)
