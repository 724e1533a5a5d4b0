"""GPU parity of the expert-parallel path.

* emulated: W virtual ranks on one GPU -- every rank's dispatch, expert and combine kernels run
  for real, the two all-to-alls are done by slicing on the device.  Checks the output against the
  fake-quantised oracle over all tokens and the per-rank expert counts against the routing.
* multi-GPU: W processes with NCCL (needs >= 2 GPUs; skipped otherwise), same check.
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle.layer import fp8_oracle, rel_fro
from _util import make_layer_inputs

pytestmark = pytest.mark.gpu

TOL_FP8 = 1e-2


def _exchange(send_bufs, counts):
    """All-to-all by slicing: send_bufs[s] is rank s's rank-major buffer, counts[s][d] its split sizes."""
    W = len(send_bufs)
    offs = [np.concatenate([[0], np.cumsum(c)]) for c in counts]
    return [torch.cat([send_bufs[s][offs[s][d]:offs[s][d] + counts[s][d]] for s in range(W)]) for d in range(W)]


@pytest.mark.parametrize("W,T,H,I,E,K", [(4, 200, 512, 256, 16, 4), (2, 333, 256, 128, 8, 8), (8, 64, 256, 128, 64, 8)])
def test_ep_emulated_ranks(W, T, H, I, E, K):
    assert torch.cuda.is_available()
    import torch.nn.functional as F

    from sonicmoe.ep import NativeStages
    from sonicmoe.ops import weight_prep

    x, rw, w1, w2 = make_layer_inputs(W * T, H, I, E, seed=W + T)
    dev = torch.device("cuda", 0)
    xg, rwg = x.to(dev), rw.to(dev)
    El = E // W
    st = NativeStages()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    w1p = [weight_prep(w1[r * El:(r + 1) * El].to(dev)) for r in range(W)]
    w2p = [weight_prep(w2[r * El:(r + 1) * El].to(dev)) for r in range(W)]
    states = []
    for r in range(W):
        xr = xg[r * T:(r + 1) * T].contiguous()
        states.append(st.dispatch(xr, F.linear(xr, rwg), E, K, W, r, True, False, err))
    send_counts = [s.send_counts.cpu().tolist() for s in states]
    recv = _exchange([s.records for s in states], send_counts)
    recv_counts = [[send_counts[s][d] for s in range(W)] for d in range(W)]
    outs, freqs = [], []
    for d in range(W):
        o, f = st.expert(recv[d].contiguous(), recv[d].shape[0], H, I, El, K, w1p[d], w2p[d], err)
        outs.append(o)
        freqs.append(f)
    ret = _exchange(outs, recv_counts)
    o_all = torch.cat([st.combine(ret[s].contiguous(), states[s].ret_row, T, K, H) for s in range(W)])
    torch.cuda.synchronize()
    assert err.item() == 0
    logits = torch.cat([s.router_logits for s in states]).float().cpu().numpy()
    o_ref, _, idx = fp8_oracle(x.float().numpy(), logits, w1.float().numpy(), w2.float().numpy(), K)
    np.testing.assert_array_equal(torch.cat(freqs).cpu().numpy(), np.bincount(idx.reshape(-1), minlength=E))
    assert rel_fro(o_all.float().cpu().numpy(), o_ref.numpy()) <= TOL_FP8


@pytest.mark.parametrize("W,T,H,I,E,K", [(4, 200, 512, 256, 16, 4), (3, 150, 256, 128, 12, 8)])
def test_ep_p2p_kernels_emulated_ranks(W, T, H, I, E, K):
    """The peer-memory stages with W buffers on one GPU: the expert stage reads each source's
    segment out of that source's send buffer, the combine reads each partial row out of the
    destination's output rows -- the same address arithmetic the IPC-mapped peers use."""
    import torch.nn.functional as F

    from sonicmoe.ep import NativeStages
    from sonicmoe.ops import weight_prep

    x, rw, w1, w2 = make_layer_inputs(W * T, H, I, E, seed=3 * W + T)
    dev = torch.device("cuda", 0)
    xg, rwg = x.to(dev), rw.to(dev)
    El = E // W
    st = NativeStages()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rb = st.record_bytes(H, K)
    send = [torch.empty(T * min(K, W), rb, dtype=torch.uint8, device=dev) for _ in range(W)]
    outs = [torch.empty(W * T, H, dtype=torch.bfloat16, device=dev) for _ in range(W)]
    states = []
    for r in range(W):
        xr = xg[r * T:(r + 1) * T].contiguous()
        states.append(st.dispatch(xr, F.linear(xr, rwg), E, K, W, r, True, False, err, records=send[r]))
    C = [s_.send_counts.cpu().tolist() for s_ in states]
    freqs = []
    for d in range(W):
        w1p = weight_prep(w1[d * El:(d + 1) * El].to(dev))
        w2p = weight_prep(w2[d * El:(d + 1) * El].to(dev))
        recv_counts = [C[s_][d] for s_ in range(W)]
        seg_off = [sum(C[s_][:d]) for s_ in range(W)]
        freqs.append(st.expert_p2p([b.data_ptr() for b in send], seg_off, recv_counts, H, I, El, K, w1p, w2p,
                                   outs[d].data_ptr(), err, dev))
    o_all = []
    for s_ in range(W):
        recv_start = [sum(C[q][d] for q in range(s_)) for d in range(W)]
        o_all.append(st.combine_p2p([o.data_ptr() for o in outs], C[s_], recv_start, states[s_].ret_row, T, K, H, dev))
    o_all = torch.cat(o_all)
    torch.cuda.synchronize()
    assert err.item() == 0
    logits = torch.cat([s_.router_logits for s_ in states]).float().cpu().numpy()
    o_ref, _, idx = fp8_oracle(x.float().numpy(), logits, w1.float().numpy(), w2.float().numpy(), K)
    np.testing.assert_array_equal(torch.cat(freqs).cpu().numpy(), np.bincount(idx.reshape(-1), minlength=E))
    assert rel_fro(o_all.float().cpu().numpy(), o_ref.numpy()) <= TOL_FP8


def _gpu_layer_inputs(T, H, I, E, seed):
    """Same distributions as make_layer_inputs, drawn on the GPU expert by expert (config 4's bf16
    weights are 22 GB; no host copy of all of them)."""
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    rw = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w1 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device=dev)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16, device=dev)
    for e in range(E):
        w1[e] = (torch.randn(2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w2[e] = (torch.randn(H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    return x, rw, w1, w2


def _home_emulated(W, T, H, I, E, K, seed, corrupt=False, inputs=make_layer_inputs, device_counts=False,
                   bad_count=False):
    """Home-down stages with W virtual ranks on one GPU: every owner's up GEMM stores its rows into
    the W separate home buffers (the peer-store address arithmetic), then every home runs the down
    projection over its own plan with all experts' w2.  With device_counts the owners' up stages
    read the count matrix from device memory (sm_ep_expert_up_home, grids sized for W * T records);
    bad_count plants a count past the send region there."""
    import torch.nn.functional as F

    from sonicmoe import ops
    from sonicmoe.ep import NativeStages
    from sonicmoe.ops import weight_prep

    x, rw, w1, w2 = inputs(W * T, H, I, E, seed=seed)
    dev = torch.device("cuda", 0)
    xg, rwg = x.to(dev), rw.to(dev)
    El = E // W
    st = NativeStages()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rb = st.record_bytes(H, K)
    home_rows = ops.max_padded_blocks(T * K, E) * 128
    send = [torch.empty(T * min(K, W), rb, dtype=torch.uint8, device=dev) for _ in range(W)]
    home_q = [torch.empty(home_rows, I, dtype=torch.uint8, device=dev) for _ in range(W)]
    home_sf = [torch.zeros(home_rows // 128, -(-I // 512), 512, dtype=torch.uint8, device=dev) for _ in range(W)]
    states, plans, logits = [], [], []
    for r in range(W):
        xr = xg[r * T:(r + 1) * T].contiguous()
        lg = F.linear(xr, rwg)
        scores, idx = ops.router_topk(lg, K, True, False)
        plan = ops.route_plan(idx, E, err)
        states.append(st.dispatch_records(xr, scores, idx, plan, E, W, err, records=send[r]))
        plans.append(plan)
        logits.append(lg)
    C = [s_.send_counts.cpu().tolist() for s_ in states]
    if corrupt:
        # one record of rank 0 names a home row past the end of the home buffer
        meta = (H + H // 128 + 15) // 16 * 16 + 8 * K
        row = send[0][0, meta:meta + 4 * K].view(torch.int32)
        row[:] = torch.where(row >= 0, torch.full_like(row, home_rows + 5), row)
    w2_full = weight_prep(w2.to(dev))
    counts = torch.stack([s_.send_counts for s_ in states]).view(-1).contiguous()  # [W * W], row = source
    if bad_count:
        counts[W - 1] = T * min(K, W) + 1  # source 0's segment for the last rank runs past its send region
    freqs = []
    for d in range(W):
        w1p = weight_prep(w1[d * El:(d + 1) * El].to(dev))
        if device_counts:
            freqs.append(st.expert_up_home([b.data_ptr() for b in send], counts, W, d, T * min(K, W), W * T, H, I,
                                           El, K, w1p, [q.data_ptr() for q in home_q],
                                           [f.data_ptr() for f in home_sf], home_rows, err, dev))
            continue
        recv_counts = [C[s_][d] for s_ in range(W)]
        seg_off = [sum(C[s_][:d]) for s_ in range(W)]
        freqs.append(st.expert_up_p2p([b.data_ptr() for b in send], seg_off, recv_counts, H, I, El, K, w1p,
                                      [q.data_ptr() for q in home_q], [f.data_ptr() for f in home_sf], home_rows,
                                      err, dev))
    outs = []
    for r in range(W):
        o = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
        ops.moe_down_combine(home_q[r], home_sf[r], w2_full, plans[r], states[r].topk_scores.view(-1), T, err, out=o)
        outs.append(o)
    torch.cuda.synchronize()
    return x, w1, w2, torch.cat(outs), torch.cat(logits), torch.cat(freqs), err.item()


@pytest.mark.parametrize("W,T,H,I,E,K", [(4, 200, 512, 256, 16, 4), (3, 150, 256, 128, 12, 8),
                                         (2, 333, 256, 384, 8, 8)])
@pytest.mark.parametrize("device_counts", [False, True])
def test_ep_home_kernels_emulated_ranks(W, T, H, I, E, K, device_counts):
    """Up projection at the experts' owners with its rows stored into the tokens' home buffers,
    down projection + combine at home: same output as the single-GPU layer's oracle, with the
    segment table passed from the host or resolved on the device from the count matrix."""
    x, w1, w2, o_all, logits, freq, e = _home_emulated(W, T, H, I, E, K, seed=5 * W + T,
                                                       device_counts=device_counts)
    assert e == 0
    o_ref, _, idx = fp8_oracle(x.float().numpy(), logits.float().cpu().numpy(), w1.float().numpy(),
                               w2.float().numpy(), K)
    np.testing.assert_array_equal(freq.cpu().numpy(), np.bincount(idx.reshape(-1), minlength=E))
    assert rel_fro(o_all.float().cpu().numpy(), o_ref.numpy()) <= TOL_FP8


def test_ep_home_config4_shape_256_experts_8_ranks():
    """Config 4's expert-parallel layout: E = 256 experts sharded 32 per rank over 8 emulated ranks,
    H = 7168, I = 2048, top-8, at a reduced token count (64 tokens per rank).  Every owner's up GEMM
    stores its rows into the 8 home buffers, every home runs the down projection over all 256
    experts' w2.  Expert counts exact for all tokens; the full rows of 8 sampled tokens within 1e-2
    of the per-token fake-quantised oracle."""
    from oracle.layer import fp8_oracle_rows
    from oracle.routing import topk_route

    W, T, H, I, E, K = 8, 64, 7168, 2048, 256, 8
    x, w1, w2, o_all, logits, freq, e = _home_emulated(W, T, H, I, E, K, seed=404, inputs=_gpu_layer_inputs)
    assert e == 0
    scores, idx = topk_route(logits.float().cpu().numpy(), K, True, False)
    np.testing.assert_array_equal(freq.cpu().numpy(), np.bincount(idx.reshape(-1), minlength=E))
    rows = np.sort(np.random.RandomState(4).choice(W * T, 8, replace=False))
    o_ref = fp8_oracle_rows(x[torch.from_numpy(rows).cuda()].float().cpu().numpy(), scores[rows], idx[rows],
                            lambda ex: (w1[ex].float().cpu().numpy(), w2[ex].float().cpu().numpy()))
    assert rel_fro(o_all[torch.from_numpy(rows).cuda()].float().cpu().numpy(), o_ref.numpy()) <= TOL_FP8


def test_ep_home_bad_return_row_is_reported():
    """A record whose home row lies past the home buffer: the up epilogue drops those rows and
    writes error 202 instead of storing outside the buffer."""
    *_, e = _home_emulated(2, 64, 256, 128, 8, 4, seed=9, corrupt=True)
    assert e == 202


def test_ep_home_device_count_out_of_range_is_reported():
    """A count in the device-side matrix whose segment runs past the source's send region: the
    owner's table is left empty (no record is read) and error 203 is written."""
    *_, e = _home_emulated(3, 64, 256, 128, 12, 4, seed=10, device_counts=True, bad_count=True)
    assert e == 203


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, W, port, q, T, H, I, E, K, transport, chunks):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "sonic-moe_b200"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    import torch.distributed as dist

    from _util import make_layer_inputs as mk
    from sonicmoe.ep import ExpertParallelMoE

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=W, timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        x, rw, w1, w2 = mk(W * T, H, I, E, seed=77)
        El = E // W
        moe = ExpertParallelMoE(rw.to(dev), w1[rank * El:(rank + 1) * El].to(dev),
                                w2[rank * El:(rank + 1) * El].to(dev), E, K, transport=transport, max_tokens=T,
                                hidden_size=H, chunks=chunks)
        for _ in range(2):  # twice: the shared buffers are reused across forwards
            out, logits, freq = moe.forward(x[rank * T:(rank + 1) * T].to(dev))
        torch.cuda.synchronize()
        q.put((rank, out.float().cpu().numpy(), logits.float().cpu().numpy(), freq.cpu().numpy()))
        moe.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("transport,chunks", [("p2p", 1), ("p2p", 2), ("p2p", 3), ("copy", 1), ("copy", 2),
                                              ("copy", 3), ("copy", 6), ("nccl", 1), ("nccl", 2), ("home", 1),
                                              ("home", 2), ("home", 3)])
def test_ep_multi_gpu(transport, chunks):
    """W processes, one per GPU.  chunks > 1 runs the pipelined forward (dispatch, expert stage and
    combine of different token chunks on different streams); chunks=3 and 6 leave the last chunk
    short (6 is the copy transport's default at 8 ranks)."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    import torch.multiprocessing as mp

    W = 4 if n >= 4 else 2
    T, H, I, E, K = 256, 512, 256, 16, 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, W, port, q, T, H, I, E, K, transport, chunks))
             for r in range(W)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(W):
        r, o, lg, f = q.get(timeout=300)
        res[r] = (o, lg, f)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    x, rw, w1, w2 = make_layer_inputs(W * T, H, I, E, seed=77)
    out = np.concatenate([res[r][0] for r in range(W)])
    logits = np.concatenate([res[r][1] for r in range(W)])
    o_ref, _, idx = fp8_oracle(x.float().numpy(), logits, w1.float().numpy(), w2.float().numpy(), K)
    np.testing.assert_array_equal(np.concatenate([res[r][2] for r in range(W)]), np.bincount(idx.reshape(-1), minlength=E))
    assert rel_fro(out, o_ref.numpy()) <= TOL_FP8


def _world1_worker(port, q, T, H, I, E, K, transport, chunks):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "sonic-moe_b200"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    import torch.distributed as dist

    from _util import make_layer_inputs as mk
    from sonicmoe.ep import ExpertParallelMoE

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        x, rw, w1, w2 = mk(T, H, I, E, seed=91)
        moe = ExpertParallelMoE(rw.to(dev), w1.to(dev), w2.to(dev), E, K, transport=transport, max_tokens=T,
                                hidden_size=H, chunks=chunks)
        for _ in range(2):
            out, logits, freq = moe.forward(x.to(dev))
        moe.check_errors()
        res = [out.float().cpu().numpy(), logits.float().cpu().numpy(), freq.cpu().numpy()]
        if transport == "home":
            # plant an invalid home buffer size: every row past the first 128-row block has no home
            # row, so the up epilogue's bounds check drops it and records error 202 (the down
            # projection then reads only inside the real buffer); the forward must report it
            full = moe._home_rows
            moe._home_rows = 128
            moe.forward(x.to(dev))
            try:
                moe.check_errors()
                res.append("no error")
            except RuntimeError as e:
                res.append(str(e))
            moe._home_rows = full
            moe.forward(x.to(dev))
            moe.check_errors()  # the next forward is clean again
        q.put(("ok", res))
        moe.close()
    except Exception as e:  # report instead of hanging the parent
        q.put(("exception", repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport,chunks", [("home", 1), ("home", 2), ("home", 3), ("p2p", 1), ("p2p", 2),
                                              ("copy", 2), ("nccl", 1)])
def test_ep_world1_transports(transport, chunks):
    """Every transport's host orchestration on a one-rank NCCL group (runs on a one-GPU box):
    output within 1e-2 of the fake-quantised oracle, exact expert counts; for the home transport,
    an up-projection row without a home row makes check_errors() raise with code 202."""
    import torch.multiprocessing as mp

    T, H, I, E, K = 384, 512, 256, 16, 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_world1_worker, args=(_free_port(), q, T, H, I, E, K, transport, chunks))
    p.start()
    status, res = q.get(timeout=300)
    p.join(timeout=120)
    assert status == "ok", res
    assert p.exitcode == 0
    out, logits, freq = res[:3]
    x, rw, w1, w2 = make_layer_inputs(T, H, I, E, seed=91)
    o_ref, _, idx = fp8_oracle(x.float().numpy(), logits, w1.float().numpy(), w2.float().numpy(), K)
    np.testing.assert_array_equal(freq, np.bincount(idx.reshape(-1), minlength=E))
    assert rel_fro(out, o_ref.numpy()) <= TOL_FP8
    if transport == "home":
        assert "device error 202" in res[3], res[3]
