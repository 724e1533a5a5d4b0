"""Expert-parallel host logic on CPU: 2 gloo ranks, device stages replaced by oracle stand-ins.

Checks the orchestration of sonicmoe.ep (count exchange, split sizes, the two all-to-alls and the
combine) against the single-process fake-quantised oracle over all tokens, and that a bad count
injected on one rank makes every rank raise (the validation is agreed collectively, so nobody
waits in a collective the others skipped).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

T_PER_RANK, H, I, E, K, W = 48, 256, 128, 8, 3, 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs():
    g = torch.Generator().manual_seed(5)
    x = torch.randn(W * T_PER_RANK, H, generator=g).to(torch.bfloat16)
    rw = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    return x, rw, w1, w2


def _worker(rank, port, bad_rank, q, err_rank=None, err_code=0):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "sonic-moe_b200"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    from _ep_fakes import FakeStages
    from sonicmoe.ep import ExpertParallelMoE

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=W, timeout=datetime.timedelta(seconds=60))
    try:
        x, rw, w1, w2 = _inputs()
        El = E // W
        moe = ExpertParallelMoE(rw, w1[rank * El:(rank + 1) * El], w2[rank * El:(rank + 1) * El], E, K,
                                stages=FakeStages(bad_count_rank=bad_rank, err_code_rank=err_rank, err_code=err_code))
        xs = x[rank * T_PER_RANK:(rank + 1) * T_PER_RANK].float()
        if err_rank is not None:
            # forward 1 records the error; it surfaces at forward 2's count exchange on every rank,
            # and check_errors() reports it after a single forward
            msgs = []
            moe.forward(xs.to(torch.bfloat16))
            try:
                moe.forward(xs.to(torch.bfloat16))
                msgs.append("no error")
            except RuntimeError as e:
                msgs.append(str(e))
            moe.forward(xs.to(torch.bfloat16))
            try:
                moe.check_errors()
                msgs.append("no error")
            except RuntimeError as e:
                msgs.append(str(e))
            q.put((rank, "errors", msgs, None))
            return
        try:
            out, logits, freq = moe.forward(xs.to(torch.bfloat16))
            # exchange accounting behind the multi-GPU roofline: bytes this rank received from the
            # other rank = its records x record bytes + the partial rows of this rank's records
            ex = moe.last_exchange
            rb = FakeStages().record_bytes(H, K)
            assert ex["bytes_in"] == ex["records_in_remote"] * rb + ex["rows_back_remote"] * H * 2
            assert ex["records_in_remote"] > 0 and ex["rows_back_remote"] > 0
            q.put((rank, "ok", out.float().numpy(), logits.float().numpy()))
        except RuntimeError as e:
            q.put((rank, "error", str(e), None))
    finally:
        dist.destroy_process_group()


def _run(bad_rank, err_rank=None, err_code=0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, bad_rank, q, err_rank, err_code)) for r in range(W)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(W):
        r, status, a, b = q.get(timeout=240)
        res[r] = (status, a, b)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_ep_two_ranks_matches_single_process_oracle():
    from oracle.layer import fp8_oracle, rel_fro

    res = _run(bad_rank=None)
    assert all(res[r][0] == "ok" for r in range(W)), res
    x, rw, w1, w2 = _inputs()
    out = np.concatenate([res[r][1] for r in range(W)])
    logits = np.concatenate([res[r][2] for r in range(W)])
    o_ref, _, _ = fp8_oracle(x.float().numpy(), logits, w1.float().numpy(), w2.float().numpy(), K)
    assert rel_fro(out, o_ref.numpy()) < 5e-3  # bf16 rounding of the per-rank partial rows only


def test_ep_bad_count_aborts_every_rank():
    res = _run(bad_rank=1)
    assert all(res[r][0] == "error" for r in range(W)), res
    assert "negative record count" in res[1][1]
    assert "peer rank" in res[0][1]


def test_ep_device_error_raises_on_every_rank():
    """A device error word set by one rank's expert stage (code 202, made on the host by the
    stand-in) is all-reduced with MAX, so both ranks raise with that code: at the next forward's
    count exchange, or from check_errors() after the last forward."""
    res = _run(bad_rank=None, err_rank=1, err_code=202)
    for r in range(W):
        status, msgs, _ = res[r]
        assert status == "errors", res[r]
        assert all("device error 202" in m for m in msgs), (r, msgs)


def test_check_counts():
    from sonicmoe.ep import check_counts

    assert check_counts([1, 2], [3, 4], 10) == ""
    assert "negative" in check_counts([1, -1], [0, 0], 10)
    assert "exceed" in check_counts([6, 6], [0, 0], 10)


def test_home_transport_arguments():
    """The home transport needs the native stages (its up stage stores into peer memory), and sized
    shared buffers; both are checked before any buffer is allocated."""
    from _ep_fakes import FakeStages
    from sonicmoe.ep import ExpertParallelMoE

    x, rw, w1, w2 = _inputs()
    with pytest.raises(ValueError, match="native stages"):
        ExpertParallelMoE(rw, w1, w2, E, K, stages=FakeStages(), transport="home")
    with pytest.raises(ValueError, match="max_tokens and hidden_size"):
        ExpertParallelMoE(rw, w1, w2, E, K, transport="home", chunks=2)
    with pytest.raises(ValueError, match="unknown transport"):
        ExpertParallelMoE(rw, w1, w2, E, K, stages=FakeStages(), transport="bogus")


def test_default_transport():
    """One process or device-stage stand-ins: NCCL; otherwise the home-down transport (measured best
    at 2, 4 and 8 ranks), pipelined over 4 token chunks from 8 ranks, 2 at 5-7, one up to 4; the copy
    transport keeps 6 chunks from 8 ranks; small batches run in one chunk."""
    from sonicmoe.ep import default_chunks, default_transport

    assert default_transport(1) == "nccl"
    assert default_transport(8, native=False) == "nccl"
    for w in (2, 3, 4, 6, 8, 16):
        assert default_transport(w) == "home" and default_transport(w, chunks=3) == "home"
    assert [default_chunks("home", w, 32768) for w in (2, 3, 4, 6, 8)] == [1, 1, 1, 2, 4]
    assert default_chunks("home", 8, 2048) == 1
    assert default_chunks("copy", 8, 32768) == 6 and default_chunks("copy", 4, 32768) == 1
    assert default_chunks("p2p", 8, 32768) == 1


def test_check_count_matrix_same_verdict_on_every_rank():
    """Every rank validates the whole all-gathered matrix: a bad row of rank 1 fails on both ranks,
    with rank 1's own message there and a peer message on rank 0."""
    from sonicmoe.ep import check_count_matrix

    ok = [[3, 4], [5, 6]]
    assert check_count_matrix(ok, 12, 20, 0) == "" and check_count_matrix(ok, 12, 20, 1) == ""
    bad = [[3, 4], [5, -1]]
    assert "negative record count" in check_count_matrix(bad, 12, 20, 1)
    m0 = check_count_matrix(bad, 12, 20, 0)
    assert "peer rank (1)" in m0 and "negative" in m0
    over = [[3, 9], [5, 9]]  # rank 1 receives 18 records, more than its output region of 12
    assert "exceed the output region" in check_count_matrix(over, 20, 12, 1)
    assert "peer rank (1)" in check_count_matrix(over, 20, 12, 0)


def test_async_error_words_raise_two_forwards_later_on_every_rank():
    """Forwards that never wait on the host queue their reduced error word; forward n checks forward
    n - 2 (a fixed point, identical on every rank, since the words are MAX-reduced), check_errors()
    checks everything left.  Events are stand-ins here (the host logic only)."""
    from sonicmoe.ep import ExpertParallelMoE

    class _Done:
        def synchronize(self):
            pass

    moe = object.__new__(ExpertParallelMoE)
    moe._err_async = []
    words = [0, 0, 202, 0]
    raised_at = None
    for n, code in enumerate(words):
        try:
            moe._poll_async_errors()  # the start of forward n
        except RuntimeError as e:
            raised_at = n
            assert "device error 202" in str(e)
        moe._err_async.append((_Done(), torch.tensor([code], dtype=torch.int32)))  # forward n's word
    assert raised_at is None  # forward 2's word is read at the start of forward 4
    with pytest.raises(RuntimeError, match="device error 202"):
        moe._poll_async_errors()
    assert moe._err_async == []
    moe._err_async.append((_Done(), torch.tensor([0], dtype=torch.int32)))
    moe._err_async.append((_Done(), torch.tensor([203], dtype=torch.int32)))
    moe._poll_async_errors()  # the newest stays queued
    with pytest.raises(RuntimeError, match="device error 203"):
        moe._poll_async_errors(wait=True)
