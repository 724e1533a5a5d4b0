"""Expert-parallel FP8 MoE layer forward: experts sharded over the ranks of a process group.

Four transports move the records and returned rows between the ranks of one node:

* ``"p2p"``: every rank's send buffer and output rows live in CUDA IPC memory
  mapped by all ranks; the receiver's pack kernel and the owner's combine kernel read them with
  peer loads over NVLink, so no separate all-to-all copies the data.  NCCL carries only the
  per-destination counts (an all-gather that also orders the stages) and one tiny all-reduce.
* ``"copy"``: the same shared buffers, but record segments and partial rows cross NVLink as plain
  device-to-device copies (copy engines, no SMs) into local buffers, pipelined over token chunks.
* ``"nccl"``: ``all_to_all_single`` of the records and of the partial rows.
* ``"home"`` (default on GPUs, see ``default_transport`` and ``default_chunks``): the records move
  as in ``"p2p"`` (with chunks, through copy engines), but an expert's owner runs only the up
  projection, whose epilogue stores each entry's e4m3 intermediate row (I + I/128 bytes) straight into the
  padded layout of the token's own rank over NVLink; that rank then runs the down projection with
  the fused top-k combine over its own routing plan, with every expert's w2 replicated on every
  rank (gathered once at construction).  No partial rows and no combine pass: at config 2 with 8
  ranks 0.24 GB instead of 1.2 GB comes back to each rank per forward.

With ``chunks > 1`` every transport pipelines the forward over token chunks on separate streams
(dispatch / transfer / combine of one chunk under the expert GEMMs of its neighbour).

No counterpart in the reference (it is single-GPU; expert parallelism is listed as future work in
its blog).  One process per GPU; rank d of W owns the contiguous global experts
[d*E/W, (d+1)*E/W).  Every rank routes its own tokens with the replicated router and then:

  dispatch   sm_ep_dispatch_prepare: top-k, one e4m3 record per (token, destination rank) -- a token
             routed to several experts of one rank travels once -- rank-major in token order
  exchange   NCCL all-to-all of the per-destination record counts, then of the records
  experts    sm_ep_expert_forward on the received records: local metadata, padding, the up and
             down FP8 GEMMs; each returned row is the token's score-weighted sum over this rank's
             experts (the combine is split: per rank in the down-proj epilogue, then across ranks)
  exchange   NCCL all-to-all of the bf16 partial rows back to the token owners
  combine    sm_ep_combine: fp32 sum of each token's partial rows, rounded once to bf16

The home transport instead runs: router top-k and this rank's routing plan over all E experts,
records carrying each entry's row in that plan, the count all-gather, the up stage (records pulled
from the peers' send buffers, rows stored into the tokens' home intermediates), one all-reduce,
and the down projection with the top-k combine over the rank's own plan.  In one chunk it never
waits on the host: the up stage reads the count matrix in device memory (a bad count becomes
device error 203, raised by a later forward on every rank).

The other transports read the record counts on the host between the two exchanges (one small
device-to-host copy per forward), and every rank checks them before any data moves; a bad count on
any rank makes all ranks raise together (the NCCL transport agrees on the verdict with a collective; the peer-memory
transports all-gather the whole count matrix, so every rank checks every rank's counts and
reaches the same verdict), so no rank is left waiting in a collective the others skipped.
"""
import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _native as nat
from .ops import Fp8ExpertWeights, _need, _ptr, _stream, _workspace, max_padded_blocks, weight_prep


@dataclass
class DispatchState:
    T: int
    K: int
    router_logits: torch.Tensor
    topk_scores: torch.Tensor
    topk_indices: torch.Tensor
    records: torch.Tensor  # [S_max, record_bytes] uint8, first sum(send_counts) rows valid
    ret_row: torch.Tensor  # [T*K] int32
    send_counts: torch.Tensor  # [W] int32 (device)


class _HomeRows:
    """The parts of a routing plan a chunk's record dispatch reads: the chunk's slice of s_rev and the
    plan's per-expert offsets (the home rows of its entries are rows of the whole plan)."""

    def __init__(self, s_rev, off, off_pad):
        self.s_rev, self.off, self.off_pad = s_rev, off, off_pad


class _RawRows:
    """Stand-in for a [rows, width] uint8 tensor at a raw device address (an IPC buffer)."""

    def __init__(self, ptr, rows, width):
        self.ptr, self.shape = ptr, (rows, width)

    def data_ptr(self):
        return self.ptr


class NativeStages:
    """The three device stages through the C ABI (the only implementation in the package)."""

    def __init__(self):
        self.lib = nat.load()

    def record_bytes(self, H, K):
        return self.lib.sm_ep_record_bytes(H, K)

    def dispatch(self, x, logits, E, K, W, rank, sot, norm, err, records=None):
        T, H = x.shape
        rb = self.record_bytes(H, K)
        dev = x.device
        s_max = T * min(K, W)
        if records is None:
            records = torch.empty(max(s_max, 1), rb, dtype=torch.uint8, device=dev)
        ret_row = torch.empty(T * K, dtype=torch.int32, device=dev)
        send_counts = torch.empty(W, dtype=torch.int32, device=dev)
        scores = torch.empty(T, K, dtype=torch.float32, device=dev)
        idx = torch.empty(T, K, dtype=torch.int32, device=dev)
        ws = _workspace(self.lib.sm_ep_dispatch_workspace_bytes(T, E, K, W), dev)
        nat.call(
            "sm_ep_dispatch_prepare", _ptr(x), _ptr(logits), T, H, E, K, W, rank, int(sot), int(norm), _ptr(records),
            _ptr(ret_row), _ptr(send_counts), _ptr(scores), _ptr(idx), _ptr(ws), ws.numel(), _ptr(err), _stream(),
        )
        return DispatchState(T, K, logits, scores, idx, records, ret_row, send_counts)

    def expert(self, records, R, H, I, El, K, w1: Fp8ExpertWeights, w2: Fp8ExpertWeights, err):
        dev = records.device
        out_rows = torch.empty(max(R, 1), H, dtype=torch.bfloat16, device=dev)
        freq = torch.empty(El, dtype=torch.int32, device=dev)
        ws = _workspace(self.lib.sm_ep_expert_workspace_bytes(R, H, I, El, K), dev)
        nat.call(
            "sm_ep_expert_forward", _ptr(records), R, H, I, El, K, _ptr(w1.q), _ptr(w1.sf), _ptr(w2.q), _ptr(w2.sf),
            int(w1.concat_glu), _ptr(out_rows), _ptr(freq), _ptr(ws), ws.numel(), _ptr(err), _stream(),
        )
        return out_rows[:R], freq

    def combine(self, ret, ret_row, T, K, H):
        out = torch.empty(T, H, dtype=torch.bfloat16, device=ret.device)
        nat.call("sm_ep_combine", _ptr(ret), _ptr(ret_row), T, K, H, _ptr(out), _stream())
        return out

    # ---- peer-memory stages ------------------------------------------------------------------
    @staticmethod
    def _ptrs(vals):
        return (ctypes.c_void_p * len(vals))(*vals)

    @staticmethod
    def _ints(vals):
        return (ctypes.c_int32 * len(vals))(*vals)

    def expert_p2p(self, peer_send, seg_off, recv_counts, H, I, El, K, w1, w2, out_ptr, err, device):
        W = len(peer_send)
        R = sum(recv_counts)
        freq = torch.empty(El, dtype=torch.int32, device=device)
        ws = _workspace(self.lib.sm_ep_expert_workspace_bytes(R, H, I, El, K), device)
        nat.call(
            "sm_ep_expert_forward_p2p", self._ptrs(peer_send), self._ints(seg_off), self._ints(recv_counts), W, H, I,
            El, K, _ptr(w1.q), _ptr(w1.sf), _ptr(w2.q), _ptr(w2.sf), int(w1.concat_glu), out_ptr, _ptr(freq),
            _ptr(ws), ws.numel(), _ptr(err), _stream(),
        )
        return freq

    # ---- home-down stages ----------------------------------------------------------------------
    def dispatch_records(self, x, scores, idx, plan, E, W, err, records=None):
        """Records from an already computed top-k; with `plan` (this rank's RoutePlan over all E
        experts) every record carries its entries' rows in this rank's padded layout."""
        T, H = x.shape
        K = idx.shape[1]
        rb = self.record_bytes(H, K)
        dev = x.device
        if records is None:
            records = torch.empty(max(T * min(K, W), 1), rb, dtype=torch.uint8, device=dev)
        ret_row = torch.empty(T * K, dtype=torch.int32, device=dev)
        send_counts = torch.empty(W, dtype=torch.int32, device=dev)
        ws = _workspace(self.lib.sm_ep_dispatch_workspace_bytes(T, E, K, W), dev)
        nat.call(
            "sm_ep_dispatch_records", _ptr(x), T, H, E, K, W, _ptr(scores), _ptr(idx),
            _ptr(plan.s_rev if plan else None), _ptr(plan.off if plan else None),
            _ptr(plan.off_pad if plan else None), _ptr(records), _ptr(ret_row), _ptr(send_counts), _ptr(ws),
            ws.numel(), _ptr(err), _stream(),
        )
        return DispatchState(T, K, None, scores, idx, records, ret_row, send_counts)

    def expert_up_p2p(self, peer_send, seg_off, recv_counts, H, I, El, K, w1, home_q, home_sf, home_rows, err,
                      device):
        """Up projection of the received records; each row is stored into its source rank's
        intermediate home_q[s] / home_sf[s] (peer pointers).  Returns the local expert counts."""
        W = len(peer_send)
        R = sum(recv_counts)
        freq = torch.empty(El, dtype=torch.int32, device=device)
        ws = _workspace(self.lib.sm_ep_expert_workspace_bytes(R, H, I, El, K), device)
        nat.call(
            "sm_ep_expert_up_p2p", self._ptrs(peer_send), self._ints(seg_off), self._ints(recv_counts), W, H, I, El,
            K, _ptr(w1.q), _ptr(w1.sf), int(w1.concat_glu), self._ptrs(home_q), self._ptrs(home_sf), int(home_rows),
            _ptr(freq), _ptr(ws), ws.numel(), _ptr(err), _stream(),
        )
        return freq

    def expert_up_home(self, peer_send, counts, stride, me, send_cap, recv_cap, H, I, El, K, w1, home_q, home_sf,
                       home_rows, err, device):
        """expert_up_p2p with the all-gathered count matrix left on the device (counts: int32 device
        tensor, counts[s * stride + d] = records of source s for destination d): every grid is sized for
        recv_cap records and the kernels read the segment table, so the host never waits."""
        W = len(peer_send)
        freq = torch.empty(El, dtype=torch.int32, device=device)
        ws = _workspace(self.lib.sm_ep_expert_workspace_bytes(recv_cap, H, I, El, K), device)
        nat.call(
            "sm_ep_expert_up_home", self._ptrs(peer_send), _ptr(counts), stride, me, W, send_cap, recv_cap, H, I, El,
            K, _ptr(w1.q), _ptr(w1.sf), int(w1.concat_glu), self._ptrs(home_q), self._ptrs(home_sf), int(home_rows),
            _ptr(freq), _ptr(ws), ws.numel(), _ptr(err), _stream(),
        )
        return freq

    def combine_p2p(self, peer_out, send_counts, recv_start, ret_row, T, K, H, device, out=None):
        if out is None:
            out = torch.empty(T, H, dtype=torch.bfloat16, device=device)
        nat.call(
            "sm_ep_combine_p2p", self._ptrs(peer_out), self._ints(send_counts), self._ints(recv_start),
            len(peer_out), _ptr(ret_row), T, K, H, _ptr(out), _stream(),
        )
        return out


class IpcBuffer:
    """A device buffer allocated by this rank and mapped into every rank of `group` (CUDA IPC)."""

    def __init__(self, nbytes: int, group=None):
        self.lib = nat.load()
        self.nbytes = int(nbytes)
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        nat.call("sm_ipc_alloc", self.nbytes, ctypes.byref(ptr), handle)
        self.ptr = ptr.value
        handles = [None] * dist.get_world_size(group)
        dist.all_gather_object(handles, bytes(handle), group=group)
        me = dist.get_rank(group)
        self.peers = []
        for r, h in enumerate(handles):
            if r == me:
                self.peers.append(self.ptr)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            nat.call("sm_ipc_open", hb, ctypes.byref(p))
            self.peers.append(p.value)
        self._me = me

    def unmap(self):
        """Drop this process's mappings of the peers' buffers."""
        if self.peers is None:
            return
        for r, p in enumerate(self.peers):
            if r != self._me:
                self.lib.sm_ipc_close(p)
        self.peers = None

    def free(self):
        """Free this rank's own buffer (after every peer has unmapped it)."""
        if self.ptr is not None:
            self.lib.sm_ipc_free(self.ptr)
            self.ptr = None


def check_counts(send_counts, recv_counts, capacity: int) -> str:
    """Host-side validation of one rank's exchange sizes; returns an error message or ''."""
    if any(c < 0 for c in send_counts) or any(c < 0 for c in recv_counts):
        return f"negative record count (send {send_counts}, recv {recv_counts})"
    if sum(send_counts) > capacity:
        return f"send counts {send_counts} exceed the dispatch buffer ({capacity} records)"
    return ""


def check_count_matrix(C, send_cap: int, out_cap: int, me: int) -> str:
    """Validation of a whole all-gathered count matrix C[s][d] (records from s to d), identical on
    every rank that holds the same C: the first failing rank's message (prefixed with the rank
    when it is not `me`), or ''.  Every rank therefore raises together without a second
    collective to agree on the verdict."""
    W = len(C)
    for r in range(W):
        recv = [C[s][r] for s in range(W)]
        msg = check_counts(C[r], recv, send_cap)
        if not msg and sum(recv) > out_cap:
            msg = f"{sum(recv)} received records exceed the output region ({out_cap})"
        if msg:
            return msg if r == me else f"a peer rank ({r}) failed its check: {msg}"
    return ""


def default_transport(world: int, native: bool = True, chunks: int = None) -> str:
    """Transport chosen when the caller names none, from the measurements at config 2 per rank.

    The home-down transport at every measured size: 2 ranks 4.08-4.13 ms per forward against 4.33
    for peer loads with the down projection at the owners; 4 ranks 5.11 against 6.24 ms; 8 ranks,
    pipelined over 4 token chunks, 6.28 ms against 6.87 for copy-engine transfers over 6 chunks (the
    bytes back per rank are 6x smaller for e4m3 intermediate rows than for bf16 partial rows).  5-7
    ranks are not measured; home wins at both neighbours.  Device-stage stand-ins (tests) take NCCL.
    """
    del chunks  # every chunk count is served by the home transport
    if not native or world <= 1:
        return "nccl"
    return "home"


def default_chunks(transport: str, world: int, max_tokens: int) -> int:
    """Token chunks the forward is pipelined over when the caller names none: the home transport
    at 8 and more ranks, 4 chunks (6.28 ms at config 2 against 6.92 with 2 and 8.34 with 1: the
    records of later chunks land through copy engines under the up projection of earlier ones);
    up to 4 ranks one, which also reads the exchange counts on the device and never waits on the
    host (4 ranks, per-step device times in one call: 4.93 ms against 5.23 with 2 chunks at config
    2, 4.05 against 4.62 at config 4); 5-7 ranks, not measured, 2; the copy transport 6 from 8
    ranks.  Batches under 4096 tokens per rank: one."""
    if max_tokens < 4096:
        return 1
    if transport == "home":
        return 4 if world >= 8 else (2 if world > 4 else 1)
    if transport == "copy" and world >= 8:
        return 6
    return 1


class ExpertParallelMoE:
    """FP8 SwiGLU MoE layer whose experts are sharded over `group` (torch.distributed, NCCL).

    router_w [E, H] is replicated; w1_local [E/W, 2I, H] / w2_local [E/W, H, I] are this rank's
    experts (bf16, quantised here, or prepared Fp8ExpertWeights).  forward(x) takes this rank's
    tokens [T, H] and returns (out [T, H], router_logits [T, E], local expert_frequency [E/W]).
    """

    def __init__(self, router_w, w1_local, w2_local, num_experts: int, top_k: int, group=None,
                 softmax_over_topk: bool = True, norm_topk_probs: bool = False, concat_layout: bool = False,
                 stages=None, reserve_sms: int = None, transport: str = None, max_tokens: int = None,
                 hidden_size: int = None, chunks: int = None, record_phases: bool = False):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError(f"num_experts={num_experts} is not divisible by the group size {self.world}")
        self.E = num_experts
        self.El = num_experts // self.world
        self.K = top_k
        self.sot = softmax_over_topk
        self.norm = norm_topk_probs
        if norm_topk_probs and softmax_over_topk:
            raise ValueError("`norm_topk_prob` only works with softmax-then-topk")
        self.stages = stages if stages is not None else NativeStages()
        if transport is None:
            transport = default_transport(self.world, native=stages is None, chunks=chunks)
        if transport not in ("p2p", "copy", "nccl", "home"):
            raise ValueError(f"unknown transport {transport!r}")
        if transport == "home" and stages is not None:
            raise ValueError("the home transport runs the native stages only")
        self.transport = transport
        if chunks is None:
            chunks = default_chunks(transport, self.world, max_tokens or 0)
        if chunks < 1:
            raise ValueError("chunks must be >= 1")
        self.chunks = int(chunks)
        if stages is None:
            # SMs the persistent GEMMs leave free for the dispatch / combine kernels and NCCL that run
            # alongside them when the forward is pipelined over chunks
            if reserve_sms is None:
                reserve_sms = 0
            nat.call("sm_set_gemm_sm_reserve", reserve_sms)
        self._send_buf = self._out_buf = None
        self.last_exchange = None
        # home transport: CUDA events at the phase boundaries of every forward (read with phase_times())
        self.record_phases = bool(record_phases)
        self._phase_events = None
        self._streams = None
        self._copy_streams = None
        self._home_buf = None
        # device error word of the last forward (already reduced over the ranks with MAX), read at
        # the next forward's count exchange -- where the host waits for this stream anyway -- or
        # by check_errors(); the one-chunk home transport, which never waits, uses _err_async
        self._err_pending = None
        # (event, pinned error word) of forwards that never wait on the host, oldest first
        self._err_async = []
        if transport in ("p2p", "copy", "home"):
            if max_tokens is None or hidden_size is None:
                raise ValueError("the p2p transport needs max_tokens and hidden_size to size its shared buffers")
            self.max_tokens = int(max_tokens)
            rb = self.stages.record_bytes(hidden_size, top_k)
            # one region per chunk in each shared buffer: chunk c of every rank lives at the same offset
            self._chunk_tokens = -(-self.max_tokens // self.chunks)
            self._send_cap = self._chunk_tokens * min(top_k, self.world)  # records per chunk region
            self._out_cap = self.world * self._chunk_tokens  # partial rows per chunk region
            self._send_chunk_bytes = max(self._send_cap, 1) * rb
            self._out_chunk_bytes = max(self._out_cap, 1) * hidden_size * 2
            self._send_buf = IpcBuffer(self.chunks * self._send_chunk_bytes, group)
            if transport != "home":
                self._out_buf = IpcBuffer(self.chunks * self._out_chunk_bytes, group)
            if transport == "copy" or (transport == "home" and self.chunks > 1):
                # local landing buffers: the records of every source (and, copy transport, the partial
                # rows of every owner)
                dev = torch.device("cuda", torch.cuda.current_device())
                self._recv_local = torch.empty(self.chunks, max(self._out_cap, 1), rb, dtype=torch.uint8, device=dev)
            if transport == "copy":
                self._ret_local = torch.empty(self.chunks, max(self._send_cap, 1), hidden_size, dtype=torch.bfloat16,
                                              device=dev)
        self.router_w = router_w
        prep = (lambda w, c: w) if stages is not None else (lambda w, c: w if isinstance(w, Fp8ExpertWeights)
                                                            else weight_prep(w, concat_glu=c))
        self.w1 = prep(w1_local, concat_layout)
        self.w2 = prep(w2_local, False)
        shp = tuple(self.w1.shape)
        if shp[0] != self.El:
            raise ValueError(f"w1_local holds {shp[0]} experts, expected {self.El}")
        self.I = shp[1] // 2
        if transport == "home":
            self._setup_home(hidden_size)

    def _setup_home(self, H):
        """Replicate w2 over the group and map every rank's intermediate buffer: rows of the
        padded layout of up to max_tokens * K entries over all E experts, e4m3 + scale atoms."""
        I, W = self.I, self.world
        if tuple(self.w2.shape) != (self.El, H, I):
            raise ValueError(f"w2_local has shape {tuple(self.w2.shape)}, expected {(self.El, H, I)}")
        if W > 1:
            q = torch.empty((W * self.El,) + tuple(self.w2.q.shape[1:]), dtype=torch.uint8, device=self.w2.q.device)
            sf = torch.empty((W * self.El,) + tuple(self.w2.sf.shape[1:]), dtype=torch.uint8, device=self.w2.sf.device)
            dist.all_gather_into_tensor(q, self.w2.q.contiguous(), group=self.group)
            dist.all_gather_into_tensor(sf, self.w2.sf.contiguous(), group=self.group)
            self.w2_full = Fp8ExpertWeights(q, sf, False)
        else:
            self.w2_full = self.w2
        self._home_rows = max_padded_blocks(self.max_tokens * self.K, self.E) * 128
        self._home_q_bytes = -(-self._home_rows * I // 256) * 256
        self._home_sf_shape = (self._home_rows // 128, -(-I // 512), 512)
        sf_bytes = self._home_sf_shape[0] * self._home_sf_shape[1] * 512
        self._home_buf = IpcBuffer(self._home_q_bytes + max(sf_bytes, 16), self.group)

    # ---- device error word ----------------------------------------------------------------------
    def _raise_pending(self):
        """Raise if the previous forward's kernels recorded an error on any rank.  The word was
        all-reduced with MAX, so every rank reads the same value and raises at the same point."""
        self._poll_async_errors()
        pending, self._err_pending = self._err_pending, None
        if pending is None:
            return
        code = int(pending.max().item())
        if code:
            raise RuntimeError(f"expert-parallel forward failed: device error {code} "
                               f"({nat.ERR_NAMES.get(code, 'unknown code')}); its output is not valid")

    def phase_times(self):
        """Device milliseconds of the last home-transport forward's phases (with record_phases=True):
        route + dispatch records, count exchange (the all-gather), up stage (record pull + up GEMM
        storing into the homes), error all-reduce (the cross-rank barrier), down +
        combine.  Waits for the forward."""
        ev = self._phase_events
        if ev is None:
            return None
        ev[-1].synchronize()
        names = ("dispatch", "count_exchange", "up_stage", "allreduce", "down")
        return {n: ev[i].elapsed_time(ev[i + 1]) for i, n in enumerate(names)}

    def _push_async_error(self, errs, stream):
        """Forwards without a host wait (home transport, one chunk): the reduced error word is copied
        into pinned host memory on `stream` and read by a later forward (_poll_async_errors), so the
        host does not wait for the device within a forward."""
        host = torch.empty(errs.shape, dtype=errs.dtype, pin_memory=True)
        host.copy_(errs, non_blocking=True)
        done = torch.cuda.Event()
        done.record(stream)
        self._err_async.append((done, host))

    def _poll_async_errors(self, wait: bool = False):
        """Raise for a queued forward whose error word is non-zero.  A forward is checked when the one
        after it has been queued too (the device is then still busy with that one, so the host rarely
        waits), or at once with wait.  The queue has the same length on every rank at the same call, so
        every rank raises in the same forward and no rank is left alone in a collective."""
        keep = 0 if wait else 1
        while len(self._err_async) > keep:
            done, host = self._err_async.pop(0)
            done.synchronize()
            code = int(host.max())
            if code:
                self._err_async.clear()
                raise RuntimeError(f"expert-parallel forward failed: device error {code} "
                                   f"({nat.ERR_NAMES.get(code, 'unknown code')}); its output is not valid")

    def check_errors(self):
        """Wait for the last forward and raise if any rank's kernels recorded an error.  Every
        forward also checks earlier ones, so only the last forward of a run needs this call."""
        if self._err_pending is not None and self._err_pending.is_cuda:
            torch.cuda.synchronize(self._err_pending.device)
        self._raise_pending()
        self._poll_async_errors(wait=True)

    def _reduce_err(self, err):
        if self.world > 1:
            dist.all_reduce(err, op=dist.ReduceOp.MAX, group=self.group)

    # ---- collectives -------------------------------------------------------------------------
    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        if self.world == 1:
            out.copy_(inp)
            return
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=self.group)

    def _agree(self, ok: bool, device):
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
        if self.world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        return bool(flag.item())

    def close(self):
        """Unmap and free the shared buffers (collective: call on every rank)."""
        if self._send_buf is not None:
            bufs = [b for b in (self._send_buf, self._out_buf, self._home_buf) if b is not None]
            torch.cuda.synchronize()
            dist.barrier(group=self.group)  # nobody reads or writes a peer buffer any more
            for b in bufs:
                b.unmap()
            torch.cuda.synchronize()
            dist.barrier(group=self.group)  # every peer mapping is gone
            for b in bufs:
                b.free()
            self._send_buf = self._out_buf = self._home_buf = None

    def _note_exchange(self, records_in_remote: int, records_out_remote: int, H: int, rb: int):
        """Bytes this rank received over NVLink in the last forward: records from other ranks, and
        the partial rows other ranks computed for this rank's records (roofline of the exchange)."""
        self.last_exchange = {"records_in_remote": records_in_remote, "rows_back_remote": records_out_remote,
                              "bytes_in": records_in_remote * rb + records_out_remote * H * 2}

    def _note_exchange_home(self, records_in_remote: int, entries_back_remote, rb: int):
        """Home transport: records from other ranks plus the e4m3 intermediate rows (I bytes + I/128
        scale bytes) other ranks computed for this rank's entries; the count of those entries stays
        a device tensor until read."""
        row = self.I + self.I // 128
        self.last_exchange = {"records_in_remote": records_in_remote, "entries_back_remote": entries_back_remote,
                              "bytes_in": entries_back_remote.double() * row + records_in_remote * rb}

    def _exchange_counts(self, st, stream, device):
        """Collective on `stream`: every rank's per-destination record counts of one chunk (and, since
        a rank's all-gather runs after its dispatch, the guarantee that every send region of the
        chunk is complete), validated on every rank over the whole matrix, so that all ranks reach
        the same verdict with no further collective.  Returns (C[s][d], ready event)."""
        W = self.world
        with torch.cuda.stream(stream):
            allc = torch.empty(W * W, dtype=torch.int32, device=device)
            dist.all_gather_into_tensor(allc, st.send_counts, group=self.group)
            C = allc.view(W, W).cpu().tolist()  # C[s][d]: records of this chunk from s to d
            self._raise_pending()  # the previous forward ran on this stream and has finished
            msg = check_count_matrix(C, self._send_cap, self._out_cap, self.rank)
            ev = torch.cuda.Event()
            ev.record(stream)
        if msg:
            raise RuntimeError(f"expert-parallel exchange aborted on every rank: {msg}")
        return C, ev

    def _forward_p2p(self, x: torch.Tensor):
        """Peer-memory forward, pipelined over `self.chunks` token chunks on three streams:

          main (high priority)  router, then per chunk: expert stage (records pulled from the peers'
                                send regions, FP8 GEMMs, partial rows into this rank's output region),
                                then an all-reduce that orders every rank's rows before any combine
          dispatch              chunks 1.. : top-k + records, then their count exchange
          combine               per chunk, after its all-reduce: each token pulls its partial rows

        so the dispatch of chunk c+1 and the combine of chunk c-1 run while chunk c's GEMMs hold the
        SMs they do not reserve.  Every rank issues the same collectives in the same order.
        """
        T, H = x.shape
        W, K, me, Cn = self.world, self.K, self.rank, self.chunks
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of the shared buffers")
        dev = x.device
        caller = torch.cuda.current_stream(dev)
        if self._streams is None:
            self._streams = (torch.cuda.Stream(dev, priority=-1), torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        s_main, s_disp, s_comb = self._streams
        s_main.wait_stream(caller)
        rb = self.stages.record_bytes(H, K)
        Tc = -(-T // Cn) if T else 0
        spans = [(min(T, c * Tc), min(T, (c + 1) * Tc)) for c in range(Cn)]
        with torch.cuda.stream(s_main):
            logits = F.linear(x, self.router_w.to(x.dtype))
            out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
            errs = torch.zeros(Cn, dtype=torch.int32, device=dev)
            freq = torch.zeros(self.El, dtype=torch.int32, device=dev)
            ev_logits = torch.cuda.Event()
            ev_logits.record(s_main)
        states = []
        for c, (a, b) in enumerate(spans):
            s = s_main if c == 0 else s_disp
            with torch.cuda.stream(s):
                s.wait_event(ev_logits)
                records = _RawRows(self._send_buf.ptr + c * self._send_chunk_bytes, self._send_cap, rb)
                states.append(self.stages.dispatch(x[a:b], logits[a:b], self.E, K, W, me, self.sot, self.norm,
                                                   errs[c:c + 1], records=records))
        counts = [None] * Cn
        counts[0] = self._exchange_counts(states[0], s_main, dev)
        for c in range(Cn):
            C, ev = counts[c]
            a, b = spans[c]
            with torch.cuda.stream(s_main):
                s_main.wait_event(ev)
                recv_counts = [C[s_][me] for s_ in range(W)]
                seg_off = [sum(C[s_][:me]) for s_ in range(W)]
                f = self.stages.expert_p2p([p + c * self._send_chunk_bytes for p in self._send_buf.peers], seg_off,
                                           recv_counts, H, self.I, self.El, K, self.w1, self.w2,
                                           self._out_buf.ptr + c * self._out_chunk_bytes, errs[c:c + 1], dev)
                freq += f
            if c + 1 < Cn:  # the host waits for chunk c+1's dispatch while chunk c computes
                counts[c + 1] = self._exchange_counts(states[c + 1], s_disp, dev)
            with torch.cuda.stream(s_main):
                # every rank's chunk-c rows are complete; MAX keeps one rank's code intact
                dist.all_reduce(errs[c:c + 1], op=dist.ReduceOp.MAX, group=self.group)
                ev_rows = torch.cuda.Event()
                ev_rows.record(s_main)
            with torch.cuda.stream(s_comb):
                s_comb.wait_event(ev_rows)
                states[c].ret_row.record_stream(s_comb)
                recv_start = [sum(C[q][d] for q in range(me)) for d in range(W)]
                self.stages.combine_p2p([p + c * self._out_chunk_bytes for p in self._out_buf.peers], C[me],
                                        recv_start, states[c].ret_row, b - a, K, H, dev, out=out[a:b])
        ev_done = torch.cuda.Event()
        ev_done.record(s_comb)
        caller.wait_event(ev_done)
        caller.wait_stream(s_main)
        for t in (logits, out, freq):
            t.record_stream(caller)
        self._err_pending = errs
        self._note_exchange(sum(C_[q][me] for C_, _ in counts for q in range(W) if q != me),
                            sum(C_[me][d] for C_, _ in counts for d in range(W) if d != me), H, rb)
        return out, logits, freq

    def _forward_home(self, x: torch.Tensor):
        """Home-down forward, all on one high-priority stream:

          router, top-k, this rank's routing plan over all E experts, records carrying each
          entry's row in that plan's padded layout
          count exchange (all-gather; also: every rank's records are complete, and every rank has
                          finished the down projection that read its intermediate last forward);
                          the matrix stays in device memory
          up stage       segment table resolved on the device from that matrix, records pulled from
                          the peers' send buffers, up GEMM whose epilogue stores each row into its
                          token's home intermediate (peer stores); grids sized for the most records
                          a rank can receive
          all-reduce     of the error word: every rank's rows have landed in every home
          down stage     down GEMM + top-k combine over this rank's own plan, replicated w2

        The host never waits for the device: the error word reaches pinned memory asynchronously and
        a later forward (or check_errors()) raises for it.
        """
        from . import ops

        self._poll_async_errors()

        T, H = x.shape
        W, K, me = self.world, self.K, self.rank
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of the shared buffers")
        dev = x.device
        caller = torch.cuda.current_stream(dev)
        if self._streams is None:
            self._streams = (torch.cuda.Stream(dev, priority=-1), torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        s_main = self._streams[0]
        s_main.wait_stream(caller)
        rb = self.stages.record_bytes(H, K)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)] if self.record_phases else None

        def mark(i):
            if ev is not None:
                ev[i].record(s_main)

        with torch.cuda.stream(s_main):
            mark(0)
            logits = F.linear(x, self.router_w.to(x.dtype))
            errs = torch.zeros(1, dtype=torch.int32, device=dev)
            scores, idx = ops.router_topk(logits, K, self.sot, self.norm)
            plan = ops.route_plan(idx, self.E, errs)
            records = _RawRows(self._send_buf.ptr, self._send_cap, rb)
            st = self.stages.dispatch_records(x, scores, idx, plan, self.E, W, errs, records=records)
            mark(1)
            # the count matrix stays on the device: the up stage's kernels read it (no host round trip)
            allc = torch.empty(W * W, dtype=torch.int32, device=dev)
            if W > 1:
                dist.all_gather_into_tensor(allc, st.send_counts, group=self.group)
            else:
                allc.copy_(st.send_counts)
            mark(2)
            home_q = list(self._home_buf.peers)
            home_sf = [p + self._home_q_bytes for p in home_q]
            freq = self.stages.expert_up_home(self._send_buf.peers, allc, W, me, self._send_cap, self._out_cap, H,
                                              self.I, self.El, K, self.w1, home_q, home_sf, self._home_rows, errs,
                                              dev)
            mark(3)
            # every rank's rows have landed in every home; MAX keeps one rank's code intact
            self._reduce_err(errs)
            mark(4)
            out = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
            aq = _RawRows(self._home_buf.ptr, self._home_rows, self.I)
            asf = _RawRows(self._home_buf.ptr + self._home_q_bytes, self._home_sf_shape[0], 1024)
            ops.moe_down_combine(aq, asf, self.w2_full, plan, scores.view(-1), T, errs, out=out)
            mark(5)
            remote = (idx // self.El != me).sum()
            cm = allc.view(W, W)
            records_in_remote = cm[:, me].sum() - cm[me, me]
            self._push_async_error(errs, s_main)
        self._phase_events = ev
        caller.wait_stream(s_main)
        for t in (logits, out, freq, remote, records_in_remote):
            t.record_stream(caller)
        self._note_exchange_home(records_in_remote, remote, rb)
        return out, logits, freq

    def _land_records(self, A, W, me, Cn, rb, ev_counts):
        """Copy-engine transfers of every chunk's record segments from the peers' send regions into
        this rank's landing buffer (one copy per (chunk, peer), on that peer's copy stream, all issued
        after the count exchange).  Returns per chunk: the events to wait for, the record source
        bases (own segment read in place) and their segment offsets."""
        lib_copy = lambda dst, src, nbytes, stream: nat.call("sm_copy_d2d_async", dst, src, nbytes,  # noqa: E731
                                                             stream.cuda_stream)
        in_events, bases, seg_offs = [], [], []
        for c in range(Cn):
            evs, base, seg, landed = [], [], [], 0
            for q in range(W):
                n = A[q][c][me]
                if q == me:  # this rank's own segment is read in place
                    base.append(self._send_buf.ptr + c * self._send_chunk_bytes)
                    seg.append(sum(A[me][c][:me]))
                    continue
                dst = self._recv_local[c].data_ptr() + landed * rb
                base.append(dst)
                seg.append(0)
                if n > 0:
                    cs = self._copy_streams[q]
                    cs.wait_event(ev_counts)
                    src = self._send_buf.peers[q] + c * self._send_chunk_bytes + sum(A[q][c][:me]) * rb
                    lib_copy(dst, src, n * rb, cs)
                    ev = torch.cuda.Event()
                    ev.record(cs)
                    evs.append(ev)
                landed += n
            in_events.append(evs)
            bases.append(base)
            seg_offs.append(seg)
        return in_events, bases, seg_offs

    def _forward_home_chunked(self, x: torch.Tensor):
        """Home-down forward over token chunks: one routing plan of all this rank's tokens (so every
        record's home row is global), records dispatched per chunk into the chunk's send region,
        one count exchange for all chunks, then the records of every chunk land through copy
        engines while the main stream runs the owner's up projection of the chunks already landed
        (rows stored into their homes).  After all chunks: the error all-reduce (every rank's rows are
        home) and one down projection + combine over this rank's plan."""
        from . import ops

        T, H = x.shape
        W, K, me, Cn = self.world, self.K, self.rank, self.chunks
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of the shared buffers")
        dev = x.device
        caller = torch.cuda.current_stream(dev)
        if self._streams is None:
            self._streams = (torch.cuda.Stream(dev, priority=-1), torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        if self._copy_streams is None:
            self._copy_streams = [torch.cuda.Stream(dev) for _ in range(W)]
        s_main = self._streams[0]
        s_main.wait_stream(caller)
        rb = self.stages.record_bytes(H, K)
        Tc = -(-T // Cn) if T else 0
        spans = [(min(T, c * Tc), min(T, (c + 1) * Tc)) for c in range(Cn)]
        with torch.cuda.stream(s_main):
            logits = F.linear(x, self.router_w.to(x.dtype))
            errs = torch.zeros(1, dtype=torch.int32, device=dev)
            scores, idx = ops.router_topk(logits, K, self.sot, self.norm)
            plan = ops.route_plan(idx, self.E, errs)
            states = []
            for c, (a, b) in enumerate(spans):
                records = _RawRows(self._send_buf.ptr + c * self._send_chunk_bytes, self._send_cap, rb)
                # the chunk's entries are entries [a K, b K) of the plan: its s_rev rows from there
                plan_c = _HomeRows(plan.s_rev[a * K:b * K], plan.off, plan.off_pad)
                states.append(self.stages.dispatch_records(x[a:b], scores[a:b], idx[a:b], plan_c, self.E, W, errs,
                                                           records=records))
            mine = torch.stack([st.send_counts for st in states]).contiguous()  # [Cn, W]
            allc = torch.empty(W * Cn * W, dtype=torch.int32, device=dev)
            dist.all_gather_into_tensor(allc, mine.view(-1), group=self.group)
            A = allc.view(W, Cn, W).cpu().tolist()  # A[s][c][d]: records of chunk c from s to d
            self._raise_pending()  # the previous forward ran on this stream and has finished
            msg = ""
            for c in range(Cn):  # the whole matrix on every rank: the same verdict everywhere
                msg = msg or check_count_matrix([[A[q][c][d] for d in range(W)] for q in range(W)],
                                                self._send_cap, self._out_cap, me)
            ev_counts = torch.cuda.Event()
            ev_counts.record(s_main)
        if msg:
            raise RuntimeError(f"expert-parallel exchange aborted on every rank: {msg}")
        in_events, bases, seg_offs = self._land_records(A, W, me, Cn, rb, ev_counts)
        home_q = list(self._home_buf.peers)
        home_sf = [p + self._home_q_bytes for p in home_q]
        with torch.cuda.stream(s_main):
            freq = torch.zeros(self.El, dtype=torch.int32, device=dev)
            for c in range(Cn):
                for ev in in_events[c]:
                    s_main.wait_event(ev)
                recv_counts = [A[q][c][me] for q in range(W)]
                freq += self.stages.expert_up_p2p(bases[c], seg_offs[c], recv_counts, H, self.I, self.El, K, self.w1,
                                                  home_q, home_sf, self._home_rows, errs, dev)
            # every rank's rows have landed in every home; MAX keeps one rank's code intact
            self._reduce_err(errs)
            out = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
            aq = _RawRows(self._home_buf.ptr, self._home_rows, self.I)
            asf = _RawRows(self._home_buf.ptr + self._home_q_bytes, self._home_sf_shape[0], 1024)
            ops.moe_down_combine(aq, asf, self.w2_full, plan, scores.view(-1), T, errs, out=out)
            remote = (idx // self.El != me).sum()
        caller.wait_stream(s_main)
        for t in (logits, out, freq, remote):
            t.record_stream(caller)
        for st in states:
            st.ret_row.record_stream(caller)
        self._err_pending = errs
        self._note_exchange_home(sum(A[q][c][me] for c in range(Cn) for q in range(W) if q != me), remote, rb)
        return out, logits, freq

    def _forward_copy(self, x: torch.Tensor):
        """Copy-engine forward: the peer buffers of the p2p transport, but the record segments and
        the returned partial rows cross NVLink as plain device-to-device copies (one per peer
        segment, on one stream per peer) into local buffers, so the transfers occupy no SMs and run
        under the expert GEMMs of the neighbouring chunks:

          main (high priority)  router, dispatch of every chunk, one exchange of all chunks' counts,
                                then per chunk: expert stage on the landed records, all-reduce
          copy stream per peer  all chunks' record segments from that peer (right after the
                                counts), then, per chunk after its all-reduce, the partial rows that
                                peer computed for this rank's records
          combine               per chunk: the fp32 sum of each token's partial rows (local reads)
        """
        T, H = x.shape
        W, K, me, Cn = self.world, self.K, self.rank, self.chunks
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of the shared buffers")
        dev = x.device
        lib = nat.load()
        caller = torch.cuda.current_stream(dev)
        if self._streams is None:
            self._streams = (torch.cuda.Stream(dev, priority=-1), torch.cuda.Stream(dev), torch.cuda.Stream(dev))
            self._copy_streams = [torch.cuda.Stream(dev) for _ in range(W)]
        s_main, _, s_comb = self._streams
        rb = self.stages.record_bytes(H, K)
        Tc = -(-T // Cn) if T else 0
        spans = [(min(T, c * Tc), min(T, (c + 1) * Tc)) for c in range(Cn)]
        s_main.wait_stream(caller)
        with torch.cuda.stream(s_main):
            logits = F.linear(x, self.router_w.to(x.dtype))
            out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
            errs = torch.zeros(Cn, dtype=torch.int32, device=dev)
            freq = torch.zeros(self.El, dtype=torch.int32, device=dev)
            states = []
            for c, (a, b) in enumerate(spans):
                records = _RawRows(self._send_buf.ptr + c * self._send_chunk_bytes, self._send_cap, rb)
                states.append(self.stages.dispatch(x[a:b], logits[a:b], self.E, K, W, me, self.sot, self.norm,
                                                   errs[c:c + 1], records=records))
            # counts of every chunk, every rank (the all-gather also orders every rank's dispatch
            # before any copy out of its send regions)
            mine = torch.stack([st.send_counts for st in states]).contiguous()  # [Cn, W]
            allc = torch.empty(W * Cn * W, dtype=torch.int32, device=dev)
            dist.all_gather_into_tensor(allc, mine.view(-1), group=self.group)
            A = allc.view(W, Cn, W).cpu().tolist()  # A[s][c][d]: records of chunk c from s to d
            self._raise_pending()  # the previous forward ran on this stream and has finished
            msg = ""
            for c in range(Cn):  # the whole matrix on every rank: the same verdict everywhere
                msg = msg or check_count_matrix([[A[q][c][d] for d in range(W)] for q in range(W)],
                                                self._send_cap, self._out_cap, me)
            ev_counts = torch.cuda.Event()
            ev_counts.record(s_main)
        if msg:
            raise RuntimeError(f"expert-parallel exchange aborted on every rank: {msg}")

        def copy(dst, src, nbytes, stream):
            nat.call("sm_copy_d2d_async", dst, src, nbytes, stream.cuda_stream)

        # records in: every chunk, every remote source, enqueued now
        in_events, bases, seg_offs = [], [], []
        for c in range(Cn):
            evs, base, seg, landed = [], [], [], 0
            for q in range(W):
                n = A[q][c][me]
                if q == me:  # this rank's own segment is read in place
                    base.append(self._send_buf.ptr + c * self._send_chunk_bytes)
                    seg.append(sum(A[me][c][:me]))
                    continue
                dst = self._recv_local[c].data_ptr() + landed * rb
                base.append(dst)
                seg.append(0)
                if n > 0:
                    cs = self._copy_streams[q]
                    cs.wait_event(ev_counts)
                    src = self._send_buf.peers[q] + c * self._send_chunk_bytes + sum(A[q][c][:me]) * rb
                    copy(dst, src, n * rb, cs)
                    ev = torch.cuda.Event()
                    ev.record(cs)
                    evs.append(ev)
                landed += n
            in_events.append(evs)
            bases.append(base)
            seg_offs.append(seg)
        for c in range(Cn):
            a, b = spans[c]
            with torch.cuda.stream(s_main):
                for ev in in_events[c]:
                    s_main.wait_event(ev)
                recv_counts = [A[q][c][me] for q in range(W)]
                f = self.stages.expert_p2p(bases[c], seg_offs[c], recv_counts, H, self.I, self.El, K, self.w1,
                                           self.w2, self._out_buf.ptr + c * self._out_chunk_bytes, errs[c:c + 1], dev)
                freq += f
                # every rank's chunk-c rows are complete; MAX keeps one rank's code intact
                dist.all_reduce(errs[c:c + 1], op=dist.ReduceOp.MAX, group=self.group)
                ev_rows = torch.cuda.Event()
                ev_rows.record(s_main)
            # partial rows out of every peer's output region for this rank's chunk-c records
            ret = self._ret_local[c]
            out_evs, row_bases, recv_start, off = [], [], [], 0
            for d in range(W):
                n = A[me][c][d]
                first = sum(A[q][c][d] for q in range(me))  # this rank's rows in d's region
                if d == me:
                    row_bases.append(self._out_buf.ptr + c * self._out_chunk_bytes)
                    recv_start.append(first)
                else:
                    row_bases.append(ret.data_ptr())
                    recv_start.append(off)
                    if n > 0:
                        cs = self._copy_streams[d]
                        cs.wait_event(ev_rows)
                        copy(ret.data_ptr() + off * H * 2,
                             self._out_buf.peers[d] + c * self._out_chunk_bytes + first * H * 2, n * H * 2, cs)
                        ev = torch.cuda.Event()
                        ev.record(cs)
                        out_evs.append(ev)
                off += n
            with torch.cuda.stream(s_comb):
                s_comb.wait_event(ev_rows)
                for ev in out_evs:
                    s_comb.wait_event(ev)
                states[c].ret_row.record_stream(s_comb)
                self.stages.combine_p2p(row_bases, A[me][c], recv_start, states[c].ret_row, b - a, K, H, dev,
                                        out=out[a:b])
        ev_done = torch.cuda.Event()
        ev_done.record(s_comb)
        caller.wait_event(ev_done)
        caller.wait_stream(s_main)
        for t in (logits, out, freq):
            t.record_stream(caller)
        self._err_pending = errs
        self._note_exchange(sum(A[q][c][me] for c in range(Cn) for q in range(W) if q != me),
                            sum(A[me][c][d] for c in range(Cn) for d in range(W) if d != me), H, rb)
        return out, logits, freq

    def forward(self, x: torch.Tensor, chunks: int = None):
        """This rank's tokens [T, H] -> (out [T, H] bf16, router_logits [T, E], local expert counts [E/W]).

        The tokens are processed in chunks (the constructor's `chunks`, or this call's for the
        NCCL transport): while chunk c runs through the expert GEMMs, the records of chunk c+1 and
        the partial rows of chunk c-1 move between the ranks (NCCL's stream, or the dispatch and
        combine streams of the peer-memory transport).
        """
        if self.transport == "p2p":
            return self._forward_p2p(x)
        if self.transport == "copy":
            return self._forward_copy(x)
        if self.transport == "home":
            return self._forward_home(x) if self.chunks == 1 else self._forward_home_chunked(x)
        T, H = x.shape
        W, K = self.world, self.K
        if chunks is None:
            chunks = self.chunks
        chunks = max(1, min(chunks, T)) if T > 0 else 1
        err = torch.zeros(1, dtype=torch.int32, device=x.device)
        logits = F.linear(x, self.router_w.to(x.dtype))
        bounds = [(T * c) // chunks for c in range(chunks + 1)]
        states = [
            self.stages.dispatch(x[bounds[c]:bounds[c + 1]].contiguous(), logits[bounds[c]:bounds[c + 1]].contiguous(),
                                 self.E, K, W, self.rank, self.sot, self.norm, err)
            for c in range(chunks)
        ]
        # counts of every chunk in one exchange: row d of send = counts for destination d
        send = torch.stack([s.send_counts for s in states], dim=1).contiguous()  # [W, C]
        recv = torch.empty_like(send)
        self._a2a(recv, send)
        counts = torch.stack([send, recv]).cpu()
        self._raise_pending()  # the previous forward ran on this stream and has finished
        sc = [[int(counts[0, d, c]) for d in range(W)] for c in range(chunks)]
        rc = [[int(counts[1, s_, c]) for s_ in range(W)] for c in range(chunks)]
        msg = ""
        for c in range(chunks):
            msg = msg or check_counts(sc[c], rc[c], states[c].records.shape[0])
        if not self._agree(msg == "", x.device):
            raise RuntimeError(f"expert-parallel exchange aborted on every rank: {msg or 'a peer rank failed its check'}")
        rb = states[0].records.shape[1]
        recv_rec = [torch.empty(max(sum(rc[c]), 1), rb, dtype=torch.uint8, device=x.device) for c in range(chunks)]
        ret = [torch.empty(max(sum(sc[c]), 1), H, dtype=torch.bfloat16, device=x.device) for c in range(chunks)]
        pending_rec = [None] * chunks
        pending_ret = [None] * chunks
        keep = []

        def send_records(c):
            S, R = sum(sc[c]), sum(rc[c])
            pending_rec[c] = self._a2a_async(recv_rec[c][:R], states[c].records[:S], rc[c], sc[c])

        send_records(0)
        freq = None
        for c in range(chunks):
            if c + 1 < chunks:
                send_records(c + 1)
            self._wait(pending_rec[c])
            R = sum(rc[c])
            out_rows, f = self.stages.expert(recv_rec[c][:R], R, H, self.I, self.El, K, self.w1, self.w2, err)
            freq = f if freq is None else freq + f
            keep.append(out_rows)
            pending_ret[c] = self._a2a_async(ret[c][:sum(sc[c])], out_rows, sc[c], rc[c])
        outs = []
        for c in range(chunks):
            self._wait(pending_ret[c])
            outs.append(self.stages.combine(ret[c][:sum(sc[c])], states[c].ret_row, bounds[c + 1] - bounds[c], K, H))
        out = torch.cat(outs) if chunks > 1 else outs[0]
        self._reduce_err(err)
        self._err_pending = err
        me = self.rank
        self._note_exchange(sum(rc[c][q] for c in range(chunks) for q in range(W) if q != me),
                            sum(sc[c][d] for c in range(chunks) for d in range(W) if d != me), H, rb)
        return out, logits, freq

    def _a2a_async(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
            return None
        return dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits,
                                      group=self.group, async_op=True)

    @staticmethod
    def _wait(work):
        if work is not None:
            work.wait()

    __call__ = forward
