"""Expert-parallel FP8 MoE layer forward: experts sharded over the ranks of a process group.

Two transports move the records and partial rows between the ranks of one node:

* ``"p2p"`` (default on GPUs): every rank's send buffer and output rows live in CUDA IPC memory
  mapped by all ranks; the receiver's pack kernel and the owner's combine kernel read them with
  peer loads over NVLink, so no separate all-to-all copies the data.  NCCL carries only the
  per-destination counts (an all-gather that also orders the stages) and one tiny all-reduce.
* ``"nccl"``: ``all_to_all_single`` of the records and of the partial rows.

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

The record counts are read on the host between the two exchanges (one small device-to-host copy
per forward), and every rank checks them before any data moves; a bad count on any rank makes all
ranks raise together (the check is itself a collective), so no rank is left waiting in a
collective the others skipped.
"""
import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _native as nat
from .ops import Fp8ExpertWeights, _need, _ptr, _stream, _workspace, weight_prep


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

    def combine_p2p(self, peer_out, send_counts, recv_start, ret_row, T, K, H, device):
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


class ExpertParallelMoE:
    """FP8 SwiGLU MoE layer whose experts are sharded over `group` (torch.distributed, NCCL).

    router_w [E, H] is replicated; w1_local [E/W, 2I, H] / w2_local [E/W, H, I] are this rank's
    experts (bf16, quantised here, or prepared Fp8ExpertWeights).  forward(x) takes this rank's
    tokens [T, H] and returns (out [T, H], router_logits [T, E], local expert_frequency [E/W]).
    """

    def __init__(self, router_w, w1_local, w2_local, num_experts: int, top_k: int, group=None,
                 softmax_over_topk: bool = True, norm_topk_probs: bool = False, concat_layout: bool = False,
                 stages=None, reserve_sms: int = None, transport: str = None, max_tokens: int = None,
                 hidden_size: int = None):
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
        if stages is None:
            # SMs the GEMMs leave free for communication kernels running alongside (default none)
            nat.call("sm_set_gemm_sm_reserve", 0 if reserve_sms is None else reserve_sms)
        if transport is None:
            transport = "p2p" if (stages is None and self.world > 1) else "nccl"
        if transport not in ("p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self._send_buf = self._out_buf = None
        if transport == "p2p":
            if max_tokens is None or hidden_size is None:
                raise ValueError("the p2p transport needs max_tokens and hidden_size to size its shared buffers")
            self.max_tokens = int(max_tokens)
            rb = self.stages.record_bytes(hidden_size, top_k)
            self._send_cap = self.max_tokens * min(top_k, self.world)
            self._out_cap = self.world * self.max_tokens
            self._send_buf = IpcBuffer(max(self._send_cap, 1) * rb, group)
            self._out_buf = IpcBuffer(max(self._out_cap, 1) * hidden_size * 2, group)
        self.router_w = router_w
        prep = (lambda w, c: w) if stages is not None else (lambda w, c: w if isinstance(w, Fp8ExpertWeights)
                                                            else weight_prep(w, concat_glu=c))
        self.w1 = prep(w1_local, concat_layout)
        self.w2 = prep(w2_local, False)
        shp = tuple(self.w1.shape)
        if shp[0] != self.El:
            raise ValueError(f"w1_local holds {shp[0]} experts, expected {self.El}")
        self.I = shp[1] // 2

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
            torch.cuda.synchronize()
            dist.barrier(group=self.group)  # nobody reads a peer buffer any more
            self._send_buf.unmap()
            self._out_buf.unmap()
            torch.cuda.synchronize()
            dist.barrier(group=self.group)  # every peer mapping is gone
            self._send_buf.free()
            self._out_buf.free()
            self._send_buf = self._out_buf = None

    def _forward_p2p(self, x: torch.Tensor):
        T, H = x.shape
        W, K, me = self.world, self.K, self.rank
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of the shared buffers")
        err = torch.zeros(1, dtype=torch.int32, device=x.device)
        logits = F.linear(x, self.router_w.to(x.dtype))
        rb = self.stages.record_bytes(H, K)
        records = _RawRows(self._send_buf.ptr, self._send_cap, rb)
        st = self.stages.dispatch(x, logits, self.E, K, W, me, self.sot, self.norm, err, records=records)
        # counts of every rank (and a barrier: every send buffer is complete once this returns)
        allc = torch.empty(W * W, dtype=torch.int32, device=x.device)
        dist.all_gather_into_tensor(allc, st.send_counts, group=self.group)
        C = allc.view(W, W).cpu().tolist()  # C[s][d]: records from s to d
        recv_counts = [C[s][me] for s in range(W)]
        seg_off = [sum(C[s][:me]) for s in range(W)]
        msg = check_counts(C[me], recv_counts, self._send_cap)
        if not msg and sum(recv_counts) > self._out_cap:
            msg = f"{sum(recv_counts)} received records exceed the output buffer ({self._out_cap})"
        if not self._agree(msg == "", x.device):
            raise RuntimeError(f"expert-parallel exchange aborted on every rank: {msg or 'a peer rank failed its check'}")
        freq = self.stages.expert_p2p(self._send_buf.peers, seg_off, recv_counts, H, self.I, self.El, K, self.w1,
                                      self.w2, self._out_buf.ptr, err, x.device)
        # every rank's output rows are complete once this returns
        dist.all_reduce(err, group=self.group)
        recv_start = [sum(C[s][d] for s in range(me)) for d in range(W)]
        out = self.stages.combine_p2p(self._out_buf.peers, C[me], recv_start, st.ret_row, T, K, H, x.device)
        return out, logits, freq

    # ---- forward -----------------------------------------------------------------------------
    def forward(self, x: torch.Tensor, chunks: int = None):
        """This rank's tokens [T, H] -> (out [T, H] bf16, router_logits [T, E], local expert counts [E/W]).

        The tokens are processed in `chunks` slices (default: 2 with more than one rank): while
        chunk c runs through the expert GEMMs, the records of chunk c+1 and the partial rows of
        chunk c-1 are exchanged on NCCL's stream.
        """
        if self.transport == "p2p":
            return self._forward_p2p(x)
        T, H = x.shape
        W, K = self.world, self.K
        if chunks is None:
            chunks = 1
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
