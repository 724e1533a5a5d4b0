"""Expert-parallel FP8 MoE layer forward: experts sharded over the ranks of a process group.

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


class NativeStages:
    """The three device stages through the C ABI (the only implementation in the package)."""

    def __init__(self):
        self.lib = nat.load()

    def record_bytes(self, H, K):
        return self.lib.sm_ep_record_bytes(H, K)

    def dispatch(self, x, logits, E, K, W, rank, sot, norm, err):
        T, H = x.shape
        rb = self.record_bytes(H, K)
        dev = x.device
        s_max = T * min(K, W)
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
                 stages=None):
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

    # ---- forward -----------------------------------------------------------------------------
    def forward(self, x: torch.Tensor):
        T, H = x.shape
        W, K = self.world, self.K
        err = torch.zeros(1, dtype=torch.int32, device=x.device)
        logits = F.linear(x, self.router_w.to(x.dtype))
        st = self.stages.dispatch(x, logits, self.E, K, W, self.rank, self.sot, self.norm, err)
        recv_counts = torch.empty_like(st.send_counts)
        self._a2a(recv_counts, st.send_counts)
        counts = torch.stack([st.send_counts, recv_counts]).cpu()
        sc, rc = counts[0].tolist(), counts[1].tolist()
        msg = check_counts(sc, rc, st.records.shape[0])
        if not self._agree(msg == "", x.device):
            raise RuntimeError(f"expert-parallel exchange aborted on every rank: {msg or 'a peer rank failed its check'}")
        S, R = sum(sc), sum(rc)
        rb = st.records.shape[1]
        recv = torch.empty(max(R, 1), rb, dtype=torch.uint8, device=x.device)
        self._a2a(recv[:R], st.records[:S], rc, sc)
        out_rows, freq = self.stages.expert(recv[:R], R, H, self.I, self.El, K, self.w1, self.w2, err)
        ret = torch.empty(max(S, 1), H, dtype=torch.bfloat16, device=x.device)
        self._a2a(ret[:S], out_rows, sc, rc)
        out = self.stages.combine(ret[:S], st.ret_row, T, K, H)
        return out, logits, freq

    __call__ = forward
