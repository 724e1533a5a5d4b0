"""Torch-facing wrappers of the libsonic_b200 entry points.

Every function takes/returns CUDA tensors, validates dtypes and contiguity, and enqueues the
kernels on the current torch CUDA stream (the reference's ops run on the current stream too,
``sonicmoe/functional/forward.py:43``).  Nothing here computes on the host.
"""
from dataclasses import dataclass

import torch

from . import _native as nat

_BLOCK_M = 128


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _need(t: torch.Tensor, name: str, dtype=None):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


_LOGIT_DTYPES = {torch.bfloat16: nat.DTYPE_BF16, torch.float16: nat.DTYPE_F16, torch.float32: nat.DTYPE_F32}


def router_topk(router_logits: torch.Tensor, K: int, softmax_over_topk: bool = True, norm_topk_probs: bool = False,
                scores: torch.Tensor = None, idx: torch.Tensor = None):
    """(scores fp32 [T,K], indices int32 [T,K]) -- reference ``_topk_softmax_fwd`` (forward.py:107-141).

    ``scores`` / ``idx``: optional contiguous fp32 / int32 [T, K] outputs to write into."""
    _need(router_logits, "router_logits")
    if router_logits.dtype not in _LOGIT_DTYPES:
        raise ValueError(f"unsupported logits dtype {router_logits.dtype}")
    T, E = router_logits.shape
    if scores is None:
        scores = torch.empty(T, K, dtype=torch.float32, device=router_logits.device)
    if idx is None:
        idx = torch.empty(T, K, dtype=torch.int32, device=router_logits.device)
    _need(scores, "scores", torch.float32)
    _need(idx, "idx", torch.int32)
    if tuple(scores.shape) != (T, K) or tuple(idx.shape) != (T, K):
        raise ValueError(f"outputs must be [{T}, {K}]")
    nat.call(
        "sm_router_topk",
        _ptr(router_logits),
        _LOGIT_DTYPES[router_logits.dtype],
        T,
        E,
        K,
        int(softmax_over_topk),
        int(norm_topk_probs),
        _ptr(scores),
        _ptr(idx),
        _stream(),
    )
    return scores, idx


def router_fused(x: torch.Tensor, router_w: torch.Tensor, K: int, softmax_over_topk: bool = True,
                 norm_topk_probs: bool = False, err: torch.Tensor = None):
    """Fused router (opt-in): (router_logits bf16 [T, E], scores fp32 [T, K], indices int32 [T, K]) from
    x [T, H] and router_w [E, H] in one tcgen05 kernel -- the reference's ``F.linear`` +
    ``_topk_softmax_fwd`` (functional/__init__.py:501, forward.py:107-141).  The logits come from the
    tensor core's fp32 accumulation, not cuBLAS's, so they can differ from ``F.linear`` in the last
    bf16 bit; the ranking of the logits it returns is exactly ``router_topk``'s."""
    _need(x, "x", torch.bfloat16)
    _need(router_w, "router_w", torch.bfloat16)
    T, H = x.shape
    E = router_w.shape[0]
    if router_w.shape[1] != H:
        raise ValueError(f"router_w {tuple(router_w.shape)} does not match x {tuple(x.shape)}")
    dev = x.device
    logits = torch.empty(T, E, dtype=torch.bfloat16, device=dev)
    scores = torch.empty(T, K, dtype=torch.float32, device=dev)
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    if err is None:
        err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = _workspace(nat.load().sm_router_fused_workspace(T, E), dev)
    nat.call("sm_router_fused", _ptr(x), _ptr(router_w), T, H, E, K, int(softmax_over_topk), int(norm_topk_probs),
             _ptr(logits), _ptr(scores), _ptr(idx), _ptr(ws), ws.numel(), _ptr(err), _stream())
    return logits, scores, idx


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def _outs_or_new(outs, sizes, dev):
    """The caller's contiguous int32 output tensors (checked), or new ones of the given sizes."""
    if outs is None:
        return [torch.empty(n, dtype=torch.int32, device=dev) for n in sizes]
    for t, n in zip(outs, sizes):
        _need(t, "metadata output", torch.int32)
        if t.numel() != n:
            raise ValueError(f"metadata output has {t.numel()} elements, expected {n}")
    return list(outs)


def route_metadata(topk_indices: torch.Tensor, E: int, err: torch.Tensor = None, outs=None):
    """Reference ``TC_topk_router_metadata_triton`` (triton_kernels/__init__.py:78-146).

    Returns (expert_frequency, expert_frequency_offset, x_gather_idx, s_scatter_idx, s_reverse_scatter_idx),
    written into ``outs`` (five contiguous int32 tensors) when given.
    """
    _need(topk_indices, "topk_indices", torch.int32)
    T, K = topk_indices.shape
    TK = T * K
    dev = topk_indices.device
    freq, off, xg, ss, sr = _outs_or_new(outs, (E, E + 1, TK, TK, TK), dev)
    if err is None:
        err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = _workspace(nat.load().sm_route_metadata_workspace(T, TK, E), dev)
    nat.call(
        "sm_route_metadata", _ptr(topk_indices), T, K, E, _ptr(freq), _ptr(off), _ptr(xg), _ptr(ss), _ptr(sr),
        _ptr(ws), ws.numel(), _ptr(err), _stream(),
    )
    return freq, off, xg, ss, sr


def general_route_metadata(sorted_token_idx: torch.Tensor, expert_idx: torch.Tensor, T: int, E: int, err=None,
                           outs=None):
    """Reference ``general_routing_router_metadata_triton`` (triton_kernels/__init__.py:281-353).

    Returns (freq, offset, x_gather_idx, s_scatter_idx, s_reverse_scatter_idx, token_offset[T+1]),
    written into ``outs`` (six contiguous int32 tensors) when given.
    """
    _need(sorted_token_idx, "sorted_token_idx", torch.int32)
    _need(expert_idx, "expert_idx", torch.int32)
    TK = expert_idx.numel()
    dev = expert_idx.device
    freq, off, xg, ss, sr, tok_off = _outs_or_new(outs, (E, E + 1, TK, TK, TK, T + 1), dev)
    if err is None:
        err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = _workspace(nat.load().sm_route_metadata_workspace(T, TK, E), dev)
    nat.call(
        "sm_general_route_metadata", _ptr(sorted_token_idx), _ptr(expert_idx), T, TK, E, _ptr(freq), _ptr(off),
        _ptr(xg), _ptr(ss), _ptr(sr), _ptr(tok_off), _ptr(ws), ws.numel(), _ptr(err), _stream(),
    )
    return freq, off, xg, ss, sr, tok_off


def quant_1x128(x: torch.Tensor):
    """1x128 e4m3 quantisation in token order: (q uint8 [R,C], sf atoms uint8 [ceil(R/128), ceil(C/512), 512])."""
    _need(x, "x", torch.bfloat16)
    R, C = x.shape
    q = torch.empty(R, C, dtype=torch.uint8, device=x.device)
    sf = torch.zeros(-(-R // _BLOCK_M), -(-C // 512), 512, dtype=torch.uint8, device=x.device)
    nat.call("sm_quant_1x128", _ptr(x), R, C, _ptr(q), _ptr(sf), _stream())
    return q, sf


@dataclass
class Fp8ExpertWeights:
    """e4m3 expert weights + 128x128 UE8M0 scale atoms, as produced by ``weight_prep``.

    ``q``: [E, N, K] uint8 (e4m3 bits); ``sf``: [E, N/128, ceil(K/512), 512] uint8;
    ``concat_glu``: the rows were re-blocked from a concatenated [gate; up] layout;
    ``t``: the same weight transposed for the backward GEMMs (``weight_prep_t``), when it was
    prepared alongside.
    """

    q: torch.Tensor
    sf: torch.Tensor
    concat_glu: bool
    t: "Fp8ExpertWeights" = None

    @property
    def shape(self):
        return tuple(self.q.shape)


def weight_prep(w: torch.Tensor, concat_glu: bool = False, with_t: bool = False) -> Fp8ExpertWeights:
    """Quantise expert weights [E, N, K] (bf16) to e4m3 with 128x128 UE8M0 scales; with_t also
    writes the transposed copy the backward uses (``.t``, as ``weight_prep_t`` would), in the same pass."""
    if w.dtype != torch.bfloat16:
        w = w.to(torch.bfloat16)
    w = w.contiguous()
    _need(w, "w", torch.bfloat16)
    E, N, K = w.shape
    q = torch.empty(E, N, K, dtype=torch.uint8, device=w.device)
    sf = torch.zeros(E, N // _BLOCK_M, -(-(K // 128) // 4), 512, dtype=torch.uint8, device=w.device)
    if not with_t:
        nat.call("sm_weight_prep", _ptr(w), E, N, K, int(concat_glu), _ptr(q), _ptr(sf), _stream())
        return Fp8ExpertWeights(q, sf, bool(concat_glu))
    qt = torch.empty(E, K, N, dtype=torch.uint8, device=w.device)
    sft = torch.zeros(E, K // _BLOCK_M, -(-(N // 128) // 4), 512, dtype=torch.uint8, device=w.device)
    nat.call("sm_weight_prep_with_t", _ptr(w), E, N, K, int(concat_glu), _ptr(q), _ptr(sf), _ptr(qt), _ptr(sft),
             _stream())
    return Fp8ExpertWeights(q, sf, bool(concat_glu), Fp8ExpertWeights(qt, sft, False))


def max_padded_blocks(TK: int, E: int) -> int:
    return nat.load().sm_max_padded_blocks(TK, E)


@dataclass
class RoutePlan:
    """Routing metadata plus the 128-row padded expert layout the GEMMs run on."""

    freq: torch.Tensor
    off: torch.Tensor
    x_gather: torch.Tensor
    s_scatter: torch.Tensor
    s_rev: torch.Tensor
    off_pad: torch.Tensor
    blk_expert: torch.Tensor
    n_blocks: torch.Tensor
    max_blocks: int
    tok_off: torch.Tensor = None  # explicit routing lists: entries [tok_off[t], tok_off[t+1]) of token t


def route_plan(topk_indices: torch.Tensor, E: int, err: torch.Tensor) -> RoutePlan:
    _need(topk_indices, "topk_indices", torch.int32)
    T, K = topk_indices.shape
    TK = T * K
    dev = topk_indices.device
    mb = max_padded_blocks(TK, E)
    p = RoutePlan(
        freq=torch.empty(E, dtype=torch.int32, device=dev),
        off=torch.empty(E + 1, dtype=torch.int32, device=dev),
        x_gather=torch.empty(TK, dtype=torch.int32, device=dev),
        s_scatter=torch.empty(TK, dtype=torch.int32, device=dev),
        s_rev=torch.empty(TK, dtype=torch.int32, device=dev),
        off_pad=torch.empty(E + 1, dtype=torch.int32, device=dev),
        blk_expert=torch.empty(mb + 1, dtype=torch.int32, device=dev),
        n_blocks=torch.empty(1, dtype=torch.int32, device=dev),
        max_blocks=mb,
    )
    ws = _workspace(nat.load().sm_route_metadata_workspace(T, TK, E), dev)
    nat.call(
        "sm_route_plan", _ptr(topk_indices), T, K, E, _ptr(p.freq), _ptr(p.off), _ptr(p.x_gather),
        _ptr(p.s_scatter), _ptr(p.s_rev), _ptr(p.off_pad), _ptr(p.blk_expert), _ptr(p.n_blocks), _ptr(ws),
        ws.numel(), _ptr(err), _stream(),
    )
    return p


def general_route_plan(token_indices: torch.Tensor, expert_indices: torch.Tensor, T: int, E: int,
                       err: torch.Tensor) -> RoutePlan:
    """Routing plan of explicit (token, expert) entries, token_indices sorted ascending."""
    _need(token_indices, "token_indices", torch.int32)
    _need(expert_indices, "expert_indices", torch.int32)
    TK = token_indices.numel()
    dev = token_indices.device
    mb = max_padded_blocks(TK, E)
    p = RoutePlan(
        freq=torch.empty(E, dtype=torch.int32, device=dev),
        off=torch.empty(E + 1, dtype=torch.int32, device=dev),
        x_gather=torch.empty(TK, dtype=torch.int32, device=dev),
        s_scatter=torch.empty(TK, dtype=torch.int32, device=dev),
        s_rev=torch.empty(TK, dtype=torch.int32, device=dev),
        off_pad=torch.empty(E + 1, dtype=torch.int32, device=dev),
        blk_expert=torch.empty(mb + 1, dtype=torch.int32, device=dev),
        n_blocks=torch.empty(1, dtype=torch.int32, device=dev),
        max_blocks=mb,
        tok_off=torch.empty(T + 1, dtype=torch.int32, device=dev),
    )
    ws = _workspace(nat.load().sm_route_metadata_workspace(T, TK, E), dev)
    nat.call(
        "sm_general_route_plan", _ptr(token_indices), _ptr(expert_indices), T, TK, E, _ptr(p.freq), _ptr(p.off),
        _ptr(p.x_gather), _ptr(p.s_scatter), _ptr(p.s_rev), _ptr(p.tok_off), _ptr(p.off_pad), _ptr(p.blk_expert),
        _ptr(p.n_blocks), _ptr(ws), ws.numel(), _ptr(err), _stream(),
    )
    return p


def quant_pack_general(x: torch.Tensor, expert_indices: torch.Tensor, plan: RoutePlan):
    """quant_pack for explicit routing lists (plan from general_route_plan)."""
    _need(x, "x", torch.bfloat16)
    T, H = x.shape
    xq = torch.empty(plan.max_blocks * _BLOCK_M, H, dtype=torch.uint8, device=x.device)
    xsf = torch.zeros(plan.max_blocks, -(-H // 512), 512, dtype=torch.uint8, device=x.device)
    nat.call(
        "sm_quant_pack_general", _ptr(x), T, H, _ptr(expert_indices), _ptr(plan.tok_off), _ptr(plan.s_rev),
        _ptr(plan.off), _ptr(plan.off_pad), _ptr(xq), _ptr(xsf), _stream(),
    )
    return xq, xsf


def quant_pack(x: torch.Tensor, topk_indices: torch.Tensor, plan: RoutePlan):
    """Quantise x and place each token at its K padded rows: (xq [mb*128, H], xsf atoms)."""
    _need(x, "x", torch.bfloat16)
    T, H = x.shape
    K = topk_indices.shape[1]
    xq = torch.empty(plan.max_blocks * _BLOCK_M, H, dtype=torch.uint8, device=x.device)
    xsf = torch.zeros(plan.max_blocks, -(-H // 512), 512, dtype=torch.uint8, device=x.device)
    nat.call(
        "sm_quant_pack", _ptr(x), T, H, _ptr(topk_indices), K, _ptr(plan.s_rev), _ptr(plan.off), _ptr(plan.off_pad),
        _ptr(xq), _ptr(xsf), _stream(),
    )
    return xq, xsf


def moe_up(xq, xsf, w1: Fp8ExpertWeights, plan: RoutePlan, err, preact_out: torch.Tensor = None):
    """Up projection + SwiGLU + requantisation.  With ``preact_out`` (bf16 [T*K, 2I]) the training
    forward's pre-activation h is stored too, in the reference's expert-sorted row order."""
    E, N2, H = w1.shape
    I = N2 // 2
    aq = torch.empty(plan.max_blocks * _BLOCK_M, I, dtype=torch.uint8, device=xq.device)
    asf = torch.zeros(plan.max_blocks, -(-I // 512), 512, dtype=torch.uint8, device=xq.device)
    if preact_out is not None:
        _need(preact_out, "preact_out", torch.bfloat16)
        if preact_out.dim() != 2 or preact_out.shape[1] != N2 or preact_out.shape[0] != plan.s_scatter.numel():
            raise ValueError(f"preact_out must be [T*K, {N2}] bf16")
        nat.call(
            "sm_moe_up_preact", _ptr(xq), _ptr(xsf), _ptr(w1.q), _ptr(w1.sf), H, I, E, int(w1.concat_glu),
            plan.max_blocks, _ptr(plan.blk_expert), _ptr(plan.n_blocks), _ptr(plan.off_pad), _ptr(plan.off),
            _ptr(plan.freq), _ptr(aq), _ptr(asf), _ptr(preact_out), _ptr(err), _stream(),
        )
        return aq, asf
    nat.call(
        "sm_moe_up", _ptr(xq), _ptr(xsf), _ptr(w1.q), _ptr(w1.sf), H, I, E, int(w1.concat_glu), plan.max_blocks,
        _ptr(plan.blk_expert), _ptr(plan.n_blocks), _ptr(plan.off_pad), _ptr(plan.freq), _ptr(aq), _ptr(asf),
        _ptr(err), _stream(),
    )
    return aq, asf


def moe_down_combine(aq, asf, w2: Fp8ExpertWeights, plan: RoutePlan, scores: torch.Tensor, T: int, err, out=None):
    E, H, I = w2.shape
    if out is None:
        out = torch.zeros(T, H, dtype=torch.bfloat16, device=aq.device)
    nat.call(
        "sm_moe_down_combine", _ptr(aq), _ptr(asf), _ptr(w2.q), _ptr(w2.sf), H, I, E, T, plan.max_blocks,
        _ptr(plan.blk_expert), _ptr(plan.n_blocks), _ptr(plan.off_pad), _ptr(plan.off), _ptr(plan.freq),
        _ptr(plan.s_scatter), _ptr(plan.x_gather), _ptr(scores), _ptr(out), _ptr(err), _stream(),
    )
    return out


def moe_forward(
    x: torch.Tensor,
    router_logits: torch.Tensor,
    w1: Fp8ExpertWeights,
    w2: Fp8ExpertWeights,
    K: int,
    softmax_over_topk: bool = True,
    norm_topk_probs: bool = False,
    out: torch.Tensor = None,
    expert_frequency: torch.Tensor = None,
    topk_scores: torch.Tensor = None,
    topk_indices: torch.Tensor = None,
    err: torch.Tensor = None,
):
    """The whole FP8 layer forward after the router GEMM (one C-ABI call, 7 kernels).

    The scratch workspace is a fresh tensor of the caching allocator for every call, so calls on
    different streams never share scratch (inside a captured CUDA graph it comes from the graph's
    own memory pool).
    """
    _need(x, "x", torch.bfloat16)
    _need(router_logits, "router_logits", torch.bfloat16)
    T, H = x.shape
    E, N2, H1 = w1.shape
    E2, H2, I = w2.shape
    if H1 != H or H2 != H or N2 != 2 * I or E2 != E or router_logits.shape != (T, E):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, logits {tuple(router_logits.shape)}, "
                         f"w1 {w1.shape}, w2 {w2.shape}")
    dev = x.device
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    if expert_frequency is None:
        expert_frequency = torch.empty(E, dtype=torch.int32, device=dev)
    ws = _workspace(nat.load().sm_moe_workspace_bytes(T, H, I, E, K), dev)
    nat.call(
        "sm_moe_forward", _ptr(x), _ptr(router_logits), T, H, I, E, K, int(softmax_over_topk), int(norm_topk_probs),
        int(w1.concat_glu), _ptr(w1.q), _ptr(w1.sf), _ptr(w2.q), _ptr(w2.sf), _ptr(out), _ptr(expert_frequency),
        _ptr(topk_scores), _ptr(topk_indices), _ptr(ws), ws.numel(), _ptr(err), _stream(),
    )
    return out, expert_frequency


def moe_forward_fused_router(
    x: torch.Tensor,
    router_w: torch.Tensor,
    w1: Fp8ExpertWeights,
    w2: Fp8ExpertWeights,
    K: int,
    softmax_over_topk: bool = True,
    norm_topk_probs: bool = False,
    err: torch.Tensor = None,
):
    """``moe_forward`` with the fused router in place of the caller's router GEMM (one C-ABI call):
    returns (out [T, H] bf16, router_logits [T, E] bf16, expert_frequency [E] int32)."""
    _need(x, "x", torch.bfloat16)
    _need(router_w, "router_w", torch.bfloat16)
    T, H = x.shape
    E, N2, H1 = w1.shape
    E2, H2, I = w2.shape
    if H1 != H or H2 != H or N2 != 2 * I or E2 != E or tuple(router_w.shape) != (E, H):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, router_w {tuple(router_w.shape)}, "
                         f"w1 {w1.shape}, w2 {w2.shape}")
    dev = x.device
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    logits = torch.empty(T, E, dtype=torch.bfloat16, device=dev)
    expert_frequency = torch.empty(E, dtype=torch.int32, device=dev)
    ws = _workspace(nat.load().sm_moe_workspace_bytes(T, H, I, E, K), dev)
    nat.call(
        "sm_moe_forward_fused_router", _ptr(x), _ptr(router_w), T, H, I, E, K, int(softmax_over_topk),
        int(norm_topk_probs), int(w1.concat_glu), _ptr(w1.q), _ptr(w1.sf), _ptr(w2.q), _ptr(w2.sf), _ptr(out),
        _ptr(logits), _ptr(expert_frequency), None, None, _ptr(ws), ws.numel(), _ptr(err), _stream(),
    )
    return out, logits, expert_frequency


def moe_general_forward(
    x: torch.Tensor,
    router_scores: torch.Tensor,
    token_indices: torch.Tensor,
    expert_indices: torch.Tensor,
    w1: Fp8ExpertWeights,
    w2: Fp8ExpertWeights,
    out: torch.Tensor = None,
    expert_frequency: torch.Tensor = None,
    err: torch.Tensor = None,
):
    """FP8 layer forward from explicit (token, expert, score) entries, token_indices sorted ascending."""
    _need(x, "x", torch.bfloat16)
    _need(router_scores, "router_scores", torch.float32)
    _need(token_indices, "token_indices", torch.int32)
    _need(expert_indices, "expert_indices", torch.int32)
    T, H = x.shape
    E, N2, H1 = w1.shape
    E2, H2, I = w2.shape
    TK = router_scores.numel()
    if H1 != H or H2 != H or N2 != 2 * I or E2 != E or token_indices.numel() != TK or expert_indices.numel() != TK:
        raise ValueError("shape mismatch between x, routing lists and weights")
    dev = x.device
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    if expert_frequency is None:
        expert_frequency = torch.empty(E, dtype=torch.int32, device=dev)
    nbytes = nat.load().sm_moe_general_workspace_bytes(T, TK, H, I, E)
    ws = _workspace(nbytes, dev)
    nat.call(
        "sm_moe_general_forward", _ptr(x), T, H, I, E, TK, _ptr(router_scores), _ptr(token_indices),
        _ptr(expert_indices), int(w1.concat_glu), _ptr(w1.q), _ptr(w1.sf), _ptr(w2.q), _ptr(w2.sf), _ptr(out),
        _ptr(expert_frequency), _ptr(ws), ws.numel(), _ptr(err), _stream(),
    )
    return out, expert_frequency


# ---------------------------------------------------------------------------------------------
# backward stages (FP8, interleaved SwiGLU); see include/sonic_b200.h for the data layouts


def weight_prep_t(w: Fp8ExpertWeights) -> Fp8ExpertWeights:
    """W^T as a backward GEMM's K-major operand, from the forward's prepared weight: e4m3 [E, N, K] ->
    [E, K, N], the same values and 128x128 block scales read transposed (for a concatenated w1 the K
    order is the prepared weight's re-blocked row order).  A weight prepared with ``with_t`` returns
    the copy it already holds."""
    if w.t is not None:
        return w.t
    E, N, K = w.shape
    q = torch.empty(E, K, N, dtype=torch.uint8, device=w.q.device)
    sf = torch.zeros(E, K // _BLOCK_M, -(-(N // 128) // 4), 512, dtype=torch.uint8, device=w.q.device)
    nat.call("sm_weight_prep_t", _ptr(w.q), _ptr(w.sf), E, N, K, _ptr(q), _ptr(sf), _stream())
    return Fp8ExpertWeights(q, sf, False)


def moe_dact(doq, dosf, w2t: Fp8ExpertWeights, plan: RoutePlan, scores_flat: torch.Tensor, preact: torch.Tensor, err,
             dscores: torch.Tensor = None, concat_layout: bool = False, with_q: bool = True):
    """dA' = dO W2 per entry fused with the SwiGLU backward: (dh_q, dh_sf, dh_bf16, a_prime, dscores).
    with_q=False: no e4m3 copy of dH (dh_q = dh_sf = None; ``tq_pack_dual`` makes it)."""
    E, I, H = w2t.shape
    rows = plan.max_blocks * _BLOCK_M
    dev = doq.device
    dh_q = torch.empty(rows, 2 * I, dtype=torch.uint8, device=dev) if with_q else None
    dh_sf = torch.zeros(plan.max_blocks, -(-(2 * I) // 512), 512, dtype=torch.uint8, device=dev) if with_q else None
    dh = torch.empty(rows, 2 * I, dtype=torch.bfloat16, device=dev)
    a_prime = torch.empty(rows, I, dtype=torch.bfloat16, device=dev)
    if dscores is None:
        dscores = torch.zeros(preact.shape[0], dtype=torch.float32, device=dev)
    _need(preact, "preact", torch.bfloat16)
    nat.call(
        "sm_moe_dact", _ptr(doq), _ptr(dosf), _ptr(w2t.q), _ptr(w2t.sf), H, I, E, plan.max_blocks,
        _ptr(plan.blk_expert), _ptr(plan.n_blocks), _ptr(plan.off_pad), _ptr(plan.off), _ptr(plan.freq),
        _ptr(plan.s_scatter), _ptr(scores_flat), _ptr(preact), int(concat_layout), _ptr(dh_q), _ptr(dh_sf), _ptr(dh),
        _ptr(a_prime), _ptr(dscores), _ptr(err), _stream(),
    )
    return dh_q, dh_sf, dh, a_prime, dscores


def tq_pack(src: torch.Tensor, plan: RoutePlan, padded: bool):
    """Transposed, column-quantised weight-gradient operand [C, rows] of padded rows (gathered token
    rows of src [T, C] when not ``padded``)."""
    _need(src, "src", torch.bfloat16)
    C = src.shape[1]
    rows = plan.max_blocks * _BLOCK_M
    q = torch.empty(C, rows, dtype=torch.uint8, device=src.device)
    sf = torch.zeros(C // _BLOCK_M, -(-plan.max_blocks // 4), 512, dtype=torch.uint8, device=src.device)
    nat.call(
        "sm_tq_pack", _ptr(src), C, int(padded), plan.max_blocks, _ptr(plan.blk_expert), _ptr(plan.n_blocks),
        _ptr(plan.off_pad), _ptr(plan.off), _ptr(plan.freq), _ptr(plan.x_gather), _ptr(q), _ptr(sf), _stream(),
    )
    return q, sf


def tq_pack_dual(src: torch.Tensor, plan: RoutePlan, concat_i: int = 0):
    """``tq_pack`` of a padded source plus its row-quantised copy from the same read: (out_q, out_sf,
    row_q [rows, C], row_sf) -- the dW1 operand and the dX GEMM's dH operand (column blocks re-blocked
    for a concatenated [gate | up] source when concat_i = I)."""
    _need(src, "src", torch.bfloat16)
    C = src.shape[1]
    rows = plan.max_blocks * _BLOCK_M
    dev = src.device
    q = torch.empty(C, rows, dtype=torch.uint8, device=dev)
    sf = torch.zeros(C // _BLOCK_M, -(-plan.max_blocks // 4), 512, dtype=torch.uint8, device=dev)
    rq = torch.empty(rows, C, dtype=torch.uint8, device=dev)
    rsf = torch.zeros(plan.max_blocks, -(-C // 512), 512, dtype=torch.uint8, device=dev)
    nat.call(
        "sm_tq_pack_dual", _ptr(src), C, plan.max_blocks, _ptr(plan.blk_expert), _ptr(plan.n_blocks),
        _ptr(plan.off_pad), _ptr(plan.freq), _ptr(q), _ptr(sf), _ptr(rq), _ptr(rsf), int(concat_i), _stream(),
    )
    return q, sf, rq, rsf


def moe_wgrad(aq, asf, bq, bsf, E: int, plan: RoutePlan, err):
    """Per-expert weight gradient [E, M, N] bf16 = A[:, rows_e] B[:, rows_e]^T."""
    M, N = aq.shape[0], bq.shape[0]
    out = torch.empty(E, M, N, dtype=torch.bfloat16, device=aq.device)
    nat.call("sm_moe_wgrad", _ptr(aq), _ptr(asf), _ptr(bq), _ptr(bsf), M, N, E, plan.max_blocks, _ptr(plan.off_pad),
             _ptr(out), _ptr(err), _stream())
    return out


def router_bwd(router_logits: torch.Tensor, scores: torch.Tensor, idx: torch.Tensor, dscores: torch.Tensor,
               softmax_over_topk: bool = True, norm_topk_probs: bool = False):
    """Gradient of the router logits [T, E] (fp32) from the scores' gradient [T, K]."""
    T, E = router_logits.shape
    K = idx.shape[1]
    dl = torch.empty(T, E, dtype=torch.float32, device=router_logits.device)
    nat.call("sm_router_bwd", _ptr(router_logits), _ptr(scores), _ptr(idx), _ptr(dscores.contiguous()), T, E, K,
             int(softmax_over_topk), int(norm_topk_probs), _ptr(dl), _stream())
    return dl


def moe_backward(dout: torch.Tensor, x: torch.Tensor, router_logits: torch.Tensor, w1: Fp8ExpertWeights,
                 w2: Fp8ExpertWeights, scores: torch.Tensor, idx: torch.Tensor, plan: RoutePlan, preact: torch.Tensor,
                 softmax_over_topk: bool, norm_topk_probs: bool, err, general: bool = False):
    """The layer backward from dO [T, H]: (dx [T, H] bf16, dlogits [T, E] fp32, dw1 [E, 2I, H] bf16,
    dw2 [E, H, I] bf16, dscores [T, K] fp32).  w1 / w2: the forward's prepared e4m3 expert weights
    ([E, 2I, H] / [E, H, I]; w1 interleaved or concatenated, as prepared); the backward GEMMs use them
    transposed, and dw1 comes back in the caller's w1 row order.

    general=True: explicit routing lists (plan from ``general_route_plan``, ``idx`` = the entries'
    expert ids [TK], ``scores`` = the router scores [TK]); dlogits is None and dscores [TK] is the
    gradient of the router scores."""
    T, H = dout.shape
    E = w1.shape[0]
    K = 1 if general else idx.shape[1]
    dout = dout.contiguous()
    doq, dosf = quant_pack_general(dout, idx, plan) if general else quant_pack(dout, idx, plan)
    w2t = weight_prep_t(w2)
    _, _, dh, a_prime, ds = moe_dact(doq, dosf, w2t, plan, scores.view(-1), preact, err,
                                     concat_layout=w1.concat_glu, with_q=False)
    del doq, dosf, w2t
    # one read of dH: the dW1 operand (transposed, column-quantised) and the dX operand (row-quantised)
    dht_q, dht_sf, dh_q, dh_sf = tq_pack_dual(dh, plan, concat_i=dh.shape[1] // 2 if w1.concat_glu else 0)
    del dh
    w1t = weight_prep_t(w1)
    dx = torch.zeros(T, H, dtype=torch.bfloat16, device=dout.device)
    E1, H1, N2 = w1t.shape
    nat.call(
        "sm_moe_down_combine", _ptr(dh_q), _ptr(dh_sf), _ptr(w1t.q), _ptr(w1t.sf), H, N2, E, T, plan.max_blocks,
        _ptr(plan.blk_expert), _ptr(plan.n_blocks), _ptr(plan.off_pad), _ptr(plan.off), _ptr(plan.freq),
        _ptr(plan.s_scatter), _ptr(plan.x_gather), None, _ptr(dx), _ptr(err), _stream(),
    )
    del dh_q, dh_sf, w1t
    dot_q, dot_sf = tq_pack(dout, plan, padded=False)
    apt_q, apt_sf = tq_pack(a_prime, plan, padded=True)
    dw2 = moe_wgrad(dot_q, dot_sf, apt_q, apt_sf, E, plan, err)  # [E, H, I]
    del dot_q, dot_sf, apt_q, apt_sf, a_prime
    xt_q, xt_sf = tq_pack(x.contiguous(), plan, padded=False)
    dw1 = moe_wgrad(dht_q, dht_sf, xt_q, xt_sf, E, plan, err)  # [E, 2I, H]
    if general:
        return dx, None, dw1, dw2, ds
    ds = ds.view(T, K)
    dlogits = router_bwd(router_logits, scores, idx, ds, softmax_over_topk, norm_topk_probs)
    return dx, dlogits, dw1, dw2, ds
