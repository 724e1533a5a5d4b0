"""Functional API of the reference (``sonicmoe/functional/__init__.py``), on the FP8 B200 engine.

Same names, arguments and return values as the reference:

* ``moe_TC_softmax_topk_layer`` (reference ``functional/__init__.py:482-557``)
* ``moe_general_routing_inputs`` (reference ``functional/__init__.py:571-652``)
* ``TC_topk_router_metadata_triton`` / ``general_routing_router_metadata_triton`` and
  ``_topk_softmax_fwd`` (reference ``triton_kernels/__init__.py:78-146, 281-353``,
  ``forward.py:107-141``), here backed by the CUDA metadata and router kernels.

Weight-format contract (reference ``functional/__init__.py:560-566``): ``w1`` is the
``(2I, H, E)`` view of ``c_fc.weight`` ``[E, 2I, H]`` (stride order (2, 0, 1)), interleaved
``[g0, u0, g1, u1, ...]`` or, with ``concat_layout=True``, ``[g0..g_{I-1}, u0..u_{I-1}]``;
``w2`` is the ``(H, I, E)`` view of ``c_proj.weight`` ``[E, H, I]``.  The bf16 weights are
quantised to e4m3 with 128x128 UE8M0 block scales on first use and cached per weight version;
already prepared :class:`~sonicmoe.ops.Fp8ExpertWeights` may be passed instead.

Op boundary: as in the reference, the router top-k (``sonicmoe::_topk_fwd``,
``sonicmoe::_softmax_topk_fwd``, in ``forward.py``) and the routing metadata
(``triton_kernels::TC_topk_router_metadata``, ``triton_kernels::general_routing_router_metadata``)
are ``torch.library.custom_op``s writing into caller-allocated outputs; the engine's layer forward
after the router GEMM is one more registered op per entry point (``sonicmoe::fp8_moe_tc_forward``,
``sonicmoe::fp8_moe_general_forward``, with fake implementations for tracing), so ``torch.compile``
traces a whole ``MoE`` forward without a graph break.

Training: with ``is_inference_mode_enabled=False`` while autograd is recording and an input or
weight requires grad, ``moe_TC_softmax_topk_layer`` and ``moe_general_routing_inputs`` run the
training forward (the up GEMM also stores the pre-activation h) inside an autograd function whose
backward is the engine's FP8 backward (``ops.moe_backward``: dx, the router logits' or router
scores' gradient, dw1, dw2), as the reference's ``_UpProjection`` / ``_DownProjection`` / router
functions do.

Differences from the reference, all explicit errors: biases and activations other than SwiGLU
raise ``NotImplementedError`` (the FP8 engine implements the bias-free SwiGLU layer); the backward
covers ``moe_TC_softmax_topk_layer`` and ``moe_general_routing_inputs`` (both w1 layouts,
I % 256 == 0) -- the fused router and prepared e4m3 weights raise ``NotImplementedError`` when a
gradient is requested, instead of returning an output whose weights would never receive one.
"""
import weakref

import torch
import torch.nn.functional as F

from .. import ops
from ..enums import ActivationType
from ..ops import Fp8ExpertWeights
from .forward import _topk_fwd, _topk_softmax_fwd  # noqa: F401  (registers the router ops)

__all__ = [
    "moe_TC_softmax_topk_layer",
    "moe_general_routing_inputs",
    "TC_topk_router_metadata_triton",
    "general_routing_router_metadata_triton",
    "prepare_fp8_weights",
    "Fp8ExpertWeights",
]

# Prepared FP8 weights, per tensor that owns the weight's storage (the root of its view chain):
# id(owner) -> (weak reference to owner, {layout: (state, prepared)}).  An entry is dropped when its
# tensor is freed, so a new weight tensor that happens to be allocated at a freed one's address can
# never see the old tensor's FP8 copy.  (Tensors cannot be weak dictionary keys: their == is
# elementwise.)
_WEIGHT_CACHE: dict = {}


def _forget(key: int, ref) -> None:
    entry = _WEIGHT_CACHE.get(key)
    if entry is not None and entry[0] is ref:
        del _WEIGHT_CACHE[key]


def _as_expert_major(w: torch.Tensor) -> torch.Tensor:
    """(N, K, E) reference view -> [E, N, K] tensor (a view when w came from permute(1, 2, 0))."""
    return w.permute(2, 0, 1)


def _storage_owner(t: torch.Tensor) -> torch.Tensor:
    while t._base is not None:
        t = t._base
    return t


def prepare_fp8_weights(w, concat_glu: bool = False, with_t: bool = False) -> Fp8ExpertWeights:
    """e4m3 + 128x128 UE8M0 version of an expert weight given in the reference's (N, K, E) view.

    Cached on the tensor that owns the weight's storage, for its current (data pointer, version
    counter, shape, strides, layout): repeated forwards with unchanged weights quantise once, an
    in-place update or a storage swap re-quantises, and the entry is dropped with the tensor.
    with_t (training): the result also holds the transposed copy the backward reads (prepared in the
    same pass over the weight, or added to a cached entry that lacks it).
    """
    if isinstance(w, Fp8ExpertWeights):
        return w
    owner = _storage_owner(w)
    layout = (tuple(w.shape), tuple(w.stride()), bool(concat_glu), w.dtype)
    state = (w.data_ptr(), w._version)
    entry = _WEIGHT_CACHE.get(id(owner))
    per_owner = entry[1] if entry is not None and entry[0]() is owner else None
    if per_owner is not None:
        hit = per_owner.get(layout)
        if hit is not None and hit[0] == state:
            if with_t and hit[1].t is None:
                hit[1].t = ops.weight_prep_t(hit[1])
            return hit[1]
    with torch.no_grad():
        prepared = ops.weight_prep(_as_expert_major(w.detach()), concat_glu=concat_glu, with_t=with_t)
    if per_owner is None:
        key = id(owner)
        ref = weakref.ref(owner, lambda r, k=key: _forget(k, r))
        per_owner = {}
        _WEIGHT_CACHE[key] = (ref, per_owner)
    per_owner[layout] = (state, prepared)  # only the newest version of each layout is kept
    return prepared


def _check_common(b1, b2, activation_type):
    assert ((b1 is None) and (b2 is None)) or (
        (b1 is not None) and (b2 is not None)
    ), "b1 and b2 has to be None or not None at the same time!"
    if b1 is not None:
        raise NotImplementedError("the FP8 engine implements the bias-free layer (b1 = b2 = None)")
    if isinstance(activation_type, str):
        activation_type = ActivationType(activation_type)
    if activation_type != ActivationType.SWIGLU:
        raise NotImplementedError(f"the FP8 engine implements SwiGLU only, got {activation_type}")
    return activation_type


def _wants_training(is_inference_mode_enabled, *tensors) -> bool:
    """True when autograd must see the layer: a training-mode call while grad is recorded and an input
    or weight requires grad."""
    if is_inference_mode_enabled or not torch.is_grad_enabled():
        return False
    return any(isinstance(t, torch.Tensor) and t.requires_grad for t in tensors)


class _FP8MoEFunction(torch.autograd.Function):
    """Training forward + FP8 backward of the token-choice layer after the router GEMM (the reference's
    router function, _UpProjection and _DownProjection autograd functions,
    functional/__init__.py:174-202, 227-479).  Inputs: x [T, H] bf16, router_logits [T, E], w1 / w2 in
    the reference's (2I, H, E) / (H, I, E) views (interleaved or concatenated gate/up rows); outputs
    (o, expert_frequency)."""

    @staticmethod
    def forward(ctx, x, router_logits, w1, w2, K, softmax_over_topk, norm_topk_probs, concat_layout):
        w1q = prepare_fp8_weights(w1, concat_glu=concat_layout, with_t=True)
        w2q = prepare_fp8_weights(w2, concat_glu=False, with_t=True)
        T, H = x.shape
        E = router_logits.shape[1]
        I = w1q.shape[1] // 2
        dev = x.device
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        scores, idx = ops.router_topk(router_logits, K, softmax_over_topk, norm_topk_probs)
        plan = ops.route_plan(idx, E, err)
        xq, xsf = ops.quant_pack(x, idx, plan)
        h = torch.empty(T * K, 2 * I, dtype=torch.bfloat16, device=dev)
        aq, asf = ops.moe_up(xq, xsf, w1q, plan, err, preact_out=h)
        del xq, xsf
        out = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
        ops.moe_down_combine(aq, asf, w2q, plan, scores, T, err, out=out)
        ctx.save_for_backward(x, router_logits, w1, w2, scores, idx, h, err, plan.freq, plan.off, plan.x_gather,
                              plan.s_scatter, plan.s_rev, plan.off_pad, plan.blk_expert, plan.n_blocks)
        ctx.max_blocks = plan.max_blocks
        ctx.modes = (bool(softmax_over_topk), bool(norm_topk_probs), bool(concat_layout))
        freq = plan.freq.clone()
        ctx.mark_non_differentiable(freq)
        return out, freq

    @staticmethod
    def backward(ctx, dout, _dfreq):
        (x, router_logits, w1, w2, scores, idx, h, err, freq, off, x_gather, s_scatter, s_rev, off_pad, blk_expert,
         n_blocks) = ctx.saved_tensors
        plan = ops.RoutePlan(freq, off, x_gather, s_scatter, s_rev, off_pad, blk_expert, n_blocks, ctx.max_blocks)
        sot, norm, concat = ctx.modes
        # the e4m3 weights the forward ran with (cached per weight version), read transposed
        w1q = prepare_fp8_weights(w1, concat_glu=concat)
        w2q = prepare_fp8_weights(w2, concat_glu=False)
        dx, dlogits, dw1, dw2, _ = ops.moe_backward(dout.to(torch.bfloat16).contiguous(), x, router_logits, w1q, w2q,
                                                    scores, idx, plan, h, sot, norm, err)
        code = int(err.item())
        if code:
            raise RuntimeError(f"FP8 MoE backward: device error {code}")
        return (dx, dlogits.to(router_logits.dtype), dw1.permute(1, 2, 0).to(w1.dtype), dw2.permute(1, 2, 0).to(w2.dtype),
                None, None, None, None)


@torch.library.custom_op("sonicmoe::fp8_moe_tc_forward", mutates_args=())
def _fp8_moe_tc_forward(
    x: torch.Tensor,
    router_logits: torch.Tensor,
    w1: torch.Tensor,
    w2: torch.Tensor,
    K: int,
    is_softmax_over_topk: bool,
    norm_topk_probs: bool,
    concat_layout: bool,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Engine part of ``moe_TC_softmax_topk_layer`` after the router GEMM: (o [T, H] bf16,
    expert_frequency [E] int32).  w1 / w2 are the reference's (2I, H, E) / (H, I, E) views."""
    w1q = prepare_fp8_weights(w1, concat_glu=concat_layout)
    w2q = prepare_fp8_weights(w2, concat_glu=False)
    return ops.moe_forward(x, router_logits, w1q, w2q, K, is_softmax_over_topk, norm_topk_probs)


@_fp8_moe_tc_forward.register_fake
def _(x, router_logits, w1, w2, K, is_softmax_over_topk, norm_topk_probs, concat_layout):
    return x.new_empty(x.shape, dtype=torch.bfloat16), x.new_empty(router_logits.shape[1], dtype=torch.int32)


@torch.library.custom_op("sonicmoe::fp8_moe_tc_forward_fused_router", mutates_args=())
def _fp8_moe_tc_forward_fused_router(
    x: torch.Tensor,
    router_w: torch.Tensor,
    w1: torch.Tensor,
    w2: torch.Tensor,
    K: int,
    is_softmax_over_topk: bool,
    norm_topk_probs: bool,
    concat_layout: bool,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``moe_TC_softmax_topk_layer`` with the fused router (router GEMM + top-k in one kernel):
    (o [T, H] bf16, router_logits [T, E] bf16, expert_frequency [E] int32)."""
    w1q = prepare_fp8_weights(w1, concat_glu=concat_layout)
    w2q = prepare_fp8_weights(w2, concat_glu=False)
    return ops.moe_forward_fused_router(x, router_w, w1q, w2q, K, is_softmax_over_topk, norm_topk_probs)


@_fp8_moe_tc_forward_fused_router.register_fake
def _(x, router_w, w1, w2, K, is_softmax_over_topk, norm_topk_probs, concat_layout):
    E = router_w.shape[0]
    return (x.new_empty(x.shape, dtype=torch.bfloat16), x.new_empty((x.shape[0], E), dtype=torch.bfloat16),
            x.new_empty(E, dtype=torch.int32))


@torch.library.custom_op("sonicmoe::fp8_moe_general_forward", mutates_args=())
def _fp8_moe_general_forward(
    x: torch.Tensor,
    router_scores: torch.Tensor,
    token_indices: torch.Tensor,
    expert_indices: torch.Tensor,
    w1: torch.Tensor,
    w2: torch.Tensor,
    concat_layout: bool,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Engine part of ``moe_general_routing_inputs``: (o [T, H] bf16, expert_frequency [E] int32)."""
    w1q = prepare_fp8_weights(w1, concat_glu=concat_layout)
    w2q = prepare_fp8_weights(w2, concat_glu=False)
    return ops.moe_general_forward(x, router_scores, token_indices, expert_indices, w1q, w2q)


@_fp8_moe_general_forward.register_fake
def _(x, router_scores, token_indices, expert_indices, w1, w2, concat_layout):
    return x.new_empty(x.shape, dtype=torch.bfloat16), x.new_empty(w2.shape[-1], dtype=torch.int32)


class _FP8MoEGeneralFunction(torch.autograd.Function):
    """Training forward + FP8 backward of the layer over explicit routing lists
    (``moe_general_routing_inputs``, reference functional/__init__.py:571-652 with its autograd
    functions): gradients for x, the router scores and the expert weights."""

    @staticmethod
    def forward(ctx, x, router_scores, token_indices, expert_indices, w1, w2, concat_layout):
        w1q = prepare_fp8_weights(w1, concat_glu=concat_layout, with_t=True)
        w2q = prepare_fp8_weights(w2, concat_glu=False, with_t=True)
        T, H = x.shape
        E = w2q.shape[0]
        I = w2q.shape[2]
        TK = router_scores.numel()
        dev = x.device
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        plan = ops.general_route_plan(token_indices, expert_indices, T, E, err)
        xq, xsf = ops.quant_pack_general(x, expert_indices, plan)
        h = torch.empty(TK, 2 * I, dtype=torch.bfloat16, device=dev)
        aq, asf = ops.moe_up(xq, xsf, w1q, plan, err, preact_out=h)
        del xq, xsf
        out = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
        ops.moe_down_combine(aq, asf, w2q, plan, router_scores, T, err, out=out)
        ctx.save_for_backward(x, router_scores, expert_indices, w1, w2, h, err, plan.freq, plan.off, plan.x_gather,
                              plan.s_scatter, plan.s_rev, plan.off_pad, plan.blk_expert, plan.n_blocks, plan.tok_off)
        ctx.max_blocks = plan.max_blocks
        ctx.concat = bool(concat_layout)
        freq = plan.freq.clone()
        ctx.mark_non_differentiable(freq)
        return out, freq

    @staticmethod
    def backward(ctx, dout, _dfreq):
        (x, router_scores, expert_indices, w1, w2, h, err, freq, off, x_gather, s_scatter, s_rev, off_pad,
         blk_expert, n_blocks, tok_off) = ctx.saved_tensors
        plan = ops.RoutePlan(freq, off, x_gather, s_scatter, s_rev, off_pad, blk_expert, n_blocks, ctx.max_blocks,
                             tok_off)
        w1q = prepare_fp8_weights(w1, concat_glu=ctx.concat)
        w2q = prepare_fp8_weights(w2, concat_glu=False)
        dx, _, dw1, dw2, ds = ops.moe_backward(dout.to(torch.bfloat16).contiguous(), x, None, w1q, w2q,
                                               router_scores, expert_indices, plan, h, True, False, err, general=True)
        code = int(err.item())
        if code:
            raise RuntimeError(f"FP8 MoE backward: device error {code}")
        return (dx, ds.to(router_scores.dtype), None, None, dw1.permute(1, 2, 0).to(w1.dtype),
                dw2.permute(1, 2, 0).to(w2.dtype), None)


def moe_TC_softmax_topk_layer(
    x: torch.Tensor,
    router_w: torch.Tensor,
    w1,
    b1,
    w2,
    b2,
    K: int,
    stream_id: int,
    activation_type=ActivationType.SWIGLU,
    is_inference_mode_enabled: bool = False,
    is_softmax_over_topk: bool = True,
    norm_topk_probs: bool = False,
    concat_layout: bool = False,
    *,
    fused_router: bool = False,
):
    """Token-choice top-k MoE layer forward.  Returns (o [T, H], router_logits [T, E], expert_frequency [E]).

    ``stream_id`` is ignored, as in the reference (the current torch stream is used).

    ``fused_router`` (keyword only; not in the reference): compute the router logits and their top-k
    in one tcgen05 kernel instead of ``F.linear`` + the top-k kernel.  Its logits come from the
    tensor core's fp32 accumulation, so they can differ from ``F.linear``'s in the last bf16 bit (and
    a near-tie can then route to another expert); needs E % 32 == 0, 32 <= E <= 256, H % 64 == 0.
    """
    _check_common(b1, b2, activation_type)
    if norm_topk_probs and is_softmax_over_topk:
        raise ValueError("`norm_topk_prob` only works with softmax-then-topk")
    training = _wants_training(is_inference_mode_enabled, x, router_w, w1, w2)
    if training and (fused_router or isinstance(w1, Fp8ExpertWeights) or isinstance(w2, Fp8ExpertWeights)):
        raise NotImplementedError("the FP8 backward covers bf16 weights with the F.linear router "
                                  "(no fused_router or prepared weights)")
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    x = x.contiguous()
    if training:
        router_logits = F.linear(x, router_w.to(x.dtype))
        o, expert_frequency = _FP8MoEFunction.apply(x, router_logits, w1, w2, K, is_softmax_over_topk,
                                                    norm_topk_probs, concat_layout)
        return o, router_logits, expert_frequency
    if fused_router:
        rw = router_w.to(x.dtype).contiguous()
        if isinstance(w1, Fp8ExpertWeights) or isinstance(w2, Fp8ExpertWeights):
            w1q = prepare_fp8_weights(w1, concat_glu=concat_layout)
            w2q = prepare_fp8_weights(w2, concat_glu=False)
            if w1q.concat_glu != bool(concat_layout):
                raise ValueError("prepared w1 layout does not match concat_layout")
            o, router_logits, expert_frequency = ops.moe_forward_fused_router(
                x, rw, w1q, w2q, K, is_softmax_over_topk, norm_topk_probs)
        else:
            o, router_logits, expert_frequency = _fp8_moe_tc_forward_fused_router(
                x, rw, w1, w2, K, is_softmax_over_topk, norm_topk_probs, concat_layout)
        return o, router_logits, expert_frequency
    router_logits = F.linear(x, router_w.to(x.dtype))
    if isinstance(w1, Fp8ExpertWeights) or isinstance(w2, Fp8ExpertWeights):
        # already prepared e4m3 weights (a host-side object, not a tensor): eager call
        w1q = prepare_fp8_weights(w1, concat_glu=concat_layout)
        w2q = prepare_fp8_weights(w2, concat_glu=False)
        if w1q.concat_glu != bool(concat_layout):
            raise ValueError("prepared w1 layout does not match concat_layout")
        o, expert_frequency = ops.moe_forward(
            x, router_logits.contiguous(), w1q, w2q, K, is_softmax_over_topk, norm_topk_probs
        )
    else:
        o, expert_frequency = _fp8_moe_tc_forward(
            x, router_logits.contiguous(), w1, w2, K, is_softmax_over_topk, norm_topk_probs, concat_layout
        )
    return o, router_logits, expert_frequency


def moe_general_routing_inputs(
    x: torch.Tensor,
    router_scores: torch.Tensor,
    token_indices: torch.Tensor,
    expert_indices: torch.Tensor,
    w1,
    b1,
    w2,
    b2,
    E: int,
    stream_id: int,
    activation_type=ActivationType.SWIGLU,
    is_inference_mode_enabled: bool = False,
    concat_layout: bool = False,
):
    """MoE forward from explicit (token, expert, score) lists; token_indices must be sorted ascending.

    Returns (o [T, H], expert_frequency [E]).  ``E`` is taken from ``w2`` as in the reference
    (``functional/__init__.py:592``).
    """
    _check_common(b1, b2, activation_type)
    training = _wants_training(is_inference_mode_enabled, x, router_scores, w1, w2)
    if training and (isinstance(w1, Fp8ExpertWeights) or isinstance(w2, Fp8ExpertWeights)):
        raise NotImplementedError("the FP8 backward covers bf16 weights (no prepared weights)")
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    x = x.contiguous()
    if router_scores.dtype != torch.float32:
        router_scores = router_scores.float()
    args = (x, router_scores.contiguous(), token_indices.to(torch.int32).contiguous(),
            expert_indices.to(torch.int32).contiguous())
    if training:
        return _FP8MoEGeneralFunction.apply(*args, w1, w2, concat_layout)
    if isinstance(w1, Fp8ExpertWeights) or isinstance(w2, Fp8ExpertWeights):
        w1q = prepare_fp8_weights(w1, concat_glu=concat_layout)
        w2q = prepare_fp8_weights(w2, concat_glu=False)
        return ops.moe_general_forward(*args, w1q, w2q)
    return _fp8_moe_general_forward(*args, w1, w2, concat_layout)


@torch.library.custom_op(
    "triton_kernels::TC_topk_router_metadata",
    mutates_args={"expert_frequency", "expert_frequency_offset", "x_gather_idx", "s_scatter_idx",
                  "s_reverse_scatter_idx"},
)
def TC_topk_router_metadata_triton(
    topk_router_indices: torch.Tensor,
    E: int,
    expert_frequency: torch.Tensor,
    expert_frequency_offset: torch.Tensor,
    x_gather_idx: torch.Tensor,
    s_scatter_idx: torch.Tensor,
    s_reverse_scatter_idx: torch.Tensor,
) -> None:
    """Reference op and signature (triton_kernels/__init__.py:68-86): fills the five int32 outputs in
    place (directly when they are contiguous int32, else through a copy)."""
    outs = (expert_frequency, expert_frequency_offset, x_gather_idx, s_scatter_idx, s_reverse_scatter_idx)
    idx = topk_router_indices.to(torch.int32).contiguous()
    if all(t.dtype == torch.int32 and t.is_contiguous() for t in outs):
        ops.route_metadata(idx, E, outs=outs)
        return
    for dst, src in zip(outs, ops.route_metadata(idx, E)):
        dst.copy_(src)


@torch.library.custom_op(
    "triton_kernels::general_routing_router_metadata",
    mutates_args={"expert_frequency", "expert_frequency_offset", "x_gather_idx", "s_scatter_idx",
                  "s_reverse_scatter_idx", "num_activated_expert_per_token_offset"},
)
def general_routing_router_metadata_triton(
    sorted_selected_T: torch.Tensor,
    selected_E: torch.Tensor,
    T: int,
    E: int,
    expert_frequency: torch.Tensor,
    expert_frequency_offset: torch.Tensor,
    x_gather_idx: torch.Tensor,
    s_scatter_idx: torch.Tensor,
    s_reverse_scatter_idx: torch.Tensor,
    num_activated_expert_per_token_offset: torch.Tensor,
) -> None:
    """Reference op and signature (triton_kernels/__init__.py:270-292): fills the six int32 outputs in place."""
    outs = (expert_frequency, expert_frequency_offset, x_gather_idx, s_scatter_idx, s_reverse_scatter_idx,
            num_activated_expert_per_token_offset)
    tok = sorted_selected_T.to(torch.int32).contiguous()
    ex = selected_E.to(torch.int32).contiguous()
    if all(t.dtype == torch.int32 and t.is_contiguous() for t in outs):
        ops.general_route_metadata(tok, ex, T, E, outs=outs)
        return
    for dst, src in zip(outs, ops.general_route_metadata(tok, ex, T, E)):
        dst.copy_(src)
