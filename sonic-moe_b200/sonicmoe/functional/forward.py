"""Registered router ops of the reference (``sonicmoe/functional/forward.py``), on the CUDA router.

Same op names, arguments and in-place outputs as the reference's ``torch.library.custom_op``s, so
code that calls ``torch.ops.sonicmoe._softmax_topk_fwd`` / ``_topk_fwd`` and compiled graphs that
contain them keep working:

* ``sonicmoe::_topk_fwd`` (reference ``forward.py:18-58``): top-k of each row (softmax over the
  top-k, or top-k of the softmax with optional renormalisation), values and indices written into
  the caller's tensors.
* ``sonicmoe::_softmax_topk_fwd`` (reference ``forward.py:107-141``): the same with the reference's
  argument order (E, K).  The reference falls back to ``torch.topk`` outside ``E <= 4096, K <= 16,
  E % 8 == 0``; this engine's router covers E <= 4096 and K <= 32 for any E, so it has no fallback.

The reference's third op, ``sonicmoe::_router_forward`` (``forward.py:64-85``, the gather-and-sum of
the down projection's [T*K, H] output), has no counterpart: the down-projection GEMM here adds each
entry's score-weighted row into the token's output row in its epilogue, so no [T*K, H] buffer exists.
"""
import torch

from .. import ops


def _write_topk(logits, k, values, indices, is_softmax_over_topk, norm_topk_probs):
    direct = values.dtype == torch.float32 and values.is_contiguous() and indices.dtype == torch.int32 \
        and indices.is_contiguous()
    if direct:
        ops.router_topk(logits.contiguous(), k, is_softmax_over_topk, norm_topk_probs, scores=values, idx=indices)
        return
    s, i = ops.router_topk(logits.contiguous(), k, is_softmax_over_topk, norm_topk_probs)
    values.copy_(s.to(values.dtype))
    indices.copy_(i.to(indices.dtype))


@torch.library.custom_op("sonicmoe::_topk_fwd", mutates_args={"values", "indices"})
def _topk_fwd(
    x: torch.Tensor,
    k: int,
    values: torch.Tensor,
    indices: torch.Tensor,
    is_softmax_over_topk: bool,
    norm_topk_probs: bool,
) -> None:
    """Top-k of each row of x [M, N] into values / indices [M, k] (reference forward.py:18-58)."""
    _write_topk(x, k, values, indices, is_softmax_over_topk, norm_topk_probs)


@torch.library.custom_op("sonicmoe::_softmax_topk_fwd", mutates_args={"topk_router_score", "topk_router_indices"})
def _topk_softmax_fwd(
    router_logits: torch.Tensor,
    topk_router_score: torch.Tensor,
    topk_router_indices: torch.Tensor,
    E: int,
    K: int,
    is_softmax_over_topk: bool,
    norm_topk_probs: bool,
) -> None:
    """Router top-k + softmax into the caller's [T, K] outputs (reference forward.py:107-141)."""
    if router_logits.size(1) != E:
        raise ValueError(f"router_logits has {router_logits.size(1)} columns, E = {E}")
    _write_topk(router_logits, K, topk_router_score, topk_router_indices, is_softmax_over_topk, norm_topk_probs)
