"""Top-k router restatement (test infrastructure; see ``oracle/__init__.py``).

Follows ``sonicmoe/functional/topk.py`` of the reference:

* ``topk.py:143-198``  (TOPK_OVER_SOFTMAX) full-row log-softmax before selection:
  ``logp = x - (max + log(sum_exp))``.
* ``topk.py:200-215``  the column index is written into the low ``log2(next_pow2(E))`` mantissa
  bits of the float32 score, inverted (``~col``) when the score is ``>= 0`` so that on equal
  scores the LOWER column wins; the original low bits are discarded (for top-k-over-softmax
  this truncates the log-probabilities before ranking).
* ``topk.py:222-234``  descending top-k, then the bits are cleared and the index decoded
  (``~enc`` when the cleared score is ``>= 0``).
* ``topk.py:237-260``  softmax over the k selected values (SOFTMAX_OVER_TOPK) or ``exp`` of the
  log-probabilities, optionally renormalised to sum to one (``norm_topk_prob``).

What this restatement fixes that the reference leaves to its GPU runtime: the exp/log
implementation (``oracle.mathfn``) and the order of the floating-point sums.  The sum of
``exp(x - max)`` over a row is taken lane by lane and then by an xor-butterfly over 32 lanes,
exactly as the CUDA router does it (``lane_layout`` below), so scores and indices are bit-exact
between the CUDA router and this file.  Ranking compares the encoded floats as a total order
(IEEE order, no flush of subnormals).
"""
import numpy as np

from .mathfn import exp_f32, log_f32

F32 = np.float32


def next_pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (int(n) - 1).bit_length()


def lane_vec(E: int) -> int:
    """Elements per lane per load step in the warp-per-row router (8, 4, 2 or 1)."""
    for v in (8, 4, 2):
        if E % (32 * v) == 0:
            return v
    return 1


def lane_layout(E: int):
    """Column order of each of the 32 lanes: list of 32 integer arrays (columns < E only)."""
    V = lane_vec(E)
    steps = -(-E // (32 * V))
    cols = []
    for lane in range(32):
        c = [j * 32 * V + lane * V + v for j in range(steps) for v in range(V)]
        cols.append(np.array([x for x in c if x < E], dtype=np.int64))
    return cols


def _row_sum_exp(x: np.ndarray, mx: np.ndarray) -> np.ndarray:
    """sum_c exp(x[:, c] - mx) with the CUDA router's association order. x: [T, E] float32."""
    T, E = x.shape
    partial = np.zeros((T, 32), dtype=F32)
    for lane, cols in enumerate(lane_layout(E)):
        s = np.zeros(T, dtype=F32)
        for c in cols:
            s = (s + exp_f32((x[:, c] - mx).astype(F32))).astype(F32)
        partial[:, lane] = s
    off = 16
    while off >= 1:
        partner = np.arange(32) ^ off
        partial = (partial + partial[:, partner]).astype(F32)
        off //= 2
    return partial[:, 0]


def order_key(bits: np.ndarray) -> np.ndarray:
    """uint32 key whose unsigned order is the IEEE total order of the float32 bit patterns."""
    bits = bits.astype(np.uint32)
    neg = (bits >> np.uint32(31)).astype(bool)
    return np.where(neg, ~bits, bits | np.uint32(0x80000000)).astype(np.uint32)


def topk_route(logits, K: int, softmax_over_topk: bool = True, norm_topk_probs: bool = False):
    """Reference router semantics.  logits: [T, E] array of bf16/fp16/fp32 values (as float).

    Returns (scores float32 [T, K], indices int32 [T, K]), both in descending score order.
    """
    x = np.ascontiguousarray(np.asarray(logits, dtype=F32))
    T, E = x.shape
    if norm_topk_probs and softmax_over_topk:
        raise ValueError("norm_topk_probs only applies to top-k over softmax (topk.py:53-54)")
    if not (1 <= K <= E):
        raise ValueError(f"need 1 <= K <= E, got K={K}, E={E}")
    if T == 0:
        return np.zeros((0, K), F32), np.zeros((0, K), np.int32)

    if not softmax_over_topk:
        mx = x.max(axis=1).astype(F32)
        s = _row_sum_exp(x, mx)
        log_norm = (mx + log_f32(s)).astype(F32)
        x = (x - log_norm[:, None]).astype(F32)

    log_n = int(np.log2(next_pow2(E)))
    mask = np.uint32((1 << log_n) - 1)
    col = np.arange(E, dtype=np.uint32)[None, :]
    bits = x.view(np.uint32)
    enc = np.where(x >= 0, (~col) & mask, col & mask).astype(np.uint32)
    bits = ((bits & ~mask) | enc).astype(np.uint32)

    key = order_key(bits)
    order = np.argsort(-key.astype(np.int64), axis=1, kind="stable")[:, :K]
    sel = np.take_along_axis(bits, order, axis=1)
    enc_sel = sel & mask
    vals = (sel & ~mask).astype(np.uint32).view(F32)
    idx = np.where(vals >= 0, (~enc_sel) & mask, enc_sel).astype(np.int32)

    if softmax_over_topk:
        vmax = vals.max(axis=1).astype(F32)
        ex = exp_f32((vals - vmax[:, None]).astype(F32))
        ssum = np.zeros(T, dtype=F32)
        for i in range(K):
            ssum = (ssum + ex[:, i]).astype(F32)
        scores = (ex / ssum[:, None]).astype(F32)
    else:
        scores = exp_f32(vals)
        if norm_topk_probs:
            ssum = np.zeros(T, dtype=F32)
            for i in range(K):
                ssum = (ssum + scores[:, i]).astype(F32)
            scores = (scores / ssum[:, None]).astype(F32)
    return scores.astype(F32), idx


def torch_fallback_route(logits, K: int, softmax_over_topk: bool = True, norm_topk_probs: bool = False):
    """The reference's torch routing (``sonicmoe/functional/forward.py:128-141``), in numpy/torch.

    Used to pin ``topk_route`` on inputs without ties.
    """
    import torch

    lt = torch.as_tensor(np.asarray(logits, dtype=F32))
    if softmax_over_topk:
        r = lt.topk(K, dim=-1)
        vals = r.values.softmax(dim=-1, dtype=torch.float32)
        return vals.numpy(), r.indices.to(torch.int32).numpy()
    probs = lt.softmax(dim=-1, dtype=torch.float32)
    r = probs.topk(K, dim=-1)
    vals = r.values
    if norm_topk_probs:
        vals = vals / vals.sum(dim=-1, keepdim=True)
    return vals.numpy(), r.indices.to(torch.int32).numpy()
