"""Backward of the FP8 layer, restated on the CPU (test infrastructure; see ``oracle/__init__.py``).

The reference's backward (``sonicmoe/functional/backward.py`` and the autograd functions of
``sonicmoe/functional/__init__.py:174-202, 227-479``) for the bias-free SwiGLU layer with
interleaved w1, in float64, with the operands of each GEMM fake-quantised where the engine
quantises them:

* ``dA'[r] = q1x128(dO)[t_r] W2q[e_r]``      (down-projection backward, ``gemm_dact`` at
  ``backward.py:211-278``; ``W2q`` the forward's 128x128-block e4m3 weight)
* ``a = silu(g) u`` from the bf16 pre-activation ``h``, ``dS[r] = <dA'[r], a>``,
  ``a'[r] = s_r a``, ``dg = s_r dA' u silu'(g)``, ``du = s_r dA' silu(g)``
* ``dx[t] = sum_k q1x128(bf16(dH))[r] W1q[e_r]``    (``gemm`` + ``token_broadcast_backward``,
  ``backward.py:173-206, 281-305``)
* ``dW2[e] = qcol(dO rows)^T qcol(a')``, ``dW1[e] = qcol(dH)^T qcol(x rows)`` over the expert's rows
  of the padded layout, ``qcol`` = one UE8M0 scale per 128 consecutive padded rows of a column, the
  operands rounded to bf16 first (the varlen-K ``gemm`` calls, ``__init__.py:339-348, 465-473``)
* router: ``dlogits`` from ``dS`` (``backward.py:308-430``: softmax over the top-k, or top-k of the
  softmax, optionally renormalised).
"""
import numpy as np
import torch

from . import metadata, quant


def _bf16(a: np.ndarray) -> np.ndarray:
    return torch.as_tensor(np.asarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def _q1x128(a: np.ndarray) -> np.ndarray:
    q, s = quant.quant_1x128(np.asarray(a, dtype=np.float32))
    return quant.dequant_1x128(q, s).astype(np.float64)


def router_backward(logits, scores, idx, ds, softmax_over_topk=True, norm_topk_probs=False):
    """dlogits [T, E] (float64) of the router from the scores' gradient ds [T, K]."""
    lg = np.asarray(logits, dtype=np.float64)
    T, E = lg.shape
    s = np.asarray(scores, dtype=np.float64)
    g = np.asarray(ds, dtype=np.float64)
    idx = np.asarray(idx)
    dl = np.zeros((T, E))
    rows = np.arange(T)[:, None]
    if softmax_over_topk:
        dot = (g * s).sum(1, keepdims=True)
        dl[rows, idx] = s * (g - dot)
        return dl
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    p_sel = p[rows, idx]
    dp_sel = (g - (g * s).sum(1, keepdims=True)) / p_sel.sum(1, keepdims=True) if norm_topk_probs else g
    dot = (dp_sel * p_sel).sum(1, keepdims=True)
    dp = np.zeros((T, E))
    dp[rows, idx] = dp_sel
    return p * (dp - dot)


def _fp8_backward_entries(x, dout, w1, w2, tok, e, s, meta, h, concat_layout):
    """Expert part of the backward over explicit entries (token tok[f], expert e[f], score s[f])."""
    T, H = x.shape
    E, N2, _ = np.asarray(w1).shape
    I = N2 // 2
    freq, off, s_rev = meta
    off_pad, _, nblk = metadata.padded_layout(freq)
    prow = (np.asarray(s_rev).astype(np.int64) - off[e] + off_pad[e]).astype(np.int64)  # padded row of entry f
    w1d = quant.dequant_128x128(*quant.quant_128x128(np.asarray(w1, dtype=np.float32))).astype(np.float64)
    w2d = quant.dequant_128x128(*quant.quant_128x128(np.asarray(w2, dtype=np.float32))).astype(np.float64)
    TK = tok.shape[0]
    # h rows are in expert-sorted order: entry f sits at row s_rev[f]
    hf = np.asarray(h, dtype=np.float64)[s_rev]
    g, u = (hf[:, :I], hf[:, I:]) if concat_layout else (hf[:, 0::2], hf[:, 1::2])
    sig = 1.0 / (1.0 + np.exp(-g))
    a = g * sig * u
    dod = _q1x128(dout)
    dap = np.zeros((TK, I))
    for ex in np.unique(e):
        r = np.nonzero(e == ex)[0]
        dap[r] = dod[tok[r]] @ w2d[ex]
    ds = (dap * a).sum(1)
    da = s[:, None] * dap
    dg, du = da * u * sig * (1.0 + g * (1.0 - sig)), da * g * sig
    dh = np.empty((TK, 2 * I))
    if concat_layout:
        dh[:, :I], dh[:, I:] = dg, du
    else:
        dh[:, 0::2], dh[:, 1::2] = dg, du
    a_prime = s[:, None] * a
    dhq = _q1x128(_bf16(dh))  # the dX GEMM's e4m3 dH is quantised from the bf16 dH
    dx = np.zeros((T, H))
    for ex in np.unique(e):
        r = np.nonzero(e == ex)[0]
        np.add.at(dx, tok[r], dhq[r] @ w1d[ex])
    rows_pad = int(nblk) * 128

    def colq(rows_vals, C):
        p = np.zeros((rows_pad, C), dtype=np.float32)
        p[prow] = _bf16(rows_vals)
        return _q1x128(p.T)  # [C, rows_pad]: 1x128 groups along the padded rows

    dot_ = colq(dout[tok], H)
    apt = colq(a_prime, I)
    dht = colq(dh, 2 * I)
    xt = colq(x[tok], H)
    dw2 = np.zeros((E, H, I))
    dw1 = np.zeros((E, 2 * I, H))
    for ex in range(E):
        c0, c1 = int(off_pad[ex]), int(off_pad[ex + 1])
        if c1 > c0:
            dw2[ex] = dot_[:, c0:c1] @ apt[:, c0:c1].T
            dw1[ex] = dht[:, c0:c1] @ xt[:, c0:c1].T
    return dx, dw1, dw2, ds


def fp8_backward(x, dout, w1, w2, scores, idx, h, softmax_over_topk=True, norm_topk_probs=False, logits=None,
                 concat_layout=False):
    """(dx [T, H], dw1 [E, 2I, H], dw2 [E, H, I], ds [T, K], dlogits [T, E] or None), float64.

    x, dout [T, H]; w1 [E, 2I, H], w2 [E, H, I] (bf16 values as float); scores / idx [T, K] the
    forward's routing; h [T*K, 2I] the stored pre-activation in expert-sorted entry order.  With
    concat_layout the gate / up halves of w1, h and dH are [gate | up] instead of interleaved; dH's 1x128
    groups along 2I are then gate-only and up-only groups, as in the engine."""
    x = np.asarray(x, dtype=np.float32)
    dout = np.asarray(dout, dtype=np.float32)
    idx = np.asarray(idx)
    T, K = idx.shape
    E = np.asarray(w1).shape[0]
    freq, off, _, _, s_rev = metadata.tc_metadata(idx, E)
    tok = np.arange(T * K) // K
    e = idx.reshape(-1).astype(np.int64)
    s = np.asarray(scores, dtype=np.float64).reshape(-1)
    dx, dw1, dw2, ds = _fp8_backward_entries(x, dout, w1, w2, tok, e, s, (freq, off, s_rev), h, concat_layout)
    ds = ds.reshape(T, K)
    dl = None if logits is None else router_backward(logits, scores, idx, ds, softmax_over_topk, norm_topk_probs)
    return dx, dw1, dw2, ds, dl


def fp8_backward_general(x, dout, w1, w2, router_scores, token_idx, expert_idx, h, concat_layout=False):
    """(dx [T, H], dw1, dw2, d router_scores [TK]), float64, of the layer over explicit entries
    (``moe_general_routing_inputs``; token_idx sorted ascending); h [TK, 2I] in expert-sorted order."""
    x = np.asarray(x, dtype=np.float32)
    dout = np.asarray(dout, dtype=np.float32)
    T = x.shape[0]
    E = np.asarray(w1).shape[0]
    tok = np.asarray(token_idx).astype(np.int64)
    e = np.asarray(expert_idx).astype(np.int64)
    freq, off, _, _, s_rev, _ = metadata.general_metadata(tok, e, T, E)
    s = np.asarray(router_scores, dtype=np.float64)
    return _fp8_backward_entries(x, dout, w1, w2, tok, e, s, (freq, off, s_rev), h, concat_layout)
