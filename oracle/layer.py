"""MoE layer forward restatements (test infrastructure; see ``oracle/__init__.py``).

``reference_port``  -- the reference's eager torch backend, ``MoE.forward(kernel_backend_moe=torch)``:
    router ``F.linear`` (``sonicmoe/moe.py:280``), ``topk`` (``moe.py:362-368``), fp32 softmax over
    the k values cast back to the input dtype (``moe.py:288-289``), ``sort`` of the flat expert ids
    (``moe.py:303``), ``bincount`` (``moe.py:305``), gather by ``sorted_scattered_idxs // K``
    (``moe.py:339-345``), per-expert ``F.linear`` (``moe.py:144-147``), SwiGLU with even rows =
    gate and odd rows = up (``moe.py:23-26``), gate scaling and ``index_add`` into an fp32
    ``[T, H]`` buffer (``moe.py:354-356``).  Same torch operations in the same order, so on CPU it
    reproduces the reference bit for bit (pinned by ``tests/golden/layer_*.npz``).  It is also the
    timed CPU baseline of ``bench.py``.

``expert_loop``  -- the per-expert reference loop of ``benchmarks/moe-cute.py:204-244``: routing by
    torch top-k, ``swiglu(h, concat_layout)`` (``moe-cute.py:22-27``), ``ref_o[T_idx] += w2_out *
    score``; it covers top-k-over-softmax (+renorm) and the concatenated w1 layout, which the MoE
    module cannot select.  Here it takes the routing as an argument and runs in float64.

``fp8_oracle``  -- ``expert_loop`` on fake-quantised operands: x dequantised from its 1x128 e4m3
    groups, w1/w2 from their 128x128 blocks, the SwiGLU output re-quantised 1x128 and dequantised
    before the down projection (the "reference FP8 path" the north star's 1e-2 bound refers to).

``fp8_oracle_rows``  -- the same math for a subset of tokens, given their routing, quantising only
    the experts they touch: the check at full configuration sizes, where the whole layer on the
    CPU would take hours.
"""
import numpy as np
import torch
import torch.nn.functional as F

from . import quant
from .routing import topk_route


def swiglu_interleaved(h):
    return h[..., 1::2] * F.silu(h[..., ::2])


def reference_port(x, router_w, w1, w2, K: int):
    """Reference eager MoE forward on CPU.  w1: [E, 2I, H] interleaved, w2: [E, H, I]. Returns (o fp32, logits)."""
    T, H = x.shape
    E = w1.shape[0]
    logits = F.linear(x, router_w)
    if K == 1:
        vals, sel = logits.max(dim=-1, keepdim=True)
    else:
        vals, sel = logits.topk(K, dim=-1)
    gates = F.softmax(vals.float(), dim=-1).type_as(x)
    flat = sel.flatten()
    _, sorted_pos = flat.sort()
    freq = flat.bincount(minlength=E).to(torch.int32)
    fan_in = sorted_pos // K
    batch_gates = gates.flatten()[sorted_pos]
    h = x[fan_in].split(freq.tolist(), dim=0)
    h = [F.linear(h[e], w1[e]) for e in range(E)]
    h = [swiglu_interleaved(t) for t in h]
    y = torch.cat([F.linear(h[e], w2[e]) for e in range(E)], dim=0)
    y = y * batch_gates.unsqueeze(-1)
    o = torch.zeros((T, H), dtype=torch.float32, device=x.device).index_add(0, fan_in, y)
    return o, logits, freq


def expert_loop(x, w1, w2, scores, idx, concat_layout: bool, dtype=torch.float64):
    """o[t] = sum_k score[t,k] * w2[e] @ swiglu(w1[e] @ x[t]) with e = idx[t,k] (float64 by default)."""
    x = torch.as_tensor(x).to(dtype)
    w1 = torch.as_tensor(w1).to(dtype)
    w2 = torch.as_tensor(w2).to(dtype)
    scores = torch.as_tensor(np.asarray(scores)).to(dtype)
    idx = torch.as_tensor(np.asarray(idx)).long()
    T, H = x.shape
    E, N2, _ = w1.shape
    I = N2 // 2
    o = torch.zeros((T, H), dtype=dtype)
    for e in range(E):
        t_idx, k_idx = torch.nonzero(idx == e, as_tuple=True)
        if t_idx.numel() == 0:
            continue
        h = x[t_idx] @ w1[e].T
        if concat_layout:
            a = F.silu(h[:, :I]) * h[:, I:]
        else:
            a = swiglu_interleaved(h)
        y = a @ w2[e].T
        o.index_add_(0, t_idx, y * scores[t_idx, k_idx, None])
    return o


def fp8_oracle(x, logits, w1, w2, K: int, softmax_over_topk=True, norm_topk_probs=False, concat_layout=False):
    """Fake-quantised FP8 layer: returns (o float64 [T,H], scores, idx).

    x: [T, H] activations (the bf16 values as float32), w1: [E, 2I, H] in the caller's layout
    (interleaved or concatenated), w2: [E, H, I], logits: [T, E] (bf16 values as float32).
    """
    x = np.asarray(x, dtype=np.float32)
    w1 = np.asarray(w1, dtype=np.float32)
    w2 = np.asarray(w2, dtype=np.float32)
    scores, idx = topk_route(logits, K, softmax_over_topk, norm_topk_probs)
    xq, xs = quant.quant_1x128(x)
    xd = quant.dequant_1x128(xq, xs)
    w1q, w1s = quant.quant_128x128(w1)
    w1d = quant.dequant_128x128(w1q, w1s)
    w2q, w2s = quant.quant_128x128(w2)
    w2d = quant.dequant_128x128(w2q, w2s)

    xt = torch.as_tensor(xd).double()
    w1t = torch.as_tensor(w1d).double()
    w2t = torch.as_tensor(w2d).double()
    T, H = x.shape
    E, N2, _ = w1.shape
    I = N2 // 2
    idx_t = torch.as_tensor(idx).long()
    sc_t = torch.as_tensor(scores).double()
    o = torch.zeros((T, H), dtype=torch.float64)
    for e in range(E):
        t_idx, k_idx = torch.nonzero(idx_t == e, as_tuple=True)
        if t_idx.numel() == 0:
            continue
        h = xt[t_idx] @ w1t[e].T
        if concat_layout:
            a = F.silu(h[:, :I]) * h[:, I:]
        else:
            a = swiglu_interleaved(h)
        aq, as_ = quant.quant_1x128(a.float().numpy())
        ad = torch.as_tensor(quant.dequant_1x128(aq, as_)).double()
        y = ad @ w2t[e].T
        o.index_add_(0, t_idx, y * sc_t[t_idx, k_idx, None])
    return o, scores, idx


def fp8_general_oracle(x, router_scores, token_idx, expert_idx, w1, w2, concat_layout=False):
    """Fake-quantised FP8 layer for explicit routing lists (``moe_general_routing_inputs``,
    reference functional/__init__.py:571-652): o[t] = sum over entries f with token t of
    score[f] * W2q[e] requant(swiglu(W1q[e] xq[t])), e = expert_idx[f]."""
    x = np.asarray(x, dtype=np.float32)
    w1 = np.asarray(w1, dtype=np.float32)
    w2 = np.asarray(w2, dtype=np.float32)
    xq, xs = quant.quant_1x128(x)
    xt = torch.as_tensor(quant.dequant_1x128(xq, xs)).double()
    w1q, w1s = quant.quant_128x128(w1)
    w1t = torch.as_tensor(quant.dequant_128x128(w1q, w1s)).double()
    w2q, w2s = quant.quant_128x128(w2)
    w2t = torch.as_tensor(quant.dequant_128x128(w2q, w2s)).double()
    T, H = x.shape
    E, N2, _ = w1.shape
    I = N2 // 2
    tok = torch.as_tensor(np.asarray(token_idx)).long()
    exp_ = torch.as_tensor(np.asarray(expert_idx)).long()
    sc = torch.as_tensor(np.asarray(router_scores, dtype=np.float32)).double()
    o = torch.zeros((T, H), dtype=torch.float64)
    for e in range(E):
        sel = torch.nonzero(exp_ == e, as_tuple=True)[0]
        if sel.numel() == 0:
            continue
        h = xt[tok[sel]] @ w1t[e].T
        a = F.silu(h[:, :I]) * h[:, I:] if concat_layout else swiglu_interleaved(h)
        aq, as_ = quant.quant_1x128(a.float().numpy())
        ad = torch.as_tensor(quant.dequant_1x128(aq, as_)).double()
        o.index_add_(0, tok[sel], (ad @ w2t[e].T) * sc[sel, None])
    return o


def fp8_oracle_rows(x_rows, scores_rows, idx_rows, expert_weights, concat_layout=False):
    """Fake-quantised FP8 layer output [n, H] (float64) of n tokens.

    x_rows: [n, H] activations (bf16 values as float32); scores_rows / idx_rows: [n, K] routing of
    those tokens (K may be ragged by padding idx with -1); expert_weights(e) -> (w1_e [2I, H],
    w2_e [H, I]) float32 in the caller's layout.  Each touched expert is quantised once with the
    same 128x128 blocks as the whole-layer oracle (through ``quant.fake_quant_128x128_fast``, which
    is pinned bit for bit to the spec path), so per row the result equals ``fp8_oracle``'s.
    """
    x_rows = np.asarray(x_rows, dtype=np.float32)
    idx_rows = np.asarray(idx_rows)
    scores_rows = np.asarray(scores_rows, dtype=np.float32)
    xq, xs = quant.quant_1x128(x_rows)
    xt = torch.as_tensor(quant.dequant_1x128(xq, xs)).double()
    n, H = x_rows.shape
    o = torch.zeros((n, H), dtype=torch.float64)
    for e in np.unique(idx_rows[idx_rows >= 0]):
        w1e, w2e = expert_weights(int(e))
        w1e = np.asarray(w1e, dtype=np.float32)[None]
        w2e = np.asarray(w2e, dtype=np.float32)[None]
        w1t = torch.as_tensor(quant.fake_quant_128x128_fast(w1e)[0]).double()
        w2t = torch.as_tensor(quant.fake_quant_128x128_fast(w2e)[0]).double()
        I = w1t.shape[0] // 2
        t_idx, k_idx = np.nonzero(idx_rows == e)
        t_idx = torch.as_tensor(t_idx).long()
        h = xt[t_idx] @ w1t.T
        a = F.silu(h[:, :I]) * h[:, I:] if concat_layout else swiglu_interleaved(h)
        aq, as_ = quant.quant_1x128(a.float().numpy())
        ad = torch.as_tensor(quant.dequant_1x128(aq, as_)).double()
        sc = torch.as_tensor(scores_rows[t_idx.numpy(), k_idx]).double()
        o.index_add_(0, t_idx, (ad @ w2t.T) * sc[:, None])
    return o


def rel_fro(a, b) -> float:
    """||a - b||_F / ||b||_F in float64."""
    a = torch.as_tensor(np.asarray(a, dtype=np.float64)) if not torch.is_tensor(a) else a.double()
    b = torch.as_tensor(np.asarray(b, dtype=np.float64)) if not torch.is_tensor(b) else b.double()
    den = torch.linalg.norm(b).item()
    return torch.linalg.norm(a - b).item() / (den if den > 0 else 1.0)
