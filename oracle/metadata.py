"""Routing metadata restatement (test infrastructure; see ``oracle/__init__.py``).

``tc_metadata`` follows ``tests/metadata_test.py:17-35`` of the reference
(``_ref_TC_topk_router_metadata``): bincount, exclusive cumsum with ``offset[E] = T*K``,
``s_scatter_idx = argsort(flat, stable=True)``, its inverse, and ``x_gather_idx = s_scatter // K``.
This is also what the reference Triton kernels produce (``triton_kernels/bitmatrix.py:63-147``:
the sort key carries the pre-sort offset, so entries of one expert stay in flat order).

``general_metadata`` follows ``tests/metadata_test.py:38-70`` (``_ref_general_routing_metadata``).

``padded_layout`` is this build's own addition: every expert's rows start on a 128-row boundary
(the GEMM tile height), so a GEMM tile never straddles two experts and the block scale factors
of a tile live in one 512-byte atom.
"""
import numpy as np

BLOCK_M = 128  # rows of one block of the padded layout
PAD_M = 128  # experts are padded to multiples of this


def tc_metadata(topk_indices, E: int):
    idx = np.asarray(topk_indices).astype(np.int64)
    T, K = idx.shape
    TK = T * K
    flat = idx.reshape(-1)
    freq = np.bincount(flat, minlength=E).astype(np.int32)[:E]
    off = np.zeros(E + 1, dtype=np.int32)
    off[1:] = np.cumsum(freq)
    s_scatter = np.argsort(flat, kind="stable").astype(np.int32)
    s_rev = np.empty(TK, dtype=np.int32)
    s_rev[s_scatter] = np.arange(TK, dtype=np.int32)
    x_gather = (s_scatter // max(K, 1)).astype(np.int32)
    return freq, off, x_gather, s_scatter, s_rev


def general_metadata(sorted_token_idx, expert_idx, T: int, E: int):
    tok = np.asarray(sorted_token_idx).astype(np.int64)
    exp_ = np.asarray(expert_idx).astype(np.int64)
    TK = exp_.shape[0]
    freq = np.bincount(exp_, minlength=E).astype(np.int32)[:E]
    off = np.zeros(E + 1, dtype=np.int32)
    off[1:] = np.cumsum(freq)
    s_scatter = np.argsort(exp_, kind="stable").astype(np.int32)
    s_rev = np.empty(TK, dtype=np.int32)
    s_rev[s_scatter] = np.arange(TK, dtype=np.int32)
    x_gather = tok[s_scatter].astype(np.int32)
    counts = np.bincount(tok, minlength=T).astype(np.int32)[:T]
    tok_off = np.zeros(T + 1, dtype=np.int32)
    tok_off[1:] = np.cumsum(counts)
    return freq, off, x_gather, s_scatter, s_rev, tok_off


def padded_layout(freq):
    """Padded expert-major layout: every expert's rows start on a 128-row block and are padded to a
    multiple of PAD_M rows (so an expert always owns whole pairs of blocks).

    Returns (off_pad [E+1] int32 in rows, blk_expert [n_blocks] int32, n_blocks).
    """
    freq = np.asarray(freq).astype(np.int64)
    nblk = (freq + PAD_M - 1) // PAD_M * (PAD_M // BLOCK_M)
    blk_off = np.zeros(len(freq) + 1, dtype=np.int64)
    blk_off[1:] = np.cumsum(nblk)
    blk_expert = np.repeat(np.arange(len(freq), dtype=np.int32), nblk)
    return (blk_off * BLOCK_M).astype(np.int32), blk_expert.astype(np.int32), int(blk_off[-1])


def padded_rows(topk_indices, s_rev, off, off_pad):
    """Padded row of every flat (token, k) entry: s_rev - off[e] + off_pad[e]."""
    e = np.asarray(topk_indices).reshape(-1).astype(np.int64)
    return (np.asarray(s_rev).astype(np.int64) - off[e] + off_pad[e]).astype(np.int64)
