"""FP8 e4m3 block quantiser specification (test infrastructure; see ``oracle/__init__.py``).

PARITY UNPINNED: the reference has no FP8 quantiser (its only "quantization" string is the
autotuner bucketing comment at ``sonicmoe/functional/__init__.py:104``), so this module is the
specification the CUDA quantiser is held to, bit for bit.  It is cross-checked against torch's
``float8_e4m3fn`` conversion in ``tests/test_oracle_quant.py``.

Spec (one group = 1x128 activation values along K, or a 128x128 weight block):

1. ``amax = max |x|`` in float32 (inputs are bf16, so this is exact).
2. ``s = amax / 448`` (float32, IEEE round-to-nearest-even division).
3. ``e = ceil(log2(s))`` taken exactly from the bits of ``s`` (subnormal ``s`` included), clamped
   to ``[-127, 127]``; ``amax == 0`` gives ``e = -127``.  The scale is ``2^e`` and is stored as
   one UE8M0 byte ``e + 127`` -- the scale format the tcgen05 block-scaled MMA consumes.
4. ``q = e4m3(x * 2^-e)``: round to nearest even, saturating to +-448 (the multiply is exact).

Dequantised value: ``float(q) * 2^e``.

Scale-factor storage ("SF atoms").  A 512-byte atom holds the UE8M0 bytes of 128 rows x 4
consecutive 128-wide K blocks; byte ``16*(r % 32) + 4*((r % 128) // 32) + (kb % 4)`` belongs to row
``r`` and K block ``kb``.  That is the per-lane order in which ``tcgen05.cp ... 32x128b.warpx4``
places scale factors into tensor memory (lane ``r % 32``, column ``(r % 128) // 32``, byte = K block),
and the MMA selects the byte with its scale-factor id.  Activation atoms are indexed
``[row // 128][kb // 4]``; weight atoms ``[expert][n // 128][kb // 4]`` with every row of a 128-row
block holding the block's scale.
"""
import numpy as np

F32 = np.float32
E4M3_MAX = 448.0


def ceil_log2_f32(s: np.ndarray) -> np.ndarray:
    """Exact ceil(log2(s)) for non-negative float32 s (s == 0 -> -127), clamped to [-127, 127]."""
    s = np.asarray(s, dtype=F32)
    bits = s.view(np.uint32).astype(np.int64)
    ex = (bits >> 23) & 0xFF
    man = bits & 0x7FFFFF
    normal = ex > 0
    e_norm = np.where(man == 0, ex - 127, ex - 126)
    # subnormal: s = man * 2^-149 -> ceil(log2 man) - 149
    man_c = np.maximum(man, 1)
    ceil_l2 = np.ceil(np.log2(man_c.astype(np.float64))).astype(np.int64)
    # log2 of a power of two is exact in float64, so ceil is exact for integers < 2^23
    e_sub = ceil_l2 - 149
    e = np.where(normal, e_norm, np.where(man == 0, -127, e_sub))
    return np.clip(e, -127, 127).astype(np.int32)


def e4m3_encode(v) -> np.ndarray:
    """float32 -> e4m3fn bit patterns (uint8), round-to-nearest-even, saturating at +-448."""
    v = np.asarray(v, dtype=np.float64)
    sign = (np.signbit(v)).astype(np.uint8) << 7
    a = np.abs(v)
    code = np.zeros(a.shape, dtype=np.int64)
    sub = a < 2.0 ** -6
    code_sub = np.rint(a / 2.0 ** -9).astype(np.int64)  # 0..8; 8 == smallest normal, code 0x08
    with np.errstate(divide="ignore"):
        ex = np.floor(np.log2(np.where(sub, 1.0, a))).astype(np.int64)
    m = np.rint(a / np.exp2(ex - 3)).astype(np.int64)  # 8..16
    carry = m >= 16
    ex = np.where(carry, ex + 1, ex)
    m = np.where(carry, 8, m)
    code_norm = ((ex + 7) << 3) | (m - 8)
    code = np.where(sub, code_sub, code_norm)
    code = np.where(a >= E4M3_MAX, 0x7E, code)
    code = np.minimum(code, 0x7E)
    return (code.astype(np.uint8) | sign).astype(np.uint8)


def e4m3_decode(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    ex = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(ex == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(ex - 7))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (sign * val).astype(F32)


def quant_groups(x: np.ndarray):
    """Quantise the last axis (length 128) of x as one group.  Returns (q uint8 [...,128], e8m0 uint8 [...])."""
    x = np.asarray(x, dtype=F32)
    amax = np.abs(x).max(axis=-1).astype(F32)
    s = (amax / F32(E4M3_MAX)).astype(F32)
    e = ceil_log2_f32(s)
    inv = np.exp2(-e.astype(np.float64)).astype(F32)  # exact power of two
    q = e4m3_encode((x * inv[..., None]).astype(F32))
    return q, (e + 127).astype(np.uint8)


def quant_1x128(x: np.ndarray):
    """Activation quantiser: x [R, C] (C % 128 == 0) -> (q [R, C] uint8, e8m0 [R, C//128] uint8)."""
    x = np.asarray(x, dtype=F32)
    R, C = x.shape
    assert C % 128 == 0, "K must be a multiple of 128"
    q, sf = quant_groups(x.reshape(R, C // 128, 128))
    return q.reshape(R, C), sf


def dequant_1x128(q: np.ndarray, sf: np.ndarray) -> np.ndarray:
    R, C = q.shape
    v = e4m3_decode(q).reshape(R, C // 128, 128).astype(np.float64)
    sc = np.exp2(sf.astype(np.float64) - 127.0)
    return (v * sc[..., None]).reshape(R, C).astype(F32)


def quant_128x128(w: np.ndarray):
    """Weight quantiser: w [E, N, K] (N, K % 128 == 0) -> (q [E,N,K] uint8, e8m0 [E, N//128, K//128])."""
    w = np.asarray(w, dtype=F32)
    E, N, K = w.shape
    assert N % 128 == 0 and K % 128 == 0
    blocks = w.reshape(E, N // 128, 128, K // 128, 128).transpose(0, 1, 3, 2, 4).reshape(E, N // 128, K // 128, 128 * 128)
    qb, sf = quant_groups(blocks)
    q = qb.reshape(E, N // 128, K // 128, 128, 128).transpose(0, 1, 3, 2, 4).reshape(E, N, K)
    return q, sf


def dequant_128x128(q: np.ndarray, sf: np.ndarray) -> np.ndarray:
    E, N, K = q.shape
    v = e4m3_decode(q).astype(np.float64)
    sc = np.exp2(sf.astype(np.float64) - 127.0)
    sc_full = np.repeat(np.repeat(sc, 128, axis=1), 128, axis=2)
    return (v * sc_full).astype(F32)


def concat_to_blocked(w1: np.ndarray) -> np.ndarray:
    """Concatenated SwiGLU weight [E, 2I, H] ([gate; up]) -> 128-row blocked [g0, u0, g1, u1, ...].

    Block j of the result holds gate rows [128j, 128j+128) followed by up rows [I+128j, I+128j+128).
    The 128x128 scale blocks of the concatenated layout map one-to-one onto the blocked layout.
    """
    E, N2, H = w1.shape
    I = N2 // 2
    g = w1[:, :I].reshape(E, I // 128, 128, H)
    u = w1[:, I:].reshape(E, I // 128, 128, H)
    return np.stack([g, u], axis=2).reshape(E, N2, H)


def act_sf_atoms(sf: np.ndarray) -> np.ndarray:
    """Per-row e8m0 [R, G] -> SF atoms [ceil(R/128), ceil(G/4), 512] (zero-filled)."""
    R, G = sf.shape
    MB, KG = -(-R // 128), -(-G // 4)
    out = np.zeros((MB, KG, 512), dtype=np.uint8)
    r = np.arange(R)[:, None]
    g = np.arange(G)[None, :]
    byte = 16 * (r % 32) + 4 * ((r % 128) // 32) + (g % 4)
    out[(r // 128).repeat(G, 1), (g // 4).repeat(R, 0), byte] = sf
    return out


def weight_sf_atoms(sf: np.ndarray) -> np.ndarray:
    """Per-block e8m0 [E, NB, G] -> SF atoms [E, NB, ceil(G/4), 512]."""
    E, NB, G = sf.shape
    KG = -(-G // 4)
    out = np.zeros((E, NB, KG, 512), dtype=np.uint8)
    for g in range(G):
        for lane in range(32):
            for c in range(4):
                out[:, :, g // 4, 16 * lane + 4 * c + (g % 4)] = sf[:, :, g]
    return out


def fake_quant_128x128_fast(w: np.ndarray) -> np.ndarray:
    """Dequantised 128x128-block e4m3 weights, ``dequant_128x128(*quant_128x128(w))``, computed
    with torch's ``float8_e4m3fn`` conversion (IEEE round to nearest even) instead of the
    element-by-element encoder above, for the full-size parity tests (tens of millions of values
    per expert).  The scale step is the spec's own (``ceil_log2_f32`` of the float32 quotient
    amax / 448), and every scaled value lies in [-448, 448], where torch's conversion needs no
    saturation; ``tests/test_oracle.py`` pins the result bit for bit against the spec path."""
    import torch

    wt = torch.as_tensor(np.asarray(w, dtype=F32))
    E, N, K = wt.shape
    assert N % 128 == 0 and K % 128 == 0
    blocks = wt.view(E, N // 128, 128, K // 128, 128)
    amax = blocks.abs().amax(dim=(2, 4))  # [E, N/128, K/128], exact
    e = torch.from_numpy(ceil_log2_f32((amax.numpy() / F32(E4M3_MAX)).astype(F32)).astype(np.float32))
    inv = torch.exp2(-e)[:, :, None, :, None]  # exact powers of two
    q = (blocks * inv).to(torch.float8_e4m3fn).to(torch.float32)
    return (q * torch.exp2(e)[:, :, None, :, None]).reshape(E, N, K).numpy()
