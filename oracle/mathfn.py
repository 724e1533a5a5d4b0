"""Float32 exp / log with a fixed sequence of IEEE single operations (test infrastructure).

The CUDA router (``sonic-moe_b200/csrc/router.cu``) evaluates the same formulas with
``__fmul_rn`` / ``__fadd_rn`` / ``__fdiv_rn`` (no FMA contraction, no flush-to-zero), so every
intermediate is the correctly rounded single-precision result on both sides and the outputs
agree bit for bit.  numpy float32 arithmetic is IEEE single with round-to-nearest-even.

exp: Cody-Waite range reduction x = n*ln2 + r (ln2 split into a 16-bit head and a tail) and the
degree-7 Taylor polynomial of e^r evaluated by Horner's rule; e^x = p(r) * 2^n.
log: s = m * 2^e with m in [sqrt(1/2), sqrt(2)); log m = 2*atanh(f/(2+f)), f = m - 1, with the
atanh series to the z^11 term; log s = e*ln2_hi + (log m + e*ln2_lo).

Both are written from the mathematics above (no library constants beyond ln2, log2(e), sqrt(2)
and 1/k!); they are accurate to a few ulp on the domain the router uses (x <= 0 for exp,
s >= 1 for log).
"""
import numpy as np

F32 = np.float32

LOG2E = F32(1.4426950408889634)
LN2_HI = F32(0.693145751953125)  # 0x3F317200: low 9 mantissa bits zero -> n*LN2_HI exact
LN2_LO = F32(0.6931471805599453 - 0.693145751953125)
SQRT2 = F32(1.4142135623730951)
# 1/k! for k = 7..2, then 1, 1
EXP_C = [F32(1.0 / 5040.0), F32(1.0 / 720.0), F32(1.0 / 120.0), F32(1.0 / 24.0), F32(1.0 / 6.0), F32(0.5)]
# 2/(2k+1) for k = 5..0
LOG_C = [F32(2.0 / 11.0), F32(2.0 / 9.0), F32(2.0 / 7.0), F32(2.0 / 5.0), F32(2.0 / 3.0), F32(2.0)]


def exp_f32(x):
    """e^x in float32 (array in, array out).  0 below 2^-126 range, +inf above 2^127."""
    x = np.asarray(x, dtype=F32)
    with np.errstate(invalid="ignore", over="ignore", under="ignore"):
        t = x * LOG2E
        nf = np.rint(t).astype(F32)
        r = (x - nf * LN2_HI).astype(F32)
        r = (r - nf * LN2_LO).astype(F32)
        p = EXP_C[0]
        for c in EXP_C[1:]:
            p = (p * r).astype(F32)
            p = (p + c).astype(F32)
        for _ in range(2):  # the 1/1! and 1/0! terms
            p = (p * r).astype(F32)
            p = (p + F32(1.0)).astype(F32)
        n_clip = np.clip(np.nan_to_num(nf, nan=0.0), -126, 127).astype(np.int32)
        scale = ((n_clip + 127).astype(np.uint32) << np.uint32(23)).view(F32)
        out = (p * scale).astype(F32)
        out = np.where(nf < F32(-126.0), F32(0.0), out)
        out = np.where(nf > F32(127.0), F32(np.inf), out)
        out = np.where(np.isnan(x), x, out)
    return out.astype(F32)


def log_f32(s):
    """Natural log in float32 for positive normal inputs (array in, array out)."""
    s = np.asarray(s, dtype=F32)
    bits = s.view(np.uint32)
    e = ((bits >> np.uint32(23)) & np.uint32(0xFF)).astype(np.int32) - 127
    m = ((bits & np.uint32(0x7FFFFF)) | np.uint32(0x3F800000)).view(F32)
    big = m > SQRT2
    m = np.where(big, (m * F32(0.5)).astype(F32), m).astype(F32)
    e = np.where(big, e + 1, e)
    f = (m - F32(1.0)).astype(F32)
    z = (f / (F32(2.0) + f).astype(F32)).astype(F32)
    w = (z * z).astype(F32)
    p = LOG_C[0]
    for c in LOG_C[1:]:
        p = (p * w).astype(F32)
        p = (p + c).astype(F32)
    logm = (z * p).astype(F32)
    ef = e.astype(F32)
    t = (logm + (ef * LN2_LO).astype(F32)).astype(F32)
    out = ((ef * LN2_HI).astype(F32) + t).astype(F32)
    return out
