"""CPU oracle for the fused FP8 quant+GEMV decode path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only to check or to time the CPU reference path.  The product
(``fp8gq``) never imports it and has no CPU fallback.

It restates, in numpy (byte / integer work and fp32 scalar arithmetic) and in
torch-on-CPU (the timed reference path), the algorithm of
wafik/sglang-triton-fusion:

* activation group quant -- ``kernels/fused_gemv_quant.py:35-43`` (the inline
  copy of sglang ``fp8_kernel.py:170-173``), repeated in
  ``kernels/fused_gemv_quant_tm.py:38-41`` (M==1) and ``:65-70`` (TM rows):
  ``amax = max(max|x|, 1e-10)``; ``sx = amax / 448``;
  ``xq = e4m3_rne(clamp(x * (1 / sx), -448, 448))``.
* block-scaled weight dequant -- ``benchmarks/bench_sglang_fp8.py:54-55``:
  ``Wq.float() * Ws.repeat_interleave(128, 0).repeat_interleave(128, 1)``.
* the contraction -- ``kernels/fused_gemv_quant_tm.py:44-46`` /
  ``:74-77``: ``out[m, n] = sum_b (sum_{k in b} xq[m,k] W[n,k]) * sx[m,b] * Ws[n/128, b]``
  stored as bf16.
* SwiGLU prologue -- ``kernels/fused_swiglu_quant_gemv.py:38-46``:
  ``act = g * sigmoid(g) * u`` in fp32 on the ``[gate | up]`` halves, then
  the same group quant on the fp32 act (not a bf16-rounded act).

Parity is pinned by ``tests/golden/`` (fixtures produced by running the
reference's own Triton kernels in Triton's CPU interpreter; see
``tests/golden/make_golden.py``) and by the known-answer cases of
``benchmarks/stress_tests.py:148-199``.

Arithmetic conventions (these are what "bit-exact" means for this path):

* every fp32 operation is one IEEE-754 binary32 operation rounded to nearest
  even; no fused multiply-add is used anywhere the bytes depend on it;
* ``sx = amax / 448`` is an IEEE division and ``1 / sx`` an IEEE reciprocal
  (sglang's formula as evaluated by torch; Triton's GPU ``/`` is an
  approximate division, which is why the torch restatement, not the Triton
  kernel, is the bit-level target);
* fp32 -> e4m3fn is round-to-nearest-even on a value already clamped to
  [-448, 448]; the sign of a value that rounds to zero is kept (0x80), which
  is what ``torch.Tensor.to(torch.float8_e4m3fn)`` does;
* ``sigmoid(g) = 1 / (1 + exp(-g))`` with ``exp`` evaluated by
  :func:`exp_f32` (Cody-Waite reduction + Cephes ``expf`` minimax polynomial,
  every step an explicit fp32 multiply or add), so the CUDA kernels can run
  the identical sequence and the SwiGLU quant bytes are reproducible bit for
  bit on both sides.
"""
from __future__ import annotations

import numpy as np

GROUP = 128                      # 1x128 activation groups, 128x128 weight blocks
E4M3_MAX = np.float32(448.0)     # largest finite e4m3fn value
EPS = np.float32(1e-10)          # amax floor, kernels/fused_gemv_quant_tm.py:144

_F32 = np.float32


# --------------------------------------------------------------------------
# e4m3fn and bf16 codecs (written from the format definitions)
# --------------------------------------------------------------------------

def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    """e4m3fn byte -> float32.  1 sign, 4 exponent (bias 7), 3 mantissa bits;
    exponent 0 is subnormal (m * 2^-9); 0x7F / 0xFF are NaN; no infinities."""
    c = np.asarray(codes, dtype=np.uint8).astype(np.int32)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    mag = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    out = (sign * mag).astype(np.float32)
    out[(c & 0x7F) == 0x7F] = np.nan
    return out


E4M3_TABLE = e4m3_decode(np.arange(256, dtype=np.uint8))


def e4m3_encode_rne(y: np.ndarray) -> np.ndarray:
    """float32 in [-448, 448] -> e4m3fn byte, round to nearest, ties to even.

    Subnormal range (|y| < 2^-6): the code is rint(|y| * 2^9), which runs
    continuously into the first normal code 0x08.  Normal range: round the
    fp32 significand to 3 bits (RNE, carry allowed into the exponent) and
    rebias the exponent from 127 to 7.  The sign bit is copied, so values that
    round to zero keep their sign.
    """
    y = np.asarray(y, dtype=np.float32)
    if np.any(~np.isfinite(y)) or np.any(np.abs(y) > E4M3_MAX):
        raise ValueError("e4m3_encode_rne expects finite values clamped to +-448")
    bits = y.view(np.uint32)
    sign = ((bits >> 24) & 0x80).astype(np.uint8)
    mag_bits = bits & np.uint32(0x7FFFFFFF)
    a = mag_bits.view(np.float32)
    sub = a < _F32(2.0 ** -6)
    # subnormal: exact scaling by a power of two, then RNE to an integer
    code_sub = np.rint(a * _F32(512.0)).astype(np.int64)
    # normal: RNE of the 23-bit fraction down to 3 bits on the raw bits
    mb = mag_bits.astype(np.int64)
    rounded = (mb + 0x7FFFF + ((mb >> 20) & 1)) >> 20
    code_norm = rounded - ((127 - 7) << 3)
    code = np.where(sub, code_sub, code_norm).astype(np.uint8)
    return code | sign


def bf16_round(y: np.ndarray) -> np.ndarray:
    """float32 -> bf16 (RNE) returned as float32 values."""
    bits = np.asarray(y, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(np.asarray(y, dtype=np.float32))
    if np.any(nan):
        out = out.copy()
        out[nan] = np.nan
    return out


def bf16_bits(y: np.ndarray) -> np.ndarray:
    """float32 values that are already bf16 -> uint16 bit patterns."""
    return (np.asarray(y, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------
# activation group quant (kernels/fused_gemv_quant.py:35-43)
# --------------------------------------------------------------------------

def group_quant(x: np.ndarray):
    """x: float32 [M, K] (bf16 values), K % 128 == 0.

    Returns (xq uint8 [M, K], sx float32 [M, K/128]).
    Mirrors kernels/fused_gemv_quant.py:40-43 step by step."""
    x = np.asarray(x, dtype=np.float32)
    M, K = x.shape
    if K % GROUP:
        raise ValueError("K must be a multiple of 128")
    g = x.reshape(M, K // GROUP, GROUP)
    absmax = np.maximum(np.abs(g).max(axis=-1), EPS)          # :40
    sx = (absmax / E4M3_MAX).astype(np.float32)               # :41
    sinv = (_F32(1.0) / sx).astype(np.float32)                # :42
    y = (g * sinv[..., None]).astype(np.float32)              # :43
    y = np.clip(y, -E4M3_MAX, E4M3_MAX)
    xq = e4m3_encode_rne(y).reshape(M, K)
    return xq, sx


# --------------------------------------------------------------------------
# SwiGLU prologue (kernels/fused_swiglu_quant_gemv.py:40-42)
# --------------------------------------------------------------------------

# Cody-Waite split of ln 2 and the degree-5 minimax polynomial for
# (e^r - 1 - r) / r^2 on |r| <= ln2/2, as published in the Cephes math
# library (S. L. Moshier, expf.c).
_LOG2E = _F32(1.44269504088896341)
_C1 = _F32(0.693359375)
_C2 = _F32(-2.12194440e-4)
_P = [_F32(1.9875691500e-4), _F32(1.3981999507e-3), _F32(8.3334519073e-3),
      _F32(4.1665795894e-2), _F32(1.6666665459e-1), _F32(5.0000001201e-1)]
EXP_HI = _F32(88.0)    # exp(x) for x > 88 is returned as +inf
EXP_LO = _F32(-88.0)   # exp(x) for x < -88 is returned as 0


def exp_f32(x: np.ndarray) -> np.ndarray:
    """exp in fp32 by an explicit sequence of fp32 multiplies and adds.

    n = rint(x * log2 e); r = (x - n*C1) - n*C2; p = 1 + r + r^2 * P(r);
    result = p * 2^n (two power-of-two factors so 2^n never leaves the normal
    range).  Accurate to about 1 ulp on [-88, 88] (checked against float64
    in the tests); the CUDA kernels evaluate the same sequence."""
    x = np.asarray(x, dtype=np.float32)
    xc = np.clip(x, EXP_LO, EXP_HI)
    n = np.rint(xc * _LOG2E).astype(np.float32)
    r = (xc - n * _C1).astype(np.float32)
    r = (r - n * _C2).astype(np.float32)
    p = _P[0]
    for c in _P[1:]:
        p = (p * r + c).astype(np.float32)
    r2 = (r * r).astype(np.float32)
    p = (p * r2).astype(np.float32)
    p = (p + r).astype(np.float32)
    p = (p + _F32(1.0)).astype(np.float32)
    ni = n.astype(np.int32)
    h1 = ni // 2
    h2 = ni - h1
    s1 = ((h1 + 127).astype(np.uint32) << 23).view(np.float32)
    s2 = ((h2 + 127).astype(np.uint32) << 23).view(np.float32)
    out = ((p * s1).astype(np.float32) * s2).astype(np.float32)
    out = np.where(x > EXP_HI, _F32(np.inf), out)
    out = np.where(x < EXP_LO, _F32(0.0), out)
    out = np.where(np.isnan(x), _F32(np.nan), out)
    return out.astype(np.float32)


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """act = g * sigmoid(g) * u in fp32, sigmoid(g) = 1 / (1 + exp(-g)),
    evaluated left to right as (g * s) * u (kernels/fused_swiglu_quant_gemv.py:42)."""
    g = np.asarray(g, dtype=np.float32)
    u = np.asarray(u, dtype=np.float32)
    e = exp_f32(-g)
    s = (_F32(1.0) / (_F32(1.0) + e).astype(np.float32)).astype(np.float32)
    return ((g * s).astype(np.float32) * u).astype(np.float32)


def swiglu_quant(gu: np.ndarray):
    """gu: float32 [M, 2I] ([gate | up], bf16 values) -> (xq, sx, act)."""
    gu = np.asarray(gu, dtype=np.float32)
    M, two_i = gu.shape
    I = two_i // 2
    act = silu_mul(gu[:, :I], gu[:, I:])
    xq, sx = group_quant(act)
    return xq, sx, act


# --------------------------------------------------------------------------
# the stand-alone SwiGLU writers (kernels/fused_swiglu_fp8.py)
# --------------------------------------------------------------------------

WRITER_SCALE_FLOOR = np.float32(1e-30)


def swiglu_writer(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """fused_swiglu (kernels/fused_swiglu_fp8.py:19-27): y = g * sigmoid(g) * u
    in fp32, stored as bf16 (RNE).  Returns the bf16 values as float32."""
    return bf16_round(silu_mul(g, u))


def swiglu_quant_writer(g: np.ndarray, u: np.ndarray):
    """fused_swiglu_quant (kernels/fused_swiglu_fp8.py:30-45), a different
    formula from the GEMV prologue's: per 128-group
      scale = max(amax / 448, 1e-30)            (:41, IEEE division)
      q     = e4m3_rne(clamp(y / scale, +-448)) (:42, IEEE division, no reciprocal)
    g, u: float32 [M, I] (bf16 values), I % 128 == 0.
    Returns (q uint8 [M, I], scale float32 [M, I/128], y float32 [M, I])."""
    y = silu_mul(g, u)
    M, I = y.shape
    if I % GROUP:
        raise ValueError("I must be a multiple of 128")
    yg = y.reshape(M, I // GROUP, GROUP)
    am = np.abs(yg).max(axis=-1).astype(np.float32)
    scale = np.maximum((am / E4M3_MAX).astype(np.float32), WRITER_SCALE_FLOOR).astype(np.float32)
    q = np.clip((yg / scale[..., None]).astype(np.float32), -E4M3_MAX, E4M3_MAX).astype(np.float32)
    return e4m3_encode_rne(q).reshape(M, I), scale, y


# --------------------------------------------------------------------------
# block dequant and the contraction
# --------------------------------------------------------------------------

def dequant_weight(wq: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """Wq uint8 [N, K] e4m3 codes, Ws float32 [N/128, K/128] -> float32 [N, K]
    (benchmarks/bench_sglang_fp8.py:54-55)."""
    w = E4M3_TABLE[np.asarray(wq, dtype=np.uint8)]
    ws = np.asarray(ws, dtype=np.float32)
    N, K = w.shape
    return (w.reshape(N // GROUP, GROUP, K // GROUP, GROUP)
            * ws[:, None, :, None]).reshape(N, K).astype(np.float32)


def gemv_from_quant(xq: np.ndarray, sx: np.ndarray, wq: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """Exact (float64-accumulated) block-scaled contraction, returned in fp64.

    out[m, n] = sum_b (sum_{k in b} xq[m,k] W[n,k]) * (sx[m,b] * Ws[n/128,b])
    with the per-block factor formed in fp32 as the reference does
    (kernels/fused_gemv_quant_tm.py:45)."""
    xv = E4M3_TABLE[np.asarray(xq, dtype=np.uint8)].astype(np.float64)
    wv = E4M3_TABLE[np.asarray(wq, dtype=np.uint8)]
    M, K = xv.shape
    N = wv.shape[0]
    sx = np.asarray(sx, np.float32)
    ws = np.asarray(ws, np.float32)
    out = np.zeros((M, N), np.float64)
    for b in range(K // GROUP):
        cols = slice(b * GROUP, (b + 1) * GROUP)
        part = xv[:, cols] @ wv[:, cols].astype(np.float64).T          # exact: <= 2^-18 granularity
        scale = (sx[:, b][:, None] * np.repeat(ws[:, b], GROUP)[None, :]).astype(np.float32)
        out += part * scale.astype(np.float64)
    return out


def fused_gemv_quant(x: np.ndarray, wq: np.ndarray, ws: np.ndarray):
    """Oracle of fused_gemv_quant (kernels/fused_gemv_quant_tm.py:83-102).

    x float32 [M, K] (bf16 values), wq uint8 [N, K], ws float32 [N/128, K/128].
    Returns (out_bf16_as_f32 [M, N], exact_f64 [M, N], xq, sx)."""
    xq, sx = group_quant(x)
    exact = gemv_from_quant(xq, sx, wq, ws)
    return bf16_round(exact.astype(np.float32)), exact, xq, sx


def fused_swiglu_q_gemm(gu: np.ndarray, wq: np.ndarray, ws: np.ndarray):
    """Oracle of fused_swiglu_q_gemm (kernels/fused_swiglu_quant_gemv.py:54-67)."""
    xq, sx, act = swiglu_quant(gu)
    exact = gemv_from_quant(xq, sx, wq, ws)
    return bf16_round(exact.astype(np.float32)), exact, xq, sx


# --------------------------------------------------------------------------
# add + RMSNorm prologue (kernels/fused_rmsnorm.py:14-27, decode dtypes)
# --------------------------------------------------------------------------

RMS_EPS = np.float32(1e-6)


def add_rmsnorm(x: np.ndarray, r: np.ndarray, w: np.ndarray, eps=RMS_EPS):
    """Fused add + RMSNorm as the kernels evaluate it, every step one rounded
    fp32 operation (no fused multiply-add), so the CUDA kernels match bit for
    bit.  The reference kernel (kernels/fused_rmsnorm.py:14-27) computes
        s = x + r;  residual_out = s;  rstd = rsqrt(mean(s^2) + eps);
        out = s * rstd * w
    Here x, r are bf16 [M, K] (float32 values), w the bf16 norm weight [K]:
      s     = f32(x) + f32(r)                    residual_out = bf16(s)
      ssq   = sum of s^2 in a fixed order: per 16-element chunk left to right,
              the 8 chunks of a 128-group pairwise ((c0+c1)+(c2+c3)) +
              ((c4+c5)+(c6+c7)), the K/128 group sums left to right
      rstd  = 1 / sqrt(ssq / K + eps)            (IEEE division and sqrt)
      out   = bf16((s * rstd) * w)
    Returns (out, residual_out, rstd) as float32 arrays ([M, K], [M, K], [M])."""
    x = np.asarray(x, np.float32)
    r = np.asarray(r, np.float32)
    return _rmsnorm_of_sum((x + r).astype(np.float32), w, eps)


def reduce_add_rmsnorm(partials, r: np.ndarray, w: np.ndarray, eps=RMS_EPS):
    """add_rmsnorm whose x is the sum of the partial outputs of a K-sharded
    (row-parallel) linear, one bf16 [M, K] array per rank, added in rank order
    in fp32 before the residual:
        s = ((p_0 + p_1) + ... + p_{n-1}) + r
    (one partial: add_rmsnorm).  The reference is single-GPU; this is what an
    all-reduce of the partials followed by its add + RMSNorm
    (kernels/fused_rmsnorm.py:14-27) computes, with the order of the
    additions fixed.  Returns (out, residual_out, rstd)."""
    parts = [np.asarray(p, np.float32) for p in partials]
    if not parts:
        raise ValueError("at least one partial")
    acc = parts[0]
    for p in parts[1:]:
        acc = (acc + p).astype(np.float32)
    return _rmsnorm_of_sum((acc + np.asarray(r, np.float32)).astype(np.float32), w, eps)


def _rmsnorm_of_sum(s: np.ndarray, w, eps):
    """The norm of add_rmsnorm applied to the fp32 sum s."""
    w = np.asarray(w, np.float32)
    M, K = s.shape
    if K % GROUP:
        raise ValueError("K must be a multiple of 128")
    sq = (s * s).astype(np.float32).reshape(M, K // GROUP, 8, 16)
    c = np.zeros(sq.shape[:3], np.float32)
    for k in range(16):                                            # chunk sums, left to right
        c = (c + sq[..., k]).astype(np.float32)
    p01 = (c[..., 0] + c[..., 1]).astype(np.float32)
    p23 = (c[..., 2] + c[..., 3]).astype(np.float32)
    p45 = (c[..., 4] + c[..., 5]).astype(np.float32)
    p67 = (c[..., 6] + c[..., 7]).astype(np.float32)
    g = ((p01 + p23).astype(np.float32) + (p45 + p67).astype(np.float32)).astype(np.float32)
    ssq = np.zeros(M, np.float32)
    for b in range(K // GROUP):                                    # group sums, left to right
        ssq = (ssq + g[:, b]).astype(np.float32)
    var = (ssq / np.float32(K)).astype(np.float32)
    rstd = (np.float32(1.0) / np.sqrt((var + np.float32(eps)).astype(np.float32))).astype(np.float32)
    h = ((s * rstd[:, None]).astype(np.float32) * w[None, :]).astype(np.float32)
    return bf16_round(h), bf16_round(s), rstd


def fused_add_rmsnorm_gemv_quant(x, r, nw, wq, ws, eps=RMS_EPS):
    """The GEMV fed by the add + RMSNorm prologue: quantises the bf16 norm
    output exactly as fused_gemv_quant quantises its input.  Returns
    (out_bf16_as_f32, exact_f64, xq, sx, residual_out)."""
    h, res, _ = add_rmsnorm(x, r, nw, eps)
    xq, sx = group_quant(h)
    exact = gemv_from_quant(xq, sx, wq, ws)
    return bf16_round(exact.astype(np.float32)), exact, xq, sx, res


def fused_reduce_add_rmsnorm_gemv_quant(partials, r, nw, wq, ws, eps=RMS_EPS):
    """fused_add_rmsnorm_gemv_quant fed by reduce_add_rmsnorm (the sum of the
    partials in rank order, then the residual).  Returns
    (out_bf16_as_f32, exact_f64, xq, sx, residual_out)."""
    h, res, _ = reduce_add_rmsnorm(partials, r, nw, eps)
    xq, sx = group_quant(h)
    exact = gemv_from_quant(xq, sx, wq, ws)
    return bf16_round(exact.astype(np.float32)), exact, xq, sx, res


# --------------------------------------------------------------------------
# tolerances used by the reference's own self-tests
# --------------------------------------------------------------------------

def bf16_ulp_at(v: float) -> float:
    """ulp of bf16 at magnitude v (kernels/fused_gemv_quant.py:107)."""
    if v <= 0:
        return 2.0 ** -133
    return 2.0 ** (np.floor(np.log2(v)) - 7)


def ref_atol(ref: np.ndarray, ulps: float) -> float:
    """atol = ulps * ulp_bf16(max|ref|) + 1e-3 (kernels/fused_gemv_quant.py:107-108,
    kernels/fused_gemv_quant_tm.py:138-140)."""
    return ulps * bf16_ulp_at(float(np.abs(ref).max())) + 1e-3


def rms_tolerance_ok(got: np.ndarray, ref: np.ndarray, rtol: float = 1e-2, atol_rel_rms: float = 1e-2):
    """|got - ref| <= rtol*|ref| + atol_rel_rms * RMS(ref), elementwise."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    return bool(np.all(np.abs(got - ref) <= rtol * np.abs(ref) + atol_rel_rms * rms))


# --------------------------------------------------------------------------
# synthetic inputs (seeded) -- the shapes and value distributions of the
# reference's benchmark cases; no dataset is involved
# --------------------------------------------------------------------------

def make_activation(M: int, K: int, seed: int, std: float = 1.0, outlier_frac: float = 0.01,
                    outlier_scale: float = 20.0) -> np.ndarray:
    """bf16 ~N(0, std^2) with `outlier_frac` of the channels scaled by
    `outlier_scale` (channels picked by a seeded permutation).  Seeded torch
    CPU generator; returns float32 holding bf16 values."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    x = torch.randn(M, K, generator=g) * float(std)
    n_out = int(round(outlier_frac * K))
    if n_out:
        ch = torch.randperm(K, generator=g)[:n_out]
        x[:, ch] *= float(outlier_scale)
    return x.to(torch.bfloat16).float().numpy()


def quantize_weight_blocks(w: np.ndarray):
    """bf16/fp32 W [N, K] -> (Wq uint8, Ws float32 [N/128, K/128]) with
    ws = max(amax_block, eps) / 448 and Wq = e4m3_rne(clamp(W / ws, +-448)),
    every step an fp32 operation (torch on CPU; its e4m3 cast is the RNE cast
    e4m3_encode_rne implements, which the tests check)."""
    import torch
    t = torch.as_tensor(np.asarray(w, np.float32))
    N, K = t.shape
    blk = t.view(N // GROUP, GROUP, K // GROUP, GROUP)
    amax = blk.abs().amax(dim=(1, 3)).clamp_min(float(EPS))
    ws = amax / float(E4M3_MAX)
    q = (blk / ws[:, None, :, None]).clamp(-float(E4M3_MAX), float(E4M3_MAX)).to(torch.float8_e4m3fn)
    return q.view(torch.uint8).reshape(N, K).numpy(), ws.numpy().astype(np.float32)


def make_weight(N: int, K: int, seed: int, std: float = 0.02):
    """Weight ~N(0, std^2) in bf16, block-quantised to e4m3 (seeded)."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    w = (torch.randn(N, K, generator=g) * float(std)).to(torch.bfloat16).float()
    return quantize_weight_blocks(w.numpy())


# --------------------------------------------------------------------------
# the reference PyTorch path on CPU (quantise, dequantise, matmul) -- the
# timed CPU baseline; torch is imported lazily
# --------------------------------------------------------------------------

def torch_reference_path(x, wq, ws, act_from_gate_up: bool = False):
    """CPU torch restatement of the reference path used as the CPU baseline.

    x: torch bf16 [M, K] (or [M, 2I] when act_from_gate_up), wq: torch
    float8_e4m3fn [N, K], ws: torch float32 [N/128, K/128].  Group quant
    (kernels/fused_gemv_quant.py:40-43), dequant of both operands
    (benchmarks/bench_sglang_fp8.py:54-55), fp32 matmul, bf16 output."""
    import torch
    xf = x.float()
    if act_from_gate_up:
        i = xf.shape[1] // 2
        g, u = xf[:, :i], xf[:, i:]
        xf = g * torch.sigmoid(g) * u
    M, K = xf.shape
    grp = xf.view(M, K // GROUP, GROUP)
    absmax = grp.abs().amax(-1, keepdim=True).clamp_min(float(EPS))
    sx = absmax / 448.0
    xq = (grp * (1.0 / sx)).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    xd = (xq.float() * sx).view(M, K)
    wd = wq.float() * ws.repeat_interleave(GROUP, 0).repeat_interleave(GROUP, 1)
    return (xd @ wd.T).to(torch.bfloat16)
