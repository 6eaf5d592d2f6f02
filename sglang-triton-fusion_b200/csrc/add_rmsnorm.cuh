// Stand-alone fused add + RMSNorm (the reference's add_rmsnorm_kernel,
// kernels/fused_rmsnorm.py:14-27) with the evaluation order the GEMV
// prologues use: out = bf16((s * rstd) * w), residual_out = bf16(s),
// s = x + r.  One CTA per row; the fused GEMV entry points compute the same
// bits inside their prologue, this kernel serves the norm on its own and the
// bit-exact tests.
#pragma once

#include "fp8gq_device.cuh"

namespace fp8gq {

constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ r, int64_t ldr,
    const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* __restrict__ out, int64_t ldo,
    __nv_bfloat16* __restrict__ res_out, int64_t ldro, int K) {
  extern __shared__ float gsum[];     // [K/128 + 1]
  grid_dependency_wait();
  const int m = blockIdx.x;
  const int tid = threadIdx.x;
  const int n_chunks = K / 16;
  const __nv_bfloat16* xr = x + m * ldx;
  const __nv_bfloat16* rr = r + m * ldr;
  for (int c0 = 0; c0 < n_chunks; c0 += kNormThreads) {
    const int c = c0 + tid;
    const bool valid = c < n_chunks;
    float sv[16];
    if (valid) {
      const uint4* xp = reinterpret_cast<const uint4*>(xr + 16 * c);
      const uint4* rp = reinterpret_cast<const uint4*>(rr + 16 * c);
      add16(sv, xp[0], xp[1], rp[0], rp[1]);
      if (res_out) {
        uint4 a, b;
        pack_bf16x16(sv, a, b);
        uint4* op = reinterpret_cast<uint4*>(res_out + m * ldro + 16 * c);
        op[0] = a;
        op[1] = b;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) sv[e] = 0.0f;
    }
    const float gs = octet_sum(sumsq16(sv));
    if (valid && (c & 7) == 0) gsum[c >> 3] = gs;
  }
  __syncthreads();
  if (tid == 0) {
    float a = 0.0f;
    for (int b = 0; b < K / 128; ++b) a = __fadd_rn(a, gsum[b]);
    gsum[K / 128] = rms_rstd(a, K, eps);
  }
  __syncthreads();
  const float rstd = gsum[K / 128];
  for (int c = tid; c < n_chunks; c += kNormThreads) {
    const uint4* xp = reinterpret_cast<const uint4*>(xr + 16 * c);
    const uint4* rp = reinterpret_cast<const uint4*>(rr + 16 * c);
    const uint4* wp = reinterpret_cast<const uint4*>(w + 16 * c);
    float sv[16], h[16];
    add16(sv, xp[0], xp[1], rp[0], rp[1]);
    norm16(h, sv, rstd, wp[0], wp[1]);
    uint4 a, b;
    pack_bf16x16(h, a, b);
    uint4* op = reinterpret_cast<uint4*>(out + m * ldo + 16 * c);
    op[0] = a;
    op[1] = b;
  }
  grid_launch_dependents();
}

}  // namespace fp8gq
