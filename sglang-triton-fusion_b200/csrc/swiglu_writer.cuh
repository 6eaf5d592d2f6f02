// Stand-alone SwiGLU writers for large M (prefill): y = g * sigmoid(g) * u,
// stored as bf16 (fused_swiglu, kernels/fused_swiglu_fp8.py:19-27) or
// quantised per 128-group with that module's own formula
// (fused_swiglu_quant, kernels/fused_swiglu_fp8.py:30-45):
//   scale = max(amax / 448, 1e-30),  q = e4m3_rne(clamp(y / scale, +-448))
// -- true IEEE divisions, unlike the GEMV prologue's x * (1 / sx).
//
// HBM-bound streaming: a half-warp owns one 128-group (8 values per lane,
// 16-byte loads of gate and up, evict-first), grid-stride over the groups.
#pragma once

#include "fp8gq_device.cuh"

namespace fp8gq {

constexpr float kWriterScaleFloor = 1e-30f;

// 8 bf16 values (16 bytes) of gate and up -> 8 fp32 activations.
__device__ __forceinline__ void swiglu8(float (&y)[8], uint4 g, uint4 u) {
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
  const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    y[2 * e] = silu_mul(bf16_lo(gw[e]), bf16_lo(uw[e]));
    y[2 * e + 1] = silu_mul(bf16_hi(gw[e]), bf16_hi(uw[e]));
  }
}

// Two values -> two e4m3 codes (v0 in the low byte): y / scale (IEEE
// division), clamp to +-448, round to nearest even.
__device__ __forceinline__ uint16_t quant_pair_div(float v0, float v1, float scale) {
  const float y0 = fminf(fmaxf(__fdiv_rn(v0, scale), -kE4m3Max), kE4m3Max);
  const float y1 = fminf(fmaxf(__fdiv_rn(v1, scale), -kE4m3Max), kE4m3Max);
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(make_float2(y0, y1), __NV_SATFINITE, __NV_E4M3));
}

// Streaming 16-byte load (read once: cache-streaming hint).
__device__ __forceinline__ uint4 ldg_stream(const void* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }

template <bool kQuant>
__global__ void __launch_bounds__(256) swiglu_writer_kernel(const __nv_bfloat16* __restrict__ gate, int64_t ldg,
                                                            const __nv_bfloat16* __restrict__ up, int64_t ldu,
                                                            void* __restrict__ out, int64_t ldo,
                                                            float* __restrict__ scale_out, int M, int I) {
  grid_dependency_wait();
  const int gpr = I / kGroup;
  const int64_t ngroups = static_cast<int64_t>(M) * gpr;
  const int lane = threadIdx.x & 31;
  const int l16 = lane & 15;
  const unsigned half_mask = 0xFFFFu << (lane & 16);
  for (int64_t gid = static_cast<int64_t>(blockIdx.x) * 16 + (threadIdx.x >> 4); gid < ngroups;
       gid += static_cast<int64_t>(gridDim.x) * 16) {
    const int m = static_cast<int>(gid / gpr);
    const int col = static_cast<int>(gid - static_cast<int64_t>(m) * gpr) * kGroup + l16 * 8;
    const uint4 g = ldg_stream(gate + m * ldg + col);
    const uint4 u = ldg_stream(up + m * ldu + col);
    float y[8];
    swiglu8(y, g, u);
    if constexpr (!kQuant) {
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * e], y[2 * e + 1]);
        ow[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + m * ldo + col) = o;
    } else {
      float amax = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(y[e]));
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(half_mask, amax, off, 16));
      const float s = fmaxf(__fdiv_rn(amax, kE4m3Max), kWriterScaleFloor);
      uint2 q;
      q.x = quant_pair_div(y[0], y[1], s) | (static_cast<uint32_t>(quant_pair_div(y[2], y[3], s)) << 16);
      q.y = quant_pair_div(y[4], y[5], s) | (static_cast<uint32_t>(quant_pair_div(y[6], y[7], s)) << 16);
      *reinterpret_cast<uint2*>(static_cast<uint8_t*>(out) + m * ldo + col) = q;
      if (l16 == 0) scale_out[gid] = s;
    }
  }
  grid_launch_dependents();
}

}  // namespace fp8gq
