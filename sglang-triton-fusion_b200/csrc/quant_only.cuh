// Stand-alone activation group quant (and SwiGLU + group quant): one warp
// per 128-group, 4 values per lane.  Same device functions as the fused
// kernels' prologues, so its bytes are the fused kernels' bytes.  The tile
// kernel also runs it ahead of itself for large M (its pre-quantised feed).
#pragma once

#include "fp8gq_device.cuh"

namespace fp8gq {

template <bool kSwiglu>
__global__ void __launch_bounds__(256) group_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                          int64_t ldx, int M, int K,
                                                          uint8_t* __restrict__ xq,
                                                          float* __restrict__ sx_out) {
  grid_dependency_wait();   // the activation comes from the stream's previous work
  grid_launch_dependents();
  const int groups_per_row = K / kGroup;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  if (gid >= static_cast<int64_t>(M) * groups_per_row) return;
  const int lane = threadIdx.x & 31;
  const int m = static_cast<int>(gid / groups_per_row);
  const int b = static_cast<int>(gid % groups_per_row);
  const int col = b * kGroup + 4 * lane;
  float v[4];
  if constexpr (kSwiglu) {
    const uint2 g = *reinterpret_cast<const uint2*>(x + m * ldx + col);
    const uint2 u = *reinterpret_cast<const uint2*>(x + m * ldx + K + col);
    v[0] = silu_mul(bf16_lo(g.x), bf16_lo(u.x));
    v[1] = silu_mul(bf16_hi(g.x), bf16_hi(u.x));
    v[2] = silu_mul(bf16_lo(g.y), bf16_lo(u.y));
    v[3] = silu_mul(bf16_hi(g.y), bf16_hi(u.y));
  } else {
    const uint2 a = *reinterpret_cast<const uint2*>(x + m * ldx + col);
    v[0] = bf16_lo(a.x);
    v[1] = bf16_hi(a.x);
    v[2] = bf16_lo(a.y);
    v[3] = bf16_hi(a.y);
  }
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float s = group_scale(amax);
  const float sinv = __frcp_rn(s);
  const uint32_t q = quant_pair(v[0], v[1], sinv) | (static_cast<uint32_t>(quant_pair(v[2], v[3], sinv)) << 16);
  *reinterpret_cast<uint32_t*>(xq + static_cast<int64_t>(m) * K + col) = q;
  if (lane == 0) sx_out[static_cast<int64_t>(m) * groups_per_row + b] = s;
}

// Launch over M rows of K (programmatic dependent launch).
inline cudaError_t launch_group_quant(bool swiglu, const __nv_bfloat16* x, int64_t ldx, int M, int K, uint8_t* xq,
                                     float* sx, cudaStream_t stream) {
  const int64_t groups = static_cast<int64_t>(M) * (K / kGroup);
  const int64_t blocks = (groups + 7) / 8;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  return swiglu ? launch_with_pdl(group_quant_kernel<true>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                                  x, ldx, M, K, xq, sx)
                : launch_with_pdl(group_quant_kernel<false>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                                  stream, x, ldx, M, K, xq, sx);
}

}  // namespace fp8gq
