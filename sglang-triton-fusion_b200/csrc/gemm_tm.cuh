// Tile kernel: fused quant + block-scaled GEMM for M tokens on the 5th-gen
// tensor cores (tcgen05, kind::f8f6f4, e4m3 x e4m3 -> fp32 in TMEM).
// Replaces gemv_quant_tm_kernel (kernels/fused_gemv_quant_tm.py:49-80) and,
// with the SwiGLU prologue, swiglu_q_gemm_kernel for M > 1
// (kernels/fused_swiglu_quant_gemv.py:26-51).
//
// Swap-AB: the MMA's M dimension is 128 weight rows (one 128x128 scale
// block), its N dimension the MT tokens of a pass (16, 32 or 64), K = 32 per
// instruction, four instructions per 128-wide K block.  Each weight tile is
// read from HBM once for all MT tokens.
//
// The scales are per (token, 128-K block) and per (128-row, 128-K block), so
// the K blocks cannot share an accumulator: every K block's MMAs write their
// own TMEM buffer (a ring of NACC buffers), and the epilogue warps read it
// back (tcgen05.ld), multiply by sx[m, b] * ws[nb, b] and add into fp32
// registers -- the per-block promotion of kernels/fused_gemv_quant_tm.py:77.
//
// Work split (stream-K): the N/128 x K/128 tiles are numbered row-block
// major; CTA i of G takes tiles [i*U/G, (i+1)*U/G).  A row block covered by
// one CTA is stored directly; a row block split between CTAs leaves fp32
// partial sums in the caller's workspace, and the CTA that finishes it last
// (atomic counter per row block) adds the partials in CTA order -- the result
// does not depend on timing -- stores bf16 and re-zeroes the counter.
//
// Warp roles (320 threads, one CTA per SM):
//   warp 0      TMA producer: 128x128-byte weight tiles (SWIZZLE_128B) into
//               the stage ring (no multicast).
//   warp 1      TMEM allocator and MMA issuer (one elected lane).
//   warps 2-5   activation producers: quantise x (or silu(g)*u) for the
//               stage's K block into the swizzled B tile, write sx.
//   warps 6-9   epilogue: TMEM -> registers, scale, accumulate, store.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "fp8gq_device.cuh"

namespace fp8gq {

constexpr int kTmThreads = 320;
constexpr int kTmNAcc = 4;          // TMEM accumulator buffers
constexpr int kTmSxRing = 32;       // >= stages + accumulators + 1
constexpr int kTmATileBytes = 128 * 128;
// The workspace starts with one split-K counter per 128-row block, in a region
// of fixed size so that the partial sums of one shape never land on the
// counters of another shape that shares the workspace.
constexpr int kTmMaxRowBlocks = 4096;                       // N <= 524288
constexpr size_t kTmCounterBytes = static_cast<size_t>(kTmMaxRowBlocks) * 4;

struct TmParams {
  const __nv_bfloat16* x;   // [M, ldx] (plain) or [M, ldx] with [gate | up] (SwiGLU)
  int64_t ldx;
  const float* ws;          // [N/128, ldws]
  int64_t ldws;
  __nv_bfloat16* out;       // [M, ldo]
  int64_t ldo;
  int M;                    // valid tokens in this pass (<= MT)
  int N, K;
  int KB;                   // K / 128
  int64_t U;                // (N/128) * KB tiles
  int* counters;            // [kTmMaxRowBlocks], zero on entry and exit
  float* partials;          // [G][2][MT][128]
  uint8_t* xq_out;          // optional [M, K]
  float* sx_out;            // optional [M, K/128]
};

template <int MT>
struct TmCfg {
  static constexpr int kStages = 8;
  static constexpr int kBTileBytes = MT * 128;
  static constexpr int kStageBytes = kTmATileBytes + kBTileBytes;
  static constexpr int kTmemCols = (kTmNAcc * MT <= 32) ? 32 : (kTmNAcc * MT <= 64) ? 64
                                   : (kTmNAcc * MT <= 128) ? 128 : 256;
  // ring | full[S] empty[S] acc_full[NACC] tmem_empty[NACC] sx_full[SXR] drain
  //      | tmem addr, flag | sx ring
  static constexpr size_t kBarOffset = static_cast<size_t>(kStages) * kStageBytes;
  static constexpr size_t kMiscOffset = kBarOffset + (2 * kStages + 2 * kTmNAcc + kTmSxRing + 1) * 8;
  static constexpr size_t kSxOffset = kMiscOffset + 16;
  static constexpr size_t kSmemBytes = kSxOffset + kTmSxRing * MT * 4 + 1024;  // +1 KB alignment slack
};

// ----------------------------------------------------------------- PTX --
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* tmap, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// K-major operand in the 128-byte swizzle layout: 8-row atoms of 1024 bytes
// stacked at SBO = 1024; version 1 (tcgen05); layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;               // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;        // SBO
  d |= static_cast<uint64_t>(1u) << 46;                // version
  d |= static_cast<uint64_t>(2u) << 61;                // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D fp32, A and B e4m3, both K-major, M = 128, N = MT.
template <int MT>
__device__ __forceinline__ uint32_t idesc_f8() {
  return (1u << 4) | (static_cast<uint32_t>(MT >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------------- kernel --
template <int MT, bool kSwiglu>
__global__ void __launch_bounds__(kTmThreads, 1)
gemm_tm_kernel(const __grid_constant__ CUtensorMap tmap_w, const TmParams p) {
  using Cfg = TmCfg<MT>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* tmem_empty = acc_full + kTmNAcc;
  uint64_t* sx_full = tmem_empty + kTmNAcc;   // activation producers -> epilogue, per sx slot
  uint64_t* drain = sx_full + kTmSxRing;      // MMA completion on the error path
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOffset);  // [0] tmem base, [1] last flag
  float* sx_ring = reinterpret_cast<float*>(smem + Cfg::kSxOffset);      // [kTmSxRing][MT]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int64_t G = gridDim.x;
  const int64_t u0 = (static_cast<int64_t>(blockIdx.x) * p.U) / G;
  const int64_t u1 = (static_cast<int64_t>(blockIdx.x + 1) * p.U) / G;
  const int J = static_cast<int>(u1 - u0);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1 + 4);    // TMA arrive_expect_tx + 4 activation warps
      mbar_init(&empty[s], 1);       // tcgen05.commit
    }
    for (int a = 0; a < kTmNAcc; ++a) {
      mbar_init(&acc_full[a], 1);    // tcgen05.commit
      mbar_init(&tmem_empty[a], 4);  // 4 epilogue warps
    }
    for (int r = 0; r < kTmSxRing; ++r) mbar_init(&sx_full[r], 4);  // 4 activation warps
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&misc[0])),
                 "r"(Cfg::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = misc[0];
  bool ok = true;

  if (warp == 0) {
    // --------------------------------------------------- TMA producer --
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int issued = 0;
      for (int j = 0; j < J && ok; ++j) {
        const int s = j % S;
        if (j >= S) ok = mbar_wait(&empty[s], ((j / S) & 1) ^ 1, kSiteTmA);
        if (!ok) break;
        const int64_t u = u0 + j;
        const int nb = static_cast<int>(u / p.KB);
        const int kb = static_cast<int>(u % p.KB);
        mbar_arrive_expect_tx(&full[s], kTmATileBytes);
        tma_load_2d(smem + static_cast<size_t>(s) * Cfg::kStageBytes, &tmap_w, kb * 128, nb * 128,
                    &full[s], pol);
        issued = j + 1;
      }
      if (!ok) {
        // let the copies already issued land before the CTA can exit
        for (int j = (issued > S ? issued - S : 0); j < issued; ++j)
          mbar_wait(&full[j % S], (j / S) & 1, kSiteTmA);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------- MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = idesc_f8<MT>();
      for (int j = 0; j < J && ok; ++j) {
        const int s = j % S;
        const int a = j % kTmNAcc;
        if (j >= kTmNAcc) ok = mbar_wait(&tmem_empty[a], ((j / kTmNAcc) & 1) ^ 1, kSiteTmTmem);
        if (!ok) break;
        ok = mbar_wait(&full[s], (j / S) & 1, kSiteTmB);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + static_cast<size_t>(s) * Cfg::kStageBytes);
        const uint32_t b_addr = a_addr + kTmATileBytes;
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(a * MT);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8(d_tmem, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32), idesc,
                 kk > 0 ? 1u : 0u);
        mma_commit(&empty[s]);
        mma_commit(&acc_full[a]);
      }
      if (!ok) {
        // wait for every MMA issued so far before TMEM can be released
        mma_commit(drain);
        mbar_wait(drain, 0, kSiteTmB);
      }
    }
  } else if (warp < 6) {
    // ----------------------------------------- activation producers --
    const int t = tid - 64;             // 0..127
    const int chunk = t & 7;            // 16-byte chunk of the 128-wide K block
    const int row0 = t >> 3;            // 0..15
    for (int j = 0; j < J && ok; ++j) {
      const int s = j % S;
      if (j >= S) ok = mbar_wait(&empty[s], ((j / S) & 1) ^ 1, kSiteTmA);
      if (!ok) break;
      const int64_t u = u0 + j;
      const int nb = static_cast<int>(u / p.KB);
      const int kb = static_cast<int>(u % p.KB);
      uint8_t* btile = smem + static_cast<size_t>(s) * Cfg::kStageBytes + kTmATileBytes;
      float* sxs = sx_ring + (j % kTmSxRing) * MT;
#pragma unroll
      for (int i = 0; i < MT / 16; ++i) {
        const int m = row0 + 16 * i;
        float v[16];
        if (m < p.M) {
          const __nv_bfloat16* xr = p.x + static_cast<int64_t>(m) * p.ldx + kb * 128 + chunk * 16;
          if constexpr (kSwiglu) {
            const uint4* gp = reinterpret_cast<const uint4*>(xr);
            const uint4* up = reinterpret_cast<const uint4*>(xr + p.K);
            const uint4 g_a = gp[0], g_b = gp[1], u_a = up[0], u_b = up[1];
            const uint32_t gw[8] = {g_a.x, g_a.y, g_a.z, g_a.w, g_b.x, g_b.y, g_b.z, g_b.w};
            const uint32_t uw[8] = {u_a.x, u_a.y, u_a.z, u_a.w, u_b.x, u_b.y, u_b.z, u_b.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              v[2 * e] = silu_mul(bf16_lo(gw[e]), bf16_lo(uw[e]));
              v[2 * e + 1] = silu_mul(bf16_hi(gw[e]), bf16_hi(uw[e]));
            }
          } else {
            const uint4* xp = reinterpret_cast<const uint4*>(xr);
            const uint4 a = xp[0], b = xp[1];
            const uint32_t xw[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              v[2 * e] = bf16_lo(xw[e]);
              v[2 * e + 1] = bf16_hi(xw[e]);
            }
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = 0.0f;
        }
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[e]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        const float sx = group_scale(amax);
        const float sinv = __frcp_rn(sx);
        uint4 packed;
        packed.x = quant_pair(v[0], v[1], sinv) | (static_cast<uint32_t>(quant_pair(v[2], v[3], sinv)) << 16);
        packed.y = quant_pair(v[4], v[5], sinv) | (static_cast<uint32_t>(quant_pair(v[6], v[7], sinv)) << 16);
        packed.z = quant_pair(v[8], v[9], sinv) | (static_cast<uint32_t>(quant_pair(v[10], v[11], sinv)) << 16);
        packed.w = quant_pair(v[12], v[13], sinv) | (static_cast<uint32_t>(quant_pair(v[14], v[15], sinv)) << 16);
        if (m >= p.M) packed = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(btile + m * 128 + ((chunk ^ (m & 7)) << 4)) = packed;
        if (chunk == 0) sxs[m] = sx;
        if (nb == 0 && m < p.M) {
          if (p.xq_out)
            *reinterpret_cast<uint4*>(p.xq_out + static_cast<int64_t>(m) * p.K + kb * 128 + chunk * 16) = packed;
          if (p.sx_out && chunk == 0) p.sx_out[static_cast<int64_t>(m) * p.KB + kb] = sx;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full[s]);
        mbar_arrive(&sx_full[j % kTmSxRing]);
      }
    }
  } else {
    // -------------------------------------------------------- epilogue --
    const int q = warp & 3;                  // TMEM lane quarter of this warp
    const int row = 32 * q + lane;           // weight row within the 128-row block
    const uint32_t t_lane = static_cast<uint32_t>(32 * q) << 16;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    int seg_j0 = 0;
    for (int j = 0; j < J; ++j) {
      const int a = j % kTmNAcc;
      const int64_t u = u0 + j;
      const int nb = static_cast<int>(u / p.KB);
      const int kb = static_cast<int>(u % p.KB);
      if (j == 0 || kb == 0) {
        seg_j0 = j;
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
      }
      if (ok) ok = mbar_wait(&acc_full[a], (j / kTmNAcc) & 1, kSiteTmAcc);
      if (ok) ok = mbar_wait(&sx_full[j % kTmSxRing], (j / kTmSxRing) & 1, kSiteTmAcc);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const float sw = __ldg(p.ws + static_cast<int64_t>(nb) * p.ldws + kb);
      const float* sxs = sx_ring + (j % kTmSxRing) * MT;
#pragma unroll
      for (int c = 0; c < MT / 16; ++c) {
        float v[16];
        if (ok) {
          tmem_ld16(tmem_base + t_lane + static_cast<uint32_t>(a * MT + 16 * c), v);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[16 * c + i] = fmaf(v[i], sxs[16 * c + i] * sw, acc[16 * c + i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[a]);

      if (kb == p.KB - 1 || j == J - 1) {
        const int n = nb * 128 + row;
        const bool whole = (u - (j - seg_j0)) % p.KB == 0 && kb == p.KB - 1;
        if (whole) {
#pragma unroll
          for (int m = 0; m < MT; ++m)
            if (m < p.M) p.out[static_cast<int64_t>(m) * p.ldo + n] = __float2bfloat16_rn(acc[m]);
        } else {
          // partial row block: publish, count, and let the last CTA reduce
          const int slot = (seg_j0 == 0) ? 0 : 1;
          float* mine = p.partials + ((static_cast<int64_t>(blockIdx.x) * 2 + slot) * MT) * 128;
#pragma unroll
          for (int m = 0; m < MT; ++m)
            if (m < p.M) mine[m * 128 + row] = acc[m];
          __threadfence();
          named_bar_sync(2, 128);
          const int64_t first_u = static_cast<int64_t>(nb) * p.KB;
          const int64_t last_u = first_u + p.KB - 1;
          const int64_t i_lo = ((first_u + 1) * G - 1) / p.U;
          const int64_t i_hi = ((last_u + 1) * G - 1) / p.U;
          if (tid == 192) {
            const int old = atomicAdd(&p.counters[nb], 1);
            const bool last = (old == static_cast<int>(i_hi - i_lo));
            misc[1] = last ? 1u : 0u;
            if (last) p.counters[nb] = 0;
          }
          named_bar_sync(2, 128);
          if (misc[1]) {
            __threadfence();
            float sum[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) sum[m] = 0.0f;
            for (int64_t i = i_lo; i <= i_hi; ++i) {
              const int64_t ui0 = (i * p.U) / G;
              const int si = (ui0 / p.KB == nb) ? 0 : 1;
              const float* pi = p.partials + ((i * 2 + si) * MT) * 128;
#pragma unroll
              for (int m = 0; m < MT; ++m)
                if (m < p.M) sum[m] += __ldcg(pi + m * 128 + row);
            }
#pragma unroll
            for (int m = 0; m < MT; ++m)
              if (m < p.M) p.out[static_cast<int64_t>(m) * p.ldo + n] = __float2bfloat16_rn(sum[m]);
          }
          named_bar_sync(2, 128);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(Cfg::kTmemCols));
  }
}

// --------------------------------------------------------------- host --
inline int tm_token_tile(int M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

inline int tm_grid(int64_t U, int sm_count) {
  return static_cast<int>(U < sm_count ? U : sm_count);
}

inline size_t tm_workspace_bytes_for(int M, int N, int K, int sm_count) {
  const int MT = tm_token_tile(M);
  const int64_t U = static_cast<int64_t>(N / kGroup) * (K / kGroup);
  const int G = tm_grid(U, sm_count);
  return kTmCounterBytes + static_cast<size_t>(G) * 2 * MT * 128 * sizeof(float);
}

inline size_t tm_workspace_bytes(int M, int N, int K) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return tm_workspace_bytes_for(M, N, K, sms);
}

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Weight tensor map: 2-D uint8 [N rows, K bytes] with row stride ldw, box
// 128 x 128 bytes, 128-byte swizzle (the UMMA K-major SW128 layout).
inline bool make_weight_tmap(CUtensorMap* map, const void* w, int N, int K, int64_t ldw) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldw)};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MT, bool S>
int launch_tm_pass(const CUtensorMap& tmap, const TmParams& p, int grid, int max_smem, cudaStream_t stream) {
  using Cfg = TmCfg<MT>;
  if (Cfg::kSmemBytes > static_cast<size_t>(max_smem)) return 8;  // FP8GQ_ERR_UNSUPPORTED
  auto fn = gemm_tm_kernel<MT, S>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(Cfg::kSmemBytes)) != cudaSuccess)
    return 7;  // FP8GQ_ERR_LAUNCH
  fn<<<grid, kTmThreads, Cfg::kSmemBytes, stream>>>(tmap, p);
  return cudaGetLastError() == cudaSuccess ? 0 : 7;
}

// Runs ceil(M / MT) passes of at most MT tokens; every pass reuses the
// workspace (its counters are zero again when a pass ends).
inline int launch_tm(bool swiglu, const void* x, int64_t ldx, const void* w, int64_t ldw, const float* ws,
                     int64_t ldws, void* out, int64_t ldo, int M, int N, int K, uint8_t* xq_out,
                     float* sx_out, void* workspace, size_t workspace_bytes, int sm_count, int max_smem,
                     cudaStream_t stream) {
  const int MT = tm_token_tile(M);
  if (N / kGroup > kTmMaxRowBlocks) return 8;  // FP8GQ_ERR_UNSUPPORTED
  const size_t need = tm_workspace_bytes_for(M, N, K, sm_count);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return 5;  // FP8GQ_ERR_WORKSPACE
  CUtensorMap tmap;
  if (!make_weight_tmap(&tmap, w, N, K, ldw)) return 7;
  TmParams p;
  p.ldx = ldx;
  p.ws = ws;
  p.ldws = ldws;
  p.ldo = ldo;
  p.N = N;
  p.K = K;
  p.KB = K / kGroup;
  p.U = static_cast<int64_t>(N / kGroup) * p.KB;
  p.counters = static_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kTmCounterBytes);
  const int grid = tm_grid(p.U, sm_count);
  for (int m0 = 0; m0 < M; m0 += MT) {
    p.x = static_cast<const __nv_bfloat16*>(x) + static_cast<int64_t>(m0) * ldx;
    p.out = static_cast<__nv_bfloat16*>(out) + static_cast<int64_t>(m0) * ldo;
    p.M = (M - m0 < MT) ? (M - m0) : MT;
    p.xq_out = xq_out ? xq_out + static_cast<int64_t>(m0) * K : nullptr;
    p.sx_out = sx_out ? sx_out + static_cast<int64_t>(m0) * (K / kGroup) : nullptr;
    int st;
    if (MT == 16)
      st = swiglu ? launch_tm_pass<16, true>(tmap, p, grid, max_smem, stream)
                  : launch_tm_pass<16, false>(tmap, p, grid, max_smem, stream);
    else if (MT == 32)
      st = swiglu ? launch_tm_pass<32, true>(tmap, p, grid, max_smem, stream)
                  : launch_tm_pass<32, false>(tmap, p, grid, max_smem, stream);
    else
      st = swiglu ? launch_tm_pass<64, true>(tmap, p, grid, max_smem, stream)
                  : launch_tm_pass<64, false>(tmap, p, grid, max_smem, stream);
    if (st) return st;
  }
  return 0;
}

}  // namespace fp8gq
