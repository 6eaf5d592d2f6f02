// Tile kernel: fused quant + block-scaled GEMM for M tokens on the 5th-gen
// tensor cores (tcgen05, kind::f8f6f4, e4m3 x e4m3 -> fp32 in TMEM).
// Replaces gemv_quant_tm_kernel (kernels/fused_gemv_quant_tm.py:49-80) and,
// with the SwiGLU prologue, swiglu_q_gemm_kernel
// (kernels/fused_swiglu_quant_gemv.py:26-51).
//
// Swap-AB: the MMA's M dimension is 128 weight rows (one 128x128 scale
// block), its N dimension the MT token columns of a pass (16, 32 or 64),
// K = 32 per instruction, four instructions per 128-wide K block.  Each weight
// tile is read from HBM once for all tokens of the pass.
//
// Per-block promotion.  The scales are per (token, 128-K block) and per
// (128-row, 128-K block), so products of different K blocks may not be summed
// before they are scaled (kernels/fused_gemv_quant_tm.py:77).  Each K block
// therefore gets its own fp32 columns in TMEM: with M tokens padded to
// SW = next power of two (<= MT), a 16-column accumulator holds KPB = MT / SW
// consecutive K blocks side by side (K block q of the group in columns
// [q*SW, (q+1)*SW)), and the activation tile of K block q carries the
// quantised tokens in those rows of B and zeros elsewhere.  The epilogue warps
// read a group once (tcgen05.ld), scale column c by sx[m, b_q] * ws[nb, b_q]
// and accumulate in registers.  At M = 1 that is one TMEM read per 16 K
// blocks; at M = 16 (or MT = 32, 64) one per K block.
//
// Work split (stream-K): the N/128 x K/128 tiles are numbered row-block
// major; CTA i of G takes tiles [i*U/G, (i+1)*U/G).  A row block covered by
// one CTA is stored directly; a row block split between CTAs leaves fp32
// partial sums in the workspace, and the CTA that finishes it last (atomic
// counter per row block) adds the partials in CTA order -- the result does not
// depend on timing -- stores bf16 and re-zeroes the counter.
//
// Warp roles (320 threads, one CTA per SM):
//   warp 0      TMA producer: the 128x128-byte weight tile (SWIZZLE_128B) and
//               the bf16 activation tile(s) of the K block (no multicast).
//   warp 1      TMEM allocator and MMA issuer (one elected lane).
//   warps 2-5   activation producers: with P of them active (P divides the
//               ring depth), warp w takes the CTA's K blocks j = w-2 mod P,
//               quantises x (or silu(g)*u) from shared memory into the
//               swizzled B tile and publishes sx; P K blocks are quantised
//               at once.
//   warps 6-9   epilogue: TMEM -> registers, scale, accumulate, store.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "fp8gq_device.cuh"

namespace fp8gq {

constexpr int kTmThreads = 320;
constexpr int kTmMaxAcc = 4;        // TMEM accumulator buffers (columns reserved for 4)
constexpr int kTmSxRing = 64;       // > stages + accumulators * K blocks per group
static_assert((kTmSxRing & (kTmSxRing - 1)) == 0, "the sx ring is indexed with a mask");
constexpr int kTmATileBytes = 128 * 128;
// The workspace starts with one split-K counter per 128-row block, in a region
// of fixed size so that the partial sums of one shape never land on the
// counters of another shape that shares the workspace.
constexpr int kTmMaxRowBlocks = 4096;                       // N <= 524288
constexpr size_t kTmCounterBytes = static_cast<size_t>(kTmMaxRowBlocks) * 4;
constexpr size_t kTmSmemBudgetSm = 228 * 1024;   // shared memory per SM
constexpr size_t kTmSmemReservedPerCta = 1024;   // what the runtime keeps per resident CTA

// CTAs per SM: the 16-token tile runs two per SM (two MMA issue streams and
// two pipelines per SM; its registers and TMEM columns allow it), the wider
// token tiles one.
template <int MT>
constexpr int tm_ctas_per_sm() { return MT == 16 ? 2 : 1; }
constexpr int kTmWsCache = 512;     // block scales of the CTA's tiles kept in shared memory

struct TmParams {
  const float* ws;          // [N/128, ldws]
  int64_t ldws;
  __nv_bfloat16* out;       // [M, ldo]
  int64_t ldo;
  int M;                    // valid tokens in this pass (<= MT)
  int sw;                   // token slot width: next power of two >= M (MT == 16), else MT
  int lg_sw;                // log2(sw)
  int kpb;                  // K blocks per accumulator group = MT / sw
  int nacc;                 // accumulator buffers in use (<= kTmMaxAcc)
  int stages;               // ring depth
  int N, K;
  int KB;                   // K / 128
  int64_t U;                // (N/128) * KB tiles
  uint32_t x_tile_bytes;    // bytes of one activation box (M rows x 128 bf16)
  int early_weights;        // weights and block scales are static: load them before the grid-dependency wait
  int* counters;            // [kTmMaxRowBlocks], zero on entry and exit
  float* partials;          // [G][2][MT][128]
  uint8_t* xq_out;          // optional [M, K]
  float* sx_out;            // optional [M, K/128]
};

template <int MT, bool kSwiglu>
struct TmCfg {
  static constexpr int kCtasPerSm = tm_ctas_per_sm<MT>();
  static constexpr size_t kTmSmemBudget =
      (kTmSmemBudgetSm / kCtasPerSm - kTmSmemReservedPerCta) < 227 * 1024
          ? (kTmSmemBudgetSm / kCtasPerSm - kTmSmemReservedPerCta) : 227 * 1024;
  static constexpr int kBTileBytes = MT * 128;
  static constexpr int kXTileBytes = MT * 256 * (kSwiglu ? 2 : 1);   // room for MT rows
  static constexpr int kStageBytes = kTmATileBytes + kBTileBytes + kXTileBytes;
  static constexpr int kTmemCols = (kTmMaxAcc * MT <= 32) ? 32 : (kTmMaxAcc * MT <= 64) ? 64
                                   : (kTmMaxAcc * MT <= 128) ? 128 : 256;
  static constexpr int kNumBars = 3 * 8 /*full, xfull, empty*/ + 2 * kTmMaxAcc + kTmSxRing + 1;
  static constexpr size_t kFixedBytes = kNumBars * 8 + 16 + kTmSxRing * MT * 4 + kTmWsCache * 4 + 1024;
  static constexpr int kFit =
      ((kTmSmemBudget - kFixedBytes) / kStageBytes) < 8 ? static_cast<int>((kTmSmemBudget - kFixedBytes) / kStageBytes)
                                                        : 8;
  // The activation warps take K blocks round robin; their number divides the
  // ring depth, so every stage is only ever waited on by one of them, use
  // after use, and a phase-parity wait can never see a stale phase.
  static constexpr int kStages = kFit >= 4 ? (kFit / 4) * 4 : kFit;
  static constexpr int kProducerWarps = kStages >= 4 ? 4 : kStages;
  // ring | full[8] xfull[8] empty[8] acc_full[ACC] tmem_empty[ACC] sx_tag[SXR] (8 B each) drain | misc
  //      | sx ring | ws cache
  static constexpr size_t kBarOffset = static_cast<size_t>(kStages) * kStageBytes;
  static constexpr size_t kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr size_t kSxOffset = kMiscOffset + 16;
  static constexpr size_t kWsOffset = kSxOffset + kTmSxRing * MT * 4;
  static constexpr size_t kSmemBytes = kWsOffset + kTmWsCache * 4 + 1024;  // +1 KB alignment slack
  static_assert(kStages >= 2, "stage ring does not fit in shared memory");
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

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
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

// Poll a shared-memory tag until it equals `want` (bounded like mbar_wait).
__device__ __forceinline__ bool tag_wait(volatile uint32_t* tag, uint32_t want) {
  if (*tag == want) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (*tag == want) return true;
    if ((it & 255u) == 0u && global_ns() - t0 > kWaitLimitNs) {
      record_error(kSiteTmAcc);
      return false;
    }
  }
}

__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

// Walks a CTA's tiles in order with no integer division on the way (the
// issuing roles are single threads, so their loop bodies must stay short).
// pos is the tile's place inside its accumulator group: groups are runs of
// kpb consecutive K blocks that never cross a row-block boundary.
struct TileCursor {
  int nb, kb, pos;     // row block, K block, position in the accumulator group
  int s;               // stage of the ring
  uint32_t ph;         // parity of that stage's current use
  __device__ __forceinline__ void init(int64_t u0, int KB) {
    nb = static_cast<int>(u0 / KB);
    kb = static_cast<int>(u0 - static_cast<int64_t>(nb) * KB);
    pos = 0;
    s = 0;
    ph = 0;
  }
  __device__ __forceinline__ void next(int KB, int kpb, int S) {
    if (++kb == KB) {
      kb = 0;
      ++nb;
      pos = 0;
    } else {
      pos = (pos + 1 == kpb) ? 0 : pos + 1;
    }
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
  }
};

// Accumulator buffer of the current group and the parity of its use.
struct AccCursor {
  int g = -1, a = -1;
  uint32_t round = 0;
  __device__ __forceinline__ void start_group(int nacc) {
    ++g;
    if (++a == nacc) {
      a = 0;
      round ^= 1u;
    }
  }
};

// ------------------------------------------------------------- kernel --
template <int MT, bool kSwiglu>
__global__ void __launch_bounds__(kTmThreads, tm_ctas_per_sm<MT>())
gemm_tm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
               const TmParams p) {
  using Cfg = TmCfg<MT, kSwiglu>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* xfull = full + 8;
  uint64_t* empty = xfull + 8;
  uint64_t* acc_full = empty + 8;
  uint64_t* tmem_empty = acc_full + kTmMaxAcc;
  // sequence tags: sx_tag[j % ring] = j + 1 once K block j's scales are in the
  // sx ring (a plain shared-memory flag; the epilogue polls it)
  volatile uint32_t* sx_tag = reinterpret_cast<volatile uint32_t*>(tmem_empty + kTmMaxAcc);
  uint64_t* drain = tmem_empty + kTmMaxAcc + kTmSxRing;  // MMA completion on the error path
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOffset);  // [0] tmem base, [1] last flag
  float* sx_ring = reinterpret_cast<float*>(smem + Cfg::kSxOffset);      // [kTmSxRing][MT]
  float* ws_cache = reinterpret_cast<float*>(smem + Cfg::kWsOffset);     // [min(J, kTmWsCache)]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int64_t G = gridDim.x;
  const int64_t u0 = (static_cast<int64_t>(blockIdx.x) * p.U) / G;
  const int64_t u1 = (static_cast<int64_t>(blockIdx.x + 1) * p.U) / G;
  const int J = static_cast<int>(u1 - u0);
  const int kpb = p.kpb;
  const int nacc = p.nacc;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1 + 1);    // TMA arrive_expect_tx + the activation warp of the K block
      mbar_init(&xfull[s], 1);       // TMA arrive_expect_tx (activation tile)
      mbar_init(&empty[s], 1);       // tcgen05.commit
    }
    for (int a = 0; a < kTmMaxAcc; ++a) {
      mbar_init(&acc_full[a], 1);    // tcgen05.commit
      mbar_init(&tmem_empty[a], 4);  // 4 epilogue warps
    }
    for (int r = 0; r < kTmSxRing; ++r) sx_tag[r] = 0u;
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

  // Block scales of this CTA's tiles, ws_cache[j] = ws[nb(j), kb(j)] (the host
  // launches only shapes with J <= kTmWsCache), and -- when the caller declared
  // the weights static -- the weight tiles of the first ring of stages are
  // fetched before the grid-dependency wait, overlapping the previous kernel's
  // tail.  Activations, outputs and the workspace are touched only after it.
  const bool early = p.early_weights != 0;
  const int n_pre = early ? (J < S ? J : S) : 0;
  auto load_ws_cache = [&]() {
    for (int j = tid; j < J; j += kTmThreads) {
      const int64_t u = u0 + j;
      ws_cache[j] = __ldg(p.ws + (u / p.KB) * p.ldws + (u % p.KB));
    }
  };
  if (early) {
    load_ws_cache();
    if (tid == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      TileCursor c;
      c.init(u0, p.KB);
      for (int j = 0; j < n_pre; ++j, c.next(p.KB, kpb, S)) {
        mbar_arrive_expect_tx(&full[c.s], kTmATileBytes);
        tma_load_2d(smem + c.s * Cfg::kStageBytes, &tmap_w, c.kb * 128, c.nb * 128, &full[c.s], pol_w);
      }
    }
  }
  grid_dependency_wait();
  if (!early) load_ws_cache();
  __syncthreads();

  if (warp == 0) {
    // --------------------------------------------------- TMA producer --
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const uint32_t xbytes = p.x_tile_bytes * (kSwiglu ? 2u : 1u);
      int issued = 0;
      TileCursor c;
      c.init(u0, p.KB);
      for (int j = 0; j < J && ok; ++j, c.next(p.KB, kpb, S)) {
        const int s = c.s;
        if (j >= S) ok = mbar_wait(&empty[s], c.ph ^ 1u, kSiteTmA);
        if (!ok) break;
        uint8_t* stage = smem + s * Cfg::kStageBytes;
        uint8_t* xt = stage + kTmATileBytes + Cfg::kBTileBytes;
        if (j >= n_pre) {
          mbar_arrive_expect_tx(&full[s], kTmATileBytes);
          tma_load_2d(stage, &tmap_w, c.kb * 128, c.nb * 128, &full[s], pol_w);
        }
        mbar_arrive_expect_tx(&xfull[s], xbytes);
        tma_load_2d(xt, &tmap_x, c.kb * 128, 0, &xfull[s], pol_x);
        if constexpr (kSwiglu) tma_load_2d(xt + p.x_tile_bytes, &tmap_x, p.K + c.kb * 128, 0, &xfull[s], pol_x);
        issued = j + 1;
      }
      grid_launch_dependents();
      if (!ok) {
        // let the copies already issued land before the CTA can exit
        for (int j = (issued > S ? issued - S : 0); j < issued; ++j) {
          mbar_wait(&full[j % S], (j / S) & 1, kSiteTmA);
          mbar_wait(&xfull[j % S], (j / S) & 1, kSiteTmA);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------- MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = idesc_f8<MT>();
      // descriptors of stage 0's A tile; a stage, a K step and the B tile are
      // offsets in the 14-bit start-address field (addresses < 256 KB)
      const uint64_t desc0 = smem_desc_sw128(smem_u32(smem));
      AccCursor acc;
      uint32_t d_tmem = tmem_base;
      TileCursor c;
      c.init(u0, p.KB);
      for (int j = 0; j < J && ok; ++j, c.next(p.KB, kpb, S)) {
        if (c.pos == 0) {
          acc.start_group(nacc);
          if (acc.g >= nacc) ok = mbar_wait(&tmem_empty[acc.a], acc.round ^ 1u, kSiteTmTmem);
          if (!ok) break;
          d_tmem = tmem_base + static_cast<uint32_t>(acc.a * MT);
        }
        ok = mbar_wait(&full[c.s], c.ph, kSiteTmB);
        if (!ok) break;
        tc_fence_after();
        const uint64_t da = desc0 + static_cast<uint64_t>((c.s * Cfg::kStageBytes) >> 4);
        const uint64_t db = da + (kTmATileBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8(d_tmem, da + 2 * kk, db + 2 * kk, idesc, (c.pos > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&empty[c.s]);
        const bool group_end = (c.pos == kpb - 1) || (c.kb == p.KB - 1) || (j == J - 1);
        if (group_end) mma_commit(&acc_full[acc.a]);
      }
      if (!ok) {
        // wait for every MMA issued so far before TMEM can be released
        mma_commit(drain);
        mbar_wait(drain, 0, kSiteTmB);
      }
    }
  } else if (warp < 6) {
    // ----------------------------------------- activation producers --
    // Lane l covers the 16-byte chunk l % 8 of B-tile rows l / 8 + 4 i.
    constexpr int NPW = Cfg::kProducerWarps;  // this warp takes j = w4, w4 + NPW, ...
    const int w4 = warp - 2;
    const int chunk = lane & 7;         // 16-byte chunk of the 128-wide K block
    const int row0 = lane >> 3;         // 0..3
    TileCursor c;
    c.init(u0, p.KB);
    for (int k = 0; k < w4; ++k) c.next(p.KB, kpb, S);
    for (int j = w4; w4 < NPW && j < J && ok; j += NPW) {
      if (j > w4) {
        for (int k = 0; k < NPW; ++k) c.next(p.KB, kpb, S);
      }
      const int s = c.s;
      ok = mbar_wait(&xfull[s], c.ph, kSiteTmA);
      if (!ok) break;
      const int nb = c.nb;
      const int kb = c.kb;
      const int pos = c.pos;
      uint8_t* stage = smem + s * Cfg::kStageBytes;
      uint8_t* btile = stage + kTmATileBytes;
      const __nv_bfloat16* xt = reinterpret_cast<const __nv_bfloat16*>(btile + Cfg::kBTileBytes);
      float* sxs = sx_ring + (j & (kTmSxRing - 1)) * MT;
#pragma unroll
      for (int i = 0; i < MT / 4; ++i) {
        const int br = row0 + 4 * i;           // row of the B tile (a token column of the MMA)
        const int m = br - pos * p.sw;         // token held by this row in K block slot `pos`
        const bool live = m >= 0 && m < p.sw && m < p.M;
        uint4 packed = make_uint4(0u, 0u, 0u, 0u);
        if (__any_sync(0xffffffffu, live)) {   // rows of a lane octet are all live or all not
          float v[16];
          if (live) {
            const __nv_bfloat16* xr = xt + m * 128 + chunk * 16;
            if constexpr (kSwiglu) {
              const uint4* gp = reinterpret_cast<const uint4*>(xr);
              const uint4* up = reinterpret_cast<const uint4*>(xr + p.x_tile_bytes / 2);
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
          if (live) {
            const float sx = group_scale(amax);
            const float sinv = __frcp_rn(sx);
            packed.x = quant_pair(v[0], v[1], sinv) | (static_cast<uint32_t>(quant_pair(v[2], v[3], sinv)) << 16);
            packed.y = quant_pair(v[4], v[5], sinv) | (static_cast<uint32_t>(quant_pair(v[6], v[7], sinv)) << 16);
            packed.z = quant_pair(v[8], v[9], sinv) | (static_cast<uint32_t>(quant_pair(v[10], v[11], sinv)) << 16);
            packed.w = quant_pair(v[12], v[13], sinv) | (static_cast<uint32_t>(quant_pair(v[14], v[15], sinv)) << 16);
            if (chunk == 0) sxs[m] = sx;
            if (nb == 0) {
              if (p.xq_out)
                *reinterpret_cast<uint4*>(p.xq_out + static_cast<int64_t>(m) * p.K + kb * 128 + chunk * 16) = packed;
              if (p.sx_out && chunk == 0) p.sx_out[static_cast<int64_t>(m) * p.KB + kb] = sx;
            }
          }
        }
        *reinterpret_cast<uint4*>(btile + br * 128 + ((chunk ^ (br & 7)) << 4)) = packed;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full[s]);
        __threadfence_block();
        sx_tag[j & (kTmSxRing - 1)] = static_cast<uint32_t>(j + 1);
      }
    }
  } else {
    // -------------------------------------------------------- epilogue --
    const int q4 = warp & 3;                 // TMEM lane quarter of this warp
    const int row = 32 * q4 + lane;          // weight row within the 128-row block
    const uint32_t t_lane = static_cast<uint32_t>(32 * q4) << 16;
    float acc[MT];                           // per TMEM column: token c % sw of slot c / sw
#pragma unroll
    for (int c = 0; c < MT; ++c) acc[c] = 0.0f;
    int seg_j0 = 0, seg_kb0 = 0;
    AccCursor accc;
    TileCursor cur;
    cur.init(u0, p.KB);
    for (int j = 0; j < J; ++j, cur.next(p.KB, kpb, S)) {
      const int nb = cur.nb;
      const int kb = cur.kb;
      const int pos = cur.pos;
      if (pos == 0) accc.start_group(nacc);
      if (j == 0 || kb == 0) {
        seg_j0 = j;
        seg_kb0 = kb;
#pragma unroll
        for (int c = 0; c < MT; ++c) acc[c] = 0.0f;
      }
      const bool group_end = (pos == kpb - 1) || (kb == p.KB - 1) || (j == J - 1);
      if (!group_end) continue;
      const int a = accc.a;
      if (ok) ok = mbar_wait(&acc_full[a], accc.round, kSiteTmAcc);
      if (lane == 0) {
        for (int q = 0; q <= pos && ok; ++q) ok = tag_wait(sx_tag + ((j - pos + q) & (kTmSxRing - 1)),
                                                         static_cast<uint32_t>(j - pos + q + 1));
        __threadfence_block();
      }
      ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
      tc_fence_after();
      const int jq0 = j - pos;                 // first K block of the group
#pragma unroll
      for (int c16 = 0; c16 < MT / 16; ++c16) {
        float v[16];
        if (ok) {
          tmem_ld16(tmem_base + t_lane + static_cast<uint32_t>(a * MT + 16 * c16), v);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c = 16 * c16 + i;
          const int q = c >> p.lg_sw;
          const int m = c & (p.sw - 1);
          if (q <= pos && m < p.M) {
            const float sxv = sx_ring[((jq0 + q) & (kTmSxRing - 1)) * MT + m];
            const float wsv = ws_cache[jq0 + q];
            acc[c] = fmaf(v[i], sxv * wsv, acc[c]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[a]);

      if (kb == p.KB - 1 || j == J - 1) {
        // fold the K-block slots: column m then holds token m's sum
#pragma unroll
        for (int h = MT / 2; h >= 1; h >>= 1)
          if (p.sw <= h) {
#pragma unroll
            for (int c = 0; c < h; ++c) acc[c] += acc[c + h];
          }
        const int n = nb * 128 + row;
        const bool whole = seg_kb0 == 0 && kb == p.KB - 1;
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
          // the barrier orders every epilogue thread's partial stores before the
          // release half of the counter update; its acquire half orders the
          // reduction's loads of the other CTAs' partials after their stores
          named_bar_sync(2, 128);
          const int64_t first_u = static_cast<int64_t>(nb) * p.KB;
          const int64_t last_u = first_u + p.KB - 1;
          const int64_t i_lo = ((first_u + 1) * G - 1) / p.U;
          const int64_t i_hi = ((last_u + 1) * G - 1) / p.U;
          if (tid == 192) {
            const int old = atomic_add_acq_rel_gpu(&p.counters[nb], 1);
            const bool last = (old == static_cast<int>(i_hi - i_lo));
            misc[1] = last ? 1u : 0u;
            if (last) p.counters[nb] = 0;
          }
          named_bar_sync(2, 128);
          if (misc[1]) {
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

// Resident CTA slots for the token tile (the most CTAs one launch may use).
inline int tm_slots(int sm_count, int MT) { return sm_count * (MT == 16 ? tm_ctas_per_sm<16>() : 1); }

// Grid size.  Preferred: an aligned split -- every CTA takes one row block's
// K range cut in S equal parts (S a power of two dividing K/128), so the
// split-K hand-off involves only the S CTAs of a row block and S = 1 needs
// none -- with NB * S the largest such count <= 1.3 x SMs (measured on B200:
// about one CTA per SM with long K runs beats two with short runs plus
// hand-offs).  Otherwise stream-K over all resident slots.
inline int tm_grid(int64_t U, int sm_count, int MT, int NB = 0, int KB = 0) {
  const int64_t slots = tm_slots(sm_count, MT);
  if (NB > 0 && KB > 0) {
    const int64_t cap = (static_cast<int64_t>(sm_count) * 13) / 10;
    int64_t best = 0;
    for (int S = 1; S <= KB; S *= 2)
      if (KB % S == 0 && static_cast<int64_t>(NB) * S <= cap && static_cast<int64_t>(NB) * S <= slots)
        best = static_cast<int64_t>(NB) * S;
    if (best >= sm_count / 2) return static_cast<int>(best);
  }
  return static_cast<int>(U < slots ? U : slots);
}

inline size_t tm_workspace_bytes_for(int M, int N, int K, int sm_count) {
  const int MT = tm_token_tile(M);
  const int64_t U = static_cast<int64_t>(N / kGroup) * (K / kGroup);
  const int G = tm_slots(sm_count, MT) < U ? tm_slots(sm_count, MT) : static_cast<int>(U);
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

// Activation tensor map: 2-D bf16 [rows, cols] with row stride ldx elements,
// box 128 columns x `rows` rows, no swizzle (rows land 256 bytes apart).
inline bool make_act_tmap(CUtensorMap* map, const void* x, int rows, int64_t cols, int64_t ldx) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldx) * 2};
  cuuint32_t box[2] = {128, static_cast<cuuint32_t>(rows)};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MT, bool S>
int launch_tm_pass(const CUtensorMap& tw, const CUtensorMap& tx, TmParams p, int grid, int max_smem,
                   cudaStream_t stream) {
  using Cfg = TmCfg<MT, S>;
  if (Cfg::kSmemBytes > static_cast<size_t>(max_smem)) return 8;  // FP8GQ_ERR_UNSUPPORTED
  auto fn = gemm_tm_kernel<MT, S>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(Cfg::kSmemBytes)) != cudaSuccess)
    return 7;  // FP8GQ_ERR_LAUNCH
  p.stages = Cfg::kStages;
  if (launch_with_pdl(fn, dim3(grid), dim3(kTmThreads), Cfg::kSmemBytes, stream, tw, tx, p) != cudaSuccess)
    return 7;
  return cudaGetLastError() == cudaSuccess ? 0 : 7;
}

// Runs ceil(M / MT) passes of at most MT tokens; every pass reuses the
// workspace (its counters are zero again when a pass ends).
inline int launch_tm(bool swiglu, const void* x, int64_t ldx, const void* w, int64_t ldw, const float* ws,
                     int64_t ldws, void* out, int64_t ldo, int M, int N, int K, uint8_t* xq_out,
                     float* sx_out, void* workspace, size_t workspace_bytes, int sm_count, int max_smem,
                     cudaStream_t stream, int early_weights = 0, int grid_override = 0) {
  const int MT = tm_token_tile(M);
  if (N / kGroup > kTmMaxRowBlocks) return 8;  // FP8GQ_ERR_UNSUPPORTED
  const size_t need = tm_workspace_bytes_for(M, N, K, sm_count);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return 5;  // FP8GQ_ERR_WORKSPACE
  CUtensorMap tmap_w;
  if (!make_weight_tmap(&tmap_w, w, N, K, ldw)) return 7;
  TmParams p;
  p.ws = ws;
  p.ldws = ldws;
  p.ldo = ldo;
  p.N = N;
  p.K = K;
  p.KB = K / kGroup;
  p.U = static_cast<int64_t>(N / kGroup) * p.KB;
  p.counters = static_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kTmCounterBytes);
  const int grid = grid_override > 0 ? (grid_override < p.U ? grid_override : static_cast<int>(p.U))
                                      : tm_grid(p.U, sm_count, MT, N / kGroup, p.KB);
  if (grid > tm_slots(sm_count, MT)) return 8;  // partial-sum slots exist for at most this many CTAs
  if ((p.U + grid - 1) / grid + 1 > kTmWsCache) return 8;  // FP8GQ_ERR_UNSUPPORTED: tiles per CTA
  const int64_t xcols = swiglu ? 2 * static_cast<int64_t>(K) : K;
  for (int m0 = 0; m0 < M; m0 += MT) {
    const __nv_bfloat16* xp = static_cast<const __nv_bfloat16*>(x) + static_cast<int64_t>(m0) * ldx;
    p.out = static_cast<__nv_bfloat16*>(out) + static_cast<int64_t>(m0) * ldo;
    p.M = (M - m0 < MT) ? (M - m0) : MT;
    int sw = 1, lg = 0;
    if (MT == 16) {
      while (sw < p.M) { sw <<= 1; ++lg; }
    } else {
      sw = MT;
      lg = (MT == 32) ? 5 : 6;
    }
    p.sw = sw;
    p.lg_sw = lg;
    p.kpb = MT / sw;
    p.nacc = p.kpb >= 8 ? 2 : kTmMaxAcc;
    p.x_tile_bytes = static_cast<uint32_t>(p.M) * 256u;
    p.early_weights = early_weights;
    p.xq_out = xq_out ? xq_out + static_cast<int64_t>(m0) * K : nullptr;
    p.sx_out = sx_out ? sx_out + static_cast<int64_t>(m0) * (K / kGroup) : nullptr;
    CUtensorMap tmap_x;
    if (!make_act_tmap(&tmap_x, xp, p.M, xcols, ldx)) return 7;
    int st;
    if (MT == 16)
      st = swiglu ? launch_tm_pass<16, true>(tmap_w, tmap_x, p, grid, max_smem, stream)
                  : launch_tm_pass<16, false>(tmap_w, tmap_x, p, grid, max_smem, stream);
    else if (MT == 32)
      st = swiglu ? launch_tm_pass<32, true>(tmap_w, tmap_x, p, grid, max_smem, stream)
                  : launch_tm_pass<32, false>(tmap_w, tmap_x, p, grid, max_smem, stream);
    else
      st = swiglu ? launch_tm_pass<64, true>(tmap_w, tmap_x, p, grid, max_smem, stream)
                  : launch_tm_pass<64, false>(tmap_w, tmap_x, p, grid, max_smem, stream);
    if (st) return st;
  }
  return 0;
}

}  // namespace fp8gq
