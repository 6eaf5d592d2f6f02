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
// Activation modes.  Streaming: each stage also carries the bf16 activation
// tile of its K block (TMA), which an activation warp quantises into the B
// tile once it lands.  Resident (the host picks it when the CTA's M x K-range
// bytes fit in the ring's activation space, e.g. every M = 1 decode shape):
// after the grid-dependency wait the CTA quantises its whole K range once
// into shared memory, and an activation warp only copies the prebuilt bytes
// into a stage's B tile as soon as the MMA has released that stage -- the B
// tile is ready long before the weight tile lands, so only the weight stream
// is on the critical path.
//
// Warp roles (320 threads):
//   warp 0      TMA producer: the 128x128-byte weight tile (SWIZZLE_128B) and,
//               streaming, the bf16 activation tile(s) of the K block (no
//               multicast).  Starts right after the grid-dependency wait.
//   warp 1      TMEM allocator and MMA issuer (one elected lane).
//   warps 2-5   activation producers: with P of them active (P divides the
//               ring depth), warp w takes the CTA's K blocks j = w-2 mod P and
//               fills their B tiles (and, streaming, publishes sx).
//   warps 6-9   epilogue: TMEM -> registers, scale, accumulate, store.
//   Warps 2-9 also load the CTA's block scales and, resident, quantise the
//   activation in the prologue.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <tuple>

#include "fp8gq_device.cuh"
#include "quant_only.cuh"

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

constexpr int kTmMaxStages = 8;     // ring depth limit (barrier arrays are sized for it)
constexpr int kTmMaxCluster = 16;   // largest split-K cluster (16: B200's non-portable size)
constexpr int64_t kTmPushMaxBytes = 16 * 1024;   // largest receive area of a split-K reduction by push
constexpr int kTmMaxPortableCluster = 8;   // clusters above this need the non-portable attribute

// CTAs per SM the 16-token tile may run at (two MMA issue streams and two
// pipelines per SM; its registers and TMEM columns allow it); the wider token
// tiles run one.  A grid of at most one CTA per SM gets the whole SM's shared
// memory instead, for a deeper ring.
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
  int stages;               // ring depth S (<= kTmMaxStages)
  int npw;                  // activation warps in use (divides S)
  uint32_t b_off, x_off, bar_off;   // shared-memory layout (bytes from the 1 KB-aligned base)
  int N, K;
  int KB;                   // K / 128
  int64_t U;                // (N/128) * KB tiles
  uint32_t x_tile_bytes;    // bytes of one activation box (M rows x 128 bf16)
  const __nv_bfloat16* x;   // activation rows of this pass (resident mode reads them directly)
  int64_t ldx;
  int resident;             // resident activation mode
  int prequant;             // pre-quantised feed: B tiles by TMA from xq (tmap_x), scales from sx_pre
  const float* sx_pre;      // [M, K/128] scales of the pre-quantised activation
  int csize;                // split-K cluster size (1: none; the CTAs of a row block form a cluster)
  int red_push;             // cluster split-K by push: the other CTAs copy their partials to rank 0
  uint32_t red_off;         // push: rank 0's receive area [csize - 1][M][128] fp32 (bytes from the base)
  int early_weights;        // weights and block scales are static: load them before the grid-dependency wait
  int* counters;            // [kTmMaxRowBlocks], zero on entry and exit
  float* partials;          // [G][2][MT][128]
  uint8_t* xq_out;          // optional [M, K]
  float* sx_out;            // optional [M, K/128]
  GatherParams gather;      // N-sharded output written to every rank (world > 0)
  NormParams norm;          // add + RMSNorm prologue (resident activation only)
};

// Shared memory, from the 1 KB-aligned base:
//   A tiles [S][16 KB] | B tiles [S][MT x 128 B] | activation region (streaming:
//   [S] bf16 tiles; resident: xq of the K range) | full[8] xfull[8] empty[8]
//   acc_full[ACC] tmem_empty[ACC] sx_tag[SXR] (8 B each) drain | misc[4] |
//   sx ring (resident: sx of the K range) | ws cache | add + RMSNorm sums
// In cluster mode the A-tile area holds the CTA's split-K partial sums once
// its MMAs are done.
template <int MT, bool kSwiglu>
struct TmCfg {
  static constexpr int kBTileBytes = MT * 128;
  static constexpr int kXTileBytes = MT * 256 * (kSwiglu ? 2 : 1);   // room for MT rows
  static constexpr int kTmemCols = (kTmMaxAcc * MT <= 32) ? 32 : (kTmMaxAcc * MT <= 64) ? 64
                                   : (kTmMaxAcc * MT <= 128) ? 128 : 256;
  static constexpr int kNumBars = 3 * kTmMaxStages /*full, xfull, empty*/ + 2 * kTmMaxAcc + kTmSxRing + 1;
  static constexpr size_t kTailBytes = kNumBars * 8 + 16 + kTmSxRing * MT * 4 + kTmWsCache * 4;
  static constexpr size_t kAlignSlack = 1024;
  static_assert(kBTileBytes % 1024 == 0, "SW128 tiles need 1 KB alignment");
  static_assert(MT * 128 * 4 <= 2 * kTmATileBytes, "cluster partial sums must fit in two A tiles");
};

// Ring depth from the bytes left for it: 8, 6, 4, 3, 2 or 1 stages, so that
// the activation warps (4, 3, 4, 3, 2, 1 of them) divide the depth -- each
// stage is then only ever waited on by one of them, use after use, and a
// phase-parity wait can never see a stale phase.
inline int tm_pick_stages(int64_t fit) {
  return fit >= 8 ? 8 : fit >= 6 ? 6 : fit >= 4 ? 4 : static_cast<int>(fit < 0 ? 0 : fit);
}
inline int tm_producer_warps(int S) { return S % 4 == 0 ? 4 : S % 3 == 0 ? 3 : S; }

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

// Fetch a tensor map (a __grid_constant__ kernel parameter) into the TMA
// descriptor cache ahead of its first use.
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Cluster-wide barrier: every thread of every CTA of the cluster arrives; the
// release/acquire pair orders shared-memory writes before it with
// distributed-shared-memory reads after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared-memory address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
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
    if ((it & 255u) == 0u && global_ns() - t0 > wait_limit_ns()) {
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
  __device__ __forceinline__ void init(int nb0, int kb0) {
    nb = nb0;
    kb = kb0;
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

// 16 activation values of one lane from two 16-byte words of bf16 (and, for
// SwiGLU, the two matching words of the up half): act = silu(g) * u.
template <bool kSwiglu>
__device__ __forceinline__ void act16(float (&v)[16], uint4 a, uint4 b, uint4 ua, uint4 ub) {
  const uint32_t xw[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  if constexpr (kSwiglu) {
    const uint32_t uw[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[2 * e] = silu_mul(bf16_lo(xw[e]), bf16_lo(uw[e]));
      v[2 * e + 1] = silu_mul(bf16_hi(xw[e]), bf16_hi(uw[e]));
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[2 * e] = bf16_lo(xw[e]);
      v[2 * e + 1] = bf16_hi(xw[e]);
    }
  }
}

// Group quant over a lane octet (8 lanes x 16 values = one 128-wide group):
// octet amax by shuffles, then this lane's 16 e4m3 bytes and the group scale.
// All 32 lanes call it together; `live` is uniform within an octet (a dead
// octet holds zeros and returns zeros).
__device__ __forceinline__ uint4 quant16_octet(const float (&v)[16], bool live, float& sx) {
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[e]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  uint4 packed = make_uint4(0u, 0u, 0u, 0u);
  sx = 0.0f;
  if (live) {
    sx = group_scale(amax);
    const float sinv = __frcp_rn(sx);
    packed.x = quant_pair(v[0], v[1], sinv) | (static_cast<uint32_t>(quant_pair(v[2], v[3], sinv)) << 16);
    packed.y = quant_pair(v[4], v[5], sinv) | (static_cast<uint32_t>(quant_pair(v[6], v[7], sinv)) << 16);
    packed.z = quant_pair(v[8], v[9], sinv) | (static_cast<uint32_t>(quant_pair(v[10], v[11], sinv)) << 16);
    packed.w = quant_pair(v[12], v[13], sinv) | (static_cast<uint32_t>(quant_pair(v[14], v[15], sinv)) << 16);
  }
  return packed;
}

// Reads every field of the parameter block once.  A parameter's first use in
// a warp can stall it for several hundred cycles (constant-cache miss); doing
// them all at kernel entry, before the grid-dependency wait, moves those
// misses off the pipeline's critical path.
__device__ __forceinline__ void tm_touch_params(const TmParams& p) {
  uint64_t t = reinterpret_cast<uint64_t>(p.ws) ^ static_cast<uint64_t>(p.ldws) ^
               reinterpret_cast<uint64_t>(p.out) ^ static_cast<uint64_t>(p.ldo) ^
               reinterpret_cast<uint64_t>(p.x) ^ static_cast<uint64_t>(p.ldx) ^ static_cast<uint64_t>(p.U) ^
               reinterpret_cast<uint64_t>(p.counters) ^ reinterpret_cast<uint64_t>(p.partials) ^
               reinterpret_cast<uint64_t>(p.xq_out) ^ reinterpret_cast<uint64_t>(p.sx_out);
  uint32_t u = static_cast<uint32_t>(p.M ^ p.sw ^ p.lg_sw ^ p.kpb ^ p.nacc ^ p.stages ^ p.npw ^ p.N ^ p.K ^ p.KB ^
                                     p.resident ^ p.csize ^ p.early_weights ^ p.gather.world ^
                                     p.gather.wait_input ^ p.norm.norm ^ p.prequant) ^
               p.b_off ^ p.x_off ^ p.bar_off ^ p.x_tile_bytes;
  asm volatile("" ::"l"(t), "r"(u));
}

// Place of the CTA's tile j in its accumulator group (TileCursor::pos after j
// steps from the CTA's first tile, K block kb0): groups restart at the CTA's
// first tile and at every row-block boundary.
__device__ __forceinline__ int tile_pos(int j, int kb0, int KB, int kpb) {
  const int t = kb0 + j;
  const int jstart = t < KB ? 0 : j - t % KB;
  return (j - jstart) & (kpb - 1);
}

// ------------------------------------------------------------- kernel --
// kTagged: the gather uses tagged words; kCluster: a cluster split-K launch
// (csize > 1).  Separate instances, so that each kernel carries only the code
// of its own protocol and reduction.
template <int MT, bool kSwiglu, bool kTagged = false, bool kCluster = false>
__global__ void __launch_bounds__(kTmThreads, tm_ctas_per_sm<MT>())
gemm_tm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
               const TmParams p) {
  using Cfg = TmCfg<MT, kSwiglu>;
  const int S = p.stages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* const a_tiles = smem;                       // [S][128 x 128 B] weight tiles
  uint8_t* const b_tiles = smem + p.b_off;             // [S][MT x 128 B] quantised activation tiles
  // streaming: [S] bf16 activation tiles; resident: xq of the K range, [slot][M][128 B]
  uint8_t* const x_tiles = smem + p.x_off;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* xfull = full + kTmMaxStages;
  uint64_t* empty = xfull + kTmMaxStages;
  uint64_t* acc_full = empty + kTmMaxStages;
  uint64_t* tmem_empty = acc_full + kTmMaxAcc;
  // sequence tags: sx_tag[j % ring] = j + 1 once K block j's scales are in the
  // sx ring (a plain shared-memory flag; the epilogue polls it)
  volatile uint32_t* sx_tag = reinterpret_cast<volatile uint32_t*>(tmem_empty + kTmMaxAcc);
  uint64_t* drain = tmem_empty + kTmMaxAcc + kTmSxRing;  // MMA completion on the error path
  uint32_t* misc = reinterpret_cast<uint32_t*>(drain + 1);  // [0] tmem base, [1] last flag, [2..3] red_full
  uint64_t* red_full = reinterpret_cast<uint64_t*>(misc + 2);  // push: the other ranks' partials have landed
  // streaming: [kTmSxRing][MT] ring indexed by j; resident: [slot][M]
  float* sx_ring = reinterpret_cast<float*>(misc + 4);
  float* ws_cache = sx_ring + kTmSxRing * MT;          // [min(J, kTmWsCache)]
  float* norm_sum = ws_cache + kTmWsCache;             // add + RMSNorm: [M][K/128] group sums, then rstd [M]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  tm_touch_params(p);

  const int64_t G = gridDim.x;
  const int64_t u0 = (static_cast<int64_t>(blockIdx.x) * p.U) / G;
  const int64_t u1 = (static_cast<int64_t>(blockIdx.x + 1) * p.U) / G;
  const int J = static_cast<int>(u1 - u0);
  const int kpb = p.kpb;
  const int nacc = p.nacc;
  // Resident K range: a CTA whose tiles cover a whole row block's K range
  // (J >= KB) keeps every K block, slot = kb; otherwise its J tiles have J
  // distinct K blocks (kb0, kb0 + 1, ... mod KB), slot = j.
  const bool resident = p.resident != 0;
  // Pre-quantised feed (large M, where the resident feed does not fit and
  // every CTA would otherwise quantise the same activation): a group-quant
  // kernel ran just before this one; B tiles arrive by TMA with the weight
  // tiles (the e4m3 rows land K-major in the 128-byte swizzle, rows past M
  // are zero-filled), scales are loaded like the resident ones.
  const bool prequant = p.prequant != 0;
  const bool sx_res = resident || prequant;    // scales of the K range in shared memory from the prologue
  const bool res_full = J >= p.KB;
  const int nkb = res_full ? p.KB : J;
  // the CTA's first tile (row block nb0, K block kb0): the only 64-bit
  // divisions, done before the grid-dependency wait
  const int nb0 = static_cast<int>(u0 / p.KB);
  const int kb0 = static_cast<int>(u0 - static_cast<int64_t>(nb0) * p.KB);
  // tagged words: the input carries this rank's last sequence number, the
  // output the one after it (read after the grid-dependency wait)
  constexpr bool tagged = kTagged;
  const bool tagged_in = tagged && p.gather.wait_input;
  unsigned int tag_in = 0u, tag_out = 0u;
  // output element (token m, column n of this launch): local, or to every
  // rank (tagged: all 32 lanes together, consecutive columns on consecutive
  // lanes -- true of every call below)
  auto store_out = [&](int m, int n, __nv_bfloat16 v) {
    if constexpr (kTagged)
      gather_store_tagged(p.gather, m, n, v, tag_out);
    else if (gather_publishes(p.gather))
      gather_store(p.gather, m, n, v);
    else
      p.out[static_cast<int64_t>(m) * p.ldo + n] = v;
  };

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&tmap_w);
      if (!resident) prefetch_tensormap(&tmap_x);
    }
    if (lane < S) {
      mbar_init(&full[lane], prequant ? 1 : 2);   // TMA arrive_expect_tx (+ the activation warp of the K block)
      mbar_init(&xfull[lane], 1);        // TMA arrive_expect_tx (activation tile)
      mbar_init(&empty[lane], 1);        // tcgen05.commit
    }
    if (lane < kTmMaxAcc) {
      mbar_init(&acc_full[lane], 1);     // tcgen05.commit
      mbar_init(&tmem_empty[lane], 4);   // 4 epilogue warps
    }
    if (lane == 0) mbar_init(drain, 1);
    if (kCluster && lane == 0 && p.red_push && cluster_rank() == 0) {
      // one phase: the bytes of csize - 1 partials
      mbar_init(red_full, 1);
      mbar_arrive_expect_tx(red_full, static_cast<uint32_t>((p.csize - 1) * p.M * 128 * 4));
    }
    for (int r = lane; r < kTmSxRing; r += 32) sx_tag[r] = 0u;
    fence_mbar_init();
  } else if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&misc[0])),
                 "r"(Cfg::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // push: rank 0's barrier is initialised before any CTA of the cluster
  // copies into it (the matching wait is at the reduction, long after)
  if (kCluster && p.red_push) asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
  const uint32_t tmem_base = misc[0];
  bool ok = true;

  // Block scales of this CTA's tiles, ws_cache[j] = ws[nb(j), kb(j)] (the host
  // launches only shapes with J <= kTmWsCache), loaded by warps 2-9; and --
  // when the caller declared the weights static -- the weight tiles of the
  // first ring of stages are fetched before the grid-dependency wait,
  // overlapping the previous kernel's tail.  Activations, outputs and the
  // workspace are touched only after it.
  const bool early = p.early_weights != 0;
  const int n_pre = (early && !prequant) ? (J < S ? J : S) : 0;
  auto ws_at = [&](int j) {
    const int t = kb0 + j;
    const int dn = t / p.KB;
    return __ldg(p.ws + static_cast<int64_t>(nb0 + dn) * p.ldws + (t - dn * p.KB));
  };
  auto load_ws_cache = [&]() {
    for (int j = tid - 64; j < J; j += kTmThreads - 64) ws_cache[j] = ws_at(j);
  };
  // resident: the B tiles of the first ring start as zeros (the live rows are
  // written once the activation is quantised); shared memory only, so this is
  // done before the grid-dependency wait (barrier 1 below orders it before
  // those writes)
  const int nfirst = J < S ? J : S;
  if (resident && warp >= 2)
    for (int i = tid - 64; i < nfirst * (Cfg::kBTileBytes / 16); i += kTmThreads - 64)
      reinterpret_cast<uint4*>(b_tiles)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (early) {
    if (warp >= 2) load_ws_cache();
    if (tid == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      TileCursor c;
      c.init(nb0, kb0);
      for (int j = 0; j < n_pre; ++j, c.next(p.KB, kpb, S)) {
        mbar_arrive_expect_tx(&full[c.s], kTmATileBytes);
        tma_load_2d(a_tiles + c.s * kTmATileBytes, &tmap_w, c.kb * 128, c.nb * 128, &full[c.s], pol_w);
      }
    }
  }
  grid_dependency_wait();
  if constexpr (kTagged) {
    tag_in = gather_seq_now(p.gather);
    tag_out = tag_after(tag_in);
  }
  if (p.gather.wait_input && !tagged) {
    // The activation comes from other ranks: the warps that read it wait for
    // every rank's flag -- warps 2-9, and with the streaming feed the TMA warp
    // too (it loads the activation tiles).  Otherwise warps 0 and 1 start the
    // weight stream and the MMA loop at once: the flags cover the activation,
    // not the weights, and the MMAs wait for B tiles built after this wait.
    // (The pre-quantised feed is never chosen for such a launch: its quant
    // kernel would read the activation before the wait.)  A wait that gives
    // up has recorded the error word; the kernel then runs to its end on
    // whatever the activation holds (as the row kernel does), so every role
    // keeps its normal path.
    const bool tma_reads_x = !resident && !prequant;
    if (tma_reads_x || warp >= 2) {
      if (warp == 2) gather_wait_input(p.gather, lane);
      if (tma_reads_x)
        __syncthreads();
      else
        named_bar_sync(1, kTmThreads - 64);
    }
  }
  // Warps 0 and 1 start their loops at once; warps 2-9 first finish the block
  // scales and, resident, quantise the CTA's K range (8 warps x 4 lane octets,
  // one 128-wide group per octet and pass), then meet at barrier 1.
  if (warp >= 2) {
    // the first block-scale load of each thread is issued before the
    // activation loads, and stored after them: one round trip for both
    const int jw = tid - 64;
    float ws_first = 0.0f;
    if (!early && jw < J) ws_first = ws_at(jw);
    // resident: the first ring's B tiles are built here as well (zeroed before
    // the wait, the live rows written as they are quantised), so the first
    // MMAs wait only for their weight tiles
    if (resident) {
      named_bar_sync(1, kTmThreads - 64);
      const int oct = (warp - 2) * 4 + (lane >> 3);
      const int chunk = lane & 7;
      const int ngroups = p.M * nkb;
      // group g of this pass: token m = g / nkb, slot r = g % nkb, K block kb
      auto group_of = [&](int g, int& m, int& r, int& kb) {
        m = g / nkb;
        r = g - m * nkb;
        kb = res_full ? r : kb0 + r;
        if (kb >= p.KB) kb -= p.KB;
      };
      // a quantised group: resident bytes and scale, the first ring's B
      // tiles, the optional outputs
      auto commit = [&](int m, int r, int kb, uint4 packed, float sx) {
        *reinterpret_cast<uint4*>(x_tiles + (static_cast<int64_t>(r) * p.M + m) * 128 + chunk * 16) = packed;
        if (chunk == 0) sx_ring[r * p.M + m] = sx;
        // first-ring tiles j < nfirst that use slot r: j = r (slot = tile),
        // or j = r - kb0 mod KB and every KB after it (slot = K block)
        int jj = r;
        int step = nfirst;
        if (res_full) {
          jj = r - kb0;
          if (jj < 0) jj += p.KB;
          step = p.KB;
        }
        for (; jj < nfirst; jj += step) {
          const int br = tile_pos(jj, kb0, p.KB, kpb) * p.sw + m;
          *reinterpret_cast<uint4*>(b_tiles + jj * Cfg::kBTileBytes + br * 128 + ((chunk ^ (br & 7)) << 4)) = packed;
        }
        if (kb >= u0 && kb < u1) {
          // this CTA holds tile (row block 0, kb): it writes the optional outputs
          if (p.xq_out)
            *reinterpret_cast<uint4*>(p.xq_out + static_cast<int64_t>(m) * p.K + kb * 128 + chunk * 16) = packed;
          if (p.sx_out && chunk == 0) p.sx_out[static_cast<int64_t>(m) * p.KB + kb] = sx;
        }
      };
      if (!kSwiglu && p.norm.norm) {
        // (reduce +) add + RMSNorm: x is the sum of p.norm.nsrc sources in
        // source order (the partials of a K-sharded linear), then + residual.
        // Every CTA first sums the squares of the whole rows
        // (all K blocks, not only its own) -- chunk sums, octet sums per
        // 128-group into norm_sum[m][b] -- and one thread per token adds the
        // groups in order
        float* gsum = norm_sum;
        const int ng_all = p.M * p.KB;
        for (int g0 = 0; g0 < ng_all; g0 += 32) {
          const int g = g0 + oct;
          const bool live = g < ng_all;
          const int m = live ? g / p.KB : 0;
          const int b = live ? g - m * p.KB : 0;
          float sv[16];
          if (live) {
            addn16(sv, p.x + static_cast<int64_t>(m) * p.ldx + b * 128 + chunk * 16, p.norm.src_stride, p.norm.nsrc,
                   p.norm.res + static_cast<int64_t>(m) * p.norm.ldr + b * 128 + chunk * 16);
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) sv[e] = 0.0f;
          }
          const float gs = octet_sum(sumsq16(sv));
          if (live && chunk == 0) gsum[m * p.KB + b] = gs;
          if (live && blockIdx.x == 0 && p.norm.res_out) {
            uint4 wa, wb;
            pack_bf16x16(sv, wa, wb);
            uint4* op =
                reinterpret_cast<uint4*>(p.norm.res_out + static_cast<int64_t>(m) * p.norm.ldro + b * 128 + chunk * 16);
            op[0] = wa;
            op[1] = wb;
          }
        }
        named_bar_sync(1, kTmThreads - 64);
        if (tid - 64 < p.M) {
          const int m = tid - 64;
          float acc_s = 0.0f;
          for (int b = 0; b < p.KB; ++b) acc_s = __fadd_rn(acc_s, gsum[m * p.KB + b]);
          gsum[p.M * p.KB + m] = rms_rstd(acc_s, p.K, p.norm.eps);
        }
        named_bar_sync(1, kTmThreads - 64);
        // then the CTA's own K blocks: the bf16 norm output, quantised
        for (int g0 = 0; g0 < ngroups; g0 += 32) {
          const int g = g0 + oct;
          const bool live = g < ngroups;
          int m = 0, r = 0, kb = 0;
          if (live) group_of(g, m, r, kb);
          float v[16];
          if (live) {
            const uint4* wr = reinterpret_cast<const uint4*>(p.norm.w + kb * 128 + chunk * 16);
            float sv[16];
            addn16(sv, p.x + static_cast<int64_t>(m) * p.ldx + kb * 128 + chunk * 16, p.norm.src_stride, p.norm.nsrc,
                   p.norm.res + static_cast<int64_t>(m) * p.norm.ldr + kb * 128 + chunk * 16);
            norm16(v, sv, gsum[p.M * p.KB + m], __ldg(wr), __ldg(wr + 1));
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = 0.0f;
          }
          float sx;
          const uint4 packed = quant16_octet(v, live, sx);
          if (live) commit(m, r, kb, packed, sx);
        }
      } else if (tagged_in) {
        // Tagged input words (word i of a row holds elements 2i, 2i + 1):
        // the loads of kPasses passes are issued first, as below, then each
        // group's words are polled until they carry this rank's last sequence
        // number.  A thread that gave up does not wait again.
        constexpr int kPasses = kSwiglu ? 1 : 2;
        const uint64_t* xw0 = reinterpret_cast<const uint64_t*>(p.x);
        bool live_in = true;
        auto words_of = [&](int m, int kb) {
          return xw0 + ((static_cast<int64_t>(m) * p.ldx + kb * 128 + chunk * 16) >> 1);
        };
        for (int g0 = 0; g0 < ngroups; g0 += 32 * kPasses) {
          uint64_t wv[kPasses][kSwiglu ? 16 : 8];
#pragma unroll
          for (int i = 0; i < kPasses; ++i) {
            const int g = g0 + 32 * i + oct;
            if (g < ngroups) {
              int m, r, kb;
              group_of(g, m, r, kb);
              tagged_issue8(words_of(m, kb), wv[i]);
              if constexpr (kSwiglu) tagged_issue8(words_of(m, kb) + p.K / 2, wv[i] + 8);
            }
          }
#pragma unroll
          for (int i = 0; i < kPasses; ++i) {
            if (g0 + 32 * i >= ngroups) break;   // uniform across the warp
            const int g = g0 + 32 * i + oct;
            const bool live = g < ngroups;
            int m = 0, r = 0, kb = 0;
            if (live) group_of(g, m, r, kb);
            float v[16];
            if (live) {
              uint32_t xw[8], uw[8];
              tagged_finish8(words_of(m, kb), tag_in, wv[i], xw, live_in);
              if constexpr (kSwiglu) tagged_finish8(words_of(m, kb) + p.K / 2, tag_in, wv[i] + 8, uw, live_in);
              const uint4 a = make_uint4(xw[0], xw[1], xw[2], xw[3]);
              const uint4 b = make_uint4(xw[4], xw[5], xw[6], xw[7]);
              if constexpr (kSwiglu)
                act16<true>(v, a, b, make_uint4(uw[0], uw[1], uw[2], uw[3]), make_uint4(uw[4], uw[5], uw[6], uw[7]));
              else
                act16<false>(v, a, b, a, b);
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] = 0.0f;
            }
            float sx;
            const uint4 packed = quant16_octet(v, live, sx);
            if (live) commit(m, r, kb, packed, sx);
          }
        }
      } else {
        // The loads of kPasses passes are issued before any of them is
        // quantised (L2-coherent loads: the activation may come from the
        // kernel before this one in the stream), so a pass costs one L2 round
        // trip per kPasses passes rather than one each.
        constexpr int kPasses = kSwiglu ? 2 : 4;
        constexpr int kWords = kSwiglu ? 4 : 2;
        for (int g0 = 0; g0 < ngroups; g0 += 32 * kPasses) {
          uint4 wd[kPasses][kWords];
#pragma unroll
          for (int i = 0; i < kPasses; ++i) {
            const int g = g0 + 32 * i + oct;
            if (g < ngroups) {
              int m, r, kb;
              group_of(g, m, r, kb);
              const uint4* xr = reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(m) * p.ldx + kb * 128 +
                                                               chunk * 16);
              wd[i][0] = __ldcg(xr);
              wd[i][1] = __ldcg(xr + 1);
              if constexpr (kSwiglu) {
                const uint4* ur = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(xr) + p.K);
                wd[i][kWords - 2] = __ldcg(ur);
                wd[i][kWords - 1] = __ldcg(ur + 1);
              }
            }
          }
#pragma unroll
          for (int i = 0; i < kPasses; ++i) {
            if (g0 + 32 * i >= ngroups) break;   // uniform across the warp
            const int g = g0 + 32 * i + oct;
            const bool live = g < ngroups;
            int m = 0, r = 0, kb = 0;
            if (live) group_of(g, m, r, kb);
            float v[16];
            if (live) {
              act16<kSwiglu>(v, wd[i][0], wd[i][1], wd[i][kWords - 2], wd[i][kWords - 1]);
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] = 0.0f;
            }
            float sx;
            const uint4 packed = quant16_octet(v, live, sx);
            if (live) commit(m, r, kb, packed, sx);
          }
        }
      }
    }
    if (prequant) {
      // scales of the CTA's K range, [slot][M] as in the resident feed
      for (int i = tid - 64; i < nkb * p.M; i += kTmThreads - 64) {
        const int r = i / p.M;
        const int m = i - r * p.M;
        int kb = res_full ? r : kb0 + r;
        if (kb >= p.KB) kb -= p.KB;
        sx_ring[i] = __ldcg(p.sx_pre + static_cast<int64_t>(m) * p.KB + kb);
      }
    }
    if (!early) {
      if (jw < J) ws_cache[jw] = ws_first;
      for (int j = jw + (kTmThreads - 64); j < J; j += kTmThreads - 64) ws_cache[j] = ws_at(j);
    }
    if (resident) fence_proxy_async_smem();   // B tiles written here are read by the MMA
    named_bar_sync(1, kTmThreads - 64);
    if (resident && tid == 64)
      for (int j = 0; j < nfirst; ++j) mbar_arrive(&full[j]);
  }

  if (warp == 0) {
    // --------------------------------------------------- TMA producer --
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const uint32_t xbytes = p.x_tile_bytes * (kSwiglu ? 2u : 1u);
      int issued = 0;
      TileCursor c;
      c.init(nb0, kb0);
      for (int j = 0; j < J && ok; ++j, c.next(p.KB, kpb, S)) {
        const int s = c.s;
        if (j >= S) ok = mbar_wait(&empty[s], c.ph ^ 1u, kSiteTmA);
        if (!ok) break;
        if (prequant) {
          // the box's MT rows start at row -pos * sw of the M-row tensor: the
          // tokens land in rows pos * sw + m of the B tile, every other row is
          // the zero fill of a row outside the tensor
          mbar_arrive_expect_tx(&full[s], kTmATileBytes + Cfg::kBTileBytes);
          tma_load_2d(a_tiles + s * kTmATileBytes, &tmap_w, c.kb * 128, c.nb * 128, &full[s], pol_w);
          tma_load_2d(b_tiles + s * Cfg::kBTileBytes, &tmap_x, c.kb * 128, -(c.pos * p.sw), &full[s], pol_x);
        } else if (j >= n_pre) {
          mbar_arrive_expect_tx(&full[s], kTmATileBytes);
          tma_load_2d(a_tiles + s * kTmATileBytes, &tmap_w, c.kb * 128, c.nb * 128, &full[s], pol_w);
        }
        if (!resident && !prequant) {
          uint8_t* xt = x_tiles + s * static_cast<uint32_t>(Cfg::kXTileBytes);
          mbar_arrive_expect_tx(&xfull[s], xbytes);
          tma_load_2d(xt, &tmap_x, c.kb * 128, 0, &xfull[s], pol_x);
          if constexpr (kSwiglu) tma_load_2d(xt + p.x_tile_bytes, &tmap_x, p.K + c.kb * 128, 0, &xfull[s], pol_x);
        }
        issued = j + 1;
      }
      grid_launch_dependents();
      if (!ok) {
        // let the copies already issued land before the CTA can exit
        for (int j = (issued > S ? issued - S : 0); j < issued; ++j) {
          mbar_wait(&full[j % S], (j / S) & 1, kSiteTmA);
          if (!resident && !prequant) mbar_wait(&xfull[j % S], (j / S) & 1, kSiteTmA);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------- MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = idesc_f8<MT>();
      // descriptors of stage 0's A and B tiles; a stage and a K step are
      // offsets in the 14-bit start-address field (addresses < 256 KB)
      const uint64_t desc_a0 = smem_desc_sw128(smem_u32(a_tiles));
      const uint64_t desc_b0 = smem_desc_sw128(smem_u32(b_tiles));
      AccCursor acc;
      uint32_t d_tmem = tmem_base;
      TileCursor c;
      c.init(nb0, kb0);
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
        const uint64_t da = desc_a0 + static_cast<uint64_t>((c.s * kTmATileBytes) >> 4);
        const uint64_t db = desc_b0 + static_cast<uint64_t>((c.s * Cfg::kBTileBytes) >> 4);
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
    const int NPW = p.npw;                    // this warp takes j = w4, w4 + NPW, ...
    const int w4 = warp - 2;
    const int chunk = lane & 7;         // 16-byte chunk of the 128-wide K block
    const int row0 = lane >> 3;         // 0..3
    // resident: the first ring's tiles were built in the prologue
    const int j_first = w4 + (resident ? S : 0);
    TileCursor c;
    c.init(nb0, kb0);
    for (int k = 0; k < j_first; ++k) c.next(p.KB, kpb, S);
    for (int j = j_first; w4 < NPW && !prequant && j < J && ok; j += NPW) {
      if (j > j_first) {
        for (int k = 0; k < NPW; ++k) c.next(p.KB, kpb, S);
      }
      const int s = c.s;
      const int pos = c.pos;
      uint8_t* btile = b_tiles + s * Cfg::kBTileBytes;
      if (resident) {
        // copy the prebuilt bytes once the MMA has released the stage
        if (j >= S) ok = mbar_wait(&empty[s], c.ph ^ 1u, kSiteTmA);
        if (!ok) break;
        const int r = res_full ? c.kb : j;
        const uint8_t* xq = x_tiles + static_cast<int64_t>(r) * p.M * 128 + chunk * 16;
#pragma unroll
        for (int i = 0; i < MT / 4; ++i) {
          const int br = row0 + 4 * i;
          const int m = br - pos * p.sw;
          const bool live = m >= 0 && m < p.sw && m < p.M;
          const uint4 packed = live ? *reinterpret_cast<const uint4*>(xq + m * 128) : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(btile + br * 128 + ((chunk ^ (br & 7)) << 4)) = packed;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
        continue;
      }
      ok = mbar_wait(&xfull[s], c.ph, kSiteTmA);
      if (!ok) break;
      const int nb = c.nb;
      const int kb = c.kb;
      const __nv_bfloat16* xt =
          reinterpret_cast<const __nv_bfloat16*>(x_tiles + s * static_cast<uint32_t>(Cfg::kXTileBytes));
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
            const uint4* xp = reinterpret_cast<const uint4*>(xt + m * 128 + chunk * 16);
            const uint4 xa = xp[0], xb = xp[1];
            uint4 ua = xa, ub = xb;
            if constexpr (kSwiglu) {
              const uint4* up = reinterpret_cast<const uint4*>(xt + p.x_tile_bytes / 2 + m * 128 + chunk * 16);
              ua = up[0];
              ub = up[1];
            }
            act16<kSwiglu>(v, xa, xb, ua, ub);
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = 0.0f;
          }
          float sx;
          packed = quant16_octet(v, live, sx);
          if (live) {
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
    // (publishing without an input wait: no store may overtake a rank still
    // inside its previous publishing kernel; the MMA pipeline runs meanwhile)
    gather_wait_store(p.gather, lane);
    const int q4 = warp & 3;                 // TMEM lane quarter of this warp
    const int row = 32 * q4 + lane;          // weight row within the 128-row block
    const uint32_t t_lane = static_cast<uint32_t>(32 * q4) << 16;
    float acc[MT];                           // per TMEM column: token c % sw of slot c / sw
#pragma unroll
    for (int c = 0; c < MT; ++c) acc[c] = 0.0f;
    int seg_j0 = 0, seg_kb0 = 0;
    AccCursor accc;
    TileCursor cur;
    cur.init(nb0, kb0);
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
      const int jq0 = j - pos;                 // first K block of the group
      const int rq0 = res_full ? kb - pos : jq0;   // its resident slot
      // Column c of the group holds token m = c % sw of K block q = c / sw;
      // its scale is sx[m, q] * ws[q].  All loads are in bounds (unused
      // columns read entry 0) so they issue back to back; resident scales of
      // the first kPre columns are loaded before the accumulator is ready.
      auto col_scale = [&](int c, bool& use) {
        const int q = c >> p.lg_sw;
        const int m = c & (p.sw - 1);
        use = q <= pos && m < p.M;
        const int qc = use ? q : 0;
        const int mc = use ? m : 0;
        const int si = sx_res ? (rq0 + qc) * p.M + mc : ((jq0 + qc) & (kTmSxRing - 1)) * MT + mc;
        return sx_ring[si] * ws_cache[jq0 + qc];
      };
      // One K block per group (kpb == 1, i.e. sw == MT): column c is token c of
      // K block jq0, and its sx values are contiguous -- the resident slot
      // rq0's M entries, or streaming ring row jq0 -- so they are read at fixed
      // offsets from one base, without col_scale's per-column index arithmetic
      // (which costs more than the rest of the per-K-block epilogue).  Columns
      // c >= M read on past the slot, still inside the sx ring and ws cache
      // regions (nkb * M <= kTmSxRing * MT), and are masked off.  Same products
      // as col_scale, so the results do not change.
      const bool one_kb = kpb == 1;
      const float* sx_grp = sx_res ? sx_ring + rq0 * p.M : sx_ring + (jq0 & (kTmSxRing - 1)) * MT;
      auto live_mask = [&](int c0) -> uint32_t {   // columns c0 .. c0 + 15 that hold a token
        const int n = p.M - c0;
        return n >= 16 ? 0xffffu : n <= 0 ? 0u : (1u << n) - 1u;
      };
      constexpr bool kPre = MT == 16;         // the 16-token tile: all scales in registers up front
      float scl[16];
      uint32_t pre_mask = 0;                   // bit c: column c holds a live (token, K block)
      auto load_scales = [&]() {
        if constexpr (kPre) {
          if (one_kb) {
            const float wsv = ws_cache[jq0];
#pragma unroll
            for (int c = 0; c < 16; ++c) scl[c] = sx_grp[c] * wsv;
            pre_mask = live_mask(0);
          } else if (sx_res && p.M == p.sw) {
            // M a power of two: the group's pos + 1 K blocks fill columns
            // 0 .. (pos + 1) * M - 1 and their sx values are contiguous too
            // (slots rq0, rq0 + 1, ... of M entries each); the ws index is
            // clamped to the group's last K block
#pragma unroll
            for (int c = 0; c < 16; ++c) scl[c] = sx_grp[c] * ws_cache[jq0 + min(c >> p.lg_sw, pos)];
            pre_mask = live_mask(p.M - (pos + 1) * p.sw);
          } else {
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              bool u;
              scl[c] = col_scale(c, u);
              pre_mask |= u ? (1u << c) : 0u;
            }
          }
        }
      };
      if (sx_res) load_scales();
      if (ok) ok = mbar_wait(&acc_full[a], accc.round, kSiteTmAcc);
      if (!sx_res && lane == 0) {
        for (int q = 0; q <= pos && ok; ++q) ok = tag_wait(sx_tag + ((j - pos + q) & (kTmSxRing - 1)),
                                                         static_cast<uint32_t>(j - pos + q + 1));
        __threadfence_block();
      }
      ok = __all_sync(0xffffffffu, ok) != 0;   // tcgen05.ld below is warp-collective
      if (!sx_res) load_scales();
      tc_fence_after();
#pragma unroll
      for (int c16 = 0; c16 < MT / 16; ++c16) {
        float v[16];
        float sc[16];
        uint32_t m16 = 0;
        if constexpr (kPre) {
#pragma unroll
          for (int i = 0; i < 16; ++i) sc[i] = scl[i];
          m16 = pre_mask;
        } else if (one_kb) {
          const float wsv = ws_cache[jq0];
#pragma unroll
          for (int i = 0; i < 16; ++i) sc[i] = sx_grp[16 * c16 + i] * wsv;
          m16 = live_mask(16 * c16);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            bool u;
            sc[i] = col_scale(16 * c16 + i, u);
            m16 |= u ? (1u << i) : 0u;
          }
        }
        if (ok) {
          tmem_ld16(tmem_base + t_lane + static_cast<uint32_t>(a * MT + 16 * c16), v);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if ((m16 >> i) & 1u) acc[16 * c16 + i] = fmaf(v[i], sc[i], acc[16 * c16 + i]);
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
            if (m < p.M) store_out(m, n, __float2bfloat16_rn(acc[m]));
        } else if (kCluster) {
          // cluster split-K: the partial sums stay in this CTA's shared memory
          // (the A tiles are free: every MMA has completed) and are reduced
          // across the cluster at the end of the kernel
          float* part = reinterpret_cast<float*>(a_tiles);
#pragma unroll
          for (int m = 0; m < MT; ++m)
            if (m < p.M) part[m * 128 + row] = acc[m];
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
            // the partials of up to kRed CTAs are loaded together (one L2 round
            // trip per kRed rather than per CTA) and added in CTA order
            // Every contributor after i_lo starts inside this row block (its
            // slot 0); i_lo's slot is 0 only if its range starts at the row
            // block's first tile.
            constexpr int kRed = 8;
            const int si_lo = ((i_lo * p.U) / G == first_u) ? 0 : 1;
            for (int64_t i0 = i_lo; i0 <= i_hi; i0 += kRed) {
              const int cnt = static_cast<int>(i_hi - i0 + 1 < kRed ? i_hi - i0 + 1 : kRed);
              // float offset of contributor q's partial slot (< 2^32: at most 296 x 2 x 64 x 128)
              auto off = [&](int q) {
                const int64_t i = i0 + (q < cnt ? q : 0);
                return static_cast<uint32_t>(((i * 2 + (i == i_lo ? si_lo : 0)) * MT) * 128 + row);
              };
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                if (m < p.M) {
                  float v[kRed];
#pragma unroll
                  for (int q = 0; q < kRed; ++q) v[q] = q < cnt ? __ldcg(p.partials + off(q) + m * 128) : 0.0f;
#pragma unroll
                  for (int q = 0; q < kRed; ++q)
                    if (q < cnt) sum[m] += v[q];
                }
              }
            }
#pragma unroll
            for (int m = 0; m < MT; ++m)
              if (m < p.M) store_out(m, n, __float2bfloat16_rn(sum[m]));
          }
          named_bar_sync(2, 128);
        }
      }
    }
  }

  if (kCluster && p.red_push) {
    // Cluster split-K reduction by push: every other CTA of the cluster copies
    // its [M][128] partial sums (one bulk copy, shared memory to rank 0's
    // shared memory) and is done; rank 0 waits for their bytes on red_full and
    // adds the partials in rank order -- the same sums as the pull form below
    // -- with one barrier wait instead of two cluster barriers.
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
    const int rank = static_cast<int>(cluster_rank());
    const int nbc = static_cast<int>(u0 / p.KB);
    float* part = reinterpret_cast<float*>(a_tiles);
    float* red = reinterpret_cast<float*>(smem + p.red_off);
    const uint32_t pbytes = static_cast<uint32_t>(p.M * 128 * 4);
    if (warp >= 6) {
      if (rank != 0) {
        fence_proxy_async_smem();   // this thread's partial stores before the copy reads them
        named_bar_sync(2, 128);
        if (tid == 192) {
          asm volatile(
              "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                  dsmem_addr(red + (rank - 1) * p.M * 128, 0)),
              "r"(smem_u32(part)), "r"(pbytes), "r"(dsmem_addr(red_full, 0))
              : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // part stays until it is read
        }
      } else {
        named_bar_sync(2, 128);     // this CTA's own partial: written by the other epilogue threads
        mbar_wait(red_full, 0, kSiteTmFixup);
        for (int e = tid - 192; e < p.M * 128; e += 128) {
          float sum = 0.0f;
          sum += part[e];
          for (int q = 1; q < p.csize; ++q) sum += red[(q - 1) * p.M * 128 + e];
          store_out(e >> 7, nbc * 128 + (e & 127), __float2bfloat16_rn(sum));
        }
      }
    }
  } else if (kCluster) {
    // Cluster split-K reduction.  The CTAs of a cluster are the csize K parts
    // of one row block; after the barrier, epilogue thread t of cluster rank r
    // reduces elements e = r*128 + t (+ 128*csize ...) of the [M][128] partial
    // sums, reading every rank's value over distributed shared memory and
    // adding them in rank order (the result does not depend on timing).
    cluster_sync_all();
    if (warp >= 6) {
      const int rank = static_cast<int>(cluster_rank());
      const int nbc = static_cast<int>(u0 / p.KB);
      const float* part = reinterpret_cast<const float*>(a_tiles);
      for (int e = rank * 128 + (tid - 192); e < p.M * 128; e += 128 * p.csize) {
        // every rank's value is requested before any is added: one round trip
        // over distributed shared memory rather than one per rank
        float v[kTmMaxCluster];
#pragma unroll
        for (int q = 0; q < kTmMaxCluster; ++q) v[q] = q < p.csize ? ld_dsmem(dsmem_addr(part + e, q)) : 0.0f;
        float sum = 0.0f;
#pragma unroll
        for (int q = 0; q < kTmMaxCluster; ++q)
          if (q < p.csize) sum += v[q];
        store_out(e >> 7, nbc * 128 + (e & 127), __float2bfloat16_rn(sum));
      }
    }
    cluster_sync_all();   // this CTA's shared memory stays until the cluster has read it
  }

  tc_fence_before();
  __syncthreads();
  if (gather_publishes(p.gather) && tid == 0) gather_cta_done(p.gather, gridDim.x);
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

// Whether M tokens may take the pre-quantised feed: every pass has one K
// block per accumulator group (16-token tile with M > 8, or a wider tile).
// The pre-quantised feed may serve any M (the workspace then holds the
// quantised activation); the auto choice takes it where the activation cannot
// stay resident, or where the resident prologue -- every CTA quantising M x
// (its K blocks) groups of the same activation -- would cost more than the
// group-quant launch: M x (K blocks per CTA) >= kTmPrequantMinGroups.
inline bool tm_prequant_shape(int M) { return M >= 1; }
constexpr int64_t kTmPrequantMinGroups = 72;

inline size_t tm_align256(size_t b) { return (b + 255) / 256 * 256; }

// Workspace: split-K counters, partial sums of up to one CTA per resident
// slot, and (shapes that may be pre-quantised) the quantised activation and
// its scales.
inline size_t tm_partials_end(int M, int N, int K, int sm_count) {
  const int MT = tm_token_tile(M);
  const int64_t U = static_cast<int64_t>(N / kGroup) * (K / kGroup);
  const int G = tm_slots(sm_count, MT) < U ? tm_slots(sm_count, MT) : static_cast<int>(U);
  return kTmCounterBytes + static_cast<size_t>(G) * 2 * MT * 128 * sizeof(float);
}

inline size_t tm_workspace_bytes_for(int M, int N, int K, int sm_count) {
  size_t b = tm_partials_end(M, N, K, sm_count);
  if (tm_prequant_shape(M))
    b = tm_align256(b) + tm_align256(static_cast<size_t>(M) * K) +
        tm_align256(static_cast<size_t>(M) * (K / kGroup) * sizeof(float));
  return b;
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

// Pre-quantised activation map: 2-D uint8 [rows, K] (row stride K), box 128
// bytes x MT rows in the 128-byte swizzle -- a B tile; rows outside the tensor
// (past `rows`, or before row 0 when the load starts at a negative row) are
// zero-filled.
inline bool make_xq_tmap(CUtensorMap* map, const void* xq, int rows, int K, int MT) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
  cuuint32_t box[2] = {128, static_cast<cuuint32_t>(MT)};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(xq), dims, strides, box, estr,
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

// Host-side caches for the per-call set-up of a launch.  A tensor map
// depends only on the address, the shape, the row stride and the box, so an
// encoded one is reused for the same operand (a decode loop calls every
// linear on the same weights and activation buffers); the table is cleared
// when it grows past kTmapCacheMax entries.
struct TmapKey {
  int dev, kind, rows, box_rows;
  const void* ptr;
  int64_t cols, ld;
  bool operator<(const TmapKey& o) const {
    return std::tie(dev, kind, rows, box_rows, ptr, cols, ld) <
           std::tie(o.dev, o.kind, o.rows, o.box_rows, o.ptr, o.cols, o.ld);
  }
};
constexpr size_t kTmapCacheMax = 8192;

// kind 0: weight (make_weight_tmap), 1: bf16 activation (make_act_tmap),
// 2: pre-quantised activation (make_xq_tmap, box_rows = MT)
inline bool cached_tmap(CUtensorMap* map, int kind, const void* ptr, int rows, int64_t cols, int64_t ld,
                        int box_rows) {
  static std::mutex mu;
  static std::map<TmapKey, CUtensorMap> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const TmapKey key{dev, kind, rows, box_rows, ptr, cols, ld};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *map = it->second;
      return true;
    }
  }
  bool ok = kind == 0   ? make_weight_tmap(map, ptr, rows, static_cast<int>(cols), ld)
            : kind == 1 ? make_act_tmap(map, ptr, rows, cols, ld)
                        : make_xq_tmap(map, ptr, rows, static_cast<int>(cols), box_rows);
  if (!ok) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() >= kTmapCacheMax) cache.clear();
  cache.emplace(key, *map);
  return true;
}

// cudaFuncAttributeMaxDynamicSharedMemorySize raised to the device's limit
// once per kernel and device (launches then pass their own smaller sizes).
inline cudaError_t ensure_max_smem(const void* fn, int max_smem) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_pair(dev, fn);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = done.find(key);
    if (it != done.end() && it->second >= max_smem) return cudaSuccess;
  }
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  done[key] = max_smem;
  return cudaSuccess;
}

// cudaFuncAttributeNonPortableClusterSizeAllowed set once per kernel and
// device, before a cluster of more than 8 CTAs is queried or launched.
inline cudaError_t ensure_nonportable_clusters(const void* fn) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, bool> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_pair(dev, fn);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess) done[key] = true;
  return e;
}

// Shared-memory plan of one pass: ring depth, activation mode and layout.
struct TmPlan {
  int stages, npw, resident;
  uint32_t b_off, x_off, bar_off;
  size_t smem;
};

// A grid of at most one CTA per SM (or a token tile that always runs one) gets
// the SM's whole shared memory; otherwise the 16-token tile gets half.  The
// resident activation mode -- M x (the CTA's K blocks) quantised bytes, their
// scales in the sx ring -- is used when it still leaves at least 4 stages.
template <int MT, bool SW>
inline bool tm_plan(TmPlan* pl, int M, int64_t U, int64_t KB, int grid, int sm_count, int max_smem,
                    int resident_mode, int64_t extra_tail = 0, bool prequant = false) {
  using Cfg = TmCfg<MT, SW>;
  const bool one_per_sm = tm_ctas_per_sm<MT>() == 1 || grid <= sm_count;
  int64_t budget = one_per_sm ? max_smem
                              : static_cast<int64_t>(kTmSmemBudgetSm / tm_ctas_per_sm<MT>() - kTmSmemReservedPerCta);
  if (budget > max_smem) budget = max_smem;
  const int64_t avail = budget - static_cast<int64_t>(Cfg::kTailBytes + Cfg::kAlignSlack) - extra_tail;
  if (avail <= 0) return false;
  const int64_t jmax = (U + grid - 1) / grid;
  const int64_t nkb = jmax < KB ? jmax : KB;
  int S = 0;
  bool res = false;
  int64_t xbytes = 0;
  if (resident_mode != 0 && nkb * M <= static_cast<int64_t>(kTmSxRing) * MT) {
    const int64_t rbytes = (nkb * M * 128 + 1023) / 1024 * 1024;
    const int sr = tm_pick_stages((avail - rbytes) / (kTmATileBytes + Cfg::kBTileBytes));
    if (sr >= 4) {
      S = sr;
      res = true;
      xbytes = rbytes;
    }
  }
  if (!res && prequant) {
    // B tiles come by TMA like the weight tiles: no activation region
    S = tm_pick_stages(avail / (kTmATileBytes + Cfg::kBTileBytes));
    xbytes = 0;
  } else if (!res) {
    S = tm_pick_stages(avail / (kTmATileBytes + Cfg::kBTileBytes + Cfg::kXTileBytes));
    xbytes = static_cast<int64_t>(S) * Cfg::kXTileBytes;
  }
  if (S < 2) return false;
  pl->stages = S;
  pl->npw = tm_producer_warps(S);
  pl->resident = res ? 1 : 0;
  pl->b_off = static_cast<uint32_t>(S * kTmATileBytes);
  pl->x_off = pl->b_off + static_cast<uint32_t>(S * Cfg::kBTileBytes);
  pl->bar_off = pl->x_off + static_cast<uint32_t>(xbytes);
  pl->smem = pl->bar_off + Cfg::kTailBytes + Cfg::kAlignSlack + static_cast<size_t>(extra_tail);
  return pl->smem <= static_cast<size_t>(max_smem);
}

template <int MT, bool SW>
int launch_tm_pass(const CUtensorMap& tw, const CUtensorMap& tx, TmParams p, int grid, int sm_count,
                   int max_smem, cudaStream_t stream, int resident_mode, int csize) {
  TmPlan pl;
  // add + RMSNorm: group sums and rstd per token after the ws cache, and the
  // resident feed (the prologue is the only place the norm is computed)
  const int64_t norm_bytes = p.norm.norm ? ((static_cast<int64_t>(p.M) * (p.KB + 1) * 4 + 15) / 16) * 16 : 0;
  if (!tm_plan<MT, SW>(&pl, p.M, p.U, p.KB, grid, sm_count, max_smem, p.prequant ? 0 : resident_mode, norm_bytes,
                       p.prequant != 0))
    return 8;  // FP8GQ_ERR_UNSUPPORTED
  if (p.norm.norm && !pl.resident) return 8;
  // tagged input words are read by the resident prologue only
  if (p.gather.tagged && p.gather.wait_input && !pl.resident) return 8;
  // cluster split-K by push when rank 0's receive area fits beside the
  // same feed (the ring may lose a stage); otherwise the pull form
  p.red_push = 0;
  p.red_off = 0;
  if (csize > 1) {
    const int64_t red_bytes = static_cast<int64_t>(csize - 1) * p.M * 128 * 4;
    TmPlan pp;
    if (red_bytes <= kTmPushMaxBytes &&
        tm_plan<MT, SW>(&pp, p.M, p.U, p.KB, grid, sm_count, max_smem, p.prequant ? 0 : resident_mode,
                        norm_bytes + red_bytes + 16, p.prequant != 0) &&
        pp.resident == pl.resident) {
      pl = pp;
      p.red_push = 1;
      p.red_off = static_cast<uint32_t>((pl.bar_off + TmCfg<MT, SW>::kTailBytes + norm_bytes + 15) / 16 * 16);
    }
  }
  p.stages = pl.stages;
  p.npw = pl.npw;
  p.resident = pl.resident;
  p.b_off = pl.b_off;
  p.x_off = pl.x_off;
  p.bar_off = pl.bar_off;
  p.csize = csize;
  auto go = [&](auto fn) -> int {
    if (ensure_max_smem(reinterpret_cast<const void*>(fn), max_smem) != cudaSuccess) return 7;  // FP8GQ_ERR_LAUNCH
    if (csize > kTmMaxPortableCluster && ensure_nonportable_clusters(reinterpret_cast<const void*>(fn)) != cudaSuccess)
      return 7;
    if (launch_with_pdl_cluster(fn, dim3(grid), dim3(kTmThreads), pl.smem, stream, csize, tw, tx, p) != cudaSuccess)
      return 7;
    return cudaGetLastError() == cudaSuccess ? 0 : 7;
  };
  if (p.gather.world > 0 && p.gather.tagged) {
    // tagged words: calls of at most 16 tokens, the 16-token tile only
    if constexpr (MT == 16)
      return csize > 1 ? go(gemm_tm_kernel<16, SW, true, true>) : go(gemm_tm_kernel<16, SW, true, false>);
    else
      return 8;
  }
  return csize > 1 ? go(gemm_tm_kernel<MT, SW, false, true>) : go(gemm_tm_kernel<MT, SW, false, false>);
}

// How many clusters of `csize` CTAs with `smem` bytes each can be resident at
// once (cudaOccupancyMaxActiveClusters), cached per device and configuration.
template <int MT, bool SW>
int tm_max_clusters(int csize, size_t smem, int max_smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, csize, smem);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto fn = gemm_tm_kernel<MT, SW, false, true>;
  int n = 0;
  if (ensure_max_smem(reinterpret_cast<const void*>(fn), max_smem) == cudaSuccess &&
      (csize <= kTmMaxPortableCluster || ensure_nonportable_clusters(reinterpret_cast<const void*>(fn)) == cudaSuccess)) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(csize);
    cfg.blockDim = dim3(kTmThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(csize);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  cache[key] = n;
  return n;
}

// Grid of a launch.  First choice: the widest aligned split -- the S CTAs of
// a row block share its K range (any 1 <= S <= min(KB, 16); the K blocks
// split as evenly as the integers allow) and reduce in a cluster -- whose
// grid fits the resident CTA slots and whose clusters are all resident in one
// wave (measured on B200: a second wave, e.g. 16 clusters of 8 one-per-SM
// CTAs where 15 fit, costs more than a narrower split).  The occupancy query
// counts one CTA per SM; a grid above the SM count runs two CTAs per SM, where
// a cluster of S CTAs needs ceil(S/2) SMs, so its capacity is the query's for
// clusters of ceil(S/2) (measured: 2048 x 12288 at M = 1 takes 9.9 us with 16
// clusters of 12 at two per SM against 13.3 us with 16 clusters of 4 at one).
// Wider splits hand off through the workspace and stream-K spreads the tiles
// over all slots; both only when no cluster split of at least 2 (or with half
// the SMs) exists.  With need_resident, only grids whose plan keeps the
// activation resident.
template <int MT, bool SW>
int tm_choose_grid_uncached(int NB, int KB, int64_t U, int M, int sm_count, int max_smem, int resident_mode,
                            bool need_resident, int64_t extra_tail) {
  const int64_t slots = tm_slots(sm_count, MT);
  const int mp = M < MT ? M : MT;
  auto usable = [&](int64_t G, bool cluster, int S) {
    TmPlan pl;
    if (!tm_plan<MT, SW>(&pl, mp, U, KB, static_cast<int>(G), sm_count, max_smem, resident_mode, extra_tail))
      return false;
    if (need_resident && !pl.resident) return false;
    if (!cluster) return true;
    const bool one_per_sm = tm_ctas_per_sm<MT>() == 1 || G <= sm_count;
    const int span = one_per_sm ? S : (S + 1) / 2;      // SMs a cluster occupies
    return span < 2 || tm_max_clusters<MT, SW>(span, pl.smem, max_smem) >= NB;
  };
  int64_t best = 0;
  for (int S = 1; S <= KB && S <= kTmMaxCluster; ++S) {
    const int64_t G = static_cast<int64_t>(NB) * S;
    if (G > slots) break;
    // (the same grid whichever hand-off runs, so the results do not depend on it)
    if (usable(G, S > 1, S)) best = G;
  }
  if (best > 0 && (best / NB >= 2 || best >= sm_count / 2)) return static_cast<int>(best);
  int64_t wide = 0;
  for (int S = 2 * kTmMaxPortableCluster; S <= KB; S *= 2) {
    const int64_t G = static_cast<int64_t>(NB) * S;
    if (KB % S || G > slots) continue;
    if (usable(G, false, S)) wide = G;
  }
  if (wide >= sm_count / 2) return static_cast<int>(wide);
  for (int64_t G : {U < slots ? U : slots, U < sm_count ? U : static_cast<int64_t>(sm_count)})
    if (usable(G, false, 1)) return static_cast<int>(G);
  return best > 0 ? static_cast<int>(best) : 0;
}

// tm_choose_grid_uncached, remembered per device and argument set (a decode
// loop asks for the same few shapes on every call).
template <int MT, bool SW>
int tm_choose_grid(int NB, int KB, int64_t U, int M, int sm_count, int max_smem, int resident_mode,
                   bool need_resident, int64_t extra_tail) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int, int, int64_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const int mp = M < MT ? M : MT;
  const auto key = std::make_tuple(dev, NB, KB, mp, max_smem, resident_mode, need_resident ? 1 : 0, extra_tail);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int g = tm_choose_grid_uncached<MT, SW>(NB, KB, U, M, sm_count, max_smem, resident_mode, need_resident,
                                                extra_tail);
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() >= kTmapCacheMax) cache.clear();
  cache.emplace(key, g);
  return g;
}

// Runs ceil(M / MT) passes of at most MT tokens; every pass reuses the
// workspace (its counters are zero again when a pass ends).  resident_mode
// picks the activation feed: 0 streaming only; 1 auto (resident where it fits,
// pre-quantised where it does not or where the resident prologue costs more:
// kTmPrequantMinGroups); 2 pre-quantised wherever its scales fit; 3 resident
// wherever it fits, pre-quantised only where it does not.  cluster_mode 0
// forces the split-K hand-off through the workspace (clusters are used for
// aligned splits of 2 to 8 CTAs otherwise).
inline int launch_tm(bool swiglu, const void* x, int64_t ldx, const void* w, int64_t ldw, const float* ws,
                     int64_t ldws, void* out, int64_t ldo, int M, int N, int K, uint8_t* xq_out,
                     float* sx_out, void* workspace, size_t workspace_bytes, int sm_count, int max_smem,
                     cudaStream_t stream, int early_weights = 0, int grid_override = 0,
                     int resident_mode = 1, int cluster_mode = 1, const GatherParams* gather = nullptr,
                     const NormParams* norm = nullptr) {
  const int MT = tm_token_tile(M);
  if (N / kGroup > kTmMaxRowBlocks) return 8;  // FP8GQ_ERR_UNSUPPORTED
  // tagged words: one launch per call (its sequence number tags every word)
  if (gather && gather->tagged && M > MT) return 8;
  const size_t need = tm_workspace_bytes_for(M, N, K, sm_count);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return 5;  // FP8GQ_ERR_WORKSPACE
  CUtensorMap tmap_w;
  if (!cached_tmap(&tmap_w, 0, w, N, K, ldw, 0)) return 7;
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
  int grid = 0;
  if (grid_override > 0) {
    grid = grid_override < p.U ? grid_override : static_cast<int>(p.U);
  } else {
    // the add + RMSNorm prologue needs the resident feed and room for its
    // sums; tagged input words need the resident feed too
    const bool need_res = (norm && norm->norm) || (gather && gather->tagged && gather->wait_input);
    const int mp = M < MT ? M : MT;
    const int64_t nb_bytes = need_res ? ((static_cast<int64_t>(mp) * (p.KB + 1) * 4 + 15) / 16) * 16 : 0;
    const int NBr = N / kGroup;
    if (MT == 16)
      grid = swiglu ? tm_choose_grid<16, true>(NBr, p.KB, p.U, M, sm_count, max_smem, resident_mode, need_res,
                                               nb_bytes)
                    : tm_choose_grid<16, false>(NBr, p.KB, p.U, M, sm_count, max_smem, resident_mode, need_res,
                                                nb_bytes);
    else if (MT == 32)
      grid = swiglu ? tm_choose_grid<32, true>(NBr, p.KB, p.U, M, sm_count, max_smem, resident_mode, need_res,
                                               nb_bytes)
                    : tm_choose_grid<32, false>(NBr, p.KB, p.U, M, sm_count, max_smem, resident_mode, need_res,
                                                nb_bytes);
    else
      grid = swiglu ? tm_choose_grid<64, true>(NBr, p.KB, p.U, M, sm_count, max_smem, resident_mode, need_res,
                                               nb_bytes)
                    : tm_choose_grid<64, false>(NBr, p.KB, p.U, M, sm_count, max_smem, resident_mode, need_res,
                                                nb_bytes);
    if (grid <= 0) return 8;  // FP8GQ_ERR_UNSUPPORTED: no plan fits
  }
  if (grid > tm_slots(sm_count, MT)) return 8;  // partial-sum slots exist for at most this many CTAs
  if ((p.U + grid - 1) / grid + 1 > kTmWsCache) return 8;  // FP8GQ_ERR_UNSUPPORTED: tiles per CTA
  // aligned split: every CTA takes 1/split of one row block's K range
  const int NB = N / kGroup;
  const int split = (grid % NB == 0) ? grid / NB : 0;
  // (any split works: with G = NB * split, CTA i's stream-K range
  // [i*U/G, (i+1)*U/G) starts at row block i / split's first tile exactly when
  // i is a multiple of split, so the split CTAs of a row block cover it
  // alone, with floor(KB/split) or ceil(KB/split) K blocks each)
  const bool aligned = split > 0 && split <= p.KB;
  const int csize = (cluster_mode != 0 && aligned && split >= 2 && split <= kTmMaxCluster) ? split : 1;
  const int64_t xcols = swiglu ? 2 * static_cast<int64_t>(K) : K;
  // Pre-quantised feed: large M whose activation does not stay resident at
  // this grid -- quantise it once here (into xq_out / sx_out when given, else
  // the workspace) instead of in every CTA.  Not for a launch that waits for
  // other ranks' activation (the quant kernel would read it before the wait).
  bool pre = false;
  uint8_t* pre_xq = nullptr;
  float* pre_sx = nullptr;
  if (resident_mode != 0 && tm_prequant_shape(M) && !(norm && norm->norm) && !(gather && gather->wait_input)) {
    const int mp0 = M < MT ? M : MT;
    TmPlan pl0;
    bool ok0;
    if (MT == 16)
      ok0 = swiglu ? tm_plan<16, true>(&pl0, mp0, p.U, p.KB, grid, sm_count, max_smem, resident_mode)
                   : tm_plan<16, false>(&pl0, mp0, p.U, p.KB, grid, sm_count, max_smem, resident_mode);
    else if (MT == 32)
      ok0 = swiglu ? tm_plan<32, true>(&pl0, mp0, p.U, p.KB, grid, sm_count, max_smem, resident_mode)
                   : tm_plan<32, false>(&pl0, mp0, p.U, p.KB, grid, sm_count, max_smem, resident_mode);
    else
      ok0 = swiglu ? tm_plan<64, true>(&pl0, mp0, p.U, p.KB, grid, sm_count, max_smem, resident_mode)
                   : tm_plan<64, false>(&pl0, mp0, p.U, p.KB, grid, sm_count, max_smem, resident_mode);
    const int64_t jmax = (p.U + grid - 1) / grid;
    const int64_t nkb = jmax < p.KB ? jmax : p.KB;
    const bool legal = nkb * mp0 <= static_cast<int64_t>(kTmSxRing) * MT;   // scales fit the sx region
    const bool res_fits = ok0 && pl0.resident;
    pre = legal && (resident_mode == 2 || !res_fits ||
                    (resident_mode == 1 && nkb * mp0 >= kTmPrequantMinGroups));
  }
  if (pre) {
    uint8_t* region = static_cast<uint8_t*>(workspace) + tm_align256(tm_partials_end(M, N, K, sm_count));
    pre_xq = xq_out ? xq_out : region;
    pre_sx = sx_out ? sx_out : reinterpret_cast<float*>(region + tm_align256(static_cast<size_t>(M) * K));
    if (launch_group_quant(swiglu, static_cast<const __nv_bfloat16*>(x), ldx, M, K, pre_xq, pre_sx, stream) !=
        cudaSuccess)
      return 7;
  }
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
    p.x = xp;
    p.ldx = ldx;
    p.early_weights = early_weights;
    p.gather = gather ? *gather : GatherParams{};
    p.norm = norm ? *norm : NormParams{};
    if (norm && norm->norm) {
      p.norm.res = norm->res + static_cast<int64_t>(m0) * norm->ldr;
      if (norm->res_out) p.norm.res_out = norm->res_out + static_cast<int64_t>(m0) * norm->ldro;
    }
    if (gather) {
      // this pass's rows of every rank's output; only the first pass waits
      if (!gather->local_out)
        for (int r = 0; r < gather->world; ++r) p.gather.out[r] = gather->out[r] + static_cast<int64_t>(m0) * gather->ldo;
      if (m0 > 0) p.gather.wait_input = 0;
    }
    p.xq_out = (xq_out && !pre) ? xq_out + static_cast<int64_t>(m0) * K : nullptr;
    p.sx_out = (sx_out && !pre) ? sx_out + static_cast<int64_t>(m0) * (K / kGroup) : nullptr;
    p.prequant = pre ? 1 : 0;
    p.sx_pre = pre ? pre_sx + static_cast<int64_t>(m0) * p.KB : nullptr;
    CUtensorMap tmap_x;
    if (pre) {
      if (!cached_tmap(&tmap_x, 2, pre_xq + static_cast<int64_t>(m0) * K, p.M, K, K, MT)) return 7;
    } else if (gather && gather->tagged && gather->wait_input) {
      tmap_x = tmap_w;   // tagged words are not bf16 rows; the resident prologue reads them, no TMA
    } else if (!cached_tmap(&tmap_x, 1, xp, p.M, xcols, ldx, 0)) {
      return 7;
    }
    int st;
    if (MT == 16)
      st = swiglu ? launch_tm_pass<16, true>(tmap_w, tmap_x, p, grid, sm_count, max_smem, stream, resident_mode, csize)
                  : launch_tm_pass<16, false>(tmap_w, tmap_x, p, grid, sm_count, max_smem, stream, resident_mode, csize);
    else if (MT == 32)
      st = swiglu ? launch_tm_pass<32, true>(tmap_w, tmap_x, p, grid, sm_count, max_smem, stream, resident_mode, csize)
                  : launch_tm_pass<32, false>(tmap_w, tmap_x, p, grid, sm_count, max_smem, stream, resident_mode, csize);
    else
      st = swiglu ? launch_tm_pass<64, true>(tmap_w, tmap_x, p, grid, sm_count, max_smem, stream, resident_mode, csize)
                  : launch_tm_pass<64, false>(tmap_w, tmap_x, p, grid, sm_count, max_smem, stream, resident_mode, csize);
    if (st) return st;
  }
  return 0;
}

}  // namespace fp8gq
