// Stack runner: one persistent launch that runs a whole list of block-FP8
// linears -- a decode step's qkv, o, gate_up, down (SwiGLU) of every layer --
// in list order, each one the fused activation quant + block-scaled GEMM of
// the tile kernel (gemm_tm.cuh; kernels/fused_gemv_quant_tm.py:49-80 and
// kernels/fused_swiglu_quant_gemv.py:26-51 for the arithmetic).
//
// Why one launch.  A linear launched on its own pays a fixed cost at both
// ends -- the grid boundary, the first activation load and MMA, the last
// MMA and the stores -- during which HBM is idle; for the 4-25 MB decode
// weights that is a third of the time.  Here the weights of the next linear
// do not depend on anything: each CTA's TMA warp runs straight on into the
// next linear's weight tiles while the same CTA's MMAs still wait for that
// linear's activation, so the ring (8 stages of 16 KB per SM) keeps HBM busy
// across the dependency.
//
// Dependencies.  Linear l reads its activation only once every CTA has
// finished linear dep(l) (the latest earlier linear whose output overlaps
// this input, or whose input or output this output overlaps; the host works
// it out).  CTA i counts itself done with linear l on done[l] (release, GPU
// scope) after its stores; waiters poll with acquire loads.  CTAs take the
// linears in the same order, so done[d] == G means every CTA has finished
// every linear up to d.  The grid is one CTA per SM and launched as a
// cooperative grid, so every CTA is resident and every wait ends.
//
// Work split (per linear, stream-K): the N/128 x K/128 tiles, row-block
// major, over Gl = min(G, U) CTAs; CTA i < Gl takes tiles [i*U/Gl, (i+1)*U/Gl).  A row block split between
// CTAs leaves fp32 partial sums in the plan's scratch, and the CTA that
// finishes it last adds them in CTA order (tile-kernel protocol).  Partial
// slots and split counters alternate between two banks by linear parity; a
// CTA writes linear l's partials only after done[l-2] == G (every reader of
// that bank is past it).
//
// Token layout, MMA, TMEM groups and epilogue scaling are the tile kernel's
// (swap-AB tcgen05 kind::f8f6f4, 128 weight rows x 16 token columns, K blocks
// of a group side by side in a 16-column accumulator, per-(token, K block)
// scale sx * ws applied in the epilogue).  Per linear, the activation warps
// load the block scales of the CTA's tiles, wait for the linear's dependency,
// and quantise the activation of the CTA's K blocks once into shared memory
// (the activation is a few KB, in L2); each stage's B tile is then a copy of
// prebuilt bytes, and the tile's scales go into a ring the epilogue reads.
// Where M x (K blocks) does not fit the resident region, the owning warp
// quantises each K block from global memory instead.
//
// Warp roles (320 threads): warp 0 TMA producer (weights only), warp 1 TMEM
// allocator and MMA issuer, warps 2-5 activation producers, warps 6-9
// epilogue.  Every wait is bounded (2 s) and also gives up as soon as any
// CTA has recorded a device error; a CTA that gave up skips the rest of its
// work but still counts itself done for every linear and drains its copies
// and MMAs before it exits.
#pragma once

#include "gemm_tm.cuh"

namespace fp8gq {

constexpr int kStThreads = 320;
constexpr int kStMT = 16;                 // token tile (M <= 16)
constexpr int kStMaxStages = 12;
constexpr int kStRing = 64;               // scale ring, in tiles (> stages + 2 groups of 16)
constexpr int kStMaxLinears = 4096;
constexpr int kStMaxRowBlocks = 4096;     // N <= 524288
constexpr int kStBTileBytes = kStMT * 128;
constexpr int kStTmemCols = 64;           // 4 accumulator buffers of 16 columns
constexpr int kStWsLin = 1024;            // block scales of a CTA's tiles of one linear kept in shared memory

// One linear of the list, as the kernel reads it (device memory, 256 bytes).
struct alignas(64) StackLinear {
  CUtensorMap tmap_w;               // weight [N, K] e4m3, 128 x 128-byte boxes, SW128
  const float* ws;                  // [N/128, ldws]
  const __nv_bfloat16* x;           // [M, ldx]; SwiGLU: [gate | up], 2K columns
  __nv_bfloat16* out;               // [M, ldo]
  int64_t ldws, ldx, ldo;
  int64_t U;                        // (N/128) * (K/128)
  int N, K, KB, swiglu;
  int dep;                          // wait for done[dep] == G before reading x (-1: none)
  int pad[7];
};
static_assert(sizeof(StackLinear) == 256, "StackLinear is 256 bytes");

struct StackParams {
  const StackLinear* lin;   // [n]
  unsigned int* done;       // [n] CTAs done with linear l; zero on entry and on exit
  unsigned int* exit_count; // CTAs that finished the launch
  int* counters;            // [2][kStMaxRowBlocks] split-K counters, zero on entry and exit
  float* partials;          // [2][G][2][M][128]
  int n, M, sw, lg_sw, kpb, nacc, stages, npw;
  uint32_t b_off, bar_off, res_off;
  int res_groups;           // (token, K block) groups the resident region holds
};

// Shared memory from the 1 KB-aligned base: A tiles [S][16 KB] | B tiles
// [S][2 KB] | wfull[12] bfull[12] empty[12] acc_full[4] tmem_empty[4] drain (8 B each) |
// misc[4] | sx_tag[64] | ws_ring[64] | sx_ring[64][16]
constexpr size_t kStTailBytes = (3 * kStMaxStages + 2 * kTmMaxAcc + 1) * 8 + 16 + kStRing * 4 + kStRing * 4 +
                                kStRing * kStMT * 4;

// Bounded wait helpers: give up after the wait limit, or at once when another
// CTA (or an earlier launch) has recorded a device error.
__device__ __forceinline__ bool st_error_seen() {
  return *reinterpret_cast<volatile unsigned int*>(&g_device_error) != 0u;
}

__device__ __forceinline__ bool st_mbar_wait(uint64_t* bar, uint32_t parity, unsigned int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u) {
      if (st_error_seen()) return false;
      if (global_ns() - t0 > wait_limit_ns()) {
        record_error(site);
        return false;
      }
    }
  }
}

__device__ __forceinline__ unsigned int ld_acquire_gpu_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until *p >= want (every CTA done with a linear).
__device__ __forceinline__ bool st_wait_count(const unsigned int* p, unsigned int want) {
  if (ld_acquire_gpu_u32(p) >= want) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (ld_acquire_gpu_u32(p) >= want) return true;
    if ((it & 63u) == 0u) {
      if (st_error_seen()) return false;
      if (global_ns() - t0 > wait_limit_ns()) {
        record_error(kSiteStackDep);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void red_release_gpu_add(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The tensor map sits in global memory (written by a copy before the
// launch): order it for the TMA unit and pull it into its cache.
__device__ __forceinline__ void st_acquire_tensormap(const CUtensorMap* map) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(reinterpret_cast<uint64_t>(map))
               : "memory");
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// CTA i's range of linear l: J tiles from row block nb0, K block kb0.  A
// linear with U tiles is spread over Gl = min(G, U) CTAs, so that every CTA
// below Gl holds at least one tile (the split-K hand-off counts on it); CTAs
// from Gl on have none.
struct StRange {
  int64_t u0, U, Gl;
  int J, nb0, kb0, KB;
};

__device__ __forceinline__ StRange st_range(const StackLinear* L, int64_t G, int64_t i) {
  StRange r;
  r.U = __ldg(&L->U);
  r.KB = __ldg(&L->KB);
  r.Gl = r.U < G ? r.U : G;
  const int64_t ic = i < r.Gl ? i : r.Gl;
  r.u0 = (ic * r.U) / r.Gl;
  const int64_t u1 = i < r.Gl ? ((i + 1) * r.U) / r.Gl : r.u0;
  r.J = static_cast<int>(u1 - r.u0);
  r.nb0 = static_cast<int>(r.u0 / r.KB);
  r.kb0 = static_cast<int>(r.u0 - static_cast<int64_t>(r.nb0) * r.KB);
  return r;
}

// Tile walk inside one linear (no division on the way); the ring stage and
// its parity continue from linear to linear.
struct StCursor {
  int nb, kb, pos;
  __device__ __forceinline__ void init(const StRange& r) {
    nb = r.nb0;
    kb = r.kb0;
    pos = 0;
  }
  __device__ __forceinline__ void next(int KB, int kpb) {
    if (++kb == KB) {
      kb = 0;
      ++nb;
      pos = 0;
    } else {
      pos = (pos + 1 == kpb) ? 0 : pos + 1;
    }
  }
};

struct StRing {
  int s = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next(int S) {
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
  }
};

__global__ void __launch_bounds__(kStThreads, 1) stack_kernel(const StackParams p) {
  const int S = p.stages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* const a_tiles = smem;
  uint8_t* const b_tiles = smem + p.b_off;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + p.bar_off);   // weight tile landed (TMA bytes)
  uint64_t* bfull = wfull + kStMaxStages;                            // B tile written (activation warp)
  uint64_t* empty = bfull + kStMaxStages;
  uint64_t* acc_full = empty + kStMaxStages;
  uint64_t* tmem_empty = acc_full + kTmMaxAcc;
  uint64_t* drain = tmem_empty + kTmMaxAcc;
  uint32_t* misc = reinterpret_cast<uint32_t*>(drain + 1);            // [0] tmem base, [1] last flag
  volatile uint32_t* sx_tag = misc + 4;                               // [kStRing]
  float* ws_ring = reinterpret_cast<float*>(misc + 4 + kStRing);      // [kStRing]
  float* sx_ring = ws_ring + kStRing;                                 // [kStRing][16]
  // per-linear activation region: res_xq [res_groups][128 B], sx_res
  // [res_groups], ws_lin [kStWsLin]
  uint8_t* res_xq = smem + p.res_off;
  float* sx_res = reinterpret_cast<float*>(res_xq + static_cast<size_t>(p.res_groups) * 128);
  float* ws_lin = sx_res + p.res_groups;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int64_t G = gridDim.x;
  const int64_t cta = blockIdx.x;
  const int kpb = p.kpb;
  const int nacc = p.nacc;

  if (warp == 0) {
    if (lane < S) {
      mbar_init(&wfull[lane], 1);      // TMA arrive_expect_tx
      mbar_init(&bfull[lane], 1);      // the activation warp of the stage
      mbar_init(&empty[lane], 1);      // tcgen05.commit
    }
    if (lane < kTmMaxAcc) {
      mbar_init(&acc_full[lane], 1);   // tcgen05.commit
      mbar_init(&tmem_empty[lane], 4); // 4 epilogue warps
    }
    if (lane == 0) mbar_init(drain, 1);
    for (int r = lane; r < kStRing; r += 32) sx_tag[r] = 0u;
    fence_mbar_init();
  } else if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&misc[0])),
                 "r"(kStTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = misc[0];

  if (warp == 0) {
    // ----------------------------------------------------- TMA producer --
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      bool ok = true;
      StRing rg;
      int64_t issued = 0;
      for (int l = 0; l < p.n && ok; ++l) {
        const StackLinear* L = p.lin + l;
        const StRange r = st_range(L, G, cta);
        if (r.J == 0) continue;
        st_acquire_tensormap(&L->tmap_w);
        StCursor c;
        c.init(r);
        for (int j = 0; j < r.J; ++j, c.next(r.KB, kpb), rg.next(S)) {
          if (issued >= S) ok = st_mbar_wait(&empty[rg.s], rg.ph ^ 1u, kSiteStackRing);
          if (!ok) break;
          mbar_arrive_expect_tx(&wfull[rg.s], kTmATileBytes);
          tma_load_2d(a_tiles + rg.s * kTmATileBytes, &L->tmap_w, c.kb * 128, c.nb * 128, &wfull[rg.s], pol_w);
          ++issued;
        }
      }
      // let every copy issued land before the CTA can exit (the last S
      // stages hold the copies that may still be in flight)
      for (int64_t t = (issued > S ? issued - S : 0); t < issued; ++t)
        mbar_wait(&wfull[t % S], static_cast<uint32_t>((t / S) & 1), kSiteStackRing);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = idesc_f8<kStMT>();
      const uint64_t desc_a0 = smem_desc_sw128(smem_u32(a_tiles));
      const uint64_t desc_b0 = smem_desc_sw128(smem_u32(b_tiles));
      bool ok = true;
      StRing rg;
      AccCursor acc;
      uint32_t d_tmem = tmem_base;
      for (int l = 0; l < p.n && ok; ++l) {
        const StRange r = st_range(p.lin + l, G, cta);
        StCursor c;
        c.init(r);
        for (int j = 0; j < r.J; ++j, c.next(r.KB, kpb), rg.next(S)) {
          if (c.pos == 0) {
            acc.start_group(nacc);
            if (acc.g >= nacc) ok = st_mbar_wait(&tmem_empty[acc.a], acc.round ^ 1u, kSiteStackRing);
            if (!ok) break;
            d_tmem = tmem_base + static_cast<uint32_t>(acc.a * kStMT);
          }
          ok = st_mbar_wait(&wfull[rg.s], rg.ph, kSiteStackRing) && st_mbar_wait(&bfull[rg.s], rg.ph, kSiteStackRing);
          if (!ok) break;
          tc_fence_after();
          const uint64_t da = desc_a0 + static_cast<uint64_t>((rg.s * kTmATileBytes) >> 4);
          const uint64_t db = desc_b0 + static_cast<uint64_t>((rg.s * kStBTileBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f8(d_tmem, da + 2 * kk, db + 2 * kk, idesc, (c.pos > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty[rg.s]);
          const bool group_end = (c.pos == kpb - 1) || (c.kb == r.KB - 1) || (j == r.J - 1);
          if (group_end) mma_commit(&acc_full[acc.a]);
        }
      }
      // every MMA issued must complete before TMEM is released
      mma_commit(drain);
      mbar_wait(drain, 0, kSiteStackRing);
    }
  } else if (warp < 6) {
    // ----------------------------------------- activation producers --
    // Per linear, all four warps together: the block scales of the CTA's
    // tiles into ws_lin, the dependency wait, then (resident feed) the
    // activation of the CTA's K blocks quantised once into res_xq / sx_res.
    // Then warp w copies the B tiles of the tiles t (numbered over the whole
    // list) with t % npw == w - 2 (npw divides S, so a stage is always the
    // same warp's) from the resident bytes, or -- where M x (K blocks) does
    // not fit -- quantises each K block from global memory itself.  The four
    // warps meet at named barrier 4 at every linear, on every path.
    const int NPW = p.npw;
    const int w4 = warp - 2;
    const int aw = tid - 64;                  // 0 .. 127
    const int chunk = lane & 7;
    const int row0 = lane >> 3;
    const int oct = w4 * 4 + (lane >> 3);     // lane octet among the four warps, 0 .. 15
    const int M = p.M;
    const int sw = p.sw;
    bool ok = true;
    int64_t t = 0;            // tile number over the list
    StRing rg;
    for (int l = 0; l < p.n; ++l) {
      const StackLinear* L = p.lin + l;
      const StRange r = st_range(L, G, cta);
      if (r.J == 0) continue;                 // the same for the four warps
      const int dep = __ldg(&L->dep);
      const int swiglu = __ldg(&L->swiglu);
      const __nv_bfloat16* x = L->x;
      const int64_t ldx = __ldg(&L->ldx);
      const float* ws = L->ws;
      const int64_t ldws = __ldg(&L->ldws);
      const int K = __ldg(&L->K);
      const bool res_full = r.J >= r.KB;      // resident slot = K block; else slot = tile j
      const int nkb = res_full ? r.KB : r.J;
      const bool resident = M * nkb <= p.res_groups;
      const bool ws_pre = r.J <= kStWsLin;
      // the previous linear's copies (readers of res_xq, sx_res, ws_lin) are done
      named_bar_sync(4, 128);
      if (ws_pre) {
        for (int j = aw; j < r.J; j += 128) {
          const int tk = r.kb0 + j;
          const int dn = tk / r.KB;
          ws_lin[j] = __ldg(ws + static_cast<int64_t>(r.nb0 + dn) * ldws + (tk - dn * r.KB));
        }
      }
      if (dep >= 0) {
        uint32_t okd = ok ? 1u : 0u;
        if (ok && lane == 0) okd = st_wait_count(p.done + dep, static_cast<unsigned int>(G)) ? 1u : 0u;
        __syncwarp();
        ok = __shfl_sync(0xffffffffu, okd, 0) != 0;
      }
      if (resident) {
        // group g: token m = g / nkb, slot q = g % nkb; the loads of kPasses
        // passes are issued before any of them is quantised (one L2 round
        // trip for up to 64 groups)
        constexpr int kPasses = 4;
        const int ngroups = M * nkb;
        for (int g0 = 0; g0 < ngroups; g0 += 16 * kPasses) {
          uint4 wd[kPasses][4];
#pragma unroll
          for (int i = 0; i < kPasses; ++i) {
            const int g = g0 + 16 * i + oct;
            if (ok && g < ngroups) {
              const int m = g / nkb;
              const int q = g - m * nkb;
              int kb = res_full ? q : r.kb0 + q;
              if (kb >= r.KB) kb -= r.KB;
              const uint4* xr =
                  reinterpret_cast<const uint4*>(x + static_cast<int64_t>(m) * ldx + kb * 128 + chunk * 16);
              wd[i][0] = __ldcg(xr);
              wd[i][1] = __ldcg(xr + 1);
              if (swiglu) {
                const uint4* ur = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(xr) + K);
                wd[i][2] = __ldcg(ur);
                wd[i][3] = __ldcg(ur + 1);
              }
            }
          }
#pragma unroll
          for (int i = 0; i < kPasses; ++i) {
            if (g0 + 16 * i >= ngroups) continue;   // the same for every lane
            const int g = g0 + 16 * i + oct;
            const bool live = ok && g < ngroups;  // the same within a lane octet
            const int m = live ? g / nkb : 0;
            const int q = live ? g - m * nkb : 0;
            float v[16];
            if (live) {
              if (swiglu)
                act16<true>(v, wd[i][0], wd[i][1], wd[i][2], wd[i][3]);
              else
                act16<false>(v, wd[i][0], wd[i][1], wd[i][0], wd[i][1]);
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] = 0.0f;
            }
            float sx;
            const uint4 packed = quant16_octet(v, live, sx);
            if (live) {
              *reinterpret_cast<uint4*>(res_xq + (static_cast<int64_t>(q) * M + m) * 128 + chunk * 16) = packed;
              if (chunk == 0) sx_res[q * M + m] = sx;
            }
          }
        }
      }
      if (resident || ws_pre) named_bar_sync(4, 128);   // resident bytes, scales and ws_lin written
      StCursor c;
      c.init(r);
      for (int j = 0; j < r.J; ++j, c.next(r.KB, kpb), rg.next(S), ++t) {
        if (static_cast<int>(t % NPW) != w4 || !ok) continue;
        const float wsv = ws_pre ? ws_lin[j] : __ldg(ws + static_cast<int64_t>(c.nb) * ldws + c.kb);
        uint8_t* btile = b_tiles + rg.s * kStBTileBytes;
        float* sxs = sx_ring + (t & (kStRing - 1)) * kStMT;
        if (resident) {
          if (t >= S) {
            uint32_t oke = 1;
            if (lane == 0) oke = st_mbar_wait(&empty[rg.s], rg.ph ^ 1u, kSiteStackRing) ? 1u : 0u;
            __syncwarp();
            ok = __shfl_sync(0xffffffffu, oke, 0) != 0;
            if (!ok) continue;
          }
          const int q = res_full ? c.kb : j;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int br = row0 + 4 * i;
            const int m = br - c.pos * sw;
            const bool live = m >= 0 && m < sw && m < M;
            uint4 packed = make_uint4(0u, 0u, 0u, 0u);
            if (live) {
              packed = *reinterpret_cast<const uint4*>(res_xq + (static_cast<int64_t>(q) * M + m) * 128 + chunk * 16);
              if (chunk == 0) sxs[m] = sx_res[q * M + m];
            }
            *reinterpret_cast<uint4*>(btile + br * 128 + ((chunk ^ (br & 7)) << 4)) = packed;
          }
        } else {
          // M x (K blocks) does not fit the resident region: quantise this
          // K block from global memory, one row of the lane's four at a time
          if (t >= S) {
            uint32_t oke = 1;
            if (lane == 0) oke = st_mbar_wait(&empty[rg.s], rg.ph ^ 1u, kSiteStackRing) ? 1u : 0u;
            __syncwarp();
            ok = __shfl_sync(0xffffffffu, oke, 0) != 0;
            if (!ok) continue;
          }
#pragma unroll 1
          for (int i = 0; i < 4; ++i) {
            const int br = row0 + 4 * i;             // row br of the B tile holds token br - pos*sw
            const int m = br - c.pos * sw;
            const bool live = m >= 0 && m < sw && m < M;
            uint4 packed = make_uint4(0u, 0u, 0u, 0u);
            if (__any_sync(0xffffffffu, live)) {    // rows of a lane octet are all live or all not
              float v[16];
              if (live) {
                const uint4* xr =
                    reinterpret_cast<const uint4*>(x + static_cast<int64_t>(m) * ldx + c.kb * 128 + chunk * 16);
                const uint4 xa = __ldcg(xr), xb = __ldcg(xr + 1);
                if (swiglu) {
                  const uint4* ur = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(xr) + K);
                  act16<true>(v, xa, xb, __ldcg(ur), __ldcg(ur + 1));
                } else {
                  act16<false>(v, xa, xb, xa, xb);
                }
              } else {
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = 0.0f;
              }
              float sx;
              packed = quant16_octet(v, live, sx);
              if (live && chunk == 0) sxs[m] = sx;
            }
            *reinterpret_cast<uint4*>(btile + br * 128 + ((chunk ^ (br & 7)) << 4)) = packed;
          }
        }
        if (lane == 0) ws_ring[t & (kStRing - 1)] = wsv;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bfull[rg.s]);
          __threadfence_block();
          sx_tag[t & (kStRing - 1)] = static_cast<uint32_t>(t + 1);
        }
      }
    }
  } else {
    // -------------------------------------------------------- epilogue --
    const int q4 = warp & 3;
    const int row = 32 * q4 + lane;
    const uint32_t t_lane = static_cast<uint32_t>(32 * q4) << 16;
    const int M = p.M;
    const int sw = p.sw;
    bool ok = true;
    int64_t t = 0;
    AccCursor accc;
    float acc[kStMT];
#pragma unroll
    for (int cc = 0; cc < kStMT; ++cc) acc[cc] = 0.0f;
    for (int l = 0; l < p.n; ++l) {
      const StackLinear* L = p.lin + l;
      const StRange r = st_range(L, G, cta);
      const int bank = l & 1;
      __nv_bfloat16* out = L->out;
      const int64_t ldo = __ldg(&L->ldo);
      int seg_j0 = 0, seg_kb0 = 0;
      // The partial bank of linear l was last used by linear l - 2: before
      // any partial of l is written every CTA must be past l - 2.  Checked
      // here, at the start of the linear, off the path of its last group.
      if (l >= 2 && r.J > 0) {
        uint32_t okw = ok ? 1u : 0u;
        if (ok && lane == 0) okw = st_wait_count(p.done + (l - 2), static_cast<unsigned int>(G)) ? 1u : 0u;
        __syncwarp();
        ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
      }
      StCursor c;
      c.init(r);
      for (int j = 0; j < r.J; ++j, c.next(r.KB, kpb), ++t) {
        const int nb = c.nb;
        const int kb = c.kb;
        const int pos = c.pos;
        if (pos == 0) accc.start_group(nacc);
        if (j == 0 || kb == 0) {
          seg_j0 = j;
          seg_kb0 = kb;
#pragma unroll
          for (int cc = 0; cc < kStMT; ++cc) acc[cc] = 0.0f;
        }
        const bool group_end = (pos == kpb - 1) || (kb == r.KB - 1) || (j == r.J - 1);
        if (!group_end) continue;
        // After a failed wait the warp keeps the same path (every named
        // barrier below is reached by all four epilogue warps) but skips
        // its waits and TMEM reads.
        const int a = accc.a;
        const int64_t tq0 = t - pos;          // first tile of the group
        if (ok) ok = st_mbar_wait(&acc_full[a], accc.round, kSiteStackRing);
        if (ok && lane == 0) {
          for (int q = 0; q <= pos && ok; ++q) {
            const int64_t tq = tq0 + q;
            volatile uint32_t* tag = sx_tag + (tq & (kStRing - 1));
            const uint32_t want = static_cast<uint32_t>(tq + 1);
            if (*tag != want) {
              const uint64_t t0 = global_ns();
              for (uint32_t it = 1; *tag != want; ++it)
                if ((it & 255u) == 0u && (st_error_seen() || global_ns() - t0 > wait_limit_ns())) {
                  record_error(kSiteStackRing);
                  ok = false;
                  break;
                }
            }
          }
          __threadfence_block();
        }
        ok = __all_sync(0xffffffffu, ok) != 0;   // tcgen05.ld below is warp-collective
        // column cc holds token cc % sw of the group's K block cc / sw; its
        // scale is sx[token, K block] * ws[row block, K block]
        float scl[16];
        uint32_t mask = 0;
#pragma unroll
        for (int cc = 0; cc < 16; ++cc) {
          const int q = cc >> p.lg_sw;
          const int m = cc & (sw - 1);
          const bool use = q <= pos && m < M;
          const int64_t tq = tq0 + (use ? q : 0);
          const int slot = static_cast<int>(tq & (kStRing - 1));
          scl[cc] = sx_ring[slot * kStMT + (use ? m : 0)] * ws_ring[slot];
          mask |= use ? (1u << cc) : 0u;
        }
        if (ok) {
          tc_fence_after();
          float v[16];
          tmem_ld16(tmem_base + t_lane + static_cast<uint32_t>(a * kStMT), v);
#pragma unroll
          for (int cc = 0; cc < 16; ++cc)
            if ((mask >> cc) & 1u) acc[cc] = fmaf(v[cc], scl[cc], acc[cc]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[a]);

        if (kb == r.KB - 1 || j == r.J - 1) {
          // fold the K-block slots: column m then holds token m's sum
#pragma unroll
          for (int h = kStMT / 2; h >= 1; h >>= 1)
            if (sw <= h) {
#pragma unroll
              for (int cc = 0; cc < h; ++cc) acc[cc] += acc[cc + h];
            }
          const int n = nb * 128 + row;
          const bool whole = seg_kb0 == 0 && kb == r.KB - 1;   // the same for the four warps
          if (whole) {
#pragma unroll
            for (int m = 0; m < kStMT; ++m)
              if (m < M) out[static_cast<int64_t>(m) * ldo + n] = __float2bfloat16_rn(acc[m]);
          } else {
            // partial row block: publish, count, and let the last CTA reduce
            // (the bank is free: see the wait at the start of the linear)
            const int slot = (seg_j0 == 0) ? 0 : 1;
            float* mine = p.partials + (((static_cast<int64_t>(bank) * G + cta) * 2 + slot) * M) * 128;
#pragma unroll
            for (int m = 0; m < kStMT; ++m)
              if (m < M) mine[m * 128 + row] = acc[m];
            // the barrier orders every epilogue thread's partial stores
            // before the release half of the counter update; its acquire
            // half orders the reduction's loads after the other CTAs' stores
            named_bar_sync(2, 128);
            const int64_t first_u = static_cast<int64_t>(nb) * r.KB;
            const int64_t last_u = first_u + r.KB - 1;
            const int64_t i_lo = ((first_u + 1) * r.Gl - 1) / r.U;   // owners of its first and last tile
            const int64_t i_hi = ((last_u + 1) * r.Gl - 1) / r.U;
            int* counter = p.counters + bank * kStMaxRowBlocks + nb;
            if (tid == 192) {
              const int old = atomic_add_acq_rel_gpu(counter, 1);
              const bool last = (old == static_cast<int>(i_hi - i_lo));
              misc[1] = last ? 1u : 0u;
              if (last) *counter = 0;
            }
            named_bar_sync(2, 128);
            if (misc[1]) {
              float sum[kStMT];
#pragma unroll
              for (int m = 0; m < kStMT; ++m) sum[m] = 0.0f;
              // the partials of up to 8 CTAs are loaded together and added
              // in CTA order
              const int si_lo = ((i_lo * r.U) / r.Gl == first_u) ? 0 : 1;
              for (int64_t i0 = i_lo; i0 <= i_hi; i0 += 8) {
                const int cnt = static_cast<int>(i_hi - i0 + 1 < 8 ? i_hi - i0 + 1 : 8);
                // float offset of contributor q's partial slot (< 2^32: 2 x 148 x 2 x 16 x 128);
                // every contributor after i_lo starts inside this row block (slot 0)
                auto off = [&](int q) {
                  const int64_t i = i0 + (q < cnt ? q : 0);
                  return static_cast<uint32_t>(
                      (((static_cast<int64_t>(bank) * G + i) * 2 + (i == i_lo ? si_lo : 0)) * M) * 128 + row);
                };
#pragma unroll
                for (int m = 0; m < kStMT; ++m) {
                  if (m < M) {
                    float v[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) v[q] = q < cnt ? __ldcg(p.partials + off(q) + m * 128) : 0.0f;
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                      if (q < cnt) sum[m] += v[q];
                  }
                }
              }
#pragma unroll
              for (int m = 0; m < kStMT; ++m)
                if (m < M) out[static_cast<int64_t>(m) * ldo + n] = __float2bfloat16_rn(sum[m]);
            }
            named_bar_sync(2, 128);
          }
        }
      }
      // this CTA is done with linear l: after every epilogue thread's
      // stores, one release add (a CTA that gave up still counts itself, so
      // that the others are not held up)
      named_bar_sync(3, 128);
      if (tid == 192) red_release_gpu_add(p.done + l, 1u);
    }
  }

  // ------------------------------------------------------------- exit --
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    // the last CTA out resets the done counters for the next launch (every
    // CTA has passed all of its waits by now)
    const int old = atomic_add_acq_rel_gpu(reinterpret_cast<int*>(p.exit_count), 1);
    if (old == static_cast<int>(G) - 1) {
      for (int l = 0; l < p.n; ++l) p.done[l] = 0u;
      *p.exit_count = 0u;
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kStTmemCols));
  }
}

// --------------------------------------------------------------- host --

// Device bytes of a plan: the linear table, done counters, split counters
// and the partial-sum banks (two banks of G CTAs x 2 slots x M x 128 fp32).
inline size_t st_table_bytes(int n) { return tm_align256(static_cast<size_t>(n) * sizeof(StackLinear)); }
inline size_t st_done_bytes(int n) { return tm_align256(static_cast<size_t>(n + 1) * 4); }
inline size_t st_counter_bytes() { return tm_align256(static_cast<size_t>(2) * kStMaxRowBlocks * 4); }
inline size_t st_partial_bytes(int M, int G) { return static_cast<size_t>(2) * G * 2 * M * 128 * 4; }
inline size_t st_plan_bytes(int n, int M, int G) {
  return st_table_bytes(n) + st_done_bytes(n) + st_counter_bytes() + st_partial_bytes(M, G);
}

// Ring depth: 8 stages (or 6 or 4 where shared memory is short; the
// activation warps in use divide the depth), leaving the rest of the shared
// memory to the per-linear resident activation.
inline int st_pick_stages(int64_t fit) { return fit >= 8 ? 8 : fit >= 6 ? 6 : fit >= 4 ? 4 : 0; }

// Shared-memory layout of a launch with S stages: the ring, the barrier and
// ring tail, then the resident activation region with what is left.
struct StLayout {
  uint32_t b_off, bar_off, res_off;
  int res_groups;
  size_t smem;
};
inline bool st_layout(int S, int max_smem, StLayout* lo) {
  lo->b_off = static_cast<uint32_t>(S * kTmATileBytes);
  lo->bar_off = lo->b_off + static_cast<uint32_t>(S * kStBTileBytes);
  lo->res_off = lo->bar_off + static_cast<uint32_t>((kStTailBytes + 15) / 16 * 16);
  // 4 KB below the per-block limit: headroom for the runtime's own
  // per-block shared memory, so that one CTA per SM always fits
  const int64_t left = static_cast<int64_t>(max_smem) - 4096 - 1024 - lo->res_off - kStWsLin * 4;
  if (left < 0) return false;
  lo->res_groups = static_cast<int>(left / (128 + 4));
  lo->smem = 1024 + lo->res_off + static_cast<size_t>(lo->res_groups) * (128 + 4) + kStWsLin * 4;
  return lo->smem <= static_cast<size_t>(max_smem);
}

}  // namespace fp8gq
