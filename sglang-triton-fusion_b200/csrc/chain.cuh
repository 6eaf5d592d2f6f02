// A decode step's M == 1 linears in one persistent launch, linked by tagged
// words (the chain runner).
//
// Each linear of the list is N-sharded as in the gathered calls: this rank
// holds rows [col0, col0 + N) of the full output, and its CTAs store them as
// tagged words (two bf16 columns and a sequence number per 64-bit word) into
// every rank's output buffer of that linear.  A linear whose input is the
// output of an earlier linear of the list (`src`) polls the words it reads
// until they carry that linear's sequence number -- written by this rank's
// other CTAs and by the other ranks alike -- so the list runs with no grid
// barrier, no flag and no kernel boundary between linears.  The weights are
// static: the producer warp streams the CTA's weight rows of every linear, in
// list order, through one ring of shared-memory stages, so the stream for the
// next linears continues while the consumers wait for an input.
//
// Work split and math are the row kernel's (gemv_row.cuh): CTA b of G owns
// the contiguous row groups [b*U/G, (b+1)*U/G) of each linear (U groups of R
// rows; rows in pairs when R == 1, since a tagged word holds two columns),
// T consumer threads split K into 16-column chunks, the activation is
// quantised per thread into registers, and each row's dot product is a
// per-chunk fp32 sum scaled by sx * ws, reduced across the warps through a
// shared-memory window -- the row kernel's steps in the row kernel's order.
//
// All CTAs must be resident at once (one CTA waits for another's output):
// the launch is cooperative.  Every wait is bounded (the peer limit for
// words and flags, twice that for the ring), so a lost peer or a CTA that
// never ran ends the kernel with the error word set, not a hang.
#pragma once

#include "fp8gq_device.cuh"
#include "gemv_row.cuh"

namespace fp8gq {

constexpr int kChainThreads = 256;        // consumer threads (8 warps) + one producer warp
constexpr int kChainC = 3;                // 16-column chunks per thread: K <= 3 * 256 * 16 = 12288
constexpr int kChainMaxK = kChainC * kChainThreads * 16;
constexpr int kChainSlotBytes = 16384;    // one ring stage: R rows of K bytes, R * K <= 16 KB
constexpr int kChainRingBytes = 96 * 1024;

// One linear of a chain as the kernel reads it (device memory, filled by
// fp8gq_chain_prepare).
struct ChainLin {
  const void* x;            // src >= 0: words of linear src's output row; src < 0: bf16 row
  const uint8_t* w;         // [N, ldw] e4m3: this rank's rows
  const float* ws;          // [N/128, ldws]
  int64_t ldw, ldws;
  int N, K;                 // rows of this rank; input columns (of gate and of up with swiglu)
  int src;                  // the linear whose output x is, or -1 (bf16 input)
  int swiglu;               // x is [gate | up], 2K columns
  int col0;                 // this rank's first column in the full output
  int R;                    // rows per ring stage (1, 2 or 4)
  int units;                // work units: N / R row groups, N / 2 row pairs when R == 1
  int unit_stages;          // ring stages per unit (2 when R == 1, else 1)
  uint64_t* out[kMaxGatherRanks];   // rank r's output words of this linear
};

struct ChainParams {
  const ChainLin* lin;
  int n;                    // linears in the list
  int stages;               // ring depth
  unsigned int* flags[kMaxGatherRanks];   // rank q's flag array, as mapped here
  unsigned int* counter;    // this rank: CTAs done with the list
  unsigned int* seq;        // this rank: sequence number before the list
  int world, rank;
};

// The sequence numbers of a list of n linears after s: s + 1 .. s + n, or
// 1 .. n where that range would pass 0 (0 is never a tag).
__device__ __forceinline__ unsigned int chain_base(unsigned int s, int n) {
  return (s + static_cast<unsigned int>(n) < s) ? 0u : s;
}

// The consumer part of one linear for one CTA: this CTA's ring stages of it
// (n_stages of them, starting at stage counter gs), its rows' dot products
// with the quantised activation held in xh / sx_c / blk, the window reduction
// and the tagged stores.  Returns the stage counter after the linear.
template <int R>
__device__ __forceinline__ int chain_rows(const ChainParams& p, const ChainLin& L, int row_begin, int n_stages,
                                          int gs, const uint32_t (&xh)[kChainC][8], const float (&sx_c)[kChainC],
                                          const int (&blk)[kChainC], uint8_t* smem, uint64_t* full,
                                          uint64_t* empty, float* window, int tid, int warp, int lane,
                                          unsigned int tag_out, bool& ok, bool& store_wait, unsigned int s_prev) {
  constexpr int T = kChainThreads;
  constexpr int n_cwarps = T / 32;
  const int n_chunks = L.K / 16;
  float s_cur[kChainC];
  int nb_cur = -1;
  int win_buf = 0;
  const int my_row_in_group = row_of_lane<R>(lane);
  const bool row_writer = (lane & ((32 / R) - 1)) == 0;
  for (int j = 0; j < n_stages; ++j, ++gs) {
    const int s = gs % p.stages;
    if (ok) ok = mbar_wait(&full[s], (gs / p.stages) & 1, kSiteRowFull);
    const int row0 = row_begin + j * R;
    const int nb = row0 >> 7;
    if (nb != nb_cur) {
      nb_cur = nb;
#pragma unroll
      for (int i = 0; i < kChainC; ++i) {
        const int c = tid + T * i;
        s_cur[i] = (c < n_chunks) ? sx_c[i] * __ldg(L.ws + static_cast<int64_t>(nb) * L.ldws + blk[i]) : 0.0f;
      }
    }
    float acc[R];
    const uint8_t* stage = smem + static_cast<size_t>(s) * kChainSlotBytes;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      acc[r] = 0.0f;
#pragma unroll
      for (int i = 0; i < kChainC; ++i) {
        const int c = tid + T * i;
        if (c < n_chunks && ok) {
          const uint4 wv = *reinterpret_cast<const uint4*>(stage + r * L.K + 16 * c);
          acc[r] = fmaf(dot16_e4m3(wv, xh[i]), s_cur[i], acc[r]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const float rs = warp_reduce_rows<R>(acc, lane);
    const int row_in_win = (j * R) % kRowWindow;
    float* win = window + (win_buf * n_cwarps) * kRowWindow;
    if (row_writer) win[warp * kRowWindow + row_in_win + my_row_in_group] = rs;

    const int done_rows = (j + 1) * R;
    if (done_rows % kRowWindow == 0 || j == n_stages - 1) {
      named_bar_sync(1, T);
      if (warp == 0) {
        if (store_wait) {
          // the list's first stores: every rank has finished its previous
          // list (its own flag slot), so nobody still reads these buffers
          if (lane < p.world) {
            const unsigned int* flag = p.flags[lane] + lane;
            const uint64_t t0 = global_ns();
            for (uint32_t it = 0;; ++it) {
              if (static_cast<int>(ld_acquire_sys_u32(flag) - s_prev) >= 0) break;
              if ((it & 255u) == 255u && global_ns() - t0 > peer_wait_limit_ns()) {
                record_error(kSiteGather);
                break;
              }
            }
          }
          __syncwarp();
          store_wait = false;
        }
        const int wrow0 = ((done_rows - 1) / kRowWindow) * kRowWindow;
        const int nrows = done_rows - wrow0;
        float sum = 0.0f;
        if (lane < nrows)
          for (int w = 0; w < n_cwarps; ++w) sum += win[w * kRowWindow + lane];
        const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(sum));
        const uint32_t hi = __shfl_down_sync(0xffffffffu, lo, 1);
        if (lane < nrows && !(lane & 1)) {
          const int64_t wi = (static_cast<int64_t>(L.col0) + row_begin + wrow0 + lane) >> 1;
          const uint64_t word = static_cast<uint64_t>(lo | (hi << 16)) | (static_cast<uint64_t>(tag_out) << 32);
#pragma unroll 1
          for (int r = 0; r < p.world; ++r)
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(L.out[r] + wi), "l"(word) : "memory");
        }
      }
      win_buf ^= 1;
    }
  }
  return gs;
}

__global__ void __launch_bounds__(kChainThreads + 32, 2) chain_kernel(const ChainParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int T = kChainThreads;
  constexpr int n_cwarps = T / 32;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(p.stages) * kChainSlotBytes);
  uint64_t* empty = full + p.stages;
  float* window = reinterpret_cast<float*>(empty + p.stages);   // [2][n_cwarps][32]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = gridDim.x;
  const int b = blockIdx.x;

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], n_cwarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // ------------------------------------------------------------ producer --
  if (warp == n_cwarps) {
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int gs = 0;
      bool ok = true;
      // the weights are static: no wait before streaming them
      for (int li = 0; li < p.n && ok; ++li) {
        const ChainLin& L = p.lin[li];
        const int u0 = static_cast<int>((static_cast<int64_t>(b) * L.units) / G);
        const int u1 = static_cast<int>((static_cast<int64_t>(b + 1) * L.units) / G);
        const int n_st = (u1 - u0) * L.unit_stages;
        const int row_begin = u0 * L.unit_stages * L.R;
        const uint32_t bytes = static_cast<uint32_t>(L.R * L.K);
        for (int j = 0; j < n_st; ++j, ++gs) {
          const int s = gs % p.stages;
          if (gs >= p.stages && !mbar_wait(&empty[s], ((gs / p.stages) & 1) ^ 1, kSiteRowEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], bytes);
          const int64_t row0 = row_begin + static_cast<int64_t>(j) * L.R;
          uint8_t* dst = smem + static_cast<size_t>(s) * kChainSlotBytes;
          if (L.ldw == L.K) {
            bulk_g2s(dst, L.w + row0 * L.K, bytes, &full[s], pol);
          } else {
            for (int r = 0; r < L.R; ++r)
              bulk_g2s(dst + r * L.K, L.w + (row0 + r) * L.ldw, static_cast<uint32_t>(L.K), &full[s], pol);
          }
        }
      }
      grid_launch_dependents();
    }
    return;
  }

  // ----------------------------------------------------------- consumers --
  // the activation of the first linear and the sequence number belong to the
  // stream's previous work
  grid_dependency_wait();
  const unsigned int s_prev = *reinterpret_cast<volatile unsigned int*>(p.seq);
  const unsigned int s0 = chain_base(s_prev, p.n);
  int gs = 0;
  bool ok = true;
  bool live = true;          // false once a word poll gave up: no further waits
  bool store_wait = true;    // warp 0 polls the ranks' flag slots before the first stores
  for (int li = 0; li < p.n; ++li) {
    const ChainLin& L = p.lin[li];
    const int u0 = static_cast<int>((static_cast<int64_t>(b) * L.units) / G);
    const int u1 = static_cast<int>((static_cast<int64_t>(b + 1) * L.units) / G);
    const int n_st = (u1 - u0) * L.unit_stages;
    if (n_st == 0) continue;
    const int row_begin = u0 * L.unit_stages * L.R;
    const unsigned int tag_in = s0 + static_cast<unsigned int>(L.src) + 1u;
    const unsigned int tag_out = s0 + static_cast<unsigned int>(li) + 1u;

    // the activation, quantised into registers (as the row kernel's prologue)
    const int n_chunks = L.K / 16;
    uint32_t xh[kChainC][8];
    float sx_c[kChainC];
    int blk[kChainC];
#pragma unroll
    for (int i = 0; i < kChainC; ++i) {
      const int c = tid + T * i;
      const bool valid = c < n_chunks;
      float v[16];
      if (valid) {
        uint32_t gw[8], uw[8];
        if (L.src >= 0) {
          const uint64_t* gp = static_cast<const uint64_t*>(L.x) + 8 * c;
          uint64_t gv[8];
          tagged_issue8(gp, gv);
          if (L.swiglu) {
            const uint64_t* up = static_cast<const uint64_t*>(L.x) + L.K / 2 + 8 * c;
            uint64_t uv[8];
            tagged_issue8(up, uv);
            tagged_finish8(up, tag_in, uv, uw, live);
          }
          tagged_finish8(gp, tag_in, gv, gw, live);
        } else {
          const uint4* gp = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(L.x) + 16 * c);
          const uint4 a = gp[0], bq = gp[1];
          gw[0] = a.x; gw[1] = a.y; gw[2] = a.z; gw[3] = a.w;
          gw[4] = bq.x; gw[5] = bq.y; gw[6] = bq.z; gw[7] = bq.w;
          if (L.swiglu) {
            const uint4* up =
                reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(L.x) + L.K + 16 * c);
            const uint4 ua = up[0], ub = up[1];
            uw[0] = ua.x; uw[1] = ua.y; uw[2] = ua.z; uw[3] = ua.w;
            uw[4] = ub.x; uw[5] = ub.y; uw[6] = ub.z; uw[7] = ub.w;
          }
        }
        if (L.swiglu) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            v[2 * e] = silu_mul(bf16_lo(gw[e]), bf16_lo(uw[e]));
            v[2 * e + 1] = silu_mul(bf16_hi(gw[e]), bf16_hi(uw[e]));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            v[2 * e] = bf16_lo(gw[e]);
            v[2 * e + 1] = bf16_hi(gw[e]);
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
#pragma unroll
      for (int e = 0; e < 8; ++e) xh[i][e] = e4m3x2_to_f16x2(quant_pair(v[2 * e], v[2 * e + 1], sinv));
      sx_c[i] = sx;
      blk[i] = c >> 3;
    }

    switch (L.R) {
      case 4:
        gs = chain_rows<4>(p, L, row_begin, n_st, gs, xh, sx_c, blk, smem, full, empty, window, tid, warp, lane,
                           tag_out, ok, store_wait, s_prev);
        break;
      case 2:
        gs = chain_rows<2>(p, L, row_begin, n_st, gs, xh, sx_c, blk, smem, full, empty, window, tid, warp, lane,
                           tag_out, ok, store_wait, s_prev);
        break;
      default:
        gs = chain_rows<1>(p, L, row_begin, n_st, gs, xh, sx_c, blk, smem, full, empty, window, tid, warp, lane,
                           tag_out, ok, store_wait, s_prev);
        break;
    }
    named_bar_sync(1, T);     // the window is reused by the next linear
  }

  // the last CTA to finish moves this rank's sequence number past the list and
  // raises its own flag slot (the next list's first stores wait for it)
  named_bar_sync(1, T);
  if (tid == 0) {
    unsigned int old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.counter) : "memory");
    if (old == static_cast<unsigned int>(G) - 1u) {
      *p.counter = 0u;
      const unsigned int s = s0 + static_cast<unsigned int>(p.n);
      *p.seq = s;
      asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p.flags[p.rank] + p.rank), "r"(s) : "memory");
    }
  }
}

}  // namespace fp8gq
