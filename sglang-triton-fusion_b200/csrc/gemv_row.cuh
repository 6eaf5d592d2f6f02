// M == 1 fused quant + GEMV on CUDA cores (replaces gemv_quant_row_kernel,
// kernels/fused_gemv_quant_tm.py:25-46, and swiglu_q_gemm_kernel at M == 1,
// kernels/fused_swiglu_quant_gemv.py:26-51).
//
// Work split.  The N weight rows are cut into row groups of R rows; CTA i of
// G owns the contiguous row groups [i*NG/G, (i+1)*NG/G), so every CTA streams
// one contiguous slice of W and computes whole dot products: no split-K, no
// scratch memory, one bf16 store per row.
//
// Pipeline.  One producer warp issues 1-D bulk copies (TMA) of R rows
// (R*K bytes) into a ring of shared-memory stages; `full[s]` counts the bytes,
// `empty[s]` counts the consumer warps that are done with the stage.
//
// Consumers.  T threads (T % 32 == 0) split K: thread t owns the 16-byte
// column chunks t, t+T, ..., t+(C-1)T, i.e. the same K positions in every
// row, so its slice of the quantised activation is computed once and kept in
// registers (as f16 pairs: every e4m3 value is exact in f16).  For each row it
// forms 16-product partial sums per chunk with fp32 accumulation
// (fma.rn.f32.f16: products are exact), scales each by sx[b] * ws[n/128, b]
// -- all 16 columns of a chunk lie in one 128-block b -- and sums; a warp
// butterfly reduces the R rows at once, and per-warp row sums go through a
// double-buffered 32-row window in shared memory where warp 0 adds them up
// and stores bf16.
#pragma once

#include "fp8gq_device.cuh"

namespace fp8gq {

struct RowParams {
  const __nv_bfloat16* x;   // [K] (plain) or [2K] = [gate | up] (SwiGLU)
  const uint8_t* w;         // [N, ldw] e4m3
  int64_t ldw;
  const float* ws;          // [N/128, ldws]
  int64_t ldws;
  __nv_bfloat16* out;       // [N]
  int N, K;
  int n_groups;             // N / R
  int stages;               // ring depth
  uint8_t* xq_out;          // optional [K]
  float* sx_out;            // optional [K/128]
  int early_weights;        // weights are static: fetch the first stages before the grid-dependency wait
  GatherParams gather;      // N-sharded output written to every rank (world > 0)
  NormParams norm;          // add + RMSNorm prologue (plain kernel only)
};

constexpr int kRowMaxConsumerThreads = 384;  // the launcher never picks T > 384
constexpr int kRowWindow = 32;  // rows per reduction window

// Shared-memory layout after the ring: full[stages], empty[stages],
// window[2][n_consumer_warps][32] fp32.
__host__ __device__ inline size_t row_smem_bytes(int stages, int stage_bytes, int n_cwarps) {
  size_t ring = static_cast<size_t>(stages) * stage_bytes;
  size_t bars = static_cast<size_t>(2 * stages) * sizeof(uint64_t);
  size_t win = static_cast<size_t>(2 * n_cwarps * kRowWindow) * sizeof(float);
  return ring + bars + win;
}

// Sum of 16 exact products xq[k] * w[k] in fp32 (two accumulators).
__device__ __forceinline__ float dot16_e4m3(const uint4 wv, const uint32_t (&xh)[8]) {
  float a0 = 0.0f, a1 = 0.0f;
  const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t wlo = e4m3x2_to_f16x2(static_cast<uint16_t>(words[q] & 0xFFFFu));
    const uint32_t whi = e4m3x2_to_f16x2(static_cast<uint16_t>(words[q] >> 16));
    asm("{\n\t.reg .b16 w0, w1, x0, x1;\n\t"
        "mov.b32 {w0, w1}, %2;\n\t"
        "mov.b32 {x0, x1}, %3;\n\t"
        "fma.rn.f32.f16 %0, w0, x0, %0;\n\t"
        "fma.rn.f32.f16 %1, w1, x1, %1;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(wlo), "r"(xh[2 * q]));
    asm("{\n\t.reg .b16 w0, w1, x0, x1;\n\t"
        "mov.b32 {w0, w1}, %2;\n\t"
        "mov.b32 {x0, x1}, %3;\n\t"
        "fma.rn.f32.f16 %0, w0, x0, %0;\n\t"
        "fma.rn.f32.f16 %1, w1, x1, %1;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(whi), "r"(xh[2 * q + 1]));
  }
  return a0 + a1;
}

// Butterfly over the warp that reduces R per-lane values at once.  Returns
// the full warp sum of row `row_of_lane(lane)` in every lane.
template <int R>
__device__ __forceinline__ float warp_reduce_rows(float (&v)[R], int lane) {
  int n = R;
  int off = 16;
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    if (n > 1) {
      const int half = n / 2;
      const bool up = (lane & off) != 0;
#pragma unroll
      for (int k = 0; k < R / 2; ++k) {
        if (k < half) {
          const float send = up ? v[k] : v[k + half];
          const float keep = up ? v[k + half] : v[k];
          v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      n = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
    off >>= 1;
  }
  return v[0];
}

template <int R>
__device__ __forceinline__ int row_of_lane(int lane) {
  int row = 0, n = R, off = 16;
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    if (n > 1) {
      const int half = n / 2;
      if (lane & off) row += half;
      n = half;
    }
    off >>= 1;
  }
  return row;
}

// kTagged: the gather uses tagged words (a separate instance, so that the
// plain kernel's code is unchanged by the protocol).
template <int C, int R, bool kSwiglu, bool kTagged = false>
__global__ void __launch_bounds__(kRowMaxConsumerThreads + 32, 1)
gemv_row_kernel(const RowParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int stage_bytes = R * p.K;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(p.stages) * stage_bytes);
  uint64_t* empty = full + p.stages;
  const int n_cwarps = blockDim.x / 32 - 1;
  const int T = n_cwarps * 32;
  float* window = reinterpret_cast<float*>(empty + p.stages);  // [2][n_cwarps][32]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // tagged words pair columns 2i, 2i + 1 in one store: with one row per group
  // the CTAs split the rows in pairs (the host checks n_groups is even)
  constexpr int gu = (R == 1 && kTagged) ? 2 : 1;
  const int g0 = gu * static_cast<int>((static_cast<int64_t>(blockIdx.x) * (p.n_groups / gu)) / gridDim.x);
  const int g1 = gu * static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * (p.n_groups / gu)) / gridDim.x);
  const int n_my = g1 - g0;

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
      auto issue = [&](int j) {
        const int s = j % p.stages;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(stage_bytes));
        const int64_t row0 = static_cast<int64_t>(g0 + j) * R;
        uint8_t* dst = smem + static_cast<size_t>(s) * stage_bytes;
        if (p.ldw == p.K) {
          bulk_g2s(dst, p.w + row0 * p.K, static_cast<uint32_t>(stage_bytes), &full[s], pol);
        } else {
#pragma unroll
          for (int r = 0; r < R; ++r)
            bulk_g2s(dst + r * p.K, p.w + (row0 + r) * p.ldw, static_cast<uint32_t>(p.K), &full[s], pol);
        }
      };
      // static weights: fill the ring before the grid-dependency wait
      const int n_pre = p.early_weights ? (n_my < p.stages ? n_my : p.stages) : 0;
      for (int j = 0; j < n_pre; ++j) issue(j);
      grid_dependency_wait();
      for (int j = n_pre; j < n_my; ++j) {
        const int s = j % p.stages;
        if (j >= p.stages) {
          if (!mbar_wait(&empty[s], ((j / p.stages) & 1) ^ 1, kSiteRowEmpty)) break;
        }
        issue(j);
      }
      grid_launch_dependents();
    }
    return;
  }
  // the activation and the output belong to the stream's previous work
  grid_dependency_wait();
  bool in_ok = true;
  // tagged words: the input carries this rank's last sequence number, the
  // output the one after it
  constexpr bool tagged = kTagged;
  const unsigned int tag_in = tagged ? gather_seq_now(p.gather) : 0u;
  const unsigned int tag_out = tag_after(tag_in);
  const bool tagged_in = tagged && p.gather.wait_input;
  bool tag_live = true;
  if (p.gather.wait_input && !tagged) {
    // the activation is a gathered output: every rank's slice must be here
    if (warp == 0) {
      const bool w_ok = gather_wait_input(p.gather, lane);
      if (lane == 0) window[0] = w_ok ? 1.0f : 0.0f;
    }
    named_bar_sync(1, T);
    in_ok = window[0] != 0.0f;
    named_bar_sync(1, T);
  }

  // ------------------------------------------------- consumers: prologue --
  // Quantise this thread's chunks of the activation (whole 128-groups are
  // shared by 8 consecutive lanes, so the group amax is a 3-step shuffle).
  const int n_chunks = p.K / 16;
  // (reduce +) add + RMSNorm: first the row's sum of squares (chunk sums, octet
  // sums per 128-group into shared memory, then one thread adds the groups in
  // order); x is the sum of p.norm.nsrc sources, see addn16
  float rstd = 0.0f;
  if (!kSwiglu && p.norm.norm) {
    float* gsum = window;                 // [K/128 + 1] until the main loop
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = tid + T * i;
      const bool valid = c < n_chunks;
      float sv[16];
      if (valid) {
        addn16(sv, p.x + 16 * c, p.norm.src_stride, p.norm.nsrc, p.norm.res + 16 * c);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) sv[e] = 0.0f;
      }
      const float gs = octet_sum(sumsq16(sv));
      if (valid && (c & 7) == 0) gsum[c >> 3] = gs;
      if (valid && blockIdx.x == 0 && p.norm.res_out) {
        uint4 a, b;
        pack_bf16x16(sv, a, b);
        uint4* op = reinterpret_cast<uint4*>(p.norm.res_out + 16 * c);
        op[0] = a;
        op[1] = b;
      }
    }
    named_bar_sync(1, T);
    if (tid == 0) {
      float a = 0.0f;
      for (int b = 0; b < p.K / 128; ++b) a = __fadd_rn(a, gsum[b]);
      gsum[p.K / 128] = rms_rstd(a, p.K, p.norm.eps);
    }
    named_bar_sync(1, T);
    rstd = gsum[p.K / 128];
    named_bar_sync(1, T);                 // the window is reused below
  }
  uint32_t xh[C][8];
  float sx_c[C];
  int blk[C];
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const int c = tid + T * i;
    const bool valid = c < n_chunks;
    float v[16];
    if (valid) {
      if constexpr (kSwiglu) {
        uint32_t gw[8], uw[8];
        if (tagged_in) {
          // word i of the row holds elements 2i, 2i + 1: gate at 8c, up at (K + 16c) / 2
          const uint64_t* gp = reinterpret_cast<const uint64_t*>(p.x) + 8 * c;
          const uint64_t* up = reinterpret_cast<const uint64_t*>(p.x) + p.K / 2 + 8 * c;
          uint64_t gv[8], uv[8];
          tagged_issue8(gp, gv);
          tagged_issue8(up, uv);
          tagged_finish8(gp, tag_in, gv, gw, tag_live);
          tagged_finish8(up, tag_in, uv, uw, tag_live);
        } else {
          const uint4* gp = reinterpret_cast<const uint4*>(p.x + 16 * c);
          const uint4* up = reinterpret_cast<const uint4*>(p.x + p.K + 16 * c);
          const uint4 g_a = gp[0], g_b = gp[1], u_a = up[0], u_b = up[1];
          gw[0] = g_a.x; gw[1] = g_a.y; gw[2] = g_a.z; gw[3] = g_a.w;
          gw[4] = g_b.x; gw[5] = g_b.y; gw[6] = g_b.z; gw[7] = g_b.w;
          uw[0] = u_a.x; uw[1] = u_a.y; uw[2] = u_a.z; uw[3] = u_a.w;
          uw[4] = u_b.x; uw[5] = u_b.y; uw[6] = u_b.z; uw[7] = u_b.w;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          v[2 * e] = silu_mul(bf16_lo(gw[e]), bf16_lo(uw[e]));
          v[2 * e + 1] = silu_mul(bf16_hi(gw[e]), bf16_hi(uw[e]));
        }
      } else {
        if (tagged_in) {
          const uint64_t* wp = reinterpret_cast<const uint64_t*>(p.x) + 8 * c;
          uint64_t wv[8];
          uint32_t xw[8];
          tagged_issue8(wp, wv);
          tagged_finish8(wp, tag_in, wv, xw, tag_live);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            v[2 * e] = bf16_lo(xw[e]);
            v[2 * e + 1] = bf16_hi(xw[e]);
          }
        } else if (p.norm.norm) {
          const uint4* wp = reinterpret_cast<const uint4*>(p.norm.w + 16 * c);
          float sv[16];
          addn16(sv, p.x + 16 * c, p.norm.src_stride, p.norm.nsrc, p.norm.res + 16 * c);
          norm16(v, sv, rstd, wp[0], wp[1]);
        } else {
          const uint4* xp = reinterpret_cast<const uint4*>(p.x + 16 * c);
          const uint4 a = xp[0], b = xp[1];
          const uint32_t xw[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            v[2 * e] = bf16_lo(xw[e]);
            v[2 * e + 1] = bf16_hi(xw[e]);
          }
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
    uint16_t q[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      q[e] = quant_pair(v[2 * e], v[2 * e + 1], sinv);
      xh[i][e] = e4m3x2_to_f16x2(q[e]);
    }
    sx_c[i] = sx;
    blk[i] = c >> 3;
    if (valid && blockIdx.x == 0) {
      if (p.xq_out) {
        uint4 packed;
        packed.x = q[0] | (static_cast<uint32_t>(q[1]) << 16);
        packed.y = q[2] | (static_cast<uint32_t>(q[3]) << 16);
        packed.z = q[4] | (static_cast<uint32_t>(q[5]) << 16);
        packed.w = q[6] | (static_cast<uint32_t>(q[7]) << 16);
        *reinterpret_cast<uint4*>(p.xq_out + 16 * c) = packed;
      }
      if (p.sx_out && (c & 7) == 0) p.sx_out[c >> 3] = sx;
    }
  }

  // ------------------------------------------------ consumers: main loop --
  const int row_begin = g0 * R;
  const int rows_my = n_my * R;
  float s_cur[C];
  int nb_cur = -1;
  bool ok = true;
  int win_buf = 0;
  bool store_wait = true;   // publishing: warp 0 waits for the ranks before its first store
  const int my_row_in_group = row_of_lane<R>(lane);
  const bool row_writer = (lane & ((32 / R) - 1)) == 0;

  for (int j = 0; j < n_my; ++j) {
    const int s = j % p.stages;
    if (ok) ok = mbar_wait(&full[s], (j / p.stages) & 1, kSiteRowFull);
    const int row0 = row_begin + j * R;
    const int nb = row0 >> 7;
    if (nb != nb_cur) {
      nb_cur = nb;
#pragma unroll
      for (int i = 0; i < C; ++i) {
        const int c = tid + T * i;
        s_cur[i] = (c < n_chunks) ? sx_c[i] * __ldg(p.ws + static_cast<int64_t>(nb) * p.ldws + blk[i]) : 0.0f;
      }
    }
    float acc[R];
    const uint8_t* stage = smem + static_cast<size_t>(s) * stage_bytes;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      acc[r] = 0.0f;
#pragma unroll
      for (int i = 0; i < C; ++i) {
        const int c = tid + T * i;
        if (c < n_chunks && ok) {
          const uint4 wv = *reinterpret_cast<const uint4*>(stage + r * p.K + 16 * c);
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
    if (done_rows % kRowWindow == 0 || j == n_my - 1) {
      named_bar_sync(1, T);
      if (warp == 0) {
        if (store_wait) {
          gather_wait_store(p.gather, lane);
          store_wait = false;
        }
        const int wrow0 = ((done_rows - 1) / kRowWindow) * kRowWindow;
        const int nrows = done_rows - wrow0;
        if constexpr (kTagged) {
          // rows come in pairs here (even row_begin, even row counts): the
          // even lane stores rows lane, lane + 1 as one tagged word
          float sum = 0.0f;
          if (lane < nrows)
            for (int w = 0; w < n_cwarps; ++w) sum += win[w * kRowWindow + lane];
          const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(sum));
          const uint32_t hi = __shfl_down_sync(0xffffffffu, lo, 1);
          if (lane < nrows && !(lane & 1))
            gather_store_pair(p.gather, 0, row_begin + wrow0 + lane, lo | (hi << 16), tag_out);
        } else if (lane < nrows) {
          float sum = 0.0f;
          for (int w = 0; w < n_cwarps; ++w) sum += win[w * kRowWindow + lane];
          const __nv_bfloat16 v = __float2bfloat16_rn(sum);
          if (gather_publishes(p.gather))
            gather_store(p.gather, 0, row_begin + wrow0 + lane, v);
          else
            p.out[row_begin + wrow0 + lane] = v;
        }
      }
      win_buf ^= 1;
    }
  }
  (void)rows_my;
  (void)in_ok;
  if (gather_publishes(p.gather)) {
    named_bar_sync(1, T);   // every output store of this CTA is issued
    if (tid == 0) gather_cta_done(p.gather, gridDim.x);
  }
}

}  // namespace fp8gq
