// Device-side building blocks shared by the fp8gq kernels (sm_100a):
// the activation group quant, the SwiGLU prologue, e4m3/f16 conversions,
// mbarriers and 1-D bulk (TMA) copies with bounded waits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>
#include <type_traits>
#include <utility>

namespace fp8gq {

constexpr int kGroup = 128;          // 1x128 activation groups, 128x128 weight blocks
constexpr float kE4m3Max = 448.0f;   // largest finite e4m3fn value
constexpr float kEps = 1e-10f;       // amax floor (kernels/fused_gemv_quant_tm.py:144)

// Error word written when a bounded wait gives up (read by fp8gq_device_error).
// Low 16 bits: site id; bit 31: set.  libfp8gq is one translation unit
// (fp8gq_api.cu), which is where this definition lands.
__device__ unsigned int g_device_error = 0;

enum ErrorSite : unsigned int {
  kSiteRowFull = 1,      // row kernel consumer waiting for a weight stage
  kSiteRowEmpty = 2,     // row kernel producer waiting for a free stage
  kSiteTmA = 3,          // tile kernel waits (A/B/accumulator/TMEM rings)
  kSiteTmB = 4,
  kSiteTmAcc = 5,
  kSiteTmTmem = 6,
  kSiteTmFixup = 7,      // tile kernel split-K partial-sum hand-off
  kSiteGather = 8,       // waiting for the peers' output slices of a gathered linear
  kSiteStackRing = 9,    // stack runner: a ring, accumulator or scale wait inside a CTA
  kSiteStackDep = 10,    // stack runner: waiting for every CTA to finish an earlier linear
};

__device__ __forceinline__ void record_error(unsigned int site) {
  atomicCAS(&g_device_error, 0u, 0x80000000u | site);
}

// ---------------------------------------------------------------------------
// timing for bounded waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every wait in these kernels is for work that completes in microseconds: of
// the same CTA or grid, or a peer GPU's kernel of the same step.  A wait for
// the peers' flags gives up after the peer limit (2 s by default); a wait for
// work inside the same kernel after twice that, so that when a peer is lost
// the peer wait is the one that gives up and reports it, and the waits queued
// behind it complete once it has.  The limit is a device variable so that a
// test can shorten it (fp8gq_set_wait_limit_ns) and make a wait run out on
// purpose; it is read only on the slow path of a wait, after its first polls
// failed.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ uint64_t peer_wait_limit_ns() {
  return *reinterpret_cast<volatile unsigned long long*>(&g_wait_limit_ns);
}
__device__ __forceinline__ uint64_t wait_limit_ns() { return 2 * peer_wait_limit_ns(); }

// ---------------------------------------------------------------------------
// mbarrier + 1-D bulk copy (TMA, no tensor map, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false (and the error
// word set) if that takes longer than the wait limit (wait_limit_ns).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u && global_ns() - t0 > wait_limit_ns()) {
      record_error(site);
      return false;
    }
  }
}

// mbar_wait by lane 0 only; the other lanes of the (converged) warp wait at
// __syncwarp, which also orders what lane 0 observed before their accesses.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, unsigned int site, int lane) {
  uint32_t ok = 1;
  if (lane == 0) ok = mbar_wait(bar, parity, site) ? 1u : 0u;
  __syncwarp();
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global to this CTA's shared memory; completion is counted on `bar`.  The
// weight stream is read once, so it is marked evict-first in L2.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar, uint64_t l2_policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(l2_policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Programmatic dependent launch.  A kernel launched with
// launch_with_pdl may start while the previous kernel in the stream is still
// running; it does its set-up, then waits here before it touches anything the
// previous kernel may write (activations, outputs, workspace).  Outside a
// programmatic launch the wait is a no-op.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next programmatically launched kernel in the stream be scheduled
// (it still waits for this grid to finish before reading our results).
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// activation quant (sglang formula, bit-exact with the oracle)
// ---------------------------------------------------------------------------

// Scale of a group from its max |value|: amax floored at 1e-10, IEEE division
// by 448 (kernels/fused_gemv_quant.py:40-41).
__device__ __forceinline__ float group_scale(float amax) {
  return __fdiv_rn(fmaxf(amax, kEps), kE4m3Max);
}

// Two fp32 values -> two e4m3 codes (v0 in the low byte): y = v * (1/sx)
// (IEEE multiply), clamp to +-448, round to nearest even
// (kernels/fused_gemv_quant.py:42-43).
__device__ __forceinline__ uint16_t quant_pair(float v0, float v1, float sinv) {
  float y0 = fminf(fmaxf(__fmul_rn(v0, sinv), -kE4m3Max), kE4m3Max);
  float y1 = fminf(fmaxf(__fmul_rn(v1, sinv), -kE4m3Max), kE4m3Max);
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(make_float2(y0, y1), __NV_SATFINITE, __NV_E4M3));
}

// Two e4m3 codes (low byte first) -> f16x2 (exact: every e4m3 value is an f16).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t two) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
  return static_cast<uint32_t>(h.x) | (static_cast<uint32_t>(h.y) << 16);
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// ---------------------------------------------------------------------------
// SwiGLU prologue: act = (g * sigmoid(g)) * u, sigmoid(g) = 1 / (1 + exp(-g))
// (kernels/fused_swiglu_quant_gemv.py:40-42).  exp is evaluated by the
// Cody-Waite reduction and the degree-5 minimax polynomial published in the
// Cephes library (S. L. Moshier, expf.c), one rounded fp32 operation per
// step and no fused multiply-add, so the CPU oracle evaluates the identical
// sequence and the quantised bytes agree bit for bit.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float exp_cw(float x) {
  const float kLog2e = 1.44269504088896341f;
  const float kC1 = 0.693359375f;
  const float kC2 = -2.12194440e-4f;
  // Branch-free: the polynomial runs on x clamped to [-88, 88] (inputs in
  // range are unchanged), and the out-of-range and NaN results are selected
  // at the end, so that the unrolled evaluations of a lane interleave.
  const float xc = fminf(fmaxf(x, -88.0f), 88.0f);
  const float n = rintf(__fmul_rn(xc, kLog2e));
  float r = __fsub_rn(xc, __fmul_rn(n, kC1));
  r = __fsub_rn(r, __fmul_rn(n, kC2));
  float p = 1.9875691500e-4f;
  p = __fadd_rn(__fmul_rn(p, r), 1.3981999507e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 8.3334519073e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 4.1665795894e-2f);
  p = __fadd_rn(__fmul_rn(p, r), 1.6666665459e-1f);
  p = __fadd_rn(__fmul_rn(p, r), 5.0000001201e-1f);
  p = __fmul_rn(p, __fmul_rn(r, r));
  p = __fadd_rn(p, r);
  p = __fadd_rn(p, 1.0f);
  const int ni = static_cast<int>(n);
  const int h1 = ni >> 1;                  // floor(n / 2)
  const int h2 = ni - h1;
  const float s1 = __int_as_float((h1 + 127) << 23);
  const float s2 = __int_as_float((h2 + 127) << 23);
  float out = __fmul_rn(__fmul_rn(p, s1), s2);
  out = x > 88.0f ? __int_as_float(0x7f800000) : out;
  out = x < -88.0f ? 0.0f : out;
  return x != x ? x : out;
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  const float e = exp_cw(-g);
  const float s = __frcp_rn(__fadd_rn(1.0f, e));
  return __fmul_rn(__fmul_rn(g, s), u);
}

// ---------------------------------------------------------------------------
// add + RMSNorm prologue (kernels/fused_rmsnorm.py:14-27): s = x + r in fp32,
// rstd = 1 / sqrt(mean(s^2) + eps), out = bf16((s * rstd) * w).  The sum of
// squares has a fixed order -- per 16-value chunk left to right, the 8
// chunks of a 128-group pairwise, the groups left to right -- and every step
// is one rounded fp32 operation, so the CPU oracle reproduces it bit for bit.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sumsq16(const float (&v)[16]) {
  float a = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) a = __fadd_rn(a, __fmul_rn(v[e], v[e]));
  return a;
}

// Sum over a lane octet (8 consecutive lanes): ((c0+c1)+(c2+c3))+((c4+c5)+(c6+c7)),
// the same bits on every lane of the octet.  All 32 lanes call it together.
__device__ __forceinline__ float octet_sum(float c) {
  c = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 1));
  c = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 2));
  c = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 4));
  return c;
}

constexpr int kMaxSumSources = 8;    // partial outputs summed by the reduce prologue (one per rank)

__device__ __forceinline__ float rms_rstd(float ssq, int K, float eps) {
  const float var = __fdiv_rn(ssq, static_cast<float>(K));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// 16 values s = x + r from two 16-byte words of bf16 each.
__device__ __forceinline__ void add16(float (&s)[16], uint4 xa, uint4 xb, uint4 ra, uint4 rb) {
  const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
  const uint32_t rw[8] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    s[2 * e] = __fadd_rn(bf16_lo(xw[e]), bf16_lo(rw[e]));
    s[2 * e + 1] = __fadd_rn(bf16_hi(xw[e]), bf16_hi(rw[e]));
  }
}

// 16 values s = ((x_0 + x_1) + ... + x_{n-1}) + r, added left to right in
// fp32: n >= 1 bf16 sources `stride` elements apart (the partial outputs of a
// K-sharded linear, one per rank, in rank order), then the residual.  With
// n == 1 it is add16's single addition.  L2-coherent loads: the sources may
// have been stored into this GPU's memory by other GPUs.
__device__ __forceinline__ void addn16(float (&s)[16], const __nv_bfloat16* x, int64_t stride, int n,
                                       const __nv_bfloat16* r) {
  const uint4* x0 = reinterpret_cast<const uint4*>(x);
  const uint4 a0 = __ldcg(x0), b0 = __ldcg(x0 + 1);
  const uint32_t w0[8] = {a0.x, a0.y, a0.z, a0.w, b0.x, b0.y, b0.z, b0.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    s[2 * e] = bf16_lo(w0[e]);
    s[2 * e + 1] = bf16_hi(w0[e]);
  }
#pragma unroll
  for (int i = 1; i < kMaxSumSources; ++i) {
    if (i < n) {
      const uint4* xi = reinterpret_cast<const uint4*>(x + i * stride);
      const uint4 a = __ldcg(xi), b = __ldcg(xi + 1);
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s[2 * e] = __fadd_rn(s[2 * e], bf16_lo(w[e]));
        s[2 * e + 1] = __fadd_rn(s[2 * e + 1], bf16_hi(w[e]));
      }
    }
  }
  const uint4* rp = reinterpret_cast<const uint4*>(r);
  const uint4 ra = __ldcg(rp), rb = __ldcg(rp + 1);
  const uint32_t rw[8] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    s[2 * e] = __fadd_rn(s[2 * e], bf16_lo(rw[e]));
    s[2 * e + 1] = __fadd_rn(s[2 * e + 1], bf16_hi(rw[e]));
  }
}

// Norm output bf16((s * rstd) * w) for 16 values (w: two 16-byte words of
// bf16), returned as the float values of the bf16 results.
__device__ __forceinline__ void norm16(float (&h)[16], const float (&s)[16], float rstd, uint4 wa, uint4 wb) {
  const uint32_t ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    h[2 * e] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(s[2 * e], rstd), bf16_lo(ww[e]))));
    h[2 * e + 1] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(s[2 * e + 1], rstd), bf16_hi(ww[e]))));
  }
}

// 16 bf16 values (round to nearest even) packed into two 16-byte words.
__device__ __forceinline__ void pack_bf16x16(const float (&s)[16], uint4& a, uint4& b) {
  uint32_t w[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(s[2 * e], s[2 * e + 1]);
    w[e] = *reinterpret_cast<const uint32_t*>(&h);
  }
  a = make_uint4(w[0], w[1], w[2], w[3]);
  b = make_uint4(w[4], w[5], w[6], w[7]);
}

// Parameters of the add + RMSNorm prologue (norm = 0: none).  The activation
// x may be the sum of nsrc sources (x, x + src_stride, ...), see addn16.
struct NormParams {
  const __nv_bfloat16* res;   // residual [M, ldr]
  const __nv_bfloat16* w;     // norm weight [K]
  __nv_bfloat16* res_out;     // sum + residual [M, ldro], written once (by CTA 0)
  int64_t ldr, ldro;
  float eps;
  int norm;
  int nsrc;                   // sources summed into x (0 or 1: x alone)
  int64_t src_stride;         // elements from one source to the next
};

// ---------------------------------------------------------------------------
// N-sharded output gather over peer memory (one process per GPU, NVLink)
// ---------------------------------------------------------------------------
constexpr int kMaxGatherRanks = 8;

// A kernel with world > 0 writes its output slice (columns col0 .. col0 + N)
// into the same columns of every rank's full output buffer -- plain stores
// through the peers' mapped pointers -- and its last CTA then raises this
// rank's flag on every rank to the rank's new sequence number.  A kernel with
// wait_input set reads its activation only after every rank's flag has
// reached this rank's sequence number, i.e. after every slice of the last
// gathered output has landed here.  All ranks run the same sequence of
// gathered kernels, so their sequence numbers advance together.
//
// Stores into a peer never overtake that peer: a publishing kernel stores
// into the ranks' buffers only once every rank's flag has reached this rank's
// sequence number, i.e. once every rank has finished its previous publishing
// kernel (with wait_input that is the input wait itself; without it the
// storing warps wait the same way before their first store).  So everything a
// rank queued before its previous publishing call -- readers of the buffer
// about to be overwritten included -- is complete before any rank writes into
// its buffers again.
//
// A K-sharded (row-parallel) linear uses the same stores for its partial
// output: out[r] points at this rank's slab in rank r's buffer of per-rank
// partials, col0 = 0.  A kernel with local_out set only waits (wait_input) and
// writes its own output locally, publishing nothing: the column-parallel
// linear that reduces those partials in its prologue.
//
// Tagged words (tagged = 1): the flags above cost a system-scope fence in the
// last CTA of every publishing kernel (it waits for every NVLink store of the
// kernel to be acknowledged) and a second round of peer stores after it.
// With tagged words each store carries its own proof of arrival instead: a
// 64-bit word holds two bf16 outputs (columns 2i, 2i + 1 of a row; low half
// first) and, in its high 32 bits, the sequence number of the kernel that
// wrote it, stored with one single-copy-atomic 64-bit store.  The buffers
// hold M x ldo / 2 words.  A kernel whose input is a tagged output
// (wait_input) polls the very words it reads until each carries the
// sequence number of this rank's last publishing kernel; no fence and no flag
// sits between a producer's stores and its consumer.  Write-after-read needs
// no wait either when the input is the last gathered output: every output
// word of the consumer depends on every input word, and each input word from
// rank q was written after q's kernel had read its own input -- the buffer
// the consumer is about to overwrite (with two buffers in turn).  A
// publishing kernel without wait_input instead waits, before its first
// store, until every rank's own flag slot flags[q][q] -- raised with a local
// store by q's last CTA, no fence -- shows that q has finished its previous
// publishing kernel.  Tagged kernels are single launches (M <= 16) whose
// input, when waited for, is the output of the last publishing kernel.
struct GatherParams {
  __nv_bfloat16* out[kMaxGatherRanks];   // rank r's full output [M, ldo], as mapped here (tagged: words)
  unsigned int* flags[kMaxGatherRanks];  // rank r's flags[world], as mapped here
  unsigned int* counter;                 // this rank: CTAs of the running kernel that are done
  unsigned int* seq;                     // this rank: sequence number of its last gathered kernel
  int64_t ldo;
  int col0;                              // first column of this rank's slice
  int world;                             // 0: no gather (plain local output)
  int rank;
  int wait_input;
  int local_out;                         // 1: output to the local `out` only, no flags raised
  int tagged;                            // 1: tagged words, see above
};

// Whether a kernel's output goes to every rank (and raises the flags).
__device__ __forceinline__ bool gather_publishes(const GatherParams& g) { return g.world > 0 && !g.local_out; }

__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Output element (m, n) of this rank's slice, to every rank.
__device__ __forceinline__ void gather_store(const GatherParams& g, int64_t m, int64_t n, __nv_bfloat16 v) {
  const int64_t off = m * g.ldo + g.col0 + n;
#pragma unroll 1
  for (int r = 0; r < g.world; ++r) g.out[r][off] = v;
}

// ---- tagged words ----------------------------------------------------------

// The sequence number after s (0 is skipped: a zero-filled buffer never
// carries a valid tag).
__device__ __forceinline__ unsigned int tag_after(unsigned int s) {
  const unsigned int t = s + 1u;
  return t ? t : 1u;
}

// This rank's last publishing sequence number; read after the grid-dependency
// wait (the previous publishing kernel's last CTA wrote it).  A publishing
// kernel tags its words with tag_after() of it; a waiting kernel expects it.
__device__ __forceinline__ unsigned int gather_seq_now(const GatherParams& g) {
  return *reinterpret_cast<volatile unsigned int*>(g.seq);
}

// Output columns n, n + 1 (n even) of token m of this rank's slice as one
// tagged word, to every rank.
__device__ __forceinline__ void gather_store_pair(const GatherParams& g, int64_t m, int64_t n, uint32_t pair,
                                                  unsigned int tag) {
  const int64_t w = (m * g.ldo + g.col0 + n) >> 1;
  const uint64_t word = static_cast<uint64_t>(pair) | (static_cast<uint64_t>(tag) << 32);
#pragma unroll 1
  for (int r = 0; r < g.world; ++r)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(reinterpret_cast<uint64_t*>(g.out[r]) + w), "l"(word)
                 : "memory");
}

// Tagged output element (m, n) held by this lane, with column n + 1 held by
// the next lane: the even lane stores the pair.  All 32 lanes call it
// together (the shuffle), with consecutive columns on consecutive lanes.
__device__ __forceinline__ void gather_store_tagged(const GatherParams& g, int64_t m, int64_t n, __nv_bfloat16 v,
                                                    unsigned int tag) {
  const uint32_t lo = __bfloat16_as_ushort(v);
  const uint32_t hi = __shfl_down_sync(0xffffffffu, lo, 1);
  if (!(n & 1)) gather_store_pair(g, m, n, lo | (hi << 16), tag);
}

// Eight tagged words (16 bf16 elements) at w, 16-byte aligned: issue the
// loads (relaxed, system scope: the words are written by other GPUs).
__device__ __forceinline__ void tagged_issue8(const uint64_t* w, uint64_t v[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                 : "=l"(v[2 * i]), "=l"(v[2 * i + 1])
                 : "l"(w + 2 * i)
                 : "memory");
}

// The issued words v of tagged_issue8(w): reload until each carries `tag`,
// then their bf16 pairs into xw.  `live` (per thread) turns false, with the
// error word set, once the peer limit has passed; later calls of a thread
// that gave up do not wait again, so a lost peer costs a kernel one limit.
__device__ __forceinline__ void tagged_finish8(const uint64_t* w, unsigned int tag, uint64_t v[8], uint32_t xw[8],
                                               bool& live) {
  auto all_tagged = [&]() {
    bool ok = true;
#pragma unroll
    for (int e = 0; e < 8; ++e) ok &= static_cast<unsigned int>(v[e] >> 32) == tag;
    return ok;
  };
  if (live && !all_tagged()) {
    const uint64_t t0 = global_ns();
    for (;;) {
      tagged_issue8(w, v);
      if (all_tagged()) break;
      if (global_ns() - t0 > peer_wait_limit_ns()) {
        record_error(kSiteGather);
        live = false;
        break;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) xw[e] = static_cast<uint32_t>(v[e]);
}

// One thread per CTA, after a barrier that follows every gather_store of the
// CTA: count the CTA (acq_rel at GPU scope: the barrier puts the CTA's stores
// before the release); the last one, having acquired every other CTA's count,
// publishes the slice to every rank with a system-scope release, which by
// cumulativity covers the stores of all CTAs.
__device__ __forceinline__ void gather_cta_done(const GatherParams& g, unsigned int ncta) {
  unsigned int old;
  asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(g.counter) : "memory");
  if (old == ncta - 1u && g.tagged) {
    // tagged words: the outputs carry their own sequence number; only the
    // local counters and this rank's own flag slot change (no fence)
    *g.counter = 0u;
    const unsigned int s = tag_after(*g.seq);
    *g.seq = s;
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(g.flags[g.rank] + g.rank), "r"(s) : "memory");
  } else if (old == ncta - 1u) {
    *g.counter = 0u;                     // ready for the next gathered kernel on this stream
    const unsigned int s = *g.seq + 1u;
    *g.seq = s;
    // one system-scope release fence, then plain (relaxed, system-scope) flag stores
    asm volatile("fence.acq_rel.sys;" ::: "memory");
#pragma unroll 1
    for (int r = 0; r < g.world; ++r)
      asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(g.flags[r] + g.rank), "r"(s) : "memory");
  }
}

// One warp (all 32 lanes), after grid_dependency_wait: wait (bounded) until
// every rank's slice of this rank's last gathered output has arrived -- lane r
// watches rank r's flag.  False on every lane (and the error word set) on
// timeout.
__device__ __forceinline__ bool gather_wait_input(const GatherParams& g, int lane) {
  const unsigned int s = *reinterpret_cast<volatile unsigned int*>(g.seq);
  bool ok = true;
  if (lane < g.world) {
    const unsigned int* flag = g.flags[g.rank] + lane;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0;; ++it) {
      if (static_cast<int>(ld_acquire_sys_u32(flag) - s) >= 0) break;
      if ((it & 255u) == 255u && global_ns() - t0 > peer_wait_limit_ns()) {
        record_error(kSiteGather);
        ok = false;
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok) != 0;
}

// One warp (all 32 lanes), before its first store of a publishing kernel's
// output: the stores may not overtake a rank still inside its previous
// publishing kernel.  A kernel with wait_input has made that wait already; for
// any other publishing kernel this is the same bounded wait.
__device__ __forceinline__ void gather_wait_store(const GatherParams& g, int lane) {
  if (!gather_publishes(g) || g.wait_input) return;
  if (!g.tagged) {
    gather_wait_input(g, lane);
    return;
  }
  // tagged: lane q watches rank q's own flag slot over NVLink until rank q
  // has finished this rank's previous publishing kernel
  const unsigned int s = gather_seq_now(g);
  bool ok = true;
  if (lane < g.world) {
    const unsigned int* flag = g.flags[lane] + lane;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0;; ++it) {
      if (static_cast<int>(ld_acquire_sys_u32(flag) - s) >= 0) break;
      if ((it & 255u) == 255u && global_ns() - t0 > peer_wait_limit_ns()) {
        record_error(kSiteGather);
        ok = false;
        break;
      }
    }
  }
  __syncwarp();
  (void)ok;
}

// ---------------------------------------------------------------------------
// Host: recorded launches.  A decode loop calls the same linears on the same
// buffers every step, so the per-call host work -- argument checks, routing,
// tensor-map encoding, grid choice, the parameter block -- can be done once.
// While a LaunchRecord is installed on the calling host thread (RecordScope),
// launch_with_pdl_cluster stores each launch (kernel, grid, block, shared
// memory, cluster size and the parameter bytes) instead of issuing it;
// launch_recorded issues them later on any stream.  A record is plain data,
// valid at any address (the runtime copies each parameter from the pointer it
// is given), so callers may copy it.
// ---------------------------------------------------------------------------
constexpr int kRecMaxLaunches = 3;    // group quant + up to two tile-kernel passes
constexpr int kRecMaxArgs = 12;
constexpr int kRecArgBytes = 1024;

struct RecordedLaunch {
  const void* fn;
  dim3 grid, block;
  size_t smem;
  int cluster_x;
  int nargs;
  uint16_t arg_off[kRecMaxArgs];
  uint16_t arg_size[kRecMaxArgs];
  unsigned char args[kRecArgBytes];
};

struct LaunchRecord {
  uint64_t magic;
  int device;
  int n;
  int overflow;
  int reserved;
  RecordedLaunch launch[kRecMaxLaunches];
};
constexpr uint64_t kRecMagic = 0x66703867714c5031ull;   // "fp8gqLP1"

inline LaunchRecord*& current_recorder() {
  static thread_local LaunchRecord* rec = nullptr;
  return rec;
}

// Installs `rec` as this thread's recorder for the scope's lifetime.
struct RecordScope {
  LaunchRecord* prev;
  explicit RecordScope(LaunchRecord* rec) : prev(current_recorder()) { current_recorder() = rec; }
  ~RecordScope() { current_recorder() = prev; }
  RecordScope(const RecordScope&) = delete;
  RecordScope& operator=(const RecordScope&) = delete;
};

template <typename... KArgs, typename... Args>
inline cudaError_t record_launch(LaunchRecord* rec, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 int cluster_x, Args&&... args) {
  static_assert(sizeof...(KArgs) == sizeof...(Args), "one value per kernel parameter");
  static_assert(sizeof...(KArgs) <= kRecMaxArgs, "too many kernel parameters to record");
  if (rec->n >= kRecMaxLaunches) {
    rec->overflow = 1;
    return cudaErrorInvalidValue;
  }
  RecordedLaunch& L = rec->launch[rec->n];
  L.fn = reinterpret_cast<const void*>(kernel);
  L.grid = grid;
  L.block = block;
  L.smem = smem;
  L.cluster_x = cluster_x;
  L.nargs = 0;
  size_t off = 0;
  bool fits = true;
  auto put = [&](const auto& v) {
    using T = std::decay_t<decltype(v)>;
    off = (off + alignof(T) - 1) / alignof(T) * alignof(T);
    if (off + sizeof(T) > static_cast<size_t>(kRecArgBytes)) {
      fits = false;
      return;
    }
    std::memcpy(L.args + off, &v, sizeof(T));
    L.arg_off[L.nargs] = static_cast<uint16_t>(off);
    L.arg_size[L.nargs] = static_cast<uint16_t>(sizeof(T));
    ++L.nargs;
    off += sizeof(T);
  };
  (put(static_cast<std::decay_t<KArgs>>(std::forward<Args>(args))), ...);
  if (!fits) {
    rec->overflow = 1;
    return cudaErrorInvalidValue;
  }
  ++rec->n;
  return cudaSuccess;
}

inline void pdl_config(cudaLaunchConfig_t& cfg, cudaLaunchAttribute (&attr)[2], dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, int cluster_x) {
  cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cluster_x > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
}

// Issues a record's launches on `stream`, in order.
inline cudaError_t launch_recorded(const LaunchRecord& rec, cudaStream_t stream) {
  for (int i = 0; i < rec.n; ++i) {
    const RecordedLaunch& L = rec.launch[i];
    void* argv[kRecMaxArgs];
    for (int a = 0; a < L.nargs; ++a) argv[a] = const_cast<unsigned char*>(L.args) + L.arg_off[a];
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    pdl_config(cfg, attr, L.grid, L.block, L.smem, stream, L.cluster_x);
    const cudaError_t e = cudaLaunchKernelExC(&cfg, L.fn, argv);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Host: launch with programmatic stream serialization (the kernel pairs it with
// grid_dependency_wait / grid_launch_dependents) and, for cluster_x > 1,
// thread-block clusters of cluster_x consecutive CTAs -- or, with a recorder
// installed on this thread, record the launch.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_with_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                           cudaStream_t stream, int cluster_x, Args&&... args) {
  if (LaunchRecord* rec = current_recorder())
    return record_launch(rec, kernel, grid, block, smem, cluster_x, std::forward<Args>(args)...);
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[2];
  pdl_config(cfg, attr, grid, block, smem, stream, cluster_x);
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_with_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                   cudaStream_t stream, Args&&... args) {
  return launch_with_pdl_cluster(kernel, grid, block, smem, stream, 1, std::forward<Args>(args)...);
}

}  // namespace fp8gq
