// C ABI of libfp8gq (declared in include/fp8gq.h): argument checks, kernel
// selection and launch.  No allocation happens here; the tile kernel's scratch
// is the caller's workspace.
#include <cuda_runtime.h>

#include <atomic>
#include <map>
#include <tuple>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "../../include/fp8gq.h"
#include "fp8gq_device.cuh"
#include "gemm_tm.cuh"
#include "gemv_row.cuh"
#include "quant_only.cuh"
#include "swiglu_writer.cuh"
#include "add_rmsnorm.cuh"
#include "stack.cuh"
#include "chain.cuh"

using namespace fp8gq;

namespace {

constexpr int kMaxDevices = 64;
constexpr uint64_t kMinWaitLimitNs = 1000000ull;        // 1 ms
constexpr uint64_t kMaxWaitLimitNs = 20000000000ull;    // 20 s

struct DeviceInfo {
  int sm_count = 0;
  int cc_major = 0;
  int max_smem_optin = 0;
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];
std::atomic<int> g_static_weights{0};
std::atomic<int> g_tm_options{0};   // FP8GQ_TM_* bits

// launch_tm's activation-feed mode for the option bits (at most one feed bit is set)
int tm_resident_mode() {
  const int f = g_tm_options.load(std::memory_order_relaxed);
  return (f & FP8GQ_TM_STREAM_ACTIVATIONS) ? 0 : (f & FP8GQ_TM_PREQUANT_ACTIVATIONS) ? 2
         : (f & FP8GQ_TM_RESIDENT_ACTIVATIONS) ? 3 : 1;
}
int tm_cluster_mode() { return (g_tm_options.load(std::memory_order_relaxed) & FP8GQ_TM_WORKSPACE_SPLITK) ? 0 : 1; }

int device_info(DeviceInfo* out, int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FP8GQ_ERR_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.sm_count == 0) {
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess) {
      d.sm_count = 0;
      return FP8GQ_ERR_DEVICE;
    }
  }
  if (d.cc_major != 10) return FP8GQ_ERR_DEVICE;
  *out = d;
  if (dev_out) *dev_out = dev;
  return FP8GQ_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(const void* x, const void* w, const float* ws, const void* out, int M, int N, int K,
                 int64_t ldw, int64_t ldws, int64_t ldo) {
  if (!x || !w || !ws || !out) return FP8GQ_ERR_NULL_POINTER;
  if (M < 1 || N <= 0 || K <= 0 || (N % kGroup) != 0 || (K % kGroup) != 0) return FP8GQ_ERR_SHAPE;
  if (ldw < K || ldws < K / kGroup || ldo < N) return FP8GQ_ERR_STRIDE;
  if (!aligned16(x) || !aligned16(w) || (ldw % 16) != 0) return FP8GQ_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(ws) & 3u) != 0 || (reinterpret_cast<uintptr_t>(out) & 1u) != 0)
    return FP8GQ_ERR_ALIGNMENT;
  return FP8GQ_OK;
}

// FP8GQ_ERR_LAUNCH for a failed CUDA call; with FP8GQ_DEBUG set in the
// environment the CUDA error is also printed to stderr.
int cuda_fail(cudaError_t e, const char* what) {
  static const bool debug = std::getenv("FP8GQ_DEBUG") != nullptr;
  if (debug) std::fprintf(stderr, "fp8gq: %s: %s\n", what, cudaGetErrorString(e));
  return FP8GQ_ERR_LAUNCH;
}

inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? FP8GQ_OK : FP8GQ_ERR_LAUNCH;
}

// ----------------------------------------------------------------- row --
using RowKernel = void (*)(const RowParams);

template <int C, int R, bool S, bool T>
RowKernel row_fn() {
  return gemv_row_kernel<C, R, S, T>;
}

constexpr int kRowCs[] = {1, 2, 3, 4, 6, 8};
constexpr int kRowRs[] = {1, 2, 4};

// S: SwiGLU input; T: tagged-word gather
template <bool S, bool T = false>
RowKernel row_lookup(int ci, int ri) {
  static const RowKernel table[6][3] = {
      {row_fn<1, 1, S, T>(), row_fn<1, 2, S, T>(), row_fn<1, 4, S, T>()},
      {row_fn<2, 1, S, T>(), row_fn<2, 2, S, T>(), row_fn<2, 4, S, T>()},
      {row_fn<3, 1, S, T>(), row_fn<3, 2, S, T>(), row_fn<3, 4, S, T>()},
      {row_fn<4, 1, S, T>(), row_fn<4, 2, S, T>(), row_fn<4, 4, S, T>()},
      {row_fn<6, 1, S, T>(), row_fn<6, 2, S, T>(), row_fn<6, 4, S, T>()},
      {row_fn<8, 1, S, T>(), row_fn<8, 2, S, T>(), row_fn<8, 4, S, T>()},
  };
  return table[ci][ri];
}

constexpr int kRowMaxK = 8 * 384 * 16;      // C = 8 chunks of 16 per thread, T <= 384
// M == 1 routing: the row kernel (CUDA cores, no split-K) wins on small
// weights, where the tile kernel's fixed prologue and split-K hand-off cost
// more than they save; the tile kernel wins above this many weight bytes
// (measured on B200 with the Qwen3-8B decode shapes: 16.8 MB row, 25.2 MB tile).
constexpr int64_t kRowPreferBytes = 20ll << 20;

bool m1_uses_row(int N, int K) { return K <= kRowMaxK && static_cast<int64_t>(N) * K <= kRowPreferBytes; }
constexpr int kRowRingBytes = 96 * 1024;    // per CTA; two CTAs per SM

// Resident CTAs per SM of a row-kernel configuration (occupancy query,
// cached per kernel, block size and shared memory).
int row_ctas_per_sm(RowKernel fn, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int, size_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, reinterpret_cast<const void*>(fn), threads, smem);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem) != cudaSuccess) n = 0;
  cudaGetLastError();
  cache.emplace(key, n);
  return n;
}

int launch_row(bool swiglu, const void* x, const void* w, int64_t ldw, const float* ws, int64_t ldws,
               void* out, int N, int K, uint8_t* xq_out, float* sx_out, cudaStream_t stream,
               const GatherParams* gather = nullptr, const NormParams* norm = nullptr) {
  DeviceInfo di;
  int dev = 0;
  int st = device_info(&di, &dev);
  if (st != FP8GQ_OK) return st;
  if (K > kRowMaxK) return FP8GQ_ERR_UNSUPPORTED;
  const int n_chunks = K / 16;
  const int c_need = (n_chunks + 383) / 384;
  // rows per ring stage: the most (4, 2 or 1) whose stage is at most 16 KB
  // (fewer rows per stage cost more per byte than their better balance over
  // the CTAs saves: measured on B200, o_proj 4096 x 4096 takes 6.8 us with
  // 4-row stages and 7.5 us with 2-row stages)
  int ri = 2;
  while (ri > 0 && kRowRs[ri] * K > 16384) --ri;
  const int R = kRowRs[ri];
  const int stage_bytes = R * K;
  int stages = kRowRingBytes / stage_bytes;
  if (stages > 16) stages = 16;
  if (stages < 2) stages = 2;
  // Chunks per thread C (and T = the consumer threads that split K): the
  // fewest that cover K, unless that CTA does not fit twice on an SM (many
  // threads x many registers, e.g. K = 12288 at C = 2: 416 threads x 85
  // registers) and a larger C with fewer threads does -- two CTAs per SM
  // stream faster, and a grid of more CTAs than are resident would run a
  // second wave.
  int ci = 0;
  while (kRowCs[ci] < c_need) ++ci;
  int T = 0, per_sm = 0;
  size_t smem = 0;
  RowKernel fn = nullptr;
  for (int cj = ci; cj < 6; ++cj) {
    const int Cj = kRowCs[cj];
    const int Tj = ((n_chunks + Cj - 1) / Cj + 31) / 32 * 32;
    const size_t sj = row_smem_bytes(stages, stage_bytes, Tj / 32);
    if (sj > static_cast<size_t>(di.max_smem_optin)) continue;
    const bool tg = gather && gather->world > 0 && gather->tagged;
    RowKernel fj = swiglu ? (tg ? row_lookup<true, true>(cj, ri) : row_lookup<true>(cj, ri))
                          : (tg ? row_lookup<false, true>(cj, ri) : row_lookup<false>(cj, ri));
    if (ensure_max_smem(reinterpret_cast<const void*>(fj), di.max_smem_optin) != cudaSuccess) return FP8GQ_ERR_LAUNCH;
    const int pj = row_ctas_per_sm(fj, Tj + 32, sj);
    if (pj < 1) continue;
    if (fn == nullptr || pj > per_sm) {
      T = Tj;
      smem = sj;
      fn = fj;
      per_sm = pj;
    }
    if (pj >= 2) break;
  }
  if (fn == nullptr) return FP8GQ_ERR_UNSUPPORTED;

  RowParams p;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.w = static_cast<const uint8_t*>(w);
  p.ldw = ldw;
  p.ws = ws;
  p.ldws = ldws;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.N = N;
  p.K = K;
  p.n_groups = N / R;
  p.stages = stages;
  p.xq_out = xq_out;
  p.sx_out = sx_out;
  p.gather = gather ? *gather : GatherParams{};
  p.norm = norm ? *norm : NormParams{};
  p.early_weights = g_static_weights.load(std::memory_order_relaxed);
  // at most two CTAs per SM, and never more than are resident at once
  int grid = (per_sm < 2 ? per_sm : 2) * di.sm_count;
  // tagged words with one row per group: the CTAs take rows in pairs
  const int units = (R == 1 && gather && gather->tagged) ? p.n_groups / 2 : p.n_groups;
  if (grid > units) grid = units;
  if (launch_with_pdl(fn, dim3(grid), dim3(T + 32), smem, stream, p) != cudaSuccess) return FP8GQ_ERR_LAUNCH;
  return launch_status();
}

int launch_quant(bool swiglu, const void* x, int64_t ldx, int M, int K, uint8_t* xq, float* sx,
                 cudaStream_t stream) {
  DeviceInfo di;
  int st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  if (launch_group_quant(swiglu, static_cast<const __nv_bfloat16*>(x), ldx, M, K, xq, sx, stream) != cudaSuccess)
    return FP8GQ_ERR_LAUNCH;
  return launch_status();
}

int launch_swiglu_writer(bool quant, const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out,
                         int64_t ldo, float* scale, int M, int I, cudaStream_t stream) {
  DeviceInfo di;
  int st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  const int64_t groups = static_cast<int64_t>(M) * (I / kGroup);
  int64_t blocks = (groups + 15) / 16;
  const int64_t cap = static_cast<int64_t>(di.sm_count) * 8;
  if (blocks > cap) blocks = cap;
  auto g = static_cast<const __nv_bfloat16*>(gate);
  auto u = static_cast<const __nv_bfloat16*>(up);
  cudaError_t e = quant ? launch_with_pdl(swiglu_writer_kernel<true>, dim3(static_cast<unsigned>(blocks)), dim3(256),
                                          0, stream, g, ldg, u, ldu, out, ldo, scale, M, I)
                        : launch_with_pdl(swiglu_writer_kernel<false>, dim3(static_cast<unsigned>(blocks)), dim3(256),
                                          0, stream, g, ldg, u, ldu, out, ldo, scale, M, I);
  if (e != cudaSuccess) return FP8GQ_ERR_LAUNCH;
  return launch_status();
}

int check_swiglu_writer(const void* gate, int64_t ldg, const void* up, int64_t ldu, const void* out, int64_t ldo,
                        int M, int I, int out_bytes) {
  if (!gate || !up || !out) return FP8GQ_ERR_NULL_POINTER;
  if (M < 1 || I <= 0 || I % kGroup) return FP8GQ_ERR_SHAPE;
  if (ldg < I || ldu < I || ldo < I) return FP8GQ_ERR_STRIDE;
  if ((reinterpret_cast<uintptr_t>(gate) & 15u) || (reinterpret_cast<uintptr_t>(up) & 15u) || (ldg % 8) ||
      (ldu % 8) || (reinterpret_cast<uintptr_t>(out) & (out_bytes == 2 ? 15u : 7u)) ||
      ((ldo * out_bytes) % (out_bytes == 2 ? 16 : 8)))
    return FP8GQ_ERR_ALIGNMENT;
  return FP8GQ_OK;
}

// Waits (bounded) until every rank's slice of this rank's last gathered
// output has arrived; one thread.
__global__ void gather_wait_kernel(const GatherParams g) {
  grid_dependency_wait();
  gather_wait_input(g, threadIdx.x & 31);
  grid_launch_dependents();
}

int to_gather_params(const fp8gq_gather* gather, GatherParams* g) {
  if (!gather || !gather->counter || !gather->seq) return FP8GQ_ERR_NULL_POINTER;
  if (gather->world < 1 || gather->world > FP8GQ_MAX_GATHER_RANKS || gather->rank < 0 ||
      gather->rank >= gather->world || gather->col0 < 0 || gather->ldo < 1)
    return FP8GQ_ERR_SHAPE;
  *g = GatherParams{};
  for (int r = 0; r < gather->world; ++r) {
    if (!gather->out[r] || !gather->flags[r]) return FP8GQ_ERR_NULL_POINTER;
    if ((reinterpret_cast<uintptr_t>(gather->out[r]) & 1u) || (reinterpret_cast<uintptr_t>(gather->flags[r]) & 3u))
      return FP8GQ_ERR_ALIGNMENT;
    g->out[r] = static_cast<__nv_bfloat16*>(gather->out[r]);
    g->flags[r] = gather->flags[r];
  }
  g->counter = gather->counter;
  g->seq = gather->seq;
  g->ldo = gather->ldo;
  g->col0 = gather->col0;
  g->world = gather->world;
  g->rank = gather->rank;
  g->wait_input = gather->wait_input ? 1 : 0;
  g->local_out = gather->local_out ? 1 : 0;
  g->tagged = gather->tagged ? 1 : 0;
  if (g->tagged) {
    // words of two columns: even col0 and ldo (16-byte rows), aligned buffers
    if (g->local_out) return FP8GQ_ERR_UNSUPPORTED;
    if ((gather->ldo % 8) || (gather->col0 % 2)) return FP8GQ_ERR_ALIGNMENT;
    for (int r = 0; r < gather->world; ++r)
      if (reinterpret_cast<uintptr_t>(gather->out[r]) & 15u) return FP8GQ_ERR_ALIGNMENT;
  }
  return FP8GQ_OK;
}

// This rank's own output slice (for the shape checks and the plain-output
// argument): element col0 of its full output, or its word for tagged words.
void* own_slice(const fp8gq_gather* gather) {
  if (gather->tagged) return static_cast<uint64_t*>(gather->out[gather->rank]) + gather->col0 / 2;
  return static_cast<__nv_bfloat16*>(gather->out[gather->rank]) + gather->col0;
}

// A tagged call: one launch (M <= 16); a waited-for input is read as words
// (16-byte aligned rows of ld / 2 words).
int check_tagged(const fp8gq_gather* gather, const void* x, int64_t ldx, int M) {
  if (!gather->tagged) return FP8GQ_OK;
  if (M > 16) return FP8GQ_ERR_UNSUPPORTED;
  if (gather->wait_input && ((reinterpret_cast<uintptr_t>(x) & 15u) || (ldx % 8))) return FP8GQ_ERR_ALIGNMENT;
  return FP8GQ_OK;
}

// Tagged words -> bf16: each thread polls 8 words (16 columns of a row) of
// this rank's full output until they carry its last sequence number.
__global__ void gather_decode_kernel(const GatherParams g, __nv_bfloat16* out, int64_t ldo, int M, int N) {
  grid_dependency_wait();
  const unsigned int tag = gather_seq_now(g);
  const uint64_t* words = reinterpret_cast<const uint64_t*>(g.out[g.rank]);
  const int per_row = N / 16;
  const int64_t total = static_cast<int64_t>(M) * per_row;
  bool live = true;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / per_row;
    const int64_t c = i - m * per_row;
    const uint64_t* w = words + ((m * g.ldo) >> 1) + 8 * c;
    uint64_t v[8];
    uint32_t xw[8];
    tagged_issue8(w, v);
    tagged_finish8(w, tag, v, xw, live);
    uint4* o = reinterpret_cast<uint4*>(out + m * ldo + 16 * c);
    o[0] = make_uint4(xw[0], xw[1], xw[2], xw[3]);
    o[1] = make_uint4(xw[4], xw[5], xw[6], xw[7]);
  }
  grid_launch_dependents();
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange, resolved through the runtime (no -lcuda at link time).
AddressRangeFn address_range_fn() {
  static std::once_flag once;
  static AddressRangeFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(ptr);
  });
  return fn;
}

}  // namespace

extern "C" {

int fp8gq_version(void) { return FP8GQ_VERSION; }

const char* fp8gq_status_string(int status) {
  switch (status) {
    case FP8GQ_OK: return "ok";
    case FP8GQ_ERR_NULL_POINTER: return "a required pointer is NULL";
    case FP8GQ_ERR_SHAPE: return "bad shape: need M >= 1 and K, N positive multiples of 128";
    case FP8GQ_ERR_ALIGNMENT: return "misaligned operand: x, w and gu need 16-byte alignment and 16-byte row strides";
    case FP8GQ_ERR_STRIDE: return "a row stride is smaller than its row";
    case FP8GQ_ERR_WORKSPACE: return "workspace missing or too small (see fp8gq_workspace_bytes)";
    case FP8GQ_ERR_DEVICE: return "current CUDA device is not compute capability 10.x (B200, sm_100a)";
    case FP8GQ_ERR_LAUNCH: return "CUDA kernel launch failed";
    case FP8GQ_ERR_UNSUPPORTED: return "shape not supported by the selected kernel";
    case FP8GQ_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait gave up (fp8gq_device_error has the site)";
    case FP8GQ_ERR_SCRATCH_LIMIT:
      return "shape needs more split-K scratch than the 8 MiB device buffer of fp8gq_gemv_quant_tm_noalloc";
    default: return "unknown fp8gq status";
  }
}

int fp8gq_gemv_quant_row(const void* x, const void* w, int64_t ldw, const float* ws, int64_t ldws,
                         void* out, int N, int K, uint8_t* xq_out, float* sx_out,
                         fp8gq_stream_t stream) {
  int st = check_common(x, w, ws, out, 1, N, K, ldw, ldws, N);
  if (st != FP8GQ_OK) return st;
  return launch_row(false, x, w, ldw, ws, ldws, out, N, K, xq_out, sx_out,
                    static_cast<cudaStream_t>(stream));
}

size_t fp8gq_workspace_bytes(int M, int N, int K) {
  if (M < 1 || N <= 0 || K <= 0 || N % kGroup || K % kGroup) return 0;
  if (M == 1 && m1_uses_row(N, K)) return 0;
  return tm_workspace_bytes(M, N, K);
}

int fp8gq_gemv_quant_tm(const void* x, int64_t ldx, const void* w, int64_t ldw, const float* ws,
                        int64_t ldws, void* out, int64_t ldo, int M, int N, int K, uint8_t* xq_out,
                        float* sx_out, void* workspace, size_t workspace_bytes,
                        fp8gq_stream_t stream) {
  int st = check_common(x, w, ws, out, M, N, K, ldw, ldws, ldo);
  if (st != FP8GQ_OK) return st;
  if (ldx < K || (ldx % 8) != 0) return ldx < K ? FP8GQ_ERR_STRIDE : FP8GQ_ERR_ALIGNMENT;
  DeviceInfo di;
  st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  return launch_tm(false, x, ldx, w, ldw, ws, ldws, out, ldo, M, N, K, xq_out, sx_out, workspace,
                   workspace_bytes, di.sm_count, di.max_smem_optin, static_cast<cudaStream_t>(stream),
                   g_static_weights.load(std::memory_order_relaxed), 0, tm_resident_mode(),
                   tm_cluster_mode());
}

int fp8gq_fused_gemv_quant(const void* x, int64_t ldx, const void* w, int64_t ldw, const float* ws,
                           int64_t ldws, void* out, int64_t ldo, int M, int N, int K, uint8_t* xq_out,
                           float* sx_out, void* workspace, size_t workspace_bytes,
                           fp8gq_stream_t stream) {
  if (M == 1 && m1_uses_row(N, K)) {
    int st = check_common(x, w, ws, out, M, N, K, ldw, ldws, ldo);
    if (st != FP8GQ_OK) return st;
    return launch_row(false, x, w, ldw, ws, ldws, out, N, K, xq_out, sx_out,
                      static_cast<cudaStream_t>(stream));
  }
  return fp8gq_gemv_quant_tm(x, ldx, w, ldw, ws, ldws, out, ldo, M, N, K, xq_out, sx_out, workspace,
                             workspace_bytes, stream);
}

int fp8gq_fused_swiglu_q_gemm(const void* gu, int64_t ldgu, const void* w, int64_t ldw,
                              const float* ws, int64_t ldws, void* out, int64_t ldo, int M, int N,
                              int I, uint8_t* xq_out, float* sx_out, void* workspace,
                              size_t workspace_bytes, fp8gq_stream_t stream) {
  int st = check_common(gu, w, ws, out, M, N, I, ldw, ldws, ldo);
  if (st != FP8GQ_OK) return st;
  if (ldgu < 2 * static_cast<int64_t>(I)) return FP8GQ_ERR_STRIDE;
  if (ldgu % 8) return FP8GQ_ERR_ALIGNMENT;
  if (M == 1 && m1_uses_row(N, I))
    return launch_row(true, gu, w, ldw, ws, ldws, out, N, I, xq_out, sx_out,
                      static_cast<cudaStream_t>(stream));
  DeviceInfo di;
  st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  return launch_tm(true, gu, ldgu, w, ldw, ws, ldws, out, ldo, M, N, I, xq_out, sx_out, workspace,
                   workspace_bytes, di.sm_count, di.max_smem_optin, static_cast<cudaStream_t>(stream),
                   g_static_weights.load(std::memory_order_relaxed), 0, tm_resident_mode(),
                   tm_cluster_mode());
}

int fp8gq_group_quant(const void* x, int64_t ldx, int M, int K, uint8_t* xq, float* sx,
                      fp8gq_stream_t stream) {
  if (!x || !xq || !sx) return FP8GQ_ERR_NULL_POINTER;
  if (M < 1 || K <= 0 || K % kGroup) return FP8GQ_ERR_SHAPE;
  if (ldx < K) return FP8GQ_ERR_STRIDE;
  if ((reinterpret_cast<uintptr_t>(x) & 7u) || (ldx % 4) || (reinterpret_cast<uintptr_t>(xq) & 3u) ||
      (reinterpret_cast<uintptr_t>(sx) & 3u))
    return FP8GQ_ERR_ALIGNMENT;
  return launch_quant(false, x, ldx, M, K, xq, sx, static_cast<cudaStream_t>(stream));
}

int fp8gq_swiglu_group_quant(const void* gu, int64_t ldgu, int M, int I, uint8_t* xq, float* sx,
                             fp8gq_stream_t stream) {
  if (!gu || !xq || !sx) return FP8GQ_ERR_NULL_POINTER;
  if (M < 1 || I <= 0 || I % kGroup) return FP8GQ_ERR_SHAPE;
  if (ldgu < 2 * static_cast<int64_t>(I)) return FP8GQ_ERR_STRIDE;
  if ((reinterpret_cast<uintptr_t>(gu) & 7u) || (ldgu % 4) || (reinterpret_cast<uintptr_t>(xq) & 3u) ||
      (reinterpret_cast<uintptr_t>(sx) & 3u))
    return FP8GQ_ERR_ALIGNMENT;
  return launch_quant(true, gu, ldgu, M, I, xq, sx, static_cast<cudaStream_t>(stream));
}

int fp8gq_add_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, const void* norm_w,
                      float eps, void* out, int64_t ldo, void* residual_out, int64_t ldro, int M, int K,
                      fp8gq_stream_t stream) {
  if (!x || !residual || !norm_w || !out) return FP8GQ_ERR_NULL_POINTER;
  if (M < 1 || K <= 0 || K % kGroup) return FP8GQ_ERR_SHAPE;
  if (ldx < K || ldr < K || ldo < K || (residual_out && ldro < K)) return FP8GQ_ERR_STRIDE;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(residual) |
                        reinterpret_cast<uintptr_t>(norm_w) | reinterpret_cast<uintptr_t>(out) |
                        reinterpret_cast<uintptr_t>(residual_out);
  if ((mis & 15u) || (ldx % 8) || (ldr % 8) || (ldo % 8) || (residual_out && (ldro % 8))) return FP8GQ_ERR_ALIGNMENT;
  DeviceInfo di;
  int st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  const size_t smem = static_cast<size_t>(K / kGroup + 1) * sizeof(float);
  if (smem > static_cast<size_t>(di.max_smem_optin)) return FP8GQ_ERR_UNSUPPORTED;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(add_rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
          cudaSuccess)
    return FP8GQ_ERR_LAUNCH;
  if (launch_with_pdl(add_rmsnorm_kernel, dim3(M), dim3(kNormThreads), smem, static_cast<cudaStream_t>(stream),
                      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(residual), ldr,
                      static_cast<const __nv_bfloat16*>(norm_w), eps, static_cast<__nv_bfloat16*>(out), ldo,
                      static_cast<__nv_bfloat16*>(residual_out), ldro, K) != cudaSuccess)
    return FP8GQ_ERR_LAUNCH;
  return launch_status();
}

int fp8gq_fused_reduce_add_rmsnorm_gemv_quant(const void* x, int nsrc, int64_t src_stride, int64_t ldx,
                                              const void* residual, int64_t ldr, const void* norm_w, float eps,
                                              const void* w, int64_t ldw, const float* ws, int64_t ldws, void* out,
                                              int64_t ldo, void* residual_out, int64_t ldro, int M, int N, int K,
                                              uint8_t* xq_out, float* sx_out, const fp8gq_gather* wait,
                                              void* workspace, size_t workspace_bytes, fp8gq_stream_t stream) {
  int st = check_common(x, w, ws, out, M, N, K, ldw, ldws, ldo);
  if (st != FP8GQ_OK) return st;
  if (!residual || !norm_w) return FP8GQ_ERR_NULL_POINTER;
  if (nsrc < 1 || nsrc > kMaxSumSources) return FP8GQ_ERR_SHAPE;
  if (ldx < K || ldr < K || (residual_out && ldro < K)) return FP8GQ_ERR_STRIDE;
  // the sources must not overlap one another's rows
  if (nsrc > 1 && src_stride < static_cast<int64_t>(M - 1) * ldx + K) return FP8GQ_ERR_STRIDE;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(residual) | reinterpret_cast<uintptr_t>(norm_w) |
                        reinterpret_cast<uintptr_t>(residual_out);
  if ((mis & 15u) || (ldx % 8) || (ldr % 8) || (residual_out && (ldro % 8)) || (nsrc > 1 && src_stride % 8))
    return FP8GQ_ERR_ALIGNMENT;
  if (residual_out) {
    // CTA 0 writes residual_out while other CTAs still read the residual and
    // the sources
    auto span = [](const void* p, int64_t elems) {
      const uintptr_t b = reinterpret_cast<uintptr_t>(p);
      return std::make_pair(b, b + static_cast<uintptr_t>(elems * 2));
    };
    const auto o = span(residual_out, static_cast<int64_t>(M - 1) * ldro + K);
    const auto r = span(residual, static_cast<int64_t>(M - 1) * ldr + K);
    const auto xs = span(x, static_cast<int64_t>(nsrc - 1) * src_stride + static_cast<int64_t>(M - 1) * ldx + K);
    if ((r.first < o.second && o.first < r.second) || (xs.first < o.second && o.first < xs.second))
      return FP8GQ_ERR_UNSUPPORTED;
  }
  GatherParams g{};
  if (wait) {
    // only the input wait: flags, seq, world and rank of the descriptor
    if (wait->tagged) return FP8GQ_ERR_UNSUPPORTED;   // the norm prologue reads bf16 sources
    if (!wait->seq) return FP8GQ_ERR_NULL_POINTER;
    if (wait->world < 2 || wait->world > FP8GQ_MAX_GATHER_RANKS || wait->rank < 0 || wait->rank >= wait->world)
      return FP8GQ_ERR_SHAPE;
    for (int q = 0; q < wait->world; ++q) {
      if (!wait->flags[q]) return FP8GQ_ERR_NULL_POINTER;
      if (reinterpret_cast<uintptr_t>(wait->flags[q]) & 3u) return FP8GQ_ERR_ALIGNMENT;
      g.flags[q] = wait->flags[q];
    }
    g.seq = wait->seq;
    g.world = wait->world;
    g.rank = wait->rank;
    g.wait_input = 1;
    g.local_out = 1;
  }
  NormParams nrm{};
  nrm.res = static_cast<const __nv_bfloat16*>(residual);
  nrm.w = static_cast<const __nv_bfloat16*>(norm_w);
  nrm.res_out = static_cast<__nv_bfloat16*>(residual_out);
  nrm.ldr = ldr;
  nrm.ldro = ldro;
  nrm.eps = eps;
  nrm.norm = 1;
  nrm.nsrc = nsrc;
  nrm.src_stride = src_stride;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const GatherParams* gp = wait ? &g : nullptr;
  if (M == 1 && m1_uses_row(N, K)) return launch_row(false, x, w, ldw, ws, ldws, out, N, K, xq_out, sx_out, s, gp, &nrm);
  DeviceInfo di;
  st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  return launch_tm(false, x, ldx, w, ldw, ws, ldws, out, ldo, M, N, K, xq_out, sx_out, workspace, workspace_bytes,
                   di.sm_count, di.max_smem_optin, s, g_static_weights.load(std::memory_order_relaxed), 0,
                   1, tm_cluster_mode(), gp, &nrm);
}

int fp8gq_fused_add_rmsnorm_gemv_quant(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                                       const void* norm_w, float eps, const void* w, int64_t ldw, const float* ws,
                                       int64_t ldws, void* out, int64_t ldo, void* residual_out, int64_t ldro,
                                       int M, int N, int K, uint8_t* xq_out, float* sx_out, void* workspace,
                                       size_t workspace_bytes, fp8gq_stream_t stream) {
  return fp8gq_fused_reduce_add_rmsnorm_gemv_quant(x, 1, 0, ldx, residual, ldr, norm_w, eps, w, ldw, ws, ldws, out,
                                                   ldo, residual_out, ldro, M, N, K, xq_out, sx_out, nullptr,
                                                   workspace, workspace_bytes, stream);
}

int fp8gq_fused_gemv_quant_gather(const void* x, int64_t ldx, const void* w, int64_t ldw, const float* ws,
                                  int64_t ldws, int M, int N, int K, const fp8gq_gather* gather,
                                  void* workspace, size_t workspace_bytes, fp8gq_stream_t stream) {
  GatherParams g;
  int st = to_gather_params(gather, &g);
  if (st != FP8GQ_OK) return st;
  if (gather->ldo < static_cast<int64_t>(gather->col0) + N) return FP8GQ_ERR_STRIDE;
  // the rank's own output slice stands in for `out` in the shape checks
  void* own = own_slice(gather);
  st = check_common(x, w, ws, own, M, N, K, ldw, ldws, gather->ldo);
  if (st != FP8GQ_OK) return st;
  st = check_tagged(gather, x, ldx, M);
  if (st != FP8GQ_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 1 && m1_uses_row(N, K)) return launch_row(false, x, w, ldw, ws, ldws, own, N, K, nullptr, nullptr, s, &g);
  if (ldx < K || (ldx % 8) != 0) return ldx < K ? FP8GQ_ERR_STRIDE : FP8GQ_ERR_ALIGNMENT;
  DeviceInfo di;
  st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  return launch_tm(false, x, ldx, w, ldw, ws, ldws, own, gather->ldo, M, N, K, nullptr, nullptr, workspace,
                   workspace_bytes, di.sm_count, di.max_smem_optin, s, g_static_weights.load(std::memory_order_relaxed),
                   0, tm_resident_mode(), tm_cluster_mode(), &g);
}

int fp8gq_fused_swiglu_q_gemm_gather(const void* gu, int64_t ldgu, const void* w, int64_t ldw, const float* ws,
                                     int64_t ldws, int M, int N, int I, const fp8gq_gather* gather,
                                     void* workspace, size_t workspace_bytes, fp8gq_stream_t stream) {
  GatherParams g;
  int st = to_gather_params(gather, &g);
  if (st != FP8GQ_OK) return st;
  if (gather->ldo < static_cast<int64_t>(gather->col0) + N) return FP8GQ_ERR_STRIDE;
  void* own = own_slice(gather);
  st = check_common(gu, w, ws, own, M, N, I, ldw, ldws, gather->ldo);
  if (st != FP8GQ_OK) return st;
  st = check_tagged(gather, gu, ldgu, M);
  if (st != FP8GQ_OK) return st;
  if (ldgu < 2 * static_cast<int64_t>(I)) return FP8GQ_ERR_STRIDE;
  if (ldgu % 8) return FP8GQ_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 1 && m1_uses_row(N, I)) return launch_row(true, gu, w, ldw, ws, ldws, own, N, I, nullptr, nullptr, s, &g);
  DeviceInfo di;
  st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  return launch_tm(true, gu, ldgu, w, ldw, ws, ldws, own, gather->ldo, M, N, I, nullptr, nullptr, workspace,
                   workspace_bytes, di.sm_count, di.max_smem_optin, s, g_static_weights.load(std::memory_order_relaxed),
                   0, tm_resident_mode(), tm_cluster_mode(), &g);
}

int fp8gq_gather_wait(const fp8gq_gather* gather, fp8gq_stream_t stream) {
  GatherParams g;
  int st = to_gather_params(gather, &g);
  if (st != FP8GQ_OK) return st;
  if (g.tagged) return FP8GQ_ERR_UNSUPPORTED;   // tagged words: fp8gq_gather_decode
  if (launch_with_pdl(gather_wait_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), g) != cudaSuccess)
    return FP8GQ_ERR_LAUNCH;
  return launch_status();
}

int fp8gq_gather_decode(const fp8gq_gather* gather, int M, int N, void* out, int64_t ldo, fp8gq_stream_t stream) {
  GatherParams g;
  int st = to_gather_params(gather, &g);
  if (st != FP8GQ_OK) return st;
  if (!g.tagged) return FP8GQ_ERR_UNSUPPORTED;   // flags: fp8gq_gather_wait
  if (!out) return FP8GQ_ERR_NULL_POINTER;
  if (M < 1 || N <= 0 || N % kGroup) return FP8GQ_ERR_SHAPE;
  if (ldo < N || gather->ldo < N) return FP8GQ_ERR_STRIDE;
  if (!aligned16(out) || (ldo % 8)) return FP8GQ_ERR_ALIGNMENT;
  DeviceInfo di;
  st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  const int64_t chunks = static_cast<int64_t>(M) * (N / 16);
  int64_t blocks = (chunks + 255) / 256;
  if (blocks > di.sm_count) blocks = di.sm_count;
  if (launch_with_pdl(gather_decode_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                      static_cast<cudaStream_t>(stream), g, static_cast<__nv_bfloat16*>(out), ldo, M, N) != cudaSuccess)
    return FP8GQ_ERR_LAUNCH;
  return launch_status();
}

int fp8gq_ipc_get(const void* ptr, void* handle64, uint64_t* offset) {
  if (!ptr || !handle64 || !offset) return FP8GQ_ERR_NULL_POINTER;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  auto range = address_range_fn();
  if (!range) return FP8GQ_ERR_DEVICE;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return FP8GQ_ERR_DEVICE;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return FP8GQ_ERR_DEVICE;
  std::memcpy(handle64, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return FP8GQ_OK;
}

int fp8gq_ipc_open(const void* handle64, uint64_t offset, void** base, void** ptr) {
  if (!handle64 || !base || !ptr) return FP8GQ_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  void* b = nullptr;
  if (cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return FP8GQ_ERR_DEVICE;
  *base = b;
  *ptr = static_cast<uint8_t*>(b) + offset;
  return FP8GQ_OK;
}

int fp8gq_ipc_close(void* base) {
  if (!base) return FP8GQ_ERR_NULL_POINTER;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? FP8GQ_OK : FP8GQ_ERR_DEVICE;
}

int fp8gq_swiglu(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out, int64_t ldo, int M,
                 int I, fp8gq_stream_t stream) {
  const int st = check_swiglu_writer(gate, ldg, up, ldu, out, ldo, M, I, 2);
  if (st != FP8GQ_OK) return st;
  return launch_swiglu_writer(false, gate, ldg, up, ldu, out, ldo, nullptr, M, I,
                              static_cast<cudaStream_t>(stream));
}

int fp8gq_swiglu_quant(const void* gate, int64_t ldg, const void* up, int64_t ldu, uint8_t* q, int64_t ldq,
                       float* scale, int M, int I, fp8gq_stream_t stream) {
  int st = check_swiglu_writer(gate, ldg, up, ldu, q, ldq, M, I, 1);
  if (st != FP8GQ_OK) return st;
  if (!scale) return FP8GQ_ERR_NULL_POINTER;
  if (reinterpret_cast<uintptr_t>(scale) & 3u) return FP8GQ_ERR_ALIGNMENT;
  return launch_swiglu_writer(true, gate, ldg, up, ldu, q, ldq, scale, M, I, static_cast<cudaStream_t>(stream));
}

int fp8gq_set_static_weights(int enable) {
  return g_static_weights.exchange(enable ? 1 : 0);
}

int fp8gq_set_tm_options(int flags) {
  constexpr int kFeed = FP8GQ_TM_STREAM_ACTIVATIONS | FP8GQ_TM_PREQUANT_ACTIVATIONS | FP8GQ_TM_RESIDENT_ACTIVATIONS;
  if (flags & ~(kFeed | FP8GQ_TM_WORKSPACE_SPLITK)) return -1;
  const int feed = flags & kFeed;
  if (feed & (feed - 1)) return -1;   // more than one activation feed
  return g_tm_options.exchange(flags);
}

int fp8gq_set_wait_limit_ns(uint64_t limit_ns, uint64_t* previous) {
  if (limit_ns < kMinWaitLimitNs || limit_ns > kMaxWaitLimitNs) return FP8GQ_ERR_UNSUPPORTED;
  unsigned long long old = 0;
  if (cudaMemcpyFromSymbol(&old, g_wait_limit_ns, sizeof(old)) != cudaSuccess) return FP8GQ_ERR_LAUNCH;
  const unsigned long long v = limit_ns;
  if (cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v)) != cudaSuccess) return FP8GQ_ERR_LAUNCH;
  if (previous) *previous = old;
  return FP8GQ_OK;
}

int fp8gq_device_error(uint32_t* code, int clear) {
  if (!code) return FP8GQ_ERR_NULL_POINTER;
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return FP8GQ_ERR_LAUNCH;
  *code = v;
  if (clear && v) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)) != cudaSuccess) return FP8GQ_ERR_LAUNCH;
  }
  return FP8GQ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Stack runner (stack.cuh): plan preparation and launch.
// ---------------------------------------------------------------------------
namespace {

// Byte range [lo, hi) an [M, cols] bf16 operand with row stride ld covers.
struct ByteRange {
  uintptr_t lo, hi;
};
ByteRange bf16_range(const void* p, int M, int64_t cols, int64_t ld) {
  const uintptr_t lo = reinterpret_cast<uintptr_t>(p);
  return {lo, lo + static_cast<uintptr_t>(((M - 1) * ld + cols) * 2)};
}
bool overlaps(ByteRange a, ByteRange b) { return a.lo < b.hi && b.lo < a.hi; }

int stack_check(const fp8gq_stack_linear* lin, int n, int M) {
  if (!lin) return FP8GQ_ERR_NULL_POINTER;
  if (n < 1 || n > kStMaxLinears || M < 1 || M > kStMT) return FP8GQ_ERR_SHAPE;
  for (int l = 0; l < n; ++l) {
    const fp8gq_stack_linear& L = lin[l];
    int st = check_common(L.x, L.w, L.ws, L.out, M, L.N, L.K, L.ldw, L.ldws, L.ldo);
    if (st != FP8GQ_OK) return st;
    const int64_t cols = L.swiglu ? 2 * static_cast<int64_t>(L.K) : L.K;
    if (L.ldx < cols) return FP8GQ_ERR_STRIDE;
    if (L.ldx % 8) return FP8GQ_ERR_ALIGNMENT;
    if (L.N / kGroup > kStMaxRowBlocks) return FP8GQ_ERR_UNSUPPORTED;
    if (L.reserved != 0 || (L.swiglu != 0 && L.swiglu != 1)) return FP8GQ_ERR_UNSUPPORTED;
  }
  return FP8GQ_OK;
}

void stack_deps(const fp8gq_stack_linear* lin, int n, int M, int* dep) {
  for (int l = 0; l < n; ++l) {
    const fp8gq_stack_linear& L = lin[l];
    const ByteRange xl = bf16_range(L.x, M, L.swiglu ? 2 * static_cast<int64_t>(L.K) : L.K, L.ldx);
    const ByteRange ol = bf16_range(L.out, M, L.N, L.ldo);
    dep[l] = -1;
    for (int i = l - 1; i >= 0; --i) {
      const fp8gq_stack_linear& P = lin[i];
      const ByteRange xi = bf16_range(P.x, M, P.swiglu ? 2 * static_cast<int64_t>(P.K) : P.K, P.ldx);
      const ByteRange oi = bf16_range(P.out, M, P.N, P.ldo);
      if (overlaps(xl, oi) || overlaps(ol, xi) || overlaps(ol, oi)) {
        dep[l] = i;
        break;
      }
    }
  }
}

}  // namespace

extern "C" {

size_t fp8gq_stack_plan_bytes(int n, int M) {
  DeviceInfo di;
  if (n < 1 || n > kStMaxLinears || M < 1 || M > kStMT || device_info(&di, nullptr) != FP8GQ_OK) return 0;
  return st_plan_bytes(n, M, di.sm_count);
}

int fp8gq_stack_dependencies(const fp8gq_stack_linear* lin, int n, int M, int* dep) {
  if (!dep) return FP8GQ_ERR_NULL_POINTER;
  const int st = stack_check(lin, n, M);
  if (st != FP8GQ_OK) return st;
  stack_deps(lin, n, M, dep);
  return FP8GQ_OK;
}

int fp8gq_stack_prepare(const fp8gq_stack_linear* lin, int n, int M, void* device_mem, size_t bytes,
                        fp8gq_stack_plan* plan, fp8gq_stream_t stream) {
  if (!plan || !device_mem) return FP8GQ_ERR_NULL_POINTER;
  int st = stack_check(lin, n, M);
  if (st != FP8GQ_OK) return st;
  DeviceInfo di;
  int dev = 0;
  st = device_info(&di, &dev);
  if (st != FP8GQ_OK) return st;
  const int G = di.sm_count;
  if (bytes < st_plan_bytes(n, M, G) || (reinterpret_cast<uintptr_t>(device_mem) & 255u))
    return FP8GQ_ERR_WORKSPACE;
  // ring depth from the shared memory one CTA per SM may use (the resident
  // activation region takes what the ring leaves)
  const int64_t avail = static_cast<int64_t>(di.max_smem_optin) - static_cast<int64_t>(kStTailBytes) - 1024 -
                        kStWsLin * 4 - 64 * 132;
  const int S = st_pick_stages(avail / (kTmATileBytes + kStBTileBytes));
  StLayout lo;
  if (S < 4 || !st_layout(S, di.max_smem_optin, &lo)) return FP8GQ_ERR_UNSUPPORTED;
  std::vector<int> dep(n);
  stack_deps(lin, n, M, dep.data());
  std::vector<StackLinear> table(n);
  for (int l = 0; l < n; ++l) {
    const fp8gq_stack_linear& L = lin[l];
    StackLinear& T = table[l];
    std::memset(&T, 0, sizeof(T));
    if (!make_weight_tmap(&T.tmap_w, L.w, L.N, L.K, L.ldw)) return FP8GQ_ERR_LAUNCH;
    T.ws = L.ws;
    T.x = static_cast<const __nv_bfloat16*>(L.x);
    T.out = static_cast<__nv_bfloat16*>(L.out);
    T.ldws = L.ldws;
    T.ldx = L.ldx;
    T.ldo = L.ldo;
    T.N = L.N;
    T.K = L.K;
    T.KB = L.K / kGroup;
    T.U = static_cast<int64_t>(L.N / kGroup) * T.KB;
    T.swiglu = L.swiglu;
    T.dep = dep[l];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(device_mem);
  if (cudaMemcpyAsync(base, table.data(), static_cast<size_t>(n) * sizeof(StackLinear), cudaMemcpyHostToDevice,
                      s) != cudaSuccess)
    return FP8GQ_ERR_LAUNCH;
  // done counters, the exit counter and the split counters start at zero
  if (cudaMemsetAsync(base + st_table_bytes(n), 0, st_done_bytes(n) + st_counter_bytes(), s) != cudaSuccess)
    return FP8GQ_ERR_LAUNCH;
  std::memset(plan, 0, sizeof(*plan));
  plan->device = device_mem;
  plan->bytes = bytes;
  plan->n = n;
  plan->M = M;
  plan->device_id = dev;
  plan->grid = G;
  plan->stages = S;
  plan->npw = tm_producer_warps(S);
  int sw = 1, lg = 0;
  while (sw < M) {
    sw <<= 1;
    ++lg;
  }
  plan->sw = sw;
  plan->lg_sw = lg;
  plan->kpb = kStMT / sw;
  plan->nacc = plan->kpb >= 8 ? 2 : kTmMaxAcc;
  plan->smem = lo.smem;
  return FP8GQ_OK;
}

int fp8gq_stack_run(const fp8gq_stack_plan* plan, fp8gq_stream_t stream) {
  if (!plan || !plan->device) return FP8GQ_ERR_NULL_POINTER;
  DeviceInfo di;
  int dev = 0;
  int st = device_info(&di, &dev);
  if (st != FP8GQ_OK) return st;
  if (dev != plan->device_id || plan->grid != di.sm_count) return FP8GQ_ERR_DEVICE;
  if (plan->n < 1 || plan->n > kStMaxLinears || plan->M < 1 || plan->M > kStMT || plan->stages < 4 ||
      plan->stages > kStMaxStages || plan->smem > static_cast<size_t>(di.max_smem_optin))
    return FP8GQ_ERR_UNSUPPORTED;
  uint8_t* base = static_cast<uint8_t*>(plan->device);
  const int n = plan->n;
  StackParams p;
  p.lin = reinterpret_cast<const StackLinear*>(base);
  p.done = reinterpret_cast<unsigned int*>(base + st_table_bytes(n));
  p.exit_count = p.done + n;
  p.counters = reinterpret_cast<int*>(base + st_table_bytes(n) + st_done_bytes(n));
  p.partials = reinterpret_cast<float*>(base + st_table_bytes(n) + st_done_bytes(n) + st_counter_bytes());
  p.n = n;
  p.M = plan->M;
  p.sw = plan->sw;
  p.lg_sw = plan->lg_sw;
  p.kpb = plan->kpb;
  p.nacc = plan->nacc;
  p.stages = plan->stages;
  p.npw = plan->npw;
  StLayout lo;
  if (!st_layout(plan->stages, di.max_smem_optin, &lo) || lo.smem != plan->smem) return FP8GQ_ERR_UNSUPPORTED;
  p.b_off = lo.b_off;
  p.bar_off = lo.bar_off;
  p.res_off = lo.res_off;
  p.res_groups = lo.res_groups;
  cudaError_t e = cudaFuncSetAttribute(stack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(plan->smem));
  if (e != cudaSuccess) return cuda_fail(e, "stack_kernel shared memory attribute");
  // every CTA must be resident at once (they wait for one another): one CTA
  // per SM, launched as a cooperative grid, which the runtime refuses rather
  // than run partly
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stack_kernel, kStThreads, plan->smem);
  if (e != cudaSuccess) return cuda_fail(e, "stack_kernel occupancy");
  if (per_sm < 1) {
    if (std::getenv("FP8GQ_DEBUG")) {
      cudaFuncAttributes fa;
      int per_sm0 = -1;
      cudaFuncGetAttributes(&fa, stack_kernel);
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm0, stack_kernel, kStThreads, 0);
      std::fprintf(stderr, "fp8gq: stack_kernel regs %d, max threads %d, static smem %zu, local %zu, "
                   "max dynamic smem %d; CTAs per SM with %zu B: 0, with 0 B: %d\n", fa.numRegs,
                   fa.maxThreadsPerBlock, fa.sharedSizeBytes, fa.localSizeBytes, fa.maxDynamicSharedSizeBytes,
                   plan->smem, per_sm0);
    }
    return cuda_fail(cudaErrorInvalidConfiguration, "stack_kernel: no CTA fits on an SM");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan->grid);
  cfg.blockDim = dim3(kStThreads);
  cfg.dynamicSmemBytes = plan->smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, stack_kernel, p);
  if (e != cudaSuccess) return cuda_fail(e, "stack_kernel launch");
  e = cudaGetLastError();
  return e == cudaSuccess ? FP8GQ_OK : cuda_fail(e, "stack_kernel launch");
}

// ------------------------------------------------------------ chain runner --

size_t fp8gq_chain_plan_bytes(int n) {
  if (n < 1) return 0;
  return (static_cast<size_t>(n) * sizeof(ChainLin) + 255) / 256 * 256;
}

int fp8gq_chain_prepare(const fp8gq_chain_linear* lin, int n, const fp8gq_gather* gather, void* device_mem,
                        size_t bytes, fp8gq_chain_plan* plan) {
  if (!lin || !gather || !device_mem || !plan) return FP8GQ_ERR_NULL_POINTER;
  if (n < 1) return FP8GQ_ERR_SHAPE;
  if (bytes < fp8gq_chain_plan_bytes(n)) return FP8GQ_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(device_mem) & 255u) return FP8GQ_ERR_ALIGNMENT;
  if (!gather->counter || !gather->seq) return FP8GQ_ERR_NULL_POINTER;
  const int world = gather->world;
  if (world < 1 || world > FP8GQ_MAX_GATHER_RANKS || gather->rank < 0 || gather->rank >= world)
    return FP8GQ_ERR_SHAPE;
  for (int q = 0; q < world; ++q) {
    if (!gather->flags[q]) return FP8GQ_ERR_NULL_POINTER;
    if (reinterpret_cast<uintptr_t>(gather->flags[q]) & 3u) return FP8GQ_ERR_ALIGNMENT;
  }
  DeviceInfo di;
  int dev = 0;
  int st = device_info(&di, &dev);
  if (st != FP8GQ_OK) return st;
  std::vector<ChainLin> table(static_cast<size_t>(n));
  for (int i = 0; i < n; ++i) {
    const fp8gq_chain_linear& a = lin[i];
    ChainLin& c = table[static_cast<size_t>(i)];
    if (!a.x || !a.w || !a.ws) return FP8GQ_ERR_NULL_POINTER;
    if (a.N <= 0 || a.K <= 0 || a.N % kGroup || a.K % kGroup || a.K > kChainMaxK) return FP8GQ_ERR_SHAPE;
    if (a.src < -1 || a.src >= i || a.reserved != 0) return FP8GQ_ERR_SHAPE;
    if (a.ldw < a.K || a.ldws < a.K / kGroup) return FP8GQ_ERR_STRIDE;
    if (!aligned16(a.w) || (a.ldw % 16) || !aligned16(a.x) || (reinterpret_cast<uintptr_t>(a.ws) & 3u) ||
        a.col0 < 0 || (a.col0 % 2))
      return FP8GQ_ERR_ALIGNMENT;
    for (int r = 0; r < world; ++r) {
      if (!a.out[r]) return FP8GQ_ERR_NULL_POINTER;
      if (!aligned16(a.out[r])) return FP8GQ_ERR_ALIGNMENT;
    }
    c.x = a.x;
    c.w = static_cast<const uint8_t*>(a.w);
    c.ws = a.ws;
    c.ldw = a.ldw;
    c.ldws = a.ldws;
    c.N = a.N;
    c.K = a.K;
    c.src = a.src;
    c.swiglu = a.swiglu ? 1 : 0;
    c.col0 = a.col0;
    // rows per stage: the most (4, 2 or 1) whose stage is at most 16 KB, as
    // the row kernel; with one row per stage the CTAs take rows in pairs (a
    // tagged word holds two columns)
    c.R = (4 * a.K <= kChainSlotBytes) ? 4 : (2 * a.K <= kChainSlotBytes) ? 2 : 1;
    c.unit_stages = c.R == 1 ? 2 : 1;
    c.units = c.R == 1 ? a.N / 2 : a.N / c.R;
    for (int r = 0; r < kMaxGatherRanks; ++r) c.out[r] = r < world ? static_cast<uint64_t*>(a.out[r]) : nullptr;
  }
  cudaError_t e = cudaMemcpy(device_mem, table.data(), table.size() * sizeof(ChainLin), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "chain table copy");
  const int stages = kChainRingBytes / kChainSlotBytes;
  const size_t smem = static_cast<size_t>(stages) * kChainSlotBytes + 2 * stages * sizeof(uint64_t) +
                      2 * (kChainThreads / 32) * kRowWindow * sizeof(float);
  if (smem > static_cast<size_t>(di.max_smem_optin)) return FP8GQ_ERR_UNSUPPORTED;
  e = cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_fail(e, "chain_kernel shared memory attribute");
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, chain_kernel, kChainThreads + 32, smem);
  if (e != cudaSuccess) return cuda_fail(e, "chain_kernel occupancy");
  if (per_sm < 1) return FP8GQ_ERR_UNSUPPORTED;
  if (per_sm > 2) per_sm = 2;
  *plan = fp8gq_chain_plan{};
  plan->device = device_mem;
  plan->bytes = bytes;
  plan->n = n;
  plan->device_id = dev;
  plan->grid = per_sm * di.sm_count;
  plan->stages = stages;
  plan->world = world;
  plan->rank = gather->rank;
  plan->smem = smem;
  for (int q = 0; q < world; ++q) plan->flags[q] = gather->flags[q];
  plan->counter = gather->counter;
  plan->seq = gather->seq;
  return FP8GQ_OK;
}

int fp8gq_chain_run(const fp8gq_chain_plan* plan, fp8gq_stream_t stream) {
  if (!plan || !plan->device || !plan->counter || !plan->seq) return FP8GQ_ERR_NULL_POINTER;
  DeviceInfo di;
  int dev = 0;
  int st = device_info(&di, &dev);
  if (st != FP8GQ_OK) return st;
  if (dev != plan->device_id) return FP8GQ_ERR_DEVICE;
  if (plan->n < 1 || plan->world < 1 || plan->world > FP8GQ_MAX_GATHER_RANKS || plan->grid < 1 ||
      plan->stages != kChainRingBytes / kChainSlotBytes || plan->smem > static_cast<size_t>(di.max_smem_optin) ||
      plan->grid > 2 * di.sm_count)
    return FP8GQ_ERR_UNSUPPORTED;
  ChainParams p;
  p.lin = static_cast<const ChainLin*>(plan->device);
  p.n = plan->n;
  p.stages = plan->stages;
  for (int q = 0; q < kMaxGatherRanks; ++q) p.flags[q] = q < plan->world ? plan->flags[q] : nullptr;
  p.counter = plan->counter;
  p.seq = plan->seq;
  p.world = plan->world;
  p.rank = plan->rank;
  cudaError_t e = cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(plan->smem));
  if (e != cudaSuccess) return cuda_fail(e, "chain_kernel shared memory attribute");
  // every CTA must be resident at once (they wait for one another's words):
  // a cooperative grid, which the runtime refuses rather than run partly
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan->grid);
  cfg.blockDim = dim3(kChainThreads + 32);
  cfg.dynamicSmemBytes = plan->smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, chain_kernel, p);
  if (e != cudaSuccess) return cuda_fail(e, "chain_kernel launch");
  e = cudaGetLastError();
  return e == cudaSuccess ? FP8GQ_OK : cuda_fail(e, "chain_kernel launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// fp8gq_gemv_quant_tm_noalloc: the tile kernel with its split-K scratch in a
// fixed device array instead of a caller-provided workspace, for callers that
// cannot allocate (see include/fp8gq.h).  Nothing here allocates.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = FP8GQ_NOALLOC_SCRATCH_BYTES;

// Zero-initialised when the library's module loads on a device; holds the
// split-K counters (first kTmCounterBytes) and the partial sums.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is looked up
// once per device with that device current, and kept for the life of the
// process (a cudaDeviceReset between calls would leave it stale; the entry
// point's documentation says not to do that).
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FP8GQ_ERR_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return FP8GQ_ERR_LAUNCH;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return FP8GQ_OK;
}

}  // namespace

extern "C" int fp8gq_gemv_quant_tm_noalloc(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                           const float* ws, int64_t ldws, void* out, int64_t ldo,
                                           int M, int N, int K, uint8_t* xq_out, float* sx_out,
                                           fp8gq_stream_t stream) {
  int st = check_common(x, w, ws, out, M, N, K, ldw, ldws, ldo);
  if (st != FP8GQ_OK) return st;
  if (ldx < K || (ldx % 8) != 0) return ldx < K ? FP8GQ_ERR_STRIDE : FP8GQ_ERR_ALIGNMENT;
  DeviceInfo di;
  st = device_info(&di, nullptr);
  if (st != FP8GQ_OK) return st;
  if (N / kGroup > kTmMaxRowBlocks || tm_workspace_bytes_for(M, N, K, di.sm_count) > kNoAllocScratchBytes)
    return FP8GQ_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st != FP8GQ_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the split-K counters must start at zero
  if (cudaMemsetAsync(scratch, 0, kTmCounterBytes, s) != cudaSuccess) return FP8GQ_ERR_LAUNCH;
  return launch_tm(false, x, ldx, w, ldw, ws, ldws, out, ldo, M, N, K, xq_out, sx_out, scratch,
                   kNoAllocScratchBytes, di.sm_count, di.max_smem_optin, s,
                   g_static_weights.load(std::memory_order_relaxed), 0, tm_resident_mode(),
                   tm_cluster_mode());
}

// ---------------------------------------------------------------------------
// Prepared launches: the entry points above, recorded once and issued later
// (fp8gq_prepare_* / fp8gq_launch_plans in include/fp8gq.h).
// ---------------------------------------------------------------------------
namespace {

static_assert(sizeof(LaunchRecord) <= sizeof(fp8gq_launch_plan), "fp8gq_launch_plan too small for a record");
static_assert(alignof(LaunchRecord) <= alignof(fp8gq_launch_plan), "fp8gq_launch_plan under-aligned");

// Runs `issue` (an entry point called with a null stream) with a recorder
// installed, so that its launches land in `plan` instead of a stream.
template <typename F>
int prepare_into(fp8gq_launch_plan* plan, F&& issue) {
  if (!plan) return FP8GQ_ERR_NULL_POINTER;
  LaunchRecord* rec = reinterpret_cast<LaunchRecord*>(plan);
  std::memset(rec, 0, sizeof(*rec));
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FP8GQ_ERR_DEVICE;
  rec->device = dev;
  int st;
  {
    RecordScope scope(rec);
    st = issue();
  }
  if (st == FP8GQ_OK && (rec->overflow || rec->n == 0)) st = FP8GQ_ERR_UNSUPPORTED;
  rec->magic = st == FP8GQ_OK ? kRecMagic : 0;
  return st;
}

}  // namespace

extern "C" {

int fp8gq_prepare_fused_gemv_quant(const void* x, int64_t ldx, const void* w, int64_t ldw, const float* ws,
                                   int64_t ldws, void* out, int64_t ldo, int M, int N, int K, uint8_t* xq_out,
                                   float* sx_out, void* workspace, size_t workspace_bytes, fp8gq_launch_plan* plan) {
  return prepare_into(plan, [&] {
    return fp8gq_fused_gemv_quant(x, ldx, w, ldw, ws, ldws, out, ldo, M, N, K, xq_out, sx_out, workspace,
                                  workspace_bytes, nullptr);
  });
}

int fp8gq_prepare_fused_swiglu_q_gemm(const void* gu, int64_t ldgu, const void* w, int64_t ldw, const float* ws,
                                      int64_t ldws, void* out, int64_t ldo, int M, int N, int I, uint8_t* xq_out,
                                      float* sx_out, void* workspace, size_t workspace_bytes,
                                      fp8gq_launch_plan* plan) {
  return prepare_into(plan, [&] {
    return fp8gq_fused_swiglu_q_gemm(gu, ldgu, w, ldw, ws, ldws, out, ldo, M, N, I, xq_out, sx_out, workspace,
                                     workspace_bytes, nullptr);
  });
}

int fp8gq_prepare_fused_gemv_quant_gather(const void* x, int64_t ldx, const void* w, int64_t ldw, const float* ws,
                                          int64_t ldws, int M, int N, int K, const fp8gq_gather* gather,
                                          void* workspace, size_t workspace_bytes, fp8gq_launch_plan* plan) {
  return prepare_into(plan, [&] {
    return fp8gq_fused_gemv_quant_gather(x, ldx, w, ldw, ws, ldws, M, N, K, gather, workspace, workspace_bytes,
                                         nullptr);
  });
}

int fp8gq_prepare_fused_swiglu_q_gemm_gather(const void* gu, int64_t ldgu, const void* w, int64_t ldw,
                                             const float* ws, int64_t ldws, int M, int N, int I,
                                             const fp8gq_gather* gather, void* workspace, size_t workspace_bytes,
                                             fp8gq_launch_plan* plan) {
  return prepare_into(plan, [&] {
    return fp8gq_fused_swiglu_q_gemm_gather(gu, ldgu, w, ldw, ws, ldws, M, N, I, gather, workspace,
                                            workspace_bytes, nullptr);
  });
}

int fp8gq_prepare_fused_reduce_add_rmsnorm_gemv_quant(
    const void* x, int nsrc, int64_t src_stride, int64_t ldx, const void* residual, int64_t ldr, const void* norm_w,
    float eps, const void* w, int64_t ldw, const float* ws, int64_t ldws, void* out, int64_t ldo, void* residual_out,
    int64_t ldro, int M, int N, int K, uint8_t* xq_out, float* sx_out, const fp8gq_gather* wait, void* workspace,
    size_t workspace_bytes, fp8gq_launch_plan* plan) {
  return prepare_into(plan, [&] {
    return fp8gq_fused_reduce_add_rmsnorm_gemv_quant(x, nsrc, src_stride, ldx, residual, ldr, norm_w, eps, w, ldw,
                                                     ws, ldws, out, ldo, residual_out, ldro, M, N, K, xq_out, sx_out,
                                                     wait, workspace, workspace_bytes, nullptr);
  });
}

int fp8gq_prepare_gather_wait(const fp8gq_gather* gather, fp8gq_launch_plan* plan) {
  return prepare_into(plan, [&] { return fp8gq_gather_wait(gather, nullptr); });
}

int fp8gq_prepare_gather_decode(const fp8gq_gather* gather, int M, int N, void* out, int64_t ldo,
                                fp8gq_launch_plan* plan) {
  return prepare_into(plan, [&] { return fp8gq_gather_decode(gather, M, N, out, ldo, nullptr); });
}

int fp8gq_launch_plans(const fp8gq_launch_plan* plans, int n, fp8gq_stream_t stream) {
  if (n < 0) return FP8GQ_ERR_SHAPE;
  if (n > 0 && !plans) return FP8GQ_ERR_NULL_POINTER;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FP8GQ_ERR_DEVICE;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n; ++i) {
    const LaunchRecord* rec = reinterpret_cast<const LaunchRecord*>(plans + i);
    if (rec->magic != kRecMagic || rec->n < 1 || rec->n > kRecMaxLaunches) return FP8GQ_ERR_UNSUPPORTED;
    if (rec->device != dev) return FP8GQ_ERR_DEVICE;
    const cudaError_t e = launch_recorded(*rec, s);
    if (e != cudaSuccess) return cuda_fail(e, "fp8gq_launch_plans");
  }
  return FP8GQ_OK;
}

}  // extern "C"
