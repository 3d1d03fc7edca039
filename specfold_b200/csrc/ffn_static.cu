// sf_fused_ffn_scatter_static: the fused FFN of the folded verify forward (post-attention
// RMSNorm -> gate/up + SiLU -> down -> scatter) for callers that cannot allocate device
// memory.
//
// Why it exists: sf_fused_ffn_scatter needs scratch the caller provides (the normalised
// rows, the SwiGLU activations, split-K partial sums).  Some callers cannot call
// cudaMalloc at all -- code running inside a CUDA graph being captured, allocator-less
// embedded runtimes, or hosts whose memory pool is owned by someone else.  This variant
// takes only inputs and outputs and keeps its scratch in a file-scope __device__ array
// of fixed size, so it calls no cudaMalloc, cudaFree or allocating library routine.
//
// Costs and rules (also in include/specfold_b200.h):
//  * kScratchBytes (32 MiB) of device memory on every GPU where this module is loaded,
//    held until the process exits.  With CUDA's default lazy module loading that is the
//    first call on the device.
//  * The first call on each device resolves the array's device address with
//    cudaGetSymbolAddress (with that device current); make that first call before any
//    stream capture.  The address is cached per device index for the life of the
//    process, so it is stale after cudaDeviceReset: no calls after a reset.
//  * All calls share the one array and it keeps the previous call's contents: the
//    split-K counters are cleared at every call; calls that overlap on the GPU (two
//    streams, or two host threads) race on the array and must be serialised by the caller.
//  * Shapes whose scratch would exceed kScratchBytes are rejected with SF_ERR_ARG.
#include <mutex>

#include "../../include/specfold_b200.h"
#include "sf_kernels.cuh"

namespace sf {
int report_error(int code, const char* msg);
int report_cuda(cudaError_t e, const char* what);
}  // namespace sf

using namespace sf;

namespace {

constexpr size_t kScratchBytes = 32ull << 20;
// split-K tile counters at the start of the GEMM scratch: the same region every GEMM of
// the library keeps there, so that clearing it here clears every counter a launch reads
constexpr size_t kCounterRegion = kGemmCounterBytes;
constexpr int kMaxDevices = 64;

// In host code this name is only a stand-in: the kernels get the address that
// cudaGetSymbolAddress returns.
__device__ __align__(256) unsigned char g_ffn_scratch[kScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return report_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return report_error(SF_ERR_ARG, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ffn_scratch);
    if (e != cudaSuccess) return report_cuda(e, "cudaGetSymbolAddress(scratch)");
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return SF_OK;
}

}  // namespace

extern "C" int sf_fused_ffn_scatter_static(int dtype, const void* hp_all, const void* ln_w,
                                           const void* w_gate, const void* w_up,
                                           const void* w_down, const int64_t* rows,
                                           const int32_t* count, void* ffn_buf, int bucket,
                                           float eps, int D, int I, int* err, void* stream) {
  if ((dtype != SF_DTYPE_F32 && dtype != SF_DTYPE_BF16) || !hp_all || !ln_w || !w_gate ||
      !w_up || !w_down || !rows || !count || !ffn_buf || D <= 0 || I <= 0 || D % 64 ||
      I % 64 || bucket < 1)
    return report_error(SF_ERR_ARG, "bad ffn arguments");
  // the tensor-core GEMMs stream the weights through TMA, which needs 16-byte aligned
  // bases; checked here, before anything is queued, as sf_fused_ffn_scatter does
  if (dtype == SF_DTYPE_BF16) {
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    if (!a16(w_gate) || !a16(w_up) || !a16(w_down))
      return report_error(SF_ERR_ARG, "ffn (static scratch): weights must be 16-byte aligned");
  }
  const size_t es = dtype == SF_DTYPE_BF16 ? 2 : 4;
  // scratch layout: [GEMM scratch (counters first)] [xn bucket x D] [act bucket x I] [rstd]
  const size_t g_gu = gemm_ws_need(dtype, bucket, 2 * I, D, EPI_SWIGLU, I);
  const size_t g_dn = gemm_ws_need(dtype, bucket, D, I, EPI_SCATTER, 0);
  const size_t g = up256(std::max(std::max(g_gu, g_dn), kCounterRegion));
  const size_t xn_off = g;
  const size_t act_off = xn_off + up256(static_cast<size_t>(bucket) * D * es);
  const size_t rstd_off = act_off + up256(static_cast<size_t>(bucket) * I * es);
  const size_t total = rstd_off + up256(static_cast<size_t>(bucket) * 4);
  if (total > kScratchBytes) {
    char msg[160];
    snprintf(msg, sizeof(msg),
             "ffn (static scratch): shape needs %zu bytes of scratch, the limit is %zu",
             total, kScratchBytes);
    return report_error(SF_ERR_ARG, msg);
  }
  void* base = nullptr;
  int s = scratch_address(&base);
  if (s) return s;
  char* sc = static_cast<char*>(base);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the previous call leaves its contents behind: counters must start at zero
  cudaError_t e = cudaMemsetAsync(sc, 0, kCounterRegion, st);
  if (e != cudaSuccess) return report_cuda(e, "clear static scratch counters");

  RmsRowsParams r{};
  r.x = hp_all;
  r.rows = rows;
  r.count = count;
  r.n = bucket;
  r.n_src = INT64_MAX;
  r.w = ln_w;
  r.out = sc + xn_off;
  r.rstd = reinterpret_cast<float*>(sc + rstd_off);
  r.D = D;
  r.eps = eps;
  r.err = err;
  e = launch_rmsnorm_rows(dtype, r, st);
  if (e != cudaSuccess) return report_cuda(e, "ffn norm");

  GemmArgs a{};
  a.dtype = dtype;
  a.X = sc + xn_off;
  a.W = w_gate;
  a.W2 = w_up;
  a.n_out = 2 * I;
  a.K = D;
  a.rows_cap = bucket;
  a.count = count;
  a.epi.kind = EPI_SWIGLU;
  a.epi.out = sc + act_off;
  a.epi.inter = I;
  a.ws = sc;
  a.ws_bytes = g;
  a.err = err;
  e = gemm(a, st);
  if (e != cudaSuccess) return report_cuda(e, "gate/up");

  GemmArgs d{};
  d.dtype = dtype;
  d.X = sc + act_off;
  d.W = w_down;
  d.n_out = D;
  d.K = I;
  d.rows_cap = bucket;
  d.count = count;
  d.epi.kind = EPI_SCATTER;
  d.epi.out = ffn_buf;
  d.epi.rows = rows;
  d.epi.ld_out = D;
  d.ws = sc;
  d.ws_bytes = g;
  d.err = err;
  e = gemm(d, st);
  if (e != cudaSuccess) return report_cuda(e, "down");
  return SF_OK;
}
