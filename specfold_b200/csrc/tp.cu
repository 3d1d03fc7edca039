// Tensor parallelism of the folded verify forward (the 14B configuration): each rank
// holds a head / intermediate shard of every layer; the two row-sharded projections
// (o_proj and down) produce fp32 partial sums that are all-reduced over NVLink, then the
// residual add (o_proj) and the row scatter (down) run on the reduced sums.
//
// NCCL is loaded at run time (dlopen "libnccl.so.2"): the process's own copy when torch
// already loaded it, the system one otherwise; the library has no link-time dependency
// on it.  The communicator is this library's own (ncclCommInitRank on an id that rank 0
// creates and the host broadcasts), so the all-reduces are plain stream operations that
// a CUDA graph of the forward captures.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "sf_kernels.cuh"

namespace sf {

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce &&
             api.error_string;
  });
  return api;
}

}  // namespace

const char* tp_error_string(int r) {
  const NcclApi& a = nccl();
  return a.ok ? a.error_string(static_cast<ncclResult_t>(r)) : "NCCL not loadable";
}

int tp_unique_id(void* out, int bytes) {
  const NcclApi& a = nccl();
  if (!a.ok) return -1;
  if (bytes < static_cast<int>(sizeof(ncclUniqueId))) return -2;
  return static_cast<int>(a.get_unique_id(static_cast<ncclUniqueId*>(out)));
}

int tp_comm_init(const void* id, int nranks, int rank, void** comm) {
  const NcclApi& a = nccl();
  if (!a.ok) return -1;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  const ncclResult_t r = a.comm_init_rank(&c, nranks, uid, rank);
  *comm = c;
  return static_cast<int>(r);
}

int tp_comm_destroy(void* comm) {
  const NcclApi& a = nccl();
  if (!a.ok) return -1;
  return static_cast<int>(a.comm_destroy(static_cast<ncclComm_t>(comm)));
}

int tp_allreduce_f32(void* comm, float* buf, size_t n, cudaStream_t st) {
  const NcclApi& a = nccl();
  if (!a.ok) return -1;
  return static_cast<int>(
      a.all_reduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st));
}

// hp[i] = T(resid[i] + T(sum[i])): the EPI_RESID arithmetic on the all-reduced sums
template <typename T>
__global__ void __launch_bounds__(256) resid_add_kernel(const float* __restrict__ sum,
                                                        const T* __restrict__ resid, T* out,
                                                        int64_t n) {
  for (int64_t i = (blockIdx.x * 256ll + threadIdx.x) * 4; i < n; i += 256ll * gridDim.x * 4) {
    const float4 s = *reinterpret_cast<const float4*>(sum + i);
    float r[4], o[4];
    const float sv[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      r[k] = Elt<T>::to_f(resid[i + k]);
      o[k] = __fadd_rn(r[k], Elt<T>::rnd(sv[k]));
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) out[i + k] = Elt<T>::from_f(o[k]);
  }
}

// out[rows[j]][:] = T(sum[j][:]) for j < min(*count, n): the EPI_SCATTER arithmetic
template <typename T>
__global__ void __launch_bounds__(256) scatter_rows_kernel(const float* __restrict__ sum,
                                                           const int64_t* rows,
                                                           const int32_t* count, int n, int D,
                                                           int64_t n_out_rows, T* out, int* err) {
  const int j = blockIdx.x;
  const int cnt = min(*count, n);
  if (j >= cnt) return;
  const int64_t r = rows[j];
  if (r < 0 || r >= n_out_rows) {
    if (threadIdx.x == 0) flag_error(err, SF_DEV_ERR_INDEX);
    return;
  }
  for (int d = threadIdx.x * 4; d < D; d += 256 * 4) {
    const float4 s = *reinterpret_cast<const float4*>(sum + static_cast<int64_t>(j) * D + d);
    out[r * D + d] = Elt<T>::from_f(s.x);
    out[r * D + d + 1] = Elt<T>::from_f(s.y);
    out[r * D + d + 2] = Elt<T>::from_f(s.z);
    out[r * D + d + 3] = Elt<T>::from_f(s.w);
  }
}

cudaError_t launch_resid_add(int dtype, const float* sum, const void* resid, void* out, int64_t n,
                             cudaStream_t st) {
  if (n % 4 != 0) return cudaErrorInvalidValue;
  const int blocks = static_cast<int>(std::min<int64_t>((n / 4 + 255) / 256, 148 * 8));
  if (dtype == BF16)
    resid_add_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        sum, static_cast<const __nv_bfloat16*>(resid), static_cast<__nv_bfloat16*>(out), n);
  else
    resid_add_kernel<float><<<blocks, 256, 0, st>>>(sum, static_cast<const float*>(resid),
                                                    static_cast<float*>(out), n);
  return launched();
}

cudaError_t launch_scatter_rows(int dtype, const float* sum, const int64_t* rows,
                                const int32_t* count, int n, int D, int64_t n_out_rows, void* out,
                                int* err, cudaStream_t st) {
  if (D % 4 != 0 || n <= 0) return n <= 0 ? cudaSuccess : cudaErrorInvalidValue;
  if (dtype == BF16)
    scatter_rows_kernel<__nv_bfloat16><<<n, 256, 0, st>>>(sum, rows, count, n, D, n_out_rows,
                                                          static_cast<__nv_bfloat16*>(out), err);
  else
    scatter_rows_kernel<float><<<n, 256, 0, st>>>(sum, rows, count, n, D, n_out_rows,
                                                  static_cast<float*>(out), err);
  return launched();
}

// ------------------------------------------------------------------ peer-memory reduce
// The NCCL all-reduce of a 5 MB fp32 partial costs ~40 us per call on two B200s; the two
// per layer made the tensor-parallel step slower than one GPU.  Instead every rank keeps
// its partial sums in an exchange buffer that every other rank has mapped (CUDA IPC over
// NVLink), and the kernel that consumes the sum -- the residual add after o_proj, the row
// scatter after down -- reads all ranks' partials straight from their memory:
//   * at its start, one thread publishes "my partial of (layer, kind) is complete" into
//     every peer's flag slot for this rank (a release store at system scope after a
//     system fence; the partial was written by the previous kernel on this stream);
//   * one thread per CTA waits (bounded) until every peer's slot in the local flags
//     shows the same sequence number, then the CTA sums the ranks' partials in rank
//     order (identical on every rank: the gate that follows decides the same folds) and
//     applies the epilogue arithmetic of the unsharded forward.
// Sequence numbers grow monotonically: seq = epoch * 2L + 2 * layer + kind with a per-rank
// epoch bumped by one kernel at the start of every forward (both ranks run the same
// forwards), so a captured graph replays with fresh numbers.  Reuse of a partial region is
// safe without a second handshake: a rank overwrites its o_proj (down) partial of the
// next layer only after its own down (o_proj) reduce, which waited for every peer to
// have started -- hence, in stream order, finished -- the reduce that reads it.

namespace {

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// publish this rank's partial (thread 0 of CTA 0) and wait for every peer's (thread 0 of
// every CTA); false after a timeout (SF_DEV_ERR_TIMEOUT set)
__device__ bool tp_handshake(const TpPeers& t, int kind, int seq, int* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int q = 0; q < t.size; ++q)
        if (q != t.rank) st_release_sys(t.flags[q] + 2 * t.rank + kind, seq);
    }
    bool ok = true;
    const uint64_t t0 = globaltimer();
    for (int q = 0; q < t.size && ok; ++q) {
      if (q == t.rank) continue;
      const int* f = t.flags[t.rank] + 2 * q + kind;
      while (ld_acquire_sys(f) - seq < 0) {
        if (globaltimer() - t0 > kWaitNs) {
          flag_error(err, SF_DEV_ERR_TIMEOUT);
          ok = false;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

__global__ void tp_epoch_kernel(unsigned* epoch) { *epoch += 1u; }

// Every rank's float4 at element offsets i + k * stride (k < kU), all loads in flight
// before any is used (the peers' are NVLink round trips); acc[k] = sum in rank order.
// S >= t.size bounds the register array (2, 4 or 8 ranks).
constexpr int kU = 4;
template <int S>
__device__ __forceinline__ void tp_gather_sum(const TpPeers& t, int64_t off, int64_t i,
                                              int64_t stride, int64_t n, float4* acc) {
  float4 v[S][kU];
#pragma unroll
  for (int q = 0; q < S; ++q)
#pragma unroll
    for (int k = 0; k < kU; ++k)
      if (q < t.size && i + k * stride < n)
        v[q][k] = __ldcv(reinterpret_cast<const float4*>(t.part[q] + off + i + k * stride));
#pragma unroll
  for (int k = 0; k < kU; ++k) {
    acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < S; ++q)
      if (q < t.size && i + k * stride < n) {
        acc[k].x += v[q][k].x; acc[k].y += v[q][k].y; acc[k].z += v[q][k].z; acc[k].w += v[q][k].w;
      }
  }
}

// hp[i] = T(resid[i] + T(sum_q part_q[i])), i < n (the EPI_RESID arithmetic)
template <int S, typename T>
__global__ void __launch_bounds__(256) tp_reduce_resid_kernel(TpPeers t, int layer, int L,
                                                              const T* __restrict__ resid,
                                                              T* out, int64_t n, int* err) {
  const int seq = static_cast<int>(*t.epoch) * 2 * L + 2 * layer;
  if (!tp_handshake(t, 0, seq, err)) return;
  const int64_t stride = 256ll * gridDim.x * 4;
  for (int64_t i = (blockIdx.x * 256ll + threadIdx.x) * 4; i < n; i += stride * kU) {
    float4 acc[kU];
    tp_gather_sum<S>(t, 0, i, stride, n, acc);
#pragma unroll
    for (int k = 0; k < kU; ++k) {
      const int64_t e = i + k * stride;
      if (e >= n) break;
      const float sv[4] = {acc[k].x, acc[k].y, acc[k].z, acc[k].w};
#pragma unroll
      for (int c = 0; c < 4; ++c)
        out[e + c] = Elt<T>::from_f(__fadd_rn(Elt<T>::to_f(resid[e + c]), Elt<T>::rnd(sv[c])));
    }
  }
}

// out[rows[j]][:] = T(sum_q part_q[j][:]) for j < min(*count, n) (the EPI_SCATTER
// arithmetic); the down partials sit after the o_proj ones in every exchange buffer
template <int S, typename T>
__global__ void __launch_bounds__(256) tp_reduce_scatter_kernel(TpPeers t, int layer, int L,
                                                                int64_t part_off,
                                                                const int64_t* rows,
                                                                const int32_t* count, int n,
                                                                int D, int64_t n_out_rows,
                                                                T* out, int* err) {
  const int seq = static_cast<int>(*t.epoch) * 2 * L + 2 * layer + 1;
  if (!tp_handshake(t, 1, seq, err)) return;
  const int cnt = min(*count, n);
  const int64_t total = static_cast<int64_t>(cnt) * D;
  const int64_t stride = 256ll * gridDim.x * 4;
  for (int64_t i = (blockIdx.x * 256ll + threadIdx.x) * 4; i < total; i += stride * kU) {
    float4 acc[kU];
    tp_gather_sum<S>(t, part_off, i, stride, total, acc);
#pragma unroll
    for (int k = 0; k < kU; ++k) {
      const int64_t e = i + k * stride;
      if (e >= total) break;
      const int64_t j = e / D, d = e % D;
      const int64_t r = rows[j];
      if (r < 0 || r >= n_out_rows) {
        flag_error(err, SF_DEV_ERR_INDEX);
        continue;
      }
      out[r * D + d] = Elt<T>::from_f(acc[k].x);
      out[r * D + d + 1] = Elt<T>::from_f(acc[k].y);
      out[r * D + d + 2] = Elt<T>::from_f(acc[k].z);
      out[r * D + d + 3] = Elt<T>::from_f(acc[k].w);
    }
  }
}

int reduce_grid(int64_t n) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n / 4 / kU + 255) / 256, 148 * 4)));
}

}  // namespace

cudaError_t launch_tp_epoch(const TpPeers& t, cudaStream_t st) {
  tp_epoch_kernel<<<1, 1, 0, st>>>(t.epoch);
  return launched();
}

template <int S>
void reduce_resid_s(int dtype, const TpPeers& t, int layer, int L, const void* resid, void* out,
                    int64_t n, int* err, cudaStream_t st) {
  const int blocks = reduce_grid(n);
  if (dtype == BF16)
    tp_reduce_resid_kernel<S, __nv_bfloat16><<<blocks, 256, 0, st>>>(
        t, layer, L, static_cast<const __nv_bfloat16*>(resid), static_cast<__nv_bfloat16*>(out),
        n, err);
  else
    tp_reduce_resid_kernel<S, float><<<blocks, 256, 0, st>>>(
        t, layer, L, static_cast<const float*>(resid), static_cast<float*>(out), n, err);
}

cudaError_t launch_tp_reduce_resid(int dtype, const TpPeers& t, int layer, int L,
                                   const void* resid, void* out, int64_t n, int* err,
                                   cudaStream_t st) {
  if (n % 4 != 0 || t.size < 1 || t.size > kMaxTp) return cudaErrorInvalidValue;
  if (t.size <= 2) reduce_resid_s<2>(dtype, t, layer, L, resid, out, n, err, st);
  else if (t.size <= 4) reduce_resid_s<4>(dtype, t, layer, L, resid, out, n, err, st);
  else reduce_resid_s<8>(dtype, t, layer, L, resid, out, n, err, st);
  return launched();
}

template <int S>
void reduce_scatter_s(int dtype, const TpPeers& t, int layer, int L, const int64_t* rows,
                      const int32_t* count, int n, int D, int64_t n_out_rows, void* out, int* err,
                      cudaStream_t st) {
  const int blocks = reduce_grid(static_cast<int64_t>(n) * D);
  const int64_t off = t.part_elems;
  if (dtype == BF16)
    tp_reduce_scatter_kernel<S, __nv_bfloat16><<<blocks, 256, 0, st>>>(
        t, layer, L, off, rows, count, n, D, n_out_rows, static_cast<__nv_bfloat16*>(out), err);
  else
    tp_reduce_scatter_kernel<S, float><<<blocks, 256, 0, st>>>(
        t, layer, L, off, rows, count, n, D, n_out_rows, static_cast<float*>(out), err);
}

cudaError_t launch_tp_reduce_scatter(int dtype, const TpPeers& t, int layer, int L,
                                     const int64_t* rows, const int32_t* count, int n, int D,
                                     int64_t n_out_rows, void* out, int* err, cudaStream_t st) {
  if (D % 4 != 0 || n <= 0) return n <= 0 ? cudaSuccess : cudaErrorInvalidValue;
  if (t.size < 1 || t.size > kMaxTp) return cudaErrorInvalidValue;
  if (t.size <= 2) reduce_scatter_s<2>(dtype, t, layer, L, rows, count, n, D, n_out_rows, out, err, st);
  else if (t.size <= 4) reduce_scatter_s<4>(dtype, t, layer, L, rows, count, n, D, n_out_rows, out, err, st);
  else reduce_scatter_s<8>(dtype, t, layer, L, rows, count, n, D, n_out_rows, out, err, st);
  return launched();
}

}  // namespace sf
