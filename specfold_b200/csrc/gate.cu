// Fold gate, deterministic row compaction, RMSNorm row preparation and the residual
// combine of the folded verify forward.
//
//   gate_rows_kernel   : optional combine (hidden = hp + ffn[src]) fused with the
//                        per-row statistics of the next layer's gate -- rstd and the
//                        recompute decision ||x - x_par|| > delta ||x_par||
//                        (fastdllm_v2_folded.py:139-141 / triton_kernels.py:199-232)
//   compact_kernel     : rows / seg / segcnt / count / src and the normalised A operand
//                        of the QKV projection (triton_kernels.py:18-26,233-239)
//   rmsnorm_rows_kernel: RMSNorm of (optionally gathered) rows, for the FFN input and the
//                        final norm (triton_kernels.py:90-99, fastdllm_v2_folded.py:365)
//   combine_kernel     : hidden = hp + ffn[src*N + n] (fastdllm_v2_folded.py:361)
//
// All are latency/HBM bound.  Rows are walked in chunks of kChunkVec 16-byte vectors per
// lane whose loads are all issued before any is used, so a row costs a couple of memory
// round trips instead of one per vector.
#include "sf_kernels.cuh"

namespace sf {

constexpr int kChunkVec = 8;   // 16-byte vectors per lane in flight per chunk

// One CTA per block position n; warp b handles branch b's row r = b*N + n.
// With hp != nullptr the row is first rebuilt as hidden = T(hp + ffn[src*N+n]) and
// written to `hidden` (the previous layer's combine); otherwise `hidden` is read.
constexpr int kGateWarps = 8;   // warps per gate CTA; warp w takes branches w, w+8, ...

template <typename T>
__global__ void __launch_bounds__(32 * kGateWarps) gate_rows_kernel(GateRowsParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* rows_s = reinterpret_cast<T*>(smem_raw);  // [B1][D]
  constexpr int V = Elt<T>::kVec;
  constexpr int STEP = 32 * V * kChunkVec;
  const int n = blockIdx.x;
  const int wid = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int D = p.D, N = p.N, B1 = p.B1;
  T* hidden = reinterpret_cast<T*>(p.hidden);
  for (int b = wid; b < B1; b += kGateWarps) {
  const int64_t r = static_cast<int64_t>(b) * N + n;
  T* mine = rows_s + static_cast<size_t>(b) * D;

  float ss = 0.f;
  if (p.hp != nullptr) {
    const T* hp = reinterpret_cast<const T*>(p.hp) + r * D;
    int64_t s = p.src[r];
    if (s < 0 || s >= B1) { flag_error(p.err, SF_DEV_ERR_INDEX); s = b; }
    const T* ff = reinterpret_cast<const T*>(p.ffn) + (s * N + n) * D;
    for (int base = 0; base < D; base += STEP) {
      float a[kChunkVec][V], c[kChunkVec][V];
#pragma unroll
      for (int i = 0; i < kChunkVec; ++i) {
        const int d = base + (lane + 32 * i) * V;
        if (d < D) {
          load_vec<T>(hp + d, a[i]);
          load_vec<T>(ff + d, c[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < kChunkVec; ++i) {
        const int d = base + (lane + 32 * i) * V;
        if (d < D) {
#pragma unroll
          for (int k = 0; k < V; ++k) {
            a[i][k] = Elt<T>::rnd(a[i][k] + c[i][k]);
            ss = fmaf(a[i][k], a[i][k], ss);
          }
          store_vec<T>(hidden + r * D + d, a[i]);
          store_vec<T>(mine + d, a[i]);
        }
      }
    }
  } else {
    const T* x = hidden + r * D;
    for (int base = 0; base < D; base += STEP) {
      float a[kChunkVec][V];
#pragma unroll
      for (int i = 0; i < kChunkVec; ++i) {
        const int d = base + (lane + 32 * i) * V;
        if (d < D) load_vec<T>(x + d, a[i]);
      }
#pragma unroll
      for (int i = 0; i < kChunkVec; ++i) {
        const int d = base + (lane + 32 * i) * V;
        if (d < D) {
#pragma unroll
          for (int k = 0; k < V; ++k) ss = fmaf(a[i][k], a[i][k], ss);
          store_vec<T>(mine + d, a[i]);
        }
      }
    }
  }
  ss = warp_sum(ss);
  if (p.rstd && lane == 0) p.rstd[r] = 1.0f / sqrtf(ss / static_cast<float>(D) + p.eps);
  }
  if (p.rec == nullptr) return;   // combine-only use
  __syncthreads();

  for (int b = wid; b < B1; b += kGateWarps) {
  const int64_t r = static_cast<int64_t>(b) * N + n;
  const T* mine = rows_s + static_cast<size_t>(b) * D;
  int recompute = 1;
  int64_t par = 0;
  if (b > 0) {
    par = p.par_idx[b];
    if (par < 0 || par >= B1 || par == b) { flag_error(p.err, SF_DEV_ERR_INDEX); par = 0; }
    const T* pr = rows_s + static_cast<size_t>(par) * D;
    float dd = 0.f, pp = 0.f;
    for (int d = lane * V; d < D; d += 32 * V) {
      float a[V], c[V];
      load_vec<T>(mine + d, a);
      load_vec<T>(pr + d, c);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float diff = Elt<T>::rnd(a[i] - c[i]);   // x - x_par in the model dtype
        dd = fmaf(diff, diff, dd);
        pp = fmaf(c[i], c[i], pp);
      }
    }
    dd = warp_sum(dd);
    pp = warp_sum(pp);
    // norms returned in the model dtype, threshold delta * ||x_par|| rounded likewise
    const float dn = Elt<T>::rnd(sqrtf(dd));
    const float pn = Elt<T>::rnd(sqrtf(pp));
    const float thr = Elt<T>::rnd(pn * p.delta);
    recompute = dn > thr ? 1 : 0;
  }
  if (lane == 0) {
    p.rec[r] = static_cast<int8_t>(recompute);
    p.f[r] = recompute ? b : par;
  }
  }
}

// out = T(w * T(x * rs)) for one row, chunked (x may alias nothing written here).
template <typename T>
__device__ __forceinline__ void norm_row_write(const T* x, const T* lw, T* out, int D, int lane,
                                               float rs) {
  constexpr int V = Elt<T>::kVec;
  constexpr int STEP = 32 * V * kChunkVec;
  for (int base = 0; base < D; base += STEP) {
    float a[kChunkVec][V], g[kChunkVec][V];
#pragma unroll
    for (int i = 0; i < kChunkVec; ++i) {
      const int d = base + (lane + 32 * i) * V;
      if (d < D) {
        load_vec<T>(x + d, a[i]);
        load_vec<T>(lw + d, g[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < kChunkVec; ++i) {
      const int d = base + (lane + 32 * i) * V;
      if (d < D) {
#pragma unroll
        for (int k = 0; k < V; ++k) a[i][k] = g[i][k] * Elt<T>::rnd(a[i][k] * rs);
        store_vec<T>(out + d, a[i]);
      }
    }
  }
}

template <typename T>
__device__ __forceinline__ float row_sumsq_chunked(const T* x, int D, int lane) {
  constexpr int V = Elt<T>::kVec;
  constexpr int STEP = 32 * V * kChunkVec;
  float acc = 0.f;
  for (int base = 0; base < D; base += STEP) {
    float a[kChunkVec][V];
#pragma unroll
    for (int i = 0; i < kChunkVec; ++i) {
      const int d = base + (lane + 32 * i) * V;
      if (d < D) load_vec<T>(x + d, a[i]);
    }
#pragma unroll
    for (int i = 0; i < kChunkVec; ++i) {
      const int d = base + (lane + 32 * i) * V;
      if (d < D) {
#pragma unroll
        for (int k = 0; k < V; ++k) acc = fmaf(a[i][k], a[i][k], acc);
      }
    }
  }
  return warp_sum(acc);
}

// Block-wide exclusive scan of 0/1 flags (BN <= kMaxRows) -> slot per row.
// Every CTA recomputes it (BN bytes); CTA 0 writes the bookkeeping.
template <typename T>
__global__ void __launch_bounds__(256) compact_kernel(CompactParams p) {
  __shared__ int s_slot[kMaxRows];
  __shared__ int8_t s_f[kMaxRows];   // parent-or-self branch per flat row
  __shared__ int s_warp[8];
  const int BN = p.B1 * p.N;
  const int tid = threadIdx.x;
  constexpr int kPer = kMaxRows / 256;
  int flags[kPer];
  int local = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int r = tid * kPer + i;
    flags[i] = (r < BN) ? (p.rec[r] != 0) : 0;
    local += flags[i];
  }
  // warp-inclusive scan of per-thread totals
  const int lane = tid & 31, w = tid >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[w] = incl;
  __syncthreads();
  int wbase = 0, total = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < w) wbase += s_warp[i];
    total += s_warp[i];
  }
  int run = wbase + incl - local;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int r = tid * kPer + i;
    if (r < kMaxRows) s_slot[r] = flags[i] ? run : -1;
    // folded rows are listed in order too: slot = r - (recomputed rows before r)
    if (blockIdx.x == 0 && p.frows != nullptr && r < BN && !flags[i]) p.frows[r - run] = r;
    run += flags[i];
  }

  if (blockIdx.x == 0) {
    for (int r = tid; r < BN; r += blockDim.x) {
      int64_t fv = p.f[r];
      if (fv < 0 || fv >= p.B1) { flag_error(p.err, SF_DEV_ERR_INDEX); fv = 0; }
      s_f[r] = static_cast<int8_t>(fv);
    }
  }
  __syncthreads();

  if (blockIdx.x == 0) {
    if (tid == 0) *p.count = total;
    for (int r = tid; r < BN; r += blockDim.x) {
      const int s = s_slot[r];
      if (s >= 0 && s < p.bucket) p.rows[s] = r;
      // src: follow f (branch indices) to the recomputing ancestor
      const int n = r % p.N;
      int c = s_f[r];
      int hops = 0;
      while (hops <= p.B1) {
        const int nx = s_f[c * p.N + n];
        if (nx == c) break;
        c = nx;
        ++hops;
      }
      if (hops > p.B1) flag_error(p.err, SF_DEV_ERR_DEPTH);
      p.src[r] = c;
    }
    // per-branch segments: i-th recomputed row of branch b
    for (int b = tid; b < p.B1; b += blockDim.x) {
      int k = 0;
      for (int n = 0; n < p.N; ++n) {
        const int r = b * p.N + n;
        if (s_slot[r] >= 0) p.seg[static_cast<int64_t>(b) * p.N + (k++)] = r;
      }
      p.segcnt[b] = k;
    }
  }

  // normalised A operand of the QKV projection: xn[slot] = T(w * T(x * rstd))
  if (p.xn == nullptr) return;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  for (int r = blockIdx.x * (blockDim.x >> 5) + w; r < BN; r += warps_total) {
    const int s = s_slot[r];
    if (s < 0 || s >= p.bucket) continue;
    norm_row_write<T>(reinterpret_cast<const T*>(p.hidden) + static_cast<int64_t>(r) * p.D,
                      reinterpret_cast<const T*>(p.ln_w),
                      reinterpret_cast<T*>(p.xn) + static_cast<int64_t>(s) * p.D, p.D, lane,
                      p.rstd[r]);
  }
}

// src only (src_resolve_kernel): one thread per flat row.
__global__ void src_resolve_kernel(const int64_t* f, int64_t* src, int B1, int N, int* err) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B1 * N) return;
  const int n = r % N;
  int64_t c = f[r];
  int hops = 0;
  while (hops <= B1) {
    if (c < 0 || c >= B1) { flag_error(err, SF_DEV_ERR_INDEX); c = 0; break; }
    const int64_t nx = f[c * N + n];
    if (nx == c) break;
    c = nx;
    ++hops;
  }
  if (hops > B1) flag_error(err, SF_DEV_ERR_DEPTH);
  src[r] = c;
}

// out[i] = T(w * T(x[row(i)] * rstd)), row(i) = rows ? rows[i] : i, for i < min(*count, n).
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(RmsRowsParams p) {
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int n = p.n;
  if (p.count) n = min(n, *p.count);
  if (w >= n) return;
  int64_t row = p.rows ? p.rows[w] : w;
  if (row < 0 || row >= p.n_src) { flag_error(p.err, SF_DEV_ERR_INDEX); return; }
  const T* x = reinterpret_cast<const T*>(p.x) + row * p.D;
  const float ss = row_sumsq_chunked<T>(x, p.D, lane);
  const float rs = 1.0f / sqrtf(ss / static_cast<float>(p.D) + p.eps);
  if (p.rstd && lane == 0) p.rstd[w] = rs;
  norm_row_write<T>(x, reinterpret_cast<const T*>(p.w),
                    reinterpret_cast<T*>(p.out) + static_cast<int64_t>(w) * p.D, p.D, lane, rs);
}

// hidden[r] = T(hp[r] + ffn[src[r]*N + n]); one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) combine_kernel(const T* hp, const T* ffn,
                                                     const int64_t* src, T* hidden, int B1,
                                                     int N, int D, int* err) {
  constexpr int V = Elt<T>::kVec;
  constexpr int STEP = 32 * V * kChunkVec;
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= B1 * N) return;
  const int n = r % N;
  int64_t s = src[r];
  if (s < 0 || s >= B1) { flag_error(err, SF_DEV_ERR_INDEX); s = r / N; }
  const T* a = hp + static_cast<int64_t>(r) * D;
  const T* c = ffn + (s * N + n) * D;
  T* o = hidden + static_cast<int64_t>(r) * D;
  for (int base = 0; base < D; base += STEP) {
    float x[kChunkVec][V], y[kChunkVec][V];
#pragma unroll
    for (int i = 0; i < kChunkVec; ++i) {
      const int d = base + (lane + 32 * i) * V;
      if (d < D) {
        load_vec<T>(a + d, x[i]);
        load_vec<T>(c + d, y[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < kChunkVec; ++i) {
      const int d = base + (lane + 32 * i) * V;
      if (d < D) {
#pragma unroll
        for (int k = 0; k < V; ++k) x[i][k] = x[i][k] + y[i][k];
        store_vec<T>(o + d, x[i]);
      }
    }
  }
}

// ------------------------------------------------------------------------ launchers
template <typename T>
static cudaError_t launch_gate_rows_t(const GateRowsParams& p, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(p.B1) * p.D * sizeof(T);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(gate_rows_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kMaxGateSmem);
    configured = true;
  }
  gate_rows_kernel<T><<<p.N, 32 * std::min(p.B1, kGateWarps), smem, st>>>(p);
  return launched();
}
cudaError_t launch_gate_rows(int dtype, const GateRowsParams& p, cudaStream_t st) {
  return dtype == BF16 ? launch_gate_rows_t<__nv_bfloat16>(p, st) : launch_gate_rows_t<float>(p, st);
}

cudaError_t launch_compact(int dtype, const CompactParams& p, cudaStream_t st) {
  const int BN = p.B1 * p.N;
  const int grid = p.xn ? (BN + 7) / 8 : 1;
  if (dtype == BF16) compact_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p);
  else compact_kernel<float><<<grid, 256, 0, st>>>(p);
  return launched();
}

cudaError_t launch_src_resolve(const int64_t* f, int64_t* src, int B1, int N, int* err,
                               cudaStream_t st) {
  const int BN = B1 * N;
  src_resolve_kernel<<<(BN + 127) / 128, 128, 0, st>>>(f, src, B1, N, err);
  return launched();
}

cudaError_t launch_rmsnorm_rows(int dtype, const RmsRowsParams& p, cudaStream_t st) {
  const int grid = (p.n + 7) / 8;
  if (grid == 0) return cudaSuccess;
  if (dtype == BF16) rmsnorm_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p);
  else rmsnorm_rows_kernel<float><<<grid, 256, 0, st>>>(p);
  return launched();
}

cudaError_t launch_combine(int dtype, const void* hp, const void* ffn, const int64_t* src,
                           void* hidden, int B1, int N, int D, int* err, cudaStream_t st) {
  const int grid = (B1 * N + 7) / 8;
  if (dtype == BF16)
    combine_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(hp), static_cast<const __nv_bfloat16*>(ffn), src,
        static_cast<__nv_bfloat16*>(hidden), B1, N, D, err);
  else
    combine_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(hp),
                                                static_cast<const float*>(ffn), src,
                                                static_cast<float*>(hidden), B1, N, D, err);
  return launched();
}

}  // namespace sf
