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

// Same output, one CTA per row: every element of the row is loaded once into registers
// (one memory round trip), the sum of squares is a block reduction, and the row is
// normalised from the registers (D <= 256 * kVec * MAXV).
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) rmsnorm_cta_kernel(RmsRowsParams p) {
  constexpr int V = Elt<T>::kVec;
  __shared__ float s_part[8];
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  int n = p.n;
  if (p.count) n = min(n, *p.count);
  if (i >= n) return;
  const int64_t row = p.rows ? p.rows[i] : i;
  if (row < 0 || row >= p.n_src) {
    if (threadIdx.x == 0) flag_error(p.err, SF_DEV_ERR_INDEX);
    return;
  }
  const T* x = reinterpret_cast<const T*>(p.x) + row * p.D;
  const T* w = reinterpret_cast<const T*>(p.w);
  float a[MAXV][V], g[MAXV][V];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < MAXV; ++u) {
    const int d = (threadIdx.x + 256 * u) * V;
    if (d < p.D) {
      load_vec<T>(x + d, a[u]);
      load_vec<T>(w + d, g[u]);
    }
  }
#pragma unroll
  for (int u = 0; u < MAXV; ++u) {
    const int d = (threadIdx.x + 256 * u) * V;
    if (d < p.D) {
#pragma unroll
      for (int k = 0; k < V; ++k) ss = fmaf(a[u][k], a[u][k], ss);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) tot += s_part[k];
  const float rs = 1.0f / sqrtf(tot / static_cast<float>(p.D) + p.eps);
  if (p.rstd && threadIdx.x == 0) p.rstd[i] = rs;
  T* out = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(i) * p.D;
#pragma unroll
  for (int u = 0; u < MAXV; ++u) {
    const int d = (threadIdx.x + 256 * u) * V;
    if (d < p.D) {
#pragma unroll
      for (int k = 0; k < V; ++k) a[u][k] = g[u][k] * Elt<T>::rnd(a[u][k] * rs);
      store_vec<T>(out + d, a[u]);
    }
  }
}

// hidden[r] = T(hp[r] + ffn[src[r]*N + n]); one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) combine_kernel(const T* hp, const T* ffn,
                                                     const int64_t* src, T* hidden, int B1,
                                                     int N, int D, int* err) {
  constexpr int V = Elt<T>::kVec;
  constexpr int STEP = 32 * V * kChunkVec;
  pdl_trigger();
  pdl_wait();
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

// ------------------------------------------------------------------------ parent map
// par_idx[i] for the B1 branches of a verify block (fastdllm_v2_folded.py:55-75): the
// first branch j whose set of positions differing from the main branch (row 0) is a
// subset of branch i's with exactly one element fewer; 0 (the main branch) otherwise.
// One CTA; runs on the device so the forward needs no host round trip before launch.
__global__ void __launch_bounds__(256) parent_map_kernel(const int64_t* ids, int B1, int N,
                                                         int64_t* par_idx) {
  __shared__ uint8_t diff[kMaxRows];
  __shared__ int cnt[kMaxBranches];
  __shared__ uint8_t esc[kMaxBranches * kMaxBranches];   // esc[i][j]: j differs where i does not
  const int BN = B1 * N;
  for (int r = threadIdx.x; r < BN; r += blockDim.x) diff[r] = ids[r] != ids[r % N] ? 1 : 0;
  __syncthreads();
  for (int i = threadIdx.x; i < B1; i += blockDim.x) {
    int c = 0;
    for (int n = 0; n < N; ++n) c += diff[i * N + n];
    cnt[i] = c;
  }
  for (int q = threadIdx.x; q < B1 * B1; q += blockDim.x) {
    const int i = q / B1, j = q % B1;
    uint8_t e = 0;
    for (int n = 0; n < N && !e; ++n) e = diff[j * N + n] && !diff[i * N + n];
    esc[q] = e;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < B1; i += blockDim.x) {
    int par = 0;
    if (i > 0) {
      for (int j = 0; j < B1; ++j) {
        if (j != i && cnt[j] == cnt[i] - 1 && !esc[i * B1 + j]) {
          par = j;
          break;
        }
      }
    }
    par_idx[i] = par;
  }
}

cudaError_t launch_parent_map(const int64_t* ids, int B1, int N, int64_t* par_idx,
                              cudaStream_t st) {
  if (B1 < 1 || B1 > kMaxBranches || N < 1 || B1 * N > kMaxRows) return cudaErrorInvalidValue;
  parent_map_kernel<<<1, 256, 0, st>>>(ids, B1, N, par_idx);
  return launched();
}

// ------------------------------------------------------------------------ fused gate
// gate_compact_kernel: the previous layer's combine, the delta gate, the compaction and
// the normalised QKV input of one layer in a single cooperative launch.
//   phase 1  CTA (n, s) owns position n and D-slice s of every branch row r = b*N + n:
//            hidden = T(hp + ffn[src*N+n]) (or the input rows at layer 0) into shared
//            memory, and its slice of sum(x^2), sum(T(x - x_par)^2), sum(x_par^2);
//   barrier  every CTA's partial sums are published (bounded spin on a counter);
//   phase 2  every CTA adds the S slices of every row in slice order (deterministic) and
//            takes the gate decisions (residual_delta_gate_kernel, triton_kernels.py:
//            199-241), the slot scan and, in CTA 0, rows / count / src / segments;
//   phase 3  each CTA writes xn[slot] = T(w * T(x * rstd)) for its own slice of the
//            recomputed rows straight from shared memory (triton_kernels.py:30-87 input).
// The slices keep ~N*S CTAs busy on the loads where one CTA per position left most SMs
// idle, and the two launches of gate + compaction become one.
template <typename T>
__global__ void __launch_bounds__(256) gate_compact_kernel(GateCompactParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* rows_s = reinterpret_cast<T*>(smem_raw);   // [B1][slice]
  __shared__ int s_slot[kMaxRows];
  __shared__ int8_t s_rec[kMaxRows];
  __shared__ int8_t s_f[kMaxRows];
  __shared__ float s_rstd[kMaxBranches];
  __shared__ int s_warp[8];
  constexpr int V = Elt<T>::kVec;
  constexpr int CV = 4;                          // vectors per lane in flight
  pdl_trigger();
  pdl_wait();
  const int n = blockIdx.x / p.S, sl = blockIdx.x % p.S;
  const int d0 = sl * p.slice;
  const int len = min(p.D, d0 + p.slice) - d0;   // a multiple of V
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B1 = p.B1, N = p.N, D = p.D, BN = B1 * N;
  T* hidden = reinterpret_cast<T*>(p.hidden);

  // ---- phase 1: rows of position n, slice [d0, d0 + len)
  for (int b = warp; b < B1; b += 8) {
    const int64_t r = static_cast<int64_t>(b) * N + n;
    T* mine = rows_s + static_cast<size_t>(b) * p.slice;
    float ss = 0.f;
    const T* hpr = nullptr;
    const T* ffr = nullptr;
    if (p.hp != nullptr) {
      int64_t s = p.src_prev[r];
      if (s < 0 || s >= B1) { flag_error(p.err, SF_DEV_ERR_INDEX); s = b; }
      hpr = reinterpret_cast<const T*>(p.hp) + r * D + d0;
      ffr = reinterpret_cast<const T*>(p.ffn) + (s * N + n) * D + d0;
    }
    for (int base = 0; base < len; base += 32 * V * CV) {
      float a[CV][V], c[CV][V];
#pragma unroll
      for (int i = 0; i < CV; ++i) {
        const int d = base + (lane + 32 * i) * V;
        if (d < len) {
          if (hpr != nullptr) {
            load_vec<T>(hpr + d, a[i]);
            load_vec<T>(ffr + d, c[i]);
          } else {
            load_vec<T>(hidden + r * D + d0 + d, a[i]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < CV; ++i) {
        const int d = base + (lane + 32 * i) * V;
        if (d < len) {
          if (hpr != nullptr) {
#pragma unroll
            for (int k = 0; k < V; ++k) a[i][k] = Elt<T>::rnd(a[i][k] + c[i][k]);
            store_vec<T>(hidden + r * D + d0 + d, a[i]);
          }
#pragma unroll
          for (int k = 0; k < V; ++k) ss = fmaf(a[i][k], a[i][k], ss);
          store_vec<T>(mine + d, a[i]);
        }
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) p.red[(r * p.S + sl) * 4] = ss;
  }
  __syncthreads();
  for (int b = warp; b < B1; b += 8) {
    const int64_t r = static_cast<int64_t>(b) * N + n;
    float dd = 0.f, pp = 0.f;
    if (b > 0) {
      int64_t par = p.par_idx[b];
      if (par < 0 || par >= B1 || par == b) { flag_error(p.err, SF_DEV_ERR_INDEX); par = 0; }
      const T* mine = rows_s + static_cast<size_t>(b) * p.slice;
      const T* pr = rows_s + static_cast<size_t>(par) * p.slice;
      for (int d = lane * V; d < len; d += 32 * V) {
        float a[V], c[V];
        load_vec<T>(mine + d, a);
        load_vec<T>(pr + d, c);
#pragma unroll
        for (int k = 0; k < V; ++k) {
          const float diff = Elt<T>::rnd(a[k] - c[k]);   // x - x_par in the model dtype
          dd = fmaf(diff, diff, dd);
          pp = fmaf(c[k], c[k], pp);
        }
      }
      dd = warp_sum(dd);
      pp = warp_sum(pp);
    }
    if (lane == 0) {
      p.red[(r * p.S + sl) * 4 + 1] = dd;
      p.red[(r * p.S + sl) * 4 + 2] = pp;
    }
  }

  // ---- grid barrier: every CTA's partial sums are visible
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    atomicAdd(p.bar, 1u);
    const uint64_t t0 = globaltimer();
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.bar) : "memory");
      if (static_cast<int>(v - p.bar_target) >= 0) break;
      if (globaltimer() - t0 > kWaitNs) { flag_error(p.err, SF_DEV_ERR_TIMEOUT); break; }
    }
  }
  __syncthreads();

  // ---- phase 2: decisions of every row (slice sums in slice order), then the scan
  for (int r = tid; r < BN; r += 256) {
    const int b = r / N;
    float ss = 0.f, dd = 0.f, pp = 0.f;
    for (int s = 0; s < p.S; ++s) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(p.red + (static_cast<int64_t>(r) * p.S + s) * 4));
      ss += v.x;
      dd += v.y;
      pp += v.z;
    }
    int recompute = 1;
    int fv = b;
    if (b > 0) {
      // norms returned in the model dtype, threshold delta * ||x_par|| rounded likewise
      const float dn = Elt<T>::rnd(sqrtf(dd));
      const float pn = Elt<T>::rnd(sqrtf(pp));
      const float thr = Elt<T>::rnd(pn * p.delta);
      recompute = dn > thr ? 1 : 0;
      if (!recompute) {
        int64_t par = p.par_idx[b];
        if (par < 0 || par >= B1) par = 0;
        fv = static_cast<int>(par);
      }
    }
    s_rec[r] = static_cast<int8_t>(recompute);
    s_f[r] = static_cast<int8_t>(fv);
    if (r % N == n) s_rstd[b] = 1.0f / sqrtf(ss / static_cast<float>(D) + p.eps);
  }
  __syncthreads();
  constexpr int kPer = kMaxRows / 256;
  int flags[kPer];
  int local = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int r = tid * kPer + i;
    flags[i] = r < BN ? s_rec[r] : 0;
    local += flags[i];
  }
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int run = incl - local, total = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < warp) run += s_warp[i];
    total += s_warp[i];
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int r = tid * kPer + i;
    if (r < kMaxRows) s_slot[r] = flags[i] ? run : -1;
    run += flags[i];
  }
  __syncthreads();

  if (blockIdx.x == 0) {
    if (tid == 0) *p.count = total;
    for (int r = tid; r < BN; r += 256) {
      p.rec[r] = s_rec[r];
      p.f[r] = s_f[r];
      const int s = s_slot[r];
      if (s >= 0 && s < p.bucket) p.rows[s] = r;
      // src: follow f (branch indices) to the recomputing ancestor
      const int nn = r % N;
      int c = s_f[r];
      int hops = 0;
      while (hops <= B1) {
        const int nx = s_f[c * N + nn];
        if (nx == c) break;
        c = nx;
        ++hops;
      }
      if (hops > B1) flag_error(p.err, SF_DEV_ERR_DEPTH);
      p.src[r] = c;
    }
    for (int b = tid; b < B1; b += 256) {
      int k = 0;
      for (int nn = 0; nn < N; ++nn) {
        const int r = b * N + nn;
        if (s_slot[r] >= 0) p.seg[static_cast<int64_t>(b) * N + (k++)] = r;
      }
      p.segcnt[b] = k;
    }
  }

  // ---- phase 3: normalised QKV input of this CTA's recomputed rows
  const T* lw = reinterpret_cast<const T*>(p.ln_w) + d0;
  for (int b = warp; b < B1; b += 8) {
    const int r = b * N + n;
    const int s = s_slot[r];
    if (s < 0 || s >= p.bucket) continue;
    const T* mine = rows_s + static_cast<size_t>(b) * p.slice;
    T* out = reinterpret_cast<T*>(p.xn) + static_cast<int64_t>(s) * D + d0;
    const float rs = s_rstd[b];
    for (int d = lane * V; d < len; d += 32 * V) {
      float a[V], g[V];
      load_vec<T>(mine + d, a);
      load_vec<T>(lw + d, g);
#pragma unroll
      for (int k = 0; k < V; ++k) a[k] = g[k] * Elt<T>::rnd(a[k] * rs);
      store_vec<T>(out + d, a);
    }
  }
}

// D-slices per position: about one CTA per SM in all, at least 64 elements per slice;
// the slice is a multiple of 8 elements (16-byte vectors)
static int gate_slice(int N, int D) {
  int S = std::max(1, 148 / std::max(1, N));
  S = std::min(S, std::max(1, D / 64));
  return ((D + S - 1) / S + 7) / 8 * 8;
}
int gate_compact_slices(int N, int D) {
  const int slice = gate_slice(N, D);
  return (D + slice - 1) / slice;
}

// ------------------------------------------------------------------------ launchers
template <typename T>
static cudaError_t launch_gate_compact_t(GateCompactParams p, cudaStream_t st) {
  p.slice = gate_slice(p.N, p.D);
  p.S = gate_compact_slices(p.N, p.D);
  const size_t smem = static_cast<size_t>(p.B1) * p.slice * sizeof(T);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gate_compact_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  if (smem > 160 * 1024) return cudaErrorInvalidValue;
  // the CTAs meet at a grid barrier: all must be resident at once
  cudaError_t e = launch_ex(gate_compact_kernel<T>, dim3(p.N * p.S), dim3(256), smem, st, true, p);
  if (e != cudaSuccess) return e;
  return launched();
}

cudaError_t launch_gate_compact(int dtype, const GateCompactParams& p, cudaStream_t st) {
  if (p.B1 > kMaxBranches || p.B1 * p.N > kMaxRows || p.D % 8 != 0) return cudaErrorInvalidValue;
  return dtype == BF16 ? launch_gate_compact_t<__nv_bfloat16>(p, st)
                       : launch_gate_compact_t<float>(p, st);
}


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
  if (p.n <= 0) return cudaSuccess;
  const int vec = dtype == BF16 ? 8 : 4;
  if (p.D % vec == 0 && p.D <= 256 * vec * 4) {
    const cudaError_t e =
        dtype == BF16 ? launch_ex(rmsnorm_cta_kernel<__nv_bfloat16, 4>, dim3(p.n), dim3(256), 0, st, false, p)
                      : launch_ex(rmsnorm_cta_kernel<float, 4>, dim3(p.n), dim3(256), 0, st, false, p);
    if (e != cudaSuccess) return e;
    return launched();
  }
  const int grid = (p.n + 7) / 8;
  if (dtype == BF16) rmsnorm_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p);
  else rmsnorm_rows_kernel<float><<<grid, 256, 0, st>>>(p);
  return launched();
}

cudaError_t launch_combine(int dtype, const void* hp, const void* ffn, const int64_t* src,
                           void* hidden, int B1, int N, int D, int* err, cudaStream_t st) {
  const int grid = (B1 * N + 7) / 8;
  cudaError_t e;
  if (dtype == BF16)
    e = launch_ex(combine_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, false,
                  static_cast<const __nv_bfloat16*>(hp), static_cast<const __nv_bfloat16*>(ffn), src,
                  static_cast<__nv_bfloat16*>(hidden), B1, N, D, err);
  else
    e = launch_ex(combine_kernel<float>, dim3(grid), dim3(256), 0, st, false,
                  static_cast<const float*>(hp), static_cast<const float*>(ffn), src,
                  static_cast<float*>(hidden), B1, N, D, err);
  if (e != cudaSuccess) return e;
  return launched();
}

}  // namespace sf
