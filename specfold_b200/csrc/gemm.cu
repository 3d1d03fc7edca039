// Weight-streaming GEMMs of the folded verify forward with fused epilogues.
//
// Shape: acc[j][f] = sum_k X[j][k] * W[f][k] for a handful of activation rows j (the
// recomputed rows, <= B1*N) against a large weight matrix W [n_out, K].  At the model
// shapes this is HBM-bound on the weight stream, so the bf16 path is a tcgen05 kernel
// in "swap-AB" form: 128 weight rows are the MMA's M operand, the activation rows its
// N operand (N = rows rounded up to 16), both staged in shared memory by TMA in the
// 128-byte swizzle layout, the fp32 accumulator in TMEM.  Few output tiles (QKV,
// o_proj, down) are split along K across CTAs; the last CTA of a tile sums the
// partials in split order (deterministic) and runs the epilogue.
//
// Epilogues (EpiKind) reproduce the rounding points of the PyTorch folded forward:
//   QKV     F.linear + bias rounded to the model dtype, then q*c + rot(q)*s with every
//           op rounded (fastdllm_v2_folded.py:153-157; triton_kernels.py:65-87)
//   RESID   x + T(O @ Wo^T) (fastdllm_v2_folded.py:207-208, :351)
//   SWIGLU  T(silu(T(g))) * T(u) (fastdllm_v2_folded.py:216; triton_kernels.py:133)
//   SCATTER ffn_buf[rows[j]] = T(acc) (triton_kernels.py:171-173)
//   LOGITS  lm_head with the Fast-dLLM shift (fastdllm_v2_generation.py:121-126)
//
// fp32 models use a SIMT kernel (tcgen05 has no fp32-exact kind) followed by the same
// epilogue as a separate pass.
#include <cudaTypedefs.h>

#include <mutex>

#include "sf_kernels.cuh"

namespace sf {

// ------------------------------------------------------------------ epilogue core
template <typename T>
__device__ __forceinline__ float ldf(const void* p, int64_t i) {
  return Elt<T>::to_f(reinterpret_cast<const T*>(p)[i]);
}
template <typename T>
__device__ __forceinline__ void stf(void* p, int64_t i, float v) {
  reinterpret_cast<T*>(p)[i] = Elt<T>::from_f(v);
}

// partner feature (natural index) of f for the paired epilogues
__device__ __forceinline__ int epi_partner(const EpiParams& e, int f) {
  if (e.kind == EPI_QKV) return f ^ (e.hd >> 1);
  if (e.kind == EPI_SWIGLU) return f < e.inter ? f + e.inter : f - e.inter;
  return f;
}
// does feature f produce an output (SWIGLU: only the gate half)
__device__ __forceinline__ bool epi_emits(const EpiParams& e, int f) {
  return e.kind != EPI_SWIGLU || f < e.inter;
}

// v = acc for (row j, feature f), vp = acc of the partner feature.
template <typename T>
__device__ __forceinline__ void epi_apply(const EpiParams& e, int j, int f, float v, float vp) {
  switch (e.kind) {
    case EPI_RAW:
      reinterpret_cast<float*>(e.out)[static_cast<int64_t>(j) * e.ld_out + f] = v;
      break;
    case EPI_QKV: {
      const int fp = f ^ (e.hd >> 1);
      float x = v, xp = vp;
      if (e.bias) {
        x = __fadd_rn(x, ldf<T>(e.bias, f));
        xp = __fadd_rn(xp, ldf<T>(e.bias, fp));
      }
      x = Elt<T>::rnd(x);
      xp = Elt<T>::rnd(xp);
      const int64_t row = e.rows[j];
      const int n = static_cast<int>(row % e.N);
      float out = x;
      if (f < e.q_dim + e.kv_dim) {  // q and k heads: RoPE (rotate-half)
        const int d = f % e.hd;
        const float c = ldf<T>(e.cos, static_cast<int64_t>(n) * e.hd + d);
        const float s = ldf<T>(e.sin, static_cast<int64_t>(n) * e.hd + d);
        const float rot = d < (e.hd >> 1) ? -xp : xp;
        out = Elt<T>::rnd(__fadd_rn(Elt<T>::rnd(__fmul_rn(x, c)), Elt<T>::rnd(__fmul_rn(rot, s))));
        if (f < e.q_dim && e.q_scale) out = Elt<T>::rnd(__fmul_rn(out, Elt<T>::rnd(e.q_scale[n])));
      }
      if (f < e.q_dim)
        stf<T>(e.out, row * e.q_dim + f, out);
      else
        stf<T>(e.out2, row * (2 * e.kv_dim) + (f - e.q_dim), out);
      break;
    }
    case EPI_RESID: {
      const int64_t i = static_cast<int64_t>(j) * e.ld_out + f;
      stf<T>(e.out, i, __fadd_rn(ldf<T>(e.resid, i), Elt<T>::rnd(v)));
      break;
    }
    case EPI_SWIGLU: {
      const float g = Elt<T>::rnd(v), u = Elt<T>::rnd(vp);
      const float s = Elt<T>::rnd(g / (1.0f + expf(-g)));
      stf<T>(e.out, static_cast<int64_t>(j) * e.inter + f, __fmul_rn(s, u));
      break;
    }
    case EPI_SCATTER:
      stf<T>(e.out, e.rows[j] * e.ld_out + f, v);
      break;
    case EPI_LOGITS: {
      const int n = j % e.N;
      const int64_t b = j / e.N;
      if (e.shift) {
        if (n + 1 < e.N) stf<T>(e.out, (b * e.N + n + 1) * e.ld_out + f, v);
        if (n == 0) stf<T>(e.out, (b * e.N) * e.ld_out + f, v);
      } else {
        stf<T>(e.out, static_cast<int64_t>(j) * e.ld_out + f, v);
      }
      break;
    }
    default:
      break;
  }
}

// ------------------------------------------------------------------ SIMT path
// raw[j][f] = sum_k X[j][k] W[f][k] (fp32), 64x64 tile, 256 threads, 4x4 per thread.
template <typename T>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const T* __restrict__ X,
                                                        const T* __restrict__ W,
                                                        const T* __restrict__ W2, int n_out,
                                                        int K, int rows_cap,
                                                        const int32_t* count, int inter,
                                                        float* __restrict__ raw) {
  constexpr int BM = 64, BF = 64, BK = 16;
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BF + 4];
  int rows = rows_cap;
  if (count) rows = min(rows, *count);
  const int j0 = blockIdx.y * BM, f0 = blockIdx.x * BF;
  if (j0 >= rows) return;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      const int r = i / BK, k = i % BK;
      const int j = j0 + r, kk = k0 + k;
      xs[k][r] = (j < rows && kk < K) ? Elt<T>::to_f(X[static_cast<int64_t>(j) * K + kk]) : 0.f;
      const int f = f0 + r;
      float wv = 0.f;
      if (f < n_out && kk < K) {
        if (W2 != nullptr && f >= inter)
          wv = Elt<T>::to_f(W2[static_cast<int64_t>(f - inter) * K + kk]);
        else
          wv = Elt<T>::to_f(W[static_cast<int64_t>(f) * K + kk]);
      }
      ws[k][r] = wv;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[k][ty * 4 + i];
        b[i] = ws[k][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[i][q] = fmaf(a[i], b[q], acc[i][q]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = j0 + ty * 4 + i;
    if (j >= rows) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int f = f0 + tx * 4 + q;
      if (f < n_out) raw[static_cast<int64_t>(j) * n_out + f] = acc[i][q];
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) epilogue_kernel(const float* __restrict__ raw, int n_out,
                                                       int rows_cap, const int32_t* count,
                                                       EpiParams e) {
  int rows = rows_cap;
  if (count) rows = min(rows, *count);
  const int64_t total = static_cast<int64_t>(rows) * n_out;
  for (int64_t i = blockIdx.x * 256ll + threadIdx.x; i < total; i += 256ll * gridDim.x) {
    const int j = static_cast<int>(i / n_out), f = static_cast<int>(i % n_out);
    if (!epi_emits(e, f)) continue;
    const int fp = epi_partner(e, f);
    const float v = raw[static_cast<int64_t>(j) * n_out + f];
    const float vp = (fp >= 0 && fp < n_out) ? raw[static_cast<int64_t>(j) * n_out + fp] : 0.f;
    epi_apply<T>(e, j, f, v, vp);
  }
}

// ------------------------------------------------------------------ tcgen05 path
//
// One CTA of 192 threads: warp 0 issues TMA loads, warp 1 owns TMEM and issues the
// MMAs, warps 2-5 (one per TMEM lane quarter) run the epilogue.  CTAs are persistent
// over "units" (tile, split); with more than one unit per CTA the accumulator is
// double-buffered in TMEM so the epilogue of one unit overlaps the next unit's
// mainloop.  Split-K units of a tile run concurrently (cooperative launch): each
// publishes fp32 partials, waits (bounded) until all splits of its tile have, then
// reduces its own slice of rows in split order -- deterministic and parallel.
constexpr int kTcThreads = 192;
constexpr int kTileF = 128;                      // weight rows per tile (MMA M)
constexpr int kBK = 64;                          // K per stage: one 128-byte swizzle row
constexpr int kMaxPassRows = 256;                // MMA N limit
constexpr int kWBytes = kTileF * kBK * 2;        // 16 KB
constexpr int kXBoxRows = 64;
constexpr int kXBoxBytes = kXBoxRows * kBK * 2;  // 8 KB
constexpr int kChunk = 32;                       // rows per epilogue chunk
constexpr int kTileLd = kTileF + 4;              // padded fp32 row of the transposed chunk
constexpr int kTileTBytes = kChunk * kTileLd * 4;
// Workspace: split-K tile counters (arrivals, departures) at offset 0 -- a fixed place
// that no other data overlaps, kept zero between launches -- then fp32 partials.
constexpr size_t kCounterBytes = 16384;
constexpr int kMaxCounterTiles = static_cast<int>(kCounterBytes / 8);

struct TcParams {
  int n_out, K, rows_cap;
  const int32_t* count;
  int mode;            // 0: 128-row tiles of W; 1: SWIGLU, 64 gate + 64 up rows per tile
  int inter;
  int n_tiles, splits, kb_total, kb_per_split, n_units;
  int stages, x_boxes_max, double_buf;
  float* partial;      // [splits][rows_cap][n_out] when splits > 1
  int* counters;       // [2 * n_tiles]
  EpiParams epi;
  int* err;
};

// natural feature index of tile-local weight row l, or -1 past the end
__device__ __forceinline__ int tc_feature(const TcParams& p, int tile, int l) {
  if (p.mode == 1) {
    const int g = tile * 64 + (l & 63);
    if (g >= p.inter) return -1;
    return l < 64 ? g : p.inter + g;
  }
  const int f = tile * kTileF + l;
  return f < p.n_out ? f : -1;
}

template <typename T>
__device__ __forceinline__ void ld8(const void* base, int64_t i, float* v) {
  load_vec<T>(reinterpret_cast<const T*>(base) + i, v);
  if (Elt<T>::kVec == 4) load_vec<T>(reinterpret_cast<const T*>(base) + i + 4, v + 4);
}
template <typename T>
__device__ __forceinline__ void st8(void* base, int64_t i, const float* v) {
  store_vec<T>(reinterpret_cast<T*>(base) + i, v);
  if (Elt<T>::kVec == 4) store_vec<T>(reinterpret_cast<T*>(base) + i + 4, v + 4);
}

// Epilogue of 8 consecutive tile-local weight rows l0..l0+7 for activation row j:
// v = their accumulators, vp = the partner rows' (RoPE pair / SwiGLU up half).
__device__ __forceinline__ void epi_group8(const TcParams& p, int tile, int j, int l0,
                                           const float* v, const float* vp) {
  using T = __nv_bfloat16;
  const EpiParams& e = p.epi;
  const int f0 = tc_feature(p, tile, l0);
  if (f0 < 0) return;
  float o[8];
  switch (e.kind) {
    case EPI_RAW:
      store_vec<float>(reinterpret_cast<float*>(e.out) + static_cast<int64_t>(j) * e.ld_out + f0, v);
      store_vec<float>(reinterpret_cast<float*>(e.out) + static_cast<int64_t>(j) * e.ld_out + f0 + 4, v + 4);
      return;
    case EPI_QKV: {
      const int64_t row = e.rows[j];
      const int n = static_cast<int>(row % e.N);
      const int fp0 = f0 ^ (e.hd >> 1);
      float x[8], xp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) { x[i] = v[i]; xp[i] = vp[i]; }
      if (e.bias) {
        float b[8], bp[8];
        ld8<T>(e.bias, f0, b);
        ld8<T>(e.bias, fp0, bp);
#pragma unroll
        for (int i = 0; i < 8; ++i) { x[i] = __fadd_rn(x[i], b[i]); xp[i] = __fadd_rn(xp[i], bp[i]); }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) { o[i] = Elt<T>::rnd(x[i]); xp[i] = Elt<T>::rnd(xp[i]); }
      if (f0 < e.q_dim + e.kv_dim) {
        const int d0 = f0 % e.hd;
        float c[8], s[8];
        ld8<T>(e.cos, static_cast<int64_t>(n) * e.hd + d0, c);
        ld8<T>(e.sin, static_cast<int64_t>(n) * e.hd + d0, s);
        const bool first = d0 < (e.hd >> 1);
        const float qs = (f0 < e.q_dim && e.q_scale) ? Elt<T>::rnd(e.q_scale[n]) : 1.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float rot = first ? -xp[i] : xp[i];
          float r = Elt<T>::rnd(__fadd_rn(Elt<T>::rnd(__fmul_rn(o[i], c[i])),
                                          Elt<T>::rnd(__fmul_rn(rot, s[i]))));
          if (f0 < e.q_dim && e.q_scale) r = Elt<T>::rnd(__fmul_rn(r, qs));
          o[i] = r;
        }
      }
      if (f0 < e.q_dim) {
        st8<T>(e.out, row * e.q_dim + f0, o);
        if (e.q_comp) {   // query-major copy per kv head for the tensor-core attention
          const int G = e.q_dim / e.kv_dim;
          const int h = f0 / e.hd;
          st8<T>(e.q_comp,
                 ((static_cast<int64_t>(h / G) * e.q_comp_rows + static_cast<int64_t>(j) * G +
                   h % G) * e.hd) + f0 % e.hd, o);
        }
      } else {
        st8<T>(e.out2, row * (2 * e.kv_dim) + (f0 - e.q_dim), o);
      }
      return;
    }
    case EPI_RESID: {
      const int64_t i0 = static_cast<int64_t>(j) * e.ld_out + f0;
      float r[8];
      ld8<T>(e.resid, i0, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __fadd_rn(r[i], Elt<T>::rnd(v[i]));
      st8<T>(e.out, i0, o);
      return;
    }
    case EPI_SWIGLU: {
      if (f0 >= e.inter) return;   // up half: consumed by its gate partner
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float g = Elt<T>::rnd(v[i]), u = Elt<T>::rnd(vp[i]);
        o[i] = __fmul_rn(Elt<T>::rnd(g / (1.0f + expf(-g))), u);
      }
      st8<T>(e.out, static_cast<int64_t>(j) * e.inter + f0, o);
      return;
    }
    case EPI_SCATTER:
      st8<T>(e.out, e.rows[j] * e.ld_out + f0, v);
      return;
    case EPI_LOGITS: {
      const int n = j % e.N;
      const int64_t b = j / e.N;
      if (e.shift) {
        if (n + 1 < e.N) st8<T>(e.out, (b * e.N + n + 1) * e.ld_out + f0, v);
        if (n == 0) st8<T>(e.out, (b * e.N) * e.ld_out + f0, v);
      } else {
        st8<T>(e.out, static_cast<int64_t>(j) * e.ld_out + f0, v);
      }
      return;
    }
    default:
      return;
  }
}

// tile-local partner of weight row l0 (first of a group of 8)
__device__ __forceinline__ int tc_partner_l(const TcParams& p, int l0) {
  if (p.epi.kind == EPI_QKV) return l0 ^ (p.epi.hd >> 1);
  if (p.epi.kind == EPI_SWIGLU) return l0 ^ 64;
  return l0;
}

// AND over the 128 epilogue threads (named barrier 1): keeps every branch that
// guards a named barrier uniform, whatever each thread saw of the abort flag.
__device__ __forceinline__ bool epi_vote_all(bool x) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(x))
      : "memory");
  return r != 0;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmW2,
                   const __grid_constant__ CUtensorMap tmX, TcParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int stage_bytes = kWBytes + p.x_boxes_max * kXBoxBytes;
  unsigned char* stage_base = smem;
  float* tileT = reinterpret_cast<float*>(smem + p.stages * stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.stages * stage_bytes + kTileTBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  uint64_t* acc_full = bars + 2 * p.stages;      // [2]
  uint64_t* acc_empty = acc_full + 2;            // [2]
  uint64_t* drain = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int rows = p.rows_cap;
  if (p.count) rows = min(rows, *p.count);
  if (rows <= 0) return;                         // uniform over the grid
  const int n_pass = (rows + kMaxPassRows - 1) / kMaxPassRows;
  const uint32_t tmem_cols = p.double_buf ? 512u : 256u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
    if (p.mode == 1) tma_prefetch_desc(&tmW2);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int it = 0;
      for (int u = blockIdx.x; u < p.n_units && !*abort_flag; u += gridDim.x) {
        const int tile = u / p.splits, split = u % p.splits;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        for (int pass = 0; pass < n_pass && !*abort_flag; ++pass) {
          const int prow0 = pass * kMaxPassRows;
          const int prows = min(kMaxPassRows, rows - prow0);
          const int nbox = (prows + kXBoxRows - 1) / kXBoxRows;
          const uint32_t bytes = kWBytes + nbox * kXBoxBytes;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % p.stages;
            const uint32_t ph = (it / p.stages) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, p.err)) { *abort_flag = 1; break; }
            unsigned char* st = stage_base + s * stage_bytes;
            mbar_arrive_expect_tx(&full[s], bytes);
            const int kx = kb * kBK;
            if (p.mode == 1) {
              tma_load_2d(st, &tmW, &full[s], kx, tile * 64, pol_w);
              tma_load_2d(st + kWBytes / 2, &tmW2, &full[s], kx, tile * 64, pol_w);
            } else {
              tma_load_2d(st, &tmW, &full[s], kx, tile * kTileF, pol_w);
            }
            for (int b = 0; b < nbox; ++b)
              tma_load_2d(st + kWBytes + b * kXBoxBytes, &tmX, &full[s], kx,
                          prow0 + b * kXBoxRows, pol_x);
          }
        }
      }
      // no copy into this CTA's shared memory may still be in flight at exit
      for (int i = max(0, it - p.stages); i < it; ++i)
        mbar_wait(&full[i % p.stages], (i / p.stages) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0, acc_it = 0;
      for (int u = blockIdx.x; u < p.n_units && !*abort_flag; u += gridDim.x) {
        const int split = u % p.splits;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        for (int pass = 0; pass < n_pass; ++pass, ++acc_it) {
          const int prows = min(kMaxPassRows, rows - pass * kMaxPassRows);
          const int n_mma = ((prows + 15) / 16) * 16;
          const uint32_t idesc = idesc_bf16(128, n_mma);
          const int buf = p.double_buf ? (acc_it & 1) : 0;
          const uint32_t par = p.double_buf ? ((acc_it >> 1) & 1) : (acc_it & 1);
          if (!mbar_wait(&acc_empty[buf], par ^ 1, p.err)) { *abort_flag = 1; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem + static_cast<uint32_t>(buf * 256);
          bool ok = true;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % p.stages;
            const uint32_t ph = (it / p.stages) & 1;
            if (*abort_flag || !mbar_wait(&full[s], ph, p.err)) { *abort_flag = 1; ok = false; break; }
            tc_fence_after();
            const uint32_t a0 = smem_u32(stage_base + s * stage_bytes);
            const uint32_t b0 = a0 + kWBytes;
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              umma_f16(d_tmem, sdesc_kmajor_sw128(a0 + k * 32), sdesc_kmajor_sw128(b0 + k * 32),
                       idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            umma_commit(&empty[s]);
          }
          if (!ok) break;
          umma_commit(&acc_full[buf]);
        }
      }
      umma_commit(drain);                 // every issued MMA done before TMEM is freed
      mbar_wait(drain, 0, p.err);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;               // TMEM lane quarter of this warp
    const int l = q * 32 + lane;          // tile-local weight row == TMEM lane
    const int et = threadIdx.x - 64;      // 0..127 within the epilogue warps
    int acc_it = 0;
    for (int u = blockIdx.x; u < p.n_units; u += gridDim.x) {
      const int tile = u / p.splits, split = u % p.splits;
      const int f = tc_feature(p, tile, l);
      for (int pass = 0; pass < n_pass; ++pass, ++acc_it) {
        const int prow0 = pass * kMaxPassRows;
        const int prows = min(kMaxPassRows, rows - prow0);
        const int buf = p.double_buf ? (acc_it & 1) : 0;
        const uint32_t par = p.double_buf ? ((acc_it >> 1) & 1) : (acc_it & 1);
        const bool ready = epi_vote_all(!*abort_flag && mbar_wait(&acc_full[buf], par, p.err));
        if (!ready) *abort_flag = 1;
        tc_fence_after();
        for (int c0 = 0; ready && c0 < prows; c0 += kChunk) {
          float v[kChunk];
          const uint32_t ta = tmem + (static_cast<uint32_t>(q * 32) << 16) +
                              static_cast<uint32_t>(buf * 256 + c0);
          tmem_ld16(ta, v);
          tmem_ld16(ta + 16, v + 16);
          tmem_ld_wait();
          if (p.splits > 1) {
            if (f >= 0) {
              float* part = p.partial +
                            (static_cast<int64_t>(split) * p.rows_cap + prow0 + c0) * p.n_out + f;
#pragma unroll
              for (int i = 0; i < kChunk; ++i)
                if (c0 + i < prows) part[static_cast<int64_t>(i) * p.n_out] = v[i];
            }
          } else {
#pragma unroll
            for (int i = 0; i < kChunk; ++i) tileT[i * kTileLd + l] = v[i];
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const int nr = min(kChunk, prows - c0);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int item = et + 128 * k;
              const int r = item >> 4, l0 = (item & 15) * 8;
              if (r < nr) {
                const float* a = tileT + r * kTileLd + l0;
                const float* b = tileT + r * kTileLd + tc_partner_l(p, l0);
                float va[8], vb[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) { va[i] = a[i]; vb[i] = b[i]; }
                epi_group8(p, tile, prow0 + c0 + r, l0, va, vb);
              }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
          }
        }
        tc_fence_before();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      if (p.splits > 1) {
        // all splits of this tile publish, then each reduces its own slice of rows
        __threadfence();
        bool go = epi_vote_all(!*abort_flag);
        if (et == 0 && go) {
          atomicAdd(&p.counters[2 * tile], 1);
          const uint64_t t0 = globaltimer();
          while (ld_acquire(&p.counters[2 * tile]) < p.splits) {
            if (globaltimer() - t0 > kWaitNs) {
              flag_error(p.err, SF_DEV_ERR_TIMEOUT);
              *abort_flag = 1;
              break;
            }
          }
        }
        go = epi_vote_all(!*abort_flag);
        const int slice = (rows + p.splits - 1) / p.splits;
        const int r0 = split * slice, r1 = min(rows, r0 + slice);
        for (int c0 = r0; go && c0 < r1; c0 += kChunk) {
          const int nr = min(kChunk, r1 - c0);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int item = et + 128 * k;
            const int r = item >> 4, l0 = (item & 15) * 8;
            if (r >= nr) continue;
            const int fa = tc_feature(p, tile, l0);
            if (fa < 0) continue;
            const int fb = tc_feature(p, tile, tc_partner_l(p, l0));
            float va[8] = {}, vb[8] = {};
            for (int s = 0; s < p.splits; ++s) {
              const float* row = p.partial + (static_cast<int64_t>(s) * p.rows_cap + c0 + r) * p.n_out;
              const float4 a0 = __ldcg(reinterpret_cast<const float4*>(row + fa));
              const float4 a1 = __ldcg(reinterpret_cast<const float4*>(row + fa + 4));
              va[0] += a0.x; va[1] += a0.y; va[2] += a0.z; va[3] += a0.w;
              va[4] += a1.x; va[5] += a1.y; va[6] += a1.z; va[7] += a1.w;
              if (fb >= 0 && fb != fa) {
                const float4 b0 = __ldcg(reinterpret_cast<const float4*>(row + fb));
                const float4 b1 = __ldcg(reinterpret_cast<const float4*>(row + fb + 4));
                vb[0] += b0.x; vb[1] += b0.y; vb[2] += b0.z; vb[3] += b0.w;
                vb[4] += b1.x; vb[5] += b1.y; vb[6] += b1.z; vb[7] += b1.w;
              }
            }
            epi_group8(p, tile, c0 + r, l0, va, fb == fa ? va : vb);
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (et == 0 && go) {
          const int prev = atomicAdd(&p.counters[2 * tile + 1], 1);
          if (prev == p.splits - 1) {      // everyone has passed the wait: reset
            p.counters[2 * tile] = 0;
            p.counters[2 * tile + 1] = 0;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, tmem_cols);
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 row-major [rows][cols], box [box_rows][64], 128-byte swizzle
static bool make_tmap(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols,
                      uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

struct TcPlan {
  int n_tiles, splits, kb_total, kb_per_split;
};
static TcPlan tc_plan(int n_out, int K, int mode, int inter, int rows_cap) {
  TcPlan pl;
  pl.n_tiles = mode == 1 ? (inter + 63) / 64 : (n_out + kTileF - 1) / kTileF;
  pl.kb_total = (K + kBK - 1) / kBK;
  const int sms = num_sms();
  int splits = 1;
  // few tiles: split K so that tiles x splits fills the SMs (one pass of rows only)
  if (rows_cap <= kMaxPassRows && pl.n_tiles < sms / 2 && pl.n_tiles <= kMaxCounterTiles) {
    splits = std::max(1, std::min(sms / pl.n_tiles, pl.kb_total / 4));
  }
  pl.kb_per_split = (pl.kb_total + splits - 1) / splits;
  pl.splits = (pl.kb_total + pl.kb_per_split - 1) / pl.kb_per_split;  // no empty split
  return pl;
}

size_t gemm_ws_need(int dtype, int rows_cap, int n_out, int K, int kind, int inter) {
  // SIMT path: raw fp32 result after the (untouched) counter region
  if (dtype != BF16) return kCounterBytes + static_cast<size_t>(rows_cap) * n_out * 4;
  const int mode = kind == EPI_SWIGLU ? 1 : 0;
  const TcPlan pl = tc_plan(n_out, K, mode, inter, rows_cap);
  if (pl.splits <= 1) return 0;
  return kCounterBytes + static_cast<size_t>(pl.splits) * rows_cap * n_out * 4;
}

int gemm_path_is_tc(int dtype) { return dtype == BF16; }

static cudaError_t gemm_tc(const GemmArgs& a, cudaStream_t st) {
  const int mode = a.epi.kind == EPI_SWIGLU ? 1 : 0;
  const int inter = a.epi.inter;
  if (a.n_out % 8 != 0 || (mode == 1 && inter % 8 != 0)) return cudaErrorInvalidValue;
  const TcPlan pl = tc_plan(a.n_out, a.K, mode, inter, a.rows_cap);
  TcParams p{};
  p.n_out = a.n_out;
  p.K = a.K;
  p.rows_cap = a.rows_cap;
  p.count = a.count;
  p.mode = mode;
  p.inter = inter;
  p.n_tiles = pl.n_tiles;
  p.splits = pl.splits;
  p.kb_total = pl.kb_total;
  p.kb_per_split = pl.kb_per_split;
  p.n_units = pl.n_tiles * pl.splits;
  const int sms = num_sms();
  const int grid = pl.splits > 1 ? p.n_units : std::min(p.n_units, sms);
  p.double_buf = (p.n_units > grid || a.rows_cap > kMaxPassRows) ? 1 : 0;
  const int max_pass_rows = std::min(a.rows_cap, kMaxPassRows);
  p.x_boxes_max = (max_pass_rows + kXBoxRows - 1) / kXBoxRows;
  const int stage_bytes = kWBytes + p.x_boxes_max * kXBoxBytes;
  const int budget = 222 * 1024 - kTileTBytes - 1024 - 256;
  p.stages = std::max(2, std::min(8, budget / stage_bytes));
  const size_t smem = 1024 + static_cast<size_t>(p.stages) * stage_bytes + kTileTBytes + 256;
  if (pl.splits > 1) {
    const size_t need = kCounterBytes + static_cast<size_t>(pl.splits) * a.rows_cap * a.n_out * 4;
    if (a.ws == nullptr || a.ws_bytes < need) return cudaErrorInvalidValue;
    p.counters = static_cast<int*>(a.ws);
    p.partial = reinterpret_cast<float*>(static_cast<char*>(a.ws) + kCounterBytes);
  }
  p.epi = a.epi;
  p.err = a.err;

  CUtensorMap tmW, tmW2, tmX;
  const uint32_t wrows = mode == 1 ? 64 : kTileF;
  const int w_rows_total = mode == 1 ? inter : a.n_out;
  if (!make_tmap(&tmW, a.W, w_rows_total, a.K, wrows)) return cudaErrorInvalidValue;
  if (!make_tmap(&tmW2, mode == 1 ? a.W2 : a.W, w_rows_total, a.K, wrows))
    return cudaErrorInvalidValue;
  if (!make_tmap(&tmX, a.X, a.rows_cap, a.K, kXBoxRows)) return cudaErrorInvalidValue;

  static int configured_smem = 0;
  if (configured_smem < static_cast<int>(smem)) {
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured_smem = static_cast<int>(smem);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (pl.splits > 1) {
    // the split CTAs of a tile wait for one another: all must be resident at once
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, tc_gemm_kernel, tmW, tmW2, tmX, p);
  if (e != cudaSuccess) return e;
  return launched();
}

template <typename T>
static cudaError_t gemm_simt_t(const GemmArgs& a, cudaStream_t st) {
  // raw fp32 result in the workspace, then the epilogue pass
  const size_t need = kCounterBytes + static_cast<size_t>(a.rows_cap) * a.n_out * 4;
  if (a.ws == nullptr || a.ws_bytes < need) return cudaErrorInvalidValue;
  float* raw = reinterpret_cast<float*>(static_cast<char*>(a.ws) + kCounterBytes);
  dim3 grid((a.n_out + 63) / 64, (a.rows_cap + 63) / 64);
  simt_gemm_kernel<T><<<grid, 256, 0, st>>>(static_cast<const T*>(a.X), static_cast<const T*>(a.W),
                                            static_cast<const T*>(a.W2), a.n_out, a.K,
                                            a.rows_cap, a.count, a.epi.inter, raw);
  cudaError_t e = launched();
  if (e != cudaSuccess) return e;
  const int64_t total = static_cast<int64_t>(a.rows_cap) * a.n_out;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  epilogue_kernel<T><<<blocks, 256, 0, st>>>(raw, a.n_out, a.rows_cap, a.count, a.epi);
  return launched();
}

cudaError_t gemm(const GemmArgs& a, cudaStream_t st) {
  if (a.rows_cap <= 0 || a.n_out <= 0 || a.K <= 0) return cudaErrorInvalidValue;
  if (a.dtype == BF16) {
    if (a.K % 8 != 0) return cudaErrorInvalidValue;
    return gemm_tc(a, st);
  }
  return gemm_simt_t<float>(a, st);
}

// bf16 SIMT variant for cross-checking the tensor-core kernel in tests
cudaError_t gemm_simt_bf16(const GemmArgs& a, cudaStream_t st) {
  return gemm_simt_t<__nv_bfloat16>(a, st);
}

}  // namespace sf
