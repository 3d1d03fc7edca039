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
constexpr int kTcThreads = 192;        // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kTileF = 128;            // weight rows per tile (MMA M)
constexpr int kBK = 64;                // K elements per stage (one 128-byte swizzle row)
constexpr int kMaxPassRows = 256;      // MMA N limit
constexpr int kWBytes = kTileF * kBK * 2;       // 16 KB
constexpr int kXBoxRows = 64;
constexpr int kXBoxBytes = kXBoxRows * kBK * 2;  // 8 KB
constexpr int kXchBytes = 128 * 17 * 4;          // epilogue exchange (16 cols + pad)

struct TcParams {
  int n_out, K, rows_cap;
  const int32_t* count;
  int mode;            // 0: 128-row tiles of W; 1: SWIGLU, 64 gate + 64 up rows per tile
  int inter;
  int n_tiles, splits, kb_total, kb_per_split;
  int stages, x_boxes_max;   // smem layout
  float* partial;      // [splits][rows_cap][n_out] when splits > 1
  int* counters;       // [n_tiles]
  EpiParams epi;
  int* err;
};

__device__ __forceinline__ int tc_feature(const TcParams& p, int tile, int l) {
  if (p.mode == 1) {
    const int g = tile * 64 + (l & 63);
    if (g >= p.inter) return -1;
    return l < 64 ? g : p.inter + g;
  }
  const int f = tile * kTileF + l;
  return f < p.n_out ? f : -1;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmW2,
                   const __grid_constant__ CUtensorMap tmX, TcParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the swizzle atoms
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int stage_bytes = kWBytes + p.x_boxes_max * kXBoxBytes;
  unsigned char* stage_base = smem;
  float* xch = reinterpret_cast<float*>(smem + p.stages * stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.stages * stage_bytes + kXchBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  uint64_t* acc_full = bars + 2 * p.stages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  int rows = p.rows_cap;
  if (p.count) rows = min(rows, *p.count);
  if (rows <= 0) return;
  const int n_pass = (rows + kMaxPassRows - 1) / kMaxPassRows;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
  if (kb0 >= kb1) return;   // host guarantees every split has work
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
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
      // make sure no copy into this CTA's shared memory is still in flight
      const int issued = it;
      for (int i = max(0, issued - p.stages); i < issued; ++i)
        mbar_wait(&full[i % p.stages], (i / p.stages) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0;
      for (int pass = 0; pass < n_pass; ++pass) {
        const int prows = min(kMaxPassRows, rows - pass * kMaxPassRows);
        const int n_mma = ((prows + 15) / 16) * 16;
        const uint32_t idesc = idesc_bf16(128, n_mma);
        if (pass > 0 && !mbar_wait(acc_empty, (pass - 1) & 1, p.err)) { *abort_flag = 1; break; }
        tc_fence_after();
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % p.stages;
          const uint32_t ph = (it / p.stages) & 1;
          if (*abort_flag || !mbar_wait(&full[s], ph, p.err)) { *abort_flag = 1; ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(stage_base + s * stage_bytes);
          const uint32_t b0 = a0 + kWBytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            umma_f16(tmem, sdesc_kmajor_sw128(a0 + k * 32), sdesc_kmajor_sw128(b0 + k * 32),
                     idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(acc_full);
      }
      // all issued MMAs complete before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0, p.err);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int l = q * 32 + lane;            // tile-local weight row == TMEM lane
    const int f = tc_feature(p, tile, l);
    const int lp = (p.epi.kind == EPI_QKV) ? (l ^ (p.epi.hd >> 1)) : (l ^ 64);
    const bool emits = f >= 0 && epi_emits(p.epi, f);
    for (int pass = 0; pass < n_pass; ++pass) {
      const int prow0 = pass * kMaxPassRows;
      const int prows = min(kMaxPassRows, rows - prow0);
      if (!mbar_wait(acc_full, pass & 1, p.err)) { *abort_flag = 1; break; }
      tc_fence_after();
      for (int c0 = 0; c0 < prows; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, v);
        tmem_ld_wait();
        if (p.splits > 1) {
          if (f >= 0) {
            float* part = p.partial + (static_cast<int64_t>(split) * p.rows_cap + prow0 + c0) * p.n_out + f;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (c0 + i < prows) part[static_cast<int64_t>(i) * p.n_out] = v[i];
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) xch[l * 17 + i] = v[i];
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (emits) {
            for (int i = 0; i < 16 && c0 + i < prows; ++i)
              epi_apply<__nv_bfloat16>(p.epi, prow0 + c0 + i, f, v[i], xch[lp * 17 + i]);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
      }
      tc_fence_before();
      if (lane == 0) mbar_arrive(acc_empty);
    }
    if (p.splits > 1 && !*abort_flag) {
      // publish partials; the last CTA of this tile reduces and applies the epilogue
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        const int prev = atomicAdd(&p.counters[tile], 1);
        *last_flag = (prev == p.splits - 1) ? 1 : 0;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*last_flag) {
        __threadfence();
        for (int c0 = 0; c0 < rows; c0 += 16) {
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
          if (f >= 0) {
            for (int s = 0; s < p.splits; ++s) {
              const float* part = p.partial + (static_cast<int64_t>(s) * p.rows_cap + c0) * p.n_out + f;
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (c0 + i < rows) v[i] += __ldcg(part + static_cast<int64_t>(i) * p.n_out);
            }
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) xch[l * 17 + i] = v[i];
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (emits) {
            for (int i = 0; i < 16 && c0 + i < rows; ++i)
              epi_apply<__nv_bfloat16>(p.epi, c0 + i, f, v[i], xch[lp * 17 + i]);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
        if (threadIdx.x == 64) p.counters[tile] = 0;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 256);
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
static TcPlan tc_plan(int n_out, int K, int mode, int inter) {
  TcPlan pl;
  pl.n_tiles = mode == 1 ? (inter + 63) / 64 : (n_out + kTileF - 1) / kTileF;
  pl.kb_total = (K + kBK - 1) / kBK;
  const int sms = num_sms();
  int splits = 1;
  if (pl.n_tiles < sms / 2) {
    splits = (sms + pl.n_tiles - 1) / pl.n_tiles;
    if (splits > sms / pl.n_tiles && sms / pl.n_tiles >= 1) splits = sms / pl.n_tiles;
    splits = std::max(1, std::min(splits, pl.kb_total / 4));
  }
  pl.kb_per_split = (pl.kb_total + splits - 1) / splits;
  pl.splits = (pl.kb_total + pl.kb_per_split - 1) / pl.kb_per_split;  // no empty split
  return pl;
}

// Workspace layout of the tensor-core path: kCounterBytes of split-K tile counters at
// offset 0 (a fixed place, so every GEMM finds them zero: the last CTA of a tile resets
// its counter), then the fp32 partial sums [splits][rows_cap][n_out].
constexpr size_t kCounterBytes = 16384;
constexpr int kMaxCounters = static_cast<int>(kCounterBytes / 4);

size_t gemm_ws_need(int dtype, int rows_cap, int n_out, int K, int kind, int inter) {
  // SIMT path: raw fp32 result after the (untouched) counter region
  if (dtype != BF16) return kCounterBytes + static_cast<size_t>(rows_cap) * n_out * 4;
  const int mode = kind == EPI_SWIGLU ? 1 : 0;
  const TcPlan pl = tc_plan(n_out, K, mode, inter);
  if (pl.splits <= 1) return 0;
  return kCounterBytes + static_cast<size_t>(pl.splits) * rows_cap * n_out * 4;
}

int gemm_path_is_tc(int dtype) { return dtype == BF16; }

static cudaError_t gemm_tc(const GemmArgs& a, cudaStream_t st) {
  const int mode = a.epi.kind == EPI_SWIGLU ? 1 : 0;
  const int inter = a.epi.inter;
  TcPlan pl = tc_plan(a.n_out, a.K, mode, inter);
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
  const int max_pass_rows = std::min(a.rows_cap, kMaxPassRows);
  p.x_boxes_max = (max_pass_rows + kXBoxRows - 1) / kXBoxRows;
  const int stage_bytes = kWBytes + p.x_boxes_max * kXBoxBytes;
  const int budget = 220 * 1024 - kXchBytes;
  p.stages = std::max(2, std::min(8, budget / stage_bytes));
  const size_t smem = 1024 + static_cast<size_t>(p.stages) * stage_bytes + kXchBytes + 256;
  // workspace: tile counters at offset 0, partials after
  if (pl.splits > 1) {
    const size_t need = kCounterBytes + static_cast<size_t>(pl.splits) * a.rows_cap * a.n_out * 4;
    if (a.ws == nullptr || a.ws_bytes < need || pl.n_tiles > kMaxCounters)
      return cudaErrorInvalidValue;
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
  dim3 grid(pl.n_tiles, pl.splits);
  tc_gemm_kernel<<<grid, kTcThreads, smem, st>>>(tmW, tmW2, tmX, p);
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
