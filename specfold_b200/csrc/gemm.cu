// Projections of the folded verify forward: dispatch, and the SIMT path used for fp32
// models (tcgen05 has no fp32-exact kind); bf16 runs the tensor-core kernel in
// gemm_tc.cu.  The SIMT path computes acc[j][f] = sum_k X[j][k] * W[f][k] into an fp32
// scratch, then applies the epilogue in a second pass.
//
// Epilogues (EpiKind) reproduce the rounding points of the PyTorch folded forward:
//   QKV     F.linear + bias rounded to the model dtype, then q*c + rot(q)*s with every
//           op rounded (fastdllm_v2_folded.py:153-157; triton_kernels.py:65-87)
//   RESID   x + T(O @ Wo^T) (fastdllm_v2_folded.py:207-208, :351)
//   SWIGLU  T(silu(T(g))) * T(u) (fastdllm_v2_folded.py:216; triton_kernels.py:133)
//   SCATTER ffn_buf[rows[j]] = T(acc) (triton_kernels.py:171-173)
//   LOGITS  lm_head with the Fast-dLLM shift (fastdllm_v2_generation.py:121-126)
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

template <typename T>
static cudaError_t gemm_simt_t(const GemmArgs& a, cudaStream_t st) {
  // raw fp32 result in the workspace, then the epilogue pass
  const size_t need = kGemmCounterBytes + static_cast<size_t>(a.rows_cap) * a.n_out * 4;
  if (a.ws == nullptr || a.ws_bytes < need) return cudaErrorInvalidValue;
  float* raw = reinterpret_cast<float*>(static_cast<char*>(a.ws) + kGemmCounterBytes);
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

size_t gemm_ws_need(int dtype, int rows_cap, int n_out, int K, int kind, int inter) {
  // SIMT path: raw fp32 result after the (untouched) counter region
  if (dtype != BF16) return kGemmCounterBytes + static_cast<size_t>(rows_cap) * n_out * 4;
  return gemm_tc_ws_need(rows_cap, n_out, K, kind, inter);
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
