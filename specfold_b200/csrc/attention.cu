// Attention of the recomputed rows with retained softmax state, and the exact
// chain-correction merge of the folded rows.
//
// attn_simt_kernel: one CTA per (recomputed row, kv head); every query head of the
//   kv group streams the prefix cache and then the N in-block keys taken through the
//   source map kv_buf[src[b*N+j]*N + j] (specfold_flash_attn_gqa_kernel,
//   triton_kernels.py:301-361; PyTorch: fastdllm_v2_folded.py:164-181).  Online softmax
//   in fp32; writes O (normalised), M = row max, Z = sum of exp.
//
// merge_kernel: one CTA per (folded row, kv head).  Starts from the source row's
//   (m, Z, O) and, for every branch on the chain from the row's branch up to (not
//   including) its source branch, replaces the contribution of each key that branch
//   recomputed: old key = what the parent saw at that position, new key = the branch's
//   own (specfold_chain_correction_gqa_kernel, triton_kernels.py:364-429; PyTorch:
//   fastdllm_v2_folded.py:183-204, which applies the same update one branch at a time).
#include "sf_kernels.cuh"

namespace sf {

constexpr int kAttnKeys = 32;   // keys per smem tile (one per lane)
constexpr int kMaxGroup = 16;   // q heads per kv head

// With part_O != nullptr the prefix keys were already folded into per-split partials
// (unnormalised O, running max m, sum l) by the tensor-core kernel: the state starts
// from their log-sum-exp merge and only the in-block keys are added here.
template <typename T, int HD>
__global__ void __launch_bounds__(128) attn_simt_kernel(AttnParams p, const float* part_O,
                                                        const float* part_ml, int splits,
                                                        int q_rows) {
  constexpr int DPL = HD / 32;  // dims per lane
  __shared__ float qs[kMaxGroup][HD];
  __shared__ float ks[kAttnKeys][HD + 1];
  __shared__ float vs[kAttnKeys][HD + 1];
  __shared__ int64_t krow[kAttnKeys];

  const int slot = blockIdx.x, kvh = blockIdx.y;
  const int count = min(*p.count, p.bucket);
  if (slot >= count) return;
  const int64_t r = p.rows[slot];
  const int64_t BN = static_cast<int64_t>(p.B1) * p.N;
  if (r < 0 || r >= BN) { flag_error(p.err, SF_DEV_ERR_INDEX); return; }
  const int64_t b = r / p.N;
  const int G = p.H / p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = p.H * HD, kvd = 2 * p.Hkv * HD;
  const T* qb = reinterpret_cast<const T*>(p.q_buf);
  const T* kvb = reinterpret_cast<const T*>(p.kv_buf);
  const T* pk = reinterpret_cast<const T*>(p.pk);
  const T* pv = reinterpret_cast<const T*>(p.pv);

  for (int i = threadIdx.x; i < G * HD; i += 128) {
    const int g = i / HD, d = i % HD;
    qs[g][d] = Elt<T>::to_f(qb[r * qd + (kvh * G + g) * HD + d]);
  }
  float m[4], l[4], acc[4][DPL];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int t = 0; t < DPL; ++t) acc[i][t] = 0.f;
  }
  if (part_O != nullptr) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int g = warp + 4 * i;
      if (g >= G) break;
      const int64_t qi = static_cast<int64_t>(slot) * G + g;
      float mx = -INFINITY;
      for (int s = 0; s < splits; ++s)
        mx = fmaxf(mx, part_ml[2 * ((static_cast<int64_t>(s) * p.Hkv + kvh) * q_rows + qi)]);
      m[i] = mx;
      for (int s = 0; s < splits; ++s) {
        const int64_t base = (static_cast<int64_t>(s) * p.Hkv + kvh) * q_rows + qi;
        const float ms = part_ml[2 * base];
        if (ms == -INFINITY) continue;
        const float w = expf(ms - mx);
        l[i] += part_ml[2 * base + 1] * w;
#pragma unroll
        for (int t = 0; t < DPL; ++t) acc[i][t] = fmaf(part_O[base * HD + lane + 32 * t], w, acc[i][t]);
      }
    }
  }
  const int total = p.P + p.N;
  const int key_begin = part_O != nullptr ? p.P : 0;
  for (int k0 = key_begin; k0 < total; k0 += kAttnKeys) {
    __syncthreads();
    if (threadIdx.x < kAttnKeys) {
      const int key = k0 + threadIdx.x;
      int64_t kr = -1;
      if (key >= p.P && key < total) {
        const int j = key - p.P;
        int64_t s = p.src[b * p.N + j];
        if (s < 0 || s >= p.B1) { flag_error(p.err, SF_DEV_ERR_INDEX); s = 0; }
        kr = s * p.N + j;
      }
      krow[threadIdx.x] = kr;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kAttnKeys * HD; i += 128) {
      const int t = i / HD, d = i % HD;
      const int key = k0 + t;
      float kv = 0.f, vv = 0.f;
      if (key < p.P) {
        const int64_t o = kvh * p.kv_head_stride + static_cast<int64_t>(key) * HD + d;
        kv = Elt<T>::to_f(pk[o]);
        vv = Elt<T>::to_f(pv[o]);
      } else if (key < total) {
        const int64_t o = krow[t] * kvd;
        kv = Elt<T>::to_f(kvb[o + kvh * HD + d]);
        vv = Elt<T>::to_f(kvb[o + (p.Hkv + kvh) * HD + d]);
      }
      ks[t][d] = kv;
      vs[t][d] = vv;
    }
    __syncthreads();
    const bool valid = (k0 + lane) < total;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int g = warp + 4 * i;
      if (g >= G) break;
      float s = 0.f;
#pragma unroll 8
      for (int d = 0; d < HD; ++d) s = fmaf(qs[g][d], ks[lane][d], s);
      s = valid ? s * p.scale : -INFINITY;
      const float mt = warp_max(s);
      const float mn = fmaxf(m[i], mt);
      const float alpha = expf(m[i] - mn);
      const float e = valid ? expf(s - mn) : 0.f;
      l[i] = l[i] * alpha + warp_sum(e);
#pragma unroll
      for (int t = 0; t < DPL; ++t) acc[i][t] *= alpha;
#pragma unroll 4
      for (int jj = 0; jj < kAttnKeys; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, e, jj);
#pragma unroll
        for (int t = 0; t < DPL; ++t) acc[i][t] = fmaf(pj, vs[jj][lane + 32 * t], acc[i][t]);
      }
      m[i] = mn;
    }
  }
  T* O = reinterpret_cast<T*>(p.O);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int g = warp + 4 * i;
    if (g >= G) break;
    const int h = kvh * G + g;
#pragma unroll
    for (int t = 0; t < DPL; ++t)
      O[r * qd + h * HD + lane + 32 * t] = Elt<T>::from_f(acc[i][t] / l[i]);
    if (lane == 0) {
      p.M[r * p.H + h] = m[i];
      p.Z[r * p.H + h] = l[i];
    }
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(128) merge_kernel(MergeParams p) {
  constexpr int DPL = HD / 32;
  const int64_t r = blockIdx.x;
  const int kvh = blockIdx.y;
  if (p.rec[r] != 0) return;
  const int N = p.N, B1 = p.B1;
  const int64_t b = r / N, n = r % N;
  int64_t srow = p.src[r];
  if (srow < 0 || srow >= B1) { flag_error(p.err, SF_DEV_ERR_INDEX); return; }
  const int G = p.H / p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = p.H * HD, kvd = 2 * p.Hkv * HD;
  const T* qb = reinterpret_cast<const T*>(p.q_buf);
  const T* kvb = reinterpret_cast<const T*>(p.kv_buf);
  T* O = reinterpret_cast<T*>(p.O);
  const int64_t sflat = srow * N + n;

  for (int g = warp; g < G; g += 4) {
    const int h = kvh * G + g;
    float q[DPL], num[DPL];
#pragma unroll
    for (int t = 0; t < DPL; ++t) q[t] = Elt<T>::to_f(qb[sflat * qd + h * HD + lane + 32 * t]);
    const float m0 = p.M[sflat * p.H + h];
    const float Z0 = p.Z[sflat * p.H + h];
    auto score = [&](int64_t row) {
      float s = 0.f;
#pragma unroll
      for (int t = 0; t < DPL; ++t)
        s = fmaf(q[t], Elt<T>::to_f(kvb[row * kvd + kvh * HD + lane + 32 * t]), s);
      return warp_sum(s) * p.scale;
    };
    // pass 1: new running max over every key that changed along the chain
    float mn = m0;
    int64_t cur = b;
    int hops = 0;
    while (cur != srow && hops < B1) {
      const int cnt = p.segcnt[cur];
      for (int e = 0; e < cnt; ++e) mn = fmaxf(mn, score(p.seg[cur * N + e]));
      cur = p.par_idx[cur];
      ++hops;
    }
    if (cur != srow) { flag_error(p.err, SF_DEV_ERR_DEPTH); continue; }
    // pass 2: rescale and swap old for new contributions
    float Z = Z0 * expf(m0 - mn);
#pragma unroll
    for (int t = 0; t < DPL; ++t)
      num[t] = Elt<T>::to_f(O[sflat * qd + h * HD + lane + 32 * t]) * Z;
    cur = b;
    while (cur != srow) {
      const int64_t pc = p.par_idx[cur];
      const int cnt = p.segcnt[cur];
      for (int e = 0; e < cnt; ++e) {
        const int64_t rn = p.seg[cur * N + e];
        const int64_t pos = rn % N;
        const int64_t ro = p.src[pc * N + pos] * N + pos;
        const float ao = expf(score(ro) - mn);
        const float an = expf(score(rn) - mn);
        Z = Z - ao + an;
#pragma unroll
        for (int t = 0; t < DPL; ++t) {
          const float vo = Elt<T>::to_f(kvb[ro * kvd + (p.Hkv + kvh) * HD + lane + 32 * t]);
          const float vn = Elt<T>::to_f(kvb[rn * kvd + (p.Hkv + kvh) * HD + lane + 32 * t]);
          num[t] = num[t] - ao * vo + an * vn;
        }
      }
      cur = pc;
    }
#pragma unroll
    for (int t = 0; t < DPL; ++t) O[r * qd + h * HD + lane + 32 * t] = Elt<T>::from_f(num[t] / Z);
    if (lane == 0) {
      p.M[r * p.H + h] = mn;
      p.Z[r * p.H + h] = Z;
    }
  }
}

template <typename T>
__global__ void kv_append_kernel(T* ck, T* cv, int64_t cs, const T* nk, const T* nv, int64_t ns,
                                 int Hkv, int hd, int P, int n) {
  constexpr int V = Elt<T>::kVec;
  const int per_head = n * hd / V;
  const int64_t total = static_cast<int64_t>(Hkv) * per_head;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int h = static_cast<int>(i / per_head);
    const int64_t e = (i % per_head) * V;   // element within the head's [n, hd] block
    const int64_t src = h * ns + e;
    const int64_t dst = h * cs + static_cast<int64_t>(P) * hd + e;
    *reinterpret_cast<uint4*>(ck + dst) = *reinterpret_cast<const uint4*>(nk + src);
    *reinterpret_cast<uint4*>(cv + dst) = *reinterpret_cast<const uint4*>(nv + src);
  }
}

// ------------------------------------------------------------------------ launchers
template <typename T>
static cudaError_t attn_t(const AttnParams& p, const float* part_O, const float* part_ml,
                          int splits, int q_rows, cudaStream_t st) {
  dim3 grid(p.bucket, p.Hkv);
  if (p.hd == 128)
    attn_simt_kernel<T, 128><<<grid, 128, 0, st>>>(p, part_O, part_ml, splits, q_rows);
  else if (p.hd == 64)
    attn_simt_kernel<T, 64><<<grid, 128, 0, st>>>(p, part_O, part_ml, splits, q_rows);
  else
    return cudaErrorInvalidValue;
  return launched();
}
cudaError_t launch_attention_simt(int dtype, const AttnParams& p, cudaStream_t st) {
  if (p.H % p.Hkv != 0 || p.H / p.Hkv > kMaxGroup) return cudaErrorInvalidValue;
  return dtype == BF16 ? attn_t<__nv_bfloat16>(p, nullptr, nullptr, 0, 0, st)
                       : attn_t<float>(p, nullptr, nullptr, 0, 0, st);
}
cudaError_t launch_attention_simt_partials(int dtype, const AttnParams& p, const float* part_O,
                                           const float* part_ml, int splits, int q_rows,
                                           cudaStream_t st) {
  if (p.H % p.Hkv != 0 || p.H / p.Hkv > kMaxGroup) return cudaErrorInvalidValue;
  return dtype == BF16 ? attn_t<__nv_bfloat16>(p, part_O, part_ml, splits, q_rows, st)
                       : attn_t<float>(p, part_O, part_ml, splits, q_rows, st);
}

template <typename T>
static cudaError_t merge_t(const MergeParams& p, cudaStream_t st) {
  dim3 grid(p.B1 * p.N, p.Hkv);
  if (p.hd == 128) merge_kernel<T, 128><<<grid, 128, 0, st>>>(p);
  else if (p.hd == 64) merge_kernel<T, 64><<<grid, 128, 0, st>>>(p);
  else return cudaErrorInvalidValue;
  return launched();
}
cudaError_t launch_merge(int dtype, const MergeParams& p, cudaStream_t st) {
  if (p.H % p.Hkv != 0) return cudaErrorInvalidValue;
  return dtype == BF16 ? merge_t<__nv_bfloat16>(p, st) : merge_t<float>(p, st);
}

cudaError_t launch_kv_append(int dtype, void* ck, void* cv, int64_t c_stride, const void* nk,
                             const void* nv, int64_t n_stride, int Hkv, int hd, int P, int n,
                             cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int vec = dtype == BF16 ? 8 : 4;
  if (hd % vec != 0) return cudaErrorInvalidValue;
  const int64_t total = static_cast<int64_t>(Hkv) * n * hd / vec;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 1184));
  if (dtype == BF16)
    kv_append_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        static_cast<__nv_bfloat16*>(ck), static_cast<__nv_bfloat16*>(cv), c_stride,
        static_cast<const __nv_bfloat16*>(nk), static_cast<const __nv_bfloat16*>(nv), n_stride,
        Hkv, hd, P, n);
  else
    kv_append_kernel<float><<<blocks, 256, 0, st>>>(
        static_cast<float*>(ck), static_cast<float*>(cv), c_stride, static_cast<const float*>(nk),
        static_cast<const float*>(nv), n_stride, Hkv, hd, P, n);
  return launched();
}


}  // namespace sf
