// Greedy top-p sampling of the verify step's logits: per row, the argmax token and its
// probability after top-p filtering, without sorting the vocabulary.
//
// The reference (FastDLLMModelExecutor.sample_with_top_p, fastdllm_model_executor.py:
// 130-155, called through _sample_with_top_p at fastdllm_v2_generation.py:346 with
// temperature 0) sorts every row, takes T(softmax) of the sorted logits (T = the logits'
// dtype), cumulative sums (fp32 accumulation, each prefix rounded to T), keeps the
// sorted prefix up to and including the first position whose cumulative sum exceeds
// top_p, re-normalises over the kept tokens and returns argmax and the probabilities;
// the decode loop then reads the probability of the argmax token only (:348-351).
//
// Here, one CTA per row:
//   1. m = max logit, Z = sum exp(l - m) (fp32, fixed-order block reduction);
//   2. a radix select over an order-preserving key of the logit (12 + 12 + 8 bits; two
//      levels for bf16, whose low 16 key bits are zero) finds the logit value at which
//      the sorted cumulative sum of p = T(exp(l - m) / Z) first exceeds top_p: each
//      level histograms the rows under the current key prefix (count, sum of p, sum of
//      exp(l - m)) and walks its bins from the top; sums are 2^-40 fixed point, so the
//      histogram is independent of the order the atomics land in;
//   3. within the tokens of that exact logit, the cumulative sum is continued token by
//      token to find how many of them are kept; Z_kept = exp sum of the tokens above
//      + kept * exp(l* - m);
//   4. conf = T(1 / Z_kept), the probability of the maximal logit after filtering, and
//      the token is the smallest index whose filtered probability T(exp(l - m) / Z_kept)
//      equals it (torch.argmax returns the first maximal element).
// Cumulative sums are exact here where the reference's fp32 scan rounds; the two can
// differ only for a prefix sum within fp32 rounding of the top_p boundary.
#include <climits>
#include <cstdint>

#include "sf_kernels.cuh"

namespace sf {

namespace {

constexpr int kSampleThreads = 512;
constexpr int kBins = 4096;
constexpr float kFix = 1099511627776.0f;   // 2^40

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
template <typename T>
__device__ __forceinline__ float round_t(float x) {
  return Elt<T>::rnd(x);
}
__device__ __forceinline__ unsigned long long to_fix(float v) {
  return __float2ull_rn(v * kFix);
}
__device__ __forceinline__ float from_fix(unsigned long long v) {
  return static_cast<float>(static_cast<double>(v) * (1.0 / 1099511627776.0));
}

__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < kSampleThreads / 32; ++w) r = fmaxf(r, red[w]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
  for (int w = 0; w < kSampleThreads / 32; ++w) r += red[w];
  __syncthreads();
  return r;
}
__device__ __forceinline__ long long block_min_ll(long long v, long long* red) {
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  long long r = red[0];
  for (int w = 1; w < kSampleThreads / 32; ++w) r = min(r, red[w]);
  __syncthreads();
  return r;
}

struct Walk {               // result of one level's bin walk
  int bin;                  // first bin (from the top) where the cumulative sum crosses, or -1
  unsigned long long p_above, e_above;   // sums over the bins above it (all bins if none)
};

template <typename T>
__global__ void __launch_bounds__(kSampleThreads) sample_top_p_kernel(
    const T* __restrict__ logits, int64_t row_stride, int V, float top_p, int64_t* tokens,
    T* conf) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* hp = reinterpret_cast<unsigned long long*>(smem);   // [kBins]
  unsigned long long* he = hp + kBins;                                     // [kBins]
  uint32_t* cnt = reinterpret_cast<uint32_t*>(he + kBins);                 // [kBins]
  __shared__ float red[kSampleThreads / 32];
  __shared__ long long redl[kSampleThreads / 32];
  __shared__ unsigned long long sp[kSampleThreads / 32], se[kSampleThreads / 32];
  __shared__ Walk walk;

  const T* x = logits + static_cast<int64_t>(blockIdx.x) * row_stride;
  const int tid = threadIdx.x;

  float mx = -INFINITY;
  for (int i = tid; i < V; i += kSampleThreads) mx = fmaxf(mx, Elt<T>::to_f(x[i]));
  const float m = block_max(mx, red);
  // level-0 bin of a logit: bins of 1/128 logit below the maximum, the last bin holding
  // every token more than 32 below it (their total probability is under V * e^-32);
  // monotone in l (the subtraction and the scaling by 128 are)
  auto bin0 = [&](float l) {
    const float d = (m - l) * 128.0f;
    const int db = d < static_cast<float>(kBins - 1) ? static_cast<int>(d) : kBins - 1;
    return kBins - 1 - db;                     // larger logit -> higher bin
  };
  // the normaliser and the level-0 bin counts in one pass
  for (int b = tid; b < kBins; b += kSampleThreads) cnt[b] = 0;
  __syncthreads();
  float z = 0.f;
  for (int i = tid; i < V; i += kSampleThreads) {
    const float l = Elt<T>::to_f(x[i]);
    z += expf(l - m);
    atomicAdd(&cnt[bin0(l)], 1u);
  }
  const float Z = block_sum(z, red);

  // ---- select of the crossing logit.  Level 0 (bins of bin0): the bin counts bound the
  // probability in each bin (p of a bin-d token lies within exp(-(d+1)/128)/Z and
  // exp(-d/128)/Z, give or take the rounding to T), which brackets the crossing bin;
  // an exact pass then sums p and exp(l - m) over the bins above the bracket in
  // registers and histograms only the bracket.  Later levels refine inside the crossing
  // bin's order-key range [klo, khi] with bins of 2^shift keys until one key is left.
  uint32_t klo = 0, khi = 0xFFFFFFFFu;
  unsigned long long p_above = 0, e_above = 0;
  bool crossed = true;
  int final_bin = -1, lv0_bin = -1;
  constexpr int per = kBins / kSampleThreads;
  {
    // cumulative bounds from the top bin; thread t owns bins [kBins-1-8t-7, kBins-1-8t]
    float lo_c[per], hi_c[per], lsum = 0.f, hsum = 0.f;
#pragma unroll
    for (int j = 0; j < per; ++j) {
      const int b = kBins - 1 - (tid * per + j);
      const int d = kBins - 1 - b;
      const float c = static_cast<float>(cnt[b]);
      const float phi = expf(-static_cast<float>(d) / 128.0f) / Z * (1.0f + 1.0f / 64.0f);
      const float plo = d == kBins - 1 ? 0.f : expf(-static_cast<float>(d + 1) / 128.0f) / Z * (1.0f - 1.0f / 64.0f);
      lsum += c * plo;
      hsum += c * phi;
      lo_c[j] = lsum;
      hi_c[j] = hsum;
    }
    // inclusive prefix over threads (warp shuffles + warps above)
    float il = lsum, ih = hsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float vl = __shfl_up_sync(0xffffffffu, il, o), vh = __shfl_up_sync(0xffffffffu, ih, o);
      if ((tid & 31) >= o) { il += vl; ih += vh; }
    }
    __shared__ float wl[kSampleThreads / 32], wh[kSampleThreads / 32];
    __shared__ int s_start, s_end;
    if ((tid & 31) == 31) { wl[tid >> 5] = il; wh[tid >> 5] = ih; }
    if (tid == 0) { s_start = -1; s_end = 0; }
    __syncthreads();
    float bl = il - lsum, bh = ih - hsum;
    for (int w = 0; w < (tid >> 5); ++w) { bl += wl[w]; bh += wh[w]; }
#pragma unroll
    for (int j = 0; j < per; ++j) {
      const int b = kBins - 1 - (tid * per + j);
      const float cl = bl + lo_c[j], ch = bh + hi_c[j];
      const float pl = bl + (j ? lo_c[j - 1] : 0.f), ph = bh + (j ? hi_c[j - 1] : 0.f);
      // first bin (from the top) where the upper / lower cumulative bound crosses
      if (round_t<T>(ch) > top_p && round_t<T>(ph) <= top_p) s_start = b;
      if (round_t<T>(cl) > top_p && round_t<T>(pl) <= top_p) s_end = b;
    }
    __syncthreads();
    const int b_start = s_start, b_end = s_end;
    if (b_start < 0) {
      crossed = false;                     // even the upper bound never crosses
    } else {
      // exact pass: register sums above the bracket, a histogram of the bracket
      for (int b = tid; b < kBins; b += kSampleThreads) { hp[b] = 0; he[b] = 0; }
      __syncthreads();
      unsigned long long rp = 0, re = 0;
      for (int i = tid; i < V; i += kSampleThreads) {
        const float l = Elt<T>::to_f(x[i]);
        const int b = bin0(l);
        if (b < b_end) continue;
        const float e = expf(l - m);
        const unsigned long long fp = to_fix(round_t<T>(__fdiv_rn(e, Z))), fe = to_fix(e);
        if (b > b_start) {
          rp += fp;
          re += fe;
        } else {
          atomicAdd(&hp[b], fp);
          atomicAdd(&he[b], fe);
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        rp += __shfl_xor_sync(0xffffffffu, rp, o);
        re += __shfl_xor_sync(0xffffffffu, re, o);
      }
      if ((tid & 31) == 0) { sp[tid >> 5] = rp; se[tid >> 5] = re; }
      if (tid == 0) walk.bin = -1;
      __syncthreads();
      if (tid == 0) {
        unsigned long long bp = 0, be = 0;
        for (int w = 0; w < kSampleThreads / 32; ++w) { bp += sp[w]; be += se[w]; }
        for (int b = b_start; b >= b_end; --b) {
          const unsigned long long np = bp + hp[b];
          if (np != bp && round_t<T>(from_fix(np)) > top_p) {
            walk.bin = b;
            walk.p_above = bp;
            walk.e_above = be;
            break;
          }
          bp = np;
          be += he[b];
        }
      }
      __syncthreads();
      if (walk.bin < 0) {
        crossed = false;
      } else {
        const int b = walk.bin;
        p_above = walk.p_above;
        e_above = walk.e_above;
        // a key range holding the bin's logit interval, widened for the rounding of the
        // bin arithmetic (values of the neighbouring bins inside it are excluded by the
        // level-0 bin test of the later levels)
        const int d = kBins - 1 - b;
        constexpr uint32_t kMargin = 1u << 12;
        const uint32_t k_hi = order_key(d == 0 ? m : m - static_cast<float>(d) / 128.0f);
        const uint32_t k_lo = d == kBins - 1 ? 0u : order_key(m - static_cast<float>(d + 1) / 128.0f);
        klo = k_lo > kMargin ? k_lo - kMargin : 0u;
        khi = k_hi < 0xFFFFFFFFu - kMargin ? k_hi + kMargin : 0xFFFFFFFFu;
        lv0_bin = b;
      }
      __syncthreads();
    }
  }
  for (int lv = 1; lv < 6 && crossed; ++lv) {
    const uint32_t span = khi - klo;
    const int shift = max(0, 32 - __clz(span) - 12);
    for (int b = tid; b < kBins; b += kSampleThreads) { hp[b] = 0; he[b] = 0; cnt[b] = 0; }
    __syncthreads();
    for (int i = tid; i < V; i += kSampleThreads) {
      const float l = Elt<T>::to_f(x[i]);
      const uint32_t key = order_key(l);
      if (key < klo || key > khi) continue;
      if (bin0(l) != lv0_bin) continue;        // counted in a neighbouring level-0 bin
      const int b = static_cast<int>((key - klo) >> shift);
      const float e = expf(l - m);
      const float p = round_t<T>(__fdiv_rn(e, Z));
      if (shift == 0) atomicAdd(&cnt[b], 1u);  // counts: the exact-key level only
      atomicAdd(&hp[b], to_fix(p));
      atomicAdd(&he[b], to_fix(e));
    }
    __syncthreads();
    // suffix sums from the top bin: thread t owns bins [kBins-1-8t-7, kBins-1-8t]
    unsigned long long mp = 0, me = 0;
#pragma unroll
    for (int j = 0; j < per; ++j) {
      const int b = kBins - 1 - (tid * per + j);
      mp += hp[b];
      me += he[b];
    }
    // exclusive scan of (mp, me) over threads: warp shuffles, then the warps above
    unsigned long long ip = mp, ie = me;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long vp = __shfl_up_sync(0xffffffffu, ip, o);
      const unsigned long long ve = __shfl_up_sync(0xffffffffu, ie, o);
      if ((tid & 31) >= o) { ip += vp; ie += ve; }
    }
    if ((tid & 31) == 31) { sp[tid >> 5] = ip; se[tid >> 5] = ie; }
    if (tid == 0) walk.bin = -1;
    __syncthreads();
    unsigned long long bp = p_above + ip - mp, be = e_above + ie - me;
    for (int w = 0; w < (tid >> 5); ++w) { bp += sp[w]; be += se[w]; }
#pragma unroll
    for (int j = 0; j < per; ++j) {
      const int b = kBins - 1 - (tid * per + j);
      const unsigned long long np = bp + hp[b];
      if (np != bp && round_t<T>(from_fix(np)) > top_p && round_t<T>(from_fix(bp)) <= top_p) {
        walk.bin = b;            // the crossing is unique: the prefix sums only grow
        walk.p_above = bp;
        walk.e_above = be;
      }
      bp = np;
      be += he[b];
    }
    __syncthreads();
    if (walk.bin < 0) {          // never crosses: every token is kept
      crossed = false;
      break;
    }
    const int b = walk.bin;
    p_above = walk.p_above;
    e_above = walk.e_above;
    klo = klo + (static_cast<uint32_t>(b) << shift);
    khi = min(khi, klo + ((1u << shift) - 1u));
    if (shift == 0) { final_bin = b; break; }
    __syncthreads();
  }
  if (final_bin < 0) crossed = false;          // not narrowed to one key: keep every token
  // the crossing value's order key
  const uint32_t key_star = klo;

  // ---- the crossing value: how many of its tokens are kept; the kept normaliser
  float Zk;
  uint32_t key_lo;               // tokens with key >= key_lo are kept (candidates)
  if (crossed) {
    const uint32_t c = cnt[final_bin];
    const float lstar = key_value(key_star);
    const float estar = expf(lstar - m);
    const float pstar = round_t<T>(__fdiv_rn(estar, Z));
    float s = from_fix(p_above);
    uint32_t kept = c;
    for (uint32_t k = 1; k <= c; ++k) {
      s += pstar;
      if (round_t<T>(s) > top_p) { kept = k; break; }
    }
    Zk = from_fix(e_above) + static_cast<float>(kept) * estar;
    key_lo = key_star;
  } else {
    Zk = Z;
    key_lo = 0;
  }
  const float qmax = round_t<T>(__fdiv_rn(1.0f, Zk));

  // ---- argmax of the filtered probabilities: first index attaining qmax.  Only logits
  // with exp(l - m) within a few ulps of 1 can round to qmax (bf16: 2^-8 relative, so
  // l > m - 1/64 is a safe superset; fp32: l > m - 2^-16).
  const float window = sizeof(T) == 2 ? 1.0f / 64.0f : 1.0f / 65536.0f;
  long long best = LLONG_MAX;
  for (int i = tid; i < V; i += kSampleThreads) {
    const float l = Elt<T>::to_f(x[i]);
    if (l < m - window || order_key(l) < key_lo) continue;
    const float q = round_t<T>(__fdiv_rn(expf(l - m), Zk));
    if (q == qmax) { best = i; break; }          // strided: the first hit is this thread's smallest
  }
  best = block_min_ll(best, redl);
  if (tid == 0) {
    tokens[blockIdx.x] = best == LLONG_MAX ? 0 : best;
    conf[blockIdx.x] = Elt<T>::from_f(qmax);
  }
}

}  // namespace

size_t sample_top_p_smem() { return kBins * (2 * sizeof(unsigned long long) + sizeof(uint32_t)); }

cudaError_t launch_sample_top_p(int dtype, const void* logits, int64_t rows, int V,
                                int64_t row_stride, float top_p, int64_t* tokens, void* conf,
                                cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const size_t smem = sample_top_p_smem();
  if (dtype == BF16) {
    static bool configured = false;
    if (!configured) {
      cudaError_t e = cudaFuncSetAttribute(sample_top_p_kernel<__nv_bfloat16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      configured = true;
    }
    sample_top_p_kernel<__nv_bfloat16><<<static_cast<unsigned>(rows), kSampleThreads, smem, st>>>(
        static_cast<const __nv_bfloat16*>(logits), row_stride, V, top_p, tokens,
        static_cast<__nv_bfloat16*>(conf));
  } else {
    static bool configured = false;
    if (!configured) {
      cudaError_t e = cudaFuncSetAttribute(sample_top_p_kernel<float>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      configured = true;
    }
    sample_top_p_kernel<float><<<static_cast<unsigned>(rows), kSampleThreads, smem, st>>>(
        static_cast<const float*>(logits), row_stride, V, top_p, tokens, static_cast<float*>(conf));
  }
  return launched();
}

}  // namespace sf
