// Exact chain-correction merge of the folded rows' attention state
// (specfold_chain_correction_gqa_kernel, triton_kernels.py:364-429; PyTorch reference
// fastdllm_v2_folded.py:183-204, which applies the same update one branch at a time).
//
// A folded row (b, n) inherits the query and the softmax state (m0, Z0, O0) of its
// source row src[b, n].  Between the source branch and b, every branch on the parent
// chain recomputed some positions e and so replaced the key/value the source saw at e
// (old = the parent's, kv_buf[src[par*N+e]*N+e]) with its own (new, kv_buf[cur*N+e]).
// The exact state for b is
//     m  = max(m0, max over new keys of q.k_new * scale)
//     Z  = Z0 exp(m0 - m) + sum_e (exp(s_new - m) - exp(s_old - m))
//     O  = (O0 Z0 exp(m0 - m) + sum_e (exp(s_new - m) v_new - exp(s_old - m) v_old)) / Z
// (the changes telescope along the chain).
//
// One CTA per (folded row, kv head).  The chain's entries are listed once in shared
// memory; each warp takes every fourth entry and keeps, per query head, an online state
// (reference max, sum and vector of the swapped contributions relative to it), with
// kMergeBatch entries' K/V rows in flight at a time.  The four warp states and the
// source state are merged in a fixed order, so results are deterministic.
#include "sf_kernels.cuh"

namespace sf {

constexpr int kMergeHeads = 8;   // query heads held in registers at a time
constexpr int kMergeBatch = 2;   // entries per warp whose loads are in flight together

template <typename T, int HD>
__global__ void __launch_bounds__(128, 4) merge_kernel(MergeParams p) {
  constexpr int DPL = HD / 32;
  __shared__ int s_new[kMaxRows], s_old[kMaxRows];
  __shared__ int s_br[kMaxBranches], s_par[kMaxBranches], s_off[kMaxBranches + 1];
  __shared__ int s_levels, s_total;
  __shared__ float s_m[4][kMergeHeads];
  __shared__ float s_z[4][kMergeHeads];
  __shared__ float s_o[4][kMergeHeads][HD];

  const int N = p.N, B1 = p.B1;
  int64_t r = blockIdx.x;
  const int kvh = blockIdx.y;
  if (p.frows != nullptr) {   // the compaction listed the folded rows: CTAs take them in order
    if (static_cast<int>(blockIdx.x) >= B1 * N - *p.count) return;
    r = p.frows[blockIdx.x];
  } else if (p.rec[r] != 0) {
    return;
  }
  const int64_t b = r / N, n = r % N;
  const int64_t srow = p.src[r];
  if (srow < 0 || srow >= B1) {
    if (threadIdx.x == 0) flag_error(p.err, SF_DEV_ERR_INDEX);
    return;
  }
  const int G = p.H / p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = p.H * HD, kvd = 2 * p.Hkv * HD;
  const T* qb = reinterpret_cast<const T*>(p.q_buf);
  const T* kvb = reinterpret_cast<const T*>(p.kv_buf);
  T* O = reinterpret_cast<T*>(p.O);
  const int64_t sflat = srow * N + n;

  // the chain b -> ... -> (child of srow), with each branch's entry offset
  if (threadIdx.x == 0) {
    int64_t cur = b;
    int off = 0, L = 0;
    while (cur != srow && L < B1) {
      const int cnt = p.segcnt[cur];
      const int64_t pc = p.par_idx[cur];
      s_br[L] = static_cast<int>(cur);
      s_par[L] = static_cast<int>(pc);
      s_off[L] = off;
      off += cnt;
      cur = pc;
      ++L;
      if (cur < 0 || cur >= B1) break;
    }
    s_off[L] = off;
    s_levels = (cur == srow) ? L : -1;
    s_total = off;
    if (cur != srow) flag_error(p.err, SF_DEV_ERR_DEPTH);
  }
  __syncthreads();
  const int levels = s_levels, total = s_total;
  if (levels < 0) return;
  for (int e = threadIdx.x; e < total; e += blockDim.x) {
    int l = 0;
    while (l + 1 < levels && s_off[l + 1] <= e) ++l;
    const int i = e - s_off[l];
    const int64_t rn = p.seg[static_cast<int64_t>(s_br[l]) * N + i];
    const int64_t pos = rn % N;
    const int64_t ro = p.src[static_cast<int64_t>(s_par[l]) * N + pos] * N + pos;
    s_new[e] = static_cast<int>(rn);
    s_old[e] = static_cast<int>(ro);
  }
  __syncthreads();

  for (int g0 = 0; g0 < G; g0 += kMergeHeads) {
    const int gn = min(kMergeHeads, G - g0);
    float q[kMergeHeads][DPL];
#pragma unroll
    for (int gi = 0; gi < kMergeHeads; ++gi)
#pragma unroll
      for (int t = 0; t < DPL; ++t)
        q[gi][t] = gi < gn ? Elt<T>::to_f(qb[sflat * qd + (kvh * G + g0 + gi) * HD + lane + 32 * t])
                           : 0.f;
    // this warp's online state per head, relative to mr
    float mr[kMergeHeads], zl[kMergeHeads], ol[kMergeHeads][DPL];
#pragma unroll
    for (int gi = 0; gi < kMergeHeads; ++gi) {
      mr[gi] = -INFINITY;
      zl[gi] = 0.f;
#pragma unroll
      for (int t = 0; t < DPL; ++t) ol[gi][t] = 0.f;
    }
    for (int e0 = warp * kMergeBatch; e0 < total; e0 += 4 * kMergeBatch) {
      float kn[kMergeBatch][DPL], ko[kMergeBatch][DPL], vn[kMergeBatch][DPL], vo[kMergeBatch][DPL];
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) {
        const int e = e0 + u;
        const int64_t rn = e < total ? s_new[e] : s_new[e0];
        const int64_t ro = e < total ? s_old[e] : s_old[e0];
#pragma unroll
        for (int t = 0; t < DPL; ++t) {
          const int d = lane + 32 * t;
          kn[u][t] = Elt<T>::to_f(kvb[rn * kvd + kvh * HD + d]);
          ko[u][t] = Elt<T>::to_f(kvb[ro * kvd + kvh * HD + d]);
          vn[u][t] = Elt<T>::to_f(kvb[rn * kvd + (p.Hkv + kvh) * HD + d]);
          vo[u][t] = Elt<T>::to_f(kvb[ro * kvd + (p.Hkv + kvh) * HD + d]);
        }
      }
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) {
        if (e0 + u >= total) break;
#pragma unroll
        for (int gi = 0; gi < kMergeHeads; ++gi) {
          if (gi >= gn) break;
          float sn = 0.f, so = 0.f;
#pragma unroll
          for (int t = 0; t < DPL; ++t) {
            sn = fmaf(q[gi][t], kn[u][t], sn);
            so = fmaf(q[gi][t], ko[u][t], so);
          }
          sn = warp_sum(sn) * p.scale;
          so = warp_sum(so) * p.scale;
          if (sn > mr[gi]) {   // new reference max: rescale what this warp holds
            const float c = expf(mr[gi] - sn);
            zl[gi] *= c;
#pragma unroll
            for (int t = 0; t < DPL; ++t) ol[gi][t] *= c;
            mr[gi] = sn;
          }
          const float an = expf(sn - mr[gi]);
          const float ao = expf(so - mr[gi]);
          zl[gi] += an - ao;
#pragma unroll
          for (int t = 0; t < DPL; ++t) ol[gi][t] += an * vn[u][t] - ao * vo[u][t];
        }
      }
    }
#pragma unroll
    for (int gi = 0; gi < kMergeHeads; ++gi) {
      if (lane == 0) {
        s_m[warp][gi] = mr[gi];
        s_z[warp][gi] = zl[gi];
      }
#pragma unroll
      for (int t = 0; t < DPL; ++t) s_o[warp][gi][lane + 32 * t] = ol[gi][t];
    }
    __syncthreads();
    for (int gi = warp; gi < gn; gi += 4) {
      const int h = kvh * G + g0 + gi;
      const float m0 = p.M[sflat * p.H + h];
      float mn = m0;
#pragma unroll
      for (int w = 0; w < 4; ++w) mn = fmaxf(mn, s_m[w][gi]);
      float cw[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) cw[w] = s_m[w][gi] == -INFINITY ? 0.f : expf(s_m[w][gi] - mn);
      const float Zs = p.Z[sflat * p.H + h] * expf(m0 - mn);
      float Z = Zs;
#pragma unroll
      for (int w = 0; w < 4; ++w) Z += s_z[w][gi] * cw[w];
#pragma unroll
      for (int t = 0; t < DPL; ++t) {
        const int d = lane + 32 * t;
        float num = Elt<T>::to_f(O[sflat * qd + h * HD + d]) * Zs;
#pragma unroll
        for (int w = 0; w < 4; ++w) num += s_o[w][gi][d] * cw[w];
        O[r * qd + h * HD + d] = Elt<T>::from_f(num / Z);
      }
      if (lane == 0) {
        p.M[r * p.H + h] = mn;
        p.Z[r * p.H + h] = Z;
      }
    }
    __syncthreads();
  }
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
  if (p.H % p.Hkv != 0 || p.B1 * p.N > kMaxRows || p.B1 > kMaxBranches)
    return cudaErrorInvalidValue;
  return dtype == BF16 ? merge_t<__nv_bfloat16>(p, st) : merge_t<float>(p, st);
}

}  // namespace sf
