// Attention of the recomputed rows with retained softmax state (SIMT part) and the
// block KV-cache append.
//
// attn_simt_kernel: one CTA per (recomputed row, kv head); every query head of the kv
//   group attends to keys taken 32 at a time into shared memory: the prefix cache, then
//   the N in-block keys kv_buf[src[b*N+j]*N + j] (specfold_flash_attn_gqa_kernel,
//   triton_kernels.py:301-361; PyTorch: fastdllm_v2_folded.py:164-181).  Online softmax
//   in fp32; writes O (normalised), M = row max, Z = sum of exp.  On the bf16 path with
//   a prefix, the tensor-core kernel (attention_tc.cu) has already reduced the prefix to
//   per-split partials: the state starts from their log-sum-exp merge and only the
//   in-block keys are added here.  On the fp32 path it covers every key.
//
// kv_append_kernel: cache[h, P + t, :] = new[h, t, :] with 16-byte vectors.
// kv_commit_kernel: the same append from the forward's own kv_buf (branch 0's rows), at a
//   prefix length read on the device (the block commit forward of a decode loop).
//
// The chain-correction merge of the folded rows lives in merge.cu.
#include "sf_kernels.cuh"

namespace sf {

constexpr int kAttnKeys = 32;   // keys per smem tile (one per lane)
constexpr int kMaxGroup = 16;   // q heads per kv head

template <typename T, int HD>
__global__ void __launch_bounds__(128) attn_simt_kernel(AttnParams p, const float* part_O,
                                                        const float* part_ml, int splits,
                                                        int q_rows) {
  constexpr int DPL = HD / 32;           // dims per lane
  constexpr int V = Elt<T>::kVec;        // elements per 16-byte vector
  constexpr int VPR = HD / V;            // vectors per row
  constexpr int TILE_VEC = kAttnKeys * VPR / 128;   // vectors per thread per K (or V) tile
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
  const int P = prefix_len(p.P_dev, p.P, p.err);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = p.H * HD, kvd = 2 * p.Hkv * HD;
  const T* qb = reinterpret_cast<const T*>(p.q_buf);
  const T* kvb = reinterpret_cast<const T*>(p.kv_buf);
  const T* pk = reinterpret_cast<const T*>(p.pk);
  const T* pv = reinterpret_cast<const T*>(p.pv);

  for (int i = threadIdx.x; i < G * VPR; i += 128) {
    const int g = i / VPR, d0 = (i % VPR) * V;
    float v[V];
    load_vec<T>(qb + r * qd + (kvh * G + g) * HD + d0, v);
#pragma unroll
    for (int k = 0; k < V; ++k) qs[g][d0 + k] = v[k];
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
      // lane s holds split s's (m, l)
      float ms = -INFINITY, ls = 0.f;
      if (lane < splits) {
        const int64_t base = (static_cast<int64_t>(lane) * p.Hkv + kvh) * q_rows + qi;
        ms = part_ml[2 * base];
        ls = part_ml[2 * base + 1];
      }
      const float mx = warp_max(ms);
      const float w = (ms == -INFINITY) ? 0.f : expf(ms - mx);
      m[i] = mx;
      l[i] = warp_sum(ls * w);
      for (int s = 0; s < splits; ++s) {
        const float ws = __shfl_sync(0xffffffffu, w, s);
        if (ws == 0.f) continue;
        const int64_t base = (static_cast<int64_t>(s) * p.Hkv + kvh) * q_rows + qi;
#pragma unroll
        for (int t = 0; t < DPL; ++t) acc[i][t] = fmaf(part_O[base * HD + lane + 32 * t], ws, acc[i][t]);
      }
    }
  }
  const int total = P + p.N;
  const int key_begin = part_O != nullptr ? P : 0;
  for (int k0 = key_begin; k0 < total; k0 += kAttnKeys) {
    __syncthreads();
    if (threadIdx.x < kAttnKeys) {
      const int key = k0 + threadIdx.x;
      int64_t kr = -1;
      if (key >= P && key < total) {
        const int j = key - P;
        int64_t s = p.src[b * p.N + j];
        if (s < 0 || s >= p.B1) { flag_error(p.err, SF_DEV_ERR_INDEX); s = 0; }
        kr = s * p.N + j;
      }
      krow[threadIdx.x] = kr;
    }
    __syncthreads();
    // all of this thread's K and V vectors of the tile are in flight at once
    float kv[TILE_VEC][V], vv[TILE_VEC][V];
#pragma unroll
    for (int u = 0; u < TILE_VEC; ++u) {
      const int idx = threadIdx.x + 128 * u;
      const int t = idx / VPR, d0 = (idx % VPR) * V;
      const int key = k0 + t;
      if (key < P) {
        const int64_t o = kvh * p.kv_head_stride + static_cast<int64_t>(key) * HD + d0;
        load_vec<T>(pk + o, kv[u]);
        load_vec<T>(pv + o, vv[u]);
      } else if (key < total) {
        const int64_t o = krow[t] * kvd;
        load_vec<T>(kvb + o + kvh * HD + d0, kv[u]);
        load_vec<T>(kvb + o + (p.Hkv + kvh) * HD + d0, vv[u]);
      } else {
#pragma unroll
        for (int k = 0; k < V; ++k) kv[u][k] = vv[u][k] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < TILE_VEC; ++u) {
      const int idx = threadIdx.x + 128 * u;
      const int t = idx / VPR, d0 = (idx % VPR) * V;
#pragma unroll
      for (int k = 0; k < V; ++k) {
        ks[t][d0 + k] = kv[u][k];
        vs[t][d0 + k] = vv[u][k];
      }
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

// attn_rows_kernel: the attention output of EVERY row r = b*N + n of the block, recomputed
// or folded, in one pass.  A row's query is that of its recomputing ancestor
// src_row = src[r]*N + n (a folded row inherits the hidden state, hence q, of src_row;
// specfold_chain_correction_gqa_kernel, triton_kernels.py:393-394); its keys are the
// prefix plus branch b's own block keys kv_buf[src[b*N+j]*N + j].  The prefix part is
// shared by every row with the same query, so on the tensor-core path it comes from
// src_row's split partials (its retained softmax state over the prefix) and only the N
// block keys are visited here; otherwise the prefix keys are visited too.  This rebuilds
// a folded row from its partner's retained state directly, where the reference walks
// the ancestor chain and telescopes old/new key contributions (:396-428): the same
// softmax, with no cancellation.  M is the true row max (the reference keeps the
// running max m_new of the telescoping for folded rows); M and Z are not read by the
// rest of the forward.
//
// One CTA per (branch b, kv head, group of rpc positions); warp w owns tasks
// (position, q head) w, w+8, ... (at most kRowTasks per CTA).  Keys are staged 32 at a
// time in shared memory and shared by all the CTA's tasks.
constexpr int kRowTasks = 32;

template <int DPL>
struct VecF;
template <> struct VecF<4> { using type = float4; };
template <> struct VecF<2> { using type = float2; };

// DPL consecutive floats <-> array
__device__ __forceinline__ void vec_get(const float4& v, float* o) { o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w; }
__device__ __forceinline__ void vec_get(const float2& v, float* o) { o[0] = v.x; o[1] = v.y; }

template <typename T, int HD>
__global__ void __launch_bounds__(256) attn_rows_kernel(AttnParams p, const float* part_O,
                                                        const float* part_ml, int splits,
                                                        int part_rows, int rpc) {
  constexpr int DPL = HD / 32;            // consecutive dims per lane (4 or 2)
  using VD = typename VecF<DPL>::type;
  constexpr int V = Elt<T>::kVec;
  constexpr int VPR = HD / V;
  constexpr int KS = HD + 4;              // padded smem row: 16-byte aligned, conflict-free
  constexpr int TILE_VEC = (kAttnKeys * VPR + 255) / 256;
  constexpr int TPW = kRowTasks / 8;      // tasks per warp
  extern __shared__ __align__(16) float sm_rows[];
  float* qs = sm_rows;                                  // [kRowTasks][HD]
  float* ks = qs + kRowTasks * HD;                      // [32][KS]
  float* vs = ks + kAttnKeys * KS;                      // [32][KS]
  __shared__ int s_src[kMaxRows];                       // branch b's src per position

  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int n0 = blockIdx.z * rpc;
  const int nrows = min(rpc, p.N - n0);
  if (nrows <= 0) return;
  const int G = p.H / p.Hkv;
  const int ntasks = nrows * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = p.H * HD, kvd = 2 * p.Hkv * HD;
  const T* qb = reinterpret_cast<const T*>(p.q_buf);
  const T* kvb = reinterpret_cast<const T*>(p.kv_buf);
  const T* pk = reinterpret_cast<const T*>(p.pk);
  const T* pv = reinterpret_cast<const T*>(p.pv);

  // recomputing ancestor of every position of branch b: query rows of this CTA's
  // positions and rows of the branch's block keys
  for (int j = threadIdx.x; j < p.N; j += 256) {
    int64_t s = p.src[static_cast<int64_t>(b) * p.N + j];
    if (s < 0 || s >= p.B1) { flag_error(p.err, SF_DEV_ERR_INDEX); s = b; }
    s_src[j] = static_cast<int>(s);
  }
  __syncthreads();

  // prefix keys this branch sees: all P' (verify), or P' + b * N (prefill block b)
  const KeyRange kr = attn_keys(p.P_dev, p.P, p.prefill_rows, p.err);
  const int P = p.prefill_rows > 0 ? kr.base + b * p.N : kr.keys;
  const int key_begin = part_O != nullptr ? P : 0;
  const int total = P + p.N;
  float kv[TILE_VEC][V], vv[TILE_VEC][V];
  // keys [k0, k0 + 32) into registers: prefix cache, then branch b's block keys
  auto load_tile = [&](int k0) {
#pragma unroll
    for (int u = 0; u < TILE_VEC; ++u) {
      const int idx = threadIdx.x + 256 * u;
      const int t = idx / VPR, d0 = (idx % VPR) * V;
      const int key = k0 + t;
      if (t < kAttnKeys && key < P) {
        const int64_t o = kvh * p.kv_head_stride + static_cast<int64_t>(key) * HD + d0;
        load_vec<T>(pk + o, kv[u]);
        load_vec<T>(pv + o, vv[u]);
      } else if (t < kAttnKeys && key < total) {
        const int j = key - P;
        const int64_t o = (static_cast<int64_t>(s_src[j]) * p.N + j) * kvd;
        load_vec<T>(kvb + o + kvh * HD + d0, kv[u]);
        load_vec<T>(kvb + o + (p.Hkv + kvh) * HD + d0, vv[u]);
      } else {
#pragma unroll
        for (int k = 0; k < V; ++k) kv[u][k] = vv[u][k] = 0.f;
      }
    }
  };
  if (key_begin < total) load_tile(key_begin);

  // queries (every task's q row) into shared memory as fp32
  for (int i = threadIdx.x; i < kRowTasks * VPR; i += 256) {
    const int t = i / VPR, d0 = (i % VPR) * V;
    float v[V];
    if (t < ntasks) {
      const int n = n0 + t / G;
      const int64_t qrow = static_cast<int64_t>(s_src[n]) * p.N + n;
      load_vec<T>(qb + qrow * qd + (kvh * G + t % G) * HD + d0, v);
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k) v[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < V; ++k) qs[t * HD + d0 + k] = v[k];
  }

  float m[TPW], l[TPW], acc[TPW][DPL];
#pragma unroll
  for (int i = 0; i < TPW; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[i][d] = 0.f;
  }
  if (part_O != nullptr) {
    // the ancestor row's prefix state: merge of its split partials (lane s: split s's m, l)
    float pm[TPW], pl[TPW];
#pragma unroll
    for (int i = 0; i < TPW; ++i) {
      pm[i] = -INFINITY;
      pl[i] = 0.f;
      const int t = warp + 8 * i;
      if (t < ntasks && lane < splits) {
        const int n = n0 + t / G;
        const int64_t qi = (static_cast<int64_t>(s_src[n]) * p.N + n) * G + t % G;
        const int64_t base = (static_cast<int64_t>(lane) * p.Hkv + kvh) * part_rows + qi;
        pm[i] = part_ml[2 * base];
        pl[i] = part_ml[2 * base + 1];
      }
    }
#pragma unroll
    for (int i = 0; i < TPW; ++i) {
      const int t = warp + 8 * i;
      if (t >= ntasks) break;
      const int n = n0 + t / G;
      const int64_t qi = (static_cast<int64_t>(s_src[n]) * p.N + n) * G + t % G;
      const float mx = warp_max(pm[i]);
      const float w = (pm[i] == -INFINITY) ? 0.f : expf(pm[i] - mx);
      m[i] = mx;
      l[i] = warp_sum(pl[i] * w);
      for (int s0 = 0; s0 < splits; s0 += 4) {
        float o[4][DPL];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (s0 + u < splits) {
            const int64_t base = (static_cast<int64_t>(s0 + u) * p.Hkv + kvh) * part_rows + qi;
            vec_get(__ldcg(reinterpret_cast<const VD*>(part_O + base * HD) + lane), o[u]);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float ws = __shfl_sync(0xffffffffu, w, (s0 + u) & 31);
          if (s0 + u < splits) {
#pragma unroll
            for (int d = 0; d < DPL; ++d) acc[i][d] = fmaf(o[u][d], ws, acc[i][d]);
          }
        }
      }
    }
  }
  for (int k0 = key_begin; k0 < total; k0 += kAttnKeys) {
    __syncthreads();
#pragma unroll
    for (int u = 0; u < TILE_VEC; ++u) {
      const int idx = threadIdx.x + 256 * u;
      const int t = idx / VPR, d0 = (idx % VPR) * V;
      if (t < kAttnKeys) {
#pragma unroll
        for (int k = 0; k < V; k += 4) {
          *reinterpret_cast<float4*>(ks + t * KS + d0 + k) =
              make_float4(kv[u][k], kv[u][k + 1], kv[u][k + 2], kv[u][k + 3]);
          *reinterpret_cast<float4*>(vs + t * KS + d0 + k) =
              make_float4(vv[u][k], vv[u][k + 1], vv[u][k + 2], vv[u][k + 3]);
        }
      }
    }
    __syncthreads();
    if (k0 + kAttnKeys < total) load_tile(k0 + kAttnKeys);   // next tile in flight meanwhile
    const bool valid = (k0 + lane) < total;
    // scores: lane = key; each K row read once for all of the warp's tasks
    float sc[TPW];
#pragma unroll
    for (int i = 0; i < TPW; ++i) sc[i] = 0.f;
    const float4* kr4 = reinterpret_cast<const float4*>(ks + lane * KS);
#pragma unroll 4
    for (int d4 = 0; d4 < HD / 4; ++d4) {
      const float4 kk = kr4[d4];
#pragma unroll
      for (int i = 0; i < TPW; ++i) {
        const float4 qq = reinterpret_cast<const float4*>(qs + (warp + 8 * i) * HD)[d4];
        sc[i] = fmaf(qq.x, kk.x, sc[i]);
        sc[i] = fmaf(qq.y, kk.y, sc[i]);
        sc[i] = fmaf(qq.z, kk.z, sc[i]);
        sc[i] = fmaf(qq.w, kk.w, sc[i]);
      }
    }
    float e[TPW];
#pragma unroll
    for (int i = 0; i < TPW; ++i) {
      e[i] = 0.f;
      if (warp + 8 * i >= ntasks) continue;
      const float s = valid ? sc[i] * p.scale : -INFINITY;
      const float mt = warp_max(s);
      const float mn = fmaxf(m[i], mt);
      const float alpha = m[i] == -INFINITY ? 0.f : expf(m[i] - mn);
      e[i] = valid ? expf(s - mn) : 0.f;
      l[i] = l[i] * alpha + warp_sum(e[i]);
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[i][d] *= alpha;
      m[i] = mn;
    }
    // P V: lane owns DPL consecutive dims; each V row read once for all tasks
#pragma unroll 4
    for (int jj = 0; jj < kAttnKeys; ++jj) {
      float vvv[DPL];
      vec_get(*reinterpret_cast<const VD*>(vs + jj * KS + lane * DPL), vvv);
#pragma unroll
      for (int i = 0; i < TPW; ++i) {
        const float pj = __shfl_sync(0xffffffffu, e[i], jj);
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[i][d] = fmaf(pj, vvv[d], acc[i][d]);
      }
    }
  }
  T* O = reinterpret_cast<T*>(p.O);
#pragma unroll
  for (int i = 0; i < TPW; ++i) {
    const int t = warp + 8 * i;
    if (t >= ntasks) break;
    const int64_t r = static_cast<int64_t>(b) * p.N + n0 + t / G;
    const int h = kvh * G + t % G;
#pragma unroll
    for (int d = 0; d < DPL; ++d)
      O[r * qd + h * HD + lane * DPL + d] = Elt<T>::from_f(acc[i][d] / l[i]);
    if (lane == 0) {
      p.M[r * p.H + h] = m[i];
      p.Z[r * p.H + h] = l[i];
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

// cache[h, P' + n, :] = kv_buf[n][(h | Hkv + h) * hd : ...] for the block's N rows of
// branch 0, P' read on the device: the commit forward's append of the committed block
template <typename T>
__global__ void kv_commit_kernel(const T* kvb, T* ck, T* cv, int64_t cs, const int32_t* P_dev,
                                 int P_max, int N, int Hkv, int hd, int* err) {
  constexpr int V = Elt<T>::kVec;
  const int P = prefix_len(P_dev, P_max, err);
  const int vecs_row = hd / V;
  const int64_t per_head = static_cast<int64_t>(N) * vecs_row;
  const int64_t total = static_cast<int64_t>(Hkv) * per_head;
  const int64_t kvd = 2LL * Hkv * hd;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int h = static_cast<int>(i / per_head);
    const int rem = static_cast<int>(i % per_head);
    const int n = rem / vecs_row, d0 = (rem % vecs_row) * V;
    const int64_t src = n * kvd + static_cast<int64_t>(h) * hd + d0;
    const int64_t dst = h * cs + static_cast<int64_t>(P + n) * hd + d0;
    *reinterpret_cast<uint4*>(ck + dst) = *reinterpret_cast<const uint4*>(kvb + src);
    *reinterpret_cast<uint4*>(cv + dst) =
        *reinterpret_cast<const uint4*>(kvb + src + static_cast<int64_t>(Hkv) * hd);
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
  if (p.H % p.Hkv != 0 || p.H / p.Hkv > kMaxGroup || splits > 32) return cudaErrorInvalidValue;
  return dtype == BF16 ? attn_t<__nv_bfloat16>(p, part_O, part_ml, splits, q_rows, st)
                       : attn_t<float>(p, part_O, part_ml, splits, q_rows, st);
}

template <typename T, int HD>
static cudaError_t rows_t(const AttnParams& p, const float* part_O, const float* part_ml,
                          int splits, int q_rows, cudaStream_t st) {
  const int G = p.H / p.Hkv;
  // positions per CTA: as few as keep the grid within one wave at two CTAs per SM
  // (register-bound), at most kRowTasks / G
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int slots = std::max(1, 2 * sms / std::max(1, p.B1 * p.Hkv));
  int rpc = (p.N + slots - 1) / slots;
  rpc = std::max(1, std::min(std::min(p.N, kRowTasks / G), rpc));
  const dim3 grid(p.B1, p.Hkv, (p.N + rpc - 1) / rpc);
  const size_t smem = (static_cast<size_t>(kRowTasks) * HD + 2 * kAttnKeys * (HD + 4)) * 4;
  static size_t configured = 0;
  if (configured < smem) {
    cudaError_t e = cudaFuncSetAttribute(attn_rows_kernel<T, HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured = smem;
  }
  const cudaError_t e = launch_ex(attn_rows_kernel<T, HD>, grid, dim3(256), smem, st, false, p,
                                 part_O, part_ml, splits, q_rows, rpc);
  if (e != cudaSuccess) return e;
  return launched();
}

cudaError_t launch_attention_rows_partials(int dtype, const AttnParams& p, const float* part_O,
                                           const float* part_ml, int splits, int q_rows,
                                           cudaStream_t st) {
  const int G = p.Hkv > 0 ? p.H / p.Hkv : 0;
  if (G <= 0 || p.H % p.Hkv != 0 || G > kRowTasks || splits > 32 ||
      p.B1 * p.N > kMaxRows || p.N > kMaxRows)
    return cudaErrorInvalidValue;
  if (dtype == BF16) {
    if (p.hd == 128) return rows_t<__nv_bfloat16, 128>(p, part_O, part_ml, splits, q_rows, st);
    if (p.hd == 64) return rows_t<__nv_bfloat16, 64>(p, part_O, part_ml, splits, q_rows, st);
  } else {
    if (p.hd == 128) return rows_t<float, 128>(p, part_O, part_ml, splits, q_rows, st);
    if (p.hd == 64) return rows_t<float, 64>(p, part_O, part_ml, splits, q_rows, st);
  }
  return cudaErrorInvalidValue;
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

cudaError_t launch_kv_commit(int dtype, const void* kv_buf, void* ck, void* cv, int64_t c_stride,
                             const int32_t* P_dev, int P, int N, int Hkv, int hd, int* err,
                             cudaStream_t st) {
  const int vec = dtype == BF16 ? 8 : 4;
  if (hd % vec != 0 || N <= 0) return cudaErrorInvalidValue;
  const int64_t total = static_cast<int64_t>(Hkv) * N * hd / vec;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 592));
  if (dtype == BF16)
    kv_commit_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(kv_buf), static_cast<__nv_bfloat16*>(ck),
        static_cast<__nv_bfloat16*>(cv), c_stride, P_dev, P, N, Hkv, hd, err);
  else
    kv_commit_kernel<float><<<blocks, 256, 0, st>>>(
        static_cast<const float*>(kv_buf), static_cast<float*>(ck), static_cast<float*>(cv),
        c_stride, P_dev, P, N, Hkv, hd, err);
  return launched();
}

}  // namespace sf
