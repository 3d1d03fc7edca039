// Attention of every block row (recomputed or folded) on the tcgen05 tensor cores, with
// S and O accumulated in TMEM: the bf16 path with a prefix, head_dim 128, N <= 32 block
// keys.  The prefix part of every ancestor row's softmax is already reduced to split
// partials by attn_prefix_kernel (attention_tc.cu).
//
// The math is that of attn_rows_kernel (attention.cu): a row r = b*N + n takes the query
// of its recomputing ancestor src_row = src[r]*N + n (triton_kernels.py:393-394), that
// query's retained prefix state, and branch b's own N block keys kv_buf[src[b*N+j]*N+j]
// (the in-block tile of specfold_flash_attn_gqa_kernel, triton_kernels.py:343-361).
//
// One CTA per (branch b, kv head, tile of tasks); task t = n*G + g is position n of the
// branch with q head kvh*G + g, and a tile of up to 128 tasks is the MMA's M = 128 rows
// (64-task tiles, the other rows zero, when 128 would leave SMs idle):
//   1. every thread gathers the tile's query rows, the branch's block keys and values
//      into shared memory in the 128-byte-swizzled layouts the MMA descriptors read
//      (query and keys K-major, values MN-major), and merges each task's split
//      partials into the prefix state (m_pre, l_pre, O_pre = sum_s w_s O_s);
//   2. one thread issues S = Q K^T (M 128, N 32, K = head_dim) into TMEM;
//   3. warps 0-3 (one task row per thread, TMEM lane quarter = warp) read their S row,
//      update the prefix state by the block scores and write P = exp(s - m) in bf16,
//      K-major, the rounding the reference applies before its P V dot;
//   4. one thread issues O_blk = P V (M 128, N = head_dim, K 32) into TMEM;
//   5. all sixteen warps (four per lane quarter, a quarter of the dims each) read O_blk and store
//      O = (exp(m_pre - m) O_pre + O_blk) / l in bf16; M = m, Z = l.
// Every mbarrier wait is bounded; TMEM is freed on every path.
#include <cstdlib>
#include <mutex>

#include "sf_kernels.cuh"

namespace sf {

namespace {

constexpr int kTcTasks = 128;        // tasks per CTA = MMA M
constexpr int kTcKeys = 32;          // block keys (MMA N of S, K of P V)
constexpr int kTcSplits = 16;        // prefix split partials merged per task
// sixteen warps: the split merge and the gathers are bound by the loads each SM keeps in
// flight, so more warps per CTA (one CTA per SM) move the partials faster
constexpr int kTcThreads = 512;

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// byte offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

template <int HD>
__global__ void __launch_bounds__(kTcThreads, 1)
    attn_rows_tc_kernel(AttnParams p, const float* part_O, const float* part_ml, int splits,
                        int part_rows, int tpc) {
  static_assert(HD == 128, "head_dim 128");
  using T = __nv_bfloat16;
  constexpr int KCH = HD / 64;                       // 64-dim boxes per row
  constexpr int kQBox = kTcTasks * 128;              // one 64-dim box of the query tile
  constexpr int kKBox = kTcKeys * 128;               // one 64-dim box of K (or V)
  constexpr int LDO = HD + 4;                        // fp32 row of the merged prefix output
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* sQ = smem;                          // [KCH][128 rows][128 B]
  unsigned char* sK = sQ + KCH * kQBox;              // [KCH][32 keys][128 B]
  unsigned char* sV = sK + KCH * kKBox;              // [KCH][32 keys][128 B] (MN-major)
  unsigned char* sP = sV + KCH * kKBox;              // [128 rows][128 B] (keys 0..31 used)
  float* sO = reinterpret_cast<float*>(sP + kTcTasks * 128);   // [128][LDO]
  float* sW = sO + kTcTasks * LDO;                   // [128][kTcSplits]
  float* sM = sW + kTcTasks * kTcSplits;             // [128] prefix max, then the new max
  float* sL = sM + kTcTasks;                         // [128] prefix sum, then the new sum
  float* sA = sL + kTcTasks;                         // [128] rescale of the prefix output
  uint64_t* bars = reinterpret_cast<uint64_t*>(sA + kTcTasks);
  uint64_t* s_full = bars;
  uint64_t* o_full = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  __shared__ int s_src[kTcKeys];

  // launched with programmatic stream serialization when that is enabled: every read of
  // an earlier kernel's output (src, queries, block K / V, split partials) comes after
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int G = p.H / p.Hkv;
  const int t0 = blockIdx.z * tpc;                   // tpc <= 128 tasks of this CTA
  const int ntasks = min(tpc, p.N * G - t0);
  if (ntasks <= 0) return;                           // uniform per CTA
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = p.H * HD;
  const int64_t kvd = 2LL * p.Hkv * HD;
  const T* qb = reinterpret_cast<const T*>(p.q_buf);
  const T* kvb = reinterpret_cast<const T*>(p.kv_buf);

  if (tid == 0) {
    mbar_init(s_full, 1);
    mbar_init(o_full, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);                      // S: columns [0, 32); O: [128, 256)
    tmem_relinquish();
  }
  if (tid < p.N) {
    int64_t s = p.src[static_cast<int64_t>(b) * p.N + tid];
    if (s < 0 || s >= p.B1) { flag_error(p.err, SF_DEV_ERR_INDEX); s = b; }
    s_src[tid] = static_cast<int>(s);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  // ---- 1. query rows, block K / V (zeros past the tasks / keys) into the swizzled tiles;
  // every load of a thread is issued before any of its stores
  {
    constexpr int VPR = HD / 8;                       // 16-byte chunks per row
    constexpr int QV = kTcTasks * VPR / kTcThreads;   // query chunks per thread
    constexpr int KV = kTcKeys * VPR / kTcThreads;    // key / value chunks per thread
    uint4 qv[QV], kv[KV], vv[KV];
#pragma unroll
    for (int u = 0; u < QV; ++u) {
      const int i = tid + u * kTcThreads, r = i / VPR, c = i % VPR;
      qv[u] = make_uint4(0, 0, 0, 0);
      if (r < ntasks) {
        const int t = t0 + r, n = t / G, g = t % G;
        const int64_t qrow = static_cast<int64_t>(s_src[n]) * p.N + n;
        qv[u] = *reinterpret_cast<const uint4*>(qb + qrow * qd + (kvh * G + g) * HD + c * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < KV; ++u) {
      const int i = tid + u * kTcThreads, j = i / VPR, c = i % VPR;
      kv[u] = vv[u] = make_uint4(0, 0, 0, 0);
      if (j < p.N) {
        const int64_t o = (static_cast<int64_t>(s_src[j]) * p.N + j) * kvd;
        kv[u] = *reinterpret_cast<const uint4*>(kvb + o + kvh * HD + c * 8);
        vv[u] = *reinterpret_cast<const uint4*>(kvb + o + (p.Hkv + kvh) * HD + c * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < QV; ++u) {
      const int i = tid + u * kTcThreads, r = i / VPR, c = i % VPR;
      *reinterpret_cast<uint4*>(sQ + (c >> 3) * kQBox + sw128(r, c & 7)) = qv[u];
    }
    // K: row = key, K-major over the dims; V: row = key, MN-major over the dims (the
    // same byte pattern: 64 dims per 128-byte row, one box per 64 dims)
#pragma unroll
    for (int u = 0; u < KV; ++u) {
      const int i = tid + u * kTcThreads, j = i / VPR, c = i % VPR;
      *reinterpret_cast<uint4*>(sK + (c >> 3) * kKBox + sw128(j, c & 7)) = kv[u];
      *reinterpret_cast<uint4*>(sV + (c >> 3) * kKBox + sw128(j, c & 7)) = vv[u];
    }
  }
  fence_async_smem();
  __syncthreads();

  // ---- 2. S = Q K^T
  if (tid == 0) {
    tc_fence_after();
    const uint32_t id_s = idesc_bf16(128, kTcKeys);
    const uint32_t q_s = smem_u32(sQ), k_s = smem_u32(sK);
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk)
      umma_f16(tS, sdesc_kmajor_sw128(q_s + (kk >> 2) * kQBox + (kk & 3) * 32),
               sdesc_kmajor_sw128(k_s + (kk >> 2) * kKBox + (kk & 3) * 32), id_s,
               kk > 0 ? 1u : 0u);
    umma_commit(s_full);
  }

  // ---- 1b. prefix state of every task from its ancestor row's split partials
  if (tid < kTcTasks) {
    float mx = -INFINITY;
    float ms[kTcSplits];
    int64_t qi = 0;
    if (tid < ntasks) {
      const int t = t0 + tid, n = t / G;
      qi = (static_cast<int64_t>(s_src[n]) * p.N + n) * G + t % G;
    }
#pragma unroll
    for (int s = 0; s < kTcSplits; ++s) {
      ms[s] = -INFINITY;
      if (s < splits && tid < ntasks)
        ms[s] = part_ml[2 * ((static_cast<int64_t>(s) * p.Hkv + kvh) * part_rows + qi)];
      mx = fmaxf(mx, ms[s]);
    }
    float l = 0.f;
#pragma unroll
    for (int s = 0; s < kTcSplits; ++s) {
      const float w = ms[s] == -INFINITY ? 0.f : expf(ms[s] - mx);
      sW[tid * kTcSplits + s] = w;
      if (s < splits && tid < ntasks)
        l = fmaf(part_ml[2 * ((static_cast<int64_t>(s) * p.Hkv + kvh) * part_rows + qi) + 1], w, l);
    }
    sM[tid] = mx;
    sL[tid] = l;
  }
  __syncthreads();
  // merged prefix output: items (row, 4 dims), two items per thread at a time with all
  // their split partials (four splits per round) in flight together (four items spilled
  // at sixteen warps' 128 registers per thread)
  constexpr int DQ = HD / 4;
  constexpr int IT = 2;
  for (int i0 = tid; i0 < kTcTasks * DQ; i0 += IT * kTcThreads) {
    float4 acc[IT];
    int64_t base[IT];
    bool live[IT];
#pragma unroll
    for (int k = 0; k < IT; ++k) {
      const int i = i0 + k * kTcThreads, r = i / DQ, dq = i % DQ;
      acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      live[k] = i < kTcTasks * DQ && r < ntasks;
      base[k] = 0;
      if (live[k]) {
        const int t = t0 + r, n = t / G;
        const int64_t qi = (static_cast<int64_t>(s_src[n]) * p.N + n) * G + t % G;
        base[k] = qi * HD + dq * 4;
      }
    }
    for (int s0 = 0; s0 < splits; s0 += 4) {
      float4 o[IT][4];
#pragma unroll
      for (int k = 0; k < IT; ++k)
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (live[k] && s0 + u < splits)
            o[k][u] = __ldcg(reinterpret_cast<const float4*>(
                part_O + (static_cast<int64_t>(s0 + u) * p.Hkv + kvh) * part_rows * HD + base[k]));
#pragma unroll
      for (int k = 0; k < IT; ++k) {
        const int r = (i0 + k * kTcThreads) / DQ;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (live[k] && s0 + u < splits) {
            const float w = sW[r * kTcSplits + s0 + u];
            acc[k].x = fmaf(o[k][u].x, w, acc[k].x);
            acc[k].y = fmaf(o[k][u].y, w, acc[k].y);
            acc[k].z = fmaf(o[k][u].z, w, acc[k].z);
            acc[k].w = fmaf(o[k][u].w, w, acc[k].w);
          }
      }
    }
#pragma unroll
    for (int k = 0; k < IT; ++k) {
      const int i = i0 + k * kTcThreads;
      if (i < kTcTasks * DQ)
        *reinterpret_cast<float4*>(sO + (i / DQ) * LDO + (i % DQ) * 4) = acc[k];
    }
  }

  // ---- 3. softmax of the block scores on top of the prefix state, P in bf16
  bool ok = true;
  if (warp < 4) {
    const int r = warp * 32 + lane;                  // task row == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    ok = mbar_wait(s_full, 0, p.err);
    float sv[kTcKeys];
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      tmem_ld16(tS + lane_off, sv);
      tmem_ld16(tS + lane_off + 16, sv + 16);
      tmem_ld_wait();
    } else {
      ok = false;
#pragma unroll
      for (int j = 0; j < kTcKeys; ++j) sv[j] = 0.f;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kTcKeys; ++j) {
      sv[j] = j < p.N ? sv[j] * p.scale : -INFINITY;
      mx = fmaxf(mx, sv[j]);
    }
    const float m_pre = sM[r];
    const float m = fmaxf(m_pre, mx);
    const float al = m_pre == -INFINITY ? 0.f : expf(m_pre - m);
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < kTcKeys / 8; ++c) {
      uint32_t pk[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float e0 = expf(sv[8 * c + 2 * h] - m), e1 = expf(sv[8 * c + 2 * h + 1] - m);
        sum += e0 + e1;
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(e0, e1);
        pk[h] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      *reinterpret_cast<uint4*>(sP + sw128(r, c)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    sM[r] = m;
    sL[r] = fmaf(sL[r], al, sum);
    sA[r] = al;
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // ---- 4. O_blk = P V
  if (tid == 0) {
    const uint32_t id_pv = idesc_bf16(128, HD, 0, 1);
    const uint32_t p_s = smem_u32(sP), v_s = smem_u32(sV);
#pragma unroll
    for (int kk = 0; kk < kTcKeys / 16; ++kk)
      umma_f16(tO, sdesc_kmajor_sw128(p_s + kk * 32), sdesc_mnmajor_sw128(v_s + kk * 2048, kKBox),
               id_pv, kk > 0 ? 1u : 0u);
    umma_commit(o_full);
  }

  // ---- 5. O = (al * O_pre + O_blk) / l
  {
    const int q = warp & 3, part = warp >> 2;       // lane quarter, quarter of the dims
    const int r = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const bool done = mbar_wait(o_full, 0, p.err);
    const bool go = __all_sync(0xffffffffu, done);
    if (go) tc_fence_after();
    const float al = sA[r];
    const int t = t0 + r;
    const bool live = go && r < ntasks;
    const int n = t / G, h = kvh * G + t % G;
    const int64_t row = static_cast<int64_t>(b) * p.N + n;
    T* O = reinterpret_cast<T*>(p.O);
#pragma unroll
    for (int c = 0; c < HD / 4; c += 16) {
      float o[16];
      if (go) {
        tmem_ld16(tO + lane_off + part * (HD / 4) + c, o);
        tmem_ld_wait();
      }
      if (live) {
        const int d0 = part * (HD / 4) + c;
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float f0 = (al * sO[r * LDO + d0 + 2 * e] + o[2 * e]) / sL[r];
          const float f1 = (al * sO[r * LDO + d0 + 2 * e + 1] + o[2 * e + 1]) / sL[r];
          const __nv_bfloat162 b2 = __floats2bfloat162_rn(f0, f1);
          pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        uint4* dst = reinterpret_cast<uint4*>(O + row * qd + h * HD + d0);
        dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
    }
    if (live && part == 0) {
      p.M[row * p.H + h] = sM[r];
      p.Z[row * p.H + h] = sL[r];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

template <int HD>
cudaError_t rows_tc(const AttnParams& p, const float* part_O, const float* part_ml, int splits,
                    int part_rows, cudaStream_t st) {
  const int G = p.H / p.Hkv;
  // 128 tasks per CTA (the MMA's M), or 64 (the other rows zero) when that leaves fewer
  // than one CTA per SM: the gathers and the split merge, not the MMAs, set the time
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int tiles128 = (p.N * G + kTcTasks - 1) / kTcTasks;
  int tpc = p.B1 * p.Hkv * tiles128 < sms ? kTcTasks / 2 : kTcTasks;
  static const int forced = [] {       // SF_ROWS_TC_TASKS: tasks per CTA (32, 64 or 128)
    const char* v = getenv("SF_ROWS_TC_TASKS");
    const int t = v ? atoi(v) : 0;
    return (t == 32 || t == 64 || t == 128) ? t : 0;
  }();
  if (forced) tpc = forced;
  const dim3 grid(p.B1, p.Hkv, (p.N * G + tpc - 1) / tpc);
  constexpr int KCH = HD / 64;
  const size_t smem = 1024 + KCH * kTcTasks * 128 + 2 * KCH * kTcKeys * 128 + kTcTasks * 128 +
                      (static_cast<size_t>(kTcTasks) * (HD + 4) + kTcTasks * kTcSplits +
                       3 * kTcTasks) * 4 + 64;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(attn_rows_tc_kernel<HD>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem));
  });
  if (attr != cudaSuccess) return attr;
  const cudaError_t e = launch_ex(attn_rows_tc_kernel<HD>, grid, dim3(kTcThreads), smem, st,
                                  false, p, part_O, part_ml, splits, part_rows, tpc);
  if (e != cudaSuccess) return e;
  return launched();
}

}  // namespace

bool attention_rows_tc_ok(int dtype, const AttnParams& p, int splits) {
  const int G = p.Hkv > 0 ? p.H / p.Hkv : 0;
  return dtype == BF16 && p.hd == 128 && G >= 1 && p.H % p.Hkv == 0 && p.N >= 1 &&
         p.N <= kTcKeys && splits >= 1 && splits <= kTcSplits && p.B1 * p.N <= kMaxRows;
}

cudaError_t launch_attention_rows_tc(const AttnParams& p, const float* part_O,
                                     const float* part_ml, int splits, int part_rows,
                                     cudaStream_t st) {
  if (p.hd == 128) return rows_tc<128>(p, part_O, part_ml, splits, part_rows, st);
  return cudaErrorInvalidValue;
}

}  // namespace sf
