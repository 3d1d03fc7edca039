// Attention of every block row (recomputed or folded) on the tensor cores: the bf16 path
// with a prefix, where the prefix part of each ancestor row's softmax is already reduced
// to split partials by attn_prefix_kernel (attention_tc.cu).
//
// Same result as attn_rows_kernel (attention.cu), which states the math: a row r = b*N+n
// uses the query of its recomputing ancestor src_row = src[r]*N + n (triton_kernels.py:
// 393-394), that query's retained prefix state, and branch b's own N block keys
// kv_buf[src[b*N+j]*N + j].  Here one CTA takes up to 32 (position, q head) tasks of one
// (branch, kv head); the 32 x N scores and the 32 x hd block output are mma.sync
// m16n8k16 bf16 tiles (two warps, one 16-task tile each): at N = 32 the block is 64 MMA
// instructions per tile, where the SIMT loop spent several thousand FMAs per warp.
//   1. stage src of the branch; load q rows, block K and V (bf16) into padded shared
//      memory, and the split partials (m, l) of every task;
//   2. merge the split partials of every (task, 4 dims) into the prefix state
//      O_pre = sum_s w_s O_s, w_s = exp(m_s - m_pre), l_pre = sum_s w_s l_s;
//   3. S = q K^T (fp32), online-softmax update of (m_pre, l_pre) by the block scores,
//      P = exp(S - m) in bf16 as the A fragments of O_blk = P V;
//   4. O = (exp(m_pre - m) O_pre + O_blk) / l, stored in bf16; M = m, Z = l.
// P in bf16 is the rounding the reference's Triton kernels apply before their P V dot.
#include <mutex>

#include "sf_kernels.cuh"

namespace sf {

namespace {

constexpr int kMmaTasks = 32;      // tasks (rows of the MMA A operand) per CTA
constexpr int kMmaKeys = 32;       // block keys handled (N <= 32)
constexpr int kMaxSplitsMma = 16;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_trans(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
// D += A (16x16 bf16, row) * B (16x8 bf16, col), fp32 accumulate
__device__ __forceinline__ void mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int HD>
__global__ void __launch_bounds__(256) attn_rows_mma_kernel(AttnParams p, const float* part_O,
                                                            const float* part_ml, int splits,
                                                            int part_rows, int rpc) {
  using T = __nv_bfloat16;
  constexpr int LDB = HD + 8;          // bf16 row of q / K / V: conflict-free ldmatrix
  constexpr int LDO = HD + 4;          // fp32 row of the merged prefix output
  constexpr int DQ = HD / 4;           // 4-dim groups per row
  constexpr int VPR = HD / 8;          // 16-byte vectors per bf16 row
  extern __shared__ __align__(16) unsigned char sm_mma[];
  T* sQ = reinterpret_cast<T*>(sm_mma);                 // [32][LDB]
  T* sK = sQ + kMmaTasks * LDB;                         // [32][LDB]
  T* sV = sK + kMmaKeys * LDB;                          // [32][LDB]
  float* sO = reinterpret_cast<float*>(sV + kMmaKeys * LDB);   // [32][LDO]
  float* sW = sO + kMmaTasks * LDO;                     // [32][kMaxSplitsMma] split weights
  float* sM = sW + kMmaTasks * kMaxSplitsMma;           // [32] prefix max
  float* sL = sM + kMmaTasks;                           // [32] prefix sum
  __shared__ int s_src[kMaxRows];

  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int n0 = blockIdx.z * rpc;
  const int nrows = min(rpc, p.N - n0);
  if (nrows <= 0) return;
  const int G = p.H / p.Hkv;
  const int ntasks = nrows * G;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = p.H * HD, kvd = 2 * p.Hkv * HD;
  const T* qb = reinterpret_cast<const T*>(p.q_buf);
  const T* kvb = reinterpret_cast<const T*>(p.kv_buf);

  for (int j = tid; j < p.N; j += 256) {
    int64_t s = p.src[static_cast<int64_t>(b) * p.N + j];
    if (s < 0 || s >= p.B1) { flag_error(p.err, SF_DEV_ERR_INDEX); s = b; }
    s_src[j] = static_cast<int>(s);
  }
  __syncthreads();

  // ---- 1. q rows, block K / V (16-byte vectors, zero past the tasks / keys)
  for (int i = tid; i < kMmaTasks * VPR; i += 256) {
    const int t = i / VPR, d = (i % VPR) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < ntasks) {
      const int n = n0 + t / G;
      const int64_t qrow = static_cast<int64_t>(s_src[n]) * p.N + n;
      v = *reinterpret_cast<const uint4*>(qb + qrow * qd + (kvh * G + t % G) * HD + d);
    }
    *reinterpret_cast<uint4*>(sQ + t * LDB + d) = v;
  }
  for (int i = tid; i < kMmaKeys * VPR; i += 256) {
    const int j = i / VPR, d = (i % VPR) * 8;
    uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    if (j < p.N) {
      const int64_t o = (static_cast<int64_t>(s_src[j]) * p.N + j) * kvd;
      kv = *reinterpret_cast<const uint4*>(kvb + o + kvh * HD + d);
      vv = *reinterpret_cast<const uint4*>(kvb + o + (p.Hkv + kvh) * HD + d);
    }
    *reinterpret_cast<uint4*>(sK + j * LDB + d) = kv;
    *reinterpret_cast<uint4*>(sV + j * LDB + d) = vv;
  }
  // split (m, l) of every task -> weights w_s = exp(m_s - m_pre), m_pre, l_pre
  if (tid < kMmaTasks) {
    const int t = tid;
    float ms[kMaxSplitsMma], ls[kMaxSplitsMma];
    float mx = -INFINITY;
    int64_t qi = 0;
    if (t < ntasks) {
      const int n = n0 + t / G;
      qi = (static_cast<int64_t>(s_src[n]) * p.N + n) * G + t % G;
    }
#pragma unroll
    for (int s = 0; s < kMaxSplitsMma; ++s) {
      ms[s] = -INFINITY;
      ls[s] = 0.f;
      if (s < splits && t < ntasks) {
        const int64_t base = (static_cast<int64_t>(s) * p.Hkv + kvh) * part_rows + qi;
        ms[s] = part_ml[2 * base];
        ls[s] = part_ml[2 * base + 1];
      }
      mx = fmaxf(mx, ms[s]);
    }
    float l = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxSplitsMma; ++s) {
      const float w = ms[s] == -INFINITY ? 0.f : expf(ms[s] - mx);
      sW[t * kMaxSplitsMma + s] = w;
      l = fmaf(ls[s], w, l);
    }
    sM[t] = mx;
    sL[t] = l;
  }
  __syncthreads();

  // ---- 2. merged prefix output O_pre = sum_s w_s O_s (relative to m_pre)
  for (int i = tid; i < kMmaTasks * DQ; i += 256) {
    const int t = i / DQ, dq = i % DQ;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < ntasks) {
      const int n = n0 + t / G;
      const int64_t qi = (static_cast<int64_t>(s_src[n]) * p.N + n) * G + t % G;
      float4 o[kMaxSplitsMma];
#pragma unroll
      for (int s = 0; s < kMaxSplitsMma; ++s)
        if (s < splits) {
          const int64_t base = (static_cast<int64_t>(s) * p.Hkv + kvh) * part_rows + qi;
          o[s] = __ldcg(reinterpret_cast<const float4*>(part_O + base * HD) + dq);
        }
#pragma unroll
      for (int s = 0; s < kMaxSplitsMma; ++s)
        if (s < splits) {
          const float w = sW[t * kMaxSplitsMma + s];
          acc.x = fmaf(o[s].x, w, acc.x);
          acc.y = fmaf(o[s].y, w, acc.y);
          acc.z = fmaf(o[s].z, w, acc.z);
          acc.w = fmaf(o[s].w, w, acc.w);
        }
    }
    *reinterpret_cast<float4*>(sO + t * LDO + dq * 4) = acc;
  }
  __syncthreads();
  if (warp >= 2) return;

  // ---- 3. warp w: tasks [16w, 16w + 16)
  const int g = lane >> 2, c = lane & 3;
  const int r0 = 16 * warp + g, r1 = r0 + 8;       // this thread's two task rows
  const uint32_t q_base = static_cast<uint32_t>(__cvta_generic_to_shared(sQ));
  const uint32_t k_base = static_cast<uint32_t>(__cvta_generic_to_shared(sK));
  const uint32_t v_base = static_cast<uint32_t>(__cvta_generic_to_shared(sV));
  float s_acc[kMmaKeys / 8][4];
#pragma unroll
  for (int nt = 0; nt < kMmaKeys / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) s_acc[nt][e] = 0.f;
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4(q_base + ((16 * warp + (lane & 15)) * LDB + kk * 16 + (lane >> 4) * 8) * 2, a0, a1, a2, a3);
#pragma unroll
    for (int nt = 0; nt < kMmaKeys / 8; ++nt) {
      uint32_t b0, b1;
      ldsm_x2(k_base + ((8 * nt + (lane & 7)) * LDB + kk * 16 + ((lane >> 3) & 1) * 8) * 2, b0, b1);
      mma_bf16(s_acc[nt], a0, a1, a2, a3, b0, b1);
    }
  }
  // softmax update of the prefix state by this block's keys (rows r0, r1)
  const float m_pre0 = sM[r0], m_pre1 = sM[r1];
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < kMmaKeys / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = 8 * nt + 2 * c + e;
      const bool valid = key < p.N;
      s_acc[nt][e] = valid ? s_acc[nt][e] * p.scale : -INFINITY;
      s_acc[nt][2 + e] = valid ? s_acc[nt][2 + e] * p.scale : -INFINITY;
      mx0 = fmaxf(mx0, s_acc[nt][e]);
      mx1 = fmaxf(mx1, s_acc[nt][2 + e]);
    }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float m0 = fmaxf(m_pre0, mx0), m1 = fmaxf(m_pre1, mx1);
  const float al0 = m_pre0 == -INFINITY ? 0.f : expf(m_pre0 - m0);
  const float al1 = m_pre1 == -INFINITY ? 0.f : expf(m_pre1 - m1);
  float sum0 = 0.f, sum1 = 0.f;
  uint32_t pa[kMmaKeys / 8][2];        // P rows r0 / r1 of each 8-key tile, bf16 pairs
#pragma unroll
  for (int nt = 0; nt < kMmaKeys / 8; ++nt) {
    const float e0 = expf(s_acc[nt][0] - m0), e1 = expf(s_acc[nt][1] - m0);
    const float e2 = expf(s_acc[nt][2] - m1), e3 = expf(s_acc[nt][3] - m1);
    sum0 += e0 + e1;
    sum1 += e2 + e3;
    pa[nt][0] = pack_bf16(e0, e1);
    pa[nt][1] = pack_bf16(e2, e3);
  }
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
  const float l0 = fmaf(sL[r0], al0, sum0), l1 = fmaf(sL[r1], al1, sum1);

  // ---- O_blk = P V, 8 dims per tile; merged with the prefix output and stored
  T* O = reinterpret_cast<T*>(p.O);
  const int t0 = r0, t1 = r1;
  const bool st0 = t0 < ntasks, st1 = t1 < ntasks;
  const int64_t row0 = static_cast<int64_t>(b) * p.N + n0 + (st0 ? t0 / G : 0);
  const int64_t row1 = static_cast<int64_t>(b) * p.N + n0 + (st1 ? t1 / G : 0);
  const int h0 = kvh * G + (st0 ? t0 % G : 0), h1 = kvh * G + (st1 ? t1 % G : 0);
#pragma unroll
  for (int dt = 0; dt < HD / 8; ++dt) {
    float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < kMmaKeys / 16; ++kk) {
      uint32_t b0, b1;
      ldsm_x2_trans(v_base + ((16 * kk + (lane & 15)) * LDB + dt * 8) * 2, b0, b1);
      mma_bf16(o, pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b0, b1);
    }
    const int d = dt * 8 + 2 * c;
    const float f00 = (al0 * sO[t0 * LDO + d] + o[0]) / l0;
    const float f01 = (al0 * sO[t0 * LDO + d + 1] + o[1]) / l0;
    const float f10 = (al1 * sO[t1 * LDO + d] + o[2]) / l1;
    const float f11 = (al1 * sO[t1 * LDO + d + 1] + o[3]) / l1;
    if (st0)
      *reinterpret_cast<__nv_bfloat162*>(O + row0 * qd + h0 * HD + d) = __floats2bfloat162_rn(f00, f01);
    if (st1)
      *reinterpret_cast<__nv_bfloat162*>(O + row1 * qd + h1 * HD + d) = __floats2bfloat162_rn(f10, f11);
  }
  if (c == 0) {
    if (st0) {
      p.M[row0 * p.H + h0] = m0;
      p.Z[row0 * p.H + h0] = l0;
    }
    if (st1) {
      p.M[row1 * p.H + h1] = m1;
      p.Z[row1 * p.H + h1] = l1;
    }
  }
}

template <int HD>
cudaError_t rows_mma(const AttnParams& p, const float* part_O, const float* part_ml, int splits,
                     int part_rows, cudaStream_t st) {
  const int G = p.H / p.Hkv;
  const int rpc = std::max(1, std::min(p.N, kMmaTasks / G));
  const dim3 grid(p.B1, p.Hkv, (p.N + rpc - 1) / rpc);
  constexpr int LDB = HD + 8, LDO = HD + 4;
  const size_t smem = static_cast<size_t>(kMmaTasks + 2 * kMmaKeys) * LDB * 2 +
                      (static_cast<size_t>(kMmaTasks) * LDO + kMmaTasks * kMaxSplitsMma +
                       2 * kMmaTasks) * 4;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(attn_rows_mma_kernel<HD>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem));
  });
  if (attr != cudaSuccess) return attr;
  const cudaError_t e = launch_ex(attn_rows_mma_kernel<HD>, grid, dim3(256), smem, st, false, p,
                                  part_O, part_ml, splits, part_rows, rpc);
  if (e != cudaSuccess) return e;
  return launched();
}

}  // namespace

bool attention_rows_mma_ok(int dtype, const AttnParams& p, int splits) {
  const int G = p.Hkv > 0 ? p.H / p.Hkv : 0;
  return dtype == BF16 && (p.hd == 128 || p.hd == 64) && G >= 1 && G <= kMmaTasks &&
         p.N <= kMmaKeys && splits >= 1 && splits <= kMaxSplitsMma && p.B1 * p.N <= kMaxRows;
}

cudaError_t launch_attention_rows_mma(const AttnParams& p, const float* part_O,
                                      const float* part_ml, int splits, int part_rows,
                                      cudaStream_t st) {
  if (p.hd == 128) return rows_mma<128>(p, part_O, part_ml, splits, part_rows, st);
  if (p.hd == 64) return rows_mma<64>(p, part_O, part_ml, splits, part_rows, st);
  return cudaErrorInvalidValue;
}

}  // namespace sf
