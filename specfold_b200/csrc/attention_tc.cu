// Tensor-core (tcgen05) attention over the shared prefix KV cache, split along the keys.
//
// Every recomputed row's queries attend to the same prefix keys of their kv head, so
// the prefix part is a dense flash-attention tile problem: queries of one kv head are
// packed (slot*G + g) 128 to a tile by the QKV epilogue (or pack_q_kernel), keys are
// streamed from the cache by TMA in blocks of 128, and per block
//     S = Q K^T              tcgen05.mma, accumulator in TMEM
//     softmax                4 warps, one query row per thread, running (m, l)
//     O += P V               P (bf16) from shared memory, V as the MN-major operand
// Each (query tile, kv head, key split) CTA writes its unnormalised partial (O, m, l)
// in fp32; attn_simt_kernel then merges the splits and adds the N in-block keys,
// which differ per branch (specfold_flash_attn_gqa_kernel, triton_kernels.py:301-361,
// covers both parts in one program per (row, kv head)).
//
// Warp 0 issues TMA, warp 1 owns TMEM and issues MMAs, warps 2-5 run the softmax.
// All mbarrier waits are bounded (sf_common.cuh).
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "sf_kernels.cuh"

namespace sf {

constexpr int kAttThreads = 320;   // TMA warp, MMA warp, 8 softmax warps
constexpr int kQT = 128;            // queries per tile (MMA M)
constexpr int kKB = 128;            // keys per block
constexpr int kMaxKvSplits = 16;
constexpr int kKeysPerSplit = 256;  // at least two key blocks per split

struct AttnTcParams {
  const int32_t* count;
  int bucket, G, q_rows, P, kv_rows, splits, keys_per_split, Hkv;
  float scale;
  float* part_O;    // [splits][Hkv][part_rows][HD]
  float* part_ml;   // [splits][Hkv][part_rows][2]
  // partial row of query qi = slot*G + g: qi itself, or rows[slot]*G + g (indexed by the
  // flat block row, for consumers that look rows up without the compaction order)
  const int64_t* rows;
  int part_rows;
  int* err;
  // device prefix length (nullptr: P).  P is then the bound the grid was sized for
  // (splits = kv_splits(P)); the kernel derives the split layout of the actual length the
  // way the host does, and the splits beyond it write empty partials (m = -inf, l = 0).
  const int32_t* P_dev;
  // batched prefill: rows of the prefill blocks (0 = off) and the block length; query
  // row of flat block row r attends to keys [0, P' + (r / block_N) * block_N)
  int prefill_rows, block_N;
};

// key splits of a prefix of P keys: at least kKeysPerSplit keys each, at most kMaxKvSplits
__host__ __device__ __forceinline__ int kv_splits_of(int P) {
  if (P <= 0) return 0;
  const int s = (P + kKeysPerSplit - 1) / kKeysPerSplit;
  return s < 1 ? 1 : (s > kMaxKvSplits ? kMaxKvSplits : s);
}
__host__ __device__ __forceinline__ int keys_per_split_of(int P, int S) {
  return S > 0 ? ((P + S - 1) / S + kKB - 1) / kKB * kKB : 0;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// AND over the 256 softmax threads (named barrier 1): keeps the softmax warps, which meet
// at named barriers, on the same iteration whatever each saw of a failed wait.
__device__ __forceinline__ bool softmax_vote(bool x) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 256, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(x))
      : "memory");
  return r != 0;
}

template <int HD>
__global__ void __launch_bounds__(kAttThreads, 1)
    attn_prefix_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, AttnTcParams p) {
  constexpr int KCH = HD / 64;                 // 64-column TMA boxes per row
  constexpr int kBox = 128 * 64 * 2;           // one 128-row box: 16 KB
  constexpr int QBYTES = KCH * kBox;
  constexpr int KVBYTES = KCH * kBox;
  constexpr int PBYTES = 2 * kBox;             // 128 queries x 128 keys bf16
  constexpr int HALF_KEYS = kKB / 2;           // keys (S columns) per softmax half
  constexpr int HALF_DIMS = HD / 2;            // O columns per softmax half
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* sQ = smem;
  unsigned char* sK = sQ + QBYTES;             // [2][KVBYTES]
  unsigned char* sV = sK + 2 * KVBYTES;        // [2][KVBYTES]
  unsigned char* sP = sV + 2 * KVBYTES;
  float* s_red = reinterpret_cast<float*>(sP + PBYTES);     // [2][128] half-row max / sum
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_red + 2 * kQT);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;    // [2]
  uint64_t* kv_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;     // [2] (S double-buffered in TMEM)
  uint64_t* p_full = bars + 7;
  uint64_t* pv_done = bars + 8;
  uint64_t* drain = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  pdl_trigger();
  pdl_wait();
  const int kvh = blockIdx.x, split = blockIdx.y, qt = blockIdx.z;
  const int count = min(*p.count, p.bucket);
  const int Mq = count * p.G;
  const int q0 = qt * kQT;
  if (q0 >= Mq) return;                        // uniform per CTA
  int P = p.P, kps = p.keys_per_split, P_base = p.P;
  if (p.P_dev != nullptr || p.prefill_rows > 0) {
    const KeyRange kr = attn_keys(p.P_dev, p.P, p.prefill_rows, p.err);
    P = kr.keys;
    P_base = kr.base;
    kps = keys_per_split_of(P, kv_splits_of(P));
  }
  // per query row: the keys it may see (prefill: its block's prefix; otherwise all P)
  auto row_limit = [&](int qi) -> int {
    if (p.prefill_rows == 0) return P;
    const int slot = min(qi, Mq - 1) / p.G;
    const int64_t fr = p.rows != nullptr ? p.rows[slot] : slot;
    return P_base + static_cast<int>(fr / p.block_N) * p.block_N;
  };
  const int k_begin = split * kps;
  // the tile's last row has the largest limit (rows ascend within a tile)
  const int k_end = min(min(P, row_limit(min(q0 + kQT, Mq) - 1)), k_begin + kps);
  const int nb = k_end > k_begin ? (k_end - k_begin + kKB - 1) / kKB : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
    }
    mbar_init(p_full, 256);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 2 * kKB;          // S buffers at columns 0 and 128

  if (warp == 0) {
    if (lane == 0 && nb > 0) {
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_last();   // every query tile of this head rereads it
      mbar_arrive_expect_tx(q_full, QBYTES);
      for (int c = 0; c < KCH; ++c)
        tma_load_2d(sQ + c * kBox, &tmQ, q_full, c * 64, kvh * p.q_rows + q0, pol_q);
      int issued = 0;
      for (int i = 0; i < nb; ++i) {
        const int s = i & 1;
        if (!mbar_wait(&kv_empty[s], ((i >> 1) & 1) ^ 1, p.err)) { *abort_flag = 1; break; }
        mbar_arrive_expect_tx(&kv_full[s], 2 * KVBYTES);
        const int krow = kvh * p.kv_rows + k_begin + i * kKB;
        for (int c = 0; c < KCH; ++c) {
          tma_load_2d(sK + s * KVBYTES + c * kBox, &tmK, &kv_full[s], c * 64, krow, pol_kv);
          tma_load_2d(sV + s * KVBYTES + c * kBox, &tmV, &kv_full[s], c * 64, krow, pol_kv);
        }
        ++issued;
      }
      mbar_wait(q_full, 0, p.err);
      for (int i = max(0, issued - 2); i < issued; ++i)
        mbar_wait(&kv_full[i & 1], (i >> 1) & 1, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0 && nb > 0) {
      const uint32_t id_s = idesc_bf16(128, kKB);          // S = Q K^T, both K-major
      const uint32_t id_pv = idesc_bf16(128, HD, 0, 1);    // O += P V, V MN-major
      const uint32_t q_s = smem_u32(sQ);
      // S(i) = Q K(i)^T into TMEM buffer i & 1
      auto issue_s = [&](int i) -> bool {
        if (!mbar_wait(&kv_full[i & 1], (i >> 1) & 1, p.err)) return false;
        tc_fence_after();
        const uint32_t k_s = smem_u32(sK + (i & 1) * KVBYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16(tmem + (i & 1) * kKB, sdesc_kmajor_sw128(q_s + (kk >> 2) * kBox + (kk & 3) * 32),
                   sdesc_kmajor_sw128(k_s + (kk >> 2) * kBox + (kk & 3) * 32), id_s,
                   kk > 0 ? 1u : 0u);
        umma_commit(&s_full[i & 1]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, p.err) && issue_s(0) && (nb < 2 || issue_s(1));
      for (int i = 0; ok && i < nb; ++i) {
        if (!mbar_wait(p_full, i & 1, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t p_s = smem_u32(sP), v_s = smem_u32(sV + (i & 1) * KVBYTES);
#pragma unroll
        for (int kk = 0; kk < kKB / 16; ++kk)
          umma_f16(tO, sdesc_kmajor_sw128(p_s + (kk >> 2) * kBox + (kk & 3) * 32),
                   sdesc_mnmajor_sw128(v_s + kk * 2048, kBox), id_pv,
                   (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(pv_done);
        umma_commit(&kv_empty[i & 1]);
        // the softmax of block i has read S buffer i & 1 (p_full): block i + 2 may reuse it
        if (i + 2 < nb && !issue_s(i + 2)) { ok = false; break; }
      }
      if (!ok) *abort_flag = 1;
      umma_commit(drain);
      mbar_wait(drain, 0, p.err);
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    // Two warps per TMEM lane quarter: half hh takes keys [hh*64, hh*64+64) of S and
    // dims [hh*HD/2, ...) of O for the 32 query rows of its quarter.
    const int q = warp & 3;
    const int hh = (warp - 2) >> 2;
    const int r = q * 32 + lane;                          // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const float sl2 = p.scale * 1.4426950408889634f;     // scores in log2 units
    float m = -INFINITY, l = 0.f;                         // m: full row; l: this half's keys
    bool ok = true;
    const int k_row = min(k_end, row_limit(q0 + r));      // this row's keys end here
    for (int i = 0; i < nb; ++i) {
      ok = softmax_vote(ok && !*abort_flag && mbar_wait(&s_full[i & 1], (i >> 1) & 1, p.err));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tS = tmem + (i & 1) * kKB + hh * HALF_KEYS;
      const int nv = min(kKB, k_row - (k_begin + i * kKB)) - hh * HALF_KEYS;   // valid keys here
      float v[HALF_KEYS];
#pragma unroll
      for (int c = 0; c < HALF_KEYS; c += 16) tmem_ld16(tS + lane_off + c, v + c);
      tmem_ld_wait();
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < HALF_KEYS; ++j)
        if (j < nv) mx = fmaxf(mx, v[j] * sl2);
      s_red[hh * kQT + r] = mx;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      const float mn = fmaxf(m, fmaxf(mx, s_red[(hh ^ 1) * kQT + r]));
      // a row with no valid key yet (prefill rows whose limit ends before this block)
      // keeps m = -inf: exponents then use 0 as the reference, and every term is zero
      const float mref = mn == -INFINITY ? 0.f : mn;
      const float alpha = exp2f(m - mref);
      if (i > 0) {
        // P V of the previous block must be done: it reads sP and accumulates into O
        ok = softmax_vote(mbar_wait(pv_done, (i - 1) & 1, p.err));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
          for (int c = 0; c < HALF_DIMS; c += 32) {
            float o[32];
            tmem_ld16(tO + lane_off + hh * HALF_DIMS + c, o);
            tmem_ld16(tO + lane_off + hh * HALF_DIMS + c + 16, o + 16);
            tmem_ld_wait();
            uint32_t u[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) u[j] = __float_as_uint(o[j] * alpha);
            tmem_st16(tO + lane_off + hh * HALF_DIMS + c, u);
            tmem_st16(tO + lane_off + hh * HALF_DIMS + c + 16, u + 16);
          }
          tmem_st_wait();
        }
      }
      // P = exp2(s*scale*log2e - m) in bf16, written in the 128-byte-swizzled K-major
      // layout the P V MMA reads (keys hh*64.. form the second 64-key box)
      float sum = 0.f;
#pragma unroll
      for (int g8 = 0; g8 < HALF_KEYS / 8; ++g8) {
        uint32_t pk[4];
#pragma unroll
        for (int h2 = 0; h2 < 4; ++h2) {
          const int j0 = g8 * 8 + 2 * h2;
          const float e0 = j0 < nv ? exp2f(fmaf(v[j0], sl2, -mref)) : 0.f;
          const float e1 = j0 + 1 < nv ? exp2f(fmaf(v[j0 + 1], sl2, -mref)) : 0.f;
          sum += e0 + e1;
          const __nv_bfloat162 b2 = __floats2bfloat162_rn(e0, e1);
          pk[h2] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        unsigned char* dst = sP + hh * kBox + r * 128 + ((g8 ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l = l * alpha + sum;
      m = mn;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && nb > 0) ok = softmax_vote(mbar_wait(pv_done, (nb - 1) & 1, p.err));
    // full-row sum: the two halves' partial sums
    s_red[hh * kQT + r] = l;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float l_row = l + s_red[(hh ^ 1) * kQT + r];
    const int qi = q0 + r;
    int64_t pq = qi;
    if (p.rows != nullptr && qi < Mq) pq = p.rows[qi / p.G] * p.G + qi % p.G;
    const int64_t base = (static_cast<int64_t>(split) * p.Hkv + kvh) * p.part_rows + pq;
    if (ok && nb > 0) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HALF_DIMS; c += 32) {
        float o[32];
        tmem_ld16(tO + lane_off + hh * HALF_DIMS + c, o);
        tmem_ld16(tO + lane_off + hh * HALF_DIMS + c + 16, o + 16);
        tmem_ld_wait();
        if (qi < Mq) {
          float4* dst = reinterpret_cast<float4*>(p.part_O + base * HD + hh * HALF_DIMS + c);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            dst[j] = make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        }
      }
    } else if (qi < Mq) {
      m = -INFINITY;
      for (int d = 0; d < HALF_DIMS; ++d) p.part_O[base * HD + hh * HALF_DIMS + d] = 0.f;
    }
    if (qi < Mq && hh == 0) {
      // m in natural-log units for the consumers
      p.part_ml[2 * base] = (ok && nb > 0) ? m * 0.6931471805599453f : -INFINITY;
      p.part_ml[2 * base + 1] = (ok && nb > 0) ? l_row : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// q_comp[kvh][slot*G + g][:] = q_buf[rows[slot]][(kvh*G + g)*hd : ...]
__global__ void pack_q_kernel(const __nv_bfloat16* q_buf, const int64_t* rows,
                              const int32_t* count, int bucket, int H, int Hkv, int hd,
                              int q_rows, __nv_bfloat16* q_comp) {
  const int slot = blockIdx.x;
  const int n = min(*count, bucket);
  if (slot >= n) return;
  const int G = H / Hkv;
  const int64_t r = rows[slot];
  const int vecs = H * hd / 8;
  for (int i = threadIdx.x; i < vecs; i += blockDim.x) {
    const int e = i * 8;
    const int h = e / hd, d = e % hd;
    const int kvh = h / G, g = h % G;
    const uint4 v = *reinterpret_cast<const uint4*>(q_buf + r * H * hd + e);
    *reinterpret_cast<uint4*>(q_comp + ((static_cast<int64_t>(kvh) * q_rows + slot * G + g) * hd + d)) = v;
  }
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 att_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

static bool att_tmap(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols) {
  auto fn = att_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int kv_splits(int P) { return kv_splits_of(P); }

static size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

size_t attn_scratch_bytes(int dtype, int bucket, int H, int Hkv, int hd, int P,
                          bool need_q_comp, int rows_total) {
  if (dtype != BF16 || P <= 0) return 0;
  const int G = H / Hkv;
  const size_t q_rows = static_cast<size_t>(bucket) * G;
  const size_t part_rows = static_cast<size_t>(std::max(bucket, rows_total)) * G;
  const int S = kv_splits(P);
  size_t b = 0;
  if (need_q_comp) b += up256(Hkv * q_rows * hd * 2);
  b += up256(static_cast<size_t>(S) * Hkv * part_rows * hd * 4);
  b += up256(static_cast<size_t>(S) * Hkv * part_rows * 2 * 4);
  return b;
}

cudaError_t launch_attention_simt_partials(int dtype, const AttnParams& p, const float* part_O,
                                           const float* part_ml, int splits, int q_rows,
                                           cudaStream_t st);

struct PrefixPartials {
  const float* part_O;
  const float* part_ml;
  int splits, q_rows;
};

// prefix part of every recomputed row's attention: per-split partials in the scratch
template <int HD>
static cudaError_t prefix_partials(const AttnParams& a, cudaStream_t st, PrefixPartials* out,
                                   bool by_row) {
  const int G = a.H / a.Hkv;
  const int q_rows = a.bucket * G;
  const int S = kv_splits(a.P);
  const bool pack = a.q_comp == nullptr;
  const int rows_total = by_row ? a.B1 * a.N : 0;
  if (a.scratch == nullptr ||
      a.scratch_bytes < attn_scratch_bytes(BF16, a.bucket, a.H, a.Hkv, HD, a.P, pack, rows_total))
    return cudaErrorInvalidValue;
  if (a.kv_head_stride % HD != 0) return cudaErrorInvalidValue;
  char* sc = static_cast<char*>(a.scratch);
  const void* q_comp = a.q_comp;
  if (pack) {
    q_comp = sc;
    pack_q_kernel<<<a.bucket, 128, 0, st>>>(static_cast<const __nv_bfloat16*>(a.q_buf), a.rows,
                                            a.count, a.bucket, a.H, a.Hkv, HD, q_rows,
                                            reinterpret_cast<__nv_bfloat16*>(sc));
    cudaError_t e = launched();
    if (e != cudaSuccess) return e;
    sc += up256(static_cast<size_t>(a.Hkv) * q_rows * HD * 2);
  }
  AttnTcParams p{};
  p.count = a.count;
  p.bucket = a.bucket;
  p.G = G;
  p.q_rows = q_rows;
  p.P = a.P;
  p.kv_rows = static_cast<int>(a.kv_head_stride / HD);
  p.splits = S;
  p.keys_per_split = keys_per_split_of(a.P, S);
  p.P_dev = a.P_dev;
  p.prefill_rows = a.prefill_rows;
  p.block_N = a.N;
  p.Hkv = a.Hkv;
  p.scale = a.scale;
  p.part_rows = std::max(a.bucket, rows_total) * G;
  p.rows = by_row ? a.rows : nullptr;
  p.part_O = reinterpret_cast<float*>(sc);
  p.part_ml = reinterpret_cast<float*>(sc + up256(static_cast<size_t>(S) * a.Hkv * p.part_rows * HD * 4));
  p.err = a.err;
  CUtensorMap tq, tk, tv;
  if (!att_tmap(&tq, q_comp, static_cast<uint64_t>(a.Hkv) * q_rows, HD) ||
      !att_tmap(&tk, a.pk, static_cast<uint64_t>(a.Hkv) * p.kv_rows, HD) ||
      !att_tmap(&tv, a.pv, static_cast<uint64_t>(a.Hkv) * p.kv_rows, HD))
    return cudaErrorInvalidValue;
  constexpr int kBox = 128 * 64 * 2;
  const size_t smem = 1024 + (HD / 64) * kBox * 5 + 2 * kBox + 2 * kQT * 4 + 256;
  static int configured = 0;
  if (configured < static_cast<int>(smem)) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefix_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured = static_cast<int>(smem);
  }
  // (kv head, split) fastest: the CTAs of the live query tiles (count * G rows, known
  // only on the device) come first in launch order and run in the first wave.  (Query
  // tiles fastest, so that the tiles of one key split read it from L2 together, cut the
  // DRAM reads at P = 32768 on the 8B shape from 933 MB but was 5-10 us slower at every
  // prefix >= 16K: the kernel is not DRAM-bound there, and the dead tiles interleave.)
  dim3 grid(a.Hkv, S, (q_rows + kQT - 1) / kQT);
  cudaError_t e = launch_ex(attn_prefix_kernel<HD>, grid, dim3(kAttThreads), smem, st, false, tq,
                            tk, tv, p);
  if (e == cudaSuccess) e = launched();
  if (e != cudaSuccess) return e;
  out->part_O = p.part_O;
  out->part_ml = p.part_ml;
  out->splits = S;
  out->q_rows = p.part_rows;
  return cudaSuccess;
}

// SF_ROWS_MMA=0: the SIMT rows kernel instead of the tensor-core one (read once)
static bool rows_mma_enabled() {
  static const bool on = [] {
    const char* v = getenv("SF_ROWS_MMA");
    return v == nullptr || atoi(v) != 0;
  }();
  return on;
}

// SF_ROWS_TC=0: the rows pass on mma.sync tiles instead of tcgen05 (read once)
static bool rows_tc_enabled() {
  static const bool on = [] {
    const char* v = getenv("SF_ROWS_TC");
    return v == nullptr || atoi(v) != 0;
  }();
  return on;
}

static bool prefix_on_tc(int dtype, const AttnParams& p) {
  return dtype == BF16 && p.P > 0 && p.pk != nullptr;
}

static cudaError_t prefix_partials_hd(const AttnParams& p, cudaStream_t st, PrefixPartials* pp,
                                      bool by_row) {
  if (p.hd == 128) return prefix_partials<128>(p, st, pp, by_row);
  if (p.hd == 64) return prefix_partials<64>(p, st, pp, by_row);
  return cudaErrorInvalidValue;
}

cudaError_t launch_attention(int dtype, const AttnParams& p, cudaStream_t st) {
  if (!prefix_on_tc(dtype, p)) return launch_attention_simt(dtype, p, st);
  PrefixPartials pp{};
  cudaError_t e = prefix_partials_hd(p, st, &pp, false);
  if (e != cudaSuccess) return e;
  return launch_attention_simt_partials(BF16, p, pp.part_O, pp.part_ml, pp.splits, pp.q_rows, st);
}

cudaError_t launch_attention_rows(int dtype, const AttnParams& p, cudaStream_t st) {
  if (!prefix_on_tc(dtype, p)) return launch_attention_rows_partials(dtype, p, nullptr, nullptr, 0, 0, st);
  PrefixPartials pp{};
  cudaError_t e = prefix_partials_hd(p, st, &pp, true);
  if (e != cudaSuccess) return e;
  if (attention_rows_tc_ok(dtype, p, pp.splits) && rows_tc_enabled())
    return launch_attention_rows_tc(p, pp.part_O, pp.part_ml, pp.splits, pp.q_rows, st);
  if (attention_rows_mma_ok(dtype, p, pp.splits) && rows_mma_enabled())
    return launch_attention_rows_mma(p, pp.part_O, pp.part_ml, pp.splits, pp.q_rows, st);
  return launch_attention_rows_partials(BF16, p, pp.part_O, pp.part_ml, pp.splits, pp.q_rows, st);
}

}  // namespace sf
