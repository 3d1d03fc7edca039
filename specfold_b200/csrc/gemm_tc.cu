// Tensor-core (tcgen05) weight-streaming GEMM of the folded verify forward, bf16.
//
// acc[j][f] = sum_k X[j][k] * W[f][k] for the few activation rows j (recomputed rows,
// <= B1*N) against a large weight matrix W [n_out, K].  At the model shapes this is
// HBM-bound on the weight stream, so the kernel is built around it:
//   * "swap-AB": 128 weight rows are the MMA's M operand, the activation rows its N
//     operand (N = rows rounded up to 16), fp32 accumulators in TMEM;
//   * a CTA streams `sub` (1, 2 or 4) 128-row weight tiles per pipeline stage against
//     one shared activation stage, so the activations (re-read from L2 by every CTA)
//     cost 1/sub as much per weight byte -- the L2->SM traffic, not HBM, is what limits
//     the weight stream when every stage carries as many activation bytes as weight;
//   * weights optionally pre-arranged in 128x64 blocks (weight_tiles_bytes), making a
//     stage's 16 KB of each tile one contiguous read;
//   * TMA loads (128-byte swizzle, no multicast), stage count sized in the kernel from
//     the actual row count;
//   * persistent CTAs over units (tile group, K split); with several units per CTA the
//     accumulators are double-buffered so one unit's epilogue overlaps the next mainloop;
//   * few tile groups (QKV, o_proj, down) split K across co-resident CTAs (cooperative
//     launch): each publishes fp32 partials, waits (bounded) for its group's other
//     splits, and reduces its own slice of rows in split order -- deterministic.
// Warp 0 issues TMA, warp 1 owns TMEM and issues MMAs, warps 2-9 run the epilogue (two
// warps per TMEM lane quarter, alternating 16-row chunks: the epilogue is latency-bound,
// and with one warp per SM sub-partition the last unit's epilogue dominated the tail).
//
// Epilogues reproduce the rounding points of the PyTorch folded forward:
//   QKV     F.linear + bias rounded to the model dtype, then q*c + rot(q)*s with every
//           op rounded (fastdllm_v2_folded.py:153-157; triton_kernels.py:65-87); also
//           writes the query copy the tensor-core attention reads
//   RESID   x + T(O @ Wo^T) (fastdllm_v2_folded.py:207-208, :351)
//   SWIGLU  T(silu(T(g))) * T(u) (fastdllm_v2_folded.py:216; triton_kernels.py:133)
//   SCATTER ffn_buf[rows[j]] = T(acc) (triton_kernels.py:171-173)
//   LOGITS  lm_head with the Fast-dLLM shift (fastdllm_v2_generation.py:121-126)
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <vector>

#include "sf_kernels.cuh"

namespace sf {

constexpr int kEpiWarps = 8;                     // two warps per TMEM lane quarter
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kTcThreads = 64 + kEpiThreads;
constexpr int kTileF = 128;                      // weight rows per tile (MMA M)
constexpr int kBK = 64;                          // K per stage: one 128-byte swizzle row
constexpr int kMaxPassRows = 256;                // MMA N limit
constexpr int kWBytes = kTileF * kBK * 2;        // 16 KB per tile per stage
constexpr int kXRowBytes = kBK * 2;              // one activation row of a stage
constexpr int kChunk = 16;                       // rows (TMEM columns) per epilogue chunk
constexpr int kTileLd = kTileF + 4;              // padded fp32 row of the transposed chunk
constexpr int kTileTBytes = 2 * kChunk * kTileLd * 4;   // one transposed chunk per half
constexpr int kMaxStages = 8;
constexpr int kSmemFixed = kTileTBytes + 1024 + 256;   // transposed chunks, alignment, barriers

// activation rows one pass loads: 128-row boxes while more than 64 remain, then one
// 64-row box (fewer, larger TMA requests than 64-row boxes alone)
__host__ __device__ __forceinline__ int x_rows_loaded(int prows) {
  const int n128 = prows > 64 ? (prows - 64 + 127) / 128 : 0;
  const int rest = prows - n128 * 128;
  return n128 * 128 + (rest > 0 ? 64 : 0);
}
// split-K counters (arrivals, departures) per tile group at offset 0 of the workspace
constexpr int kMaxCounterTiles = static_cast<int>(kGemmCounterBytes / 8);

struct TcParams {
  int n_out, K, rows_cap;
  const int32_t* count;
  int mode;            // 0: 128-row tiles of W; 1: SWIGLU, 64 gate + 64 up rows per tile
  int inter;
  int n_tiles;         // 128-row weight tiles
  int sub;             // tiles per unit sharing one activation stage (1, 2 or 4)
  int n_groups;        // ceil(n_tiles / sub)
  int splits, kb_total, kb_per_split, n_units;
  int w_tiled;         // weights in the [tile][kb][128][64] layout
  int stage_budget;    // shared-memory bytes for the pipeline stages
  int defer_reduce;    // split phase whose reduction the next phase's norm performs
  int no_dep;          // phase k > 0 that does not read phase k-1's output
  WPrefetch next_pf;   // the next GEMM's first weight blocks, pulled into L2 by the
                       // producer once it has issued its own last load
  float* partial;      // [splits][rows_cap][n_out] when splits > 1
  int* counters;       // [2 * n_groups]
  EpiParams epi;
  int* err;
};

// natural feature index of tile-local weight row l, or -1 past the end
__device__ __forceinline__ int tc_feature(const TcParams& p, int tile, int l) {
  if (tile >= p.n_tiles) return -1;
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

// The operands of a QKV output group that do not depend on the GEMM: the bias at the
// group's features f and at its RoPE partner's fp, cos / sin at (n, f % hd) (q and k
// features only) and, with `both`, at (n, fp % hd) for the partner's own group; bf16 x 8.
struct QkvOps {
  uint4 b, bp, c, s, cp, sp;
  float qs;
};
__device__ __forceinline__ void qkv_ops_load(const EpiParams& e, int64_t row, int f, int fp,
                                             bool both, QkvOps& o) {
  using T = __nv_bfloat16;
  const int n = static_cast<int>(row % e.N);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  const T* bias = reinterpret_cast<const T*>(e.bias);
  o.b = bias ? *reinterpret_cast<const uint4*>(bias + f) : z;
  o.bp = bias ? *reinterpret_cast<const uint4*>(bias + fp) : z;
  o.c = o.s = o.cp = o.sp = z;
  if (f < e.q_dim + e.kv_dim) {
    const int64_t base = static_cast<int64_t>(n) * e.hd;
    o.c = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(e.cos) + base + f % e.hd);
    o.s = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(e.sin) + base + f % e.hd);
    if (both) {
      o.cp = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(e.cos) + base + fp % e.hd);
      o.sp = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(e.sin) + base + fp % e.hd);
    }
  }
  o.qs = (f < e.q_dim && e.q_scale) ? e.q_scale[n] : 1.0f;
}
__device__ __forceinline__ void bf16x8_get(const uint4& u, float* out) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}
// QKV output group f0..f0+7 of activation row j (block row `row`): + bias, bf16, RoPE with
// the partner values vp, q scale, scatter (q rows, the query-major q copy, k / v rows).
__device__ __forceinline__ void qkv_emit8(const EpiParams& e, int j, int64_t row, int f0,
                                          const float* v, const float* vp, const uint4& braw,
                                          const uint4& bpraw, const uint4& craw,
                                          const uint4& sraw, float qs_raw) {
  using T = __nv_bfloat16;
  float x[8], xp[8], o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) { x[i] = v[i]; xp[i] = vp[i]; }
  if (e.bias) {
    float b[8], bp[8];
    bf16x8_get(braw, b);
    bf16x8_get(bpraw, bp);
#pragma unroll
    for (int i = 0; i < 8; ++i) { x[i] = __fadd_rn(x[i], b[i]); xp[i] = __fadd_rn(xp[i], bp[i]); }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) { o[i] = Elt<T>::rnd(x[i]); xp[i] = Elt<T>::rnd(xp[i]); }
  if (f0 < e.q_dim + e.kv_dim) {
    const int d0 = f0 % e.hd;
    float c[8], s[8];
    bf16x8_get(craw, c);
    bf16x8_get(sraw, s);
    const bool first = d0 < (e.hd >> 1);
    const float qs = (f0 < e.q_dim && e.q_scale) ? Elt<T>::rnd(qs_raw) : 1.0f;
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
}

// Epilogue of 8 consecutive tile-local weight rows l0..l0+7 for activation row j:
// v = their accumulators, vp = the partner rows' (RoPE pair / SwiGLU up half).  The kind
// is a template parameter: one kernel per epilogue keeps each kernel's code small (the
// epilogue loop of an all-kinds kernel missed in the instruction cache).
template <int KIND>
__device__ __forceinline__ void epi_group8(const TcParams& p, int tile, int j, int l0,
                                           const float* v, const float* vp) {
  using T = __nv_bfloat16;
  const EpiParams& e = p.epi;
  const int f0 = tc_feature(p, tile, l0);
  if (f0 < 0) return;
  float o[8];
  switch (KIND) {
    case EPI_RAW:
      store_vec<float>(reinterpret_cast<float*>(e.out) + static_cast<int64_t>(j) * e.ld_out + f0, v);
      store_vec<float>(reinterpret_cast<float*>(e.out) + static_cast<int64_t>(j) * e.ld_out + f0 + 4, v + 4);
      return;
    case EPI_QKV: {
      const int64_t row = e.rows[j];
      QkvOps ops;
      qkv_ops_load(e, row, f0, f0 ^ (e.hd >> 1), false, ops);
      qkv_emit8(e, j, row, f0, v, vp, ops.b, ops.bp, ops.c, ops.s, ops.qs);
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
      // silu in fp32 with the hardware exp and divide intrinsics; their few-ulp fp32
      // error sits far below the bf16 rounding that follows
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float g = Elt<T>::rnd(v[i]), u = Elt<T>::rnd(vp[i]);
        o[i] = __fmul_rn(Elt<T>::rnd(__fdividef(g, 1.0f + __expf(-g))), u);
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
// groups of 8 tile rows per activation row that produce output (SwiGLU: the gate half;
// its up partner rides along)
template <int KIND>
constexpr int kGroupsOut = KIND == EPI_SWIGLU ? 8 : 16;

__device__ __forceinline__ void vec_get(const float4& v, float* o) {
  o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}

template <int KIND>
__device__ __forceinline__ int tc_partner_l(const TcParams& p, int l0) {
  if (KIND == EPI_QKV) return l0 ^ (p.epi.hd >> 1);
  if (KIND == EPI_SWIGLU) return l0 ^ 64;
  return l0;
}

// AND over the 256 epilogue threads (named barrier 1): keeps every branch that
// guards a named barrier uniform, whatever each thread saw of the abort flag.
__device__ __forceinline__ bool epi_vote_all(bool x) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 256, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(x))
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void epi_sync_all() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// the four warps of one epilogue half (named barriers 2 and 3)
__device__ __forceinline__ void epi_sync_half(int h) {
  asm volatile("bar.sync %0, 128;" ::"r"(2 + h) : "memory");
}

// Sum over splits s of partial[s][row][f..f+7], in split order (deterministic), four
// splits' loads in flight at a time.
__device__ __forceinline__ void sum_splits8(const float* partial, int splits, int64_t split_stride,
                                            int64_t off, float* acc) {
  int s = 0;
  for (; s + 4 <= splits; s += 4) {
    float4 a[8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float* q = partial + (s + u) * split_stride + off;
      a[2 * u] = __ldcg(reinterpret_cast<const float4*>(q));
      a[2 * u + 1] = __ldcg(reinterpret_cast<const float4*>(q + 4));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      acc[0] += a[2 * u].x; acc[1] += a[2 * u].y; acc[2] += a[2 * u].z; acc[3] += a[2 * u].w;
      acc[4] += a[2 * u + 1].x; acc[5] += a[2 * u + 1].y;
      acc[6] += a[2 * u + 1].z; acc[7] += a[2 * u + 1].w;
    }
  }
  for (; s < splits; ++s) {
    const float* q = partial + s * split_stride + off;
    const float4 a0 = __ldcg(reinterpret_cast<const float4*>(q));
    const float4 a1 = __ldcg(reinterpret_cast<const float4*>(q + 4));
    acc[0] += a0.x; acc[1] += a0.y; acc[2] += a0.z; acc[3] += a0.w;
    acc[4] += a1.x; acc[5] += a1.y; acc[6] += a1.z; acc[7] += a1.w;
  }
}

// sum_splits8 of two groups at once (both groups' loads in flight together; each sum in
// split order, as sum_splits8)
__device__ __forceinline__ void sum_splits8_pair(const float* partial, int splits,
                                                 int64_t split_stride, int64_t off_a,
                                                 int64_t off_b, float* acc_a, float* acc_b) {
  int s = 0;
  for (; s + 4 <= splits; s += 4) {                // four splits' loads in flight
    float4 a[16];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float* qa = partial + (s + u) * split_stride + off_a;
      const float* qb = partial + (s + u) * split_stride + off_b;
      a[4 * u] = __ldcg(reinterpret_cast<const float4*>(qa));
      a[4 * u + 1] = __ldcg(reinterpret_cast<const float4*>(qa + 4));
      a[4 * u + 2] = __ldcg(reinterpret_cast<const float4*>(qb));
      a[4 * u + 3] = __ldcg(reinterpret_cast<const float4*>(qb + 4));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float va[8], vb[8];
      vec_get(a[4 * u], va); vec_get(a[4 * u + 1], va + 4);
      vec_get(a[4 * u + 2], vb); vec_get(a[4 * u + 3], vb + 4);
#pragma unroll
      for (int i = 0; i < 8; ++i) { acc_a[i] += va[i]; acc_b[i] += vb[i]; }
    }
  }
  for (; s + 2 <= splits; s += 2) {
    float4 a[8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float* qa = partial + (s + u) * split_stride + off_a;
      const float* qb = partial + (s + u) * split_stride + off_b;
      a[4 * u] = __ldcg(reinterpret_cast<const float4*>(qa));
      a[4 * u + 1] = __ldcg(reinterpret_cast<const float4*>(qa + 4));
      a[4 * u + 2] = __ldcg(reinterpret_cast<const float4*>(qb));
      a[4 * u + 3] = __ldcg(reinterpret_cast<const float4*>(qb + 4));
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float va[8], vb[8];
      vec_get(a[4 * u], va); vec_get(a[4 * u + 1], va + 4);
      vec_get(a[4 * u + 2], vb); vec_get(a[4 * u + 3], vb + 4);
#pragma unroll
      for (int i = 0; i < 8; ++i) { acc_a[i] += va[i]; acc_b[i] += vb[i]; }
    }
  }
  for (; s < splits; ++s) {
    float va[8], vb[8];
    const float* qa = partial + s * split_stride + off_a;
    const float* qb = partial + s * split_stride + off_b;
    vec_get(__ldcg(reinterpret_cast<const float4*>(qa)), va);
    vec_get(__ldcg(reinterpret_cast<const float4*>(qa + 4)), va + 4);
    vec_get(__ldcg(reinterpret_cast<const float4*>(qb)), vb);
    vec_get(__ldcg(reinterpret_cast<const float4*>(qb + 4)), vb + 4);
#pragma unroll
    for (int i = 0; i < 8; ++i) { acc_a[i] += va[i]; acc_b[i] += vb[i]; }
  }
}

// L2 prefetch of another GEMM's weights (see WPrefetch): worker w of n takes units
// w, w + n, ...; every (unit, tile) is one contiguous range of the tile layout.
__device__ __forceinline__ void issue_w_prefetch(const WPrefetch& f, int worker, int n_workers) {
  if (f.w == nullptr) return;
  for (int u = worker; u < f.n_units; u += n_workers) {
    const int grp = u / f.splits, split = u % f.splits;
    const int kb0 = split * f.kb_per_split;
    const int npf = min(min(f.kb_total, kb0 + f.kb_per_split) - kb0, f.npf);
    for (int t = 0; t < f.sub; ++t) {
      const int tile = grp * f.sub + t;
      if (tile >= f.n_tiles) break;
      const char* a = static_cast<const char*>(f.w) + (static_cast<int64_t>(tile) * f.kb_total + kb0) * kWBytes;
      for (int c = 0; c < npf; c += 4)
        prefetch_l2_bulk(a + static_cast<int64_t>(c) * kWBytes, min(4, npf - c) * kWBytes);
    }
  }
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------------------------ GEMM chains
// One launch may run up to three GEMMs back to back ("phases"), each optionally preceded
// by an RMSNorm of its activation rows.  Phase k's activations come from phase k-1's
// output, directly or through that norm (o_proj -> norm -> gate_up -> down).  Units of
// all phases are spread over the same persistent CTAs; a phase waits for its
// activations through device counters, and only before its first activation load: the
// weight blocks of its first stages are already in flight while the previous phase (or
// the norm) finishes.
constexpr int kMaxPhases = 3;

struct PreNorm {           // out[i] = T(w * T(x[rows[i]] * rstd)), i < min(*count, n)
  const void* x;
  const int64_t* rows;
  const int32_t* count;
  const void* w;
  void* out;
  int n;
  int64_t n_src;
  int D;
  float eps;
  const int8_t* rec;               // recompute flags (deferred reduction only)
};

struct ChainParams {
  TcParams ph[kMaxPhases];
  PreNorm norm[kMaxPhases];        // norm[k].x != nullptr: RMSNorm writing phase k's input
  int n_phases;
  int unit_base[kMaxPhases + 1];   // units of phase k: [unit_base[k], unit_base[k+1])
  int stage_budget;
  int max_sub;
  int ctas_per_sm;                 // CTAs sharing an SM's TMEM
  // counters, zero at launch: dep[2k] CTAs done with norm k, dep[2k+1] units of phase k
  // done (the latter only counted for phases whose output a later phase reads)
  unsigned* dep;
  int* err;
};

// what phase k's activation loads wait for: (counter, target), or counter == nullptr
__device__ __forceinline__ const unsigned* phase_dep(const ChainParams& c, int k, unsigned* target) {
  if (c.norm[k].x != nullptr) {
    *target = gridDim.x;
    return c.dep + 2 * k;
  }
  if (k > 0 && !c.ph[k].no_dep) {
    *target = static_cast<unsigned>(c.ph[k - 1].n_units);
    return c.dep + 2 * (k - 1) + 1;
  }
  return nullptr;
}

// bounded wait for a device counter to reach target (acquire)
__device__ __forceinline__ bool wait_counter(const unsigned* c, unsigned target, int* err) {
  const uint64_t t0 = globaltimer();
  while (true) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
    if (static_cast<int>(v - target) >= 0) return true;
    if (globaltimer() - t0 > kWaitNs) {
      flag_error(err, SF_DEV_ERR_TIMEOUT);
      return false;
    }
  }
}
// generic-proxy stores by other CTAs are read next by this thread's TMA (async proxy)
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

struct EpiCtx {
  uint32_t tmem;
  int acc_cols, buf_cols;
  int q, l, et, h, eh;
  float* tileT;
  volatile int* abort_flag;
};

// Epilogue of one unit (all passes of its activation rows) for phase parameters p.
template <int KIND>
__device__ __forceinline__ void epi_unit(const TcParams& p, const EpiCtx& x, int lu, int rows,
                                         int& acc_it, bool double_buf, uint64_t* acc_full,
                                         uint64_t* acc_empty) {
  const int n_pass = (rows + kMaxPassRows - 1) / kMaxPassRows;
  const int grp = lu / p.splits, split = lu % p.splits;
  const int lane = threadIdx.x & 31;
  for (int pass = 0; pass < n_pass; ++pass, ++acc_it) {
    const int prow0 = pass * kMaxPassRows;
    const int prows = min(kMaxPassRows, rows - prow0);
    const int buf = double_buf ? (acc_it & 1) : 0;
    const uint32_t par = double_buf ? ((acc_it >> 1) & 1) : (acc_it & 1);
    const bool ready = epi_vote_all(!*x.abort_flag && mbar_wait(&acc_full[buf], par, p.err));
    if (!ready) *x.abort_flag = 1;
    tc_fence_after();
    for (int t = 0; ready && t < p.sub; ++t) {
      const int tile = grp * p.sub + t;
      if (tile >= p.n_tiles) break;
      for (int c0 = x.h * kChunk; c0 < prows; c0 += 2 * kChunk) {
        float v[kChunk];
        const uint32_t ta = x.tmem + (static_cast<uint32_t>(x.q * 32) << 16) +
                            static_cast<uint32_t>(buf * x.buf_cols + t * x.acc_cols + c0);
        tmem_ld16(ta, v);
        tmem_ld_wait();
        const int nr = min(kChunk, prows - c0);
        if (p.splits > 1) {
          // fp32 partial of this split, row-major, straight from the registers: lane l
          // holds feature f(l) of rows c0.., so each row is one 128-byte store per warp
          const int f = tc_feature(p, tile, x.l);
          if (f >= 0) {
            float* part = p.partial + (static_cast<int64_t>(split) * p.rows_cap + prow0 + c0) * p.n_out + f;
#pragma unroll
            for (int i = 0; i < kChunk; ++i)
              if (i < nr) __stcg(part + static_cast<int64_t>(i) * p.n_out, v[i]);
          }
          continue;
        }
#pragma unroll
        for (int i = 0; i < kChunk; ++i) x.tileT[i * kTileLd + x.l] = v[i];
        epi_sync_half(x.h);
        {
#pragma unroll
          for (int k = 0; k < kChunk * kGroupsOut<KIND> / 128; ++k) {
            const int item = x.eh + 128 * k;
            const int r = item / kGroupsOut<KIND>, l0 = (item % kGroupsOut<KIND>) * 8;
            if (r < nr) {
              const float4* a = reinterpret_cast<const float4*>(x.tileT + r * kTileLd + l0);
              const float4* b =
                  reinterpret_cast<const float4*>(x.tileT + r * kTileLd + tc_partner_l<KIND>(p, l0));
              float va[8], vb[8];
              vec_get(a[0], va); vec_get(a[1], va + 4);
              vec_get(b[0], vb); vec_get(b[1], vb + 4);
              epi_group8<KIND>(p, tile, prow0 + c0 + r, l0, va, vb);
            }
          }
        }
        epi_sync_half(x.h);
      }
    }
    tc_fence_before();
    if (lane == 0) mbar_arrive(&acc_empty[buf]);
  }
  if (p.splits > 1 && !p.defer_reduce) {
    // every split of this tile group publishes, then each reduces its slice of rows
    __threadfence();
    bool go = epi_vote_all(!*x.abort_flag);
    // QKV: the block row of this thread's first item does not depend on the GEMM; loaded
    // while the other splits finish, it leaves one round of loads after the wait (bias,
    // cos / sin and the partials together) where each item chained several
    int64_t pre_row = -1;
    if constexpr (KIND == EPI_QKV) {
      const int sl = (rows + p.splits - 1) / p.splits;
      const int pr = split * sl + x.et / 8;
      if (go && x.et / 8 < sl && pr < rows) pre_row = p.epi.rows[pr];
    }
    if (x.et == 0 && go) {
      atomicAdd(&p.counters[2 * grp], 1);
      const uint64_t t0 = globaltimer();
      while (ld_acquire(&p.counters[2 * grp]) < p.splits) {
        if (globaltimer() - t0 > kWaitNs) {
          flag_error(p.err, SF_DEV_ERR_TIMEOUT);
          *x.abort_flag = 1;
          break;
        }
      }
    }
    go = epi_vote_all(!*x.abort_flag);
    const int slice = (rows + p.splits - 1) / p.splits;
    const int r0 = split * slice, r1 = min(rows, r0 + slice);
    const int64_t split_stride = static_cast<int64_t>(p.rows_cap) * p.n_out;
    // items: (tile t, row r, group of 8 weight rows l0 that emits output).  QKV: one item
    // per RoPE pair (l0 in the lower half of its head), which sums both halves once and
    // emits both -- every partial is read once
    constexpr bool kPair = KIND == EPI_QKV;
    constexpr int GPR = kPair ? 8 : kGroupsOut<KIND>;
    const int n_items = go ? p.sub * max(0, r1 - r0) * GPR : 0;
    for (int item = x.et; item < n_items; item += kEpiThreads) {
      const int t = item / ((r1 - r0) * GPR);
      const int rem = item - t * (r1 - r0) * GPR;
      const int r = r0 + rem / GPR;
      int l0 = (rem % GPR) * 8;
      if (kPair) {
        const int half = p.epi.hd >> 1;
        l0 = (l0 / half) * p.epi.hd + l0 % half;
      }
      const int tile = grp * p.sub + t;
      if (tile >= p.n_tiles) continue;
      if constexpr (KIND == EPI_QKV) {
        const int fa = tc_feature(p, tile, l0);
        const int fb = tc_feature(p, tile, tc_partner_l<KIND>(p, l0));
        if (item == x.et && t == 0 && pre_row >= 0 && fa >= 0 && fb >= 0 && fb != fa) {
          QkvOps ops;
          qkv_ops_load(p.epi, pre_row, fa, fb, true, ops);
          float va[8] = {}, vb[8] = {};
          const int64_t row_off = static_cast<int64_t>(r) * p.n_out;
          sum_splits8_pair(p.partial, p.splits, split_stride, row_off + fa, row_off + fb, va, vb);
          qkv_emit8(p.epi, r, pre_row, fa, va, vb, ops.b, ops.bp, ops.c, ops.s, ops.qs);
          qkv_emit8(p.epi, r, pre_row, fb, vb, va, ops.bp, ops.b, ops.cp, ops.sp, ops.qs);
          continue;
        }
      }
      const int fa = tc_feature(p, tile, l0);
      if (fa < 0) continue;
      const int lp = tc_partner_l<KIND>(p, l0);
      const int fb = tc_feature(p, tile, lp);
      float va[8] = {}, vb[8] = {};
      const int64_t row_off = static_cast<int64_t>(r) * p.n_out;
      sum_splits8(p.partial, p.splits, split_stride, row_off + fa, va);
      if (fb >= 0 && fb != fa) sum_splits8(p.partial, p.splits, split_stride, row_off + fb, vb);
      epi_group8<KIND>(p, tile, r, l0, va, fb == fa ? va : vb);
      if (kPair && fb >= 0 && fb != fa) epi_group8<KIND>(p, tile, r, lp, vb, va);
    }
    epi_sync_all();
    if (x.et == 0 && go) {
      const int prev = atomicAdd(&p.counters[2 * grp + 1], 1);
      if (prev == p.splits - 1) {      // everyone has passed the wait: reset
        p.counters[2 * grp] = 0;
        p.counters[2 * grp + 1] = 0;
      }
    }
  }
}

// RMSNorm of rows i = blockIdx.x, blockIdx.x + gridDim.x, ... by the 256 epilogue
// threads (D <= 256 * 8 * MAXV): one load of the row into registers, block reduction,
// normalised from the registers (the rmsnorm_cta_kernel arithmetic).
template <int MAXV>
__device__ __forceinline__ void pre_norm_rows(const PreNorm& pr, int et, float* red, int* err) {
  using T = __nv_bfloat16;
  constexpr int V = 8;
  int n = pr.n;
  if (pr.count) n = min(n, *pr.count);
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int64_t row = pr.rows ? pr.rows[i] : i;
    const bool okrow = row >= 0 && row < pr.n_src;
    if (!okrow && et == 0) flag_error(err, SF_DEV_ERR_INDEX);
    const T* xr = reinterpret_cast<const T*>(pr.x) + (okrow ? row : 0) * pr.D;
    const T* w = reinterpret_cast<const T*>(pr.w);
    float a[MAXV][V], g[MAXV][V];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < MAXV; ++u) {
      const int d = (et + kEpiThreads * u) * V;
      if (d < pr.D) {
        load_vec<T>(xr + d, a[u]);
        load_vec<T>(w + d, g[u]);
#pragma unroll
        for (int k = 0; k < V; ++k) ss = fmaf(a[u][k], a[u][k], ss);
      }
    }
    ss = warp_sum(ss);
    if ((et & 31) == 0) red[et >> 5] = ss;
    epi_sync_all();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < kEpiWarps; ++k) tot += red[k];
    epi_sync_all();
    const float rs = 1.0f / sqrtf(tot / static_cast<float>(pr.D) + pr.eps);
    T* out = reinterpret_cast<T*>(pr.out) + static_cast<int64_t>(i) * pr.D;
#pragma unroll
    for (int u = 0; u < MAXV; ++u) {
      const int d = (et + kEpiThreads * u) * V;
      if (d < pr.D) {
#pragma unroll
        for (int k = 0; k < V; ++k) a[u][k] = g[u][k] * Elt<T>::rnd(a[u][k] * rs);
        if (okrow) store_vec<T>(out + d, a[u]);
      }
    }
  }
}

// The split reduction of a residual GEMM (EPI_RESID, partials of every row) fused with the
// RMSNorm that reads it: for the recomputed rows r = rows[i], i < min(*count, n),
//   x[r]   = T(resid[r] + T(sum_s partial[s][r]))   (the EPI_RESID arithmetic, split order)
//   out[i] = T(w * T(x[r] * rstd))                  (the pre_norm_rows arithmetic)
// from the same registers: one pass over the partials instead of a reduction, a device
// counter hop and a re-read.
template <int MAXV>
__device__ __forceinline__ void pre_resid_norm_rows(const PreNorm& pr, const TcParams& g, int et,
                                                    float* red, int* err) {
  using T = __nv_bfloat16;
  constexpr int V = 8;
  int n = pr.n;
  if (pr.count) n = min(n, *pr.count);
  const int64_t split_stride = static_cast<int64_t>(g.rows_cap) * g.n_out;
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int64_t row = pr.rows[i];
    const bool okrow = row >= 0 && row < pr.n_src && row < g.rows_cap;
    if (!okrow && et == 0) flag_error(err, SF_DEV_ERR_INDEX);
    const int64_t r = okrow ? row : 0;
    const T* w = reinterpret_cast<const T*>(pr.w);
    float a[MAXV][V];
    uint4 gw[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < MAXV; ++u) {
      const int d = (et + kEpiThreads * u) * V;
      if (d < pr.D) {
        float v[V] = {}, rs[V];
        gw[u] = *reinterpret_cast<const uint4*>(w + d);
        sum_splits8(g.partial, g.splits, split_stride, r * g.n_out + d, v);
        ld8<T>(g.epi.resid, r * g.epi.ld_out + d, rs);
#pragma unroll
        for (int k = 0; k < V; ++k) a[u][k] = Elt<T>::rnd(__fadd_rn(rs[k], Elt<T>::rnd(v[k])));
        if (okrow) st8<T>(g.epi.out, r * g.epi.ld_out + d, a[u]);
#pragma unroll
        for (int k = 0; k < V; ++k) ss = fmaf(a[u][k], a[u][k], ss);
      }
    }
    ss = warp_sum(ss);
    if ((et & 31) == 0) red[et >> 5] = ss;
    epi_sync_all();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < kEpiWarps; ++k) tot += red[k];
    epi_sync_all();
    const float rsd = 1.0f / sqrtf(tot / static_cast<float>(pr.D) + pr.eps);
    T* out = reinterpret_cast<T*>(pr.out) + static_cast<int64_t>(i) * pr.D;
#pragma unroll
    for (int u = 0; u < MAXV; ++u) {
      const int d = (et + kEpiThreads * u) * V;
      if (d < pr.D) {
        const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&gw[u]);
#pragma unroll
        for (int k = 0; k < V / 2; ++k) {
          const float2 wf = __bfloat1622float2(wp[k]);
          a[u][2 * k] = wf.x * Elt<T>::rnd(a[u][2 * k] * rsd);
          a[u][2 * k + 1] = wf.y * Elt<T>::rnd(a[u][2 * k + 1] * rsd);
        }
        if (okrow) store_vec<T>(out + d, a[u]);
      }
    }
  }
}

// The rest of that residual GEMM's output: x[r] for the rows the norm did not reduce (not
// flagged for recompute; every row when the compaction overflowed its bucket).  Runs after
// the norm has released the next phase.
__device__ __forceinline__ void resid_rows_rest(const PreNorm& pr, const TcParams& g, int et) {
  using T = __nv_bfloat16;
  const bool all = pr.count != nullptr && *pr.count > pr.n;
  const int64_t split_stride = static_cast<int64_t>(g.rows_cap) * g.n_out;
  const int groups = g.n_out / 8;
  for (int r = blockIdx.x; r < g.rows_cap; r += gridDim.x) {
    if (!all && r < pr.n_src && pr.rec[r] != 0) continue;   // uniform over the CTA
    for (int q = et; q < groups; q += kEpiThreads) {
      const int d = q * 8;
      float v[8] = {}, rs[8], o[8];
      sum_splits8(g.partial, g.splits, split_stride, static_cast<int64_t>(r) * g.n_out + d, v);
      ld8<T>(g.epi.resid, static_cast<int64_t>(r) * g.epi.ld_out + d, rs);
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = __fadd_rn(rs[k], Elt<T>::rnd(v[k]));
      st8<T>(g.epi.out, static_cast<int64_t>(r) * g.epi.ld_out + d, o);
    }
  }
}

// NV: 0 for chains without a fused norm (its code left out: the single GEMMs and the
// lm_head), else the 8-element vectors per thread the norm keeps in registers (D <= 2048
// NV).  The norm's arrays set the register pressure of the whole kernel: sized for
// D <= 8192 they made every chain kernel spill (the QKV GEMM 388 bytes per thread).
template <int K0, int K1, int K2, int NV>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_chain_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW2_0,
                    const __grid_constant__ CUtensorMap tmX0, const __grid_constant__ CUtensorMap tmX64_0,
                    const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmX1,
                    const __grid_constant__ CUtensorMap tmX64_1, const __grid_constant__ CUtensorMap tmW2,
                    const __grid_constant__ CUtensorMap tmX2, const __grid_constant__ CUtensorMap tmX64_2,
                    ChainParams c) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW0);
    tma_prefetch_desc(&tmX0);
    tma_prefetch_desc(&tmX64_0);
    if (c.ph[0].mode == 1 && !c.ph[0].w_tiled) tma_prefetch_desc(&tmW2_0);
    if (c.n_phases > 1) {
      tma_prefetch_desc(&tmW1);
      tma_prefetch_desc(&tmX1);
      tma_prefetch_desc(&tmX64_1);
    }
    if (c.n_phases > 2) {
      tma_prefetch_desc(&tmW2);
      tma_prefetch_desc(&tmX2);
      tma_prefetch_desc(&tmX64_2);
    }
  }
  pdl_trigger();
  pdl_wait();
  int rows_ph[kMaxPhases] = {0, 0, 0};
  int max_rows = 0;
  for (int k = 0; k < c.n_phases; ++k) {
    int r = c.ph[k].rows_cap;
    if (c.ph[k].count) r = min(r, *c.ph[k].count);
    rows_ph[k] = max(r, 0);
    max_rows = max(max_rows, rows_ph[k]);
  }
  if (max_rows <= 0) return;                     // uniform over the grid
  // stage layout from the actual row counts: phase k puts its sub_k weight tiles first and its activation rows right
  // after them; the stage size is the largest over the phases
  int stage_bytes = 0, buf_cols_i = 0;
  int acc_ph[kMaxPhases] = {128, 128, 128};
  for (int k = 0; k < c.n_phases; ++k) {
    const int xr = rows_ph[k] > 0 ? x_rows_loaded(min(rows_ph[k], kMaxPassRows)) : 0;
    stage_bytes = max(stage_bytes, c.ph[k].sub * kWBytes + xr * kXRowBytes);
    // TMEM columns per accumulator from the phase's actual rows
    acc_ph[k] = rows_ph[k] <= 128 ? 128 : 256;
    buf_cols_i = max(buf_cols_i, c.ph[k].sub * acc_ph[k]);
  }
  const int stages = min(kMaxStages, c.stage_budget / stage_bytes);
  // TMEM: double-buffered when two accumulators fit (one unit's epilogue overlaps the next)
  const bool double_buf = 2 * buf_cols_i * c.ctas_per_sm <= 512;
  const uint32_t buf_cols = buf_cols_i;
  const uint32_t tmem_cols = (double_buf ? 2u : 1u) * buf_cols;
  unsigned char* stage_base = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + c.stage_budget + kTileTBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* acc_full = bars + 2 * kMaxStages;    // [2]
  uint64_t* acc_empty = acc_full + 2;            // [2]
  uint64_t* drain = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 2);   // [kEpiWarps] norm partial sums
  const int total_units = c.unit_base[c.n_phases];

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
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
      // activation loads of the stages issued before a phase's input was ready
      struct Pending { unsigned char* st; uint64_t* bar; int kx, prow0, x_rows; };
      Pending pend[kMaxStages];
      int npend = 0;
      bool dep_ok[kMaxPhases];
      for (int k = 0; k < kMaxPhases; ++k) {
        unsigned tg;
        dep_ok[k] = k >= c.n_phases || phase_dep(c, k, &tg) == nullptr;
      }
      int it = 0;
      for (int u = blockIdx.x; u < total_units && !*abort_flag; u += gridDim.x) {
        const int ph = u >= c.unit_base[2] ? 2 : (u >= c.unit_base[1] ? 1 : 0);
        const TcParams& p = c.ph[ph];
        const CUtensorMap* mW = ph == 2 ? &tmW2 : (ph ? &tmW1 : &tmW0);
        const CUtensorMap* mX = ph == 2 ? &tmX2 : (ph ? &tmX1 : &tmX0);
        const CUtensorMap* mX64 = ph == 2 ? &tmX64_2 : (ph ? &tmX64_1 : &tmX64_0);
        const int rows = rows_ph[ph];
        const int n_pass = (rows + kMaxPassRows - 1) / kMaxPassRows;
        const int lu = u - c.unit_base[ph];
        const int grp = lu / p.splits, split = lu % p.splits;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        auto flush = [&]() -> bool {
          unsigned tg = 0;
          const unsigned* dc = phase_dep(c, ph, &tg);
          if (dc != nullptr && !wait_counter(dc, tg, c.err)) return false;
          fence_proxy_async_global();
          for (int k = 0; k < npend; ++k)
            for (int r = 0; r < pend[k].x_rows; r += 128) {
              const bool wide = pend[k].x_rows - r > 64;
              tma_load_2d(pend[k].st + p.sub * kWBytes + r * kXRowBytes, wide ? mX : mX64, pend[k].bar,
                          pend[k].kx, pend[k].prow0 + r, pol_x);
            }
          npend = 0;
          dep_ok[ph] = true;
          return true;
        };
        for (int pass = 0; pass < n_pass && !*abort_flag; ++pass) {
          const int prow0 = pass * kMaxPassRows;
          const int prows = min(kMaxPassRows, rows - prow0);
          const int x_rows = x_rows_loaded(prows);
          const uint32_t bytes = p.sub * kWBytes + x_rows * kXRowBytes;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % stages;
            const uint32_t phs = (it / stages) & 1;
            if (!mbar_wait(&empty[s], phs ^ 1, p.err)) { *abort_flag = 1; break; }
            unsigned char* st = stage_base + s * stage_bytes;
            mbar_arrive_expect_tx(&full[s], bytes);
            const int kx = kb * kBK;
            for (int t = 0; t < p.sub; ++t) {
              const int tile = grp * p.sub + t;
              unsigned char* wdst = st + t * kWBytes;
              if (p.w_tiled) {
                tma_load_2d(wdst, mW, &full[s], 0, (tile * p.kb_total + kb) * kTileF, pol_w);
              } else if (p.mode == 1) {
                tma_load_2d(wdst, &tmW0, &full[s], kx, tile * 64, pol_w);
                tma_load_2d(wdst + kWBytes / 2, &tmW2_0, &full[s], kx, tile * 64, pol_w);
              } else {
                tma_load_2d(wdst, mW, &full[s], kx, tile * kTileF, pol_w);
              }
            }
            if (dep_ok[ph]) {
              for (int r = 0; r < x_rows; r += 128) {
                const bool wide = x_rows - r > 64;
                tma_load_2d(st + p.sub * kWBytes + r * kXRowBytes, wide ? mX : mX64, &full[s], kx,
                            prow0 + r, pol_x);
              }
            } else {
              pend[npend++] = {st, &full[s], kx, prow0, x_rows};
              // every stage holds weights waiting for activations: wait for the input now
              if (npend == stages && !flush()) { *abort_flag = 1; break; }
            }
          }
        }
        if (npend > 0 && !*abort_flag && !flush()) *abort_flag = 1;
      }
      // HBM is about to idle for this kernel's tail: start the next GEMM's weights
      if (!*abort_flag) issue_w_prefetch(c.ph[c.n_phases - 1].next_pf, blockIdx.x, gridDim.x);
      // no copy into this CTA's shared memory may still be in flight at exit
      for (int i = max(0, it - stages); i < it; ++i)
        mbar_wait(&full[i % stages], (i / stages) & 1, c.err);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0, acc_it = 0;
      for (int u = blockIdx.x; u < total_units && !*abort_flag; u += gridDim.x) {
        const int ph = u >= c.unit_base[2] ? 2 : (u >= c.unit_base[1] ? 1 : 0);
        const TcParams& p = c.ph[ph];
        const int rows = rows_ph[ph];
        const int n_pass = (rows + kMaxPassRows - 1) / kMaxPassRows;
        const int lu = u - c.unit_base[ph];
        const int split = lu % p.splits;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        bool ok = true;
        for (int pass = 0; pass < n_pass && ok; ++pass, ++acc_it) {
          const int prows = min(kMaxPassRows, rows - pass * kMaxPassRows);
          const int n_mma = ((prows + 15) / 16) * 16;
          const uint32_t idesc = idesc_bf16(128, n_mma);
          const int buf = double_buf ? (acc_it & 1) : 0;
          const uint32_t par = double_buf ? ((acc_it >> 1) & 1) : (acc_it & 1);
          if (!mbar_wait(&acc_empty[buf], par ^ 1, p.err)) { *abort_flag = 1; ok = false; break; }
          tc_fence_after();
          const uint32_t d0 = tmem + buf * buf_cols;
          for (int i = 0; i < kb1 - kb0; ++i, ++it) {
            const int s = it % stages;
            const uint32_t phs = (it / stages) & 1;
            if (*abort_flag || !mbar_wait(&full[s], phs, p.err)) { *abort_flag = 1; ok = false; break; }
            tc_fence_after();
            const uint32_t a0 = smem_u32(stage_base + s * stage_bytes);
            const uint32_t b0 = a0 + p.sub * kWBytes;
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              const uint64_t bd = sdesc_kmajor_sw128(b0 + k * 32);
              for (int t = 0; t < p.sub; ++t)
                umma_f16(d0 + t * acc_ph[ph], sdesc_kmajor_sw128(a0 + t * kWBytes + k * 32), bd,
                         idesc, (i > 0 || k > 0) ? 1u : 0u);
            }
            umma_commit(&empty[s]);
          }
          if (!ok) break;
          umma_commit(&acc_full[buf]);
        }
        if (!ok) break;
      }
      umma_commit(drain);                 // every issued MMA done before TMEM is freed
      mbar_wait(drain, 0, c.err);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // Two warps per TMEM lane quarter: half h takes the even (h = 0) or odd (h = 1)
    // chunks of kChunk activation rows, so two chunks are in flight per SM sub-partition.
    EpiCtx x;
    x.tmem = tmem;
    x.buf_cols = buf_cols;
    x.q = warp & 3;                       // TMEM lane quarter of this warp
    x.l = x.q * 32 + lane;                // tile-local weight row == TMEM lane
    x.et = threadIdx.x - 64;              // 0..255 within the epilogue warps
    x.h = x.et >> 7;                      // epilogue half
    x.eh = x.et & 127;                    // thread within the half
    x.tileT = reinterpret_cast<float*>(smem + c.stage_budget) + x.h * kChunk * kTileLd;
    x.abort_flag = abort_flag;
    int acc_it = 0;
    for (int k = 0; k < c.n_phases; ++k) {
      if (NV > 0 && c.norm[k].x != nullptr) {
        // the norm reads every row of the previous phase's output
        if (k > 0) {
          bool ok = true;
          if (x.et == 0)
            ok = wait_counter(c.dep + 2 * (k - 1) + 1, static_cast<unsigned>(c.ph[k - 1].n_units), c.err);
          if (!epi_vote_all(ok && !*abort_flag)) *abort_flag = 1;
        }
        const bool fused = k > 0 && c.ph[k - 1].defer_reduce;
        if constexpr (NV > 0) {
          if (!*abort_flag) {
            if (fused) pre_resid_norm_rows<NV>(c.norm[k], c.ph[k - 1], x.et, red, c.err);
            else pre_norm_rows<NV>(c.norm[k], x.et, red, c.err);
          }
        }
        epi_sync_all();
        if (x.et == 0) {
          __threadfence();
          fence_proxy_async_global();
          atomicAdd(c.dep + 2 * k, 1u);
        }
        // the residual rows no later phase reads, while phase k streams its weights
        if constexpr (NV > 0)
          if (fused && !*abort_flag) resid_rows_rest(c.norm[k], c.ph[k - 1], x.et);
      }
      // this CTA's units of phase k: u = blockIdx.x + j * gridDim.x in the phase's range
      const int base = c.unit_base[k];
      const int first = base + ((static_cast<int>(blockIdx.x) - base) % static_cast<int>(gridDim.x) +
                                static_cast<int>(gridDim.x)) % static_cast<int>(gridDim.x);
      for (int u = first; u < c.unit_base[k + 1]; u += gridDim.x) {
        const int lu = u - base;
        x.acc_cols = acc_ph[k];
        if (k == 0)
          epi_unit<K0>(c.ph[0], x, lu, rows_ph[0], acc_it, double_buf, acc_full, acc_empty);
        else if (k == 1)
          epi_unit<K1>(c.ph[1], x, lu, rows_ph[1], acc_it, double_buf, acc_full, acc_empty);
        else
          epi_unit<K2>(c.ph[2], x, lu, rows_ph[2], acc_it, double_buf, acc_full, acc_empty);
        if (k + 1 < c.n_phases && !c.ph[k + 1].no_dep) {
          // this unit's output is the next phase's input
          epi_sync_all();
          if (x.et == 0) {
            __threadfence();
            fence_proxy_async_global();
            atomicAdd(c.dep + 2 * k + 1, 1u);
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
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
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

// Tuning, read once from the environment: SF_GEMM_SUB (weight tiles per CTA stage: 0 =
// chosen per GEMM, or 1 / 2 / 4 wherever TMEM allows), SF_GEMM_SMEM_KB (shared memory
// per CTA; below ~113 two CTAs share an SM) and SF_QKV_SPLITS (split-K of the QKV GEMM).
constexpr int kDefaultSmemKb = 170;
constexpr int kMaxSmemKb = 226;
struct TcTuning {
  int sub = 0;
  int smem_kb = kDefaultSmemKb;
  int pf_mb = 0;       // SF_GEMM_PF_MB: L2 prefetch budget for the next GEMM's weights
                       // (off: measured, the step got slower at 40 and 80 MB)
  int qkv_splits = 0;  // SF_QKV_SPLITS: split-K count of the QKV GEMM (0: chosen)
  int pf_kind_mb[6] = {-1, -1, -1, -1, -1, -1};   // SF_GEMM_PF_MB_<kind>: the budget of the
                                                  // GEMM with epilogue <kind> (0..5) only
};
static const TcTuning& tc_tuning() {
  static TcTuning t;
  static std::once_flag once;
  std::call_once(once, [] {
    if (const char* v = getenv("SF_GEMM_SUB")) {
      const int s = atoi(v);
      t.sub = (s == 1 || s == 2 || s == 4) ? s : 0;
    }
    if (const char* v = getenv("SF_GEMM_SMEM_KB")) t.smem_kb = std::max(64, std::min(kMaxSmemKb, atoi(v)));
    if (const char* v = getenv("SF_GEMM_PF_MB")) t.pf_mb = std::max(0, std::min(96, atoi(v)));
    if (const char* v = getenv("SF_QKV_SPLITS")) t.qkv_splits = std::max(0, std::min(16, atoi(v)));
    for (int k = 0; k < 6; ++k) {
      char name[32];
      snprintf(name, sizeof(name), "SF_GEMM_PF_MB_%d", k);
      if (const char* v = getenv(name)) t.pf_kind_mb[k] = std::max(0, std::min(96, atoi(v)));
    }
  });
  return t;
}

struct TcPlan {
  int n_tiles, sub, n_groups, splits, kb_total, kb_per_split, acc_cols, double_buf, grid;
  int stage_budget, ctas_per_sm;
};
static TcPlan tc_plan(int n_out, int K, int kind, int inter, int rows_cap) {
  const int mode = kind == EPI_SWIGLU ? 1 : 0;
  TcPlan pl{};
  pl.n_tiles = mode == 1 ? (inter + 63) / 64 : (n_out + kTileF - 1) / kTileF;
  pl.kb_total = (K + kBK - 1) / kBK;
  const TcTuning& tune = tc_tuning();
  pl.acc_cols = rows_cap <= 128 ? 128 : 256;
  const int sms = num_sms();
  // Weight tiles per stage: each CTA re-reads the activations from L2 for every stage, so
  // `sub` tiles per stage cut that traffic per weight byte by `sub`.  Chosen where the
  // tile groups still fill the SMs without splitting K (a wider unit under split-K
  // multiplies the fp32 partials instead); TMEM holds sub x acc_cols columns.
  if (tune.sub > 0) {
    pl.sub = tune.sub;
  } else if (pl.n_tiles >= 2 * sms) {
    pl.sub = 2;
  } else {
    // split-K regime: two tiles per stage when each split still streams >= 16 k-blocks
    // (the doubled partials are a fixed cost per CTA; the halved activation re-reads pay
    // over a long K range, e.g. the down projection)
    const int g2 = (pl.n_tiles + 1) / 2;
    const int s2 = std::max(1, std::min(sms / g2, pl.kb_total / 4));
    pl.sub = (pl.n_tiles >= 2 && pl.kb_total / s2 >= 16) ? 2 : 1;
  }
  while (pl.sub > 1 && (pl.sub * pl.acc_cols > 512 || pl.n_tiles < pl.sub)) pl.sub >>= 1;
  pl.stage_budget = tune.smem_kb * 1024 - kSmemFixed;
  pl.ctas_per_sm = std::max(1, (227 * 1024) / (tune.smem_kb * 1024 + 1024));
  pl.n_groups = (pl.n_tiles + pl.sub - 1) / pl.sub;
  int splits = 1;
  // few tile groups: split K so that groups x splits fills the SMs (one pass of rows)
  if (rows_cap <= kMaxPassRows && pl.n_groups < sms / 2 && pl.n_groups <= kMaxCounterTiles)
    splits = std::max(1, std::min(sms / pl.n_groups, pl.kb_total / 4));
  // (every split of a group must be resident at once: at most the SMs' CTA slots)
  if (kind == EPI_QKV && tune.qkv_splits > 0 && splits > 1)
    splits = std::max(1, std::min(std::min(tune.qkv_splits, pl.kb_total),
                                  sms * pl.ctas_per_sm / std::max(1, pl.n_groups)));
  pl.kb_per_split = (pl.kb_total + splits - 1) / splits;
  pl.splits = (pl.kb_total + pl.kb_per_split - 1) / pl.kb_per_split;  // no empty split
  const int n_units = pl.n_groups * pl.splits;
  pl.grid = pl.splits > 1 ? n_units : std::min(n_units, sms * pl.ctas_per_sm);
  const bool want_double = n_units > pl.grid || rows_cap > kMaxPassRows;
  // TMEM (512 columns per SM) is shared by the CTAs resident on an SM
  pl.double_buf = (want_double && 2 * pl.sub * pl.acc_cols * pl.ctas_per_sm <= 512) ? 1 : 0;
  return pl;
}

WPrefetch gemm_prefetch_plan(const GemmArgs& a) {
  WPrefetch f{};
  if (a.dtype != BF16 || !a.w_tiled || a.W == nullptr) return f;
  const TcPlan pl = tc_plan(a.n_out, a.K, a.epi.kind, a.epi.inter, a.rows_cap);
  const int64_t per_kb = static_cast<int64_t>(pl.n_groups) * pl.splits * pl.sub * kWBytes;
  const TcTuning& tune = tc_tuning();
  const int kind_mb = a.epi.kind >= 0 && a.epi.kind < 6 ? tune.pf_kind_mb[a.epi.kind] : -1;
  const int64_t budget = static_cast<int64_t>(kind_mb >= 0 ? kind_mb : tune.pf_mb) << 20;
  const int npf = static_cast<int>(std::min<int64_t>(pl.kb_per_split, per_kb > 0 ? budget / per_kb : 0));
  if (npf <= 0) return f;
  f.w = a.W;
  f.n_tiles = pl.n_tiles;
  f.sub = pl.sub;
  f.splits = pl.splits;
  f.kb_total = pl.kb_total;
  f.kb_per_split = pl.kb_per_split;
  f.n_units = pl.n_groups * pl.splits;
  f.npf = npf;
  return f;
}

static int wave_tail_tiles0(int n_out, int K, int kind, int rows_cap, int* splits1);

size_t gemm_tc_ws_need(int rows_cap, int n_out, int K, int kind, int inter) {
  const TcPlan pl = tc_plan(n_out, K, kind, inter, rows_cap);
  if (pl.splits <= 1) {
    int s1 = 0;
    const int tiles0 = wave_tail_tiles0(n_out, K, kind, rows_cap, &s1);
    if (tiles0 <= 0) return 0;
    return kGemmCounterBytes + static_cast<size_t>(s1) * rows_cap * (n_out - tiles0 * kTileF) * 4;
  }
  return kGemmCounterBytes + static_cast<size_t>(pl.splits) * rows_cap * n_out * 4;
}

int gemm_path_is_tc(int dtype) { return dtype == BF16; }

// Phase parameters and tensor maps of one GEMM (counters at `counters`, partials after
// the counter region of the workspace).
static cudaError_t make_phase(const GemmArgs& a, int* counters, TcParams* out, TcPlan* plan,
                              CUtensorMap* tmW, CUtensorMap* tmW2, CUtensorMap* tmX,
                              CUtensorMap* tmX64) {
  const int mode = a.epi.kind == EPI_SWIGLU ? 1 : 0;
  const int inter = a.epi.inter;
  if (a.n_out % 8 != 0 || (mode == 1 && inter % 8 != 0)) return cudaErrorInvalidValue;
  const TcPlan pl = tc_plan(a.n_out, a.K, a.epi.kind, inter, a.rows_cap);
  TcParams p{};
  p.n_out = a.n_out;
  p.K = a.K;
  p.rows_cap = a.rows_cap;
  p.count = a.count;
  p.mode = mode;
  p.inter = inter;
  p.n_tiles = pl.n_tiles;
  p.sub = pl.sub;
  p.n_groups = pl.n_groups;
  p.splits = pl.splits;
  p.kb_total = pl.kb_total;
  p.kb_per_split = pl.kb_per_split;
  p.n_units = pl.n_groups * pl.splits;
  p.w_tiled = a.w_tiled ? 1 : 0;
  p.stage_budget = pl.stage_budget;
  p.next_pf = a.next_pf;

  if (pl.splits > 1) {
    const size_t need = kGemmCounterBytes + static_cast<size_t>(pl.splits) * a.rows_cap * a.n_out * 4;
    if (a.ws == nullptr || a.ws_bytes < need) return cudaErrorInvalidValue;
    p.counters = counters;
    p.partial = reinterpret_cast<float*>(static_cast<char*>(a.ws) + kGemmCounterBytes);
  }
  p.epi = a.epi;
  p.err = a.err;
  if (p.w_tiled) {
    const uint64_t blocks = static_cast<uint64_t>(pl.n_tiles) * pl.kb_total * kTileF;
    if (!make_tmap(tmW, a.W, blocks, kBK, kTileF)) return cudaErrorInvalidValue;
    *tmW2 = *tmW;
  } else {
    const uint32_t wrows = mode == 1 ? 64 : kTileF;
    const int w_rows_total = mode == 1 ? inter : a.n_out;
    if (!make_tmap(tmW, a.W, w_rows_total, a.K, wrows)) return cudaErrorInvalidValue;
    if (!make_tmap(tmW2, mode == 1 ? a.W2 : a.W, w_rows_total, a.K, wrows))
      return cudaErrorInvalidValue;
  }
  if (!make_tmap(tmX, a.X, a.rows_cap, a.K, 128) || !make_tmap(tmX64, a.X, a.rows_cap, a.K, 64))
    return cudaErrorInvalidValue;
  *out = p;
  *plan = pl;
  return cudaSuccess;
}

using ChainFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap,
                         CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap,
                         ChainParams);

// the instantiation for the phase kinds k[0..n) and the norm's vector count nv (0: none)
template <int NV>
static ChainFn chain_kernel_nv(int n, const int* k) {
  if (n == 2 && k[0] == EPI_SWIGLU && k[1] == EPI_SCATTER)
    return tc_chain_kernel<EPI_SWIGLU, EPI_SCATTER, EPI_SCATTER, NV>;
  // tensor parallel: the down projection's fp32 partial sums go to the exchange
  if (n == 2 && k[0] == EPI_SWIGLU && k[1] == EPI_RAW)
    return tc_chain_kernel<EPI_SWIGLU, EPI_RAW, EPI_RAW, NV>;
  if (n == 3 && k[0] == EPI_RESID && k[1] == EPI_SWIGLU && k[2] == EPI_SCATTER)
    return tc_chain_kernel<EPI_RESID, EPI_SWIGLU, EPI_SCATTER, NV>;
  return nullptr;
}
static ChainFn chain_kernel(int n, const int* k, int nv) {
  if (nv == 3) return chain_kernel_nv<3>(n, k);
  if (nv == 4) return chain_kernel_nv<4>(n, k);
  if (nv != 0) return nullptr;
  if (n == 1) {
    switch (k[0]) {
      case EPI_RAW: return tc_chain_kernel<EPI_RAW, EPI_RAW, EPI_RAW, 0>;
      case EPI_QKV: return tc_chain_kernel<EPI_QKV, EPI_QKV, EPI_QKV, 0>;
      case EPI_RESID: return tc_chain_kernel<EPI_RESID, EPI_RESID, EPI_RESID, 0>;
      case EPI_SWIGLU: return tc_chain_kernel<EPI_SWIGLU, EPI_SWIGLU, EPI_SWIGLU, 0>;
      case EPI_SCATTER: return tc_chain_kernel<EPI_SCATTER, EPI_SCATTER, EPI_SCATTER, 0>;
      case EPI_LOGITS: return tc_chain_kernel<EPI_LOGITS, EPI_LOGITS, EPI_LOGITS, 0>;
      default: return nullptr;
    }
  }
  // a long GEMM and its wave tail (independent phases of one epilogue kind)
  if (n == 2 && k[0] == k[1] && (k[0] == EPI_LOGITS || k[0] == EPI_RAW))
    return k[0] == EPI_LOGITS ? tc_chain_kernel<EPI_LOGITS, EPI_LOGITS, EPI_LOGITS, 0>
                              : tc_chain_kernel<EPI_RAW, EPI_RAW, EPI_RAW, 0>;
  return nullptr;
}

static void set_norm(PreNorm* d, const PreNormArgs* s) {
  d->x = s->x;
  d->rows = s->rows;
  d->count = s->count;
  d->w = s->w;
  d->out = s->out;
  d->n = s->n;
  d->n_src = s->n_src;
  d->D = s->D;
  d->eps = s->eps;
  d->rec = s->rec;
}

// indep: bit k set -> phase k does not read phase k-1's output (no counter wait)
static cudaError_t chain_launch(const GemmArgs* g, int n, const PreNormArgs* const* norms,
                                unsigned* dep, cudaStream_t st, unsigned indep) {
  if (n < 1 || n > kMaxPhases) return cudaErrorInvalidValue;
  bool any_norm = false, any_dep = false;
  for (int k = 0; k < n; ++k) {
    any_norm = any_norm || (norms != nullptr && norms[k] != nullptr);
    any_dep = any_dep || (k > 0 && !((indep >> k) & 1u));
    if (k > 0 && ((indep >> k) & 1u) && norms != nullptr && norms[k] != nullptr)
      return cudaErrorInvalidValue;
  }
  if ((any_dep || any_norm) && dep == nullptr) return cudaErrorInvalidValue;
  ChainParams c{};
  CUtensorMap tm[kMaxPhases][4];
  TcPlan pl[kMaxPhases];
  int kinds[kMaxPhases];
  int max_norm_d = 0;
  int* counters = static_cast<int*>(g[0].ws);
  for (int k = 0; k < n; ++k) {
    // untiled SwiGLU reads its up half through phase 0's second weight map: phase 0 only
    if (k > 0 && !g[k].w_tiled && g[k].epi.kind == EPI_SWIGLU) return cudaErrorInvalidValue;
    cudaError_t e = make_phase(g[k], counters, &c.ph[k], &pl[k], &tm[k][0], &tm[k][1], &tm[k][2],
                               &tm[k][3]);
    if (e != cudaSuccess) return e;
    c.ph[k].no_dep = (k > 0 && ((indep >> k) & 1u)) ? 1 : 0;
    if (pl[k].splits > 1) counters += 2 * pl[k].n_groups;   // each split phase its own counters
    kinds[k] = g[k].epi.kind;
    if (norms != nullptr && norms[k] != nullptr) {
      if (norms[k]->D % 8 != 0 || norms[k]->D > kEpiThreads * 8 * 4) return cudaErrorInvalidValue;
      max_norm_d = std::max(max_norm_d, norms[k]->D);
      set_norm(&c.norm[k], norms[k]);
    }
  }
  // a split-K residual GEMM over every row followed by the norm of its output: the norm
  // performs the split reduction (pre_resid_norm_rows / resid_rows_rest)
  static const bool defer_on = getenv("SF_DEFER") == nullptr || atoi(getenv("SF_DEFER")) != 0;
  for (int k = 1; k < n; ++k)
    if (defer_on && norms != nullptr && norms[k] != nullptr && norms[k]->rec != nullptr && norms[k]->rows != nullptr &&
        g[k - 1].epi.kind == EPI_RESID && pl[k - 1].splits > 1 && g[k - 1].count == nullptr &&
        norms[k]->x == g[k - 1].epi.out && g[k - 1].epi.ld_out == g[k - 1].n_out &&
        norms[k]->D == g[k - 1].n_out && g[k - 1].n_out % 8 == 0) {
      // the deferred partials are read after the norm has released phase k, while later
      // split phases write theirs: they get a region of their own, after the largest of
      // the other split phases' (which run one after another and share theirs)
      size_t other = 0;
      for (int j = 0; j < n; ++j)
        if (j != k - 1 && pl[j].splits > 1)
          other = std::max(other, static_cast<size_t>(pl[j].splits) * g[j].rows_cap * g[j].n_out * 4);
      const size_t mine = static_cast<size_t>(pl[k - 1].splits) * g[k - 1].rows_cap * g[k - 1].n_out * 4;
      if (g[k - 1].ws == nullptr || kGemmCounterBytes + other + mine > g[k - 1].ws_bytes) continue;
      c.ph[k - 1].partial = reinterpret_cast<float*>(static_cast<char*>(g[k - 1].ws) + kGemmCounterBytes + other);
      c.ph[k - 1].defer_reduce = 1;
    }
  for (int k = n; k < kMaxPhases; ++k) tm[k][0] = tm[k][1] = tm[k][2] = tm[k][3] = tm[0][0];
  if (counters - static_cast<int*>(g[0].ws) > kMaxCounterTiles * 2) return cudaErrorInvalidValue;
  c.n_phases = n;
  int grid = 0;
  bool coop = n > 1 || any_norm;
  c.unit_base[0] = 0;
  for (int k = 0; k < kMaxPhases; ++k) {
    c.unit_base[k + 1] = c.unit_base[k] + (k < n ? c.ph[k].n_units : 0);
    if (k >= n) continue;
    grid = std::max(grid, pl[k].grid);
    c.max_sub = std::max(c.max_sub, pl[k].sub);
    coop = coop || pl[k].splits > 1;
  }
  // split phases: every unit on its own resident CTA (the splits of a group wait on each
  // other); the persistent grid serves all phases
  for (int k = 0; k < n; ++k)
    if (pl[k].splits > 1 && c.ph[k].n_units > grid) return cudaErrorInvalidValue;
  c.stage_budget = pl[0].stage_budget;
  c.ctas_per_sm = pl[0].ctas_per_sm;
  // the lm_head streams 256 activation rows with two weight tiles per stage (64 KB
  // stages): at the default budget it keeps two stages in flight and waits on latency;
  // the largest budget gives it three (measured 301 -> 275 us per step at the 7B shape;
  // the other GEMMs measured no faster or slower with it)
  bool all_logits = tc_tuning().smem_kb == kDefaultSmemKb;
  for (int k = 0; k < n; ++k) all_logits = all_logits && g[k].epi.kind == EPI_LOGITS;
  if (all_logits) {
    c.stage_budget = kMaxSmemKb * 1024 - kSmemFixed;
    c.ctas_per_sm = 1;
  }

  c.err = g[0].err;
  c.dep = dep;

  const int nv = max_norm_d == 0 ? 0 : (max_norm_d <= kEpiThreads * 8 * 3 ? 3 : 4);
  ChainFn kern = chain_kernel(n, kinds, nv);
  if (kern == nullptr) return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(c.stage_budget) + kSmemFixed;
  {
    static std::mutex mu;
    static std::vector<std::pair<std::pair<int, ChainFn>, size_t>> configured;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    bool done = false;
    for (auto& cf : configured)
      if (cf.first.first == dev && cf.first.second == kern && cf.second >= smem) done = true;
    if (!done) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      configured.push_back({{dev, kern}, smem});
    }
  }
  cudaError_t e = launch_ex(kern, dim3(grid), dim3(kTcThreads), smem, st, coop, tm[0][0],
                            tm[0][1], tm[0][2], tm[0][3], tm[1][0], tm[1][2], tm[1][3], tm[2][0],
                            tm[2][2], tm[2][3], c);
  if (e != cudaSuccess) return e;
  return launched();
}

cudaError_t gemm_chain(const GemmArgs* g, int n, const PreNormArgs* const* norms, unsigned* dep,
                       cudaStream_t st) {
  return chain_launch(g, n, norms, dep, st, 0u);
}

// Wave tail of a long unsplit GEMM (the lm_head: 594 two-tile units on 148 CTAs leave a
// fifth round of 2 units, a whole unit's time with the GPU nearly idle): when the last
// round is at most a quarter full, its tiles become a second, independent phase of the
// same launch, split over K across the CTAs that would otherwise idle.  Same MMAs per
// tile; only the unit boundaries move (the split sums add in split order).
// tiles of the full rounds (0: no tail split) and the tail phase's split count
static int wave_tail_tiles0(int n_out, int K, int kind, int rows_cap, int* splits1) {
  if ((kind != EPI_LOGITS && kind != EPI_RAW) || rows_cap > kMaxPassRows) return 0;
  const TcPlan pl = tc_plan(n_out, K, kind, 0, rows_cap);
  if (pl.splits > 1) return 0;
  const int n_units = pl.n_groups * pl.splits;
  const int rem = n_units % pl.grid;
  if (rem == 0 || rem * 4 > pl.grid) return 0;
  const int tiles0 = (n_units - rem) * pl.sub;
  const TcPlan p1 = tc_plan(n_out - tiles0 * kTileF, K, kind, 0, rows_cap);
  if (p1.splits <= 1 || p1.n_groups * p1.splits > pl.grid) return 0;
  *splits1 = p1.splits;
  return tiles0;
}

static bool split_wave_tail(const GemmArgs& a, GemmArgs* g) {
  if (a.dtype != BF16) return false;
  int s1 = 0;
  const int tiles0 = wave_tail_tiles0(a.n_out, a.K, a.epi.kind, a.rows_cap, &s1);
  if (tiles0 <= 0) return false;
  const TcPlan pl = tc_plan(a.n_out, a.K, a.epi.kind, 0, a.rows_cap);
  const int n1 = a.n_out - tiles0 * kTileF;
  const size_t need = kGemmCounterBytes + static_cast<size_t>(s1) * a.rows_cap * n1 * 4;
  if (a.ws == nullptr || a.ws_bytes < need) return false;
  g[0] = a;
  g[0].n_out = tiles0 * kTileF;
  g[1] = a;
  g[1].n_out = n1;
  const size_t w_off = a.w_tiled ? static_cast<size_t>(tiles0) * pl.kb_total * kWBytes
                                 : static_cast<size_t>(tiles0) * kTileF * a.K * 2;
  g[1].W = static_cast<const char*>(a.W) + w_off;
  const size_t esz = a.epi.kind == EPI_RAW ? 4 : 2;
  g[1].epi.out = static_cast<char*>(a.epi.out) + static_cast<size_t>(tiles0) * kTileF * esz;
  g[0].next_pf = WPrefetch{};
  return true;
}

cudaError_t gemm_tc(const GemmArgs& a, cudaStream_t st) {
  static const bool tail_on = getenv("SF_WAVE_TAIL") == nullptr || atoi(getenv("SF_WAVE_TAIL")) != 0;
  GemmArgs g[2];
  if (tail_on && split_wave_tail(a, g)) return chain_launch(g, 2, nullptr, nullptr, st, 2u);
  return chain_launch(&a, 1, nullptr, nullptr, st, 0u);
}

// ------------------------------------------------------------------ weight tiling
// dst[(t*kb_total + kb)*128 + r][c] = W row (t, r) at column kb*64 + c (zero past the
// matrix).  mode 1: r < 64 -> gate row t*64 + r, r >= 64 -> up row t*64 + r - 64.
// One thread per 16-byte destination vector (K is a multiple of 8).
__global__ void pack_tiles_kernel(const __nv_bfloat16* W, const __nv_bfloat16* W2, int n_out,
                                  int K, int mode, int inter, int n_tiles, int kb_total,
                                  __nv_bfloat16* dst) {
  const int64_t total = static_cast<int64_t>(n_tiles) * kb_total * kTileF * (kBK / 8);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = static_cast<int>(i % (kBK / 8));
    const int64_t row = i / (kBK / 8);
    const int r = static_cast<int>(row % kTileF);
    const int64_t tk = row / kTileF;
    const int kb = static_cast<int>(tk % kb_total);
    const int t = static_cast<int>(tk / kb_total);
    const int col = kb * kBK + v * 8;
    const __nv_bfloat16* src = nullptr;
    if (mode == 1) {
      const int g = t * 64 + (r & 63);
      if (g < inter) src = (r < 64 ? W : W2) + static_cast<int64_t>(g) * K;
    } else {
      const int f = t * kTileF + r;
      if (f < n_out) src = W + static_cast<int64_t>(f) * K;
    }
    uint4 val = make_uint4(0, 0, 0, 0);
    if (src != nullptr && col < K) val = *reinterpret_cast<const uint4*>(src + col);
    *reinterpret_cast<uint4*>(dst + row * kBK + v * 8) = val;
  }
}

size_t weight_tiles_bytes(int n_out, int K, int mode, int inter) {
  const int n_tiles = mode == 1 ? (inter + 63) / 64 : (n_out + kTileF - 1) / kTileF;
  const int kb_total = (K + kBK - 1) / kBK;
  return static_cast<size_t>(n_tiles) * kb_total * kTileF * kBK * 2;
}

cudaError_t pack_weight_tiles(const void* W, const void* W2, int n_out, int K, int mode,
                              int inter, void* dst, cudaStream_t st) {
  if (K % 8 != 0 || (mode == 1 && W2 == nullptr)) return cudaErrorInvalidValue;
  const int n_tiles = mode == 1 ? (inter + 63) / 64 : (n_out + kTileF - 1) / kTileF;
  const int kb_total = (K + kBK - 1) / kBK;
  const int64_t total = static_cast<int64_t>(n_tiles) * kb_total * kTileF * (kBK / 8);
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  pack_tiles_kernel<<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(W),
                                            static_cast<const __nv_bfloat16*>(W2), n_out, K,
                                            mode, inter, n_tiles, kb_total,
                                            static_cast<__nv_bfloat16*>(dst));
  return launched();
}

}  // namespace sf
