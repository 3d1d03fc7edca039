// Internal launcher interface shared by the .cu files of the library.
#pragma once

#include <utility>

#include "sf_common.cuh"

namespace sf {

constexpr int kMaxBranches = 32;         // B1 limit (one warp per branch in the gate)
constexpr int kMaxRows = 1024;           // B1*N limit of the compaction scan
constexpr int kMaxGateSmem = 227 * 1024;

// Launch with programmatic stream serialization (the kernel may begin while the previous
// one finishes; it calls pdl_wait() before touching what that kernel produces), plus the
// cooperative attribute when the kernel's CTAs wait on one another.  If the driver
// refuses the combination, the launch is repeated without the programmatic attribute.
// The programmatic attribute is set only with SF_PDL=1 in the environment (read once).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, bool cooperative, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++na;
  if (cooperative) {
    attr[na].id = cudaLaunchAttributeCooperative;
    attr[na].val.cooperative = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e == cudaErrorInvalidValue || e == cudaErrorNotSupported) {
    (void)cudaGetLastError();
    cfg.attrs = attr + 1;
    cfg.numAttrs = na - 1;
    e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  }
  return e;
}

// number of kernels this library has launched (all threads, all devices)
void count_launch(int n = 1);
// launch status of the kernel just launched; counts it when it launched
inline cudaError_t launched(int n = 1) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) count_launch(n);
  return e;
}

struct GateRowsParams {
  const void* hp;          // combine input (nullptr: gate on `hidden` as is)
  const void* ffn;         // [BN+1, D]
  const int64_t* src;      // previous layer's src (combine)
  void* hidden;            // [BN, D] read, or written by the combine
  const int64_t* par_idx;  // [B1]
  float* rstd;             // [BN] or nullptr
  int8_t* rec;             // [BN] (nullptr: combine + rstd only)
  int64_t* f;              // [BN]
  float delta, eps;
  int B1, N, D;
  int* err;
};

struct CompactParams {
  const int8_t* rec;
  const int64_t* f;
  int64_t* rows;           // [bucket]
  int32_t* count;          // [1]
  int64_t* seg;            // [BN]
  int32_t* segcnt;         // [B1]
  int64_t* src;            // [BN]
  const void* hidden;      // [BN, D] gate input (for xn)
  const float* rstd;       // [BN]
  const void* ln_w;        // [D]
  void* xn;                // [bucket, D] or nullptr
  int32_t* frows;          // [BN] folded rows in ascending order, or nullptr
  int B1, N, D, bucket;
  int* err;
};

struct RmsRowsParams {
  const void* x;           // [n_src, D]
  const int64_t* rows;     // gather index or nullptr
  const int32_t* count;    // device row count or nullptr
  int n;                   // rows to produce (upper bound)
  int64_t n_src;           // rows in x
  const void* w;           // [D]
  void* out;               // [n, D]
  float* rstd;             // [n] or nullptr
  int D;
  float eps;
  int* err;
};

struct GateCompactParams {
  const void* hp;          // previous layer's o_proj output (nullptr at layer 0)
  const void* ffn;         // [BN+1, D] previous layer's FFN rows
  const int64_t* src_prev; // previous layer's src (read before the grid barrier)
  void* hidden;            // [BN, D] read (layer 0) or written by the combine
  const int64_t* par_idx;  // [B1]
  const void* ln_w;        // [D] input RMSNorm weight
  int8_t* rec;             // [BN]
  int64_t* f;              // [BN]
  int64_t* rows;           // [bucket]
  int32_t* count;          // [1]
  int64_t* seg;            // [BN]
  int32_t* segcnt;         // [B1]
  int64_t* src;            // [BN] (written after the barrier; may alias src_prev)
  void* xn;                // [bucket, D]
  float* red;              // [BN][S][4] partial sums
  unsigned* bar;           // grid barrier counter (zero at the start of the forward)
  unsigned bar_target;     // counter value to wait for (cumulative over layers)
  float delta, eps;
  int B1, N, D, bucket;
  int S, slice;            // set by the launcher
  int* err;
};
int gate_compact_slices(int N, int D);
cudaError_t launch_parent_map(const int64_t* ids, int B1, int N, int64_t* par_idx,
                              cudaStream_t st);
cudaError_t launch_gate_compact(int dtype, const GateCompactParams& p, cudaStream_t st);

cudaError_t launch_gate_rows(int dtype, const GateRowsParams& p, cudaStream_t st);
cudaError_t launch_compact(int dtype, const CompactParams& p, cudaStream_t st);
cudaError_t launch_src_resolve(const int64_t* f, int64_t* src, int B1, int N, int* err,
                               cudaStream_t st);
cudaError_t launch_rmsnorm_rows(int dtype, const RmsRowsParams& p, cudaStream_t st);
cudaError_t launch_combine(int dtype, const void* hp, const void* ffn, const int64_t* src,
                           void* hidden, int B1, int N, int D, int* err, cudaStream_t st);

// ------------------------------------------------------------------ GEMM + epilogues
// out-features f in [0, n_out), activation rows j in [0, rows): acc[j][f] =
// sum_k X[j][k] * W[f][k]; the epilogue turns acc into the layer output.
enum EpiKind : int {
  EPI_RAW = 0,       // ws fp32 [rows][n_out] (tests)
  EPI_QKV = 1,       // + bias, RoPE on q/k, q scale, scatter to q_buf / kv_buf at rows[j]
  EPI_RESID = 2,     // out[j][f] = T(resid[j][f] + T(acc))
  EPI_SWIGLU = 3,    // W = [Wg; Wu] (n_out = 2I): act[j][f] = T(T(silu(T(g))) * T(u))
  EPI_SCATTER = 4,   // out[rows[j]][f] = T(acc)
  EPI_LOGITS = 5,    // logits[b][n'][f] with the Fast-dLLM shift when shift != 0
};

struct EpiParams {
  int kind;
  void* out;               // q_buf / hp / act / ffn_buf / logits / raw fp32
  void* out2;              // kv_buf
  const void* resid;       // EPI_RESID
  const void* bias;        // EPI_QKV (nullable)
  const void* cos;         // [N, hd]
  const void* sin;
  const float* q_scale;    // [N] nullable
  const int64_t* rows;     // row index map (QKV / SCATTER)
  int ld_out;              // leading dimension of `out` (elements)
  int q_dim, kv_dim, hd, N;
  int inter;               // SWIGLU: I
  int shift;               // LOGITS
  void* q_comp;            // QKV: optional query copy [Hkv][q_comp_rows][hd], row slot*G + g
  int q_comp_rows;         //      (the A operand layout of the tensor-core attention)
};

// Weights of a GEMM to pull into L2 ahead of it: the first npf k-blocks of every (unit,
// tile) of its plan, in the order its producer reads them (tile layout only).
struct WPrefetch {
  const void* w;           // nullptr: nothing to prefetch
  int n_tiles, sub, splits, kb_total, kb_per_split, n_units, npf;
};

struct GemmArgs {
  int dtype;
  const void* X;           // [rows_cap, K] activations (row-major)
  const void* W;           // [n_out, K] weights (row-major); SWIGLU: gate half
  const void* W2;          // SWIGLU: up half [I, K]
  int n_out, K;
  int rows_cap;            // static bound on rows (allocation of X)
  const int32_t* count;    // device row count (nullptr: rows_cap rows)
  EpiParams epi;
  void* ws;
  size_t ws_bytes;
  int* err;
  int w_tiled;             // W (and W2) already in the tile layout of pack_weight_tiles
  WPrefetch next_pf;       // optional: the next GEMM's weights to pull into L2
};
WPrefetch gemm_prefetch_plan(const GemmArgs& next);

// RMSNorm of the activation rows of a chain's first GEMM, done inside the chain launch:
// out[i] = T(w * T(x[rows[i]] * rstd)) for i < min(*count, n) (bf16, D <= 8192)
struct PreNormArgs {
  const void* x;
  const int64_t* rows;
  const int32_t* count;
  const void* w;
  void* out;
  int n;
  int64_t n_src;
  int D;
  float eps;
  // optional: the recompute flag per source row (rows[] lists the flagged ones).  With it,
  // when x is the output of a split-K residual GEMM (EPI_RESID, all rows) that precedes
  // the norm in the chain, that GEMM leaves its split reduction to the norm: flagged rows
  // are reduced, stored and normalised in one pass, the others stored after the norm.
  const int8_t* rec;
};
// Up to three bf16 GEMMs in one persistent launch, each reading the previous one's
// output (g[k].X == what g[k-1]'s epilogue writes, or what norms[k] writes from it);
// norms[k] (nullable array, nullable entries) is an RMSNorm writing g[k].X.
// dep: 2 * n device counters, zero before the launch.  Shares g[0].ws.
cudaError_t gemm_chain(const GemmArgs* g, int n, const PreNormArgs* const* norms, unsigned* dep,
                       cudaStream_t st);

// Weight tile layout for the tensor-core GEMM: [n_tiles][k_blocks][128 rows][64] so
// that the 16 KB a pipeline stage needs is one contiguous read.  mode 1 (SwiGLU) puts
// rows [64 gate | 64 up] of the same 64 output features in each 128-row block.
size_t weight_tiles_bytes(int n_out, int K, int mode, int inter);
cudaError_t pack_weight_tiles(const void* W, const void* W2, int n_out, int K, int mode,
                              int inter, void* dst, cudaStream_t st);

// GEMM scratch: kGemmCounterBytes of split-K tile counters at offset 0 (kept zero between
// launches; nothing else ever lands there), then partial sums / the SIMT raw result.
constexpr size_t kGemmCounterBytes = 16384;
size_t gemm_ws_need(int dtype, int rows_cap, int n_out, int K, int kind, int inter);
size_t gemm_tc_ws_need(int rows_cap, int n_out, int K, int kind, int inter);
cudaError_t gemm_tc(const GemmArgs& a, cudaStream_t st);
cudaError_t gemm_simt_bf16(const GemmArgs& a, cudaStream_t st);
cudaError_t gemm(const GemmArgs& a, cudaStream_t st);
int gemm_path_is_tc(int dtype);

// ------------------------------------------------------------------ attention
struct AttnParams {
  const void* q_buf;       // [BN+1, H*hd]
  const void* pk;          // [Hkv, .., hd] prefix keys (head stride kv_head_stride)
  const void* pv;
  int64_t kv_head_stride;
  const void* kv_buf;      // [BN+1, 2*Hkv*hd]
  const int64_t* src;      // [BN]
  const int64_t* rows;     // [bucket]
  const int32_t* count;
  const int8_t* rec;       // [BN] recompute flags (launch_attention_rows: slot of a row)
  void* O;                 // [BN, H*hd]
  float* M;                // [BN, H]
  float* Z;
  int P, N, bucket, H, Hkv, hd, B1;
  float scale;
  int* err;
  // tensor-core path (bf16): compact queries written by the QKV epilogue (nullptr: the
  // launcher packs them from q_buf into the scratch) and fp32 split-KV partials
  const void* q_comp;
  void* scratch;
  size_t scratch_bytes;
  // prefix length read on the device when the kernel runs (decode loops: one captured
  // launch serves every prefix length); nullptr = P.  P then bounds it and sizes the grid.
  const int32_t* P_dev;
  // batched prefill (block-causal): the B1 branches are consecutive blocks of N tokens
  // whose keys and values are already in the cache after the prefix; P (and *P_dev)
  // count the prefix before them and row (b, n) attends to the cache's first
  // P' + b * N keys plus its own block.  prefill_rows = B1 * N (0 = off); the launcher
  // passes P + prefill_rows as the key bound.
  int prefill_rows;
};

// The prefix length a kernel attends to: *P_dev when given, clamped to the bound P the
// launch was sized for (a larger value flags SF_DEV_ERR_INDEX and is clamped).
__device__ __forceinline__ int prefix_len(const int32_t* P_dev, int P, int* err) {
  if (P_dev == nullptr) return P;
  const int v = *P_dev;
  if (v < 0 || v > P) {
    flag_error(err, SF_DEV_ERR_INDEX);
    return v < 0 ? 0 : P;
  }
  return v;
}

// keys of the cache an attention launch covers: P' = the prefix before any prefill rows,
// keys = P' + prefill_rows (a prefill block b sees P' + b * N of them)
struct KeyRange {
  int base, keys;
};
__device__ __forceinline__ KeyRange attn_keys(const int32_t* P_dev, int P_bound, int prefill_rows,
                                              int* err) {
  const int base = prefix_len(P_dev, P_bound - prefill_rows, err);
  return {base, base + prefill_rows};
}
// rows_total > 0: room for partials indexed by flat block row (launch_attention_rows)
size_t attn_scratch_bytes(int dtype, int bucket, int H, int Hkv, int hd, int P,
                          bool need_q_comp, int rows_total = 0);
// recomputed rows only (the flash-attention operator)
cudaError_t launch_attention(int dtype, const AttnParams& p, cudaStream_t st);
cudaError_t launch_attention_simt(int dtype, const AttnParams& p, cudaStream_t st);
// every row of the block, folded rows from their recomputing ancestor's query and prefix
// state (the fused forward's attention + chain correction in one pass)
cudaError_t launch_attention_rows(int dtype, const AttnParams& p, cudaStream_t st);
cudaError_t launch_attention_rows_partials(int dtype, const AttnParams& p, const float* part_O,
                                           const float* part_ml, int splits, int q_rows,
                                           cudaStream_t st);
// the same on the tensor cores (mma.sync block of <= 32 keys): bf16, hd 64 / 128, N <= 32
bool attention_rows_mma_ok(int dtype, const AttnParams& p, int splits);
cudaError_t launch_attention_rows_mma(const AttnParams& p, const float* part_O,
                                      const float* part_ml, int splits, int part_rows,
                                      cudaStream_t st);
// the same rows pass with S and O on tcgen05 (TMEM accumulators): bf16, head_dim 128,
// N <= 32 block keys, <= 16 prefix splits
bool attention_rows_tc_ok(int dtype, const AttnParams& p, int splits);
cudaError_t launch_attention_rows_tc(const AttnParams& p, const float* part_O,
                                     const float* part_ml, int splits, int part_rows,
                                     cudaStream_t st);

struct MergeParams {
  const void* q_buf;
  const void* kv_buf;
  const int64_t* src;
  const int64_t* par_idx;
  const int8_t* rec;
  const int64_t* seg;
  const int32_t* segcnt;
  const int32_t* frows;    // folded rows listed by the compaction, or nullptr (scan all)
  const int32_t* count;    // recomputed rows (BN - count rows are folded), with frows
  void* O;
  float* M;
  float* Z;
  int B1, N, H, Hkv, hd;
  float scale;
  int* err;
};
cudaError_t launch_merge(int dtype, const MergeParams& p, cudaStream_t st);

// ------------------------------------------------------------------ tensor parallel
const char* tp_error_string(int r);
int tp_unique_id(void* out, int bytes);
int tp_comm_init(const void* id, int nranks, int rank, void** comm);
int tp_comm_destroy(void* comm);
int tp_allreduce_f32(void* comm, float* buf, size_t n, cudaStream_t st);

// Tensor parallelism over peer memory (tp.cu): every rank's exchange buffer, as mapped in
// this process (own one included), laid out as [flags: kMaxTp x 2 int32][epoch][pad to
// kTpHeader bytes][o_proj partials: part_elems fp32][down partials: part_elems fp32].
constexpr int kMaxTp = 8;
constexpr size_t kTpHeader = 512;
struct TpPeers {
  float* part[kMaxTp];       // each rank's partial regions (o_proj, then down)
  int* flags[kMaxTp];        // each rank's flag array: [rank q][kind] = last seq of q
  unsigned* epoch;           // this rank's forward counter
  int64_t part_elems;        // fp32 elements of one partial region
  int rank, size;
};
cudaError_t launch_tp_epoch(const TpPeers& t, cudaStream_t st);
cudaError_t launch_tp_reduce_resid(int dtype, const TpPeers& t, int layer, int L,
                                   const void* resid, void* out, int64_t n, int* err,
                                   cudaStream_t st);
cudaError_t launch_tp_reduce_scatter(int dtype, const TpPeers& t, int layer, int L,
                                     const int64_t* rows, const int32_t* count, int n, int D,
                                     int64_t n_out_rows, void* out, int* err, cudaStream_t st);
cudaError_t launch_resid_add(int dtype, const float* sum, const void* resid, void* out, int64_t n,
                             cudaStream_t st);
cudaError_t launch_scatter_rows(int dtype, const float* sum, const int64_t* rows,
                                const int32_t* count, int n, int D, int64_t n_out_rows, void* out,
                                int* err, cudaStream_t st);

// Block commit inside the forward: the first N rows of kv_buf (branch 0's keys and values)
// appended to the prefix cache at positions [P', P' + N), P' = prefix_len(P_dev, P).
cudaError_t launch_kv_commit(int dtype, const void* kv_buf, void* ck, void* cv, int64_t c_stride,
                             const int32_t* P_dev, int P, int N, int Hkv, int hd, int* err,
                             cudaStream_t st);
cudaError_t launch_kv_append(int dtype, void* ck, void* cv, int64_t c_stride, const void* nk,
                             const void* nv, int64_t n_stride, int Hkv, int hd, int P, int n,
                             cudaStream_t st);

int draft_max_topk();
int draft_max_positions();
cudaError_t launch_draft_blocks(int dtype, const void* logits, int64_t row_stride, int n_pos,
                                int V, int K, int conf_fp32, const uint8_t* mask,
                                const int32_t* pairs, const int32_t* node_off, int n_nodes,
                                const int64_t* block, int block_len, int pos_offset,
                                int64_t* drafts, int32_t* valid, float* conf, int64_t* top,
                                cudaStream_t st);

cudaError_t launch_sample_top_p(int dtype, const void* logits, int64_t rows, int V,
                                int64_t row_stride, float top_p, int64_t* tokens, void* conf,
                                cudaStream_t st);

}  // namespace sf
