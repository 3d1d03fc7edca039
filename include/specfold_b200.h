/*
 * specfold_b200.h -- C ABI of the B200 (sm_100a) folded multi-branch verify forward.
 *
 * One entry point per launch of the reference's fused path
 * (specfold/generate/fastdllm_v2_folded.py:237-370, nld_folded.py:255-394 and the
 * Triton kernels in specfold/generate/triton_kernels.py), plus the whole layer loop
 * as a single call.  Plain pointers and sizes only; every pointer is device memory
 * unless documented otherwise.  Buffers are owned by the caller; the library
 * allocates no device memory.  `stream` is a cudaStream_t passed as void*.
 *
 * Element types: `dtype` is SF_DTYPE_F32 or SF_DTYPE_BF16 and applies to every
 * hidden-state, weight and Q/K/V/O table argument; softmax state (M, Z), rstd and
 * RoPE q-scales are always float32, indices int64, counters int32.
 *
 * Layouts (row-major unless stated; BN = B1*N flat rows, row r = b*N + n):
 *   Hf        [BN, D]                 layer input hidden states
 *   q_buf     [BN+1, H*hd]            RoPE'd queries, row BN is the trash row
 *   kv_buf    [BN+1, 2*Hkv*hd]        RoPE'd keys (heads 0..Hkv-1) then values
 *   prefix_k/v [Hkv, >=P, hd] each    head h at offset h*kv_head_stride elements
 *   O_tab     [BN, H*hd]; M_tab, Z_tab [BN, H] float32
 *
 * Every function returns 0 (SF_OK) or a status code; sf_last_error() describes the
 * last failure of the calling thread.  Launch errors are reported, kernel faults
 * surface at the caller's next synchronisation.  Kernels that wait on barriers give
 * up after a bounded time and set bits in `err` (a device int32, see SF_DEV_*).
 */
#ifndef SPECFOLD_B200_H
#define SPECFOLD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  SF_OK = 0,
  SF_ERR_ARG = 1,          /* bad shape / null pointer / unsupported combination */
  SF_ERR_CUDA = 2,         /* CUDA runtime error on launch */
  SF_ERR_UNSUPPORTED = 3,  /* device is not sm_100 or feature missing */
  SF_ERR_WORKSPACE = 4     /* workspace too small */
};
enum { SF_DTYPE_F32 = 0, SF_DTYPE_BF16 = 1 };
/* bits of the device error word */
enum { SF_DEV_TIMEOUT = 1, SF_DEV_INDEX = 2, SF_DEV_DEPTH = 4, SF_DEV_TMEM = 8 };

const char* sf_last_error(void);
int sf_abi_version(void);
/* 0 when the current device is an sm_100 part the kernels run on */
int sf_check_device(void);

/* ------------------------------------------------------------------ fold gate ----
 * Replaces residual_delta_gate_kernel (triton_kernels.py:199-239, launched at
 * fastdllm_v2_folded.py:306-309) together with src_resolve_kernel
 * (triton_kernels.py:18-26, launched at :310).  Same arguments and outputs, with
 * the recompute test written the way the PyTorch reference decides it
 * (fastdllm_v2_folded.py:139-141): ||x - x_par|| > delta * ||x_par|| with the
 * difference, both norms and the threshold rounded to the model dtype.
 * Compaction is deterministic: rows[] lists the recomputed flat rows in ascending
 * order (branch-major, position-ascending), seg[b*N + i] the i-th recomputed row of
 * branch b.  Also writes xn[slot] = RMSNorm(Hf[rows[slot]]) * ln_w in the model dtype
 * (the A operand of the QKV projection) when xn != NULL.
 * f and src hold branch indices; count[0] and segcnt[0..B1) must be zero on entry
 * (they are accumulated, as in the reference).                                     */
int sf_residual_delta_gate(int dtype, const void* Hf, const int64_t* par_idx, float* rstd,
                           int64_t* f, int8_t* rec, int64_t* rows, int32_t* count,
                           int64_t* seg, int32_t* segcnt, int64_t* src, void* xn,
                           const void* ln_w, float delta, int B1, int N, int D, int bucket,
                           float eps, int* err, void* stream);

/* src_resolve_kernel (triton_kernels.py:18-26): src[b,n] = nearest recomputing
 * ancestor branch, following f (branch indices) until a fixed point.               */
int sf_src_resolve(const int64_t* f, int64_t* src, int B1, int N, int* err, void* stream);

/* ------------------------------------------------------------- projections -------
 * Workspace for every GEMM-based entry point below: sf_gemm_workspace_bytes(...)
 * bytes of device memory (split-K partial sums and tile counters; tile counters must
 * be zero on the first use and are left zero by every call).                        */
size_t sf_workspace_bytes(int BN, int D, int H, int Hkv, int hd, int I, int V);
/* zero the tile counters inside a fresh workspace.  A call that set a device error
 * bit (SF_DEV_TIMEOUT in particular) may leave counters nonzero: run sf_workspace_init
 * on the workspace again before reusing it after any device error. */
int sf_workspace_init(void* ws, size_t ws_bytes, void* stream);

/* fused_ln_qkv_rope_scatter_kernel (triton_kernels.py:29-87, launched at
 * fastdllm_v2_folded.py:313-319): Q/K/V of the recomputed rows, + bias, RoPE on q
 * and k (rotate-half, cos/sin [N, hd] in the model dtype), optional per-position
 * q scale (llama-4, nld_folded.py:175-176; NULL = 1), scattered to q_buf / kv_buf
 * at the flat row.  xn is the normalised compacted input written by the gate;
 * w_qkv = [Wq; Wk; Wv] ((H+2Hkv)*hd x D), b_qkv the matching bias (NULL = none).   */
int sf_fused_ln_qkv_rope_scatter(int dtype, const void* xn, const void* w_qkv,
                                 const void* b_qkv, const int64_t* rows, const int32_t* count,
                                 const void* cos, const void* sin, const float* q_scale,
                                 void* q_buf, void* kv_buf, int D, int N, int bucket, int H,
                                 int Hkv, int hd, void* ws, size_t ws_bytes, int* err,
                                 void* stream);

/* specfold_flash_attn_gqa_kernel (triton_kernels.py:301-361, launched at
 * fastdllm_v2_folded.py:329-333): attention of each recomputed row over the prefix
 * cache (P keys) and the N in-block keys kv_buf[src[b*N+j]*N + j]; writes O (model
 * dtype, normalised), M (row max) and Z (sum of exp) at the flat row.  P may be 0.
 * Takes B1 in addition to the reference's arguments (bounds check of src) and, for
 * bf16 with P > 0 (tensor-core prefix pass, split along the keys), a workspace of
 * sf_attn_workspace_bytes(...) bytes; kv_head_stride must be a multiple of hd.      */
int sf_flash_attn_gqa(int dtype, const void* q_buf, const void* prefix_k, const void* prefix_v,
                      int64_t kv_head_stride, const void* kv_buf, const int64_t* src,
                      const int64_t* rows, const int32_t* count, void* O_tab, float* M_tab,
                      float* Z_tab, int P, int N, float scale, int bucket, int B1, int H,
                      int Hkv, int hd, void* ws, size_t ws_bytes, int* err, void* stream);
size_t sf_attn_workspace_bytes(int dtype, int bucket, int H, int Hkv, int hd, int P);

/* specfold_chain_correction_gqa_kernel (triton_kernels.py:364-429, launched at
 * fastdllm_v2_folded.py:334-338): for every folded row (rec == 0) start from the
 * source row's (m, Z, O) and apply the exact update for every key that changed along
 * the branch chain up to the source; writes O, M, Z at the folded row.              */
int sf_chain_correction_gqa(int dtype, const void* q_buf, const void* kv_buf,
                            const int64_t* src, const int64_t* par_idx, const int8_t* rec,
                            const int64_t* seg, const int32_t* segcnt, void* O_tab,
                            float* M_tab, float* Z_tab, int B1, int N, float scale, int H,
                            int Hkv, int hd, int* err, void* stream);

/* torch.addmm(Hf, O_tab, Wo^T) at fastdllm_v2_folded.py:351 (all BN rows):
 * hp = Hf + O_tab @ Wo^T, the matmul rounded to the model dtype before the add.     */
int sf_o_proj_residual(int dtype, const void* Hf, const void* O_tab, const void* w_o,
                       void* hp, int BN, int D, int q_dim, void* ws, size_t ws_bytes,
                       int* err, void* stream);

/* fused_ffn_scatter (triton_kernels.py:176-194, called at fastdllm_v2_folded.py:354-359
 * with store_ffn_only=True): for each recomputed row rows[slot], slot < count:
 * ffn_buf[rows[slot]] = down(silu(gate(z)) * up(z)), z = RMSNorm(hp_all[rows[slot]]) *
 * ln_w.  Reads hp_all directly (the reference gathers hp_all[rows] first).  act_buf
 * [bucket, I] and xn_buf [bucket, D] (model dtype) and rstd_buf [bucket] are scratch. */
int sf_fused_ffn_scatter(int dtype, const void* hp_all, const void* ln_w, const void* w_gate,
                         const void* w_up, const void* w_down, const int64_t* rows,
                         const int32_t* count, void* ffn_buf, int bucket, void* act_buf,
                         void* xn_buf, float* rstd_buf, float eps, int D, int I, void* ws,
                         size_t ws_bytes, int* err, void* stream);

/* sf_fused_ffn_scatter without caller-provided scratch.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory (code inside a
 * stream capture, runtimes without an allocator, hosts whose memory pool belongs to
 * someone else).  Same inputs and outputs as sf_fused_ffn_scatter minus act_buf,
 * xn_buf, rstd_buf and the workspace; the scratch is a fixed 32 MiB __device__ array
 * inside the library, held on every GPU where the library's module is loaded until the
 * process exits.  It calls no cudaMalloc/cudaFree.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress, that device current): make it before any stream capture.
 *    The address is kept for the life of the process; after cudaDeviceReset on that
 *    device it is stale, so do not call this entry point again after a reset.
 *  - Shapes needing more than 32 MiB of scratch return SF_ERR_ARG.
 *  - All calls share the array and it keeps the last call's contents (the split-K
 *    counters are cleared at each call); calls that overlap on the GPU race and must be
 *    serialised by the caller.                                                       */
int sf_fused_ffn_scatter_static(int dtype, const void* hp_all, const void* ln_w,
                                const void* w_gate, const void* w_up, const void* w_down,
                                const int64_t* rows, const int32_t* count, void* ffn_buf,
                                int bucket, float eps, int D, int I, int* err, void* stream);

/* hidden = hp_all + ffn_buf[src*N + n] (fastdllm_v2_folded.py:361).                 */
int sf_combine(int dtype, const void* hp_all, const void* ffn_buf, const int64_t* src,
               void* hidden, int B1, int N, int D, int* err, void* stream);

/* final norm + lm_head (+ the Fast-dLLM logit shift when shift != 0)
 * (fastdllm_v2_folded.py:365-366, fastdllm_v2_generation.py:121-126;
 * nld_folded.py:389-390 without shift).  logits [B1, N, V]; xn_buf [BN, D] scratch. */
int sf_final_norm_lm_head(int dtype, const void* hidden, const void* norm_w,
                          const void* lm_w, void* logits, void* xn_buf, int B1, int N, int D,
                          int V, float eps, int shift, void* ws, size_t ws_bytes, int* err,
                          void* stream);

/* Block KV commit: append n_new committed positions to a preallocated cache,
 * cache_{k,v}[h, P + t, :] = new_{k,v}[h, t, :], t < n_new.  Replaces the torch.cat
 * inside DynamicCache.update (modeling_ministral.py:154-158 via nld_generation.py:
 * 279-289; the Fast-dLLM remote code at fastdllm_v2_generation.py:560-575).
 * cache head stride = cache_head_stride elements, new head stride = new_head_stride. */
int sf_kv_append(int dtype, void* cache_k, void* cache_v, int64_t cache_head_stride,
                 const void* new_k, const void* new_v, int64_t new_head_stride, int Hkv,
                 int hd, int P, int n_new, void* stream);

/* Greedy top-p sampling of logits rows (temperature 0): tokens[r] = the argmax token,
 * conf[r] = its probability after top-p filtering, in the logits' dtype -- what the
 * decode loops take from FastDLLMModelExecutor.sample_with_top_p
 * (fastdllm_model_executor.py:130-155; used at fastdllm_v2_generation.py:346-351) --
 * computed per row by a radix select of the nucleus boundary instead of a vocabulary
 * sort.  logits [rows][row_stride] (row_stride >= V elements), tokens int64 [rows],
 * conf [rows]; 0 < top_p. */
int sf_sample_top_p_greedy(int dtype, const void* logits, int64_t rows, int V,
                           int64_t row_stride, float top_p, int64_t* tokens, void* conf,
                           void* stream);

/* Draft blocks from the calibration graph (FastDLLMV2SpeculativeGeneration.
 * get_draft_blocks, fastdllm_v2_generation.py:387-474; NLDDiffusionGeneration.
 * get_draft_blocks, nld_generation.py:108-151): confidence of each of the n_pos
 * positions = its maximal softmax probability (conf_fp32 = 1: fp32, as NLD; 0: in the
 * logits' dtype, as Fast-dLLM); for node k with pairs[node_off[k]..node_off[k+1]) of
 * (pos_rank, vocab_rank), drafts[k] = block with block[pos_offset + p] = the
 * vocab_rank-th most likely token of p, p = the pos_rank-th most confident masked
 * position; valid[k] = 0 when the node needs more masked positions than there are
 * (the reference skips it).  Ties rank the larger value, then the smaller index first.
 * logits [n_pos][row_stride] (>= V), mask uint8 [n_pos], pairs int32 [n_pairs][2],
 * node_off int32 [n_nodes + 1], block int64 [block_len], drafts int64
 * [n_nodes][block_len], valid int32 [n_nodes], all on the device; K = largest
 * vocab_rank + 1 (<= 16), n_pos <= 1024; ws: sf_draft_workspace_bytes(n_pos, K) bytes. */
size_t sf_draft_workspace_bytes(int n_pos, int K);
int sf_draft_blocks(int dtype, const void* logits, int64_t row_stride, int n_pos, int V, int K,
                    int conf_fp32, const uint8_t* mask, const int32_t* pairs,
                    const int32_t* node_off, int n_nodes, const int64_t* block, int block_len,
                    int pos_offset, int64_t* drafts, int32_t* valid, void* ws, size_t ws_bytes,
                    void* stream);

/* ------------------------------------------------------------ whole forward -------
 * The full per-layer loop of SpecFoldTritonFastDLLMV2Generation._batched_block_forward
 * (fastdllm_v2_folded.py:296-366) in one call: gate -> QKV -> attention -> chain
 * correction -> o_proj -> FFN -> combine for every layer, then final norm + lm_head.
 * Host-side work that stays in the caller: the parent map (:263-265), embedding
 * lookup and RoPE tables (:267-271), and the fold counters / overflow check (:363-369). */
typedef struct sf_layer {
  const void* w_qkv;      /* [(H+2Hkv)*hd, D] */
  const void* b_qkv;      /* [(H+2Hkv)*hd] or NULL */
  const void* ln1_w;      /* input_layernorm.weight [D] */
  const void* w_o;        /* o_proj.weight [D, H*hd] */
  const void* ln2_w;      /* post_attention_layernorm.weight [D] */
  const void* w_gate;     /* [I, D] */
  const void* w_up;       /* [I, D] */
  const void* w_down;     /* [D, I] */
  const void* prefix_k;   /* [Hkv, >=P, hd] or NULL when P == 0 */
  const void* prefix_v;
} sf_layer;

typedef struct sf_verify_args {
  int dtype;
  int B1, N, D, H, Hkv, hd, I, V, L;
  int P;                       /* prefix length (0 = no prefix cache) */
  int64_t kv_head_stride;      /* elements between prefix heads */
  int bucket;                  /* compaction capacity (<= B1*N) */
  float delta, eps, scale;     /* recompute threshold, RMSNorm eps, attention scale */
  int shift_logits;            /* 1 for Fast-dLLM, 0 for NLD */
  int weights_tiled;           /* bf16 only: w_qkv, w_o, w_gate (gate+up), w_down and lm_w
                                  are in the tile layout of sf_pack_weight_tiles (w_up is
                                  then unused) */
  const sf_layer* layers;      /* HOST array of L layers */
  const void* final_norm_w;    /* [D] */
  const void* lm_w;            /* [V, D] */
  const int64_t* par_idx;      /* [B1] parent branch (0 for main) */
  const void* hidden_in;       /* [B1*N, D] embeddings */
  const void* cos;             /* [N, hd] */
  const void* sin;             /* [N, hd] */
  const float* q_scale;        /* [N] or NULL */
  void* logits;                /* [B1, N, V] */
  int32_t* count_slab;         /* [L] recomputed rows per layer (zeroed by the call) */
  int32_t* segcnt_slab;        /* [L*B1] recomputed rows per layer and branch (zeroed by
                                  the call) */
  int8_t* rec_slab;            /* [L*B1*N] fold masks per layer, or NULL */
  void* ws;                    /* sf_verify_workspace_bytes(...) bytes */
  size_t ws_bytes;
  int* err;                    /* device error word (SF_DEV_*), zeroed by the call */
  void* stream;
  /* tensor parallelism (the 14B configuration: attention heads and the intermediate
   * dimension sharded over tp_size ranks).  tp_size <= 1: off.  Otherwise
   * H, Hkv and I are this rank's shard, the weights and prefix K/V are its shards, and
   * tp_comm comes from sf_tp_comm_init; o_proj and down are all-reduced in fp32. */
  void* tp_comm;
  int tp_size;
  /* Decode-loop support (both optional; zero / NULL = off).
   * P_dev: device int32 holding the prefix length actually used, read when the
   *   launches run (0 <= *P_dev <= P; a larger value sets SF_DEV_INDEX and is clamped).
   *   P then only bounds it: it sizes the grids and the workspace, and the prefix heads
   *   must hold kv_head_stride >= P * hd elements.  The launches no longer depend on the
   *   prefix length, so the captured graph of one argument set serves every block of a
   *   decode.  cos / sin (and q_scale) must hold the rows of positions [*P_dev, +N).
   * commit: the block commit forward (B1 == 1): every layer also writes its block rows'
   *   keys (after RoPE) and values into prefix_k / prefix_v at positions [P', P' + N),
   *   P' = *P_dev or P -- the append of the reference's cache update
   *   (fastdllm_v2_generation.py:562-568 -> DynamicCache.update); the prefix tensors are
   *   then written, and kv_head_stride must be >= (P + N) * hd.  A commit forward may
   *   pass logits == NULL: the last layer's combine, the final norm and the LM head are
   *   then skipped (the prompt blocks of a prefill, whose logits are not read). */
  const int32_t* P_dev;
  int commit;
  /* tensor parallelism over peer memory (sf_tp_peers_init) instead of tp_comm: the
   * o_proj and down partial sums stay in each rank's exchange buffer and the kernels
   * that consume them read every rank's partial over NVLink (no NCCL on the layer path). */
  void* tp_peers;
  /* prefill != 0 (with commit, a negative delta and shift_logits 0): the B1 "branches"
   * are B1 consecutive blocks of N prompt tokens at positions [P', P' + B1 * N) -- one
   * block-causal forward instead of B1 commit forwards.  Every layer appends all B1 * N
   * rows' keys and values to the cache before its attention; row (b, n) attends to the
   * cache's first P' + b * N keys and to its own block bidirectionally.  cos / sin (and
   * q_scale) hold B1 * N rows; logits, when not NULL, are [1, N, V] of the last block;
   * kv_head_stride must be >= (P + B1 * N) * hd. */
  int prefill;
} sf_verify_args;

/* Tensor-parallel communicator (NCCL, loaded at run time).  Rank 0 calls
 * sf_tp_unique_id (128 bytes), the host broadcasts it, every rank calls
 * sf_tp_comm_init on its own device.  Release captured graphs (sf_release_graphs)
 * before sf_tp_comm_destroy. */
int sf_tp_unique_id(void* id_out, int bytes);
int sf_tp_comm_init(const void* id, int nranks, int rank, void** comm_out);
int sf_tp_comm_destroy(void* comm);
/* Tensor parallelism over peer memory.  Each rank allocates an exchange buffer of
 * sf_tp_exchange_bytes(B1*N, D) bytes of device memory, zero-filled, maps every other
 * rank's buffer into its address space (CUDA IPC; NVLink peers) and passes the table of
 * device pointers -- xbufs[q] = rank q's buffer as seen from this process, its own at
 * xbufs[rank], a HOST array of `size` pointers -- to sf_tp_peers_init; the returned
 * handle goes into sf_verify_args.tp_peers.  Every rank must run the same sequence of
 * forwards; a missing peer makes the waiting kernels give up after a bounded time with
 * SF_DEV_TIMEOUT.  (No counterpart in the reference, which is single-GPU; this replaces
 * the NCCL all-reduce of sf_tp_comm_init for the two reductions per layer.) */
size_t sf_tp_exchange_bytes(int BN, int D);
int sf_tp_peers_init(int rank, int size, void* const* xbufs, int BN, int D, void** peers_out);
int sf_tp_peers_destroy(void* peers);
/* CUDA IPC of the exchange buffers (64-byte handles): sf_tp_ipc_export gives the handle
 * of the allocation holding `ptr` and ptr's offset in it; sf_tp_ipc_open maps a peer's
 * allocation into the CURRENT device's context (peer access enabled for it), the
 * buffer is then base + offset; sf_tp_ipc_close unmaps it. */
int sf_tp_ipc_export(const void* ptr, void* handle_out, int bytes, size_t* offset_out);
int sf_tp_ipc_open(const void* handle, int bytes, void** base_out);
int sf_tp_ipc_close(void* base);
/* Destroys every CUDA graph the forward captured (all devices). */
int sf_release_graphs(void);

/* The parent map of a verify block on the device: par_idx[i] = the first branch whose
 * set of positions differing from the main branch (row 0 of ids) is a subset of
 * branch i's with one element fewer, else 0 (SpecFold*Generation._build_parent_map,
 * fastdllm_v2_folded.py:55-75; the reference computes it on the host after a sync).
 * ids [B1, N] int64 on the device. */
int sf_parent_map(const int64_t* ids, int B1, int N, int64_t* par_idx, void* stream);

/* ------------------------------------------------------------------ measurement ----
 * Kernels launched by this library so far (all host threads).                       */
long long sf_launch_count(void);
/* CUDA-event timing of sf_folded_verify_forward's launches, per kernel kind (host-side
 * events only).  sf_profile_begin(capacity) arms up to `capacity` timed launches on the
 * calling thread; sf_profile_end() waits for them and sums per kind;
 * sf_profile_kind(k, &ms, &calls) reads kind k (0 <= k < sf_profile_kinds()).       */
int sf_profile_begin(int capacity);
int sf_profile_end(void);
int sf_profile_kinds(void);
const char* sf_profile_name(int kind);
int sf_profile_kind(int kind, double* total_ms, int* calls);

/* Weight tile layout for the tensor-core projections (bf16): [n_tiles][K/64][128][64],
 * i.e. every 128-row x 64-column block of W stored contiguously, so one pipeline stage
 * is one 16 KB read.  mode 0: W [n_out, K]; mode 1 (SwiGLU): each 128-row block holds
 * 64 rows of W (gate) then the same 64 rows of W2 (up), n_out = 2*inter.  Packing is a
 * one-time copy per model (the reference packs [Wq;Wk;Wv] and [Wg;Wu] likewise,
 * fastdllm_v2_folded.py:77-87).                                                      */
size_t sf_weight_tiles_bytes(int n_out, int K, int mode, int inter);
int sf_pack_weight_tiles(const void* W, const void* W2, int n_out, int K, int mode, int inter,
                         void* dst, void* stream);

size_t sf_verify_workspace_bytes(int dtype, int B1, int N, int D, int H, int Hkv, int hd, int I,
                                 int V, int P);
/* Runs the forward on args->stream.  The launches of one argument set (every field but
 * `stream`, and the contents of the layer table) are captured into a CUDA graph on the
 * second call with that set and replayed afterwards: keep buffers at fixed addresses
 * across steps to benefit; the data behind the pointers may change freely.  SF_GRAPH=0
 * in the environment launches directly every time. */
int sf_folded_verify_forward(const sf_verify_args* args);

#ifdef __cplusplus
}
#endif
#endif /* SPECFOLD_B200_H */
