// Draft construction from the calibration graph on the GPU.
//
// The decode loops build the next step's draft blocks from the main block's logits
// (FastDLLMV2SpeculativeGeneration.get_draft_blocks, fastdllm_v2_generation.py:387-474;
// NLDDiffusionGeneration.get_draft_blocks, nld_generation.py:108-151): every masked
// position's confidence is its maximal softmax probability; for each graph node with
// pairs (pos_rank, vocab_rank), the pos_rank-th most confident masked position receives
// its vocab_rank-th most likely token, on a copy of the block; a node needing more
// masked positions than there are is skipped.  The reference runs a full-vocabulary
// topk per (node, pair) and syncs with the host per node.
//
// Here: one CTA per position computes the confidence and the top-K tokens (K = the
// largest vocab_rank + 1 over the graph), then one CTA ranks the masked positions and
// writes every node's draft.  Ties: a larger value first, then the smaller index (for
// positions and tokens alike).
#include <cstdint>

#include "sf_kernels.cuh"

namespace sf {

namespace {

constexpr int kDraftThreads = 512;
constexpr int kMaxTopK = 16;

// a thread's running top-K (value desc, index asc), kept sorted in registers
struct TopK {
  float v[kMaxTopK];
  int i[kMaxTopK];
};
__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  return a > b || (a == b && ia < ib);
}
__device__ __forceinline__ void topk_insert(TopK& t, int K, float v, int idx) {
  if (!better(v, idx, t.v[K - 1], t.i[K - 1])) return;
  int p = K - 1;
  while (p > 0 && better(v, idx, t.v[p - 1], t.i[p - 1])) {
    t.v[p] = t.v[p - 1];
    t.i[p] = t.i[p - 1];
    --p;
  }
  t.v[p] = v;
  t.i[p] = idx;
}

template <typename T>
__global__ void __launch_bounds__(kDraftThreads) draft_rows_kernel(
    const T* __restrict__ logits, int64_t row_stride, int V, int K, int conf_fp32, float* conf,
    int64_t* top) {
  __shared__ float red[kDraftThreads / 32];
  __shared__ float cand_v[kDraftThreads / 32][kMaxTopK];
  __shared__ int cand_i[kDraftThreads / 32][kMaxTopK];
  const T* x = logits + static_cast<int64_t>(blockIdx.x) * row_stride;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;

  TopK t;
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) { t.v[k] = -INFINITY; t.i[k] = INT32_MAX; }
  float mx = -INFINITY;
  for (int i = tid; i < V; i += kDraftThreads) {
    const float l = Elt<T>::to_f(x[i]);
    mx = fmaxf(mx, l);
    topk_insert(t, K, l, i);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[w] = mx;
  __syncthreads();
  float m = red[0];
  for (int j = 1; j < kDraftThreads / 32; ++j) m = fmaxf(m, red[j]);
  __syncthreads();
  float z = 0.f;
  for (int i = tid; i < V; i += kDraftThreads) z += expf(Elt<T>::to_f(x[i]) - m);
  for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  if (lane == 0) red[w] = z;

  // warp merge of the per-thread lists: K rounds of a warp arg-best over the heads
  int head = 0;
  for (int r = 0; r < K; ++r) {
    float v = head < K ? t.v[head] : -INFINITY;
    int ix = head < K ? t.i[head] : INT32_MAX;
    float bv = v;
    int bi = ix;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (ix == bi && head < K) ++head;          // the lane whose head won advances
    if (lane == 0) { cand_v[w][r] = bv; cand_i[w][r] = bi; }
  }
  __syncthreads();
  if (w == 0) {
    // block merge: the 16 warp lists, K rounds again (lane j reads list j)
    int h2 = 0;
    for (int r = 0; r < K; ++r) {
      const bool has = lane < kDraftThreads / 32 && h2 < K;
      float bv = has ? cand_v[lane][h2] : -INFINITY;
      int bi = has ? cand_i[lane][h2] : INT32_MAX;
      const int mine = bi;
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
      }
      if (has && mine == bi) ++h2;
      if (lane == 0) top[static_cast<int64_t>(blockIdx.x) * K + r] = bi;
    }
    if (lane == 0) {
      float Z = 0.f;
      for (int j = 0; j < kDraftThreads / 32; ++j) Z += red[j];
      const float c = __fdiv_rn(1.0f, Z);       // exp(m - m) / Z: the maximal probability
      conf[blockIdx.x] = conf_fp32 ? c : Elt<T>::rnd(c);
    }
  }
}

// ranks the masked positions, then writes each node's draft (pairs applied in order)
__global__ void __launch_bounds__(256) draft_assemble_kernel(
    const float* conf, const int64_t* top, int K, const uint8_t* mask, int n_pos,
    const int32_t* pairs, const int32_t* node_off, int n_nodes, const int64_t* block,
    int block_len, int pos_offset, int64_t* drafts, int32_t* valid) {
  __shared__ int ranked[1024];
  __shared__ int n_masked;
  const int tid = threadIdx.x;
  if (tid == 0) n_masked = 0;
  __syncthreads();
  for (int i = tid; i < n_pos; i += blockDim.x) {
    if (!mask[i]) continue;
    int r = 0;
    for (int j = 0; j < n_pos; ++j)
      if (mask[j] && (conf[j] > conf[i] || (conf[j] == conf[i] && j < i))) ++r;
    ranked[r] = i;
    atomicAdd(&n_masked, 1);
  }
  __syncthreads();
  for (int nd = 0; nd < n_nodes; ++nd) {
    int64_t* d = drafts + static_cast<int64_t>(nd) * block_len;
    for (int i = tid; i < block_len; i += blockDim.x) d[i] = block[i];
    __syncthreads();
    if (tid == 0) {
      int max_rank = -1;
      bool ranks_ok = node_off[nd + 1] > node_off[nd];
      for (int q = node_off[nd]; q < node_off[nd + 1]; ++q) {
        max_rank = max(max_rank, pairs[2 * q]);
        ranks_ok = ranks_ok && pairs[2 * q] >= 0 && pairs[2 * q + 1] >= 0 && pairs[2 * q + 1] < K;
      }
      const bool ok = ranks_ok && max_rank < n_masked;
      valid[nd] = ok ? 1 : 0;
      if (ok)
        for (int q = node_off[nd]; q < node_off[nd + 1]; ++q) {
          const int pos = ranked[pairs[2 * q]];
          const int vr = pairs[2 * q + 1];
          d[pos_offset + pos] = top[static_cast<int64_t>(pos) * K + vr];
        }
    }
    __syncthreads();
  }
}

}  // namespace

int draft_max_topk() { return kMaxTopK; }
int draft_max_positions() { return 1024; }

cudaError_t launch_draft_blocks(int dtype, const void* logits, int64_t row_stride, int n_pos,
                                int V, int K, int conf_fp32, const uint8_t* mask,
                                const int32_t* pairs, const int32_t* node_off, int n_nodes,
                                const int64_t* block, int block_len, int pos_offset,
                                int64_t* drafts, int32_t* valid, float* conf, int64_t* top,
                                cudaStream_t st) {
  if (n_pos > 0) {
    if (dtype == BF16)
      draft_rows_kernel<__nv_bfloat16><<<n_pos, kDraftThreads, 0, st>>>(
          static_cast<const __nv_bfloat16*>(logits), row_stride, V, K, conf_fp32, conf, top);
    else
      draft_rows_kernel<float><<<n_pos, kDraftThreads, 0, st>>>(
          static_cast<const float*>(logits), row_stride, V, K, conf_fp32, conf, top);
    cudaError_t e = launched();
    if (e != cudaSuccess) return e;
  }
  draft_assemble_kernel<<<1, 256, 0, st>>>(conf, top, K, mask, n_pos, pairs, node_off, n_nodes,
                                           block, block_len, pos_offset, drafts, valid);
  return launched();
}

}  // namespace sf
