// extern "C" entry points of libspecfold_b200 (declared in include/specfold_b200.h) and
// the whole-forward layer loop.
#include <cstring>
#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <mutex>
#include <unordered_set>
#include <cstdlib>
#include <string>
#include <vector>

#include "../../include/specfold_b200.h"
#include "sf_kernels.cuh"

using namespace sf;

namespace sf {
static std::atomic<long long> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
// Programmatic dependent launch is off unless SF_PDL=1: measured on the verify forward
// (captured as a CUDA graph) it did not shorten the step.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("SF_PDL");
    return v != nullptr && atoi(v) != 0;
  }();
  return on;
}
}  // namespace sf

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SF_OK;
  return fail(SF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

size_t esize(int dtype) { return dtype == SF_DTYPE_BF16 ? 2 : 4; }

bool dtype_ok(int dtype) { return dtype == SF_DTYPE_F32 || dtype == SF_DTYPE_BF16; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

int check_dims(int dtype, int D, int hd, int H, int Hkv) {
  if (!dtype_ok(dtype)) return fail(SF_ERR_ARG, "dtype %d not supported", dtype);
  if (D <= 0 || D % 64 != 0) return fail(SF_ERR_ARG, "hidden size %d must be a multiple of 64", D);
  if (hd != 64 && hd != 128) return fail(SF_ERR_ARG, "head_dim %d must be 64 or 128", hd);
  if (H <= 0 || Hkv <= 0 || H % Hkv != 0 || H / Hkv > 16)
    return fail(SF_ERR_ARG, "heads %d / kv heads %d unsupported", H, Hkv);
  return SF_OK;
}

// GEMM workspace need for one projection (rows_cap activation rows)
size_t ws_gemm(int dtype, int rows, int n_out, int K, int kind, int inter) {
  return gemm_ws_need(dtype, rows, n_out, K, kind, inter);
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// ---------------------------------------------------------------- profiling
// CUDA-event timing of the forward's launches, per kernel kind.  Host-side events
// only; one host thread at a time.
enum ProfKind {
  K_GATE = 0, K_COMPACT, K_QKV, K_ATTN, K_MERGE, K_OPROJ, K_FFN_NORM, K_GATEUP, K_DOWN,
  K_COMBINE, K_FINAL_NORM, K_LM_HEAD, K_FFN, K_TP_REDUCE, K_NUM
};
const char* kProfNames[K_NUM] = {"gate", "compact", "qkv", "attention", "merge", "o_proj",
                                 "ffn_norm", "gate_up", "down", "combine", "final_norm",
                                 "lm_head", "ffn", "tp_reduce"};
struct Profiler {
  bool on = false;
  std::vector<cudaEvent_t> ev;
  std::vector<int> kind;
  int used = 0, dropped = 0;
  double total_ms[K_NUM] = {};
  int calls[K_NUM] = {};
};
Profiler g_prof;

void prof_mark(int kind, cudaStream_t st, bool start) {
  if (!g_prof.on) return;
  if (start) {
    if (2 * (g_prof.used + 1) > static_cast<int>(g_prof.ev.size())) {
      ++g_prof.dropped;
      g_prof.kind.push_back(-1);
      return;
    }
    cudaEventRecord(g_prof.ev[2 * g_prof.used], st);
  } else {
    if (2 * (g_prof.used + 1) > static_cast<int>(g_prof.ev.size())) return;
    cudaEventRecord(g_prof.ev[2 * g_prof.used + 1], st);
    if (static_cast<int>(g_prof.kind.size()) <= g_prof.used) g_prof.kind.resize(g_prof.used + 1);
    g_prof.kind[g_prof.used] = kind;
    ++g_prof.used;
  }
}

template <typename F>
int timed(int kind, cudaStream_t st, F&& fn) {
  prof_mark(kind, st, true);
  const int r = fn();
  prof_mark(kind, st, false);
  return r;
}

// Carves the forward's scratch out of one buffer.
struct Carve {
  char* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<char*>(b)) {}
  void* take(size_t bytes) {
    void* p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  }
};

// device counters of the forward (zeroed per call): [0] the gate's grid barrier,
// [kSyncFfn + 2*layer ..] the FFN chain's dependencies
constexpr size_t kSyncBytes = 4096;
constexpr int kSyncFfn = 16;
// SF_CHAIN: 0 = separate launches, 1 = the FFN chained, 2 (default) = o_proj + FFN chained
static int chain_level() {
  static const int lvl = [] {
    const char* v = getenv("SF_CHAIN");
    return v == nullptr ? 2 : std::max(0, std::min(2, atoi(v)));
  }();
  return lvl;
}

struct FwdBufs {
  void *q_buf, *kv_buf, *O, *ffn, *act, *hbuf, *hp, *xn, *gemm_ws, *q_comp, *attn_ws;
  float *M, *Z, *rstd, *rstd2;
  int64_t *f, *src, *seg, *rows;
  int8_t* rec;
  float* gate_red;        // gate partial sums [BN][S][4]
  float* tp_sum;          // tensor parallel: fp32 partial sums [BN][D] of o_proj / down
  unsigned* sync;         // grid barrier counter (zeroed per forward)
  size_t gemm_ws_bytes, attn_ws_bytes, total;
};

FwdBufs carve_forward(void* ws, int dtype, int B1, int N, int D, int H, int Hkv, int hd, int I,
                      int V, int bucket, int P) {
  const size_t es = esize(dtype);
  const int BN = B1 * N, qd = H * hd, kvd = Hkv * hd;
  Carve c(ws);
  FwdBufs b{};
  b.q_buf = c.take((BN + 1) * static_cast<size_t>(qd) * es);
  b.kv_buf = c.take((BN + 1) * static_cast<size_t>(2 * kvd) * es);
  b.O = c.take(static_cast<size_t>(BN) * qd * es);
  b.M = static_cast<float*>(c.take(static_cast<size_t>(BN) * H * 4));
  b.Z = static_cast<float*>(c.take(static_cast<size_t>(BN) * H * 4));
  b.ffn = c.take((BN + 1) * static_cast<size_t>(D) * es);
  b.act = c.take(static_cast<size_t>(bucket) * I * es);
  b.hbuf = c.take(static_cast<size_t>(BN) * D * es);
  b.hp = c.take(static_cast<size_t>(BN) * D * es);
  b.xn = c.take(static_cast<size_t>(BN) * D * es);
  b.rstd = static_cast<float*>(c.take(static_cast<size_t>(BN) * 4));
  b.rstd2 = static_cast<float*>(c.take(static_cast<size_t>(bucket) * 4));
  b.f = static_cast<int64_t*>(c.take(static_cast<size_t>(BN) * 8));
  b.src = static_cast<int64_t*>(c.take(static_cast<size_t>(BN) * 8));
  b.seg = static_cast<int64_t*>(c.take(static_cast<size_t>(BN) * 8));
  b.rows = static_cast<int64_t*>(c.take(static_cast<size_t>(bucket) * 8));
  b.rec = static_cast<int8_t*>(c.take(static_cast<size_t>(BN)));
  b.gate_red = static_cast<float*>(
      c.take(static_cast<size_t>(BN) * gate_compact_slices(N, D) * 4 * sizeof(float)));
  b.sync = static_cast<unsigned*>(c.take(kSyncBytes));
  b.tp_sum = static_cast<float*>(c.take(static_cast<size_t>(BN) * D * sizeof(float)));
  size_t g = 0;
  g = std::max(g, ws_gemm(dtype, bucket, qd + 2 * kvd, D, EPI_QKV, 0));
  g = std::max(g, ws_gemm(dtype, BN, D, qd, EPI_RESID, 0));
  g = std::max(g, ws_gemm(dtype, bucket, 2 * I, D, EPI_SWIGLU, I));
  g = std::max(g, ws_gemm(dtype, bucket, D, I, EPI_SCATTER, 0));
  g = std::max(g, ws_gemm(dtype, BN, V, D, EPI_LOGITS, 0));
  // a prefill forward runs its LM head on the last block's N rows only
  g = std::max(g, ws_gemm(dtype, N, V, D, EPI_LOGITS, 0));
  // the chained o_proj's partials live beside the later phases' (its split reduction is
  // deferred to the post-attention norm)
  const size_t o_ws = ws_gemm(dtype, BN, D, qd, EPI_RESID, 0);
  if (o_ws > kGemmCounterBytes) g += o_ws - kGemmCounterBytes;
  b.gemm_ws_bytes = g;
  b.gemm_ws = c.take(g + 256);
  // tensor-core attention: query copy per kv head + split-KV partials
  const bool tc_attn = dtype == SF_DTYPE_BF16 && P > 0;
  b.q_comp = tc_attn ? c.take(static_cast<size_t>(bucket) * H * hd * es) : nullptr;
  b.attn_ws_bytes = attn_scratch_bytes(dtype, bucket, H, Hkv, hd, P, false, BN);
  b.attn_ws = b.attn_ws_bytes ? c.take(b.attn_ws_bytes) : nullptr;
  b.total = c.off;
  return b;
}

}  // namespace

namespace sf {
// lets other translation units of the library set sf_last_error()
int report_error(int code, const char* msg) { return fail(code, "%s", msg); }
int report_cuda(cudaError_t e, const char* what) { return cuda_status(e, what); }
}  // namespace sf

extern "C" {

const char* sf_last_error(void) { return g_err.c_str(); }

int sf_abi_version(void) { return 1; }

int sf_check_device(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return fail(SF_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                dev, major, minor);
  return SF_OK;
}

int sf_residual_delta_gate(int dtype, const void* Hf, const int64_t* par_idx, float* rstd,
                           int64_t* f, int8_t* rec, int64_t* rows, int32_t* count,
                           int64_t* seg, int32_t* segcnt, int64_t* src, void* xn,
                           const void* ln_w, float delta, int B1, int N, int D, int bucket,
                           float eps, int* err, void* stream) {
  if (!dtype_ok(dtype)) return fail(SF_ERR_ARG, "bad dtype");
  if (B1 < 1 || B1 > kMaxBranches || N < 1 || B1 * N > kMaxRows)
    return fail(SF_ERR_ARG, "B1=%d N=%d outside the supported range", B1, N);
  if (D % 64 != 0 || bucket < 1 || bucket > B1 * N)
    return fail(SF_ERR_ARG, "D=%d bucket=%d unsupported", D, bucket);
  if (static_cast<size_t>(B1) * D * esize(dtype) > static_cast<size_t>(kMaxGateSmem))
    return fail(SF_ERR_ARG, "B1*D too large for the gate");
  if (!Hf || !par_idx || !rstd || !f || !rec || !rows || !count || !seg || !segcnt || !src ||
      (xn && !ln_w))
    return fail(SF_ERR_ARG, "null pointer");
  GateRowsParams g{};
  g.hidden = const_cast<void*>(Hf);
  g.par_idx = par_idx;
  g.rstd = rstd;
  g.rec = rec;
  g.f = f;
  g.delta = delta;
  g.eps = eps;
  g.B1 = B1;
  g.N = N;
  g.D = D;
  g.err = err;
  int s = cuda_status(launch_gate_rows(dtype, g, S(stream)), "gate");
  if (s) return s;
  CompactParams c{};
  c.rec = rec;
  c.f = f;
  c.rows = rows;
  c.count = count;
  c.seg = seg;
  c.segcnt = segcnt;
  c.src = src;
  c.hidden = Hf;
  c.rstd = rstd;
  c.ln_w = ln_w;
  c.xn = xn;
  c.B1 = B1;
  c.N = N;
  c.D = D;
  c.bucket = bucket;
  c.err = err;
  return cuda_status(launch_compact(dtype, c, S(stream)), "compact");
}

int sf_src_resolve(const int64_t* f, int64_t* src, int B1, int N, int* err, void* stream) {
  if (!f || !src || B1 < 1 || N < 1) return fail(SF_ERR_ARG, "bad arguments");
  return cuda_status(launch_src_resolve(f, src, B1, N, err, S(stream)), "src_resolve");
}

size_t sf_workspace_bytes(int BN, int D, int H, int Hkv, int hd, int I, int V) {
  size_t g = 0;
  const int qd = H * hd, kvd = Hkv * hd;
  for (int dt = 0; dt < 2; ++dt) {
    g = std::max(g, ws_gemm(dt, BN, qd + 2 * kvd, D, EPI_QKV, 0));
    g = std::max(g, ws_gemm(dt, BN, D, qd, EPI_RESID, 0));
    g = std::max(g, ws_gemm(dt, BN, 2 * I, D, EPI_SWIGLU, I));
    g = std::max(g, ws_gemm(dt, BN, D, I, EPI_SCATTER, 0));
    g = std::max(g, ws_gemm(dt, BN, V, D, EPI_LOGITS, 0));
  }
  return g + 512;
}

int sf_workspace_init(void* ws, size_t ws_bytes, void* stream) {
  if (!ws) return fail(SF_ERR_ARG, "null workspace");
  return cuda_status(cudaMemsetAsync(ws, 0, ws_bytes, S(stream)), "workspace init");
}

static int run_gemm(GemmArgs& a, void* stream, const char* what) {
  if (a.dtype == SF_DTYPE_BF16) {
    if (!aligned16(a.X) || !aligned16(a.W) || (a.W2 && !aligned16(a.W2)))
      return fail(SF_ERR_ARG, "%s: operands must be 16-byte aligned", what);
  }
  const size_t need = gemm_ws_need(a.dtype, a.rows_cap, a.n_out, a.K, a.epi.kind, a.epi.inter);
  if (need > a.ws_bytes)
    return fail(SF_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", what, a.ws_bytes, need);
  return cuda_status(gemm(a, S(stream)), what);
}

int sf_fused_ln_qkv_rope_scatter(int dtype, const void* xn, const void* w_qkv,
                                 const void* b_qkv, const int64_t* rows, const int32_t* count,
                                 const void* cos, const void* sin, const float* q_scale,
                                 void* q_buf, void* kv_buf, int D, int N, int bucket, int H,
                                 int Hkv, int hd, void* ws, size_t ws_bytes, int* err,
                                 void* stream) {
  int s = check_dims(dtype, D, hd, H, Hkv);
  if (s) return s;
  if (!xn || !w_qkv || !rows || !count || !cos || !sin || !q_buf || !kv_buf)
    return fail(SF_ERR_ARG, "null pointer");
  GemmArgs a{};
  a.dtype = dtype;
  a.X = xn;
  a.W = w_qkv;
  a.n_out = (H + 2 * Hkv) * hd;
  a.K = D;
  a.rows_cap = bucket;
  a.count = count;
  a.epi.kind = EPI_QKV;
  a.epi.out = q_buf;
  a.epi.out2 = kv_buf;
  a.epi.bias = b_qkv;
  a.epi.cos = cos;
  a.epi.sin = sin;
  a.epi.q_scale = q_scale;
  a.epi.rows = rows;
  a.epi.q_dim = H * hd;
  a.epi.kv_dim = Hkv * hd;
  a.epi.hd = hd;
  a.epi.N = N;
  a.ws = ws;
  a.ws_bytes = ws_bytes;
  a.err = err;
  return run_gemm(a, stream, "qkv");
}

int sf_flash_attn_gqa(int dtype, const void* q_buf, const void* prefix_k, const void* prefix_v,
                      int64_t kv_head_stride, const void* kv_buf, const int64_t* src,
                      const int64_t* rows, const int32_t* count, void* O_tab, float* M_tab,
                      float* Z_tab, int P, int N, float scale, int bucket, int B1, int H,
                      int Hkv, int hd, void* ws, size_t ws_bytes, int* err, void* stream) {
  int s = check_dims(dtype, 64, hd, H, Hkv);
  if (s) return s;
  if (P < 0 || (P > 0 && (!prefix_k || !prefix_v)) || !q_buf || !kv_buf || !src || !rows ||
      !count || !O_tab || !M_tab || !Z_tab || N < 1 || bucket < 1 || B1 < 1 || bucket > B1 * N)
    return fail(SF_ERR_ARG, "bad attention arguments");
  if (P > 0 && kv_head_stride < static_cast<int64_t>(P) * hd)
    return fail(SF_ERR_ARG, "kv_head_stride %lld < P*hd", static_cast<long long>(kv_head_stride));
  if (P > 0 && kv_head_stride % hd != 0)
    return fail(SF_ERR_ARG, "kv_head_stride must be a multiple of head_dim");
  const size_t need = attn_scratch_bytes(dtype, bucket, H, Hkv, hd, P, true);
  if (need > 0 && (!ws || ws_bytes < need))
    return fail(SF_ERR_WORKSPACE, "attention workspace %zu < %zu bytes", ws_bytes, need);
  AttnParams p{};
  p.q_buf = q_buf;
  p.pk = prefix_k;
  p.pv = prefix_v;
  p.kv_head_stride = kv_head_stride;
  p.kv_buf = kv_buf;
  p.src = src;
  p.rows = rows;
  p.count = count;
  p.O = O_tab;
  p.M = M_tab;
  p.Z = Z_tab;
  p.P = P;
  p.N = N;
  p.bucket = bucket;
  p.H = H;
  p.Hkv = Hkv;
  p.hd = hd;
  p.B1 = B1;
  p.scale = scale;
  p.err = err;
  p.q_comp = nullptr;   // packed from q_buf into the workspace
  p.scratch = ws;
  p.scratch_bytes = ws_bytes;
  return cuda_status(launch_attention(dtype, p, S(stream)), "attention");
}

size_t sf_attn_workspace_bytes(int dtype, int bucket, int H, int Hkv, int hd, int P) {
  return attn_scratch_bytes(dtype, bucket, H, Hkv, hd, P, true);
}

int sf_chain_correction_gqa(int dtype, const void* q_buf, const void* kv_buf,
                            const int64_t* src, const int64_t* par_idx, const int8_t* rec,
                            const int64_t* seg, const int32_t* segcnt, void* O_tab,
                            float* M_tab, float* Z_tab, int B1, int N, float scale, int H,
                            int Hkv, int hd, int* err, void* stream) {
  int s = check_dims(dtype, 64, hd, H, Hkv);
  if (s) return s;
  if (!q_buf || !kv_buf || !src || !par_idx || !rec || !seg || !segcnt || !O_tab || !M_tab ||
      !Z_tab || B1 < 1 || N < 1)
    return fail(SF_ERR_ARG, "bad merge arguments");
  MergeParams p{};
  p.q_buf = q_buf;
  p.kv_buf = kv_buf;
  p.src = src;
  p.par_idx = par_idx;
  p.rec = rec;
  p.seg = seg;
  p.segcnt = segcnt;
  p.O = O_tab;
  p.M = M_tab;
  p.Z = Z_tab;
  p.B1 = B1;
  p.N = N;
  p.H = H;
  p.Hkv = Hkv;
  p.hd = hd;
  p.scale = scale;
  p.err = err;
  return cuda_status(launch_merge(dtype, p, S(stream)), "chain correction");
}

int sf_o_proj_residual(int dtype, const void* Hf, const void* O_tab, const void* w_o, void* hp,
                       int BN, int D, int q_dim, void* ws, size_t ws_bytes, int* err,
                       void* stream) {
  if (!dtype_ok(dtype) || !Hf || !O_tab || !w_o || !hp || BN < 1 || D % 64 || q_dim % 64)
    return fail(SF_ERR_ARG, "bad o_proj arguments");
  GemmArgs a{};
  a.dtype = dtype;
  a.X = O_tab;
  a.W = w_o;
  a.n_out = D;
  a.K = q_dim;
  a.rows_cap = BN;
  a.epi.kind = EPI_RESID;
  a.epi.out = hp;
  a.epi.resid = Hf;
  a.epi.ld_out = D;
  a.ws = ws;
  a.ws_bytes = ws_bytes;
  a.err = err;
  return run_gemm(a, stream, "o_proj");
}

int sf_fused_ffn_scatter(int dtype, const void* hp_all, const void* ln_w, const void* w_gate,
                         const void* w_up, const void* w_down, const int64_t* rows,
                         const int32_t* count, void* ffn_buf, int bucket, void* act_buf,
                         void* xn_buf, float* rstd_buf, float eps, int D, int I, void* ws,
                         size_t ws_bytes, int* err, void* stream) {
  if (!dtype_ok(dtype) || !hp_all || !ln_w || !w_gate || !w_up || !w_down || !rows || !count ||
      !ffn_buf || !act_buf || !xn_buf || D % 64 || I % 64 || bucket < 1)
    return fail(SF_ERR_ARG, "bad ffn arguments");
  RmsRowsParams r{};
  r.x = hp_all;
  r.rows = rows;
  r.count = count;
  r.n = bucket;
  r.n_src = INT64_MAX;
  r.w = ln_w;
  r.out = xn_buf;
  r.rstd = rstd_buf;
  r.D = D;
  r.eps = eps;
  r.err = err;
  int s = cuda_status(launch_rmsnorm_rows(dtype, r, S(stream)), "ffn norm");
  if (s) return s;
  GemmArgs a{};
  a.dtype = dtype;
  a.X = xn_buf;
  a.W = w_gate;
  a.W2 = w_up;
  a.n_out = 2 * I;
  a.K = D;
  a.rows_cap = bucket;
  a.count = count;
  a.epi.kind = EPI_SWIGLU;
  a.epi.out = act_buf;
  a.epi.inter = I;
  a.ws = ws;
  a.ws_bytes = ws_bytes;
  a.err = err;
  s = run_gemm(a, stream, "gate/up");
  if (s) return s;
  GemmArgs d{};
  d.dtype = dtype;
  d.X = act_buf;
  d.W = w_down;
  d.n_out = D;
  d.K = I;
  d.rows_cap = bucket;
  d.count = count;
  d.epi.kind = EPI_SCATTER;
  d.epi.out = ffn_buf;
  d.epi.rows = rows;
  d.epi.ld_out = D;
  d.ws = ws;
  d.ws_bytes = ws_bytes;
  d.err = err;
  return run_gemm(d, stream, "down");
}

int sf_combine(int dtype, const void* hp_all, const void* ffn_buf, const int64_t* src,
               void* hidden, int B1, int N, int D, int* err, void* stream) {
  if (!dtype_ok(dtype) || !hp_all || !ffn_buf || !src || !hidden || D % 64)
    return fail(SF_ERR_ARG, "bad combine arguments");
  return cuda_status(launch_combine(dtype, hp_all, ffn_buf, src, hidden, B1, N, D, err, S(stream)),
                     "combine");
}

int sf_final_norm_lm_head(int dtype, const void* hidden, const void* norm_w, const void* lm_w,
                          void* logits, void* xn_buf, int B1, int N, int D, int V, float eps,
                          int shift, void* ws, size_t ws_bytes, int* err, void* stream) {
  if (!dtype_ok(dtype) || !hidden || !norm_w || !lm_w || !logits || !xn_buf || D % 64 || V < 1)
    return fail(SF_ERR_ARG, "bad lm_head arguments");
  const int BN = B1 * N;
  RmsRowsParams r{};
  r.x = hidden;
  r.n = BN;
  r.n_src = BN;
  r.w = norm_w;
  r.out = xn_buf;
  r.D = D;
  r.eps = eps;
  r.err = err;
  int s = cuda_status(launch_rmsnorm_rows(dtype, r, S(stream)), "final norm");
  if (s) return s;
  GemmArgs a{};
  a.dtype = dtype;
  a.X = xn_buf;
  a.W = lm_w;
  a.n_out = V;
  a.K = D;
  a.rows_cap = BN;
  a.epi.kind = EPI_LOGITS;
  a.epi.out = logits;
  a.epi.ld_out = V;
  a.epi.N = N;
  a.epi.shift = shift;
  a.ws = ws;
  a.ws_bytes = ws_bytes;
  a.err = err;
  return run_gemm(a, stream, "lm_head");
}

int sf_kv_append(int dtype, void* cache_k, void* cache_v, int64_t cache_head_stride,
                 const void* new_k, const void* new_v, int64_t new_head_stride, int Hkv, int hd,
                 int P, int n_new, void* stream) {
  if (!dtype_ok(dtype) || !cache_k || !cache_v || !new_k || !new_v || Hkv < 1 || P < 0 ||
      n_new < 0)
    return fail(SF_ERR_ARG, "bad kv_append arguments");
  const int vec = dtype == SF_DTYPE_BF16 ? 8 : 4;
  if (hd % vec || cache_head_stride % vec || new_head_stride % vec || !aligned16(cache_k) ||
      !aligned16(cache_v) || !aligned16(new_k) || !aligned16(new_v))
    return fail(SF_ERR_ARG, "kv_append needs 16-byte aligned rows");
  if (cache_head_stride < static_cast<int64_t>(P + n_new) * hd)
    return fail(SF_ERR_ARG, "cache capacity %lld < (P + n) * hd",
                static_cast<long long>(cache_head_stride));
  if (new_head_stride < static_cast<int64_t>(n_new) * hd)
    return fail(SF_ERR_ARG, "new_head_stride too small");
  return cuda_status(launch_kv_append(dtype, cache_k, cache_v, cache_head_stride, new_k, new_v,
                                      new_head_stride, Hkv, hd, P, n_new, S(stream)),
                     "kv_append");
}

size_t sf_draft_workspace_bytes(int n_pos, int K) {
  if (n_pos < 0 || K < 1) return 0;
  return ((static_cast<size_t>(n_pos) * 4 + 255) / 256) * 256 + static_cast<size_t>(n_pos) * K * 8;
}

int sf_draft_blocks(int dtype, const void* logits, int64_t row_stride, int n_pos, int V, int K,
                    int conf_fp32, const uint8_t* mask, const int32_t* pairs,
                    const int32_t* node_off, int n_nodes, const int64_t* block, int block_len,
                    int pos_offset, int64_t* drafts, int32_t* valid, void* ws, size_t ws_bytes,
                    void* stream) {
  if (!dtype_ok(dtype) || (n_pos > 0 && !logits) || !mask || !node_off || !block ||
      (n_nodes > 0 && (!drafts || !valid)) || n_pos < 0 || V < 1 || row_stride < V || n_nodes < 0 ||
      block_len < 1)
    return fail(SF_ERR_ARG, "bad draft_blocks arguments");
  if (K < 1 || K > draft_max_topk() || K > V)
    return fail(SF_ERR_ARG, "draft_blocks: K = %d outside [1, %d] or above V", K, draft_max_topk());
  if (n_pos > draft_max_positions() || pos_offset < 0 || pos_offset + n_pos > block_len)
    return fail(SF_ERR_ARG, "draft_blocks: positions [%d, %d) outside the block of %d (at most %d)",
                pos_offset, pos_offset + n_pos, block_len, draft_max_positions());
  const size_t need = sf_draft_workspace_bytes(n_pos, K);
  if (!ws || ws_bytes < need) return fail(SF_ERR_WORKSPACE, "draft_blocks: workspace %zu < %zu", ws_bytes, need);
  float* conf = static_cast<float*>(ws);
  int64_t* top = reinterpret_cast<int64_t*>(static_cast<char*>(ws) +
                                            ((static_cast<size_t>(n_pos) * 4 + 255) / 256) * 256);
  return cuda_status(launch_draft_blocks(dtype, logits, row_stride, n_pos, V, K, conf_fp32, mask,
                                         pairs, node_off, n_nodes, block, block_len, pos_offset,
                                         drafts, valid, conf, top, S(stream)),
                     "draft_blocks");
}

int sf_sample_top_p_greedy(int dtype, const void* logits, int64_t rows, int V,
                           int64_t row_stride, float top_p, int64_t* tokens, void* conf,
                           void* stream) {
  if (!dtype_ok(dtype) || !logits || !tokens || !conf || rows < 0 || V < 1 || row_stride < V ||
      !(top_p > 0.0f))
    return fail(SF_ERR_ARG, "bad sample_top_p_greedy arguments");
  if (rows > 0x7FFFFFFF) return fail(SF_ERR_ARG, "sample_top_p_greedy: too many rows");
  return cuda_status(launch_sample_top_p(dtype, logits, rows, V, row_stride, top_p, tokens, conf,
                                         S(stream)),
                     "sample_top_p_greedy");
}

size_t sf_verify_workspace_bytes(int dtype, int B1, int N, int D, int H, int Hkv, int hd, int I,
                                 int V, int P) {
  return carve_forward(nullptr, dtype, B1, N, D, H, Hkv, hd, I, V, B1 * N, P).total + 256;
}

static int forward_launches(const sf_verify_args* a, const FwdBufs& b, cudaStream_t st);
static int forward_graph(const sf_verify_args* a, const FwdBufs& b);
static bool graphs_enabled() {
  static const bool on = [] {
    const char* v = getenv("SF_GRAPH");
    return v == nullptr || atoi(v) != 0;
  }();
  return on;
}

int sf_folded_verify_forward(const sf_verify_args* a) {
  if (!a) return fail(SF_ERR_ARG, "null args");
  const int dtype = a->dtype;
  int s = check_dims(dtype, a->D, a->hd, a->H, a->Hkv);
  if (s) return s;
  const int B1 = a->B1, N = a->N, D = a->D, H = a->H, Hkv = a->Hkv, hd = a->hd, I = a->I,
            V = a->V, L = a->L;
  const int BN = B1 * N;
  if (B1 < 1 || B1 > kMaxBranches || N < 1 || BN > kMaxRows || L < 1 || I % 64 || V < 1 ||
      kSyncFfn + 8 * L > static_cast<int>(kSyncBytes / 4))
    return fail(SF_ERR_ARG, "shape B1=%d N=%d L=%d I=%d V=%d unsupported", B1, N, L, I, V);
  const int bucket = a->bucket;
  if (bucket < 1 || bucket > BN) return fail(SF_ERR_ARG, "bucket %d outside [1, %d]", bucket, BN);
  if (static_cast<size_t>(B1) * D * esize(dtype) > static_cast<size_t>(kMaxGateSmem))
    return fail(SF_ERR_ARG, "B1*D too large for the gate");
  if (!a->layers || !a->final_norm_w || !a->lm_w || !a->par_idx || !a->hidden_in || !a->cos ||
      !a->sin || (!a->logits && !a->commit) || !a->count_slab || !a->segcnt_slab || !a->ws)
    return fail(SF_ERR_ARG, "null pointer in verify args");
  if (a->P < 0 || (a->P > 0 && a->kv_head_stride < static_cast<int64_t>(a->P) * hd))
    return fail(SF_ERR_ARG, "prefix length / stride mismatch");
  if (a->tp_size > 1 && ((a->tp_comm == nullptr && a->tp_peers == nullptr) || D % 4 != 0))
    return fail(SF_ERR_ARG, "tensor parallel forward needs a communicator (sf_tp_comm_init) "
                            "or a peer table (sf_tp_peers_init)");
  if (a->tp_size > 1 && a->tp_peers != nullptr) {
    const TpPeers* tp = static_cast<const TpPeers*>(a->tp_peers);
    if (tp->size != a->tp_size || tp->part_elems < static_cast<int64_t>(BN) * D)
      return fail(SF_ERR_ARG, "peer table: %d ranks / %lld partial elements, the forward needs "
                              "%d / %lld", tp->size, static_cast<long long>(tp->part_elems),
                  a->tp_size, static_cast<long long>(BN) * D);
  }
  if (a->commit && ((B1 != 1 && !a->prefill) ||
                    a->kv_head_stride < static_cast<int64_t>(a->P + BN) * hd || hd % 8 != 0))
    return fail(SF_ERR_ARG, "commit forward needs B1 == 1 (or prefill) and kv_head_stride >= "
                            "(P + B1 * N) * hd");
  if (a->prefill && (!a->commit || a->delta >= 0.f || a->shift_logits || a->tp_size > 1))
    return fail(SF_ERR_ARG, "prefill needs commit, a negative delta (dense), no logit shift "
                            "and no tensor parallelism");
  // prefill: the attention covers the prompt blocks' keys as well (its scratch is sized
  // for P + B1 * N keys; sf_verify_workspace_bytes with that P gives the size)
  FwdBufs b = carve_forward(a->ws, dtype, B1, N, D, H, Hkv, hd, I, V, bucket,
                            a->P + (a->prefill ? BN : 0));
  if (b.total > a->ws_bytes)
    return fail(SF_ERR_WORKSPACE, "workspace %zu < %zu bytes", a->ws_bytes, b.total);
  for (int li = 0; li < L; ++li) {
    const sf_layer& ly = a->layers[li];
    if (!ly.w_qkv || !ly.ln1_w || !ly.w_o || !ly.ln2_w || !ly.w_gate ||
        (!ly.w_up && !a->weights_tiled) || !ly.w_down ||
        ((a->P > 0 || a->commit) && (!ly.prefix_k || !ly.prefix_v)))
      return fail(SF_ERR_ARG, "layer %d: null weight", li);
  }
  if (g_prof.on || !graphs_enabled()) return forward_launches(a, b, S(a->stream));
  return forward_graph(a, b);
}

// The launches of one verify forward on stream st (validated arguments).
static int tp_status(int r) {
  if (r == 0) return 0;
  return fail(SF_ERR_CUDA, "tensor-parallel all-reduce: %s", tp_error_string(r));
}

// L2 prefetch plan of a GEMM of the forward (only the fields that shape its plan)
static WPrefetch pf_plan(int dtype, int tiled, const void* W, int n_out, int K, int rows_cap,
                         int kind, int inter) {
  GemmArgs g{};
  g.dtype = dtype;
  g.w_tiled = tiled;
  g.W = W;
  g.n_out = n_out;
  g.K = K;
  g.rows_cap = rows_cap;
  g.epi.kind = kind;
  g.epi.inter = inter;
  return gemm_prefetch_plan(g);
}

static int forward_launches(const sf_verify_args* a, const FwdBufs& b, cudaStream_t st) {
  const int dtype = a->dtype;
  const int B1 = a->B1, N = a->N, D = a->D, H = a->H, Hkv = a->Hkv, hd = a->hd, I = a->I,
            V = a->V, L = a->L;
  const int BN = B1 * N;
  const int bucket = a->bucket;
  int s = 0;
  const int qd = H * hd, kvd = Hkv * hd;
  // split-K tile counters (first 16 KB of the GEMM scratch) start at zero
  if (b.gemm_ws_bytes > 0) {
    s = cuda_status(cudaMemsetAsync(b.gemm_ws, 0, std::min<size_t>(b.gemm_ws_bytes, kGemmCounterBytes), st),
                    "memset");
    if (s) return s;
  }
  s = cuda_status(cudaMemsetAsync(a->count_slab, 0, sizeof(int32_t) * L, st), "memset");
  if (s) return s;
  s = cuda_status(cudaMemsetAsync(b.sync, 0, kSyncBytes, st), "memset");
  if (s) return s;
  s = cuda_status(cudaMemsetAsync(a->segcnt_slab, 0, sizeof(int32_t) * L * B1, st), "memset");
  if (s) return s;
  if (a->err) {
    s = cuda_status(cudaMemsetAsync(a->err, 0, sizeof(int32_t), st), "memset");
    if (s) return s;
  }
  const TpPeers* peers = a->tp_size > 1 ? static_cast<const TpPeers*>(a->tp_peers) : nullptr;
  if (peers && (s = cuda_status(launch_tp_epoch(*peers, st), "tp epoch"))) return s;

  for (int li = 0; li < L; ++li) {
    const sf_layer& ly = a->layers[li];
    const void* Hf = li == 0 ? a->hidden_in : b.hbuf;
    int8_t* rec = a->rec_slab ? a->rec_slab + static_cast<int64_t>(li) * BN : b.rec;
    int32_t* count = a->count_slab + li;
    int32_t* segcnt = a->segcnt_slab + static_cast<int64_t>(li) * B1;

    // previous layer's combine + delta gate + compaction + normalised QKV input
    GateCompactParams g{};
    g.hp = li == 0 ? nullptr : b.hp;
    g.ffn = b.ffn;
    g.src_prev = b.src;
    g.hidden = const_cast<void*>(Hf);
    g.par_idx = a->par_idx;
    g.ln_w = ly.ln1_w;
    g.rec = rec;
    g.f = b.f;
    g.rows = b.rows;
    g.count = count;
    g.seg = b.seg;
    g.segcnt = segcnt;
    g.src = b.src;
    g.xn = b.xn;
    g.red = b.gate_red;
    g.bar = b.sync;
    g.bar_target = static_cast<unsigned>(li + 1) * static_cast<unsigned>(N * gate_compact_slices(N, D));
    g.delta = a->delta;
    g.eps = a->eps;
    g.B1 = B1;
    g.N = N;
    g.D = D;
    g.bucket = bucket;
    g.err = a->err;
    if ((s = timed(K_GATE, st, [&] { return cuda_status(launch_gate_compact(dtype, g, st), "gate"); })))
      return s;

    GemmArgs q{};
    q.dtype = dtype;
    q.X = b.xn;
    q.W = ly.w_qkv;
    q.w_tiled = a->weights_tiled;
    q.n_out = qd + 2 * kvd;
    q.K = D;
    q.rows_cap = bucket;
    q.count = count;
    q.epi.kind = EPI_QKV;
    q.epi.out = b.q_buf;
    q.epi.out2 = b.kv_buf;
    q.epi.bias = ly.b_qkv;
    q.epi.cos = a->cos;
    q.epi.sin = a->sin;
    q.epi.q_scale = a->q_scale;
    q.epi.rows = b.rows;
    q.epi.q_dim = qd;
    q.epi.kv_dim = kvd;
    q.epi.hd = hd;
    // prefill: every row has its own position (RoPE tables of B1 * N rows)
    q.epi.N = a->prefill ? BN : N;
    q.epi.q_comp = b.q_comp;
    q.epi.q_comp_rows = bucket * (H / Hkv);
    q.ws = b.gemm_ws;
    q.ws_bytes = b.gemm_ws_bytes;
    q.err = a->err;
    // each GEMM's producer pulls the next GEMM's first weight blocks into L2
    const int tl = a->weights_tiled;
    q.next_pf = pf_plan(dtype, tl, ly.w_o, D, qd, BN, EPI_RESID, 0);
    if ((s = timed(K_QKV, st, [&] { return run_gemm(q, st, "qkv"); }))) return s;

    AttnParams at{};
    at.q_buf = b.q_buf;
    at.pk = ly.prefix_k;
    at.pv = ly.prefix_v;
    at.kv_head_stride = a->kv_head_stride;
    at.kv_buf = b.kv_buf;
    at.src = b.src;
    at.rows = b.rows;
    at.count = count;
    at.O = b.O;
    at.M = b.M;
    at.Z = b.Z;
    at.P = a->P;
    at.N = N;
    at.bucket = bucket;
    at.H = H;
    at.Hkv = Hkv;
    at.hd = hd;
    at.B1 = B1;
    at.scale = a->scale;
    at.err = a->err;
    at.q_comp = b.q_comp;
    at.scratch = b.attn_ws;
    at.scratch_bytes = b.attn_ws_bytes;
    at.rec = rec;
    at.P_dev = a->P_dev;
    if (a->prefill) {
      // every block's keys and values join the cache first: block b attends to the
      // prefix and blocks 0..b-1 there, and to itself from kv_buf
      if ((s = cuda_status(launch_kv_commit(dtype, b.kv_buf, const_cast<void*>(ly.prefix_k),
                                            const_cast<void*>(ly.prefix_v), a->kv_head_stride,
                                            a->P_dev, a->P, BN, Hkv, hd, a->err, st),
                           "kv commit (prefill)")))
        return s;
      at.prefill_rows = BN;
      at.P = a->P + BN;
    }
    // every row: recomputed rows attend with their own query, folded rows are rebuilt
    // from their recomputing ancestor's query and retained prefix state
    if ((s = timed(K_ATTN, st, [&] { return cuda_status(launch_attention_rows(dtype, at, st), "attention"); })))
      return s;
    if (a->commit && !a->prefill) {
      // the committed block's keys and values join the prefix cache (its rows [P', P' + N)
      // are not read by this layer's attention, which covers [0, P'))
      if ((s = cuda_status(launch_kv_commit(dtype, b.kv_buf, const_cast<void*>(ly.prefix_k),
                                            const_cast<void*>(ly.prefix_v), a->kv_head_stride,
                                            a->P_dev, a->P, N, Hkv, hd, a->err, st),
                           "kv commit")))
        return s;
    }

    GemmArgs o{};
    o.dtype = dtype;
    o.X = b.O;
    o.W = ly.w_o;
    o.w_tiled = a->weights_tiled;
    o.n_out = D;
    o.K = qd;
    o.rows_cap = BN;
    o.epi.kind = EPI_RESID;
    o.epi.out = b.hp;
    o.epi.resid = Hf;
    o.epi.ld_out = D;
    o.ws = b.gemm_ws;
    o.ws_bytes = b.gemm_ws_bytes;
    o.err = a->err;
    o.next_pf = pf_plan(dtype, tl, ly.w_gate, 2 * I, D, bucket, EPI_SWIGLU, I);
    if (a->tp_size > 1) {
      // tensor parallel: this rank's heads give a partial o_proj sum; all-reduce, then
      // hp = T(x + T(sum)) as the unsharded epilogue does
      GemmArgs op = o;
      op.epi.kind = EPI_RAW;
      op.epi.out = peers ? peers->part[peers->rank] : b.tp_sum;
      op.epi.resid = nullptr;
      op.epi.ld_out = D;
      op.next_pf = WPrefetch{};
      if ((s = timed(K_OPROJ, st, [&] { return run_gemm(op, st, "o_proj (tp)"); }))) return s;
      if ((s = timed(K_TP_REDUCE, st, [&] {
             if (peers)
               return cuda_status(launch_tp_reduce_resid(dtype, *peers, li, L, Hf, b.hp,
                                                         static_cast<int64_t>(BN) * D, a->err, st),
                                  "tp reduce (o_proj)");
             int r = tp_status(tp_allreduce_f32(a->tp_comm, b.tp_sum, static_cast<size_t>(BN) * D, st));
             if (r) return r;
             return cuda_status(launch_resid_add(dtype, b.tp_sum, Hf, b.hp, static_cast<int64_t>(BN) * D, st),
                                "residual add");
           })))
        return s;
    }
    const bool chained = dtype == SF_DTYPE_BF16 && a->weights_tiled && chain_level() > 0 &&
                         a->tp_size <= 1;
    if (a->tp_size <= 1 && !(chained && chain_level() >= 2))
      if ((s = timed(K_OPROJ, st, [&] { return run_gemm(o, st, "o_proj"); }))) return s;

    GemmArgs gu{};
    gu.dtype = dtype;
    gu.X = b.xn;
    gu.W = ly.w_gate;
    gu.w_tiled = a->weights_tiled;
    gu.W2 = ly.w_up;
    gu.n_out = 2 * I;
    gu.K = D;
    gu.rows_cap = bucket;
    gu.count = count;
    gu.epi.kind = EPI_SWIGLU;
    gu.epi.out = b.act;
    gu.epi.inter = I;
    gu.ws = b.gemm_ws;
    gu.ws_bytes = b.gemm_ws_bytes;
    gu.err = a->err;
    gu.next_pf = pf_plan(dtype, tl, ly.w_down, D, I, bucket, EPI_SCATTER, 0);

    GemmArgs dn{};
    dn.dtype = dtype;
    dn.X = b.act;
    dn.W = ly.w_down;
    dn.w_tiled = a->weights_tiled;
    dn.n_out = D;
    dn.K = I;
    dn.rows_cap = bucket;
    dn.count = count;
    dn.epi.kind = EPI_SCATTER;
    dn.epi.out = b.ffn;
    dn.epi.rows = b.rows;
    dn.epi.ld_out = D;
    dn.ws = b.gemm_ws;
    dn.ws_bytes = b.gemm_ws_bytes;
    dn.err = a->err;
    dn.next_pf = li + 1 < L ? pf_plan(dtype, tl, a->layers[li + 1].w_qkv, qd + 2 * kvd, D, bucket, EPI_QKV, 0)
                            : pf_plan(dtype, tl, a->lm_w, V, D, BN, EPI_LOGITS, 0);

    if (a->tp_size > 1) {
      // this rank's intermediate shard: gate/up + down partial sums, all-reduce, scatter
      GemmArgs dp = dn;
      dp.epi.kind = EPI_RAW;
      dp.epi.out = peers ? peers->part[peers->rank] + peers->part_elems : b.tp_sum;
      dp.epi.rows = nullptr;
      dp.epi.ld_out = D;
      dp.next_pf = WPrefetch{};
      const bool tp_chain = dtype == SF_DTYPE_BF16 && a->weights_tiled && chain_level() > 0;
      if (tp_chain) {
        PreNormArgs pre{};
        pre.x = b.hp;
        pre.rows = b.rows;
        pre.count = count;
        pre.w = ly.ln2_w;
        pre.out = b.xn;
        pre.n = bucket;
        pre.n_src = BN;
        pre.D = D;
        pre.eps = a->eps;
        const GemmArgs chain[2] = {gu, dp};
        const PreNormArgs* norms[2] = {&pre, nullptr};
        if ((s = timed(K_FFN, st, [&] {
               return cuda_status(gemm_chain(chain, 2, norms, b.sync + kSyncFfn + 8 * li, st),
                                  "ffn (tp)");
             })))
          return s;
      } else {
        RmsRowsParams r{};
        r.x = b.hp;
        r.rows = b.rows;
        r.count = count;
        r.n = bucket;
        r.n_src = BN;
        r.w = ly.ln2_w;
        r.out = b.xn;
        r.rstd = b.rstd2;
        r.D = D;
        r.eps = a->eps;
        r.err = a->err;
        if ((s = timed(K_FFN_NORM, st, [&] { return cuda_status(launch_rmsnorm_rows(dtype, r, st), "ffn norm"); })))
          return s;
        if ((s = timed(K_GATEUP, st, [&] { return run_gemm(gu, st, "gate/up"); }))) return s;
        if ((s = timed(K_DOWN, st, [&] { return run_gemm(dp, st, "down (tp)"); }))) return s;
      }
      if ((s = timed(K_TP_REDUCE, st, [&] {
             if (peers)
               return cuda_status(launch_tp_reduce_scatter(dtype, *peers, li, L, b.rows, count,
                                                           bucket, D, BN + 1, b.ffn, a->err, st),
                                  "tp reduce (down)");
             int r = tp_status(tp_allreduce_f32(a->tp_comm, b.tp_sum, static_cast<size_t>(bucket) * D, st));
             if (r) return r;
             return cuda_status(launch_scatter_rows(dtype, b.tp_sum, b.rows, count, bucket, D, BN + 1,
                                                    b.ffn, a->err, st),
                                "ffn scatter");
           })))
        return s;
      continue;
    }
    if (chained) {
      // post-attention RMSNorm + gate/up + down in one launch (fastdllm_v2_folded.py:
      // 209-219; triton_kernels.py:103-174)
      PreNormArgs pre{};
      pre.x = b.hp;
      pre.rows = b.rows;
      pre.count = count;
      pre.w = ly.ln2_w;
      pre.out = b.xn;
      pre.n = bucket;
      pre.n_src = BN;
      pre.D = D;
      pre.eps = a->eps;
      pre.rec = rec;   // the o_proj split reduction happens in the norm (gemm_chain)
      if (chain_level() >= 2) {
        // o_proj + residual, then the norm, gate/up and down: one launch
        const GemmArgs chain[3] = {o, gu, dn};
        const PreNormArgs* norms[3] = {nullptr, &pre, nullptr};
        if ((s = timed(K_FFN, st, [&] {
               return cuda_status(gemm_chain(chain, 3, norms, b.sync + kSyncFfn + 8 * li, st),
                                  "o_proj + ffn");
             })))
          return s;
      } else {
        const GemmArgs chain[2] = {gu, dn};
        const PreNormArgs* norms[2] = {&pre, nullptr};
        if ((s = timed(K_FFN, st, [&] {
               return cuda_status(gemm_chain(chain, 2, norms, b.sync + kSyncFfn + 8 * li, st), "ffn");
             })))
          return s;
      }
      continue;
    }

    RmsRowsParams r{};
    r.x = b.hp;
    r.rows = b.rows;
    r.count = count;
    r.n = bucket;
    r.n_src = BN;
    r.w = ly.ln2_w;
    r.out = b.xn;
    r.rstd = b.rstd2;
    r.D = D;
    r.eps = a->eps;
    r.err = a->err;
    if ((s = timed(K_FFN_NORM, st, [&] { return cuda_status(launch_rmsnorm_rows(dtype, r, st), "ffn norm"); })))
      return s;
    if ((s = timed(K_GATEUP, st, [&] { return run_gemm(gu, st, "gate/up"); }))) return s;
    if ((s = timed(K_DOWN, st, [&] { return run_gemm(dn, st, "down"); }))) return s;
  }
  // a commit forward whose logits nobody reads (a prompt block of a prefill) ends here
  if (a->logits == nullptr) return SF_OK;
  // last layer's combine, final norm, lm_head
  if ((s = timed(K_COMBINE, st, [&] {
         return cuda_status(launch_combine(dtype, b.hp, b.ffn, b.src, b.hbuf, B1, N, D, a->err, st),
                            "combine");
       })))
    return s;
  RmsRowsParams r{};
  // prefill: the logits of the last block only ([1, N, V], the rows a decode loop reads)
  const int lm_rows = a->prefill ? N : BN;
  const size_t lm_off = static_cast<size_t>(BN - lm_rows) * D * esize(dtype);
  r.x = static_cast<const char*>(b.hbuf) + lm_off;
  r.n = lm_rows;
  r.n_src = lm_rows;
  r.w = a->final_norm_w;
  r.out = b.xn;
  r.D = D;
  r.eps = a->eps;
  r.err = a->err;
  if ((s = timed(K_FINAL_NORM, st, [&] { return cuda_status(launch_rmsnorm_rows(dtype, r, st), "final norm"); })))
    return s;
  GemmArgs lm{};
  lm.dtype = dtype;
  lm.X = b.xn;
  lm.W = a->lm_w;
  lm.w_tiled = a->weights_tiled;
  lm.n_out = V;
  lm.K = D;
  lm.rows_cap = lm_rows;
  lm.epi.kind = EPI_LOGITS;
  lm.epi.out = a->logits;
  lm.epi.ld_out = V;
  lm.epi.N = N;
  lm.epi.shift = a->shift_logits;
  lm.ws = b.gemm_ws;
  lm.ws_bytes = b.gemm_ws_bytes;
  lm.err = a->err;
  return timed(K_LM_HEAD, st, [&] { return run_gemm(lm, st, "lm_head"); });
}

// ------------------------------------------------------------------ CUDA graphs
// A verify step is ~230 kernel launches whose host cost (tensor-map encoding, launch
// calls) exceeds the GPU time of the small kernels.  The launches of one argument set
// are captured once, on a private stream, into a CUDA graph; a call with byte-identical
// arguments (same pointers, shapes, scalars, layer table) replays it with one launch on
// the caller's stream.  Data behind the pointers may change freely between calls.
namespace {

struct GraphEntry {
  int device;
  std::string key;
  cudaGraphExec_t exec;
  long long launches;   // kernels in the graph (the library's launch counter advances by it)
  unsigned long long last_use;
};
std::mutex g_graph_mu;
std::vector<GraphEntry> g_graphs;
std::unordered_set<std::string> g_seen;
unsigned long long g_graph_clock = 0;
constexpr size_t kMaxGraphs = 16;

std::string graph_key(const sf_verify_args* a) {
  sf_verify_args c = *a;
  c.stream = nullptr;
  c.layers = nullptr;
  std::string k(reinterpret_cast<const char*>(&c), sizeof(c));
  k.append(reinterpret_cast<const char*>(a->layers), sizeof(sf_layer) * a->L);
  return k;
}

cudaStream_t capture_stream(int device) {
  static std::mutex mu;
  static std::vector<cudaStream_t> streams;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(streams.size()) <= device) streams.resize(device + 1, nullptr);
  if (!streams[device]) cudaStreamCreateWithFlags(&streams[device], cudaStreamNonBlocking);
  return streams[device];
}

}  // namespace

int sf_release_graphs(void) {
  std::lock_guard<std::mutex> lock(g_graph_mu);
  int dev0 = 0;
  cudaGetDevice(&dev0);
  for (auto& e : g_graphs) {
    cudaSetDevice(e.device);
    cudaGraphExecDestroy(e.exec);
  }
  cudaSetDevice(dev0);
  g_graphs.clear();
  g_seen.clear();
  return 0;
}

static int forward_graph(const sf_verify_args* a, const FwdBufs& b) {
  int dev = 0;
  int s = cuda_status(cudaGetDevice(&dev), "get device");
  if (s) return s;
  const std::string key = graph_key(a);
  cudaStream_t st = S(a->stream);
  {
    std::lock_guard<std::mutex> lock(g_graph_mu);
    for (auto& e : g_graphs) {
      if (e.device == dev && e.key == key) {
        e.last_use = ++g_graph_clock;
        s = cuda_status(cudaGraphLaunch(e.exec, st), "graph launch");
        if (!s) count_launch(static_cast<int>(e.launches));
        return s;
      }
    }
  }
  {
    // the first call of an argument set runs directly (it also performs the one-time
    // per-kernel setup); the second is captured
    std::lock_guard<std::mutex> lock(g_graph_mu);
    const std::string skey = std::to_string(dev) + ":" + key;
    if (g_seen.insert(skey).second) {
      if (g_seen.size() > 4 * kMaxGraphs) g_seen.clear();
      return forward_launches(a, b, st);
    }
  }
  cudaStream_t cs = capture_stream(dev);
  if (!cs) return fail(SF_ERR_CUDA, "could not create the capture stream");
  const long long before = g_launches.load();
  s = cuda_status(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
  if (s) return s;
  const int rs = forward_launches(a, b, cs);
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(cs, &g);
  if (rs) {
    if (g) cudaGraphDestroy(g);
    return rs;
  }
  if (ce != cudaSuccess || !g) {
    if (g) cudaGraphDestroy(g);
    return cuda_status(ce != cudaSuccess ? ce : cudaErrorUnknown, "end capture");
  }
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return cuda_status(ie, "graph instantiate");
  const long long n = g_launches.load() - before;
  g_launches.fetch_sub(n);            // counted when the graph runs, not when captured
  {
    std::lock_guard<std::mutex> lock(g_graph_mu);
    if (g_graphs.size() >= kMaxGraphs) {
      auto lru = g_graphs.begin();
      for (auto it = g_graphs.begin(); it != g_graphs.end(); ++it)
        if (it->last_use < lru->last_use) lru = it;
      cudaGraphExecDestroy(lru->exec);
      g_graphs.erase(lru);
    }
    g_graphs.push_back({dev, key, exec, n, ++g_graph_clock});
  }
  s = cuda_status(cudaGraphLaunch(exec, st), "graph launch");
  if (!s) count_launch(static_cast<int>(n));
  return s;
}

int sf_tp_unique_id(void* id_out, int bytes) {
  if (!id_out) return fail(SF_ERR_ARG, "null pointer");
  const int r = tp_unique_id(id_out, bytes);
  if (r == -1) return fail(SF_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  if (r == -2) return fail(SF_ERR_ARG, "id buffer smaller than 128 bytes");
  return r ? fail(SF_ERR_CUDA, "ncclGetUniqueId: %s", tp_error_string(r)) : 0;
}

int sf_tp_comm_init(const void* id, int nranks, int rank, void** comm_out) {
  if (!id || !comm_out || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(SF_ERR_ARG, "bad communicator arguments");
  const int r = tp_comm_init(id, nranks, rank, comm_out);
  if (r == -1) return fail(SF_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  return r ? fail(SF_ERR_CUDA, "ncclCommInitRank: %s", tp_error_string(r)) : 0;
}

size_t sf_tp_exchange_bytes(int BN, int D) {
  if (BN < 1 || D < 1) return 0;
  return kTpHeader + 2 * static_cast<size_t>(BN) * D * sizeof(float);
}

int sf_tp_peers_init(int rank, int size, void* const* xbufs, int BN, int D, void** peers_out) {
  if (!xbufs || !peers_out || size < 2 || size > kMaxTp || rank < 0 || rank >= size || BN < 1 ||
      D < 1 || D % 4 != 0)
    return fail(SF_ERR_ARG, "peer table: bad arguments");
  TpPeers* t = new TpPeers{};
  t->rank = rank;
  t->size = size;
  t->part_elems = static_cast<int64_t>(BN) * D;
  for (int q = 0; q < size; ++q) {
    if (!xbufs[q] || !aligned16(xbufs[q])) {
      delete t;
      return fail(SF_ERR_ARG, "peer table: exchange buffer %d null or unaligned", q);
    }
    char* base = static_cast<char*>(xbufs[q]);
    t->flags[q] = reinterpret_cast<int*>(base);
    t->part[q] = reinterpret_cast<float*>(base + kTpHeader);
  }
  t->epoch = reinterpret_cast<unsigned*>(static_cast<char*>(xbufs[rank]) + 2 * kMaxTp * sizeof(int));
  *peers_out = t;
  return SF_OK;
}

int sf_tp_peers_destroy(void* peers) {
  delete static_cast<TpPeers*>(peers);
  return SF_OK;
}

// CUDA IPC of an exchange buffer.  The buffer may sit inside a larger allocation (a caching
// allocator's block): the handle names the allocation and the offset locates the buffer.
// Opening maps the peer's allocation into the CURRENT device's context, with peer access
// enabled for it -- the device whose kernels read it.
namespace {
using AddrRangeFn = int (*)(unsigned long long*, size_t*, unsigned long long);
AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(ptr);
  });
  return fn;
}
}  // namespace

int sf_tp_ipc_export(const void* ptr, void* handle_out, int bytes, size_t* offset_out) {
  if (!ptr || !handle_out || !offset_out || bytes < static_cast<int>(sizeof(cudaIpcMemHandle_t)))
    return fail(SF_ERR_ARG, "ipc export: bad arguments");
  AddrRangeFn fn = addr_range_fn();
  if (!fn) return fail(SF_ERR_UNSUPPORTED, "cuMemGetAddressRange not available");
  unsigned long long base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<unsigned long long>(ptr)) != 0)
    return fail(SF_ERR_ARG, "ipc export: pointer is not device memory");
  cudaIpcMemHandle_t h;
  int s = cuda_status(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  if (s) return s;
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return SF_OK;
}

int sf_tp_ipc_open(const void* handle, int bytes, void** base_out) {
  if (!handle || !base_out || bytes < static_cast<int>(sizeof(cudaIpcMemHandle_t)))
    return fail(SF_ERR_ARG, "ipc open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess),
                     "cudaIpcOpenMemHandle");
}

int sf_tp_ipc_close(void* base) {
  if (!base) return fail(SF_ERR_ARG, "ipc close: null pointer");
  return cuda_status(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}

int sf_tp_comm_destroy(void* comm) {
  if (!comm) return 0;
  const int r = tp_comm_destroy(comm);
  return r ? fail(SF_ERR_CUDA, "ncclCommDestroy: %s", tp_error_string(r)) : 0;
}

int sf_parent_map(const int64_t* ids, int B1, int N, int64_t* par_idx, void* stream) {
  if (!ids || !par_idx) return fail(SF_ERR_ARG, "null pointer");
  if (B1 < 1 || B1 > kMaxBranches || N < 1 || B1 * N > kMaxRows)
    return fail(SF_ERR_ARG, "parent map shape B1=%d N=%d unsupported", B1, N);
  return cuda_status(launch_parent_map(ids, B1, N, par_idx, S(stream)), "parent map");
}

size_t sf_weight_tiles_bytes(int n_out, int K, int mode, int inter) {
  return weight_tiles_bytes(n_out, K, mode, inter);
}

int sf_pack_weight_tiles(const void* W, const void* W2, int n_out, int K, int mode, int inter,
                         void* dst, void* stream) {
  if (!W || !dst || K <= 0 || K % 8 || (mode != 0 && mode != 1) || (mode == 1 && (!W2 || inter <= 0)) ||
      (mode == 0 && n_out <= 0) || !aligned16(W) || !aligned16(dst) || (W2 && !aligned16(W2)))
    return fail(SF_ERR_ARG, "bad weight tiling arguments");
  return cuda_status(pack_weight_tiles(W, W2, n_out, K, mode, inter, dst, S(stream)),
                     "pack weight tiles");
}

long long sf_launch_count(void) { return sf::g_launches.load(); }

int sf_profile_begin(int capacity) {
  for (cudaEvent_t e : g_prof.ev) cudaEventDestroy(e);
  g_prof = Profiler();
  if (capacity <= 0) return SF_OK;
  g_prof.ev.resize(2 * static_cast<size_t>(capacity));
  for (auto& e : g_prof.ev) {
    cudaError_t r = cudaEventCreate(&e);
    if (r != cudaSuccess) return cuda_status(r, "cudaEventCreate");
  }
  g_prof.on = true;
  return SF_OK;
}

int sf_profile_end(void) {
  g_prof.on = false;
  for (int i = 0; i < g_prof.used; ++i) {
    cudaError_t r = cudaEventSynchronize(g_prof.ev[2 * i + 1]);
    if (r != cudaSuccess) return cuda_status(r, "cudaEventSynchronize");
    float ms = 0.f;
    r = cudaEventElapsedTime(&ms, g_prof.ev[2 * i], g_prof.ev[2 * i + 1]);
    if (r != cudaSuccess) return cuda_status(r, "cudaEventElapsedTime");
    const int k = g_prof.kind[i];
    if (k >= 0 && k < K_NUM) {
      g_prof.total_ms[k] += ms;
      g_prof.calls[k] += 1;
    }
  }
  if (g_prof.dropped) return fail(SF_ERR_ARG, "profile capacity exceeded (%d launches dropped)", g_prof.dropped);
  return SF_OK;
}

int sf_profile_kinds(void) { return K_NUM; }

const char* sf_profile_name(int kind) {
  return (kind >= 0 && kind < K_NUM) ? kProfNames[kind] : "";
}

int sf_profile_kind(int kind, double* total_ms, int* calls) {
  if (kind < 0 || kind >= K_NUM || !total_ms || !calls) return fail(SF_ERR_ARG, "bad profile kind");
  *total_ms = g_prof.total_ms[kind];
  *calls = g_prof.calls[kind];
  return SF_OK;
}

}  // extern "C"
