// hakm_runtime.cu — device context and C ABI of libhakm_cuda.
//
// hakmc_create binds the same tensors hakm_ctx_new binds (src/model.c:17-76)
// from an MLF2 image in host memory, uploads them once in a kernel-friendly
// device layout (same bytes, re-ordered), sizes the fp32 KV cache
// [seq][layer][max_seq][kv_dim] like the reference's, and captures one decode
// step as a CUDA graph. A step is: embedding, then per layer
//   qkv  (rmsnorm+q8 prologue; Q4_K q/k rows with bias+RoPE+K append; Q6_K v
//         rows with bias+V append)
//   attn (GQA decode attention)
//   wo   (q8 prologue; Q4_K + residual)
//   ffn  (rmsnorm+q8 prologue; Q4_K gate/up interleaved + SwiGLU)
//   down (fp32; Q6_K + residual)
// then lm_head (rmsnorm; Q6_K logits + argmax + step finalisation).
#include "../../include/hakm_cuda.h"
#include "hakm_internal.h"
#include "hakm_tmap.h"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <unistd.h>
#include <mutex>
#include <string>
#include <vector>

using namespace hakm;

// ------------------------------------------------------------ errors

static thread_local std::string g_err;

static void set_err(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
}

#define CK(call)                                                                    \
  do {                                                                              \
    cudaError_t e_ = (call);                                                        \
    if (e_ != cudaSuccess) {                                                        \
      set_err("%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
      return HAKMC_ECUDA;                                                           \
    }                                                                               \
  } while (0)

extern "C" const char* hakmc_last_error(void) { return g_err.c_str(); }
extern "C" int hakmc_version(void) { return 100; }

// ------------------------------------------------------------ MLF2 parsing

// MLF2 v2 (include/mlf2.h:55-87 of mithraeums/hako): 128-byte header,
// 104-byte directory entries, tensor data relative to data_off.
namespace {

struct MTensor {
  std::string name;
  uint32_t type = 0, n_dims = 0;
  uint64_t dims[4] = {0, 0, 0, 0};
  const uint8_t* data = nullptr;
  uint64_t nbytes = 0;
};

struct MImage {
  uint32_t n_layers, d_model, n_heads, n_kv, head_dim, ffn, ctx, vocab, flags;
  float theta, eps;
  std::map<std::string, MTensor> t;
};

template <class T>
T rd(const uint8_t* p) {
  T v;
  memcpy(&v, p, sizeof v);
  return v;
}

int parse_mlf2(const uint8_t* img, size_t size, MImage& m) {
  if (!img || size < 128) { set_err("MLF2 image too small"); return HAKMC_EFORMAT; }
  if (memcmp(img, "MLF2", 4) != 0) { set_err("bad magic (not MLF2)"); return HAKMC_EFORMAT; }
  if (rd<uint32_t>(img + 4) != 2) { set_err("unsupported MLF2 version %u", rd<uint32_t>(img + 4)); return HAKMC_EFORMAT; }
  m.n_layers = rd<uint32_t>(img + 12); m.d_model = rd<uint32_t>(img + 16);
  m.n_heads = rd<uint32_t>(img + 20); m.n_kv = rd<uint32_t>(img + 24);
  m.head_dim = rd<uint32_t>(img + 28); m.ffn = rd<uint32_t>(img + 32);
  m.ctx = rd<uint32_t>(img + 36); m.vocab = rd<uint32_t>(img + 40);
  m.theta = rd<float>(img + 44); m.eps = rd<float>(img + 48);
  m.flags = rd<uint32_t>(img + 52);
  const uint32_t nt = rd<uint32_t>(img + 56);
  const uint64_t toff = rd<uint64_t>(img + 60), doff = rd<uint64_t>(img + 76);
  if (toff + (uint64_t)nt * 104 > size || doff > size) { set_err("corrupt offsets"); return HAKMC_EFORMAT; }
  for (uint32_t i = 0; i < nt; i++) {
    const uint8_t* e = img + toff + (size_t)i * 104;
    MTensor t;
    t.name.assign((const char*)e, strnlen((const char*)e, 48));
    t.type = rd<uint32_t>(e + 48);
    t.n_dims = rd<uint32_t>(e + 52);
    for (int d = 0; d < 4; d++) t.dims[d] = rd<uint64_t>(e + 56 + 8 * d);
    const uint64_t rel = rd<uint64_t>(e + 88);
    t.nbytes = rd<uint64_t>(e + 96);
    if (doff + rel + t.nbytes > size) { set_err("tensor %s past end of image", t.name.c_str()); return HAKMC_EFORMAT; }
    t.data = img + doff + rel;
    m.t[t.name] = t;
  }
  return 0;
}

size_t row_bytes(uint32_t type, int n_in) {
  if (type == W_Q4K) return (size_t)(n_in / QK) * Q4K_BYTES;
  if (type == W_Q6K) return (size_t)(n_in / QK) * Q6K_BYTES;
  if (type == 0) return (size_t)n_in * 4;
  return 0;
}

}  // namespace

// RoPE (cos, sin) pairs of one position as the reference's build computes
// them (hakm_hostmath.c).
extern "C" void hakm_host_rope_row(float* cs, int head_dim, int pos, float theta);

// ------------------------------------------------------------ context

// token_dev word where forward_batch keeps the single-sequence API's last
// pick while it runs other sequences through the step kernel
constexpr int TOKEN_SAVE = 8;
// forward_batch: batches of at least this many sequences take the batched pass
constexpr int BATCH_ROWS_MIN = 8;

struct DevMat {         // one weight matrix on the device (layout: hakm_internal.h)
  int type = 0, rows = 0, cols = 0;
  uint8_t* w = nullptr;
  // tensor parallelism: w holds only this GPU's rows (Seg::w_row0 / w_rows)
  int shard_row0 = 0, shard_rows = 0;
};

struct DevLayer {
  float *attn_norm, *ffn_norm, *bqk, *bv;
  DevMat wqk, wv, wo, wgu, down;
};

struct UpStage;

struct hakmc_ctx {
  int device = 0, num_sms = 148;
  int L, D, H, KVH, hd, KV, F, V, max_seq, max_batch;
  float theta, eps;
  bool tied = false, pdl = true;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.f;
  std::vector<void*> allocs;
  std::vector<DevLayer> layers;
  DevMat tok_embd, lm_head;
  float* out_norm = nullptr;
  // KV cache [seq][layer][max_seq][KV]
  float *k_cache = nullptr, *v_cache = nullptr;
  // activations (sequence 0 for the single-sequence graph)
  float *xb, *q, *k, *v, *att, *hbuf, *logits, *rope_cs, *attn_part;
  int *token_dev, *pos_dev, *step_dev, *token_log, *prompt_dev;
  int prompt_cap = 0;
  unsigned long long* argmax_key;
  unsigned int* done_counter;
  const uint32_t* rsq = nullptr;  // rsqrtss table of this host (rsqrt_table_device)
  int* err_flag = nullptr;    // set by a kernel whose bounded wait gave up
  int token_log_cap = 0;
  int* h_pinned = nullptr;    // pinned staging: [0] token in, [1] argmax out
  float* logits_pinned = nullptr;
  int pos = 0;                // host mirror of *pos_dev
  int run_layers = 0;
  std::map<int, cudaGraphExec_t> graphs;  // keyed by attention split count
  // persistent step kernel: device program of one step for run_layers layers
  bool use_step = true;        // HAKMC_STEP=0 selects the per-phase graphs
  PhaseDesc* prog_dev = nullptr;
  int prog_cap = 0, prog_layers = -1;
  UpStage* up = nullptr;             // weight-upload staging, while loading
  CUtensorMap* tmaps_dev = nullptr;  // the program's chunk-stream tensor maps
  size_t tmaps_cap = 0;
  SegRange* ranges_dev = nullptr;  // [phase][cta][segment] rows of the step program
  size_t ranges_cap = 0;
  StepArgs step = {};
  size_t attn_part_floats = 0;    // attention scratch of one sequence
  unsigned int* step_bar = nullptr;
  unsigned int* step_tickets = nullptr;
  unsigned long long* step_keys = nullptr;
  // tagged exchange vectors of the step kernel: xb (two buffers), q, k, v, att, h
  uint64_t *xb_ll = nullptr, *q_ll = nullptr, *k_ll = nullptr, *v_ll = nullptr, *att_ll = nullptr,
           *h_ll = nullptr;
  size_t ll_words = 0;         // all of them, contiguous from xb_ll
  uint32_t tag_base = 1;       // first tag of the next launch
  bool step_ran = false;       // the exchange vectors hold the latest q/k/v/att/h
  // tensor parallelism (hakmc_tp_connect): regions every rank addresses
  int tp_rank = 0, tp_world = 1;
  unsigned int* step_xbar = nullptr;  // cross-GPU step counter, never reset
  unsigned int xbar_base = 0;         // steps run in tensor-parallel launches so far
  void* xr_ptr[XR_COUNT] = {};
  size_t xr_size[XR_COUNT] = {};
  void* peer_ptr[TP_MAX][XR_COUNT] = {};
  bool peer_ipc[TP_MAX] = {};         // opened through IPC (closed at destroy)
  // row-batched passes (hakmc_prefill_batched, batched decode): buffers for
  // pf_rows rows
  int pf_rows = 0;
  float *pf_x = nullptr, *pf_xn = nullptr, *pf_qk = nullptr, *pf_v = nullptr, *pf_q = nullptr, *pf_att = nullptr,
        *pf_gu = nullptr, *pf_h = nullptr, *pf_tmp = nullptr, *pf_xs = nullptr;
  int8_t* pf_xq = nullptr;
  int* row_io = nullptr;  // batched decode: [max_batch] tokens, positions, picks
  // batched decode: one captured graph per (rows, layers, attention score
  // capacity); dropped whenever a buffer it names is reallocated
  std::map<uint64_t, cudaGraphExec_t> bgraphs;
};

static int dalloc(hakmc_ctx* c, void** p, size_t n) {
  cudaError_t e = cudaMalloc(p, n ? n : 16);
  if (e != cudaSuccess) {
    set_err("cudaMalloc(%zu): %s", n, cudaGetErrorString(e));
    return HAKMC_ENOMEM;
  }
  c->allocs.push_back(*p);
  return 0;
}

static void drop_bgraphs(hakmc_ctx* c) {
  for (auto& kv : c->bgraphs) cudaGraphExecDestroy(kv.second);
  c->bgraphs.clear();
}

// Free one dalloc'd buffer before the context goes (a buffer being regrown).
static void dfree(hakmc_ctx* c, void* p) {
  if (!p) return;
  drop_bgraphs(c);  // a captured batched-decode graph may name this buffer
  for (size_t i = 0; i < c->allocs.size(); i++)
    if (c->allocs[i] == p) {
      cudaFree(p);
      c->allocs.erase(c->allocs.begin() + (long)i);
      return;
    }
}

// Pinned staging of the weight upload: two host buffers and two device
// buffers used in turn, so the host copy of one slice of rows (from the
// mapped file, in device row order) overlaps the transfer and the device
// repack of the previous one. Held only while a context loads.
struct UpStage {
  static constexpr size_t BYTES = 32u << 20;
  uint8_t* host[2] = {nullptr, nullptr};
  uint8_t* dev[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  bool used[2] = {false, false};
  int k = 0;
  cudaError_t open() {
    for (int b = 0; b < 2; b++) {
      cudaError_t e = cudaHostAlloc((void**)&host[b], BYTES, cudaHostAllocDefault);
      if (e == cudaSuccess) e = cudaMalloc((void**)&dev[b], BYTES);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  ~UpStage() {
    for (int b = 0; b < 2; b++) {
      if (done[b]) { cudaEventSynchronize(done[b]); cudaEventDestroy(done[b]); }
      if (dev[b]) cudaFree(dev[b]);
      if (host[b]) cudaFreeHost(host[b]);
    }
  }
};

// Upload rows of a Q4_K / Q6_K matrix. `order[i]` is the source row of device
// row i (identity when empty). Q6_K rows are split into 208-byte bodies (bytes
// reordered by lane class) and an fp16 d plane (hakmc_q6k_pack layout): the
// verbatim rows go to the device and the repack kernel lays them out there.
static int upload_mat(hakmc_ctx* c, DevMat& dm, const MTensor& t, int exp_cols, int exp_rows,
                      const std::vector<int>& order, const MTensor* t2 = nullptr) {
  if (t.type != W_Q4K && t.type != W_Q6K) {
    set_err("tensor %s: type %u unsupported on the device (Q4_K/Q6_K only)", t.name.c_str(), t.type);
    return HAKMC_EFORMAT;
  }
  if ((int)t.dims[0] != exp_cols || (int)t.dims[1] != exp_rows || exp_cols % QK) {
    set_err("tensor %s: dims [%llu,%llu], expected [%d,%d]", t.name.c_str(),
            (unsigned long long)t.dims[0], (unsigned long long)t.dims[1], exp_cols, exp_rows);
    return HAKMC_EFORMAT;
  }
  const size_t rb = row_bytes(t.type, exp_cols);
  if (t.nbytes < rb * exp_rows) { set_err("tensor %s: short data", t.name.c_str()); return HAKMC_EFORMAT; }
  int rows = exp_rows;
  if (t2) {  // interleave t (even device rows) with t2 (odd device rows)
    if (t2->type != t.type || t2->dims[0] != t.dims[0] || t2->dims[1] != t.dims[1]) {
      set_err("tensors %s/%s must share type and shape", t.name.c_str(), t2->name.c_str());
      return HAKMC_EFORMAT;
    }
    rows = 2 * exp_rows;
  }
  dm.type = (int)t.type;
  dm.rows = rows;
  dm.cols = exp_cols;
  const int nb = exp_cols / QK;
  auto src_row = [&](int i) -> const uint8_t* {
    if (t2) return ((i & 1) ? t2->data : t.data) + (size_t)(i >> 1) * rb;
    const int s = order.empty() ? i : order[i];
    return t.data + (size_t)s * rb;
  };
  const size_t drb = dev_row_bytes((int)t.type, nb);
  int e = dalloc(c, (void**)&dm.w, (size_t)rows * drb);
  if (e) return e;
  UpStage& U = *c->up;
  const int per = (int)std::max<size_t>(1, UpStage::BYTES / rb);  // rows per slice
  if ((size_t)per * rb > UpStage::BYTES) { set_err("tensor %s: rows too long to stage", t.name.c_str()); return HAKMC_EFORMAT; }
  for (int r0 = 0; r0 < rows; r0 += per) {
    const int n = std::min(per, rows - r0), b = U.k++ & 1;
    if (U.used[b]) CK(cudaEventSynchronize(U.done[b]));  // the slice before last has left this buffer
    for (int i = 0; i < n; i++) memcpy(U.host[b] + (size_t)i * rb, src_row(r0 + i), rb);
    uint8_t* dst = dm.w + (size_t)r0 * drb;
    if (t.type == W_Q4K) {  // the device row is the verbatim row
      CK(cudaMemcpyAsync(dst, U.host[b], (size_t)n * rb, cudaMemcpyHostToDevice, c->stream));
    } else {
      CK(cudaMemcpyAsync(U.dev[b], U.host[b], (size_t)n * rb, cudaMemcpyHostToDevice, c->stream));
      CK(launch_q6k_pack(dst, U.dev[b], n, exp_cols, c->stream));
    }
    CK(cudaEventRecord(U.done[b], c->stream));
    U.used[b] = true;
  }
  return 0;
}

static int upload_f32(hakmc_ctx* c, float** dst, const MTensor* t, int n, const std::vector<int>& order) {
  if (!t) { *dst = nullptr; return 0; }
  if (t->type != 0 || (int)t->dims[0] != n || t->nbytes < (size_t)n * 4) {
    set_err("tensor %s: expected %d f32", t->name.c_str(), n);
    return HAKMC_EFORMAT;
  }
  std::vector<float> h(n);
  const float* s = reinterpret_cast<const float*>(t->data);
  for (int i = 0; i < n; i++) h[i] = s[order.empty() ? i : order[i]];
  int e = dalloc(c, (void**)dst, (size_t)n * 4);
  if (e) return e;
  CK(cudaMemcpy(*dst, h.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
  return 0;
}

// Device row 2p+t of head h holds source row h*hd + p + t*hd/2, so the two
// halves of every NeoX rotation pair (src/nn.c:36-41) meet in one chunk.
static std::vector<int> rope_pair_order(int n_heads, int hd) {
  std::vector<int> o((size_t)n_heads * hd);
  for (int h = 0; h < n_heads; h++)
    for (int p = 0; p < hd / 2; p++) {
      o[h * hd + 2 * p] = h * hd + p;
      o[h * hd + 2 * p + 1] = h * hd + p + hd / 2;
    }
  return o;
}

static Seg make_seg(const DevMat& m, int epi, float* out) {
  Seg s = {};
  s.w = m.w;
  s.w_row0 = m.shard_row0;
  s.w_rows = m.shard_rows;
  s.type = m.type;
  s.n_rows = m.rows;
  s.epi = epi;
  s.out = out;
  return s;
}

static void finish_params(PhaseParams& p) {
  p.need_q8 = 0;
  p.need_q6 = 0;
  for (int i = 0; i < p.n_seg; i++) {
    if (p.seg[i].type == W_Q4K) p.need_q8 = 1;
    if (p.seg[i].type == W_Q6K) p.need_q6 = 1;
  }
}

static unsigned long long* g_trace = nullptr;  // set only inside hakmc_trace_phase


enum { PH_QKV = 0, PH_ATTN = 1, PH_WO = 2, PH_FFN = 3, PH_DOWN = 4, PH_LMHEAD = 5 };

// One phase of layer l (l ignored for PH_LMHEAD) as a PhaseDesc. `timing`
// leaves out the step-finalisation side effects of the per-phase lm_head
// kernel, so a phase can be relaunched on its own (and the step program,
// which finalises inside the step kernel, uses it too).
static PhaseDesc make_phase(hakmc_ctx* c, int l, int ph, int n_split, bool timing, int seq = 0) {
  const size_t lstride = (size_t)c->max_seq * c->KV;
  DevLayer& y = c->layers[l < c->L ? l : 0];
  // cache slot `seq`
  float* kc = c->k_cache + ((size_t)seq * c->L + l) * lstride;
  float* vc = c->v_cache + ((size_t)seq * c->L + l) * lstride;
  PhaseDesc d = {};
  d.kind = PK_GEMV;
  PhaseParams& p = d.g;
  switch (ph) {
    case PH_QKV:
      p.n_in = c->D; p.act = ACT_RMS; p.x = c->xb; p.norm_w = y.attn_norm; p.eps = c->eps;
      p.n_seg = 2;
      p.seg[0] = make_seg(y.wqk, EPI_ROPE_QK, c->q);
      p.seg[0].out2 = c->k; p.seg[0].cache = kc; p.seg[0].split = c->D; p.seg[0].bias = y.bqk;
      p.seg[1] = make_seg(y.wv, EPI_V_CACHE, c->v);
      p.seg[1].cache = vc; p.seg[1].bias = y.bv;
      p.rope_cs = c->rope_cs; p.pos_dev = c->pos_dev; p.head_dim = c->hd; p.kv_dim = c->KV;
      break;
    case PH_ATTN: {
      d.kind = PK_ATTN;
      AttnParams& a = d.a;
      a.q = c->q; a.k_cache = kc; a.v_cache = vc; a.out = c->att; a.pos_dev = c->pos_dev;
      a.n_heads = c->H; a.n_kv = c->KVH; a.head_dim = c->hd; a.scale = host_rsqrt_nr((float)c->hd);
      // one scratch: sequences run their steps one after another
      a.part = c->attn_part; a.score_stride = c->max_seq;
      break;
    }
    case PH_WO:
      p.n_in = c->D; p.act = ACT_F32; p.x = c->att;
      p.n_seg = 1;
      p.seg[0] = make_seg(y.wo, EPI_RESID, c->xb);
      break;
    case PH_FFN:
      p.n_in = c->D; p.act = ACT_RMS; p.x = c->xb; p.norm_w = y.ffn_norm; p.eps = c->eps;
      p.n_seg = 1;
      p.seg[0] = make_seg(y.wgu, EPI_SWIGLU, c->hbuf);
      break;
    case PH_DOWN:
      p.n_in = c->F; p.act = ACT_F32; p.x = c->hbuf;
      p.n_seg = 1;
      p.seg[0] = make_seg(y.down, EPI_RESID, c->xb);
      break;
    default:  // final norm + lm_head + argmax (+ step finalisation)
      p.n_in = c->D; p.act = ACT_RMS; p.x = c->xb; p.norm_w = c->out_norm; p.eps = c->eps;
      p.n_seg = 1;
      p.seg[0] = make_seg(c->lm_head, EPI_ARGMAX, c->logits + (size_t)seq * c->V);
      p.argmax_key = c->argmax_key;
      d.skip_forced = 1;
      if (!timing) {
        p.done_counter = c->done_counter;
        p.next_token = c->token_dev; p.token_log = c->token_log; p.step_dev = c->step_dev;
        p.token_log_cap = c->token_log_cap;
        p.pos_inc = c->pos_dev;
      }
      break;
  }
  if (d.kind == PK_GEMV) {
    finish_params(p);
    p.err_flag = c->err_flag;
    p.rsq = c->rsq;
  }
  (void)n_split;
  return d;
}

static cudaError_t enqueue_phase(hakmc_ctx* c, int l, int ph, int n_split, bool timing) {
  PhaseDesc d = make_phase(c, l, ph, n_split, timing);
  if (d.kind == PK_ATTN) return launch_attention(d.a, c->stream, c->pdl);
  d.g.trace = g_trace;
  return launch_phase(d.g, c->num_sms, c->stream, c->pdl);
}

// Enqueue one decode step for sequence 0 on c->stream.
static cudaError_t enqueue_step(hakmc_ctx* c, int n_split) {
  cudaError_t e = launch_embed_q6k(c->xb, c->tok_embd.w, c->token_dev, c->D, c->stream, c->pdl);
  if (e != cudaSuccess) return e;
  for (int l = 0; l < c->run_layers; l++)
    for (int ph = PH_QKV; ph <= PH_DOWN; ph++)
      if ((e = enqueue_phase(c, l, ph, n_split, false)) != cudaSuccess) return e;
  return enqueue_phase(c, 0, PH_LMHEAD, n_split, false);
}

// Key of the captured per-phase step graph: the attention kernel reads the
// position from the device, so one graph serves every position.
static int n_split_for(const hakmc_ctx*, int) { return 1; }

static int get_graph(hakmc_ctx* c, int n_split, cudaGraphExec_t* out) {
  auto it = c->graphs.find(n_split);
  if (it != c->graphs.end()) { *out = it->second; return 0; }
  cudaGraph_t g = nullptr;
  CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  cudaError_t e = enqueue_step(c, n_split);
  cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    set_err("graph capture failed: %s / %s", cudaGetErrorString(e), cudaGetErrorString(e2));
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    return HAKMC_ECUDA;
  }
  cudaGraphExec_t ge = nullptr;
  e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) { set_err("graph instantiate: %s", cudaGetErrorString(e)); return HAKMC_ECUDA; }
  c->graphs[n_split] = ge;
  *out = ge;
  return 0;
}

// Capture (once) every step graph positions [p0, p1) will use, so no capture
// happens between timed launches.
static int ensure_graphs(hakmc_ctx* c, int p0, int p1) {
  for (int p = p0; p < p1 && p < c->max_seq; p++) {
    cudaGraphExec_t g;
    const int r = get_graph(c, n_split_for(c, p), &g);
    if (r) return r;
  }
  return 0;
}

static void drop_graphs(hakmc_ctx* c) {
  for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
  c->graphs.clear();
}

// One step at the host-mirrored position (token already in token_dev).
static int launch_one(hakmc_ctx* c) {
  if (c->pos >= c->max_seq) { set_err("position %d beyond max_seq %d", c->pos, c->max_seq); return HAKMC_ERANGE; }
  cudaGraphExec_t g;
  int r = get_graph(c, n_split_for(c, c->pos), &g);
  if (r) return r;
  CK(cudaGraphLaunch(g, c->stream));
  c->pos++;
  return 0;
}

// Device program of one decode step for run_layers layers (rebuilt when that
// changes) and its shared-memory plan. Phase i of the program has tag index
// i + 1 (0 is the embedding); each phase names the index of the phase whose
// output it reads.
// The step program of sequence `seq` (its exchange vectors, cache slot,
// logits, attention scratch and tickets) for run_layers layers.
static void build_program(hakmc_ctx* c, int seq, std::vector<PhaseDesc>& prog) {
  prog.clear();
  const size_t lo = (size_t)seq * c->ll_words;
  uint64_t* xb0 = c->xb_ll + lo;
  uint64_t* xb1 = c->xb_ll + lo + c->D;
  uint64_t *q_ll = c->q_ll + lo, *k_ll = c->k_ll + lo, *v_ll = c->v_ll + lo, *att_ll = c->att_ll + lo,
           *h_ll = c->h_ll + lo;
  int xb0_src = 0;  // phase that last wrote xb buffer 0 (the embedding first)
  for (int l = 0; l < c->run_layers; l++) {
    const int base = 5 * l + 1;  // tag index of this layer's qkv phase
    PhaseDesc qkv = make_phase(c, l, PH_QKV, 1, true, seq);
    qkv.x_ll = xb0; qkv.x_src = xb0_src;
    qkv.out_ll[0] = q_ll; qkv.out2_ll = k_ll; qkv.out_ll[1] = v_ll;
    PhaseDesc at = make_phase(c, l, PH_ATTN, 1, true, seq);
    at.x_ll = q_ll; at.res_ll = k_ll; at.v_ll = v_ll; at.x_src = base;
    at.out_ll[0] = att_ll; at.layer = l;
    PhaseDesc wo = make_phase(c, l, PH_WO, 1, true, seq);
    wo.x_ll = att_ll; wo.x_src = base + 1;
    wo.res_ll = xb0; wo.res_src = xb0_src; wo.out_ll[0] = xb1;
    PhaseDesc ffn = make_phase(c, l, PH_FFN, 1, true, seq);
    ffn.x_ll = xb1; ffn.x_src = base + 2; ffn.out_ll[0] = h_ll;
    PhaseDesc down = make_phase(c, l, PH_DOWN, 1, true, seq);
    down.x_ll = h_ll; down.x_src = base + 3;
    down.res_ll = xb1; down.res_src = base + 2; down.out_ll[0] = xb0;
    xb0_src = base + 4;
    prog.push_back(qkv); prog.push_back(at); prog.push_back(wo); prog.push_back(ffn); prog.push_back(down);
  }
  PhaseDesc lm = make_phase(c, 0, PH_LMHEAD, 1, true, seq);
  lm.x_ll = xb0; lm.x_src = xb0_src;
  prog.push_back(lm);
}

// Device program of one decode step for run_layers layers (rebuilt when that
// changes) and its shared-memory plan. Phase i of the program has tag index
// i + 1 (0 is the embedding); each phase names the index of the phase whose
// output it reads.
static int ensure_program(hakmc_ctx* c) {
  if (c->prog_layers == c->run_layers) return 0;
  std::vector<PhaseDesc> prog;
  build_program(c, 0, prog);
  StepArgs a = {};
  if (!plan_step(prog.data(), (int)prog.size(), c->num_sms * c->tp_world, a)) {
    set_err("step kernel: shapes do not fit its shared-memory plan");
    return HAKMC_EINVAL;
  }
  {
    // tensor maps of the chunk-streamed segments: two per segment, boxes of
    // st_chunk_rows and st_chunk_rows - 4 rows x one chunk
    std::vector<CUtensorMap> maps;
    std::vector<std::pair<int, int>> where;
    for (size_t ph = 0; ph < prog.size(); ph++) {
      const PhaseDesc& D = prog[ph];
      if (D.kind != PK_GEMV) continue;
      for (int s = 0; s < D.g.n_seg; s++) {
        const int cr = D.st_chunk_rows[s];
        if (!cr) continue;
        const Seg& S = D.g.seg[s];
        const uint64_t rowB = dev_row_bytes(W_Q6K, D.g.n_in / QK);
        CUtensorMap m[2];
        for (int k = 0; k < 2; k++)
          if (!encode_tmap_2d(&m[k], CU_TENSOR_MAP_DATA_TYPE_UINT64, S.w, rowB / 8,
                              (uint64_t)(S.w_rows ? S.w_rows : S.n_rows), rowB,
                              Q6K_CHUNK / 8, (uint32_t)std::max(4, cr - 4 * k))) {
            set_err("step kernel: tensor map of a %d x %d Q6_K matrix rejected", S.n_rows, D.g.n_in);
            return HAKMC_EINVAL;
          }
        maps.push_back(m[0]);
        maps.push_back(m[1]);
        where.push_back({(int)ph, s});
      }
    }
    if (maps.size() > c->tmaps_cap) {
      dfree(c, c->tmaps_dev);
      c->tmaps_dev = nullptr;
      c->tmaps_cap = 0;
      const int r = dalloc(c, (void**)&c->tmaps_dev, maps.size() * sizeof(CUtensorMap));
      if (r) return r;
      c->tmaps_cap = maps.size();
    }
    if (!maps.empty())
      CK(cudaMemcpy(c->tmaps_dev, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
    for (size_t i = 0; i < where.size(); i++)
      prog[where[i].first].st_map[where[i].second] = c->tmaps_dev + 2 * i;
  }
  if ((int)prog.size() > c->prog_cap) {
    void* p = nullptr;
    const int r = dalloc(c, &p, prog.size() * sizeof(PhaseDesc));
    if (r) return r;
    c->prog_dev = (PhaseDesc*)p;
    c->prog_cap = (int)prog.size();
  }
  CK(cudaMemcpy(c->prog_dev, prog.data(), prog.size() * sizeof(PhaseDesc), cudaMemcpyHostToDevice));
  {
    std::vector<SegRange> tab(prog.size() * (size_t)c->num_sms * MAX_SEGS);
    step_ranges(prog.data(), (int)prog.size(), c->num_sms * c->tp_world, c->tp_rank * c->num_sms, c->num_sms,
                tab.data());
    if (tab.size() > c->ranges_cap) {
      void* p = nullptr;
      const int r = dalloc(c, &p, tab.size() * sizeof(SegRange));
      if (r) return r;
      c->ranges_dev = (SegRange*)p;
      c->ranges_cap = tab.size();
    }
    CK(cudaMemcpy(c->ranges_dev, tab.data(), tab.size() * sizeof(SegRange), cudaMemcpyHostToDevice));
  }
  a.prog = c->prog_dev;
  a.ranges = c->ranges_dev;
  a.n_phases = (int)prog.size();
  a.token_dev = c->token_dev;
  a.pos_dev = c->pos_dev;
  a.token_log = c->token_log;
  a.token_log_cap = c->token_log_cap;
  a.keys = c->step_keys;
  a.bar = c->step_bar;
  a.tickets = c->step_tickets;
  a.err_flag = c->err_flag;
  a.tok_embd = c->tok_embd.w;
  a.xb_ll = c->xb_ll;
  a.xb_plain = c->xb;
  a.D = c->D;
  a.n_layers = c->run_layers;
  a.skip_last = 1;  // the program ends with lm_head
  a.head_dim = c->hd;
  c->step = a;
  c->prog_layers = c->run_layers;
  return 0;
}

// n_steps decode steps from the host-mirrored position in one launch of the
// step kernel. Steps 0..n_forced-1 take forced_dev[] as input (else step 0
// takes token_dev); the pick of step j goes to token_log[j - log_base].
static int run_steps(hakmc_ctx* c, int n_steps, int n_forced, const int* forced_dev, int log_base,
                     unsigned long long* trace = nullptr, int trace_k = 0, int seq = 0) {
  if (n_steps <= 0) return 0;
  if (c->pos + n_steps > c->max_seq) { set_err("position %d beyond max_seq %d", c->pos + n_steps, c->max_seq); return HAKMC_ERANGE; }
  int r = ensure_program(c);
  if (r) return r;
  StepArgs a = c->step;
  a.kv_off = (long long)seq * c->L * c->max_seq * c->KV;  // cache layout [seq][layer][max_seq][KV]
  a.n_steps = n_steps;
  a.pos0 = c->pos;
  a.n_forced = n_forced;
  a.forced = forced_dev;
  a.log_base = log_base;
  a.trace = trace;
  a.trace_k = trace_k;
  // tags of this launch: tag_base .. tag_base + n_steps * (n_phases + 1) - 1;
  // before they would wrap, the vectors are cleared and tags restart at 1
  const uint64_t span = (uint64_t)n_steps * (uint64_t)(a.n_phases + 1);
  if ((uint64_t)c->tag_base + span >= 0xFFFFFFF0ull) {
    // peers write into these words without a host round trip: clearing them
    // under tensor parallelism could erase a peer's early write
    if (c->tp_world > 1) { set_err("tag space of the tensor-parallel group used up: recreate the contexts"); return HAKMC_ERANGE; }
    CK(cudaMemsetAsync(c->xb_ll, 0, c->ll_words * 8, c->stream));
    c->tag_base = 1;
  }
  a.tp_rank = c->tp_rank;
  a.tp_world = c->tp_world;
  for (int rr = 0; rr < c->tp_world; rr++)
    for (int x = 0; x < XR_COUNT; x++)
      a.tp_delta[rr][x] = rr == c->tp_rank ? 0
                                           : (long long)((const char*)c->peer_ptr[rr][x] - (const char*)c->xr_ptr[x]);
  a.xbar = c->step_xbar;
  a.xbar_base = c->xbar_base;
  a.tag_base = c->tag_base;
  c->tag_base += (uint32_t)span;
  CK(cudaMemsetAsync(c->step_bar, 0, 4, c->stream));
  CK(cudaMemsetAsync(c->step_tickets, 0, 64 * 4, c->stream));
  CK(cudaMemsetAsync(c->step_keys, 0, 3 * 8, c->stream));
  CK(launch_step(a, c->num_sms, c->stream));
  c->pos += n_steps;
  c->step_ran = true;
  if (c->tp_world > 1) c->xbar_base += (unsigned)n_steps;
  return 0;
}

// After a synchronised call: a kernel whose bounded wait gave up leaves the
// error flag set (and its outputs unusable).
static int check_flag(hakmc_ctx* c) {
  CK(cudaMemcpy(&c->h_pinned[4], c->err_flag, 4, cudaMemcpyDeviceToHost));
  if (c->h_pinned[4]) {
    CK(cudaMemset(c->err_flag, 0, 4));
    set_err("a kernel wait timed out; outputs of this call are invalid");
    return HAKMC_ETIMEOUT;
  }
  return 0;
}

extern "C" void hakmc_destroy(hakmc_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  drop_graphs(c);
  for (int rr = 0; rr < TP_MAX; rr++)
    if (c->peer_ipc[rr])
      for (int x = 0; x < XR_COUNT; x++)
        if (c->peer_ptr[rr][x]) cudaIpcCloseMemHandle(c->peer_ptr[rr][x]);
  drop_bgraphs(c);
  for (void* p : c->allocs) cudaFree(p);
  if (c->h_pinned) cudaFreeHost(c->h_pinned);
  if (c->logits_pinned) cudaFreeHost(c->logits_pinned);
  if (c->ev0) cudaEventDestroy(c->ev0);
  if (c->ev1) cudaEventDestroy(c->ev1);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

static int create_impl(hakmc_ctx* c, const uint8_t* img, size_t size) {
  MImage m;
  int r = parse_mlf2(img, size, m);
  if (r) return r;
  c->L = (int)m.n_layers; c->D = (int)m.d_model; c->H = (int)m.n_heads; c->KVH = (int)m.n_kv;
  c->hd = (int)m.head_dim; c->KV = c->KVH * c->hd; c->F = (int)m.ffn; c->V = (int)m.vocab;
  c->theta = m.theta; c->eps = m.eps; c->tied = (m.flags & 2u) != 0;
  c->run_layers = c->L;
  if (c->D % QK || c->F % QK || c->H % c->KVH || c->H * c->hd != c->D || (c->hd != 64 && c->hd != 128) ||
      c->H / c->KVH > 8 || c->KV % 4) {
    set_err("unsupported shape: d %d heads %d/%d hd %d ffn %d", c->D, c->H, c->KVH, c->hd, c->F);
    return HAKMC_EINVAL;
  }
  auto need = [&](const std::string& n) -> const MTensor* {
    auto it = m.t.find(n);
    if (it == m.t.end()) { set_err("missing tensor %s", n.c_str()); return nullptr; }
    return &it->second;
  };
  auto opt = [&](const std::string& n) -> const MTensor* {
    auto it = m.t.find(n);
    return it == m.t.end() ? nullptr : &it->second;
  };
  CK(cudaSetDevice(c->device));
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, c->device));
  c->num_sms = prop.multiProcessorCount;
  CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  CK(cudaEventCreate(&c->ev0));
  CK(cudaEventCreate(&c->ev1));
  const char* pe = getenv("HAKMC_PDL");
  c->pdl = !(pe && pe[0] == '0');
  const char* se = getenv("HAKMC_STEP");
  c->use_step = !(se && se[0] == '0');
  // weight staging for the uploads below; released when this returns
  UpStage stage;
  struct Unset {
    hakmc_ctx* c;
    ~Unset() { c->up = nullptr; }
  } unset{c};
  CK(stage.open());
  c->up = &stage;

  const MTensor *te = need("token_embd.weight"), *on = need("output_norm.weight");
  if (!te || !on) return HAKMC_EFORMAT;
  const MTensor* ow = c->tied ? te : need("output.weight");
  if (!ow) return HAKMC_EFORMAT;
  std::vector<int> none;
  if (te->type != W_Q6K) { set_err("token_embd: only Q6_K embeddings are supported"); return HAKMC_EFORMAT; }
  if ((r = upload_mat(c, c->tok_embd, *te, c->D, c->V, none))) return r;
  if (c->tied) c->lm_head = c->tok_embd;
  else if ((r = upload_mat(c, c->lm_head, *ow, c->D, c->V, none))) return r;
  if ((r = upload_f32(c, &c->out_norm, on, c->D, none))) return r;

  const std::vector<int> qo = rope_pair_order(c->H, c->hd), ko = rope_pair_order(c->KVH, c->hd);
  std::vector<int> qko(qo);
  for (int i : ko) qko.push_back(c->D + i);
  c->layers.resize(c->L);
  char nm[96];
  for (int l = 0; l < c->L; l++) {
    DevLayer& y = c->layers[l];
    auto T = [&](const char* s) { snprintf(nm, sizeof nm, "blk.%d.%s", l, s); return std::string(nm); };
    const MTensor *an = need(T("attn_norm.weight")), *fn = need(T("ffn_norm.weight")),
                  *wq = need(T("attn_q.weight")), *wk = need(T("attn_k.weight")),
                  *wv = need(T("attn_v.weight")), *wo = need(T("attn_output.weight")),
                  *wg = need(T("ffn_gate.weight")), *wu = need(T("ffn_up.weight")),
                  *wd = need(T("ffn_down.weight"));
    if (!an || !fn || !wq || !wk || !wv || !wo || !wg || !wu || !wd) return HAKMC_EFORMAT;
    const MTensor *bq = opt(T("attn_q.bias")), *bk = opt(T("attn_k.bias")), *bv = opt(T("attn_v.bias"));
    if ((r = upload_f32(c, &y.attn_norm, an, c->D, none))) return r;
    if ((r = upload_f32(c, &y.ffn_norm, fn, c->D, none))) return r;
    // q and k rows share one Q4_K/Q6_K segment: concatenate, then pair-order
    if (wq->type != wk->type) { set_err("attn_q/attn_k types differ"); return HAKMC_EFORMAT; }
    {
      MTensor cat = *wq;
      const size_t rb = row_bytes(wq->type, c->D);
      std::vector<uint8_t> buf(rb * (size_t)(c->D + c->KV));
      if (wq->nbytes < rb * c->D || wk->nbytes < rb * c->KV || (int)wk->dims[1] != c->KV ||
          (int)wk->dims[0] != c->D) {
        set_err("attn_q/attn_k shape mismatch");
        return HAKMC_EFORMAT;
      }
      memcpy(buf.data(), wq->data, rb * c->D);
      memcpy(buf.data() + rb * c->D, wk->data, rb * c->KV);
      cat.data = buf.data(); cat.nbytes = buf.size(); cat.dims[1] = (uint64_t)(c->D + c->KV);
      if ((r = upload_mat(c, y.wqk, cat, c->D, c->D + c->KV, qko))) return r;
    }
    if (bq && bk) {
      std::vector<float> b((size_t)(c->D + c->KV));
      if (bq->type || bk->type || (int)bq->dims[0] != c->D || (int)bk->dims[0] != c->KV) {
        set_err("q/k bias shape"); return HAKMC_EFORMAT;
      }
      for (int i = 0; i < c->D + c->KV; i++)
        b[i] = qko[i] < c->D ? reinterpret_cast<const float*>(bq->data)[qko[i]]
                             : reinterpret_cast<const float*>(bk->data)[qko[i] - c->D];
      if ((r = dalloc(c, (void**)&y.bqk, b.size() * 4))) return r;
      CK(cudaMemcpy(y.bqk, b.data(), b.size() * 4, cudaMemcpyHostToDevice));
    } else if (bq || bk) {
      set_err("layer %d: only one of attn_q/attn_k bias present", l);
      return HAKMC_EFORMAT;
    } else {
      y.bqk = nullptr;
    }
    if ((r = upload_mat(c, y.wv, *wv, c->D, c->KV, none))) return r;
    if ((r = upload_f32(c, &y.bv, bv, c->KV, none))) return r;
    if ((r = upload_mat(c, y.wo, *wo, c->D, c->D, none))) return r;
    if ((r = upload_mat(c, y.wgu, *wg, c->D, c->F, none, wu))) return r;
    if ((r = upload_mat(c, y.down, *wd, c->F, c->D, none))) return r;
  }

  // KV cache and activations
  const size_t kv = (size_t)c->max_batch * c->L * c->max_seq * c->KV;
  if ((r = dalloc(c, (void**)&c->k_cache, kv * 4))) return r;
  if ((r = dalloc(c, (void**)&c->v_cache, kv * 4))) return r;
  CK(cudaMemset(c->k_cache, 0, kv * 4));
  CK(cudaMemset(c->v_cache, 0, kv * 4));
  const int B = c->max_batch;
  if ((r = dalloc(c, (void**)&c->xb, (size_t)B * c->D * 4))) return r;
  if ((r = dalloc(c, (void**)&c->q, (size_t)B * c->D * 4))) return r;
  if ((r = dalloc(c, (void**)&c->k, (size_t)B * c->KV * 4))) return r;
  if ((r = dalloc(c, (void**)&c->v, (size_t)B * c->KV * 4))) return r;
  if ((r = dalloc(c, (void**)&c->att, (size_t)B * c->D * 4))) return r;
  if ((r = dalloc(c, (void**)&c->hbuf, (size_t)B * c->F * 4))) return r;
  if ((r = dalloc(c, (void**)&c->logits, (size_t)B * c->V * 4))) return r;
  // attention score rows: one per (query head, dimension slice) unit
  c->attn_part_floats = attention_scratch_floats(c->H, c->hd, c->max_seq);
  if ((r = dalloc(c, (void**)&c->attn_part, c->attn_part_floats * 4))) return r;
  if (!(c->rsq = rsqrt_table_device(c->device))) {
    set_err("rsqrtss table: this host's estimate is not a function of exponent parity and 10 mantissa bits");
    return HAKMC_EINVAL;
  }
  // [sequence] plus a save slot (forward_batch, TOKEN_SAVE)
  if ((r = dalloc(c, (void**)&c->token_dev, 4 * std::max(4 * B, TOKEN_SAVE + 1)))) return r;
  if ((r = dalloc(c, (void**)&c->pos_dev, 16 * B))) return r;
  if ((r = dalloc(c, (void**)&c->step_dev, 16))) return r;
  c->token_log_cap = c->max_seq + 8;
  if ((r = dalloc(c, (void**)&c->token_log, (size_t)c->token_log_cap * 4))) return r;
  if ((r = dalloc(c, (void**)&c->argmax_key, 8 * B))) return r;
  if ((r = dalloc(c, (void**)&c->done_counter, 4 * B))) return r;
  if ((r = dalloc(c, (void**)&c->err_flag, 16))) return r;
  if ((r = dalloc(c, (void**)&c->step_bar, 32))) return r;
  if ((r = dalloc(c, (void**)&c->step_keys, 32))) return r;
  if ((r = dalloc(c, (void**)&c->step_tickets, 64 * 4))) return r;
  if ((r = dalloc(c, (void**)&c->step_xbar, 16))) return r;
  CK(cudaMemset(c->step_xbar, 0, 16));
  CK(cudaMemset(c->step_bar, 0, 32));
  CK(cudaMemset(c->step_keys, 0, 32));
  CK(cudaMemset(c->step_tickets, 0, 64 * 4));
  {
    // exchange vectors, 16-byte aligned pieces of one allocation
    auto up2 = [](size_t n) { return (n + 1) & ~(size_t)1; };
    const size_t nD = up2(c->D), nKV = up2(c->KV), nF = up2(c->F);
    c->ll_words = 2 * nD + nD + 2 * nKV + nD + nF;
    if ((r = dalloc(c, (void**)&c->xb_ll, c->ll_words * 8))) return r;
    CK(cudaMemset(c->xb_ll, 0, c->ll_words * 8));
    c->q_ll = c->xb_ll + 2 * nD;
    c->k_ll = c->q_ll + nD;
    c->v_ll = c->k_ll + nKV;
    c->att_ll = c->v_ll + nKV;
    c->h_ll = c->att_ll + nD;
  }
  c->xr_ptr[XR_LL] = c->xb_ll;          c->xr_size[XR_LL] = c->ll_words * 8;
  c->xr_ptr[XR_KCACHE] = c->k_cache;    c->xr_size[XR_KCACHE] = kv * 4;
  c->xr_ptr[XR_VCACHE] = c->v_cache;    c->xr_size[XR_VCACHE] = kv * 4;
  c->xr_ptr[XR_LOGITS] = c->logits;     c->xr_size[XR_LOGITS] = (size_t)B * c->V * 4;
  c->xr_ptr[XR_KEYS] = c->step_keys;    c->xr_size[XR_KEYS] = 32;
  c->xr_ptr[XR_XBAR] = c->step_xbar;    c->xr_size[XR_XBAR] = 16;
  CK(cudaMemset(c->err_flag, 0, 16));
  CK(cudaMemset(c->token_dev, 0, 16 * B));
  CK(cudaMemset(c->pos_dev, 0, 16 * B));
  CK(cudaMemset(c->step_dev, 0, 16));
  CK(cudaMemset(c->argmax_key, 0, 8 * B));
  CK(cudaMemset(c->done_counter, 0, 4 * B));

  // RoPE table as the reference's build computes it (src/nn.c:35-37 through
  // glibc's vector powf/cosf/sinf: hakm_host_rope_row)
  {
    const int half = c->hd / 2;
    std::vector<float> cs((size_t)c->max_seq * half * 2);
    for (int p = 0; p < c->max_seq; p++) hakm_host_rope_row(cs.data() + (size_t)p * half * 2, c->hd, p, c->theta);
    if ((r = dalloc(c, (void**)&c->rope_cs, cs.size() * 4))) return r;
    CK(cudaMemcpy(c->rope_cs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  }
  CK(cudaMallocHost((void**)&c->h_pinned, 64));
  CK(cudaMallocHost((void**)&c->logits_pinned, (size_t)c->V * 4));
  CK(cudaDeviceSynchronize());
  return 0;
}

extern "C" hakmc_ctx* hakmc_create(const void* image, size_t size, int max_seq, int max_batch, int device) {
  if (max_seq <= 0 || max_batch <= 0) { set_err("max_seq and max_batch must be positive"); return nullptr; }
  hakmc_ctx* c = new hakmc_ctx();
  c->device = device;
  c->max_seq = max_seq;
  c->max_batch = max_batch;
  if (create_impl(c, (const uint8_t*)image, size) != 0) {
    std::string keep = g_err;
    hakmc_destroy(c);
    g_err = keep;
    return nullptr;
  }
  return c;
}

extern "C" void hakmc_reset(hakmc_ctx* c) {
  if (!c) return;
  hakmc_set_pos(c, 0);
}

extern "C" int hakmc_pos(const hakmc_ctx* c) { return c ? c->pos : -1; }
extern "C" int hakmc_vocab(const hakmc_ctx* c) { return c ? c->V : -1; }
extern "C" int hakmc_dim(const hakmc_ctx* c) { return c ? c->D : -1; }
extern "C" int hakmc_n_layers(const hakmc_ctx* c) { return c ? c->L : -1; }
extern "C" float hakmc_last_device_ms(const hakmc_ctx* c) { return c ? c->last_ms : -1.f; }

extern "C" int hakmc_set_pos(hakmc_ctx* c, int pos) {
  if (!c || pos < 0 || pos > c->max_seq) { set_err("bad position"); return HAKMC_EINVAL; }
  CK(cudaSetDevice(c->device));
  c->h_pinned[2] = pos;
  CK(cudaMemcpyAsync(c->pos_dev, &c->h_pinned[2], 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  c->pos = pos;
  return 0;
}

extern "C" int hakmc_set_layers(hakmc_ctx* c, int n) {
  if (!c) return HAKMC_EINVAL;
  const int nl = (n < 0 || n > c->L) ? c->L : n;
  if (nl != c->run_layers) {
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    drop_graphs(c);
    c->run_layers = nl;
  }
  return 0;
}

extern "C" int hakmc_forward(hakmc_ctx* c, int token, float* logits, int* argmax) {
  if (!c) return HAKMC_EINVAL;
  if (token < 0 || token >= c->V) { set_err("token %d out of range", token); return HAKMC_EINVAL; }
  CK(cudaSetDevice(c->device));
  c->h_pinned[0] = token;
  CK(cudaEventRecord(c->ev0, c->stream));
  CK(cudaMemcpyAsync(c->token_dev, &c->h_pinned[0], 4, cudaMemcpyHostToDevice, c->stream));
  int r = c->use_step ? run_steps(c, 1, 1, c->token_dev, 0) : launch_one(c);
  if (r) return r;
  CK(cudaMemcpyAsync(&c->h_pinned[1], c->token_dev, 4, cudaMemcpyDeviceToHost, c->stream));
  if (logits) CK(cudaMemcpyAsync(c->logits_pinned, c->logits, (size_t)c->V * 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaEventRecord(c->ev1, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  CK(cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1));
  if ((r = check_flag(c))) return r;
  if (argmax) *argmax = c->h_pinned[1];
  if (logits) memcpy(logits, c->logits_pinned, (size_t)c->V * 4);
  return 0;
}

extern "C" int hakmc_generate(hakmc_ctx* c, const int* prompt, int n_prompt, int n_gen, int* out) {
  if (!c || !prompt || n_prompt <= 0 || n_gen < 0 || (n_gen > 0 && !out)) return HAKMC_EINVAL;
  if (c->pos + n_prompt + n_gen - 1 > c->max_seq) { set_err("sequence exceeds max_seq"); return HAKMC_ERANGE; }
  if (c->pos + n_prompt + n_gen > c->token_log_cap) { set_err("token log too small"); return HAKMC_ERANGE; }
  for (int i = 0; i < n_prompt; i++)
    if (prompt[i] < 0 || prompt[i] >= c->V) { set_err("prompt token out of range"); return HAKMC_EINVAL; }
  CK(cudaSetDevice(c->device));
  if (n_prompt > c->prompt_cap) {
    void* p = nullptr;
    int r = dalloc(c, &p, (size_t)n_prompt * 4);
    if (r) return r;
    c->prompt_dev = (int*)p;
    c->prompt_cap = n_prompt;
  }
  if (!c->use_step) {
    const int r = ensure_graphs(c, c->pos, c->pos + n_prompt + n_gen);
    if (r) return r;
  }
  std::vector<int> pp(prompt, prompt + n_prompt);
  CK(cudaMemcpyAsync(c->prompt_dev, pp.data(), (size_t)n_prompt * 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemsetAsync(c->step_dev, 0, 4, c->stream));
  CK(cudaEventRecord(c->ev0, c->stream));
  int log_off = n_prompt - 1;  // token_log index of the first generated token
  if (c->use_step) {
    // prompt and generation in one launch: the pick of the last prompt step
    // is the first generated token
    const int r = run_steps(c, n_prompt + (n_gen > 0 ? n_gen : 1) - 1, n_prompt, c->prompt_dev, n_prompt - 1);
    if (r) return r;
    log_off = 0;
  } else {
    for (int i = 0; i < n_prompt; i++) {
      CK(cudaMemcpyAsync(c->token_dev, c->prompt_dev + i, 4, cudaMemcpyDeviceToDevice, c->stream));
      int r = launch_one(c);
      if (r) return r;
    }
    for (int g = 1; g < n_gen; g++) {
      int r = launch_one(c);
      if (r) return r;
    }
  }
  CK(cudaEventRecord(c->ev1, c->stream));
  if (n_gen > 0)
    CK(cudaMemcpyAsync(out, c->token_log + log_off, (size_t)n_gen * 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  CK(cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1));
  return check_flag(c);
}

extern "C" int hakmc_prefill(hakmc_ctx* c, const int* tokens, int n, float* logits, int* argmax) {
  if (!c || !tokens || n <= 0) { set_err("prefill: need at least one token"); return HAKMC_EINVAL; }
  if (c->pos + n > c->max_seq) { set_err("prefill: sequence exceeds max_seq"); return HAKMC_ERANGE; }
  for (int i = 0; i < n; i++)
    if (tokens[i] < 0 || tokens[i] >= c->V) { set_err("prefill: token %d out of range", tokens[i]); return HAKMC_EINVAL; }
  CK(cudaSetDevice(c->device));
  if (n > c->prompt_cap) {
    void* p = nullptr;
    const int r = dalloc(c, &p, (size_t)n * 4);
    if (r) return r;
    c->prompt_dev = (int*)p;
    c->prompt_cap = n;
  }
  std::vector<int> pp(tokens, tokens + n);
  CK(cudaMemcpyAsync(c->prompt_dev, pp.data(), (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaEventRecord(c->ev0, c->stream));
  if (c->use_step) {
    const int r = run_steps(c, n, n, c->prompt_dev, n - 1);
    if (r) return r;
  } else {
    for (int i = 0; i < n; i++) {
      CK(cudaMemcpyAsync(c->token_dev, c->prompt_dev + i, 4, cudaMemcpyDeviceToDevice, c->stream));
      const int r = launch_one(c);
      if (r) return r;
    }
  }
  CK(cudaEventRecord(c->ev1, c->stream));
  CK(cudaMemcpyAsync(&c->h_pinned[1], c->token_dev, 4, cudaMemcpyDeviceToHost, c->stream));
  if (logits) CK(cudaMemcpyAsync(c->logits_pinned, c->logits, (size_t)c->V * 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  CK(cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1));
  const int r = check_flag(c);
  if (r) return r;
  if (argmax) *argmax = c->h_pinned[1];
  if (logits) memcpy(logits, c->logits_pinned, (size_t)c->V * 4);
  return 0;
}

// ------------------------------------------------------------ batched prefill
//
// The rows of a prompt chunk go through every layer together, each weight
// byte read once per chunk (hakm_rows.cu, hakm_mma.cu, hakm_prefill.cu):
// Q4_K matmuls on the tensor cores, Q6_K matmuls as fp32 lane chains,
// attention of each row over the cache, which the chunk's own K/V rows enter
// first. Every kernel keeps the reference's roundings, so each row equals
// what hakm_forward gives at its position bit for bit. Then the last row's
// final norm, lm_head and argmax run as in a decode step.

constexpr int PF_ROWS_DEFAULT = 1024;

// Buffers for chunks of `rows` rows (regrown when a larger chunk comes).
static int pf_ensure(hakmc_ctx* c, int rows) {
  if (rows <= c->pf_rows) return 0;
  float** fb[] = {&c->pf_x, &c->pf_xn, &c->pf_qk, &c->pf_v, &c->pf_q, &c->pf_att, &c->pf_gu, &c->pf_h, &c->pf_tmp,
                  &c->pf_xs};
  for (float** b : fb) { dfree(c, *b); *b = nullptr; }
  dfree(c, c->pf_xq);
  c->pf_xq = nullptr;
  c->pf_rows = 0;
  const size_t M = (size_t)rows, K = (size_t)std::max(c->D, c->F);
  const size_t n[] = {M * c->D, M * c->D, M * (c->D + c->KV), M * c->KV, M * c->D, M * c->D, M * 2 * c->F,
                      M * c->F, M * c->D, M * K / 32};
  for (size_t i = 0; i < sizeof(n) / sizeof(n[0]); i++) {
    const int r = dalloc(c, (void**)fb[i], n[i] * 4);
    if (r) return r;
  }
  const int r = dalloc(c, (void**)&c->pf_xq, M * K);
  if (r) return r;
  c->pf_rows = rows;
  return 0;
}

// out[M][W.rows] (+)= W x (+ bias) for M rows: Q4_K on the q8 codes (xq,
// xs) on the tensor cores, Q6_K on the fp32 rows xn. Accumulating Q4_K
// products go through pf_tmp, then one add (the reference's order: the
// product, then +=).
static cudaError_t pf_matmul(hakmc_ctx* c, float* out, const DevMat& W, const float* xn, const int8_t* xq,
                             const float* xs, const float* bias, int M, bool accumulate) {
  if (W.type == W_Q6K) return launch_rx_q6k_gemm(out, W.w, xn, bias, W.rows, W.cols, M, accumulate, c->stream);
  float* dst = accumulate ? c->pf_tmp : out;
  cudaError_t e = launch_q4k_mma(dst, W.w, xq, xs, bias, W.rows, W.cols, M, c->err_flag, c->num_sms, c->stream);
  if (e != cudaSuccess || !accumulate) return e;
  return launch_pf_add(out, c->pf_tmp, (size_t)M * W.rows, c->stream);
}

// The layers for M rows already embedded in pf_x. Row r is at position
// row_pos[r] with its cache slot_stride floats after row r-1's, or (row_pos
// null) at pos0 + r of sequence 0; n_max >= every row's position + 1.
static cudaError_t pf_layers(hakmc_ctx* c, int M, int pos0, const int* row_pos, size_t slot_stride, int n_max) {
  const int D = c->D, KV = c->KV, F = c->F;
  const size_t lstride = (size_t)c->max_seq * KV;
  const float scale = host_rsqrt_nr((float)c->hd);
  cudaStream_t s = c->stream;
  cudaError_t e = cudaSuccess;
  for (int l = 0; l < c->run_layers && e == cudaSuccess; l++) {
    const DevLayer& y = c->layers[l];
    float* kc = c->k_cache + (size_t)l * lstride;
    float* vc = c->v_cache + (size_t)l * lstride;
    // attention block (src/model.c:102-146)
    if ((e = launch_rx_norm_quant(c->pf_x, y.attn_norm, M, D, c->eps, c->rsq, c->pf_xn, c->pf_xq, c->pf_xs, s)))
      break;
    if ((e = pf_matmul(c, c->pf_qk, y.wqk, c->pf_xn, c->pf_xq, c->pf_xs, y.bqk, M, false))) break;
    if ((e = pf_matmul(c, c->pf_v, y.wv, c->pf_xn, c->pf_xq, c->pf_xs, y.bv, M, false))) break;
    if ((e = launch_pf_rope_kv(c->pf_qk, c->pf_v, c->pf_q, kc, vc, c->rope_cs, M, pos0, row_pos, slot_stride, D, KV,
                               c->hd, s)))
      break;
    if ((e = launch_rx_attention(c->pf_att, c->pf_q, kc, vc, M, pos0, row_pos, n_max, slot_stride, c->H, c->KVH,
                                 c->hd, scale, s)))
      break;
    if (y.wo.type == W_Q4K && (e = launch_quantize_q8(c->pf_att, M * D, c->pf_xq, c->pf_xs, s))) break;
    if ((e = pf_matmul(c, c->pf_x, y.wo, c->pf_att, c->pf_xq, c->pf_xs, nullptr, M, true))) break;
    // feed-forward block (src/model.c:148-156)
    if ((e = launch_rx_norm_quant(c->pf_x, y.ffn_norm, M, D, c->eps, c->rsq, c->pf_xn, c->pf_xq, c->pf_xs, s)))
      break;
    if ((e = pf_matmul(c, c->pf_gu, y.wgu, c->pf_xn, c->pf_xq, c->pf_xs, nullptr, M, false))) break;
    if ((e = launch_rx_swiglu(c->pf_h, c->pf_gu, M, F, s))) break;
    if (y.down.type == W_Q4K && (e = launch_quantize_q8(c->pf_h, M * F, c->pf_xq, c->pf_xs, s))) break;
    e = pf_matmul(c, c->pf_x, y.down, c->pf_h, c->pf_xq, c->pf_xs, nullptr, M, true);
  }
  return e;
}

// One chunk: rows tokens_dev[0..M) at positions pos0.. of sequence 0 through
// run_layers layers; leaves the residual rows in pf_x.
static cudaError_t pf_chunk(hakmc_ctx* c, const int* tokens_dev, int M, int pos0) {
  const cudaError_t e = launch_pf_embed(c->pf_x, c->tok_embd.w, tokens_dev, M, c->D, c->stream);
  return e != cudaSuccess ? e : pf_layers(c, M, pos0, nullptr, 0, pos0 + M);
}

extern "C" int hakmc_prefill_batched(hakmc_ctx* c, const int* tokens, int n, int chunk_rows, float* logits,
                                     int* argmax) {
  if (!c || !tokens || n <= 0) { set_err("prefill: need at least one token"); return HAKMC_EINVAL; }
  if (c->tp_world > 1) return hakmc_prefill(c, tokens, n, logits, argmax);
  if (c->pos + n > c->max_seq) { set_err("prefill: sequence exceeds max_seq"); return HAKMC_ERANGE; }
  for (int i = 0; i < n; i++)
    if (tokens[i] < 0 || tokens[i] >= c->V) { set_err("prefill: token %d out of range", tokens[i]); return HAKMC_EINVAL; }
  // the batched attention keeps a row's scores in shared memory
  if (rx_attention_smem_bytes(c->hd, c->pos + n) > RX_ATTN_SMEM_MAX) return hakmc_prefill(c, tokens, n, logits, argmax);
  CK(cudaSetDevice(c->device));
  const int rows = std::min(n, chunk_rows > 0 ? chunk_rows : PF_ROWS_DEFAULT);
  int r = pf_ensure(c, rows);
  if (r) return r;
  if (n > c->prompt_cap) {
    void* p = nullptr;
    r = dalloc(c, &p, (size_t)n * 4);
    if (r) return r;
    dfree(c, c->prompt_dev);
    c->prompt_dev = (int*)p;
    c->prompt_cap = n;
  }
  std::vector<int> pp(tokens, tokens + n);
  CK(cudaMemcpyAsync(c->prompt_dev, pp.data(), (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaEventRecord(c->ev0, c->stream));
  int last = 0;
  for (int i = 0; i < n; i += rows) {
    const int M = std::min(rows, n - i);
    CK(pf_chunk(c, c->prompt_dev + i, M, c->pos + i));
    last = M;
  }
  // the last row's final norm + lm_head + argmax, as a decode step ends:
  // the residual row goes to xb, the position word to that row's position
  // (the lm_head kernel moves it on by one and leaves the pick in token_dev)
  CK(cudaMemcpyAsync(c->xb, c->pf_x + (size_t)(last - 1) * c->D, (size_t)c->D * 4, cudaMemcpyDeviceToDevice,
                     c->stream));
  c->h_pinned[2] = c->pos + n - 1;
  CK(cudaMemcpyAsync(c->pos_dev, &c->h_pinned[2], 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemsetAsync(c->step_dev, 0, 4, c->stream));
  CK(enqueue_phase(c, 0, PH_LMHEAD, 1, false));
  CK(cudaEventRecord(c->ev1, c->stream));
  CK(cudaMemcpyAsync(&c->h_pinned[1], c->token_dev, 4, cudaMemcpyDeviceToHost, c->stream));
  if (logits) CK(cudaMemcpyAsync(c->logits_pinned, c->logits, (size_t)c->V * 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  CK(cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1));
  c->pos += n;
  c->step_ran = false;
  r = check_flag(c);
  if (r) return r;
  if (argmax) *argmax = c->h_pinned[1];
  if (logits) memcpy(logits, c->logits_pinned, (size_t)c->V * 4);
  return 0;
}

extern "C" void hakmc_free(hakmc_ctx* c) { hakmc_destroy(c); }

extern "C" int hakmc_decode(hakmc_ctx* c, int n_steps, int* out) {
  if (!c || n_steps < 0) return HAKMC_EINVAL;
  if (c->pos + n_steps > c->max_seq) { set_err("sequence exceeds max_seq"); return HAKMC_ERANGE; }
  if (n_steps > c->token_log_cap) { set_err("token log too small"); return HAKMC_ERANGE; }
  CK(cudaSetDevice(c->device));
  if (c->use_step) {
    const int r = ensure_program(c);
    if (r) return r;
  } else {
    const int r = ensure_graphs(c, c->pos, c->pos + n_steps);
    if (r) return r;
  }
  // token_log[i] records the argmax of step i, i.e. the input of step i+1; the
  // first input is the argmax already waiting in token_dev
  CK(cudaMemsetAsync(c->step_dev, 0, 4, c->stream));
  if (out && n_steps > 0) CK(cudaMemcpyAsync(out, c->token_dev, 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaEventRecord(c->ev0, c->stream));
  if (c->use_step) {
    const int r = run_steps(c, n_steps, 0, nullptr, 0);
    if (r) return r;
  } else {
    for (int i = 0; i < n_steps; i++) {
      int r = launch_one(c);
      if (r) return r;
    }
  }
  CK(cudaEventRecord(c->ev1, c->stream));
  if (out && n_steps > 1)
    CK(cudaMemcpyAsync(out + 1, c->token_log, (size_t)(n_steps - 1) * 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  CK(cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1));
  return check_flag(c);
}

extern "C" int hakmc_time_phase(hakmc_ctx* c, int phase, int iters, float* avg_ms) {
  if (!c || phase < 0 || phase > PH_LMHEAD || iters <= 0 || !avg_ms) return HAKMC_EINVAL;
  if (c->tp_world > 1) { set_err("time_phase: one GPU only (tensor-parallel weights are shards)"); return HAKMC_EINVAL; }
  CK(cudaSetDevice(c->device));
  const int ns = n_split_for(c, c->pos < c->max_seq ? c->pos : c->max_seq - 1);
  for (int i = 0; i < 3; i++) CK(enqueue_phase(c, i % c->L, phase, ns, true));  // warm-up
  CK(cudaEventRecord(c->ev0, c->stream));
  for (int i = 0; i < iters; i++) CK(enqueue_phase(c, i % c->L, phase, ns, true));
  CK(cudaEventRecord(c->ev1, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  float ms = 0.f;
  CK(cudaEventElapsedTime(&ms, c->ev0, c->ev1));
  *avg_ms = ms / iters;
  return 0;
}

extern "C" int hakmc_trace_phase(hakmc_ctx* c, int phase, int layer, unsigned long long* stamps, int max_ctas) {
  if (c && c->tp_world > 1) { set_err("trace_phase: one GPU only (tensor-parallel weights are shards)"); return HAKMC_EINVAL; }
  if (!c || phase < 0 || phase > PH_LMHEAD || phase == PH_ATTN || !stamps || layer < 0 || layer >= c->L)
    return HAKMC_EINVAL;
  CK(cudaSetDevice(c->device));
  const size_t n = (size_t)max_ctas * 8;
  unsigned long long* d = nullptr;
  CK(cudaMalloc(&d, n * 8));
  CK(cudaMemset(d, 0, n * 8));
  const int ns = n_split_for(c, c->pos < c->max_seq ? c->pos : c->max_seq - 1);
  g_trace = d;
  cudaError_t e = enqueue_phase(c, layer, phase, ns, true);
  g_trace = nullptr;
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess) e = cudaMemcpy(stamps, d, n * 8, cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) { set_err("trace: %s", cudaGetErrorString(e)); return HAKMC_ECUDA; }
  return max_ctas < c->num_sms ? max_ctas : c->num_sms;
}

// ------------------------------------------------------------ tensor parallelism

namespace {
struct TpHandle {
  uint32_t magic, version;
  int32_t pid, device;
  int32_t vocab, dim, layers, max_seq, max_batch, pad;
  uint64_t size[XR_COUNT];
  uint64_t ptr[XR_COUNT];                // for ranks in the same process
  cudaIpcMemHandle_t ipc[XR_COUNT];      // for ranks in other processes
};
constexpr uint32_t TP_MAGIC = 0x48414b54u;  // "HAKT"
}  // namespace

extern "C" size_t hakmc_tp_handle_bytes(void) { return sizeof(TpHandle); }

extern "C" int hakmc_tp_export(hakmc_ctx* c, void* handle) {
  if (!c || !handle) return HAKMC_EINVAL;
  CK(cudaSetDevice(c->device));
  TpHandle h;
  memset(&h, 0, sizeof h);
  h.magic = TP_MAGIC; h.version = 1; h.pid = (int32_t)getpid(); h.device = c->device;
  h.vocab = c->V; h.dim = c->D; h.layers = c->L; h.max_seq = c->max_seq; h.max_batch = c->max_batch;
  for (int x = 0; x < XR_COUNT; x++) {
    h.size[x] = c->xr_size[x];
    h.ptr[x] = (uint64_t)(uintptr_t)c->xr_ptr[x];
    CK(cudaIpcGetMemHandle(&h.ipc[x], c->xr_ptr[x]));
  }
  memcpy(handle, &h, sizeof h);
  return 0;
}

// Tensor parallelism: keep only this GPU's rows of every matrix the step
// program splits (the lm_head too unless it is the embedding, which every
// token needs whole). A GPU's rows of a segment are the ranges of its CTAs,
// which run on cyclically (the split of each segment is rotated), so they
// are kept from the first CTA's first row on, wrapping past the last row.
static int shard_weights(hakmc_ctx* c) {
  const int keep = c->run_layers;
  c->run_layers = c->L;
  std::vector<PhaseDesc> prog;
  build_program(c, 0, prog);
  c->run_layers = keep;
  const int ns = c->num_sms;
  std::vector<SegRange> tab(prog.size() * (size_t)ns * MAX_SEGS);
  step_ranges(prog.data(), (int)prog.size(), ns * c->tp_world, c->tp_rank * ns, ns, tab.data());
  std::vector<DevMat*> mats;
  for (int l = 0; l < c->L; l++) {
    DevLayer& y = c->layers[l];
    for (DevMat* m : {&y.wqk, &y.wv, &y.wo, &y.wgu, &y.down}) mats.push_back(m);
  }
  if (!c->tied) mats.push_back(&c->lm_head);
  for (DevMat* m : mats) {
    int ph = -1, sg = -1;
    for (size_t i = 0; i < prog.size() && ph < 0; i++)
      if (prog[i].kind == PK_GEMV)
        for (int s = 0; s < prog[i].g.n_seg; s++)
          if (prog[i].g.seg[s].w == m->w) { ph = (int)i; sg = s; break; }
    if (ph < 0) continue;
    const int n = m->rows;
    int lo = -1, owned = 0, next = -1;
    for (int lc = 0; lc < ns; lc++) {
      const SegRange& r = tab[((size_t)ph * ns + lc) * MAX_SEGS + sg];
      if (r.row1 <= r.row0) continue;
      if (lo < 0) lo = r.row0;
      else if (r.row0 != next % n) { set_err("tp_connect: rows of a matrix are not contiguous"); return HAKMC_EINVAL; }
      owned += r.row1 - r.row0;
      next = r.row1;
    }
    if (lo < 0 || owned >= n) continue;
    const size_t rowB = dev_row_bytes(m->type, m->cols / QK);
    uint8_t* w = nullptr;
    int e = dalloc(c, (void**)&w, (size_t)owned * rowB);
    if (e) return e;
    const int first = std::min(owned, n - lo);
    CK(cudaMemcpy(w, m->w + (size_t)lo * rowB, (size_t)first * rowB, cudaMemcpyDeviceToDevice));
    if (owned > first) CK(cudaMemcpy(w + (size_t)first * rowB, m->w, (size_t)(owned - first) * rowB,
                                     cudaMemcpyDeviceToDevice));
    dfree(c, m->w);
    m->w = w;
    m->shard_row0 = lo;
    m->shard_rows = owned;
  }
  return 0;
}

extern "C" int hakmc_tp_connect(hakmc_ctx* c, int rank, int world, const void* handles) {
  if (!c || !handles || world < 1 || world > TP_MAX || rank < 0 || rank >= world) {
    set_err("tp_connect: world must be 1..%d and rank within it", TP_MAX);
    return HAKMC_EINVAL;
  }
  if (!c->use_step) { set_err("tp_connect: tensor parallelism needs the step kernel (HAKMC_STEP unset)"); return HAKMC_EINVAL; }
  if (c->tp_world > 1) { set_err("tp_connect: already connected"); return HAKMC_EINVAL; }
  CK(cudaSetDevice(c->device));
  const TpHandle* hs = static_cast<const TpHandle*>(handles);
  for (int rr = 0; rr < world; rr++) {
    const TpHandle& h = hs[rr];
    if (h.magic != TP_MAGIC || h.version != 1 || h.vocab != c->V || h.dim != c->D || h.layers != c->L ||
        h.max_seq != c->max_seq || h.max_batch != c->max_batch) {
      set_err("tp_connect: rank %d's context differs (model, max_seq or max_batch)", rr);
      return HAKMC_EINVAL;
    }
    for (int x = 0; x < XR_COUNT; x++)
      if (h.size[x] != c->xr_size[x]) { set_err("tp_connect: rank %d's regions differ in size", rr); return HAKMC_EINVAL; }
  }
  if (hs[rank].pid != (int32_t)getpid() || hs[rank].device != c->device ||
      hs[rank].ptr[XR_LL] != (uint64_t)(uintptr_t)c->xr_ptr[XR_LL]) {
    set_err("tp_connect: handle %d is not this context's", rank);
    return HAKMC_EINVAL;
  }
  CK(cudaDeviceSynchronize());
  for (int rr = 0; rr < world; rr++) {
    if (rr == rank) continue;
    const TpHandle& h = hs[rr];
    if (h.pid == (int32_t)getpid()) {
      int can = 0;
      CK(cudaDeviceCanAccessPeer(&can, c->device, h.device));
      if (!can) { set_err("tp_connect: device %d cannot access device %d", c->device, h.device); return HAKMC_EINVAL; }
      cudaError_t e = cudaDeviceEnablePeerAccess(h.device, 0);
      if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
        set_err("tp_connect: peer access to device %d: %s", h.device, cudaGetErrorString(e));
        return HAKMC_ECUDA;
      }
      cudaGetLastError();
      for (int x = 0; x < XR_COUNT; x++) c->peer_ptr[rr][x] = (void*)(uintptr_t)h.ptr[x];
    } else {
      c->peer_ipc[rr] = true;
      for (int x = 0; x < XR_COUNT; x++)
        CK(cudaIpcOpenMemHandle(&c->peer_ptr[rr][x], h.ipc[x], cudaIpcMemLazyEnablePeerAccess));
    }
  }
  for (int x = 0; x < XR_COUNT; x++) c->peer_ptr[rank][x] = c->xr_ptr[x];
  c->tp_rank = rank;
  c->tp_world = world;
  c->prog_layers = -1;  // rebuild the program: rows over all GPUs' CTAs
  return world > 1 ? shard_weights(c) : 0;
}

extern "C" int hakmc_tp_rank(const hakmc_ctx* c) { return c ? c->tp_rank : -1; }
extern "C" int hakmc_tp_world(const hakmc_ctx* c) { return c ? c->tp_world : -1; }

extern "C" int hakmc_trace_step(hakmc_ctx* c, unsigned long long* stamps, int max_phases) {
  if (!c || !stamps || max_phases <= 0) return HAKMC_EINVAL;
  if (c->pos >= c->max_seq) { set_err("position beyond max_seq"); return HAKMC_ERANGE; }
  CK(cudaSetDevice(c->device));
  const size_t n = (size_t)c->num_sms * max_phases * 4;
  unsigned long long* d = nullptr;
  CK(cudaMalloc(&d, n * 8));
  cudaError_t e = cudaMemset(d, 0, n * 8);
  int r = e == cudaSuccess ? run_steps(c, 1, 0, nullptr, 0, d, max_phases) : HAKMC_ECUDA;
  if (r == 0) {
    e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess) e = cudaMemcpy(stamps, d, n * 8, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) { set_err("trace_step: %s", cudaGetErrorString(e)); r = HAKMC_ECUDA; }
  }
  cudaFree(d);
  if (r) return r;
  if ((r = check_flag(c))) return r;
  return c->num_sms;
}

// Batched decode: one pass of the layers in which row r is sequence r (input
// tokens[r] at position pos[r], cache slot r), so every weight byte read
// serves all n rows (the kernels of the batched prompt path; attention reads
// each row's own slot up to its position). Then every row's final norm,
// lm_head and greedy pick. Leaves the residual rows in xb[0..n), the logits
// in logits[0..n).
static int batch_decode(hakmc_ctx* c, const int* tokens, const int* pos, int n, float* logits, int* argmax) {
  int r = pf_ensure(c, n);
  if (!r && !c->row_io) r = dalloc(c, (void**)&c->row_io, (size_t)3 * c->max_batch * 4);
  if (r) return r;
  const int D = c->D, B = c->max_batch;
  int* tok_dev = c->row_io;
  int* pos_dev = c->row_io + B;
  int* pick_dev = c->row_io + 2 * B;
  cudaStream_t s = c->stream;
  CK(cudaMemcpyAsync(tok_dev, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(pos_dev, pos, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  int max_pos = 0;
  for (int i = 0; i < n; i++) max_pos = std::max(max_pos, pos[i]);
  const size_t slot = (size_t)c->L * c->max_seq * c->KV;
  // score capacity of the attention launch: a multiple of 1024, so a
  // captured graph serves the next steps until the positions pass it
  const int n_cap = std::min((max_pos + 1 + 1023) / 1024 * 1024, c->max_seq);
  // the kernels of the step, captured once per (rows, layers, score
  // capacity) into a graph: ~15 launches per layer
  const uint64_t key = ((uint64_t)n << 48) | ((uint64_t)c->run_layers << 32) | (uint64_t)n_cap;
  auto enqueue = [&]() -> cudaError_t {
    cudaError_t e = launch_pf_embed(c->pf_x, c->tok_embd.w, tok_dev, n, D, s);
    if (e == cudaSuccess) e = pf_layers(c, n, 0, pos_dev, slot, n_cap);
    // final norm, lm_head, greedy pick per row (src/model.c:159-164, src/sample.c:28-32)
    if (e == cudaSuccess)
      e = launch_rx_norm_quant(c->pf_x, c->out_norm, n, D, c->eps, c->rsq, c->pf_xn, c->pf_xq, c->pf_xs, s);
    if (e == cudaSuccess) e = pf_matmul(c, c->logits, c->lm_head, c->pf_xn, c->pf_xq, c->pf_xs, nullptr, n, false);
    if (e == cudaSuccess) e = launch_pf_argmax(pick_dev, c->logits, n, c->V, s);
    return e;
  };
  cudaGraphExec_t ge = nullptr;
  auto it = c->bgraphs.find(key);
  if (it != c->bgraphs.end()) {
    ge = it->second;
  } else {
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      const cudaError_t e1 = enqueue();
      e = cudaStreamEndCapture(s, &g);
      if (e1 != cudaSuccess) e = e1;
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&ge, g, 0);
    if (g) cudaGraphDestroy(g);
    if (e == cudaSuccess) {
      c->bgraphs[key] = ge;
    } else {
      ge = nullptr;  // not capturable here: launch the kernels directly
      cudaGetLastError();
    }
  }
  CK(cudaEventRecord(c->ev0, s));
  if (ge) CK(cudaGraphLaunch(ge, s));
  else CK(enqueue());
  CK(cudaEventRecord(c->ev1, s));
  CK(cudaMemcpyAsync(c->xb, c->pf_x, (size_t)n * D * 4, cudaMemcpyDeviceToDevice, s));
  if (argmax) CK(cudaMemcpyAsync(argmax, pick_dev, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
  if (logits) CK(cudaMemcpyAsync(logits, c->logits, (size_t)n * c->V * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  CK(cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1));
  return check_flag(c);
}

extern "C" int hakmc_forward_batch(hakmc_ctx* c, const int* tokens, const int* pos, int n_seq,
                                   float* logits, int* argmax) {
  if (!c || !tokens || !pos || n_seq <= 0 || n_seq > c->max_batch) { set_err("bad batch"); return HAKMC_EINVAL; }
  for (int i = 0; i < n_seq; i++) {
    if (tokens[i] < 0 || tokens[i] >= c->V) { set_err("token %d out of range", tokens[i]); return HAKMC_EINVAL; }
    if (pos[i] < 0 || pos[i] >= c->max_seq) { set_err("position %d beyond max_seq %d", pos[i], c->max_seq); return HAKMC_ERANGE; }
  }
  CK(cudaSetDevice(c->device));
  // BATCH_ROWS_MIN or more sequences on one GPU: one batched pass (weights
  // read once), while a row's attention scores fit in shared memory. Fewer
  // run the step kernel per sequence. Both give the same bits.
  if (n_seq >= BATCH_ROWS_MIN && c->tp_world == 1 && rx_attention_smem_bytes(c->hd, c->max_seq) <= RX_ATTN_SMEM_MAX)
    return batch_decode(c, tokens, pos, n_seq, logits, argmax);
  if (!c->use_step) { set_err("forward_batch runs on the step kernel (HAKMC_STEP=0 is set)"); return HAKMC_EINVAL; }
  // sequence 0 is also the single-sequence API's: its position and last pick
  // (the input hakmc_decode continues from) are restored afterwards
  const int saved_pos = c->pos;
  CK(cudaMemcpyAsync(c->token_dev + TOKEN_SAVE, c->token_dev, 4, cudaMemcpyDeviceToDevice, c->stream));
  int r = 0;
  float dev_ms = 0.f;  // the step launches' device time, summed
  for (int i = 0; i < n_seq && !r; i++) {
    c->pos = pos[i];
    c->h_pinned[0] = tokens[i];
    CK(cudaMemcpyAsync(c->token_dev, &c->h_pinned[0], 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaEventRecord(c->ev0, c->stream));
    r = run_steps(c, 1, 1, c->token_dev, 0, nullptr, 0, i);
    if (r) break;
    CK(cudaEventRecord(c->ev1, c->stream));
    CK(cudaMemcpyAsync(&c->h_pinned[1], c->token_dev, 4, cudaMemcpyDeviceToHost, c->stream));
    if (logits) CK(cudaMemcpyAsync(c->logits_pinned, c->logits, (size_t)c->V * 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, c->ev0, c->ev1));
    dev_ms += ms;
    c->last_ms = dev_ms;
    r = check_flag(c);
    if (r) break;
    if (argmax) argmax[i] = c->h_pinned[1];
    if (logits) memcpy(logits + (size_t)i * c->V, c->logits_pinned, (size_t)c->V * 4);
  }
  c->pos = saved_pos;
  c->h_pinned[2] = saved_pos;
  CK(cudaMemcpyAsync(c->pos_dev, &c->h_pinned[2], 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemcpyAsync(c->token_dev, c->token_dev + TOKEN_SAVE, 4, cudaMemcpyDeviceToDevice, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  return r;
}

extern "C" int hakmc_hidden(hakmc_ctx* c, int seq, float* out) {
  if (!c || !out || seq < 0 || seq >= c->max_batch) return HAKMC_EINVAL;
  CK(cudaSetDevice(c->device));
  CK(cudaMemcpyAsync(out, c->xb + (size_t)seq * c->D, (size_t)c->D * 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  return 0;
}

extern "C" int hakmc_debug_read(hakmc_ctx* c, int which, float* out) {
  if (!c || !out) return HAKMC_EINVAL;
  const float* src[7] = {c->xb, c->q, c->k, c->v, c->att, c->hbuf, c->logits};
  const int n[7] = {c->D, c->D, c->KV, c->KV, c->D, c->F, c->V};
  if (which < 0 || which > 6) return HAKMC_EINVAL;
  CK(cudaSetDevice(c->device));
  if (c->step_ran && which >= 1 && which <= 5) {
    // the step kernel keeps these as tagged words: unpack into the plain buffer
    const uint64_t* ll[6] = {nullptr, c->q_ll, c->k_ll, c->v_ll, c->att_ll, c->h_ll};
    CK(launch_ll_unpack(const_cast<float*>(src[which]), ll[which], n[which], c->stream));
  }
  CK(cudaMemcpyAsync(out, src[which], (size_t)n[which] * 4, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  return 0;
}

extern "C" int hakmc_fill_kv(hakmc_ctx* c, int seq, const float* k, const float* v, int n_pos) {
  if (!c || !k || !v || seq < 0 || seq >= c->max_batch || n_pos < 0 || n_pos > c->max_seq) {
    set_err("bad fill_kv arguments");
    return HAKMC_EINVAL;
  }
  CK(cudaSetDevice(c->device));
  const size_t row = (size_t)n_pos * c->KV * 4;
  for (int l = 0; l < c->L; l++) {
    const size_t off = (((size_t)seq * c->L + l) * c->max_seq) * c->KV;
    CK(cudaMemcpy(c->k_cache + off, k + (size_t)l * n_pos * c->KV, row, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->v_cache + off, v + (size_t)l * n_pos * c->KV, row, cudaMemcpyHostToDevice));
  }
  if (seq == 0) return hakmc_set_pos(c, n_pos);
  return 0;
}

extern "C" int hakmc_fill_kv_normal(hakmc_ctx* c, int seq, int n_pos, unsigned long long seed) {
  if (!c || seq < 0 || seq >= c->max_batch || n_pos < 0 || n_pos > c->max_seq) {
    set_err("bad fill_kv_normal arguments");
    return HAKMC_EINVAL;
  }
  CK(cudaSetDevice(c->device));
  const size_t lstride = (size_t)c->max_seq * c->KV, off = (size_t)seq * c->L * lstride;
  if (n_pos > 0) {
    CK(launch_pf_fill_normal(c->k_cache + off, lstride, (size_t)n_pos * c->KV, c->L, seed * 2 + 1, c->stream));
    CK(launch_pf_fill_normal(c->v_cache + off, lstride, (size_t)n_pos * c->KV, c->L, seed * 2 + 2, c->stream));
  }
  CK(cudaStreamSynchronize(c->stream));
  if (seq == 0) return hakmc_set_pos(c, n_pos);
  return 0;
}

// ------------------------------------------------------------ kernel-level API

namespace {
// Small per-device scratch the kernel-level entry points share: a position
// word, attention partials and tickets, a RoPE row and argmax words. Grown on
// demand; one per device for the life of the process.
struct DevScratch {
  int* pos = nullptr;
  unsigned* counters = nullptr;
  float* part = nullptr;
  size_t part_floats = 0;
  float* rope = nullptr;
  size_t rope_floats = 0;
  unsigned long long* key = nullptr;
  unsigned* done = nullptr;
  int* tok = nullptr;
};
std::mutex g_scr_mu;
std::map<int, DevScratch> g_scr;

int scratch(DevScratch** out, size_t part_floats, size_t rope_floats) {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_scr_mu);
  DevScratch& s = g_scr[dev];
  if (!s.pos) {
    CK(cudaMalloc(&s.pos, 64));
    CK(cudaMalloc(&s.counters, 64 * 4));
    CK(cudaMemset(s.counters, 0, 64 * 4));
    CK(cudaMalloc(&s.key, 64));
    CK(cudaMemset(s.key, 0, 64));
    CK(cudaMalloc(&s.done, 64));
    CK(cudaMemset(s.done, 0, 64));
    CK(cudaMalloc(&s.tok, 64));
  }
  if (part_floats > s.part_floats) {
    CK(cudaDeviceSynchronize());
    if (s.part) cudaFree(s.part);
    CK(cudaMalloc(&s.part, part_floats * 4));
    s.part_floats = part_floats;
  }
  if (rope_floats > s.rope_floats) {
    CK(cudaDeviceSynchronize());
    if (s.rope) cudaFree(s.rope);
    CK(cudaMalloc(&s.rope, rope_floats * 4));
    s.rope_floats = rope_floats;
  }
  *out = &s;
  return 0;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
}  // namespace

#define CKL(expr)                                                                           \
  do {                                                                                      \
    cudaError_t e_ = (expr);                                                                \
    if (e_ != cudaSuccess) { set_err("%s: %s", #expr, cudaGetErrorString(e_)); return HAKMC_ECUDA; } \
  } while (0)

extern "C" int hakmc_quantize_q8_32(const float* x, int n, int8_t* xq, float* xs, void* stream) {
  if (!x || !xq || !xs || n <= 0 || n % 32) { set_err("quantize: n must be a positive multiple of 32"); return HAKMC_EINVAL; }
  CKL(launch_quantize_q8(x, n, xq, xs, (cudaStream_t)stream));
  return 0;
}

static int gemv_common(float* out, const void* w, int type, const float* x, const int8_t* xq, const float* xs,
                       const float* bias, int n_out, int n_in, int act, void* stream) {
  if (!out || !w || n_out <= 0 || n_in <= 0 || n_in % QK) { set_err("gemv: n_in must be a positive multiple of 256"); return HAKMC_EINVAL; }
  if (!aligned16(w) || (x && !aligned16(x)) || (xq && !aligned16(xq))) { set_err("gemv: buffers must be 16-byte aligned"); return HAKMC_EINVAL; }
  PhaseParams p = {};
  p.n_in = n_in; p.act = act; p.x = x; p.xq = xq; p.xs = xs;
  p.n_seg = 1;
  Seg s = {};
  s.w = (const uint8_t*)w;
  s.type = type;
  s.n_rows = n_out;
  s.epi = EPI_STORE;
  s.out = out;
  s.bias = bias;
  p.seg[0] = s;
  finish_params(p);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (phase_smem_bytes(p, sms) > (size_t)PHASE_SMEM_MAX) { set_err("gemv: n_in too large"); return HAKMC_EINVAL; }
  CKL(launch_phase(p, sms, (cudaStream_t)stream, false));
  return 0;
}

extern "C" int hakmc_gemv_q4k_q8(float* out, const void* w, const int8_t* xq, const float* xs, const float* bias,
                                 int n_out, int n_in, void* stream) {
  if (!xq || !xs) return HAKMC_EINVAL;
  return gemv_common(out, w, W_Q4K, nullptr, xq, xs, bias, n_out, n_in, ACT_Q8, stream);
}

static int device_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// Which batches go to the tensor cores (hakm_mma.cu): their MMAs take the
// integer work that bounds the dp4a kernel as the batch grows. Measured on
// the config-1 shapes: above 16 activations always; from 9 (where the dp4a
// kernel runs its 16-wide instance) once the matrix has 16M weights or more
// in at least 64 row tiles of 128 (the tensor-core kernel never splits a
// row along K, so a long-K matrix of few rows runs on few SMs); the rest
// stay on dp4a, whose launch is lighter.
static bool use_tensor_cores(int n_out, int n_in, int n_batch) {
  if (n_batch > 16) return true;
  return n_batch > 8 && (long long)n_out * n_in >= (16ll << 20) && (n_out + 127) / 128 >= 64;
}

extern "C" size_t hakmc_gemv_q4k_q8_batch_scratch(int n_out, int n_in, int n_batch) {
  if (n_out <= 0 || n_in <= 0 || n_in % QK || n_batch <= 0) return 0;
  const int sms = device_sms();
  // the dp4a kernel's partials and tickets (the tensor-core kernel needs none)
  return (q4k_batch_scratch_bytes(n_out, n_in, n_batch, sms) + 255) & ~(size_t)255;
}

extern "C" int hakmc_gemv_q4k_q8_batch(float* out, const void* w, const int8_t* xq, const float* xs,
                                       const float* bias, int n_out, int n_in, int n_batch, void* scratch,
                                       size_t scratch_bytes, void* stream) {
  if (!out || !w || !xq || !xs || n_out <= 0 || n_in <= 0 || n_in % QK || n_batch <= 0) {
    set_err("gemv batch: n_in must be a positive multiple of 256, n_batch >= 1");
    return HAKMC_EINVAL;
  }
  if (!aligned16(w) || !aligned16(xq)) { set_err("gemv batch: w and xq must be 16-byte aligned"); return HAKMC_EINVAL; }
  const int sms = device_sms();
  const size_t bytes = hakmc_gemv_q4k_q8_batch_scratch(n_out, n_in, n_batch);
  if (scratch && (scratch_bytes < bytes || !aligned16(scratch))) {
    set_err("gemv batch: scratch needs %zu bytes, 16-byte aligned", bytes);
    return HAKMC_EINVAL;
  }
  const cudaStream_t st = (cudaStream_t)stream;
  if (use_tensor_cores(n_out, n_in, n_batch) && aligned16(xs)) {
    CKL(launch_q4k_mma(out, (const uint8_t*)w, xq, xs, bias, n_out, n_in, n_batch, nullptr, sms, st));
    return 0;
  }
  void* s = scratch;
  if (!s) {  // stream-ordered scratch for callers that pass none
    CKL(cudaMallocAsync(&s, bytes, st));
    const size_t t0 = q4k_batch_ticket_offset(n_out, n_in, n_batch, sms);
    const cudaError_t e = cudaMemsetAsync((char*)s + t0, 0, bytes - t0, st);
    if (e != cudaSuccess) { cudaFreeAsync(s, st); CKL(e); }
  }
  const cudaError_t e = launch_q4k_batch(out, (const uint8_t*)w, xq, xs, bias, n_out, n_in, n_batch, s, nullptr,
                                         sms, st);
  if (!scratch) CKL(cudaFreeAsync(s, st));
  CKL(e);
  return 0;
}

extern "C" size_t hakmc_gemm_q4k_q8_scratch(int n_out, int n_in, int n_batch) {
  (void)n_out, (void)n_in, (void)n_batch;
  return 0;  // the kernel never splits K, so it needs no scratch
}

extern "C" int hakmc_gemm_q4k_q8(float* out, const void* w, const int8_t* xq, const float* xs, const float* bias,
                                 int n_out, int n_in, int n_batch, void* scratch, size_t scratch_bytes,
                                 void* stream) {
  (void)scratch, (void)scratch_bytes;
  if (!out || !w || !xq || !xs || n_out <= 0 || n_in <= 0 || n_in % QK || n_batch <= 0) {
    set_err("gemm: n_in must be a positive multiple of 256, n_batch >= 1");
    return HAKMC_EINVAL;
  }
  if (!aligned16(w) || !aligned16(xq) || !aligned16(xs)) {
    set_err("gemm: w, xq and xs must be 16-byte aligned");
    return HAKMC_EINVAL;
  }
  CKL(launch_q4k_mma(out, (const uint8_t*)w, xq, xs, bias, n_out, n_in, n_batch, nullptr, device_sms(),
                     (cudaStream_t)stream));
  return 0;
}

extern "C" int hakmc_attention_rows(float* out, const float* q, const float* k_cache, const float* v_cache,
                                    int rows, int pos0, const int* row_pos, int max_pos, size_t slot_stride,
                                    int n_heads, int n_kv, int head_dim, void* stream) {
  if (!out || !q || !k_cache || !v_cache || rows <= 0 || max_pos < 0 || n_heads <= 0 || n_kv <= 0 ||
      n_heads % n_kv || (head_dim != 64 && head_dim != 128) || (!row_pos && (pos0 < 0 || pos0 + rows - 1 > max_pos))) {
    set_err("attention_rows: bad arguments");
    return HAKMC_EINVAL;
  }
  if (rx_attention_smem_bytes(head_dim, max_pos + 1) > RX_ATTN_SMEM_MAX) {
    set_err("attention_rows: %d positions exceed the shared-memory score row", max_pos + 1);
    return HAKMC_ERANGE;
  }
  CKL(launch_rx_attention(out, q, k_cache, v_cache, rows, pos0, row_pos, max_pos + 1, slot_stride, n_heads, n_kv,
                          head_dim, host_rsqrt_nr((float)head_dim), (cudaStream_t)stream));
  return 0;
}

extern "C" int hakmc_gemm_q6k(float* out, const void* w, const float* x, const float* bias, int n_out, int n_in,
                              int n_batch, int accumulate, void* stream) {
  if (!out || !w || !x || n_out <= 0 || n_in <= 0 || n_in % QK || n_batch <= 0) {
    set_err("gemm_q6k: n_in must be a positive multiple of 256, n_batch >= 1");
    return HAKMC_EINVAL;
  }
  if (!aligned16(w)) { set_err("gemm_q6k: w must be 16-byte aligned"); return HAKMC_EINVAL; }
  CKL(launch_rx_q6k_gemm(out, (const uint8_t*)w, x, bias, n_out, n_in, n_batch, accumulate != 0,
                         (cudaStream_t)stream));
  return 0;
}

extern "C" int hakmc_gemv_q4k(float* out, const void* w, const float* x, const float* bias, int n_out, int n_in,
                              void* stream) {
  if (!x) return HAKMC_EINVAL;
  return gemv_common(out, w, W_Q4K, x, nullptr, nullptr, bias, n_out, n_in, ACT_F32, stream);
}

extern "C" int hakmc_q4k_subsums(int32_t* iqx, int32_t* ix, const void* w, const int8_t* xq, int n_out, int n_in,
                                 void* stream) {
  if (!iqx || !ix || !w || !xq || n_out <= 0 || n_in <= 0 || n_in % QK) return HAKMC_EINVAL;
  CKL(launch_q4k_subsums(iqx, ix, (const uint8_t*)w, xq, n_out, n_in, (cudaStream_t)stream));
  return 0;
}

extern "C" size_t hakmc_q6k_packed_bytes(int n_rows, int n_in) {
  return (size_t)n_rows * dev_row_bytes(W_Q6K, n_in / QK);
}

extern "C" int hakmc_q6k_pack(void* dst, const void* src, int n_rows, int n_in, void* stream) {
  if (!dst || !src || n_rows <= 0 || n_in <= 0 || n_in % QK) return HAKMC_EINVAL;
  CKL(launch_q6k_pack((uint8_t*)dst, (const uint8_t*)src, n_rows, n_in, (cudaStream_t)stream));
  return 0;
}

extern "C" int hakmc_gemv_q6k(float* out, const void* w, const float* x, const float* bias, int n_out, int n_in,
                              void* stream) {
  if (!x) return HAKMC_EINVAL;
  return gemv_common(out, w, W_Q6K, x, nullptr, nullptr, bias, n_out, n_in, ACT_F32, stream);
}

extern "C" int hakmc_lmhead_argmax(float* logits, int* argmax, const void* w, const float* x, const float* norm_w,
                                   float eps, int n_vocab, int n_in, void* stream) {
  if (!argmax || !w || !x || n_vocab <= 0 || n_in % QK || !aligned16(w) || !aligned16(x)) return HAKMC_EINVAL;
  DevScratch* s;
  int r = scratch(&s, 0, 0);
  if (r) return r;
  PhaseParams p = {};
  p.n_in = n_in; p.act = norm_w ? ACT_RMS : ACT_F32; p.x = x; p.norm_w = norm_w; p.eps = eps;
  p.n_seg = 1;
  Seg sg = {};
  sg.w = (const uint8_t*)w;
  sg.type = W_Q6K; sg.n_rows = n_vocab; sg.epi = EPI_ARGMAX; sg.out = logits;
  p.seg[0] = sg;
  p.argmax_key = s->key; p.done_counter = s->done; p.next_token = argmax;
  finish_params(p);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (norm_w && !(p.rsq = rsqrt_table_device(dev))) { set_err("lmhead_argmax: no rsqrtss table"); return HAKMC_ECUDA; }
  CKL(launch_phase(p, sms, (cudaStream_t)stream, false));
  return 0;
}

extern "C" int hakmc_dequant(float* out, const void* w, int type, int n_rows, int n_in, void* stream) {
  if (!out || !w || n_rows <= 0 || n_in % QK || (type != W_Q4K && type != W_Q6K)) return HAKMC_EINVAL;
  CKL(launch_dequant(out, (const uint8_t*)w, type, n_rows, n_in, (cudaStream_t)stream));
  return 0;
}

extern "C" int hakmc_rmsnorm(float* y, const float* x, const float* w, int n, float eps, void* stream) {
  if (!y || !x || !w || n <= 0 || n % 8) return HAKMC_EINVAL;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  const uint32_t* rsq = rsqrt_table_device(dev);
  if (!rsq) { set_err("rmsnorm: no rsqrtss table for device %d", dev); return HAKMC_ECUDA; }
  CKL(launch_rmsnorm(y, x, w, n, eps, rsq, (cudaStream_t)stream));
  return 0;
}

extern "C" int hakmc_attention(float* out, const float* q, const float* kc, const float* vc, int pos, int n_heads,
                               int n_kv, int head_dim, void* stream) {
  if (!out || !q || !kc || !vc || pos < 0 || n_kv <= 0 || n_heads % n_kv || (head_dim != 64 && head_dim != 128)) {
    set_err("attention: unsupported arguments");
    return HAKMC_EINVAL;
  }
  DevScratch* s;
  int r = scratch(&s, attention_scratch_floats(n_heads, head_dim, pos + 1), 0);
  if (r) return r;
  cudaStream_t st = (cudaStream_t)stream;
  CKL(cudaMemcpyAsync(s->pos, &pos, 4, cudaMemcpyHostToDevice, st));
  AttnParams a = {};
  a.q = q; a.k_cache = kc; a.v_cache = vc; a.out = out; a.pos_dev = s->pos;
  a.n_heads = n_heads; a.n_kv = n_kv; a.head_dim = head_dim; a.scale = host_rsqrt_nr((float)head_dim);
  a.part = s->part; a.score_stride = pos + 1;
  CKL(launch_attention(a, st, false));
  CKL(cudaStreamSynchronize(st));
  return 0;
}

extern "C" int hakmc_attention_noalloc(float* out, const float* q, const float* kc, const float* vc, int pos,
                                       int n_heads, int n_kv, int head_dim, void* stream) {
  if (!out || !q || !kc || !vc || pos < 0 || n_kv <= 0 || n_heads % n_kv || (head_dim != 64 && head_dim != 128)) {
    set_err("attention_noalloc: unsupported arguments");
    return HAKMC_EINVAL;
  }
  const size_t need = attention_scratch_floats(n_heads, head_dim, pos + 1);
  if (need > noalloc_part_floats()) {
    set_err("attention_noalloc: %d heads x %d positions need %zu scratch floats, the fixed array holds %zu "
            "(use hakmc_attention)", n_heads, pos + 1, need, noalloc_part_floats());
    return HAKMC_ERANGE;
  }
  CKL(attention_noalloc(out, q, kc, vc, pos, n_heads, n_kv, head_dim, (cudaStream_t)stream));
  return 0;
}

extern "C" int hakmc_plan_rows(const int* seg_rows, int n_seg, int grid, int cta, int* ranges) {
  if (!seg_rows || !ranges || n_seg < 1 || n_seg > MAX_SEGS || grid < 1 || cta < 0 || cta >= grid) return HAKMC_EINVAL;
  PhaseDesc d = {};
  d.kind = PK_GEMV;
  d.g.n_in = QK;
  d.g.n_seg = n_seg;
  for (int s = 0; s < n_seg; s++) {
    if (seg_rows[s] < 1) return HAKMC_EINVAL;
    d.g.seg[s].n_rows = seg_rows[s];
  }
  SegRange sr[MAX_SEGS];
  step_ranges(&d, 1, grid, cta, 1, sr);
  for (int s = 0; s < n_seg; s++) { ranges[2 * s] = sr[s].row0; ranges[2 * s + 1] = sr[s].row1; }
  return 0;
}

extern "C" int hakmc_plan_attn_units(int n_heads, int head_dim, int rank, int world, int* units, int cap) {
  if (n_heads < 1 || head_dim < ATTN_SLICE || head_dim % ATTN_SLICE || world < 1 || rank < 0 || rank >= world)
    return HAKMC_EINVAL;
  const int n = attn_units_local(attn_units(n_heads, head_dim), rank, world);
  for (int i = 0; i < n && i < cap; i++) units[i] = attn_unit_of(rank, world, i);
  return n;
}

namespace {
// Per-device scratch of the sampler: the sort keys / indices (4n words) and
// the generator state and pick.
struct SampleScratch {
  uint32_t* words = nullptr;
  size_t cap = 0;
  unsigned long long* io = nullptr;  // [0] rng, [1] pick (int)
};
std::mutex g_smp_mu;
std::map<int, SampleScratch> g_smp;

int sample_on(float* logits, int n, float temp, float top_p, int top_k, unsigned long long* rng, int* token,
              cudaStream_t st) {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (!(temp > 0.0f)) {  // greedy: first index of the maximum (src/sample.c:28-32)
    DevScratch* s;
    int r = scratch(&s, 0, 0);
    if (r) return r;
    CK(launch_pf_argmax(s->tok, logits, 1, n, st));
    CK(cudaMemcpyAsync(token, s->tok, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return 0;
  }
  if (n < 9) { set_err("sample: vocabulary below 9 entries"); return HAKMC_EINVAL; }
  const uint32_t* rcp = rcp_table_device(dev);
  if (!rcp) { set_err("sample: no rcpss table for this host"); return HAKMC_ECUDA; }
  std::lock_guard<std::mutex> lk(g_smp_mu);
  SampleScratch& S = g_smp[dev];
  if (!S.io) CK(cudaMalloc(&S.io, 64));
  const size_t need = sample_scratch_words(n);
  if (need > S.cap) {
    CK(cudaStreamSynchronize(st));
    if (S.words) cudaFree(S.words);
    S.words = nullptr;
    CK(cudaMalloc(&S.words, need * 4));
    S.cap = need;
  }
  CK(cudaMemcpyAsync(S.io, rng, 8, cudaMemcpyHostToDevice, st));
  CK(launch_sample(logits, n, temp, top_p, top_k, rcp, S.words, S.io, reinterpret_cast<int*>(S.io + 1), st));
  unsigned long long back[2];
  CK(cudaMemcpyAsync(back, S.io, 16, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  *rng = back[0];
  *token = (int)(uint32_t)back[1];
  return 0;
}
}  // namespace

extern "C" int hakmc_sample(float* logits, int n, float temp, float top_p, int top_k, unsigned long long* rng,
                            int* token, void* stream) {
  if (!logits || n <= 0 || !rng || !token) return HAKMC_EINVAL;
  return sample_on(logits, n, temp, top_p, top_k, rng, token, (cudaStream_t)stream);
}

extern "C" int hakmc_sample_last(hakmc_ctx* c, float temp, float top_p, int top_k, unsigned long long* rng,
                                 int* token) {
  if (!c || !rng || !token) return HAKMC_EINVAL;
  CK(cudaSetDevice(c->device));
  return sample_on(c->logits, c->V, temp, top_p, top_k, rng, token, c->stream);
}

extern "C" int hakmc_test_expf(float* out, const float* in, int n, int variant, void* stream) {
  if (!out || !in || n < 0 || variant < 0 || variant > 2) return HAKMC_EINVAL;
  CKL(launch_exp_probe(out, in, n, variant, (cudaStream_t)stream));
  return 0;
}

extern "C" int hakmc_rope_neox(float* x, int n_heads, int head_dim, int pos, float theta, void* stream) {
  if (!x || n_heads <= 0 || head_dim <= 0 || head_dim % 2 || pos < 0) return HAKMC_EINVAL;
  const int half = head_dim / 2;
  DevScratch* s;
  int r = scratch(&s, 0, (size_t)half * 2);
  if (r) return r;
  std::vector<float> cs((size_t)half * 2);
  hakm_host_rope_row(cs.data(), head_dim, pos, theta);
  cudaStream_t st = (cudaStream_t)stream;
  CKL(cudaMemcpyAsync(s->rope, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, st));
  CKL(launch_rope(x, s->rope, nullptr, n_heads, head_dim, st));
  CKL(cudaStreamSynchronize(st));
  return 0;
}
