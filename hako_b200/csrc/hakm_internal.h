// hakm_internal.h — declarations shared by the kernels and the runtime of
// libhakm_cuda. Internal: not part of the C ABI (include/hakm_cuda.h).
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace hakm {

constexpr int QK = 256;            // k-quant super-block (src/quant.h:9)
constexpr int Q4K_BYTES = 144;     // block_q4_K (src/quant.h:12-17)
constexpr int Q6K_BYTES = 210;     // block_q6_K (src/quant.h:19-24)
constexpr int Q6K_BODY = 208;      // {ql, qh, scales} part of a block_q6_K
constexpr int MAX_SEGS = 3;

enum WType { W_Q4K = 12, W_Q6K = 14 };

// Device layouts. A row is cut into chunks of 8 super-blocks (2048 columns):
//  Q4_K: verbatim 144-byte blocks, so a chunk is 1152 contiguous bytes.
//  Q6_K: a chunk holds the 208-byte bodies of its (up to) 8 blocks, then their
//        8 fp16 d values: 1680 bytes = 8 * 210, the verbatim byte count; a
//        short last chunk is padded to 16 bytes. Every chunk starts 16-byte
//        aligned, so a stage of chunks is one bulk copy per row.
//        A body keeps the block's bytes, reordered "by lane class": the
//        reference's Q6_K dot adds the products of element i into lane i % 8
//        of its vectorized loop, and the device gives each such lane chain to
//        one thread, which then needs the code bits of elements l, l+8, ...
//        (l = i % 8). Bytes 24l .. 24l+23 hold them for class l: per half n
//        of the block (12 bytes at 24l + 12n), W0[b] = ql[64n + 8b + l],
//        W1[b] = ql[64n + 32 + 8b + l], WH[b] = qh[32n + 8b + l] (b = 0..3);
//        bytes 192..207 are the 16 int8 scales, unchanged. Element
//        i = 8(16n + 4k + b) + l is nibble (k < 2 ? low : high) of
//        (k even ? W0 : W1)[b] with bits 2k..2k+1 of WH[b] on top, the
//        element map of dequant_q6_K (src/quant.c:94-123).
constexpr int CHUNK_BLOCKS = 8;
constexpr int Q4K_CHUNK = CHUNK_BLOCKS * Q4K_BYTES;  // 1152
constexpr int Q6K_CHUNK = CHUNK_BLOCKS * Q6K_BYTES;  // 1680

__host__ __device__ inline int n_chunks(int nb) { return (nb + CHUNK_BLOCKS - 1) / CHUNK_BLOCKS; }
__host__ __device__ inline int q6_chunk_blocks(int nb, int c) {
  const int m = nb - CHUNK_BLOCKS * c;
  return m < CHUNK_BLOCKS ? m : CHUNK_BLOCKS;
}
__host__ __device__ inline int chunk_bytes(int type, int nb, int c) {
  const int m = q6_chunk_blocks(nb, c);
  return type == W_Q4K ? m * Q4K_BYTES : ((m * Q6K_BYTES + 15) & ~15);
}
// Position in the device body of byte `src` (0..207) of a verbatim body.
__host__ __device__ inline int q6k_body_pos(int src) {
  if (src < 128) {  // ql
    const int n = src >> 6, h = (src >> 5) & 1, j = src & 31;
    return 24 * (j & 7) + 12 * n + 4 * h + (j >> 3);
  }
  if (src < 192) {  // qh
    const int p = src - 128, n = p >> 5, j = p & 31;
    return 24 * (j & 7) + 12 * n + 8 + (j >> 3);
  }
  return src;  // scales
}
__host__ __device__ inline size_t dev_row_bytes(int type, int nb) {
  if (type == W_Q4K) return (size_t)nb * Q4K_BYTES;
  const int full = nb / CHUNK_BLOCKS, rem = nb % CHUNK_BLOCKS;
  return (size_t)full * Q6K_CHUNK + (rem ? (size_t)((rem * Q6K_BYTES + 15) & ~15) : 0);
}


// How the GEMV prologue builds the activation it keeps in shared memory.
enum ActMode {
  ACT_Q8 = 0,    // int8 xq / fp32 xs given in global memory
  ACT_F32 = 1,   // fp32 x in global memory (quantized in smem for Q4_K rows)
  ACT_RMS = 2,   // rmsnorm(x) * norm_w computed in smem, then as ACT_F32
};

// What each finished row does with its dot product.
enum Epi {
  EPI_STORE = 0,      // out[r] = acc (+ bias[r])
  EPI_RESID = 1,      // out[r] += acc                     (residual add)
  EPI_ROPE_QK = 2,    // rows are RoPE pairs; q out / k out + K cache write
  EPI_SWIGLU = 3,     // rows are (gate, up) pairs; out[i] = silu(g) * u
  EPI_V_CACHE = 4,    // out = acc + bias, written to the V cache at pos
  EPI_ARGMAX = 5,     // logits (optional) + running argmax key
};

// One block of output rows that share a weight type and an epilogue.
struct Seg {
  const uint8_t* w;      // rows in the device layout above
  const float* bias;     // device row order, may be null
  float* out;            // primary output
  float* out2;           // EPI_ROPE_QK: k output (rows >= split)
  float* cache;          // EPI_ROPE_QK: K cache layer base; EPI_V_CACHE: V cache base
  int type;
  int n_rows;
  int epi;
  int split;             // EPI_ROPE_QK: first k row (= q rows)
  // tensor parallelism: w holds only this GPU's rows, w_rows of them,
  // cyclically from row w_row0 (rows w_row0 .. n_rows-1, then 0 ..);
  // w_rows 0: all rows
  int w_row0, w_rows;
};

struct PhaseParams {
  int n_in;              // K (multiple of 256)
  int act;               // ActMode
  const float* x;        // ACT_F32 / ACT_RMS input
  const float* norm_w;   // ACT_RMS weight
  float eps;
  const int8_t* xq;      // ACT_Q8 input
  const float* xs;
  int need_q8;           // some segment is Q4_K (int8 activation in the prologue)
  int need_q6;           // some segment is Q6_K (fp32 activation, by lane class, in the prologue)
  const uint32_t* rsq;   // ACT_RMS: the rsqrtss table (2048 words, see rsqrt_est)
  int n_seg;
  Seg seg[MAX_SEGS];
  // filled by launch_phase: ring geometry and per-CTA partial-sum slots
  int n_stages, stage_bytes, part_floats;
  // position-dependent epilogues
  const float* rope_cs;  // [max_seq][head_dim/2] (cos, sin) pairs
  const int* pos_dev;    // current position (device)
  int head_dim;
  int kv_dim;
  // argmax epilogue
  unsigned long long* argmax_key;
  // step finalisation by the last CTA (lm_head phase): next token, pos++
  unsigned int* done_counter;
  int* next_token;       // written with the argmax
  int* token_log;        // token_log[step] = argmax (may be null)
  int token_log_cap;     // entries in token_log; steps beyond it are not logged
  int* step_dev;         // step counter for token_log (may be null)
  int* pos_inc;          // position to increment (may be null)
  int* err_flag;         // set non-zero when a bounded wait gives up (may be null)
  unsigned long long* trace;  // per-CTA %globaltimer stamps (measurement hook, may be null)
};

// ---- streaming GEMV phases (hakm_stream.cu) ----
cudaError_t launch_phase(const PhaseParams& p, int num_sms, cudaStream_t s, bool pdl);
size_t phase_smem_bytes(const PhaseParams& p, int grid);
constexpr int PHASE_SMEM_MAX = 220 * 1024;

// ---- small kernels (hakm_kernels.cu) ----

cudaError_t launch_quantize_q8(const float* x, int n, int8_t* xq, float* xs, cudaStream_t s);
// Batched Q4_K x q8_32 matmul (hakm_batch.cu). scratch: scratch_bytes,
// the words from ticket_offset on zero (the launches leave them zero).
cudaError_t launch_q4k_batch(float* out, const uint8_t* w, const int8_t* xq, const float* xs, const float* bias,
                             int n_out, int n_in, int n_batch, void* scratch, int* err_flag, int num_sms,
                             cudaStream_t st);
size_t q4k_batch_scratch_bytes(int n_out, int n_in, int n_batch, int num_sms);
size_t q4k_batch_ticket_offset(int n_out, int n_in, int n_batch, int num_sms);
// out[n][r] = sum over c < nch of part[c][n][r] (+ bias[r]), in order.
cudaError_t launch_chunk_sum(float* out, const float* part, const float* bias, int n_out, int n_batch, int nch,
                             int num_sms, cudaStream_t st);
// Tensor-core (tcgen05 kind::i8) batched Q4_K x q8_32 matmul (hakm_mma.cu):
// every output equals the reference's q4k_vec_dot (+ bias) bit for bit.
cudaError_t launch_q4k_mma(float* out, const uint8_t* w, const int8_t* xq, const float* xs, const float* bias,
                           int n_out, int n_in, int n_batch, int* err_flag, int num_sms, cudaStream_t st);
cudaError_t launch_q4k_subsums(int32_t* iqx, int32_t* ix, const uint8_t* w, const int8_t* xq,
                               int n_out, int n_in, cudaStream_t s);
cudaError_t launch_q6k_pack(uint8_t* dst, const uint8_t* src, int n_rows, int n_in, cudaStream_t s);
cudaError_t launch_dequant(float* out, const uint8_t* w, int type, int n_rows, int n_in, cudaStream_t s);
cudaError_t launch_rmsnorm(float* y, const float* x, const float* w, int n, float eps, const uint32_t* rsq,
                           cudaStream_t s);
cudaError_t launch_embed_q6k(float* xb, const uint8_t* w, const int* token, int n_in, cudaStream_t s,
                             bool pdl);
cudaError_t launch_rope(float* x, const float* rope_cs, const int* pos_dev, int n_heads, int head_dim,
                        cudaStream_t s);

// ---- row-wise kernels of the row-batched passes (hakm_prefill.cu) ----
cudaError_t launch_pf_embed(float* x, const uint8_t* w, const int* tokens, int M, int D, cudaStream_t s);
cudaError_t launch_pf_rope_kv(const float* qk, const float* v, float* q, float* kc, float* vc, const float* rope_cs,
                              int M, int pos0, const int* row_pos, size_t slot_stride, int D, int KV, int hd,
                              cudaStream_t s);
cudaError_t launch_pf_argmax(int* out, const float* logits, int M, int V, cudaStream_t s);
cudaError_t launch_pf_fill_normal(float* dst, size_t ystride, size_t n, int blocks_y, uint64_t seed, cudaStream_t s);
cudaError_t launch_pf_add(float* x, const float* o, size_t n, cudaStream_t s);

// ---- row-batched kernels with the reference's roundings (hakm_rows.cu) ----
// Each row's results equal the single-row decode path's bit for bit.
// rmsnorm of M rows of D (a multiple of 256, at most 8192) into xn and/or
// their q8_32 codes (xq, xs); either output may be null.
cudaError_t launch_rx_norm_quant(const float* x, const float* w, int M, int D, float eps, const uint32_t* rsq,
                                 float* xn, int8_t* xq, float* xs, cudaStream_t s);
// out[m][n] (+)= Q6_K row n . x[m] (+ bias[n]), m < M.
cudaError_t launch_rx_q6k_gemm(float* out, const uint8_t* w, const float* x, const float* bias, int n_out, int K,
                               int M, bool accumulate, cudaStream_t s);
cudaError_t launch_rx_swiglu(float* h, const float* gu, int M, int F, cudaStream_t s);
// Attention of `rows` rows: row r at row_pos[r] with its cache slot_stride
// floats after row r-1's, or (row_pos null) at pos0 + r over one cache;
// n_max >= every row's position + 1.
constexpr size_t RX_ATTN_SMEM_MAX = 200 * 1024;
size_t rx_attention_smem_bytes(int hd, int n_max);
cudaError_t launch_rx_attention(float* out, const float* q, const float* kc, const float* vc, int rows, int pos0,
                                const int* row_pos, int n_max, size_t slot_stride, int H, int KVH, int hd,
                                float scale, cudaStream_t s);

struct AttnParams {
  const float* q;        // [H*hd]
  const float* k_cache;  // layer base [max_seq][kv_dim]
  const float* v_cache;
  float* out;            // [H*hd]
  const int* pos_dev;    // attend over positions 0..pos
  int n_heads, n_kv, head_dim;
  float scale;           // 1.0f/sqrtf(head_dim) as the reference's build computes it
  float* part;           // scratch: per unit, score_stride floats (scores, exps, probabilities)
  int score_stride;      // >= positions attended (pos + 1)
};
// Attention work units: (query head, slice of ATTN_SLICE dimensions).
constexpr int ATTN_SLICE = 32;
__host__ __device__ inline int attn_units(int n_heads, int head_dim) { return n_heads * (head_dim / ATTN_SLICE); }
// With tensor parallelism rank r of `world` runs units r, r + world, ...:
// attn_units_local of them, the i-th being attn_unit_of(r, world, i).
__host__ __device__ inline int attn_units_local(int n_units, int rank, int world) {
  return (n_units - rank + world - 1) / world;
}
__host__ __device__ inline int attn_unit_of(int rank, int world, int i) { return rank + world * i; }
cudaError_t launch_attention(const AttnParams& a, cudaStream_t s, bool pdl);
// hakmc_attention_noalloc: scratch in a static device array, no allocation
cudaError_t attention_noalloc(float* out, const float* q, const float* kc, const float* vc, int pos, int n_heads,
                              int n_kv, int head_dim, cudaStream_t stream);
size_t noalloc_part_floats();
// Scratch floats of launch_attention for n positions.
size_t attention_scratch_floats(int n_heads, int head_dim, int n_pos);
// Sampling for temperature > 0 (hakm_sample.cu): logits[0..n) (n >= 9)
// become probabilities in place; scratch: sample_scratch_words(n) words;
// rng_dev / out_dev: the generator state (in/out) and the pick.
size_t sample_scratch_words(int n);
cudaError_t launch_sample(float* logits, int n, float temp, float top_p, int top_k, const uint32_t* rcp_tab,
                          uint32_t* scratch, unsigned long long* rng_dev, int* out_dev, cudaStream_t s);
// The rcpss table of this host on device `dev` (made on first use).
const uint32_t* rcp_table_device(int dev);
// The device's exp restatements on n inputs (variant 0 scalar, 1 8-wide, 2 4-wide).
cudaError_t launch_exp_probe(float* out, const float* in, int n, int variant, cudaStream_t s);
// The rsqrtss table of this host on device `dev` (made on first use).
const uint32_t* rsqrt_table_device(int dev);
// 1.0f/sqrtf(v) as the reference's build computes it, on the host.
float host_rsqrt_nr(float v);

// Rows of one segment that one CTA computes, and where its per-(row, chunk)
// partial sums start in shared memory.
struct SegRange {
  int row0, row1;
  int wdelta;  // device row rt of the segment is row rt - wdelta of its weights (0 unless they are a shard)
  int part_base;
};

// ---- persistent decode-step kernel (hakm_step.cu) ----

// Tensor parallelism: device regions every GPU of a group can address in
// every other (identical sizes on all ranks, so an address moves to rank r
// by that region's byte offset).
constexpr int TP_MAX = 8;
enum XRegion { XR_LL = 0, XR_KCACHE = 1, XR_VCACHE = 2, XR_LOGITS = 3, XR_KEYS = 4, XR_XBAR = 5, XR_COUNT = 6 };
enum PhaseKind { PK_GEMV = 0, PK_ATTN = 1 };

// One phase of the device-resident step program. Phases exchange vectors as
// tagged words: uint64 = (tag << 32) | float bits, tag = tag_base + step *
// (n_phases + 1) + index of the writing phase (0 = embedding, prog[i] = i+1).
struct alignas(16) PhaseDesc {  // copied to shared memory as 16-byte words
  int kind;          // PhaseKind
  int skip_forced;   // skipped on forced (prompt) steps whose pick is not needed: lm_head
  PhaseParams g;     // PK_GEMV geometry, weights, biases, caches, norm and rope tables
  AttnParams a;      // PK_ATTN geometry, caches, split scratch (n_split / pos_dev / q / out unused)
  const uint64_t* x_ll;  // input vector (GEMV activation; attention q)
  int x_src;             // index of the phase that wrote it
  const uint64_t* res_ll;  // EPI_RESID: previous residual; attention: current k row
  int res_src;
  const uint64_t* v_ll;  // attention: current v row (written by phase x_src)
  uint64_t* out_ll[MAX_SEGS];  // per segment: q / v / xb / h; attention: att
  uint64_t* out2_ll;     // EPI_ROPE_QK: k
  int layer;             // attention: layer index (split tickets)
  // stage geometry of each GEMV segment (plan_step): rows per stage, row
  // bytes, chunks per row, and ceil(2^16 / chunks) for unit -> (group, chunk)
  int st_rows[MAX_SEGS], st_row_bytes[MAX_SEGS], st_nch[MAX_SEGS], st_rn[MAX_SEGS];
  int st_unit_rows[MAX_SEGS];  // rows per unit: 4, or 2 where a CTA holds few rows (shorter latency)
  // Q6_K segments whose CTAs hold a few long rows stream chunk by chunk: a
  // stage is st_chunk_rows[s] rows x one 8-block chunk, one 2-D tensor copy
  // through st_map[s] (two CUtensorMaps in device memory: boxes of
  // st_chunk_rows and st_chunk_rows - 4 rows, the second for CTAs with
  // fewer rows), so every row's chains run at once. 0: stages of whole rows.
  int st_chunk_rows[MAX_SEGS];
  const void* st_map[MAX_SEGS];
  // byte offset, within the shared activation region, of the per-thread
  // epilogue records (past this phase's activation); -1: no room, no records
  int epi_rec_off;
};


struct StepArgs {
  const PhaseDesc* prog;   // device array, n_phases entries (one decode step)
  int n_phases;
  int n_steps;             // decode steps run by the launch
  int pos0;                // position of step 0
  int n_forced;            // steps 0..n_forced-1 take forced[step] as input token
  const int* forced;
  int* token_dev;          // in: input of step 0 when n_forced == 0; out: last pick
  int* pos_dev;            // out: pos0 + n_steps
  long long kv_off;        // elements from the K/V cache pointers to this launch's sequence
  int* token_log;          // pick of step j at token_log[j - log_base] (may be null)
  int token_log_cap;
  int log_base;
  unsigned long long* keys;  // [3] running argmax keys, by step % 3
  unsigned int* bar;       // step barrier counter, zero at launch
  unsigned int* tickets;   // attention split tickets [n_kv], zero at launch, monotonic
  const SegRange* ranges;  // [n_phases][grid][MAX_SEGS]: each CTA's rows of each GEMV phase
  int* err_flag;
  const uint8_t* tok_embd; // Q6_K embedding rows (device layout)
  uint64_t* xb_ll;         // embedding output (xb buffer 0)
  float* xb_plain;         // final residual as plain floats (CTA 0, lm_head phase)
  int D;
  int n_layers;            // attention phases per step (split tickets)
  int skip_last;           // the last phase (lm_head) is skipped on forced steps but the last
  // tensor parallelism (tp_world 1: none). Rows of every GEMV phase are split
  // over the tp_world * grid CTAs of all GPUs; outputs go to every GPU.
  int tp_rank, tp_world;
  long long tp_delta[TP_MAX][XR_COUNT];  // byte offset from this GPU's region to rank r's
  unsigned int* xbar;      // cross-GPU step counter (XR_XBAR): +1 per GPU per step, never reset
  unsigned int xbar_base;  // steps completed before this launch
  int head_dim;            // attention head size (64 or 128): selects the kernel instance
  uint32_t tag_base;
  // shared-memory plan (plan_step)
  int n_stages, slot_bytes, region_bytes, part_floats;
  // measurement hook: per CTA and phase k < trace_k, %globaltimer stamps
  // [cta][k][4] = phase start, activation built, stages done, epilogue done
  unsigned long long* trace;
  int trace_k;
};

// Fills the shared-memory plan of `a` for this program (grid: the CTAs of all
// GPUs the rows split over); false if it cannot fit. With `chunked`, Q6_K
// segments of few long rows per CTA stream chunk by chunk (their
// st_chunk_rows set; the caller then supplies their tensor maps).
bool plan_step(PhaseDesc* prog_host, int n_phases, int grid, StepArgs& a, bool chunked = true);
// The row table of StepArgs::ranges for this program: the rows of CTAs
// cta0 .. cta0 + n_ctas - 1 of a grid of `grid` CTAs (all GPUs' CTAs).
void step_ranges(const PhaseDesc* prog_host, int n_phases, int grid, int cta0, int n_ctas, SegRange* out);
size_t step_smem_bytes(const StepArgs& a);
cudaError_t launch_step(const StepArgs& a, int grid, cudaStream_t s);
// Unpacks n tagged words into floats (debug reads of the exchange buffers).
cudaError_t launch_ll_unpack(float* out, const uint64_t* in, int n, cudaStream_t s);
constexpr int STEP_SMEM_MAX = 224 * 1024;  // dynamic; the opt-in limit (227 KB) also covers the ~2.2 KB static

}  // namespace hakm
