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
constexpr int Q6K_BODY = 208;      // packed device layout: {ql, qh, scales} per block
constexpr int ROWS_PER_CHUNK = 4;  // rows a warp reduces together
constexpr int MAX_SEGS = 3;

enum WType { W_Q4K = 12, W_Q6K = 14 };

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
  const uint8_t* w;      // Q4_K: verbatim rows; Q6_K: packed bodies
  const uint16_t* wd;    // Q6_K: fp16 d plane [n_rows][nb]
  const float* bias;     // device row order, may be null
  float* out;            // primary output
  float* out2;           // EPI_ROPE_QK: k output (rows >= split)
  float* cache;          // EPI_ROPE_QK: K cache layer base; EPI_V_CACHE: V cache base
  int type;
  int n_rows;
  int epi;
  int split;             // EPI_ROPE_QK: first k row (= q rows)
  int chunk_begin;       // first global chunk id of this segment
};

struct PhaseParams {
  int n_in;              // K (multiple of 256)
  int act;               // ActMode
  const float* x;        // ACT_F32 / ACT_RMS input
  const float* norm_w;   // ACT_RMS weight
  float eps;
  const int8_t* xq;      // ACT_Q8 input
  const float* xs;
  int need_q8;           // some segment is Q4_K (quantize in the prologue)
  int n_seg;
  Seg seg[MAX_SEGS];
  int total_chunks;
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
};

// ---- launchers (hakm_kernels.cu) ----
size_t phase_smem_bytes(const PhaseParams& p);
cudaError_t launch_phase(const PhaseParams& p, int grid, cudaStream_t s, bool pdl);
int phase_grid(const PhaseParams& p, int num_sms);

cudaError_t launch_quantize_q8(const float* x, int n, int8_t* xq, float* xs, cudaStream_t s);
cudaError_t launch_q4k_subsums(int32_t* iqx, int32_t* ix, const uint8_t* w, const int8_t* xq,
                               int n_out, int n_in, cudaStream_t s);
cudaError_t launch_q6k_pack(uint8_t* dst, const uint8_t* src, int n_rows, int n_in, cudaStream_t s);
cudaError_t launch_dequant(float* out, const uint8_t* w, int type, int n_rows, int n_in, cudaStream_t s);
cudaError_t launch_rmsnorm(float* y, const float* x, const float* w, int n, float eps, cudaStream_t s);
cudaError_t launch_embed_q6k(float* xb, const uint8_t* wb, const uint16_t* wd, const int* token,
                             int n_in, unsigned long long* argmax_key, cudaStream_t s, bool pdl);
cudaError_t launch_rope(float* x, const float* rope_cs, const int* pos_dev, int n_heads, int head_dim,
                        cudaStream_t s);

struct AttnParams {
  const float* q;        // [H*hd]
  const float* k_cache;  // layer base [max_seq][kv_dim]
  const float* v_cache;
  float* out;            // [H*hd]
  const int* pos_dev;    // attend over positions 0..pos
  int n_heads, n_kv, head_dim;
  float scale;
  int n_split;           // grid.y; chunks of ATTN_CHUNK positions
  float* part;           // scratch [n_kv][n_split][G][2 + hd]
  unsigned int* counters;  // [n_kv], self-resetting
};
constexpr int ATTN_CHUNK = 256;
cudaError_t launch_attention(const AttnParams& a, cudaStream_t s, bool pdl);
size_t attention_scratch_floats(int n_kv, int n_split, int group, int head_dim);

}  // namespace hakm
