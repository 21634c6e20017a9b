// C interface between the CUDA translation units and the Python binding.  Plain pointers and
// integers only, so the .cu files compile without the PyTorch headers.
#pragma once
#include <stdint.h>
#include "comm.h"

#ifdef __cplusplus
extern "C" {
#endif

enum { MNG_BF16 = 0, MNG_E4M3 = 1, MNG_E5M2 = 2 };
enum { MNG_EPI_STORE = 0, MNG_EPI_RELU2 = 1, MNG_EPI_DPRE = 2, MNG_EPI_NULL = 3 /* no output: profiling aid */ };

// D[b] = epi(A[b] (MxK) * B[b]^T (NxK)).  a_mn / b_mn: operand is stored [K, rows] instead of [rows, K].
typedef struct {
  const void* a;
  const void* b;
  int M, N, K, batch;
  int dtype_a, dtype_b;
  int a_mn, b_mn;
  long long lda, ldb;                 // row stride of the stored arrays, in elements
  long long a_bstride, b_bstride;     // batch strides in elements
  int epilogue;
  int bn;                             // CTA tile width: 128 or 256; 512 = 256 x 256 tile on a pair of CTAs (cta_group::2)
  int out_f32;
  void* out;
  long long ldc, c_bstride;
  const void* cin;                    // STORE: addend (beta); DPRE: saved post activations
  float alpha, beta;
  const float* alpha_ptr;             // optional device scalar folded into alpha
  const float* alpha2_ptr;            // a second one (STORE, DPRE)
  const float* beta_ptr;              // optional device scalar folded into beta (STORE)
  float* dot_out;                     // DPRE: *dot_out += sum(acc * post) over the whole product (fp32 atomics), or null
  void* out2;                         // epilogues that split the N columns over several [M, out_cols] outputs
  void* out3;
  int out_cols;
  const float* row_scale;
  const float* col_scale;
  void* out8;                         // RELU2: e4m3 copy of the output
  const float* act_scale;
  unsigned int* amax_bits;
  int max_ctas;                       // 0 = one CTA per SM
  int symmetric;                      // STORE, M == N a multiple of 128: the product is symmetric; only the upper-triangular
                                      // 128 x 128 tiles are computed and every off-diagonal tile is stored twice
  void* stream;
  uint32_t* status;
} GemmDesc;

int mng_gemm(const GemmDesc* g);

// ---- pointwise / normalisation (pointwise.cu) ---------------------------------------------------
// y = x / rms(x) per row of `cols` bf16 elements; optional e4m3 copy with one scale per row
// (scale = amax/448) for the row-scaled FP8 GEMMs.
int mng_rmsnorm_fwd(const void* x, void* y, void* y8, float* row_scale, float* rstd, long long rows, int cols, void* stream);
int mng_rmsnorm_bwd(const void* x, const void* dy, const float* rstd, void* dx, long long rows, int cols, int accumulate,
                    void* stream);
int mng_rmsnorm_bwd_add(const void* x, const void* dy, const float* rstd, const void* addend, void* dx, long long rows,
                        int cols, void* stream);
// dx = norm backward + (*addend_scale) * addend; *dot_out += sum(addend * x)  (fp32 atomics, one per block).
int mng_rmsnorm_bwd_add_scaled(const void* x, const void* dy, const float* rstd, const void* addend,
                               const float* addend_scale, float* dot_out, void* dx, long long rows, int cols, void* stream);
// Row-wise e4m3 quantisation: q = x / s, s[r] = amax(x[r,:])/448 (bf16 in).
int mng_quant_rows_e4m3(const void* x, void* q, float* scale, long long rows, int cols, void* stream);
// dst[c, r] = src[r, c] (optionally += ), bf16; 32x32 tiles through shared memory.
int mng_transpose_bf16(const void* src, void* dst, long long rows, long long cols, int accumulate, void* stream);
// dst[c, r] = src[r, c] for 1-byte elements (fp8 activations); rows, cols multiples of 64.
int mng_transpose_u8(const void* src, void* dst, long long rows, long long cols, void* stream);
// Row-scaled e4m3 quantisation of the transpose: q[c, :] = src[:, c] / s[c], s[c] = amax(src[:, c]) / 448.
// `amax_scratch`: `cols` 32-bit words of scratch memory owned by the caller.
int mng_quant_transpose_e4m3(const void* src, void* q, float* scale, unsigned int* amax_scratch, long long rows,
                             long long cols, void* stream);

// All FP8 copies of a [layers, 2, hid, dim] bf16 MLP bank in one call (five launches): fc8 [layers, hid, dim] with
// fc_scale [layers, hid]; projT8 [layers, dim, hid] with projT_scale [layers, dim]; act_scale / amax_bits / used /
// next: [layers].  amax_scratch: layers * dim words.
int mng_mlp_weight_refresh(const void* bank, int layers, int hid, int dim, void* fc8, float* fc_scale, void* projT8,
                           float* projT_scale, unsigned int* amax_scratch, float* act_scale, unsigned int* amax_bits,
                           float* used_scales, float* next_scales, int bootstrap, void* stream);

// Saturating static-scale e4m3 cast of a bf16 [rows, cols] matrix, as is (q) and / or transposed (qT); either may be
// null.  rows, cols multiples of 64.
int mng_quant_static_dual(const void* src, void* q, void* qT, long long rows, long long cols, float scale, void* stream);

// lm_head GEMM fused with the soft-capped cross entropy: no [T, V] logits in memory.  x8 [T, K], wT8 [V, K] e4m3;
// losses [T] fp32; dlogits [T, V] e5m2 (times grad_mul); scratch: slab_sum T * ceil(V/128), ztgt T * 4, rowc T floats.
// n_predict <= 3.
int mng_lmhead_ce_fused(const void* x8, const void* wT8, int T, int V, int K, float alpha, const long long* targets,
                        const float* mtp_w, int n_predict, const long long* prefix_targets, const float* prefix_w, float A,
                        float B, float C, float grad_mul, float* losses, void* dlogits_e5m2, float* slab_sum, float* ztgt,
                        float* rowc, void* stream, uint32_t* status);

// QKV projection with the attention pre-processing in its epilogue (epi_qkv.cuh): x [T, K] bf16, w [3*H*128, K] bf16
// (rows ordered q heads, k heads, v heads) -> q, k, v [T, H*128] bf16, rstd_q / rstd_k [T, H] fp32, k_last [H, 64] bf16.
// lam: device scalar multiplied into the projection; cos_t / sin_t: fp32 [positions, 32]; ve / vgate optional.
int mng_qkv_proj(const void* x, const void* w, int T, int K, int H, const float* lam, const float* cos_t, const float* sin_t,
                 const void* ve, const void* vgate, int vgate_stride, void* q, void* k, void* v, float* rstd_q, float* rstd_k,
                 void* k_last, int paired, int key_offset, void* stream, uint32_t* status);
// Backward of the pre-processing from its outputs (no copy of the raw projection is kept): d_qkv [T, 3*H*128].
int mng_qkv_post_bwd_from_out(const void* q, const void* k, const void* k_last, const float* cos_t, const float* sin_t,
                              const float* rstd_q, const float* rstd_k, const void* dq, const void* dk, const void* dv,
                              const void* ve, const void* vgate, int vgate_stride, void* d_qkv, void* d_ve, void* d_vgate,
                              int d_vgate_stride, long long T, int H, int paired, int key_offset, void* stream);

// ---- softcapped cross entropy (ce.cu) -------------------------------------------------------------
// One CTA per token row: z = A*sigmoid((logit+B)/C), loss = sum_k w_k (lse - z[t_{i+k}]) + w_p (lse - z[p_i]),
// dlogits (e5m2 or bf16) = grad_mul * d loss / d logit.
int mng_softcap_ce(const void* logits_bf16, const long long* targets, const float* mtp_weights, int n_predict,
                   const long long* prefix_targets, const float* prefix_weight, float* losses, void* dlogits,
                   int dlogits_is_e5m2, long long rows, int vocab, long long ld_logits, float A, float B, float C,
                   float grad_mul, void* stream);

// ---- optimizer (optim.cu) ---------------------------------------------------------------------------
// Gradients are summed over `grads.n` ranks' buffers (peer pointers) and scaled by grad_mul; updated
// values are stored to every buffer in `params`.  `off` = element offset of this rank's shard.
typedef struct {
  PeerPtrs grads;
  PeerPtrs params;
  long long off;
  float* exp_avg;
  float* exp_avg_sq;
  long long n;
  int p_is_f32;
  float beta1, beta2, eps, step_size, eff_wd, grad_mul;
  // Row masks (optional, local memory): row_mask[r * mask_stride + row] != 0 iff rank r's gradient row `row` (rows of
  // row_elems elements, counted from the parameter's start) may be non-zero.  Rows whose byte is 0 are not loaded from
  // rank r at all: a sparse pull over NVLink for embedding-type gradients.  row_elems must be a multiple of 8.
  const unsigned char* row_mask;
  long long mask_stride;
  int row_elems;
} AdamDesc;
int mng_adam(const AdamDesc* d, void* stream);

// One launch for up to MNG_SMALL_ADAM_MAX small replicated parameters.  base: the address of one buffer (an arena) on every
// rank, or a single null entry when p_off / g_off are absolute addresses; each rank reads all ranks' gradients and updates
// its own copy.
#define MNG_SMALL_ADAM_MAX 16
typedef struct {
  long long p_off, g_off;   // byte offsets of the parameter and of its gradient from base
  float* m;
  float* v;
  long long n;
  int is_f32;               // parameter and gradient dtype: fp32 or bf16
  float beta1, beta2, eps, step_size, eff_wd;
} SmallAdamEntry;
typedef struct {
  PeerPtrs base;
  int count;
  float gmul;               // gradient multiplier (1 / ranks)
  SmallAdamEntry e[MNG_SMALL_ADAM_MAX];
} SmallAdamTable;
int mng_adam_small(const SmallAdamTable* t, void* stream);
int mng_fill_zero(void* p, long long bytes, void* stream);

//   g = bf16(grad_mul * sum_r grads[r]); buf = lerp(buf, g, 1-mu); u = lerp(g, buf, mu);
//   out = bf16(u); sumsq[mat] = sum(out^2)
int mng_nesterov(const PeerPtrs* grads, long long off, float* buf, void* out_bf16, float* sumsq, long long mats,
                 long long per_mat, float momentum, float grad_mul, void* stream);
// x[mat] /= bf16(bf16(||x[mat]||_F) * 1.02) + 1e-6   (bf16, in place)
int mng_scale_by_norm(void* x_bf16, const float* sumsq, long long mats, long long per_mat, void* stream);
// NorMuon second-moment normalisation + cautious weight decay on bf16 weight + uint16 mantissa.
//   red_rows != 0: statistics per row (reduce over columns), else per column (reduce over rows).
//   scale_scratch: mats * (max(rows, cols) + 65) floats, all zero before the first call (the kernels leave the
//   counters at its end zero again).  Learning rate of matrix m = lr_base * lr_mul_per_mat[m].
int mng_normuon_apply(const PeerPtrs* params, long long off, void* mantissa_u16, const void* v_bf16, float* second_mom,
                      float* scale_scratch, long long mats, int rows, int cols, int red_rows, float beta2, float eff_wd,
                      float lr_base, const float* lr_mul_per_mat, void* stream);
// ---- fused glue (glue.cu) -----------------------------------------------------------------------------
#define LC_MAX_TERMS 6
typedef struct {
  const void* x;            // [rows, cols] bf16
  const float* scalar;      // device scalar s (null = 1)
  const void* gate;         // per-row coefficient source g (null = 1): element [row*gate_stride + gate_col]
  long long gate_stride;
  int gate_col;
  int gate_bf16;            // gate dtype: 1 = bf16, 0 = fp32
  float addc;               // coefficient = addc + s * g(row)
} LinTerm;
typedef struct { LinTerm t[LC_MAX_TERMS]; int k; } LinCombArgs;
typedef struct {
  void* dx;                 // [rows, cols] bf16 or null
  int dx_accumulate;        // 1: dx += coefficient * g (dx holds the contributions of earlier calls), 0: dx = ...
  void* dgate;              // bf16 buffer (zero-initialised by the caller) or null; written at [row*stride + col]
  long long dgate_stride;
  int dgate_col;
  float* dscalar;           // fp32 accumulator (zeroed by the caller) or null
} LinGrad;
typedef struct { LinGrad t[LC_MAX_TERMS]; } LinCombGrads;
int mng_lincomb_fwd(const LinCombArgs* a, void* out, long long rows, int cols, void* stream);
int mng_lincomb_bwd(const LinCombArgs* a, const LinCombGrads* g, const void* gout, long long rows, int cols, void* stream);

int mng_qkv_post_fwd(const void* qkv, const float* cos_t, const float* sin_t, const void* ve, const void* vgate,
                     int vgate_stride, const void* vadd, void* q, void* k, void* v, float* rstd_q, float* rstd_k,
                     long long T, int H, int paired, int key_offset, int split, void* stream);
int mng_qkv_post_bwd(const void* qkv, const float* cos_t, const float* sin_t, const float* rstd_q, const float* rstd_k,
                     const void* dq, const void* dk, const void* dv, const void* ve, const void* vgate, int vgate_stride,
                     void* d_qkv, void* d_ve, void* d_vgate, int d_vgate_stride, long long T, int H, int paired,
                     int key_offset, int split, void* stream);
int mng_xsa_gate_fwd(const void* y, const void* v, const void* alpha, int alpha_stride, const void* gate, int gate_stride,
                     void* out, long long T, int H, void* stream);
int mng_xsa_gate_bwd(const void* y, const void* v, const void* alpha, int alpha_stride, const void* gate, int gate_stride,
                     const void* dout, void* dy, void* dv, void* dalpha, int dalpha_stride, void* dgate, int dgate_stride,
                     long long T, int H, void* stream);

// ---- weight-side helpers (weights.cu) ------------------------------------------------------------------
// dW = sum_s parts[s] (fp32 [S, n]); grad (bf16, slices g0 = elements [0, n0), g1 = the rest) += lam * dW;
// *dlam = <dW, W>.  partials: MNG_BANK_GRAD_BLOCKS floats of scratch; counter: one word, zero before and after.
#define MNG_BANK_GRAD_BLOCKS 592
int mng_bank_grad_acc(const float* parts, int S, long long n, const void* W, const float* lam, void* g0, long long n0,
                      void* g1, float* partials, unsigned int* counter, float* dlam, void* stream);

// ---- gate / MUDD MLP tail (gatemlp.cu): out = (gelu(pre) W2^T + b2) * scale, pre [rows, 64], n <= 48 outputs --------
// scale = *scale_ptr (rounded to bf16) when scale_ptr is given, else scale_const.
#define MNG_GATE_TAIL_BLOCKS 296
int mng_gate_tail_fwd(const void* pre, const void* W2, long long w2_ld, const void* b2, const float* scale_ptr,
                      float scale_const, void* out, long long rows, int n, void* stream);
// dpre [rows, 64] bf16; dW2 [n, 64] and db2 [n] bf16; *dscale fp32 (may be null).
// partials: MNG_GATE_TAIL_BLOCKS * (n*64 + n + 1) floats of scratch.
int mng_gate_tail_bwd(const void* pre, const void* W2, long long w2_ld, const void* b2, const float* scale_ptr,
                      float scale_const, const void* dout, long long dout_ld, void* dpre, float* partials, void* dW2,
                      long long dw2_ld, void* db2, float* dscale, long long rows, int n, void* stream);

// ---- DC cross-head mixing (dc.cu) ---------------------------------------------------------------------
int mng_dc_mix_fwd(const float* S, const void* w1, const int* doc_start, void* P, void* a, long long T, int H, int window,
                   void* stream);
int mng_dc_fold(const void* part, void* out, long long T, int H, void* stream);
int mng_dc_mix_bwd(const float* dM, const void* P, const void* a, const void* w1, const void* w2, void* dS, float* g_w1,
                   float* g_w2, long long T, int H, float scale, void* stream);

// ---- embedding backward (embed.cu): grad[sorted_ids[j], :] += g[perm[j], :], accumulated in place (bf16) ----
int mng_embed_bwd(const void* g, const long long* sorted_ids, const long long* perm, void* grad, long long n, int D,
                  long long table_rows, void* stream);

// Debug build (-DMNG_BOUNDS_CHECK): source line of the last out-of-range index seen by the kernels of a translation
// unit since the previous query (0 = none; always 0 in the regular build).
unsigned int mng_bounds_embed(void);
unsigned int mng_bounds_glue(void);
unsigned int mng_bounds_dc(void);
unsigned int mng_bounds_optim(void);

// ---- attention forward (attn_sm100.cu) ------------------------------------------------------------------
// q, k, v: [T, H, 128] bf16 with token stride `row_stride` elements (heads contiguous); doc_start[i] = first token of
// i's document; keys j with max(doc_start[i], i - window) <= j <= i.  out [T, H, 128] bf16 contiguous, lse [H, T] fp32.
int mng_attn_fwd(const void* q, const void* k, const void* v, const int* doc_start, void* out, float* lse, int T, int H,
                 long long row_stride, int window, float scale, void* stream, uint32_t* status);

// Backward of the same attention: dq, dk, dv [T, H, 128] bf16 contiguous from q, k, v, the forward's out and lse and
// the incoming gradient dout (contiguous).  doc_end[i] = first token of the next document.  delta, lse2: [H, T] fp32
// scratch owned by the caller.  T must be a multiple of 4.
int mng_attn_bwd(const void* q, const void* k, const void* v, const void* out, const void* dout, const float* lse,
                 const int* doc_start, const int* doc_end, void* dq, void* dk, void* dv, float* delta, float* lse2, int T,
                 int H, long long row_stride, int window, float scale, void* stream, uint32_t* status);

// Barrier across ranks on signal pads (bounded wait; sets *status on expiry).
int mng_peer_barrier(const PeerPtrs* pads, int rank, uint32_t epoch, uint32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
