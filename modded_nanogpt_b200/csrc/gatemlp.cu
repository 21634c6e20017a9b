// Tail of the small gate / MUDD MLPs: out = (gelu(pre) W2^T + b2) * scale for pre = x W1^T of width 64 and at most
// 48 outputs per token (`train_gpt.py:1465-1467` gate MLPs with 26 / 41 coefficients, `:1601-1610`, `:1677-1680`
// MUDD with 14 / 5).  The wide product x W1^T (and its two backward products) run on the tcgen05 GEMM; everything
// after it is one kernel per direction here, so neither the hidden activation nor its gradient with respect to the
// activation ever exist in global memory.
//
// Rounding points follow the op-by-op bf16 evaluation: h = bf16(gelu(pre)), y = bf16(h W2^T), y = bf16(y + b2),
// out = bf16(y * scale).
#include "api.h"
#include "ptx.cuh"

namespace mng {

constexpr int GM_HID = 64;
constexpr int GM_MAX_OUT = 48;
constexpr int GM_ROWS = 128;                 // rows (= threads) per block

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16(v)); }
__device__ __forceinline__ float gelu_f(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }
__device__ __forceinline__ float gelu_grad_f(float x) {
  return 0.5f * (1.f + erff(x * 0.70710678118654752f)) + x * 0.3989422804014327f * __expf(-0.5f * x * x);
}

__device__ __forceinline__ void load_row64(const __nv_bfloat16* p, float (&v)[GM_HID]) {
#pragma unroll
  for (int c = 0; c < GM_HID / 8; ++c) {
    const uint4 u = reinterpret_cast<const uint4*>(p)[c];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 f = __bfloat1622float2(h[t]);
      v[c * 8 + 2 * t] = f.x;
      v[c * 8 + 2 * t + 1] = f.y;
    }
  }
}

__global__ void __launch_bounds__(GM_ROWS)
gate_tail_fwd_kernel(const __nv_bfloat16* __restrict__ pre, const __nv_bfloat16* __restrict__ W2, long long w2_ld,
                     const __nv_bfloat16* __restrict__ b2, const float* __restrict__ scale_ptr, float scale_const,
                     __nv_bfloat16* __restrict__ out, long long rows, int n) {
  __shared__ float w2s[GM_MAX_OUT][GM_HID];
  __shared__ float b2s[GM_MAX_OUT];
  for (int i = threadIdx.x; i < n * GM_HID; i += GM_ROWS) w2s[i / GM_HID][i % GM_HID] = __bfloat162float(W2[(i / GM_HID) * w2_ld + i % GM_HID]);
  for (int i = threadIdx.x; i < n; i += GM_ROWS) b2s[i] = __bfloat162float(b2[i]);
  __syncthreads();
  const float scale = scale_ptr ? bf16r(*scale_ptr) : scale_const;
  const long long row = (long long)blockIdx.x * GM_ROWS + threadIdx.x;
  if (row >= rows) return;
  float h[GM_HID];
  load_row64(pre + row * GM_HID, h);
#pragma unroll
  for (int j = 0; j < GM_HID; ++j) h[j] = bf16r(gelu_f(h[j]));
  __nv_bfloat16* o = out + row * n;
  for (int i = 0; i < n; ++i) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < GM_HID; ++j) acc += h[j] * w2s[i][j];
    o[i] = __float2bfloat16(bf16r(bf16r(acc) + b2s[i]) * scale);
  }
}

// Backward of the tail.  Per row: do_i = dout_i * scale, dh_j = sum_i do_i W2[i][j], dpre_j = dh_j gelu'(pre_j).
// Per block (persistent over row chunks): partial sums of dW2 = do^T h, db2 = sum do, dscale = sum dout_i y_i, kept in
// registers across chunks and written once to `partials[block][n*64 + n + 1]`.  The block-level products use a
// 6 x 4 register tile per thread (8 x 16 threads cover 48 x 64 outputs) over the chunk's rows staged in shared memory.
constexpr int GM_DO_LD = GM_MAX_OUT + 1, GM_H_LD = GM_HID + 1;

__global__ void __launch_bounds__(GM_ROWS)
gate_tail_bwd_kernel(const __nv_bfloat16* __restrict__ pre, const __nv_bfloat16* __restrict__ W2, long long w2_ld,
                     const __nv_bfloat16* __restrict__ b2, const float* __restrict__ scale_ptr, float scale_const,
                     const __nv_bfloat16* __restrict__ dout, long long dout_ld, __nv_bfloat16* __restrict__ dpre,
                     float* __restrict__ partials, long long rows, int n) {
  extern __shared__ float gm_smem[];
  float (*w2s)[GM_HID] = reinterpret_cast<float (*)[GM_HID]>(gm_smem);                 // [48][64]
  float* b2s = gm_smem + GM_MAX_OUT * GM_HID;                                          // [48]
  float* do_s = b2s + GM_MAX_OUT;                                                      // [128][49]
  float* h_s = do_s + GM_ROWS * GM_DO_LD;                                              // [128][65]
  float* red = h_s + GM_ROWS * GM_H_LD;                                                // [4]
  for (int i = threadIdx.x; i < GM_MAX_OUT * GM_HID; i += GM_ROWS)
    w2s[i / GM_HID][i % GM_HID] = (i / GM_HID) < n ? __bfloat162float(W2[(i / GM_HID) * w2_ld + i % GM_HID]) : 0.f;
  for (int i = threadIdx.x; i < GM_MAX_OUT; i += GM_ROWS) b2s[i] = i < n ? __bfloat162float(b2[i]) : 0.f;
  const float scale = scale_ptr ? bf16r(*scale_ptr) : scale_const;
  const int ti = threadIdx.x >> 4, tj = threadIdx.x & 15;       // register tile: outputs i in [6 ti, +6), j in [4 tj, +4)
  float accw[6][4], accb[6];
#pragma unroll
  for (int a = 0; a < 6; ++a) {
    accb[a] = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) accw[a][b] = 0.f;
  }
  float dsc = 0.f;
  __syncthreads();

  const long long chunks = (rows + GM_ROWS - 1) / GM_ROWS;
  for (long long ch = blockIdx.x; ch < chunks; ch += gridDim.x) {
    const long long row = ch * GM_ROWS + threadIdx.x;
    const bool live = row < rows;
    float h[GM_HID], dh[GM_HID];
#pragma unroll
    for (int j = 0; j < GM_HID; ++j) { h[j] = 0.f; dh[j] = 0.f; }
    if (live) {
      load_row64(pre + row * GM_HID, h);
#pragma unroll
      for (int j = 0; j < GM_HID; ++j) h[j] = bf16r(gelu_f(h[j]));
    }
#pragma unroll
    for (int j = 0; j < GM_HID; ++j) h_s[threadIdx.x * GM_H_LD + j] = h[j];
    for (int i = 0; i < GM_MAX_OUT; ++i) {
      float d = 0.f;
      if (i < n) {
        const float g = live ? __bfloat162float(dout[row * dout_ld + i]) : 0.f;
        d = g * scale;
        float y = 0.f;
#pragma unroll
        for (int j = 0; j < GM_HID; ++j) {
          dh[j] += d * w2s[i][j];
          y += h[j] * w2s[i][j];
        }
        dsc += g * bf16r(bf16r(y) + b2s[i]);
      }
      do_s[threadIdx.x * GM_DO_LD + i] = d;
    }
    if (live) {
      float p[GM_HID];
      load_row64(pre + row * GM_HID, p);
      uint4* o = reinterpret_cast<uint4*>(dpre + row * GM_HID);
#pragma unroll
      for (int c = 0; c < GM_HID / 8; ++c) {
        float v[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = dh[c * 8 + t] * gelu_grad_f(p[c * 8 + t]);
        uint4 w;
        w.x = pack_bf16x2(v[0], v[1]); w.y = pack_bf16x2(v[2], v[3]); w.z = pack_bf16x2(v[4], v[5]); w.w = pack_bf16x2(v[6], v[7]);
        o[c] = w;
      }
    }
    __syncthreads();
    for (int r = 0; r < GM_ROWS; ++r) {
      float dv[6], hv[4];
#pragma unroll
      for (int a = 0; a < 6; ++a) dv[a] = do_s[r * GM_DO_LD + ti * 6 + a];
#pragma unroll
      for (int b = 0; b < 4; ++b) hv[b] = h_s[r * GM_H_LD + tj * 4 + b];
#pragma unroll
      for (int a = 0; a < 6; ++a) {
        accb[a] += dv[a];
#pragma unroll
        for (int b = 0; b < 4; ++b) accw[a][b] += dv[a] * hv[b];
      }
    }
    __syncthreads();
  }
  const int n_out = n * GM_HID + n;
  float* mine = partials + (long long)blockIdx.x * (n_out + 1);
#pragma unroll
  for (int a = 0; a < 6; ++a) {
    const int i = ti * 6 + a;
    if (i < n) {
#pragma unroll
      for (int b = 0; b < 4; ++b) mine[i * GM_HID + tj * 4 + b] = accw[a][b];
      if (tj == 0) mine[n * GM_HID + i] = accb[a];
    }
  }
  dsc = warp_sum(dsc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = dsc;
  __syncthreads();
  if (threadIdx.x == 0) mine[n_out] = red[0] + red[1] + red[2] + red[3];
}

// out[k] = sum_b partials[b][k] in block order (deterministic); dW2 / db2 entries to bf16, dscale to fp32.
__global__ void gate_tail_reduce_kernel(const float* __restrict__ partials, int blocks, int n_out, __nv_bfloat16* __restrict__ dW2,
                                        long long dw2_ld, int n, __nv_bfloat16* __restrict__ db2, float* __restrict__ dscale) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k > n_out) return;
  float s = 0.f;
  for (int b = 0; b < blocks; ++b) s += partials[(long long)b * (n_out + 1) + k];
  if (k < n * GM_HID) dW2[(k / GM_HID) * dw2_ld + k % GM_HID] = __float2bfloat16(s);
  else if (k < n_out) db2[k - n * GM_HID] = __float2bfloat16(s);
  else if (dscale) *dscale = s;
}

constexpr int GM_BWD_SMEM = (GM_MAX_OUT * GM_HID + GM_MAX_OUT + GM_ROWS * GM_DO_LD + GM_ROWS * GM_H_LD + 4) * 4;

}  // namespace mng

using namespace mng;

extern "C" int mng_gate_tail_fwd(const void* pre, const void* W2, long long w2_ld, const void* b2, const float* scale_ptr,
                                 float scale_const, void* out, long long rows, int n, void* stream) {
  if (n < 1 || n > GM_MAX_OUT || rows <= 0) return -1;
  gate_tail_fwd_kernel<<<(unsigned)((rows + GM_ROWS - 1) / GM_ROWS), GM_ROWS, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(pre), reinterpret_cast<const __nv_bfloat16*>(W2), w2_ld,
      reinterpret_cast<const __nv_bfloat16*>(b2), scale_ptr, scale_const, reinterpret_cast<__nv_bfloat16*>(out), rows, n);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// partials: MNG_GATE_TAIL_BLOCKS * (n*64 + n + 1) floats of scratch.  dW2 [n, 64] (row pitch dw2_ld), db2 [n] bf16;
// dscale fp32 or null.
extern "C" int mng_gate_tail_bwd(const void* pre, const void* W2, long long w2_ld, const void* b2, const float* scale_ptr,
                                 float scale_const, const void* dout, long long dout_ld, void* dpre, float* partials,
                                 void* dW2, long long dw2_ld, void* db2, float* dscale, long long rows, int n, void* stream) {
  if (n < 1 || n > GM_MAX_OUT || rows <= 0) return -1;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(gate_tail_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GM_BWD_SMEM) != cudaSuccess) return -3;
    attr = true;
  }
  long long chunks = (rows + GM_ROWS - 1) / GM_ROWS;
  const int blocks = (int)(chunks < MNG_GATE_TAIL_BLOCKS ? chunks : MNG_GATE_TAIL_BLOCKS);
  cudaStream_t st = (cudaStream_t)stream;
  gate_tail_bwd_kernel<<<blocks, GM_ROWS, GM_BWD_SMEM, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(pre), reinterpret_cast<const __nv_bfloat16*>(W2), w2_ld,
      reinterpret_cast<const __nv_bfloat16*>(b2), scale_ptr, scale_const, reinterpret_cast<const __nv_bfloat16*>(dout), dout_ld,
      reinterpret_cast<__nv_bfloat16*>(dpre), partials, rows, n);
  const int n_out = n * GM_HID + n;
  gate_tail_reduce_kernel<<<(n_out + 1 + 127) / 128, 128, 0, st>>>(partials, blocks, n_out, reinterpret_cast<__nv_bfloat16*>(dW2),
                                                                  dw2_ld, n, reinterpret_cast<__nv_bfloat16*>(db2), dscale);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
