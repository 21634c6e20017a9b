// Weight-side helpers of the projections whose weights live in parameter banks.
//
// bank_grad_acc: the weight-gradient GEMM of a bank-backed linear layer y = x (lam W)^T runs split along the token
// dimension (one fp32 partial product per split, written by the batched tcgen05 GEMM).  This kernel folds the
// splits and finishes the layer's parameter gradients in one pass over the weight-sized data:
//     dW      = sum_s parts[s]                         (unscaled: dy^T x)
//     grad   += lam * dW                               (bf16, in place, into up to two bank-gradient slices)
//     dlam    = <dW, W>                                (fp32; deterministic two-level reduction)
// It replaces a scaled copy of the weight, an fp32 product + reduction and one addcmul per slice
// (`train_gpt.py:1103`, `:1161`: the reference multiplies the weight by the scalar and lets autograd do this).
#include "api.h"
#include "ptx.cuh"

namespace mng {

constexpr int BGA_THREADS = 256;

__global__ void __launch_bounds__(BGA_THREADS)
bank_grad_acc_kernel(const float* __restrict__ parts, int S, long long n, const __nv_bfloat16* __restrict__ W,
                     const float* __restrict__ lam_ptr, __nv_bfloat16* __restrict__ g0, long long n0,
                     __nv_bfloat16* __restrict__ g1, float* __restrict__ partials, unsigned int* __restrict__ counter,
                     float* __restrict__ dlam) {
  const float lam = *lam_ptr;
  float dot = 0.f;
  for (long long i = ((long long)blockIdx.x * BGA_THREADS + threadIdx.x) * 8; i < n; i += (long long)gridDim.x * BGA_THREADS * 8) {
    float d[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) d[t] = 0.f;
    for (int s = 0; s < S; ++s) {
      const float4 a = *reinterpret_cast<const float4*>(parts + s * n + i);
      const float4 b = *reinterpret_cast<const float4*>(parts + s * n + i + 4);
      d[0] += a.x; d[1] += a.y; d[2] += a.z; d[3] += a.w;
      d[4] += b.x; d[5] += b.y; d[6] += b.z; d[7] += b.w;
    }
    const uint4 wu = *reinterpret_cast<const uint4*>(W + i);
    const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wu);
    __nv_bfloat16* g = i < n0 ? g0 + i : g1 + (i - n0);
    uint4 gu = *reinterpret_cast<const uint4*>(g);
    __nv_bfloat162* gh = reinterpret_cast<__nv_bfloat162*>(&gu);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 w = __bfloat1622float2(wh[t]);
      const float2 o = __bfloat1622float2(gh[t]);
      dot += d[2 * t] * w.x + d[2 * t + 1] * w.y;
      gh[t] = __floats2bfloat162_rn(o.x + lam * d[2 * t], o.y + lam * d[2 * t + 1]);
    }
    *reinterpret_cast<uint4*>(g) = gu;
  }
  // block sum -> partials[block]; the last block to finish adds the partials in index order
  __shared__ float red[BGA_THREADS / 32];
  __shared__ bool last;
  dot = warp_sum(dot);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = dot;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < BGA_THREADS / 32; ++w) s += red[w];
    partials[blockIdx.x] = s;
    __threadfence();
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x < 32) {
    __threadfence();
    float s = 0.f;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += 32) s += reinterpret_cast<volatile float*>(partials)[b];
    s = warp_sum(s);
    if (threadIdx.x == 0) {
      *dlam = s;
      *counter = 0;                                      // ready for the next launch on this stream
    }
  }
}

// Saturating e4m3 cast of src / scale (one static scale for the whole tensor, `train_gpt.py:78-79`) of a row-major
// bf16 [rows, cols] matrix, written as is (q, may be null) and / or transposed (qT [cols, rows], may be null) in one
// pass: 64 x 64 tiles through shared memory, 16-byte accesses on every side.  rows, cols multiples of 64.
__global__ void __launch_bounds__(256)
quant_static_dual_kernel(const __nv_bfloat16* __restrict__ src, uint8_t* __restrict__ q, uint8_t* __restrict__ qT, long long rows,
                         long long cols, float inv_scale) {
  __shared__ uint8_t tile[64][64 + 16];
  const long long r0 = (long long)blockIdx.y * 64, c0 = (long long)blockIdx.x * 64;
  const int a = threadIdx.x >> 2, seg = threadIdx.x & 3;            // row a of the tile, 16 columns from seg * 16
  const __nv_bfloat16* sp = src + (r0 + a) * cols + c0 + seg * 16;
  uint32_t w[4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 u = reinterpret_cast<const uint4*>(sp)[h];
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 f0 = __bfloat1622float2(b2[0]), f1 = __bfloat1622float2(b2[1]);
    const float2 f2 = __bfloat1622float2(b2[2]), f3 = __bfloat1622float2(b2[3]);
    w[2 * h] = (uint32_t)pack_e4m3x2(f0.x * inv_scale, f0.y * inv_scale) | ((uint32_t)pack_e4m3x2(f1.x * inv_scale, f1.y * inv_scale) << 16);
    w[2 * h + 1] = (uint32_t)pack_e4m3x2(f2.x * inv_scale, f2.y * inv_scale) | ((uint32_t)pack_e4m3x2(f3.x * inv_scale, f3.y * inv_scale) << 16);
  }
  const uint4 packed = make_uint4(w[0], w[1], w[2], w[3]);
  if (q) *reinterpret_cast<uint4*>(q + (r0 + a) * cols + c0 + seg * 16) = packed;
  if (qT) {
    *reinterpret_cast<uint4*>(&tile[a][seg * 16]) = packed;
    __syncthreads();
    uint8_t v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = tile[seg * 16 + j][a];
    *reinterpret_cast<uint4*>(qT + (c0 + a) * rows + r0 + seg * 16) = *reinterpret_cast<const uint4*>(v);
  }
}

}  // namespace mng

using namespace mng;

extern "C" int mng_quant_static_dual(const void* src, void* q, void* qT, long long rows, long long cols, float scale, void* stream) {
  if (rows <= 0 || cols <= 0 || (rows % 64) || (cols % 64) || rows / 64 > 65535 || scale <= 0.f) return -1;
  dim3 grid((unsigned)(cols / 64), (unsigned)(rows / 64));
  quant_static_dual_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)src, (uint8_t*)q, (uint8_t*)qT, rows, cols,
                                                                   1.f / scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// parts: [S, n] fp32; W: [n] bf16; g0 covers elements [0, n0), g1 (may be null when n0 == n) the rest.
// partials: `BANK_GRAD_BLOCKS` floats of scratch; counter: one zero-initialised word that the kernel leaves at zero.
extern "C" int mng_bank_grad_acc(const float* parts, int S, long long n, const void* W, const float* lam, void* g0,
                                 long long n0, void* g1, float* partials, unsigned int* counter, float* dlam, void* stream) {
  if (n <= 0 || (n % 8) || (n0 % 8) || n0 > n || S < 1 || (n0 < n && !g1)) return -1;
  long long want = (n / 8 + BGA_THREADS - 1) / BGA_THREADS;
  const int blocks = (int)(want < MNG_BANK_GRAD_BLOCKS ? want : MNG_BANK_GRAD_BLOCKS);
  bank_grad_acc_kernel<<<blocks, BGA_THREADS, 0, (cudaStream_t)stream>>>(
      parts, S, n, reinterpret_cast<const __nv_bfloat16*>(W), lam, reinterpret_cast<__nv_bfloat16*>(g0), n0,
      reinterpret_cast<__nv_bfloat16*>(g1), partials, counter, dlam);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
