// Bandwidth-bound row kernels: RMSNorm forward (with fused row-scaled e4m3 quantisation for the
// FP8 GEMMs) and backward, row quantisation, tiled transposes.  One warp per row, 16-byte accesses.
#include "api.h"
#include "ptx.cuh"

namespace mng {

constexpr int ROW_WARPS = 8;

// cols must be a multiple of 256 (32 lanes x 8 bf16) and <= 256 * MAXV.
template <int MAXV>
__global__ void __launch_bounds__(ROW_WARPS * 32)
rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, uint8_t* __restrict__ y8,
                   float* __restrict__ row_scale, float* __restrict__ rstd_out, long long rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nv = cols >> 8;
  const __nv_bfloat16* xr = x + row * cols;
  float v[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (i < nv) {
      uint4 u = *reinterpret_cast<const uint4*>(xr + (i * 32 + lane) * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float2 f = __bfloat1622float2(h[t]);
        v[i][2 * t] = f.x; v[i][2 * t + 1] = f.y;
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / cols + eps);
  if (rstd_out && lane == 0) rstd_out[row] = rstd;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (i < nv) {
      uint4 w;
      uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        __nv_bfloat162 b = __floats2bfloat162_rn(v[i][2 * t] * rstd, v[i][2 * t + 1] * rstd);
        wp[t] = *reinterpret_cast<uint32_t*>(&b);
        float2 f = __bfloat1622float2(b);          // quantise what the bf16 consumer would see
        v[i][2 * t] = f.x; v[i][2 * t + 1] = f.y;
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
      if (y) *reinterpret_cast<uint4*>(y + row * cols + (i * 32 + lane) * 8) = w;
    }
  }
  if (y8) {
    amax = fmaxf(warp_max(amax), 1e-12f);
    const float s = amax / 448.f, inv = 448.f / amax;
    if (lane == 0) row_scale[row] = s;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (i < nv) {
        uint2 w;
        w.x = pack_e4m3x2(v[i][0] * inv, v[i][1] * inv) | ((uint32_t)pack_e4m3x2(v[i][2] * inv, v[i][3] * inv) << 16);
        w.y = pack_e4m3x2(v[i][4] * inv, v[i][5] * inv) | ((uint32_t)pack_e4m3x2(v[i][6] * inv, v[i][7] * inv) << 16);
        *reinterpret_cast<uint2*>(y8 + row * cols + (i * 32 + lane) * 8) = w;
      }
    }
  }
}

// dx = rstd * (dy - xhat * mean(dy * xhat)) [+ s * addend],  xhat = x * rstd.   `addend` may be `dx` itself (accumulate).
// s = *addend_scale (1 when null).  With dot_out, *dot_out += sum(addend * x) over all rows: when the addend is the
// gradient g of y = s * x + ..., that sum is the gradient of s.
template <int MAXV>
__global__ void __launch_bounds__(ROW_WARPS * 32)
rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy, const float* __restrict__ rstd_in,
                   const __nv_bfloat16* addend, __nv_bfloat16* dx, long long rows, int cols, float eps,
                   const float* __restrict__ addend_scale = nullptr, float* __restrict__ dot_out = nullptr) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  __shared__ float blk_dot[ROW_WARPS];
  if (dot_out) {                                        // block-uniform: every warp takes part in the block sum
    if (lane == 0) blk_dot[threadIdx.x >> 5] = 0.f;
  }
  const float as = addend_scale ? *addend_scale : 1.f;
  float adot = 0.f;
  if (row < rows) {
  const int nv = cols >> 8;
  float xv[MAXV][8], gv[MAXV][8];
  uint4 old[MAXV];                                        // the addend is loaded with x and dy, not after the row sums
  float ss = 0.f, dot = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
    if (i < nv && addend) old[i] = *reinterpret_cast<const uint4*>(addend + row * cols + (i * 32 + lane) * 8);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (i < nv) {
      uint4 u = *reinterpret_cast<const uint4*>(x + row * cols + (i * 32 + lane) * 8);
      uint4 g = *reinterpret_cast<const uint4*>(dy + row * cols + (i * 32 + lane) * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
      const __nv_bfloat162* k = reinterpret_cast<const __nv_bfloat162*>(&g);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float2 a = __bfloat1622float2(h[t]), b = __bfloat1622float2(k[t]);
        xv[i][2 * t] = a.x; xv[i][2 * t + 1] = a.y; gv[i][2 * t] = b.x; gv[i][2 * t + 1] = b.y;
        ss += a.x * a.x + a.y * a.y;
        dot += a.x * b.x + a.y * b.y;
      }
    }
  }
  ss = warp_sum(ss);
  dot = warp_sum(dot);
  const float rstd = rstd_in ? rstd_in[row] : rsqrtf(ss / cols + eps);
  const float c = dot * rstd * rstd * rstd / cols;       // mean(dy*xhat) * rstd, with xhat = x*rstd
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (i < nv) {
      __nv_bfloat16* o = dx + row * cols + (i * 32 + lane) * 8;
      float r[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) r[t] = gv[i][t] * rstd - xv[i][t] * c;
      if (addend) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&old[i]);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float2 f = __bfloat1622float2(h[t]);
          r[2 * t] += as * f.x; r[2 * t + 1] += as * f.y;
          adot += f.x * xv[i][2 * t] + f.y * xv[i][2 * t + 1];
        }
      }
      uint4 w;
      w.x = pack_bf16x2(r[0], r[1]); w.y = pack_bf16x2(r[2], r[3]); w.z = pack_bf16x2(r[4], r[5]); w.w = pack_bf16x2(r[6], r[7]);
      *reinterpret_cast<uint4*>(o) = w;
    }
  }
  }
  if (dot_out) {
    adot = warp_sum(adot);
    if (lane == 0) blk_dot[threadIdx.x >> 5] = adot;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < ROW_WARPS; ++w) s += blk_dot[w];
      atomicAdd(dot_out, s);
    }
  }
}

template <int MAXV>
__global__ void __launch_bounds__(ROW_WARPS * 32)
quant_rows_kernel(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ q, float* __restrict__ scale, long long rows, int cols,
                  long long group_rows, long long group_stride) {
  // source row r lives at x + (r / group_rows) * group_stride + (r % group_rows) * cols: lets one launch walk the
  // [hid, dim] matrices of a [layers, 2, hid, dim] parameter bank; outputs are dense
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  x += (row / group_rows) * group_stride + (row % group_rows) * cols - row * cols;
  const int nv = cols >> 8;
  float v[MAXV][8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (i < nv) {
      uint4 u = *reinterpret_cast<const uint4*>(x + row * cols + (i * 32 + lane) * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float2 f = __bfloat1622float2(h[t]);
        v[i][2 * t] = f.x; v[i][2 * t + 1] = f.y;
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
  amax = fmaxf(warp_max(amax), 1e-12f);
  const float inv = 448.f / amax;
  if (lane == 0) scale[row] = amax / 448.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (i < nv) {
      uint2 w;
      w.x = pack_e4m3x2(v[i][0] * inv, v[i][1] * inv) | ((uint32_t)pack_e4m3x2(v[i][2] * inv, v[i][3] * inv) << 16);
      w.y = pack_e4m3x2(v[i][4] * inv, v[i][5] * inv) | ((uint32_t)pack_e4m3x2(v[i][6] * inv, v[i][7] * inv) << 16);
      *reinterpret_cast<uint2*>(q + row * cols + (i * 32 + lane) * 8) = w;
    }
  }
}

// 64x64 bf16 tile transpose through padded shared memory; coalesced on both sides.
__global__ void __launch_bounds__(256)
transpose_bf16_kernel(const __nv_bfloat16* __restrict__ src, __nv_bfloat16* __restrict__ dst, long long rows, long long cols,
                      int accumulate) {
  __shared__ __nv_bfloat16 tile[64][66];
  const long long r0 = (long long)blockIdx.y * 64, c0 = (long long)blockIdx.x * 64;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  for (int i = ty; i < 64; i += 4) {
    const long long r = r0 + i, c = c0 + tx;
    tile[i][tx] = (r < rows && c < cols) ? src[r * cols + c] : __float2bfloat16(0.f);
  }
  __syncthreads();
  for (int i = ty; i < 64; i += 4) {
    const long long c = c0 + i, r = r0 + tx;
    if (c < cols && r < rows) {
      __nv_bfloat16 v = tile[tx][i];
      if (accumulate) v = __float2bfloat16(__bfloat162float(v) + __bfloat162float(dst[c * rows + r]));
      dst[c * rows + r] = v;
    }
  }
}

// Column amax of a [rows, cols] bf16 matrix (atomic max on float bits), then quantise the transpose.
__global__ void __launch_bounds__(256)
col_amax_kernel(const __nv_bfloat16* __restrict__ src, unsigned int* __restrict__ amax_bits, long long rows, long long cols,
                long long src_bstride = 0) {
  src += blockIdx.z * src_bstride;                     // gridDim.z matrices, one amax row of `cols` words each
  amax_bits += blockIdx.z * cols;
  // Block = 256 columns x 64 rows; a warp reads one row segment of 256 columns with 16-byte loads, the eight
  // warps' maxima are combined in shared memory, one atomic per column and block.  Ragged column edges (cols
  // not a multiple of 8) take the scalar path.
  __shared__ float part[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long c0 = (long long)blockIdx.x * 256 + lane * 8;
  const long long r_begin = (long long)blockIdx.y * 64;
  float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const bool vec = (cols % 8 == 0) && c0 + 8 <= cols;
  for (long long r = r_begin + warp; r < rows && r < r_begin + 64; r += 8) {
    if (vec) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + r * cols + c0);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __bfloat1622float2(h[t]);
        m[2 * t] = fmaxf(m[2 * t], fabsf(f.x));
        m[2 * t + 1] = fmaxf(m[2 * t + 1], fabsf(f.y));
      }
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t)
        if (c0 + t < cols) m[t] = fmaxf(m[t], fabsf(__bfloat162float(src[r * cols + c0 + t])));
    }
  }
#pragma unroll
  for (int t = 0; t < 8; ++t) part[warp][lane * 8 + t] = m[t];
  __syncthreads();
  float best = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) best = fmaxf(best, part[w][threadIdx.x]);
  const long long c = (long long)blockIdx.x * 256 + threadIdx.x;
  if (c < cols && best > 0.f) atomicMax(amax_bits + c, __float_as_uint(best));
}

__global__ void __launch_bounds__(256)
quant_transpose_kernel(const __nv_bfloat16* __restrict__ src, uint8_t* __restrict__ q, const unsigned int* __restrict__ amax_bits,
                       float* __restrict__ scale, long long rows, long long cols, long long src_bstride = 0) {
  src += blockIdx.z * src_bstride;
  q += blockIdx.z * rows * cols;
  amax_bits += blockIdx.z * cols;
  scale += blockIdx.z * cols;
  __shared__ float tile[64][65];
  const long long r0 = (long long)blockIdx.y * 64, c0 = (long long)blockIdx.x * 64;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  for (int i = ty; i < 64; i += 4) {
    const long long r = r0 + i, c = c0 + tx;
    tile[i][tx] = (r < rows && c < cols) ? __bfloat162float(src[r * cols + c]) : 0.f;
  }
  __syncthreads();
  for (int i = ty; i < 64; i += 4) {
    const long long c = c0 + i, r = r0 + tx;
    if (c < cols && r < rows) {
      const float amax = fmaxf(__uint_as_float(amax_bits[c]), 1e-12f);
      if (blockIdx.y == 0 && tx == 0) scale[c] = amax / 448.f;
      q[c * rows + r] = (uint8_t)(pack_e4m3x2(tile[tx][i] * (448.f / amax), 0.f) & 0xff);
    }
  }
}

}  // namespace mng

using namespace mng;

#define DISPATCH_COLS(KERNEL, ...)                                                            \
  do {                                                                                        \
    if (cols % 256 != 0 || cols > 4096) return -1;                                            \
    const unsigned grid = (unsigned)((rows + ROW_WARPS - 1) / ROW_WARPS);                     \
    if (cols <= 256) KERNEL<1><<<grid, ROW_WARPS * 32, 0, (cudaStream_t)stream>>>(__VA_ARGS__);        \
    else if (cols <= 768) KERNEL<3><<<grid, ROW_WARPS * 32, 0, (cudaStream_t)stream>>>(__VA_ARGS__);   \
    else if (cols <= 1024) KERNEL<4><<<grid, ROW_WARPS * 32, 0, (cudaStream_t)stream>>>(__VA_ARGS__);  \
    else if (cols <= 3072) KERNEL<12><<<grid, ROW_WARPS * 32, 0, (cudaStream_t)stream>>>(__VA_ARGS__); \
    else KERNEL<16><<<grid, ROW_WARPS * 32, 0, (cudaStream_t)stream>>>(__VA_ARGS__);                   \
    return cudaGetLastError() == cudaSuccess ? 0 : -2;                                        \
  } while (0)

static const float kRmsEps = 1.1920929e-07f;   // F.rms_norm(eps=None) uses the eps of the fp32 computation dtype, also for bf16 input

extern "C" int mng_rmsnorm_fwd(const void* x, void* y, void* y8, float* row_scale, float* rstd, long long rows, int cols,
                               void* stream) {
  if (rows == 0) return 0;
  DISPATCH_COLS(rmsnorm_fwd_kernel, (const __nv_bfloat16*)x, (__nv_bfloat16*)y, (uint8_t*)y8, row_scale, rstd, rows, cols, kRmsEps);
}

extern "C" int mng_rmsnorm_bwd(const void* x, const void* dy, const float* rstd, void* dx, long long rows, int cols,
                               int accumulate, void* stream) {
  if (rows == 0) return 0;
  DISPATCH_COLS(rmsnorm_bwd_kernel, (const __nv_bfloat16*)x, (const __nv_bfloat16*)dy, rstd,
                accumulate ? (const __nv_bfloat16*)dx : nullptr, (__nv_bfloat16*)dx, rows, cols, kRmsEps);
}

// dx = norm backward + addend: the sum autograd would otherwise form with a separate pass when the normalised tensor
// also feeds a residual path.
extern "C" int mng_rmsnorm_bwd_add(const void* x, const void* dy, const float* rstd, const void* addend, void* dx,
                                   long long rows, int cols, void* stream) {
  if (rows == 0) return 0;
  DISPATCH_COLS(rmsnorm_bwd_kernel, (const __nv_bfloat16*)x, (const __nv_bfloat16*)dy, rstd, (const __nv_bfloat16*)addend,
                (__nv_bfloat16*)dx, rows, cols, kRmsEps);
}

// The same with the addend scaled by a device scalar, and sum(addend * x) added to *dot_out (see the kernel).
extern "C" int mng_rmsnorm_bwd_add_scaled(const void* x, const void* dy, const float* rstd, const void* addend,
                                          const float* addend_scale, float* dot_out, void* dx, long long rows, int cols,
                                          void* stream) {
  if (rows == 0) return 0;
  DISPATCH_COLS(rmsnorm_bwd_kernel, (const __nv_bfloat16*)x, (const __nv_bfloat16*)dy, rstd, (const __nv_bfloat16*)addend,
                (__nv_bfloat16*)dx, rows, cols, kRmsEps, addend_scale, dot_out);
}

extern "C" int mng_quant_rows_e4m3(const void* x, void* q, float* scale, long long rows, int cols, void* stream) {
  if (rows == 0) return 0;
  DISPATCH_COLS(quant_rows_kernel, (const __nv_bfloat16*)x, (uint8_t*)q, scale, rows, cols, rows, 0LL);
}

// dst[c, r] = src[r, c] for 1-byte elements; rows and cols multiples of 64.  64 x 64 tiles through shared memory,
// 16-byte global accesses on both sides.
__global__ void __launch_bounds__(256)
transpose_u8_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, long long rows, long long cols) {
  __shared__ uint8_t tile[64][64 + 16];
  const long long r0 = (long long)blockIdx.y * 64, c0 = (long long)blockIdx.x * 64;
  const int a = threadIdx.x >> 2, seg = threadIdx.x & 3;
  *reinterpret_cast<uint4*>(&tile[a][seg * 16]) = *reinterpret_cast<const uint4*>(src + (r0 + a) * cols + c0 + seg * 16);
  __syncthreads();
  uint8_t v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = tile[seg * 16 + j][a];
  *reinterpret_cast<uint4*>(dst + (c0 + a) * rows + r0 + seg * 16) = *reinterpret_cast<const uint4*>(v);
}

extern "C" int mng_transpose_u8(const void* src, void* dst, long long rows, long long cols, void* stream) {
  if (rows % 64 || cols % 64) return -1;
  dim3 grid((unsigned)(cols / 64), (unsigned)(rows / 64));
  transpose_u8_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)src, (uint8_t*)dst, rows, cols);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_transpose_bf16(const void* src, void* dst, long long rows, long long cols, int accumulate, void* stream) {
  dim3 grid((unsigned)((cols + 63) / 64), (unsigned)((rows + 63) / 64));
  transpose_bf16_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)src, (__nv_bfloat16*)dst, rows, cols, accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// `amax_scratch` holds `cols` 32-bit words of caller-provided scratch (zeroed here).
extern "C" int mng_quant_transpose_e4m3(const void* src, void* q, float* scale, unsigned int* amax_scratch, long long rows,
                                        long long cols, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (cudaMemsetAsync(amax_scratch, 0, sizeof(unsigned int) * cols, s) != cudaSuccess) return -3;
  dim3 g1((unsigned)((cols + 255) / 256), (unsigned)((rows + 63) / 64));
  col_amax_kernel<<<g1, 256, 0, s>>>((const __nv_bfloat16*)src, amax_scratch, rows, cols);
  dim3 g2((unsigned)((cols + 63) / 64), (unsigned)((rows + 63) / 64));
  quant_transpose_kernel<<<g2, 256, 0, s>>>((const __nv_bfloat16*)src, (uint8_t*)q, amax_scratch, scale, rows, cols);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Refresh of the FP8 copies of a [layers, 2, hid, dim] MLP parameter bank in five launches for all layers:
// row-scaled e4m3 of the up projections, column-amax + transposing quantiser of the down projections, and the
// per-layer scale bookkeeping (delayed activation scales from the amax seen since the last refresh,
// `train_gpt.py:1670-1675`; per-layer maxima of the down-projection scales for the state_dict buffers).
namespace mng {
__global__ void mlp_scales_kernel(const float* __restrict__ projT_scale, float* __restrict__ act_scale, unsigned int* __restrict__ amax_bits,
                                  float* __restrict__ used, float* __restrict__ next, int dim, int bootstrap) {
  const int l = blockIdx.x;
  float m = 0.f;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) m = fmaxf(m, projT_scale[(long long)l * dim + c]);
  __shared__ float red[8];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    used[l] = bootstrap ? m : next[l];
    next[l] = m * 1.12f;
    const float seen = __uint_as_float(amax_bits[l]);
    if (seen > 0.f) act_scale[l] = fmaxf(seen, 1e-12f) * (1.80f / 448.0f);
    amax_bits[l] = 0u;
  }
}
}  // namespace mng

extern "C" int mng_mlp_weight_refresh(const void* bank, int layers, int hid, int dim, void* fc8, float* fc_scale, void* projT8,
                                      float* projT_scale, unsigned int* amax_scratch, float* act_scale, unsigned int* amax_bits,
                                      float* used_scales, float* next_scales, int bootstrap, void* stream) {
  if (layers <= 0 || hid <= 0 || dim <= 0 || layers > 65535) return -1;
  cudaStream_t s = (cudaStream_t)stream;
  const __nv_bfloat16* w = (const __nv_bfloat16*)bank;
  const long long lstride = 2LL * hid * dim;
  {
    const long long rows = (long long)layers * hid;
    const int cols = dim;
    if (cols % 256 != 0 || cols > 4096) return -1;
    const unsigned grid = (unsigned)((rows + ROW_WARPS - 1) / ROW_WARPS);
    const __nv_bfloat16* x = w;
    uint8_t* q = (uint8_t*)fc8;
    if (cols <= 256) quant_rows_kernel<1><<<grid, ROW_WARPS * 32, 0, s>>>(x, q, fc_scale, rows, cols, (long long)hid, lstride);
    else if (cols <= 768) quant_rows_kernel<3><<<grid, ROW_WARPS * 32, 0, s>>>(x, q, fc_scale, rows, cols, (long long)hid, lstride);
    else if (cols <= 1024) quant_rows_kernel<4><<<grid, ROW_WARPS * 32, 0, s>>>(x, q, fc_scale, rows, cols, (long long)hid, lstride);
    else if (cols <= 3072) quant_rows_kernel<12><<<grid, ROW_WARPS * 32, 0, s>>>(x, q, fc_scale, rows, cols, (long long)hid, lstride);
    else quant_rows_kernel<16><<<grid, ROW_WARPS * 32, 0, s>>>(x, q, fc_scale, rows, cols, (long long)hid, lstride);
  }
  if (cudaMemsetAsync(amax_scratch, 0, sizeof(unsigned int) * (size_t)layers * dim, s) != cudaSuccess) return -3;
  const __nv_bfloat16* proj = w + (long long)hid * dim;                 // [l, 1] = down projection [hid, dim]
  dim3 g1((unsigned)((dim + 255) / 256), (unsigned)((hid + 63) / 64), (unsigned)layers);
  col_amax_kernel<<<g1, 256, 0, s>>>(proj, amax_scratch, hid, dim, lstride);
  dim3 g2((unsigned)((dim + 63) / 64), (unsigned)((hid + 63) / 64), (unsigned)layers);
  quant_transpose_kernel<<<g2, 256, 0, s>>>(proj, (uint8_t*)projT8, amax_scratch, projT_scale, hid, dim, lstride);
  mlp_scales_kernel<<<layers, 256, 0, s>>>(projT_scale, act_scale, amax_bits, used_scales, next_scales, dim, bootstrap);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// ---------------------------------------------------------------------------------------------------
// Allocation-free variant of mng_quant_transpose_e4m3 (see noalloc.h): the column-amax scratch lives
// in this file-scope device array instead of caller memory.
#include "noalloc.h"

#include <mutex>

static __device__ __align__(256) unsigned int g_static_amax_scratch[MNG_STATIC_SCRATCH_COLS];

namespace {
constexpr int kMaxDevices = 64;
void* g_static_scratch_addr[kMaxDevices] = {};   // device address of the array, per device ordinal
std::mutex g_static_scratch_mu;

// `g_static_amax_scratch` named in host code is only a host-side handle; the address a kernel can use
// has to be asked for, once per device, while that device is current.
int static_scratch_ptr(unsigned int** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MNG_ERR_SYMBOL;
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (g_static_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_amax_scratch) != cudaSuccess || p == nullptr) return MNG_ERR_SYMBOL;
    g_static_scratch_addr[dev] = p;
  }
  *out = static_cast<unsigned int*>(g_static_scratch_addr[dev]);
  return MNG_OK;
}
}  // namespace

extern "C" int mng_quant_transpose_e4m3_static(const void* src, void* q, float* scale, long long rows, long long cols,
                                               void* stream) {
  if (rows <= 0 || cols <= 0) return MNG_ERR_BAD_SHAPE;
  if (cols > MNG_STATIC_SCRATCH_COLS || rows > MNG_STATIC_MAX_ROWS) return MNG_ERR_TOO_LARGE;
  unsigned int* scratch = nullptr;
  const int rc = static_scratch_ptr(&scratch);
  if (rc != MNG_OK) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  // the array still holds the previous call's maxima: clear the words this call will use
  if (cudaMemsetAsync(scratch, 0, sizeof(unsigned int) * cols, s) != cudaSuccess) return MNG_ERR_LAUNCH;
  dim3 g1((unsigned)((cols + 255) / 256), (unsigned)((rows + 63) / 64));
  mng::col_amax_kernel<<<g1, 256, 0, s>>>((const __nv_bfloat16*)src, scratch, rows, cols);
  dim3 g2((unsigned)((cols + 63) / 64), (unsigned)((rows + 63) / 64));
  mng::quant_transpose_kernel<<<g2, 256, 0, s>>>((const __nv_bfloat16*)src, (uint8_t*)q, scratch, scale, rows, cols);
  return cudaGetLastError() == cudaSuccess ? MNG_OK : MNG_ERR_LAUNCH;
}

extern "C" const char* mng_static_strerror(int code) {
  switch (code) {
    case MNG_OK: return "ok";
    case MNG_ERR_TOO_LARGE:
      return "cols exceeds MNG_STATIC_SCRATCH_COLS (65536, the size of the built-in scratch array) or rows exceeds "
             "MNG_STATIC_MAX_ROWS (4194240, the launch grid's limit)";
    case MNG_ERR_SYMBOL: return "could not resolve the device address of the built-in scratch array on the current device";
    case MNG_ERR_BAD_SHAPE: return "rows and cols must be positive";
    case MNG_ERR_LAUNCH: return "memset or kernel launch failed";
    default: return "unknown code";
  }
}
