// Cross-head mixing step of the dynamically-composable-MHA correction.  The score and value
// products run as windowed, batched tcgen05 GEMMs (one 128-query block against the 256 keys
// [128*blk - 128, 128*blk + 128)); these two kernels do what sits between them, one warp per query:
//   fwd: masked softmax per head over the last `window` same-document keys, a = sum_h w1_h P_h
//   bwd: from dM_h = dOut_h V^T:  g_w2, da, g_w1 and dS_h = scale * P_h w1_h (da - g_w1_h)
// Math of `dc_triton_kernels.py:252-440` (forward) and `:489-896` (backward).
#include "api.h"
#include "ptx.cuh"

namespace mng {

constexpr int DC_WARPS = 8;
constexpr int DC_R = 256;        // keys per block window
constexpr int DC_MAXH = 8;

// S: [H, nblk, 128, 256] fp32 scores (already scaled).  P: same shape bf16.  a: [nblk, 128, 256] bf16.
__global__ void __launch_bounds__(DC_WARPS * 32)
dc_mix_fwd_kernel(const float* __restrict__ S, const __nv_bfloat16* __restrict__ w1, const int* __restrict__ doc_start,
                  __nv_bfloat16* __restrict__ P, __nv_bfloat16* __restrict__ a, long long T, int H, int window) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * DC_WARPS + (threadIdx.x >> 5);
  if (t >= T) return;
  const long long blk = t >> 7;
  const long long k0 = blk * 128 - 128;              // key position of column 0
  int ds = doc_start[t];
  if (!MNG_IN_RANGE(ds, t + 1)) ds = (int)t;                  // debug build only: a document cannot start after its token
  const long long head_stride = T * DC_R;            // nblk*128*256
  bool valid[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const long long kp = k0 + lane * 8 + i;
    valid[i] = kp <= t && t - kp < window && kp >= ds;
  }
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int h = 0; h < H; ++h) {
    const float* s = S + h * head_stride + t * DC_R + lane * 8;
    float4 s0 = *reinterpret_cast<const float4*>(s), s1 = *reinterpret_cast<const float4*>(s + 4);
    float v[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float mx = -3.0e38f;
#pragma unroll
    for (int i = 0; i < 8; ++i) if (valid[i]) mx = fmaxf(mx, v[i]);
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) { v[i] = valid[i] ? __expf(v[i] - mx) : 0.f; sum += v[i]; }
    sum = warp_sum(sum);
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    const float w = __bfloat162float(w1[t * H + h]);
    float p[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) { p[i] = v[i] * inv; acc[i] += w * p[i]; }
    uint4 o;
    o.x = pack_bf16x2(p[0], p[1]); o.y = pack_bf16x2(p[2], p[3]); o.z = pack_bf16x2(p[4], p[5]); o.w = pack_bf16x2(p[6], p[7]);
    *reinterpret_cast<uint4*>(P + h * head_stride + t * DC_R + lane * 8) = o;
  }
  uint4 o;
  o.x = pack_bf16x2(acc[0], acc[1]); o.y = pack_bf16x2(acc[2], acc[3]); o.z = pack_bf16x2(acc[4], acc[5]); o.w = pack_bf16x2(acc[6], acc[7]);
  *reinterpret_cast<uint4*>(a + t * DC_R + lane * 8) = o;
}

// dM: [H, nblk, 128, 256] fp32.  Outputs: dS [H, nblk, 128, 256] bf16, g_w1, g_w2 [T, H] fp32.
__global__ void __launch_bounds__(DC_WARPS * 32)
dc_mix_bwd_kernel(const float* __restrict__ dM, const __nv_bfloat16* __restrict__ P, const __nv_bfloat16* __restrict__ a,
                  const __nv_bfloat16* __restrict__ w1, const __nv_bfloat16* __restrict__ w2, __nv_bfloat16* __restrict__ dS,
                  float* __restrict__ g_w1, float* __restrict__ g_w2, long long T, int H, float scale) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * DC_WARPS + (threadIdx.x >> 5);
  if (t >= T) return;
  const long long head_stride = T * DC_R;
  float av[8];
  {
    uint4 u = *reinterpret_cast<const uint4*>(a + t * DC_R + lane * 8);
    const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) { float2 f = __bfloat1622float2(hh[i]); av[2 * i] = f.x; av[2 * i + 1] = f.y; }
  }
  float da[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int h = 0; h < H; ++h) {
    const float* m = dM + h * head_stride + t * DC_R + lane * 8;
    float4 m0 = *reinterpret_cast<const float4*>(m), m1 = *reinterpret_cast<const float4*>(m + 4);
    const float mv[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
    const float wv2 = __bfloat162float(w2[t * H + h]);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) { dot += av[i] * mv[i]; da[i] += wv2 * mv[i]; }
    dot = warp_sum(dot);
    if (lane == 0) g_w2[t * H + h] = dot;
  }
  for (int h = 0; h < H; ++h) {
    uint4 u = *reinterpret_cast<const uint4*>(P + h * head_stride + t * DC_R + lane * 8);
    const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
    float p[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) { float2 f = __bfloat1622float2(hh[i]); p[2 * i] = f.x; p[2 * i + 1] = f.y; }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) dot += p[i] * da[i];
    dot = warp_sum(dot);
    if (lane == 0) g_w1[t * H + h] = dot;
    const float c = scale * __bfloat162float(w1[t * H + h]);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = c * p[i] * (da[i] - dot);
    uint4 w;
    w.x = pack_bf16x2(o[0], o[1]); w.y = pack_bf16x2(o[2], o[3]); w.z = pack_bf16x2(o[4], o[5]); w.w = pack_bf16x2(o[6], o[7]);
    *reinterpret_cast<uint4*>(dS + h * head_stride + t * DC_R + lane * 8) = w;
  }
}

}  // namespace mng

using namespace mng;

MNG_DEFINE_BOUNDS_QUERY(dc)

extern "C" int mng_dc_mix_fwd(const float* S, const void* w1, const int* doc_start, void* P, void* a, long long T, int H,
                              int window, void* stream) {
  if (T % 128 || H > DC_MAXH || window > 128) return -1;
  const unsigned grid = (unsigned)((T + DC_WARPS - 1) / DC_WARPS);
  dc_mix_fwd_kernel<<<grid, DC_WARPS * 32, 0, (cudaStream_t)stream>>>(S, (const __nv_bfloat16*)w1, doc_start, (__nv_bfloat16*)P,
                                                                      (__nv_bfloat16*)a, T, H, window);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Fold of the windowed key/value gradients.  part [H, nblk, 256, 128] bf16: row j of block b's window is position
// 128*b - 128 + j, so position t = 128*b + r gets part[h, b, 128 + r] + part[h, b + 1, r].  out [T, H, 128] bf16.
// One thread per 8 elements.
__global__ void __launch_bounds__(256)
dc_fold_kernel(const __nv_bfloat16* __restrict__ part, __nv_bfloat16* __restrict__ out, long long T, int H) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;      // over T * H * 16
  if (i >= T * H * 16) return;
  const int seg = (int)(i & 15);
  const long long th = i >> 4;
  const long long t = th / H;
  const int h = (int)(th - t * H);
  const long long nblk = T >> 7, b = t >> 7;
  const int r = (int)(t & 127);
  const __nv_bfloat16* hi = part + (((long long)h * nblk + b) * 256 + 128 + r) * 128 + seg * 8;
  uint4 u = *reinterpret_cast<const uint4*>(hi);
  if (b + 1 < nblk) {
    const uint4 v = *reinterpret_cast<const uint4*>(part + (((long long)h * nblk + b + 1) * 256 + r) * 128 + seg * 8);
    __nv_bfloat162* a2 = reinterpret_cast<__nv_bfloat162*>(&u);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) a2[k] = __hadd2(a2[k], b2[k]);
  }
  *reinterpret_cast<uint4*>(out + th * 128 + seg * 8) = u;
}

extern "C" int mng_dc_fold(const void* part, void* out, long long T, int H, void* stream) {
  if (T % 128) return -1;
  const long long n = T * H * 16;
  dc_fold_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)part, (__nv_bfloat16*)out, T, H);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_dc_mix_bwd(const float* dM, const void* P, const void* a, const void* w1, const void* w2, void* dS,
                              float* g_w1, float* g_w2, long long T, int H, float scale, void* stream) {
  if (T % 128 || H > DC_MAXH) return -1;
  const unsigned grid = (unsigned)((T + DC_WARPS - 1) / DC_WARPS);
  dc_mix_bwd_kernel<<<grid, DC_WARPS * 32, 0, (cudaStream_t)stream>>>(dM, (const __nv_bfloat16*)P, (const __nv_bfloat16*)a,
                                                                      (const __nv_bfloat16*)w1, (const __nv_bfloat16*)w2,
                                                                      (__nv_bfloat16*)dS, g_w1, g_w2, T, H, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
