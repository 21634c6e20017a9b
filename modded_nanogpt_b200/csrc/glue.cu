// Fused "glue" between the GEMMs: the residual / skip / MUDD mixes, the post-processing of the
// QKV projection (QK RMSNorm, rotary, key offset, value-embedding add) and the attention output
// gating (XSA + per-head gate), each as one forward and one backward kernel.  All of them stream
// [T, D] bf16 tensors once, one warp per row (or per head row), 16-byte accesses.
#include "api.h"
#include "ptx.cuh"

namespace mng {

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    float2 v = __bfloat1622float2(h[t]);
    f[2 * t] = v.x; f[2 * t + 1] = v.y;
  }
}
__device__ __forceinline__ void cvt8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    float2 v = __bfloat1622float2(h[t]);
    f[2 * t] = v.x; f[2 * t + 1] = v.y;
  }
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 w;
  w.x = pack_bf16x2(f[0], f[1]); w.y = pack_bf16x2(f[2], f[3]); w.z = pack_bf16x2(f[4], f[5]); w.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = w;
}
__device__ __forceinline__ float gate_at(const void* g, int is_bf16, long long idx) {
  return is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g)[idx]) : reinterpret_cast<const float*>(g)[idx];
}

// =====================================================================================================
// out[t,:] = sum_j c_j(t) * x_j[t,:],   c_j(t) = addc_j + s_j * g_j(t)
//   s_j : fp32 device scalar (or 1),  g_j(t) : element [t*stride + col] of a gate tensor (or 1).
constexpr int LC_WARPS = 8;

template <int MAXV>
__global__ void __launch_bounds__(LC_WARPS * 32)
lincomb_fwd_kernel(LinCombArgs a, __nv_bfloat16* __restrict__ out, long long rows, int cols) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * LC_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nv = cols >> 8;
  float acc[MAXV][8];
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[i][t] = 0.f;
  for (int j = 0; j < a.k; ++j) {
    const LinTerm& tm = a.t[j];
    float c = tm.scalar ? *tm.scalar : 1.f;
    if (tm.gate && MNG_IN_RANGE(tm.gate_col, tm.gate_stride)) c *= gate_at(tm.gate, tm.gate_bf16, row * tm.gate_stride + tm.gate_col);
    c += tm.addc;
    const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(tm.x) + row * cols;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (i < nv) {
        float f[8];
        ld8(x + (i * 32 + lane) * 8, f);
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[i][t] += c * f[t];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
    if (i < nv) st8(out + row * cols + (i * 32 + lane) * 8, acc[i]);
}

// Backward: dx_j = c_j(t) * g (optional), dgate_j[t] = s_j * <g, x_j>(t) (optional, bf16 column of a
// zero-initialised buffer), dscalar_j += sum_t g_j(t) * <g, x_j>(t) (optional, fp32 atomics per CTA).
template <int MAXV>
__global__ void __launch_bounds__(LC_WARPS * 32)
lincomb_bwd_kernel(LinCombArgs a, LinCombGrads gr, const __nv_bfloat16* __restrict__ g, long long rows, int cols) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long row = (long long)blockIdx.x * LC_WARPS + warp;
  const bool live = row < rows;
  const int nv = cols >> 8;
  __shared__ float s_part[LC_MAX_TERMS][LC_WARPS];
  float gv[MAXV][8];
  if (live) {
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
      if (i < nv) ld8(g + row * cols + (i * 32 + lane) * 8, gv[i]);
  }
  // Terms are handled two at a time with all of their loads (x for the dot products, dx where it is accumulated
  // into) issued before the first use: the stores of one term would otherwise fence off the loads of the next.
  for (int j0 = 0; j0 < a.k; j0 += 2) {
    uint4 rx[2][MAXV], rd[2][MAXV];
    // two terms of one tensor share a gradient buffer (the first writes, the second adds): then the second one's
    // read has to follow the first one's store
    const bool late1 = j0 + 1 < a.k && gr.t[j0 + 1].dx != nullptr && gr.t[j0 + 1].dx == gr.t[j0].dx;
    if (live) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = j0 + u;
        if (j < a.k) {
          const LinGrad& og = gr.t[j];
          const bool need_dot = og.dgate || og.dscalar;
          const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(a.t[j].x) + row * cols;
          const __nv_bfloat16* dx = og.dx ? reinterpret_cast<const __nv_bfloat16*>(og.dx) + row * cols : nullptr;
#pragma unroll
          for (int i = 0; i < MAXV; ++i) {
            if (i < nv) {
              if (need_dot) rx[u][i] = *reinterpret_cast<const uint4*>(x + (i * 32 + lane) * 8);
              if (dx && og.dx_accumulate && !(u == 1 && late1)) rd[u][i] = *reinterpret_cast<const uint4*>(dx + (i * 32 + lane) * 8);
            }
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int j = j0 + u;
      if (j >= a.k) break;
      const LinTerm& tm = a.t[j];
      const LinGrad& og = gr.t[j];
      float spart = 0.f;
      if (live) {
        const float s = tm.scalar ? *tm.scalar : 1.f;
        const float gt = tm.gate ? gate_at(tm.gate, tm.gate_bf16, row * tm.gate_stride + tm.gate_col) : 1.f;
        const float c = tm.addc + s * gt;
        float dot = 0.f;
        const bool need_dot = og.dgate || og.dscalar;
        __nv_bfloat16* dx = og.dx ? reinterpret_cast<__nv_bfloat16*>(og.dx) + row * cols : nullptr;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
          if (i < nv) {
            if (need_dot) {
              float f[8];
              cvt8(rx[u][i], f);
#pragma unroll
              for (int t = 0; t < 8; ++t) dot += gv[i][t] * f[t];
            }
            if (dx) {
              float o[8];
              if (og.dx_accumulate) {
                if (u == 1 && late1) rd[u][i] = *reinterpret_cast<const uint4*>(dx + (i * 32 + lane) * 8);
                cvt8(rd[u][i], o);
#pragma unroll
                for (int t = 0; t < 8; ++t) o[t] = fmaf(c, gv[i][t], o[t]);
              } else {
#pragma unroll
                for (int t = 0; t < 8; ++t) o[t] = c * gv[i][t];
              }
              st8(dx + (i * 32 + lane) * 8, o);
            }
          }
        }
        if (need_dot) {
          dot = warp_sum(dot);
          if (og.dgate && lane == 0)
            reinterpret_cast<__nv_bfloat16*>(og.dgate)[row * og.dgate_stride + og.dgate_col] = __float2bfloat16(s * dot);
          spart = gt * dot;
        }
      }
      if (og.dscalar && lane == 0) s_part[j][warp] = spart;
    }
  }
  __syncthreads();
  if (threadIdx.x < a.k && gr.t[threadIdx.x].dscalar) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < LC_WARPS; ++w) tot += s_part[threadIdx.x][w];
    atomicAdd(gr.t[threadIdx.x].dscalar, tot);
  }
}

// =====================================================================================================
// QKV post-processing.  One warp per (token, head) row of 128 elements; lane l owns dims 4l..4l+3.
//   q,k: RMSNorm over the head (eps = fp32 epsilon), rotary, optional key offset;
//        layout 0 (track 1): dims 0..63 rotate as interleaved pairs (2i, 2i+1), dims 64..127 are stationary;
//                            key offset: k[t, 64:] <- k_normed[t-1, 64:] for t >= 1;
//        layout 1 (track 2, split halves): dim d < 32 rotates with dim d + 64, dims 32..63 and 96..127 are
//                            stationary and are the ones the key offset takes from the previous token;
//   v  : v + vgate[t,h] * ve[t,h,:] + vadd[t,h,:]   (both optional).
// cos/sin: fp32 [positions, 32].  position = t, or 2t + (h & 1) for paired-head layers.
constexpr int QP_WARPS = 8;
constexpr float HEAD_EPS = 1.1920929e-07f;   // eps of the fp32 computation dtype, as F.rms_norm(eps=None)

template <bool split>                         // rotary layout, compile-time so that each layout carries only its own shuffles
__global__ void __launch_bounds__(QP_WARPS * 32)
qkv_post_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                    const __nv_bfloat16* __restrict__ ve, const __nv_bfloat16* __restrict__ vgate, int vgate_stride,
                    const __nv_bfloat16* __restrict__ vadd, __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                    __nv_bfloat16* __restrict__ v, float* __restrict__ rstd_q, float* __restrict__ rstd_k, long long T, int H,
                    int paired, int key_offset) {
  const int lane = threadIdx.x & 31;
  const long long idx = (long long)blockIdx.x * QP_WARPS + (threadIdx.x >> 5);     // (t, h)
  if (idx >= T * H) return;
  const long long t = idx / H;
  const int h = (int)(idx % H);
  const long long ld = 3LL * H * 128;
  const long long pos = paired ? 2 * t + (h & 1) : t;
  float cs[2] = {1.f, 1.f}, sn[2] = {0.f, 0.f};
  float c4[4] = {1.f, 1.f, 1.f, 1.f}, s4[4] = {0.f, 0.f, 0.f, 0.f};
  const bool rot = split ? ((lane & 15) < 8) : (lane < 16);      // lanes whose dims rotate
  if (!split && lane < 16) {
    cs[0] = cos_t[pos * 32 + 2 * lane]; cs[1] = cos_t[pos * 32 + 2 * lane + 1];
    sn[0] = sin_t[pos * 32 + 2 * lane]; sn[1] = sin_t[pos * 32 + 2 * lane + 1];
  }
  if (split && rot) {
    const float4 c = *reinterpret_cast<const float4*>(cos_t + pos * 32 + 4 * (lane & 7));
    const float4 s = *reinterpret_cast<const float4*>(sin_t + pos * 32 + 4 * (lane & 7));
    c4[0] = c.x; c4[1] = c.y; c4[2] = c.z; c4[3] = c.w;
    s4[0] = s.x; s4[1] = s.y; s4[2] = s.z; s4[3] = s.w;
  }
#pragma unroll
  for (int which = 0; which < 2; ++which) {        // 0 = q, 1 = k
    const __nv_bfloat16* src = qkv + t * ld + (which * H + h) * 128 + lane * 4;
    uint2 u = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 a = __bfloat1622float2(hh[0]), b = __bfloat1622float2(hh[1]);
    float ss = warp_sum(a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y);
    const float r = rsqrtf(ss * (1.f / 128.f) + HEAD_EPS);
    if (lane == 0) (which ? rstd_k : rstd_q)[idx] = r;
    // normalised values rounded to bf16, as the separate norm op would produce them
    float n0 = __bfloat162float(__float2bfloat16(a.x * r)), n1 = __bfloat162float(__float2bfloat16(a.y * r));
    float n2 = __bfloat162float(__float2bfloat16(b.x * r)), n3 = __bfloat162float(__float2bfloat16(b.y * r));
    float o0, o1, o2, o3;
    // split layout: the partner values live 16 lanes away (dims d and d + 64)
    float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
    if (split) {
      p0 = __shfl_xor_sync(0xffffffffu, n0, 16); p1 = __shfl_xor_sync(0xffffffffu, n1, 16);
      p2 = __shfl_xor_sync(0xffffffffu, n2, 16); p3 = __shfl_xor_sync(0xffffffffu, n3, 16);
    }
    if (split && rot) {   // x1' = c x1 + s x2 (lanes 0-7), x2' = c x2 - s x1 (lanes 16-23)
      const float sg = lane < 16 ? 1.f : -1.f;
      o0 = c4[0] * n0 + sg * s4[0] * p0; o1 = c4[1] * n1 + sg * s4[1] * p1;
      o2 = c4[2] * n2 + sg * s4[2] * p2; o3 = c4[3] * n3 + sg * s4[3] * p3;
    } else if (!split && lane < 16) {      // pairs (x0,x1): x0' = c x0 + s x1, x1' = c x1 - s x0
      o0 = cs[0] * n0 + sn[0] * n1; o1 = cs[0] * n1 - sn[0] * n0;
      o2 = cs[1] * n2 + sn[1] * n3; o3 = cs[1] * n3 - sn[1] * n2;
    } else {
      o0 = n0; o1 = n1; o2 = n2; o3 = n3;
      if (which == 1 && key_offset && t > 0) {
        // stationary half of k comes from the previous token: recompute its norm from qkv[t-1]
        const __nv_bfloat16* ps = qkv + (t - 1) * ld + (H + h) * 128;
        uint2 pu = *reinterpret_cast<const uint2*>(ps + lane * 4);
        const __nv_bfloat162* ph = reinterpret_cast<const __nv_bfloat162*>(&pu);
        float2 pa = __bfloat1622float2(ph[0]), pb = __bfloat1622float2(ph[1]);
        o0 = pa.x; o1 = pa.y; o2 = pb.x; o3 = pb.y;      // scaled below with the previous row's rstd
      }
    }
    if (which == 1 && key_offset && t > 0) {
      // all lanes take part in the previous row's sum of squares
      const __nv_bfloat16* ps = qkv + (t - 1) * ld + (H + h) * 128;
      uint2 pu = *reinterpret_cast<const uint2*>(ps + lane * 4);
      const __nv_bfloat162* ph = reinterpret_cast<const __nv_bfloat162*>(&pu);
      float2 pa = __bfloat1622float2(ph[0]), pb = __bfloat1622float2(ph[1]);
      const float pss = warp_sum(pa.x * pa.x + pa.y * pa.y + pb.x * pb.x + pb.y * pb.y);
      const float pr = rsqrtf(pss * (1.f / 128.f) + HEAD_EPS);
      if (!rot) { o0 *= pr; o1 *= pr; o2 *= pr; o3 *= pr; }
    }
    uint2 w;
    w.x = pack_bf16x2(o0, o1); w.y = pack_bf16x2(o2, o3);
    *reinterpret_cast<uint2*>((which ? k : q) + idx * 128 + lane * 4) = w;
  }
  {
    const __nv_bfloat16* src = qkv + t * ld + (2 * H + h) * 128 + lane * 4;
    uint2 u = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 a = __bfloat1622float2(hh[0]), b = __bfloat1622float2(hh[1]);
    if (ve) {
      const float gt = vgate ? __bfloat162float(vgate[t * vgate_stride + h]) : 1.f;
      uint2 e = *reinterpret_cast<const uint2*>(ve + idx * 128 + lane * 4);
      const __nv_bfloat162* eh = reinterpret_cast<const __nv_bfloat162*>(&e);
      float2 ea = __bfloat1622float2(eh[0]), eb = __bfloat1622float2(eh[1]);
      a.x += gt * ea.x; a.y += gt * ea.y; b.x += gt * eb.x; b.y += gt * eb.y;
    }
    if (vadd) {
      uint2 e = *reinterpret_cast<const uint2*>(vadd + idx * 128 + lane * 4);
      const __nv_bfloat162* eh = reinterpret_cast<const __nv_bfloat162*>(&e);
      float2 ea = __bfloat1622float2(eh[0]), eb = __bfloat1622float2(eh[1]);
      a.x += ea.x; a.y += ea.y; b.x += eb.x; b.y += eb.y;
    }
    uint2 w;
    w.x = pack_bf16x2(a.x, a.y); w.y = pack_bf16x2(b.x, b.y);
    *reinterpret_cast<uint2*>(v + idx * 128 + lane * 4) = w;
  }
}

// Backward of the above.  dq, dk, dv: [T, H, 128].  Writes d_qkv [T, 3*H*128], and optionally
// d_ve = vgate * dv, d_vgate[t,h] = <dv, ve> (bf16 column buffer), d_vadd = dv is the caller's alias.
template <bool split>
__global__ void __launch_bounds__(QP_WARPS * 32)
qkv_post_bwd_kernel(const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                    const float* __restrict__ rstd_q, const float* __restrict__ rstd_k, const __nv_bfloat16* __restrict__ dq,
                    const __nv_bfloat16* __restrict__ dk, const __nv_bfloat16* __restrict__ dv, const __nv_bfloat16* __restrict__ ve,
                    const __nv_bfloat16* __restrict__ vgate, int vgate_stride, __nv_bfloat16* __restrict__ d_qkv,
                    __nv_bfloat16* __restrict__ d_ve, __nv_bfloat16* __restrict__ d_vgate, int d_vgate_stride, long long T, int H,
                    int paired, int key_offset) {
  const int lane = threadIdx.x & 31;
  const long long idx = (long long)blockIdx.x * QP_WARPS + (threadIdx.x >> 5);
  if (idx >= T * H) return;
  const long long t = idx / H;
  const int h = (int)(idx % H);
  const long long ld = 3LL * H * 128;
  const long long pos = paired ? 2 * t + (h & 1) : t;
  float cs[2] = {1.f, 1.f}, sn[2] = {0.f, 0.f};
  float c4[4] = {1.f, 1.f, 1.f, 1.f}, s4[4] = {0.f, 0.f, 0.f, 0.f};
  const bool rot = split ? ((lane & 15) < 8) : (lane < 16);
  if (!split && lane < 16) {
    cs[0] = cos_t[pos * 32 + 2 * lane]; cs[1] = cos_t[pos * 32 + 2 * lane + 1];
    sn[0] = sin_t[pos * 32 + 2 * lane]; sn[1] = sin_t[pos * 32 + 2 * lane + 1];
  }
  if (split && rot) {
    const float4 c = *reinterpret_cast<const float4*>(cos_t + pos * 32 + 4 * (lane & 7));
    const float4 s = *reinterpret_cast<const float4*>(sin_t + pos * 32 + 4 * (lane & 7));
    c4[0] = c.x; c4[1] = c.y; c4[2] = c.z; c4[3] = c.w;
    s4[0] = s.x; s4[1] = s.y; s4[2] = s.z; s4[3] = s.w;
  }
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const __nv_bfloat16* gsrc = (which ? dk : dq) + idx * 128 + lane * 4;
    uint2 gu = *reinterpret_cast<const uint2*>(gsrc);
    const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gu);
    float2 ga = __bfloat1622float2(gh[0]), gb = __bfloat1622float2(gh[1]);
    float d0, d1, d2, d3;                    // gradient w.r.t. the normalised (pre-rotary) values
    float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
    if (split) {
      q0 = __shfl_xor_sync(0xffffffffu, ga.x, 16); q1 = __shfl_xor_sync(0xffffffffu, ga.y, 16);
      q2 = __shfl_xor_sync(0xffffffffu, gb.x, 16); q3 = __shfl_xor_sync(0xffffffffu, gb.y, 16);
    }
    if (split && rot) {                      // transpose of [c s; -s c] over the (d, d + 64) pairs
      const float sg = lane < 16 ? -1.f : 1.f;
      d0 = c4[0] * ga.x + sg * s4[0] * q0; d1 = c4[1] * ga.y + sg * s4[1] * q1;
      d2 = c4[2] * gb.x + sg * s4[2] * q2; d3 = c4[3] * gb.y + sg * s4[3] * q3;
    } else if (!split && lane < 16) {        // transpose of the rotation
      d0 = cs[0] * ga.x - sn[0] * ga.y; d1 = cs[0] * ga.y + sn[0] * ga.x;
      d2 = cs[1] * gb.x - sn[1] * gb.y; d3 = cs[1] * gb.y + sn[1] * gb.x;
    } else if (which == 1 && key_offset) {
      // normalised k[t, 64:] feeds output row t+1 (and row 0 feeds itself as well)
      d0 = d1 = d2 = d3 = 0.f;
      if (t + 1 < T) {
        uint2 nu = *reinterpret_cast<const uint2*>(dk + (idx + H) * 128 + lane * 4);
        const __nv_bfloat162* nh = reinterpret_cast<const __nv_bfloat162*>(&nu);
        float2 na = __bfloat1622float2(nh[0]), nb = __bfloat1622float2(nh[1]);
        d0 = na.x; d1 = na.y; d2 = nb.x; d3 = nb.y;
      }
      if (t == 0) { d0 += ga.x; d1 += ga.y; d2 += gb.x; d3 += gb.y; }
    } else {
      d0 = ga.x; d1 = ga.y; d2 = gb.x; d3 = gb.y;
    }
    const __nv_bfloat16* src = qkv + t * ld + (which * H + h) * 128 + lane * 4;
    uint2 u = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 a = __bfloat1622float2(hh[0]), b = __bfloat1622float2(hh[1]);
    const float r = (which ? rstd_k : rstd_q)[idx];
    // y = x r,  r = (mean x^2 + eps)^-1/2 :  dx = r (dy - y <dy, y> / 128)
    const float dot = warp_sum(d0 * a.x + d1 * a.y + d2 * b.x + d3 * b.y) * r * r * r * (1.f / 128.f);
    uint2 w;
    w.x = pack_bf16x2(d0 * r - a.x * dot, d1 * r - a.y * dot);
    w.y = pack_bf16x2(d2 * r - b.x * dot, d3 * r - b.y * dot);
    *reinterpret_cast<uint2*>(d_qkv + t * ld + (which * H + h) * 128 + lane * 4) = w;
  }
  {
    uint2 gu = *reinterpret_cast<const uint2*>(dv + idx * 128 + lane * 4);
    *reinterpret_cast<uint2*>(d_qkv + t * ld + (2 * H + h) * 128 + lane * 4) = gu;
    if (ve) {
      const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gu);
      float2 ga = __bfloat1622float2(gh[0]), gb = __bfloat1622float2(gh[1]);
      const float gt = vgate ? __bfloat162float(vgate[t * vgate_stride + h]) : 1.f;
      if (d_ve) {
        uint2 w;
        w.x = pack_bf16x2(gt * ga.x, gt * ga.y); w.y = pack_bf16x2(gt * gb.x, gt * gb.y);
        *reinterpret_cast<uint2*>(d_ve + idx * 128 + lane * 4) = w;
      }
      if (d_vgate) {
        uint2 e = *reinterpret_cast<const uint2*>(ve + idx * 128 + lane * 4);
        const __nv_bfloat162* eh = reinterpret_cast<const __nv_bfloat162*>(&e);
        float2 ea = __bfloat1622float2(eh[0]), eb = __bfloat1622float2(eh[1]);
        const float dot = warp_sum(ga.x * ea.x + ga.y * ea.y + gb.x * eb.x + gb.y * eb.y);
        if (lane == 0) d_vgate[t * d_vgate_stride + h] = __float2bfloat16(dot);
      }
    }
  }
}

// Backward of the QKV post-processing from its OUTPUTS (interleaved-pair layout): for the projection whose epilogue
// already produced q, k, v (csrc/epi_qkv.cuh) no copy of the raw projection exists.  The normalised pre-rotary values
// are recovered from the outputs - the rotation is orthogonal, so n = R^T(out) for the rotating dims; the stationary
// half of k sits one row down when the key offset is on (the last token's in k_last) - and
//   d_x = rstd * (d_n - n * <d_n, n> / 128)        with d_n = R^T(d_out) (and the offset undone).
__global__ void __launch_bounds__(QP_WARPS * 32)
qkv_post_bwd_from_out_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                             const __nv_bfloat16* __restrict__ k_last, const float* __restrict__ cos_t,
                             const float* __restrict__ sin_t, const float* __restrict__ rstd_q, const float* __restrict__ rstd_k,
                             const __nv_bfloat16* __restrict__ dq, const __nv_bfloat16* __restrict__ dk,
                             const __nv_bfloat16* __restrict__ dv, const __nv_bfloat16* __restrict__ ve,
                             const __nv_bfloat16* __restrict__ vgate, int vgate_stride, __nv_bfloat16* __restrict__ d_qkv,
                             __nv_bfloat16* __restrict__ d_ve, __nv_bfloat16* __restrict__ d_vgate, int d_vgate_stride,
                             long long T, int H, int paired, int key_offset) {
  const int lane = threadIdx.x & 31;
  const long long idx = (long long)blockIdx.x * QP_WARPS + (threadIdx.x >> 5);
  if (idx >= T * H) return;
  const long long t = idx / H;
  const int h = (int)(idx % H);
  const long long ld = 3LL * H * 128;
  const long long pos = paired ? 2 * t + (h & 1) : t;
  float cs[2] = {1.f, 1.f}, sn[2] = {0.f, 0.f};
  const bool rot = lane < 16;                           // lane l owns dims 4l..4l+3: pairs 2l and 2l+1 rotate for l < 16
  if (rot) {
    cs[0] = cos_t[pos * 32 + 2 * lane]; cs[1] = cos_t[pos * 32 + 2 * lane + 1];
    sn[0] = sin_t[pos * 32 + 2 * lane]; sn[1] = sin_t[pos * 32 + 2 * lane + 1];
  }
  auto cvt4 = [](uint2 u, float (&f)[4]) {
    const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(hh[0]), b = __bfloat1622float2(hh[1]);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  };
  auto ldu = [](const __nv_bfloat16* p) { return *reinterpret_cast<const uint2*>(p); };
  auto unrot = [&](float (&f)[4]) {                     // transpose of the rotation on the two pairs of this lane
    const float a0 = f[0], a1 = f[1], b0 = f[2], b1 = f[3];
    f[0] = cs[0] * a0 - sn[0] * a1; f[1] = cs[0] * a1 + sn[0] * a0;
    f[2] = cs[1] * b0 - sn[1] * b1; f[3] = cs[1] * b1 + sn[1] * b0;
  };
  // every load of this (token, head) is issued before the first row sum: one memory round trip per warp
  const long long e = idx * 128 + lane * 4;
  const bool shifted = !rot && key_offset;              // stationary half of k: lives one row down
  const uint2 uq = ldu(q + e), udq = ldu(dq + e), uk = ldu(k + e), udk = ldu(dk + e), udv = ldu(dv + e);
  uint2 uk2 = make_uint2(0u, 0u), udk2 = make_uint2(0u, 0u), uve = make_uint2(0u, 0u);
  if (shifted) {
    if (t + 1 < T) { uk2 = ldu(k + e + H * 128); udk2 = ldu(dk + e + H * 128); }
    else if (t != 0) uk2 = ldu(k_last + h * 64 + (lane - 16) * 4);
  }
  if (ve && d_vgate) uve = ldu(ve + e);
  const float rq = rstd_q[idx], rk = rstd_k[idx];
  const float gt = (ve && vgate) ? __bfloat162float(vgate[t * vgate_stride + h]) : 1.f;
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    float n[4], d[4];
    cvt4(which ? uk : uq, n);
    cvt4(which ? udk : udq, d);
    if (rot) {
      unrot(n);
      unrot(d);
    } else if (which == 1 && key_offset) {
      // n[t, 64:] was stored at row t + 1 (and at row 0 for t = 0); its gradient arrives from there
      float g0[4] = {0.f, 0.f, 0.f, 0.f};
      if (t == 0) {
#pragma unroll
        for (int u = 0; u < 4; ++u) g0[u] = d[u];       // row 0 kept its own stationary half: n = out, gradient d
      }
      if (t + 1 < T) {
        float dd[4];
        cvt4(udk2, dd);
        if (t != 0) cvt4(uk2, n);
#pragma unroll
        for (int u = 0; u < 4; ++u) d[u] = dd[u] + g0[u];
      } else {
        if (t != 0) cvt4(uk2, n);
#pragma unroll
        for (int u = 0; u < 4; ++u) d[u] = g0[u];
      }
    }
    const float r = which ? rk : rq;
    const float s = warp_sum(d[0] * n[0] + d[1] * n[1] + d[2] * n[2] + d[3] * n[3]) * (1.f / 128.f);
    uint2 w;
    w.x = pack_bf16x2(r * (d[0] - n[0] * s), r * (d[1] - n[1] * s));
    w.y = pack_bf16x2(r * (d[2] - n[2] * s), r * (d[3] - n[3] * s));
    *reinterpret_cast<uint2*>(d_qkv + t * ld + (which * H + h) * 128 + lane * 4) = w;
  }
  {
    *reinterpret_cast<uint2*>(d_qkv + t * ld + (2 * H + h) * 128 + lane * 4) = udv;
    if (ve) {
      float g[4];
      cvt4(udv, g);
      if (d_ve) {
        uint2 w;
        w.x = pack_bf16x2(gt * g[0], gt * g[1]); w.y = pack_bf16x2(gt * g[2], gt * g[3]);
        *reinterpret_cast<uint2*>(d_ve + e) = w;
      }
      if (d_vgate) {
        float ev[4];
        cvt4(uve, ev);
        const float dot = warp_sum(g[0] * ev[0] + g[1] * ev[1] + g[2] * ev[2] + g[3] * ev[3]);
        if (lane == 0) d_vgate[t * d_vgate_stride + h] = __float2bfloat16(dot);
      }
    }
  }
}

// =====================================================================================================
// Attention output gating, one warp per (token, head):
//   y' = (y - tanh(alpha[t,h]) * (<y,v> / max(<v,v>, 1e-8)) * v) * gate[t,h]      (alpha, gate optional)
__global__ void __launch_bounds__(QP_WARPS * 32)
xsa_gate_fwd_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ alpha,
                    int alpha_stride, const __nv_bfloat16* __restrict__ gate, int gate_stride, __nv_bfloat16* __restrict__ out,
                    long long T, int H) {
  const int lane = threadIdx.x & 31;
  const long long idx = (long long)blockIdx.x * QP_WARPS + (threadIdx.x >> 5);
  if (idx >= T * H) return;
  const long long t = idx / H;
  const int h = (int)(idx % H);
  uint2 yu = *reinterpret_cast<const uint2*>(y + idx * 128 + lane * 4);
  // the per-head scalars are fetched with the rows, not behind the row sums
  const float alpha_raw = alpha ? __bfloat162float(alpha[t * alpha_stride + h]) : 0.f;
  const float gt = gate ? __bfloat162float(gate[t * gate_stride + h]) : 1.f;
  const __nv_bfloat162* yh = reinterpret_cast<const __nv_bfloat162*>(&yu);
  float2 ya = __bfloat1622float2(yh[0]), yb = __bfloat1622float2(yh[1]);
  float o0 = ya.x, o1 = ya.y, o2 = yb.x, o3 = yb.y;
  if (alpha) {
    uint2 vu = *reinterpret_cast<const uint2*>(v + idx * 128 + lane * 4);
    const __nv_bfloat162* vh = reinterpret_cast<const __nv_bfloat162*>(&vu);
    float2 va = __bfloat1622float2(vh[0]), vb = __bfloat1622float2(vh[1]);
    const float yv = warp_sum(ya.x * va.x + ya.y * va.y + yb.x * vb.x + yb.y * vb.y);
    const float vv = fmaxf(warp_sum(va.x * va.x + va.y * va.y + vb.x * vb.x + vb.y * vb.y), 1e-8f);
    const float c = tanhf(alpha_raw) * yv / vv;
    o0 -= c * va.x; o1 -= c * va.y; o2 -= c * vb.x; o3 -= c * vb.y;
  }
  if (gate) {
    o0 *= gt; o1 *= gt; o2 *= gt; o3 *= gt;
  }
  uint2 w;
  w.x = pack_bf16x2(o0, o1); w.y = pack_bf16x2(o2, o3);
  *reinterpret_cast<uint2*>(out + idx * 128 + lane * 4) = w;
}

__global__ void __launch_bounds__(QP_WARPS * 32)
xsa_gate_bwd_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ alpha,
                    int alpha_stride, const __nv_bfloat16* __restrict__ gate, int gate_stride, const __nv_bfloat16* __restrict__ dout,
                    __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ dv, __nv_bfloat16* __restrict__ dalpha,
                    int dalpha_stride, __nv_bfloat16* __restrict__ dgate, int dgate_stride, long long T, int H) {
  const int lane = threadIdx.x & 31;
  const long long idx = (long long)blockIdx.x * QP_WARPS + (threadIdx.x >> 5);
  if (idx >= T * H) return;
  const long long t = idx / H;
  const int h = (int)(idx % H);
  // every load first: the per-head scalars would otherwise be fetched behind the row sums
  uint2 yu = *reinterpret_cast<const uint2*>(y + idx * 128 + lane * 4);
  uint2 gu = *reinterpret_cast<const uint2*>(dout + idx * 128 + lane * 4);
  uint2 vu = make_uint2(0u, 0u);
  if (alpha) vu = *reinterpret_cast<const uint2*>(v + idx * 128 + lane * 4);
  const float alpha_raw = alpha ? __bfloat162float(alpha[t * alpha_stride + h]) : 0.f;
  const float gt = gate ? __bfloat162float(gate[t * gate_stride + h]) : 1.f;
  const __nv_bfloat162* yh = reinterpret_cast<const __nv_bfloat162*>(&yu);
  const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gu);
  float2 ya = __bfloat1622float2(yh[0]), yb = __bfloat1622float2(yh[1]);
  float2 ga = __bfloat1622float2(gh[0]), gb = __bfloat1622float2(gh[1]);
  float Y[4] = {ya.x, ya.y, yb.x, yb.y}, G[4] = {ga.x, ga.y, gb.x, gb.y}, V[4] = {0, 0, 0, 0};
  float c = 0.f, th = 0.f, yv = 0.f, vv = 1.f;
  bool clamped = false;
  if (alpha) {
    const __nv_bfloat162* vh = reinterpret_cast<const __nv_bfloat162*>(&vu);
    float2 va = __bfloat1622float2(vh[0]), vb = __bfloat1622float2(vh[1]);
    V[0] = va.x; V[1] = va.y; V[2] = vb.x; V[3] = vb.y;
    yv = warp_sum(Y[0] * V[0] + Y[1] * V[1] + Y[2] * V[2] + Y[3] * V[3]);
    vv = warp_sum(V[0] * V[0] + V[1] * V[1] + V[2] * V[2] + V[3] * V[3]);
    clamped = vv < 1e-8f;
    vv = fmaxf(vv, 1e-8f);
    th = tanhf(alpha_raw);
    c = th * yv / vv;
  }
  // z = y - c v ; out = z * gt
  if (dgate) {
    float zdot = warp_sum(G[0] * (Y[0] - c * V[0]) + G[1] * (Y[1] - c * V[1]) + G[2] * (Y[2] - c * V[2]) + G[3] * (Y[3] - c * V[3]));
    if (lane == 0) dgate[t * dgate_stride + h] = __float2bfloat16(zdot);
  }
  float dz[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) dz[i] = G[i] * gt;
  float DY[4] = {dz[0], dz[1], dz[2], dz[3]}, DV[4] = {0, 0, 0, 0};
  if (alpha) {
    const float dzv = warp_sum(dz[0] * V[0] + dz[1] * V[1] + dz[2] * V[2] + dz[3] * V[3]);   // <dz, v>
    // c = th * yv / vv:  dc = -<dz, v>
    const float dc = -dzv;
    if (dalpha && lane == 0) dalpha[t * dalpha_stride + h] = __float2bfloat16(dc * (yv / vv) * (1.f - th * th));
    const float dyv = dc * th / vv;                          // d/d<y,v>
    const float dvv = clamped ? 0.f : -dc * th * yv / (vv * vv);   // d/d<v,v>
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      DY[i] += dyv * V[i];
      DV[i] = -c * dz[i] + dyv * Y[i] + 2.f * dvv * V[i];
    }
    if (dv) {
      uint2 w;
      w.x = pack_bf16x2(DV[0], DV[1]); w.y = pack_bf16x2(DV[2], DV[3]);
      *reinterpret_cast<uint2*>(dv + idx * 128 + lane * 4) = w;
    }
  }
  uint2 w;
  w.x = pack_bf16x2(DY[0], DY[1]); w.y = pack_bf16x2(DY[2], DY[3]);
  *reinterpret_cast<uint2*>(dy + idx * 128 + lane * 4) = w;
}

}  // namespace mng

using namespace mng;

#define LC_DISPATCH(KERNEL, ...)                                                                       \
  do {                                                                                                 \
    if (cols % 256 != 0 || cols > 1024) return -1;                                                     \
    const unsigned grid = (unsigned)((rows + LC_WARPS - 1) / LC_WARPS);                                \
    if (cols <= 256) KERNEL<1><<<grid, LC_WARPS * 32, 0, (cudaStream_t)stream>>>(__VA_ARGS__);         \
    else if (cols <= 768) KERNEL<3><<<grid, LC_WARPS * 32, 0, (cudaStream_t)stream>>>(__VA_ARGS__);    \
    else KERNEL<4><<<grid, LC_WARPS * 32, 0, (cudaStream_t)stream>>>(__VA_ARGS__);                     \
    return cudaGetLastError() == cudaSuccess ? 0 : -2;                                                 \
  } while (0)

MNG_DEFINE_BOUNDS_QUERY(glue)

extern "C" int mng_lincomb_fwd(const LinCombArgs* a, void* out, long long rows, int cols, void* stream) {
  if (rows == 0) return 0;
  if (a->k < 1 || a->k > LC_MAX_TERMS) return -3;
  LC_DISPATCH(lincomb_fwd_kernel, *a, (__nv_bfloat16*)out, rows, cols);
}

extern "C" int mng_lincomb_bwd(const LinCombArgs* a, const LinCombGrads* g, const void* gout, long long rows, int cols, void* stream) {
  if (rows == 0) return 0;
  if (a->k < 1 || a->k > LC_MAX_TERMS) return -3;
  LC_DISPATCH(lincomb_bwd_kernel, *a, *g, (const __nv_bfloat16*)gout, rows, cols);
}

extern "C" int mng_qkv_post_fwd(const void* qkv, const float* cos_t, const float* sin_t, const void* ve, const void* vgate,
                                int vgate_stride, const void* vadd, void* q, void* k, void* v, float* rstd_q, float* rstd_k,
                                long long T, int H, int paired, int key_offset, int split, void* stream) {
  if (T == 0) return 0;
  const unsigned grid = (unsigned)((T * H + QP_WARPS - 1) / QP_WARPS);
  auto kern = split ? qkv_post_fwd_kernel<true> : qkv_post_fwd_kernel<false>;
  kern<<<grid, QP_WARPS * 32, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)qkv, cos_t, sin_t, (const __nv_bfloat16*)ve, (const __nv_bfloat16*)vgate, vgate_stride,
      (const __nv_bfloat16*)vadd, (__nv_bfloat16*)q, (__nv_bfloat16*)k, (__nv_bfloat16*)v, rstd_q, rstd_k, T, H, paired, key_offset);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_qkv_post_bwd(const void* qkv, const float* cos_t, const float* sin_t, const float* rstd_q, const float* rstd_k,
                                const void* dq, const void* dk, const void* dv, const void* ve, const void* vgate,
                                int vgate_stride, void* d_qkv, void* d_ve, void* d_vgate, int d_vgate_stride, long long T, int H,
                                int paired, int key_offset, int split, void* stream) {
  if (T == 0) return 0;
  const unsigned grid = (unsigned)((T * H + QP_WARPS - 1) / QP_WARPS);
  auto kern = split ? qkv_post_bwd_kernel<true> : qkv_post_bwd_kernel<false>;
  kern<<<grid, QP_WARPS * 32, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)qkv, cos_t, sin_t, rstd_q, rstd_k, (const __nv_bfloat16*)dq, (const __nv_bfloat16*)dk,
      (const __nv_bfloat16*)dv, (const __nv_bfloat16*)ve, (const __nv_bfloat16*)vgate, vgate_stride, (__nv_bfloat16*)d_qkv,
      (__nv_bfloat16*)d_ve, (__nv_bfloat16*)d_vgate, d_vgate_stride, T, H, paired, key_offset);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_qkv_post_bwd_from_out(const void* q, const void* k, const void* k_last, const float* cos_t, const float* sin_t,
                                         const float* rstd_q, const float* rstd_k, const void* dq, const void* dk, const void* dv,
                                         const void* ve, const void* vgate, int vgate_stride, void* d_qkv, void* d_ve,
                                         void* d_vgate, int d_vgate_stride, long long T, int H, int paired, int key_offset,
                                         void* stream) {
  const unsigned grid = (unsigned)((T * H + QP_WARPS - 1) / QP_WARPS);
  qkv_post_bwd_from_out_kernel<<<grid, QP_WARPS * 32, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)k_last, cos_t, sin_t, rstd_q, rstd_k,
      (const __nv_bfloat16*)dq, (const __nv_bfloat16*)dk, (const __nv_bfloat16*)dv, (const __nv_bfloat16*)ve,
      (const __nv_bfloat16*)vgate, vgate_stride, (__nv_bfloat16*)d_qkv, (__nv_bfloat16*)d_ve, (__nv_bfloat16*)d_vgate,
      d_vgate_stride, T, H, paired, key_offset);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_xsa_gate_fwd(const void* y, const void* v, const void* alpha, int alpha_stride, const void* gate,
                                int gate_stride, void* out, long long T, int H, void* stream) {
  if (T == 0) return 0;
  const unsigned grid = (unsigned)((T * H + QP_WARPS - 1) / QP_WARPS);
  xsa_gate_fwd_kernel<<<grid, QP_WARPS * 32, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)y, (const __nv_bfloat16*)v, (const __nv_bfloat16*)alpha, alpha_stride, (const __nv_bfloat16*)gate,
      gate_stride, (__nv_bfloat16*)out, T, H);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_xsa_gate_bwd(const void* y, const void* v, const void* alpha, int alpha_stride, const void* gate,
                                int gate_stride, const void* dout, void* dy, void* dv, void* dalpha, int dalpha_stride,
                                void* dgate, int dgate_stride, long long T, int H, void* stream) {
  if (T == 0) return 0;
  const unsigned grid = (unsigned)((T * H + QP_WARPS - 1) / QP_WARPS);
  xsa_gate_bwd_kernel<<<grid, QP_WARPS * 32, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)y, (const __nv_bfloat16*)v, (const __nv_bfloat16*)alpha, alpha_stride, (const __nv_bfloat16*)gate,
      gate_stride, (const __nv_bfloat16*)dout, (__nv_bfloat16*)dy, (__nv_bfloat16*)dv, (__nv_bfloat16*)dalpha, dalpha_stride,
      (__nv_bfloat16*)dgate, dgate_stride, T, H);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
