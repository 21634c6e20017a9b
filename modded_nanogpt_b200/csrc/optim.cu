// Optimizer kernels (the math of `train_gpt.py:724-864`: Nesterov momentum, NorMuon variance reduction, cautious weight
// decay on a split fp32 master, Adam).  Each one can fold the neighbouring collective into its memory traffic:
// gradients are read from every rank's buffer through NVLink peer pointers (reduce-scatter /
// all-reduce fused into the first read) and updated weights are stored straight into every rank's
// parameter tensor (all-gather fused into the last write).  When the buffers also have an NVSwitch
// multicast address (PeerPtrs::mc), the gradient read is one `multimem.ld_reduce` (the switch sums the
// ranks' copies: 1/n of the bytes arrive) and the weight write one `multimem.st`.  With nranks == 1
// the same kernels are the plain single-GPU update.  Cross-rank ordering is provided by `mng_peer_barrier` launched
// before (gradients complete everywhere) and after (weights visible everywhere).
#include "api.h"
#include "comm.h"
#include "ptx.cuh"

namespace mng {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    float2 v = __bfloat1622float2(h[t]);
    f[2 * t] = v.x; f[2 * t + 1] = v.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 w;
  w.x = pack_bf16x2(f[0], f[1]); w.y = pack_bf16x2(f[2], f[3]); w.z = pack_bf16x2(f[4], f[5]); w.w = pack_bf16x2(f[6], f[7]);
  return w;
}

// ---------------------------------------------------------------------------------------------------
// Adam with cautious weight decay on a shard of n elements (n % 8 == 0 for bf16, % 4 for fp32).
//   g = mean over ranks of grads[r][off + i];  m,v fp32;  u = step*m/(sqrt(v)+eps);
//   u += wd * p * [u*p > 0];  p -= u  (p rounded to its dtype);  p written to params[r][off + i].
template <bool F32>
__global__ void __launch_bounds__(256)
adam_kernel(PeerPtrs grads, PeerPtrs params, long long off, float* __restrict__ m, float* __restrict__ v, long long n,
            float beta1, float beta2, float eps, float step_size, float eff_wd, float gmul,
            const unsigned char* __restrict__ row_mask, long long mask_stride, int row_elems) {
  constexpr int VEC = F32 ? 4 : 8;
  const long long nvec = n / VEC;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long long)gridDim.x * blockDim.x) {
    const long long e = off + i * VEC;
    float g[VEC], p[VEC];
#pragma unroll
    for (int t = 0; t < VEC; ++t) g[t] = 0.f;
    const long long row = row_mask ? e / row_elems : 0;     // a vector never straddles rows (row_elems % 8 == 0)
    if (grads.mc) {
      // one load through the multicast address: the switch reads every rank's copy and returns the sum
      bool any = true;
      if (row_mask && MNG_IN_RANGE(row, mask_stride)) {
        any = false;
        for (int r = 0; r < grads.n; ++r) any |= row_mask[r * mask_stride + row] != 0;
      }
      if (any) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(grads.mc) + e * (F32 ? 4 : 2);
        if constexpr (F32) {
          const float4 x = multimem_ld_sum_f32x4(src);
          g[0] = x.x; g[1] = x.y; g[2] = x.z; g[3] = x.w;
        } else {
          const uint4 x = multimem_ld_sum_bf16x8(src);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float2 v2 = __bfloat1622float2(h[t]);
            g[2 * t] = v2.x; g[2 * t + 1] = v2.y;
          }
        }
      }
    } else {
      // all peers' loads are issued before the first is consumed: one NVLink round trip instead of grads.n
      uint4 raw[MNG_MAX_RANKS];
#pragma unroll
      for (int r = 0; r < MNG_MAX_RANKS; ++r) {
        if (r < grads.n) {
          if (row_mask && MNG_IN_RANGE(row, mask_stride) && row_mask[r * mask_stride + row] == 0)
            raw[r] = make_uint4(0u, 0u, 0u, 0u);             // rank r did not touch this row: nothing crosses NVLink
          else
            raw[r] = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(grads.p[r]) + e * (F32 ? 4 : 2));
        }
      }
#pragma unroll
      for (int r = 0; r < MNG_MAX_RANKS; ++r) {
        if (r < grads.n) {
          if constexpr (F32) {
            const float* x = reinterpret_cast<const float*>(&raw[r]);
            g[0] += x[0]; g[1] += x[1]; g[2] += x[2]; g[3] += x[3];
          } else {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[r]);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const float2 v2 = __bfloat1622float2(h[t]);
              g[2 * t] += v2.x; g[2 * t + 1] += v2.y;
            }
          }
        }
      }
    }
    if constexpr (F32) {
      float4 x = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(params.p[params.self]) + e);
      p[0] = x.x; p[1] = x.y; p[2] = x.z; p[3] = x.w;
    } else {
      load8(reinterpret_cast<const __nv_bfloat16*>(params.p[params.self]) + e, *reinterpret_cast<float(*)[8]>(p));
    }
    float mm[VEC], vv[VEC];
#pragma unroll
    for (int t = 0; t < VEC; t += 4) {
      float4 a = *reinterpret_cast<const float4*>(m + i * VEC + t), b = *reinterpret_cast<const float4*>(v + i * VEC + t);
      mm[t] = a.x; mm[t + 1] = a.y; mm[t + 2] = a.z; mm[t + 3] = a.w;
      vv[t] = b.x; vv[t + 1] = b.y; vv[t + 2] = b.z; vv[t + 3] = b.w;
    }
#pragma unroll
    for (int t = 0; t < VEC; ++t) {
      float gg = g[t] * gmul;
      if constexpr (!F32) gg = __bfloat162float(__float2bfloat16(gg));   // the averaged gradient travels as bf16
      mm[t] = mm[t] * beta1 + gg * (1.f - beta1);
      vv[t] = vv[t] * beta2 + gg * gg * (1.f - beta2);
      float u = step_size * (mm[t] / (sqrtf(vv[t]) + eps));
      if (u * p[t] > 0.f) u += eff_wd * p[t];
      p[t] -= u;
    }
#pragma unroll
    for (int t = 0; t < VEC; t += 4) {
      *reinterpret_cast<float4*>(m + i * VEC + t) = make_float4(mm[t], mm[t + 1], mm[t + 2], mm[t + 3]);
      *reinterpret_cast<float4*>(v + i * VEC + t) = make_float4(vv[t], vv[t + 1], vv[t + 2], vv[t + 3]);
    }
    if (params.mc) {                                          // one store through the switch lands on every rank
      if constexpr (F32) multimem_st_f32x4(reinterpret_cast<float*>(params.mc) + e, make_float4(p[0], p[1], p[2], p[3]));
      else multimem_st_bf16x8(reinterpret_cast<__nv_bfloat16*>(params.mc) + e, pack8(*reinterpret_cast<float(*)[8]>(p)));
    } else {
      for (int r = 0; r < params.n; ++r) {
        if constexpr (F32) {
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(params.p[r]) + e) = make_float4(p[0], p[1], p[2], p[3]);
        } else {
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(params.p[r]) + e) = pack8(*reinterpret_cast<float(*)[8]>(p));
        }
      }
    }
  }
}

// One launch for a batch of small replicated parameters (gates, scalars, the MUDD matrices; `train_gpt.py:597-599`
// issues one all-reduce and `:840-864` one compiled update per such parameter): blockIdx.y picks the parameter, elements are handled one by one so that no size or alignment rule applies.  Every rank sums all ranks'
// gradients in the same order and updates its own copy, so the copies stay bitwise equal.
__global__ void __launch_bounds__(256)
adam_small_kernel(const __grid_constant__ SmallAdamTable t) {
  const SmallAdamEntry& e = t.e[blockIdx.y];
  const uint8_t* own = reinterpret_cast<const uint8_t*>(t.base.p[t.base.self]);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < e.n; i += (long long)gridDim.x * blockDim.x) {
    float g = 0.f;
#pragma unroll
    for (int r = 0; r < MNG_MAX_RANKS; ++r) {
      if (r < t.base.n) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(t.base.p[r]) + e.g_off;
        g += e.is_f32 ? reinterpret_cast<const float*>(src)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src)[i]);
      }
    }
    g *= t.gmul;
    if (!e.is_f32) g = __bfloat162float(__float2bfloat16(g));
    uint8_t* pp = const_cast<uint8_t*>(own) + e.p_off;
    float p = e.is_f32 ? reinterpret_cast<float*>(pp)[i] : __bfloat162float(reinterpret_cast<__nv_bfloat16*>(pp)[i]);
    const float mm = e.m[i] * e.beta1 + g * (1.f - e.beta1);
    const float vv = e.v[i] * e.beta2 + g * g * (1.f - e.beta2);
    e.m[i] = mm;
    e.v[i] = vv;
    float u = e.step_size * (mm / (sqrtf(vv) + e.eps));
    if (u * p > 0.f) u += e.eff_wd * p;
    p -= u;
    if (e.is_f32) reinterpret_cast<float*>(pp)[i] = p;
    else reinterpret_cast<__nv_bfloat16*>(pp)[i] = __float2bfloat16(p);
  }
}

// ---------------------------------------------------------------------------------------------------
// Reduce-scatter + Nesterov momentum:  g = gmul * sum_r grads[r][off+i] (rounded to bf16, as the
// averaged gradient would be on the wire);  buf = lerp(buf, g, 1-mu);  u = lerp(g, buf, mu);
// out = bf16(u);  sumsq[matrix] += out^2.   per_mat % 8 == 0.
__global__ void __launch_bounds__(256)
nesterov_kernel(PeerPtrs grads, long long off, float* __restrict__ buf, __nv_bfloat16* __restrict__ out,
                float* __restrict__ sumsq, long long mats, long long per_mat, float mu, float gmul, int its) {
  // A CTA takes chunks of its x 8 groups (its <= 16) of 32 vectors (32 KB of gradient) in grid-stride order; inside a chunk its eight
  // warps interleave.  A warp keeps the sum of squares of its groups in a register and adds it to the matrix's total
  // at the end of the chunk or when the matrix changes: `its` times fewer adds to one address (they serialise) than one
  // per group, while neighbouring CTAs still sweep neighbouring addresses.
  const long long vec_per_mat = per_mat / 8;                 // a multiple of 32: a group never straddles matrices
  const long long ngroups = mats * vec_per_mat / 32;
  const long long per_chunk = 8LL * its;
  const long long nchunks = (ngroups + per_chunk - 1) / per_chunk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x) {
  float ss = 0.f;
  long long cur = -1;
  for (int it = 0; it < its; ++it) {
    const long long grp = chunk * per_chunk + it * 8 + warp;
    if (grp >= ngroups) break;
    const long long i = grp * 32 + lane;
    const long long mat = i / vec_per_mat;
    if (mat != cur) {                                        // warp-uniform
      if (cur >= 0) {
        ss = warp_sum(ss);
        if (lane == 0) atomicAdd(sumsq + cur, ss);
      }
      ss = 0.f;
      cur = mat;
    }
    float g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (grads.mc) {
      const uint4 x = multimem_ld_sum_bf16x8(reinterpret_cast<const __nv_bfloat16*>(grads.mc) + off + i * 8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 v2 = __bfloat1622float2(h2[t]);
        g[2 * t] = v2.x; g[2 * t + 1] = v2.y;
      }
    } else {
      uint4 raw[MNG_MAX_RANKS];
#pragma unroll
      for (int r = 0; r < MNG_MAX_RANKS; ++r)
        if (r < grads.n) raw[r] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(grads.p[r]) + off + i * 8);
#pragma unroll
      for (int r = 0; r < MNG_MAX_RANKS; ++r) {
        if (r < grads.n) {
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[r]);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float2 v2 = __bfloat1622float2(h2[t]);
            g[2 * t] += v2.x; g[2 * t + 1] += v2.y;
          }
        }
      }
    }
    float b[8], u[8];
    float4 b0 = *reinterpret_cast<const float4*>(buf + i * 8), b1 = *reinterpret_cast<const float4*>(buf + i * 8 + 4);
    b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float gg = __bfloat162float(__float2bfloat16(g[t] * gmul));
      b[t] = b[t] + (1.f - mu) * (gg - b[t]);
      u[t] = __bfloat162float(__float2bfloat16(b[t] - (b[t] - gg) * (1.f - mu)));   // lerp(g, buf, mu), mu >= 0.5
      ss += u[t] * u[t];
    }
    *reinterpret_cast<float4*>(buf + i * 8) = make_float4(b[0], b[1], b[2], b[3]);
    *reinterpret_cast<float4*>(buf + i * 8 + 4) = make_float4(b[4], b[5], b[6], b[7]);
    *reinterpret_cast<uint4*>(out + i * 8) = pack8(u);
  }
  if (cur >= 0) {
    ss = warp_sum(ss);
    if (lane == 0) atomicAdd(sumsq + cur, ss);
  }
  }
}

__global__ void __launch_bounds__(256)
scale_by_norm_kernel(__nv_bfloat16* __restrict__ x, const float* __restrict__ sumsq, long long mats, long long per_mat) {
  const long long vec_per_mat = per_mat / 8;
  const long long nvec = mats * vec_per_mat;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long long)gridDim.x * blockDim.x) {
    // X / (||X||_F * 1.02 + 1e-6) with the norm and the quotient rounded to bf16 like the tensor ops they replace
    const float nrm = __bfloat162float(__float2bfloat16(sqrtf(sumsq[i / vec_per_mat])));
    const float den = __bfloat162float(__float2bfloat16(__bfloat162float(__float2bfloat16(nrm * 1.02f)) + 1e-6f));
    float f[8];
    load8(x + i * 8, f);
#pragma unroll
    for (int t = 0; t < 8; ++t) f[t] = f[t] / den;
    *reinterpret_cast<uint4*>(x + i * 8) = pack8(f);
  }
}

// ---------------------------------------------------------------------------------------------------
// NorMuon: per-row (or per-column) mean square of v -> EMA second moment -> rescale keeping the
// Frobenius norm -> cautious weight decay + step on the fp32 master (bf16 weight | uint16 mantissa)
// -> bf16 weight stored to every rank.  The statistics kernel runs `chunks` CTAs per matrix, each over a
// slice of the rows (columns); the last CTA of a matrix to finish (a counter per matrix, left at zero
// again) sums the slices' partial norms in a fixed order and applies the norm-preserving ratio, so the
// result does not depend on the order in which the CTAs ran.  Then a grid-stride update kernel.
constexpr int NORMUON_MAX_CHUNKS = 32;
__global__ void __launch_bounds__(1024)
normuon_stats_kernel(const __nv_bfloat16* __restrict__ v, float* __restrict__ second_mom, float* __restrict__ scale_out,
                     float* __restrict__ partials, unsigned int* __restrict__ counters, int rows, int cols, int red_rows,
                     float beta2) {
  // red_rows: one statistic per row (mean over columns); else one per column (mean over rows).
  const long long mat = blockIdx.y;
  const int chunk = blockIdx.x, chunks = gridDim.x;
  const __nv_bfloat16* vm = v + mat * (long long)rows * cols;
  const int nstat = red_rows ? rows : cols;
  const int nred = red_rows ? cols : rows;
  const int per = (nstat + chunks - 1) / chunks;
  const int s_lo = chunk * per, s_hi = min(nstat, s_lo + per);
  float* sm = second_mom + mat * nstat;
  float* sc = scale_out + mat * nstat;
  __shared__ float s_a[32], s_b[32];
  __shared__ bool s_last;
  float tot_old = 0.f, tot_new = 0.f;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  if (red_rows) {
    for (int r = s_lo + warp; r < s_hi; r += nwarps) {
      float ss = 0.f;
      for (int c = lane * 8; c < cols; c += 256) {
        float f[8];
        load8(vm + (long long)r * cols + c, f);
#pragma unroll
        for (int t = 0; t < 8; ++t) ss += f[t] * f[t];
      }
      ss = warp_sum(ss);
      if (lane == 0) {
        const float mean = ss / nred;
        const float s = sm[r] + (1.f - beta2) * (mean - sm[r]);
        sm[r] = s;
        const float step = rsqrtf(fmaxf(s, 1e-10f));
        sc[r] = step;
        tot_old += ss;
        tot_new += ss * step * step;
      }
    }
  } else {
    // a CTA owns at most 128 columns: thread (rg, cl) sums rows rg, rg + 8, ... of column s_lo + cl, then the eight
    // row groups are added through shared memory
    __shared__ float s_col[8][128];
    const int cl = threadIdx.x & 127, rg = threadIdx.x >> 7;
    const int c = s_lo + cl;
    float part = 0.f;
    if (c < s_hi) {
      for (int r = rg; r < rows; r += 8) {
        const float f = __bfloat162float(vm[(long long)r * cols + c]);
        part += f * f;
      }
    }
    s_col[rg][cl] = part;
    __syncthreads();
    if (rg == 0 && c < s_hi) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += s_col[k][cl];
      const float mean = ss / nred;
      const float s = sm[c] + (1.f - beta2) * (mean - sm[c]);
      sm[c] = s;
      const float step = rsqrtf(fmaxf(s, 1e-10f));
      sc[c] = step;
      tot_old += ss;
      tot_new += ss * step * step;
    }
  }
  tot_old = warp_sum(tot_old);
  tot_new = warp_sum(tot_new);
  if (lane == 0) { s_a[warp] = tot_old; s_b[warp] = tot_new; }
  __syncthreads();
  if (warp == 0) {
    float a = lane < nwarps ? s_a[lane] : 0.f, b = lane < nwarps ? s_b[lane] : 0.f;
    a = warp_sum(a); b = warp_sum(b);
    if (lane == 0) {
      float* part = partials + (mat * NORMUON_MAX_CHUNKS + chunk) * 2;
      part[0] = a; part[1] = b;
      __threadfence();                                       // partials and this CTA's sc[] before the count
      const unsigned int done = atomicAdd(counters + mat, 1u);
      s_last = done == (unsigned int)chunks - 1;
      if (s_last) counters[mat] = 0u;                        // ready for the next call
    }
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (threadIdx.x == 0) {
    float a = 0.f, b = 0.f;
    const volatile float* part = partials + mat * NORMUON_MAX_CHUNKS * 2;
    for (int k = 0; k < chunks; ++k) { a += part[2 * k]; b += part[2 * k + 1]; }
    s_a[0] = sqrtf(a);
    s_b[0] = fmaxf(sqrtf(b), 1e-10f);
  }
  __syncthreads();
  const float ratio = s_a[0] / s_b[0];
  volatile float* scv = sc;
  for (int i = threadIdx.x; i < nstat; i += blockDim.x) scv[i] = __bfloat162float(__float2bfloat16(scv[i] * ratio));
}

__global__ void __launch_bounds__(256)
normuon_update_kernel(PeerPtrs params, long long off, unsigned short* __restrict__ mantissa, const __nv_bfloat16* __restrict__ v,
                      const float* __restrict__ scale, long long mats, int rows, int cols, int red_rows, float eff_wd,
                      float lr_base, const float* __restrict__ lr_mul_per_mat) {
  const long long per_mat = (long long)rows * cols;
  const long long nvec = mats * per_mat / 8;
  const int nstat = red_rows ? rows : cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long long)gridDim.x * blockDim.x) {
    const long long e = i * 8;
    const long long mat = e / per_mat;
    const long long in_mat = e - mat * per_mat;
    const int r = (int)(in_mat / cols), c = (int)(in_mat % cols);
    const float lr = lr_base * lr_mul_per_mat[mat];
    float g[8];
    load8(v + e, g);
    const float* sc = scale + mat * nstat;
    uint4 pw = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(params.p[params.self]) + off + e);
    uint4 mw = *reinterpret_cast<const uint4*>(mantissa + e);
    const unsigned short* ph = reinterpret_cast<const unsigned short*>(&pw);
    const unsigned short* ml = reinterpret_cast<const unsigned short*>(&mw);
    uint4 po, mo;
    unsigned short* poh = reinterpret_cast<unsigned short*>(&po);
    unsigned short* mol = reinterpret_cast<unsigned short*>(&mo);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float s = red_rows ? sc[r] : sc[c + t];
      const float gg = __bfloat162float(__float2bfloat16(g[t] * s));         // v * bf16 scale, held in bf16
      const float p = __uint_as_float(((uint32_t)ph[t] << 16) | ml[t]);
      const float decay = (gg * p >= 0.f) ? p * eff_wd * lr : 0.f;
      const float pn = p - decay - gg * lr;
      const uint32_t bits = __float_as_uint(pn);
      poh[t] = (unsigned short)(bits >> 16);
      mol[t] = (unsigned short)(bits & 0xffff);
    }
    *reinterpret_cast<uint4*>(mantissa + e) = mo;
    if (params.mc) {
      multimem_st_bf16x8(reinterpret_cast<__nv_bfloat16*>(params.mc) + off + e, po);
    } else {
      for (int q = 0; q < params.n; ++q) *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(params.p[q]) + off + e) = po;
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// Cross-rank barrier on signal pads.  pads[r] points to rank r's pad: an array of `nranks` 32-bit
// epoch slots.  Every rank publishes `epoch` into slot [rank] of every pad, then waits (bounded)
// until all slots of its own pad have reached `epoch`.
__global__ void peer_barrier_kernel(PeerPtrs pads, int rank, uint32_t epoch, uint32_t* status) {
  const int t = threadIdx.x;
  if (t < pads.n) {
    __threadfence_system();
    uint32_t* dst = reinterpret_cast<uint32_t*>(pads.p[t]) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(pads.p[rank]) + t;
    const long long t0 = clock64();
    uint32_t seen;
    while (true) {
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(seen) : "l"(mine) : "memory");
      if ((int32_t)(seen - epoch) >= 0) break;
      if (clock64() - t0 > kWaitBudgetCycles) { atomicCAS(status, 0u, ERR_WAIT_PEER); break; }
      __nanosleep(200);
    }
    __threadfence_system();
  }
}

static inline unsigned grid_for(long long nvec) {
  long long g = (nvec + 255) / 256;
  const long long cap = 148 * 8;
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace mng

using namespace mng;

MNG_DEFINE_BOUNDS_QUERY(optim)

extern "C" int mng_adam(const AdamDesc* d, void* stream) {
  const AdamDesc& a = *d;
  if (a.n == 0) return 0;
  const int vec = a.p_is_f32 ? 4 : 8;
  if (a.n % vec || a.off % vec) return -1;
  if (a.row_mask && (a.row_elems <= 0 || a.row_elems % 8 || a.mask_stride <= 0)) return -3;
  const unsigned grid = grid_for(a.n / vec);
  if (a.p_is_f32)
    adam_kernel<true><<<grid, 256, 0, (cudaStream_t)stream>>>(a.grads, a.params, a.off, a.exp_avg, a.exp_avg_sq, a.n, a.beta1,
                                                              a.beta2, a.eps, a.step_size, a.eff_wd, a.grad_mul, a.row_mask,
                                                              a.mask_stride, a.row_elems);
  else
    adam_kernel<false><<<grid, 256, 0, (cudaStream_t)stream>>>(a.grads, a.params, a.off, a.exp_avg, a.exp_avg_sq, a.n, a.beta1,
                                                               a.beta2, a.eps, a.step_size, a.eff_wd, a.grad_mul, a.row_mask,
                                                               a.mask_stride, a.row_elems);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_adam_small(const SmallAdamTable* t, void* stream) {
  if (t->count < 1 || t->count > MNG_SMALL_ADAM_MAX) return -1;
  long long most = 1;
  for (int i = 0; i < t->count; ++i) most = t->e[i].n > most ? t->e[i].n : most;
  const unsigned gx = (unsigned)((most + 255) / 256 > 64 ? 64 : (most + 255) / 256);
  adam_small_kernel<<<dim3(gx, (unsigned)t->count), 256, 0, (cudaStream_t)stream>>>(*t);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_fill_zero(void* p, long long bytes, void* stream) {
  return cudaMemsetAsync(p, 0, (size_t)bytes, (cudaStream_t)stream) == cudaSuccess ? 0 : -2;
}

extern "C" int mng_nesterov(const PeerPtrs* grads, long long off, float* buf, void* out_bf16, float* sumsq, long long mats,
                            long long per_mat, float momentum, float grad_mul, void* stream) {
  if (per_mat % 256) return -1;                              // 32 vectors of 8: a warp's group stays inside one matrix
  cudaStream_t s = (cudaStream_t)stream;
  cudaMemsetAsync(sumsq, 0, sizeof(float) * mats, s);
  // chunk length: long enough to thin out the adds to one address, short enough that every SM has several chunks
  const long long groups = mats * per_mat / 256;
  long long its = groups / (8LL * 148 * 4);
  its = its < 1 ? 1 : (its > 16 ? 16 : its);
  const long long nchunks = (groups + 8 * its - 1) / (8 * its);
  const unsigned grid = (unsigned)(nchunks < 148 * 8 ? nchunks : 148 * 8);
  nesterov_kernel<<<grid, 256, 0, s>>>(*grads, off, buf, (__nv_bfloat16*)out_bf16, sumsq, mats, per_mat, momentum, grad_mul, (int)its);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_scale_by_norm(void* x, const float* sumsq, long long mats, long long per_mat, void* stream) {
  if (per_mat % 8) return -1;
  scale_by_norm_kernel<<<grid_for(mats * per_mat / 8), 256, 0, (cudaStream_t)stream>>>((__nv_bfloat16*)x, sumsq, mats, per_mat);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_normuon_apply(const PeerPtrs* params, long long off, void* mantissa, const void* v, float* second_mom,
                                 float* scale_scratch, long long mats, int rows, int cols, int red_rows, float beta2, float eff_wd,
                                 float lr_base, const float* lr_mul_per_mat, void* stream) {
  // scale_scratch: mats * nstat scales, then mats * 64 partial norms, then mats counters (zero on entry, left zero)
  if (cols % 8) return -1;
  cudaStream_t s = (cudaStream_t)stream;
  const int nstat = red_rows ? rows : cols;
  float* partials = scale_scratch + mats * nstat;
  unsigned int* counters = reinterpret_cast<unsigned int*>(partials + mats * NORMUON_MAX_CHUNKS * 2);
  // rows: slices of >= 128 rows; columns: slices of exactly <= 128 columns (the kernel's shared-memory layout)
  int chunks = (nstat + 127) / 128;
  if (!red_rows && chunks > NORMUON_MAX_CHUNKS) return -4;
  chunks = chunks < 1 ? 1 : (chunks > NORMUON_MAX_CHUNKS ? NORMUON_MAX_CHUNKS : chunks);
  normuon_stats_kernel<<<dim3(chunks, (unsigned)mats), 1024, 0, s>>>((const __nv_bfloat16*)v, second_mom, scale_scratch, partials,
                                                                     counters, rows, cols, red_rows, beta2);
  normuon_update_kernel<<<grid_for(mats * (long long)rows * cols / 8), 256, 0, s>>>(
      *params, off, (unsigned short*)mantissa, (const __nv_bfloat16*)v, scale_scratch, mats, rows, cols, red_rows, eff_wd,
      lr_base, lr_mul_per_mat);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mng_peer_barrier(const PeerPtrs* pads, int rank, uint32_t epoch, uint32_t* status, void* stream) {
  peer_barrier_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(*pads, rank, epoch, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
