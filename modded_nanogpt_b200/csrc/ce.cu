// Softcapped cross-entropy, forward and gradient in one pass over the logits.
//
// One CTA per token row.  z = A*sigmoid((logit+B)/C) is bounded by A, so the log-sum-exp needs no
// running maximum: sum_j exp(z_j - A) stays within fp32 range.  The row of sigmoids is parked in
// shared memory as bf16 (vocab*2 bytes) between the reduction and the gradient sweep, so the
// logits are read from HBM exactly once and the gradient is written exactly once:
//   loss_i  = sum_k w_k (lse - z[t_{i+k}]) + w_p (lse - z[p_i])            (k < n_predict, i+k < rows)
//   dlogit  = grad_mul * (A/C) * (S_w * softmax(z) - [targets]) * s(1-s)
// Same contract as the reference kernel `triton_kernels.py:914-1171` (S_w sums all MTP weights,
// targets past the end of the batch drop out of the loss but not of S_w, prefix target < 0 = none).
#include "api.h"
#include "ptx.cuh"

namespace mng {

constexpr int CE_MAX_PREDICT = 8;

__device__ __forceinline__ float fast_sigmoid(float u) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u * 0.5f));
  return 0.5f + 0.5f * t;
}

// CACHE_E: also park exp(z - A) (bf16) next to the sigmoids so the gradient sweep needs no second
// exponential: 2 instead of 3 special-function evaluations per logit, which is what bounds this kernel
// once the logits stream at HBM speed.  Needs 4*vocab bytes of shared memory (one 1024-thread CTA per SM).
template <bool OUT_E5M2, bool CACHE_E, int CE_THREADS>
__global__ void __launch_bounds__(CE_THREADS, CACHE_E ? 1 : 2)
softcap_ce_kernel(const __nv_bfloat16* __restrict__ logits, const long long* __restrict__ targets,
                  const float* __restrict__ mtp_weights, int n_predict, const long long* __restrict__ prefix_targets,
                  const float* __restrict__ prefix_weight_ptr, float* __restrict__ losses, void* __restrict__ dlogits,
                  long long rows, int vocab, long long ld, float A, float B, float C, float grad_mul) {
  extern __shared__ __nv_bfloat16 sig[];
  __nv_bfloat16* ex = sig + vocab;                 // only touched when CACHE_E
  __shared__ float red[CE_THREADS / 32];
  __shared__ float s_lse, s_inv;
  const long long row = blockIdx.x;
  const __nv_bfloat16* lrow = logits + row * ld;
  const float inv_c = 1.f / C, b_over_c = B / C;
  const int nvec = vocab >> 3;

  float part = 0.f;
  for (int i = threadIdx.x; i < nvec; i += CE_THREADS) {
    uint4 u = *reinterpret_cast<const uint4*>(lrow + i * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    uint4 w, we;
    uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
    uint32_t* ep = reinterpret_cast<uint32_t*>(&we);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float2 f = __bfloat1622float2(h[t]);
      __nv_bfloat162 s2 = __floats2bfloat162_rn(fast_sigmoid(f.x * inv_c + b_over_c), fast_sigmoid(f.y * inv_c + b_over_c));
      wp[t] = *reinterpret_cast<uint32_t*>(&s2);
      float2 s = __bfloat1622float2(s2);
      const float e0 = __expf(A * s.x - A), e1 = __expf(A * s.y - A);
      part += e0 + e1;
      if constexpr (CACHE_E) ep[t] = pack_bf16x2(e0, e1);
    }
    *reinterpret_cast<uint4*>(sig + i * 8) = w;
    if constexpr (CACHE_E) *reinterpret_cast<uint4*>(ex + i * 8) = we;
  }
  part = warp_sum(part);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < CE_THREADS / 32; ++i) tot += red[i];
    s_lse = A + __logf(tot);
    s_inv = 1.f / tot;
  }
  __syncthreads();
  const float lse = s_lse, inv_tot = s_inv;

  const float prefix_weight = prefix_weight_ptr ? prefix_weight_ptr[0] : 0.f;
  const long long ptgt = prefix_targets ? prefix_targets[row] : -1;
  const bool pvalid = ptgt >= 0 && ptgt < vocab;
  float S_w = pvalid ? prefix_weight : 0.f;
  for (int k = 0; k < n_predict; ++k) S_w += mtp_weights[k];

  if (threadIdx.x == 0) {
    float loss = 0.f;
    for (int k = 0; k < n_predict; ++k) {
      const long long ti = row + k;
      if (ti < rows) {
        const long long t = targets[ti];
        if (t >= 0 && t < vocab) loss += mtp_weights[k] * (lse - A * __bfloat162float(sig[t]));
      }
    }
    if (pvalid) loss += prefix_weight * (lse - A * __bfloat162float(sig[ptgt]));
    losses[row] = loss;
  }

  const float gscale = grad_mul * (A * inv_c);
  for (int i = threadIdx.x; i < nvec; i += CE_THREADS) {
    uint4 u = *reinterpret_cast<const uint4*>(sig + i * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float g[8];
    if constexpr (CACHE_E) {
      uint4 ue = *reinterpret_cast<const uint4*>(ex + i * 8);
      const __nv_bfloat162* he = reinterpret_cast<const __nv_bfloat162*>(&ue);
      const float c = gscale * S_w * inv_tot;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float2 s = __bfloat1622float2(h[t]), e = __bfloat1622float2(he[t]);
        g[2 * t] = c * e.x * s.x * (1.f - s.x);
        g[2 * t + 1] = c * e.y * s.y * (1.f - s.y);
      }
    } else {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float2 s = __bfloat1622float2(h[t]);
        g[2 * t] = gscale * S_w * __expf(A * s.x - lse) * s.x * (1.f - s.x);
        g[2 * t + 1] = gscale * S_w * __expf(A * s.y - lse) * s.y * (1.f - s.y);
      }
    }
    if constexpr (OUT_E5M2) {
      uint2 w;
      w.x = pack_e5m2x2(g[0], g[1]) | ((uint32_t)pack_e5m2x2(g[2], g[3]) << 16);
      w.y = pack_e5m2x2(g[4], g[5]) | ((uint32_t)pack_e5m2x2(g[6], g[7]) << 16);
      *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(dlogits) + row * ld + i * 8) = w;
    } else {
      uint4 w;
      w.x = pack_bf16x2(g[0], g[1]); w.y = pack_bf16x2(g[2], g[3]); w.z = pack_bf16x2(g[4], g[5]); w.w = pack_bf16x2(g[6], g[7]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dlogits) + row * ld + i * 8) = w;
    }
  }
  __syncthreads();

  // Target columns: subtract the weights of every prediction that lands on the column.  Threads
  // that hit the same column compute the same value, so concurrent writes agree.
  if (threadIdx.x <= n_predict) {
    const int i = threadIdx.x;
    long long tgt = -1;
    bool valid;
    if (i < n_predict) {
      valid = row + i < rows;
      if (valid) tgt = targets[row + i];
      valid = valid && tgt >= 0 && tgt < vocab;
    } else {
      tgt = ptgt;
      valid = pvalid;
    }
    if (valid) {
      const float s = __bfloat162float(sig[tgt]);
      float hit = 0.f;
      for (int k = 0; k < n_predict; ++k)
        if (row + k < rows && targets[row + k] == tgt) hit += mtp_weights[k];
      if (pvalid && ptgt == tgt) hit += prefix_weight;
      const float gv = gscale * (S_w * __expf(A * s - lse) - hit) * s * (1.f - s);
      if constexpr (OUT_E5M2)
        reinterpret_cast<uint8_t*>(dlogits)[row * ld + tgt] = (uint8_t)(pack_e5m2x2(gv, 0.f) & 0xff);
      else
        reinterpret_cast<__nv_bfloat16*>(dlogits)[row * ld + tgt] = __float2bfloat16(gv);
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// Streaming variant: persistent 512-thread CTAs, two per SM, each walking rows blockIdx.x, +gridDim.x, ...
// A row of logits arrives in shared memory by one bulk async copy (cp.async.bulk, completion on an
// mbarrier) and is rewritten in place: raw logit -> bf16(exp(z-A) * s * (1-s)), the only per-column
// quantity the gradient sweep needs; the sigmoids at the (at most n_predict+1) target columns are
// recomputed from global memory while the copy is in flight.  The two CTAs of an SM run out of phase, so
// one CTA's copy and store-heavy gradient sweep overlap the other's special-function-heavy first sweep.
// One row buffer of vocab*2 bytes per CTA.  Needs vocab % 16 == 0 and 16-byte aligned rows.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :
               : "r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

constexpr int CE_STREAM_THREADS = 512;

template <bool OUT_E5M2>
__global__ void __launch_bounds__(CE_STREAM_THREADS, 2)
softcap_ce_stream_kernel(const __nv_bfloat16* __restrict__ logits, const long long* __restrict__ targets,
                         const float* __restrict__ mtp_weights, int n_predict,
                         const long long* __restrict__ prefix_targets, const float* __restrict__ prefix_weight_ptr,
                         float* __restrict__ losses, void* __restrict__ dlogits, long long rows, int vocab, long long ld,
                         float A, float B, float C, float grad_mul) {
  constexpr int TH = CE_STREAM_THREADS;
  extern __shared__ __align__(128) unsigned char ce_smem[];
  __nv_bfloat16* const buf = reinterpret_cast<__nv_bfloat16*>(ce_smem);
  __shared__ __align__(8) uint64_t bar;
  __shared__ float red[TH / 32];
  __shared__ uint32_t s_abort;
  const int tid = threadIdx.x, lane = tid & 31;
  const uint32_t bytes = (uint32_t)vocab * 2u;
  if (tid == 0) {
    mbar_init(&bar, 1);
    s_abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  const float half_inv_c = 0.5f / C, half_b_over_c = 0.5f * B / C;
  const float k2 = A * 1.4426950408889634f;            // exp(A*s - A) = exp2(k2*s - k2)
  const float gscale = grad_mul * (A / C);
  const float prefix_weight = prefix_weight_ptr ? prefix_weight_ptr[0] : 0.f;
  float w_sum = 0.f;
  for (int k = 0; k < n_predict; ++k) w_sum += mtp_weights[k];
  const int nvec = vocab >> 3;

  int it = 0;
  for (long long row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
    const __nv_bfloat16* lrow = logits + row * ld;
    if (tid == 0) {
      fence_proxy_async_smem();                         // the buffer was last touched by generic-proxy accesses
      mbar_expect_tx(&bar, bytes);
      bulk_load_1d(buf, lrow, bytes, &bar);
    }
    // this thread's target column (threads 0..n_predict): logit straight from global memory
    long long tgt = -1;
    bool tvalid = false;
    float tw = 0.f, ts = 0.f, hit = 0.f;
    const long long ptgt = prefix_targets ? prefix_targets[row] : -1;
    const bool pvalid = ptgt >= 0 && ptgt < vocab;
    if (tid <= n_predict) {
      if (tid < n_predict) {
        if (row + tid < rows) tgt = targets[row + tid];
        tw = mtp_weights[tid];
      } else {
        tgt = pvalid ? ptgt : -1;
        tw = prefix_weight;
      }
      tvalid = tgt >= 0 && tgt < vocab;
      if (tvalid) {
        float t;
        asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(__bfloat162float(lrow[tgt]) * half_inv_c + half_b_over_c));
        ts = 0.5f + 0.5f * t;
        for (int k = 0; k < n_predict; ++k)
          if (row + k < rows && targets[row + k] == tgt) hit += mtp_weights[k];
        if (pvalid && ptgt == tgt) hit += prefix_weight;
      }
    }
    if (!mbar_wait(&bar, (uint32_t)it & 1u, &s_abort)) s_abort = 1;
    __syncthreads();
    if (s_abort) {                                      // the copy never landed: mark what is left and leave
      for (long long r = row; r < rows; r += gridDim.x)
        if (tid == 0) losses[r] = __int_as_float(0x7fc00000);
      break;
    }

    float part = 0.f;
#pragma unroll 2
    for (int i = tid; i < nvec; i += TH) {
      uint4 u = *reinterpret_cast<const uint4*>(buf + i * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
      uint4 w;
      uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __bfloat1622float2(h[t]);
        float t0, t1;
        asm("tanh.approx.f32 %0, %1;" : "=f"(t0) : "f"(f.x * half_inv_c + half_b_over_c));
        asm("tanh.approx.f32 %0, %1;" : "=f"(t1) : "f"(f.y * half_inv_c + half_b_over_c));
        const float s0 = 0.5f + 0.5f * t0, s1 = 0.5f + 0.5f * t1;
        const float e0 = exp2f(k2 * s0 - k2), e1 = exp2f(k2 * s1 - k2);
        part += e0 + e1;
        wp[t] = pack_bf16x2(e0 * s0 * (0.5f - 0.5f * t0), e1 * s1 * (0.5f - 0.5f * t1));
      }
      *reinterpret_cast<uint4*>(buf + i * 8) = w;
    }
    part = warp_sum(part);
    if (lane == 0) red[tid >> 5] = part;
    __syncthreads();
    const float tot = warp_sum(lane < TH / 32 ? red[lane] : 0.f);
    const float lse = A + __logf(tot), inv_tot = 1.f / tot;
    const float S_w = w_sum + (pvalid ? prefix_weight : 0.f);

    if (tid < 32) {                                     // loss: the target threads all sit in warp 0
      float l = tvalid ? tw * (lse - A * ts) : 0.f;
      l = warp_sum(l);
      if (tid == 0) losses[row] = l;
    }

    const float c = gscale * S_w * inv_tot;
    if constexpr (OUT_E5M2) {
      uint8_t* drow = reinterpret_cast<uint8_t*>(dlogits) + row * ld;
#pragma unroll 2
      for (int i = tid; i < (vocab >> 4); i += TH) {
        const uint4 u0 = *reinterpret_cast<const uint4*>(buf + i * 16);
        const uint4 u1 = *reinterpret_cast<const uint4*>(buf + i * 16 + 8);
        const __nv_bfloat162* h0 = reinterpret_cast<const __nv_bfloat162*>(&u0);
        const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
        uint32_t o[4];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const float2 a = __bfloat1622float2(h0[2 * t]), b = __bfloat1622float2(h0[2 * t + 1]);
          o[t] = pack_e5m2x2(c * a.x, c * a.y) | ((uint32_t)pack_e5m2x2(c * b.x, c * b.y) << 16);
          const float2 d = __bfloat1622float2(h1[2 * t]), e = __bfloat1622float2(h1[2 * t + 1]);
          o[2 + t] = pack_e5m2x2(c * d.x, c * d.y) | ((uint32_t)pack_e5m2x2(c * e.x, c * e.y) << 16);
        }
        *reinterpret_cast<uint4*>(drow + i * 16) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    } else {
      __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(dlogits) + row * ld;
#pragma unroll 2
      for (int i = tid; i < nvec; i += TH) {
        const uint4 u = *reinterpret_cast<const uint4*>(buf + i * 8);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
        uint4 w;
        uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 a = __bfloat1622float2(h[t]);
          wp[t] = pack_bf16x2(c * a.x, c * a.y);
        }
        *reinterpret_cast<uint4*>(drow + i * 8) = w;
      }
    }
    __syncthreads();                                    // sweep done: the buffer is free, fix-ups may follow

    if (tid <= n_predict && tvalid) {                   // target columns: same value from every thread that hits one
      const float gv = gscale * (S_w * exp2f(k2 * ts - k2) * inv_tot - hit) * ts * (1.f - ts);
      if constexpr (OUT_E5M2)
        reinterpret_cast<uint8_t*>(dlogits)[row * ld + tgt] = (uint8_t)(pack_e5m2x2(gv, 0.f) & 0xff);
      else
        reinterpret_cast<__nv_bfloat16*>(dlogits)[row * ld + tgt] = __float2bfloat16(gv);
    }
  }
}

}  // namespace mng

using namespace mng;

extern "C" int mng_softcap_ce(const void* logits, const long long* targets, const float* mtp_weights, int n_predict,
                              const long long* prefix_targets, const float* prefix_weight, float* losses, void* dlogits,
                              int dlogits_is_e5m2, long long rows, int vocab, long long ld, float A, float B, float C,
                              float grad_mul, void* stream) {
  if (rows == 0) return 0;
  if (vocab % 8 || ld % 8 || n_predict > CE_MAX_PREDICT || n_predict < 1) return -1;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t smem1 = (size_t)vocab * 2, smem2 = (size_t)vocab * 4;
  if (vocab % 16 == 0 && (ld * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(dlogits) & 15) == 0 && smem1 <= 110 * 1024) {
    static int sms = 0;
    if (sms == 0) {
      int dev = 0;
      if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return -5;
      if (cudaFuncSetAttribute(softcap_ce_stream_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 110 * 1024) != cudaSuccess ||
          cudaFuncSetAttribute(softcap_ce_stream_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 110 * 1024) != cudaSuccess)
        return -3;
    }
    const unsigned grid = (unsigned)(rows < 2 * sms ? rows : 2 * sms);
    if (dlogits_is_e5m2)
      softcap_ce_stream_kernel<true><<<grid, CE_STREAM_THREADS, smem1, st>>>((const __nv_bfloat16*)logits, targets, mtp_weights, n_predict,
                                                                prefix_targets, prefix_weight, losses, dlogits, rows, vocab, ld,
                                                                A, B, C, grad_mul);
    else
      softcap_ce_stream_kernel<false><<<grid, CE_STREAM_THREADS, smem1, st>>>((const __nv_bfloat16*)logits, targets, mtp_weights, n_predict,
                                                                 prefix_targets, prefix_weight, losses, dlogits, rows, vocab, ld,
                                                                 A, B, C, grad_mul);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
  }
  const bool cache = smem2 <= 220 * 1024;
  if (!cache && smem1 > 200 * 1024) return -2;
#define CE_LAUNCH(E5, CACHE, TH, SMEM)                                                                              \
  do {                                                                                                              \
    static bool set = false;                                                                                        \
    auto kern = softcap_ce_kernel<E5, CACHE, TH>;                                                                   \
    if (!set) {                                                                                                     \
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024) != cudaSuccess) return -3; \
      set = true;                                                                                                   \
    }                                                                                                               \
    kern<<<(unsigned)rows, TH, SMEM, st>>>((const __nv_bfloat16*)logits, targets, mtp_weights, n_predict, prefix_targets, \
                                           prefix_weight, losses, dlogits, rows, vocab, ld, A, B, C, grad_mul);       \
  } while (0)
  if (dlogits_is_e5m2) {
    if (cache) CE_LAUNCH(true, true, 1024, smem2); else CE_LAUNCH(true, false, 256, smem1);
  } else {
    if (cache) CE_LAUNCH(false, true, 1024, smem2); else CE_LAUNCH(false, false, 256, smem1);
  }
#undef CE_LAUNCH
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
