// Tile epilogues that fuse the soft-capped cross entropy into the FP8 lm_head GEMM (CTA-pair kernel), so that the
// [tokens, vocab] logits never exist in memory (`triton_kernels.py:1208-1292` materialises them in bf16 and runs a
// separate loss kernel over them):
//
//   pass 1  TEpiCeStats   logits tile -> z = A * sigmoid((logit + B) / C) -> per row and per 128-column slab the sum of
//                         exp(z - A) (z is bounded by A, so no running maximum is needed), plus z at the row's target
//                         columns.  Stores nothing tile-sized.
//   (ce_finish_kernel: slab sums -> lse, loss, S_w / sum per row)
//   pass 2  TEpiCeGrad    the same GEMM again; the epilogue turns the accumulators straight into
//                         dlogit = g * (S_w * softmax(z) - [targets]) * s (1 - s) in e5m2 (bulk tensor stores).
//
// Per-row state lives in registers across the four 32-column chunks a warp owns (tile hooks of the pair kernel).
// A target column that falls into the warp's slab is handled at the start of the tile by re-reading that single
// accumulator column from TMEM (warp-uniform tcgen05.ld of one column; the lane that owns the row keeps its value):
// no per-element compares in the chunk loops.  Both epilogues are bound by the special-function unit (one tanh and
// one exponential per logit), so three of four exponentials are evaluated by a polynomial on the FMA pipe.
#pragma once
#include "gemm_sm100_pair.cuh"

namespace mng {

constexpr int CE_FUSED_TARGETS = 4;        // up to 3 multi-token-prediction targets + the prefix target

struct CeEpiParams {
  const long long* targets;                // [rows]
  const long long* prefix_targets;         // [rows] or null
  const float* mtp_w;                      // [n_predict]
  const float* prefix_w;                   // [1] or null
  int n_predict;
  float alpha;                             // dequantisation: logit = acc * alpha
  float A, half_inv_c, half_b_over_c;      // sigmoid(u) = 0.5 + 0.5 tanh(u / 2), u = (logit + B) / C
  float k2;                                // A * log2(e): exp(A s - A) = exp2(k2 s - k2)
  float* slab_sum;                         // pass 1: [rows, slabs]
  int slabs;
  float* ztgt;                             // pass 1: [rows, 4]
  const float* rowc;                       // pass 2: [rows]  S_w / sum
  float gscale;                            // pass 2: grad_mul * A / C
};

struct CeEpiState {
  uint32_t taddr;                          // TMEM address of the warp's 128-column slab (set by the kernel)
  long long cached_row;                    // row whose targets t[], w[] hold (-1 = none): tiles of one row block follow
  long long t[CE_FUSED_TARGETS];           // each other along N, so the target loads are skipped most of the time
  float w[CE_FUSED_TARGETS];
  int d[CE_FUSED_TARGETS];                 // target column - first column of the slab (huge negative = not in this slab)
  float hitacc[CE_FUSED_TARGETS];          // accumulator value at that column
  float hitw[CE_FUSED_TARGETS];            // pass 2: weight landing on that column
  float sum, rowc;
  int cw;                                  // columns of the slab already consumed
  __device__ CeEpiState() : cached_row(-1) {}
};

__device__ __forceinline__ float ce_sigmoid_half(float acc, const CeEpiParams& p) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(fmaf(acc, p.alpha * p.half_inv_c, p.half_b_over_c)));
  return fmaf(0.5f, t, 0.5f);
}
// Two sigmoids with one special-function instruction: tanh.approx on a bf16 pair.  bf16 precision is what the
// reference keeps of the sigmoid (it stores it as bf16 before forming z, `triton_kernels.py:1003-1009`).
__device__ __forceinline__ void ce_sigmoid2(float a0, float a1, const CeEpiParams& p, float& s0, float& s1) {
  const float c = p.alpha * p.half_inv_c;
  const uint32_t u = pack_bf16x2(fmaf(a0, c, p.half_b_over_c), fmaf(a1, c, p.half_b_over_c));
  uint32_t t;
  asm("tanh.approx.bf16x2 %0, %1;" : "=r"(t) : "r"(u));
  s0 = fmaf(0.5f, __uint_as_float(t << 16), 0.5f);
  s1 = fmaf(0.5f, __uint_as_float(t & 0xffff0000u), 0.5f);
}
__device__ __forceinline__ float ce_exp2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// The epilogues send every other exponential to the polynomial: that balances the two pipes (8 issue slots of the FMA
// pipe cost what one special-function instruction costs in its unit).


// value of accumulator column `col` (0..127 within the slab) of this lane's row, for every lane that asks; warp collective
__device__ __forceinline__ float ce_reload(const CeEpiState& st, bool hit, int col) {
  float mine = 0.f;
  unsigned m = __ballot_sync(0xffffffffu, hit);
  const int lane = threadIdx.x & 31;
  while (m) {
    const int src = __ffs(m) - 1;
    m &= m - 1;
    const int c = __shfl_sync(0xffffffffu, col, src);
    const uint32_t v = tmem_ld1(st.taddr + c);
    tmem_ld_wait();
    if (lane == src) mine = __uint_as_float(v);
  }
  return mine;
}

__device__ __forceinline__ void ce_tile_begin(const CeEpiParams& p, CeEpiState& st, long long row, int n0, int M, int N, bool grad) {
  if (st.cached_row != row) {
    st.cached_row = row;
#pragma unroll
    for (int k = 0; k < CE_FUSED_TARGETS - 1; ++k) {
      st.t[k] = -1;
      st.w[k] = 0.f;
      if (k < p.n_predict && row + k < M) {
        st.t[k] = p.targets[row + k];
        st.w[k] = p.mtp_w[k];
      }
    }
    st.t[3] = (p.prefix_targets && row < M) ? p.prefix_targets[row] : -1;
    st.w[3] = p.prefix_w ? p.prefix_w[0] : 0.f;
    if (grad) {
      st.rowc = row < M ? p.rowc[row] : 0.f;
#pragma unroll
      for (int k = 0; k < CE_FUSED_TARGETS; ++k) {
        float h = 0.f;
#pragma unroll
        for (int j = 0; j < CE_FUSED_TARGETS; ++j)
          if (st.t[j] == st.t[k] && st.t[j] >= 0 && st.t[j] < N) h += st.w[j];
        st.hitw[k] = h;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < CE_FUSED_TARGETS; ++k) {
    const bool valid = st.t[k] >= 0 && st.t[k] < N && row < M;
    const long long dd = st.t[k] - n0;
    const bool hit = valid && dd >= 0 && dd < 128;
    st.d[k] = hit ? (int)dd : -(1 << 30);
    if (__any_sync(0xffffffffu, hit)) st.hitacc[k] = ce_reload(st, hit, (int)dd);
  }
  st.sum = 0.f;
  st.cw = 0;
}

struct TEpiCeStats {
  static constexpr bool kCin = false, kOut8 = false, kStore16 = false, kTileHooks = true;
  using Params = CeEpiParams;
  using State = CeEpiState;
  __device__ static void finish(const Params&, State&) {}
  __device__ static void tile_begin(const Params& p, State& st, int, long long row, int n0, int M, int N) {
    ce_tile_begin(p, st, row, n0, M, N, false);
#pragma unroll
    for (int k = 0; k < CE_FUSED_TARGETS; ++k)
      if (st.d[k] >= 0) p.ztgt[row * CE_FUSED_TARGETS + k] = p.A * ce_sigmoid_half(st.hitacc[k], p);
  }
  __device__ static void apply(const Params& p, State& st, const float (&acc)[32], const uint4 (&)[4], uint4 (&)[4], uint4 (&)[2],
                               int, long long, int col0, int, int N) {
    if (col0 >= N) return;                                   // N is a multiple of 32: the chunk is inside or outside
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      float a, b;
      ce_sigmoid2(acc[j], acc[j + 1], p, a, b);
      s0 += ce_exp2(fmaf(p.k2, a, -p.k2));
      s1 += exp2_fma(fmaf(p.k2, b, -p.k2));
    }
    st.sum += s0 + s1;
  }
  __device__ static void tile_end(const Params& p, State& st, int, long long row, int n0, int M, int N) {
    if (row < M && n0 < N) p.slab_sum[row * p.slabs + (n0 >> 7)] = st.sum;
  }
};

struct TEpiCeGrad {
  static constexpr bool kCin = false, kOut8 = true, kStore16 = false, kTileHooks = true;
  using Params = CeEpiParams;
  using State = CeEpiState;
  __device__ static void finish(const Params&, State&) {}
  __device__ static void tile_begin(const Params& p, State& st, int, long long row, int n0, int M, int N) {
    ce_tile_begin(p, st, row, n0, M, N, true);
  }
  // two neighbouring columns -> e5m2 pair
  __device__ static uint32_t grad2(const Params& p, float c, float a0, float a1) {
    float s0, s1;
    ce_sigmoid2(a0, a1, p, s0, s1);
    const float e0 = ce_exp2(fmaf(p.k2, s0, -p.k2)), e1 = exp2_fma(fmaf(p.k2, s1, -p.k2));
    return (uint32_t)pack_e5m2x2(c * e0 * fmaf(-s0, s0, s0), c * e1 * fmaf(-s1, s1, s1));
  }
  __device__ static void apply(const Params& p, State& st, const float (&acc)[32], const uint4 (&)[4], uint4 (&)[4], uint4 (&out8)[2],
                               int, long long, int col0, int, int N) {
    const int cw = st.cw;
    st.cw += 32;
    uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0, w4 = 0, w5 = 0, w6 = 0, w7 = 0;
    if (col0 < N) {
      const float c = p.gscale * st.rowc;
#define MNG_CE_WORD(T) (grad2(p, c, acc[4 * T], acc[4 * T + 1]) | (grad2(p, c, acc[4 * T + 2], acc[4 * T + 3]) << 16))
      w0 = MNG_CE_WORD(0); w1 = MNG_CE_WORD(1); w2 = MNG_CE_WORD(2); w3 = MNG_CE_WORD(3);
      w4 = MNG_CE_WORD(4); w5 = MNG_CE_WORD(5); w6 = MNG_CE_WORD(6); w7 = MNG_CE_WORD(7);
#undef MNG_CE_WORD
#pragma unroll
      for (int k = 0; k < CE_FUSED_TARGETS; ++k) {
        const int dd = st.d[k] - cw;
        if (dd >= 0 && dd < 32) {                            // a target column of this row: exact formula with the hit weight
          const float sg = ce_sigmoid_half(st.hitacc[k], p);
          const float e = ce_exp2(fmaf(p.k2, sg, -p.k2));
          const float g = p.gscale * (st.rowc * e - st.hitw[k]) * sg * (1.f - sg);
          const uint32_t byte = (uint32_t)pack_e5m2x2(g, 0.f) & 0xffu;
          const int sh = (dd & 3) * 8, wi = dd >> 2;
          const uint32_t keep = ~(0xffu << sh), put = byte << sh;
          if (wi == 0) w0 = (w0 & keep) | put;
          if (wi == 1) w1 = (w1 & keep) | put;
          if (wi == 2) w2 = (w2 & keep) | put;
          if (wi == 3) w3 = (w3 & keep) | put;
          if (wi == 4) w4 = (w4 & keep) | put;
          if (wi == 5) w5 = (w5 & keep) | put;
          if (wi == 6) w6 = (w6 & keep) | put;
          if (wi == 7) w7 = (w7 & keep) | put;
        }
      }
    }
    out8[0] = make_uint4(w0, w1, w2, w3);
    out8[1] = make_uint4(w4, w5, w6, w7);
  }
  __device__ static void tile_end(const Params&, State&, int, long long, int, int, int) {}
};

// Per row: sum of the slab sums -> lse = A + log(sum); loss as in csrc/ce.cu; rowc = S_w / sum.  One warp per row.
__global__ void __launch_bounds__(256)
ce_finish_kernel(CeEpiParams p, float* __restrict__ losses, float* __restrict__ rowc, long long rows, int vocab) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  float s = 0.f;
  for (int i = lane; i < p.slabs; i += 32) s += p.slab_sum[row * p.slabs + i];
  s = warp_sum(s);
  if (lane == 0) {
    const float lse = p.A + __logf(s);
    const float pw = p.prefix_w ? p.prefix_w[0] : 0.f;
    const long long pt = p.prefix_targets ? p.prefix_targets[row] : -1;
    const bool pvalid = pt >= 0 && pt < vocab;
    float S_w = pvalid ? pw : 0.f, loss = 0.f;
    for (int k = 0; k < p.n_predict; ++k) {
      S_w += p.mtp_w[k];
      if (row + k < rows) {
        const long long t = p.targets[row + k];
        if (t >= 0 && t < vocab) loss += p.mtp_w[k] * (lse - p.ztgt[row * CE_FUSED_TARGETS + k]);
      }
    }
    if (pvalid) loss += pw * (lse - p.ztgt[row * CE_FUSED_TARGETS + 3]);
    losses[row] = loss;
    rowc[row] = S_w / s;
  }
}

}  // namespace mng
