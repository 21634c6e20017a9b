// Tile epilogue that turns the QKV projection's accumulators straight into attention operands
// (`train_gpt.py:1103-1116` does this with separate ops after the GEMM):
//   q, k:  x = bf16(lam * acc);  n = bf16(x * rstd),  rstd = (mean_d x^2 + eps)^-1/2 over the head's 128 dims;
//          dims 0..63 rotate as interleaved pairs (2i, 2i+1) with the angle of position t (2t + (h & 1) for paired-head
//          layers), dims 64..127 stay; with the partial key offset the stationary half of k is stored one row down
//          (k[t, 64:] <- n[t-1, 64:], row 0 keeps its own), by shifting the bulk store of that box;
//   v:     bf16(lam * acc) + vgate[t, h] * ve[t, h, :].
// The GEMM has N = 3 * H * 128 columns ordered [q heads | k heads | v heads]; an epilogue warp owns 32 rows x 128
// columns = one head of 32 tokens, one token per lane, so the per-head norm needs no cross-thread traffic: the sum of
// squares is formed by a first sweep over the warp's TMEM columns at the start of the tile.  Outputs are three
// contiguous [T, H * 128] tensors (bulk tensor stores), plus rstd_q / rstd_k [T, H] and k_last [H, 64] (the
// stationary half of the last token's key, which the shift pushes out of the tensor) for the backward.
#pragma once
#include "gemm_sm100_pair.cuh"

namespace mng {

struct QkvEpiParams {
  const float* lam;                 // device scalar
  const float* cos_t;               // [positions, 32] fp32
  const float* sin_t;
  const __nv_bfloat16* ve;          // [T, H*128] or null
  const __nv_bfloat16* vgate;       // [T, >= H] (row stride vgate_stride) or null (gate 1)
  int vgate_stride;
  float* rstd_q;                    // [T, H]
  float* rstd_k;
  __nv_bfloat16* k_out;             // [T, H*128]: row 0 of the shifted half is written with plain stores
  __nv_bfloat16* k_last;            // [H, 64]
  int H, paired, key_offset;
};

struct QkvEpiState {
  uint32_t taddr;
  float lam, rstd;
  int which, h;                     // 0 = q, 1 = k, 2 = v; head
  long long pos;
  int cw;
};

constexpr float QKV_HEAD_EPS = 1.1920929e-07f;

struct TEpiQkv {
  static constexpr bool kCin = false, kOut8 = false, kStore16 = true, kTileHooks = true, kCustomStore = true;
  using Params = QkvEpiParams;
  using State = QkvEpiState;
  __device__ static void finish(const Params&, State&) {}

  __device__ static void tile_begin(const Params& p, State& st, int, long long row, int n0, int M, int N) {
    const int HD = p.H * 128;
    st.which = n0 / HD;
    st.h = (n0 - st.which * HD) >> 7;
    st.lam = *p.lam;
    st.pos = p.paired ? 2 * row + (st.h & 1) : row;
    st.cw = 0;
    st.rstd = 1.f;
    if (st.which < 2) {
      float ss = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(st.taddr + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float a = __uint_as_float(v[j]) * st.lam, b = __uint_as_float(v[j + 1]) * st.lam;
          const uint32_t u = pack_bf16x2(a, b);             // the projection's output as a bf16 tensor would hold it
          a = __uint_as_float(u << 16);
          b = __uint_as_float(u & 0xffff0000u);
          ss = fmaf(a, a, fmaf(b, b, ss));
        }
      }
      st.rstd = rsqrtf(ss * (1.f / 128.f) + QKV_HEAD_EPS);
      if (row < M) (st.which == 0 ? p.rstd_q : p.rstd_k)[row * p.H + st.h] = st.rstd;
    }
  }

  __device__ static void apply(const Params& p, State& st, const float (&acc)[32], const uint4 (&)[4], uint4 (&out)[4], uint4 (&)[2],
                               int, long long row, int, int M, int) {
    const int cw = st.cw;                                    // first dim of this chunk within the head: 0, 32, 64, 96
    st.cw += 32;
    float x[32];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const uint32_t u = pack_bf16x2(acc[j] * st.lam, acc[j + 1] * st.lam);
      x[j] = __uint_as_float(u << 16);
      x[j + 1] = __uint_as_float(u & 0xffff0000u);
    }
    const bool live = row < M;
    if (st.which == 2) {
      if (p.ve && live) {
        const float g = p.vgate ? __bfloat162float(p.vgate[row * p.vgate_stride + st.h]) : 1.f;
        const uint4* e = reinterpret_cast<const uint4*>(p.ve + (row * p.H + st.h) * 128 + cw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 u = e[q];
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float2 f = __bfloat1622float2(h2[t]);
            x[q * 8 + 2 * t] = fmaf(g, f.x, x[q * 8 + 2 * t]);
            x[q * 8 + 2 * t + 1] = fmaf(g, f.y, x[q * 8 + 2 * t + 1]);
          }
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {                      // normalised values, rounded like the separate norm op
        const uint32_t u = pack_bf16x2(x[j] * st.rstd, x[j + 1] * st.rstd);
        x[j] = __uint_as_float(u << 16);
        x[j + 1] = __uint_as_float(u & 0xffff0000u);
      }
      if (cw < 64) {                                         // rotary pairs cw/2 .. cw/2 + 15
        const float4* cs = reinterpret_cast<const float4*>(p.cos_t + st.pos * 32 + (cw >> 1));
        const float4* sn = reinterpret_cast<const float4*>(p.sin_t + st.pos * 32 + (cw >> 1));
        if (live) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 c4 = cs[q], s4 = sn[q];
            const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const float a = x[q * 8 + 2 * t], b = x[q * 8 + 2 * t + 1];
              x[q * 8 + 2 * t] = fmaf(cc[t], a, ss[t] * b);
              x[q * 8 + 2 * t + 1] = fmaf(cc[t], b, -ss[t] * a);
            }
          }
        }
      } else if (st.which == 1 && p.key_offset && live) {
        // the shifted store leaves out row 0 (keeps its own values) and drops the last row's (kept for the backward)
        if (row == 0 || row == M - 1) {
          __nv_bfloat16* dst = row == 0 ? p.k_out + st.h * 128 + cw : p.k_last + st.h * 64 + (cw - 64);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(x[q * 8], x[q * 8 + 1]); w.y = pack_bf16x2(x[q * 8 + 2], x[q * 8 + 3]);
            w.z = pack_bf16x2(x[q * 8 + 4], x[q * 8 + 5]); w.w = pack_bf16x2(x[q * 8 + 6], x[q * 8 + 7]);
            reinterpret_cast<uint4*>(dst)[q] = w;
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      out[q].x = pack_bf16x2(x[q * 8], x[q * 8 + 1]); out[q].y = pack_bf16x2(x[q * 8 + 2], x[q * 8 + 3]);
      out[q].z = pack_bf16x2(x[q * 8 + 4], x[q * 8 + 5]); out[q].w = pack_bf16x2(x[q * 8 + 6], x[q * 8 + 7]);
    }
  }

  __device__ static void tile_end(const Params&, State&, int, long long, int, int, int) {}

  // lane 0: the warp's two staged boxes (dims 0..63 and 64..127 of one head, 32 tokens) to q, k or v
  __device__ static void issue_stores(const Params& p, const PairMaps& maps, uint8_t* stg, int b, int m0, int n0, int M, int N) {
    if (n0 >= N) return;
    const int HD = p.H * 128;
    const int which = n0 / HD;
    const int col = n0 - which * HD;
    const CUtensorMap* m = which == 0 ? &maps.out : (which == 1 ? &maps.out2 : &maps.out3);
    tma_store_3d(m, stg, col, m0, b);
    const int shift = (which == 1 && p.key_offset) ? 1 : 0;
    tma_store_3d(m, stg + 4096, col + 64, m0 + shift, b);
  }
};

}  // namespace mng
