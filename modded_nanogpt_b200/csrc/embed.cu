// Embedding backward that accumulates straight into the (persistent) bf16 gradient table.
//
// Input: token rows sorted by table row (sorted_ids, perm), upstream gradient g [n, D].  The sorted
// list is cut into chunks of EMB_CHUNK entries, one CTA each; a CTA walks its chunk, sums runs of equal
// ids in fp32 registers and flushes each run once.  A run that lies wholly inside the chunk has a single
// writer and is added with a plain read-modify-write; a run that continues into a neighbouring chunk
// (a frequent token) is added with bf16x2 atomics, one per chunk and element.  No dense [V, D] temporary,
// no zero fill, no separate accumulate pass (the reference goes through ATen's dense embedding backward
// and autograd's accumulate for `embed`, `value_embeds` and `bigram_embed`, `train_gpt.py:1531-1541`).
#include "api.h"
#include "ptx.cuh"

namespace mng {

constexpr int EMB_CHUNK = 128;

__device__ __forceinline__ void emb_flush(__nv_bfloat16* dst, const float (&acc)[8], bool atomic) {
  if (atomic) {
    __nv_bfloat162* d2 = reinterpret_cast<__nv_bfloat162*>(dst);
#pragma unroll
    for (int t = 0; t < 4; ++t) atomicAdd(d2 + t, __floats2bfloat162_rn(acc[2 * t], acc[2 * t + 1]));
  } else {
    uint4 u = *reinterpret_cast<const uint4*>(dst);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    uint4 w;
    uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float2 f = __bfloat1622float2(h[t]);
      wp[t] = pack_bf16x2(f.x + acc[2 * t], f.y + acc[2 * t + 1]);
    }
    *reinterpret_cast<uint4*>(dst) = w;
  }
}

// blockDim.x = D / 8 (each thread owns 8 consecutive columns)
__global__ void embed_bwd_kernel(const __nv_bfloat16* __restrict__ g, const long long* __restrict__ sorted_ids,
                                 const long long* __restrict__ perm, __nv_bfloat16* __restrict__ grad, long long n, int D,
                                 long long table_rows) {
  const long long begin = (long long)blockIdx.x * EMB_CHUNK;
  const long long end = begin + EMB_CHUNK < n ? begin + EMB_CHUNK : n;
  const int col = threadIdx.x * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  long long cur = sorted_ids[begin];
  bool open_left = begin > 0 && sorted_ids[begin - 1] == cur;       // the run started in an earlier chunk
  for (long long j = begin; j < end; j += 4) {
    long long id[4], src[4];
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long jj = j + u < end ? j + u : end - 1;
      id[u] = sorted_ids[jj];
      src[u] = perm[jj];
      if (!MNG_IN_RANGE(src[u], n)) src[u] = 0;               // debug build only: a bad permutation entry reads row 0
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const uint4*>(g + src[u] * D + col);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j + u >= end) break;
      if (id[u] != cur) {
        if (MNG_IN_RANGE(cur, table_rows)) emb_flush(grad + cur * D + col, acc, open_left);
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[t] = 0.f;
        cur = id[u];
        open_left = false;
      }
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float2 f = __bfloat1622float2(h[t]);
        acc[2 * t] += f.x; acc[2 * t + 1] += f.y;
      }
    }
  }
  const bool open_right = end < n && sorted_ids[end] == cur;
  if (MNG_IN_RANGE(cur, table_rows)) emb_flush(grad + cur * D + col, acc, open_left || open_right);
}

}  // namespace mng

MNG_DEFINE_BOUNDS_QUERY(embed)

extern "C" int mng_embed_bwd(const void* g, const long long* sorted_ids, const long long* perm, void* grad, long long n, int D,
                             long long table_rows, void* stream) {
  if (n == 0) return 0;
  if (D % 8 || D / 8 > 1024) return -1;
  const unsigned grid = (unsigned)((n + mng::EMB_CHUNK - 1) / mng::EMB_CHUNK);
  mng::embed_bwd_kernel<<<grid, D / 8, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)g, sorted_ids, perm,
                                                                   (__nv_bfloat16*)grad, n, D, table_rows);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
