// Causal, document-masked sliding-window attention forward for sm_100a (head dim 128, bf16).
//
//   o[i,h,:] = softmax_j( scale * q[i,h,:].k[j,h,:] ) v[j,h,:]   over keys j of i's document with i-window <= j <= i
//   lse[h,i] = log sum_j exp(scale * q.k)                         (natural log; what a flash-attention backward expects)
//
// Same contract as the reference's `flash_attn_varlen_func(..., causal=True, window_size=(W, 0))` call
// (`train_gpt.py:1139-1141`) on one packed sequence; documents are given as `doc_start[i]` = index of the
// first token of the document that holds token i.
//
// One work item = 128 queries of one head.  CTAs of 192 threads, two per SM (96 KB of shared memory and 256 TMEM
// columns each), so that one CTA's softmax overlaps the other's MMAs; a CTA claims item after item from a device counter:
//   warp 0    TMA producer: claims the items, Q tile once per item, then K and V tiles of 128 keys (single buffers,
//             refilled as soon as the MMA that read them has completed);
//   warp 1    tcgen05 issuer: S = Q K^T (both operands K-major from shared memory) into TMEM columns [0,128);
//             O += P V with P read from TMEM (bf16, aliasing S) and V MN-major from shared memory, into [128,256);
//   warps 2-5 softmax: thread = query row.  Two passes over the S tile in TMEM (row maximum, then
//             exponentials): p = exp2(s*c - m), bf16 P written back over S, row sums in fp32.  The running
//             maximum only moves when it grows by more than 8 (factor 256), so the O accumulator is rescaled
//             rarely; the final division by the row sum makes the result exact either way.
// Key blocks run from max(doc_start[q0], q0 - window) to the tile's last query: blocks before the window or
// the document never load.  Every mbarrier wait is bounded.
#include "api.h"
#include "ptx.cuh"

#include <cstdlib>
#include <mutex>
#include <string>

// All soft-max exponentials stay on the special-function unit: moving every other one to the FMA pipe (exp2_fma in
// ptx.cuh) measured 19 % slower in the forward and 5 % slower in the backward on B200 - these kernels are bound by the
// latency of their S -> P -> PV chains, not by the throughput of that unit.

namespace mng {

constexpr int ATT_THREADS = 192;
constexpr int ATT_TILE_BYTES = 128 * 128 * 2;     // 128 rows x 128 dims bf16 = two 16 KB boxes
constexpr int ATT_SMEM = 3 * ATT_TILE_BYTES + 1024 /*barriers*/ + 1024 /*alignment*/;

struct AttnParams {
  const int* doc_start;
  __nv_bfloat16* out;
  float* lse;
  int T, H, window;
  float scale_log2;       // softmax scale * log2(e)
  int* work;              // items beyond the first of each CTA are claimed here; null = static stride of gridDim.x
};

// Work counter of the forward kernel (items beyond the first of each CTA are claimed from it); zeroed by a memset that
// precedes the launch on the stream.  One per device: forward calls on different streams of one device must not overlap.
static __device__ int g_atf_work[1];

// Persistent: two CTAs per SM; a CTA starts on item blockIdx.x and claims further items (item = (128-query tile, head),
// heads fastest, long-history tiles first) from a device counter, so that packed documents of different lengths balance
// out.  TMEM, the barriers and the K/V buffers live across items and every barrier phase runs on counters that continue
// across items: the next item's Q / K / V loads and its first score MMAs overlap the drain of the previous item's
// accumulator (per-tile fixed cost of the one-CTA-per-tile launch: 7.9 us of a ~17 us tile at the training shapes).
// The producer publishes each item number in a two-slot ring in shared memory before it signals q_full; -1 ends the walk.
__global__ void __launch_bounds__(ATT_THREADS, 2)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, AttnParams p, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + ATT_TILE_BYTES;
  uint8_t* sV = smem + 2 * ATT_TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 3 * ATT_TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 2;
  uint64_t* v_full = bars + 3;
  uint64_t* v_empty = bars + 4;
  uint64_t* s_full = bars + 5;
  uint64_t* p_ready = bars + 6;
  uint64_t* o_done = bars + 7;
  uint64_t* q_empty = bars + 8;      // the item's score MMAs have read Q: the producer may load the next item's
  uint64_t* o_free = bars + 9;       // the four soft-max warps have drained O: the next item's PV MMAs may overwrite it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  volatile int* item_ring = reinterpret_cast<volatile int*>(tmem_slot + 2);   // [2]: item of the it-th step of this CTA

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (p.T + 127) / 128;
  const int items = tiles * p.H;
  // query tile start, head, first key and number of 128-key blocks of an item
  auto item_geom = [&](int item, int& h, int& q0, int& kv_lo, int& nb) {
    const int tile = item / p.H;
    h = item - tile * p.H;
    q0 = (tiles - 1 - tile) * 128;                           // late (long-history) tiles first
    const int q_last = min(q0 + 127, p.T - 1);
    kv_lo = max(p.doc_start[q0], q0 - p.window);
    nb = (q_last - kv_lo) / 128 + 1;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(k_full, 1);
    mbar_init(k_empty, 1);
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_ready, 4);
    mbar_init(o_done, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_free, 4);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_S = *tmem_slot;
  const uint32_t tmem_O = tmem_S + 128;
#define ATT_FAIL(code)                                                          \
  do {                                                                          \
    if (*abort_flag == 0) { *abort_flag = (code); atomicCAS(status, 0u, (code)); } \
  } while (0)

  if (warp == 0) {
    if (lane == 0) {
      uint32_t jt = 0, it = 0;                               // blocks / items issued so far by this CTA
      int item = blockIdx.x;
      bool ok = true;
      while (ok) {
        // Q buffer and ring slot it & 1 are free once the score MMAs of the item before have completed
        if (!mbar_wait(q_empty, (it & 1) ^ 1, abort_flag)) { ATT_FAIL(ERR_WAIT_SMEM_EMPTY); break; }
        if (item >= items) {
          item_ring[it & 1] = -1;
          mbar_arrive(q_full);                               // no copy: a plain arrive completes the phase
          break;
        }
        item_ring[it & 1] = item;
        int h, q0, kv_lo, nb;
        item_geom(item, h, q0, kv_lo, nb);
        mbar_expect_tx(q_full, ATT_TILE_BYTES);
        tma_load_3d(sQ, &tq, q_full, 0, h, q0);
        tma_load_3d(sQ + 16384, &tq, q_full, 64, h, q0);
        for (int j = 0; j < nb; ++j, ++jt) {
          const int kb = kv_lo + j * 128;
          if (!mbar_wait(k_empty, (jt & 1) ^ 1, abort_flag)) { ATT_FAIL(ERR_WAIT_SMEM_EMPTY); ok = false; break; }
          mbar_expect_tx(k_full, ATT_TILE_BYTES);
          tma_load_3d(sK, &tk, k_full, 0, h, kb);
          tma_load_3d(sK + 16384, &tk, k_full, 64, h, kb);
          if (!mbar_wait(v_empty, (jt & 1) ^ 1, abort_flag)) { ATT_FAIL(ERR_WAIT_SMEM_EMPTY); ok = false; break; }
          mbar_expect_tx(v_full, ATT_TILE_BYTES);
          tma_load_3d(sV, &tv, v_full, 0, h, kb);
          tma_load_3d(sV + 16384, &tv, v_full, 64, h, kb);
        }
        item = p.work ? (int)gridDim.x + atomicAdd(p.work, 1) : item + (int)gridDim.x;
        ++it;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC_S = make_idesc(1, 1, 0, 0, 128, 128);
      constexpr uint32_t IDESC_PV = make_idesc(1, 1, 0, 1, 128, 128);
      // descriptors differ only in the 14-bit start-address field (address >> 4): build once, then add offsets
      const uint64_t dQ = make_smem_desc(smem_u32(sQ), 16, 1024), dK = make_smem_desc(smem_u32(sK), 16, 1024);
      const uint64_t dV = make_smem_desc(smem_u32(sV), 16384, 1024);
      uint32_t jt = 0;
      bool ok = true;
      for (uint32_t it = 0; ok; ++it) {
        if (!mbar_wait(q_full, it & 1, abort_flag)) { ATT_FAIL(ERR_WAIT_TMA_FULL); break; }
        const int item = item_ring[it & 1];
        if (item < 0) {
          mbar_arrive(s_full);                               // wakes the soft-max warps, which then read the end mark
          break;
        }
        int h, q0, kv_lo, nb;
        item_geom(item, h, q0, kv_lo, nb);
        for (int j = 0; j < nb; ++j, ++jt) {
          if (!mbar_wait(k_full, jt & 1, abort_flag)) { ATT_FAIL(ERR_WAIT_TMA_FULL); ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t off = ((k >> 2) * 16384 + (k & 3) * 32) >> 4;
            umma_f16(tmem_S, dQ + off, dK + off, IDESC_S, k != 0);
          }
          umma_commit(k_empty);
          if (j == nb - 1) umma_commit(q_empty);             // last reader of this item's Q
          umma_commit(s_full);
          if (!mbar_wait(p_ready, jt & 1, abort_flag)) { ATT_FAIL(ERR_WAIT_TMEM_EMPTY); ok = false; break; }
          if (!mbar_wait(v_full, jt & 1, abort_flag)) { ATT_FAIL(ERR_WAIT_TMA_FULL); ok = false; break; }
          if (j == 0 && !mbar_wait(o_free, (it & 1) ^ 1, abort_flag)) { ATT_FAIL(ERR_WAIT_TMEM_EMPTY); ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 8; ++k)                        // 16 keys per MMA: 8 TMEM columns of packed bf16
            umma_f16_ts(tmem_O, tmem_S + k * 8, dV + ((k * 2048) >> 4), IDESC_PV, (j | k) != 0);
          umma_commit(v_empty);
          umma_commit(o_done);
        }
      }
    }
  } else {
    const int sub = warp & 3;                                // TMEM sub-partition of this warp
    const int r = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const float c = p.scale_log2;
    uint32_t jt = 0;
    bool alive = true;
    for (uint32_t it = 0; alive; ++it) {
      // The first score tile of the step (or the issuing thread's end signal) also tells that the ring slot is written.
      // s_full runs at most one phase ahead of these warps (the next score MMA needs their p_ready); q_full can run two
      // phases ahead of them when an item has a single block, so it cannot be waited on here.
      if (!mbar_wait(s_full, jt & 1, abort_flag)) { ATT_FAIL(ERR_WAIT_TMEM_FULL); break; }
      const int item = item_ring[it & 1];
      if (item < 0) break;
      int h, q0, kv_lo, nb;
      item_geom(item, h, q0, kv_lo, nb);
      const int i = q0 + r;
      const bool row_ok = i < p.T;
      const int lo_i = row_ok ? max(p.doc_start[i], i - p.window) : 0;
      const int hi_i = row_ok ? i : -1;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nb; ++j, ++jt) {
        const int kb = kv_lo + j * 128;
        if (j > 0 && !mbar_wait(s_full, jt & 1, abort_flag)) { ATT_FAIL(ERR_WAIT_TMEM_FULL); alive = false; break; }
        tc_fence_after();
        const bool full = kb >= lo_i && kb + 127 <= hi_i;    // no masking needed for this row in this block
        const unsigned span = (unsigned)(hi_i - lo_i);
        const bool any_vis = hi_i >= lo_i;
        // the whole 128-column row of S in registers: four loads in flight, one wait
        uint32_t v0[32], v1[32], v2[32], v3[32];
        tmem_ld32(tmem_S + lane_off, v0);
        tmem_ld32(tmem_S + lane_off + 32, v1);
        tmem_ld32(tmem_S + lane_off + 64, v2);
        tmem_ld32(tmem_S + lane_off + 96, v3);
        tmem_ld_wait();
        float mx = -INFINITY;
        if (full) {
#pragma unroll
          for (int t = 0; t < 32; ++t)
            mx = fmaxf(mx, fmaxf(fmaxf(__uint_as_float(v0[t]), __uint_as_float(v1[t])), fmaxf(__uint_as_float(v2[t]), __uint_as_float(v3[t]))));
        } else {
          const int col0 = kb - lo_i;
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            if (!((unsigned)(col0 + t) <= span && any_vis)) v0[t] = 0xff800000u;          // -inf: exp2 gives exactly 0
            if (!((unsigned)(col0 + 32 + t) <= span && any_vis)) v1[t] = 0xff800000u;
            if (!((unsigned)(col0 + 64 + t) <= span && any_vis)) v2[t] = 0xff800000u;
            if (!((unsigned)(col0 + 96 + t) <= span && any_vis)) v3[t] = 0xff800000u;
            mx = fmaxf(mx, fmaxf(fmaxf(__uint_as_float(v0[t]), __uint_as_float(v1[t])), fmaxf(__uint_as_float(v2[t]), __uint_as_float(v3[t]))));
          }
        }
        mx *= c;
        float alpha = 1.f;
        if (mx > m_used + 8.f || (m_used == -INFINITY && mx > -INFINITY)) {
          alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - mx);
          m_used = mx;
          l *= alpha;
        }
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {  // rescale the accumulator rows of this warp
          if (!mbar_wait(o_done, (jt - 1) & 1, abort_flag)) { ATT_FAIL(ERR_WAIT_TMEM_FULL); alive = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t v[32];
            tmem_ld32(tmem_O + lane_off + cc * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 32; ++t) v[t] = __float_as_uint(__uint_as_float(v[t]) * alpha);
            tmem_st32(tmem_O + lane_off + cc * 32, v);
          }
        }
        // rows that have seen no key yet keep m_used = -inf: use 0 so that exp2(-inf - 0) = 0 and not NaN
        const float mneg = (m_used == -INFINITY) ? 0.f : -m_used;
        auto emit = [&](const uint32_t (&vv)[32], int cc) {
          uint32_t pk[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const float p0 = exp2f(fmaf(__uint_as_float(vv[2 * t]), c, mneg));
            const float p1 = exp2f(fmaf(__uint_as_float(vv[2 * t + 1]), c, mneg));
            l += p0 + p1;
            pk[t] = pack_bf16x2(p0, p1);
          }
          tmem_st16(tmem_S + lane_off + cc * 16, pk);
        };
        emit(v0, 0);
        emit(v1, 1);
        emit(v2, 2);
        emit(v3, 3);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_ready);
      }
      if (!alive) break;
      if (!mbar_wait(o_done, (jt - 1) & 1, abort_flag)) { ATT_FAIL(ERR_WAIT_TMEM_FULL); break; }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.out + ((size_t)i * p.H + h) * 128;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t v[32];
        tmem_ld32(tmem_O + lane_off + cc * 32, v);
        tmem_ld_wait();
        if (cc == 3) {                                       // this warp's rows of O are in registers: release the accumulator
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(o_free);
        }
        if (row_ok) {
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[8 * t]) * inv, __uint_as_float(v[8 * t + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[8 * t + 2]) * inv, __uint_as_float(v[8 * t + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[8 * t + 4]) * inv, __uint_as_float(v[8 * t + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[8 * t + 6]) * inv, __uint_as_float(v[8 * t + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + cc * 32 + t * 8) = w;
          }
        }
      }
      if (row_ok) p.lse[(size_t)h * p.T + i] = (m_used + log2f(l)) * 0.6931471805599453f;
    }
  }
#undef ATT_FAIL

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (*abort_flag != 0) {
      const long long t0 = clock64();
      while (clock64() - t0 < 2000000LL) { __nanosleep(1000); }
    }
    tc_fence_after();
    tmem_dealloc(tmem_S, 256);
  }
}

// ---- host ---------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn attn_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [T, H, 128] bf16 (token stride `row_stride` elements) as {d, head, token} with boxes of 64 dims x 1 head x box_rows tokens
static int attn_map(CUtensorMap* m, const void* ptr, int T, int H, long long row_stride, int box_rows = 128) {
  EncodeTiledFn enc = attn_encode();
  if (!enc) return -1;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (row_stride * 2) % 16) return -2;
  cuuint64_t dims[3] = {128, (cuuint64_t)H, (cuuint64_t)T};
  cuuint64_t strides[2] = {256, (cuuint64_t)row_stride * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -100 - (int)r;
}

}  // namespace mng

using namespace mng;

extern "C" int mng_attn_fwd(const void* q, const void* k, const void* v, const int* doc_start, void* out, float* lse, int T,
                            int H, long long row_stride, int window, float scale, void* stream, uint32_t* status) {
  if (T <= 0 || H <= 0) return 0;
  static thread_local bool ctx_bound = false;
  if (!ctx_bound) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaSetDevice(dev);
    cudaFree(nullptr);
    ctx_bound = true;
  }
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = attn_map(&tq, q, T, H, row_stride))) return rc;
  if ((rc = attn_map(&tk, k, T, H, row_stride))) return rc - 1000;
  if ((rc = attn_map(&tv, v, T, H, row_stride))) return rc - 2000;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM) != cudaSuccess) return -3;
    attr = true;
  }
  // the work counter is a __device__ symbol: its address and the SM count belong to the current device
  constexpr int kMaxDevices = 64;
  static int* work_of[kMaxDevices] = {};
  static int sms_of[kMaxDevices] = {};
  static std::mutex mu;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -6;
  int* work = nullptr;
  int sms = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!work_of[dev]) {
      if (cudaGetSymbolAddress(reinterpret_cast<void**>(&work_of[dev]), g_atf_work) != cudaSuccess ||
          cudaDeviceGetAttribute(&sms_of[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        work_of[dev] = nullptr;
        return -6;
      }
    }
    work = work_of[dev];
    sms = sms_of[dev];
  }
  // MNG_ATTN_FWD=tile: one CTA per (tile, head) item (same kernel, no claims)
  static const bool per_item = [] { const char* e = getenv("MNG_ATTN_FWD"); return e && std::string(e) == "tile"; }();
  const int items = ((T + 127) / 128) * H;
  const int resident = 2 * sms;                              // two CTAs per SM (shared memory and TMEM columns)
  const bool claim = !per_item && items > resident;
  if (claim && cudaMemsetAsync(work, 0, sizeof(int), (cudaStream_t)stream) != cudaSuccess) return -5;
  AttnParams p{doc_start, reinterpret_cast<__nv_bfloat16*>(out), lse, T, H, window, scale * 1.4426950408889634f,
               claim ? work : nullptr};
  dim3 grid(claim ? resident : items);
  attn_fwd_kernel<<<grid, ATT_THREADS, ATT_SMEM, (cudaStream_t)stream>>>(tq, tk, tv, p, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

// =====================================================================================================
// Backward.  Two launches of one templated kernel, both with the forward's structure (owner tile resident,
// the other side streamed, everything recomputed from q, k, v, dO and the forward's log-sum-exp):
//
//   DKV = true   owner = 128 keys (K, V tiles), stream = blocks of 64 queries (Q, dO, lse, delta):
//                S^T = K Q^T, dP^T = V dO^T (lanes = keys), P^T = exp2(S^T c - lse), dS^T = P^T (dP^T - delta) scale,
//                dV += P^T dO, dK += dS^T Q          (P^T, dS^T as bf16 A operands read from TMEM)
//   DKV = false  owner = 128 queries (Q, dO tiles), stream = blocks of 64 keys (K, V):
//                S = Q K^T, dP = dO V^T (lanes = queries), dS = P (dP - delta) scale, dQ += dS K
//
// The score tiles are computed twice (once per launch) so that no gradient needs atomics or a second pass:
// each output row is written exactly once.  TMEM: two S buffers [0,64) [64,128), two dP buffers [128,192)
// [192,256), accumulators [256,384) and [384,512).  With two score buffers the issuing thread runs one block
// ahead: S/dP of block n+1 are computed while the element-wise warps turn block n into P / dS, whose
// accumulating MMAs then overlap the element-wise work on block n+1.  The bf16 operands alias the fp32
// tiles they were computed from (each element-wise warp writes only inside the 32 columns it has read).
// 576 threads: warp 0 TMA (4-stage ring of stream blocks), warp 1 MMA, warps 2-17 element-wise (warp w: TMEM
// lanes (w%4)*32.., columns ((w-2)/4)*16.. of the block; sixteen warps because the work is bound by
// TMEM round-trip latency, not by issue slots).  delta[h,i] = sum_d dO[i,h,d] O[i,h,d] and
// lse2 = lse * log2(e) come from a small pre-kernel.
namespace mng {

constexpr int ATB_THREADS = 576;                          // 2 + 16 warps
constexpr int ATB_STAGES = 4;
constexpr int ATB_BLK = 64;                               // stream rows per block
constexpr int ATB_YTILE = ATB_BLK * 128 * 2;              // 16 KB: two boxes of 64 rows x 64 dims
constexpr int ATB_VEC_BYTES = ATB_STAGES * 2 * ATB_BLK * 4;
constexpr int ATB_SMEM = 2 * ATT_TILE_BYTES + ATB_STAGES * 2 * ATB_YTILE + ATB_VEC_BYTES + 1024 + 1024;

struct AttnBwdParams {
  const int* doc_start;     // [T]
  const int* doc_end;       // [T] first token of the next document
  const float* lse2;        // [H, T] log-sum-exp in log2 units
  const float* delta;       // [H, T] rowsum(dO o O) * scale
  __nv_bfloat16* out1;      // DKV: dK, else dQ     [T, H, 128]
  __nv_bfloat16* out2;      // DKV: dV
  int T, H, window;
  float scale_log2, scale;
  int* work_counter;        // items beyond the first of each CTA are claimed here; null = static stride of gridDim.x
};

// Work counters of the two backward kernels of one call (dK/dV, dQ); the prep kernel, which precedes both on the stream,
// zeroes them.  One set per device: backward calls on different streams of one device must not overlap.
static __device__ int g_atb_work[2];

__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                     const float* __restrict__ lse, float* __restrict__ delta, float* __restrict__ lse2, int T,
                                     int H, float scale) {
  const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 4;      // (token, head) pair: 16 lanes each
  const int part = threadIdx.x & 15;
  float acc = 0.f;
  if (blockIdx.x == 0 && threadIdx.x < 2) g_atb_work[threadIdx.x] = 0;
  if (row < (long long)T * H) {
    const uint4 a = *reinterpret_cast<const uint4*>(o + row * 128 + part * 8);
    const uint4 b = *reinterpret_cast<const uint4*>(dout + row * 128 + part * 8);
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 x = __bfloat1622float2(a2[t]), y = __bfloat1622float2(b2[t]);
      acc += x.x * y.x + x.y * y.y;
    }
  }
#pragma unroll
  for (int s = 8; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if (part == 0 && row < (long long)T * H) {
    const int i = (int)(row / H), h = (int)(row % H);
    delta[(size_t)h * T + i] = acc * scale;       // pre-multiplied: dS = P (dP scale - delta scale)
    lse2[(size_t)h * T + i] = lse[(size_t)h * T + i] * 1.4426950408889634f;
  }
}

__device__ __forceinline__ void attn_bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :
               : "r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <bool DKV>
__global__ void __launch_bounds__(ATB_THREADS, 1)
attn_bwd_kernel(const __grid_constant__ CUtensorMap tx1, const __grid_constant__ CUtensorMap tx2,
                const __grid_constant__ CUtensorMap ty1, const __grid_constant__ CUtensorMap ty2, AttnBwdParams p,
                uint32_t* status) {
  // Persistent: CTA c works on items c, c + gridDim.x, ...; item = (128-row owner tile, head), heads fastest.  TMEM is
  // allocated once; the stream ring, the score buffers and every barrier phase run on counters that continue across
  // items, so the next item's owner-tile load and first score MMAs overlap the previous item's accumulator drain.
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sX1 = smem;
  uint8_t* sX2 = smem + ATT_TILE_BYTES;
  uint8_t* sY = smem + 2 * ATT_TILE_BYTES;                  // stage s: Y1 at sY + s*2*YTILE, Y2 right after
  float* vec = reinterpret_cast<float*>(sY + ATB_STAGES * 2 * ATB_YTILE);   // stage s: lse2 at vec + s*128, delta at +64
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(vec) + ATB_VEC_BYTES);
  uint64_t* x_full = bars + 0;
  uint64_t* y_full = bars + 1;                     // [4]
  uint64_t* y_empty = y_full + ATB_STAGES;         // [4]
  uint64_t* sdp_full = y_empty + ATB_STAGES;       // [2]
  uint64_t* pds_ready = sdp_full + 2;              // [2]
  uint64_t* acc_done = pds_ready + 2;              // accumulators of the item complete
  uint64_t* x_free = acc_done + 1;                 // owner tiles no longer read by any MMA
  uint64_t* acc_free = x_free + 1;                 // accumulators drained by the 16 element-wise warps
  uint64_t* item_full = acc_free + 1;              // [2] item ring: the producer publishes the ids it claimed
  uint64_t* item_empty = item_full + 2;            // [2] read by the MMA thread and the 16 element-wise warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + 2);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  volatile int* item_slot = reinterpret_cast<volatile int*>(tmem_slot + 2);    // [2], -1 = no more work

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (p.T + 127) / 128;
  const int items = tiles * p.H;

  // owner tile start, head, stream start row and number of 64-row blocks of an item
  auto item_geom = [&](int item, int& h, int& r0, int& s0, int& nb) {
    const int tile = item / p.H;
    h = item - tile * p.H;
    r0 = (DKV ? tile : tiles - 1 - tile) * 128;
    const int r_last = min(r0 + 127, p.T - 1);
    if (DKV) {
      s0 = r0;
      const int i_max = min(min(r_last + p.window, p.doc_end[r_last] - 1), p.T - 1);
      nb = (i_max - s0) / ATB_BLK + 1;
    } else {
      s0 = max(p.doc_start[r0], r0 - p.window);
      nb = (r_last - s0) / ATB_BLK + 1;
    }
  };

  if (threadIdx.x == 0) {
    mbar_init(x_full, 1);
    for (int s = 0; s < ATB_STAGES; ++s) {
      mbar_init(&y_full[s], 1);
      mbar_init(&y_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sdp_full[s], 1);
      mbar_init(&pds_ready[s], 16);
    }
    mbar_init(acc_done, 1);
    mbar_init(x_free, 1);
    mbar_init(acc_free, 16);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&item_full[s], 1);
      mbar_init(&item_empty[s], 17);
    }
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tx1);
    tma_prefetch_desc(&tx2);
    tma_prefetch_desc(&ty1);
    tma_prefetch_desc(&ty2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tmem_slot;
  const uint32_t tm_S = tm, tm_dP = tm + 128, tm_A1 = tm + 256, tm_A2 = tm + 384;
#define ATB_FAIL(code)                                                          \
  do {                                                                          \
    if (*abort_flag == 0) { *abort_flag = (code); atomicCAS(status, 0u, (code)); } \
  } while (0)

  if (warp == 0) {
    if (lane == 0) {
      int gn = 0, it = 0, next = blockIdx.x;
      bool ok = true;
      for (; ok; ++it) {
        const int item = next < items ? next : -1;
        if (!mbar_wait(&item_empty[it & 1], ((it >> 1) & 1) ^ 1, abort_flag)) { ATB_FAIL(ERR_WAIT_SMEM_EMPTY); break; }
        item_slot[it & 1] = item;
        mbar_arrive(&item_full[it & 1]);
        if (item < 0) break;
        next = p.work_counter ? (int)gridDim.x + atomicAdd(p.work_counter, 1) : item + (int)gridDim.x;   // claimed early, used next round
        int h, r0, s0, nb;
        item_geom(item, h, r0, s0, nb);
        if (!mbar_wait(x_free, (it & 1) ^ 1, abort_flag)) { ATB_FAIL(ERR_WAIT_SMEM_EMPTY); break; }
        mbar_expect_tx(x_full, 2 * ATT_TILE_BYTES);
        tma_load_3d(sX1, &tx1, x_full, 0, h, r0);
        tma_load_3d(sX1 + 16384, &tx1, x_full, 64, h, r0);
        tma_load_3d(sX2, &tx2, x_full, 0, h, r0);
        tma_load_3d(sX2 + 16384, &tx2, x_full, 64, h, r0);
        for (int n = 0; n < nb; ++n, ++gn) {
          const int st = gn % ATB_STAGES, srow = s0 + n * ATB_BLK;
          if (!mbar_wait(&y_empty[st], ((gn / ATB_STAGES) & 1) ^ 1, abort_flag)) { ATB_FAIL(ERR_WAIT_SMEM_EMPTY); ok = false; break; }
          uint8_t* y1 = sY + st * 2 * ATB_YTILE;
          uint8_t* y2 = y1 + ATB_YTILE;
          uint32_t bytes = 2 * ATB_YTILE;
          const int cnt = min(ATB_BLK, p.T - srow);
          if (DKV) bytes += 2u * cnt * 4u;
          mbar_expect_tx(&y_full[st], bytes);
          tma_load_3d(y1, &ty1, &y_full[st], 0, h, srow);
          tma_load_3d(y1 + ATB_YTILE / 2, &ty1, &y_full[st], 64, h, srow);
          tma_load_3d(y2, &ty2, &y_full[st], 0, h, srow);
          tma_load_3d(y2 + ATB_YTILE / 2, &ty2, &y_full[st], 64, h, srow);
          if (DKV) {
            attn_bulk_load(vec + st * 2 * ATB_BLK, p.lse2 + (size_t)h * p.T + srow, cnt * 4, &y_full[st]);
            attn_bulk_load(vec + st * 2 * ATB_BLK + ATB_BLK, p.delta + (size_t)h * p.T + srow, cnt * 4, &y_full[st]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC_SS = make_idesc(1, 1, 0, 0, 128, ATB_BLK);
      constexpr uint32_t IDESC_TS = make_idesc(1, 1, 0, 1, 128, 128);
      const uint64_t dX1 = make_smem_desc(smem_u32(sX1), 16, 1024), dX2 = make_smem_desc(smem_u32(sX2), 16, 1024);
      const uint64_t dYk = make_smem_desc(smem_u32(sY), 16, 1024);                 // stream tile as K-major B (scores)
      const uint64_t dYm = make_smem_desc(smem_u32(sY), ATB_YTILE / 2, 1024);      // the same bytes as MN-major B (accumulation)
      const uint32_t x1l = (uint32_t)dX1, x1h = (uint32_t)(dX1 >> 32), x2l = (uint32_t)dX2, x2h = (uint32_t)(dX2 >> 32);
      // Per block g (numbered across all items of this CTA): scores of g, then the accumulation of g-1.  The owner
      // tiles are only read by score MMAs, so they are released right after an item's last score MMA and the next
      // item's tiles load under its last block.  (Issuing the next item's first scores before the last accumulation
      // measured 5% slower: the accumulation gates the drain.)
#define ATB_XO(k) ((((k) >> 2) * 16384 + ((k) & 3) * 32) >> 4)
#define ATB_YO(k) ((((k) >> 2) * (ATB_YTILE / 2) + ((k) & 3) * 32) >> 4)
#define ATB_ACOL(k) (b * ATB_BLK + (k) * 16)
      bool ok = true;
      // accumulate global block gm from its bf16 operands in TMEM; `first`/`last`: position in its item, `itm`: item ordinal
      auto accumulate = [&](int gm, bool first, bool last, int itm) {
        const int st = gm % ATB_STAGES, b = gm & 1;
        const uint64_t dY1 = dYm + ((st * 2 * ATB_YTILE) >> 4), dY2 = dY1 + (ATB_YTILE >> 4);
        if (first && itm > 0) {                              // the previous item's accumulators must have been drained
          if (!mbar_wait(acc_free, (itm - 1) & 1, abort_flag)) { ATB_FAIL(ERR_WAIT_TMEM_EMPTY); ok = false; return; }
        }
        if (!mbar_wait(&pds_ready[b], (gm >> 1) & 1, abort_flag)) { ATB_FAIL(ERR_WAIT_TMEM_EMPTY); ok = false; return; }
        tc_fence_after();
        const uint32_t y1l = (uint32_t)dY1, y1h = (uint32_t)(dY1 >> 32), y2l = (uint32_t)dY2, y2h = (uint32_t)(dY2 >> 32);
        if (first) {
          if (DKV) umma_f16_ts_lo<false>(tm_A2, tm_S + ATB_ACOL(0), y2l, y2h, IDESC_TS);
          umma_f16_ts_lo<false>(tm_A1, tm_dP + ATB_ACOL(0), y1l, y1h, IDESC_TS);
        } else {
          if (DKV) umma_f16_ts_lo<true>(tm_A2, tm_S + ATB_ACOL(0), y2l, y2h, IDESC_TS);
          umma_f16_ts_lo<true>(tm_A1, tm_dP + ATB_ACOL(0), y1l, y1h, IDESC_TS);
        }
#pragma unroll
        for (int k = 1; k < ATB_BLK / 16; ++k) {              // 16 stream rows per MMA: 8 TMEM columns of packed bf16
          if (DKV) umma_f16_ts_lo<true>(tm_A2, tm_S + ATB_ACOL(k), y2l + ((k * 2048) >> 4), y2h, IDESC_TS);   // dV += P^T dO
          umma_f16_ts_lo<true>(tm_A1, tm_dP + ATB_ACOL(k), y1l + ((k * 2048) >> 4), y1h, IDESC_TS);           // dK += dS^T Q / dQ += dS K
        }
        umma_commit(&y_empty[st]);
        if (last) umma_commit(acc_done);
      };
      int g = 0;                                             // global block index
      bool pend = false, pend_first = false, pend_last = false;   // block g-1 waits for its accumulation
      int pend_it = 0;
      for (int it = 0; ok; ++it) {
        if (!mbar_wait(&item_full[it & 1], (it >> 1) & 1, abort_flag)) { ATB_FAIL(ERR_WAIT_TMA_FULL); break; }
        const int item = item_slot[it & 1];
        mbar_arrive(&item_empty[it & 1]);
        if (item < 0) break;
        int h, r0, s0, nb;
        item_geom(item, h, r0, s0, nb);
        if (pend) {                                          // finish the previous item first: its drain is on the critical path
          accumulate(g - 1, pend_first, pend_last, pend_it);
          pend = false;
          if (!ok) break;
        }
        if (!mbar_wait(x_full, it & 1, abort_flag)) { ATB_FAIL(ERR_WAIT_TMA_FULL); break; }
        for (int n = 0; ok && n < nb; ++n, ++g) {
          const int st = g % ATB_STAGES, b = g & 1;          // scores of block g into buffer g & 1
          const uint64_t dY1 = dYk + ((st * 2 * ATB_YTILE) >> 4), dY2 = dY1 + (ATB_YTILE >> 4);
          if (!mbar_wait(&y_full[st], (g / ATB_STAGES) & 1, abort_flag)) { ATB_FAIL(ERR_WAIT_TMA_FULL); ok = false; break; }
          tc_fence_after();
          const uint32_t y1l = (uint32_t)dY1, y1h = (uint32_t)(dY1 >> 32), y2l = (uint32_t)dY2, y2h = (uint32_t)(dY2 >> 32);
          const uint32_t dS = tm_S + b * ATB_BLK, dD = tm_dP + b * ATB_BLK;
          umma_f16_lo<false>(dS, x1l + ATB_XO(0), x1h, y1l + ATB_YO(0), y1h, IDESC_SS);
          umma_f16_lo<false>(dD, x2l + ATB_XO(0), x2h, y2l + ATB_YO(0), y2h, IDESC_SS);
#pragma unroll
          for (int k = 1; k < 8; ++k) {
            umma_f16_lo<true>(dS, x1l + ATB_XO(k), x1h, y1l + ATB_YO(k), y1h, IDESC_SS);
            umma_f16_lo<true>(dD, x2l + ATB_XO(k), x2h, y2l + ATB_YO(k), y2h, IDESC_SS);
          }
          umma_commit(&sdp_full[b]);
          if (n == nb - 1) umma_commit(x_free);
          if (pend) accumulate(g - 1, pend_first, pend_last, pend_it);
          pend = true;
          pend_first = n == 0;
          pend_last = n == nb - 1;
          pend_it = it;
        }
      }
      if (ok && pend) accumulate(g - 1, pend_first, pend_last, pend_it);
    }
  } else {
    const int sub = warp & 3, quarter = (warp - 2) >> 2;     // TMEM lanes sub*32.., block columns quarter*16..
    const int r = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const float c = p.scale_log2, sc = p.scale;
    bool alive = true;
    int gn = 0, it = 0;
    for (; alive; ++it) {
      if (!mbar_wait(&item_full[it & 1], (it >> 1) & 1, abort_flag)) { ATB_FAIL(ERR_WAIT_TMA_FULL); break; }
      const int item = item_slot[it & 1];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[it & 1]);
      if (item < 0) break;
      int h, r0, s0, nb;
      item_geom(item, h, r0, s0, nb);
      const int g = r0 + r;                                  // owner row: a key (DKV) or a query
      const bool row_ok = g < p.T;
      int lo, hi;                                            // visible stream rows for this owner row
      float my_lse2 = 0.f, my_delta = 0.f;
      if (DKV) {
        lo = g;
        hi = row_ok ? min(min(g + p.window, p.doc_end[g] - 1), p.T - 1) : -1;
      } else {
        lo = row_ok ? max(p.doc_start[g], g - p.window) : 0;
        hi = row_ok ? g : -1;
        if (row_ok) {
          my_lse2 = p.lse2[(size_t)h * p.T + g];
          my_delta = p.delta[(size_t)h * p.T + g];
        }
      }
      const bool any_vis = hi >= lo;
      const unsigned span = (unsigned)(hi - lo);
      for (int n = 0; n < nb; ++n, ++gn) {
        const int st = gn % ATB_STAGES, b = gn & 1, srow = s0 + n * ATB_BLK;
        if (!mbar_wait(&sdp_full[b], (gn >> 1) & 1, abort_flag)) { ATB_FAIL(ERR_WAIT_TMEM_FULL); alive = false; break; }
        tc_fence_after();
        const float* vl = vec + st * 2 * ATB_BLK + quarter * 16;
        const float* vd = vl + ATB_BLK;
        const uint32_t col = lane_off + b * ATB_BLK + quarter * 16;
        uint32_t s[16], d[16];
        tmem_ld16(tm_S + col, s);
        tmem_ld16(tm_dP + col, d);
        tmem_ld_wait();
        uint32_t pk_p[8], pk_ds[8];
        const int col0 = srow + quarter * 16 - lo;
        const bool full = any_vis && col0 >= 0 && (unsigned)(col0 + 15) <= span;     // all 16 columns visible for this row
        if (__all_sync(0xffffffffu, full)) {
#pragma unroll
          for (int t = 0; t < 16; t += 4) {
            float l2[4], dl[4];
            if (DKV) {
              *reinterpret_cast<float4*>(l2) = *reinterpret_cast<const float4*>(vl + t);
              *reinterpret_cast<float4*>(dl) = *reinterpret_cast<const float4*>(vd + t);
            } else {
#pragma unroll
              for (int u = 0; u < 4; ++u) { l2[u] = my_lse2; dl[u] = my_delta; }
            }
            float pv[4], dv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              pv[u] = exp2f(fmaf(__uint_as_float(s[t + u]), c, -l2[u]));
              dv[u] = pv[u] * fmaf(__uint_as_float(d[t + u]), sc, -dl[u]);
            }
            pk_p[t >> 1] = pack_bf16x2(pv[0], pv[1]);
            pk_p[(t >> 1) + 1] = pack_bf16x2(pv[2], pv[3]);
            pk_ds[t >> 1] = pack_bf16x2(dv[0], dv[1]);
            pk_ds[(t >> 1) + 1] = pack_bf16x2(dv[2], dv[3]);
          }
        } else {
#pragma unroll
          for (int t = 0; t < 16; t += 2) {
            float pv[2], dv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float l2 = DKV ? vl[t + u] : my_lse2;
              const float dl = DKV ? vd[t + u] : my_delta;
              const bool vis = any_vis && (unsigned)(col0 + t + u) <= span;
              const float pe = exp2f(fmaf(__uint_as_float(s[t + u]), c, -l2));
              pv[u] = vis ? pe : 0.f;
              dv[u] = vis ? pe * fmaf(__uint_as_float(d[t + u]), sc, -dl) : 0.f;
            }
            pk_p[t >> 1] = pack_bf16x2(pv[0], pv[1]);
            pk_ds[t >> 1] = pack_bf16x2(dv[0], dv[1]);
          }
        }
        if (DKV) tmem_st8(tm_S + col, pk_p);
        tmem_st8(tm_dP + col, pk_ds);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pds_ready[b]);
      }
      if (!alive) break;
      if (!mbar_wait(acc_done, it & 1, abort_flag)) { ATB_FAIL(ERR_WAIT_TMEM_FULL); alive = false; break; }
      tc_fence_after();
#pragma unroll 1
      for (int which = 0; which < (DKV ? 2 : 1); ++which) {
        __nv_bfloat16* orow = (which == 0 ? p.out1 : p.out2) + ((size_t)g * p.H + h) * 128 + quarter * 32;
        uint32_t v[32];
        tmem_ld32((which == 0 ? tm_A1 : tm_A2) + lane_off + quarter * 32, v);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[8 * t]), __uint_as_float(v[8 * t + 1]));
            w.y = pack_bf16x2(__uint_as_float(v[8 * t + 2]), __uint_as_float(v[8 * t + 3]));
            w.z = pack_bf16x2(__uint_as_float(v[8 * t + 4]), __uint_as_float(v[8 * t + 5]));
            w.w = pack_bf16x2(__uint_as_float(v[8 * t + 6]), __uint_as_float(v[8 * t + 7]));
            *reinterpret_cast<uint4*>(orow + t * 8) = w;
          }
        }
      }
      tc_fence_before();                                     // accumulator reads done before the next item's first accumulating MMA
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_free);
    }
  }
#undef ATB_FAIL

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (*abort_flag != 0) {
      const long long t0 = clock64();
      while (clock64() - t0 < 2000000LL) { __nanosleep(1000); }
    }
    tc_fence_after();
    tmem_dealloc(tm, 512);
  }
}

}  // namespace mng

extern "C" int mng_attn_bwd(const void* q, const void* k, const void* v, const void* out, const void* dout, const float* lse,
                            const int* doc_start, const int* doc_end, void* dq, void* dk, void* dv, float* delta, float* lse2,
                            int T, int H, long long row_stride, int window, float scale, void* stream, uint32_t* status) {
  if (T <= 0 || H <= 0) return 0;
  if (T % 4) return -5;                                    // rows of the [H, T] vectors must stay 16-byte aligned
  CUtensorMap tq, tk, tv, tdo, sq, sk, sv, sdo;            // owner maps (128-row boxes) and stream maps (64-row boxes)
  int rc;
  const long long ds = (long long)H * 128;
  if ((rc = attn_map(&tq, q, T, H, row_stride, 128)) || (rc = attn_map(&sq, q, T, H, row_stride, ATB_BLK))) return rc;
  if ((rc = attn_map(&tk, k, T, H, row_stride, 128)) || (rc = attn_map(&sk, k, T, H, row_stride, ATB_BLK))) return rc - 1000;
  if ((rc = attn_map(&tv, v, T, H, row_stride, 128)) || (rc = attn_map(&sv, v, T, H, row_stride, ATB_BLK))) return rc - 2000;
  if ((rc = attn_map(&tdo, dout, T, H, ds, 128)) || (rc = attn_map(&sdo, dout, T, H, ds, ATB_BLK))) return rc - 3000;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_bwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATB_SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(attn_bwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATB_SMEM) != cudaSuccess)
      return -3;
    attr = true;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const long long rows = (long long)T * H;
  attn_bwd_prep_kernel<<<(unsigned)((rows * 16 + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(out), reinterpret_cast<const __nv_bfloat16*>(dout), lse, delta, lse2, T, H, scale);
  const float c = scale * 1.4426950408889634f;
  // one persistent CTA per SM; MNG_ATTN_BWD=tile launches one CTA per (tile, head) item instead (same kernel)
  // MNG_ATTN_BWD=static keeps the persistent grid but strides the items instead of claiming them from the counter
  static const std::string mode = [] { const char* e = getenv("MNG_ATTN_BWD"); return std::string(e ? e : ""); }();
  static const bool per_item = mode == "tile";
  // the work counters are a __device__ symbol: its address and the SM count belong to the current device
  constexpr int kMaxDevices = 64;
  static int* work_of[kMaxDevices] = {};
  static int sms_of[kMaxDevices] = {};
  static std::mutex mu;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -6;
  int* work = nullptr;
  int sms = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!work_of[dev]) {
      if (cudaGetSymbolAddress(reinterpret_cast<void**>(&work_of[dev]), g_atb_work) != cudaSuccess ||
          cudaDeviceGetAttribute(&sms_of[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        work_of[dev] = nullptr;
        return -6;
      }
    }
    work = work_of[dev];
    sms = sms_of[dev];
  }
  int* const w0 = mode == "static" ? nullptr : work;
  const int items = ((T + 127) / 128) * H;
  dim3 grid(per_item ? items : (items < sms ? items : sms));
  AttnBwdParams pa{doc_start, doc_end, lse2, delta, reinterpret_cast<__nv_bfloat16*>(dk), reinterpret_cast<__nv_bfloat16*>(dv),
                   T, H, window, c, scale, w0};
  attn_bwd_kernel<true><<<grid, ATB_THREADS, ATB_SMEM, st>>>(tk, tv, sq, sdo, pa, status);
  AttnBwdParams pb{doc_start, doc_end, lse2, delta, reinterpret_cast<__nv_bfloat16*>(dq), nullptr, T, H, window, c, scale, w0 ? w0 + 1 : nullptr};
  attn_bwd_kernel<false><<<grid, ATB_THREADS, ATB_SMEM, st>>>(tq, tdo, sk, sv, pb, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
