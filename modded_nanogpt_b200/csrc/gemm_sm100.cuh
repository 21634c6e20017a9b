// Persistent warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[b] = epilogue( A[b] (M x K) * B[b]^T (N x K) )          fp32 accumulation in TMEM
//
// * operands bf16 (kind::f16) or e4m3/e5m2 (kind::f8f6f4), each either K-major (row-major [rows,K])
//   or MN-major (row-major [K,rows]); tiles arrive by TMA (128-byte swizzle) into a multi-stage
//   shared-memory ring, one elected thread issues tcgen05.mma, accumulators live in TMEM and are
//   double buffered so the epilogue of tile i overlaps the main loop of tile i+1;
// * CTA tile 128 x BN (BN = 128 or 256), K step = 128 bytes of K per operand row;
// * warp 0 = TMA producer, warp 1 = MMA issuer (+ TMEM allocation), warps 2..9 = epilogue (warp w reads
//   the 32-lane TMEM sub-partition `w % 4`; warps 2..5 take the left half of the tile's columns, 6..9 the right);
// * epilogues are functors applied to 32-column register fragments (see epilogues in gemm_sm100.cu);
// * no cluster launch, no multicast loads; every mbarrier wait is bounded.
#pragma once
#include "ptx.cuh"

namespace mng {

constexpr int GEMM_BM = 128;
constexpr int GEMM_THREADS = 320;
constexpr int GEMM_EPI_WARPS = 8;
constexpr int GEMM_STAGE_K_BYTES = 128;   // bytes of K per row and stage (one swizzle span)

struct GemmShape {
  int M, N, K, batch;
  int symmetric;   // single-CTA kernel with BN = 128 only: M == N and the product is symmetric, so only the tiles on and
                   // above the diagonal are computed (the epilogue mirrors them: `triton_kernels.py:51-55` does the same)
};

// Tile index -> (batch, first row, first column).  Symmetric mode walks the upper triangle row by row.
template <int BN>
__device__ __forceinline__ void gemm_tile_coords(const GemmShape& shape, int tile, int tiles_m, int tiles_n, int& b, int& m0, int& n0) {
  if (shape.symmetric) {
    const int per = tiles_n * (tiles_n + 1) / 2;
    b = tile / per;
    int r = tile - b * per, i = 0;
    while (r >= tiles_n - i) { r -= tiles_n - i; ++i; }      // row i holds tiles_n - i tiles: columns i .. tiles_n - 1
    m0 = i * GEMM_BM;
    n0 = (i + r) * BN;
  } else {
    b = tile / (tiles_m * tiles_n);
    const int r = tile - b * tiles_m * tiles_n;
    m0 = (r / tiles_n) * GEMM_BM;
    n0 = (r % tiles_n) * BN;
  }
}

template <int BN, int ES>   // ES = operand element size in bytes
struct GemmSmem {
  static constexpr int A_BYTES = GEMM_BM * GEMM_STAGE_K_BYTES;        // 16 KB
  static constexpr int B_BYTES = BN * GEMM_STAGE_K_BYTES;             // 16 / 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int STG_BYTES = 4096;                                  // epilogue staging per warp
  static constexpr int TOTAL = STAGES * STAGE_BYTES + BAR_BYTES + 8 * STG_BYTES + 1024;   // + alignment slack
};

// Per-warp staging buffer that turns the "one thread = one row" fragments of tcgen05.ld into
// coalesced global traffic.  A warp holds 32 rows x B bytes (B = 32, 64 or 128: 32 columns of 1-, 2-
// or 4-byte elements) as 16-byte chunks with an XOR swizzle that keeps both access patterns free of
// bank conflicts: thread r writes/reads its own row; then B/16 adjacent lanes cover one row, so a warp
// store instruction writes 512 contiguous-per-row bytes (full 32-byte sectors) instead of 32 scattered
// 16-byte pieces.  All methods are warp collectives (every lane must call them).
struct ChunkIO {
  uint8_t* stg;      // 4 KB of shared memory owned by this warp
  int lane;
  template <int B>
  __device__ __forceinline__ static int swz(int j, int row) {
    if constexpr (B == 128) return j ^ (row & 7);
    else if constexpr (B == 64) return j ^ ((row >> 1) & 3);
    else return j ^ ((row >> 2) & 1);
  }
  template <int B>
  __device__ __forceinline__ void put(int j, uint4 v) {                 // chunk j of this lane's row
    *reinterpret_cast<uint4*>(stg + lane * B + swz<B>(j, lane) * 16) = v;
  }
  template <int B>
  __device__ __forceinline__ uint4 get(int j) const {
    return *reinterpret_cast<const uint4*>(stg + lane * B + swz<B>(j, lane) * 16);
  }
  // rows [row0, row0+32) x bytes [col_byte0, col_byte0+B) of a row-major array with row pitch ld_bytes
  template <int B>
  __device__ __forceinline__ void store_rows(void* gbase, long long ld_bytes, long long row0, long long col_byte0, int M) {
    constexpr int LPR = B / 16, RPI = 32 / LPR;
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 32 / RPI; ++it) {
      const int row = it * RPI + lane / LPR, j = lane % LPR;
      const uint4 v = *reinterpret_cast<const uint4*>(stg + row * B + swz<B>(j, row) * 16);
      if (row0 + row < M)
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(gbase) + (row0 + row) * ld_bytes + col_byte0 + j * 16) = v;
    }
    __syncwarp();
  }
  template <int B>
  __device__ __forceinline__ void load_rows(const void* gbase, long long ld_bytes, long long row0, long long col_byte0, int M) {
    constexpr int LPR = B / 16, RPI = 32 / LPR;
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 32 / RPI; ++it) {
      const int row = it * RPI + lane / LPR, j = lane % LPR;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (row0 + row < M)
        v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(gbase) + (row0 + row) * ld_bytes + col_byte0 + j * 16);
      *reinterpret_cast<uint4*>(stg + row * B + swz<B>(j, row) * 16) = v;
    }
    __syncwarp();
  }
};

// Epilogue contract:
//   struct Epi { struct Params {...}; struct State {...};
//     __device__ static void apply(const Params&, State&, ChunkIO&, const float (&acc)[32], int batch,
//                                  long long row0, int col0, int M, int N);
//     __device__ static void finish(const Params&, State&);   // once per epilogue thread, after its last tile
//   }
// `acc[j]` is element (row0 + lane, col0 + j) of the tile product.  `apply` is called by all 32 lanes of
// the warp (it uses warp-collective staging); rows/cols beyond M/N must not be written.

template <int BN, int ES, bool A_MN, bool B_MN, uint32_t A_FMT, uint32_t B_FMT, class Epi>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                    GemmShape shape, typename Epi::Params ep, uint32_t* status) {
  using SM = GemmSmem<BN, ES>;
  constexpr int STAGES = SM::STAGES;
  constexpr int BK = GEMM_STAGE_K_BYTES / ES;           // elements of K per stage (64 bf16 / 128 fp8)
  constexpr int UMMA_K = 32 / ES;                       // 16 for 16-bit, 32 for 8-bit operands
  constexpr int KSTEPS = BK / UMMA_K;                   // 4
  constexpr uint32_t IDESC = make_idesc(A_FMT, B_FMT, A_MN ? 1 : 0, B_MN ? 1 : 0, GEMM_BM, BN);
  constexpr int CHUNK_ELEMS = 128 / ES;                 // MN-major: elements per 128-byte chunk
  constexpr int A_CHUNKS = GEMM_BM / CHUNK_ELEMS;       // MN-major A: boxes per stage
  constexpr int B_CHUNKS = BN / CHUNK_ELEMS;
  constexpr uint32_t CHUNK_BYTES = BK * 128;            // one [BK x 128 B] box

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bars = smem + STAGES * SM::STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(bars);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile uint32_t* abort_flag = tmem_base_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (shape.M + GEMM_BM - 1) / GEMM_BM;
  const int tiles_n = (shape.N + BN - 1) / BN;
  const int num_tiles = (shape.symmetric ? tiles_n * (tiles_n + 1) / 2 : tiles_m * tiles_n) * shape.batch;
  const int num_kb = (shape.K + BK - 1) / BK;
  constexpr uint32_t TMEM_COLS = 2 * BN;                // two accumulator buffers (256 or 512 columns)

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull_bar[s], 1);
      mbar_init(&tempty_bar[s], GEMM_EPI_WARPS);        // one arrival per epilogue warp
    }
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        int b, m0, n0;
        gemm_tile_coords<BN>(shape, tile, tiles_m, tiles_n, b, m0, n0);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) {
            if (*abort_flag == 0) { *abort_flag = ERR_WAIT_SMEM_EMPTY; atomicCAS(status, 0u, ERR_WAIT_SMEM_EMPTY); }
            goto producer_done;
          }
          uint8_t* sa = smem + stage * SM::STAGE_BYTES;
          uint8_t* sb = sa + SM::A_BYTES;
          mbar_expect_tx(&full_bar[stage], SM::STAGE_BYTES);
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_3d(sa, &tma_a, &full_bar[stage], k0, m0, b);
          } else {
#pragma unroll
            for (int c = 0; c < A_CHUNKS; ++c)
              tma_load_3d(sa + c * CHUNK_BYTES, &tma_a, &full_bar[stage], m0 + c * CHUNK_ELEMS, k0, b);
          }
          if constexpr (!B_MN) {
            tma_load_3d(sb, &tma_b, &full_bar[stage], k0, n0, b);
          } else {
#pragma unroll
            for (int c = 0; c < B_CHUNKS; ++c)
              tma_load_3d(sb + c * CHUNK_BYTES, &tma_b, &full_bar[stage], n0 + c * CHUNK_ELEMS, k0, b);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  producer_done:;
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort_flag)) {
          if (*abort_flag == 0) { *abort_flag = ERR_WAIT_TMEM_EMPTY; atomicCAS(status, 0u, ERR_WAIT_TMEM_EMPTY); }
          goto mma_done;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
            if (*abort_flag == 0) { *abort_flag = ERR_WAIT_TMA_FULL; atomicCAS(status, 0u, ERR_WAIT_TMA_FULL); }
            goto mma_done;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * SM::STAGE_BYTES);
          const uint32_t sb = sa + SM::A_BYTES;
#pragma unroll
          for (int k = 0; k < KSTEPS; ++k) {
            // K-major: advance 32 bytes along the swizzled row; MN-major: advance UMMA_K rows of 128 bytes.
            const uint64_t da = A_MN ? make_smem_desc(sa + k * UMMA_K * 128, CHUNK_BYTES, 1024)
                                     : make_smem_desc(sa + k * 32, 16, 1024);
            const uint64_t db = B_MN ? make_smem_desc(sb + k * UMMA_K * 128, CHUNK_BYTES, 1024)
                                     : make_smem_desc(sb + k * 32, 16, 1024);
            if constexpr (ES == 2) umma_f16(tmem_d, da, db, IDESC, (kb | k) != 0);
            else umma_f8(tmem_d, da, db, IDESC, (kb | k) != 0);
          }
          umma_commit(&empty_bar[stage]);               // slot is free once these MMAs have read it
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        umma_commit(&tfull_bar[acc]);                   // accumulator complete
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  mma_done:;
  } else {
    // ------------------------------ epilogue warps ----------------------------------------------
    const int q = warp & 3;                             // TMEM sub-partition of this warp
    const int c_begin = ((warp - 2) >> 2) * (BN / 64);  // first 32-column chunk of this warp's half
    int acc = 0;
    uint32_t acc_phase = 0;
    typename Epi::State est{};                         // per-thread state carried across tiles (e.g. a running max)
    ChunkIO io{bars + SM::BAR_BYTES + (warp - 2) * SM::STG_BYTES, lane};
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int b, m0, n0;
      gemm_tile_coords<BN>(shape, tile, tiles_m, tiles_n, b, m0, n0);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag)) {
        if (*abort_flag == 0) { *abort_flag = ERR_WAIT_TMEM_FULL; atomicCAS(status, 0u, ERR_WAIT_TMEM_FULL); }
        break;
      }
      tc_fence_after();
      const long long row0 = m0 + q * 32;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = c_begin; c < c_begin + BN / 64; ++c) {
        uint32_t v[32];
        tmem_ld32(taddr + c * 32, v);
        tmem_ld_wait();
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
        if (n0 + c * 32 < shape.N) Epi::apply(ep, est, io, f, b, row0, n0 + c * 32, shape.M, shape.N);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    Epi::finish(ep, est);
  }

  // ------------------------------ common exit ---------------------------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (*abort_flag != 0) {
      // give copies still in flight time to land before the shared memory and TMEM are released
      const long long t0 = clock64();
      while (clock64() - t0 < 2000000LL) { __nanosleep(1000); }
    }
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace mng
