// CTA-pair variant of the persistent tcgen05 GEMM: a cluster of two CTAs on neighbouring SMs computes
// one 256 x 256 output tile per step with tcgen05.mma.cta_group::2, and the output path runs entirely
// through TMA: optional addend / saved-activation tiles are prefetched into shared memory while the tile's
// MMAs run, results are written back with bulk tensor stores.
//
// Why: measured on B200 with K = 768 the load + MMA pipeline alone sustains the cuBLAS rate, but an
// epilogue that stores (and, for the MLP backward, loads) through the LSU path costs 30-130 % on top: the
// eight epilogue warps stall on their own global accesses and the accumulator buffers are released late.
// With bulk stores the warps only write shared memory.
//
// Layout of the work inside a pair (rank = %cluster_ctarank):
//   * A tile rows   [m0 + rank*128, +128)            -> own shared memory, own TMA loads
//   * B tile rows   [n0 + rank*128, +128)            -> own shared memory, own TMA loads
//   * accumulator   rows [m0 + rank*128, +128) x 256 -> own TMEM (2 buffers x 256 columns)
//   * rank 0 ("leader") waits for both CTAs' bytes on ITS full barrier (the peer's loads signal it through
//     the .cta_group::2 form of the copy; no load is multicast) and issues every MMA; its
//     tcgen05.commit arrives on the slot-free / accumulator-ready barriers of both CTAs;
//   * epilogue warp w (2..9) owns rows (w%4)*32..+32 and columns ((w-2)/4)*128..+128 of its CTA's half tile,
//     staged as two 32 x 128-byte boxes (64 bf16 columns each, 128-byte swizzle) plus, for the fp8 copy,
//     one 32 x 128-byte box; it arrives on the leader's accumulator-free barrier as soon as its last
//     TMEM load has landed.
// Every wait is bounded; both CTAs meet at a cluster barrier before TMEM is released.
//
// Tile epilogue contract:
//   struct Epi { static constexpr bool kCin, kOut8; struct Params; struct State;
//     __device__ static void apply(const Params&, State&, const float (&acc)[32], const uint4 (&cin)[4],
//                                  uint4 (&out)[4], uint4 (&out8)[2], int batch, long long row, int col0, int M, int N);
//     __device__ static void finish(const Params&, State&); }
// acc[j] = element (row, col0 + j); cin / out hold the same 32 positions as bf16; out8 as e4m3.
// Optional members (detected below): `static constexpr bool kStore16 = false` - no bf16 output at all (only the
// 8-bit copy, or nothing); `static constexpr bool kTileHooks = true` - the epilogue keeps per-row state over the
// 128 columns a warp owns in a tile: the kernel sets st.taddr to the TMEM address of the warp's 128-column slab and
// calls tile_begin(ep, st, b, row, n0, M, N) before the four chunks (it may re-read single accumulator columns with
// tmem_ld1 there), and tile_end(ep, st, b, row, n0, M, N) after them.  For these epilogues the chunk loop is
// unrolled and the TMEM load of chunk c + 1 is in flight while chunk c is processed.
// `static constexpr bool kCustomStore = true`: the epilogue issues the bulk stores of the warp's two staged
// 32 x 64 boxes itself - issue_stores(ep, maps, stg, b, m0, n0, M, N), called by lane 0 - e.g. to route column ranges
// to different output tensors or to shift a box by a row.
#pragma once
#include "gemm_sm100.cuh"

namespace mng {

template <class E, class = void> struct epi_store16 { static constexpr bool value = true; };
template <class E> struct epi_store16<E, decltype((void)E::kStore16)> { static constexpr bool value = E::kStore16; };
template <class E, class = void> struct epi_custom_store { static constexpr bool value = false; };
template <class E> struct epi_custom_store<E, decltype((void)E::kCustomStore)> { static constexpr bool value = E::kCustomStore; };
template <class E, class = void> struct epi_hooks { static constexpr bool value = false; };
template <class E> struct epi_hooks<E, decltype((void)E::kTileHooks)> { static constexpr bool value = E::kTileHooks; };

template <bool OUT8>
struct GemmPairSmem {
  static constexpr int BN = 256;
  static constexpr int A_BYTES = GEMM_BM * GEMM_STAGE_K_BYTES;         // 16 KB: 128 rows of A
  static constexpr int B_BYTES = (BN / 2) * GEMM_STAGE_K_BYTES;        // 16 KB: this CTA's half of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = OUT8 ? 4 : 5;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int BOX_BYTES = 4096;                               // 32 rows x 128 bytes
  static constexpr int WARP_STG_BYTES = (OUT8 ? 3 : 2) * BOX_BYTES;
  static constexpr int TOTAL = STAGES * STAGE_BYTES + BAR_BYTES + GEMM_EPI_WARPS * WARP_STG_BYTES + 1024;
};

struct PairMaps {
  CUtensorMap a, b, out, cin, out8;
  CUtensorMap out2, out3;       // epilogues with `kCustomStore`: further bf16 outputs (same box shape as `out`)
};

template <int ES, bool A_MN, bool B_MN, uint32_t A_FMT, uint32_t B_FMT, class Epi>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_tcgen05_pair_kernel(const __grid_constant__ PairMaps maps, GemmShape shape, typename Epi::Params ep, uint32_t* status) {
  using SM = GemmPairSmem<Epi::kOut8>;
  constexpr int BN = 256, BNH = 128, BM2 = 2 * GEMM_BM;
  constexpr int STAGES = SM::STAGES;
  constexpr int BK = GEMM_STAGE_K_BYTES / ES;
  constexpr int UMMA_K = 32 / ES;
  constexpr int KSTEPS = BK / UMMA_K;
  constexpr uint32_t IDESC = make_idesc(A_FMT, B_FMT, A_MN ? 1 : 0, B_MN ? 1 : 0, BM2, BN);
  constexpr int CHUNK_ELEMS = 128 / ES;
  constexpr int A_CHUNKS = GEMM_BM / CHUNK_ELEMS;
  constexpr int B_CHUNKS = BNH / CHUNK_ELEMS;
  constexpr uint32_t CHUNK_BYTES = BK * 128;
  constexpr bool STORE16 = epi_store16<Epi>::value;
  constexpr bool HOOKS = epi_hooks<Epi>::value;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bars = smem + STAGES * SM::STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(bars);      // used in the leader only
  uint64_t* empty_bar = full_bar + STAGES;                     // per CTA, signalled by the leader's commits
  uint64_t* tfull_bar = empty_bar + STAGES;                    // per CTA, signalled by the leader's commits
  uint64_t* tempty_bar = tfull_bar + 2;                        // used in the leader only: 2 x 8 epilogue warps
  uint64_t* cin_bar = tempty_bar + 2;                          // one per epilogue warp: its addend boxes have landed
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(cin_bar + GEMM_EPI_WARPS);
  volatile uint32_t* abort_flag = tmem_base_slot + 1;
  uint8_t* stg_base = bars + SM::BAR_BYTES;                    // 1024-byte aligned

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = (int)cluster_id_x();
  const int num_pairs = (int)cluster_count_x();
  const int tiles_m = (shape.M + BM2 - 1) / BM2;
  const int tiles_n = (shape.N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n * shape.batch;
  const int num_kb = (shape.K + BK - 1) / BK;
  constexpr uint32_t TMEM_COLS = 2 * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull_bar[s], 1);
      mbar_init(&tempty_bar[s], 2 * GEMM_EPI_WARPS);
    }
    for (int s = 0; s < GEMM_EPI_WARPS; ++s) mbar_init(&cin_bar[s], 1);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&maps.a);
    tma_prefetch_desc(&maps.b);
    if constexpr (STORE16) tma_prefetch_desc(&maps.out);
    if constexpr (epi_custom_store<Epi>::value) {
      tma_prefetch_desc(&maps.out2);
      tma_prefetch_desc(&maps.out3);
    }
    if constexpr (Epi::kCin) tma_prefetch_desc(&maps.cin);
    if constexpr (Epi::kOut8) tma_prefetch_desc(&maps.out8);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();                                          // the peer's barriers exist before anything signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer (both CTAs) ------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = pair; tile < num_tiles; tile += num_pairs) {
        const int b = tile / (tiles_m * tiles_n);
        const int r = tile - b * tiles_m * tiles_n;
        const int m0 = (r / tiles_n) * BM2 + (int)rank * GEMM_BM;
        const int n0 = (r % tiles_n) * BN + (int)rank * BNH;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) {
            if (*abort_flag == 0) { *abort_flag = ERR_WAIT_SMEM_EMPTY; atomicCAS(status, 0u, ERR_WAIT_SMEM_EMPTY); }
            goto producer_done;
          }
          uint8_t* sa = smem + stage * SM::STAGE_BYTES;
          uint8_t* sb = sa + SM::A_BYTES;
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (rank == 0) mbar_expect_tx(&full_bar[stage], 2 * SM::STAGE_BYTES);     // both CTAs' bytes
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_3d_pair(sa, &maps.a, fb, k0, m0, b);
          } else {
#pragma unroll
            for (int c = 0; c < A_CHUNKS; ++c) tma_load_3d_pair(sa + c * CHUNK_BYTES, &maps.a, fb, m0 + c * CHUNK_ELEMS, k0, b);
          }
          if constexpr (!B_MN) {
            tma_load_3d_pair(sb, &maps.b, fb, k0, n0, b);
          } else {
#pragma unroll
            for (int c = 0; c < B_CHUNKS; ++c) tma_load_3d_pair(sb + c * CHUNK_BYTES, &maps.b, fb, n0 + c * CHUNK_ELEMS, k0, b);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  producer_done:;
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (leader only) ------------------------------------
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = pair; tile < num_tiles; tile += num_pairs) {
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
            const uint64_t da = A_MN ? make_smem_desc(sa + k * UMMA_K * 128, CHUNK_BYTES, 1024)
                                     : make_smem_desc(sa + k * 32, 16, 1024);
            const uint64_t db = B_MN ? make_smem_desc(sb + k * UMMA_K * 128, CHUNK_BYTES, 1024)
                                     : make_smem_desc(sb + k * 32, 16, 1024);
            if constexpr (ES == 2) umma_f16_pair(tmem_d, da, db, IDESC, (kb | k) != 0);
            else umma_f8_pair(tmem_d, da, db, IDESC, (kb | k) != 0);
          }
          umma_commit_pair(&empty_bar[stage], 3);            // slot free in both CTAs
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        umma_commit_pair(&tfull_bar[acc], 3);                // accumulator ready in both CTAs
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  mma_done:;
  } else {
    // ------------------------------ epilogue warps (both CTAs) ----------------------------------
    const int ew = warp - 2;
    const int q = warp & 3;                                    // TMEM sub-partition = 32-row group of the tile
    const int half = ew >> 2;                                  // which 128 columns
    uint8_t* stg = stg_base + ew * SM::WARP_STG_BYTES;
    const int sw = lane & 7;
    int acc = 0;
    uint32_t acc_phase = 0, cin_phase = 0;
    typename Epi::State est{};

    auto tile_coords = [&](int tile, int& b, int& m0, int& n0) {
      b = tile / (tiles_m * tiles_n);
      const int r = tile - b * tiles_m * tiles_n;
      m0 = (r / tiles_n) * BM2 + (int)rank * GEMM_BM + q * 32;
      n0 = (r % tiles_n) * BN + half * 128;
    };
    auto load_cin = [&](int tile) {                            // lane 0 only; the staging boxes must be free
      int b, m0, n0;
      tile_coords(tile, b, m0, n0);
      mbar_expect_tx(&cin_bar[ew], 2 * SM::BOX_BYTES);
      tma_load_3d(stg, &maps.cin, &cin_bar[ew], n0, m0, b);
      tma_load_3d(stg + SM::BOX_BYTES, &maps.cin, &cin_bar[ew], n0 + 64, m0, b);
    };
    if constexpr (Epi::kCin) {
      if (lane == 0 && pair < num_tiles) load_cin(pair);
    }

    for (int tile = pair; tile < num_tiles; tile += num_pairs) {
      int b, m0, n0;
      tile_coords(tile, b, m0, n0);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag)) {
        if (*abort_flag == 0) { *abort_flag = ERR_WAIT_TMEM_FULL; atomicCAS(status, 0u, ERR_WAIT_TMEM_FULL); }
        break;
      }
      if constexpr (Epi::kCin) {
        if (!mbar_wait(&cin_bar[ew], cin_phase, abort_flag)) {
          if (*abort_flag == 0) { *abort_flag = ERR_WAIT_TMA_FULL; atomicCAS(status, 0u, ERR_WAIT_TMA_FULL); }
          break;
        }
        cin_phase ^= 1;
      }
      tc_fence_after();
      if constexpr (!Epi::kCin && (STORE16 || Epi::kOut8)) {
        // the previous tile's bulk stores have had a whole tile of MMA time to read the staging boxes: waiting
        // here, not right after issuing them, keeps the warp from idling on the store engine
        if (lane == 0) tma_store_wait_read<0>();
        __syncwarp();
      }
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + half * 128;
      // one chunk: registers -> epilogue functor -> staging boxes
      auto do_chunk = [&](int c, const uint32_t (&v)[32]) {
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
        uint8_t* rowp = stg + (c >> 1) * SM::BOX_BYTES + lane * 128;
        const int cb = (c & 1) * 4;
        uint4 cin[4], out[4], out8[2];
        if constexpr (Epi::kCin) {
#pragma unroll
          for (int j = 0; j < 4; ++j) cin[j] = *reinterpret_cast<const uint4*>(rowp + (((cb + j) ^ sw) << 4));
        }
        Epi::apply(ep, est, f, cin, out, out8, b, (long long)m0 + lane, n0 + c * 32, shape.M, shape.N);
        if constexpr (STORE16) {
#pragma unroll
          for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(rowp + (((cb + j) ^ sw) << 4)) = out[j];
        }
        if constexpr (Epi::kOut8) {
          uint8_t* rowp8 = stg + 2 * SM::BOX_BYTES + lane * 128;
#pragma unroll
          for (int j = 0; j < 2; ++j) *reinterpret_cast<uint4*>(rowp8 + (((c * 2 + j) ^ sw) << 4)) = out8[j];
        }
      };
      auto release_acc = [&]() {                               // everything this warp needs is in registers
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[acc]), 0));
      };
      if constexpr (HOOKS) {
        est.taddr = taddr;
        Epi::tile_begin(ep, est, b, (long long)m0 + lane, n0, shape.M, shape.N);
        uint32_t va[32], vb[32];
        tmem_ld32(taddr, va);
        tmem_ld_wait();
        tmem_ld32(taddr + 32, vb);
        do_chunk(0, va);
        tmem_ld_wait();
        tmem_ld32(taddr + 64, va);
        do_chunk(1, vb);
        tmem_ld_wait();
        tmem_ld32(taddr + 96, vb);
        do_chunk(2, va);
        tmem_ld_wait();
        release_acc();
        do_chunk(3, vb);
        Epi::tile_end(ep, est, b, (long long)m0 + lane, n0, shape.M, shape.N);
      } else {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(taddr + c * 32, v);
          tmem_ld_wait();
          if (c == 3) release_acc();
          do_chunk(c, v);
        }
      }
      if constexpr (!(STORE16 || Epi::kOut8)) {                // nothing staged for the store engine: next tile
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
        continue;
      }
      fence_proxy_async_smem();                                // generic-proxy writes -> visible to the bulk stores
      __syncwarp();
      if (lane == 0) {
        if (m0 < shape.M) {
          if constexpr (epi_custom_store<Epi>::value) {
            Epi::issue_stores(ep, maps, stg, b, m0, n0, shape.M, shape.N);
          } else if constexpr (STORE16) {
            if (n0 < shape.N) tma_store_3d(&maps.out, stg, n0, m0, b);
            if (n0 + 64 < shape.N) tma_store_3d(&maps.out, stg + SM::BOX_BYTES, n0 + 64, m0, b);
          }
          if constexpr (Epi::kOut8) {
            if (n0 < shape.N) tma_store_3d(&maps.out8, stg + 2 * SM::BOX_BYTES, n0, m0, b);
          }
        }
        tma_store_commit();
        if constexpr (Epi::kCin) {
          tma_store_wait_read<0>();                            // boxes may be overwritten: by the next addend tile
          if (tile + num_pairs < num_tiles) load_cin(tile + num_pairs);
        }
      }
      __syncwarp();
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    Epi::finish(ep, est);
    if (lane == 0) tma_store_wait_all<0>();
  }

  // ------------------------------ common exit ---------------------------------------------------
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  if (warp == 1 && *abort_flag != 0) {
    const long long t0 = clock64();
    while (clock64() - t0 < 2000000LL) { __nanosleep(1000); }
  }
  cluster_sync_all();                                          // nobody signals or reads the peer after this
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace mng
