// Raw tcgen05.mma issue-rate probe for sm_100a: one CTA per SM, one thread issues a long run of MMAs of one shape
// (operands: whatever is in shared memory / TMEM) and times them with clock64.
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -I. -o bench_mma_rate bench_mma_rate.cu && ./bench_mma_rate
#include "modded_nanogpt_b200/csrc/ptx.cuh"
#include <cstdio>
using namespace mng;
template <int N, bool TS, int NACC>
__global__ void __launch_bounds__(128, 1) probe(long long* out, int reps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) { mbar_init(&bar, 1); mbar_fence_init(); }
  if (warp == 0) { tmem_alloc(&slot, 512); tmem_relinquish(); }
  tc_fence_before(); __syncthreads(); tc_fence_after();
  const uint32_t tm = slot;
  if (threadIdx.x == 0) {
    constexpr uint32_t IDESC = make_idesc(1, 1, 0, 0, 128, N);
    const uint64_t dA = make_smem_desc(smem_u32(smem), 16, 1024), dB = make_smem_desc(smem_u32(smem + 32768), 16, 1024);
    const long long t0 = clock64();
    for (int r = 0; r < reps; ++r) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
          const uint32_t off = ((k >> 2) * 16384 + (k & 3) * 32) >> 4;
          if (TS) umma_f16_ts(tm + a * N, tm + 448 + k * 8, dB + off, IDESC, 1);
          else umma_f16(tm + a * N, dA + off, dB + off, IDESC, 1);
        }
      }
    }
    umma_commit(&bar);
    volatile uint32_t ab = 0;
    mbar_wait(&bar, 0, &ab);
    const long long t1 = clock64();
    if (blockIdx.x == 0) out[0] = t1 - t0;
  }
  tc_fence_before(); __syncthreads();
  if (warp == 0) { tc_fence_after(); tmem_dealloc(tm, 512); }
}
template <int N, bool TS, int NACC>
void run(const char* name, long long* d, int grid) {
  auto k = probe<N, TS, NACC>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
  const int reps = 200;
  k<<<grid, 128, 100 * 1024>>>(d, reps);
  k<<<grid, 128, 100 * 1024>>>(d, reps);
  cudaDeviceSynchronize();
  long long h = 0; cudaMemcpy(&h, d, 8, cudaMemcpyDeviceToHost);
  printf("%-34s grid %3d: %7.1f clks per MMA (math %d)  err=%s\n", name, grid, (double)h / (reps * 8 * NACC), N / 2, cudaGetErrorString(cudaGetLastError()));
}
int main() {
  long long* d; cudaMalloc(&d, 64);
  for (int grid : {1, 148}) {
    run<64, false, 1>("SS N=64  one chain", d, grid);
    run<64, false, 2>("SS N=64  two chains interleaved", d, grid);
    run<128, false, 1>("SS N=128 one chain", d, grid);
    run<128, false, 2>("SS N=128 two chains", d, grid);
    run<256, false, 1>("SS N=256 one chain", d, grid);
    run<64, true, 1>("TS N=64  one chain", d, grid);
    run<128, true, 1>("TS N=128 one chain", d, grid);
    run<128, true, 2>("TS N=128 two chains", d, grid);
    run<256, true, 1>("TS N=256 one chain", d, grid);
  }
  return 0;
}
