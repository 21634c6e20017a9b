// Allocation-free entry point.  This has no counterpart in the reference trainer: it exists for
// users of this library whose host code is not allowed to allocate device memory at the point of
// the call - a runtime that hands out all device memory up front and forbids cudaMalloc afterwards,
// a plugin living inside another framework's memory pool, a latency-critical loop where an
// allocation (and the implicit synchronisation it can cause) is unacceptable.
//
// `mng_quant_transpose_e4m3_static` computes the same result as `mng_quant_transpose_e4m3`
// (api.h): q[c, :] = src[:, c] / s[c] rounded to e4m3, s[c] = max|src[:, c]| / 448, for a row-major
// bf16 matrix `src` of `rows` x `cols`.  The regular entry point needs `cols` 32-bit words of
// scratch from its caller; this one keeps that scratch inside the library, in a file-scope
// `static __device__` array of MNG_STATIC_SCRATCH_COLS words (256 KiB), which every GPU that loads
// the library holds from load until the process exits.
//
// Rules for callers:
//   * `cols` must not exceed MNG_STATIC_SCRATCH_COLS and `rows` must not exceed MNG_STATIC_MAX_ROWS
//     (the kernels tile rows in blocks of 64 along a grid dimension that holds 65,535 blocks); larger
//     inputs are refused with MNG_ERR_TOO_LARGE and nothing is launched.  Inputs and outputs are
//     still the caller's.
//   * The first call on each device resolves the device address of the scratch array
//     (cudaGetSymbolAddress, with that device current).  Make that first call outside of any
//     stream capture; later calls only enqueue a memset and two kernels on `stream`.
//   * The entry point calls no cudaMalloc / cudaFree and no allocating library routine.
//   * All calls share the one array, which keeps whatever the previous call left in it; each call
//     clears the part it uses before use.  Two calls whose GPU work overlaps in time (different
//     streams, or different host threads on different streams) race on it and must be serialised
//     by the caller.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define MNG_STATIC_SCRATCH_COLS 65536
#define MNG_STATIC_MAX_ROWS (65535LL * 64)

enum {
  MNG_OK = 0,
  MNG_ERR_TOO_LARGE = -22,     // cols > MNG_STATIC_SCRATCH_COLS or rows > MNG_STATIC_MAX_ROWS
  MNG_ERR_SYMBOL = -23,        // the scratch array's device address could not be resolved
  MNG_ERR_BAD_SHAPE = -24,     // rows <= 0 or cols <= 0
  MNG_ERR_LAUNCH = -25,        // memset or kernel launch failed
};

int mng_quant_transpose_e4m3_static(const void* src_bf16, void* q_e4m3, float* scale, long long rows, long long cols,
                                    void* stream);

// Human-readable text for the codes above.
const char* mng_static_strerror(int code);

#ifdef __cplusplus
}
#endif
