// Allocation-free entry point of the small-M (decode) bf16 GEMM.
//
// This entry point has no counterpart in the reference; it exists for callers
// of this library that cannot allocate device memory themselves: code that
// runs where cudaMalloc is not allowed or not wanted (a host framework that
// owns every allocation through its own pool, a plugin loaded into a process
// whose allocator must not be bypassed, a real-time path that may not enter
// the driver's allocator).  The regular entry point needs a caller-allocated
// fp32 split-K workspace and a ticket array; this one uses scratch compiled
// into the library instead.
//
//   C[M, N] = A[M, K] . W[N, K]^T (+ bias[N]),  bf16 in / out, fp32 accumulate,
//   1 <= M <= 128.
//
// Scratch: a file-scope device array of LL_NOALLOC_WS_FLOATS floats (4 MiB)
// for split-K partial sums and LL_NOALLOC_TICKETS ints for the split-K tickets.
// A call whose split-K partials (splits * M * N floats) or tile count
// (ceil(N / 128)) exceed them is rejected with LL_NOALLOC_E_TOO_LARGE before
// anything is launched; ll_gemm_small_m_noalloc_error_string() names it.
//
// The first call on each device does a one-time set-up: it looks up the device
// address of the scratch (cudaGetSymbolAddress, with that device current) and
// caches it.  Under CUDA's default lazy module loading that lookup is also what
// loads this file's module onto the device, and with it the static scratch: a
// one-time allocation made by the driver, not by this code.  A caller that may
// not enter the allocator at all should therefore make one call per device
// during its initialisation, before any stream capture; the device then holds
// the scratch until the process exits.  Every later call allocates nothing: no
// cudaMalloc, cudaFree or allocating library routine; the tickets it uses are
// cleared with cudaMemsetAsync on the caller's stream before the launch.
//
// All calls on a device share one scratch array, which keeps the contents of
// the last call.  Calls whose executions overlap on the GPU (different
// streams without ordering between them) race on it and give wrong results;
// serialize them on one stream or order them with events.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

#define LL_NOALLOC_WS_FLOATS (1u << 20)
#define LL_NOALLOC_TICKETS 4096

#define LL_NOALLOC_OK 0
#define LL_NOALLOC_E_TOO_LARGE (-8)
#define LL_NOALLOC_E_SYMBOL (-9)

#ifdef __cplusplus
extern "C" {
#endif

// Returns 0 on success or a negative code; `err` (may be NULL) receives the
// device-side timeout code of the kernel's bounded waits, as for the regular
// entry point.
int ll_gemm_bf16_small_m_noalloc(const __nv_bfloat16* A, int lda, const __nv_bfloat16* W, int ldw,
                                 __nv_bfloat16* C, int ldc, const __nv_bfloat16* bias, int M, int N, int K,
                                 int* err, cudaStream_t stream);

const char* ll_gemm_small_m_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
