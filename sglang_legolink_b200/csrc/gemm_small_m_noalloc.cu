// Allocation-free variant of the small-M GEMM entry point; see
// gemm_small_m_noalloc.h for who needs it and the rules that come with it.
// It has no counterpart in the reference.  The GEMM itself is the unchanged
// ll_gemm_bf16_small_m (gemm_tcgen05.cu); only where its scratch lives differs.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "gemm_small_m_noalloc.h"

using bf16 = __nv_bfloat16;

extern "C" int ll_gemm_bf16_small_m(const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc,
                                    const bf16* bias, int M, int N, int K, int splits, float* ws, size_t ws_floats,
                                    int* tickets, int* err, cudaStream_t stream);
extern "C" int ll_gemm_small_m_splits(int N, int K);

// The scratch itself.  In host code these names are host-side stand-ins, not
// device addresses: only the addresses looked up below may be passed to a kernel.
static __device__ __align__(256) float g_noalloc_ws[LL_NOALLOC_WS_FLOATS];
static __device__ __align__(256) int g_noalloc_tickets[LL_NOALLOC_TICKETS];

namespace {

constexpr int kMaxDevices = 64;

struct ScratchAddrs {
  float* ws = nullptr;
  int* tickets = nullptr;
};

std::mutex g_mu;
ScratchAddrs g_addrs[kMaxDevices];

// Looks up (once per device, with that device current) the device addresses
// of the scratch arrays.
int scratch_for_current_device(ScratchAddrs* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return LL_NOALLOC_E_SYMBOL;
  std::lock_guard<std::mutex> lock(g_mu);
  ScratchAddrs& a = g_addrs[dev];
  if (a.ws == nullptr || a.tickets == nullptr) {
    void* ws = nullptr;
    void* tk = nullptr;
    if (cudaGetSymbolAddress(&ws, g_noalloc_ws) != cudaSuccess) return LL_NOALLOC_E_SYMBOL;
    if (cudaGetSymbolAddress(&tk, g_noalloc_tickets) != cudaSuccess) return LL_NOALLOC_E_SYMBOL;
    a.ws = static_cast<float*>(ws);
    a.tickets = static_cast<int*>(tk);
  }
  *out = a;
  return LL_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) const char* ll_gemm_small_m_noalloc_error_string(int code) {
  switch (code) {
    case LL_NOALLOC_OK: return "ok";
    case LL_NOALLOC_E_TOO_LARGE:
      return "problem too large for the library's static scratch (split-K partials above 1048576 floats or "
             "more than 4096 output tiles of 128 columns); use ll_gemm_bf16_small_m with caller-provided scratch";
    case LL_NOALLOC_E_SYMBOL: return "could not resolve the device address of the static scratch";
    case -3: return "unsupported shape (M must be 1..128; K, lda and ldw multiples of 8)";
    default: return "launch or tensor-map failure (see ll_gemm_bf16_small_m return codes)";
  }
}

extern "C" __attribute__((visibility("default"))) int ll_gemm_bf16_small_m_noalloc(
    const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc, const bf16* bias, int M, int N, int K,
    int* err, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return LL_NOALLOC_OK;
  if (M > 128) return -3;
  const int splits = ll_gemm_small_m_splits(N, K);
  const long long tiles = (N + 127) / 128;
  const long long need = splits > 1 ? (long long)splits * M * N : 0;
  if (need > (long long)LL_NOALLOC_WS_FLOATS || tiles > LL_NOALLOC_TICKETS) return LL_NOALLOC_E_TOO_LARGE;
  ScratchAddrs s;
  const int rc = scratch_for_current_device(&s);
  if (rc != LL_NOALLOC_OK) return rc;
  if (splits > 1) {
    // Tickets must start at zero; the array keeps whatever the last call left.
    if (cudaMemsetAsync(s.tickets, 0, sizeof(int) * tiles, stream) != cudaSuccess) return -5;
  }
  return ll_gemm_bf16_small_m(A, lda, W, ldw, C, ldc, bias, M, N, K, splits, s.ws, (size_t)LL_NOALLOC_WS_FLOATS,
                              s.tickets, err, stream);
}
