// Epilogues of the small-M (decode) GEMM, shared with the host bindings.
// Plain C layout; the kernel takes it as a __grid_constant__ argument.
//
// The decode layer runs as four GEMVs and the attention kernel.  The work
// the reference does in separate kernels between them moves into the GEMVs'
// final stores (patched_sglang_files/python/sglang/srt/models/qwen2.py:
// 170-200 for the layer order, 91-106 for RoPE):
//
//   qkv GEMV      -> LL_EPI_QKV_ROPE: per-head RMSNorm (Qwen3), RoPE, Q to
//                    q_out, K/V to this step's pool slot.  A 128-feature tile
//                    of the qkv product is exactly one head (head_dim 128).
//   o_proj / down -> LL_EPI_RESIDUAL: r = bf16(y) + res; res = bf16(r);
//                    h = bf16(r * norm_w); sumsq_out[m] += sum(r^2).
//
// Row sums of squares are 64-bit fixed point in units of 2^-24
// (LL_SUMSQ_ONE): each output tile adds its part with an integer atomic, and
// integer addition does not depend on the order in which the tiles finish,
// so a decode step gives the same bits every time it runs (a float atomic
// add would not, and greedy decoding of near-tied logits then drifts).
//   gate_up / qkv / lm_head read such an h: with scale_sumsq set, the
//                    accumulator of row m is multiplied by
//                    rsqrt(scale_sumsq[m] / K + scale_eps) before the bias,
//                    which is the RMSNorm of the row applied after the dot
//                    product (W . (r * norm_w) * rstd) instead of before it.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
#include <cuda_bf16.h>
typedef __nv_bfloat16 ll_bf16_t;
#else
typedef uint16_t ll_bf16_t;
#endif

#define LL_SUMSQ_ONE 16777216.0f

enum {
  LL_EPI_STORE = 0,
  LL_EPI_SWIGLU = 1,    // interleaved gate/up (groups of 16) -> silu(gate) * up, N / 2 columns
  LL_EPI_RESIDUAL = 2,
  LL_EPI_QKV_ROPE = 3,
};

struct LLSmallMEpi {
  int mode;
  // row scale (an RMSNorm folded after the product); null: none.
  // Fixed-point sums of squares (units of 1 / LL_SUMSQ_ONE).
  const unsigned long long* scale_sumsq;
  float scale_eps;
  // LL_EPI_RESIDUAL: [M, ld] rows; res is read and written in place
  ll_bf16_t* res;
  const ll_bf16_t* norm_w;
  ll_bf16_t* h_out;
  unsigned long long* sumsq_out;  // [M] fixed point, zeroed before the GEMV
  int ld;
  // LL_EPI_QKV_ROPE
  const int* positions;        // [M]
  const int64_t* slots;        // [M] pool slots (page * page_size + offset)
  const float* cos_sin;        // [max_pos, 128]: cos of the 64 frequencies, then sin
  ll_bf16_t* q_out;            // [M, Hq, 128]
  ll_bf16_t* k_pool;           // this layer's [pages, Hkv, page_size, 128]
  ll_bf16_t* v_pool;
  const ll_bf16_t* q_norm_w;   // [128] or null
  const ll_bf16_t* k_norm_w;
  int Hq, Hkv, page_size;
  float eps;
  int64_t slot_limit;  // slots in this layer's pool (pages * page_size): larger slots are refused
  int max_pos;         // rows of cos_sin: larger positions are refused
};

#ifdef __cplusplus
extern "C" {
#endif
// Small-M GEMM C = A . W^T (+ bias) with an epilogue.  C may be null for the
// residual and qkv epilogues.  w_tiled: W in tile-major layout.
int ll_gemm_bf16_small_m_epi(const void* A, int lda, const void* W, int ldw, void* C, int ldc, const void* bias,
                             int M, int N, int K, int splits, float* ws, size_t ws_floats, int* tickets, int* err,
                             int w_tiled, const struct LLSmallMEpi* epi, void* stream);
#ifdef __cplusplus
}
#endif
