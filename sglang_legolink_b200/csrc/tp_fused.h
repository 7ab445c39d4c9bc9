// Kernel arguments of the fused tensor-parallel path (gemm_tcgen05.cu,
// tp_fused.cu), shared with the host bindings.  Plain C layout.
#pragma once

#define LL_MAX_TP_RANKS 8

// 2-SM GEMM hooks.  wait_cnt != nullptr: the producer waits until
// *wait_cnt >= wait_target before loading A.  Scatter epilogue: row r goes to
// rank d = r / rows_per_rank's slot buffer `slot[d]`, into the region of the
// storing rank, which is tiled as [R/32][N/32] tiles of 32 rows x 32 columns
// (2 KB each, row-major inside); each 32-row x 256-column slice it stored
// adds 1 to `cnt[d]` (published at the end of the GEMM).
struct LLTpArgs {
  void* slot[LL_MAX_TP_RANKS];
  unsigned long long* cnt[LL_MAX_TP_RANKS];
  const unsigned long long* wait_cnt;
  unsigned long long wait_target;
  int rank, world, rows_per_rank;
};

// Reduce + RMSNorm + all-gather: g[d] / g_cnt[d] are rank d's gather buffer
// and counter; slot_cnt / slot_target gate the read of this rank's slots.
struct LLTpGather {
  void* g[LL_MAX_TP_RANKS];
  unsigned long long* g_cnt[LL_MAX_TP_RANKS];
  const unsigned long long* slot_cnt;
  unsigned long long slot_target;
  int rank, world, rows_per_rank;
};

// Decode boundary (one-shot all-reduce + residual + RMSNorm): part[d] is
// rank d's partial rows of this call, cnt[d] rank d's arrival counter, epoch
// this rank's [calls completed, CTA ticket] (device memory, so a CUDA graph
// replays the boundary unchanged).
// mc != nullptr: the multicast (NVLS) address of this call's partial rows
// in every rank's buffer; each element's sum over the ranks is then one
// multimem load reduced in the NVLink switch instead of `world` peer loads.
struct LLTpDecode {
  const void* part[LL_MAX_TP_RANKS];
  unsigned long long* cnt[LL_MAX_TP_RANKS];
  unsigned long long* epoch;
  const void* mc;
  int rank, world;
};

// Greedy token over vocab-sharded logits: slot[d] is rank d's record array
// [2 parities][rmax rows][LL_MAX_TP_RANKS source ranks] of LLTpArgmaxRec;
// epoch this rank's [calls completed, CTA ticket] (device memory).
struct LLTpArgmax {
  void* slot[LL_MAX_TP_RANKS];
  unsigned long long* epoch;
  int rank, world, rmax;
};

// One source rank's (max, global index) for one row, tagged with the call's
// epoch; the tag is stored after the pair with release semantics.
struct LLTpArgmaxRec {
  unsigned long long pair;  // float bits of the max << 32 | global index
  unsigned long long tag;
};

#ifdef __cplusplus
extern "C" {
#endif
int ll_tp_argmax(const void* logits, int vocab_local, int ld, int vocab_start, int rows, int* out,
                 const struct LLTpArgmax* ta, int* err, void* stream);
int ll_gemm_bf16_tp(const void* A, int lda, const void* W, int ldw, void* C, int ldc, const void* bias, int M, int N,
                    int K, int epilogue, const struct LLTpArgs* tp, int* err, void* stream);
int ll_tp_reduce_norm_gather(const void* slots, void* residual, const void* w, float eps, int H, int rows,
                             const struct LLTpGather* tg, int* err, void* stream);
int ll_tp_reduce_norm_gather_grid(int rows, int H);
int ll_tp_wait(const void* cnt, unsigned long long target, int* err, void* stream);
int ll_tp_decode_allreduce_norm(void* residual, const void* w, void* out, float eps, int H, int rows,
                                const struct LLTpDecode* td, int* err, void* stream);
#ifdef __cplusplus
}
#endif
