// PyTorch bindings for the sm_100a kernels.  Kernel sources (*.cu) expose
// plain C entry points; this file checks tensors and forwards pointers and
// the current CUDA stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

using bf16 = __nv_bfloat16;

#include "gemm_epi.h"
#include "tp_fused.h"

extern "C" {
int ll_gemm_bf16(const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc, const bf16* bias, int M, int N,
                 int K, int epilogue, int bn, int* err, cudaStream_t stream);
int ll_gemm_bf16_small_m(const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc, const bf16* bias, int M,
                         int N, int K, int splits, float* ws, size_t ws_floats, int* tickets, int* err,
                         cudaStream_t stream);
int ll_gemm_small_m_splits(int N, int K);
int ll_gemm_bf16_small_m_ex(const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc, const bf16* bias,
                            int M, int N, int K, int splits, float* ws, size_t ws_floats, int* tickets, int* err,
                            int flags, cudaStream_t stream);
int ll_rmsnorm(bf16* out, const bf16* x, bf16* residual, const bf16* w, int rows, int hidden, float eps,
               cudaStream_t stream);
int ll_rope_qkv_write(const bf16* qkv, const int* positions, const int64_t* slots, const float* cos_sin, bf16* q_out,
                      bf16* k_pool, bf16* v_pool, const bf16* q_norm_w, const bf16* k_norm_w, int T, int Hq, int Hkv,
                      int head_dim, int page_size, int qkv_ld, float eps, int64_t slot_limit, int max_pos, int* err,
                      cudaStream_t stream);
int ll_kv_link_rope(bf16* dst_k, bf16* dst_v, const bf16* src_k, const bf16* src_v, const int64_t* src_slots,
                    const int64_t* dst_slots, const int* local_pos, const int* global_pos, const float* cos_sin, int n,
                    int num_layers, int Hkv, int head_dim, int src_page_size, int dst_page_size,
                    int64_t src_layer_stride, int64_t dst_layer_stride, int64_t src_slot_limit,
                    int64_t dst_slot_limit, int max_pos, int* err, cudaStream_t stream);
int ll_swiglu(bf16* out, const bf16* gu, int T, int inter, cudaStream_t stream);
int ll_embedding(bf16* out, const int* ids, const bf16* table, int T, int hidden, int vocab_start, int vocab_end,
                 cudaStream_t stream);
int ll_argmax(int* out, const bf16* logits, int rows, int vocab, int ld, cudaStream_t stream);
int ll_attn_prefill(const bf16* q, const bf16* kpool, const bf16* vpool, const int* q_indptr, const int* q_pos,
                    const int* page_table, int pt_stride, const int* tiles, int ntiles, bf16* out, int Hq, int Hkv,
                    int head_dim, int page_size, float scale, cudaStream_t stream);
int ll_attn_decode(const bf16* q, const bf16* kpool, const bf16* vpool, int num_pages, const int* page_table,
                   int pt_stride, const int* kv_lens, bf16* out, float* ws_o, float* ws_ml, int B, int Hq, int Hkv,
                   int head_dim, int page_size, int nsplit, float scale, int* err, cudaStream_t stream);
int ll_attn_prefill_tc(const bf16* q, const bf16* k_pool, const bf16* v_pool, int L, int pages, int layer,
                       const int* q_indptr, const int* q_pos, const int* page_table, int pt_stride, const int* tiles,
                       int ntiles, bf16* out, int Hq, int Hkv, int head_dim, int page_size, float scale, int* err,
                       int nsplit, float* ws_o, float* ws_ml, int combine_rows, cudaStream_t stream);
int ll_attn_prefill_tc_set_variant(int v);
int ll_attn_prefill_tc_trace(unsigned long long* host, int n);
}

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bfloat16")
#define CHECK_I32(x) TORCH_CHECK((x).scalar_type() == at::kInt, #x " must be int32")
#define CHECK_I64(x) TORCH_CHECK((x).scalar_type() == at::kLong, #x " must be int64")
#define CHECK_F32(x) TORCH_CHECK((x).scalar_type() == at::kFloat, #x " must be float32")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_ALIGN16(x) \
  TORCH_CHECK(reinterpret_cast<uintptr_t>((x).data_ptr()) % 16 == 0, #x " must start on a 16-byte boundary")

inline bf16* bp(const at::Tensor& t) { return reinterpret_cast<bf16*>(t.data_ptr()); }
inline bf16* bp_opt(const c10::optional<at::Tensor>& t) { return t.has_value() ? bp(*t) : nullptr; }
inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_rc(int rc, const char* what) { TORCH_CHECK(rc == 0, what, " failed with code ", rc); }

// out[M, N] = a[M, K] @ w[N, K]^T (+ bias).  a/out may be row-strided views.
void gemm(const at::Tensor& a, const at::Tensor& w, const c10::optional<at::Tensor>& bias, at::Tensor& out,
          int64_t epilogue, int64_t bn, const at::Tensor& err) {
  CHECK_CUDA(a); CHECK_BF16(a); CHECK_BF16(w); CHECK_BF16(out); CHECK_CONTIG(w);
  TORCH_CHECK(a.dim() == 2 && w.dim() == 2 && out.dim() == 2);
  TORCH_CHECK(a.stride(1) == 1 && out.stride(1) == 1, "inner dim must be contiguous");
  const int M = a.size(0), K = a.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K);
  if (epilogue == 1) {
    TORCH_CHECK(out.size(1) == N / 2 && out.size(0) == M);
  } else {
    TORCH_CHECK(out.size(1) == N && out.size(0) == M);
  }
  if (bias.has_value()) { CHECK_BF16(*bias); TORCH_CHECK(bias->numel() == N); }
  c10::cuda::CUDAGuard g(a.device());
  check_rc(ll_gemm_bf16(bp(a), a.stride(0), bp(w), w.stride(0), bp(out), out.stride(0), bp_opt(bias), M, N, K,
                        (int)epilogue, (int)bn, err.data_ptr<int>(), cur_stream()),
           "ll_gemm_bf16");
}

// Tensor-parallel GEMM (2-SM kernel): epilogue 0 plain, 1 SwiGLU, 2 scatter
// into the owners' slot buffers.  Pointer lists are device addresses.
void gemm_tp(const at::Tensor& a, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
             const c10::optional<at::Tensor>& out, int64_t epilogue, int64_t N_out_ld, std::vector<int64_t> slot_ptrs,
             std::vector<int64_t> cnt_ptrs, int64_t wait_cnt, int64_t wait_target, int64_t rank, int64_t world,
             int64_t rows_per_rank, const at::Tensor& err) {
  CHECK_CUDA(a); CHECK_BF16(a); CHECK_BF16(w); CHECK_CONTIG(w);
  TORCH_CHECK(a.dim() == 2 && w.dim() == 2 && a.stride(1) == 1);
  const int M = a.size(0), K = a.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K);
  TORCH_CHECK((int64_t)slot_ptrs.size() <= LL_MAX_TP_RANKS && (int64_t)cnt_ptrs.size() <= LL_MAX_TP_RANKS);
  LLTpArgs tp{};
  for (size_t i = 0; i < slot_ptrs.size(); ++i) tp.slot[i] = reinterpret_cast<void*>(slot_ptrs[i]);
  for (size_t i = 0; i < cnt_ptrs.size(); ++i) tp.cnt[i] = reinterpret_cast<unsigned long long*>(cnt_ptrs[i]);
  tp.wait_cnt = reinterpret_cast<const unsigned long long*>(wait_cnt);
  tp.wait_target = (unsigned long long)wait_target;
  tp.rank = (int)rank;
  tp.world = (int)world;
  tp.rows_per_rank = (int)rows_per_rank;
  void* c = nullptr;
  int ldc = (int)N_out_ld;
  if (out.has_value()) {
    CHECK_BF16(*out);
    TORCH_CHECK(out->dim() == 2 && out->stride(1) == 1 && out->size(0) == M);
    TORCH_CHECK(out->size(1) == (epilogue == 1 ? N / 2 : N));
    c = out->data_ptr();
    ldc = out->stride(0);
  }
  if (bias.has_value()) { CHECK_BF16(*bias); TORCH_CHECK(bias->numel() == N); }
  c10::cuda::CUDAGuard g(a.device());
  check_rc(ll_gemm_bf16_tp(a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), c, ldc,
                           bias.has_value() ? bias->data_ptr() : nullptr, M, N, K, (int)epilogue, &tp,
                           err.data_ptr<int>(), cur_stream()),
           "ll_gemm_bf16_tp");
}

// Owner side of the fused TP boundary: sum slots (optional) + residual ->
// residual, RMSNorm -> every rank's gather buffer.  Returns the grid (the
// per-rank increment of every G counter is world x grid).
int64_t tp_reduce_norm_gather(const c10::optional<at::Tensor>& slots, at::Tensor& residual, const at::Tensor& w,
                              double eps, int64_t rows, std::vector<int64_t> g_ptrs, std::vector<int64_t> g_cnt_ptrs,
                              int64_t slot_cnt, int64_t slot_target, int64_t rank, int64_t world,
                              int64_t rows_per_rank, const at::Tensor& err) {
  CHECK_CUDA(residual); CHECK_BF16(residual); CHECK_CONTIG(residual); CHECK_BF16(w);
  TORCH_CHECK((int64_t)g_ptrs.size() == world && (int64_t)g_cnt_ptrs.size() == world && world <= LL_MAX_TP_RANKS);
  const int H = residual.size(1);
  TORCH_CHECK(residual.size(0) >= rows && w.numel() == H);
  if (slots.has_value()) {
    CHECK_BF16(*slots); CHECK_CONTIG(*slots);
    TORCH_CHECK(slots->numel() >= world * rows_per_rank * H);
  }
  LLTpGather tg{};
  for (int i = 0; i < world; ++i) {
    tg.g[i] = reinterpret_cast<void*>(g_ptrs[i]);
    tg.g_cnt[i] = reinterpret_cast<unsigned long long*>(g_cnt_ptrs[i]);
  }
  tg.slot_cnt = reinterpret_cast<const unsigned long long*>(slot_cnt);
  tg.slot_target = (unsigned long long)slot_target;
  tg.rank = (int)rank;
  tg.world = (int)world;
  tg.rows_per_rank = (int)rows_per_rank;
  c10::cuda::CUDAGuard g(residual.device());
  check_rc(ll_tp_reduce_norm_gather(slots.has_value() ? slots->data_ptr() : nullptr, residual.data_ptr(),
                                    w.data_ptr(), (float)eps, H, (int)rows, &tg, err.data_ptr<int>(), cur_stream()),
           "ll_tp_reduce_norm_gather");
  return ll_tp_reduce_norm_gather_grid((int)rows, H);
}

void tp_wait(int64_t cnt, int64_t target, const at::Tensor& err) {
  c10::cuda::CUDAGuard g(err.device());
  check_rc(ll_tp_wait(reinterpret_cast<const void*>(cnt), (unsigned long long)target, err.data_ptr<int>(),
                      cur_stream()),
           "ll_tp_wait");
}

// Decode TP boundary: residual [rows, H] += sum over ranks of part[d] rows;
// out = RMSNorm(residual) * w.  epoch: this rank's int64 [2] (zeroed once).
void tp_decode_allreduce_norm_nvls(at::Tensor& residual, const at::Tensor& w, at::Tensor& out, double eps,
                                   int64_t rows, std::vector<int64_t> part_ptrs, std::vector<int64_t> cnt_ptrs,
                                   at::Tensor& epoch, int64_t rank, int64_t world, const at::Tensor& err,
                                   int64_t mc_ptr) {
  CHECK_CUDA(residual); CHECK_BF16(residual); CHECK_CONTIG(residual); CHECK_BF16(w); CHECK_BF16(out);
  CHECK_CONTIG(out); CHECK_ALIGN16(residual); CHECK_ALIGN16(out); CHECK_ALIGN16(w);
  TORCH_CHECK(epoch.scalar_type() == at::kLong && epoch.numel() >= 2 && epoch.is_cuda());
  TORCH_CHECK((int64_t)part_ptrs.size() == world && (int64_t)cnt_ptrs.size() == world && world <= LL_MAX_TP_RANKS);
  const int H = residual.size(1);
  TORCH_CHECK(residual.size(0) >= rows && out.size(0) >= rows && out.size(1) == H && w.numel() == H);
  LLTpDecode td{};
  for (int i = 0; i < world; ++i) {
    TORCH_CHECK(part_ptrs[i] % 16 == 0, "partial buffer must be 16-byte aligned");
    td.part[i] = reinterpret_cast<const void*>(part_ptrs[i]);
    td.cnt[i] = reinterpret_cast<unsigned long long*>(cnt_ptrs[i]);
  }
  td.epoch = reinterpret_cast<unsigned long long*>(epoch.data_ptr<int64_t>());
  TORCH_CHECK(mc_ptr % 16 == 0, "multicast address must be 16-byte aligned");
  td.mc = reinterpret_cast<const void*>(mc_ptr);
  td.rank = (int)rank;
  td.world = (int)world;
  c10::cuda::CUDAGuard g(residual.device());
  check_rc(ll_tp_decode_allreduce_norm(residual.data_ptr(), w.data_ptr(), out.data_ptr(), (float)eps, H, (int)rows,
                                       &td, err.data_ptr<int>(), cur_stream()),
           "ll_tp_decode_allreduce_norm");
}

void tp_decode_allreduce_norm(at::Tensor& residual, const at::Tensor& w, at::Tensor& out, double eps, int64_t rows,
                              std::vector<int64_t> part_ptrs, std::vector<int64_t> cnt_ptrs, at::Tensor& epoch,
                              int64_t rank, int64_t world, const at::Tensor& err) {
  tp_decode_allreduce_norm_nvls(residual, w, out, eps, rows, std::move(part_ptrs), std::move(cnt_ptrs), epoch, rank,
                                world, err, 0);
}

// Greedy token ids [rows] over vocab-sharded logits [rows, vocab_local]
// (this rank's shard starting at vocab_start): records pushed to every
// rank's slot array (device addresses), epoch this rank's int64 [2].
void tp_argmax(const at::Tensor& logits, int64_t vocab_start, at::Tensor& out, std::vector<int64_t> slot_ptrs,
               at::Tensor& epoch, int64_t rank, int64_t world, int64_t rmax, const at::Tensor& err) {
  CHECK_CUDA(logits); CHECK_BF16(logits); CHECK_I32(out);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && out.is_contiguous() && out.numel() >= logits.size(0));
  TORCH_CHECK(epoch.scalar_type() == at::kLong && epoch.numel() >= 2 && epoch.is_cuda());
  TORCH_CHECK((int64_t)slot_ptrs.size() == world && world <= LL_MAX_TP_RANKS);
  LLTpArgmax ta{};
  for (int i = 0; i < world; ++i) {
    TORCH_CHECK(slot_ptrs[i] % 16 == 0, "argmax slot array must be 16-byte aligned");
    ta.slot[i] = reinterpret_cast<void*>(slot_ptrs[i]);
  }
  ta.epoch = reinterpret_cast<unsigned long long*>(epoch.data_ptr<int64_t>());
  ta.rank = (int)rank;
  ta.world = (int)world;
  ta.rmax = (int)rmax;
  c10::cuda::CUDAGuard g(logits.device());
  check_rc(ll_tp_argmax(logits.data_ptr(), (int)logits.size(1), (int)logits.stride(0), (int)vocab_start,
                        (int)logits.size(0), out.data_ptr<int>(), &ta, err.data_ptr<int>(), cur_stream()),
           "ll_tp_argmax");
}

// swiglu: w is the interleaved gate/up weight and out holds silu(gate) * up
// (N / 2 columns).
void gemm_small_m(const at::Tensor& a, const at::Tensor& w, const c10::optional<at::Tensor>& bias, at::Tensor& out,
                  int64_t splits, at::Tensor& ws, at::Tensor& tickets, const at::Tensor& err, bool swiglu) {
  CHECK_CUDA(a); CHECK_BF16(a); CHECK_BF16(w); CHECK_BF16(out); CHECK_CONTIG(w); CHECK_F32(ws); CHECK_I32(tickets);
  TORCH_CHECK(a.stride(1) == 1 && out.stride(1) == 1);
  // w: [N, K] row-major, or tile-major [N/128, K/64, 128, 64].
  const bool tiled = w.dim() == 4;
  const int M = a.size(0), K = a.size(1);
  const int N = tiled ? (int)(w.size(0) * 128) : (int)w.size(0);
  if (tiled) {
    TORCH_CHECK(w.size(2) == 128 && w.size(3) == 64 && w.size(1) * 64 == K, "bad tile-major weight shape");
  } else {
    TORCH_CHECK(w.size(1) == K);
  }
  TORCH_CHECK(out.size(0) == M && out.size(1) == (swiglu ? N / 2 : N));
  c10::cuda::CUDAGuard g(a.device());
  check_rc(ll_gemm_bf16_small_m_ex(bp(a), a.stride(0), bp(w), tiled ? K : (int)w.stride(0), bp(out), out.stride(0),
                                   bp_opt(bias), M, N, K, (int)splits, ws.data_ptr<float>(), (size_t)ws.numel(),
                                   tickets.data_ptr<int>(), err.data_ptr<int>(), (tiled ? 1 : 0) | (swiglu ? 2 : 0),
                                   cur_stream()),
           "ll_gemm_bf16_small_m");
}

int64_t gemm_small_m_splits(int64_t N, int64_t K) { return ll_gemm_small_m_splits((int)N, (int)K); }

template <typename T>
static T* opt_ptr(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

// Small-M GEMM with a decode-layer epilogue (gemm_epi.h): mode 0 store,
// 1 SwiGLU, 2 residual + norm weight + row sum of squares, 3 qkv heads with
// QK-norm, RoPE and the KV write.  scale_sumsq: rows' sums of squares of an
// unnormalised input (RMSNorm applied after the product).
void gemm_small_m_epi(const at::Tensor& a, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                      const c10::optional<at::Tensor>& out, int64_t splits, at::Tensor& ws, at::Tensor& tickets,
                      const at::Tensor& err, int64_t mode, const c10::optional<at::Tensor>& scale_sumsq,
                      double scale_eps, const c10::optional<at::Tensor>& res, const c10::optional<at::Tensor>& norm_w,
                      const c10::optional<at::Tensor>& h_out, const c10::optional<at::Tensor>& sumsq_out,
                      const c10::optional<at::Tensor>& positions, const c10::optional<at::Tensor>& slots,
                      const c10::optional<at::Tensor>& cos_sin, const c10::optional<at::Tensor>& q_out,
                      const c10::optional<at::Tensor>& k_pool_l, const c10::optional<at::Tensor>& v_pool_l,
                      const c10::optional<at::Tensor>& q_norm_w, const c10::optional<at::Tensor>& k_norm_w,
                      int64_t Hq, int64_t Hkv, int64_t page_size, double eps) {
  CHECK_CUDA(a); CHECK_BF16(a); CHECK_BF16(w); CHECK_CONTIG(w); CHECK_F32(ws); CHECK_I32(tickets);
  TORCH_CHECK(a.stride(1) == 1);
  const bool tiled = w.dim() == 4;
  const int M = a.size(0), K = a.size(1);
  const int N = tiled ? (int)(w.size(0) * 128) : (int)w.size(0);
  if (tiled) {
    TORCH_CHECK(w.size(2) == 128 && w.size(3) == 64 && w.size(1) * 64 == K, "bad tile-major weight shape");
  } else {
    TORCH_CHECK(w.size(1) == K);
  }
  LLSmallMEpi e{};
  e.mode = (int)mode;
  if (scale_sumsq.has_value()) {
    TORCH_CHECK(scale_sumsq->scalar_type() == at::kLong && scale_sumsq->is_contiguous(),
                "scale_sumsq: int64 fixed-point sums of squares");
    TORCH_CHECK(scale_sumsq->numel() >= M);
  }
  e.scale_sumsq = opt_ptr<const unsigned long long>(scale_sumsq);
  e.scale_eps = (float)scale_eps;
  int ldc = 0;
  if (mode == LL_EPI_STORE || mode == LL_EPI_SWIGLU) {
    TORCH_CHECK(out.has_value(), "this epilogue writes `out`");
    CHECK_BF16(*out);
    TORCH_CHECK(out->stride(1) == 1 && out->size(0) == M && out->size(1) == (mode == LL_EPI_SWIGLU ? N / 2 : N));
    ldc = out->stride(0);
  } else if (mode == LL_EPI_RESIDUAL) {
    TORCH_CHECK(res.has_value() && norm_w.has_value() && h_out.has_value() && sumsq_out.has_value());
    CHECK_BF16(*res); CHECK_BF16(*norm_w); CHECK_BF16(*h_out);
    TORCH_CHECK(sumsq_out->scalar_type() == at::kLong && sumsq_out->is_contiguous(),
                "sumsq_out: int64 fixed-point sums of squares");
    TORCH_CHECK(res->size(0) == M && res->size(1) == N && res->stride(1) == 1 && h_out->sizes() == res->sizes() &&
                h_out->strides() == res->strides() && norm_w->numel() == N && sumsq_out->numel() >= M);
    e.res = opt_ptr<ll_bf16_t>(res);
    e.norm_w = opt_ptr<const ll_bf16_t>(norm_w);
    e.h_out = opt_ptr<ll_bf16_t>(h_out);
    e.sumsq_out = opt_ptr<unsigned long long>(sumsq_out);
    e.ld = res->stride(0);
  } else if (mode == LL_EPI_QKV_ROPE) {
    TORCH_CHECK(positions.has_value() && slots.has_value() && cos_sin.has_value() && q_out.has_value() &&
                k_pool_l.has_value() && v_pool_l.has_value());
    CHECK_I32(*positions); CHECK_I64(*slots); CHECK_F32(*cos_sin); CHECK_BF16(*q_out); CHECK_BF16(*k_pool_l);
    CHECK_BF16(*v_pool_l); CHECK_CONTIG(*q_out); CHECK_CONTIG(*k_pool_l); CHECK_CONTIG(*v_pool_l);
    CHECK_CONTIG(*cos_sin);
    TORCH_CHECK(cos_sin->size(-1) == 128 && q_out->numel() >= (int64_t)M * Hq * 128 && positions->numel() >= M &&
                slots->numel() >= M);
    TORCH_CHECK(k_pool_l->size(-1) == 128 && k_pool_l->size(-3) == Hkv && k_pool_l->size(-2) == page_size);
    if (q_norm_w.has_value()) CHECK_BF16(*q_norm_w);
    if (k_norm_w.has_value()) CHECK_BF16(*k_norm_w);
    e.positions = opt_ptr<const int>(positions);
    e.slots = opt_ptr<const int64_t>(slots);
    e.cos_sin = opt_ptr<const float>(cos_sin);
    e.q_out = opt_ptr<ll_bf16_t>(q_out);
    e.k_pool = opt_ptr<ll_bf16_t>(k_pool_l);
    e.v_pool = opt_ptr<ll_bf16_t>(v_pool_l);
    e.q_norm_w = opt_ptr<const ll_bf16_t>(q_norm_w);
    e.k_norm_w = opt_ptr<const ll_bf16_t>(k_norm_w);
    e.Hq = (int)Hq;
    e.Hkv = (int)Hkv;
    e.page_size = (int)page_size;
    e.eps = (float)eps;
    e.slot_limit = k_pool_l->size(0) * page_size;
    e.max_pos = (int)cos_sin->size(0);
  } else {
    TORCH_CHECK(false, "unknown epilogue mode");
  }
  c10::cuda::CUDAGuard g(a.device());
  check_rc(ll_gemm_bf16_small_m_epi(a.data_ptr(), a.stride(0), w.data_ptr(), tiled ? K : (int)w.stride(0),
                                    out.has_value() ? out->data_ptr() : nullptr, ldc,
                                    bias.has_value() ? bias->data_ptr() : nullptr, M, N, K, (int)splits,
                                    ws.data_ptr<float>(), (size_t)ws.numel(), tickets.data_ptr<int>(),
                                    err.data_ptr<int>(), tiled ? 1 : 0, &e, cur_stream()),
           "ll_gemm_bf16_small_m_epi");
}

void rmsnorm(at::Tensor& out, const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w,
             double eps) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(out); CHECK_BF16(w); CHECK_CONTIG(x); CHECK_CONTIG(out);
  const int hidden = x.size(-1);
  const int rows = x.numel() / hidden;
  bf16* res = nullptr;
  if (residual.has_value()) { CHECK_BF16(*residual); CHECK_CONTIG(*residual); res = bp(*residual); }
  c10::cuda::CUDAGuard g(x.device());
  check_rc(ll_rmsnorm(bp(out), bp(x), res, bp(w), rows, hidden, (float)eps, cur_stream()), "ll_rmsnorm");
}

void rope_qkv_write(const at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& slots,
                    const at::Tensor& cos_sin, at::Tensor& q_out, at::Tensor& k_pool_l, at::Tensor& v_pool_l,
                    const c10::optional<at::Tensor>& q_norm_w, const c10::optional<at::Tensor>& k_norm_w,
                    int64_t Hq, int64_t Hkv, int64_t head_dim, double eps, const at::Tensor& err) {
  CHECK_CUDA(qkv); CHECK_BF16(qkv); CHECK_I32(positions); CHECK_I64(slots); CHECK_F32(cos_sin);
  CHECK_BF16(q_out); CHECK_BF16(k_pool_l); CHECK_BF16(v_pool_l); CHECK_I32(err);
  TORCH_CHECK(qkv.stride(1) == 1);
  const int T = qkv.size(0);
  const int ps = k_pool_l.size(2);
  const int64_t slot_limit = k_pool_l.size(0) * ps;  // this layer's pool: [pages, Hkv, ps, D]
  c10::cuda::CUDAGuard g(qkv.device());
  check_rc(ll_rope_qkv_write(bp(qkv), positions.data_ptr<int>(), slots.data_ptr<int64_t>(), cos_sin.data_ptr<float>(),
                             bp(q_out), bp(k_pool_l), bp(v_pool_l), bp_opt(q_norm_w), bp_opt(k_norm_w), T, Hq, Hkv,
                             head_dim, ps, qkv.stride(0), (float)eps, slot_limit, (int)cos_sin.size(0),
                             err.data_ptr<int>(), cur_stream()),
           "ll_rope_qkv_write");
}

// Pools are [L, pages, Hkv, page_size, D].  src pools may be raw peer
// addresses (src_k_ptr/src_v_ptr != 0) for the cross-replica link.
void kv_link_rope(at::Tensor& k_pool, at::Tensor& v_pool, int64_t src_k_ptr, int64_t src_v_ptr,
                  int64_t src_page_size, int64_t src_layer_stride, const at::Tensor& src_slots,
                  const at::Tensor& dst_slots, const at::Tensor& local_pos, const at::Tensor& global_pos,
                  const at::Tensor& cos_sin, const at::Tensor& err) {
  CHECK_CUDA(k_pool); CHECK_BF16(k_pool); CHECK_BF16(v_pool); CHECK_I64(src_slots); CHECK_I64(dst_slots);
  CHECK_I32(local_pos); CHECK_I32(global_pos); CHECK_F32(cos_sin); CHECK_CONTIG(k_pool); CHECK_CONTIG(v_pool);
  CHECK_I32(err);
  const int L = k_pool.size(0), Hkv = k_pool.size(2), ps = k_pool.size(3), D = k_pool.size(4);
  const int n = src_slots.numel();
  const bf16* sk = src_k_ptr ? reinterpret_cast<const bf16*>(src_k_ptr) : bp(k_pool);
  const bf16* sv = src_v_ptr ? reinterpret_cast<const bf16*>(src_v_ptr) : bp(v_pool);
  const int sps = src_k_ptr ? (int)src_page_size : ps;
  const int64_t sls = src_k_ptr ? src_layer_stride : k_pool.stride(0);
  // slots in a pool: one layer's elements / (Hkv * D) = pages * page_size
  const int64_t src_limit = sls / ((int64_t)Hkv * D), dst_limit = k_pool.stride(0) / ((int64_t)Hkv * D);
  c10::cuda::CUDAGuard g(k_pool.device());
  check_rc(ll_kv_link_rope(bp(k_pool), bp(v_pool), sk, sv, src_slots.data_ptr<int64_t>(), dst_slots.data_ptr<int64_t>(),
                           local_pos.data_ptr<int>(), global_pos.data_ptr<int>(), cos_sin.data_ptr<float>(), n, L, Hkv,
                           D, sps, ps, sls, k_pool.stride(0), src_limit, dst_limit, (int)cos_sin.size(0),
                           err.data_ptr<int>(), cur_stream()),
           "ll_kv_link_rope");
}

void swiglu(at::Tensor& out, const at::Tensor& gu) {
  CHECK_CUDA(gu); CHECK_BF16(gu); CHECK_CONTIG(gu); CHECK_CONTIG(out);
  c10::cuda::CUDAGuard g(gu.device());
  check_rc(ll_swiglu(bp(out), bp(gu), gu.size(0), gu.size(1) / 2, cur_stream()), "ll_swiglu");
}

void embedding(at::Tensor& out, const at::Tensor& ids, const at::Tensor& table, int64_t vocab_start) {
  CHECK_CUDA(ids); CHECK_I32(ids); CHECK_BF16(table); CHECK_CONTIG(table); CHECK_CONTIG(out);
  c10::cuda::CUDAGuard g(ids.device());
  check_rc(ll_embedding(bp(out), ids.data_ptr<int>(), bp(table), ids.numel(), table.size(1), (int)vocab_start,
                        (int)(vocab_start + table.size(0)), cur_stream()),
           "ll_embedding");
}

void argmax(at::Tensor& out, const at::Tensor& logits) {
  CHECK_CUDA(logits); CHECK_BF16(logits); CHECK_I32(out);
  TORCH_CHECK(logits.stride(1) == 1);
  c10::cuda::CUDAGuard g(logits.device());
  check_rc(ll_argmax(out.data_ptr<int>(), bp(logits), logits.size(0), logits.size(1), logits.stride(0), cur_stream()),
           "ll_argmax");
}

void attn_prefill(const at::Tensor& q, const at::Tensor& k_pool_l, const at::Tensor& v_pool_l,
                  const at::Tensor& q_indptr, const at::Tensor& q_pos, const at::Tensor& page_table,
                  const at::Tensor& tiles, at::Tensor& out, double scale) {
  CHECK_CUDA(q); CHECK_BF16(q); CHECK_CONTIG(q); CHECK_I32(q_indptr); CHECK_I32(q_pos); CHECK_I32(page_table);
  CHECK_I32(tiles); CHECK_CONTIG(tiles); CHECK_ALIGN16(tiles); CHECK_CONTIG(out);
  const int Hq = q.size(1), D = q.size(2);
  const int Hkv = k_pool_l.size(1), ps = k_pool_l.size(2);
  c10::cuda::CUDAGuard g(q.device());
  check_rc(ll_attn_prefill(bp(q), bp(k_pool_l), bp(v_pool_l), q_indptr.data_ptr<int>(), q_pos.data_ptr<int>(),
                           page_table.data_ptr<int>(), page_table.stride(0), tiles.data_ptr<int>(), tiles.size(0),
                           bp(out), Hq, Hkv, D, ps, (float)scale, cur_stream()),
           "ll_attn_prefill");
}

// k_pool / v_pool: whole pools [L, pages, Hkv, ps, D]; `layer` selects one.
void attn_prefill_tc(const at::Tensor& q, const at::Tensor& k_pool, const at::Tensor& v_pool, int64_t layer,
                     const at::Tensor& q_indptr, const at::Tensor& q_pos, const at::Tensor& page_table,
                     const at::Tensor& tiles, at::Tensor& out, double scale, const at::Tensor& err, int64_t nsplit,
                     const c10::optional<at::Tensor>& ws_o, const c10::optional<at::Tensor>& ws_ml) {
  CHECK_CUDA(q); CHECK_BF16(q); CHECK_CONTIG(q); CHECK_BF16(k_pool); CHECK_BF16(v_pool); CHECK_CONTIG(k_pool);
  CHECK_CONTIG(v_pool); CHECK_I32(q_indptr); CHECK_I32(q_pos); CHECK_I32(page_table); CHECK_I32(tiles);
  CHECK_CONTIG(tiles); CHECK_ALIGN16(tiles); CHECK_CONTIG(out);
  TORCH_CHECK(k_pool.dim() == 5 && k_pool.sizes() == v_pool.sizes());
  TORCH_CHECK(layer >= 0 && layer < k_pool.size(0));
  const int T = q.size(0), Hq = q.size(1), D = q.size(2);
  float* wo = nullptr;
  float* wml = nullptr;
  if (nsplit > 1) {
    TORCH_CHECK(ws_o.has_value() && ws_ml.has_value(), "split attention needs its workspaces");
    TORCH_CHECK(ws_o->scalar_type() == at::kFloat && ws_ml->scalar_type() == at::kFloat);
    TORCH_CHECK(ws_o->is_contiguous() && ws_ml->is_contiguous());
    TORCH_CHECK(ws_o->numel() >= (int64_t)T * Hq * nsplit * D && ws_ml->numel() >= (int64_t)T * Hq * nsplit * 2,
                "split attention workspace too small");
    wo = ws_o->data_ptr<float>();
    wml = ws_ml->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(q.device());
  check_rc(ll_attn_prefill_tc(bp(q), bp(k_pool), bp(v_pool), k_pool.size(0), k_pool.size(1), (int)layer,
                              q_indptr.data_ptr<int>(), q_pos.data_ptr<int>(), page_table.data_ptr<int>(),
                              page_table.stride(0), tiles.data_ptr<int>(), tiles.size(0), bp(out), Hq,
                              k_pool.size(2), D, k_pool.size(3), (float)scale, err.data_ptr<int>(), (int)nsplit, wo,
                              wml, T * Hq, cur_stream()),
           "ll_attn_prefill_tc");
}

void attn_decode(const at::Tensor& q, const at::Tensor& k_pool_l, const at::Tensor& v_pool_l,
                 const at::Tensor& page_table, const at::Tensor& kv_lens, at::Tensor& out, at::Tensor& ws_o,
                 at::Tensor& ws_ml, int64_t nsplit, double scale, const at::Tensor& err) {
  CHECK_CUDA(q); CHECK_BF16(q); CHECK_CONTIG(q); CHECK_I32(page_table); CHECK_I32(kv_lens); CHECK_CONTIG(out);
  const int B = q.size(0), Hq = q.size(1), D = q.size(2);
  const int Hkv = k_pool_l.size(1), ps = k_pool_l.size(2);
  if (nsplit > 1) {
    TORCH_CHECK(ws_o.numel() >= (int64_t)B * Hq * nsplit * D && ws_ml.numel() >= (int64_t)B * Hq * nsplit * 2,
                "decode workspace too small");
  }
  c10::cuda::CUDAGuard g(q.device());
  TORCH_CHECK(k_pool_l.is_contiguous() && v_pool_l.is_contiguous() && k_pool_l.sizes() == v_pool_l.sizes());
  check_rc(ll_attn_decode(bp(q), bp(k_pool_l), bp(v_pool_l), (int)k_pool_l.size(0), page_table.data_ptr<int>(),
                          page_table.stride(0), kv_lens.data_ptr<int>(), bp(out), ws_o.data_ptr<float>(),
                          ws_ml.data_ptr<float>(), B, Hq, Hkv, D, ps, (int)nsplit, (float)scale,
                          err.data_ptr<int>(), cur_stream()),
           "ll_attn_decode");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels for the LegoLink B200 runtime";
  m.def("gemm", &gemm);
  m.def("gemm_small_m", &gemm_small_m);
  m.def("gemm_small_m_splits", &gemm_small_m_splits);
  m.def("gemm_small_m_epi", &gemm_small_m_epi);
  m.def("rmsnorm", &rmsnorm);
  m.def("rope_qkv_write", &rope_qkv_write);
  m.def("kv_link_rope", &kv_link_rope);
  m.def("swiglu", &swiglu);
  m.def("embedding", &embedding);
  m.def("argmax", &argmax);
  m.def("attn_prefill", &attn_prefill);
  m.def("attn_decode", &attn_decode);
  m.def("attn_prefill_tc", &attn_prefill_tc);
  m.def("gemm_tp", &gemm_tp);
  m.def("tp_reduce_norm_gather", &tp_reduce_norm_gather);
  m.def("tp_wait", &tp_wait);
  m.def("tp_decode_allreduce_norm", &tp_decode_allreduce_norm);
  m.def("tp_argmax", &tp_argmax);
  m.def("tp_decode_allreduce_norm_nvls", &tp_decode_allreduce_norm_nvls);
  m.def("attn_prefill_tc_set_variant", [](int64_t v) { return ll_attn_prefill_tc_set_variant((int)v); });
  m.def("attn_prefill_tc_trace", []() {
    auto t = at::zeros({256 * 20}, at::kLong);
    const int n = ll_attn_prefill_tc_trace(reinterpret_cast<unsigned long long*>(t.data_ptr<int64_t>()), 256 * 20);
    TORCH_CHECK(n > 0, "trace copy failed");
    return t.view({256, 20});
  });
}
