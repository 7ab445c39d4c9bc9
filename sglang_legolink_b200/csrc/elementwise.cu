// Memory-bound kernels: RMSNorm (+ fused residual add), QKV split + per-head
// RMSNorm (Qwen3) + RoPE + paged KV write, the LegoLink KV link with RoPE
// delta rotation, SwiGLU, embedding gather and greedy argmax.
//
// Reference counterparts: sgl-kernel norms / activation / rope used by
// patched_sglang_files/python/sglang/srt/models/qwen2.py:91-106,170-200,257-288;
// the fused KV link kernel legolink_triton.py:302-547 and its torch path
// pic_runtime.py:5533-5598 / 6025-6057.
#include <cuda_runtime.h>

#include "common.cuh"

namespace ll {

// ----------------------------------------------------------------- RMSNorm
// One CTA per row; each thread keeps VPT 16-byte vectors in registers.
template <int VPT, bool ADD>
__global__ void __launch_bounds__(256) rmsnorm_kernel(bf16* __restrict__ out, const bf16* __restrict__ x,
                                                      bf16* __restrict__ residual, const bf16* __restrict__ w,
                                                      int hidden, float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int nvec = hidden / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * hidden);
  uint4* rr = reinterpret_cast<uint4*>(residual + (size_t)row * hidden);
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < nvec) {
      uint4 a = xr[idx];
      const uint32_t* au = reinterpret_cast<const uint32_t*>(&a);
      if constexpr (ADD) {
        uint4 b = rr[idx];
        const uint32_t* bu = reinterpret_cast<const uint32_t*>(&b);
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 fa = unpack_bf16x2(au[j]), fb = unpack_bf16x2(bu[j]);
          v[i][2 * j] = fa.x + fb.x;
          v[i][2 * j + 1] = fa.y + fb.y;
          o[j] = pack_bf16x2(v[i][2 * j], v[i][2 * j + 1]);
        }
        rr[idx] = make_uint4(o[0], o[1], o[2], o[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 fa = unpack_bf16x2(au[j]);
          v[i][2 * j] = fa.x;
          v[i][2 * j + 1] = fa.y;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)hidden + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * hidden);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < nvec) {
      uint4 wv = wr[idx];
      const uint32_t* wu = reinterpret_cast<const uint32_t*>(&wv);
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 fw = unpack_bf16x2(wu[j]);
        o[j] = pack_bf16x2(v[i][2 * j] * inv * fw.x, v[i][2 * j + 1] * inv * fw.y);
      }
      orow[idx] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ------------------------------------------------- QKV split + RoPE + KV write
// One CTA per token.  Warp k handles heads k, k+nwarps, ... over the list
// [Hq query heads | Hkv key heads | Hkv value heads].  Lane l holds elements
// {l, l+32} of the first rotary half and {l+64, l+96} of the second half
// (head_dim 128), so each rotate-half pair is lane-local.
// Pool layout: [pages, Hkv, page_size, D] for this layer.
__global__ void __launch_bounds__(256) rope_qkv_write_kernel(
    const bf16* __restrict__ qkv, const int* __restrict__ positions, const int64_t* __restrict__ slots,
    const float* __restrict__ cos_sin, bf16* __restrict__ q_out, bf16* __restrict__ k_pool,
    bf16* __restrict__ v_pool, const bf16* __restrict__ q_norm_w, const bf16* __restrict__ k_norm_w, int Hq,
    int Hkv, int page_size, int qkv_ld, float eps, int64_t slot_limit, int max_pos, int* err) {
  constexpr int D = 128;
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int pos = positions[t];
  const int64_t slot = slots[t];
  if (slot < 0 || slot >= slot_limit || pos < 0 || pos >= max_pos) {  // checked, recorded, skipped
    if (threadIdx.x == 0) record_error(err, kErrBadIndex);
    return;
  }
  const int64_t page = slot / page_size, off = slot % page_size;
  const float* cs = cos_sin + (size_t)pos * D;
  const float c0 = cs[lane], c1 = cs[lane + 32];
  const float s0 = cs[64 + lane], s1 = cs[64 + lane + 32];
  const bf16* row = qkv + (size_t)t * qkv_ld;
  for (int h = warp; h < Hq + 2 * Hkv; h += nw) {
    const bf16* src = row + h * D;
    float a0 = __bfloat162float(src[lane]), a1 = __bfloat162float(src[lane + 32]);
    float b0 = __bfloat162float(src[lane + 64]), b1 = __bfloat162float(src[lane + 96]);
    bf16* dst;
    if (h < Hq + Hkv) {
      const bf16* nw_ = (h < Hq) ? q_norm_w : k_norm_w;
      if (nw_ != nullptr) {
        float ss = warp_sum(a0 * a0 + a1 * a1 + b0 * b0 + b1 * b1);
        float inv = rsqrtf(ss / (float)D + eps);
        a0 = a0 * inv * __bfloat162float(nw_[lane]);
        a1 = a1 * inv * __bfloat162float(nw_[lane + 32]);
        b0 = b0 * inv * __bfloat162float(nw_[lane + 64]);
        b1 = b1 * inv * __bfloat162float(nw_[lane + 96]);
      }
      const float r_a0 = a0 * c0 - b0 * s0, r_b0 = b0 * c0 + a0 * s0;
      const float r_a1 = a1 * c1 - b1 * s1, r_b1 = b1 * c1 + a1 * s1;
      a0 = r_a0; b0 = r_b0; a1 = r_a1; b1 = r_b1;
      if (h < Hq) {
        dst = q_out + ((size_t)t * Hq + h) * D;
      } else {
        dst = k_pool + (((size_t)page * Hkv + (h - Hq)) * page_size + off) * D;
      }
    } else {
      dst = v_pool + (((size_t)page * Hkv + (h - Hq - Hkv)) * page_size + off) * D;
    }
    dst[lane] = __float2bfloat16(a0);
    dst[lane + 32] = __float2bfloat16(a1);
    dst[lane + 64] = __float2bfloat16(b0);
    dst[lane + 96] = __float2bfloat16(b1);
  }
}

// ------------------------------------------------------- KV link + RoPE remap
// One warp per linked token, looping over all layers.  8 lanes per KV head:
// lane j of a group loads elements [8j, 8j+8) and [64+8j, 64+8j+8) so both
// members of every rotate-half pair are in the same thread, as 2 x 16-byte
// loads for K and 2 for V.  The delta rotation
//   dc = gc*lc + gs*ls,  ds = gs*lc - gc*ls
// is computed once per token (fp32, __fmul_rn/__fadd_rn: no contraction, the
// same rounding points as the fp32 statement) and applied to K in fp32 with a
// single rounding to bf16.  Tokens with local == global position are copied.
// src_k/src_v may point at a peer GPU's pool (cross-replica link).
__global__ void __launch_bounds__(256) kv_link_rope_kernel(
    bf16* __restrict__ dst_k, bf16* __restrict__ dst_v, const bf16* __restrict__ src_k,
    const bf16* __restrict__ src_v, const int64_t* __restrict__ src_slots, const int64_t* __restrict__ dst_slots,
    const int* __restrict__ local_pos, const int* __restrict__ global_pos, const float* __restrict__ cos_sin,
    int n, int num_layers, int Hkv, int src_page_size, int dst_page_size, int64_t src_layer_stride,
    int64_t dst_layer_stride, int64_t src_slot_limit, int64_t dst_slot_limit, int max_pos, int* err,
    int layer_groups) {
  constexpr int D = 128;
  // warp -> (token, group of layers): few tokens spread their layers over
  // several warps so that the dependent per-layer round trips overlap
  const int64_t gwl = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gwl >= (int64_t)n * layer_groups) return;
  const int gw = (int)(gwl / layer_groups), lgrp = (int)(gwl % layer_groups);
  const int lpg = (num_layers + layer_groups - 1) / layer_groups;
  const int layer0 = lgrp * lpg, layer1 = min(num_layers, layer0 + lpg);
  const int j = lane & 7;         // chunk within the head
  const int hsub = lane >> 3;     // 0..3: head offset within this pass
  const int lp = local_pos[gw], gp = global_pos[gw];
  {
    const int64_t s0 = src_slots[gw], d0 = dst_slots[gw];
    if (s0 < 0 || s0 >= src_slot_limit || d0 < 0 || d0 >= dst_slot_limit || lp < 0 || lp >= max_pos || gp < 0 ||
        gp >= max_pos) {  // checked, recorded, skipped (the whole row, every layer)
      if (lane == 0 && lgrp == 0) record_error(err, kErrBadIndex);
      return;
    }
  }
  const bool same = (lp == gp);
  float dc[8], ds[8];
  if (!same) {
    const float* lcs = cos_sin + (size_t)lp * D;
    const float* gcs = cos_sin + (size_t)gp * D;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int f = 8 * j + e;
      const float lc = lcs[f], ls = lcs[64 + f], gc = gcs[f], gs = gcs[64 + f];
      dc[e] = __fadd_rn(__fmul_rn(gc, lc), __fmul_rn(gs, ls));
      ds[e] = __fsub_rn(__fmul_rn(gs, lc), __fmul_rn(gc, ls));
    }
  }
  const int64_t ss = src_slots[gw], dsl = dst_slots[gw];
  const int64_t sp = ss / src_page_size, so = ss % src_page_size;
  const int64_t dp = dsl / dst_page_size, dof = dsl % dst_page_size;
  for (int layer = layer0; layer < layer1; ++layer) {
    for (int h0 = 0; h0 < Hkv; h0 += 4) {
      const int h = h0 + hsub;
      if (h >= Hkv) continue;
      const size_t soff = (size_t)layer * src_layer_stride + (((size_t)sp * Hkv + h) * src_page_size + so) * D;
      const size_t doff = (size_t)layer * dst_layer_stride + (((size_t)dp * Hkv + h) * dst_page_size + dof) * D;
      const uint4 ka = *reinterpret_cast<const uint4*>(src_k + soff + 8 * j);
      const uint4 kb = *reinterpret_cast<const uint4*>(src_k + soff + 64 + 8 * j);
      const uint4 va = *reinterpret_cast<const uint4*>(src_v + soff + 8 * j);
      const uint4 vb = *reinterpret_cast<const uint4*>(src_v + soff + 64 + 8 * j);
      uint4 oa = ka, ob = kb;
      if (!same) {
        const uint32_t* au = reinterpret_cast<const uint32_t*>(&ka);
        const uint32_t* bu = reinterpret_cast<const uint32_t*>(&kb);
        uint32_t* oau = reinterpret_cast<uint32_t*>(&oa);
        uint32_t* obu = reinterpret_cast<uint32_t*>(&ob);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 x1 = unpack_bf16x2(au[e]), x2 = unpack_bf16x2(bu[e]);
          const float c_0 = dc[2 * e], c_1 = dc[2 * e + 1], s_0 = ds[2 * e], s_1 = ds[2 * e + 1];
          const float o1x = __fsub_rn(__fmul_rn(x1.x, c_0), __fmul_rn(x2.x, s_0));
          const float o1y = __fsub_rn(__fmul_rn(x1.y, c_1), __fmul_rn(x2.y, s_1));
          const float o2x = __fadd_rn(__fmul_rn(x2.x, c_0), __fmul_rn(x1.x, s_0));
          const float o2y = __fadd_rn(__fmul_rn(x2.y, c_1), __fmul_rn(x1.y, s_1));
          oau[e] = pack_bf16x2(o1x, o1y);
          obu[e] = pack_bf16x2(o2x, o2y);
        }
      }
      *reinterpret_cast<uint4*>(dst_k + doff + 8 * j) = oa;
      *reinterpret_cast<uint4*>(dst_k + doff + 64 + 8 * j) = ob;
      *reinterpret_cast<uint4*>(dst_v + doff + 8 * j) = va;
      *reinterpret_cast<uint4*>(dst_v + doff + 64 + 8 * j) = vb;
    }
  }
}

// ------------------------------------------------------------------ SwiGLU
// gu rows are [2*inter] interleaved in groups of 16: columns [32j, 32j+16)
// are gate features [16j, 16j+16) and [32j+16, 32j+32) the matching up
// features.  out[t, 16j+i] = silu(gate) * up.
__global__ void swiglu_kernel(bf16* __restrict__ out, const bf16* __restrict__ gu, int T, int inter) {
  pdl_trigger();
  pdl_wait();
  const size_t nvec = (size_t)T * inter / 8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nvec; i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = (i * 8) / inter, c = (i * 8) % inter;
    const size_t gcol = (c / 16) * 32 + (c % 16);
    const uint4 g = *reinterpret_cast<const uint4*>(gu + t * 2 * inter + gcol);
    const uint4 u = *reinterpret_cast<const uint4*>(gu + t * 2 * inter + gcol + 16);
    const uint32_t* gp = reinterpret_cast<const uint32_t*>(&g);
    const uint32_t* up = reinterpret_cast<const uint32_t*>(&u);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = unpack_bf16x2(gp[j]), b = unpack_bf16x2(up[j]);
      o[j] = pack_bf16x2(a.x / (1.f + __expf(-a.x)) * b.x, a.y / (1.f + __expf(-a.y)) * b.y);
    }
    *reinterpret_cast<uint4*>(out + t * inter + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// --------------------------------------------------------------- embedding
__global__ void embedding_kernel(bf16* __restrict__ out, const int* __restrict__ ids, const bf16* __restrict__ table,
                                 int hidden, int vocab_start, int vocab_end) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int id = ids[t];
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)t * hidden);
  const bool mine = id >= vocab_start && id < vocab_end;
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)(mine ? id - vocab_start : 0) * hidden);
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) o[i] = mine ? src[i] : make_uint4(0, 0, 0, 0);
}

// ------------------------------------------------------------------ argmax
// One CTA per row; ties resolve to the smallest index (torch.argmax order).
__global__ void __launch_bounds__(1024) argmax_kernel(int* __restrict__ out, const bf16* __restrict__ logits,
                                                      int vocab, int ld) {
  pdl_trigger();
  pdl_wait();
  const bf16* row = logits + (size_t)blockIdx.x * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  // 16-byte loads (8 logits) with several in flight per thread; each thread
  // visits its indices in increasing order, so a strict '>' keeps the first.
  const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  const int nvec = vec ? vocab / 8 : 0;
  const uint4* rv = reinterpret_cast<const uint4*>(row);
#pragma unroll 4
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    const uint4 x = __ldg(rv + v);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&x);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(u[j]);
      if (f.x > best) { best = f.x; bi = 8 * v + 2 * j; }
      if (f.y > best) { best = f.y; bi = 8 * v + 2 * j + 1; }
    }
  }
  for (int i = nvec * 8 + threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = __bfloat162float(row[i]);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    best = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) out[blockIdx.x] = bi;
  }
}

}  // namespace ll

using namespace ll;

extern "C" int ll_rmsnorm(bf16* out, const bf16* x, bf16* residual, const bf16* w, int rows, int hidden, float eps,
                          cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (hidden % 8) return -3;
  const int nvec = hidden / 8;
  const int threads = 256;
  const int vpt = (nvec + threads - 1) / threads;
#define LL_RMS(V)                                                                                           \
  do {                                                                                                      \
    if (residual)                                                                                           \
      launch_pdl(rmsnorm_kernel<V, true>, dim3(rows), dim3(threads), 0, stream, out, x, residual, w, hidden, \
                 eps);                                                                                      \
    else                                                                                                    \
      launch_pdl(rmsnorm_kernel<V, false>, dim3(rows), dim3(threads), 0, stream, out, x, residual, w,       \
                 hidden, eps);                                                                              \
  } while (0)
  if (vpt <= 1) LL_RMS(1);
  else if (vpt <= 2) LL_RMS(2);
  else if (vpt <= 4) LL_RMS(4);
  else if (vpt <= 8) LL_RMS(8);
  else return -3;
#undef LL_RMS
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

extern "C" int ll_rope_qkv_write(const bf16* qkv, const int* positions, const int64_t* slots, const float* cos_sin,
                                 bf16* q_out, bf16* k_pool, bf16* v_pool, const bf16* q_norm_w, const bf16* k_norm_w,
                                 int T, int Hq, int Hkv, int head_dim, int page_size, int qkv_ld, float eps,
                                 int64_t slot_limit, int max_pos, int* err, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (head_dim != 128) return -3;
  launch_pdl(rope_qkv_write_kernel, dim3(T), dim3(256), 0, stream, qkv, positions, slots, cos_sin, q_out, k_pool,
             v_pool, q_norm_w, k_norm_w, Hq, Hkv, page_size, qkv_ld, eps, slot_limit, max_pos, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

extern "C" int ll_kv_link_rope(bf16* dst_k, bf16* dst_v, const bf16* src_k, const bf16* src_v,
                               const int64_t* src_slots, const int64_t* dst_slots, const int* local_pos,
                               const int* global_pos, const float* cos_sin, int n, int num_layers, int Hkv,
                               int head_dim, int src_page_size, int dst_page_size, int64_t src_layer_stride,
                               int64_t dst_layer_stride, int64_t src_slot_limit, int64_t dst_slot_limit,
                               int max_pos, int* err, cudaStream_t stream) {
  if (n <= 0) return 0;
  if (head_dim != 128) return -3;
  const int threads = 256;
  // about one resident wave of warps (148 SMs x 64 warps): fewer tokens
  // than that split their layers over several warps
  constexpr int64_t kTargetWarps = 148 * 64;
  int groups = (int)((kTargetWarps + n - 1) / n);
  groups = groups < 1 ? 1 : (groups > num_layers ? num_layers : groups);
  const int blocks = (int)(((int64_t)n * groups * 32 + threads - 1) / threads);
  kv_link_rope_kernel<<<blocks, threads, 0, stream>>>(dst_k, dst_v, src_k, src_v, src_slots, dst_slots, local_pos,
                                                      global_pos, cos_sin, n, num_layers, Hkv, src_page_size,
                                                      dst_page_size, src_layer_stride, dst_layer_stride,
                                                      src_slot_limit, dst_slot_limit, max_pos, err, groups);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

extern "C" int ll_swiglu(bf16* out, const bf16* gu, int T, int inter, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (inter % 16) return -3;
  const size_t nvec = (size_t)T * inter / 8;
  int blocks = (int)((nvec + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(swiglu_kernel, dim3(blocks), dim3(256), 0, stream, out, gu, T, inter);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

extern "C" int ll_embedding(bf16* out, const int* ids, const bf16* table, int T, int hidden, int vocab_start,
                            int vocab_end, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (hidden % 8) return -3;
  launch_pdl(embedding_kernel, dim3(T), dim3(128), 0, stream, out, ids, table, hidden, vocab_start, vocab_end);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

extern "C" int ll_argmax(int* out, const bf16* logits, int rows, int vocab, int ld, cudaStream_t stream) {
  if (rows <= 0) return 0;
  launch_pdl(argmax_kernel, dim3(rows), dim3(1024), 0, stream, out, logits, vocab, ld);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}
