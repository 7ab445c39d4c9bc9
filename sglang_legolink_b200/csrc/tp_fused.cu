// Tensor-parallel layer boundary without a collective library call.
//
// Row-parallel GEMMs (o_proj, down_proj) of a TP layer produce partial sums
// that the reference reduces with an NCCL all-reduce (reference
// patched_sglang_files/python/sglang/srt/models/qwen2.py:80-86,162-168, the
// RowParallelLinear path).  Here the sequence is split into `world` row
// ranges of `rows_per_rank` rows (R, a multiple of 32) and:
//
//   1. the 2-SM GEMM's epilogue (kEpiScatter, gemm_tcgen05.cu) stores each
//      output row straight into its owner's slot buffer over NVLink (tiled
//      32 x 32, so each warp store instruction writes 512 contiguous bytes) while
//      the tensor cores work on the next tile, and bumps the owner's
//      arrival counter by the 32-row slices it stored, once at the end of the
//      GEMM (reduce-scatter fused into the GEMM);
//   2. tp_reduce_norm_gather_kernel (this file) runs on every owner: it waits
//      for all slices, sums the world slots in fp32, adds the residual,
//      stores the new residual, applies RMSNorm and writes the normalised
//      row into EVERY rank's gather buffer G over NVLink (the all-gather,
//      fused into the norm), then bumps every rank's G counter;
//   3. the next column-parallel GEMM (QKV / gate-up) waits on its G counter
//      in its producer warp and TMA-loads A from the local G.
//
// Counters only grow: the host keeps the cumulative target of each one, so
// no counter is ever reset between layers.  Every wait is bounded
// (wait_counter_geq in common.cuh) and reports kErrPeerFlagTimeout.
#include <cuda_runtime.h>

#include "common.cuh"
#include "tp_fused.h"

namespace ll {

using TpGather = LLTpGather;

// One CTA of TPB = 128 threads per row (grid-strided over as many CTAs as
// are resident at once, so there is no partial second wave); each thread
// keeps VPT 16-byte vectors of the row in registers, and its VPT vectors of
// the norm weight for the whole loop (one load per CTA instead of an L2
// round trip per row after the reduction).
constexpr int TPB = 128;
template <int VPT>
__global__ void __launch_bounds__(TPB)
    tp_reduce_norm_gather_kernel(const bf16* __restrict__ slots, bf16* __restrict__ residual,
                                 const bf16* __restrict__ w, float eps, int H, int rows,
                                 const __grid_constant__ TpGather tg, int* err) {
  __shared__ int s_ok;
  __shared__ float red[TPB / 32];
  const int R = tg.rows_per_rank;
  if (threadIdx.x == 0) s_ok = tg.slot_cnt == nullptr ? 1 : (wait_counter_geq(tg.slot_cnt, tg.slot_target, err) ? 1 : 0);
  __syncthreads();
  const int nvec = H / 8;
  uint4 wv[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * TPB;
    wv[i] = idx < nvec ? reinterpret_cast<const uint4*>(w)[idx] : make_uint4(0, 0, 0, 0);
  }
  if (s_ok) {
    for (int row = blockIdx.x; row < rows; row += gridDim.x) {
      uint4* rr = reinterpret_cast<uint4*>(residual + (size_t)row * H);
      float v[VPT][8];
      // residual, then each source rank's slot (all VPT loads of one slot are
      // independent and issue back to back)
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = threadIdx.x + i * TPB;
        uint4 b = idx < nvec ? rr[idx] : make_uint4(0, 0, 0, 0);
        const uint32_t* bu = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(bu[j]);
          v[i][2 * j] = f.x;
          v[i][2 * j + 1] = f.y;
        }
      }
      if (slots != nullptr) {
#pragma unroll 2
        for (int s = 0; s < tg.world; ++s) {
          // source s's slot is tiled: [R/32][H/32] tiles of 32 x 32 (2 KB
          // each); 16-byte vector idx of the row is in tile column idx / 4
          const uint4* sr = reinterpret_cast<const uint4*>(slots + (size_t)s * R * H) +
                            (size_t)(row >> 5) * (size_t)(H >> 5) * 128 + (row & 31) * 4;
          uint4 a[VPT];
#pragma unroll
          for (int i = 0; i < VPT; ++i) {
            const int idx = threadIdx.x + i * TPB;
            // L2-only loads: the slots were written by other GPUs.
            a[i] = idx < nvec ? __ldcg(sr + (idx >> 2) * 128 + (idx & 3)) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int i = 0; i < VPT; ++i) {
            const uint32_t* au = reinterpret_cast<const uint32_t*>(&a[i]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = unpack_bf16x2(au[j]);
              v[i][2 * j] += f.x;
              v[i][2 * j + 1] += f.y;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          const int idx = threadIdx.x + i * TPB;
          if (idx < nvec) {
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = pack_bf16x2(v[i][2 * j], v[i][2 * j + 1]);
            rr[idx] = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < TPB / 32; ++i) tot += red[i];
      __syncthreads();
      const float rstd = rsqrtf(tot / H + eps);
      const size_t grow = (size_t)tg.rank * R + row;  // row index in every rank's G
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = threadIdx.x + i * TPB;
        if (idx < nvec) {
          const uint32_t* wu = reinterpret_cast<const uint32_t*>(&wv[i]);
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack_bf16x2(wu[j]);
            o[j] = pack_bf16x2(v[i][2 * j] * rstd * f.x, v[i][2 * j + 1] * rstd * f.y);
          }
          const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
          for (int d = 0; d < tg.world; ++d) reinterpret_cast<uint4*>(static_cast<bf16*>(tg.g[d]) + grow * H)[idx] = ov;
        }
      }
    }
  }
  // Publish: every thread's peer stores, then one release-add per rank.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < tg.world) red_release_sys_add(tg.g_cnt[threadIdx.x], 1ull);
}

}  // namespace ll

using namespace ll;

typedef void (*TpRngKern)(const bf16*, bf16*, const bf16*, float, int, int, const TpGather, int*);

static TpRngKern tp_rng_kernel(int H) {
  switch ((H / 8 + TPB - 1) / TPB) {
    case 1: return tp_reduce_norm_gather_kernel<1>;
    case 2: return tp_reduce_norm_gather_kernel<2>;
    case 3: return tp_reduce_norm_gather_kernel<3>;
    case 4: return tp_reduce_norm_gather_kernel<4>;
    case 5: return tp_reduce_norm_gather_kernel<5>;
    case 6: return tp_reduce_norm_gather_kernel<6>;
    default: return tp_reduce_norm_gather_kernel<8>;
  }
}

// Grid used by ll_tp_reduce_norm_gather for `rows` rows of width H: the CTAs
// that are resident at once (the same on every rank of one GPU type, so each
// rank's G counter grows by world x this per call).
extern "C" int ll_tp_reduce_norm_gather_grid(int rows, int H) {
  static int sms = 0, per_sm[9] = {};
  const int vpt = (H / 8 + TPB - 1) / TPB;
  const int slot = vpt > 6 ? 8 : vpt;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  if (per_sm[slot] == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, tp_rng_kernel(H), TPB, 0) != cudaSuccess || n <= 0) n = 4;
    per_sm[slot] = n;
  }
  const int g = per_sm[slot] * sms;
  return rows < g ? rows : g;
}

// slots: this rank's [world][R][H] slot buffer, or nullptr for a plain
// norm + all-gather (the first layer).  residual: this rank's [R][H] rows.
extern "C" int ll_tp_reduce_norm_gather(const void* slots_, void* residual_, const void* w_, float eps, int H,
                                        int rows, const LLTpGather* tg, int* err, void* stream_) {
  const bf16* slots = static_cast<const bf16*>(slots_);
  bf16* residual = static_cast<bf16*>(residual_);
  const bf16* w = static_cast<const bf16*>(w_);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (H % 32 || H > 8 * TPB * 8 || rows <= 0 || rows > tg->rows_per_rank || tg->rows_per_rank % 32) return -3;
  if (tg->world < 1 || tg->world > LL_MAX_TP_RANKS) return -3;
  const int grid = ll_tp_reduce_norm_gather_grid(rows, H);
  tp_rng_kernel(H)<<<grid, TPB, 0, stream>>>(slots, residual, w, eps, H, rows, *tg, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

namespace ll {
// One thread waits (bounded) for a gather counter so that later kernels on
// the stream may read the gathered rows with ordinary loads.
__global__ void tp_wait_kernel(const unsigned long long* cnt, unsigned long long target, int* err) {
  if (threadIdx.x == 0) {
    wait_counter_geq(cnt, target, err);
    __threadfence();
  }
}
}  // namespace ll

extern "C" int ll_tp_wait(const void* cnt, unsigned long long target, int* err, void* stream) {
  ll::tp_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const unsigned long long*>(cnt),
                                                                       target, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

// ---------------------------------------------------------------- decode
// Decode boundary of a TP layer: each rank's row-parallel GEMV wrote its
// partial rows [rows][H] into its own symmetric buffer; this kernel, on every
// rank, is a one-shot all-reduce fused with the residual add and RMSNorm:
//
//   * CTA 0 announces "my partial is complete" by a release-add of 1 to every
//     rank's arrival counter (the GEMV before it on the stream has finished);
//   * each CTA waits (bounded) until its own counter reaches world x epoch;
//   * one CTA per row loads the row from every rank's buffer over NVLink (all
//     loads of a rank issued back to back), sums residual + partials in fp32
//     in rank order (so every rank computes the same bits), stores the new
//     residual and writes RMSNorm(residual) * w;
//   * the last CTA advances this rank's epoch.
//
// The caller alternates two partial buffers between consecutive calls.  A
// rank rewrites buffer b only in call i + 2, after passing call i + 1's wait,
// which every peer joins only after finishing its call-i reads of b, so no
// end-of-call barrier is needed.
namespace ll {
constexpr int TPD = 256;
// residual (bf16) + sum (bf16, already reduced over the ranks) in fp32 ->
// residual; RMSNorm(residual) * w -> out (one CTA per row, TPD threads).
template <int VPT>
__device__ __forceinline__ void res_add_norm_store(const uint4 (&res_v)[VPT], const uint4 (&sum_v)[VPT],
                                                   const uint4 (&w_v)[VPT], uint4* rr, bf16* out, int row, int H,
                                                   int nvec, float eps, float* red) {
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const uint32_t* bu = reinterpret_cast<const uint32_t*>(&res_v[i]);
    const uint32_t* su = reinterpret_cast<const uint32_t*>(&sum_v[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(bu[j]), g = unpack_bf16x2(su[j]);
      v[i][2 * j] = f.x + g.x;
      v[i][2 * j + 1] = f.y + g.y;
    }
    const int idx = threadIdx.x + i * TPD;
    if (idx < nvec) {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[j] = pack_bf16x2(v[i][2 * j], v[i][2 * j + 1]);
        ss += v[i][2 * j] * v[i][2 * j] + v[i][2 * j + 1] * v[i][2 * j + 1];
      }
      rr[idx] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < TPD / 32; ++i) tot += red[i];
  const float rstd = rsqrtf(tot / H + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * H);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * TPD;
    if (idx < nvec) {
      const uint32_t* wu = reinterpret_cast<const uint32_t*>(&w_v[i]);
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(wu[j]);
        o[j] = pack_bf16x2(v[i][2 * j] * rstd * f.x, v[i][2 * j + 1] * rstd * f.y);
      }
      orow[idx] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// WMAX: compile-time bound on the world size, so that the loads of every
// rank's partial row are issued together after the wait (one NVLink round
// trip instead of one per pair of ranks).  The residual row and the norm
// weights do not depend on the other ranks and are loaded before the wait
// for their arrivals.
template <int VPT, int WMAX>
__global__ void __launch_bounds__(TPD)
    tp_decode_allreduce_norm_kernel(bf16* __restrict__ residual, const bf16* __restrict__ w, bf16* __restrict__ out,
                                    float eps, int H, int rows, const __grid_constant__ LLTpDecode td, int* err) {
  __shared__ int s_ok;
  __shared__ unsigned long long s_e;
  __shared__ float red[TPD / 32];
  const int nvec = H / 8;
  const int row = blockIdx.x;
  const bool live = row < rows;
  uint4* rr = reinterpret_cast<uint4*>(residual + (size_t)row * H);
  // The next GEMV may launch now: its CTAs stream their weights while this
  // boundary waits for the other ranks, and read our output only after
  // their own pdl_wait (this grid complete).
  pdl_trigger();
  uint4 res_v[VPT], w_v[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {  // norm weights: written by no kernel
    const int idx = threadIdx.x + i * TPD;
    w_v[i] = (live && idx < nvec) ? reinterpret_cast<const uint4*>(w)[idx] : make_uint4(0, 0, 0, 0);
  }
  // The partial rows, the residual and the epoch are written by earlier
  // kernels, which may still run while this one is resident.
  pdl_wait();
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * TPD;
    res_v[i] = (live && idx < nvec) ? rr[idx] : make_uint4(0, 0, 0, 0);
  }
  if (threadIdx.x == 0) {
    const unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(td.epoch) + 1ull;
    s_e = e;
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int d = 0; d < td.world; ++d) red_release_sys_add(td.cnt[d], 1ull);
    }
    s_ok = wait_counter_geq(td.cnt[td.rank], e * (unsigned long long)td.world, err) ? 1 : 0;
  }
  __syncthreads();
  if (s_ok && live && td.mc != nullptr) {
    // NVLS: every element's sum over the ranks comes from the switch in one
    // multimem load (bf16 result, fp32 accumulation), then residual + norm
    const uint4* mr = reinterpret_cast<const uint4*>(static_cast<const bf16*>(td.mc) + (size_t)row * H);
    uint4 sm[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * TPD;
      if (idx < nvec) {
        uint32_t r0, r1, r2, r3;
        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                     : "l"(mr + idx)
                     : "memory");
        sm[i] = make_uint4(r0, r1, r2, r3);
      } else {
        sm[i] = make_uint4(0, 0, 0, 0);
      }
    }
    res_add_norm_store<VPT>(res_v, sm, w_v, rr, out, row, H, nvec, eps, red);
  } else if (s_ok && live) {
    uint4 a[WMAX][VPT];
#pragma unroll
    for (int d = 0; d < WMAX; ++d) {
      if (d < td.world) {
        const uint4* pr = reinterpret_cast<const uint4*>(static_cast<const bf16*>(td.part[d]) + (size_t)row * H);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          const int idx = threadIdx.x + i * TPD;
          a[d][i] = idx < nvec ? __ldcg(pr + idx) : make_uint4(0, 0, 0, 0);  // not through L1: peer data
        }
      }
    }
    float v[VPT][8];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const uint32_t* bu = reinterpret_cast<const uint32_t*>(&res_v[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(bu[j]);
        v[i][2 * j] = f.x;
        v[i][2 * j + 1] = f.y;
      }
    }
    // residual + partials in rank order: every rank computes the same bits
#pragma unroll
    for (int d = 0; d < WMAX; ++d) {
      if (d < td.world) {
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          const uint32_t* au = reinterpret_cast<const uint32_t*>(&a[d][i]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack_bf16x2(au[j]);
            v[i][2 * j] += f.x;
            v[i][2 * j + 1] += f.y;
          }
        }
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * TPD;
      if (idx < nvec) {
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // the norm reads the fp32 sum, as the unfused add + RMSNorm does
          o[j] = pack_bf16x2(v[i][2 * j], v[i][2 * j + 1]);
          ss += v[i][2 * j] * v[i][2 * j] + v[i][2 * j + 1] * v[i][2 * j + 1];
        }
        rr[idx] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < TPD / 32; ++i) tot += red[i];
    const float rstd = rsqrtf(tot / H + eps);
    uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * H);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * TPD;
      if (idx < nvec) {
        const uint32_t* wu = reinterpret_cast<const uint32_t*>(&w_v[i]);
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(wu[j]);
          o[j] = pack_bf16x2(v[i][2 * j] * rstd * f.x, v[i][2 * j + 1] * rstd * f.y);
        }
        orow[idx] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* ticket = reinterpret_cast<unsigned int*>(td.epoch + 1);
    if (atomicAdd(ticket, 1u) == gridDim.x - 1) {
      *reinterpret_cast<volatile unsigned int*>(ticket) = 0u;
      __threadfence();
      *reinterpret_cast<volatile unsigned long long*>(td.epoch) = s_e;
    }
  }
}
}  // namespace ll

// One CTA per row; every rank must make the same sequence of calls.
extern "C" int ll_tp_decode_allreduce_norm(void* residual, const void* w, void* out, float eps, int H, int rows,
                                           const LLTpDecode* td, int* err, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (H % 8 || H > 8 * TPD * 4 || rows <= 0 || rows > 1024) return -3;
  if (td->world < 1 || td->world > LL_MAX_TP_RANKS || td->rank < 0 || td->rank >= td->world) return -3;
  const int vpt = (H / 8 + TPD - 1) / TPD;
  bf16* r = static_cast<bf16*>(residual);
  const bf16* wp = static_cast<const bf16*>(w);
  bf16* o = static_cast<bf16*>(out);
#define LL_TPD(V, W) \
  ll::launch_pdl(ll::tp_decode_allreduce_norm_kernel<V, W>, dim3(rows), dim3(ll::TPD), 0, stream, r, wp, o, eps, H, rows, *td, err)
#define LL_TPD_W(V)                    \
  do {                                 \
    if (td->world <= 2) LL_TPD(V, 2);  \
    else if (td->world <= 4) LL_TPD(V, 4); \
    else LL_TPD(V, 8);                 \
  } while (0)
  switch (vpt) {
    case 1: LL_TPD_W(1); break;
    case 2: LL_TPD_W(2); break;
    case 3: LL_TPD_W(3); break;
    default: LL_TPD_W(4); break;
  }
#undef LL_TPD_W
#undef LL_TPD
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

// ------------------------------------------------------- vocab-sharded argmax
// Greedy sampling when the LM head is split over the vocabulary (reference:
// the logits all-gather of the tensor-parallel LM head, replaced there by a
// gather of per-rank (max, index) pairs): one kernel per call on every rank.
//   * CTA i takes row i: block argmax of this rank's logits shard (ties: the
//     smallest index, as torch.argmax);
//   * it stores (max, vocab_start + index) into row i's record for this rank
//     in EVERY rank's slot array (peer stores over NVLink), then the record's
//     tag = epoch with release semantics;
//   * it waits (bounded) until the W records of row i in its own slot carry
//     this epoch, and writes the index of the largest max (ties: the lowest
//     rank, whose vocabulary range comes first -> the smallest token id).
// Records alternate between two parities by epoch: a rank writes parity p
// again only in call e + 2, after passing call e + 1's wait, which every
// peer joins only after finishing its call-e reads.  The epoch lives in
// device memory (advanced by the last CTA), so a CUDA graph replays the
// call unchanged.
namespace ll {
constexpr int TPA = 512;
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(TPA)
    tp_argmax_kernel(const bf16* __restrict__ logits, int vocab, int ld, int vocab_start, int rows,
                     int* __restrict__ out, const __grid_constant__ LLTpArgmax ta, int* err) {
  __shared__ float sv[TPA / 32];
  __shared__ int si[TPA / 32];
  __shared__ unsigned long long s_e;
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) s_e = *reinterpret_cast<volatile unsigned long long*>(ta.epoch) + 1ull;
  const int i = blockIdx.x;
  const bf16* row = logits + (size_t)i * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = threadIdx.x; v < vocab; v += TPA) {  // increasing per thread: '>' keeps the first
    const float x = __bfloat162float(row[v]);
    if (x > best) {
      best = x;
      bi = v;
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
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    best = threadIdx.x < TPA / 32 ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < TPA / 32 ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
  }
  const unsigned long long e = s_e;
  const int par = (int)(e & 1ull);
  // lanes 0..world-1 of warp 0: push this rank's pair to every rank
  if (threadIdx.x < 32) {
    const int gidx = bi == 0x7fffffff ? vocab_start : vocab_start + bi;
    const unsigned long long pair =
        ((unsigned long long)__float_as_uint(__shfl_sync(0xffffffffu, best, 0)) << 32) |
        (unsigned int)__shfl_sync(0xffffffffu, gidx, 0);
    const int d = threadIdx.x;
    if (d < ta.world) {
      LLTpArgmaxRec* rec = static_cast<LLTpArgmaxRec*>(ta.slot[d]) +
                           ((size_t)par * ta.rmax + i) * LL_MAX_TP_RANKS + ta.rank;
      rec->pair = pair;
      st_release_sys_u64(&rec->tag, e);
    }
    // wait for every rank's record of this row in this rank's slot
    bool ok = true;
    float rv = -INFINITY;
    int ri = 0x7fffffff;
    if (d < ta.world) {
      LLTpArgmaxRec* own = static_cast<LLTpArgmaxRec*>(ta.slot[ta.rank]) +
                           ((size_t)par * ta.rmax + i) * LL_MAX_TP_RANKS + d;
      if (ld_acquire_sys(&own->tag) != e) {
        const unsigned long long start = globaltimer_ns();
        uint32_t iter = 0;
        while (true) {
          __nanosleep(32);
          if (ld_acquire_sys(&own->tag) == e) break;
          if ((++iter & 63u) == 0 && globaltimer_ns() - start > kWaitLimitNs) {
            record_error(err, kErrPeerFlagTimeout);
            ok = false;
            break;
          }
        }
      }
      if (ok) {
        const unsigned long long pv = *reinterpret_cast<volatile unsigned long long*>(&own->pair);
        rv = __uint_as_float((unsigned int)(pv >> 32));
        ri = (int)(unsigned int)(pv & 0xffffffffull);
      }
    }
    // largest max; ties to the lowest rank (the smallest token id)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, rv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, ri, o);
      if (ov > rv || (ov == rv && oi < ri)) {
        rv = ov;
        ri = oi;
      }
    }
    const bool all_ok = __all_sync(0xffffffffu, ok);
    if (threadIdx.x == 0 && i < rows) out[i] = all_ok ? ri : -1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* ticket = reinterpret_cast<unsigned int*>(ta.epoch + 1);
    if (atomicAdd(ticket, 1u) == gridDim.x - 1) {
      *reinterpret_cast<volatile unsigned int*>(ticket) = 0u;
      __threadfence();
      *reinterpret_cast<volatile unsigned long long*>(ta.epoch) = e;
    }
  }
}
}  // namespace ll

// One CTA per row (rows <= rmax); every rank must make the same sequence of
// calls with the same row count.
extern "C" int ll_tp_argmax(const void* logits, int vocab_local, int ld, int vocab_start, int rows, int* out,
                            const LLTpArgmax* ta, int* err, void* stream_) {
  if (rows <= 0) return 0;
  if (rows > ta->rmax || ta->world < 1 || ta->world > LL_MAX_TP_RANKS || ta->rank < 0 || ta->rank >= ta->world ||
      vocab_local <= 0)
    return -3;
  launch_pdl(ll::tp_argmax_kernel, dim3(rows), dim3(ll::TPA), 0, static_cast<cudaStream_t>(stream_),
             static_cast<const ll::bf16*>(logits), vocab_local, ld, vocab_start, rows, out, *ta, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

