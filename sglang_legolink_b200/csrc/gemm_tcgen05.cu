// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
//   C[M, N] = A[M, K] . W[N, K]^T (+ bias[N])          (nn.Linear layout)
//
// Two kernels share the same pipeline pieces:
//
// * gemm_tcgen05_kernel -- persistent, one CTA per SM, 128 x BN output tiles.
//   warp 0 issues TMA loads of A/W k-blocks into a STAGES-deep shared-memory
//   ring (128-byte swizzle), warp 1 allocates TMEM and one elected thread
//   issues tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM accumulators,
//   warps 2..5 drain the other accumulator (tcgen05.ld) so the epilogue of
//   tile i overlaps the main loop of tile i+1.
//   Epilogues: plain (+bias) and SwiGLU, where W's rows are interleaved in
//   groups of 16 (gate rows, then the matching up rows) so that every
//   32-column chunk of the accumulator yields 16 outputs silu(g) * u.
//
// * gemm_swapab_kernel -- for small M (decode): computes C^T = W . A^T so the
//   weight tile fills the M=128 side of the MMA and the few activation rows
//   sit on the N side (N = 16/32/64/128).  K is split across CTAs so that
//   every SM streams weights; partial sums go to an fp32 workspace and the
//   last CTA of each output tile (atomic ticket) reduces and writes bf16.
//
// The reference runs these GEMMs through cuBLAS via torch linear layers
// (reference patched_sglang_files/python/sglang/srt/models/qwen2.py:63-217).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "gemm_epi.h"
#include "tp_fused.h"

namespace ll {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
// ll_gemm_bf16_small_m_ex flags
constexpr int LL_SMALL_M_W_TILED = 1;
constexpr int LL_SMALL_M_SWIGLU = 2;

enum Epilogue : int { kEpiPlain = 0, kEpiSwiGLU = 1, kEpiScatter = 2 };

// Tensor-parallel hooks of the 2-SM kernel (tp_fused.h, tp_fused.cu).
using TpArgs = LLTpArgs;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES) + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16(x)); }
// Named barrier 1 over the 128 epilogue threads (warps 2-5).
__device__ __forceinline__ void bar_sync_128() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Same barrier, returning whether `p` held in all 128 threads.
__device__ __forceinline__ bool bar_and_128(bool p) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n bar.red.and.pred po, 1, 128, pi;\n"
      " selp.u32 %0, 1, 0, po;\n}"
      : "=r"(r)
      : "r"((uint32_t)p)
      : "memory");
  return r != 0;
}

// Tile order: groups of `group_m` m-blocks, m fastest inside a group, so
// the tiles in flight at once (one per SM or SM pair) share a few A row
// blocks and a few W column blocks; plain m-fastest order re-streams all of
// A from HBM once per W column block when A does not fit in L2.  W is read
// from HBM once per group, so the host makes a group as large as keeps its
// A rows L2-resident (gemm_group_m).
constexpr int GEMM_GROUP_M = 8;
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group_m, int& mb, int& nb) {
  const int per_group = group_m * num_n;
  const int first_m = (t / per_group) * group_m;
  const int gm = min(num_m - first_m, group_m);
  const int r = t % per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        bf16* __restrict__ C, const bf16* __restrict__ bias, int M, int N, int K, int ldc,
                        int* err, int group_m) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + GEMM_BM - 1) / GEMM_BM;
  const int num_n = (N + BN - 1) / BN;
  const int ntiles = num_m * num_n;
  const int num_kb = (K + GEMM_BK - 1) / GEMM_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, group_m, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, err, kErrSmemEmptyTimeout)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::B_BYTES);
          tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * GEMM_BK, mb * GEMM_BM);
          tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB, &full[stage], kb * GEMM_BK, nb * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Give in-flight bulk copies time to land before the CTA exits.
        unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(GEMM_BM, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, aphase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], aphase ^ 1, err, kErrTmemEmptyTimeout)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, kErrTmaFullTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128_kmajor(smem_u32(sA + stage * Cfg::A_BYTES));
          const uint64_t bd = umma_desc_sw128_kmajor(smem_u32(sB + stage * Cfg::B_BYTES));
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            umma_bf16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          aphase ^= 1;
        }
      }
      // Drain: wait until every MMA this thread issued has completed before
      // the accumulator memory is released.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    // Epilogue warps 2..5: warp (w % 4) owns TMEM lanes [32*(w%4), +32).
    const int q = warp & 3;
    int acc = 0;
    uint32_t aphase = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      int mb, nb;
        tile_coords(t, num_m, num_n, group_m, mb, nb);
      if (!mbar_wait(&tfull[acc], aphase, err, kErrTmemFullTimeout)) break;
      tc_fence_after();
      const int row = mb * GEMM_BM + q * 32 + lane;
      const uint32_t tbase = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + c, r);
        tmem_ld_wait();
        const int col0 = nb * BN + c;
        if (row < M && col0 < N) {
          if constexpr (EPI == kEpiSwiGLU) {
            // 16 gate columns then the 16 matching up columns.
            bf16* dst = C + (size_t)row * ldc + (col0 >> 1);
            uint32_t packed[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float g0 = __uint_as_float(r[2 * i]), g1 = __uint_as_float(r[2 * i + 1]);
              float u0 = __uint_as_float(r[16 + 2 * i]), u1 = __uint_as_float(r[16 + 2 * i + 1]);
              if (bias != nullptr) {
                g0 += __bfloat162float(bias[col0 + 2 * i]);
                g1 += __bfloat162float(bias[col0 + 2 * i + 1]);
                u0 += __bfloat162float(bias[col0 + 16 + 2 * i]);
                u1 += __bfloat162float(bias[col0 + 16 + 2 * i + 1]);
              }
              packed[i] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
            }
            uint4* d4 = reinterpret_cast<uint4*>(dst);
            d4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            d4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
          } else {
            bf16* dst = C + (size_t)row * ldc + col0;
            if (col0 + 32 <= N) {
              uint32_t packed[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                float a0 = __uint_as_float(r[2 * i]), a1 = __uint_as_float(r[2 * i + 1]);
                if (bias != nullptr) {
                  a0 += __bfloat162float(bias[col0 + 2 * i]);
                  a1 += __bfloat162float(bias[col0 + 2 * i + 1]);
                }
                packed[i] = pack_bf16x2(a0, a1);
              }
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
            } else {
              for (int i = 0; i < 32 && col0 + i < N; ++i) {
                float a = __uint_as_float(r[i]);
                if (bias != nullptr) a += __bfloat162float(bias[col0 + i]);
                dst[i] = __float2bfloat16(a);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        aphase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
}

// ---------------------------------------------------------------------------
// Fixed-point row sum of squares -> float (see gemm_epi.h).
__device__ __forceinline__ float sumsq_value(unsigned long long x) {
  return __ull2float_rn(x) * (1.f / LL_SUMSQ_ONE);
}

// Four consecutive bf16 <-> float (8-byte accesses; the caller guarantees
// the alignment).
__device__ __forceinline__ void ld_bf16x4(const bf16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  v[0] = __low2float(a);
  v[1] = __high2float(a);
  v[2] = __low2float(b);
  v[3] = __high2float(b);
}
__device__ __forceinline__ void st_bf16x4(bf16* p, float v0, float v1, float v2, float v3) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v0, v1), b = __floats2bfloat162_rn(v2, v3);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// Sum over a 32-feature group held as 4 consecutive features by each of 8
// lanes (lanes 8g..8g+7 hold features 32g..32g+31).  The additions pair the
// same features in the same order as warp_sum() over one feature per lane
// (feature distance 16, 8, 4 across lanes, then 2 and 1 inside the thread),
// so the result has the same bits as the one-feature-per-lane epilogue.
__device__ __forceinline__ float group32_sum(float y0, float y1, float y2, float y3) {
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) {
    y0 += __shfl_xor_sync(0xffffffffu, y0, o);
    y1 += __shfl_xor_sync(0xffffffffu, y1, o);
    y2 += __shfl_xor_sync(0xffffffffu, y2, o);
    y3 += __shfl_xor_sync(0xffffffffu, y3, o);
  }
  return (y0 + y2) + (y1 + y3);
}

// Tile epilogue of the small-M kernel for 2 <= M <= 16 rows.  The four
// epilogue warps hold the 16 x 128 output tile as warp q = rows 4q..4q+3,
// lane = features 4*lane..4*lane+3, so every row of the tile lives in ONE
// warp: a row's sums over the tile (QK-norm, the residual epilogue's sum of
// squares) and the RoPE rotate-half partner (feature f +- 64 = lane ^ 16) are
// warp shuffles, and the four warps emit their rows at the same time with no
// block barrier.  The split-K fix-up loads each thread's 4 rows x 4 features
// of up to four splits at once (16-byte loads).  The per-element arithmetic
// and the order of every sum are those of the one-row-at-a-time epilogue, so
// both give the same bits.
template <int MODE>
struct TileEpi {
  int q, lane, f0, feat0, m0;
  bool fvalid;
  float tb[4], tw[4];        // bias, norm weight (residual: norm_w; qkv: q/k norm)
  float rs[4];               // per-row scale
  float tres[4][4];          // residual rows
  float tc[4][4], ts[4][4];  // RoPE cos / sin of the four rows
  int tpos[4];
  int64_t tslot[4];

  // Operands that do not depend on the product (call after pdl_wait).
  __device__ __forceinline__ void prefetch(const bf16* __restrict__ bias, int M, int N, int K, int nb,
                                           const LLSmallMEpi& epi) {
    fvalid = feat0 < N;
#pragma unroll
    for (int c = 0; c < 4; ++c) tb[c] = tw[c] = 0.f;
    if (bias != nullptr && fvalid) ld_bf16x4(bias + feat0, tb);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + j;
      rs[j] = (epi.scale_sumsq != nullptr && m < M)
                  ? rsqrtf(sumsq_value(__ldcg(epi.scale_sumsq + m)) / (float)K + epi.scale_eps)
                  : 1.f;
    }
    if constexpr (MODE == LL_EPI_RESIDUAL) {
      if (fvalid) ld_bf16x4(epi.norm_w + feat0, tw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int c = 0; c < 4; ++c) tres[j][c] = 0.f;
        if (m0 + j < M && fvalid) ld_bf16x4(epi.res + (size_t)(m0 + j) * epi.ld + feat0, tres[j]);
      }
    }
    if constexpr (MODE == LL_EPI_QKV_ROPE) {
      const bf16* nw = nb < epi.Hq ? epi.q_norm_w : (nb < epi.Hq + epi.Hkv ? epi.k_norm_w : nullptr);
      if (nw != nullptr) ld_bf16x4(nw + f0, tw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int m = m0 + j;
        tpos[j] = m < M ? epi.positions[m] : 0;
        tslot[j] = m < M ? epi.slots[m] : 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) tc[j][c] = ts[j][c] = 0.f;
        if (m < M && nb < epi.Hq + epi.Hkv && tpos[j] >= 0 && tpos[j] < epi.max_pos) {
          const float4 cv = *reinterpret_cast<const float4*>(epi.cos_sin + (size_t)tpos[j] * 128 + (f0 & 63));
          const float4 sv = *reinterpret_cast<const float4*>(epi.cos_sin + (size_t)tpos[j] * 128 + 64 + (f0 & 63));
          tc[j][0] = cv.x, tc[j][1] = cv.y, tc[j][2] = cv.z, tc[j][3] = cv.w;
          ts[j][0] = sv.x, ts[j][1] = sv.y, ts[j][2] = sv.z, ts[j][3] = sv.w;
        }
      }
    }
  }

  // Emits row j (m = m0 + j < M) from its four accumulator values.  Called
  // by the whole warp (shuffles); lanes past N store nothing.
  __device__ __forceinline__ void emit(int j, const float (&a)[4], bf16* __restrict__ C, int ldc, int M, int nb,
                                       const LLSmallMEpi& epi, int* err) {
    const int m = m0 + j;
    float v[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      v[c] = a[c];
      if (epi.scale_sumsq != nullptr) v[c] *= rs[j];
      v[c] += tb[c];
    }
    if constexpr (MODE == LL_EPI_STORE) {
      if (fvalid) st_bf16x4(C + (size_t)m * ldc + feat0, v[0], v[1], v[2], v[3]);
    } else if constexpr (MODE == LL_EPI_SWIGLU) {
      // gate features on lanes 8g..8g+3, the matching up features on lane ^ 4
      float u[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) u[c] = __shfl_xor_sync(0xffffffffu, v[c], 4);
      if ((lane & 4) == 0 && fvalid)
        st_bf16x4(C + (size_t)m * ldc + (feat0 >> 5) * 16 + (feat0 & 15), silu_f(v[0]) * u[0], silu_f(v[1]) * u[1],
                  silu_f(v[2]) * u[2], silu_f(v[3]) * u[3]);
    } else if constexpr (MODE == LL_EPI_RESIDUAL) {
      float r[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) r[c] = fvalid ? bf16_round(v[c]) + tres[j][c] : 0.f;
      if (fvalid) {
        const size_t i = (size_t)m * epi.ld + feat0;
        st_bf16x4(epi.res + i, r[0], r[1], r[2], r[3]);
        st_bf16x4(epi.h_out + i, r[0] * tw[0], r[1] * tw[1], r[2] * tw[2], r[3] * tw[3]);
      }
      const float ss = group32_sum(r[0] * r[0], r[1] * r[1], r[2] * r[2], r[3] * r[3]);
      if ((lane & 7) == 0 && fvalid) atomicAdd(epi.sumsq_out + m, __float2ull_rn(ss * LL_SUMSQ_ONE));
    } else {  // LL_EPI_QKV_ROPE: this tile is head nb of [Hq | Hkv keys | Hkv values]
      const int64_t slot = tslot[j];
      const int pos_m = tpos[j];
      if (slot < 0 || slot >= epi.slot_limit || pos_m < 0 || pos_m >= epi.max_pos) {
        if (lane == 0) record_error(err, kErrBadIndex);
        return;
      }
      float x[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) x[c] = bf16_round(v[c]);
      const int64_t page = slot / epi.page_size, off = slot % epi.page_size;
      bf16* dst;
      if (nb < epi.Hq + epi.Hkv) {
        const bf16* nw = nb < epi.Hq ? epi.q_norm_w : epi.k_norm_w;
        if (nw != nullptr) {
          const float gs = group32_sum(x[0] * x[0], x[1] * x[1], x[2] * x[2], x[3] * x[3]);
          const float s0 = __shfl_sync(0xffffffffu, gs, 0), s1 = __shfl_sync(0xffffffffu, gs, 8);
          const float s2 = __shfl_sync(0xffffffffu, gs, 16), s3 = __shfl_sync(0xffffffffu, gs, 24);
          const float tot = (s0 + s1) + (s2 + s3);
#pragma unroll
          for (int c = 0; c < 4; ++c) x[c] = x[c] * rsqrtf(tot / 128.f + epi.eps) * tw[c];
        }
        float p[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) p[c] = __shfl_xor_sync(0xffffffffu, x[c], 16);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float cc = tc[j][c], sn = ts[j][c];
          x[c] = f0 < 64 ? x[c] * cc - p[c] * sn : x[c] * cc + p[c] * sn;
        }
        dst = nb < epi.Hq ? epi.q_out + ((size_t)m * epi.Hq + nb) * 128
                          : epi.k_pool + (((size_t)page * epi.Hkv + (nb - epi.Hq)) * epi.page_size + off) * 128;
      } else {
        dst = epi.v_pool + (((size_t)page * epi.Hkv + (nb - epi.Hq - epi.Hkv)) * epi.page_size + off) * 128;
      }
      st_bf16x4(dst + f0, x[0], x[1], x[2], x[3]);
    }
  }
};

// Small-M (swap-AB, split-K) kernel.
//   D^T[128 features, BNX rows] = W_tile[128, K] . A[BNX, K]^T
// grid = (feature tiles, splits); each CTA does k-blocks [kb0, kb1).
template <int BNX, int RING_KB>
struct SwapCfg {
  static constexpr int W_BYTES = GEMM_BM * GEMM_BK * 2;  // 16 KB
  static constexpr int X_BYTES = BNX * GEMM_BK * 2;
  // A ring of RING_KB: 108 KB lets two CTAs share an SM (one CTA's tail then
  // overlaps the next CTA's start, and two independent streams keep twice
  // the weight bytes in flight); 72 KB leaves room for a third CTA, so the
  // next kernel's CTAs can become resident and start streaming their weights
  // while this kernel's last CTAs finish.
  static constexpr int STAGES = (RING_KB * 1024) / (W_BYTES + X_BYTES);
  static constexpr int TMEM_COLS = BNX < 32 ? 32 : BNX;
  static constexpr int SMEM = STAGES * (W_BYTES + X_BYTES) + 1024 + 256;
};

// kRowPrefetch (M > 1): the epilogue loads the per-row operands and split-K
// partials of kRowChunk rows before emitting any of them.  M == 1 launches
// the plain epilogue, a separate instantiation, so the batch-1 decode kernel
// keeps its smaller code and register count.  MODE >= 0 compiles a single
// epilogue mode (the decode instantiations, M <= 16): the kernel then holds
// only that mode's code, so a launch fetches less cold code (instruction
// fetch stalls led the 16-row epilogue's stall profile); MODE = -1 takes the
// mode from `epi` at run time.
//
// kTile (BNX == 16, 2 <= M <= 16, MODE >= 0): the tile epilogue (TileEpi)
// instead of the one-row-at-a-time one.
template <int BNX, int RING_KB, bool kRowPrefetch, int MODE = -1, bool kTile = false>
__global__ void __launch_bounds__(192, 2)
    gemm_swapab_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                       bf16* __restrict__ C, const bf16* __restrict__ bias, int M, int N, int K, int ldc,
                       int kb_per_split, float* __restrict__ ws, int* __restrict__ tickets, int* err,
                       int w_tiled, const __grid_constant__ LLSmallMEpi epi) {
  const int mode = MODE >= 0 ? MODE : epi.mode;
  using Cfg = SwapCfg<BNX, RING_KB>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * Cfg::W_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sX + STAGES * Cfg::X_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  __shared__ int s_last;
  __shared__ float s_head[GEMM_BM];  // LL_EPI_QKV_ROPE: one row of the head (rotate-half partner exchange)
  __shared__ float s_red[4];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = blockIdx.x;  // feature tile
  const int split = blockIdx.y, nsplit = gridDim.y;
  const int num_kb = (K + GEMM_BK - 1) / GEMM_BK;
  const int kb0 = split * kb_per_split;
  const int kb1 = min(num_kb, kb0 + kb_per_split);
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmW);
      prefetch_tmap(&tmX);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // The weights do not depend on the previous kernel: start streaming the
      // first ring's worth of them before waiting for it, then add the
      // activation tiles once its output is visible.
      const int pre = (kb1 - kb0) < STAGES ? (kb1 - kb0) : STAGES;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], Cfg::W_BYTES + Cfg::X_BYTES);
        if (w_tiled)  // one contiguous 16 KB tile
          tma_load_4d_(sW + i * Cfg::W_BYTES, &tmW, &full[i], 0, 0, kb0 + i, nb);
        else
          tma_load_2d(sW + i * Cfg::W_BYTES, &tmW, &full[i], (kb0 + i) * GEMM_BK, nb * GEMM_BM);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(sX + i * Cfg::X_BYTES, &tmX, &full[i], (kb0 + i) * GEMM_BK, 0);
      if (pre == STAGES) phase = 1;  // stage wrapped around exactly once
      for (int kb = kb0 + pre; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err, kErrSmemEmptyTimeout)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], Cfg::W_BYTES + Cfg::X_BYTES);
        if (w_tiled)
          tma_load_4d_(sW + stage * Cfg::W_BYTES, &tmW, &full[stage], 0, 0, kb, nb);
        else
          tma_load_2d(sW + stage * Cfg::W_BYTES, &tmW, &full[stage], kb * GEMM_BK, nb * GEMM_BM);
        tma_load_2d(sX + stage * Cfg::X_BYTES, &tmX, &full[stage], kb * GEMM_BK, 0);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) {
        unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(GEMM_BM, BNX);
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, err, kErrTmaFullTimeout)) break;
        tc_fence_after();
        const uint64_t ad = umma_desc_sw128_kmajor(smem_u32(sW + stage * Cfg::W_BYTES));
        const uint64_t bd = umma_desc_sw128_kmajor(smem_u32(sX + stage * Cfg::X_BYTES));
#pragma unroll
        for (int k = 0; k < GEMM_BK / 16; ++k)
          umma_bf16(tmem_base, ad + 2 * k, bd + 2 * k, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      umma_commit(tfull);
    }
    __syncwarp();
  } else if constexpr (kTile) {
    static_assert(BNX == 16 && MODE >= 0, "tile epilogue: 16-row kernels of one mode");
    const int q = warp & 3;
    TileEpi<MODE> te;
    te.q = q;
    te.lane = lane;
    te.f0 = 4 * lane;
    te.feat0 = nb * GEMM_BM + te.f0;
    te.m0 = 4 * q;
    pdl_wait();  // outputs / workspace may still be in use by the previous kernel
    te.prefetch(bias, M, N, K, nb, epi);
    const bool ok = bar_and_128(mbar_wait(tfull, 0, err, kErrTmemFullTimeout));
    tc_fence_after();
    // this warp's TMEM lanes: features q*32 .. q*32+31, columns = rows
    uint32_t r[32];
    tmem_ld_32x32b_x32(tmem_base + (uint32_t(q * 32) << 16), r);  // columns >= 16 unused
    tmem_ld_wait();
    float acc[4][4];
    bool emit_rows = ok;
    if (nsplit == 1) {
      // Transpose through stage 0 of the ring (every MMA that read it has
      // completed: tfull was committed after the last one).
      float* sT = reinterpret_cast<float*>(sW);
#pragma unroll
      for (int m = 0; m < 16; ++m) sT[m * GEMM_BM + q * 32 + lane] = __uint_as_float(r[m]);
      bar_sync_128();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 t = *reinterpret_cast<const float4*>(sT + (te.m0 + j) * GEMM_BM + te.f0);
        acc[j][0] = t.x, acc[j][1] = t.y, acc[j][2] = t.z, acc[j][3] = t.w;
      }
    } else {
      const int feat = nb * GEMM_BM + q * 32 + lane;
      if (feat < N) {
        float* w = ws + ((size_t)split * M) * N;
        const bool empty_split = (kb1 <= kb0);
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (m < M) w[(size_t)m * N + feat] = empty_split ? 0.f : __uint_as_float(r[m]);
      }
      // Split-K fix-up: the last CTA of this feature tile reduces all splits.
      __threadfence();
      bar_sync_128();
      if (threadIdx.x == 64) {
        const int prev = atomicAdd(&tickets[nb], 1);
        s_last = (prev == nsplit - 1);
      }
      bar_sync_128();
      emit_rows = ok && s_last;
      if (s_last) {
        __threadfence();
        const size_t sstride = (size_t)M * N;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[j][c] = 0.f;
        if (te.fvalid) {
          // four splits of the thread's four rows in flight at a time, each
          // element summed in split order
#pragma unroll 1
          for (int s0 = 0; s0 < nsplit; s0 += 4) {
            float4 part[4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int sp = 0; sp < 4; ++sp)
                part[j][sp] = (te.m0 + j < M && s0 + sp < nsplit)
                                  ? __ldcg(reinterpret_cast<const float4*>(
                                        ws + (s0 + sp) * sstride + (size_t)(te.m0 + j) * N + te.feat0))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int sp = 0; sp < 4; ++sp)
                if (s0 + sp < nsplit) {
                  acc[j][0] += part[j][sp].x;
                  acc[j][1] += part[j][sp].y;
                  acc[j][2] += part[j][sp].z;
                  acc[j][3] += part[j][sp].w;
                }
          }
        }
        if (threadIdx.x == 64) tickets[nb] = 0;  // ready for the next launch / graph replay
      }
    }
    if (emit_rows) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (te.m0 + j < M) te.emit(j, acc[j], C, ldc, M, nb, epi, err);
    }
  } else {
    const int q = warp & 3;
    const int f = q * 32 + lane;             // feature within the tile
    const int feat = nb * GEMM_BM + f;       // output column of C
    pdl_wait();  // outputs / workspace may still be in use by the previous kernel
    // Epilogue operands that do not depend on this product are loaded now,
    // while the main loop runs: per-row scalars in lane `row` (rows < 32,
    // read back with a shuffle), per-feature values and row 0's per-element
    // values in registers.  Other rows load at use.
    float pf_rstd = 1.f;
    if (epi.scale_sumsq != nullptr && lane < M)
      pf_rstd = rsqrtf(sumsq_value(__ldcg(epi.scale_sumsq + lane)) / (float)K + epi.scale_eps);
    const float pf_bias = (bias != nullptr && feat < N) ? __bfloat162float(bias[feat]) : 0.f;
    float pf_res0 = 0.f, pf_w = 0.f, pf_c0 = 0.f, pf_s0 = 0.f;
    int pf_pos = 0;
    int64_t pf_slot = 0;
    if (mode == LL_EPI_RESIDUAL && feat < N) {
      pf_res0 = __bfloat162float(epi.res[feat]);
      pf_w = __bfloat162float(epi.norm_w[feat]);
    } else if (mode == LL_EPI_QKV_ROPE) {
      if (lane < M) {
        pf_pos = epi.positions[lane];
        pf_slot = epi.slots[lane];
      }
      const int p0 = __shfl_sync(0xffffffffu, pf_pos, 0);
      if (p0 >= 0 && p0 < epi.max_pos) {  // an out-of-range row 0 is refused in the epilogue
        pf_c0 = epi.cos_sin[(size_t)p0 * 128 + (f & 63)];
        pf_s0 = epi.cos_sin[(size_t)p0 * 128 + 64 + (f & 63)];
      }
      const bf16* nw = nb < epi.Hq ? epi.q_norm_w : (nb < epi.Hq + epi.Hkv ? epi.k_norm_w : nullptr);
      if (nw != nullptr) pf_w = __bfloat162float(nw[f]);
    }
    // The four epilogue warps agree on `ok`: the epilogues below use named
    // barriers, which every one of the 128 threads must reach.
    const bool ok = bar_and_128(mbar_wait(tfull, 0, err, kErrTmemFullTimeout));
    tc_fence_after();
    const bool empty_split = (kb1 <= kb0);
    const uint32_t tbase = tmem_base + (uint32_t(q * 32) << 16);
    // Per-row operands of the epilogue (row scale, residual, position, slot,
    // RoPE cos/sin).  They are loaded for a chunk of kRowChunk rows before
    // any of those rows is emitted, so a batch of M rows waits on M /
    // kRowChunk L2 round trips instead of one per row.  Called by all 128
    // threads for the same m (the shuffles need whole warps).
    struct RowPf {
      float rs, res, c, s;
      int pos;
      int64_t slot;
    };
    auto row_pf = [&](int m) -> RowPf {
      RowPf p{1.f, 0.f, pf_c0, pf_s0, 0, 0};
      if (epi.scale_sumsq != nullptr) {
        const float rs = __shfl_sync(0xffffffffu, pf_rstd, m & 31);
        p.rs = m < 32 ? rs : (m < M ? rsqrtf(sumsq_value(__ldcg(epi.scale_sumsq + m)) / (float)K + epi.scale_eps) : 1.f);
      }
      if (mode == LL_EPI_RESIDUAL) {
        if (m < M && feat < N) p.res = m == 0 ? pf_res0 : __bfloat162float(epi.res[(size_t)m * epi.ld + feat]);
      } else if (mode == LL_EPI_QKV_ROPE) {
        const int pm0 = __shfl_sync(0xffffffffu, pf_pos, m & 31);
        const int64_t sl = __shfl_sync(0xffffffffu, pf_slot, m & 31);
        p.pos = m < 32 ? pm0 : (m < M ? epi.positions[m] : 0);
        p.slot = m < 32 ? sl : (m < M ? epi.slots[m] : 0);
        if (m > 0 && m < M && nb < epi.Hq + epi.Hkv && p.pos >= 0 && p.pos < epi.max_pos) {
          const float* cs = epi.cos_sin + (size_t)p.pos * 128;
          p.c = cs[f & 63];
          p.s = cs[64 + (f & 63)];
        }
      }
      return p;
    };
    constexpr int kRowChunk = 4;
    // Final value of (row m, feature feat), called by all 128 threads for
    // the same m.  Features past N (N % 32 == 0: whole warps) store nothing.
    auto emit = [&](int m, float v, const RowPf& p) {
      if (epi.scale_sumsq != nullptr) v *= p.rs;
      v += pf_bias;
      if (mode == LL_EPI_STORE) {
        if (feat < N) C[(size_t)m * ldc + feat] = __float2bfloat16(v);
      } else if (mode == LL_EPI_SWIGLU) {
        // gate/up interleaved in groups of 16: lanes 0-15 hold gate
        // features, lanes 16-31 the matching up features
        const float u = __shfl_down_sync(0xffffffffu, v, 16);
        if (lane < 16 && feat < N) C[(size_t)m * ldc + (feat >> 5) * 16 + lane] = __float2bfloat16(silu_f(v) * u);
      } else if (mode == LL_EPI_RESIDUAL) {
        float r = 0.f;
        if (feat < N) {
          const size_t i = (size_t)m * epi.ld + feat;
          r = bf16_round(v) + p.res;
          epi.res[i] = __float2bfloat16(r);
          epi.h_out[i] = __float2bfloat16(r * pf_w);
        }
        const float ss = warp_sum(r * r);
        if (lane == 0) atomicAdd(epi.sumsq_out + m, __float2ull_rn(ss * LL_SUMSQ_ONE));
      } else {  // LL_EPI_QKV_ROPE: this tile is head nb of [Hq | Hkv keys | Hkv values]
        float x = bf16_round(v);
        const int64_t slot = p.slot;
        const int pos_m = p.pos;
        // checked per row (the same for all 128 threads, so the barriers
        // below stay uniform): a bad slot or position is recorded, not written
        if (slot < 0 || slot >= epi.slot_limit || pos_m < 0 || pos_m >= epi.max_pos) {
          if (threadIdx.x == 64) record_error(err, kErrBadIndex);
          return;
        }
        const int64_t page = slot / epi.page_size, off = slot % epi.page_size;
        bf16* dst;
        if (nb < epi.Hq + epi.Hkv) {
          const bf16* nw = nb < epi.Hq ? epi.q_norm_w : epi.k_norm_w;
          if (nw != nullptr) {
            const float ss = warp_sum(x * x);
            if (lane == 0) s_red[q] = ss;
            bar_sync_128();
            const float tot = (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]);
            x = x * rsqrtf(tot / 128.f + epi.eps) * pf_w;
          }
          s_head[f] = x;
          bar_sync_128();
          const float c = p.c, sn = p.s;
          x = f < 64 ? x * c - s_head[f + 64] * sn : x * c + s_head[f - 64] * sn;
          bar_sync_128();  // s_head / s_red are free for the next row
          dst = nb < epi.Hq ? epi.q_out + ((size_t)m * epi.Hq + nb) * 128
                            : epi.k_pool + (((size_t)page * epi.Hkv + (nb - epi.Hq)) * epi.page_size + off) * 128;
        } else {
          dst = epi.v_pool + (((size_t)page * epi.Hkv + (nb - epi.Hq - epi.Hkv)) * epi.page_size + off) * 128;
        }
        dst[f] = __float2bfloat16(x);
      }
    };
#pragma unroll 1
    for (int c = 0; c < BNX; c += 32) {
      uint32_t r[32];
      if constexpr (BNX >= 32) {
        tmem_ld_32x32b_x32(tbase + c, r);
      } else {
        tmem_ld_32x32b_x32(tbase, r);  // columns >= BNX hold garbage; ignored
      }
      tmem_ld_wait();
      if (!ok) continue;
      const int ncols = BNX < 32 ? BNX : 32;
      if (nsplit == 1) {
        if constexpr (kRowPrefetch) {
#pragma unroll
          for (int i0 = 0; i0 < ncols; i0 += kRowChunk) {
            if (c + i0 >= M) break;
            RowPf pf[kRowChunk];
#pragma unroll
            for (int j = 0; j < kRowChunk; ++j) pf[j] = row_pf(c + i0 + j);
#pragma unroll
            for (int j = 0; j < kRowChunk; ++j)
              if (i0 + j < ncols && c + i0 + j < M) emit(c + i0 + j, __uint_as_float(r[i0 + j]), pf[j]);
          }
        } else {
          for (int i = 0; i < ncols && c + i < M; ++i) emit(c + i, __uint_as_float(r[i]), row_pf(c + i));
        }
      } else if (feat < N) {
        float* w = ws + ((size_t)split * M) * N;
        for (int i = 0; i < ncols; ++i) {
          const int m = c + i;
          if (m < M) w[(size_t)m * N + feat] = empty_split ? 0.f : __uint_as_float(r[i]);
        }
      }
    }
    if (nsplit > 1) {
      // Split-K fix-up: the last CTA of this feature tile reduces all splits.
      __threadfence();
      bar_sync_128();
      if (threadIdx.x == 64) {
        const int prev = atomicAdd(&tickets[nb], 1);
        s_last = (prev == nsplit - 1);
      }
      bar_sync_128();
      if (s_last) {
        __threadfence();
        const size_t sstride = (size_t)M * N;
        if constexpr (!kRowPrefetch) {
          for (int m = 0; m < M; ++m) {
            // all partials in flight at once, then summed in split order
            float part[16];
            const float* src = ws + (size_t)m * N + feat;
#pragma unroll
            for (int sp = 0; sp < 16; ++sp) part[sp] = (sp < nsplit && feat < N) ? __ldcg(src + sp * sstride) : 0.f;
            float sum = 0.f;
#pragma unroll
            for (int sp = 0; sp < 16; ++sp) sum += part[sp];
            for (int sp = 16; sp < nsplit; ++sp)
              if (feat < N) sum += __ldcg(src + sp * sstride);
            if (ok) emit(m, sum, row_pf(m));
          }
        } else {
#pragma unroll 1
        for (int m0 = 0; m0 < M; m0 += kRowChunk) {
          // the partials of kRowChunk rows and their epilogue operands are
          // all in flight at once; each row is then summed in split order
          float part[kRowChunk][16];
#pragma unroll
          for (int j = 0; j < kRowChunk; ++j) {
            const float* src = ws + (size_t)(m0 + j) * N + feat;
#pragma unroll
            for (int sp = 0; sp < 16; ++sp)
              part[j][sp] = (m0 + j < M && sp < nsplit && feat < N) ? __ldcg(src + sp * sstride) : 0.f;
          }
          RowPf pf[kRowChunk];
#pragma unroll
          for (int j = 0; j < kRowChunk; ++j) pf[j] = row_pf(m0 + j);
#pragma unroll
          for (int j = 0; j < kRowChunk; ++j) {
            const int m = m0 + j;
            if (m >= M) break;
            const float* src = ws + (size_t)m * N + feat;
            float sum = 0.f;
#pragma unroll
            for (int sp = 0; sp < 16; ++sp) sum += part[j][sp];
            for (int sp = 16; sp < nsplit; ++sp)
              if (feat < N) sum += __ldcg(src + sp * sstride);
            if (ok) emit(m, sum, pf[j]);
          }
        }
        }
        if (threadIdx.x == 64) tickets[nb] = 0;  // ready for the next launch / graph replay
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
}

// ---------------------------------------------------------------------------
// 2-SM variant (cta_group::2): a cluster of two CTAs computes a 256 x BN
// tile.  CTA r of the pair loads A rows [128r, 128r+128) and B rows
// [BN/2 * r, BN/2 * (r+1)) of the tile into its own shared memory; the
// leader (r = 0) issues tcgen05.mma.cta_group::2 (M=256, N=BN, K=16), which
// reads both CTAs' operands and accumulates rows [128r, 128r+128) into CTA
// r's TMEM.  Per SM this moves 32 KB of operands per 64-deep k-block instead
// of 48 KB for the same FLOPs, so a 6-deep ring hides more load latency.
// Both CTAs' TMA loads complete on the leader's `full` barrier; the leader's
// commits arrive on both CTAs' `empty` / `tfull` barriers (commit multicast);
// the epilogue warps of both CTAs release an accumulator on the leader's
// `tempty` barrier.  No TMA load uses cluster multicast.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tma_load_2d_2sm(void* smem_dst, const void* tmap, uint32_t leader_bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void umma_bf16_2sm(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrive on the barrier at this offset in both CTAs of the pair once every
// MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit_2sm_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}

__device__ __forceinline__ void umma_commit_2sm_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Bulk tensor store of a shared-memory box to global memory (bulk-group
// completion), and the waits on this thread's outstanding groups.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_group_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One warp's 32-row x 64-byte box of C (32 bf16 columns per row) staged for
// a bulk tensor store: lane = row, `v` its 16 packed bf16 pairs; 16-byte chunk
// k of row r lands at chunk k ^ ((r >> 1) & 3) (the 64-byte swizzle the
// store's tensor map names), so the four st.shared.v4 of a quarter-warp hit
// distinct banks.
__device__ __forceinline__ void epi_stage_row64(uint8_t* box, int lane, const uint32_t (&v)[16]) {
  uint4* row = reinterpret_cast<uint4*>(box + lane * 64);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    row[k ^ ((lane >> 1) & 3)] = make_uint4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}

template <int EPI>
__device__ __forceinline__ void epi_store_chunk(const uint32_t (&r)[32], bf16* __restrict__ C,
                                                const bf16* __restrict__ bias, int row, int col0, int M, int N,
                                                int ldc) {
  if (row >= M || col0 >= N) return;
  if constexpr (EPI == kEpiSwiGLU) {
    bf16* dst = C + (size_t)row * ldc + (col0 >> 1);
    uint32_t packed[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float g0 = __uint_as_float(r[2 * i]), g1 = __uint_as_float(r[2 * i + 1]);
      float u0 = __uint_as_float(r[16 + 2 * i]), u1 = __uint_as_float(r[16 + 2 * i + 1]);
      if (bias != nullptr) {
        g0 += __bfloat162float(bias[col0 + 2 * i]);
        g1 += __bfloat162float(bias[col0 + 2 * i + 1]);
        u0 += __bfloat162float(bias[col0 + 16 + 2 * i]);
        u1 += __bfloat162float(bias[col0 + 16 + 2 * i + 1]);
      }
      packed[i] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    d4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    d4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  } else {
    bf16* dst = C + (size_t)row * ldc + col0;
    if (col0 + 32 <= N) {
      uint32_t packed[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float a0 = __uint_as_float(r[2 * i]), a1 = __uint_as_float(r[2 * i + 1]);
        if (bias != nullptr) {
          a0 += __bfloat162float(bias[col0 + 2 * i]);
          a1 += __bfloat162float(bias[col0 + 2 * i + 1]);
        }
        packed[i] = pack_bf16x2(a0, a1);
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
    } else {
      for (int i = 0; i < 32 && col0 + i < N; ++i) {
        float a = __uint_as_float(r[i]);
        if (bias != nullptr) a += __bfloat162float(bias[col0 + i]);
        dst[i] = __float2bfloat16(a);
      }
    }
  }
}

template <int BN>
struct Gemm2Cfg {
  static constexpr int STAGES = 6;
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;       // this CTA's 128 rows of A
  static constexpr int B_BYTES = (BN / 2) * GEMM_BK * 2;      // this CTA's half of the B tile
  static constexpr int TMEM_COLS = 2 * BN;
  // epilogue staging: 4 warps x 2 buffers x one 32-row x 64-byte box
  static constexpr int EPI_BYTES = 4 * 2 * 32 * 64;
  static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES) + EPI_BYTES + 1024 + 256;
};

template <int BN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_tcgen05_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmC, int c_bulk, bf16* __restrict__ C,
                            const bf16* __restrict__ bias, int M, int N, int K, int ldc, int* err,
                            const __grid_constant__ TpArgs tp, int group_m) {
  using Cfg = Gemm2Cfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sEpi = sB + STAGES * Cfg::B_BYTES;  // [4 warps][2][32 rows x 64 B], 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + Cfg::EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m = (M + 2 * GEMM_BM - 1) / (2 * GEMM_BM);
  const int num_n = (N + BN - 1) / BN;
  const int ntiles = num_m * num_n;
  const int num_kb = (K + GEMM_BK - 1) / GEMM_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // 4 epilogue warps x 2 CTAs (used on the leader)
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)Cfg::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      if (tp.wait_cnt != nullptr) {
        ok = wait_counter_geq(tp.wait_cnt, tp.wait_target, err);
        fence_proxy_async_global();  // peers' generic stores -> this CTA's TMA (async proxy) reads
      }
      for (int t = pair; t < ntiles && ok; t += npairs) {
        int mb, nb;
        tile_coords(t, num_m, num_n, group_m, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, err, kErrSmemEmptyTimeout)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = mapa_shared(smem_u32(&full[stage]), 0);
          if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
          tma_load_2d_2sm(sA + stage * Cfg::A_BYTES, &tmA, leader_full, kb * GEMM_BK,
                          mb * 2 * GEMM_BM + (int)crank * GEMM_BM);
          tma_load_2d_2sm(sB + stage * Cfg::B_BYTES, &tmB, leader_full, kb * GEMM_BK,
                          nb * BN + (int)crank * (BN / 2));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && crank == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(2 * GEMM_BM, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, aphase = 0;
      bool ok = true;
      for (int t = pair; t < ntiles && ok; t += npairs) {
        if (!mbar_wait(&tempty[acc], aphase ^ 1, err, kErrTmemEmptyTimeout)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, kErrTmaFullTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128_kmajor(smem_u32(sA + stage * Cfg::A_BYTES));
          const uint64_t bd = umma_desc_sw128_kmajor(smem_u32(sB + stage * Cfg::B_BYTES));
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k)
            umma_bf16_2sm(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit_2sm_both(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_2sm_both(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          aphase ^= 1;
        }
      }
      umma_commit_2sm_local(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const uint32_t leader_tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t leader_tempty1 = mapa_shared(smem_u32(&tempty[1]), 0);
    int acc = 0;
    uint32_t aphase = 0;
    // kEpiScatter: slices stored per owner rank, published once at the end
    // (one system fence per warp instead of one per tile).
    uint32_t sent[LL_MAX_TP_RANKS] = {0, 0, 0, 0, 0, 0, 0, 0};
    int nbox = 0;  // bulk-stored boxes of this warp (c_bulk)
    for (int t = pair; t < ntiles; t += npairs) {
      int mb, nb;
        tile_coords(t, num_m, num_n, group_m, mb, nb);
      if (!mbar_wait(&tfull[acc], aphase, err, kErrTmemFullTimeout)) break;
      tc_fence_after();
      const int row0 = mb * 2 * GEMM_BM + (int)crank * GEMM_BM + q * 32;  // this warp's 32-row slice
      const int row = row0 + lane;
      const uint32_t tbase = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN);
      if constexpr (EPI == kEpiScatter) {
        // rows_per_rank is a multiple of 32, so the slice has one owner.
        // The owner's slot for this rank is tiled: [R/32][N/32] tiles of 32
        // rows x 32 columns, each tile 2 KB contiguous, so the warp's chunk
        // (its 32 rows x 32 columns) is one contiguous 2 KB run.  The chunk
        // goes through the warp's shared-memory box (lane = row, 64-byte
        // swizzle) and is read back so that in store k the warp writes rows
        // 8k..8k+7 -- 512 contiguous bytes per NVLink store instruction.
        const int d = row0 / tp.rows_per_rank;
        const int R = tp.rows_per_rank;
        bf16* slot_rows = row0 < M ? static_cast<bf16*>(tp.slot[d]) + (size_t)tp.rank * R * N +
                                         (size_t)((row0 - d * R) >> 5) * (size_t)(N >> 5) * 1024
                                   : nullptr;
        uint8_t* box = sEpi + q * 2 * 2048;
        const int q4 = lane & 3, rw = lane >> 2;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          const int col0 = nb * BN + c;
          if (slot_rows == nullptr || col0 >= N) continue;  // warp-uniform
          uint32_t p[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) p[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
          __syncwarp();  // the previous chunk's reads of the box are done
          epi_stage_row64(box, lane, p);
          __syncwarp();
          bf16* tile = slot_rows + (size_t)(col0 >> 5) * 1024;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int row = 8 * k + rw;
            const uint4 v = *reinterpret_cast<const uint4*>(box + row * 64 + ((q4 ^ ((row >> 1) & 3)) << 4));
            *reinterpret_cast<uint4*>(tile + row * 32 + 8 * q4) = v;
          }
        }
        if (row0 < M) {
#pragma unroll
          for (int i = 0; i < LL_MAX_TP_RANKS; ++i) sent[i] += (i == d) ? 1u : 0u;
        }
      } else if (c_bulk) {
        // TMEM -> registers (bias, SwiGLU, bf16) -> a swizzled 32 x 64-byte
        // box in shared memory -> one bulk tensor store per box, issued by
        // lane 0: every global write is a whole 64-byte row segment instead
        // of 16 bytes of 32 different rows.  The warp alternates two boxes
        // and reuses one once the store before last has read it.  Rows past
        // M and columns past N are clipped by the store.
        uint8_t* boxes = sEpi + q * 2 * 2048;
        const int row0w = mb * 2 * GEMM_BM + (int)crank * GEMM_BM + q * 32;
        constexpr int STEP = EPI == kEpiSwiGLU ? 64 : 32;  // accumulator columns per box
#pragma unroll 1
        for (int c = 0; c < BN; c += STEP) {
          const int col0 = nb * BN + c;
          uint32_t v[16];
          if constexpr (EPI == kEpiSwiGLU) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t r[32];
              tmem_ld_32x32b_x32(tbase + c + 32 * hh, r);
              tmem_ld_wait();
              const int cb = col0 + 32 * hh;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                float g0 = __uint_as_float(r[2 * i]), g1 = __uint_as_float(r[2 * i + 1]);
                float u0 = __uint_as_float(r[16 + 2 * i]), u1 = __uint_as_float(r[16 + 2 * i + 1]);
                if (bias != nullptr && cb < N) {  // N % 32 == 0: a 32-column group is wholly in or out
                  g0 += __bfloat162float(bias[cb + 2 * i]);
                  g1 += __bfloat162float(bias[cb + 2 * i + 1]);
                  u0 += __bfloat162float(bias[cb + 16 + 2 * i]);
                  u1 += __bfloat162float(bias[cb + 16 + 2 * i + 1]);
                }
                v[8 * hh + i] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
              }
            }
          } else {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tbase + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float a0 = __uint_as_float(r[2 * i]), a1 = __uint_as_float(r[2 * i + 1]);
              if (bias != nullptr) {
                if (col0 + 2 * i < N) a0 += __bfloat162float(bias[col0 + 2 * i]);
                if (col0 + 2 * i + 1 < N) a1 += __bfloat162float(bias[col0 + 2 * i + 1]);
              }
              v[i] = pack_bf16x2(a0, a1);
            }
          }
          if (col0 >= N || row0w >= M) continue;  // warp-uniform: the box is wholly outside C
          uint8_t* box = boxes + (nbox & 1) * 2048;
          if (nbox >= 2 && lane == 0) bulk_wait_group_read1();
          __syncwarp();
          epi_stage_row64(box, lane, v);
          fence_proxy_async();  // this lane's shared writes -> the bulk copy (async proxy)
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, box, EPI == kEpiSwiGLU ? col0 / 2 : col0, row0w);
            bulk_commit_group();
          }
          ++nbox;
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          epi_store_chunk<EPI>(r, C, bias, row, nb * BN + c, M, N, ldc);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc == 0 ? leader_tempty0 : leader_tempty1);
      if (++acc == 2) {
        acc = 0;
        aphase ^= 1;
      }
    }
    if (lane == 0 && nbox > 0) bulk_wait_group0();  // this warp's bulk stores are complete
    if constexpr (EPI == kEpiScatter) {
      __threadfence_system();  // this lane's peer stores are visible system-wide
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < LL_MAX_TP_RANKS; ++i)
          if (i < tp.world && sent[i] != 0) red_release_sys_add(tp.cnt[i], (unsigned long long)sent[i]);
      }
    }
  }

  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"((uint32_t)Cfg::TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host side.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix (cols contiguous),
// box = [box_rows, 64 cols], 128-byte swizzle, zero fill out of bounds.
static int make_tmap_2d(CUtensorMap* tm, const void* ptr, int rows, int cols, int ld, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// Store map of C for the bulk-store epilogue: box of 32 rows x 32 bf16
// columns (64 bytes) with the 64-byte swizzle.  Returns 0 when C qualifies
// (16-byte aligned base and row pitch).
static int make_tmap_c(CUtensorMap* tm, const void* ptr, int rows, int cols, int ld) {
  if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15) || (ld % 8)) return -3;
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// Bulk-store epilogue: LL_GEMM_BULK_STORE=1 selects it, 0 the per-thread
// stores; unset: kGemmBulkStoreDefault.
constexpr int kGemmBulkStoreDefault = 1;
static bool gemm_bulk_store_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("LL_GEMM_BULK_STORE");
    v = e != nullptr && e[0] != '\0' ? (e[0] == '0' ? 0 : 1) : kGemmBulkStoreDefault;
  }
  return v == 1;
}

// m-blocks per tile group: as many as keep the group's A rows (block_rows x
// K bf16 each) within ~40 MB of L2, at least 8; LL_GEMM_GROUP_M=<n> fixes it.
static int gemm_group_m(int M, int K, int block_rows) {
  static int fixed = -1;
  if (fixed < 0) {
    const char* e = getenv("LL_GEMM_GROUP_M");
    fixed = e != nullptr ? atoi(e) : 0;
    if (fixed < 0) fixed = 0;
  }
  const int num_m = (M + block_rows - 1) / block_rows;
  int g = fixed;
  if (g == 0) {
    const double per_block = (double)block_rows * (double)K * 2.0;
    g = (int)((40.0 * 1024 * 1024) / per_block);
    if (g < GEMM_GROUP_M) g = GEMM_GROUP_M;
  }
  if (g > num_m) g = num_m;
  return g < 1 ? 1 : g;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

static int max_smem_optin() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  }
  return n;
}

template <typename Kern>
static void set_smem(Kern k, int bytes) {
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace ll

using namespace ll;

// Returns 0 on success, <0 on a host-side error (bad shape / tensor map).
extern "C" int ll_gemm_bf16(const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc, const bf16* bias,
                            int M, int N, int K, int epilogue, int bn, int* err, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((K % 8) || (lda % 8) || (ldw % 8)) return -3;
  if (epilogue == kEpiSwiGLU && (N % 32)) return -4;
  CUtensorMap tA, tB;
  const int BN = (bn == 128) ? 128 : 256;
  if (BN == 256 && M > 2 * GEMM_BM) {
    // 2-SM tiles (256 x 256 per CTA pair).
    if (make_tmap_2d(&tA, A, M, K, lda, GEMM_BM)) return -2;
    if (make_tmap_2d(&tB, W, N, K, ldw, BN / 2)) return -2;
    const int ntiles2 = ((M + 2 * GEMM_BM - 1) / (2 * GEMM_BM)) * ((N + BN - 1) / BN);
    const int pairs = ntiles2 < num_sms() / 2 ? ntiles2 : num_sms() / 2;
    CUtensorMap tC;
    const int c_bulk = gemm_bulk_store_enabled() &&
                       make_tmap_c(&tC, C, M, epilogue == kEpiSwiGLU ? N / 2 : N, ldc) == 0;
    if (!c_bulk) tC = tA;  // not read
#define LL_LAUNCH2(EPI_)                                                                              \
  do {                                                                                                \
    auto kern = gemm_tcgen05_2sm_kernel<256, EPI_>;                                                   \
    if (Gemm2Cfg<256>::SMEM > max_smem_optin()) return -7;                                            \
    static bool init = false;                                                                         \
    if (!init) {                                                                                      \
      set_smem(kern, Gemm2Cfg<256>::SMEM);                                                            \
      init = true;                                                                                    \
    }                                                                                                 \
    kern<<<2 * pairs, 192, Gemm2Cfg<256>::SMEM, stream>>>(tA, tB, tC, c_bulk, C, bias, M, N, K, ldc, err, \
                                                           TpArgs{}, gemm_group_m(M, K, 2 * GEMM_BM)); \
  } while (0)
    if (epilogue == kEpiSwiGLU) LL_LAUNCH2(kEpiSwiGLU); else LL_LAUNCH2(kEpiPlain);
#undef LL_LAUNCH2
    return cudaGetLastError() == cudaSuccess ? 0 : -5;
  }
  if (make_tmap_2d(&tA, A, M, K, lda, GEMM_BM)) return -2;
  if (make_tmap_2d(&tB, W, N, K, ldw, BN)) return -2;
  const int ntiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + BN - 1) / BN);
  const int grid = ntiles < num_sms() ? ntiles : num_sms();
#define LL_LAUNCH(BN_, EPI_)                                                                          \
  do {                                                                                                \
    auto kern = gemm_tcgen05_kernel<BN_, EPI_>;                                                       \
    if (GemmCfg<BN_>::SMEM > max_smem_optin()) return -7;                                             \
    static bool init = false;                                                                         \
    if (!init) {                                                                                      \
      set_smem(kern, GemmCfg<BN_>::SMEM);                                                             \
      init = true;                                                                                    \
    }                                                                                                 \
    kern<<<grid, 192, GemmCfg<BN_>::SMEM, stream>>>(tA, tB, C, bias, M, N, K, ldc, err,               \
                                                    gemm_group_m(M, K, GEMM_BM));                   \
  } while (0)
  if (BN == 256) {
    if (epilogue == kEpiSwiGLU) LL_LAUNCH(256, kEpiSwiGLU); else LL_LAUNCH(256, kEpiPlain);
  } else {
    if (epilogue == kEpiSwiGLU) LL_LAUNCH(128, kEpiSwiGLU); else LL_LAUNCH(128, kEpiPlain);
  }
#undef LL_LAUNCH
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

extern "C" int ll_gemm_small_m_splits(int N, int K);

// Tensor-parallel GEMM on the 2-SM kernel: `tp` carries the optional wait on
// the all-gathered A and, for epilogue kEpiScatter, the owners' slot buffers
// and counters.  Requires M > 256; kEpiScatter also needs
// M == world * rows_per_rank with rows_per_rank a multiple of 32.
extern "C" int ll_gemm_bf16_tp(const void* A_, int lda, const void* W_, int ldw, void* C_, int ldc, const void* bias_,
                               int M, int N, int K, int epilogue, const LLTpArgs* tp, int* err, void* stream_) {
  const bf16* A = static_cast<const bf16*>(A_);
  const bf16* W = static_cast<const bf16*>(W_);
  bf16* C = static_cast<bf16*>(C_);
  const bf16* bias = static_cast<const bf16*>(bias_);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (M <= 2 * GEMM_BM || N <= 0 || K <= 0) return -3;
  if ((K % 8) || (lda % 8) || (ldw % 8) || (ldc % 8)) return -3;
  if (epilogue == kEpiSwiGLU && (N % 32)) return -4;
  if (epilogue == kEpiScatter &&
      (tp->world < 1 || tp->world > LL_MAX_TP_RANKS || tp->rows_per_rank % 32 || M != tp->world * tp->rows_per_rank ||
       N % 32 || bias_ != nullptr))
    return -4;
  CUtensorMap tA, tB;
  if (make_tmap_2d(&tA, A, M, K, lda, GEMM_BM)) return -2;
  if (make_tmap_2d(&tB, W, N, K, ldw, 128)) return -2;
  const int ntiles2 = ((M + 2 * GEMM_BM - 1) / (2 * GEMM_BM)) * ((N + 255) / 256);
  const int pairs = ntiles2 < num_sms() / 2 ? ntiles2 : num_sms() / 2;
  if (Gemm2Cfg<256>::SMEM > max_smem_optin()) return -7;
  // The scatter epilogue stores into peers' slot buffers with per-thread
  // stores; the local outputs take the bulk-store epilogue.
  CUtensorMap tC;
  const int c_bulk = epilogue != kEpiScatter && gemm_bulk_store_enabled() &&
                     make_tmap_c(&tC, C, M, epilogue == kEpiSwiGLU ? N / 2 : N, ldc) == 0;
  if (!c_bulk) tC = tA;  // not read
#define LL_LAUNCH_TP(EPI_)                                                                            \
  do {                                                                                                \
    auto kern = gemm_tcgen05_2sm_kernel<256, EPI_>;                                                   \
    static bool init = false;                                                                         \
    if (!init) {                                                                                      \
      set_smem(kern, Gemm2Cfg<256>::SMEM);                                                            \
      init = true;                                                                                    \
    }                                                                                                 \
    kern<<<2 * pairs, 192, Gemm2Cfg<256>::SMEM, stream>>>(tA, tB, tC, c_bulk, C, bias, M, N, K, ldc, err, \
                                                           *tp, gemm_group_m(M, K, 2 * GEMM_BM));    \
  } while (0)
  if (epilogue == kEpiSwiGLU) LL_LAUNCH_TP(kEpiSwiGLU);
  else if (epilogue == kEpiScatter) LL_LAUNCH_TP(kEpiScatter);
  else LL_LAUNCH_TP(kEpiPlain);
#undef LL_LAUNCH_TP
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

// Tile-major weights: W stored as [N/128][K/64][128][64] so that every TMA
// box of the small-M kernel is one contiguous 16 KB block (row-major W reads
// 128 rows x 128 B scattered by the row pitch).
static int make_tmap_w_tiled(CUtensorMap* tm, const void* ptr, int N, int K) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[4] = {64, 128, (cuuint64_t)(K / 64), (cuuint64_t)(N / 128)};
  cuuint64_t strides[3] = {128, 16384, (cuuint64_t)16384 * (K / 64)};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

extern "C" int ll_gemm_bf16_small_m_ex(const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc,
                                       const bf16* bias, int M, int N, int K, int splits, float* ws,
                                       size_t ws_floats, int* tickets, int* err, int flags, cudaStream_t stream);

// Small-M path.  ws must hold splits*M*N floats, tickets ceil(N/128) ints
// (zero-initialised once; the kernel leaves them zero).  splits <= 0 picks a
// split count that puts about one CTA on every SM.
extern "C" int ll_gemm_bf16_small_m(const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc,
                                    const bf16* bias, int M, int N, int K, int splits, float* ws, size_t ws_floats,
                                    int* tickets, int* err, cudaStream_t stream) {
  return ll_gemm_bf16_small_m_ex(A, lda, W, ldw, C, ldc, bias, M, N, K, splits, ws, ws_floats, tickets, err, 0,
                                 stream);
}

// Shared-memory ring of the small-M kernel in KB: 108 (default) or 72
// (LL_GEMV_RING_KB=72: three CTAs fit on an SM).
static int small_m_ring_kb() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("LL_GEMV_RING_KB");
    v = (e != nullptr && atoi(e) == 72) ? 72 : 108;
  }
  return v;
}

// LL_GEMV_MODE_KERNELS=0 launches the runtime-mode decode kernels instead of
// the per-mode ones (an A/B switch; default on).
static bool small_m_mode_kernels() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("LL_GEMV_MODE_KERNELS");
    v = (e != nullptr && atoi(e) == 0) ? 0 : 1;
  }
  return v == 1;
}

// LL_GEMV_TILE_EPI=0 keeps 2..16-row launches on the one-row-at-a-time
// epilogue (an A/B switch; default: the tile epilogue).
static bool small_m_tile_epi() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("LL_GEMV_TILE_EPI");
    v = (e != nullptr && atoi(e) == 0) ? 0 : 1;
  }
  return v == 1;
}

static bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Whether a 2..16-row launch meets the tile epilogue's vector widths: four
// consecutive features per thread (8-byte bf16 and 16-byte fp32 accesses).
static bool small_m_tile_ok(const bf16* C, int ldc, const bf16* bias, int M, int N, const float* ws,
                            const LLSmallMEpi& epi) {
  if (M < 2 || M > 16 || (N % 32) || !aligned_to(ws, 16) || !aligned_to(bias, 8)) return false;
  switch (epi.mode) {
    case LL_EPI_STORE:
    case LL_EPI_SWIGLU:
      return (ldc % 4) == 0 && aligned_to(C, 8);
    case LL_EPI_RESIDUAL:
      return (epi.ld % 4) == 0 && aligned_to(epi.res, 8) && aligned_to(epi.h_out, 8) && aligned_to(epi.norm_w, 8);
    case LL_EPI_QKV_ROPE:
      return aligned_to(epi.q_out, 8) && aligned_to(epi.k_pool, 8) && aligned_to(epi.v_pool, 8) &&
             aligned_to(epi.q_norm_w, 8) && aligned_to(epi.k_norm_w, 8) && aligned_to(epi.cos_sin, 16);
    default:
      return false;
  }
}

static int small_m_launch(const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc, const bf16* bias, int M,
                          int N, int K, int splits, float* ws, size_t ws_floats, int* tickets, int* err, int w_tiled,
                          const LLSmallMEpi& epi, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (M > 128) return -3;
  if ((K % 8) || (lda % 8) || (ldw % 8)) return -3;
  if (w_tiled && ((N % 128) || (K % 64))) return -3;
  switch (epi.mode) {
    case LL_EPI_STORE:
      if (C == nullptr) return -3;
      break;
    case LL_EPI_SWIGLU:
      if (C == nullptr || (N % 32)) return -3;
      break;
    case LL_EPI_RESIDUAL:
      if ((N % 32) || epi.res == nullptr || epi.norm_w == nullptr || epi.h_out == nullptr ||
          epi.sumsq_out == nullptr || epi.ld < N)
        return -3;
      break;
    case LL_EPI_QKV_ROPE:
      if (N != (epi.Hq + 2 * epi.Hkv) * GEMM_BM || epi.Hq <= 0 || epi.Hkv <= 0 || epi.page_size <= 0 ||
          epi.positions == nullptr || epi.slots == nullptr || epi.cos_sin == nullptr || epi.q_out == nullptr ||
          epi.k_pool == nullptr || epi.v_pool == nullptr || epi.slot_limit <= 0 || epi.max_pos <= 0)
        return -3;
      break;
    default:
      return -3;
  }
  const int ntiles = (N + GEMM_BM - 1) / GEMM_BM;
  const int num_kb = (K + GEMM_BK - 1) / GEMM_BK;
  if (splits <= 0) {
    splits = ll_gemm_small_m_splits(N, K);
    // 2..16 rows (the tile epilogue): at most 8 splits, the cap that
    // ops._small_m_splits applies, so both routes sum in the same order
    if (M > 1 && M <= 16 && splits > 8) splits = 8;
  }
  int kb_per = (num_kb + splits - 1) / splits;
  splits = (num_kb + kb_per - 1) / kb_per;
  if (splits > 1 && (ws == nullptr || tickets == nullptr || ws_floats < (size_t)splits * M * N)) return -6;
  const int BNX = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
  CUtensorMap tW, tX;
  if (w_tiled ? make_tmap_w_tiled(&tW, W, N, K) : make_tmap_2d(&tW, W, N, K, ldw, GEMM_BM)) return -2;
  if (make_tmap_2d(&tX, A, M, K, lda, BNX)) return -2;
  dim3 grid(ntiles, splits);
#define LL_LAUNCH_SMT(BNX_, RING_, PF_, MODE_, TILE_)                                                    \
  do {                                                                                                   \
    auto kern = gemm_swapab_kernel<BNX_, RING_, PF_, MODE_, TILE_>;                                      \
    using C_ = SwapCfg<BNX_, RING_>;                                                                     \
    if (C_::SMEM > max_smem_optin()) return -7;                                                          \
    static bool init = false;                                                                            \
    if (!init) {                                                                                         \
      set_smem(kern, C_::SMEM);                                                                          \
      init = true;                                                                                       \
    }                                                                                                    \
    launch_pdl(kern, grid, dim3(192), C_::SMEM, stream, tW, tX, C, bias, M, N, K, ldc, kb_per, ws, tickets, \
               err, w_tiled, epi);                                                                       \
  } while (0)
#define LL_LAUNCH_SM(BNX_, RING_, PF_, MODE_) LL_LAUNCH_SMT(BNX_, RING_, PF_, MODE_, false)
#define LL_LAUNCH_S(BNX_, RING_, PF_) LL_LAUNCH_SM(BNX_, RING_, PF_, -1)
// 2..16 rows on the tile epilogue, one instantiation per mode
#define LL_LAUNCH_T16()                                                                  \
  do {                                                                                   \
    switch (epi.mode) {                                                                  \
      case LL_EPI_STORE: LL_LAUNCH_SMT(16, 108, true, LL_EPI_STORE, true); break;       \
      case LL_EPI_SWIGLU: LL_LAUNCH_SMT(16, 108, true, LL_EPI_SWIGLU, true); break;     \
      case LL_EPI_RESIDUAL: LL_LAUNCH_SMT(16, 108, true, LL_EPI_RESIDUAL, true); break; \
      default: LL_LAUNCH_SMT(16, 108, true, LL_EPI_QKV_ROPE, true); break;              \
    }                                                                                    \
  } while (0)
// the decode sizes (M <= 16) on the default ring: one instantiation per epilogue mode
#define LL_LAUNCH_S16(PF_)                                     \
  do {                                                         \
    switch (epi.mode) {                                        \
      case LL_EPI_STORE: LL_LAUNCH_SM(16, 108, PF_, LL_EPI_STORE); break;       \
      case LL_EPI_SWIGLU: LL_LAUNCH_SM(16, 108, PF_, LL_EPI_SWIGLU); break;     \
      case LL_EPI_RESIDUAL: LL_LAUNCH_SM(16, 108, PF_, LL_EPI_RESIDUAL); break; \
      default: LL_LAUNCH_SM(16, 108, PF_, LL_EPI_QKV_ROPE); break;              \
    }                                                          \
  } while (0)
  if (small_m_ring_kb() == 72) {
    switch (BNX) {
      case 16:
        if (M == 1) LL_LAUNCH_S(16, 72, false);
        else LL_LAUNCH_S(16, 72, true);
        break;
      case 32: LL_LAUNCH_S(32, 72, true); break;
      case 64: LL_LAUNCH_S(64, 72, true); break;
      default: LL_LAUNCH_S(128, 72, true); break;
    }
  } else {
    switch (BNX) {
      case 16:
        if (small_m_mode_kernels()) {
          if (M == 1) LL_LAUNCH_S16(false);
          else if (small_m_tile_epi() && small_m_tile_ok(C, ldc, bias, M, N, ws, epi)) LL_LAUNCH_T16();
          else LL_LAUNCH_S16(true);
        } else if (M == 1) {
          LL_LAUNCH_S(16, 108, false);
        } else {
          LL_LAUNCH_S(16, 108, true);
        }
        break;
      case 32: LL_LAUNCH_S(32, 108, true); break;
      case 64: LL_LAUNCH_S(64, 108, true); break;
      default: LL_LAUNCH_S(128, 108, true); break;
    }
  }
#undef LL_LAUNCH_T16
#undef LL_LAUNCH_S16
#undef LL_LAUNCH_S
#undef LL_LAUNCH_SM
#undef LL_LAUNCH_SMT
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

// Same, with flags: LL_SMALL_M_W_TILED for tile-major W (N % 128 == 0,
// K % 64 == 0); LL_SMALL_M_SWIGLU to write silu(gate) * up of the
// interleaved gate/up product (C: M x N/2; N % 32 == 0).
extern "C" int ll_gemm_bf16_small_m_ex(const bf16* A, int lda, const bf16* W, int ldw, bf16* C, int ldc,
                                       const bf16* bias, int M, int N, int K, int splits, float* ws,
                                       size_t ws_floats, int* tickets, int* err, int flags, cudaStream_t stream) {
  LLSmallMEpi epi{};
  epi.mode = (flags & LL_SMALL_M_SWIGLU) ? LL_EPI_SWIGLU : LL_EPI_STORE;
  return small_m_launch(A, lda, W, ldw, C, ldc, bias, M, N, K, splits, ws, ws_floats, tickets, err,
                        flags & LL_SMALL_M_W_TILED, epi, stream);
}

extern "C" int ll_gemm_bf16_small_m_epi(const void* A, int lda, const void* W, int ldw, void* C, int ldc,
                                        const void* bias, int M, int N, int K, int splits, float* ws,
                                        size_t ws_floats, int* tickets, int* err, int w_tiled,
                                        const LLSmallMEpi* epi, void* stream) {
  if (epi == nullptr) return -3;
  return small_m_launch(static_cast<const bf16*>(A), lda, static_cast<const bf16*>(W), ldw, static_cast<bf16*>(C),
                        ldc, static_cast<const bf16*>(bias), M, N, K, splits, ws, ws_floats, tickets, err, w_tiled,
                        *epi, static_cast<cudaStream_t>(stream));
}

// Split count that keeps the grid within one wave of resident CTAs (two per
// SM): floor(2 * SMs / tiles), so no SM runs a third CTA while others idle.
extern "C" int ll_gemm_small_m_splits(int N, int K) {
  const int ntiles = (N + GEMM_BM - 1) / GEMM_BM;
  const int num_kb = (K + GEMM_BK - 1) / GEMM_BK;
  int splits = 2 * num_sms() / ntiles;
  if (splits > num_kb / 2) splits = num_kb / 2;
  // The fix-up keeps 16 partials per row in flight; each split past 16 adds
  // a dependent L2 round trip per row (a 1280-feature GEMV at 16 rows took
  // 53 us with 27 splits).
  if (splits > 16) splits = 16;
  if (splits < 1) splits = 1;
  int kb_per = (num_kb + splits - 1) / splits;
  return (num_kb + kb_per - 1) / kb_per;
}
