// Paged GQA attention, causal by logical position.
//
// attn_prefill_kernel: query rows at arbitrary positions (full prefill of a
//   Compile, the sparse boundary-repair rows of a Link, or any extend); each
//   row attends to key positions [0, pos] of its own request.  The reference
//   gets this from upstream Triton extend attention or FlashInfer
//   BlockSparse / paged-prefill wrappers with an explicit logical-causal mask
//   (reference patched_sglang_files/python/sglang/srt/flashinfer_sparse_repair.py:
//   1217-1318, 1395-1502; pic_runtime.py:4153-4488).  Here one launch covers
//   every repair row of every layer's attention, with no per-row forward loop.
//   Work unit: (request, kv head, 64 packed rows) where a packed row is a
//   (token, q-head-of-this-group) pair, so the K/V tile is loaded once for
//   all g = Hq/Hkv query heads.  4 warps x 16 rows, 64-key K/V blocks in a
//   double-buffered cp.async ring with XOR-swizzled rows, QK^T and PV on
//   mma.sync m16n8k16 (bf16 in, fp32 accumulate), online softmax in fp32.
//
// attn_decode_kernel: one query token per request; split-KV over 1-warp CTAs
//   (16 rows = the token's g heads), partials combined by attn_combine_kernel.
//   The default decode path is the TMA-fed 4-warp kernel in attention_tc.cu;
//   this one is the comparison point (LL_DECODE_V1=1).
#include <cuda_runtime.h>

#include <cstdlib>

#include "common.cuh"

namespace ll {

constexpr int AT_D = 128;
constexpr int AT_ROW_BYTES = AT_D * 2;  // 256

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * AT_ROW_BYTES + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

// ---------------------------------------------------------------- prefill
constexpr int PF_BM = 64;   // packed rows per CTA
constexpr int PF_BN = 64;   // keys per block
constexpr int PF_SMEM = (PF_BM + 4 * PF_BN) * AT_ROW_BYTES;  // Q + 2x(K,V) = 80 KB

__device__ __forceinline__ void pf_load_kv(uint32_t sK, uint32_t sV, const bf16* kpool, const bf16* vpool,
                                           const int* pt, int blk, int max_pos, int hk, int Hkv, int ps) {
  const int tid = threadIdx.x;
  const int c = tid & 15;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int kr = (tid >> 4) + 8 * i;
    const int key = blk * PF_BN + kr;
    const bool ok = key <= max_pos;
    size_t off = 0;
    if (ok) {
      const int page = pt[key / ps];
      off = (((size_t)page * Hkv + hk) * ps + (key % ps)) * AT_D + c * 8;
    }
    cp_async16(sK + swz(kr, c), kpool + off, ok);
    cp_async16(sV + swz(kr, c), vpool + off, ok);
  }
}

__global__ void __launch_bounds__(128, 2)
    attn_prefill_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kpool, const bf16* __restrict__ vpool,
                        const int* __restrict__ q_indptr, const int* __restrict__ q_pos,
                        const int* __restrict__ page_table, int pt_stride, const int4* __restrict__ tiles,
                        bf16* __restrict__ out, int Hq, int Hkv, int ps, float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + PF_BM * AT_ROW_BYTES;
  const uint32_t sV0 = sK0 + 2 * PF_BN * AT_ROW_BYTES;
  const int4 tile = tiles[blockIdx.x];
  const int b = tile.x, hk = tile.y, row0 = tile.z, max_pos = tile.w;
  const int g = Hq / Hkv;
  const int s = q_indptr[b];
  const int nrows = (q_indptr[b + 1] - s) * g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int* pt = page_table + (size_t)b * pt_stride;

  // Q tile (rows are (token, head) pairs of this kv-head group).
  {
    const int c = tid & 15;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = (tid >> 4) + 8 * i;
      const int pr = row0 + r;
      const bool ok = pr < nrows;
      size_t off = 0;
      if (ok) off = ((size_t)(s + pr / g) * Hq + hk * g + pr % g) * AT_D + c * 8;
      cp_async16(sQ + swz(r, c), q + off, ok);
    }
  }
  pf_load_kv(sK0, sV0, kpool, vpool, pt, 0, max_pos, hk, Hkv, ps);
  cp_async_commit();

  const int ra = warp * 16 + (lane >> 2), rb = ra + 8;
  const int pos_a = (row0 + ra < nrows) ? q_pos[s + (row0 + ra) / g] : -1;
  const int pos_b = (row0 + rb < nrows) ? q_pos[s + (row0 + rb) / g] : -1;
  int wmax = max(pos_a, pos_b);
  int wmin = min(pos_a < 0 ? 0x7fffffff : pos_a, pos_b < 0 ? 0x7fffffff : pos_b);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
    wmin = min(wmin, __shfl_xor_sync(0xffffffffu, wmin, o));
  }

  float O[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) O[i][0] = O[i][1] = O[i][2] = O[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  uint32_t qf[8][4];
  const int nblocks = max_pos / PF_BN + 1;

  for (int blk = 0; blk < nblocks; ++blk) {
    const int st = blk & 1;
    if (blk + 1 < nblocks) {
      pf_load_kv(sK0 + (st ^ 1) * PF_BN * AT_ROW_BYTES, sV0 + (st ^ 1) * PF_BN * AT_ROW_BYTES, kpool, vpool, pt,
                 blk + 1, max_pos, hk, Hkv, ps);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (blk == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        ldsm_x4(sQ + swz(r, 2 * kk + (lane >> 4)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const int kbase = blk * PF_BN;
    if (kbase <= wmax) {
      const uint32_t sK = sK0 + st * PF_BN * AT_ROW_BYTES;
      const uint32_t sV = sV0 + st * PF_BN * AT_ROW_BYTES;
      float S[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) S[i][0] = S[i][1] = S[i][2] = S[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          const int key = np * 16 + (lane & 7) + 8 * (lane >> 4);
          ldsm_x4(sK + swz(key, 2 * kk + ((lane >> 3) & 1)), b0, b1, b2, b3);
          mma16816(S[2 * np], qf[kk], b0, b1);
          mma16816(S[2 * np + 1], qf[kk], b2, b3);
        }
      }
      // scale + mask
      const bool need_mask = kbase + PF_BN - 1 > wmin;
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kbase + nt * 8 + 2 * (lane & 3) + e;
          float va = S[nt][e] * scale_log2, vb = S[nt][2 + e] * scale_log2;
          if (need_mask) {
            if (key > pos_a) va = -INFINITY;
            if (key > pos_b) vb = -INFINITY;
          }
          S[nt][e] = va;
          S[nt][2 + e] = vb;
          mx_a = fmaxf(mx_a, va);
          mx_b = fmaxf(mx_b, vb);
        }
      }
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      const float al_a = (mn_a == -INFINITY) ? 1.f : fast_exp2(m_a - mn_a);
      const float al_b = (mn_b == -INFINITY) ? 1.f : fast_exp2(m_b - mn_b);
      const float sub_a = (mn_a == -INFINITY) ? 0.f : mn_a;
      const float sub_b = (mn_b == -INFINITY) ? 0.f : mn_b;
      m_a = mn_a;
      m_b = mn_b;
      float rs_a = 0.f, rs_b = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        S[nt][0] = fast_exp2(S[nt][0] - sub_a);
        S[nt][1] = fast_exp2(S[nt][1] - sub_a);
        S[nt][2] = fast_exp2(S[nt][2] - sub_b);
        S[nt][3] = fast_exp2(S[nt][3] - sub_b);
        rs_a += S[nt][0] + S[nt][1];
        rs_b += S[nt][2] + S[nt][3];
      }
      l_a = l_a * al_a + rs_a;
      l_b = l_b * al_b + rs_b;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        O[i][0] *= al_a;
        O[i][1] *= al_a;
        O[i][2] *= al_b;
        O[i][3] *= al_b;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t a[4];
        a[0] = pack_bf16x2(S[2 * j][0], S[2 * j][1]);
        a[1] = pack_bf16x2(S[2 * j][2], S[2 * j][3]);
        a[2] = pack_bf16x2(S[2 * j + 1][0], S[2 * j + 1][1]);
        a[3] = pack_bf16x2(S[2 * j + 1][2], S[2 * j + 1][3]);
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int key = 16 * j + (lane & 7) + 8 * ((lane >> 3) & 1);
          ldsm_x4_t(sV + swz(key, 2 * dp + (lane >> 4)), b0, b1, b2, b3);
          mma16816(O[2 * dp], a, b0, b1);
          mma16816(O[2 * dp + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();
  }

  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f;
  const float inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  const int pra = row0 + ra, prb = row0 + rb;
  bf16* oa = pra < nrows ? out + ((size_t)(s + pra / g) * Hq + hk * g + pra % g) * AT_D : nullptr;
  bf16* ob = prb < nrows ? out + ((size_t)(s + prb / g) * Hq + hk * g + prb % g) * AT_D : nullptr;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = nt * 8 + 2 * (lane & 3);
    if (oa) *reinterpret_cast<uint32_t*>(oa + d) = pack_bf16x2(O[nt][0] * inv_a, O[nt][1] * inv_a);
    if (ob) *reinterpret_cast<uint32_t*>(ob + d) = pack_bf16x2(O[nt][2] * inv_b, O[nt][3] * inv_b);
  }
}

// ----------------------------------------------------------------- decode
constexpr int DC_BN = 32;  // keys per block
constexpr int DC_SMEM = (16 + 4 * DC_BN) * AT_ROW_BYTES;  // Q(16 rows) + 2x(K,V) = 36 KB

__device__ __forceinline__ void dc_load_kv(uint32_t sK, uint32_t sV, const bf16* kpool, const bf16* vpool,
                                           const int* pt, int k0, int kend, int hk, int Hkv, int ps) {
  const int lane = threadIdx.x;
  const int c = lane & 15;
#pragma unroll
  for (int i = 0; i < DC_BN / 2; ++i) {
    const int kr = (lane >> 4) + 2 * i;
    const int key = k0 + kr;
    const bool ok = key < kend;
    size_t off = 0;
    if (ok) {
      const int page = pt[key / ps];
      off = (((size_t)page * Hkv + hk) * ps + (key % ps)) * AT_D + c * 8;
    }
    cp_async16(sK + swz(kr, c), kpool + off, ok);
    cp_async16(sV + swz(kr, c), vpool + off, ok);
  }
}

// grid (B*Hkv, nsplit), block 32.  q [B, Hq, D].  Writes either the final
// output (nsplit == 1) or unnormalised partials: ws_o [B*Hq, nsplit, D],
// ws_ml [B*Hq, nsplit, 2] = (max in log2 domain, sum).
__global__ void __launch_bounds__(32)
    attn_decode_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kpool, const bf16* __restrict__ vpool,
                       const int* __restrict__ page_table, int pt_stride, const int* __restrict__ kv_lens,
                       bf16* __restrict__ out, float* __restrict__ ws_o, float* __restrict__ ws_ml, int Hq, int Hkv,
                       int ps, float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + 16 * AT_ROW_BYTES;
  const uint32_t sV0 = sK0 + 2 * DC_BN * AT_ROW_BYTES;
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x / Hkv, hk = blockIdx.x % Hkv;
  const int split = blockIdx.y, nsplit = gridDim.y;
  const int g = Hq / Hkv;
  const int lane = threadIdx.x;
  const int kv_len = kv_lens[b];
  int chunk = (kv_len + nsplit - 1) / nsplit;
  chunk = (chunk + DC_BN - 1) / DC_BN * DC_BN;
  const int kbeg = split * chunk;
  const int kend = min(kv_len, kbeg + chunk);
  const int* pt = page_table + (size_t)b * pt_stride;

  {
    const int c = lane & 15;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = (lane >> 4) + 2 * i;
      const bool ok = r < g;
      const size_t off = ok ? (((size_t)b * Hq + hk * g + r) * AT_D + c * 8) : 0;
      cp_async16(sQ + swz(r, c), q + off, ok);
    }
  }
  const int nblocks = kend > kbeg ? (kend - kbeg + DC_BN - 1) / DC_BN : 0;
  if (nblocks > 0) dc_load_kv(sK0, sV0, kpool, vpool, pt, kbeg, kend, hk, Hkv, ps);
  cp_async_commit();

  float O[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) O[i][0] = O[i][1] = O[i][2] = O[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  uint32_t qf[8][4];
  if (nblocks == 0) {
    cp_async_wait<0>();
    __syncwarp();
  }
  for (int blk = 0; blk < nblocks; ++blk) {
    const int st = blk & 1;
    const int k0 = kbeg + blk * DC_BN;
    if (blk + 1 < nblocks) {
      dc_load_kv(sK0 + (st ^ 1) * DC_BN * AT_ROW_BYTES, sV0 + (st ^ 1) * DC_BN * AT_ROW_BYTES, kpool, vpool, pt,
                 k0 + DC_BN, kend, hk, Hkv, ps);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();
    if (blk == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int r = (lane & 7) + 8 * ((lane >> 3) & 1);
        ldsm_x4(sQ + swz(r, 2 * kk + (lane >> 4)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const uint32_t sK = sK0 + st * DC_BN * AT_ROW_BYTES;
    const uint32_t sV = sV0 + st * DC_BN * AT_ROW_BYTES;
    float S[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) S[i][0] = S[i][1] = S[i][2] = S[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b0, b1, b2, b3;
        const int key = np * 16 + (lane & 7) + 8 * (lane >> 4);
        ldsm_x4(sK + swz(key, 2 * kk + ((lane >> 3) & 1)), b0, b1, b2, b3);
        mma16816(S[2 * np], qf[kk], b0, b1);
        mma16816(S[2 * np + 1], qf[kk], b2, b3);
      }
    }
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = k0 + nt * 8 + 2 * (lane & 3) + e;
        float va = S[nt][e] * scale_log2, vb = S[nt][2 + e] * scale_log2;
        if (key >= kend) va = vb = -INFINITY;
        S[nt][e] = va;
        S[nt][2 + e] = vb;
        mx_a = fmaxf(mx_a, va);
        mx_b = fmaxf(mx_b, vb);
      }
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float al_a = (mn_a == -INFINITY) ? 1.f : fast_exp2(m_a - mn_a);
    const float al_b = (mn_b == -INFINITY) ? 1.f : fast_exp2(m_b - mn_b);
    const float sub_a = (mn_a == -INFINITY) ? 0.f : mn_a;
    const float sub_b = (mn_b == -INFINITY) ? 0.f : mn_b;
    m_a = mn_a;
    m_b = mn_b;
    float rs_a = 0.f, rs_b = 0.f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      S[nt][0] = fast_exp2(S[nt][0] - sub_a);
      S[nt][1] = fast_exp2(S[nt][1] - sub_a);
      S[nt][2] = fast_exp2(S[nt][2] - sub_b);
      S[nt][3] = fast_exp2(S[nt][3] - sub_b);
      rs_a += S[nt][0] + S[nt][1];
      rs_b += S[nt][2] + S[nt][3];
    }
    l_a = l_a * al_a + rs_a;
    l_b = l_b * al_b + rs_b;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      O[i][0] *= al_a;
      O[i][1] *= al_a;
      O[i][2] *= al_b;
      O[i][3] *= al_b;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t a[4];
      a[0] = pack_bf16x2(S[2 * j][0], S[2 * j][1]);
      a[1] = pack_bf16x2(S[2 * j][2], S[2 * j][3]);
      a[2] = pack_bf16x2(S[2 * j + 1][0], S[2 * j + 1][1]);
      a[3] = pack_bf16x2(S[2 * j + 1][2], S[2 * j + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int key = 16 * j + (lane & 7) + 8 * ((lane >> 3) & 1);
        ldsm_x4_t(sV + swz(key, 2 * dp + (lane >> 4)), b0, b1, b2, b3);
        mma16816(O[2 * dp], a, b0, b1);
        mma16816(O[2 * dp + 1], a, b2, b3);
      }
    }
    __syncwarp();
  }
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const int ra = lane >> 2, rb = ra + 8;
  if (nsplit == 1) {
    const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f, inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int d = nt * 8 + 2 * (lane & 3);
      if (ra < g)
        *reinterpret_cast<uint32_t*>(out + ((size_t)b * Hq + hk * g + ra) * AT_D + d) =
            pack_bf16x2(O[nt][0] * inv_a, O[nt][1] * inv_a);
      if (rb < g)
        *reinterpret_cast<uint32_t*>(out + ((size_t)b * Hq + hk * g + rb) * AT_D + d) =
            pack_bf16x2(O[nt][2] * inv_b, O[nt][3] * inv_b);
    }
  } else {
    const size_t ia = ((size_t)b * Hq + hk * g + ra) * nsplit + split;
    const size_t ib = ((size_t)b * Hq + hk * g + rb) * nsplit + split;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int d = nt * 8 + 2 * (lane & 3);
      if (ra < g) *reinterpret_cast<float2*>(ws_o + ia * AT_D + d) = make_float2(O[nt][0], O[nt][1]);
      if (rb < g) *reinterpret_cast<float2*>(ws_o + ib * AT_D + d) = make_float2(O[nt][2], O[nt][3]);
    }
    if ((lane & 3) == 0) {
      if (ra < g) *reinterpret_cast<float2*>(ws_ml + ia * 2) = make_float2(m_a, l_a);
      if (rb < g) *reinterpret_cast<float2*>(ws_ml + ib * 2) = make_float2(m_b, l_b);
    }
  }
}

// grid (B*Hq), block 128 (one thread per head_dim element).  The split
// maxima and weights are computed cooperatively in shared memory, then each
// thread reduces its head_dim column over the splits (coalesced reads).
// 256 threads: the split maxima and weights are computed cooperatively in
// shared memory; then each of the 8 warps sums a strided subset of the
// splits (lane l owns head_dim elements [4l, 4l+4) via float4 loads, 8 loads
// in flight per lane) and the warps' partial vectors are added in shared
// memory.  A thread-per-element loop over the splits is latency-bound.
constexpr int CB_MAX_SPLITS = 1024;
constexpr int CB_THREADS = 256;
__global__ void __launch_bounds__(CB_THREADS) attn_combine_kernel(bf16* __restrict__ out,
                                                                  const float* __restrict__ ws_o,
                                                                  const float* __restrict__ ws_ml, int nsplit) {
  __shared__ float w[CB_MAX_SPLITS];
  __shared__ float red[CB_THREADS / 32];
  __shared__ float4 part[CB_THREADS / 32][32];
  pdl_trigger();
  pdl_wait();
  const size_t row = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  constexpr int NW = CB_THREADS / 32;
  const float2* ml = reinterpret_cast<const float2*>(ws_ml) + row * nsplit;
  float M = -INFINITY;
  for (int sp = t; sp < nsplit; sp += CB_THREADS) M = fmaxf(M, ml[sp].x);
  M = warp_max(M);
  if (lane == 0) red[warp] = M;
  __syncthreads();
  M = red[0];
#pragma unroll
  for (int i = 1; i < NW; ++i) M = fmaxf(M, red[i]);
  __syncthreads();
  float den = 0.f;
  for (int sp = t; sp < nsplit; sp += CB_THREADS) {
    const float2 v = ml[sp];
    const float wt = (v.x == -INFINITY || M == -INFINITY) ? 0.f : exp2f(v.x - M);
    w[sp] = wt;
    den += wt * v.y;
  }
  den = warp_sum(den);
  if (lane == 0) red[warp] = den;
  __syncthreads();
  den = 0.f;
#pragma unroll
  for (int i = 0; i < NW; ++i) den += red[i];
  const float4* o = reinterpret_cast<const float4*>(ws_o + row * (size_t)nsplit * AT_D) + lane;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
  for (int sp = warp; sp < nsplit; sp += NW) {
    const float4 v = __ldcg(o + (size_t)sp * (AT_D / 4));
    const float wt = w[sp];
    acc.x += wt * v.x;
    acc.y += wt * v.y;
    acc.z += wt * v.z;
    acc.w += wt * v.w;
  }
  part[warp][lane] = acc;
  __syncthreads();
  if (warp == 0) {
    float4 s = part[0][lane];
#pragma unroll
    for (int i = 1; i < NW; ++i) {
      const float4 p = part[i][lane];
      s.x += p.x;
      s.y += p.y;
      s.z += p.z;
      s.w += p.w;
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
    uint2 pk = make_uint2(pack_bf16x2(s.x * inv, s.y * inv), pack_bf16x2(s.z * inv, s.w * inv));
    *reinterpret_cast<uint2*>(out + row * AT_D + 4 * lane) = pk;
  }
}

}  // namespace ll

using namespace ll;

extern "C" int ll_attn_prefill(const bf16* q, const bf16* kpool, const bf16* vpool, const int* q_indptr,
                               const int* q_pos, const int* page_table, int pt_stride, const int* tiles, int ntiles,
                               bf16* out, int Hq, int Hkv, int head_dim, int page_size, float scale,
                               cudaStream_t stream) {
  if (ntiles <= 0) return 0;
  if (head_dim != AT_D || Hq % Hkv) return -3;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
    init = true;
  }
  attn_prefill_kernel<<<ntiles, 128, PF_SMEM, stream>>>(q, kpool, vpool, q_indptr, q_pos, page_table, pt_stride,
                                                        reinterpret_cast<const int4*>(tiles), out, Hq, Hkv,
                                                        page_size, scale * 1.4426950408889634f);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

extern "C" int ll_attn_decode_tma(const bf16* q, const bf16* k_pool, const bf16* v_pool, int pages,
                                  const int* page_table, int pt_stride, const int* kv_lens, bf16* out, float* ws_o,
                                  float* ws_ml, int B, int Hq, int Hkv, int page_size, int nsplit, float scale_log2,
                                  int new_tokens, int* err, cudaStream_t stream);

// Decode attention runs on the TMA-fed kernel (attention_tc.cu);
// LL_DECODE_V1=1 selects the one-warp cp.async kernel above, kept as the
// comparison point (and used for page sizes that do not divide 64).
static bool decode_tma_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("LL_DECODE_V1");
    v = (e != nullptr && e[0] == '1') ? 0 : 1;
  }
  return v == 1;
}

// Few splits per row (the prefill key-range splits): one warp per row, lane
// l owns columns [4l, 4l + 4); every split's (max, sum) and 16-byte slice of
// O are loaded before any is used, so a warp has all its loads in flight at
// once; 8 rows per CTA.
constexpr int CW_ROWS = 8;
template <int MAXS>
__global__ void __launch_bounds__(32 * CW_ROWS) attn_combine_warp_kernel(bf16* __restrict__ out,
                                                                         const float* __restrict__ ws_o,
                                                                         const float* __restrict__ ws_ml, int rows,
                                                                         int nsplit) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const size_t row = (size_t)blockIdx.x * CW_ROWS + (threadIdx.x >> 5);
  if (row >= (size_t)rows) return;
  const float2* ml = reinterpret_cast<const float2*>(ws_ml) + row * nsplit;
  const float4* o = reinterpret_cast<const float4*>(ws_o + row * (size_t)nsplit * AT_D) + lane;
  float2 m[MAXS];
  float4 v[MAXS];
#pragma unroll
  for (int sp = 0; sp < MAXS; ++sp) {
    if (sp < nsplit) {
      m[sp] = __ldcg(ml + sp);
      v[sp] = __ldcg(o + (size_t)sp * (AT_D / 4));
    }
  }
  float M = -INFINITY;
#pragma unroll
  for (int sp = 0; sp < MAXS; ++sp)
    if (sp < nsplit) M = fmaxf(M, m[sp].x);
  float den = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int sp = 0; sp < MAXS; ++sp) {
    if (sp < nsplit) {
      const float wt = (m[sp].x == -INFINITY || M == -INFINITY) ? 0.f : exp2f(m[sp].x - M);
      den += wt * m[sp].y;
      acc.x += wt * v[sp].x;
      acc.y += wt * v[sp].y;
      acc.z += wt * v[sp].z;
      acc.w += wt * v[sp].w;
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  *reinterpret_cast<uint2*>(out + row * AT_D + 4 * lane) =
      make_uint2(pack_bf16x2(acc.x * inv, acc.y * inv), pack_bf16x2(acc.z * inv, acc.w * inv));
}

// Combine of split-KV partials: rows x nsplit partials [rows][nsplit][128]
// (fp32) with (max log2, sum) each -> out [rows][128] (bf16).
extern "C" int ll_attn_combine(bf16* out, const float* ws_o, const float* ws_ml, int rows, int nsplit,
                               cudaStream_t stream) {
  if (rows <= 0 || nsplit < 1 || nsplit > CB_MAX_SPLITS) return -3;
  const dim3 grid((rows + CW_ROWS - 1) / CW_ROWS), block(32 * CW_ROWS);
  if (nsplit <= 8)
    launch_pdl(attn_combine_warp_kernel<8>, grid, block, 0, stream, out, ws_o, ws_ml, rows, nsplit);
  else if (nsplit <= 16)
    launch_pdl(attn_combine_warp_kernel<16>, grid, block, 0, stream, out, ws_o, ws_ml, rows, nsplit);
  else
    launch_pdl(attn_combine_kernel, dim3(rows), dim3(CB_THREADS), 0, stream, out, ws_o, ws_ml, nsplit);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

extern "C" int ll_attn_decode(const bf16* q, const bf16* kpool, const bf16* vpool, int num_pages,
                              const int* page_table, int pt_stride, const int* kv_lens, bf16* out, float* ws_o,
                              float* ws_ml, int B, int Hq, int Hkv, int head_dim, int page_size, int nsplit,
                              float scale, int* err, cudaStream_t stream) {
  if (B <= 0) return 0;
  if (head_dim != AT_D || Hq % Hkv || Hq / Hkv > 16) return -3;
  if (nsplit < 1) nsplit = 1;
  if (nsplit > CB_MAX_SPLITS) return -3;
  if (nsplit > 1 && (ws_o == nullptr || ws_ml == nullptr)) return -6;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DC_SMEM);
    init = true;
  }
  dim3 grid(B * Hkv, nsplit);
  const float sl2 = scale * 1.4426950408889634f;
  if (decode_tma_enabled() && page_size >= 4 && 64 % page_size == 0) {
    // One query per request: only its own key (the last) may have been
    // written by the previous kernel; the TMA kernel streams the older keys
    // before waiting on it.  Every other K/V writer is separated from this
    // launch by a stream-ordered copy (each decode step starts with its
    // input copies), so it has completed.
    const int rc = ll_attn_decode_tma(q, kpool, vpool, num_pages, page_table, pt_stride, kv_lens, out, ws_o, ws_ml,
                                      B, Hq, Hkv, page_size, nsplit, sl2, 1, err, stream);
    if (rc != 0) return rc;
  } else {
    launch_pdl(attn_decode_kernel, grid, dim3(32), DC_SMEM, stream, q, kpool, vpool, page_table, pt_stride, kv_lens,
               out, ws_o, ws_ml, Hq, Hkv, page_size, sl2);
  }
  if (nsplit > 1)
    launch_pdl(attn_combine_kernel, dim3(B * Hq), dim3(CB_THREADS), 0, stream, out, ws_o, ws_ml, nsplit);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}
