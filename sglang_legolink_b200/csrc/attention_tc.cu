// Prefill / sparse-repair attention on the 5th-generation tensor cores.
//
// Same contract as attn_prefill_kernel (attention.cu): query rows at arbitrary
// positions, keys = the request's paged KV, causal by logical position, GQA
// rows packed as (token, q-head-of-the-group) pairs.  One CTA owns TC_NT = 2
// tiles of 128 packed rows of one (request, kv head) and walks 64-key blocks;
// both tiles share every K/V block:
//
//   warp 0      TMA producer: K and V pages of each block (one box of
//               page_size keys x 64 dims per page and half), 2-stage ring.
//   warp 1      MMA issuer (one thread), per block j: S(t, j) = Q_t K_j^T for
//               both tiles into their TMEM S double buffers (M=128, N=64,
//               K=16 x 8), then O_t += P(t, j-1) V_{j-1} (M=128, N=128,
//               K=16 x 4; V is the MN-major B operand).
//   warps 2..9  two softmax warpgroups, one per tile, one query row per
//               thread (TMEM lane = row): read S with tcgen05.ld, mask by
//               position, online max/sum in fp32 (log2 domain), write P (bf16)
//               to shared memory in the 128-byte swizzled K-major layout the
//               MMA reads.  O stays in TMEM; it is rescaled (tcgen05.ld/st)
//               only when a row's running max grows by more than 2^8, so
//               P <= 256 and most blocks skip the rescale.  While one
//               warpgroup runs its softmax the tensor core works on the other
//               tile.
//
// Barriers: kv_full/kv_empty per stage; s_full/s_empty and p_full/p_empty
// per tile and double buffer; q_full, o_full.  Every wait is bounded
// (common.cuh).
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace ll {

constexpr int TC_BM = 128;        // packed query rows per tile
constexpr int TC_NT = 2;          // tiles per CTA
constexpr int TC_BN = 64;         // keys per block
constexpr int TC_D = 128;
constexpr int TC_STAGES = 2;
constexpr int TC_Q_BYTES = TC_BM * TC_D * 2;         // 32 KB per tile: [2 halves][128 rows][128 B]
constexpr int TC_Q_HALF = TC_BM * 128;               // 16 KB
constexpr int TC_KV_BYTES = TC_BN * TC_D * 2;        // 16 KB: [2 halves][64 rows][128 B]
constexpr int TC_KV_HALF = TC_BN * 128;              // 8 KB
constexpr int TC_P_BYTES = TC_BM * TC_BN * 2;        // 16 KB: [128 rows][128 B]
constexpr int TC_SMEM = TC_NT * TC_Q_BYTES + 2 * TC_STAGES * TC_KV_BYTES + TC_NT * 2 * TC_P_BYTES + 1024 + 512;
constexpr uint32_t TC_TMEM_COLS = 512;               // per tile t: S0 [256t, +64) S1 [+64, +128) O [+128, +256)
constexpr int TC_THREADS = 64 + 128 * TC_NT;
constexpr float TC_RESCALE_THRESHOLD = 8.0f;         // log2 units

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Descriptor of an MN-major operand in the 128-byte swizzle: atoms of 8 K-rows
// x 128 B (64 bf16 along N); `lbo` = bytes between 64-wide N groups, `sbo` =
// bytes between 8-row K groups.
__device__ __forceinline__ uint64_t umma_desc_sw128_mnmajor(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void cp_async16_tc(uint32_t saddr, const void* g, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(n) : "memory");
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           const bf16* __restrict__ q, const int* __restrict__ q_indptr,
                           const int* __restrict__ q_pos, const int* __restrict__ page_table, int pt_stride,
                           const int4* __restrict__ tiles, bf16* __restrict__ out, int Hq, int Hkv, int ps,
                           int layer, float scale_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [TC_NT][Q]
  uint8_t* sK = sQ + TC_NT * TC_Q_BYTES;                // [STAGES][KV]
  uint8_t* sV = sK + TC_STAGES * TC_KV_BYTES;
  uint8_t* sP = sV + TC_STAGES * TC_KV_BYTES;           // [TC_NT][2][P]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + TC_NT * 2 * TC_P_BYTES);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = kv_full + TC_STAGES;
  uint64_t* s_full = kv_empty + TC_STAGES;    // [TC_NT][2]
  uint64_t* s_empty = s_full + 2 * TC_NT;
  uint64_t* p_full = s_empty + 2 * TC_NT;
  uint64_t* p_empty = p_full + 2 * TC_NT;
  uint64_t* q_full = p_empty + 2 * TC_NT;
  uint64_t* o_full = q_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int4 tile = tiles[blockIdx.x];
  const int b = tile.x, hk = tile.y, row0 = tile.z, max_pos = tile.w;
  const int g = Hq / Hkv;
  const int s0 = q_indptr[b];
  const int nrows = (q_indptr[b + 1] - s0) * g;
  const int nb = max_pos / TC_BN + 1;
  const int* pt = page_table + (size_t)b * pt_stride;

  if (threadIdx.x == 0) {
    for (int i = 0; i < TC_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2 * TC_NT; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(q_full, 4 * TC_NT);
    mbar_init(o_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TC_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      const int pages_per_block = TC_BN / ps;
      bool ok = true;
      for (int j = 0; j < nb && ok; ++j) {
        const int st = j % TC_STAGES, n = j / TC_STAGES;
        if (!mbar_wait(&kv_empty[st], (n & 1) ^ 1, err, kErrSmemEmptyTimeout)) { ok = false; break; }
        mbar_arrive_expect_tx(&kv_full[st], 2 * TC_KV_BYTES);
        for (int p = 0; p < pages_per_block; ++p) {
          const int key0 = j * TC_BN + p * ps;
          const int ycoord = key0 <= max_pos ? pt[key0 / ps] * Hkv + hk : -1;  // -1: out of range, zero fill
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint8_t* dk = sK + st * TC_KV_BYTES + h * TC_KV_HALF + p * ps * 128;
            uint8_t* dv = sV + st * TC_KV_BYTES + h * TC_KV_HALF + p * ps * 128;
            tma_load_4d(dk, &tmK, &kv_full[st], 64 * h, 0, ycoord, layer);
            tma_load_4d(dv, &tmV, &kv_full[st], 64 * h, 0, ycoord, layer);
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
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16_f32(TC_BM, TC_BN);
      constexpr uint32_t idesc_pv = umma_idesc_bf16_f32(TC_BM, TC_D) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(q_full, 0, err, kErrTmaFullTimeout);
      tc_fence_after();
      // O_t += P(t, i) V_i for both tiles, then release K_i/V_i.
      auto issue_pv = [&](int i) -> bool {
        const int pb = i & 1;
        const int st = i % TC_STAGES;
        const uint32_t vbase = smem_u32(sV + st * TC_KV_BYTES);
#pragma unroll
        for (int t = 0; t < TC_NT; ++t) {
          if (!mbar_wait(&p_full[2 * t + pb], (i >> 1) & 1, err, kErrTmemFullTimeout)) return false;
          tc_fence_after();
          const uint32_t pbase = smem_u32(sP + (2 * t + pb) * TC_P_BYTES);
#pragma unroll
          for (int k = 0; k < TC_BN / 16; ++k) {
            const uint64_t ad = umma_desc_sw128_kmajor(pbase + 32 * k);
            const uint64_t bd = umma_desc_sw128_mnmajor(vbase + k * 16 * 128, TC_KV_HALF, 1024);
            umma_bf16(tmem + 256 * t + 128, ad, bd, idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&p_empty[2 * t + pb]);
        }
        umma_commit(&kv_empty[st]);
        return true;
      };
      for (int j = 0; j < nb && ok; ++j) {
        const int st = j % TC_STAGES, sb = j & 1;
        if (!mbar_wait(&kv_full[st], (j / TC_STAGES) & 1, err, kErrTmaFullTimeout)) { ok = false; break; }
        const uint32_t kbase = smem_u32(sK + st * TC_KV_BYTES);
#pragma unroll
        for (int t = 0; t < TC_NT; ++t) {
          if (!mbar_wait(&s_empty[2 * t + sb], ((j >> 1) & 1) ^ 1, err, kErrTmemEmptyTimeout)) { ok = false; break; }
          tc_fence_after();
          const uint32_t qbase = smem_u32(sQ + t * TC_Q_BYTES);
#pragma unroll
          for (int k = 0; k < TC_D / 16; ++k) {
            const uint64_t ad = umma_desc_sw128_kmajor(qbase + (k >> 2) * TC_Q_HALF + (k & 3) * 32);
            const uint64_t bd = umma_desc_sw128_kmajor(kbase + (k >> 2) * TC_KV_HALF + (k & 3) * 32);
            umma_bf16(tmem + 256 * t + sb * TC_BN, ad, bd, idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[2 * t + sb]);
        }
        if (!ok) break;
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(nb - 1);
      umma_commit(o_full);  // also drains every MMA issued above
      mbar_wait(o_full, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- softmax
    const int t = (warp - 2) >> 2;        // tile of this warpgroup
    const int qd = warp & 3;              // TMEM lane quarter of this warp
    const int r = qd * 32 + lane;         // query row of this thread within the tile
    const int pr = row0 + t * TC_BM + r;
    const bool valid = pr < nrows;
    const int tok = s0 + pr / g;
    const int head = hk * g + pr % g;
    const int pos = valid ? q_pos[tok] : -1;
    uint8_t* sQt = sQ + t * TC_Q_BYTES;
    // Q row -> shared memory (two 128-B halves, 128-B swizzle), then signal.
    {
      const bf16* src = q + ((size_t)tok * Hq + head) * TC_D;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const int h = c >> 3, cc = c & 7;
        const uint32_t dst = smem_u32(sQt) + h * TC_Q_HALF + r * 128 + ((cc ^ (r & 7)) << 4);
        cp_async16_tc(dst, valid ? (const void*)(src + c * 8) : (const void*)q, valid);
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    }
    const uint32_t lane_base = tmem + (uint32_t(qd * 32) << 16) + 256 * t;
    uint64_t* sf = s_full + 2 * t;
    uint64_t* se = s_empty + 2 * t;
    uint64_t* pf = p_full + 2 * t;
    uint64_t* pe = p_empty + 2 * t;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&sf[sb], (j >> 1) & 1, err, kErrTmemFullTimeout)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[64];
      tmem_ld_32x32b_x32(lane_base + sb * TC_BN, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
      tmem_ld_32x32b_x32(lane_base + sb * TC_BN + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&se[sb]);
      const int kbase = j * TC_BN;
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        float v = __uint_as_float(s[i]) * scale_log2;
        if (kbase + i > pos) v = -INFINITY;
        s[i] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
      const float m_new = fmaxf(m_run, mx);
      const bool grow = m_new > m_run + TC_RESCALE_THRESHOLD;  // false while m_new == -inf
      const float m_use = grow ? m_new : m_run;
      const float o_scale = (grow && m_run != -INFINITY) ? ex2(m_run - m_new) : 1.f;
      // P buffer sb of this tile is free once PV of block j-2 finished.
      if (!mbar_wait(&pe[sb], ((j >> 1) & 1) ^ 1, err, kErrTmemEmptyTimeout)) { ok = false; break; }
      if (j > 0 && __any_sync(0xffffffffu, o_scale != 1.f)) {
        // O must be stable: PV of block j-1 complete.
        const int pb = (j - 1) & 1;
        if (!mbar_wait(&pe[pb], ((j - 1) >> 1) & 1, err, kErrTmemEmptyTimeout)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < TC_D; c += 32) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(lane_base + 128 + c, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * o_scale);
          tmem_st_32x32b_x32(lane_base + 128 + c, o);
        }
        tmem_st_wait();
      }
      l_run *= o_scale;
      m_run = m_use;
      // P = exp2(s - m) as bf16 into the swizzled K-major tile.
      float sum = 0.f;
      const uint32_t prow = smem_u32(sP + (2 * t + sb) * TC_P_BYTES) + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = __uint_as_float(s[8 * c + 2 * e]), bb = __uint_as_float(s[8 * c + 2 * e + 1]);
          const float pa = (m_use == -INFINITY) ? 0.f : ex2(a - m_use);
          const float pb = (m_use == -INFINITY) ? 0.f : ex2(bb - m_use);
          sum += pa + pb;
          pk[e] = pack_bf16x2(pa, pb);
        }
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(prow + ((c ^ (r & 7)) << 4)), "r"(pk[0]),
                     "r"(pk[1]), "r"(pk[2]), "r"(pk[3])
                     : "memory");
      }
      l_run += sum;
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pf[sb]);
    }
    // ----------------------------------------------------------- epilogue
    if (ok && mbar_wait(o_full, 0, err, kErrTmemFullTimeout)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      bf16* dst = out + ((size_t)tok * Hq + head) * TC_D;
#pragma unroll 1
      for (int c = 0; c < TC_D; c += 32) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(lane_base + 128 + c, o);
        tmem_ld_wait();
        if (valid) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
          uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TC_TMEM_COLS);
}

typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 encode_fn() {
  static EncodeTiledFn2 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn2>(p);
  }
  return fn;
}

// 4-D map over a pool [L, pages, Hkv, ps, D=128] viewed as {D, ps, pages*Hkv, L};
// box = {64, ps, 1, 1} with the 128-byte swizzle.
static int make_pool_map(CUtensorMap* tm, const void* base, int L, int pages, int Hkv, int ps) {
  EncodeTiledFn2 enc = encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[4] = {(cuuint64_t)TC_D, (cuuint64_t)ps, (cuuint64_t)pages * Hkv, (cuuint64_t)L};
  cuuint64_t strides[3] = {(cuuint64_t)TC_D * 2, (cuuint64_t)ps * TC_D * 2, (cuuint64_t)pages * Hkv * ps * TC_D * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)ps, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

}  // namespace ll

using namespace ll;

// k_pool / v_pool: whole pools [L, pages, Hkv, ps, 128]; `layer` selects the layer.
extern "C" int ll_attn_prefill_tc(const bf16* q, const bf16* k_pool, const bf16* v_pool, int L, int pages, int layer,
                                  const int* q_indptr, const int* q_pos, const int* page_table, int pt_stride,
                                  const int* tiles, int ntiles, bf16* out, int Hq, int Hkv, int head_dim,
                                  int page_size, float scale, int* err, cudaStream_t stream) {
  if (ntiles <= 0) return 0;
  if (head_dim != TC_D || Hq % Hkv) return -3;
  if (page_size <= 0 || page_size > TC_BN || TC_BN % page_size) return -3;
  if (Hq / Hkv > TC_BM) return -3;
  CUtensorMap tk, tv;
  if (make_pool_map(&tk, k_pool, L, pages, Hkv, page_size)) return -2;
  if (make_pool_map(&tv, v_pool, L, pages, Hkv, page_size)) return -2;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    init = true;
  }
  attn_prefill_tc_kernel<<<ntiles, TC_THREADS, TC_SMEM, stream>>>(tk, tv, q, q_indptr, q_pos, page_table, pt_stride,
                                                           reinterpret_cast<const int4*>(tiles), out, Hq, Hkv,
                                                           page_size, layer, scale * 1.4426950408889634f, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}
