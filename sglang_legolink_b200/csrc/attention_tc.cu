// Prefill / sparse-repair attention on the 5th-generation tensor cores.
//
// Same contract as attn_prefill_kernel (attention.cu): query rows at arbitrary
// positions, keys = the request's paged KV, causal by logical position, GQA
// rows packed as (token, q-head-of-the-group) pairs.  One CTA owns TC_NT = 2
// tiles of 128 packed rows of one (request, kv head) and walks 128-key blocks;
// both tiles share every K/V block.
//
//   warp 0      TMA producer: K and V pages of each block (one box of
//               page_size keys x 64 dims per page and half) into separate
//               K and V rings, so K of block j+1 streams while V of block j
//               is still in use.
//   warp 1      MMA issuer (one thread).  Per block j and tile t:
//                 O_t += P_t(j-1) V_{j-1}   A = P from TMEM, B = V (MN-major)
//                 S_t  = Q_t K_j^T          A = Q, B = K from shared memory
//               P_t aliases the first 64 columns of S_t (bf16 pairs), so
//               each tile needs 256 TMEM columns (S/P 128 + O 128).  The
//               tensor pipe executes one thread's MMAs in issue order, so
//               S_t(j) overwriting P_t(j-1) after the PV MMA that reads it
//               is safe.  While softmax t works on S_t(j), the tensor core
//               runs the other tile's PV and S MMAs (ping-pong).
//   warps 2,3   idle (their registers go to the softmax warpgroups).
//   softmax     CS warpgroups per tile (CS = 1: warps 4..11; CS = 2: warps
//               4..19), one query row per thread (TMEM lane = row); with
//               CS = 2 each of the two warpgroups of a tile takes 64 of the
//               128 key columns of every row, so each warp's dependent chain
//               (TMEM load, max, exp2, pack, TMEM store) is half as long and
//               twice as many warps hide each other's latency.  The two
//               halves of a row exchange their maxima through shared memory
//               behind a bounded mbarrier wait.  Per row: tcgen05.ld S,
//               causal mask, online max/sum in fp32 (log2 domain), P =
//               exp2(S*scale - m) as bf16 written back to TMEM with
//               tcgen05.st.  O stays in TMEM; it is rescaled in place only
//               when a row's running max grows by more than 2^8, so P <= 256
//               and most blocks skip the rescale.  At the end: O / l ->
//               global memory (each half writes its 64 of the 128 columns).
//
// Barriers: k_full/k_empty, v_full/v_empty per stage; s_full, p_full per
// tile; q_full, o_full; with CS = 2, one max-exchange barrier per (tile,
// TMEM lane quarter).  Every wait is bounded (common.cuh).
#include <cstdlib>
#include <type_traits>

#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace ll {

constexpr int TC_BM = 128;        // packed query rows per tile
constexpr int TC_NT = 2;          // tiles per CTA
constexpr int TC_BN = 128;        // keys per block
constexpr int TC_D = 128;
constexpr int TC_KS = 2;          // K ring stages
constexpr int TC_VS = 2;          // V ring stages
constexpr int TC_Q_BYTES = TC_BM * TC_D * 2;         // 32 KB per tile: [2 halves][128 rows][128 B]
constexpr int TC_Q_HALF = TC_BM * 128;               // 16 KB
constexpr int TC_KV_BYTES = TC_BN * TC_D * 2;        // 32 KB: [2 halves][128 keys][128 B]
constexpr int TC_KV_HALF = TC_BN * 128;              // 16 KB
constexpr int TC_SMEM_BASE = TC_NT * TC_Q_BYTES + (TC_KS + TC_VS) * TC_KV_BYTES + 1024 + 256;
constexpr uint32_t TC_TMEM_COLS = 512;               // S_t/P_t at 128t, O_t at 256 + 128t
// Per softmax column split CS: threads, shared memory and the register split
// (setmaxnreg).  Warpgroup 0 (producer, MMA, 2 idle warps) gives registers
// back and the softmax warpgroups take them; the sum stays within the launch
// allocation (threads x launch registers) and, per SM sub-partition (one
// warp of every warpgroup), within 16384.
//   CS = 1: 384 threads at 168: 4 x 32 x 80 + 8 x 32 x 208 = 63488 <= 64512;
//           per sub-partition 32 x (80 + 2 x 208) = 15872.
//   CS = 2: 640 threads at 96:  4 x 32 x 88 + 16 x 32 x 96 = 60416 <= 61440;
//           per sub-partition 32 x (88 + 4 x 96) = 15104.  (With 64 for
//           warpgroup 0 its MMA loop spills.)  Shared memory adds the max /
//           sum exchange buffer [tile][parity][half][128].
template <int CS>
struct TcCfg {
  static constexpr int THREADS = 128 + 128 * TC_NT * CS;
  static constexpr int REGS_LAUNCH = CS == 1 ? 168 : 96;
  static constexpr int REGS_CTRL = CS == 1 ? 80 : 88;
  static constexpr int REGS_SOFTMAX = CS == 1 ? 208 : 96;
  static constexpr int NC = TC_BN / CS;              // key columns per softmax thread
  static constexpr int XBUF_BYTES = CS == 1 ? 0 : TC_NT * 2 * CS * TC_BM * 4;
  static constexpr int SMEM = TC_SMEM_BASE + XBUF_BYTES;
  static_assert(4 * REGS_CTRL + 4 * TC_NT * CS * REGS_SOFTMAX <= (THREADS / 32) * REGS_LAUNCH,
                "register split exceeds the launch allocation");
  static_assert(32 * (REGS_CTRL + TC_NT * CS * REGS_SOFTMAX) <= 16384, "register split exceeds a sub-partition");
  static_assert(THREADS * REGS_LAUNCH <= 65536, "launch registers exceed the SM");
};
static_assert(TC_Q_HALF == TC_KV_HALF, "Q and K halves share descriptor offsets");
constexpr float TC_RESCALE_THRESHOLD = 8.0f;         // log2 units

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, for x <= 16: x = n + f with n = rint(x) (the
// 1.5 * 2^23 add leaves n in the low mantissa bits of t) and f in
// [-0.5, 0.5]; 2^f from a degree-3 polynomial whose coefficients are a
// relative-error Lawson (iteratively reweighted least-squares) fit of 2^f on
// Chebyshev nodes of [-0.5, 0.5] (max relative error 7.5e-5, below the bf16
// half-ulp 2^-9 that P is rounded to); 2^n is added to the exponent field.
// x is clamped at -126 so the exponent never wraps: masked (-inf) scores give
// a denormal below 1e-38 instead of 0.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = __fadd_rn(x, 12582912.f);
  const float f = __fsub_rn(x, __fsub_rn(t, 12582912.f));
  float p = fmaf(f, 0.05517166f, 0.24261113f);
  p = fmaf(p, f, 0.69326097f);
  p = fmaf(p, f, 0.99992806f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

// Two non-negative finite floats -> bf16x2 (lo in the low half) on the ALU
// pipe: add half an ulp of bf16 and keep the high halves (round half up; the
// tie case differs from round-to-nearest-even only on exact ties).
__device__ __forceinline__ uint32_t pack_bf16x2_alu(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo) + 0x8000u, __float_as_uint(hi) + 0x8000u, 0x7632);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
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

// D(tmem) (+)= A(tmem) * B(smem): A is M x K with row m in TMEM lane m and
// K elements packed two per 32-bit column.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
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

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
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

// 5-D box load: {x, y, z, w, v} coordinates (x innermost).
__device__ __forceinline__ void tma_load_5d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z,
                                            int w, int v) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, "
      "%7}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v)
      : "memory");
}

__device__ __forceinline__ void cp_async16_tc(uint32_t saddr, const void* g, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(n) : "memory");
}

// POLY8 of every 8 scores take exp2 on the FMA pipe (exp2_poly) instead of
// the MUFU pipe; ALU_PACK rounds P to bf16 on the ALU pipe.  Both move work
// off the MUFU/XU pipe.
// TRACE: CTA 0 records clock64() at the handoffs of each block into
// g_attn_trace (diagnostic build only; read with ll_attn_prefill_tc_trace).
constexpr int TC_TRACE_EV = 20;
constexpr int TC_TRACE_BLOCKS = 256;
__device__ unsigned long long g_attn_trace[TC_TRACE_BLOCKS * TC_TRACE_EV];
#define TC_TR(j, e)                                                                   \
  do {                                                                                \
    if (TRACE && blockIdx.x == 0 && (j) < TC_TRACE_BLOCKS)                            \
      g_attn_trace[(j) * TC_TRACE_EV + (e)] = clock64();                              \
  } while (0)

// SCHED 1: the row max over 8 independent chains, and the block's P values
// all computed before any TMEM store (one stream of exp2s, four stores at
// the end) instead of a store after every 32 columns.
template <int CS, int POLY8, bool ALU_PACK, bool TRACE = false, int SCHED = 0>
__global__ void __launch_bounds__(TcCfg<CS>::THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           const bf16* __restrict__ q, const int* __restrict__ q_indptr,
                           const int* __restrict__ q_pos, const int* __restrict__ page_table, int pt_stride,
                           const int4* __restrict__ tiles, bf16* __restrict__ out, int Hq, int Hkv, int ps,
                           int layer, float scale_log2, int* err, int nsplit_arg, float* __restrict__ ws_o,
                           float* __restrict__ ws_ml) {
  using Cfg = TcCfg<CS>;
  constexpr int NC = Cfg::NC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [TC_NT][Q]
  uint8_t* sK = sQ + TC_NT * TC_Q_BYTES;                // [KS][KV]
  uint8_t* sV = sK + TC_KS * TC_KV_BYTES;               // [VS][KV]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + TC_VS * TC_KV_BYTES);
  uint64_t* k_full = bars;
  uint64_t* k_empty = k_full + TC_KS;
  uint64_t* v_full = k_empty + TC_KS;
  uint64_t* v_empty = v_full + TC_VS;
  uint64_t* s_full = v_empty + TC_VS;   // [TC_NT]
  uint64_t* p_full = s_full + TC_NT;    // [TC_NT]
  uint64_t* q_full = p_full + TC_NT;
  uint64_t* o_full = q_full + 1;
  uint64_t* x_bar = o_full + 1;         // [TC_NT][4] CS == 2: max / sum exchange per lane quarter
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_bar + 4 * TC_NT);
  float* xbuf = reinterpret_cast<float*>(smem + TC_SMEM_BASE - 1024);  // [TC_NT][2][CS][TC_BM]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int4 tile = tiles[blockIdx.x];
  // tile.y = kv head | split << 8 | split count << 16 (split count 0 = 1):
  // with a split count S > 1 this CTA walks the split-th of S equal key
  // ranges of the tile and writes an unnormalised partial (fp32 O, running
  // max in the log2 domain, row sum) for attn_combine_kernel.
  const int b = tile.x, hk = tile.y & 0xff, row0 = tile.z, max_pos = tile.w;
  const int split = (tile.y >> 8) & 0xff, nsplit = max(1, tile.y >> 16);
  if (nsplit != max(1, nsplit_arg) || (nsplit > 1 && (ws_o == nullptr || ws_ml == nullptr))) {
    if (threadIdx.x == 0) record_error(err, kErrBadIndex);  // work list and launch disagree: nothing written
    return;
  }
  const int g = Hq / Hkv;
  const int s0 = q_indptr[b];
  const int nrows = (q_indptr[b + 1] - s0) * g;
  const int nb_all = max_pos / TC_BN + 1;
  const int chunk = (nb_all + nsplit - 1) / nsplit;
  const int jb = min(nb_all, split * chunk);   // first key block of this CTA
  const int nb = min(nb_all, jb + chunk) - jb;  // its key blocks (0 for an empty split)
  const int* pt = page_table + (size_t)b * pt_stride;

  if (threadIdx.x == 0) {
    for (int i = 0; i < TC_KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < TC_VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < TC_NT; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4 * CS);
    }
    for (int i = 0; i < 4 * TC_NT; ++i) mbar_init(&x_bar[i], 64);  // both halves' 32 threads
    mbar_init(q_full, 4 * TC_NT * CS);
    mbar_init(o_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TC_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Cfg::REGS_CTRL));
    if (warp == 0) {
      // ------------------------------------------------------------ producer
      // The whole warp: lane p owns page p of a block (page_size >= 4, so a
      // block spans at most 32 pages).  Its page-table entry for block j+1 is
      // loaded while block j streams, and each lane issues its own page's
      // TMA boxes, so neither the page-table latency nor the TMA issue is
      // serialised on one thread.
      if (lane == 0) {
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
      }
      const int ppb = TC_BN / ps;
      auto page_of = [&](int j) -> int {
        const int key0 = j * TC_BN + lane * ps;
        if (lane >= ppb || key0 > max_pos) return -1;  // -1: out of range, zero fill
        if (key0 / ps >= pt_stride) {  // past the page-table row: recorded, zero fill
          record_error(err, kErrBadIndex);
          return -1;
        }
        return pt[key0 / ps] * Hkv + hk;
      };
      auto load_block = [&](const CUtensorMap* tm, uint8_t* dst, uint64_t* bar, int y) {
        if (lane == 0) mbar_arrive_expect_tx(bar, TC_KV_BYTES);
        __syncwarp();
        if (lane < ppb) {
#pragma unroll
          for (int h = 0; h < 2; ++h) tma_load_4d(dst + h * TC_KV_HALF + lane * ps * 128, tm, bar, 64 * h, 0, y, layer);
        }
      };
      bool ok = true;
      int y_next = nb > 0 ? page_of(jb) : -1;
      for (int j = 0; j < nb; ++j) {  // j: block of this CTA's range (ring index); jb + j: key block
        const int y = y_next;
        if (j + 1 < nb) y_next = page_of(jb + j + 1);
        const int sk = j % TC_KS, sv = j % TC_VS;
        bool w = true;
        if (lane == 0) w = mbar_wait(&k_empty[sk], ((j / TC_KS) & 1) ^ 1, err, kErrSmemEmptyTimeout);
        if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
        load_block(&tmK, sK + sk * TC_KV_BYTES, &k_full[sk], y);
        if (lane == 0) w = mbar_wait(&v_empty[sv], ((j / TC_VS) & 1) ^ 1, err, kErrSmemEmptyTimeout);
        if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
        load_block(&tmV, sV + sv * TC_KV_BYTES, &v_full[sv], y);
      }
      if (!ok && lane == 0) {
        unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {
        }
      }
      __syncwarp();
    } else if (warp == 1) {
      // ----------------------------------------------------------------- MMA
      if (lane == 0) {
        constexpr uint32_t idesc_s = umma_idesc_bf16_f32(TC_BM, TC_BN);
        constexpr uint32_t idesc_pv = umma_idesc_bf16_f32(TC_BM, TC_D) | (1u << 16);  // B (V) MN-major
        bool ok = mbar_wait(q_full, 0, err, kErrTmaFullTimeout);
        tc_fence_after();
        // Descriptors advance by adding byte offsets / 16 to their address
        // field (shared addresses stay below 256 KB, so it never carries).
        const uint64_t q_desc0 = umma_desc_sw128_kmajor(smem_u32(sQ));
        const uint64_t k_desc0 = umma_desc_sw128_kmajor(smem_u32(sK));
        const uint64_t v_desc0 = umma_desc_sw128_mnmajor(smem_u32(sV), TC_KV_HALF, 1024);
        // O_t += P_t(i) V_i (P from TMEM columns [128t, 128t + 64)).
        auto issue_pv = [&](int t, int i) {
          const uint64_t vd = v_desc0 + (uint64_t)(((i % TC_VS) * TC_KV_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < TC_BN / 16; ++k)
            umma_bf16_ts(tmem + 256 + 128 * t, tmem + 128 * t + 8 * k, vd + (uint64_t)((k * 16 * 128) >> 4), idesc_pv,
                         (i > 0 || k > 0) ? 1u : 0u);
        };
        for (int j = 0; j < nb && ok; ++j) {
          const int sk = j % TC_KS;
          const uint64_t kd = k_desc0 + (uint64_t)((sk * TC_KV_BYTES) >> 4);
#pragma unroll
          for (int t = 0; t < TC_NT; ++t) {
            if (j > 0) {
              if (!mbar_wait(&p_full[t], (j - 1) & 1, err, kErrTmemFullTimeout)) { ok = false; break; }
              TC_TR(j, 7 + t);
              if (t == 0 && !mbar_wait(&v_full[(j - 1) % TC_VS], ((j - 1) / TC_VS) & 1, err, kErrTmaFullTimeout)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_pv(t, j - 1);
              if (t == TC_NT - 1) umma_commit(&v_empty[(j - 1) % TC_VS]);
            }
            if (t == 0) {  // K_j is needed only from here: PV of block j-1 did not wait for it
              if (!mbar_wait(&k_full[sk], (j / TC_KS) & 1, err, kErrTmaFullTimeout)) { ok = false; break; }
              TC_TR(j, 6);
              tc_fence_after();
            }
            const uint64_t qd = q_desc0 + (uint64_t)((t * TC_Q_BYTES) >> 4);
#pragma unroll
            for (int k = 0; k < TC_D / 16; ++k) {
              const uint32_t off = ((k >> 2) * TC_Q_HALF + (k & 3) * 32) >> 4;  // TC_Q_HALF == TC_KV_HALF
              umma_bf16(tmem + 128 * t, qd + off, kd + off, idesc_s, k > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[t]);
            TC_TR(j, 9 + t);
          }
          if (!ok) break;
          umma_commit(&k_empty[sk]);
        }
        if (ok && nb > 0) {
          const int i = nb - 1;
          for (int t = 0; t < TC_NT && ok; ++t) {
            if (!mbar_wait(&p_full[t], i & 1, err, kErrTmemFullTimeout)) { ok = false; break; }
            if (t == 0 && !mbar_wait(&v_full[i % TC_VS], (i / TC_VS) & 1, err, kErrTmaFullTimeout)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, i);
          }
          if (ok) umma_commit(&v_empty[i % TC_VS]);
        }
        umma_commit(o_full);  // also drains every MMA issued above
        mbar_wait(o_full, 0, nullptr, 0);
      }
      __syncwarp();
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Cfg::REGS_SOFTMAX));
    // ------------------------------------------------------------- softmax
    const int sg = (warp - 4) >> 2;       // softmax warpgroup
    const int t = sg / CS;                // tile of this warpgroup
    const int h = sg % CS;                // its share of the key columns: [h * NC, (h + 1) * NC)
    const int qd = warp & 3;              // TMEM lane quarter of this warp
    const int r = qd * 32 + lane;         // query row of this thread within the tile
    const int pr = row0 + t * TC_BM + r;
    const bool valid = pr < nrows;
    const int tok = s0 + pr / g;
    const int head = hk * g + pr % g;
    const int pos = valid ? q_pos[tok] : -1;
    uint8_t* sQt = sQ + t * TC_Q_BYTES;
    // Q row -> shared memory (two 128-B halves, 128-B swizzle; with CS = 2
    // each half-thread copies 8 of the row's 16 chunks), then signal.
    {
      const bf16* src = q + ((size_t)tok * Hq + head) * TC_D;
#pragma unroll
      for (int i = 0; i < 16 / CS; ++i) {
        const int c = h * (16 / CS) + i;
        const int hh = c >> 3, cc = c & 7;
        const uint32_t dst = smem_u32(sQt) + hh * TC_Q_HALF + r * 128 + ((cc ^ (r & 7)) << 4);
        cp_async16_tc(dst, valid ? (const void*)(src + c * 8) : (const void*)q, valid);
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    }
    const uint32_t lane_base = tmem + (uint32_t(qd * 32) << 16);
    const uint32_t s_col = lane_base + 128 * t + h * NC;        // this thread's S columns
    const uint32_t p_col = lane_base + 128 * t + h * (NC / 2);  // its P (bf16 pairs)
    const uint32_t o_col = lane_base + 256 + 128 * t + h * (TC_D / CS);
    uint64_t* xb = &x_bar[t * 4 + qd];
    // exchange slot of (tile, parity, half) for this row
    auto xslot = [&](int par, int hh) -> float* { return xbuf + ((t * 2 + par) * CS + hh) * TC_BM + r; };
    // Both halves of a row publish a value and read the other's; false when
    // the (bounded) wait gave up, which it records.
    auto exchange = [&](int phase, float v, float& other) -> bool {
      *xslot(phase & 1, h) = v;
      mbar_arrive(xb);
      if (!mbar_wait(xb, phase & 1, err, kErrTmemFullTimeout)) return false;
      other = *xslot(phase & 1, h ^ 1);
      return true;
    };
    float m_run = -INFINITY, l_run = 0.f;
    // Blocks before jd are visible to every row of this tile (positions
    // ascend, so the tile's first row has its smallest position) and skip
    // the causal mask; the mask is compiled into a separate copy of the
    // block step so unmasked blocks carry none of its per-score selects.
    const int pr0 = row0 + t * TC_BM;
    const int tile_min_pos = pr0 < nrows ? q_pos[s0 + pr0 / g] : -1;
    const int jd = min((tile_min_pos + 1) / TC_BN, nb);
    auto step = [&](int j, auto mask_c) -> bool {
      constexpr bool MASK = decltype(mask_c)::value;
      if (!mbar_wait(&s_full[t], j & 1, err, kErrTmemFullTimeout)) return false;
      if (r == 0 && h == 0) TC_TR(j, 3 * t);
      tc_fence_after();
      uint32_t s[NC];
#pragma unroll
      for (int c = 0; c < NC / 32; ++c)
        tmem_ld_32x32b_x32(s_col + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&s[32 * c]));
      tmem_ld_wait();
      if (r == 0 && h == 0) TC_TR(j, 3 * t + 1);
      if (MASK) {
        const int lim = pos - (jb + j) * TC_BN - h * NC;  // scores with index > lim are masked
#pragma unroll
        for (int i = 0; i < NC; ++i)
          if (i > lim) s[i] = __float_as_uint(-INFINITY);
      }
      if (r == 0 && t == 0 && h == 0) TC_TR(j, 17);
      float mx;
      if constexpr (SCHED == 1) {
        float m8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) m8[u] = fmaxf(__uint_as_float(s[2 * u]), __uint_as_float(s[2 * u + 1]));
#pragma unroll
        for (int i = 16; i < NC; i += 16) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            m8[u] = fmax3(m8[u], __uint_as_float(s[i + 2 * u]), __uint_as_float(s[i + 2 * u + 1]));
        }
        mx = fmaxf(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], fmax3(m8[5], m8[6], m8[7])));
      } else {
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < NC; i += 8) {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            m4[u] = fmax3(m4[u], __uint_as_float(s[i + 2 * u]), __uint_as_float(s[i + 2 * u + 1]));
        }
        mx = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
      }
      if constexpr (CS == 2) {
        float other;
        if (!exchange(j, mx, other)) return false;
        mx = fmaxf(mx, other);
      }
      if (r == 0 && t == 0 && h == 0) TC_TR(j, 11);
      const float m_new = fmaxf(m_run, mx * scale_log2);
      const bool grow = m_new > m_run + TC_RESCALE_THRESHOLD;  // false while m_new == -inf
      const float m_use = grow ? m_new : m_run;
      const float o_scale = (grow && m_run != -INFINITY) ? ex2(m_run - m_new) : 1.f;
      const float neg_m = m_use == -INFINITY ? 0.f : -m_use;
      // P = exp2(S*scale - m) as bf16 pairs over this thread's share of the
      // first 64 columns of S.
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      if constexpr (SCHED == 1) {
        // the P values overwrite the scores they come from (s[e] holds pair
        // e once s[2e], s[2e+1] are consumed), then four stores
#pragma unroll
        for (int e = 0; e < NC / 2; ++e) {
          const float xa = fmaf(__uint_as_float(s[2 * e]), scale_log2, neg_m);
          const float xb2 = fmaf(__uint_as_float(s[2 * e + 1]), scale_log2, neg_m);
          const float pa = ((2 * e) & 7) < POLY8 ? exp2_poly(xa) : ex2(xa);
          const float pb = ((2 * e + 1) & 7) < POLY8 ? exp2_poly(xb2) : ex2(xb2);
          sum4[e & 3] += pa + pb;
          s[e] = ALU_PACK ? pack_bf16x2_alu(pa, pb) : pack_bf16x2(pa, pb);
        }
#pragma unroll
        for (int c = 0; c < NC / 32; ++c)
          tmem_st_32x32b_x16(p_col + 16 * c, *reinterpret_cast<const uint32_t(*)[16]>(&s[16 * c]));
        if (r == 0 && t == 0 && h == 0) TC_TR(j, 15);
      } else {
        for (int c = 0; c < NC / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int i0 = 32 * c + 2 * e;
            const float xa = fmaf(__uint_as_float(s[i0]), scale_log2, neg_m);
            const float xb2 = fmaf(__uint_as_float(s[i0 + 1]), scale_log2, neg_m);
            const float pa = (i0 & 7) < POLY8 ? exp2_poly(xa) : ex2(xa);
            const float pb = ((i0 + 1) & 7) < POLY8 ? exp2_poly(xb2) : ex2(xb2);
            sum4[e & 3] += pa + pb;
            pk[e] = ALU_PACK ? pack_bf16x2_alu(pa, pb) : pack_bf16x2(pa, pb);
          }
          tmem_st_32x32b_x16(p_col + 16 * c, pk);
          if (r == 0 && t == 0 && h == 0) TC_TR(j, 12 + c);
        }
      }
      const float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
      // O is stable here: PV of block j-1 was issued before S(j) and the
      // commit that signalled S(j) covers it.  Each half rescales its
      // share of O's columns (both halves see the same row maxima).
      if (__any_sync(0xffffffffu, o_scale != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < TC_D / CS; c += 32) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(o_col + c, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * o_scale);
          tmem_st_32x32b_x32(o_col + c, o);
        }
      }
      tmem_st_wait();
      if (r == 0 && t == 0 && h == 0) TC_TR(j, 16);
      l_run = l_run * o_scale + sum;
      m_run = m_use;
      tc_fence_before();
      __syncwarp();
      if (r == 0 && h == 0) TC_TR(j, 3 * t + 2);
      if (lane == 0) mbar_arrive(&p_full[t]);
      return true;
    };
    bool ok = true;
    int j = 0;  // block of this CTA's range; jb + j is the key block
    for (; j < nb && jb + j < jd && ok; ++j) ok = step(j, std::false_type{});
    for (; j < nb && ok; ++j) ok = step(j, std::true_type{});
    // ----------------------------------------------------------- epilogue
    if (ok && mbar_wait(o_full, 0, err, kErrTmemFullTimeout)) {
      float l_tot = l_run;
      if constexpr (CS == 2) {
        float other = 0.f;
        ok = exchange(nb, l_run, other);  // the row sum is the two halves' sums
        l_tot += other;
      }
      tc_fence_after();
      if (nsplit > 1) {
        // partial of this key range: O as accumulated (fp32, not divided by
        // the row sum) and (running max, row sum); an empty range writes
        // zeros and a max of -inf, which the combine weighs by 0
        const size_t prow = ((size_t)tok * Hq + head) * nsplit + split;
        float4* po = reinterpret_cast<float4*>(ws_o + prow * TC_D + h * (TC_D / CS));
#pragma unroll 1
        for (int c = 0; c < TC_D / CS; c += 32) {
          uint32_t o[32];
          if (nb > 0) {
            tmem_ld_32x32b_x32(o_col + c, o);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0u;
          }
          if (valid) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              po[c / 4 + i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                          __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
          }
        }
        if (valid && h == 0) reinterpret_cast<float2*>(ws_ml)[prow] = make_float2(m_run, l_tot);
      }
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
      bf16* dst = out + ((size_t)tok * Hq + head) * TC_D + h * (TC_D / CS);
#pragma unroll 1
      for (int c = 0; c < TC_D / CS && ok && nsplit == 1; c += 32) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(o_col + c, o);
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

// 5-D map over the same pool viewed as {D, ps, Hkv, pages, L}; box =
// {64, ps, 1, run, 1}: `run` consecutive pages of one kv head in one box.
static int make_pool_run_map(CUtensorMap* tm, const void* base, int L, int pages, int Hkv, int ps, int run) {
  EncodeTiledFn2 enc = encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[5] = {(cuuint64_t)TC_D, (cuuint64_t)ps, (cuuint64_t)Hkv, (cuuint64_t)pages, (cuuint64_t)L};
  cuuint64_t strides[4] = {(cuuint64_t)TC_D * 2, (cuuint64_t)ps * TC_D * 2, (cuuint64_t)Hkv * ps * TC_D * 2,
                           (cuuint64_t)pages * Hkv * ps * TC_D * 2};
  cuuint32_t box[5] = {64, (cuuint32_t)ps, 1, (cuuint32_t)run, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

typedef void (*Kern)(CUtensorMap, CUtensorMap, const bf16*, const int*, const int*, const int*, int, const int4*,
                     bf16*, int, int, int, int, float, int*, int, float*, float*);
// Builds of the kernel, LL_ATTN_VARIANT=<index> selects one:
//   0  CS = 1, exp2 on MUFU        3  CS = 2, exp2 on MUFU
//   1  CS = 1, bf16 pack on ALU    4  CS = 2, 2 of 8 exp2 on the FMA pipe
//   2  CS = 1, 2 of 8 exp2 on FMA  5, 6  clock64() trace builds of 0 and 3
struct TcBuild {
  Kern kern;
  int threads, smem;
};
template <int CS, int POLY8, bool ALU_PACK, bool TRACE = false, int SCHED = 0>
constexpr TcBuild tc_build() {
  return {attn_prefill_tc_kernel<CS, POLY8, ALU_PACK, TRACE, SCHED>, TcCfg<CS>::THREADS, TcCfg<CS>::SMEM};
}
//   7  CS = 1, SCHED 1 (8-chain max, P stored after the whole row)
//   8  CS = 1, SCHED 1, 2 of 8 exp2 on FMA   9  trace build of 7
constexpr int kNumVariants = 10;
static const TcBuild kVariants[kNumVariants] = {
    tc_build<1, 0, false>(),       tc_build<1, 0, true>(),  tc_build<1, 2, true>(), tc_build<2, 0, false>(),
    tc_build<2, 2, true>(),        tc_build<1, 0, false, true>(), tc_build<2, 0, false, true>(),
    tc_build<1, 0, false, false, 1>(), tc_build<1, 2, false, false, 1>(), tc_build<1, 0, false, true, 1>()};
constexpr int kDefaultVariant = 7;  // SCHED 1: 0.521 vs 0.533 ms on the Link repair case

static int g_attn_variant = -1;

static int attn_tc_variant() {
  if (g_attn_variant < 0) {
    const char* e = getenv("LL_ATTN_VARIANT");
    g_attn_variant = e != nullptr ? atoi(e) : kDefaultVariant;
    if (g_attn_variant < 0 || g_attn_variant >= kNumVariants) g_attn_variant = kDefaultVariant;
  }
  return g_attn_variant;
}

// ----------------------------------------------------------------- decode
// One query token per request, split-KV.  grid (B*Hkv, nsplit), block 160:
// warps 0-3 compute, warp 4 is the TMA producer.  A CTA owns one contiguous
// key range of one (request, kv head); its page-table entries are copied to
// shared memory once, then 64-key K/V blocks arrive by TMA (one box of
// page_size keys x 64 dims per page and half, 128-byte swizzle) in a 3-stage
// ring, 16 bulk copies per block instead of 2048 16-byte copies.  Warp w takes
// keys [16w, 16w+16) of every block with its own online softmax on mma.sync
// m16n8k16 (16 rows = the token's g query heads); the warps' (m, l, O) are
// merged in shared memory.  Output: final rows (nsplit == 1) or unnormalised
// partials [B*Hq, nsplit, D] + (max log2, sum) for attn_combine_kernel.
constexpr int DT_BN = 64;
constexpr int DT_STAGES = 3;
constexpr int DT_THREADS = 160;
constexpr int DT_MAXP = 1024;
constexpr int DT_HALF = DT_BN * 128;                 // 8 KB: one 64-dim half of a 64-key block
constexpr int DT_KV = 2 * DT_HALF;                   // 16 KB per K (or V) block
constexpr int dt_smem(int stages) { return 1024 + 4096 + stages * 2 * DT_KV + DT_MAXP * 4 + 128; }
constexpr int DT_SMEM = dt_smem(DT_STAGES);  // 3 stages (default)
constexpr int DT_SMEM2 = dt_smem(2);          // 2 stages (LL_DECODE_STAGES=2): fits beside two 72 KB GEMV CTAs

__device__ __forceinline__ uint32_t dt_swz(int key, int c16) {  // TMA 128-byte swizzle, two 64-dim halves
  return (uint32_t)((c16 >> 3) * DT_HALF + key * 128 + (((c16 & 7) ^ (key & 7)) << 4));
}
__device__ __forceinline__ uint32_t dt_qswz(int row, int c16) {  // Q: 256-byte rows, XOR swizzle
  return (uint32_t)(row * 256 + ((c16 ^ (row & 7)) << 4));
}
__device__ __forceinline__ void dt_ldsm(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void dt_ldsm_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void dt_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int ST>
__global__ void __launch_bounds__(DT_THREADS)
    attn_decode_tma_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           const __grid_constant__ CUtensorMap tmKr, const __grid_constant__ CUtensorMap tmVr,
                           const bf16* __restrict__ q, const int* __restrict__ page_table, int pt_stride,
                           const int* __restrict__ kv_lens, bf16* __restrict__ out, float* __restrict__ ws_o,
                           float* __restrict__ ws_ml, int Hq, int Hkv, int ps, float scale_log2, int new_tokens,
                           int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sKV = smem;                                  // [stage][K|V][2 halves][64 keys][128 B]
  uint8_t* sQb = sKV + ST * 2 * DT_KV;           // 16 rows x 256 B
  int* spage = reinterpret_cast<int*>(sQb + 4096);
  uint64_t* full = reinterpret_cast<uint64_t*>(spage + DT_MAXP);
  uint64_t* empty = full + ST;
  const uint32_t sQ = smem_u32(sQb);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmKr);
    prefetch_tmap(&tmVr);
  }
  pdl_trigger();
  // Before the wait on the previous kernel: the kv lengths and page table
  // (written before this step's first kernel) and the K/V of every key but
  // the newest `new_tokens` of each request (written by earlier steps).  Only
  // Q and those newest keys come from the previous kernel (rope + KV write),
  // so the page list and the first blocks stream in while it finishes.
  const int b = blockIdx.x / Hkv, hk = blockIdx.x % Hkv;
  const int split = blockIdx.y, nsplit = gridDim.y;
  const int g = Hq / Hkv;
  int kv_len = kv_lens[b];
  if (kv_len < 0 || kv_len > pt_stride * ps) {  // more keys than the page-table row holds: recorded, clamped
    if (threadIdx.x == 0) record_error(err, kErrBadIndex);
    kv_len = kv_len < 0 ? 0 : pt_stride * ps;
  }
  const int fresh0 = kv_len - new_tokens;  // keys >= fresh0 are read only after the wait
  int chunk = (kv_len + nsplit - 1) / nsplit;
  chunk = (chunk + DT_BN - 1) / DT_BN * DT_BN;
  const int kbeg = min(kv_len, split * chunk);
  const int kend = min(kv_len, kbeg + chunk);
  const int nblocks = (kend - kbeg + DT_BN - 1) / DT_BN;
  const int* pt = page_table + (size_t)b * pt_stride;
  const int p0 = kbeg / ps;
  const int npages = kend > kbeg ? (kend - 1) / ps - p0 + 1 : 0;
  for (int i = tid; i < npages && i < DT_MAXP; i += DT_THREADS) spage[i] = pt[p0 + i];
  __syncthreads();  // barriers initialised, page list in shared memory

  float O[16][4];
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  if (warp == 4) {
    // ---------------------------------------------------------- producer
    // The whole warp issues: lane (p, h, kv) = (lane >> 2, (lane >> 1) & 1,
    // lane & 1) owns one box of page p, so a block's 16 boxes (page_size 16)
    // go out in one instruction instead of 16 serial ones from one thread.
    const int pages_per_block = DT_BN / ps;
    const int p = lane >> 2, h = (lane >> 1) & 1, isv = lane & 1;
    bool waited = false;
    for (int blk = 0; blk < nblocks; ++blk) {
      const int st = blk % ST;
      if (!waited && kbeg + (blk + 1) * DT_BN > fresh0) {
        pdl_wait();  // this block holds keys the previous kernel wrote
        waited = true;
      }
      bool w = true;
      if (lane == 0) {
        w = mbar_wait(&empty[st], ((blk / ST) & 1) ^ 1, err, kErrSmemEmptyTimeout);
        if (w) mbar_arrive_expect_tx(&full[st], 2 * DT_KV);
      }
      if (!__shfl_sync(0xffffffffu, w, 0)) break;
      // A block whose pages are one ascending run (the usual case: the
      // allocator hands out ascending runs) goes as 4 boxes of the whole
      // block -- fewer, larger TMA boxes stream several times faster.
      const int lp0 = (kbeg + blk * DT_BN) / ps - p0;
      bool run = kbeg + (blk + 1) * DT_BN <= kend && lp0 + pages_per_block <= DT_MAXP;
      if (run) {
        const int base_page = spage[lp0];
        const int i = lane < pages_per_block ? lane : 0;
        run = __all_sync(0xffffffffu, spage[lp0 + i] == base_page + i);
        if (run) {
          if (lane < 4) {
            const int hh = lane >> 1, vv = lane & 1;
            uint8_t* dst = sKV + st * 2 * DT_KV + vv * DT_KV + hh * DT_HALF;
            tma_load_5d(dst, vv ? &tmVr : &tmKr, &full[st], 64 * hh, 0, hk, base_page, 0);
          }
          continue;
        }
      }
      for (int pp = p; pp < pages_per_block; pp += 8) {
        const int key0 = kbeg + blk * DT_BN + pp * ps;
        const int lp = key0 / ps - p0;
        const int y = key0 < kend ? (lp < DT_MAXP ? spage[lp] : pt[p0 + lp]) * Hkv + hk : -1;  // -1: zero fill
        uint8_t* dst = sKV + st * 2 * DT_KV + isv * DT_KV + h * DT_HALF + pp * ps * 128;
        tma_load_4d(dst, isv ? &tmV : &tmK, &full[st], 64 * h, 0, y, 0);
      }
    }
  } else {
    // ---------------------------------------------------------- consumers
    pdl_wait();  // Q (and the outputs' previous readers) belong to earlier kernels
    {
      const int c = tid & 15;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int r = (tid >> 4) + 8 * i;
        const bool ok = r < g;
        const bf16* src = ok ? q + (((size_t)b * Hq + hk * g + r) * 128 + c * 8) : q;
        const int n = ok ? 16 : 0;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sQ + dt_qswz(r, c)), "l"(src), "r"(n)
                     : "memory");
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four compute warps: Q in shared memory
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) O[i][0] = O[i][1] = O[i][2] = O[i][3] = 0.f;
    uint32_t qf[8][4];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int r = (lane & 7) + 8 * ((lane >> 3) & 1);
      dt_ldsm(sQ + dt_qswz(r, 2 * kk + (lane >> 4)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
    for (int blk = 0; blk < nblocks; ++blk) {
      const int st = blk % ST;
      if (!mbar_wait(&full[st], (blk / ST) & 1, err, kErrTmaFullTimeout)) break;
      const uint32_t sK = smem_u32(sKV + st * 2 * DT_KV);
      const uint32_t sV = sK + DT_KV;
      const int k0 = kbeg + blk * DT_BN + 16 * warp;  // this warp's 16 keys
      if (k0 + 16 > kend) {
        // Rows past the last key hold whatever the page held: zero this
        // warp's V rows there so that P = 0 never meets a non-finite V.
        const int r = lane >> 1;
        if (k0 + r >= kend) {
          uint4* vrow0 = reinterpret_cast<uint4*>(sKV + st * 2 * DT_KV + DT_KV + (lane & 1) * DT_HALF +
                                                  (16 * warp + r) * 128);
#pragma unroll
          for (int i = 0; i < 8; ++i) vrow0[i] = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      float S[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i) S[i][0] = S[i][1] = S[i][2] = S[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t b0, b1, b2, b3;
        const int key = 16 * warp + (lane & 7) + 8 * (lane >> 4);
        dt_ldsm(sK + dt_swz(key, 2 * kk + ((lane >> 3) & 1)), b0, b1, b2, b3);
        dt_mma(S[0], qf[kk], b0, b1);
        dt_mma(S[1], qf[kk], b2, b3);
      }
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
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
      const float al_a = (mn_a == -INFINITY) ? 1.f : ex2(m_a - mn_a);
      const float al_b = (mn_b == -INFINITY) ? 1.f : ex2(m_b - mn_b);
      const float sub_a = (mn_a == -INFINITY) ? 0.f : mn_a;
      const float sub_b = (mn_b == -INFINITY) ? 0.f : mn_b;
      m_a = mn_a;
      m_b = mn_b;
      float rs_a = 0.f, rs_b = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        S[nt][0] = ex2(S[nt][0] - sub_a);
        S[nt][1] = ex2(S[nt][1] - sub_a);
        S[nt][2] = ex2(S[nt][2] - sub_b);
        S[nt][3] = ex2(S[nt][3] - sub_b);
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
      uint32_t a[4];
      a[0] = pack_bf16x2(S[0][0], S[0][1]);
      a[1] = pack_bf16x2(S[0][2], S[0][3]);
      a[2] = pack_bf16x2(S[1][0], S[1][1]);
      a[3] = pack_bf16x2(S[1][2], S[1][3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int key = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1);
        dt_ldsm_t(sV + dt_swz(key, 2 * dp + (lane >> 4)), b0, b1, b2, b3);
        dt_mma(O[2 * dp], a, b0, b1);
        dt_mma(O[2 * dp + 1], a, b2, b3);
      }
      fence_proxy_async();  // generic accesses of the stage before the next TMA write
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  }
  // ---- merge the four compute warps (every issued block was consumed, so
  // the ring is free).  Only the g real query rows are written; the slices
  // use an XOR swizzle (column ^ 8 * row) so that a warp's float2 stores and
  // the summing threads' float4 loads are free of bank conflicts.
  __syncthreads();
  float* sm = reinterpret_cast<float*>(sKV);  // [4 warps][16 rows] m, then l
  float* sw = sm + 2 * 4 * 16;                // [4 warps][16 rows][128] fp32, scaled partial O
  const int ra = lane >> 2, rb = ra + 8;
  if (warp < 4 && (lane & 3) == 0) {
    sm[warp * 16 + ra] = m_a;
    sm[warp * 16 + rb] = m_b;
    sm[64 + warp * 16 + ra] = l_a;
    sm[64 + warp * 16 + rb] = l_b;
  }
  __syncthreads();
  if (warp < 4) {
    float Ma = -INFINITY, Mb = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      Ma = fmaxf(Ma, sm[w * 16 + ra]);
      Mb = fmaxf(Mb, sm[w * 16 + rb]);
    }
    const float fa = (m_a == -INFINITY) ? 0.f : ex2(m_a - Ma);
    const float fb = (m_b == -INFINITY) ? 0.f : ex2(m_b - Mb);
    float* mine = sw + warp * 16 * 128;
    if (ra < g) {
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        const int d = (nt * 8 + 2 * (lane & 3)) ^ (ra << 3);
        *reinterpret_cast<float2*>(&mine[ra * 128 + d]) = make_float2(O[nt][0] * fa, O[nt][1] * fa);
      }
    }
    if (rb < g) {
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        const int d = (nt * 8 + 2 * (lane & 3)) ^ (rb << 3);
        *reinterpret_cast<float2*>(&mine[rb * 128 + d]) = make_float2(O[nt][2] * fb, O[nt][3] * fb);
      }
    }
  }
  __syncthreads();
  // thread -> 16 consecutive columns of one row: sum the four slices and
  // write the final row (nsplit == 1) or this split's partial
  if (tid < 128 && (tid >> 3) < g) {
    const int r = tid >> 3, d0 = (tid & 7) * 16;
    float M = -INFINITY, Lsum = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm[w * 16 + r]);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = sm[w * 16 + r];
      Lsum += (mw == -INFINITY) ? 0.f : sm[64 + w * 16 + r] * ex2(mw - M);
    }
    float acc[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = r * 128 + ((d0 + 4 * i) ^ (r << 3));
      float4 a4 = *reinterpret_cast<const float4*>(&sw[e]);
#pragma unroll
      for (int w = 1; w < 4; ++w) {
        const float4 v = *reinterpret_cast<const float4*>(&sw[w * 16 * 128 + e]);
        a4.x += v.x;
        a4.y += v.y;
        a4.z += v.z;
        a4.w += v.w;
      }
      acc[4 * i] = a4.x;
      acc[4 * i + 1] = a4.y;
      acc[4 * i + 2] = a4.z;
      acc[4 * i + 3] = a4.w;
    }
    const size_t row = (size_t)b * Hq + hk * g + r;
    if (nsplit == 1) {
      const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pk[i] = pack_bf16x2(acc[2 * i] * inv, acc[2 * i + 1] * inv);
      uint4* dst = reinterpret_cast<uint4*>(out + row * 128 + d0);
      dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    } else {
      const size_t idx = row * nsplit + split;
      float4* dst = reinterpret_cast<float4*>(ws_o + idx * 128 + d0);
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
      if ((tid & 7) == 0) *reinterpret_cast<float2*>(ws_ml + idx * 2) = make_float2(M, Lsum);
    }
  }
}

}  // namespace ll

using namespace ll;

// k_pool / v_pool: whole pools [L, pages, Hkv, ps, 128]; `layer` selects the layer.
extern "C" int ll_attn_combine(bf16* out, const float* ws_o, const float* ws_ml, int rows, int nsplit,
                               cudaStream_t stream);

// tiles: one int4 per CTA (see the kernel).  nsplit > 1: every tile appears
// as nsplit work items over equal key ranges, each writes a partial for row
// (token * Hq + head) into ws_o [rows][nsplit][128] / ws_ml [rows][nsplit][2],
// and the combine (rows = tokens * Hq) writes `out`.
extern "C" int ll_attn_prefill_tc(const bf16* q, const bf16* k_pool, const bf16* v_pool, int L, int pages, int layer,
                                  const int* q_indptr, const int* q_pos, const int* page_table, int pt_stride,
                                  const int* tiles, int ntiles, bf16* out, int Hq, int Hkv, int head_dim,
                                  int page_size, float scale, int* err, int nsplit, float* ws_o, float* ws_ml,
                                  int combine_rows, cudaStream_t stream) {
  if (ntiles <= 0) return 0;
  if (head_dim != TC_D || Hq % Hkv || Hkv > 256) return -3;
  if (nsplit < 1 || nsplit > 255 || (nsplit > 1 && (ws_o == nullptr || ws_ml == nullptr || combine_rows <= 0)))
    return -3;
  if (page_size < 4 || page_size > TC_BN || TC_BN % page_size) return -3;  // one producer lane per page
  if (Hq / Hkv > TC_BM) return -3;
  CUtensorMap tk, tv;
  if (make_pool_map(&tk, k_pool, L, pages, Hkv, page_size)) return -2;
  if (make_pool_map(&tv, v_pool, L, pages, Hkv, page_size)) return -2;
  const int v = attn_tc_variant();
  const TcBuild& bd = kVariants[v];
  Kern kern = bd.kern;
  // A launch whose registers or shared memory cannot fit one CTA on an SM is
  // refused here: such launches crashed the host process inside the driver
  // instead of returning an error.
  static int fits[kNumVariants] = {};  // 0: not checked yet, 1: fits, 2: refused
  if (fits[v] == 0) {
    int n = 0;
    fits[v] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bd.smem) == cudaSuccess &&
                      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, bd.threads, bd.smem) == cudaSuccess &&
                      n >= 1
                  ? 1
                  : 2;
  }
  if (fits[v] != 1) return -7;
  kern<<<ntiles, bd.threads, bd.smem, stream>>>(tk, tv, q, q_indptr, q_pos, page_table, pt_stride,
                                                reinterpret_cast<const int4*>(tiles), out, Hq, Hkv, page_size, layer,
                                                scale * 1.4426950408889634f, err, nsplit, ws_o, ws_ml);
  if (cudaGetLastError() != cudaSuccess) return -5;
  if (nsplit > 1) return ll_attn_combine(out, ws_o, ws_ml, combine_rows, nsplit, stream);
  return 0;
}

// Selects the build (kVariants index) for later launches; -2 goes back to
// the default (LL_ATTN_VARIANT, else kDefaultVariant); any other negative or
// out-of-range index only queries.  Returns the number of builds.
extern "C" int ll_attn_prefill_tc_set_variant(int v) {
  if (v >= 0 && v < kNumVariants) g_attn_variant = v;
  if (v == -2) g_attn_variant = -1;
  return kNumVariants;
}

// Copies the clock64() trace of the last TRACE-variant launch (blocks x 12
// events) to host memory; returns the number of values copied.
extern "C" int ll_attn_prefill_tc_trace(unsigned long long* host, int n) {
  n = n < TC_TRACE_BLOCKS * TC_TRACE_EV ? n : TC_TRACE_BLOCKS * TC_TRACE_EV;
  if (cudaMemcpyFromSymbol(host, g_attn_trace, n * sizeof(unsigned long long)) != cudaSuccess) return -1;
  return n;
}

// Decode attention (split-KV partials or final rows); the caller launches the
// combine when nsplit > 1.  k_pool / v_pool: ONE layer's pool [pages, Hkv,
// page_size, 128].  page_size must divide 64 and be >= 4.
extern "C" int ll_attn_decode_tma(const bf16* q, const bf16* k_pool, const bf16* v_pool, int pages,
                                  const int* page_table, int pt_stride, const int* kv_lens, bf16* out, float* ws_o,
                                  float* ws_ml, int B, int Hq, int Hkv, int page_size, int nsplit, float scale_log2,
                                  int new_tokens, int* err, cudaStream_t stream) {
  if (page_size < 4 || DT_BN % page_size || Hq / Hkv > 16) return -3;
  CUtensorMap tk, tv, tkr, tvr;
  if (make_pool_map(&tk, k_pool, 1, pages, Hkv, page_size)) return -2;
  if (make_pool_map(&tv, v_pool, 1, pages, Hkv, page_size)) return -2;
  if (make_pool_run_map(&tkr, k_pool, 1, pages, Hkv, page_size, DT_BN / page_size)) return -2;
  if (make_pool_run_map(&tvr, v_pool, 1, pages, Hkv, page_size, DT_BN / page_size)) return -2;
  static int stages = -1;
  if (stages < 0) {
    const char* e = getenv("LL_DECODE_STAGES");
    stages = (e != nullptr && atoi(e) == 2) ? 2 : 3;
  }
  auto kern = stages == 2 ? attn_decode_tma_kernel<2> : attn_decode_tma_kernel<3>;
  const int smem = stages == 2 ? DT_SMEM2 : DT_SMEM;
  static int fits = -1;
  if (fits < 0) {
    int n = 0;
    fits = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess &&
                   cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, DT_THREADS, smem) == cudaSuccess && n >= 1
               ? 1
               : 0;
  }
  if (!fits) return -7;
  launch_pdl(kern, dim3(B * Hkv, nsplit), dim3(DT_THREADS), smem, stream, tk, tv, tkr, tvr, q, page_table, pt_stride,
             kv_lens, out, ws_o, ws_ml, Hq, Hkv, page_size, scale_log2, new_tokens, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}
