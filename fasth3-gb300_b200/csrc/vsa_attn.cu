// FP8 block-sparse VSA attention (fine step) for sm_100a: tcgen05 MMAs on E4M3 Q/K/V with TMEM accumulators, TMA
// staging, one persistent CTA per SM.
//
// Semantics (BASELINE config 4 and fastvideo/models/dits/h3fast/vsa_fp8.cuh:10-15, 716-764): for each (head, query
// tile) softmax attention of its rows over the keys of its selected 64-key tiles (keys past vbs[b] masked), scores
// scaled by sm_scale and the Q/K scales, fp32 online softmax, output bf16 heads-first [heads, rows_pad, 128], optional
// log2-domain LSE [heads, rows_pad]. P is stored as E4M3 with the V tile scale folded in: P' = 2^(x - m + 6) *
// (sv_b / sv_head) (<= 2^8 < 448 with the lazy-rescale bound of 2^2), and the row sum carries the same 2^6, so
// O = (sum P' V8) * sv_head / l. P' is split into two E4M3 terms, hi = e4m3(P') and lo = e4m3(P' - hi), both
// multiplied with V into the same accumulator: one E4M3 term alone leaves ~3% relative noise on O when V is noise-like
// (BASELINE config 4's N(0,1) data), two terms leave ~2^-8.
//
// Work item = (head, pair of query tiles t0 = 2p, t1 = 2p+1): the 128 query rows form one M=128 MMA operand, and the
// pair walks the ascending union of its two selection lists; a row whose tile did not select a key tile writes P = 0
// for it. CTA = 6 warps:
//   warp 0   builds the union list (bitmaps + warp prefix sums) and loads Q (per item) and K/V tiles (ring) by TMA
//   warp 1   TMEM allocation, MMA issue: S_j = Q K_j^T (4 x K32, into one of two S buffers), O += P_j V_j
//            (2 x K32 for each of the two P terms, P from TMEM, V as an MN-major operand), S one key tile ahead
//   warps 2-5 softmax (thread = query row, warp w owns TMEM lanes 32*(w%4)..), lazy O rescale, epilogue
// Every wait is bounded (2 s) and records H3B_ETIMEOUT in a device status word.
#include "common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

namespace h3b {

__device__ int g_attn_status = 0;

namespace {

using namespace sm100;

constexpr int D = 128;
constexpr int TILE = 64;
constexpr int KV_STAGES = 6;
constexpr int U_MAX = 4096;  // union entries per work item (a union of two subsets of n <= 4096 tiles)
constexpr float P_SHIFT = 6.f;
constexpr float RESCALE_LOG2 = 2.f;
constexpr uint64_t kLimitNs = 2000000000ull;
// TMEM columns
constexpr uint32_t COL_O = 0, COL_S = 128, COL_P = 256;  // P buffer b: hi at COL_P + 32b, lo at + 16

struct AttnArgs {
  const int32_t* idx;     // [heads, n_ext, n]
  const int32_t* num;     // [heads, n_ext]
  const int32_t* vbs;     // [n_ext]
  const float* qs;        // [heads, n_ext] per-tile Q scale, or NULL (scale folded in coef)
  const float* ks;        // [heads, n_ext] per-tile K scale, or NULL
  const float* vs;        // [heads, n_ext] per-tile V scale
  const float* vs_head;   // [heads]
  float coef;             // sm_scale * log2(e) (* static Q/K scales when qs/ks are NULL)
  bf16* out;              // [heads, rows_pad, 128]
  float* lse;             // [heads, rows_pad] or NULL
  int heads, n, n_ext;
  int64_t rows_pad;
  int items;
};

// ------------------------------------------------------------------------------------------------ shared storage
struct __align__(1024) Smem {
  uint8_t q[2][2 * TILE * D];        // two Q buffers of 128 rows x 128 B (1024-aligned, 128-byte swizzle)
  uint8_t kv[KV_STAGES][2][TILE * D];  // K tile, V tile
  uint32_t ulist[2][U_MAX];            // (tile | member bits << 16)
  uint32_t bm[2][128];                 // selection bitmaps of the two query tiles (n <= 4096)
  int ucount[2];
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
  uint64_t list_full[2], list_empty[2];
  uint64_t s_full[2], s_free[2], p_full[2];
  uint64_t pv_done, o_full, o_empty, drain;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// PV: O += P (TMEM, M=128 rows x K32 e4m3) * V (SMEM, MN-major)
__device__ __forceinline__ void mma_e4m3_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void tmem_st_16cols(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_32cols(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory descriptor of an MN-major operand tile: rows of 128 bytes along N, 128-byte swizzle, 8-row groups
// (8 K-steps) 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)2 << 61);
}

// kind::f8f6f4 e4m3 x e4m3 -> f32, M = 128, N = n; B major MN (bit 16) when b_mn.
__host__ __device__ constexpr uint32_t idesc_e4m3_mn(int n, bool b_mn) {
  return (1u << 4) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__global__ void __launch_bounds__(192, 1)
    vsa_fp8_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.q_full[i], 1);
      mbar_init(&sm.q_empty[i], 1);
      mbar_init(&sm.list_full[i], 1);
      mbar_init(&sm.list_empty[i], 5);  // the MMA thread + 4 softmax warps
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], 4);
      mbar_init(&sm.p_full[i], 4);
    }
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    mbar_init(&sm.pv_done, 1);
    mbar_init(&sm.o_full, 1);
    mbar_init(&sm.o_empty, 4);
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  auto fail = [&]() {
    *abort_flag = 1;
    atomicExch(&g_attn_status, H3B_ETIMEOUT);
  };
  const int pairs = a.n_ext / 2;

  if (warp == 0) {
    // -------------------------------------------------------------- union lists + TMA producer
    uint32_t list_phase[2] = {0, 0}, q_phase[2] = {0, 0};
    int stage = 0;
    uint32_t kv_phase = 0;
    bool ok = true;
    int it = 0;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
      const int buf = it & 1;
      const int h = item / pairs, p = item - h * pairs;
      const int t0 = 2 * p, t1 = 2 * p + 1;
      // wait until the consumers of this list buffer (two items ago) are done
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&sm.list_empty[buf], list_phase[buf] ^ 1, abort_flag, kLimitNs))) {
        if (lane == 0) fail();
        ok = false;
        break;
      }
      list_phase[buf] ^= 1;
      const int words = (a.n + 31) / 32;
      for (int w = lane; w < words; w += 32) {
        sm.bm[0][w] = 0u;
        sm.bm[1][w] = 0u;
      }
      __syncwarp();
      const int n0 = a.num[(size_t)h * a.n_ext + t0], n1 = a.num[(size_t)h * a.n_ext + t1];
      const int32_t* l0 = a.idx + ((size_t)h * a.n_ext + t0) * a.n;
      const int32_t* l1 = a.idx + ((size_t)h * a.n_ext + t1) * a.n;
      for (int i = lane; i < n0; i += 32) {
        const int b = l0[i];
        if (b >= 0 && b < a.n) atomicOr(&sm.bm[0][b >> 5], 1u << (b & 31));
      }
      for (int i = lane; i < n1; i += 32) {
        const int b = l1[i];
        if (b >= 0 && b < a.n) atomicOr(&sm.bm[1][b >> 5], 1u << (b & 31));
      }
      __syncwarp();
      // ascending union: word-level exclusive prefix of popcounts across the warp
      int base = 0;
      for (int w0 = 0; w0 < words; w0 += 32) {
        const int w = w0 + lane;
        const uint32_t b0 = w < words ? sm.bm[0][w] : 0u, b1 = w < words ? sm.bm[1][w] : 0u;
        uint32_t u = b0 | b1;
        const int c = __popc(u);
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        int pos = base + incl - c;
        while (u) {
          const int bit = __ffs(u) - 1;
          u &= u - 1;
          const uint32_t m = ((b0 >> bit) & 1u) | (((b1 >> bit) & 1u) << 1);
          if (pos < U_MAX) sm.ulist[buf][pos] = (uint32_t)(w * 32 + bit) | (m << 16);
          ++pos;
        }
        base += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) {
        sm.ucount[buf] = base < U_MAX ? base : U_MAX;
        mbar_arrive(&sm.list_full[buf]);
      }
      __syncwarp();
      const int U = base < U_MAX ? base : U_MAX;
      if (lane == 0) {
        // Q pair
        if (!mbar_wait_bounded(&sm.q_empty[buf], q_phase[buf] ^ 1, abort_flag, kLimitNs)) {
          fail();
          ok = false;
        } else {
          q_phase[buf] ^= 1;
          mbar_arrive_expect_tx(&sm.q_full[buf], 2 * TILE * D);
          tma_load_3d(&sm.q[buf][0], &tmQ, 0, t0 * TILE, h, &sm.q_full[buf]);
          tma_load_3d(&sm.q[buf][TILE * D], &tmQ, 0, t1 * TILE, h, &sm.q_full[buf]);
          for (int j = 0; j < U && ok; ++j) {
            const int b = (int)(sm.ulist[buf][j] & 0xFFFFu);
            if (!mbar_wait_bounded(&sm.kv_empty[stage], kv_phase ^ 1, abort_flag, kLimitNs)) {
              fail();
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&sm.kv_full[stage], 2 * TILE * D);
            tma_load_3d(&sm.kv[stage][0][0], &tmK, 0, b * TILE, h, &sm.kv_full[stage]);
            tma_load_3d(&sm.kv[stage][1][0], &tmV, 0, b * TILE, h, &sm.kv_full[stage]);
            if (++stage == KV_STAGES) {
              stage = 0;
              kv_phase ^= 1;
            }
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = idesc_e4m3_mn(TILE, false);
      const uint32_t idesc_pv = idesc_e4m3_mn(D, true);
      uint32_t list_phase[2] = {0, 0}, q_phase[2] = {0, 0}, s_phase[2] = {0, 0}, p_phase[2] = {0, 0};
      uint32_t o_phase = 0;
      int stage = 0;
      uint32_t kv_phase = 0;
      int sbuf_next = 0;  // S buffer of the next S MMA
      int pbuf = 0;       // P buffer of the next PV (persists across items, like the softmax side)
      bool ok = true;
      int it = 0;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
        const int buf = it & 1;
        if (!mbar_wait_bounded(&sm.list_full[buf], list_phase[buf], abort_flag, kLimitNs)) { fail(); break; }
        list_phase[buf] ^= 1;
        const int U = sm.ucount[buf];
        if (!mbar_wait_bounded(&sm.q_full[buf], q_phase[buf], abort_flag, kLimitNs)) { fail(); break; }
        q_phase[buf] ^= 1;
        tc_fence_after();
        const uint64_t dq = desc_k_sw128(smem_addr(&sm.q[buf][0]));
        // S_j for j = 0 .. U-1 issued one ahead of PV_j; K/V stage of tile j is stage0 + j (mod ring)
        int s_stage = stage;
        uint32_t s_kvphase = kv_phase;
        auto issue_s = [&](int j) -> bool {
          const int sb = sbuf_next;
          if (!mbar_wait_bounded(&sm.kv_full[s_stage], s_kvphase, abort_flag, kLimitNs)) return false;
          if (!mbar_wait_bounded(&sm.s_free[sb], s_phase[sb] ^ 1, abort_flag, kLimitNs)) return false;
          s_phase[sb] ^= 1;
          tc_fence_after();
          const uint64_t dk = desc_k_sw128(smem_addr(&sm.kv[s_stage][0][0]));
#pragma unroll
          for (int i = 0; i < 4; ++i) mma_e4m3(tmem + COL_S + sb * TILE, dq + 2 * i, dk + 2 * i, idesc_s, i != 0);
          tc_commit(&sm.s_full[sb]);
          sbuf_next ^= 1;
          if (++s_stage == KV_STAGES) {
            s_stage = 0;
            s_kvphase ^= 1;
          }
          (void)j;
          return true;
        };
        if (U > 0 && !issue_s(0)) { fail(); break; }
        for (int j = 0; j < U; ++j) {
          if (j + 1 < U && !issue_s(j + 1)) { fail(); ok = false; break; }
          if (j == U - 1) tc_commit(&sm.q_empty[buf]);  // last S of the item has been issued: Q buffer reusable
          if (j == 0) {  // O is about to be overwritten: the previous item's epilogue must have read it
            if (!mbar_wait_bounded(&sm.o_empty, o_phase ^ 1, abort_flag, kLimitNs)) { fail(); ok = false; break; }
            o_phase ^= 1;
          }
          if (!mbar_wait_bounded(&sm.p_full[pbuf], p_phase[pbuf], abort_flag, kLimitNs)) { fail(); ok = false; break; }
          p_phase[pbuf] ^= 1;
          tc_fence_after();
          const uint64_t dv = desc_mn_sw128(smem_addr(&sm.kv[stage][1][0]));
#pragma unroll
          for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int i = 0; i < 2; ++i)
              mma_e4m3_ts(tmem + COL_O, tmem + COL_P + pbuf * 32 + t * 16 + 8 * i,
                          dv + (uint64_t)((i * 32 * D) >> 4), idesc_pv, (j | i | t) != 0);
          tc_commit(&sm.kv_empty[stage]);
          tc_commit(&sm.pv_done);
          pbuf ^= 1;
          if (++stage == KV_STAGES) {
            stage = 0;
            kv_phase ^= 1;
          }
        }
        if (!ok) break;
        if (U == 0) {
          tc_commit(&sm.q_empty[buf]);
          if (!mbar_wait_bounded(&sm.o_empty, o_phase ^ 1, abort_flag, kLimitNs)) { fail(); break; }
          o_phase ^= 1;
        }
        tc_commit(&sm.o_full);
        mbar_arrive(&sm.list_empty[buf]);
      }
      tc_commit(&sm.drain);
      volatile int no_abort = 0;
      if (!mbar_wait_bounded(&sm.drain, 0, &no_abort, kLimitNs)) fail();
    }
  } else {
    // -------------------------------------------------------------- softmax + epilogue
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // query row of the pair: 0-63 tile t0, 64-127 tile t1
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t my_bit = r < TILE ? 1u : 2u;
    uint32_t list_phase[2] = {0, 0}, s_phase[2] = {0, 0};
    uint32_t o_phase = 0;
    uint32_t pv_count = 0;  // PV commits seen by this CTA so far (pv_done phase bookkeeping)
    int sbuf = 0, pbuf_g = 0;
    int it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
      const int buf = it & 1;
      const int h = item / pairs, p = item - h * pairs;
      const int tq = r < TILE ? 2 * p : 2 * p + 1;
      const int rr = r & (TILE - 1);
      bool got = mbar_wait_bounded(&sm.list_full[buf], list_phase[buf], abort_flag, kLimitNs);
      if (!__all_sync(0xffffffffu, got)) { if (lane == 0) fail(); ok = false; break; }
      list_phase[buf] ^= 1;
      const int U = sm.ucount[buf];
      const float qscale = a.qs ? a.qs[(size_t)h * a.n_ext + tq] : 1.f;
      const float vhead = a.vs_head[h];
      const float inv_vhead = 1.f / vhead;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < U; ++j) {
        const uint32_t e = sm.ulist[buf][j];
        const int b = (int)(e & 0xFFFFu);
        const bool member = (e >> 16) & my_bit;
        got = mbar_wait_bounded(&sm.s_full[sbuf], s_phase[sbuf], abort_flag, kLimitNs);
        if (!__all_sync(0xffffffffu, got)) { if (lane == 0) fail(); ok = false; break; }
        s_phase[sbuf] ^= 1;
        __syncwarp();
        tc_fence_after();
        uint32_t sr[2][32];
        tmem_ld_32cols(tmem + lane_off + COL_S + sbuf * TILE, sr[0]);
        tmem_ld_32cols(tmem + lane_off + COL_S + sbuf * TILE + 32, sr[1]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_free[sbuf]);
        sbuf ^= 1;
        const int kv_valid = a.vbs[b];
        const float coef = a.coef * qscale * (a.ks ? a.ks[(size_t)h * a.n_ext + b] : 1.f);
        const float vratio = a.vs[(size_t)h * a.n_ext + b] * inv_vhead;
        float x[64];
        float m8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) m8[u] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float s = __uint_as_float(sr[c >> 5][c & 31]) * coef;
          x[c] = (member && c < kv_valid) ? s : -INFINITY;
          m8[c & 7] = fmaxf(m8[c & 7], x[c]);  // eight independent chains: one warp per sub-partition hides little latency
        }
        const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        // lazy rescale: move the reference max only when the row max grows by more than 2^RESCALE_LOG2
        const bool grow = member && mx > m_ref + RESCALE_LOG2;
        const bool need_o = grow && l > 0.f;
        float alpha = 1.f;
        if (grow) {
          alpha = l > 0.f ? ex2(m_ref - mx) : 1.f;
          m_ref = mx;
        }
        if (__any_sync(0xffffffffu, need_o)) {
          // O must hold every PV issued before this tile: wait for PV_{j-1}
          if (j > 0) {
            got = mbar_wait_bounded(&sm.pv_done, (pv_count - 1) & 1, abort_flag, kLimitNs);
            if (!__all_sync(0xffffffffu, got)) { if (lane == 0) fail(); ok = false; break; }
          }
          tc_fence_after();
#pragma unroll 1
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t o[32];
            tmem_ld_32cols(tmem + lane_off + COL_O + c0, o);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st_32cols(tmem + lane_off + COL_O + c0, o);
          }
          tmem_st_wait();
        }
        l *= alpha;
        const float base = P_SHIFT - m_ref;
        uint32_t pw[16], pl[16];
        float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          float ev[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            ev[u] = x[c + u] == -INFINITY ? 0.f : ex2(x[c + u] + base);
            l4[u] += ev[u];
            ev[u] *= vratio;
          }
          const uint32_t hi = e4m3x4(ev[0], ev[1], ev[2], ev[3]);
          pw[c >> 2] = hi;
          pl[c >> 2] = e4m3x4(ev[0] - e4m3_to_float(hi & 0xFFu), ev[1] - e4m3_to_float((hi >> 8) & 0xFFu),
                              ev[2] - e4m3_to_float((hi >> 16) & 0xFFu), ev[3] - e4m3_to_float(hi >> 24));
        }
        l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
        tmem_st_16cols(tmem + lane_off + COL_P + pbuf_g * 32, pw);
        tmem_st_16cols(tmem + lane_off + COL_P + pbuf_g * 32 + 16, pl);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[pbuf_g]);
        pbuf_g ^= 1;
        ++pv_count;
      }
      if (!ok) break;
      // epilogue: O * sv_head / l -> bf16 rows; the list buffer is released once every tile was consumed
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.list_empty[buf]);
      got = mbar_wait_bounded(&sm.o_full, o_phase, abort_flag, kLimitNs);
      if (!__all_sync(0xffffffffu, got)) { if (lane == 0) fail(); ok = false; break; }
      o_phase ^= 1;
      __syncwarp();
      tc_fence_after();
      const float oscale = l > 0.f ? vhead / l : 0.f;
      const bool row_ok = rr < a.vbs[tq];
      bf16* dst = a.out + ((size_t)h * a.rows_pad + (size_t)tq * TILE + rr) * D;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t o[32];
        tmem_ld_32cols(tmem + lane_off + COL_O + c0, o);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float f[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) f[u] = l > 0.f ? __uint_as_float(o[c + u]) * oscale : 0.f;
            store8(dst + c0 + c, f);
          }
        }
      }
      if (a.lse && row_ok)
        a.lse[(size_t)h * a.rows_pad + (size_t)tq * TILE + rr] = l > 0.f ? m_ref + __log2f(l) - P_SHIFT : -INFINITY;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.o_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// [heads, rows_pad, 128] e4m3 as a 3D tensor map with a {128 B, 64 rows, 1 head} box, 128-byte swizzle
int make_map(CUtensorMap* m, const void* base, int heads, int64_t rows_pad) {
  auto fn = encode_fn();
  if (!fn) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows_pad, (cuuint64_t)heads};
  cuuint64_t strides[2] = {(cuuint64_t)D, (cuuint64_t)rows_pad * D};
  cuuint32_t box[3] = {(cuuint32_t)D, (cuuint32_t)TILE, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return H3B_OK;
}

}  // namespace
}  // namespace h3b

using namespace h3b;

extern "C" int h3b_vsa_fp8(const void* qb, const void* kb, const void* vb, const int32_t* idx, const int32_t* num,
                           const int32_t* vbs, const float* qs_blk, const float* ks_blk, const float* vs_blk,
                           const float* vs_head, float qk_coef, void* out, float* lse, int heads, int n, int n_ext,
                           int64_t rows_pad, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(qb && kb && vb && idx && num && vbs && vs_blk && vs_head && out, "vsa_fp8: null pointer");
  H3B_REQUIRE((qs_blk == nullptr) == (ks_blk == nullptr), "vsa_fp8: give both or neither per-tile Q/K scales");
  H3B_REQUIRE(heads > 0 && n > 0 && n_ext >= n && n_ext % 2 == 0 && n <= 4096,
              "vsa_fp8: need n_ext even, n_ext >= n, n <= 4096 tiles");
  H3B_REQUIRE(rows_pad == (int64_t)n_ext * TILE, "vsa_fp8: rows_pad must equal n_ext * 64");
  H3B_REQUIRE(aligned(qb, 16) && aligned(kb, 16) && aligned(vb, 16) && aligned(out, 16),
              "vsa_fp8: 16-byte aligned operands");
  CUtensorMap mq, mk, mv;
  if (int rc = make_map(&mq, qb, heads, rows_pad)) return rc;
  if (int rc = make_map(&mk, kb, heads, rows_pad)) return rc;
  if (int rc = make_map(&mv, vb, heads, rows_pad)) return rc;
  AttnArgs a{idx, num, vbs, qs_blk, ks_blk, vs_blk, vs_head, qk_coef, static_cast<bf16*>(out), lse, heads, n, n_ext,
             rows_pad, heads * (n_ext / 2)};
  const int smem = (int)sizeof(Smem) + 1024;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(vsa_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return set_error(H3B_ECUDA, "vsa_fp8: cannot reserve %d bytes of shared memory", smem);
    attr = true;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = a.items < sms ? a.items : sms;
  vsa_fp8_kernel<<<grid, 192, smem, stream>>>(mq, mk, mv, a);
  H3B_LAUNCH_CHECK("vsa_fp8");
  return H3B_OK;
}

extern "C" int h3b_vsa_status(int* status, int reset) {
  clear_error();
  H3B_REQUIRE(status, "vsa_status: null pointer");
  if (cudaMemcpyFromSymbol(status, g_attn_status, sizeof(int)) != cudaSuccess)
    return set_error(H3B_ECUDA, "vsa_status: read failed");
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int)) != cudaSuccess)
      return set_error(H3B_ECUDA, "vsa_status: reset failed");
  }
  return H3B_OK;
}
