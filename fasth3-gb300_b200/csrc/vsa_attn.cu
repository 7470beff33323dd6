// FP8 block-sparse VSA attention (fine step) for sm_100a: tcgen05 MMAs with TMEM accumulators, TMA staging, one
// persistent CTA per SM.
//
// Semantics (BASELINE config 4 and fastvideo/models/dits/h3fast/vsa_fp8.cuh:10-15, 716-764): for each (head, query
// tile) softmax attention of its rows over the keys of its selected 64-key tiles (keys past vbs_kv[b] masked), scores
// scaled by the softmax scale and the Q/K scales, fp32 online softmax with a lazy rescale (the running maximum moves
// only when a tile's maximum exceeds it by more than 2^4), bf16 output, optional log2-domain LSE.
//
// Arithmetic: S = Q8 K8^T on E4M3 operands (kind::f8f6f4). P = 2^(S*coef - m) is evaluated in f16x2 (one
// ex2.approx.f16x2 per two keys; the exponent argument is at most 4 in magnitude for every key that matters, where f16
// resolves it to 2^-9) and multiplied with V in f16 (kind::f16). V is stored E4M3 with one scale per (head, tile); each
// V tile is converted once per use into f16 in shared memory with the tile's scale ratio sv_b / sv_head folded in, so
// O = (sum P V') * sv_head / l and the row sum l = sum P needs no per-tile correction. The conversion is shared by the
// 128 query rows of a work item. (The reference's kernel quantizes P to E4M3 instead; f16 P keeps the attention
// output within ~2^-9 of exact attention over the same E4M3 Q/K/V.)
//
// Operand layout: Q/out and K/V are each [chunks * heads, rows_chunk, 128] ("planes" of rows_chunk rows). Query tile t
// of head h lives in plane (t / tiles_per_chunk) * heads + h at row (t % tiles_per_chunk) * 64. With one chunk this is
// the plain heads-first [heads, rows, 128] layout; with P chunks it is exactly what an all-to-all over P ranks
// delivers ([source rank][local head][rows]), so sequence-parallel callers attend in place without a permute copy.
// K/V may be a different tensor with its own tile count (cross-attention to text tokens).
//
// Work item = (head, pair of query tiles t0 = 2p, t1 = 2p+1): the 128 query rows form one M=128 MMA operand and the
// pair walks the ascending union of its two selection lists; a row whose tile did not select a key tile gets P = 0
// there. CTA = 10 warps:
//   warp 0     union list (bitmaps + warp prefix sums); TMA loads of the Q pair (per item) and K/V tiles (ring)
//   warp 1     TMEM allocation, MMA issue: S_j = Q K_j^T (E4M3, 4 x K32, two S buffers, one key tile ahead of PV),
//              O += P_j V'_j (f16, 4 x K16, P from TMEM, V' from shared memory as an MN-major operand)
//   warps 2-5  V converters: E4M3 V tile -> f16 V' (scale ratio folded in), 128-byte-swizzled MN-major layout
//   warps 6-9  softmax + epilogue: one query row per thread (TMEM lane), the 64 scores of a key tile in registers
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
constexpr int KV_STAGES = 4;  // E4M3 K/V tiles
constexpr int VF_STAGES = 3;  // f16 V' tiles
constexpr int N_MAX = 4096;   // key tiles (bitmap words: 128)
constexpr int U_MAX = N_MAX;  // the union of two subsets of N_MAX tiles
constexpr int CONV_WARPS = 4;
constexpr int SOFT_WARPS = 4;
constexpr int THREADS = (2 + CONV_WARPS + SOFT_WARPS) * 32;
constexpr float RESCALE_LOG2 = 4.f;
constexpr uint64_t kLimitNs = 2000000000ull;
// TMEM columns: O [0,128), S buffers [128,192) [192,256), P buffers (f16, 64 keys = 32 columns) [256,288) [288,320)
constexpr uint32_t COL_O = 0, COL_S = 128, COL_P = 256;

struct AttnArgs {
  const int32_t* idx;
  const int32_t* num;
  const int32_t* vbs_q;
  const int32_t* vbs_kv;
  const float* qs;
  const float* ks;
  const float* vs;
  const float* vs_head;
  float coef;
  bf16* out;
  float* lse;
  int heads, n_q_ext, n_kv;
  int idx_ld, q_scale_ld, kv_scale_ld;
  int tpc_q, tpc_kv;  // tiles per chunk
  int64_t rows_chunk_q;
  int items;
};

struct __align__(1024) Smem {
  uint8_t q[2][2 * TILE * D];
  uint8_t kv[KV_STAGES][2][TILE * D];
  uint8_t vf[VF_STAGES][2][TILE * 128];  // [half of d][key][64 d] f16, 128-byte rows, 128-byte swizzle
  uint32_t ulist[2][U_MAX];
  uint32_t bm[2][N_MAX / 32];
  int ucount[2];
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
  uint64_t vf_full[VF_STAGES], vf_empty[VF_STAGES];
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

__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                           uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
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

// 2^x for two keys: x0 (low half) and x1 rounded to f16, exponentiated in f16x2
__device__ __forceinline__ uint32_t ex2_f16x2(float x0, float x1) {
  uint32_t h, e;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(x1), "f"(x0));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(e) : "r"(h));
  return e;
}

__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// two E4M3 bytes (low byte first) -> f16x2 scaled by an f16x2 factor
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2_scaled(uint16_t v, uint32_t scale2) {
  uint32_t h, d;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(v));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(h), "r"(scale2));
  return d;
}

// K-major e4m3 tiles use desc_k_sw128; V' is MN-major: 64 f16 of d (128 bytes) per row, rows = keys, 8-row groups
// 1024 bytes apart (SBO), the two 64-column halves of d `lbo` bytes apart (LBO), 128-byte swizzle.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// fp32 accumulate, A and B of the same 8/16-bit type (E4M3 under kind::f8f6f4, f16 under kind::f16), A K-major,
// B K-major or MN-major, M = 128
__host__ __device__ constexpr uint32_t idesc_mn(int n, bool b_mn) {
  return (1u << 4) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void fail_cta(volatile int* abort_flag) {
  *abort_flag = 1;
  atomicExch(&g_attn_status, H3B_ETIMEOUT);
}

// a wait every lane of the warp takes; false (and the CTA marked aborted) if it gave up
__device__ __forceinline__ bool warp_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int lane) {
  const bool got = mbar_wait_bounded(bar, parity, abort_flag, kLimitNs);
  if (__all_sync(0xffffffffu, got)) return true;
  if (lane == 0) fail_cta(abort_flag);
  return false;
}

__global__ void __launch_bounds__(THREADS, 1)
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
      mbar_init(&sm.list_empty[i], 1 + CONV_WARPS + SOFT_WARPS);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], SOFT_WARPS);
      mbar_init(&sm.p_full[i], SOFT_WARPS);
    }
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1 + CONV_WARPS);  // K read by the S MMA, V read by the converters
    }
    for (int s = 0; s < VF_STAGES; ++s) {
      mbar_init(&sm.vf_full[s], CONV_WARPS);
      mbar_init(&sm.vf_empty[s], 1);
    }
    mbar_init(&sm.pv_done, 1);
    mbar_init(&sm.o_full, 1);
    mbar_init(&sm.o_empty, SOFT_WARPS);
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
#define fail() fail_cta(abort_flag)
#define warp_wait(bar, parity) warp_wait_bounded((bar), (parity), abort_flag, lane)
  const int pairs = a.n_q_ext / 2;

  if (warp == 0) {
    // -------------------------------------------------------------- union lists + TMA producer
    uint32_t list_phase = 0, q_phase = 0;
    int stage = 0;
    uint32_t kv_phase = 0;
    bool ok = true;
    int it = 0;
    const int words = (a.n_kv + 31) / 32;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
      const int buf = it & 1;
      const int h = item / pairs, p = item - h * pairs;
      const int t0 = 2 * p, t1 = 2 * p + 1;
      if (!warp_wait(&sm.list_empty[buf], (((list_phase >> buf) & 1u) ^ 1u))) break;
      list_phase ^= 1u << buf;
      for (int w = lane; w < words; w += 32) {
        sm.bm[0][w] = 0u;
        sm.bm[1][w] = 0u;
      }
      __syncwarp();
      const int n0 = a.num[(size_t)h * a.n_q_ext + t0], n1 = a.num[(size_t)h * a.n_q_ext + t1];
      const int32_t* l0 = a.idx + ((size_t)h * a.n_q_ext + t0) * a.idx_ld;
      const int32_t* l1 = a.idx + ((size_t)h * a.n_q_ext + t1) * a.idx_ld;
      for (int i = lane; i < n0 && i < a.idx_ld; i += 32) {
        const int b = l0[i];
        if (b >= 0 && b < a.n_kv) atomicOr(&sm.bm[0][b >> 5], 1u << (b & 31));
      }
      for (int i = lane; i < n1 && i < a.idx_ld; i += 32) {
        const int b = l1[i];
        if (b >= 0 && b < a.n_kv) atomicOr(&sm.bm[1][b >> 5], 1u << (b & 31));
      }
      __syncwarp();
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
          sm.ulist[buf][pos++] = (uint32_t)(w * 32 + bit) | (m << 16);
        }
        base += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) {
        sm.ucount[buf] = base;
        mbar_arrive(&sm.list_full[buf]);
      }
      __syncwarp();
      const int U = base;
      if (lane == 0) {
        if (!mbar_wait_bounded(&sm.q_empty[buf], (((q_phase >> buf) & 1u) ^ 1u), abort_flag, kLimitNs)) {
          fail();
          ok = false;
        } else {
          q_phase ^= 1u << buf;
          mbar_arrive_expect_tx(&sm.q_full[buf], 2 * TILE * D);
          for (int s = 0; s < 2; ++s) {
            const int t = s ? t1 : t0;
            tma_load_3d(&sm.q[buf][s * TILE * D], &tmQ, 0, (t % a.tpc_q) * TILE, (t / a.tpc_q) * a.heads + h,
                        &sm.q_full[buf]);
          }
          for (int j = 0; j < U && ok; ++j) {
            const int b = (int)(sm.ulist[buf][j] & 0xFFFFu);
            if (!mbar_wait_bounded(&sm.kv_empty[stage], kv_phase ^ 1, abort_flag, kLimitNs)) {
              fail();
              ok = false;
              break;
            }
            const int y = (b % a.tpc_kv) * TILE, z = (b / a.tpc_kv) * a.heads + h;
            mbar_arrive_expect_tx(&sm.kv_full[stage], 2 * TILE * D);
            tma_load_3d(&sm.kv[stage][0][0], &tmK, 0, y, z, &sm.kv_full[stage]);
            tma_load_3d(&sm.kv[stage][1][0], &tmV, 0, y, z, &sm.kv_full[stage]);
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
      const uint32_t idesc_s = idesc_mn(TILE, false);
      const uint32_t idesc_pv = idesc_mn(D, true);
      uint32_t list_phase = 0, q_phase = 0, s_phase = 0, p_phase = 0;
      uint32_t o_phase = 0;
      int s_stage = 0, vstage = 0;
      uint32_t s_kvphase = 0, vf_phase = 0;
      int sbuf_next = 0, pbuf = 0;
      bool ok = true;
      int it = 0;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
        const int buf = it & 1;
        if (!mbar_wait_bounded(&sm.list_full[buf], ((list_phase >> buf) & 1u), abort_flag, kLimitNs)) { fail(); break; }
        list_phase ^= 1u << buf;
        const int U = sm.ucount[buf];
        if (!mbar_wait_bounded(&sm.q_full[buf], ((q_phase >> buf) & 1u), abort_flag, kLimitNs)) { fail(); break; }
        q_phase ^= 1u << buf;
        tc_fence_after();
        const uint64_t dq = desc_k_sw128(smem_addr(&sm.q[buf][0]));
        // j = -1 issues S(0) only; step j issues S(j+1) (one key tile ahead) and then PV(j)
        for (int j = -1; j < U; ++j) {
          if (j + 1 < U) {
            const int sb = sbuf_next;
            if (!mbar_wait_bounded(&sm.kv_full[s_stage], s_kvphase, abort_flag, kLimitNs) ||
                !mbar_wait_bounded(&sm.s_free[sb], (((s_phase >> sb) & 1u) ^ 1u), abort_flag, kLimitNs)) {
              fail();
              ok = false;
              break;
            }
            s_phase ^= 1u << sb;
            tc_fence_after();
            const uint64_t dk = desc_k_sw128(smem_addr(&sm.kv[s_stage][0][0]));
#pragma unroll
            for (int i = 0; i < 4; ++i) mma_e4m3(tmem + COL_S + sb * TILE, dq + 2 * i, dk + 2 * i, idesc_s, i != 0);
            tc_commit(&sm.s_full[sb]);
            tc_commit(&sm.kv_empty[s_stage]);  // the K half of the stage is consumed
            sbuf_next ^= 1;
            if (++s_stage == KV_STAGES) {
              s_stage = 0;
              s_kvphase ^= 1;
            }
          }
          if (j < 0) continue;
          if (j == U - 1) tc_commit(&sm.q_empty[buf]);
          if (j == 0) {
            if (!mbar_wait_bounded(&sm.o_empty, o_phase ^ 1, abort_flag, kLimitNs)) { fail(); ok = false; break; }
            o_phase ^= 1;
          }
          if (!mbar_wait_bounded(&sm.p_full[pbuf], ((p_phase >> pbuf) & 1u), abort_flag, kLimitNs)) { fail(); ok = false; break; }
          p_phase ^= 1u << pbuf;
          if (!mbar_wait_bounded(&sm.vf_full[vstage], vf_phase, abort_flag, kLimitNs)) { fail(); ok = false; break; }
          tc_fence_after();
          const uint64_t dv = desc_mn_sw128(smem_addr(&sm.vf[vstage][0][0]), TILE * 128);
#pragma unroll
          for (int i = 0; i < 4; ++i)  // K = 16 keys per MMA: 8 TMEM columns of P, 16 rows (2048 bytes) of V'
            mma_f16_ts(tmem + COL_O, tmem + COL_P + pbuf * 32 + 8 * i, dv + (uint64_t)((i * 16 * 128) >> 4),
                       idesc_pv, (j | i) != 0);
          tc_commit(&sm.vf_empty[vstage]);
          tc_commit(&sm.pv_done);
          pbuf ^= 1;
          if (++vstage == VF_STAGES) {
            vstage = 0;
            vf_phase ^= 1;
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
  } else if (warp < 2 + CONV_WARPS) {
    // -------------------------------------------------------------- V converters: E4M3 -> f16 V' = v * sv_b/sv_head
    const int ct = (warp - 2) * 32 + lane;
    uint32_t list_phase = 0;
    int stage = 0, vstage = 0;
    uint32_t kv_phase = 0, vf_phase = 0;
    bool ok = true;
    int it = 0;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
      const int buf = it & 1;
      const int h = item / pairs;
      if (!warp_wait(&sm.list_full[buf], ((list_phase >> buf) & 1u))) break;
      list_phase ^= 1u << buf;
      const int U = sm.ucount[buf];
      const float inv_vhead = 1.f / a.vs_head[h];
      float vs_next = U > 0 ? a.vs[(size_t)h * a.kv_scale_ld + (sm.ulist[buf][0] & 0xFFFFu)] : 0.f;
      for (int j = 0; j < U; ++j) {
        const __half2 r2 = __float2half2_rn(vs_next * inv_vhead);
        const uint32_t scale2 = *reinterpret_cast<const uint32_t*>(&r2);
        if (j + 1 < U) vs_next = a.vs[(size_t)h * a.kv_scale_ld + (sm.ulist[buf][j + 1] & 0xFFFFu)];
        if (!warp_wait(&sm.kv_full[stage], kv_phase)) { ok = false; break; }
        if (!warp_wait(&sm.vf_empty[vstage], vf_phase ^ 1)) { ok = false; break; }
        const uint8_t* src = &sm.kv[stage][1][0];
        uint8_t* dst = &sm.vf[vstage][0][0];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int u = ct + 128 * i;
          const int key = u >> 3, c = u & 7;  // 16 E4M3 values: d = 16c .. 16c+15
          const uint4 raw = *reinterpret_cast<const uint4*>(src + key * 128 + ((c ^ (key & 7)) << 4));
          const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
          uint32_t f[8];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            f[2 * q] = e4m3x2_to_f16x2_scaled((uint16_t)(w[q] & 0xFFFFu), scale2);
            f[2 * q + 1] = e4m3x2_to_f16x2_scaled((uint16_t)(w[q] >> 16), scale2);
          }
          uint8_t* half_base = dst + (c >> 2) * (TILE * 128) + key * 128;
          const int dc0 = (c & 3) * 2;
          *reinterpret_cast<uint4*>(half_base + ((dc0 ^ (key & 7)) << 4)) = make_uint4(f[0], f[1], f[2], f[3]);
          *reinterpret_cast<uint4*>(half_base + (((dc0 + 1) ^ (key & 7)) << 4)) = make_uint4(f[4], f[5], f[6], f[7]);
        }
        fence_proxy_async_smem();  // the generic-proxy stores become visible to the tensor core
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.vf_full[vstage]);
          mbar_arrive(&sm.kv_empty[stage]);
        }
        if (++stage == KV_STAGES) {
          stage = 0;
          kv_phase ^= 1;
        }
        if (++vstage == VF_STAGES) {
          vstage = 0;
          vf_phase ^= 1;
        }
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.list_empty[buf]);
    }
  } else {
    // -------------------------------------------------------------- softmax + epilogue (warps 6..9)
    const int q4 = warp & 3;       // a warp reaches only the TMEM lanes 32*(warp%4) .. +31
    const int r = q4 * 32 + lane;  // query row of the item = TMEM lane
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t my_bit = r < TILE ? 1u : 2u;  // warp-uniform
    uint32_t list_phase = 0, s_phase = 0;
    uint32_t o_phase = 0;
    uint32_t pv_count = 0;
    int sbuf = 0, pbuf = 0;
    int it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
      const int buf = it & 1;
      const int h = item / pairs, p = item - h * pairs;
      const int tq = r < TILE ? 2 * p : 2 * p + 1;
      const int rr = r & (TILE - 1);
      if (!warp_wait(&sm.list_full[buf], ((list_phase >> buf) & 1u))) break;
      list_phase ^= 1u << buf;
      const int U = sm.ucount[buf];
      const float qcoef = a.coef * (a.qs ? a.qs[(size_t)h * a.q_scale_ld + tq] : 1.f);
      float m_ref = -INFINITY, l = 0.f;
      // per-tile scalars of key tile j+1 are loaded while tile j is processed (global loads off the critical path)
      int vbs_next = 0;
      float ks_next = 1.f;
      if (U > 0) {
        const int b0 = (int)(sm.ulist[buf][0] & 0xFFFFu);
        vbs_next = a.vbs_kv[b0];
        if (a.ks) ks_next = a.ks[(size_t)h * a.kv_scale_ld + b0];
      }
      for (int j = 0; j < U; ++j) {
        const uint32_t e = sm.ulist[buf][j];
        const bool member = (e >> 16) & my_bit;
        const int vbs_j = vbs_next;
        const float ks_j = ks_next;
        if (j + 1 < U) {
          const int bn = (int)(sm.ulist[buf][j + 1] & 0xFFFFu);
          vbs_next = a.vbs_kv[bn];
          if (a.ks) ks_next = a.ks[(size_t)h * a.kv_scale_ld + bn];
        }
        if (!warp_wait(&sm.s_full[sbuf], ((s_phase >> sbuf) & 1u))) { ok = false; break; }
        s_phase ^= 1u << sbuf;
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld_32cols(tmem + lane_off + COL_S + sbuf * TILE, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tmem_ld_32cols(tmem + lane_off + COL_S + sbuf * TILE + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_free[sbuf]);
        sbuf ^= 1;
        const int kv_valid = member ? vbs_j : 0;
        if (kv_valid < TILE) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= kv_valid) sr[c] = __float_as_uint(-INFINITY);
        }
        const float coef = qcoef * ks_j;
        float m8[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) m8[c] = __uint_as_float(sr[c]);
#pragma unroll
        for (int c = 8; c < 64; ++c) m8[c & 7] = fmaxf(m8[c & 7], __uint_as_float(sr[c]));
        const float mraw = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                 fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        const float mx = mraw * coef;  // coef > 0
        // lazy rescale: the running maximum moves only when this tile's maximum exceeds it by more than 2^4
        const bool grow = mx > m_ref + RESCALE_LOG2;
        const bool had_mass = m_ref != -INFINITY;
        float alpha = 1.f;
        if (grow) {
          alpha = had_mass ? ex2(m_ref - mx) : 1.f;
          m_ref = mx;
        }
        if (__any_sync(0xffffffffu, grow && had_mass)) {
          if (j > 0 && !warp_wait(&sm.pv_done, (pv_count - 1) & 1)) { ok = false; break; }
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
        uint32_t pw[32];
        if (m_ref == -INFINITY) {
#pragma unroll
          for (int c = 0; c < 32; ++c) pw[c] = 0u;
        } else {
          const float nb = -m_ref;
          uint32_t acc[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            pw[c] = ex2_f16x2(fmaf(__uint_as_float(sr[2 * c]), coef, nb),
                              fmaf(__uint_as_float(sr[2 * c + 1]), coef, nb));
            acc[c & 3] = hadd2(acc[c & 3], pw[c]);
          }
          const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&acc[0]));
          const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&acc[1]));
          const float2 s2 = __half22float2(*reinterpret_cast<const __half2*>(&acc[2]));
          const float2 s3 = __half22float2(*reinterpret_cast<const __half2*>(&acc[3]));
          l += ((s0.x + s0.y) + (s1.x + s1.y)) + ((s2.x + s2.y) + (s3.x + s3.y));
        }
        tmem_st_32cols(tmem + lane_off + COL_P + pbuf * 32, pw);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[pbuf]);
        pbuf ^= 1;
        ++pv_count;
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.list_empty[buf]);
      if (!warp_wait(&sm.o_full, o_phase)) break;
      o_phase ^= 1;
      tc_fence_after();
      const float vhead = a.vs_head[h];
      const float oscale = l > 0.f ? vhead / l : 0.f;
      const bool row_ok = rr < a.vbs_q[tq];
      const size_t orow =
          (size_t)((tq / a.tpc_q) * a.heads + h) * (size_t)a.rows_chunk_q + (size_t)(tq % a.tpc_q) * TILE + rr;
      bf16* dst = a.out + orow * D;
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
      if (a.lse && row_ok) a.lse[orow] = l > 0.f ? m_ref + __log2f(l) : -INFINITY;
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
#undef fail
#undef warp_wait

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

// [planes, rows, 128] e4m3 as a 3D tensor map with a {128 B, 64 rows, 1 plane} box, 128-byte swizzle
int make_map(CUtensorMap* m, const void* base, int64_t planes, int64_t rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)planes};
  cuuint64_t strides[2] = {(cuuint64_t)D, (cuuint64_t)rows * D};
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

extern "C" int h3b_vsa_fp8_ex(const h3b_vsa_args* x, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(x, "vsa_fp8: null argument block");
  H3B_REQUIRE(x->q && x->k && x->v && x->idx && x->num && x->vbs_q && x->vbs_kv && x->vs && x->vs_head && x->out,
              "vsa_fp8: null pointer");
  H3B_REQUIRE((x->qs == nullptr) == (x->ks == nullptr), "vsa_fp8: give both or neither per-tile Q/K scales");
  H3B_REQUIRE(x->heads > 0 && x->n_q_ext > 0 && x->n_q_ext % 2 == 0, "vsa_fp8: n_q_ext must be positive and even");
  H3B_REQUIRE(x->n_kv > 0 && x->n_kv <= N_MAX, "vsa_fp8: 1 <= n_kv <= %d key tiles", N_MAX);
  H3B_REQUIRE(x->idx_ld >= 1 && x->kv_scale_ld >= x->n_kv && (!x->qs || x->q_scale_ld >= x->n_q_ext),
              "vsa_fp8: bad idx / scale strides");
  H3B_REQUIRE(x->chunks_q > 0 && x->chunks_kv > 0 && x->rows_chunk_q > 0 && x->rows_chunk_kv > 0 &&
                  x->rows_chunk_q % TILE == 0 && x->rows_chunk_kv % TILE == 0,
              "vsa_fp8: chunk row counts must be positive multiples of 64");
  const int tpc_q = (int)(x->rows_chunk_q / TILE), tpc_kv = (int)(x->rows_chunk_kv / TILE);
  H3B_REQUIRE((int64_t)tpc_q * x->chunks_q >= x->n_q_ext && (int64_t)tpc_kv * x->chunks_kv >= x->n_kv,
              "vsa_fp8: chunks do not cover the tiles");
  H3B_REQUIRE(aligned(x->q, 16) && aligned(x->k, 16) && aligned(x->v, 16) && aligned(x->out, 16),
              "vsa_fp8: 16-byte aligned operands");
  CUtensorMap mq, mk, mv;
  if (int rc = make_map(&mq, x->q, (int64_t)x->chunks_q * x->heads, x->rows_chunk_q)) return rc;
  if (int rc = make_map(&mk, x->k, (int64_t)x->chunks_kv * x->heads, x->rows_chunk_kv)) return rc;
  if (int rc = make_map(&mv, x->v, (int64_t)x->chunks_kv * x->heads, x->rows_chunk_kv)) return rc;
  AttnArgs a{x->idx, x->num, x->vbs_q, x->vbs_kv, x->qs, x->ks, x->vs, x->vs_head, x->qk_coef,
             static_cast<bf16*>(x->out), x->lse, x->heads, x->n_q_ext, x->n_kv, x->idx_ld, x->q_scale_ld,
             x->kv_scale_ld, tpc_q, tpc_kv, x->rows_chunk_q, x->heads * (x->n_q_ext / 2)};
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
  vsa_fp8_kernel<<<grid, THREADS, smem, stream>>>(mq, mk, mv, a);
  H3B_LAUNCH_CHECK("vsa_fp8");
  return H3B_OK;
}

extern "C" int h3b_vsa_fp8(const void* qb, const void* kb, const void* vb, const int32_t* idx, const int32_t* num,
                           const int32_t* vbs, const float* qs_blk, const float* ks_blk, const float* vs_blk,
                           const float* vs_head, float qk_coef, void* out, float* lse, int heads, int n, int n_ext,
                           int64_t rows_pad, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(rows_pad == (int64_t)n_ext * TILE && n <= n_ext, "vsa_fp8: rows_pad must be n_ext * 64, n <= n_ext");
  h3b_vsa_args x{};
  x.q = qb;
  x.k = kb;
  x.v = vb;
  x.out = out;
  x.lse = lse;
  x.idx = idx;
  x.num = num;
  x.vbs_q = vbs;
  x.vbs_kv = vbs;
  x.qs = qs_blk;
  x.ks = ks_blk;
  x.vs = vs_blk;
  x.vs_head = vs_head;
  x.qk_coef = qk_coef;
  x.heads = heads;
  x.n_q_ext = n_ext;
  x.n_kv = n;            // key tiles: the real tiles (the padding tile is never selected)
  x.idx_ld = n;          // idx [heads, n_ext, n]
  x.q_scale_ld = n_ext;  // scales [heads, n_ext]
  x.kv_scale_ld = n_ext;
  x.rows_chunk_q = rows_pad;
  x.rows_chunk_kv = rows_pad;
  x.chunks_q = 1;
  x.chunks_kv = 1;
  return h3b_vsa_fp8_ex(&x, stream);
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
