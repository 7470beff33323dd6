// FP8 block-sparse VSA attention (fine step) for sm_100a: tcgen05 MMAs with TMEM accumulators, TMA staging, one
// persistent CTA per SM.
//
// Semantics (BASELINE config 4 and fastvideo/models/dits/h3fast/vsa_fp8.cuh:10-15, 716-764): for each (head, query
// tile) softmax attention of its rows over the keys of its selected 64-key tiles (keys past vbs_kv[b] masked), scores
// scaled by the softmax scale and the Q/K scales, fp32 online softmax with a lazy rescale (the running maximum moves
// only when a tile's maximum exceeds it by more than 2^4), bf16 output, optional log2-domain LSE.
//
// Arithmetic: S = Q8 K8^T on E4M3 operands (kind::f8f6f4), or on int8 codes (kind::i8, s32 accumulation, exact;
// h3b_vsa_args.qk_int8) whose integer S is converted to float before the softmax. P = 2^(S*coef - m) is evaluated in f16x2 (one
// ex2.approx.f16x2 per two keys; the exponent argument is at most 4 in magnitude for every key that matters, where f16
// resolves it to 2^-9), multiplied by the key tile's V-scale ratio sv_b / sv_head (P') after the row sum l = sum P is
// taken, and multiplied with V in f16 (kind::f16): V is stored E4M3 with one scale per (head, tile) and each V tile is
// converted exactly into f16 in shared memory once per use, so O = (sum P' V8) * sv_head / l. (The reference's kernel
// quantizes P to E4M3 instead; f16 P keeps the output within ~2^-9 of exact attention over the same E4M3 Q/K/V.)
//
// Operand layout: Q/out and K/V are each [chunks * heads, rows_chunk, 128] ("planes" of rows_chunk rows). Query tile t
// of head h lives in plane (t / tiles_per_chunk) * heads + h at row (t % tiles_per_chunk) * 64. With one chunk this is
// the plain heads-first [heads, rows, 128] layout; with P chunks it is exactly what an all-to-all over P ranks
// delivers ([source rank][local head][rows]), so sequence-parallel callers attend in place without a permute copy.
// K/V may be a different tensor with its own tile count (cross-attention to text tokens).
//
// Work item = (head, query tiles t0 = 2p and t1 = 2p+1), each with its own list of selected key tiles. The two tiles
// run as two M=64 MMA streams in the two half-subpartitions of TMEM (tile t0 in lanes 0-15 of each 32-lane quarter,
// t1 in lanes 16-31), so one 32-lane warp holds 16 rows of each tile and no MMA row computes a key tile its query tile
// did not select. Step j processes key tile j of both lists. Steps alternate between two softmax warpgroups (split-KV
// inside the CTA): each keeps its own running maximum, row sum and O accumulator, and the two partial results are
// merged in the epilogue. CTA = 11 warps:
//   warp 0      key-tile lists (from the top-k output) and TMA loads: the Q pair per item, K tiles and V tiles (two
//               rings: K is released by the S MMA, V only after the softmax converted it)
//   warps 1, 2  MMA issue for the even / odd steps (warp 1 also allocates TMEM): S_j = Q K_j^T (E4M3, M=64 N=64,
//               4 x K32 per tile) as soon as the warpgroup has read S_{j-2}, O_{j%2} += P_j V'_j (f16, M=64 N=128,
//               4 x K16 per tile, P from TMEM, V' from shared memory as an MN-major operand)
//   warps 3-6   steps of even index, warps 7-10 steps of odd index: the softmax with one query row per thread (TMEM
//               lane) and the 64 scores of a key tile in registers, then the step's E4M3 V tiles into f16 V'
//               (128-byte-swizzled MN-major layout); the epilogue merges the two warpgroups' partial results (each
//               writes half of the columns)
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
constexpr int K_STAGES = 4;   // E4M3 K tiles of both query tiles (consumed by the S MMAs)
constexpr int V_STAGES = 4;   // V ring slots (barriers): E4M3 V tiles of both query tiles (consumed by the conversion
                              // after the softmax), or 3 of f16 V tiles (consumed by the PV MMAs)
template <bool VF16>
constexpr int v_stages() { return 4; }
constexpr int N_MAX = 2048;   // key tiles
constexpr int L_MAX = 1024;   // longest selection list (more selected key tiles set H3B_EINVAL in the status word)
constexpr int SOFT_WARPS = 8;  // two warpgroups
constexpr int THREADS = (3 + SOFT_WARPS) * 32;  // producer, two MMA issuers, two softmax warpgroups
constexpr float RESCALE_LOG2 = 4.f;
constexpr uint64_t kLimitNs = 2000000000ull;
// TMEM columns: O of even / odd steps [0,128) [128,256), S of even / odd steps [256,320) [320,384), P (f16, 64 keys =
// 32 columns) of even / odd steps [384,416) [416,448). Query tile t1 uses the same columns at lane offset 16.
constexpr uint32_t COL_O = 0, COL_S = 256, COL_P = 384;
constexpr uint32_t LANE_B = 16u << 16;

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
  // pair mode (topk_pairs' format): idx / num hold one union list per (head, pair of query tiles) and u_mem a
  // membership byte per union entry (bit 0: tile 2p selected it, bit 1: tile 2p+1); NULL: one list per query tile
  const uint8_t* u_mem;
};

struct __align__(1024) Smem {
  uint8_t q[2][TILE * D];                    // [query tile] E4M3, 128-byte swizzle
  uint8_t k[K_STAGES][2][TILE * D];          // [stage][query tile]
  // V: with E4M3 V, the ring [4 stages][query tile][64 keys x 128 B] then the converted tiles V'
  // [warpgroup][query tile][half of d][64 keys x 128 B] (also the epilogue's output staging boxes); with f16 V, the
  // ring [4 stages][query tile][half of d][64 keys x 128 B] (the epilogue stores its rows directly)
  uint8_t vbuf[128 * 1024];
  uint16_t list[2][2][L_MAX];                // [buffer][query tile] selected key tiles
  float ml[2][2][2][128];                    // [item parity][max, sum][warpgroup][TMEM lane]
  int cnt[2][2];                             // [buffer][query tile] list lengths
  uint64_t q_full, q_empty;
  uint64_t k_full[K_STAGES], k_empty[K_STAGES];
  uint64_t v_full[V_STAGES], v_empty[V_STAGES];
  uint64_t list_full[2], list_empty[2];
  uint64_t s_full[2], s_free[2], p_full[2], pv_done[2];
  uint64_t ml_bar, o_full, o_empty, drain[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ uint8_t* v8_slot(Smem& sm, int stage, int s) { return sm.vbuf + (stage * 2 + s) * TILE * D; }
__device__ __forceinline__ uint8_t* vconv(Smem& sm, int w, int s) {
  return sm.vbuf + 64 * 1024 + (w * 2 + s) * 2 * TILE * 128;
}
__device__ __forceinline__ uint8_t* v16_slot(Smem& sm, int stage, int s) {
  return sm.vbuf + (stage * 2 + s) * 2 * TILE * 128;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// 3D tiled TMA store from this CTA's shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const void* src, const CUtensorMap* map, int32_t x, int32_t y, int32_t z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(smem_addr(src))
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


__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max of three floats in one instruction (sm_100)

// 2^(s * coef + nb) for two keys: both exponent arguments by one paired fp32 fused multiply-add (sm_100), rounded to
// f16 (s0 in the low half) and exponentiated in f16x2
__device__ __forceinline__ uint32_t ex2_pair(uint32_t s0, uint32_t s1, uint64_t coef2, uint64_t nb2) {
  uint32_t e;
  asm("{\n\t.reg .b64 s, x;\n\t.reg .f32 x0, x1;\n\t.reg .b32 h;\n\t"
      "mov.b64 s, {%1, %2};\n\t"
      "fma.rn.f32x2 x, s, %3, %4;\n\t"
      "mov.b64 {x0, x1}, x;\n\t"
      "cvt.rn.f16x2.f32 h, x1, x0;\n\t"
      "ex2.approx.f16x2 %0, h;\n\t}"
      : "=r"(e)
      : "r"(s0), "r"(s1), "l"(coef2), "l"(nb2));
  return e;
}

__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
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

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// two E4M3 bytes (low byte first) -> f16x2 (exact)
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(v));
  return h;
}

// K-major e4m3 tiles use desc_k_sw128; V' is MN-major: 64 f16 of d (128 bytes) per row, rows = keys, 8-row groups
// 1024 bytes apart (SBO), the two 64-column halves of d `lbo` bytes apart (LBO), 128-byte swizzle.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// fp32 accumulate, A and B of the same 8/16-bit type (E4M3 under kind::f8f6f4, f16 under kind::f16), A K-major,
// B K-major or MN-major
__host__ __device__ constexpr uint32_t idesc_mn(int m, int n, bool b_mn) {
  return (1u << 4) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// kind::i8: signed 8-bit A and B (format 1 in bits 7-9 and 10-12), s32 accumulate (format 2 in bits 4-5), both
// K-major
__host__ __device__ constexpr uint32_t idesc_s8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_s8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// an s32 accumulator word x -> the float x + 1.5 * 2^23, exact for |x| < 2^22 (|Q K^T| <= 128 * 127 * 127 < 2^21
// here): the integer added to the bit pattern of 1.5 * 2^23 lands in the mantissa of a float of that binade. The
// softmax keeps this biased value (order-preserving); the bias leaves the row maximum exactly and enters the
// exponent's constant term, fl(nb - 1.5 * 2^23 * coef), whose one rounding shifts every exponent of the step by at
// most 0.75 * coef (less than one integer unit of S).
constexpr float kS32Bias = 12582912.f;
__device__ __forceinline__ uint32_t s32_bits_to_biased_f32_bits(uint32_t x) { return (uint32_t)((int)x + 0x4B400000); }

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

// SH: the two query tiles of an item share one key list (the list of tile 2p; cross-attention to text, dense
// layers): each step loads one K and one V tile, and S and PV run as single M = 128 MMAs over both tiles (full
// datapath; row r of the pair in TMEM lane r, tile 2p in lanes 0-63) instead of two M = 64 streams.
template <bool QKI8, bool VF16, bool SH = false>
__global__ void __launch_bounds__(THREADS, 1)
    vsa_fp8_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 2);  // the last S MMA of each issuer
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.list_full[i], 1);
      mbar_init(&sm.list_empty[i], 2 + SOFT_WARPS);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], SOFT_WARPS / 2);
      mbar_init(&sm.p_full[i], SOFT_WARPS / 2);
      mbar_init(&sm.pv_done[i], 1);
    }
    for (int s = 0; s < K_STAGES; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);  // the S MMAs of the step have read the K tiles
    }
    for (int s = 0; s < V_STAGES; ++s) {
      mbar_init(&sm.v_full[s], 1);
      // E4M3 V: the step's warpgroup has converted the V tiles; f16 V: the step's PV MMAs have read them
      mbar_init(&sm.v_empty[s], VF16 ? 1 : SOFT_WARPS / 2);
    }
    mbar_init(&sm.ml_bar, SOFT_WARPS);
    mbar_init(&sm.o_full, 2);  // the last PV MMA of each issuer
    mbar_init(&sm.o_empty, SOFT_WARPS);
    mbar_init(&sm.drain[0], 1);
    mbar_init(&sm.drain[1], 1);
    sm.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmO);
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
    // -------------------------------------------------------------- key-tile lists + TMA producer
    uint32_t list_phase = 0, q_phase = 0, k_phase = 0, v_phase = 0;
    int kst = 0, vst = 0;
    bool ok = true;
    int it = 0;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
      const int buf = it & 1;
      const int h = item / pairs, p = item - h * pairs;
      const int t0 = 2 * p, t1 = 2 * p + 1;
      if (!warp_wait(&sm.list_empty[buf], ((list_phase >> buf) & 1u) ^ 1u)) break;
      list_phase ^= 1u << buf;
      int n[2];
      if (a.u_mem) {
        // the pair's union list, ascending, split by membership into each query tile's own list (ballot
        // compaction keeps the ascending order)
        const size_t urow = (size_t)h * pairs + p;
        const int u = min(max(a.num[urow], 0), a.idx_ld);
        const int32_t* src = a.idx + urow * a.idx_ld;
        const uint8_t* mem = a.u_mem + urow * a.idx_ld;
        const uint32_t below = (1u << lane) - 1u;
        int c[2] = {0, 0};
        for (int base = 0; base < u; base += 32) {
          const int i = base + lane;
          const uint32_t mb = i < u ? mem[i] : 0u;
          const uint16_t col = i < u ? (uint16_t)min(max(src[i], 0), a.n_kv - 1) : (uint16_t)0;
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const bool in = (mb >> s) & 1u;
            const uint32_t m = __ballot_sync(0xffffffffu, in);
            const int pos = c[s] + __popc(m & below);
            if (in && pos < L_MAX) sm.list[buf][s][pos] = col;
            c[s] += __popc(m);
          }
        }
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          n[s] = min(c[s], L_MAX);
          if (c[s] > L_MAX && lane == 0) atomicExch(&g_attn_status, H3B_EINVAL);
        }
      } else {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const int t = (s && !SH) ? t1 : t0;
          const int want = min(max(a.num[(size_t)h * a.n_q_ext + t], 0), a.idx_ld);
          n[s] = min(want, L_MAX);
          if (want > L_MAX && lane == 0) atomicExch(&g_attn_status, H3B_EINVAL);
          const int32_t* src = a.idx + ((size_t)h * a.n_q_ext + t) * a.idx_ld;
          for (int i = lane; i < n[s]; i += 32) sm.list[buf][s][i] = (uint16_t)min(max(src[i], 0), a.n_kv - 1);
        }
      }
      __syncwarp();
      if (lane == 0) {
        sm.cnt[buf][0] = n[0];
        sm.cnt[buf][1] = n[1];
        mbar_arrive(&sm.list_full[buf]);
      }
      __syncwarp();
      const int U = max(n[0], n[1]);
      if (lane == 0) {
        if (!mbar_wait_bounded(&sm.q_empty, q_phase ^ 1, abort_flag, kLimitNs)) {
          fail();
          ok = false;
        } else {
          q_phase ^= 1;
          mbar_arrive_expect_tx(&sm.q_full, 2 * TILE * D);
          for (int s = 0; s < 2; ++s) {
            const int t = s ? t1 : t0;
            tma_load_3d(&sm.q[s][0], &tmQ, 0, (t % a.tpc_q) * TILE, (t / a.tpc_q) * a.heads + h, &sm.q_full);
          }
          for (int j = 0; j < U && ok; ++j) {
            const bool has0 = j < n[0], has1 = !SH && j < n[1];  // shared lists: one K and one V tile per step
            const uint32_t bytes = (has0 ? TILE * D : 0) + (has1 ? TILE * D : 0);
            if (!mbar_wait_bounded(&sm.k_empty[kst], ((k_phase >> kst) & 1u) ^ 1u, abort_flag, kLimitNs)) {
              fail();
              ok = false;
              break;
            }
            k_phase ^= 1u << kst;
            mbar_arrive_expect_tx(&sm.k_full[kst], bytes);
#pragma unroll
            for (int s = 0; s < 2; ++s) {
              if (s ? !has1 : !has0) continue;
              const int b = sm.list[buf][s][j];
              tma_load_3d(&sm.k[kst][s][0], &tmK, 0, (b % a.tpc_kv) * TILE, (b / a.tpc_kv) * a.heads + h,
                          &sm.k_full[kst]);
            }
            if (++kst == K_STAGES) kst = 0;
            if (!mbar_wait_bounded(&sm.v_empty[vst], ((v_phase >> vst) & 1u) ^ 1u, abort_flag, kLimitNs)) {
              fail();
              ok = false;
              break;
            }
            v_phase ^= 1u << vst;
            mbar_arrive_expect_tx(&sm.v_full[vst], VF16 ? 2 * bytes : bytes);
#pragma unroll
            for (int s = 0; s < 2; ++s) {
              if (s ? !has1 : !has0) continue;
              const int b = sm.list[buf][s][j];
              if constexpr (VF16) {  // 64 keys x 128 f16 as two 128-byte-wide boxes (the halves of d)
                for (int half = 0; half < 2; ++half)
                  tma_load_3d(v16_slot(sm, vst, s) + half * TILE * 128, &tmV, 128 * half, (b % a.tpc_kv) * TILE,
                              (b / a.tpc_kv) * a.heads + h, &sm.v_full[vst]);
              } else {
                tma_load_3d(v8_slot(sm, vst, s), &tmV, 0, (b % a.tpc_kv) * TILE, (b / a.tpc_kv) * a.heads + h,
                            &sm.v_full[vst]);
              }
            }
            if (++vst == v_stages<VF16>()) vst = 0;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
  } else if (warp == 1 || warp == 2) {
    // -------------------------------------------------------------- MMA issuers: warp 1 even steps, warp 2 odd steps
    if (lane == 0) {
      const int w = warp - 1;
      constexpr int MQ = SH ? 2 * TILE : TILE;  // query rows per MMA
      const uint32_t idesc_s = QKI8 ? idesc_s8(MQ, TILE) : idesc_mn(MQ, TILE, false);
      const uint32_t idesc_pv = idesc_mn(MQ, D, true);
      uint32_t list_phase = 0, q_phase = 0, s_phase = 0, p_phase = 0, o_phase = 0;
      uint32_t gbase = 0;  // steps of all earlier items: step j is K-ring use gbase + j
      bool ok = true;
      int it = 0;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
        const int buf = it & 1;
        if (!mbar_wait_bounded(&sm.list_full[buf], (list_phase >> buf) & 1u, abort_flag, kLimitNs)) { fail(); break; }
        list_phase ^= 1u << buf;
        const int n0 = sm.cnt[buf][0], n1 = sm.cnt[buf][1];
        const int U = max(n0, n1);
        if (!mbar_wait_bounded(&sm.q_full, q_phase, abort_flag, kLimitNs)) { fail(); break; }
        q_phase ^= 1;
        tc_fence_after();
        const uint64_t dq0 = desc_k_sw128(smem_addr(&sm.q[0][0]));
        const uint64_t dq1 = desc_k_sw128(smem_addr(&sm.q[1][0]));
        uint32_t started = 0;  // bit s: O of this issuer's parity, query tile s, has been written this item
        const int last_s = U > w ? w + ((U - 1 - w) / 2) * 2 : -1;  // this issuer's last step
        if (last_s < 0) tc_commit(&sm.q_empty);
        // j = w - 2 issues S(w) only; step j issues S(j+2) (into S buffer w, once warpgroup w has read S(j)) and then
        // PV(j)
        for (int j = w - 2; j < U; j += 2) {
          const int js = j + 2;
          if (js < U) {
            const uint32_t g = gbase + (uint32_t)js;
            const int kst = (int)(g % K_STAGES);
            if (!mbar_wait_bounded(&sm.s_free[w], (s_phase & 1u) ^ 1u, abort_flag, kLimitNs) ||
                !mbar_wait_bounded(&sm.k_full[kst], (g / K_STAGES) & 1u, abort_flag, kLimitNs)) {
              fail();
              ok = false;
              break;
            }
            s_phase ^= 1;
            tc_fence_after();
#pragma unroll
            for (int s = 0; s < 2; ++s) {
              if (js >= (s ? n1 : n0) || (SH && s)) continue;
              const uint32_t lo = s ? LANE_B : 0u;
              const uint64_t dk = desc_k_sw128(smem_addr(&sm.k[kst][s][0]));
              const uint64_t dq = s ? dq1 : dq0;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                if constexpr (QKI8)
                  mma_s8(tmem + lo + COL_S + 64 * w, dq + 2 * i, dk + 2 * i, idesc_s, i != 0);
                else
                  mma_e4m3(tmem + lo + COL_S + 64 * w, dq + 2 * i, dk + 2 * i, idesc_s, i != 0);
              }
            }
            tc_commit(&sm.s_full[w]);
            tc_commit(&sm.k_empty[kst]);  // the K tiles of the stage are consumed
            if (js == last_s) tc_commit(&sm.q_empty);
          }
          if (j < w) continue;
          if (j == w) {
            if (!mbar_wait_bounded(&sm.o_empty, o_phase ^ 1, abort_flag, kLimitNs)) { fail(); ok = false; break; }
            o_phase ^= 1;
          }
          if (!mbar_wait_bounded(&sm.p_full[w], p_phase & 1u, abort_flag, kLimitNs)) {  // P and V' of step j ready
            fail();
            ok = false;
            break;
          }
          p_phase ^= 1;
          const uint32_t gv = gbase + (uint32_t)j;
          const int vstage = (int)(gv % (uint32_t)v_stages<VF16>());
          if constexpr (VF16) {  // the f16 V tiles of step j landed
            if (!mbar_wait_bounded(&sm.v_full[vstage], (gv / (uint32_t)v_stages<VF16>()) & 1u, abort_flag,
                                   kLimitNs)) {
              fail();
              ok = false;
              break;
            }
          }
          tc_fence_after();
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            if (j >= (s ? n1 : n0) || (SH && s)) continue;
            const uint32_t lo = s ? LANE_B : 0u;
            const uint64_t dv =
                desc_mn_sw128(smem_addr(VF16 ? v16_slot(sm, vstage, s) : vconv(sm, w, s)), TILE * 128);
            const uint32_t bit = 1u << s;
#pragma unroll
            for (int i = 0; i < 4; ++i)  // K = 16 keys per MMA: 8 TMEM columns of P, 16 rows (2048 bytes) of V'
              mma_f16_ts(tmem + lo + COL_O + 128 * w, tmem + lo + COL_P + 32 * w + 8 * i,
                         dv + (uint64_t)((i * 16 * 128) >> 4), idesc_pv, ((started & bit) || i) ? 1u : 0u);
            started |= bit;
          }
          tc_commit(&sm.pv_done[w]);
          if constexpr (VF16) tc_commit(&sm.v_empty[vstage]);  // the V tiles of the stage are consumed
        }
        if (!ok) break;
        if (U <= w) {  // no step of this parity: O of this parity is not used, but the epilogue waits for both
          if (!mbar_wait_bounded(&sm.o_empty, o_phase ^ 1, abort_flag, kLimitNs)) { fail(); break; }
          o_phase ^= 1;
        }
        gbase += (uint32_t)U;
        tc_commit(&sm.o_full);
        mbar_arrive(&sm.list_empty[buf]);
      }
      tc_commit(&sm.drain[w]);
      volatile int no_abort = 0;
      if (!mbar_wait_bounded(&sm.drain[w], 0, &no_abort, kLimitNs)) fail();
    }
  } else {
    // -------------------------------------------------------------- softmax (steps of parity w) + epilogue
    const int w = (warp - 3) >> 2;               // warpgroup: 0 = even steps, 1 = odd steps
    const int q4 = warp & 3;                     // TMEM lane quarter this warp may access
    // query tile and row of this thread's TMEM lane: M = 64 streams put tile t0 in lanes 0-15 and t1 in lanes 16-31
    // of each quarter; an M = 128 MMA (shared lists) puts t0 in lanes 0-63 and t1 in lanes 64-127
    const int tsel = SH ? (q4 >> 1) : (lane >> 4);
    const int rt = SH ? 32 * (q4 & 1) + lane : 16 * q4 + (lane & 15);
    const int tl = q4 * 32 + lane;               // TMEM lane
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    uint32_t list_phase = 0, s_phase = 0, ml_phase = 0, o_phase = 0;
    uint32_t pv_count = 0;  // PV MMAs of this warpgroup's parity issued so far (all items)
    uint32_t gbase = 0;     // steps of all earlier items: step j of this item is ring use gbase + j
    int it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
      const int buf = it & 1;
      const int h = item / pairs, p = item - h * pairs;
      const int tq = 2 * p + tsel;
      if (!warp_wait(&sm.list_full[buf], (list_phase >> buf) & 1u)) break;
      list_phase ^= 1u << buf;
      const int n_me = sm.cnt[buf][tsel];
      const int U = max(sm.cnt[buf][0], sm.cnt[buf][1]);
      const float qcoef = a.coef * (a.qs ? a.qs[(size_t)h * a.q_scale_ld + tq] : 1.f);
      const float* ksh = a.ks ? a.ks + (size_t)h * a.kv_scale_ld : nullptr;
      const float* vsh = a.vs + (size_t)h * a.kv_scale_ld;
      const int n0 = sm.cnt[buf][0], n1 = sm.cnt[buf][1];
      const float inv_vhead = 1.f / a.vs_head[h];
      float m_ref = -INFINITY, l = 0.f;
      // per-tile scalars of this warpgroup's next key tile are loaded one step ahead (global loads off the critical
      // path; their values are only used in the next iteration)
      int vbs_next = 0;
      float ks_next = 1.f, vs_next = 0.f;
      if (w < n_me) {
        const int b0 = sm.list[buf][tsel][w];
        vbs_next = a.vbs_kv[b0];
        vs_next = vsh[b0];
        if (ksh) ks_next = ksh[b0];
      }
      for (int j = w; j < U; j += 2) {
        const bool valid = j < n_me;
        const int vbs_j = valid ? vbs_next : 0;
        const float ks_j = ks_next, vs_j = vs_next;
        if (j + 2 < n_me) {
          const int bn = sm.list[buf][tsel][j + 2];
          vbs_next = a.vbs_kv[bn];
          vs_next = vsh[bn];
          if (ksh) ks_next = ksh[bn];
        }
        const uint32_t g = gbase + (uint32_t)j;
        const int stage = (int)(g % V_STAGES);
        // ---- softmax of step j
        if (!warp_wait(&sm.s_full[w], (s_phase >> w) & 1u)) { ok = false; break; }
        s_phase ^= 1u << w;
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld_32cols(tmem + lane_off + COL_S + 64 * w, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tmem_ld_32cols(tmem + lane_off + COL_S + 64 * w + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_free[w]);
        if constexpr (QKI8) {
#pragma unroll
          for (int c = 0; c < 64; ++c) sr[c] = s32_bits_to_biased_f32_bits(sr[c]);
        }
        if (__any_sync(0xffffffffu, vbs_j < TILE)) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= vbs_j) sr[c] = __float_as_uint(-INFINITY);
        }
        const float coef = qcoef * ks_j;
        // row maximum: four chains of three-input maxima
        float m4[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) m4[c] = fmaxf(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1]));
#pragma unroll
        for (int c = 4; c < 32; ++c)
          m4[c & 3] = fmax3(m4[c & 3], __uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1]));
        float mraw = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
        if constexpr (QKI8) {
          if (mraw != -INFINITY) mraw = __fsub_rn(mraw, kS32Bias);  // exact
        }
        const float mx = mraw == -INFINITY ? -INFINITY : mraw * coef;  // coef > 0
        const bool grow = mx > m_ref + RESCALE_LOG2;
        const bool had_mass = m_ref != -INFINITY;
        float alpha = 1.f;
        if (grow) {
          alpha = had_mass ? ex2(m_ref - mx) : 1.f;
          m_ref = mx;
        }
        if (__any_sync(0xffffffffu, grow && had_mass)) {
          // the previous PV of this parity must have landed in O before O is rescaled
          if (pv_count > 0 && !warp_wait(&sm.pv_done[w], (pv_count - 1) & 1u)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t o[32];
            tmem_ld_32cols(tmem + lane_off + COL_O + 128 * w + c0, o);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st_32cols(tmem + lane_off + COL_O + 128 * w + c0, o);
          }
          tmem_st_wait();
        }
        l *= alpha;
        uint32_t pw[32];
        if (m_ref == -INFINITY) {
#pragma unroll
          for (int c = 0; c < 32; ++c) pw[c] = 0u;
        } else {
          const float nb = QKI8 ? fmaf(-kS32Bias, coef, -m_ref) : -m_ref;
          uint32_t acc[4] = {0u, 0u, 0u, 0u};
          const __half2 vr2 = __float2half2_rn(vs_j * inv_vhead);  // P' = P * sv_b / sv_head: V' is V8 itself
          const uint32_t vr = *reinterpret_cast<const uint32_t*>(&vr2);
          const uint64_t coef2 = pack_f32x2(coef, coef), nb2 = pack_f32x2(nb, nb);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const uint32_t e = ex2_pair(sr[2 * c], sr[2 * c + 1], coef2, nb2);
            acc[c & 3] = hadd2(acc[c & 3], e);
            pw[c] = hmul2(e, vr);
          }
          const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&acc[0]));
          const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&acc[1]));
          const float2 s2 = __half22float2(*reinterpret_cast<const __half2*>(&acc[2]));
          const float2 s3 = __half22float2(*reinterpret_cast<const __half2*>(&acc[3]));
          l += ((s0.x + s0.y) + (s1.x + s1.y)) + ((s2.x + s2.y) + (s3.x + s3.y));
        }
        // this warpgroup's previous PV (step j-2) reads the P and V' buffers this step overwrites: it was issued when
        // that step ended and has normally completed while P was computed
        if (pv_count > 0 && !warp_wait(&sm.pv_done[w], (pv_count - 1) & 1u)) { ok = false; break; }
        tmem_st_32cols(tmem + lane_off + COL_P + 32 * w, pw);
        // ---- V' of this step (E4M3 V only: f16 V tiles are read by the PV MMAs as they land)
        if constexpr (!VF16) {
        if (!warp_wait(&sm.v_full[stage], (g / V_STAGES) & 1u)) { ok = false; break; }
        {
          // 16 E4M3 values (d = 16c .. 16c+15) of one key per thread and chunk; a warp covers 8 consecutive keys x 4
          // chunks per load, so its 16-byte loads and stores each touch every bank group four times (no bank
          // conflicts). All eight loads (both query tiles) are issued before the conversions.
          uint4 raw[2][4];
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            if (j >= (s ? n1 : n0) || (SH && s)) continue;  // warpgroup-uniform
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int key = (lane & 7) + 8 * (q4 + 4 * (i & 1)), c = (lane >> 3) + 4 * (i >> 1);
              raw[s][i] = *reinterpret_cast<const uint4*>(v8_slot(sm, stage, s) + key * 128 + ((c ^ (key & 7)) << 4));
            }
          }
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            if (j >= (s ? n1 : n0) || (SH && s)) continue;
            uint8_t* dst = vconv(sm, w, s);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int key = (lane & 7) + 8 * (q4 + 4 * (i & 1)), c = (lane >> 3) + 4 * (i >> 1);
              const uint32_t wv[4] = {raw[s][i].x, raw[s][i].y, raw[s][i].z, raw[s][i].w};
              uint32_t f[8];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                f[2 * q] = e4m3x2_to_f16x2((uint16_t)(wv[q] & 0xFFFFu));
                f[2 * q + 1] = e4m3x2_to_f16x2((uint16_t)(wv[q] >> 16));
              }
              uint8_t* half_base = dst + (c >> 2) * (TILE * 128) + key * 128;
              const int dc0 = (c & 3) * 2;
              *reinterpret_cast<uint4*>(half_base + ((dc0 ^ (key & 7)) << 4)) = make_uint4(f[0], f[1], f[2], f[3]);
              *reinterpret_cast<uint4*>(half_base + (((dc0 + 1) ^ (key & 7)) << 4)) =
                  make_uint4(f[4], f[5], f[6], f[7]);
            }
          }
        }
        fence_proxy_async_smem();  // the generic-proxy stores become visible to the tensor core
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (!VF16) mbar_arrive(&sm.v_empty[stage]);  // the V tiles are consumed
          mbar_arrive(&sm.p_full[w]);  // P of step j in TMEM (and, E4M3 V, V' of step j in shared memory)
        }
        ++pv_count;
      }
      if (!ok) break;
      gbase += (uint32_t)U;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.list_empty[buf]);
      // merge the two warpgroups' partial results: exchange (max, sum) per row through shared memory
      const int par = it & 1;
      sm.ml[par][0][w][tl] = m_ref;
      sm.ml[par][1][w][tl] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.ml_bar);
      if (!warp_wait(&sm.ml_bar, ml_phase)) break;
      ml_phase ^= 1;
      const float m_other = sm.ml[par][0][w ^ 1][tl], l_other = sm.ml[par][1][w ^ 1][tl];
      const float m0 = w ? m_other : m_ref, m1 = w ? m_ref : m_other;  // selects, not a runtime-indexed array
      const float l0 = w ? l_other : l, l1 = w ? l : l_other;
      const float M = fmaxf(m0, m1);
      const float f0 = (M == -INFINITY || m0 == -INFINITY) ? 0.f : ex2(m0 - M);
      const float f1 = (M == -INFINITY || m1 == -INFINITY) ? 0.f : ex2(m1 - M);
      const float L = l0 * f0 + l1 * f1;
      if (!warp_wait(&sm.o_full, o_phase)) break;
      o_phase ^= 1;
      tc_fence_after();
      const float vhead = a.vs_head[h];
      const float oscale = L > 0.f ? vhead / L : 0.f;
      const bool row_ok = rt < a.vbs_q[tq];
      const size_t orow =
          (size_t)((tq / a.tpc_q) * a.heads + h) * (size_t)a.rows_chunk_q + (size_t)(tq % a.tpc_q) * TILE + rt;
      const float g0 = f0 * oscale, g1 = f1 * oscale;
      // warpgroup w writes output columns 64w .. 64w+63 of both query tiles: each row (TMEM lane) is staged as 128
      // bytes of bf16 in a 64-row box per query tile (128-byte swizzle; the V' buffer of this warpgroup is idle here:
      // every PV of the item has completed), then one thread stores both boxes with TMA. Rows past the tile's length
      // are written as zeros (padding rows of the tile's 64-row slot).
      uint8_t* box = vconv(sm, w, tsel);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c0 = 64 * w + 32 * cc;
        uint32_t o0[32], o1[32];
        tmem_ld_32cols(tmem + lane_off + COL_O + c0, o0);
        tmem_ld_32cols(tmem + lane_off + COL_O + 128 + c0, o1);
        tmem_ld_wait();
        if (cc == 1) {  // both accumulators read: the next item's PV MMAs may overwrite them
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.o_empty);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t pk[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c = 8 * j + 2 * u;
            // a partial with no mass contributes nothing (its O may be stale)
            const float x0 = (g0 != 0.f ? __uint_as_float(o0[c]) * g0 : 0.f) + (g1 != 0.f ? __uint_as_float(o1[c]) * g1 : 0.f);
            const float x1 =
                (g0 != 0.f ? __uint_as_float(o0[c + 1]) * g0 : 0.f) + (g1 != 0.f ? __uint_as_float(o1[c + 1]) * g1 : 0.f);
            pk[u] = row_ok ? pack_bf16x2(x0, x1) : 0u;
          }
          if constexpr (VF16) {  // the row's 128 bytes of this warpgroup's columns, stored directly
            *reinterpret_cast<uint4*>(a.out + orow * D + c0 + 8 * j) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          } else {
            const int chunk = 4 * cc + j;  // 16-byte chunk of the 128-byte box row
            *reinterpret_cast<uint4*>(box + rt * 128 + ((chunk ^ (rt & 7)) << 4)) =
                make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        }
      }
      if constexpr (!VF16) {
        fence_proxy_async_smem();
        asm volatile("bar.sync %0, 128;" ::"r"(1 + w) : "memory");  // the warpgroup's rows are staged
        if (warp == 3 + 4 * w && lane == 0) {
#pragma unroll
          for (int s2 = 0; s2 < 2; ++s2) {
            const int t = 2 * p + s2;
            tma_store_3d(vconv(sm, w, s2), &tmO, 64 * w, (t % a.tpc_q) * TILE, (t / a.tpc_q) * a.heads + h);
          }
          bulk_commit_group();
          bulk_wait_read<0>();  // the boxes are read before the next conversion overwrites the V' buffer
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + w) : "memory");
      }
      if (a.lse && row_ok && w == 0) a.lse[orow] = L > 0.f ? M + __log2f(L) : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
#undef fail
#undef warp_wait
}

#include "vsa_ws.cuh"

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
// bf16 output [planes, rows, 128] with a {64 columns, 64 rows, 1 plane} box (128-byte rows, 128-byte swizzle)
int make_out_map(CUtensorMap* m, const void* base, int64_t planes, int64_t rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)planes};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)rows * D * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)TILE, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return H3B_OK;
}

// f16 V [planes, rows, 128] as bytes [planes, rows, 256]: 128-byte-wide boxes of 64 rows (one half of d each)
int make_map_v16(CUtensorMap* m, const void* base, int64_t planes, int64_t rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)(2 * D), (cuuint64_t)rows, (cuuint64_t)planes};
  cuuint64_t strides[2] = {(cuuint64_t)(2 * D), (cuuint64_t)rows * 2 * D};
  cuuint32_t box[3] = {128, (cuuint32_t)TILE, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return H3B_OK;
}

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

namespace h3b {
namespace {
int vsa_launch(const h3b_vsa_args* x, const uint8_t* u_mem, bool v16, cudaStream_t stream, bool shared = false);
}  // namespace
}  // namespace h3b

extern "C" int h3b_vsa_fp8_ex(const h3b_vsa_args* x, cudaStream_t stream) {
  clear_error();
  return h3b::vsa_launch(x, nullptr, false, stream);
}

extern "C" int h3b_vsa_fp8_ex_v16(const h3b_vsa_args* x, cudaStream_t stream) {
  clear_error();
  return h3b::vsa_launch(x, nullptr, true, stream);
}

extern "C" int h3b_vsa_fp8_shared(const h3b_vsa_args* x, cudaStream_t stream) {
  clear_error();
  return h3b::vsa_launch(x, nullptr, false, stream, true);
}

extern "C" int h3b_vsa_fp8_shared_v16(const h3b_vsa_args* x, cudaStream_t stream) {
  clear_error();
  return h3b::vsa_launch(x, nullptr, true, stream, true);
}

extern "C" int h3b_vsa_pair(const h3b_vsa_args* x, const uint8_t* u_mem, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(u_mem, "vsa_pair: null membership bytes");
  return h3b::vsa_launch(x, u_mem, false, stream);
}

extern "C" int h3b_vsa_pair_v16(const h3b_vsa_args* x, const uint8_t* u_mem, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(u_mem, "vsa_pair: null membership bytes");
  return h3b::vsa_launch(x, u_mem, true, stream);
}

namespace h3b {
namespace {
int vsa_launch(const h3b_vsa_args* x, const uint8_t* u_mem, bool v16, cudaStream_t stream, bool shared) {
  H3B_REQUIRE(x, "vsa_fp8: null argument block");
  H3B_REQUIRE(!shared || !x->qk_int8, "vsa_fp8_shared: E4M3 QK^T only");
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
  CUtensorMap mq, mk, mv, mo;
  if (int rc = make_map(&mq, x->q, (int64_t)x->chunks_q * x->heads, x->rows_chunk_q)) return rc;
  if (int rc = make_map(&mk, x->k, (int64_t)x->chunks_kv * x->heads, x->rows_chunk_kv)) return rc;
  if (int rc = v16 ? make_map_v16(&mv, x->v, (int64_t)x->chunks_kv * x->heads, x->rows_chunk_kv)
                    : make_map(&mv, x->v, (int64_t)x->chunks_kv * x->heads, x->rows_chunk_kv))
    return rc;
  if (int rc = make_out_map(&mo, x->out, (int64_t)x->chunks_q * x->heads, x->rows_chunk_q)) return rc;
  AttnArgs a{x->idx, x->num, x->vbs_q, x->vbs_kv, x->qs, x->ks, x->vs, x->vs_head, x->qk_coef,
             static_cast<bf16*>(x->out), x->lse, x->heads, x->n_q_ext, x->n_kv, x->idx_ld, x->q_scale_ld,
             x->kv_scale_ld, tpc_q, tpc_kv, x->rows_chunk_q, x->heads * (x->n_q_ext / 2), u_mem};
  const int smem = (int)sizeof(Smem) + 1024;
  auto kern = shared ? (v16 ? vsa_fp8_kernel<false, true, true> : vsa_fp8_kernel<false, false, true>)
             : x->qk_int8 ? (v16 ? vsa_fp8_kernel<true, true> : vsa_fp8_kernel<true, false>)
                          : (v16 ? vsa_fp8_kernel<false, true> : vsa_fp8_kernel<false, false>);
  static PerDevice setup[6];  // the shared-memory reservation per instantiation and device; the value is the SM count
  int sms = 0;
  if (int rc = setup[shared ? 4 + (v16 ? 1 : 0) : (x->qk_int8 ? 1 : 0) + (v16 ? 2 : 0)].get([&](int* v) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
          return set_error(H3B_ECUDA, "vsa_fp8: cannot reserve %d bytes of shared memory", smem);
        *v = current_sms();
        return H3B_OK;
      }, &sms))
    return rc;
  const int grid = a.items < sms ? a.items : sms;
  kern<<<grid, THREADS, smem, stream>>>(mq, mk, mv, mo, a);
  H3B_LAUNCH_CHECK("vsa_fp8");
  return H3B_OK;
}
}  // namespace
}  // namespace h3b

namespace h3b {
namespace {
// The wide-step kernel (vsa_ws.cuh): E4M3 Q/K, f16 V, one key list per query tile.
int vsa_ws_launch(const h3b_vsa_args* x, cudaStream_t stream) {
  H3B_REQUIRE(x, "vsa_fp8_ws: null argument block");
  H3B_REQUIRE(!x->qk_int8, "vsa_fp8_ws: E4M3 QK^T only");
  H3B_REQUIRE(x->q && x->k && x->v && x->idx && x->num && x->vbs_q && x->vbs_kv && x->vs && x->vs_head && x->out,
              "vsa_fp8_ws: null pointer");
  H3B_REQUIRE((x->qs == nullptr) == (x->ks == nullptr), "vsa_fp8_ws: give both or neither per-tile Q/K scales");
  H3B_REQUIRE(x->heads > 0 && x->n_q_ext > 0 && x->n_q_ext % 2 == 0, "vsa_fp8_ws: n_q_ext must be positive and even");
  H3B_REQUIRE(x->n_kv > 0 && x->n_kv <= N_MAX, "vsa_fp8_ws: 1 <= n_kv <= %d key tiles", N_MAX);
  H3B_REQUIRE(x->idx_ld >= 1 && x->kv_scale_ld >= x->n_kv && (!x->qs || x->q_scale_ld >= x->n_q_ext),
              "vsa_fp8_ws: bad idx / scale strides");
  H3B_REQUIRE(x->chunks_q > 0 && x->chunks_kv > 0 && x->rows_chunk_q > 0 && x->rows_chunk_kv > 0 &&
                  x->rows_chunk_q % TILE == 0 && x->rows_chunk_kv % TILE == 0,
              "vsa_fp8_ws: chunk row counts must be positive multiples of 64");
  const int tpc_q = (int)(x->rows_chunk_q / TILE), tpc_kv = (int)(x->rows_chunk_kv / TILE);
  H3B_REQUIRE((int64_t)tpc_q * x->chunks_q >= x->n_q_ext && (int64_t)tpc_kv * x->chunks_kv >= x->n_kv,
              "vsa_fp8_ws: chunks do not cover the tiles");
  H3B_REQUIRE(aligned(x->q, 16) && aligned(x->k, 16) && aligned(x->v, 16) && aligned(x->out, 16),
              "vsa_fp8_ws: 16-byte aligned operands");
  CUtensorMap mq, mk, mv;
  if (int rc = make_map(&mq, x->q, (int64_t)x->chunks_q * x->heads, x->rows_chunk_q)) return rc;
  if (int rc = make_map(&mk, x->k, (int64_t)x->chunks_kv * x->heads, x->rows_chunk_kv)) return rc;
  if (int rc = make_map_v16(&mv, x->v, (int64_t)x->chunks_kv * x->heads, x->rows_chunk_kv)) return rc;
  AttnArgs a{x->idx, x->num, x->vbs_q, x->vbs_kv, x->qs, x->ks, x->vs, x->vs_head, x->qk_coef,
             static_cast<bf16*>(x->out), x->lse, x->heads, x->n_q_ext, x->n_kv, x->idx_ld, x->q_scale_ld,
             x->kv_scale_ld, tpc_q, tpc_kv, x->rows_chunk_q, x->heads * (x->n_q_ext / 2), nullptr};
  const int smem = (int)sizeof(ws::Smem) + 1024;
  static PerDevice setup;  // the shared-memory reservation per device; the value is the SM count
  int sms = 0;
  if (int rc = setup.get([&](int* v) {
        if (cudaFuncSetAttribute(vsa_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
          return set_error(H3B_ECUDA, "vsa_fp8_ws: cannot reserve %d bytes of shared memory", smem);
        *v = current_sms();
        return H3B_OK;
      }, &sms))
    return rc;
  const int grid = a.items < sms ? a.items : sms;
  vsa_ws_kernel<<<grid, ws::THREADS, smem, stream>>>(mq, mk, mv, a);
  H3B_LAUNCH_CHECK("vsa_fp8_ws");
  return H3B_OK;
}
}  // namespace
}  // namespace h3b

extern "C" int h3b_vsa_fp8_ws(const h3b_vsa_args* x, cudaStream_t stream) {
  clear_error();
  return h3b::vsa_ws_launch(x, stream);
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

namespace h3b {
int attn_status_async(int* dst, int clear, cudaStream_t stream) {
  if (cudaMemcpyFromSymbolAsync(dst, g_attn_status, sizeof(int), 0, cudaMemcpyDefault, stream) != cudaSuccess)
    return set_error(H3B_ECUDA, "status: reading the attention status word failed");
  if (clear) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_status) != cudaSuccess || cudaMemsetAsync(p, 0, sizeof(int), stream) != cudaSuccess)
      return set_error(H3B_ECUDA, "status: clearing the attention status word failed");
  }
  return H3B_OK;
}
}  // namespace h3b

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
