// Persistent, warp-specialized tcgen05 GEMMs for the DiT linears, fp32 accumulators in tensor memory and a fused
// epilogue (scales, bias, GELU-tanh, gated residual, bf16 store):
//   gemm_fp8_kernel        FP8 (kind::f8f6f4, e4m3 x e4m3), one CTA per SM, 128x256 tiles
//   gemm_nvfp4_pair_kernel NVFP4 (kind::mxf4nvf4 block16, e2m1 x e2m1 with ue4m3 scales per 16 K-elements) on CTA
//                          pairs (cta_group::2), 256x192 tiles; described where it is defined
//
// gemm_fp8_kernel: CTA = 10 warps, one CTA per SM (the shared-memory footprint forbids two):
//   warp 0   TMA producer: A/B tiles (128-byte swizzle)
//   warp 1   TMEM allocator + MMA issuer (one thread): 4 MMAs per 128-byte K block
//   warps 2-9 epilogue: TMEM -> registers -> epilogue math -> global (warp w reads TMEM lanes 32*(w%4)..+31; warps
//            2-5 take the first half of the tile's columns, warps 6-9 the second)
// Two accumulator buffers in TMEM let the epilogue of tile j overlap the main loop of tile j+1.
// Every mbarrier wait is bounded (2 s); on expiry the CTA records H3B_ETIMEOUT in a device status word, the other
// roles abandon their loops, in-flight copies and MMAs are drained (again bounded) and TMEM is freed.
#include "common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <algorithm>

namespace h3b {

__device__ int g_gemm_status = 0;

namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int KB_BYTES = 128;  // one swizzle atom of K per stage
constexpr uint64_t kWaitLimitNs = 2000000000ull;

template <int BN>
struct Cfg8 {
  static constexpr int kStages = 4;
  static constexpr int kABytes = BM * KB_BYTES;
  static constexpr int kBBytes = BN * KB_BYTES;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAccCols = BN;
  static constexpr int kThreads = 320;  // 2 + 8 epilogue warps (two per TMEM lane quarter, half the columns each)
  static constexpr int kTmemCols = 512;
  static constexpr int kElemsPerKB = 128;
  // barriers + bookkeeping after the stages
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256;
  static_assert(2 * BN <= kTmemCols, "TMEM budget");
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
};

struct Epi {
  float alpha;
  const float* alpha_dev;
  const float* row_scale;
  const float* col_scale;
  int col_scalar;
  const bf16* bias;
  int act;
  const bf16* residual;
  int64_t ldr;
  const bf16* gate;
  bf16* D;
  int64_t ldd;
  // NVFP4 re-quantization of the output for the next GEMM instead of the bf16 store (NVFP4 pair kernel only)
  uint8_t* q;              // [M, N/2] packed e2m1, element 2i in the low nibble
  uint8_t* q_sf;           // [pad128(M), N/16] ue4m3 block scales in 128x4 atoms
  const float* q_scale;    // device scalar: the fixed global scale s (blocks encoded under gs = 1/s)
};

struct Problem {
  int M, N, K;
  int m_blocks, n_blocks, k_blocks;
  int num_tiles;
  const uint8_t* sfa;  // NVFP4 scale atoms
  const uint8_t* sfb;
  int sfb_groups;      // 128-row groups present in the B scale buffer
};

__device__ __forceinline__ void tile_coords(int tile, const Problem& p, int& mb, int& nb) {
  constexpr int GN = 8;  // n-blocks per raster group: the group's B tiles stay in L2 while A streams
  const int per_group = p.m_blocks * GN;
  const int g = tile / per_group;
  const int in = tile - g * per_group;
  const int gn = min(GN, p.n_blocks - g * GN);
  mb = in / gn;
  nb = g * GN + (in - mb * gn);
}

__device__ __forceinline__ float gelu_tanh(float v) {
  float t;
  const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * v * (1.f + t);
}

// Epilogue of one accumulator row: this thread's TMEM lane (tbase = lane address + accumulator column) holds output
// row m, columns nb*BN .. nb*BN+BN-1; this call stores tile columns c_lo .. c_hi-1.
template <int BN>
__device__ __forceinline__ void store_rows(const Problem& p, const Epi& e, float alpha, uint32_t tbase, int m, int nb,
                                           int c_lo, int c_hi) {
  const bool row_ok = m < p.M;
  const float rs = alpha * ((e.row_scale && row_ok) ? e.row_scale[m] : 1.f);
#pragma unroll 1
  for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
    uint32_t r[32];
    tmem_ld_32cols(tbase + c0, r);
    tmem_ld_wait();
    const int n0 = nb * BN + c0;
    if (!row_ok || n0 >= p.N) continue;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int n = min(n0 + i, p.N - 1);
      float x = __uint_as_float(r[i]) * rs;
      if (e.col_scale) x *= e.col_scale[e.col_scalar ? 0 : n];
      if (e.bias) x += __bfloat162float(e.bias[n]);
      if (e.act == H3B_ACT_GELU_TANH) x = gelu_tanh(x);
      v[i] = x;
    }
    if (e.residual) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        const int n = n0 + i;
        if (n < p.N) {
          float res[8], g[8];
          load8(e.residual + (int64_t)m * e.ldr + n, res);
          load8(e.gate + n, g);
#pragma unroll
          for (int u = 0; u < 8; ++u) v[i + u] = res[u] + g[u] * v[i + u];
        }
      }
    }
    bf16* dst = e.D + (int64_t)m * e.ldd + n0;
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      if (n0 + i < p.N) {
        float w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) w[u] = v[i + u];
        store8(dst + i, w);
      }
    }
  }
}

// Epilogue of one warp's 32 accumulator rows (TMEM lanes 32q .. 32q+31), chunks c_begin .. c_end-1 of 32 columns,
// through shared memory and TMA: per chunk each lane turns its row into bf16 inside a 32 x 64-byte staging box
// (64-byte swizzle, so the 16-byte accesses of a quarter-warp hit distinct banks) and lane 0 writes the box with one
// tensor store (full sectors; rows >= M and columns >= N are clipped by the tensor map). With a gated residual the box
// is first filled with the residual's 32 x 32 block by a TMA load issued at the start of the chunk (completing on the
// box's mbarrier while the accumulator is read and scaled), so the residual is read with full-sector loads and updated
// in place. One box per warp: before it is refilled, the store that last read it has finished reading. `lphase` holds
// the parity of the box's load barrier.
// Per-chunk pieces of the epilogue. epi_issue_residual: with a gated residual, lane 0 puts the chunk's 32 x 32
// residual block in flight into the box (which the previous store has finished reading). epi_finish: scale, bias,
// activation and residual of the chunk's 32 raw accumulator words, bf16 into the box, one tensor store. Returns false
// when the residual block never arrived.
__device__ __forceinline__ void epi_issue_residual(const Epi& e, const CUtensorMap* tmR, uint8_t* box,
                                                   uint64_t* box_bar, int n0, int m0) {
  const int lane = threadIdx.x & 31;
  if (e.residual && lane == 0) {
    bulk_wait_read<0>();
    mbar_arrive_expect_tx(box_bar, 2048);
    tma_load_2d(box, tmR, n0, m0, box_bar);
  }
  __syncwarp();  // tcgen05.ld after this is warp-collective: reconverge after the lane-0 branch
}

__device__ __forceinline__ bool epi_finish(const Problem& p, const Epi& e, const CUtensorMap* tmD, float rs,
                                           const uint32_t (&r)[32], int n0, int m0, uint8_t* box, uint64_t* box_bar,
                                           uint32_t& lphase, volatile int* abort_flag) {
  const int lane = threadIdx.x & 31;
  const bool res = e.residual != nullptr;
  const int sw = (lane >> 1) & 3;
  uint8_t* row = box + lane * 64;
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int n = min(n0 + i, p.N - 1);
    float x = __uint_as_float(r[i]) * rs;
    if (e.col_scale) x *= e.col_scale[e.col_scalar ? 0 : n];
    if (e.bias) x += __bfloat162float(e.bias[n]);
    if (e.act == H3B_ACT_GELU_TANH) x = gelu_tanh(x);
    v[i] = x;
  }
  if (e.q) {
    // NVFP4 of the row's 32 values (two 16-element blocks) from their bf16 roundings -- the values a bf16 output
    // would hold -- under the fixed global factor gs = 1/s: the block math of the activation quantizers
    const int m = m0 + lane;
    const float gs = 1.f / *e.q_scale;
    uint32_t codes[4], bits[2];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      float vmax = 0.f;
#pragma unroll
      for (int i = 16 * b; i < 16 * b + 16; ++i) {
        v[i] = to_bf16_and_back(v[i]);
        vmax = fmaxf(vmax, fabsf(v[i]));
      }
      const float mult = nvfp4_block_scale(vmax, gs, &bits[b]);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float* u = v + 16 * b + 8 * j;
        codes[2 * b + j] = e2m1x4(u[0] * mult, u[1] * mult, u[2] * mult, u[3] * mult) |
                           (e2m1x4(u[4] * mult, u[5] * mult, u[6] * mult, u[7] * mult) << 16);
      }
    }
    if (m < p.M) {
      *reinterpret_cast<uint4*>(e.q + (size_t)m * (p.N / 2) + n0 / 2) = make_uint4(codes[0], codes[1], codes[2], codes[3]);
      *reinterpret_cast<uint16_t*>(e.q_sf + sf_atom_offset(m, n0 / 16, p.N / 16)) = (uint16_t)(bits[0] | (bits[1] << 8));
    }
    return true;
  }
  if (res) {
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(box_bar, lphase & 1u, abort_flag, kWaitLimitNs))) return false;
    lphase ^= 1u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 w = *reinterpret_cast<const uint4*>(row + ((j ^ sw) << 4));
      float rv[8], g[8];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 t = __bfloat1622float2(h[u]);
        rv[2 * u] = t.x;
        rv[2 * u + 1] = t.y;
      }
      load8(e.gate + min(n0 + 8 * j, p.N - 8), g);
#pragma unroll
      for (int u = 0; u < 8; ++u) v[8 * j + u] = rv[u] + g[u] * v[8 * j + u];
    }
  } else {
    // without a residual the box is first needed here: the previous store's read overlapped the accumulator read
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * j], v[8 * j + 1]);
    w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
    w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
    w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
    *reinterpret_cast<uint4*>(row + ((j ^ sw) << 4)) = w;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmD, n0, m0, box);
    bulk_commit_group();
  }
  return true;
}

__device__ __forceinline__ float epi_row_scale(const Problem& p, const Epi& e, float alpha, int m0) {
  const int m = m0 + (threadIdx.x & 31);
  return alpha * ((e.row_scale && m < p.M) ? e.row_scale[m] : 1.f);
}

// Epilogue of one warp's 32 accumulator rows (TMEM lanes 32q .. 32q+31), chunks c_begin .. c_end-1 of 32 columns,
// through shared memory and TMA: per chunk each lane turns its row into bf16 inside a 32 x 64-byte staging box
// (64-byte swizzle, so the 16-byte accesses of a quarter-warp hit distinct banks) and lane 0 writes the box with one
// tensor store (full sectors; rows >= M and columns >= N are clipped by the tensor map). With a gated residual the box
// is first filled with the residual's 32 x 32 block by a TMA load issued at the start of the chunk (completing on the
// box's mbarrier while the accumulator is read and scaled), so the residual is read with full-sector loads and updated
// in place. One box per warp: before it is refilled, the store that last read it has finished reading. `lphase` holds
// the parity of the box's load barrier.
template <int BN>
__device__ __forceinline__ void store_rows_tma(const Problem& p, const Epi& e, const CUtensorMap* tmD,
                                               const CUtensorMap* tmR, float alpha, uint32_t tbase, int m0, int nb,
                                               int c_begin, int c_end, uint8_t* box, uint64_t* box_bar,
                                               uint32_t& lphase, volatile int* abort_flag, bool& ok) {
  const float rs = epi_row_scale(p, e, alpha, m0);
#pragma unroll 1
  for (int c = c_begin; c < c_end; ++c) {
    const int n0 = nb * BN + 32 * c;
    if (m0 >= p.M || n0 >= p.N) break;  // warp-uniform: this and later chunks lie outside the output
    epi_issue_residual(e, tmR, box, box_bar, n0, m0);
    uint32_t r[32];
    tmem_ld_32cols(tbase + 32 * c, r);
    tmem_ld_wait();
    if (!epi_finish(p, e, tmD, rs, r, n0, m0, box, box_bar, lphase, abort_flag)) {
      ok = false;
      return;
    }
  }
}

// As store_rows_tma for NC chunks whose accumulator words the caller has already read into registers (so it could
// release the TMEM accumulator before the stores).
template <int BN, int NC>
__device__ __forceinline__ void store_rows_regs(const Problem& p, const Epi& e, const CUtensorMap* tmD,
                                                const CUtensorMap* tmR, float alpha, const uint32_t (&acc)[NC][32],
                                                int m0, int nb, int c_begin, uint8_t* box, uint64_t* box_bar,
                                                uint32_t& lphase, volatile int* abort_flag, bool& ok) {
  const float rs = epi_row_scale(p, e, alpha, m0);
#pragma unroll
  for (int cc = 0; cc < NC; ++cc) {
    const int n0 = nb * BN + 32 * (c_begin + cc);
    if (m0 >= p.M || n0 >= p.N) break;
    epi_issue_residual(e, tmR, box, box_bar, n0, m0);
    if (!epi_finish(p, e, tmD, rs, acc[cc], n0, m0, box, box_bar, lphase, abort_flag)) {
      ok = false;
      return;
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(Cfg8<BN>::kThreads, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Problem p,
                const Epi e) {
  using C = Cfg8<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;

  auto fail = [&]() {
    *abort_flag = 1;
    atomicExch(&g_gemm_status, H3B_ETIMEOUT);
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;  // loads armed but possibly not consumed, for the error-path drain
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, kWaitLimitNs)) {
            fail();
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * C::kStageBytes;
          uint8_t* sB = sA + C::kABytes;
          mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          tma_load_2d(sA, &tmA, kb * KB_BYTES, m0, &full[stage]);
          tma_load_2d(sB, &tmB, kb * KB_BYTES, n0, &full[stage]);
          issued = min(issued + 1, C::kStages);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // drain: every armed stage completes its transaction bytes once its copies land
        for (int i = 0; i < C::kStages; ++i) {
          int s = stage - 1 - i;
          uint32_t ph = phase;
          if (s < 0) {
            s += C::kStages;
            ph ^= 1;
          }
          if (i < issued) {
            volatile int no_abort = 0;
            mbar_wait_bounded(&full[s], ph, &no_abort, kWaitLimitNs / 4);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_e4m3(BN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      int j = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++j) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        const int buf = j & 1;
        if (!mbar_wait_bounded(&acc_empty[buf], (((acc_phase >> buf) & 1u) ^ 1u), abort_flag, kWaitLimitNs)) {
          fail();
          break;
        }
        acc_phase ^= 1u << buf;
        tc_fence_after();
        const uint32_t d = tmem + buf * C::kAccCols;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, kWaitLimitNs)) {
            fail();
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sA = smem + stage * C::kStageBytes;
          uint8_t* sB = sA + C::kABytes;
          const uint64_t da = desc_k_sw128(smem_addr(sA));
          const uint64_t db = desc_k_sw128(smem_addr(sB));
#pragma unroll
          for (int i = 0; i < 4; ++i) mma_e4m3(d, da + 2 * i, db + 2 * i, idesc, (kb | i) != 0);
          tc_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
      }
      // drain: wait until every MMA and copy issued above has finished before TMEM is freed
      tc_commit(drain);
      volatile int no_abort = 0;
      if (!mbar_wait_bounded(drain, 0, &no_abort, kWaitLimitNs)) fail();
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;         // TMEM lane quarter this warp may access
    const int half = warp < 6 ? 0 : 1;  // warps 2-5: tile columns 0 .. BN/2-1, warps 6-9: the rest
    const float alpha = e.alpha * (e.alpha_dev ? *e.alpha_dev : 1.f);
    uint32_t acc_phase = 0;
    int j = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++j) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int buf = j & 1;
      const bool got = mbar_wait_bounded(&acc_full[buf], ((acc_phase >> buf) & 1u), abort_flag, kWaitLimitNs);
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) fail();
        break;
      }
      acc_phase ^= 1u << buf;
      __syncwarp();
      tc_fence_after();
      store_rows<BN>(p, e, alpha, tmem + ((uint32_t)(q * 32) << 16) + buf * C::kAccCols, mb * BM + q * 32 + lane,
                     nb, half * (BN / 2), half * (BN / 2) + BN / 2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}


// ------------------------------------------------------------------------------------------------ NVFP4, CTA pairs
// 256 x 192 output tiles on a cluster of two CTAs (two SMs) with cta_group::2 MMAs: CTA r of the pair loads rows
// 128r .. 128r+127 of the A tile and rows 96r .. 96r+95 of the B tile, and holds output rows 128r .. 128r+127 in its
// TMEM; the even CTA issues every MMA (M = 256, N = 192) over both CTAs' shared memory. Per SM this halves the B
// bytes per MMA against a single-CTA 128 x 192 tile, and the smaller stage leaves room for six of them.
// Warps of each CTA (14):
//   warp 0    TMA producer: its A and B halves (cta_group::2 loads completing on the even CTA's stage barrier) and its
//             scale atoms (bulk copies completing on its own barrier)
//   warp 1    TMEM allocation (both CTAs); in the even CTA, lane 0 issues the MMAs
//   warps 2-5, 10-13 epilogue of this CTA's 128 rows (warp w reads TMEM lanes 32*(w%4) .. +31; warps 2-5 take
//             columns 0-95 of the tile, warps 10-13 columns 96-191), so a tile drains within the next tile's main loop
//   warps 6-9 scale factors: each warp writes the stage's scale atoms into its own 32 TMEM lanes with tcgen05.st (the
//             replicated image a 32x128b.warpx4 tcgen05.cp would produce) in a ring of TMEM slots, so the tensor
//             pipe runs MMAs only (a tcgen05.cp costs tensor-pipe time in proportion to the bytes it writes)
// Barriers the even CTA's MMA thread waits on live in the even CTA: one per stage, which completes when both CTAs'
// A/B halves have landed and the eight scale warps of the pair have written the stage's scale slot (one wait per
// stage keeps the issuing thread's gaps between MMAs short), and one per accumulator, drained by both epilogues. The
// odd CTA's producer, scale warps and epilogue reach them through shared::cluster addresses. Each producer issues its
// scale copies before its A/B copies, so the scale warps' TMEM writes are not queued behind 28 KB of operand tiles.
#ifndef H3B_PAIR_ACC_BUFS
#define H3B_PAIR_ACC_BUFS 2
#endif
#ifndef H3B_PAIR_KSTAGE
#define H3B_PAIR_KSTAGE 1
#endif
struct PairCfg {
  static constexpr int BN = 192;         // N of one MMA / output tile
  static constexpr int kBRows = BN / 2;  // B rows each CTA loads
  static constexpr int KS = H3B_PAIR_KSTAGE;  // 256-deep K blocks per stage
  static constexpr int kStages = KS == 1 ? 6 : 3;
  static constexpr int kAKb = BM * KB_BYTES;          // one K block of A (128 rows x 128 bytes)
  static constexpr int kBKb = kBRows * KB_BYTES;      // one K block of this CTA's B rows
  static constexpr int kABytes = KS * kAKb;
  static constexpr int kBBytes = KS * kBKb;
  static constexpr int kSfaBytes = KS * 2048;         // four 512-byte atoms per K block
  static constexpr int kSfbBytes = KS * 4096;         // the same for two 128-row groups of B
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  // Accumulator buffers and scale slots in TMEM. Two accumulators let a tile's epilogue overlap the next tile's
  // MMAs, but leave room for three scale slots only, so a stage's scales can be written only once the MMAs of the
  // stage three back have completed; with one accumulator there is a slot per stage (the scale writes then wait
  // on the same completions as the producer) and the epilogue reads the accumulator into registers and releases it
  // before its stores. A scales take 16 columns (4 K blocks x 4), the B scales of the tile's 192 rows 24 (4 K blocks
  // x 6, row 32c + r of the tile in column c, lane r).
  static constexpr int kAccBufs = H3B_PAIR_ACC_BUFS;
  static constexpr int kSfCol = kAccBufs * BN;
  static constexpr int kSfSlotCols = 40 * KS;
  static constexpr int kSfSlots = kAccBufs == 1 ? kStages : 3;
  static_assert(KS == 1 || kAccBufs == 1, "two K blocks per stage leave TMEM for one accumulator only");
  static constexpr int kThreads = 448;
  static constexpr int kTmemCols = 512;
  static constexpr int kEpiWarps = 8;                 // two per TMEM lane quarter, each on half of the columns
  static constexpr int kEpiBytes = kEpiWarps * 2048;  // per epilogue warp one 32 x 64-byte output staging box
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 /*align*/ + 512;
  static_assert(kAccBufs * BN + kSfSlotCols * kSfSlots <= kTmemCols, "TMEM budget");
  static_assert(kSfCol % 8 == 0 && kSfSlotCols % 8 == 0, "scale slots are written 8 columns at a time");
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
};

__global__ void __launch_bounds__(PairCfg::kThreads, 1)
    gemm_nvfp4_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmR,
                           const Problem p, const Epi e) {
  using C = PairCfg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_boxes = smem + C::kStages * C::kStageBytes;
  // [stage] even CTA: A/B halves landed (transaction bytes) and the eight scale warps wrote the stage's slot
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_boxes + C::kEpiBytes);
  // [stage] the MMAs reading the stage have completed: one commit per stage into the even CTA's barrier; an even-CTA
  // scale warp relays each completion to the odd CTA's barrier
  uint64_t* empty = full + C::kStages;
  uint64_t* sf_loaded = empty + C::kStages;         // [stage] this CTA's scale atoms landed
  uint64_t* acc_full = sf_loaded + C::kStages;      // [buffer] the tile's MMAs have completed
  uint64_t* acc_empty = acc_full + 2;               // [buffer] even CTA: both epilogues drained the accumulator
  uint64_t* drain = acc_empty + 2;
  uint64_t* box_bar = drain + 1;                    // [epilogue warp] residual block landed in its box
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(box_bar + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  // shared::cluster address of a barrier of this CTA's layout, in CTA r of the pair
  auto in_cta = [&](uint64_t* bar, uint32_t r) { return map_to_cta(smem_addr(bar), r); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1 + 8);  // the even producer's arrive.expect_tx + 4 scale warps x 2 CTAs
      mbar_init(&empty[s], 1);
      mbar_init(&sf_loaded[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * C::kEpiWarps);  // epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 8; ++i) mbar_init(&box_bar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmD);
    if (e.residual) prefetch_tmap(&tmR);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_slot, C::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers are initialised before either CTA signals into the other
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;

  auto fail = [&]() {
    *abort_flag = 1;
    atomicExch(&g_gemm_status, H3B_ETIMEOUT);
  };
  const int m_blocks2 = (p.m_blocks + 1) >> 1;
  const int ksteps = (p.k_blocks + C::KS - 1) / C::KS;  // stages per tile
  Problem pp = p;  // tile raster over 256-row blocks
  pp.m_blocks = m_blocks2;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer (each CTA loads its halves)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      const size_t kstride = (size_t)(p.K / 64) * 512;  // scale bytes per 128-row group
      for (int tile = cluster; tile < p.num_tiles && ok; tile += clusters) {
        int mb2, nb;
        tile_coords(tile, pp, mb2, nb);
        const int mblk = 2 * mb2 + (int)rank;
        const int n0 = nb * C::BN;
        const uint8_t* sfa_src = p.sfa + (size_t)min(mblk, p.m_blocks - 1) * kstride;
        const int g0 = n0 >> 7;
        const int g1 = min(g0 + 1, p.sfb_groups - 1);
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, kWaitLimitNs)) {
            fail();
            ok = false;
            break;
          }
          const int kb0 = ks * C::KS, nk = min(C::KS, p.k_blocks - kb0);
          uint8_t* sA = smem + stage * C::kStageBytes;
          uint8_t* sB = sA + C::kABytes;
          uint8_t* sSFA = sB + C::kBBytes;
          uint8_t* sSFB = sSFA + C::kSfaBytes;
          const uint32_t full0 = in_cta(&full[stage], 0);
          const uint32_t sf_bytes = (uint32_t)nk * 2048;
          mbar_arrive_expect_tx(&sf_loaded[stage], 3 * sf_bytes);
          bulk_load(sSFA, sfa_src + (size_t)kb0 * 2048, sf_bytes, &sf_loaded[stage]);
          bulk_load(sSFB, p.sfb + (size_t)g0 * kstride + (size_t)kb0 * 2048, sf_bytes, &sf_loaded[stage]);
          bulk_load(sSFB + C::kSfbBytes / 2, p.sfb + (size_t)g1 * kstride + (size_t)kb0 * 2048, sf_bytes,
                    &sf_loaded[stage]);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * nk * (C::kAKb + C::kBKb));
          for (int h = 0; h < nk; ++h) {
            tma_load_2d_pair(sA + h * C::kAKb, &tmA, (kb0 + h) * KB_BYTES, mblk * BM, full0);
            tma_load_2d_pair(sB + h * C::kBKb, &tmB, (kb0 + h) * KB_BYTES, n0 + (int)rank * C::kBRows, full0);
          }
          issued = min(issued + 1, C::kStages);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // drain this CTA's scale copies (its A/B copies complete on the even CTA's barrier, drained there)
        for (int i = 0; i < C::kStages; ++i) {
          int s = stage - 1 - i;
          uint32_t ph = phase;
          if (s < 0) {
            s += C::kStages;
            ph ^= 1;
          }
          if (i < issued) {
            volatile int no_abort = 0;
            mbar_wait_bounded(&sf_loaded[s], ph, &no_abort, kWaitLimitNs / 4);
            // the stage barrier also counts scale-warp arrivals that an aborting pair may never make; its bound (far
            // above the latency of a copy) ends the wait then
            if (rank == 0) mbar_wait_bounded(&full[s], ph, &no_abort, kWaitLimitNs / 64);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA, one thread)
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = idesc_nvf4_m256(C::BN);
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0, sf_n = 0;
      int j = 0;
      bool ok = true;
      for (int tile = cluster; tile < p.num_tiles && ok; tile += clusters, ++j) {
        int mb2, nb;
        tile_coords(tile, pp, mb2, nb);
        const int buf = j % C::kAccBufs;
        if (!mbar_wait_spin(&acc_empty[buf], (((acc_phase >> buf) & 1u) ^ 1u), abort_flag, kWaitLimitNs)) {
          fail();
          break;
        }
        acc_phase ^= 1u << buf;
        tc_fence_after();
        const uint32_t d = tmem + buf * C::BN;
        for (int ks = 0; ks < ksteps; ++ks) {
          const int slot = (int)(sf_n % C::kSfSlots);
          const int nk = min(C::KS, p.k_blocks - ks * C::KS);
          if (!mbar_wait_spin(&full[stage], phase, abort_flag, kWaitLimitNs)) {
            fail();
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sA = smem + stage * C::kStageBytes;
          const uint32_t sfa = tmem + C::kSfCol + C::kSfSlotCols * slot, sfb = sfa + 16 * C::KS;
#pragma unroll
          for (int h = 0; h < C::KS; ++h) {
            if (h < nk) {
              const uint64_t da = desc_k_sw128(smem_addr(sA + h * C::kAKb));
              const uint64_t db = desc_k_sw128(smem_addr(sA + C::kABytes + h * C::kBKb));
#pragma unroll
              for (int i = 0; i < 4; ++i)
                mma_nvf4_pair(d, da + 2 * i, db + 2 * i, idesc, (ks | h | i) != 0, sfa + 4 * (4 * h + i),
                              sfb + 6 * (4 * h + i));
            }
          }
          tc_commit_pair(smem_addr(&empty[stage]));  // one commit per stage: each extra one costs tensor-pipe time
          ++sf_n;
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair(in_cta(&acc_full[buf], 0));
        tc_commit_pair(in_cta(&acc_full[buf], 1));
      }
      tc_commit_pair(in_cta(drain, 0));
      volatile int no_abort = 0;
      if (!mbar_wait_spin(drain, 0, &no_abort, kWaitLimitNs)) fail();
    }
  } else if (warp >= 6 && warp < 10) {
    // ------------------------------------------------------------------ scale factors into this CTA's TMEM
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    int stage = 0;
    uint32_t phase = 0, sf_n = 0;
    bool ok = true;
    for (int tile = cluster; tile < p.num_tiles && ok; tile += clusters) {
      int mb2, nb;
      tile_coords(tile, pp, mb2, nb);
      // the tile's 192 B rows start at word 0 or 2 (rows 0 or 64 of a 128-row group) of the first group's atoms
      const bool mid = ((nb * C::BN) & 127) != 0;
      for (int ks = 0; ks < ksteps; ++ks) {
        const int slot = (int)(sf_n % C::kSfSlots);
        // the stage's atoms are read into registers first, so the slot wait (MMA completion) is followed only by
        // the TMEM stores
        if (!__all_sync(0xffffffffu, mbar_wait_spin(&sf_loaded[stage], phase, abort_flag, kWaitLimitNs))) {
          if (lane == 0) fail();
          ok = false;
          break;
        }
        const uint8_t* sSFA = smem + stage * C::kStageBytes + C::kABytes + C::kBBytes;
        const uint8_t* sSFB = sSFA + C::kSfaBytes;
        // (a tail stage with fewer K blocks writes its unused columns from stale atoms; no MMA reads them)
        uint32_t a[16 * C::KS], b[24 * C::KS];
#pragma unroll
        for (int i = 0; i < 4 * C::KS; ++i) {
          const uint4 x = *reinterpret_cast<const uint4*>(sSFA + 512 * i + 16 * lane);
          const uint4 y = *reinterpret_cast<const uint4*>(sSFB + 512 * i + 16 * lane);
          const uint4 z = *reinterpret_cast<const uint4*>(sSFB + C::kSfbBytes / 2 + 512 * i + 16 * lane);
          a[4 * i] = x.x, a[4 * i + 1] = x.y, a[4 * i + 2] = x.z, a[4 * i + 3] = x.w;
          // words w0 .. w0+5 of (first group's atom, second group's atom)
          b[6 * i] = mid ? y.z : y.x;
          b[6 * i + 1] = mid ? y.w : y.y;
          b[6 * i + 2] = mid ? z.x : y.z;
          b[6 * i + 3] = mid ? z.y : y.w;
          b[6 * i + 4] = mid ? z.z : z.x;
          b[6 * i + 5] = mid ? z.w : z.y;
        }
        // the slot was last read by the MMAs of stage sf_n - kSfSlots: wait for their completion (and, in the even
        // CTA, pass it on to the odd CTA's barrier of that stage for its producer and scale warps)
        if (sf_n >= C::kSfSlots) {
          const uint32_t prev = sf_n - C::kSfSlots;
          const int ps = (int)(prev % C::kStages);
          if (!__all_sync(0xffffffffu,
                          mbar_wait_spin(&empty[ps], (prev / C::kStages) & 1u, abort_flag, kWaitLimitNs))) {
            if (lane == 0) fail();
            ok = false;
            break;
          }
          if (rank == 0 && warp == 6 && lane == 0) mbar_arrive_cluster(in_cta(&empty[ps], 1));
        }
        tc_fence_after();
        const uint32_t sfa = tmem + lane_off + C::kSfCol + C::kSfSlotCols * slot;
#pragma unroll
        for (int c = 0; c < 2 * C::KS; ++c) tmem_st_8cols(sfa + 8 * c, a + 8 * c);
#pragma unroll
        for (int c = 0; c < 3 * C::KS; ++c) tmem_st_8cols(sfa + 16 * C::KS + 8 * c, b + 8 * c);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(in_cta(&full[stage], 0));
        ++sf_n;
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (this CTA's 128 rows)
    const int q = warp & 3;
    const float alpha = e.alpha * (e.alpha_dev ? *e.alpha_dev : 1.f);
    const int ew = warp < 6 ? warp - 2 : warp - 6;  // epilogue warp 0..7
    const int half = warp < 6 ? 0 : 1;              // columns 0-95 or 96-191 of the tile
    uint8_t* box = epi_boxes + ew * 2048;
    uint32_t acc_phase = 0, lphase = 0;
    bool ok = true;
    int j = 0;
    for (int tile = cluster; tile < p.num_tiles; tile += clusters, ++j) {
      int mb2, nb;
      tile_coords(tile, pp, mb2, nb);
      const int buf = j % C::kAccBufs;
      const bool got = mbar_wait_bounded(&acc_full[buf], ((acc_phase >> buf) & 1u), abort_flag, kWaitLimitNs);
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) fail();
        break;
      }
      acc_phase ^= 1u << buf;
      __syncwarp();
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * C::BN;
      const int m0 = (2 * mb2 + (int)rank) * BM + q * 32;
      if constexpr (C::kAccBufs == 1) {
        // read this warp's 96 columns, release the accumulator to the next tile's MMAs, then scale and store
        uint32_t acc[3][32];
#pragma unroll
        for (int cc = 0; cc < 3; ++cc) tmem_ld_32cols(tbase + 32 * (3 * half + cc), acc[cc]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(in_cta(&acc_empty[buf], 0));
        store_rows_regs<C::BN, 3>(p, e, &tmD, &tmR, alpha, acc, m0, nb, 3 * half, box, box_bar + ew, lphase,
                                  abort_flag, ok);
        if (!ok) {
          if (lane == 0) fail();
          break;
        }
      } else {
        store_rows_tma<C::BN>(p, e, &tmD, &tmR, alpha, tbase, m0, nb, 3 * half, 3 * half + 3, box, box_bar + ew,
                              lphase, abort_flag, ok);
        if (!ok) {
          if (lane == 0) fail();
          break;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(in_cta(&acc_empty[buf], 0));
      }
    }
    if (lane == 0) bulk_wait_all();  // the output stores have completed before the CTA exits
  }

  tc_fence_before();
  cluster_sync_all();  // nothing signals into either CTA after this point
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------ host side
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

// Row-major byte matrix [rows, cols_bytes] as a 2D tensor map with box {128 bytes, box_rows}, 128-byte swizzle.
int make_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols_bytes, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols_bytes};
  cuuint32_t box[2] = {(cuuint32_t)KB_BYTES, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return H3B_OK;
}

// Output matrix bf16 [rows, cols] with row stride ld elements as a 2D tensor map with a 32 x 32 box (64-byte rows,
// 64-byte swizzle): the epilogue's staging box.
int make_tmap_out(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld) {
  auto fn = encode_fn();
  if (!fn) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return H3B_OK;
}

int num_sms() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

template <int BN>
int run_gemm_fp8(const void* A, const void* B, int64_t M, int64_t N, int64_t K, const h3b_epilogue* epi,
                 cudaStream_t stream) {
  using C = Cfg8<BN>;
  const int64_t kbytes = K;
  CUtensorMap ta, tb;
  int rc = make_tmap(&ta, A, M, kbytes, BM);
  if (rc) return rc;
  rc = make_tmap(&tb, B, N, kbytes, BN);
  if (rc) return rc;
  Problem p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.m_blocks = (int)((M + BM - 1) / BM);
  p.n_blocks = (int)((N + BN - 1) / BN);
  p.k_blocks = (int)(K / C::kElemsPerKB);
  p.num_tiles = p.m_blocks * p.n_blocks;
  p.sfa = nullptr;
  p.sfb = nullptr;
  p.sfb_groups = 0;
  Epi e{epi->alpha,
        epi->alpha_dev,
        epi->row_scale,
        epi->col_scale,
        epi->col_scale_scalar,
        static_cast<const bf16*>(epi->bias),
        epi->act,
        static_cast<const bf16*>(epi->residual),
        epi->ldr,
        static_cast<const bf16*>(epi->gate),
        static_cast<bf16*>(epi->D),
        epi->ldd};
  auto kern = gemm_fp8_kernel<BN>;
  static PerDevice setup;  // the shared-memory reservation, per device; the value is the SM count
  int sms = 0;
  if (int rc = setup.get([&](int* v) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) != cudaSuccess)
          return set_error(H3B_ECUDA, "gemm: cannot reserve %d bytes of shared memory", C::kSmemBytes);
        *v = num_sms();
        return H3B_OK;
      }, &sms))
    return rc;
  const int grid = std::min(p.num_tiles, sms);
  kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(ta, tb, p, e);
  H3B_LAUNCH_CHECK("gemm");
  return H3B_OK;
}

int run_gemm_nvfp4_pair(const void* A, const uint8_t* sfa, const void* B, const uint8_t* sfb, int64_t M, int64_t N,
                        int64_t K, const h3b_epilogue* epi, uint8_t* q, uint8_t* q_sf, const float* q_scale,
                        cudaStream_t stream) {
  using C = PairCfg;
  CUtensorMap ta, tb;
  int rc = make_tmap(&ta, A, M, K / 2, BM);
  if (rc) return rc;
  rc = make_tmap(&tb, B, N, K / 2, C::kBRows);
  if (rc) return rc;
  CUtensorMap td, tr;
  // with re-quantization the output maps are unused: they are built over the code buffer (as bf16 [M, N/4])
  void* dbase = q ? static_cast<void*>(q) : epi->D;
  const int64_t dcols = q ? N / 4 : N, dld = q ? N / 4 : epi->ldd;
  rc = make_tmap_out(&td, dbase, M, dcols, dld);
  if (rc) return rc;
  rc = epi->residual ? make_tmap_out(&tr, epi->residual, M, N, epi->ldr) : make_tmap_out(&tr, dbase, M, dcols, dld);
  if (rc) return rc;
  Problem p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.m_blocks = (int)((M + BM - 1) / BM);
  p.n_blocks = (int)((N + C::BN - 1) / C::BN);
  p.k_blocks = (int)(K / 256);
  p.num_tiles = ((p.m_blocks + 1) / 2) * p.n_blocks;  // 256-row x 192-column tiles
  p.sfa = sfa;
  p.sfb = sfb;
  p.sfb_groups = (int)((N + 127) / 128);
  Epi e{epi->alpha,
        epi->alpha_dev,
        epi->row_scale,
        epi->col_scale,
        epi->col_scale_scalar,
        static_cast<const bf16*>(epi->bias),
        epi->act,
        static_cast<const bf16*>(epi->residual),
        epi->ldr,
        static_cast<const bf16*>(epi->gate),
        static_cast<bf16*>(epi->D),
        epi->ldd,
        q,
        q_sf,
        q_scale};
  auto kern = gemm_nvfp4_pair_kernel;
  static PerDevice setup;  // the shared-memory reservation and the resident CTA pairs, per device
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int max_clusters = 0;
  if (int rc = setup.get([&](int* v) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) != cudaSuccess)
          return set_error(H3B_ECUDA, "gemm: cannot reserve %d bytes of shared memory", C::kSmemBytes);
        cfg.gridDim = dim3(2 * (num_sms() / 2));
        if (cudaOccupancyMaxActiveClusters(v, kern, &cfg) != cudaSuccess || *v <= 0)
          return set_error(H3B_ECUDA, "gemm: no CTA pair of %d bytes of shared memory fits", C::kSmemBytes);
        return H3B_OK;
      }, &max_clusters))
    return rc;
  cfg.gridDim = dim3(2 * std::min(p.num_tiles, max_clusters));
  const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, ta, tb, td, tr, p, e);
  if (le != cudaSuccess) {
    cudaGetLastError();
    return set_error(H3B_ECUDA, "gemm: CTA-pair launch failed: %s", cudaGetErrorString(le));
  }
  H3B_LAUNCH_CHECK("gemm");
  return H3B_OK;
}

int check_epilogue(const h3b_epilogue* epi, int64_t N) {
  H3B_REQUIRE(epi && epi->D, "gemm: epilogue and its output D are required");
  H3B_REQUIRE(epi->ldd >= N && epi->ldd % 8 == 0 && aligned(epi->D, 16), "gemm: ldd >= N, multiple of 8, D 16-byte aligned");
  H3B_REQUIRE(epi->act == H3B_ACT_NONE || epi->act == H3B_ACT_GELU_TANH, "gemm: act %d", epi->act);
  H3B_REQUIRE(!epi->residual || (epi->gate && epi->ldr >= N && epi->ldr % 8 == 0 && aligned(epi->residual, 16) &&
                                 aligned(epi->gate, 16)),
              "gemm: residual needs gate, ldr >= N (multiple of 8) and 16-byte alignment");
  return H3B_OK;
}

}  // namespace
}  // namespace h3b

using namespace h3b;

extern "C" int h3b_gemm_fp8(const void* A, const void* B, int64_t M, int64_t N, int64_t K, const h3b_epilogue* epi,
                            cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(A && B, "gemm_fp8: null operand");
  H3B_REQUIRE(K > 0 && K % 128 == 0, "gemm_fp8: K must be a positive multiple of 128 (got %lld)", (long long)K);
  H3B_REQUIRE(N > 0 && N % 16 == 0 && M >= 0, "gemm_fp8: N must be a positive multiple of 16");
  H3B_REQUIRE(aligned(A, 16) && aligned(B, 16), "gemm_fp8: A and B must be 16-byte aligned");
  if (int rc = check_epilogue(epi, N)) return rc;
  if (M == 0) return H3B_OK;
  return run_gemm_fp8<256>(A, B, M, N, K, epi, stream);
}

extern "C" int h3b_gemm_nvfp4(const void* A, const uint8_t* sfa, const void* B, const uint8_t* sfb, int64_t M,
                              int64_t N, int64_t K, const h3b_epilogue* epi, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(A && B && sfa && sfb, "gemm_nvfp4: null operand");
  H3B_REQUIRE(K > 0 && K % 256 == 0, "gemm_nvfp4: K must be a positive multiple of 256 (got %lld)", (long long)K);
  H3B_REQUIRE(N > 0 && N % 16 == 0 && M >= 0, "gemm_nvfp4: N must be a positive multiple of 16");
  H3B_REQUIRE(aligned(A, 16) && aligned(B, 16) && aligned(sfa, 16) && aligned(sfb, 16),
              "gemm_nvfp4: operands and scales must be 16-byte aligned");
  if (int rc = check_epilogue(epi, N)) return rc;
  if (M == 0) return H3B_OK;
  return run_gemm_nvfp4_pair(A, sfa, B, sfb, M, N, K, epi, nullptr, nullptr, nullptr, stream);
}

extern "C" int h3b_gemm_nvfp4_requant(const void* A, const uint8_t* sfa, const void* B, const uint8_t* sfb,
                                      int64_t M, int64_t N, int64_t K, const h3b_epilogue* epi, uint8_t* q,
                                      uint8_t* q_sf, const float* q_scale, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(A && B && sfa && sfb, "gemm_nvfp4_requant: null operand");
  H3B_REQUIRE(K > 0 && K % 256 == 0, "gemm_nvfp4_requant: K must be a positive multiple of 256 (got %lld)",
              (long long)K);
  H3B_REQUIRE(N > 0 && N % 32 == 0 && M >= 0, "gemm_nvfp4_requant: N must be a positive multiple of 32");
  H3B_REQUIRE(aligned(A, 16) && aligned(B, 16) && aligned(sfa, 16) && aligned(sfb, 16),
              "gemm_nvfp4_requant: operands and scales must be 16-byte aligned");
  H3B_REQUIRE(epi && !epi->D && !epi->residual,
              "gemm_nvfp4_requant: the epilogue writes q/q_sf only (D and residual must be NULL)");
  H3B_REQUIRE(epi->act == H3B_ACT_NONE || epi->act == H3B_ACT_GELU_TANH, "gemm_nvfp4_requant: act %d", epi->act);
  H3B_REQUIRE(q && q_sf && q_scale && aligned(q, 16) && aligned(q_sf, 2),
              "gemm_nvfp4_requant: q (16-byte aligned), q_sf and q_scale are required");
  if (M == 0) return H3B_OK;
  return run_gemm_nvfp4_pair(A, sfa, B, sfb, M, N, K, epi, q, q_sf, q_scale, stream);
}

namespace h3b {
namespace {
// Self-test of the bounded-wait path: one warp waits on an mbarrier that nothing arrives on, with the wait helper the
// kernels use; when the limit expires it records H3B_ETIMEOUT in the device status word and returns.
__global__ void selftest_wait_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  volatile int no_abort = 0;
  const bool got = mbar_wait_bounded(&bar, 0, &no_abort, limit_ns);
  if (!__all_sync(0xffffffffu, got) && threadIdx.x == 0) atomicExch(&g_gemm_status, H3B_ETIMEOUT);
}
}  // namespace
}  // namespace h3b

extern "C" int h3b_selftest_wait_timeout(uint64_t limit_ns, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(limit_ns > 0 && limit_ns <= 2000000000ull, "selftest_wait_timeout: limit must be in (0, 2 s]");
  selftest_wait_kernel<<<1, 32, 0, stream>>>(limit_ns);
  H3B_LAUNCH_CHECK("selftest_wait_timeout");
  return H3B_OK;
}

namespace h3b {
int gemm_status_async(int* dst, int clear, cudaStream_t stream) {
  if (cudaMemcpyFromSymbolAsync(dst, g_gemm_status, sizeof(int), 0, cudaMemcpyDefault, stream) != cudaSuccess)
    return set_error(H3B_ECUDA, "status: reading the GEMM status word failed");
  if (clear) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_status) != cudaSuccess || cudaMemsetAsync(p, 0, sizeof(int), stream) != cudaSuccess)
      return set_error(H3B_ECUDA, "status: clearing the GEMM status word failed");
  }
  return H3B_OK;
}
}  // namespace h3b

extern "C" int h3b_device_status(int* status) {
  clear_error();
  H3B_REQUIRE(status, "device_status: null pointer");
  if (cudaMemcpyFromSymbol(status, g_gemm_status, sizeof(int)) != cudaSuccess)
    return set_error(H3B_ECUDA, "device_status: read failed");
  return H3B_OK;
}

extern "C" int h3b_reset_device_status(void) {
  clear_error();
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int)) != cudaSuccess)
    return set_error(H3B_ECUDA, "reset_device_status: write failed");
  return H3B_OK;
}
