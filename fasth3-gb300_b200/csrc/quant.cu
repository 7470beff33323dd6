// Activation quantizers of the DiT block: gated residual + RMSNorm/LayerNorm + adaLN modulate + FP8/NVFP4 row
// quantization, the plain per-token FP8 quantizer, and the per-tensor NVFP4 quantizer.
//
// Built with --use_fast_math like the reference extension (fastvideo/models/dits/h3fast/__init__.py:42), and every
// per-element expression below is written in the same operand order as the reference kernel
// (fastvideo/models/dits/h3fast/h3fast.cu:188-265): with the same flags the compiler emits the same approximate
// reciprocal, rsqrt and contractions, which is what makes the quantized bytes bit-identical to the reference's.
// The RMSNorm row sum of squares uses the reference's reduction tree (8 contiguous elements per thread summed in order,
// warp butterfly, warp partials butterflied again), so its rounding is the same too. The LayerNorm variant has no
// reference counterpart; its summation order is defined below and restated by the oracle.
#include "common.cuh"
#include "sm100.cuh"

#include <algorithm>

namespace h3b {
namespace {

struct RowArgs {
  const bf16* x;
  const bf16* y;
  const float* sy;
  const bf16* gate;
  int64_t gate_ld;
  const int32_t* idx;
  const bf16* nw;
  const bf16* shift;
  const bf16* scale;
  int64_t tab_ld;
  bf16* xo;
  uint8_t* h;
  uint8_t* hsf;
  float* hs;
  float eps;
  int64_t rows;
};

// Persistent CTAs of C/8 threads, thread t owns elements [8t, 8t+8) of a row; a CTA walks rows r, r + grid, ... and
// loads the next row while it reduces and quantizes the current one (the per-row arithmetic is unchanged).
template <int C, bool BRANCH, int NORM, bool FP4>
__global__ void __launch_bounds__(C / 8, 2) resid_norm_quant_kernel(const RowArgs a) {
  constexpr int NW = C / 8 / 32;
  __shared__ float stage[32];
  const int t = threadIdx.x;
  int64_t r = blockIdx.x;
  if (r >= a.rows) return;
  uint4 vn = ld8_raw(a.x + r * C + t * 8), bn = make_uint4(0u, 0u, 0u, 0u);
  if constexpr (BRANCH) bn = ld8_raw(a.y + r * C + t * 8);
  for (; r < a.rows; r += gridDim.x) {
    const int64_t tab = a.idx ? (int64_t)a.idx[r] : 0;
    float v[8], b[8];
    unpack8(vn, v);
    if constexpr (BRANCH) unpack8(bn, b);
    const int64_t rn = r + gridDim.x;
    if (rn < a.rows) {
      vn = ld8_raw(a.x + rn * C + t * 8);
      if constexpr (BRANCH) bn = ld8_raw(a.y + rn * C + t * 8);
    }
    if constexpr (BRANCH) {
      float g[8];
      load8(a.gate + tab * a.gate_ld + t * 8, g);
      const float s = a.sy[r];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = to_bf16_and_back(v[i] + g[i] * (s * b[i]));
      store8(a.xo + r * C + t * 8, v);
    }
    if constexpr (NORM != H3B_NORM_NONE) {
      float sc[8], sf[8];
      load8(a.scale + tab * a.tab_ld + t * 8, sc);
      load8(a.shift + tab * a.tab_ld + t * 8, sf);
      float am = 0.f;
      if constexpr (NORM == H3B_NORM_RMS) {
        float wv[8];
        load8(a.nw + t * 8, wv);
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
        ss = block_allreduce<NW, false>(ss, stage);
        const float rs = rsqrtf(ss / C + a.eps);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[i] = v[i] * rs * wv[i] * (1.f + sc[i]) + sf[i];
          am = fmaxf(am, fabsf(v[i]));
        }
      } else {  // LayerNorm without affine parameters, two passes over the registers
        float s1 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) s1 += v[i];
        const float mean = block_allreduce<NW, false>(s1, stage) / C;
        float s2 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[i] -= mean;
          s2 += v[i] * v[i];
        }
        const float rs = rsqrtf(block_allreduce<NW, false>(s2, stage) / C + a.eps);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[i] = v[i] * rs * (1.f + sc[i]) + sf[i];
          am = fmaxf(am, fabsf(v[i]));
        }
      }
      am = block_allreduce<NW, true>(am, stage);
      if constexpr (FP4) {
        const float s = fmaxf(am / kFp4Range, kMinScaleFp4);
        const float gs = 1.f / s;
        // a 16-element block spans lanes t and t^1
        float vmax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) vmax = fmaxf(vmax, fabsf(v[i]));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
        uint32_t bits;
        const float m = nvfp4_block_scale(vmax, gs, &bits);
        const uint32_t lo = e2m1x4(v[0] * m, v[1] * m, v[2] * m, v[3] * m);
        const uint32_t hi = e2m1x4(v[4] * m, v[5] * m, v[6] * m, v[7] * m);
        *reinterpret_cast<uint32_t*>(a.h + r * (C / 2) + t * 4) = lo | (hi << 16);
        if ((t & 1) == 0) a.hsf[sf_atom_offset(r, t >> 1, C / 16)] = (uint8_t)bits;
        if (t == 0) a.hs[r] = s;
      } else {
        const float s = fmaxf(am / kFp8Max, kMinScaleFp8);
        const float inv = 1.f / s;
        uint2 o;
        o.x = e4m3x4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv);
        o.y = e4m3x4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv);
        *reinterpret_cast<uint2*>(a.h + r * C + t * 8) = o;
        if (t == 0) a.hs[r] = s;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------ LayerNorm
// The LayerNorm variant (no reference counterpart: the DiT block's norm1/norm2 with the adaLN modulate, and the affine
// norm3 given as a table) has one summation order for every kernel below, defined by a thread layout: a row of
// C = 8 K G elements is shared by G threads (a whole number of warps), thread t owning the 8-element chunks
// t, t + G, ..., t + (K - 1) G, with K the largest of 5, 4, 3, 2 that gives whole warps (else 1). A thread sums its
// values with two float32 accumulators (even and odd elements of each chunk, chunk by chunk), adds the two, the warp
// butterflies the thread sums, and the warp sums are added in warp order. The sum of squares of (x - mean) is formed
// the same way with one fused multiply-add per element.
template <int C>
struct LnRowShape {
  static constexpr int kChunks = C / 8;
  static constexpr int pick() {
    for (int k = 5; k > 1; --k)
      if (kChunks % k == 0 && (kChunks / k) % 32 == 0) return k;
    return 1;
  }
  static constexpr int K = pick();
  static constexpr int G = kChunks / K;
  static constexpr int NW = G / 32;
  static_assert(G % 32 == 0, "the LayerNorm row layout needs whole warps");
};

// one thread's share of the row sum from its chunks' values v[8 K]: the pair accumulators, then their sum
template <int E>
__device__ __forceinline__ float ln_thread_sum(const float (&v)[E]) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < E; i += 2) add2(s0, s1, v[i], v[i + 1]);
  return s0 + s1;
}
template <int E>
__device__ __forceinline__ float ln_thread_sumsq(const float (&d)[E]) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < E; i += 2) sq_acc2(s0, s1, d[i], d[i + 1]);
  return s0 + s1;
}

__device__ int g_rows_status = 0;
constexpr uint64_t kRowWaitLimitNs = 1000000000ull;

// Row-per-CTA LayerNorm quantizer for the common case of one modulation row for all tokens (or a per-token table row
// given by idx) and no residual branch. G threads per CTA walk rows r, r + grid, ...; thread 0 keeps kLnStages rows
// in flight as 1D bulk copies into a ring of shared-memory row buffers (mbarrier completion), so the loads need no
// registers and many rows are in flight per SM. A thread reads its chunks once into registers and keeps them there
// through both statistics, the modulate and the quantization; the modulate factors (1 + scale, shift) of its columns
// stay in registers for the whole launch when the table row is shared. Three CTA reductions per row (sum, sum of
// squares, maximum). Every wait is bounded: on expiry the CTA records H3B_ETIMEOUT in the row kernels' status word,
// waits (bounded) for its copies in flight and returns.
constexpr int kLnStages = 4;
template <int C>
constexpr int ln_rows_smem_bytes() {
  return kLnStages * C * 2 + kLnStages * 8 + 3 * 32 * 4;
}

template <int C, bool FP4, bool IDX>
__global__ void __launch_bounds__(LnRowShape<C>::G, (LnRowShape<C>::G <= 128 ? 3 : 2))
    layer_norm_quant_rows_kernel(const RowArgs a) {
  using Sh = LnRowShape<C>;
  constexpr int K = Sh::K, G = Sh::G, NW = Sh::NW, E = 8 * K;
  constexpr uint32_t kRowBytes = C * 2;
  extern __shared__ __align__(16) uint8_t ln_smem[];
  bf16* ring = reinterpret_cast<bf16*>(ln_smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(ln_smem + (size_t)kLnStages * kRowBytes);
  float* red = reinterpret_cast<float*>(full + kLnStages);  // [3][32]: warp sums, sums of squares, maxima
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int64_t step = gridDim.x;
  if (t == 0) {
    for (int s = 0; s < kLnStages; ++s) sm100::mbar_init(&full[s], 1);
    sm100::fence_mbar_init();
    for (int s = 0; s < kLnStages; ++s) {
      const int64_t r = blockIdx.x + s * step;
      if (r < a.rows) {
        sm100::mbar_arrive_expect_tx(&full[s], kRowBytes);
        sm100::bulk_load(ring + (size_t)s * C, a.x + r * C, kRowBytes, &full[s]);
      }
    }
  }
  float a1[E], sh[E];
  auto factors = [&](int64_t tab) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int c = (t + G * k) * 8;
      float sc[8], sf[8];
      load8_nc(a.scale + tab * a.tab_ld + c, sc);
      load8_nc(a.shift + tab * a.tab_ld + c, sf);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        a1[8 * k + i] = 1.f + sc[i];
        sh[8 * k + i] = sf[i];
      }
    }
  };
  if constexpr (!IDX) factors(0);
  __syncthreads();
  volatile int no_abort = 0;
  uint32_t it = 0;
  for (int64_t r = blockIdx.x; r < a.rows; r += step, ++it) {
    const uint32_t s = it % kLnStages;
    if constexpr (IDX) factors(a.idx[r]);
    const bool ok = sm100::mbar_wait_bounded(&full[s], (it / kLnStages) & 1u, &no_abort, kRowWaitLimitNs);
    float v[E];
    const bf16* row = ring + (size_t)s * C;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(row + (t + G * k) * 8), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[8 * k + i] = f[i];
    }
    const float ts = warp_allreduce<false>(ln_thread_sum(v));
    if (lane == 0) red[w] = ts;
    if (__syncthreads_or(!ok)) {  // a row never arrived: record it, drain this CTA's copies, leave
      if (t == 0) {
        atomicExch(&g_rows_status, H3B_ETIMEOUT);
        for (int j = 0; j < kLnStages; ++j) {
          if (r + j * step >= a.rows) break;
          const uint32_t ij = it + j;
          sm100::mbar_wait_bounded(&full[ij % kLnStages], (ij / kLnStages) & 1u, &no_abort, kRowWaitLimitNs / 8);
        }
      }
      return;
    }
    if (t == 0) {  // every thread has read buffer s (before the barrier): refill it with row r + kLnStages * step
      const int64_t rn = r + kLnStages * step;
      if (rn < a.rows) {
        sm100::fence_proxy_async_smem();
        sm100::mbar_arrive_expect_tx(&full[s], kRowBytes);
        sm100::bulk_load(ring + (size_t)s * C, a.x + rn * C, kRowBytes, &full[s]);
      }
    }
    float tot = red[0];
#pragma unroll
    for (int q = 1; q < NW; ++q) tot += red[q];
    const float mean = tot / C;
#pragma unroll
    for (int i = 0; i < E; i += 2) sub2(v[i], v[i + 1], mean, mean);
    const float tq = warp_allreduce<false>(ln_thread_sumsq(v));
    if (lane == 0) red[32 + w] = tq;
    __syncthreads();
    float tot2 = red[32];
#pragma unroll
    for (int q = 1; q < NW; ++q) tot2 += red[32 + q];
    const float rs = rsqrtf(tot2 / C + a.eps);
    float cm[K];
    float am = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
#pragma unroll
      for (int i = 8 * k; i < 8 * k + 8; i += 2) {
        mul2(v[i], v[i + 1], rs, rs);
        fma2(v[i], v[i + 1], a1[i], a1[i + 1], sh[i], sh[i + 1]);
      }
      const float* u = v + 8 * k;
      float m = fmaxf(fabsf(u[0]), fabsf(u[1]));
#pragma unroll
      for (int i = 2; i < 8; ++i) m = fmaxf(m, fabsf(u[i]));
      cm[k] = m;
      am = fmaxf(am, m);
    }
    am = warp_allreduce<true>(am);
    if (lane == 0) red[64 + w] = am;
    __syncthreads();
    am = red[64];
#pragma unroll
    for (int q = 1; q < NW; ++q) am = fmaxf(am, red[64 + q]);
    const float gscale = FP4 ? fmaxf(am / kFp4Range, kMinScaleFp4) : fmaxf(am / kFp8Max, kMinScaleFp8);
    const float inv = 1.f / gscale;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int chunk = t + G * k;
      float* u = v + 8 * k;
      if constexpr (FP4) {
        // a 16-element block spans chunks 2m and 2m+1: threads t and t^1 of the same k (G is even)
        const float vmax = fmaxf(cm[k], __shfl_xor_sync(0xffffffffu, cm[k], 1));
        uint32_t bits;
        const float mult = nvfp4_block_scale(vmax, inv, &bits);
#pragma unroll
        for (int i = 0; i < 8; i += 2) mul2(u[i], u[i + 1], mult, mult);
        const uint32_t lo = e2m1x4(u[0], u[1], u[2], u[3]);
        const uint32_t hi = e2m1x4(u[4], u[5], u[6], u[7]);
        *reinterpret_cast<uint32_t*>(a.h + r * (C / 2) + chunk * 4) = lo | (hi << 16);
        if ((t & 1) == 0) a.hsf[sf_atom_offset(r, chunk >> 1, C / 16)] = (uint8_t)bits;
      } else {
#pragma unroll
        for (int i = 0; i < 8; i += 2) mul2(u[i], u[i + 1], inv, inv);
        uint2 o;
        o.x = e4m3x4(u[0], u[1], u[2], u[3]);
        o.y = e4m3x4(u[4], u[5], u[6], u[7]);
        *reinterpret_cast<uint2*>(a.h + r * C + chunk * 8) = o;
      }
    }
    if (t == 0) a.hs[r] = gscale;
  }
}

// The shared-table form of the row kernel: one CTA per SM holding ln_groups() row groups of G threads, each group
// working on its own rows with its own ring of kLnGroupStages bulk-copied row buffers and named barriers, so several
// rows are in flight per SM while the adaLN table row -- the same for all tokens -- sits once in shared memory as
// float32 pairs (1 + scale, shift), formed once per CTA exactly as the register form forms them. The arithmetic and
// the summation order are those of layer_norm_quant_rows_kernel.
template <int C>
constexpr int ln_groups() {
  return LnRowShape<C>::G <= 128 ? 6 : 4;
}
constexpr int kLnGroupStages = 2;
template <int C>
constexpr int ln_group_smem_bytes() {
  return 2 * C * 4 + ln_groups<C>() * (kLnGroupStages * C * 2 + kLnGroupStages * 8 + 3 * 32 * 4);
}

__device__ __forceinline__ void bar_group(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ bool bar_group_or(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

template <int C, bool FP4>
__global__ void __launch_bounds__(LnRowShape<C>::G * ln_groups<C>(), 1)
    layer_norm_quant_groups_kernel(const RowArgs a) {
  using Sh = LnRowShape<C>;
  constexpr int K = Sh::K, G = Sh::G, NW = Sh::NW, E = 8 * K, RG = ln_groups<C>();
  constexpr uint32_t kRowBytes = C * 2;
  extern __shared__ __align__(16) uint8_t ln_smem[];
  // [4][C/8] float4: for pair p of chunk c, (1 + scale, 1 + scale, shift, shift) of columns 8c+2p, 8c+2p+1 -- a
  // warp's reads of one pair index are contiguous
  float4* tb = reinterpret_cast<float4*>(ln_smem);
  const int grp = threadIdx.x / G, t = threadIdx.x - grp * G, lane = t & 31, w = t >> 5;
  uint8_t* gbase = ln_smem + 8 * C + (size_t)grp * (kLnGroupStages * C * 2 + kLnGroupStages * 8 + 3 * 32 * 4);
  bf16* ring = reinterpret_cast<bf16*>(gbase);
  uint64_t* full = reinterpret_cast<uint64_t*>(gbase + (size_t)kLnGroupStages * kRowBytes);
  float* red = reinterpret_cast<float*>(full + kLnGroupStages);  // [3][32]
  const int bar_id = 1 + grp;
  const int64_t step = (int64_t)gridDim.x * RG;
  const int64_t first = (int64_t)blockIdx.x * RG + grp;
  if (t == 0) {
    for (int s = 0; s < kLnGroupStages; ++s) sm100::mbar_init(&full[s], 1);
    sm100::fence_mbar_init();
    for (int s = 0; s < kLnGroupStages; ++s) {
      const int64_t r = first + s * step;
      if (r < a.rows) {
        sm100::mbar_arrive_expect_tx(&full[s], kRowBytes);
        sm100::bulk_load(ring + (size_t)s * C, a.x + r * C, kRowBytes, &full[s]);
      }
    }
  }
  for (int c = threadIdx.x; c < C / 8; c += G * RG) {
    float sc[8], sf[8];
    load8_nc(a.scale + 8 * c, sc);
    load8_nc(a.shift + 8 * c, sf);
#pragma unroll
    for (int p = 0; p < 4; ++p)
      tb[p * (C / 8) + c] = make_float4(1.f + sc[2 * p], 1.f + sc[2 * p + 1], sf[2 * p], sf[2 * p + 1]);
  }
  // this thread's output offsets: codes / scale-byte columns of its chunks (the row part is added per row)
  int sf_col[K];
#pragma unroll
  for (int k = 0; k < K; ++k) sf_col[k] = (int)sf_atom_offset(0, (t + G * k) >> 1, C / 16);
  __syncthreads();
  volatile int no_abort = 0;
  uint32_t it = 0;
  for (int64_t r = first; r < a.rows; r += step, ++it) {
    const uint32_t s = it % kLnGroupStages;
    const bool ok = sm100::mbar_wait_bounded(&full[s], (it / kLnGroupStages) & 1u, &no_abort, kRowWaitLimitNs);
    float v[E];
    const bf16* row = ring + (size_t)s * C;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(row + (t + G * k) * 8), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[8 * k + i] = f[i];
    }
    const float ts = warp_allreduce<false>(ln_thread_sum(v));
    if (lane == 0) red[w] = ts;
    if (bar_group_or(bar_id, G, !ok)) {  // a row never arrived: record it, drain this group's copies, leave
      if (t == 0) {
        atomicExch(&g_rows_status, H3B_ETIMEOUT);
        for (int j = 0; j < kLnGroupStages; ++j) {
          if (r + j * step >= a.rows) break;
          const uint32_t ij = it + j;
          sm100::mbar_wait_bounded(&full[ij % kLnGroupStages], (ij / kLnGroupStages) & 1u, &no_abort,
                                   kRowWaitLimitNs / 8);
        }
      }
      return;
    }
    if (t == 0) {  // every thread of the group has read buffer s (before the barrier): refill it
      const int64_t rn = r + kLnGroupStages * step;
      if (rn < a.rows) {
        sm100::fence_proxy_async_smem();
        sm100::mbar_arrive_expect_tx(&full[s], kRowBytes);
        sm100::bulk_load(ring + (size_t)s * C, a.x + rn * C, kRowBytes, &full[s]);
      }
    }
    float tot = red[0];
#pragma unroll
    for (int q = 1; q < NW; ++q) tot += red[q];
    const float mean = tot / C;
#pragma unroll
    for (int i = 0; i < E; i += 2) sub2(v[i], v[i + 1], mean, mean);
    const float tq = warp_allreduce<false>(ln_thread_sumsq(v));
    if (lane == 0) red[32 + w] = tq;
    bar_group(bar_id, G);
    float tot2 = red[32];
#pragma unroll
    for (int q = 1; q < NW; ++q) tot2 += red[32 + q];
    const float rs = rsqrtf(tot2 / C + a.eps);
    float cm[K];
    float am = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const float4 ab = tb[(i / 2) * (C / 8) + t + G * k];
        mul2(v[8 * k + i], v[8 * k + i + 1], rs, rs);
        fma2(v[8 * k + i], v[8 * k + i + 1], ab.x, ab.y, ab.z, ab.w);
      }
      const float* u = v + 8 * k;
      float m = fmax3(fabsf(u[0]), fabsf(u[1]), fabsf(u[2]));
      m = fmax3(m, fabsf(u[3]), fabsf(u[4]));
      m = fmax3(m, fabsf(u[5]), fabsf(u[6]));
      m = fmaxf(m, fabsf(u[7]));
      cm[k] = m;
      am = fmaxf(am, m);
    }
    am = warp_allreduce<true>(am);
    if (lane == 0) red[64 + w] = am;
    bar_group(bar_id, G);
    am = red[64];
#pragma unroll
    for (int q = 1; q < NW; ++q) am = fmaxf(am, red[64 + q]);
    const float gscale = FP4 ? fmaxf(am / kFp4Range, kMinScaleFp4) : fmaxf(am / kFp8Max, kMinScaleFp8);
    const float inv = 1.f / gscale;
    uint8_t* hrow = a.h + r * (FP4 ? C / 2 : C);
    uint8_t* sfrow = FP4 ? a.hsf + sf_atom_offset(r, 0, C / 16) : nullptr;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int chunk = t + G * k;
      float* u = v + 8 * k;
      if constexpr (FP4) {
        const float vmax = fmaxf(cm[k], __shfl_xor_sync(0xffffffffu, cm[k], 1));
        uint32_t bits;
        const float mult = nvfp4_block_scale(vmax, inv, &bits);
#pragma unroll
        for (int i = 0; i < 8; i += 2) mul2(u[i], u[i + 1], mult, mult);
        const uint32_t lo = e2m1x4(u[0], u[1], u[2], u[3]);
        const uint32_t hi = e2m1x4(u[4], u[5], u[6], u[7]);
        *reinterpret_cast<uint32_t*>(hrow + chunk * 4) = lo | (hi << 16);
        if ((t & 1) == 0) sfrow[sf_col[k]] = (uint8_t)bits;
      } else {
#pragma unroll
        for (int i = 0; i < 8; i += 2) mul2(u[i], u[i + 1], inv, inv);
        uint2 o;
        o.x = e4m3x4(u[0], u[1], u[2], u[3]);
        o.y = e4m3x4(u[4], u[5], u[6], u[7]);
        *reinterpret_cast<uint2*>(hrow + chunk * 8) = o;
      }
    }
    if (t == 0) a.hs[r] = gscale;
  }
}

// LayerNorm with the gated residual branch in front (x + gate * (sy * y) written to xo, then normalized): one
// warp per row, lane l owns the 8-element chunks l, l+32, l+64, ... (coalesced); the row is staged in shared memory
// (bf16) by asynchronous copies. The row statistics follow the LayerNorm order above: lane l plays thread 32q + l of
// each of the NW warps of the row layout in turn (one butterfly per warp), so the results equal the row-per-CTA
// kernel's. No block barriers, so many rows are in flight per SM. With one adaLN table
// row for all tokens (idx NULL) the CTA first copies it into shared memory (bf16: half the bytes the two modulate
// passes read per row against a float32 copy; 1 + scale is formed per element as in the idx path, so the values are
// the same). One CTA per SM with as many row buffers as fit beside the table (20 warps at C = 5120).
constexpr int kLnSmemBudget = 227 * 1024;
template <int C>
constexpr int ln_warps() {
  return (kLnSmemBudget - 4 * C) / (2 * C) < 20 ? (kLnSmemBudget - 4 * C) / (2 * C) : 20;
}
template <int C>
constexpr int ln_smem_bytes() {
  return ln_warps<C>() * C * 2 + 2 * C * 2;  // row buffers + bf16 table (scale, shift)
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int C, bool BRANCH, bool FP4>
__global__ void __launch_bounds__(ln_warps<C>() * 32, 1) layer_norm_quant_warp_kernel(const RowArgs a) {
  constexpr int LN_WARPS = ln_warps<C>();
  constexpr int J = C / 256;  // chunks per lane
  extern __shared__ __align__(16) uint8_t ln_smem[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  bf16* row = reinterpret_cast<bf16*>(ln_smem) + (size_t)wid * C;
  bf16* tb_scale = reinterpret_cast<bf16*>(ln_smem + (size_t)LN_WARPS * C * sizeof(bf16));
  bf16* tb_shift = tb_scale + C;
  const bool tab_smem = a.idx == nullptr;
  if (tab_smem) {
    for (int c = threadIdx.x * 8; c < C; c += LN_WARPS * 32 * 8) {
      *reinterpret_cast<uint4*>(tb_scale + c) = *reinterpret_cast<const uint4*>(a.scale + c);
      *reinterpret_cast<uint4*>(tb_shift + c) = *reinterpret_cast<const uint4*>(a.shift + c);
    }
    __syncthreads();
  }
  // the modulate factors of the 8 columns at c: (1 + scale) and shift, from shared memory or from table row tab
  auto modulate_factors = [&](int64_t tab, int c, float (&a1)[8], float (&sf)[8]) {
    if (tab_smem) {
      float sc[8];
      unpack8(*reinterpret_cast<const uint4*>(tb_scale + c), sc);
      unpack8(*reinterpret_cast<const uint4*>(tb_shift + c), sf);
#pragma unroll
      for (int i = 0; i < 8; ++i) a1[i] = 1.f + sc[i];
    } else {
      float sc[8];
      load8(a.scale + tab * a.tab_ld + c, sc);
      load8(a.shift + tab * a.tab_ld + c, sf);
#pragma unroll
      for (int i = 0; i < 8; ++i) a1[i] = 1.f + sc[i];
    }
  };
  const int64_t warps = (int64_t)gridDim.x * LN_WARPS;
  for (int64_t r = (int64_t)blockIdx.x * LN_WARPS + wid; r < a.rows; r += warps) {
    const int64_t tab = a.idx ? (int64_t)a.idx[r] : 0;
    __syncwarp();  // the previous row's reads of the buffer are done
#pragma unroll 4
    for (int j = 0; j < J; ++j) cp_async16(row + (lane + 32 * j) * 8, a.x + r * C + (lane + 32 * j) * 8);
    cp_async_wait_all();
    __syncwarp();
    if constexpr (BRANCH) {
      const float sy = a.sy[r];
#pragma unroll 2
      for (int j = 0; j < J; ++j) {
        const int c = (lane + 32 * j) * 8;
        float v[8], b[8], g[8];
        unpack8(*reinterpret_cast<const uint4*>(row + c), v);
        load8(a.y + r * C + c, b);
        load8(a.gate + tab * a.gate_ld + c, g);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = to_bf16_and_back(v[i] + g[i] * (sy * b[i]));
        store8(a.xo + r * C + c, v);
        store8(row + c, v);  // v is bf16-exact
      }
    }
    // row statistics in the LayerNorm order: lane l plays thread 32 q + l of warp q of the row layout
    using Sh = LnRowShape<C>;
    float tot = 0.f;
#pragma unroll 1
    for (int q = 0; q < Sh::NW; ++q) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int k = 0; k < Sh::K; ++k) {
        float v[8];
        unpack8(*reinterpret_cast<const uint4*>(row + (32 * q + lane + Sh::G * k) * 8), v);
#pragma unroll
        for (int i = 0; i < 8; i += 2) add2(s0, s1, v[i], v[i + 1]);
      }
      const float part = warp_allreduce<false>(s0 + s1);
      tot = q == 0 ? part : tot + part;
    }
    const float mean = tot / C;
    float tot2 = 0.f;
#pragma unroll 1
    for (int q = 0; q < Sh::NW; ++q) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int k = 0; k < Sh::K; ++k) {
        float v[8];
        unpack8(*reinterpret_cast<const uint4*>(row + (32 * q + lane + Sh::G * k) * 8), v);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          sub2(v[i], v[i + 1], mean, mean);
          sq_acc2(s0, s1, v[i], v[i + 1]);
        }
      }
      const float part = warp_allreduce<false>(s0 + s1);
      tot2 = q == 0 ? part : tot2 + part;
    }
    const float rs = rsqrtf(tot2 / C + a.eps);
    float am = 0.f;
#pragma unroll 2
    for (int j = 0; j < J; ++j) {
      const int c = (lane + 32 * j) * 8;
      float v[8], a1[8], sf[8];
      unpack8(*reinterpret_cast<const uint4*>(row + c), v);
      modulate_factors(tab, c, a1, sf);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[i] -= mean;
        v[i] = v[i] * rs * a1[i] + sf[i];
        am = fmaxf(am, fabsf(v[i]));
      }
    }
    am = warp_allreduce<true>(am);
    const float s = FP4 ? fmaxf(am / kFp4Range, kMinScaleFp4) : fmaxf(am / kFp8Max, kMinScaleFp8);
    const float inv = 1.f / s;
#pragma unroll 2
    for (int j = 0; j < J; ++j) {
      const int chunk = lane + 32 * j, c = chunk * 8;
      float v[8], a1[8], sf[8];
      unpack8(*reinterpret_cast<const uint4*>(row + c), v);
      modulate_factors(tab, c, a1, sf);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[i] -= mean;
        v[i] = v[i] * rs * a1[i] + sf[i];
      }
      if constexpr (FP4) {
        // a 16-element block spans chunks 2m and 2m+1: lanes l and l^1 of the same j
        float vmax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) vmax = fmaxf(vmax, fabsf(v[i]));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
        uint32_t bits;
        const float m = nvfp4_block_scale(vmax, inv, &bits);
        const uint32_t lo = e2m1x4(v[0] * m, v[1] * m, v[2] * m, v[3] * m);
        const uint32_t hi = e2m1x4(v[4] * m, v[5] * m, v[6] * m, v[7] * m);
        *reinterpret_cast<uint32_t*>(a.h + r * (C / 2) + chunk * 4) = lo | (hi << 16);
        if ((lane & 1) == 0) a.hsf[sf_atom_offset(r, chunk >> 1, C / 16)] = (uint8_t)bits;
      } else {
        uint2 o;
        o.x = e4m3x4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv);
        o.y = e4m3x4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv);
        *reinterpret_cast<uint2*>(a.h + r * C + c) = o;
      }
    }
    if (lane == 0) a.hs[r] = s;
  }
}

// Shared-table LayerNorm launch: one CTA per SM (fewer when there are fewer row groups' worth of rows).
template <int C, bool FP4>
int launch_ln_groups(const RowArgs& a, int sms, cudaStream_t st) {
  constexpr int lsm = ln_group_smem_bytes<C>();
  static PerDevice setup;
  int done = 0;
  if (int rc = setup.get([&](int* v) {
        if (cudaFuncSetAttribute(layer_norm_quant_groups_kernel<C, FP4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 lsm) != cudaSuccess)
          return set_error(H3B_ECUDA, "resid_norm_quant: cannot reserve %d bytes of shared memory", lsm);
        *v = 1;
        return H3B_OK;
      }, &done))
    return rc;
  constexpr int RG = ln_groups<C>();
  const int64_t need = (a.rows + RG - 1) / RG;
  layer_norm_quant_groups_kernel<C, FP4>
      <<<(unsigned)(need < sms ? need : sms), LnRowShape<C>::G * RG, lsm, st>>>(a);
  return H3B_OK;
}

// The reference's RMSNorm row form (gated residual, RMSNorm with weights, adaLN modulate, FP8 / NVFP4) with row
// groups: G threads per row (the LayerNorm layout, thread t owning the 8-element chunks t, t + G, ...), RG groups per
// CTA, each group on its own rows with the next row in flight in registers. The reference's kernel has a thread per
// 8-element chunk and reduces the row's sum of squares thread by thread in element order, butterflies each warp and
// butterflies the warp partials again (zeros past the last warp); here thread t plays the reference's threads
// t + G k, so each of its warps butterflies once per k (the reference's warp w + (G/32) k), the partials are staged in
// shared memory and every warp butterflies them the same way: the sum, and so every byte, is the reference's.
template <int C>
constexpr int rms_groups() {
  return LnRowShape<C>::G <= 96 ? 5 : (LnRowShape<C>::G <= 128 ? 3 : 2);
}

template <int C, bool BRANCH, bool FP4>
__global__ void __launch_bounds__(LnRowShape<C>::G * rms_groups<C>(), 1) rms_norm_quant_groups_kernel(const RowArgs a) {
  using Sh = LnRowShape<C>;
  constexpr int K = Sh::K, G = Sh::G, NW = Sh::NW, RG = rms_groups<C>();
  constexpr int NWV = C / 8 / 32;  // warps of the reference's row layout
  static_assert(NWV <= 32, "at most 32 warps in the reference layout");
  __shared__ float stage[RG][32];
  __shared__ float red[RG][NW];
  const int grp = threadIdx.x / G, t = threadIdx.x - grp * G, lane = t & 31, w = t >> 5;
  const int bar = 1 + grp;
  const int64_t step = (int64_t)gridDim.x * RG;
  int64_t r = (int64_t)blockIdx.x * RG + grp;
  if (r >= a.rows) return;  // group-uniform; a group without rows takes no part in any barrier
  uint4 xn[K], yn[K];
  auto load = [&](int64_t row) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int c = (t + G * k) * 8;
      xn[k] = ld8_raw(a.x + row * C + c);
      if constexpr (BRANCH) yn[k] = ld8_raw(a.y + row * C + c);
    }
  };
  load(r);
  for (; r < a.rows; r += step) {
    const int64_t tab = a.idx ? (int64_t)a.idx[r] : 0;
    float v[K][8];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      unpack8(xn[k], v[k]);
      if constexpr (BRANCH) {
        float b[8], g[8];
        unpack8(yn[k], b);
        const int c = (t + G * k) * 8;
        load8(a.gate + tab * a.gate_ld + c, g);
        const float s = a.sy[r];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[k][i] = to_bf16_and_back(v[k][i] + g[i] * (s * b[i]));
        store8(a.xo + r * C + c, v[k]);
      }
    }
    if (r + step < a.rows) load(r + step);
    // the sum of squares in the reference's tree
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[k][i] * v[k][i];
      ss = warp_allreduce<false>(ss);
      if (lane == 0) stage[grp][w + NW * k] = ss;
    }
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(G) : "memory");
    float ss = lane < NWV ? stage[grp][lane] : 0.f;
    ss = warp_allreduce<false>(ss);
    const float rs = rsqrtf(ss / C + a.eps);
    float am = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int c = (t + G * k) * 8;
      float sc[8], sf[8], wv[8];
      load8(a.scale + tab * a.tab_ld + c, sc);
      load8(a.shift + tab * a.tab_ld + c, sf);
      load8(a.nw + c, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[k][i] = v[k][i] * rs * wv[i] * (1.f + sc[i]) + sf[i];
        am = fmaxf(am, fabsf(v[k][i]));
      }
    }
    am = warp_allreduce<true>(am);
    if (lane == 0) red[grp][w] = am;
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(G) : "memory");
    am = red[grp][0];
#pragma unroll
    for (int q = 1; q < NW; ++q) am = fmaxf(am, red[grp][q]);
    if constexpr (FP4) {
      const float s = fmaxf(am / kFp4Range, kMinScaleFp4);
      const float gs = 1.f / s;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int chunk = t + G * k;
        float vmax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) vmax = fmaxf(vmax, fabsf(v[k][i]));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));  // the block's other half: thread t^1, same k
        uint32_t bits;
        const float m = nvfp4_block_scale(vmax, gs, &bits);
        const uint32_t lo = e2m1x4(v[k][0] * m, v[k][1] * m, v[k][2] * m, v[k][3] * m);
        const uint32_t hi = e2m1x4(v[k][4] * m, v[k][5] * m, v[k][6] * m, v[k][7] * m);
        *reinterpret_cast<uint32_t*>(a.h + r * (C / 2) + chunk * 4) = lo | (hi << 16);
        if ((t & 1) == 0) a.hsf[sf_atom_offset(r, chunk >> 1, C / 16)] = (uint8_t)bits;
      }
      if (t == 0) a.hs[r] = s;
    } else {
      const float s = fmaxf(am / kFp8Max, kMinScaleFp8);
      const float inv = 1.f / s;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int chunk = t + G * k;
        uint2 o;
        o.x = e4m3x4(v[k][0] * inv, v[k][1] * inv, v[k][2] * inv, v[k][3] * inv);
        o.y = e4m3x4(v[k][4] * inv, v[k][5] * inv, v[k][6] * inv, v[k][7] * inv);
        *reinterpret_cast<uint2*>(a.h + r * C + chunk * 8) = o;
      }
      if (t == 0) a.hs[r] = s;
    }
  }
}

// Row-per-CTA LayerNorm launch: as many CTAs as are resident on the device (occupancy queried once per device).
template <int C, bool FP4, bool IDX>
int launch_ln_rows(const RowArgs& a, int sms, cudaStream_t st) {
  constexpr int lsm = ln_rows_smem_bytes<C>();
  static_assert(lsm <= 48 * 1024, "the row ring fits the default dynamic shared-memory limit");
  static PerDevice occupancy;
  int per_sm = 0;
  if (int rc = occupancy.get([&](int* v) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, layer_norm_quant_rows_kernel<C, FP4, IDX>,
                                                          LnRowShape<C>::G, lsm) != cudaSuccess || n < 1)
          return set_error(H3B_ECUDA, "resid_norm_quant: occupancy query failed");
        *v = n;
        return H3B_OK;
      }, &per_sm))
    return rc;
  const int64_t cap = (int64_t)sms * per_sm;
  layer_norm_quant_rows_kernel<C, FP4, IDX>
      <<<(unsigned)(a.rows < cap ? a.rows : cap), LnRowShape<C>::G, lsm, st>>>(a);
  return H3B_OK;
}

template <int C>
int launch_resid_norm_quant(const RowArgs& a, bool branch, int norm, bool fp4, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t resident = (int64_t)sms * 2;  // two resident CTAs per SM (the launch bounds)
  const dim3 grid((unsigned)(a.rows < resident ? a.rows : resident)), block(C / 8);
#define H3B_RNQ(B, N, Q) resid_norm_quant_kernel<C, B, N, Q><<<grid, block, 0, st>>>(a)
  if (norm == H3B_NORM_NONE) {
    H3B_RNQ(true, H3B_NORM_NONE, false);
  } else if (norm == H3B_NORM_RMS) {
    constexpr int RG = rms_groups<C>();
    const int64_t need = (a.rows + RG - 1) / RG;
    const dim3 g3((unsigned)(need < sms ? need : sms)), b3(LnRowShape<C>::G * RG);
#define H3B_RMS(B, Q) rms_norm_quant_groups_kernel<C, B, Q><<<g3, b3, 0, st>>>(a)
    if (branch) {
      if (fp4) H3B_RMS(true, true); else H3B_RMS(true, false);
    } else {
      if (fp4) H3B_RMS(false, true); else H3B_RMS(false, false);
    }
#undef H3B_RMS
  } else {
    constexpr int LN_WARPS = ln_warps<C>();
    const int64_t blocks = (a.rows + LN_WARPS - 1) / LN_WARPS, cap = (int64_t)sms;
    const dim3 g2((unsigned)(blocks < cap ? blocks : cap)), b2(LN_WARPS * 32);
    const int lsm = ln_smem_bytes<C>();
    // the shared-memory attribute is set on each instantiation's first launch on a device only (later launches may
    // be inside a CUDA-graph capture)
#define H3B_LNQ(B, Q)                                                                                    \
  do {                                                                                                   \
    static PerDevice setup;                                                                              \
    int done_ = 0;                                                                                       \
    if (int rc_ = setup.get([&](int* v) {                                                                \
          if (cudaFuncSetAttribute(layer_norm_quant_warp_kernel<C, B, Q>,                                \
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, lsm) != cudaSuccess)     \
            return set_error(H3B_ECUDA, "resid_norm_quant: cannot reserve %d bytes of shared memory", lsm); \
          *v = 1;                                                                                        \
          return H3B_OK;                                                                                 \
        }, &done_))                                                                                      \
      return rc_;                                                                                        \
    layer_norm_quant_warp_kernel<C, B, Q><<<g2, b2, lsm, st>>>(a);                                       \
  } while (0)
    if (branch) {
      if (fp4) H3B_LNQ(true, true); else H3B_LNQ(true, false);
    } else if (a.idx) {
      if (int rc = fp4 ? launch_ln_rows<C, true, true>(a, sms, st) : launch_ln_rows<C, false, true>(a, sms, st))
        return rc;
    } else {
      if (int rc = fp4 ? launch_ln_groups<C, true>(a, sms, st) : launch_ln_groups<C, false>(a, sms, st)) return rc;
    }
#undef H3B_LNQ
  }
#undef H3B_RNQ
  H3B_LAUNCH_CHECK("resid_norm_quant");
  return H3B_OK;
}

// ------------------------------------------------------------------------------------------- plain FP8 per row
// One CTA per row; the row is read twice (amax, then quantize; the second read is served from L1/L2). Max is exact
// in any order, so the bytes do not depend on the thread layout.
__global__ void __launch_bounds__(256) quant_fp8_rows_kernel(const bf16* __restrict__ x, int64_t ld, int K,
                                                             uint8_t* __restrict__ q, float* __restrict__ s_out) {
  __shared__ float stage[32];
  const int64_t r = blockIdx.x;
  const bf16* row = x + r * ld;
  float am = 0.f;
  for (int c = threadIdx.x * 8; c < K; c += 256 * 8) {
    float f[8];
    load8(row + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(f[i]));
  }
  am = block_allreduce<8, true>(am, stage);
  const float s = fmaxf(am / kFp8Max, kMinScaleFp8);
  const float inv = 1.f / s;
  for (int c = threadIdx.x * 8; c < K; c += 256 * 8) {
    float f[8];
    load8(row + c, f);
    uint2 o;
    o.x = e4m3x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv);
    o.y = e4m3x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv);
    *reinterpret_cast<uint2*>(q + r * K + c) = o;
  }
  if (threadIdx.x == 0) s_out[r] = s;
}

// ------------------------------------------------------------------------------------------- per-tensor amax
// One warp per row at a time, eight 512-byte row segments in flight per warp (every load instruction reads 512
// contiguous bytes).
__global__ void __launch_bounds__(256, 4) amax_kernel(const bf16* __restrict__ x, int64_t ld, int64_t rows, int K,
                                                      float* __restrict__ amax) {
  __shared__ float stage[32];
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * 8;
  float am = 0.f;
  for (int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += nwarps) {
    const bf16* src = x + r * ld;
    for (int c0 = 0; c0 < K; c0 += 8 * 256) {
      uint4 raw[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int col = c0 + u * 256 + 8 * lane;
        raw[u] = col < K ? __ldg(reinterpret_cast<const uint4*>(src + col)) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float f[8];
        unpack8(raw[u], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) am = fmaxf(am, fabsf(f[j]));
      }
    }
  }
  am = block_allreduce<8, true>(am, stage);
  if (threadIdx.x == 0 && am > 0.f) atomicMax(reinterpret_cast<int*>(amax), __float_as_int(am));
}

// ------------------------------------------------------------------------------------------- per-tensor NVFP4
// Warp-cooperative, one warp per row at a time: a unit is 512 consecutive elements of the row and lane l holds the
// 16-element block 16l .. 16l+15 (two 16-byte loads; a warp's loads cover 1 KB of the row), so each lane owns whole
// blocks: one block scale per lane and block, no shuffles, its 8 code bytes in one store and its scale byte in one
// byte store. A warp converts 2 units while the next 2 units' loads are in flight; a row's last unit may be partial
// (K is a multiple of 64; lanes past K are masked). Rows past `rows` up to the next multiple of 128 get zero scales
// (the atom layout's padding). The per-element arithmetic is the block math of h3fast.cu:99-119.
constexpr int kQuantUnits = 2;

__global__ void __launch_bounds__(256, 3) quant_nvfp4_tensor_kernel(const bf16* __restrict__ x, int64_t ld, int64_t rows,
                                                                    int K, const float* __restrict__ amax,
                                                                    uint8_t* __restrict__ q, uint8_t* __restrict__ sf,
                                                                    float* __restrict__ s_out) {
  const float s = fmaxf(*amax / kFp4Range, kMinScaleFp4);
  const float gs = 1.f / s;
  const int lane = threadIdx.x & 31;
  const int64_t rows_pad = (rows + 127) / 128 * 128;
  const int64_t sf_cols = K / 16;
  if (blockIdx.x == 0 && threadIdx.x == 0) s_out[0] = s;
  const int64_t nwarps = (int64_t)gridDim.x * 8;
  constexpr int U = kQuantUnits;
  auto load = [&](int64_t r, int c0, uint4 (&raw)[U][2]) {
    const bf16* src = x + r * ld;
    const bool row_live = r < rows;
#pragma unroll
    for (int t = 0; t < U; ++t) {
      const int col = c0 + t * 512 + 16 * lane;
      const bool live = row_live && col < K;
      raw[t][0] = live ? __ldg(reinterpret_cast<const uint4*>(src + col)) : make_uint4(0u, 0u, 0u, 0u);
      raw[t][1] = live ? __ldg(reinterpret_cast<const uint4*>(src + col + 8)) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  int c0 = 0;
  uint4 cur[U][2], nxt[U][2];
  if (r < rows_pad) load(r, c0, cur);
  while (r < rows_pad) {
    int c1 = c0 + U * 512;
    int64_t r1 = r;
    if (c1 >= K) {
      c1 = 0;
      r1 = r + nwarps;
    }
    if (r1 < rows_pad) load(r1, c1, nxt);
    const bool row_live = r < rows;
    const size_t sf_row = sf_atom_offset(r, 0, sf_cols);
#pragma unroll
    for (int t = 0; t < U; ++t) {
      const int col = c0 + t * 512 + 16 * lane;
      if (col < K) {
        const int c = col >> 4;  // this lane's block
        uint32_t bits = 0;
        if (row_live) {
          float f[16];
          unpack8(cur[t][0], *reinterpret_cast<float(*)[8]>(&f[0]));
          unpack8(cur[t][1], *reinterpret_cast<float(*)[8]>(&f[8]));
          float vmax = fmax3(fabsf(f[0]), fabsf(f[1]), fabsf(f[2]));
#pragma unroll
          for (int i = 3; i < 15; i += 2) vmax = fmax3(vmax, fabsf(f[i]), fabsf(f[i + 1]));
          vmax = fmaxf(vmax, fabsf(f[15]));
          const float m = nvfp4_block_scale(vmax, gs, &bits);
#pragma unroll
          for (int i = 0; i < 16; i += 2) mul2(f[i], f[i + 1], m, m);
          *reinterpret_cast<uint2*>(q + r * (K / 2) + col / 2) = make_uint2(e2m1x8(f), e2m1x8(f + 8));
        }
        sf[sf_row + (size_t)(c >> 2) * 512 + (c & 3)] = (uint8_t)bits;
      }
    }
#pragma unroll
    for (int t = 0; t < U; ++t) {
      cur[t][0] = nxt[t][0];
      cur[t][1] = nxt[t][1];
    }
    r = r1;
    c0 = c1;
  }
}

// Grid of a grid-stride kernel: as many CTAs as are resident at once (no partial last wave), at most `need`.
template <typename Kern>
int resident_grid(Kern kern, int threads, int64_t need) {
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0) != cudaSuccess || per_sm < 1) per_sm = 1;
  const int64_t cap = (int64_t)sms * per_sm;
  return (int)std::max<int64_t>(1, std::min<int64_t>(cap, need));
}

}  // namespace

int quant_nvfp4_tensor_launch(const bf16* x, int64_t ld, int64_t rows, int K, const float* amax, uint8_t* q,
                              uint8_t* sf, float* s_out, cudaStream_t st) {
  const int64_t rows_pad = (rows + 127) / 128 * 128;
  quant_nvfp4_tensor_kernel<<<resident_grid(quant_nvfp4_tensor_kernel, 256, (rows_pad + 7) / 8), 256, 0, st>>>(
      x, ld, rows, K, amax, q, sf, s_out);
  H3B_LAUNCH_CHECK("quant_nvfp4_tensor");
  return H3B_OK;
}

int amax_launch(const bf16* x, int64_t ld, int64_t rows, int K, float* amax, cudaStream_t st) {
  amax_kernel<<<resident_grid(amax_kernel, 256, (rows + 7) / 8), 256, 0, st>>>(x, ld, rows, K, amax);
  H3B_LAUNCH_CHECK("amax");
  return H3B_OK;
}

}  // namespace h3b

namespace h3b {
// The row kernels' status word (H3B_ETIMEOUT when a LayerNorm row copy never completed), read in stream order.
int rows_status_async(int* dst, int clear, cudaStream_t stream) {
  if (cudaMemcpyFromSymbolAsync(dst, g_rows_status, sizeof(int), 0, cudaMemcpyDefault, stream) != cudaSuccess)
    return set_error(H3B_ECUDA, "status: reading the row kernels' status word failed");
  if (clear) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_rows_status) != cudaSuccess || cudaMemsetAsync(p, 0, sizeof(int), stream) != cudaSuccess)
      return set_error(H3B_ECUDA, "status: clearing the row kernels' status word failed");
  }
  return H3B_OK;
}
}  // namespace h3b

using namespace h3b;

extern "C" int h3b_resid_norm_quant(const void* x, const void* y, const float* sy, const void* gate, int64_t gate_ld,
                                    const int32_t* idx, int norm, const void* nw, const void* shift,
                                    const void* scale, int64_t tab_ld, void* xo, void* h, uint8_t* hsf, float* hs,
                                    float eps, int64_t rows, int C, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(x != nullptr && rows >= 0, "resid_norm_quant: x is null or rows < 0");
  H3B_REQUIRE(norm == H3B_NORM_NONE || norm == H3B_NORM_RMS || norm == H3B_NORM_LAYER, "resid_norm_quant: norm %d",
              norm);
  const bool branch = y != nullptr;
  H3B_REQUIRE(branch || norm != H3B_NORM_NONE, "resid_norm_quant: nothing to do (no y and no norm)");
  H3B_REQUIRE(!branch || (sy && gate && xo), "resid_norm_quant: the branch needs sy, gate and xo");
  H3B_REQUIRE(norm == H3B_NORM_NONE || (shift && scale && h && hs), "resid_norm_quant: the norm needs shift, scale, h, hs");
  H3B_REQUIRE(norm != H3B_NORM_RMS || nw, "resid_norm_quant: RMSNorm needs nw");
  H3B_REQUIRE(aligned(x, 16) && (!y || aligned(y, 16)) && (!xo || aligned(xo, 16)) && (!h || aligned(h, 8)),
              "resid_norm_quant: x, y, xo need 16-byte and h 8-byte alignment");
  H3B_REQUIRE((gate_ld % 8) == 0 && (tab_ld % 8) == 0, "resid_norm_quant: gate_ld and tab_ld must be multiples of 8");
  if (rows == 0) return H3B_OK;
  RowArgs a{static_cast<const bf16*>(x), static_cast<const bf16*>(y), sy, static_cast<const bf16*>(gate), gate_ld,
            idx, static_cast<const bf16*>(nw), static_cast<const bf16*>(shift), static_cast<const bf16*>(scale),
            tab_ld, static_cast<bf16*>(xo), static_cast<uint8_t*>(h), hsf, hs, eps, rows};
  const bool fp4 = hsf != nullptr;
  switch (C) {
    case 3072: return launch_resid_norm_quant<3072>(a, branch, norm, fp4, stream);
    case 4096: return launch_resid_norm_quant<4096>(a, branch, norm, fp4, stream);
    case 5120: return launch_resid_norm_quant<5120>(a, branch, norm, fp4, stream);
    case 5376: return launch_resid_norm_quant<5376>(a, branch, norm, fp4, stream);
    default: return set_error(H3B_EINVAL, "resid_norm_quant: unsupported width C=%d (3072, 4096, 5120, 5376)", C);
  }
}

extern "C" int h3b_quant_fp8_rows(const void* x, int64_t ld, int64_t rows, int K, void* q, float* s,
                                  cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(K > 0 && K % 8 == 0 && ld % 8 == 0 && ld >= K, "quant_fp8_rows: K and ld must be multiples of 8, ld >= K");
  H3B_REQUIRE(rows >= 0, "quant_fp8_rows: rows < 0");
  if (rows == 0) return H3B_OK;
  H3B_REQUIRE(x && q && s, "quant_fp8_rows: null pointer");
  H3B_REQUIRE(aligned(x, 16) && aligned(q, 8), "quant_fp8_rows: x needs 16-byte and q 8-byte alignment");
  quant_fp8_rows_kernel<<<(unsigned)rows, 256, 0, stream>>>(static_cast<const bf16*>(x), ld, K,
                                                             static_cast<uint8_t*>(q), s);
  H3B_LAUNCH_CHECK("quant_fp8_rows");
  return H3B_OK;
}

extern "C" int h3b_amax_bf16(const void* x, int64_t ld, int64_t rows, int K, float* amax, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(K > 0 && K % 8 == 0 && ld % 8 == 0 && ld >= K, "amax_bf16: K and ld must be multiples of 8, ld >= K");
  if (rows <= 0) return H3B_OK;
  H3B_REQUIRE(x && amax && aligned(x, 16), "amax_bf16: null pointer or x not 16-byte aligned");
  return amax_launch(static_cast<const bf16*>(x), ld, rows, K, amax, stream);
}

extern "C" int h3b_quant_nvfp4_tensor(const void* x, int64_t ld, int64_t rows, int K, const float* amax, void* q,
                                      uint8_t* sf, float* s_out, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(x && amax && q && sf && s_out, "quant_nvfp4_tensor: null pointer");
  H3B_REQUIRE(K > 0 && K % 64 == 0 && ld % 8 == 0 && ld >= K, "quant_nvfp4_tensor: K multiple of 64, ld multiple of 8");
  H3B_REQUIRE(aligned(x, 16) && aligned(q, 16) && aligned(sf, 4), "quant_nvfp4_tensor: x, q 16-byte and sf 4-byte aligned");
  if (rows == 0) return H3B_OK;
  return quant_nvfp4_tensor_launch(static_cast<const bf16*>(x), ld, rows, K, amax, static_cast<uint8_t*>(q), sf,
                                   s_out, stream);
}

extern "C" size_t h3b_quant_nvfp4_workspace_bytes(void) { return 256; }

extern "C" int h3b_quant_nvfp4(const void* x, int64_t ld, int64_t rows, int K, void* q, uint8_t* sf, float* s_out,
                               void* workspace, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(workspace && aligned(workspace, 256), "quant_nvfp4: workspace must be non-null and 256-byte aligned");
  H3B_REQUIRE(x && q && sf && s_out, "quant_nvfp4: null pointer");
  H3B_REQUIRE(K > 0 && K % 64 == 0 && ld % 8 == 0 && ld >= K, "quant_nvfp4: K multiple of 64, ld multiple of 8");
  H3B_REQUIRE(aligned(x, 16) && aligned(q, 16) && aligned(sf, 4), "quant_nvfp4: x, q 16-byte and sf 4-byte aligned");
  float* amax = static_cast<float*>(workspace);
  if (cudaMemsetAsync(amax, 0, sizeof(float), stream) != cudaSuccess)
    return set_error(H3B_ECUDA, "quant_nvfp4: memset of the workspace failed");
  if (rows == 0) return H3B_OK;
  int rc = amax_launch(static_cast<const bf16*>(x), ld, rows, K, amax, stream);
  if (rc) return rc;
  return quant_nvfp4_tensor_launch(static_cast<const bf16*>(x), ld, rows, K, amax, static_cast<uint8_t*>(q), sf,
                                   s_out, stream);
}

// ------------------------------------------------------------------------------------------- per-row NVFP4, any K
// One CTA per row: amax pass, then the 16-element block quantizer of h3fast.cu:121-138 with the row's global factor
// gs = 1/s, s = max(amax/(448*6), 1e-12) (the reference's per-row NVFP4 form, as in swiglu_quant's FP4 output).
namespace h3b {
namespace {
__global__ void __launch_bounds__(256) quant_nvfp4_rows_kernel(const bf16* __restrict__ x, int64_t ld, int K,
                                                               uint8_t* __restrict__ q, uint8_t* __restrict__ sf,
                                                               float* __restrict__ s_rows) {
  __shared__ float stage[32];
  const int64_t r = blockIdx.x;
  const bf16* row = x + r * ld;
  float am = 0.f;
  for (int c = threadIdx.x * 8; c < K; c += 256 * 8) {
    float f[8];
    load8(row + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(f[i]));
  }
  am = block_allreduce<8, true>(am, stage);
  const float s = fmaxf(am / kFp4Range, kMinScaleFp4);
  const float gs = 1.f / s;
  const int blocks = K / 16;
  for (int b = threadIdx.x; b < blocks; b += 256) {
    float f[8], e[8];
    load8(row + b * 16, f);
    load8(row + b * 16 + 8, e);
    float vmax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) vmax = fmaxf(vmax, fmaxf(fabsf(f[j]), fabsf(e[j])));
    uint32_t bits;
    const float m = nvfp4_block_scale(vmax, gs, &bits);
    uint2 o;
    o.x = e2m1x4(f[0] * m, f[1] * m, f[2] * m, f[3] * m) | (e2m1x4(f[4] * m, f[5] * m, f[6] * m, f[7] * m) << 16);
    o.y = e2m1x4(e[0] * m, e[1] * m, e[2] * m, e[3] * m) | (e2m1x4(e[4] * m, e[5] * m, e[6] * m, e[7] * m) << 16);
    *reinterpret_cast<uint2*>(q + r * (K / 2) + b * 8) = o;
    sf[sf_atom_offset(r, b, blocks)] = (uint8_t)bits;
  }
  if (threadIdx.x == 0) s_rows[r] = s;
}
}  // namespace
}  // namespace h3b

extern "C" int h3b_quant_nvfp4_rows(const void* x, int64_t ld, int64_t rows, int K, void* q, uint8_t* sf,
                                    float* s_rows, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(K > 0 && K % 64 == 0 && ld % 8 == 0 && ld >= K, "quant_nvfp4_rows: K multiple of 64, ld multiple of 8");
  if (rows <= 0) return H3B_OK;
  H3B_REQUIRE(x && q && sf && s_rows, "quant_nvfp4_rows: null pointer");
  H3B_REQUIRE(aligned(x, 16) && aligned(q, 8), "quant_nvfp4_rows: x 16-byte, q 8-byte aligned");
  quant_nvfp4_rows_kernel<<<(unsigned)rows, 256, 0, stream>>>(static_cast<const bf16*>(x), ld, K,
                                                               static_cast<uint8_t*>(q), sf, s_rows);
  H3B_LAUNCH_CHECK("quant_nvfp4_rows");
  return H3B_OK;
}
