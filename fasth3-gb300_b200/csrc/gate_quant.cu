// Attention output -> next GEMM's input: gather each compact token row from the attention kernel's heads-first padded
// layout, optionally merge it with a dense-pass output by log-sum-exp, add gate * compressed-branch output, and
// quantize the row to FP8 (row scale) or NVFP4 (row global scale + ue4m3 block scales).
//
// Semantics of attn_gate_quant (fastvideo/models/dits/h3fast/h3fast.cu:688-741). Built with --use_fast_math and the
// reference's expression order, one CTA per row with W/8 threads (thread t owns elements 8t..8t+7 of head t/16), so
// the quantized bytes are bit-identical to the reference's.
#include "common.cuh"

namespace h3b {
namespace {

constexpr int D = 128;

struct GateArgs {
  const bf16* ob;
  const bf16* g;
  const float* sg;
  const bf16* oc;
  const int32_t* slot;
  int64_t rows_pad;
  int n_tiles;
  int tile;
  uint8_t* a;
  uint8_t* asf;
  float* sa;
  const bf16* o1;
  const float* lse1a;
  const float* lse1b;
  int n1;
  const float* lse2;
  int64_t rows;
};

// Persistent CTAs: a CTA walks rows r, r + grid, ...; the next row's attention output is loaded (its slot one more row
// ahead) while the current row is reduced and quantized. The per-row arithmetic is unchanged.
template <int W, bool GATE, bool FP4, bool MERGE>
__global__ void __launch_bounds__(W / 8, 2) gate_quant_kernel(const GateArgs p) {
  constexpr int NW = W / 8 / 32, H = W / D;
  __shared__ float stage[32];
  const int t = threadIdx.x, h = t / (D / 8), d0 = (t % (D / 8)) * 8;
  int64_t r = blockIdx.x;
  if (r >= p.rows) return;
  const int64_t g = gridDim.x;
  int sl_next = p.slot[r];
  uint4 on = ld8_raw(p.ob + ((size_t)h * p.rows_pad + sl_next) * D + d0);
  int sl_next2 = r + g < p.rows ? p.slot[r + g] : 0;
  for (; r < p.rows; r += g) {
  const int sl = sl_next;
  float o[8];
  unpack8(on, o);
  if (r + g < p.rows) {
    sl_next = sl_next2;
    on = ld8_raw(p.ob + ((size_t)h * p.rows_pad + sl_next) * D + d0);
    if (r + 2 * g < p.rows) sl_next2 = p.slot[r + 2 * g];
  }
  if constexpr (MERGE) {
    float od[8];
    load8(p.o1 + ((size_t)r * H + h) * D + d0, od);
    const float l1 = (r < p.n1 ? p.lse1a[(size_t)h * p.n1 + r] : p.lse1b[(size_t)h * (p.rows - p.n1) + (r - p.n1)]) *
                     1.4426950408889634f;
    const float l2 = r < p.n1 ? -INFINITY : p.lse2[(size_t)h * p.rows_pad + sl];
    const float m = fmaxf(l1, l2);
    const float w1 = m == -INFINITY ? 0.f : exp2f(l1 - m), w2 = m == -INFINITY ? 0.f : exp2f(l2 - m);
    const float inv = (w1 + w2) > 0.f ? 1.f / (w1 + w2) : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (w1 * od[i] + (w2 > 0.f ? w2 * o[i] : 0.f)) * inv;
  }
  if constexpr (GATE) {
    float gv[8], cv[8];
    load8(p.g + r * W + t * 8, gv);
    load8(p.oc + ((size_t)h * p.n_tiles + sl / p.tile) * D + d0, cv);
    const float s = p.sg[r];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] += cv[i] * (s * gv[i]);
  }
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(o[i]));
  am = block_allreduce<NW, true>(am, stage);
  if constexpr (FP4) {
    const float s = fmaxf(am / kFp4Range, kMinScaleFp4);
    const float gs = 1.f / s;
    float vmax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) vmax = fmaxf(vmax, fabsf(o[i]));
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
    uint32_t bits;
    const float m = nvfp4_block_scale(vmax, gs, &bits);
    const uint32_t lo = e2m1x4(o[0] * m, o[1] * m, o[2] * m, o[3] * m);
    const uint32_t hi = e2m1x4(o[4] * m, o[5] * m, o[6] * m, o[7] * m);
    *reinterpret_cast<uint32_t*>(p.a + r * (W / 2) + t * 4) = lo | (hi << 16);
    if ((t & 1) == 0) p.asf[sf_atom_offset(r, t >> 1, W / 16)] = (uint8_t)bits;
    if (t == 0) p.sa[r] = s;
  } else {
    const float s = fmaxf(am / kFp8Max, kMinScaleFp8);
    const float inv = 1.f / s;
    uint2 u;
    u.x = e4m3x4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
    u.y = e4m3x4(o[4] * inv, o[5] * inv, o[6] * inv, o[7] * inv);
    *reinterpret_cast<uint2*>(p.a + r * W + t * 8) = u;
    if (t == 0) p.sa[r] = s;
  }
  }
}

// The plain form (no gate branch, no merge: the block's attention output straight into the next GEMM's input) with
// row groups: a CTA per SM holds RG groups of G threads, each group working on its own rows r, r + step, ...
// with the next row's attention output in flight in registers; thread t of a group owns the 8-element chunks
// t, t + G, ... of the row (a warp's 16-byte loads cover two heads' 256-byte segments), and the row maximum is reduced
// over the group's warps with a named barrier, so many rows are in flight per SM without the 20-warp block reduction
// of the one-row-per-CTA form. The per-element arithmetic is gate_quant_kernel's (bit-identical bytes).
template <int W>
struct GqShape {
  static constexpr int kChunks = W / 8;
  static constexpr int pick() {
    for (int k = 5; k > 1; --k)
      if (kChunks % k == 0 && (kChunks / k) % 32 == 0) return k;
    return 1;
  }
  static constexpr int K = pick();
  static constexpr int G = kChunks / K;
  static constexpr int NW = G / 32;
  static constexpr int RG = G <= 128 ? 5 : 3;
  static_assert(G % 32 == 0 && G % 2 == 0, "whole warps, even thread count");
};

__device__ __forceinline__ void gq_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

template <int W, bool FP4>
__global__ void __launch_bounds__(GqShape<W>::G * GqShape<W>::RG, 1) gate_quant_groups_kernel(const GateArgs p) {
  using Sh = GqShape<W>;
  constexpr int K = Sh::K, G = Sh::G, NW = Sh::NW, RG = Sh::RG;
  __shared__ float red[RG][2][NW];
  const int grp = threadIdx.x / G, t = threadIdx.x - grp * G, lane = t & 31, w = t >> 5;
  const int64_t step = (int64_t)gridDim.x * RG;
  int64_t r = (int64_t)blockIdx.x * RG + grp;
  if (r >= p.rows) return;  // group-uniform; a group with no rows takes no part in any barrier
  int hk[K], dk[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int c = t + G * k;
    hk[k] = c / (D / 8);
    dk[k] = (c % (D / 8)) * 8;
  }
  uint4 nxt[K];
  auto load = [&](int64_t row) {
    const int sl = p.slot[row];
#pragma unroll
    for (int k = 0; k < K; ++k) nxt[k] = ld8_raw(p.ob + ((size_t)hk[k] * p.rows_pad + sl) * D + dk[k]);
  };
  load(r);
  int par = 0;
  for (; r < p.rows; r += step, par ^= 1) {
    float o[K][8];
#pragma unroll
    for (int k = 0; k < K; ++k) unpack8(nxt[k], o[k]);
    if (r + step < p.rows) load(r + step);
    float cm[K];
    float am = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float m = fmax3(fabsf(o[k][0]), fabsf(o[k][1]), fabsf(o[k][2]));
      m = fmax3(m, fabsf(o[k][3]), fabsf(o[k][4]));
      m = fmax3(m, fabsf(o[k][5]), fabsf(o[k][6]));
      cm[k] = fmaxf(m, fabsf(o[k][7]));
      am = fmaxf(am, cm[k]);
    }
    am = warp_allreduce<true>(am);
    if (lane == 0) red[grp][par][w] = am;
    gq_bar(1 + grp, G);
    am = red[grp][par][0];
#pragma unroll
    for (int q = 1; q < NW; ++q) am = fmaxf(am, red[grp][par][q]);
    if constexpr (FP4) {
      const float s = fmaxf(am / kFp4Range, kMinScaleFp4);
      const float gs = 1.f / s;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int c = t + G * k;
        // a 16-element block spans chunks 2m and 2m+1: threads t and t^1 of the same k (G is even)
        const float vmax = fmaxf(cm[k], __shfl_xor_sync(0xffffffffu, cm[k], 1));
        uint32_t bits;
        const float m = nvfp4_block_scale(vmax, gs, &bits);
        const uint32_t lo = e2m1x4(o[k][0] * m, o[k][1] * m, o[k][2] * m, o[k][3] * m);
        const uint32_t hi = e2m1x4(o[k][4] * m, o[k][5] * m, o[k][6] * m, o[k][7] * m);
        *reinterpret_cast<uint32_t*>(p.a + r * (W / 2) + c * 4) = lo | (hi << 16);
        if ((t & 1) == 0) p.asf[sf_atom_offset(r, c >> 1, W / 16)] = (uint8_t)bits;
      }
      if (t == 0) p.sa[r] = s;
    } else {
      const float s = fmaxf(am / kFp8Max, kMinScaleFp8);
      const float inv = 1.f / s;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int c = t + G * k;
        uint2 u;
        u.x = e4m3x4(o[k][0] * inv, o[k][1] * inv, o[k][2] * inv, o[k][3] * inv);
        u.y = e4m3x4(o[k][4] * inv, o[k][5] * inv, o[k][6] * inv, o[k][7] * inv);
        *reinterpret_cast<uint2*>(p.a + r * W + c * 8) = u;
      }
      if (t == 0) p.sa[r] = s;
    }
  }
}

template <int W>
int launch(const GateArgs& p, bool gate, bool fp4, bool merge, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t resident = (int64_t)sms * 2;  // two resident CTAs per SM (the launch bounds)
  const dim3 grid((unsigned)(p.rows < resident ? p.rows : resident)), block(W / 8);
#define H3B_GQ(G, Q, M) gate_quant_kernel<W, G, Q, M><<<grid, block, 0, st>>>(p)
  if (!gate && !merge) {  // the plain form: row groups
    using Sh = GqShape<W>;
    const int64_t need = (p.rows + Sh::RG - 1) / Sh::RG;
    const dim3 g2((unsigned)(need < sms ? need : sms)), b2(Sh::G * Sh::RG);
    if (fp4) gate_quant_groups_kernel<W, true><<<g2, b2, 0, st>>>(p);
    else gate_quant_groups_kernel<W, false><<<g2, b2, 0, st>>>(p);
  } else if (gate) {
    if (fp4) { if (merge) H3B_GQ(true, true, true); else H3B_GQ(true, true, false); }
    else { if (merge) H3B_GQ(true, false, true); else H3B_GQ(true, false, false); }
  } else {
    if (fp4) { if (merge) H3B_GQ(false, true, true); else H3B_GQ(false, true, false); }
    else { if (merge) H3B_GQ(false, false, true); else H3B_GQ(false, false, false); }
  }
#undef H3B_GQ
  H3B_LAUNCH_CHECK("attn_gate_quant");
  return H3B_OK;
}

}  // namespace
}  // namespace h3b

using namespace h3b;

extern "C" int h3b_attn_gate_quant(const void* ob, const void* g, const float* sg, const void* oc,
                                   const int32_t* slot, int64_t rows_pad, int n_tiles, int tile, void* a, uint8_t* asf,
                                   float* sa, int64_t rows, int W, const void* o1, const float* lse1a,
                                   const float* lse1b, int n1, const float* lse2, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(ob && slot && a && sa, "attn_gate_quant: null pointer");
  const bool gate = g != nullptr, merge = o1 != nullptr;
  H3B_REQUIRE(!gate || (sg && oc), "attn_gate_quant: the gate needs sg and oc");
  H3B_REQUIRE(!merge || (lse1a && lse1b && lse2 && n1 >= 0 && n1 <= rows), "attn_gate_quant: merge needs o1, lse1a, "
              "lse1b, lse2 and 0 <= n1 <= rows");
  H3B_REQUIRE(tile > 0 && n_tiles > 0, "attn_gate_quant: bad tiles");
  if (rows == 0) return H3B_OK;
  GateArgs p{static_cast<const bf16*>(ob), static_cast<const bf16*>(g), sg, static_cast<const bf16*>(oc), slot,
             rows_pad, n_tiles, tile, static_cast<uint8_t*>(a), asf, sa, static_cast<const bf16*>(o1), lse1a, lse1b,
             n1, lse2, rows};
  const bool fp4 = asf != nullptr;
  switch (W) {
    case 5120: return launch<5120>(p, gate, fp4, merge, stream);
    case 7168: return launch<7168>(p, gate, fp4, merge, stream);
    default: return set_error(H3B_EINVAL, "attn_gate_quant: unsupported width W=%d (5120, 7168)", W);
  }
}
