// VSA prologue: from q/k/v rows to the attention kernel's heads-first, tile-ordered E4M3 operands, their scales, and
// the fp32 tile means of q, k and v for the coarse (tile-score) step.
//
// Two input forms, one kernel (one CTA per (tile, head), 8 warps; warp w owns rows w, w+8, ...; lane l owns dims
// 4l..4l+3 -- the reference's work split, which fixes the float32 summation order of the tile means):
//   QKV_ROWS  the runner's form (qkv_prologue8, fastvideo/models/dits/h3fast/h3fast.cu:376-510): compact token rows
//             [rows, heads*128] with a deferred per-row GEMM scale s1; per-head RMSNorm of q and k with weights,
//             rotate-half RoPE on the first 96 dims, bf16 rounding, E4M3 Q/K with static per-layer scales, V with one
//             scale per (head, tile) and the running per-head maximum of those.
//   HEAD_MAJOR BASELINE config 4: q/k/v bf16 [heads, S, 128] in token order gathered into tiles through a
//             permutation, no norm or RoPE, and Q, K, V each with one E4M3 scale per (head, tile) (amax/448).
// Built with --use_fast_math and with the reference's expression order, so the QKV_ROWS outputs are bit-identical to
// the reference kernel's.
#include "common.cuh"

namespace h3b {
namespace {

constexpr int D = 128, ROT = 96, HALF_LANES = 12, NWARP = 8, TILE = 64, RPW = TILE / NWARP;

struct ProArgs {
  const bf16* q;
  const bf16* k;
  const bf16* v;
  int64_t ld;           // QKV_ROWS: row stride (elements)
  int64_t seqlen;       // HEAD_MAJOR: tokens per head plane
  const int32_t* perm;  // HEAD_MAJOR: tile-ordered row -> token (NULL: identity)
  const float* s1;      // QKV_ROWS: deferred row scale
  const int32_t* tile_row0;
  const int32_t* vbs;
  const bf16* wq;
  const bf16* wk;
  const bf16* cosb;
  const bf16* sinb;
  float inv_sq, inv_sk;  // static Q/K scales (QKV_ROWS with static scales)
  uint8_t* qb;
  uint8_t* kb;
  uint8_t* vb;
  float* qs_blk;  // per-tile Q/K scales (NULL with static scales)
  float* ks_blk;
  float* vs_blk;
  float* vs_head;
  float* qp;
  float* kp;
  float* vp;
  int heads;
  int64_t rows_pad;
  int n_tiles;
  int n_ext;
  float eps;
};

__device__ __forceinline__ void unpack4(uint2 u, float (&f)[4]) {
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
  float2 t = __bfloat1622float2(b[0]);
  f[0] = t.x;
  f[1] = t.y;
  t = __bfloat1622float2(b[1]);
  f[2] = t.x;
  f[3] = t.y;
}

// bf16-exact floats -> packed bf16 (lossless: every value passed here is already a bf16 value)
__device__ __forceinline__ uint2 pack4(const float (&f)[4]) {
  uint2 u;
  __nv_bfloat162 lo = __floats2bfloat162_rn(f[0], f[1]), hi = __floats2bfloat162_rn(f[2], f[3]);
  u.x = *reinterpret_cast<uint32_t*>(&lo);
  u.y = *reinterpret_cast<uint32_t*>(&hi);
  return u;
}

// Rows are loaded for all of a warp's rows before any arithmetic (eight rows x three 8-byte loads in flight per lane),
// and the rounded bf16 values are kept packed until the quantization pass; the arithmetic per element and the order of
// every float32 sum are those of the reference kernel.
template <bool ROWS, bool TILE_QK>
__global__ void __launch_bounds__(NWARP * 32, 2) prologue_kernel(const ProArgs a) {
  __shared__ float sp[3][NWARP][D];
  __shared__ float red[32];
  const int h = blockIdx.x % a.heads, ti = blockIdx.x / a.heads;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int row0 = a.tile_row0[ti], n = a.vbs[ti];
  float pq[4] = {0.f, 0.f, 0.f, 0.f}, pk[4] = {0.f, 0.f, 0.f, 0.f}, pv[4] = {0.f, 0.f, 0.f, 0.f};
  uint2 rq[RPW], rk[RPW], rv[RPW];
  float s1v[RPW];
  float qmax = 0.f, kmax = 0.f, vmax = 0.f;
  float wqv[4], wkv[4];
  const int partner = l < HALF_LANES ? l + HALF_LANES : (l < 2 * HALF_LANES ? l - HALF_LANES : l);
  const float sign = l < HALF_LANES ? -1.f : 1.f;
  const bool rot = l < 2 * HALF_LANES && a.cosb != nullptr;
  if constexpr (ROWS) {
    unpack4(*reinterpret_cast<const uint2*>(a.wq + l * 4), wqv);
    unpack4(*reinterpret_cast<const uint2*>(a.wk + l * 4), wkv);
  }
  // ---- loads
#pragma unroll
  for (int u = 0; u < RPW; ++u) {
    const int i = w + u * NWARP;
    rq[u] = rk[u] = rv[u] = make_uint2(0u, 0u);
    s1v[u] = 0.f;
    if (i < n) {
      size_t src;
      if constexpr (ROWS) {
        src = (size_t)(row0 + i) * a.ld + (size_t)h * D + l * 4;
      } else {
        int64_t tok = a.perm ? a.perm[row0 + i] : row0 + i;
        if (tok < 0 || tok >= a.seqlen) tok = 0;  // out-of-range token: read token 0 rather than fault
        src = ((size_t)h * a.seqlen + tok) * D + l * 4;
      }
      rq[u] = *reinterpret_cast<const uint2*>(a.q + src);
      rk[u] = *reinterpret_cast<const uint2*>(a.k + src);
      rv[u] = *reinterpret_cast<const uint2*>(a.v + src);
      if constexpr (ROWS) {
        const int64_t r = row0 + i;
        s1v[u] = a.s1[r];
      }
    }
  }
  // ---- per-row arithmetic
#pragma unroll
  for (int u = 0; u < RPW; ++u) {
    const int i = w + u * NWARP;
    if (i >= n) break;  // warp-uniform
    float qf[4], kf[4], vf[4];
    unpack4(rq[u], qf);
    unpack4(rk[u], kf);
    unpack4(rv[u], vf);
    float qo[4], ko[4];
    if constexpr (ROWS) {
      const float s = s1v[u];
      float sumq = 0.f, sumk = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qf[j] *= s;
        kf[j] *= s;
        vf[j] *= s;
        sumq += qf[j] * qf[j];
        sumk += kf[j] * kf[j];
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        sumq += __shfl_xor_sync(0xffffffffu, sumq, o);
        sumk += __shfl_xor_sync(0xffffffffu, sumk, o);
      }
      const float rq_ = rsqrtf(sumq / D + a.eps), rk_ = rsqrtf(sumk / D + a.eps);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qf[j] *= rq_ * wqv[j];
        kf[j] *= rk_ * wkv[j];
      }
      float c[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
      if (rot) {
        const int64_t r = row0 + i;
        unpack4(*reinterpret_cast<const uint2*>(a.cosb + r * ROT + l * 4), c);
        unpack4(*reinterpret_cast<const uint2*>(a.sinb + r * ROT + l * 4), sn);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float qr = __shfl_sync(0xffffffffu, qf[j], partner), kr = __shfl_sync(0xffffffffu, kf[j], partner);
        qo[j] = to_bf16_and_back(qf[j] * c[j] + sign * qr * sn[j]);
        ko[j] = to_bf16_and_back(kf[j] * c[j] + sign * kr * sn[j]);
        vf[j] = to_bf16_and_back(vf[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qo[j] = qf[j];
        ko[j] = kf[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      pq[j] += qo[j];
      pk[j] += ko[j];
      pv[j] += vf[j];
      qmax = fmaxf(qmax, fabsf(qo[j]));
      kmax = fmaxf(kmax, fabsf(ko[j]));
      vmax = fmaxf(vmax, fabsf(vf[j]));
    }
    rq[u] = pack4(qo);
    rk[u] = pack4(ko);
    rv[u] = pack4(vf);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sp[0][w][l * 4 + j] = pq[j];
    sp[1][w][l * 4 + j] = pk[j];
    sp[2][w][l * 4 + j] = pv[j];
  }
  vmax = block_allreduce<NWARP, true>(vmax, red);
  const float svb = fmaxf(vmax / kFp8Max, 1e-30f);
  float inv_q = a.inv_sq, inv_k = a.inv_sk;
  if constexpr (TILE_QK) {
    qmax = block_allreduce<NWARP, true>(qmax, red);
    kmax = block_allreduce<NWARP, true>(kmax, red);
    const float sqb = fmaxf(qmax / kFp8Max, 1e-30f), skb = fmaxf(kmax / kFp8Max, 1e-30f);
    inv_q = 1.f / sqb;
    inv_k = 1.f / skb;
    if (threadIdx.x == 0) {
      a.qs_blk[(size_t)h * a.n_ext + ti] = sqb;
      a.ks_blk[(size_t)h * a.n_ext + ti] = skb;
    }
  }
  if (threadIdx.x == 0) {
    a.vs_blk[(size_t)h * a.n_ext + ti] = svb;
    if (a.vs_head) atomicMax(reinterpret_cast<int*>(a.vs_head + h), __float_as_int(svb));
  }
  const float inv_v = 1.f / svb;
  const size_t plane = (size_t)h * a.rows_pad + (size_t)ti * TILE;
#pragma unroll
  for (int u = 0; u < RPW; ++u) {
    const int i = w + u * NWARP;
    if (i >= n) break;
    const size_t dst = (plane + i) * D + l * 4;
    float qv[4], kv[4], vv[4];
    unpack4(rq[u], qv);
    unpack4(rk[u], kv);
    unpack4(rv[u], vv);
    *reinterpret_cast<uint32_t*>(a.qb + dst) = e4m3x4(qv[0] * inv_q, qv[1] * inv_q, qv[2] * inv_q, qv[3] * inv_q);
    *reinterpret_cast<uint32_t*>(a.kb + dst) = e4m3x4(kv[0] * inv_k, kv[1] * inv_k, kv[2] * inv_k, kv[3] * inv_k);
    *reinterpret_cast<uint32_t*>(a.vb + dst) = e4m3x4(vv[0] * inv_v, vv[1] * inv_v, vv[2] * inv_v, vv[3] * inv_v);
  }
  const float inv = 1.f / (float)n;
  for (int e = threadIdx.x; e < 3 * D; e += NWARP * 32) {
    const int which = e / D, d = e % D;
    float acc = 0.f;
#pragma unroll
    for (int ww = 0; ww < NWARP; ++ww) acc += sp[which][ww][d];
    float* dst = which == 0 ? a.qp : (which == 1 ? a.kp : a.vp);
    dst[((size_t)h * a.n_tiles + ti) * D + d] = acc * inv;
  }
}

}  // namespace
}  // namespace h3b

using namespace h3b;

extern "C" int h3b_qkv_prologue8(const void* q, const void* k, const void* v, int64_t ld, const float* s1,
                                 const int32_t* tile_row0, const int32_t* vbs, const void* wq, const void* wk,
                                 const void* cosb, const void* sinb, float inv_sq, float inv_sk, void* qb, void* kb,
                                 void* vb, float* qs_blk, float* ks_blk, float* vs_blk, float* vs_head, float* qp,
                                 float* kp, float* vp, int heads, int64_t rows_pad, int n_tiles, int n_ext, float eps,
                                 cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(q && k && v && s1 && tile_row0 && vbs && wq && wk && qb && kb && vb && vs_blk && qp && kp && vp,
              "qkv_prologue8: null pointer");
  H3B_REQUIRE((cosb == nullptr) == (sinb == nullptr), "qkv_prologue8: give both or neither of cosb/sinb");
  H3B_REQUIRE(heads > 0 && n_tiles > 0 && n_ext >= n_tiles && rows_pad >= (int64_t)n_ext * TILE,
              "qkv_prologue8: bad heads / tiles / padding");
  H3B_REQUIRE(ld % 4 == 0 && aligned(q, 8) && aligned(k, 8) && aligned(v, 8), "qkv_prologue8: 8-byte aligned rows");
  const bool tile_qk = qs_blk != nullptr;
  H3B_REQUIRE(!tile_qk || ks_blk, "qkv_prologue8: per-tile Q/K scales need both qs_blk and ks_blk");
  ProArgs a{static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v), ld, 0, nullptr, s1,
            tile_row0, vbs, static_cast<const bf16*>(wq), static_cast<const bf16*>(wk),
            static_cast<const bf16*>(cosb), static_cast<const bf16*>(sinb), inv_sq, inv_sk,
            static_cast<uint8_t*>(qb), static_cast<uint8_t*>(kb), static_cast<uint8_t*>(vb), qs_blk, ks_blk, vs_blk,
            vs_head, qp, kp, vp, heads, rows_pad, n_tiles, n_ext, eps};
  if (tile_qk) prologue_kernel<true, true><<<n_tiles * heads, NWARP * 32, 0, stream>>>(a);
  else prologue_kernel<true, false><<<n_tiles * heads, NWARP * 32, 0, stream>>>(a);
  H3B_LAUNCH_CHECK("qkv_prologue8");
  return H3B_OK;
}

extern "C" int h3b_vsa_tile_quant(const void* q, const void* k, const void* v, int heads, int64_t seqlen,
                                  const int32_t* perm, const int32_t* tile_row0, const int32_t* vbs, void* qb,
                                  void* kb, void* vb, float* qs_blk, float* ks_blk, float* vs_blk, float* vs_head,
                                  float* qp,
                                  float* kp, float* vp, int64_t rows_pad, int n_tiles, int n_ext, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(q && k && v && tile_row0 && vbs && qb && kb && vb && qs_blk && ks_blk && vs_blk && qp && kp && vp,
              "vsa_tile_quant: null pointer");
  H3B_REQUIRE(heads > 0 && n_tiles > 0 && n_ext >= n_tiles && rows_pad >= (int64_t)n_ext * TILE && seqlen > 0,
              "vsa_tile_quant: bad heads / tiles / padding");
  H3B_REQUIRE(aligned(q, 8) && aligned(k, 8) && aligned(v, 8), "vsa_tile_quant: 8-byte aligned inputs");
  ProArgs a{static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v), 0, seqlen, perm,
            nullptr, tile_row0, vbs, nullptr, nullptr, nullptr, nullptr, 0.f, 0.f, static_cast<uint8_t*>(qb),
            static_cast<uint8_t*>(kb), static_cast<uint8_t*>(vb), qs_blk, ks_blk, vs_blk, vs_head, qp, kp, vp, heads,
            rows_pad, n_tiles, n_ext, 0.f};
  prologue_kernel<false, true><<<n_tiles * heads, NWARP * 32, 0, stream>>>(a);
  H3B_LAUNCH_CHECK("vsa_tile_quant");
  return H3B_OK;
}

// ------------------------------------------------------------------------------------------- one-tensor tile quant
// The prologue's per-tile E4M3 quantization for a single tensor (cross-attention queries, text keys and values), with
// the same work split and expression order: x * s1[row] (optional), per-head RMSNorm with weight (optional), bf16
// rounding, scale max(amax/448, 1e-30) per (head, tile), folded into xs_head with an atomic max (optional).
namespace h3b {
namespace {
struct HtqArgs {
  const bf16* x;
  int64_t ld;
  const float* s1;
  const int32_t* tile_row0;
  const int32_t* vbs;
  const bf16* w;
  uint8_t* xb;
  float* xs_blk;
  float* xs_head;
  int heads;
  int64_t rows_pad;
  int n_ext;
  float eps;
};

__global__ void __launch_bounds__(NWARP * 32) head_tile_quant_kernel(const HtqArgs a) {
  __shared__ float red[32];
  const int h = blockIdx.x % a.heads, ti = blockIdx.x / a.heads;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int row0 = a.tile_row0[ti], n = a.vbs[ti];
  float xs[RPW][4];
  float xmax = 0.f;
  float wv[4] = {1.f, 1.f, 1.f, 1.f};
  if (a.w) {
    const uint2 uw = *reinterpret_cast<const uint2*>(a.w + l * 4);
    const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&uw);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float2 t = __bfloat1622float2(hw[j]);
      wv[2 * j] = t.x;
      wv[2 * j + 1] = t.y;
    }
  }
  uint2 raw[RPW];
  float s1v[RPW];
#pragma unroll
  for (int u = 0; u < RPW; ++u) {  // all of a warp's rows are loaded before any arithmetic
    const int i = w + u * NWARP;
    raw[u] = make_uint2(0u, 0u);
    s1v[u] = 1.f;
    if (i < n) {
      const int64_t r = row0 + i;
      raw[u] = *reinterpret_cast<const uint2*>(a.x + (size_t)r * a.ld + (size_t)h * D + l * 4);
      if (a.s1) s1v[u] = a.s1[r];
    }
  }
#pragma unroll
  for (int u = 0; u < RPW; ++u) {
    const int i = w + u * NWARP;
    if (i >= n) break;  // warp-uniform
    float f[4];
    unpack4(raw[u], f);
    const float s = s1v[u];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[j] *= s;
      sum += f[j] * f[j];
    }
    if (a.w) {
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      const float rr = rsqrtf(sum / D + a.eps);
#pragma unroll
      for (int j = 0; j < 4; ++j) f[j] *= rr * wv[j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      xs[u][j] = to_bf16_and_back(f[j]);
      xmax = fmaxf(xmax, fabsf(xs[u][j]));
    }
  }
  xmax = block_allreduce<NWARP, true>(xmax, red);
  const float sb = fmaxf(xmax / kFp8Max, 1e-30f);
  if (threadIdx.x == 0) {
    a.xs_blk[(size_t)h * a.n_ext + ti] = sb;
    if (a.xs_head) atomicMax(reinterpret_cast<int*>(a.xs_head + h), __float_as_int(sb));
  }
  const float inv = 1.f / sb;
  const size_t plane = (size_t)h * a.rows_pad + (size_t)ti * TILE;
#pragma unroll
  for (int u = 0; u < RPW; ++u) {
    const int i = w + u * NWARP;
    if (i >= n) break;
    *reinterpret_cast<uint32_t*>(a.xb + (plane + i) * D + l * 4) =
        e4m3x4(xs[u][0] * inv, xs[u][1] * inv, xs[u][2] * inv, xs[u][3] * inv);
  }
}
}  // namespace
}  // namespace h3b

extern "C" int h3b_head_tile_quant(const void* x, int64_t ld, const float* s1, const int32_t* tile_row0,
                                   const int32_t* vbs, const void* w, void* xb, float* xs_blk, float* xs_head,
                                   int heads, int64_t rows_pad, int n_tiles, int n_ext, float eps,
                                   cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(x && tile_row0 && vbs && xb && xs_blk, "head_tile_quant: null pointer");
  H3B_REQUIRE(heads > 0 && n_tiles > 0 && n_ext >= n_tiles && rows_pad >= (int64_t)n_ext * TILE,
              "head_tile_quant: bad heads / tiles / padding");
  H3B_REQUIRE(ld % 4 == 0 && ld >= (int64_t)heads * D && aligned(x, 8), "head_tile_quant: 8-byte aligned rows");
  H3B_REQUIRE(!w || aligned(w, 8), "head_tile_quant: norm weight 8-byte aligned");
  HtqArgs a{static_cast<const bf16*>(x), ld, s1, tile_row0, vbs, static_cast<const bf16*>(w),
            static_cast<uint8_t*>(xb), xs_blk, xs_head, heads, rows_pad, n_ext, eps};
  head_tile_quant_kernel<<<n_tiles * heads, NWARP * 32, 0, stream>>>(a);
  H3B_LAUNCH_CHECK("head_tile_quant");
  return H3B_OK;
}
