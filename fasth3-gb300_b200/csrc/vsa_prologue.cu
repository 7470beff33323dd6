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

template <bool ROWS, bool TILE_QK>
__global__ void __launch_bounds__(NWARP * 32) prologue_kernel(const ProArgs a) {
  __shared__ float sp[3][NWARP][D];
  __shared__ float red[32];
  const int h = blockIdx.x % a.heads, ti = blockIdx.x / a.heads;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int row0 = a.tile_row0[ti], n = a.vbs[ti];
  float pq[4] = {0.f, 0.f, 0.f, 0.f}, pk[4] = {0.f, 0.f, 0.f, 0.f}, pv[4] = {0.f, 0.f, 0.f, 0.f};
  float qs[RPW][4], ks[RPW][4], vs[RPW][4];
  float qmax = 0.f, kmax = 0.f, vmax = 0.f;
  float wqv[4], wkv[4];
  const int partner = l < HALF_LANES ? l + HALF_LANES : (l < 2 * HALF_LANES ? l - HALF_LANES : l);
  const float sign = l < HALF_LANES ? -1.f : 1.f;
  const bool rot = l < 2 * HALF_LANES && a.cosb != nullptr;
  if constexpr (ROWS) {
    const uint2 uq = *reinterpret_cast<const uint2*>(a.wq + l * 4), uk = *reinterpret_cast<const uint2*>(a.wk + l * 4);
    const __nv_bfloat162* hq = reinterpret_cast<const __nv_bfloat162*>(&uq);
    const __nv_bfloat162* hk = reinterpret_cast<const __nv_bfloat162*>(&uk);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float2 t = __bfloat1622float2(hq[j]);
      wqv[2 * j] = t.x;
      wqv[2 * j + 1] = t.y;
      t = __bfloat1622float2(hk[j]);
      wkv[2 * j] = t.x;
      wkv[2 * j + 1] = t.y;
    }
  }
#pragma unroll
  for (int u = 0; u < RPW; ++u) {
    const int i = w + u * NWARP;
    if (i >= n) break;  // warp-uniform
    size_t src;
    if constexpr (ROWS) {
      src = (size_t)(row0 + i) * a.ld + (size_t)h * D + l * 4;
    } else {
      int64_t tok = a.perm ? a.perm[row0 + i] : row0 + i;
      if (tok < 0 || tok >= a.seqlen) tok = 0;  // out-of-range token: read token 0 rather than fault
      src = ((size_t)h * a.seqlen + tok) * D + l * 4;
    }
    float qf[4], kf[4], vf[4];
    {
      const uint2 u0 = *reinterpret_cast<const uint2*>(a.q + src), u1 = *reinterpret_cast<const uint2*>(a.k + src),
                  u2 = *reinterpret_cast<const uint2*>(a.v + src);
      const __nv_bfloat162* b0 = reinterpret_cast<const __nv_bfloat162*>(&u0);
      const __nv_bfloat162* b1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&u2);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float2 t = __bfloat1622float2(b0[j]);
        qf[2 * j] = t.x;
        qf[2 * j + 1] = t.y;
        t = __bfloat1622float2(b1[j]);
        kf[2 * j] = t.x;
        kf[2 * j + 1] = t.y;
        t = __bfloat1622float2(b2[j]);
        vf[2 * j] = t.x;
        vf[2 * j + 1] = t.y;
      }
    }
    float qo[4], ko[4];
    if constexpr (ROWS) {
      const int64_t r = row0 + i;
      const float s = a.s1[r];
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
      const float rq = rsqrtf(sumq / D + a.eps), rk = rsqrtf(sumk / D + a.eps);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qf[j] *= rq * wqv[j];
        kf[j] *= rk * wkv[j];
      }
      float c[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
      if (rot) {
        const uint2 uc = *reinterpret_cast<const uint2*>(a.cosb + r * ROT + l * 4);
        const uint2 us = *reinterpret_cast<const uint2*>(a.sinb + r * ROT + l * 4);
        const __nv_bfloat162* bc = reinterpret_cast<const __nv_bfloat162*>(&uc);
        const __nv_bfloat162* bs = reinterpret_cast<const __nv_bfloat162*>(&us);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float2 t = __bfloat1622float2(bc[j]);
          c[2 * j] = t.x;
          c[2 * j + 1] = t.y;
          t = __bfloat1622float2(bs[j]);
          sn[2 * j] = t.x;
          sn[2 * j + 1] = t.y;
        }
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
      qs[u][j] = qo[j];
      ks[u][j] = ko[j];
      vs[u][j] = vf[j];
    }
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
    *reinterpret_cast<uint32_t*>(a.qb + dst) =
        e4m3x4(qs[u][0] * inv_q, qs[u][1] * inv_q, qs[u][2] * inv_q, qs[u][3] * inv_q);
    *reinterpret_cast<uint32_t*>(a.kb + dst) =
        e4m3x4(ks[u][0] * inv_k, ks[u][1] * inv_k, ks[u][2] * inv_k, ks[u][3] * inv_k);
    *reinterpret_cast<uint32_t*>(a.vb + dst) =
        e4m3x4(vs[u][0] * inv_v, vs[u][1] * inv_v, vs[u][2] * inv_v, vs[u][3] * inv_v);
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
