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

#include <algorithm>

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
  int v16;  // V written as f16 (the decoded E4M3 values, 2 bytes per element) instead of E4M3 codes
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

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Persistent: each CTA walks work units (tile, 8 consecutive heads) with a grid stride and the items (tile, head) of
// a unit in head order. The q/k/v rows of the next item are copied into shared memory (cp.async, two buffers) while the
// current item is computed, so the loads' latency is off the critical path; each thread copies exactly the 8-byte
// pieces it later reads (rows w, w+8, ... of its warp, dims 4l .. 4l+3), so the copies need no block barrier. The
// tile's per-row data (the deferred GEMM scale and the RoPE cos/sin) is read once per unit. The arithmetic per
// element and the order of every float32 sum are those of the reference kernel.
constexpr int HG = 8;                                         // heads per work unit
constexpr int kProBufBytes = 3 * TILE * D * (int)sizeof(bf16);  // one item's q/k/v rows
constexpr int kProSmem = 2 * kProBufBytes;

struct UnitInfo {
  int ti, h0, row0, n;
  int32_t tok[RPW];  // HEAD_MAJOR: token of each of this thread's rows
};

// int8 codes of four floats already scaled into [-127, 127] (round to nearest even), packed low byte first
__device__ __forceinline__ uint32_t s8x4(float a, float b, float c, float d) {
  auto one = [](float v) { return (uint32_t)(min(127, max(-127, __float2int_rn(v))) & 0xFF); };
  return one(a) | (one(b) << 8) | (one(c) << 16) | (one(d) << 24);
}

// One row of the q/k/v row form, per lane 4 dims of q, k and v: the deferred row scale, per-head RMSNorm of q and k
// with weights (warp butterfly over the 128 dims), rotate-half RoPE on the first 96 dims, bf16 rounding. The
// reference's per-element operations (h3fast.cu:376-510) in the same order, two lanes of work per paired fp32
// instruction (q with k, or neighbouring dims); sign * sin is exact, so the sign is applied to the table. Returns
// the rounded values (qo, ko, vf) and their packed bf16 words. Warp-collective (shuffles).
__device__ __forceinline__ void rows_arith(float (&qf)[4], float (&kf)[4], float (&vf)[4], float s, uint2 crow,
                                           uint2 srow, bool rot, int partner, float sign, const float (&wqv)[4],
                                           const float (&wkv)[4], float eps, float (&qo)[4], float (&ko)[4],
                                           uint2& qw, uint2& kw, uint2& vw) {
#pragma unroll
  for (int j = 0; j < 4; j += 2) {
    mul2(qf[j], qf[j + 1], s, s);
    mul2(kf[j], kf[j + 1], s, s);
    mul2(vf[j], vf[j + 1], s, s);
  }
  float sumq = 0.f, sumk = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) sq_acc2(sumq, sumk, qf[j], kf[j]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float tq = __shfl_xor_sync(0xffffffffu, sumq, o), tk = __shfl_xor_sync(0xffffffffu, sumk, o);
    add2(sumq, sumk, tq, tk);
  }
  const float rq_ = rsqrtf(sumq / D + eps), rk_ = rsqrtf(sumk / D + eps);
#pragma unroll
  for (int j = 0; j < 4; j += 2) {
    float tq0 = rq_, tq1 = rq_, tk0 = rk_, tk1 = rk_;
    mul2(tq0, tq1, wqv[j], wqv[j + 1]);
    mul2(tk0, tk1, wkv[j], wkv[j + 1]);
    mul2(qf[j], qf[j + 1], tq0, tq1);
    mul2(kf[j], kf[j + 1], tk0, tk1);
  }
  float c[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
  if (rot) {
    unpack4(crow, c);
    unpack4(srow, sn);
  }
  float qr[4], kr[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qr[j] = __shfl_sync(0xffffffffu, qf[j], partner);
    kr[j] = __shfl_sync(0xffffffffu, kf[j], partner);
    sn[j] *= sign;
  }
#pragma unroll
  for (int j = 0; j < 4; j += 2) {
    mul2(qr[j], qr[j + 1], sn[j], sn[j + 1]);
    mul2(kr[j], kr[j + 1], sn[j], sn[j + 1]);
    fma2(qf[j], qf[j + 1], c[j], c[j + 1], qr[j], qr[j + 1]);
    fma2(kf[j], kf[j + 1], c[j], c[j + 1], kr[j], kr[j + 1]);
  }
  qw = make_uint2(pack_bf16x2(qf[0], qf[1]), pack_bf16x2(qf[2], qf[3]));
  kw = make_uint2(pack_bf16x2(kf[0], kf[1]), pack_bf16x2(kf[2], kf[3]));
  vw = make_uint2(pack_bf16x2(vf[0], vf[1]), pack_bf16x2(vf[2], vf[3]));
  unpack4(qw, qo);
  unpack4(kw, ko);
  unpack4(vw, vf);
}

// QK_I8: Q and K as symmetric int8 with per-(head, tile) scales max(amax / 127, 1e-30) (for the kind::i8 QK^T of the
// attention kernel); V stays E4M3.
template <bool ROWS, bool TILE_QK, bool QK_I8 = false>
__global__ void __launch_bounds__(NWARP * 32, 2) prologue_kernel(const ProArgs a) {
  extern __shared__ __align__(16) uint8_t pro_smem[];
  __shared__ float sp[3][NWARP][D];
  __shared__ float red[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int hgroups = (a.heads + HG - 1) / HG;
  const int units = a.n_tiles * hgroups;
  const int partner = l < HALF_LANES ? l + HALF_LANES : (l < 2 * HALF_LANES ? l - HALF_LANES : l);
  const float sign = l < HALF_LANES ? -1.f : 1.f;
  const bool rot = l < 2 * HALF_LANES && a.cosb != nullptr;
  float wqv[4], wkv[4];
  if constexpr (ROWS) {
    unpack4(*reinterpret_cast<const uint2*>(a.wq + l * 4), wqv);
    unpack4(*reinterpret_cast<const uint2*>(a.wk + l * 4), wkv);
  }
  auto unit_info = [&](int unit, UnitInfo& ui) {
    ui.ti = unit / hgroups;
    ui.h0 = (unit - ui.ti * hgroups) * HG;
    ui.row0 = a.tile_row0[ui.ti];
    ui.n = a.vbs[ui.ti];
    if constexpr (!ROWS) {
#pragma unroll
      for (int u = 0; u < RPW; ++u) {
        const int i = w + u * NWARP;
        int32_t tok = 0;
        if (i < ui.n) {
          tok = a.perm ? a.perm[ui.row0 + i] : ui.row0 + i;
          if (tok < 0 || tok >= a.seqlen) tok = 0;  // out-of-range token: read token 0 rather than fault
        }
        ui.tok[u] = tok;
      }
    }
  };
  // this thread's pieces of item (ui's tile, head h) into buffer b
  auto issue = [&](const UnitInfo& ui, int h, int b) {
    bf16* dst = reinterpret_cast<bf16*>(pro_smem + b * kProBufBytes);
#pragma unroll
    for (int u = 0; u < RPW; ++u) {
      const int i = w + u * NWARP;
      if (i < ui.n) {
        size_t src;
        if constexpr (ROWS) src = (size_t)(ui.row0 + i) * a.ld + (size_t)h * D + l * 4;
        else src = ((size_t)h * a.seqlen + (size_t)ui.tok[u]) * D + l * 4;
        cp_async8(dst + (0 * TILE + i) * D + l * 4, a.q + src);
        cp_async8(dst + (1 * TILE + i) * D + l * 4, a.k + src);
        cp_async8(dst + (2 * TILE + i) * D + l * 4, a.v + src);
      }
    }
  };

  int unit = blockIdx.x;
  if (unit >= units) return;  // CTA-uniform
  UnitInfo cur, nxt;
  unit_info(unit, cur);
  bool more = unit + (int)gridDim.x < units;
  if (more) unit_info(unit + gridDim.x, nxt);
  int b = 0;
  issue(cur, cur.h0, 0);
  cp_async_commit();
  for (;;) {
    const int ti = cur.ti, row0 = cur.row0, n = cur.n;
    // the tile's per-row data, once per unit
    float s1v[RPW];
    uint2 cr[RPW], sr[RPW];
#pragma unroll
    for (int u = 0; u < RPW; ++u) {
      const int i = w + u * NWARP;
      s1v[u] = 0.f;
      cr[u] = sr[u] = make_uint2(0u, 0u);
      if constexpr (ROWS) {
        if (i < n) {
          const int64_t r = row0 + i;
          s1v[u] = a.s1[r];
          if (rot) {
            cr[u] = *reinterpret_cast<const uint2*>(a.cosb + r * ROT + l * 4);
            sr[u] = *reinterpret_cast<const uint2*>(a.sinb + r * ROT + l * 4);
          }
        }
      }
    }
    const int hend = min(cur.h0 + HG, a.heads);
    for (int h = cur.h0; h < hend; ++h) {
      // the next item's rows go in flight before this one is computed
      if (h + 1 < hend) issue(cur, h + 1, b ^ 1);
      else if (more) issue(nxt, nxt.h0, b ^ 1);
      cp_async_commit();
      cp_async_wait_prev();
      // the rounded bf16 values go back into this thread's own pieces of the buffer for the quantization pass
      bf16* buf = reinterpret_cast<bf16*>(pro_smem + b * kProBufBytes);
      float pq[4] = {0.f, 0.f, 0.f, 0.f}, pk[4] = {0.f, 0.f, 0.f, 0.f}, pv[4] = {0.f, 0.f, 0.f, 0.f};
      float qmax = 0.f, kmax = 0.f, vmax = 0.f;
      // ---- per-row arithmetic
#pragma unroll
      for (int u = 0; u < RPW; ++u) {
        // rows past the tile's length are computed as zeros (branch-free, so the rows' shuffle chains overlap);
        // zeros leave every sum and maximum unchanged and are not stored
        const int i = w + u * NWARP;
        const bool valid = i < n;
        float qf[4], kf[4], vf[4];
        const uint2 zero = make_uint2(0u, 0u);
        unpack4(valid ? *reinterpret_cast<const uint2*>(buf + (0 * TILE + i) * D + l * 4) : zero, qf);
        unpack4(valid ? *reinterpret_cast<const uint2*>(buf + (1 * TILE + i) * D + l * 4) : zero, kf);
        unpack4(valid ? *reinterpret_cast<const uint2*>(buf + (2 * TILE + i) * D + l * 4) : zero, vf);
        float qo[4], ko[4];
        uint2 qw, kw, vw;  // the bf16 roundings, packed (what goes back into the buffer)
        if constexpr (ROWS) {
          rows_arith(qf, kf, vf, s1v[u], cr[u], sr[u], rot, partner, sign, wqv, wkv, a.eps, qo, ko, qw, kw, vw);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            qo[j] = qf[j];
            ko[j] = kf[j];
          }
          qw = pack4(qo);
          kw = pack4(ko);
          vw = pack4(vf);
        }
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          add2(pq[j], pq[j + 1], qo[j], qo[j + 1]);
          add2(pk[j], pk[j + 1], ko[j], ko[j + 1]);
          add2(pv[j], pv[j + 1], vf[j], vf[j + 1]);
          qmax = fmax3(qmax, fabsf(qo[j]), fabsf(qo[j + 1]));
          kmax = fmax3(kmax, fabsf(ko[j]), fabsf(ko[j + 1]));
          vmax = fmax3(vmax, fabsf(vf[j]), fabsf(vf[j + 1]));
        }
        if (valid) {
          *reinterpret_cast<uint2*>(buf + (0 * TILE + i) * D + l * 4) = qw;
          *reinterpret_cast<uint2*>(buf + (1 * TILE + i) * D + l * 4) = kw;
          *reinterpret_cast<uint2*>(buf + (2 * TILE + i) * D + l * 4) = vw;
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sp[0][w][l * 4 + j] = pq[j];
        sp[1][w][l * 4 + j] = pk[j];
        sp[2][w][l * 4 + j] = pv[j];
      }
      // the tile maxima (V, and Q/K with per-tile scales): warp butterflies, one staging round
      vmax = warp_allreduce<true>(vmax);
      if constexpr (TILE_QK) {
        qmax = warp_allreduce<true>(qmax);
        kmax = warp_allreduce<true>(kmax);
      }
      if (l == 0) {
        red[w] = vmax;
        red[NWARP + w] = qmax;
        red[2 * NWARP + w] = kmax;
      }
      __syncthreads();
      vmax = red[0];
#pragma unroll
      for (int ww = 1; ww < NWARP; ++ww) vmax = fmaxf(vmax, red[ww]);
      const float svb = fmaxf(vmax / kFp8Max, 1e-30f);
      float inv_q = a.inv_sq, inv_k = a.inv_sk;
      if constexpr (TILE_QK) {
        qmax = red[NWARP];
        kmax = red[2 * NWARP];
#pragma unroll
        for (int ww = 1; ww < NWARP; ++ww) {
          qmax = fmaxf(qmax, red[NWARP + ww]);
          kmax = fmaxf(kmax, red[2 * NWARP + ww]);
        }
        const float qk_max = QK_I8 ? 127.f : kFp8Max;
        const float sqb = fmaxf(qmax / qk_max, 1e-30f), skb = fmaxf(kmax / qk_max, 1e-30f);
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
        unpack4(*reinterpret_cast<const uint2*>(buf + (0 * TILE + i) * D + l * 4), qv);
        unpack4(*reinterpret_cast<const uint2*>(buf + (1 * TILE + i) * D + l * 4), kv);
        unpack4(*reinterpret_cast<const uint2*>(buf + (2 * TILE + i) * D + l * 4), vv);
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          mul2(qv[j], qv[j + 1], inv_q, inv_q);
          mul2(kv[j], kv[j + 1], inv_k, inv_k);
          mul2(vv[j], vv[j + 1], inv_v, inv_v);
        }
        if constexpr (QK_I8) {
          *reinterpret_cast<uint32_t*>(a.qb + dst) = s8x4(qv[0], qv[1], qv[2], qv[3]);
          *reinterpret_cast<uint32_t*>(a.kb + dst) = s8x4(kv[0], kv[1], kv[2], kv[3]);
        } else {
          *reinterpret_cast<uint32_t*>(a.qb + dst) = e4m3x4(qv[0], qv[1], qv[2], qv[3]);
          *reinterpret_cast<uint32_t*>(a.kb + dst) = e4m3x4(kv[0], kv[1], kv[2], kv[3]);
        }
        const uint32_t vcodes = e4m3x4(vv[0], vv[1], vv[2], vv[3]);
        if (a.v16)
          *reinterpret_cast<uint2*>(a.vb + 2 * dst) = e4m3x4_to_f16x4(vcodes);
        else
          *reinterpret_cast<uint32_t*>(a.vb + dst) = vcodes;
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
      __syncthreads();  // sp is rewritten by the next item
      b ^= 1;
    }
    if (!more) break;
    unit += gridDim.x;
    cur = nxt;
    more = unit + (int)gridDim.x < units;
    if (more) unit_info(unit + gridDim.x, nxt);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// The q/k/v row form with one CTA per (tile, head) item (blockIdx = tile * heads + head, so a tile's heads run side by
// side and its per-row scale and RoPE rows are read from L2 by all of them). Warp w owns rows w, w + 8, ... and lane l
// dims 4l .. 4l+3, as in the reference kernel; each warp loads its rows straight into registers one row ahead of the
// arithmetic, and the item's rounded values are staged in one 48 KB buffer for the quantization pass (the tile's
// maxima are needed first), so three CTAs share an SM. Arithmetic, rounding and summation orders are those of
// prologue_kernel (rows_arith; the per-lane row sums in row order, the warp partials in warp order).
constexpr int kItemSmem = 3 * TILE * D * (int)sizeof(bf16);

template <bool TILE_QK, bool QK_I8>
__global__ void __launch_bounds__(NWARP * 32, 3) prologue_item_kernel(const ProArgs a) {
  extern __shared__ __align__(16) uint8_t pro_smem[];
  __shared__ float sp[3][NWARP][D];
  __shared__ float red[32];
  bf16* buf = reinterpret_cast<bf16*>(pro_smem);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int h = blockIdx.x % a.heads, ti = blockIdx.x / a.heads;
  const int row0 = a.tile_row0[ti], n = a.vbs[ti];
  const int partner = l < HALF_LANES ? l + HALF_LANES : (l < 2 * HALF_LANES ? l - HALF_LANES : l);
  const float sign = l < HALF_LANES ? -1.f : 1.f;
  const bool rot = l < 2 * HALF_LANES && a.cosb != nullptr;
  float wqv[4], wkv[4];
  unpack4(*reinterpret_cast<const uint2*>(a.wq + l * 4), wqv);
  unpack4(*reinterpret_cast<const uint2*>(a.wk + l * 4), wkv);
  float pq[4] = {0.f, 0.f, 0.f, 0.f}, pk[4] = {0.f, 0.f, 0.f, 0.f}, pv[4] = {0.f, 0.f, 0.f, 0.f};
  float qmax = 0.f, kmax = 0.f, vmax = 0.f;
  // raw data of row w + 8u (zeros past the tile's length)
  uint2 nq = make_uint2(0u, 0u), nk = nq, nv = nq, ncr = nq, nsr = nq;
  float ns = 0.f;
  auto load_row = [&](int u) {
    const int i = w + u * NWARP;
    if (i < n) {
      const int64_t r = row0 + i;
      const size_t src = (size_t)r * a.ld + (size_t)h * D + l * 4;
      nq = __ldg(reinterpret_cast<const uint2*>(a.q + src));
      nk = __ldg(reinterpret_cast<const uint2*>(a.k + src));
      nv = __ldg(reinterpret_cast<const uint2*>(a.v + src));
      ns = __ldg(a.s1 + r);
      if (rot) {
        ncr = __ldg(reinterpret_cast<const uint2*>(a.cosb + r * ROT + l * 4));
        nsr = __ldg(reinterpret_cast<const uint2*>(a.sinb + r * ROT + l * 4));
      }
    }
  };
  load_row(0);
#pragma unroll 1
  for (int u = 0; u < RPW; ++u) {
    const int i = w + u * NWARP;
    if (i >= n) break;  // warp-uniform: later rows of this warp are past the tile too (zeros would change nothing)
    float qf[4], kf[4], vf[4];
    unpack4(nq, qf);
    unpack4(nk, kf);
    unpack4(nv, vf);
    const float s = ns;
    const uint2 crow = ncr, srow = nsr;
    if (u + 1 < RPW) load_row(u + 1);
    float qo[4], ko[4];
    uint2 qw, kw, vw;
    rows_arith(qf, kf, vf, s, crow, srow, rot, partner, sign, wqv, wkv, a.eps, qo, ko, qw, kw, vw);
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      add2(pq[j], pq[j + 1], qo[j], qo[j + 1]);
      add2(pk[j], pk[j + 1], ko[j], ko[j + 1]);
      add2(pv[j], pv[j + 1], vf[j], vf[j + 1]);
      qmax = fmax3(qmax, fabsf(qo[j]), fabsf(qo[j + 1]));
      kmax = fmax3(kmax, fabsf(ko[j]), fabsf(ko[j + 1]));
      vmax = fmax3(vmax, fabsf(vf[j]), fabsf(vf[j + 1]));
    }
    if constexpr (TILE_QK) {
      *reinterpret_cast<uint2*>(buf + (0 * TILE + i) * D + l * 4) = qw;
      *reinterpret_cast<uint2*>(buf + (1 * TILE + i) * D + l * 4) = kw;
    } else {  // static Q/K scales: the codes need no tile maximum and are written at once (only V is staged)
      const size_t dst = ((size_t)h * a.rows_pad + (size_t)ti * TILE + i) * D + l * 4;
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        mul2(qo[j], qo[j + 1], a.inv_sq, a.inv_sq);
        mul2(ko[j], ko[j + 1], a.inv_sk, a.inv_sk);
      }
      *reinterpret_cast<uint32_t*>(a.qb + dst) = e4m3x4(qo[0], qo[1], qo[2], qo[3]);
      *reinterpret_cast<uint32_t*>(a.kb + dst) = e4m3x4(ko[0], ko[1], ko[2], ko[3]);
    }
    *reinterpret_cast<uint2*>(buf + (2 * TILE + i) * D + l * 4) = vw;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sp[0][w][l * 4 + j] = pq[j];
    sp[1][w][l * 4 + j] = pk[j];
    sp[2][w][l * 4 + j] = pv[j];
  }
  vmax = warp_allreduce<true>(vmax);
  if constexpr (TILE_QK) {
    qmax = warp_allreduce<true>(qmax);
    kmax = warp_allreduce<true>(kmax);
  }
  if (l == 0) {
    red[w] = vmax;
    red[NWARP + w] = qmax;
    red[2 * NWARP + w] = kmax;
  }
  __syncthreads();
  vmax = red[0];
#pragma unroll
  for (int ww = 1; ww < NWARP; ++ww) vmax = fmaxf(vmax, red[ww]);
  const float svb = fmaxf(vmax / kFp8Max, 1e-30f);
  float inv_q = a.inv_sq, inv_k = a.inv_sk;
  if constexpr (TILE_QK) {
    qmax = red[NWARP];
    kmax = red[2 * NWARP];
#pragma unroll
    for (int ww = 1; ww < NWARP; ++ww) {
      qmax = fmaxf(qmax, red[NWARP + ww]);
      kmax = fmaxf(kmax, red[2 * NWARP + ww]);
    }
    const float qk_max = QK_I8 ? 127.f : kFp8Max;
    const float sqb = fmaxf(qmax / qk_max, 1e-30f), skb = fmaxf(kmax / qk_max, 1e-30f);
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
#pragma unroll 2
  for (int u = 0; u < RPW; ++u) {
    const int i = w + u * NWARP;
    if (i >= n) break;
    const size_t dst = (plane + i) * D + l * 4;
    if constexpr (TILE_QK) {
      float qv[4], kv[4];
      unpack4(*reinterpret_cast<const uint2*>(buf + (0 * TILE + i) * D + l * 4), qv);
      unpack4(*reinterpret_cast<const uint2*>(buf + (1 * TILE + i) * D + l * 4), kv);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        mul2(qv[j], qv[j + 1], inv_q, inv_q);
        mul2(kv[j], kv[j + 1], inv_k, inv_k);
      }
      if constexpr (QK_I8) {
        *reinterpret_cast<uint32_t*>(a.qb + dst) = s8x4(qv[0], qv[1], qv[2], qv[3]);
        *reinterpret_cast<uint32_t*>(a.kb + dst) = s8x4(kv[0], kv[1], kv[2], kv[3]);
      } else {
        *reinterpret_cast<uint32_t*>(a.qb + dst) = e4m3x4(qv[0], qv[1], qv[2], qv[3]);
        *reinterpret_cast<uint32_t*>(a.kb + dst) = e4m3x4(kv[0], kv[1], kv[2], kv[3]);
      }
    }
    float vv[4];
    unpack4(*reinterpret_cast<const uint2*>(buf + (2 * TILE + i) * D + l * 4), vv);
#pragma unroll
    for (int j = 0; j < 4; j += 2) mul2(vv[j], vv[j + 1], inv_v, inv_v);
    const uint32_t vcodes = e4m3x4(vv[0], vv[1], vv[2], vv[3]);
    if (a.v16)
      *reinterpret_cast<uint2*>(a.vb + 2 * dst) = e4m3x4_to_f16x4(vcodes);
    else
      *reinterpret_cast<uint32_t*>(a.vb + dst) = vcodes;
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

template <bool TILE_QK, bool QK_I8 = false>
int launch_prologue_item(const ProArgs& a, cudaStream_t stream) {
  auto kern = prologue_item_kernel<TILE_QK, QK_I8>;
  static PerDevice setup;  // the shared-memory reservation, per device
  int done = 0;
  if (int rc = setup.get([&](int* v) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kItemSmem) != cudaSuccess)
          return set_error(H3B_ECUDA, "prologue: cannot reserve %d bytes of shared memory", kItemSmem);
        *v = 1;
        return H3B_OK;
      }, &done))
    return rc;
  kern<<<(unsigned)((int64_t)a.n_tiles * a.heads), NWARP * 32, kItemSmem, stream>>>(a);
  return H3B_OK;
}

template <bool ROWS, bool TILE_QK, bool QK_I8 = false>
int launch_prologue(const ProArgs& a, cudaStream_t stream) {
  auto kern = prologue_kernel<ROWS, TILE_QK, QK_I8>;
  static PerDevice setup;  // the shared-memory reservation and the resident CTAs, per device
  int grid = 0;
  if (int rc = setup.get([&](int* v) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kProSmem) != cudaSuccess)
          return set_error(H3B_ECUDA, "prologue: cannot reserve %d bytes of shared memory", kProSmem);
        int per_sm = 1;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NWARP * 32, kProSmem) != cudaSuccess ||
            per_sm < 1)
          per_sm = 1;
        *v = current_sms() * per_sm;
        return H3B_OK;
      }, &grid))
    return rc;
  const int units = a.n_tiles * ((a.heads + HG - 1) / HG);
  kern<<<std::min(grid, units), NWARP * 32, kProSmem, stream>>>(a);
  return H3B_OK;
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
            vs_head, qp, kp, vp, heads, rows_pad, n_tiles, n_ext, eps, 0};
  const int rc = tile_qk ? launch_prologue_item<true>(a, stream) : launch_prologue_item<false>(a, stream);
  if (rc) return rc;
  H3B_LAUNCH_CHECK("qkv_prologue8");
  return H3B_OK;
}

extern "C" int h3b_qkv_prologue8_qk_int8(const void* q, const void* k, const void* v, int64_t ld, const float* s1,
                                         const int32_t* tile_row0, const int32_t* vbs, const void* wq, const void* wk,
                                         const void* cosb, const void* sinb, void* qb, void* kb, void* vb,
                                         float* qs_blk, float* ks_blk, float* vs_blk, float* vs_head, float* qp,
                                         float* kp, float* vp, int heads, int64_t rows_pad, int n_tiles, int n_ext,
                                         float eps, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(q && k && v && s1 && tile_row0 && vbs && wq && wk && qb && kb && vb && qs_blk && ks_blk && vs_blk && qp &&
                  kp && vp,
              "qkv_prologue8_qk_int8: null pointer");
  H3B_REQUIRE((cosb == nullptr) == (sinb == nullptr), "qkv_prologue8_qk_int8: give both or neither of cosb/sinb");
  H3B_REQUIRE(heads > 0 && n_tiles > 0 && n_ext >= n_tiles && rows_pad >= (int64_t)n_ext * TILE,
              "qkv_prologue8_qk_int8: bad heads / tiles / padding");
  H3B_REQUIRE(ld % 4 == 0 && aligned(q, 8) && aligned(k, 8) && aligned(v, 8),
              "qkv_prologue8_qk_int8: 8-byte aligned rows");
  ProArgs a{static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v), ld, 0, nullptr, s1,
            tile_row0, vbs, static_cast<const bf16*>(wq), static_cast<const bf16*>(wk),
            static_cast<const bf16*>(cosb), static_cast<const bf16*>(sinb), 1.f, 1.f,
            static_cast<uint8_t*>(qb), static_cast<uint8_t*>(kb), static_cast<uint8_t*>(vb), qs_blk, ks_blk, vs_blk,
            vs_head, qp, kp, vp, heads, rows_pad, n_tiles, n_ext, eps, 0};
  if (const int rc = launch_prologue_item<true, true>(a, stream)) return rc;
  H3B_LAUNCH_CHECK("qkv_prologue8_qk_int8");
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
            rows_pad, n_tiles, n_ext, 0.f, 0};
  if (const int rc = launch_prologue<false, true>(a, stream)) return rc;
  H3B_LAUNCH_CHECK("vsa_tile_quant");
  return H3B_OK;
}

extern "C" int h3b_vsa_tile_quant_v16(const void* q, const void* k, const void* v, int heads, int64_t seqlen,
                                      const int32_t* perm, const int32_t* tile_row0, const int32_t* vbs, void* qb,
                                      void* kb, void* vh, float* qs_blk, float* ks_blk, float* vs_blk, float* vs_head,
                                      float* qp, float* kp, float* vp, int64_t rows_pad, int n_tiles, int n_ext,
                                      cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(q && k && v && tile_row0 && vbs && qb && kb && vh && qs_blk && ks_blk && vs_blk && qp && kp && vp,
              "vsa_tile_quant_v16: null pointer");
  H3B_REQUIRE(heads > 0 && n_tiles > 0 && n_ext >= n_tiles && rows_pad >= (int64_t)n_ext * TILE && seqlen > 0,
              "vsa_tile_quant_v16: bad heads / tiles / padding");
  H3B_REQUIRE(aligned(q, 8) && aligned(k, 8) && aligned(v, 8) && aligned(vh, 16),
              "vsa_tile_quant_v16: 8-byte aligned inputs, 16-byte aligned f16 V");
  ProArgs a{static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v), 0, seqlen, perm,
            nullptr, tile_row0, vbs, nullptr, nullptr, nullptr, nullptr, 0.f, 0.f, static_cast<uint8_t*>(qb),
            static_cast<uint8_t*>(kb), static_cast<uint8_t*>(vh), qs_blk, ks_blk, vs_blk, vs_head, qp, kp, vp, heads,
            rows_pad, n_tiles, n_ext, 0.f, 1};
  if (const int rc = launch_prologue<false, true>(a, stream)) return rc;
  H3B_LAUNCH_CHECK("vsa_tile_quant_v16");
  return H3B_OK;
}

extern "C" int h3b_qkv_prologue8_tiles(const void* q, const void* k, const void* v, int64_t ld, const float* s1,
                                       const int32_t* tile_row0, const int32_t* vbs, const void* wq, const void* wk,
                                       const void* cosb, const void* sinb, void* qb, void* kb, void* vb,
                                       float* qs_blk, float* ks_blk, float* vs_blk, float* vs_head, float* qp,
                                       float* kp, float* vp, int heads, int64_t rows_pad, int n_tiles, int n_ext,
                                       float eps, int flags, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(q && k && v && s1 && tile_row0 && vbs && wq && wk && qb && kb && vb && qs_blk && ks_blk && vs_blk && qp &&
                  kp && vp,
              "qkv_prologue8_tiles: null pointer");
  H3B_REQUIRE((cosb == nullptr) == (sinb == nullptr), "qkv_prologue8_tiles: give both or neither of cosb/sinb");
  H3B_REQUIRE(heads > 0 && n_tiles > 0 && n_ext >= n_tiles && rows_pad >= (int64_t)n_ext * TILE,
              "qkv_prologue8_tiles: bad heads / tiles / padding");
  H3B_REQUIRE(ld % 4 == 0 && aligned(q, 8) && aligned(k, 8) && aligned(v, 8), "qkv_prologue8_tiles: 8-byte aligned rows");
  H3B_REQUIRE((flags & ~3) == 0, "qkv_prologue8_tiles: unknown flag bits %d", flags);
  const bool v16 = (flags & H3B_PRO_V_F16) != 0, i8 = (flags & H3B_PRO_QK_INT8) != 0;
  H3B_REQUIRE(!v16 || aligned(vb, 16), "qkv_prologue8_tiles: 16-byte aligned f16 V");
  ProArgs a{static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v), ld, 0, nullptr, s1,
            tile_row0, vbs, static_cast<const bf16*>(wq), static_cast<const bf16*>(wk),
            static_cast<const bf16*>(cosb), static_cast<const bf16*>(sinb), 1.f, 1.f,
            static_cast<uint8_t*>(qb), static_cast<uint8_t*>(kb), static_cast<uint8_t*>(vb), qs_blk, ks_blk, vs_blk,
            vs_head, qp, kp, vp, heads, rows_pad, n_tiles, n_ext, eps, v16 ? 1 : 0};
  const int rc = i8 ? launch_prologue_item<true, true>(a, stream) : launch_prologue_item<true>(a, stream);
  if (rc) return rc;
  H3B_LAUNCH_CHECK("qkv_prologue8_tiles");
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
  int v16;  // written as f16 (decoded E4M3 values) instead of E4M3 codes
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
  for (int u = 0; u < RPW; ++u) {  // rows past the tile's length hold zeros: computed branch-free, not stored
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
    const uint32_t codes = e4m3x4(xs[u][0] * inv, xs[u][1] * inv, xs[u][2] * inv, xs[u][3] * inv);
    if (a.v16)
      *reinterpret_cast<uint2*>(a.xb + 2 * ((plane + i) * D + l * 4)) = e4m3x4_to_f16x4(codes);
    else
      *reinterpret_cast<uint32_t*>(a.xb + (plane + i) * D + l * 4) = codes;
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
            static_cast<uint8_t*>(xb), xs_blk, xs_head, heads, rows_pad, n_ext, eps, 0};
  head_tile_quant_kernel<<<n_tiles * heads, NWARP * 32, 0, stream>>>(a);
  H3B_LAUNCH_CHECK("head_tile_quant");
  return H3B_OK;
}

extern "C" int h3b_head_tile_quant_v16(const void* x, int64_t ld, const float* s1, const int32_t* tile_row0,
                                       const int32_t* vbs, const void* w, void* xh, float* xs_blk, float* xs_head,
                                       int heads, int64_t rows_pad, int n_tiles, int n_ext, float eps,
                                       cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(x && tile_row0 && vbs && xh && xs_blk, "head_tile_quant_v16: null pointer");
  H3B_REQUIRE(heads > 0 && n_tiles > 0 && n_ext >= n_tiles && rows_pad >= (int64_t)n_ext * TILE,
              "head_tile_quant_v16: bad heads / tiles / padding");
  H3B_REQUIRE(ld % 4 == 0 && ld >= (int64_t)heads * D && aligned(x, 8) && aligned(xh, 16),
              "head_tile_quant_v16: 8-byte aligned rows, 16-byte aligned output");
  H3B_REQUIRE(!w || aligned(w, 8), "head_tile_quant_v16: norm weight 8-byte aligned");
  HtqArgs a{static_cast<const bf16*>(x), ld, s1, tile_row0, vbs, static_cast<const bf16*>(w),
            static_cast<uint8_t*>(xh), xs_blk, xs_head, heads, rows_pad, n_ext, eps, 1};
  head_tile_quant_kernel<<<n_tiles * heads, NWARP * 32, 0, stream>>>(a);
  H3B_LAUNCH_CHECK("head_tile_quant_v16");
  return H3B_OK;
}
