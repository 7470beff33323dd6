// VSA coarse step: tile scores from the tile means, top-k key-tile selection per query tile, and the compressed
// (mean-pooled) attention branch.
//
// Scores are defined bit-exactly: sc[h,i,j] = fmul(sum_d, scale) with sum_d accumulated over d = 0..127 in order, one
// correctly rounded fused multiply-add per d, so a float32 CPU restatement (an exact product added with one rounding)
// reproduces every bit and the selected tile indices are reproducible. The reference scores with cuBLAS (TF32 by default,
// fastvideo/models/dits/h3fast/__init__.py:146-149, 498-500), which no other implementation can reproduce bit for bit.
//
// Selection follows topk_rows (fastvideo/models/dits/h3fast/h3fast.cu:524-588): prefix tiles kept, per span the k
// largest keys under the order-preserving uint32 map of the float bits, ties broken toward the lowest column, the kept
// columns written in ascending order.
#include "common.cuh"

namespace h3b {
namespace {

constexpr int D = 128;

// ------------------------------------------------------------------------------------------------ scores
// Block = 128x128 outputs of one head, 256 threads, an 8x8 register tile per thread; the q and k tile means are staged
// in shared memory 32 dimensions at a time, transposed ([d][row], rows padded by 4 floats against bank conflicts).
// Each output accumulates d = 0..127 in order, one fused multiply-add per d (the order the CPU oracle restates).
constexpr int SB = 128, SCH = 32, SPAD = SB + 4;

__global__ void __launch_bounds__(256) scores_kernel(const float* __restrict__ qp, const float* __restrict__ kp,
                                                     int n, float scale, float* __restrict__ sc) {
  __shared__ __align__(16) float sq[SCH][SPAD];
  __shared__ __align__(16) float sk[SCH][SPAD];
  const int h = blockIdx.z;
  const int i0 = blockIdx.y * SB, j0 = blockIdx.x * SB;
  const float* qh = qp + (size_t)h * n * D;
  const float* kh = kp + (size_t)h * n * D;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float acc[8][8];
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[a][b] = 0.f;
  for (int dc = 0; dc < D; dc += SCH) {
    for (int e = threadIdx.x; e < SB * SCH / 4; e += 256) {
      const int r = e / (SCH / 4), d4 = (e % (SCH / 4)) * 4;
      const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 vq = i0 + r < n ? *reinterpret_cast<const float4*>(qh + (size_t)(i0 + r) * D + dc + d4) : zero;
      const float4 vk = j0 + r < n ? *reinterpret_cast<const float4*>(kh + (size_t)(j0 + r) * D + dc + d4) : zero;
      sq[d4 + 0][r] = vq.x;
      sq[d4 + 1][r] = vq.y;
      sq[d4 + 2][r] = vq.z;
      sq[d4 + 3][r] = vq.w;
      sk[d4 + 0][r] = vk.x;
      sk[d4 + 1][r] = vk.y;
      sk[d4 + 2][r] = vk.z;
      sk[d4 + 3][r] = vk.w;
    }
    __syncthreads();
#pragma unroll 4
    for (int d = 0; d < SCH; ++d) {
      const float4 a0 = *reinterpret_cast<const float4*>(&sq[d][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sq[d][ty * 8 + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sk[d][tx * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&sk[d][tx * 8 + 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) acc[a][b] = __fmaf_rn(av[a], bv[b], acc[a][b]);
    }
    __syncthreads();
  }
  const int jb = j0 + tx * 8;
#pragma unroll
  for (int a = 0; a < 8; ++a) {
    const int i = i0 + ty * 8 + a;
    if (i >= n) break;
    float* dst = sc + ((size_t)h * n + i) * n;
    if (jb + 8 <= n && (n & 3) == 0) {
      *reinterpret_cast<float4*>(dst + jb) = make_float4(__fmul_rn(acc[a][0], scale), __fmul_rn(acc[a][1], scale),
                                                         __fmul_rn(acc[a][2], scale), __fmul_rn(acc[a][3], scale));
      *reinterpret_cast<float4*>(dst + jb + 4) = make_float4(__fmul_rn(acc[a][4], scale),
                                                             __fmul_rn(acc[a][5], scale),
                                                             __fmul_rn(acc[a][6], scale),
                                                             __fmul_rn(acc[a][7], scale));
    } else {
#pragma unroll
      for (int b = 0; b < 8; ++b)
        if (jb + b < n) dst[jb + b] = __fmul_rn(acc[a][b], scale);
    }
  }
}

// ------------------------------------------------------------------------------------------------ top-k
struct Spans {
  int n;
  int start[4];
  int end[4];
  int k[4];
};

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One warp per (head, query tile). PER = keys per lane (span length <= 32 * PER).
template <int PER>
__global__ void __launch_bounds__(128) topk_kernel(const float* __restrict__ scores, int n, int n_ext, int prefix,
                                                   Spans sp, int rows, int* __restrict__ idx, int* __restrict__ num,
                                                   int split) {
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int hh = row / n, q = row - hh * n;
  int* out = idx + ((size_t)hh * n_ext + q) * n;
  const float* srow = scores + (size_t)row * n;
  if (q < prefix) {
    if (!split)
      for (int c = lane; c < n; c += 32) out[c] = c;
    if (lane == 0) num[(size_t)hh * n_ext + q] = split ? 0 : n;
    return;
  }
  int cnt = 0;
  if (!split) {
    for (int c = lane; c < prefix; c += 32) out[c] = c;
    cnt = prefix;
  }
  const uint32_t below = (1u << lane) - 1u;
  for (int s = 0; s < sp.n; ++s) {
    const int start = sp.start[s], len = sp.end[s] - start, k = sp.k[s];
    if (k >= len) {
      for (int c = lane; c < len; c += 32) out[cnt + c] = start + c;
      cnt += len;
      continue;
    }
    uint32_t key[PER];
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = p * 32 + lane;
      key[p] = c < len ? order_key(srow[start + c]) : 0u;
    }
    // the largest threshold t with count(key >= t) >= k, found bit by bit from the top
    uint32_t t = 0;
#pragma unroll 1
    for (int b = 31; b >= 0; --b) {
      const uint32_t cand = t | (1u << b);
      int c = 0;
#pragma unroll
      for (int p = 0; p < PER; ++p) c += key[p] >= cand ? 1 : 0;
      if (__reduce_add_sync(0xffffffffu, c) >= k) t = cand;
    }
    int above = 0;
#pragma unroll
    for (int p = 0; p < PER; ++p) above += key[p] > t ? 1 : 0;
    const int ties_needed = k - __reduce_add_sync(0xffffffffu, above);
    int ties_seen = 0;
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = p * 32 + lane;
      const bool valid = c < len;
      const bool eq = valid && key[p] == t;
      const uint32_t eq_mask = __ballot_sync(0xffffffffu, eq);
      const bool keep = (valid && key[p] > t) || (eq && ties_seen + __popc(eq_mask & below) < ties_needed);
      ties_seen += __popc(eq_mask);
      const uint32_t keep_mask = __ballot_sync(0xffffffffu, keep);
      if (keep) out[cnt + __popc(keep_mask & below)] = start + c;
      cnt += __popc(keep_mask);
    }
  }
  if (lane == 0) num[(size_t)hh * n_ext + q] = cnt;
}

// ------------------------------------------------------------------------------------------------ compressed branch
// oc[h,i,:] = softmax_j(sc[h,i,:]) @ vp[h,:,:] in fp32, stored bf16. One CTA (128 threads) per (head, query tile).
__global__ void __launch_bounds__(128) compressed_kernel(const float* __restrict__ sc, const float* __restrict__ vp,
                                                         int n, bf16* __restrict__ oc) {
  extern __shared__ float p[];
  __shared__ float stage[32];
  const int h = blockIdx.y, i = blockIdx.x;
  const float* row = sc + ((size_t)h * n + i) * n;
  float m = -INFINITY;
  for (int j = threadIdx.x; j < n; j += 128) m = fmaxf(m, row[j]);
  m = block_allreduce<4, true>(m, stage);
  float s = 0.f;
  for (int j = threadIdx.x; j < n; j += 128) {
    const float e = __expf(row[j] - m);
    p[j] = e;
    s += e;
  }
  s = block_allreduce<4, false>(s, stage);  // also orders the p[] writes before the reads below
  const float inv = 1.f / s;
  const float* vh = vp + (size_t)h * n * D;
  float acc = 0.f;
  for (int j = 0; j < n; ++j) acc += p[j] * vh[(size_t)j * D + threadIdx.x];
  oc[((size_t)h * n + i) * D + threadIdx.x] = __float2bfloat16_rn(acc * inv);
}

// The union of two adjacent query tiles' selections, ascending, with a membership byte per entry (bit 0: tile 2p,
// bit 1: tile 2p+1): topk_pairs' output format (fastvideo/models/dits/h3fast/h3fast.cu:590-686) built from topk_rows'
// lists. One warp per (head, pair); a byte per key column in shared memory marks the members, then a ballot
// compaction writes the columns in ascending order. Tiles past n (padding) select nothing.
constexpr int kUnionWarps = 4;
__global__ void __launch_bounds__(kUnionWarps * 32) union_pairs_kernel(const int* __restrict__ idx,
                                                                       const int* __restrict__ num, int n, int n_ext,
                                                                       int pairs_total, int* __restrict__ u_idx,
                                                                       uint8_t* __restrict__ u_mem,
                                                                       int* __restrict__ u_num) {
  extern __shared__ uint8_t umem[];
  const int wid = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int gp = blockIdx.x * kUnionWarps + wid;
  if (gp >= pairs_total) return;  // warp-uniform
  uint8_t* m = umem + (size_t)wid * n;
  const int n_pairs = n_ext / 2;
  const int hh = gp / n_pairs, pr = gp % n_pairs;
  for (int c = l; c < n; c += 32) m[c] = 0;
  __syncwarp();
  for (int t = 0; t < 2; ++t) {
    const int r = 2 * pr + t;
    if (r >= n) break;
    const int cnt = num[(size_t)hh * n_ext + r];
    const int* list = idx + ((size_t)hh * n_ext + r) * n;
    for (int j = l; j < cnt; j += 32) m[list[j]] |= (uint8_t)(1 << t);  // a list holds each column once
    __syncwarp();
  }
  const uint32_t lt = (1u << l) - 1u;
  int total = 0;
  int* oi = u_idx + (size_t)gp * n;
  uint8_t* om = u_mem + (size_t)gp * n;
  for (int c0 = 0; c0 < n; c0 += 32) {
    const int c = c0 + l;
    const uint8_t b = c < n ? m[c] : 0;
    const uint32_t any = __ballot_sync(0xffffffffu, b != 0);
    if (b) {
      const int pos = total + __popc(any & lt);
      oi[pos] = c;
      om[pos] = b;
    }
    total += __popc(any);
  }
  if (l == 0) u_num[gp] = total;
}

}  // namespace
}  // namespace h3b

using namespace h3b;

extern "C" int h3b_tile_scores(const float* qp, const float* kp, int heads, int n, float scale, float* sc,
                               cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(heads > 0 && n > 0, "tile_scores: heads and n must be positive");
  H3B_REQUIRE(qp && kp && sc, "tile_scores: null pointer");
  H3B_REQUIRE(aligned(qp, 16) && aligned(kp, 16) && aligned(sc, 16), "tile_scores: 16-byte aligned buffers");
  const dim3 grid((n + SB - 1) / SB, (n + SB - 1) / SB, heads);
  scores_kernel<<<grid, 256, 0, stream>>>(qp, kp, n, scale, sc);
  H3B_LAUNCH_CHECK("tile_scores");
  return H3B_OK;
}

extern "C" int h3b_topk_rows(const float* scores, int heads, int n, int n_ext, int prefix, int n_spans,
                             const int* starts, const int* ends, const int* ks, int* idx, int* num, int split,
                             cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(scores && idx && num && (n_spans == 0 || (starts && ends && ks)), "topk_rows: null pointer");
  H3B_REQUIRE(n > 0 && n_ext >= n && prefix >= 0 && prefix <= n && heads > 0, "topk_rows: bad n / n_ext / prefix");
  H3B_REQUIRE(n_spans >= 0 && n_spans <= 4, "topk_rows: at most 4 spans");
  Spans sp{};
  sp.n = n_spans;
  int longest = 0;
  for (int s = 0; s < n_spans; ++s) {  // host arrays
    H3B_REQUIRE(starts[s] >= 0 && ends[s] <= n && starts[s] <= ends[s] && ks[s] >= 0, "topk_rows: bad span %d", s);
    sp.start[s] = starts[s];
    sp.end[s] = ends[s];
    sp.k[s] = ks[s];
    longest = longest > ends[s] - starts[s] ? longest : ends[s] - starts[s];
  }
  const int rows = heads * n;
  const int grid = (rows + 3) / 4;
#define H3B_TOPK(P) topk_kernel<P><<<grid, 128, 0, stream>>>(scores, n, n_ext, prefix, sp, rows, idx, num, split)
  if (longest <= 16 * 32) H3B_TOPK(16);
  else if (longest <= 32 * 32) H3B_TOPK(32);
  else if (longest <= 64 * 32) H3B_TOPK(64);
  else if (longest <= 160 * 32) H3B_TOPK(160);
  else return set_error(H3B_EINVAL, "topk_rows: span of %d tiles is too long (max 5120)", longest);
#undef H3B_TOPK
  H3B_LAUNCH_CHECK("topk_rows");
  return H3B_OK;
}

extern "C" int h3b_compressed_branch(const float* sc, const float* vp, int heads, int n, void* oc,
                                     cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(sc && vp && oc && heads > 0 && n > 0, "compressed_branch: bad arguments");
  H3B_REQUIRE((size_t)n * sizeof(float) <= 48 * 1024, "compressed_branch: n = %d tiles exceeds 12288", n);
  compressed_kernel<<<dim3(n, heads), 128, n * sizeof(float), stream>>>(sc, vp, n, static_cast<bf16*>(oc));
  H3B_LAUNCH_CHECK("compressed_branch");
  return H3B_OK;
}

extern "C" int h3b_topk_pairs(const float* scores, int heads, int n, int n_ext, int prefix, int n_spans,
                              const int* starts, const int* ends, const int* ks, int* idx, int* num, int* u_idx,
                              uint8_t* u_mem, int* u_num, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(idx && num && u_idx && u_mem && u_num, "topk_pairs: null pointer");
  H3B_REQUIRE(n_ext % 2 == 0, "topk_pairs: n_ext must be even");
  // a dense (prefix) query tile selects the prefix plus every span here and every column in topk_rows: the two agree
  // when the spans tile [prefix, n)
  int covered = prefix;
  for (int s = 0; s < n_spans; ++s) {
    H3B_REQUIRE(starts && ends && starts[s] == covered, "topk_pairs: the spans must tile [prefix, n) in order");
    covered = ends[s];
  }
  H3B_REQUIRE(covered == n, "topk_pairs: the spans must tile [prefix, n) in order");
  if (cudaMemsetAsync(num, 0, sizeof(int) * (size_t)heads * n_ext, stream) != cudaSuccess)
    return set_error(H3B_ECUDA, "topk_pairs: memset failed");
  if (const int rc = h3b_topk_rows(scores, heads, n, n_ext, prefix, n_spans, starts, ends, ks, idx, num, 0, stream))
    return rc;
  const int pairs = heads * (n_ext / 2);
  const size_t smem = (size_t)kUnionWarps * n;
  H3B_REQUIRE(smem <= 48 * 1024, "topk_pairs: n = %d tiles exceeds 12288", n);
  union_pairs_kernel<<<(pairs + kUnionWarps - 1) / kUnionWarps, kUnionWarps * 32, smem, stream>>>(
      idx, num, n, n_ext, pairs, u_idx, u_mem, u_num);
  H3B_LAUNCH_CHECK("topk_pairs");
  return H3B_OK;
}
