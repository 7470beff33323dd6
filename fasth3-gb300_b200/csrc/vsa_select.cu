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
  // thread (ty, tx) owns rows 8ty.. and columns 8tx.. of the block; a warp covers 4 values of ty and 8 of tx (a 32 x 64
  // sub-block), so its shared-memory reads per d touch 32 q and 64 k values (one wavefront each) instead of 16 and 128
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ty = (warp >> 1) * 4 + (lane >> 3), tx = (warp & 1) * 8 + (lane & 7);
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
        for (int b = 0; b < 8; b += 2) fma2_acc_rn(acc[a][b], acc[a][b + 1], av[a], av[a], bv[b], bv[b + 1]);
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
// Selection semantics (the interface of topk_rows, fastvideo/models/dits/h3fast/h3fast.cu:524-588): query tiles below
// `prefix` are dense (every column, or nothing in split mode); any other row keeps the prefix columns (unless split),
// then per span the k largest scores under the order-preserving map of the float bits to uint32 (so -0.0 < +0.0 and
// NaNs sort by their bits), ties going to the lowest column, the kept columns written in ascending order.
//
// Algorithm (one warp per row and span; the span's keys -- the order-preserving uint32 map of the float bits -- in
// registers, PER per lane at column p * 32 + lane):
//   1. one read of the span, tracking each lane's smallest and largest key;
//   2. a lower bound L with at least k keys >= L, and a candidate list of the keys >= L with their columns, gathered
//      into shared memory in ascending column order (ballot compaction):
//        k <= 32: L = the smallest of the 32 lanes' largest keys (32 distinct keys are >= L); for N(0, 1)-like scores
//                 about 5% of a 2016-column span survive;
//        k > 32:  a 256-bucket histogram of the values over the span's finite range, bucket = min(255,
//                 uint(fma(v, 256 / (hi - lo), -lo * 256 / (hi - lo)))), non-decreasing in v (a span with a NaN puts
//                 everything in bucket 0); the list holds the buckets from the one containing the k-th largest up;
//   3. exact selection on the list by most-significant-digit radix levels over a key interval [lo, hi]: each level
//      histograms the list keys inside the interval by (key - lo) >> shift (256 buckets spanning the interval), finds
//      the bucket holding the `need`-th largest, drops the keys above it from `need` and narrows the interval to that
//      bucket. Every level removes at least 8 bits of the interval's width, so at most four levels leave a single key:
//      the threshold t, the k-th largest key of the span. The list entries equal to t are kept up to the `need`-th
//      in column order;
//   4. the list is written out in order: keys above t, and keys equal to t up to the last kept column.
// A span whose list would exceed 512 entries (heavy ties at the bound, or k > 32 with a wide boundary bucket) runs the
// same radix levels over the keys in registers instead, and writes its output from the registers.
struct Spans {
  int n;
  int start[4];
  int end[4];
  int k[4];
};

constexpr int kSelWarps = 4;     // rows per CTA
constexpr int kBuckets = 256;
constexpr int kListCap = 512;    // candidate list entries per warp
constexpr int kLaneBoundK = 32;  // k up to which the lane-maximum bound is used

__device__ __forceinline__ uint32_t order_key(uint32_t u) {
  return u ^ ((uint32_t)((int32_t)u >> 31) | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t key) {  // the inverse map
  return __uint_as_float(key ^ ((key & 0x80000000u) ? 0x80000000u : 0xffffffffu));
}

__device__ __forceinline__ uint32_t value_bucket(uint32_t key, float sc, float off) {
  return min(__float2uint_rz(__fmaf_rn(key_value(key), sc, off)), (uint32_t)(kBuckets - 1));
}

// The bucket holding the need-th largest entry of the histogram (counted from the top bucket down) and the number of
// entries in the buckets above it. Lane l sums buckets 8l .. 8l+7; suffix sums across lanes locate the lane.
__device__ __forceinline__ void boundary_bucket(const int* hist, int need, int& b, int& above) {
  const int lane = threadIdx.x & 31;
  const int4 h0 = *reinterpret_cast<const int4*>(hist + 8 * lane);
  const int4 h1 = *reinterpret_cast<const int4*>(hist + 8 * lane + 4);
  const int hb[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  int own = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) own += hb[j];
  int suffix = own;  // entries in buckets >= 8 * lane
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_down_sync(0xffffffffu, suffix, o);
    if (lane + o < 32) suffix += t;
  }
  const uint32_t reach = __ballot_sync(0xffffffffu, suffix >= need);  // lanes 0 .. L (suffix does not increase)
  const int L = 31 - __clz(reach);
  int higher = __shfl_down_sync(0xffffffffu, suffix, 1);  // entries in buckets >= 8 * (lane + 1)
  if (lane == 31) higher = 0;
  int bb = 0, ab = 0;
  if (lane == L) {
    int acc = higher;
#pragma unroll
    for (int j = 7; j >= 0; --j) {
      if (acc + hb[j] >= need) {
        bb = 8 * lane + j;
        ab = acc;
        break;
      }
      acc += hb[j];
    }
  }
  b = __shfl_sync(0xffffffffu, bb, L);
  above = __shfl_sync(0xffffffffu, ab, L);
}

// One radix level: `hist` holds the counts of the active keys (those in [lo, hi]) by (key - lo) >> shift. Narrows
// [lo, hi] to the bucket holding the need-th largest active key and takes the keys above it off `need`.
__device__ __forceinline__ void narrow(const int* hist, int shift, int& need, uint32_t& lo, uint32_t& hi) {
  int b, above;
  boundary_bucket(hist, need, b, above);
  need -= above;
  const uint32_t nlo = lo + ((uint32_t)b << shift);
  const uint32_t width = (1u << shift) - 1u;
  hi = (hi - nlo > width) ? nlo + width : hi;
  lo = nlo;
}

// Digits of one level: 256 buckets cover [lo, hi].
__device__ __forceinline__ int level_shift(uint32_t lo, uint32_t hi) {
  const int bits = 32 - __clz(hi - lo);
  return bits > 8 ? bits - 8 : 0;
}

// Selects the k largest of scores[start, start + len) and appends their columns (ascending) at out[cnt..]. FULL: the
// span is exactly 32 * PER long (every register slot holds a key; no per-slot bounds checks).
template <int PER, bool FULL>
__device__ __forceinline__ void select_span(const float* __restrict__ srow, int start, int len, int k,
                                            int* __restrict__ out, int& cnt, int* hist, uint32_t* lkey, int* lcol) {
  const int lane = threadIdx.x & 31;
  const uint32_t below = (1u << lane) - 1u;
  if (k <= 0 || len <= 0) return;
  if (k >= len) {
    for (int c = lane; c < len; c += 32) out[cnt + c] = start + c;
    cnt += len;
    return;
  }
  // 1. the span's keys: every load is issued before the first is used
  auto valid = [&](int p) { return FULL || p * 32 + lane < len; };
  auto live = [&](int p) { return FULL || p * 32 < len; };  // warp-uniform: slot p holds keys in some lane
  uint32_t key[PER];
#pragma unroll
  for (int p = 0; p < PER; ++p) key[p] = valid(p) ? __float_as_uint(srow[start + p * 32 + lane]) : 0u;
  uint32_t kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    if (valid(p)) {
      key[p] = order_key(key[p]);
      kmin = min(kmin, key[p]);
      kmax = max(kmax, key[p]);
    }
  }
  // 2. lower bound and candidate list; [lo, hi] = the key interval still undecided, `need` = keys wanted from it
  int need = k, n_list = 0;
  uint32_t lo, hi;
  bool listed = false;
  if (k <= kLaneBoundK) {
    const uint32_t bound = __reduce_min_sync(0xffffffffu, len >= 32 ? kmax : 0u);
    lo = bound;
    hi = __reduce_max_sync(0xffffffffu, kmax);
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      if (!live(p)) break;
      const int c = p * 32 + lane;
      const bool in = valid(p) && key[p] >= bound;
      const uint32_t m = __ballot_sync(0xffffffffu, in);
      const int pos = n_list + __popc(m & below);
      if (in && pos < kListCap) {
        lkey[pos] = key[p];
        lcol[pos] = c;
      }
      n_list += __popc(m);
    }
    listed = n_list <= kListCap;
  } else {
    float vlo = INFINITY, vhi = -INFINITY;
    bool nan = false;
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      if (!live(p)) break;
      if (valid(p)) {
        const float v = key_value(key[p]);
        if (fabsf(v) < INFINITY) {
          vlo = fminf(vlo, v);
          vhi = fmaxf(vhi, v);
        }
        nan |= v != v;
      }
    }
    vlo = -warp_allreduce<true>(-vlo);
    vhi = warp_allreduce<true>(vhi);
    nan = __any_sync(0xffffffffu, nan);
    float sc = 0.f, off = 0.f;
    if (!nan && vhi > vlo && vhi - vlo < INFINITY) {
      sc = 256.f / (vhi - vlo);
      off = -vlo * sc;
      if (!(sc < INFINITY)) sc = 0.f, off = 0.f;
    }
    for (int i = lane; i < kBuckets; i += 32) hist[i] = 0;
    __syncwarp();
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      if (!live(p)) break;
      if (valid(p)) atomicAdd(&hist[value_bucket(key[p], sc, off)], 1);
    }
    __syncwarp();
    int b, above;
    boundary_bucket(hist, k, b, above);
    const int total = above + hist[b];
    __syncwarp();  // hist is reused by the radix levels
    if (total <= kListCap) {
      uint32_t blo = 0xffffffffu, bhi = 0u;
#pragma unroll
      for (int p = 0; p < PER; ++p) {
        if (!live(p)) break;
        const int c = p * 32 + lane;
        const uint32_t vb = valid(p) ? value_bucket(key[p], sc, off) : 0u;
        const bool in = valid(p) && vb >= (uint32_t)b;
        const uint32_t m = __ballot_sync(0xffffffffu, in);
        if (in) {
          const int pos = n_list + __popc(m & below);
          lkey[pos] = key[p];
          lcol[pos] = c;
          if (vb == (uint32_t)b) {
            blo = min(blo, key[p]);
            bhi = max(bhi, key[p]);
          }
        }
        n_list += __popc(m);
      }
      lo = __reduce_min_sync(0xffffffffu, blo);
      hi = __reduce_max_sync(0xffffffffu, bhi);
      need = k - above;  // every key of a higher bucket exceeds every key of bucket b
      listed = true;
    }
  }
  // 3. radix levels down to one key t; tie_last = the last column kept among the keys equal to t
  uint32_t t;
  int tie_last = -1;
  if (listed) {
    __syncwarp();
#pragma unroll 1
    for (int level = 0; level < 5 && lo != hi; ++level) {
      const int shift = level_shift(lo, hi);
      for (int i = lane; i < kBuckets; i += 32) hist[i] = 0;
      __syncwarp();
      for (int i = lane; i < n_list; i += 32) {
        const uint32_t kk = lkey[i];
        if (kk >= lo && kk <= hi) atomicAdd(&hist[(kk - lo) >> shift], 1);
      }
      __syncwarp();
      narrow(hist, shift, need, lo, hi);
      __syncwarp();
    }
    t = lo;
    int seen = 0;
    for (int base = 0; base < n_list; base += 32) {
      const int i = base + lane;
      const bool eq = i < n_list && lkey[i] == t;
      const uint32_t m = __ballot_sync(0xffffffffu, eq);
      const uint32_t hit = __ballot_sync(0xffffffffu, eq && seen + __popc(m & below) + 1 == need);
      if (hit) {
        tie_last = lcol[base + __ffs(hit) - 1];
        break;
      }
      seen += __popc(m);
    }
    // 4. the kept list entries, in column order
    for (int base = 0; base < n_list; base += 32) {
      const int i = base + lane;
      bool keep = false;
      int c = 0;
      if (i < n_list) {
        const uint32_t kk = lkey[i];
        c = lcol[i];
        keep = kk > t || (kk == t && c <= tie_last);
      }
      const uint32_t m = __ballot_sync(0xffffffffu, keep);
      if (keep) out[cnt + __popc(m & below)] = start + c;
      cnt += __popc(m);
    }
    __syncwarp();  // the list is reused by the next span
    return;
  }
  // the same levels over the keys in registers
  lo = __reduce_min_sync(0xffffffffu, kmin);
  hi = __reduce_max_sync(0xffffffffu, kmax);
  need = k;
#pragma unroll 1
  for (int level = 0; level < 5 && lo != hi; ++level) {
    const int shift = level_shift(lo, hi);
    for (int i = lane; i < kBuckets; i += 32) hist[i] = 0;
    __syncwarp();
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      if (!live(p)) break;
      if (valid(p) && key[p] >= lo && key[p] <= hi) atomicAdd(&hist[(key[p] - lo) >> shift], 1);
    }
    __syncwarp();
    narrow(hist, shift, need, lo, hi);
    __syncwarp();
  }
  t = lo;
  int seen = 0;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    if (!live(p) || tie_last >= 0) break;
    const int c = p * 32 + lane;
    const bool eq = valid(p) && key[p] == t;
    const uint32_t m = __ballot_sync(0xffffffffu, eq);
    const uint32_t hit = __ballot_sync(0xffffffffu, eq && seen + __popc(m & below) + 1 == need);
    if (hit) tie_last = p * 32 + __ffs(hit) - 1;
    seen += __popc(m);
  }
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    if (!live(p)) break;
    const int c = p * 32 + lane;
    const bool keep = valid(p) && (key[p] > t || (key[p] == t && c <= tie_last));
    const uint32_t m = __ballot_sync(0xffffffffu, keep);
    if (keep) out[cnt + __popc(m & below)] = start + c;
    cnt += __popc(m);
  }
}

// One warp per (head, query tile) row; PER = keys per lane (span length <= 32 * PER).
template <int PER, bool FULL>
__global__ void __launch_bounds__(kSelWarps * 32, PER <= 32 ? 4 : (PER <= 64 ? 3 : 1)) select_kernel(const float* __restrict__ scores, int n, int n_ext,
                                                                int prefix, Spans sp, int rows, int* __restrict__ idx,
                                                                int* __restrict__ num, int split) {
  __shared__ __align__(16) int hist[kSelWarps][kBuckets];
  __shared__ uint32_t lkey[kSelWarps][kListCap];
  __shared__ int lcol[kSelWarps][kListCap];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kSelWarps + w;
  if (row >= rows) return;  // warp-uniform; the CTA's warps never synchronise with each other
  const int hh = row / n, q = row - hh * n;
  int* out = idx + ((size_t)hh * n_ext + q) * n;
  int* count = num + (size_t)hh * n_ext + q;
  if (q < prefix) {  // a dense query tile
    if (!split)
      for (int c = lane; c < n; c += 32) out[c] = c;
    if (lane == 0) *count = split ? 0 : n;
    return;
  }
  int cnt = 0;
  if (!split) {
    for (int c = lane; c < prefix; c += 32) out[c] = c;
    cnt = prefix;
  }
  const float* srow = scores + (size_t)row * n;
  for (int s = 0; s < sp.n; ++s)
    select_span<PER, FULL>(srow, sp.start[s], sp.end[s] - sp.start[s], sp.k[s], out, cnt, hist[w], lkey[w], lcol[w]);
  if (lane == 0) *count = cnt;
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
  const int grid = (rows + kSelWarps - 1) / kSelWarps;
#define H3B_SELECT(P, F) \
  select_kernel<P, F><<<grid, kSelWarps * 32, 0, stream>>>(scores, n, n_ext, prefix, sp, rows, idx, num, split)
  // one span of exactly 32 * PER columns (BASELINE's 512- and 2016-tile layouts): the check-free instantiation
  const bool one = n_spans == 1;
  if (one && longest == 16 * 32) H3B_SELECT(16, true);
  else if (one && longest == 63 * 32) H3B_SELECT(63, true);
  else if (one && longest == 64 * 32) H3B_SELECT(64, true);
  else if (longest <= 16 * 32) H3B_SELECT(16, false);
  else if (longest <= 32 * 32) H3B_SELECT(32, false);
  else if (longest <= 64 * 32) H3B_SELECT(64, false);
  else if (longest <= 160 * 32) H3B_SELECT(160, false);
  else return set_error(H3B_EINVAL, "topk_rows: span of %d tiles is too long (max 5120)", longest);
#undef H3B_SELECT
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
