// Token reduction around an interval of DiT blocks (horizontal token pairing): the pooling of paired rows into the
// reduced residual stream and the expansion back to full rows (H3FastRunner._pool / _expand,
// fastvideo/models/dits/h3fast/__init__.py:280-293; the same arithmetic as pool_token_pairs / expand_token_pairs,
// fastvideo/models/dits/minimax_h3_token_reduction.py:124-150).
//
// Both are row gathers of bf16 rows, HBM-bound: one warp per output row at a time, each lane moving 16-byte pieces
// (512 contiguous bytes per warp instruction), grid sized to the resident warps. All arithmetic is float32 with IEEE
// rounding, rounded to bf16 once at the store, as torch evaluates the reference's expressions on float32 tensors.
#include "common.cuh"

#include <algorithm>

namespace h3b {
namespace {

constexpr int kRedWarps = 8;

// out[r] = bf16((x[ia[r]] + x[ib[r]]) * 0.5) in float32 (an unpaired row has ia == ib and is copied exactly);
// `pooled`, when given, receives the same rows (the expansion subtracts them from the reduced output).
__global__ void __launch_bounds__(kRedWarps * 32) pool_pairs_kernel(const bf16* __restrict__ x,
                                                                    const int32_t* __restrict__ ia,
                                                                    const int32_t* __restrict__ ib, int64_t rows,
                                                                    int C, bf16* __restrict__ out,
                                                                    bf16* __restrict__ pooled) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * kRedWarps;
  for (int64_t r = (int64_t)blockIdx.x * kRedWarps + (threadIdx.x >> 5); r < rows; r += nw) {
    const bf16* a = x + (int64_t)ia[r] * C;
    const bf16* b = x + (int64_t)ib[r] * C;
    for (int c = lane * 8; c < C; c += 256) {
      float fa[8], fb[8], v[8];
      load8(a + c, fa);
      load8(b + c, fb);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fadd_rn(fa[i], fb[i]), 0.5f);
      store8(out + r * C + c, v);
      if (pooled) store8(pooled + r * C + c, v);
    }
  }
}

// x[i] = pair[i] ? bf16(x[i] + scale * (xr[par[i]] - pooled[par[i]])) : xr[par[i]], float32 arithmetic; x is updated
// in place (each row reads and writes only itself).
__global__ void __launch_bounds__(kRedWarps * 32) expand_pairs_kernel(bf16* __restrict__ x, int64_t rows,
                                                                      const bf16* __restrict__ xr,
                                                                      const bf16* __restrict__ pooled,
                                                                      const int32_t* __restrict__ par,
                                                                      const uint8_t* __restrict__ pair, int C,
                                                                      float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * kRedWarps;
  for (int64_t i = (int64_t)blockIdx.x * kRedWarps + (threadIdx.x >> 5); i < rows; i += nw) {
    const int64_t p = par[i];
    const bool paired = pair[i] != 0;
    const bf16* src = xr + p * C;
    const bf16* pool = pooled + p * C;
    bf16* dst = x + i * C;
    for (int c = lane * 8; c < C; c += 256) {
      float v[8];
      if (paired) {
        float fr[8], fp[8], fx[8];
        load8(src + c, fr);
        load8(pool + c, fp);
        load8(dst + c, fx);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __fadd_rn(__fmul_rn(__fsub_rn(fr[k], fp[k]), scale), fx[k]);
      } else {
        load8(src + c, v);
      }
      store8(dst + c, v);
    }
  }
}

template <typename Kern>
unsigned warp_grid(Kern kern, int64_t rows) {
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRedWarps * 32, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int64_t need = (rows + kRedWarps - 1) / kRedWarps;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(need, (int64_t)sms * per_sm));
}

}  // namespace
}  // namespace h3b

using namespace h3b;

extern "C" int h3b_pool_pairs(const void* x, const int32_t* ia, const int32_t* ib, int64_t rows_out, int C, void* out,
                              void* pooled, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(x && ia && ib && out, "pool_pairs: null pointer");
  H3B_REQUIRE(C > 0 && C % 8 == 0 && rows_out >= 0, "pool_pairs: C must be a positive multiple of 8");
  H3B_REQUIRE(aligned(x, 16) && aligned(out, 16) && (!pooled || aligned(pooled, 16)), "pool_pairs: 16-byte rows");
  if (rows_out == 0) return H3B_OK;
  pool_pairs_kernel<<<warp_grid(pool_pairs_kernel, rows_out), kRedWarps * 32, 0, stream>>>(
      static_cast<const bf16*>(x), ia, ib, rows_out, C, static_cast<bf16*>(out), static_cast<bf16*>(pooled));
  H3B_LAUNCH_CHECK("pool_pairs");
  return H3B_OK;
}

extern "C" int h3b_expand_pairs(void* x, int64_t rows, const void* xr, const void* pooled, const int32_t* par,
                                const uint8_t* pair, int C, float scale, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(x && xr && pooled && par && pair, "expand_pairs: null pointer");
  H3B_REQUIRE(C > 0 && C % 8 == 0 && rows >= 0, "expand_pairs: C must be a positive multiple of 8");
  H3B_REQUIRE(aligned(x, 16) && aligned(xr, 16) && aligned(pooled, 16), "expand_pairs: 16-byte rows");
  if (rows == 0) return H3B_OK;
  expand_pairs_kernel<<<warp_grid(expand_pairs_kernel, rows), kRedWarps * 32, 0, stream>>>(
      static_cast<bf16*>(x), rows, static_cast<const bf16*>(xr), static_cast<const bf16*>(pooled), par, pair, C,
      scale);
  H3B_LAUNCH_CHECK("expand_pairs");
  return H3B_OK;
}
