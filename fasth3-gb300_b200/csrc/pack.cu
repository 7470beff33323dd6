// Offline weight packing: FP8 e4m3 with per-channel or per-tensor scales, and NVFP4 (e2m1 + ue4m3 block scales in the
// 128x4 atom layout + an fp32 per-tensor scale).
//
// Built WITHOUT fast math: the FP8 path restates quantize_fp8_weight (patches/fastvideo-a01c50a.patch:384-394), which
// torch evaluates with IEEE division, and it keeps torch's rounding steps: the scale is rounded to the weight dtype
// (bf16) before the division, the quotient is rounded to bf16, clamped to +-448, then rounded to e4m3.
#include "common.cuh"

#include <algorithm>

namespace h3b {

int amax_launch(const bf16* x, int64_t ld, int64_t rows, int K, float* amax, cudaStream_t st);
int quant_nvfp4_tensor_launch(const bf16* x, int64_t ld, int64_t rows, int K, const float* amax, uint8_t* q,
                              uint8_t* sf, float* s_out, cudaStream_t st);

namespace {

__device__ __forceinline__ uint32_t pack_one(float w, float sbf) {
  float v = __bfloat162float(__float2bfloat16_rn(w / sbf));
  v = fminf(fmaxf(v, -kFp8Max), kFp8Max);
  return (uint32_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

// One CTA per output channel. With `global_amax` the row uses the tensor's scale instead of its own.
__global__ void __launch_bounds__(256) pack_fp8_kernel(const bf16* __restrict__ w, int K, const float* global_amax,
                                                       uint8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ float stage[32];
  const int64_t n = blockIdx.x;
  const bf16* row = w + n * K;
  float am;
  if (global_amax) {
    am = *global_amax;
  } else {
    am = 0.f;
    for (int c = threadIdx.x * 8; c < K; c += 256 * 8) {
      float f[8];
      load8(row + c, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(f[i]));
    }
    am = block_allreduce<8, true>(am, stage);
  }
  const float s = fmaxf(am / kFp8Max, kMinScaleFp8);
  const float sbf = __bfloat162float(__float2bfloat16_rn(s));
  for (int c = threadIdx.x * 8; c < K; c += 256 * 8) {
    float f[8];
    load8(row + c, f);
    uint2 o;
    o.x = pack_one(f[0], sbf) | (pack_one(f[1], sbf) << 8) | (pack_one(f[2], sbf) << 16) | (pack_one(f[3], sbf) << 24);
    o.y = pack_one(f[4], sbf) | (pack_one(f[5], sbf) << 8) | (pack_one(f[6], sbf) << 16) | (pack_one(f[7], sbf) << 24);
    *reinterpret_cast<uint2*>(q + n * K + c) = o;
  }
  if (threadIdx.x == 0) {
    if (!global_amax) scale[n] = s;
    else if (n == 0) scale[0] = s;
  }
}

// LoRA merge on the base weight's FP8 grid (fastvideo/models/dits/h3fast/__init__.py:82-92, `_on_grid`): the merged
// fp32 weight keeps the base scale s0 of its row (or tensor) while amax <= 1.05 * 448 * s0 -- evaluated as torch does
// for a float32 tensor and a Python scalar: fl32(470.4f * s0) -- and otherwise gets its own max(amax / 448, 1e-12);
// codes are e4m3(clamp(m / s, +-448)) with IEEE division. One CTA per row; `tensor_amax` set selects the tensor form.
__global__ void __launch_bounds__(256) fp8_on_grid_kernel(const float* __restrict__ m, int K,
                                                          const float* __restrict__ base, const float* tensor_amax,
                                                          uint8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ float stage[32];
  const int64_t n = blockIdx.x;
  const float* row = m + n * K;
  float am;
  if (tensor_amax) {
    am = *tensor_amax;
  } else {
    am = 0.f;
    for (int c = threadIdx.x * 4; c < K; c += 256 * 4) {
      const float4 f = *reinterpret_cast<const float4*>(row + c);
      am = fmaxf(am, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
    }
    am = block_allreduce<8, true>(am, stage);
  }
  const float s0 = tensor_amax ? base[0] : base[n];
  const float lim = __fmul_rn(470.4f, s0);
  const float s = am <= lim ? s0 : fmaxf(__fdiv_rn(am, kFp8Max), 1e-12f);
  for (int c = threadIdx.x * 4; c < K; c += 256 * 4) {
    const float4 f = *reinterpret_cast<const float4*>(row + c);
    const float v[4] = {f.x, f.y, f.z, f.w};
    uint32_t o = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x = fminf(fmaxf(__fdiv_rn(v[i], s), -kFp8Max), kFp8Max);
      o |= (uint32_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3) << (8 * i);
    }
    *reinterpret_cast<uint32_t*>(q + n * K + c) = o;
  }
  if (threadIdx.x == 0) {
    if (!tensor_amax) scale[n] = s;
    else if (n == 0) scale[0] = s;
  }
}

// max |x| over an fp32 matrix into *amax (non-negative floats order like their bit patterns as integers).
__global__ void __launch_bounds__(256) amax_f32_kernel(const float* __restrict__ x, int64_t n, float* amax) {
  __shared__ float stage[32];
  float am = 0.f;
  for (int64_t i = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 4; i < n; i += (int64_t)gridDim.x * 256 * 4) {
    const float4 f = *reinterpret_cast<const float4*>(x + i);
    am = fmaxf(am, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
  }
  am = block_allreduce<8, true>(am, stage);
  if (threadIdx.x == 0 && am > 0.f) atomicMax(reinterpret_cast<int*>(amax), __float_as_int(am));
}

}  // namespace
}  // namespace h3b

using namespace h3b;

extern "C" int h3b_quant_fp8_on_grid(const float* merged, int64_t N, int K, const float* base_scale, int per_row,
                                     void* wq, float* wscale, void* workspace, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(merged && base_scale && wq && wscale, "quant_fp8_on_grid: null pointer");
  H3B_REQUIRE(K > 0 && K % 4 == 0 && N >= 0, "quant_fp8_on_grid: K must be a positive multiple of 4");
  H3B_REQUIRE(aligned(merged, 16) && aligned(wq, 4), "quant_fp8_on_grid: merged 16-byte, wq 4-byte aligned");
  if (N == 0) return H3B_OK;
  const float* tam = nullptr;
  if (!per_row) {
    H3B_REQUIRE(workspace && aligned(workspace, 256), "quant_fp8_on_grid: tensor mode needs a 256-byte aligned workspace");
    float* amax = static_cast<float*>(workspace);
    if (cudaMemsetAsync(amax, 0, sizeof(float), stream) != cudaSuccess)
      return set_error(H3B_ECUDA, "quant_fp8_on_grid: workspace memset failed");
    const int64_t n = N * (int64_t)K;
    const int64_t blocks = std::min<int64_t>((n / 4 + 255) / 256, 148 * 8);
    amax_f32_kernel<<<(unsigned)blocks, 256, 0, stream>>>(merged, n, amax);
    H3B_LAUNCH_CHECK("quant_fp8_on_grid (amax)");
    tam = amax;
  }
  fp8_on_grid_kernel<<<(unsigned)N, 256, 0, stream>>>(merged, K, base_scale, tam, static_cast<uint8_t*>(wq), wscale);
  H3B_LAUNCH_CHECK("quant_fp8_on_grid");
  return H3B_OK;
}

extern "C" int h3b_pack_weight_fp8(const void* w, int64_t N, int K, int granularity, void* wq, float* wscale,
                                   void* workspace, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(w && wq && wscale, "pack_weight_fp8: null pointer");
  H3B_REQUIRE(granularity == H3B_GRAN_TENSOR || granularity == H3B_GRAN_CHANNEL, "pack_weight_fp8: granularity %d",
              granularity);
  H3B_REQUIRE(K > 0 && K % 8 == 0 && N >= 0, "pack_weight_fp8: K must be a positive multiple of 8");
  H3B_REQUIRE(aligned(w, 16) && aligned(wq, 8), "pack_weight_fp8: w 16-byte, wq 8-byte aligned");
  if (N == 0) return H3B_OK;
  const float* gam = nullptr;
  if (granularity == H3B_GRAN_TENSOR) {
    H3B_REQUIRE(workspace && aligned(workspace, 256), "pack_weight_fp8: tensor mode needs a 256-byte aligned workspace");
    float* amax = static_cast<float*>(workspace);
    if (cudaMemsetAsync(amax, 0, sizeof(float), stream) != cudaSuccess)
      return set_error(H3B_ECUDA, "pack_weight_fp8: workspace memset failed");
    int rc = amax_launch(static_cast<const bf16*>(w), K, N, K, amax, stream);
    if (rc) return rc;
    gam = amax;
  }
  pack_fp8_kernel<<<(unsigned)N, 256, 0, stream>>>(static_cast<const bf16*>(w), K, gam, static_cast<uint8_t*>(wq),
                                                    wscale);
  H3B_LAUNCH_CHECK("pack_weight_fp8");
  return H3B_OK;
}

extern "C" int h3b_pack_weight_nvfp4(const void* w, int64_t N, int K, void* wq, uint8_t* wsf, float* wscale,
                                     void* workspace, cudaStream_t stream) {
  clear_error();
  H3B_REQUIRE(w && wq && wsf && wscale, "pack_weight_nvfp4: null pointer");
  H3B_REQUIRE(K > 0 && K % 64 == 0 && N >= 0, "pack_weight_nvfp4: K must be a positive multiple of 64");
  H3B_REQUIRE(workspace && aligned(workspace, 256), "pack_weight_nvfp4: needs a 256-byte aligned workspace");
  H3B_REQUIRE(aligned(w, 16) && aligned(wq, 16) && aligned(wsf, 4), "pack_weight_nvfp4: w, wq 16-byte, wsf 4-byte aligned");
  float* amax = static_cast<float*>(workspace);
  if (cudaMemsetAsync(amax, 0, sizeof(float), stream) != cudaSuccess)
    return set_error(H3B_ECUDA, "pack_weight_nvfp4: workspace memset failed");
  if (N == 0) return H3B_OK;
  int rc = amax_launch(static_cast<const bf16*>(w), K, N, K, amax, stream);
  if (rc) return rc;
  return quant_nvfp4_tensor_launch(static_cast<const bf16*>(w), K, N, K, amax, static_cast<uint8_t*>(wq), wsf,
                                   wscale, stream);
}
