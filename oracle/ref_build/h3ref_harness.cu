// TEST INFRASTRUCTURE ONLY: the reference's memory-bound kernels, compiled from the reference source where it lies
// (fastvideo/models/dits/h3fast/h3fast.cu, included read-only through -I, never copied) for sm_100a, so that a B200
// can produce golden outputs of the reference itself.
//
// Adds (1) definitions for the attention ops h3fast.cu declares but whose sources (h3attn8.cu, h3attn16*.cu) are not
// compiled here, raising if called; (2) extern "C" launchers of the reference templates at BASELINE.json's widths
// (C = 5120, attention width 5120 at 40 heads); (3) a per-tensor NVFP4 launcher that applies the reference's own block
// quantizer st_fp4x16 (h3fast.cu:121-138) with one global factor gs = 1/s for the whole tensor.
#include "h3fast.cu"

torch::Tensor vsa_fp8_op(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
                         double, torch::Tensor, torch::Tensor, std::optional<torch::Tensor>) {
  TORCH_CHECK(false, "h3ref harness: vsa_fp8 is not built for sm_100a");
}
torch::Tensor vsa_pair_op(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
                          torch::Tensor, double, std::optional<torch::Tensor>, std::optional<torch::Tensor>,
                          std::optional<torch::Tensor>) {
  TORCH_CHECK(false, "h3ref harness: vsa_pair is not built for sm_100a");
}
std::vector<torch::Tensor> vsa_bf16_op(torch::Tensor, torch::Tensor, torch::Tensor, c10::optional<torch::Tensor>,
                                       torch::Tensor, torch::Tensor, torch::Tensor, double, bool) {
  TORCH_CHECK(false, "h3ref harness: vsa_bf16 is not built here");
}
std::vector<torch::Tensor> vsa_bf16_blk128_op(torch::Tensor, torch::Tensor, torch::Tensor,
                                              c10::optional<torch::Tensor>, torch::Tensor, torch::Tensor,
                                              torch::Tensor, double, bool) {
  TORCH_CHECK(false, "h3ref harness: vsa_bf16_blk128 is not built here");
}

namespace {

__global__ void h3ref_amax_kernel(const bf16* __restrict__ x, int64_t n, float* __restrict__ out) {
  float m = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(__bfloat162float(x[i])));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(~0u, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(out), __float_as_int(m));
}

// One thread per 16-element block; the global factor is the tensor's, computed the way the row kernels compute theirs.
__global__ void h3ref_nvfp4_tensor_kernel(const bf16* __restrict__ x, int64_t rows, int K,
                                          const float* __restrict__ amax, uint8_t* __restrict__ q,
                                          uint8_t* __restrict__ sf, float* __restrict__ s_out) {
  const float s = fmaxf(*amax / kFp4Range, kMinScale4);
  const float gs = 1.f / s;
  const int blocks = K / 16;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i == 0) *s_out = s;
  if (i >= rows * blocks) return;
  const int64_t r = i / blocks;
  const int t = (int)(i % blocks);
  float f[2][8];
  ld8(x + r * K + t * 16, f[0]);
  ld8(x + r * K + t * 16 + 8, f[1]);
  st_fp4x16(q + r * (K / 2), sf, f, gs, r, t, blocks);
}

}  // namespace

extern "C" int h3ref_resid_norm_quant_5120(const void* x, const void* y, const float* sy, const void* gate,
                                           int64_t gate_ld, const int* idx, const void* nw, const void* shift,
                                           const void* scale, int64_t tab_ld, void* xo, void* h, uint8_t* hsf,
                                           float* hs, float eps, int64_t rows, cudaStream_t st) {
  constexpr int C = 5120;
  const bool branch = y != nullptr, norm = nw != nullptr, fp4 = hsf != nullptr;
#define H3REF_L(B, N, Q)                                                                                            \
  resid_norm_quant<C, B, N, Q, 1><<<(unsigned)rows, C / 8, 0, st>>>(                                                \
      (const bf16*)x, (const bf16*)y, sy, (const bf16*)gate, idx, (const bf16*)nw, (const bf16*)shift,              \
      (const bf16*)scale, gate_ld, tab_ld, (bf16*)xo, (fp8s*)h, hsf, hs, eps, rows)
  if (branch && norm) {
    if (fp4) H3REF_L(true, true, true);
    else H3REF_L(true, true, false);
  } else if (branch) {
    H3REF_L(true, false, false);
  } else if (fp4) {
    H3REF_L(false, true, true);
  } else {
    H3REF_L(false, true, false);
  }
#undef H3REF_L
  return (int)cudaGetLastError();
}

extern "C" int h3ref_quant_nvfp4_tensor(const void* x, int64_t rows, int K, float* amax_ws, void* q, uint8_t* sf,
                                        float* s_out, cudaStream_t st) {
  cudaMemsetAsync(amax_ws, 0, sizeof(float), st);
  h3ref_amax_kernel<<<256, 256, 0, st>>>((const bf16*)x, rows * K, amax_ws);
  const int64_t n = rows * (K / 16);
  h3ref_nvfp4_tensor_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const bf16*)x, rows, K, amax_ws,
                                                                        (uint8_t*)q, sf, s_out);
  return (int)cudaGetLastError();
}

extern "C" int h3ref_attn_gate_quant_5120(const void* ob, const void* g, const float* sg, const void* oc,
                                          const int* slot, int64_t rows_pad, int n_tiles, int tile, void* a,
                                          uint8_t* asf, float* sa, int64_t rows, cudaStream_t st) {
  constexpr int W = 5120;
  const bool gate = g != nullptr, fp4 = asf != nullptr;
#define H3REF_G(G, Q)                                                                                               \
  attn_gate_quant<W, G, Q, false><<<(unsigned)rows, W / 8, 0, st>>>(                                                \
      (const bf16*)ob, (const bf16*)g, sg, (const bf16*)oc, slot, rows_pad, n_tiles, tile, (fp8s*)a, asf, sa, nullptr, \
      nullptr, nullptr, 0, nullptr)
  if (gate) {
    if (fp4) H3REF_G(true, true);
    else H3REF_G(true, false);
  } else if (fp4) {
    H3REF_G(false, true);
  } else {
    H3REF_G(false, false);
  }
#undef H3REF_G
  return (int)cudaGetLastError();
}
