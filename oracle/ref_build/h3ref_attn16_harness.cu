// TEST INFRASTRUCTURE ONLY: the reference's BF16 VSA block-sparse attention (FastVideo's Blackwell kernel as vendored
// by the reference: fastvideo/models/dits/h3fast/h3attn16.cu, vsa_bf16.cuh, vsa_bf16_launch.cuh), compiled from the
// reference source where it lies (included read-only through -I, never copied) for sm_100a with VSA_LDRED off --
// tcgen05.ld.red, its default row-maximum path, exists on sm_103a only. It is the timing bar for this library's FP8
// attention on the same B200 and is never part of the product.
#define VSA_LDRED false
#include "h3attn16.cu"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("vsa_bf16", &vsa_bf16_op, "the reference's BF16 VSA forward (64-token blocks, [B, H, S, D])");
}
