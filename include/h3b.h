/*
 * h3b: C ABI of the B200 (sm_100a) quantized DiT-block hot path.
 *
 * Conventions shared by every entry point:
 *   - pointers are device pointers unless a parameter says "host"; the caller allocates every buffer;
 *   - bf16 tensors are row-major with the stated leading dimension in elements;
 *   - e4m3 ("fp8") tensors are raw bytes (OCP E4M3, torch.float8_e4m3fn);
 *   - NVFP4 tensors are two e2m1 codes per byte, element 2i in the low nibble; their block scales are ue4m3 bytes
 *     (one per 16 consecutive K-elements) stored in 512-byte atoms of 128 rows x 4 scale columns
 *     (byte offset (r/128)*(K/64)*512 + (c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4), rows padded to 128;
 *   - every call is asynchronous on `stream` and returns 0 (H3B_OK) or an H3B_E* code; h3b_last_error() gives the
 *     message of the calling thread's last failure.
 *
 * Each declaration names the reference interface it replaces (chronarion/fasth3-gb300, FastVideo a01c50a overlay).
 */
#ifndef H3B_H_
#define H3B_H_

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3B_OK 0
#define H3B_EINVAL 1   /* bad argument: shape, alignment, null pointer, unsupported width */
#define H3B_ECUDA 2    /* a CUDA runtime call or launch failed */
#define H3B_ETIMEOUT 3 /* a kernel's bounded wait expired; see h3b_device_status */

/* Message of the calling thread's last failed call ("" if none). */
const char* h3b_last_error(void);
/* Library version string. */
const char* h3b_version(void);

/* ---------------------------------------------------------------------------------------------------------------
 * Row quantizers.
 * Replaces resid_norm_quant_op (fastvideo/models/dits/h3fast/h3fast.cu:831-858; kernel :188-265).
 *
 *   branch  (y != NULL):  x' = bf16(x + gate[idx[r]] * (sy[r] * y)), written to xo (xo may alias x)
 *   norm    (norm != H3B_NORM_NONE): v = norm(x') * nw * (1 + scale[idx[r]]) + shift[idx[r]]
 *           H3B_NORM_RMS: x' * rsqrt(mean(x'^2) + eps) * nw     (nw: bf16 [C])
 *           H3B_NORM_LAYER: (x' - mean) * rsqrt(var + eps)       (no affine; nw ignored)
 *   quant   (norm != NONE): per-row FP8 (hsf == NULL): hs[r] = max(amax/448, 1/(448*512)), h = e4m3(v * (1/hs[r]))
 *                           per-row NVFP4 (hsf != NULL): hs[r] = max(amax/(448*6), 1e-12), h = e2m1 codes [rows, C/2],
 *                           block scales into hsf (rows padded to 128).
 *   Tables shift/scale are bf16 rows of stride tab_ld elements selected by idx; gate rows have stride gate_ld.
 *   C must be one of 3072, 5120, 5376 (multiples of 1024 up to 8192 accepted).
 * ------------------------------------------------------------------------------------------------------------- */
#define H3B_NORM_NONE 0
#define H3B_NORM_RMS 1
#define H3B_NORM_LAYER 2

int h3b_resid_norm_quant(const void* x, const void* y, const float* sy, const void* gate, int64_t gate_ld,
                         const int32_t* idx, int norm, const void* nw, const void* shift, const void* scale,
                         int64_t tab_ld, void* xo, void* h, uint8_t* hsf, float* hs, float eps, int64_t rows, int C,
                         cudaStream_t stream);

/* Plain per-token FP8 quantizer of a bf16 matrix [rows, K] (leading dim ld):
 * s[r] = max(amax_r/448, 1/(448*512)), q = e4m3(x * (1/s[r])). The activation side of an FP8 linear
 * (same row formula as h3fast.cu:256-262). */
int h3b_quant_fp8_rows(const void* x, int64_t ld, int64_t rows, int K, void* q, float* s, cudaStream_t stream);

/* Per-tensor absolute maximum of a bf16 matrix [rows, K] (leading dim ld) folded into *amax with an atomic max
 * (as the bit pattern of a non-negative float). *amax must hold 0 or a previous partial maximum. */
int h3b_amax_bf16(const void* x, int64_t ld, int64_t rows, int K, float* amax, cudaStream_t stream);

/* NVFP4 quantizer with a per-tensor global scale (the block math of h3fast.cu:99-119 with
 * gs = 1/s): s = max(amax/(448*6), 1e-12) with amax read from device memory, q = e2m1 codes [rows, K/2],
 * sf = ue4m3 block scales in the 128x4 atom layout (rows padded to 128; padding rows are written as zero),
 * s_out[0] = s. K must be a multiple of 64. */
int h3b_quant_nvfp4_tensor(const void* x, int64_t ld, int64_t rows, int K, const float* amax, void* q, uint8_t* sf,
                           float* s_out, cudaStream_t stream);

/* One call of the two above: amax pass then quantization. `workspace` is device scratch of at least
 * h3b_quant_nvfp4_workspace_bytes() bytes, 256-byte aligned; the call zeroes it itself. */
size_t h3b_quant_nvfp4_workspace_bytes(void);
int h3b_quant_nvfp4(const void* x, int64_t ld, int64_t rows, int K, void* q, uint8_t* sf, float* s_out,
                    void* workspace, cudaStream_t stream);

/* h3b_quant_nvfp4 for callers that cannot allocate device memory (no counterpart in the reference). A host that
 * only hands the library the tensors it owns -- a plugin running inside an engine whose device memory is planned up
 * front, or a foreign-language host with a fixed buffer set -- cannot call cudaMalloc for a workspace mid-run. This
 * variant keeps its scratch in a 256-byte static device array (present on every GPU that loads the library until the
 * process exits) and allocates nothing. The first call on each device looks up the array's device address; make that
 * first call before any stream capture. Every call on a device shares the array and zeroes it first, so calls that
 * overlap on the GPU (e.g. on two streams) race and must be serialized by the caller. Same arguments and results as
 * h3b_quant_nvfp4 without the workspace; a build whose scratch need exceeds the array is rejected with H3B_EINVAL. */
int h3b_quant_nvfp4_noalloc(const void* x, int64_t ld, int64_t rows, int K, void* q, uint8_t* sf, float* s_out,
                            cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Offline weight packing.
 * FP8: replaces quantize_fp8_weight (patches/fastvideo-a01c50a.patch:384-394):
 *   channel: s[n] = max(amax_n/448, FP8_MIN_SCALE); wq = e4m3(clamp(bf16(w / bf16(s[n])), +-448))
 *   tensor:  s[0] = max(amax/448, FP8_MIN_SCALE);   wq = e4m3(clamp(bf16(w / bf16(s[0])), +-448))
 *   with FP8_MIN_SCALE = 1/(448*512). `workspace` (>= 256 bytes, 256-aligned) is used by the tensor mode only.
 * NVFP4: the packed-weight format FastVideo's NVFP4 linear reads (_nvfp4_weight [N, K/2], _nvfp4_weight_scale in the
 *   128x4 layout, _weight_global_sf) as consumed at fastvideo/models/dits/h3fast/__init__.py:393-402: per-tensor
 *   s = max(amax/(448*6), 1e-12), block math as h3b_quant_nvfp4. Same workspace rule as h3b_quant_nvfp4.
 * ------------------------------------------------------------------------------------------------------------- */
#define H3B_GRAN_TENSOR 0
#define H3B_GRAN_CHANNEL 1
int h3b_pack_weight_fp8(const void* w, int64_t N, int K, int granularity, void* wq, float* wscale, void* workspace,
                        cudaStream_t stream);
int h3b_pack_weight_nvfp4(const void* w, int64_t N, int K, void* wq, uint8_t* wsf, float* wscale, void* workspace,
                          cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * tcgen05 GEMMs with a fused epilogue.
 * FP8 replaces torch._scaled_mm(a, w.T, scale_a, scale_b) in H3FastRunner._gemm
 *   (fastvideo/models/dits/h3fast/__init__.py:378-392), NVFP4 replaces FlashInfer mm_fp4 (:393-404).
 *
 *   acc[m, n] = sum_k A[m, k] * B[n, k]                        (fp32 in tensor memory)
 *   v = acc * alpha * (row_scale ? row_scale[m] : 1) * (col_scale ? col_scale[n] : 1) + (bias ? bias[n] : 0)
 *   v = act(v)                                                 (H3B_ACT_GELU_TANH: 0.5 v (1 + tanh(0.79788456 (v + 0.044715 v^3))))
 *   out = residual ? residual[m, n] + gate[n] * v : v         (gate: bf16 [N], required with residual)
 *   D[m, n] = bf16(out)
 * A: [M, K] K-major, B: [N, K] K-major (FP8: bytes, NVFP4: packed nibbles with block scales in the 128x4 layout).
 * Requirements: K % 128 == 0 (FP8) or K % 256 == 0 (NVFP4); N % 16 == 0; 16-byte aligned base pointers;
 * ldd, ldr multiples of 8. M is arbitrary (rows past M are masked).
 * ------------------------------------------------------------------------------------------------------------- */
#define H3B_ACT_NONE 0
#define H3B_ACT_GELU_TANH 1

typedef struct h3b_epilogue {
  float alpha;
  const float* alpha_dev; /* device scalar multiplied into alpha (e.g. a per-tensor activation scale), or NULL */
  const float* row_scale; /* [M] or NULL */
  const float* col_scale; /* [N], or [1] when col_scale_scalar != 0, or NULL */
  int col_scale_scalar;
  const void* bias;       /* bf16 [N] or NULL */
  int act;                /* H3B_ACT_* */
  const void* residual;   /* bf16 [M, ldr] or NULL; may alias D */
  int64_t ldr;
  const void* gate;       /* bf16 [N]; required when residual != NULL */
  void* D;                /* bf16 [M, ldd] */
  int64_t ldd;
} h3b_epilogue;

int h3b_gemm_fp8(const void* A, const void* B, int64_t M, int64_t N, int64_t K, const h3b_epilogue* epi,
                 cudaStream_t stream);
int h3b_gemm_nvfp4(const void* A, const uint8_t* sfa, const void* B, const uint8_t* sfb, int64_t M, int64_t N,
                   int64_t K, const h3b_epilogue* epi, cudaStream_t stream);

/* Status word written by kernels whose bounded waits expired (0 = none since the last reset); reset with
 * h3b_reset_device_status. Both synchronize the current device. */
int h3b_device_status(int* status);
int h3b_reset_device_status(void);

#ifdef __cplusplus
}
#endif

#endif /* H3B_H_ */
