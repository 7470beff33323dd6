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

/* Per-row NVFP4 quantizer of a bf16 matrix [rows, K] (leading dim ld), any K multiple of 64: s_rows[r] =
 * max(amax_r/(448*6), 1e-12), block math of h3fast.cu:121-138 with gs = 1/s_rows[r] (the reference's per-row FP4
 * output of swiglu_quant / attn_gate_quant / resid_norm_quant, here for the FFN intermediate of any width). The padding
 * rows of sf are not written. */
int h3b_quant_nvfp4_rows(const void* x, int64_t ld, int64_t rows, int K, void* q, uint8_t* sf, float* s_rows,
                         cudaStream_t stream);

/* One call of the two above: amax pass then quantization. `workspace` is device scratch of at least
 * h3b_quant_nvfp4_workspace_bytes() bytes, 256-byte aligned; the call zeroes it itself. */
size_t h3b_quant_nvfp4_workspace_bytes(void);
int h3b_quant_nvfp4(const void* x, int64_t ld, int64_t rows, int K, void* q, uint8_t* sf, float* s_out,
                    void* workspace, cudaStream_t stream);

/* h3b_quant_nvfp4 for callers that cannot allocate device memory (no counterpart in the reference). A host that
 * only hands the library the tensors it owns -- a plugin running inside an engine whose device memory is planned up
 * front, or a foreign-language host with a fixed buffer set -- cannot call cudaMalloc for a workspace mid-run. This
 * variant keeps its scratch in a 256-byte static device array (present on every GPU that loads the library until the
 * process exits) and allocates nothing. The first call on each device looks up the array's device address (and so
 * does the first call after the thread's context on that device changed, e.g. after cudaDeviceReset); make that first
 * call before any stream capture. Every call on a device shares the array and zeroes it first, so calls that
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

/* LoRA merge on the base weight's FP8 grid: replaces `_on_grid` (fastvideo/models/dits/h3fast/__init__.py:82-92),
 * which H3FastRunner._merged_fp8 (:354-376) applies to W + scale * B @ A (merged in fp32). merged fp32 [N, K];
 * base_scale fp32 [N] (per_row = 1) or [1] (per_row = 0). Per row (or for the tensor): amax = max|merged|;
 * s = base_scale when amax <= fl32(470.4f * base_scale), else max(amax / 448, 1e-12); wq = e4m3(clamp(merged / s,
 * +-448)) with IEEE division; wscale = s. `workspace` (>= 256 bytes, 256-aligned) is used when per_row = 0. */
int h3b_quant_fp8_on_grid(const float* merged, int64_t N, int K, const float* base_scale, int per_row, void* wq,
                          float* wscale, void* workspace, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Token reduction around an interval of blocks (horizontal pairs of video tokens): replace H3FastRunner._pool and
 * _expand (fastvideo/models/dits/h3fast/__init__.py:280-293), whose arithmetic is pool_token_pairs /
 * expand_token_pairs (fastvideo/models/dits/minimax_h3_token_reduction.py:124-150). Rows are bf16 [*, C], C % 8 == 0,
 * 16-byte aligned; float32 arithmetic, one bf16 rounding at the store.
 *   pool:   out[r] = (x[ia[r]] + x[ib[r]]) * 0.5 for r < rows_out (ia == ib copies); pooled (may be NULL) gets the same.
 *   expand: x[i] = pair[i] ? x[i] + scale * (xr[par[i]] - pooled[par[i]]) : xr[par[i]] for i < rows (in place).
 * ------------------------------------------------------------------------------------------------------------- */
int h3b_pool_pairs(const void* x, const int32_t* ia, const int32_t* ib, int64_t rows_out, int C, void* out,
                   void* pooled, cudaStream_t stream);
int h3b_expand_pairs(void* x, int64_t rows, const void* xr, const void* pooled, const int32_t* par,
                     const uint8_t* pair, int C, float scale, cudaStream_t stream);

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
/* NVFP4 GEMM whose epilogue re-quantizes its output for the next NVFP4 GEMM instead of storing bf16 (the reference
 * writes the fc_in output and re-quantizes it in a separate pass, fastvideo/models/dits/h3fast/h3fast.cu:781-817, with
 * a per-row global scale that needs the whole row). Each output value (alpha, row/col scales, bias, activation as in
 * h3b_gemm_nvfp4) is rounded to bf16 -- the value a bf16 output would hold -- and encoded with the activation
 * quantizers' block math under a FIXED global scale s = *q_scale (device float, e.g. a calibrated per-layer
 * constant): ue4m3 block scale sat(vmax / 6 / s) per 16 columns, e2m1 codes of v * (1/s) / block scale; magnitudes
 * above 2688 * s saturate. q: [M, N/2] packed (element 2i in the low nibble); q_sf: [pad128(M), N/16] in 128x4 atoms
 * (padding rows are not written). epi->D and epi->residual must be NULL; N a multiple of 32. The next GEMM takes
 * s as its alpha. */
int h3b_gemm_nvfp4_requant(const void* A, const uint8_t* sfa, const void* B, const uint8_t* sfb, int64_t M, int64_t N,
                           int64_t K, const h3b_epilogue* epi, uint8_t* q, uint8_t* q_sf, const float* q_scale,
                           cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * VSA coarse step and prologue, and the attention-output gate.
 * ------------------------------------------------------------------------------------------------------------- */

/* Replaces qkv_prologue8_op (fastvideo/models/dits/h3fast/h3fast.cu:889-927; kernel :376-510) for 64-token tiles.
 * q/k/v: bf16 rows [rows, heads*128] with row stride ld, in compact tile order; s1: deferred GEMM row scale [rows];
 * tile_row0/vbs: first row and row count of each tile [n_tiles]; wq/wk: RMSNorm weights bf16 [128]; cosb/sinb: bf16
 * [rows, 96] (RoPE on the first 96 dims, rotate-half pairs (d, d+48)). Outputs, heads-first and padded to rows_pad =
 * n_ext*64 rows per head: qb/kb/vb e4m3 [heads, rows_pad, 128]; vs_blk [heads, n_ext] V scale per tile
 * (max(amax/448, 1e-30)); vs_head [heads] folded with an atomic max (caller zeroes; may be NULL); qp/kp/vp fp32
 * [heads, n_tiles, 128] tile means. Q/K scales: static (inv_sq, inv_sk: 1/scale) when qs_blk == NULL, else one scale
 * per (head, tile) like V, written to qs_blk/ks_blk [heads, n_ext]. */
/* cosb == sinb == NULL skips the rotation (cross-attention queries and text keys). */
int h3b_qkv_prologue8(const void* q, const void* k, const void* v, int64_t ld, const float* s1,
                      const int32_t* tile_row0, const int32_t* vbs, const void* wq, const void* wk, const void* cosb,
                      const void* sinb, float inv_sq, float inv_sk, void* qb, void* kb, void* vb, float* qs_blk,
                      float* ks_blk, float* vs_blk, float* vs_head, float* qp, float* kp, float* vp, int heads,
                      int64_t rows_pad, int n_tiles, int n_ext, float eps, cudaStream_t stream);

/* h3b_qkv_prologue8 with per-tile scales, Q and K as symmetric int8 for the attention's kind::i8 QK^T (the
 * INT8 QK^T that sm_100a offers and the reference could not use on sm_103a, fastvideo/models/dits/h3fast/vsa_fp8.cuh:7-9):
 * qs_blk/ks_blk[h, t] = max(amax / 127, 1e-30) of the tile's rounded bf16 values, codes = clamp(rint(x / s), +-127)
 * (x times the fast-math reciprocal of s); V, the means and the V scales as h3b_qkv_prologue8. */
int h3b_qkv_prologue8_qk_int8(const void* q, const void* k, const void* v, int64_t ld, const float* s1,
                              const int32_t* tile_row0, const int32_t* vbs, const void* wq, const void* wk,
                              const void* cosb, const void* sinb, void* qb, void* kb, void* vb, float* qs_blk,
                              float* ks_blk, float* vs_blk, float* vs_head, float* qp, float* kp, float* vp, int heads,
                              int64_t rows_pad, int n_tiles, int n_ext, float eps, cudaStream_t stream);

/* The per-tile form the block runner uses (no reference counterpart; the tile and scale math are qkv_prologue8's):
 * per-(head, tile) scales for Q, K and V; flags H3B_PRO_QK_INT8 writes Q and K as int8 (as
 * h3b_qkv_prologue8_qk_int8), H3B_PRO_V_F16 writes V as f16 [heads, rows_pad, 128] -- the decoded E4M3 values, so
 * the attention kernel's PV operand is loaded as is (h3b_vsa_fp8_ex_v16) instead of converted on every use. */
#define H3B_PRO_QK_INT8 1
#define H3B_PRO_V_F16 2
int h3b_qkv_prologue8_tiles(const void* q, const void* k, const void* v, int64_t ld, const float* s1,
                            const int32_t* tile_row0, const int32_t* vbs, const void* wq, const void* wk,
                            const void* cosb, const void* sinb, void* qb, void* kb, void* vb, float* qs_blk,
                            float* ks_blk, float* vs_blk, float* vs_head, float* qp, float* kp, float* vp, int heads,
                            int64_t rows_pad, int n_tiles, int n_ext, float eps, int flags, cudaStream_t stream);

/* BASELINE config 4's prologue (no reference counterpart for its layout; the tile and scale math are qkv_prologue8's):
 * q/k/v bf16 [heads, seqlen, 128] in token order; perm [rows] maps tile-ordered rows to tokens (NULL = identity);
 * per-tile E4M3 scales for Q, K and V (max(amax/448, 1e-30)); vs_head [heads] (caller zeroes) takes the per-head
 * maximum of the V scales; other outputs as h3b_qkv_prologue8. */
int h3b_vsa_tile_quant(const void* q, const void* k, const void* v, int heads, int64_t seqlen, const int32_t* perm,
                       const int32_t* tile_row0, const int32_t* vbs, void* qb, void* kb, void* vb, float* qs_blk,
                       float* ks_blk, float* vs_blk, float* vs_head, float* qp, float* kp, float* vp, int64_t rows_pad,
                       int n_tiles, int n_ext, cudaStream_t stream);
/* h3b_vsa_tile_quant with V written as f16 [heads, rows_pad, 128] (the decoded E4M3 values) for h3b_vsa_fp8_ex_v16. */
int h3b_vsa_tile_quant_v16(const void* q, const void* k, const void* v, int heads, int64_t seqlen,
                           const int32_t* perm, const int32_t* tile_row0, const int32_t* vbs, void* qb, void* kb,
                           void* vh, float* qs_blk, float* ks_blk, float* vs_blk, float* vs_head, float* qp, float* kp,
                           float* vp, int64_t rows_pad, int n_tiles, int n_ext, cudaStream_t stream);

/* One tensor of h3b_qkv_prologue8's per-tile E4M3 form (no reference counterpart; the cross-attention queries, text
 * keys and text values of the DiT block): x bf16 rows [rows, heads*128] with row stride ld in tile order; optional
 * deferred row scale s1 [rows]; optional per-head RMSNorm weight w bf16 [128] (NULL: no norm); no RoPE. Writes xb e4m3
 * [heads, rows_pad, 128], xs_blk [heads, n_ext] = max(amax/448, 1e-30) per (head, tile), and folds the per-head
 * maximum into xs_head [heads] with an atomic max (caller zeroes; may be NULL). */
int h3b_head_tile_quant(const void* x, int64_t ld, const float* s1, const int32_t* tile_row0, const int32_t* vbs,
                        const void* w, void* xb, float* xs_blk, float* xs_head, int heads, int64_t rows_pad,
                        int n_tiles, int n_ext, float eps, cudaStream_t stream);
/* h3b_head_tile_quant writing f16 [heads, rows_pad, 128] (the decoded E4M3 values): text values for the f16-V
 * attention. */
int h3b_head_tile_quant_v16(const void* x, int64_t ld, const float* s1, const int32_t* tile_row0, const int32_t* vbs,
                            const void* w, void* xh, float* xs_blk, float* xs_head, int heads, int64_t rows_pad,
                            int n_tiles, int n_ext, float eps, cudaStream_t stream);

/* FP8 block-sparse VSA attention, fine step (replaces vsa_fp8_op, fastvideo/models/dits/h3fast/h3attn8.cu:1-42 and
 * vsa_fp8.cuh:782-871). qb/kb/vb e4m3 [heads, rows_pad, 128] (rows_pad = n_ext*64, tile order);
 * idx/num from h3b_topk_rows ([heads, n_ext, n], [heads, n_ext], padding tiles num 0); vbs [n_ext] valid rows per
 * tile; Q/K scales either per tile (qs_blk/ks_blk [heads, n_ext]) or folded into qk_coef; V per tile vs_blk and the
 * per-head maximum vs_head [heads]; qk_coef = softmax scale * log2(e) (* static Q and K scales). Output bf16
 * [heads, rows_pad, 128] (rows past vbs untouched), optional log2-domain LSE [heads, rows_pad]. n <= 4096, n_ext even. */
int h3b_vsa_fp8(const void* qb, const void* kb, const void* vb, const int32_t* idx, const int32_t* num,
                const int32_t* vbs, const float* qs_blk, const float* ks_blk, const float* vs_blk, const float* vs_head,
                float qk_coef, void* out, float* lse, int heads, int n, int n_ext, int64_t rows_pad,
                cudaStream_t stream);

/* The general form of h3b_vsa_fp8 (no reference counterpart: it adds the layouts the sequence-parallel block and the
 * cross-attention need). Q/out are [chunks_q * heads, rows_chunk_q, 128] and K/V [chunks_kv * heads, rows_chunk_kv,
 * 128]: query tile t of head h is plane (t / (rows_chunk_q/64)) * heads + h, row (t % (rows_chunk_q/64)) * 64 -- one
 * chunk is the plain heads-first layout, P chunks is what an all-to-all over P ranks delivers. Key tiles may be a
 * different tensor (cross-attention). idx row (h, t) starts at (h * n_q_ext + t) * idx_ld; num [h * n_q_ext + t];
 * qs [h * q_scale_ld + t]; ks/vs [h * kv_scale_ld + b]; lse indexed like out rows. */
typedef struct h3b_vsa_args {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  float* lse;
  const int32_t* idx;
  const int32_t* num;
  const int32_t* vbs_q;  /* [n_q_ext] */
  const int32_t* vbs_kv; /* [n_kv] */
  const float* qs;       /* or NULL: static Q/K scales folded into qk_coef */
  const float* ks;
  const float* vs;
  const float* vs_head;  /* [heads] */
  float qk_coef;
  int heads;
  int n_q_ext;           /* even */
  int n_kv;              /* <= 4096 */
  int idx_ld;
  int q_scale_ld;
  int kv_scale_ld;
  int64_t rows_chunk_q;
  int64_t rows_chunk_kv;
  int chunks_q;
  int chunks_kv;
  int qk_int8;           /* nonzero: q and k hold int8 codes (symmetric, per-tile scales qs/ks = amax/127) and
                            S = Q K^T runs as tcgen05 kind::i8 with s32 accumulation (exact), else E4M3 */
} h3b_vsa_args;
int h3b_vsa_fp8_ex(const h3b_vsa_args* args, cudaStream_t stream);
/* h3b_vsa_fp8_ex with V given as f16 [planes, rows, 128] holding the E4M3 values (h3b_qkv_prologue8_tiles with
 * H3B_PRO_V_F16): the PV MMAs read the V tiles as the TMA lands them, with no per-use conversion. */
int h3b_vsa_fp8_ex_v16(const h3b_vsa_args* args, cudaStream_t stream);
/* Replaces vsa_pair_op (fastvideo/models/dits/h3fast/h3attn8.cu:44-77; kernel vsa_pair.cuh:140-770): the same
 * attention driven by topk_pairs' output (h3b_topk_pairs) -- per (head, pair of adjacent 64-token query tiles) the
 * ascending union of both tiles' selections in args->idx [heads * n_q_ext/2, idx_ld] with its length in args->num
 * [heads * n_q_ext/2], and u_mem [heads * n_q_ext/2, idx_ld] one membership byte per union entry (bit 0: tile 2p
 * selected the key tile, bit 1: tile 2p+1). Every query row attends exactly its own tile's selection. A 128-token
 * tile is run as a pair whose 128-key blocks appear as two 64-key blocks selected by both halves (byte 3). The other
 * fields as h3b_vsa_fp8_ex; each tile's list holds at most 1024 key tiles (H3B_EINVAL in the status word beyond). */
int h3b_vsa_pair(const h3b_vsa_args* args, const uint8_t* u_mem, cudaStream_t stream);
/* h3b_vsa_pair with f16 V (as h3b_vsa_fp8_ex_v16). */
int h3b_vsa_pair_v16(const h3b_vsa_args* args, const uint8_t* u_mem, cudaStream_t stream);
/* h3b_vsa_fp8_ex for key lists shared by each pair of query tiles (no counterpart in the reference, whose
 * cross-attention is a dense FlashAttention call): the list of query tile 2p (idx/num rows of the even tile) applies
 * to tiles 2p and 2p+1, as for cross-attention to text tokens or a dense layer. One K and one V tile per step serve
 * both query tiles, and S = Q K^T and O += P V run as M = 128 MMAs over the pair. Same arguments and outputs as
 * h3b_vsa_fp8_ex; qk_int8 must be 0. The _v16 form takes f16 V like h3b_vsa_fp8_ex_v16. */
int h3b_vsa_fp8_shared(const h3b_vsa_args* args, cudaStream_t stream);
int h3b_vsa_fp8_shared_v16(const h3b_vsa_args* args, cudaStream_t stream);
/* Replaces vsa_fp8_op (fastvideo/models/dits/h3fast/h3attn8.cu:1-42) like h3b_vsa_fp8_ex_v16 --
 * same arguments (f16 V holding the E4M3 values, E4M3 Q/K: qk_int8 must be 0), same outputs within the accumulation
 * order inside the MMAs -- on the wide-step kernel: each query tile's key tiles run as two streams (even and odd list
 * entries) that one weight-stationary M = 64 MMA advances together (S: N = 128, PV: N = 256), so the whole 128-lane
 * datapath works on one query tile; the streams are merged by log-sum-exp in the epilogue. */
int h3b_vsa_fp8_ws(const h3b_vsa_args* args, cudaStream_t stream);
/* Status word of the attention kernel's bounded waits (0 = none); reset != 0 clears it. Synchronizes the device. */
int h3b_vsa_status(int* status, int reset);

/* Tile scores sc[h, i, j] = scale * sum_d qp[h,i,d] kp[h,j,d] in fp32 with a fixed order (d ascending, one fused
 * multiply-add per d), replacing the runner's torch.baddbmm (fastvideo/models/dits/h3fast/__init__.py:498-500,
 * TF32 there) with a bit-reproducible definition. qp/kp [heads, n, 128], sc [heads, n, n]. */
int h3b_tile_scores(const float* qp, const float* kp, int heads, int n, float scale, float* sc, cudaStream_t stream);

/* Replaces topk_rows_op (fastvideo/models/dits/h3fast/h3fast.cu:929-957; kernel :524-588). scores [heads*n, n];
 * spans given as HOST arrays starts/ends/ks [n_spans <= 4]; idx [heads, n_ext, n], num [heads, n_ext]. Prefix query
 * tiles are dense (or empty with split); per span the k largest (ties to the lowest column), ascending. */
int h3b_topk_rows(const float* scores, int heads, int n, int n_ext, int prefix, int n_spans, const int* starts,
                  const int* ends, const int* ks, int* idx, int* num, int split, cudaStream_t stream);

/* Replaces topk_pairs_op (fastvideo/models/dits/h3fast/h3fast.cu:959-987; kernel :590-686): per (head, pair of
 * adjacent query tiles 2p, 2p+1) the ascending union of both tiles' topk_rows selections with a membership byte per
 * entry (bit 0: tile 2p selected it, bit 1: tile 2p+1), u_idx/u_mem [heads * n_ext/2, n], u_num [heads * n_ext/2].
 * Pad tiles (>= n) select nothing; prefix query tiles are dense. The spans must tile [prefix, n) in order. idx/num:
 * scratch of topk_rows' shape ([heads, n_ext, n], [heads, n_ext]). */
int h3b_topk_pairs(const float* scores, int heads, int n, int n_ext, int prefix, int n_spans, const int* starts,
                   const int* ends, const int* ks, int* idx, int* num, int* u_idx, uint8_t* u_mem, int* u_num,
                   cudaStream_t stream);

/* The compressed (mean-pooled) attention branch: oc[h,i,:] = softmax_j(sc[h,i,:]) @ vp[h,:,:], stored bf16
 * [heads, n, 128] (fastvideo/models/dits/h3fast/__init__.py:505-511). */
int h3b_compressed_branch(const float* sc, const float* vp, int heads, int n, void* oc, cudaStream_t stream);

/* Replaces attn_gate_quant_op (fastvideo/models/dits/h3fast/h3fast.cu:1003-1029; kernel :688-741): row r of the
 * output gathers ob [heads, rows_pad, 128] at slot[r]; with o1 it is merged with o1 [rows, heads, 128] by log-sum-exp
 * (lse1a [heads, n1] for rows < n1, lse1b [heads, rows-n1] for the rest, natural log; lse2 [heads, rows_pad], log2);
 * with g it adds oc[h, slot/tile] * (sg[r] * g[r]) (g bf16 [rows, W]); then FP8 (asf == NULL: a [rows, W], sa row
 * scale) or NVFP4 (a [rows, W/2] codes, asf 128x4 scales, sa row global scale). W = heads*128 in {5120, 7168}. */
int h3b_attn_gate_quant(const void* ob, const void* g, const float* sg, const void* oc, const int32_t* slot,
                        int64_t rows_pad, int n_tiles, int tile, void* a, uint8_t* asf, float* sa, int64_t rows, int W,
                        const void* o1, const float* lse1a, const float* lse1b, int n1, const float* lse2,
                        cudaStream_t stream);

/* ---- Peer-memory transport of the sequence-parallel head exchange (no counterpart in the reference, whose fused
 * runner is single-GPU: patches/fastvideo-a01c50a.patch:644-645; FastVideo's stock path runs the same exchange as NCCL
 * all-to-alls, patch:12-13). One allocation per rank holds its receive buffers and flag words; every rank of the node
 * maps every other rank's allocation (CUDA IPC), the sender's copy engines write chunks into the receiver's buffers,
 * and a flag word written after the copies releases the receiver's bounded wait. */
typedef struct h3b_peer_handle {
  unsigned char bytes[64]; /* a CUDA IPC memory handle */
} h3b_peer_handle;
/* cudaMalloc of `bytes` on `device` (which must be the calling thread's current device), zero-filled. */
int h3b_peer_alloc(int device, size_t bytes, void** ptr);
int h3b_peer_free(void* ptr);
/* The IPC handle of an allocation made by h3b_peer_alloc, for another process of the node to open. */
int h3b_peer_export(const void* ptr, h3b_peer_handle* handle);
/* Maps a peer's allocation into this process (peer access enabled on first use); *ptr is its base address here. */
int h3b_peer_open(const h3b_peer_handle* handle, void** ptr);
int h3b_peer_close(void* ptr);
/* Stream-ordered 2D copy (height rows of `width` bytes, pitches in bytes) between any two of: local device memory,
 * a mapped peer allocation. Runs on the copy engines. */
int h3b_peer_copy2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t height,
                    cudaStream_t stream);
/* Writes `epoch` to a flag word (local or in a mapped peer allocation) after the stream's earlier work, preceded by
 * a system-scope fence, so a reader that sees the value also sees the data copied before it on this stream. */
int h3b_peer_signal(uint32_t* flag, uint32_t epoch, cudaStream_t stream);
/* One 2D region of h3b_peer_put: `height` rows of `width` bytes, pitches in bytes. */
typedef struct h3b_peer_copy {
  void* dst;
  const void* src;
  size_t dpitch;
  size_t spitch;
  size_t width;
  size_t height;
} h3b_peer_copy;
#define H3B_PEER_PUT_MAX_COPIES 64
#define H3B_PEER_PUT_MAX_FLAGS 16
/* Stream-ordered: copies up to 64 2D regions with the SMs (stores into a mapped peer allocation travel over NVLink),
 * then writes `epoch` into each of flags[0..n_flags) once every copied byte is visible system-wide, so a reader that
 * sees a flag sees all the copies. One kernel, for small transfers to many peers, where a run of h3b_peer_copy2d and
 * h3b_peer_signal calls is bound by the copy engines' per-copy latency. Addresses, pitches and widths are multiples
 * of 4 bytes. `counter` is a device word of the caller, zero before the call and left zero after it, with at most
 * one put in flight per counter. The copies and flags arrays are read on the host. */
int h3b_peer_put(const h3b_peer_copy* copies, int n_copies, uint32_t* const* flags, int n_flags, uint32_t epoch,
                 uint32_t* counter, cudaStream_t stream);
/* Enqueues a one-block kernel that waits until every one of flags[0..count) reaches `epoch` (32-bit wrap-around
 * compare). The wait is bounded (limit_ns per flag, at most 10 s; 0 means 10 s); when it expires the kernel sets the
 * exchange status word (dst[3] of h3b_status_async) to H3B_ETIMEOUT and returns, and later waits return at once
 * until the word is cleared. Later work on the stream sees everything written before the flags. */
int h3b_peer_wait(const uint32_t* flags, int count, uint32_t epoch, uint64_t limit_ns, cudaStream_t stream);

/* Status word written by kernels whose bounded waits expired (0 = none since the last reset); reset with
 * h3b_reset_device_status. Both synchronize the current device. */
int h3b_device_status(int* status);
int h3b_reset_device_status(void);
/* The kernels' device status words, read in stream order (no counterpart in the reference, whose kernels have no
 * bounded waits): dst[0] = the GEMMs' word (H3B_ETIMEOUT when a bounded wait expired), dst[1] = the attention's
 * (H3B_ETIMEOUT, or H3B_EINVAL when a selection list exceeded the 1024 key tiles the kernel holds), dst[2] = the row
 * kernels' (H3B_ETIMEOUT when a LayerNorm row copy never completed), dst[3] = the exchange waits' (H3B_ETIMEOUT when a
 * peer's flag did not arrive, h3b_peer_wait). dst is device memory or page-locked host memory for four ints; with
 * `clear` the words are reset after the read. A step that
 * enqueues this after its last kernel and checks dst once the stream reaches it learns of any failure in the step. */
int h3b_status_async(int* dst, int clear, cudaStream_t stream);
/* Exercises the bounded-wait path without a fault: one warp waits on an mbarrier nothing arrives on, with the kernels'
 * wait helper, gives up after limit_ns (<= 2 s) and sets the status word to H3B_ETIMEOUT; the context stays usable. */
int h3b_selftest_wait_timeout(uint64_t limit_ns, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* H3B_H_ */
