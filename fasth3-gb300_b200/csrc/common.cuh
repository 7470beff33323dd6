// Shared host/device helpers for the h3b C-ABI library (sm_100a only).
//
// Error model of every entry point: it returns 0 on success or a nonzero H3B_E* code and leaves a message in a
// thread-local buffer that h3b_last_error() returns. Nothing here allocates device memory; callers own all buffers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include <cstdio>
#include <cstdarg>
#include <mutex>

#include "../../include/h3b.h"

namespace h3b {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------------------------------------ host-side errors
int set_error(int code, const char* fmt, ...);
void clear_error();

#define H3B_REQUIRE(cond, ...)                                                                                     \
  do {                                                                                                             \
    if (!(cond)) return ::h3b::set_error(H3B_EINVAL, __VA_ARGS__);                                                \
  } while (0)

#define H3B_LAUNCH_CHECK(what)                                                                                     \
  do {                                                                                                             \
    cudaError_t e_ = cudaGetLastError();                                                                           \
    if (e_ != cudaSuccess) return ::h3b::set_error(H3B_ECUDA, "%s: %s", what, cudaGetErrorString(e_));            \
  } while (0)

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// A launch setting computed once per device (cudaFuncSetAttribute and occupancy queries apply to the current device:
// a host that drives several GPUs from one process needs them on each). Thread-safe; an init that fails (nonzero
// return) is not cached, so the next call retries.
constexpr int kMaxDevices = 64;
struct PerDevice {
  std::mutex m;
  int value[kMaxDevices] = {};
  bool ready[kMaxDevices] = {};

  template <class Init>
  int get(Init&& init, int* out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
      return set_error(H3B_ECUDA, "no usable current device (at most %d)", kMaxDevices);
    std::lock_guard<std::mutex> lock(m);
    if (!ready[dev]) {
      int v = 0;
      if (const int rc = init(&v)) return rc;
      value[dev] = v;
      ready[dev] = true;
    }
    *out = value[dev];
    return H3B_OK;
  }
};

inline int current_sms() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// ------------------------------------------------------------------------------------------------ device helpers
constexpr float kFp8Max = 448.f;
constexpr float kMinScaleFp8 = 1.f / (448.f * 512.f);  // floor of a per-row FP8 scale (all-zero rows)
constexpr float kFp4Range = 448.f * 6.f;              // largest |x| reachable as ue4m3 block scale x e2m1 code
constexpr float kMinScaleFp4 = 1e-12f;

// Eight bf16 from one 16-byte load, widened to fp32.
// 8 bf16 as raw bits (a prefetch: nothing waits on the load until unpack8 reads the registers)
__device__ __forceinline__ uint4 ld8_raw(const bf16* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void load8(const bf16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void load8_nc(const bf16* p, float (&f)[8]) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(bf16* p, const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// two fp32 -> bf16x2 (round to nearest even), a in the low half
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float to_bf16_and_back(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Two fp32 -> two saturating round-to-nearest-even e4m3 bytes (first argument in the low byte).
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  return e4m3x2(a, b) | (e4m3x2(c, d) << 16);
}

// Four E4M3 codes (low byte first) -> four f16 (exact: every E4M3 value is an f16 value), low code in the low half.
__device__ __forceinline__ uint2 e4m3x4_to_f16x4(uint32_t codes) {
  uint2 r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r.x) : "h"((uint16_t)(codes & 0xFFFFu)));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r.y) : "h"((uint16_t)(codes >> 16)));
  return r;
}

__device__ __forceinline__ float e4m3_to_float(uint32_t byte) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)byte, __NV_E4M3);
  return __half2float(__half(h));
}

// Four fp32 -> four e2m1 nibbles (saturating, round-to-nearest-even) in the low 16 bits; element 0 in the lowest
// nibble. cvt...e2m1x2 puts its first source operand in the high nibble, so the pair is passed swapped.
__device__ __forceinline__ uint32_t e2m1x4(float a, float b, float c, float d) {
  uint32_t r;
  asm("{\n\t.reg .b8 lo, hi;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 lo, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 hi, %4, %3;\n\t"
      "mov.b32 %0, {lo, hi, lo, hi};\n\t}"
      : "=r"(r)
      : "f"(a), "f"(b), "f"(c), "f"(d));
  return r & 0xffffu;
}

// Eight fp32 -> eight e2m1 nibbles in one word (element 0 in the lowest nibble; the same codes as two e2m1x4).
__device__ __forceinline__ uint32_t e2m1x8(const float* v) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return r;
}

// Byte offset of scale (row, col) in the 128x4-atom layout that tcgen05 block-scaled MMA reads (one 512-byte atom per
// 128 rows x 4 scale columns; inside it row r sits at (r % 32) * 16 + ((r % 128) / 32) * 4).
__host__ __device__ __forceinline__ size_t sf_atom_offset(int64_t row, int64_t col, int64_t sf_cols) {
  return (size_t)(row >> 7) * (size_t)(sf_cols >> 2) * 512 + (size_t)(col >> 2) * 512 + (size_t)(row & 31) * 16 +
         (size_t)((row & 127) >> 5) * 4 + (size_t)(col & 3);
}

// The ue4m3 block scale of one 16-element block whose largest magnitude is vmax, under the global factor gs (so the
// scale stays inside the e4m3 range), and the multiplier that maps the block onto e2m1 codes (0 for an empty block).
__device__ __forceinline__ float nvfp4_block_scale(float vmax, float gs, uint32_t* bits) {
  *bits = (uint32_t)__nv_cvt_float_to_fp8(gs * (vmax * (1.f / 6.f)), __NV_SATFINITE, __NV_E4M3);
  const float sf = e4m3_to_float(*bits);
  return (vmax != 0.f && sf != 0.f) ? gs / sf : 0.f;
}

// Paired fp32 arithmetic (sm_100 f32x2): two independent operations in one instruction, each rounded to nearest and
// flushed to zero like the scalar instructions of the fast-math build, so the results equal two scalar operations.
__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 a, b;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %3};\n\t"
      "add.rn.ftz.f32x2 a, a, b;\n\tmov.b64 {%0, %1}, a;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}
__device__ __forceinline__ void sub2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 a, b;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %3};\n\t"
      "sub.rn.ftz.f32x2 a, a, b;\n\tmov.b64 {%0, %1}, a;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}
__device__ __forceinline__ void mul2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 a, b;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %3};\n\t"
      "mul.rn.ftz.f32x2 a, a, b;\n\tmov.b64 {%0, %1}, a;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}
// a = a * b + c
__device__ __forceinline__ void fma2(float& a0, float& a1, float b0, float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 a, b, c;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %3};\n\tmov.b64 c, {%4, %5};\n\t"
      "fma.rn.ftz.f32x2 a, a, b, c;\n\tmov.b64 {%0, %1}, a;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
// three-input maximum (sm_100 max.f32 with three sources)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// acc += x * y for a pair, IEEE rounding without flush to zero (one correctly rounded fused multiply-add per lane)
__device__ __forceinline__ void fma2_acc_rn(float& acc0, float& acc1, float x0, float x1, float y0, float y1) {
  asm("{\n\t.reg .b64 a, x, y;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "fma.rn.f32x2 a, x, y, a;\n\tmov.b64 {%0, %1}, a;\n\t}"
      : "+f"(acc0), "+f"(acc1)
      : "f"(x0), "f"(x1), "f"(y0), "f"(y1));
}
// acc += d * d for a pair
__device__ __forceinline__ void sq_acc2(float& acc0, float& acc1, float d0, float d1) {
  asm("{\n\t.reg .b64 a, d;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 d, {%2, %3};\n\t"
      "fma.rn.ftz.f32x2 a, d, d, a;\n\tmov.b64 {%0, %1}, a;\n\t}"
      : "+f"(acc0), "+f"(acc1)
      : "f"(d0), "f"(d1));
}

// Butterfly reductions. Every lane ends with the same value: at each stage lanes l and l^o add the same two operands.
template <bool MAX>
__device__ __forceinline__ float warp_allreduce(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, u) : v + u;
  }
  return v;
}

// Block-wide all-reduce over NW warps: per-warp butterfly, warp partials staged in shared memory, then the same
// butterfly over 32 lanes with zeros past NW. The staging buffer is reusable after the call returns.
template <int NW, bool MAX>
__device__ __forceinline__ float block_allreduce(float v, float* stage) {
  static_assert(NW <= 32, "at most 32 warps");
  v = warp_allreduce<MAX>(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) stage[w] = v;
  __syncthreads();
  float r = l < NW ? stage[l] : 0.f;
  r = warp_allreduce<MAX>(r);
  __syncthreads();
  return r;
}

}  // namespace h3b
