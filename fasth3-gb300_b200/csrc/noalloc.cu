// Per-tensor NVFP4 quantization for callers that cannot allocate device memory.
//
// h3b_quant_nvfp4 needs a few bytes of device scratch (the tensor's running absolute maximum) and asks its caller for
// them. Some callers have no way to provide that: a host that hands the library only the tensors it owns (a plugin
// entry point inside an engine whose device memory is planned ahead of time, or a foreign-language host driving the
// C ABI with a fixed buffer set) must not call cudaMalloc mid-run, because an allocation can synchronize the device
// and fragment a pool that was sized up front. This file gives them h3b_quant_nvfp4_noalloc, whose scratch lives in a
// file-scope device array that the CUDA runtime places on every GPU that loads the library and keeps until the process
// exits. The entry point calls no cudaMalloc, cudaFree or allocating library routine.
#include "common.cuh"

#include <cuda.h>
#include <mutex>

namespace h3b {

int amax_launch(const bf16* x, int64_t ld, int64_t rows, int K, float* amax, cudaStream_t st);
int quant_nvfp4_tensor_launch(const bf16* x, int64_t ld, int64_t rows, int K, const float* amax, uint8_t* q,
                              uint8_t* sf, float* s_out, cudaStream_t st);

namespace {

// 256 bytes of device scratch shared by every call on a device. Host code must not use this name as a device address
// (on the host it is only a stand-in symbol); the address comes from cudaGetSymbolAddress below.
constexpr size_t kScratchBytes = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mutex;  // kMaxDevices: common.cuh
void* g_scratch_addr[kMaxDevices] = {nullptr};
CUcontext g_scratch_ctx[kMaxDevices] = {nullptr};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  return fn;
}

// Resolves the array's device address on the current device. The lookup runs on the first call on a device and again
// whenever the thread's current context on that device is not the one the cached address belongs to (after
// cudaDeviceReset, or under a context the caller created); a failed lookup is not cached, the next call retries.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(H3B_ECUDA, "quant_nvfp4_noalloc: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(H3B_EINVAL, "quant_nvfp4_noalloc: device %d is beyond the %d devices supported", dev, kMaxDevices);
  const CtxGetCurrentFn get = ctx_get_current();
  if (!get) return set_error(H3B_ECUDA, "quant_nvfp4_noalloc: cuCtxGetCurrent is unavailable");
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS) return set_error(H3B_ECUDA, "quant_nvfp4_noalloc: cannot read the current context");
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_addr[dev] == nullptr || ctx == nullptr || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // binds the runtime's context if none is
    if (e != cudaSuccess || p == nullptr) {
      g_scratch_addr[dev] = nullptr;
      return set_error(H3B_ECUDA, "quant_nvfp4_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                       cudaGetErrorString(e));
    }
    if (get(&ctx) != CUDA_SUCCESS) ctx = nullptr;  // a null context key makes the next call look up again
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_addr[dev];
  return H3B_OK;
}

}  // namespace
}  // namespace h3b

using namespace h3b;

extern "C" int h3b_quant_nvfp4_noalloc(const void* x, int64_t ld, int64_t rows, int K, void* q, uint8_t* sf,
                                       float* s_out, cudaStream_t stream) {
  clear_error();
  const size_t need = h3b_quant_nvfp4_workspace_bytes();
  H3B_REQUIRE(need <= kScratchBytes,
              "quant_nvfp4_noalloc: needs %zu bytes of scratch but the static array holds %zu", need, kScratchBytes);
  H3B_REQUIRE(x && q && sf && s_out, "quant_nvfp4_noalloc: null pointer");
  H3B_REQUIRE(K > 0 && K % 64 == 0 && ld % 8 == 0 && ld >= K, "quant_nvfp4_noalloc: K multiple of 64, ld multiple of 8");
  H3B_REQUIRE(rows >= 0, "quant_nvfp4_noalloc: rows < 0");
  H3B_REQUIRE(aligned(x, 16) && aligned(q, 16) && aligned(sf, 4),
              "quant_nvfp4_noalloc: x, q 16-byte and sf 4-byte aligned");
  void* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  float* amax = static_cast<float*>(scratch);
  // the array keeps the previous call's maximum: it must start from zero
  if (cudaMemsetAsync(amax, 0, sizeof(float), stream) != cudaSuccess)
    return set_error(H3B_ECUDA, "quant_nvfp4_noalloc: clearing the scratch failed");
  if (rows == 0) return H3B_OK;
  if (int rc = amax_launch(static_cast<const bf16*>(x), ld, rows, K, amax, stream)) return rc;
  return quant_nvfp4_tensor_launch(static_cast<const bf16*>(x), ld, rows, K, amax, static_cast<uint8_t*>(q), sf,
                                   s_out, stream);
}
