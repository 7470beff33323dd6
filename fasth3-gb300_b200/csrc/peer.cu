// Peer-memory transport for the sequence-parallel head exchange.
//
// The reference's fused runner is single-GPU (patches/fastvideo-a01c50a.patch:644-645); FastVideo's stock multi-GPU
// path exchanges heads with NCCL all-to-alls inside DistributedAttention (patch:12-13). Here each rank's receive
// buffers live in one device allocation that every rank of the node maps (CUDA IPC over NVLink). The sender's copy
// engines write each chunk straight into the receiver's buffer (cudaMemcpy2DAsync between local and peer-mapped
// memory: no SM is used, so the copies run beside the attention kernels), and a flag word per (sender, exchange) in
// the receiver's allocation, written after the copy in stream order with a system-scope fence (cuStreamWriteValue32),
// releases the receiver. The receiver waits on the flags with a one-block kernel whose wait is bounded: after
// kPeerWaitLimitNs it gives up, records H3B_ETIMEOUT in the exchange status word (dst[3] of h3b_status_async) and
// returns, so the context stays usable and the host learns of it after the step.
//
// Flags hold the sender's running exchange count (an epoch): a receiver waits until flag - epoch >= 0 (32-bit
// wrap-around compare), so the words are never reset.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "sm100.cuh"

namespace h3b {

__device__ int g_peer_status = 0;
constexpr uint64_t kPeerWaitLimitNs = 10ull * 1000ull * 1000ull * 1000ull;

namespace {

__global__ void peer_wait_kernel(const uint32_t* __restrict__ flags, int count, uint32_t epoch, uint64_t limit_ns) {
  // once a wait has expired, the exchanges that follow in the same step are not waited for again (the step's result
  // is already void and the host raises when it reads the status word), so a lost peer costs one limit, not one per
  // exchange
  if (*reinterpret_cast<volatile int*>(&g_peer_status) != 0) return;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const uint64_t t0 = sm100::globaltimer_ns();
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (sm100::globaltimer_ns() - t0 > limit_ns) {
        atomicExch(&g_peer_status, H3B_ETIMEOUT);
        break;
      }
      __nanosleep(200);
    }
  }
}

// h3b_peer_put: the copies (row geometry in units of 1 << shift bytes) and flags, passed by value
struct PutCopy {
  char* dst;
  const char* src;
  uint64_t dpitch, spitch;
  uint64_t row_units, units;
};
struct PutArgs {
  PutCopy c[H3B_PEER_PUT_MAX_COPIES];
  uint32_t* flags[H3B_PEER_PUT_MAX_FLAGS];
  uint32_t* counter;
  int n, n_flags;
  uint32_t epoch;
};

// Every thread copies a grid-strided share of each region, four units in flight at a time; then each thread fences at
// system scope, and the block's thread 0 (after the barrier and its own system fence, which covers the writes of the
// block it observed) counts the block in. The block that counts last fences again and writes the flags with release
// semantics at system scope: a reader whose acquire load sees a flag sees every byte of every copy. The counter is
// left at zero for the next put. Nothing here waits on another block or GPU.
template <typename U>
__global__ void __launch_bounds__(256) peer_put_kernel(const __grid_constant__ PutArgs a) {
  const uint64_t nthr = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int c = 0; c < a.n; ++c) {
    const PutCopy& d = a.c[c];
    for (uint64_t u0 = tid; u0 < d.units; u0 += 4 * nthr) {
      U v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t u = u0 + k * nthr;
        if (u < d.units) {
          const uint64_t row = u / d.row_units, col = u - row * d.row_units;
          v[k] = *reinterpret_cast<const U*>(d.src + row * d.spitch + col * sizeof(U));
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t u = u0 + k * nthr;
        if (u < d.units) {
          const uint64_t row = u / d.row_units, col = u - row * d.row_units;
          *reinterpret_cast<U*>(d.dst + row * d.dpitch + col * sizeof(U)) = v[k];
        }
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(a.counter, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int f = 0; f < a.n_flags; ++f)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flags[f]), "r"(a.epoch) : "memory");
      atomicExch(a.counter, 0u);
    }
  }
}

typedef CUresult (*WriteValueFn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

WriteValueFn write_value_fn() {
  static WriteValueFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<WriteValueFn>(p);
  }
  return fn;
}

}  // namespace

int peer_status_async(int* dst, int clear, cudaStream_t stream) {
  if (cudaMemcpyFromSymbolAsync(dst, g_peer_status, sizeof(int), 0, cudaMemcpyDefault, stream) != cudaSuccess)
    return set_error(H3B_ECUDA, "status: reading the exchange status word failed");
  if (clear) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_peer_status) != cudaSuccess || cudaMemsetAsync(p, 0, sizeof(int), stream) != cudaSuccess)
      return set_error(H3B_ECUDA, "status: clearing the exchange status word failed");
  }
  return H3B_OK;
}

}  // namespace h3b

using h3b::set_error;

static_assert(sizeof(h3b_peer_handle) == sizeof(cudaIpcMemHandle_t), "h3b_peer_handle must hold a CUDA IPC handle");

extern "C" int h3b_peer_alloc(int device, size_t bytes, void** ptr) {
  h3b::clear_error();
  H3B_REQUIRE(ptr && bytes > 0, "peer_alloc: null pointer or zero size");
  int cur = -1;
  H3B_REQUIRE(cudaGetDevice(&cur) == cudaSuccess && cur == device, "peer_alloc: device %d is not the current device",
              device);
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return set_error(H3B_ECUDA, "peer_alloc: cudaMalloc of %zu bytes failed", bytes);
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return set_error(H3B_ECUDA, "peer_alloc: clearing %zu bytes failed", bytes);
  }
  return H3B_OK;
}

extern "C" int h3b_peer_free(void* ptr) {
  h3b::clear_error();
  if (!ptr) return H3B_OK;
  if (cudaFree(ptr) != cudaSuccess) return set_error(H3B_ECUDA, "peer_free: cudaFree failed");
  return H3B_OK;
}

extern "C" int h3b_peer_export(const void* ptr, h3b_peer_handle* handle) {
  h3b::clear_error();
  H3B_REQUIRE(ptr && handle, "peer_export: null pointer");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess)
    return set_error(H3B_ECUDA, "peer_export: cudaIpcGetMemHandle failed (the pointer must come from h3b_peer_alloc)");
  memcpy(handle->bytes, &h, sizeof(h));
  return H3B_OK;
}

extern "C" int h3b_peer_open(const h3b_peer_handle* handle, void** ptr) {
  h3b::clear_error();
  H3B_REQUIRE(handle && ptr, "peer_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof(h));
  *ptr = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(H3B_ECUDA, "peer_open: cudaIpcOpenMemHandle failed (%s)", cudaGetErrorString(e));
  return H3B_OK;
}

extern "C" int h3b_peer_close(void* ptr) {
  h3b::clear_error();
  if (!ptr) return H3B_OK;
  if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) return set_error(H3B_ECUDA, "peer_close: cudaIpcCloseMemHandle failed");
  return H3B_OK;
}

extern "C" int h3b_peer_copy2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t height,
                               cudaStream_t stream) {
  h3b::clear_error();
  H3B_REQUIRE(dst && src, "peer_copy2d: null pointer");
  H3B_REQUIRE(width <= dpitch && width <= spitch, "peer_copy2d: width %zu exceeds a pitch", width);
  if (width == 0 || height == 0) return H3B_OK;
  const cudaError_t e = height == 1 ? cudaMemcpyAsync(dst, src, width, cudaMemcpyDefault, stream)
                                    : cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDefault, stream);
  if (e != cudaSuccess) return set_error(H3B_ECUDA, "peer_copy2d: copy failed (%s)", cudaGetErrorString(e));
  return H3B_OK;
}

extern "C" int h3b_peer_signal(uint32_t* flag, uint32_t epoch, cudaStream_t stream) {
  h3b::clear_error();
  H3B_REQUIRE(flag && (reinterpret_cast<uintptr_t>(flag) & 3u) == 0, "peer_signal: null or unaligned flag");
  auto fn = h3b::write_value_fn();
  H3B_REQUIRE(fn, "peer_signal: cuStreamWriteValue32 is not available");
  // default flags: the write is ordered after the stream's earlier work and preceded by a system-wide fence
  if (fn(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag), epoch, 0) != CUDA_SUCCESS)
    return set_error(H3B_ECUDA, "peer_signal: cuStreamWriteValue32 failed");
  return H3B_OK;
}

extern "C" int h3b_peer_put(const h3b_peer_copy* copies, int n_copies, uint32_t* const* flags, int n_flags,
                            uint32_t epoch, uint32_t* counter, cudaStream_t stream) {
  h3b::clear_error();
  H3B_REQUIRE(n_copies >= 0 && n_copies <= H3B_PEER_PUT_MAX_COPIES, "peer_put: %d copies (at most %d)", n_copies,
              H3B_PEER_PUT_MAX_COPIES);
  H3B_REQUIRE(n_flags >= 0 && n_flags <= H3B_PEER_PUT_MAX_FLAGS, "peer_put: %d flags (at most %d)", n_flags,
              H3B_PEER_PUT_MAX_FLAGS);
  H3B_REQUIRE(n_copies == 0 || copies, "peer_put: null copies");
  H3B_REQUIRE(n_flags == 0 || flags, "peer_put: null flags");
  H3B_REQUIRE(counter && (reinterpret_cast<uintptr_t>(counter) & 3u) == 0, "peer_put: null or unaligned counter");
  h3b::PutArgs a;
  memset(&a, 0, sizeof(a));
  // 16-byte units when every address, pitch and width allows them, else 4-byte units
  uintptr_t bits = 0;
  for (int i = 0; i < n_copies; ++i) {
    const h3b_peer_copy& c = copies[i];
    if (c.width == 0 || c.height == 0) continue;
    H3B_REQUIRE(c.dst && c.src, "peer_put: copy %d has a null pointer", i);
    H3B_REQUIRE(c.width <= c.dpitch && c.width <= c.spitch, "peer_put: copy %d's width exceeds a pitch", i);
    bits |= reinterpret_cast<uintptr_t>(c.dst) | reinterpret_cast<uintptr_t>(c.src) | c.dpitch | c.spitch | c.width;
  }
  H3B_REQUIRE((bits & 3u) == 0, "peer_put: addresses, pitches and widths must be multiples of 4 bytes");
  const int shift = (bits & 15u) == 0 ? 4 : 2;
  uint64_t total = 0;
  for (int i = 0; i < n_copies; ++i) {
    const h3b_peer_copy& c = copies[i];
    if (c.width == 0 || c.height == 0) continue;
    h3b::PutCopy& d = a.c[a.n++];
    d.dst = static_cast<char*>(c.dst);
    d.src = static_cast<const char*>(c.src);
    d.dpitch = c.dpitch;
    d.spitch = c.spitch;
    d.row_units = c.width >> shift;
    d.units = d.row_units * c.height;
    total += d.units;
  }
  for (int f = 0; f < n_flags; ++f) {
    H3B_REQUIRE(flags[f] && (reinterpret_cast<uintptr_t>(flags[f]) & 3u) == 0, "peer_put: flag %d null or unaligned",
                f);
    a.flags[f] = flags[f];
  }
  a.n_flags = n_flags;
  a.counter = counter;
  a.epoch = epoch;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t want = (total + 4 * 256 - 1) / (4 * 256);
  const int blocks = (int)(want < 1 ? 1 : (want > (uint64_t)(2 * sms) ? 2 * sms : want));
  if (shift == 4)
    h3b::peer_put_kernel<int4><<<blocks, 256, 0, stream>>>(a);
  else
    h3b::peer_put_kernel<uint32_t><<<blocks, 256, 0, stream>>>(a);
  H3B_LAUNCH_CHECK("peer_put");
  return H3B_OK;
}

extern "C" int h3b_peer_wait(const uint32_t* flags, int count, uint32_t epoch, uint64_t limit_ns, cudaStream_t stream) {
  h3b::clear_error();
  H3B_REQUIRE(flags && count > 0 && count <= 4096, "peer_wait: null flags or count %d outside 1..4096", count);
  H3B_REQUIRE(limit_ns <= h3b::kPeerWaitLimitNs, "peer_wait: limit above %llu ns",
              (unsigned long long)h3b::kPeerWaitLimitNs);
  const int threads = count < 128 ? ((count + 31) / 32) * 32 : 128;
  h3b::peer_wait_kernel<<<1, threads, 0, stream>>>(flags, count, epoch, limit_ns ? limit_ns : h3b::kPeerWaitLimitNs);
  H3B_LAUNCH_CHECK("peer_wait");
  return H3B_OK;
}
