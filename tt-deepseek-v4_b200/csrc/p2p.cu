// Peer-memory exchange for the sequence split: the small all-gathers of one
// decode step (per layer G x 16 KB of top-k candidates and G x 128 KB of
// attention partials) done as direct NVLink stores into every peer's
// receive buffer plus a per-rank flag, instead of a library collective
// whose fixed cost (~20 us per call inside a graph) exceeds the transfer
// (~0.2 us at 770 GB/s) a hundredfold.
//
// Buffers that peers write are allocated here with cudaMalloc (one
// allocation per rank, exported once as a CUDA IPC handle and mapped by
// every other rank of the node).  Only plain st.global / ld.acquire go to
// peer memory; no TMA and no library kernel ever reads it.
//
// Ordering: a publishing CTA makes its peer stores visible system-wide
// (fence.sc.sys) before its arrival on a local counter; the last CTA for a
// destination then release-stores the step's epoch into that destination's
// flag slot for this rank.  The consumer waits (acquire, bounded) until
// every rank's flag reaches the epoch.  Epochs grow by one per decode step
// and never repeat, so a flag left from an earlier step never passes a
// wait.  Reuse of a receive buffer by the next step is safe because a rank
// publishes step s + 1 only after it has waited on every peer's later
// exchange of step s (each peer finished reading by then, stream order).
#include "common.cuh"
#include <cuda.h>
#include <string.h>

namespace dsa {
namespace p2p {

constexpr int kThreads = 512;
constexpr size_t kChunk = 32 * 1024;       // bytes one CTA stores to one destination
constexpr int kStatusTimeout = 2;

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// grid (chunks, G): CTA (x, g) stores chunk x of src to destination g, then
// the last CTA of destination g raises its flag.
__global__ void __launch_bounds__(kThreads) publish_kernel(const uint4* __restrict__ src, size_t n16,
                                                           const unsigned long long* __restrict__ dst,
                                                           const unsigned long long* __restrict__ flag,
                                                           const uint32_t* __restrict__ epoch,
                                                           uint32_t* __restrict__ done) {
  const int g = blockIdx.y;
  uint4* d = reinterpret_cast<uint4*>(dst[g]);
  const size_t per = kChunk / 16;
  const size_t i0 = size_t(blockIdx.x) * per, i1 = min(n16, i0 + per);
  for (size_t i = i0 + threadIdx.x; i < i1; i += kThreads) d[i] = __ldg(src + i);
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t old = atomicAdd(done + g, 1u);
    if (old == gridDim.x - 1) {
      done[g] = 0;  // every CTA of this destination has arrived: reset for the next call
      __threadfence_system();
      st_release_sys_u32(reinterpret_cast<uint32_t*>(flag[g]), *epoch);
    }
  }
}

// One warp: lane i < G waits until flags[i] >= epoch.
__global__ void wait_kernel(const uint32_t* __restrict__ flags, int G, const uint32_t* __restrict__ epoch,
                            int32_t* __restrict__ status, long long spin) {
  const int i = threadIdx.x;
  const uint32_t e = *epoch;
  if (i < G) {
    const long long t0 = clock64();
    while (ld_acquire_sys_u32(flags + i) < e) {
      if (clock64() - t0 > spin) {
        if (status) atomicOr(status, kStatusTimeout);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncwarp();
}

__global__ void bump_kernel(uint32_t* c) { *c += 1u; }

}  // namespace p2p
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_p2p_alloc(size_t bytes, void** ptr) {
  clear_error();
  DSA_CHECK_ARG(ptr && bytes > 0, "p2p_alloc: bad arguments");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) {
    set_error("p2p_alloc: %s", cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

extern "C" int dsa_p2p_free(void* ptr) {
  clear_error();
  if (!ptr) return DSA_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_error("p2p_free: %s", cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

extern "C" size_t dsa_p2p_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

namespace {
// cuMemGetAddressRange (driver API), resolved once through the runtime
typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  }
  return fn;
}
}  // namespace

// IPC handle of the allocation holding ptr, and ptr's byte offset in it (a
// buffer from a caching allocator is usually a piece of a larger cudaMalloc).
extern "C" int dsa_p2p_export(void* ptr, void* handle, uint64_t* offset) {
  clear_error();
  DSA_CHECK_ARG(ptr && handle && offset, "p2p_export: null pointer");
  AddrRangeFn fn = addr_range_fn();
  if (!fn) {
    set_error("p2p_export: cuMemGetAddressRange unavailable");
    return DSA_ERR_CUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error("p2p_export: cuMemGetAddressRange failed");
    return DSA_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    set_error("p2p_export: %s", cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  *offset = uint64_t(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return DSA_OK;
}

extern "C" int dsa_p2p_import(const void* handle, void** ptr) {
  clear_error();
  DSA_CHECK_ARG(ptr && handle, "p2p_import: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("p2p_import: %s", cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

extern "C" int dsa_p2p_close(void* ptr) {
  clear_error();
  if (!ptr) return DSA_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_error("p2p_close: %s", cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

extern "C" int dsa_p2p_publish(const void* src, size_t bytes, const unsigned long long* dst_ptrs,
                               const unsigned long long* flag_ptrs, const uint32_t* epoch, int G, uint32_t* done,
                               dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(src && dst_ptrs && flag_ptrs && epoch && done, "p2p_publish: null pointer");
  DSA_CHECK_ARG(G > 0 && G <= 64 && bytes > 0 && bytes % 16 == 0 && aligned(src, 16),
                "p2p_publish: need 0 < G <= 64 and a 16-byte aligned source of whole 16-byte words");
  const size_t chunks = (bytes + p2p::kChunk - 1) / p2p::kChunk;
  DSA_CHECK_ARG(chunks <= 65535, "p2p_publish: %zu bytes is too large", bytes);
  p2p::publish_kernel<<<dim3(unsigned(chunks), G), p2p::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), bytes / 16, dst_ptrs, flag_ptrs, epoch, done);
  DSA_CHECK_LAUNCH("p2p_publish");
  return DSA_OK;
}

extern "C" int dsa_p2p_wait(const uint32_t* flags, int G, const uint32_t* epoch, int32_t* status,
                            dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(flags && epoch && G > 0 && G <= 32, "p2p_wait: bad arguments");
  p2p::wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flags, G, epoch, status,
                                                                         wait_limit_cycles());
  DSA_CHECK_LAUNCH("p2p_wait");
  return DSA_OK;
}

extern "C" int dsa_counter_bump(uint32_t* counter, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(counter, "counter_bump: null pointer");
  p2p::bump_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(counter);
  DSA_CHECK_LAUNCH("counter_bump");
  return DSA_OK;
}
