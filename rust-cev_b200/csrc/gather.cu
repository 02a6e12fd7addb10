// The cfg5 head all-gather fused into the attention epilogue, over NVLink
// peer memory (KV-head split of the LFM2 attention layers across ranks).
//
// Every rank cudaMallocs its gathered buffers and a flag array, exports them
// with cudaIpcGetMemHandle and opens its peers' (lazy peer access; no
// multicast object).  The attention call of rank r stores each output row to
// every rank's buffer at rank r's head columns (plain 16-byte P2P stores
// from the epilogue); gather_signal_kernel then raises flag[r] = epoch in
// every rank's flag array, and gather_wait_kernel on each rank waits (bounded)
// until all flags of its own array reach the epoch before the replicated
// output projection reads the buffer.  Replaces the NCCL all-gather of
// lfm2.rs:145-171's per-head outputs under the KV-head split.
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace cevk {

constexpr int kMaxRanks = 8;
constexpr int kErrGatherTimeout = 2;

struct FlagPtrs {
  int* p[kMaxRanks];
};

// Runs after this rank's attention kernel on the same stream: its peer
// stores are complete; publish them with a system-scope release.
__global__ void gather_signal_kernel(FlagPtrs flags, int world, int rank, int epoch) {
  const int i = threadIdx.x;
  if (i >= world) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flags.p[i] + rank), "r"(epoch) : "memory");
}

__global__ void gather_wait_kernel(const int* flags, int world, int epoch, long long limit) {
  if (threadIdx.x != 0) return;
  const long long t0 = clock64();
  for (int s = 0; s < world; ++s) {
    for (;;) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flags + s) : "memory");
      if (v - epoch >= 0) break;  // epochs only grow
      if (clock64() - t0 > limit) {
        if (atomicExch(&g_device_error, kErrGatherTimeout) == 0) {
          g_device_error_info[0] = (int)blockIdx.x;
          g_device_error_info[1] = s;
          g_device_error_info[2] = v;
          g_device_error_info[3] = epoch;
        }
        return;
      }
      __nanosleep(64);
    }
  }
}

// Device-side epochs: the signal kernel advances this rank's epoch counter
// and publishes it; the wait kernel reads the same counter.  A CUDA graph
// can then replay the same launches, each replay a new epoch.
__global__ void gather_signal_dev_kernel(FlagPtrs flags, int world, int rank, int* epoch_ctr) {
  __shared__ int e;
  if (threadIdx.x == 0) {
    e = *epoch_ctr + 1;
    *epoch_ctr = e;
  }
  __syncthreads();
  const int i = threadIdx.x;
  if (i >= world) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flags.p[i] + rank), "r"(e) : "memory");
}

__global__ void gather_wait_dev_kernel(const int* flags, int world, const int* epoch_ctr, long long limit) {
  if (threadIdx.x != 0) return;
  const int epoch = *epoch_ctr;  // this rank's signal kernel ran earlier on the stream
  const long long t0 = clock64();
  for (int s = 0; s < world; ++s) {
    for (;;) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flags + s) : "memory");
      if (v - epoch >= 0) break;
      if (clock64() - t0 > limit) {
        if (atomicExch(&g_device_error, kErrGatherTimeout) == 0) {
          g_device_error_info[0] = (int)blockIdx.x;
          g_device_error_info[1] = s;
          g_device_error_info[2] = v;
          g_device_error_info[3] = epoch;
        }
        return;
      }
      __nanosleep(64);
    }
  }
}

// One contiguous range of 16-byte words copied to each destination (this
// rank's buffer and its peers', over NVLink); every word is loaded once.
struct DstPtrs {
  uint4* p[kMaxRanks];
};
__global__ void __launch_bounds__(256) rows_to_peers_kernel(const uint4* __restrict__ src, DstPtrs dst, int n_dst,
                                                            long long n16) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const uint4 v = src[i];
    for (int d = 0; d < n_dst; ++d) dst.p[d][i] = v;
  }
}

// Signal and wait in one launch (device-side epoch): the head gather's
// handshake after the attention call.
__device__ __forceinline__ void signal_then_wait(const FlagPtrs& flags, int world, int rank, int* epoch_ctr,
                                                 const int* own, long long limit) {
  __shared__ int e;
  if (threadIdx.x == 0) {
    e = *epoch_ctr + 1;
    *epoch_ctr = e;
  }
  __syncthreads();
  if ((int)threadIdx.x < world) {
    __threadfence_system();
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flags.p[threadIdx.x] + rank), "r"(e) : "memory");
  }
  if (threadIdx.x != 0) return;
  const long long t0 = clock64();
  for (int s = 0; s < world; ++s) {
    for (;;) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(own + s) : "memory");
      if (v - e >= 0) break;
      if (clock64() - t0 > limit) {
        if (atomicExch(&g_device_error, kErrGatherTimeout) == 0) {
          g_device_error_info[0] = (int)blockIdx.x;
          g_device_error_info[1] = s;
          g_device_error_info[2] = v;
          g_device_error_info[3] = e;
        }
        return;
      }
      __nanosleep(64);
    }
  }
}

__global__ void gather_sync_dev_kernel(FlagPtrs flags, int world, int rank, int* epoch_ctr, const int* own,
                                       long long limit) {
  signal_then_wait(flags, world, rank, epoch_ctr, own, limit);
}

// The token split's residual all-gather in one launch: every block copies
// its share of this rank's rows to each destination, fences them and takes
// a ticket; the last block to finish (all stores fenced before their
// tickets) resets the ticket, raises this rank's epoch flag everywhere and
// waits (bounded) for every rank's.
__global__ void __launch_bounds__(256) rows_gather_dev_kernel(const uint4* __restrict__ src, DstPtrs dst, int n_dst,
                                                              long long n16, FlagPtrs flags, int world, int rank,
                                                              int* epoch_ctr, const int* own, long long limit,
                                                              unsigned* ticket) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const uint4 v = src[i];
    for (int d = 0; d < n_dst; ++d) dst.p[d][i] = v;
  }
  __shared__ bool last;
  __threadfence_system();  // every thread's peer stores, before the block's ticket
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  if (threadIdx.x == 0) *ticket = 0u;
  __threadfence_system();
  signal_then_wait(flags, world, rank, epoch_ctr, own, limit);
}

}  // namespace cevk

using namespace cevk;

extern "C" {

int cevk_ipc_alloc(int64_t bytes, void** dev_ptr) {
  if (!dev_ptr || bytes <= 0) return set_error(CEVK_E_SHAPE, "ipc_alloc: bad arguments");
  *dev_ptr = nullptr;
  cudaError_t e = cudaMalloc(dev_ptr, (size_t)bytes);
  if (e == cudaSuccess) e = cudaMemset(*dev_ptr, 0, (size_t)bytes);
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "ipc_alloc: %s", cudaGetErrorString(e));
  return CEVK_OK;
}

int cevk_ipc_free(void* dev_ptr) {
  const cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "ipc_free: %s", cudaGetErrorString(e));
  return CEVK_OK;
}

int cevk_ipc_handle(const void* dev_ptr, void* handle) {
  if (!dev_ptr || !handle) return set_error(CEVK_E_SHAPE, "ipc_handle: null argument");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "ipc_handle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == CEVK_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return CEVK_OK;
}

int cevk_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return set_error(CEVK_E_SHAPE, "ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "ipc_open: %s", cudaGetErrorString(e));
  return CEVK_OK;
}

int cevk_ipc_close(void* dev_ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "ipc_close: %s", cudaGetErrorString(e));
  return CEVK_OK;
}

int cevk_gather_signal(int32_t* const* flags, int32_t world, int32_t rank, int32_t epoch, void* stream) {
  if (!flags || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || epoch <= 0)
    return set_error(CEVK_E_SHAPE, "gather_signal: world %d rank %d epoch %d", world, rank, epoch);
  FlagPtrs f{};
  for (int i = 0; i < world; ++i) {
    if (!flags[i]) return set_error(CEVK_E_SHAPE, "gather_signal: null flag array %d", i);
    f.p[i] = flags[i];
  }
  gather_signal_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(f, world, rank, epoch);
  return check_launch("gather_signal_kernel");
}

int cevk_gather_wait(const int32_t* flags, int32_t world, int32_t epoch, int64_t limit_cycles, void* stream) {
  if (!flags || world < 1 || world > kMaxRanks || epoch <= 0 || limit_cycles <= 0)
    return set_error(CEVK_E_SHAPE, "gather_wait: world %d epoch %d", world, epoch);
  gather_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flags, world, epoch, limit_cycles);
  return check_launch("gather_wait_kernel");
}

int cevk_gather_signal_dev(int32_t* const* flags, int32_t world, int32_t rank, int32_t* epoch, void* stream) {
  if (!flags || !epoch || world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return set_error(CEVK_E_SHAPE, "gather_signal_dev: world %d rank %d", world, rank);
  FlagPtrs f{};
  for (int i = 0; i < world; ++i) {
    if (!flags[i]) return set_error(CEVK_E_SHAPE, "gather_signal_dev: null flag array %d", i);
    f.p[i] = flags[i];
  }
  gather_signal_dev_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(f, world, rank, epoch);
  return check_launch("gather_signal_dev_kernel");
}

int cevk_gather_wait_dev(const int32_t* flags, int32_t world, const int32_t* epoch, int64_t limit_cycles,
                         void* stream) {
  if (!flags || !epoch || world < 1 || world > kMaxRanks || limit_cycles <= 0)
    return set_error(CEVK_E_SHAPE, "gather_wait_dev: world %d", world);
  gather_wait_dev_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flags, world, epoch, limit_cycles);
  return check_launch("gather_wait_dev_kernel");
}

int cevk_gather_sync_dev(int32_t* const* flags, int32_t world, int32_t rank, int32_t* epoch, const int32_t* own_flags,
                         int64_t limit_cycles, void* stream) {
  if (!flags || !epoch || !own_flags || world < 1 || world > kMaxRanks || rank < 0 || rank >= world ||
      limit_cycles <= 0)
    return set_error(CEVK_E_SHAPE, "gather_sync_dev: world %d rank %d", world, rank);
  FlagPtrs f{};
  for (int i = 0; i < world; ++i) {
    if (!flags[i]) return set_error(CEVK_E_SHAPE, "gather_sync_dev: null flag array %d", i);
    f.p[i] = flags[i];
  }
  gather_sync_dev_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(f, world, rank, epoch, own_flags,
                                                                               limit_cycles);
  return check_launch("gather_sync_dev_kernel");
}

int cevk_rows_gather_dev(const void* src, void* const* dst, int32_t n_dst, int64_t bytes, int32_t* const* flags,
                         int32_t world, int32_t rank, int32_t* epoch, const int32_t* own_flags, int64_t limit_cycles,
                         uint32_t* ticket, void* stream) {
  if (!src || !dst || n_dst < 1 || n_dst > kMaxRanks || bytes < 0 || (bytes & 15) || ((uintptr_t)src & 15) ||
      !flags || !epoch || !own_flags || !ticket || world < 1 || world > kMaxRanks || rank < 0 || rank >= world ||
      limit_cycles <= 0)
    return set_error(CEVK_E_SHAPE, "rows_gather_dev: %d destinations, %lld bytes, world %d", n_dst,
                     (long long)bytes, world);
  DstPtrs d{};
  for (int i = 0; i < n_dst; ++i) {
    if (!dst[i] || ((uintptr_t)dst[i] & 15)) return set_error(CEVK_E_SHAPE, "rows_gather_dev: destination %d", i);
    d.p[i] = reinterpret_cast<uint4*>(dst[i]);
  }
  FlagPtrs f{};
  for (int i = 0; i < world; ++i) {
    if (!flags[i]) return set_error(CEVK_E_SHAPE, "rows_gather_dev: null flag array %d", i);
    f.p[i] = flags[i];
  }
  const long long n16 = bytes / 16;
  const long long blocks = std::max<long long>(1, std::min<long long>((n16 + 255) / 256, 148 * 8));
  rows_gather_dev_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(src), d, n_dst, n16, f, world, rank, epoch, own_flags, limit_cycles, ticket);
  return check_launch("rows_gather_dev_kernel");
}

int cevk_rows_to_peers(const void* src, void* const* dst, int32_t n_dst, int64_t bytes, void* stream) {
  if (!src || !dst || n_dst < 1 || n_dst > kMaxRanks || bytes < 0 || (bytes & 15) || ((uintptr_t)src & 15))
    return set_error(CEVK_E_SHAPE, "rows_to_peers: %d destinations, %lld bytes", n_dst, (long long)bytes);
  DstPtrs d{};
  for (int i = 0; i < n_dst; ++i) {
    if (!dst[i] || ((uintptr_t)dst[i] & 15)) return set_error(CEVK_E_SHAPE, "rows_to_peers: destination %d", i);
    d.p[i] = reinterpret_cast<uint4*>(dst[i]);
  }
  const long long n16 = bytes / 16;
  if (n16 == 0) return CEVK_OK;
  const long long blocks = std::min<long long>((n16 + 255) / 256, 148 * 8);
  rows_to_peers_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(src), d, n_dst, n16);
  return check_launch("rows_to_peers_kernel");
}

}  // extern "C"
