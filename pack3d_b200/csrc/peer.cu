// Peer-memory exchange for the z-slab sharding (one process per GPU on one node).
//
// Each rank allocates one region of device memory and hands its CUDA IPC handle to the other
// ranks, which map it into their address space (NVLink peer memory).  A rank's region holds
// the buffers its slab kernels read -- its keys / values with the halo planes around them
// and the summaries of every rank -- and two counters.  Per layer call a rank:
//
//   1. waits (one thread, bounded) until every peer has finished reading what it pushed in
//      the previous call: its `credits` counter, raised by one by every peer per call;
//   2. pushes (p3d_peer_push, many CTAs): its summaries into every peer's summary buffer and
//      its boundary planes into the neighbours' halo rows, with 16-byte stores over NVLink;
//      every CTA then adds one to each target's `arrivals` counter (release, system scope)
//      and copies this rank's own rows into its own region;
//   3. waits (one thread, bounded) until every peer's push has arrived: its `arrivals`
//      counter, raised by ctas per peer per call;
//   4. runs its kernels on its region, then raises every peer's `credits` by one.
//
// The counters only grow (64-bit), and the expected values live in device memory and are
// advanced by the wait kernel itself, so a CUDA graph captured over a call replays
// correctly.  A wait that runs out of time sets kErrTimeout | kErrPeer in this file's error
// word (read by p3d_device_errors) and returns; nothing spins without a bound.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"
#include "../../include/pack3d_b200.h"

namespace p3d {
namespace {

using sm100::global_timer_ns;
using sm100::kErrTimeout;

constexpr unsigned kErrPeer = 32u;
__device__ unsigned g_peer_errors = 0;

constexpr int kPushThreads = 512;

struct PushParams {
  p3d_peer_copy copy[P3D_PEER_MAX_COPIES];
  unsigned long long *arrive[P3D_PEER_MAX_TARGETS];
  int n_copies, n_remote, n_arrive;
};

// copy.rows rows of copy.row_bytes bytes (a multiple of 16), strided in bytes on both sides;
// this CTA takes every gridDim.x-th 16-byte word, four words in flight per thread.
__device__ __forceinline__ void copy_rows(const p3d_peer_copy &c) {
  const int64_t words_per_row = c.row_bytes >> 4;
  const int64_t words = c.rows * words_per_row;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const char *src = static_cast<const char *>(c.src);
  char *dst = static_cast<char *>(c.dst);
  for (; w + 3 * stride < words; w += 4 * stride) {
    uint4 v[4];
    int64_t off_d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t wu = w + u * stride;
      const int64_t r = wu / words_per_row, k = wu - r * words_per_row;
      v[u] = __ldg(reinterpret_cast<const uint4 *>(src + r * c.src_stride) + k);
      off_d[u] = r * c.dst_stride + (k << 4);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) *reinterpret_cast<uint4 *>(dst + off_d[u]) = v[u];
  }
  for (; w < words; w += stride) {
    const int64_t r = w / words_per_row, k = w - r * words_per_row;
    *reinterpret_cast<uint4 *>(dst + r * c.dst_stride + (k << 4)) =
        __ldg(reinterpret_cast<const uint4 *>(src + r * c.src_stride) + k);
  }
}

__global__ void __launch_bounds__(kPushThreads) peer_push_kernel(const __grid_constant__ PushParams p) {
  for (int i = 0; i < p.n_remote; ++i) copy_rows(p.copy[i]);
  // every thread's peer stores are ordered before the CTA's arrivals
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < p.n_arrive; ++i) {
      asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(p.arrive[i]) : "memory");
    }
  }
  for (int i = p.n_remote; i < p.n_copies; ++i) copy_rows(p.copy[i]);
}

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long *a) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// One thread: wait until *counter >= *expected (at most timeout_ns), then *expected += step.
__global__ void peer_wait_kernel(const unsigned long long *counter, unsigned long long *expected,
                                 unsigned long long step, uint64_t timeout_ns) {
  const unsigned long long target = *expected;
  const uint64_t t0 = global_timer_ns();
  while (load_acquire_sys(counter) < target) {
    if (global_timer_ns() - t0 > timeout_ns) {
      atomicOr(&g_peer_errors, kErrTimeout | kErrPeer);
      break;
    }
    __nanosleep(200);
  }
  *expected = target + step;
}

struct SignalParams {
  unsigned long long *counter[P3D_PEER_MAX_TARGETS];
  int n;
};

// One thread: add one to every counter (release, system scope), after this stream's
// earlier work.
__global__ void peer_signal_kernel(const __grid_constant__ SignalParams p) {
  __threadfence_system();
  for (int i = 0; i < p.n; ++i) asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(p.counter[i]) : "memory");
}

}  // namespace

int take_peer_errors(unsigned *flags) {
  unsigned v = 0, zero = 0;
  P3D_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_peer_errors, sizeof(v)));
  P3D_CUDA_TRY(cudaMemcpyToSymbol(g_peer_errors, &zero, sizeof(zero)));
  *flags |= v;
  return P3D_OK;
}

}  // namespace p3d

using namespace p3d;

extern "C" {

int p3d_peer_alloc(size_t bytes, void **ptr, void *handle) {
  P3D_CHECK_ARG(ptr && handle && bytes > 0, "p3d_peer_alloc: null output or empty region");
  *ptr = nullptr;
  void *p = nullptr;
  P3D_CUDA_TRY(cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    P3D_CUDA_TRY(e);
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return P3D_OK;
}

int p3d_peer_free(void *ptr) {
  P3D_CHECK_ARG(ptr != nullptr, "p3d_peer_free: null region");
  P3D_CUDA_TRY(cudaFree(ptr));
  return P3D_OK;
}

int p3d_peer_open(const void *handle, void **ptr) {
  P3D_CHECK_ARG(ptr && handle, "p3d_peer_open: null handle or output");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  P3D_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return P3D_OK;
}

int p3d_peer_close(void *ptr) {
  P3D_CHECK_ARG(ptr != nullptr, "p3d_peer_close: null mapping");
  P3D_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return P3D_OK;
}

int p3d_peer_push(const p3d_peer_copy *copies, int n_copies, int n_remote, uint64_t *const *arrive, int n_arrive,
                  int ctas, void *stream) {
  P3D_CHECK_ARG(n_copies >= 0 && n_copies <= P3D_PEER_MAX_COPIES && n_remote >= 0 && n_remote <= n_copies,
                "p3d_peer_push: %d copies (%d remote), at most %d", n_copies, n_remote, P3D_PEER_MAX_COPIES);
  P3D_CHECK_ARG(n_arrive >= 0 && n_arrive <= P3D_PEER_MAX_TARGETS, "p3d_peer_push: %d targets, at most %d",
                n_arrive, P3D_PEER_MAX_TARGETS);
  P3D_CHECK_ARG(ctas >= 1 && ctas <= 4096, "p3d_peer_push: ctas must be in [1, 4096]");
  P3D_CHECK_ARG(n_copies == 0 || copies != nullptr, "p3d_peer_push: null copies");
  P3D_CHECK_ARG(n_arrive == 0 || arrive != nullptr, "p3d_peer_push: null targets");
  PushParams p;
  std::memset(&p, 0, sizeof(p));
  for (int i = 0; i < n_copies; ++i) {
    const p3d_peer_copy &c = copies[i];
    P3D_CHECK_ARG(c.rows >= 0 && c.row_bytes >= 0 && c.row_bytes % 16 == 0, "p3d_peer_push: copy %d: row bytes %lld "
                  "not a multiple of 16", i, (long long)c.row_bytes);
    P3D_CHECK_ARG(c.rows == 0 || c.row_bytes == 0 || (c.src && c.dst), "p3d_peer_push: copy %d: null pointer", i);
    P3D_CHECK_ARG(reinterpret_cast<uintptr_t>(c.src) % 16 == 0 && reinterpret_cast<uintptr_t>(c.dst) % 16 == 0 &&
                      c.src_stride % 16 == 0 && c.dst_stride % 16 == 0,
                  "p3d_peer_push: copy %d: addresses and strides must be 16-byte aligned", i);
    p.copy[i] = c;
  }
  for (int i = 0; i < n_arrive; ++i) {
    P3D_CHECK_ARG(arrive[i] != nullptr && reinterpret_cast<uintptr_t>(arrive[i]) % 8 == 0,
                  "p3d_peer_push: target %d: null or unaligned counter", i);
    p.arrive[i] = reinterpret_cast<unsigned long long *>(arrive[i]);
  }
  p.n_copies = n_copies;
  p.n_remote = n_remote;
  p.n_arrive = n_arrive;
  peer_push_kernel<<<ctas, kPushThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  P3D_CUDA_TRY(cudaGetLastError());
  return P3D_OK;
}

int p3d_peer_wait(const uint64_t *counter, uint64_t *expected, uint64_t step, double timeout_s, void *stream) {
  P3D_CHECK_ARG(counter && expected, "p3d_peer_wait: null counter");
  P3D_CHECK_ARG(reinterpret_cast<uintptr_t>(counter) % 8 == 0 && reinterpret_cast<uintptr_t>(expected) % 8 == 0,
                "p3d_peer_wait: unaligned counter");
  P3D_CHECK_ARG(timeout_s > 0.0 && timeout_s <= 600.0, "p3d_peer_wait: timeout must be in (0, 600] s");
  peer_wait_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const unsigned long long *>(counter), reinterpret_cast<unsigned long long *>(expected),
      static_cast<unsigned long long>(step), static_cast<uint64_t>(timeout_s * 1e9));
  P3D_CUDA_TRY(cudaGetLastError());
  return P3D_OK;
}

int p3d_peer_signal(uint64_t *const *counters, int n, void *stream) {
  P3D_CHECK_ARG(n >= 0 && n <= P3D_PEER_MAX_TARGETS && (n == 0 || counters), "p3d_peer_signal: bad targets");
  SignalParams p;
  std::memset(&p, 0, sizeof(p));
  for (int i = 0; i < n; ++i) {
    P3D_CHECK_ARG(counters[i] != nullptr && reinterpret_cast<uintptr_t>(counters[i]) % 8 == 0,
                  "p3d_peer_signal: target %d: null or unaligned counter", i);
    p.counter[i] = reinterpret_cast<unsigned long long *>(counters[i]);
  }
  p.n = n;
  peer_signal_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(p);
  P3D_CUDA_TRY(cudaGetLastError());
  return P3D_OK;
}

}  // extern "C"
