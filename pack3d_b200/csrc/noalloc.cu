// Forward pass without any device allocation: p3d_attn_fwd_noalloc.
//
// Some callers cannot allocate device memory at all: plugins running inside a host
// framework that owns every byte of device memory and hands out none (inference servers
// with a fixed arena, sandboxed plugin hosts), and hard-real-time loops that must not
// hit the device-wide synchronisation that cudaMalloc / cudaFree may cause.  Such a
// caller still provides its inputs and outputs, but cannot provide the scratch buffer
// p3d_attn_fwd asks for.  This entry point runs the neighbour-table (indexed) forward,
// whose only scratch is the local-branch output ol [B, H, N, D], and keeps that scratch
// in a fixed array compiled into the library.
//
// The array is a file-scope __device__ object, so every GPU that loads the library holds
// its kScratchBytes until the process exits.  Host code cannot use the array's name as a
// device address (it names a host-side shadow); the device address is obtained with
// cudaGetSymbolAddress once per device, with that device current, on the first call made
// on it -- so that first call should come before any stream capture.  All calls share the
// array and it keeps the last call's contents: nothing in it needs to start at zero (the
// local kernel writes every element before the global kernel reads it), and two calls
// whose kernels overlap on the GPU (different streams, no ordering) race on it.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace p3d {
namespace {

// Largest local-branch output the fixed scratch holds: B * H * N * D * sizeof(dtype) bytes.
constexpr size_t kScratchBytes = size_t(16) << 20;  // 16 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_address(void **out) {
  static std::mutex mu;
  static void *addr[kMaxDevices] = {};
  int dev = 0;
  P3D_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(P3D_ERR_DEVICE, "p3d_attn_fwd_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void *p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr)
      return fail(P3D_ERR_CUDA, "p3d_attn_fwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(err));
    addr[dev] = p;
  }
  *out = addr[dev];
  return P3D_OK;
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" int p3d_attn_fwd_noalloc(const p3d_operator *op, void *y, void *sk, void *sv, void *stream) {
  // The same argument checks as p3d_attn_fwd (the shared validate(); the forward reads no
  // reverse adjacency); only the scratch size is checked here.
  if (int st = validate(op)) return st;
  P3D_CHECK_ARG(y && sk && sv, "p3d_attn_fwd_noalloc: y, sk and sv are required");
  const size_t need = (size_t)op->batch * op->heads * op->tokens * op->head_dim * dtype_size(op->dtype);
  if (need > kScratchBytes)
    return fail(P3D_ERR_UNSUPPORTED,
                "p3d_attn_fwd_noalloc: the local-branch scratch needs %zu bytes but the fixed scratch holds %zu "
                "(B*H*N*D*sizeof(dtype) must not exceed it); use p3d_attn_fwd with a workspace",
                need, kScratchBytes);
  void *scratch = nullptr;
  if (int st = scratch_address(&scratch)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int st = launch_pool_fwd(pool_args(op, sk, sv), s)) return st;
  const IndexedArgs a = indexed_args(op, sk, sv);
  if (int st = launch_local_fwd_indexed(a, scratch, nullptr, s)) return st;
  return launch_global_fwd_mix(a, scratch, y, nullptr, nullptr, s);
}
