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
  P3D_CHECK_ARG(op != nullptr && y && sk && sv, "p3d_attn_fwd_noalloc: null argument");
  P3D_CHECK_ARG(dtype_ok(op->dtype) && dtype_ok(op->gate_dtype), "p3d_attn_fwd_noalloc: unknown dtype");
  P3D_CHECK_ARG(op->batch >= 1 && op->heads >= 1 && op->kv_heads >= 1 && op->tokens >= 1 &&
                    op->heads % op->kv_heads == 0,
                "p3d_attn_fwd_noalloc: bad batch / head / token counts");
  P3D_CHECK_ARG(op->head_dim >= 2 && op->head_dim <= 128 && op->head_dim % 2 == 0,
                "p3d_attn_fwd_noalloc: head_dim %d unsupported", op->head_dim);
  P3D_CHECK_ARG(op->temperature > 0.f && op->temperature < __builtin_huge_valf(),
                "p3d_attn_fwd_noalloc: temperature must be finite and positive");
  P3D_CHECK_ARG(op->width >= 1 && op->width <= 128 && op->slots >= 1 && op->slots <= 64 && op->pool_size >= 1 &&
                    op->pool_size <= 32 && op->fine_blocks >= 1,
                "p3d_attn_fwd_noalloc: bad geometry description");
  P3D_CHECK_ARG(op->q && op->kl && op->vl && op->kg && op->vg && op->gate && op->pool_weight && op->slot_bias &&
                    op->local_scale && op->global_scale && op->neighbors && op->blocks,
                "p3d_attn_fwd_noalloc: null input");
  const size_t need = (size_t)op->batch * op->heads * op->tokens * op->head_dim * dtype_size(op->dtype);
  if (need > kScratchBytes)
    return fail(P3D_ERR_UNSUPPORTED,
                "p3d_attn_fwd_noalloc: the local-branch scratch needs %zu bytes but the fixed scratch holds %zu "
                "(B*H*N*D*sizeof(dtype) must not exceed it); use p3d_attn_fwd with a workspace",
                need, kScratchBytes);
  void *scratch = nullptr;
  if (int st = scratch_address(&scratch)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  PoolArgs pa{};
  pa.k = op->kg;
  pa.v = op->vg;
  pa.weight = op->pool_weight;
  pa.bias = op->slot_bias;
  pa.blocks = op->blocks;
  pa.fine_blocks = op->fine_blocks;
  pa.slots = op->slots;
  pa.pool_size = op->pool_size;
  pa.summaries = (op->fine_blocks + op->pool_size - 1) / op->pool_size;
  pa.sk = sk;
  pa.sv = sv;
  pa.dtype = op->dtype;
  pa.bg = op->batch * op->kv_heads;
  pa.tokens = op->tokens;
  pa.head_dim = op->head_dim;
  pa.temperature = op->temperature;
  pa.vec = dtype_size(op->dtype) == 2 && op->head_dim % 8 == 0 && ((uintptr_t)op->kg & 15) == 0 &&
           ((uintptr_t)op->vg & 15) == 0;
  if (int st = launch_pool_fwd(pa, s)) return st;

  IndexedArgs a{};
  a.dtype = op->dtype;
  a.gate_dtype = op->gate_dtype;
  a.batch = op->batch;
  a.heads = op->heads;
  a.kv_heads = op->kv_heads;
  a.tokens = op->tokens;
  a.head_dim = op->head_dim;
  a.summaries = pa.summaries;
  a.q = op->q;
  a.kl = op->kl;
  a.vl = op->vl;
  a.sk = sk;
  a.sv = sv;
  a.neighbors = op->neighbors;
  a.width = op->width;
  a.reverse = op->reverse_neighbors;
  a.reverse_width = op->reverse_width;
  a.gate = op->gate;
  a.sl = op->local_scale;
  a.sg = op->global_scale;
  if (int st = launch_local_fwd_indexed(a, scratch, nullptr, s)) return st;
  return launch_global_fwd_mix(a, scratch, y, nullptr, nullptr, s);
}
