// C ABI entry points: argument validation, workspace layout and stage dispatch.
#include <stdarg.h>
#include <stdio.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace p3d {

static thread_local char g_last_error[512] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int device_info(DeviceInfo *info) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  static bool filled[64] = {};
  int dev = 0;
  P3D_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(P3D_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!filled[dev]) {
    cudaDeviceProp prop;
    P3D_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
    cache[dev].sm_count = prop.multiProcessorCount;
    cache[dev].major = prop.major;
    cache[dev].minor = prop.minor;
    cache[dev].smem_optin = prop.sharedMemPerBlockOptin;
    filled[dev] = true;
  }
  *info = cache[dev];
  return P3D_OK;
}

int summaries_of(const p3d_operator *op) { return (op->fine_blocks + op->pool_size - 1) / op->pool_size; }

int validate(const p3d_operator *op) {
  P3D_CHECK_ARG(op != nullptr, "null operator descriptor");
  P3D_CHECK_ARG(dtype_ok(op->dtype) && dtype_ok(op->gate_dtype), "unknown dtype");
  P3D_CHECK_ARG((op->options & ~(P3D_OPT_INDEXED_ONLY | P3D_OPT_DY_ROWS)) == 0u, "unknown option bits 0x%x",
                op->options);
  P3D_CHECK_ARG(op->batch >= 1 && op->heads >= 1 && op->tokens >= 1 && op->kv_heads >= 1,
                "batch, heads, kv_heads and tokens must be positive");
  P3D_CHECK_ARG(op->heads % op->kv_heads == 0, "query heads must be divisible by KV heads");
  P3D_CHECK_ARG(op->head_dim >= 2 && op->head_dim <= 128 && op->head_dim % 2 == 0,
                "head_dim %d unsupported (even, <= 128)", op->head_dim);
  P3D_CHECK_ARG(op->temperature > 0.f && op->temperature < __builtin_huge_valf(),
                "temperature must be finite and positive");
  P3D_CHECK_ARG(op->width >= 1 && op->width <= 128, "neighbour width must be in [1,128]");
  P3D_CHECK_ARG(op->slots >= 1 && op->slots <= 64, "fine-block slots must be in [1,64]");
  P3D_CHECK_ARG(op->pool_size >= 1 && op->pool_size <= 32, "pool_size must be in [1,32]");
  P3D_CHECK_ARG(op->fine_blocks >= 1, "no fine blocks");
  P3D_CHECK_ARG(op->q && op->kl && op->vl && op->kg && op->vg && op->gate, "null input tensor");
  P3D_CHECK_ARG(op->pool_weight && op->slot_bias && op->local_scale && op->global_scale, "null parameter");
  P3D_CHECK_ARG(op->neighbors && op->blocks, "null geometry table");
  P3D_CHECK_ARG((int64_t)op->batch * op->heads * op->tokens * op->head_dim < (int64_t(1) << 40),
                "tensor too large");
  if (op->stencil) {
    P3D_CHECK_ARG(op->grid[0] >= 1 && op->grid[1] >= 1 && op->grid[2] >= 1, "bad stencil grid");
    P3D_CHECK_ARG((int64_t)op->grid[0] * op->grid[1] * op->grid[2] == op->tokens,
                  "stencil grid does not match the token count");
    P3D_CHECK_ARG(op->radius[0] >= 0 && op->radius[1] >= 0 && op->radius[2] >= 0, "bad stencil radius");
  }
  return P3D_OK;
}

IndexedArgs indexed_args(const p3d_operator *op, const void *sk, const void *sv) {
  IndexedArgs a{};
  a.dtype = op->dtype;
  a.gate_dtype = op->gate_dtype;
  a.batch = op->batch;
  a.heads = op->heads;
  a.kv_heads = op->kv_heads;
  a.tokens = op->tokens;
  a.head_dim = op->head_dim;
  a.summaries = summaries_of(op);
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
  return a;
}

PoolArgs pool_args(const p3d_operator *op, void *sk, void *sv) {
  PoolArgs p{};
  p.k = op->kg;
  p.v = op->vg;
  p.weight = op->pool_weight;
  p.bias = op->slot_bias;
  p.blocks = op->blocks;
  p.fine_blocks = op->fine_blocks;
  p.slots = op->slots;
  p.pool_size = op->pool_size;
  p.summaries = summaries_of(op);
  p.sk = sk;
  p.sv = sv;
  p.dtype = op->dtype;
  p.bg = op->batch * op->kv_heads;
  p.tokens = op->tokens;
  p.head_dim = op->head_dim;
  p.temperature = op->temperature;
  p.vec = dtype_size(op->dtype) == 2 && op->head_dim % 8 == 0 && ((uintptr_t)op->kg & 15) == 0 &&
          ((uintptr_t)op->vg & 15) == 0;
  return p;
}

namespace {

// Bump allocator over a caller-provided workspace (256-byte aligned slices).
struct Carver {
  char *base;
  size_t used = 0, cap;
  Carver(void *b, size_t c) : base(static_cast<char *>(b)), cap(c) {}
  template <typename T>
  T *take(size_t count) {
    used = (used + 255) & ~size_t(255);
    T *p = base ? reinterpret_cast<T *>(base + used) : nullptr;
    used += count * sizeof(T);
    return p;
  }
  bool ok() const { return base != nullptr && used <= cap; }
};

bool use_stencil_path(const p3d_operator *op, unsigned flags) {
  if (flags & P3D_FWD_FORCE_INDEXED) return false;
  if (!op->stencil || (op->options & P3D_OPT_INDEXED_ONLY)) return false;
  return stencil_fwd_supported(op->dtype, op->head_dim, op->radius, summaries_of(op));
}

// Forward workspace: indexed path needs an ol buffer when the caller saves no state;
// the stencil path needs the per-(batch, kv-head) summary-norm bound and, when storage is
// permuted, raster-ordered copies of q, kl, vl.
size_t fwd_layout(const p3d_operator *op, unsigned flags, void *base, size_t cap, void **ol_ws,
                  void **q_r, void **kl_r, void **vl_r, float **kbound) {
  Carver c(base, cap);
  const size_t es = dtype_size(op->dtype);
  const size_t q_elems = (size_t)op->batch * op->heads * op->tokens * op->head_dim;
  const size_t kv_elems = (size_t)op->batch * op->kv_heads * op->tokens * op->head_dim;
  if (use_stencil_path(op, flags)) {
    *kbound = c.take<float>((size_t)op->batch * op->kv_heads);
    if (op->raster_to_packed && !(flags & P3D_FWD_RASTER_QKV)) {
      *q_r = c.take<char>(q_elems * es);
      *kl_r = c.take<char>(kv_elems * es);
      *vl_r = c.take<char>(kv_elems * es);
    }
  } else if (!(flags & P3D_FWD_SAVE_STATE)) {
    *ol_ws = c.take<char>(q_elems * es);
  }
  return c.used;
}

// dst[r, :] = src[map[r], :] for every (batch*head) slab: gathers packed rows into raster order.
__global__ void gather_rows_kernel(const uint4 *src, uint4 *dst, const int32_t *map, int64_t slabs,
                                   int tokens, int row_vecs) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = slabs * tokens * row_vecs;
  if (t >= total) return;
  const int v = (int)(t % row_vecs);
  const int64_t rest = t / row_vecs;
  const int r = (int)(rest % tokens);
  const int64_t slab = rest / tokens;
  dst[(slab * tokens + r) * row_vecs + v] = src[(slab * tokens + map[r]) * row_vecs + v];
}

// dst[slab, r] = src[slab, map[r]]: per-row fp32 values (logsumexp, Delta) into raster order.
__global__ void gather_vals_kernel(const float *src, float *dst, const int32_t *map, int64_t slabs, int tokens) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= slabs * tokens) return;
  const int r = (int)(t % tokens);
  const int64_t slab = t / tokens;
  dst[t] = src[slab * tokens + map[r]];
}

int gather_vals(const float *src, float *dst, const int32_t *map, int64_t slabs, int tokens, cudaStream_t s) {
  const int64_t total = slabs * tokens;
  if (!total) return P3D_OK;
  gather_vals_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(src, dst, map, slabs, tokens);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int gather_rows(const void *src, void *dst, const int32_t *map, int64_t slabs, int tokens, size_t row_bytes,
                cudaStream_t s) {
  if (row_bytes % 16 || ((uintptr_t)src & 15) || ((uintptr_t)dst & 15))
    return fail(P3D_ERR_UNSUPPORTED, "row gather needs 16-byte rows");
  const int row_vecs = (int)(row_bytes / 16);
  const int64_t total = slabs * tokens * row_vecs;
  if (!total) return P3D_OK;
  gather_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      static_cast<const uint4 *>(src), static_cast<uint4 *>(dst), map, slabs, tokens, row_vecs);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

// The tensor-core backward needs what the tensor-core forward needs, and at least two
// summaries (with one the global softmax is constant: no score gradient, reference
// kernels.py:198-199).
// The z-slab (multi-GPU) backward is built and tested for radius 2, the benchmark configurations' radius;
// the single-GPU tensor-core kernels take radius 1 or 2.
bool radius_two(const p3d_operator *op) { return op->radius[0] == 2 && op->radius[1] == 2 && op->radius[2] == 2; }

bool use_stencil_bwd(const p3d_operator *op) {
  return op->stencil && !(op->options & P3D_OPT_INDEXED_ONLY) && summaries_of(op) >= 2 &&
         stencil_fwd_supported(op->dtype, op->head_dim, op->radius, summaries_of(op));
}

// Global dSK / dSV on tensor cores: any token order, 16-bit dtypes, at least two summaries.
bool use_tc_global_dkv(const p3d_operator *op) {
  return !(op->options & P3D_OPT_INDEXED_ONLY) && global_dkv_tc_supported(op->dtype, op->head_dim, summaries_of(op));
}

struct BwdBuffers {
  void *dol, *dog;
  void *q_r, *kl_r, *vl_r, *dol_r, *dog_r;  // raster-order copies (tensor-core path, permuted storage)
  float *lse_g_r, *delta_g_r;               // raster-order copies for the tensor-core global dSK / dSV
  float *delta_l, *delta_g, *dsl_part, *dsg_part, *dk_part, *dv_part, *dsk, *dsv, *dw_part, *db_part, *tmp;
  int64_t mix_rows, pool_rows;
  int splits, per_split;  // global dSK / dSV partials (per_split: tensor-core kernel only)
};

size_t bwd_layout(const p3d_operator *op, void *base, size_t cap, BwdBuffers *b) {
  Carver c(base, cap);
  const size_t es = dtype_size(op->dtype);
  const int M = summaries_of(op);
  const int64_t rows = (int64_t)op->batch * op->heads * op->tokens;
  const int64_t bh = (int64_t)op->batch * op->heads;
  const int64_t bg = (int64_t)op->batch * op->kv_heads;
  const int chunk = mix_bwd_chunk_rows();
  b->mix_rows = bh * ((op->tokens + chunk - 1) / chunk);
  b->pool_rows = bg * M;
  b->per_split = 0;
  if (use_tc_global_dkv(op)) {
    DeviceInfo info{};
    if (device_info(&info) != P3D_OK) info.sm_count = 148;
    global_dkv_tc_splits(op->batch, op->heads, op->kv_heads, op->tokens, M, info.sm_count, &b->splits,
                         &b->per_split);
  } else {
    b->splits = global_dkv_splits(op->tokens);
  }
  const int64_t d = op->head_dim;
  b->dol = c.take<char>(rows * d * es);
  b->dog = c.take<char>(rows * d * es);
  b->q_r = b->kl_r = b->vl_r = b->dol_r = b->dog_r = nullptr;
  b->lse_g_r = b->delta_g_r = nullptr;
  if (use_stencil_bwd(op) && op->raster_to_packed) {
    const int64_t kv_rows = bg * op->tokens;
    b->q_r = c.take<char>(rows * d * es);
    b->dol_r = c.take<char>(rows * d * es);
    b->dog_r = c.take<char>(rows * d * es);
    b->kl_r = c.take<char>(kv_rows * d * es);
    b->vl_r = c.take<char>(kv_rows * d * es);
    if (use_tc_global_dkv(op)) {
      b->lse_g_r = c.take<float>(rows);
      b->delta_g_r = c.take<float>(rows);
    }
  }
  b->delta_l = c.take<float>(rows);
  b->delta_g = c.take<float>(rows);
  b->dsl_part = c.take<float>(b->mix_rows * d);
  b->dsg_part = c.take<float>(b->mix_rows * d);
  b->dk_part = c.take<float>(bg * b->splits * M * d);
  b->dv_part = c.take<float>(bg * b->splits * M * d);
  b->dsk = c.take<float>(bg * M * d);
  b->dsv = c.take<float>(bg * M * d);
  b->dw_part = c.take<float>(b->pool_rows * d);
  b->db_part = c.take<float>(b->pool_rows * op->slots);
  const int64_t tmp = std::max({sum_rows_tmp(b->mix_rows, d), sum_rows_tmp(b->pool_rows, d),
                                sum_rows_tmp(b->pool_rows, op->slots)});
  b->tmp = c.take<float>(tmp);
  return c.used;
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" {

const char *p3d_strerror(int status) {
  switch (status) {
    case P3D_OK: return "success";
    case P3D_ERR_INVALID_ARGUMENT: return "invalid argument";
    case P3D_ERR_UNSUPPORTED: return "unsupported input";
    case P3D_ERR_CUDA: return "CUDA error";
    case P3D_ERR_WORKSPACE: return "workspace missing or too small";
    case P3D_ERR_DEVICE: return "no usable device";
    default: return "unknown status";
  }
}

const char *p3d_last_error(void) { return g_last_error; }

int p3d_abi_version(void) { return P3D_ABI_VERSION; }

int p3d_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int count = 0;
  for (int i = 0; i < n; ++i) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, i) == cudaSuccess && prop.major == 10) ++count;
  }
  return count;
}

int p3d_device_errors(unsigned *flags) {
  P3D_CHECK_ARG(flags != nullptr, "p3d_device_errors: null output");
  *flags = 0;
  if (int st = take_fwd_errors(flags)) return st;
  if (int st = take_proj_errors(flags)) return st;
  if (int st = take_peer_errors(flags)) return st;
  return take_bwd_errors(flags);
}

int p3d_pool_fwd(const void *k, const void *v, const float *weight, const float *bias, const int32_t *blocks,
                 int fine_blocks, int slots, int pool_size, void *sk, void *sv, float *sk32, float *sv32,
                 int dtype, int batch, int kv_heads, int tokens, int head_dim, float temperature,
                 void *stream) {
  P3D_CHECK_ARG(dtype_ok(dtype), "p3d_pool_fwd: unknown dtype");
  P3D_CHECK_ARG(k && v && weight && bias && blocks && sk && sv, "p3d_pool_fwd: null pointer");
  P3D_CHECK_ARG(slots >= 1 && slots <= 64 && pool_size >= 1 && pool_size <= 32 && fine_blocks >= 1,
                "p3d_pool_fwd: bad block table");
  P3D_CHECK_ARG(head_dim >= 1 && head_dim <= 128, "p3d_pool_fwd: head_dim must be in [1,128]");
  P3D_CHECK_ARG(temperature > 0.f, "p3d_pool_fwd: temperature must be positive");
  PoolArgs p{};
  p.k = k; p.v = v; p.weight = weight; p.bias = bias; p.blocks = blocks;
  p.fine_blocks = fine_blocks; p.slots = slots; p.pool_size = pool_size;
  p.summaries = (fine_blocks + pool_size - 1) / pool_size;
  p.sk = sk; p.sv = sv; p.sk32 = sk32; p.sv32 = sv32;
  p.dtype = dtype; p.bg = batch * kv_heads; p.tokens = tokens; p.head_dim = head_dim;
  p.temperature = temperature;
  p.vec = dtype_size(dtype) == 2 && head_dim % 8 == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0;
  return launch_pool_fwd(p, static_cast<cudaStream_t>(stream));
}

size_t p3d_attn_fwd_workspace(const p3d_operator *op, unsigned flags) {
  if (validate(op) != P3D_OK) return 0;
  void *a = nullptr, *b = nullptr, *c = nullptr, *d = nullptr;
  float *e = nullptr;
  return fwd_layout(op, flags, nullptr, 0, &a, &b, &c, &d, &e);
}

int p3d_stencil_fwd_supported(int dtype, int head_dim, int rz, int ry, int rx, int summaries) {
  const int radius[3] = {rz, ry, rx};
  return stencil_fwd_supported(dtype, head_dim, radius, summaries) ? 1 : 0;
}

int p3d_summary_bound(const void *sk, int dtype, int batch, int kv_heads, int summaries, int head_dim,
                      float *bound, void *stream) {
  P3D_CHECK_ARG(sk && bound, "p3d_summary_bound: null pointer");
  P3D_CHECK_ARG(batch >= 1 && kv_heads >= 1 && summaries >= 1, "p3d_summary_bound: bad shape");
  return launch_summary_bound(sk, dtype, batch * kv_heads, summaries, head_dim, bound,
                              static_cast<cudaStream_t>(stream));
}

int p3d_attn_fwd(const p3d_operator *op, void *y, void *sk, void *sv, void *ol, void *og, float *lse_l,
                 float *lse_g, unsigned flags, void *workspace, size_t workspace_bytes, void *stream) {
  if (int st = validate(op)) return st;
  P3D_CHECK_ARG(y && sk && sv, "p3d_attn_fwd: y, sk and sv are required");
  P3D_CHECK_ARG((flags & ~(unsigned)(P3D_FWD_SAVE_STATE | P3D_FWD_FORCE_INDEXED | P3D_FWD_SUMMARIES_GIVEN |
                                     P3D_FWD_Y_ROWS | P3D_FWD_RASTER_QKV)) == 0u,
                "p3d_attn_fwd: unknown flags 0x%x", flags);
  if ((flags & P3D_FWD_RASTER_QKV) && !use_stencil_path(op, flags))
    return fail(P3D_ERR_UNSUPPORTED, "p3d_attn_fwd: raster-ordered q, kl, vl need the tensor-core stencil path");
  const bool save = flags & P3D_FWD_SAVE_STATE;
  P3D_CHECK_ARG(!save || (ol && og && lse_l && lse_g), "p3d_attn_fwd: saving state needs ol, og, lse_l, lse_g");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void *ol_ws = nullptr, *q_r = nullptr, *kl_r = nullptr, *vl_r = nullptr;
  float *kbound = nullptr;
  const size_t need = fwd_layout(op, flags, nullptr, 0, &ol_ws, &q_r, &kl_r, &vl_r, &kbound);
  if (need > 0) {
    if (!workspace || workspace_bytes < need)
      return fail(P3D_ERR_WORKSPACE, "p3d_attn_fwd: workspace of %zu bytes required", need);
    fwd_layout(op, flags, workspace, workspace_bytes, &ol_ws, &q_r, &kl_r, &vl_r, &kbound);
  }
  if (!(flags & P3D_FWD_SUMMARIES_GIVEN))
    if (int st = launch_pool_fwd(pool_args(op, sk, sv), s)) return st;
  if (use_stencil_path(op, flags)) {
    StencilFwdArgs a{};
    a.radius = op->radius[0];
    a.dtype = op->dtype;
    a.gate_dtype = op->gate_dtype;
    a.batch = op->batch;
    a.heads = op->heads;
    a.kv_heads = op->kv_heads;
    a.head_dim = op->head_dim;
    a.summaries = summaries_of(op);
    for (int i = 0; i < 3; ++i) a.grid[i] = op->grid[i];
    a.global_planes = a.k_planes = op->grid[0];
    a.q_z0 = a.k_z0 = 0;
    a.q = op->q;
    a.kl = op->kl;
    a.vl = op->vl;
    if (op->raster_to_packed && !(flags & P3D_FWD_RASTER_QKV)) {
      const size_t row_bytes = (size_t)op->head_dim * dtype_size(op->dtype);
      if (int st = gather_rows(op->q, q_r, op->raster_to_packed, (int64_t)op->batch * op->heads, op->tokens,
                               row_bytes, s))
        return st;
      if (int st = gather_rows(op->kl, kl_r, op->raster_to_packed, (int64_t)op->batch * op->kv_heads,
                               op->tokens, row_bytes, s))
        return st;
      if (int st = gather_rows(op->vl, vl_r, op->raster_to_packed, (int64_t)op->batch * op->kv_heads,
                               op->tokens, row_bytes, s))
        return st;
      a.q = q_r;
      a.kl = kl_r;
      a.vl = vl_r;
    }
    a.raster_to_packed = op->raster_to_packed;
    a.sk = sk;
    a.sv = sv;
    a.gate = op->gate;
    a.sl = op->local_scale;
    a.sg = op->global_scale;
    a.y = y;
    a.ol = save ? ol : nullptr;
    a.og = save ? og : nullptr;
    a.lse_l = save ? lse_l : nullptr;
    a.lse_g = save ? lse_g : nullptr;
    a.y_rows = (flags & P3D_FWD_Y_ROWS) != 0;
    if (int st = launch_summary_bound(sk, op->dtype, op->batch * op->kv_heads, a.summaries, op->head_dim, kbound, s))
      return st;
    a.summary_bound = kbound;
    return launch_stencil_fwd(a, s);
  }
  IndexedArgs a = indexed_args(op, sk, sv);
  a.y_rows = (flags & P3D_FWD_Y_ROWS) != 0;
  void *ol_buf = save ? ol : ol_ws;
  if (int st = launch_local_fwd_indexed(a, ol_buf, save ? lse_l : nullptr, s)) return st;
  return launch_global_fwd_mix(a, ol_buf, y, save ? og : nullptr, save ? lse_g : nullptr, s);
}

int p3d_attn_fwd_slab(const p3d_operator *op, const p3d_slab *slab, void *y, const void *sk, const void *sv,
                      void *ol, void *og, float *lse_l, float *lse_g, unsigned flags, void *stream) {
  if (int st = validate(op)) return st;
  P3D_CHECK_ARG(slab != nullptr && y && sk && sv, "p3d_attn_fwd_slab: slab, y, sk and sv are required");
  const bool save = flags & P3D_FWD_SAVE_STATE;
  P3D_CHECK_ARG(!save || (ol && og && lse_l && lse_g), "p3d_attn_fwd_slab: saving state needs ol, og, lse_l, lse_g");
  P3D_CHECK_ARG((flags & ~(unsigned)(P3D_FWD_SAVE_STATE | P3D_FWD_SUMMARIES_GIVEN | P3D_FWD_Y_ROWS)) == 0u,
                "p3d_attn_fwd_slab: unsupported flags 0x%x", flags);
  P3D_CHECK_ARG(op->stencil && !op->raster_to_packed,
                "p3d_attn_fwd_slab: needs a complete stencil in raster storage");
  P3D_CHECK_ARG(!(op->options & P3D_OPT_INDEXED_ONLY), "p3d_attn_fwd_slab: has no indexed form");
  if (!stencil_fwd_supported(op->dtype, op->head_dim, op->radius, slab->summaries))
    return fail(P3D_ERR_UNSUPPORTED, "p3d_attn_fwd_slab: needs bf16/f16, head_dim 16/32/48/64, radius 1 or 2 and sm_100");
  const int nz = op->grid[0], r = op->radius[0];
  const int need_lo = std::max(0, slab->center_z0 - r);
  const int need_hi = std::min(slab->global_planes, slab->center_z0 + nz + r);
  P3D_CHECK_ARG(slab->global_planes >= 1 && slab->center_z0 >= 0 && slab->center_z0 + nz <= slab->global_planes,
                "p3d_attn_fwd_slab: rank planes [%d, %d) outside the volume of %d planes", slab->center_z0,
                slab->center_z0 + nz, slab->global_planes);
  P3D_CHECK_ARG(slab->halo_z0 <= need_lo && slab->halo_z0 + slab->halo_planes >= need_hi && slab->halo_z0 >= 0 &&
                    slab->halo_z0 + slab->halo_planes <= slab->global_planes,
                "p3d_attn_fwd_slab: kl/vl planes [%d, %d) do not cover [%d, %d)", slab->halo_z0,
                slab->halo_z0 + slab->halo_planes, need_lo, need_hi);
  P3D_CHECK_ARG(slab->summaries >= 1, "p3d_attn_fwd_slab: no summaries");
  StencilFwdArgs a{};
  a.radius = op->radius[0];
  a.dtype = op->dtype;
  a.gate_dtype = op->gate_dtype;
  a.batch = op->batch;
  a.heads = op->heads;
  a.kv_heads = op->kv_heads;
  a.head_dim = op->head_dim;
  a.summaries = slab->summaries;
  for (int i = 0; i < 3; ++i) a.grid[i] = op->grid[i];
  a.global_planes = slab->global_planes;
  a.q_z0 = slab->center_z0;
  a.k_z0 = slab->halo_z0;
  a.k_planes = slab->halo_planes;
  a.q = op->q;
  a.kl = op->kl;
  a.vl = op->vl;
  a.raster_to_packed = nullptr;
  a.sk = sk;
  a.sv = sv;
  a.gate = op->gate;
  a.sl = op->local_scale;
  a.sg = op->global_scale;
  a.y = y;
  a.ol = save ? ol : nullptr;
  a.og = save ? og : nullptr;
  a.lse_l = save ? lse_l : nullptr;
  a.lse_g = save ? lse_g : nullptr;
  a.y_rows = (flags & P3D_FWD_Y_ROWS) != 0;
  a.summary_bound = slab->summary_bound;
  P3D_CHECK_ARG(slab->tile_z_begin >= 0 && slab->tile_z_end >= 0 &&
                    (slab->tile_z_end == 0 || slab->tile_z_begin < slab->tile_z_end),
                "p3d_attn_fwd_slab: bad tile range [%d, %d)", slab->tile_z_begin, slab->tile_z_end);
  a.tile_z_begin = slab->tile_z_begin;
  a.tile_z_end = slab->tile_z_end;
  return launch_stencil_fwd(a, static_cast<cudaStream_t>(stream));
}

size_t p3d_attn_bwd_workspace(const p3d_operator *op) {
  if (validate(op) != P3D_OK) return 0;
  BwdBuffers b;
  return bwd_layout(op, nullptr, 0, &b);
}

int p3d_attn_bwd(const p3d_operator *op, const void *dy, const void *sk, const void *sv, const void *ol,
                 const void *og, const float *lse_l, const float *lse_g, void *dq, void *dkl, void *dvl, void *dkg,
                 void *dvg, void *dgate, float *dweight, float *dbias, float *dlocal_scale, float *dglobal_scale,
                 void *workspace, size_t workspace_bytes, void *stream) {
  if (int st = validate(op)) return st;
  P3D_CHECK_ARG(dy && sk && sv && ol && og && lse_l && lse_g, "p3d_attn_bwd: missing saved state");
  P3D_CHECK_ARG(dq && dkl && dvl && dkg && dvg && dgate && dweight && dbias && dlocal_scale && dglobal_scale,
                "p3d_attn_bwd: missing gradient output");
  P3D_CHECK_ARG(op->reverse_neighbors && op->reverse_width >= 1 && op->reverse_width <= 128,
                "p3d_attn_bwd: reverse adjacency required");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  BwdBuffers b;
  const size_t need = bwd_layout(op, nullptr, 0, &b);
  if (!workspace || workspace_bytes < need)
    return fail(P3D_ERR_WORKSPACE, "p3d_attn_bwd: workspace of %zu bytes required", need);
  bwd_layout(op, workspace, workspace_bytes, &b);
  const int d = op->head_dim, M = summaries_of(op);
  const int64_t bh = (int64_t)op->batch * op->heads, bg = (int64_t)op->batch * op->kv_heads;

  MixBwdArgs mix{};
  mix.dtype = op->dtype;
  mix.gate_dtype = op->gate_dtype;
  mix.bh = (int)bh;
  mix.tokens = op->tokens;
  mix.head_dim = d;
  mix.chunk_rows = mix_bwd_chunk_rows();
  mix.heads = op->heads;
  mix.dy_rows = (op->options & P3D_OPT_DY_ROWS) ? 1 : 0;
  mix.dy = dy;
  mix.ol = ol;
  mix.og = og;
  mix.gate = op->gate;
  mix.sl = op->local_scale;
  mix.sg = op->global_scale;
  mix.dol = b.dol;
  mix.dog = b.dog;
  mix.delta_l = b.delta_l;
  mix.delta_g = b.delta_g;
  mix.dgate = dgate;
  mix.dsl_part = b.dsl_part;
  mix.dsg_part = b.dsg_part;
  if (int st = launch_mix_bwd(mix, s)) return st;

  const IndexedArgs a = indexed_args(op, sk, sv);
  if (use_stencil_bwd(op)) {
    StencilBwdArgs t{};
    t.radius = op->radius[0];
    t.dtype = op->dtype;
    t.batch = op->batch;
    t.heads = op->heads;
    t.kv_heads = op->kv_heads;
    t.head_dim = d;
    t.summaries = M;
    for (int i = 0; i < 3; ++i) t.grid[i] = op->grid[i];
    t.global_planes = t.k_planes = op->grid[0];
    t.q_z0 = t.k_z0 = 0;
    t.q = op->q;
    t.kl = op->kl;
    t.vl = op->vl;
    t.dol = b.dol;
    t.dog = b.dog;
    if (op->raster_to_packed) {
      const size_t row_bytes = (size_t)d * dtype_size(op->dtype);
      const void *src[5] = {op->q, op->kl, op->vl, b.dol, b.dog};
      void *dst[5] = {b.q_r, b.kl_r, b.vl_r, b.dol_r, b.dog_r};
      const int64_t heads[5] = {bh, bg, bg, bh, bh};
      for (int i = 0; i < 5; ++i)
        if (int st = gather_rows(src[i], dst[i], op->raster_to_packed, heads[i], op->tokens, row_bytes, s)) return st;
      t.q = b.q_r;
      t.kl = b.kl_r;
      t.vl = b.vl_r;
      t.dol = b.dol_r;
      t.dog = b.dog_r;
    }
    t.sk = sk;
    t.sv = sv;
    t.lse_l = lse_l;
    t.lse_g = lse_g;
    t.delta_l = b.delta_l;
    t.delta_g = b.delta_g;
    t.raster_to_packed = op->raster_to_packed;
    t.dq = dq;
    t.dkl = dkl;
    t.dvl = dvl;
    t.q_halo = t.q;
    t.dol_halo = t.dol;
    t.lse_l_halo = lse_l;
    t.delta_l_halo = b.delta_l;
    t.x_z0 = 0;
    t.x_planes = op->grid[0];
    if (int st = launch_stencil_bwd_dq(t, s)) return st;
    if (int st = launch_stencil_bwd_dkv(t, s)) return st;
  } else {
    if (int st = launch_local_dq_indexed(a, b.dol, lse_l, b.delta_l, dq, s)) return st;
    if (int st = launch_local_dkv_indexed(a, b.dol, lse_l, b.delta_l, dkl, dvl, s)) return st;
    if (int st = launch_global_dq(a, b.dog, lse_g, b.delta_g, dq, s)) return st;
  }
  if (use_tc_global_dkv(op)) {
    GlobalDkvArgs g{};
    g.dtype = op->dtype;
    g.batch = op->batch;
    g.heads = op->heads;
    g.kv_heads = op->kv_heads;
    g.tokens = op->tokens;
    g.head_dim = d;
    g.summaries = M;
    g.splits = b.splits;
    g.per_split = b.per_split;
    g.q = op->q;
    g.dog = b.dog;
    g.sk = sk;
    g.sv = sv;
    g.lse_g = lse_g;
    g.delta_g = b.delta_g;
    if (b.lse_g_r) {
      // Permuted storage: visit the queries in raster order, as raster storage does, so that
      // the fixed-order query sums (and with them dK_g, dV_g) do not depend on the storage.
      if (int st = gather_vals(lse_g, b.lse_g_r, op->raster_to_packed, bh, op->tokens, s)) return st;
      if (int st = gather_vals(b.delta_g, b.delta_g_r, op->raster_to_packed, bh, op->tokens, s)) return st;
      g.q = b.q_r;
      g.dog = b.dog_r;
      g.lse_g = b.lse_g_r;
      g.delta_g = b.delta_g_r;
    }
    g.dk_part = b.dk_part;
    g.dv_part = b.dv_part;
    if (int st = launch_global_dkv_tc(g, s)) return st;
  } else {
    if (int st = launch_global_dkv(a, b.dog, lse_g, b.delta_g, b.splits, b.dk_part, b.dv_part, s)) return st;
  }
  if (int st = launch_sum_middle(b.dk_part, b.dsk, bg, b.splits, (int64_t)M * d, s)) return st;
  if (int st = launch_sum_middle(b.dv_part, b.dsv, bg, b.splits, (int64_t)M * d, s)) return st;

  PoolBwdArgs pb{};
  pb.k = op->kg;
  pb.v = op->vg;
  pb.weight = op->pool_weight;
  pb.bias = op->slot_bias;
  pb.blocks = op->blocks;
  pb.fine_blocks = op->fine_blocks;
  pb.slots = op->slots;
  pb.pool_size = op->pool_size;
  pb.summaries = M;
  pb.dsk = b.dsk;
  pb.dsv = b.dsv;
  pb.dk = dkg;
  pb.dv = dvg;
  pb.dw_part = b.dw_part;
  pb.db_part = b.db_part;
  pb.dtype = op->dtype;
  pb.bg = (int)bg;
  pb.tokens = op->tokens;
  pb.head_dim = d;
  pb.temperature = op->temperature;
  pb.vec = pool_args(op, nullptr, nullptr).vec;
  if (int st = launch_pool_bwd(pb, s)) return st;

  if (int st = launch_sum_rows(b.dw_part, dweight, b.pool_rows, d, b.tmp, s)) return st;
  if (int st = launch_sum_rows(b.db_part, dbias, b.pool_rows, op->slots, b.tmp, s)) return st;
  if (int st = launch_sum_rows(b.dsl_part, dlocal_scale, b.mix_rows, d, b.tmp, s)) return st;
  if (int st = launch_sum_rows(b.dsg_part, dglobal_scale, b.mix_rows, d, b.tmp, s)) return st;
  return P3D_OK;
}


// ------------------------------------------------------------------ staged backward
// The backward in three stages, for callers that interleave their own communication:
// the z-slab sharding runs mix -> (halo exchange) -> attention -> (reduce-scatter of the
// summary gradients) -> pooling.  p3d_attn_bwd is the composition of the same kernels.

static size_t mix_layout(const p3d_operator *op, void *base, size_t cap, float **dsl_part, float **dsg_part,
                         float **tmp, int64_t *mix_rows) {
  Carver c(base, cap);
  const int chunk = mix_bwd_chunk_rows();
  const int64_t bh = (int64_t)op->batch * op->heads;
  *mix_rows = bh * ((op->tokens + chunk - 1) / chunk);
  *dsl_part = c.take<float>(*mix_rows * op->head_dim);
  *dsg_part = c.take<float>(*mix_rows * op->head_dim);
  *tmp = c.take<float>(sum_rows_tmp(*mix_rows, op->head_dim));
  return c.used;
}

size_t p3d_bwd_mix_workspace(const p3d_operator *op) {
  if (validate(op) != P3D_OK) return 0;
  float *a, *b, *t;
  int64_t r;
  return mix_layout(op, nullptr, 0, &a, &b, &t, &r);
}

int p3d_bwd_mix(const p3d_operator *op, const void *dy, const void *ol, const void *og, void *dol, void *dog,
                float *delta_l, float *delta_g, void *dgate, float *dlocal_scale, float *dglobal_scale, void *workspace,
                size_t workspace_bytes, void *stream) {
  if (int st = validate(op)) return st;
  P3D_CHECK_ARG(dy && ol && og && dol && dog && delta_l && delta_g && dgate && dlocal_scale && dglobal_scale,
                "p3d_bwd_mix: null argument");
  float *dsl_part, *dsg_part, *tmp;
  int64_t mix_rows;
  const size_t need = mix_layout(op, nullptr, 0, &dsl_part, &dsg_part, &tmp, &mix_rows);
  if (!workspace || workspace_bytes < need)
    return fail(P3D_ERR_WORKSPACE, "p3d_bwd_mix: workspace of %zu bytes required", need);
  mix_layout(op, workspace, workspace_bytes, &dsl_part, &dsg_part, &tmp, &mix_rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  MixBwdArgs mix{};
  mix.dtype = op->dtype;
  mix.gate_dtype = op->gate_dtype;
  mix.bh = op->batch * op->heads;
  mix.tokens = op->tokens;
  mix.head_dim = op->head_dim;
  mix.chunk_rows = mix_bwd_chunk_rows();
  mix.heads = op->heads;
  mix.dy_rows = (op->options & P3D_OPT_DY_ROWS) ? 1 : 0;
  mix.dy = dy;
  mix.ol = ol;
  mix.og = og;
  mix.gate = op->gate;
  mix.sl = op->local_scale;
  mix.sg = op->global_scale;
  mix.dol = dol;
  mix.dog = dog;
  mix.delta_l = delta_l;
  mix.delta_g = delta_g;
  mix.dgate = dgate;
  mix.dsl_part = dsl_part;
  mix.dsg_part = dsg_part;
  if (int st = launch_mix_bwd(mix, s)) return st;
  if (int st = launch_sum_rows(dsl_part, dlocal_scale, mix_rows, op->head_dim, tmp, s)) return st;
  return launch_sum_rows(dsg_part, dglobal_scale, mix_rows, op->head_dim, tmp, s);
}

static int check_slab(const p3d_operator *op, const p3d_slab *slab, const char *what) {
  P3D_CHECK_ARG(slab != nullptr, "%s: null slab", what);
  P3D_CHECK_ARG(op->stencil && !op->raster_to_packed, "%s: needs a complete stencil in raster storage", what);
  P3D_CHECK_ARG(!(op->options & P3D_OPT_INDEXED_ONLY), "%s: has no indexed form", what);
  if (!stencil_fwd_supported(op->dtype, op->head_dim, op->radius, slab->summaries) || slab->summaries < 2 ||
      !radius_two(op) || !global_dkv_tc_supported(op->dtype, op->head_dim, slab->summaries))
    return fail(P3D_ERR_UNSUPPORTED, "%s: needs bf16/f16, head_dim 16/32/48/64, radius 2, >= 2 summaries, sm_100",
                what);
  const int nz = op->grid[0], r = op->radius[0];
  const int need_lo = std::max(0, slab->center_z0 - r);
  const int need_hi = std::min(slab->global_planes, slab->center_z0 + nz + r);
  P3D_CHECK_ARG(slab->global_planes >= 1 && slab->center_z0 >= 0 && slab->center_z0 + nz <= slab->global_planes,
                "%s: rank planes [%d, %d) outside the volume of %d planes", what, slab->center_z0,
                slab->center_z0 + nz, slab->global_planes);
  P3D_CHECK_ARG(slab->halo_z0 <= need_lo && slab->halo_z0 + slab->halo_planes >= need_hi && slab->halo_z0 >= 0 &&
                    slab->halo_z0 + slab->halo_planes <= slab->global_planes,
                "%s: halo planes [%d, %d) do not cover [%d, %d)", what, slab->halo_z0,
                slab->halo_z0 + slab->halo_planes, need_lo, need_hi);
  return P3D_OK;
}

static size_t attn_slab_layout(const p3d_operator *op, int summaries, void *base, size_t cap, float **dk_part,
                               float **dv_part, int *splits, int *per_split) {
  Carver c(base, cap);
  DeviceInfo info{};
  if (device_info(&info) != P3D_OK) info.sm_count = 148;
  global_dkv_tc_splits(op->batch, op->heads, op->kv_heads, op->tokens, summaries, info.sm_count, splits, per_split);
  const int64_t n = (int64_t)op->batch * op->kv_heads * *splits * summaries * op->head_dim;
  *dk_part = c.take<float>(n);
  *dv_part = c.take<float>(n);
  return c.used;
}

size_t p3d_bwd_attn_slab_workspace(const p3d_operator *op, const p3d_slab *slab) {
  if (validate(op) != P3D_OK || !slab) return 0;
  float *a, *b;
  int sp, per;
  return attn_slab_layout(op, slab->summaries, nullptr, 0, &a, &b, &sp, &per);
}

int p3d_bwd_attn_slab(const p3d_operator *op, const p3d_slab *slab, const void *sk, const void *sv,
                      const float *lse_l, const float *lse_g, const void *dol, const void *dog, const float *delta_l,
                      const float *delta_g, const void *q_halo, const void *dol_halo, const float *lse_l_halo,
                      const float *delta_l_halo, void *dq, void *dkl, void *dvl, float *dsk, float *dsv,
                      void *workspace, size_t workspace_bytes, void *stream) {
  if (int st = validate(op)) return st;
  if (int st = check_slab(op, slab, "p3d_bwd_attn_slab")) return st;
  P3D_CHECK_ARG(sk && sv && lse_l && lse_g && dol && dog && delta_l && delta_g && q_halo && dol_halo && lse_l_halo &&
                    delta_l_halo && dq && dkl && dvl && dsk && dsv,
                "p3d_bwd_attn_slab: null argument");
  float *dk_part, *dv_part;
  int splits, per_split;
  const size_t need = attn_slab_layout(op, slab->summaries, nullptr, 0, &dk_part, &dv_part, &splits, &per_split);
  if (!workspace || workspace_bytes < need)
    return fail(P3D_ERR_WORKSPACE, "p3d_bwd_attn_slab: workspace of %zu bytes required", need);
  attn_slab_layout(op, slab->summaries, workspace, workspace_bytes, &dk_part, &dv_part, &splits, &per_split);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  StencilBwdArgs t{};
  t.radius = op->radius[0];
  t.dtype = op->dtype;
  t.batch = op->batch;
  t.heads = op->heads;
  t.kv_heads = op->kv_heads;
  t.head_dim = op->head_dim;
  t.summaries = slab->summaries;
  for (int i = 0; i < 3; ++i) t.grid[i] = op->grid[i];
  t.global_planes = slab->global_planes;
  t.q_z0 = slab->center_z0;
  t.k_z0 = slab->halo_z0;
  t.k_planes = slab->halo_planes;
  t.q = op->q;
  t.kl = op->kl;
  t.vl = op->vl;
  t.dol = dol;
  t.dog = dog;
  t.sk = sk;
  t.sv = sv;
  t.lse_l = lse_l;
  t.lse_g = lse_g;
  t.delta_l = delta_l;
  t.delta_g = delta_g;
  t.raster_to_packed = nullptr;
  t.dq = dq;
  t.dkl = dkl;
  t.dvl = dvl;
  t.q_halo = q_halo;
  t.dol_halo = dol_halo;
  t.lse_l_halo = lse_l_halo;
  t.delta_l_halo = delta_l_halo;
  t.x_z0 = slab->halo_z0;
  t.x_planes = slab->halo_planes;
  if (int st = launch_stencil_bwd_dq(t, s)) return st;
  if (int st = launch_stencil_bwd_dkv(t, s)) return st;
  GlobalDkvArgs g{};
  g.dtype = op->dtype;
  g.batch = op->batch;
  g.heads = op->heads;
  g.kv_heads = op->kv_heads;
  g.tokens = op->tokens;
  g.head_dim = op->head_dim;
  g.summaries = slab->summaries;
  g.splits = splits;
  g.per_split = per_split;
  g.q = op->q;
  g.dog = dog;
  g.sk = sk;
  g.sv = sv;
  g.lse_g = lse_g;
  g.delta_g = delta_g;
  g.dk_part = dk_part;
  g.dv_part = dv_part;
  if (int st = launch_global_dkv_tc(g, s)) return st;
  const int64_t bg = (int64_t)op->batch * op->kv_heads;
  if (int st = launch_sum_middle(dk_part, dsk, bg, splits, (int64_t)slab->summaries * op->head_dim, s)) return st;
  return launch_sum_middle(dv_part, dsv, bg, splits, (int64_t)slab->summaries * op->head_dim, s);
}

static size_t pool_bwd_layout(int64_t pool_rows, int dim, int slots, void *base, size_t cap, float **dw_part,
                              float **db_part, float **tmp) {
  Carver c(base, cap);
  *dw_part = c.take<float>(pool_rows * dim);
  *db_part = c.take<float>(pool_rows * slots);
  *tmp = c.take<float>(std::max(sum_rows_tmp(pool_rows, dim), sum_rows_tmp(pool_rows, slots)));
  return c.used;
}

size_t p3d_pool_bwd_workspace(int fine_blocks, int slots, int pool_size, int batch, int kv_heads, int head_dim) {
  if (fine_blocks < 1 || slots < 1 || pool_size < 1 || batch < 1 || kv_heads < 1 || head_dim < 1) return 0;
  const int64_t rows = (int64_t)batch * kv_heads * ((fine_blocks + pool_size - 1) / pool_size);
  float *a, *b, *t;
  return pool_bwd_layout(rows, head_dim, slots, nullptr, 0, &a, &b, &t);
}

int p3d_pool_bwd(const void *k, const void *v, const float *weight, const float *bias, const int32_t *blocks,
                 int fine_blocks, int slots, int pool_size, const float *dsk, const float *dsv, void *dk, void *dv,
                 float *dweight, float *dbias, int dtype, int batch, int kv_heads, int tokens, int head_dim,
                 float temperature, void *workspace, size_t workspace_bytes, void *stream) {
  P3D_CHECK_ARG(dtype_ok(dtype), "p3d_pool_bwd: unknown dtype");
  P3D_CHECK_ARG(k && v && weight && bias && blocks && dsk && dsv && dk && dv && dweight && dbias,
                "p3d_pool_bwd: null pointer");
  P3D_CHECK_ARG(fine_blocks >= 1 && slots >= 1 && slots <= 64 && pool_size >= 1 && pool_size <= 32,
                "p3d_pool_bwd: bad blocks description");
  P3D_CHECK_ARG(batch >= 1 && kv_heads >= 1 && tokens >= 1 && head_dim >= 2 && head_dim <= 128,
                "p3d_pool_bwd: bad extents");
  P3D_CHECK_ARG(temperature > 0.f && temperature < __builtin_huge_valf(), "p3d_pool_bwd: bad temperature");
  const int M = (fine_blocks + pool_size - 1) / pool_size;
  const int64_t rows = (int64_t)batch * kv_heads * M;
  float *dw_part, *db_part, *tmp;
  const size_t need = pool_bwd_layout(rows, head_dim, slots, nullptr, 0, &dw_part, &db_part, &tmp);
  if (!workspace || workspace_bytes < need)
    return fail(P3D_ERR_WORKSPACE, "p3d_pool_bwd: workspace of %zu bytes required", need);
  pool_bwd_layout(rows, head_dim, slots, workspace, workspace_bytes, &dw_part, &db_part, &tmp);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PoolBwdArgs pb{};
  pb.k = k;
  pb.v = v;
  pb.weight = weight;
  pb.bias = bias;
  pb.blocks = blocks;
  pb.fine_blocks = fine_blocks;
  pb.slots = slots;
  pb.pool_size = pool_size;
  pb.summaries = M;
  pb.dsk = dsk;
  pb.dsv = dsv;
  pb.dk = dk;
  pb.dv = dv;
  pb.dw_part = dw_part;
  pb.db_part = db_part;
  pb.dtype = dtype;
  pb.bg = batch * kv_heads;
  pb.tokens = tokens;
  pb.head_dim = head_dim;
  pb.temperature = temperature;
  pb.vec = dtype_size(dtype) == 2 && head_dim % 8 == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0;
  if (int st = launch_pool_bwd(pb, s)) return st;
  if (int st = launch_sum_rows(dw_part, dweight, rows, head_dim, tmp, s)) return st;
  return launch_sum_rows(db_part, dbias, rows, slots, tmp, s);
}

}  // extern "C"
