// Stage (b): two-stage summary pooling, forward and backward.
//
// Restates compression.py:28-44 (forward) and the VJP that autograd takes through
// it (the reference Triton kernels _pool / _pool_bwd, kernels.py:13-40,243-272):
//   fine stage   a = softmax_slots(k . w / T + bias[slot]) over valid slots,
//                fine = sum_slots a * member
//   coarse stage summary m = mean of the fine summaries of the nonempty fine
//                blocks [m*P, (m+1)*P).
// One warp owns one (summary, batch*kv-head) pair.  The slot softmax runs with a
// lane per slot (two slots per lane, V <= 64) and warp-shuffle max / sum; the
// weighted member sums run with a lane per channel, broadcasting each slot's
// weight and row index from its owner lane, so member rows are read coalesced.
// Backward writes per-summary partials of dW / dBias that a fixed-order
// reduction sums -- no atomics, bit-reproducible.
#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace p3d {
namespace {

using sm100::add2;
using sm100::fma2;
using sm100::mul2;

constexpr int kWarps = 4;
constexpr float kNegInf = -__builtin_huge_valf();

template <typename T>
__device__ __forceinline__ float row_dot(const T *row, const float *w, int d, bool vec) {
  return dot_row<T>(row, w, d, vec);
}

struct FineWeights {
  float a[2];     // softmax weight of slots lane and lane+32 (0 for empty)
  int idx[2];     // member token row (-1 for empty)
  bool nonempty;  // warp-uniform
};

// Slot softmax of fine block f (lane owns slots lane, lane+32).
template <typename T>
__device__ __forceinline__ FineWeights fine_weights(const T *K, const int32_t *blocks, int f, int slots,
                                                   const float *w, const float *bias, int d, float inv_temp,
                                                   bool vec) {
  const int lane = threadIdx.x & 31;
  FineWeights fw;
  float logit[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int s = lane + 32 * j;
    fw.idx[j] = s < slots ? blocks[(int64_t)f * slots + s] : -1;
    logit[j] = kNegInf;
    if (fw.idx[j] >= 0) logit[j] = row_dot(K + (int64_t)fw.idx[j] * d, w, d, vec) * inv_temp + bias[s];
  }
  const float mx = warp_max(fmaxf(logit[0], logit[1]));
  fw.nonempty = mx != kNegInf;
  float e[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) e[j] = fw.idx[j] >= 0 ? expf(logit[j] - mx) : 0.f;
  const float sum = warp_sum(e[0] + e[1]);
  const float inv = fw.nonempty ? 1.f / sum : 0.f;
  fw.a[0] = e[0] * inv;
  fw.a[1] = e[1] * inv;
  return fw;
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) pool_fwd_kernel(PoolArgs p) {
  extern __shared__ float smem[];
  float *w = smem;                 // [D]
  float *bias = smem + p.head_dim; // [V]
  for (int i = threadIdx.x; i < p.head_dim; i += blockDim.x) w[i] = p.weight[i];
  for (int i = threadIdx.x; i < p.slots; i += blockDim.x) bias[i] = p.bias[i];
  __syncthreads();
  const int warp = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int M = p.summaries;
  if (warp >= M * p.bg) return;
  const int m = warp % M, bg = warp / M;
  const int d = p.head_dim;
  const T *K = static_cast<const T *>(p.k) + (int64_t)bg * p.tokens * d;
  const T *V = static_cast<const T *>(p.v) + (int64_t)bg * p.tokens * d;
  const float inv_temp = 1.f / p.temperature;
  float acc_k[4] = {0.f, 0.f, 0.f, 0.f}, acc_v[4] = {0.f, 0.f, 0.f, 0.f};
  int count = 0;
  const int f_end = min(p.fine_blocks, (m + 1) * p.pool_size);
  for (int f = m * p.pool_size; f < f_end; ++f) {
    const FineWeights fw = fine_weights(K, p.blocks, f, p.slots, w, bias, d, inv_temp, p.vec);
    if (!fw.nonempty) continue;
    ++count;
    for (int s = 0; s < p.slots; ++s) {
      const int owner = s & 31, j = s >> 5;
      const float a = __shfl_sync(0xffffffffu, j ? fw.a[1] : fw.a[0], owner);
      const int idx = __shfl_sync(0xffffffffu, j ? fw.idx[1] : fw.idx[0], owner);
      if (idx < 0) continue;
      const T *kr = K + (int64_t)idx * d, *vr = V + (int64_t)idx * d;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int ch = lane + 32 * c;
        if (ch < d) {
          acc_k[c] = fmaf(a, to_f32<T>(kr[ch]), acc_k[c]);
          acc_v[c] = fmaf(a, to_f32<T>(vr[ch]), acc_v[c]);
        }
      }
    }
  }
  const float inv_count = 1.f / (float)count;  // every coarse group holds a nonempty block
  const int64_t out = ((int64_t)bg * M + m) * d;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int ch = lane + 32 * c;
    if (ch < d) {
      const float sk = acc_k[c] * inv_count, sv = acc_v[c] * inv_count;
      static_cast<T *>(p.sk)[out + ch] = from_f32<T>(sk);
      static_cast<T *>(p.sv)[out + ch] = from_f32<T>(sv);
      if (p.sk32) p.sk32[out + ch] = sk;
      if (p.sv32) p.sv32[out + ch] = sv;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) pool_bwd_kernel(PoolBwdArgs p) {
  extern __shared__ float smem[];
  const int d = p.head_dim;
  float *w = smem;                       // [D]
  float *bias = w + d;                   // [V]
  float *grad = bias + p.slots + (threadIdx.x >> 5) * 2 * d;  // per warp: dfine_k [D], dfine_v [D]
  for (int i = threadIdx.x; i < d; i += blockDim.x) w[i] = p.weight[i];
  for (int i = threadIdx.x; i < p.slots; i += blockDim.x) bias[i] = p.bias[i];
  __syncthreads();
  const int warp = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int M = p.summaries;
  if (warp >= M * p.bg) return;
  const int m = warp % M, bg = warp / M;
  const T *K = static_cast<const T *>(p.k) + (int64_t)bg * p.tokens * d;
  const T *V = static_cast<const T *>(p.v) + (int64_t)bg * p.tokens * d;
  T *DK = static_cast<T *>(p.dk) + (int64_t)bg * p.tokens * d;
  T *DV = static_cast<T *>(p.dv) + (int64_t)bg * p.tokens * d;
  const float inv_temp = 1.f / p.temperature;
  const int f_begin = m * p.pool_size, f_end = min(p.fine_blocks, (m + 1) * p.pool_size);
  // Number of nonempty fine blocks of this summary (the coarse mean's divisor).
  int count = 0;
  for (int f = f_begin; f < f_end; ++f) {
    const bool any = (lane < p.slots && p.blocks[(int64_t)f * p.slots + lane] >= 0) ||
                     (lane + 32 < p.slots && p.blocks[(int64_t)f * p.slots + lane + 32] >= 0);
    count += __any_sync(0xffffffffu, any) ? 1 : 0;
  }
  const float inv_count = 1.f / (float)count;
  const int64_t srow = ((int64_t)bg * M + m) * d;
  for (int ch = lane; ch < d; ch += 32) {
    grad[ch] = p.dsk[srow + ch] * inv_count;
    grad[d + ch] = p.dsv[srow + ch] * inv_count;
  }
  __syncwarp();
  float dw[4] = {0.f, 0.f, 0.f, 0.f};
  float db[2] = {0.f, 0.f};
  for (int f = f_begin; f < f_end; ++f) {
    const FineWeights fw = fine_weights(K, p.blocks, f, p.slots, w, bias, d, inv_temp, p.vec);
    if (!fw.nonempty) continue;
    // da_s = member_k . dfine_k + member_v . dfine_v; ds = a * (da - sum a*da)
    float da[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      da[j] = 0.f;
      if (fw.idx[j] >= 0)
        da[j] = row_dot(K + (int64_t)fw.idx[j] * d, grad, d, p.vec) +
                row_dot(V + (int64_t)fw.idx[j] * d, grad + d, d, p.vec);
    }
    const float mean = warp_sum(fw.a[0] * da[0] + fw.a[1] * da[1]);
    float ds[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      ds[j] = fw.a[j] * (da[j] - mean);
      db[j] += ds[j];
    }
    for (int s = 0; s < p.slots; ++s) {
      const int owner = s & 31, j = s >> 5;
      const float a = __shfl_sync(0xffffffffu, j ? fw.a[1] : fw.a[0], owner);
      const float dsv = __shfl_sync(0xffffffffu, j ? ds[1] : ds[0], owner);
      const int idx = __shfl_sync(0xffffffffu, j ? fw.idx[1] : fw.idx[0], owner);
      if (idx < 0) continue;
      const T *kr = K + (int64_t)idx * d;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int ch = lane + 32 * c;
        if (ch < d) {
          const float wt = w[ch] * inv_temp;
          DK[(int64_t)idx * d + ch] = from_f32<T>(fmaf(a, grad[ch], dsv * wt));
          DV[(int64_t)idx * d + ch] = from_f32<T>(a * grad[d + ch]);
          dw[c] = fmaf(dsv, to_f32<T>(kr[ch]) * inv_temp, dw[c]);
        }
      }
    }
  }
  const int64_t prow = (int64_t)bg * M + m;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int ch = lane + 32 * c;
    if (ch < d) p.dw_part[prow * d + ch] = dw[c];
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int s = lane + 32 * j;
    if (s < p.slots) p.db_part[prow * p.slots + s] = db[j];
  }
}

// ---------------------------------------------------------------- staged 16-bit path
// The kernels above read each member row from global memory once per use, with one lane per
// slot for the dot products and dependent 2-byte loads per channel for the sums: latency-
// bound at a fraction of HBM bandwidth.  For 16-bit rows with 16-byte-aligned rows and a
// head_dim of 8, 16, 32, 48, 64 or 128, the staged kernels below (one warp per summary, as
// above; the head_dim a template parameter, so every index is compile-time arithmetic and
// the loops unroll) gather a fine block's member K and V rows into the warp's shared memory
// with 16-byte cp.async copies -- consecutive lanes on consecutive chunks of a row, one
// coalesced segment per row -- and take every use from there: each K / V byte crosses HBM
// once.  The V rows are in flight while the slot softmax runs on K.
//
// Slot softmax and the backward's per-slot dots run with a lane per slot (two slots per
// lane) in channel order, as the kernels above.  The weighted member sums (and the
// backward's dweight) run with a lane per (slot group, 16-byte chunk): lane = group * C +
// chunk for C = D / 8 chunks and G = 32 / C groups, group g taking slots g, g + G, ...; the
// group partials meet in shared memory and are added in group order -- deterministic, but a
// different summation order from the kernels above (agreement to fp32 rounding).
//
// Staged K rows are padded to an odd number of 16-byte chunks: a lane-per-row read of one
// chunk column then touches 8 distinct 16-byte bank groups in each quarter-warp phase.  V
// rows stay unpadded (their (group, chunk) reads already spread over the banks), which keeps
// a warp's staging small enough for 16 resident warps per SM.  Each CTA (two warps) starts
// its first gather before loading the pooling weights, so the weight load, the block-table
// load and the gather overlap.
constexpr int kStageWarps = 2;

template <int D>
struct Staging {
  static constexpr int kChunks = D / 8;          // 16-byte chunks per row
  static constexpr int kStride = kChunks | 1;    // padded row stride (chunks)
  static constexpr int kGroups = 32 / kChunks;   // slot groups of the (group, chunk) lane map
  static constexpr int kSlotIters = (64 + kGroups - 1) / kGroups;  // a group's slots (<= 64)
  static constexpr size_t kHead = ((size_t)4 * (D + 64) + 15) & ~(size_t)15;  // w [D], bias [64]
  // One warp: k rows [slots][kStride] and v rows [slots][kChunks] (at least the 2 KB group-
  // partials scratch they host afterwards), idx [64], a [64] (, ds [64], grad [2D] in the
  // backward).
  static __host__ __device__ size_t rows(int slots) {
    const size_t r = (size_t)slots * (kStride + kChunks) * 16;
    return r < 2048 ? 2048 : r;
  }
  static __host__ __device__ size_t per_warp(int slots, bool bwd) { return rows(slots) + 64 * 4 * (bwd ? 3 : 2) + (bwd ? 8 * D : 0); }
};

struct Stage {
  uint4 *k, *v;    // [slots][kStride], [slots][kChunks] 16-byte chunks
  float *scratch;  // overlays k / v once the rows are consumed: [32 lanes][16] fp32
  int *idx;        // [64] member row per slot (-1: empty)
  float *a, *ds;   // [64] slot weights (, slot score gradients)
  float *grad;     // [2D] fp32 (backward)
};

template <int D>
__device__ __forceinline__ Stage stage_at(unsigned char *smem, int slots, bool bwd) {
  using G = Staging<D>;
  const size_t rows = G::rows(slots);
  unsigned char *mine = smem + G::kHead + (threadIdx.x >> 5) * G::per_warp(slots, bwd);
  Stage S;
  S.k = reinterpret_cast<uint4 *>(mine);
  S.v = S.k + (size_t)slots * G::kStride;
  S.scratch = reinterpret_cast<float *>(mine);
  S.idx = reinterpret_cast<int *>(mine + rows);
  S.a = reinterpret_cast<float *>(S.idx + 64);
  S.ds = bwd ? S.a + 64 : nullptr;
  S.grad = bwd ? S.a + 128 : nullptr;
  return S;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Stage fine block f: slot table into idx (and two registers per lane), then the K rows and
// the V rows as two cp.async groups (row r <- member row idx[r]; empty slots skipped).
template <typename T, int D>
__device__ __forceinline__ void stage_block(const Stage &S, const T *K, const T *V, const int32_t *blocks, int f,
                                            int slots, int (&idx)[2]) {
  constexpr int C = Staging<D>::kChunks;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int s = lane + 32 * j;
    idx[j] = s < slots ? blocks[(int64_t)f * slots + s] : -1;
    S.idx[s] = idx[j];
  }
  __syncwarp();
  constexpr int kIters = (64 * C + 31) / 32;  // slots <= 64: compile-time trip count, predicated
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    uint4 *dst = pass ? S.v : S.k;
    const int stride = pass ? C : Staging<D>::kStride;
    const T *src = pass ? V : K;
#pragma unroll
    for (int i = 0; i < kIters; ++i) {
      const int e = lane + 32 * i, r = e / C, c = e - r * C;
      if (e < slots * C) {
        const int row = S.idx[r];
        if (row >= 0) cp_async16(dst + r * stride + c, src + (int64_t)row * D + c * 8);
      }
    }
    cp_async_commit();
  }
}

// Dots of two staged 16-bit rows with an fp32 shared vector, each in channel order (dot_row's
// order), as one packed f32x2 chain: .x for row0, .y for row1.
template <typename T, int D>
__device__ __forceinline__ float2 staged_dot2(const uint4 *row0, const uint4 *row1, const float *w) {
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    const uint4 r0 = row0[c], r1 = row1[c];
    const uint32_t u0[4] = {r0.x, r0.y, r0.z, r0.w}, u1[4] = {r1.x, r1.y, r1.z, r1.w};
    const float4 w0 = *reinterpret_cast<const float4 *>(w + 8 * c);
    const float4 w1 = *reinterpret_cast<const float4 *>(w + 8 * c + 4);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = unpack2<T>(u0[i]), b = unpack2<T>(u1[i]);
      acc = fma2(make_float2(a.x, b.x), make_float2(wv[2 * i], wv[2 * i]), acc);
      acc = fma2(make_float2(a.y, b.y), make_float2(wv[2 * i + 1], wv[2 * i + 1]), acc);
    }
  }
  return acc;
}

// acc[i] += a * chunk[i] over the 8 channels of a 16-byte chunk (pairs packed f32x2).
template <typename T>
__device__ __forceinline__ void axpy8(float a, const uint4 &raw, float2 (&acc)[4]) {
  const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
  const float2 aa = make_float2(a, a);
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = fma2(aa, unpack2<T>(u[i]), acc[i]);
}

__device__ __forceinline__ uint32_t bits16(__half v) { return __half_as_ushort(v); }
__device__ __forceinline__ uint32_t bits16(__nv_bfloat16 v) { return __bfloat16_as_ushort(v); }
// Two fp32 values rounded to T, packed low-first.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float x, float y) {
  return bits16(from_f32<T>(x)) | (bits16(from_f32<T>(y)) << 16);
}

// Slot softmax of a staged fine block (lane owns slots lane, lane+32); fine_weights' math.
template <typename T, int D>
__device__ __forceinline__ FineWeights staged_weights(const Stage &S, const int (&idx)[2], const float *w,
                                                      const float *bias, float inv_temp) {
  const int lane = threadIdx.x & 31;
  FineWeights fw;
  // an empty slot reads staged row 0 (in bounds, possibly stale) and its dot is discarded
  const float2 dot = staged_dot2<T, D>(S.k + (idx[0] >= 0 ? lane : 0) * Staging<D>::kStride,
                                       S.k + (idx[1] >= 0 ? lane + 32 : 0) * Staging<D>::kStride, w);
  float logit[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    fw.idx[j] = idx[j];
    logit[j] = idx[j] >= 0 ? (j ? dot.y : dot.x) * inv_temp + bias[lane + 32 * j] : kNegInf;
  }
  const float mx = warp_max(fmaxf(logit[0], logit[1]));
  fw.nonempty = mx != kNegInf;
  float e[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) e[j] = idx[j] >= 0 ? expf(logit[j] - mx) : 0.f;
  const float sum = warp_sum(e[0] + e[1]);
  const float inv = fw.nonempty ? 1.f / sum : 0.f;
  fw.a[0] = e[0] * inv;
  fw.a[1] = e[1] * inv;
  return fw;
}

__device__ __forceinline__ uint64_t valid_slots(const int (&idx)[2]) {
  const uint64_t lo = __ballot_sync(0xffffffffu, idx[0] >= 0), hi = __ballot_sync(0xffffffffu, idx[1] >= 0);
  return lo | (hi << 32);
}

// Park this lane's 8 group partials at offset off of its 16-float scratch row.
__device__ __forceinline__ void park8(float *scratch, int off, const float2 (&part)[4]) {
  float *mine = scratch + (threadIdx.x & 31) * 16 + off;
  *reinterpret_cast<float4 *>(mine) = make_float4(part[0].x, part[0].y, part[1].x, part[1].y);
  *reinterpret_cast<float4 *>(mine + 4) = make_float4(part[2].x, part[2].y, part[3].x, part[3].y);
}
// Output channel o summed over the groups in order (partials at offset off).
template <int D>
__device__ __forceinline__ float sum_groups(const float *scratch, int o, int off) {
  constexpr int C = Staging<D>::kChunks, G = Staging<D>::kGroups;
  const float *col = scratch + (o >> 3) * 16 + (o & 7) + off;
  float sum = 0.f;
#pragma unroll
  for (int g = 0; g < G; ++g) sum += col[g * C * 16];
  return sum;
}

template <typename T, int D>
__global__ void __launch_bounds__(kStageWarps * 32, 8) pool_fwd_staged_kernel(PoolArgs p) {
  using G = Staging<D>;
  extern __shared__ __align__(16) unsigned char stage_smem[];
  const int V = p.slots, M = p.summaries;
  const int warp = blockIdx.x * kStageWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const bool has = warp < M * p.bg;  // warp-uniform
  const int m = has ? warp % M : 0, bg = has ? warp / M : 0;
  const Stage S = stage_at<D>(stage_smem, V, false);
  const T *K = static_cast<const T *>(p.k) + (int64_t)bg * p.tokens * D;
  const T *Vt = static_cast<const T *>(p.v) + (int64_t)bg * p.tokens * D;
  const int f_begin = m * p.pool_size, f_end = min(p.fine_blocks, (m + 1) * p.pool_size);
  int idx[2];
  if (has) stage_block<T, D>(S, K, Vt, p.blocks, f_begin, V, idx);
  float *w = reinterpret_cast<float *>(stage_smem);
  float *bias = w + D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) w[i] = p.weight[i];
  for (int i = threadIdx.x; i < V; i += blockDim.x) bias[i] = p.bias[i];
  __syncthreads();
  if (!has) return;
  const float inv_temp = 1.f / p.temperature;
  const int grp = lane / G::kChunks, chunk = lane - grp * G::kChunks;  // (slot group, chunk) lane map
  const bool mapped = grp < G::kGroups;
  float2 acc_k[4], acc_v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc_k[i] = acc_v[i] = make_float2(0.f, 0.f);
  int count = 0;
  for (int f = f_begin; f < f_end; ++f) {
    if (f != f_begin) stage_block<T, D>(S, K, Vt, p.blocks, f, V, idx);
    cp_async_wait<1>();  // K rows
    __syncwarp();
    const FineWeights fw = staged_weights<T, D>(S, idx, w, bias, inv_temp);
    S.a[lane] = fw.a[0];
    S.a[lane + 32] = fw.a[1];
    const uint64_t valid = valid_slots(idx);
    cp_async_wait<0>();  // V rows
    __syncwarp();
    if (fw.nonempty) {
      ++count;
      if (mapped) {
#pragma unroll 4
        for (int it = 0; it < G::kSlotIters; ++it) {
          const int s = grp + G::kGroups * it;
          if (s < V && ((valid >> s) & 1)) {
            const float a = S.a[s];
            axpy8<T>(a, S.k[s * G::kStride + chunk], acc_k);
            axpy8<T>(a, S.v[s * G::kChunks + chunk], acc_v);
          }
        }
      }
    }
    __syncwarp();  // the next fine block (or the scratch) overwrites the rows
  }
  park8(S.scratch, 0, acc_k);
  park8(S.scratch, 8, acc_v);
  __syncwarp();
  const float inv_count = 1.f / (float)count;  // every coarse group holds a nonempty block
  const int64_t out = ((int64_t)bg * M + m) * D;
  for (int o = lane; o < D; o += 32) {
    const float sk = sum_groups<D>(S.scratch, o, 0) * inv_count;
    const float sv = sum_groups<D>(S.scratch, o, 8) * inv_count;
    static_cast<T *>(p.sk)[out + o] = from_f32<T>(sk);
    static_cast<T *>(p.sv)[out + o] = from_f32<T>(sv);
    if (p.sk32) p.sk32[out + o] = sk;
    if (p.sv32) p.sv32[out + o] = sv;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kStageWarps * 32, 7) pool_bwd_staged_kernel(PoolBwdArgs p) {
  using G = Staging<D>;
  extern __shared__ __align__(16) unsigned char stage_smem[];
  const int V = p.slots, M = p.summaries;
  const int warp = blockIdx.x * kStageWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const bool has = warp < M * p.bg;  // warp-uniform
  const int m = has ? warp % M : 0, bg = has ? warp / M : 0;
  const Stage S = stage_at<D>(stage_smem, V, true);
  const T *K = static_cast<const T *>(p.k) + (int64_t)bg * p.tokens * D;
  const T *Vt = static_cast<const T *>(p.v) + (int64_t)bg * p.tokens * D;
  T *DK = static_cast<T *>(p.dk) + (int64_t)bg * p.tokens * D;
  T *DV = static_cast<T *>(p.dv) + (int64_t)bg * p.tokens * D;
  const int f_begin = m * p.pool_size, f_end = min(p.fine_blocks, (m + 1) * p.pool_size);
  int idx[2];
  if (has) stage_block<T, D>(S, K, Vt, p.blocks, f_begin, V, idx);
  // the summary's gradient rows and its block-table entries load while the rows gather
  constexpr int kCh = (D + 31) / 32;
  const int64_t srow = ((int64_t)bg * M + m) * D;
  float gk[kCh], gv[kCh];
#pragma unroll
  for (int i = 0; i < kCh; ++i) {
    const int ch = lane + 32 * i;
    gk[i] = has && ch < D ? p.dsk[srow + ch] : 0.f;
    gv[i] = has && ch < D ? p.dsv[srow + ch] : 0.f;
  }
  int count = 0;  // nonempty fine blocks: the coarse mean's divisor
  for (int f = f_begin; has && f < f_end; ++f) {
    const bool any = (lane < V && p.blocks[(int64_t)f * V + lane] >= 0) ||
                     (lane + 32 < V && p.blocks[(int64_t)f * V + lane + 32] >= 0);
    count += __any_sync(0xffffffffu, any) ? 1 : 0;
  }
  float *w = reinterpret_cast<float *>(stage_smem);
  float *bias = w + D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) w[i] = p.weight[i];
  for (int i = threadIdx.x; i < V; i += blockDim.x) bias[i] = p.bias[i];
  __syncthreads();
  if (!has) return;
  const float inv_temp = 1.f / p.temperature;
  const int grp = lane / G::kChunks, chunk = lane - grp * G::kChunks;
  const bool mapped = grp < G::kGroups;
  const float inv_count = 1.f / (float)count;
#pragma unroll
  for (int i = 0; i < kCh; ++i) {
    const int ch = lane + 32 * i;
    if (ch < D) {
      S.grad[ch] = gk[i] * inv_count;
      S.grad[D + ch] = gv[i] * inv_count;
    }
  }
  float2 dw[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) dw[i] = make_float2(0.f, 0.f);
  float db[2] = {0.f, 0.f};
  for (int f = f_begin; f < f_end; ++f) {
    if (f != f_begin) stage_block<T, D>(S, K, Vt, p.blocks, f, V, idx);
    cp_async_wait<1>();
    __syncwarp();  // (also publishes grad)
    const FineWeights fw = staged_weights<T, D>(S, idx, w, bias, inv_temp);
    cp_async_wait<0>();
    __syncwarp();
    if (fw.nonempty) {
      // da_s = member_k . dfine_k + member_v . dfine_v; ds = a * (da - sum a*da)
      const int r0 = idx[0] >= 0 ? lane : 0, r1 = idx[1] >= 0 ? lane + 32 : 0;  // empty: row 0, discarded
      const float2 dk = staged_dot2<T, D>(S.k + r0 * G::kStride, S.k + r1 * G::kStride, S.grad);
      const float2 dv = staged_dot2<T, D>(S.v + r0 * G::kChunks, S.v + r1 * G::kChunks, S.grad + D);
      const float da[2] = {idx[0] >= 0 ? dk.x + dv.x : 0.f, idx[1] >= 0 ? dk.y + dv.y : 0.f};
      const float mean = warp_sum(fw.a[0] * da[0] + fw.a[1] * da[1]);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float ds = fw.a[j] * (da[j] - mean);
        db[j] += ds;
        S.a[lane + 32 * j] = fw.a[j];
        S.ds[lane + 32 * j] = ds;
      }
      const uint64_t valid = valid_slots(idx);
      __syncwarp();
      // dK / dV member rows: lane per (row, 16-byte chunk), one 16-byte store each.
#pragma unroll 2
      for (int i = 0; i < (64 * G::kChunks + 31) / 32; ++i) {
        const int e = lane + 32 * i, r = e / G::kChunks, c = e - r * G::kChunks;
        if (e >= V * G::kChunks) break;  // e grows with i
        const int row = S.idx[r];
        if (row < 0) continue;
        const float a = S.a[r], dsv = S.ds[r];
        float gk[8], gv[8], wc[8];  // this chunk's 8 channels of dfine_k, dfine_v, w
        *reinterpret_cast<float4 *>(gk) = *reinterpret_cast<const float4 *>(S.grad + 8 * c);
        *reinterpret_cast<float4 *>(gk + 4) = *reinterpret_cast<const float4 *>(S.grad + 8 * c + 4);
        *reinterpret_cast<float4 *>(gv) = *reinterpret_cast<const float4 *>(S.grad + D + 8 * c);
        *reinterpret_cast<float4 *>(gv + 4) = *reinterpret_cast<const float4 *>(S.grad + D + 8 * c + 4);
        *reinterpret_cast<float4 *>(wc) = *reinterpret_cast<const float4 *>(w + 8 * c);
        *reinterpret_cast<float4 *>(wc + 4) = *reinterpret_cast<const float4 *>(w + 8 * c + 4);
        uint32_t pk[4], pv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pk[i] = pack2<T>(fmaf(a, gk[2 * i], dsv * (wc[2 * i] * inv_temp)),
                           fmaf(a, gk[2 * i + 1], dsv * (wc[2 * i + 1] * inv_temp)));
          pv[i] = pack2<T>(a * gv[2 * i], a * gv[2 * i + 1]);
        }
        *reinterpret_cast<uint4 *>(DK + (int64_t)row * D + 8 * c) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4 *>(DV + (int64_t)row * D + 8 * c) = make_uint4(pv[0], pv[1], pv[2], pv[3]);
      }
      // dweight partial: dw[ch] += ds_s * k_s[ch] / T, (slot group, chunk) lanes.
      if (mapped) {
        const float2 it2 = make_float2(inv_temp, inv_temp);
#pragma unroll 4
        for (int it = 0; it < G::kSlotIters; ++it) {
          const int s = grp + G::kGroups * it;
          if (s < V && ((valid >> s) & 1)) {
            const float2 dsv = make_float2(S.ds[s], S.ds[s]);
            const uint4 raw = S.k[s * G::kStride + chunk];
            const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) dw[i] = fma2(dsv, mul2(unpack2<T>(u[i]), it2), dw[i]);
          }
        }
      }
    }
    __syncwarp();  // the next fine block (or the scratch) overwrites the rows
  }
  park8(S.scratch, 0, dw);
  __syncwarp();
  const int64_t prow = (int64_t)bg * M + m;
  for (int o = lane; o < D; o += 32) p.dw_part[prow * D + o] = sum_groups<D>(S.scratch, o, 0);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int s = lane + 32 * j;
    if (s < V) p.db_part[prow * V + s] = db[j];
  }
}

}  // namespace

static bool aligned(const void *p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

template <typename T, int D>
static int pool_fwd_staged(const PoolArgs &p, cudaStream_t stream) {
  const unsigned blocks = (unsigned)(((int64_t)p.summaries * p.bg + kStageWarps - 1) / kStageWarps);
  static size_t seen[kMaxDevices] = {};
  const size_t bytes = Staging<D>::kHead + kStageWarps * Staging<D>::per_warp(p.slots, false);
  if (int st = smem_optin(pool_fwd_staged_kernel<T, D>, bytes, seen)) return st;
  pool_fwd_staged_kernel<T, D><<<blocks, kStageWarps * 32, bytes, stream>>>(p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

template <typename T, int D>
static int pool_bwd_staged(const PoolBwdArgs &p, cudaStream_t stream) {
  const unsigned blocks = (unsigned)(((int64_t)p.summaries * p.bg + kStageWarps - 1) / kStageWarps);
  static size_t seen[kMaxDevices] = {};
  const size_t bytes = Staging<D>::kHead + kStageWarps * Staging<D>::per_warp(p.slots, true);
  if (int st = smem_optin(pool_bwd_staged_kernel<T, D>, bytes, seen)) return st;
  pool_bwd_staged_kernel<T, D><<<blocks, kStageWarps * 32, bytes, stream>>>(p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

template <typename T>
static int launch_pool_fwd_t(const PoolArgs &p, cudaStream_t stream) {
  const int warps = p.summaries * p.bg;
  const int blocks = (warps + kWarps - 1) / kWarps;
  if constexpr (sizeof(T) == 2) {
    if (p.vec) {
      switch (p.head_dim) {
        case 8: return pool_fwd_staged<T, 8>(p, stream);
        case 16: return pool_fwd_staged<T, 16>(p, stream);
        case 32: return pool_fwd_staged<T, 32>(p, stream);
        case 48: return pool_fwd_staged<T, 48>(p, stream);
        case 64: return pool_fwd_staged<T, 64>(p, stream);
        case 128: return pool_fwd_staged<T, 128>(p, stream);
        default: break;
      }
    }
  }
  const size_t smem = sizeof(float) * (p.head_dim + p.slots);
  pool_fwd_kernel<T><<<blocks, kWarps * 32, smem, stream>>>(p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_pool_fwd(const PoolArgs &p, cudaStream_t stream) {
  if ((int64_t)p.summaries * p.bg == 0) return P3D_OK;
  switch (p.dtype) {
    case P3D_F16: return launch_pool_fwd_t<__half>(p, stream);
    case P3D_BF16: return launch_pool_fwd_t<__nv_bfloat16>(p, stream);
    default: return launch_pool_fwd_t<float>(p, stream);
  }
}

template <typename T>
static int launch_pool_bwd_t(const PoolBwdArgs &p, cudaStream_t stream) {
  const int warps = p.summaries * p.bg;
  const int blocks = (warps + kWarps - 1) / kWarps;
  if constexpr (sizeof(T) == 2) {
    if (p.vec && aligned(p.dk, 16) && aligned(p.dv, 16)) {
      switch (p.head_dim) {
        case 8: return pool_bwd_staged<T, 8>(p, stream);
        case 16: return pool_bwd_staged<T, 16>(p, stream);
        case 32: return pool_bwd_staged<T, 32>(p, stream);
        case 48: return pool_bwd_staged<T, 48>(p, stream);
        case 64: return pool_bwd_staged<T, 64>(p, stream);
        case 128: return pool_bwd_staged<T, 128>(p, stream);
        default: break;
      }
    }
  }
  const size_t smem = sizeof(float) * (p.head_dim + p.slots + kWarps * 2 * p.head_dim);
  pool_bwd_kernel<T><<<blocks, kWarps * 32, smem, stream>>>(p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_pool_bwd(const PoolBwdArgs &p, cudaStream_t stream) {
  if ((int64_t)p.summaries * p.bg == 0) return P3D_OK;
  switch (p.dtype) {
    case P3D_F16: return launch_pool_bwd_t<__half>(p, stream);
    case P3D_BF16: return launch_pool_bwd_t<__nv_bfloat16>(p, stream);
    default: return launch_pool_bwd_t<float>(p, stream);
  }
}

}  // namespace p3d
