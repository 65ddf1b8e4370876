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

namespace p3d {
namespace {

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

}  // namespace

template <typename T>
static int launch_pool_fwd_t(const PoolArgs &p, cudaStream_t stream) {
  const int warps = p.summaries * p.bg;
  const int blocks = (warps + kWarps - 1) / kWarps;
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
