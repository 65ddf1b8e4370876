// Layer glue of the PACK3D attention layer on the inference path (attention.py:53-89):
//
//   p3d_layer_norm  LayerNorm over the channel dimension (nn.LayerNorm, attention.py:64):
//                   one warp per token row, fp32 mean / variance, 16-byte accesses.
//   p3d_qkv_split   the projection split of attention.py:70-81 in one pass: reads the
//                   row-major to_q / to_kv outputs [B, N, H*D] and [B, N, 4*G*D] (to_kv's
//                   channel blocks are kl, vl, kg, vg) and writes the five head-major
//                   tensors [B, H|G, N, D]; q, kl and kg are rotated by the axial RoPE
//                   phase table exactly as p3d_rope does (rotary.py:11-45), vl and vg
//                   copied.  Replaces three rotations and two strided copies.
//   p3d_qkv_merge   its backward (rotary.py:66-70 inverse rotation, then the transposes and
//                   the chunk concatenation autograd would do): the five head-major
//                   gradients -> the row-major to_q / to_kv output gradients, dq / dkl / dkg
//                   rotated back by the same table (sine negated, products rounded as in
//                   p3d_rope's inverse), so the result equals rotation + copies bit for bit.
//   p3d_layer_norm_bwd  LayerNorm backward: dx per row (mean / rstd recomputed as in the
//                   forward), fp32 per-warp partials of dweight / dbias reduced in fixed order.
// All are HBM bound: one read and one write of every byte.
#include "common.cuh"
#include "kernels.cuh"

namespace p3d {
namespace {

constexpr int kWarps = 8;

template <typename T>
__device__ __forceinline__ void load8(const T *src, float (&v)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4 *>(src);
  const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = to_f32<T>(e[i]);
}

template <typename T>
__device__ __forceinline__ void store8(T *dst, const float (&v)[8]) {
  uint4 raw;
  T *e = reinterpret_cast<T *>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(v[i]);
  *reinterpret_cast<uint4 *>(dst) = raw;
}

// o = round(o) + r in fp32: the LayerNorm input gradient rounded to the storage type, then the
// residual branch's gradient added as a separate elementwise add of two T tensors would (the
// caller's store rounds the sum), so the fused form is bit-identical to the two-step one.
template <typename T>
__device__ __forceinline__ void add_rounded8(float (&o)[8], const float (&r)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = to_f32<T>(from_f32<T>(o[i])) + r[i];
}

// ---------------------------------------------------------------------------- LayerNorm
template <typename T, int kChunks>
__global__ void __launch_bounds__(kWarps * 32)
    layer_norm_kernel(const T *x, const T *weight, const T *bias, T *y, int64_t rows, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T *xr = x + row * dim;
  float v[kChunks][8];
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (c < dim) {
      load8<T>(xr + c, v[k]);
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += v[k][i];
    }
  }
  const float mean = warp_sum(sum) / (float)dim;
  float sq = 0.f;
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (c < dim) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[k][i] - mean;
        sq += d * d;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(sq) / (float)dim + eps);
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (c < dim) {
      float w[8], b[8], o[8];
      load8<T>(weight + c, w);
      load8<T>(bias + c, b);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[k][i] - mean) * rstd * w[i] + b[i];
      store8<T>(y + row * dim + c, o);
    }
  }
}

// LayerNorm backward: each warp walks rows with a grid stride; per row, with mean / rstd
// recomputed exactly as the forward computes them,
//   xhat = (x - mean) rstd,  g = dy w,  dx = rstd (g - mean(g) - xhat mean(g xhat)),
// and the warp's fp32 partials of dweight = sum dy xhat, dbias = sum dy are written per warp
// (reduced afterwards in fixed order: bitwise-repeatable).
constexpr int kLnBwdBlocks = 1024;  // at most 8192 warps: the partials' row count

template <typename T, int kChunks, bool kRes>
__global__ void __launch_bounds__(kWarps * 32)
    layer_norm_bwd_kernel(const T *x, const T *weight, const T *dy, const T *dres, T *dx, float *dw_part,
                          float *db_part, int64_t rows, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_id = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t n_warps = (int64_t)gridDim.x * kWarps;
  float w[kChunks][8], accw[kChunks][8], accb[kChunks][8];
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const int c = (lane + 32 * k) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) accw[k][i] = accb[k][i] = w[k][i] = 0.f;
    if (c < dim) load8<T>(weight + c, w[k]);
  }
  const float inv_dim = 1.f / (float)dim;
  for (int64_t row = warp_id; row < rows; row += n_warps) {
    float v[kChunks][8], g[kChunks][8];
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      const int c = (lane + 32 * k) * 8;
      if (c < dim) {
        load8<T>(x + row * dim + c, v[k]);
        load8<T>(dy + row * dim + c, g[k]);
#pragma unroll
        for (int i = 0; i < 8; ++i) sum += v[k][i];
      }
    }
    const float mean = warp_sum(sum) / (float)dim;
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      const int c = (lane + 32 * k) * 8;
      if (c < dim) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float d = v[k][i] - mean;
          sq += d * d;
        }
      }
    }
    const float rstd = rsqrtf(warp_sum(sq) / (float)dim + eps);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      const int c = (lane + 32 * k) * 8;
      if (c < dim) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xhat = (v[k][i] - mean) * rstd;
          const float gw = g[k][i] * w[k][i];
          s1 += gw;
          s2 += gw * xhat;
          accw[k][i] += g[k][i] * xhat;
          accb[k][i] += g[k][i];
          v[k][i] = xhat;
          g[k][i] = gw;
        }
      }
    }
    const float m1 = warp_sum(s1) * inv_dim, m2 = warp_sum(s2) * inv_dim;
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      const int c = (lane + 32 * k) * 8;
      if (c < dim) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = rstd * (g[k][i] - m1 - v[k][i] * m2);
        if constexpr (kRes) {
          float r[8];
          load8<T>(dres + row * dim + c, r);
          add_rounded8<T>(o, r);
        }
        store8<T>(dx + row * dim + c, o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (c < dim) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dw_part[warp_id * dim + c + i] = accw[k][i];
        db_part[warp_id * dim + c + i] = accb[k][i];
      }
    }
  }
}

// ------------------------------------------------------- LayerNorm, segment layout
// For dim = 64 K (K <= 4): a row is a segment of 8 lanes, lane l of the segment holding the
// row's 16-byte chunks l + 8 j (j < K), so each j reads one 128-byte line per row; a warp pass
// covers 4 rows.  Row sums reduce inside the segment (3 xor shuffles instead of 5 across the
// warp), all 32 lanes work for any such dim, and in the forward the next row group's loads
// (a grid-stride walk) are issued before the current one is reduced.
// Same per-element arithmetic as the kernels above; the row sums add in a different order.
template <int S>
__device__ __forceinline__ float seg_sum(float v) {
#pragma unroll
  for (int o = 1; o < S; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ void unpack8x(const uint4 &raw, float (&v)[8]) {
  const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack2<T>(u[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T, int K>
__global__ void __launch_bounds__(kWarps * 32, 3)
    layer_norm_seg_kernel(const T *x, const T *weight, const T *bias, T *y, int64_t rows, float eps) {
  constexpr int D = 64 * K;
  const int lane = threadIdx.x & 31, seg = lane >> 3, l = lane & 7;
  const int64_t n_warps = (int64_t)gridDim.x * kWarps;
  auto load_group = [&](int64_t g, uint4 (&raw)[K]) {
    const int64_t row = 4 * g + seg;
#pragma unroll
    for (int j = 0; j < K; ++j)
      raw[j] = row < rows ? *reinterpret_cast<const uint4 *>(x + row * D + 8 * (l + 8 * j)) : make_uint4(0u, 0u, 0u, 0u);
  };
  int64_t g = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  uint4 raw[K];
  load_group(g, raw);
  for (; 4 * g < rows; g += n_warps) {
    float v[K][8];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      unpack8x<T>(raw[j], v[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += v[j][i];
    }
    load_group(g + n_warps, raw);  // the next row group is in flight during this one's math
    const float mean = seg_sum<8>(sum) / (float)D;
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[j][i] - mean;
        sq += d * d;
      }
    const float rstd = rsqrtf(seg_sum<8>(sq) / (float)D + eps);
    const int64_t row = 4 * g + seg;
    if (row < rows) {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        float w[8], b[8], o[8];
        load8<T>(weight + 8 * (l + 8 * j), w);  // L1-resident after the first row group
        load8<T>(bias + 8 * (l + 8 * j), b);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = (v[j][i] - mean) * rstd * w[i] + b[i];
        store8<T>(y + row * D + 8 * (l + 8 * j), o);
      }
    }
  }
}

template <typename T, int K, bool kRes>
__global__ void __launch_bounds__(kWarps * 32, 2)
    layer_norm_bwd_seg_kernel(const T *x, const T *weight, const T *dy, const T *dres, T *dx, float *dw_part,
                              float *db_part, int64_t rows, float eps) {
  constexpr int D = 64 * K;
  const int lane = threadIdx.x & 31, seg = lane >> 3, l = lane & 7;
  const int64_t warp_id = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t n_warps = (int64_t)gridDim.x * kWarps;
  float accw[K][8], accb[K][8];
#pragma unroll
  for (int j = 0; j < K; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) accw[j][i] = accb[j][i] = 0.f;
  const float inv_dim = 1.f / (float)D;
  for (int64_t g = warp_id; 4 * g < rows; g += n_warps) {
    const int64_t row = 4 * g + seg;
    const bool on = row < rows;
    uint4 rx[K], rg[K], rr[kRes ? K : 1];
#pragma unroll
    for (int j = 0; j < K; ++j) {
      rx[j] = rg[j] = make_uint4(0u, 0u, 0u, 0u);
      if (on) {
        rx[j] = *reinterpret_cast<const uint4 *>(x + row * D + 8 * (l + 8 * j));
        rg[j] = *reinterpret_cast<const uint4 *>(dy + row * D + 8 * (l + 8 * j));
        if constexpr (kRes) rr[j] = *reinterpret_cast<const uint4 *>(dres + row * D + 8 * (l + 8 * j));
      }
    }
    float v[K][8], gr[K][8];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      unpack8x<T>(rx[j], v[j]);
      unpack8x<T>(rg[j], gr[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += v[j][i];
    }
    const float mean = seg_sum<8>(sum) / (float)D;
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[j][i] - mean;
        sq += d * d;
      }
    const float rstd = rsqrtf(seg_sum<8>(sq) / (float)D + eps);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      float w[8];
      load8<T>(weight + 8 * (l + 8 * j), w);  // L1-resident after the first row group
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xhat = (v[j][i] - mean) * rstd;
        const float gw = gr[j][i] * w[i];
        s1 += gw;
        s2 += gw * xhat;
        accw[j][i] += gr[j][i] * xhat;  // rows outside the tensor load zeros: no contribution
        accb[j][i] += gr[j][i];
        v[j][i] = xhat;
        gr[j][i] = gw;
      }
    }
    const float m1 = seg_sum<8>(s1) * inv_dim, m2 = seg_sum<8>(s2) * inv_dim;
    if (on) {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = rstd * (gr[j][i] - m1 - v[j][i] * m2);
        if constexpr (kRes) {
          float r[8];
          unpack8x<T>(rr[j], r);
          add_rounded8<T>(o, r);
        }
        store8<T>(dx + row * D + 8 * (l + 8 * j), o);
      }
    }
  }
  // the four segments' partials of each channel, then segment 0 writes the warp's row
#pragma unroll
  for (int j = 0; j < K; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      accw[j][i] += __shfl_xor_sync(0xffffffffu, accw[j][i], 8);
      accw[j][i] += __shfl_xor_sync(0xffffffffu, accw[j][i], 16);
      accb[j][i] += __shfl_xor_sync(0xffffffffu, accb[j][i], 8);
      accb[j][i] += __shfl_xor_sync(0xffffffffu, accb[j][i], 16);
    }
  if (seg == 0) {
#pragma unroll
    for (int j = 0; j < K; ++j) {
      float *pw = dw_part + warp_id * D + 8 * (l + 8 * j), *pb = db_part + warp_id * D + 8 * (l + 8 * j);
      *reinterpret_cast<float4 *>(pw) = make_float4(accw[j][0], accw[j][1], accw[j][2], accw[j][3]);
      *reinterpret_cast<float4 *>(pw + 4) = make_float4(accw[j][4], accw[j][5], accw[j][6], accw[j][7]);
      *reinterpret_cast<float4 *>(pb) = make_float4(accb[j][0], accb[j][1], accb[j][2], accb[j][3]);
      *reinterpret_cast<float4 *>(pb + 4) = make_float4(accb[j][4], accb[j][5], accb[j][6], accb[j][7]);
    }
  }
}

// ---------------------------------------------------------------------- projection split
struct SplitParams {
  const void *qp, *kvp;
  void *out[5];  // q, kl, vl, kg, vg
  int batch, heads, kv_heads, tokens;
  const int64_t *coords;  // [N, 3]
  int pairs[3];
  int start[3];           // first phase-table entry of each axis
  const float *phases;    // (cos, sin) per (axis, coordinate, pair)
  int raster_qkv;         // split: q, kl, vl rows at the token's raster index (ey x ex planes)
  int ey, ex;
  int q_stride, kv_stride;  // elements between consecutive tokens' rows of qp / kvp
  const void *gate_logits;  // split only, or null: [token][head][2] logits at gate_stride per token
  int gate_stride;
  void *gate;               // [B, H, N]: softmax over each logit pair, second entry
};

constexpr int kTokensPerWarp = 4;
constexpr int kGateRounds = 2;  // lanes x rounds cover the (token, head) gates of a warp: heads <= 16

template <typename T>
__device__ __forceinline__ T *pick(const SplitParams &p, int part) {  // out[1 + part] without a local array
  void *o = part == 0 ? p.out[1] : part == 1 ? p.out[2] : part == 2 ? p.out[3] : p.out[4];
  return static_cast<T *>(o);
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &raw, float (&v)[8]) {
  const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack2<T>(u[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// (cos, sin) of rotation pair `pair` at the token's coordinates: pairs [0, pairs[0]) turn
// with z, the next pairs[1] with y, the rest with x.  Selects, not indexing: keeps c and p
// in registers.
__device__ __forceinline__ float2 pair_phase(const SplitParams &p, const int64_t (&c)[3], int pair) {
  int64_t entry;
  if (pair < p.pairs[0]) {
    entry = p.start[0] + c[0] * p.pairs[0] + pair;
  } else if (pair < p.pairs[0] + p.pairs[1]) {
    entry = p.start[1] + c[1] * p.pairs[1] + (pair - p.pairs[0]);
  } else {
    entry = p.start[2] + c[2] * p.pairs[2] + (pair - p.pairs[0] - p.pairs[1]);
  }
  return *reinterpret_cast<const float2 *>(p.phases + 2 * entry);
}

// One pass over a token's head rows (q heads, then the kl, vl, kg, vg heads): MERGE = false
// is the split (row-major projections -> head-major, q / kl / kg rotated), MERGE = true its
// backward (head-major gradients -> row-major projection gradients, rotated back).  Lane =
// row * C + chunk for C = D / 8 chunks per head row and 32 / C rows per warp pass, so a
// lane always holds the same 4 pairs of a head row: it reads their (cos, sin) once per token
// and every rotation is lane-local.  kBatch passes of loads are issued before the first
// rotation.  Each product and sum is rounded separately, as the reference's elementwise torch
// arithmetic (rotary.py).
template <typename T, int D, bool MERGE>
__global__ void __launch_bounds__(kWarps * 32, 4) qkv_pass_kernel(SplitParams p) {
  constexpr int C = D / 8;       // 16-byte chunks per head row
  constexpr int kRows = 32 / C;  // head rows per warp pass
  constexpr int kBatch = 4;      // passes loaded ahead of the rotations
  const int lane = threadIdx.x & 31;
  const int sub = lane / C, grp = lane - sub * C;
  const bool on = sub < kRows;
  const int b = blockIdx.y;
  const int n_begin = (blockIdx.x * kWarps + (threadIdx.x >> 5)) * kTokensPerWarp;
  const int rows = p.heads + 4 * p.kv_heads;  // head rows per token
  const int qw = p.q_stride, kvw = p.kv_stride;  // elements between projection rows
  T *qrow_w = static_cast<T *>(const_cast<void *>(p.qp)), *kvrow_w = static_cast<T *>(const_cast<void *>(p.kvp));
  // the gate logit pairs of this warp's tokens (split with a gate only), loaded first so that
  // their latency overlaps the head rows
  uint32_t gate_pair[kGateRounds] = {};
  if (!MERGE && p.gate_logits != nullptr) {
#pragma unroll
    for (int r = 0; r < kGateRounds; ++r) {
      const int k = lane + 32 * r, t = k / p.heads, h = k - t * p.heads, n = n_begin + t;
      if (k < kTokensPerWarp * p.heads && n < p.tokens)
        gate_pair[r] = __ldg(reinterpret_cast<const uint32_t *>(static_cast<const T *>(p.gate_logits) +
                                                                ((int64_t)b * p.tokens + n) * p.gate_stride + 2 * h));
    }
  }
  for (int base = 0; base < rows; base += kRows * kBatch) {
    // token-independent: each pass's head row, its head-major tensor row of token 0, its
    // offset in the projection rows, whether it rotates
    T *head[kBatch];
    int off[kBatch];
    bool isq[kBatch], rot[kBatch], act[kBatch], to_raster[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int hr = base + i * kRows + sub;
      act[i] = on && hr < rows;
      const int r = act[i] ? hr : 0;
      isq[i] = r < p.heads;
      if (isq[i]) {
        head[i] = static_cast<T *>(p.out[0]) + ((int64_t)b * p.heads + r) * p.tokens * D + 8 * grp;
        off[i] = r * D + 8 * grp;
        rot[i] = true;
        to_raster[i] = true;
      } else {
        const int x = r - p.heads, part = x / p.kv_heads, g = x - part * p.kv_heads;  // 0 kl, 1 vl, 2 kg, 3 vg
        head[i] = pick<T>(p, part) + ((int64_t)b * p.kv_heads + g) * p.tokens * D + 8 * grp;
        off[i] = x * D + 8 * grp;
        rot[i] = (part & 1) == 0;
        to_raster[i] = part <= 1;  // kl, vl (kg, vg stay in token order for the pooling)
      }
    }
    for (int t = 0; t < kTokensPerWarp; ++t) {
      const int n = n_begin + t;
      if (n >= p.tokens) break;  // warp-uniform
      T *qrow = qrow_w + ((int64_t)b * p.tokens + n) * qw;
      T *kvrow = kvrow_w + ((int64_t)b * p.tokens + n) * kvw;
      uint4 raw[kBatch];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        raw[i] = make_uint4(0u, 0u, 0u, 0u);
        if (act[i])
          raw[i] = *reinterpret_cast<const uint4 *>(MERGE ? head[i] + (int64_t)n * D : (isq[i] ? qrow : kvrow) + off[i]);
      }
      const int64_t c[3] = {p.coords[3 * (int64_t)n], p.coords[3 * (int64_t)n + 1], p.coords[3 * (int64_t)n + 2]};
      // destination row of q, kl, vl: the token's row, or its raster index for the raster form
      const int64_t nr = (!MERGE && p.raster_qkv) ? (c[0] * p.ey + c[1]) * p.ex + c[2] : n;
      float2 cs[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        cs[j] = pair_phase(p, c, 4 * grp + j);
        if (MERGE) cs[j].y = -cs[j].y;  // the inverse rotation: sine negated
      }
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        if (!act[i]) continue;
        float v[8];
        unpack8<T>(raw[i], v);
        if (rot[i]) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float even = v[2 * j], odd = v[2 * j + 1];
            v[2 * j] = __fsub_rn(__fmul_rn(even, cs[j].x), __fmul_rn(odd, cs[j].y));
            v[2 * j + 1] = __fadd_rn(__fmul_rn(even, cs[j].y), __fmul_rn(odd, cs[j].x));
          }
        }
        store8<T>(MERGE ? (isq[i] ? qrow : kvrow) + off[i] : head[i] + (to_raster[i] ? nr : (int64_t)n) * D, v);
      }
    }
  }
  if (!MERGE && p.gate_logits != nullptr) {
    // the gate of the reference layer (attention.py:84-86): softmax over each head's logit pair,
    // second entry, in fp32 (expf, then a division) and rounded to the storage type once; a
    // lane per (token, head), its pair loaded before the head rows (gate_pair)
    T *gate = static_cast<T *>(p.gate);
#pragma unroll
    for (int r = 0; r < kGateRounds; ++r) {
      const int k = lane + 32 * r, t = k / p.heads, h = k - t * p.heads, n = n_begin + t;
      if (k >= kTokensPerWarp * p.heads || n >= p.tokens) continue;
      const float2 l = unpack2<T>(gate_pair[r]);
      const float m = fmaxf(l.x, l.y);
      const float e0 = expf(l.x - m), e1 = expf(l.y - m);
      gate[((int64_t)b * p.heads + h) * p.tokens + n] = from_f32<T>(e1 / (e0 + e1));
    }
  }
}

template <typename T>
int launch_merge(const SplitParams &p, int head_dim, cudaStream_t s) {
  const dim3 grid((unsigned)((p.tokens + kWarps * kTokensPerWarp - 1) / (kWarps * kTokensPerWarp)),
                  (unsigned)p.batch);
  switch (head_dim) {
    case 16: qkv_pass_kernel<T, 16, true><<<grid, kWarps * 32, 0, s>>>(p); break;
    case 32: qkv_pass_kernel<T, 32, true><<<grid, kWarps * 32, 0, s>>>(p); break;
    case 48: qkv_pass_kernel<T, 48, true><<<grid, kWarps * 32, 0, s>>>(p); break;
    case 64: qkv_pass_kernel<T, 64, true><<<grid, kWarps * 32, 0, s>>>(p); break;
    case 128: qkv_pass_kernel<T, 128, true><<<grid, kWarps * 32, 0, s>>>(p); break;
    default: return fail(P3D_ERR_UNSUPPORTED, "p3d_qkv_merge: head_dim %d", head_dim);
  }
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

template <typename T>
int launch_split(const SplitParams &p, int head_dim, cudaStream_t s) {
  const dim3 grid((unsigned)((p.tokens + kWarps * kTokensPerWarp - 1) / (kWarps * kTokensPerWarp)),
                  (unsigned)p.batch);
  switch (head_dim) {
    case 16: qkv_pass_kernel<T, 16, false><<<grid, kWarps * 32, 0, s>>>(p); break;
    case 32: qkv_pass_kernel<T, 32, false><<<grid, kWarps * 32, 0, s>>>(p); break;
    case 48: qkv_pass_kernel<T, 48, false><<<grid, kWarps * 32, 0, s>>>(p); break;
    case 64: qkv_pass_kernel<T, 64, false><<<grid, kWarps * 32, 0, s>>>(p); break;
    case 128: qkv_pass_kernel<T, 128, false><<<grid, kWarps * 32, 0, s>>>(p); break;
    default: return fail(P3D_ERR_UNSUPPORTED, "p3d_qkv_split: head_dim %d", head_dim);
  }
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

template <typename T>
int launch_ln(const void *x, const void *w, const void *b, void *y, int64_t rows, int dim, float eps,
              cudaStream_t s) {
  if (dim % 64 == 0 && dim <= 256) {  // segment layout: 4 rows per warp pass, grid-stride
    DeviceInfo info{};
    if (int st = device_info(&info)) return st;
    const int64_t want = (rows + 4 * kWarps - 1) / (4 * kWarps), cap = (int64_t)info.sm_count * 3;
    const unsigned blocks = (unsigned)(want < cap ? want : cap);
    auto seg = [&](auto kernel) {
      kernel<<<blocks, kWarps * 32, 0, s>>>(static_cast<const T *>(x), static_cast<const T *>(w),
                                            static_cast<const T *>(b), static_cast<T *>(y), rows, eps);
    };
    switch (dim / 64) {
      case 1: seg(layer_norm_seg_kernel<T, 1>); break;
      case 2: seg(layer_norm_seg_kernel<T, 2>); break;
      case 3: seg(layer_norm_seg_kernel<T, 3>); break;
      default: seg(layer_norm_seg_kernel<T, 4>); break;
    }
    P3D_LAUNCH_CHECK();
    return P3D_OK;
  }
  const unsigned blocks = (unsigned)((rows + kWarps - 1) / kWarps);
  const int chunks = (dim / 8 + 31) / 32;
  auto args = [&](auto kernel) {
    kernel<<<blocks, kWarps * 32, 0, s>>>(static_cast<const T *>(x), static_cast<const T *>(w),
                                          static_cast<const T *>(b), static_cast<T *>(y), rows, dim, eps);
  };
  switch (chunks) {
    case 1: args(layer_norm_kernel<T, 1>); break;
    case 2: args(layer_norm_kernel<T, 2>); break;
    case 3: args(layer_norm_kernel<T, 3>); break;
    case 4: args(layer_norm_kernel<T, 4>); break;
    default: return fail(P3D_ERR_UNSUPPORTED, "p3d_layer_norm: dim %d above 1024", dim);
  }
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

template <typename T, bool kRes>
int launch_ln_bwd(const void *x, const void *w, const void *dy, const void *dres, void *dx, float *dw_part,
                  float *db_part, int64_t rows, int dim, float eps, unsigned blocks, cudaStream_t s) {
  if (dim % 64 == 0 && dim <= 192) {  // segment layout (same grid: one partials row per warp)
    auto seg = [&](auto kernel) {
      kernel<<<blocks, kWarps * 32, 0, s>>>(static_cast<const T *>(x), static_cast<const T *>(w),
                                            static_cast<const T *>(dy), static_cast<const T *>(dres),
                                            static_cast<T *>(dx), dw_part, db_part, rows, eps);
    };
    switch (dim / 64) {
      case 1: seg(layer_norm_bwd_seg_kernel<T, 1, kRes>); break;
      case 2: seg(layer_norm_bwd_seg_kernel<T, 2, kRes>); break;
      default: seg(layer_norm_bwd_seg_kernel<T, 3, kRes>); break;
    }
    P3D_LAUNCH_CHECK();
    return P3D_OK;
  }
  const int chunks = (dim / 8 + 31) / 32;
  auto args = [&](auto kernel) {
    kernel<<<blocks, kWarps * 32, 0, s>>>(static_cast<const T *>(x), static_cast<const T *>(w),
                                          static_cast<const T *>(dy), static_cast<const T *>(dres),
                                          static_cast<T *>(dx), dw_part, db_part, rows, dim, eps);
  };
  switch (chunks) {
    case 1: args(layer_norm_bwd_kernel<T, 1, kRes>); break;
    case 2: args(layer_norm_bwd_kernel<T, 2, kRes>); break;
    case 3: args(layer_norm_bwd_kernel<T, 3, kRes>); break;
    case 4: args(layer_norm_bwd_kernel<T, 4, kRes>); break;
    default: return fail(P3D_ERR_UNSUPPORTED, "p3d_layer_norm_bwd: dim %d above 1024", dim);
  }
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

template <typename T>
int launch_ln_bwd_any(const void *x, const void *w, const void *dy, const void *dres, void *dx, float *dw_part,
                      float *db_part, int64_t rows, int dim, float eps, unsigned blocks, cudaStream_t s) {
  return dres ? launch_ln_bwd<T, true>(x, w, dy, dres, dx, dw_part, db_part, rows, dim, eps, blocks, s)
              : launch_ln_bwd<T, false>(x, w, dy, dres, dx, dw_part, db_part, rows, dim, eps, blocks, s);
}

unsigned ln_bwd_blocks(int64_t rows) {
  const int64_t b = (rows + kWarps - 1) / kWarps;
  return (unsigned)(b < kLnBwdBlocks ? (b > 0 ? b : 1) : kLnBwdBlocks);
}

// workspace: dweight / dbias partials [warps, dim] each, then the row-sum scratch
size_t ln_bwd_layout(int64_t rows, int dim, void *base, float **dw_part, float **db_part, float **tmp) {
  const int64_t warps = (int64_t)ln_bwd_blocks(rows) * kWarps;
  const size_t part = (size_t)warps * dim * sizeof(float);
  char *p = static_cast<char *>(base);
  *dw_part = reinterpret_cast<float *>(p);
  *db_part = reinterpret_cast<float *>(p + part);
  *tmp = reinterpret_cast<float *>(p + 2 * part);
  return 2 * part + (size_t)sum_rows_tmp(warps, dim) * sizeof(float);
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" int p3d_layer_norm(const void *x, const void *weight, const void *bias, void *y, int dtype, int64_t rows,
                              int dim, float eps, void *stream) {
  P3D_CHECK_ARG(dtype == P3D_BF16 || dtype == P3D_F16, "p3d_layer_norm: bf16 or f16 only");
  P3D_CHECK_ARG(x && weight && bias && y, "p3d_layer_norm: null pointer");
  P3D_CHECK_ARG(rows >= 0 && dim >= 8 && dim % 8 == 0, "p3d_layer_norm: dim must be a positive multiple of 8");
  P3D_CHECK_ARG(aligned16(x) && aligned16(weight) && aligned16(bias) && aligned16(y),
                "p3d_layer_norm: 16-byte aligned tensors required");
  P3D_CHECK_ARG(eps >= 0.f, "p3d_layer_norm: negative eps");
  if (rows == 0) return P3D_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == P3D_BF16 ? launch_ln<__nv_bfloat16>(x, weight, bias, y, rows, dim, eps, s)
                           : launch_ln<__half>(x, weight, bias, y, rows, dim, eps, s);
}

namespace {
// Arguments shared by p3d_qkv_split and p3d_qkv_merge (names as in p3d_qkv_split).
int check_split(const char *name, const void *const (&ptrs)[7], int dtype, int batch, int heads, int kv_heads,
                int tokens, int head_dim, const int64_t *coords, int pz, int py, int px, const float *phases, int ez,
                int ey, int ex) {
  P3D_CHECK_ARG(dtype == P3D_BF16 || dtype == P3D_F16, "%s: bf16 or f16 only", name);
  for (const void *t : ptrs) P3D_CHECK_ARG(t != nullptr, "%s: null pointer", name);
  P3D_CHECK_ARG(coords && phases, "%s: null pointer", name);
  P3D_CHECK_ARG(batch >= 0 && heads >= 1 && kv_heads >= 1 && heads % kv_heads == 0 && tokens >= 0,
                "%s: bad batch / head / token counts", name);
  P3D_CHECK_ARG(head_dim % 8 == 0 && 2 * (pz + py + px) == head_dim && pz >= 0 && py >= 0 && px >= 0,
                "%s: pairs (%d,%d,%d) do not allocate head_dim %d", name, pz, py, px, head_dim);
  P3D_CHECK_ARG(ez >= 1 && ey >= 1 && ex >= 1, "%s: bad table extents", name);
  for (const void *t : ptrs) P3D_CHECK_ARG(aligned16(t), "%s: 16-byte aligned tensors required", name);
  P3D_CHECK_ARG(batch <= 65535, "%s: batch above 65535", name);
  return P3D_OK;
}
}  // namespace

extern "C" size_t p3d_layer_norm_bwd_workspace(int64_t rows, int dim) {
  if (rows < 1 || dim < 8) return 0;
  float *a, *b, *t;
  return ln_bwd_layout(rows, dim, nullptr, &a, &b, &t);
}

namespace {
int layer_norm_bwd(const char *name, const void *x, const void *weight, const void *dy, const void *dres, void *dx,
                   float *dweight, float *dbias, int dtype, int64_t rows, int dim, float eps, void *workspace,
                   size_t workspace_bytes, void *stream) {
  P3D_CHECK_ARG(dtype == P3D_BF16 || dtype == P3D_F16, "%s: bf16 or f16 only", name);
  P3D_CHECK_ARG(x && weight && dy && dx && dweight && dbias, "%s: null pointer", name);
  P3D_CHECK_ARG(rows >= 1 && dim >= 8 && dim % 8 == 0, "%s: rows >= 1, dim a positive multiple of 8", name);
  P3D_CHECK_ARG(aligned16(x) && aligned16(weight) && aligned16(dy) && aligned16(dx) && aligned16(dres),
                "%s: 16-byte aligned tensors required", name);
  P3D_CHECK_ARG(eps >= 0.f, "%s: negative eps", name);
  float *dw_part, *db_part, *tmp;
  const size_t need = ln_bwd_layout(rows, dim, workspace, &dw_part, &db_part, &tmp);
  if (!workspace || workspace_bytes < need)
    return fail(P3D_ERR_WORKSPACE, "%s: workspace of %zu bytes required", name, need);
  P3D_CHECK_ARG(((uintptr_t)workspace & 15) == 0, "%s: 16-byte aligned workspace required", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned blocks = ln_bwd_blocks(rows);
  const int st =
      dtype == P3D_BF16
          ? launch_ln_bwd_any<__nv_bfloat16>(x, weight, dy, dres, dx, dw_part, db_part, rows, dim, eps, blocks, s)
          : launch_ln_bwd_any<__half>(x, weight, dy, dres, dx, dw_part, db_part, rows, dim, eps, blocks, s);
  if (st) return st;
  const int64_t warps = (int64_t)blocks * kWarps;
  if (int e = launch_sum_rows(dw_part, dweight, warps, dim, tmp, s)) return e;
  return launch_sum_rows(db_part, dbias, warps, dim, tmp, s);
}
}  // namespace

extern "C" int p3d_layer_norm_bwd(const void *x, const void *weight, const void *dy, void *dx, float *dweight,
                                  float *dbias, int dtype, int64_t rows, int dim, float eps, void *workspace,
                                  size_t workspace_bytes, void *stream) {
  return layer_norm_bwd("p3d_layer_norm_bwd", x, weight, dy, nullptr, dx, dweight, dbias, dtype, rows, dim, eps,
                        workspace, workspace_bytes, stream);
}

extern "C" int p3d_layer_norm_bwd_residual(const void *x, const void *weight, const void *dy, const void *dres,
                                           void *dx, float *dweight, float *dbias, int dtype, int64_t rows, int dim,
                                           float eps, void *workspace, size_t workspace_bytes, void *stream) {
  P3D_CHECK_ARG(dres, "p3d_layer_norm_bwd_residual: null pointer");
  return layer_norm_bwd("p3d_layer_norm_bwd_residual", x, weight, dy, dres, dx, dweight, dbias, dtype, rows, dim,
                        eps, workspace, workspace_bytes, stream);
}

extern "C" int p3d_qkv_split(const void *qp, const void *kvp, void *q, void *kl, void *vl, void *kg, void *vg,
                             int dtype, int batch, int heads, int kv_heads, int tokens, int head_dim,
                             const int64_t *coords, int pz, int py, int px, const float *phases, int ez, int ey,
                             int ex, unsigned flags, void *stream) {
  const void *const ptrs[7] = {qp, kvp, q, kl, vl, kg, vg};
  if (int st = check_split("p3d_qkv_split", ptrs, dtype, batch, heads, kv_heads, tokens, head_dim, coords, pz, py,
                           px, phases, ez, ey, ex))
    return st;
  P3D_CHECK_ARG((flags & ~P3D_SPLIT_RASTER_QKV) == 0u, "p3d_qkv_split: unknown flags 0x%x", flags);
  P3D_CHECK_ARG(!(flags & P3D_SPLIT_RASTER_QKV) || (int64_t)ez * ey * ex == tokens,
                "p3d_qkv_split: raster rows need the coordinate extents to be the token grid (%d x %d x %d != %d)",
                ez, ey, ex, tokens);
  if ((int64_t)batch * tokens == 0) return P3D_OK;
  SplitParams p{};
  p.qp = qp;
  p.kvp = kvp;
  p.out[0] = q;
  p.out[1] = kl;
  p.out[2] = vl;
  p.out[3] = kg;
  p.out[4] = vg;
  p.batch = batch;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.tokens = tokens;
  p.coords = coords;
  p.pairs[0] = pz;
  p.pairs[1] = py;
  p.pairs[2] = px;
  p.start[0] = 0;
  p.start[1] = ez * pz;
  p.start[2] = ez * pz + ey * py;
  p.phases = phases;
  p.raster_qkv = (flags & P3D_SPLIT_RASTER_QKV) ? 1 : 0;
  p.ey = ey;
  p.ex = ex;
  p.q_stride = heads * head_dim;
  p.kv_stride = 4 * kv_heads * head_dim;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == P3D_BF16 ? launch_split<__nv_bfloat16>(p, head_dim, s) : launch_split<__half>(p, head_dim, s);
}

// gate[b, h, n] = softmax(logits[b, n, 2h .. 2h + 1])[1] (attention.py:84-86), in fp32 with expf and
// a division, rounded once; a thread per (head, token) in gate order (coalesced stores), logits
// read as one 4-byte pair.
template <typename T>
__global__ void __launch_bounds__(256) gate_pairs_kernel(const T *logits, int stride, T *gate, int heads,
                                                         int tokens, int64_t total) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bh = k / tokens, n = k - bh * tokens, b = bh / heads;
    const int h = (int)(bh - b * heads);
    const float2 l = unpack2<T>(__ldg(reinterpret_cast<const uint32_t *>(logits + (b * tokens + n) * stride + 2 * h)));
    const float m = fmaxf(l.x, l.y);
    const float e0 = expf(l.x - m), e1 = expf(l.y - m);
    gate[k] = from_f32<T>(e1 / (e0 + e1));
  }
}

extern "C" int p3d_gate_pairs(const void *logits, int stride, void *gate, int dtype, int batch, int heads,
                              int tokens, void *stream) {
  P3D_CHECK_ARG(dtype == P3D_BF16 || dtype == P3D_F16, "p3d_gate_pairs: bf16 or f16 only");
  P3D_CHECK_ARG(logits && gate, "p3d_gate_pairs: null pointer");
  P3D_CHECK_ARG(batch >= 0 && heads >= 1 && tokens >= 0 && stride >= 2 * heads && stride % 2 == 0,
                "p3d_gate_pairs: bad shape (stride %d for %d heads)", stride, heads);
  P3D_CHECK_ARG(((uintptr_t)logits & 3) == 0, "p3d_gate_pairs: logits must be 4-byte aligned");
  const int64_t total = (int64_t)batch * tokens * heads;
  if (total == 0) return P3D_OK;
  DeviceInfo info{};
  if (int st = device_info(&info)) return st;
  const int64_t want = (total + 255) / 256, cap = (int64_t)info.sm_count * 8;
  const unsigned blocks = (unsigned)(want < cap ? want : cap);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == P3D_BF16)
    gate_pairs_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(logits), stride,
                                                             static_cast<__nv_bfloat16 *>(gate), heads, tokens, total);
  else
    gate_pairs_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half *>(logits), stride,
                                                     static_cast<__half *>(gate), heads, tokens, total);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

extern "C" int p3d_qkv_gate_split(const void *proj, int proj_cols, void *q, void *kl, void *vl, void *kg, void *vg,
                                  void *gate, int dtype, int batch, int heads, int kv_heads, int tokens, int head_dim,
                                  const int64_t *coords, int pz, int py, int px, const float *phases, int ez, int ey,
                                  int ex, unsigned flags, void *stream) {
  const void *const ptrs[7] = {proj, gate, q, kl, vl, kg, vg};
  if (int st = check_split("p3d_qkv_gate_split", ptrs, dtype, batch, heads, kv_heads, tokens, head_dim, coords, pz,
                           py, px, phases, ez, ey, ex))
    return st;
  P3D_CHECK_ARG((flags & ~P3D_SPLIT_RASTER_QKV) == 0u, "p3d_qkv_gate_split: unknown flags 0x%x", flags);
  P3D_CHECK_ARG(!(flags & P3D_SPLIT_RASTER_QKV) || (int64_t)ez * ey * ex == tokens,
                "p3d_qkv_gate_split: raster rows need the coordinate extents to be the token grid (%d x %d x %d != %d)",
                ez, ey, ex, tokens);
  P3D_CHECK_ARG(heads <= 32 * kGateRounds / kTokensPerWarp, "p3d_qkv_gate_split: at most %d heads",
                32 * kGateRounds / kTokensPerWarp);
  const int used = (heads + 4 * kv_heads) * head_dim + 2 * heads;
  P3D_CHECK_ARG(proj_cols >= used && proj_cols % 8 == 0,
                "p3d_qkv_gate_split: proj_cols %d must cover the %d projection columns and be a multiple of 8",
                proj_cols, used);
  if ((int64_t)batch * tokens == 0) return P3D_OK;
  const size_t es = 2;
  SplitParams p{};
  p.qp = proj;
  p.kvp = static_cast<const char *>(proj) + es * heads * head_dim;
  p.out[0] = q;
  p.out[1] = kl;
  p.out[2] = vl;
  p.out[3] = kg;
  p.out[4] = vg;
  p.batch = batch;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.tokens = tokens;
  p.coords = coords;
  p.pairs[0] = pz;
  p.pairs[1] = py;
  p.pairs[2] = px;
  p.start[0] = 0;
  p.start[1] = ez * pz;
  p.start[2] = ez * pz + ey * py;
  p.phases = phases;
  p.raster_qkv = (flags & P3D_SPLIT_RASTER_QKV) ? 1 : 0;
  p.ey = ey;
  p.ex = ex;
  p.q_stride = p.kv_stride = p.gate_stride = proj_cols;
  p.gate_logits = static_cast<const char *>(proj) + es * (heads + 4 * kv_heads) * head_dim;
  p.gate = gate;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == P3D_BF16 ? launch_split<__nv_bfloat16>(p, head_dim, s) : launch_split<__half>(p, head_dim, s);
}

extern "C" int p3d_qkv_merge(const void *dq, const void *dkl, const void *dvl, const void *dkg, const void *dvg,
                             void *dqp, void *dkvp, int dtype, int batch, int heads, int kv_heads, int tokens,
                             int head_dim, const int64_t *coords, int pz, int py, int px, const float *phases, int ez,
                             int ey, int ex, void *stream) {
  const void *const ptrs[7] = {dqp, dkvp, dq, dkl, dvl, dkg, dvg};
  if (int st = check_split("p3d_qkv_merge", ptrs, dtype, batch, heads, kv_heads, tokens, head_dim, coords, pz, py,
                           px, phases, ez, ey, ex))
    return st;
  if ((int64_t)batch * tokens == 0) return P3D_OK;
  SplitParams p{};
  p.qp = dqp;
  p.kvp = dkvp;
  p.out[0] = const_cast<void *>(dq);
  p.out[1] = const_cast<void *>(dkl);
  p.out[2] = const_cast<void *>(dvl);
  p.out[3] = const_cast<void *>(dkg);
  p.out[4] = const_cast<void *>(dvg);
  p.batch = batch;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.tokens = tokens;
  p.coords = coords;
  p.pairs[0] = pz;
  p.pairs[1] = py;
  p.pairs[2] = px;
  p.start[0] = 0;
  p.start[1] = ez * pz;
  p.start[2] = ez * pz + ey * py;
  p.phases = phases;
  p.q_stride = heads * head_dim;
  p.kv_stride = 4 * kv_heads * head_dim;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == P3D_BF16 ? launch_merge<__nv_bfloat16>(p, head_dim, s) : launch_merge<__half>(p, head_dim, s);
}
