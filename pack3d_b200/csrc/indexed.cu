// Indexed attention kernels: every dtype, any validated graph (neighbour table),
// head_dim <= 128, GQA.  They serve the fp32 path, custom graphs from
// prepare_geometry and the backward until the tensor-core kernels cover it.
//
// Restated from the reference core (reference.py:20-31) and its Triton kernels
// _local_fwd, _global_fwd, _mix_bwd, _local_dq, _local_dkv, _global_dq,
// _global_dkv (kernels.py:44-239):
//   local    s = q.k / sqrt(D) over valid neighbours, masked softmax, all-masked -> 0
//   global   online softmax over all summaries
//   mix      y = sl*ol + (gate*sg)*og
//   backward dS = P (dP - Delta), Delta = rowsum(dO * O); local dK/dV through the
//            reverse adjacency (owner writes, no atomics); global dSK/dSV as
//            query-split partials summed in a fixed order.
// One warp per output row: lanes own neighbours / summaries for the scores and
// channels for the weighted sums (scores broadcast by shuffle).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace p3d {
namespace {

constexpr int kWarps = 8;
constexpr float kInf = __builtin_huge_valf();

struct RowIds {
  int64_t row;   // warp's output row id
  int i, bh, b, h, bg;
};

__device__ __forceinline__ bool query_row(const IndexedArgs &a, RowIds &r) {
  r.row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (r.row >= (int64_t)a.batch * a.heads * a.tokens) return false;
  r.i = (int)(r.row % a.tokens);
  r.bh = (int)(r.row / a.tokens);
  r.b = r.bh / a.heads;
  r.h = r.bh % a.heads;
  r.bg = r.b * a.kv_heads + r.h / (a.heads / a.kv_heads);
  return true;
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) local_fwd_kernel(IndexedArgs a, T *ol, float *lse, bool vec) {
  extern __shared__ float smem[];
  const int d = a.head_dim, lane = threadIdx.x & 31;
  float *qs = smem + (threadIdx.x >> 5) * d;
  RowIds r;
  if (!query_row(a, r)) return;
  const int64_t qoff = r.row * d;
  row_to_smem(static_cast<const T *>(a.q) + qoff, qs, d);
  const T *K = static_cast<const T *>(a.kl) + (int64_t)r.bg * a.tokens * d;
  const T *V = static_cast<const T *>(a.vl) + (int64_t)r.bg * a.tokens * d;
  const int32_t *nb = a.neighbors + (int64_t)r.i * a.width;
  const float root = sqrtf((float)d);
  float s[4];
  int idx[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int c = lane + 32 * k;
    idx[k] = c < a.width ? nb[c] : -1;
    s[k] = idx[k] >= 0 ? dot_row(K + (int64_t)idx[k] * d, qs, d, vec) / root : -kInf;
  }
  const float mx = warp_max(fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3])));
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float l = 0.f;
  if (mx != -kInf) {
    float e[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) e[k] = idx[k] >= 0 ? expf(s[k] - mx) : 0.f;
    l = warp_sum(e[0] + e[1] + e[2] + e[3]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (32 * k >= a.width) break;
      for (int src = 0; src < 32; ++src) {
        const int id = __shfl_sync(0xffffffffu, idx[k], src);
        const float p = __shfl_sync(0xffffffffu, e[k], src);
        if (id < 0) continue;
        const T *vr = V + (int64_t)id * d;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int ch = lane + 32 * c;
          if (ch < d) acc[c] = fmaf(p, to_f32<T>(vr[ch]), acc[c]);
        }
      }
    }
  }
  const float inv = mx != -kInf ? 1.f / l : 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int ch = lane + 32 * c;
    if (ch < d) ol[qoff + ch] = from_f32<T>(acc[c] * inv);
  }
  if (lse && lane == 0) lse[r.row] = mx != -kInf ? mx + logf(l) : kInf;
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
    global_fwd_mix_kernel(IndexedArgs a, const T *ol, T *y, T *og, float *lse, bool vec) {
  extern __shared__ float smem[];
  const int d = a.head_dim, lane = threadIdx.x & 31, M = a.summaries;
  float *qs = smem + (threadIdx.x >> 5) * d;
  RowIds r;
  if (!query_row(a, r)) return;
  const int64_t qoff = r.row * d;
  row_to_smem(static_cast<const T *>(a.q) + qoff, qs, d);
  const T *SK = static_cast<const T *>(a.sk) + (int64_t)r.bg * M * d;
  const T *SV = static_cast<const T *>(a.sv) + (int64_t)r.bg * M * d;
  const float root = sqrtf((float)d);
  float run_max = -kInf, run_sum = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j0 = 0; j0 < M; j0 += 32) {
    const int j = j0 + lane;
    const float s = j < M ? dot_row(SK + (int64_t)j * d, qs, d, vec) / root : -kInf;
    const float new_max = fmaxf(run_max, warp_max(s));
    const float alpha = expf(run_max - new_max);
    const float e = j < M ? expf(s - new_max) : 0.f;
    run_sum = run_sum * alpha + warp_sum(e);
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[c] *= alpha;
    const int count = min(32, M - j0);
    for (int src = 0; src < count; ++src) {
      const float p = __shfl_sync(0xffffffffu, e, src);
      const T *vr = SV + (int64_t)(j0 + src) * d;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int ch = lane + 32 * c;
        if (ch < d) acc[c] = fmaf(p, to_f32<T>(vr[ch]), acc[c]);
      }
    }
    run_max = new_max;
  }
  const float inv = 1.f / run_sum;
  const float gate = load_any(a.gate, a.gate_dtype, r.row);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int ch = lane + 32 * c;
    if (ch < d) {
      const float o = acc[c] * inv;
      const float local = to_f32<T>(ol[qoff + ch]);
      // y = sl * ol + (gate * sg) * og, each product rounded as in the reference
      const float v = __fadd_rn(__fmul_rn(a.sl[ch], local), __fmul_rn(__fmul_rn(gate, a.sg[ch]), o));
      y[(a.y_rows ? ((int64_t)r.b * a.tokens + r.i) * a.heads + r.h : r.row) * d + ch] = from_f32<T>(v);
      if (og) og[qoff + ch] = from_f32<T>(o);
    }
  }
  if (lse && lane == 0) lse[r.row] = run_max + logf(run_sum);
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) mix_bwd_kernel(MixBwdArgs a) {
  const int d = a.head_dim, lane = threadIdx.x & 31;
  const int chunks = (a.tokens + a.chunk_rows - 1) / a.chunk_rows;
  const int64_t wid = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (wid >= (int64_t)a.bh * chunks) return;
  const int bh = (int)(wid / chunks);
  const int r0 = (int)(wid % chunks) * a.chunk_rows;
  const int r1 = min(a.tokens, r0 + a.chunk_rows);
  const T *dy = static_cast<const T *>(a.dy), *ol = static_cast<const T *>(a.ol);
  const T *og = static_cast<const T *>(a.og);
  T *dol = static_cast<T *>(a.dol), *dog = static_cast<T *>(a.dog);
  float dsl[4] = {0.f, 0.f, 0.f, 0.f}, dsg[4] = {0.f, 0.f, 0.f, 0.f};
  for (int i = r0; i < r1; ++i) {
    const int64_t row = (int64_t)bh * a.tokens + i;
    const int64_t dy_row = a.dy_rows ? ((int64_t)(bh / a.heads) * a.tokens + i) * a.heads + bh % a.heads : row;
    const float gate = load_any(a.gate, a.gate_dtype, row);
    float dl = 0.f, dg = 0.f, dgate = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int ch = lane + 32 * c;
      if (ch >= d) continue;
      const int64_t off = row * d + ch;
      const float g_y = to_f32<T>(dy[dy_row * d + ch]), o_l = to_f32<T>(ol[off]), o_g = to_f32<T>(og[off]);
      // Delta uses the same rounded branch gradients the attention VJPs consume.
      const float g_l = round_to<T>(g_y * a.sl[ch]);
      const float g_g = round_to<T>((g_y * gate) * a.sg[ch]);
      dol[off] = from_f32<T>(g_l);
      dog[off] = from_f32<T>(g_g);
      dl = fmaf(g_l, o_l, dl);
      dg = fmaf(g_g, o_g, dg);
      dgate = fmaf(g_y * o_g, a.sg[ch], dgate);
      dsl[c] = fmaf(g_y, o_l, dsl[c]);
      dsg[c] = fmaf(g_y * o_g, gate, dsg[c]);
    }
    dl = warp_sum(dl);
    dg = warp_sum(dg);
    dgate = warp_sum(dgate);
    if (lane == 0) {
      a.delta_l[row] = dl;
      a.delta_g[row] = dg;
      store_any(a.dgate, a.gate_dtype, row, dgate);
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int ch = lane + 32 * c;
    if (ch < d) {
      a.dsl_part[wid * d + ch] = dsl[c];
      a.dsg_part[wid * d + ch] = dsg[c];
    }
  }
}

// The mix backward for 16-bit rows with D in {8, 16, 32, 48, 64, 128} and 16-byte-aligned
// tensors: the same per-element arithmetic as mix_bwd_kernel, laid out for bandwidth.  A row
// is a segment of S lanes (S = the power of two >= D / 8), one 16-byte chunk per lane, so a
// warp pass covers 32 / S rows and kBatch passes of loads are issued before the first use.
// The per-row sums (Delta_l, Delta_g, dgate) reduce inside the segment (xor shuffles); the
// per-channel sums (dsl, dsg) accumulate per lane over the lane's rows and combine across
// segments at the end.  Summation orders differ from mix_bwd_kernel (fp32 rounding).
template <int D>
struct MixVec {
  static constexpr int kC = D / 8;  // chunks per row
  static constexpr int kS = kC <= 1 ? 1 : kC <= 2 ? 2 : kC <= 4 ? 4 : kC <= 8 ? 8 : 16;  // lanes per row
  static constexpr int kR = 32 / kS;  // rows per warp pass
  static constexpr int kBatch = 4;    // passes loaded ahead
};

template <typename T>
__device__ __forceinline__ void unpack8f(const uint4 &raw, float (&v)[8]) {
  const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack2<T>(u[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2f(float x, float y) {
  const T lo = from_f32<T>(x), hi = from_f32<T>(y);
  uint16_t a, b;
  memcpy(&a, &lo, 2);
  memcpy(&b, &hi, 2);
  return (uint32_t)a | ((uint32_t)b << 16);
}

template <int S>
__device__ __forceinline__ float segment_sum(float v) {
#pragma unroll
  for (int o = 1; o < S; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, int D>
__global__ void __launch_bounds__(kWarps * 32) mix_bwd_vec_kernel(MixBwdArgs a) {
  using G = MixVec<D>;
  const int lane = threadIdx.x & 31, seg = lane / G::kS, c = lane % G::kS;
  const bool on = c < G::kC;
  const int chunks = (a.tokens + a.chunk_rows - 1) / a.chunk_rows;
  const int64_t wid = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (wid >= (int64_t)a.bh * chunks) return;
  const int bh = (int)(wid / chunks);
  const int r0 = (int)(wid % chunks) * a.chunk_rows;
  const int r1 = min(a.tokens, r0 + a.chunk_rows);
  const T *dy = static_cast<const T *>(a.dy), *ol = static_cast<const T *>(a.ol);
  const T *og = static_cast<const T *>(a.og);
  T *dol = static_cast<T *>(a.dol), *dog = static_cast<T *>(a.dog);
  float sl[8], sg[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    sl[e] = on ? a.sl[8 * c + e] : 0.f;
    sg[e] = on ? a.sg[8 * c + e] : 0.f;
  }
  float dsl[8], dsg[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) dsl[e] = dsg[e] = 0.f;
  for (int base = r0; base < r1; base += G::kR * G::kBatch) {
    uint4 rgy[G::kBatch], rlo[G::kBatch], rgo[G::kBatch];  // raw 16-byte chunks, unpacked on use
    float gate[G::kBatch];
#pragma unroll
    for (int i = 0; i < G::kBatch; ++i) {
      const int t = base + i * G::kR + seg;
      const int tt = t < r1 ? t : r0;
      const int64_t row = (int64_t)bh * a.tokens + tt;
      const int64_t off = row * D + 8 * c;
      const int64_t dy_row = a.dy_rows ? ((int64_t)(bh / a.heads) * a.tokens + tt) * a.heads + bh % a.heads : row;
      rgy[i] = rlo[i] = rgo[i] = make_uint4(0u, 0u, 0u, 0u);
      if (on && t < r1) {
        rgy[i] = *reinterpret_cast<const uint4 *>(dy + dy_row * D + 8 * c);
        rlo[i] = *reinterpret_cast<const uint4 *>(ol + off);
        rgo[i] = *reinterpret_cast<const uint4 *>(og + off);
      }
      gate[i] = load_any(a.gate, a.gate_dtype, row);
    }
#pragma unroll
    for (int i = 0; i < G::kBatch; ++i) {
      if (base + i * G::kR >= r1) break;  // warp-uniform
      const int t = base + i * G::kR + seg;
      const bool valid = on && t < r1;
      const int64_t row = (int64_t)bh * a.tokens + t;
      float gy[8], lo[8], go[8];
      unpack8f<T>(rgy[i], gy);
      unpack8f<T>(rlo[i], lo);
      unpack8f<T>(rgo[i], go);
      float dl = 0.f, dg = 0.f, dgate = 0.f;
      uint32_t pl[4], pg[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float g_l[2], g_g[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float g_y = gy[e + h];
          // Delta uses the same rounded branch gradients the attention VJPs consume.
          g_l[h] = round_to<T>(g_y * sl[e + h]);
          g_g[h] = round_to<T>((g_y * gate[i]) * sg[e + h]);
          dl = fmaf(g_l[h], lo[e + h], dl);
          dg = fmaf(g_g[h], go[e + h], dg);
          dgate = fmaf(g_y * go[e + h], sg[e + h], dgate);
          if (valid) {
            dsl[e + h] = fmaf(g_y, lo[e + h], dsl[e + h]);
            dsg[e + h] = fmaf(g_y * go[e + h], gate[i], dsg[e + h]);
          }
        }
        pl[e / 2] = pack2f<T>(g_l[0], g_l[1]);
        pg[e / 2] = pack2f<T>(g_g[0], g_g[1]);
      }
      if (valid) {
        *reinterpret_cast<uint4 *>(dol + row * D + 8 * c) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
        *reinterpret_cast<uint4 *>(dog + row * D + 8 * c) = make_uint4(pg[0], pg[1], pg[2], pg[3]);
      }
      dl = segment_sum<G::kS>(dl);
      dg = segment_sum<G::kS>(dg);
      dgate = segment_sum<G::kS>(dgate);
      if (c == 0 && t < r1) {
        a.delta_l[row] = dl;
        a.delta_g[row] = dg;
        store_any(a.dgate, a.gate_dtype, row, dgate);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
#pragma unroll
    for (int o = G::kS; o < 32; o <<= 1) {
      dsl[e] += __shfl_xor_sync(0xffffffffu, dsl[e], o);
      dsg[e] += __shfl_xor_sync(0xffffffffu, dsg[e], o);
    }
  }
  if (seg == 0 && on) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      a.dsl_part[wid * D + 8 * c + e] = dsl[e];
      a.dsg_part[wid * D + 8 * c + e] = dsg[e];
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
    local_dq_kernel(IndexedArgs a, const T *dol, const float *lse_l, const float *delta_l, T *dq, bool vec) {
  extern __shared__ float smem[];
  const int d = a.head_dim, lane = threadIdx.x & 31;
  float *qs = smem + (threadIdx.x >> 5) * 2 * d, *dos = qs + d;
  RowIds r;
  if (!query_row(a, r)) return;
  const int64_t qoff = r.row * d;
  row_to_smem(static_cast<const T *>(a.q) + qoff, qs, d);
  row_to_smem(dol + qoff, dos, d);
  const T *K = static_cast<const T *>(a.kl) + (int64_t)r.bg * a.tokens * d;
  const T *V = static_cast<const T *>(a.vl) + (int64_t)r.bg * a.tokens * d;
  const int32_t *nb = a.neighbors + (int64_t)r.i * a.width;
  const float root = sqrtf((float)d);
  const float lse = lse_l[r.row], delta = delta_l[r.row];
  float ds[4];
  int idx[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int c = lane + 32 * k;
    idx[k] = c < a.width ? nb[c] : -1;
    ds[k] = 0.f;
    if (idx[k] >= 0) {
      const float s = dot_row(K + (int64_t)idx[k] * d, qs, d, vec) / root;
      const float p = expf(s - lse);
      const float dp = dot_row(V + (int64_t)idx[k] * d, dos, d, vec);
      ds[k] = p * (dp - delta) / root;
    }
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (32 * k >= a.width) break;
    for (int src = 0; src < 32; ++src) {
      const int id = __shfl_sync(0xffffffffu, idx[k], src);
      const float g = __shfl_sync(0xffffffffu, ds[k], src);
      if (id < 0) continue;
      const T *kr = K + (int64_t)id * d;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int ch = lane + 32 * c;
        if (ch < d) acc[c] = fmaf(g, to_f32<T>(kr[ch]), acc[c]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int ch = lane + 32 * c;
    if (ch < d) dq[qoff + ch] = from_f32<T>(acc[c]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) local_dkv_kernel(IndexedArgs a, const T *dol, const float *lse_l,
                                                                const float *delta_l, T *dkl, T *dvl, bool vec) {
  extern __shared__ float smem[];
  const int d = a.head_dim, lane = threadIdx.x & 31;
  float *ks = smem + (threadIdx.x >> 5) * 2 * d, *vs = ks + d;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);  // (bg, j)
  if (row >= (int64_t)a.batch * a.kv_heads * a.tokens) return;
  const int j = (int)(row % a.tokens);
  const int bg = (int)(row / a.tokens);
  const int b = bg / a.kv_heads, g = bg % a.kv_heads, rep = a.heads / a.kv_heads;
  row_to_smem(static_cast<const T *>(a.kl) + row * d, ks, d);
  row_to_smem(static_cast<const T *>(a.vl) + row * d, vs, d);
  const int32_t *rev = a.reverse + (int64_t)j * a.reverse_width;
  const float root = sqrtf((float)d);
  float dk[4] = {0.f, 0.f, 0.f, 0.f}, dv[4] = {0.f, 0.f, 0.f, 0.f};
  for (int hh = 0; hh < rep; ++hh) {
    const int bh = b * a.heads + g * rep + hh;
    const T *Q = static_cast<const T *>(a.q) + (int64_t)bh * a.tokens * d;
    const T *DO = dol + (int64_t)bh * a.tokens * d;
    const float *LSE = lse_l + (int64_t)bh * a.tokens, *DEL = delta_l + (int64_t)bh * a.tokens;
    for (int k = 0; k < (a.reverse_width + 31) / 32; ++k) {
      const int c = lane + 32 * k;
      const int i = c < a.reverse_width ? rev[c] : -1;
      float p = 0.f, gs = 0.f;
      if (i >= 0) {
        const float s = dot_row(Q + (int64_t)i * d, ks, d, vec) / root;
        p = expf(s - LSE[i]);
        const float dp = dot_row(DO + (int64_t)i * d, vs, d, vec);
        gs = p * (dp - DEL[i]) / root;
      }
      for (int src = 0; src < 32; ++src) {
        const int id = __shfl_sync(0xffffffffu, i, src);
        const float pp = __shfl_sync(0xffffffffu, p, src);
        const float gg = __shfl_sync(0xffffffffu, gs, src);
        if (id < 0) continue;
        const T *qr = Q + (int64_t)id * d, *dr = DO + (int64_t)id * d;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int ch = lane + 32 * cc;
          if (ch < d) {
            dk[cc] = fmaf(gg, to_f32<T>(qr[ch]), dk[cc]);
            dv[cc] = fmaf(pp, to_f32<T>(dr[ch]), dv[cc]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int ch = lane + 32 * c;
    if (ch < d) {
      dkl[row * d + ch] = from_f32<T>(dk[c]);
      dvl[row * d + ch] = from_f32<T>(dv[c]);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) global_dq_kernel(IndexedArgs a, const T *dog, const float *lse_g,
                                                                const float *delta_g, T *dq, bool vec) {
  extern __shared__ float smem[];
  const int d = a.head_dim, lane = threadIdx.x & 31, M = a.summaries;
  float *qs = smem + (threadIdx.x >> 5) * 2 * d, *dos = qs + d;
  RowIds r;
  if (!query_row(a, r)) return;
  const int64_t qoff = r.row * d;
  row_to_smem(static_cast<const T *>(a.q) + qoff, qs, d);
  row_to_smem(dog + qoff, dos, d);
  const T *SK = static_cast<const T *>(a.sk) + (int64_t)r.bg * M * d;
  const T *SV = static_cast<const T *>(a.sv) + (int64_t)r.bg * M * d;
  const float root = sqrtf((float)d);
  const float lse = lse_g[r.row], delta = delta_g[r.row];
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j0 = 0; j0 < M; j0 += 32) {
    const int j = j0 + lane;
    float g = 0.f;
    if (j < M && M > 1) {  // one summary: softmax is constant, no score gradient
      const float s = dot_row(SK + (int64_t)j * d, qs, d, vec) / root;
      const float p = expf(s - lse);
      const float dp = dot_row(SV + (int64_t)j * d, dos, d, vec);
      g = p * (dp - delta) / root;
    }
    const int count = min(32, M - j0);
    for (int src = 0; src < count; ++src) {
      const float gg = __shfl_sync(0xffffffffu, g, src);
      const T *kr = SK + (int64_t)(j0 + src) * d;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int ch = lane + 32 * c;
        if (ch < d) acc[c] = fmaf(gg, to_f32<T>(kr[ch]), acc[c]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int ch = lane + 32 * c;
    if (ch < d) {
      // Local and global query gradients are each rounded to storage, then added.
      const float local = to_f32<T>(dq[qoff + ch]);
      dq[qoff + ch] = from_f32<T>(local + round_to<T>(acc[c]));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
    global_dkv_kernel(IndexedArgs a, const T *dog, const float *lse_g, const float *delta_g, int splits,
                      float *dk_part, float *dv_part, bool vec) {
  extern __shared__ float smem[];
  const int d = a.head_dim, lane = threadIdx.x & 31, M = a.summaries;
  float *ks = smem + (threadIdx.x >> 5) * 2 * d, *vs = ks + d;
  const int64_t wid = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (wid >= (int64_t)M * splits * a.batch * a.kv_heads) return;
  const int j = (int)(wid % M);
  const int split = (int)((wid / M) % splits);
  const int bg = (int)(wid / ((int64_t)M * splits));
  const int b = bg / a.kv_heads, g = bg % a.kv_heads, rep = a.heads / a.kv_heads;
  row_to_smem(static_cast<const T *>(a.sk) + ((int64_t)bg * M + j) * d, ks, d);
  row_to_smem(static_cast<const T *>(a.sv) + ((int64_t)bg * M + j) * d, vs, d);
  const int per = (a.tokens + splits - 1) / splits;
  const int r0 = split * per, r1 = min(a.tokens, r0 + per);
  const float root = sqrtf((float)d);
  float dk[4] = {0.f, 0.f, 0.f, 0.f}, dv[4] = {0.f, 0.f, 0.f, 0.f};
  for (int hh = 0; hh < rep; ++hh) {
    const int bh = b * a.heads + g * rep + hh;
    const T *Q = static_cast<const T *>(a.q) + (int64_t)bh * a.tokens * d;
    const T *DO = dog + (int64_t)bh * a.tokens * d;
    const float *LSE = lse_g + (int64_t)bh * a.tokens, *DEL = delta_g + (int64_t)bh * a.tokens;
    for (int i0 = r0; i0 < r1; i0 += 32) {
      const int i = i0 + lane;
      float p = 0.f, gs = 0.f;
      if (i < r1) {
        if (M > 1) {
          const float s = dot_row(Q + (int64_t)i * d, ks, d, vec) / root;
          p = expf(s - LSE[i]);
          const float dp = dot_row(DO + (int64_t)i * d, vs, d, vec);
          gs = p * (dp - DEL[i]) / root;
        } else {
          p = 1.f;  // a single summary takes the whole softmax mass
        }
      }
      const int count = min(32, r1 - i0);
      for (int src = 0; src < count; ++src) {
        const float pp = __shfl_sync(0xffffffffu, p, src);
        const float gg = __shfl_sync(0xffffffffu, gs, src);
        const T *qr = Q + (int64_t)(i0 + src) * d, *dr = DO + (int64_t)(i0 + src) * d;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int ch = lane + 32 * c;
          if (ch < d) {
            dk[c] = fmaf(gg, to_f32<T>(qr[ch]), dk[c]);
            dv[c] = fmaf(pp, to_f32<T>(dr[ch]), dv[c]);
          }
        }
      }
    }
  }
  const int64_t out = (((int64_t)bg * splits + split) * M + j) * d;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int ch = lane + 32 * c;
    if (ch < d) {
      dk_part[out + ch] = dk[c];
      dv_part[out + ch] = dv[c];
    }
  }
}

__global__ void sum_middle_kernel(const float *in, float *out, int64_t outer, int S, int64_t C) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= outer * C) return;
  const int64_t a = t / C, c = t % C;
  float acc = 0.f;
  for (int s = 0; s < S; ++s) acc += in[(a * S + s) * C + c];
  out[t] = acc;
}

// Column sums of a row-major [R, C] fp32 matrix, in a fixed order (bitwise repeatable).
// Block (x, g) sums rows [g*rows_per_group, ...) of the column chunk x (kSumCols columns):
// thread t takes column t % kSumCols and every S-th row from sub-row t / kSumCols (S =
// kSumThreads / kSumCols), and the S partials of a column are added in sub-row order.
constexpr int kSumThreads = 256, kSumCols = 64;
__global__ void __launch_bounds__(kSumThreads) sum_rows_kernel(const float *in, float *out, int64_t R, int64_t C,
                                                               int rows_per_group) {
  __shared__ float part[kSumThreads];
  const int cols = C < kSumCols ? (int)C : kSumCols;
  const int subs = kSumThreads / cols;
  const int t = threadIdx.x, cl = t % cols, sub = t / cols;
  const int64_t c = (int64_t)blockIdx.x * kSumCols + cl;
  const int64_t group = blockIdx.y;
  const int64_t r0 = group * rows_per_group, r1 = std::min<int64_t>(R, r0 + rows_per_group);
  float acc = 0.f;
  if (sub < subs && c < C)
    for (int64_t r = r0 + sub; r < r1; r += subs) acc += in[r * C + c];
  part[t] = acc;
  __syncthreads();
  if (sub == 0 && c < C) {
    float total = 0.f;
    for (int s = 0; s < subs; ++s) total += part[s * cols + cl];
    out[group * C + c] = total;
  }
}

bool vec_ok(const IndexedArgs &a) {
  const int es = dtype_size(a.dtype);
  if (es != 2 || a.head_dim % 8) return false;
  for (const void *p : {a.q, a.kl, a.vl, a.sk, a.sv})
    if (p && ((uintptr_t)p & 15)) return false;
  return true;
}

size_t row_smem(int head_dim, int rows) { return sizeof(float) * (size_t)kWarps * rows * head_dim; }

}  // namespace

#define P3D_BY_DTYPE(dtype, T, ...)                  \
  switch (dtype) {                                   \
    case P3D_F16: { using T = __half; __VA_ARGS__; break; }          \
    case P3D_BF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }  \
    default: { using T = float; __VA_ARGS__; break; }                \
  }

static int grid_for(int64_t warps) { return (int)((warps + kWarps - 1) / kWarps); }

int launch_local_fwd_indexed(const IndexedArgs &a, void *ol, float *lse_l, cudaStream_t s) {
  const int64_t rows = (int64_t)a.batch * a.heads * a.tokens;
  if (!rows) return P3D_OK;
  const bool vec = vec_ok(a);
  P3D_BY_DTYPE(a.dtype, T,
               local_fwd_kernel<T><<<grid_for(rows), kWarps * 32, row_smem(a.head_dim, 1), s>>>(
                   a, static_cast<T *>(ol), lse_l, vec));
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_global_fwd_mix(const IndexedArgs &a, const void *ol, void *y, void *og, float *lse_g, cudaStream_t s) {
  const int64_t rows = (int64_t)a.batch * a.heads * a.tokens;
  if (!rows) return P3D_OK;
  const bool vec = vec_ok(a);
  P3D_BY_DTYPE(a.dtype, T,
               global_fwd_mix_kernel<T><<<grid_for(rows), kWarps * 32, row_smem(a.head_dim, 1), s>>>(
                   a, static_cast<const T *>(ol), static_cast<T *>(y), static_cast<T *>(og), lse_g, vec));
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_mix_bwd(const MixBwdArgs &a, cudaStream_t s) {
  const int chunks = (a.tokens + a.chunk_rows - 1) / a.chunk_rows;
  const int64_t warps = (int64_t)a.bh * chunks;
  if (!warps) return P3D_OK;
  const bool vec = a.dtype != P3D_F32 && ((uintptr_t)a.dy & 15) == 0 && ((uintptr_t)a.ol & 15) == 0 &&
                   ((uintptr_t)a.og & 15) == 0 && ((uintptr_t)a.dol & 15) == 0 && ((uintptr_t)a.dog & 15) == 0;
  auto by_dim = [&](auto tag) -> bool {
    using T = decltype(tag);
    switch (a.head_dim) {
      case 8: mix_bwd_vec_kernel<T, 8><<<grid_for(warps), kWarps * 32, 0, s>>>(a); return true;
      case 16: mix_bwd_vec_kernel<T, 16><<<grid_for(warps), kWarps * 32, 0, s>>>(a); return true;
      case 32: mix_bwd_vec_kernel<T, 32><<<grid_for(warps), kWarps * 32, 0, s>>>(a); return true;
      case 48: mix_bwd_vec_kernel<T, 48><<<grid_for(warps), kWarps * 32, 0, s>>>(a); return true;
      case 64: mix_bwd_vec_kernel<T, 64><<<grid_for(warps), kWarps * 32, 0, s>>>(a); return true;
      case 128: mix_bwd_vec_kernel<T, 128><<<grid_for(warps), kWarps * 32, 0, s>>>(a); return true;
      default: return false;
    }
  };
  bool done = false;
  if (vec) done = a.dtype == P3D_BF16 ? by_dim(__nv_bfloat16{}) : by_dim(__half{});
  if (!done) P3D_BY_DTYPE(a.dtype, T, mix_bwd_kernel<T><<<grid_for(warps), kWarps * 32, 0, s>>>(a));
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_local_dq_indexed(const IndexedArgs &a, const void *dol, const float *lse_l, const float *delta_l,
                            void *dq, cudaStream_t s) {
  const int64_t rows = (int64_t)a.batch * a.heads * a.tokens;
  if (!rows) return P3D_OK;
  const bool vec = vec_ok(a) && ((uintptr_t)dol & 15) == 0;
  P3D_BY_DTYPE(a.dtype, T,
               local_dq_kernel<T><<<grid_for(rows), kWarps * 32, row_smem(a.head_dim, 2), s>>>(
                   a, static_cast<const T *>(dol), lse_l, delta_l, static_cast<T *>(dq), vec));
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_local_dkv_indexed(const IndexedArgs &a, const void *dol, const float *lse_l, const float *delta_l,
                             void *dkl, void *dvl, cudaStream_t s) {
  const int64_t rows = (int64_t)a.batch * a.kv_heads * a.tokens;
  if (!rows) return P3D_OK;
  const bool vec = vec_ok(a) && ((uintptr_t)dol & 15) == 0;
  P3D_BY_DTYPE(a.dtype, T,
               local_dkv_kernel<T><<<grid_for(rows), kWarps * 32, row_smem(a.head_dim, 2), s>>>(
                   a, static_cast<const T *>(dol), lse_l, delta_l, static_cast<T *>(dkl),
                   static_cast<T *>(dvl), vec));
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_global_dq(const IndexedArgs &a, const void *dog, const float *lse_g, const float *delta_g, void *dq,
                     cudaStream_t s) {
  const int64_t rows = (int64_t)a.batch * a.heads * a.tokens;
  if (!rows) return P3D_OK;
  const bool vec = vec_ok(a) && ((uintptr_t)dog & 15) == 0;
  P3D_BY_DTYPE(a.dtype, T,
               global_dq_kernel<T><<<grid_for(rows), kWarps * 32, row_smem(a.head_dim, 2), s>>>(
                   a, static_cast<const T *>(dog), lse_g, delta_g, static_cast<T *>(dq), vec));
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_global_dkv(const IndexedArgs &a, const void *dog, const float *lse_g, const float *delta_g, int splits,
                      float *dk_part, float *dv_part, cudaStream_t s) {
  const int64_t warps = (int64_t)a.summaries * splits * a.batch * a.kv_heads;
  if (!warps) return P3D_OK;
  const bool vec = vec_ok(a) && ((uintptr_t)dog & 15) == 0;
  P3D_BY_DTYPE(a.dtype, T,
               global_dkv_kernel<T><<<grid_for(warps), kWarps * 32, row_smem(a.head_dim, 2), s>>>(
                   a, static_cast<const T *>(dog), lse_g, delta_g, splits, dk_part, dv_part, vec));
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_sum_middle(const float *in, float *out, int64_t outer, int S, int64_t C, cudaStream_t s) {
  const int64_t total = outer * C;
  if (!total) return P3D_OK;
  sum_middle_kernel<<<(int)((total + 255) / 256), 256, 0, s>>>(in, out, outer, S, C);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

int launch_sum_rows(const float *in, float *out, int64_t R, int64_t C, float *tmp, cudaStream_t s) {
  if (!C) return P3D_OK;
  const int64_t groups = (R + kSumRowsPerGroup - 1) / kSumRowsPerGroup;
  const unsigned col_blocks = (unsigned)((C + kSumCols - 1) / kSumCols);
  if (groups <= 1) {
    sum_rows_kernel<<<dim3(col_blocks, 1), kSumThreads, 0, s>>>(in, out, R, C, kSumRowsPerGroup);
    P3D_LAUNCH_CHECK();
    return P3D_OK;
  }
  if (groups > 65535) return fail(P3D_ERR_UNSUPPORTED, "sum_rows: too many rows (%lld)", (long long)R);
  sum_rows_kernel<<<dim3(col_blocks, (unsigned)groups), kSumThreads, 0, s>>>(in, tmp, R, C, kSumRowsPerGroup);
  P3D_LAUNCH_CHECK();
  sum_rows_kernel<<<dim3(col_blocks, 1), kSumThreads, 0, s>>>(tmp, out, groups, C, (int)groups);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

}  // namespace p3d
