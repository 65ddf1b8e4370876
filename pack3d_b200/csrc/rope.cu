// Stage (a): axial rotary embedding of projected queries / keys.
//
// Restates the rotation of the reference's rope.py:35-48 (per-axis interleaved
// pairs, fp32 angles, product/difference rounded separately, result cast back to
// the storage dtype) as a bandwidth kernel: each thread rotates four planar pairs
// (eight channels) of one token row, reading the strided projection view and
// writing a contiguous head-major row.  With an fp32 (cos, sin) table built on the
// host from the same fp32 angles as the reference, the output is bit-identical.
#include <stdarg.h>

#include <algorithm>

#include "common.cuh"

namespace p3d {
namespace {

constexpr int kPairsPerThread = 4;

struct RopeParams {
  const void *x;
  int64_t sb, sh, sn, sd;
  void *out;
  int batch, heads, tokens, head_dim;
  const int64_t *coords;
  int64_t csn, csa;
  int pairs[3];
  const float *freqs;
  const float *phases;
  int extent[3];
  int packed, inverse;
};

template <typename T, bool kVector, typename Index>
__global__ void __launch_bounds__(256) rope_kernel(RopeParams p) {
  const int half = p.head_dim / 2;
  const int groups = (half + kPairsPerThread - 1) / kPairsPerThread;
  const Index total = (Index)p.batch * p.tokens * groups;
  const Index stride = (Index)gridDim.x * blockDim.x;
  for (Index t = (Index)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    // A thread owns one group of kPairsPerThread pairs of one token and walks all its heads:
    // the token's coordinates and the group's (cos, sin) are fetched once and reused for
    // every head row.  Consecutive threads take consecutive groups of one token, so each
    // head row's channels are read and written as contiguous runs.  Index is 32-bit whenever
    // the thread count allows: the divisions are the costliest arithmetic here.
    const Index bn = t / groups;
    const int grp = (int)(t - bn * groups);
    const int b = (int)(bn / p.tokens), n = (int)(bn - (Index)b * p.tokens);
    const int pair0 = grp * kPairsPerThread;
    const int npairs = min(kPairsPerThread, half - pair0);
    // the token's coordinates (the packed encoding uses the row index on axis 0)
    int64_t coord3[3] = {n, 0, 0};
    if (!p.packed)
#pragma unroll
      for (int a = 0; a < 3; ++a) coord3[a] = p.coords[n * p.csn + a * p.csa];
    float cs[kPairsPerThread], sn[kPairsPerThread];
#pragma unroll
    for (int j = 0; j < kPairsPerThread; ++j) {
      cs[j] = 1.f;
      sn[j] = 0.f;
      if (j >= npairs) continue;
      const int pair = pair0 + j;
      int axis, local, start;
      if (pair < p.pairs[0]) {
        axis = 0; local = pair; start = 0;
      } else if (pair < p.pairs[0] + p.pairs[1]) {
        axis = 1; local = pair - p.pairs[0]; start = p.extent[0] * p.pairs[0];
      } else {
        axis = 2; local = pair - p.pairs[0] - p.pairs[1];
        start = p.extent[0] * p.pairs[0] + p.extent[1] * p.pairs[1];
      }
      const int64_t coord = axis == 0 ? coord3[0] : axis == 1 ? coord3[1] : coord3[2];
      if (p.phases != nullptr) {
        const float2 e = *reinterpret_cast<const float2 *>(p.phases + 2 * (start + coord * p.pairs[axis] + local));
        cs[j] = e.x;
        sn[j] = e.y;
      } else {
        const float angle = __fmul_rn((float)coord, p.freqs[pair]);
        sincosf(angle, &sn[j], &cs[j]);
      }
      if (p.inverse) sn[j] = -sn[j];
    }
    for (int h = 0; h < p.heads; ++h) {
      const T *src = static_cast<const T *>(p.x) + b * p.sb + h * p.sh + n * p.sn;
      T *dst = static_cast<T *>(p.out) + (((int64_t)b * p.heads + h) * p.tokens + n) * p.head_dim;
      float vals[2 * kPairsPerThread];
      if (kVector && npairs == kPairsPerThread) {
        // 8 contiguous, 8-element-aligned channels (checked on the host).
        if constexpr (sizeof(T) == 2) {
          const uint4 raw = *reinterpret_cast<const uint4 *>(src + 2 * pair0);
          const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
          for (int i = 0; i < 8; ++i) vals[i] = to_f32<T>(e[i]);
        } else {
          const float4 a = *reinterpret_cast<const float4 *>(src + 2 * pair0);
          const float4 c = *reinterpret_cast<const float4 *>(src + 2 * pair0 + 4);
          vals[0] = a.x; vals[1] = a.y; vals[2] = a.z; vals[3] = a.w;
          vals[4] = c.x; vals[5] = c.y; vals[6] = c.z; vals[7] = c.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 2 * kPairsPerThread; ++i)
          vals[i] = (i < 2 * npairs) ? to_f32<T>(src[(int64_t)(2 * pair0 + i) * p.sd]) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < kPairsPerThread; ++j) {
        const float even = vals[2 * j], odd = vals[2 * j + 1];
        // (even*c - odd*s, even*s + odd*c) with each product rounded: no FMA contraction.
        vals[2 * j] = __fsub_rn(__fmul_rn(even, cs[j]), __fmul_rn(odd, sn[j]));
        vals[2 * j + 1] = __fadd_rn(__fmul_rn(even, sn[j]), __fmul_rn(odd, cs[j]));
      }
      if (npairs == kPairsPerThread && sizeof(T) == 2 && ((uintptr_t)(dst + 2 * pair0) & 15) == 0) {
        uint4 raw;
        T *e = reinterpret_cast<T *>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(vals[i]);
        *reinterpret_cast<uint4 *>(dst + 2 * pair0) = raw;
      } else {
        for (int i = 0; i < 2 * npairs; ++i) dst[2 * pair0 + i] = from_f32<T>(vals[i]);
      }
    }
  }
}

template <typename T>
int launch_rope(const RopeParams &p, bool vector, cudaStream_t stream) {
  const int half = p.head_dim / 2;
  const int groups = (half + kPairsPerThread - 1) / kPairsPerThread;
  const int64_t total = (int64_t)p.batch * p.tokens * groups;
  DeviceInfo info;
  if (int st = device_info(&info)) return st;
  const int64_t want = (total + 255) / 256;
  const int blocks = (int)std::min<int64_t>(want, (int64_t)info.sm_count * 16);
  if (blocks == 0) return P3D_OK;
  // 32-bit index arithmetic while the last thread index (plus one grid stride) fits
  const bool narrow = total + (int64_t)blocks * 256 < (int64_t(1) << 31);
  if (vector)
    narrow ? rope_kernel<T, true, uint32_t><<<blocks, 256, 0, stream>>>(p)
           : rope_kernel<T, true, uint64_t><<<blocks, 256, 0, stream>>>(p);
  else
    narrow ? rope_kernel<T, false, uint32_t><<<blocks, 256, 0, stream>>>(p)
           : rope_kernel<T, false, uint64_t><<<blocks, 256, 0, stream>>>(p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

}  // namespace
}  // namespace p3d

extern "C" int p3d_rope(const void *x, int64_t sb, int64_t sh, int64_t sn, int64_t sd, void *out, int dtype,
                        int batch, int heads, int tokens, int head_dim, const int64_t *coords,
                        int64_t coord_sn, int64_t coord_sa, int pz, int py, int px, const float *freqs,
                        const float *phases, int ez, int ey, int ex, int packed, int inverse, void *stream) {
  using namespace p3d;
  P3D_CHECK_ARG(dtype_ok(dtype), "p3d_rope: unknown dtype %d", dtype);
  P3D_CHECK_ARG(batch >= 0 && heads >= 0 && tokens >= 0, "p3d_rope: negative extent");
  P3D_CHECK_ARG(head_dim > 0 && head_dim % 2 == 0, "p3d_rope: head_dim must be positive and even");
  P3D_CHECK_ARG(pz >= 0 && py >= 0 && px >= 0 && 2 * (pz + py + px) == head_dim,
                "p3d_rope: pairs (%d,%d,%d) do not allocate head_dim %d", pz, py, px, head_dim);
  P3D_CHECK_ARG(!packed || (py == 0 && px == 0), "p3d_rope: packed positions need pairs (D/2,0,0)");
  P3D_CHECK_ARG(x && out, "p3d_rope: null tensor");
  P3D_CHECK_ARG(packed || coords, "p3d_rope: coordinates required unless packed");
  P3D_CHECK_ARG(phases || freqs, "p3d_rope: need a phase table or frequencies");
  P3D_CHECK_ARG(!phases || (ez >= 0 && ey >= 0 && ex >= 0), "p3d_rope: bad table extents");
  if ((int64_t)batch * heads * tokens == 0) return P3D_OK;
  RopeParams p{};
  p.x = x; p.sb = sb; p.sh = sh; p.sn = sn; p.sd = sd; p.out = out;
  p.batch = batch; p.heads = heads; p.tokens = tokens; p.head_dim = head_dim;
  p.coords = coords; p.csn = coord_sn; p.csa = coord_sa;
  p.pairs[0] = pz; p.pairs[1] = py; p.pairs[2] = px;
  p.freqs = freqs; p.phases = phases;
  p.extent[0] = ez; p.extent[1] = ey; p.extent[2] = ex;
  p.packed = packed; p.inverse = inverse;
  const int es = dtype_size(dtype);
  const bool vector = sd == 1 && ((uintptr_t)x % 16 == 0) && (sb * es) % 16 == 0 && (sh * es) % 16 == 0 &&
                      (sn * es) % 16 == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case P3D_F16: return launch_rope<__half>(p, vector, s);
    case P3D_BF16: return launch_rope<__nv_bfloat16>(p, vector, s);
    default: return launch_rope<float>(p, vector, s);
  }
}
