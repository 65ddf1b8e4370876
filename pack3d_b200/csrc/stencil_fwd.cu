// Stage (c): fused local + global attention forward on tensor cores (tcgen05 / TMEM / TMA).
//
// Restates reference.py:20-31 (and the Triton _local_fwd/_global_fwd pair,
// kernels.py:44-103) for a complete radius-2 voxel stencil in bf16 / f16:
//   y = sl * softmax_local(q kl^T / sqrt(D)) vl + (gate * sg) * softmax_global(q sk^T / sqrt(D)) sv
//
// Work unit (one CTA): one (batch, head) and an 8x4x8 (z, y, x) box of queries,
// split into two 128-row query tiles A (z 0..3) and B (z 4..7).  Rows are ordered
// (z, y, x), so softmax warp w of a tile owns query plane z = w and TMEM lanes
// 32w..32w+31.
//
// Chunk sequence per tile (both tiles in lockstep, one shared smem ring):
//   chunks 0..7   local: halo plane z-2+c of the tile, an 8x12 (y, x) window = 96
//                 keys; a key is used iff it lies in the query's 5x5x5 cube and in
//                 the volume (coordinate test, no neighbour table).  A warp whose
//                 query plane is more than 2 planes away writes a zero P block.
//   chunks 8..    global: 128 summaries per chunk.
// Two independent online softmaxes (max / sum per row in registers, conditional
// rescale of the TMEM accumulator only when the running max grows by > 2^8),
// accumulators O_local and O_global in TMEM; the epilogue normalises both and
// writes y (and optionally ol, og, lse_l, lse_g) through the raster->packed map.
//
// Roles: warps 0-3 softmax tile A, warps 4-7 softmax tile B, warp 8 TMA producer,
// warp 9 MMA issuer (one thread).  Operands live in shared memory in the
// SWIZZLE_32B layout: Q / K are K-major boxes of 16 channels, V is the same bytes
// read MN-major; P goes back into the S columns of TMEM as bf16/f16 pairs and
// feeds the PV MMA as the TMEM A operand.  Every mbarrier wait is bounded.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace p3d {
namespace {
using namespace sm100;

__device__ unsigned g_fwd_errors = 0;  // failure bits of the kernels in this file

constexpr int kR = 2;                               // stencil radius handled here
constexpr int kTZ = 4, kTY = 4, kTX = 8;            // one 128-row query tile
constexpr int kHY = kTY + 2 * kR, kHX = kTX + 2 * kR, kHZ = kTZ + 2 * kR;
constexpr int kPlane = kHY * kHX;                   // 96 keys per halo plane
constexpr int kLocalChunks = kHZ;                   // 8 halo planes per tile
constexpr int kSumRows = 128;                       // summaries per global chunk
constexpr int kRows = 128;                          // queries per tile
constexpr int kThreads = 320;
constexpr int kProducerWarp = 8, kMmaWarp = 9;
constexpr uint32_t kTmemCols = 512;
constexpr float kNegInf = -__builtin_huge_valf();

static_assert(kPlane % 16 == 0, "halo plane must be a multiple of the MMA K step");

template <int D>
struct Cfg {
  static constexpr int kK = D / 16;                 // 16-channel boxes per row
  static constexpr int kBoxQ = kRows * 32;          // one box = rows x 32 bytes
  static constexpr int kBoxP = kPlane * 32;
  static constexpr int kBoxS = kSumRows * 32;
  static constexpr int kQBytes = kK * kBoxQ;        // one query tile
  static constexpr int kPlaneBytes = kK * kBoxP;    // one halo plane of K (or V)
  static constexpr int kSumBytes = kK * kBoxS;      // one summary chunk of K (or V)
  static constexpr int kStageRaw = (4 * kPlaneBytes > 2 * kSumBytes) ? 4 * kPlaneBytes : 2 * kSumBytes;
  static constexpr int kStageBytes = (kStageRaw + 1023) / 1024 * 1024;
  static constexpr int kStages = D <= 48 ? 4 : 3;
  // + alignment slack; at least 116 KB so that one CTA (which owns all 512 TMEM columns) fits per SM
  static constexpr int kSmemNeed = 2 * kQBytes + kStages * kStageBytes + 1024;
  static constexpr int kSmemBytes = kSmemNeed > 116 * 1024 ? kSmemNeed : 116 * 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// TMEM columns of tile t: S/P [t*256, +128), O_global [+128, +D), O_local [+192, +D).
constexpr uint32_t kColS = 0, kColOg = 128, kColOl = 192;

enum Bar { kQFull = 0, kFull = 1, kEmpty = 5, kSReady = 9, kPReady = 11, kPvDone = 13, kOReady = 15, kNumBars = 17 };

struct FwdParams {
  int Z, Y, X, tiles_z, tiles_y, tiles_x;
  int heads, kv_heads, summaries, global_chunks;
  int64_t tokens;
  float sc;          // log2(e) / sqrt(D): scores -> exp2 domain
  float inv_sqrt_d;
  const void *gate;
  int gate_dtype;
  const float *sl, *sg;
  const int32_t *map;  // raster -> packed rows (nullptr: raster storage)
  void *y, *ol, *og;
  float *lse_l, *lse_g;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return BF16 ? pack_bf16(lo, hi) : pack_f16(lo, hi);
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  if constexpr (BF16) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162 *>(&v);
    return __bfloat1622float2(h);
  } else {
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
  }
}

// Online-softmax bookkeeping of one branch for one row.  Rescales the TMEM
// accumulator only when some row of the warp raised its max by more than 2^8.
template <int D>
__device__ __forceinline__ void update_max(float &m, float &l, float mx, float sc, uint32_t t_o) {
  const float m_new = fmaxf(m, mx);
  const bool first = (m == kNegInf);
  const bool need = !first && (m_new - m) * sc > 8.f;
  if (first) m = m_new;
  if (__any_sync(0xffffffffu, need)) {
    const float factor = need ? ex2_approx((m - m_new) * sc) : 1.f;
    uint32_t o[16];
#pragma unroll
    for (int c = 0; c < D / 16; ++c) {
      tmem_ld16(t_o + 16 * c, o);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
      tmem_st16(t_o + 16 * c, o);
    }
    if (need) {
      l *= factor;
      m = m_new;
    }
  }
}

// Exponentiate `n` scores (in registers) against max m, pack to 16-bit pairs and store
// them as P into TMEM columns [t_p, t_p + n/2).  Returns the row sum of p.
template <int N, bool BF16>
__device__ __forceinline__ float exp_store(const float *s, float m, float sc, uint32_t t_p) {
  const float msc = (m == kNegInf) ? 0.f : m * sc;
  float sum = 0.f;
#pragma unroll
  for (int g = 0; g < N / 32; ++g) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float p0 = ex2_approx(fmaf(s[32 * g + 2 * i], sc, -msc));
      const float p1 = ex2_approx(fmaf(s[32 * g + 2 * i + 1], sc, -msc));
      sum += p0 + p1;
      pk[i] = pack2<BF16>(p0, p1);
    }
    tmem_st16(t_p + 16 * g, pk);
  }
  return sum;
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    stencil_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkl,
                       const __grid_constant__ CUtensorMap tvl, const __grid_constant__ CUtensorMap tsk,
                       const __grid_constant__ CUtensorMap tsv, const FwdParams p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kNumBars];
  __shared__ uint32_t tmem_holder;
  __shared__ float s_sl[D], s_sg[D];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // ---- work unit
  int unit = blockIdx.x;
  const int tx = unit % p.tiles_x;
  unit /= p.tiles_x;
  const int ty = unit % p.tiles_y;
  unit /= p.tiles_y;
  const int tz = unit % p.tiles_z;
  const int bh = unit / p.tiles_z;
  const int x0 = tx * kTX, y0 = ty * kTY, z0 = tz * 2 * kTZ;
  const int b = bh / p.heads, h = bh % p.heads;
  const int bg = b * p.kv_heads + h / (p.heads / p.kv_heads);
  const int n_chunks = kLocalChunks + p.global_chunks;

  // ---- shared memory carve-up (1024-byte aligned)
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t q_smem = base;                        // tile A, then tile B
  const uint32_t ring = base + 2 * C::kQBytes;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (tid == 0) {
    mbar_init(bar(kQFull), 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar(kFull + s), 1);
      mbar_init(bar(kEmpty + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kSReady + t), 1);
      mbar_init(bar(kPReady + t), 4);
      mbar_init(bar(kPvDone + t), 1);
      mbar_init(bar(kOReady + t), 1);
    }
    fence_mbar_init();
  }
  for (int i = tid; i < D; i += kThreads) {
    s_sl[i] = p.sl[i];
    s_sg[i] = p.sg[i];
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tq);
    prefetch_tmap(&tkl);
    prefetch_tmap(&tvl);
    prefetch_tmap(&tsk);
    prefetch_tmap(&tsv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(bar(kQFull), 2 * C::kQBytes);
      for (int t = 0; t < 2; ++t)
        for (int c = 0; c < C::kK; ++c)
          tma_load_5d(q_smem + t * C::kQBytes + c * C::kBoxQ, &tq, bar(kQFull), 16 * c, x0, y0, z0 + kTZ * t, bh);
      for (int ch = 0; ch < n_chunks; ++ch) {
        const int s = ch % C::kStages;
        if (ch >= C::kStages && !mbar_wait(bar(kEmpty + s), ((ch / C::kStages) + 1) & 1, &g_fwd_errors)) break;
        const uint32_t stage = ring + s * C::kStageBytes;
        const uint32_t full = bar(kFull + s);
        if (ch < kLocalChunks) {
          mbar_expect_tx(full, 4 * C::kPlaneBytes);
          for (int t = 0; t < 2; ++t) {
            const int z = z0 + kTZ * t - kR + ch;
            for (int c = 0; c < C::kK; ++c) {
              tma_load_5d(stage + t * C::kPlaneBytes + c * C::kBoxP, &tkl, full, 16 * c, x0 - kR, y0 - kR, z, bg);
              tma_load_5d(stage + (2 + t) * C::kPlaneBytes + c * C::kBoxP, &tvl, full, 16 * c, x0 - kR, y0 - kR, z,
                          bg);
            }
          }
        } else {
          const int g = ch - kLocalChunks;
          mbar_expect_tx(full, 2 * C::kSumBytes);
          for (int c = 0; c < C::kK; ++c) {
            tma_load_3d(stage + c * C::kBoxS, &tsk, full, 16 * c, g * kSumRows, bg);
            tma_load_3d(stage + C::kSumBytes + c * C::kBoxS, &tsv, full, 16 * c, g * kSumRows, bg);
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_local = idesc_f16(128, kPlane, BF16, false);
      constexpr uint32_t idesc_global = idesc_f16(128, kSumRows, BF16, false);
      constexpr uint32_t idesc_pv = idesc_f16(128, D, BF16, true);
      bool ok = mbar_wait(bar(kQFull), 0, &g_fwd_errors);
      for (int ch = 0; ok && ch <= n_chunks; ++ch) {
        if (ch < n_chunks) {
          ok = mbar_wait(bar(kFull + ch % C::kStages), (ch / C::kStages) & 1, &g_fwd_errors);
          if (!ok) break;
          tc_fence_after();
        }
        for (int t = 0; t < 2 && ok; ++t) {
          const uint32_t t_s = tmem + t * 256 + kColS;
          if (ch > 0) {
            // O_t += P_t(ch-1) V(ch-1)
            const int c = ch - 1;
            ok = mbar_wait(bar(kPReady + t), c & 1, &g_fwd_errors);
            if (!ok) break;
            tc_fence_after();
            const uint32_t stage = ring + (c % C::kStages) * C::kStageBytes;
            const bool local = c < kLocalChunks;
            const uint32_t v_base = local ? stage + (2 + t) * C::kPlaneBytes : stage + C::kSumBytes;
            const uint32_t lbo = local ? C::kBoxP : C::kBoxS;
            const int ksteps = (local ? kPlane : kSumRows) / 16;
            const uint32_t t_o = tmem + t * 256 + (local ? kColOl : kColOg);
            const bool first = (c == 0) || (c == kLocalChunks);
            for (int j = 0; j < ksteps; ++j)
              mma_ts(t_o, t_s + 8 * j, desc_sw32(v_base + j * 512, lbo, 256), idesc_pv, (first && j == 0) ? 0u : 1u);
            if (ch == n_chunks) {
              mma_commit(bar(kOReady + t));
            } else {
              // S(ch) overwrites the P(ch-1) columns: wait until the PV MMA has read them.
              mma_commit(bar(kPvDone + t));
              ok = mbar_wait(bar(kPvDone + t), c & 1, &g_fwd_errors);
              if (!ok) break;
            }
          }
          if (ch < n_chunks) {
            // S_t = Q_t K(ch)^T
            const uint32_t stage = ring + (ch % C::kStages) * C::kStageBytes;
            const bool local = ch < kLocalChunks;
            const uint32_t k_base = local ? stage + t * C::kPlaneBytes : stage;
            const uint32_t box = local ? C::kBoxP : C::kBoxS;
            const uint32_t idesc = local ? idesc_local : idesc_global;
            const uint32_t q_t = q_smem + t * C::kQBytes;
            for (int c = 0; c < C::kK; ++c)
              mma_ss(t_s, desc_sw32(q_t + c * C::kBoxQ, 16, 256), desc_sw32(k_base + c * box, 16, 256), idesc,
                     c > 0 ? 1u : 0u);
            mma_commit(bar(kSReady + t));
          }
        }
        if (ok && ch > 0 && ch < n_chunks) mma_commit(bar(kEmpty + (ch - 1) % C::kStages));
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2, w = warp & 3;
    const uint32_t lanes = (uint32_t)(w * 32) << 16;
    const uint32_t t_s = tmem + lanes + t * 256 + kColS;
    const uint32_t t_og = tmem + lanes + t * 256 + kColOg;
    const uint32_t t_ol = tmem + lanes + t * 256 + kColOl;
    const int qz = w, qy = lane >> 3, qx = lane & 7;
    const int zq = z0 + kTZ * t + qz, yq = y0 + qy, xq = x0 + qx;
    const bool row_ok = zq < p.Z && yq < p.Y && xq < p.X;
    uint32_t mask[3] = {0u, 0u, 0u};
#pragma unroll
    for (int hy = 0; hy < kHY; ++hy) {
#pragma unroll
      for (int hx = 0; hx < kHX; ++hx) {
        const int c = hy * kHX + hx, yy = y0 - kR + hy, xx = x0 - kR + hx;
        const bool in = (unsigned)(hy - qy) <= 2u * kR && (unsigned)(hx - qx) <= 2u * kR && yy >= 0 && yy < p.Y &&
                        xx >= 0 && xx < p.X;
        if (in) mask[c >> 5] |= 1u << (c & 31);
      }
    }
    const float sc = p.sc;
    float m_l = kNegInf, l_l = 0.f, m_g = kNegInf, l_g = 0.f;
    bool ok = true;
    for (int ch = 0; ch < n_chunks; ++ch) {
      ok = mbar_wait(bar(kSReady + t), ch & 1, &g_fwd_errors);
      if (!ok) break;
      tc_fence_after();
      if (ch < kLocalChunks) {
        const int zp = z0 + kTZ * t - kR + ch;
        const bool need = (unsigned)(ch - qz) <= 2u * kR && zp >= 0 && zp < p.Z;  // warp-uniform
        if (need) {
          float s[kPlane];
#pragma unroll
          for (int g = 0; g < kPlane / 32; ++g) tmem_ld32(t_s + 32 * g, reinterpret_cast<uint32_t *>(s + 32 * g));
          tmem_wait_ld();
          float mx = kNegInf;
#pragma unroll
          for (int i = 0; i < kPlane; ++i) {
            s[i] = (mask[i >> 5] >> (i & 31)) & 1u ? s[i] : kNegInf;
            mx = fmaxf(mx, s[i]);
          }
          update_max<D>(m_l, l_l, mx, sc, t_ol);
          l_l += exp_store<kPlane, BF16>(s, m_l, sc, t_s);
        } else {
          uint32_t zero[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) zero[i] = 0u;
#pragma unroll
          for (int g = 0; g < kPlane / 32; ++g) tmem_st16(t_s + 16 * g, zero);
        }
      } else {
        const int g0 = (ch - kLocalChunks) * kSumRows;
        const int valid = min(kSumRows, p.summaries - g0);
        float s[kSumRows];
#pragma unroll
        for (int g = 0; g < kSumRows / 32; ++g) tmem_ld32(t_s + 32 * g, reinterpret_cast<uint32_t *>(s + 32 * g));
        tmem_wait_ld();
        float mx = kNegInf;
        if (valid == kSumRows) {
#pragma unroll
          for (int i = 0; i < kSumRows; ++i) mx = fmaxf(mx, s[i]);
        } else {
#pragma unroll
          for (int i = 0; i < kSumRows; ++i) {
            s[i] = i < valid ? s[i] : kNegInf;
            mx = fmaxf(mx, s[i]);
          }
        }
        update_max<D>(m_g, l_g, mx, sc, t_og);
        l_g += exp_store<kSumRows, BF16>(s, m_g, sc, t_s);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kPReady + t));
    }
    // ---- epilogue: normalise both branches, mix, store through the row map
    if (ok) ok = mbar_wait(bar(kOReady + t), 0, &g_fwd_errors);
    if (ok) {
      tc_fence_after();
      uint32_t ol[D], og[D];
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        tmem_ld16(t_ol + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(ol + 16 * c));
        tmem_ld16(t_og + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(og + 16 * c));
      }
      tmem_wait_ld();
      if (row_ok) {
        int64_t rr = ((int64_t)zq * p.Y + yq) * p.X + xq;
        if (p.map) rr = p.map[rr];
        const int64_t row = (int64_t)bh * p.tokens + rr;
        const float gate = load_any(p.gate, p.gate_dtype, row);
        const float inv_l = l_l > 0.f ? 1.f / l_l : 0.f;
        const float inv_g = 1.f / l_g;
        uint32_t packed_y[D / 2], packed_l[D / 2], packed_g[D / 2];
#pragma unroll
        for (int i = 0; i < D / 2; ++i) {
          float yv[2], lv[2], gv[2];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int d = 2 * i + k;
            lv[k] = __uint_as_float(ol[d]) * inv_l;
            gv[k] = __uint_as_float(og[d]) * inv_g;
            yv[k] = __fadd_rn(__fmul_rn(s_sl[d], lv[k]), __fmul_rn(__fmul_rn(gate, s_sg[d]), gv[k]));
          }
          packed_y[i] = pack2<BF16>(yv[0], yv[1]);
          packed_l[i] = pack2<BF16>(lv[0], lv[1]);
          packed_g[i] = pack2<BF16>(gv[0], gv[1]);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.y) + row * D);
#pragma unroll
        for (int v = 0; v < D / 8; ++v)
          dst[v] = make_uint4(packed_y[4 * v], packed_y[4 * v + 1], packed_y[4 * v + 2], packed_y[4 * v + 3]);
        if (p.ol) {
          uint4 *dl = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.ol) + row * D);
          uint4 *dg = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.og) + row * D);
#pragma unroll
          for (int v = 0; v < D / 8; ++v) {
            dl[v] = make_uint4(packed_l[4 * v], packed_l[4 * v + 1], packed_l[4 * v + 2], packed_l[4 * v + 3]);
            dg[v] = make_uint4(packed_g[4 * v], packed_g[4 * v + 1], packed_g[4 * v + 2], packed_g[4 * v + 3]);
          }
          p.lse_l[row] = m_l * p.inv_sqrt_d + logf(l_l);
          p.lse_g[row] = m_g * p.inv_sqrt_d + logf(l_g);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------- host side

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
  });
  return fn;
}

int encode(CUtensorMap *map, int dtype, const void *ptr, int rank, const uint64_t *dims, const uint64_t *strides,
           const uint32_t *box) {
  EncodeTiled fn = encode_fn();
  if (!fn) return fail(P3D_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t elem[5] = {1, 1, 1, 1, 1};
  const CUresult r = fn(map, dtype == P3D_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        rank, const_cast<void *>(ptr), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(P3D_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return P3D_OK;
}

template <int D, bool BF16>
int launch_t(const StencilFwdArgs &a, cudaStream_t stream) {
  using C = Cfg<D>;
  const int Z = a.grid[0], Y = a.grid[1], X = a.grid[2];
  const uint64_t es = 2;
  const uint64_t bh = (uint64_t)a.batch * a.heads, bgs = (uint64_t)a.batch * a.kv_heads;
  CUtensorMap tq, tkl, tvl, tsk, tsv;
  {
    const uint64_t dims[5] = {(uint64_t)D, (uint64_t)X, (uint64_t)Y, (uint64_t)Z, bh};
    const uint64_t strides[4] = {D * es, X * D * es, (uint64_t)Y * X * D * es, (uint64_t)Z * Y * X * D * es};
    const uint32_t box[5] = {16, kTX, kTY, kTZ, 1};
    if (int st = encode(&tq, a.dtype, a.q, 5, dims, strides, box)) return st;
  }
  {
    const uint64_t dims[5] = {(uint64_t)D, (uint64_t)X, (uint64_t)Y, (uint64_t)Z, bgs};
    const uint64_t strides[4] = {D * es, X * D * es, (uint64_t)Y * X * D * es, (uint64_t)Z * Y * X * D * es};
    const uint32_t box[5] = {16, kHX, kHY, 1, 1};
    if (int st = encode(&tkl, a.dtype, a.kl, 5, dims, strides, box)) return st;
    if (int st = encode(&tvl, a.dtype, a.vl, 5, dims, strides, box)) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)a.summaries, bgs};
    const uint64_t strides[2] = {D * es, (uint64_t)a.summaries * D * es};
    const uint32_t box[3] = {16, kSumRows, 1};
    if (int st = encode(&tsk, a.dtype, a.sk, 3, dims, strides, box)) return st;
    if (int st = encode(&tsv, a.dtype, a.sv, 3, dims, strides, box)) return st;
  }
  FwdParams p{};
  p.Z = Z;
  p.Y = Y;
  p.X = X;
  p.tiles_z = (Z + 2 * kTZ - 1) / (2 * kTZ);
  p.tiles_y = (Y + kTY - 1) / kTY;
  p.tiles_x = (X + kTX - 1) / kTX;
  p.heads = a.heads;
  p.kv_heads = a.kv_heads;
  p.summaries = a.summaries;
  p.global_chunks = (a.summaries + kSumRows - 1) / kSumRows;
  p.tokens = (int64_t)Z * Y * X;
  p.sc = 1.4426950408889634f / sqrtf((float)D);
  p.inv_sqrt_d = 1.f / sqrtf((float)D);
  p.gate = a.gate;
  p.gate_dtype = a.gate_dtype;
  p.sl = a.sl;
  p.sg = a.sg;
  p.map = a.raster_to_packed;
  p.y = a.y;
  p.ol = a.ol;
  p.og = a.og;
  p.lse_l = a.lse_l;
  p.lse_g = a.lse_g;
  const int64_t units = (int64_t)bh * p.tiles_z * p.tiles_y * p.tiles_x;
  if (units <= 0) return P3D_OK;
  if (units > 0x7fffffff) return fail(P3D_ERR_UNSUPPORTED, "too many tiles");
  auto kernel = stencil_fwd_kernel<D, BF16>;
  static bool configured = false;
  if (!configured) {
    P3D_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    configured = true;
  }
  kernel<<<(unsigned)units, kThreads, C::kSmemBytes, stream>>>(tq, tkl, tvl, tsk, tsv, p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

}  // namespace

bool stencil_fwd_supported(int dtype, int head_dim, const int radius[3], int summaries) {
  if (dtype != P3D_BF16 && dtype != P3D_F16) return false;
  if (head_dim != 16 && head_dim != 32 && head_dim != 48 && head_dim != 64) return false;
  if (radius[0] != kR || radius[1] != kR || radius[2] != kR) return false;
  if (summaries < 1) return false;
  DeviceInfo info;
  if (device_info(&info) != P3D_OK || info.major != 10) return false;
  return true;
}

int launch_stencil_fwd(const StencilFwdArgs &a, cudaStream_t s) {
  const bool bf16 = a.dtype == P3D_BF16;
  switch (a.head_dim) {
    case 16: return bf16 ? launch_t<16, true>(a, s) : launch_t<16, false>(a, s);
    case 32: return bf16 ? launch_t<32, true>(a, s) : launch_t<32, false>(a, s);
    case 48: return bf16 ? launch_t<48, true>(a, s) : launch_t<48, false>(a, s);
    case 64: return bf16 ? launch_t<64, true>(a, s) : launch_t<64, false>(a, s);
    default: return fail(P3D_ERR_UNSUPPORTED, "stencil forward: head_dim %d", a.head_dim);
  }
}

}  // namespace p3d

namespace p3d {
int take_fwd_errors(unsigned *flags) {
  unsigned v = 0, zero = 0;
  P3D_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_fwd_errors, sizeof(v)));
  P3D_CUDA_TRY(cudaMemcpyToSymbol(g_fwd_errors, &zero, sizeof(zero)));
  *flags |= v;
  return P3D_OK;
}
}  // namespace p3d
