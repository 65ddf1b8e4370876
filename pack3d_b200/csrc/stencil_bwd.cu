// Stage (d), query side: dQ of the fused local + global attention on tensor cores.
//
// Restates the query-gradient half of the reference backward (kernels.py:131-150 local,
// :180-206 global; stencil.py:91-147 for the spatial local form) for a complete radius-1
// or radius-2 voxel stencil in bf16 / f16.  With P recomputed from the saved logsumexp,
//   dS = P * (dO V^T - Delta) / sqrt(D),   dQ = dS K
// per branch (local: dO = dO_l, K/V = the 3x3x3 or 5x5x5 neighbours; global: dO = dO_g, K/V = all
// summaries).  dS is rounded to the storage dtype before the product (the reference does
// the same for the global branch, kernels.py:197); here the rounded operand is P (dP -
// Delta) and the 1/sqrt(D) is applied once to the fp32 dQ accumulator (one multiply per
// output instead of one per score; the rounding is relative, so the result agrees within
// the dtype's rounding).  The two branch gradients are each rounded, then added and
// rounded again (kernels.py:202-206).
//
// Work unit and chunk sequence are those of the forward kernel (stencil_fwd.cu): one
// (batch, head) and a 4x4x8 tile of 128 queries per CTA, two CTAs per SM; 8 local chunks
// (halo planes of an 8x12 window) then ceil(M/96) global chunks at radius 2; 6 planes of a
// 6x10 window padded to 64 keys, and 64-summary chunks, at radius 1 (BGeo).  TMEM (256
// columns) holds S [0, W), dP [W, 2W) and the dQ accumulator [2W, 2W + D), W the chunk
// width (96 or 64).  Per chunk the MMA thread
// issues S = Q K^T and dP = dO V^T; the softmax warps turn them into dS, written back as
// 16-bit pairs over the first W/2 dP columns, and the MMA thread accumulates dQ += dS K with
// dS as the TMEM A operand and the K chunk (already in shared memory for S) read MN-major
// as B.  S of the next chunk is issued as soon as the softmax warps have released this
// chunk, while dQ of this chunk runs; dP of the next chunk waits for dQ to finish reading
// dS.
//
// Roles: warps 0-3 softmax, warp 4 TMA producer, warp 5 MMA issuer.  Every
// mbarrier wait is bounded and every parity wait is unambiguous: each barrier completes
// once per chunk (the ring's release barriers once per stage use) and each waiter awaits
// its completions in order, its next completion needing the waiter's own next step.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace p3d {
namespace {
using namespace sm100;

__device__ unsigned g_bwd_errors = 0;  // failure bits of the kernels in this file

constexpr int kTZ = 4, kTY = 4, kTX = 8;
constexpr int kRows = 128;

// Chunk geometry of a radius-R stencil (R = 1 or 2), as in the forward kernel: a halo plane
// of a 4x4x8 tile is a kHY x kHX window of kWin keys (or queries), padded to kKeys (a
// multiple of 32); the padding rows of the ring are zero and masked.
template <int R>
struct BGeo {
  static constexpr int kR = R;
  static constexpr int kHY = kTY + 2 * R, kHX = kTX + 2 * R, kHZ = kTZ + 2 * R;
  static constexpr int kWin = kHY * kHX;                // 96 (R = 2), 60 (R = 1)
  static constexpr int kKeys = (kWin + 31) / 32 * 32;   // 96, 64
  static constexpr int kLocalChunks = kHZ;              // 8, 6
  static constexpr int kSumRows = kKeys;
  static constexpr int kHalf = kKeys / 2;               // query columns per softmax warp (dK / dV)
  static_assert(kKeys % 32 == 0 && kHalf % 16 == 0, "chunk width must suit the MMA and TMEM shapes");
};
constexpr int kThreads = 320;
constexpr int kProducerWarp = 8, kMmaWarp = 9;
constexpr uint32_t kTmemCols = 512;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr float kLog2e = 1.4426950408889634f;

constexpr int kDqThreads = 192;                   // one tile per CTA, two CTAs per SM
constexpr int kDqProducerWarp = 4, kDqMmaWarp = 5;
constexpr uint32_t kDqTmemCols = 256;

template <int D, int KEYS>
struct DqCfg {
  static constexpr int kK = D / 16;
  static constexpr int kBoxQ = kRows * 32;
  static constexpr int kBoxK = KEYS * 32;
  static constexpr int kQBytes = kK * kBoxQ;      // the 128-row tile of Q, dO_l or dO_g
  static constexpr int kKeyBytes = kK * kBoxK;    // one chunk of K or V
  static constexpr int kStageBytes = (2 * kKeyBytes + 1023) / 1024 * 1024;
  static constexpr int kParkBytes = kRows * D * 2;
  static constexpr int kFixed = 3 * kQBytes + kParkBytes + 1024;
  // two CTAs per SM (<= 113 KB each), never three (> 76 KB: a third CTA's TMEM
  // allocation would have to wait)
  static constexpr int kMaxSmem = 113 * 1024, kMinSmem = 78 * 1024;
  static constexpr int kRoom = (kMaxSmem - kFixed) / kStageBytes;
  static constexpr int kStages = kRoom > 4 ? 4 : kRoom;
  static constexpr int kSmemNeed = kFixed + kStages * kStageBytes;
  static constexpr int kSmemBytes = kSmemNeed > kMinSmem ? kSmemNeed : kMinSmem;
  static_assert(kStages >= 2, "the ring must hold two chunks");
  static_assert(kSmemBytes <= kMaxSmem, "shared memory budget");
};

enum DqBar {
  kQFull = 0,
  kFull = 1,                 // [stage]
  kEmpty = kFull + 4,        // [stage]: arrived by the MMA thread once dQ of the chunk it held completed
  kSReady = kEmpty + 4,      // S(c) complete
  kSFree = kSReady + 1,      // the 4 softmax warps hold S(c) in registers (count 4)
  kDPReady = kSFree + 1,     // dP(c) complete
  kDSReady = kDPReady + 1,   // the 4 softmax warps stored dS(c) (count 4)
  kDQDone = kDSReady + 1,    // dQ(c) complete
  kDrain = kDQDone + 1,
  kNumBars = kDrain + 1
};

struct DqParams {
  int Z, Y, X, tiles_z, tiles_y, tiles_x;  // Z: planes of the query (centre) buffer
  int Zg, qz0, kz0;  // global planes; global z of query-buffer plane 0 and of K/V-buffer plane 0
  int heads, kv_heads, summaries, global_chunks;
  int64_t tokens;
  float sc;        // log2(e) / sqrt(D)
  float inv_sqrt_d;
  const float *lse_l, *lse_g, *delta_l, *delta_g;  // [B*H, N] in the layout's row order
  const int32_t *map;                               // raster -> packed rows (nullptr: raster)
  void *dq;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return BF16 ? pack_bf16(lo, hi) : pack_f16(lo, hi);
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  if constexpr (BF16) {  // exact: the bf16 bit patterns shifted into fp32 position
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  } else {
    return __half22float2(*reinterpret_cast<const __half2 *>(&v));
  }
}

template <bool BF16>
__device__ __forceinline__ float round_storage(float v) {
  const float2 r = unpack2<BF16>(pack2<BF16>(v, 0.f));
  return r.x;
}

template <int D, bool BF16, int R>
__global__ void __launch_bounds__(kDqThreads, 2)
    stencil_bwd_dq_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdol,
                          const __grid_constant__ CUtensorMap tdog, const __grid_constant__ CUtensorMap tkl,
                          const __grid_constant__ CUtensorMap tvl, const __grid_constant__ CUtensorMap tsk,
                          const __grid_constant__ CUtensorMap tsv, const DqParams p) {
  using G = BGeo<R>;
  constexpr int kR = G::kR, kHY = G::kHY, kHX = G::kHX, kWin = G::kWin, kKeys = G::kKeys;
  constexpr int kLocalChunks = G::kLocalChunks, kSumRows = G::kSumRows;
  // TMEM: S [0, kKeys), dP [kKeys, 2 kKeys) (dS written back over its first half), dQ after
  constexpr uint32_t kColS = 0, kColDP = kKeys, kColDQ = 2 * kKeys;
  using C = DqCfg<D, kKeys>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kNumBars];
  __shared__ uint32_t tmem_holder;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int unit = blockIdx.x;
  const int tx = unit % p.tiles_x;
  unit /= p.tiles_x;
  const int ty = unit % p.tiles_y;
  unit /= p.tiles_y;
  const int tz = unit % p.tiles_z;
  const int bh = unit / p.tiles_z;
  const int x0 = tx * kTX, y0 = ty * kTY, z0 = tz * kTZ;
  const int b = bh / p.heads, h = bh % p.heads;
  const int bg = b * p.kv_heads + h / (p.heads / p.kv_heads);
  const int n_chunks = kLocalChunks + p.global_chunks;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t q_smem = base;                     // Q
  const uint32_t dol_smem = base + C::kQBytes;      // dO_l
  const uint32_t dog_smem = base + 2 * C::kQBytes;  // dO_g
  const uint32_t ring = base + 3 * C::kQBytes;
  uint8_t *park_base = smem_raw + (base - raw) + 3 * C::kQBytes + C::kStages * C::kStageBytes;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (tid == 0) {
    mbar_init(bar(kQFull), 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar(kFull + s), 1);
      mbar_init(bar(kEmpty + s), 1);
    }
    mbar_init(bar(kSReady), 1);
    mbar_init(bar(kSFree), 4);
    mbar_init(bar(kDPReady), 1);
    mbar_init(bar(kDSReady), 4);
    mbar_init(bar(kDQDone), 1);
    mbar_init(bar(kDrain), 1);
    fence_mbar_init();
  }
  if constexpr (kWin < kKeys) {
    // local chunks fill kWin of the kKeys rows of each box: the rest reads as zeros (see the
    // forward kernel) until a global chunk reuses the stage
    uint4 *ring_v = reinterpret_cast<uint4 *>(smem_raw + (base - raw) + 3 * C::kQBytes);
    for (int i = tid; i < C::kStages * C::kStageBytes / 16; i += kDqThreads) ring_v[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (warp == kDqMmaWarp) {
    tmem_alloc(smem_u32(&tmem_holder), kDqTmemCols);
    tmem_relinquish();
  }
  if (warp == kDqProducerWarp && lane == 0) {
    prefetch_tmap(&tq);
    prefetch_tmap(&tdol);
    prefetch_tmap(&tdog);
    prefetch_tmap(&tkl);
    prefetch_tmap(&tvl);
    prefetch_tmap(&tsk);
    prefetch_tmap(&tsv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;

  if (warp == kDqProducerWarp) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(bar(kQFull), 3 * C::kQBytes);
      for (int c = 0; c < C::kK; ++c) {
        tma_load_5d(q_smem + c * C::kBoxQ, &tq, bar(kQFull), 16 * c, x0, y0, z0, bh);
        tma_load_5d(dol_smem + c * C::kBoxQ, &tdol, bar(kQFull), 16 * c, x0, y0, z0, bh);
        tma_load_5d(dog_smem + c * C::kBoxQ, &tdog, bar(kQFull), 16 * c, x0, y0, z0, bh);
      }
      int issued = 0;
      for (int ch = 0; ch < n_chunks; ++ch) {
        const int s = ch % C::kStages;
        // kEmpty[s] completes once per use of stage s: this is completion ch/kStages - 1.
        // Completion - 1 was awaited here a ring turn ago (or this is the first), and
        // completion + 1 needs chunk ch, which is not loaded yet.
        if (ch >= C::kStages &&
            !mbar_wait(bar(kEmpty + s), (ch / C::kStages - 1) & 1, &g_bwd_errors, kWaitNs, kErrProducer))
          break;
        const uint32_t stage = ring + s * C::kStageBytes;
        const uint32_t full = bar(kFull + s);
        mbar_expect_tx(full, ch < kLocalChunks ? 2 * C::kK * kWin * 32 : 2 * C::kKeyBytes);
        if (ch < kLocalChunks) {
          const int z = p.qz0 + z0 - kR + ch - p.kz0;  // plane in the K/V buffer
          for (int c = 0; c < C::kK; ++c) {
            tma_load_5d(stage + c * C::kBoxK, &tkl, full, 16 * c, x0 - kR, y0 - kR, z, bg);
            tma_load_5d(stage + C::kKeyBytes + c * C::kBoxK, &tvl, full, 16 * c, x0 - kR, y0 - kR, z, bg);
          }
        } else {
          const int g = ch - kLocalChunks;
          for (int c = 0; c < C::kK; ++c) {
            tma_load_3d(stage + c * C::kBoxK, &tsk, full, 16 * c, g * kSumRows, bg);
            tma_load_3d(stage + C::kKeyBytes + c * C::kBoxK, &tsv, full, 16 * c, g * kSumRows, bg);
          }
        }
        issued = ch + 1;
      }
      mbar_wait(bar(kQFull), 0, &g_bwd_errors, kWaitNs, kErrTeardown);
      for (int ch = issued > C::kStages ? issued - C::kStages : 0; ch < issued; ++ch)
        mbar_wait(bar(kFull + ch % C::kStages), (ch / C::kStages) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
    }
  } else if (warp == kDqMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(128, kKeys, BF16, false);  // S and dP: N = kKeys, K-major B
      constexpr uint32_t idesc_dq = idesc_f16(128, D, BF16, true);     // dQ: N = D, B = K read MN-major
      uint32_t commits[kNumBars];
      for (int i = 0; i < kNumBars; ++i) commits[i] = 0u;
      auto commit = [&](int bidx) {
        mma_commit(bar(bidx));
        ++commits[bidx];
      };
      const uint64_t desc_q = desc_sw32(q_smem, 16, 256);
      const uint64_t desc_dol = desc_sw32(dol_smem, 16, 256), desc_dog = desc_sw32(dog_smem, 16, 256);
      const uint64_t desc_k = desc_sw32(ring, 16, 256);          // K / V chunks, K-major
      const uint64_t desc_kmn = desc_sw32(ring, C::kBoxK, 256);  // K chunks read MN-major
      auto stage_off = [&](int c) { return (uint32_t)((c % C::kStages) * C::kStageBytes) >> 4; };
      auto issue_s = [&](int c) {
        const uint64_t bk = desc_k + stage_off(c);
#pragma unroll
        for (int kk = 0; kk < C::kK; ++kk)
          mma_ss(tmem + kColS, desc_q + kk * (C::kBoxQ >> 4), bk + kk * (C::kBoxK >> 4), idesc_s, kk > 0 ? 1u : 0u);
        commit(kSReady);
      };
      auto issue_dp = [&](int c) {
        const uint64_t ad = c < kLocalChunks ? desc_dol : desc_dog;
        const uint64_t bv = desc_k + stage_off(c) + (C::kKeyBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < C::kK; ++kk)
          mma_ss(tmem + kColDP, ad + kk * (C::kBoxQ >> 4), bv + kk * (C::kBoxK >> 4), idesc_s, kk > 0 ? 1u : 0u);
        commit(kDPReady);
      };
      auto issue_dq = [&](int c) {
        const uint64_t bk = desc_kmn + stage_off(c);
        const bool first = (c == 0) || (c == kLocalChunks);  // dQ restarts for the global branch
#pragma unroll
        for (int j = 0; j < kKeys / 16; ++j)
          mma_ts(tmem + kColDQ, tmem + kColDP + 8 * j, bk + j * (512 >> 4), idesc_dq, (first && j == 0) ? 0u : 1u);
        commit(kDQDone);
      };
      auto wait_bar = [&](int bidx, int completion) -> bool {
        if (!mbar_wait(bar(bidx), completion & 1, &g_bwd_errors, kWaitNs, kErrMma)) return false;
        tc_fence_after();
        return true;
      };
      auto wait_full = [&](int c) { return wait_bar(kFull + c % C::kStages, c / C::kStages); };
      // Prologue: S and dP of chunk 0.  Steady state per chunk c:
      //   [S(c) in registers] S(c+1), [dS(c)] dQ(c), [dQ(c) done] release stage c, dP(c+1)
      // S(c+1) overwrites S(c) once the softmax warps hold it in registers, so it runs while
      // they compute P(c) and dS(c); dP(c+1) overwrites dS(c), which dQ(c) reads
      // (tcgen05.mma ops are ordered only when they share an accumulator), hence the wait
      // for dQ(c) -- whose completion also frees chunk c's ring stage (S(c) and dP(c) were
      // complete before the softmax warps used them).
      bool ok = wait_bar(kQFull, 0) && wait_full(0);
      if (ok) {
        issue_s(0);
        issue_dp(0);
      }
      for (int c = 0; ok && c < n_chunks; ++c) {
        const bool more = c + 1 < n_chunks;
        if (more) {
          ok = wait_bar(kSFree, c) && wait_full(c + 1);
          if (!ok) break;
          issue_s(c + 1);
        }
        ok = wait_bar(kDSReady, c);
        if (!ok) break;
        issue_dq(c);
        if (!more) break;
        ok = wait_bar(kDQDone, c);
        if (!ok) break;
        mbar_arrive(bar(kEmpty + c % C::kStages));
        issue_dp(c + 1);
      }
      commit(kDrain);
      for (int i = 0; i < kNumBars; ++i)
        if (commits[i]) mbar_wait(bar(i), (commits[i] - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int w = warp;
    const uint32_t t_tile = tmem + ((uint32_t)(w * 32) << 16);
    const int row = w * 32 + lane;
    const int qz = w, qy = lane >> 3, qx = lane & 7;
    const int zq = z0 + qz, yq = y0 + qy, xq = x0 + qx;
    const bool row_ok = zq < p.Z && yq < p.Y && xq < p.X;
    int64_t grow = 0;
    float lse2_l = __builtin_huge_valf(), lse2_g = __builtin_huge_valf(), delta_l = 0.f, delta_g = 0.f;
    if (row_ok) {
      int64_t rr = ((int64_t)zq * p.Y + yq) * p.X + xq;
      if (p.map) rr = p.map[rr];
      grow = (int64_t)bh * p.tokens + rr;
      lse2_l = p.lse_l[grow] * kLog2e;  // +inf for a row with no valid neighbour: P = 0
      lse2_g = p.lse_g[grow] * kLog2e;
      delta_l = p.delta_l[grow];
      delta_g = p.delta_g[grow];
    }
    uint32_t *park = reinterpret_cast<uint32_t *>(park_base + (size_t)row * D * 2);
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
    const float sc = p.sc, inv_sqrt_d = p.inv_sqrt_d;
    auto wait_warp = [&](int bidx, int completion) -> bool {
      const bool r = mbar_wait(bar(bidx), completion & 1, &g_bwd_errors, kWaitNs, kErrSoftmax);
      const bool all = __all_sync(0xffffffffu, r);
      if (all) tc_fence_after();
      return all;
    };
    bool ok = true;
    for (int ch = 0; ch < n_chunks; ++ch) {
      if (ch == kLocalChunks) {
        // Local branch done once dQ(7) has completed: round it to the storage dtype, park it.
        ok = wait_warp(kDQDone, kLocalChunks - 1);
        if (!ok) break;
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t o[16];
          tmem_ld16(t_tile + kColDQ + 16 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            park[8 * c + i] =
                pack2<BF16>(__uint_as_float(o[2 * i]) * inv_sqrt_d, __uint_as_float(o[2 * i + 1]) * inv_sqrt_d);
        }
      }
      const bool local = ch < kLocalChunks;
      const int zp = p.qz0 + z0 - kR + ch;  // global plane of this local chunk
      const bool active = !local || ((unsigned)(ch - qz) <= 2u * kR && zp >= 0 && zp < p.Zg);  // warp-uniform
      const float lse2 = local ? lse2_l : lse2_g, delta = local ? delta_l : delta_g;
      ok = wait_warp(kSReady, ch);
      if (!ok) break;
      float pr[kKeys];
      if (active) {
#pragma unroll
        for (int g = 0; g < kKeys / 32; ++g) tmem_ld32(t_tile + kColS + 32 * g, reinterpret_cast<uint32_t *>(pr + 32 * g));
        tmem_wait_ld();
      }
      // S(ch) is in registers (or not needed): the S buffer may take S(ch+1)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kSFree));
      if (active) {
        int valid = kKeys;
        if (!local) valid = min(kKeys, p.summaries - (ch - kLocalChunks) * kSumRows);
        if (local || valid < kKeys) {
#pragma unroll
          for (int i = 0; i < kKeys; ++i) {
            const bool use = local ? ((mask[i >> 5] >> (i & 31)) & 1u) != 0u : i < valid;
            pr[i] = use ? ex2_approx(fmaf(pr[i], sc, -lse2)) : 0.f;
          }
        } else {  // a full global chunk: no mask, paired scale
          const float2 sc2 = make_float2(sc, sc), nl2 = make_float2(-lse2, -lse2);
#pragma unroll
          for (int i = 0; i < kKeys; i += 2) {
            const float2 x = fma2(make_float2(pr[i], pr[i + 1]), sc2, nl2);
            pr[i] = ex2_approx(x.x);
            pr[i + 1] = ex2_approx(x.y);
          }
        }
      }
      ok = wait_warp(kDPReady, ch);
      if (!ok) break;
      if (active) {
#pragma unroll
        for (int g = 0; g < kKeys / 32; ++g) {
          uint32_t dp[32];
          tmem_ld32(t_tile + kColDP + 32 * g, dp);
          tmem_wait_ld();
          uint32_t pk[16];
          // dS = P (dP - Delta); its 1/sqrt(D) is applied to the dQ accumulator
          const float2 nd2 = make_float2(-delta, -delta);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 t = add2(make_float2(__uint_as_float(dp[2 * i]), __uint_as_float(dp[2 * i + 1])), nd2);
            const float2 d = mul2(make_float2(pr[32 * g + 2 * i], pr[32 * g + 2 * i + 1]), t);
            pk[i] = pack2<BF16>(d.x, d.y);
          }
          // dS group g goes to dP columns [16g, 16g + 16): already read (groups are read in order)
          tmem_st16(t_tile + kColDP + 16 * g, pk);
        }
      } else {
        uint32_t zero[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) zero[i] = 0u;
#pragma unroll
        for (int g = 0; g < kKeys / 32; ++g) tmem_st16(t_tile + kColDP + 16 * g, zero);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kDSReady));
    }
    // ---- epilogue: dq = round(round(dQ_l) + round(dQ_g)) through the row map
    if (ok) ok = wait_warp(kDQDone, n_chunks - 1);
    if (ok) {
      uint32_t acc[D];
#pragma unroll
      for (int c = 0; c < D / 16; ++c) tmem_ld16(t_tile + kColDQ + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(acc + 16 * c));
      tmem_wait_ld();
      if (row_ok) {
        uint32_t out[D / 2];
#pragma unroll
        for (int i = 0; i < D / 2; ++i) {
          const float2 l = unpack2<BF16>(park[i]);
          const float g0 = round_storage<BF16>(__uint_as_float(acc[2 * i]) * inv_sqrt_d);
          const float g1 = round_storage<BF16>(__uint_as_float(acc[2 * i + 1]) * inv_sqrt_d);
          out[i] = pack2<BF16>(l.x + g0, l.y + g1);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.dq) + grow * D);
#pragma unroll
        for (int v = 0; v < D / 8; ++v) dst[v] = make_uint4(out[4 * v], out[4 * v + 1], out[4 * v + 2], out[4 * v + 3]);
      }
    }
    tmem_wait_st();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kDqMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kDqTmemCols);
  }
}

template <int D, bool BF16, int R>
int launch_dq_t(const StencilBwdArgs &a, cudaStream_t stream) {
  using G = BGeo<R>;
  constexpr int kHY = G::kHY, kHX = G::kHX, kSumRows = G::kSumRows;
  using C = DqCfg<D, G::kKeys>;
  const int Z = a.grid[0], Y = a.grid[1], X = a.grid[2];
  const uint64_t es = 2;
  const uint64_t bh = (uint64_t)a.batch * a.heads, bgs = (uint64_t)a.batch * a.kv_heads;
  CUtensorMap tq, tdol, tdog, tkl, tvl, tsk, tsv;
  {
    const uint64_t dims[5] = {(uint64_t)D, (uint64_t)X, (uint64_t)Y, (uint64_t)Z, bh};
    const uint64_t strides[4] = {D * es, X * D * es, (uint64_t)Y * X * D * es, (uint64_t)Z * Y * X * D * es};
    const uint32_t box[5] = {16, kTX, kTY, kTZ, 1};
    if (int st = encode_operand(&tq, a.dtype, a.q, 5, dims, strides, box)) return st;
    if (int st = encode_operand(&tdol, a.dtype, a.dol, 5, dims, strides, box)) return st;
    if (int st = encode_operand(&tdog, a.dtype, a.dog, 5, dims, strides, box)) return st;
  }
  {
    const uint64_t dims[5] = {(uint64_t)D, (uint64_t)X, (uint64_t)Y, (uint64_t)a.k_planes, bgs};
    const uint64_t strides[4] = {D * es, X * D * es, (uint64_t)Y * X * D * es,
                                 (uint64_t)a.k_planes * Y * X * D * es};
    const uint32_t box[5] = {16, kHX, kHY, 1, 1};
    if (int st = encode_operand(&tkl, a.dtype, a.kl, 5, dims, strides, box)) return st;
    if (int st = encode_operand(&tvl, a.dtype, a.vl, 5, dims, strides, box)) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)a.summaries, bgs};
    const uint64_t strides[2] = {D * es, (uint64_t)a.summaries * D * es};
    const uint32_t box[3] = {16, kSumRows, 1};
    if (int st = encode_operand(&tsk, a.dtype, a.sk, 3, dims, strides, box)) return st;
    if (int st = encode_operand(&tsv, a.dtype, a.sv, 3, dims, strides, box)) return st;
  }
  DqParams p{};
  p.Z = Z;
  p.Zg = a.global_planes;
  p.qz0 = a.q_z0;
  p.kz0 = a.k_z0;
  p.Y = Y;
  p.X = X;
  p.tiles_z = (Z + kTZ - 1) / kTZ;
  p.tiles_y = (Y + kTY - 1) / kTY;
  p.tiles_x = (X + kTX - 1) / kTX;
  p.heads = a.heads;
  p.kv_heads = a.kv_heads;
  p.summaries = a.summaries;
  p.global_chunks = (a.summaries + kSumRows - 1) / kSumRows;
  p.tokens = (int64_t)Z * Y * X;
  p.sc = kLog2e / sqrtf((float)D);
  p.inv_sqrt_d = 1.f / sqrtf((float)D);
  p.lse_l = a.lse_l;
  p.lse_g = a.lse_g;
  p.delta_l = a.delta_l;
  p.delta_g = a.delta_g;
  p.map = a.raster_to_packed;
  p.dq = a.dq;
  const int64_t units = (int64_t)bh * p.tiles_z * p.tiles_y * p.tiles_x;
  if (units <= 0) return P3D_OK;
  if (units > 0x7fffffff) return fail(P3D_ERR_UNSUPPORTED, "too many tiles");
  auto kernel = stencil_bwd_dq_kernel<D, BF16, R>;
  static size_t seen[kMaxDevices] = {};
  if (int st = smem_optin(kernel, C::kSmemBytes, seen)) return st;
  kernel<<<(unsigned)units, kDqThreads, C::kSmemBytes, stream>>>(tq, tdol, tdog, tkl, tvl, tsk, tsv, p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}


// ============================================================================ global dSK / dSV
//
// Restates the summary-gradient half of the global branch (kernels.py:210-239): for a
// tile of 128 summaries (TMEM lanes) and a stream of 128-query chunks (columns),
//   S^T = SK Q^T, dP^T = SV dO_g^T, P^T = exp(S^T / sqrt(D) - lse), dS^T = P^T (dP^T - Delta) / sqrt(D)
//   dSV += P^T dO_g,  dSK += dS^T Q          (P^T and dS^T rounded to the storage dtype)
// over the query chunks of one split (the rounded dS^T operand is P^T (dP^T - Delta); the
// 1/sqrt(D) multiplies the fp32 dSK accumulator once, when it is written); splits write fp32 partials [B*G, splits, M, D] that a
// fixed-order reduction sums.  The global branch ignores the geometry, so this kernel serves
// any token order.  Summary rows past M read zeros and are not written; query columns past
// N get lse = +inf (P = 0).
//
// TMEM: S^T [0, 128), dP^T [128, 256), P^T [256, 320), dS^T [320, 384) (16-bit pairs),
// dSK [384, 384 + D), dSV [384 + D, 384 + 2D).  Eight softmax warps: warp w serves TMEM
// lanes 32(w%4).. and query columns 64(w/4)..+64.  Per chunk the MMA thread issues S^T and
// dP^T; the softmax warps pull them into registers and release the buffers (the next
// chunk's S^T / dP^T start at once), then store P^T / dS^T once the previous chunk's dSV /
// dSK products are done with them, and the MMA thread accumulates dSV and dSK.
constexpr int kGRows = 128;   // summaries per tile
constexpr int kGCols = 128;   // queries per chunk
constexpr uint32_t kGColS = 0, kGColDP = 128, kGColP = 256, kGColDS = 320, kGColAcc = 384;

template <int D>
struct GkvCfg {
  static constexpr int kK = D / 16;
  static constexpr int kBox = 128 * 32;                 // 128 rows x 16 channels
  static constexpr int kTileBytes = kK * kBox;          // one 128-row operand tile
  static constexpr int kRowVals = kGCols * 4;           // one chunk of lse (or Delta), fp32
  static constexpr int kStageBytes = (2 * kTileBytes + 2 * kRowVals + 1023) / 1024 * 1024;
  static constexpr int kFixed = 2 * kTileBytes + 1024;
  static constexpr int kRoom = (227 * 1024 - 2048 - kFixed) / kStageBytes;
  static constexpr int kStages = kRoom > 4 ? 4 : kRoom;
  static constexpr int kSmemNeed = kFixed + kStages * kStageBytes;
  static constexpr int kSmemBytes = kSmemNeed > 116 * 1024 ? kSmemNeed : 116 * 1024;
  static_assert(kStages >= 2, "the ring must hold two chunks");
  static_assert(kGColAcc + 2 * D <= 512, "TMEM budget");
};

enum GkvBar {
  kGKvFull = 0,
  kGFull = 1,                  // [stage]: Q, dO_g copies (tx) + lse / Delta stores (one arrive)
  kGEmpty = kGFull + 4,        // [stage]: released by the commit after dSV / dSK of its chunk
  kGSReady = kGEmpty + 4,      // S^T(c) and dP^T(c) complete
  kGSFree = kGSReady + 1,      // the 8 softmax warps have read S^T(c), dP^T(c) (count 8)
  kGPdsReady = kGSFree + 1,    // the 8 softmax warps stored P^T(c), dS^T(c) (count 8)
  kGPdsFree = kGPdsReady + 1,  // dSV(c), dSK(c) complete
  kGDrain = kGPdsFree + 1,
  kGNumBars = kGDrain + 1
};

struct GkvParams {
  int heads, kv_heads, rep, tokens, summaries, m_tiles, splits, q_chunks, per_split;
  int bulk_vals;  // lse / Delta rows are 16-byte aligned (N % 4 == 0): bulk-copy them
  float sc, inv_sqrt_d;
  const float *lse_g, *delta_g;  // [B*H, N]
  float *dk_part, *dv_part;      // [B*G, splits, M, D]
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    global_dkv_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                         const __grid_constant__ CUtensorMap tsk, const __grid_constant__ CUtensorMap tsv,
                         const GkvParams p) {
  using C = GkvCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kGNumBars];
  __shared__ uint32_t tmem_holder;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x % p.splits;
  const int mt = (blockIdx.x / p.splits) % p.m_tiles;
  const int bg = blockIdx.x / (p.splits * p.m_tiles);
  const int b = bg / p.kv_heads, g = bg % p.kv_heads;
  const int m0 = mt * kGRows;
  const int total = p.rep * p.q_chunks;
  const int c_begin = split * p.per_split;
  const int n_chunks = min(total, c_begin + p.per_split) - c_begin;  // >= 1 (host)

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sk_smem = base, sv_smem = base + C::kTileBytes;
  const uint32_t ring = base + 2 * C::kTileBytes;
  uint8_t *ring_ptr = smem_raw + (base - raw) + 2 * C::kTileBytes;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (tid == 0) {
    mbar_init(bar(kGKvFull), 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar(kGFull + s), 2);
      mbar_init(bar(kGEmpty + s), 1);
    }
    mbar_init(bar(kGSReady), 1);
    mbar_init(bar(kGSFree), 8);
    mbar_init(bar(kGPdsReady), 8);
    mbar_init(bar(kGPdsFree), 1);
    mbar_init(bar(kGDrain), 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tq);
    prefetch_tmap(&tdo);
    prefetch_tmap(&tsk);
    prefetch_tmap(&tsv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;
  auto chunk_head = [&](int c) { return b * p.heads + g * p.rep + (c_begin + c) / p.q_chunks; };
  auto chunk_row0 = [&](int c) { return ((c_begin + c) % p.q_chunks) * kGCols; };

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ producer (whole warp)
    if (lane == 0) {
      mbar_expect_tx(bar(kGKvFull), 2 * C::kTileBytes);
      for (int c = 0; c < C::kK; ++c) {
        tma_load_3d(sk_smem + c * C::kBox, &tsk, bar(kGKvFull), 16 * c, m0, bg);
        tma_load_3d(sv_smem + c * C::kBox, &tsv, bar(kGKvFull), 16 * c, m0, bg);
      }
    }
    int issued = 0;
    for (int ch = 0; ch < n_chunks; ++ch) {
      const int s = ch % C::kStages;
      // kGEmpty[s]: completion ch/kStages - 1 (the same unambiguity argument as the dQ kernel)
      bool ok = true;
      if (lane == 0 && ch >= C::kStages)
        ok = mbar_wait(bar(kGEmpty + s), (ch / C::kStages - 1) & 1, &g_bwd_errors, kWaitNs, kErrProducer);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      const uint32_t stage = ring + s * C::kStageBytes;
      const uint32_t full = bar(kGFull + s);
      const int bh = chunk_head(ch), n0 = chunk_row0(ch);
      const int64_t r0 = (int64_t)bh * p.tokens + n0;
      const uint32_t rows = (uint32_t)min(kGCols, p.tokens - n0);
      // lse and Delta of the chunk's queries (columns past the last row are masked by the
      // softmax warps): bulk copies beside the tensor tiles, or plain loads in registers
      // first, then stores (so the loads are not serialised behind the stores).
      const uint32_t vals_smem = stage + 2 * C::kTileBytes;
      if (lane == 0) {
        mbar_expect_tx(full, 2 * C::kTileBytes + (p.bulk_vals ? 2 * rows * 4 : 0));
        for (int c = 0; c < C::kK; ++c) {
          tma_load_3d(stage + c * C::kBox, &tq, full, 16 * c, n0, bh);
          tma_load_3d(stage + C::kTileBytes + c * C::kBox, &tdo, full, 16 * c, n0, bh);
        }
        if (p.bulk_vals) {
          bulk_load(vals_smem, p.lse_g + r0, rows * 4, full);
          bulk_load(vals_smem + C::kRowVals, p.delta_g + r0, rows * 4, full);
        }
      }
      if (!p.bulk_vals) {
        float *vals = reinterpret_cast<float *>(ring_ptr + (size_t)s * C::kStageBytes + 2 * C::kTileBytes);
        float l[kGCols / 32], dl[kGCols / 32];
#pragma unroll
        for (int k = 0; k < kGCols / 32; ++k) {
          const int j = lane + 32 * k;
          l[k] = j < (int)rows ? __ldg(p.lse_g + r0 + j) : 0.f;
          dl[k] = j < (int)rows ? __ldg(p.delta_g + r0 + j) : 0.f;
        }
#pragma unroll
        for (int k = 0; k < kGCols / 32; ++k) {
          vals[lane + 32 * k] = l[k];
          vals[kGCols + lane + 32 * k] = dl[k];
        }
        __syncwarp();
      }
      if (lane == 0) mbar_arrive(full);
      issued = ch + 1;
    }
    if (lane == 0) {
      mbar_wait(bar(kGKvFull), 0, &g_bwd_errors, kWaitNs, kErrTeardown);
      for (int ch = issued > C::kStages ? issued - C::kStages : 0; ch < issued; ++ch)
        mbar_wait(bar(kGFull + ch % C::kStages), (ch / C::kStages) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(128, kGCols, BF16, false);
      constexpr uint32_t idesc_acc = idesc_f16(128, D, BF16, true);
      uint32_t commits[kGNumBars];
      for (int i = 0; i < kGNumBars; ++i) commits[i] = 0u;
      auto commit = [&](int bidx) {
        mma_commit(bar(bidx));
        ++commits[bidx];
      };
      auto stage_of = [&](int c) { return ring + (c % C::kStages) * C::kStageBytes; };
      auto issue_s_dp = [&](int c) {
        const uint32_t q = stage_of(c), dov = stage_of(c) + C::kTileBytes;
        for (int kk = 0; kk < C::kK; ++kk)
          mma_ss(tmem + kGColS, desc_sw32(sk_smem + kk * C::kBox, 16, 256), desc_sw32(q + kk * C::kBox, 16, 256),
                 idesc_s, kk > 0 ? 1u : 0u);
        for (int kk = 0; kk < C::kK; ++kk)
          mma_ss(tmem + kGColDP, desc_sw32(sv_smem + kk * C::kBox, 16, 256), desc_sw32(dov + kk * C::kBox, 16, 256),
                 idesc_s, kk > 0 ? 1u : 0u);
        commit(kGSReady);
      };
      auto issue_acc = [&](int c) {
        const uint32_t q = stage_of(c), dov = stage_of(c) + C::kTileBytes;
        for (int j = 0; j < kGCols / 16; ++j)
          mma_ts(tmem + kGColAcc + D, tmem + kGColP + 8 * j, desc_sw32(dov + j * 512, C::kBox, 256), idesc_acc,
                 (c == 0 && j == 0) ? 0u : 1u);
        for (int j = 0; j < kGCols / 16; ++j)
          mma_ts(tmem + kGColAcc, tmem + kGColDS + 8 * j, desc_sw32(q + j * 512, C::kBox, 256), idesc_acc,
                 (c == 0 && j == 0) ? 0u : 1u);
        commit(kGPdsFree);
        commit(kGEmpty + c % C::kStages);  // every reader of chunk c's stage is issued
      };
      auto wait_bar = [&](int bidx, int completion) -> bool {
        if (!mbar_wait(bar(bidx), completion & 1, &g_bwd_errors, kWaitNs, kErrMma)) return false;
        tc_fence_after();
        return true;
      };
      auto wait_full = [&](int c) { return wait_bar(kGFull + c % C::kStages, c / C::kStages); };
      bool ok = wait_bar(kGKvFull, 0) && wait_full(0);
      if (ok) issue_s_dp(0);
      for (int c = 0; ok && c < n_chunks; ++c) {
        ok = wait_bar(kGSFree, c);
        if (!ok) break;
        if (c + 1 < n_chunks) {
          ok = wait_full(c + 1);
          if (!ok) break;
          issue_s_dp(c + 1);
        }
        ok = wait_bar(kGPdsReady, c);
        if (!ok) break;
        issue_acc(c);
      }
      commit(kGDrain);
      for (int i = 0; i < kGNumBars; ++i)
        if (commits[i]) mbar_wait(bar(i), (commits[i] - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
    }
  } else {
    // ------------------------------------------------------------------ softmax (8 warps) + epilogue
    const int quarter = warp & 3, half = warp >> 2;
    const uint32_t t_lanes = tmem + ((uint32_t)(quarter * 32) << 16);
    const int row = quarter * 32 + lane;  // summary m0 + row
    const float sc = p.sc, inv_sqrt_d = p.inv_sqrt_d;
    auto wait_warp = [&](int bidx, int completion) -> bool {
      const bool r = mbar_wait(bar(bidx), completion & 1, &g_bwd_errors, kWaitNs, kErrSoftmax);
      const bool all = __all_sync(0xffffffffu, r);
      if (all) tc_fence_after();
      return all;
    };
    bool ok = true;
    for (int ch = 0; ch < n_chunks; ++ch) {
      ok = wait_warp(kGSReady, ch);
      if (!ok) break;
      const float4 *vals = reinterpret_cast<const float4 *>(ring_ptr + (size_t)(ch % C::kStages) * C::kStageBytes +
                                                            2 * C::kTileBytes);
      const int valid = min(kGCols, p.tokens - chunk_row0(ch));  // query columns inside the volume
      uint32_t pw[2][16], dw[2][16];
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const int col0 = 64 * half + 32 * gi;
        uint32_t sv[32], dv[32];
        tmem_ld32(t_lanes + kGColS + col0, sv);
        tmem_ld32(t_lanes + kGColDP + col0, dv);
        tmem_wait_ld();
        // P^T = exp2(S^T sc - lse log2e); dS^T = P^T (dP^T - Delta) (its 1/sqrt(D) is applied
        // to the dSK accumulator at the end)
        if (col0 + 32 <= valid) {  // every column inside the volume: paired, no masks
          const float2 sc2 = make_float2(sc, sc), nl2e = make_float2(-kLog2e, -kLog2e);
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            const int j = col0 + 4 * i4;
            const float4 l4 = vals[j / 4], d4 = vals[(kGCols + j) / 4];
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              const int i = 4 * i4 + 2 * h2;
              const float2 l2 = h2 ? make_float2(l4.z, l4.w) : make_float2(l4.x, l4.y);
              const float2 nd2 = h2 ? make_float2(-d4.z, -d4.w) : make_float2(-d4.x, -d4.y);
              const float2 x =
                  fma2(make_float2(__uint_as_float(sv[i]), __uint_as_float(sv[i + 1])), sc2, mul2(l2, nl2e));
              const float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
              const float2 dd = mul2(pp, add2(make_float2(__uint_as_float(dv[i]), __uint_as_float(dv[i + 1])), nd2));
              pw[gi][2 * i4 + h2] = pack2<BF16>(pp.x, pp.y);
              dw[gi][2 * i4 + h2] = pack2<BF16>(dd.x, dd.y);
            }
          }
        } else {
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            const int j = col0 + 4 * i4;
            const float4 l4 = vals[j / 4], d4 = vals[(kGCols + j) / 4];
            const float ls[4] = {l4.x, l4.y, l4.z, l4.w}, ds[4] = {d4.x, d4.y, d4.z, d4.w};
            float pp[4], dd[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 4 * i4 + e;
              // columns past the volume may hold stale values: they give exact zeros
              const bool in = j + e < valid;
              pp[e] = in ? ex2_approx(fmaf(__uint_as_float(sv[i]), sc, -ls[e] * kLog2e)) : 0.f;
              dd[e] = in ? pp[e] * (__uint_as_float(dv[i]) - ds[e]) : 0.f;
            }
            pw[gi][2 * i4] = pack2<BF16>(pp[0], pp[1]);
            pw[gi][2 * i4 + 1] = pack2<BF16>(pp[2], pp[3]);
            dw[gi][2 * i4] = pack2<BF16>(dd[0], dd[1]);
            dw[gi][2 * i4 + 1] = pack2<BF16>(dd[2], dd[3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kGSFree));
      if (ch > 0) {
        ok = wait_warp(kGPdsFree, ch - 1);  // dSV / dSK of the previous chunk no longer read P^T / dS^T
        if (!ok) break;
      }
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        tmem_st16(t_lanes + kGColP + 32 * half + 16 * gi, pw[gi]);
        tmem_st16(t_lanes + kGColDS + 32 * half + 16 * gi, dw[gi]);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kGPdsReady));
    }
    if (ok) ok = wait_warp(kGPdsFree, n_chunks - 1);
    if (ok) {
      // warps 0-3 write dSK rows, warps 4-7 dSV rows
      uint32_t acc[D];
      const uint32_t col = kGColAcc + (half ? D : 0);
#pragma unroll
      for (int c = 0; c < D / 16; ++c) tmem_ld16(t_lanes + col + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(acc + 16 * c));
      tmem_wait_ld();
      const int m = m0 + row;
      if (m < p.summaries) {
        float *dst = (half ? p.dv_part : p.dk_part) + (((int64_t)bg * p.splits + split) * p.summaries + m) * D;
        const float scale = half ? 1.f : inv_sqrt_d;  // dSK: the 1/sqrt(D) of dS
#pragma unroll
        for (int v = 0; v < D / 4; ++v)
          reinterpret_cast<float4 *>(dst)[v] =
              make_float4(__uint_as_float(acc[4 * v]) * scale, __uint_as_float(acc[4 * v + 1]) * scale,
                          __uint_as_float(acc[4 * v + 2]) * scale, __uint_as_float(acc[4 * v + 3]) * scale);
      }
    }
    tmem_wait_st();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool BF16>
int launch_gkv_t(const GlobalDkvArgs &a, cudaStream_t stream) {
  using C = GkvCfg<D>;
  const uint64_t es = 2;
  const uint64_t bh = (uint64_t)a.batch * a.heads, bgs = (uint64_t)a.batch * a.kv_heads;
  CUtensorMap tq, tdo, tsk, tsv;
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)a.tokens, bh};
    const uint64_t strides[2] = {D * es, (uint64_t)a.tokens * D * es};
    const uint32_t box[3] = {16, kGCols, 1};
    if (int st = encode_operand(&tq, a.dtype, a.q, 3, dims, strides, box)) return st;
    if (int st = encode_operand(&tdo, a.dtype, a.dog, 3, dims, strides, box)) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)a.summaries, bgs};
    const uint64_t strides[2] = {D * es, (uint64_t)a.summaries * D * es};
    const uint32_t box[3] = {16, kGRows, 1};
    if (int st = encode_operand(&tsk, a.dtype, a.sk, 3, dims, strides, box)) return st;
    if (int st = encode_operand(&tsv, a.dtype, a.sv, 3, dims, strides, box)) return st;
  }
  GkvParams p{};
  p.heads = a.heads;
  p.kv_heads = a.kv_heads;
  p.rep = a.heads / a.kv_heads;
  p.tokens = a.tokens;
  p.summaries = a.summaries;
  p.m_tiles = (a.summaries + kGRows - 1) / kGRows;
  p.q_chunks = (a.tokens + kGCols - 1) / kGCols;
  p.splits = a.splits;
  p.per_split = a.per_split;
  p.bulk_vals = a.tokens % 4 == 0 && ((uintptr_t)a.lse_g & 15) == 0 && ((uintptr_t)a.delta_g & 15) == 0;
  p.sc = kLog2e / sqrtf((float)D);
  p.inv_sqrt_d = 1.f / sqrtf((float)D);
  p.lse_g = a.lse_g;
  p.delta_g = a.delta_g;
  p.dk_part = a.dk_part;
  p.dv_part = a.dv_part;
  const int64_t units = (int64_t)bgs * p.m_tiles * p.splits;
  if (units <= 0) return P3D_OK;
  if (units > 0x7fffffff) return fail(P3D_ERR_UNSUPPORTED, "too many tiles");
  auto kernel = global_dkv_tc_kernel<D, BF16>;
  static size_t seen[kMaxDevices] = {};
  if (int st = smem_optin(kernel, C::kSmemBytes, seen)) return st;
  kernel<<<(unsigned)units, kThreads, C::kSmemBytes, stream>>>(tq, tdo, tsk, tsv, p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}


// ============================================================================ local dK / dV
//
// Restates the key-gradient half of the local branch (kernels.py:154-176; stencil.py:91-147
// with QUERY false) on tensor cores.  A CTA owns one (batch, kv-head) and a 4x4x8 (z, y, x)
// box of 128 keys (TMEM lanes, row order (z, y, x) as for the forward's query tiles) and
// streams, for every query head of its group, the 8 query halo planes z0-2 .. z0+5 (8x12
// windows, 96 queries each):
//   S^T = K Q^T, dP^T = V dO_l^T, P^T = exp(S^T / sqrt(D) - lse_l) on the key's 5x5x5 cube,
//   dS^T = P^T (dP^T - Delta_l) / sqrt(D),   dV += P^T dO_l,  dK += dS^T Q.
// The neighbourhood is symmetric (key j is in query i's clipped cube iff i is in j's), so
// the mask is the forward's with the roles swapped.  P^T and dS^T are rounded to the
// storage dtype for the products (the reference keeps them in fp32; the difference is far
// inside the bf16 tolerance).  Each CTA writes its own keys' dK / dV: no atomics, no
// partials.
//
// TMEM (W = kKeys, 96 at radius 2): S^T [0, W), dP^T [W, 2W), P^T [2W, 2.5W), dS^T
// [2.5W, 3W), dK [3W, 3W + D), dV [3W + D, 3W + 2D).  Eight softmax warps (warp w: TMEM
// lanes 32(w%4).., query columns (W/2)(w/4)..+W/2); the protocol is the global dSK / dSV
// kernel's.
template <int D, int KEYS>
struct LkvCfg {
  static constexpr uint32_t kLColS = 0, kLColDP = KEYS, kLColP = 2 * KEYS, kLColDS = 2 * KEYS + KEYS / 2,
                            kLColAcc = 3 * KEYS;
  static constexpr int kK = D / 16;
  static constexpr int kBoxT = kRows * 32;           // key tile: 128 rows x 16 channels
  static constexpr int kBoxP = KEYS * 32;            // query plane: KEYS rows x 16 channels
  static constexpr int kTileBytes = kK * kBoxT;
  static constexpr int kPlaneBytes = kK * kBoxP;
  static constexpr int kVals = KEYS * 4;              // lse (or Delta) of one plane, fp32
  static constexpr int kStageBytes = (2 * kPlaneBytes + 2 * kVals + 1023) / 1024 * 1024;
  static constexpr int kFixed = 2 * kTileBytes + 1024;
  static constexpr int kRoom = (227 * 1024 - 2048 - kFixed) / kStageBytes;
  static constexpr int kStages = kRoom > 4 ? 4 : kRoom;
  static constexpr int kSmemNeed = kFixed + kStages * kStageBytes;
  static constexpr int kSmemBytes = kSmemNeed > 116 * 1024 ? kSmemNeed : 116 * 1024;
  static_assert(kStages >= 2, "the ring must hold two chunks");
  static_assert(kLColAcc + 2 * D <= 512, "TMEM budget");
};

struct LkvParams {
  int Z, Y, X, tiles_z, tiles_y, tiles_x;  // Z: planes of the key (centre) buffer
  int Zg, cz0, kz0;      // global planes; global z of the first key plane and of kl / vl plane 0
  int xz0;               // global z of plane 0 of the query-side buffers (q, dO_l, lse_l, Delta_l)
  int heads, kv_heads, rep;
  int64_t tokens;        // rows of the key buffer's grid (outputs)
  int64_t xtokens;       // rows of the query-side buffers per (batch, head)
  float sc, inv_sqrt_d;
  const float *lse_l, *delta_l;  // [B*H, xtokens] in the layout's row order
  const int32_t *map;            // raster -> packed rows (nullptr: raster)
  void *dkl, *dvl;               // [B*G, N, D] in the layout's row order
};

template <int D, bool BF16, int R>
__global__ void __launch_bounds__(kThreads, 1)
    stencil_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tkl, const __grid_constant__ CUtensorMap tvl,
                           const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                           const LkvParams p) {
  using G = BGeo<R>;
  constexpr int kR = G::kR, kHX = G::kHX, kWin = G::kWin, kKeys = G::kKeys, kHalf = G::kHalf;
  constexpr int kLocalChunks = G::kLocalChunks;
  using C = LkvCfg<D, kKeys>;
  constexpr uint32_t kLColS = C::kLColS, kLColDP = C::kLColDP, kLColP = C::kLColP, kLColDS = C::kLColDS,
                     kLColAcc = C::kLColAcc;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kGNumBars];
  __shared__ uint32_t tmem_holder;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int unit = blockIdx.x;
  const int tx = unit % p.tiles_x;
  unit /= p.tiles_x;
  const int ty = unit % p.tiles_y;
  unit /= p.tiles_y;
  const int tz = unit % p.tiles_z;
  const int bg = unit / p.tiles_z;
  const int b = bg / p.kv_heads, g = bg % p.kv_heads;
  const int x0 = tx * kTX, y0 = ty * kTY, z0 = tz * kTZ;
  const int n_chunks = p.rep * kLocalChunks;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t k_smem = base, v_smem = base + C::kTileBytes;
  const uint32_t ring = base + 2 * C::kTileBytes;
  uint8_t *ring_ptr = smem_raw + (base - raw) + 2 * C::kTileBytes;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (tid == 0) {
    mbar_init(bar(kGKvFull), 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar(kGFull + s), 2);
      mbar_init(bar(kGEmpty + s), 1);
    }
    mbar_init(bar(kGSReady), 1);
    mbar_init(bar(kGSFree), 8);
    mbar_init(bar(kGPdsReady), 8);
    mbar_init(bar(kGPdsFree), 1);
    mbar_init(bar(kGDrain), 1);
    fence_mbar_init();
  }
  if constexpr (kWin < kKeys) {
    // the query planes fill kWin of the kKeys rows of each box: the rest reads as zeros
    uint4 *ring_v = reinterpret_cast<uint4 *>(ring_ptr);
    for (int i = tid; i < C::kStages * C::kStageBytes / 16; i += kThreads) ring_v[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tkl);
    prefetch_tmap(&tvl);
    prefetch_tmap(&tq);
    prefetch_tmap(&tdo);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;
  // chunk c: query head b*H + g*rep + c/8, query plane z0 - 2 + c%8
  auto chunk_head = [&](int c) { return b * p.heads + g * p.rep + c / kLocalChunks; };
  auto chunk_plane = [&](int c) { return p.cz0 + z0 - kR + c % kLocalChunks; };  // global z

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ producer (whole warp)
    if (lane == 0) {
      mbar_expect_tx(bar(kGKvFull), 2 * C::kTileBytes);
      for (int c = 0; c < C::kK; ++c) {
        tma_load_5d(k_smem + c * C::kBoxT, &tkl, bar(kGKvFull), 16 * c, x0, y0, p.cz0 + z0 - p.kz0, bg);
        tma_load_5d(v_smem + c * C::kBoxT, &tvl, bar(kGKvFull), 16 * c, x0, y0, p.cz0 + z0 - p.kz0, bg);
      }
    }
    int issued = 0;
    for (int ch = 0; ch < n_chunks; ++ch) {
      const int s = ch % C::kStages;
      bool ok = true;
      if (lane == 0 && ch >= C::kStages)
        ok = mbar_wait(bar(kGEmpty + s), (ch / C::kStages - 1) & 1, &g_bwd_errors, kWaitNs, kErrProducer);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      const uint32_t stage = ring + s * C::kStageBytes;
      const uint32_t full = bar(kGFull + s);
      const int bh = chunk_head(ch), zp = chunk_plane(ch);
      if (lane == 0) {
        mbar_expect_tx(full, 2 * C::kK * kWin * 32);
        for (int c = 0; c < C::kK; ++c) {
          tma_load_5d(stage + c * C::kBoxP, &tq, full, 16 * c, x0 - kR, y0 - kR, zp - p.xz0, bh);
          tma_load_5d(stage + C::kPlaneBytes + c * C::kBoxP, &tdo, full, 16 * c, x0 - kR, y0 - kR, zp - p.xz0,
                      bh);
        }
      }
      // lse (as log2) and Delta of the plane's kWin queries; +inf outside the volume and on
      // the padding columns (P = 0).
      // All loads are issued before any store, so they overlap.
      float *vals = reinterpret_cast<float *>(ring_ptr + (size_t)s * C::kStageBytes + 2 * C::kPlaneBytes);
      float l[kKeys / 32], dl[kKeys / 32];
#pragma unroll
      for (int k = 0; k < kKeys / 32; ++k) {
        const int j = lane + 32 * k;
        const int qy = y0 - kR + j / kHX, qx = x0 - kR + j % kHX;
        const bool in = j < kWin && zp >= 0 && zp < p.Zg && qy >= 0 && qy < p.Y && qx >= 0 && qx < p.X;
        l[k] = __builtin_huge_valf();
        dl[k] = 0.f;
        if (in) {
          int64_t r = ((int64_t)(zp - p.xz0) * p.Y + qy) * p.X + qx;
          if (p.map) r = __ldg(p.map + r);
          const int64_t row = (int64_t)bh * p.xtokens + r;
          l[k] = __ldg(p.lse_l + row) * kLog2e;
          dl[k] = __ldg(p.delta_l + row);
        }
      }
#pragma unroll
      for (int k = 0; k < kKeys / 32; ++k) {
        vals[lane + 32 * k] = l[k];
        vals[kKeys + lane + 32 * k] = dl[k];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(full);
      issued = ch + 1;
    }
    if (lane == 0) {
      mbar_wait(bar(kGKvFull), 0, &g_bwd_errors, kWaitNs, kErrTeardown);
      for (int ch = issued > C::kStages ? issued - C::kStages : 0; ch < issued; ++ch)
        mbar_wait(bar(kGFull + ch % C::kStages), (ch / C::kStages) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(128, kKeys, BF16, false);
      constexpr uint32_t idesc_acc = idesc_f16(128, D, BF16, true);
      uint32_t commits[kGNumBars];
      for (int i = 0; i < kGNumBars; ++i) commits[i] = 0u;
      auto commit = [&](int bidx) {
        mma_commit(bar(bidx));
        ++commits[bidx];
      };
      auto stage_of = [&](int c) { return ring + (c % C::kStages) * C::kStageBytes; };
      auto issue_s_dp = [&](int c) {
        const uint32_t q = stage_of(c), dov = stage_of(c) + C::kPlaneBytes;
        for (int kk = 0; kk < C::kK; ++kk)
          mma_ss(tmem + kLColS, desc_sw32(k_smem + kk * C::kBoxT, 16, 256), desc_sw32(q + kk * C::kBoxP, 16, 256),
                 idesc_s, kk > 0 ? 1u : 0u);
        for (int kk = 0; kk < C::kK; ++kk)
          mma_ss(tmem + kLColDP, desc_sw32(v_smem + kk * C::kBoxT, 16, 256), desc_sw32(dov + kk * C::kBoxP, 16, 256),
                 idesc_s, kk > 0 ? 1u : 0u);
        commit(kGSReady);
      };
      auto issue_acc = [&](int c) {
        const uint32_t q = stage_of(c), dov = stage_of(c) + C::kPlaneBytes;
        for (int j = 0; j < kKeys / 16; ++j)
          mma_ts(tmem + kLColAcc + D, tmem + kLColP + 8 * j, desc_sw32(dov + j * 512, C::kBoxP, 256), idesc_acc,
                 (c == 0 && j == 0) ? 0u : 1u);
        for (int j = 0; j < kKeys / 16; ++j)
          mma_ts(tmem + kLColAcc, tmem + kLColDS + 8 * j, desc_sw32(q + j * 512, C::kBoxP, 256), idesc_acc,
                 (c == 0 && j == 0) ? 0u : 1u);
        commit(kGPdsFree);
        commit(kGEmpty + c % C::kStages);
      };
      auto wait_bar = [&](int bidx, int completion) -> bool {
        if (!mbar_wait(bar(bidx), completion & 1, &g_bwd_errors, kWaitNs, kErrMma)) return false;
        tc_fence_after();
        return true;
      };
      auto wait_full = [&](int c) { return wait_bar(kGFull + c % C::kStages, c / C::kStages); };
      bool ok = wait_bar(kGKvFull, 0) && wait_full(0);
      if (ok) issue_s_dp(0);
      for (int c = 0; ok && c < n_chunks; ++c) {
        ok = wait_bar(kGSFree, c);
        if (!ok) break;
        if (c + 1 < n_chunks) {
          ok = wait_full(c + 1);
          if (!ok) break;
          issue_s_dp(c + 1);
        }
        ok = wait_bar(kGPdsReady, c);
        if (!ok) break;
        issue_acc(c);
      }
      commit(kGDrain);
      for (int i = 0; i < kGNumBars; ++i)
        if (commits[i]) mbar_wait(bar(i), (commits[i] - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
    }
  } else {
    // ------------------------------------------------------------------ softmax (8 warps) + epilogue
    const int quarter = warp & 3, half = warp >> 2;
    const uint32_t t_lanes = tmem + ((uint32_t)(quarter * 32) << 16);
    const int kz = z0 + quarter, kyl = lane >> 3, kxl = lane & 7;
    const int ky = y0 + kyl, kx = x0 + kxl;
    const bool row_ok = kz < p.Z && ky < p.Y && kx < p.X;
    // this warp's kHalf query columns of the halo window that lie in the key's cube
    uint64_t mask = 0ull;
#pragma unroll
    for (int i = 0; i < kHalf; ++i) {
      const int j = kHalf * half + i, hy = j / kHX, hx = j % kHX;
      if (j < kWin && (unsigned)(hy - kyl) <= 2u * kR && (unsigned)(hx - kxl) <= 2u * kR) mask |= 1ull << i;
    }
    if (!row_ok) mask = 0ull;
    const float sc = p.sc, inv_sqrt_d = p.inv_sqrt_d;
    auto wait_warp = [&](int bidx, int completion) -> bool {
      const bool r = mbar_wait(bar(bidx), completion & 1, &g_bwd_errors, kWaitNs, kErrSoftmax);
      const bool all = __all_sync(0xffffffffu, r);
      if (all) tc_fence_after();
      return all;
    };
    bool ok = true;
    for (int ch = 0; ch < n_chunks; ++ch) {
      ok = wait_warp(kGSReady, ch);
      if (!ok) break;
      const int zp = chunk_plane(ch);
      const bool active = (unsigned)(zp - (p.cz0 + kz) + kR) <= 2u * kR;  // warp-uniform
      const float *vals = reinterpret_cast<const float *>(ring_ptr + (size_t)(ch % C::kStages) * C::kStageBytes +
                                                          2 * C::kPlaneBytes);
      uint32_t pw[kHalf / 16][8], dw[kHalf / 16][8];
      if (active) {
#pragma unroll
        for (int gi = 0; gi < kHalf / 16; ++gi) {
          const int col0 = kHalf * half + 16 * gi;
          uint32_t sv[16], dv[16];
          tmem_ld16(t_lanes + kLColS + col0, sv);
          tmem_ld16(t_lanes + kLColDP + col0, dv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int j = col0 + 2 * i, bit = 16 * gi + 2 * i;
            const float p0 = (mask >> bit) & 1ull ? ex2_approx(fmaf(__uint_as_float(sv[2 * i]), sc, -vals[j])) : 0.f;
            const float p1 =
                (mask >> (bit + 1)) & 1ull ? ex2_approx(fmaf(__uint_as_float(sv[2 * i + 1]), sc, -vals[j + 1])) : 0.f;
            const float d0 = p0 * (__uint_as_float(dv[2 * i]) - vals[kKeys + j]) * inv_sqrt_d;
            const float d1 = p1 * (__uint_as_float(dv[2 * i + 1]) - vals[kKeys + j + 1]) * inv_sqrt_d;
            pw[gi][i] = pack2<BF16>(p0, p1);
            dw[gi][i] = pack2<BF16>(d0, d1);
          }
        }
      } else {
#pragma unroll
        for (int gi = 0; gi < kHalf / 16; ++gi)
#pragma unroll
          for (int i = 0; i < 8; ++i) pw[gi][i] = dw[gi][i] = 0u;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kGSFree));
      if (ch > 0) {
        ok = wait_warp(kGPdsFree, ch - 1);
        if (!ok) break;
      }
#pragma unroll
      for (int gi = 0; gi < kHalf / 16; ++gi) {
        tmem_st8(t_lanes + kLColP + (kHalf / 2) * half + 8 * gi, pw[gi]);
        tmem_st8(t_lanes + kLColDS + (kHalf / 2) * half + 8 * gi, dw[gi]);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kGPdsReady));
    }
    if (ok) ok = wait_warp(kGPdsFree, n_chunks - 1);
    if (ok) {
      // warps 0-3 write dK rows, warps 4-7 dV rows (storage dtype)
      uint32_t acc[D];
      const uint32_t col = kLColAcc + (half ? D : 0);
#pragma unroll
      for (int c = 0; c < D / 16; ++c) tmem_ld16(t_lanes + col + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(acc + 16 * c));
      tmem_wait_ld();
      if (row_ok) {
        int64_t r = ((int64_t)kz * p.Y + ky) * p.X + kx;
        if (p.map) r = p.map[r];
        uint16_t *dst = static_cast<uint16_t *>(half ? p.dvl : p.dkl) + ((int64_t)bg * p.tokens + r) * D;
        uint32_t out[D / 2];
#pragma unroll
        for (int i = 0; i < D / 2; ++i) out[i] = pack2<BF16>(__uint_as_float(acc[2 * i]), __uint_as_float(acc[2 * i + 1]));
#pragma unroll
        for (int v = 0; v < D / 8; ++v)
          reinterpret_cast<uint4 *>(dst)[v] = make_uint4(out[4 * v], out[4 * v + 1], out[4 * v + 2], out[4 * v + 3]);
      }
    }
    tmem_wait_st();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool BF16, int R>
int launch_lkv_t(const StencilBwdArgs &a, cudaStream_t stream) {
  using G = BGeo<R>;
  constexpr int kHY = G::kHY, kHX = G::kHX;
  using C = LkvCfg<D, G::kKeys>;
  const int Z = a.grid[0], Y = a.grid[1], X = a.grid[2];
  const uint64_t es = 2;
  const uint64_t bh = (uint64_t)a.batch * a.heads, bgs = (uint64_t)a.batch * a.kv_heads;
  CUtensorMap tkl, tvl, tq, tdo;
  {
    const uint64_t dims[5] = {(uint64_t)D, (uint64_t)X, (uint64_t)Y, (uint64_t)a.k_planes, bgs};
    const uint64_t strides[4] = {D * es, X * D * es, (uint64_t)Y * X * D * es,
                                 (uint64_t)a.k_planes * Y * X * D * es};
    const uint32_t box[5] = {16, kTX, kTY, kTZ, 1};
    if (int st = encode_operand(&tkl, a.dtype, a.kl, 5, dims, strides, box)) return st;
    if (int st = encode_operand(&tvl, a.dtype, a.vl, 5, dims, strides, box)) return st;
  }
  {
    const uint64_t dims[5] = {(uint64_t)D, (uint64_t)X, (uint64_t)Y, (uint64_t)a.x_planes, bh};
    const uint64_t strides[4] = {D * es, X * D * es, (uint64_t)Y * X * D * es,
                                 (uint64_t)a.x_planes * Y * X * D * es};
    const uint32_t box[5] = {16, kHX, kHY, 1, 1};
    if (int st = encode_operand(&tq, a.dtype, a.q_halo, 5, dims, strides, box)) return st;
    if (int st = encode_operand(&tdo, a.dtype, a.dol_halo, 5, dims, strides, box)) return st;
  }
  LkvParams p{};
  p.Z = Z;
  p.Y = Y;
  p.X = X;
  p.tiles_z = (Z + kTZ - 1) / kTZ;
  p.tiles_y = (Y + kTY - 1) / kTY;
  p.tiles_x = (X + kTX - 1) / kTX;
  p.heads = a.heads;
  p.kv_heads = a.kv_heads;
  p.rep = a.heads / a.kv_heads;
  p.tokens = (int64_t)Z * Y * X;
  p.Zg = a.global_planes;
  p.cz0 = a.q_z0;
  p.kz0 = a.k_z0;
  p.xz0 = a.x_z0;
  p.xtokens = (int64_t)a.x_planes * Y * X;
  p.sc = kLog2e / sqrtf((float)D);
  p.inv_sqrt_d = 1.f / sqrtf((float)D);
  p.lse_l = a.lse_l_halo;
  p.delta_l = a.delta_l_halo;
  p.map = a.raster_to_packed;
  p.dkl = a.dkl;
  p.dvl = a.dvl;
  const int64_t units = (int64_t)bgs * p.tiles_z * p.tiles_y * p.tiles_x;
  if (units <= 0) return P3D_OK;
  if (units > 0x7fffffff) return fail(P3D_ERR_UNSUPPORTED, "too many tiles");
  auto kernel = stencil_bwd_dkv_kernel<D, BF16, R>;
  static size_t seen[kMaxDevices] = {};
  if (int st = smem_optin(kernel, C::kSmemBytes, seen)) return st;
  kernel<<<(unsigned)units, kThreads, C::kSmemBytes, stream>>>(tkl, tvl, tq, tdo, p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

}  // namespace

template <int R>
static int launch_dq_radius(const StencilBwdArgs &a, cudaStream_t s) {
  const bool bf16 = a.dtype == P3D_BF16;
  switch (a.head_dim) {
    case 16: return bf16 ? launch_dq_t<16, true, R>(a, s) : launch_dq_t<16, false, R>(a, s);
    case 32: return bf16 ? launch_dq_t<32, true, R>(a, s) : launch_dq_t<32, false, R>(a, s);
    case 48: return bf16 ? launch_dq_t<48, true, R>(a, s) : launch_dq_t<48, false, R>(a, s);
    case 64: return bf16 ? launch_dq_t<64, true, R>(a, s) : launch_dq_t<64, false, R>(a, s);
    default: return fail(P3D_ERR_UNSUPPORTED, "stencil backward: head_dim %d", a.head_dim);
  }
}

int launch_stencil_bwd_dq(const StencilBwdArgs &a, cudaStream_t s) {
  switch (a.radius) {
    case 1: return launch_dq_radius<1>(a, s);
    case 2: return launch_dq_radius<2>(a, s);
    default: return fail(P3D_ERR_UNSUPPORTED, "stencil backward: radius %d", a.radius);
  }
}

// Query-chunk splits of the global dSK / dSV kernel: a CTA count that fills whole waves
// (at least four when the work allows), every split non-empty.
void global_dkv_tc_splits(int batch, int heads, int kv_heads, int tokens, int summaries, int sm_count, int *splits,
                          int *per_split) {
  const int64_t base = (int64_t)batch * kv_heads * ((summaries + kGRows - 1) / kGRows);
  const int64_t total = (int64_t)(heads / kv_heads) * ((tokens + kGCols - 1) / kGCols);
  const int sms = sm_count > 0 ? sm_count : 148;
  int best_s = 1;
  double best_eff = -1.0;
  for (int s = 1; s <= 64 && s <= total; ++s) {
    const int64_t per = (total + s - 1) / s;
    if (s > 1 && per < 8) break;
    const int64_t s_eff = (total + per - 1) / per;
    const int64_t ctas = base * s_eff;
    const int64_t waves = (ctas + sms - 1) / sms;
    const double eff = (double)ctas / (double)(waves * sms);
    if (ctas >= 4 * sms && eff >= 0.9) {
      best_s = (int)s_eff;
      break;
    }
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best_s = (int)s_eff;
    }
  }
  *per_split = (int)((total + best_s - 1) / best_s);
  *splits = (int)((total + *per_split - 1) / *per_split);
}

bool global_dkv_tc_supported(int dtype, int head_dim, int summaries) {
  if (dtype != P3D_BF16 && dtype != P3D_F16) return false;
  if (head_dim != 16 && head_dim != 32 && head_dim != 48 && head_dim != 64) return false;
  if (summaries < 2) return false;
  DeviceInfo info;
  return device_info(&info) == P3D_OK && info.major == 10;
}

int launch_global_dkv_tc(const GlobalDkvArgs &a, cudaStream_t s) {
  const bool bf16 = a.dtype == P3D_BF16;
  switch (a.head_dim) {
    case 16: return bf16 ? launch_gkv_t<16, true>(a, s) : launch_gkv_t<16, false>(a, s);
    case 32: return bf16 ? launch_gkv_t<32, true>(a, s) : launch_gkv_t<32, false>(a, s);
    case 48: return bf16 ? launch_gkv_t<48, true>(a, s) : launch_gkv_t<48, false>(a, s);
    case 64: return bf16 ? launch_gkv_t<64, true>(a, s) : launch_gkv_t<64, false>(a, s);
    default: return fail(P3D_ERR_UNSUPPORTED, "global dSK/dSV: head_dim %d", a.head_dim);
  }
}

template <int R>
static int launch_dkv_radius(const StencilBwdArgs &a, cudaStream_t s) {
  const bool bf16 = a.dtype == P3D_BF16;
  switch (a.head_dim) {
    case 16: return bf16 ? launch_lkv_t<16, true, R>(a, s) : launch_lkv_t<16, false, R>(a, s);
    case 32: return bf16 ? launch_lkv_t<32, true, R>(a, s) : launch_lkv_t<32, false, R>(a, s);
    case 48: return bf16 ? launch_lkv_t<48, true, R>(a, s) : launch_lkv_t<48, false, R>(a, s);
    case 64: return bf16 ? launch_lkv_t<64, true, R>(a, s) : launch_lkv_t<64, false, R>(a, s);
    default: return fail(P3D_ERR_UNSUPPORTED, "stencil backward: head_dim %d", a.head_dim);
  }
}

int launch_stencil_bwd_dkv(const StencilBwdArgs &a, cudaStream_t s) {
  switch (a.radius) {
    case 1: return launch_dkv_radius<1>(a, s);
    case 2: return launch_dkv_radius<2>(a, s);
    default: return fail(P3D_ERR_UNSUPPORTED, "stencil backward: radius %d", a.radius);
  }
}

int take_bwd_errors(unsigned *flags) {
  unsigned v = 0, zero = 0;
  P3D_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_bwd_errors, sizeof(v)));
  P3D_CUDA_TRY(cudaMemcpyToSymbol(g_bwd_errors, &zero, sizeof(zero)));
  *flags |= v;
  return P3D_OK;
}

}  // namespace p3d
