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
  static_assert(kKeys % 32 == 0, "chunk width must suit the MMA and TMEM shapes");
};
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
    // Lane 0 issues (measured 0.15 ms faster here than the warp-wide elected form the dK / dV
    // kernels use).
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(128, kKeys, BF16, false);  // S and dP: N = kKeys, K-major B
      constexpr uint32_t idesc_dq = idesc_f16(128, D, BF16, true);     // dQ: N = D, B = K read MN-major
      int n_s = 0, n_dp = 0, n_dq = 0;  // commits to kSReady, kDPReady, kDQDone (for the teardown)
      const uint64_t desc_q = desc_sw32(q_smem, 16, 256);
      const uint64_t desc_dol = desc_sw32(dol_smem, 16, 256), desc_dog = desc_sw32(dog_smem, 16, 256);
      const uint64_t desc_k = desc_sw32(ring, 16, 256);          // K / V chunks, K-major
      const uint64_t desc_kmn = desc_sw32(ring, C::kBoxK, 256);  // K chunks read MN-major
      auto stage_off = [&](int c) { return (uint32_t)((c % C::kStages) * C::kStageBytes) >> 4; };
      auto issue_s = [&](int c) {
        const uint64_t bk = desc_k + stage_off(c);
#pragma unroll
        for (int kk = 0; kk < C::kK; ++kk)
          mma_ss(tmem + kColS, desc_q + kk * (C::kBoxQ >> 4), bk + kk * (C::kBoxK >> 4), idesc_s,
                      kk > 0 ? 1u : 0u);
        mma_commit(bar(kSReady));
        ++n_s;
      };
      auto issue_dp = [&](int c) {
        const uint64_t ad = c < kLocalChunks ? desc_dol : desc_dog;
        const uint64_t bv = desc_k + stage_off(c) + (C::kKeyBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < C::kK; ++kk)
          mma_ss(tmem + kColDP, ad + kk * (C::kBoxQ >> 4), bv + kk * (C::kBoxK >> 4), idesc_s,
                      kk > 0 ? 1u : 0u);
        mma_commit(bar(kDPReady));
        ++n_dp;
      };
      auto issue_dq = [&](int c) {
        const uint64_t bk = desc_kmn + stage_off(c);
        const bool first = (c == 0) || (c == kLocalChunks);  // dQ restarts for the global branch
#pragma unroll
        for (int j = 0; j < kKeys / 16; ++j)
          mma_ts(tmem + kColDQ, tmem + kColDP + 8 * j, bk + j * (512 >> 4), idesc_dq,
                      (first && j == 0) ? 0u : 1u);
        mma_commit(bar(kDQDone));
        ++n_dq;
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
      // the drain commit's arrival means every operation completed; then each barrier's last
      // commit has arrived or is about to
      mma_commit(bar(kDrain));
      mbar_wait(bar(kDrain), 0, &g_bwd_errors, kWaitNs, kErrTeardown);
      if (n_s) mbar_wait(bar(kSReady), (n_s - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
      if (n_dp) mbar_wait(bar(kDPReady), (n_dp - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
      if (n_dq) mbar_wait(bar(kDQDone), (n_dq - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
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


// ============================================================================ dK / dV side
//
// Two kernels give the key-side gradients: global_dkv_tc_kernel (summaries, any token order)
// and stencil_bwd_dkv_kernel (the local keys of a complete stencil).  Both put 128 keys (or
// summaries) on the TMEM lanes and stream chunks of 32 queries as columns:
//   S^T = K Q^T, dP^T = V dO^T, P^T = exp(S^T / sqrt(D) - lse), dS^T = P^T (dP^T - Delta),
//   dV += P^T dO,  dK += dS^T Q        (the 1/sqrt(D) of dS multiplies dK once, at the end)
// with P^T and dS^T rounded to the storage dtype for the products (the rounded dS^T operand
// is P^T (dP^T - Delta); the rounding is relative, so it agrees within the dtype's rounding).
//
// They run two CTAs per SM: the tensor cores are fed by one issuing warp per CTA, and
// while one CTA's softmax warps work the other CTA's products run.  Each CTA holds 256 TMEM
// columns: an S^T buffer [0, 64), a dP^T buffer [64, 128), then -- for head_dim <= 48 -- a
// 32-column P^T buffer, then the accumulators dK, dV (D columns each).  The softmax warps
// write dS^T back over the dP^T columns they read, as 16-bit pairs, and P^T into its own
// buffer (or, for head_dim 64, where no room is left, over S^T).  S^T(c) and dP^T(c) commit
// to separate barriers: the warps load S^T, release it (so that, with a separate P^T buffer,
// S^T(c + 1) is issued at once and runs while they exponentiate), then wait for dP^T.  Per
// chunk the MMA warp waits for P^T / dS^T of chunk c, issues its dV / dK products, releases
// the chunk's ring stage, waits for those products to complete (tcgen05.mma operations are
// ordered only when they share an accumulator, and dP^T(c + 1) overwrites dS^T(c)), then
// issues dP^T(c + 1) (and S^T(c + 1) when P^T lives over S^T).  tests/stencil_protocol.py
// (run_ip) replays this barrier protocol with the hardware's parity semantics, tensor-core
// operations completing in order only per accumulator, and each warp's TMEM contents.
//
// Roles: eight softmax warps (warp w serves TMEM lanes 32(w % 4).. and query columns
// [32(w / 4), 32(w / 4) + 32) of a chunk), the TMA producer warp (query chunks by TMA, lse /
// Delta beside them), the MMA warp, which issues warp-wide (every lane runs the loop with the
// same operands and elect.sync picks the issuing lane).  Every wait is bounded.
constexpr uint32_t kKvTmemCols = 256;
constexpr int kKvCols = 64;          // queries per chunk
constexpr int kKvSoft = 8;           // softmax warps
constexpr int kKvW = 4 * kKvCols / kKvSoft;  // columns per softmax warp (32)
constexpr int kKvProducer = kKvSoft, kKvMma = kKvSoft + 1, kKvThreads = 32 * (kKvSoft + 2);
constexpr int kKvMaxStages = 8;
// Of every 8 exp2 pairs of a softmax warp, this many run as the degree-3 polynomial on the
// FMA pipe (exp2_poly2, relative error < 1e-4, far below the 16-bit rounding of P) instead of
// the MUFU: 0 / 2 / 3 / 4 measured 11.06 / 10.96 / 11.14 / 11.23 ms for the config-3 backward.
constexpr int kKvPolyPairs = 2;
static_assert(kKvW == 32, "a softmax warp serves 32 columns (two groups of 16)");

enum KvBar {
  kVKvFull = 0,                            // the K and V (or SK and SV) tiles landed
  kVFull = 1,                              // [stage]: query chunk copies (tx) + the producer's lse / Delta stores
  kVEmpty = kVFull + kKvMaxStages,         // [stage]: committed after the dV / dK products of the chunk it held
  kVSReady = kVEmpty + kKvMaxStages,       // S^T of a chunk complete
  kVSFree = kVSReady + 1,                  // every softmax warp loaded its S^T columns
  kVDPReady = kVSFree + 1,                 // dP^T of a chunk complete
  kVPdsReady = kVDPReady + 1,              // every softmax warp stored its P^T, dS^T of a chunk
  kVAccDone = kVPdsReady + 1,              // the dV / dK products of a chunk complete
  kVAccReady = kVAccDone + 1,              // every product complete: the accumulators are final
  kVNumBars = kVAccReady + 1
};

template <int D>
struct KvCfg {
  // a P^T buffer of its own when it fits beside S^T, dP^T and the accumulators
  static constexpr bool kSepP = 2 * kKvCols + kKvCols / 2 + 2 * D <= (int)kKvTmemCols;
  static constexpr uint32_t kColS = 0, kColDP = kKvCols;
  static constexpr uint32_t kColP = kSepP ? 2 * kKvCols : 0;
  static constexpr uint32_t kColAcc = kSepP ? 2 * kKvCols + kKvCols / 2 : 2 * kKvCols;
  // TMEM column of the P^T pairs of query group j (queries 16j .. 16j + 15), and of the
  // dS^T pairs: softmax warps of column half h store their group g at the start of their
  // own range (dS^T, in-place P^T: 32h + 8g) or packed (separate P^T: 16h + 8g = 8j)
  static constexpr uint32_t p_col(int j) { return kColP + (kSepP ? 8 * j : 32 * (j / 2) + 8 * (j % 2)); }
  static constexpr uint32_t ds_col(int j) { return kColDP + 32 * (j / 2) + 8 * (j % 2); }
  static constexpr int kK = D / 16;
  static constexpr int kBoxT = kRows * 32;       // key / summary tile: 128 rows x 16 channels
  static constexpr int kBoxC = kKvCols * 32;     // query chunk: kKvCols rows x 16 channels
  static constexpr int kTileBytes = kK * kBoxT;
  static constexpr int kChunkBytes = kK * kBoxC;
  static constexpr int kVals = kKvCols * 4;      // lse (or Delta) of one chunk, fp32
  static constexpr int kStageBytes = (2 * kChunkBytes + 2 * kVals + 1023) / 1024 * 1024;
  static constexpr int kFixed = 2 * kTileBytes + 1024;
  // two CTAs per SM (<= 113 KB each), never three (> 76 KB: a third CTA's TMEM allocation
  // would have to wait)
  static constexpr int kMaxSmem = 113 * 1024, kMinSmem = 78 * 1024;
  static constexpr int kRoom = (kMaxSmem - kFixed) / kStageBytes;
  static constexpr int kStages = kRoom > kKvMaxStages ? kKvMaxStages : kRoom;
  static constexpr int kSmemNeed = kFixed + kStages * kStageBytes;
  static constexpr int kSmemBytes = kSmemNeed > kMinSmem ? kSmemNeed : kMinSmem;
  static_assert(kStages >= 2, "the ring must hold the chunk in flight and the next");
  static_assert(kSmemBytes <= kMaxSmem, "shared memory budget");
  static_assert(kColAcc + 2 * D <= kKvTmemCols, "TMEM budget");
};

__device__ __forceinline__ void kv_init(uint64_t *bars, int stages) {
  mbar_init(smem_u32(&bars[kVKvFull]), 1);
  for (int s = 0; s < stages; ++s) {
    mbar_init(smem_u32(&bars[kVFull + s]), 2);
    mbar_init(smem_u32(&bars[kVEmpty + s]), 1);
  }
  mbar_init(smem_u32(&bars[kVSReady]), 1);
  mbar_init(smem_u32(&bars[kVSFree]), kKvSoft);
  mbar_init(smem_u32(&bars[kVDPReady]), 1);
  mbar_init(smem_u32(&bars[kVPdsReady]), kKvSoft);
  mbar_init(smem_u32(&bars[kVAccDone]), 1);
  mbar_init(smem_u32(&bars[kVAccReady]), 1);
  fence_mbar_init();
}

// The producer warp: `tiles()` (lane 0) starts the K / V tile copies on kVKvFull;
// `chunk(c, s, wait_stage)` (whole warp) may issue its lse / Delta loads, then calls
// wait_stage() (false: give up), then fills ring stage s with chunk c -- lane 0 issues the
// copies with their expect_tx, every lane may store lse / Delta -- and returns whether it
// got the stage.
template <int kStages, class Tiles, class Chunk>
__device__ __forceinline__ void kv_producer_role(uint64_t *bars, int n_chunks, int lane, Tiles tiles, Chunk chunk) {
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  if (lane == 0) tiles();
  int issued = 0;
  for (int ch = 0; ch < n_chunks; ++ch) {
    const int s = ch % kStages;
    // kVEmpty[s]: completion ch / kStages - 1, committed after the products of chunk
    // ch - kStages; its next completion needs this stage refilled first
    auto wait_stage = [&]() -> bool {
      bool ok = true;
      if (lane == 0 && ch >= kStages)
        ok = mbar_wait(bar(kVEmpty + s), (ch / kStages - 1) & 1, &g_bwd_errors, kWaitNs, kErrProducer);
      return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    };
    if (!chunk(ch, s, wait_stage)) break;
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(kVFull + s));
    issued = ch + 1;
  }
  if (lane == 0) {  // no copy may still be in flight when the CTA exits
    mbar_wait(bar(kVKvFull), 0, &g_bwd_errors, kWaitNs, kErrTeardown);
    for (int ch = issued > kStages ? issued - kStages : 0; ch < issued; ++ch)
      mbar_wait(bar(kVFull + ch % kStages), (ch / kStages) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
  }
}

// The whole MMA warp: s(c) issues S^T of chunk c, dp(c) its dP^T, acc(c) its dV / dK
// products, with the warp-wide (elected-lane) MMA forms; every lane waits on the barriers.
template <int kStages, bool kSepP, class IssueS, class IssueDP, class Acc>
__device__ __forceinline__ void kv_mma_role(uint64_t *bars, int n_chunks, IssueS s_mma, IssueDP dp_mma, Acc acc) {
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  int n_s = 0, n_dp = 0, n_acc = 0;  // chunks whose S^T, dP^T, products were issued
  auto wait_bar = [&](int b, int completion) -> bool {
    const bool r = mbar_wait(bar(b), completion & 1, &g_bwd_errors, kWaitNs, kErrMma);
    if (!__all_sync(0xffffffffu, r)) return false;
    tc_fence_after();
    return true;
  };
  auto issue_s = [&](int c) {
    s_mma(c);
    mma_commit_warp(bar(kVSReady));
    n_s = c + 1;
  };
  auto issue_dp = [&](int c) {
    dp_mma(c);
    mma_commit_warp(bar(kVDPReady));
    n_dp = c + 1;
  };
  bool ok = wait_bar(kVKvFull, 0) && wait_bar(kVFull, 0);
  if (ok) {
    issue_s(0);
    issue_dp(0);
  }
  for (int c = 0; ok && c < n_chunks; ++c) {
    const bool more = c + 1 < n_chunks;
    if (kSepP && more) {
      // S^T(c + 1) overwrites S^T(c) once every warp holds its columns (sfree: completion c;
      // the warps' next arrivals need S^T(c + 1))
      ok = wait_bar(kVSFree, c) && wait_bar(kVFull + (c + 1) % kStages, (c + 1) / kStages);
      if (!ok) break;
      issue_s(c + 1);
    }
    ok = wait_bar(kVPdsReady, c);  // completion c; the next arrivals need dP^T(c + 1)
    if (!ok) break;
    acc(c);
    mma_commit_warp(bar(kVEmpty + c % kStages));
    mma_commit_warp(bar(kVAccDone));
    n_acc = c + 1;
    if (more) {
      // dP^T(c + 1) (and, with P^T over S^T, S^T(c + 1)) overwrite what the products of
      // chunk c read: they must have completed
      ok = wait_bar(kVAccDone, c);
      if (!kSepP) ok = ok && wait_bar(kVFull + (c + 1) % kStages, (c + 1) / kStages);
      if (!ok) break;
      if (!kSepP) issue_s(c + 1);
      issue_dp(c + 1);
    }
  }
  mma_commit_warp(bar(kVAccReady));
  // drain: the last commit first (every operation then complete), then each barrier's last
  // completion, so that no arrival is in flight when the CTA exits.  kVEmpty[s] was committed
  // once per chunk c < n_acc with c % kStages == s.
  mbar_wait(bar(kVAccReady), 0, &g_bwd_errors, kWaitNs, kErrTeardown);
  if (n_s) mbar_wait(bar(kVSReady), (n_s - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
  if (n_dp) mbar_wait(bar(kVDPReady), (n_dp - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
  if (n_acc) mbar_wait(bar(kVAccDone), (n_acc - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
  for (int s = 0; s < kStages; ++s) {
    const int times = n_acc / kStages + (s < n_acc % kStages ? 1 : 0);
    if (times > 0) mbar_wait(bar(kVEmpty + s), (times - 1) & 1, &g_bwd_errors, kWaitNs, kErrTeardown);
  }
}

// Softmax-warp wait: every lane polls; the warp proceeds only if all lanes saw the phase.
__device__ __forceinline__ bool kv_wait_warp(uint64_t *bars, int b, int completion) {
  // (suspending try_wait, as mbar_wait does: spinning on try_wait or test_wait instead
  // measured 0.3 ms slower over the config-3 backward -- the spinning warps take issue slots)
  const bool r = mbar_wait(smem_u32(&bars[b]), completion & 1, &g_bwd_errors, kWaitNs, kErrSoftmax);
  const bool all = __all_sync(0xffffffffu, r);
  if (all) tc_fence_after();
  return all;
}

// One chunk of a softmax warp, columns [col0, col0 + 32) of its 32 TMEM lanes: wait for S^T,
// load it, release it (sfree), exponentiate, wait for dP^T, load it, form dS^T = P^T (dP^T -
// Delta) and store both as 16-bit pairs (P^T at C::p_col, dS^T at C::ds_col of the warp's
// two query groups).  l, d: the chunk's per-column -lse log2(e) and -Delta in shared memory;
// mask: bit i for column col0 + i, a masked column gives
// exact zeros whatever its inputs; active false: the warp's rows take no query of this
// chunk and store zeros.  Returns false if a wait timed out.
template <class C, bool BF16, bool MASKED>
__device__ __forceinline__ bool kv_chunk(uint64_t *bars, int ch, uint32_t t_lanes, int col0, const float *l,
                                         const float *d, float sc, uint32_t mask, bool active) {
  float pf[kKvW];
  if (!kv_wait_warp(bars, kVSReady, ch)) return false;
  if (active) {
#pragma unroll
    for (int g = 0; g < kKvW / 16; ++g) {  // S^T in groups of 16 columns, exponentiated as loaded
      uint32_t sv[16];
      tmem_ld16(t_lanes + C::kColS + col0 + 16 * g, sv);
      tmem_wait_ld();
      if (g + 1 == kKvW / 16) {  // every column loaded: S^T may be overwritten
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(smem_u32(&bars[kVSFree]));
      }
      const float2 sc2 = make_float2(sc, sc);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = 16 * g + 2 * i;
        const float2 l2 = *reinterpret_cast<const float2 *>(l + col0 + k);
        const float2 x = fma2(make_float2(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])), sc2, l2);
        // kKvPolyPairs of every 8 pairs take the FMA-pipe polynomial, the rest the MUFU
        const float2 e = i < 8 - kKvPolyPairs ? make_float2(ex2_approx(x.x), ex2_approx(x.y)) : exp2_poly2(x);
        pf[k] = e.x;
        pf[k + 1] = e.y;
      }
    }
  } else {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(smem_u32(&bars[kVSFree]));
  }
  // dpready(c) also means the products of chunk c - 1 completed: the P^T buffer is free
  if (!kv_wait_warp(bars, kVDPReady, ch)) return false;
  const int j0 = col0 / 16;  // the warp's first query group
#pragma unroll
  for (int g = 0; g < kKvW / 16; ++g) {
    uint32_t pw[8], dw[8];
    if (active) {
      uint32_t dv[16];
      tmem_ld16(t_lanes + C::kColDP + col0 + 16 * g, dv);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = 16 * g + 2 * i;
        const float2 d2 = *reinterpret_cast<const float2 *>(d + col0 + k);
        float2 pp = make_float2(pf[k], pf[k + 1]);
        float2 dd = mul2(pp, add2(make_float2(__uint_as_float(dv[2 * i]), __uint_as_float(dv[2 * i + 1])), d2));
        if (MASKED) {  // selects, not products
          const bool b0 = (mask >> k) & 1u, b1 = (mask >> (k + 1)) & 1u;
          pp = make_float2(b0 ? pp.x : 0.f, b1 ? pp.y : 0.f);
          dd = make_float2(b0 ? dd.x : 0.f, b1 ? dd.y : 0.f);
        }
        pw[i] = pack2<BF16>(pp.x, pp.y);
        dw[i] = pack2<BF16>(dd.x, dd.y);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) pw[i] = dw[i] = 0u;
    }
    // dS^T group g lands on dP^T columns this warp has already loaded (its own first 16)
    tmem_st8(t_lanes + C::p_col(j0 + g), pw);
    tmem_st8(t_lanes + C::ds_col(j0 + g), dw);
  }
  tmem_wait_st();
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(smem_u32(&bars[kVPdsReady]));
  return true;
}

// The MMAs of one chunk, shared by both kernels: kt the 128-row K (or V) tile, qc the
// chunk's Q (or dO) box, col the TMEM buffer (S^T or dP^T).
template <int D, bool BF16>
__device__ __forceinline__ void kv_issue_scores(uint32_t tmem, uint32_t col, uint32_t kt, uint32_t qc) {
  using C = KvCfg<D>;
  constexpr uint32_t idesc_s = idesc_f16(128, kKvCols, BF16, false);
#pragma unroll
  for (int kk = 0; kk < C::kK; ++kk)
    mma_ss_warp(tmem + col, desc_sw32(kt + kk * C::kBoxT, 16, 256), desc_sw32(qc + kk * C::kBoxC, 16, 256), idesc_s,
                kk > 0 ? 1u : 0u);
}

template <int D, bool BF16>
__device__ __forceinline__ void kv_issue_acc(uint32_t tmem, uint32_t q, uint32_t dov, bool first) {
  using C = KvCfg<D>;
  constexpr uint32_t idesc_acc = idesc_f16(128, D, BF16, true);
  // dV += P^T dO and dK += dS^T Q: A from TMEM (query group j: 16 queries as 8 columns of
  // pairs), B the chunk's dO / Q read MN-major (16 query rows of 32 bytes per step)
#pragma unroll
  for (int j = 0; j < kKvCols / 16; ++j)
    mma_ts_warp(tmem + C::kColAcc + D, tmem + C::p_col(j), desc_sw32(dov + j * 512, C::kBoxC, 256), idesc_acc,
                (first && j == 0) ? 0u : 1u);
#pragma unroll
  for (int j = 0; j < kKvCols / 16; ++j)
    mma_ts_warp(tmem + C::kColAcc, tmem + C::ds_col(j), desc_sw32(q + j * 512, C::kBoxC, 256), idesc_acc,
                (first && j == 0) ? 0u : 1u);
}

// The epilogue's accumulator rows: warps 0-3 take dK (scaled by 1/sqrt(D)), warps 4-7 dV.
template <int D>
__device__ __forceinline__ void kv_load_acc(uint32_t t_lanes, int half, uint32_t (&acc)[D]) {
#pragma unroll
  for (int c = 0; c < D / 16; ++c)
    tmem_ld16(t_lanes + KvCfg<D>::kColAcc + (half ? D : 0) + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(acc + 16 * c));
  tmem_wait_ld();
}

// ------------------------------------------------------------------ global dSK / dSV
//
// Restates the summary-gradient half of the global branch (kernels.py:210-239): a CTA owns
// one (batch, kv-head), a tile of 128 summaries and one split of the query chunks (every
// query head of the group); splits write fp32 partials [B*G, splits, M, D] that a
// fixed-order reduction sums.  The global branch ignores the geometry, so this kernel serves
// any token order.  Summary rows past M read zeros and are not written; query columns past
// N are masked (P = 0).
constexpr int kGRows = 128;      // summaries per tile
constexpr int kGCols = kKvCols;  // queries per chunk

struct GkvParams {
  int heads, kv_heads, rep, tokens, summaries, m_tiles, splits, q_chunks, per_split;
  float sc, inv_sqrt_d;
  const float *lse_g, *delta_g;  // [B*H, N]
  float *dk_part, *dv_part;      // [B*G, splits, M, D]
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kKvThreads, 2)
    global_dkv_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                         const __grid_constant__ CUtensorMap tsk, const __grid_constant__ CUtensorMap tsv,
                         const GkvParams p) {
  using C = KvCfg<D>;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kVNumBars];
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

  if (tid == 0) kv_init(bars, kStages);
  if (warp == kKvMma) {
    tmem_alloc(smem_u32(&tmem_holder), kKvTmemCols);
    tmem_relinquish();
  }
  if (warp == kKvProducer && lane == 0) {
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
  auto stage_of = [&](int c) { return ring + (uint32_t)((c % kStages) * C::kStageBytes); };

  if (warp == kKvProducer) {
    auto tiles = [&]() {
      const uint32_t full = smem_u32(&bars[kVKvFull]);
      mbar_expect_tx(full, 2 * C::kTileBytes);
      for (int c = 0; c < C::kK; ++c) {
        tma_load_3d(sk_smem + c * C::kBoxT, &tsk, full, 16 * c, m0, bg);
        tma_load_3d(sv_smem + c * C::kBoxT, &tsv, full, 16 * c, m0, bg);
      }
    };
    auto chunk = [&](int ch, int s, auto wait_stage) -> bool {
      const uint32_t stage = ring + s * C::kStageBytes, full = smem_u32(&bars[kVFull + s]);
      const int bh = chunk_head(ch), n0 = chunk_row0(ch);
      const int64_t r0 = (int64_t)bh * p.tokens + n0;
      const uint32_t rows = (uint32_t)min(kGCols, p.tokens - n0);
      // -lse log2(e) and -Delta of the chunk's queries, formed once here rather than by every
      // softmax lane (columns past N: zeros, masked there).  The loads go out before the
      // stage wait and are first used after the chunk's copies are issued.
      float l[kGCols / 32], dl[kGCols / 32];
#pragma unroll
      for (int k = 0; k < kGCols / 32; ++k) {
        const int j = lane + 32 * k;
        l[k] = -0.f;
        dl[k] = -0.f;
        if (j < (int)rows) {
          l[k] = __ldg(p.lse_g + r0 + j);
          dl[k] = __ldg(p.delta_g + r0 + j);
        }
      }
      if (!wait_stage()) return false;
      if (lane == 0) {
        mbar_expect_tx(full, 2 * C::kChunkBytes);
        for (int c = 0; c < C::kK; ++c) {
          tma_load_3d(stage + c * C::kBoxC, &tq, full, 16 * c, n0, bh);
          tma_load_3d(stage + C::kChunkBytes + c * C::kBoxC, &tdo, full, 16 * c, n0, bh);
        }
      }
      float *vals = reinterpret_cast<float *>(ring_ptr + (size_t)s * C::kStageBytes + 2 * C::kChunkBytes);
#pragma unroll
      for (int k = 0; k < kGCols / 32; ++k) {
        vals[lane + 32 * k] = -l[k] * kLog2e;
        vals[kGCols + lane + 32 * k] = -dl[k];
      }
      return true;
    };
    kv_producer_role<kStages>(bars, n_chunks, lane, tiles, chunk);
  } else if (warp == kKvMma) {
    kv_mma_role<kStages, C::kSepP>(
        bars, n_chunks, [&](int c) { kv_issue_scores<D, BF16>(tmem, C::kColS, sk_smem, stage_of(c)); },
        [&](int c) { kv_issue_scores<D, BF16>(tmem, C::kColDP, sv_smem, stage_of(c) + C::kChunkBytes); },
        [&](int c) { kv_issue_acc<D, BF16>(tmem, stage_of(c), stage_of(c) + C::kChunkBytes, c == 0); });
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3, half = warp >> 2, col0 = half * kKvW;
    const uint32_t t_lanes = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sc = p.sc;
    bool ok = true;
    for (int ch = 0; ch < n_chunks && ok; ++ch) {
      const float *vals =
          reinterpret_cast<const float *>(ring_ptr + (size_t)(ch % kStages) * C::kStageBytes + 2 * C::kChunkBytes);
      const int valid = min(kGCols, p.tokens - chunk_row0(ch)) - col0;  // this warp's columns inside the volume
      if (valid >= kKvW) {
        ok = kv_chunk<C, BF16, false>(bars, ch, t_lanes, col0, vals, vals + kGCols, sc, ~0u, true);
      } else {  // columns past the volume may hold stale lse / Delta: masked to exact zeros
        const uint32_t mask = valid > 0 ? ~0u >> (32 - valid) : 0u;
        ok = kv_chunk<C, BF16, true>(bars, ch, t_lanes, col0, vals, vals + kGCols, sc, mask, valid > 0);
      }
    }
    if (ok) ok = kv_wait_warp(bars, kVAccReady, 0);
    if (ok) {
      const int m = m0 + quarter * 32 + lane;
      uint32_t acc[D];
      kv_load_acc<D>(t_lanes, half, acc);
      if (m < p.summaries) {
        float *dst = (half ? p.dv_part : p.dk_part) + (((int64_t)bg * p.splits + split) * p.summaries + m) * D;
        const float scale = half ? 1.f : p.inv_sqrt_d;
#pragma unroll
        for (int v = 0; v < D / 4; ++v)
          reinterpret_cast<float4 *>(dst)[v] =
              make_float4(__uint_as_float(acc[4 * v]) * scale, __uint_as_float(acc[4 * v + 1]) * scale,
                          __uint_as_float(acc[4 * v + 2]) * scale, __uint_as_float(acc[4 * v + 3]) * scale);
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kKvMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kKvTmemCols);
  }
}

template <int D, bool BF16>
int launch_gkv_t(const GlobalDkvArgs &a, cudaStream_t stream) {
  using C = KvCfg<D>;
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
  p.sc = kLog2e / sqrtf((float)D);
  p.inv_sqrt_d = 1.f / sqrtf((float)D);
  p.lse_g = a.lse_g;
  p.delta_g = a.delta_g;
  p.dk_part = a.dk_part;
  p.dv_part = a.dv_part;
  const int64_t units = (int64_t)bgs * p.m_tiles * p.splits;
  if (units <= 0) return P3D_OK;
  if (units > 0x7fffffff) return fail(P3D_ERR_UNSUPPORTED, "too many tiles");
  const int64_t total = (int64_t)p.rep * p.q_chunks;
  if (p.per_split < 1 || (int64_t)p.splits * p.per_split < total || (int64_t)(p.splits - 1) * p.per_split >= total)
    return fail(P3D_ERR_INVALID_ARGUMENT, "global dSK/dSV: splits do not cover the query chunks");
  auto kernel = global_dkv_tc_kernel<D, BF16>;
  static size_t seen[kMaxDevices] = {};
  if (int st = smem_optin(kernel, C::kSmemBytes, seen)) return st;
  kernel<<<(unsigned)units, kKvThreads, C::kSmemBytes, stream>>>(tq, tdo, tsk, tsv, p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}


// ------------------------------------------------------------------ local dK / dV
//
// Restates the key-gradient half of the local branch (kernels.py:154-176; stencil.py:91-147
// with QUERY false) on tensor cores.  A CTA owns one (batch, kv-head) and an 8 x 4 x 4 (z, y,
// x) box of 128 keys (TMEM lanes in (z, y, x) order, so softmax warp w holds key planes
// 2(w % 4) and 2(w % 4) + 1 of the box) and streams, for every query head of the group, the
// 8 + 2R query planes z0 - R .. z0 + 7 + R of its neighbourhood.  A plane is the (4 + 2R) x
// (4 + 2R) window of queries around the box, taken as one chunk (64 queries at radius 2; 36,
// padded, at radius 1) or, with 32-query chunks, as two of (2 + R) rows each.  The
// neighbourhood is symmetric (key j is
// in query i's clipped cube iff i is in j's), so a key takes a query iff both lie in the
// volume and |dz|, |dy|, |dx| <= R.  Each CTA writes its own keys' dK / dV in the storage
// dtype: no atomics, no partials.
template <int R>
struct KGeo {
  static constexpr int kBZ = 8, kBY = 4, kBX = 4;
  static constexpr int kHY = kBY + 2 * R, kHX = kBX + 2 * R;
  static constexpr int kParts = kHY * kHX <= kKvCols ? 1 : 2;  // chunks per plane
  static constexpr int kRowsH = kHY / kParts;           // window rows per chunk
  static constexpr int kWin = kRowsH * kHX;             // queries per chunk
  static constexpr int kPlanes = kBZ + 2 * R;           // 12, 10
  static_assert(kWin <= kKvCols, "a chunk's window rows must fit its columns");
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
__global__ void __launch_bounds__(kKvThreads, 2)
    stencil_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tkl, const __grid_constant__ CUtensorMap tvl,
                           const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                           const LkvParams p) {
  using G = KGeo<R>;
  constexpr int kHX = G::kHX, kRowsH = G::kRowsH, kWin = G::kWin, kPlanes = G::kPlanes;
  using C = KvCfg<D>;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kVNumBars];
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
  const int x0 = tx * G::kBX, y0 = ty * G::kBY, z0 = tz * G::kBZ;
  constexpr int kParts = G::kParts;
  const int n_chunks = p.rep * kPlanes * kParts;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t k_smem = base, v_smem = base + C::kTileBytes;
  const uint32_t ring = base + 2 * C::kTileBytes;
  uint8_t *ring_ptr = smem_raw + (base - raw) + 2 * C::kTileBytes;

  if (tid == 0) kv_init(bars, kStages);
  if constexpr (kWin < kKvCols) {
    // the query windows fill kWin of the kKvCols rows of each box: the rest reads as zeros
    uint4 *ring_v = reinterpret_cast<uint4 *>(ring_ptr);
    for (int i = tid; i < kStages * C::kStageBytes / 16; i += kKvThreads) ring_v[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (warp == kKvMma) {
    tmem_alloc(smem_u32(&tmem_holder), kKvTmemCols);
    tmem_relinquish();
  }
  if (warp == kKvProducer && lane == 0) {
    prefetch_tmap(&tkl);
    prefetch_tmap(&tvl);
    prefetch_tmap(&tq);
    prefetch_tmap(&tdo);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;
  // chunk c: query head b*H + g*rep + c / (kParts kPlanes), query plane z0 - R + (c /
  // kParts) % kPlanes, window rows kRowsH (c % kParts) ..
  auto chunk_head = [&](int c) { return b * p.heads + g * p.rep + c / (kParts * kPlanes); };
  auto chunk_plane = [&](int c) { return (c / kParts) % kPlanes; };  // relative to z0 - R
  auto stage_of = [&](int c) { return ring + (uint32_t)((c % kStages) * C::kStageBytes); };

  if (warp == kKvProducer) {
    auto tiles = [&]() {
      const uint32_t full = smem_u32(&bars[kVKvFull]);
      mbar_expect_tx(full, 2 * C::kTileBytes);
      for (int c = 0; c < C::kK; ++c) {
        tma_load_5d(k_smem + c * C::kBoxT, &tkl, full, 16 * c, x0, y0, p.cz0 + z0 - p.kz0, bg);
        tma_load_5d(v_smem + c * C::kBoxT, &tvl, full, 16 * c, x0, y0, p.cz0 + z0 - p.kz0, bg);
      }
    };
    auto chunk = [&](int ch, int s, auto wait_stage) -> bool {
      const uint32_t stage = ring + s * C::kStageBytes, full = smem_u32(&bars[kVFull + s]);
      const int bh = chunk_head(ch), zp = p.cz0 + z0 - R + chunk_plane(ch), hy0 = kRowsH * (ch % kParts);
      // lse and Delta of the chunk's queries (column j: window row hy0 + j / kHX, column
      // j % kHX); +inf and -0 outside the volume and on the padding columns (P = 0).  The loads
      // go out before the stage wait and are first used after the chunk's copies are issued,
      // so the copies do not wait for them.
      constexpr int kPer = kKvCols / 32;
      float l[kPer], dl[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int j = lane + 32 * k;
        const int qy = y0 - R + hy0 + j / kHX, qx = x0 - R + j % kHX;
        const bool in = j < kWin && zp >= 0 && zp < p.Zg && qy >= 0 && qy < p.Y && qx >= 0 && qx < p.X;
        l[k] = __builtin_huge_valf();
        dl[k] = -0.f;
        if (in) {
          int64_t r = ((int64_t)(zp - p.xz0) * p.Y + qy) * p.X + qx;
          if (p.map) r = __ldg(p.map + r);
          const int64_t row = (int64_t)bh * p.xtokens + r;
          l[k] = __ldg(p.lse_l + row);
          dl[k] = __ldg(p.delta_l + row);
        }
      }
      if (!wait_stage()) return false;
      if (lane == 0) {
        mbar_expect_tx(full, 2 * C::kK * kWin * 32);
        for (int c = 0; c < C::kK; ++c) {
          tma_load_5d(stage + c * C::kBoxC, &tq, full, 16 * c, x0 - R, y0 - R + hy0, zp - p.xz0, bh);
          tma_load_5d(stage + C::kChunkBytes + c * C::kBoxC, &tdo, full, 16 * c, x0 - R, y0 - R + hy0, zp - p.xz0,
                      bh);
        }
      }
      float *vals = reinterpret_cast<float *>(ring_ptr + (size_t)s * C::kStageBytes + 2 * C::kChunkBytes);
#pragma unroll
      for (int k = 0; k < kPer; ++k) {  // -lse log2(e) (-inf where masked) and -Delta
        vals[lane + 32 * k] = -l[k] * kLog2e;
        vals[kKvCols + lane + 32 * k] = -dl[k];
      }
      return true;
    };
    kv_producer_role<kStages>(bars, n_chunks, lane, tiles, chunk);
  } else if (warp == kKvMma) {
    kv_mma_role<kStages, C::kSepP>(
        bars, n_chunks, [&](int c) { kv_issue_scores<D, BF16>(tmem, C::kColS, k_smem, stage_of(c)); },
        [&](int c) { kv_issue_scores<D, BF16>(tmem, C::kColDP, v_smem, stage_of(c) + C::kChunkBytes); },
        [&](int c) { kv_issue_acc<D, BF16>(tmem, stage_of(c), stage_of(c) + C::kChunkBytes, c == 0); });
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3, half = warp >> 2, col0 = half * kKvW;
    const uint32_t t_lanes = tmem + ((uint32_t)(quarter * 32) << 16);
    const int zl = 2 * quarter + (lane >> 4), kyl = (lane >> 2) & 3, kxl = lane & 3;  // key within the box
    const int kz = z0 + zl, ky = y0 + kyl, kx = x0 + kxl;
    const bool row_ok = kz < p.Z && ky < p.Y && kx < p.X;
    // this warp's chunk columns inside the key's (y, x) square, per chunk of a plane (bit
    // i: column col0 + i)
    uint32_t mask0 = 0u, mask1 = 0u;
#pragma unroll
    for (int hh = 0; hh < kParts; ++hh)
#pragma unroll
      for (int i = 0; i < kKvW; ++i) {
        const int j = col0 + i, hy = kRowsH * hh + j / kHX, hx = j % kHX;
        if (row_ok && j < kWin && (unsigned)(hy - kyl) <= 2u * R && (unsigned)(hx - kxl) <= 2u * R)
          (hh ? mask1 : mask0) |= 1u << i;
      }
    const float sc = p.sc;
    bool ok = true;
    for (int ch = 0; ch < n_chunks && ok; ++ch) {
      const int pl = chunk_plane(ch);  // query plane z0 - R + pl
      const float *vals =
          reinterpret_cast<const float *>(ring_ptr + (size_t)(ch % kStages) * C::kStageBytes + 2 * C::kChunkBytes);
      // the plane reaches one of the warp's key planes (warp-uniform); lanes of the other plane
      // take the chunk through a zero mask
      const bool active = (unsigned)(pl - 2 * quarter) <= 2u * R + 1u;
      const uint32_t m = (unsigned)(pl - zl) <= 2u * R ? ((ch % kParts) ? mask1 : mask0) : 0u;
      ok = kv_chunk<C, BF16, true>(bars, ch, t_lanes, col0, vals, vals + kKvCols, sc, m, active);
    }
    if (ok) ok = kv_wait_warp(bars, kVAccReady, 0);
    if (ok) {
      int64_t r = ((int64_t)kz * p.Y + ky) * p.X + kx;
      if (row_ok && p.map) r = p.map[r];
      uint32_t acc[D];
      kv_load_acc<D>(t_lanes, half, acc);
      if (row_ok) {  // storage dtype; warps 0-3 write dK (scaled by 1/sqrt(D)), 4-7 dV
        const float scale = half ? 1.f : p.inv_sqrt_d;
        uint16_t *dst = static_cast<uint16_t *>(half ? p.dvl : p.dkl) + ((int64_t)bg * p.tokens + r) * D;
        uint32_t out[D / 2];
#pragma unroll
        for (int i = 0; i < D / 2; ++i)
          out[i] = pack2<BF16>(__uint_as_float(acc[2 * i]) * scale, __uint_as_float(acc[2 * i + 1]) * scale);
#pragma unroll
        for (int v = 0; v < D / 8; ++v)
          reinterpret_cast<uint4 *>(dst)[v] = make_uint4(out[4 * v], out[4 * v + 1], out[4 * v + 2], out[4 * v + 3]);
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kKvMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kKvTmemCols);
  }
}

template <int D, bool BF16, int R>
int launch_lkv_t(const StencilBwdArgs &a, cudaStream_t stream) {
  using G = KGeo<R>;
  using C = KvCfg<D>;
  const int Z = a.grid[0], Y = a.grid[1], X = a.grid[2];
  const uint64_t es = 2;
  const uint64_t bh = (uint64_t)a.batch * a.heads, bgs = (uint64_t)a.batch * a.kv_heads;
  CUtensorMap tkl, tvl, tq, tdo;
  {
    const uint64_t dims[5] = {(uint64_t)D, (uint64_t)X, (uint64_t)Y, (uint64_t)a.k_planes, bgs};
    const uint64_t strides[4] = {D * es, X * D * es, (uint64_t)Y * X * D * es,
                                 (uint64_t)a.k_planes * Y * X * D * es};
    const uint32_t box[5] = {16, G::kBX, G::kBY, G::kBZ, 1};
    if (int st = encode_operand(&tkl, a.dtype, a.kl, 5, dims, strides, box)) return st;
    if (int st = encode_operand(&tvl, a.dtype, a.vl, 5, dims, strides, box)) return st;
  }
  {
    const uint64_t dims[5] = {(uint64_t)D, (uint64_t)X, (uint64_t)Y, (uint64_t)a.x_planes, bh};
    const uint64_t strides[4] = {D * es, X * D * es, (uint64_t)Y * X * D * es,
                                 (uint64_t)a.x_planes * Y * X * D * es};
    const uint32_t box[5] = {16, G::kHX, G::kRowsH, 1, 1};  // one chunk's window rows
    if (int st = encode_operand(&tq, a.dtype, a.q_halo, 5, dims, strides, box)) return st;
    if (int st = encode_operand(&tdo, a.dtype, a.dol_halo, 5, dims, strides, box)) return st;
  }
  LkvParams p{};
  p.Z = Z;
  p.Y = Y;
  p.X = X;
  p.tiles_z = (Z + G::kBZ - 1) / G::kBZ;
  p.tiles_y = (Y + G::kBY - 1) / G::kBY;
  p.tiles_x = (X + G::kBX - 1) / G::kBX;
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
  kernel<<<(unsigned)units, kKvThreads, C::kSmemBytes, stream>>>(tkl, tvl, tq, tdo, p);
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
  const int sms = 2 * (sm_count > 0 ? sm_count : 148);  // two CTAs per SM
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
