// Stage (c): fused local + global attention forward on tensor cores (tcgen05 / TMEM / TMA).
//
// Restates reference.py:20-31 (and the Triton _local_fwd/_global_fwd pair,
// kernels.py:44-103) for a complete radius-2 voxel stencil in bf16 / f16:
//   y = sl * softmax_local(q kl^T / sqrt(D)) vl + (gate * sg) * softmax_global(q sk^T / sqrt(D)) sv
//
// Work unit (one CTA): one (batch, head) and a 4x4x8 (z, y, x) tile of 128 queries.
// Rows are ordered (z, y, x), so softmax warp w owns query plane z = w and TMEM lanes
// 32w..32w+31.  Two CTAs share an SM (each owns 256 TMEM columns and its own MMA issuer:
// an issuing thread blocks ~60 cycles per tcgen05.mma and ~140 per commit, so two issuers
// per SM double the rate at which the tensor pipe is fed).
//
// Chunk sequence, 96 keys each:
//   chunks 0..7   local: halo plane z-2+c of the tile, its 8x12 (y, x) window.  A key
//                 is used iff it lies in the query's 5x5x5 cube and in the volume
//                 (coordinate test, no neighbour table).  A warp whose query plane is
//                 more than 2 planes away writes a zero P block.
//   chunks 8..    global: 96 summaries per chunk.
// TMEM (256 columns): two 96-column S buffers and one accumulator O.  The QK^T MMA of
// chunk c+2 and the PV MMA of chunk c run while the softmax warps work on chunk c+1.  O
// holds the local accumulator during chunks 0..7; when they are done the normalised
// local output is parked in shared memory, rounded to the storage dtype as the
// reference rounds it before the mix, and O then accumulates the global branch.
// Two independent online softmaxes (max / sum per row in registers, conditional
// rescale of O only when the running max grows by > 2^8).  The epilogue normalises the
// global branch, mixes and writes y (and optionally ol, og, lse_l, lse_g) through the
// raster->packed row map.
//
// Roles: warps 0-3 softmax, warp 4 TMA producer, warp 5 MMA issuer (one thread).
// Operands live in shared memory in the SWIZZLE_32B layout: Q / K are K-major boxes of
// 16 channels, V is the same bytes read MN-major; P goes back into its S buffer in TMEM
// as bf16/f16 pairs and feeds the PV MMA as the TMEM A operand.  Every mbarrier wait is
// bounded.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace p3d {
namespace {
using namespace sm100;

__device__ unsigned g_fwd_errors = 0;  // failure bits of the kernels in this file

constexpr int kTZ = 4, kTY = 4, kTX = 8;            // one 128-row query tile
constexpr int kRows = 128;                          // queries per tile
constexpr int kThreads = 192;
constexpr int kProducerWarp = 4, kMmaWarp = 5;
constexpr uint32_t kTmemCols = 256;                 // two CTAs per SM
constexpr float kNegInf = -__builtin_huge_valf();
constexpr uint64_t kWaitNs = 2000000000ull;        // every mbarrier wait gives up after 2 s

// Chunk geometry of a radius-R stencil (R = 1 or 2): a local chunk is one halo plane of the
// tile, a kHY x kHX (y, x) window; chunks are kKeys wide (the window rounded up to 32 keys;
// the padding rows of every ring stage are zero and masked) and global chunks take kKeys
// summaries.  TMEM: S buffers [0, kKeys) and [kKeys, 2 kKeys), O [2 kKeys, 2 kKeys + D).
template <int R>
struct Geo {
  static constexpr int kR = R;
  static constexpr int kHY = kTY + 2 * R, kHX = kTX + 2 * R, kHZ = kTZ + 2 * R;
  static constexpr int kWin = kHY * kHX;                // 96 (R = 2), 60 (R = 1)
  static constexpr int kKeys = (kWin + 31) / 32 * 32;   // 96, 64
  static constexpr int kLocalChunks = kHZ;              // 8, 6 halo planes per tile
  static constexpr int kSumRows = kKeys;                // summaries per global chunk
  static constexpr uint32_t kSBuf = kKeys, kColO = 2 * kKeys;
  static_assert(kKeys % 32 == 0 && kKeys <= 96, "chunk size must suit the MMA, TMEM and register budgets");
};

template <int D, int KEYS>
struct Cfg {
  static constexpr int kK = D / 16;                 // 16-channel boxes per row
  static constexpr int kBoxQ = kRows * 32;          // one box = rows x 32 bytes
  static constexpr int kBoxK = KEYS * 32;           // 3072 (96 keys), 2048 (64)
  static constexpr int kQBytes = kK * kBoxQ;        // the query tile
  static constexpr int kKeyBytes = kK * kBoxK;      // one chunk of K (or V)
  static constexpr int kStageBytes = (2 * kKeyBytes + 1023) / 1024 * 1024;  // K, V
  static constexpr int kOlBytes = kRows * D * 2;    // parked local output
  static constexpr int kFixed = kQBytes + kOlBytes + 1024;
  // Two CTAs per SM: at most 113 KB each; and more than a third of the SM's 228 KB, so
  // that a third CTA (whose TMEM allocation would have to wait) never lands on an SM.
  static constexpr int kMaxSmem = 113 * 1024, kMinSmem = 78 * 1024;
  // 3 or 4 stages: at least chunks c .. c+2 resident (S of chunk c+2 is issued while PV of
  // chunk c may still read its stage); at most 4, the size of the per-stage barrier arrays.
  static constexpr int kRoom = (kMaxSmem - kFixed) / kStageBytes;
  static constexpr int kStages = kRoom > 4 ? 4 : kRoom;
  static constexpr int kSmemNeed = kFixed + kStages * kStageBytes;
  static constexpr int kSmemBytes = kSmemNeed > kMinSmem ? kSmemNeed : kMinSmem;
  static_assert(kStages >= 3 && kStages <= 4, "the ring must hold chunks c .. c+2");
  static_assert(kSmemBytes <= kMaxSmem, "shared memory budget");
};

// S(c) is complete when its commit arrives: S(0), S(1) commit to kSReady[c], and S(c),
// c >= 2, to kEmpty[(c-2) % kStages]: S(c) is issued after PV(c-2) has completed (and every
// MMA before it), so its completion is also the moment chunk c-2's ring stage is free.
// One release barrier per stage keeps every parity wait unambiguous (see the producer).
enum Bar {
  kQFull = 0,
  kFull = 1,                  // [stage]
  kSReady = kFull + 4,        // [buf] (chunks 0 and 1)
  kEmpty = kSReady + 2,       // [stage]: released by S(c + 2), c the chunk it held
  kPReady = kEmpty + 4,       // [buf] (count 4: the softmax warps stored P)
  kPvDone = kPReady + 2,      // [buf]: PV of the chunk that last used the buffer is done
  kOReady = kPvDone + 2,
  kDrain = kOReady + 1,       // MMA thread: every MMA it issued has completed
  kNumBars = kDrain + 1
};

struct FwdParams {
  int Z, Y, X, tiles_z, tiles_y, tiles_x;  // Z: planes of the query (centre) buffer
  int Zg, qz0, kz0;  // global planes; global z of query-buffer plane 0 and of K/V-buffer plane 0
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
  int y_rows;  // y is [B, N, H, D] (token-major) instead of [B, H, N, D]
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

// Online-softmax bookkeeping of one branch for one row, split in two so that the
// scores are dead before the accumulator is touched:
//   begin_max  picks the reference max for this chunk's exponentials.  The running
//              max only moves when it grows by more than 2^8 (or on the first chunk);
//              otherwise the stale max is kept and p <= 2^8.
//   finish_max rescales the TMEM accumulator row and the running sum when the max
//              moved (warp-collective TMEM access, per-row factor) and adds this
//              chunk's sum.
struct MaxUpdate {
  float m_use;   // max the exponentials of this chunk are taken against
  float factor;  // accumulator rescale factor (1 when the max did not move)
  bool rescale;
};

__device__ __forceinline__ MaxUpdate begin_max(float m, float mx, float sc) {
  const float m_new = fmaxf(m, mx);
  MaxUpdate u;
  u.rescale = (m != kNegInf) && (m_new - m) * sc > 8.f;
  u.m_use = (m == kNegInf || u.rescale) ? m_new : m;
  u.factor = u.rescale ? ex2_approx((m - m_new) * sc) : 1.f;
  return u;
}

template <int D>
__device__ __forceinline__ void rescale_rows(float factor, uint32_t t_o) {
  uint32_t o[16];
#pragma unroll
  for (int c = 0; c < D / 16; ++c) {
    tmem_ld16(t_o + 16 * c, o);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
    tmem_st16(t_o + 16 * c, o);
  }
}

// Exponentiate N scores (in registers) against max m, pack to 16-bit pairs and store
// them as P into TMEM columns [t_p, t_p + N/2).  Returns the row sum of p.
template <int N, bool BF16>
__device__ __forceinline__ float exp_store(const float *s, float m, float sc, uint32_t t_p) {
  static_assert(N % 32 == 0, "N must be a multiple of 32");
  const float msc = (m == kNegInf) ? 0.f : m * sc;
  const float2 sc2 = make_float2(sc, sc), nmsc2 = make_float2(-msc, -msc);
  float2 sum[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // independent partial sums
#pragma unroll
  for (int g = 0; g < N / 32; ++g) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      // fmaf(s, sc, -msc) on each lane of the pair
      const float2 x = fma2(make_float2(s[32 * g + 2 * i], s[32 * g + 2 * i + 1]), sc2, nmsc2);
      float p0, p1;
      if ((i & 3) == 3) {  // a quarter of the exponentials on the FMA pipe: the MUFU is the bound
        const float2 e = exp2_poly2(x);
        p0 = e.x;
        p1 = e.y;
      } else {
        p0 = ex2_approx(x.x);
        p1 = ex2_approx(x.y);
      }
      sum[i & 1] = add2(sum[i & 1], make_float2(p0, p1));
      pk[i] = pack2<BF16>(p0, p1);
    }
    tmem_st16(t_p + 16 * g, pk);
  }
  const float2 t = add2(sum[0], sum[1]);
  return t.x + t.y;
}

// Row maximum of N registers as a tree (8 independent chains, then pairwise).
template <int N>
__device__ __forceinline__ float row_max(const float *s) {
  static_assert(N % 16 == 0, "N must be a multiple of 16");
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) m[k] = fmaxf(s[2 * k], s[2 * k + 1]);
#pragma unroll
  for (int i = 16; i < N; i += 16) {
#pragma unroll
    for (int k = 0; k < 8; ++k) m[k] = max3(m[k], s[i + 2 * k], s[i + 2 * k + 1]);
  }
  return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
}

template <int D, bool BF16, int R>
__global__ void __launch_bounds__(kThreads, 2)
    stencil_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkl,
                       const __grid_constant__ CUtensorMap tvl, const __grid_constant__ CUtensorMap tsk,
                       const __grid_constant__ CUtensorMap tsv, const FwdParams p) {
  using G = Geo<R>;
  constexpr int kR = G::kR, kHY = G::kHY, kHX = G::kHX, kWin = G::kWin, kKeys = G::kKeys;
  constexpr int kLocalChunks = G::kLocalChunks, kSumRows = G::kSumRows;
  constexpr uint32_t kSBuf = G::kSBuf, kColO = G::kColO;
  using C = Cfg<D, kKeys>;
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
  const int x0 = tx * kTX, y0 = ty * kTY, z0 = tz * kTZ;
  const int b = bh / p.heads, h = bh % p.heads;
  const int bg = b * p.kv_heads + h / (p.heads / p.kv_heads);
  const int n_chunks = kLocalChunks + p.global_chunks;

  // ---- shared memory carve-up (1024-byte aligned)
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t q_smem = base;
  const uint32_t ring = base + C::kQBytes;
  uint8_t *ol_park = smem_raw + (base - raw) + C::kQBytes + C::kStages * C::kStageBytes;  // [row][D]
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (tid == 0) {
    mbar_init(bar(kQFull), 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar(kFull + s), 1);
      mbar_init(bar(kEmpty + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(kSReady + i), 1);
      mbar_init(bar(kPReady + i), 4);
      mbar_init(bar(kPvDone + i), 1);
    }
    mbar_init(bar(kOReady), 1);
    mbar_init(bar(kDrain), 1);
    fence_mbar_init();
  }
  for (int i = tid; i < D; i += kThreads) {
    s_sl[i] = p.sl[i];
    s_sg[i] = p.sg[i];
  }
  if constexpr (kWin < kKeys) {
    // The TMA boxes of a local chunk fill kWin of the kKeys rows of every 16-channel box; the
    // rest must read as zeros (masked scores, zero V rows) until the global chunks, which
    // fill whole boxes, reuse the stage.  Zero the ring once, then order these generic-proxy
    // stores before the tensor cores' (async-proxy) reads.
    uint4 *ring_v = reinterpret_cast<uint4 *>(smem_raw + (base - raw) + C::kQBytes);
    for (int i = tid; i < C::kStages * C::kStageBytes / 16; i += kThreads) ring_v[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
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
      mbar_expect_tx(bar(kQFull), C::kQBytes);
      for (int c = 0; c < C::kK; ++c)
        tma_load_5d(q_smem + c * C::kBoxQ, &tq, bar(kQFull), 16 * c, x0, y0, z0, bh);
      int issued = 0;
      for (int ch = 0; ch < n_chunks; ++ch) {
        const int s = ch % C::kStages;
        // kEmpty[s] completes once per use of stage s: this is completion ch/kStages - 1.
        // A parity wait only tells it from its neighbours if both are ruled out: the one
        // before was awaited here a ring turn ago (or this is the first), and the one
        // after is S(ch + 2), which needs chunk ch + 2, not loaded yet.
        if (ch >= C::kStages &&
            !mbar_wait(bar(kEmpty + s), (ch / C::kStages - 1) & 1, &g_fwd_errors, kWaitNs, kErrProducer))
          break;
        const uint32_t stage = ring + s * C::kStageBytes;
        const uint32_t full = bar(kFull + s);
        // a local chunk's boxes hold kWin rows each, a global chunk's all kKeys (rows past M
        // are zero-filled and still counted)
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
      // Never leave copies in flight into shared memory this CTA is about to give up: wait
      // (bounded) for the Q tile and the last loads of every stage.  On the normal path
      // these phases completed long ago; after a timed-out wait they may still be landing.
      mbar_wait(bar(kQFull), 0, &g_fwd_errors, kWaitNs, kErrTeardown);
      for (int ch = issued > C::kStages ? issued - C::kStages : 0; ch < issued; ++ch)
        mbar_wait(bar(kFull + ch % C::kStages), (ch / C::kStages) & 1, &g_fwd_errors, kWaitNs, kErrTeardown);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(128, kKeys, BF16, false);
      constexpr uint32_t idesc_pv = idesc_f16(128, D, BF16, true);
      // Commits issued per barrier: teardown waits for the last phase of each, so that no
      // arrive from a commit can land after the CTA has exited.
      uint32_t commits[kNumBars];
      for (int i = 0; i < kNumBars; ++i) commits[i] = 0u;
      auto commit = [&](int b_idx) {
        mma_commit(bar(b_idx));
        ++commits[b_idx];
      };
      // Shared-memory descriptors are built once; an operand's descriptor is its base plus
      // (byte offset >> 4), one add per MMA (addresses stay inside the 14-bit field).
      const uint64_t desc_q = desc_sw32(q_smem, 16, 256);          // the Q tile, K-major
      const uint64_t desc_k = desc_sw32(ring, 16, 256);            // K chunks in the ring, K-major
      const uint64_t desc_v = desc_sw32(ring, C::kBoxK, 256);      // V chunks in the ring, MN-major
      // S(ch) = Q K(ch)^T into S buffer ch%2, then signal the softmax warps.
      auto issue_s = [&](int ch) {
        const uint64_t bk = desc_k + ((uint32_t)((ch % C::kStages) * C::kStageBytes) >> 4);
        const uint32_t t_s = tmem + (ch & 1) * kSBuf;
#pragma unroll
        for (int c = 0; c < C::kK; ++c)
          mma_ss(t_s, desc_q + c * (C::kBoxQ >> 4), bk + c * (C::kBoxK >> 4), idesc_s, c > 0 ? 1u : 0u);
        commit(ch >= 2 ? kEmpty + (ch - 2) % C::kStages : kSReady + ch);
      };
      // O += P(c) V(c) once the softmax warps have written P(c).
      auto issue_pv = [&](int c) -> bool {
        if (!mbar_wait(bar(kPReady + (c & 1)), (c >> 1) & 1, &g_fwd_errors, kWaitNs, kErrMma)) return false;
        tc_fence_after();
        const uint64_t bv = desc_v + ((uint32_t)((c % C::kStages) * C::kStageBytes + C::kKeyBytes) >> 4);
        const uint32_t t_p = tmem + (c & 1) * kSBuf, t_o = tmem + kColO;
        const bool first = (c == 0) || (c == kLocalChunks);  // O restarts for the global branch
#pragma unroll
        for (int j = 0; j < kKeys / 16; ++j)
          mma_ts(t_o, t_p + 8 * j, bv + j * (512 >> 4), idesc_pv, (first && j == 0) ? 0u : 1u);
        commit(kPvDone + (c & 1));
        return true;
      };
      auto wait_full = [&](int ch) -> bool {
        if (!mbar_wait(bar(kFull + ch % C::kStages), (ch / C::kStages) & 1, &g_fwd_errors, kWaitNs, kErrMma))
          return false;
        tc_fence_after();
        return true;
      };
      // S(c+2) writes the TMEM columns that PV(c) reads as its A operand (P(c)).
      // tcgen05.mma ops are only ordered among themselves when they share an accumulator,
      // so PV(c) must have completed before S(c+2) is issued.
      auto wait_pv = [&](int c) -> bool {
        if (!mbar_wait(bar(kPvDone + (c & 1)), (c >> 1) & 1, &g_fwd_errors, kWaitNs, kErrMma)) return false;
        tc_fence_after();
        return true;
      };
      // Prologue: both S buffers.  Steady state per chunk c: PV(c), [PV(c) done] S(c+2).
      bool ok = mbar_wait(bar(kQFull), 0, &g_fwd_errors, kWaitNs, kErrMma);
      for (int ch = 0; ok && ch < 2; ++ch) {
        ok = wait_full(ch);
        if (!ok) break;
        issue_s(ch);
      }
      for (int c = 0; ok && c < n_chunks; ++c) {
        ok = issue_pv(c);
        if (!ok || c + 2 >= n_chunks) continue;
        ok = wait_full(c + 2) && wait_pv(c);
        if (!ok) break;
        issue_s(c + 2);  // its commit also releases chunk c's stage to the producer
      }
      if (ok) commit(kOReady);
      // TMEM is freed after the final __syncthreads: make sure every MMA issued above has
      // completed, and every commit has arrived, first -- on the normal path and after a
      // timed-out wait alike.
      commit(kDrain);
      for (int i = 0; i < kNumBars; ++i)
        if (commits[i]) mbar_wait(bar(i), (commits[i] - 1) & 1, &g_fwd_errors, kWaitNs, kErrTeardown);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int w = warp;
    const uint32_t lanes = (uint32_t)(w * 32) << 16;
    const uint32_t t_tile = tmem + lanes;
    const uint32_t t_o = t_tile + kColO;
    const int row = w * 32 + lane;
    const int qz = w, qy = lane >> 3, qx = lane & 7;
    const int zq = z0 + qz, yq = y0 + qy, xq = x0 + qx;
    const bool row_ok = zq < p.Z && yq < p.Y && xq < p.X;
    uint32_t *park = reinterpret_cast<uint32_t *>(ol_park + (size_t)row * D * 2);
    // keys of the 8x12 halo window inside this query's cube and inside the volume
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
    // Bounded wait with a warp-uniform result: the warp reconverges and leaves together,
    // so the warp-collective TMEM loads and stores that follow run on the whole warp.
    auto wait_warp = [&](uint32_t b_addr, uint32_t parity) -> bool {
      const bool r = mbar_wait(b_addr, parity, &g_fwd_errors, kWaitNs, kErrSoftmax);
      const bool all = __all_sync(0xffffffffu, r);
      if (all) tc_fence_after();
      return all;
    };
    // Completion of PV(c), needed before O is read or rescaled.  Testing the phase only
    // when needed is sound: the next completion of that buffer's barrier is PV(c+2), which
    // needs this warp's P of chunk c+2.
    auto wait_pv_done = [&](int c) -> bool { return wait_warp(bar(kPvDone + (c & 1)), (c >> 1) & 1); };
    for (int ch = 0; ch < n_chunks; ++ch) {
      const int buf = ch & 1;
      const uint32_t t_s = t_tile + buf * kSBuf;
      if (ch == kLocalChunks) {
        // Local branch done: park its normalised output (storage dtype) and free O.
        ok = wait_pv_done(kLocalChunks - 1);
        if (!ok) break;
        const float inv_l = l_l > 0.f ? 1.f / l_l : 0.f;
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t o[16];
          tmem_ld16(t_o + 16 * c, o);
          tmem_wait_ld();
          uint4 v[2];
          uint32_t *pv = reinterpret_cast<uint32_t *>(v);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            pv[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
          reinterpret_cast<uint4 *>(park)[2 * c] = v[0];
          reinterpret_cast<uint4 *>(park)[2 * c + 1] = v[1];
        }
        tc_fence_before();
      }
      // S(ch) complete (the barrier map is described at enum Bar).  Each is completion
      // number k of its barrier with k - 1 awaited by this warp before (or k = 0), and
      // completion k + 1 needs this warp's P of a later chunk.
      if (ch >= 2)
        ok = wait_warp(bar(kEmpty + (ch - 2) % C::kStages), ((ch - 2) / C::kStages) & 1);
      else
        ok = wait_warp(bar(kSReady + ch), 0);
      if (!ok) break;
      const bool local = ch < kLocalChunks;
      const int zp = p.qz0 + z0 - kR + ch;  // global plane of this local chunk
      const bool active = !local || ((unsigned)(ch - qz) <= 2u * kR && zp >= 0 && zp < p.Zg);  // warp-uniform
      if (active) {
        float s[kKeys];
#pragma unroll
        for (int g = 0; g < kKeys / 32; ++g) tmem_ld32(t_s + 32 * g, reinterpret_cast<uint32_t *>(s + 32 * g));
        tmem_wait_ld();
        if (local) {
#pragma unroll
          for (int i = 0; i < kKeys; ++i) s[i] = (mask[i >> 5] >> (i & 31)) & 1u ? s[i] : kNegInf;
        } else {
          const int valid = p.summaries - (ch - kLocalChunks) * kSumRows;
          if (valid < kSumRows) {
#pragma unroll
            for (int i = 0; i < kSumRows; ++i) s[i] = i < valid ? s[i] : kNegInf;
          }
        }
        const MaxUpdate u = begin_max(local ? m_l : m_g, row_max<kKeys>(s), sc);
        const float sum = exp_store<kKeys, BF16>(s, u.m_use, sc, t_s);
        if (__any_sync(0xffffffffu, u.rescale)) {
          ok = wait_pv_done(ch - 1);
          if (!ok) break;
          rescale_rows<D>(u.factor, t_o);
        }
        if (local) {
          l_l = l_l * u.factor + sum;
          m_l = u.m_use;
        } else {
          l_g = l_g * u.factor + sum;
          m_g = u.m_use;
        }
      } else {
        uint32_t zero[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) zero[i] = 0u;
#pragma unroll
        for (int g = 0; g < kKeys / 32; ++g) tmem_st16(t_s + 16 * g, zero);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kPReady + buf));
    }
    // ---- epilogue: normalise the global branch, mix, store through the row map
    if (ok) ok = wait_warp(bar(kOReady), 0);
    if (ok) {
      uint32_t og[D];
#pragma unroll
      for (int c = 0; c < D / 16; ++c) tmem_ld16(t_o + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(og + 16 * c));
      tmem_wait_ld();
      if (row_ok) {
        int64_t rr = ((int64_t)zq * p.Y + yq) * p.X + xq;
        if (p.map) rr = p.map[rr];
        const int64_t grow = (int64_t)bh * p.tokens + rr;
        const float gate = load_any(p.gate, p.gate_dtype, grow);
        const float inv_g = 1.f / l_g;
        uint32_t packed_y[D / 2], packed_g[D / 2];
#pragma unroll
        for (int i = 0; i < D / 2; ++i) {
          const float2 lv = unpack2<BF16>(park[i]);
          const float g0 = __uint_as_float(og[2 * i]) * inv_g, g1 = __uint_as_float(og[2 * i + 1]) * inv_g;
          const float y0v = __fadd_rn(__fmul_rn(s_sl[2 * i], lv.x), __fmul_rn(__fmul_rn(gate, s_sg[2 * i]), g0));
          const float y1v =
              __fadd_rn(__fmul_rn(s_sl[2 * i + 1], lv.y), __fmul_rn(__fmul_rn(gate, s_sg[2 * i + 1]), g1));
          packed_y[i] = pack2<BF16>(y0v, y1v);
          packed_g[i] = pack2<BF16>(g0, g1);
        }
        const int64_t yrow = p.y_rows ? ((int64_t)b * p.tokens + rr) * p.heads + h : grow;
        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.y) + yrow * D);
#pragma unroll
        for (int v = 0; v < D / 8; ++v)
          dst[v] = make_uint4(packed_y[4 * v], packed_y[4 * v + 1], packed_y[4 * v + 2], packed_y[4 * v + 3]);
        if (p.ol) {
          uint4 *dl = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.ol) + grow * D);
          uint4 *dg = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.og) + grow * D);
#pragma unroll
          for (int v = 0; v < D / 8; ++v) {
            dl[v] = reinterpret_cast<const uint4 *>(park)[v];
            dg[v] = make_uint4(packed_g[4 * v], packed_g[4 * v + 1], packed_g[4 * v + 2], packed_g[4 * v + 3]);
          }
          p.lse_l[grow] = m_l * p.inv_sqrt_d + logf(l_l);
          p.lse_g[grow] = m_g * p.inv_sqrt_d + logf(l_g);
        }
      }
    }
    tmem_wait_st();  // a warp that left the chunk loop early may still have TMEM stores in flight
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------- host side

template <int D, bool BF16, int R>
int launch_t(const StencilFwdArgs &a, cudaStream_t stream) {
  using G = Geo<R>;
  constexpr int kHY = G::kHY, kHX = G::kHX, kSumRows = G::kSumRows;
  using C = Cfg<D, G::kKeys>;
  const int Z = a.grid[0], Y = a.grid[1], X = a.grid[2];
  const uint64_t es = 2;
  const uint64_t bh = (uint64_t)a.batch * a.heads, bgs = (uint64_t)a.batch * a.kv_heads;
  CUtensorMap tq, tkl, tvl, tsk, tsv;
  {
    const uint64_t dims[5] = {(uint64_t)D, (uint64_t)X, (uint64_t)Y, (uint64_t)Z, bh};
    const uint64_t strides[4] = {D * es, X * D * es, (uint64_t)Y * X * D * es, (uint64_t)Z * Y * X * D * es};
    const uint32_t box[5] = {16, kTX, kTY, kTZ, 1};
    if (int st = encode_operand(&tq, a.dtype, a.q, 5, dims, strides, box)) return st;
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
  FwdParams p{};
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
  p.y_rows = a.y_rows;
  const int64_t units = (int64_t)bh * p.tiles_z * p.tiles_y * p.tiles_x;
  if (units <= 0) return P3D_OK;
  if (units > 0x7fffffff) return fail(P3D_ERR_UNSUPPORTED, "too many tiles");
  auto kernel = stencil_fwd_kernel<D, BF16, R>;
  static size_t seen[kMaxDevices] = {};
  if (int st = smem_optin(kernel, C::kSmemBytes, seen)) return st;
  kernel<<<(unsigned)units, kThreads, C::kSmemBytes, stream>>>(tq, tkl, tvl, tsk, tsv, p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

}  // namespace

bool stencil_fwd_supported(int dtype, int head_dim, const int radius[3], int summaries) {
  if (dtype != P3D_BF16 && dtype != P3D_F16) return false;
  if (head_dim != 16 && head_dim != 32 && head_dim != 48 && head_dim != 64) return false;
  if (radius[0] != radius[1] || radius[1] != radius[2] || (radius[0] != 1 && radius[0] != 2)) return false;
  if (summaries < 1) return false;
  DeviceInfo info;
  if (device_info(&info) != P3D_OK || info.major != 10) return false;
  return true;
}

template <int R>
int launch_fwd_radius(const StencilFwdArgs &a, cudaStream_t s) {
  const bool bf16 = a.dtype == P3D_BF16;
  switch (a.head_dim) {
    case 16: return bf16 ? launch_t<16, true, R>(a, s) : launch_t<16, false, R>(a, s);
    case 32: return bf16 ? launch_t<32, true, R>(a, s) : launch_t<32, false, R>(a, s);
    case 48: return bf16 ? launch_t<48, true, R>(a, s) : launch_t<48, false, R>(a, s);
    case 64: return bf16 ? launch_t<64, true, R>(a, s) : launch_t<64, false, R>(a, s);
    default: return fail(P3D_ERR_UNSUPPORTED, "stencil forward: head_dim %d", a.head_dim);
  }
}

int launch_stencil_fwd(const StencilFwdArgs &a, cudaStream_t s) {
  switch (a.radius) {
    case 1: return launch_fwd_radius<1>(a, s);
    case 2: return launch_fwd_radius<2>(a, s);
    default: return fail(P3D_ERR_UNSUPPORTED, "stencil forward: radius %d", a.radius);
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
