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
// TMEM (256 columns): one 96-column S buffer, two 48-column P buffers (16-bit pairs; chunk c
// uses buffer c % 2) and the accumulator O.  The softmax warps release S as soon as it is in
// their registers, so the QK^T MMA of chunk c+1 runs while they exponentiate chunk c, and the
// PV MMA of chunk c runs while they work on chunk c+1.  O holds the local accumulator during chunks 0..7;
// when they are done the normalised local output is parked in shared memory, rounded to
// the storage dtype as the reference rounds it before the mix, and O then accumulates the
// global branch.  Two independent online softmaxes: the local one tracks its maximum (in
// registers; O is rescaled only when it grows by > 2^8); the global one takes its
// exponentials against a per-row upper bound of its scores when the summaries' norms give
// one that is tight enough, so it needs no maximum at all.  The epilogue normalises the
// global branch, mixes and writes y (and optionally ol, og, lse_l, lse_g) through the
// raster->packed row map.
//
// Roles: warps 0-3 softmax, warp 4 TMA producer, warp 5 MMA issuer (one thread).
// Operands live in shared memory in the SWIZZLE_32B layout: Q / K are K-major boxes of
// 16 channels, V is the same bytes read MN-major; P is written to its TMEM buffer as
// bf16/f16 pairs and feeds the PV MMA as the TMEM A operand.  Every mbarrier wait is
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
constexpr int kSoftmaxWarps = 4;                    // one per 32-row quarter of the tile
constexpr int kThreads = 32 * (kSoftmaxWarps + 2);
constexpr int kProducerWarp = kSoftmaxWarps, kMmaWarp = kSoftmaxWarps + 1;
constexpr uint32_t kTmemCols = 256;                 // two CTAs per SM
constexpr float kNegInf = -__builtin_huge_valf();
constexpr uint64_t kWaitNs = 2000000000ull;        // every mbarrier wait gives up after 2 s

// Chunk geometry of a radius-R stencil (R = 1 or 2): a local chunk is one halo plane of the
// tile, a kHY x kHX (y, x) window; chunks are kKeys wide (the window rounded up to 32 keys;
// the padding rows of every ring stage are zero and masked) and global chunks take kKeys
// summaries.  TMEM: the S buffer [0, kKeys), P buffers 0 and 1 (16-bit pairs, kKeys / 2
// columns each) [kKeys, 2 kKeys), O [2 kKeys, 2 kKeys + D).
template <int R>
struct Geo {
  static constexpr int kR = R;
  static constexpr int kHY = kTY + 2 * R, kHX = kTX + 2 * R, kHZ = kTZ + 2 * R;
  static constexpr int kWin = kHY * kHX;                // 96 (R = 2), 60 (R = 1)
  static constexpr int kKeys = (kWin + 31) / 32 * 32;   // 96, 64
  static constexpr int kLocalChunks = kHZ;              // 8, 6 halo planes per tile
  static constexpr int kSumRows = kKeys;                // summaries per global chunk
  static constexpr uint32_t kColS = 0, kColP = kKeys, kPStride = kKeys / 2, kColO = 2 * kKeys;
  static_assert(kKeys % 32 == 0 && kKeys <= 96, "chunk size must suit the MMA, TMEM and register budgets");
  static_assert(kPStride % 16 == 0, "P buffers start on 16-column boundaries (tcgen05.st pieces)");
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

// Barrier map (one 128-row tile; the executable model is tests/stencil_protocol.py):
//   S(c) commits to kSFull.  The four softmax warps arrive on kSFree once they have loaded
//   S(c) into registers, and S(c + 1) may then overwrite it -- so the next S is computed
//   while the softmax warps still work on this one.  They arrive on kPFull[c % 2] once P(c)
//   is in P buffer c % 2 (one barrier per buffer: the warps may finish chunk c + 1 before
//   the MMA thread has seen chunk c's arrivals, but not chunk c + 2, whose S is issued only
//   after PV(c)); PV(c) commits to kPFree (O quiet: it may be read or rescaled until
//   PV(c + 1) is issued) and to kEmpty[c % kStages] (both MMAs that read the ring stage of
//   chunk c have completed: the producer may refill it).  P buffer c % 2 needs no wait of its
//   own: PV(c - 2), its last reader, was issued before S(c), and the kSFull commit of S(c),
//   which the warps wait for first, arrives only once every MMA issued before it completed.
//   Every parity wait has the completions before and after the awaited one ruled out.
enum Bar {
  kQFull = 0,
  kFull = 1,                  // [stage]
  kEmpty = kFull + 4,         // [stage]: released by PV(c), c the chunk it held
  kSFull = kEmpty + 4,        // S(c) complete
  kSFree = kSFull + 1,        // count 4: the softmax warps loaded S(c)
  kPFull = kSFree + 1,        // [c % 2], count 4: the softmax warps stored P(c)
  kPFree = kPFull + 2,        // PV(c) complete
  kOReady = kPFree + 1,
  kDrain = kOReady + 1,       // MMA thread: every MMA it issued has completed
  kNumBars = kDrain + 1
};

struct FwdParams {
  int Z, Y, X, tiles_z, tiles_y, tiles_x;  // Z: planes of the query (centre) buffer; tiles_z: of the range run
  int tz0;                                 // first 4-plane query tile of the range
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
  const float *kbound;  // [B*G] max_j |sk_j|, or nullptr: the global branch tracks its maximum
};

// Fixed-reference global softmax (see the softmax warps): used when the largest p of every row
// is at least 2^-fixed_range, so that it is a normal number of the 16-bit type P is stored in
// (bf16 keeps fp32's exponent range; f16's smallest normal is 2^-14, and below 2^-24 a p would
// be stored as zero).  kPolyEighths of every 8 exponential pairs go to the FMA pipe.
template <bool BF16>
__device__ __forceinline__ constexpr float fixed_range() {
  return BF16 ? 64.f : 14.f;
}
constexpr int kPolyEighths = 2;

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

// Exponentiate N scores (in registers) against max m and pack them to 16-bit pairs in
// pk[N/2] (P for the TMEM store).  A quarter of the pairs use the polynomial on the FMA pipe.
// Returns the row sum of p.
template <int N, bool BF16>
__device__ __forceinline__ float exp_pack(const float *s, float m, float sc, uint32_t *pk) {
  static_assert(N % 16 == 0, "N must be a multiple of 16");
  const float msc = (m == kNegInf) ? 0.f : m * sc;
  const float2 sc2 = make_float2(sc, sc), nmsc2 = make_float2(-msc, -msc);
  float2 sum[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // independent partial sums
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    // fmaf(s, sc, -msc) on each lane of the pair
    const float2 x = fma2(make_float2(s[2 * i], s[2 * i + 1]), sc2, nmsc2);
    float2 e;
    if ((i & 3) == 3) {  // a quarter of the exponentials on the FMA pipe: the MUFU is the bound
      e = exp2_poly2(x);
    } else {
      e.x = ex2_approx(x.x);
      e.y = ex2_approx(x.y);
    }
    sum[i & 1] = add2(sum[i & 1], e);
    pk[i] = pack2<BF16>(e.x, e.y);
  }
  const float2 t = add2(sum[0], sum[1]);
  return t.x + t.y;
}

// exp_pack for the fixed-reference global branch: every x = s sc - msc lies in
// [-fixed_range(), 0] (up to rounding), so no maximum, no rescale and no clamp are needed; a
// share kPoly of every 8 pairs is evaluated by the polynomial on the FMA pipe, the rest on
// the MUFU, interleaved.  Returns the row sum of p.
template <int N, bool BF16, int kPoly>
__device__ __forceinline__ float exp_pack_fixed(const float *s, float msc, float sc, uint32_t *pk) {
  static_assert(N % 16 == 0, "N must be a multiple of 16");
  const float2 sc2 = make_float2(sc, sc), nmsc2 = make_float2(-msc, -msc);
  float2 sum[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    const float2 x = fma2(make_float2(s[2 * i], s[2 * i + 1]), sc2, nmsc2);
    float2 e;
    if (((i * kPoly) & 7) < kPoly) {
      e = exp2_poly2_inrange(x);
    } else {
      e.x = ex2_approx(x.x);
      e.y = ex2_approx(x.y);
    }
    sum[i & 1] = add2(sum[i & 1], e);
    pk[i] = pack2<BF16>(e.x, e.y);
  }
  const float2 t = add2(sum[0], sum[1]);
  return t.x + t.y;
}

// TMEM columns [OFF, OFF + W) of this warp's 32 lanes (t: the warp's lane base, column 0 of
// the allocation, which is 32-column aligned), loaded (ld_span, then tmem_wait_ld) or stored
// (st_span, then tmem_wait_st) as .x32 / .x16 / .x8 pieces that each start at a multiple of
// their own width.
template <int OFF, int W>
__device__ __forceinline__ void ld_span(uint32_t t, uint32_t *r) {
  static_assert(OFF % 8 == 0 && W % 8 == 0, "TMEM spans are whole 8-column groups");
  if constexpr (W == 0) {
    return;
  } else if constexpr (OFF % 32 == 0 && W >= 32) {
    tmem_ld32(t + OFF, r);
    ld_span<OFF + 32, W - 32>(t, r + 32);
  } else if constexpr (OFF % 16 == 0 && W >= 16) {
    tmem_ld16(t + OFF, *reinterpret_cast<uint32_t(*)[16]>(r));
    ld_span<OFF + 16, W - 16>(t, r + 16);
  } else {
    tmem_ld8(t + OFF, r);
    ld_span<OFF + 8, W - 8>(t, r + 8);
  }
}
template <int OFF, int W>
__device__ __forceinline__ void st_span(uint32_t t, const uint32_t *r) {
  static_assert(OFF % 8 == 0 && W % 8 == 0, "TMEM spans are whole 8-column groups");
  if constexpr (W == 0) {
    return;
  } else if constexpr (OFF % 16 == 0 && W >= 16) {
    tmem_st16(t + OFF, r);
    st_span<OFF + 16, W - 16>(t, r + 16);
  } else {
    tmem_st8(t + OFF, r);
    st_span<OFF + 8, W - 8>(t, r + 8);
  }
}

// O *= factor on TMEM columns [OFF, OFF + W) (this warp's channels; per-row factor).
template <int OFF, int W>
__device__ __forceinline__ void rescale_span(float factor, uint32_t t) {
  uint32_t o[W];
  ld_span<OFF, W>(t, o);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < W; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
  st_span<OFF, W>(t, o);
}

// Squared Euclidean norm of query row `row` of the Q tile in shared memory: D/16 boxes of
// 128 rows x 32 bytes (16 channels).  The 32-byte swizzle only permutes the two 16-byte halves
// of a row, which the sum does not see.
template <int D, bool BF16>
__device__ __forceinline__ float q_row_sq(const uint8_t *q_tile, int row) {
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < D / 16; ++c) {
    const uint4 *src = reinterpret_cast<const uint4 *>(q_tile + c * kRows * 32 + row * 32);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 v = src[h];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack2<BF16>(w[k]);
        acc = fmaf(f.x, f.x, acc);
        acc = fmaf(f.y, f.y, acc);
      }
    }
  }
  return acc;
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
  constexpr uint32_t kColO = G::kColO;
  using C = Cfg<D, kKeys>;
  static_assert(kColO + D <= kTmemCols, "S, both P buffers and O must fit the CTA's TMEM columns");
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
  const int tz = p.tz0 + unit % p.tiles_z;
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
  const uint8_t *q_tile = smem_raw + (base - raw);                                       // generic view of Q
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (tid == 0) {
    mbar_init(bar(kQFull), 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar(kFull + s), 1);
      mbar_init(bar(kEmpty + s), 1);
    }
    mbar_init(bar(kSFull), 1);
    mbar_init(bar(kSFree), kSoftmaxWarps);
    mbar_init(bar(kPFull), kSoftmaxWarps);
    mbar_init(bar(kPFull + 1), kSoftmaxWarps);
    mbar_init(bar(kPFree), 1);
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
      // Operations issued, for the teardown: it waits for the last phase of every barrier
      // committed to, so that no arrive from a commit can land after the CTA has exited.
      int n_s = 0, n_pv = 0;
      bool o_ready = false;
      // Shared-memory descriptors are built once; an operand's descriptor is its base plus
      // (byte offset >> 4), one add per MMA (addresses stay inside the 14-bit field).
      const uint64_t desc_q = desc_sw32(q_smem, 16, 256);          // the Q tile, K-major
      const uint64_t desc_k = desc_sw32(ring, 16, 256);            // K chunks in the ring, K-major
      const uint64_t desc_v = desc_sw32(ring, C::kBoxK, 256);      // V chunks in the ring, MN-major
      // S(ch) = Q K(ch)^T into the S buffer, then signal the softmax warps.
      auto issue_s = [&](int ch) {
        const uint64_t bk = desc_k + ((uint32_t)((ch % C::kStages) * C::kStageBytes) >> 4);
        const uint32_t t_s = tmem + G::kColS;
#pragma unroll
        for (int c = 0; c < C::kK; ++c)
          mma_ss(t_s, desc_q + c * (C::kBoxQ >> 4), bk + c * (C::kBoxK >> 4), idesc_s, c > 0 ? 1u : 0u);
        mma_commit(bar(kSFull));
        ++n_s;
      };
      // O += P(c) V(c); its completion frees the P buffer and O, and releases the ring stage.
      auto issue_pv = [&](int c) {
        const uint64_t bv = desc_v + ((uint32_t)((c % C::kStages) * C::kStageBytes + C::kKeyBytes) >> 4);
        const uint32_t t_p = tmem + G::kColP + (uint32_t)(c & 1) * G::kPStride, t_o = tmem + kColO;
        const bool first = (c == 0) || (c == kLocalChunks);  // O restarts for the global branch
#pragma unroll
        for (int j = 0; j < kKeys / 16; ++j)
          mma_ts(t_o, t_p + 8 * j, bv + j * (512 >> 4), idesc_pv, (first && j == 0) ? 0u : 1u);
        mma_commit(bar(kPFree));
        mma_commit(bar(kEmpty + c % C::kStages));
        ++n_pv;
      };
      auto wait_bar = [&](int b_idx, uint32_t parity) -> bool {
        if (!mbar_wait(bar(b_idx), parity, &g_fwd_errors, kWaitNs, kErrMma)) return false;
        tc_fence_after();
        return true;
      };
      auto wait_full = [&](int ch) -> bool { return wait_bar(kFull + ch % C::kStages, (ch / C::kStages) & 1); };
      // Per chunk c: S(c + 1) as soon as the softmax warps have loaded S(c) (and chunk c + 1
      // has landed), then PV(c) once they have stored P(c).
      bool ok = wait_bar(kQFull, 0) && n_chunks > 0 && wait_full(0);
      if (ok) issue_s(0);
      for (int c = 0; ok && c < n_chunks; ++c) {
        if (c + 1 < n_chunks) {
          ok = wait_full(c + 1) && wait_bar(kSFree, c & 1);
          if (!ok) break;
          issue_s(c + 1);
        }
        ok = wait_bar(kPFull + (c & 1), (c >> 1) & 1);
        if (!ok) break;
        issue_pv(c);
      }
      if (ok) {
        mma_commit(bar(kOReady));
        o_ready = true;
      }
      // TMEM is freed after the final __syncthreads: make sure every MMA issued above has
      // completed, and every commit has arrived, first -- on the normal path and after a
      // timed-out wait alike.  The drain commit's arrival means every operation completed;
      // then each barrier's last commit has arrived or is about to.
      mma_commit(bar(kDrain));
      mbar_wait(bar(kDrain), 0, &g_fwd_errors, kWaitNs, kErrTeardown);
      if (n_s) mbar_wait(bar(kSFull), (n_s - 1) & 1, &g_fwd_errors, kWaitNs, kErrTeardown);
      if (n_pv) mbar_wait(bar(kPFree), (n_pv - 1) & 1, &g_fwd_errors, kWaitNs, kErrTeardown);
      if (o_ready) mbar_wait(bar(kOReady), 0, &g_fwd_errors, kWaitNs, kErrTeardown);
      for (int st = 0; st < C::kStages; ++st) {  // kEmpty[st]: once per PV of a chunk c with c % kStages == st
        const int times = n_pv / C::kStages + (st < n_pv % C::kStages ? 1 : 0);
        if (times) mbar_wait(bar(kEmpty + st), (times - 1) & 1, &g_fwd_errors, kWaitNs, kErrTeardown);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    // Warp w owns TMEM lanes 32w .. 32w + 31: the 32 queries of plane z = w.
    const int w = warp;
    const uint32_t t_tile = tmem + ((uint32_t)(w * 32) << 16);
    const int row = w * 32 + lane;
    const int qz = w, qy = lane >> 3, qx = lane & 7;
    const int zq = z0 + qz, yq = y0 + qy, xq = x0 + qx;
    const bool row_ok = zq < p.Z && yq < p.Y && xq < p.X;
    // The row's storage index and gate, loaded now so that the epilogue does not wait on them.
    int64_t rr = 0, grow = 0;
    float gate = 0.f;
    if (row_ok) {
      rr = ((int64_t)zq * p.Y + yq) * p.X + xq;
      if (p.map) rr = p.map[rr];
      grow = (int64_t)bh * p.tokens + rr;
      gate = load_any(p.gate, p.gate_dtype, grow);
    }
    uint32_t *park = reinterpret_cast<uint32_t *>(ol_park + (size_t)row * D * 2);
    // keys of the halo window inside this query's cube and inside the volume
    uint32_t mask[kKeys / 32] = {};
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
    // Completion c of kPFree: PV(c) has completed, so O may be read or rescaled (until this
    // warp's next kPFull arrival lets PV(c + 1) be issued).  A warp that waits for it has
    // waited for completion c - 1 at its previous chunk (it skips these waits only from its
    // first fixed-reference global chunk on), and completion c + 1 needs this warp's P of
    // chunk c + 1, so the parity wait is exact.
    auto wait_pfree = [&](int c) -> bool { return wait_warp(bar(kPFree), c & 1); };
    // This warp's rows of S are in registers: S(c + 1) may overwrite the S buffer.
    auto release_s = [&]() {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kSFree));
    };
    // Global-branch reference value.  By Cauchy-Schwarz every global score of this row (raw
    // q.sk) is at most u = |q| max_j |sk_j|.  Taking the exponentials against u itself puts
    // every p = 2^((s - u) sc) in [2^(-2 u sc), 1]: with 2 u sc <= fixed_range() for every row
    // of the warp there is no running maximum to track, no rescale of O and no clamp in the
    // polynomial exp2, and the row's largest p is a normal number of P's storage type.  The
    // softmax is the same function of the scores (only its reference point moves); otherwise,
    // or without a bound, the warp tracks the maximum.
    bool fixed_g = false;
    if (p.kbound != nullptr) {
      ok = wait_warp(bar(kQFull), 0);
      if (ok) {
        const float u = sqrtf(q_row_sq<D, BF16>(q_tile, row)) * __ldg(p.kbound + bg);
        fixed_g = __all_sync(0xffffffffu, 2.f * u * sc <= fixed_range<BF16>());
        if (fixed_g) m_g = u;
      }
    }
    for (int ch = 0; ok && ch < n_chunks; ++ch) {
      if (ch == kLocalChunks) {
        // Local branch done: park its normalised output (storage dtype) and free O.
        ok = wait_pfree(kLocalChunks - 1);
        if (!ok) break;
        const float inv_l = l_l > 0.f ? 1.f / l_l : 0.f;
        uint32_t o[D];
        ld_span<kColO, D>(t_tile, o);
        tmem_wait_ld();
#pragma unroll
        for (int v = 0; v < D / 8; ++v) {
          uint4 pw;
          uint32_t *pv = reinterpret_cast<uint32_t *>(&pw);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            pv[i] = pack2<BF16>(__uint_as_float(o[8 * v + 2 * i]) * inv_l, __uint_as_float(o[8 * v + 2 * i + 1]) * inv_l);
          reinterpret_cast<uint4 *>(park)[v] = pw;
        }
        tc_fence_before();
      }
      // S(ch) complete: completion ch of kSFull (completion ch + 1 needs this warp's kSFree
      // arrival for chunk ch).
      ok = wait_warp(bar(kSFull), ch & 1);
      if (!ok) break;
      const bool local = ch < kLocalChunks;
      const int zp = p.qz0 + z0 - kR + ch;  // global plane of this local chunk
      const bool active = !local || ((unsigned)(ch - qz) <= 2u * kR && zp >= 0 && zp < p.Zg);  // warp-uniform
      uint32_t pk[kKeys / 2];
      bool rescale = false;
      float factor = 1.f;
      if (active) {
        float s[kKeys];
        ld_span<G::kColS, kKeys>(t_tile, reinterpret_cast<uint32_t *>(s));
        tmem_wait_ld();
        release_s();
        const int valid = local ? kKeys : p.summaries - (ch - kLocalChunks) * kSumRows;
        if (local) {
#pragma unroll
          for (int i = 0; i < kKeys; ++i) s[i] = (mask[i >> 5] >> (i & 31)) & 1u ? s[i] : kNegInf;
        } else if (valid < kSumRows) {
#pragma unroll
          for (int i = 0; i < kSumRows; ++i) s[i] = i < valid ? s[i] : kNegInf;
        }
        if (!local && fixed_g) {
          // the last, partial chunk has masked (-inf) scores: the clamped form maps them to 0
          l_g += valid < kSumRows ? exp_pack<kKeys, BF16>(s, m_g, sc, pk)
                                  : exp_pack_fixed<kKeys, BF16, kPolyEighths>(s, m_g * sc, sc, pk);
        } else {
          const MaxUpdate u = begin_max(local ? m_l : m_g, row_max<kKeys>(s), sc);
          const float sum = exp_pack<kKeys, BF16>(s, u.m_use, sc, pk);
          rescale = __any_sync(0xffffffffu, u.rescale);
          factor = u.factor;
          if (local) {
            l_l = l_l * u.factor + sum;
            m_l = u.m_use;
          } else {
            l_g = l_g * u.factor + sum;
            m_g = u.m_use;
          }
        }
      } else {
        release_s();
#pragma unroll
        for (int i = 0; i < kKeys / 2; ++i) pk[i] = 0u;   // a zero P block: no key of this plane is in range
      }
      // P buffer ch % 2 is free: its last reader PV(ch - 2) completed before S(ch) did (see
      // the barrier map).  O may be rescaled only once PV(ch - 1) has completed: the warp
      // waits for that on every chunk except the global chunks of the fixed-reference path,
      // which never rescale (and, so that every kPFree parity wait stays exact, never wait).
      if (ch >= 1 && !(fixed_g && !local)) {
        ok = wait_pfree(ch - 1);
        if (!ok) break;
      }
      if (rescale) rescale_span<kColO, D>(factor, t_tile);
      st_span<G::kColP, kKeys / 2>(t_tile + (uint32_t)(ch & 1) * G::kPStride, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kPFull + (ch & 1)));
    }
    // ---- epilogue: normalise the global branch, mix, store through the row map
    if (ok) ok = wait_warp(bar(kOReady), 0);
    if (ok) {
      uint32_t og[D];
      ld_span<kColO, D>(t_tile, og);
      tmem_wait_ld();
      if (row_ok) {
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
  const int all_z = (Z + kTZ - 1) / kTZ;
  const int tz_end = a.tile_z_end > 0 ? std::min(a.tile_z_end, all_z) : all_z;
  p.tz0 = std::max(0, a.tile_z_begin);
  p.tiles_z = tz_end - p.tz0;
  if (p.tiles_z <= 0) return P3D_OK;  // an empty tile range
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
  p.kbound = a.summary_bound;
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

// bound[bg] = max_j |sk[bg, j, :]| for the fixed-reference global softmax: blockIdx.y is the
// (batch, kv-head), blockIdx.x a slice of its summary rows, a thread per row; squared norms in
// fp32, a block maximum, then an atomic maximum on the float's bits (non-negative floats order
// as unsigned integers; bound[] starts at zero).  The norm is rounded up by 2^-10 so that
// rounding in the norm cannot put it below a score.
template <bool BF16>
__global__ void __launch_bounds__(128) summary_bound_kernel(const uint32_t *sk, int M, int D, float *bound) {
  __shared__ float part[4];
  const uint32_t *base = sk + (int64_t)blockIdx.y * M * (D / 2);
  float best = 0.f;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < M; j += gridDim.x * blockDim.x) {
    const uint32_t *row = base + (int64_t)j * (D / 2);
    float acc = 0.f;
    for (int d = 0; d < D / 2; ++d) {
      const float2 f = unpack2<BF16>(__ldg(row + d));
      acc = fmaf(f.x, f.x, acc);
      acc = fmaf(f.y, f.y, acc);
    }
    best = fmaxf(best, acc);
  }
  for (int o = 16; o; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = fmaxf(best, part[w]);
    const float b = sqrtf(best) * (1.f + 1.f / 1024.f);
    atomicMax(reinterpret_cast<unsigned *>(bound) + blockIdx.y, __float_as_uint(b));
  }
}

}  // namespace

int launch_summary_bound(const void *sk, int dtype, int bg, int summaries, int head_dim, float *bound,
                         cudaStream_t stream) {
  if (dtype != P3D_BF16 && dtype != P3D_F16) return fail(P3D_ERR_UNSUPPORTED, "summary bound: 16-bit summaries only");
  if (head_dim < 2 || head_dim % 2 || summaries < 1 || bg < 1)
    return fail(P3D_ERR_INVALID_ARGUMENT, "summary bound: bad shape");
  if (((uintptr_t)sk & 3) != 0) return fail(P3D_ERR_INVALID_ARGUMENT, "summary bound: misaligned summaries");
  if (bg > 65535) return fail(P3D_ERR_UNSUPPORTED, "summary bound: too many (batch, kv-head) pairs");
  P3D_CUDA_TRY(cudaMemsetAsync(bound, 0, sizeof(float) * (size_t)bg, stream));
  const dim3 grid((unsigned)std::min((summaries + 127) / 128, 64), (unsigned)bg);
  const uint32_t *src = static_cast<const uint32_t *>(sk);
  if (dtype == P3D_BF16)
    summary_bound_kernel<true><<<grid, 128, 0, stream>>>(src, summaries, head_dim, bound);
  else
    summary_bound_kernel<false><<<grid, 128, 0, stream>>>(src, summaries, head_dim, bound);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

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
