// Fused projection + split + axial RoPE (inference and training forward of the layer glue).
//
// The layer computes qp = LN(x) Wq^T and kvp = LN(x) Wkv^T (attention.py:53-89; the reference
// runs them as two nn.Linear calls) and then splits them head-major, rotating q, kl and kg
// (rotary.py).  p3d_qkv_split does the split from the bf16 projections in HBM; this kernel
// removes the projections' round trip through HBM: for a 128-token tile it multiplies on the
// tensor cores (tcgen05, fp32 accumulators in TMEM) and its epilogue rounds each projection
// to the storage type -- as the GEMM's output would be -- then rotates and stores head-major
// exactly as p3d_qkv_split does from that rounded value.
//
// Columns of Z = [q | kl | vl | kg | vg] are split into groups of G_h head rows (q groups,
// then kv groups; a group never straddles q and kv).  A CTA owns one group: its slice of W
// (G_h D rows x dim) stays in shared memory while it walks token tiles t = c, c + n, ... .
// The CTAs of the different groups walk the same tiles at about the same time, so each X
// tile comes from HBM once and from L2 for the other groups.
//
// Roles (576 threads): warp 0 TMA producer (W slice once, X tiles through a 2-stage ring),
// warp 1 MMA issuer (Z tile into one of two TMEM accumulators), warps 2-17 epilogue: a token
// row (TMEM lane) per thread, four warps per lane quarter splitting the group's heads.  The
// RoPE phase table is staged in shared memory once per CTA (rows at an odd pitch, so that a
// warp's tokens read it without bank conflicts); a token's coordinates are fetched
// a tile ahead, so the epilogue does not wait on global loads.  Every wait is bounded (2 s): on a timeout the kernel records an
// error bit (p3d_device_errors), drains its copies and MMAs and frees TMEM.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace p3d {
namespace {

using namespace sm100;

__device__ unsigned g_proj_errors = 0;

constexpr int kSplit = 4;                        // epilogue warps per TMEM lane quarter
constexpr int kEpilogueThreads = 128 * kSplit;
constexpr int kThreads = 64 + kEpilogueThreads;
constexpr int kProducerWarp = 0, kMmaWarp = 1;  // warps 2..: epilogue
constexpr int kMaxTableFloats = 8192;           // phase tables up to 32 KB live in shared memory
constexpr int kEpilogueWarps = kEpilogueThreads / 32;
constexpr int kStageRows = 16;                  // rows of a warp's head staged per pass (half its 32)
constexpr int kGateRows = 16;                   // gate logit rows (2 H <= 16, zero-padded) beside the last group's W
constexpr int kTile = 128;                      // tokens per tile (MMA M)
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int kTmemCols = 512;

enum : int {
  kWFull = 0,
  kXFull = 1,       // [2]
  kXEmpty = 3,      // [2]
  kAccFull = 5,     // [2]
  kAccEmpty = 7,    // [2], one arrival per epilogue warp
  kDrain = 9,
  kNumBars = 10
};

struct ProjParams {
  int rows;            // B * N token rows of X
  int tokens;          // N
  int kc;              // dim / 64: 64-channel (128-byte, SWIZZLE_128B) boxes along K
  int heads, kv_heads;
  int group_heads;     // head rows per group (G_h)
  int groups_q;        // groups over the q head rows; the rest cover the 4 kv_heads kv head rows
  int groups;
  int ctas_per_group;
  void *out[5];        // q [B,H,N,D], kl, vl, kg, vg [B,G,N,D]
  const int64_t *coords;
  int pairs[3], start[3];
  const float *phases;
  int table_floats;    // 2 * (ez pz + ey py + ex px)
  // The shared-memory copy of the table: the rows of axis a start at entry tstart[a] and are
  // tpitch[a] = pairs[a] | 1 entries apart (an odd pitch: the 32 tokens of a warp, consecutive
  // along x, then read their (cos, sin) from distinct banks instead of 16 lanes per bank);
  // staged when its smem_floats <= kMaxTableFloats.
  int tstart[3], tpitch[3], smem_floats;
  int table_in_smem;   // the table is staged (it fits beside the W slice and X ring)
  int stage_out;       // per-warp output staging in shared memory (kStageRows rows of D values)
  int raster_qkv, ey, ex;  // q, kl, vl rows at each token's raster index (c0 ey + c1) ex + c2
  int64_t kv_rows, kv_row0;  // kl, vl: [B, G, kv_rows, D], token row n at kv_row0 + n
  // The gate (attention.py:84-86) in the CTAs of the last group (vg head rows: no rotation, the
  // lightest epilogue): gate_cols = 2 H logit rows of wg
  // [2H, dim] (nn.Linear weight, bias bg [2H]) beside the group's W slice, zero-padded to
  // kGateRows; gate [B, H, N] = softmax(logit pair of head h)[1].  0: no gate.
  int gate_cols;
  const void *wg, *bg;
  void *gate;
};

// (cos, sin) of rotation pair `pair` of a token at coordinates c, from the table `tab` whose
// axis-a rows start at entry st[a] and are pitch[a] entries apart.
__device__ __forceinline__ float2 pair_cs(const ProjParams &p, const float *tab, const int *st, const int *pitch,
                                          const int (&c)[3], int pair) {
  int entry;
  if (pair < p.pairs[0]) {
    entry = st[0] + c[0] * pitch[0] + pair;
  } else if (pair < p.pairs[0] + p.pairs[1]) {
    entry = st[1] + c[1] * pitch[1] + (pair - p.pairs[0]);
  } else {
    entry = st[2] + c[2] * pitch[2] + (pair - p.pairs[0] - p.pairs[1]);
  }
  return *reinterpret_cast<const float2 *>(tab + 2 * entry);
}

template <bool BF16>
__device__ __forceinline__ float2 unpack_pair(uint32_t v) {  // exact
  if constexpr (BF16) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  } else {
    return __half22float2(*reinterpret_cast<const __half2 *>(&v));
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  return BF16 ? pack_bf16(lo, hi) : pack_f16(lo, hi);
}

// Pairs per axis of balanced_pairs(D) (rope.py: D / 2 pairs dealt evenly over z, y, x, the
// remainder first): when the call uses them, the epilogue knows every pair's axis at compile
// time and reads its (cos, sin) at a constant offset from the token's per-axis table row.
template <int D>
struct Balanced {
  static constexpr int kShare = D / 2 / 3, kExtra = D / 2 % 3;
  static constexpr int count(int axis) { return kShare + (axis < kExtra ? 1 : 0); }
  static constexpr int axis_of(int pair) { return pair < count(0) ? 0 : pair < count(0) + count(1) ? 1 : 2; }
  static constexpr int first(int axis) { return axis == 0 ? 0 : axis == 1 ? count(0) : count(0) + count(1); }
};

template <bool BF16, int D, bool kBalanced>
__global__ void __launch_bounds__(kThreads, 1)
    proj_split_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap twq,
                      const __grid_constant__ CUtensorMap twkv, const ProjParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.group_heads * D;                 // projection columns of the group
  const int group0 = blockIdx.x % p.groups;
  const bool has_gate = p.gate_cols > 0 && group0 == p.groups - 1;
  const int Gp = G + (has_gate ? kGateRows : 0);   // accumulator columns (MMA N): + the gate logits
  const uint32_t x_atom = kTile * 128;             // bytes of one 64-channel box of an X tile
  const uint32_t w_atom = (uint32_t)Gp * 128;      // of the W slice (Gp multiple of 16: 1024-aligned)
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t w_smem = base;
  const uint32_t x_smem = w_smem + p.kc * w_atom;  // 2 stages of kc * x_atom
  const uint32_t x_stage = p.kc * x_atom;
  const uint32_t bars = x_smem + 2 * x_stage;
  // after the barriers: the epilogue warps' output staging (if any), then the phase table
  const uint32_t stage_off = (bars + 8u * kNumBars + 15u - raw) / 16u * 16u;
  const uint32_t stage_bytes = p.stage_out ? (uint32_t)kEpilogueWarps * kStageRows * D * 2u : 0u;
  float *table = reinterpret_cast<float *>(smem_raw + stage_off + stage_bytes);
  __shared__ uint32_t tmem_holder;
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };

  const int group = group0, slot = blockIdx.x / p.groups;
  const bool is_q = group < p.groups_q;
  const int head0 = (is_q ? group : group - p.groups_q) * p.group_heads;  // first head row of the group
  const int n_tiles = (p.rows + kTile - 1) / kTile;
  const int my_tiles = slot < n_tiles ? (n_tiles - 1 - slot) / p.ctas_per_group + 1 : 0;

  if (threadIdx.x == 0) {
    mbar_init(bar(kWFull), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(kXFull + s), 1);
      mbar_init(bar(kXEmpty + s), 1);
      mbar_init(bar(kAccFull + s), 1);
      mbar_init(bar(kAccEmpty + s), kEpilogueThreads / 32);
    }
    mbar_init(bar(kDrain), 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tx);
    prefetch_tmap(is_q ? &twq : &twkv);
  }
  const bool table_in_smem = p.table_in_smem != 0;
  if (table_in_smem) {
    // entry e of the table (axis a, coordinate c, pair k: e = start[a] + c pairs[a] + k) goes
    // to tstart[a] + c tpitch[a] + k
    for (int e = threadIdx.x; 2 * e < p.table_floats; e += kThreads) {
      const int a = e < p.start[1] ? 0 : e < p.start[2] ? 1 : 2;
      const int local = e - p.start[a], c = local / p.pairs[a], k = local - c * p.pairs[a];
      reinterpret_cast<float2 *>(table)[p.tstart[a] + c * p.tpitch[a] + k] =
          reinterpret_cast<const float2 *>(p.phases)[e];
    }
  }
  if (has_gate) {
    // the gate's logit rows after the group's G rows of every 64-channel box, in the layout
    // the TMA writes there (128-byte rows, 16-byte chunk j of row r at j ^ (r mod 8); G is a
    // multiple of 8), rows past 2 H zero
    const uint16_t *wg = static_cast<const uint16_t *>(p.wg);
    for (int e = threadIdx.x; e < p.kc * kGateRows * 8; e += kThreads) {
      const int c = e / (kGateRows * 8), r = (e / 8) % kGateRows, j = e % 8;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < p.gate_cols) v = *reinterpret_cast<const uint4 *>(wg + (int64_t)r * (p.kc * 64) + 64 * c + 8 * j);
      const uint32_t at = w_smem + c * w_atom + (uint32_t)(G + r) * 128u + (uint32_t)((j ^ (r & 7)) * 16);
      *reinterpret_cast<uint4 *>(smem_raw + (at - raw)) = v;
    }
    fence_proxy_async_smem();  // generic-proxy writes, read by the tensor core (async proxy)
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const CUtensorMap *tw = is_q ? &twq : &twkv;
      mbar_expect_tx(bar(kWFull), p.kc * (uint32_t)G * 128u);  // the TMA copies G rows per box
      for (int c = 0; c < p.kc; ++c) tma_load_3d(w_smem + c * w_atom, tw, bar(kWFull), 64 * c, head0 * D, 0);
      int issued = 0;
      for (int i = 0; i < my_tiles; ++i) {
        const int s = i & 1, t = slot + i * p.ctas_per_group;
        // XEmpty[s] completes once per use of stage s; completion i/2 - 1 frees it for tile i.
        // Its neighbours are ruled out: the one before was awaited a ring turn ago, the one
        // after needs tile i, not loaded yet.
        if (i >= 2 && !mbar_wait(bar(kXEmpty + s), ((i >> 1) - 1) & 1, &g_proj_errors, kWaitNs, kErrProducer)) break;
        const uint32_t st = x_smem + s * x_stage;
        mbar_expect_tx(bar(kXFull + s), p.kc * x_atom);
        for (int c = 0; c < p.kc; ++c) tma_load_3d(st + c * x_atom, &tx, bar(kXFull + s), 64 * c, t * kTile, 0);
        issued = i + 1;
      }
      // no copies in flight into shared memory this CTA gives up
      mbar_wait(bar(kWFull), 0, &g_proj_errors, kWaitNs, kErrTeardown);
      for (int i = issued > 2 ? issued - 2 : 0; i < issued; ++i)
        mbar_wait(bar(kXFull + (i & 1)), (i >> 1) & 1, &g_proj_errors, kWaitNs, kErrTeardown);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kTile, Gp, BF16, false);
      int n_mma = 0;  // tiles whose MMAs were issued (each commits kXEmpty and kAccFull of its stage)
      const uint64_t desc_w = desc_sw128(w_smem, 1024);  // K-major, 8-row groups of 128-byte rows
      const uint64_t desc_x = desc_sw128(x_smem, 1024);
      bool ok = mbar_wait(bar(kWFull), 0, &g_proj_errors, kWaitNs, kErrMma);
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int s = i & 1, a = i & 1;
        ok = mbar_wait(bar(kXFull + s), (i >> 1) & 1, &g_proj_errors, kWaitNs, kErrMma);
        // accumulator a was last used by tile i - 2: the epilogue must have read it out
        if (ok && i >= 2) ok = mbar_wait(bar(kAccEmpty + a), ((i >> 1) - 1) & 1, &g_proj_errors, kWaitNs, kErrMma);
        if (!ok) break;
        tc_fence_after();
        const uint64_t dx = desc_x + ((uint32_t)(s * x_stage) >> 4);
        for (int c = 0; c < p.kc; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)  // K = 16 slices: 32 bytes along the 128-byte rows
            mma_ss(tmem + a * Gp, dx + ((c * x_atom + 32 * k) >> 4), desc_w + ((c * w_atom + 32 * k) >> 4), idesc,
                   (c | k) ? 1u : 0u);
        mma_commit(bar(kXEmpty + s));
        mma_commit(bar(kAccFull + a));
        n_mma = i + 1;
      }
      // drain: the last commit first, then each barrier's last phase (stage / accumulator s was
      // committed once per tile i < n_mma with i % 2 == s)
      mma_commit(bar(kDrain));
      mbar_wait(bar(kDrain), 0, &g_proj_errors, kWaitNs, kErrTeardown);
      for (int st = 0; st < 2; ++st) {
        const int times = n_mma / 2 + (st < n_mma % 2 ? 1 : 0);
        if (times) {
          mbar_wait(bar(kXEmpty + st), (times - 1) & 1, &g_proj_errors, kWaitNs, kErrTeardown);
          mbar_wait(bar(kAccFull + st), (times - 1) & 1, &g_proj_errors, kWaitNs, kErrTeardown);
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp & 3;                   // TMEM lanes this warp may access
    const int split = (warp - 2) >> 2;              // heads j = split, split + kSplit, ...
    const int r = quarter * 32 + lane;              // token row within the tile = TMEM lane
    const uint32_t t_lanes = tmem + ((uint32_t)(quarter * 32) << 16);
    const float *tab = table_in_smem ? table : p.phases;
    int tst[3], tpitch[3];  // row start and pitch (entries) of each axis in `tab`
#pragma unroll
    for (int ax = 0; ax < 3; ++ax) {
      tst[ax] = table_in_smem ? p.tstart[ax] : p.start[ax];
      tpitch[ax] = table_in_smem ? p.tpitch[ax] : p.pairs[ax];
    }
    const int head_rows = is_q ? p.heads : 4 * p.kv_heads;
    // coordinates of this thread's token in tile i (fetched one tile ahead)
    auto fetch = [&](int i, int (&c)[3]) {
      const int row = (slot + i * p.ctas_per_group) * kTile + r;
      c[0] = c[1] = c[2] = 0;
      if (i < my_tiles && row < p.rows) {
        const int n = row % p.tokens;
        c[0] = (int)p.coords[3 * (int64_t)n];
        c[1] = (int)p.coords[3 * (int64_t)n + 1];
        c[2] = (int)p.coords[3 * (int64_t)n + 2];
      }
    };
    int cnext[3];
    fetch(0, cnext);
    for (int i = 0; i < my_tiles; ++i) {
      const int a = i & 1, t = slot + i * p.ctas_per_group;
      const int c3[3] = {cnext[0], cnext[1], cnext[2]};
      fetch(i + 1, cnext);
      const bool ready = mbar_wait(bar(kAccFull + a), (i >> 1) & 1, &g_proj_errors, kWaitNs, kErrSoftmax);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int row = t * kTile + r;
      const bool valid = row < p.rows;
      const int b = valid ? row / p.tokens : 0, n = valid ? row - b * p.tokens : 0;
      for (int j = split; j < p.group_heads; j += kSplit) {
        const int hr = head0 + j;  // head row within q, or within the 4 kv parts
        if (hr >= head_rows) break;  // a short last group (warp-uniform)
        uint32_t acc[D];
#pragma unroll
        for (int q16 = 0; q16 < D / 16; ++q16)
          tmem_ld16(t_lanes + a * Gp + j * D + 16 * q16, *reinterpret_cast<uint32_t(*)[16]>(acc + 16 * q16));
        tmem_wait_ld();
        int part = 0, hh = hr;
        if (!is_q) {
          part = hr / p.kv_heads;
          hh = hr - part * p.kv_heads;
        }
        const bool rot = is_q || (part & 1) == 0;  // q, kl, kg
        const int ht = is_q ? p.heads : p.kv_heads;
        uint32_t packed[D / 2];
#pragma unroll
        for (int q2 = 0; q2 < D / 2; ++q2) {
          // the projection pair rounded to the storage type (as the GEMM output would be)
          packed[q2] = pack_pair<BF16>(__uint_as_float(acc[2 * q2]), __uint_as_float(acc[2 * q2 + 1]));
        }
        if (rot && valid) {
          // the token's table row of each axis (balanced pairs: pair q2 sits at a constant
          // offset from the row of its axis)
          const float *row_axis[3];
#pragma unroll
          for (int ax = 0; ax < 3; ++ax) row_axis[ax] = tab + 2 * (tst[ax] + c3[ax] * tpitch[ax]);
#pragma unroll
          for (int q2 = 0; q2 < D / 2; ++q2) {
            const float2 e_o = unpack_pair<BF16>(packed[q2]);
            float2 c;
            if constexpr (kBalanced) {  // q2 is a constant in each unrolled step: the axis folds
              const int ax = Balanced<D>::axis_of(q2);
              c = *reinterpret_cast<const float2 *>(row_axis[ax] + 2 * (q2 - Balanced<D>::first(ax)));
            } else {
              c = pair_cs(p, tab, tst, tpitch, c3, q2);
            }
            const float even = __fsub_rn(__fmul_rn(e_o.x, c.x), __fmul_rn(e_o.y, c.y));
            const float odd = __fadd_rn(__fmul_rn(e_o.x, c.y), __fmul_rn(e_o.y, c.x));
            packed[q2] = pack_pair<BF16>(even, odd);
          }
        }
        // a select chain, not p.out[1 + part]: a runtime index would move the parameters to local memory
        void *o = is_q ? p.out[0] : part == 0 ? p.out[1] : part == 1 ? p.out[2] : part == 2 ? p.out[3] : p.out[4];
        // q, kl, vl go to the token's raster row in the raster form (kg, vg stay in token order)
        const int64_t nd = (p.raster_qkv && (is_q || part <= 1)) ? ((int64_t)c3[0] * p.ey + c3[1]) * p.ex + c3[2] : n;
        const bool kv_local = !is_q && part <= 1;
        const int64_t head_rows = kv_local ? p.kv_rows : (int64_t)p.tokens;
        const int64_t row = kv_local ? p.kv_row0 + nd : nd;
        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(o) + (((int64_t)b * ht + hh) * head_rows + row) * D);
        // When the warp's 32 rows are one contiguous run of the output (every row valid, one
        // batch, token order), each thread's D values go through shared memory, kStageRows rows
        // at a time, and the warp writes the run as whole 512-byte spans; a thread's own row
        // would otherwise be D / 8 stores at a D-element stride, each touching as many lines
        // as there are threads.
        uint4 *const dst0 = reinterpret_cast<uint4 *>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(dst), 0));
        const bool run = p.stage_out && __all_sync(0xffffffffu, valid && dst == dst0 + lane * (D / 8));
        if (run) {
          uint4 *stg = reinterpret_cast<uint4 *>(smem_raw + stage_off) + (warp - 2) * (kStageRows * D / 8);
          constexpr int kChunks = kStageRows * D / 8;  // 16-byte pieces per pass
#pragma unroll
          for (int h2 = 0; h2 < 32 / kStageRows; ++h2) {
            if (lane / kStageRows == h2) {
#pragma unroll
              for (int v = 0; v < D / 8; ++v)
                stg[(lane % kStageRows) * (D / 8) + v] =
                    make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
            }
            __syncwarp();
            uint4 *out = dst0 + h2 * kChunks;
#pragma unroll
            for (int k = lane; k < kChunks; k += 32) out[k] = stg[k];
            __syncwarp();
          }
        } else if (valid) {
#pragma unroll
          for (int v = 0; v < D / 8; ++v)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
      }
      if (has_gate) {
        // this thread's token's gate (heads split over the warps of the lane quarter as the
        // group's heads are): each logit rounded to the storage type with its bias added (as
        // the gate Linear's output would be), then the pair softmax of p3d_gate_pairs, stored
        // at gate[b, h, n]
        using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
        uint32_t gl[kGateRows];
        tmem_ld16(t_lanes + a * Gp + G, *reinterpret_cast<uint32_t(*)[kGateRows]>(gl));
        tmem_wait_ld();
        if (valid) {
          const T *bg = static_cast<const T *>(p.bg);
          T *gate = static_cast<T *>(p.gate);
#pragma unroll
          for (int hg = 0; hg < kGateRows / 2; ++hg) {
            if (2 * hg < p.gate_cols && hg % kSplit == split) {
              const float l0 = to_f32<T>(from_f32<T>(__uint_as_float(gl[2 * hg]) + to_f32<T>(bg[2 * hg])));
              const float l1 = to_f32<T>(from_f32<T>(__uint_as_float(gl[2 * hg + 1]) + to_f32<T>(bg[2 * hg + 1])));
              const float m = fmaxf(l0, l1);
              const float e0 = expf(l0 - m), e1 = expf(l1 - m);
              gate[((int64_t)b * p.heads + hg) * p.tokens + n] = from_f32<T>(e1 / (e0 + e1));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kAccEmpty + a));
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <bool BF16, int D>
int launch_proj(const ProjArgs &a, cudaStream_t stream) {
  const uint64_t es = 2;
  const int K = a.dim;
  CUtensorMap tx, twq, twkv;
  const int gh = a.group_heads;
  {
    const uint64_t dims[3] = {(uint64_t)K, (uint64_t)a.rows, 1};
    const uint64_t strides[2] = {K * es, (uint64_t)a.rows * K * es};
    const uint32_t box[3] = {64, kTile, 1};
    if (int st = encode_operand_sw128(&tx, a.dtype, a.x, 3, dims, strides, box)) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)K, (uint64_t)a.heads * D, 1};
    const uint64_t strides[2] = {K * es, (uint64_t)a.heads * D * K * es};
    const uint32_t box[3] = {64, (uint32_t)(gh * D), 1};
    if (int st = encode_operand_sw128(&twq, a.dtype, a.wq, 3, dims, strides, box)) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)K, (uint64_t)4 * a.kv_heads * D, 1};
    const uint64_t strides[2] = {K * es, (uint64_t)4 * a.kv_heads * D * K * es};
    const uint32_t box[3] = {64, (uint32_t)(gh * D), 1};
    if (int st = encode_operand_sw128(&twkv, a.dtype, a.wkv, 3, dims, strides, box)) return st;
  }
  ProjParams p{};
  p.rows = a.rows;
  p.tokens = a.tokens;
  p.kc = K / 64;
  p.heads = a.heads;
  p.kv_heads = a.kv_heads;
  p.group_heads = gh;
  p.groups_q = (a.heads + gh - 1) / gh;
  p.groups = p.groups_q + (4 * a.kv_heads + gh - 1) / gh;
  DeviceInfo info{};
  if (int st = device_info(&info)) return st;
  p.ctas_per_group = info.sm_count / p.groups > 0 ? info.sm_count / p.groups : 1;
  for (int i = 0; i < 5; ++i) p.out[i] = a.out[i];
  p.kv_rows = a.kv_rows;
  p.kv_row0 = a.kv_row0;
  p.coords = a.coords;
  int tstart = 0;
  for (int i = 0; i < 3; ++i) {
    p.pairs[i] = a.pairs[i];
    p.start[i] = a.start[i];
    p.tpitch[i] = a.pairs[i] | 1;
    p.tstart[i] = tstart;
    tstart += a.ext[i] * p.tpitch[i];
  }
  p.smem_floats = 2 * tstart;
  p.phases = a.phases;
  p.table_floats = a.table_floats;
  p.raster_qkv = a.raster_qkv;
  p.ey = a.ey;
  p.ex = a.ex;
  p.gate_cols = a.gate_cols;
  p.wg = a.wg;
  p.bg = a.bg;
  p.gate = a.gate;
  // shared memory: the W slice and the X ring (always), the phase table when it has at most
  // kMaxTableFloats entries (the budget proj_group_heads reserves for it), then the output
  // staging of the epilogue warps if it still fits
  const size_t table_bytes = 4 * (size_t)p.smem_floats;
  const size_t stage_bytes = (size_t)kEpilogueWarps * kStageRows * D * 2;
  size_t smem = proj_smem_bytes(a.dim, gh * D + (a.gate_cols > 0 ? kGateRows : 0)) - 4 * (size_t)kMaxTableFloats;
  p.table_in_smem = p.smem_floats <= kMaxTableFloats ? 1 : 0;
  p.stage_out = smem + stage_bytes + (p.table_in_smem ? table_bytes : 0) + 1024 <= info.smem_optin ? 1 : 0;
  if (p.stage_out) smem += stage_bytes;
  if (p.table_in_smem) smem += table_bytes;
  const bool balanced = p.pairs[0] == Balanced<D>::count(0) && p.pairs[1] == Balanced<D>::count(1) &&
                        p.pairs[2] == Balanced<D>::count(2);
  auto kernel = balanced ? proj_split_kernel<BF16, D, true> : proj_split_kernel<BF16, D, false>;
  static size_t seen[2][kMaxDevices] = {};
  if (int st = smem_optin(kernel, smem, seen[balanced ? 1 : 0])) return st;
  kernel<<<p.groups * p.ctas_per_group, kThreads, smem, stream>>>(tx, twq, twkv, p);
  P3D_LAUNCH_CHECK();
  return P3D_OK;
}

}  // namespace

size_t proj_smem_bytes(int dim, int group_cols) {
  // W slice + 2 X stages (64-channel boxes of 128-byte rows) + barriers + the phase table (at
  // most kMaxTableFloats) + 1024 alignment slack
  return (size_t)(dim / 64) * group_cols * 128 + 2 * (size_t)(dim / 64) * kTile * 128 + 8 * kNumBars + 16 +
         4 * (size_t)kMaxTableFloats + 1024;
}

int proj_group_heads(int head_dim, int heads, int kv_heads, int dim, size_t smem_limit) {
  int gh = 256 / head_dim;  // MMA N <= 256 and 2 accumulators in 512 TMEM columns
  if (gh > heads) gh = heads;
  if (gh > 4 * kv_heads) gh = 4 * kv_heads;
  // the W slice shrinks with the group (+ 1 KB of static shared memory)
  while (gh > 1 && proj_smem_bytes(dim, gh * head_dim) + 1024 > smem_limit) --gh;
  return gh < 1 ? 1 : gh;
}

int launch_proj_split(const ProjArgs &a, cudaStream_t stream) {
  if (a.rows == 0) return P3D_OK;
  const bool bf16 = a.dtype == P3D_BF16;
  switch (a.head_dim) {
    case 16: return bf16 ? launch_proj<true, 16>(a, stream) : launch_proj<false, 16>(a, stream);
    case 32: return bf16 ? launch_proj<true, 32>(a, stream) : launch_proj<false, 32>(a, stream);
    case 48: return bf16 ? launch_proj<true, 48>(a, stream) : launch_proj<false, 48>(a, stream);
    case 64: return bf16 ? launch_proj<true, 64>(a, stream) : launch_proj<false, 64>(a, stream);
    case 128: return bf16 ? launch_proj<true, 128>(a, stream) : launch_proj<false, 128>(a, stream);
    default: return fail(P3D_ERR_UNSUPPORTED, "p3d_qkv_project: head_dim %d", a.head_dim);
  }
}

int take_proj_errors(unsigned *flags) {
  unsigned v = 0, zero = 0;
  P3D_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_proj_errors, sizeof(v)));
  P3D_CUDA_TRY(cudaMemcpyToSymbol(g_proj_errors, &zero, sizeof(zero)));
  *flags |= v;
  return P3D_OK;
}

}  // namespace p3d

using namespace p3d;

extern "C" int p3d_qkv_project_supported(int dtype, int dim, int heads, int kv_heads, int head_dim) {
  if (dtype != P3D_BF16 && dtype != P3D_F16) return 0;
  if (head_dim != 16 && head_dim != 32 && head_dim != 48 && head_dim != 64 && head_dim != 128) return 0;
  if (dim < 64 || dim % 64 != 0 || heads < 1 || kv_heads < 1 || heads % kv_heads != 0) return 0;
  DeviceInfo info{};
  if (device_info(&info) != P3D_OK) return 0;
  const int gh = proj_group_heads(head_dim, heads, kv_heads, dim, info.smem_optin);
  return proj_smem_bytes(dim, gh * head_dim) + 1024 <= info.smem_optin ? 1 : 0;
}

extern "C" int p3d_qkv_gate_project_supported(int dtype, int dim, int heads, int kv_heads, int head_dim) {
  if (!p3d_qkv_project_supported(dtype, dim, heads, kv_heads, head_dim) || 2 * heads > kGateRows) return 0;
  DeviceInfo info{};
  if (device_info(&info) != P3D_OK) return 0;
  // the last group carries the gate's logit rows: its MMA N and its two TMEM accumulators grow by kGateRows
  const int cols = proj_group_heads(head_dim, heads, kv_heads, dim, info.smem_optin) * head_dim + kGateRows;
  return cols <= 256 && proj_smem_bytes(dim, cols) + 1024 <= info.smem_optin ? 1 : 0;
}

namespace {
int qkv_project(const char *name, const void *x, const void *wq, const void *wkv, const void *wg, const void *bg,
                void *q, void *kl, void *vl, void *kg, void *vg, void *gate, int dtype, int batch, int heads,
                int kv_heads, int tokens, int dim, int head_dim, const int64_t *coords, int pz, int py, int px,
                const float *phases, int ez, int ey, int ex, int64_t kv_rows, int64_t kv_row0, unsigned flags,
                void *stream) {
  P3D_CHECK_ARG(x && wq && wkv && q && kl && vl && kg && vg && coords && phases, "%s: null pointer", name);
  if (kv_rows == 0) kv_rows = tokens;
  P3D_CHECK_ARG(kv_row0 >= 0 && kv_row0 + tokens <= kv_rows, "%s: kl / vl rows [%lld, %lld) outside "
                "%lld rows", name, (long long)kv_row0, (long long)(kv_row0 + tokens), (long long)kv_rows);
  P3D_CHECK_ARG((flags & ~P3D_SPLIT_RASTER_QKV) == 0u, "%s: unknown flags 0x%x", name, flags);
  P3D_CHECK_ARG(!(flags & P3D_SPLIT_RASTER_QKV) || (int64_t)ez * ey * ex == tokens,
                "%s: raster rows need the coordinate extents to be the token grid (%d x %d x %d != %d)",
                name, ez, ey, ex, tokens);
  P3D_CHECK_ARG(batch >= 0 && tokens >= 0 && (int64_t)batch * tokens < (int64_t(1) << 31),
                "%s: bad batch / token counts", name);
  P3D_CHECK_ARG(pz >= 0 && py >= 0 && px >= 0 && 2 * (pz + py + px) == head_dim && ez >= 1 && ey >= 1 && ex >= 1,
                "%s: bad rotation pairs / extents", name);
  for (const void *t : {x, wq, wkv, (const void *)q, (const void *)kl, (const void *)vl, (const void *)kg,
                        (const void *)vg})
    P3D_CHECK_ARG(((uintptr_t)t & 15) == 0, "%s: 16-byte aligned tensors required", name);
  if (wg) {
    P3D_CHECK_ARG(bg && gate, "%s: null pointer", name);
    P3D_CHECK_ARG(((uintptr_t)wg & 15) == 0 && ((uintptr_t)bg & 1) == 0 && ((uintptr_t)gate & 1) == 0,
                  "%s: 16-byte aligned gate weight required", name);
  }
  if (!(wg ? p3d_qkv_gate_project_supported : p3d_qkv_project_supported)(dtype, dim, heads, kv_heads, head_dim))
    return fail(P3D_ERR_UNSUPPORTED, "%s: unsupported shape (dtype %d, dim %d, heads %d/%d, D %d)", name, dtype, dim,
                heads, kv_heads, head_dim);
  ProjArgs a{};
  a.dtype = dtype;
  a.rows = batch * tokens;
  a.tokens = tokens;
  a.dim = dim;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.head_dim = head_dim;
  DeviceInfo info{};
  if (int st = device_info(&info)) return st;
  a.group_heads = proj_group_heads(head_dim, heads, kv_heads, dim, info.smem_optin);
  a.x = x;
  a.wq = wq;
  a.wkv = wkv;
  a.kv_rows = kv_rows;
  a.kv_row0 = kv_row0;
  a.out[0] = q;
  a.out[1] = kl;
  a.out[2] = vl;
  a.out[3] = kg;
  a.out[4] = vg;
  a.raster_qkv = (flags & P3D_SPLIT_RASTER_QKV) ? 1 : 0;
  a.ey = ey;
  a.ex = ex;
  a.coords = coords;
  a.pairs[0] = pz;
  a.pairs[1] = py;
  a.pairs[2] = px;
  a.start[0] = 0;
  a.start[1] = ez * pz;
  a.start[2] = ez * pz + ey * py;
  a.ext[0] = ez;
  a.ext[1] = ey;
  a.ext[2] = ex;
  a.phases = phases;
  a.table_floats = 2 * (ez * pz + ey * py + ex * px);
  a.gate_cols = wg ? 2 * heads : 0;
  a.wg = wg;
  a.bg = bg;
  a.gate = gate;
  return launch_proj_split(a, static_cast<cudaStream_t>(stream));
}
}  // namespace

extern "C" int p3d_qkv_project(const void *x, const void *wq, const void *wkv, void *q, void *kl, void *vl, void *kg,
                               void *vg, int dtype, int batch, int heads, int kv_heads, int tokens, int dim,
                               int head_dim, const int64_t *coords, int pz, int py, int px, const float *phases,
                               int ez, int ey, int ex, int64_t kv_rows, int64_t kv_row0, unsigned flags,
                               void *stream) {
  return qkv_project("p3d_qkv_project", x, wq, wkv, nullptr, nullptr, q, kl, vl, kg, vg, nullptr, dtype, batch, heads,
                     kv_heads, tokens, dim, head_dim, coords, pz, py, px, phases, ez, ey, ex, kv_rows, kv_row0, flags,
                     stream);
}

extern "C" int p3d_qkv_gate_project(const void *x, const void *wq, const void *wkv, const void *wg, const void *bg,
                                    void *q, void *kl, void *vl, void *kg, void *vg, void *gate, int dtype, int batch,
                                    int heads, int kv_heads, int tokens, int dim, int head_dim, const int64_t *coords,
                                    int pz, int py, int px, const float *phases, int ez, int ey, int ex,
                                    int64_t kv_rows, int64_t kv_row0, unsigned flags, void *stream) {
  P3D_CHECK_ARG(wg, "p3d_qkv_gate_project: null pointer");
  return qkv_project("p3d_qkv_gate_project", x, wq, wkv, wg, bg, q, kl, vl, kg, vg, gate, dtype, batch, heads,
                     kv_heads, tokens, dim, head_dim, coords, pz, py, px, phases, ez, ey, ex, kv_rows, kv_row0, flags,
                     stream);
}
