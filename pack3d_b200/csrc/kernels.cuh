// Internal launch interfaces between the C ABI (capi.cu) and the kernel files.
#pragma once

#include "common.cuh"

namespace p3d {

// Shared by every entry point that takes a p3d_operator (capi.cu): the argument checks of
// p3d_attn_fwd / p3d_attn_bwd and the descriptor -> launch-argument conversions.
int summaries_of(const p3d_operator *op);
int validate(const p3d_operator *op);

struct PoolArgs {
  const void *k, *v;  // [BG, N, D]
  const float *weight, *bias;
  const int32_t *blocks;
  int fine_blocks, slots, pool_size, summaries;
  void *sk, *sv;      // [BG, M, D] dtype
  float *sk32, *sv32; // optional fp32 copies
  int dtype, bg, tokens, head_dim;
  float temperature;
  bool vec;           // 16-byte row loads allowed
};
int launch_pool_fwd(const PoolArgs &p, cudaStream_t stream);

struct PoolBwdArgs {
  const void *k, *v;
  const float *weight, *bias;
  const int32_t *blocks;
  int fine_blocks, slots, pool_size, summaries;
  const float *dsk, *dsv;  // [BG, M, D] fp32
  void *dk, *dv;           // [BG, N, D] dtype
  float *dw_part;          // [BG*M, D]
  float *db_part;          // [BG*M, V]
  int dtype, bg, tokens, head_dim;
  float temperature;
  bool vec;
};
int launch_pool_bwd(const PoolBwdArgs &p, cudaStream_t stream);

// ---- indexed (neighbour-table) kernels: every dtype, every head_dim <= 128 --------------
struct IndexedArgs {
  int dtype, gate_dtype;
  int batch, heads, kv_heads, tokens, head_dim, summaries;
  const void *q, *kl, *vl, *sk, *sv;    // sk, sv [B,G,M,D] dtype
  const int32_t *neighbors;
  int width;
  const int32_t *reverse;
  int reverse_width;
  const void *gate;
  const float *sl, *sg;
  int y_rows;  // global/mix forward: y token-major [B,N,H,D]
};

// Local branch forward: ol [B,H,N,D] dtype, lse_l [B,H,N] fp32 (nullable; +inf for all-masked rows).
IndexedArgs indexed_args(const p3d_operator *op, const void *sk, const void *sv);
PoolArgs pool_args(const p3d_operator *op, void *sk, void *sv);
int launch_local_fwd_indexed(const IndexedArgs &a, void *ol, float *lse_l, cudaStream_t s);
// Global branch forward + mix: y, og (nullable), lse_g (nullable).
int launch_global_fwd_mix(const IndexedArgs &a, const void *ol, void *y, void *og, float *lse_g,
                          cudaStream_t s);

// Backward pieces.
// ---- fused projection + split + axial RoPE (csrc/proj.cu) ---------------------------------
struct ProjArgs {
  int dtype;                    // P3D_BF16 / P3D_F16
  int rows, tokens, dim;        // rows = batch * tokens of x [rows, dim]
  int heads, kv_heads, head_dim;
  int group_heads;              // head rows per column group (proj_group_heads)
  const void *x, *wq, *wkv;     // wq [heads*D, dim], wkv [4*kv_heads*D, dim] (nn.Linear weights)
  void *out[5];                 // q [B,H,N,D], kl, vl, kg, vg [B,G,N,D]
  const int64_t *coords;        // [N, 3]
  int pairs[3], start[3];
  int ext[3];                   // coordinate extents (rows of the phase table per axis)
  const float *phases;
  int table_floats;             // floats in the phase table
  int raster_qkv, ey, ex;       // q, kl, vl rows at each token's raster index (ey x ex planes)
  int64_t kv_rows, kv_row0;     // kl, vl: [B, G, kv_rows, D], token row n at kv_row0 + n
  int gate_cols;                // 2 * heads with the gate folded in (wg [2H, dim], bg [2H], gate [B,H,N]), else 0
  const void *wg, *bg;
  void *gate;
};
int proj_group_heads(int head_dim, int heads, int kv_heads, int dim, size_t smem_limit);
size_t proj_smem_bytes(int dim, int group_cols);
int launch_proj_split(const ProjArgs &a, cudaStream_t stream);
int take_proj_errors(unsigned *flags);
int take_peer_errors(unsigned *flags);  // peer.cu

struct MixBwdArgs {
  int dtype, gate_dtype, bh, tokens, head_dim, chunk_rows;
  int heads, dy_rows;  // dy_rows: dy is [B,N,H,D] (row (b,h,i) at ((b N + i) H + h) D)
  const void *dy, *ol, *og, *gate;
  const float *sl, *sg;
  void *dol, *dog;         // dtype
  float *delta_l, *delta_g;
  void *dgate;             // gate dtype
  float *dsl_part, *dsg_part;  // [bh * ceil(N/chunk_rows), D]
};
int launch_mix_bwd(const MixBwdArgs &a, cudaStream_t s);
inline int mix_bwd_chunk_rows() { return 128; }

int launch_local_dq_indexed(const IndexedArgs &a, const void *dol, const float *lse_l, const float *delta_l,
                            void *dq, cudaStream_t s);
int launch_local_dkv_indexed(const IndexedArgs &a, const void *dol, const float *lse_l, const float *delta_l,
                             void *dkl, void *dvl, cudaStream_t s);
// Adds the global-branch dQ into dq (which holds the local-branch dQ).
int launch_global_dq(const IndexedArgs &a, const void *dog, const float *lse_g, const float *delta_g, void *dq,
                     cudaStream_t s);
// Global-branch dSK / dSV split partials [B*G, splits, M, D] fp32.
int launch_global_dkv(const IndexedArgs &a, const void *dog, const float *lse_g, const float *delta_g,
                      int splits, float *dk_part, float *dv_part, cudaStream_t s);
inline int global_dkv_splits(int tokens) {
  int s = (tokens + 1023) / 1024;
  return s < 1 ? 1 : (s > 32 ? 32 : s);
}

// Deterministic reductions.
// out[a, c] = sum_{s < S} in[(a * S + s) * C + c]
int launch_sum_middle(const float *in, float *out, int64_t outer, int S, int64_t C, cudaStream_t s);
// out[c] = sum_{r < R} in[r * C + c]; tmp needs ceil(R / 256) * C floats.
int launch_sum_rows(const float *in, float *out, int64_t R, int64_t C, float *tmp, cudaStream_t s);
constexpr int kSumRowsPerGroup = 128;  // rows per first-pass group of launch_sum_rows
inline int64_t sum_rows_tmp(int64_t R, int64_t C) { return ((R + kSumRowsPerGroup - 1) / kSumRowsPerGroup) * C; }

// ---- tensor-core (tcgen05) fused forward on complete voxel stencils --------------------
struct StencilFwdArgs {
  int dtype, gate_dtype;
  int batch, heads, kv_heads, head_dim, summaries;
  int grid[3];                        // query (centre) buffer: grid[0] planes of grid[1] x grid[2]
  // z-slab extents (whole volume: global_planes = k_planes = grid[0], q_z0 = k_z0 = 0):
  int global_planes;                  // planes of the whole volume (keys outside are masked)
  int q_z0;                           // global z of the query buffer's first plane
  int k_z0, k_planes;                 // global z and plane count of the kl / vl buffers
  const void *q, *kl, *vl, *sk, *sv;  // q/kl/vl in raster order (contiguous [B,H|G,Z,Y,X,D])
  const int32_t *raster_to_packed;    // output row map (NULL = raster)
  const void *gate;
  const float *sl, *sg;
  void *y, *ol, *og;                  // ol/og nullable
  float *lse_l, *lse_g;               // nullable
  int y_rows;                         // y token-major [B,N,H,D]
  int radius;                         // stencil radius (1 or 2, all axes)
  const float *summary_bound;         // [B*G] max_j |sk_j| (launch_summary_bound), or NULL
  int tile_z_begin, tile_z_end;       // 4-plane query tiles [begin, end) of the buffer; 0, 0: all
};
// bound[bg] = max over the summaries j of |sk[bg, j, :]| (fp32 Euclidean norm, rounded up by
// 2^-10), sk [BG, M, D] in a 16-bit dtype: the stencil forward's per-row bound on the global
// scores.
int launch_summary_bound(const void *sk, int dtype, int bg, int summaries, int head_dim, float *bound,
                         cudaStream_t stream);
// Read-and-clear the device failure bits of the tensor-core kernel files (OR-ed into *flags).
int take_fwd_errors(unsigned *flags);

bool stencil_fwd_supported(int dtype, int head_dim, const int radius[3], int summaries);
int launch_stencil_fwd(const StencilFwdArgs &a, cudaStream_t s);

// Tensor-core backward over a complete radius-2 stencil (stencil_bwd.cu).
struct StencilBwdArgs {
  int dtype;
  int radius;                           // stencil radius (1 or 2, all axes)
  int batch, heads, kv_heads, head_dim, summaries;
  int grid[3];                          // centre buffer (queries for dQ, keys for dK / dV)
  // z-slab extents (whole volume: global_planes = k_planes = grid[0], q_z0 = k_z0 = 0):
  int global_planes, q_z0, k_z0, k_planes;
  const void *q, *kl, *vl, *dol, *dog;  // raster order (contiguous [B,H|G,Z,Y,X,D])
  const void *sk, *sv;                  // [B,G,M,D]
  const float *lse_l, *lse_g, *delta_l, *delta_g;  // [B*H, N] in the layout's row order
  const int32_t *raster_to_packed;      // row map of lse / delta / outputs (NULL = raster)
  void *dq;                             // [B,H,N,D] in the layout's row order
  void *dkl, *dvl;                      // [B,G,N,D] in the layout's row order
  // query-side buffers of the local dK / dV (whole volume: the centre buffers, x_z0 = 0,
  // x_planes = grid[0]; a z-slab: the rank's planes plus the neighbours' halo planes)
  const void *q_halo, *dol_halo;
  const float *lse_l_halo, *delta_l_halo;
  int x_z0, x_planes;
};
int launch_stencil_bwd_dq(const StencilBwdArgs &a, cudaStream_t s);
int launch_stencil_bwd_dkv(const StencilBwdArgs &a, cudaStream_t s);

// Tensor-core global dSK / dSV split partials (any token order).
struct GlobalDkvArgs {
  int dtype;
  int batch, heads, kv_heads, tokens, head_dim, summaries;
  int splits, per_split;          // from global_dkv_tc_splits
  const void *q, *dog;            // [B,H,N,D]
  const void *sk, *sv;            // [B,G,M,D]
  const float *lse_g, *delta_g;   // [B*H, N]
  float *dk_part, *dv_part;       // [B*G, splits, M, D]
};
bool global_dkv_tc_supported(int dtype, int head_dim, int summaries);
void global_dkv_tc_splits(int batch, int heads, int kv_heads, int tokens, int summaries, int sm_count, int *splits,
                          int *per_split);
int launch_global_dkv_tc(const GlobalDkvArgs &a, cudaStream_t s);
int take_bwd_errors(unsigned *flags);

}  // namespace p3d
