/*
 * pack3d_b200 -- C ABI of the Blackwell (sm_100a) PACK3D operator library.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream and returns a
 * p3d_status.  Nothing here allocates device memory: outputs, saved state
 * and workspaces are provided by the caller (the Python host layer uses
 * torch tensors for that).  No entry point aborts the process; on failure
 * p3d_last_error() describes the problem (thread-local).
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   p3d_rope           src/pack3d/backends/triton/rotary.py:94-106  rotate_projections()
 *                      (kernel _rotate rotary.py:11-45, inverse for _Rotary.backward :66-70)
 *   p3d_pool_fwd       src/pack3d/backends/triton/kernels.py:13-40  _pool
 *   p3d_attn_fwd       src/pack3d/backends/triton/kernels.py:289-311 forward()
 *   p3d_attn_bwd       src/pack3d/backends/triton/kernels.py:314-356 backward()
 *   p3d_*_workspace    (no counterpart: the reference allocates scratch with torch.empty,
 *                      kernels.py:275-277,319-351)
 */
#ifndef PACK3D_B200_H
#define PACK3D_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define P3D_ABI_VERSION 5

#if defined(__GNUC__)
#define P3D_API __attribute__((visibility("default")))
#else
#define P3D_API
#endif

typedef enum {
  P3D_OK = 0,
  P3D_ERR_INVALID_ARGUMENT = 1, /* shape / dtype / pointer / limit violation */
  P3D_ERR_UNSUPPORTED = 2,      /* valid input outside what the library implements */
  P3D_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed */
  P3D_ERR_WORKSPACE = 4,        /* workspace pointer missing or too small */
  P3D_ERR_DEVICE = 5            /* no usable sm_100 device */
} p3d_status;

typedef enum { P3D_F32 = 0, P3D_F16 = 1, P3D_BF16 = 2 } p3d_dtype;

/* Attention-forward flags. */
#define P3D_FWD_SAVE_STATE 1u   /* write ol, og, lse_l, lse_g for the backward */
#define P3D_FWD_FORCE_INDEXED 2u /* use the indexed (neighbour-table) kernels even on a stencil */
#define P3D_FWD_SUMMARIES_GIVEN 4u /* sk, sv already hold the pooled summaries: skip stage (b) */
#define P3D_FWD_Y_ROWS 8u /* write y token-major, [B,N,H,D] (the layout to_out reads), not [B,H,N,D] */
/* q, kl, vl are stored in raster order (rows at each token's raster index; p3d_qkv_split with
 * P3D_SPLIT_RASTER_QKV) although the layout is permuted: the tensor-core forward reads them as
 * they are instead of gathering raster copies.  Needs the tensor-core path
 * (p3d_stencil_fwd_supported); y, gate and the saved state keep the layout's row order. */
#define P3D_FWD_RASTER_QKV 16u

/* p3d_qkv_split flags: write q, kl, vl at each token's raster index (z * ey + y) * ex + x of its
 * coordinates (the extents must then be the token grid); kg, vg keep the token rows. */
#define P3D_SPLIT_RASTER_QKV 1u

/* Static description string of a status code. */
P3D_API const char *p3d_strerror(int status);
/* Detail of the last failure on the calling thread ("" if none). */
P3D_API const char *p3d_last_error(void);
P3D_API int p3d_abi_version(void);
/* Number of visible sm_100 devices (0 without a GPU); never fails. */
P3D_API int p3d_device_count(void);
/* Read and clear the device-side failure flags of the current device.  Bit 0: a
 * bounded wait inside a tensor-core kernel timed out and the kernel unwound; bits
 * 1-4 name the waiting role (2 TMA producer, 4 MMA issuer, 8 softmax / epilogue,
 * 16 a drain before tensor memory is freed); bit 5 (32): a peer-exchange wait
 * (p3d_peer_wait) ran out.  Synchronises with the device.  No
 * reference counterpart (the Triton kernels have no device-side waits). */
P3D_API int p3d_device_errors(unsigned *flags);

/*
 * Axial rotary embedding of a strided [B, H, N, D] tensor into a contiguous
 * [B, H, N, D] output (same dtype).  Element (b,h,n,d) of x is read at
 * x + b*sb + h*sh + n*sn + d*sd (strides in elements).  Pair i of axis a
 * (axes z,y,x own pairs pz,py,px in that channel order, interleaved
 * (even, odd)) turns by coord[n][a] * freqs[i] radians, where freqs holds the
 * concatenated per-axis frequency vectors (pz + py + px floats) and
 * coord[n][a] = coords[n*coord_sn + a*coord_sa].  If phases != NULL it holds
 * (cos, sin) float pairs for every (axis, coordinate value, pair): axis a's
 * block starts at entry sum_{a'<a} extent[a'] * pairs[a'] and coordinate c,
 * pair i is entry start + c * pairs[a] + i; coordinates must then lie in
 * [0, extent[a]).  packed != 0 uses the row index n as the axis-0 position
 * (packed-sequence RoPE; pairs must be (D/2, 0, 0)).  inverse != 0 applies the
 * transposed rotation (the backward).  Replaces rotary.py:94-106.
 */
P3D_API int p3d_rope(const void *x, int64_t sb, int64_t sh, int64_t sn, int64_t sd, void *out, int dtype,
             int batch, int heads, int tokens, int head_dim, const int64_t *coords, int64_t coord_sn,
             int64_t coord_sa, int pz, int py, int px, const float *freqs, const float *phases,
             int ez, int ey, int ex, int packed, int inverse, void *stream);

/*
 * Two-stage summary pooling (compression.py:7-44, kernels.py:13-40):
 * k, v [B, G, N, D] (dtype) -> sk, sv [B, G, M, D] (dtype), M = ceil(F / pool).
 * blocks [F, V] int32 token rows (-1 = empty slot); weight [D], bias [V] fp32.
 * If sk32/sv32 are non-NULL the fp32 summaries are written there as well.
 */
P3D_API int p3d_pool_fwd(const void *k, const void *v, const float *weight, const float *bias,
                 const int32_t *blocks, int fine_blocks, int slots, int pool_size, void *sk, void *sv,
                 float *sk32, float *sv32, int dtype, int batch, int kv_heads, int tokens, int head_dim,
                 float temperature, void *stream);

/*
 * Layer glue (reference attention.py:53-89), HBM-bound helpers of the layer's inference path.
 * p3d_layer_norm: y = LayerNorm(x) over the last dimension (nn.LayerNorm, attention.py:64),
 *   x, y [rows, dim], weight, bias [dim], all in dtype (bf16 / f16), fp32 statistics.
 * p3d_qkv_split: from the projections qp [B,N,H*D] (to_q) and kvp [B,N,4*G*D] (to_kv, channel
 *   blocks kl, vl, kg, vg; attention.py:70-72) write q, kl, vl, kg, vg [B,H|G,N,D]; q, kl, kg
 *   rotated by the axial RoPE phase table (the table of p3d_rope, rotary.py:74-85; coordinates
 *   coords [N,3]), vl, vg copied.  One pass in place of three rotations and two strided copies
 *   (rotary.py:94-106 and the .contiguous() copies of autograd.py:13).
 */
P3D_API int p3d_layer_norm(const void *x, const void *weight, const void *bias, void *y, int dtype, int64_t rows,
                   int dim, float eps, void *stream);
P3D_API int p3d_qkv_split(const void *qp, const void *kvp, void *q, void *kl, void *vl, void *kg, void *vg,
                  int dtype, int batch, int heads, int kv_heads, int tokens, int head_dim, const int64_t *coords,
                  int pz, int py, int px, const float *phases, int ez, int ey, int ex, unsigned flags,
                  void *stream);

/* p3d_qkv_gate_split: p3d_qkv_split plus the layer's gate, from one GEMM output.  proj is
 *   [B*N, proj_cols] (row stride proj_cols elements, a multiple of 8): columns [0, H*D) the to_q
 *   projection, the next 4*G*D the to_kv projection, the next 2*H the gate logits (head-major
 *   pairs, as nn.Linear(dim, 2H) of attention.py:64 lays them out); further columns are
 *   ignored.  q .. vg as p3d_qkv_split; gate [B, H, N] = softmax over each logit pair, second
 *   entry (attention.py:84-86), computed in fp32 and rounded once.  Replaces the to_q / to_kv
 *   / gate Linear outputs' reshapes, the rotations and the gate softmax of attention.py:70-86
 *   in one pass; the caller runs one GEMM with the three weights stacked. */
/* p3d_gate_pairs: the layer's gate from its Linear's output: logits [B*N, stride] (row stride in
 *   elements; columns 2h, 2h + 1 are head h's pair), gate [B, H, N] = softmax over each pair,
 *   second entry (attention.py:84-86), in fp32, rounded once.  Used beside p3d_qkv_project. */
P3D_API int p3d_gate_pairs(const void *logits, int stride, void *gate, int dtype, int batch, int heads, int tokens,
                   void *stream);

P3D_API int p3d_qkv_gate_split(const void *proj, int proj_cols, void *q, void *kl, void *vl, void *kg, void *vg,
                       void *gate, int dtype, int batch, int heads, int kv_heads, int tokens, int head_dim,
                       const int64_t *coords, int pz, int py, int px, const float *phases, int ez, int ey, int ex,
                       unsigned flags, void *stream);

/*
 * p3d_qkv_project: the projections and the split in one kernel -- the two nn.Linear calls of
 *   attention.py:70-72 (to_q, to_kv; weights wq [H*D, dim], wkv [4*G*D, dim], no bias) on x
 *   [B*N, dim], followed by p3d_qkv_split: each projection is rounded to dtype, as the GEMM's
 *   output would be, then rotated and stored head-major as p3d_qkv_split stores it.  The
 *   projections never reach HBM.  flags: P3D_SPLIT_RASTER_QKV as for p3d_qkv_split.  Shapes
 *   p3d_qkv_project_supported() rejects return P3D_ERR_UNSUPPORTED (callers then run the
 *   GEMMs and p3d_qkv_split).  kl and vl are stored [B, G, kv_rows, D] with token row n at
 *   row kv_row0 + n (kv_rows 0: tokens, the dense layout): a z-slab rank writes its keys and
 *   values straight between the halo rows of its extended buffers.
 */
P3D_API int p3d_qkv_project_supported(int dtype, int dim, int heads, int kv_heads, int head_dim);
P3D_API int p3d_qkv_project(const void *x, const void *wq, const void *wkv, void *q, void *kl, void *vl, void *kg,
                    void *vg, int dtype, int batch, int heads, int kv_heads, int tokens, int dim, int head_dim,
                    const int64_t *coords, int pz, int py, int px, const float *phases, int ez, int ey, int ex,
                    int64_t kv_rows, int64_t kv_row0, unsigned flags, void *stream);
/*
 * p3d_qkv_gate_project: p3d_qkv_project with the gate Linear folded in -- attention.py:84-86
 *   (`self.gate(x)`, its pair softmax and the transpose), the job of a third GEMM and
 *   p3d_gate_pairs: wg [2*heads, dim] and bg [2*heads] (nn.Linear weight and bias, dtype),
 *   gate [B, H, N] = softmax(logits[b, n, 2h .. 2h + 1])[1], each logit rounded to dtype with
 *   its bias added, as the Linear's output would be.  q, kl, vl, kg, vg are the bits
 *   p3d_qkv_project writes.  p3d_qkv_gate_project_supported() (heads <= 8 and room for the
 *   logit rows beside the last column group's) rejects: P3D_ERR_UNSUPPORTED.
 */
P3D_API int p3d_qkv_gate_project_supported(int dtype, int dim, int heads, int kv_heads, int head_dim);
P3D_API int p3d_qkv_gate_project(const void *x, const void *wq, const void *wkv, const void *wg, const void *bg,
                         void *q, void *kl, void *vl, void *kg, void *vg, void *gate, int dtype, int batch,
                         int heads, int kv_heads, int tokens, int dim, int head_dim, const int64_t *coords,
                         int pz, int py, int px, const float *phases, int ez, int ey, int ex, int64_t kv_rows,
                         int64_t kv_row0, unsigned flags, void *stream);

/*
 * Layer glue of the training path (their backward halves):
 * p3d_qkv_merge: the backward of p3d_qkv_split -- replaces _Rotary.backward (rotary.py:66-70,
 *   the inverse rotation of dq, dkl, dkg) and the transposes / chunk concatenation autograd
 *   does for attention.py:70-72: dq [B,H,N,D], dkl, dvl, dkg, dvg [B,G,N,D] -> dqp [B,N,H*D],
 *   dkvp [B,N,4*G*D] (channel blocks kl, vl, kg, vg).  Same arguments as p3d_qkv_split;
 *   bit-identical to rotating back with p3d_rope (inverse = 1) and copying.
 * p3d_layer_norm_bwd: the backward of p3d_layer_norm (nn.LayerNorm, attention.py:64): dx
 *   [rows, dim] in dtype, dweight and dbias [dim] fp32 (sums over rows in fixed order,
 *   bitwise repeatable); workspace of p3d_layer_norm_bwd_workspace(rows, dim) bytes.
 * p3d_layer_norm_bwd_residual: p3d_layer_norm_bwd with dres [rows, dim] (dtype), the gradient
 *   that reaches the LayerNorm's input through the layer's outer residual (attention.py:64 and
 *   :89, `residual + to_out(...)` with `x = norm(residual)`): dx = round(LayerNorm dx) + dres,
 *   rounded to dtype -- the same bits as autograd's sum of the two gradients, in one pass.
 *   Same workspace.
 */
P3D_API int p3d_qkv_merge(const void *dq, const void *dkl, const void *dvl, const void *dkg, const void *dvg,
                  void *dqp, void *dkvp, int dtype, int batch, int heads, int kv_heads, int tokens, int head_dim,
                  const int64_t *coords, int pz, int py, int px, const float *phases, int ez, int ey, int ex,
                  void *stream);
P3D_API size_t p3d_layer_norm_bwd_workspace(int64_t rows, int dim);
P3D_API int p3d_layer_norm_bwd(const void *x, const void *weight, const void *dy, void *dx, float *dweight,
                       float *dbias, int dtype, int64_t rows, int dim, float eps, void *workspace,
                       size_t workspace_bytes, void *stream);
P3D_API int p3d_layer_norm_bwd_residual(const void *x, const void *weight, const void *dy, const void *dres,
                                void *dx, float *dweight, float *dbias, int dtype, int64_t rows, int dim,
                                float eps, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Geometry tables (host code, no GPU): the native builders behind pack3d_b200.geometry for
 * complete voxel stencils -- replace the tensor passes of build_layout's neighbour table and
 * prepare_geometry's reverse adjacency (reference geometry.py:224-266, 54-101) and of
 * TokenLayout.repack (geometry.py:190-220); bit-identical, multithreaded over rows
 * (threads <= 0: all hardware threads).
 * p3d_stencil_neighbors: order [n] int64 (packed row -> raster index of a Z x Y x X grid) ->
 *   neighbors [n, W] int32 (W = prod(2r+1), offsets z-major from -r, -1 outside) and sorted
 *   [n, W] (each row's valid entries ascending, -1 last); *max_valid = widest row.
 * p3d_repack_neighbors: new row i = old row perm[i]: nb_new [n, W] = old table transported,
 *   sorted and *max_valid as above.
 */
P3D_API int p3d_stencil_neighbors(int Z, int Y, int X, int rz, int ry, int rx, const int64_t *order, int64_t n,
                          int32_t *neighbors, int32_t *sorted, int32_t *max_valid, int threads);
P3D_API int p3d_repack_neighbors(int64_t n, int width, const int32_t *nb_old, const int64_t *perm,
                         int32_t *nb_new, int32_t *sorted, int32_t *max_valid, int threads);

/* Operator arguments shared by forward and backward (all device pointers, contiguous). */
typedef struct {
  int32_t batch, heads, kv_heads, tokens, head_dim;
  int32_t dtype;      /* p3d_dtype of q, kl, vl, kg, vg, y, ol, og, sk, sv, dq.. dvg */
  int32_t gate_dtype; /* p3d_dtype of gate and dgate */
  float temperature;
  const void *q, *kl, *vl, *kg, *vg; /* q [B,H,N,D]; the others [B,G,N,D]; q/kl/kg rotated */
  const float *pool_weight;          /* [D] */
  const float *slot_bias;            /* [V] */
  const void *gate;                  /* [B,H,N] */
  const float *local_scale;          /* [D] */
  const float *global_scale;         /* [D] */
  /* geometry */
  const int32_t *neighbors; /* [N, width], -1 pads */
  int32_t width;
  const int32_t *reverse_neighbors; /* [N, reverse_width] */
  int32_t reverse_width;
  const int32_t *blocks; /* [fine_blocks, slots] */
  int32_t fine_blocks, slots, pool_size;
  /* complete voxel stencil (optional): grid extents, radius, raster->packed row map */
  int32_t stencil; /* nonzero when the neighbour table is the full radius stencil of the grid */
  int32_t grid[3];
  int32_t radius[3];
  const int32_t *raster_to_packed; /* [N] or NULL for raster storage */
  uint32_t options;                 /* P3D_OPT_* bits (0: pick the fastest kernels) */
} p3d_operator;

/* p3d_operator.options: run only the neighbour-table (indexed) kernels, as the reference's
 * Triton backend is structured -- for comparison and testing. */
#define P3D_OPT_INDEXED_ONLY 1u
/* p3d_operator.options: the dy of p3d_attn_bwd / p3d_bwd_mix is token-major, [B,N,H,D] (the
 * layout of the output projection's input gradient), instead of [B,H,N,D]. */
#define P3D_OPT_DY_ROWS 2u

/*
 * Forward (kernels.py:289-311).  Writes y [B,H,N,D] and the summaries sk, sv
 * [B,G,M,D].  With P3D_FWD_SAVE_STATE also ol, og [B,H,N,D] (dtype) and
 * lse_l, lse_g [B,H,N] fp32 (all-masked local rows store +inf).
 * workspace: p3d_attn_fwd_workspace() bytes (may be 0).
 */
P3D_API int p3d_attn_fwd(const p3d_operator *op, void *y, void *sk, void *sv, void *ol, void *og, float *lse_l,
                 float *lse_g, unsigned flags, void *workspace, size_t workspace_bytes, void *stream);
P3D_API size_t p3d_attn_fwd_workspace(const p3d_operator *op, unsigned flags);

/* 1 when p3d_attn_fwd runs the tensor-core stencil kernel for these properties of a complete
 * stencil (16-bit dtype, head_dim 16/32/48/64, radius 1 or 2 on all axes, at least one
 * summary, an sm_100 device current), else 0.  No reference counterpart. */
P3D_API int p3d_stencil_fwd_supported(int dtype, int head_dim, int rz, int ry, int rx, int summaries);

/*
 * bound[b*G + g] = max over the summaries j of |sk[b, g, j, :]| (fp32 Euclidean norm, rounded
 * up by 2^-10), sk [B,G,M,D] bf16 / f16.  By Cauchy-Schwarz |q| * bound bounds every global
 * score of query row q (before the 1/sqrt(D) scale).  p3d_attn_fwd computes it itself; the
 * z-slab forward takes it through p3d_slab.summary_bound.  No reference counterpart (the
 * Triton kernels track a running maximum).
 */
P3D_API int p3d_summary_bound(const void *sk, int dtype, int batch, int kv_heads, int summaries, int head_dim,
                      float *bound, void *stream);

/*
 * z-slab extents of one rank when a volume is sharded across GPUs along z.  No counterpart
 * in the reference, which runs on one GPU.  op->q, op->gate, y, ol, og, lse_* describe this
 * rank's planes [center_z0, center_z0 + op->grid[0]); op->kl / op->vl hold the planes
 * [halo_z0, halo_z0 + halo_planes): this rank's own plus the neighbours' halo planes
 * (radius planes each side, clipped to the volume).
 */
typedef struct {
  int32_t global_planes; /* z extent of the whole volume */
  int32_t center_z0;     /* global z of this rank's first plane */
  int32_t halo_z0;       /* global z of the first plane of op->kl / op->vl */
  int32_t halo_planes;   /* planes in op->kl / op->vl */
  int32_t summaries;     /* rows of the gathered sk / sv: the summaries of all ranks */
  /* Optional [B*G] fp32 bound of p3d_summary_bound() on the gathered sk, or NULL.  With it
   * the global softmax takes its exponentials against the per-row score bound instead of a
   * running maximum (the faster form); p3d_attn_fwd_slab reads it, the backward does not. */
  const float *summary_bound;
  /* p3d_attn_fwd_slab only: run the 4-plane query tiles [tile_z_begin, tile_z_end) of this
   * rank's planes (tile_z_end 0: up to the last tile; 0, 0: all of them).  A caller overlapping the halo exchange runs the tiles
   * whose neighbourhood lies in its own planes first and the others once the halo planes of
   * op->kl / op->vl have arrived; op->kl / op->vl must hold every plane the tiles run read. */
  int32_t tile_z_begin, tile_z_end;
} p3d_slab;

/*
 * Forward of one z-slab on tensor cores (complete radius-2 stencil, raster storage,
 * 16-bit dtypes): local attention over op->kl / op->vl with halo planes, global attention
 * over the gathered summaries sk, sv [B,G,slab->summaries,D] (pooled per rank with
 * p3d_pool_fwd and all-gathered by the caller).  Writes y (and with P3D_FWD_SAVE_STATE ol,
 * og, lse_l, lse_g) for this rank's rows.  Needs no workspace.  No counterpart in the
 * reference (single-GPU only); the halo exchange and all-gather replace nothing there.
 */
P3D_API int p3d_attn_fwd_slab(const p3d_operator *op, const p3d_slab *slab, void *y, const void *sk, const void *sv,
                      void *ol, void *og, float *lse_l, float *lse_g, unsigned flags, void *stream);

/*
 * The backward in stages, for callers that interleave communication between them (the
 * z-slab sharding: mix -> halo exchange -> attention -> reduce-scatter of dsk, dsv ->
 * pooling).  p3d_attn_bwd runs the same kernels in one call.
 *
 * p3d_bwd_mix (kernels.py:107-127 _mix_bwd): dol = dy*sl, dog = dy*gate*sg [B,H,N,D] (dtype),
 *   delta_l/g = rowsum(dO*O) [B,H,N] fp32, dgate [B,H,N] (gate dtype), and dlocal_scale,
 *   dglobal_scale [D] fp32 summed over op's rows.
 * p3d_bwd_attn_slab (kernels.py:131-239 on one z-slab; no reference counterpart for the
 *   slab form): op->q, dol, dog, lse_*, delta_* are this rank's rows; op->kl / op->vl and
 *   q_halo, dol_halo, lse_l_halo, delta_l_halo hold the slab's halo planes (extents of
 *   p3d_slab, as for p3d_attn_fwd_slab); sk, sv the gathered summaries.  Writes dq, dkl,
 *   dvl for this rank's rows and dsk, dsv [B,G,slab->summaries,D] fp32: this rank's
 *   queries' contribution to every summary's gradient.
 * p3d_pool_bwd (kernels.py:243-272 _pool_bwd): the pooling VJP from fp32 dsk, dsv
 *   [B,G,M,D]: dk, dv [B,G,N,D] (dtype) and dweight [D], dbias [V] fp32.
 */
P3D_API int p3d_bwd_mix(const p3d_operator *op, const void *dy, const void *ol, const void *og, void *dol, void *dog,
                float *delta_l, float *delta_g, void *dgate, float *dlocal_scale, float *dglobal_scale,
                void *workspace, size_t workspace_bytes, void *stream);
P3D_API size_t p3d_bwd_mix_workspace(const p3d_operator *op);
P3D_API int p3d_bwd_attn_slab(const p3d_operator *op, const p3d_slab *slab, const void *sk, const void *sv,
                      const float *lse_l, const float *lse_g, const void *dol, const void *dog,
                      const float *delta_l, const float *delta_g, const void *q_halo, const void *dol_halo,
                      const float *lse_l_halo, const float *delta_l_halo, void *dq, void *dkl, void *dvl,
                      float *dsk, float *dsv, void *workspace, size_t workspace_bytes, void *stream);
P3D_API size_t p3d_bwd_attn_slab_workspace(const p3d_operator *op, const p3d_slab *slab);
P3D_API int p3d_pool_bwd(const void *k, const void *v, const float *weight, const float *bias, const int32_t *blocks,
                 int fine_blocks, int slots, int pool_size, const float *dsk, const float *dsv, void *dk, void *dv,
                 float *dweight, float *dbias, int dtype, int batch, int kv_heads, int tokens, int head_dim,
                 float temperature, void *workspace, size_t workspace_bytes, void *stream);
P3D_API size_t p3d_pool_bwd_workspace(int fine_blocks, int slots, int pool_size, int batch, int kv_heads,
                              int head_dim);

/*
 * Peer-memory exchange of the z-slab sharding (one process per GPU on one node).  No
 * counterpart in the reference, which runs on one GPU.  Each rank allocates one region
 * (p3d_peer_alloc: device memory, zeroed, with its 64-byte CUDA IPC handle) and maps the
 * other ranks' regions from their handles (p3d_peer_open: NVLink peer memory, valid on the
 * calling process's device).  Per layer call a rank waits for its peers' credits
 * (p3d_peer_wait), pushes its rows into the peers' regions (p3d_peer_push), waits for the
 * peers' pushes (p3d_peer_wait), runs its kernels on its own region and then raises every
 * peer's credit (p3d_peer_signal).  Counters are 64-bit, only grow, and live in the regions;
 * the expected values live in device memory and advance on the device, so a CUDA graph
 * captured over a call replays correctly.
 */
#define P3D_PEER_HANDLE_BYTES 64
#define P3D_PEER_MAX_COPIES 32
#define P3D_PEER_MAX_TARGETS 16
typedef struct {
  const void *src;   /* this process's memory */
  void *dst;         /* a peer's mapped region, or this process's memory */
  int64_t rows;      /* rows of row_bytes bytes (a multiple of 16) */
  int64_t row_bytes;
  int64_t src_stride, dst_stride;  /* bytes between rows (multiples of 16; 16-byte aligned pointers) */
} p3d_peer_copy;
P3D_API int p3d_peer_alloc(size_t bytes, void **ptr, void *handle);
P3D_API int p3d_peer_free(void *ptr);
P3D_API int p3d_peer_open(const void *handle, void **ptr);
P3D_API int p3d_peer_close(void *ptr);
/* copies[0, n_remote) are written first; then each of the ctas CTAs adds one to every
 * arrive[i] (release, system scope) after its part of them; then copies[n_remote,
 * n_copies) (rows that no peer waits for).  A consumer of the remote rows waits for
 * ctas arrivals per pusher. */
P3D_API int p3d_peer_push(const p3d_peer_copy *copies, int n_copies, int n_remote, uint64_t *const *arrive,
                  int n_arrive, int ctas, void *stream);
/* One device thread: wait until *counter >= *expected (acquire, system scope), for at most
 * timeout_s seconds, then *expected += step.  A wait that runs out sets bits 1 | 32 of
 * p3d_device_errors and returns. */
P3D_API int p3d_peer_wait(const uint64_t *counter, uint64_t *expected, uint64_t step, double timeout_s,
                  void *stream);
/* One device thread, after the stream's earlier work: add one to each counter (release,
 * system scope). */
P3D_API int p3d_peer_signal(uint64_t *const *counters, int n, void *stream);

/*
 * Forward (inference, no saved state) that allocates nothing and needs no workspace.
 * No counterpart in the reference.  For callers that cannot allocate device memory --
 * plugins inside a host framework that owns all device memory, or real-time loops that
 * must avoid the device synchronisation cudaMalloc / cudaFree can cause.  The caller
 * passes inputs (op) and outputs y [B,H,N,D], sk, sv [B,G,M,D] as for p3d_attn_fwd.
 * Runs the neighbour-table kernels; their one scratch buffer (the local-branch output,
 * B*H*N*D*sizeof(dtype) bytes, at most 16 MiB -- larger inputs return
 * P3D_ERR_UNSUPPORTED) lives in a fixed array inside the library that every GPU loading
 * the library keeps until process exit.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress), so make that first call before any stream
 * capture.  All calls share the array: calls whose kernels overlap on the GPU race.
 */
P3D_API int p3d_attn_fwd_noalloc(const p3d_operator *op, void *y, void *sk, void *sv, void *stream);

/*
 * Backward (kernels.py:314-356) from the saved forward state.  Writes dq
 * [B,H,N,D], dkl, dvl, dkg, dvg [B,G,N,D] (dtype), dgate [B,H,N] (gate_dtype)
 * and fp32 dweight [D], dbias [V], dlocal_scale [D], dglobal_scale [D].
 * Deterministic: no floating-point atomics, fixed reduction order.
 */
P3D_API int p3d_attn_bwd(const p3d_operator *op, const void *dy, const void *sk, const void *sv, const void *ol,
                 const void *og, const float *lse_l, const float *lse_g, void *dq, void *dkl, void *dvl,
                 void *dkg, void *dvg, void *dgate, float *dweight, float *dbias, float *dlocal_scale,
                 float *dglobal_scale, void *workspace, size_t workspace_bytes, void *stream);
P3D_API size_t p3d_attn_bwd_workspace(const p3d_operator *op);

#ifdef __cplusplus
}
#endif
#endif /* PACK3D_B200_H */
