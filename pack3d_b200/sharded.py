"""z-slab sharding of a PACK3D volume across GPUs (one process per GPU).

The reference runs on one GPU; this module spreads one volume over ``world`` ranks along
z.  Rank r owns planes ``[r*Z/world, (r+1)*Z/world)`` stored in raster order, so its
tokens are a contiguous range of the global raster order.  The plane count per rank is a
multiple of the summary block depth, so every summary (4x4x4 block) lies inside one rank.

Forward of the attention core on one rank (``sharded_core_forward``):

1. pool the rank's own blocks into summaries (``p3d_pool_fwd``);
2. all-gather the summaries of every rank (the global branch attends to all of them; its
   softmax and sum do not depend on their order, which is rank-major here);
3. exchange halo planes of the rotated local keys / values with the neighbouring ranks --
   ``radius`` planes each side, clipped to the volume -- through NCCL point-to-point
   send / receive;
4. run the fused tensor-core forward on the rank's planes with keys / values from its
   planes plus the halo (``p3d_attn_fwd_slab``).

Communication per layer and rank: 2 x radius planes of kl and vl each way, and the
summaries of all ranks (M x D per kv-head); both are small next to the compute.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native
from .geometry import TokenLayout, build_layout
from .ops import _as_gate, _device_tables, _f32, _operator


@dataclass(frozen=True)
class ZSlabs:
    """The z-partition of a ``(Z, Y, X)`` volume over ``world`` ranks, seen from ``rank``."""

    grid: tuple
    world: int
    rank: int
    radius: int = 2
    block_depth: int = 4

    def __post_init__(self):
        z = self.grid[0]
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError("rank must lie in [0, world)")
        if z % self.world or (z // self.world) % self.block_depth:
            raise ValueError(f"{z} planes do not split into {self.world} slabs of whole "
                             f"{self.block_depth}-plane summary blocks")

    @property
    def planes(self):
        return self.grid[0] // self.world

    @property
    def z0(self):
        return self.rank * self.planes

    @property
    def halo_lo(self):
        """Planes received from the rank below (0 at the bottom of the volume)."""
        return min(self.radius, self.z0)

    @property
    def halo_hi(self):
        """Planes received from the rank above (0 at the top of the volume)."""
        return min(self.radius, self.grid[0] - self.z0 - self.planes)

    @property
    def halo_z0(self):
        return self.z0 - self.halo_lo

    @property
    def halo_planes(self):
        return self.halo_lo + self.planes + self.halo_hi

    @property
    def plane_tokens(self):
        return self.grid[1] * self.grid[2]

    @property
    def tokens(self):
        return self.planes * self.plane_tokens

    def token_range(self):
        """This rank's rows of the global raster order."""
        return self.z0 * self.plane_tokens, (self.z0 + self.planes) * self.plane_tokens


@dataclass(frozen=True)
class SlabLayout:
    """One rank's planes of a raster-stored volume.

    ``local`` is the complete layout of the slab's own grid (its geometry -- neighbour
    table, blocks, stencil tag -- drives pooling and the kernels); ``coords`` are global
    ``(z, y, x)``, so RoPE turns every token by its position in the whole volume
    (``grid_shape``).
    """

    grid_shape: tuple
    slabs: ZSlabs
    local: TokenLayout
    coords: torch.Tensor

    @property
    def geometry(self):
        return self.local.geometry

    def to(self, device):
        return SlabLayout(self.grid_shape, self.slabs, self.local.to(device), self.coords.to(device))

    def check_unmodified(self):
        self.local.check_unmodified()


def slab_layout(grid, block_shape=(4, 4, 4), *, radius=2, pool_size=1, slabs: ZSlabs):
    """Raster-stored layout of this rank's planes of ``grid``."""
    if tuple(grid) != tuple(slabs.grid) or block_shape[0] != slabs.block_depth or radius != slabs.radius:
        raise ValueError("the slab partition must match the grid, block depth and radius")
    local = build_layout((slabs.planes, grid[1], grid[2]), block_shape, radius=radius, pool_size=pool_size)
    local = local.repack(local.order.argsort())
    coords = local.coords.clone()
    coords[:, 0] += slabs.z0
    return SlabLayout(tuple(grid), slabs, local, coords)


def exchange_halos(t, slabs: ZSlabs, group=None):
    """``t`` [B, G, planes*Y*X, D] (this rank's planes, raster) -> [B, G, halo_planes*Y*X, D].

    Sends this rank's first ``radius`` planes down and its last ``radius`` planes up, and
    receives the neighbours' in one batch of point-to-point operations.
    """
    b, g, n, d = t.shape
    if n != slabs.tokens:
        raise ValueError("tensor rows do not match the slab")
    pt = slabs.plane_tokens
    rank_of = (lambda r: r) if group is None else (lambda r: dist.get_global_rank(group, r))
    ops, recv_lo, recv_hi = [], None, None
    if slabs.halo_lo:
        lo = slabs.halo_lo * pt
        recv_lo = torch.empty((b, g, lo, d), dtype=t.dtype, device=t.device)
        ops.append(dist.P2POp(dist.isend, t[:, :, :lo].contiguous(), rank_of(slabs.rank - 1), group))
        ops.append(dist.P2POp(dist.irecv, recv_lo, rank_of(slabs.rank - 1), group))
    if slabs.halo_hi:
        hi = slabs.halo_hi * pt
        recv_hi = torch.empty((b, g, hi, d), dtype=t.dtype, device=t.device)
        ops.append(dist.P2POp(dist.isend, t[:, :, n - hi:].contiguous(), rank_of(slabs.rank + 1), group))
        ops.append(dist.P2POp(dist.irecv, recv_hi, rank_of(slabs.rank + 1), group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    parts = [p for p in (recv_lo, t, recv_hi) if p is not None]
    return torch.cat(parts, dim=2) if len(parts) > 1 else t.contiguous()


def gather_summaries(s, group=None):
    """``s`` [B, G, M_rank, D] -> [B, G, world*M_rank, D], rank-major."""
    world = dist.get_world_size(group)
    if world == 1:
        return s.contiguous()
    parts = [torch.empty_like(s) for _ in range(world)]
    dist.all_gather(parts, s.contiguous(), group=group)
    return torch.cat(parts, dim=2)


def pool_summaries(kg, vg, weight, bias, geometry, temperature=1.0):
    """This rank's summaries: pooling of its own blocks (``p3d_pool_fwd``)."""
    b, g, n, d = kg.shape
    tables = _device_tables(geometry, kg.device)
    m = geometry.num_summaries
    sk = torch.empty((b, g, m, d), dtype=kg.dtype, device=kg.device)
    sv = torch.empty_like(sk)
    w32, b32 = _f32(weight), _f32(bias)
    fine, slots = geometry.blocks.shape
    with torch.cuda.device(kg.device):
        status = _native.lib().p3d_pool_fwd(
            _native.ptr(kg), _native.ptr(vg), _native.ptr(w32), _native.ptr(b32), _native.ptr(tables["blocks"]),
            fine, slots, geometry.pool_size, _native.ptr(sk), _native.ptr(sv), None, None,
            _native.DTYPE_CODE[kg.dtype], b, g, n, d, float(temperature), _native.stream_of(kg.device))
    _native.check(status, "p3d_pool_fwd")
    return sk, sv


def slab_forward(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, geometry, slabs: ZSlabs, temperature=1.0,
                 save_state=False):
    """``p3d_attn_fwd_slab`` on one rank: returns ``(y, state)``.

    ``kl_ext`` / ``vl_ext`` hold the rank's planes plus its halo planes; ``sk`` / ``sv`` the
    gathered summaries of all ranks.
    """
    b, h, n, d = q.shape
    if n != slabs.tokens or kl_ext.shape[2] != slabs.halo_planes * slabs.plane_tokens:
        raise ValueError("q / kl rows do not match the slab")
    gate = _as_gate(gate, q).contiguous()
    w32, b32, sl32, sg32 = (_f32(t) for t in (weight, bias, sl, sg))
    op, keep = _operator(q, kl_ext, vl_ext, kl_ext, vl_ext, w32, b32, gate, sl32, sg32, geometry, temperature)
    if geometry.stencil is None or op.raster_to_packed:
        raise ValueError("slab forward needs the complete stencil of a raster-stored slab")
    slab = _native.Slab(slabs.grid[0], slabs.z0, slabs.halo_z0, slabs.halo_planes, sk.shape[2])
    y = torch.empty_like(q)
    ol = og = lse_l = lse_g = None
    flags = 0
    if save_state:
        ol, og = torch.empty_like(q), torch.empty_like(q)
        lse_l = torch.empty((b, h, n), dtype=torch.float32, device=q.device)
        lse_g = torch.empty_like(lse_l)
        flags = _native.FWD_SAVE_STATE
    with torch.cuda.device(q.device):
        status = _native.lib().p3d_attn_fwd_slab(op, ctypes.byref(slab), _native.ptr(y), _native.ptr(sk),
                                                 _native.ptr(sv), _native.ptr(ol), _native.ptr(og),
                                                 _native.ptr(lse_l), _native.ptr(lse_g), flags,
                                                 _native.stream_of(q.device))
    _native.check(status, "p3d_attn_fwd_slab")
    del keep
    return y, ((sk, sv, ol, og, lse_l, lse_g) if save_state else ())


def sharded_core_forward(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, slabs: ZSlabs, group=None,
                         temperature=1.0):
    """The attention core of one rank's planes (inference): pool, gather, exchange, attend."""
    sk_rank, sv_rank = pool_summaries(kg, vg, weight, bias, geometry, temperature)
    sk, sv = gather_summaries(sk_rank, group), gather_summaries(sv_rank, group)
    kl_ext, vl_ext = exchange_halos(kl, slabs, group), exchange_halos(vl, slabs, group)
    y, _ = slab_forward(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, geometry, slabs, temperature)
    return y


def sharded_layer_forward(layer, x, layout: SlabLayout, group=None):
    """``PACK3DAttention.forward`` (reference attention.py:53-89) on one rank's planes.

    ``x`` [B, rank tokens, dim] holds this rank's tokens in raster order.  LayerNorm,
    projections, gate and output projection are per token and run locally; RoPE uses the
    global coordinates; the attention core runs sharded (``sharded_core_forward``).
    Inference only: the sharded backward is not provided.
    """
    from .rope import balanced_pairs, rotate_projections
    if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in layer.parameters())):
        raise NotImplementedError("the sharded layer runs inference only; wrap the call in torch.no_grad()")
    layout.check_unmodified()
    if layer.position_encoding != "axial":
        raise ValueError("the sharded layer supports axial position encoding only")
    b, n = x.shape[0], x.shape[1]
    if n != layout.slabs.tokens or x.shape[2] != layer.dim:
        raise ValueError("x must be [batch, rank tokens, dim]")
    h, g, d = layer.heads, layer.kv_heads, layer.head_dim
    xn = layer.norm(x)
    q = layer.to_q(xn).reshape(b, n, h, d).transpose(1, 2)
    kl, vl, kg, vg = (t.reshape(b, n, g, d).transpose(1, 2) for t in layer.to_kv(xn).chunk(4, -1))
    q, kl, kg = rotate_projections(q, kl, kg, layout.coords, balanced_pairs(d), layout.grid_shape, packed=False)
    gate = layer.gate(xn).reshape(b, n, h, 2).softmax(-1)[..., 1].transpose(1, 2).contiguous()
    y = sharded_core_forward(q, kl, vl.contiguous(), kg, vg.contiguous(), layer.pool_weight, layer.slot_bias, gate,
                             layer.local_scale, layer.global_scale, layout.geometry, layout.slabs, group,
                             layer.temperature)
    return x + layer.to_out(y.transpose(1, 2).reshape(b, n, -1))
