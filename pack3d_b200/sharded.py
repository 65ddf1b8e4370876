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
    """Raster-stored layout of this rank's planes of ``grid``.

    Only ``pool_size=1`` is accepted: each summary is then one fine block, a cube that lies
    inside one rank, so the ranks' summaries are exactly the whole volume's.  With coarser
    pooling a rank would group consecutive fine blocks of its own Morton block order, which
    differs from the whole volume's, and summaries would pool the wrong blocks.
    """
    if tuple(grid) != tuple(slabs.grid) or block_shape[0] != slabs.block_depth or radius != slabs.radius:
        raise ValueError("the slab partition must match the grid, block depth and radius")
    if pool_size != 1:
        raise ValueError("z-slab sharding supports pool_size=1 only (each summary one fine block)")
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


def exchange_slab(kl, vl, sk_rank, sv_rank, slabs: ZSlabs, group=None):
    """The forward's whole exchange as one batch of point-to-point operations: the halo
    planes of ``kl`` and ``vl`` with both neighbours and this rank's summaries with every
    rank (an all-gather written as sends and receives, so that it shares the batch).

    Returns ``(kl_ext, vl_ext, sk, sv)`` as :func:`exchange_halos` and
    :func:`gather_summaries` would.
    """
    world = dist.get_world_size(group)
    b, g, n, d = kl.shape
    if n != slabs.tokens or vl.shape != kl.shape:
        raise ValueError("tensor rows do not match the slab")
    pt = slabs.plane_tokens
    rank_of = (lambda r: r) if group is None else (lambda r: dist.get_global_rank(group, r))
    ops = []
    halos = {}
    for name, t in (("k", kl), ("v", vl)):
        if slabs.halo_lo:
            lo = slabs.halo_lo * pt
            halos[name, "lo"] = torch.empty((b, g, lo, d), dtype=t.dtype, device=t.device)
            ops.append(dist.P2POp(dist.isend, t[:, :, :lo].contiguous(), rank_of(slabs.rank - 1), group))
            ops.append(dist.P2POp(dist.irecv, halos[name, "lo"], rank_of(slabs.rank - 1), group))
        if slabs.halo_hi:
            hi = slabs.halo_hi * pt
            halos[name, "hi"] = torch.empty((b, g, hi, d), dtype=t.dtype, device=t.device)
            ops.append(dist.P2POp(dist.isend, t[:, :, n - hi:].contiguous(), rank_of(slabs.rank + 1), group))
            ops.append(dist.P2POp(dist.irecv, halos[name, "hi"], rank_of(slabs.rank + 1), group))
    sk_rank, sv_rank = sk_rank.contiguous(), sv_rank.contiguous()
    parts = {name: [None] * world for name in ("k", "v")}
    for name, s in (("k", sk_rank), ("v", sv_rank)):
        for r in range(world):
            if r == slabs.rank:
                parts[name][r] = s
                continue
            parts[name][r] = torch.empty_like(s)
            ops.append(dist.P2POp(dist.isend, s, rank_of(r), group))
            ops.append(dist.P2POp(dist.irecv, parts[name][r], rank_of(r), group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    ext = []
    for name, t in (("k", kl), ("v", vl)):
        pieces = [p for p in (halos.get((name, "lo")), t, halos.get((name, "hi"))) if p is not None]
        ext.append(torch.cat(pieces, dim=2) if len(pieces) > 1 else t.contiguous())
    return ext[0], ext[1], torch.cat(parts["k"], dim=2), torch.cat(parts["v"], dim=2)


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


def _summary_bound(sk, device):
    """Per-(batch, kv-head) bound of the gathered summaries' norms (``p3d_summary_bound``): the
    forward's fixed-reference global softmax takes its exponentials against a score bound per
    query row instead of a running maximum."""
    b, g, m, d = sk.shape
    bound = torch.empty(b * g, dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        _native.check(_native.lib().p3d_summary_bound(_native.ptr(sk), _native.DTYPE_CODE[sk.dtype], b, g, m, d,
                                                      _native.ptr(bound), _native.stream_of(device)),
                      "p3d_summary_bound")
    return bound


TILE_PLANES = 4   # planes of one query tile of p3d_attn_fwd_slab (4 x 4 x 8 = 128 rows)


def interior_tiles(slabs: ZSlabs):
    """The query tiles of this rank whose keys and values lie in its own planes or outside
    the volume -- none in a halo plane: ``(begin, end)``, empty when ``begin >= end``.  Tile t
    covers planes ``[4t, 4t + 4)`` of the rank and reads ``radius`` planes more on each side."""
    tiles = -(-slabs.planes // TILE_PLANES)
    reach = -(-slabs.radius // TILE_PLANES)
    return (reach if slabs.halo_lo else 0), tiles - (reach if slabs.halo_hi else 0)


class _SlabCall:
    """One rank's ``p3d_attn_fwd_slab`` set up once and launched over ranges of its 4-plane
    query tiles (the pointers of ``kl_ext`` / ``vl_ext`` are fixed here; a range may run only
    once every plane its tiles read has been written)."""

    def __init__(self, q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, geometry, slabs, temperature,
                 save_state, y_rows):
        b, h, n, d = q.shape
        if n != slabs.tokens or kl_ext.shape[2] != slabs.halo_planes * slabs.plane_tokens:
            raise ValueError("q / kl rows do not match the slab")
        self.device = q.device
        self.gate = _as_gate(gate, q).contiguous()
        self.f32 = tuple(_f32(t) for t in (weight, bias, sl, sg))
        self.op, self.keep = _operator(q, kl_ext, vl_ext, kl_ext, vl_ext, *self.f32[:2], self.gate, *self.f32[2:],
                                       geometry, temperature)
        if geometry.stencil is None or self.op.raster_to_packed:
            raise ValueError("slab forward needs the complete stencil of a raster-stored slab")
        self.sk, self.sv = sk, sv
        self.bound = _summary_bound(sk, q.device)
        self.slabs = slabs
        self.tiles_z = -(-slabs.planes // TILE_PLANES)
        if y_rows:
            self.y = torch.empty((b, n, h, d), dtype=q.dtype, device=q.device).transpose(1, 2)
        else:
            self.y = torch.empty_like(q)
        self.state = (None,) * 4
        self.flags = _native.FWD_Y_ROWS if y_rows else 0
        if save_state:
            ol, og = torch.empty_like(q), torch.empty_like(q)
            lse_l = torch.empty((b, h, n), dtype=torch.float32, device=q.device)
            self.state = (ol, og, lse_l, torch.empty_like(lse_l))
            self.flags |= _native.FWD_SAVE_STATE

    def run(self, tile_z_begin=0, tile_z_end=0):
        """Launch the query tiles ``[tile_z_begin, tile_z_end)`` (0, 0: all of them)."""
        slabs = self.slabs
        slab = _native.Slab(slabs.grid[0], slabs.z0, slabs.halo_z0, slabs.halo_planes, self.sk.shape[2],
                            ctypes.c_void_p(self.bound.data_ptr()), tile_z_begin, tile_z_end)
        with torch.cuda.device(self.device):
            status = _native.lib().p3d_attn_fwd_slab(self.op, ctypes.byref(slab), _native.ptr(self.y),
                                                     _native.ptr(self.sk), _native.ptr(self.sv),
                                                     *[_native.ptr(t) for t in self.state], self.flags,
                                                     _native.stream_of(self.device))
        _native.check(status, "p3d_attn_fwd_slab")

    def result(self):
        ol, og, lse_l, lse_g = self.state
        return self.y, ((self.sk, self.sv, ol, og, lse_l, lse_g) if self.flags & _native.FWD_SAVE_STATE else ())


def slab_forward(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, geometry, slabs: ZSlabs, temperature=1.0,
                 save_state=False, y_rows=False):
    """``p3d_attn_fwd_slab`` on one rank: returns ``(y, state)``.

    ``kl_ext`` / ``vl_ext`` hold the rank's planes plus its halo planes; ``sk`` / ``sv`` the
    gathered summaries of all ranks.  With ``y_rows`` y is stored token-major ([B, N, H, D];
    the returned [B, H, N, D] tensor is a view of it).
    """
    call = _SlabCall(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, geometry, slabs, temperature,
                     save_state, y_rows)
    call.run()
    return call.result()


class _DeviceBytes:
    """A raw device allocation seen by ``torch.as_tensor`` (CUDA array interface)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 2,
                                         "strides": None}


class SlabPeers:
    """The peer-memory exchange of one z-slab partition (``p3d_peer_*``): every rank's region
    of device memory, mapped into every other rank's process over NVLink.

    A rank's region holds what its slab kernel reads -- its keys / values with the halo
    planes around them ([B, G, halo_planes * Y * X, D] each) and the summaries of every rank
    ([B, G, world * M, D] each, rank-major) -- and two counters.  :meth:`exchange` waits for
    the peers' credits, pushes this rank's summaries to every peer and its boundary planes
    to its neighbours (one kernel, 16-byte stores over NVLink), copies its own rows into its
    region and waits for the peers' pushes; :meth:`release` raises every peer's credit once
    this rank's kernels have read the region.  Building one is collective (the ranks trade
    IPC handles through the process group) and must happen outside stream capture; the calls
    after it capture into CUDA graphs.  :meth:`close` (collective) unmaps and frees.
    """

    ARRIVALS, CREDITS, HEADER = 0, 128, 4096

    def __init__(self, slabs: ZSlabs, batch, kv_heads, head_dim, summaries, dtype, device, group=None, ctas=None,
                 timeout_s=10.0):
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("SlabPeers is set up outside stream capture (its first call runs eagerly)")
        self.world = dist.get_world_size(group)
        if dist.get_rank(group) != slabs.rank:
            raise ValueError("the slab partition's rank is not this process's rank in the group")
        if slabs.planes < slabs.radius:
            raise ValueError("a rank's planes must cover the halo depth")
        self.slabs, self.group, self.device, self.dtype = slabs, group, torch.device(device), dtype
        self.shape = (batch, kv_heads, head_dim, summaries)
        self.timeout_s = float(timeout_s)
        props = torch.cuda.get_device_properties(self.device)
        self.ctas = int(ctas or 2 * props.multi_processor_count)
        es = torch.empty((), dtype=dtype).element_size()
        pt = slabs.plane_tokens
        self.row_bytes = head_dim * es
        rows_max = (slabs.planes + 2 * slabs.radius) * pt
        align = lambda v: -(-v // 4096) * 4096  # noqa: E731
        self.ext_bytes = align(batch * kv_heads * rows_max * self.row_bytes)
        self.summ_bytes = align(batch * kv_heads * self.world * summaries * self.row_bytes)
        self.offsets = {"k": self.HEADER, "v": self.HEADER + self.ext_bytes,
                        "sk": self.HEADER + 2 * self.ext_bytes, "sv": self.HEADER + 2 * self.ext_bytes + self.summ_bytes}
        self.nbytes = self.HEADER + 2 * self.ext_bytes + 2 * self.summ_bytes
        lib = _native.lib()
        handle = ctypes.create_string_buffer(_native.PEER_HANDLE_BYTES)
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _native.check(lib.p3d_peer_alloc(self.nbytes, ctypes.byref(own), handle), "p3d_peer_alloc")
        self.own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.bases = [None] * self.world
        self.opened = []
        for r in range(self.world):
            if r == slabs.rank:
                self.bases[r] = self.own
                continue
            ptr = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                _native.check(lib.p3d_peer_open(ctypes.create_string_buffer(handles[r], len(handles[r])),
                                                ctypes.byref(ptr)), "p3d_peer_open")
            self.bases[r] = ptr.value
            self.opened.append(ptr.value)
        region = torch.as_tensor(_DeviceBytes(self.own, self.nbytes), device=self.device)
        self.region = region
        b, g, d, m = self.shape
        rows = slabs.halo_planes * pt
        view = lambda key, n_rows: region[self.offsets[key]:self.offsets[key] + b * g * n_rows * self.row_bytes].view(  # noqa: E731
            dtype).view(b, g, n_rows, d)
        self.kl_ext, self.vl_ext = view("k", rows), view("v", rows)
        self.sk, self.sv = view("sk", self.world * m), view("sv", self.world * m)
        # expected arrivals (every peer pushes with `ctas` CTAs) and credits (one per peer)
        self.expected = torch.tensor([(self.world - 1) * self.ctas, 0], dtype=torch.int64, device=self.device)
        peers = [r for r in range(self.world) if r != slabs.rank]
        self._arrive = (ctypes.c_void_p * max(1, len(peers)))(*[self.bases[r] + self.ARRIVALS for r in peers])
        self._credit = (ctypes.c_void_p * max(1, len(peers)))(*[self.bases[r] + self.CREDITS for r in peers])
        self.peers = peers

    def _ext_rows(self, rank):
        s = ZSlabs(self.slabs.grid, self.world, rank, self.slabs.radius, self.slabs.block_depth)
        return s, s.halo_planes * s.plane_tokens

    def _copies(self, kl, vl, sk_rank, sv_rank):
        """(remote copies, local copies) of one call, as ``p3d_peer_copy`` records.  Every input
        is [B, G, rows, D] with contiguous rows per head (:func:`_head_stride`); kl / vl already
        in place between this rank's halo rows (``p3d_qkv_project`` with ``kv_out``) are not
        copied again."""
        s, rb = self.slabs, self.row_bytes
        b, g, d, m = self.shape
        pt, n = s.plane_tokens, s.tokens
        remote, local = [], []

        def rec(src, src_off, dst, rows_each, dst_rows):
            return (src.data_ptr() + src_off * rb, dst, b * g, rows_each * rb, _head_stride(src), dst_rows * rb)

        for key, t in (("sk", sk_rank), ("sv", sv_rank)):
            for r in range(self.world):
                dst = self.bases[r] + self.offsets[key] + s.rank * m * rb
                (local if r == s.rank else remote).append(rec(t, 0, dst, m, self.world * m))
        own_rows = s.halo_planes * pt
        for key, t in (("k", kl), ("v", vl)):
            if s.halo_lo:   # my first planes are the lower neighbour's upper halo
                nb, rows = self._ext_rows(s.rank - 1)
                dst = self.bases[s.rank - 1] + self.offsets[key] + (nb.halo_lo + nb.planes) * pt * rb
                remote.append(rec(t, 0, dst, nb.halo_hi * pt, rows))
            if s.halo_hi:   # my last planes are the upper neighbour's lower halo
                nb, rows = self._ext_rows(s.rank + 1)
                dst = self.bases[s.rank + 1] + self.offsets[key]
                remote.append(rec(t, n - nb.halo_lo * pt, dst, nb.halo_lo * pt, rows))
            dst = self.own + self.offsets[key] + s.halo_lo * pt * rb
            if t.data_ptr() != dst or _head_stride(t) != own_rows * rb:
                local.append(rec(t, 0, dst, n, own_rows))
        return remote, local

    def kv_out(self):
        """``(kl_ext, vl_ext, row0)``: where ``p3d_qkv_project`` writes this rank's kl / vl so
        that :meth:`exchange` copies nothing locally."""
        return self.kl_ext, self.vl_ext, self.slabs.halo_lo * self.slabs.plane_tokens

    def exchange(self, kl, vl, sk_rank, sv_rank):
        """``(kl_ext, vl_ext, sk, sv)`` as :func:`exchange_slab` returns them, as views of this
        rank's region (valid until :meth:`release`)."""
        b, g, d, m = self.shape
        want = (b, g, self.slabs.tokens, d)
        if tuple(kl.shape) != want or tuple(vl.shape) != want or tuple(sk_rank.shape) != (b, g, m, d) or \
                tuple(sv_rank.shape) != (b, g, m, d) or any(t.dtype != self.dtype for t in (kl, vl, sk_rank, sv_rank)):
            raise ValueError("exchange inputs do not match the peer regions")
        kl, vl, sk_rank, sv_rank = (t if _head_stride(t) else t.contiguous() for t in (kl, vl, sk_rank, sv_rank))
        remote, local = self._copies(kl, vl, sk_rank, sv_rank)
        copies = (_native.PeerCopy * len(remote + local))(*[_native.PeerCopy(*c) for c in remote + local])
        lib, stream = _native.lib(), _native.stream_of(self.device)
        exp = self.expected.data_ptr()
        with torch.cuda.device(self.device):
            if self.peers:
                _native.check(lib.p3d_peer_wait(self.own + self.CREDITS, exp + 8, len(self.peers), self.timeout_s,
                                                stream), "p3d_peer_wait")
            _native.check(lib.p3d_peer_push(copies, len(copies), len(remote), self._arrive, len(self.peers),
                                            self.ctas, stream), "p3d_peer_push")
            if self.peers:
                _native.check(lib.p3d_peer_wait(self.own + self.ARRIVALS, exp, len(self.peers) * self.ctas,
                                                self.timeout_s, stream), "p3d_peer_wait")
        return self.kl_ext, self.vl_ext, self.sk, self.sv

    def release(self):
        """Raise every peer's credit: this rank's kernels that read its region are enqueued."""
        if self.peers:
            with torch.cuda.device(self.device):
                _native.check(_native.lib().p3d_peer_signal(self._credit, len(self.peers),
                                                            _native.stream_of(self.device)), "p3d_peer_signal")

    def close(self):
        """Collective: wait for every rank's work, then unmap the peers' regions and free this one."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _native.lib()
        with torch.cuda.device(self.device):
            for ptr in self.opened:
                _native.check(lib.p3d_peer_close(ptr), "p3d_peer_close")
            self.opened = []
            self.region = self.kl_ext = self.vl_ext = self.sk = self.sv = None
            if self.own:
                _native.check(lib.p3d_peer_free(self.own), "p3d_peer_free")
                self.own = None
        dist.barrier(group=self.group)


def _head_stride(t):
    """Bytes between the heads of a [B, G, rows, D] tensor whose rows are contiguous within a
    head and whose heads are evenly spaced across the batch; None for other layouts."""
    b, g, n, d = t.shape
    if t.stride(3) != 1 or (n > 1 and t.stride(2) != d) or (b > 1 and t.stride(0) != g * t.stride(1)):
        return None
    return t.stride(1) * t.element_size()


_PEERS = {}


def slab_peers(slabs: ZSlabs, batch, kv_heads, head_dim, summaries, dtype, device, group=None):
    """The cached :class:`SlabPeers` for this partition, shapes and group (built on first use)."""
    key = (slabs, batch, kv_heads, head_dim, summaries, dtype, torch.device(device), id(group))
    if key not in _PEERS:
        _PEERS[key] = SlabPeers(slabs, batch, kv_heads, head_dim, summaries, dtype, device, group)
    return _PEERS[key]


def release_peers():
    """Collective: close every cached :class:`SlabPeers` (before the process group is destroyed)."""
    for key in list(_PEERS):
        _PEERS.pop(key).close()


def peer_exchange_supported(head_dim, dtype, device, group=None):
    """More than one rank, and rows the peer exchange can move (16-byte words: a row of
    head_dim elements must be a multiple of 16 bytes)."""
    es = torch.empty((), dtype=dtype).element_size()
    return torch.device(device).type == "cuda" and dist.get_world_size(group) > 1 and (head_dim * es) % 16 == 0


def sharded_core_forward(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, slabs: ZSlabs, group=None,
                         temperature=1.0):
    """The attention core of one rank's planes (inference): pool, exchange (:func:`peer_forward`)
    and attend."""
    sk_rank, sv_rank = pool_summaries(kg, vg, weight, bias, geometry, temperature)
    return peer_forward(q, kl, vl, sk_rank, sv_rank, weight, bias, gate, sl, sg, geometry, slabs, group, temperature)


def peer_forward(q, kl, vl, sk_rank, sv_rank, weight, bias, gate, sl, sg, geometry, slabs: ZSlabs, group=None,
                 temperature=1.0, y_rows=False):
    """Exchange and attend on one rank: the halo planes and summaries through the peer
    regions (:class:`SlabPeers`) when the rows allow it and more than one rank runs, else one
    NCCL point-to-point batch (:func:`exchange_slab`); then ``p3d_attn_fwd_slab``.  Returns y."""
    if peer_exchange_supported(kl.shape[3], kl.dtype, kl.device, group):
        b, g, _, d = kl.shape
        peers = slab_peers(slabs, b, g, d, sk_rank.shape[2], kl.dtype, kl.device, group)
        kl_ext, vl_ext, sk, sv = peers.exchange(kl, vl, sk_rank, sv_rank)
        y, _ = slab_forward(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, geometry, slabs, temperature,
                            y_rows=y_rows)
        peers.release()
        return y
    kl_ext, vl_ext, sk, sv = exchange_slab(kl, vl, sk_rank, sv_rank, slabs, group)
    y, _ = slab_forward(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, geometry, slabs, temperature,
                        y_rows=y_rows)
    return y


def sharded_layer_forward(layer, x, layout: SlabLayout, group=None):
    """``PACK3DAttention.forward`` (reference attention.py:53-89) on one rank's planes.

    ``x`` [B, rank tokens, dim] holds this rank's tokens in raster order.  LayerNorm,
    projections, gate and output projection are per token and run locally; RoPE uses the
    global coordinates; the attention core runs sharded (``sharded_core_forward``).
    Differentiable: the core's backward is sharded (``sharded_core_backward``); parameter
    gradients are this rank's share, to be summed over ranks like any replicated layer's.
    """
    from .rope import balanced_pairs, rotate_projections
    layout.check_unmodified()
    if layer.position_encoding != "axial":
        raise ValueError("the sharded layer supports axial position encoding only")
    b, n = x.shape[0], x.shape[1]
    if n != layout.slabs.tokens or x.shape[2] != layer.dim:
        raise ValueError("x must be [batch, rank tokens, dim]")
    h, g, d = layer.heads, layer.kv_heads, layer.head_dim
    if layer._fast_inference(x):
        # the fused glue of the single-GPU inference path writing kl, vl into this rank's peer
        # region, the peer exchange, token-major y
        kv_out = None
        if peer_exchange_supported(d, x.dtype, x.device, group):
            kv_out = slab_peers(layout.slabs, b, g, d, layout.geometry.num_summaries, x.dtype, x.device,
                                group).kv_out()
        x, q, kl, vl, kg, vg, gate = layer._inference_glue(x, layout.coords, layout.grid_shape, kv_out=kv_out)
        sk_rank, sv_rank = pool_summaries(kg, vg, layer.pool_weight, layer.slot_bias, layout.geometry,
                                          layer.temperature)
        y = peer_forward(q, kl, vl, sk_rank, sv_rank, layer.pool_weight, layer.slot_bias, gate, layer.local_scale,
                         layer.global_scale, layout.geometry, layout.slabs, group, layer.temperature, y_rows=True)
        return layer._out_residual(x, y)
    xn = layer.norm(x)
    q = layer.to_q(xn).reshape(b, n, h, d).transpose(1, 2)
    kl, vl, kg, vg = (t.reshape(b, n, g, d).transpose(1, 2) for t in layer.to_kv(xn).chunk(4, -1))
    q, kl, kg = rotate_projections(q, kl, kg, layout.coords, balanced_pairs(d), layout.grid_shape, packed=False)
    gate = layer.gate(xn).reshape(b, n, h, 2).softmax(-1)[..., 1].transpose(1, 2).contiguous()
    args = (q, kl, vl.contiguous(), kg, vg.contiguous(), layer.pool_weight, layer.slot_bias, gate, layer.local_scale,
            layer.global_scale, layout.geometry, layout.slabs, group, layer.temperature)
    if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in layer.parameters())):
        y = sharded_core(*args)
    else:
        y = sharded_core_forward(*args)
    return x + layer.to_out(y.transpose(1, 2).reshape(b, n, -1))


# ----------------------------------------------------------------------------- backward
#
# Backward of the attention core on one rank (``sharded_core_backward``):
#
# 1. mix backward of the rank's rows (``p3d_bwd_mix``): dO_l, dO_g, Delta_l, Delta_g, the
#    gate gradient and the rank's share of the branch-scale gradients;
# 2. exchange halo planes of q, dO_l, lse_l and Delta_l: the local dK / dV of a key is
#    computed by the key's owner from every query that attends to it, including the
#    neighbours' (no dK / dV is sent back);
# 3. dQ, local dK / dV and the rank's contribution to every summary gradient
#    (``p3d_bwd_attn_slab``);
# 4. reduce-scatter the summary gradients to the ranks that own the summaries;
# 5. pooling backward of the rank's own summaries (``p3d_pool_bwd``).
#
# Parameter gradients (pooling weight and bias, branch scales) are this rank's
# contributions, as for any layer whose parameters are replicated: the caller sums them
# over ranks with its other parameter gradients.

def _workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def slab_mix_backward(dy, q, kl, vl, kg, vg, weight, bias, gate, sl, sg, ol, og, geometry, temperature=1.0):
    """Stage 1 on one rank: ``(dol, dog, delta_l, delta_g, dgate, dsl, dsg)``."""
    b, h, n, d = q.shape
    gate_k = _as_gate(gate, q).contiguous()
    w32, b32, sl32, sg32 = (_f32(t) for t in (weight, bias, sl, sg))
    op, keep = _operator(q, kl, vl, kg, vg, w32, b32, gate_k, sl32, sg32, geometry, temperature)
    dol, dog = torch.empty_like(q), torch.empty_like(q)
    f32 = dict(dtype=torch.float32, device=q.device)
    delta_l, delta_g = torch.empty((b, h, n), **f32), torch.empty((b, h, n), **f32)
    dgate = torch.empty_like(gate_k)
    dsl, dsg = torch.empty(d, **f32), torch.empty(d, **f32)
    lib = _native.lib()
    ws = _workspace(lib.p3d_bwd_mix_workspace(op), q.device)
    with torch.cuda.device(q.device):
        status = lib.p3d_bwd_mix(op, _native.ptr(dy), _native.ptr(ol), _native.ptr(og), _native.ptr(dol),
                                 _native.ptr(dog), _native.ptr(delta_l), _native.ptr(delta_g), _native.ptr(dgate),
                                 _native.ptr(dsl), _native.ptr(dsg), _native.ptr(ws), ws.numel(),
                                 _native.stream_of(q.device))
    _native.check(status, "p3d_bwd_mix")
    del keep
    return dol, dog, delta_l, delta_g, dgate, dsl, dsg


def slab_attention_backward(q, kl_ext, vl_ext, sk, sv, lse_l, lse_g, dol, dog, delta_l, delta_g, q_ext, dol_ext,
                            lse_l_ext, delta_l_ext, weight, bias, gate, sl, sg, geometry, slabs: ZSlabs,
                            temperature=1.0):
    """Stage 3 on one rank: ``(dq, dkl, dvl, dsk, dsv)``; dsk, dsv [B, G, M_all, D] fp32."""
    b, h, n, d = q.shape
    g = kl_ext.shape[1]
    gate_k = _as_gate(gate, q).contiguous()
    w32, b32, sl32, sg32 = (_f32(t) for t in (weight, bias, sl, sg))
    op, keep = _operator(q, kl_ext, vl_ext, kl_ext, vl_ext, w32, b32, gate_k, sl32, sg32, geometry, temperature)
    slab = _native.Slab(slabs.grid[0], slabs.z0, slabs.halo_z0, slabs.halo_planes, sk.shape[2])
    dq = torch.empty_like(q)
    dkl = torch.empty((b, g, n, d), dtype=q.dtype, device=q.device)
    dvl = torch.empty_like(dkl)
    dsk = torch.empty((b, g, sk.shape[2], d), dtype=torch.float32, device=q.device)
    dsv = torch.empty_like(dsk)
    lib = _native.lib()
    ws = _workspace(lib.p3d_bwd_attn_slab_workspace(op, ctypes.byref(slab)), q.device)
    args = [sk, sv, lse_l, lse_g, dol, dog, delta_l, delta_g, q_ext, dol_ext, lse_l_ext, delta_l_ext, dq, dkl, dvl,
            dsk, dsv]
    with torch.cuda.device(q.device):
        status = lib.p3d_bwd_attn_slab(op, ctypes.byref(slab), *[_native.ptr(t) for t in args], _native.ptr(ws),
                                       ws.numel(), _native.stream_of(q.device))
    _native.check(status, "p3d_bwd_attn_slab")
    del keep
    return dq, dkl, dvl, dsk, dsv


def slab_pool_backward(kg, vg, weight, bias, geometry, dsk, dsv, temperature=1.0):
    """Stage 5 on one rank: ``(dkg, dvg, dweight, dbias)`` from its summaries' gradients."""
    b, g, n, d = kg.shape
    tables = _device_tables(geometry, kg.device)
    fine, slots = geometry.blocks.shape
    dkg, dvg = torch.empty_like(kg), torch.empty_like(vg)
    f32 = dict(dtype=torch.float32, device=kg.device)
    dw, db = torch.empty(d, **f32), torch.empty(slots, **f32)
    w32, b32 = _f32(weight), _f32(bias)
    # bound to names: a temporary whose pointer alone is passed is freed (and its block reused) before the launch
    dsk, dsv = dsk.contiguous(), dsv.contiguous()
    lib = _native.lib()
    ws = _workspace(lib.p3d_pool_bwd_workspace(fine, slots, geometry.pool_size, b, g, d), kg.device)
    with torch.cuda.device(kg.device):
        status = lib.p3d_pool_bwd(_native.ptr(kg), _native.ptr(vg), _native.ptr(w32), _native.ptr(b32),
                                  _native.ptr(tables["blocks"]), fine, slots, geometry.pool_size,
                                  _native.ptr(dsk), _native.ptr(dsv), _native.ptr(dkg),
                                  _native.ptr(dvg), _native.ptr(dw), _native.ptr(db), _native.DTYPE_CODE[kg.dtype], b,
                                  g, n, d, float(temperature), _native.ptr(ws), ws.numel(),
                                  _native.stream_of(kg.device))
    _native.check(status, "p3d_pool_bwd")
    return dkg, dvg, dw, db


def scatter_summary_grads(ds, group=None):
    """Sum ``ds`` [B, G, world*M_rank, D] over ranks; each rank keeps its own M_rank rows."""
    world = dist.get_world_size(group)
    if world == 1:
        return ds.contiguous()
    b, g, m_all, d = ds.shape
    m = m_all // world
    chunks = ds.reshape(b, g, world, m, d).permute(2, 0, 1, 3, 4).contiguous()
    out = torch.empty((b, g, m, d), dtype=ds.dtype, device=ds.device)
    if dist.get_backend(group) == "nccl":
        dist.reduce_scatter_tensor(out, chunks.reshape(-1), group=group)
    else:   # gloo has no reduce-scatter: all-reduce, keep this rank's part
        dist.all_reduce(chunks, group=group)
        out.copy_(chunks[dist.get_rank(group)])
    return out


def _exchange_rows(t, slabs, group):
    """Halo exchange of a per-row tensor [B, H, N] (lse, Delta)."""
    return exchange_halos(t.unsqueeze(-1).contiguous(), slabs, group).squeeze(-1)


class _ShardedCore(torch.autograd.Function):
    """The sharded attention core with its sharded backward (first order)."""

    @staticmethod
    def forward(ctx, q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, slabs, group, temperature):
        q, kl, vl, kg, vg, gate = (t.contiguous() for t in (q, kl, vl, kg, vg, gate))
        sk_rank, sv_rank = pool_summaries(kg, vg, weight, bias, geometry, temperature)
        sk, sv = gather_summaries(sk_rank, group), gather_summaries(sv_rank, group)
        kl_ext, vl_ext = exchange_halos(kl, slabs, group), exchange_halos(vl, slabs, group)
        y, state = slab_forward(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, geometry, slabs, temperature,
                                save_state=True)
        _, _, ol, og, lse_l, lse_g = state
        ctx.save_for_backward(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, kl_ext, vl_ext, sk, sv, ol, og, lse_l,
                              lse_g)
        ctx.geometry, ctx.slabs, ctx.group, ctx.temperature = geometry, slabs, group, temperature
        return y

    @staticmethod
    def backward(ctx, dy):
        (q, kl, vl, kg, vg, weight, bias, gate, sl, sg, kl_ext, vl_ext, sk, sv, ol, og, lse_l,
         lse_g) = ctx.saved_tensors
        grads = sharded_core_backward(dy.contiguous(), (q, kl, vl, kg, vg, weight, bias, gate, sl, sg),
                                      (kl_ext, vl_ext, sk, sv, ol, og, lse_l, lse_g), ctx.geometry, ctx.slabs,
                                      ctx.group, ctx.temperature)
        return (*grads, None, None, None, None)


def sharded_core_backward(dy, inputs, saved, geometry, slabs: ZSlabs, group=None, temperature=1.0):
    """All ten input gradients of this rank's core (parameter gradients: this rank's share)."""
    q, kl, vl, kg, vg, weight, bias, gate, sl, sg = inputs
    kl_ext, vl_ext, sk, sv, ol, og, lse_l, lse_g = saved
    dol, dog, delta_l, delta_g, dgate, dsl, dsg = slab_mix_backward(dy, q, kl, vl, kg, vg, weight, bias, gate, sl,
                                                                    sg, ol, og, geometry, temperature)
    q_ext, dol_ext = exchange_halos(q, slabs, group), exchange_halos(dol, slabs, group)
    lse_l_ext, delta_l_ext = _exchange_rows(lse_l, slabs, group), _exchange_rows(delta_l, slabs, group)
    dq, dkl, dvl, dsk, dsv = slab_attention_backward(q, kl_ext, vl_ext, sk, sv, lse_l, lse_g, dol, dog, delta_l,
                                                     delta_g, q_ext, dol_ext, lse_l_ext, delta_l_ext, weight, bias,
                                                     gate, sl, sg, geometry, slabs, temperature)
    dsk_rank, dsv_rank = scatter_summary_grads(dsk, group), scatter_summary_grads(dsv, group)
    dkg, dvg, dw, db = slab_pool_backward(kg, vg, weight, bias, geometry, dsk_rank, dsv_rank, temperature)
    return (dq, dkl, dvl, dkg, dvg, dw.to(weight.dtype), db.to(bias.dtype), dgate.to(gate.dtype), dsl.to(sl.dtype),
            dsg.to(sg.dtype))


def sharded_core(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, slabs: ZSlabs, group=None, temperature=1.0):
    """This rank's attention core output; differentiable (sharded backward)."""
    return _ShardedCore.apply(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, slabs, group,
                              float(temperature))
