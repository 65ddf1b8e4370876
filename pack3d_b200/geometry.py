"""Token layouts and validated coordinate graphs (host side, built once on the CPU).

API-compatible with the reference's ``src/pack3d/geometry.py``:
``Pack3DGeometry`` (:11-50), ``prepare_geometry`` (:54-101),
``grid_coordinates`` (:112-115), the Morton code (:118-126), ``TokenLayout``
with ``pack / unpack / repack`` (:129-220) and ``build_layout`` (:224-266).
The tables are bit-identical to the reference's (pinned by golden digests);
the construction is vectorised so a 64^3 radius-2 layout builds in seconds.

Beyond the reference, every layout made by ``build_layout`` carries a
*stencil tag* -- the grid shape, the neighbourhood radius and the
raster->packed row map -- for every radius, not only radius one.  The tag is
what lets the CUDA kernels derive each query's neighbourhood from voxel
coordinates instead of reading the neighbour table.  ``repack`` transports
the tag by composing the map with the permutation, exactly as the reference
transports its radius-one tag (:211-217).  Graphs built directly with
``prepare_geometry`` carry no tag and use the indexed kernels.
"""
from __future__ import annotations

import math
from itertools import product

import torch
from torch import Tensor

_SEAL = object()

MAX_NEIGHBORS = 128       # local / reverse degree (reference geometry.py:71,94)
MAX_SLOTS = 64            # canonical fine-block slots (geometry.py:71)
MAX_POOL = 32             # fine blocks per summary (geometry.py:66)


class Pack3DGeometry:
    """Validated neighbour / reverse-neighbour / fine-block tables.

    Construct only through :func:`prepare_geometry`.  Tensors are treated as
    immutable: their version counters are recorded and any in-place change
    makes :meth:`check_unmodified` raise ``RuntimeError``.
    """

    __slots__ = ("neighbors", "reverse_neighbors", "blocks", "pool_size", "num_tokens",
                 "_radius_one_grid", "_raster_to_packed", "_stencil", "_stencil_map",
                 "_versions", "_cache")

    def __init__(self, neighbors, reverse_neighbors, blocks, pool_size, num_tokens, *, _seal=None,
                 _radius_one_grid=None, _raster_to_packed=None, _stencil=None, _stencil_map=None):
        if _seal is not _SEAL:
            raise ValueError("Use prepare_geometry() to validate indices before launching CUDA")
        self.neighbors = neighbors
        self.reverse_neighbors = reverse_neighbors
        self.blocks = blocks
        self.pool_size = pool_size
        self.num_tokens = num_tokens
        self._radius_one_grid = _radius_one_grid
        self._raster_to_packed = _raster_to_packed
        self._stencil = _stencil            # (grid_shape, radius) of a complete grid stencil
        self._stencil_map = _stencil_map    # raster -> packed int32 map, None when identity
        self._cache = {}
        self._versions = self._tensor_versions()

    def __setattr__(self, name, value):
        if hasattr(self, "_versions") and name != "_cache":
            raise AttributeError("Pack3DGeometry is immutable")
        object.__setattr__(self, name, value)

    def _tracked(self):
        extra = [t for t in (self._raster_to_packed, self._stencil_map) if t is not None]
        return (*self.tensors, *extra)

    def _tensor_versions(self):
        return tuple(t._version for t in self._tracked())

    @property
    def tensors(self):
        return self.neighbors, self.reverse_neighbors, self.blocks

    @property
    def num_summaries(self):
        return -(-self.blocks.shape[0] // self.pool_size)

    @property
    def stencil(self):
        """``(grid_shape, radius)`` when the graph is a complete voxel stencil, else ``None``."""
        return self._stencil

    def check_unmodified(self):
        if self._tensor_versions() != self._versions:
            raise RuntimeError("Geometry changed after validation; prepare it again")

    @torch.inference_mode(False)
    def to(self, device):
        self.check_unmodified()
        move = (lambda t: None if t is None else t.to(device))
        return Pack3DGeometry(*(t.to(device) for t in self.tensors), self.pool_size, self.num_tokens,
                              _seal=_SEAL, _radius_one_grid=self._radius_one_grid,
                              _raster_to_packed=move(self._raster_to_packed), _stencil=self._stencil,
                              _stencil_map=move(self._stencil_map))

    def _retag(self, **changes):
        fields = dict(_radius_one_grid=self._radius_one_grid, _raster_to_packed=self._raster_to_packed,
                      _stencil=self._stencil, _stencil_map=self._stencil_map)
        fields.update(changes)
        return Pack3DGeometry(*self.tensors, self.pool_size, self.num_tokens, _seal=_SEAL, **fields)

    def __repr__(self):
        return (f"Pack3DGeometry(tokens={self.num_tokens}, width={self.neighbors.shape[1]}, "
                f"fine_blocks={self.blocks.shape[0]}, slots={self.blocks.shape[1]}, "
                f"pool_size={self.pool_size}, stencil={self._stencil})")


def _reverse_adjacency(nb):
    """For each token j, the ascending list of rows i whose neighbour list holds j."""
    n = nb.shape[0]
    valid = nb >= 0
    dst = nb[valid]
    src = torch.arange(n).repeat_interleave(valid.sum(1))
    # Row-major enumeration already sorts src; a stable sort by dst keeps that order.
    order = torch.sort(dst, stable=True).indices
    src, dst = src[order], dst[order]
    counts = torch.bincount(dst, minlength=n)
    width = max(1, int(counts.max()) if counts.numel() else 1)
    if width > MAX_NEIGHBORS:
        raise ValueError("reverse local degree exceeds 128")
    starts = torch.cumsum(counts, 0) - counts
    column = torch.arange(dst.numel()) - starts[dst]
    reverse = torch.full((n, width), -1, dtype=torch.int32)
    reverse[dst, column] = src.to(torch.int32)
    return reverse


@torch.inference_mode(False)
def prepare_geometry(neighbors: Tensor, blocks: Tensor, pool_size: int) -> Pack3DGeometry:
    """Validate a local graph and a fine-block partition on the CPU, once.

    ``neighbors[i]`` lists the keys of query ``i`` (-1 pads); ``blocks[f]``
    lists fine block ``f``'s member tokens by canonical slot (-1 = empty
    slot); consecutive groups of ``pool_size`` fine blocks form one summary.
    Mirrors the reference's checks and messages (``geometry.py:54-101``) and
    builds the reverse adjacency used by race-free local K/V gradients.
    """
    return _prepare(neighbors, blocks, pool_size, symmetric=False)


def _prepare(neighbors, blocks, pool_size, *, symmetric):
    """``symmetric=True`` is for graphs known to satisfy ``j in nb[i] <=> i in nb[j]``
    (complete voxel stencils and their repacks): the reverse list of ``j`` is then
    its own neighbour list in ascending order, read off the sorted rows."""
    for name, value in (("neighbors", neighbors), ("blocks", blocks)):
        if value.ndim != 2 or value.dtype not in (torch.int32, torch.int64):
            raise ValueError(f"{name} must be a rank-two integer tensor")
        if min(value.shape) == 0:
            raise ValueError(f"{name} must be nonempty")
    if type(pool_size) is not int or not 1 <= pool_size <= MAX_POOL:
        raise ValueError("pool_size must be an integer in [1,32]")
    nb = neighbors.detach().to(device="cpu", dtype=torch.int64).contiguous().clone()
    members = blocks.detach().to(device="cpu", dtype=torch.int64).contiguous().clone()
    n = nb.shape[0]
    if nb.shape[1] > MAX_NEIGHBORS or members.shape[1] > MAX_SLOTS:
        raise ValueError("at most 128 neighbors and 64 fine-block slots are supported")
    if max(nb.numel(), members.numel()) >= 2**31:
        raise ValueError("geometry exceeds the 32-bit kernel indexing limit")
    for name, value in (("neighbors", nb), ("blocks", members)):
        if bool(((value < -1) | (value >= n)).any()):
            raise ValueError(f"{name} contains an out-of-range token")
    # Sort each row with the -1 pads last; equal neighbours then sit side by side.
    ordered = torch.where(nb >= 0, nb, n).sort(dim=1).values
    if bool(((ordered[:, 1:] == ordered[:, :-1]) & (ordered[:, 1:] < n)).any()):
        raise ValueError("duplicate local edges are not supported")
    covered = members[members >= 0]
    if covered.numel() != n or not bool((torch.bincount(covered, minlength=n) == 1).all()):
        raise ValueError("fine blocks must partition every token exactly once")
    nonempty = (members >= 0).any(dim=1)
    groups = -(-members.shape[0] // pool_size)
    padded = torch.zeros(groups * pool_size, dtype=torch.bool)
    padded[:members.shape[0]] = nonempty
    if not bool(padded.view(groups, pool_size).any(1).all()):
        raise ValueError("an entirely empty coarse group is unsupported")
    if symmetric:
        width = max(1, int((nb >= 0).sum(1).max()))
        reverse = ordered[:, :width].masked_fill(ordered[:, :width] == n, -1).to(torch.int32)
    else:
        reverse = _reverse_adjacency(nb)
    return Pack3DGeometry(nb.to(torch.int32), reverse, members.to(torch.int32), pool_size, n, _seal=_SEAL)


def _triple(value, name, *, allow_zero=False):
    values = (value,) * 3 if type(value) is int else tuple(value)
    least = 0 if allow_zero else 1
    if len(values) != 3 or any(type(v) is not int or v < least for v in values):
        raise ValueError(f"{name} must contain three integers >= {least}")
    return values


def grid_coordinates(shape):
    """CPU int64 ``[Z*Y*X, 3]`` voxel coordinates ``(z, y, x)`` in raster order."""
    z, y, x = _triple(shape, "shape")
    axes = torch.meshgrid(torch.arange(z), torch.arange(y), torch.arange(x), indexing="ij")
    return torch.stack(axes, -1).reshape(-1, 3)


def morton_codes(coords):
    """Interleave coordinate bits, axis 0 (z) lowest: bit ``b`` of axis ``a`` -> ``3b + a``."""
    top = int(coords.max()) if coords.numel() else 0
    bits = top.bit_length()
    if bits > 20:
        raise ValueError("Morton coordinates exceed the supported int64 range")
    code = torch.zeros(coords.shape[0], dtype=torch.int64)
    for bit in range(bits):
        code |= ((coords >> bit) & 1).mul(torch.tensor([1, 2, 4]) << (3 * bit)).sum(1)
    return code


def _compose_map(old_map, inverse, n):
    """raster -> new row, given raster -> old row (None = identity) and old row -> new row."""
    mapping = inverse if old_map is None else inverse[old_map.cpu().long()]
    return None if torch.equal(mapping, torch.arange(n)) else mapping.to(torch.int32)


class TokenLayout:
    """A complete unpadded 3D field stored in an explicit token order.

    ``order[i]`` is packed row ``i``'s raster index and ``coords[i]`` its
    ``(z, y, x)``; ``geometry`` holds the graph over packed rows.  All
    tensors are immutable; ``repack`` transports the graph to a new order.
    """

    __slots__ = ("grid_shape", "order", "coords", "geometry", "_versions")

    def __init__(self, grid_shape, order, coords, geometry):
        shape = _triple(grid_shape, "grid_shape")
        n = math.prod(shape)
        if order.shape != (n,) or order.dtype != torch.int64:
            raise ValueError("order must be an int64 permutation of the grid")
        if coords.shape != (n, 3) or coords.dtype != torch.int64:
            raise ValueError("coords must be int64 [tokens, 3]")
        host_order = order.detach().cpu()
        if not torch.equal(host_order.sort().values, torch.arange(n)):
            raise ValueError("order must be a permutation")
        if not torch.equal(coords.detach().cpu(), grid_coordinates(shape)[host_order]):
            raise ValueError("coordinates do not agree with order")
        if n != geometry.num_tokens or any(t.device != order.device for t in (coords, *geometry.tensors)):
            raise ValueError("layout and geometry must agree on token count and device")
        object.__setattr__(self, "grid_shape", shape)
        object.__setattr__(self, "order", order)
        object.__setattr__(self, "coords", coords)
        object.__setattr__(self, "geometry", geometry)
        object.__setattr__(self, "_versions", (order._version, coords._version))

    def __setattr__(self, name, value):
        raise AttributeError("TokenLayout is immutable")

    def check_unmodified(self):
        self.geometry.check_unmodified()
        if self._versions != (self.order._version, self.coords._version):
            raise RuntimeError("layout changed in place; construct a new layout")

    @torch.inference_mode(False)
    def to(self, device):
        """Move the metadata to a device; coordinates and membership are unchanged."""
        self.check_unmodified()
        return TokenLayout(self.grid_shape, self.order.to(device), self.coords.to(device),
                           self.geometry.to(device))

    def pack(self, grid):
        """``[batch, Z, Y, X, channels]`` -> ``[batch, tokens, channels]`` in this layout's order."""
        self.check_unmodified()
        if grid.ndim != 5 or tuple(grid.shape[1:4]) != self.grid_shape:
            raise ValueError("input must match [batch,Z,Y,X,channels]")
        return grid.flatten(1, 3).index_select(1, self.order.to(grid.device))

    def unpack(self, packed):
        """Inverse of :meth:`pack`."""
        self.check_unmodified()
        if packed.ndim != 3 or packed.shape[1] != self.geometry.num_tokens:
            raise ValueError("packed input must have shape [batch,tokens,channels]")
        raster = packed.index_select(1, self.order.argsort().to(packed.device))
        return raster.reshape(packed.shape[0], *self.grid_shape, packed.shape[-1])

    @torch.inference_mode(False)
    def repack(self, permutation):
        """New row ``i`` is old row ``permutation[i]``; the graph is transported, never rebuilt.

        Fine-block rows, canonical slot columns and coarse groups keep their
        identity; only token row indices change (reference ``geometry.py:190-220``).
        """
        self.check_unmodified()
        n = self.geometry.num_tokens
        p = torch.as_tensor(permutation).detach().cpu()
        if p.dtype not in (torch.int32, torch.int64) or p.shape != (n,):
            raise ValueError("permutation must be an integer vector with one entry per token")
        p = p.long()
        if not torch.equal(p.sort().values, torch.arange(n)):
            raise ValueError("permutation must contain every token exactly once")
        inverse = torch.empty_like(p)
        inverse[p] = torch.arange(n)
        old = self.geometry
        blocks = old.blocks.cpu().long()
        blocks = torch.where(blocks >= 0, inverse[blocks.clamp_min(0)], -1)
        lib = _native_geometry() if old._stencil is not None else None
        if lib is not None:
            nb, reverse = _native_repack_tables(lib, old.neighbors.cpu(), p)
            geom = _geometry_from_tables(nb, reverse, blocks.to(torch.int32), old.pool_size, n)
        else:
            nb = old.neighbors.cpu()[p].long()
            nb = torch.where(nb >= 0, inverse[nb.clamp_min(0)], -1)
            geom = _prepare(nb, blocks, old.pool_size, symmetric=old._stencil is not None)
        tags = {}
        if old._radius_one_grid is not None:
            tags.update(_radius_one_grid=old._radius_one_grid,
                        _raster_to_packed=_compose_map(old._raster_to_packed, inverse, n))
        if old._stencil is not None:
            tags.update(_stencil=old._stencil, _stencil_map=_compose_map(old._stencil_map, inverse, n))
        if tags:
            geom = geom._retag(**tags)
        moved = TokenLayout(self.grid_shape, self.order.cpu()[p].clone(), self.coords.cpu()[p].clone(), geom)
        return moved.to(self.order.device)


def _native_geometry():
    """The library's host builders (``p3d_stencil_neighbors`` / ``p3d_repack_neighbors``: one
    multithreaded pass, bit-identical to the tensor formulation in this module), or None
    when the library is not built -- the tensor formulation then builds the same tables."""
    try:
        from . import _native
        return _native.lib()
    except (OSError, RuntimeError):
        return None


def _native_check(status, what):
    from . import _native
    _native.check(status, what)


def _geometry_from_tables(nb32, reverse32, blocks32, pool_size, n):
    """A geometry from natively built stencil tables (valid by construction: every checked
    property of ``_prepare`` holds for a complete stencil and its repacks)."""
    if type(pool_size) is not int or not 1 <= pool_size <= MAX_POOL:
        raise ValueError("pool_size must be an integer in [1,32]")
    if nb32.shape[1] > MAX_NEIGHBORS or blocks32.shape[1] > MAX_SLOTS:
        raise ValueError("at most 128 neighbors and 64 fine-block slots are supported")
    if max(nb32.numel(), blocks32.numel()) >= 2**31:
        raise ValueError("geometry exceeds the 32-bit kernel indexing limit")
    return Pack3DGeometry(nb32, reverse32, blocks32, pool_size, n, _seal=_SEAL)


def _native_stencil_tables(lib, shape, radius, order):
    """``(neighbors, reverse)`` int32 of the complete stencil over packed rows ``order``."""
    import ctypes
    n, width = order.shape[0], math.prod(2 * r + 1 for r in radius)
    order = order.contiguous()
    nb = torch.empty((n, width), dtype=torch.int32)
    ordered = torch.empty_like(nb)
    widest = ctypes.c_int32(0)
    _native_check(lib.p3d_stencil_neighbors(*shape, *radius, ctypes.c_void_p(order.data_ptr()), n,
                                            ctypes.c_void_p(nb.data_ptr()), ctypes.c_void_p(ordered.data_ptr()),
                                            ctypes.byref(widest), 0), "p3d_stencil_neighbors")
    return nb, ordered[:, :max(1, widest.value)].contiguous()


def _native_repack_tables(lib, neighbors, permutation):
    """``(neighbors, reverse)`` int32 of a symmetric graph transported by ``permutation``."""
    import ctypes
    nb_old = neighbors.to(torch.int32).contiguous()
    n, width = nb_old.shape
    perm = permutation.to(torch.int64).contiguous()
    nb = torch.empty_like(nb_old)
    ordered = torch.empty_like(nb_old)
    widest = ctypes.c_int32(0)
    _native_check(lib.p3d_repack_neighbors(n, width, ctypes.c_void_p(nb_old.data_ptr()),
                                           ctypes.c_void_p(perm.data_ptr()), ctypes.c_void_p(nb.data_ptr()),
                                           ctypes.c_void_p(ordered.data_ptr()), ctypes.byref(widest), 0),
                  "p3d_repack_neighbors")
    return nb, ordered[:, :max(1, widest.value)].contiguous()


def _stencil_neighbors(coords, inverse, shape, radius):
    """Neighbour table: one column per offset, z-major ``itertools.product`` order, -1 outside."""
    n = coords.shape[0]
    extent = torch.tensor(shape)
    strides = torch.tensor([shape[1] * shape[2], shape[2], 1])
    columns = []
    for offset in product(*(range(-r, r + 1) for r in radius)):
        target = coords + torch.tensor(offset)
        inside = ((target >= 0) & (target < extent)).all(-1)
        raster = (target * strides).sum(-1).clamp(0, n - 1)
        columns.append(torch.where(inside, inverse[raster], -1))
    return torch.stack(columns, 1)


@torch.inference_mode(False)
def build_layout(grid_shape, block_shape=(2, 2, 2), *, radius=1, pool_size=4,
                 layout="native_block_morton"):
    """Prepare an unpadded 3D layout on the CPU, once, outside any timed region.

    ``native_block_morton`` orders fine blocks by the Morton code of their
    block coordinate and tokens within a block by the Morton code of their
    slot; ``raster_block`` keeps raster order and groups consecutive raster
    tokens by block *volume* (reference ``geometry.py:224-266``).  The local
    graph holds every in-grid offset within ``radius`` (the query included).
    """
    shape = _triple(grid_shape, "grid_shape")
    block = _triple(block_shape, "block_shape")
    rad = _triple(radius, "radius", allow_zero=True)
    if any(s % b for s, b in zip(shape, block)):
        raise ValueError("build_layout requires an unpadded grid divisible by block_shape")
    if math.prod(block) > MAX_SLOTS or math.prod(2 * r + 1 for r in rad) > MAX_NEIGHBORS:
        raise ValueError("layout exceeds supported block or neighborhood width")
    coords = grid_coordinates(shape)
    n = coords.shape[0]
    if layout == "native_block_morton":
        size = torch.tensor(block)
        slot = morton_codes(coords % size)
        key = morton_codes(coords // size) * (int(slot.max()) + 1) + slot
        order = key.argsort()
    elif layout == "raster_block":
        order = torch.arange(n)
    else:
        raise ValueError("layout must be raster_block or native_block_morton")
    coords = coords[order]
    inverse = torch.empty_like(order)
    inverse[order] = torch.arange(n)
    blocks = torch.arange(n).reshape(-1, math.prod(block))
    lib = _native_geometry()
    if lib is not None:
        nb, reverse = _native_stencil_tables(lib, shape, rad, order)
        geom = _geometry_from_tables(nb, reverse, blocks.to(torch.int32), pool_size, n)
    else:
        geom = _prepare(_stencil_neighbors(coords, inverse, shape, rad), blocks, pool_size, symmetric=True)
    raster = layout == "raster_block"
    tags = dict(_stencil=(shape, rad), _stencil_map=None if raster else inverse.to(torch.int32))
    if rad == (1, 1, 1) and n >= 4096 and shape[0] >= 2 and shape[1] >= 2 and shape[2] >= 4:
        tags.update(_radius_one_grid=shape, _raster_to_packed=None if raster else inverse.to(torch.int32))
    return TokenLayout(shape, order, coords, geom._retag(**tags))
