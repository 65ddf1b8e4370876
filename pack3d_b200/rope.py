"""Stage (a): axial RoPE on the GPU, mirroring the reference's rotary interface.

``rotate_projections`` has the signature of the reference's
``src/pack3d/backends/triton/rotary.py:94-106`` and returns contiguous
head-major rotated tensors with an autograd backward (the inverse rotation,
``rotary.py:58-70``).  The work runs in ``p3d_rope`` (C ABI).

The (cos, sin) phase table is computed once per (device, pairs, grid extents)
on the host with exactly the fp32 operations of ``src/pack3d/rope.py:43-46``
-- ``base ** (-i / count)`` times the integer coordinate -- so the rotation is
bit-identical to the reference.  Packed-sequence positions, or extents whose
table would exceed ``TABLE_LIMIT`` entries, rotate with on-device ``sincosf``
of the same fp32 angles.
"""
from __future__ import annotations

import threading

import torch
from torch.autograd.function import once_differentiable

from . import _native

TABLE_LIMIT = 65536
BASE = 10000.0


def balanced_pairs(head_dim):
    """Pairs per (z, y, x) axis: ``head_dim // 2`` dealt evenly, remainder first (rope.py:7-12)."""
    if type(head_dim) is not int or head_dim <= 0 or head_dim % 2:
        raise ValueError("head_dim must be a positive even integer")
    share, extra = divmod(head_dim // 2, 3)
    return tuple(share + (1 if axis < extra else 0) for axis in range(3))


def _frequencies(count):
    return BASE ** (-torch.arange(count, dtype=torch.float32) / count)


_tables = {}
_tables_lock = threading.Lock()


def phase_tables(device, pairs, extents):
    """``(freqs, phases)`` on ``device``: concatenated per-axis frequencies and, when
    ``extents`` is given and small enough, the (cos, sin) table of every
    (axis, coordinate, pair)."""
    key = (str(device), tuple(pairs), tuple(extents) if extents else None)
    with _tables_lock:
        hit = _tables.get(key)
    if hit is not None:
        return hit
    with torch.inference_mode(False):
        freqs = torch.cat([_frequencies(c) for c in pairs if c] or [torch.zeros(0)])
        phases = None
        if extents and sum(e * c for e, c in zip(extents, pairs)) <= TABLE_LIMIT:
            parts = []
            for extent, count in zip(extents, pairs):
                if count:
                    angle = torch.arange(extent, dtype=torch.float32)[:, None] * _frequencies(count)
                    parts.append(angle.flatten())
            angle = torch.cat(parts)
            phases = torch.stack((angle.cos(), angle.sin()), -1).contiguous().to(device)
        entry = (freqs.to(device), phases)
    with _tables_lock:
        _tables[key] = entry
    return entry


def _rotate(x, coords, pairs, extents, packed, inverse):
    b, h, n, d = x.shape
    out = torch.empty((b, h, n, d), dtype=x.dtype, device=x.device)
    freqs, phases = phase_tables(x.device, pairs, None if packed else extents)
    use_table = phases is not None
    coords_ptr, csn, csa = None, 0, 0
    if not packed:
        coords = coords.to(device=x.device, dtype=torch.int64)
        coords_ptr, (csn, csa) = _native.ptr(coords), coords.stride()
    ez, ey, ex = (extents if use_table else (0, 0, 0))
    with torch.cuda.device(x.device):
        status = _native.lib().p3d_rope(
            _native.ptr(x), *x.stride(), _native.ptr(out), _native.DTYPE_CODE[x.dtype], b, h, n, d,
            coords_ptr, csn, csa, *pairs, _native.ptr(freqs), _native.ptr(phases) if use_table else None,
            ez, ey, ex, int(packed), int(inverse), _native.stream_of(x.device))
    _native.check(status, "p3d_rope")
    return out


class _Rotary(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, coords, pairs, extents, packed):
        ctx.save_for_backward(coords)
        ctx.pairs, ctx.extents, ctx.packed = pairs, extents, packed
        return _rotate(x, coords, pairs, extents, packed, inverse=False)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        coords, = ctx.saved_tensors
        return _rotate(grad, coords, ctx.pairs, ctx.extents, ctx.packed, inverse=True), None, None, None, None


def rotate_projections(q, kl, kg, coords, pairs, grid_shape, *, packed):
    """Rotate ``q``, local ``k`` and global ``k`` (``[B, heads, N, D]``, any strides)
    into contiguous head-major tensors.  ``coords`` is ``[N, 3]`` (ignored when
    ``packed``: packed-sequence RoPE uses the row index on axis 0)."""
    pairs = tuple(int(p) for p in pairs)
    for t in (q, kl, kg):
        if t.ndim != 4 or t.device.type != "cuda" or t.dtype not in _native.DTYPE_CODE:
            raise ValueError("rotate_projections needs CUDA fp32/fp16/bf16 [B, heads, N, D] tensors")
        if sum(pairs) * 2 != t.shape[-1]:
            raise ValueError("pairs must allocate every rotary pair across three axes")
    extents = tuple(int(s) for s in grid_shape)
    return tuple(_Rotary.apply(x, coords, pairs, extents, bool(packed)) for x in (q, kl, kg))
