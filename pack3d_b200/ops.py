"""The operator boundary: ``pack3d_streamed`` over the C ABI.

Mirrors the reference's ``src/pack3d/backends/triton/autograd.py:8-64``:
validation, an explicit CUDA check, an autograd Function with an explicit
first-order backward that saves 19 tensors (10 inputs, 6 forward states, 3
geometry tables) and never an ``N x M`` buffer, and a gradient-free
inference short cut that saves nothing.  All compute is in
``libpack3d_b200.so``; nothing here falls back to PyTorch arithmetic.
"""
from __future__ import annotations

import torch
from torch.autograd.function import once_differentiable

from . import _native
from ._validation import check_cuda, validate_inputs
from .geometry import Pack3DGeometry

_GATE_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _device_tables(geometry, device):
    """int32 device copies of the geometry tables the kernels read (cached per device)."""
    key = ("tables", str(device))
    hit = geometry._cache.get(key)
    if hit is None:
        def dev(t):
            return None if t is None else t.to(device=device, dtype=torch.int32).contiguous()
        hit = {"neighbors": dev(geometry.neighbors), "reverse": dev(geometry.reverse_neighbors),
               "blocks": dev(geometry.blocks), "map": dev(geometry._stencil_map)}
        geometry._cache[key] = hit
    return hit


def _f32(t):
    return t.detach().to(torch.float32).contiguous()


def _operator(q, kl, vl, kg, vg, w32, b32, gate, sl32, sg32, geometry, temperature):
    """Fill a ``p3d_operator`` descriptor; the returned tuple keeps every buffer alive."""
    b, h, n, d = q.shape
    tables = _device_tables(geometry, q.device)
    op = _native.Operator()
    op.batch, op.heads, op.kv_heads, op.tokens, op.head_dim = b, h, kl.shape[1], n, d
    op.dtype = _native.DTYPE_CODE[q.dtype]
    op.gate_dtype = _native.DTYPE_CODE[gate.dtype]
    op.temperature = float(temperature)
    for name, t in (("q", q), ("kl", kl), ("vl", vl), ("kg", kg), ("vg", vg), ("pool_weight", w32),
                    ("slot_bias", b32), ("gate", gate), ("local_scale", sl32), ("global_scale", sg32)):
        setattr(op, name, t.data_ptr())
    op.neighbors, op.width = tables["neighbors"].data_ptr(), geometry.neighbors.shape[1]
    op.reverse_neighbors, op.reverse_width = tables["reverse"].data_ptr(), geometry.reverse_neighbors.shape[1]
    op.blocks = tables["blocks"].data_ptr()
    op.fine_blocks, op.slots = geometry.blocks.shape
    op.pool_size = geometry.pool_size
    if geometry.stencil is not None:
        grid, radius = geometry.stencil
        op.stencil = 1
        op.grid[:] = grid
        op.radius[:] = radius
        op.raster_to_packed = None if tables["map"] is None else tables["map"].data_ptr()
    return op, tables


def _workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _as_gate(gate, q):
    return gate if gate.dtype in _GATE_DTYPES else gate.to(torch.float32)


def raster_qkv_applies(geometry, dtype, head_dim, device):
    """True when the layout stores tokens out of raster order and the tensor-core stencil
    forward runs for it: q, kl, vl may then be produced at raster rows (``p3d_qkv_split``
    with ``SPLIT_RASTER_QKV``) and handed to :func:`forward` with ``raster_qkv=True``."""
    if geometry.stencil is None or geometry._stencil_map is None or dtype not in (torch.bfloat16, torch.float16):
        return False
    _, radius = geometry.stencil
    with torch.cuda.device(device):
        return bool(_native.lib().p3d_stencil_fwd_supported(_native.DTYPE_CODE[dtype], int(head_dim), *radius,
                                                            geometry.num_summaries))


def forward(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, temperature, *, save_state=True,
            force_indexed=False, summaries=None, y_rows=False, raster_qkv=False):
    """Launch the forward; returns ``(y, (sk, sv, ol, og, lse_l, lse_g))`` (empty state when not saving).

    ``summaries=(sk, sv)`` supplies already pooled summaries and runs stage (c) alone.
    ``y_rows`` writes y token-major: the result is a [B, H, N, D] view of a [B, N, H, D]
    tensor, so ``y.transpose(1, 2).reshape(B, N, H * D)`` needs no copy.
    ``raster_qkv``: q, kl, vl hold their rows at raster positions (see :func:`raster_qkv_applies`);
    kg, vg, gate and y keep the layout's row order.
    """
    b, h, n, d = q.shape
    g = kl.shape[1]
    gate = _as_gate(gate, q).contiguous()
    w32, b32, sl32, sg32 = (_f32(t) for t in (weight, bias, sl, sg))
    op, keep = _operator(q, kl, vl, kg, vg, w32, b32, gate, sl32, sg32, geometry, temperature)
    m = geometry.num_summaries
    empty = lambda *shape, dtype=q.dtype: torch.empty(shape, dtype=dtype, device=q.device)  # noqa: E731
    y = empty(b, n, h, d).permute(0, 2, 1, 3) if y_rows else empty(b, h, n, d)
    flags = (_native.FWD_SAVE_STATE if save_state else 0) | (_native.FWD_FORCE_INDEXED if force_indexed else 0)
    flags |= _native.FWD_Y_ROWS if y_rows else 0
    flags |= _native.FWD_RASTER_QKV if raster_qkv else 0
    if summaries is None:
        sk, sv = empty(b, g, m, d), empty(b, g, m, d)
    else:
        sk, sv = summaries
        if sk.shape != (b, g, m, d) or sv.shape != sk.shape or sk.dtype != q.dtype or not sk.is_contiguous():
            raise ValueError("given summaries must be contiguous [B, G, M, D] in the input dtype")
        flags |= _native.FWD_SUMMARIES_GIVEN
    ol = og = lse_l = lse_g = None
    if save_state:
        ol, og = empty(b, h, n, d), empty(b, h, n, d)
        lse_l, lse_g = empty(b, h, n, dtype=torch.float32), empty(b, h, n, dtype=torch.float32)
    handle = _native.lib()
    ws = _workspace(handle.p3d_attn_fwd_workspace(op, flags), q.device)
    with torch.cuda.device(q.device):
        status = handle.p3d_attn_fwd(op, _native.ptr(y), _native.ptr(sk), _native.ptr(sv), _native.ptr(ol),
                                     _native.ptr(og), _native.ptr(lse_l), _native.ptr(lse_g), flags,
                                     _native.ptr(ws), ws.numel(), _native.stream_of(q.device))
    _native.check(status, "p3d_attn_fwd")
    del keep
    return y, ((sk, sv, ol, og, lse_l, lse_g) if save_state else ())


def backward(dy, inputs, saved, geometry, temperature, *, force_indexed=False, dy_rows=False):
    """Launch the backward; returns the ten input gradients in the inputs' dtypes.

    ``force_indexed`` runs the neighbour-table kernels even on a complete stencil.
    ``dy_rows``: dy is a [B, H, N, D] view of a contiguous [B, N, H, D] tensor (token-major).
    """
    q, kl, vl, kg, vg, weight, bias, gate, sl, sg = inputs
    sk, sv, ol, og, lse_l, lse_g = saved
    gate_k = _as_gate(gate, q).contiguous()
    w32, b32, sl32, sg32 = (_f32(t) for t in (weight, bias, sl, sg))
    op, keep = _operator(q, kl, vl, kg, vg, w32, b32, gate_k, sl32, sg32, geometry, temperature)
    if force_indexed:
        op.options |= _native.OPT_INDEXED_ONLY
    if dy_rows:
        op.options |= _native.OPT_DY_ROWS
    dq, dkl, dvl, dkg, dvg = (torch.empty_like(t) for t in (q, kl, vl, kg, vg))
    dgate = torch.empty_like(gate_k)
    d = q.shape[-1]
    f32 = dict(dtype=torch.float32, device=q.device)
    dw, dsl, dsg = torch.empty(d, **f32), torch.empty(d, **f32), torch.empty(d, **f32)
    db = torch.empty(bias.shape[0], **f32)
    handle = _native.lib()
    ws = _workspace(handle.p3d_attn_bwd_workspace(op), q.device)
    with torch.cuda.device(q.device):
        status = handle.p3d_attn_bwd(op, _native.ptr(dy), _native.ptr(sk), _native.ptr(sv), _native.ptr(ol),
                                     _native.ptr(og), _native.ptr(lse_l), _native.ptr(lse_g), _native.ptr(dq),
                                     _native.ptr(dkl), _native.ptr(dvl), _native.ptr(dkg), _native.ptr(dvg),
                                     _native.ptr(dgate), _native.ptr(dw), _native.ptr(db), _native.ptr(dsl),
                                     _native.ptr(dsg), _native.ptr(ws), ws.numel(),
                                     _native.stream_of(q.device))
    _native.check(status, "p3d_attn_bwd")
    del keep
    return (dq, dkl, dvl, dkg, dvg, dw.to(weight.dtype), db.to(bias.dtype), dgate.to(gate.dtype),
            dsl.to(sl.dtype), dsg.to(sg.dtype))


def _token_major(t):
    """True when the [B, H, N, D] tensor t is a view of a contiguous [B, N, H, D] tensor."""
    return t.transpose(1, 2).is_contiguous()


class _Pack3D(torch.autograd.Function):
    """The core as an autograd function.  ``y_rows`` returns y token-major (a [B, H, N, D]
    view of a [B, N, H, D] tensor, as the layer's output projection reads it); a gradient
    arriving in that layout is consumed without a copy (``P3D_OPT_DY_ROWS``)."""

    @staticmethod
    def forward(ctx, q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, temperature, y_rows=False):
        inputs = tuple(t.contiguous() for t in (q, kl, vl, kg, vg, weight, bias, gate, sl, sg))
        y, saved = forward(*inputs, geometry, temperature, y_rows=y_rows)
        ctx.save_for_backward(*inputs, *saved, *geometry.tensors)
        ctx.geometry, ctx.temperature = geometry, temperature
        return y

    @staticmethod
    @once_differentiable
    def backward(ctx, dy):
        ctx.geometry.check_unmodified()
        saved = ctx.saved_tensors
        if dy.is_contiguous():
            grads = backward(dy, saved[:10], saved[10:16], ctx.geometry, ctx.temperature)
        elif _token_major(dy):
            grads = backward(dy, saved[:10], saved[10:16], ctx.geometry, ctx.temperature, dy_rows=True)
        else:
            grads = backward(dy.contiguous(), saved[:10], saved[10:16], ctx.geometry, ctx.temperature)
        return (*grads, None, None, None)


def pack3d_token_major(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry: Pack3DGeometry, *,
                       temperature=1.0):
    """:func:`pack3d_streamed` with y returned token-major: a [B, H, N, D] view of a [B, N, H, D]
    tensor, so ``y.transpose(1, 2).reshape(B, N, H * D)`` (the output projection's input) is
    free, and its gradient reaches the backward without a transpose copy."""
    validate_inputs(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, temperature)
    check_cuda(q)
    inputs = (q, kl, vl, kg, vg, weight, bias, gate, sl, sg)
    if torch.is_grad_enabled() and any(t.requires_grad for t in inputs):
        return _Pack3D.apply(*inputs, geometry, float(temperature), True)
    y, _ = forward(*(t.contiguous() for t in inputs), geometry, float(temperature), save_state=False, y_rows=True)
    return y


def pack3d_streamed(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry: Pack3DGeometry, *,
                    temperature=1.0, backend="b200"):
    """Local-residual / global-gated PACK3D core on rotated projections.

    ``y = sl * softmax_local(q kl^T / sqrt(D)) vl + gate * sg * softmax_global(q sk^T / sqrt(D)) sv``
    with ``sk, sv`` the pooled summaries of ``kg, vg``.  Same signature and
    contract as the reference's ``pack3d_streamed`` (autograd.py:40-64) with
    ``backend="b200"``.  Unsupported inputs raise; nothing falls back.
    """
    validate_inputs(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, temperature)
    if backend != "b200":
        raise ValueError(f"unknown explicit backend {backend!r}")
    check_cuda(q)
    inputs = (q, kl, vl, kg, vg, weight, bias, gate, sl, sg)
    if torch.is_grad_enabled() and any(t.requires_grad for t in inputs):
        return _Pack3D.apply(*inputs, geometry, float(temperature))
    y, _ = forward(*(t.contiguous() for t in inputs), geometry, float(temperature), save_state=False)
    return y
