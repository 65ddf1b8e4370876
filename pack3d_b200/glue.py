"""Fused layer glue for the training path of :class:`PACK3DAttention` (reference
``attention.py:53-89``): autograd functions over the library's glue kernels.

* :func:`layer_norm` -- ``nn.LayerNorm`` (``attention.py:64``) as ``p3d_layer_norm`` with
  ``p3d_layer_norm_bwd`` as its backward (dweight / dbias summed in fixed order);
  :func:`layer_norm_residual` also hands x on to the outer residual (``attention.py:89``) and
  adds that branch's gradient inside the same backward kernel.
* :func:`qkv_split` -- the projection split of ``attention.py:70-81``: the row-major
  ``to_q`` / ``to_kv`` outputs become rotated head-major q, kl, kg and head-major vl, vg in
  one ``p3d_qkv_split`` pass; its backward, ``p3d_qkv_merge``, rotates dq, dkl, dkg back and
  writes the row-major projection gradients in one pass (bit-identical to the inverse
  rotation of ``rotary.py:66-70`` followed by autograd's transposes and concatenation).

16-bit tensors on the GPU only; the layer falls back to its per-op path otherwise.
"""
from __future__ import annotations

import torch
from torch.autograd.function import once_differentiable

from . import _native


def _empty_ws(nbytes, device):
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def _ln_forward(ctx, x, weight, bias, eps):
    x = x.contiguous()
    y = torch.empty_like(x)
    rows, dim = x.numel() // x.shape[-1], x.shape[-1]
    with torch.cuda.device(x.device):
        _native.check(_native.lib().p3d_layer_norm(_native.ptr(x), _native.ptr(weight), _native.ptr(bias),
                                                   _native.ptr(y), _native.DTYPE_CODE[x.dtype], rows, dim,
                                                   float(eps), _native.stream_of(x.device)), "p3d_layer_norm")
    ctx.save_for_backward(x, weight)
    ctx.eps = float(eps)
    return x, y


def _ln_backward(ctx, dy, dres=None):
    """``(dx, dweight, dbias, None)``; with ``dres`` (the residual branch's gradient of x) the
    kernel adds it into dx (``p3d_layer_norm_bwd_residual``)."""
    x, weight = ctx.saved_tensors
    dy = dy.contiguous()
    rows, dim = x.numel() // x.shape[-1], x.shape[-1]
    dx = torch.empty_like(x)
    f32 = dict(dtype=torch.float32, device=x.device)
    dw, db = torch.empty(dim, **f32), torch.empty(dim, **f32)
    lib = _native.lib()
    ws = _empty_ws(lib.p3d_layer_norm_bwd_workspace(rows, dim), x.device)
    tail = (_native.ptr(dx), _native.ptr(dw), _native.ptr(db), _native.DTYPE_CODE[x.dtype], rows, dim, ctx.eps,
            _native.ptr(ws), ws.numel(), _native.stream_of(x.device))
    with torch.cuda.device(x.device):
        if dres is None:
            _native.check(lib.p3d_layer_norm_bwd(_native.ptr(x), _native.ptr(weight), _native.ptr(dy), *tail),
                          "p3d_layer_norm_bwd")
        else:
            # bound to a name: a temporary whose pointer alone is passed could be freed before the launch
            dres = dres.to(x.dtype).contiguous()
            _native.check(lib.p3d_layer_norm_bwd_residual(_native.ptr(x), _native.ptr(weight), _native.ptr(dy),
                                                          _native.ptr(dres), *tail), "p3d_layer_norm_bwd_residual")
    return dx, dw.to(weight.dtype), db.to(weight.dtype), None


class _LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        return _ln_forward(ctx, x, weight, bias, eps)[1]

    @staticmethod
    @once_differentiable
    def backward(ctx, dy):
        return _ln_backward(ctx, dy)


def layer_norm(x, norm):
    """``norm(x)`` for an ``nn.LayerNorm`` over the last dimension, in the library kernels."""
    return _LayerNorm.apply(x, norm.weight, norm.bias, norm.eps)


class _LayerNormResidual(torch.autograd.Function):
    """``(norm(x), x)``: the second output is x itself, which the layer's outer residual
    (``attention.py:89``) reads, so both gradients of x arrive in one backward call and
    ``p3d_layer_norm_bwd_residual`` adds the residual's into the LayerNorm's dx in the same pass
    -- the bits autograd's separate add of the two would give, one elementwise pass fewer."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        ctx.set_materialize_grads(False)
        xc, y = _ln_forward(ctx, x, weight, bias, eps)
        return y, xc

    @staticmethod
    @once_differentiable
    def backward(ctx, dy, dres):
        if dy is None:
            return (None if dres is None else dres), None, None, None
        return _ln_backward(ctx, dy, dres)


def layer_norm_residual(x, norm):
    """``(norm(x), x)`` with the two gradients of x summed inside the LayerNorm backward kernel;
    the second output is the residual operand of the layer's output GEMM."""
    return _LayerNormResidual.apply(x, norm.weight, norm.bias, norm.eps)


class _QKVSplit(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qp, kvp, coords, phases, pairs, extents, heads, kv_heads, head_dim):
        b, n = qp.shape[0], qp.shape[1]
        qp, kvp = qp.contiguous(), kvp.contiguous()
        dev, dt = qp.device, qp.dtype
        q = torch.empty((b, heads, n, head_dim), dtype=dt, device=dev)
        kl, vl, kg, vg = (torch.empty((b, kv_heads, n, head_dim), dtype=dt, device=dev) for _ in range(4))
        with torch.cuda.device(dev):
            _native.check(_native.lib().p3d_qkv_split(
                _native.ptr(qp), _native.ptr(kvp), _native.ptr(q), _native.ptr(kl), _native.ptr(vl), _native.ptr(kg),
                _native.ptr(vg), _native.DTYPE_CODE[dt], b, heads, kv_heads, n, head_dim, _native.ptr(coords), *pairs,
                _native.ptr(phases), *extents, 0, _native.stream_of(dev)), "p3d_qkv_split")
        ctx.save_for_backward(coords, phases)
        ctx.meta = (pairs, extents, heads, kv_heads, head_dim, b, n, dt)
        return q, kl, vl, kg, vg

    @staticmethod
    @once_differentiable
    def backward(ctx, dq, dkl, dvl, dkg, dvg):
        coords, phases = ctx.saved_tensors
        pairs, extents, heads, kv_heads, head_dim, b, n, dt = ctx.meta
        dqp, dkvp = _merge(dq, dkl, dvl, dkg, dvg, coords, phases, pairs, extents, heads, kv_heads, head_dim, b, n,
                           dt)
        return dqp, dkvp, None, None, None, None, None, None, None


def qkv_split(qp, kvp, coords, phases, pairs, extents, heads, kv_heads, head_dim):
    """Differentiable ``p3d_qkv_split``: ``(q, kl, vl, kg, vg)`` head-major, q / kl / kg rotated.

    ``coords`` int64 ``[N, 3]`` and ``phases`` (the RoPE table of ``rope.phase_tables``) on the
    projections' device."""
    return _QKVSplit.apply(qp, kvp, coords, phases, tuple(int(p) for p in pairs), tuple(int(e) for e in extents),
                           int(heads), int(kv_heads), int(head_dim))


def _merge(dq, dkl, dvl, dkg, dvg, coords, phases, pairs, extents, heads, kv_heads, head_dim, b, n, dt):
    """``p3d_qkv_merge``: head-major gradients -> the projection gradients (dqp, dkvp)."""
    dev = coords.device

    def grad(t, h):
        if t is None:
            return torch.zeros((b, h, n, head_dim), dtype=dt, device=dev)
        return t.to(dt).contiguous()

    dq = grad(dq, heads)
    dkl, dvl, dkg, dvg = (grad(t, kv_heads) for t in (dkl, dvl, dkg, dvg))
    dqp = torch.empty((b, n, heads * head_dim), dtype=dt, device=dev)
    dkvp = torch.empty((b, n, 4 * kv_heads * head_dim), dtype=dt, device=dev)
    with torch.cuda.device(dev):
        _native.check(_native.lib().p3d_qkv_merge(
            _native.ptr(dq), _native.ptr(dkl), _native.ptr(dvl), _native.ptr(dkg), _native.ptr(dvg),
            _native.ptr(dqp), _native.ptr(dkvp), _native.DTYPE_CODE[dt], b, heads, kv_heads, n, head_dim,
            _native.ptr(coords), *pairs, _native.ptr(phases), *extents, _native.stream_of(dev)), "p3d_qkv_merge")
    return dqp, dkvp


def project_supported(x, wq, wkv, heads, kv_heads, head_dim):
    """Whether ``p3d_qkv_project`` runs this shape (16-bit, contiguous 16-byte-aligned weights)."""
    if x.dtype not in (torch.bfloat16, torch.float16) or not x.is_cuda:
        return False
    if not (wq.is_contiguous() and wkv.is_contiguous() and wq.dtype == x.dtype and wkv.dtype == x.dtype):
        return False
    if wq.data_ptr() % 16 or wkv.data_ptr() % 16:
        return False
    with torch.cuda.device(x.device):
        return bool(_native.lib().p3d_qkv_project_supported(_native.DTYPE_CODE[x.dtype], x.shape[-1], heads,
                                                            kv_heads, head_dim))


def gate_project_supported(x, wg, bg, heads, kv_heads, head_dim):
    """Whether ``p3d_qkv_gate_project`` folds this gate Linear (weight ``wg``, bias ``bg``) into
    the fused projection (project_supported must hold too)."""
    if not (wg.is_contiguous() and bg.is_contiguous() and wg.dtype == x.dtype and bg.dtype == x.dtype):
        return False
    if wg.data_ptr() % 16 or bg.data_ptr() % 2:
        return False
    with torch.cuda.device(x.device):
        return bool(_native.lib().p3d_qkv_gate_project_supported(_native.DTYPE_CODE[x.dtype], x.shape[-1], heads,
                                                                 kv_heads, head_dim))


def project_split_raw(x, wq, wkv, coords, phases, pairs, extents, heads, kv_heads, head_dim, raster_qkv=False,
                      kv_out=None, gate=None):
    """``p3d_qkv_project`` on x [B, N, dim] (no autograd): ``(q, kl, vl, kg, vg)``; ``raster_qkv``
    stores q, kl, vl at each token's raster row.  ``kv_out = (kl_ext, vl_ext, row0)`` writes kl
    and vl into rows ``[row0, row0 + N)`` of the given [B, G, rows, D] buffers (a z-slab rank's
    extended buffers) and returns those row ranges as kl, vl.  ``gate = (wg, bg)`` folds the gate
    Linear and its pair softmax in (``p3d_qkv_gate_project``) and appends the gate [B, H, N]."""
    b, n, dim = x.shape
    x = x.contiguous()
    dev, dt = x.device, x.dtype
    q = torch.empty((b, heads, n, head_dim), dtype=dt, device=dev)
    kg, vg = (torch.empty((b, kv_heads, n, head_dim), dtype=dt, device=dev) for _ in range(2))
    kv_rows = row0 = 0
    if kv_out is None:
        kl, vl = (torch.empty((b, kv_heads, n, head_dim), dtype=dt, device=dev) for _ in range(2))
        dst_k, dst_v = kl, vl
    else:
        dst_k, dst_v, row0 = kv_out
        want = (b, kv_heads, dst_k.shape[2], head_dim)
        if tuple(dst_k.shape) != want or tuple(dst_v.shape) != want or not (dst_k.is_contiguous() and
                                                                           dst_v.is_contiguous()):
            raise ValueError("kv_out buffers must be contiguous [B, G, rows, D]")
        kv_rows = dst_k.shape[2]
        kl, vl = dst_k[:, :, row0:row0 + n], dst_v[:, :, row0:row0 + n]
    tail = (_native.DTYPE_CODE[dt], b, heads, kv_heads, n, dim, head_dim, _native.ptr(coords), *pairs,
            _native.ptr(phases), *extents, kv_rows, row0, _native.SPLIT_RASTER_QKV if raster_qkv else 0,
            _native.stream_of(dev))
    with torch.cuda.device(dev):
        if gate is None:
            _native.check(_native.lib().p3d_qkv_project(
                _native.ptr(x), _native.ptr(wq), _native.ptr(wkv), _native.ptr(q), _native.ptr(dst_k),
                _native.ptr(dst_v), _native.ptr(kg), _native.ptr(vg), *tail), "p3d_qkv_project")
            return q, kl, vl, kg, vg
        wg, bg = gate
        g = torch.empty((b, heads, n), dtype=dt, device=dev)
        _native.check(_native.lib().p3d_qkv_gate_project(
            _native.ptr(x), _native.ptr(wq), _native.ptr(wkv), _native.ptr(wg), _native.ptr(bg), _native.ptr(q),
            _native.ptr(dst_k), _native.ptr(dst_v), _native.ptr(kg), _native.ptr(vg), _native.ptr(g), *tail),
            "p3d_qkv_gate_project")
    return q, kl, vl, kg, vg, g


class _QKVProject(torch.autograd.Function):
    """The projections (to_q, to_kv: no bias) and the split in one kernel, and the gate logits
    (``x Wg^T + bg``) on the same input; backward: the merge, then dx = dqp Wq + dkvp Wkv +
    dgl Wg with each GEMM accumulating into the first one's output (no elementwise add of
    separate input gradients), and the weight gradients."""

    @staticmethod
    def forward(ctx, x, wq, wkv, wg, bg, coords, phases, pairs, extents, heads, kv_heads, head_dim):
        x = x.contiguous()
        outs = project_split_raw(x, wq, wkv, coords, phases, pairs, extents, heads, kv_heads, head_dim)
        b, n, dim = x.shape
        gl = torch.addmm(bg, x.view(b * n, dim), wg.t()).view(b, n, -1)
        ctx.save_for_backward(x, wq, wkv, wg, coords, phases)
        ctx.meta = (pairs, extents, heads, kv_heads, head_dim)
        return (*outs, gl)

    @staticmethod
    @once_differentiable
    def backward(ctx, dq, dkl, dvl, dkg, dvg, dgl):
        x, wq, wkv, wg, coords, phases = ctx.saved_tensors
        pairs, extents, heads, kv_heads, head_dim = ctx.meta
        b, n, dim = x.shape
        dqp, dkvp = _merge(dq, dkl, dvl, dkg, dvg, coords, phases, pairs, extents, heads, kv_heads, head_dim, b, n,
                           x.dtype)
        dqp2, dkvp2, x2 = dqp.view(b * n, -1), dkvp.view(b * n, -1), x.view(b * n, dim)
        dx = torch.mm(dqp2, wq).addmm_(dkvp2, wkv)
        dgl2 = dgl.reshape(b * n, -1) if dgl is not None else None
        if dgl2 is not None:
            dx.addmm_(dgl2, wg)
        need = ctx.needs_input_grad
        dwq = torch.mm(dqp2.t(), x2) if need[1] else None
        dwkv = torch.mm(dkvp2.t(), x2) if need[2] else None
        dwg = torch.mm(dgl2.t(), x2) if dgl2 is not None and need[3] else None
        dbg = dgl2.sum(0) if dgl2 is not None and need[4] else None
        return dx.view(b, n, dim), dwq, dwkv, dwg, dbg, None, None, None, None, None, None, None


def qkv_project(x, wq, wkv, wg, bg, coords, phases, pairs, extents, heads, kv_heads, head_dim):
    """Differentiable ``x -> (x Wq^T, x Wkv^T) -> split`` and the gate logits ``x Wg^T + bg``:
    ``(q, kl, vl, kg, vg, gate_logits)``, the split head-major with q / kl / kg rotated,
    through ``p3d_qkv_project`` (check ``project_supported`` first)."""
    return _QKVProject.apply(x, wq, wkv, wg, bg, coords, phases, tuple(int(p) for p in pairs),
                             tuple(int(e) for e in extents), int(heads), int(kv_heads), int(head_dim))


class _Projections(torch.autograd.Function):
    """``x Wq^T``, ``x Wkv^T`` and ``x Wg^T + bg`` (to_q, to_kv, gate) on one input, whose
    gradient is accumulated by the GEMMs themselves (dx = dqp Wq, then += dkvp Wkv and
    += dgl Wg in place) instead of by two elementwise adds of three separate gradients."""

    @staticmethod
    def forward(ctx, x, wq, wkv, wg, bg):
        b, n, dim = x.shape
        x2 = x.reshape(b * n, dim)
        qp = torch.mm(x2, wq.t()).view(b, n, -1)
        kvp = torch.mm(x2, wkv.t()).view(b, n, -1)
        gl = torch.addmm(bg, x2, wg.t()).view(b, n, -1)
        ctx.save_for_backward(x, wq, wkv, wg)
        return qp, kvp, gl

    @staticmethod
    @once_differentiable
    def backward(ctx, dqp, dkvp, dgl):
        x, wq, wkv, wg = ctx.saved_tensors
        b, n, dim = x.shape
        x2 = x.reshape(b * n, dim)
        grads = [(t.reshape(b * n, -1) if t is not None else None, w) for t, w in ((dqp, wq), (dkvp, wkv), (dgl, wg))]
        dx = None
        for g, w in grads:
            if g is None:
                continue
            dx = torch.mm(g, w) if dx is None else dx.addmm_(g, w)
        if dx is None:
            dx = torch.zeros_like(x2)
        dw = [torch.mm(g.t(), x2) if g is not None and ctx.needs_input_grad[i + 1] else None
              for i, (g, _) in enumerate(grads)]
        dbg = grads[2][0].sum(0) if grads[2][0] is not None and ctx.needs_input_grad[4] else None
        return dx.view(b, n, dim), dw[0], dw[1], dw[2], dbg


def projections(x, to_q, to_kv, gate):
    """``(to_q(x), to_kv(x), gate(x))`` for bias-free to_q / to_kv and a biased gate, with the
    input gradient accumulated inside the GEMMs."""
    return _Projections.apply(x, to_q.weight, to_kv.weight, gate.weight, gate.bias)
