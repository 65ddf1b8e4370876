"""The PACK3D attention layer with the B200 backend.

Same constructor, parameters (and therefore state-dict names) and forward as
the reference's ``src/pack3d/attention.py:12-89``: LayerNorm, Q and 4-way KV
projections (cuBLAS through PyTorch), axial or packed-sequence RoPE of q /
local k / global k, the 2-way gate softmax, the core, the output projection
and the outer residual.  RoPE and the core run in ``libpack3d_b200.so``.
The only backend is ``"b200"``: an explicit request that never falls back.
"""
import math

import torch
from torch import nn

from ._validation import HEAD_DIMS, check_cuda
from .geometry import TokenLayout
from .ops import pack3d_streamed, pack3d_token_major
from . import glue
from .rope import balanced_pairs, phase_tables, rotate_projections


class PACK3DAttention(nn.Module):
    """Local residual plus gated compressed attention and an outer residual.

    Input / output ``[batch, packed_tokens, dim]``; the layout travels with the
    tokens.  Separate local / global K/V projections, one learned fine atom,
    two-stage compression.

    Two attributes choose between equivalent implementations; both paths compute the same
    layer within the bf16 tolerance:

    * ``fused_glue`` (default True): 16-bit CUDA calls run LayerNorm, the projection split
      with its RoPE, and their backward halves in the library's kernels, and feed the core's
      token-major output to ``to_out`` together with the residual in one GEMM.  False keeps
      the per-op PyTorch path.
    * ``fused_projection`` (default True): with ``fused_glue``, run the two projections and
      the split with its RoPE in one tensor-core kernel (``p3d_qkv_project``) where it
      supports the shape (16-bit, dim a multiple of 64); the projections never reach HBM.
      False runs cuBLAS GEMMs and the split kernel instead.
    """

    def __init__(self, dim, *, heads=4, kv_heads=2, head_dim=32, block_volume=8, backend="b200",
                 position_encoding="axial", temperature=1.0):
        super().__init__()
        if any(type(v) is not int or v <= 0 for v in (dim, heads, kv_heads, head_dim, block_volume)):
            raise ValueError("dimensions must be positive integers")
        if heads % kv_heads or head_dim not in HEAD_DIMS or block_volume > 64:
            raise ValueError("unsupported grouped-head dimensions or block volume")
        if backend != "b200":
            raise ValueError("backend must be explicitly b200")
        if position_encoding not in ("axial", "packed"):
            raise ValueError("position_encoding must be axial or packed")
        if not math.isfinite(temperature) or temperature <= 0:
            raise ValueError("temperature must be finite and positive")
        self.dim, self.heads, self.kv_heads, self.head_dim = dim, heads, kv_heads, head_dim
        self.backend, self.position_encoding = backend, position_encoding
        self.temperature = float(temperature)
        self.norm = nn.LayerNorm(dim)
        self.to_q = nn.Linear(dim, heads * head_dim, bias=False)
        self.to_kv = nn.Linear(dim, 4 * kv_heads * head_dim, bias=False)
        self.pool_weight = nn.Parameter(torch.empty(head_dim))
        nn.init.uniform_(self.pool_weight, -1 / math.sqrt(head_dim), 1 / math.sqrt(head_dim))
        self.slot_bias = nn.Parameter(torch.empty(block_volume))
        nn.init.normal_(self.slot_bias, std=0.02)
        self.gate = nn.Linear(dim, heads * 2)
        nn.init.zeros_(self.gate.bias)
        self.local_scale = nn.Parameter(torch.ones(head_dim))
        self.global_scale = nn.Parameter(torch.full((head_dim,), 0.25))
        self.to_out = nn.Linear(heads * head_dim, dim, bias=False)
        # 16-bit CUDA training calls run LayerNorm and the projection split (with RoPE) in the
        # fused library kernels of pack3d_b200.glue; False keeps the per-op PyTorch path.
        self.fused_glue = True
        # p3d_qkv_project (projections + split + RoPE in one tensor-core kernel, the projections
        # never written to HBM) where it supports the shape: 0.22 ms at config 1 against 0.36 ms
        # for the stacked cuBLAS GEMM and p3d_qkv_gate_split; False keeps the latter
        self.fused_projection = True

    def forward(self, x, layout: TokenLayout):
        layout.check_unmodified()
        if x.ndim != 3 or x.shape[0] == 0 or x.shape[1:] != (layout.geometry.num_tokens, self.dim):
            raise ValueError("x must be [batch,layout_tokens,dim] with a nonempty batch")
        if x.device != layout.coords.device:
            raise ValueError("x and layout are on different devices; move both with .to(device)")
        if layout.geometry.blocks.shape[1] != len(self.slot_bias):
            raise ValueError("layout canonical slot count must match block_volume")
        if self.backend != "b200":
            raise ValueError("unknown backend; implicit fallback is disabled")
        residual, b, n = x, x.shape[0], x.shape[1]
        if self._fast_inference(x):
            return self._forward_inference(x, layout)
        packed = self.position_encoding == "packed"
        pairs = (self.head_dim // 2, 0, 0) if packed else balanced_pairs(self.head_dim)
        phases = self._fused_glue_table(x, layout, pairs)
        if phases is not None:
            # the fused training glue: LayerNorm and the projection split (with RoPE) and their
            # backward halves in the library kernels (pack3d_b200.glue)
            # the residual operand is the LayerNorm's second output: both gradients of x meet in
            # one backward kernel (p3d_layer_norm_bwd_residual) instead of an extra add
            x, residual = glue.layer_norm_residual(x, self.norm)
            coords = layout.coords.to(device=x.device, dtype=torch.int64).contiguous()
            if self.fused_projection and glue.project_supported(x, self.to_q.weight, self.to_kv.weight, self.heads,
                                                                self.kv_heads, self.head_dim):
                q, kl, vl, kg, vg, gate_logits = glue.qkv_project(x, self.to_q.weight, self.to_kv.weight,
                                                                  self.gate.weight, self.gate.bias, coords, phases,
                                                                  pairs, layout.grid_shape, self.heads,
                                                                  self.kv_heads, self.head_dim)
            else:
                qp, kvp, gate_logits = glue.projections(x, self.to_q, self.to_kv, self.gate)
                q, kl, vl, kg, vg = glue.qkv_split(qp, kvp, coords, phases, pairs,
                                                   layout.grid_shape, self.heads, self.kv_heads, self.head_dim)
        else:
            x = self.norm(x)
            q = self.to_q(x).reshape(b, n, self.heads, self.head_dim).transpose(1, 2)
            kl, vl, kg, vg = (t.reshape(b, n, self.kv_heads, self.head_dim).transpose(1, 2)
                              for t in self.to_kv(x).chunk(4, -1))
            check_cuda(q)
            q, kl, kg = rotate_projections(q, kl, kg, layout.coords, pairs, layout.grid_shape, packed=packed)
        if phases is None:
            gate_logits = self.gate(x)
        gates = gate_logits.reshape(b, n, self.heads, 2).softmax(-1)
        gate = gates[..., 1].transpose(1, 2)
        if phases is not None:
            # token-major core output: to_out reads it, and takes the residual, in one GEMM
            out = pack3d_token_major(q, kl, vl, kg, vg, self.pool_weight, self.slot_bias, gate, self.local_scale,
                                     self.global_scale, layout.geometry, temperature=self.temperature)
            return self._out_residual(residual, out)
        out = pack3d_streamed(q, kl, vl, kg, vg, self.pool_weight, self.slot_bias, gate, self.local_scale,
                              self.global_scale, layout.geometry, temperature=self.temperature)
        return residual + self.to_out(out.transpose(1, 2).reshape(b, n, -1))

    def _fused_glue_table(self, x, layout, pairs):
        """The RoPE phase table when the fused training glue applies (16-bit CUDA tensors of
        the layer's dtype, axial RoPE, 16-byte rows), else None."""
        if not (self.fused_glue and x.is_cuda and x.dtype in (torch.bfloat16, torch.float16)
                and self.position_encoding == "axial" and self.dim % 8 == 0 and self.head_dim % 8 == 0
                and all(p.dtype == x.dtype for p in self.parameters())):
            return None
        _, phases = phase_tables(x.device, pairs, tuple(int(e) for e in layout.grid_shape))
        return phases

    def _fast_inference(self, x):
        """Gradient-free 16-bit axial calls take the fused glue path (same arithmetic)."""
        return (not torch.is_grad_enabled() or not (x.requires_grad or any(p.requires_grad for p in self.parameters()))) \
            and x.dtype in (torch.bfloat16, torch.float16) and self.position_encoding == "axial" \
            and x.is_cuda and self.dim % 8 == 0 and self.head_dim % 8 == 0 \
            and all(p.dtype == x.dtype for p in self.parameters())

    def _forward_inference(self, x, layout):
        """The same layer as :meth:`forward` with the glue fused into library kernels.

        LayerNorm runs in ``p3d_layer_norm``; one ``p3d_qkv_split`` pass turns the two
        projection outputs into rotated q / kl / kg and head-major vl / vg; the core writes
        its output token-major so the output projection reads it without a transpose copy.
        """
        from .ops import forward as core_forward, raster_qkv_applies
        # permuted storage (Morton blocks): the split writes q, kl, vl at raster rows, so the
        # tensor-core stencil kernel reads them without a gather pass
        extents = tuple(int(e) for e in layout.grid_shape)
        raster = (phase_tables(x.device, balanced_pairs(self.head_dim), extents)[1] is not None
                  and raster_qkv_applies(layout.geometry, x.dtype, self.head_dim, x.device))
        x, q, kl, vl, kg, vg, gate = self._inference_glue(x, layout.coords, layout.grid_shape, raster_qkv=raster)
        w32, b32, sl32, sg32 = self._core_params_f32()
        y, _ = core_forward(q, kl, vl, kg, vg, w32, b32, gate, sl32, sg32, layout.geometry, self.temperature,
                            save_state=False, y_rows=True, raster_qkv=raster)
        return self._out_residual(x, y)

    def _out_residual(self, x, y_rows):
        """``x + to_out(y)`` for a token-major core output, the residual added inside the GEMM."""
        b, n = x.shape[0], x.shape[1]
        out = torch.addmm(x.reshape(b * n, self.dim), y_rows.transpose(1, 2).reshape(b * n, -1), self.to_out.weight.t())
        return out.view(b, n, self.dim)

    def _inference_glue(self, x, coords, grid_shape, raster_qkv=False, kv_out=None):
        """LayerNorm, projections, RoPE at ``coords`` (extents ``grid_shape``) and the gate of
        the fused inference path: ``(x, q, kl, vl, kg, vg, gate)``, head-major.  ``raster_qkv``
        stores the rows of q, kl, vl at each token's raster index (the extents must be the
        token grid).  ``kv_out = (kl_ext, vl_ext, row0)``: kl and vl are rows
        ``[row0, row0 + N)`` of those [B, G, rows, D] buffers (a z-slab rank's extended
        buffers); the fused projection writes them there, the other forms copy them in."""
        glue_out = self._inference_glue_rows(x, coords, grid_shape, raster_qkv, kv_out)
        if kv_out is None or glue_out[2].data_ptr() == kv_out[0][:, :, kv_out[2]:].data_ptr():
            return glue_out
        x, q, kl, vl, kg, vg, gate = glue_out
        n = kl.shape[2]
        kl_ext, vl_ext, row0 = kv_out
        kl_ext[:, :, row0:row0 + n].copy_(kl)
        vl_ext[:, :, row0:row0 + n].copy_(vl)
        return x, q, kl_ext[:, :, row0:row0 + n], vl_ext[:, :, row0:row0 + n], kg, vg, gate

    def _inference_glue_rows(self, x, coords, grid_shape, raster_qkv, kv_out):
        from . import _native
        from .rope import phase_tables
        b, n = x.shape[0], x.shape[1]
        h, g, d = self.heads, self.kv_heads, self.head_dim
        x = x.contiguous()
        xn = torch.empty_like(x)
        dev = x.device
        code = _native.DTYPE_CODE[x.dtype]
        lib = _native.lib()
        stream = _native.stream_of(dev)
        with torch.cuda.device(dev):
            _native.check(lib.p3d_layer_norm(_native.ptr(x), _native.ptr(self.norm.weight), _native.ptr(self.norm.bias),
                                             _native.ptr(xn), code, b * n, self.dim, float(self.norm.eps), stream),
                          "p3d_layer_norm")
        pairs = balanced_pairs(d)
        extents = tuple(int(e) for e in grid_shape)
        _, phases = phase_tables(dev, pairs, extents)
        if raster_qkv and phases is None:
            raise ValueError("raster-ordered q, kl, vl need a phase table")
        if phases is not None and self.fused_projection and glue.project_supported(xn, self.to_q.weight,
                                                                                  self.to_kv.weight, h, g, d):
            # projections, split and RoPE in one kernel: the projections never reach HBM; the
            # gate folded in (its logit rows beside the first q group's), or else from its own
            # GEMM and p3d_gate_pairs
            coords = coords.to(device=dev, dtype=torch.int64).contiguous()
            if glue.gate_project_supported(xn, self.gate.weight, self.gate.bias, h, g, d):
                return (x, *glue.project_split_raw(xn, self.to_q.weight, self.to_kv.weight, coords, phases, pairs,
                                                   extents, h, g, d, raster_qkv=raster_qkv, kv_out=kv_out,
                                                   gate=(self.gate.weight, self.gate.bias)))
            q, kl, vl, kg, vg = glue.project_split_raw(xn, self.to_q.weight, self.to_kv.weight, coords, phases, pairs,
                                                       extents, h, g, d, raster_qkv=raster_qkv, kv_out=kv_out)
            logits = torch.addmm(self.gate.bias, xn.view(b * n, self.dim), self.gate.weight.t())
            gate = torch.empty((b, h, n), dtype=x.dtype, device=dev)
            with torch.cuda.device(dev):
                _native.check(lib.p3d_gate_pairs(_native.ptr(logits), logits.shape[1], _native.ptr(gate), code, b, h,
                                                 n, stream), "p3d_gate_pairs")
            return x, q, kl, vl, kg, vg, gate
        if phases is not None and h <= 16:
            # one GEMM for to_q, to_kv and gate (weights stacked, gate bias in the epilogue); one
            # pass splits, rotates and forms the gate (p3d_qkv_gate_split, up to 16 heads)
            w, bias = self._stacked_projection(x.dtype, dev)
            proj = torch.addmm(bias, xn.view(b * n, self.dim), w.t())
            qp = kvp = None
        else:
            qp, kvp = self.to_q(xn), self.to_kv(xn)
        if phases is None:   # coordinate extents too large for a table: the general RoPE path
            q, kl, kg = rotate_projections(qp.reshape(b, n, h, d).transpose(1, 2),
                                           *(t.reshape(b, n, g, d).transpose(1, 2) for t in kvp.chunk(4, -1)[0::2]),
                                           coords, pairs, extents, packed=False)
            vl, vg = (t.reshape(b, n, g, d).transpose(1, 2).contiguous() for t in kvp.chunk(4, -1)[1::2])
        elif qp is None:
            coords = coords.to(device=dev, dtype=torch.int64).contiguous()
            q = torch.empty((b, h, n, d), dtype=x.dtype, device=dev)
            kl, vl, kg, vg = (torch.empty((b, g, n, d), dtype=x.dtype, device=dev) for _ in range(4))
            gate = torch.empty((b, h, n), dtype=x.dtype, device=dev)
            with torch.cuda.device(dev):
                _native.check(lib.p3d_qkv_gate_split(_native.ptr(proj), proj.shape[1], _native.ptr(q), _native.ptr(kl),
                                                     _native.ptr(vl), _native.ptr(kg), _native.ptr(vg),
                                                     _native.ptr(gate), code, b, h, g, n, d, _native.ptr(coords),
                                                     *pairs, _native.ptr(phases), *extents,
                                                     _native.SPLIT_RASTER_QKV if raster_qkv else 0, stream),
                              "p3d_qkv_gate_split")
            return x, q, kl, vl, kg, vg, gate
        else:
            coords = coords.to(device=dev, dtype=torch.int64).contiguous()
            q = torch.empty((b, h, n, d), dtype=x.dtype, device=dev)
            kl, vl, kg, vg = (torch.empty((b, g, n, d), dtype=x.dtype, device=dev) for _ in range(4))
            with torch.cuda.device(dev):
                _native.check(lib.p3d_qkv_split(_native.ptr(qp), _native.ptr(kvp), _native.ptr(q), _native.ptr(kl),
                                                _native.ptr(vl), _native.ptr(kg), _native.ptr(vg), code, b, h, g, n, d,
                                                _native.ptr(coords), *pairs, _native.ptr(phases), *extents,
                                                _native.SPLIT_RASTER_QKV if raster_qkv else 0, stream),
                              "p3d_qkv_split")
        gate = self.gate(xn).reshape(b, n, h, 2).softmax(-1)[..., 1].transpose(1, 2).contiguous()
        return x, q, kl, vl, kg, vg, gate

    def _core_params_f32(self):
        """``(pool_weight, slot_bias, local_scale, global_scale)`` in fp32, as the core's kernels
        take them, cached until any of them changes (inference calls would otherwise convert
        them on every call)."""
        params = (self.pool_weight, self.slot_bias, self.local_scale, self.global_scale)
        key = tuple((t.data_ptr(), t._version, t.device) for t in params)
        hit = getattr(self, "_params_f32", None)
        if hit is None or hit[0] != key:
            with torch.inference_mode(False), torch.no_grad():
                hit = (key, tuple(t.detach().to(torch.float32).contiguous() for t in params))
            self._params_f32 = hit
        return hit[1]

    def _stacked_projection(self, dtype, device):
        """``(W, bias)``: the to_q, to_kv and gate weights stacked row-wise (zero rows pad the
        count to a multiple of 8) and the matching bias (zero, zero, gate bias), cached until
        any of those parameters changes."""
        params = (self.to_q.weight, self.to_kv.weight, self.gate.weight, self.gate.bias)
        key = (dtype, device) + tuple((t.data_ptr(), t._version) for t in params)
        hit = getattr(self, "_stacked", None)
        if hit is not None and hit[0] == key:
            return hit[1], hit[2]
        with torch.inference_mode(False), torch.no_grad():
            rows = self.to_q.weight.shape[0] + self.to_kv.weight.shape[0] + self.gate.weight.shape[0]
            pad = -rows % 8
            w = torch.cat([self.to_q.weight, self.to_kv.weight, self.gate.weight,
                           self.gate.weight.new_zeros(pad, self.dim)]).to(device=device, dtype=dtype).contiguous()
            bias = torch.cat([self.gate.bias.new_zeros(self.to_q.weight.shape[0] + self.to_kv.weight.shape[0]),
                              self.gate.bias, self.gate.bias.new_zeros(pad)]).to(device=device, dtype=dtype)
        self._stacked = (key, w, bias)
        return w, bias
