"""The fused layer glue of the inference path: p3d_qkv_split, p3d_layer_norm, token-major y."""
import pytest
import torch

from pack3d_b200 import PACK3DAttention, _native, build_layout
from pack3d_b200 import ops as p3d_ops
from pack3d_b200.rope import balanced_pairs, phase_tables, rotate_projections

pytestmark = pytest.mark.gpu


def _layout(grid, raster=True):
    layout = build_layout(grid, (4, 4, 4), radius=2, pool_size=1)
    return layout.repack(layout.order.argsort()) if raster else layout


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("h,g,d", [(4, 4, 48), (4, 2, 32), (2, 1, 16), (2, 2, 64), (3, 1, 128), (6, 3, 48)])
def test_qkv_split_matches_rotation_and_copies(cuda_device, dtype, h, g, d):
    layout = _layout((8, 12, 16), raster=False).to(cuda_device)
    b, n = 2, layout.geometry.num_tokens
    gen = torch.Generator(device=cuda_device).manual_seed(h + g + d)
    qp = torch.randn(b, n, h * d, device=cuda_device, generator=gen).to(dtype)
    kvp = torch.randn(b, n, 4 * g * d, device=cuda_device, generator=gen).to(dtype)
    pairs = balanced_pairs(d)
    extents = layout.grid_shape
    _, phases = phase_tables(cuda_device, pairs, extents)
    outs = [torch.empty((b, h, n, d), dtype=dtype, device=cuda_device)]
    outs += [torch.empty((b, g, n, d), dtype=dtype, device=cuda_device) for _ in range(4)]
    coords = layout.coords.contiguous()
    with torch.cuda.device(cuda_device):
        _native.check(_native.lib().p3d_qkv_split(
            _native.ptr(qp), _native.ptr(kvp), *[_native.ptr(t) for t in outs], _native.DTYPE_CODE[dtype], b, h, g, n,
            d, _native.ptr(coords), *pairs, _native.ptr(phases), *extents, 0, _native.stream_of(cuda_device)),
            "p3d_qkv_split")
    q, kl, vl, kg, vg = outs
    chunks = [t.reshape(b, n, g, d).transpose(1, 2) for t in kvp.chunk(4, -1)]
    wq, wkl, wkg = rotate_projections(qp.reshape(b, n, h, d).transpose(1, 2), chunks[0], chunks[2], layout.coords,
                                      pairs, extents, packed=False)
    assert torch.equal(q, wq) and torch.equal(kl, wkl) and torch.equal(kg, wkg)
    assert torch.equal(vl, chunks[1].contiguous()) and torch.equal(vg, chunks[3].contiguous())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("h,g,d", [(4, 4, 48), (2, 1, 32)])
def test_qkv_split_raster_rows_are_the_token_rows_permuted(cuda_device, dtype, h, g, d):
    """SPLIT_RASTER_QKV puts each token's q, kl, vl at its raster index and leaves kg, vg in
    token order: the same values as the plain split, with q, kl, vl rows permuted."""
    layout = _layout((8, 12, 16), raster=False).to(cuda_device)
    b, n = 2, layout.geometry.num_tokens
    gen = torch.Generator(device=cuda_device).manual_seed(7 * h + d)
    qp = torch.randn(b, n, h * d, device=cuda_device, generator=gen).to(dtype)
    kvp = torch.randn(b, n, 4 * g * d, device=cuda_device, generator=gen).to(dtype)
    pairs = balanced_pairs(d)
    extents = layout.grid_shape
    _, phases = phase_tables(cuda_device, pairs, extents)
    coords = layout.coords.contiguous()
    results = []
    for flags in (0, _native.SPLIT_RASTER_QKV):
        outs = [torch.empty((b, h, n, d), dtype=dtype, device=cuda_device)]
        outs += [torch.empty((b, g, n, d), dtype=dtype, device=cuda_device) for _ in range(4)]
        with torch.cuda.device(cuda_device):
            _native.check(_native.lib().p3d_qkv_split(
                _native.ptr(qp), _native.ptr(kvp), *[_native.ptr(t) for t in outs], _native.DTYPE_CODE[dtype], b, h,
                g, n, d, _native.ptr(coords), *pairs, _native.ptr(phases), *extents, flags,
                _native.stream_of(cuda_device)), "p3d_qkv_split")
        results.append(outs)
    plain, raster = results
    c = coords
    row = (c[:, 0] * extents[1] + c[:, 1]) * extents[2] + c[:, 2]      # raster index of token row i
    for i, name in enumerate(("q", "kl", "vl")):
        assert torch.equal(raster[i][:, :, row], plain[i]), name
    for i, name in ((3, "kg"), (4, "vg")):
        assert torch.equal(raster[i], plain[i]), name
    # the raster form needs the extents to be the token grid
    with pytest.raises(ValueError, match="token grid"):
        _native.check(_native.lib().p3d_qkv_split(
            _native.ptr(qp), _native.ptr(kvp), *[_native.ptr(t) for t in plain], _native.DTYPE_CODE[dtype], b, h, g,
            n, d, _native.ptr(coords), *pairs, _native.ptr(phases), extents[0] + 1, extents[1], extents[2],
            _native.SPLIT_RASTER_QKV, _native.stream_of(cuda_device)), "p3d_qkv_split")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("h,g,d", [(4, 4, 48), (3, 1, 32), (2, 2, 64)])
def test_qkv_gate_split_matches_the_split_and_the_torch_gate(cuda_device, dtype, h, g, d):
    """p3d_qkv_gate_split on one stacked projection buffer (q, kv, gate logits, padding columns)
    gives the split's q .. vg bit for bit and the layer's gate (softmax over each logit pair,
    second entry) as torch computes it."""
    layout = _layout((8, 12, 16), raster=False).to(cuda_device)
    b, n = 2, layout.geometry.num_tokens
    gen = torch.Generator(device=cuda_device).manual_seed(31 * h + d)
    used = (h + 4 * g) * d + 2 * h
    cols = used + (-used % 8) + 8  # padding columns beyond the ones the kernel reads
    proj = (torch.randn(b, n, cols, device=cuda_device, generator=gen) * 2).to(dtype)
    qp, kvp = proj[..., :h * d].contiguous(), proj[..., h * d:(h + 4 * g) * d].contiguous()
    logits = proj[..., (h + 4 * g) * d:used]
    pairs = balanced_pairs(d)
    extents = layout.grid_shape
    _, phases = phase_tables(cuda_device, pairs, extents)
    coords = layout.coords.contiguous()
    lib = _native.lib()
    want = [torch.empty((b, h, n, d), dtype=dtype, device=cuda_device)]
    want += [torch.empty((b, g, n, d), dtype=dtype, device=cuda_device) for _ in range(4)]
    got = [torch.empty_like(t) for t in want]
    gate = torch.empty((b, h, n), dtype=dtype, device=cuda_device)
    code, stream = _native.DTYPE_CODE[dtype], _native.stream_of(cuda_device)
    with torch.cuda.device(cuda_device):
        _native.check(lib.p3d_qkv_split(_native.ptr(qp), _native.ptr(kvp), *[_native.ptr(t) for t in want], code, b,
                                        h, g, n, d, _native.ptr(coords), *pairs, _native.ptr(phases), *extents, 0,
                                        stream), "p3d_qkv_split")
        _native.check(lib.p3d_qkv_gate_split(_native.ptr(proj), cols, *[_native.ptr(t) for t in got],
                                             _native.ptr(gate), code, b, h, g, n, d, _native.ptr(coords), *pairs,
                                             _native.ptr(phases), *extents, 0, stream), "p3d_qkv_gate_split")
    for name, w, o in zip(("q", "kl", "vl", "kg", "vg"), want, got):
        assert torch.equal(w, o), name
    want_gate = logits.reshape(b, n, h, 2).softmax(-1)[..., 1].transpose(1, 2)
    step = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    assert (gate.float() - want_gate.float()).abs().max().item() <= step, "gate"
    assert torch.equal(gate, want_gate) or (gate != want_gate).float().mean().item() < 1e-3
    # the column count must cover the projections and keep rows 16-byte aligned
    with pytest.raises(ValueError, match="proj_cols"):
        _native.check(lib.p3d_qkv_gate_split(_native.ptr(proj), used - 2, *[_native.ptr(t) for t in got],
                                             _native.ptr(gate), code, b, h, g, n, d, _native.ptr(coords), *pairs,
                                             _native.ptr(phases), *extents, 0, stream), "p3d_qkv_gate_split")


@pytest.mark.parametrize("dim", [192, 384, 64, 128, 256, 40])
def test_layer_norm_matches_torch(cuda_device, dim):
    # 64 k <= 256: segment layout (4 rows per warp pass; 2999 rows leave a ragged last group)
    gen = torch.Generator(device=cuda_device).manual_seed(dim)
    x = (torch.randn(1, 2999, dim, device=cuda_device, generator=gen) * 3 + 1).to(torch.bfloat16)
    norm = torch.nn.LayerNorm(dim).to(cuda_device, torch.bfloat16)
    with torch.no_grad():
        norm.weight.normal_()
        norm.bias.normal_()
    y = torch.empty_like(x)
    with torch.cuda.device(cuda_device):
        _native.check(_native.lib().p3d_layer_norm(_native.ptr(x), _native.ptr(norm.weight), _native.ptr(norm.bias),
                                                   _native.ptr(y), _native.BF16, 2999, dim, 1e-5,
                                                   _native.stream_of(cuda_device)), "p3d_layer_norm")
    want = norm(x)
    err = (y.float() - want.float()).abs()
    # one bf16 step of the larger magnitude at most
    assert (err <= 2.0 ** -7 * torch.maximum(y.float().abs(), want.float().abs()) + 1e-3).all()


@pytest.mark.parametrize("raster", [True, False])
def test_token_major_output_matches(cuda_device, raster):
    import oracle
    from cases import grid_inputs
    layout = _layout((8, 8, 16), raster)
    n = layout.geometry.num_tokens
    raw = grid_inputs(n, 2, 4, 4, 48, torch.float32, 4, True)
    rot = [oracle.axial_rope(raw[i], layout.coords) if i in (0, 1, 3) else raw[i] for i in range(5)]
    inputs = [t.to(torch.bfloat16).to(cuda_device) for t in rot] + [t.to(cuda_device) for t in raw[5:]]
    geom = layout.geometry.to(cuda_device)
    for force_indexed in (False, True):
        y, _ = p3d_ops.forward(*inputs, geom, 1.0, save_state=False, force_indexed=force_indexed)
        y_rows, _ = p3d_ops.forward(*inputs, geom, 1.0, save_state=False, force_indexed=force_indexed, y_rows=True)
        assert y_rows.shape == y.shape and y_rows.transpose(1, 2).is_contiguous()
        assert torch.equal(y_rows, y)


def test_fast_inference_layer_matches_the_autograd_path(cuda_device):
    layout = _layout((16, 16, 16)).to(cuda_device)
    torch.manual_seed(0)
    layer = PACK3DAttention(192, heads=4, kv_heads=4, head_dim=48, block_volume=64).to(cuda_device, torch.bfloat16)
    x = torch.randn(2, layout.geometry.num_tokens, 192, device=cuda_device).to(torch.bfloat16)
    with torch.no_grad():
        fast = layer(x, layout)
    slow = layer(x.clone().requires_grad_(), layout)
    with torch.no_grad():
        assert layer._fast_inference(x)
    assert not layer._fast_inference(x.clone().requires_grad_())
    assert (fast.float() - slow.detach().float()).abs().max().item() <= 2e-2 * max(1.0, slow.abs().max().item())
    assert _native.device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("h,g,d", [(4, 4, 48), (4, 2, 32), (8, 8, 48), (3, 1, 128), (2, 1, 16)])
def test_qkv_merge_is_the_exact_backward_of_the_split(cuda_device, dtype, h, g, d):
    from pack3d_b200 import glue
    from pack3d_b200.rope import _rotate
    layout = _layout((8, 12, 16), raster=False).to(cuda_device)
    b, n = 2, layout.geometry.num_tokens
    gen = torch.Generator(device=cuda_device).manual_seed(h + 3 * g + d)
    pairs = balanced_pairs(d)
    extents = layout.grid_shape
    _, phases = phase_tables(cuda_device, pairs, extents)
    coords = layout.coords.to(torch.int64).contiguous()
    grads = [torch.randn(b, h, n, d, device=cuda_device, generator=gen).to(dtype)]
    grads += [torch.randn(b, g, n, d, device=cuda_device, generator=gen).to(dtype) for _ in range(4)]
    qp = torch.randn(b, n, h * d, device=cuda_device, generator=gen).to(dtype).requires_grad_()
    kvp = torch.randn(b, n, 4 * g * d, device=cuda_device, generator=gen).to(dtype).requires_grad_()
    outs = glue.qkv_split(qp, kvp, coords, phases, pairs, extents, h, g, d)
    torch.autograd.backward(outs, grads)
    # the per-op backward: inverse rotation (p3d_rope), then the transposes and the concatenation
    inv = lambda t: _rotate(t, layout.coords, pairs, tuple(extents), False, inverse=True)  # noqa: E731
    dq, dkl, dvl, dkg, dvg = inv(grads[0]), inv(grads[1]), grads[2], inv(grads[3]), grads[4]
    want_q = dq.transpose(1, 2).reshape(b, n, h * d)
    want_kv = torch.cat([t.transpose(1, 2).reshape(b, n, g * d) for t in (dkl, dvl, dkg, dvg)], -1)
    assert torch.equal(qp.grad, want_q) and torch.equal(kvp.grad, want_kv)


@pytest.mark.parametrize("dim", [192, 384, 64, 128, 40])
def test_layer_norm_backward_matches_torch(cuda_device, dim):
    from pack3d_b200 import glue
    gen = torch.Generator(device=cuda_device).manual_seed(dim)
    x = (torch.randn(2, 2999, dim, device=cuda_device, generator=gen) * 2 + 0.5).to(torch.bfloat16)
    dy = torch.randn(2, 2999, dim, device=cuda_device, generator=gen).to(torch.bfloat16)
    norm = torch.nn.LayerNorm(dim).to(cuda_device, torch.bfloat16)
    with torch.no_grad():
        norm.weight.normal_()
        norm.bias.normal_()
    xa = x.clone().requires_grad_()
    glue.layer_norm(xa, norm).backward(dy)
    got = (xa.grad, norm.weight.grad.clone(), norm.bias.grad.clone())
    norm.zero_grad()
    # fp32 reference of the same op
    w32 = norm.weight.detach().float().requires_grad_()
    b32 = norm.bias.detach().float().requires_grad_()
    xc = x.float().requires_grad_()
    torch.nn.functional.layer_norm(xc, (dim,), w32, b32, norm.eps).backward(dy.float())
    want = (xc.grad, w32.grad, b32.grad)
    for g_, w_ in zip(got, want):
        tol = 2e-2 * max(1.0, w_.abs().max().item())
        assert (g_.float() - w_).abs().max().item() <= tol
    # fixed-order sums: a repeated backward is bitwise identical
    xa2 = x.clone().requires_grad_()
    norm.zero_grad()
    glue.layer_norm(xa2, norm).backward(dy)
    assert torch.equal(xa2.grad, got[0]) and torch.equal(norm.weight.grad, got[1])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dim", [192, 384, 40])
def test_layer_norm_residual_backward_is_the_two_step_sum(cuda_device, dtype, dim):
    """p3d_layer_norm_bwd_residual (through glue.layer_norm_residual feeding an addmm residual,
    as the layer does) gives the same bits as glue.layer_norm plus autograd's separate add."""
    from pack3d_b200 import glue
    gen = torch.Generator(device=cuda_device).manual_seed(dim + 7)
    x = (torch.randn(2, 1537, dim, device=cuda_device, generator=gen) * 2 + 0.5).to(dtype)
    m = torch.randn(2 * 1537, dim, device=cuda_device, generator=gen).to(dtype)
    w_out = (torch.randn(dim, dim, device=cuda_device, generator=gen) / dim ** 0.5).to(dtype)
    dy = torch.randn(2, 1537, dim, device=cuda_device, generator=gen).to(dtype)
    norm = torch.nn.LayerNorm(dim).to(cuda_device, dtype)
    with torch.no_grad():
        norm.weight.normal_()
        norm.bias.normal_()
    results = []
    for fused in (True, False):
        norm.zero_grad(set_to_none=True)
        xa = x.clone().requires_grad_()
        if fused:
            xn, res = glue.layer_norm_residual(xa, norm)
        else:
            xn, res = glue.layer_norm(xa, norm), xa
        y = torch.addmm(res.reshape(-1, dim), xn.reshape(-1, dim) * m, w_out.t()).view_as(x)
        y.backward(dy)
        results.append((y.detach(), xa.grad, norm.weight.grad.clone(), norm.bias.grad.clone()))
    for a, b in zip(*results):
        assert torch.equal(a, b)
    # the residual output alone (LayerNorm output unused): its gradient passes straight through
    xa = x.clone().requires_grad_()
    _, res = glue.layer_norm_residual(xa, norm)
    res.backward(dy)
    assert torch.equal(xa.grad, dy)
    assert _native.device_errors() == 0


def test_fused_training_glue_matches_the_per_op_path(cuda_device):
    layout = _layout((16, 16, 16)).to(cuda_device)
    torch.manual_seed(0)
    layer = PACK3DAttention(192, heads=4, kv_heads=4, head_dim=48, block_volume=64).to(cuda_device, torch.bfloat16)
    gen = torch.Generator(device=cuda_device).manual_seed(9)
    x = torch.randn(2, layout.geometry.num_tokens, 192, device=cuda_device, generator=gen).to(torch.bfloat16)
    dy = torch.randn_like(x)
    results = []
    for fused in (True, False):
        layer.fused_glue = fused
        layer.zero_grad(set_to_none=True)
        xi = x.clone().requires_grad_()
        y = layer(xi, layout)
        y.backward(dy)
        results.append((y.detach(), xi.grad, {k: p.grad.clone() for k, p in layer.named_parameters()}))
    (y0, dx0, g0), (y1, dx1, g1) = results
    tol = lambda t: 2e-2 * max(1.0, t.float().abs().max().item())  # noqa: E731
    assert (y0.float() - y1.float()).abs().max().item() <= tol(y1)
    assert (dx0.float() - dx1.float()).abs().max().item() <= tol(dx1)
    for k in g1:
        assert (g0[k].float() - g1[k].float()).abs().max().item() <= tol(g1[k]), k
    assert _native.device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gate_pairs_is_the_torch_gate(cuda_device, dtype):
    """p3d_gate_pairs: softmax over each head's logit pair, second entry, [B, H, N], from logits
    with a row stride wider than the pairs."""
    b, n, h, stride = 2, 777, 5, 16
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    logits = (torch.randn(b * n, stride, device=cuda_device, generator=gen) * 3).to(dtype)
    gate = torch.empty((b, h, n), dtype=dtype, device=cuda_device)
    with torch.cuda.device(cuda_device):
        _native.check(_native.lib().p3d_gate_pairs(_native.ptr(logits), stride, _native.ptr(gate),
                                                   _native.DTYPE_CODE[dtype], b, h, n, _native.stream_of(cuda_device)),
                      "p3d_gate_pairs")
    want = logits[:, :2 * h].reshape(b, n, h, 2).softmax(-1)[..., 1].transpose(1, 2)
    step = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    assert (gate.float() - want.float()).abs().max().item() <= step
    assert (gate != want).float().mean().item() < 1e-3
