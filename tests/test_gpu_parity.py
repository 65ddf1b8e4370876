"""GPU parity: the CUDA path against the oracle and the reference's golden vectors.

Tolerances: max-abs 1e-5 for fp32, 2e-2 for bf16
(outputs and gradients), and exact equality for RoPE with a phase table and
for repeated backward calls (determinism).
"""
import pytest
import torch

import oracle
from cases import CORE_CASES, GRID_CASES, graph_case, grid_inputs, upstream
from pack3d_b200 import (PACK3DAttention, TokenLayout, build_layout, pack3d_streamed, prepare_geometry,
                         rotate_projections)
from pack3d_b200 import ops as p3d_ops

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float64: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}
NAMES = ["q", "kl", "vl", "kg", "vg", "pool_weight", "slot_bias", "gate", "local_scale", "global_scale"]


def max_abs(a, b):
    return (a.detach().float().cpu() - b.detach().float().cpu()).abs().max().item()


def to_dev(ts, dev, dtype=None, grad=False):
    out = []
    for t in ts:
        t = t.to(dev) if dtype is None else t.to(dev, dtype)
        out.append(t.clone().requires_grad_(grad))
    return out


# ------------------------------------------------------------------------------ RoPE

@pytest.mark.parametrize("d", [16, 48, 64, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_is_bit_exact_with_table(cuda_device, d, dtype):
    grid = (5, 7, 9)
    layout = build_layout(grid, 1, radius=0, pool_size=1)
    coords = layout.coords
    x = torch.randn(2, 3 * 6, layout.geometry.num_tokens, d).to(dtype)
    # strided projection-style views: [B, N, heads*D] viewed as [B, heads, N, D]
    proj = x.transpose(1, 2).contiguous().to(cuda_device).transpose(1, 2)
    views = proj.split(6, dim=1)
    got = rotate_projections(*views, coords.to(cuda_device), oracle.balanced_pairs(d), grid, packed=False)
    for g, v in zip(got, x.split(6, dim=1)):
        want = oracle.axial_rope(v, coords)
        assert g.is_contiguous() and g.dtype == dtype
        assert torch.equal(g.cpu(), want)


def test_rope_packed_and_backward(cuda_device):
    n, d = 65539, 16
    x = torch.randn(1, 2, n, d)
    pairs = (d // 2, 0, 0)
    seq = torch.arange(n)
    coords = torch.stack((seq, torch.zeros_like(seq), torch.zeros_like(seq)), -1)
    xd = x.to(cuda_device).requires_grad_()
    got = rotate_projections(xd, xd, xd, coords.to(cuda_device), pairs, (n, 1, 1), packed=True)[0]
    want = oracle.axial_rope(x, coords, pairs)
    torch.testing.assert_close(got.cpu(), want, atol=2e-6, rtol=2e-6)
    dy = torch.randn_like(x)
    grad, = torch.autograd.grad(got, xd, dy.to(cuda_device))
    torch.testing.assert_close(grad.cpu(), oracle.axial_rope(dy, coords, pairs, inverse=True), atol=2e-6, rtol=2e-6)


# ------------------------------------------------------------------ core, custom graphs

@pytest.mark.parametrize("case", CORE_CASES, ids=[c[0] for c in CORE_CASES])
def test_core_graph_cases_match_reference(cuda_device, golden, case):
    name, n, d, b, h, g, volume, pool, dtype, seed, temperature, empty = case
    if dtype == torch.float64:
        pytest.skip("fp64 is an oracle-only dtype")
    inputs, nb, blocks = graph_case(n, d, b, h, g, volume, pool, dtype, seed, empty)
    geom = prepare_geometry(nb, blocks, pool).to(cuda_device)
    ref = golden(f"core_{name}.pt")
    leaves = to_dev(inputs, cuda_device, grad=True)
    y = pack3d_streamed(*leaves, geom, temperature=temperature)
    tol = TOL[dtype]
    assert max_abs(y, ref["y"]) <= tol, ("y", max_abs(y, ref["y"]))
    dy = upstream(y.shape, y.dtype, seed).to(cuda_device)
    grads = torch.autograd.grad(y, leaves, dy)
    for nm, got, want in zip(NAMES, grads, ref["grads"]):
        assert got.dtype == want.dtype, nm
        # The reference's bf16 gradients are themselves rounded to bf16.  Where they exceed 2 in
        # magnitude one bf16 step is more than 2e-2, so those are held to 2e-2 relative to their
        # largest value: in the d48 bf16 case dvl (up to 4.5), dvg (2.0), dweight (2.3),
        # dlocal_scale (11.1) and dglobal_scale (2.8).  Every other gradient: plain 2e-2.
        big = dtype != torch.float32 and want.float().abs().max().item() > 2.0
        scale = want.float().abs().max().item() if big else 1.0
        assert max_abs(got, want) <= tol * scale, (nm, max_abs(got, want))
    with torch.inference_mode():
        inference = pack3d_streamed(*[t.detach() for t in leaves], geom, temperature=temperature)
    assert max_abs(inference, y) <= tol


# ---------------------------------------------------------- benchmark-shaped grid pipeline

def _grid_layout(grid):
    layout = build_layout(grid, (4, 4, 4), radius=2, pool_size=1)
    return layout.repack(layout.order.argsort())


def _pipeline(inputs, layout, temperature=1.0):
    q, kl, vl, kg, vg, *rest = inputs
    pairs = oracle.balanced_pairs(q.shape[-1])
    rq, rkl, rkg = rotate_projections(q, kl, kg, layout.coords, pairs, layout.grid_shape, packed=False)
    return pack3d_streamed(rq, rkl, vl, rkg, vg, *rest, layout.geometry, temperature=temperature)


@pytest.mark.parametrize("case", GRID_CASES, ids=[c[0] for c in GRID_CASES])
def test_grid_pipeline_matches_reference(cuda_device, golden, case):
    name, grid, b, h, g, d, dtype, seed, weighted = case
    layout = _grid_layout(grid)
    inputs = grid_inputs(layout.geometry.num_tokens, b, h, g, d, dtype, seed, weighted)
    ref = golden(f"grid_{name}.pt")
    leaves = to_dev(inputs, cuda_device, grad=True)
    y = _pipeline(leaves, layout.to(cuda_device))
    assert max_abs(y, ref["y"]) <= 1e-5
    dy = upstream(y.shape, y.dtype, seed).to(cuda_device)
    for nm, got, want in zip(NAMES, torch.autograd.grad(y, leaves, dy), ref["grads"]):
        assert max_abs(got, want) <= 1e-5 * max(1.0, want.abs().max().item()), nm


def test_config0_fp32_forward_matches_oracle(cuda_device):
    """16^3 raster, B=2, 4 heads x 48, radius 2, 4x4x4 mean pooling, fp32."""
    layout = _grid_layout((16, 16, 16))
    n = layout.geometry.num_tokens
    inputs = grid_inputs(n, 2, 4, 4, 48, torch.float32, 0, False)
    q, kl, vl, kg, vg, *rest = inputs
    rq, rkl, rkg = (oracle.axial_rope(t, layout.coords) for t in (q, kl, kg))
    geom = layout.geometry
    want = oracle.core_forward(rq, rkl, vl, rkg, vg, *rest, geom.neighbors, geom.blocks, 1)["y"]
    dev = layout.to(cuda_device)
    with torch.no_grad():
        got = _pipeline(to_dev(inputs, cuda_device), dev)
    assert max_abs(got, want) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_grid_bf16_forward_backward_matches_oracle(cuda_device, dtype):
    layout = _grid_layout((8, 8, 16))
    n = layout.geometry.num_tokens
    inputs = grid_inputs(n, 2, 4, 2, 48, dtype, 9, True)
    geom = layout.geometry
    rotated = [oracle.axial_rope(inputs[i], layout.coords) if i in (0, 1, 3) else inputs[i] for i in range(5)]
    want = oracle.core_forward(*rotated, *inputs[5:], geom.neighbors, geom.blocks, 1)["y"]
    dy = torch.randn(want.shape).to(dtype)
    leaves = to_dev(inputs, cuda_device, grad=True)
    got = _pipeline(leaves, layout.to(cuda_device))
    assert max_abs(got, want) <= 2e-2
    grads = torch.autograd.grad(got, leaves, dy.to(cuda_device))
    ref_leaves = [t.float().requires_grad_() for t in inputs]
    ref_rot = [oracle.axial_rope(ref_leaves[i], layout.coords) if i in (0, 1, 3) else ref_leaves[i]
               for i in range(5)]
    ref_y = oracle.pack3d_core(*ref_rot, *ref_leaves[5:], geom.neighbors, geom.blocks, 1, chunk=512)
    ref_grads = torch.autograd.grad(ref_y, ref_leaves, dy.float())
    # Tensor gradients (largest about 2.8) at plain 2e-2.  The parameter gradients that sum over
    # all 2 x 4 x 1024 query rows -- dweight (about 18), dlocal_scale (about 39) and
    # dglobal_scale (about 19) -- at 2e-2 relative to their largest magnitude.
    summed = {"pool_weight", "local_scale", "global_scale"}
    for nm, a, b in zip(NAMES, grads, ref_grads):
        scale = max(1.0, b.abs().max().item()) if nm in summed else 1.0
        assert max_abs(a, b) <= 2e-2 * scale, (nm, max_abs(a, b))


# ------------------------------------------------------------------ contract properties

def test_repack_equivariance(cuda_device):
    raster = _grid_layout((8, 8, 8))
    morton = build_layout((8, 8, 8), (4, 4, 4), radius=2, pool_size=1)   # native block-Morton storage
    p = morton.order                                    # Morton row i holds raster row p[i]
    inputs = grid_inputs(512, 1, 4, 4, 48, torch.bfloat16, 4, True)
    dev_r, dev_m = raster.to(cuda_device), morton.to(cuda_device)
    with torch.no_grad():
        y_r = _pipeline(to_dev(inputs, cuda_device), dev_r)
        permuted = [t[:, :, p] if i in (0, 1, 2, 3, 4, 7) else t for i, t in enumerate(inputs)]
        y_m = _pipeline(to_dev(permuted, cuda_device), dev_m)
    # Morton storage gathers its rows into raster order and runs the same arithmetic: exact.
    assert torch.equal(y_m, y_r[:, :, p.to(cuda_device)])


def test_backward_is_deterministic_and_saves_19(cuda_device):
    layout = _grid_layout((8, 8, 8))
    inputs = to_dev(grid_inputs(512, 1, 2, 1, 48, torch.bfloat16, 2, True), cuda_device, grad=True)
    rotated = rotate_projections(inputs[0], inputs[1], inputs[3], layout.coords.to(cuda_device),
                                 (8, 8, 8), layout.grid_shape, packed=False)
    saved = []
    geom = layout.to(cuda_device).geometry
    with torch.autograd.graph.saved_tensors_hooks(lambda t: saved.append(tuple(t.shape)) or t, lambda t: t):
        y = pack3d_streamed(rotated[0], rotated[1], inputs[2], rotated[2], *inputs[4:], geom)
    core_saved = [s for s in saved if s != (512, 3)]
    assert len(core_saved) == 19
    assert all(not (512 in s and geom.num_summaries in s) for s in core_saved)
    dy = torch.randn_like(y)
    g1 = torch.autograd.grad(y, inputs, dy, retain_graph=True)
    g2 = torch.autograd.grad(y, inputs, dy)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_singleton_summary_has_no_query_or_key_gradient(cuda_device, dtype):
    inputs, nb, blocks = graph_case(1, 16, 1, 1, 1, 1, 1, dtype, 18)
    geom = prepare_geometry(nb, blocks, 1).to(cuda_device)
    leaves = to_dev(inputs, cuda_device, grad=True)
    y = pack3d_streamed(*leaves, geom)
    grads = torch.autograd.grad(y, leaves, torch.randn_like(y))
    for index in (0, 1, 2, 3, 5, 6):
        assert torch.count_nonzero(grads[index]) == 0, NAMES[index]


def test_mutated_geometry_fails_backward(cuda_device):
    inputs, nb, blocks = graph_case(37, 16, 2, 4, 2, 4, 3, torch.float32, 18)
    geom = prepare_geometry(nb, blocks, 3).to(cuda_device)
    leaves = to_dev(inputs, cuda_device, grad=True)
    y = pack3d_streamed(*leaves, geom)
    geom.neighbors[1, 0] = 1
    with pytest.raises(RuntimeError, match="changed"):
        y.sum().backward()


@pytest.mark.parametrize("tag", ["f32"])
def test_layer_matches_reference(cuda_device, golden, tag):
    ref = golden(f"layer_{tag}.pt")
    t = ref["layout"]
    layer = PACK3DAttention(32, heads=ref["heads"], kv_heads=ref["kv_heads"], head_dim=ref["head_dim"],
                            block_volume=t["blocks"].shape[1])
    layer.load_state_dict(ref["state"])
    layer = layer.to(cuda_device)
    layout = build_layout((4, 4, 4), pool_size=2).to(cuda_device)
    x = ref["x"].to(cuda_device).requires_grad_()
    y = layer(x, layout)
    assert max_abs(y, ref["y"]) <= 1e-5
    grads = torch.autograd.grad(y, (x, *layer.parameters()), ref["dy"].to(cuda_device))
    for nm, got, want in zip(ref["names"], grads, ref["grads"]):
        assert max_abs(got, want) <= 2e-5 * max(1.0, want.abs().max().item()), nm


def test_indexed_and_custom_graph_paths_agree(cuda_device):
    layout = _grid_layout((8, 8, 8))
    g = layout.geometry
    custom = TokenLayout(layout.grid_shape, layout.order, layout.coords,
                         prepare_geometry(g.neighbors, g.blocks, 1)).to(cuda_device)
    inputs = to_dev(grid_inputs(512, 1, 4, 4, 48, torch.bfloat16, 6, True), cuda_device)
    with torch.no_grad():
        a = _pipeline(inputs, layout.to(cuda_device))
        b = _pipeline(inputs, custom)
    assert max_abs(a, b) <= 2e-2
    y, _ = p3d_ops.forward(*[t.contiguous() for t in inputs], custom.geometry, 1.0, save_state=False)
    assert y.shape == a.shape


@pytest.mark.parametrize("dtype,d", [(torch.bfloat16, 48), (torch.float16, 64), (torch.float32, 48), (torch.bfloat16, 16)])
def test_token_major_output_and_gradient_are_layout_only(cuda_device, dtype, d):
    """``pack3d_token_major`` / ``P3D_OPT_DY_ROWS`` change storage order only: the same y and
    bitwise the same gradients as the head-major call with a contiguous dy."""
    from pack3d_b200.ops import pack3d_token_major
    layout = _grid_layout((8, 8, 16)).to(cuda_device)
    n = layout.geometry.num_tokens
    inputs = [t.to(cuda_device) for t in grid_inputs(n, 2, 4, 2, d, dtype, 5, True)]
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    dy_rows = torch.randn(2, n, 4, d, device=cuda_device, generator=gen).to(dtype)   # [B, N, H, D]
    results = []
    for fn, dy in ((pack3d_streamed, dy_rows.transpose(1, 2).contiguous()), (pack3d_token_major, dy_rows.transpose(1, 2))):
        leaves = [t.clone().requires_grad_() for t in inputs]
        y = fn(*leaves, layout.geometry)
        grads = torch.autograd.grad(y, leaves, dy)
        results.append((y, grads))
    (y0, g0), (y1, g1) = results
    assert y1.transpose(1, 2).is_contiguous() and torch.equal(y0, y1)
    for nm, a, b in zip(NAMES, g0, g1):
        assert torch.equal(a, b), nm
