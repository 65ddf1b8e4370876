"""Parity at the benchmark configurations' own sizes (64^3 field, 4 heads x 48, radius 2, 4096
summaries), against the CPU oracle.

* Config 1: the exact layer inference path the benchmark times (``PACK3DAttention`` in bf16,
  ``inference_mode``: fused LayerNorm, projection split with RoPE, pooling, tensor-core stencil,
  output GEMM with the residual) against the oracle's layer (``attention.py:53-89``) on
  sampled query rows that include every border plane of the volume.
* Config 3: operator gradients of the training shape (batch 2).  ``dq`` and ``dgate`` at 64^3
  on sampled rows (each depends only on its own row); every gradient in full at 32^3 with
  512 summaries, where the oracle's full backward takes seconds rather than minutes.
* Config 2: Morton (Z-order) storage of the same field gives the permuted outputs and
  gradients of raster storage bit for bit, in bf16 and f16 -- the Morton path gathers its
  rows into raster order and runs the same arithmetic in the same order.

Tolerances are the benchmark contract's: max-abs 2e-2 for 16-bit outputs and gradients.
"""
import pytest
import torch

import oracle
from cases import grid_inputs
from pack3d_b200 import PACK3DAttention, _native, build_layout, pack3d_streamed

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _layout(grid, raster=True):
    layout = build_layout(grid, (4, 4, 4), radius=2, pool_size=1)
    return layout.repack(layout.order.argsort()) if raster else layout


def _border_and_sampled_rows(grid, extra, seed):
    """Every token on a face of the volume plus ``extra`` seeded interior rows."""
    z, y, x = (torch.arange(s) for s in grid)
    zz, yy, xx = torch.meshgrid(z, y, x, indexing="ij")
    face = ((zz == 0) | (zz == grid[0] - 1) | (yy == 0) | (yy == grid[1] - 1) | (xx == 0) | (xx == grid[2] - 1))
    border = face.flatten().nonzero().flatten()
    inner = (~face.flatten()).nonzero().flatten()
    pick = inner[torch.randperm(len(inner), generator=torch.Generator().manual_seed(seed))[:extra]]
    return torch.cat((border, pick)).sort().values


def test_config1_layer_inference_matches_oracle(cuda_device):
    """BASELINE config 1, the benchmark's own call: 64^3 raster field, batch 1, dim 192 =
    4 heads x 48, bf16, seeded layer (seed 0).  The oracle runs the reference layer on the same
    bf16 tensors and forms the output projection plus residual unrounded: the library adds
    the residual inside the GEMM and rounds once, the reference's eager layer rounds twice.
    The bound covers that one rounding (half a bf16 step: 0.0078 for |y| < 4)."""
    grid = (64, 64, 64)
    layout = _layout(grid)
    torch.manual_seed(0)
    layer = PACK3DAttention(192, heads=4, kv_heads=4, head_dim=48, block_volume=64).to(torch.bfloat16)
    params = {k: v.detach().clone() for k, v in layer.state_dict().items()}
    x = torch.randn(1, 64 ** 3, 192, generator=torch.Generator().manual_seed(101)).to(torch.bfloat16)
    dev_layer = layer.to(cuda_device)
    with torch.inference_mode():
        y = dev_layer(x.to(cuda_device), layout.to(cuda_device))
    torch.cuda.synchronize()
    assert _native.device_errors() == 0
    rows = _border_and_sampled_rows(grid, 4096, seed=102)
    assert len(rows) >= 4096 + 6 * 62 * 62
    want = oracle.layer_forward(x, params, layout.coords, layout.geometry.neighbors, layout.geometry.blocks, 1,
                                heads=4, kv_heads=4, head_dim=48, rows=rows, exact_output=True)
    got = y[:, rows.to(cuda_device)].float().cpu()
    err = (got - want).abs().max().item()
    assert err <= TOL, f"config-1 layer max abs error {err}"


def _operator_inputs(layout, b, h, g, d, dtype, seed):
    """Benchmark settings (mean pooling, gate 0.5, branch scales 1 / 0.25), RoPE applied by the
    oracle to the seeded pre-RoPE projections, stored in ``dtype``."""
    n = layout.geometry.num_tokens
    raw = grid_inputs(n, b, h, g, d, torch.float32, seed, False)
    rot = [oracle.axial_rope(raw[i], layout.coords) if i in (0, 1, 3) else raw[i] for i in range(5)]
    return [t.to(dtype) for t in rot] + raw[5:]


def _gpu_forward_backward(inputs, layout, dy, dev):
    leaves = [t.to(dev).requires_grad_() for t in inputs]
    geom = layout.to(dev).geometry
    y = pack3d_streamed(*leaves, geom)
    y.backward(dy.to(dev))
    torch.cuda.synchronize()
    assert _native.device_errors() == 0
    return y.detach(), [t.grad for t in leaves]


def test_config3_dq_and_dgate_rows_at_64(cuda_device):
    """BASELINE config 3 shape (64^3, batch 2, 4 heads x 48, bf16, 4096 summaries): dq and
    dgate of ~29k query rows (every border plane and 4096 interior rows) against the oracle.
    Largest |dq| here is about 2.5."""
    grid = (64, 64, 64)
    layout = _layout(grid)
    inputs = _operator_inputs(layout, 2, 4, 4, 48, torch.bfloat16, seed=301)
    dy = torch.randn(2, 4, 64 ** 3, 48, generator=torch.Generator().manual_seed(302)).to(torch.bfloat16)
    _, grads = _gpu_forward_backward(inputs, layout, dy, cuda_device)
    rows = _border_and_sampled_rows(grid, 4096, seed=303)
    geom = layout.geometry
    f32 = [t.float() for t in inputs[:5]] + inputs[5:]
    dq, dgate = oracle.core_backward_rows(dy.float(), *f32, geom.neighbors, geom.blocks, 1, rows)
    r = rows.to(cuda_device)
    err_dq = (grads[0][:, :, r].float().cpu() - dq).abs().max().item()
    err_gate = (grads[7][:, :, r].float().cpu() - dgate).abs().max().item()
    assert dq.abs().max().item() < 8
    assert err_dq <= TOL, f"dq max abs error {err_dq}"
    assert err_gate <= TOL, f"dgate max abs error {err_gate}"


def test_config3_every_gradient_at_32(cuda_device):
    """Config-3 arithmetic at 32^3 (batch 2, 4 heads x 48, bf16, 512 summaries -- several
    global chunks, a partial last one), every gradient in full against the oracle.

    The tensor gradients (dq, dkl, dvl, dkg, dvg, dgate; largest about 2.4) pass at max-abs
    2e-2.  Three parameter gradients are sums over all 2 x 4 x 32,768 query rows: dlocal_scale
    reaches about 160, dweight about 7 and dglobal_scale about 6.  Each of their terms uses the
    16-bit saved branch outputs (as the reference's GPU backward does), so their bound is 2e-2
    relative to their largest magnitude."""
    grid = (32, 32, 32)
    layout = _layout(grid)
    inputs = _operator_inputs(layout, 2, 4, 4, 48, torch.bfloat16, seed=311)
    n = layout.geometry.num_tokens
    dy = torch.randn(2, 4, n, 48, generator=torch.Generator().manual_seed(312)).to(torch.bfloat16)
    y, grads = _gpu_forward_backward(inputs, layout, dy, cuda_device)
    geom = layout.geometry
    f32 = [t.float() for t in inputs[:5]] + inputs[5:]
    want_y = oracle.core_forward(*f32, geom.neighbors, geom.blocks, 1)["y"]
    assert (y.float().cpu() - want_y).abs().max().item() <= TOL
    want = oracle.core_backward(dy.float(), *f32, geom.neighbors, geom.blocks, 1)
    names = ("dq", "dkl", "dvl", "dkg", "dvg", "dweight", "dbias", "dgate", "dlocal_scale", "dglobal_scale")
    summed = {"dweight", "dlocal_scale", "dglobal_scale"}
    for name, got, ref in zip(names, grads, want):
        err = (got.float().cpu() - ref.float()).abs().max().item()
        scale = max(1.0, ref.abs().max().item()) if name in summed else 1.0
        assert err <= TOL * scale, f"{name}: max abs error {err} (largest |ref| {ref.abs().max().item():.3g})"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_config2_morton_storage_is_the_permuted_raster_result(cuda_device, dtype):
    """the 64^3 field stored in Morton order (the native layout) gives
    exactly the raster result permuted -- output and every per-token gradient bit for bit,
    in bf16 and f16 (reference equivariance test ``tests/test_repacking.py:5-23``).  The
    summed scale gradients visit the rows in storage order, so they agree to rounding."""
    grid = (64, 64, 64)
    raster, morton = _layout(grid), _layout(grid, raster=False)
    inputs = _operator_inputs(raster, 1, 4, 4, 48, dtype, seed=321)
    n = raster.geometry.num_tokens
    dy = torch.randn(1, 4, n, 48, generator=torch.Generator().manual_seed(322)).to(dtype)
    p = morton.order                       # Morton row i holds raster token p[i]
    per_token = (0, 1, 2, 3, 4, 7)         # q, kl, vl, kg, vg, gate
    permuted = [t[:, :, p].contiguous() if i in per_token else t for i, t in enumerate(inputs)]
    y_r, g_r = _gpu_forward_backward(inputs, raster, dy, cuda_device)
    y_m, g_m = _gpu_forward_backward(permuted, morton, dy[:, :, p].contiguous(), cuda_device)
    pd = p.to(cuda_device)
    assert torch.equal(y_m, y_r[:, :, pd])
    for i, name in ((0, "dq"), (1, "dkl"), (2, "dvl"), (3, "dkg"), (4, "dvg"), (7, "dgate")):
        assert torch.equal(g_m[i], g_r[i][:, :, pd]), name
    for i, name in ((5, "dweight"), (6, "dbias")):     # summed in block order: the same order
        assert torch.equal(g_m[i], g_r[i]), name
    for i, name in ((8, "dlocal_scale"), (9, "dglobal_scale")):
        torch.testing.assert_close(g_m[i], g_r[i], atol=1e-3, rtol=1e-4, msg=name)


def test_config2_morton_layer_inference_is_the_permuted_raster_layer(cuda_device):
    """BASELINE config 2 through the layer call the benchmark times: the 64^3 field in Morton
    storage, where the projection split writes q, kl, vl at raster rows and the tensor-core
    kernel reads them without a gather pass, gives the raster layer's output permuted, bit for
    bit (LayerNorm, the projections and the output GEMM are per-row; the pooled summaries visit
    each block's slots in the same order in both layouts)."""
    from pack3d_b200 import ops as p3d_ops
    grid = (64, 64, 64)
    raster, morton = _layout(grid), _layout(grid, raster=False)
    assert p3d_ops.raster_qkv_applies(morton.geometry, torch.bfloat16, 48, cuda_device)
    assert not p3d_ops.raster_qkv_applies(raster.geometry, torch.bfloat16, 48, cuda_device)
    torch.manual_seed(0)
    layer = PACK3DAttention(192, heads=4, kv_heads=4, head_dim=48, block_volume=64).to(torch.bfloat16)
    layer = layer.to(cuda_device)
    x = torch.randn(1, 64 ** 3, 192, generator=torch.Generator().manual_seed(201)).to(torch.bfloat16)
    p = morton.order.to(cuda_device)       # Morton row i holds raster token p[i]
    x = x.to(cuda_device)
    with torch.inference_mode():
        y_r = layer(x, raster.to(cuda_device))
        y_m = layer(x[:, p].contiguous(), morton.to(cuda_device))
    torch.cuda.synchronize()
    assert _native.device_errors() == 0
    assert torch.equal(y_m, y_r[:, p])
