"""GPU parity of the tensor-core stencil forward against the indexed CUDA path and the oracle.

The indexed kernels are themselves pinned to the reference (test_gpu_parity);
here the tcgen05 path must agree with them and with the oracle on every shape
class the tile decomposition meets: partial tiles on every axis, summary counts
that are not a multiple of the 128-row chunk, GQA, bf16 and f16, every
supported head dimension, permuted (Morton) storage, and the saved state.
"""
import pytest
import torch

import oracle
from cases import grid_inputs
from pack3d_b200 import _native, build_layout
from pack3d_b200 import ops as p3d_ops

pytestmark = pytest.mark.gpu


def _layout(grid, raster=True):
    layout = build_layout(grid, (4, 4, 4), radius=2, pool_size=1)
    return layout.repack(layout.order.argsort()) if raster else layout


def _rotated_inputs(layout, b, h, g, d, dtype, seed):
    n = layout.geometry.num_tokens
    inputs = grid_inputs(n, b, h, g, d, torch.float32, seed, True)
    rot = [oracle.axial_rope(inputs[i], layout.coords) if i in (0, 1, 3) else inputs[i] for i in range(5)]
    return [t.to(dtype) for t in rot] + inputs[5:]


def _run(inputs, geom, dev, **kw):
    dev_inputs = [t.to(dev).contiguous() for t in inputs]
    return p3d_ops.forward(*dev_inputs, geom.to(dev), 1.0, **kw)


@pytest.mark.parametrize("grid,b,h,g,d,dtype", [
    ((8, 8, 16), 1, 4, 4, 48, torch.bfloat16),
    ((16, 16, 16), 2, 4, 4, 48, torch.bfloat16),       # BASELINE config-0 shape in bf16
    ((12, 8, 24), 1, 4, 2, 48, torch.float16),         # GQA, f16, M = 36 (partial chunk)
    ((4, 12, 20), 1, 2, 1, 32, torch.bfloat16),        # partial z box, x not a multiple of 8
    ((8, 8, 8), 1, 2, 2, 16, torch.bfloat16),
    ((8, 8, 8), 1, 2, 2, 64, torch.bfloat16),
    ((32, 32, 32), 1, 2, 2, 48, torch.bfloat16),       # M = 512: several global chunks
])
def test_stencil_forward_matches_indexed_and_oracle(cuda_device, grid, b, h, g, d, dtype):
    layout = _layout(grid)
    geom = layout.geometry
    inputs = _rotated_inputs(layout, b, h, g, d, dtype, seed=sum(grid) + d)
    y_tc, (sk, sv, ol, og, lse_l, lse_g) = _run(inputs, geom, cuda_device)
    y_ix, (_, _, ol_i, og_i, ll_i, lg_i) = _run(inputs, geom, cuda_device, force_indexed=True)
    torch.cuda.synchronize()
    assert _native.device_errors() == 0
    tol = 2e-2
    assert (y_tc.float() - y_ix.float()).abs().max().item() <= tol
    assert (ol.float() - ol_i.float()).abs().max().item() <= tol
    assert (og.float() - og_i.float()).abs().max().item() <= tol
    assert (lse_l - ll_i).abs().max().item() <= 1e-2
    assert (lse_g - lg_i).abs().max().item() <= 1e-2
    want = oracle.core_forward(*[t.float() if t.dtype != torch.float32 else t for t in inputs[:5]], *inputs[5:],
                               geom.neighbors, geom.blocks, 1, chunk=2048)
    assert (y_tc.float().cpu() - want["y"].float()).abs().max().item() <= tol
    # inference path (no saved state) writes the same output
    y_inf, _ = _run(inputs, geom, cuda_device, save_state=False)
    assert torch.equal(y_inf, y_tc)


def test_stencil_forward_on_morton_storage(cuda_device):
    raster = _layout((16, 16, 16))
    morton = _layout((16, 16, 16), raster=False)
    inputs = _rotated_inputs(raster, 1, 4, 4, 48, torch.bfloat16, seed=3)
    p = morton.order
    permuted = [t[:, :, p] if i in (0, 1, 2, 3, 4, 7) else t for i, t in enumerate(inputs)]
    y_r, _ = _run(inputs, raster.geometry, cuda_device, save_state=False)
    y_m, state = _run(permuted, morton.geometry, cuda_device)
    y_mi, _ = _run(permuted, morton.geometry, cuda_device, force_indexed=True, save_state=False)
    assert torch.equal(y_m, y_r[:, :, p.to(cuda_device)])     # the same arithmetic on the same rows
    assert (y_m.float() - y_mi.float()).abs().max().item() <= 2e-2
    assert _native.device_errors() == 0


def test_stencil_forward_is_deterministic(cuda_device):
    layout = _layout((16, 16, 32))
    inputs = _rotated_inputs(layout, 1, 4, 4, 48, torch.bfloat16, seed=8)
    a, _ = _run(inputs, layout.geometry, cuda_device, save_state=False)
    b, _ = _run(inputs, layout.geometry, cuda_device, save_state=False)
    assert torch.equal(a, b)


@pytest.mark.parametrize("grid,block,pool,kind,b,h,g,d,dtype", [
    ((8, 8, 16), (4, 4, 4), 1, "cubes", 1, 4, 4, 48, torch.bfloat16),
    ((8, 32, 16), (1, 4, 4), 16, "raster_block", 1, 8, 2, 64, torch.bfloat16),   # the allen15 preset, small
    ((6, 12, 20), (1, 4, 4), 4, "raster_block", 2, 4, 2, 32, torch.float16),     # partial tiles on every axis
    ((4, 8, 8), (4, 4, 4), 1, "cubes", 1, 2, 2, 16, torch.bfloat16),
])
def test_radius_one_stencil_forward_matches_indexed_and_oracle(cuda_device, grid, block, pool, kind, b, h, g, d,
                                                               dtype):
    """Radius 1: 6x10 halo windows padded to 64-key chunks, 6 halo planes."""
    if kind == "cubes":
        layout = build_layout(grid, block, radius=1, pool_size=pool)
        layout = layout.repack(layout.order.argsort())
    else:
        layout = build_layout(grid, block, radius=1, pool_size=pool, layout="raster_block")
    geom = layout.geometry
    assert geom.stencil == (tuple(grid), (1, 1, 1))
    n = geom.num_tokens
    raw = grid_inputs(n, b, h, g, d, torch.float32, sum(grid) + d, True, volume=block[0] * block[1] * block[2])
    inputs = [oracle.axial_rope(raw[i], layout.coords) if i in (0, 1, 3) else raw[i] for i in range(5)]
    inputs = [t.to(dtype) for t in inputs] + raw[5:]
    y_tc, (sk, sv, ol, og, lse_l, lse_g) = _run(inputs, geom, cuda_device)
    y_ix, (_, _, ol_i, og_i, ll_i, lg_i) = _run(inputs, geom, cuda_device, force_indexed=True)
    torch.cuda.synchronize()
    assert _native.device_errors() == 0
    tol = 2e-2
    assert (y_tc.float() - y_ix.float()).abs().max().item() <= tol
    assert (ol.float() - ol_i.float()).abs().max().item() <= tol
    assert (og.float() - og_i.float()).abs().max().item() <= tol
    assert (lse_l - ll_i).abs().max().item() <= 1e-2
    assert (lse_g - lg_i).abs().max().item() <= 1e-2
    want = oracle.core_forward(*[t.float() if t.dtype != torch.float32 else t for t in inputs[:5]], *inputs[5:],
                               geom.neighbors, geom.blocks, pool, chunk=2048)
    assert (y_tc.float().cpu() - want["y"].float()).abs().max().item() <= tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("bg,m,d", [(4, 4096, 48), (3, 300, 64), (1, 1, 16), (2, 8191, 32)])
def test_summary_bound_is_the_largest_summary_norm(cuda_device, dtype, bg, m, d):
    """p3d_summary_bound: per (batch, kv-head) the largest summary-row norm, rounded up by 2^-10
    (never below a norm the kernel's own arithmetic could see)."""
    from pack3d_b200 import _native
    gen = torch.Generator(device=cuda_device).manual_seed(bg * 1000 + m)
    sk = (torch.randn(bg, m, d, device=cuda_device, generator=gen) * 3).to(dtype)
    sk[0, m // 2] *= 4  # one row clearly the largest
    bound = torch.full((bg,), -1.0, device=cuda_device)
    with torch.cuda.device(cuda_device):
        _native.check(_native.lib().p3d_summary_bound(_native.ptr(sk), _native.DTYPE_CODE[dtype], 1, bg, m, d,
                                                      _native.ptr(bound), _native.stream_of(cuda_device)),
                      "p3d_summary_bound")
    want = sk.double().norm(dim=-1).amax(dim=-1)
    got = bound.double()
    assert torch.all(got >= want * (1 + 2.0 ** -12)), (got, want)
    assert torch.all(got <= want * (1 + 2.0 ** -9)), (got, want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_global_branch_with_a_loose_score_bound(cuda_device, dtype):
    """Queries orthogonal to every summary, both of norm 12: every global score is 0 while the
    Cauchy-Schwarz bound u = |q| max|sk| is 144, so p = 2^((0 - u) log2(e) / sqrt(D)) = 2^-30
    against the bound.  That is a normal bf16 number but below f16's range, so for f16 the
    kernel must track the row maximum instead (the global softmax is then uniform and og the
    summaries' mean, here 1)."""
    layout = _layout((8, 8, 16))
    geom = layout.geometry
    b, h, d = 1, 2, 48
    n = geom.num_tokens
    inputs = grid_inputs(n, b, h, h, d, torch.float32, 11, False)
    q = torch.zeros(b, h, n, d)
    q[..., : d // 2] = 12.0 / (d // 2) ** 0.5       # |q| = 12 in the first half of the channels
    kg = torch.zeros(b, h, n, d)
    kg[..., d // 2:] = 12.0 / (d // 2) ** 0.5      # |sk| = 12 in the second half: q . sk = 0
    vg = torch.ones(b, h, n, d)
    inputs[0], inputs[3], inputs[4] = q, kg, vg
    inputs = [t.to(dtype) if i < 5 else t for i, t in enumerate(inputs)]
    y_tc, (_, _, _, og, _, lse_g) = _run(inputs, geom, cuda_device)
    y_ix, (_, _, _, og_i, _, lg_i) = _run(inputs, geom, cuda_device, force_indexed=True)
    torch.cuda.synchronize()
    assert _native.device_errors() == 0
    assert (og.float() - 1).abs().max().item() <= 2e-2
    assert (og.float() - og_i.float()).abs().max().item() <= 2e-2
    assert (lse_g - lg_i).abs().max().item() <= 1e-2
    assert (y_tc.float() - y_ix.float()).abs().max().item() <= 2e-2
    want = oracle.core_forward(*[t.float() for t in inputs[:5]], *inputs[5:], geom.neighbors, geom.blocks, 1,
                               chunk=2048)
    assert (y_tc.float().cpu() - want["y"].float()).abs().max().item() <= 2e-2
