"""The CPU oracle reproduces the reference's own outputs (golden fixtures).

These pins are what make the oracle trustworthy as the checker for the CUDA
path: RoPE, pooling, the core with all ten gradients (both through autograd
and through the explicit chunked backward) and the whole layer.
"""
import pytest
import torch

import oracle
from cases import CORE_CASES, GRID_CASES, graph_case, grid_inputs, upstream
from pack3d_b200 import build_layout


def _tol(dtype):
    return {torch.float64: 1e-12, torch.float32: 2e-6, torch.bfloat16: 1e-2}[dtype]


def test_balanced_pairs():
    assert oracle.balanced_pairs(64) == (11, 11, 10)
    assert oracle.balanced_pairs(48) == (8, 8, 8)
    with pytest.raises(ValueError):
        oracle.balanced_pairs(15)


def test_rope_matches_reference(golden):
    for case in golden("rope.pt"):
        got = oracle.axial_rope(case["x"], case["coords"], case["pairs"])
        assert got.dtype == case["y"].dtype
        # Same fp32 operations in the same order: bit-identical.
        assert torch.equal(got, case["y"])


def test_rope_inverse_is_transpose():
    x = torch.randn(1, 2, 9, 48, dtype=torch.float64)
    c = torch.randint(0, 30, (9, 3))
    back = oracle.axial_rope(oracle.axial_rope(x, c), c, inverse=True)
    torch.testing.assert_close(back, x, atol=1e-12, rtol=1e-12)


def test_pooling_matches_reference(golden):
    for case in golden("pool.pt"):
        sk, sv = oracle.compress_summaries(case["k"], case["v"], case["w"], case["bias"], case["blocks"],
                                           case["pool_size"], case["temperature"])
        tol = _tol(case["k"].dtype) if case["k"].dtype != torch.bfloat16 else 1e-6
        torch.testing.assert_close(sk, case["sk"], atol=tol, rtol=tol)
        torch.testing.assert_close(sv, case["sv"], atol=tol, rtol=tol)


@pytest.mark.parametrize("case", CORE_CASES, ids=[c[0] for c in CORE_CASES])
def test_core_and_gradients_match_reference(golden, case):
    name, n, d, b, h, g, volume, pool, dtype, seed, temperature, empty = case
    inputs, nb, blocks = graph_case(n, d, b, h, g, volume, pool, dtype, seed, empty)
    ref = golden(f"core_{name}.pt")
    leaves = [t.clone().requires_grad_() for t in inputs]
    y = oracle.pack3d_core(*leaves, nb, blocks, pool, temperature, chunk=16)
    dy = upstream(y.shape, y.dtype, seed)
    tol = _tol(dtype)
    torch.testing.assert_close(y, ref["y"], atol=tol, rtol=tol)
    grads = torch.autograd.grad(y, leaves, dy)
    for got, want in zip(grads, ref["grads"]):
        torch.testing.assert_close(got, want, atol=tol * 5, rtol=tol * 5)
    explicit = oracle.core_backward(dy, *inputs, nb, blocks, pool, temperature, chunk=16)
    for got, want in zip(explicit, ref["grads"]):
        assert got.dtype == want.dtype
        torch.testing.assert_close(got, want, atol=tol * 5, rtol=tol * 5)
    state = oracle.core_forward(*inputs, nb, blocks, pool, temperature, chunk=16)
    torch.testing.assert_close(state["y"], ref["y"], atol=tol, rtol=tol)


@pytest.mark.parametrize("case", GRID_CASES, ids=[c[0] for c in GRID_CASES])
def test_grid_pipeline_matches_reference(golden, case):
    name, grid, b, h, g, d, dtype, seed, weighted = case
    layout = build_layout(grid, (4, 4, 4), radius=2, pool_size=1)
    layout = layout.repack(layout.order.argsort())
    geom = layout.geometry
    inputs = grid_inputs(geom.num_tokens, b, h, g, d, dtype, seed, weighted)
    ref = golden(f"grid_{name}.pt")
    leaves = [t.clone().requires_grad_() for t in inputs]
    rq, rkl, rkg = (oracle.axial_rope(t, layout.coords) for t in (leaves[0], leaves[1], leaves[3]))
    y = oracle.pack3d_core(rq, rkl, leaves[2], rkg, *leaves[4:], geom.neighbors, geom.blocks, 1, chunk=100)
    torch.testing.assert_close(y, ref["y"], atol=2e-6, rtol=2e-6)
    dy = upstream(y.shape, y.dtype, seed)
    for got, want in zip(torch.autograd.grad(y, leaves, dy), ref["grads"]):
        torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("tag", ["f64", "f32"])
def test_layer_matches_reference(golden, tag):
    ref = golden(f"layer_{tag}.pt")
    t = ref["layout"]
    params = {k: v.clone().requires_grad_() for k, v in ref["state"].items()}
    x = ref["x"].clone().requires_grad_()
    y = oracle.layer_forward(x, params, t["coords"], t["neighbors"], t["blocks"], t["pool_size"],
                             heads=ref["heads"], kv_heads=ref["kv_heads"], head_dim=ref["head_dim"])
    tol = 1e-12 if tag == "f64" else 2e-6
    torch.testing.assert_close(y, ref["y"], atol=tol, rtol=tol)
    names = ref["names"]
    leaves = [x] + [params[name] for name in names[1:]]
    for name, got, want in zip(names, torch.autograd.grad(y, leaves, ref["dy"]), ref["grads"]):
        torch.testing.assert_close(got, want, atol=tol * 10, rtol=tol * 10, msg=name)


def test_explicit_backward_matches_autograd_on_grid():
    layout = build_layout((8, 8, 8), (4, 4, 4), radius=2, pool_size=1)
    geom = layout.geometry
    inputs = grid_inputs(geom.num_tokens, 2, 4, 2, 48, torch.float64, 3, True)
    leaves = [t.clone().requires_grad_() for t in inputs]
    y = oracle.pack3d_core(*leaves, geom.neighbors, geom.blocks, 1, 0.8, chunk=128)
    dy = torch.randn_like(y)
    auto = torch.autograd.grad(y, leaves, dy)
    explicit = oracle.core_backward(dy, *inputs, geom.neighbors, geom.blocks, 1, 0.8, chunk=77)
    for a, e in zip(auto, explicit):
        torch.testing.assert_close(e, a, atol=1e-11, rtol=1e-11)
