"""Fused projection + split + axial RoPE (``p3d_qkv_project``) against the unfused path:
cuBLAS projections (rounded to the storage type) followed by ``p3d_qkv_split`` -- itself
bit-exact against the RoPE kernel the golden vectors pin.  The fused kernel accumulates the
projections in its own order, so its rounded projections may sit one storage step away from
cuBLAS's; the tolerance is two steps of the output's magnitude."""
import pytest
import torch

from pack3d_b200 import _native, build_layout
from pack3d_b200.rope import balanced_pairs, phase_tables

pytestmark = pytest.mark.gpu

# (batch, grid, dim, heads, kv_heads, head_dim, dtype)
CASES = [
    (1, (8, 12, 16), 192, 4, 4, 48, torch.bfloat16),     # config-1 shape family
    (2, (5, 7, 9), 192, 4, 4, 48, torch.bfloat16),       # 315 tokens: ragged last tile
    (2, (8, 8, 8), 256, 8, 2, 32, torch.bfloat16),       # GQA, groups of 8 heads
    (1, (6, 6, 6), 128, 6, 3, 48, torch.float16),        # 6 q heads in groups of 5: a short group
    (1, (8, 8, 8), 64, 2, 1, 64, torch.bfloat16),
    (1, (4, 8, 8), 128, 2, 2, 128, torch.float16),
    (3, (4, 4, 4), 64, 4, 2, 16, torch.bfloat16),
]


def _unfused(x, wq, wkv, coords, pairs, phases, extents, b, n, h, g, d):
    qp, kvp = x @ wq.t(), x @ wkv.t()
    outs = [torch.empty((b, h, n, d), dtype=x.dtype, device=x.device)]
    outs += [torch.empty((b, g, n, d), dtype=x.dtype, device=x.device) for _ in range(4)]
    _native.check(_native.lib().p3d_qkv_split(
        _native.ptr(qp), _native.ptr(kvp), *[_native.ptr(t) for t in outs], _native.DTYPE_CODE[x.dtype], b, h, g, n,
        d, _native.ptr(coords), *pairs, _native.ptr(phases), *extents, 0, _native.stream_of(x.device)),
        "p3d_qkv_split")
    return outs


@pytest.mark.parametrize("case", CASES, ids=[f"b{c[0]}_dim{c[2]}_h{c[3]}g{c[4]}_d{c[5]}" for c in CASES])
def test_project_matches_gemm_then_split(cuda_device, case):
    b, grid, dim, h, g, d, dtype = case
    lib = _native.lib()
    code = _native.DTYPE_CODE[dtype]
    assert lib.p3d_qkv_project_supported(code, dim, h, g, d) == 1
    layout = build_layout(grid, 1, radius=0, pool_size=1).to(cuda_device)
    n = layout.geometry.num_tokens
    gen = torch.Generator(device=cuda_device).manual_seed(dim + h + d)
    x = torch.randn(b * n, dim, device=cuda_device, generator=gen).to(dtype)
    wq = (torch.randn(h * d, dim, device=cuda_device, generator=gen) / dim ** 0.5).to(dtype)
    wkv = (torch.randn(4 * g * d, dim, device=cuda_device, generator=gen) / dim ** 0.5).to(dtype)
    pairs = balanced_pairs(d)
    extents = tuple(int(e) for e in layout.grid_shape)
    _, phases = phase_tables(cuda_device, pairs, extents)
    coords = layout.coords.to(torch.int64).contiguous()
    want = _unfused(x, wq, wkv, coords, pairs, phases, extents, b, n, h, g, d)
    got = [torch.full_like(t, float("nan")) for t in want]
    with torch.cuda.device(cuda_device):
        _native.check(lib.p3d_qkv_project(
            _native.ptr(x), _native.ptr(wq), _native.ptr(wkv), *[_native.ptr(t) for t in got], code, b, h, g, n, dim,
            d, _native.ptr(coords), *pairs, _native.ptr(phases), *extents, 0, 0, 0, _native.stream_of(cuda_device)),
            "p3d_qkv_project")
    # kl, vl between halo rows of an extended buffer (a z-slab rank's layout): the same rows,
    # nothing written outside them
    lo, extra = 3, 7
    ext = [torch.full((b, g, n + extra, d), float("nan"), dtype=dtype, device=cuda_device) for _ in range(2)]
    other = [torch.empty_like(t) for t in got]
    with torch.cuda.device(cuda_device):
        _native.check(lib.p3d_qkv_project(
            _native.ptr(x), _native.ptr(wq), _native.ptr(wkv), _native.ptr(other[0]), _native.ptr(ext[0]),
            _native.ptr(ext[1]), _native.ptr(other[3]), _native.ptr(other[4]), code, b, h, g, n, dim, d,
            _native.ptr(coords), *pairs, _native.ptr(phases), *extents, n + extra, lo, 0,
            _native.stream_of(cuda_device)), "p3d_qkv_project")
    torch.cuda.synchronize()
    assert _native.device_errors() == 0
    for e, dense in zip(ext, got[1:3]):
        assert torch.equal(e[:, :, lo:lo + n], dense)
        assert torch.isnan(e[:, :, :lo]).all() and torch.isnan(e[:, :, lo + n:]).all()
    for i in (0, 3, 4):
        assert torch.equal(other[i], got[i])
    step = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    for nm, a, w in zip(("q", "kl", "vl", "kg", "vg"), got, want):
        assert not torch.isnan(a).any(), nm
        err = (a.float() - w.float()).abs()
        bound = 2 * step * torch.maximum(a.float().abs(), w.float().abs()) + 1e-6
        assert (err <= bound).all(), (nm, err.max().item())
        # most elements agree exactly
        assert (a == w).float().mean().item() > 0.95, nm


GATE_CASES = [c for c in CASES if 2 * c[3] <= 16]


@pytest.mark.parametrize("case", GATE_CASES, ids=[f"b{c[0]}_dim{c[2]}_h{c[3]}g{c[4]}_d{c[5]}" for c in GATE_CASES])
def test_gate_project_folds_the_gate_linear(cuda_device, case):
    """p3d_qkv_gate_project: q, kl, vl, kg, vg are p3d_qkv_project's bits, and the gate is the
    separate path's (cuBLAS logits with the bias, p3d_gate_pairs) up to the logits' summation
    order: a logit may sit one storage step away, which moves the gate by at most a quarter of
    that step (softmax of a pair: dg/dl <= 1/4) plus the gate's own rounding."""
    b, grid, dim, h, g, d, dtype = case
    lib = _native.lib()
    code = _native.DTYPE_CODE[dtype]
    if not lib.p3d_qkv_gate_project_supported(code, dim, h, g, d):
        pytest.skip("no room for the gate rows at this shape")
    layout = build_layout(grid, 1, radius=0, pool_size=1).to(cuda_device)
    n = layout.geometry.num_tokens
    gen = torch.Generator(device=cuda_device).manual_seed(dim + h + d + 1)
    x = torch.randn(b * n, dim, device=cuda_device, generator=gen).to(dtype)
    wq = (torch.randn(h * d, dim, device=cuda_device, generator=gen) / dim ** 0.5).to(dtype)
    wkv = (torch.randn(4 * g * d, dim, device=cuda_device, generator=gen) / dim ** 0.5).to(dtype)
    wg = (torch.randn(2 * h, dim, device=cuda_device, generator=gen) / dim ** 0.5).to(dtype)
    bg = (torch.randn(2 * h, device=cuda_device, generator=gen) * 0.5).to(dtype)
    pairs = balanced_pairs(d)
    extents = tuple(int(e) for e in layout.grid_shape)
    _, phases = phase_tables(cuda_device, pairs, extents)
    coords = layout.coords.to(torch.int64).contiguous()
    args = (code, b, h, g, n, dim, d, _native.ptr(coords), *pairs, _native.ptr(phases), *extents, 0, 0, 0,
            _native.stream_of(cuda_device))
    plain = [torch.empty((b, h, n, d), dtype=dtype, device=cuda_device)]
    plain += [torch.empty((b, g, n, d), dtype=dtype, device=cuda_device) for _ in range(4)]
    fused = [torch.full_like(t, float("nan")) for t in plain]
    gate = torch.full((b, h, n), float("nan"), dtype=dtype, device=cuda_device)
    logits = torch.addmm(bg, x, wg.t())
    want_gate = torch.empty_like(gate)
    with torch.cuda.device(cuda_device):
        _native.check(lib.p3d_qkv_project(_native.ptr(x), _native.ptr(wq), _native.ptr(wkv),
                                          *[_native.ptr(t) for t in plain], *args), "p3d_qkv_project")
        _native.check(lib.p3d_qkv_gate_project(_native.ptr(x), _native.ptr(wq), _native.ptr(wkv), _native.ptr(wg),
                                               _native.ptr(bg), *[_native.ptr(t) for t in fused], _native.ptr(gate),
                                               *args), "p3d_qkv_gate_project")
        _native.check(lib.p3d_gate_pairs(_native.ptr(logits), 2 * h, _native.ptr(want_gate), code, b, h, n,
                                         _native.stream_of(cuda_device)), "p3d_gate_pairs")
    torch.cuda.synchronize()
    assert _native.device_errors() == 0
    for a, w in zip(fused, plain):
        assert torch.equal(a, w)
    assert not torch.isnan(gate).any()
    step = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11   # half an ulp at 1, relative
    logit_ulp = 2 * step * logits.float().abs().max().item()
    err = (gate.float() - want_gate.float()).abs().max().item()
    assert err <= 0.25 * logit_ulp + 4 * step, err
    assert (gate == want_gate).float().mean().item() > 0.9


def test_project_rejects_what_it_cannot_run(cuda_device):
    lib = _native.lib()
    assert lib.p3d_qkv_project_supported(_native.F32, 192, 4, 4, 48) == 0
    assert lib.p3d_qkv_project_supported(_native.BF16, 200, 4, 4, 48) == 0       # dim % 64
    assert lib.p3d_qkv_project_supported(_native.BF16, 96, 4, 4, 48) == 0
    assert lib.p3d_qkv_project_supported(_native.BF16, 192, 4, 4, 40) == 0       # head_dim
    assert lib.p3d_qkv_project_supported(_native.BF16, 4096, 4, 4, 48) == 0      # shared memory (X tiles alone)


@pytest.mark.parametrize("grad", [False, True])
def test_layer_with_fused_projection_matches(cuda_device, grad):
    """The layer with ``fused_projection`` (p3d_qkv_project in the forward, its autograd
    backward) against the default cuBLAS projections + p3d_qkv_split."""
    from pack3d_b200 import PACK3DAttention
    layout = build_layout((16, 16, 16), (4, 4, 4), radius=2, pool_size=1)
    layout = layout.repack(layout.order.argsort()).to(cuda_device)
    torch.manual_seed(0)
    layer = PACK3DAttention(192, heads=4, kv_heads=4, head_dim=48, block_volume=64).to(cuda_device, torch.bfloat16)
    gen = torch.Generator(device=cuda_device).manual_seed(11)
    x = torch.randn(2, layout.geometry.num_tokens, 192, device=cuda_device, generator=gen).to(torch.bfloat16)
    dy = torch.randn_like(x)
    results = []
    for fused in (True, False):
        layer.fused_projection = fused
        layer.zero_grad(set_to_none=True)
        xi = x.clone().requires_grad_(grad)
        with torch.set_grad_enabled(grad):
            y = layer(xi, layout)
        if grad:
            y.backward(dy)
            results.append((y.detach(), xi.grad, {k: p.grad.clone() for k, p in layer.named_parameters()}))
        else:
            results.append((y, None, {}))
    (y0, dx0, g0), (y1, dx1, g1) = results
    tol = lambda t: 2e-2 * max(1.0, t.float().abs().max().item())  # noqa: E731
    assert (y0.float() - y1.float()).abs().max().item() <= tol(y1)
    if grad:
        assert (dx0.float() - dx1.float()).abs().max().item() <= tol(dx1)
        for k in g1:
            assert (g0[k].float() - g1[k].float()).abs().max().item() <= tol(g1[k]), k
    assert _native.device_errors() == 0
