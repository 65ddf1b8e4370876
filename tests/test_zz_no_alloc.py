"""The allocation-free forward entry point (p3d_attn_fwd_noalloc) on a GPU.

It exists for callers that may not allocate device memory (a plugin inside a framework
that owns all device memory, a real-time loop that must avoid cudaMalloc's implicit
synchronisation).  It keeps its one scratch buffer in a fixed array inside the library,
so this test checks, through the C ABI: its output against the regular p3d_attn_fwd on
two calls in a row (the second on different inputs, so stale scratch from the first call
cannot leak into it), and that inputs beyond the fixed scratch are refused with a clear
error.  The file is named to be collected last.
"""
import pytest
import torch

from cases import grid_inputs
from pack3d_b200 import _native, build_layout
from pack3d_b200 import ops as p3d_ops

pytestmark = pytest.mark.gpu


def _case(grid, b, h, g, dtype, seed, device):
    layout = build_layout(grid, (4, 4, 4), radius=2, pool_size=1)
    layout = layout.repack(layout.order.argsort())
    inputs = [t.to(device) for t in grid_inputs(layout.geometry.num_tokens, b, h, g, 48, dtype, seed, True)]
    return inputs, layout.geometry.to(device)


def _noalloc(inputs, geom):
    q, kl, vl, kg, vg, weight, bias, gate, sl, sg = inputs
    b, h, n, d = q.shape
    f32 = [t.detach().float().contiguous() for t in (weight, bias, sl, sg)]
    op, keep = p3d_ops._operator(q, kl, vl, kg, vg, f32[0], f32[1], gate.contiguous(), f32[2], f32[3], geom, 1.0)
    y = torch.empty_like(q)
    sk = torch.empty(b, kl.shape[1], geom.num_summaries, d, dtype=q.dtype, device=q.device)
    sv = torch.empty_like(sk)
    status = _native.lib().p3d_attn_fwd_noalloc(op, _native.ptr(y), _native.ptr(sk), _native.ptr(sv),
                                                _native.stream_of(q.device))
    return status, y, (sk, sv), keep


def _regular(inputs, geom):
    y, _ = p3d_ops.forward(*inputs, geom, 1.0, save_state=False)
    return y


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
def test_noalloc_matches_regular_forward_twice(cuda_device, dtype, tol):
    first, geom1 = _case((16, 16, 16), 2, 4, 4, dtype, 0, cuda_device)
    second, geom2 = _case((8, 16, 16), 1, 4, 2, dtype, 7, cuda_device)
    for inputs, geom in ((first, geom1), (second, geom2)):
        status, y, _, keep = _noalloc(inputs, geom)
        _native.check(status, "p3d_attn_fwd_noalloc")
        torch.cuda.synchronize(cuda_device)
        want = _regular(inputs, geom)
        assert torch.isfinite(y.float()).all()
        assert (y.float() - want.float()).abs().max().item() <= tol
        del keep


def test_noalloc_refuses_inputs_beyond_its_scratch(cuda_device):
    inputs, geom = _case((32, 32, 32), 1, 4, 2, torch.float32, 1, cuda_device)  # needs 24 MiB
    status, _, _, keep = _noalloc(inputs, geom)
    assert status == 2
    assert b"fixed scratch" in _native.lib().p3d_last_error()
    del keep
