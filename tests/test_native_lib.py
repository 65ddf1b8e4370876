"""The C-ABI library builds, loads without a GPU and exports every declared symbol.

No compute entry point is called here (there may be no device); the product's
CUDA requirement is checked to fail loudly instead of falling back.
"""
import ctypes
import re
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"P3D_API\s+[\w\s\*]*?\b(p3d_\w+)\s*\(", header.read_text()))
    return names


def test_header_declares_entry_points():
    assert {"p3d_rope", "p3d_pool_fwd", "p3d_attn_fwd", "p3d_attn_bwd"} <= _declared()


def test_library_exports_every_declared_symbol():
    from pack3d_b200 import _native
    handle = _native.lib()
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)], capture_output=True, text=True)
    exported = set(re.findall(r"\bT (p3d_\w+)", nm.stdout))
    missing = _declared() - exported
    assert not missing, missing
    for name in _declared():
        assert getattr(handle, name) is not None
    assert set(_native.exported_symbols()) == _declared()


def test_library_metadata_calls():
    from pack3d_b200 import _native
    handle = _native.lib()
    assert handle.p3d_abi_version() == 5
    assert handle.p3d_strerror(0) == b"success"
    assert handle.p3d_strerror(4).startswith(b"workspace")
    assert handle.p3d_device_count() >= 0


def test_struct_layout_matches_header():
    """ctypes mirror of p3d_operator has the C layout (checked with the host compiler)."""
    from pack3d_b200 import _native
    src = ROOT / "include" / "pack3d_b200.h"
    probe = ('#include <stddef.h>\n#include <stdio.h>\n#include "%s"\nint main(void){printf("%%zu %%zu %%zu %%zu\\n",'
             ' sizeof(p3d_operator), offsetof(p3d_operator, blocks), offsetof(p3d_operator, raster_to_packed),'
             ' offsetof(p3d_operator, options));}'
             % src)
    exe = Path(__file__).resolve().parent / ".struct_probe"
    run = subprocess.run(["gcc", "-x", "c", "-", "-o", str(exe)], input=probe, text=True, capture_output=True)
    assert run.returncode == 0, run.stderr
    try:
        out = subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()
    finally:
        exe.unlink(missing_ok=True)
    op = _native.Operator
    assert [int(v) for v in out] == [ctypes_size(op), op.blocks.offset, op.raster_to_packed.offset,
                                     op.options.offset]


def ctypes_size(t):
    import ctypes
    return ctypes.sizeof(t)


def test_cpu_tensors_are_refused_not_computed():
    from pack3d_b200 import build_layout, pack3d_streamed
    layout = build_layout((4, 4, 4), (4, 4, 4), radius=2, pool_size=1)
    g = layout.geometry
    q = torch.randn(1, 1, 64, 48)
    args = (q, q, q, q, q, torch.zeros(48), torch.zeros(64), torch.zeros(1, 1, 64), torch.ones(48), torch.ones(48))
    with pytest.raises(ValueError, match="CUDA"):
        pack3d_streamed(*args, g)
    with pytest.raises(ValueError, match="backend"):
        pack3d_streamed(*args, g, backend="triton")


def test_layer_rejects_unsupported():
    from pack3d_b200 import PACK3DAttention
    for kwargs in ({"heads": 3}, {"temperature": 0}, {"backend": "reference"}, {"position_encoding": "none"},
                   {"head_dim": 40}):
        with pytest.raises(ValueError):
            PACK3DAttention(32, **kwargs)
    layer = PACK3DAttention(192, heads=4, kv_heads=4, head_dim=48, block_volume=64)
    assert [n for n, _ in layer.named_parameters()] == [
        "pool_weight", "slot_bias", "local_scale", "global_scale", "norm.weight", "norm.bias",
        "to_q.weight", "to_kv.weight", "gate.weight", "gate.bias", "to_out.weight"]


def test_import_does_not_pull_the_oracle():
    code = "import sys, pack3d_b200; assert 'oracle' not in sys.modules; assert 'triton' not in sys.modules"
    subprocess.run([sys.executable, "-c", code], check=True, cwd=str(ROOT))


def test_argument_checks_run_before_any_device_call():
    """Malformed calls of the glue and projection entry points are refused on the host, with
    a message, before anything touches a device (so they behave the same without a GPU)."""
    from pack3d_b200 import _native
    lib = _native.lib()
    dummy = 16  # a non-null, 16-byte aligned stand-in: never dereferenced on these paths
    # p3d_qkv_project: null pointer, bad rotation pairs
    st = lib.p3d_qkv_project(None, dummy, dummy, dummy, dummy, dummy, dummy, dummy, _native.BF16, 1, 4, 4, 64, 192,
                             48, dummy, 8, 8, 8, dummy, 4, 4, 4, 0, 0, 0, None)
    assert st == 1 and b"null pointer" in lib.p3d_last_error()
    st = lib.p3d_qkv_project(dummy, dummy, dummy, dummy, dummy, dummy, dummy, dummy, _native.BF16, 1, 4, 4, 64, 192,
                             48, dummy, 8, 8, 7, dummy, 4, 4, 4, 0, 0, 0, None)
    assert st == 1 and b"pairs" in lib.p3d_last_error()
    # kl / vl rows past the end of their buffers
    st = lib.p3d_qkv_project(dummy, dummy, dummy, dummy, dummy, dummy, dummy, dummy, _native.BF16, 1, 4, 4, 64, 192,
                             48, dummy, 8, 8, 8, dummy, 4, 4, 4, 70, 8, 0, None)
    assert st == 1 and b"outside" in lib.p3d_last_error()
    # the peer exchange: a row that is not whole 16-byte words, too many copies
    copy = _native.PeerCopy(dummy, dummy, 2, 24, 32, 32)
    st = lib.p3d_peer_push(ctypes.byref(copy), 1, 1, None, 0, 4, None)
    assert st == 1 and b"multiple of 16" in lib.p3d_last_error()
    st = lib.p3d_peer_push(ctypes.byref(copy), 33, 0, None, 0, 4, None)
    assert st == 1 and b"at most" in lib.p3d_last_error()
    st = lib.p3d_peer_wait(dummy, dummy, 1, 0.0, None)
    assert st == 1 and b"timeout" in lib.p3d_last_error()
    # shapes the fused kernel does not run are reported as unsupported, not computed
    assert lib.p3d_qkv_project_supported(_native.F32, 192, 4, 4, 48) == 0
    assert lib.p3d_qkv_project_supported(_native.BF16, 96, 4, 4, 48) == 0
    assert lib.p3d_qkv_project_supported(_native.BF16, 192, 4, 4, 40) == 0
    # p3d_qkv_split: heads not a multiple of kv_heads
    st = lib.p3d_qkv_split(dummy, dummy, dummy, dummy, dummy, dummy, dummy, _native.BF16, 1, 5, 3, 64, 48, dummy,
                           8, 8, 8, dummy, 4, 4, 4, 0, None)
    assert st == 1 and b"head" in lib.p3d_last_error()
    # p3d_pool_fwd: more than 64 slots per fine block
    st = lib.p3d_pool_fwd(dummy, dummy, dummy, dummy, dummy, 4, 65, 1, dummy, dummy, None, None, _native.BF16, 1, 1,
                          256, 48, 1.0, None)
    assert st == 1 and b"block table" in lib.p3d_last_error()
    # p3d_qkv_gate_project: the gate weight, bias and output are required; the weight 16-byte aligned
    proj_tail = (_native.BF16, 1, 4, 4, 64, 192, 48, dummy, 8, 8, 8, dummy, 4, 4, 4, 0, 0, 0, None)
    st = lib.p3d_qkv_gate_project(dummy, dummy, dummy, None, dummy, dummy, dummy, dummy, dummy, dummy, dummy,
                                  *proj_tail)
    assert st == 1 and b"p3d_qkv_gate_project: null pointer" in lib.p3d_last_error()
    st = lib.p3d_qkv_gate_project(dummy, dummy, dummy, dummy, dummy, dummy, dummy, dummy, dummy, dummy, None,
                                  *proj_tail)
    assert st == 1 and b"p3d_qkv_gate_project: null pointer" in lib.p3d_last_error()
    st = lib.p3d_qkv_gate_project(dummy, dummy, dummy, dummy + 8, dummy, dummy, dummy, dummy, dummy, dummy, dummy,
                                  *proj_tail)
    assert st == 1 and b"aligned gate weight" in lib.p3d_last_error()
    # p3d_layer_norm_bwd_residual: the residual gradient is required; misaligned, or no workspace
    st = lib.p3d_layer_norm_bwd_residual(dummy, dummy, dummy, None, dummy, dummy, dummy, _native.BF16, 8, 192, 1e-5,
                                         dummy, 1 << 20, None)
    assert st == 1 and b"null pointer" in lib.p3d_last_error()
    st = lib.p3d_layer_norm_bwd_residual(dummy, dummy, dummy, dummy + 2, dummy, dummy, dummy, _native.BF16, 8, 192,
                                         1e-5, dummy, 1 << 20, None)
    assert st == 1 and b"aligned" in lib.p3d_last_error()
    st = lib.p3d_layer_norm_bwd_residual(dummy, dummy, dummy, dummy, dummy, dummy, dummy, _native.BF16, 8, 192, 1e-5,
                                         None, 0, None)
    assert st == 4 and b"p3d_layer_norm_bwd_residual: workspace" in lib.p3d_last_error()


def test_fused_projection_is_not_offered_for_cpu_tensors():
    from pack3d_b200 import glue
    x = torch.zeros(1, 64, 192, dtype=torch.bfloat16)
    w = torch.zeros(192, 192, dtype=torch.bfloat16)
    assert not glue.project_supported(x, w, torch.zeros(768, 192, dtype=torch.bfloat16), 4, 4, 48)
