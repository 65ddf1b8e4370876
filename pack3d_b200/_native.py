"""ctypes binding of the in-tree C-ABI library ``lib/libpack3d_b200.so``.

The library is the product's only compute path.  Loading fails loudly when it
has not been built (``python -m pack3d_b200.build``); there is no fallback.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libpack3d_b200.so"

F32, F16, BF16 = 0, 1, 2
DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
FWD_SAVE_STATE = 1
FWD_FORCE_INDEXED = 2
FWD_SUMMARIES_GIVEN = 4
FWD_Y_ROWS = 8
FWD_RASTER_QKV = 16
SPLIT_RASTER_QKV = 1
OPT_INDEXED_ONLY = 1
OPT_DY_ROWS = 2

_c_int, _c_i64, _c_f32, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class Operator(ctypes.Structure):
    """Mirror of ``p3d_operator`` in ``include/pack3d_b200.h``."""

    _fields_ = [
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
        ("tokens", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32), ("gate_dtype", ctypes.c_int32), ("temperature", ctypes.c_float),
        ("q", _vp), ("kl", _vp), ("vl", _vp), ("kg", _vp), ("vg", _vp),
        ("pool_weight", _vp), ("slot_bias", _vp), ("gate", _vp), ("local_scale", _vp),
        ("global_scale", _vp),
        ("neighbors", _vp), ("width", ctypes.c_int32),
        ("reverse_neighbors", _vp), ("reverse_width", ctypes.c_int32),
        ("blocks", _vp), ("fine_blocks", ctypes.c_int32), ("slots", ctypes.c_int32),
        ("pool_size", ctypes.c_int32),
        ("stencil", ctypes.c_int32), ("grid", ctypes.c_int32 * 3), ("radius", ctypes.c_int32 * 3),
        ("raster_to_packed", _vp), ("options", ctypes.c_uint32),
    ]


class Slab(ctypes.Structure):
    """Mirror of ``p3d_slab`` in ``include/pack3d_b200.h``."""

    _fields_ = [("global_planes", ctypes.c_int32), ("center_z0", ctypes.c_int32), ("halo_z0", ctypes.c_int32),
                ("halo_planes", ctypes.c_int32), ("summaries", ctypes.c_int32), ("summary_bound", _vp),
                ("tile_z_begin", ctypes.c_int32), ("tile_z_end", ctypes.c_int32)]


class PeerCopy(ctypes.Structure):
    """Mirror of ``p3d_peer_copy`` in ``include/pack3d_b200.h``."""

    _fields_ = [("src", _vp), ("dst", _vp), ("rows", ctypes.c_int64), ("row_bytes", ctypes.c_int64),
                ("src_stride", ctypes.c_int64), ("dst_stride", ctypes.c_int64)]


PEER_HANDLE_BYTES = 64
PEER_MAX_COPIES = 32
PEER_MAX_TARGETS = 16

_SIGNATURES = {
    "p3d_strerror": (ctypes.c_char_p, [_c_int]),
    "p3d_last_error": (ctypes.c_char_p, []),
    "p3d_abi_version": (_c_int, []),
    "p3d_device_count": (_c_int, []),
    "p3d_device_errors": (_c_int, [ctypes.POINTER(ctypes.c_uint)]),
    "p3d_rope": (_c_int, [_vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                          _vp, _c_i64, _c_i64, _c_int, _c_int, _c_int, _vp, _vp, _c_int, _c_int, _c_int,
                          _c_int, _c_int, _vp]),
    "p3d_layer_norm": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_i64, _c_int, _c_f32, _vp]),
    "p3d_qkv_split": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                               _vp, _c_int, _c_int, _c_int, _vp, _c_int, _c_int, _c_int, ctypes.c_uint, _vp]),
    "p3d_qkv_gate_split": (_c_int, [_vp, _c_int, _vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                    _c_int, _c_int, _vp, _c_int, _c_int, _c_int, _vp, _c_int, _c_int, _c_int,
                                    ctypes.c_uint, _vp]),
    "p3d_gate_pairs": (_c_int, [_vp, _c_int, _vp, _c_int, _c_int, _c_int, _c_int, _vp]),
    "p3d_qkv_project_supported": (_c_int, [_c_int] * 5),
    "p3d_qkv_gate_project_supported": (_c_int, [_c_int] * 5),
    "p3d_qkv_gate_project": (_c_int, [_vp] * 11 + [_c_int] * 7 + [_vp] + [_c_int] * 3 + [_vp] + [_c_int] * 3 +
                             [_c_i64] * 2 + [ctypes.c_uint, _vp]),
    "p3d_qkv_project": (_c_int, [_vp] * 8 + [_c_int] * 7 + [_vp] + [_c_int] * 3 + [_vp] + [_c_int] * 3 + [_c_i64] * 2 +
                        [ctypes.c_uint, _vp]),
    "p3d_qkv_merge": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                               _vp, _c_int, _c_int, _c_int, _vp, _c_int, _c_int, _c_int, _vp]),
    "p3d_stencil_neighbors": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_i64, _vp, _vp, _vp,
                                       _c_int]),
    "p3d_repack_neighbors": (_c_int, [_c_i64, _c_int, _vp, _vp, _vp, _vp, _vp, _c_int]),
    "p3d_layer_norm_bwd_workspace": (ctypes.c_size_t, [_c_i64, _c_int]),
    "p3d_layer_norm_bwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_i64, _c_int, _c_f32, _vp,
                                    ctypes.c_size_t, _vp]),
    "p3d_layer_norm_bwd_residual": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_i64, _c_int, _c_f32,
                                             _vp, ctypes.c_size_t, _vp]),
    "p3d_pool_fwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _c_int,
                              _c_int, _c_int, _c_int, _c_int, _c_f32, _vp]),
    "p3d_attn_fwd": (_c_int, [ctypes.POINTER(Operator), _vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_uint,
                              _vp, ctypes.c_size_t, _vp]),
    "p3d_attn_fwd_workspace": (ctypes.c_size_t, [ctypes.POINTER(Operator), ctypes.c_uint]),
    "p3d_summary_bound": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp]),
    "p3d_stencil_fwd_supported": (_c_int, [_c_int] * 6),
    "p3d_attn_fwd_noalloc": (_c_int, [ctypes.POINTER(Operator), _vp, _vp, _vp, _vp]),
    "p3d_attn_fwd_slab": (_c_int, [ctypes.POINTER(Operator), ctypes.POINTER(Slab), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                   ctypes.c_uint, _vp]),
    "p3d_attn_bwd": (_c_int, [ctypes.POINTER(Operator), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                              _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "p3d_attn_bwd_workspace": (ctypes.c_size_t, [ctypes.POINTER(Operator)]),
    "p3d_peer_alloc": (_c_int, [ctypes.c_size_t, ctypes.POINTER(_vp), _vp]),
    "p3d_peer_free": (_c_int, [_vp]),
    "p3d_peer_open": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "p3d_peer_close": (_c_int, [_vp]),
    "p3d_peer_push": (_c_int, [ctypes.POINTER(PeerCopy), _c_int, _c_int, ctypes.POINTER(_vp), _c_int, _c_int, _vp]),
    "p3d_peer_wait": (_c_int, [_vp, _vp, ctypes.c_uint64, ctypes.c_double, _vp]),
    "p3d_peer_signal": (_c_int, [ctypes.POINTER(_vp), _c_int, _vp]),
    "p3d_bwd_mix": (_c_int, [ctypes.POINTER(Operator)] + [_vp] * 10 + [_vp, ctypes.c_size_t, _vp]),
    "p3d_bwd_mix_workspace": (ctypes.c_size_t, [ctypes.POINTER(Operator)]),
    "p3d_bwd_attn_slab": (_c_int, [ctypes.POINTER(Operator), ctypes.POINTER(Slab)] + [_vp] * 17 +
                          [_vp, ctypes.c_size_t, _vp]),
    "p3d_bwd_attn_slab_workspace": (ctypes.c_size_t, [ctypes.POINTER(Operator), ctypes.POINTER(Slab)]),
    "p3d_pool_bwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp,
                              _c_int, _c_int, _c_int, _c_int, _c_int, _c_f32, _vp, ctypes.c_size_t, _vp]),
    "p3d_pool_bwd_workspace": (ctypes.c_size_t, [_c_int] * 6),
}

_lock = threading.Lock()
_lib = None


def lib():
    """Load the native library once (raises if it is missing)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(f"pack3d_b200 native library missing at {LIB_PATH}; "
                                       "build it with `python -m pack3d_b200.build`")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (restype, argtypes) in _SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype, fn.argtypes = restype, argtypes
                _lib = handle
    return _lib


def check(status, what):
    if status != 0:
        handle = lib()
        detail = handle.p3d_last_error().decode(errors="replace")
        kind = handle.p3d_strerror(status).decode(errors="replace")
        error = ValueError if status in (1, 2) else RuntimeError
        raise error(f"{what}: {kind}: {detail}")


def ptr(t):
    """Device address of a tensor (or NULL for None)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def device_errors():
    """Read and clear the device-side failure flags (bit 0: a bounded wait timed out)."""
    flags = ctypes.c_uint(0)
    check(lib().p3d_device_errors(ctypes.byref(flags)), "p3d_device_errors")
    return flags.value


def exported_symbols():
    return tuple(_SIGNATURES)
