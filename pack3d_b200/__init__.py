"""pack3d_b200: a Blackwell (sm_100a) backend for the PACK3D attention operator.

Drop-in for the reference ``pack3d`` package's operator path: the same layer
(``PACK3DAttention``), geometry (``build_layout``, ``prepare_geometry``,
``TokenLayout``) and operator (``pack3d_streamed``) APIs, with every stage of
the hot path in hand-written CUDA behind the C-ABI library
``libpack3d_b200.so``.  There is no CPU path: compute entry points raise if
the native library or a CUDA device is missing.
"""
from .geometry import Pack3DGeometry, TokenLayout, build_layout, grid_coordinates, prepare_geometry

__version__ = "0.1.0"
__all__ = ["Pack3DGeometry", "TokenLayout", "build_layout", "grid_coordinates", "prepare_geometry"]
