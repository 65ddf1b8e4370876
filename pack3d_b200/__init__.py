"""pack3d_b200: a Blackwell (sm_100a) backend for the PACK3D attention operator.

Drop-in for the reference ``pack3d`` package's operator path: the same layer
(``PACK3DAttention``), geometry (``build_layout``, ``prepare_geometry``,
``TokenLayout``) and operator (``pack3d_streamed``, ``rotate_projections``)
APIs, with every stage of the hot path in hand-written CUDA behind the C-ABI
library ``lib/libpack3d_b200.so``.  There is no CPU path: compute entry points
raise if the native library or a CUDA sm_100 device is missing.
"""
from .attention import PACK3DAttention
from .geometry import Pack3DGeometry, TokenLayout, build_layout, grid_coordinates, prepare_geometry
from .ops import pack3d_streamed
from .rope import balanced_pairs, rotate_projections

__version__ = "0.1.0"
__all__ = ["PACK3DAttention", "Pack3DGeometry", "TokenLayout", "balanced_pairs", "build_layout",
           "grid_coordinates", "pack3d_streamed", "prepare_geometry", "rotate_projections"]
