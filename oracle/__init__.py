"""CPU oracle for the PACK3D operator -- TEST INFRASTRUCTURE ONLY.

This package is a plain restatement, on the CPU with PyTorch tensors, of the
reference's readable implementation of the hot path (``pack3d`` 0.1.0):

* axial RoPE .............. ``src/pack3d/rope.py:7-48``
* summary pooling ......... ``src/pack3d/compression.py:7-44``
* local + global core ..... ``src/pack3d/reference.py:8-31``
* layer glue .............. ``src/pack3d/attention.py:24-89``
* grid tables ............. ``src/pack3d/geometry.py:118-126,190-266``

It is pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``).  Only ``tests/``, ``__graft_entry__.smoke``
and the CPU-baseline / reference arms of ``bench.py`` may import it, and only
as the checker or as the timed CPU baseline -- never as the product path.
The product (``pack3d_b200``) never imports this package.
"""
from .pack3d_oracle import (  # noqa: F401
    axial_rope,
    balanced_pairs,
    compress_summaries,
    core_backward,
    core_backward_rows,
    core_forward,
    grid_layout,
    init_layer,
    layer_forward,
    morton_codes,
    pack3d_core,
)
