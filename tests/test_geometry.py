"""Geometry tables are bit-identical to the reference's (golden fixtures and digests)."""
import hashlib

import pytest
import torch

from pack3d_b200 import TokenLayout, build_layout, prepare_geometry
from pack3d_b200.geometry import grid_coordinates


def _sha(t):
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def _tables(layout):
    geom = layout.geometry
    return {"grid_shape": tuple(layout.grid_shape), "order": layout.order, "coords": layout.coords,
            "neighbors": geom.neighbors, "reverse_neighbors": geom.reverse_neighbors,
            "blocks": geom.blocks, "pool_size": geom.pool_size,
            "radius_one_grid": geom._radius_one_grid, "raster_to_packed": geom._raster_to_packed}


def _assert_same(actual, expected):
    assert set(actual) == set(expected)
    for key, want in expected.items():
        got = actual[key]
        if isinstance(want, str):                    # a SHA-256 digest of the reference table
            assert _sha(got) == want, key
        elif torch.is_tensor(want):
            assert got is not None and got.dtype == want.dtype and torch.equal(got, want), key
        else:
            assert got == want or (want is None and got is None), key


@pytest.mark.parametrize("key", ["r1_raster_4x4x8", "r1_native_4x4x8", "r2_native_8x8x8",
                                 "r_mixed_odd", "r1_native_16x16x16"])
def test_layouts_match_reference(golden, key):
    case = golden("layouts.pt")[key]
    layout = build_layout(*case["args"], **case["kwargs"])
    _assert_same(_tables(layout), case["tables"])
    _assert_same(_tables(layout.repack(case["perm"])), case["repacked"])
    _assert_same(_tables(layout.repack(layout.order.argsort())), case["raster"])


@pytest.mark.parametrize("grid", [16, 32])
def test_baseline_layout_digests(golden, grid):
    digests = golden("layout_digests.pt")
    native = build_layout((grid,) * 3, (4, 4, 4), radius=2, pool_size=1)
    _assert_same(_tables(native), digests[f"r2_b4_native_{grid}"])
    raster = native.repack(native.order.argsort())
    _assert_same(_tables(raster), digests[f"r2_b4_raster_{grid}"])


@pytest.mark.slow
def test_baseline_layout_digests_64(golden):
    digests = golden("layout_digests.pt")
    native = build_layout((64,) * 3, (4, 4, 4), radius=2, pool_size=1)
    _assert_same(_tables(native), digests["r2_b4_native_64"])
    raster = native.repack(native.order.argsort())
    _assert_same(_tables(raster), digests["r2_b4_raster_64"])


def test_stencil_tag_transport():
    layout = build_layout((8, 8, 8), (4, 4, 4), radius=2, pool_size=1)
    geom = layout.geometry
    assert geom.stencil == ((8, 8, 8), (2, 2, 2))
    torch.testing.assert_close(geom._stencil_map.long(), layout.order.argsort())
    raster = layout.repack(layout.order.argsort())
    assert raster.geometry.stencil == geom.stencil and raster.geometry._stencil_map is None
    p = torch.randperm(512, generator=torch.Generator().manual_seed(3))
    moved = raster.repack(p)
    torch.testing.assert_close(moved.geometry._stencil_map.long(), moved.order.argsort())
    custom = prepare_geometry(geom.neighbors, geom.blocks, 1)
    assert custom.stencil is None
    assert TokenLayout(layout.grid_shape, layout.order, layout.coords, custom).repack(p).geometry.stencil is None


def test_pack_roundtrip_and_transport():
    layout = build_layout((4, 4, 8), pool_size=2)
    grid = torch.randn(2, 4, 4, 8, 3)
    torch.testing.assert_close(layout.unpack(layout.pack(grid)), grid)
    p = torch.randperm(128)
    new = layout.repack(p)
    torch.testing.assert_close(new.pack(grid), layout.pack(grid)[:, p])
    torch.testing.assert_close(new.unpack(new.pack(grid)), grid)
    torch.testing.assert_close(new.coords[new.geometry.blocks.long()],
                               layout.coords[layout.geometry.blocks.long()])


@pytest.mark.parametrize("kwargs", [{"grid_shape": (3, 4, 4)}, {"radius": -1},
                                    {"block_shape": (0, 2, 2)}, {"layout": "unknown"},
                                    {"pool_size": True}, {"radius": 3}])
def test_bad_layout_rejected(kwargs):
    args = {"grid_shape": (4, 4, 4), **kwargs}
    with pytest.raises(ValueError):
        build_layout(**args)


def test_guards_and_mutation():
    layout = build_layout((2, 2, 2))
    with pytest.raises(ValueError, match="permutation"):
        layout.repack(torch.zeros(8, dtype=torch.int64))
    geom = layout.geometry
    with pytest.raises(ValueError, match="partition"):
        prepare_geometry(geom.neighbors, torch.zeros_like(geom.blocks), 4)
    with pytest.raises(ValueError, match="out-of-range"):
        prepare_geometry(geom.neighbors + 1000, geom.blocks, 4)
    with pytest.raises(ValueError, match="duplicate"):
        prepare_geometry(torch.zeros(8, 2, dtype=torch.int32), geom.blocks, 4)
    with pytest.raises(ValueError, match="empty coarse group"):
        blocks = torch.cat((torch.full((2, 8), -1, dtype=torch.int32), geom.blocks))
        prepare_geometry(geom.neighbors, blocks, 2)
    layout.coords[0, 0] += 1
    with pytest.raises(RuntimeError, match="changed"):
        layout.pack(torch.zeros(1, 2, 2, 2, 1))
    fresh = build_layout((4, 4, 4))
    fresh.geometry.neighbors[0, 0] = 1
    with pytest.raises(RuntimeError, match="changed"):
        fresh.geometry.check_unmodified()


def test_reverse_adjacency_of_custom_graph(golden):
    from cases import CORE_CASES, graph_case
    for name, n, d, b, h, g, volume, pool, dtype, seed, temperature, empty in CORE_CASES:
        _, nb, blocks = graph_case(n, d, b, h, g, volume, pool, dtype, seed, empty)
        geom = prepare_geometry(nb, blocks, pool)
        assert torch.equal(geom.reverse_neighbors, golden(f"core_{name}.pt")["reverse_neighbors"]), name


def test_grid_coordinates():
    c = grid_coordinates((2, 3, 4))
    assert c.shape == (24, 3) and c[5].tolist() == [0, 1, 1] and c[-1].tolist() == [1, 2, 3]


@pytest.mark.parametrize("grid,block,radius,pool,kind", [
    ((16, 16, 16), (4, 4, 4), 2, 1, "native_block_morton"),
    ((8, 12, 20), (4, 4, 4), 1, 4, "native_block_morton"),
    ((6, 12, 20), (1, 4, 4), 1, 4, "raster_block"),
    ((8, 8, 8), (2, 2, 2), (1, 2, 0), 2, "native_block_morton"),
    ((4, 4, 8), (2, 2, 2), 0, 1, "raster_block"),
])
def test_native_tables_equal_the_tensor_formulation(monkeypatch, grid, block, radius, pool, kind):
    """The library's host builders reproduce build_layout and repack bit for bit."""
    import pack3d_b200.geometry as geometry
    if geometry._native_geometry() is None:
        pytest.skip("library not built")
    native = build_layout(grid, block, radius=radius, pool_size=pool, layout=kind)
    perm = torch.randperm(native.geometry.num_tokens, generator=torch.Generator().manual_seed(sum(grid)))
    native_raster, native_random = native.repack(native.order.argsort()), native.repack(perm)
    monkeypatch.setattr(geometry, "_native_geometry", lambda: None)
    tensor = build_layout(grid, block, radius=radius, pool_size=pool, layout=kind)
    tensor_raster, tensor_random = tensor.repack(tensor.order.argsort()), tensor.repack(perm)
    for a, b in ((native, tensor), (native_raster, tensor_raster), (native_random, tensor_random)):
        assert torch.equal(a.order, b.order) and torch.equal(a.coords, b.coords)
        for x, y in zip(a.geometry.tensors, b.geometry.tensors):
            assert x.dtype == y.dtype == torch.int32 and torch.equal(x, y)
        assert a.geometry.stencil == b.geometry.stencil
        for tag in ("_stencil_map", "_raster_to_packed", "_radius_one_grid"):
            ta, tb = getattr(a.geometry, tag), getattr(b.geometry, tag)
            assert (ta is None and tb is None) or (torch.is_tensor(ta) and torch.equal(ta, tb)) or ta == tb
