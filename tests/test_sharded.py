"""z-slab sharding: partition, halo exchange and summary gather (CPU, gloo), the slab
forward against the whole-volume forward (one GPU, ranks emulated in turn), and the
sharded forward over NCCL (two GPUs)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pack3d_b200.sharded import ZSlabs, exchange_halos, gather_summaries, slab_layout


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_covers_the_volume_with_clipped_halos():
    grid = (32, 8, 12)
    for world in (1, 2, 4, 8):
        slabs = [ZSlabs(grid, world, r) for r in range(world)]
        assert [s.z0 for s in slabs] == [r * 32 // world for r in range(world)]
        assert sum(s.planes for s in slabs) == 32
        assert slabs[0].halo_lo == 0 and slabs[-1].halo_hi == 0
        for s in slabs[1:-1]:
            assert s.halo_lo == 2 and s.halo_hi == 2
        for s in slabs:
            assert s.halo_z0 == max(0, s.z0 - 2)
            assert s.halo_z0 + s.halo_planes == min(32, s.z0 + s.planes + 2)
    with pytest.raises(ValueError):
        ZSlabs((30, 8, 8), 2, 0)    # 15 planes: not whole 4-plane blocks
    with pytest.raises(ValueError):
        ZSlabs((32, 8, 8), 2, 2)


def test_slab_layout_has_global_coordinates():
    slabs = ZSlabs((16, 8, 8), 2, 1)
    layout = slab_layout((16, 8, 8), slabs=slabs)
    assert layout.geometry.num_tokens == 8 * 8 * 8
    assert layout.coords[:, 0].min().item() == 8 and layout.coords[:, 0].max().item() == 15
    assert layout.geometry.stencil == ((8, 8, 8), (2, 2, 2))


def _exchange_worker(rank, world, port, grid, out):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(0)
        full = torch.randn(2, 3, grid[0] * grid[1] * grid[2], 4, generator=gen)
        s = ZSlabs(grid, world, rank)
        lo, hi = s.token_range()
        ext = exchange_halos(full[:, :, lo:hi].contiguous(), s)
        pt = s.plane_tokens
        want = full[:, :, s.halo_z0 * pt:(s.halo_z0 + s.halo_planes) * pt]
        summ = torch.full((2, 3, 5, 4), float(rank))
        gathered = gather_summaries(summ)
        out[rank] = (torch.equal(ext, want), gathered[:, :, :, 0].flatten().tolist())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_halo_exchange_and_summary_gather_over_gloo(world):
    grid = (8 * world, 4, 6)
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_exchange_worker, args=(world, _free_port(), grid, out), nprocs=world, join=True)
        results = dict(out)
    for rank in range(world):
        ok, gathered = results[rank]
        assert ok, rank
        assert gathered == [float(r) for _ in range(2 * 3) for r in range(world) for _ in range(5)]


# ----------------------------------------------------------------------------- GPU


def _case(grid, dtype, seed):
    import oracle
    from cases import grid_inputs
    from pack3d_b200 import build_layout
    layout = build_layout(grid, (4, 4, 4), radius=2, pool_size=1)
    layout = layout.repack(layout.order.argsort())
    raw = grid_inputs(layout.geometry.num_tokens, 1, 4, 4, 48, torch.float32, seed, True)
    rot = [oracle.axial_rope(raw[i], layout.coords) if i in (0, 1, 3) else raw[i] for i in range(5)]
    return layout, [t.to(dtype) for t in rot] + raw[5:]


def _slab_inputs(inputs, s):
    """This rank's rows of every per-token input, and the halo-extended kl / vl."""
    lo, hi = s.token_range()
    pt = s.plane_tokens
    q, kl, vl, kg, vg, weight, bias, gate, sl, sg = inputs
    cut = lambda t: t[:, :, lo:hi].contiguous()  # noqa: E731
    ext = lambda t: t[:, :, s.halo_z0 * pt:(s.halo_z0 + s.halo_planes) * pt].contiguous()  # noqa: E731
    return (cut(q), ext(kl), ext(vl), cut(kg), cut(vg), weight, bias, cut(gate), sl, sg)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_slab_forward_matches_the_whole_volume(cuda_device, world):
    from pack3d_b200 import _native
    from pack3d_b200 import ops as p3d_ops
    from pack3d_b200.sharded import pool_summaries, slab_forward
    grid = (32, 16, 24)
    layout, inputs = _case(grid, torch.bfloat16, 11)
    dev = [t.to(cuda_device) for t in inputs]
    y_full, _ = p3d_ops.forward(*dev, layout.geometry.to(cuda_device), 1.0, save_state=False)
    slabs = [ZSlabs(grid, world, r) for r in range(world)]
    layouts = [slab_layout(grid, slabs=s).to(cuda_device) for s in slabs]
    parts = [_slab_inputs(dev, s) for s in slabs]
    pooled = [pool_summaries(p[3], p[4], p[5], p[6], lay.geometry) for p, lay in zip(parts, layouts)]
    sk = torch.cat([p[0] for p in pooled], dim=2)
    sv = torch.cat([p[1] for p in pooled], dim=2)
    for s, lay, p in zip(slabs, layouts, parts):
        q, kl_ext, vl_ext, _, _, weight, bias, gate, sl, sg = p
        y, _ = slab_forward(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, lay.geometry, s)
        lo, hi = s.token_range()
        assert (y.float() - y_full[:, :, lo:hi].float()).abs().max().item() <= 2e-2, s.rank
    assert _native.device_errors() == 0


def _nccl_worker(rank, world, port, grid, out):
    from pack3d_b200 import _native
    from pack3d_b200.sharded import sharded_core_forward
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        layout, inputs = _case(grid, torch.bfloat16, 11)
        s = ZSlabs(grid, world, rank)
        lay = slab_layout(grid, slabs=s).to(dev)
        lo, hi = s.token_range()
        q, kl, vl, kg, vg, weight, bias, gate, sl, sg = [t.to(dev) for t in inputs]
        cut = lambda t: t[:, :, lo:hi].contiguous()  # noqa: E731
        y = sharded_core_forward(cut(q), cut(kl), cut(vl), cut(kg), cut(vg), weight, bias, cut(gate), sl, sg,
                                 lay.geometry, s)
        torch.cuda.synchronize(dev)
        out[rank] = (y.cpu(), _native.device_errors())
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_forward_over_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from pack3d_b200 import ops as p3d_ops
    world, grid = 2, (32, 16, 24)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_nccl_worker, args=(world, _free_port(), grid, out), nprocs=world, join=True)
        results = dict(out)
    layout, inputs = _case(grid, torch.bfloat16, 11)
    dev = torch.device("cuda", 0)
    y_full, _ = p3d_ops.forward(*[t.to(dev) for t in inputs], layout.geometry.to(dev), 1.0, save_state=False)
    for rank in range(world):
        y, errors = results[rank]
        s = ZSlabs(grid, world, rank)
        lo, hi = s.token_range()
        assert errors == 0
        assert (y.float() - y_full[:, :, lo:hi].float().cpu()).abs().max().item() <= 2e-2, rank
