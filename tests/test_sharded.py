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

from pack3d_b200.sharded import (SlabPeers, ZSlabs, exchange_halos, exchange_slab, gather_summaries, interior_tiles,
                                 release_peers, slab_layout)


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


@pytest.mark.parametrize("radius", [1, 2])
def test_interior_tiles_read_no_halo_plane(radius):
    """A tile in the interior range reads keys / values of the rank's own planes only (planes
    outside the volume are masked, not read); every tile outside it reads a halo plane."""
    grid = (64, 8, 8)
    for world in (1, 2, 4, 8):
        for rank in range(world):
            s = ZSlabs(grid, world, rank, radius=radius)
            begin, end = interior_tiles(s)
            for t in range(s.planes // 4):
                lo = max(0, s.z0 + 4 * t - radius)
                hi = min(grid[0], s.z0 + 4 * t + 4 + radius)
                own = s.z0 <= lo and hi <= s.z0 + s.planes
                assert own == (begin <= t < end), (world, rank, t)


def test_slab_layout_has_global_coordinates():
    slabs = ZSlabs((16, 8, 8), 2, 1)
    layout = slab_layout((16, 8, 8), slabs=slabs)
    assert layout.geometry.num_tokens == 8 * 8 * 8
    assert layout.coords[:, 0].min().item() == 8 and layout.coords[:, 0].max().item() == 15
    assert layout.geometry.stencil == ((8, 8, 8), (2, 2, 2))


@pytest.mark.parametrize("grid,world", [((16, 16, 16), 4), ((16, 8, 24), 2), ((32, 8, 8), 8)])
def test_slab_summaries_are_the_whole_volume_summaries(grid, world):
    """Every rank's summaries (rank-major after the gather) are the whole volume's 4x4x4 cubes,
    each exactly once, with the same members (global raster indices)."""
    from pack3d_b200 import build_layout
    whole = build_layout(grid, (4, 4, 4), radius=2, pool_size=1)
    whole = whole.repack(whole.order.argsort())
    want = {frozenset(row.tolist()) for row in whole.geometry.blocks}
    got = []
    for rank in range(world):
        s = ZSlabs(grid, world, rank)
        layout = slab_layout(grid, slabs=s)
        lo, _ = s.token_range()
        got += [frozenset((row + lo).tolist()) for row in layout.geometry.blocks]
    assert len(got) == len(want) and set(got) == want


def test_slab_layout_refuses_coarse_pooling():
    """A rank's coarse groups follow its own block order, not the whole volume's: refused."""
    slabs = ZSlabs((16, 16, 16), 4, 1)
    for pool in (2, 8):
        with pytest.raises(ValueError, match="pool_size=1"):
            slab_layout((16, 16, 16), pool_size=pool, slabs=slabs)


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
        # the one-batch exchange of the inference path gives the same tensors
        kl, vl = full[:, :, lo:hi].contiguous(), 2 * full[:, :, lo:hi]
        kx, vx, skx, svx = exchange_slab(kl, vl, summ, summ + 0.5, s)
        same = (torch.equal(kx, want) and torch.equal(vx, 2 * want) and torch.equal(skx, gathered)
                and torch.equal(svx, gathered + 0.5))
        out[rank] = (torch.equal(ext, want) and same, gathered[:, :, :, 0].flatten().tolist())
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


@pytest.mark.gpu
def test_slab_forward_tile_ranges_compose(cuda_device):
    """The slab forward run over ranges of its query tiles (the overlapped exchange's interior
    first, the tiles at the ends after) writes the same y as one launch over all of them."""
    from pack3d_b200 import _native
    from pack3d_b200.sharded import _SlabCall, pool_summaries, slab_forward
    grid, world = (48, 16, 24), 4   # 12 planes a rank: an interior tile in the middle ranks
    layout, inputs = _case(grid, torch.bfloat16, 12)
    dev = [t.to(cuda_device) for t in inputs]
    slabs = [ZSlabs(grid, world, r) for r in range(world)]
    layouts = [slab_layout(grid, slabs=s).to(cuda_device) for s in slabs]
    parts = [_slab_inputs(dev, s) for s in slabs]
    pooled = [pool_summaries(p[3], p[4], p[5], p[6], lay.geometry) for p, lay in zip(parts, layouts)]
    sk = torch.cat([p[0] for p in pooled], dim=2)
    sv = torch.cat([p[1] for p in pooled], dim=2)
    for s, lay, p in zip(slabs, layouts, parts):
        q, kl_ext, vl_ext, _, _, weight, bias, gate, sl, sg = p
        want, _ = slab_forward(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, lay.geometry, s, y_rows=True)
        begin, end = interior_tiles(s)
        call = _SlabCall(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, lay.geometry, s, 1.0, False, True)
        call.y.zero_()
        if begin < end:
            call.run(begin, end)
        begin, end = min(begin, end), max(begin, end)   # an empty interior: all tiles after
        lo_rows, hi_rows = begin * 4 * s.plane_tokens, end * 4 * s.plane_tokens
        assert torch.equal(call.y[:, :, lo_rows:hi_rows], want[:, :, lo_rows:hi_rows]), s.rank
        assert not call.y[:, :, :lo_rows].any() and not call.y[:, :, hi_rows:].any(), s.rank
        for t0, t1 in ((0, begin), (end, call.tiles_z)):
            if t0 < t1:
                call.run(t0, t1)
        assert torch.equal(call.y, want), s.rank
    assert _native.device_errors() == 0


def _emulated_exchange(grid, world, radius, b, g, d, m, dtype=torch.bfloat16):
    """Every rank's peer-exchange copy records applied to emulated regions (host byte arrays
    at made-up base addresses): the regions' views against what the NCCL batch gives."""
    import numpy as np
    es = torch.empty((), dtype=dtype).element_size()
    gen = torch.Generator().manual_seed(3)
    full_k = torch.randn(b, g, grid[0] * grid[1] * grid[2], d, generator=gen).to(dtype)
    full_v = torch.randn(full_k.shape, generator=gen).to(dtype)
    summ = [(torch.randn(b, g, m, d, generator=gen).to(dtype), torch.randn(b, g, m, d, generator=gen).to(dtype))
            for _ in range(world)]
    peers, inputs, regions = [], [], []
    for r in range(world):
        s = ZSlabs(grid, world, r, radius=radius)
        p = SlabPeers.__new__(SlabPeers)
        p.slabs, p.world, p.shape, p.row_bytes = s, world, (b, g, d, m), d * es
        rows_max = (s.planes + 2 * radius) * s.plane_tokens
        align = lambda v: -(-v // 4096) * 4096  # noqa: E731
        p.ext_bytes = align(b * g * rows_max * p.row_bytes)
        p.summ_bytes = align(b * g * world * m * p.row_bytes)
        p.offsets = {"k": p.HEADER, "v": p.HEADER + p.ext_bytes, "sk": p.HEADER + 2 * p.ext_bytes,
                     "sv": p.HEADER + 2 * p.ext_bytes + p.summ_bytes}
        p.nbytes = p.HEADER + 2 * p.ext_bytes + 2 * p.summ_bytes
        p.bases = [(q + 1) << 40 for q in range(world)]
        p.own = p.bases[r]
        lo, hi = s.token_range()
        peers.append(p)
        inputs.append((full_k[:, :, lo:hi].contiguous(), full_v[:, :, lo:hi].contiguous()) + summ[r])
        regions.append(np.zeros(p.nbytes, dtype=np.uint8))
    sources = [t for inp in inputs for t in inp]

    def src_bytes(addr, nbytes):
        for t in sources:
            base = t.data_ptr()
            if base <= addr and addr + nbytes <= base + t.numel() * es:
                flat = t.view(torch.uint8).flatten().numpy() if dtype != torch.bfloat16 else \
                    t.view(torch.int16).flatten().numpy().view(np.uint8)
                return flat[addr - base:addr - base + nbytes]
        raise AssertionError("copy source outside every input")

    for r in range(world):
        remote, local = peers[r]._copies(*inputs[r])
        for src, dst, rows, row_bytes, src_stride, dst_stride in remote + local:
            dst_rank = (dst >> 40) - 1
            assert (dst_rank != r) == ((src, dst, rows, row_bytes, src_stride, dst_stride) in remote)
            off = dst - peers[0].bases[dst_rank]
            for i in range(rows):
                chunk = src_bytes(src + i * src_stride, row_bytes)
                o = off + i * dst_stride
                assert 0 <= o and o + row_bytes <= peers[dst_rank].nbytes
                regions[dst_rank][o:o + row_bytes] = chunk
    for r in range(world):
        p, s = peers[r], peers[r].slabs
        region = torch.from_numpy(regions[r].view(np.int16)).view(dtype) if es == 2 else None
        rows = s.halo_planes * s.plane_tokens
        view = lambda key, n: region[p.offsets[key] // es:p.offsets[key] // es + b * g * n * d].view(b, g, n, d)  # noqa: E731
        pt = s.plane_tokens
        want = full_k[:, :, s.halo_z0 * pt:(s.halo_z0 + s.halo_planes) * pt]
        assert torch.equal(view("k", rows), want), r
        assert torch.equal(view("v", rows), full_v[:, :, s.halo_z0 * pt:(s.halo_z0 + s.halo_planes) * pt]), r
        assert torch.equal(view("sk", world * m), torch.cat([x[0] for x in summ], dim=2)), r
        assert torch.equal(view("sv", world * m), torch.cat([x[1] for x in summ], dim=2)), r


@pytest.mark.parametrize("world,radius", [(2, 2), (4, 2), (4, 1), (8, 2)])
def test_peer_exchange_copies_build_the_slab_buffers(world, radius):
    """The peer exchange's copy records (every rank's, applied to emulated regions) leave in
    each rank's region exactly its planes with the halo planes around them and every rank's
    summaries in rank order -- what the NCCL exchange hands the slab kernel."""
    _emulated_exchange((8 * world, 4, 6), world, radius, 2, 3, 8, 5)


@pytest.mark.gpu
def test_peer_wait_times_out_and_reports(cuda_device):
    """A peer wait on a counter that nothing raises gives up after its limit, sets the peer
    bits of the device error flags and leaves the context usable."""
    import ctypes
    from pack3d_b200 import _native
    lib = _native.lib()
    counter = torch.zeros(2, dtype=torch.int64, device=cuda_device)
    expected = torch.tensor([1, 0], dtype=torch.int64, device=cuda_device)
    _native.device_errors()
    with torch.cuda.device(cuda_device):
        _native.check(lib.p3d_peer_wait(counter.data_ptr(), expected.data_ptr(), 5, 0.05,
                                        _native.stream_of(cuda_device)), "p3d_peer_wait")
    torch.cuda.synchronize(cuda_device)
    assert _native.device_errors() == 33
    assert expected.tolist() == [6, 0]
    # a counter that is high enough passes at once; a signal raises the counters
    counter.fill_(6)
    targets = (ctypes.c_void_p * 2)(counter.data_ptr(), counter.data_ptr() + 8)
    with torch.cuda.device(cuda_device):
        stream = _native.stream_of(cuda_device)
        _native.check(lib.p3d_peer_wait(counter.data_ptr(), expected.data_ptr(), 1, 1.0, stream), "p3d_peer_wait")
        _native.check(lib.p3d_peer_signal(targets, 2, stream), "p3d_peer_signal")
    torch.cuda.synchronize(cuda_device)
    assert _native.device_errors() == 0
    assert counter.tolist() == [7, 7] and expected.tolist() == [7, 0]


@pytest.mark.gpu
def test_peer_push_copies_strided_rows_and_arrives(cuda_device):
    """p3d_peer_push on one device: strided rows land where the records say, untouched bytes
    stay, and every CTA adds one arrival to each target."""
    import ctypes
    from pack3d_b200 import _native
    lib = _native.lib()
    gen = torch.Generator(device=cuda_device).manual_seed(4)
    src = torch.randint(-2**15, 2**15, (6, 40), dtype=torch.int16, device=cuda_device, generator=gen)
    dst = torch.zeros(6, 64, dtype=torch.int16, device=cuda_device)
    small = torch.zeros(3, 16, dtype=torch.int16, device=cuda_device)
    counters = torch.zeros(2, dtype=torch.int64, device=cuda_device)
    copies = (_native.PeerCopy * 2)(
        _native.PeerCopy(src.data_ptr() + 16, dst.data_ptr() + 32, 6, 48, 80, 128),     # words 1-3 of each row
        _native.PeerCopy(src.data_ptr(), small.data_ptr(), 3, 32, 160, 32))              # rows 0, 2, 4: words 0-1
    targets = (ctypes.c_void_p * 2)(counters.data_ptr(), counters.data_ptr() + 8)
    with torch.cuda.device(cuda_device):
        _native.check(lib.p3d_peer_push(copies, 2, 1, targets, 2, 7, _native.stream_of(cuda_device)), "p3d_peer_push")
    torch.cuda.synchronize(cuda_device)
    want = torch.zeros_like(dst)
    want[:, 16:40] = src[:, 8:32]
    assert torch.equal(dst, want)
    assert torch.equal(small, src[0::2, :16])
    assert counters.tolist() == [7, 7]
    assert _native.device_errors() == 0


def _nccl_worker(rank, world, port, grid, out):
    from pack3d_b200 import _native
    from pack3d_b200.sharded import pool_summaries, sharded_core_forward, slab_forward, slab_peers
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
        # the overlapped exchange (interior tiles while the halo planes are in flight) gives
        # bit for bit what the one-batch exchange followed by one launch gives
        skr, svr = pool_summaries(cut(kg), cut(vg), weight, bias, lay.geometry)
        kx, vx, skx, svx = exchange_slab(cut(kl), cut(vl), skr, svr, s)
        y_one, _ = slab_forward(cut(q), kx, vx, skx, svx, weight, bias, cut(gate), sl, sg, lay.geometry, s)
        # the peer exchange's buffers equal the NCCL batch's
        kb, kg_, _, kd = kl.shape
        peers = slab_peers(s, kb, kg_, kd, skr.shape[2], kl.dtype, dev)
        got = [t.clone() for t in peers.exchange(cut(kl), cut(vl), skr, svr)]
        peers.release()
        same = torch.equal(y, y_one) and all(torch.equal(a, b) for a, b in zip(got, (kx, vx, skx, svx)))
        torch.cuda.synchronize(dev)
        out[rank] = (y.cpu(), _native.device_errors(), same)
        release_peers()
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
        y, errors, same = results[rank]
        s = ZSlabs(grid, world, rank)
        lo, hi = s.token_range()
        assert errors == 0 and same, rank
        assert (y.float() - y_full[:, :, lo:hi].float().cpu()).abs().max().item() <= 2e-2, rank


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_slab_backward_matches_the_whole_volume(cuda_device, world):
    """Every stage of the sharded backward, ranks emulated in turn (exchanges = slices)."""
    from cases import upstream
    from pack3d_b200 import _native
    from pack3d_b200 import ops as p3d_ops
    from pack3d_b200.sharded import (pool_summaries, slab_attention_backward, slab_forward, slab_mix_backward,
                                     slab_pool_backward)
    grid = (32, 16, 24)
    layout, inputs = _case(grid, torch.bfloat16, 12)
    dev = [t.to(cuda_device) for t in inputs]
    geom = layout.geometry.to(cuda_device)
    n = layout.geometry.num_tokens
    dy = upstream((1, 4, n, 48), torch.bfloat16, 12).to(cuda_device)
    _, saved = p3d_ops.forward(*dev, geom, 1.0, save_state=True)
    want = p3d_ops.backward(dy, dev, saved, geom, 1.0)

    slabs = [ZSlabs(grid, world, r) for r in range(world)]
    geoms = [slab_layout(grid, slabs=s).to(cuda_device).geometry for s in slabs]
    parts = [_slab_inputs(dev, s) for s in slabs]
    pooled = [pool_summaries(p[3], p[4], p[5], p[6], g) for p, g in zip(parts, geoms)]
    sk = torch.cat([p[0] for p in pooled], dim=2)
    sv = torch.cat([p[1] for p in pooled], dim=2)
    fwd, mix = [], []
    for s, g, p in zip(slabs, geoms, parts):
        q, kl_ext, vl_ext, kg, vg, weight, bias, gate, sl, sg = p
        _, state = slab_forward(q, kl_ext, vl_ext, sk, sv, weight, bias, gate, sl, sg, g, s, save_state=True)
        lo, hi = s.token_range()
        pt = s.plane_tokens
        kl_c = kl_ext[:, :, s.halo_lo * pt:(s.halo_lo + s.planes) * pt].contiguous()
        vl_c = vl_ext[:, :, s.halo_lo * pt:(s.halo_lo + s.planes) * pt].contiguous()
        fwd.append(state)
        mix.append(slab_mix_backward(dy[:, :, lo:hi].contiguous(), q, kl_c, vl_c, kg, vg, weight, bias, gate, sl, sg,
                                     state[2], state[3], g))
    # the exchanged halos, assembled from every rank's rows
    cat = lambda i: torch.cat([m[i] for m in mix], dim=2)  # noqa: E731
    dol_all, delta_l_all = cat(0), cat(2)
    q_all = dev[0]
    lse_l_all = torch.cat([f[4] for f in fwd], dim=2)
    dsk_sum = dsv_sum = 0
    per_rank = []
    for s, g, p, f, m in zip(slabs, geoms, parts, fwd, mix):
        q, kl_ext, vl_ext, kg, vg, weight, bias, gate, sl, sg = p
        pt = s.plane_tokens
        ext = slice(s.halo_z0 * pt, (s.halo_z0 + s.halo_planes) * pt)
        dq, dkl, dvl, dsk, dsv = slab_attention_backward(
            q, kl_ext, vl_ext, sk, sv, f[4], f[5], m[0], m[1], m[2], m[3], q_all[:, :, ext].contiguous(),
            dol_all[:, :, ext].contiguous(), lse_l_all[:, :, ext].contiguous(), delta_l_all[:, :, ext].contiguous(),
            weight, bias, gate, sl, sg, g, s)
        dsk_sum, dsv_sum = dsk_sum + dsk, dsv_sum + dsv
        per_rank.append((dq, dkl, dvl))
    m_rank = sk.shape[2] // world
    dw_sum = db_sum = dsl_sum = dsg_sum = 0
    tol = lambda t: 2e-2 * max(1.0, t.float().abs().max().item())  # noqa: E731
    for r, (s, g, p, m) in enumerate(zip(slabs, geoms, parts, mix)):
        lo, hi = s.token_range()
        rows = slice(r * m_rank, (r + 1) * m_rank)
        dkg, dvg, dw, db = slab_pool_backward(p[3], p[4], p[5], p[6], g, dsk_sum[:, :, rows], dsv_sum[:, :, rows])
        dq, dkl, dvl = per_rank[r]
        for name, got, ref in (("dq", dq, want[0]), ("dkl", dkl, want[1]), ("dvl", dvl, want[2]),
                               ("dkg", dkg, want[3]), ("dvg", dvg, want[4]), ("dgate", m[4], want[7])):
            ref = ref[:, :, lo:hi]
            assert (got.float() - ref.float()).abs().max().item() <= tol(ref), (name, r)
        dw_sum, db_sum = dw_sum + dw, db_sum + db
        dsl_sum, dsg_sum = dsl_sum + m[5], dsg_sum + m[6]
    for name, got, ref in (("dweight", dw_sum, want[5]), ("dbias", db_sum, want[6]), ("dsl", dsl_sum, want[8]),
                           ("dsg", dsg_sum, want[9])):
        assert (got.float() - ref.float()).abs().max().item() <= tol(ref) + 1e-3, name
    assert _native.device_errors() == 0


def _train_worker(rank, world, port, grid, out):
    from pack3d_b200 import PACK3DAttention, _native
    from pack3d_b200.sharded import sharded_layer_forward
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        torch.manual_seed(0)
        layer = PACK3DAttention(192, heads=4, kv_heads=4, head_dim=48, block_volume=64).to(dev, torch.bfloat16)
        n = grid[0] * grid[1] * grid[2]
        gen = torch.Generator().manual_seed(5)
        x_full = torch.randn(1, n, 192, generator=gen).to(torch.bfloat16)
        dy_full = torch.randn(1, n, 192, generator=gen).to(torch.bfloat16)
        s = ZSlabs(grid, world, rank)
        lay = slab_layout(grid, slabs=s).to(dev)
        lo, hi = s.token_range()
        with torch.inference_mode():   # the fused inference path (one exchange batch)
            y_inf = sharded_layer_forward(layer, x_full[:, lo:hi].to(dev), lay).cpu()
        x = x_full[:, lo:hi].to(dev).requires_grad_()
        y = sharded_layer_forward(layer, x, lay)
        y.backward(dy_full[:, lo:hi].to(dev))
        for p in layer.parameters():            # replicated parameters: sum the ranks' shares
            dist.all_reduce(p.grad)
        torch.cuda.synchronize(dev)
        out[rank] = (y.detach().cpu(), x.grad.cpu(), {k: p.grad.cpu() for k, p in layer.named_parameters()},
                     _native.device_errors(), y_inf)
        release_peers()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_training_step_over_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from pack3d_b200 import PACK3DAttention, build_layout
    world, grid = 2, (32, 16, 24)
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_train_worker, args=(world, _free_port(), grid, out), nprocs=world, join=True)
        results = dict(out)
    dev = torch.device("cuda", 0)
    layout = build_layout(grid, (4, 4, 4), radius=2, pool_size=1)
    layout = layout.repack(layout.order.argsort()).to(dev)
    torch.manual_seed(0)
    layer = PACK3DAttention(192, heads=4, kv_heads=4, head_dim=48, block_volume=64).to(dev, torch.bfloat16)
    n = grid[0] * grid[1] * grid[2]
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(1, n, 192, generator=gen).to(torch.bfloat16).to(dev).requires_grad_()
    dy = torch.randn(1, n, 192, generator=gen).to(torch.bfloat16).to(dev)
    y = layer(x, layout)
    y.backward(dy)
    tol = lambda t: 2e-2 * max(1.0, t.float().abs().max().item())  # noqa: E731
    for rank in range(world):
        y_r, dx_r, grads, errors, y_inf = results[rank]
        lo, hi = ZSlabs(grid, world, rank).token_range()
        assert errors == 0
        assert (y_r.float() - y[:, lo:hi].detach().float().cpu()).abs().max().item() <= tol(y)
        assert (y_inf.float() - y[:, lo:hi].detach().float().cpu()).abs().max().item() <= tol(y), rank
        assert (dx_r.float() - x.grad[:, lo:hi].float().cpu()).abs().max().item() <= tol(x.grad), rank
        for name, p in layer.named_parameters():
            assert (grads[name].float() - p.grad.float().cpu()).abs().max().item() <= tol(p.grad), (name, rank)


def _graph_worker(rank, world, port, grid, out):
    """The sharded inference layer captured in a CUDA graph (its NCCL point-to-point batch
    included) and replayed: the same output as the eager call, twice in a row."""
    from pack3d_b200 import PACK3DAttention, _native
    from pack3d_b200.sharded import sharded_layer_forward
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=datetime.timedelta(seconds=60))
    graph = None
    try:
        torch.manual_seed(0)
        layer = PACK3DAttention(192, heads=4, kv_heads=4, head_dim=48, block_volume=64).to(dev, torch.bfloat16)
        n = grid[0] * grid[1] * grid[2]
        x_full = torch.randn(1, n, 192, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
        s = ZSlabs(grid, world, rank)
        lay = slab_layout(grid, slabs=s).to(dev)
        lo, hi = s.token_range()
        x = x_full[:, lo:hi].to(dev)
        with torch.inference_mode():
            want = sharded_layer_forward(layer, x, lay).clone()
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for _ in range(2):
                    sharded_layer_forward(layer, x, lay)
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                y = sharded_layer_forward(layer, x, lay)
            got = []
            for _ in range(2):
                graph.replay()
                torch.cuda.synchronize(dev)
                got.append(y.clone())
        out[rank] = ([torch.equal(g, want) for g in got], _native.device_errors())
        del graph   # a graph holding the exchange is released before its peer regions
        graph = None
        release_peers()
    finally:
        del graph   # a graph holding NCCL calls is released before the process group
        dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_inference_layer_replays_as_a_cuda_graph():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, grid = 2, (32, 16, 24)
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_graph_worker, args=(world, _free_port(), grid, out), nprocs=world, join=True)
        results = dict(out)
    for rank in range(world):
        same, errors = results[rank]
        assert errors == 0
        assert all(same), rank
