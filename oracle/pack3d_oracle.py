"""CPU restatement of the reference PACK3D hot path -- TEST INFRASTRUCTURE ONLY.

Every function names the reference lines it restates (paths are relative to
the reference project root).  The arithmetic follows the reference step for
step -- same working dtype (fp64 for fp64 inputs, else fp32), same operation
order for the rotations and the pooling -- but the attention core is
token-chunked so that grids far larger than the reference's dense guards
(``src/pack3d/reference.py:13-15``) fit in host memory.  Chunking changes no
per-row arithmetic: every output row depends only on its own scores.

``core_backward`` is an explicit, chunked restatement of the gradients that
autograd produces through ``pack3d_reference``; the CPU tests check it
against autograd on small shapes.

Nothing here touches a GPU.  The product package never imports this module.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _work_dtype(dtype):
    """fp64 stays fp64; every other floating dtype computes in fp32 (reference.py:17-18)."""
    return torch.float64 if dtype == torch.float64 else torch.float32


# --------------------------------------------------------------------- geometry

def morton_codes(coords):
    """Morton code of int64 ``[N, 3]`` coordinates -- ``src/pack3d/geometry.py:118-126``.

    Bit ``b`` of axis ``a`` lands at bit ``3 b + a``: axis 0 (z) takes the lowest bit of
    every triple.  The number of bit planes is that of the largest coordinate.
    """
    bits = int(coords.max()).bit_length()
    code = torch.zeros(len(coords), dtype=torch.int64)
    for bit in range(bits):
        for axis in range(3):
            code |= ((coords[:, axis] >> bit) & 1) << (3 * bit + axis)
    return code


def grid_layout(grid, block=(4, 4, 4), radius=2, storage="raster"):
    """Tables of a complete grid with cubic fine blocks, as the reference builds them.

    Restates ``build_layout(grid, block, radius=radius, layout="native_block_morton")``
    (``src/pack3d/geometry.py:224-266``): tokens sorted by the Morton code of their block
    and then of their slot inside the block; one neighbour column per offset of the
    ``(2r+1)^3`` cube in ``itertools.product`` order (z offset slowest), -1 where the
    neighbour leaves the grid; fine block ``f`` = packed rows ``[f V, (f+1) V)``.
    ``storage="raster"`` applies ``TokenLayout.repack(order.argsort())``
    (``geometry.py:190-220``): rows in raster order, block rows and slot columns kept,
    every index mapped to its raster row.  ``storage="morton"`` keeps the native order.

    Returns ``{"order", "coords", "neighbors", "blocks"}`` (int64, int64, int32, int32).
    """
    shape = tuple(int(v) for v in grid)
    block = tuple(int(v) for v in block)
    rad = (radius,) * 3 if isinstance(radius, int) else tuple(radius)
    if any(g % b for g, b in zip(shape, block)):
        raise ValueError("grid must be divisible by block")
    n = shape[0] * shape[1] * shape[2]
    raster = torch.stack(torch.meshgrid(*(torch.arange(s) for s in shape), indexing="ij"), -1).reshape(-1, 3)
    bt = torch.tensor(block)
    slot_code = morton_codes(raster % bt)
    order = (morton_codes(raster // bt) * (int(slot_code.max()) + 1) + slot_code).argsort()
    if storage == "raster":
        row_of = torch.arange(n)                       # raster index -> stored row
        coords = raster
        blocks = order.reshape(-1, block[0] * block[1] * block[2])
        stored_order = torch.arange(n)
    elif storage == "morton":
        row_of = order.argsort()
        coords = raster[order]
        blocks = torch.arange(n).reshape(-1, block[0] * block[1] * block[2])
        stored_order = order
    else:
        raise ValueError("storage must be raster or morton")
    extent = torch.tensor(shape)
    strides = torch.tensor([shape[1] * shape[2], shape[2], 1])
    columns = []
    for dz in range(-rad[0], rad[0] + 1):
        for dy in range(-rad[1], rad[1] + 1):
            for dx in range(-rad[2], rad[2] + 1):
                target = coords + torch.tensor((dz, dy, dx))
                valid = ((target >= 0) & (target < extent)).all(-1)
                index = (target * strides).sum(-1).clamp(0, n - 1)
                columns.append(torch.where(valid, row_of[index], -1))
    return {"order": stored_order, "coords": coords, "neighbors": torch.stack(columns, 1).to(torch.int32),
            "blocks": blocks.to(torch.int32)}


# --------------------------------------------------------------------------- RoPE

def balanced_pairs(head_dim):
    """Rotary pairs per (z, y, x) axis -- ``src/pack3d/rope.py:7-12``.

    The head dimension holds ``head_dim // 2`` planar pairs; they are dealt to
    the three axes as evenly as possible, the first axes taking the remainder.
    """
    if type(head_dim) is not int or head_dim <= 0 or head_dim % 2:
        raise ValueError("head_dim must be a positive even integer")
    total = head_dim // 2
    share, extra = divmod(total, 3)
    return tuple(share + (1 if axis < extra else 0) for axis in range(3))


def axial_rope(x, coords, pairs=None, base=10000.0, *, inverse=False):
    """Axial rotary embedding of ``[B, heads, N, D]`` -- ``src/pack3d/rope.py:15-48``.

    Axis ``a`` owns channel range ``[off_a, off_a + 2*pairs[a])`` laid out as
    interleaved (even, odd) pairs.  Pair ``i`` of that axis turns by
    ``coord_a * base ** (-i / pairs[a])`` radians, evaluated in the working
    dtype; the result is cast back to ``x.dtype``.  ``inverse`` applies the
    transposed rotation (the RoPE backward).
    """
    if pairs is None:
        pairs = balanced_pairs(x.shape[-1])
    pairs = tuple(pairs)
    if len(pairs) != 3 or sum(pairs) * 2 != x.shape[-1] or any(p < 0 for p in pairs):
        raise ValueError("pairs must allocate every rotary pair across three axes")
    work = _work_dtype(x.dtype)
    position = coords.to(work)
    pieces, offset = [], 0
    for axis, count in enumerate(pairs):
        if count == 0:
            continue
        seg = x[..., offset:offset + 2 * count].to(work).reshape(*x.shape[:-1], count, 2)
        frequency = base ** (-torch.arange(count, dtype=work) / count)
        angle = position[:, axis, None] * frequency
        cos, sin = angle.cos(), angle.sin()
        if inverse:
            sin = -sin
        even, odd = seg[..., 0], seg[..., 1]
        pieces.append(torch.stack((even * cos - odd * sin, even * sin + odd * cos), -1).flatten(-2))
        offset += 2 * count
    return torch.cat(pieces, -1).to(x.dtype)


# ----------------------------------------------------------------------- pooling

def compress_summaries(keys, values, weight, bias, blocks, pool_size, temperature=1.0):
    """Two-stage summary pooling -- ``src/pack3d/compression.py:7-44``.

    Fine stage: for fine block ``f`` with member slots ``blocks[f]`` (-1 =
    empty slot), ``a = softmax_slots(keys . weight / temperature + bias[slot])``
    over the valid slots; ``fine = sum a * member``.  Coarse stage: summary
    ``m`` is the mean of the fine summaries of the nonempty fine blocks
    ``[m*pool_size, (m+1)*pool_size)``.  Values are pooled with the same
    weights.  Differentiable.
    """
    work = _work_dtype(keys.dtype)
    index = blocks.long()
    valid = index >= 0
    k = keys.to(work)[:, :, index.clamp_min(0)]
    v = values.to(work)[:, :, index.clamp_min(0)]
    logits = (k * weight.to(work)).sum(-1) / temperature + bias.to(work)
    logits = logits.masked_fill(~valid, -torch.inf)
    fine_valid = valid.any(-1)
    logits = torch.where(fine_valid[None, None, :, None], logits, torch.zeros_like(logits))
    a = logits.softmax(-1) * valid
    fine_k = (a[..., None] * k).sum(-2)
    fine_v = (a[..., None] * v).sum(-2)
    pooled_k, pooled_v = [], []
    for start in range(0, index.shape[0], pool_size):
        stop = start + pool_size
        count = fine_valid[start:stop].sum()
        pooled_k.append(fine_k[:, :, start:stop].sum(2) / count)
        pooled_v.append(fine_v[:, :, start:stop].sum(2) / count)
    return torch.stack(pooled_k, 2), torch.stack(pooled_v, 2)


# ---------------------------------------------------------------- attention core

def _chunk_rows(n, chunk):
    chunk = n if not chunk else int(chunk)
    for start in range(0, n, chunk):
        yield start, min(n, start + chunk)


def pack3d_core(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, neighbors, blocks, pool_size,
                temperature=1.0, chunk=None):
    """Differentiable PACK3D core -- ``src/pack3d/reference.py:8-31``.

    ``y = sl * softmax_local(q kl^T / sqrt(D)) vl + gate * sg * softmax_global(q sk^T / sqrt(D)) sv``
    with two independent softmaxes, GQA by ``repeat_interleave`` of the KV
    heads, masked (-1) neighbours excluded and an all-masked local row giving
    zero.  Computes in fp32 (fp64 for fp64 inputs) and returns ``q.dtype``.
    """
    b, h, n, d = q.shape
    g = kl.shape[1]
    work = _work_dtype(q.dtype)
    qf, klf, vlf, kgf, vgf = (t.to(work) for t in (q, kl, vl, kg, vg))
    sk, sv = compress_summaries(kgf, vgf, weight, bias, blocks, pool_size, temperature)
    rep = h // g
    sk, sv = sk.repeat_interleave(rep, 1), sv.repeat_interleave(rep, 1)
    klr, vlr = klf.repeat_interleave(rep, 1), vlf.repeat_interleave(rep, 1)
    root = math.sqrt(d)
    slw, sgw = sl.to(work), sg.to(work)
    rows = []
    for start, stop in _chunk_rows(n, chunk):
        qc = qf[:, :, start:stop]
        og = ((qc @ sk.transpose(-1, -2)) / root).softmax(-1) @ sv
        ni = neighbors[start:stop].long()
        ok = ni >= 0
        lk = klr[:, :, ni.clamp_min(0)]
        lv = vlr[:, :, ni.clamp_min(0)]
        scores = (qc[..., None, :] * lk).sum(-1) / root
        scores = scores.masked_fill(~ok, -torch.inf)
        scores = torch.where(ok.any(-1)[None, None, :, None], scores, torch.zeros_like(scores))
        ol = (scores.softmax(-1)[..., None] * ok[..., None] * lv).sum(-2)
        rows.append(slw * ol + gate[:, :, start:stop].to(work)[..., None] * sgw * og)
    return torch.cat(rows, 2).to(q.dtype)


@torch.no_grad()
def core_forward(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, neighbors, blocks, pool_size,
                 temperature=1.0, chunk=4096, rows=None):
    """Forward of :func:`pack3d_core` with its intermediate state, chunked, no autograd.

    Returns a dict with ``y`` (in ``q.dtype``) and the working-precision
    intermediates ``ol, og, lse_l, lse_g, sk, sv``.  ``rows`` (a 1-D index
    tensor) restricts the query rows evaluated -- rows are independent given
    the summaries, so a sampled subset is exact for those rows.
    """
    b, h, n, d = q.shape
    g = kl.shape[1]
    work = _work_dtype(q.dtype)
    sk, sv = compress_summaries(kg.to(work), vg.to(work), weight, bias, blocks, pool_size, temperature)
    rep = h // g
    skr, svr = sk.repeat_interleave(rep, 1), sv.repeat_interleave(rep, 1)
    root = math.sqrt(d)
    slw, sgw = sl.to(work), sg.to(work)
    rows = torch.arange(n) if rows is None else rows.long()
    ys, ols, ogs, lls, lgs = [], [], [], [], []
    head_of = torch.arange(h) // rep
    klw, vlw = kl[:, head_of].to(work), vl[:, head_of].to(work)   # GQA: KV head of every query head
    for start, stop in _chunk_rows(len(rows), chunk):
        r = rows[start:stop]
        qc = q[:, :, r].to(work)
        logits = (qc @ skr.transpose(-1, -2)).div_(root)
        lg = torch.logsumexp(logits, -1)
        og = logits.sub_(lg[..., None]).exp_() @ svr
        ni = neighbors[r].long()
        ok = ni >= 0
        idx = ni.clamp_min(0)
        lk = klw[:, :, idx]                                          # [B, H, rows, W, D]
        lv = vlw[:, :, idx]
        scores = (lk @ qc[..., None]).squeeze(-1) / root
        scores = scores.masked_fill(~ok, -torch.inf)
        any_ok = ok.any(-1)[None, None, :]
        ll = torch.where(any_ok, torch.logsumexp(scores, -1), torch.full_like(scores[..., 0], -torch.inf))
        p = torch.where(any_ok[..., None], (scores - ll[..., None]).exp(), torch.zeros_like(scores))
        ol = (p[..., None, :] @ lv).squeeze(-2)
        ys.append(slw * ol + gate[:, :, r].to(work)[..., None] * sgw * og)
        ols.append(ol)
        ogs.append(og)
        lls.append(ll)
        lgs.append(lg)
    return {"y": torch.cat(ys, 2).to(q.dtype), "ol": torch.cat(ols, 2), "og": torch.cat(ogs, 2),
            "lse_l": torch.cat(lls, 2), "lse_g": torch.cat(lgs, 2), "sk": sk, "sv": sv}


def core_backward(dy, q, kl, vl, kg, vg, weight, bias, gate, sl, sg, neighbors, blocks, pool_size,
                  temperature=1.0, chunk=2048):
    """Explicit chunked gradients of :func:`pack3d_core` (first order).

    Restates what autograd computes through ``src/pack3d/reference.py:17-31``
    and ``src/pack3d/compression.py:28-44``:

    * mix: ``dOL = dy*sl``, ``dOG = dy*gate*sg``, ``dgate = sum_D dy*sg*og``,
      ``dsl = sum dy*ol``, ``dsg = sum dy*gate*og``;
    * each softmax branch: ``dS = P * (dP - rowsum(P*dP))`` with
      ``dP = dO V^T``; ``dQ = dS K / sqrt(D)``, ``dK = dS^T Q / sqrt(D)``,
      ``dV = P^T dO`` -- local dK/dV scattered back through the neighbour
      table, GQA heads summed onto their KV head;
    * pooling: autograd through :func:`compress_summaries` with the summed
      summary gradients.

    Returns ``(dq, dkl, dvl, dkg, dvg, dweight, dbias, dgate, dsl, dsg)`` in
    the dtypes of the corresponding inputs.
    """
    b, h, n, d = q.shape
    g = kl.shape[1]
    rep = h // g
    work = _work_dtype(q.dtype)
    root = math.sqrt(d)
    kgw = kg.detach().to(work).requires_grad_()
    vgw = vg.detach().to(work).requires_grad_()
    ww = weight.detach().to(work).requires_grad_()
    bw = bias.detach().to(work).requires_grad_()
    with torch.enable_grad():
        sk, sv = compress_summaries(kgw, vgw, ww, bw, blocks, pool_size, temperature)
    with torch.no_grad():
        skr, svr = sk.detach().repeat_interleave(rep, 1), sv.detach().repeat_interleave(rep, 1)
        klr = kl.to(work).repeat_interleave(rep, 1)
        vlr = vl.to(work).repeat_interleave(rep, 1)
        slw, sgw = sl.to(work), sg.to(work)
        dq = torch.zeros(b, h, n, d, dtype=work)
        dklr = torch.zeros(b, h, n, d, dtype=work)
        dvlr = torch.zeros(b, h, n, d, dtype=work)
        dskr = torch.zeros_like(skr)
        dsvr = torch.zeros_like(svr)
        dgate = torch.zeros(b, h, n, dtype=work)
        dsl = torch.zeros(d, dtype=work)
        dsg = torch.zeros(d, dtype=work)
        for start, stop in _chunk_rows(n, chunk):
            qc = q[:, :, start:stop].to(work)
            dyc = dy[:, :, start:stop].to(work)
            gc = gate[:, :, start:stop].to(work)[..., None]
            # global branch (reference.py:20-22)
            pg = ((qc @ skr.transpose(-1, -2)) / root).softmax(-1)
            og = pg @ svr
            # local branch (reference.py:23-30)
            ni = neighbors[start:stop].long()
            ok = ni >= 0
            idx = ni.clamp_min(0)
            lk, lv = klr[:, :, idx], vlr[:, :, idx]
            scores = (qc[..., None, :] * lk).sum(-1) / root
            scores = scores.masked_fill(~ok, -torch.inf)
            scores = torch.where(ok.any(-1)[None, None, :, None], scores, torch.zeros_like(scores))
            pl = scores.softmax(-1)
            a = pl * ok
            ol = (a[..., None] * lv).sum(-2)
            # mix (reference.py:31)
            dol = dyc * slw
            dog = dyc * gc * sgw
            dgate[:, :, start:stop] = (dyc * sgw * og).sum(-1)
            dsl += (dyc * ol).sum((0, 1, 2))
            dsg += (dyc * gc * og).sum((0, 1, 2))
            # global VJP
            dpg = dog @ svr.transpose(-1, -2)
            dsg_scores = pg * (dpg - (pg * dpg).sum(-1, keepdim=True)) / root
            dq[:, :, start:stop] += dsg_scores @ skr
            dskr += dsg_scores.transpose(-1, -2) @ qc
            dsvr += pg.transpose(-1, -2) @ dog
            # local VJP
            dpl = (dol[..., None, :] * lv).sum(-1) * ok
            dsl_scores = pl * (dpl - (pl * dpl).sum(-1, keepdim=True)) / root
            dq[:, :, start:stop] += (dsl_scores[..., None] * lk).sum(-2)
            flat = idx.reshape(-1)
            dklr.index_add_(2, flat, (dsl_scores[..., None] * qc[..., None, :]).reshape(b, h, -1, d))
            dvlr.index_add_(2, flat, (a[..., None] * dol[..., None, :]).reshape(b, h, -1, d))
        dsk = dskr.view(b, g, rep, -1, d).sum(2)
        dsv = dsvr.view(b, g, rep, -1, d).sum(2)
        dkl = dklr.view(b, g, rep, n, d).sum(2)
        dvl = dvlr.view(b, g, rep, n, d).sum(2)
    dkg, dvg, dweight, dbias = torch.autograd.grad((sk, sv), (kgw, vgw, ww, bw), (dsk, dsv))
    return (dq.to(q.dtype), dkl.to(kl.dtype), dvl.to(vl.dtype), dkg.to(kg.dtype), dvg.to(vg.dtype),
            dweight.to(weight.dtype), dbias.to(bias.dtype), dgate.to(gate.dtype),
            dsl.to(sl.dtype), dsg.to(sg.dtype))


@torch.no_grad()
def core_backward_rows(dy, q, kl, vl, kg, vg, weight, bias, gate, sl, sg, neighbors, blocks, pool_size, rows,
                       temperature=1.0, chunk=2048):
    """``dq`` and ``dgate`` of :func:`core_backward` for the query rows ``rows`` only.

    A query row's ``dq`` and ``dgate`` depend only on that row's scores, its upstream
    gradient and the (fixed) summaries, so the sampled rows are exact.  Same arithmetic as
    :func:`core_backward` (``reference.py:17-31`` under autograd).  Returns
    ``(dq [B, H, R, D], dgate [B, H, R])`` in the working precision.
    """
    b, h, n, d = q.shape
    g = kl.shape[1]
    rep = h // g
    work = _work_dtype(q.dtype)
    root = math.sqrt(d)
    sk, sv = compress_summaries(kg.to(work), vg.to(work), weight, bias, blocks, pool_size, temperature)
    skr, svr = sk.repeat_interleave(rep, 1), sv.repeat_interleave(rep, 1)
    klr = kl.to(work).repeat_interleave(rep, 1)
    vlr = vl.to(work).repeat_interleave(rep, 1)
    slw, sgw = sl.to(work), sg.to(work)
    rows = rows.long()
    dqs, dgates = [], []
    for start, stop in _chunk_rows(len(rows), chunk):
        r = rows[start:stop]
        qc, dyc = q[:, :, r].to(work), dy[:, :, r].to(work)
        gc = gate[:, :, r].to(work)[..., None]
        pg = ((qc @ skr.transpose(-1, -2)) / root).softmax(-1)
        og = pg @ svr
        idx_raw = neighbors[r].long()
        ok = idx_raw >= 0
        idx = idx_raw.clamp_min(0)
        lk, lv = klr[:, :, idx], vlr[:, :, idx]
        scores = (lk @ qc[..., None]).squeeze(-1) / root
        scores = scores.masked_fill(~ok, -torch.inf)
        scores = torch.where(ok.any(-1)[None, None, :, None], scores, torch.zeros_like(scores))
        pl = scores.softmax(-1)
        dol, dog = dyc * slw, dyc * gc * sgw
        dpg = dog @ svr.transpose(-1, -2)
        dq = (pg * (dpg - (pg * dpg).sum(-1, keepdim=True)) / root) @ skr
        dpl = (lv @ dol[..., None]).squeeze(-1) * ok
        dsl_scores = pl * (dpl - (pl * dpl).sum(-1, keepdim=True)) / root
        dq += (dsl_scores[..., None, :] @ lk).squeeze(-2)
        dqs.append(dq)
        dgates.append((dyc * sgw * og).sum(-1))
    return torch.cat(dqs, 2), torch.cat(dgates, 2)


# ------------------------------------------------------------------------- layer

LAYER_PARAMETERS = ("norm.weight", "norm.bias", "to_q.weight", "to_kv.weight", "pool_weight",
                    "slot_bias", "gate.weight", "gate.bias", "local_scale", "global_scale",
                    "to_out.weight")


def init_layer(dim, *, heads=4, kv_heads=2, head_dim=32, block_volume=8):
    """Freshly initialised parameters of the reference layer, by state-dict name.

    Restates the constructor ``src/pack3d/attention.py:24-51``: the same modules and
    initialisers created in the same order, so that after the same ``torch.manual_seed``
    the tensors are identical to the reference layer's (``LayerNorm``; ``to_q`` and
    ``to_kv`` without bias; ``pool_weight`` uniform in +-1/sqrt(head_dim); ``slot_bias``
    N(0, 0.02^2); the gate ``Linear`` with its bias zeroed; branch scales 1 and 0.25;
    ``to_out`` without bias).  Consumes the global RNG exactly as the constructor does.
    """
    norm = torch.nn.LayerNorm(dim)
    to_q = torch.nn.Linear(dim, heads * head_dim, bias=False)
    to_kv = torch.nn.Linear(dim, 4 * kv_heads * head_dim, bias=False)
    pool_weight = torch.empty(head_dim)
    torch.nn.init.uniform_(pool_weight, -1 / math.sqrt(head_dim), 1 / math.sqrt(head_dim))
    slot_bias = torch.empty(block_volume)
    torch.nn.init.normal_(slot_bias, std=0.02)
    gate = torch.nn.Linear(dim, heads * 2)
    torch.nn.init.zeros_(gate.bias)
    to_out = torch.nn.Linear(heads * head_dim, dim, bias=False)
    return {"norm.weight": norm.weight.detach(), "norm.bias": norm.bias.detach(),
            "to_q.weight": to_q.weight.detach(), "to_kv.weight": to_kv.weight.detach(),
            "pool_weight": pool_weight, "slot_bias": slot_bias, "gate.weight": gate.weight.detach(),
            "gate.bias": gate.bias.detach(), "local_scale": torch.ones(head_dim),
            "global_scale": torch.full((head_dim,), 0.25), "to_out.weight": to_out.weight.detach()}


def layer_forward(x, params, coords, neighbors, blocks, pool_size, *, heads, kv_heads, head_dim,
                  temperature=1.0, position_encoding="axial", chunk=None, rows=None, exact_output=False):
    """Whole PACK3D attention layer -- ``src/pack3d/attention.py:53-89``.

    LayerNorm, Q and 4-way KV projections, axial (or packed-sequence) RoPE of
    q / local k / global k, the 2-way gate softmax, the core, the output
    projection and the outer residual.  ``params`` maps the reference layer's
    state-dict names (``LAYER_PARAMETERS``) to tensors.

    ``rows`` (1-D token indices) evaluates the core and the output only for those query
    rows: the projections, RoPE and pooling still cover every token, and each output row
    depends only on them, so the sampled rows are exact.  That form runs without autograd.
    ``exact_output`` forms the output projection and the residual in the working precision
    and returns it unrounded (a checker for a fused GEMM that rounds once).
    """
    if rows is not None or exact_output:
        return _layer_rows(x, params, coords, neighbors, blocks, pool_size, heads=heads, kv_heads=kv_heads,
                           head_dim=head_dim, temperature=temperature, position_encoding=position_encoding,
                           chunk=chunk, rows=rows, exact_output=exact_output)
    b, n, dim = x.shape
    q, kl, vl, kg, vg, gate = _layer_projections(x, params, coords, heads=heads, kv_heads=kv_heads,
                                                 head_dim=head_dim, position_encoding=position_encoding)
    out = pack3d_core(q, kl, vl, kg, vg, params["pool_weight"], params["slot_bias"], gate,
                      params["local_scale"], params["global_scale"], neighbors, blocks, pool_size,
                      temperature, chunk=chunk)
    return x + F.linear(out.transpose(1, 2).reshape(b, n, -1), params["to_out.weight"])


def _layer_projections(x, params, coords, *, heads, kv_heads, head_dim, position_encoding):
    """LayerNorm, projections, RoPE and gate of ``attention.py:56-72`` for every token."""
    b, n, dim = x.shape
    xn = F.layer_norm(x, (dim,), params["norm.weight"], params["norm.bias"])
    q = F.linear(xn, params["to_q.weight"]).reshape(b, n, heads, head_dim).transpose(1, 2)
    kl, vl, kg, vg = (t.reshape(b, n, kv_heads, head_dim).transpose(1, 2)
                      for t in F.linear(xn, params["to_kv.weight"]).chunk(4, -1))
    if position_encoding == "packed":
        pairs = (head_dim // 2, 0, 0)
        seq = torch.arange(n)
        coords = torch.stack((seq, torch.zeros_like(seq), torch.zeros_like(seq)), -1)
    elif position_encoding == "axial":
        pairs = balanced_pairs(head_dim)
    else:
        raise ValueError("position_encoding must be axial or packed")
    q, kl, kg = (axial_rope(t, coords, pairs) for t in (q, kl, kg))
    gates = F.linear(xn, params["gate.weight"], params["gate.bias"]).reshape(b, n, heads, 2).softmax(-1)
    return q, kl, vl, kg, vg, gates[..., 1].transpose(1, 2)


@torch.no_grad()
def _layer_rows(x, params, coords, neighbors, blocks, pool_size, *, heads, kv_heads, head_dim, temperature,
                position_encoding, chunk, rows, exact_output):
    b, n, dim = x.shape
    q, kl, vl, kg, vg, gate = _layer_projections(x, params, coords, heads=heads, kv_heads=kv_heads,
                                                 head_dim=head_dim, position_encoding=position_encoding)
    rows = torch.arange(n) if rows is None else rows.long()
    state = core_forward(q, kl, vl, kg, vg, params["pool_weight"], params["slot_bias"], gate,
                         params["local_scale"], params["global_scale"], neighbors, blocks, pool_size, temperature,
                         chunk=chunk or 2048, rows=rows)
    out = state["y"].transpose(1, 2).reshape(b, len(rows), -1)
    if exact_output:
        work = _work_dtype(x.dtype)
        return x[:, rows].to(work) + F.linear(out.to(work), params["to_out.weight"].to(work))
    return x[:, rows] + F.linear(out, params["to_out.weight"])
