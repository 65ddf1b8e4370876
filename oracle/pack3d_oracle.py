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
    for start, stop in _chunk_rows(len(rows), chunk):
        r = rows[start:stop]
        qc = q[:, :, r].to(work)
        logits = (qc @ skr.transpose(-1, -2)) / root
        lg = torch.logsumexp(logits, -1)
        og = (logits - lg[..., None]).exp() @ svr
        ni = neighbors[r].long()
        ok = ni >= 0
        idx = ni.clamp_min(0)
        lk = kl[:, head_of][:, :, idx].to(work)
        lv = vl[:, head_of][:, :, idx].to(work)
        scores = (qc[..., None, :] * lk).sum(-1) / root
        scores = scores.masked_fill(~ok, -torch.inf)
        any_ok = ok.any(-1)[None, None, :]
        ll = torch.where(any_ok, torch.logsumexp(scores, -1), torch.full_like(scores[..., 0], -torch.inf))
        p = torch.where(any_ok[..., None], (scores - ll[..., None]).exp(), torch.zeros_like(scores))
        ol = (p[..., None] * lv).sum(-2)
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


# ------------------------------------------------------------------------- layer

LAYER_PARAMETERS = ("norm.weight", "norm.bias", "to_q.weight", "to_kv.weight", "pool_weight",
                    "slot_bias", "gate.weight", "gate.bias", "local_scale", "global_scale",
                    "to_out.weight")


def layer_forward(x, params, coords, neighbors, blocks, pool_size, *, heads, kv_heads, head_dim,
                  temperature=1.0, position_encoding="axial", chunk=None):
    """Whole PACK3D attention layer -- ``src/pack3d/attention.py:53-89``.

    LayerNorm, Q and 4-way KV projections, axial (or packed-sequence) RoPE of
    q / local k / global k, the 2-way gate softmax, the core, the output
    projection and the outer residual.  ``params`` maps the reference layer's
    state-dict names (``LAYER_PARAMETERS``) to tensors.
    """
    b, n, dim = x.shape
    residual = x
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
    gate = gates[..., 1].transpose(1, 2)
    out = pack3d_core(q, kl, vl, kg, vg, params["pool_weight"], params["slot_bias"], gate,
                      params["local_scale"], params["global_scale"], neighbors, blocks, pool_size,
                      temperature, chunk=chunk)
    return residual + F.linear(out.transpose(1, 2).reshape(b, n, -1), params["to_out.weight"])
