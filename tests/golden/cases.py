"""Seeded input recipes shared by the fixture generator and the tests.

The golden fixtures store only what the reference computed (outputs,
gradients, tables); the inputs are regenerated here from fixed seeds with
``torch.Generator`` on the CPU, so both sides see identical tensors.
"""
import torch


def graph_case(n, d, b, h, g, volume, pool, dtype, seed, empty_block=False):
    """Custom-graph case: an asymmetric 3-edge neighbour graph whose row 0 is
    all-masked, a ragged last fine block, and scaled inputs (gate in (0, 1),
    local scale near 1, global scale near 0.25).

    Returns ``(inputs, neighbors, blocks)``; ``inputs`` is the 10-tuple
    ``q, kl, vl, kg, vg, weight, bias, gate, sl, sg``.
    """
    gen = torch.Generator().manual_seed(seed)
    nb = torch.full((n, 5), -1, dtype=torch.int32)
    for i in range(n):
        edges = sorted({i, (i + 1) % n, max(i - 2, 0)})
        nb[i, :len(edges)] = torch.tensor(edges)
    nb[0] = -1
    blocks = torch.full(((n + volume - 1) // volume, volume), -1, dtype=torch.int32)
    blocks.flatten()[:n] = torch.arange(n)
    if empty_block:                       # a leading fine block with no member at all
        blocks = torch.cat((torch.full((1, volume), -1, dtype=torch.int32), blocks))
    shapes = [(b, h, n, d)] + [(b, g, n, d)] * 4 + [(d,), (volume,), (b, h, n), (d,), (d,)]
    inputs = []
    for index, shape in enumerate(shapes):
        t = torch.randn(shape, generator=gen) * (0.2 if index in (5, 6) else 0.5)
        if index == 7:
            t = t.sigmoid()
        if index == 8:
            t += 1
        if index == 9:
            t += 0.25
        inputs.append(t.to(dtype))
    return inputs, nb, blocks


def grid_inputs(n, b, h, g, d, dtype, seed, weighted, volume=64):
    """Pre-RoPE projections and operator parameters for a grid case.

    Unweighted cases use the benchmark settings: mean pooling (weight 0, slot
    bias 0), gate 0.5 and the layer's initial branch scales (1 and 0.25).
    """
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, n, d, generator=gen)
    kl, vl, kg, vg = (torch.randn(b, g, n, d, generator=gen) for _ in range(4))
    if weighted:
        weight = torch.randn(d, generator=gen) * 0.3
        bias = torch.randn(volume, generator=gen) * 0.1
        gate = torch.rand(b, h, n, generator=gen)
        sl = 1 + 0.1 * torch.randn(d, generator=gen)
        sg = 0.25 + 0.1 * torch.randn(d, generator=gen)
    else:
        weight, bias = torch.zeros(d), torch.zeros(volume)
        gate = torch.full((b, h, n), 0.5)
        sl, sg = torch.ones(d), torch.full((d,), 0.25)
    return [t.to(dtype) for t in (q, kl, vl, kg, vg, weight, bias, gate, sl, sg)]


def upstream(shape, dtype, seed):
    """Upstream gradient ``dy`` for a case generated with ``seed``."""
    return torch.randn(shape, generator=torch.Generator().manual_seed(seed + 1)).to(dtype)


# (name, n, d, b, h, g, volume, pool, dtype, seed, temperature, empty_block)
CORE_CASES = [
    ("d16_f64", 37, 16, 2, 4, 2, 4, 3, torch.float64, 18, 0.7, False),
    ("d16_f32", 37, 16, 2, 4, 2, 4, 3, torch.float32, 18, 0.7, False),
    ("d48_f32", 41, 48, 1, 4, 2, 8, 2, torch.float32, 19, 1.0, False),
    ("d48_bf16", 41, 48, 1, 4, 2, 8, 2, torch.bfloat16, 20, 1.0, False),
    ("d64_f32_empty", 131, 64, 1, 4, 2, 16, 2, torch.float32, 21, 0.7, True),
]

# (name, grid, b, h, g, d, dtype, seed, weighted)
GRID_CASES = [
    ("844_d48_mean_f32", (8, 4, 4), 1, 2, 2, 48, torch.float32, 0, False),
    ("848_d48_gqa_f32", (8, 4, 8), 1, 4, 2, 48, torch.float32, 5, True),
]
