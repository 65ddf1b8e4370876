"""Summary pooling through the C ABI (``p3d_pool_fwd`` / ``p3d_pool_bwd``).

For 16-bit rows whose base pointers are 16-byte aligned and whose head_dim is a multiple of
8, the pooling kernels stage each fine block's member rows in shared memory (16-byte
gathers, persistent warps); otherwise they read rows directly with scalar loads.  The slot
softmax and the per-slot gradient dots take the same arithmetic in the same order on both
paths, so dK, dV and dbias agree bit for bit; the weighted member sums and dweight add slot
groups in a different order, so summaries and dweight agree to fp32 rounding.  A
2-byte-shifted copy of the same data forces the direct path.  Both paths are also checked
against the oracle's pooling (``compress_summaries``, the restatement of
compression.py:7-44) in float64.
"""
import pytest
import torch

from oracle import pack3d_oracle as oracle
from pack3d_b200 import _native

pytestmark = pytest.mark.gpu

# (name, batch, kv_heads, tokens, head_dim, fine blocks, slots, pool_size, empty fraction, temperature)
CASES = [
    ("config1_like", 1, 4, 8192, 48, 128, 64, 1, 0.0, 1.0),
    ("ragged_pool3", 2, 2, 6000, 48, 90, 64, 3, 0.35, 0.7),
    ("slots27_d64", 1, 3, 4000, 64, 140, 27, 2, 0.2, 1.3),
    ("slots40_d128", 2, 1, 3000, 128, 60, 40, 4, 0.5, 1.0),
    ("d8_slots1", 1, 2, 500, 8, 300, 1, 5, 0.3, 1.0),
]


def _blocks(fine, slots, tokens, pool, empty, seed):
    """Disjoint member rows with empty slots; one all-empty fine block per coarse group of
    two or more (never the group's first, so every group keeps a nonempty block)."""
    g = torch.Generator().manual_seed(seed)
    idx = torch.randperm(tokens, generator=g)[: fine * slots].view(fine, slots).to(torch.int32)
    drop = torch.rand(fine, slots, generator=g) < empty
    drop[::pool, 0] = False
    idx[drop] = -1
    if pool >= 2:
        idx[1::pool] = -1
    return idx


def _shifted(t):
    """The same values in a buffer whose first element sits 2 bytes past a 16-byte boundary."""
    buf = torch.empty(t.numel() + 8, dtype=t.dtype, device=t.device)
    view = buf[1:1 + t.numel()].view(t.shape)
    view.copy_(t)
    assert view.data_ptr() % 16 != 0
    return view


def _pool_fwd(k, v, w, b, blocks, pool, temperature):
    bsz, g, n, d = k.shape
    fine, slots = blocks.shape
    m = (fine + pool - 1) // pool
    sk = torch.empty((bsz, g, m, d), dtype=k.dtype, device=k.device)
    sv = torch.empty_like(sk)
    sk32 = torch.empty(sk.shape, dtype=torch.float32, device=k.device)
    sv32 = torch.empty_like(sk32)
    status = _native.lib().p3d_pool_fwd(
        _native.ptr(k), _native.ptr(v), _native.ptr(w), _native.ptr(b), _native.ptr(blocks), fine, slots, pool,
        _native.ptr(sk), _native.ptr(sv), _native.ptr(sk32), _native.ptr(sv32), _native.DTYPE_CODE[k.dtype],
        bsz, g, n, d, float(temperature), _native.stream_of(k.device))
    _native.check(status, "p3d_pool_fwd")
    return sk, sv, sk32, sv32


def _pool_bwd(k, v, w, b, blocks, pool, dsk, dsv, temperature, shift_out=False):
    bsz, g, n, d = k.shape
    fine, slots = blocks.shape
    lib = _native.lib()
    dk = torch.zeros_like(k)
    dv = torch.zeros_like(v)
    if shift_out:
        dk, dv = _shifted(dk), _shifted(dv)
    dw = torch.empty(d, dtype=torch.float32, device=k.device)
    db = torch.empty(slots, dtype=torch.float32, device=k.device)
    need = lib.p3d_pool_bwd_workspace(fine, slots, pool, bsz, g, d)
    ws = torch.empty(need, dtype=torch.uint8, device=k.device)
    status = lib.p3d_pool_bwd(
        _native.ptr(k), _native.ptr(v), _native.ptr(w), _native.ptr(b), _native.ptr(blocks), fine, slots, pool,
        _native.ptr(dsk), _native.ptr(dsv), _native.ptr(dk), _native.ptr(dv), _native.ptr(dw), _native.ptr(db),
        _native.DTYPE_CODE[k.dtype], bsz, g, n, d, float(temperature), _native.ptr(ws), need,
        _native.stream_of(k.device))
    _native.check(status, "p3d_pool_bwd")
    return dk, dv, dw, db


def _case(case, dtype, device):
    name, bsz, g, n, d, fine, slots, pool, empty, temperature = case
    seed = sum(map(ord, name))
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn(bsz, g, n, d, generator=gen).to(dtype)
    v = torch.randn(bsz, g, n, d, generator=gen).to(dtype)
    w = torch.randn(d, generator=gen) * 0.3
    b = torch.randn(slots, generator=gen) * 0.5
    blocks = _blocks(fine, slots, n, pool, empty, seed)
    m = (fine + pool - 1) // pool
    dsk = torch.randn(bsz, g, m, d, generator=gen)
    dsv = torch.randn(bsz, g, m, d, generator=gen)
    host = dict(k=k, v=v, w=w, b=b, blocks=blocks, dsk=dsk, dsv=dsv, pool=pool, temperature=temperature)
    dev = {key: (t.to(device) if torch.is_tensor(t) else t) for key, t in host.items()}
    return host, dev


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_pool_staged_and_direct_paths_agree(cuda_device, case, dtype):
    _, c = _case(case, dtype, cuda_device)
    args = (c["w"], c["b"], c["blocks"], c["pool"])
    staged = _pool_fwd(c["k"], c["v"], *args, c["temperature"])
    direct = _pool_fwd(_shifted(c["k"]), _shifted(c["v"]), *args, c["temperature"])
    for nm, a, b in zip(("sk32", "sv32"), staged[2:], direct[2:]):
        assert (a - b).abs().max().item() <= 2e-6 * max(1.0, b.abs().max().item()), nm
    for nm, a, b in zip(("sk", "sv"), staged[:2], direct[:2]):  # at most one rounding step apart
        assert ((a.float() - b.float()).abs() <= b.float().abs() * 2 ** -7 + 1e-6).all(), nm
    grads = (c["dsk"], c["dsv"], c["temperature"])
    staged = _pool_bwd(c["k"], c["v"], *args, *grads)
    direct = _pool_bwd(_shifted(c["k"]), _shifted(c["v"]), *args, *grads, shift_out=True)
    for nm, a, b in zip(("dk", "dv", "dweight", "dbias"), staged, direct):
        a, b = a.contiguous(), b.contiguous()
        if nm == "dweight":
            assert (a - b).abs().max().item() <= 1e-5 * max(1.0, b.abs().max().item()), nm
        else:
            assert torch.equal(a, b), nm


def test_pool_staged_is_deterministic(cuda_device):
    _, c = _case(CASES[1], torch.bfloat16, cuda_device)
    args = (c["k"], c["v"], c["w"], c["b"], c["blocks"], c["pool"])
    first = _pool_fwd(*args, c["temperature"]) + _pool_bwd(*args, c["dsk"], c["dsv"], c["temperature"])
    again = _pool_fwd(*args, c["temperature"]) + _pool_bwd(*args, c["dsk"], c["dsv"], c["temperature"])
    for a, b in zip(first, again):
        assert torch.equal(a, b)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_pool_matches_oracle(cuda_device, case):
    h, c = _case(case, torch.bfloat16, cuda_device)
    sk, sv, sk32, sv32 = _pool_fwd(c["k"], c["v"], c["w"], c["b"], c["blocks"], c["pool"], c["temperature"])
    leaves = [h["k"].double().requires_grad_(), h["v"].double().requires_grad_(),
              h["w"].double().requires_grad_(), h["b"].double().requires_grad_()]
    want_k, want_v = oracle.compress_summaries(*leaves, h["blocks"], h["pool"], h["temperature"])
    # fp32 accumulation of bf16 members; the bf16 outputs add one rounding (2^-8 relative)
    assert (sk32.cpu().double() - want_k).abs().max() <= 1e-5
    assert (sv32.cpu().double() - want_v).abs().max() <= 1e-5
    assert (sk.cpu().double() - want_k).abs().max() <= 2e-2
    assert (sv.cpu().double() - want_v).abs().max() <= 2e-2
    grads = torch.autograd.grad((want_k * h["dsk"].double()).sum() + (want_v * h["dsv"].double()).sum(), leaves)
    got = _pool_bwd(c["k"], c["v"], c["w"], c["b"], c["blocks"], c["pool"], c["dsk"], c["dsv"], c["temperature"])
    member = torch.zeros(h["k"].shape[2], dtype=torch.bool)
    member[h["blocks"][h["blocks"] >= 0].long()] = True
    for nm, a, want in zip(("dk", "dv", "dweight", "dbias"), got, grads):
        a = a.cpu().double()
        if nm in ("dk", "dv"):
            assert not a[:, :, ~member].any(), nm  # rows outside every block stay untouched (zero)
        scale = max(1.0, want.abs().max().item())
        tol = 2e-2 if nm in ("dk", "dv") else 1e-4
        assert (a - want).abs().max() <= tol * scale, (nm, (a - want).abs().max().item())
