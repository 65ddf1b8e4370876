"""Host-side pieces of the layer glue, checked on the CPU in fp32.

``glue._Projections`` runs the three input projections of the layer (to_q, to_kv, gate) as
one autograd function that accumulates the input gradient inside its GEMMs; it must give
what autograd gives through three separate ``nn.Linear`` calls.  ``ops._token_major`` decides
whether an upstream gradient can enter the backward without a copy.
"""
import torch

from pack3d_b200 import glue
from pack3d_b200.ops import _token_major


def test_projections_match_three_linears():
    torch.manual_seed(0)
    dim, hq, hkv, hg = 24, 16, 32, 8
    to_q = torch.nn.Linear(dim, hq, bias=False)
    to_kv = torch.nn.Linear(dim, hkv, bias=False)
    gate = torch.nn.Linear(dim, hg)
    x = torch.randn(2, 5, dim, requires_grad=True)
    grads = [torch.randn(2, 5, c) for c in (hq, hkv, hg)]
    outs = glue.projections(x, to_q, to_kv, gate)
    torch.autograd.backward(outs, grads)
    got = [x.grad.clone()] + [p.grad.clone() for p in (to_q.weight, to_kv.weight, gate.weight, gate.bias)]
    for m in (to_q, to_kv, gate):
        m.zero_grad()
    x2 = x.detach().clone().requires_grad_()
    want_outs = (to_q(x2), to_kv(x2), gate(x2))
    for a, b in zip(outs, want_outs):
        torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-6)
    torch.autograd.backward(want_outs, grads)
    want = [x2.grad] + [p.grad for p in (to_q.weight, to_kv.weight, gate.weight, gate.bias)]
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-5)


def test_projections_with_unused_outputs():
    """Outputs that do not reach the loss get no gradient; the input gradient still forms."""
    torch.manual_seed(1)
    to_q, to_kv, gate = torch.nn.Linear(8, 8, bias=False), torch.nn.Linear(8, 16, bias=False), torch.nn.Linear(8, 4)
    x = torch.randn(1, 3, 8, requires_grad=True)
    qp, kvp, gl = glue.projections(x, to_q, to_kv, gate)
    qp.sum().backward()
    torch.testing.assert_close(x.grad, to_q.weight.sum(0).expand(1, 3, 8), atol=1e-6, rtol=1e-6)
    assert gate.bias.grad is None or not gate.bias.grad.any()


def test_token_major_detects_the_transposed_layout():
    b, n, h, d = 2, 7, 3, 4
    rows = torch.randn(b, n, h, d)
    assert _token_major(rows.transpose(1, 2))           # [B,H,N,D] view of [B,N,H,D]
    assert not _token_major(rows.transpose(1, 2).contiguous())
    assert not _token_major(torch.randn(b, h, n, d)[:, :, ::2])
