"""Projected-tensor contract checks of the operator boundary.

Mirrors the reference's ``src/pack3d/_validation.py:4-39`` (same messages, so
callers catching them keep working) with three deliberate differences:

* head dimension 48 is admitted -- the benchmark shape (three axes x eight
  rotary pairs); every head dimension the kernels support is listed in
  ``HEAD_DIMS``;
* the Triton register-tile budget (``_validation.py:22-24``) does not apply:
  the CUDA kernels stream slots and pool members, so any validated block table
  (<= 64 slots, pool <= 32) is accepted;
* the 32-bit indexing limit is replaced by the 64-bit addressing of the
  kernels (a tensor may hold up to 2**40 elements).
"""
import math

import torch

HEAD_DIMS = (16, 32, 48, 64, 128)
COMPUTE_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def validate_inputs(q, kl, vl, kg, vg, weight, bias, gate, sl, sg, geometry, temperature):
    geometry.check_unmodified()
    if q.ndim != 4 or min(q.shape) < 1:
        raise ValueError("Q must have shape [batch, query_heads, tokens, head_dim]")
    b, h, n, d = q.shape
    if kl.ndim != 4 or kl.shape[0] != b or kl.shape[2:] != (n, d):
        raise ValueError("local K has incompatible dimensions")
    if not 0 < kl.shape[1] <= h or h % kl.shape[1]:
        raise ValueError("query heads must be divisible by KV heads")
    if any(t.shape != kl.shape for t in (vl, kg, vg)):
        raise ValueError("all branch K/V tensors must have matching shapes")
    if any(t.dtype != q.dtype for t in (kl, vl, kg, vg)):
        raise ValueError("Q/K/V must have the same dtype")
    if d not in HEAD_DIMS:
        raise ValueError("supported head dimensions are 16, 32, 48, 64 and 128")
    if q.numel() >= 2**40:
        raise ValueError("shape exceeds the kernel indexing limit")
    if weight.shape != (d,) or bias.shape != (geometry.blocks.shape[1],):
        raise ValueError("pool scorer/slot bias shape mismatch")
    if gate.shape != (b, h, n) or sl.shape != (d,) or sg.shape != (d,):
        raise ValueError("gate or channelwise branch scale shape mismatch")
    if n != geometry.num_tokens:
        raise ValueError("geometry token count does not match Q")
    tensors = (q, kl, vl, kg, vg, weight, bias, gate, sl, sg, *geometry.tensors)
    if any(t.device != q.device for t in tensors):
        raise ValueError("all tensors and prepared geometry must be on the same device")
    if any(not t.is_floating_point() for t in tensors[:10]):
        raise ValueError("attention inputs must be floating point")
    if not math.isfinite(temperature) or temperature <= 0:
        raise ValueError("temperature must be finite and positive")


def check_cuda(q):
    """The backend runs only on CUDA sm_100 devices, in fp32 / fp16 / bf16."""
    if q.device.type != "cuda" or q.dtype not in COMPUTE_DTYPES:
        raise ValueError("b200 backend requires CUDA fp32/fp16/bf16 Q/K/V")
    major, _ = torch.cuda.get_device_capability(q.device)
    if major != 10:
        raise ValueError("b200 backend targets compute capability 10.x (sm_100a) devices")
