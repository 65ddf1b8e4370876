#!/usr/bin/env python
"""PACK3D layer benchmark on B200: bf16 forward tokens/s at 262,144 tokens.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One JSON line on rank 0.  A step is one forward of the whole ``PACK3DAttention``
layer (LayerNorm, projections, RoPE, pooling, fused local + global attention,
output projection, residual) over the 64^3 field, inputs resident in HBM, timed
with CUDA events per step (L2 flushed between steps, outside the timed events),
max over ranks.  ``e2e`` times the same public call with the input copied from
pinned host memory and the output read back every step, as a streaming pipeline
(copy-in, compute and copy-out on three streams).  ``roofline`` is the
fused stencil kernel (stage c) timed alone with CUDA events on its stream;
``cpu_baseline`` is the CPU restatement of the reference path on this host.

``--impl reference`` times the reference's CPU path (the CPU restatement; the
reference itself is Python/Triton and refuses head_dim 48) on the host cores.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "PACK3D layer bf16 fwd and fwd+bwd ms (tokens/s) at 262,144 tokens; 1-8 GPU"
CONFIG = dict(grid=(64, 64, 64), batch=1, heads=4, kv_heads=4, head_dim=48, dim=192, block=(4, 4, 4), radius=2,
              pool_size=1)
L2_FLUSH_BYTES = 256 * 1024 * 1024


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-graph", action="store_true", help="time eager launches instead of a CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--fwd-bwd-steps", type=int, default=3, help="timed fwd+bwd steps (0 disables)")
    ap.add_argument("--backward-only", type=int, default=0, metavar="N",
                    help="profiling mode: run the operator backward N times on config-3 inputs and exit")
    ap.add_argument("--rope-only", type=int, default=0, metavar="N",
                    help="profiling mode: time N iterations of the standalone rotation (p3d_rope) of q, kl, kg "
                         "views at config-1 shapes and exit")
    ap.add_argument("--config4", type=int, default=0, metavar="K",
                    help="separate mode: BASELINE config 4 (128^3 field, dim 384 = 8 heads x 48) layer forward + "
                         "backward, K timed steps, on the launch's N GPUs (z-slabs for N > 1); one JSON line")
    ap.add_argument("--allen15", type=int, default=0, metavar="K",
                    help="separate mode: the reference's published 'allen15' preset (32x128x64 raster, dim 512, "
                         "8 q-heads / 2 kv-heads x 64, radius 1, (1,4,4) raster blocks, pool 16), layer inference "
                         "and forward + backward, K timed steps each; one JSON line")
    ap.add_argument("--no-allen15", action="store_true", help="skip the allen15 preset in the N = 1 line")
    ap.add_argument("--no-config2", action="store_true", help="skip the Morton-storage (config 2) sub-object")
    ap.add_argument("--config4-steps", type=int, default=3,
                    help="timed steps of the config-4 sub-object (128^3 fwd + bwd at this N; 0 skips it)")
    ap.add_argument("--infer-only", type=int, default=0, metavar="N",
                    help="profiling mode: run the config-1 layer inference forward N times (eager) and exit")
    ap.add_argument("--train-only", type=int, default=0, metavar="N",
                    help="profiling mode: run the config-3 layer forward + backward N times and exit")
    ap.add_argument("--kernel-only", type=int, default=0, metavar="N",
                    help="profiling mode: run the stage-(c) kernel N times on the config-1 inputs and exit")
    return ap.parse_args()


def make_layout(grid):
    from pack3d_b200 import build_layout
    layout = build_layout(grid, CONFIG["block"], radius=CONFIG["radius"], pool_size=CONFIG["pool_size"])
    return layout.repack(layout.order.argsort())        # raster storage of 4x4x4 cubes


def make_layer(dtype, device):
    from pack3d_b200 import PACK3DAttention
    torch.manual_seed(0)
    layer = PACK3DAttention(CONFIG["dim"], heads=CONFIG["heads"], kv_heads=CONFIG["kv_heads"],
                            head_dim=CONFIG["head_dim"], block_volume=math.prod(CONFIG["block"]))
    return layer.to(device=device, dtype=dtype)


def mean_valid_neighbors(geometry):
    return (geometry.neighbors >= 0).sum().item() / geometry.num_tokens


# ------------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        clocks = [num(r[1]) for r in rows if num(r[1])]
        max_clk = max((num(r[2]) for r in rows if num(r[2])), default=None)
        loaded = [c for c, r in zip(clocks, rows) if num(r[3]) and num(r[3]) > 200] or clocks
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max_clk,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------- timing

def timed_steps(step, steps, stream, flush=None):
    """Per-step CUDA-event times (ms) on `stream`; the L2 flush runs between events."""
    times = []
    for _ in range(steps):
        if flush is not None:
            flush()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        step()
        end.record(stream)
        end.synchronize()
        times.append(start.elapsed_time(end))
    return times


def pipelined_e2e(call, x_host, out_shape, device, stream, steps, warmup):
    """End-to-end ms per step of ``call(x_device) -> y`` as a streaming pipeline: each step
    copies its input in from pinned host memory (one copy stream), runs the call (``stream``)
    and copies its result out to pinned host memory (another copy stream); device inputs and
    host outputs are double-buffered, so step i+1's copy-in and step i-1's copy-out overlap
    step i's compute.  Every step moves its own input in and result out inside the timed
    region; the per-step working set (~0.7 GB at config 1) exceeds L2."""
    x_dev = [torch.empty(x_host.shape, dtype=x_host.dtype, device=device) for _ in range(2)]
    y_host = [torch.empty(out_shape, dtype=x_host.dtype).pin_memory() for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def run(k):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        s_in.wait_event(start)
        s_out.wait_event(start)
        computed = []
        last_out = None
        for i in range(k):
            j = i % 2
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(computed[i - 2])   # step i-2 has read x_dev[j]
                x_dev[j].copy_(x_host, non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(s_in)
            stream.wait_event(loaded)
            with torch.inference_mode():
                y = call(x_dev[j])
            done = torch.cuda.Event()
            done.record(stream)
            computed.append(done)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                y_host[j].copy_(y, non_blocking=True)
                y.record_stream(s_out)               # y's memory is reused only after its copy-out
                last_out = torch.cuda.Event()
                last_out.record(s_out)
        stream.wait_event(last_out)
        end.record(stream)
        end.synchronize()
        return start.elapsed_time(end) / k

    run(max(warmup, 2))
    return run(steps)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one stencil_fwd_kernel launch at
# config 1, from the ncu capture summarised in profiles/stencil_fwd_config1.md (the command is
# there); refreshed together with that summary whenever the kernel changes.
STENCIL_FWD_DRAM_BYTES = 392.0e6   # 307.5 MB read + 84.5 MB written, one ncu launch
STENCIL_FWD_DRAM_SOURCE = "ncu capture of stencil_fwd_kernel at config 1 (profiles/stencil_fwd_config1.md)"


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        peaks = json.loads(path.read_text())
        return peaks.get("bf16_tflops"), peaks.get("bf16_tflops_sustained"), peaks.get("hbm_gbs"), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


# ------------------------------------------------------------------------- CPU baseline

def cpu_model():
    """The host CPU's model name (from /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_reference_step(seed=1000):
    """One config-1 layer forward on the host cores with the CPU restatement of the reference
    (``oracle``: the reference's layer, RoPE, pooling and core arithmetic in fp32, its grid
    tables and its seeded layer initialisation), over all 262,144 tokens.

    Returns ``(step, threads)``; ``step()`` runs the whole forward once.  Nothing here loads
    the B200 library: the tables, the weights and the arithmetic all come from the oracle.
    """
    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    tables = oracle.grid_layout(CONFIG["grid"], CONFIG["block"], CONFIG["radius"], "raster")
    torch.manual_seed(0)
    params = oracle.init_layer(CONFIG["dim"], heads=CONFIG["heads"], kv_heads=CONFIG["kv_heads"],
                               head_dim=CONFIG["head_dim"], block_volume=math.prod(CONFIG["block"]))
    n = math.prod(CONFIG["grid"])
    x = torch.randn(CONFIG["batch"], n, CONFIG["dim"], generator=torch.Generator().manual_seed(seed))
    rows = torch.arange(n)

    def step():
        with torch.no_grad():
            return oracle.layer_forward(x, params, tables["coords"], tables["neighbors"], tables["blocks"],
                                        CONFIG["pool_size"], heads=CONFIG["heads"], kv_heads=CONFIG["kv_heads"],
                                        head_dim=CONFIG["head_dim"], rows=rows, chunk=4096)
    return step, threads


CPU_SAMPLE = ("the whole config-1 layer forward (LayerNorm, projections, RoPE, pooling, local + global "
              "attention over all 262,144 query rows, output projection, residual), fp32, no extrapolation")


def config1_desc(parallelism):
    """The workload description both arms print as ``config``."""
    return {"workload": "BASELINE config 1: 64^3 raster field, batch 1, dim 192 = 4 heads x 48, radius-2 "
                        "5x5x5 neighbourhood, 4x4x4 mean-pool summaries (4096), layer forward",
            "grid": list(CONFIG["grid"]), "batch": CONFIG["batch"], "heads": CONFIG["heads"],
            "kv_heads": CONFIG["kv_heads"], "head_dim": CONFIG["head_dim"], "dim": CONFIG["dim"],
            "summaries": math.prod(CONFIG["grid"]) // math.prod(CONFIG["block"]), "radius": CONFIG["radius"],
            "parallelism": parallelism,
            "l2": "GPU arm: a 256 MiB write flushes L2 between timed steps (outside the timed events); "
                  "CPU arm: the per-step working set (several GB) exceeds every cache"}


# ------------------------------------------------------------------------------- GPU arm

def backward_only(args, device):
    """Profiling mode: the operator backward (stage d) alone on config-3 inputs (batch 2)."""
    from pack3d_b200 import _native
    from pack3d_b200 import ops as p3d_ops
    layout = make_layout(CONFIG["grid"]).to(device)
    geom = layout.geometry
    n, hq, g, hd = geom.num_tokens, CONFIG["heads"], CONFIG["kv_heads"], CONFIG["head_dim"]
    gen = torch.Generator(device=device).manual_seed(3)
    rnd = lambda *shape: torch.randn(*shape, device=device, generator=gen).to(torch.bfloat16)  # noqa: E731
    q, (kl, vl, kg, vg) = rnd(2, hq, n, hd), (rnd(2, g, n, hd) for _ in range(4))
    f32 = dict(device=device, dtype=torch.float32)
    params = (torch.zeros(hd, **f32), torch.zeros(64, **f32), torch.full((2, hq, n), 0.5, device=device,
              dtype=torch.bfloat16), torch.ones(hd, **f32), torch.full((hd,), 0.25, **f32))
    inputs = (q, kl, vl, kg, vg, *params)
    _, saved = p3d_ops.forward(*inputs, geom, 1.0, save_state=True)
    dy = rnd(2, hq, n, hd)
    step = lambda: p3d_ops.backward(dy, inputs, saved, geom, 1.0)  # noqa: E731
    for _ in range(max(args.warmup, 1)):
        step()
    times = timed_steps(step, args.backward_only, torch.cuda.current_stream(device))
    errors = _native.device_errors()
    print(json.dumps({"backward_only_ms": [round(t, 4) for t in times], "device_errors": errors}), flush=True)


ALLEN15 = dict(grid=(32, 128, 64), block=(1, 4, 4), radius=1, pool_size=16, dim=512, heads=8, kv_heads=2,
               head_dim=64)


def allen15(args, device):
    """``--allen15 K``: :func:`allen15_measure` as one JSON line."""
    print(json.dumps(allen15_measure(args.allen15, args.warmup, device)), flush=True)


def allen15_measure(steps, warmup, device):
    """The preset of the reference's only published timings (H200, Triton backend, batch 1:
    layer inference 4.644 ms, forward + backward 15.098 ms, bf16, raster storage), on this
    GPU: the same layer, layout, dtype and batch, eager calls, medians of CUDA-event times."""
    from pack3d_b200 import PACK3DAttention, _native, build_layout
    cfg = ALLEN15
    layout = build_layout(cfg["grid"], cfg["block"], radius=cfg["radius"], pool_size=cfg["pool_size"],
                          layout="raster_block").to(device)
    n = layout.geometry.num_tokens
    torch.manual_seed(0)
    layer = PACK3DAttention(cfg["dim"], heads=cfg["heads"], kv_heads=cfg["kv_heads"], head_dim=cfg["head_dim"],
                            block_volume=math.prod(cfg["block"])).to(device=device, dtype=torch.bfloat16)
    gen = torch.Generator(device=device).manual_seed(15)
    x = torch.randn(1, n, cfg["dim"], device=device, generator=gen).to(torch.bfloat16)
    dy = torch.randn_like(x)
    stream = torch.cuda.current_stream(device)

    def infer():
        with torch.inference_mode():
            layer(x, layout)

    xg = x.clone().requires_grad_()

    def train():
        layer.zero_grad(set_to_none=True)
        xg.grad = None
        layer(xg, layout).backward(dy)

    out = {}
    for name, fn in (("inference", infer), ("fwd_bwd", train)):
        for _ in range(max(warmup, 2)):
            fn()
        torch.cuda.synchronize(device)
        times = timed_steps(fn, steps, stream)
        out[name] = round(statistics.median(times), 4)
    errors = _native.device_errors()
    if errors:
        raise RuntimeError(f"device error flags set: {errors}")
    return {"mode": "allen15", "workload": "the reference's published 'allen15' preset: 32x128x64 raster, dim 512, "
                                           "8 q-heads / 2 kv-heads x 64, radius 1, (1,4,4) raster blocks, pool 16, "
                                           "bf16, batch 1",
            "inference_ms": out["inference"], "fwd_bwd_ms": out["fwd_bwd"],
            "reference_h200_ms": {"inference": 4.644, "fwd_bwd": 15.098},
            "tokens": n, "summaries": layout.geometry.num_summaries, "eager": True, "steps": steps}


def rope_only(args, device):
    """Profiling mode: ``rotate_projections`` (three ``p3d_rope`` calls) on strided views of the
    config-1 projection rows, as the per-op layer path calls it."""
    from pack3d_b200.rope import balanced_pairs, rotate_projections
    layout = make_layout(CONFIG["grid"]).to(device)
    n, h, d = layout.geometry.num_tokens, CONFIG["heads"], CONFIG["head_dim"]
    gen = torch.Generator(device=device).manual_seed(4)
    qp = torch.randn(1, n, h * d, device=device, generator=gen).to(torch.bfloat16)
    kvp = torch.randn(1, n, 4 * h * d, device=device, generator=gen).to(torch.bfloat16)
    q = qp.reshape(1, n, h, d).transpose(1, 2)
    kl, _, kg, _ = (t.reshape(1, n, h, d).transpose(1, 2) for t in kvp.chunk(4, -1))
    pairs = balanced_pairs(d)

    def step():
        with torch.no_grad():
            rotate_projections(q, kl, kg, layout.coords, pairs, layout.grid_shape, packed=False)
    for _ in range(max(args.warmup, 1)):
        step()
    times = timed_steps(step, args.rope_only, torch.cuda.current_stream(device))
    print(json.dumps({"rope_three_calls_ms": [round(t, 4) for t in times]}), flush=True)


def infer_only(args, device):
    """Profiling mode: the config-1 layer inference forward alone (eager calls)."""
    from pack3d_b200 import _native
    layout = make_layout(CONFIG["grid"]).to(device)
    layer = make_layer(torch.bfloat16, device)
    gen = torch.Generator(device=device).manual_seed(5)
    x = torch.randn(CONFIG["batch"], layout.geometry.num_tokens, CONFIG["dim"], device=device, generator=gen)
    x = x.to(torch.bfloat16)

    def step():
        with torch.inference_mode():
            layer(x, layout)

    for _ in range(max(args.warmup, 1)):
        step()
    times = timed_steps(step, args.infer_only, torch.cuda.current_stream(device))
    errors = _native.device_errors()
    print(json.dumps({"infer_step_ms": [round(t, 4) for t in times], "device_errors": errors}), flush=True)


def train_only(args, device):
    """Profiling mode: the config-3 layer forward + backward (batch 2) alone."""
    from pack3d_b200 import _native
    layout = make_layout(CONFIG["grid"]).to(device)
    layer = make_layer(torch.bfloat16, device)
    gen = torch.Generator(device=device).manual_seed(4)
    x = torch.randn(2, layout.geometry.num_tokens, CONFIG["dim"], device=device, generator=gen)
    x = x.to(torch.bfloat16).requires_grad_()
    dy = torch.randn_like(x)

    def step():
        layer.zero_grad(set_to_none=True)
        x.grad = None
        layer(x, layout).backward(dy)

    for _ in range(max(args.warmup, 1)):
        step()
    times = timed_steps(step, args.train_only, torch.cuda.current_stream(device))
    errors = _native.device_errors()
    print(json.dumps({"train_step_ms": [round(t, 4) for t in times], "device_errors": errors}), flush=True)


CONFIG4 = dict(grid=(128, 128, 128), batch=1, heads=8, kv_heads=8, head_dim=48, dim=384, block=(4, 4, 4), radius=2)


def config4_fwd_bwd(steps, rank, world, device):
    """the layer forward + backward on a 128^3 field (2,097,152 tokens),
    dim 384 = 8 heads x 48, bf16.  N = 1: the whole field on one GPU; N > 1: z-slabs, the
    sharded core (halo exchange, summary all-gather, summary-gradient reduce-scatter) and an
    all-reduce of the replicated parameters' gradients, as a data-parallel step would.
    The field is stored in raster order (the reference config's Morton storage is a pure
    repack of it, tested for equivariance elsewhere)."""
    from pack3d_b200 import PACK3DAttention, _native
    from pack3d_b200.sharded import ZSlabs, sharded_layer_forward, slab_layout
    grid = CONFIG4["grid"]
    if world == 1:
        layout = make_layout(grid).to(device)
        forward = lambda layer, x: layer(x, layout)  # noqa: E731
        n = math.prod(grid)
    else:
        slabs = ZSlabs(grid, world, rank, radius=CONFIG4["radius"], block_depth=CONFIG4["block"][0])
        layout = slab_layout(grid, CONFIG4["block"], radius=CONFIG4["radius"], slabs=slabs).to(device)
        forward = lambda layer, x: sharded_layer_forward(layer, x, layout)  # noqa: E731
        n = slabs.tokens
    torch.manual_seed(0)
    layer = PACK3DAttention(CONFIG4["dim"], heads=CONFIG4["heads"], kv_heads=CONFIG4["kv_heads"],
                            head_dim=CONFIG4["head_dim"], block_volume=math.prod(CONFIG4["block"]))
    layer = layer.to(device=device, dtype=torch.bfloat16)
    gen = torch.Generator(device=device).manual_seed(2000 + rank)
    x = torch.randn(CONFIG4["batch"], n, CONFIG4["dim"], device=device, generator=gen).to(torch.bfloat16)
    x.requires_grad_()
    dy = torch.randn_like(x)

    def step():
        layer.zero_grad(set_to_none=True)
        x.grad = None
        forward(layer, x).backward(dy)
        if world > 1:
            for p in layer.parameters():
                torch.distributed.all_reduce(p.grad)

    step()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    times = timed_steps(step, steps, torch.cuda.current_stream(device))
    ms = sum(times) / len(times)
    if world > 1:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    errors = _native.device_errors()
    if errors:
        raise RuntimeError(f"device error flags set: {errors}")
    total = math.prod(grid) * CONFIG4["batch"]
    return {"mode": "config4", "metric": "PACK3D layer bf16 fwd+bwd tokens/s, BASELINE config 4", "n_gpus": world,
            "steps": steps, "ms_per_step": round(ms, 3), "tokens_per_s": round(total / (ms * 1e-3), 1),
            "scaling": "strong",
            "config": {"workload": "BASELINE config 4: 128^3 field (2,097,152 tokens, raster storage), batch 1, "
                                   "dim 384 = 8 heads x 48, radius 2, 32,768 summaries; layer forward + backward "
                                   "(no optimizer)" + ("" if world == 1 else "; z-slabs over NCCL, parameter "
                                                                             "gradients all-reduced"),
                       "grid": list(grid), "dim": CONFIG4["dim"], "heads": CONFIG4["heads"],
                       "head_dim": CONFIG4["head_dim"]}}


def config2_measure(steps, device):
    """the config-1 field stored in Morton (Z-order) storage -- the
    reference's native block-Morton layout, tokens, coordinates and tables permuted together
    -- layer inference in bf16 and f16 (CUDA graph, L2 flushed between steps), next to the
    same call on raster storage.  Its outputs equal the permuted raster outputs bit for bit
    (tests/test_gpu_baseline_parity.py)."""
    from pack3d_b200 import build_layout
    layout = build_layout(CONFIG["grid"], CONFIG["block"], radius=CONFIG["radius"],
                          pool_size=CONFIG["pool_size"]).to(device)
    raster = make_layout(CONFIG["grid"]).to(device)
    stream = torch.cuda.current_stream(device)
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    out = {"workload": "BASELINE config 2: the 64^3 config-1 field in Morton storage (native block-Morton "
                       "layout), layer forward, batch 1", "steps": steps}
    for dtype, tag in ((torch.bfloat16, "bf16"), (torch.float16, "f16")):
        layer = make_layer(dtype, device)
        gen = torch.Generator(device=device).manual_seed(1000)
        x = torch.randn(CONFIG["batch"], layout.geometry.num_tokens, CONFIG["dim"], device=device,
                        generator=gen).to(dtype)
        for name, lay in (("morton", layout), ("raster", raster)):
            with torch.inference_mode():
                for _ in range(3):
                    layer(x, lay)
                side = torch.cuda.Stream(device)
                side.wait_stream(stream)
                with torch.cuda.stream(side):
                    layer(x, lay)
                stream.wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    layer(x, lay)
            for _ in range(3):
                graph.replay()
            times = timed_steps(graph.replay, steps, stream, flush_buf.zero_)
            ms = sum(times) / len(times)
            out[f"{tag}_{name}_ms"] = round(ms, 4)
            if name == "morton":
                out[f"{tag}_tokens_per_s"] = round(layout.geometry.num_tokens / (ms * 1e-3), 1)
            del graph
    return out


def sharded_phases(layer, x, layout, steps, stream, flush, max_over_ranks):
    """Per-phase CUDA-event times (ms, median over ``steps`` eager steps, then max over ranks)
    of one rank's sharded inference step, the same calls ``sharded_layer_forward`` makes:
    glue (LayerNorm, fused projection writing kl / vl into the peer region, gate), pooling,
    the peer exchange (credit wait, push, arrival wait: includes waiting for the slowest
    peer), the slab kernel (summary bound + attention), and release + output projection."""
    from pack3d_b200.sharded import pool_summaries, slab_forward, slab_peers
    b, g, d = x.shape[0], layer.kv_heads, layer.head_dim
    names = ("glue", "pooling", "exchange", "slab_attention", "output")
    samples = {k: [] for k in names}
    with torch.inference_mode():
        peers = slab_peers(layout.slabs, b, g, d, layout.geometry.num_summaries, x.dtype, x.device)
        for _ in range(steps):
            flush()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
            ev[0].record(stream)
            xr, q, kl, vl, kg, vg, gate = layer._inference_glue(x, layout.coords, layout.grid_shape,
                                                                kv_out=peers.kv_out())
            ev[1].record(stream)
            skr, svr = pool_summaries(kg, vg, layer.pool_weight, layer.slot_bias, layout.geometry, layer.temperature)
            ev[2].record(stream)
            kl_ext, vl_ext, sk, sv = peers.exchange(kl, vl, skr, svr)
            ev[3].record(stream)
            y, _ = slab_forward(q, kl_ext, vl_ext, sk, sv, layer.pool_weight, layer.slot_bias, gate,
                                layer.local_scale, layer.global_scale, layout.geometry, layout.slabs,
                                layer.temperature, y_rows=True)
            ev[4].record(stream)
            peers.release()
            layer._out_residual(xr, y)
            ev[5].record(stream)
            ev[5].synchronize()
            for i, k in enumerate(names):
                samples[k].append(ev[i].elapsed_time(ev[i + 1]))
    return {k: round(max_over_ranks(statistics.median(v)), 4) for k, v in samples.items()}


def run_sharded(args, rank, world, device):
    """N > 1: the config-1 field split into z-slabs, one per rank (the same 64^3 field at
    every N: strong scaling).  Each rank runs the layer on its planes with the halo
    exchange and the summary all-gather over NCCL (pack3d_b200.sharded)."""
    from pack3d_b200 import _native
    from pack3d_b200.rope import balanced_pairs, rotate_projections
    from pack3d_b200.sharded import (ZSlabs, exchange_halos, gather_summaries, pool_summaries,
                                     sharded_layer_forward, slab_forward, slab_layout)
    grid, b, dim = CONFIG["grid"], CONFIG["batch"], CONFIG["dim"]
    hq, g, hd = CONFIG["heads"], CONFIG["kv_heads"], CONFIG["head_dim"]
    slabs = ZSlabs(grid, world, rank, radius=CONFIG["radius"], block_depth=CONFIG["block"][0])
    layout = slab_layout(grid, CONFIG["block"], radius=CONFIG["radius"], slabs=slabs).to(device)
    geom = layout.geometry
    n_total, n = math.prod(grid), slabs.tokens
    layer = make_layer(torch.bfloat16, device)
    gen = torch.Generator(device=device).manual_seed(1000)
    lo, hi = slabs.token_range()
    x = torch.randn(b, n_total, dim, device=device, dtype=torch.bfloat16, generator=gen)[:, lo:hi].contiguous()
    stream = torch.cuda.current_stream(device)
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)

    def flush():
        flush_buf.zero_()

    def step():
        with torch.inference_mode():
            return sharded_layer_forward(layer, x, layout)

    def max_over_ranks(v):
        t = torch.tensor([v], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return t.item()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(device)
    run, graph = step, None
    if not args.no_graph:
        # the whole rank step (its peer exchange included) as one CUDA graph
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                step()
        stream.wait_stream(side)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        run = graph.replay
        for _ in range(2):
            run()
        torch.cuda.synchronize(device)
    torch.distributed.barrier()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index).__enter__()
    times = timed_steps(run, args.steps, stream, flush)
    torch.cuda.synchronize(device)
    used_graph = graph is not None
    del run, graph   # a graph holding NCCL calls is released before the process group
    torch.distributed.barrier()
    ms = max_over_ranks(sum(times) / len(times))

    # the slab forward kernel alone (halo and summaries already exchanged), for the roofline
    with torch.inference_mode():
        xn = layer.norm(x)
        q = layer.to_q(xn).reshape(b, n, hq, hd).transpose(1, 2)
        kl, vl, kg, vg = (t.reshape(b, n, g, hd).transpose(1, 2) for t in layer.to_kv(xn).chunk(4, -1))
        q, kl, kg = rotate_projections(q, kl, kg, layout.coords, balanced_pairs(hd), layout.grid_shape, packed=False)
        gate = layer.gate(xn).reshape(b, n, hq, 2).softmax(-1)[..., 1].transpose(1, 2).contiguous()
        vl, vg = vl.contiguous(), vg.contiguous()
        params = (layer.pool_weight, layer.slot_bias, gate, layer.local_scale, layer.global_scale)
        skr, svr = pool_summaries(kg, vg, layer.pool_weight, layer.slot_bias, geom)
        sk, sv = gather_summaries(skr), gather_summaries(svr)
        kl_ext, vl_ext = exchange_halos(kl, slabs), exchange_halos(vl, slabs)
        kernel = lambda: slab_forward(q, kl_ext, vl_ext, sk, sv, *params, geom, slabs)  # noqa: E731
        for _ in range(3):
            kernel()
        torch.cuda.synchronize(device)
        torch.distributed.barrier()
        kernel_ms = max_over_ranks(statistics.median(timed_steps(kernel, max(args.steps, 10), stream)))

    torch.cuda.synchronize(device)
    torch.distributed.barrier()
    phases = sharded_phases(layer, x, layout, max(args.steps, 10), stream, flush, max_over_ranks)

    x_host = x.detach().cpu().pin_memory()
    torch.cuda.synchronize(device)
    torch.distributed.barrier()
    e2e_ms = max_over_ranks(pipelined_e2e(lambda xd: sharded_layer_forward(layer, xd, layout), x_host, (b, n, dim),
                                          device, stream, args.steps, 3))
    clocks.__exit__(None, None, None)
    clock_summary = clocks.summary()
    errors = _native.device_errors()
    if max_over_ranks(float(errors)):
        raise RuntimeError(f"device error flags set: {errors}")

    full_geom = make_layout(grid).geometry
    w_bar, m = mean_valid_neighbors(full_geom), full_geom.num_summaries
    flops_total = 4.0 * b * hq * n_total * hd * (m + w_bar)
    peak, peak_sustained, _, peak_kind = measured_peaks()
    achieved = flops_total / world / (kernel_ms * 1e-3) / 1e12
    tokens = b * n_total
    return {
        "metric": METRIC,
        "value": round(tokens / (ms * 1e-3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: x ~ N(0,1) (seeded), random-init PACK3DAttention weights (seed 0)",
        "config": {"workload": "BASELINE config 1 field (64^3, batch 1, dim 192 = 4 heads x 48, radius 2, 4096 "
                               "summaries) split into z-slabs, one per GPU; layer forward",
                   "grid": list(grid), "batch": b, "heads": hq, "kv_heads": g, "head_dim": hd, "dim": dim,
                   "summaries": m, "radius": CONFIG["radius"],
                   "parallelism": f"{world} z-slabs of {slabs.planes} planes; peer-memory exchange per layer "
                                  "(p3d_peer_push over NVLink: 2 halo planes of kl, vl to each neighbour, the "
                                  "rank's summaries to every rank; bounded counter waits), no NCCL in the step",
                   "cuda_graph": used_graph,
                   "l2": "flushed between timed steps (256 MiB write outside the timed events)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "kernel": "stencil_fwd_kernel on one slab (p3d_attn_fwd_slab), max over ranks",
                     "kernel_ms": round(kernel_ms, 4), "flop_per_launch": flops_total / world,
                     "peak_kind": peak_kind, "peak_sustained": peak_sustained},
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": x_host.numel() * x_host.element_size() * world,
                "d2h_bytes_per_step": x_host.numel() * x_host.element_size() * world,   # y: x's shape and dtype
                "pipelined": "copy-in, compute and copy-out on three streams per rank; double-buffered, every "
                             "step copies its own input in and result out inside the timed region"},
        "phases_ms": dict(phases, note="eager step (no CUDA graph), each phase's median over ranks' "
                                        "steps, max over ranks; the graphed step above is the headline"),
        # per step: layer norm, fused projection, gate pairs, pooling, credit wait, push,
        # arrival wait, summary bound, slab forward, credit signal
        "gpu_launches": 10 * args.steps,
        "clocks": clock_summary,
    }


def run_b200(args, rank, world, device):
    from pack3d_b200 import _native
    from pack3d_b200 import ops as p3d_ops
    from pack3d_b200.rope import balanced_pairs, rotate_projections
    if args.backward_only:
        return backward_only(args, device)
    if args.train_only:
        return train_only(args, device)
    if args.rope_only:
        return rope_only(args, device)
    if args.infer_only:
        return infer_only(args, device)
    if args.allen15:
        return allen15(args, device)
    dtype = torch.bfloat16
    layout = make_layout(CONFIG["grid"]).to(device)
    geom = layout.geometry
    n = geom.num_tokens
    b = CONFIG["batch"]
    layer = make_layer(dtype, device)
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    x = torch.randn(b, n, CONFIG["dim"], device=device, dtype=dtype, generator=gen)
    stream = torch.cuda.current_stream(device)
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)

    def flush():
        flush_buf.zero_()

    def forward():
        with torch.inference_mode():
            return layer(x, layout)

    for _ in range(max(args.warmup, 3)):
        forward()
    torch.cuda.synchronize(device)
    use_graph = not args.no_graph and not args.kernel_only
    if use_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.inference_mode():
            side = torch.cuda.Stream(device)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                forward()
            stream.wait_stream(side)
            with torch.cuda.graph(graph):
                y_graph = layer(x, layout)
        step = graph.replay
    else:
        step = forward
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    # nvidia-smi samples every 100 ms from here through the kernel, operator and e2e timing loops
    clocks = ClockSampler(device.index).__enter__()
    times = timed_steps(step, 1 if args.kernel_only else args.steps, stream, flush)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    ms_local = sum(times) / len(times)
    ms = ms_local
    if world > 1:
        t = torch.tensor([ms_local], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()

    # ---- stage (c) kernel alone: fused local + global attention (for the roofline)
    with torch.inference_mode():
        xn = layer.norm(x)
        hq, hd, g = CONFIG["heads"], CONFIG["head_dim"], CONFIG["kv_heads"]
        q = layer.to_q(xn).reshape(b, n, hq, hd).transpose(1, 2)
        kl, vl, kg, vg = (t.reshape(b, n, g, hd).transpose(1, 2) for t in layer.to_kv(xn).chunk(4, -1))
        q, kl, kg = rotate_projections(q, kl, kg, layout.coords, balanced_pairs(hd), layout.grid_shape, packed=False)
        gate = layer.gate(xn).reshape(b, n, hq, 2).softmax(-1)[..., 1].transpose(1, 2).contiguous()
        vl, vg = vl.contiguous(), vg.contiguous()
        params = (layer.pool_weight, layer.slot_bias, gate, layer.local_scale, layer.global_scale)
        _, (sk, sv, *_rest) = p3d_ops.forward(q, kl, vl, kg, vg, *params, geom, 1.0, save_state=True)
        kernel = lambda: p3d_ops.forward(q, kl, vl, kg, vg, *params, geom, 1.0,  # noqa: E731
                                         save_state=False, summaries=(sk, sv))
        if args.kernel_only:
            times = timed_steps(kernel, args.kernel_only, stream)
            print(json.dumps({"kernel_only_ms": [round(t, 4) for t in times]}), flush=True)
            clocks.__exit__(None, None, None)
            clocks.summary()
            return None
        for _ in range(3):
            kernel()
        kernel_times = timed_steps(kernel, max(args.steps, 10), stream)
        op_fn = lambda: p3d_ops.forward(q, kl, vl, kg, vg, *params, geom, 1.0, save_state=False)  # noqa: E731
        op_times = timed_steps(op_fn, max(args.steps, 10), stream, flush)
    kernel_ms = statistics.median(kernel_times)
    w_bar = mean_valid_neighbors(geom)
    m = geom.num_summaries
    flops = 4.0 * b * hq * n * hd * (m + w_bar)
    peak, peak_sustained, hbm, peak_kind = measured_peaks()
    achieved = flops / (kernel_ms * 1e-3) / 1e12

    # ---- end to end through the public call: pinned host input in, output back out, streamed
    x_host = x.detach().cpu().pin_memory()
    e2e_ms = pipelined_e2e(lambda xd: layer(xd, layout), x_host, (b, n, CONFIG["dim"]), device, stream,
                           args.steps, 3)
    clocks.__exit__(None, None, None)
    clock_summary = clocks.summary()
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = t.item()

    # ---- fwd+bwd (BASELINE config 3 shape: batch 2), fewer steps
    fwd_bwd = None
    if args.fwd_bwd_steps > 0:
        xb = torch.randn(2, n, CONFIG["dim"], device=device, dtype=dtype, generator=gen).requires_grad_()
        dyb = torch.randn_like(xb)

        def train_step():
            layer.zero_grad(set_to_none=True)
            xb.grad = None
            layer(xb, layout).backward(dyb)

        train_step()
        torch.cuda.synchronize(device)
        fb_times = timed_steps(train_step, args.fwd_bwd_steps, stream, flush)
        fb_ms = sum(fb_times) / len(fb_times)
        if world > 1:
            t = torch.tensor([fb_ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            fb_ms = t.item()
        fwd_bwd = {"ms_per_step": round(fb_ms, 4), "tokens_per_s": round(world * 2 * n / (fb_ms * 1e-3), 1),
                   "batch": 2, "steps": args.fwd_bwd_steps, "includes": "layer forward + backward, no optimizer"}

    errors = _native.device_errors()
    if errors:
        raise RuntimeError(f"device error flags set: {errors}")
    tokens = world * b * n
    launches_per_step = 4      # library kernels per layer forward: LayerNorm, qkv split + RoPE, pooling, stencil
    line = {
        "metric": METRIC,
        "value": round(tokens / (ms * 1e-3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: x ~ N(0,1) (seeded), random-init PACK3DAttention weights (seed 0)",
        "config": config1_desc("none (one device)" if world == 1 else
                               f"{world} independent replicas (one field per GPU)"),
        "cuda_graph": use_graph,
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": STENCIL_FWD_DRAM_BYTES,
                     "traffic_source": STENCIL_FWD_DRAM_SOURCE,
                     "kernel": "stencil_fwd_kernel (stage c: fused local + global attention)",
                     "kernel_ms": round(kernel_ms, 4), "flop_per_launch": flops, "mean_valid_neighbors": w_bar,
                     "peak_kind": peak_kind, "peak_sustained": peak_sustained},
        "operator_ms": round(statistics.median(op_times), 4),
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                "d2h_bytes_per_step": x_host.numel() * x_host.element_size(),   # y has x's shape and dtype
                "pipelined": "copy-in, compute and copy-out on three streams; double-buffered, every step "
                             "copies its own input in and result out inside the timed region"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clock_summary,
        "fwd_bwd": fwd_bwd,
    }
    if use_graph:
        del graph, y_graph
    return line


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # The reference's CPU path (its CPU restatement in oracle/) on the host cores; rank 0
        # alone under torchrun.  No B200 code is imported on this arm.
        if rank != 0:
            return
        step, threads = cpu_reference_step()
        for _ in range(args.warmup):
            step()
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            step()
            times.append(time.perf_counter() - t0)
        s = sum(times) / len(times)
        n = math.prod(CONFIG["grid"]) * CONFIG["batch"]
        value = round(n / s, 1)
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(s * 1e3, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: x ~ N(0,1) (seeded), the reference layer's seeded initialisation (seed 0)",
            "config": config1_desc("none (one device)"),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "cpu": cpu_model(),
                             "kind": "port", "sample": CPU_SAMPLE + "; every step is the whole workload"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "step_s": [round(t, 3) for t in times],
        }), flush=True)
        return
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --impl b200 needs a CUDA device")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    if args.config4:
        line = config4_fwd_bwd(args.config4, rank, world, device)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    line = run_b200(args, rank, world, device) if world == 1 else run_sharded(args, rank, world, device)
    if line is None:
        return
    if world == 1 and not args.no_allen15 and not args.kernel_only:
        line["allen15"] = allen15_measure(5, 2, device)
    if world == 1 and not args.kernel_only and not args.no_config2:
        line["config2"] = config2_measure(10, device)
    if not args.kernel_only and args.config4_steps > 0:
        # the multi-GPU target (128^3, 8 heads, fwd + bwd) at this N: whole field at N = 1,
        # z-slabs for N > 1 -- the driver's 1..8 GPU runs give its scaling curve
        line["config4"] = config4_fwd_bwd(args.config4_steps, rank, world, device)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        step, threads = cpu_reference_step()
        t0 = time.perf_counter()
        step()
        cpu_s = time.perf_counter() - t0
        n = math.prod(CONFIG["grid"]) * CONFIG["batch"]
        line["cpu_baseline"] = {"value": round(n / cpu_s, 1), "unit": "tokens/s", "cores": threads,
                                "cpu": cpu_model(), "kind": "port", "sample": CPU_SAMPLE + ", timed once",
                                "measured_wall_s": round(cpu_s, 2)}
    if world > 1:
        from pack3d_b200.sharded import release_peers
        release_peers()   # the peer-exchange regions go before the process group
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
