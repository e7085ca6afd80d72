"""Benchmark: BF16 3x3-conv training step on the `xdna` device (B200).

Workload (the 3x3 conv sweep, at a large-channel
point): per GPU a batch of 128 NCHW BF16 images 256 x 72 x 72, one
Conv2d(256, 256, 3, padding=1, bias) trained with a synthetic upstream gradient
dY ~ N(0,1): forward, dgrad, wgrad (deferred, materialized by the optimizer),
bias grad and a fused Adam step; with N GPUs the gradients are averaged with
NCCL all-reduce over NVLink (data parallel, weak scaling).  Metric: training
images/s for the whole job, plus the conv's fwd+bwd TFLOP/s against the
measured dense-BF16 peak in "roofline".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the reference's CPU BF16 path for the same step
(stock PyTorch CPU kernels -- what the reference runs for these ops,
torch_xdna_device.cpp:4594-4603, 4862-4873, 5196-5198) on the host cores,
each step a bounded sample of the batch.  Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "pytorch-xdna2_b200"))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

METRIC = "train images/s at 1/2/4/8 B200; 3x3 conv fwd+bwd TFLOP/s vs BF16 peak"
B_PER_GPU, C, HW = 128, 256, 72
CPU_SAMPLE = 4  # images per CPU step (bounded sample of the same workload)


def conv_flops(b: int) -> float:
    return 2.0 * b * HW * HW * C * C * 9  # one direction (fwd, dgrad or wgrad)


def conv_traffic_bytes():
    """DRAM bytes of one fwd+dgrad+wgrad launch set at the bench shape, from the
    committed ncu summary (captured at batch 64, scaled by the batch)."""
    import re
    f = REPO / "profiles" / "conv3x3_igemm_B64_C256_HW72.md"
    if not f.is_file():
        return None
    m = re.search(r"traffic_fwd_dgrad_wgrad_bytes_B128:\s*(\d+)", f.read_text())
    return int(m.group(1)) if m else None


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


# --------------------------------------------------------------------- clocks

class Clocks:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        self.first = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            # nvidia-smi takes a moment to start: wait for its first sample (taken
            # before the timed region, so it is not counted) before timing starts
            import threading
            box = []
            t = threading.Thread(target=lambda: box.append(self.proc.stdout.readline()), daemon=True)
            t.start()
            t.join(timeout=5.0)
            self.first = box[0] if box else None
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
                self.lines = [ln for ln in out.splitlines() if ln.strip()]
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# -------------------------------------------------------------- the GPU step

def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def allreduce_max(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args):
    world, rank, local = setup_dist(args)
    import torch.nn as nn

    import xdna_train
    xdna_train.register_xdna_device()
    X = torch.device("xdna", local)
    torch.manual_seed(0)
    conv = nn.Conv2d(C, C, 3, padding=1).bfloat16().to(X)
    opt = torch.optim.Adam(conv.parameters(), lr=1e-3)
    g = torch.Generator().manual_seed(1 + rank)
    x_host = torch.randn(B_PER_GPU, C, HW, HW, generator=g).bfloat16().pin_memory()
    dy_host = torch.randn(B_PER_GPU, C, HW, HW, generator=g).bfloat16().pin_memory()
    x = x_host.to(X)
    dy = dy_host.to(X)

    if world > 1:
        import torch.distributed as dist

    def allreduce_grads():
        if world == 1:
            return
        for p in conv.parameters():
            t = xdna_train.as_cuda(p.grad)  # materializes the deferred dW first
            dist.all_reduce(t)
            t.div_(world)

    def step(xin, dyin):
        opt.zero_grad(set_to_none=True)
        xr = xin.requires_grad_(True) if not xin.requires_grad else xin
        y = conv(xr)
        y.backward(dyin)
        allreduce_grads()
        opt.step()
        return y

    for _ in range(args.warmup):
        step(x.detach(), dy)
    torch.cuda.synchronize()
    xdna_train.reset_mapped_cpu_stats()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(s)
        for _ in range(args.steps):
            step(x.detach(), dy)
        e1.record(s)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    ms = allreduce_max(ms, world)
    launches = sum(xdna_train.kernel_stats().values())
    fallbacks = xdna_train.fallback_stats()

    # ---- e2e through the public API with host buffers: H2D of x and dy, the
    # step, D2H of the updated weights (the step's result)
    w_host = torch.empty(conv.weight.shape, dtype=conv.weight.dtype).pin_memory()
    for _ in range(2):
        step(x_host.to(X, non_blocking=True), dy_host.to(X, non_blocking=True))
        w_host.copy_(conv.weight.detach(), non_blocking=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(s)
    for _ in range(args.steps):
        step(x_host.to(X, non_blocking=True), dy_host.to(X, non_blocking=True))
        w_host.copy_(conv.weight.detach(), non_blocking=True)
    e3.record(s)
    torch.cuda.synchronize()
    e2e_ms = allreduce_max(e2.elapsed_time(e3) / args.steps, world)
    del t0

    # ---- per-kernel device time of the conv directions (CUDA events on the
    # launching stream, same operands), for the roofline
    kt = kernel_times(x, dy, conv, local)

    if rank != 0:
        return None
    bf16_peak, _, peak_kind = peaks()
    flops_dir = conv_flops(B_PER_GPU)
    achieved = 3 * flops_dir / ((kt["fwd"] + kt["dgrad"] + kt["wgrad"]) * 1e-3) / 1e12
    images = B_PER_GPU * world
    line = {
        "metric": METRIC,
        "value": round(images / (ms * 1e-3), 2),
        "unit": "images/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (x, dY ~ N(0,1); random-init Conv2d weights)",
        "config": {"workload": f"conv3x3 train step: Conv2d({C},{C},3,pad=1,bias) on B{B_PER_GPU}x{C}x{HW}x{HW} "
                               "per GPU (BASELINE configs[1] sweep point), fwd+dgrad+wgrad+Adam",
                   "global_batch": images, "per_gpu_batch": B_PER_GPU, "channels": C, "hw": HW,
                   "parallelism": f"dp{world}", "l2": "inputs larger than L2 (340 MB activations per tensor)"},
        "e2e": {"value": round(images / (e2e_ms * 1e-3), 2), "unit": "images/s",
                "h2d_bytes_per_step": int(x_host.numel() * 2 + dy_host.numel() * 2),
                "d2h_bytes_per_step": int(w_host.numel() * 2)},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": bf16_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / bf16_peak, 4), "traffic": conv_traffic_bytes(),
                     "traffic_source": "ncu dram__bytes_read+write of the three kernels at B64, x2 (profiles/)",
                     "kernel": "conv3x3 implicit GEMM fwd+dgrad+wgrad (tcgen05 cta_group::2 SM-pair kernel)",
                     "per_launch_ms": {k: round(v, 4) for k, v in kt.items()},
                     "flops_per_launch": flops_dir, "peak_kind": peak_kind},
        "gpu_launches": launches,
        "clocks": clk.summary(),
        "fallback_ops": {k: v["calls"] for k, v in fallbacks.items()},
    }
    return line


def kernel_times(x, dy, conv, local, iters=10):
    """Average device time per launch of the fwd / dgrad / wgrad kernels, each
    timed alone with CUDA events on the stream they run on."""
    import ctypes

    from xdna_train import _abi
    L = _abi.lib()
    X = x.device
    st = torch.cuda.current_stream().cuda_stream
    B, C, HW = x.shape[0], x.shape[1], x.shape[2]
    ch = (C + 63) // 64
    rows = torch.empty(B * (HW + 2) * (HW + 2), ch * 64, dtype=torch.bfloat16, device=X)
    drows = torch.empty_like(rows)
    w = conv.weight.detach()
    wk = torch.empty(C, ch * 576, dtype=torch.bfloat16, device=X)
    wkd = torch.empty_like(wk)
    y = torch.empty_like(x)
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    wsb = L.b2_conv3x3_wgrad_workspace_bytes(B, C, HW, HW, C)
    ws = torch.empty(wsb, dtype=torch.uint8, device=X)
    _abi.call("b2_pack_rows_bf16", x.data_ptr(), *x.stride(), B, C, HW, HW, ch, rows.data_ptr(), st)
    _abi.call("b2_pack_rows_bf16", dy.data_ptr(), *dy.stride(), B, C, HW, HW, ch, drows.data_ptr(), st)
    _abi.call("b2_pack_weight_fwd_bf16", w.data_ptr(), C, C, ch, wk.data_ptr(), st)
    _abi.call("b2_pack_weight_dgrad_bf16", w.data_ptr(), C, C, ch, wkd.data_ptr(), st)
    fns = {
        "fwd": lambda: L.b2_conv3x3_fwd(rows.data_ptr(), wk.data_ptr(), conv.bias.data_ptr(), y.data_ptr(),
                                        *y.stride(), B, C, HW, HW, C, 0, st),
        "dgrad": lambda: L.b2_conv3x3_dgrad(drows.data_ptr(), wkd.data_ptr(), dx.data_ptr(), *dx.stride(), B, C,
                                            HW, HW, C, st),
        "wgrad": lambda: L.b2_conv3x3_wgrad(drows.data_ptr(), rows.data_ptr(), dw.data_ptr(), 0, B, C, HW, HW, C,
                                            ws.data_ptr(), wsb, st),
        "pack_rows": lambda: L.b2_pack_rows_bf16(x.data_ptr(), *x.stride(), B, C, HW, HW, ch, rows.data_ptr(), st),
    }
    out = {}
    for name, fn in fns.items():
        for _ in range(2):
            _abi.check(fn(), name)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        out[name] = a.elapsed_time(b) / iters
    code = ctypes.c_int(0)
    _abi.check(L.b2_device_status(local, ctypes.byref(code)))
    assert code.value == 0, f"device status {code.value}"
    return out


# -------------------------------------------------------- CPU reference path

def cpu_reference_step_rate(steps: int, warmup: int, sample: int = CPU_SAMPLE):
    """images/s of the reference's CPU BF16 path on a bounded sample."""
    from oracle import cpu_path
    torch.manual_seed(0)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(sample, C, HW, HW, generator=g).bfloat16()
    dy = torch.randn(sample, C, HW, HW, generator=g).bfloat16()
    w = (torch.randn(C, C, 3, 3, generator=g) * 0.02).bfloat16()
    b = torch.zeros(C).bfloat16()
    m = [torch.zeros_like(w), torch.zeros_like(b)]
    v = [torch.zeros_like(w), torch.zeros_like(b)]
    steps_t = [torch.zeros(()), torch.zeros(())]

    def one():
        cpu_path.conv3x3_fwd(x, w, b)
        _, dw, db = cpu_path.conv3x3_bwd(dy, x, w, (True, True, True))
        for t in steps_t:
            t += 1
        torch._fused_adam_([w, b], [dw, db], m, v, [], steps_t, lr=1e-3, beta1=0.9, beta2=0.999,
                           weight_decay=0.0, eps=1e-8, amsgrad=False, maximize=False)

    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dt = (time.perf_counter() - t0) / steps
    return sample / dt, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    steps, warmup = max(1, args.steps), max(1, min(args.warmup, 2))
    rate, dt = cpu_reference_step_rate(steps, warmup)
    cores = torch.get_num_threads()
    return {
        "metric": METRIC, "value": round(rate, 3), "unit": "images/s", "impl": "reference",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": steps, "warmup": warmup,
        "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (x, dY ~ N(0,1))",
        "config": {"workload": f"conv3x3 train step Conv2d({C},{C},3,pad=1,bias), {C}x{HW}x{HW} images, "
                               "fwd+dgrad+wgrad+Adam on the reference's CPU BF16 path",
                   "per_step_sample_images": CPU_SAMPLE, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(rate, 3), "unit": "images/s", "cores": cores, "kind": "reference",
                         "sample": f"{CPU_SAMPLE} images of {C}x{HW}x{HW} per step (of the {B_PER_GPU}-image "
                                   "GPU batch), stock PyTorch CPU conv/convolution_backward/_fused_adam_ = the "
                                   f"reference's CPU path; torch {torch.__version__} (reference pins 2.14)"},
        "e2e": {"value": round(rate, 3), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def kernel_probe(args):
    """Per-kernel device times of one conv shape (``--kernel-probe``): used for
    sweeps and as the small case of ncu captures."""
    import torch.nn as nn

    import xdna_train
    xdna_train.register_xdna_device()
    torch.cuda.set_device(0)
    X = torch.device("xdna", 0)
    b, c, hw = args.batch, args.channels, args.hw
    conv = nn.Conv2d(c, c, 3, padding=1).bfloat16().to(X)
    x = torch.randn(b, c, hw, hw, dtype=torch.bfloat16, device=X)
    dy = torch.randn(b, c, hw, hw, dtype=torch.bfloat16, device=X)
    kt = kernel_times(x, dy, conv, 0, iters=args.iters)
    fl = 2.0 * b * hw * hw * c * c * 9
    out = {k: {"ms": round(v, 4)} for k, v in kt.items()}
    for k in ("fwd", "dgrad", "wgrad"):
        out[k]["tflops"] = round(fl / (kt[k] * 1e-3) / 1e12, 1)
    out["pack_rows"]["gbs"] = round(2 * (x.numel() + b * (hw + 2) ** 2 * ((c + 63) // 64) * 64) / (kt["pack_rows"] * 1e-3) / 1e9, 1)
    print(json.dumps({"probe": f"B{b} C{c} HW{hw}", **out}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel-probe", action="store_true")
    ap.add_argument("--batch", type=int, default=B_PER_GPU)
    ap.add_argument("--channels", type=int, default=C)
    ap.add_argument("--hw", type=int, default=HW)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.kernel_probe:
        kernel_probe(args)
        return
    args.warmup = max(3, args.warmup) if args.impl == "ours" else args.warmup
    if args.impl == "reference":
        line = run_reference(args)
    else:
        line = run_ours(args)
        if line is not None and not args.no_cpu_baseline and line["n_gpus"] == 1:
            rate, dt = cpu_reference_step_rate(steps=3, warmup=1)
            line["cpu_baseline"] = {
                "value": round(rate, 3), "unit": "images/s", "cores": torch.get_num_threads(), "kind": "reference",
                "sample": f"{CPU_SAMPLE} images per step, 3 timed steps after 1 warmup; stock PyTorch CPU BF16 "
                          "conv/convolution_backward/_fused_adam_ (the reference's CPU path)"}
    if line is not None:
        print(json.dumps(line), flush=True)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 and args.impl == "ours":
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
