"""Benchmark of the `xdna` device on B200: BF16 training, one process per GPU.

Headline (the default; BASELINE.json's metric "train images/s at 1/2/4/8
B200; 3x3 conv fwd+bwd TFLOP/s vs BF16 peak" on its configs[4], ResNet-50):
per GPU a batch of 128 synthetic 224x224 images ~ N(0,1) (channels-last
BF16) with uniform random labels over 1000 classes, a random-init
torchvision ResNet-50 on ``torch.device("xdna")``, cross-entropy, backward
(deferred conv weight gradients materialized by the optimizer or the
all-reduce), SGD momentum 0.9 (``--optimizer adam``: the config's Adam
variant); with N GPUs the gradients are averaged by bucketed NCCL
all-reduces overlapped with backward (``xdna_train.ddp``; data parallel, weak
scaling).  The step (at N > 1 with its NCCL all-reduces) is captured into a
CUDA graph (``xdna_train.graphs.make_graphed_step``) and replayed, so the host's per-op
dispatch (about as long as the step's kernels) is out of the timed region;
``--eager`` times the step op by op, and the line carries the eager rate
beside the replayed one.  ``value`` = images/s of the whole job; ``roofline`` = the 3x3
convolution kernels' FLOPs over their device time inside the step (CUDA
event pairs around each launch, on its stream); ``e2e`` = the same step fed
from pinned host memory (images and labels copied every step, the loss read
back every step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --workload conv|readme|mlp|style     (the other configs)

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
B_PER_GPU, C, HW = 128, 256, 72  # --workload conv: the 3x3 conv layer step
CPU_SAMPLE = 4  # images per CPU step (bounded sample of the same workload)
RESNET_BATCH, RESNET_HW = 128, 224  # the headline: ResNet-50 per-GPU batch
RESNET_CPU_SAMPLE = 16  # images per CPU step of the ResNet-50 reference path


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


def peaks(sustained: bool = False):
    """(bf16 TFLOP/s, HBM GB/s, kind): the pool's measured peaks (the burst
    GEMM figure, or with ``sustained`` the figure of a seconds-long GEMM loop
    under the power cap, for kernels timed inside a long step), else the
    recipe's fallback."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        tf = d.get("bf16_tflops_sustained") if sustained else None
        return float(tf or d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return (1400.0 if sustained else 1590.0), 6650.0, "fallback"


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
        # once xdna is registered PyTorch treats it as the accelerator and
        # refuses a cuda device_id; NCCL then binds the device lazily
        acc = torch.accelerator.current_accelerator() if hasattr(torch, "accelerator") else None
        kw = {"device_id": torch.device("cuda", local)} if acc is None or acc.type == "cuda" else {}
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), **kw)
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def cuda_barrier():
    """A barrier as an all-reduce of a CUDA tensor: dist.barrier() picks its
    device from the current accelerator, which is xdna once registered, and
    NCCL has no xdna backend."""
    import torch.distributed as dist
    t = torch.zeros(1, device=torch.device("cuda", torch.cuda.current_device()))
    dist.all_reduce(t)
    torch.cuda.synchronize()


def allreduce_max(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_conv_layer(args):
    world, rank, local = setup_dist(args)
    import torch.nn as nn

    import xdna_train
    xdna_train.register_xdna_device()
    X = torch.device("xdna", local)
    torch.manual_seed(0)
    conv = nn.Conv2d(C, C, 3, padding=1).bfloat16().to(X)
    opt = torch.optim.Adam(conv.parameters(), lr=1e-3)
    g = torch.Generator().manual_seed(1 + rank)
    mf = torch.channels_last if args.channels_last else torch.contiguous_format
    if args.channels_last:
        conv = conv.to(memory_format=mf)
    x_host = torch.randn(B_PER_GPU, C, HW, HW, generator=g).bfloat16().contiguous(memory_format=mf).pin_memory()
    dy_host = torch.randn(B_PER_GPU, C, HW, HW, generator=g).bfloat16().contiguous(memory_format=mf).pin_memory()
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
        cuda_barrier()
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
        cuda_barrier()
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
        cuda_barrier()
    # The step's inputs arrive through two device buffers: the host->device
    # copy of step k+1 runs on a copy stream while step k computes (what a
    # prefetching data loader does); every step still copies its own inputs.
    copy_s = torch.cuda.Stream()
    bx = [torch.empty_like(x) for _ in range(2)]
    bd = [torch.empty_like(dy) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]

    def prefetch(i):
        with torch.cuda.stream(copy_s):
            copy_s.wait_event(used[i])  # the step that last read buffer i is done
            bx[i].copy_(x_host, non_blocking=True)
            bd[i].copy_(dy_host, non_blocking=True)
            copied[i].record(copy_s)

    for i in range(2):
        used[i].record(s)
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(s)
    copy_s.wait_stream(s)
    prefetch(0)
    for k in range(args.steps):
        i = k % 2
        s.wait_event(copied[i])
        if k + 1 < args.steps:
            prefetch(1 - i)
        step(bx[i].detach(), bd[i])
        used[i].record(s)
        w_host.copy_(conv.weight.detach(), non_blocking=True)
    e3.record(s)
    torch.cuda.synchronize()
    e2e_ms = allreduce_max(e2.elapsed_time(e3) / args.steps, world)

    # ---- the step's own launches timed in place (event pairs on their stream)
    xdna_train.kernel_timer(True)
    for _ in range(3):
        step(x.detach(), dy)
    torch.cuda.synchronize()
    xdna_train.kernel_timer(False)
    in_step = {k: round(v["ms"] / 3, 4) for k, v in xdna_train.kernel_times().items()}

    # ---- per-kernel device time of the conv directions (CUDA events on the
    # launching stream, same operands), for the roofline
    kt = kernel_times(x.contiguous(), dy.contiguous(), conv, local, nhwc=args.channels_last)
    sfx = "_nhwc" if args.channels_last else ""

    if rank != 0:
        return None
    bf16_peak, _, peak_kind = peaks()
    flops_dir = conv_flops(B_PER_GPU)
    achieved = 3 * flops_dir / ((kt["fwd" + sfx] + kt["dgrad" + sfx] + kt["wgrad" + sfx]) * 1e-3) / 1e12
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
                               "per GPU (BASELINE configs[1] sweep point), fwd+dgrad+wgrad+Adam"
                               + (", channels-last activations" if args.channels_last else ", NCHW activations"),
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
        "kernel_ms_per_step": in_step,
        "clocks": clk.summary(),
        "fallback_ops": {k: v["calls"] for k, v in fallbacks.items()},
    }
    return line


def kernel_times(x, dy, conv, local, iters=10, nhwc=False):
    """Average device time per launch of the fwd / dgrad / wgrad kernels, each
    timed alone with CUDA events on the stream they run on (``nhwc``: also
    the channels-last in-place entry points)."""
    import ctypes

    from xdna_train import _abi
    L = _abi.lib()
    X = x.device
    st = torch.cuda.current_stream().cuda_stream
    B, C, HW = x.shape[0], x.shape[1], x.shape[2]
    ch = (C + 63) // 64
    rows = torch.empty(B * (HW + 2) * (HW + 2), ch * 64, dtype=torch.bfloat16, device=X)
    drows = torch.empty_like(rows)
    w = conv.weight.detach().contiguous()
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
    if nhwc:
        # the same three directions reading channels-last x / dY in place
        xc = x.contiguous(memory_format=torch.channels_last)
        dyc = dy.contiguous(memory_format=torch.channels_last)
        yc = torch.empty_like(xc)
        dxc = torch.empty_like(xc)
        fns.update({
            "fwd_nhwc": lambda: L.b2_conv3x3_fwd_nhwc(xc.data_ptr(), xc.stride(0), xc.stride(2), xc.stride(3),
                                                      wk.data_ptr(), conv.bias.data_ptr(), yc.data_ptr(),
                                                      *yc.stride(), B, C, HW, HW, C, 0, st),
            "dgrad_nhwc": lambda: L.b2_conv3x3_dgrad_nhwc(dyc.data_ptr(), dyc.stride(0), dyc.stride(2),
                                                          dyc.stride(3), wkd.data_ptr(), dxc.data_ptr(),
                                                          *dxc.stride(), B, C, HW, HW, C, st),
            "wgrad_nhwc": lambda: L.b2_conv3x3_wgrad_nhwc(dyc.data_ptr(), dyc.stride(0), dyc.stride(2),
                                                          dyc.stride(3), xc.data_ptr(), xc.stride(0), xc.stride(2),
                                                          xc.stride(3), dw.data_ptr(), 0, B, C, HW, HW, C,
                                                          ws.data_ptr(), wsb, st),
        })
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


def run_conv_reference(args):
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


# ------------------------------------------------------- headline: ResNet-50

# in-step timer labels whose work is algorithmic bytes (HBM-bound passes)
MEM_LABELS = ("bn.", "relu_bwd_sum")


def resnet50_model(dev):
    """torchvision ResNet-50 (random init, seed 0) in bf16, channels-last."""
    from torchvision.models import resnet50
    torch.manual_seed(0)
    return resnet50(num_classes=1000).bfloat16().to(dev).to(memory_format=torch.channels_last)


def resnet50_train_flops(batch: int, hw: int = RESNET_HW):
    """Algorithmic FLOPs of one ResNet-50 training step (2 per multiply-add),
    counted from the layer shapes: every convolution and the classifier
    forward, input gradient (all but the stem, whose input needs none) and
    weight gradient.  Returns (total, of which the 3x3 stride-1 convolutions)."""
    import torch.nn as nn
    from torchvision.models import resnet50
    m = resnet50(num_classes=1000).to("meta")
    tot, c33 = [0.0], [0.0]
    stem = m.conv1

    def conv_hook(mod, inp, out):
        macs = out.numel() * mod.in_channels * mod.kernel_size[0] * mod.kernel_size[1] / mod.groups
        f = 2.0 * macs * (2 if mod is stem else 3)
        tot[0] += f
        if mod.kernel_size == (3, 3) and mod.stride == (1, 1):
            c33[0] += f

    def fc_hook(mod, inp, out):
        tot[0] += 3 * 2.0 * out.numel() * mod.in_features

    hs = [mm.register_forward_hook(conv_hook) for mm in m.modules() if isinstance(mm, nn.Conv2d)]
    hs.append(m.fc.register_forward_hook(fc_hook))
    with torch.no_grad():
        m(torch.empty(batch, 3, hw, hw, device="meta"))
    for h in hs:
        h.remove()
    return tot[0], c33[0]


def _sgd_or_adam(model, optimizer, on_device):
    # the CPU side keeps the foreach implementations: torch 2.11's CPU
    # _fused_sgd_ leaves bf16 parameters unchanged
    fused = True if on_device else None
    if optimizer == "adam":
        return torch.optim.Adam(model.parameters(), lr=1e-3, fused=fused)
    return torch.optim.SGD(model.parameters(), lr=0.1, momentum=0.9, fused=fused)


def run_resnet50(args):
    """The headline line (see the module docstring)."""
    import torch.nn.functional as F
    world, rank, local = setup_dist(args)
    import xdna_train
    from xdna_train.ddp import GradAllReduce
    xdna_train.register_xdna_device()
    X = torch.device("xdna", local)
    cl = torch.channels_last
    B = args.batch if args.batch != B_PER_GPU else RESNET_BATCH
    model = resnet50_model(X)
    opt = _sgd_or_adam(model, args.optimizer, True)
    ar = GradAllReduce(model) if world > 1 else None
    g = torch.Generator().manual_seed(1000 + rank)
    x_host = torch.empty((B, 3, RESNET_HW, RESNET_HW), dtype=torch.bfloat16, pin_memory=True)
    x_host.copy_(torch.randn(B, 3, RESNET_HW, RESNET_HW, generator=g))
    y_host = torch.randint(0, 1000, (B,), generator=g).pin_memory()
    x = x_host.to(X).contiguous(memory_format=cl)
    y = y_host.to(X)

    def step(xin, yin):
        opt.zero_grad(set_to_none=True)
        loss = F.cross_entropy(model(xin).float(), yin)
        loss.backward()
        if ar is not None:
            ar.synchronize()
        opt.step()
        return loss

    # two input buffers (the e2e loop fills one while the other is in use);
    # with CUDA graphs (the default: xdna_train.graphs, the step's kernels --
    # and at N > 1 its bucketed NCCL all-reduces -- replayed without the
    # host's per-op dispatch) one capture each
    bx = [x.clone(memory_format=cl) for _ in range(2)]
    by = [y.clone() for _ in range(2)]
    graphed = not args.eager
    s = torch.cuda.current_stream()
    if graphed:
        from xdna_train import graphs
        replays = [graphs.make_graphed_step(lambda i=i: step(bx[i], by[i]), warmup=args.warmup) for i in range(2)]
        run = lambda i: replays[i]()  # noqa: E731
    else:
        for _ in range(args.warmup):
            step(x, y)
        run = lambda i: step(bx[i], by[i])  # noqa: E731
    torch.cuda.synchronize()
    xdna_train.reset_mapped_cpu_stats()
    if world > 1:
        cuda_barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(s)
        for _ in range(args.steps):
            loss = run(0)
        e1.record(s)
        torch.cuda.synchronize()
    if world > 1:
        cuda_barrier()
    ms = allreduce_max(e0.elapsed_time(e1) / args.steps, world)
    launches = sum(xdna_train.kernel_stats().values())
    fallbacks = xdna_train.fallback_stats()
    final_loss = float(loss.item())

    # ---- e2e: every step copies its images and labels from pinned host
    # memory (on a copy stream, one step ahead, through the two device buffers
    # -- what a prefetching loader does) and reads its loss back to the host
    copy_s = torch.cuda.Stream()
    copied = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]
    loss_host = torch.empty(max(1, args.steps), dtype=torch.float32, pin_memory=True)

    def prefetch(i):
        with torch.cuda.stream(copy_s):
            copy_s.wait_event(used[i])
            bx[i].copy_(x_host, non_blocking=True)
            by[i].copy_(y_host, non_blocking=True)
            copied[i].record(copy_s)

    for i in range(2):
        used[i].record(s)
    torch.cuda.synchronize()
    if world > 1:
        cuda_barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(s)
    copy_s.wait_stream(s)
    prefetch(0)
    for k in range(args.steps):
        i = k % 2
        s.wait_event(copied[i])
        if k + 1 < args.steps:
            prefetch(1 - i)
        loss = run(i)
        used[i].record(s)
        loss_host[k:k + 1].copy_(loss.detach().reshape(1), non_blocking=True)
    e3.record(s)
    torch.cuda.synchronize()
    if world > 1:
        cuda_barrier()
    e2e_ms = allreduce_max(e2.elapsed_time(e3) / args.steps, world)
    assert torch.isfinite(loss_host[:args.steps]).all(), "non-finite loss"

    # ---- the 3x3 convolution kernels (and the other timed launch sites)
    # inside the same step: CUDA event pairs around each launch on its stream,
    # over a few more steps of the same workload
    xdna_train.reset_mapped_cpu_stats()
    xdna_train.kernel_timer(True)
    for _ in range(3):
        step(x, y)
    torch.cuda.synchronize()
    xdna_train.kernel_timer(False)
    kt = xdna_train.kernel_times()
    if graphed:  # a replay launches what the captured step launched
        launches = sum(xdna_train.kernel_stats().values()) * args.steps // 3
        fallbacks = {k: {**v, "calls": v["calls"] * args.steps // 3} for k, v in xdna_train.fallback_stats().items()}

    # ---- the same step eagerly (host dispatch per op), for comparison
    eager_ms = None
    if graphed:
        torch.cuda.synchronize()
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ne = min(args.steps, 30)
        ea.record(s)
        for _ in range(ne):
            step(x, y)
        eb.record(s)
        torch.cuda.synchronize()
        eager_ms = ea.elapsed_time(eb) / ne
        # graphs holding NCCL calls are released before the process group
        for r in replays:
            r.graph.reset()
        del replays, run

    # ---- the gradient all-reduce alone, per step (N > 1): every bucket's
    # collective, events on the launching stream
    ar_ms = None
    if ar is not None:
        import torch.distributed as dist
        cuda_barrier()
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ea.record(s)
        for _ in range(5):
            for bkt in ar.buckets:
                dist.all_reduce(xdna_train.as_cuda(bkt["flat"]), op=dist.ReduceOp.AVG)
        eb.record(s)
        torch.cuda.synchronize()
        ar_ms = allreduce_max(ea.elapsed_time(eb) / 5, world)

    if rank != 0:
        return None
    total_fl, c33_fl = resnet50_train_flops(B)
    peak_s, hbm, peak_kind = peaks(sustained=True)
    conv = {k: v for k, v in kt.items() if k.startswith("conv3x3.")}
    c_ms = sum(v["ms"] for v in conv.values())
    c_work = sum(v["work"] for v in conv.values())
    c_launch = sum(v["launches"] for v in conv.values())
    achieved = c_work / (c_ms * 1e-3) / 1e12 if c_ms > 0 else None
    images = B * world
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
        "data": "synthetic (images ~ N(0,1), uniform labels over 1000 classes; random-init ResNet-50)",
        "config": {"workload": f"ResNet-50 training step (BASELINE configs[4]), {RESNET_HW}x{RESNET_HW}, "
                               f"per-GPU batch {B}, channels-last bf16, cross-entropy, "
                               + ("Adam lr 1e-3" if args.optimizer == "adam" else "SGD momentum 0.9")
                               + (", NCCL all-reduce of bucketed gradients overlapped with backward"
                                  if world > 1 else ""),
                   "model": "resnet50", "global_batch": images, "per_gpu_batch": B, "image_hw": RESNET_HW,
                   "parallelism": f"dp{world}",
                   "execution": ("CUDA graph replay of the captured step (xdna_train.graphs)" if graphed
                                 else "eager"),
                   "l2": "inputs larger than L2 (the step's activations are tens of GB)",
                   "train_gflop_per_step_per_gpu": round(total_fl / 1e9, 1),
                   "conv3x3_s1_gflop_per_step_per_gpu": round(c33_fl / 1e9, 1)},
        "e2e": {"value": round(images / (e2e_ms * 1e-3), 2), "unit": "images/s",
                "h2d_bytes_per_step": int(x_host.numel() * x_host.element_size() + y_host.numel() * 8),
                "d2h_bytes_per_step": 4},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1) if achieved else None, "peak": peak_s,
                     "unit": "TFLOP/s", "frac": round(achieved / peak_s, 4) if achieved else None,
                     "traffic": conv_step_traffic_bytes(),
                     "kernel": "3x3 stride-1 convolutions of the step (tcgen05 implicit GEMM: fwd, dgrad, wgrad)",
                     "launches_per_step": round(c_launch / 3, 1),
                     "gflop_per_launch": round(c_work / max(1, c_launch) / 1e9, 3),
                     "ms_per_launch": round(c_ms / max(1, c_launch), 5),
                     "peak_kind": f"{peak_kind}, sustained (kernels timed inside a long step)"},
        # work is FLOPs for the convolutions and GEMMs, algorithmic bytes for
        # the BatchNorm and gradient passes (MEM_LABELS, reported as GB/s)
        "kernel_times_per_step": {k: {"launches": round(v["launches"] / 3, 1), "ms": round(v["ms"] / 3, 4),
                                      ("gbs" if k.startswith(MEM_LABELS) else "tflops"):
                                      (round(v["work"] / (v["ms"] * 1e-3) / (1e9 if k.startswith(MEM_LABELS) else 1e12), 1)
                                       if v["ms"] else None)}
                                  for k, v in sorted(kt.items())},
        "step_tflops": round(total_fl / (ms * 1e-3) / 1e12, 1),
        "eager_images_per_s": round(images / (eager_ms * 1e-3), 2) if eager_ms else None,
        "final_loss": round(final_loss, 4),
        "gpu_launches": launches,
        "clocks": clk.summary(),
        "fallback_ops": dict(sorted(((k, v["calls"]) for k, v in fallbacks.items()), key=lambda kv: -kv[1])[:10]),
    }
    if ar_ms is not None:
        line["allreduce_ms_per_step"] = round(ar_ms, 4)
        line["allreduce_buckets"] = len(ar.buckets)
    return line


def cpu_resnet50_rate(steps: int, warmup: int, sample: int = RESNET_CPU_SAMPLE, optimizer: str = "sgd"):
    """images/s of the reference's CPU BF16 path (stock PyTorch CPU ops) on
    a bounded sample of the ResNet-50 step: ``sample`` images per step."""
    import torch.nn.functional as F
    model = resnet50_model("cpu")
    opt = _sgd_or_adam(model, optimizer, False)
    g = torch.Generator().manual_seed(1000)
    x = torch.randn(sample, 3, RESNET_HW, RESNET_HW, generator=g).bfloat16().contiguous(
        memory_format=torch.channels_last)
    y = torch.randint(0, 1000, (sample,), generator=g)

    def one():
        opt.zero_grad(set_to_none=True)
        F.cross_entropy(model(x).float(), y).backward()
        opt.step()

    dt = _timed(one, steps, warmup, lambda: None)
    return sample / dt, dt


def conv_step_traffic_bytes():
    """DRAM bytes per launch of the 3x3 conv kernels in the ResNet-50 step,
    from the committed ncu summary (None until one is committed)."""
    import re
    f = REPO / "profiles" / "conv3x3_resnet50_step_traffic.md"
    if not f.is_file():
        return None
    m = re.search(r"traffic_bytes_per_launch_B128:\s*(\d+)", f.read_text())
    return int(m.group(1)) if m else None


def run_resnet50_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    steps, warmup = max(1, args.steps), max(1, min(args.warmup, 3))
    rate, dt = cpu_resnet50_rate(steps, warmup, optimizer=args.optimizer)
    cores = torch.get_num_threads()
    return {
        "metric": METRIC, "value": round(rate, 3), "unit": "images/s", "impl": "reference",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": steps, "warmup": warmup,
        "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (images ~ N(0,1), uniform labels over 1000 classes)",
        "config": {"workload": f"ResNet-50 training step (BASELINE configs[4]), {RESNET_HW}x{RESNET_HW}, "
                               "channels-last bf16, cross-entropy, "
                               + ("Adam lr 1e-3" if args.optimizer == "adam" else "SGD momentum 0.9")
                               + ", on the reference's CPU BF16 path",
                   "model": "resnet50", "per_step_sample_images": RESNET_CPU_SAMPLE, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(rate, 3), "unit": "images/s", "cores": cores, "kind": "reference",
                         "sample": f"{RESNET_CPU_SAMPLE} images of 3x{RESNET_HW}x{RESNET_HW} per step (of the "
                                   f"{RESNET_BATCH}-image GPU batch); stock PyTorch CPU ops = the reference's CPU "
                                   f"path; torch {torch.__version__} (reference pins 2.14)"},
        "e2e": {"value": round(rate, 3), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------- the other BASELINE configs
# Model definitions written from BASELINE.json's config descriptions; used by
# `--workload` and by the GPU parity tests (tests/test_gpu_workloads.py).

def make_mlp():
    """Config 3: Linear 1024-4096-4096-4096-1024 with GELU between."""
    import torch.nn as nn
    return nn.Sequential(nn.Linear(1024, 4096), nn.GELU(), nn.Linear(4096, 4096), nn.GELU(),
                         nn.Linear(4096, 4096), nn.GELU(), nn.Linear(4096, 1024))


def make_style_generator():
    """Config 4 generator: 9x9 conv 3->32, stride-2 3x3 convs to 64 and 128, 5
    residual blocks (3x3 conv-BN-ReLU, 128 ch), two (nearest 2x upsample + 3x3
    conv) stages back to 32, 9x9 conv to 3."""
    import torch.nn as nn

    def cbr(ci, co, k, s=1):
        return [nn.Conv2d(ci, co, k, stride=s, padding=k // 2, bias=False), nn.BatchNorm2d(co), nn.ReLU()]

    class Res(nn.Module):
        def __init__(self, c):
            super().__init__()
            self.body = nn.Sequential(*cbr(c, c, 3), nn.Conv2d(c, c, 3, padding=1, bias=False), nn.BatchNorm2d(c))

        def forward(self, x):
            return torch.relu(self.body(x) + x)

    layers = cbr(3, 32, 9) + cbr(32, 64, 3, 2) + cbr(64, 128, 3, 2) + [Res(128) for _ in range(5)]
    layers += [nn.Upsample(scale_factor=2, mode="nearest")] + cbr(128, 64, 3)
    layers += [nn.Upsample(scale_factor=2, mode="nearest")] + cbr(64, 32, 3)
    layers += [nn.Conv2d(32, 3, 9, padding=4)]
    return nn.Sequential(*layers)


class _ConvNormAct(torch.nn.Module):
    """[nearest 2x upsample ->] 3x3 conv (no bias) -> BatchNorm2d -> LeakyReLU(0.2)."""

    def __init__(self, ci, co, stride=1, upsample=False):
        super().__init__()
        import torch.nn as nn
        self.upsample = upsample
        self.conv = nn.Conv2d(ci, co, 3, stride=stride, padding=1, bias=False)
        self.norm = nn.BatchNorm2d(co)
        self.act = nn.LeakyReLU(0.2)

    def forward(self, x):
        if self.upsample:
            x = torch.nn.functional.interpolate(x, scale_factor=2, mode="nearest")
        return self.act(self.norm(self.conv(x)))


class _LeakyRes(torch.nn.Module):
    """LeakyReLU(BN(conv(ConvNormAct(x))) + x), 3x3 convs without bias."""

    def __init__(self, c):
        super().__init__()
        import torch.nn as nn
        self.first = _ConvNormAct(c, c)
        self.conv = nn.Conv2d(c, c, 3, padding=1, bias=False)
        self.norm = nn.BatchNorm2d(c)
        self.act = nn.LeakyReLU(0.2)

    def forward(self, x):
        return self.act(self.norm(self.conv(self.first(x))) + x)


class RefStyleNet(torch.nn.Module):
    """The reference's own benchmark generator (`benchmarks/style_net.py:64-88`,
    the network its perceptual-loss region was written for), built from that
    description: encoder 3->64 (stride 1), ->128 and ->128 (stride 2) of
    conv-BN-LeakyReLU(0.2); 5 residual blocks at 128 channels; two decoder
    stages (nearest 2x upsample + conv-BN-LeakyReLU) fed with the encoder's
    skip maps concatenated on the channel axis; a conv-BN-LeakyReLU over
    [decoder, first encoder map, input] (195 -> 64 channels) and a 1x1 conv
    with bias to 3 channels."""

    def __init__(self, cin=3, cout=3, blocks=5):
        super().__init__()
        import torch.nn as nn
        self.enc0 = _ConvNormAct(cin, 64)
        self.enc1 = _ConvNormAct(64, 128, stride=2)
        self.enc2 = _ConvNormAct(128, 128, stride=2)
        self.blocks = nn.ModuleList(_LeakyRes(128) for _ in range(blocks))
        self.dec2 = _ConvNormAct(256, 128, upsample=True)
        self.dec1 = _ConvNormAct(256, 128, upsample=True)
        self.head = _ConvNormAct(128 + 64 + cin, 64)
        self.out = nn.Conv2d(64, cout, 1)

    def forward(self, x):
        e0 = self.enc0(x)
        e1 = self.enc1(e0)
        e2 = self.enc2(e1)
        r = e2.clone()
        for b in self.blocks:
            r = b(r)
        y = self.dec2(torch.cat([r, e2], dim=1))
        y = self.dec1(torch.cat([y, e1], dim=1))
        return self.out(self.head(torch.cat([y, e0, x], dim=1)))

    def norm_act_pairs(self):
        """(BatchNorm2d, LeakyReLU) pairs with nothing between them, for
        `regions.fuse_norm_activation` (the residual tail has an add between)."""
        return [(m.norm, m.act) for m in self.modules() if isinstance(m, _ConvNormAct)]


class _ImageNetNorm(torch.nn.Module):
    """(x - mean) / std per RGB channel, the constants cast to x's dtype."""

    def __init__(self):
        super().__init__()
        self.mean = torch.tensor([0.485, 0.456, 0.406]).view(1, 3, 1, 1)
        self.std = torch.tensor([0.229, 0.224, 0.225]).view(1, 3, 1, 1)

    def forward(self, x):
        return (x - self.mean.to(x.device, x.dtype)) / self.std.to(x.device, x.dtype)


class RefStyleLoss(torch.nn.Module):
    """The reference benchmark's loss (`benchmarks/style_net.py:90-144`), from
    its description: l_perceptual * mean((f(x) - f(t))**2) over the
    concatenated flattened outputs of frozen random-init VGG19 features 0, 3
    and 5 of the ImageNet-normalised images (target side without autograd),
    plus l_l1 * L1(x, t).  The module layout is the one
    `regions.fuse_perceptual_loss` matches."""

    def __init__(self, l_l1=4.0, l_perceptual=6.0, taps=(0, 3, 5)):
        super().__init__()
        from torchvision.models import vgg19
        self.perceptual_vgg = torch.nn.Module()
        self.perceptual_vgg.model = vgg19(weights=None).eval()
        self.perceptual_vgg.feature_layers = tuple(taps)
        self.perceptual_vgg.use_norm = True
        self.perceptual_vgg.norm = _ImageNetNorm()
        for q in self.perceptual_vgg.parameters():
            q.requires_grad_(False)
        self.l_l1, self.l_perceptual = l_l1, l_perceptual

    def features(self, x):
        net, maps = self.perceptual_vgg, []
        y = net.norm(x)
        for i in range(max(net.feature_layers) + 1):
            y = net.model.features[i](y)
            if i in net.feature_layers:
                maps.append(y.clone().view(y.shape[0], -1))
        return torch.cat(maps, dim=1)

    def compute_perceptual_loss(self, x, t):
        fx = self.features(x)
        with torch.no_grad():
            ft = self.features(t)
        return ((fx - ft) ** 2).mean()

    def forward(self, x, t):
        return self.l_perceptual * self.compute_perceptual_loss(x, t) + self.l_l1 * torch.nn.functional.l1_loss(x, t)




class StyleLoss(torch.nn.Module):
    """Config 4 loss: frozen random-init VGG19 features; content MSE over the
    concatenated taps plus Gram-matrix style MSE.  Follows the module pattern
    `fuse_perceptual_loss` accepts (perceptual_vgg.model.features,
    feature_layers, compute_perceptual_loss)."""

    def __init__(self, taps=(3, 8, 17), style_weight=1e-2):
        super().__init__()
        from torchvision.models import vgg19
        self.perceptual_vgg = torch.nn.Module()
        self.perceptual_vgg.model = vgg19(weights=None)
        self.perceptual_vgg.feature_layers = tuple(taps)
        self.perceptual_vgg.use_norm = False
        for q in self.perceptual_vgg.parameters():
            q.requires_grad_(False)
        self.style_weight = style_weight

    def features(self, x):
        maps, y = [], x
        for i in range(max(self.perceptual_vgg.feature_layers) + 1):
            y = self.perceptual_vgg.model.features[i](y)
            if i in self.perceptual_vgg.feature_layers:
                maps.append(y)
        return maps

    def compute_perceptual_loss(self, x, t):
        fx, ft = self.features(x), self.features(t)
        return torch.nn.functional.mse_loss(torch.cat([a.reshape(-1) for a in fx]),
                                            torch.cat([b.reshape(-1) for b in ft]))

    @staticmethod
    def gram(f):
        b, c, h, w = f.shape
        f = f.reshape(b, c, h * w)
        return torch.bmm(f, f.transpose(1, 2)) / (c * h * w)

    def forward(self, out, target, style):
        content = self.compute_perceptual_loss(out, target)
        with torch.no_grad():
            gs = [self.gram(f) for f in self.features(style)]
        go = [self.gram(f) for f in self.features(out)]
        sl = sum(torch.nn.functional.mse_loss(a.float(), b.float()) for a, b in zip(go, gs))
        return content.float() + self.style_weight * sl


def _timed(fn, steps, warmup, device_sync):
    for _ in range(warmup):
        fn()
    device_sync()
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    device_sync()
    return (time.perf_counter() - t0) / steps


def run_workload(args):
    """One JSON line for a non-headline BASELINE config (1, 3 or 4)."""
    import torch.nn as nn
    import torch.nn.functional as F

    import xdna_train
    xdna_train.register_xdna_device()
    world, rank, local = setup_dist(args)
    X = torch.device("xdna", local)
    sync = lambda: torch.xdna.synchronize()  # noqa: E731
    cpu = lambda: None  # noqa: E731
    w = args.workload
    out = {"workload": w, "n_gpus": world, "dtype": "bf16", "data": "synthetic", "steps": args.steps,
           "warmup": args.warmup}

    def cpu_rate(make_step, steps=2, warmup=1):
        if rank != 0 or world != 1 or args.no_cpu_baseline:
            return None
        return _timed(make_step(), steps, warmup, cpu)

    def graphed(make_step, key, scale, read_loss=False):
        """The same step captured once into a CUDA graph (xdna_train.graphs)
        and replayed: the step's kernels without the host's per-op dispatch
        (``read_loss``: every replay also reads the loss on the host)."""
        if world != 1:
            return
        from xdna_train import graphs
        try:
            replay = graphs.make_graphed_step(make_step(), warmup=max(3, args.warmup))
            fn = (lambda: replay().item()) if read_loss else replay
            out[key] = round(scale / _timed(fn, args.steps, 2, sync), 2)
        except Exception as e:  # reported, not hidden: the eager figure stands
            out[key + "_error"] = f"{type(e).__name__}: {e}"[:300]

    if w == "readme":
        # config 1: Conv2d(128,128,3,pad=1) BF16, x [16,128,36,36], target 0, Adam 1e-3
        def make(dev, capturable=False):
            torch.manual_seed(0)
            model = nn.Conv2d(128, 128, 3, padding=1).bfloat16().to(dev)
            opt = torch.optim.Adam(model.parameters(), lr=1e-3, fused=True, capturable=capturable)
            x = torch.randn(16, 128, 36, 36, dtype=torch.bfloat16).to(dev)
            tgt = torch.zeros_like(x)

            def step():
                opt.zero_grad(set_to_none=True)
                loss = F.mse_loss(model(x).float(), tgt.float())
                loss.backward()
                opt.step()
            return step
        dt = _timed(make(X), args.steps, args.warmup, sync)
        out.update(metric="README Conv2d training step it/s (BASELINE config 1)", value=round(1 / dt, 2),
                   unit="it/s", ms_per_step=round(dt * 1e3, 4),
                   tflops=round(18.35e9 / dt / 1e12, 1))
        graphed(lambda: make(X, True), "graphed_it_s", 1.0)
        c = cpu_rate(lambda: make("cpu"), steps=5, warmup=1)
    elif w == "mlp":
        # config 3: MLP B512, autocast BF16 over FP32 params (FP32 master state), Adam 1e-4
        def make(dev, capturable=False):
            torch.manual_seed(0)
            model = make_mlp().to(dev)
            opt = torch.optim.Adam(model.parameters(), lr=1e-4, fused=True, capturable=capturable)
            x = torch.randn(512, 1024).to(dev)
            tgt = torch.randn(512, 1024).to(dev)
            dtype = "xdna" if torch.device(dev).type == "xdna" else "cpu"

            def step():
                opt.zero_grad(set_to_none=True)
                with torch.autocast(dtype, dtype=torch.bfloat16):
                    loss = F.mse_loss(model(x).float(), tgt)
                loss.backward()
                opt.step()
            return step
        dt = _timed(make(X), args.steps, args.warmup, sync)
        out.update(metric="MLP training TFLOP/s (BASELINE config 3)", value=round(128.85e9 / dt / 1e12, 2),
                   unit="TFLOP/s", ms_per_step=round(dt * 1e3, 4))
        graphed(lambda: make(X, True), "graphed_tflops", 128.85e9 / 1e12)
        c = cpu_rate(lambda: make("cpu"))
        if c:
            c = c  # seconds per step
    elif w == "style":
        # config 4: B40 36x36 style transfer, Adam 1e-3, with and without the region
        from xdna_train import regions

        def make(dev, fused, fuse_norm=False, capturable=False):
            torch.manual_seed(0)
            gen = make_style_generator().bfloat16().to(dev)
            crit = StyleLoss().bfloat16().to(dev)
            if fused:
                assert regions.fuse_perceptual_loss(crit)
            if fuse_norm:
                # every BatchNorm2d directly followed by its ReLU in a Sequential
                for seq in [m for m in gen.modules() if isinstance(m, nn.Sequential)]:
                    mods = list(seq)
                    for a, b in zip(mods, mods[1:]):
                        if isinstance(a, nn.BatchNorm2d) and isinstance(b, nn.ReLU):
                            assert regions.fuse_norm_activation(a, b)
            opt = torch.optim.Adam(gen.parameters(), lr=1e-3, fused=True, capturable=capturable)
            g = torch.Generator().manual_seed(1)
            x = torch.rand(40, 3, 36, 36, generator=g).bfloat16().to(dev)
            tgt = torch.rand(40, 3, 36, 36, generator=g).bfloat16().to(dev)
            sty = torch.rand(40, 3, 36, 36, generator=g).bfloat16().to(dev)

            def step():
                opt.zero_grad(set_to_none=True)
                loss = crit(gen(x), tgt, sty)
                loss.backward()
                opt.step()
            return step
        dt = _timed(make(X, False), args.steps, args.warmup, sync)
        out.update(metric="style-transfer training it/s (BASELINE config 4)", value=round(1 / dt, 2), unit="it/s",
                   ms_per_step=round(dt * 1e3, 4))
        if not args.style_plain_only:
            dtf = _timed(make(X, True), args.steps, args.warmup, sync)
            dtn = _timed(make(X, True, True), args.steps, args.warmup, sync)
            out.update(fused_perceptual_loss_it_s=round(1 / dtf, 2), fused_perceptual_and_norm_act_it_s=round(1 / dtn, 2))
            graphed(lambda: make(X, False, capturable=True), "graphed_it_s", 1.0)
            graphed(lambda: make(X, True, True, capturable=True), "graphed_fused_perceptual_and_norm_act_it_s", 1.0)

            # The reference's own benchmark network and loss (benchmarks/end_to_end_speed.py: BF16, B40 36x36,
            # Adam lr 1e-4 wd 1e-5, the loss read on the host every step), eager plain / with the perceptual
            # region / with the region and the BatchNorm+LeakyReLU pairs fused, and replayed as a CUDA graph.
            def make_ref(dev, fused, fuse_norm=False, capturable=False):
                torch.manual_seed(0)
                net = RefStyleNet().bfloat16().to(dev)
                crit = RefStyleLoss().bfloat16().to(dev)
                if fused:
                    assert regions.fuse_perceptual_loss(crit)
                if fuse_norm:
                    for bn, act in net.norm_act_pairs():
                        assert regions.fuse_norm_activation(bn, act)
                opt = torch.optim.Adam(net.parameters(), lr=1e-4, weight_decay=1e-5, fused=True,
                                       capturable=capturable)
                g = torch.Generator().manual_seed(1)
                x = (torch.rand(40, 3, 36, 36, generator=g) * 2 - 1).bfloat16().to(dev)
                tgt = torch.rand(40, 3, 36, 36, generator=g).bfloat16().to(dev)

                def step():
                    loss = crit(net(x), tgt)
                    opt.zero_grad(set_to_none=True)
                    loss.backward()
                    opt.step()
                    return loss
                return step

            def read(step):
                return lambda: step().item()
            rn = {}
            for key, fl in (("eager_it_s", (False,)), ("fused_perceptual_loss_it_s", (True,)),
                            ("fused_perceptual_and_norm_act_it_s", (True, True))):
                rn[key] = round(1 / _timed(read(make_ref(X, *fl)), args.steps, args.warmup, sync), 2)
            out["reference_stylenet"] = rn
            graphed(lambda: make_ref(X, True, True, capturable=True), "reference_stylenet_graphed_it_s", 1.0,
                    read_loss=True)
            if rank == 0 and world == 1 and not args.no_cpu_baseline:
                rn["cpu_it_s"] = round(1 / _timed(read(make_ref("cpu", False)), 2, 1, cpu), 3)
        c = cpu_rate(lambda: make("cpu", False))
    else:
        raise SystemExit(f"unknown workload {w}")
    if c:
        if w == "readme":
            unit_scale = 1 / c
        elif w == "mlp":
            unit_scale = 128.85e9 / c / 1e12
        else:
            unit_scale = 1 / c
        out["cpu_baseline"] = {"value": round(unit_scale, 3), "unit": out["unit"], "cores": torch.get_num_threads(),
                               "kind": "reference", "sample": "same step on the reference's CPU BF16 path "
                                                              "(stock PyTorch CPU ops), few steps"}
    fb = xdna_train.fallback_stats()
    out["fallback_ops_top"] = dict(sorted(((k, v["calls"]) for k, v in fb.items()), key=lambda kv: -kv[1])[:8])
    out["kernel_launches"] = xdna_train.kernel_stats()
    return out if rank == 0 else None


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
    kt = kernel_times(x, dy, conv, 0, iters=args.iters, nhwc=args.channels % 8 == 0)
    fl = 2.0 * b * hw * hw * c * c * 9
    out = {k: {"ms": round(v, 4)} for k, v in kt.items()}
    for k in kt:
        if k != "pack_rows":
            out[k]["tflops"] = round(fl / (kt[k] * 1e-3) / 1e12, 1)
    out["pack_rows"]["gbs"] = round(2 * (x.numel() + b * (hw + 2) ** 2 * ((c + 63) // 64) * 64) / (kt["pack_rows"] * 1e-3) / 1e9, 1)
    print(json.dumps({"probe": f"B{b} C{c} HW{hw}", **out}), flush=True)


SWEEP_C = (32, 64, 128, 256, 512)
SWEEP_HW = (18, 36, 72, 144)
SWEEP_B = (8, 40, 128)


def conv_sweep(args):
    """BASELINE configs[1], the whole 3x3 conv sweep (``--conv-sweep``): for
    every C_in = C_out, H = W and batch of the config, the fwd / dgrad / wgrad
    kernels and the NCHW row packer timed separately on the device (CUDA
    events around back-to-back launches after two warm-up calls, as many as
    make ~30 ms per direction, 3 to 50), with TFLOP/s and the fraction of the
    measured dense-BF16 peak (padding to 64-channel chunks not counted as
    work).  The reference's CPU path (stock PyTorch CPU conv /
    convolution_backward) is timed beside it on a one-image sample per
    (C, H), for shapes up to ~1.5 GFLOP per image and direction.  One JSON
    line per shape, then a summary line."""
    import torch.nn as nn

    import xdna_train
    xdna_train.register_xdna_device()
    torch.cuda.set_device(0)
    X = torch.device("xdna", 0)
    peak, _, kind = peaks()
    cs = [args.channels] if args.sweep_one else SWEEP_C
    hws = [args.hw] if args.sweep_one else SWEEP_HW
    bs = [args.batch] if args.sweep_one else SWEEP_B
    cpu_tf = {}
    if not args.no_cpu_baseline:
        from oracle import cpu_path
        for c in cs:
            for hw in hws:
                if hw * hw * c * c > 1.1e8:
                    continue
                g = torch.Generator().manual_seed(c + hw)
                x = torch.randn(1, c, hw, hw, generator=g).bfloat16()
                dy = torch.randn(1, c, hw, hw, generator=g).bfloat16()
                w = (torch.randn(c, c, 3, 3, generator=g) * 0.05).bfloat16()
                fl = 2.0 * hw * hw * c * c * 9
                row = {}
                for k, fn in (("fwd", lambda: cpu_path.conv3x3_fwd(x, w)),
                              ("dgrad", lambda: cpu_path.conv3x3_bwd(dy, x, w, (True, False, False))),
                              ("wgrad", lambda: cpu_path.conv3x3_bwd(dy, x, w, (False, True, False)))):
                    fn()
                    t0 = time.perf_counter()
                    fn()
                    row[k] = round(fl / (time.perf_counter() - t0) / 1e12, 3)
                cpu_tf[(c, hw)] = row
    rows = []
    for c in cs:
        torch.manual_seed(c)
        conv = nn.Conv2d(c, c, 3, padding=1).bfloat16().to(X)
        for hw in hws:
            for b in bs:
                x = torch.randn(b, c, hw, hw, dtype=torch.bfloat16, device=X)
                dy = torch.randn(b, c, hw, hw, dtype=torch.bfloat16, device=X)
                fl = 2.0 * b * hw * hw * c * c * 9
                iters = max(3, min(50, int(0.03 / (fl / 1.2e15))))
                kt = kernel_times(x, dy, conv, 0, iters=iters)
                row = {"shape": f"B{b} C{c} HW{hw}", "batch": b, "channels": c, "hw": hw,
                       "gflop_per_direction": round(fl / 1e9, 3), "iters": iters}
                for k in ("fwd", "dgrad", "wgrad"):
                    tf = fl / (kt[k] * 1e-3) / 1e12
                    row[k] = {"us": round(kt[k] * 1e3, 2), "tflops": round(tf, 1), "frac": round(tf / peak, 4)}
                row["pack_rows_us"] = round(kt["pack_rows"] * 1e3, 2)
                if (c, hw) in cpu_tf:
                    row["cpu_tflops_1img"] = cpu_tf[(c, hw)]
                rows.append(row)
                print(json.dumps(row), flush=True)
                del x, dy
            torch.xdna.empty_cache()
    summary = sweep_summary(rows)
    summary.update(peak_tflops=peak, peak_kind=kind, cpu_threads=torch.get_num_threads() if cpu_tf else None)
    print(json.dumps({"probe": "conv3x3 sweep (BASELINE configs[1])", **summary}), flush=True)


def sweep_summary(rows):
    """Totals of ``--conv-sweep`` rows: work and kernel time summed over the
    three directions, the aggregate rate, and the fraction of peak over the
    large-channel shapes (C >= 256, H = W >= 36; the sweep's >= 60 % target)."""
    dirs = ("fwd", "dgrad", "wgrad")
    tot_fl = sum(r["gflop_per_direction"] for r in rows) * len(dirs)
    tot_us = sum(r[k]["us"] for r in rows for k in dirs)
    big = [r[k]["frac"] for r in rows for k in dirs if r["channels"] >= 256 and r["hw"] >= 36]
    return {"shapes": len(rows), "sum_gflop": round(tot_fl, 1), "sum_us": round(tot_us, 1),
            "aggregate_tflops": round(tot_fl * 1e9 / (tot_us * 1e-6) / 1e12, 1) if tot_us > 0 else None,
            "large_channel_min_frac": min(big) if big else None,
            "large_channel_median_frac": statistics.median(big) if big else None}


def bn_probe(args):
    """Device time of training-mode BatchNorm2d forward + backward on one
    channels-last shape (``--bn-probe --batch B --channels C --hw H``), with the
    algorithmic bandwidth: forward 6 B/elem (x read by the sums and by the
    apply pass, y written), backward 10 B/elem (dy and x read by the sums and
    by the dx pass, dx written).  The ncu small case of the BatchNorm kernels."""
    import torch.nn as nn

    import xdna_train
    xdna_train.register_xdna_device()
    torch.cuda.set_device(0)
    X = torch.device("xdna", 0)
    b, c, hw = args.batch, args.channels, args.hw
    cl = torch.channels_last
    bn = nn.BatchNorm2d(c).bfloat16().to(X)
    x = torch.randn(b, c, hw, hw, dtype=torch.bfloat16, device=X).contiguous(memory_format=cl).requires_grad_()
    g = torch.randn(b, c, hw, hw, dtype=torch.bfloat16, device=X).contiguous(memory_format=cl)
    st = torch.cuda.current_stream()
    times = {"fwd": [], "bwd": []}
    for i in range(args.iters + 3):
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(st)
        y = bn(x)
        xdna_train.materialize(y)  # the output pass waits for a reader: run it inside the forward's timing
        e1.record(st)
        y.backward(g)
        e2.record(st)
        torch.cuda.synchronize()
        if i >= 3:
            times["fwd"].append(e0.elapsed_time(e1))
            times["bwd"].append(e1.elapsed_time(e2))
        x.grad = None
    n = x.numel()
    out = {}
    for k, bpe in (("fwd", 6), ("bwd", 10)):
        ms = sorted(times[k])[len(times[k]) // 2]
        out[k] = {"ms": round(ms, 4), "gbs": round(bpe * n / (ms * 1e-3) / 1e9, 1)}
    print(json.dumps({"probe": f"BatchNorm2d channels-last B{b} C{c} HW{hw}", **out,
                      "kernels": xdna_train.kernel_stats()}), flush=True)


def adam_probe(args):
    """Device time of one fused Adam step over ``--params`` million fp32
    parameters (FP32 master weights, the MLP config's regime) or bf16 ones
    (``--adam-bf16``), in 4 tensors, through torch.optim.Adam on the xdna
    device; algorithmic bytes per element: fp32 28 (read g, p, m, v; write p,
    m, v), bf16 14.  The ncu small case of the Adam kernel."""
    import xdna_train
    xdna_train.register_xdna_device()
    torch.cuda.set_device(0)
    X = torch.device("xdna", 0)
    dt = torch.bfloat16 if args.adam_bf16 else torch.float32
    n = int(args.params * 1e6) // 4
    params = [torch.nn.Parameter(torch.randn(n, dtype=dt, device=X)) for _ in range(4)]
    for q in params:
        q.grad = torch.randn(n, dtype=dt, device=X)
    opt = torch.optim.Adam(params, lr=1e-4)
    st = torch.cuda.current_stream()
    ts = []
    for i in range(args.iters + 3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        opt.step()
        e1.record(st)
        torch.cuda.synchronize()
        if i >= 3:
            ts.append(e0.elapsed_time(e1))
    ms = sorted(ts)[len(ts) // 2]
    # the kernel alone, through the C ABI on the optimizer's own state
    import ctypes
    from xdna_train import _abi
    arr = (_abi.AdamTensor * 4)()
    for k, q in enumerate(params):
        stt = opt.state[q]
        arr[k] = _abi.AdamTensor(q.data_ptr(), q.grad.data_ptr(), stt["exp_avg"].data_ptr(),
                                 stt["exp_avg_sq"].data_ptr(), None, stt["step"].data_ptr(), n)
    code = _abi.B2_BF16 if args.adam_bf16 else _abi.B2_F32
    hp = _abi.AdamHparams(1e-4, 0.9, 0.999, 0.0, 1e-8, 0, 0, 0, code, code, None, None, None)
    kts = []
    for i in range(args.iters + 3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        _abi.check(_abi.lib().b2_fused_adam(arr, 4, ctypes.byref(hp), st.cuda_stream))
        e1.record(st)
        torch.cuda.synchronize()
        if i >= 3:
            kts.append(e0.elapsed_time(e1))
    kms = sorted(kts)[len(kts) // 2]
    bpe = 14 if args.adam_bf16 else 28
    elems = 4 * n
    print(json.dumps({"probe": f"fused Adam {elems / 1e6:.1f} M {str(dt).split('.')[-1]} parameters",
                      "step_ms": round(ms, 4), "step_gbs": round(bpe * elems / (ms * 1e-3) / 1e9, 1),
                      "kernel_ms": round(kms, 4), "kernel_gbs": round(bpe * elems / (kms * 1e-3) / 1e9, 1),
                      "note": "step = torch.optim.Adam.step() incl. host-side work and step-counter updates",
                      "kernels": xdna_train.kernel_stats()}), flush=True)


# The MLP's GEMMs at batch 512: (M, N, K, transA, transB)
# for each layer's forward (x . W^T), input gradient (dY . W) and weight
# gradient (dY^T . x), as nn.Linear's autograd issues them.
def mlp_gemm_shapes(batch=512, dims=(1024, 4096, 4096, 4096, 1024)):
    out = []
    for fi, fo in zip(dims[:-1], dims[1:]):
        out.append((f"fwd {fi}->{fo}", batch, fo, fi, 0, 1))
        out.append((f"dX {fo}->{fi}", batch, fi, fo, 0, 0))
        out.append((f"dW {fo}x{fi}", fo, fi, batch, 1, 0))
    return out


def gemm_probe(args):
    """Device time of b2_gemm_bf16 on the MLP's GEMM shapes (``--gemm-probe``),
    beside cuBLAS (torch.matmul on CUDA tensors) for the same product: CUDA
    events around 20 back-to-back calls after warm-up, the median of
    ``--iters`` timings; TFLOP/s = 2*M*N*K / time against the measured burst
    peak.  The ncu small case of the GEMM kernel."""
    from xdna_train import _abi
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    st = torch.cuda.current_stream()
    peak, _, kind = peaks()
    reps = 20

    def med(fn):
        ts = []
        for i in range(args.iters + 3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(reps):
                fn()
            e1.record(st)
            torch.cuda.synchronize()
            if i >= 3:
                ts.append(e0.elapsed_time(e1) / reps)
        return sorted(ts)[len(ts) // 2]

    rows, tot_o, tot_l, tot_f = [], 0.0, 0.0, 0.0
    shapes = mlp_gemm_shapes(args.batch if args.batch != B_PER_GPU else 512)
    if args.shape_index >= 0:
        shapes = [shapes[args.shape_index]]
    for name, M, N, K, ta, tb in shapes:
        g = torch.Generator(device=dev).manual_seed(M + N + K)
        A = torch.randn(K if ta else M, M if ta else K, generator=g, device=dev).bfloat16()
        Bm = torch.randn(N if tb else K, K if tb else N, generator=g, device=dev).bfloat16()
        D = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        lda, ldb = A.shape[1], Bm.shape[1]
        s = st.cuda_stream
        wsb = _abi.lib().b2_gemm_bf16_workspace_bytes(M, N, K, 1)
        ws = torch.empty(max(16, wsb), dtype=torch.uint8, device=dev)
        ours = med(lambda: _abi.call("b2_gemm_bf16_ws", ta, tb, M, N, K, 1.0, A.data_ptr(), lda, 0, Bm.data_ptr(),
                                     ldb, 0, 0.0, None, _abi.B2_BF16, 0, 0, 0, D.data_ptr(), N, 0, 1, ws.data_ptr(),
                                     wsb, s))
        opA = A.t() if ta else A
        opB = Bm.t() if tb else Bm
        lib = med(lambda: torch.matmul(opA, opB))
        ref = torch.matmul(opA.float(), opB.float())
        err = ((D.float() - ref).abs().max() / ref.abs().max()).item()
        fl = 2.0 * M * N * K
        tot_o += ours
        tot_l += lib
        tot_f += fl
        row = {"shape": name, "M": M, "N": N, "K": K, "split_k_workspace": wsb,
               "ours_us": round(ours * 1e3, 2), "cublas_us": round(lib * 1e3, 2),
               "ours_tflops": round(fl / (ours * 1e-3) / 1e12, 1), "frac": round(fl / (ours * 1e-3) / 1e12 / peak, 4),
               "max_rel_err": round(err, 5)}
        rows.append(row)
        print(json.dumps(row), flush=True)
    print(json.dumps({"probe": "MLP GEMMs (BASELINE configs[2])", "ours_us_total": round(tot_o * 1e3, 1),
                      "cublas_us_total": round(tot_l * 1e3, 1),
                      "ours_tflops": round(tot_f / (tot_o * 1e-3) / 1e12, 1),
                      "cublas_tflops": round(tot_f / (tot_l * 1e-3) / 1e12, 1), "peak_tflops": peak,
                      "peak_kind": kind}), flush=True)


# ResNet-50's 1x1 convolutions at stride 1: (H*W, Cin, Cout) per layer kind
RESNET50_1X1 = [(3136, 64, 64), (3136, 64, 256), (3136, 256, 64), (3136, 256, 128), (784, 128, 512),
                (784, 512, 128), (784, 512, 256), (196, 256, 1024), (196, 1024, 256), (196, 1024, 512),
                (49, 512, 2048), (49, 2048, 512)]


def conv1x1_probe(args):
    """Device times of the channels-last 1x1 convolution kernels (forward,
    dgrad, wgrad with its ordered reduce) on ResNet-50's stride-1 shapes at
    ``--batch``, beside ATen's CUDA library kernels for the same convolution
    (``--conv1x1-probe``).  CUDA tensors and the C ABI only; nothing is
    registered.  Each timing replays 20 calls captured into one CUDA graph:
    device time for both sides.  FLOPs per direction 2*P*Cin*Cout."""
    from xdna_train import _abi
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    st = torch.cuda.current_stream()
    b = args.batch
    cl = torch.channels_last

    reps = 20

    def med(fn):
        # `reps` calls captured into one CUDA graph and replayed, so that both
        # sides are timed on the device only (no host dispatch between calls)
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                fn()
        ts = []
        for i in range(args.iters + 3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            g.replay()
            e1.record(st)
            torch.cuda.synchronize()
            if i >= 3:
                ts.append(e0.elapsed_time(e1) / reps)
        g.reset()
        return sorted(ts)[len(ts) // 2]

    rows = []
    shapes = RESNET50_1X1 if args.shape_index < 0 else [RESNET50_1X1[args.shape_index]]
    for hw2, cin, cout in shapes:
        hw = int(round(hw2 ** 0.5))
        x = torch.randn(b, cin, hw, hw, dtype=torch.bfloat16, device=dev).contiguous(memory_format=cl)
        w = torch.randn(cout, cin, 1, 1, dtype=torch.bfloat16, device=dev)
        dy = torch.randn(b, cout, hw, hw, dtype=torch.bfloat16, device=dev).contiguous(memory_format=cl)
        y = torch.empty_like(dy)
        dx = torch.empty_like(x)
        dw = torch.empty(cout, cin, dtype=torch.float32, device=dev)
        wsb = _abi.lib().b2_conv1x1_wgrad_workspace_bytes(1, b, cin, hw2, cout)
        ws = torch.empty(max(1, wsb), dtype=torch.uint8, device=dev)
        s = st.cuda_stream

        def cs():  # the stream a call is made on (the capture stream inside med)
            return torch.cuda.current_stream().cuda_stream

        ours = {
            "fwd": med(lambda: _abi.call("b2_conv1x1_fwd", x.data_ptr(), w.data_ptr(), None, y.data_ptr(), 1, b, cin,
                                         hw2, cout, cs())),
            "dgrad": med(lambda: _abi.call("b2_conv1x1_dgrad", dy.data_ptr(), w.data_ptr(), dx.data_ptr(), 1, b, cin,
                                           hw2, cout, cs())),
            "wgrad": med(lambda: _abi.call("b2_conv1x1_wgrad", dy.data_ptr(), x.data_ptr(), dw.data_ptr(),
                                           _abi.B2_F32, 1, b, cin, hw2, cout, ws.data_ptr(), wsb, cs())),
        }
        ref = torch.nn.functional.conv2d(x, w)
        yo = ref.float()
        lib = {
            "fwd": med(lambda: torch.nn.functional.conv2d(x, w)),
            "dgrad": med(lambda: torch.ops.aten.convolution_backward(dy, x, w, None, [1, 1], [0, 0], [1, 1], False,
                                                                     [0, 0], 1, [True, False, False])),
            "wgrad": med(lambda: torch.ops.aten.convolution_backward(dy, x, w, None, [1, 1], [0, 0], [1, 1], False,
                                                                     [0, 0], 1, [False, True, False])),
        }
        # the forward against the library's, as a sanity check of the timed call
        _abi.call("b2_conv1x1_fwd", x.data_ptr(), w.data_ptr(), None, y.data_ptr(), 1, b, cin, hw2, cout, s)
        err = ((y.float() - yo).abs().max() / yo.abs().max().clamp_min(1e-6)).item()
        fl = 2.0 * b * hw2 * cin * cout
        row = {"shape": f"P{b * hw2} Cin{cin} Cout{cout}", "fwd_rel_err": round(err, 5)}
        for k in ("fwd", "dgrad", "wgrad"):
            row[k] = {"ours_us": round(ours[k] * 1e3, 1), "lib_us": round(lib[k] * 1e3, 1),
                      "ours_tflops": round(fl / (ours[k] * 1e-3) / 1e12, 1)}
        rows.append(row)
        print(json.dumps(row), flush=True)
    tot_o = sum(r[k]["ours_us"] for r in rows for k in ("fwd", "dgrad", "wgrad"))
    tot_l = sum(r[k]["lib_us"] for r in rows for k in ("fwd", "dgrad", "wgrad"))
    print(json.dumps({"probe": f"conv1x1 channels-last B{b}", "ours_us_total": round(tot_o, 1),
                      "lib_us_total": round(tot_l, 1)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel-probe", action="store_true")
    ap.add_argument("--conv1x1-probe", action="store_true")
    ap.add_argument("--gemm-probe", action="store_true", help="b2_gemm_bf16 on the MLP's GEMM shapes vs cuBLAS")
    ap.add_argument("--conv-sweep", action="store_true", help="BASELINE configs[1]: every shape of the 3x3 sweep")
    ap.add_argument("--sweep-one", action="store_true", help="--conv-sweep: only --batch/--channels/--hw")
    ap.add_argument("--shape-index", type=int, default=-1, help="--conv1x1-probe / --gemm-probe: one shape of the list")
    ap.add_argument("--style-plain-only", action="store_true",
                    help="--workload style: the eager plain-loss variant only (launch-list captures)")
    ap.add_argument("--bn-probe", action="store_true")
    ap.add_argument("--adam-probe", action="store_true")
    ap.add_argument("--adam-bf16", action="store_true")
    ap.add_argument("--params", type=float, default=64.0, help="--adam-probe: millions of parameters")
    ap.add_argument("--optimizer", default="sgd", choices=["sgd", "adam"], help="--workload resnet50: optimizer")
    ap.add_argument("--workload", default="resnet50", choices=["resnet50", "conv", "readme", "mlp", "style"],
                    help="resnet50 (default, the headline) or another BASELINE config")
    ap.add_argument("--batch", type=int, default=B_PER_GPU)
    ap.add_argument("--channels", type=int, default=C)
    ap.add_argument("--hw", type=int, default=HW)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (resnet50: 100, conv: 200, others: 200)")
    ap.add_argument("--warmup", type=int, default=None, help="warm-up steps (resnet50: 20, others: 5)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="resnet50: time the eager step, not its CUDA-graph replay")
    ap.add_argument("--channels-last", action="store_true", help="--workload conv: channels-last activations")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 100 if args.workload == "resnet50" else 200
    if args.warmup is None:
        args.warmup = 20 if args.workload == "resnet50" else 5
    if args.kernel_probe:
        kernel_probe(args)
        return
    if args.conv_sweep:
        conv_sweep(args)
        return
    if args.bn_probe:
        bn_probe(args)
        return
    if args.conv1x1_probe:
        conv1x1_probe(args)
        return
    if args.gemm_probe:
        gemm_probe(args)
        return
    if args.adam_probe:
        adam_probe(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.workload not in ("conv", "resnet50"):
        line = run_workload(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            cuda_barrier()
            dist.destroy_process_group()
        return
    args.warmup = max(3, args.warmup) if args.impl == "ours" else args.warmup
    if args.impl == "reference":
        line = run_resnet50_reference(args) if args.workload == "resnet50" else run_conv_reference(args)
    elif args.workload == "resnet50":
        line = run_resnet50(args)
        if line is not None and not args.no_cpu_baseline and line["n_gpus"] == 1:
            rate, dt = cpu_resnet50_rate(steps=3, warmup=1, optimizer=args.optimizer)
            line["cpu_baseline"] = {
                "value": round(rate, 3), "unit": "images/s", "cores": torch.get_num_threads(), "kind": "reference",
                "sample": f"{RESNET_CPU_SAMPLE} images per step, 3 timed steps after 1 warm-up; the same ResNet-50 "
                          "step on stock PyTorch CPU BF16 ops (the reference's CPU path)"}
    else:
        line = run_conv_layer(args)
        if line is not None and not args.no_cpu_baseline and line["n_gpus"] == 1:
            rate, dt = cpu_reference_step_rate(steps=3, warmup=1)
            line["cpu_baseline"] = {
                "value": round(rate, 3), "unit": "images/s", "cores": torch.get_num_threads(), "kind": "reference",
                "sample": f"{CPU_SAMPLE} images per step, 3 timed steps after 1 warmup; stock PyTorch CPU BF16 "
                          "conv/convolution_backward/_fused_adam_ (the reference's CPU path)"}
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1 and args.impl == "ours":
        import torch.distributed as dist
        cuda_barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
