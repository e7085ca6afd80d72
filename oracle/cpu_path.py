"""The reference's CPU BF16 path for the offloaded training step -- TEST
INFRASTRUCTURE ONLY (tests/, smoke() and bench.py's CPU baseline).

With ``npu_mode`` 0, or for any op its NPU runtimes decline, the reference
runs the stock ATen CPU kernel on zero-copy CPU aliases of the device memory:
  convolution            torch_xdna_device.cpp:4594-4603  at::_ops::convolution::call
  convolution_backward   torch_xdna_device.cpp:4862-4873  at::_ops::convolution_backward::call
  mm / addmm / bmm       torch_xdna_device.cpp:4382, 3764, 3787
  _fused_adam_           torch_xdna_device.cpp:5196-5198 (boxed CPU fallback)
Calling the same ATen CPU ops on ``device="cpu"`` tensors is therefore the
reference's own arithmetic for this path (docs/usage.md:208-209 says the same:
mode 0 is the CPU path).  The reference pins torch 2.14; this environment has
torch 2.11, a version skew recorded next to every parity figure.
"""
from __future__ import annotations

import torch


def conv3x3_fwd(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    return torch.ops.aten.convolution(x.cpu(), w.cpu(), None if b is None else b.cpu(), [1, 1], [1, 1],
                                      [1, 1], False, [0, 0], 1)


def conv3x3_bwd(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor, mask=(True, True, False)):
    """(dX, dW, dB) of the 3x3/s1/p1 conv on the reference's CPU path."""
    return torch.ops.aten.convolution_backward(dy.cpu(), x.cpu(), w.cpu(), None, [1, 1], [1, 1], [1, 1],
                                               False, [0, 0], 1, list(mask))


def conv_train_step_cpu(x, w, bias, dy, exp_avg, exp_avg_sq, step, lr=1e-3):
    """One CPU step of the bench workload: fwd + dgrad + wgrad + fused Adam."""
    y = conv3x3_fwd(x, w, bias)
    dx, dw, db = conv3x3_bwd(dy, x, w, (True, True, True))
    step += 1
    torch._fused_adam_([w, bias], [dw, db], exp_avg, exp_avg_sq, [], [step, step.clone()], lr=lr,
                       beta1=0.9, beta2=0.999, weight_decay=0.0, eps=1e-8, amsgrad=False, maximize=False)
    return y, dx


def fp32_reference_conv(x, w, b=None):
    """FP32 conv of the same bf16 inputs (the tolerance anchor)."""
    return torch.nn.functional.conv2d(x.float().cpu(), w.float().cpu(), None if b is None else b.float().cpu(),
                                      padding=1)
