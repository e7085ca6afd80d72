"""Fused training regions on the xdna device.

Two opt-in rewrites with the public contract of torch-xdna2's
``xdna_train.regions`` (``regions.py:1-31, 392-420, 426-548`` there):

``fuse_perceptual_loss(loss_module, features_attr="perceptual_vgg")``
    The perceptual MSE of a frozen VGG-style feature stack (Conv2d, ReLU and
    2x2/2 MaxPool2d layers, selected taps) becomes one autograd node.  The
    convolutions still dispatch to the xdna backend's sm_100a kernels; the
    ReLU, ReLU + max-pool, squared-difference reduction and the backward's
    tap / ReLU / max-pool passes are single fused region kernels
    (``b2_region_*``).  Neither the tap copies nor their concatenation are
    materialized, and the loss never leaves the device.

``fuse_norm_activation(bn, act)``
    A training ``BatchNorm2d`` followed directly by its ``ReLU`` /
    ``LeakyReLU`` runs as one op: statistics plus the activated output in two
    passes over the input, the backward's parameter sums and input gradient
    in two more (``b2_region_bn_*``).

Both keep eligibility semantic -- layer types, dtypes, device, requires_grad,
training mode -- and fall back to the modules' own code for anything else.
``XDNA_REGIONS=0`` turns both off.  On this device every convolution runs on
the GPU, so the reference's per-convolution CPU/NPU placement has no
counterpart here.
"""
from __future__ import annotations

import os
import weakref

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd.function import once_differentiable
from torch.nn.modules import module as _module_globals
from torch.nn.utils import parametrize

#: Inputs smaller than this many bytes keep the eager BatchNorm / activation
#: pair (4 MB, the reference's default): below it the fused op's Python-level
#: autograd node costs more host time than the activation pass it saves.
#: ``XDNA_REGION_NORM_ACT_MIN_BYTES`` overrides it.
NORM_ACT_MIN_BYTES = int(os.environ.get("XDNA_REGION_NORM_ACT_MIN_BYTES", "4000000"))


def enabled() -> bool:
    return os.environ.get("XDNA_REGIONS", "1") != "0"


def _ext():
    from . import device
    device.register_xdna_device()
    return device._C


def _is_unmodified(m: nn.Module, cls: type) -> bool:
    """``m`` is exactly a ``cls`` whose forward nothing wraps or replaces:
    no instance-level forward, no module or global hooks, no
    parametrization -- anything the fused code would silently skip."""
    if type(m) is not cls or "forward" in m.__dict__ or parametrize.is_parametrized(m):
        return False
    if m._forward_hooks or m._forward_pre_hooks or m._backward_hooks or m._backward_pre_hooks:
        return False
    return not (_module_globals._global_forward_hooks or _module_globals._global_forward_pre_hooks)


# ---------------------------------------------------------------------------
# perceptual loss: the feature stack compiled into stages
# ---------------------------------------------------------------------------

def _stage_of(m: nn.Module):
    """(kind, key) of a layer the region runs, or None.  ``key`` captures
    everything the compiled program depends on, so a program is reused only
    while every layer still describes the same."""
    if _is_unmodified(m, nn.Conv2d):
        if m.padding_mode != "zeros" or isinstance(m.padding, str):
            return None
        return "conv", (id(m), id(m.weight), id(m.bias), tuple(m.stride), tuple(m.padding), tuple(m.dilation),
                        m.groups)
    if _is_unmodified(m, nn.ReLU):
        return "relu", (id(m),)
    if _is_unmodified(m, nn.MaxPool2d):
        two = lambda v: v in (2, (2, 2))  # noqa: E731
        if (two(m.kernel_size) and two(m.stride) and m.padding in (0, (0, 0)) and m.dilation in (1, (1, 1))
                and not m.ceil_mode and not m.return_indices):
            return "pool", (id(m),)
    return None


class _Program:
    """The layers 0..last_tap of a feature stack as stages.

    ``kinds[i]``  "conv" / "relu" / "pool";
    ``convs[i]``  the Conv2d of a conv stage (its frozen weight is read on
                  every call, so in-place weight updates are seen);
    ``taps``      sorted tap indices, ``tapped`` the same as a set;
    ``key``       the layers' descriptions at compile time."""

    __slots__ = ("kinds", "convs", "taps", "tapped", "key")

    def __init__(self, kinds, convs, taps, key):
        self.kinds, self.convs, self.taps, self.key = kinds, convs, taps, key
        self.tapped = frozenset(taps)

    @property
    def last(self) -> int:
        return self.taps[-1]


def _compile(layers, taps) -> _Program | None:
    taps = tuple(sorted({int(t) for t in taps}))
    layers = list(layers)
    if not taps or taps[0] < 0 or taps[-1] >= len(layers):
        return None
    kinds, convs, key = [], [], []
    for m in layers[: taps[-1] + 1]:
        st = _stage_of(m)
        if st is None:
            return None
        kind, k = st
        if kind == "conv" and (m.weight.requires_grad or (m.bias is not None and m.bias.requires_grad)):
            return None  # the region produces no weight gradients
        kinds.append(kind)
        convs.append(m if kind == "conv" else None)
        key.append(st)
    if kinds[0] != "conv":
        return None
    return _Program(tuple(kinds), tuple(convs), taps, tuple(key))


def _runs_here(prog: _Program, x: torch.Tensor, target: torch.Tensor) -> bool:
    """The region applies to this call: bf16 4-D xdna images of one shape, a
    target without gradient, an input that wants one (under grad mode), and
    frozen bf16 xdna feature weights."""
    if not enabled() or x.device.type != "xdna" or target.device.type != "xdna":
        return False
    if x.dtype != torch.bfloat16 or target.dtype != torch.bfloat16 or x.dim() != 4 or x.shape != target.shape:
        return False
    if target.requires_grad or (torch.is_grad_enabled() and not x.requires_grad):
        return False
    for conv in prog.convs:
        if conv is None:
            continue
        w, b = conv.weight, conv.bias
        if w.device.type != "xdna" or w.dtype != torch.bfloat16 or w.requires_grad:
            return False
        if b is not None and b.requires_grad:
            return False
    return True


def _evaluate(prog: _Program, img: torch.Tensor, retain_all: bool) -> dict:
    """Run stages 0..last on ``img``; returns {stage: output} for every stage
    (``retain_all``) or only for the taps.  A ReLU followed by a pool runs as
    one fused kernel producing both outputs."""
    ext = _ext()
    acts = {}
    cur = img
    k, end = 0, prog.last + 1
    while k < end:
        kind = prog.kinds[k]
        first = k
        if kind == "conv":
            c = prog.convs[k]
            cur = F.conv2d(cur, c.weight, c.bias, c.stride, c.padding, c.dilation, c.groups).contiguous()
            acts[k] = cur
            k += 1
        elif kind == "relu" and k + 1 < end and prog.kinds[k + 1] == "pool":
            n, ch, h, w = cur.shape
            act = torch.empty_like(cur)
            pooled = torch.empty(n, ch, h // 2, w // 2, dtype=cur.dtype, device=cur.device)
            ext.region_relu_maxpool2(cur, act, pooled)
            acts[k], acts[k + 1] = act, pooled
            cur = pooled
            k += 2
        elif kind == "relu":
            act = torch.empty_like(cur)
            ext.region_relu(cur, act)
            acts[k] = cur = act
            k += 1
        else:
            cur = F.max_pool2d(cur, 2, 2)
            acts[k] = cur
            k += 1
        if not retain_all:
            for j in range(first, k):
                if j not in prog.tapped:
                    acts.pop(j, None)
    return acts


class _PerceptualMSE(torch.autograd.Function):
    """mean over the concatenated tap elements of (f(x) - f(target))**2 for
    the compiled feature stack f; dX only (the features are frozen)."""

    @staticmethod
    def forward(ctx, prog, x, target, *weights):
        ext = _ext()
        with torch.no_grad():
            xa = _evaluate(prog, x, retain_all=True)
            ta = _evaluate(prog, target, retain_all=False)
            count = sum(xa[k].numel() for k in prog.taps)
            # per-tap sums of squares in double, left on the device
            loss = torch.stack([ext.region_sqdiff_sum_tensor(xa[k], ta[k]) for k in prog.taps]).sum() / count
        stages = sorted(xa)
        tapped = list(prog.taps)
        ctx.save_for_backward(x, *(xa[k] for k in stages), *(ta[k] for k in tapped), *weights)
        ctx.layout = (prog, stages, tapped, count)
        return loss.to(torch.bfloat16)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_loss):
        ext = _ext()
        prog, stages, tapped, count = ctx.layout
        saved = ctx.saved_tensors
        img = saved[0]
        xa = dict(zip(stages, saved[1:1 + len(stages)]))
        ta = dict(zip(tapped, saved[1 + len(stages):1 + len(stages) + len(tapped)]))
        weights = iter(saved[1 + len(stages) + len(tapped):])
        weight_of = {k: next(weights) for k in range(prog.last + 1) if prog.kinds[k] == "conv"}
        # d loss / d (tap) = 2 (f(x) - f(t)) / count.  The walk below computes
        # the gradient for an incoming gradient of 1 and scales the result by
        # grad_loss at the end, so no device value is read on the host.
        coef = 2.0 / count
        grad = None  # gradient w.r.t. the output of stage k (None: still zero)
        for k in range(prog.last, -1, -1):
            kind, out, tap = prog.kinds[k], xa[k], k in prog.tapped
            if kind == "relu":
                nxt = torch.empty_like(out)
                ext.region_relu_bwd(out, grad, out if tap else None, ta[k] if tap else None, nxt, coef)
                grad = nxt
                continue
            if tap:
                nxt = torch.empty_like(out)
                ext.region_addtap(grad, out, ta[k], nxt, coef)
                grad = nxt
            below = xa[k - 1] if k > 0 else img
            if kind == "pool":
                nxt = torch.empty_like(below)
                ext.region_maxpool2_bwd(below, grad, nxt)
                grad = nxt
            else:
                c = prog.convs[k]
                grad = torch.ops.aten.convolution_backward(grad.contiguous(), below, weight_of[k], None,
                                                           list(c.stride), list(c.padding), list(c.dilation), False,
                                                           [0, 0], c.groups, [True, False, False])[0]
        return (None, grad * grad_loss.to(grad.dtype), None) + (None,) * len(weight_of)


def _feature_parts(owner, attr):
    """(feature layers up to the last tap, taps, normalisation or None) of a
    loss module following the pattern ``<attr>.model.features`` (a
    Sequential), ``<attr>.feature_layers`` (tap indices), optional
    ``<attr>.use_norm`` / ``<attr>.norm`` (with ``mean`` / ``std``); None if
    the module does not follow it."""
    net = getattr(owner, attr, None)
    feats = getattr(getattr(net, "model", None), "features", None)
    taps = getattr(net, "feature_layers", None)
    if feats is None or taps is None or len(taps) == 0:
        return None
    norm = getattr(net, "norm", None) if getattr(net, "use_norm", False) else None
    if norm is not None and (getattr(norm, "mean", None) is None or getattr(norm, "std", None) is None):
        return None
    return list(feats)[: max(int(t) for t in taps) + 1], taps, norm


class _FusedPerceptual:
    """Installed as ``owner.compute_perceptual_loss``: the region when the
    call is eligible, the class's own method otherwise.  Holds its owner, so
    ``copy.deepcopy`` of the loss module produces a copy bound to the copy
    (whose program is recompiled against the copied layers)."""

    def __init__(self, owner, attr):
        self.owner = owner
        self.attr = attr
        self.prog = None
        self.consts = None  # (mean, std, key, device mean, device std)

    def _program(self):
        parts = _feature_parts(self.owner, self.attr)
        if parts is None:
            return None, None
        layers, taps, norm = parts
        want = tuple(sorted({int(t) for t in taps}))
        p = self.prog
        if p is None or p.taps != want or p.key != tuple(_stage_of(m) for m in layers):
            p = self.prog = _compile(layers, taps)
        return p, norm

    def _normalised(self, norm, x, t):
        """(x - mean) / std and the same for t.  Tensor constants are copied to
        the device once per device, dtype and tensor version (the eager
        normalisation copies its CPU constants on every call; with no copy
        after the first call, the region can be captured in a CUDA graph)."""
        mean, std = norm.mean, norm.std
        if not (isinstance(mean, torch.Tensor) and isinstance(std, torch.Tensor)):
            m = torch.as_tensor(mean).to(device=x.device, dtype=x.dtype).view(1, -1, 1, 1)
            s = torch.as_tensor(std).to(device=x.device, dtype=x.dtype).view(1, -1, 1, 1)
        else:
            key = (mean._version, std._version, x.device, x.dtype)
            c = self.consts
            if c is None or c[0] is not mean or c[1] is not std or c[2] != key:
                c = self.consts = (mean, std, key, mean.to(device=x.device, dtype=x.dtype).view(1, -1, 1, 1),
                                   std.to(device=x.device, dtype=x.dtype).view(1, -1, 1, 1))
            m, s = c[3], c[4]
        return (x - m) / s, (t - m) / s

    def __call__(self, input, target):
        owner = self.owner
        prog, norm = self._program() if enabled() else (None, None)
        if prog is None or not _runs_here(prog, input, target):
            return type(owner).compute_perceptual_loss(owner, input, target)
        x, t = self._normalised(norm, input, target) if norm is not None else (input, target)
        weights = [c.weight for c in prog.convs if c is not None]
        return _PerceptualMSE.apply(prog, x, t, *weights)


def fuse_perceptual_loss(loss_module, features_attr: str = "perceptual_vgg") -> bool:
    """Route ``loss_module.compute_perceptual_loss(input, target)`` through the
    fused region when the module follows the pattern (``features_attr`` with
    ``model.features``, ``feature_layers`` and optional ``use_norm`` /
    ``norm``) and its loss is the mean squared difference over the
    concatenated taps.  Returns True if installed.  Eligibility of every call
    is checked again (dtypes, device, frozen weights, gradient wanted), and a
    changed feature stack is recompiled (reference: regions.py:392-420)."""
    if not enabled() or not hasattr(loss_module, "compute_perceptual_loss"):
        return False
    parts = _feature_parts(loss_module, features_attr)
    if parts is None or _compile(parts[0], parts[1]) is None:
        return False
    loss_module.__dict__["compute_perceptual_loss"] = _FusedPerceptual(loss_module, features_attr)
    return True


# ---------------------------------------------------------------------------
# norm + activation: training BatchNorm2d and its ReLU / LeakyReLU as one op
# ---------------------------------------------------------------------------

class _BatchNormAct(torch.autograd.Function):
    """act(batch_norm(x)) in training mode, contiguous NCHW bf16 on xdna.

    Per-channel statistics over (N, H, W); the biased variance normalises and
    the unbiased one moves the running variance by ``factor``.  The backward
    needs x, the activated output y (its sign is the activation's mask), the
    weight and the fp32 per-channel mean / inverse std of the forward, and
    returns the gradients autograd asks for.  Not double differentiable."""

    @staticmethod
    def forward(ctx, x, weight, bias, running_mean, running_var, eps, slope, factor, plain_relu):
        y, stats = _ext().region_bn_forward(x, weight, bias, running_mean, running_var, eps, slope, factor)
        ctx.save_for_backward(x, y, weight, stats)
        ctx.slope, ctx.plain_relu = slope, plain_relu
        return y

    @staticmethod
    @once_differentiable
    def backward(ctx, dy):
        x, y, weight, stats = ctx.saved_tensors
        need = ctx.needs_input_grad[:3]
        grads = (None, None, None)
        if any(need):
            grads = _ext().region_bn_backward(dy, y, x, weight, stats, need[0], need[1], need[2], ctx.slope,
                                              ctx.plain_relu)
        return tuple(grads) + (None,) * 6


def _activation_slope(act):
    """Negative-side slope of a plain ReLU (0.0) or LeakyReLU; None for any
    other module, subclasses included (their forward may differ)."""
    if type(act) is nn.ReLU:
        return 0.0
    if type(act) is nn.LeakyReLU:
        return float(act.negative_slope)
    return None


def _bf16_on_device(t, n: int) -> bool:
    return (isinstance(t, torch.Tensor) and t.device.type == "xdna" and t.dtype == torch.bfloat16
            and t.is_contiguous() and t.numel() == n)


def _norm_act_applies(bn: nn.BatchNorm2d, x) -> bool:
    """Training statistics of an affine norm that tracks running statistics
    with a float momentum, on a contiguous 4-D bf16 xdna input with more than
    one value per channel and at least NORM_ACT_MIN_BYTES, with bf16 xdna
    parameters and buffers."""
    if not (enabled() and bn.training and bn.track_running_stats and bn.affine and bn.momentum is not None):
        return False
    if not isinstance(x, torch.Tensor) or x.dim() != 4 or not _bf16_on_device(x, x.numel()):
        return False
    c = x.shape[1]
    if c == 0 or x.numel() // c <= 1 or 2 * x.numel() < NORM_ACT_MIN_BYTES:
        return False
    return all(_bf16_on_device(t, c) for t in (bn.weight, bn.bias, bn.running_mean, bn.running_var))


# Fused outputs whose paired activation has not run yet: id(tensor) ->
# (weak reference to the tensor, the activation).  Keyed by identity (a
# tensor's == is elementwise); an entry leaves with its tensor.
_AWAITING_ACT: dict = {}


def _await_act(y: torch.Tensor, act: nn.Module) -> None:
    key = id(y)
    _AWAITING_ACT[key] = (weakref.ref(y, lambda _r, k=key: _AWAITING_ACT.pop(k, None)), act)


def _awaiting(t) -> nn.Module | None:
    entry = _AWAITING_ACT.get(id(t))
    return entry[1] if entry is not None and entry[0]() is t else None


class _NormForward:
    """Replaces the norm's forward: the fused op where it applies (the
    activation is looked up at every call), the class's forward otherwise."""

    def __init__(self, bn, act):
        self.bn, self.act = bn, act

    def __call__(self, x):
        bn, act = self.bn, self.act
        slope = _activation_slope(act)
        # a negative slope would break the y > 0 mask the backward uses
        if slope is None or slope < 0.0 or not _norm_act_applies(bn, x):
            return type(bn).forward(bn, x)
        bn.num_batches_tracked.add_(1)
        y = _BatchNormAct.apply(x, bn.weight, bn.bias, bn.running_mean, bn.running_var, float(bn.eps), slope,
                                float(bn.momentum), type(act) is nn.ReLU)
        _await_act(y, act)
        return y


class _ActForward:
    """Replaces the activation's forward: a tensor its norm already activated
    passes through unchanged, once; anything else is activated."""

    def __init__(self, act):
        self.act = act

    def __call__(self, x):
        if isinstance(x, torch.Tensor) and _awaiting(x) is self.act:
            _AWAITING_ACT.pop(id(x), None)
            return x
        return type(self.act).forward(self.act, x)


def paired_activation(bn: nn.Module):
    """The activation ``fuse_norm_activation`` paired with ``bn``, or None."""
    fwd = bn.__dict__.get("forward")
    return fwd.act if isinstance(fwd, _NormForward) else None


def activation_pending(t: torch.Tensor) -> bool:
    """``t`` came out of a fused norm and its paired activation has not yet
    passed it through."""
    return _awaiting(t) is not None


def fuse_norm_activation(bn: nn.BatchNorm2d, act: nn.Module) -> bool:
    """Declare that ``act`` (an ``nn.ReLU`` or ``nn.LeakyReLU``) is applied
    directly to the output of ``bn`` (an ``nn.BatchNorm2d``) and run the pair
    as one fused op where eligible (reference: regions.py:508-548).

    Only the two modules' ``forward`` are replaced (by callables holding the
    modules, so ``copy.deepcopy`` of a model holding both keeps a working
    pair); parameters, buffers and state_dict keys are untouched.  Where the
    fused op applies (training mode, contiguous bf16 NCHW xdna input, affine,
    tracked statistics with a float momentum, at least NORM_ACT_MIN_BYTES),
    ``bn(x)`` returns the activated tensor and the next call of ``act`` on
    that exact tensor returns it unchanged, once; otherwise both modules run
    their own forward.  The caller vouches for the dataflow: a pair with
    anything in between (an add, a branch) must not be declared.  Returns
    True if the pair is installed (or already was)."""
    if not enabled() or type(bn) is not nn.BatchNorm2d or _activation_slope(act) is None:
        return False
    current = paired_activation(bn)
    if current is not None:
        return current is act
    bn.__dict__["forward"] = _NormForward(bn, act)
    if not isinstance(act.__dict__.get("forward"), _ActForward):
        act.__dict__["forward"] = _ActForward(act)
    return True
