"""Training regions: a pattern of eager ops run as one autograd node.

``fuse_perceptual_loss`` replaces a frozen-VGG perceptual MSE loss

    features = frozen Sequential(conv, relu, conv, relu, maxpool, conv, ...)
    loss = mean over the concatenated selected taps of (features(x) - features(t))**2

by one autograd node (the reference's ``regions.py:1-31`` contract): the
convolutions still dispatch through the xdna backend (so they run the sm_100a
conv kernels), while ReLU, ReLU+max-pool, the squared-difference reduction and
the backward's tap/ReLU/max-pool passes run as single fused CUDA region
kernels (``b2_region_*``).  The concatenation and the tap clones of the eager
loss are never materialized.

Contract (unchanged from the reference)
  * inputs: ``x`` (bf16 xdna, requires grad), ``target`` (bf16 xdna, no grad);
    feature weights are read, never modified, and must not require grad.
  * output: a bf16 scalar, the mean over the concatenated tap elements.
  * backward produces dX only; not double-differentiable; retain_graph works.
  * numerics: bf16 storage, fp32 arithmetic in the fused kernels rounded once
    to bf16, the squared-difference sum accumulated in double on the device
    (no host synchronization; the incoming gradient scales dX at the end).
  * eligibility is semantic (layer types, dtype, device, requires_grad);
    anything else takes the module's own method.  ``XDNA_REGIONS=0`` disables.

``fuse_norm_activation`` runs a training ``BatchNorm2d`` and the ``ReLU`` /
``LeakyReLU`` applied directly to its output as one op (the reference's
``regions.py:426-548`` contract): statistics and the activated output in two
passes over the input, the backward's parameter sums and input gradient in
two more (``b2_region_bn_*``).

The reference also times CPU vs NPU placement per convolution (its
``_Placer``); on B200 every convolution runs on the GPU, so there is nothing to
place.
"""
from __future__ import annotations

import os
import types
import weakref
from dataclasses import dataclass, field

import torch
import torch.nn as nn
from torch.autograd.function import once_differentiable
from torch.nn.modules import module as _modmod
from torch.nn.utils import parametrize
import torch.nn.functional as F


_C_MOD = None


def _native():
    global _C_MOD
    if _C_MOD is None:
        from . import device
        device.register_xdna_device()
        _C_MOD = device._C
    return _C_MOD


def enabled() -> bool:
    return os.environ.get("XDNA_REGIONS", "1") != "0"


def _plain(m, cls) -> bool:
    """``m`` is exactly ``cls`` with nothing around its forward the region would skip."""
    if type(m) is not cls or "forward" in m.__dict__:
        return False
    if m._forward_hooks or m._forward_pre_hooks or m._backward_hooks or m._backward_pre_hooks:
        return False
    if _modmod._global_forward_hooks or _modmod._global_forward_pre_hooks:
        return False
    return not parametrize.is_parametrized(m)


def _layer_sig(m):
    """What the parsed chain depends on for one layer (None: unsupported).
    Re-checked on every call, so later model surgery is never missed."""
    if _plain(m, nn.Conv2d):
        if m.padding_mode != "zeros" or isinstance(m.padding, str):
            return None
        return ("conv", id(m.weight), id(m.bias), tuple(m.stride), tuple(m.padding), tuple(m.dilation), m.groups)
    if _plain(m, nn.ReLU):
        return ("relu",)
    if (_plain(m, nn.MaxPool2d) and m.kernel_size in (2, (2, 2)) and m.stride in (2, (2, 2))
            and m.padding in (0, (0, 0)) and m.dilation in (1, (1, 1)) and not m.ceil_mode
            and not m.return_indices):
        return ("maxpool2",)
    return None


@dataclass
class _Op:
    kind: str  # "conv" | "relu" | "maxpool2"
    weight: torch.Tensor | None = None
    bias: torch.Tensor | None = None
    stride: tuple = (1, 1)
    padding: tuple = (0, 0)
    dilation: tuple = (1, 1)
    groups: int = 1


@dataclass
class FrozenFeatureChain:
    ops: list
    taps: tuple
    _tapset: frozenset = field(init=False)
    sig: tuple = field(init=False, default=())

    def __post_init__(self):
        self._tapset = frozenset(self.taps)

    @classmethod
    def from_sequential(cls, layers, taps):
        """Parse ``layers[0 .. max(taps)]``; None if a layer is unsupported."""
        layers = list(layers)
        taps = tuple(sorted(set(int(t) for t in taps)))
        if not taps or taps[0] < 0 or taps[-1] >= len(layers):
            return None
        ops, sigs = [], []
        for m in layers[: taps[-1] + 1]:
            sig = _layer_sig(m)
            if sig is None:
                return None
            sigs.append(sig)
            if sig[0] == "conv":
                if m.weight.requires_grad or (m.bias is not None and m.bias.requires_grad):
                    return None
                ops.append(_Op("conv", m.weight, m.bias, tuple(m.stride), tuple(m.padding), tuple(m.dilation),
                               m.groups))
            else:
                ops.append(_Op(sig[0]))
        if ops[0].kind != "conv":
            return None
        chain = cls(ops, taps)
        chain.sig = tuple(sigs)
        return chain

    def eligible(self, x: torch.Tensor, target: torch.Tensor) -> bool:
        if not enabled() or x.device.type != "xdna" or target.device.type != "xdna":
            return False
        if x.dtype != torch.bfloat16 or target.dtype != torch.bfloat16:
            return False
        if x.dim() != 4 or x.shape != target.shape or target.requires_grad:
            return False
        if torch.is_grad_enabled() and not x.requires_grad:
            return False
        for op in self.ops:
            if op.kind != "conv":
                continue
            if op.weight.device.type != "xdna" or op.weight.dtype != torch.bfloat16:
                return False
            if op.weight.requires_grad or (op.bias is not None and op.bias.requires_grad):
                return False
        return True


def _forward_pass(chain: FrozenFeatureChain, x: torch.Tensor, keep_all: bool):
    """outs[i] = output of op i (None once neither a tap nor the next op needs it)."""
    C = _native()
    outs = [None] * len(chain.ops)
    cur = x
    i, n = 0, len(chain.ops)
    while i < n:
        op = chain.ops[i]
        if op.kind == "conv":
            cur = F.conv2d(cur, op.weight, op.bias, op.stride, op.padding, op.dilation, op.groups)
            if not cur.is_contiguous():
                cur = cur.contiguous()
            outs[i] = cur
            i += 1
        elif op.kind == "relu":
            r = torch.empty_like(cur)
            if i + 1 < n and chain.ops[i + 1].kind == "maxpool2" and cur.dim() == 4:
                p = torch.empty(cur.shape[0], cur.shape[1], cur.shape[2] // 2, cur.shape[3] // 2, dtype=cur.dtype,
                                device=cur.device)
                C.region_relu_maxpool2(cur, r, p)
                outs[i], outs[i + 1] = r, p
                cur = p
                i += 2
            else:
                C.region_relu(cur, r)
                outs[i] = r
                cur = r
                i += 1
        else:  # maxpool2 not preceded by relu
            cur = F.max_pool2d(cur, 2, 2)
            outs[i] = cur
            i += 1
        if not keep_all:
            for j in range(i - 1):
                if j not in chain._tapset:
                    outs[j] = None
    return outs


class _FrozenFeatureMSE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, chain, x, target):
        C = _native()
        with torch.no_grad():
            g_outs = _forward_pass(chain, x, keep_all=True)
            t_outs = _forward_pass(chain, target, keep_all=False)
            total = 0
            parts = []
            for k in chain.taps:
                total += g_outs[k].numel()
                # per-tap sums stay on the device: no host synchronization
                parts.append(C.region_sqdiff_sum_tensor(g_outs[k], t_outs[k]))
            sq = torch.stack(parts).sum()
        gi = [i for i, t in enumerate(g_outs) if t is not None]
        ti = [i for i, t in enumerate(t_outs) if t is not None]
        weights = [op.weight for op in chain.ops if op.kind == "conv"]
        ctx.save_for_backward(x, *[g_outs[i] for i in gi], *[t_outs[i] for i in ti], *weights)
        ctx.meta = (chain, gi, ti, total)
        return (sq / total).to(torch.bfloat16)

    @staticmethod
    @once_differentiable
    def backward(ctx, go):
        C = _native()
        chain, gi, ti, total = ctx.meta
        saved = ctx.saved_tensors
        x = saved[0]
        g_outs = [None] * len(chain.ops)
        t_outs = [None] * len(chain.ops)
        for n, i in enumerate(gi):
            g_outs[i] = saved[1 + n]
        for n, i in enumerate(ti):
            t_outs[i] = saved[1 + len(gi) + n]
        weights = iter(saved[1 + len(gi) + len(ti):])
        w_of = {k: next(weights) for k, o in enumerate(chain.ops) if o.kind == "conv"}
        # The backward is linear in the incoming gradient `go`: run it for go = 1
        # and scale dX by go at the end, so that no device value is read on the
        # host (the reference folds float(go) into the scale, regions.py:313).
        scale = 2.0 / total
        G = None  # gradient w.r.t. the output of the op being processed
        for k in range(chain.taps[-1], -1, -1):
            op = chain.ops[k]
            tapped = k in chain._tapset
            out_k = g_outs[k]
            if op.kind == "relu":
                new = torch.empty_like(out_k)
                if tapped:
                    C.region_relu_bwd(out_k, G, out_k, t_outs[k], new, scale)
                else:
                    C.region_relu_bwd(out_k, G, None, None, new, scale)
                G = new
                continue
            if tapped:  # G (+)= scale * (out - target_out)
                new = torch.empty_like(out_k)
                C.region_addtap(G, out_k, t_outs[k], new, scale)
                G = new
            src = g_outs[k - 1] if k > 0 else x
            if op.kind == "maxpool2":
                new = torch.empty_like(src)
                C.region_maxpool2_bwd(src, G, new)
                G = new
            else:  # conv: dX only
                if not G.is_contiguous():
                    G = G.contiguous()
                G = torch.ops.aten.convolution_backward(G, src, w_of[k], None, list(op.stride), list(op.padding),
                                                        list(op.dilation), False, [0, 0], op.groups,
                                                        [True, False, False])[0]
        return None, G * go.to(G.dtype), None


def frozen_feature_mse(chain: FrozenFeatureChain, x: torch.Tensor, target: torch.Tensor):
    """mean over the concatenated tap elements of (feat(x) - feat(target))**2."""
    return _FrozenFeatureMSE.apply(chain, x, target)


def _loss_chain(loss_module):
    cfg = loss_module.__dict__["_xdna_region_cfg"]
    net = getattr(loss_module, cfg["features_attr"], None)
    feats = getattr(getattr(net, "model", None), "features", None)
    taps = getattr(net, "feature_layers", None)
    if feats is None or taps is None:
        return None
    layers = list(feats)[: max(taps) + 1] if len(taps) else []
    chain = loss_module.__dict__.get("_xdna_chain")
    if chain is not None:
        want = tuple(sorted(set(int(t) for t in taps)))
        if chain.taps != want or chain.sig != tuple(_layer_sig(m) for m in layers):
            chain = None
    if chain is None:
        chain = FrozenFeatureChain.from_sequential(layers, taps)
        loss_module.__dict__["_xdna_chain"] = chain
    return chain


def _fused_compute_perceptual_loss(self, input, target):
    chain = _loss_chain(self)
    if chain is None or not enabled() or not chain.eligible(input, target):
        return type(self).compute_perceptual_loss(self, input, target)
    net = getattr(self, self.__dict__["_xdna_region_cfg"]["features_attr"])
    x, t = input, target
    norm = getattr(net, "norm", None) if getattr(net, "use_norm", False) else None
    if norm is not None:
        mean, std = getattr(norm, "mean", None), getattr(norm, "std", None)
        if mean is None or std is None:
            return type(self).compute_perceptual_loss(self, input, target)
        m, s = _norm_constants(self, mean, std, x)
        x = (x - m) / s
        t = (t - m) / s
    return frozen_feature_mse(chain, x, t)


def _norm_constants(loss_module, mean, std, x):
    """mean / std as [1, C, 1, 1] tensors of x's dtype on x's device.  The
    reference's normalisation keeps them as CPU tensors and copies them on
    every call; the copies are cached here per device, dtype and tensor
    version, so that after the first call no host-to-device copy is issued
    (a captured CUDA graph may contain none from pageable memory).  Constants
    that are not tensors (lists, tuples) are converted on every call."""
    m = torch.as_tensor(mean, dtype=x.dtype, device=x.device).view(1, -1, 1, 1) \
        if not isinstance(mean, torch.Tensor) else None
    s = torch.as_tensor(std, dtype=x.dtype, device=x.device).view(1, -1, 1, 1) \
        if not isinstance(std, torch.Tensor) else None
    if m is not None or s is not None:
        if m is None:
            m = mean.to(device=x.device, dtype=x.dtype).view(1, -1, 1, 1)
        if s is None:
            s = std.to(device=x.device, dtype=x.dtype).view(1, -1, 1, 1)
        return m, s
    key = (mean._version, std._version, x.device, x.dtype)
    hit = loss_module.__dict__.get("_xdna_norm_consts")
    if hit is not None and hit[0] is mean and hit[1] is std and hit[2] == key:
        return hit[3], hit[4]
    m = mean.to(device=x.device, dtype=x.dtype).view(1, -1, 1, 1)
    s = std.to(device=x.device, dtype=x.dtype).view(1, -1, 1, 1)
    loss_module.__dict__["_xdna_norm_consts"] = (mean, std, key, m, s)
    return m, s


def fuse_perceptual_loss(loss_module, features_attr: str = "perceptual_vgg") -> bool:
    """Route ``loss_module.compute_perceptual_loss`` through the region when the
    module follows the common pattern: ``getattr(loss_module, features_attr)``
    has ``model.features`` (a Sequential), ``feature_layers`` (tap indices),
    optional ``use_norm`` / ``norm``, and the loss is the mean squared tap
    difference.  Returns True if installed (reference: regions.py:392-420).
    Every call re-checks eligibility; the wrapper is bound to the module, so a
    deepcopy uses its own weights."""
    if not enabled():
        return False
    net = getattr(loss_module, features_attr, None)
    feats = getattr(getattr(net, "model", None), "features", None)
    taps = getattr(net, "feature_layers", None)
    if feats is None or taps is None or not hasattr(loss_module, "compute_perceptual_loss"):
        return False
    if FrozenFeatureChain.from_sequential(list(feats)[: max(taps) + 1], taps) is None:
        return False
    if getattr(net, "use_norm", False):
        norm = getattr(net, "norm", None)
        if getattr(norm, "mean", None) is None or getattr(norm, "std", None) is None:
            return False
    loss_module.__dict__["_xdna_region_cfg"] = {"features_attr": features_attr}
    loss_module.compute_perceptual_loss = types.MethodType(_fused_compute_perceptual_loss, loss_module)
    return True



# ---------------------------------------------------------------------------
# fuse_norm_activation: training BatchNorm2d + ReLU / LeakyReLU as one op
# ---------------------------------------------------------------------------

#: Inputs smaller than this many bytes keep the eager pair (the reference's
#: default, 4 MB).  The eager BatchNorm runs this backend's own kernels too;
#: below this size the fused op's Python-level autograd node costs more host
#: time than the activation pass it saves.  ``XDNA_REGION_NORM_ACT_MIN_BYTES``
#: overrides it.
_NORM_ACT_MIN_BYTES = int(os.environ.get("XDNA_REGION_NORM_ACT_MIN_BYTES", "4000000"))


class _BatchNormAct(torch.autograd.Function):
    """act(batch_norm(x)) in training mode on contiguous NCHW bf16 xdna tensors.

    Statistics over (N, H, W) per channel; the biased variance normalizes, the
    unbiased one moves the running variance (once per call, by ``factor``);
    affine weight and bias.  Backward reads x, the activated output y (its sign
    is the activation mask), the weight and the fp32 per-channel mean and
    inverse std saved by the forward; it returns the input, weight and bias
    gradients that autograd asks for.  Not double differentiable."""

    @staticmethod
    def forward(ctx, x, weight, bias, running_mean, running_var, eps, slope, factor, relu):
        # outputs allocated by the binding: one native call per direction
        y, stats = _native().region_bn_forward(x, weight, bias, running_mean, running_var, eps, slope, factor)
        ctx.save_for_backward(x, y, weight, stats)
        ctx.slope, ctx.relu = slope, relu
        return y

    @staticmethod
    @once_differentiable
    def backward(ctx, dy):
        x, y, weight, stats = ctx.saved_tensors
        want_x, want_w, want_b = ctx.needs_input_grad[:3]
        if not (want_x or want_w or want_b):
            return (None,) * 9
        dx, dw, db = _native().region_bn_backward(dy, y, x, weight, stats, want_x, want_w, want_b, ctx.slope,
                                                  ctx.relu)
        return dx, dw, db, None, None, None, None, None, None


def _bf16_xdna(t, n) -> bool:
    return (isinstance(t, torch.Tensor) and t.device.type == "xdna" and t.dtype == torch.bfloat16
            and t.is_contiguous() and t.numel() == n)


def _norm_act_eligible(bn: nn.BatchNorm2d, x) -> bool:
    """The fused op applies to training-mode statistics of an affine norm with
    tracked running statistics and a float momentum, on a contiguous 4-D bf16
    xdna input with more than one value per channel, at least
    ``_NORM_ACT_MIN_BYTES`` large, with bf16 xdna parameters and buffers."""
    if not (enabled() and bn.training and bn.track_running_stats and bn.affine) or bn.momentum is None:
        return False
    if not isinstance(x, torch.Tensor) or x.dim() != 4 or not _bf16_xdna(x, x.numel()):
        return False
    channels = x.shape[1]
    if channels == 0 or x.numel() // channels <= 1 or 2 * x.numel() < _NORM_ACT_MIN_BYTES:
        return False
    return all(_bf16_xdna(t, channels) for t in (bn.weight, bn.bias, bn.running_mean, bn.running_var))


def _act_slope(act):
    """Negative slope of a plain ReLU (0) or LeakyReLU; None for anything else
    (subclasses included: their forward could differ)."""
    if type(act) is nn.ReLU:
        return 0.0
    if type(act) is nn.LeakyReLU:
        return float(act.negative_slope)
    return None


def _fused_bn_forward(self, x):
    # Bound to the norm module itself, so copy.deepcopy rebinds it to the copy;
    # the paired activation and its slope are looked up on every call.
    act = self.__dict__.get("_xdna_pair")
    slope = None if act is None else _act_slope(act)
    # a negative slope breaks the y > 0 mask the backward relies on
    if slope is None or slope < 0.0 or not _norm_act_eligible(self, x):
        return type(self).forward(self, x)
    self.num_batches_tracked.add_(1)
    y = _BatchNormAct.apply(x, self.weight, self.bias, self.running_mean, self.running_var,
                            float(self.eps), slope, float(self.momentum), type(act) is nn.ReLU)
    y._xdna_act_for = weakref.ref(act)
    return y


def _checked_act_forward(self, x):
    # The paired norm already activated this exact tensor: pass it through,
    # once.  Any other input is activated normally.
    owner = getattr(x, "_xdna_act_for", None)
    if owner is not None and owner() is self:
        x._xdna_act_for = None
        return x
    return type(self).forward(self, x)


def fuse_norm_activation(bn: nn.BatchNorm2d, act: nn.Module) -> bool:
    """Declare that ``act`` (an ``nn.ReLU`` or ``nn.LeakyReLU``) is applied
    directly to the output of ``bn`` (an ``nn.BatchNorm2d``) and run the pair as
    one fused op where eligible (reference: regions.py:508-548).

    Parameters, buffers and state_dict keys are untouched; only the two
    ``forward`` methods are replaced, by methods bound to the modules, so a
    ``copy.deepcopy`` of a model holding both modules keeps a working pair.
    When eligible (training mode, contiguous bf16 NCHW xdna input, affine,
    tracked statistics with a float momentum, at least
    ``_NORM_ACT_MIN_BYTES``), ``bn(x)`` returns the activated tensor and the
    next call of ``act`` on that exact tensor returns it unchanged, once;
    otherwise both modules run their own forward.  The caller vouches for the
    dataflow: a pair with anything in between (an add, a branch) must not be
    declared.  Returns True if the pair is installed (or already was)."""
    if not enabled() or type(bn) is not nn.BatchNorm2d or _act_slope(act) is None:
        return False
    paired = bn.__dict__.get("_xdna_pair")
    if paired is not None:
        return paired is act
    object.__setattr__(bn, "_xdna_pair", act)  # a plain attribute, not a submodule
    bn.forward = types.MethodType(_fused_bn_forward, bn)
    fwd = act.__dict__.get("forward")
    if not (isinstance(fwd, types.MethodType) and fwd.__func__ is _checked_act_forward):
        act.forward = types.MethodType(_checked_act_forward, act)
    return True
