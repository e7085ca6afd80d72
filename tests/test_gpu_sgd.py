"""Fused SGD (b2_fused_sgd, aten::_fused_sgd_ on xdna) against the oracle's
restatement (oracle.sgd_step, bit-exact) and ATen's CUDA _fused_sgd_ on the
same inputs, through the C ABI and through torch.optim.SGD(fused=True).

torch.optim.SGD's fused path is what the reference's _prefer_fused_optimizer
selects for device parameters (xdna_train/device.py:408-436); its ResNet-50
configuration trains with SGD momentum 0.9.  The bar is
bit-exact against the oracle.  ATen's CUDA kernel evaluates the same
definition with fp32 intermediates where this library keeps the products in
double, so against it the bar is a few rounding steps of the operands'
magnitude (under cancellation an fp32 product's rounding shows at the
product's scale, not the result's).
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from xdna_train import _abi

pytestmark = pytest.mark.gpu

SIZES = [1, 7, 8, 9, 4096, 8191, 8192, 8193, 100_003]

OPTS = [
    dict(lr=0.1, momentum=0.9),
    dict(lr=0.05, momentum=0.9, weight_decay=1e-4, nesterov=True),
    dict(lr=0.01, momentum=0.8, dampening=0.1, maximize=True),
    dict(lr=0.1, momentum=0.9, first_step=True, weight_decay=5e-4),
    dict(lr=0.2, weight_decay=1e-2),  # no momentum: no buffers
    dict(lr=0.1, momentum=0.9, grad_scale=1024.0),
]


def _st():
    return torch.cuda.current_stream().cuda_stream


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _run_abi(ps, gs, bs, dtype, o):
    n = len(ps)
    arr = (_abi.SgdTensor * n)()
    for i in range(n):
        arr[i] = _abi.SgdTensor(ps[i].data_ptr(), gs[i].data_ptr(), bs[i].data_ptr() if bs else None, ps[i].numel())
    scale = None
    if o.get("grad_scale"):
        scale = torch.tensor([o["grad_scale"]], dtype=torch.float32, device=ps[0].device)
    hp = _abi.SgdHparams(o["lr"], o.get("weight_decay", 0.0), o.get("momentum", 0.0), o.get("dampening", 0.0),
                         int(o.get("nesterov", False)), int(o.get("maximize", False)), int(o.get("first_step", False)),
                         _abi.B2_BF16 if dtype == torch.bfloat16 else _abi.B2_F32, None,
                         scale.data_ptr() if scale is not None else None, None)
    _abi.check(_abi.lib().b2_fused_sgd(arr, n, ctypes.byref(hp), _st()), "b2_fused_sgd")
    torch.cuda.synchronize()


def _inputs(cuda, dtype, sizes, seed):
    g = torch.Generator().manual_seed(seed)
    ps = [torch.randn(n, generator=g).to(dtype).to(cuda) for n in sizes]
    gs = [torch.randn(n, generator=g).to(dtype).to(cuda) for n in sizes]
    bs = [torch.randn(n, generator=g).to(dtype).to(cuda) for n in sizes]
    return ps, gs, bs


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("oi", range(len(OPTS)))
def test_fused_sgd_bit_exact_vs_oracle(cuda, dtype, oi):
    o = OPTS[oi]
    ps, gs, bs = _inputs(cuda, dtype, SIZES, seed=oi)
    has_buf = o.get("momentum", 0.0) != 0.0
    bf = dtype == torch.bfloat16
    enc = _bits if bf else (lambda t: t.detach().cpu().numpy().copy())
    want = [oracle.sgd_step(enc(p), enc(g), enc(b) if has_buf else None, o["lr"], o.get("weight_decay", 0.0),
                            o.get("momentum", 0.0), o.get("dampening", 0.0), o.get("nesterov", False),
                            o.get("maximize", False), o.get("first_step", False), o.get("grad_scale"), bf16=bf)
            for p, g, b in zip(ps, gs, bs)]
    _run_abi(ps, gs, bs if has_buf else None, dtype, o)
    for (wp, wg, wb), p, g, b in zip(want, ps, gs, bs):
        assert np.array_equal(enc(p), wp)
        assert np.array_equal(enc(g), wg)
        if has_buf:
            assert np.array_equal(enc(b), wb)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_sgd_matches_aten_cuda_kernel(cuda, dtype):
    # 130 tensors (more than one launch's table), misaligned views among them
    sizes = [(i * 977) % 20011 + 1 for i in range(130)]
    for oi, o in enumerate(OPTS):
        ps, gs, bs = _inputs(cuda, dtype, sizes, seed=100 + oi)
        ps[3], gs[3], bs[3] = ps[3][1:], gs[3][1:], bs[3][1:]  # 2- or 4-byte offset: scalar path
        has_buf = o.get("momentum", 0.0) != 0.0
        rp, rg, rb = [p.clone() for p in ps], [g.clone() for g in gs], [b.clone() for b in bs]
        scale = torch.tensor(o["grad_scale"], device=cuda) if o.get("grad_scale") else None
        torch._fused_sgd_(rp, rg, rb if has_buf else [], weight_decay=o.get("weight_decay", 0.0),
                          momentum=o.get("momentum", 0.0), lr=o["lr"], dampening=o.get("dampening", 0.0),
                          nesterov=o.get("nesterov", False), maximize=o.get("maximize", False),
                          is_first_step=o.get("first_step", False), grad_scale=scale)
        _run_abi(ps, gs, bs if has_buf else None, dtype, o)
        m, wd, lr = o.get("momentum", 0.0), o.get("weight_decay", 0.0), o["lr"]
        step = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -24  # half an ulp, relative
        # magnitudes of the operands each stored value is formed from
        p_in = [p.float() for p in _inputs(cuda, dtype, sizes, seed=100 + oi)[0]]
        g_in = [g.float() for g in _inputs(cuda, dtype, sizes, seed=100 + oi)[1]]
        b_in = [b.float() for b in _inputs(cuda, dtype, sizes, seed=100 + oi)[2]]
        for lst in (p_in, g_in, b_in):
            lst[3] = lst[3][1:]
        if o.get("grad_scale"):
            g_in = [g / o["grad_scale"] for g in g_in]
        for i in range(len(ps)):
            mg = g_in[i].abs() + wd * p_in[i].abs()
            mb = (0.0 if o.get("first_step") else m) * b_in[i].abs() + mg
            mp = p_in[i].abs() + lr * (mb * (1 + m) if has_buf else mg)
            assert ((ps[i].float() - rp[i].float()).abs() <= 4 * step * mp + 1e-30).all(), f"param, opts {o}"
            if has_buf:
                assert ((bs[i].float() - rb[i].float()).abs() <= 4 * step * mb + 1e-30).all(), f"buffer, opts {o}"
            if scale is not None:
                assert ((gs[i].float() - rg[i].float()).abs() <= 2 * step * g_in[i].abs() + 1e-30).all()


def test_fused_sgd_skips_on_found_inf(cuda):
    ps, gs, bs = _inputs(cuda, torch.bfloat16, [1000, 33], seed=9)
    before = [p.clone() for p in ps]
    inf = torch.ones(1, device=cuda)
    arr = (_abi.SgdTensor * 2)(*[_abi.SgdTensor(p.data_ptr(), g.data_ptr(), b.data_ptr(), p.numel())
                                 for p, g, b in zip(ps, gs, bs)])
    hp = _abi.SgdHparams(0.1, 0.0, 0.9, 0.0, 0, 0, 0, _abi.B2_BF16, None, None, inf.data_ptr())
    _abi.check(_abi.lib().b2_fused_sgd(arr, 2, ctypes.byref(hp), _st()))
    torch.cuda.synchronize()
    for p, q in zip(ps, before):
        assert torch.equal(p, q)


def test_torch_optim_sgd_fused_runs_the_native_kernel(cuda):
    """torch.optim.SGD(fused=True) on xdna parameters -- a channels-last conv
    weight among them, as in a channels-last ResNet -- runs b2_fused_sgd with
    no fallback, and tracks ATen's CUDA kernel over three steps."""
    import xdna_train
    xdna_train.register_xdna_device()
    X = torch.device("xdna", 0)
    g = torch.Generator().manual_seed(0)
    init = [torch.randn(16, 8, 3, 3, generator=g).bfloat16().contiguous(memory_format=torch.channels_last),
            torch.randn(96, 64, generator=g).bfloat16(), torch.randn(96, generator=g).bfloat16()]
    params = [torch.nn.Parameter(t.to(X)) for t in init]
    assert params[0].is_contiguous(memory_format=torch.channels_last) and not params[0].is_contiguous()
    ref = [t.to(cuda) for t in init]
    opt = torch.optim.SGD(params, lr=0.1, momentum=0.9, weight_decay=1e-4, fused=True)
    bufs = None
    xdna_train.reset_mapped_cpu_stats()
    for step in range(3):
        grads = [torch.randn(t.shape, generator=g).bfloat16().contiguous(memory_format=torch.channels_last)
                 if t.dim() == 4 else torch.randn(t.shape, generator=g).bfloat16() for t in init]
        for q, gr in zip(params, grads):
            q.grad = gr.to(X)
        opt.step()
        gc = [gr.to(cuda) for gr in grads]
        if bufs is None:
            bufs = [torch.empty_like(r) for r in ref]
        torch._fused_sgd_(ref, gc, bufs, weight_decay=1e-4, momentum=0.9, lr=0.1, dampening=0.0, nesterov=False,
                          maximize=False, is_first_step=step == 0)
    for q, r in zip(params, ref):
        got = xdna_train.as_cuda(q.detach()).float()
        assert ((got - r.float()).abs() <= r.float().abs() * 2.0 ** -6 + 1e-6).all()
    assert xdna_train.kernel_stats().get("fused_sgd", 0) == 3
    assert "_fused_sgd_" not in xdna_train.fallback_stats()
