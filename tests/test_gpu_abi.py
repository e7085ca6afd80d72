"""Parity of libxdna_b200's sm_100a kernels, called through the C ABI, with
the CPU oracle (oracle/, pinned to the reference) and with an FP32 PyTorch
reference of the same op.

Tolerances: layouts and region kernels bit-exact; conv / GEMM
max|out - ref| <= 2e-2 * max|ref| and relative L2 error
<= 5e-3 (what fp32 accumulation + one bf16 rounding gives); Adam within 1e-6
(fp32) and bit-exact on bf16 parameters; fused BatchNorm + activation within
one bf16 ulp of the reference's host kernels, or within a small absolute floor
where cancellation leaves a near-zero result (their fp32 plane sums are added
in another order), and bit-equal on at least 99.5 % of the elements.
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from xdna_train import _abi

pytestmark = pytest.mark.gpu


def st():
    return torch.cuda.current_stream().cuda_stream


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def close(got: torch.Tensor, ref: torch.Tensor, tol=2e-2, l2=5e-3):
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert err <= tol * scale, f"max abs err {err} > {tol} * {scale}"
    assert rel <= l2, f"rel L2 {rel}"


def rows_of(x: torch.Tensor) -> torch.Tensor:
    B, Cc, H, W = x.shape
    chunks = -(-Cc // 64)
    rows = torch.empty(B * (H + 2) * (W + 2), chunks * 64, dtype=torch.bfloat16, device=x.device)
    s = x.stride()
    _abi.call("b2_pack_rows_bf16", x.data_ptr(), s[0], s[1], s[2], s[3], B, Cc, H, W, chunks, rows.data_ptr(),
              st())
    return rows


def wk_of(w: torch.Tensor, dgrad=False) -> torch.Tensor:
    Cout, Cin = w.shape[:2]
    kred = Cout if dgrad else Cin
    chunks = -(-kred // 64)
    wk = torch.empty((Cin if dgrad else Cout), chunks * 576, dtype=torch.bfloat16, device=w.device)
    name = "b2_pack_weight_dgrad_bf16" if dgrad else "b2_pack_weight_fwd_bf16"
    _abi.call(name, w.data_ptr(), Cout, Cin, chunks, wk.data_ptr(), st())
    return wk


# --------------------------------------------------------------------- packers

@pytest.mark.parametrize("shape", [(2, 70, 5, 7), (1, 3, 4, 4), (3, 64, 6, 9), (2, 130, 3, 11), (1, 64, 2, 150),
                                   (2, 64, 5, 36), (2, 96, 3, 18), (1, 70, 3, 264), (2, 128, 4, 72),
                                   # W % 8 == 0, W <= 256: the TMA packer (ragged channel chunks, one row,
                                   # W = 256, several work items per CTA)
                                   (2, 70, 5, 16), (3, 130, 4, 8), (2, 64, 1, 8), (1, 64, 3, 256),
                                   (8, 200, 40, 72)])
@pytest.mark.parametrize("channels_last", [False, True])
def test_pack_rows_bit_exact(cuda, shape, channels_last):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(*shape, generator=g).bfloat16()
    xd = x.to(cuda)
    if channels_last:
        xd = xd.contiguous(memory_format=torch.channels_last)
    got = bits(rows_of(xd))
    want = oracle.pack_rows(bits(x))
    assert np.array_equal(got, want)


@pytest.mark.parametrize("shape", [(4, 256, 9, 72), (2, 70, 5, 36), (3, 64, 6, 9), (2, 130, 7, 18), (2, 70, 5, 24),
                                   (6, 130, 30, 64)])
@pytest.mark.parametrize("channels_last", [False, True])
def test_pack_rows_dbias(cuda, shape, channels_last):
    """Packed rows bit-exact, plus dbias = sum over (b, y, x) (fixed-order fp32 sums)."""
    B, Cc, H, W = shape
    g = torch.Generator().manual_seed(3)
    x = torch.randn(*shape, generator=g).bfloat16()
    xd = x.to(cuda)
    if channels_last:
        xd = xd.contiguous(memory_format=torch.channels_last)
    ch = -(-Cc // 64)
    rows = torch.empty(B * (H + 2) * (W + 2), ch * 64, dtype=torch.bfloat16, device=cuda)
    ws_bytes = _abi.lib().b2_pack_rows_dbias_workspace_bytes(B, Cc, H, W)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
    db = torch.empty(Cc, dtype=torch.float32, device=cuda)
    db16 = torch.empty(Cc, dtype=torch.bfloat16, device=cuda)
    for out, dt in ((db, _abi.B2_F32), (db16, _abi.B2_BF16)):
        _abi.call("b2_pack_rows_dbias_bf16", xd.data_ptr(), *xd.stride(), B, Cc, H, W, ch, rows.data_ptr(),
                  out.data_ptr(), dt, ws.data_ptr(), ws_bytes, st())
    torch.cuda.synchronize()
    assert np.array_equal(bits(rows), oracle.pack_rows(bits(x)))
    ref = x.double().sum((0, 2, 3))
    assert (db.double().cpu() - ref).abs().max().item() <= 1e-4 * max(1.0, ref.abs().max().item())
    assert torch.equal(db16.cpu(), db.cpu().bfloat16())


@pytest.mark.parametrize("co_ci", [(128, 70), (100, 64), (3, 10), (256, 130)])
def test_pack_weights_bit_exact(cuda, co_ci):
    Cout, Cin = co_ci
    w = torch.randn(Cout, Cin, 3, 3).bfloat16()
    wd = w.to(cuda)
    assert np.array_equal(bits(wk_of(wd)), oracle.pack_weight(bits(w)))
    assert np.array_equal(bits(wk_of(wd, dgrad=True)), oracle.pack_weight(bits(w), dgrad=True))


@pytest.mark.parametrize("co_ci", [(128, 70), (64, 64), (3, 10), (256, 130)])
def test_pack_weights_strided_bit_exact(cuda, co_ci):
    """Packing read through the weight's strides: a channels-last (OHWI)
    weight and a transposed view give the oracle's packed forms."""
    import ctypes
    Cout, Cin = co_ci
    w = torch.randn(Cout, Cin, 3, 3).bfloat16()
    views = [w.to(cuda).contiguous(memory_format=torch.channels_last),
             w.transpose(2, 3).contiguous().to(cuda).transpose(2, 3)]
    for wd in views:
        assert wd.shape == w.shape and not wd.is_contiguous()
        for dgrad in (0, 1):
            chunks = -(-(Cout if dgrad else Cin) // 64)
            wk = torch.empty((Cin if dgrad else Cout), chunks * 576, dtype=torch.bfloat16, device=cuda)
            strides = (ctypes.c_int64 * 4)(*wd.stride())
            _abi.call("b2_pack_weight_strided_bf16", wd.data_ptr(), strides, Cout, Cin, chunks, dgrad,
                      wk.data_ptr(), st())
            assert np.array_equal(bits(wk), oracle.pack_weight(bits(w), dgrad=bool(dgrad)))


def test_nchw_nhwc_roundtrip_bit_exact(cuda):
    x = torch.randn(3, 70, 9, 13, device=cuda).bfloat16()
    y = torch.empty(3, 9 * 13, 70, dtype=torch.bfloat16, device=cuda)
    _abi.call("b2_nchw_to_nhwc_bf16", x.data_ptr(), y.data_ptr(), 3, 70, 117, st())
    assert torch.equal(y.view(3, 9, 13, 70).permute(0, 3, 1, 2), x)
    z = torch.empty_like(x)
    _abi.call("b2_nhwc_to_nchw_bf16", y.data_ptr(), z.data_ptr(), 3, 70, 117, st())
    assert torch.equal(z, x)


# ------------------------------------------------------------------------ conv

SMALL = [  # B, Cin, H, W, Cout, bias  (oracle-checked)
    (2, 64, 8, 8, 64, True),
    (3, 3, 5, 7, 10, True),
    (2, 70, 12, 37, 70, False),
    (1, 130, 6, 6, 200, True),
]
LARGE = [  # the reference's run_conv3x3w_torch.py shapes (:22-35) and the README conv
    (40, 256, 36, 36, 128, False),
    (40, 64, 36, 36, 64, True),
    (4, 195, 36, 36, 70, False),
    (40, 128, 9, 9, 128, False),
    (40, 256, 18, 18, 256, False),
    (2, 128, 14, 112, 128, False),
    (1, 64, 8, 224, 64, False),
    (16, 128, 36, 36, 128, True),
    (8, 512, 18, 18, 512, False),
    # wide convolutions on the halo kernel: windows of one and two TMA boxes,
    # the largest window that fits, and one too wide for it (the plain pair kernel)
    (2, 256, 10, 72, 256, True),
    (1, 192, 4, 150, 320, False),
    (1, 256, 3, 200, 256, False),
    # narrow layers with enough padded rows for the all-taps weight-gradient
    # kernel: a three-box input window (W = 224) with 3 -> 10 channels, and odd
    # channel counts below one 64-channel chunk
    (8, 3, 40, 224, 10, True),
    (16, 37, 40, 40, 45, False),
]


def _conv_inputs(cuda, B, Cin, H, W, Cout, bias, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, Cin, H, W, generator=g).bfloat16()
    w = ((torch.rand(Cout, Cin, 3, 3, generator=g) * 2 - 1) * (1.0 / (9 * Cin)) ** 0.5).bfloat16()
    b = torch.randn(Cout, generator=g).bfloat16() if bias else None
    dy = torch.randn(B, Cout, H, W, generator=g).bfloat16()
    return x, w, b, dy


def _gpu_conv(cuda, x, w, b, dy, out_channels_last=False):
    B, Cin, H, W = x.shape
    Cout = w.shape[0]
    xd, wd, dyd = x.to(cuda), w.to(cuda), dy.to(cuda)
    bd = b.to(cuda) if b is not None else None
    xr, dyr = rows_of(xd), rows_of(dyd)
    mf = torch.channels_last if out_channels_last else torch.contiguous_format
    y = torch.empty(B, Cout, H, W, dtype=torch.bfloat16, device=cuda, memory_format=mf)
    s = y.stride()
    _abi.call("b2_conv3x3_fwd", xr.data_ptr(), wk_of(wd).data_ptr(), 0 if bd is None else bd.data_ptr(),
              y.data_ptr(), s[0], s[1], s[2], s[3], B, Cin, H, W, Cout, 0, st())
    dx = torch.empty(B, Cin, H, W, dtype=torch.bfloat16, device=cuda, memory_format=mf)
    s = dx.stride()
    _abi.call("b2_conv3x3_dgrad", dyr.data_ptr(), wk_of(wd, dgrad=True).data_ptr(), dx.data_ptr(), s[0], s[1],
              s[2], s[3], B, Cout, H, W, Cin, st())
    ws_bytes = _abi.lib().b2_conv3x3_wgrad_workspace_bytes(B, Cin, H, W, Cout)
    ws = torch.empty(ws_bytes // 4 + 4, dtype=torch.float32, device=cuda)
    dw = torch.empty(Cout, Cin, 3, 3, dtype=torch.float32, device=cuda)
    _abi.call("b2_conv3x3_wgrad", dyr.data_ptr(), xr.data_ptr(), dw.data_ptr(), _abi.B2_F32, B, Cin, H, W, Cout,
              ws.data_ptr(), ws.numel() * 4, st())
    torch.cuda.synchronize()
    return y, dx, dw


@pytest.mark.parametrize("shape", SMALL)
def test_conv_vs_oracle(cuda, shape):
    x, w, b, dy = _conv_inputs(cuda, *shape)
    y, dx, dw = _gpu_conv(cuda, x, w, b, dy)
    close(y, torch.from_numpy(oracle.conv_fwd(bits(x), bits(w), None if b is None else bits(b))))
    close(dx, torch.from_numpy(oracle.conv_dgrad(bits(dy), bits(w))))
    close(dw, torch.from_numpy(oracle.conv_wgrad(bits(dy), bits(x))))


@pytest.mark.parametrize("shape", LARGE)
def test_conv_vs_fp32_reference(cuda, shape):
    x, w, b, dy = _conv_inputs(cuda, *shape, seed=1)
    y, dx, dw = _gpu_conv(cuda, x, w, b, dy, out_channels_last=(shape[0] % 2 == 0))
    xf, wf, dyf = x.float().to(cuda), w.float().to(cuda), dy.float().to(cuda)
    bf = b.float().to(cuda) if b is not None else None
    with torch.no_grad():
        torch.backends.cudnn.allow_tf32 = False
        y_ref = torch.nn.functional.conv2d(xf, wf, bf, padding=1)
        dx_ref, dw_ref, _ = torch.ops.aten.convolution_backward(dyf, xf, wf, None, [1, 1], [1, 1], [1, 1], False,
                                                                [0, 0], 1, [True, True, False])
    close(y, y_ref)
    close(dx, dx_ref)
    close(dw, dw_ref)


def test_conv_relu_epilogue_and_bf16_wgrad(cuda):
    x, w, b, dy = _conv_inputs(cuda, 2, 64, 9, 9, 96, True, seed=3)
    xd, wd, bd = x.to(cuda), w.to(cuda), b.to(cuda)
    y = torch.empty(2, 96, 9, 9, dtype=torch.bfloat16, device=cuda)
    xr0, wk0 = rows_of(xd), wk_of(wd)  # keep the operands alive until the kernel ran
    _abi.call("b2_conv3x3_fwd", xr0.data_ptr(), wk0.data_ptr(), bd.data_ptr(), y.data_ptr(),
              *y.stride(), 2, 64, 9, 9, 96, 1, st())
    ref = torch.from_numpy(oracle.conv_fwd(bits(x), bits(w), bits(b), relu=True))
    close(y, ref)
    assert (y >= 0).all()
    # bf16 dW output = fp32 result rounded once
    dyd = dy.to(cuda)
    ws_bytes = _abi.lib().b2_conv3x3_wgrad_workspace_bytes(2, 64, 9, 9, 96)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
    dw32 = torch.empty(96, 64, 3, 3, dtype=torch.float32, device=cuda)
    dw16 = torch.empty(96, 64, 3, 3, dtype=torch.bfloat16, device=cuda)
    xr, dyr = rows_of(xd), rows_of(dyd)
    for out, dt in ((dw32, _abi.B2_F32), (dw16, _abi.B2_BF16)):
        _abi.call("b2_conv3x3_wgrad", dyr.data_ptr(), xr.data_ptr(), out.data_ptr(), dt, 2, 64, 9, 9, 96,
                  ws.data_ptr(), ws_bytes, st())
    assert torch.equal(dw16, dw32.bfloat16())


def test_wgrad_rejects_small_workspace(cuda):
    ws = torch.empty(16, dtype=torch.uint8, device=cuda)
    t = torch.empty(1 << 16, dtype=torch.bfloat16, device=cuda)
    st_ = _abi.lib().b2_conv3x3_wgrad(t.data_ptr(), t.data_ptr(), t.data_ptr(), 0, 1, 64, 8, 8, 64, ws.data_ptr(),
                                      16, st())
    assert st_ == 5


def test_device_status_clean(cuda):
    code = ctypes.c_int(-1)
    _abi.check(_abi.lib().b2_device_status(0, ctypes.byref(code)))
    assert code.value == 0


# ------------------------------------------------------------------------ GEMM

@pytest.mark.parametrize("ta", [0, 1])
@pytest.mark.parametrize("tb", [0, 1])
@pytest.mark.parametrize("mnk", [(512, 1024, 4096), (300, 200, 136), (64, 520, 72), (1, 256, 64)])
def test_gemm_transposes(cuda, ta, tb, mnk):
    M, N, K = mnk
    g = torch.Generator().manual_seed(M + N + K)
    A = torch.randn(M, K, generator=g).bfloat16()
    Bm = torch.randn(K, N, generator=g).bfloat16()
    a_store = (A.t().contiguous() if ta else A).to(cuda)
    b_store = (Bm.t().contiguous() if tb else Bm).to(cuda)
    lda, ldb = a_store.shape[1], b_store.shape[1]
    if lda % 8 or ldb % 8:
        pytest.skip("TMA needs 16-byte aligned rows")
    D = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    _abi.call("b2_gemm_bf16", ta, tb, M, N, K, 1.0, a_store.data_ptr(), lda, 0, b_store.data_ptr(), ldb, 0, 0.0,
              None, _abi.B2_BF16, 0, 0, 0, D.data_ptr(), N, 0, 1, st())
    torch.cuda.synchronize()
    close(D, A.float() @ Bm.float())


def test_gemm_batched_bias_alpha_beta(cuda):
    g = torch.Generator().manual_seed(7)
    bt, M, N, K = 3, 200, 136, 256
    A = torch.randn(bt, M, K, generator=g).bfloat16()
    Bm = torch.randn(bt, N, K, generator=g).bfloat16()  # transB storage
    bias = torch.randn(N, generator=g).bfloat16()
    Ad, Bd, biasd = A.to(cuda), Bm.to(cuda), bias.to(cuda)
    D = torch.empty(bt, M, N, dtype=torch.bfloat16, device=cuda)
    _abi.call("b2_gemm_bf16", 0, 1, M, N, K, 0.5, Ad.data_ptr(), K, M * K, Bd.data_ptr(), K, N * K, 2.0,
              biasd.data_ptr(), _abi.B2_BF16, 0, 1, 0, D.data_ptr(), N, M * N, bt, st())
    torch.cuda.synchronize()
    ref = 0.5 * torch.bmm(A.float(), Bm.float().transpose(1, 2)) + 2.0 * bias.float()
    close(D, ref)
    # and against the oracle for one batch entry
    o = oracle.gemm(bits(A[1]), bits(Bm[1].t().contiguous()), np.broadcast_to(bias.float().numpy(), (M, N)),
                    alpha=0.5, beta=2.0)
    close(D[1], torch.from_numpy(o))


@pytest.mark.parametrize("mnk", [(512, 1024, 4096), (512, 4096, 4096), (300, 200, 1024)])
def test_gemm_split_k_with_workspace(cuda, mnk):
    """b2_gemm_bf16_ws: split-K where the output has too few tiles for the SMs,
    alpha and a broadcast bias (beta * C) applied by the ordered reduction;
    within the GEMM bound of the unsplit kernel against fp32."""
    M, N, K = mnk
    g = torch.Generator().manual_seed(M * 7 + N)
    A = torch.randn(M, K, generator=g).bfloat16()
    Bt = torch.randn(N, K, generator=g).bfloat16()  # transB storage, as nn.Linear's weight
    bias = torch.randn(N, generator=g).bfloat16()
    Ad, Bd, bd = A.to(cuda), Bt.to(cuda), bias.to(cuda)
    L = _abi.lib()
    wsb = L.b2_gemm_bf16_workspace_bytes(M, N, K, 1)
    if mnk[:2] == (512, 1024):
        assert wsb > 0  # 32 output tiles of 148 SMs: split
    ws = torch.empty(max(16, wsb), dtype=torch.uint8, device=cuda)
    D = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    D0 = torch.empty_like(D)
    for out, w, wb in ((D, ws.data_ptr(), wsb), (D0, None, 0)):
        _abi.call("b2_gemm_bf16_ws", 0, 1, M, N, K, 0.5, Ad.data_ptr(), K, 0, Bd.data_ptr(), K, 0, 1.0, bd.data_ptr(),
                  _abi.B2_BF16, 0, 1, 0, out.data_ptr(), N, 0, 1, w, wb, st())
    torch.cuda.synchronize()
    ref = 0.5 * (A.float() @ Bt.float().t()) + bias.float()
    close(D, ref)
    close(D0, ref)


def test_gemm_sm_pair_tiles_in_a_subprocess(cuda):
    """The SM-pair GEMM tiles (B2_GEMM_PAIR=1, read once per process): every
    transpose combination, 256- and 128-wide pair tiles, a bias epilogue and
    split-K partials, against fp32 -- run in a child process with the switch
    set."""
    import os
    import subprocess
    import sys
    code = r'''
import sys, torch
sys.path[:0] = [sys.argv[1], sys.argv[2]]
from xdna_train import _abi
d = torch.device("cuda", 0)
st = torch.cuda.current_stream().cuda_stream
L = _abi.lib()
for (M, N, K) in [(512, 4096, 1024), (1024, 2048, 512), (2048, 4096, 256), (512, 1024, 4096)]:
    for ta in (0, 1):
        for tb in (0, 1):
            g = torch.Generator().manual_seed(M + N + K + 2 * ta + tb)
            A = torch.randn(M, K, generator=g).bfloat16(); Bm = torch.randn(K, N, generator=g).bfloat16()
            bias = torch.randn(N, generator=g).bfloat16()
            a = (A.t().contiguous() if ta else A).to(d); b = (Bm.t().contiguous() if tb else Bm).to(d)
            D = torch.empty(M, N, dtype=torch.bfloat16, device=d)
            wsb = L.b2_gemm_bf16_workspace_bytes(M, N, K, 1)
            ws = torch.empty(max(16, wsb), dtype=torch.uint8, device=d)
            _abi.call("b2_gemm_bf16_ws", ta, tb, M, N, K, 1.0, a.data_ptr(), a.shape[1], 0, b.data_ptr(), b.shape[1],
                      0, 1.0, bias.to(d).data_ptr(), _abi.B2_BF16, 0, 1, 0, D.data_ptr(), N, 0, 1, ws.data_ptr(),
                      wsb, st)
            torch.cuda.synchronize()
            ref = A.float() @ Bm.float() + bias.float()
            err = (D.float().cpu() - ref).abs().max().item()
            assert err <= 2e-2 * ref.abs().max().item(), (M, N, K, ta, tb, err)
print("ok")
'''
    repo = Path(__file__).resolve().parent.parent
    env = dict(os.environ, B2_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-c", code, str(repo / "pytorch-xdna2_b200"), str(repo)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


# ------------------------------------------------------------------------ Adam

@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("adamw,amsgrad,wd", [(False, False, 0.0), (True, False, 0.01), (False, True, 0.1)])
def test_fused_adam_matches_cpu(cuda, dtype, adamw, amsgrad, wd):
    g = torch.Generator().manual_seed(5)
    sizes = [1, 7, 4096, 70001, 3 * 16384 + 5]
    ps = [torch.randn(n, generator=g).to(dtype) for n in sizes]
    gs = [torch.randn(n, generator=g).to(dtype) for n in sizes]
    ms = [(torch.randn(n, generator=g) * 0.1).to(dtype) for n in sizes]
    vs = [(torch.rand(n, generator=g) * 0.1).to(dtype) for n in sizes]
    xs = [(torch.rand(n, generator=g) * 0.1).to(dtype) for n in sizes] if amsgrad else []
    steps = [torch.tensor(float(i + 2)) for i in range(len(sizes))]
    dev = lambda L: [t.to(cuda) for t in L]  # noqa: E731
    P, G, M, V, X, S = dev(ps), dev(gs), dev(ms), dev(vs), dev(xs), dev(steps)
    fn = torch._fused_adamw_ if adamw else torch._fused_adam_
    fn(ps, gs, ms, vs, xs, steps, lr=1e-2, beta1=0.9, beta2=0.99, weight_decay=wd, eps=1e-8, amsgrad=amsgrad,
       maximize=False)
    arr = (_abi.AdamTensor * len(sizes))()
    for i, n in enumerate(sizes):
        arr[i] = _abi.AdamTensor(P[i].data_ptr(), G[i].data_ptr(), M[i].data_ptr(), V[i].data_ptr(),
                                 X[i].data_ptr() if amsgrad else None, S[i].data_ptr(), n)
    code = _abi.B2_F32 if dtype == torch.float32 else _abi.B2_BF16
    hp = _abi.AdamHparams(1e-2, 0.9, 0.99, wd, 1e-8, int(amsgrad), 0, int(adamw), code, code, None, None, None)
    _abi.check(_abi.lib().b2_fused_adam(arr, len(sizes), ctypes.byref(hp), st()))
    torch.cuda.synchronize()
    for got, ref in zip(P + M + V, ps + ms + vs):
        got = got.cpu().float()
        ref = ref.float()
        if dtype == torch.float32:
            assert (got - ref).abs().max().item() <= 1e-6 * max(1.0, ref.abs().max().item())
        else:  # bit-exact with torch's CPU fused Adam
            assert torch.equal(got, ref)


# --------------------------------------------------------------------- regions

@pytest.fixture(scope="module")
def reg():
    from pathlib import Path
    return np.load(Path(__file__).resolve().parent / "golden" / "regions.npz")


def _dev(a: np.ndarray, cuda):
    return torch.from_numpy(a.view(np.int16).copy()).to(cuda).view(torch.bfloat16)


@pytest.mark.parametrize("tag", ["even", "odd"])
def test_regions_bit_exact_vs_reference(cuda, reg, tag):
    a, b, base = (_dev(reg[f"{tag}_{k}"], cuda) for k in ("a", "b", "base"))
    shape = reg[f"{tag}_a"].shape
    planes, H, W = shape[0] * shape[1], shape[2], shape[3]
    n = a.numel()
    out = torch.empty_like(a)
    _abi.call("b2_region_relu_bf16", a.data_ptr(), out.data_ptr(), n, st())
    assert np.array_equal(bits(out), reg[f"{tag}_relu"])
    r = torch.empty_like(a)
    p = torch.empty(shape[0], shape[1], H // 2, W // 2, dtype=torch.bfloat16, device=cuda)
    _abi.call("b2_region_relu_maxpool2_bf16", a.data_ptr(), r.data_ptr(), p.data_ptr(), planes, H, W, st())
    assert np.array_equal(bits(r), reg[f"{tag}_relu_r"])
    assert np.array_equal(bits(p), reg[f"{tag}_pool"])
    _abi.call("b2_region_addtap_bf16", base.data_ptr(), a.data_ptr(), b.data_ptr(), out.data_ptr(), n,
              ctypes.c_float(0.37), st())
    assert np.array_equal(bits(out), reg[f"{tag}_addtap"])
    _abi.call("b2_region_addtap_bf16", None, a.data_ptr(), b.data_ptr(), out.data_ptr(), n, ctypes.c_float(-1.5),
              st())
    assert np.array_equal(bits(out), reg[f"{tag}_addtap_nobase"])
    rr = _dev(reg[f"{tag}_relu"], cuda)
    _abi.call("b2_region_relu_bwd_bf16", rr.data_ptr(), base.data_ptr(), a.data_ptr(), b.data_ptr(), out.data_ptr(),
              n, ctypes.c_float(0.25), st())
    assert np.array_equal(bits(out), reg[f"{tag}_relu_bwd"])
    _abi.call("b2_region_relu_bwd_bf16", rr.data_ptr(), base.data_ptr(), None, None, out.data_ptr(), n,
              ctypes.c_float(0.25), st())
    assert np.array_equal(bits(out), reg[f"{tag}_relu_bwd_notap"])
    gg = _dev(reg[f"{tag}_g"], cuda)
    _abi.call("b2_region_maxpool2_bwd_bf16", a.data_ptr(), gg.data_ptr(), out.data_ptr(), planes, H, W, st())
    assert np.array_equal(bits(out), reg[f"{tag}_maxpool_bwd"])
    fa, fb = _dev(reg[f"{tag}_fin_a"], cuda), _dev(reg[f"{tag}_fin_b"], cuda)
    acc = torch.zeros(1, dtype=torch.float64, device=cuda)
    _abi.call("b2_region_sqdiff_sum_bf16", fa.data_ptr(), fb.data_ptr(), n, acc.data_ptr(), st())
    want = reg[f"{tag}_sqdiff"][0]
    assert abs(acc.item() - want) <= 1e-5 * abs(want)


def test_regions_large_sqdiff(cuda):
    g = torch.Generator().manual_seed(11)
    a = torch.randn(40, 256, 18, 18, generator=g).bfloat16()
    b = torch.randn(40, 256, 18, 18, generator=g).bfloat16()
    acc = torch.zeros(1, dtype=torch.float64, device=cuda)
    ad, bd = a.to(cuda), b.to(cuda)
    _abi.call("b2_region_sqdiff_sum_bf16", ad.data_ptr(), bd.data_ptr(), a.numel(), acc.data_ptr(), st())
    want = oracle.sqdiff_sum(bits(a), bits(b))
    assert abs(acc.item() - want) <= 1e-5 * want


def test_single_cta_conv_path_still_matches(cuda):
    """Wide convolutions run the SM-pair kernel by default; B2_PAIR_MMA=0 keeps
    the single-CTA kernel.  Check that one too, in a fresh process."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    code = (
        "import sys; sys.path[:0] = [%r, %r]\n"
        "import torch\n"
        "from tests.test_gpu_abi import _conv_inputs, _gpu_conv, close\n"
        "x, w, b, dy = _conv_inputs(None, 4, 256, 18, 18, 320, True, seed=9)\n"
        "y, dx, dw = _gpu_conv(torch.device('cuda', 0), x, w, b, dy)\n"
        "with torch.no_grad():\n"
        "    xf, wf, dyf = x.float(), w.float(), dy.float()\n"
        "    y_ref = torch.nn.functional.conv2d(xf, wf, b.float(), padding=1)\n"
        "    dx_ref, dw_ref, _ = torch.ops.aten.convolution_backward(dyf, xf, wf, None, [1, 1], [1, 1], [1, 1],"
        " False, [0, 0], 1, [True, True, False])\n"
        "close(y, y_ref); close(dx, dx_ref); close(dw, dw_ref)\n"
        "print('ok')\n" % (str(root), str(root / "pytorch-xdna2_b200")))
    env = dict(os.environ, B2_PAIR_MMA="0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


# ---- fused BatchNorm + activation (region_kernels.cpp:309-460) ----------------

def _ulps(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return np.abs(a.astype(np.int32) - b.astype(np.int32))


def _bf_close(got: np.ndarray, want: np.ndarray, floor: float, exact: float = 0.995):
    """bf16 bit arrays that agree to one bf16 ulp, or to `floor` absolutely
    where the value is the small difference of larger terms (cancellation makes
    ulps of a near-zero result meaningless), with at least `exact` of the
    elements bit-equal."""
    g, w = oracle.bf16_value(got), oracle.bf16_value(want)
    err = np.abs(g - w)
    bound = np.abs(w) * 2.0 ** -7 + floor
    assert (err <= bound).all(), f"max excess {(err - bound).max()} (floor {floor})"
    assert (got == want).mean() >= exact, f"only {(got == want).mean():.5f} bit-equal"


def _gpu_bn(cuda, x, w, b, rm, rv, slope, relu, dy, ybwd=None, need=(True, True, True), update=True):
    """Runs b2_region_bn_fwd_bf16 / _bwd_bf16 on bf16-bit numpy inputs."""
    N, Cc = x.shape[:2]
    HW = int(np.prod(x.shape[2:]))
    dv = lambda a: None if a is None else _dev(a, cuda)  # noqa: E731
    xd, wd, bd, rmd, rvd, dyd = dv(x), dv(w), dv(b), dv(rm), dv(rv), dv(dy)
    y = torch.empty_like(xd)
    mean = torch.empty(Cc, dtype=torch.float32, device=cuda)
    invstd = torch.empty_like(mean)
    nws = _abi.lib().b2_region_bn_workspace_bytes(N, Cc)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda)
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _abi.call("b2_region_bn_fwd_bf16", xd.data_ptr(), p(wd), p(bd), p(rmd), p(rvd), y.data_ptr(), mean.data_ptr(),
              invstd.data_ptr(), N, Cc, HW, ctypes.c_float(1e-5), ctypes.c_float(slope), ctypes.c_float(0.1),
              int(update), ws.data_ptr(), nws, st())
    yb = y if ybwd is None else dv(ybwd)
    dx = torch.empty_like(xd) if need[0] else None
    dw = torch.empty(Cc, dtype=torch.bfloat16, device=cuda) if need[1] else None
    db = torch.empty(Cc, dtype=torch.bfloat16, device=cuda) if need[2] else None
    _abi.call("b2_region_bn_bwd_bf16", dyd.data_ptr(), yb.data_ptr(), xd.data_ptr(), p(wd), mean.data_ptr(),
              invstd.data_ptr(), p(dx), p(dw), p(db), N, Cc, HW, ctypes.c_float(slope), int(relu), ws.data_ptr(),
              nws, st())
    torch.cuda.synchronize()
    out = lambda t: None if t is None else bits(t)  # noqa: E731
    return (bits(y), mean.cpu().numpy(), invstd.cpu().numpy(), out(rmd), out(rvd), out(dx), out(dw), out(db))


@pytest.fixture(scope="module")
def bn_gold():
    return np.load(Path(__file__).resolve().parent / "golden" / "regions_bn.npz")


def test_bn_act_vs_reference_vectors(cuda, bn_gold):
    """Against the reference's own host kernels' outputs: the fp32 plane sums
    are ordered differently, so a value on a bf16 rounding boundary may land one
    ulp apart (or, for a near-zero difference of larger terms, a small absolute
    amount); nearly every element is bit-equal."""
    g = bn_gold
    for i in range(int(g["cases"][0])):
        N, Cc, H, W, relu, affine = (int(v) for v in g[f"c{i}_meta"])
        slope = float(g[f"c{i}_slope"][0])
        w = g[f"c{i}_w"] if affine else None
        b = g[f"c{i}_b"] if affine else None
        y, mean, invstd, rm, rv, dx, dw, db = _gpu_bn(cuda, g[f"c{i}_x"], w, b, g[f"c{i}_rm"], g[f"c{i}_rv"],
                                                      slope, relu, g[f"c{i}_dy"])
        M = N * H * W
        _bf_close(y, g[f"c{i}_y"], 1e-5 * np.abs(oracle.bf16_value(g[f"c{i}_y"])).max())
        np.testing.assert_allclose(mean, g[f"c{i}_mean"], rtol=0, atol=1e-6 * max(1.0, np.abs(mean).max()))
        np.testing.assert_allclose(invstd, g[f"c{i}_invstd"], rtol=1e-6)
        assert _ulps(rm, g[f"c{i}_rm_out"]).max() <= 1 and _ulps(rv, g[f"c{i}_rv_out"]).max() <= 1
        # backward on the reference's activation with planted 0 / NaN (the dz rule)
        *_, dx, dw, db = _gpu_bn(cuda, g[f"c{i}_x"], w, b, g[f"c{i}_rm"], g[f"c{i}_rv"], slope, relu,
                                 g[f"c{i}_dy"], ybwd=g[f"c{i}_ybwd"])
        _bf_close(dx, g[f"c{i}_dx"], 1e-5 * np.abs(oracle.bf16_value(g[f"c{i}_dx"])).max())
        _bf_close(dw, g[f"c{i}_dw"], 2e-6 * M, exact=0.9)
        _bf_close(db, g[f"c{i}_db"], 2e-6 * M, exact=0.9)


# warp-per-plane (>= 32 planes per SM) and block-per-plane paths, 16-byte
# vector and scalar (HW % 8 != 0) paths, N = 1, C = 1, no affine, no update
@pytest.mark.parametrize("shape,slope,relu,affine", [
    ((40, 128, 9, 9), 0.2, 0, True),      # 5120 planes, scalar
    ((64, 96, 16, 16), 0.0, 1, True),     # 6144 planes, vector
    ((2, 64, 56, 56), 0.0, 1, True),      # block per plane, vector
    ((3, 5, 7, 9), 0.2, 0, True),         # block per plane, scalar
    ((1, 32, 20, 20), 0.01, 0, False),    # N = 1, affine=False
    ((16, 1, 12, 12), 0.0, 1, True),      # C = 1
])
def test_bn_act_vs_oracle(cuda, shape, slope, relu, affine):
    rng = np.random.default_rng(sum(shape))
    N, Cc = shape[:2]
    x = oracle.bf16_bits((rng.standard_normal(shape) * 1.5 + 0.3).astype(np.float32))
    w = oracle.bf16_bits(rng.uniform(0.5, 1.5, Cc).astype(np.float32)) if affine else None
    b = oracle.bf16_bits((rng.standard_normal(Cc) * 0.3).astype(np.float32)) if affine else None
    rm = oracle.bf16_bits((rng.standard_normal(Cc) * 0.1).astype(np.float32))
    rv = oracle.bf16_bits(rng.uniform(0.5, 1.5, Cc).astype(np.float32))
    dy = oracle.bf16_bits(rng.standard_normal(shape).astype(np.float32))
    y, mean, invstd, rm2, rv2, dx, dw, db = _gpu_bn(cuda, x, w, b, rm, rv, slope, relu, dy)
    oy, omean, oinv, orm, orv = oracle.bn_fwd(x, w, b, rm, rv, 1e-5, slope, 0.1, True)
    np.testing.assert_allclose(mean, omean, rtol=0, atol=1e-6 * max(1.0, np.abs(omean).max()))
    np.testing.assert_allclose(invstd, oinv, rtol=1e-6)
    M = int(np.prod(shape)) // Cc
    _bf_close(y, oy, 1e-5 * np.abs(oracle.bf16_value(oy)).max())
    assert _ulps(rm2, orm).max() <= 1 and _ulps(rv2, orv).max() <= 1
    # backward from the GPU's own statistics, so only the backward is compared
    odx, odw, odb = oracle.bn_bwd(dy, y, x, w, mean, invstd, slope, bool(relu))
    _bf_close(dx, odx, 1e-5 * np.abs(oracle.bf16_value(odx)).max())
    _bf_close(dw, odw, 2e-6 * M, exact=0.9)
    _bf_close(db, odb, 2e-6 * M, exact=0.9)
    # only some gradients requested; no running-statistics update
    y3, _, _, rm3, rv3, dx3, dw3, db3 = _gpu_bn(cuda, x, w, b, rm, rv, slope, relu, dy, need=(False, True, False),
                                                update=False)
    assert np.array_equal(y3, y) and np.array_equal(rm3, rm) and np.array_equal(rv3, rv)
    assert dx3 is None and db3 is None and np.array_equal(dw3, dw)


def test_bn_act_rejects_small_workspace(cuda):
    t = torch.zeros(64, dtype=torch.float32, device=cuda)
    rc = _abi.lib().b2_region_bn_fwd_bf16(t.data_ptr(), None, None, None, None, t.data_ptr(), t.data_ptr(),
                                          t.data_ptr(), 2, 4, 8, ctypes.c_float(1e-5), ctypes.c_float(0.0),
                                          ctypes.c_float(0.1), 0, t.data_ptr(), 8, st())
    assert rc == 5 and b"workspace" in _abi.lib().b2_last_error()
