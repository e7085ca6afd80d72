"""The allocation-free weight gradient, b2_conv3x3_wgrad_noalloc.

Some callers of this library cannot hand it a workspace: a host framework that
reserved all device memory for its own pool up front, or a latency-critical
loop that must never reach cudaMalloc (which can synchronize the device).  For
them the library keeps wgrad's split-K partial sums in one fixed device array
(b2_conv3x3_wgrad_noalloc_max_bytes(), 16 MiB) instead of a caller workspace.

This file is collected last on purpose.  It calls the entry point through the
C ABI several times in a row -- each call reuses the array the previous one
left behind -- and checks every result against b2_conv3x3_wgrad with a
caller-provided workspace, within the conv tolerance of the other GPU tests.
It also checks that a shape whose partial sums cannot fit is refused with a
clear error instead of running.
"""
import ctypes

import pytest
import torch

from xdna_train import _abi

pytestmark = pytest.mark.gpu


def _st():
    return torch.cuda.current_stream().cuda_stream


def _rows(x):
    B, C, H, W = x.shape
    ch = -(-C // 64)
    rows = torch.empty(B * (H + 2) * (W + 2), ch * 64, dtype=torch.bfloat16, device=x.device)
    _abi.call("b2_pack_rows_bf16", x.data_ptr(), *x.stride(), B, C, H, W, ch, rows.data_ptr(), _st())
    return rows


def _close(got, ref, tol=2e-2, l2=5e-3):
    got, ref = got.float().cpu(), ref.float().cpu()
    scale = ref.abs().max().item()
    assert (got - ref).abs().max().item() <= tol * scale
    assert ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item() <= l2


# (B, Cin, H, W, Cout).  The usual split-K plan of the fourth shape (2048 padded
# rows = 32 k-blocks, 72 tiles of 148 SMs -> 2 splits) needs 2 * 9 * 512 * 512 *
# 4 B = 18.9 MB of partial sums, more than the 16 MiB array: the call cuts it to
# one split.  The others keep the usual plan (one split each for the first
# three, which all fit).
SHAPES = [(4, 128, 18, 18, 128), (1, 512, 8, 8, 512), (2, 64, 9, 13, 96), (8, 512, 14, 14, 512)]


def test_noalloc_wgrad_matches_workspace_entry_point_on_consecutive_calls(cuda):
    L = _abi.lib()
    assert L.b2_conv3x3_wgrad_noalloc_max_bytes() == 16 << 20
    g = torch.Generator().manual_seed(7)
    for B, Cin, H, W, Cout in SHAPES:
        x = torch.randn(B, Cin, H, W, generator=g).bfloat16().to(cuda)
        dy = torch.randn(B, Cout, H, W, generator=g).bfloat16().to(cuda)
        xr, dyr = _rows(x), _rows(dy)
        ws_bytes = L.b2_conv3x3_wgrad_workspace_bytes(B, Cin, H, W, Cout)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
        ref = torch.empty(Cout, Cin, 3, 3, dtype=torch.float32, device=cuda)
        _abi.call("b2_conv3x3_wgrad", dyr.data_ptr(), xr.data_ptr(), ref.data_ptr(), _abi.B2_F32, B, Cin, H, W, Cout,
                  ws.data_ptr(), ws_bytes, _st())
        got = torch.full((Cout, Cin, 3, 3), float("nan"), dtype=torch.float32, device=cuda)
        _abi.call("b2_conv3x3_wgrad_noalloc", dyr.data_ptr(), xr.data_ptr(), got.data_ptr(), _abi.B2_F32, B, Cin, H,
                  W, Cout, _st())
        got16 = torch.empty(Cout, Cin, 3, 3, dtype=torch.bfloat16, device=cuda)
        _abi.call("b2_conv3x3_wgrad_noalloc", dyr.data_ptr(), xr.data_ptr(), got16.data_ptr(), _abi.B2_BF16, B, Cin,
                  H, W, Cout, _st())
        torch.cuda.synchronize()
        _close(got, ref)
        _close(got16, ref)
    code = ctypes.c_int(-1)
    _abi.check(L.b2_device_status(torch.cuda.current_device(), ctypes.byref(code)))
    assert code.value == 0


def test_noalloc_wgrad_refuses_what_does_not_fit(cuda):
    L = _abi.lib()
    t = torch.empty(1 << 12, dtype=torch.bfloat16, device=cuda)
    # 9 * 1024 * 1024 fp32 partial sums are 37.7 MB, beyond the 16 MiB array
    st = L.b2_conv3x3_wgrad_noalloc(t.data_ptr(), t.data_ptr(), t.data_ptr(), _abi.B2_F32, 1, 1024, 4, 4, 1024,
                                    _st())
    assert st == 5  # B2_ERR_WORKSPACE
    assert b"scratch" in L.b2_last_error()
