// aten::convolution_overrideable / convolution_backward_overrideable on xdna.
//
// Replaces convolution_overrideable_xdna / convolution_backward_overrideable_xdna
// (torch_xdna_device.cpp:4524-4606, 4608-4885) and the conv3x3w runtimes they
// drive (:1990-2523, 2530-2771).  BF16 3x3 / stride 1 / pad 1 / dilation 1 /
// groups 1 convolutions run the sm_100a implicit-GEMM kernels:
//   forward   pack x -> padded-grid rows, pack w -> Wk, conv kernel (+bias)
//   dX        pack dy -> rows, pack w -> Wk' (flip + transpose), same kernel
//   dW        wgrad kernel over the dy rows and the x rows the forward kept,
//             deferred until the gradient is first read (see deferred.cpp)
//   dbias     sum of dy over (N, H, W)
// Outputs follow the input's memory format (NCHW or channels-last), written
// directly by the kernel epilogue.  Other convolutions (and set_npu_mode(0))
// take ATen's CUDA convolution on aliases -- the reference sends them to its
// CPU path the same way (:4578-4605).
#include <ATen/ops/convolution.h>
#include <ATen/ops/convolution_backward.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "xdna.h"

namespace xdna {
namespace {

bool is3x3s1p1(const at::Tensor& input, const at::Tensor& weight, at::IntArrayRef stride, at::IntArrayRef padding,
               at::IntArrayRef dilation, bool transposed, int64_t groups) {
  if (input.dim() != 4 || weight.dim() != 4 || transposed || groups != 1) return false;
  if (weight.size(2) != 3 || weight.size(3) != 3) return false;
  auto all = [](at::IntArrayRef v, int64_t x) {
    for (auto e : v)
      if (e != x) return false;
    return v.size() == 2;
  };
  return all(stride, 1) && all(padding, 1) && all(dilation, 1) && input.size(1) == weight.size(1);
}

bool bf16(const at::Tensor& t) { return !t.defined() || t.scalar_type() == at::kBFloat16; }

at::MemoryFormat out_format(const at::Tensor& input) {
  return input.suggest_memory_format() == at::MemoryFormat::ChannelsLast ? at::MemoryFormat::ChannelsLast
                                                                          : at::MemoryFormat::Contiguous;
}

int chunks_of(int64_t c) { return int((c + 63) / 64); }

at::Tensor pack_rows(const at::Tensor& x) {
  const int B = int(x.size(0)), C = int(x.size(1)), H = int(x.size(2)), W = int(x.size(3));
  const int ch = chunks_of(C);
  at::Tensor rows = empty({int64_t(B) * (H + 2) * (W + 2), int64_t(ch) * 64}, at::kBFloat16, x.device().index());
  materialize(x);
  XDNA_B2(b2_pack_rows_bf16(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), x.stride(3), B, C, H, W, ch,
                            rows.data_ptr(), stream(x.device().index())));
  count_launch("pack_rows");
  return rows;
}

at::Tensor pack_weight(const at::Tensor& w_in, bool dgrad) {
  at::Tensor w = w_in.is_contiguous() ? w_in : w_in.contiguous();
  materialize(w);
  const int Cout = int(w.size(0)), Cin = int(w.size(1));
  const int ch = chunks_of(dgrad ? Cout : Cin);
  at::Tensor wk = empty({dgrad ? Cin : Cout, int64_t(ch) * 576}, at::kBFloat16, w.device().index());
  if (dgrad)
    XDNA_B2(b2_pack_weight_dgrad_bf16(w.data_ptr(), Cout, Cin, ch, wk.data_ptr(), stream(w.device().index())));
  else
    XDNA_B2(b2_pack_weight_fwd_bf16(w.data_ptr(), Cout, Cin, ch, wk.data_ptr(), stream(w.device().index())));
  count_launch("pack_weight");
  return wk;
}

// dW into `gw` (raw pointer: a deferred job must not keep the gradient's
// storage alive, or an unread gradient could never be freed and dropped).
void launch_wgrad(const at::Tensor& dy_rows, const at::Tensor& x_rows, void* gw, at::ScalarType dtype,
                  c10::DeviceIndex dev, int B, int Cin, int H, int W, int Cout) {
  c10::cuda::CUDAGuard g(dev);
  const size_t ws_bytes = b2_conv3x3_wgrad_workspace_bytes(B, Cin, H, W, Cout);
  at::Tensor ws = empty({int64_t((ws_bytes + 15) / 16) * 4}, at::kFloat, dev);
  const int dt = dtype == at::kFloat ? B2_F32 : B2_BF16;
  XDNA_B2(b2_conv3x3_wgrad(dy_rows.data_ptr(), x_rows.data_ptr(), gw, dt, B, Cin, H, W, Cout, ws.data_ptr(),
                           size_t(ws.numel()) * 4, stream(dev)));
  count_launch("conv3x3.wgrad", 2);  // igemm + split-K reduce
}

bool deferral_enabled() {
  static const bool on = [] {
    const char* s = std::getenv("XDNA_DEFER_DW");
    return !s || std::string(s) != "0";
  }();
  return on;
}

at::Tensor convolution_overrideable(const at::Tensor& input, const at::Tensor& weight,
                                    const std::optional<at::Tensor>& bias_opt, at::IntArrayRef stride,
                                    at::IntArrayRef padding, at::IntArrayRef dilation, bool transposed,
                                    at::IntArrayRef output_padding, int64_t groups) {
  const at::Tensor bias = bias_opt.has_value() ? *bias_opt : at::Tensor();
  const bool fast = g_mode.load() > 0 && is3x3s1p1(input, weight, stride, padding, dilation, transposed, groups) &&
                    bf16(input) && bf16(weight) && bf16(bias) && input.numel() > 0;
  if (!fast) {
    count_fallback("convolution_overrideable");
    c10::cuda::CUDAGuard g(input.device().index());
    return adopt(at::convolution(to_cuda(input), to_cuda(weight), bias.defined() ? to_cuda(bias) : at::Tensor(),
                                 stride, padding, dilation, transposed, output_padding, groups));
  }
  c10::cuda::CUDAGuard g(input.device().index());
  const int B = int(input.size(0)), Cin = int(input.size(1)), H = int(input.size(2)), W = int(input.size(3));
  const int Cout = int(weight.size(0));
  at::Tensor rows = pack_rows(input);
  at::Tensor wk = pack_weight(weight, false);
  at::Tensor b = bias.defined() ? (bias.is_contiguous() ? bias : bias.contiguous()) : at::Tensor();
  if (b.defined()) materialize(b);
  at::Tensor y = empty({B, Cout, H, W}, at::kBFloat16, input.device().index(), out_format(input));
  XDNA_B2(b2_conv3x3_fwd(rows.data_ptr(), wk.data_ptr(), b.defined() ? b.data_ptr() : nullptr, y.data_ptr(),
                         y.stride(0), y.stride(1), y.stride(2), y.stride(3), B, Cin, H, W, Cout, 0,
                         stream(input.device().index())));
  count_launch("conv3x3.fwd");
  // keep the packed input for the weight gradient when one will be needed
  if (at::GradMode::is_enabled() && weight.requires_grad() && g_mode.load() > 1) attach_rows(input, rows);
  return y;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> convolution_backward_overrideable(
    const at::Tensor& grad_output, const at::Tensor& input, const at::Tensor& weight, at::IntArrayRef stride,
    at::IntArrayRef padding, at::IntArrayRef dilation, bool transposed, at::IntArrayRef output_padding, int64_t groups,
    std::array<bool, 3> output_mask) {
  const bool fast = g_mode.load() > 0 && is3x3s1p1(input, weight, stride, padding, dilation, transposed, groups) &&
                    bf16(input) && bf16(weight) && bf16(grad_output) && input.numel() > 0;
  c10::cuda::CUDAGuard g(input.device().index());
  if (!fast) {
    count_fallback("convolution_backward_overrideable");
    auto r = at::convolution_backward(to_cuda(grad_output), to_cuda(input), to_cuda(weight), std::nullopt, stride,
                                      padding, dilation, transposed, output_padding, groups, output_mask);
    return {adopt(std::get<0>(r)), adopt(std::get<1>(r)), adopt(std::get<2>(r))};
  }
  const int B = int(input.size(0)), Cin = int(input.size(1)), H = int(input.size(2)), W = int(input.size(3));
  const int Cout = int(weight.size(0));
  const c10::DeviceIndex dev = input.device().index();
  at::Tensor dx, dw, db;
  at::Tensor dy_rows;
  if (output_mask[2]) {
    // the dY packer also reduces dbias (one pass over dY, deterministic order)
    const int ch = chunks_of(Cout);
    dy_rows = empty({int64_t(B) * (H + 2) * (W + 2), int64_t(ch) * 64}, at::kBFloat16, dev);
    db = empty({Cout}, grad_output.scalar_type(), dev);
    const size_t ws_bytes = b2_pack_rows_dbias_workspace_bytes(B, Cout, H, W);
    at::Tensor ws = empty({int64_t((ws_bytes + 15) / 16) * 4}, at::kFloat, dev);
    materialize(grad_output);
    XDNA_B2(b2_pack_rows_dbias_bf16(grad_output.data_ptr(), grad_output.stride(0), grad_output.stride(1),
                                    grad_output.stride(2), grad_output.stride(3), B, Cout, H, W, ch, dy_rows.data_ptr(),
                                    db.data_ptr(), B2_BF16, ws.data_ptr(), size_t(ws.numel()) * 4, stream(dev)));
    count_launch("pack_rows_dbias", 3);  // pack + two channel-sum stages
  } else {
    dy_rows = pack_rows(grad_output);
  }
  if (output_mask[0]) {
    at::Tensor wkd = pack_weight(weight, true);
    dx = empty({B, Cin, H, W}, at::kBFloat16, dev, out_format(input));
    XDNA_B2(b2_conv3x3_dgrad(dy_rows.data_ptr(), wkd.data_ptr(), dx.data_ptr(), dx.stride(0), dx.stride(1),
                             dx.stride(2), dx.stride(3), B, Cout, H, W, Cin, stream(dev)));
    count_launch("conv3x3.dgrad");
  }
  if (output_mask[1]) {
    dw = empty({Cout, Cin, 3, 3}, weight.scalar_type(), dev);
    if (g_mode.load() > 1) {
      at::Tensor x_rows = find_rows(input);
      if (!x_rows.defined()) x_rows = pack_rows(input);
      if (deferral_enabled()) {
        defer_write(dw, [dy_rows, x_rows, gw = dw.data_ptr(), dtype = dw.scalar_type(), dev, B, Cin, H, W, Cout]() {
          launch_wgrad(dy_rows, x_rows, gw, dtype, dev, B, Cin, H, W, Cout);
        });
      } else {
        launch_wgrad(dy_rows, x_rows, dw.data_ptr(), dw.scalar_type(), dev, B, Cin, H, W, Cout);
      }
    } else {
      // mode 1: weight gradient through ATen's CUDA path
      count_fallback("convolution_backward_overrideable.dw");
      auto r = at::convolution_backward(to_cuda(grad_output), to_cuda(input), to_cuda(weight), std::nullopt, stride,
                                        padding, dilation, transposed, output_padding, groups, {false, true, false});
      to_cuda_nosync(dw).copy_(std::get<1>(r));
    }
  }
  if (output_mask[0]) note_dgrad();
  return {dx, dw, db};
}

}  // namespace

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("convolution_overrideable", convolution_overrideable);
  m.impl("convolution_backward_overrideable", convolution_backward_overrideable);
}

}  // namespace xdna
