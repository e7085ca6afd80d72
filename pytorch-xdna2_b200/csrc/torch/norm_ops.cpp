// Training-mode BatchNorm with xdna kernels: `native_batch_norm` and
// `native_batch_norm_backward` (the reference runs ATen's CPU kernels on
// aliases, torch_xdna_device.cpp:4214-4358).
//
// Fast path (b2_batch_norm_*): training mode, bf16 input of rank >= 2 that is
// contiguous (NCHW order) or 4-D channels-last with C % 8 == 0 and C <= 2048;
// weight, bias, running statistics absent or bf16 / fp32 xdna vectors of C
// elements.  save_mean / save_invstd are fp32.  Evaluation mode and every
// other case run ATen's CUDA kernels on zero-copy CUDA aliases.
#include <ATen/ops/threshold_backward.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "xdna.h"

namespace xdna {

// XDNA_BN_EPILOGUE=0 turns the folding of add_ / relu_ into BatchNorm's
// output pass off (xdna_train.set_fusion switches it at run time).
std::atomic<bool> g_bn_epilogue{[] {
  const char* s = std::getenv("XDNA_BN_EPILOGUE");
  return !s || std::string(s) != "0";
}()};

namespace {

int vec_dtype(const std::optional<at::Tensor>& t, int64_t C) {
  if (!t.has_value() || !t->defined()) return B2_BF16;  // absent: any
  if (t->device().type() != kXdna || !t->is_contiguous() || t->numel() != C) return -1;
  return t->scalar_type() == at::kBFloat16 ? B2_BF16 : t->scalar_type() == at::kFloat ? B2_F32 : -1;
}

bool defined(const std::optional<at::Tensor>& t) { return t.has_value() && t->defined(); }

const void* ptr_of(const std::optional<at::Tensor>& t) {
  if (!defined(t)) return nullptr;
  materialize(*t);
  return t->data_ptr();
}

// 0 = contiguous, 1 = channels-last (4-D), -1 = neither or not supported.
int bn_layout(const at::Tensor& x) {
  if (x.dim() == 4 && x.suggest_memory_format() == c10::MemoryFormat::ChannelsLast &&
      x.is_contiguous(c10::MemoryFormat::ChannelsLast))
    return (x.size(1) % 8 == 0 && x.size(1) <= 2048) ? 1 : -1;
  return x.is_contiguous() ? 0 : -1;
}

std::vector<at::Tensor> as_cuda(const std::vector<std::optional<at::Tensor>>& ts) {
  std::vector<at::Tensor> out;
  for (const auto& t : ts) out.push_back(defined(t) ? to_cuda(*t) : at::Tensor());
  return out;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> bn_fwd_alias(
    const at::Tensor& input, const std::optional<at::Tensor>& weight, const std::optional<at::Tensor>& bias,
    const std::optional<at::Tensor>& rm, const std::optional<at::Tensor>& rv, bool training, double momentum,
    double eps) {
  count_fallback("aten::native_batch_norm");
  c10::cuda::CUDAGuard g(input.device().index());
  auto c = as_cuda({weight, bias, rm, rv});
  auto r = at::native_batch_norm(to_cuda(input), c[0], c[1], c[2], c[3], training, momentum, eps);
  return {adopt(std::get<0>(r)), adopt(std::get<1>(r)), adopt(std::get<2>(r))};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> native_batch_norm(
    const at::Tensor& input, const std::optional<at::Tensor>& weight, const std::optional<at::Tensor>& bias,
    const std::optional<at::Tensor>& running_mean, const std::optional<at::Tensor>& running_var, bool training,
    double momentum, double eps) {
  const int64_t C = input.dim() >= 2 ? input.size(1) : 0;
  const int layout = input.dim() >= 2 ? bn_layout(input) : -1;
  const int pw = vec_dtype(weight, C), pb = vec_dtype(bias, C);
  const int rdm = vec_dtype(running_mean, C), rdv = vec_dtype(running_var, C);
  const bool params_ok = pw >= 0 && pb >= 0 && (!defined(weight) || !defined(bias) || pw == pb);
  const bool stats_ok = rdm >= 0 && rdv >= 0 && defined(running_mean) == defined(running_var) &&
                        (!defined(running_mean) || rdm == rdv);
  if (g_mode.load() == 0 || !training || input.scalar_type() != at::kBFloat16 || layout < 0 || !params_ok ||
      !stats_ok || input.numel() == 0)
    return bn_fwd_alias(input, weight, bias, running_mean, running_var, training, momentum, eps);
  const auto dev = input.device().index();
  const int64_t N = input.size(0), HW = input.numel() / (N * C);
  const auto mf = layout == 1 ? c10::MemoryFormat::ChannelsLast : c10::MemoryFormat::Contiguous;
  at::Tensor out = empty(input.sizes(), at::kBFloat16, dev, mf);
  at::Tensor stats = empty({2, C}, at::kFloat, dev);
  at::Tensor save_mean = stats[0], save_invstd = stats[1];
  const int64_t wsb = int64_t(b2_batch_norm_workspace_bytes(N, C, HW, layout));
  at::Tensor ws = empty({std::max<int64_t>(wsb, 16)}, at::kByte, dev);
  materialize(input);
  const int pdt = defined(weight) ? pw : pb;
  c10::cuda::CUDAGuard g(dev);
  if (g_bn_epilogue.load() && g_mode.load() > 1) {
    // statistics now; the output pass waits for the first reader of `out`,
    // so that a residual add_ and a relu_ on `out` fold into it
    {
      // the module's num_batches_tracked.add_(1) just before this forward,
      // if still pending, advances inside the statistics launch
      const PendingCount pc = take_pending_count(dev);
      KernelTimer kt("bn.stats", 2.0 * double(input.numel()), stream(dev));  // work: algorithmic bytes
      if (pc.counter.defined())
        XDNA_B2(b2_batch_norm_stats_count_bf16(
            input.data_ptr(), layout, pdt, const_cast<void*>(ptr_of(running_mean)),
            const_cast<void*>(ptr_of(running_var)), rdm, save_mean.data_ptr<float>(), save_invstd.data_ptr<float>(),
            N, C, HW, float(momentum), float(eps), static_cast<int64_t*>(pc.counter.data_ptr()), pc.inc,
            ws.data_ptr(), size_t(ws.numel()), stream(dev)));
      else
        XDNA_B2(b2_batch_norm_stats_bf16(input.data_ptr(), layout, pdt, const_cast<void*>(ptr_of(running_mean)),
                                         const_cast<void*>(ptr_of(running_var)), rdm, save_mean.data_ptr<float>(),
                                         save_invstd.data_ptr<float>(), N, C, HW, float(momentum), float(eps),
                                         ws.data_ptr(), size_t(ws.numel()), stream(dev)));
    }
    count_launch("batch_norm.fwd", 2);
    auto spec = std::make_shared<EpiSpec>();
    const at::Tensor w = defined(weight) ? *weight : at::Tensor();
    const at::Tensor b = defined(bias) ? *bias : at::Tensor();
    if (w.defined()) materialize(w);
    if (b.defined()) materialize(b);
    void* y = out.data_ptr();  // raw: an unread output must stay free to drop its pass
    // the output's geometry, to register it as a gated output when its pass
    // folded a relu_ and no residual (the pass runs while the output lives)
    auto geo = std::make_shared<std::pair<std::vector<int64_t>, std::vector<int64_t>>>(out.sizes().vec(),
                                                                                      out.strides().vec());
    defer_epilogue(out, {input, w, b}, spec, [input, w, b, stats, spec, y, layout, pdt, N, C, HW, dev, geo]() {
      c10::cuda::CUDAGuard guard(dev);
      const at::Tensor& r = spec->residual;
      if (spec->relu && !r.defined() && layout == 1) {
        auto src = std::make_shared<GateSource>();
        src->x = input;
        src->w = w;
        src->b = b;
        src->stats = stats;
        src->x_version = int64_t(input._version());
        src->w_version = w.defined() ? int64_t(w._version()) : 0;
        src->b_version = b.defined() ? int64_t(b._version()) : 0;
        src->pdtype = pdt;
        note_gate_source(y, geo->first, geo->second, 0, std::move(src));
      }
      KernelTimer kt(r.defined() ? "bn.apply_res" : "bn.apply", (r.defined() ? 6.0 : 4.0) * double(input.numel()),
                     stream(dev));
      XDNA_B2(b2_batch_norm_apply_bf16(input.data_ptr(), layout, w.defined() ? w.data_ptr() : nullptr,
                                       b.defined() ? b.data_ptr() : nullptr, pdt, stats[0].data_ptr<float>(),
                                       stats[1].data_ptr<float>(), r.defined() ? r.data_ptr() : nullptr,
                                       spec->relu ? 1 : 0, y, N, C, HW, stream(dev)));
      count_launch("batch_norm.fwd");
    });
    return {out, save_mean, save_invstd};
  }
  XDNA_B2(b2_batch_norm_fwd_bf16(input.data_ptr(), layout, ptr_of(weight), ptr_of(bias), pdt,
                                 const_cast<void*>(ptr_of(running_mean)), const_cast<void*>(ptr_of(running_var)),
                                 rdm, out.data_ptr(), save_mean.data_ptr<float>(), save_invstd.data_ptr<float>(), N,
                                 C, HW, float(momentum), float(eps), ws.data_ptr(), size_t(ws.numel()), stream(dev)));
  count_launch("batch_norm.fwd", 3);
  return {out, save_mean, save_invstd};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> native_batch_norm_backward(
    const at::Tensor& grad_out, const at::Tensor& input, const std::optional<at::Tensor>& weight,
    const std::optional<at::Tensor>& running_mean, const std::optional<at::Tensor>& running_var,
    const std::optional<at::Tensor>& save_mean, const std::optional<at::Tensor>& save_invstd, bool train,
    double eps, std::array<bool, 3> mask) {
  const int64_t C = input.dim() >= 2 ? input.size(1) : 0;
  const int layout = input.dim() >= 2 ? bn_layout(input) : -1;
  const int pw = vec_dtype(weight, C);
  auto f32_vec = [&](const std::optional<at::Tensor>& t) {
    return defined(t) && t->device().type() == kXdna && t->scalar_type() == at::kFloat && t->is_contiguous() &&
           t->numel() == C;
  };
  const bool fast = g_mode.load() != 0 && train && input.scalar_type() == at::kBFloat16 && layout >= 0 && pw >= 0 &&
                    grad_out.scalar_type() == at::kBFloat16 && grad_out.sizes() == input.sizes() &&
                    f32_vec(save_mean) && f32_vec(save_invstd) && input.numel() > 0;
  if (!fast) {
    count_fallback("aten::native_batch_norm_backward");
    c10::cuda::CUDAGuard g(input.device().index());
    auto c = as_cuda({weight, running_mean, running_var, save_mean, save_invstd});
    auto r = at::native_batch_norm_backward(to_cuda(grad_out), to_cuda(input), c[0], c[1], c[2], c[3], c[4], train,
                                            eps, mask);
    return {adopt(std::get<0>(r)), adopt(std::get<1>(r)), adopt(std::get<2>(r))};
  }
  const auto dev = input.device().index();
  const auto mf = layout == 1 ? c10::MemoryFormat::ChannelsLast : c10::MemoryFormat::Contiguous;
  const int64_t N = input.size(0), HW = input.numel() / (N * C);
  const auto gdt = defined(weight) ? weight->scalar_type() : at::kFloat;
  // grad_out still pending as the ReLU backward of a pending gradient sum
  // (a residual block's last BatchNorm): dz made, written and reduced in one
  // pass from the sum's two terms and the ReLU's output
  if (auto rs = layout == 1 ? find_epilogue(grad_out) : nullptr;
      rs && rs->relu_sum_a.defined() && has_pending(rs->relu_sum_a) && grad_out.is_contiguous(mf) &&
      grad_out.strides() == input.strides()) {
    at::Tensor gi, gw, gb;
    if (mask[0]) gi = empty(input.sizes(), at::kBFloat16, dev, mf);
    if (mask[1]) gw = empty({C}, gdt, dev);
    if (mask[2]) gb = empty({C}, gdt, dev);
    const int64_t wsb = int64_t(b2_batch_norm_workspace_bytes(N, C, HW, 1));
    at::Tensor ws = empty({std::max<int64_t>(wsb, 16)}, at::kByte, dev);
    materialize(rs->relu_sum_b);
    materialize(rs->relu_sum_y);
    materialize(input);
    c10::cuda::CUDAGuard guard(dev);
    KernelTimer kt("bn.bwd_relu_sum", (mask[0] ? 16.0 : 10.0) * double(input.numel()), stream(dev));
    const b2_status st = b2_batch_norm_bwd_relu_sum_bf16(
        rs->relu_sum_a.data_ptr(), rs->relu_sum_b.data_ptr(), rs->relu_sum_y.data_ptr(), input.data_ptr(),
        ptr_of(weight), pw, save_mean->data_ptr<float>(), save_invstd->data_ptr<float>(), grad_out.data_ptr(),
        mask[0] ? gi.data_ptr() : nullptr, mask[1] ? gw.data_ptr() : nullptr, mask[2] ? gb.data_ptr() : nullptr,
        gdt == at::kFloat ? B2_F32 : B2_BF16, N, C, HW, ws.data_ptr(), size_t(ws.numel()), stream(dev));
    if (st == B2_OK) {
      drop_pending(grad_out);  // dz written by the fused pass
      count_launch("batch_norm.bwd_relu_sum", mask[0] ? 3 : 2);
      return {gi, gw, gb};
    }
    TORCH_CHECK(st == B2_ERR_UNSUPPORTED, "xdna: b2_batch_norm_bwd_relu_sum_bf16 failed (", st, "): ",
                b2_last_error());
  }
  // grad_out still pending as threshold_backward(grad, y, 0) of this
  // BatchNorm's own gated output: one backward from `grad`, the ReLU's gate
  // recomputed from x (the pending pass is never run unless read elsewhere)
  if (auto spec = layout == 1 ? find_epilogue(grad_out) : nullptr; spec && spec->gate) {
    const GateSource& src = *spec->gate;
    const at::Tensor& gg = spec->gate_grad;
    const bool same_bn =
        src.x.is_same(input) && int64_t(input._version()) == src.x_version &&
        save_mean->data_ptr() == src.stats[0].data_ptr() && save_invstd->data_ptr() == src.stats[1].data_ptr() &&
        (defined(weight) ? (src.w.defined() && weight->is_same(src.w) && int64_t(src.w._version()) == src.w_version)
                         : !src.w.defined()) &&
        (!src.b.defined() || int64_t(src.b._version()) == src.b_version) && gg.is_contiguous(mf);
    if (same_bn) {
      at::Tensor gi, gw, gb;
      if (mask[0]) gi = empty(input.sizes(), at::kBFloat16, dev, mf);
      if (mask[1]) gw = empty({C}, gdt, dev);
      if (mask[2]) gb = empty({C}, gdt, dev);
      const int64_t wsb = int64_t(b2_batch_norm_workspace_bytes(N, C, HW, 1));
      at::Tensor ws = empty({std::max<int64_t>(wsb, 16)}, at::kByte, dev);
      materialize(gg);
      materialize(input);
      c10::cuda::CUDAGuard guard(dev);
      KernelTimer kt("bn.bwd_relu", (mask[0] ? 10.0 : 4.0) * double(input.numel()), stream(dev));
      const b2_status st = b2_batch_norm_relu_bwd_bf16(
          gg.data_ptr(), input.data_ptr(), src.w.defined() ? src.w.data_ptr() : nullptr,
          src.b.defined() ? src.b.data_ptr() : nullptr, src.pdtype, save_mean->data_ptr<float>(),
          save_invstd->data_ptr<float>(), mask[0] ? gi.data_ptr() : nullptr, mask[1] ? gw.data_ptr() : nullptr,
          mask[2] ? gb.data_ptr() : nullptr, gdt == at::kFloat ? B2_F32 : B2_BF16, N, C, HW, ws.data_ptr(),
          size_t(ws.numel()), stream(dev));
      if (st == B2_OK) {
        count_launch("batch_norm.bwd_relu", mask[0] ? 3 : 2);
        return {gi, gw, gb};
      }
      TORCH_CHECK(st == B2_ERR_UNSUPPORTED, "xdna: b2_batch_norm_relu_bwd_bf16 failed (", st, "): ",
                  b2_last_error());
    }
  }
  // the gradient in the input's memory order (a copy only when they differ)
  at::Tensor g = grad_out.is_contiguous(mf) ? grad_out : grad_out.contiguous(mf);
  at::Tensor gi, gw, gb;
  if (mask[0]) gi = empty(input.sizes(), at::kBFloat16, dev, mf);
  if (mask[1]) gw = empty({C}, gdt, dev);
  if (mask[2]) gb = empty({C}, gdt, dev);
  const int64_t wsb = int64_t(b2_batch_norm_workspace_bytes(N, C, HW, layout));
  at::Tensor ws = empty({std::max<int64_t>(wsb, 16)}, at::kByte, dev);
  materialize(g);
  materialize(input);
  c10::cuda::CUDAGuard guard(dev);
  KernelTimer kt("bn.bwd", (mask[0] ? 10.0 : 4.0) * double(input.numel()), stream(dev));
  XDNA_B2(b2_batch_norm_bwd_bf16(g.data_ptr(), input.data_ptr(), layout, ptr_of(weight), pw,
                                 save_mean->data_ptr<float>(), save_invstd->data_ptr<float>(),
                                 mask[0] ? gi.data_ptr() : nullptr, mask[1] ? gw.data_ptr() : nullptr,
                                 mask[2] ? gb.data_ptr() : nullptr, gdt == at::kFloat ? B2_F32 : B2_BF16, N, C, HW,
                                 ws.data_ptr(), size_t(ws.numel()), stream(dev)));
  count_launch("batch_norm.bwd", mask[0] ? 3 : 2);
  return {gi, gw, gb};
}

// ReLU backward (autograd's ReluBackward: threshold_backward(grad, result,
// 0)).  On a gated BatchNorm output the result is left pending: that
// BatchNorm's backward, its only reader, takes `grad` instead and recomputes
// the gate (b2_batch_norm_relu_bwd_bf16), so this pass never runs; any other
// reader runs it first.  Everything else takes ATen's CUDA kernel on aliases.
at::Tensor threshold_backward(const at::Tensor& grad, const at::Tensor& self, const at::Scalar& threshold) {
  const auto cl = c10::MemoryFormat::ChannelsLast;
  // the gradient is a pending sum (grad += other, left by add_): both terms
  // summed and gated in one pass; grad's own pass is never run unless read
  if (g_mode.load() > 1 && threshold.toDouble() == 0.0 && grad.scalar_type() == at::kBFloat16 &&
      self.scalar_type() == at::kBFloat16 && grad.dim() == 4 && grad.sizes() == self.sizes() &&
      grad.strides() == self.strides() && grad.is_contiguous(cl) && grad.device() == self.device()) {
    if (auto sum = find_epilogue(grad); sum && sum->pending_sum.defined() && (self.numel() % 8 == 0) &&
                                        (reinterpret_cast<uintptr_t>(self.data_ptr()) & 15) == 0) {
      const auto dev = self.device().index();
      materialize(self);
      at::Tensor dz = empty(self.sizes(), at::kBFloat16, dev, cl);
      // dz itself is left pending too: a BatchNorm backward reading it makes
      // it in its own reduction pass; any other reader runs this job
      auto rs = std::make_shared<EpiSpec>();
      rs->relu_sum_a = grad;
      rs->relu_sum_b = sum->pending_sum;
      rs->relu_sum_y = self;
      defer_epilogue(dz, {grad, sum->pending_sum, self}, rs,
                     [grad, other = sum->pending_sum, self, ptr = dz.data_ptr(), sizes = dz.sizes().vec(),
                      strides = dz.strides().vec(), dev]() {
                       c10::cuda::CUDAGuard guard(dev);
                       if (has_pending(grad)) {  // grad still holds a, its sum with `other` pending
                         KernelTimer kt("relu_bwd_sum", 8.0 * double(self.numel()), stream(dev));
                         XDNA_B2(b2_relu_bwd_sum_bf16(grad.data_ptr(), other.data_ptr(), self.data_ptr(), ptr,
                                                      self.numel(), stream(dev)));
                         count_launch("relu_bwd_sum");
                       } else {  // the sum has run in place: a plain ReLU backward of it
                         count_fallback("aten::threshold_backward");
                         at::Tensor out = at::from_blob(
                             ptr, sizes, strides, at::TensorOptions().dtype(at::kBFloat16).device(at::kCUDA, dev));
                         at::threshold_backward_out(out, to_cuda(grad), to_cuda(self), 0);
                       }
                     });
      return dz;
    }
  }
  std::shared_ptr<GateSource> src;
  if (g_bn_epilogue.load() && g_mode.load() > 1 && threshold.toDouble() == 0.0 &&
      grad.scalar_type() == at::kBFloat16 && self.scalar_type() == at::kBFloat16 && grad.dim() == 4 &&
      grad.sizes() == self.sizes() && grad.is_contiguous(cl) && self.is_contiguous(cl) &&
      grad.device() == self.device()) {
    materialize(self);  // a pending output pass registers its gate when it runs
    src = find_gate_source(self);
  }
  if (src) {
    const auto dev = self.device().index();
    at::Tensor dz = empty(self.sizes(), at::kBFloat16, dev, cl);
    auto spec = std::make_shared<EpiSpec>();
    spec->gate_grad = grad;
    spec->gate = std::move(src);
    // raw: an unread gradient must stay free to drop its pass
    defer_epilogue(dz, {grad, self}, spec,
                   [grad, self, ptr = dz.data_ptr(), sizes = dz.sizes().vec(), strides = dz.strides().vec(), dev]() {
                     c10::cuda::CUDAGuard guard(dev);
                     count_fallback("aten::threshold_backward");
                     at::Tensor out = at::from_blob(ptr, sizes, strides,
                                                    at::TensorOptions().dtype(at::kBFloat16).device(at::kCUDA, dev));
                     at::threshold_backward_out(out, to_cuda(grad), to_cuda(self), 0);
                   });
    return dz;
  }
  count_fallback("aten::threshold_backward");
  c10::cuda::CUDAGuard g(self.device().index());
  return adopt(at::threshold_backward(to_cuda(grad), to_cuda(self), threshold));
}

}  // namespace

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("native_batch_norm", native_batch_norm);
  m.impl("native_batch_norm_backward", native_batch_norm_backward);
  m.impl("threshold_backward", threshold_backward);
}

}  // namespace xdna
