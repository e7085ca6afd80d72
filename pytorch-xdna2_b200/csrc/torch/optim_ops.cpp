// aten::_fused_adam_ / _fused_adamw_ / _fused_sgd_ (and .tensor_lr) on xdna:
// one multi-tensor launch of the b2 fused Adam or SGD kernel per call.
//
// The reference had no device kernel for these; torch.optim's fused Adam
// reached its CPU kernel through the boxed fallback, which also materialized
// any deferred weight gradient first (torch_xdna_device.cpp:5124-5260,
// device.py:408-452).  Here the grads are materialized (their wgrad kernels
// enqueued) and the update runs on the same stream, bit-exact with torch's
// CPU fused Adam on bf16 parameters.  Parameters' version counters are bumped
// (the reference does that from a Python post-hook).
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "xdna.h"

namespace xdna {
namespace {

// The kernels update element i of every array together, so any dense layout
// works as long as all arrays of a parameter share it (channels-last conv
// weights and their gradients and states are dense, not contiguous).
bool dense_like(const at::Tensor& t, const at::Tensor& ref) {
  if (t.device().type() != kXdna || !t.is_non_overlapping_and_dense() || !t.sizes().equals(ref.sizes())) return false;
  for (int64_t d = 0; d < t.dim(); ++d)  // the stride of a size-1 dimension addresses nothing
    if (t.size(d) > 1 && t.stride(d) != ref.stride(d)) return false;
  return true;
}

bool supported(at::TensorList params, at::TensorList grads, at::TensorList m, at::TensorList v,
               at::TensorList vmax, at::TensorList steps, bool amsgrad, at::ScalarType& pt, at::ScalarType& st) {
  if (g_mode.load() == 0 || params.empty()) return false;
  pt = params[0].scalar_type();
  st = m.empty() ? pt : m[0].scalar_type();
  auto okdt = [](at::ScalarType t) { return t == at::kFloat || t == at::kBFloat16; };
  if (!okdt(pt) || !okdt(st)) return false;
  const size_t n = params.size();
  if (grads.size() != n || m.size() != n || v.size() != n || steps.size() != n || (amsgrad && vmax.size() != n))
    return false;
  for (size_t i = 0; i < n; ++i) {
    const at::Tensor* ts[] = {&params[i], &grads[i], &m[i], &v[i]};
    for (const at::Tensor* t : ts)
      if (!dense_like(*t, params[i])) return false;
    if (params[i].scalar_type() != pt || grads[i].scalar_type() != pt || m[i].scalar_type() != st ||
        v[i].scalar_type() != st)
      return false;
    if (amsgrad && (vmax[i].scalar_type() != st || !dense_like(vmax[i], params[i])))
      return false;
    if (steps[i].device().type() != kXdna || steps[i].scalar_type() != at::kFloat || steps[i].numel() != 1)
      return false;
  }
  return true;
}

const float* scalar_ptr(const std::optional<at::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK(t->device().type() == kXdna && t->scalar_type() == at::kFloat && t->numel() == 1,
              "xdna fused Adam: grad_scale/found_inf/lr must be float32 scalars on xdna");
  materialize(*t);
  return t->data_ptr<float>();
}

void fused_adam_impl(at::TensorList params, at::TensorList grads, at::TensorList m, at::TensorList v,
                     at::TensorList vmax, at::TensorList steps, double lr, const at::Tensor* lr_t, double beta1,
                     double beta2, double wd, double eps, bool amsgrad, bool maximize,
                     const std::optional<at::Tensor>& grad_scale, const std::optional<at::Tensor>& found_inf,
                     bool adamw) {
  for (const at::Tensor& p : params) {
    before_write(p);
    note_write(p);
  }
  at::ScalarType pt, st;
  if (!supported(params, grads, m, v, vmax, steps, amsgrad, pt, st)) {
    // unsupported layout/dtype mix: ATen's CUDA fused kernel on aliases
    count_fallback(adamw ? "_fused_adamw_" : "_fused_adam_");
    auto conv = [](at::TensorList l) {
      std::vector<at::Tensor> out;
      for (const auto& t : l) out.push_back(to_cuda(t));
      return out;
    };
    auto P = conv(params), G = conv(grads), M = conv(m), V = conv(v), X = conv(vmax), S = conv(steps);
    std::optional<at::Tensor> gs = grad_scale.has_value() ? std::optional<at::Tensor>(to_cuda(*grad_scale)) : std::nullopt;
    std::optional<at::Tensor> fi = found_inf.has_value() ? std::optional<at::Tensor>(to_cuda(*found_inf)) : std::nullopt;
    c10::cuda::CUDAGuard g(params[0].device().index());
    if (lr_t) {
      if (adamw)
        at::_fused_adamw_(P, G, M, V, X, S, to_cuda(*lr_t), beta1, beta2, wd, eps, amsgrad, maximize, gs, fi);
      else
        at::_fused_adam_(P, G, M, V, X, S, to_cuda(*lr_t), beta1, beta2, wd, eps, amsgrad, maximize, gs, fi);
    } else {
      if (adamw)
        at::_fused_adamw_(P, G, M, V, X, S, lr, beta1, beta2, wd, eps, amsgrad, maximize, gs, fi);
      else
        at::_fused_adam_(P, G, M, V, X, S, lr, beta1, beta2, wd, eps, amsgrad, maximize, gs, fi);
    }
    for (const auto& p : params) p.unsafeGetTensorImpl()->bump_version();
    note_optimizer_step();
    return;
  }
  const c10::DeviceIndex dev = params[0].device().index();
  c10::cuda::CUDAGuard g(dev);
  std::vector<b2_adam_tensor> ts(params.size());
  for (size_t i = 0; i < params.size(); ++i) {
    materialize(grads[i]);  // deferred weight gradients are computed here at the latest
    materialize(params[i]);
    ts[i].param = params[i].data_ptr();
    ts[i].grad = grads[i].data_ptr();
    ts[i].exp_avg = m[i].data_ptr();
    ts[i].exp_avg_sq = v[i].data_ptr();
    ts[i].max_exp_avg_sq = amsgrad ? vmax[i].data_ptr() : nullptr;
    ts[i].step = steps[i].data_ptr<float>();
    ts[i].numel = params[i].numel();
  }
  b2_adam_hparams hp{};
  hp.lr = lr;
  hp.beta1 = beta1;
  hp.beta2 = beta2;
  hp.weight_decay = wd;
  hp.eps = eps;
  hp.amsgrad = amsgrad;
  hp.maximize = maximize;
  hp.adamw = adamw;
  hp.param_dtype = pt == at::kFloat ? B2_F32 : B2_BF16;
  hp.state_dtype = st == at::kFloat ? B2_F32 : B2_BF16;
  hp.lr_tensor = nullptr;
  if (lr_t) {
    std::optional<at::Tensor> l(*lr_t);
    hp.lr_tensor = scalar_ptr(l);
  }
  hp.grad_scale = scalar_ptr(grad_scale);
  hp.found_inf = scalar_ptr(found_inf);
  XDNA_B2(b2_fused_adam(ts.data(), int(ts.size()), &hp, stream(dev)));
  count_launch("fused_adam");
  for (const auto& p : params) p.unsafeGetTensorImpl()->bump_version();
  note_optimizer_step();
}

void fused_adam(at::TensorList self, at::TensorList grads, at::TensorList exp_avgs, at::TensorList exp_avg_sqs,
                at::TensorList max_exp_avg_sqs, at::TensorList state_steps, double lr, double beta1, double beta2,
                double weight_decay, double eps, bool amsgrad, bool maximize,
                const std::optional<at::Tensor>& grad_scale, const std::optional<at::Tensor>& found_inf) {
  fused_adam_impl(self, grads, exp_avgs, exp_avg_sqs, max_exp_avg_sqs, state_steps, lr, nullptr, beta1, beta2,
                  weight_decay, eps, amsgrad, maximize, grad_scale, found_inf, false);
}

void fused_adam_tlr(at::TensorList self, at::TensorList grads, at::TensorList exp_avgs, at::TensorList exp_avg_sqs,
                    at::TensorList max_exp_avg_sqs, at::TensorList state_steps, const at::Tensor& lr, double beta1,
                    double beta2, double weight_decay, double eps, bool amsgrad, bool maximize,
                    const std::optional<at::Tensor>& grad_scale, const std::optional<at::Tensor>& found_inf) {
  fused_adam_impl(self, grads, exp_avgs, exp_avg_sqs, max_exp_avg_sqs, state_steps, 0.0, &lr, beta1, beta2,
                  weight_decay, eps, amsgrad, maximize, grad_scale, found_inf, false);
}

void fused_adamw(at::TensorList self, at::TensorList grads, at::TensorList exp_avgs, at::TensorList exp_avg_sqs,
                 at::TensorList max_exp_avg_sqs, at::TensorList state_steps, double lr, double beta1, double beta2,
                 double weight_decay, double eps, bool amsgrad, bool maximize,
                 const std::optional<at::Tensor>& grad_scale, const std::optional<at::Tensor>& found_inf) {
  fused_adam_impl(self, grads, exp_avgs, exp_avg_sqs, max_exp_avg_sqs, state_steps, lr, nullptr, beta1, beta2,
                  weight_decay, eps, amsgrad, maximize, grad_scale, found_inf, true);
}

void fused_adamw_tlr(at::TensorList self, at::TensorList grads, at::TensorList exp_avgs, at::TensorList exp_avg_sqs,
                     at::TensorList max_exp_avg_sqs, at::TensorList state_steps, const at::Tensor& lr, double beta1,
                     double beta2, double weight_decay, double eps, bool amsgrad, bool maximize,
                     const std::optional<at::Tensor>& grad_scale, const std::optional<at::Tensor>& found_inf) {
  fused_adam_impl(self, grads, exp_avgs, exp_avg_sqs, max_exp_avg_sqs, state_steps, 0.0, &lr, beta1, beta2,
                  weight_decay, eps, amsgrad, maximize, grad_scale, found_inf, true);
}

// aten::_fused_sgd_ (and .tensor_lr): torch.optim.SGD(fused=True), which the
// reference's _prefer_fused_optimizer selects for device parameters
// (device.py:408-436) and runs on its CPU through the boxed fallback.  An
// empty momentum-buffer list means no momentum, as in ATen's kernels.
bool sgd_supported(at::TensorList params, at::TensorList grads, at::TensorList bufs, at::ScalarType& pt) {
  if (g_mode.load() == 0 || params.empty()) return false;
  pt = params[0].scalar_type();
  if (pt != at::kFloat && pt != at::kBFloat16) return false;
  const size_t n = params.size();
  if (grads.size() != n || (!bufs.empty() && bufs.size() != n)) return false;
  for (size_t i = 0; i < n; ++i) {
    std::vector<const at::Tensor*> ts = {&params[i], &grads[i]};
    if (!bufs.empty()) ts.push_back(&bufs[i]);
    for (const at::Tensor* t : ts)
      if (!dense_like(*t, params[i]) || t->scalar_type() != pt) return false;
  }
  return true;
}

void fused_sgd_impl(at::TensorList params, at::TensorList grads, at::TensorList bufs, double wd, double momentum,
                    double lr, const at::Tensor* lr_t, double dampening, bool nesterov, bool maximize,
                    bool is_first_step, const std::optional<at::Tensor>& grad_scale,
                    const std::optional<at::Tensor>& found_inf) {
  for (const at::Tensor& p : params) {
    before_write(p);
    note_write(p);
  }
  at::ScalarType pt;
  if (!sgd_supported(params, grads, bufs, pt)) {
    count_fallback("_fused_sgd_");
    auto conv = [](at::TensorList l) {
      std::vector<at::Tensor> out;
      for (const auto& t : l) out.push_back(to_cuda(t));
      return out;
    };
    auto P = conv(params), G = conv(grads), M = conv(bufs);
    std::optional<at::Tensor> gs = grad_scale.has_value() ? std::optional<at::Tensor>(to_cuda(*grad_scale)) : std::nullopt;
    std::optional<at::Tensor> fi = found_inf.has_value() ? std::optional<at::Tensor>(to_cuda(*found_inf)) : std::nullopt;
    c10::cuda::CUDAGuard g(params[0].device().index());
    if (lr_t)
      at::_fused_sgd_(P, G, M, wd, momentum, to_cuda(*lr_t), dampening, nesterov, maximize, is_first_step, gs, fi);
    else
      at::_fused_sgd_(P, G, M, wd, momentum, lr, dampening, nesterov, maximize, is_first_step, gs, fi);
    for (const auto& p : params) p.unsafeGetTensorImpl()->bump_version();
    note_optimizer_step();
    return;
  }
  const c10::DeviceIndex dev = params[0].device().index();
  c10::cuda::CUDAGuard g(dev);
  std::vector<b2_sgd_tensor> ts(params.size());
  for (size_t i = 0; i < params.size(); ++i) {
    materialize(grads[i]);  // deferred weight gradients are computed here at the latest
    materialize(params[i]);
    if (!bufs.empty()) materialize(bufs[i]);
    ts[i].param = params[i].data_ptr();
    ts[i].grad = grads[i].data_ptr();
    ts[i].momentum_buffer = bufs.empty() ? nullptr : bufs[i].data_ptr();
    ts[i].numel = params[i].numel();
  }
  b2_sgd_hparams hp{};
  hp.lr = lr;
  hp.weight_decay = wd;
  hp.momentum = bufs.empty() ? 0.0 : momentum;
  hp.dampening = dampening;
  hp.nesterov = nesterov;
  hp.maximize = maximize;
  hp.is_first_step = is_first_step;
  hp.param_dtype = pt == at::kFloat ? B2_F32 : B2_BF16;
  hp.lr_tensor = nullptr;
  if (lr_t) {
    std::optional<at::Tensor> l(*lr_t);
    hp.lr_tensor = scalar_ptr(l);
  }
  hp.grad_scale = scalar_ptr(grad_scale);
  hp.found_inf = scalar_ptr(found_inf);
  XDNA_B2(b2_fused_sgd(ts.data(), int(ts.size()), &hp, stream(dev)));
  count_launch("fused_sgd");
  for (const auto& p : params) p.unsafeGetTensorImpl()->bump_version();
  note_optimizer_step();
}

void fused_sgd(at::TensorList self, at::TensorList grads, at::TensorList bufs, double weight_decay, double momentum,
               double lr, double dampening, bool nesterov, bool maximize, bool is_first_step,
               const std::optional<at::Tensor>& grad_scale, const std::optional<at::Tensor>& found_inf) {
  fused_sgd_impl(self, grads, bufs, weight_decay, momentum, lr, nullptr, dampening, nesterov, maximize, is_first_step,
                 grad_scale, found_inf);
}

void fused_sgd_tlr(at::TensorList self, at::TensorList grads, at::TensorList bufs, double weight_decay,
                   double momentum, const at::Tensor& lr, double dampening, bool nesterov, bool maximize,
                   bool is_first_step, const std::optional<at::Tensor>& grad_scale,
                   const std::optional<at::Tensor>& found_inf) {
  fused_sgd_impl(self, grads, bufs, weight_decay, momentum, 0.0, &lr, dampening, nesterov, maximize, is_first_step,
                 grad_scale, found_inf);
}

}  // namespace

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("_fused_sgd_", fused_sgd);
  m.impl("_fused_sgd_.tensor_lr", fused_sgd_tlr);
  m.impl("_fused_adam_", fused_adam);
  m.impl("_fused_adam_.tensor_lr", fused_adam_tlr);
  m.impl("_fused_adamw_", fused_adamw);
  m.impl("_fused_adamw_.tensor_lr", fused_adamw_tlr);
}

}  // namespace xdna
