// Boxed fallback for every aten op without an `xdna` kernel.
//
// The reference runs such ops as stock ATen CPU kernels on zero-copy CPU
// aliases of its host-mapped buffers (zero_copy_cpu_fallback,
// torch_xdna_device.cpp:5124-5260).  Here xdna memory is HBM, so the same idea
// maps every xdna tensor argument to a zero-copy CUDA alias and redispatches to
// ATen's CUDA kernel: non-hot ops (BatchNorm, activations, pooling, losses,
// elementwise, reductions, factories) stay on the GPU with no copies.
//   * pending deferred writes of every xdna argument are materialized first;
//   * mutated arguments (in-place / out=) are written through the alias; if the
//     op re-allocated an out= tensor, the new memory is adopted back;
//   * returns that alias an argument come back as views of the original xdna
//     storage; fresh results are adopted (xdna storage over the CUDA block).
// Every call is counted per op (fallback_stats); the hot-path ops never come
// here (tests assert their counters stay zero).
#include <ATen/core/dispatch/Dispatcher.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <mutex>
#include <unordered_map>

#include "xdna.h"

namespace xdna {
namespace {

struct ArgMap {
  // CUDA alias storage impl -> original xdna tensor (for view/alias returns)
  std::vector<std::pair<c10::StorageImpl*, at::Tensor>> storages;
};

c10::IValue convert_in(const c10::IValue& v, ArgMap& map, c10::DeviceIndex& dev) {
  if (v.isTensor()) {
    const at::Tensor& t = v.toTensor();
    if (t.defined() && t.device().type() == kXdna) {
      dev = t.device().index();
      at::Tensor c = to_cuda(t);
      map.storages.emplace_back(c.storage().unsafeGetStorageImpl(), t);
      return c;
    }
    return v;
  }
  if (v.isTensorList()) {
    auto list = v.toTensorList();
    c10::List<at::Tensor> out;
    out.reserve(list.size());
    for (const at::Tensor& t : list) {
      if (t.defined() && t.device().type() == kXdna) {
        dev = t.device().index();
        at::Tensor c = to_cuda(t);
        map.storages.emplace_back(c.storage().unsafeGetStorageImpl(), t);
        out.push_back(c);
      } else {
        out.push_back(t);
      }
    }
    return out;
  }
  if (v.isOptionalTensorList()) {
    auto list = v.toOptionalTensorList();
    c10::List<std::optional<at::Tensor>> out;
    for (const std::optional<at::Tensor>& ot : list) {
      if (ot.has_value() && ot->defined() && ot->device().type() == kXdna) {
        dev = ot->device().index();
        out.push_back(std::optional<at::Tensor>(to_cuda(*ot)));
      } else {
        out.push_back(ot);
      }
    }
    return out;
  }
  if (v.isDevice()) {
    c10::Device d = v.toDevice();
    if (d.type() == kXdna) {
      if (d.has_index()) dev = d.index();
      return c10::Device(c10::DeviceType::CUDA, d.has_index() ? d.index() : dev);
    }
    return v;
  }
  return v;
}

at::Tensor convert_out(const at::Tensor& r, const ArgMap& map) {
  if (!r.defined() || r.device().type() != c10::DeviceType::CUDA) return r;
  c10::StorageImpl* si = r.storage().unsafeGetStorageImpl();
  for (const auto& kv : map.storages) {
    if (kv.first == si) {
      // a view of an argument: same xdna storage, the result's geometry
      at::Tensor v = at::detail::make_tensor<c10::TensorImpl>(c10::Storage(kv.second.storage()),
                                                              kv.second.key_set(), r.dtype());
      v.unsafeGetTensorImpl()->set_sizes_and_strides(r.sizes(), r.strides(), r.storage_offset());
      return v;
    }
  }
  return adopt(r);
}

// After an op wrote through the alias of `orig`: if the alias was resized or
// re-pointed (out= resize), carry that back to the xdna tensor.
void sync_back(const at::Tensor& orig, const at::Tensor& alias) {
  auto* oi = orig.unsafeGetTensorImpl();
  if (alias.storage().mutable_data() != orig.storage().mutable_data() ||
      alias.storage().nbytes() != orig.storage().nbytes()) {
    at::Tensor adopted = adopt(alias);
    oi->set_storage_keep_dtype(adopted.storage());
  }
  if (alias.sizes() != orig.sizes() || alias.strides() != orig.strides() ||
      alias.storage_offset() != orig.storage_offset())
    oi->set_sizes_and_strides(alias.sizes(), alias.strides(), alias.storage_offset());
}

void cuda_alias_fallback(const c10::OperatorHandle& op, torch::jit::Stack* stack) {
  const auto& schema = op.schema();
  const size_t nargs = schema.arguments().size();
  const size_t nret = schema.returns().size();
  count_fallback(schema.operator_name().name + (schema.overload_name().empty() ? "" : "." + schema.overload_name()));

  ArgMap map;
  c10::DeviceIndex dev = -1;
  auto args_begin = stack->end() - nargs;
  std::vector<c10::IValue> originals(args_begin, stack->end());
  for (size_t i = 0; i < nargs; ++i) args_begin[i] = convert_in(args_begin[i], map, dev);
  // aliases of mutated arguments, to sync back after the call; deferred
  // producers that read a mutated storage run before the write lands
  std::vector<std::pair<size_t, c10::IValue>> written;
  for (size_t i = 0; i < nargs; ++i) {
    const auto* ai = schema.arguments()[i].alias_info();
    if (ai && ai->isWrite()) {
      written.emplace_back(i, args_begin[i]);
      const c10::IValue& o = originals[i];
      if (o.isTensor()) before_write(o.toTensor());
      else if (o.isTensorList())
        for (const at::Tensor& t : o.toTensorList()) before_write(t);
    }
  }

  {
    c10::cuda::OptionalCUDAGuard g;
    if (dev >= 0) g.set_index(dev);
    op.callBoxed(stack);
  }

  for (auto& w : written) {
    const c10::IValue& o = originals[w.first];
    if (o.isTensor() && o.toTensor().defined() && o.toTensor().device().type() == kXdna) {
      sync_back(o.toTensor(), w.second.toTensor());
      note_write(o.toTensor());
    } else if (o.isTensorList()) {
      auto ol = o.toTensorList();
      auto al = w.second.toTensorList();
      for (size_t k = 0; k < ol.size(); ++k) {
        const at::Tensor& ot = ol[k];
        if (ot.defined() && ot.device().type() == kXdna) {
          sync_back(ot, al[k]);
          note_write(ot);
        }
      }
    }
  }

  auto rets_begin = stack->end() - nret;
  for (size_t i = 0; i < nret; ++i) {
    const auto* ai = schema.returns()[i].alias_info();
    c10::IValue& r = rets_begin[i];
    if (ai && ai->isWrite()) {
      // in-place / out=: return the original argument with the same alias set
      bool done = false;
      for (size_t a = 0; a < nargs && !done; ++a) {
        const auto* aa = schema.arguments()[a].alias_info();
        if (aa && aa->beforeSets() == ai->beforeSets()) {
          r = originals[a];
          done = true;
        }
      }
      if (done) continue;
    }
    if (r.isTensor()) {
      r = convert_out(r.toTensor(), map);
    } else if (r.isTensorList()) {
      auto list = r.toTensorList();
      c10::List<at::Tensor> out;
      out.reserve(list.size());
      for (const at::Tensor& t : list) out.push_back(convert_out(t, map));
      r = out;
    }
  }
}

// relu_ / add_.Tensor on a pending BatchNorm output fold into its output pass
// (the residual add first, then the ReLU, in that order only); anything else
// takes the CUDA-alias path.
void relu_inplace(const c10::OperatorHandle& op, torch::jit::Stack* stack) {
  const at::Tensor self = (*stack)[stack->size() - 1].toTensor();
  if (g_bn_epilogue.load() && self.device().type() == kXdna) {
    auto spec = find_epilogue(self);
    if (spec && spec->foldable() && !spec->relu) {
      spec->relu = true;
      note_folded();
      return;  // the stack holds self, the op's return
    }
  }
  cuda_alias_fallback(op, stack);
}

std::mutex g_count_mu;
PendingCount g_count;  // at most one: a new increment runs the previous first

bool host_integer(const at::Tensor& t) {
  return t.defined() && t.device().is_cpu() && t.dim() == 0 && at::isIntegralType(t.scalar_type(), false);
}

}  // namespace

PendingCount take_pending_count(c10::DeviceIndex dev) {
  PendingCount pc;
  {
    std::lock_guard<std::mutex> lk(g_count_mu);
    if (!g_count.counter.defined() || g_count.counter.device().index() != dev) return {};
    pc = std::move(g_count);
    g_count = PendingCount{};
  }
  if (!has_pending(pc.counter)) return {};  // read (and so run) since
  drop_pending(pc.counter);
  return pc;
}

void flush_pending_count() {
  at::Tensor t;
  {
    std::lock_guard<std::mutex> lk(g_count_mu);
    t = std::move(g_count.counter);
    g_count = PendingCount{};
  }
  if (t.defined()) materialize(t);
}

namespace {

void add_inplace(const c10::OperatorHandle& op, torch::jit::Stack* stack) {
  auto args = stack->end() - 3;  // self, other, alpha
  // a module's step counter: counter.add_(k), an xdna int64 scalar and a host
  // integer -- left pending for the next training BatchNorm forward to
  // advance inside its statistics launch (no kernel of its own)
  if (g_bn_epilogue.load() && g_mode.load() > 1 && args[0].isTensor() && args[1].isTensor() &&
      args[2].isScalar() && args[2].toScalar().isIntegral(false)) {
    const at::Tensor self = args[0].toTensor();
    const at::Tensor other = args[1].toTensor();
    if (self.device().type() == kXdna && self.scalar_type() == at::kLong && self.numel() == 1 && self.dim() <= 1 &&
        self.storage().nbytes() == sizeof(int64_t) && !self.requires_grad() && host_integer(other) &&
        (reinterpret_cast<uintptr_t>(self.data_ptr()) & 7) == 0) {
      const int64_t inc = other.item<int64_t>() * args[2].toScalar().toLong();
      flush_pending_count();
      materialize(self);
      const auto dev = self.device().index();
      defer_write(self,
                  [ptr = self.data_ptr(), dev, inc]() {
                    c10::cuda::CUDAGuard guard(dev);
                    count_fallback("aten::add_.Tensor");
                    at::from_blob(ptr, {1}, at::TensorOptions().dtype(at::kLong).device(at::kCUDA, dev)).add_(inc);
                  },
                  /*kick=*/false);
      {
        std::lock_guard<std::mutex> lk(g_count_mu);
        g_count = PendingCount{self, inc};
      }
      torch::jit::drop(*stack, 3);
      stack->push_back(self);
      return;
    }
  }
  if (g_bn_epilogue.load() && args[0].isTensor() && args[1].isTensor()) {
    const at::Tensor self = args[0].toTensor();
    const at::Tensor other = args[1].toTensor();
    if (self.device().type() == kXdna && other.defined() && other.device().type() == kXdna &&
        self.scalar_type() == at::kBFloat16 && other.scalar_type() == at::kBFloat16 && args[2].toScalar().toDouble() == 1.0 &&
        other.sizes() == self.sizes() && other.strides() == self.strides() &&
        other.storage().data() != self.storage().data()) {
      auto spec = find_epilogue(self);
      if (spec && spec->foldable() && !spec->relu && !spec->residual.defined()) {
        materialize(other);
        spec->residual = other;
        add_epilogue_input(self, other);
        note_folded();
        torch::jit::drop(*stack, 3);
        stack->push_back(self);
        return;
      }
      // a gradient sum inside backward (autograd adds the two gradients of a
      // tensor used twice, e.g. a residual block's output): left pending on
      // self, so that a ReLU backward reading it sums both terms in its own
      // pass; any other reader runs the add first
      if (!spec && g_mode.load() > 1 && !at::GradMode::is_enabled() && self.dim() == 4 &&
          self.is_contiguous(at::MemoryFormat::ChannelsLast) && self.numel() >= (int64_t(1) << 20) &&
          self.numel() % 8 == 0 && (reinterpret_cast<uintptr_t>(self.data_ptr()) & 15) == 0 &&
          (reinterpret_cast<uintptr_t>(other.data_ptr()) & 15) == 0 && self.device() == other.device() &&
          !has_pending(self)) {
        materialize(other);
        auto sum = std::make_shared<EpiSpec>();
        sum->pending_sum = other;
        const auto dev = self.device().index();
        defer_epilogue(self, {other}, sum,
                       [ptr = self.data_ptr(), sizes = self.sizes().vec(), strides = self.strides().vec(), other,
                        dev]() {
                         c10::cuda::CUDAGuard guard(dev);
                         count_fallback("aten::add_.Tensor");
                         at::Tensor s = at::from_blob(ptr, sizes, strides,
                                                      at::TensorOptions().dtype(at::kBFloat16).device(at::kCUDA, dev));
                         s.add_(to_cuda(other));
                       });
        torch::jit::drop(*stack, 3);
        stack->push_back(self);
        return;
      }
    }
  }
  cuda_alias_fallback(op, stack);
}

}  // namespace

TORCH_LIBRARY_IMPL(_, PrivateUse1, m) {
  m.fallback(torch::CppFunction::makeFromBoxedFunction<&cuda_alias_fallback>());
}

// Structured ops reach a backend without kernels through a generic wrapper that
// allocates the output from the meta function and then calls the out= variant.
// For mse_loss with a reduction that wrapper hands the CUDA out= kernel a 0-dim
// output which the kernel resizes (a deprecation warning on every call); the
// functional form on the CUDA alias allocates its own output and needs one
// dispatch instead of two.
//
// The _foreach_* ops carry a CompositeExplicitAutograd kernel that a backend
// without its own kernels inherits ahead of the boxed fallback: a host loop of
// one single-tensor op per list element (an optimizer's step counters alone
// are one launch per parameter).  Routed through the CUDA aliases they reach
// ATen's CUDA multi-tensor kernels: one launch per list.
TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  const auto boxed = [] { return torch::CppFunction::makeFromBoxedFunction<&cuda_alias_fallback>(); };
  m.impl("mse_loss", boxed());
  m.impl("relu_", torch::CppFunction::makeFromBoxedFunction<&relu_inplace>());
  m.impl("add_.Tensor", torch::CppFunction::makeFromBoxedFunction<&add_inplace>());
  for (const char* op :
       {"_foreach_add_.Scalar", "_foreach_add_.List", "_foreach_add_.ScalarList", "_foreach_add_.Tensor",
        "_foreach_mul_.Scalar", "_foreach_mul_.List", "_foreach_mul_.ScalarList", "_foreach_mul_.Tensor",
        "_foreach_div_.Scalar", "_foreach_div_.List", "_foreach_div_.ScalarList", "_foreach_div_.Tensor",
        "_foreach_sub_.Scalar", "_foreach_sub_.List", "_foreach_sub_.ScalarList", "_foreach_addcmul_.Scalar",
        "_foreach_addcmul_.ScalarList", "_foreach_addcmul_.Tensor", "_foreach_addcdiv_.Scalar",
        "_foreach_addcdiv_.ScalarList", "_foreach_addcdiv_.Tensor", "_foreach_lerp_.Scalar", "_foreach_lerp_.List",
        "_foreach_lerp_.ScalarList", "_foreach_maximum_.Scalar", "_foreach_maximum_.List",
        "_foreach_maximum_.ScalarList", "_foreach_sqrt_", "_foreach_zero_", "_foreach_copy_", "_foreach_add.Scalar",
        "_foreach_add.List", "_foreach_add.ScalarList", "_foreach_add.Tensor", "_foreach_mul.Scalar",
        "_foreach_mul.List", "_foreach_mul.ScalarList", "_foreach_mul.Tensor", "_foreach_div.Scalar",
        "_foreach_div.List", "_foreach_div.ScalarList", "_foreach_div.Tensor", "_foreach_sqrt", "_foreach_neg",
        "_foreach_norm.Scalar"})
    m.impl(op, boxed());
}

}  // namespace xdna
