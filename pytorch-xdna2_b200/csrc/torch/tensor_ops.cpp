// Factories, views, resize/set_ and copies of `xdna` tensors, plus the two
// conversions everything else builds on: to_cuda() (a zero-copy CUDA view of
// an xdna tensor) and adopt() (an xdna tensor over a CUDA tensor's memory).
//
// Replaces torch_xdna_device.cpp:1001-1318 (factories, views, resize, set_,
// _copy_from with copies deferred behind a pending dW).  Copies here run on
// the device's current CUDA stream through ATen's CUDA copy kernels (H2D/D2H
// with pinned staging, D2D, dtype casts); a pending deferred write into the
// source or the destination is materialized first.
#include <ATen/EmptyTensor.h>
#include <ATen/native/Resize.h>
#include <ATen/native/TensorFactories.h>
#include <ATen/ops/as_strided_native.h>
#include <ATen/ops/view_native.h>
#include <ATen/ops/_reshape_alias_native.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "xdna.h"

namespace xdna {

void resize_storage_bytes(const c10::Storage& storage, size_t newsize);  // guard.cpp

cudaStream_t stream(c10::DeviceIndex device) { return c10::cuda::getCurrentCUDAStream(device).stream(); }

at::Tensor empty(at::IntArrayRef size, at::ScalarType dtype, c10::DeviceIndex device, c10::MemoryFormat mf) {
  c10::cuda::CUDAGuard g(device);
  return at::detail::empty_generic(size, allocator(), c10::DispatchKeySet(c10::DispatchKey::PrivateUse1), dtype, mf);
}

// ---- CUDA aliases and adoption ------------------------------------------------

namespace {

void noop_delete(void*) {}

struct AdoptCtx {
  c10::Storage cuda_storage;
};

void adopt_delete(void* ctx) {
  auto* c = static_cast<AdoptCtx*>(ctx);
  on_release(c->cuda_storage.mutable_data());
  delete c;
}

}  // namespace

bool record_adopted(const c10::DataPtr& ptr, cudaStream_t s) {
  if (ptr.get_deleter() != &adopt_delete) return false;
  auto* c = static_cast<AdoptCtx*>(ptr.get_context());
  c10::cuda::CUDACachingAllocator::recordStream(
      c->cuda_storage.data_ptr(),
      c10::cuda::getStreamFromExternal(s, c->cuda_storage.device().index()));
  return true;
}

at::Tensor to_cuda_nosync(const at::Tensor& t) {
  if (!t.defined() || t.device().type() != kXdna) return t;
  const c10::Storage& st = t.storage();
  const c10::DeviceIndex dev = t.device().index();
  c10::DataPtr dp(st.mutable_data(), st.mutable_data(), &noop_delete, c10::Device(c10::DeviceType::CUDA, dev));
  // Resizable through the CUDA allocator: an out= op that grows the alias gets
  // a new CUDA block, which the fallback then adopts back into the xdna tensor.
  c10::Storage cst(c10::Storage::use_byte_size_t(), st.nbytes(), std::move(dp),
                   c10::cuda::CUDACachingAllocator::get(), /*resizable=*/true);
  auto r = at::detail::make_tensor<c10::TensorImpl>(std::move(cst), c10::DispatchKeySet(c10::DispatchKey::CUDA),
                                                   t.dtype());
  r.unsafeGetTensorImpl()->set_sizes_and_strides(t.sizes(), t.strides(), t.storage_offset());
  if (t.is_conj()) r._set_conj(true);
  if (t.is_neg()) r._set_neg(true);
  return r;
}

at::Tensor to_cuda(const at::Tensor& t) {
  if (t.defined() && t.device().type() == kXdna) materialize(t);
  return to_cuda_nosync(t);
}

at::Tensor adopt(const at::Tensor& c) {
  if (!c.defined() || c.device().type() != c10::DeviceType::CUDA) return c;
  const c10::Storage& cst = c.storage();
  const c10::DeviceIndex dev = c.device().index();
  auto* ctx = new AdoptCtx{cst};
  c10::DataPtr dp(cst.mutable_data(), ctx, &adopt_delete, c10::Device(kXdna, dev));
  c10::Storage xs(c10::Storage::use_byte_size_t(), cst.nbytes(), std::move(dp), allocator(), /*resizable=*/true);
  auto r = at::detail::make_tensor<c10::TensorImpl>(std::move(xs), c10::DispatchKeySet(c10::DispatchKey::PrivateUse1),
                                                   c.dtype());
  r.unsafeGetTensorImpl()->set_sizes_and_strides(c.sizes(), c.strides(), c.storage_offset());
  if (c.is_conj()) r._set_conj(true);
  if (c.is_neg()) r._set_neg(true);
  return r;
}

namespace {

// ---- factories -------------------------------------------------------------------

c10::DeviceIndex dev_of(std::optional<c10::Device> d) {
  if (d.has_value() && d->has_index()) return d->index();
  return c10::cuda::current_device();
}

at::Tensor empty_memory_format(c10::IntArrayRef size, std::optional<at::ScalarType> dtype,
                               std::optional<at::Layout> layout, std::optional<at::Device> device,
                               std::optional<bool> pin_memory, std::optional<at::MemoryFormat> memory_format) {
  TORCH_CHECK(!pin_memory.value_or(false), "xdna: pin_memory applies to CPU tensors only");
  TORCH_CHECK(layout.value_or(at::kStrided) == at::kStrided, "xdna: only strided tensors are supported");
  const auto dt = dtype.value_or(at::get_default_dtype_as_scalartype());
  return empty(size, dt, dev_of(device), memory_format.value_or(at::MemoryFormat::Contiguous));
}

at::Tensor empty_strided(c10::IntArrayRef size, c10::IntArrayRef stride, std::optional<at::ScalarType> dtype,
                         std::optional<at::Layout> layout, std::optional<at::Device> device,
                         std::optional<bool> pin_memory) {
  TORCH_CHECK(layout.value_or(at::kStrided) == at::kStrided, "xdna: only strided tensors are supported");
  c10::cuda::CUDAGuard g(dev_of(device));
  const auto dt = dtype.value_or(at::get_default_dtype_as_scalartype());
  return at::detail::empty_strided_generic(size, stride, allocator(),
                                           c10::DispatchKeySet(c10::DispatchKey::PrivateUse1), dt);
}

// ---- resize / set_ -----------------------------------------------------------------

void ensure_storage(const at::Tensor& self, int64_t needed_elems) {
  const size_t need = size_t(needed_elems) * self.dtype().itemsize();
  c10::StorageImpl* st = self.unsafeGetTensorImpl()->unsafe_storage().unsafeGetStorageImpl();
  if (need > st->nbytes()) {
    c10::cuda::CUDAGuard g(self.device().index());
    resize_storage_bytes(self.storage(), need);
  }
}

const at::Tensor& resize_(const at::Tensor& self, c10::SymIntArrayRef size_sym,
                          std::optional<at::MemoryFormat> memory_format) {
  auto size = C10_AS_INTARRAYREF_SLOW(size_sym);
  materialize(self);
  auto* impl = self.unsafeGetTensorImpl();
  impl->set_sizes_contiguous(size);
  const auto mf = memory_format.value_or(at::MemoryFormat::Contiguous);
  if (mf != at::MemoryFormat::Preserve) impl->empty_tensor_restride(mf);
  if (impl->numel() > 0) ensure_storage(self, impl->storage_offset() + impl->numel());
  return self;
}

at::Tensor& set_storage(at::Tensor& self, c10::Storage source, c10::SymInt offset_sym, c10::SymIntArrayRef size_sym,
                        c10::SymIntArrayRef stride_sym) {
  const int64_t offset = offset_sym.expect_int();
  auto size = C10_AS_INTARRAYREF_SLOW(size_sym);
  auto stride = C10_AS_INTARRAYREF_SLOW(stride_sym);
  materialize(self);
  auto* impl = self.unsafeGetTensorImpl();
  impl->set_storage_keep_dtype(std::move(source));
  impl->set_storage_offset(offset);
  std::vector<int64_t> st(stride.begin(), stride.end());
  if (st.empty() && !size.empty()) {
    auto cs = c10::contiguous_strides(size);
    st.assign(cs.begin(), cs.end());
  }
  impl->set_sizes_and_strides(size, st);
  int64_t max_off = offset;
  bool empty_t = false;
  for (size_t i = 0; i < size.size(); ++i) {
    if (size[i] == 0) empty_t = true;
    max_off += (size[i] - 1) * st[i];
  }
  if (!empty_t) ensure_storage(self, max_off + 1);
  return self;
}

at::Tensor& set_source_storage(at::Tensor& self, c10::Storage source) {
  const int64_t n = int64_t(source.nbytes() / self.dtype().itemsize());
  std::vector<c10::SymInt> sz{c10::SymInt(n)}, st{c10::SymInt(1)};
  return set_storage(self, std::move(source), 0, sz, st);
}

at::Tensor& set_source_tensor(at::Tensor& self, const at::Tensor& src) {
  if (self.is_same(src)) return self;
  std::vector<c10::SymInt> sz(src.sym_sizes().begin(), src.sym_sizes().end());
  std::vector<c10::SymInt> st(src.sym_strides().begin(), src.sym_strides().end());
  return set_storage(self, src.storage(), src.sym_storage_offset(), sz, st);
}

at::Tensor& set_empty(at::Tensor& self) {
  c10::Storage s(c10::Storage::use_byte_size_t(), 0, allocator()->allocate(0), allocator(), true);
  std::vector<c10::SymInt> sz{c10::SymInt(0)}, st{};
  return set_storage(self, std::move(s), 0, sz, st);
}

// ---- copies ----------------------------------------------------------------------------

at::Tensor copy_from(const at::Tensor& self, const at::Tensor& dst, bool non_blocking) {
  if (dst.device().type() == kXdna) {
    before_write(dst);
    note_write(dst);
  }
  // self -> dst; at least one of them is on xdna.
  const bool src_x = self.device().type() == kXdna;
  const bool dst_x = dst.device().type() == kXdna;
  if (dst_x) materialize(dst);
  at::Tensor s = src_x ? to_cuda(self) : self;
  at::Tensor d = dst_x ? to_cuda_nosync(dst) : dst;
  {
    c10::cuda::OptionalCUDAGuard g;
    if (dst_x) g.set_index(dst.device().index());
    else if (src_x) g.set_index(self.device().index());
    d.copy_(s, non_blocking);
  }
  count_launch("copy");
  return dst;
}

at::Tensor copy_from_and_resize(const at::Tensor& self, const at::Tensor& dst) {
  if (dst.sizes() != self.sizes()) {
    if (dst.device().type() == kXdna) {
      std::vector<c10::SymInt> sz(self.sym_sizes().begin(), self.sym_sizes().end());
      resize_(dst, sz, std::nullopt);
    } else {
      dst.resize_(self.sizes());
    }
  }
  return copy_from(self, dst, false);
}

at::Tensor as_strided(const at::Tensor& self, c10::SymIntArrayRef size, c10::SymIntArrayRef stride,
                      std::optional<c10::SymInt> storage_offset) {
  return at::native::as_strided_tensorimpl(self, C10_AS_INTARRAYREF_SLOW(size), C10_AS_INTARRAYREF_SLOW(stride),
                                           storage_offset.has_value()
                                               ? std::optional<int64_t>(storage_offset->expect_int())
                                               : std::nullopt);
}

at::Tensor view(const at::Tensor& self, c10::SymIntArrayRef size) {
  return at::native::view(self, C10_AS_INTARRAYREF_SLOW(size));
}

at::Tensor reshape_alias(const at::Tensor& self, c10::SymIntArrayRef size, c10::SymIntArrayRef stride) {
  return at::native::_reshape_alias(self, C10_AS_INTARRAYREF_SLOW(size), C10_AS_INTARRAYREF_SLOW(stride));
}

}  // namespace

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("empty.memory_format", empty_memory_format);
  m.impl("empty_strided", empty_strided);
  m.impl("as_strided", as_strided);
  m.impl("view", view);
  m.impl("_reshape_alias", reshape_alias);
  m.impl("resize_", resize_);
  m.impl("set_.source_Storage_storage_offset", set_storage);
  m.impl("set_.source_Storage", set_source_storage);
  m.impl("set_.source_Tensor", set_source_tensor);
  m.impl("set_", set_empty);
  m.impl("_copy_from", copy_from);
  m.impl("_copy_from_and_resize", copy_from_and_resize);
}

}  // namespace xdna
