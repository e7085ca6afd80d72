// Device guard and PrivateUse1 hooks of the `xdna` device.
//
// Replaces XdnaGuardImpl / XdnaHooks (torch_xdna_device.cpp:872-928, 964-997):
// the reference had one device, dummy streams and a no-op synchronize; here
// `xdna:i` maps onto CUDA device i, with real CUDA streams and events.  A
// PrivateUse1 stream carries the id of the CUDA stream it stands for, so
// torch's stream/event machinery, ATen's CUDA kernels run through the
// CUDA-alias path and the b2 kernels all share one stream per device.
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAGeneratorImpl.h>
#include <ATen/cuda/PinnedMemoryAllocator.h>
#include <ATen/detail/PrivateUse1HooksInterface.h>
#include <c10/core/impl/DeviceGuardImplInterface.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAGuard.h>

#include "xdna.h"

namespace xdna {

bool record_adopted(const c10::DataPtr& ptr, cudaStream_t s);  // tensor_ops.cpp

namespace {

c10::Stream wrap(const c10::cuda::CUDAStream& s) {
  return c10::Stream(c10::Stream::UNSAFE, c10::Device(kXdna, s.device_index()), s.id());
}
c10::Stream as_cuda_stream(const c10::Stream& s) {
  return c10::Stream(c10::Stream::UNSAFE, c10::Device(c10::DeviceType::CUDA, s.device_index()), s.id());
}
c10::cuda::CUDAStream unwrap(const c10::Stream& s) { return c10::cuda::CUDAStream(as_cuda_stream(s)); }

const c10::impl::DeviceGuardImplInterface* cuda_impl() {
  return c10::impl::getDeviceGuardImpl(c10::DeviceType::CUDA);
}

struct XdnaGuardImpl final : public c10::impl::DeviceGuardImplInterface {
  XdnaGuardImpl() = default;
  c10::DeviceType type() const override { return kXdna; }
  c10::Device exchangeDevice(c10::Device d) const override {
    c10::Device old = getDevice();
    if (old.index() != d.index()) c10::cuda::set_device(d.index());
    return old;
  }
  c10::Device getDevice() const override { return c10::Device(kXdna, c10::cuda::current_device()); }
  void setDevice(c10::Device d) const override { c10::cuda::set_device(d.index()); }
  void uncheckedSetDevice(c10::Device d) const noexcept override { cudaSetDevice(d.index()); }
  c10::Stream getStream(c10::Device d) const override { return wrap(c10::cuda::getCurrentCUDAStream(d.index())); }
  c10::Stream getDefaultStream(c10::Device d) const override {
    return wrap(c10::cuda::getDefaultCUDAStream(d.index()));
  }
  c10::Stream getNewStream(c10::Device d, int priority = 0) const override {
    return wrap(c10::cuda::getStreamFromPool(priority, d.index()));
  }
  c10::Stream getStreamFromGlobalPool(c10::Device d, bool isHighPriority = false) const override {
    return wrap(c10::cuda::getStreamFromPool(isHighPriority, d.index()));
  }
  c10::Stream exchangeStream(c10::Stream s) const override {
    auto cs = unwrap(s);
    auto old = c10::cuda::getCurrentCUDAStream(s.device_index());
    c10::cuda::setCurrentCUDAStream(cs);
    return wrap(old);
  }
  c10::DeviceIndex deviceCount() const noexcept override { return c10::cuda::device_count(); }
  void record(void** event, const c10::Stream& stream, const c10::DeviceIndex device_index,
              const c10::EventFlag flag) const override {
    cuda_impl()->record(event, as_cuda_stream(stream), device_index, flag);
  }
  void block(void* event, const c10::Stream& stream) const override {
    cuda_impl()->block(event, as_cuda_stream(stream));
  }
  bool queryEvent(void* event) const override { return cuda_impl()->queryEvent(event); }
  void destroyEvent(void* event, const c10::DeviceIndex device_index) const noexcept override {
    cuda_impl()->destroyEvent(event, device_index);
  }
  bool queryStream(const c10::Stream& stream) const override {
    return cuda_impl()->queryStream(as_cuda_stream(stream));
  }
  void synchronizeStream(const c10::Stream& stream) const override {
    cuda_impl()->synchronizeStream(as_cuda_stream(stream));
  }
  void synchronizeEvent(void* event) const override { cuda_impl()->synchronizeEvent(event); }
  void synchronizeDevice(const c10::DeviceIndex device_index) const override {
    cuda_impl()->synchronizeDevice(device_index);
  }
  void recordDataPtrOnStream(const c10::DataPtr& data_ptr, const c10::Stream& stream) const override {
    cudaStream_t s = unwrap(stream).stream();
    if (!record_adopted(data_ptr, s)) record_stream(data_ptr, s);
  }
  double elapsedTime(void* event1, void* event2, const c10::DeviceIndex device_index) const override {
    return cuda_impl()->elapsedTime(event1, event2, device_index);
  }
};

struct XdnaHooks final : public at::PrivateUse1HooksInterface {
  bool isBuilt() const override { return true; }
  bool isAvailable() const override { return c10::cuda::device_count() > 0; }
  bool hasPrimaryContext(c10::DeviceIndex device_index) const override {
    return c10::cuda::hasPrimaryContext(device_index);
  }
  void init() const override {}
  c10::DeviceIndex deviceCount() const override { return c10::cuda::device_count(); }
  void setCurrentDevice(c10::DeviceIndex device) const override { c10::cuda::set_device(device); }
  c10::DeviceIndex getCurrentDevice() const override { return c10::cuda::current_device(); }
  c10::DeviceIndex exchangeDevice(c10::DeviceIndex device) const override {
    return c10::cuda::ExchangeDevice(device);
  }
  c10::DeviceIndex maybeExchangeDevice(c10::DeviceIndex device) const override {
    return c10::cuda::MaybeExchangeDevice(device);
  }
  const at::Generator& getDefaultGenerator(c10::DeviceIndex device_index) const override {
    // Random ops run as ATen CUDA kernels on aliases, so the device's
    // generator is the CUDA generator of the same index.
    return at::cuda::detail::getDefaultCUDAGenerator(device_index < 0 ? c10::cuda::current_device()
                                                                        : device_index);
  }
  at::Generator getNewGenerator(c10::DeviceIndex device_index) const override {
    return at::make_generator<at::CUDAGeneratorImpl>(device_index < 0 ? c10::cuda::current_device()
                                                                       : device_index);
  }
  at::Device getDeviceFromPtr(void* data) const override {
    cudaPointerAttributes attr{};
    XDNA_CUDA(cudaPointerGetAttributes(&attr, data));
    return at::Device(kXdna, c10::DeviceIndex(attr.device));
  }
  bool isPinnedPtr(const void* data) const override {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, data) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    return attr.type == cudaMemoryTypeHost;
  }
  at::Allocator* getPinnedMemoryAllocator() const override { return at::cuda::getPinnedMemoryAllocator(); }
  void resizePrivateUse1Bytes(const c10::Storage& storage, size_t newsize) const override;
};

XdnaHooks* g_hooks = nullptr;

}  // namespace

// Storage resize (torch.UntypedStorage.resize_ and tensor resize_): new block,
// copy the old bytes on the current stream, swap the data pointer.
void resize_storage_bytes(const c10::Storage& storage, size_t newsize) {
  c10::StorageImpl* impl = storage.unsafeGetStorageImpl();
  TORCH_CHECK(impl->resizable(), "xdna: trying to resize storage that is not resizable");
  const size_t old = impl->nbytes();
  if (old == newsize) return;
  c10::DataPtr fresh = allocator()->allocate(newsize);
  const size_t keep = std::min(old, newsize);
  if (keep && impl->data()) {
    int dev = 0;
    XDNA_CUDA(cudaGetDevice(&dev));
    XDNA_CUDA(cudaMemcpyAsync(fresh.get(), impl->data(), keep, cudaMemcpyDeviceToDevice,
                              stream(c10::DeviceIndex(dev))));
  }
  impl->set_data_ptr_noswap(std::move(fresh));
  impl->set_nbytes(newsize);
}

void XdnaHooks::resizePrivateUse1Bytes(const c10::Storage& storage, size_t newsize) const {
  resize_storage_bytes(storage, newsize);
}

C10_REGISTER_GUARD_IMPL(PrivateUse1, XdnaGuardImpl);

void register_hooks() {
  if (!g_hooks) {
    g_hooks = new XdnaHooks();
    at::RegisterPrivateUse1HooksInterface(g_hooks);
  }
}

}  // namespace xdna
