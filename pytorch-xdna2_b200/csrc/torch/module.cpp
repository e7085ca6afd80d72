// Python module `xdna_train._C`: device queries, modes, statistics, the
// deferred-gradient controls, CUDA aliases for NCCL, and the region kernels.
// Mirrors the reference's pybind surface (torch_xdna_device.cpp:5346-5767) for
// the functions the hot path and xdna_train's Python API use.
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include "xdna.h"

namespace xdna {

void register_hooks();  // guard.cpp

std::atomic<int> g_mode{[] {
  const char* s = std::getenv("XDNA_NPU_MODE");
  return s ? std::atoi(s) : 2;
}()};

namespace {
std::mutex g_stat_mu;
std::map<std::string, int64_t> g_launches, g_fallbacks;
}  // namespace

void count_launch(const char* what, int64_t n) {
  std::lock_guard<std::mutex> lk(g_stat_mu);
  g_launches[what] += n;
}
void count_fallback(const std::string& op) {
  std::lock_guard<std::mutex> lk(g_stat_mu);
  g_fallbacks[op] += 1;
}
std::map<std::string, int64_t> launch_stats() {
  std::lock_guard<std::mutex> lk(g_stat_mu);
  return g_launches;
}
std::map<std::string, int64_t> fallback_stats() {
  std::lock_guard<std::mutex> lk(g_stat_mu);
  return g_fallbacks;
}
void reset_stats() {
  std::lock_guard<std::mutex> lk(g_stat_mu);
  g_launches.clear();
  g_fallbacks.clear();
}

namespace {
std::atomic<bool> g_timer_on{false};
struct TimedLaunch {
  std::string label;
  double work;
  int device;
  cudaEvent_t start, end;
};
std::mutex g_timer_mu;
std::vector<TimedLaunch> g_timed;
std::map<int, std::vector<cudaEvent_t>> g_event_pool;  // per device, for reuse

cudaEvent_t timer_event(int device) {
  {
    std::lock_guard<std::mutex> lk(g_timer_mu);
    auto& pool = g_event_pool[device];
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
  }
  cudaEvent_t e = nullptr;
  XDNA_CUDA(cudaEventCreate(&e));
  return e;
}

bool capturing(cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  return cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone;
}
}  // namespace

void kernel_timer_enable(bool on) { g_timer_on.store(on); }
bool kernel_timer_enabled() { return g_timer_on.load(); }

KernelTimer::KernelTimer(const char* label, double work, cudaStream_t stream)
    : label_(label), work_(work), stream_(stream) {
  if (!g_timer_on.load(std::memory_order_relaxed) || capturing(stream)) return;
  int dev = 0;
  XDNA_CUDA(cudaGetDevice(&dev));
  start_ = timer_event(dev);
  XDNA_CUDA(cudaEventRecord(start_, stream_));
}

KernelTimer::~KernelTimer() {
  if (!start_) return;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  cudaEvent_t end = timer_event(dev);
  if (cudaEventRecord(end, stream_) != cudaSuccess) return;
  std::lock_guard<std::mutex> lk(g_timer_mu);
  g_timed.push_back({label_, work_, dev, start_, end});
}

std::map<std::string, KernelTimerRead> kernel_timer_read() {
  std::vector<TimedLaunch> recs;
  {
    std::lock_guard<std::mutex> lk(g_timer_mu);
    recs.swap(g_timed);
  }
  std::map<std::string, KernelTimerRead> out;
  for (auto& r : recs) {
    XDNA_CUDA(cudaEventSynchronize(r.end));
    float ms = 0.f;
    XDNA_CUDA(cudaEventElapsedTime(&ms, r.start, r.end));
    auto& o = out[r.label];
    o.launches += 1;
    o.ms += ms;
    o.work += r.work;
    std::lock_guard<std::mutex> lk(g_timer_mu);
    g_event_pool[r.device].push_back(r.start);
    g_event_pool[r.device].push_back(r.end);
  }
  return out;
}

namespace {

void check_bf16(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.device().type() == kXdna && t.scalar_type() == at::kBFloat16 && t.is_contiguous(),
              "xdna region kernel: ", what, " must be a contiguous bf16 xdna tensor");
}
const void* opt_ptr(const std::optional<at::Tensor>& t, const char* what) {
  if (!t.has_value() || !t->defined()) return nullptr;
  check_bf16(*t, what);
  materialize(*t);
  return t->data_ptr();
}

double region_sqdiff_sum(const at::Tensor& a, const at::Tensor& b) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  TORCH_CHECK(a.numel() == b.numel(), "region_sqdiff_sum: size mismatch");
  materialize(a);
  materialize(b);
  c10::cuda::CUDAGuard g(a.device().index());
  at::Tensor acc = empty({1}, at::kDouble, a.device().index());
  XDNA_B2(b2_region_sqdiff_sum_bf16(a.data_ptr(), b.data_ptr(), a.numel(), acc.data_ptr<double>(),
                                    stream(a.device().index())));
  count_launch("region.sqdiff_sum");
  return to_cuda(acc).item<double>();
}

// Same sum as region_sqdiff_sum, left on the device (0-dim double xdna tensor):
// no host synchronization inside a training step.
at::Tensor region_sqdiff_sum_tensor(const at::Tensor& a, const at::Tensor& b) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  TORCH_CHECK(a.numel() == b.numel(), "region_sqdiff_sum: size mismatch");
  materialize(a);
  materialize(b);
  c10::cuda::CUDAGuard g(a.device().index());
  at::Tensor acc = empty({}, at::kDouble, a.device().index());
  XDNA_B2(b2_region_sqdiff_sum_bf16(a.data_ptr(), b.data_ptr(), a.numel(), acc.data_ptr<double>(),
                                    stream(a.device().index())));
  count_launch("region.sqdiff_sum");
  return acc;
}

void region_relu(const at::Tensor& a, const at::Tensor& r) {
  check_bf16(a, "a");
  check_bf16(r, "r");
  materialize(a);
  c10::cuda::CUDAGuard g(a.device().index());
  XDNA_B2(b2_region_relu_bf16(a.data_ptr(), r.data_ptr(), a.numel(), stream(a.device().index())));
  count_launch("region.relu");
}

void region_relu_maxpool2(const at::Tensor& a, const at::Tensor& r, const at::Tensor& p) {
  check_bf16(a, "a");
  check_bf16(r, "r");
  check_bf16(p, "p");
  TORCH_CHECK(a.dim() == 4, "region_relu_maxpool2: NCHW input expected");
  materialize(a);
  c10::cuda::CUDAGuard g(a.device().index());
  XDNA_B2(b2_region_relu_maxpool2_bf16(a.data_ptr(), r.data_ptr(), p.data_ptr(), a.size(0) * a.size(1), a.size(2),
                                       a.size(3), stream(a.device().index())));
  count_launch("region.relu_maxpool2");
}

void region_addtap(const std::optional<at::Tensor>& base, const at::Tensor& a, const at::Tensor& b,
                   const at::Tensor& out, double scale) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_bf16(out, "out");
  materialize(a);
  materialize(b);
  c10::cuda::CUDAGuard g(a.device().index());
  XDNA_B2(b2_region_addtap_bf16(opt_ptr(base, "base"), a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(),
                                float(scale), stream(a.device().index())));
  count_launch("region.addtap");
}

void region_relu_bwd(const at::Tensor& r, const std::optional<at::Tensor>& base, const std::optional<at::Tensor>& a,
                     const std::optional<at::Tensor>& b, const at::Tensor& out, double scale) {
  check_bf16(r, "r");
  check_bf16(out, "out");
  materialize(r);
  c10::cuda::CUDAGuard g(r.device().index());
  XDNA_B2(b2_region_relu_bwd_bf16(r.data_ptr(), opt_ptr(base, "base"), opt_ptr(a, "a"), opt_ptr(b, "b"),
                                  out.data_ptr(), r.numel(), float(scale), stream(r.device().index())));
  count_launch("region.relu_bwd");
}

void region_maxpool2_bwd(const at::Tensor& x, const at::Tensor& gr, const at::Tensor& out) {
  check_bf16(x, "x");
  check_bf16(gr, "g");
  check_bf16(out, "out");
  TORCH_CHECK(x.dim() == 4, "region_maxpool2_bwd: NCHW input expected");
  materialize(x);
  materialize(gr);
  c10::cuda::CUDAGuard g(x.device().index());
  XDNA_B2(b2_region_maxpool2_bwd_bf16(x.data_ptr(), gr.data_ptr(), out.data_ptr(), x.size(0) * x.size(1), x.size(2),
                                      x.size(3), stream(x.device().index())));
  count_launch("region.maxpool2_bwd");
}

void check_f32(const at::Tensor& t, int64_t n, const char* what) {
  TORCH_CHECK(t.device().type() == kXdna && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == n,
              "xdna region kernel: ", what, " must be a contiguous fp32 xdna tensor of ", n, " elements");
}

at::Tensor bn_workspace(int64_t N, int64_t C, c10::DeviceIndex dev) {
  const int64_t bytes = int64_t(b2_region_bn_workspace_bytes(N, C));
  return empty({std::max<int64_t>(bytes, 16)}, at::kByte, dev);
}

// Fused training BatchNorm2d + LeakyReLU/ReLU forward on contiguous NCHW bf16
// (the reference's region_bn_fwd binding, torch_xdna_device.cpp:5521-5550).
void region_bn_fwd(const at::Tensor& x, const std::optional<at::Tensor>& w, const std::optional<at::Tensor>& b,
                   const std::optional<at::Tensor>& rm, const std::optional<at::Tensor>& rv, const at::Tensor& y,
                   const at::Tensor& mean, const at::Tensor& invstd, double eps, double slope, double factor,
                   bool update) {
  check_bf16(x, "x");
  check_bf16(y, "y");
  TORCH_CHECK(x.dim() >= 2 && y.sizes() == x.sizes(), "region_bn_fwd: x and y must be [N, C, ...] of one shape");
  const int64_t N = x.size(0), C = x.size(1), HW = C ? x.numel() / std::max<int64_t>(1, N * C) : 0;
  check_f32(mean, C, "mean");
  check_f32(invstd, C, "invstd");
  for (const auto* t : {&w, &b, &rm, &rv})
    if (t->has_value() && (*t)->defined())
      TORCH_CHECK((*t)->numel() == C, "region_bn_fwd: per-channel tensors must have C elements");
  TORCH_CHECK(!update || (rm.has_value() && rv.has_value()), "region_bn_fwd: update needs running statistics");
  materialize(x);
  const auto dev = x.device().index();
  c10::cuda::CUDAGuard g(dev);
  at::Tensor ws = bn_workspace(N, C, dev);
  XDNA_B2(b2_region_bn_fwd_bf16(x.data_ptr(), opt_ptr(w, "weight"), opt_ptr(b, "bias"),
                                const_cast<void*>(opt_ptr(rm, "running_mean")),
                                const_cast<void*>(opt_ptr(rv, "running_var")), y.data_ptr(),
                                mean.data_ptr<float>(), invstd.data_ptr<float>(), N, C, HW, float(eps), float(slope),
                                float(factor), update ? 1 : 0, ws.data_ptr(), size_t(ws.numel()), stream(dev)));
  count_launch("region.bn_fwd", 3);
}

// Backward of the fused pair: dx, dw, db each optional (region_bn_bwd,
// torch_xdna_device.cpp:5552-5580).
void region_bn_bwd(const at::Tensor& dy, const at::Tensor& y, const at::Tensor& x, const std::optional<at::Tensor>& w,
                   const at::Tensor& mean, const at::Tensor& invstd, const std::optional<at::Tensor>& dx,
                   const std::optional<at::Tensor>& dw, const std::optional<at::Tensor>& db, double slope,
                   bool relu) {
  check_bf16(dy, "dy");
  check_bf16(y, "y");
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() >= 2 && dy.sizes() == x.sizes() && y.sizes() == x.sizes(),
              "region_bn_bwd: dy, y and x must be [N, C, ...] of one shape");
  const int64_t N = x.size(0), C = x.size(1), HW = C ? x.numel() / std::max<int64_t>(1, N * C) : 0;
  check_f32(mean, C, "mean");
  check_f32(invstd, C, "invstd");
  auto out_ptr = [&](const std::optional<at::Tensor>& t, int64_t n, const char* what) -> void* {
    if (!t.has_value() || !t->defined()) return nullptr;
    check_bf16(*t, what);
    TORCH_CHECK(t->numel() == n, "region_bn_bwd: ", what, " has the wrong size");
    return t->data_ptr();
  };
  void* pdx = out_ptr(dx, x.numel(), "dx");
  void* pdw = out_ptr(dw, C, "dw");
  void* pdb = out_ptr(db, C, "db");
  materialize(dy);
  materialize(y);
  materialize(x);
  const auto dev = x.device().index();
  c10::cuda::CUDAGuard g(dev);
  at::Tensor ws = bn_workspace(N, C, dev);
  XDNA_B2(b2_region_bn_bwd_bf16(dy.data_ptr(), y.data_ptr(), x.data_ptr(), opt_ptr(w, "weight"),
                                mean.data_ptr<float>(), invstd.data_ptr<float>(), pdx, pdw, pdb, N, C, HW,
                                float(slope), relu ? 1 : 0, ws.data_ptr(), size_t(ws.numel()), stream(dev)));
  count_launch("region.bn_bwd", pdx ? 3 : 2);
}

// Allocating forms used by regions._BatchNormAct: one binding call per
// direction.  region_bn_forward returns (y, stats) with stats = [mean; invstd]
// as fp32 [2, C]; region_bn_backward returns (dx, dw, db), None where not
// requested.
std::tuple<at::Tensor, at::Tensor> region_bn_forward(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b,
                                                     const at::Tensor& rm, const at::Tensor& rv, double eps,
                                                     double slope, double factor) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() >= 2, "region_bn_forward: x must be [N, C, ...]");
  const auto dev = x.device().index();
  at::Tensor y = empty(x.sizes(), at::kBFloat16, dev);
  at::Tensor stats = empty({2, x.size(1)}, at::kFloat, dev);
  region_bn_fwd(x, w, b, rm, rv, y, stats[0], stats[1], eps, slope, factor, true);
  return {y, stats};
}

py::tuple region_bn_backward(const at::Tensor& dy, const at::Tensor& y, const at::Tensor& x, const at::Tensor& w,
                             const at::Tensor& stats, bool want_x, bool want_w, bool want_b, double slope,
                             bool relu) {
  const auto dev = x.device().index();
  const int64_t C = x.dim() >= 2 ? x.size(1) : 0;
  std::optional<at::Tensor> dx, dw, db;
  if (want_x) dx = empty(x.sizes(), at::kBFloat16, dev);
  if (want_w) dw = empty({C}, at::kBFloat16, dev);
  if (want_b) db = empty({C}, at::kBFloat16, dev);
  const at::Tensor g = dy.is_contiguous() ? dy : dy.contiguous();
  region_bn_bwd(g, y, x, w, stats[0], stats[1], dx, dw, db, slope, relu);
  auto as_py = [](const std::optional<at::Tensor>& t) { return t ? py::cast(*t) : py::none(); };
  return py::make_tuple(as_py(dx), as_py(dw), as_py(db));
}

py::dict to_dict(const std::map<std::string, int64_t>& m) {
  py::dict d;
  for (auto& kv : m) d[py::str(kv.first)] = kv.second;
  return d;
}

}  // namespace
}  // namespace xdna

PYBIND11_MODULE(_C, m) {
  using namespace xdna;
  register_hooks();
  m.doc() = "xdna device on NVIDIA B200 (PrivateUse1 over CUDA, sm_100a kernels in libxdna_b200.so)";
  m.def("abi_version", [] { return b2_abi_version(); });
  m.def("is_available", [] { return c10::cuda::device_count() > 0; });
  m.def("device_count", [] { return int(c10::cuda::device_count()); });
  m.def("current_device", [] { return int(c10::cuda::current_device()); });
  m.def("set_device", [](int d) { c10::cuda::set_device(c10::DeviceIndex(d)); });
  m.def(
      "synchronize",
      [](int d) {
        py::gil_scoped_release nogil;
        if (d < 0) d = c10::cuda::current_device();
        c10::cuda::CUDAGuard g(c10::DeviceIndex(d));
        XDNA_CUDA(cudaDeviceSynchronize());
      },
      py::arg("device") = -1);
  m.def("empty_cache", [] {
    empty_cache();
    c10::cuda::CUDACachingAllocator::emptyCache();
  });
  m.def("allocator_stats", [] { return to_dict(allocator_stats()); });
  m.def("graph_capture_begin", [](int device, uintptr_t stream, int share_pool) {
    return graph_capture_begin(device, reinterpret_cast<cudaStream_t>(stream), share_pool);
  });
  m.def("graph_capture_end", [](uintptr_t stream) {
    // a step counter still pending advances inside the capture, so that each
    // replay advances it; after a failed capture there is nothing to keep
    try {
      flush_pending_count();
    } catch (const std::exception&) {
    }
    graph_capture_end(reinterpret_cast<cudaStream_t>(stream));
  });
  m.def("graph_pool_release", [](int pool) { graph_pool_release(pool); });
  m.def("set_bn_epilogue", [](bool on) { return g_bn_epilogue.exchange(on); });
  m.def("bn_epilogue", [] { return g_bn_epilogue.load(); });
  m.def("fallback_stats", [] {
    py::dict d;
    for (auto& kv : fallback_stats()) {
      py::dict e;
      e["calls"] = kv.second;
      d[py::str(kv.first)] = e;
    }
    return d;
  });
  m.def("launch_stats", [] { return to_dict(launch_stats()); });
  m.def("kernel_timer_enable", [](bool on) { kernel_timer_enable(on); });
  m.def("kernel_timer_read", [] {
    std::map<std::string, KernelTimerRead> r;
    {
      py::gil_scoped_release nogil;
      r = kernel_timer_read();
    }
    py::dict d;
    for (auto& kv : r) {
      py::dict e;
      e["launches"] = kv.second.launches;
      e["ms"] = kv.second.ms;
      e["work"] = kv.second.work;
      d[py::str(kv.first)] = e;
    }
    return d;
  });
  m.def("reset_stats", [] { reset_stats(); });
  m.def("set_npu_mode", [](int mode) {
    TORCH_CHECK(mode >= 0 && mode <= 2, "npu mode must be 0, 1 or 2");
    g_mode.store(mode);
  });
  m.def("npu_mode", [] { return g_mode.load(); });
  m.def("async_dw_stats", [] { return to_dict(deferred_stats()); });
  m.def("materialize", [](const at::Tensor& t) { materialize(t); });
  m.def("materialize_all", [] { materialize_all(); });
  m.def("has_pending", [](const at::Tensor& t) { return has_pending(t); });
  m.def("optimizer_step_boundary", [] { note_optimizer_step(); });
  m.def("as_cuda", [](const at::Tensor& t) {
    TORCH_CHECK(t.device().type() == kXdna, "as_cuda: expected an xdna tensor");
    return to_cuda(t);
  });
  m.def("adopt", [](const at::Tensor& t) {
    TORCH_CHECK(t.device().type() == c10::DeviceType::CUDA, "adopt: expected a CUDA tensor");
    return adopt(t);
  });
  m.def("device_status", [](int d) {
    int code = 0;
    XDNA_B2(b2_device_status(d, &code));
    return code;
  });
  m.def("region_sqdiff_sum", &region_sqdiff_sum);
  m.def("region_sqdiff_sum_tensor", &region_sqdiff_sum_tensor);
  m.def("region_relu", &region_relu);
  m.def("region_relu_maxpool2", &region_relu_maxpool2);
  m.def("region_addtap", &region_addtap);
  m.def("region_relu_bwd", &region_relu_bwd);
  m.def("region_maxpool2_bwd", &region_maxpool2_bwd);
  m.def("set_conv_paths", [](std::optional<bool> conv1x1, std::optional<bool> general) {
    if (conv1x1) xdna::g_conv1x1.store(*conv1x1);
    if (general) xdna::g_conv_general.store(*general);
    return py::make_tuple(xdna::g_conv1x1.load(), xdna::g_conv_general.load());
  }, py::arg("conv1x1") = py::none(), py::arg("general") = py::none());
  m.def("region_bn_fwd", &region_bn_fwd);
  m.def("region_bn_bwd", &region_bn_bwd);
  m.def("region_bn_forward", &region_bn_forward);
  m.def("region_bn_backward", &region_bn_backward);
}
