// Shared declarations of the `xdna` PrivateUse1 backend (B200 edition).
//
// The device is a CUDA device under another name: `xdna:i` is `cuda:i`, its
// streams and events are CUDA streams and events, its storage is HBM from a
// stream-ordered caching allocator, and the hot ops run the sm_100a kernels of
// libxdna_b200.so (include/b2.h).  Everything else runs ATen's CUDA kernels on
// zero-copy CUDA aliases of the same memory (the B200 counterpart of the
// reference's zero-copy CPU fallback, torch_xdna_device.cpp:5117-5260).
#pragma once

#include <ATen/ATen.h>
#include <c10/core/Allocator.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime_api.h>

#include <atomic>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>

#include "b2.h"

namespace xdna {

constexpr c10::DeviceType kXdna = c10::DeviceType::PrivateUse1;

// ---- errors ------------------------------------------------------------
#define XDNA_B2(call)                                                              \
  do {                                                                             \
    b2_status _st = (call);                                                        \
    TORCH_CHECK(_st == B2_OK, "xdna: ", #call, " failed (", _st, "): ", b2_last_error()); \
  } while (0)

#define XDNA_CUDA(call)                                                            \
  do {                                                                             \
    cudaError_t _e = (call);                                                       \
    TORCH_CHECK(_e == cudaSuccess, "xdna: ", #call, ": ", cudaGetErrorString(_e)); \
  } while (0)

// ---- allocator (allocator.cpp) -------------------------------------------
c10::Allocator* allocator();
void record_stream(const c10::DataPtr& ptr, cudaStream_t stream);
void empty_cache();
std::map<std::string, int64_t> allocator_stats();
// CUDA graph capture: allocations on `stream` come from a private pool until
// graph_capture_end; a pool (returned id; share_pool > 0 reuses one) stays
// reserved for its graphs until graph_pool_release.
int graph_capture_begin(int device, cudaStream_t stream, int share_pool);
void graph_capture_end(cudaStream_t stream);
void graph_pool_release(int pool);
// Called by the allocator when a block is released; drops deferred work and
// packed-operand attachments keyed on that address.
void on_release(void* ptr);

// ---- tensors / streams (tensor_ops.cpp) -----------------------------------
cudaStream_t stream(c10::DeviceIndex device);  // current CUDA stream of xdna:device
at::Tensor empty(at::IntArrayRef size, at::ScalarType dtype, c10::DeviceIndex device,
                 c10::MemoryFormat mf = c10::MemoryFormat::Contiguous);
// Zero-copy CUDA view of an xdna tensor (same bytes, sizes, strides, offset).
// Materializes deferred writes into that storage first.
at::Tensor to_cuda(const at::Tensor& t);
at::Tensor to_cuda_nosync(const at::Tensor& t);
// xdna tensor over the memory of a CUDA tensor (the xdna storage keeps the
// CUDA storage alive).
at::Tensor adopt(const at::Tensor& cuda_tensor);

// ---- deferred weight gradients (deferred.cpp) -----------------------------
// A job produces the contents of one storage.  Readers run it first; freeing
// the storage before anyone read it drops it unrun (reference semantics,
// torch_xdna_device.cpp:299-482, 550-656).
// kick = false keeps the job out of the async policy's early launch (a
// producer whose whole point is to wait for a reader that may never come).
void defer_write(const at::Tensor& target, std::function<void()> job, bool kick = true);
void materialize(const at::Tensor& t);  // no-op unless t's storage has a pending job
// t's pending job and tails dropped unrun: its contents were written by a
// kernel that fused the job's work into its own pass
void drop_pending(const at::Tensor& t);
void materialize_all();
bool has_pending(const at::Tensor& t);
void note_dgrad();           // one dX computed (async policy bookkeeping)
void note_optimizer_step();  // step boundary
std::map<std::string, int64_t> deferred_stats();
extern std::atomic<int64_t> g_pending_jobs;

// Packed padded-grid rows of a conv input, attached to the input's storage by
// the forward so the weight gradient reuses them (reference: packed X attached
// to the allocation, torch_xdna_device.cpp:1968-1985).
void attach_rows(const at::Tensor& input, const at::Tensor& rows);
at::Tensor find_rows(const at::Tensor& input);

// A BatchNorm output pass that folded a relu_ and no residual: its output y
// is relu(bf16(x*scale + shift)), so the ReLU's gate can be recomputed from
// the BatchNorm's input and parameters (b2_batch_norm_relu_bwd_bf16).
struct GateSource {
  at::Tensor x, w, b, stats;  // stats: [2][C] fp32 (save_mean, save_invstd)
  int64_t x_version = 0, w_version = 0, b_version = 0;
  int pdtype = 0;
};
// Fused tails of a deferred producer (a BatchNorm whose output pass waits for
// its first reader): the in-place ops that follow it on exactly its output
// tensor (a residual add_, then a relu_) fold into that pass instead of
// running as passes of their own.  Readers materialize it as any deferred
// write; a write into a storage it reads (before_write: the CUDA-alias
// fallback, copies, out= and fused optimizer ops call it first) runs it
// before the write lands.
struct EpiSpec {
  at::Tensor residual;
  bool relu = false;
  // a pending ReLU input gradient (threshold_backward(grad, y, 0) with y a
  // gated BatchNorm output): its BatchNorm's backward reads `grad` and
  // recomputes the gate instead of running the pass; nothing folds into it
  at::Tensor gate_grad;
  std::shared_ptr<GateSource> gate;
  // a pending in-place sum (self += pending_sum, both bf16, same layout):
  // a ReLU backward on it reads both terms and sums them in its own pass
  // (b2_relu_bwd_sum_bf16); nothing folds into it
  at::Tensor pending_sum;
  // a pending ReLU backward of a pending sum: dz = gate(relu_sum_y) ?
  // bf16(relu_sum_a + relu_sum_b) : 0, relu_sum_a still holding its pre-add
  // values while its own sum is pending; the BatchNorm backward that reads dz
  // makes, writes and reduces it in one pass
  // (b2_batch_norm_bwd_relu_sum_bf16)
  at::Tensor relu_sum_a, relu_sum_b, relu_sum_y;
  // add_ / relu_ may fold into this pending output: only a BatchNorm's pass
  bool foldable() const { return !gate && !pending_sum.defined() && !relu_sum_a.defined(); }
};
// The gated BatchNorm output y (registered when its output pass is enqueued;
// dropped when y's storage is released) and its lookup by exact geometry.
void note_gate_source(void* storage_data, std::vector<int64_t> sizes, std::vector<int64_t> strides, int64_t offset,
                      std::shared_ptr<GateSource> src);
std::shared_ptr<GateSource> find_gate_source(const at::Tensor& y);
void defer_epilogue(const at::Tensor& out, const std::vector<at::Tensor>& inputs, std::shared_ptr<EpiSpec> spec,
                    std::function<void()> job);
std::shared_ptr<EpiSpec> find_epilogue(const at::Tensor& t);  // t is exactly a pending output
void add_epilogue_input(const at::Tensor& out, const at::Tensor& input);
void note_folded();  // an op folded into a pending output pass (async_dw_stats "folded_tails")
void before_write(const at::Tensor& t);
extern std::atomic<bool> g_bn_epilogue;  // fold add_ / relu_ into BatchNorm's output pass

// Packed GEMM-operand forms of frozen weights (the reference's weight-encode
// cache keyed on pointer, version counter and write epoch,
// torch_xdna_device.cpp:2200-2271): found while the weight's version, geometry
// and storage are unchanged; any write into the storage through this backend
// (note_write: the CUDA-alias fallback, copies, out= and fused optimizer ops)
// and the storage's release drop them.
at::Tensor find_packed_weight(const at::Tensor& w, int kind);
void attach_packed_weight(const at::Tensor& w, int kind, const at::Tensor& packed);
void note_write(const at::Tensor& t);

// ---- modes and counters (module.cpp) --------------------------------------
// 2: all hot-path kernels; 1: weight gradients through the CUDA-alias path;
// 0: every hot op through the CUDA-alias path (A/B switch, set_npu_mode).
extern std::atomic<int> g_mode;
// Convolutions outside the 3x3 fast path: 1x1 GEMMs / column-matrix GEMMs
// (conv_ops.cpp); off sends them to ATen's CUDA kernels.
extern std::atomic<bool> g_conv1x1;
extern std::atomic<bool> g_conv_general;
void count_launch(const char* what, int64_t n = 1);

// Per-launch device timing for measurements (the bench's roofline): while
// enabled, a KernelTimer placed around a launch records a CUDA event before
// and after it on the launching stream, with the launch's algorithmic work
// (FLOPs or bytes).  kernel_timer_read() waits for the recorded events and
// returns, per label, the launches, the summed device milliseconds and the
// summed work.  Off by default (one atomic load per launch site); launches on
// a capturing stream are not timed.
void kernel_timer_enable(bool on);
bool kernel_timer_enabled();
struct KernelTimerRead {
  int64_t launches = 0;
  double ms = 0, work = 0;
};
std::map<std::string, KernelTimerRead> kernel_timer_read();
class KernelTimer {
 public:
  KernelTimer(const char* label, double work, cudaStream_t stream);
  ~KernelTimer();
  KernelTimer(const KernelTimer&) = delete;
  KernelTimer& operator=(const KernelTimer&) = delete;

 private:
  const char* label_;
  double work_;
  cudaStream_t stream_;
  cudaEvent_t start_ = nullptr;
};
void count_fallback(const std::string& op);

// ---- a module's step counter left pending (fallback.cpp) -------------------
// `counter.add_(k)` on an xdna int64 scalar with a host integer k (a training
// BatchNorm's num_batches_tracked.add_(1)) is deferred like any write: a reader
// runs it first.  The next training BatchNorm forward on that device takes it
// (take_pending_count: the job dropped, the counter and k handed over) and
// advances the counter inside its statistics launch.  flush_pending_count
// runs a pending one now (the end of a graph capture).
struct PendingCount {
  at::Tensor counter;
  int64_t inc = 0;
};
PendingCount take_pending_count(c10::DeviceIndex dev);
void flush_pending_count();
std::map<std::string, int64_t> launch_stats();
std::map<std::string, int64_t> fallback_stats();
void reset_stats();

}  // namespace xdna
