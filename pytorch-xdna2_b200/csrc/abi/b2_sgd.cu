// Multi-tensor fused SGD (momentum, dampening, Nesterov, weight decay,
// maximize, grad scaling / inf skipping): the update `torch.optim.SGD(...,
// fused=True)` issues as aten::_fused_sgd_.  The reference reaches that op's
// CPU kernel through its boxed fallback and _prefer_fused_optimizer
// (xdna_train/device.py:408-436, torch_xdna_device.cpp:5124-5260); here it is
// one memory-bound pass per element over param, grad and momentum buffer.
//
// Arithmetic: PyTorch's fused-SGD definition with fp32 operands and the
// scalar hyper-parameters in double, each intermediate rounded where that
// definition stores it (to fp32 for the gradient, to the parameter dtype on
// store):
//   g = grad                       (grad_scale: g = fp32(g / scale), stored back)
//   maximize: g = -g
//   wd != 0: g = fp32(g + wd * p)
//   momentum != 0: b = first_step ? g : momentum * buf + (1 - dampening) * g   (double)
//                  buf <- b;  g = fp32(nesterov ? g + momentum * b : b)
//   p <- fp32(p - lr * g)
// A buffer or parameter stored as bf16 goes double -> fp32 -> bf16 (round to
// nearest even at each step), as a bf16 store of a double value does on the
// device.  Bit-exact with the oracle's restatement (oracle.sgd_step); ATen's
// CUDA _fused_sgd_ evaluates the same definition with fp32 intermediates and
// agrees to a few roundings of the operands' magnitude (tests/test_gpu_sgd.py).
#include <algorithm>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kMaxTensors = 96;
constexpr int kChunk = 8192;
constexpr int kThreads = 256;

struct SgdArgs {
  void* param[kMaxTensors];
  void* grad[kMaxTensors];
  void* buf[kMaxTensors];
  long long numel[kMaxTensors];
  int chunk_begin[kMaxTensors + 1];  // prefix sums of chunks per tensor
  unsigned char vec[kMaxTensors];    // arrays 16-byte aligned: 16-byte vector accesses
  int ntensors;
};

struct SgdScalars {
  double lr, wd, momentum, dampening;
  int nesterov, maximize, first_step, has_buf;
  const float* lr_tensor;
  const float* grad_scale;
  const float* found_inf;
};

template <typename T>
__device__ __forceinline__ float ldv(const void* p, long long i) {
  if constexpr (sizeof(T) == 2)
    return bf2f(static_cast<const uint16_t*>(p)[i]);
  else
    return static_cast<const float*>(p)[i];
}
template <typename T>
__device__ __forceinline__ void stv(void* p, long long i, float v) {
  if constexpr (sizeof(T) == 2)
    static_cast<uint16_t*>(p)[i] = f2bf(v);
  else
    static_cast<float*>(p)[i] = v;
}

// One element: p, g, b in fp32 in, the values to store out.
__device__ __forceinline__ void sgd_elem(const SgdScalars& s, double lr, float scale, float& p, float& g, float& b) {
  if (s.grad_scale) g = float(__ddiv_rn(double(g), double(scale)));
  float gg = s.maximize ? -g : g;
  if (s.wd != 0.0) gg = float(__dadd_rn(double(gg), __dmul_rn(s.wd, double(p))));
  if (s.has_buf) {
    const double bd = s.first_step ? double(gg)
                                   : __dadd_rn(__dmul_rn(s.momentum, double(b)),
                                               __dmul_rn(1.0 - s.dampening, double(gg)));
    b = float(bd);
    gg = s.nesterov ? float(__dadd_rn(double(gg), __dmul_rn(s.momentum, bd))) : float(bd);
  }
  p = float(__dsub_rn(double(p), __dmul_rn(lr, double(gg))));
}

template <typename T>
__device__ __forceinline__ void scalar_range(const SgdScalars& s, double lr, float scale, void* P, void* G, void* Bf,
                                             long long j0, long long j1, bool load_buf) {
  for (long long j = j0; j < j1; ++j) {
    float p = ldv<T>(P, j), g = ldv<T>(G, j), b = load_buf ? ldv<T>(Bf, j) : 0.f;
    sgd_elem(s, lr, scale, p, g, b);
    stv<T>(P, j, p);
    if (s.grad_scale) stv<T>(G, j, g);
    if (s.has_buf) stv<T>(Bf, j, b);
  }
}

// 16 bytes of T -> fp32 lanes and back
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float (&o)[16 / sizeof(T)]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[2 * k] = __uint_as_float(w[k] << 16);
      o[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = __uint_as_float(w[k]);
  }
}
template <typename T>
__device__ __forceinline__ uint4 pack16(const float (&v)[16 / sizeof(T)]) {
  uint32_t w[4];
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = uint32_t(f2bf(v[2 * k])) | (uint32_t(f2bf(v[2 * k + 1])) << 16);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = __float_as_uint(v[k]);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) sgd_kernel(const __grid_constant__ SgdArgs a, const SgdScalars s) {
  if (s.found_inf && *s.found_inf != 0.f) return;
  const double lr = s.lr_tensor ? double(*s.lr_tensor) : s.lr;
  const float scale = s.grad_scale ? *s.grad_scale : 1.f;
  constexpr int V = 16 / int(sizeof(T));  // elements per 16-byte vector
  const bool load_buf = s.has_buf && !s.first_step;
  const int total = a.chunk_begin[a.ntensors];
  int t = 0;
  for (int chunk = blockIdx.x; chunk < total; chunk += gridDim.x) {
    while (chunk >= a.chunk_begin[t + 1]) ++t;
    const long long begin = (long long)(chunk - a.chunk_begin[t]) * kChunk;
    const long long end = min(begin + kChunk, a.numel[t]);
    void* P = a.param[t];
    void* G = a.grad[t];
    void* Bf = a.buf[t];
    if (!a.vec[t]) {
      for (long long j = begin + threadIdx.x; j < end; j += kThreads) scalar_range<T>(s, lr, scale, P, G, Bf, j, j + 1, load_buf);
      continue;
    }
    // two 16-byte vectors per thread, all loads issued before the math
    for (long long i0 = begin + (long long)V * threadIdx.x; i0 < end; i0 += 2LL * V * kThreads) {
      const long long i1 = i0 + (long long)V * kThreads;
      if (i0 + V > end || (i1 < end && i1 + V > end)) {  // ragged tail of the tensor
        scalar_range<T>(s, lr, scale, P, G, Bf, i0, min(i0 + V, end), load_buf);
        if (i1 < end) scalar_range<T>(s, lr, scale, P, G, Bf, i1, min(i1 + V, end), load_buf);
        continue;
      }
      const int nv = i1 < end ? 2 : 1;
      uint4 up[2], ug[2], ub[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (k < nv) {
          const long long i = k ? i1 : i0;
          up[k] = *reinterpret_cast<const uint4*>(static_cast<const T*>(P) + i);
          ug[k] = *reinterpret_cast<const uint4*>(static_cast<const T*>(G) + i);
          if (load_buf) ub[k] = *reinterpret_cast<const uint4*>(static_cast<const T*>(Bf) + i);
        }
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (k < nv) {
          const long long i = k ? i1 : i0;
          float p[V], g[V], b[V];
          unpack16<T>(up[k], p);
          unpack16<T>(ug[k], g);
          unpack16<T>(ub[k], b);
#pragma unroll
          for (int e = 0; e < V; ++e) sgd_elem(s, lr, scale, p[e], g[e], b[e]);
          *reinterpret_cast<uint4*>(static_cast<T*>(P) + i) = pack16<T>(p);
          if (s.grad_scale) *reinterpret_cast<uint4*>(static_cast<T*>(G) + i) = pack16<T>(g);
          if (s.has_buf) *reinterpret_cast<uint4*>(static_cast<T*>(Bf) + i) = pack16<T>(b);
        }
      }
    }
  }
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" b2_status b2_fused_sgd(const b2_sgd_tensor* tensors, int n, const b2_sgd_hparams* hp, void* stream) {
  if (n < 0 || (n > 0 && !tensors) || !hp) return set_error(B2_ERR_INVALID, "b2_fused_sgd: bad arguments");
  if (hp->param_dtype != B2_BF16 && hp->param_dtype != B2_F32) return set_error(B2_ERR_INVALID, "b2_fused_sgd: dtype");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SgdScalars sc{};
  sc.lr = hp->lr;
  sc.wd = hp->weight_decay;
  sc.momentum = hp->momentum;
  sc.dampening = hp->dampening;
  sc.nesterov = hp->nesterov;
  sc.maximize = hp->maximize;
  sc.first_step = hp->is_first_step;
  sc.has_buf = hp->momentum != 0.0;
  sc.lr_tensor = hp->lr_tensor;
  sc.grad_scale = hp->grad_scale;
  sc.found_inf = hp->found_inf;
  auto kern = hp->param_dtype == B2_BF16 ? sgd_kernel<uint16_t> : sgd_kernel<float>;
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  static int per_sm[64][2] = {};
  int& occ = per_sm[dev][hp->param_dtype == B2_BF16 ? 0 : 1];
  if (!occ) {
    int b = 0;
    B2_TRY(check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, kThreads, 0), "occupancy"));
    occ = std::max(1, b);
  }
  const int max_grid = occ * sm_count(dev);
  SgdArgs args;
  args.ntensors = 0;
  args.chunk_begin[0] = 0;
  auto flush = [&]() -> b2_status {
    const int total = args.chunk_begin[args.ntensors];
    if (total > 0) {
      kern<<<std::min(total, max_grid), kThreads, 0, st>>>(args, sc);
      B2_TRY(check_cuda(cudaGetLastError(), "fused sgd launch"));
    }
    args.ntensors = 0;
    args.chunk_begin[0] = 0;
    return B2_OK;
  };
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  for (int i = 0; i < n; ++i) {
    const b2_sgd_tensor& t = tensors[i];
    if (t.numel <= 0) continue;
    if (!t.param || !t.grad || (sc.has_buf && !t.momentum_buffer))
      return set_error(B2_ERR_INVALID, "b2_fused_sgd: null pointer in tensor %d", i);
    const long long chunks = (t.numel + kChunk - 1) / kChunk;
    if (chunks > (1LL << 30)) return set_error(B2_ERR_UNSUPPORTED, "b2_fused_sgd: tensor %d too large", i);
    if (args.ntensors == kMaxTensors || args.chunk_begin[args.ntensors] + chunks > (1LL << 30)) B2_TRY(flush());
    const int k = args.ntensors;
    args.param[k] = t.param;
    args.grad[k] = t.grad;
    args.buf[k] = t.momentum_buffer;
    args.numel[k] = t.numel;
    args.vec[k] = al(t.param) && al(t.grad) && (!sc.has_buf || al(t.momentum_buffer));
    args.chunk_begin[k + 1] = args.chunk_begin[k] + int(chunks);
    args.ntensors = k + 1;
  }
  return flush();
}
