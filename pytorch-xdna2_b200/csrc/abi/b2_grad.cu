// The ReLU backward of a residual block's output fused with the gradient sum
// that feeds it.  In a ResNet the output y = relu(bn(...) + identity) of
// block k is the input of block k+1 twice (its first convolution and its
// identity path), so autograd first adds the two gradients that arrive for y
// (an in-place add of bf16 tensors) and then runs threshold_backward on the
// sum.  The reference runs both as ATen ops on its CPU path
// (torch_xdna_device.cpp:5124-5260); here the add is left pending and this
// kernel does both in one pass:
//
//   dz = (y > 0 or y is NaN) ? bf16(float(a) + float(b)) : +0
//
// -- ATen's add (one fp32 add, rounded to nearest even by the hardware
// conversion, as ATen's CUDA kernel does) and threshold_backward (keeps the
// gradient where !(y <= 0)), bit for bit, reading a, b, y and writing dz
// instead of reading a, b, writing the sum, reading it and y, writing dz.
// HBM-bound: 8 bytes per element instead of 12.
#include <cuda_bf16.h>

#include <algorithm>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kGradThreads = 256;

__device__ __forceinline__ uint32_t gated_sum2(uint32_t a, uint32_t b, uint32_t y) {
  uint32_t out = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t sh = 16u * uint32_t(h);
    const float fa = __uint_as_float(((a >> sh) & 0xffffu) << 16);
    const float fb = __uint_as_float(((b >> sh) & 0xffffu) << 16);
    const float fy = __uint_as_float(((y >> sh) & 0xffffu) << 16);
    uint32_t v = 0;
    if (!(fy <= 0.0f)) v = __bfloat16_as_ushort(__float2bfloat16_rn(__fadd_rn(fa, fb)));
    out |= v << sh;
  }
  return out;
}

// Four 16-byte units per thread in flight, grid-stride.
__global__ void __launch_bounds__(kGradThreads) relu_bwd_sum_kernel(const uint4* __restrict__ a,
                                                                    const uint4* __restrict__ b,
                                                                    const uint4* __restrict__ y, uint4* __restrict__ dz,
                                                                    long long units) {
  const long long stride = (long long)gridDim.x * kGradThreads;
  long long u = (long long)blockIdx.x * kGradThreads + threadIdx.x;
  auto one = [](const uint4 va, const uint4 vb, const uint4 vy) {
    return make_uint4(gated_sum2(va.x, vb.x, vy.x), gated_sum2(va.y, vb.y, vy.y), gated_sum2(va.z, vb.z, vy.z),
                      gated_sum2(va.w, vb.w, vy.w));
  };
  for (; u + 3 * stride < units; u += 4 * stride) {
    uint4 va[4], vb[4], vy[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      va[i] = __ldg(a + u + i * stride);
      vb[i] = __ldg(b + u + i * stride);
      vy[i] = __ldg(y + u + i * stride);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) dz[u + i * stride] = one(va[i], vb[i], vy[i]);
  }
  for (; u < units; u += stride) dz[u] = one(__ldg(a + u), __ldg(b + u), __ldg(y + u));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" b2_status b2_relu_bwd_sum_bf16(const void* a, const void* b, const void* y, void* dz, int64_t n,
                                          void* stream) {
  if (n < 0) return set_error(B2_ERR_INVALID, "b2_relu_bwd_sum_bf16: negative size");
  if (n == 0) return B2_OK;
  if (!a || !b || !y || !dz) return set_error(B2_ERR_INVALID, "b2_relu_bwd_sum_bf16: null pointer");
  if (n % 8 || !aligned16(a) || !aligned16(b) || !aligned16(y) || !aligned16(dz))
    return set_error(B2_ERR_UNSUPPORTED, "b2_relu_bwd_sum_bf16: needs 16-byte aligned tensors of 8k elements");
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const long long units = n / 8;
  const long long want = (units + kGradThreads * 4 - 1) / (kGradThreads * 4);
  const int grid = int(std::max<long long>(1, std::min<long long>(want, (long long)sm_count(dev) * 8)));
  relu_bwd_sum_kernel<<<grid, kGradThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(a), static_cast<const uint4*>(b), static_cast<const uint4*>(y),
      static_cast<uint4*>(dz), units);
  return check_cuda(cudaGetLastError(), "relu_bwd_sum launch");
}
