// Training BatchNorm2d + LeakyReLU/ReLU on contiguous NCHW bf16, the fused
// pair behind xdna_train.regions.fuse_norm_activation.  Same contract as the
// reference's host kernels (xdna_train/_native/region_kernels.cpp:309-460):
//
//   statistics  each (n, c) plane reduced in fp32: mean = sum / HW, then the
//               sum of squared deviations from that mean; the N planes of a
//               channel merged in double, in plane order, with Chan's
//               parallel-variance formula; invstd = 1 / sqrt(var + eps) in
//               double; running statistics (bf16) updated with the unbiased
//               variance.
//   forward     y = act(x*scale + shift), scale = w*invstd, shift = b -
//               mean*scale, act(z) = z > 0 ? z : z*slope, one rounding to bf16.
//   backward    dz = dy where y > 0 (or y is NaN and the activation is ReLU),
//               else dy*slope; db = sum dz, dw = sum dz*xhat (plane sums in
//               fp32, channel sums in double); dx = w*invstd*(dz - db/M -
//               xhat*dw/M).
//
// Every elementwise expression is evaluated with explicitly rounded fp32
// operations in the reference's order (no FMA contraction: the reference's
// host build has none), so the outputs differ from the reference only where
// the fp32 plane sums do (their summation order differs).
//
// Memory traffic (M = N*C*HW elements): forward 6 B/elem (stats read x, apply
// reads x and writes y), backward 14 B/elem (plane sums read dy, y, x; dx reads
// them again and writes dx).  Second reads of tensors smaller than L2 hit L2.
#include <algorithm>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kBnThreads = 256;

// Sum over the TPP threads of a plane group (a warp, or the whole block).
template <int TPP>
__device__ __forceinline__ float group_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  if constexpr (TPP == 32) {
    return v;
  } else {
    const int w = threadIdx.x >> 5;
    __syncthreads();  // red[] may still be read from a previous call
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float s = red[0];
#pragma unroll
    for (int k = 1; k < TPP / 32; ++k) s = __fadd_rn(s, red[k]);
    return s;
  }
}

__device__ __forceinline__ void unpack8(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    f[2 * k] = __uint_as_float(w[k] << 16);
    f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
  }
}

// Per-plane fp32 mean and sum of squared deviations.  TPP threads per plane:
// a warp (many small planes) or the whole block (few large planes).  VEC:
// 8 elements per 16-byte load (HW % 8 == 0, so every plane starts aligned).
template <int TPP, bool VEC>
__global__ void __launch_bounds__(kBnThreads) bn_plane_stats_kernel(
    const uint16_t* __restrict__ x, long long planes, long long hw, float* __restrict__ pm,
    float* __restrict__ pq) {
  __shared__ float red[kBnThreads / 32];
  constexpr int kGroups = kBnThreads / TPP;
  const int lane = threadIdx.x % TPP;
  const long long g0 = (long long)blockIdx.x * kGroups + threadIdx.x / TPP;
  const long long gstep = (long long)gridDim.x * kGroups;
  // all threads of a block run the same number of iterations (group_sum syncs)
  const long long iters = (planes + gstep - 1) / gstep;
  for (long long it = 0; it < iters; ++it) {
    const long long pl = g0 + it * gstep;
    const bool live = pl < planes;
    const uint16_t* p = x + (live ? pl : 0) * hw;
    float s = 0.0f;
    if (live) {
      if constexpr (VEC) {
        const uint4* pv = reinterpret_cast<const uint4*>(p);
        for (long long v = lane; v < hw / 8; v += TPP) {
          float f[8];
          unpack8(__ldg(pv + v), f);
#pragma unroll
          for (int k = 0; k < 8; ++k) s = __fadd_rn(s, f[k]);
        }
      } else {
        for (long long i = lane; i < hw; i += TPP) s = __fadd_rn(s, bf2f(p[i]));
      }
    }
    const float mean = __fdiv_rn(group_sum<TPP>(s, red), float(hw));
    float q = 0.0f;
    if (live) {
      if constexpr (VEC) {
        const uint4* pv = reinterpret_cast<const uint4*>(p);
        for (long long v = lane; v < hw / 8; v += TPP) {
          float f[8];
          unpack8(__ldg(pv + v), f);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float d = __fsub_rn(f[k], mean);
            q = __fadd_rn(q, __fmul_rn(d, d));
          }
        }
      } else {
        for (long long i = lane; i < hw; i += TPP) {
          const float d = __fsub_rn(bf2f(p[i]), mean);
          q = __fadd_rn(q, __fmul_rn(d, d));
        }
      }
    }
    q = group_sum<TPP>(q, red);
    if (live && lane == 0) {
      pm[pl] = mean;
      pq[pl] = q;
    }
  }
}

// One thread per channel: Chan's merge of the N plane statistics in double,
// in plane order; mean / invstd out; running statistics.
__global__ void bn_channel_stats_kernel(const float* __restrict__ pm, const float* __restrict__ pq,
                                        long long N, long long C, long long hw, float eps,
                                        float factor, int update, uint16_t* rm, uint16_t* rv,
                                        float* __restrict__ mean_out, float* __restrict__ invstd_out) {
  const long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const double nb = double(hw);
  double count = 0.0, mean = 0.0, m2 = 0.0;
  for (long long n = 0; n < N; ++n) {
    const double tot = count + nb;
    const double delta = double(pm[n * C + c]) - mean;
    mean += delta * nb / tot;
    m2 += double(pq[n * C + c]) + delta * delta * count * nb / tot;
    count = tot;
  }
  const double M = double(N) * nb;
  const double var = m2 / M;
  mean_out[c] = float(mean);
  invstd_out[c] = float(1.0 / sqrt(var + double(eps)));
  if (update) {
    const double unbiased = M > 1.0 ? var * M / (M - 1.0) : var;
    const double f = double(factor);
    rm[c] = f2bf(float((1.0 - f) * double(bf2f(rm[c])) + f * mean));
    rv[c] = f2bf(float((1.0 - f) * double(bf2f(rv[c])) + f * unbiased));
  }
}

__device__ __forceinline__ float bn_act(float xv, float scale, float shift, float slope) {
  const float z = __fadd_rn(__fmul_rn(xv, scale), shift);
  return z > 0.0f ? z : __fmul_rn(z, slope);
}

// y = act(x*scale + shift); one thread per 8 elements (VEC) or per element.
template <bool VEC>
__global__ void __launch_bounds__(kBnThreads) bn_apply_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, const uint16_t* __restrict__ b,
    const float* __restrict__ mean, const float* __restrict__ invstd, uint16_t* __restrict__ y,
    long long units, long long units_per_plane, long long C, float slope) {
  for (long long u = (long long)blockIdx.x * kBnThreads + threadIdx.x; u < units;
       u += (long long)gridDim.x * kBnThreads) {
    const long long c = (u / units_per_plane) % C;
    const float is = __ldg(invstd + c);
    const float scale = __fmul_rn(w ? bf2f(__ldg(w + c)) : 1.0f, is);
    const float shift = __fsub_rn(b ? bf2f(__ldg(b + c)) : 0.0f, __fmul_rn(__ldg(mean + c), scale));
    if constexpr (VEC) {
      float f[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(x) + u), f);
      uint4 o;
      o.x = pack_bf2(bn_act(f[0], scale, shift, slope), bn_act(f[1], scale, shift, slope));
      o.y = pack_bf2(bn_act(f[2], scale, shift, slope), bn_act(f[3], scale, shift, slope));
      o.z = pack_bf2(bn_act(f[4], scale, shift, slope), bn_act(f[5], scale, shift, slope));
      o.w = pack_bf2(bn_act(f[6], scale, shift, slope), bn_act(f[7], scale, shift, slope));
      reinterpret_cast<uint4*>(y)[u] = o;
    } else {
      y[u] = f2bf(bn_act(bf2f(x[u]), scale, shift, slope));
    }
  }
}

__device__ __forceinline__ float bn_dz(float g, float yv, float slope, int relu) {
  return ((yv > 0.0f) || (relu && yv != yv)) ? g : __fmul_rn(g, slope);
}

// Per-plane fp32 sums of dz and dz*xhat.
template <int TPP, bool VEC>
__global__ void __launch_bounds__(kBnThreads) bn_bwd_plane_kernel(
    const uint16_t* __restrict__ dy, const uint16_t* __restrict__ y, const uint16_t* __restrict__ x,
    const float* __restrict__ mean, const float* __restrict__ invstd, long long planes, long long C,
    long long hw, float slope, int relu, float* __restrict__ ps, float* __restrict__ pt) {
  __shared__ float red[kBnThreads / 32];
  constexpr int kGroups = kBnThreads / TPP;
  const int lane = threadIdx.x % TPP;
  const long long g0 = (long long)blockIdx.x * kGroups + threadIdx.x / TPP;
  const long long gstep = (long long)gridDim.x * kGroups;
  const long long iters = (planes + gstep - 1) / gstep;
  for (long long it = 0; it < iters; ++it) {
    const long long pl = g0 + it * gstep;
    const bool live = pl < planes;
    float s1 = 0.0f, s2 = 0.0f;
    if (live) {
      const long long c = pl % C;
      const float mc = __ldg(mean + c), is = __ldg(invstd + c);
      const long long off = pl * hw;
      if constexpr (VEC) {
        const uint4* dv = reinterpret_cast<const uint4*>(dy + off);
        const uint4* yv = reinterpret_cast<const uint4*>(y + off);
        const uint4* xv = reinterpret_cast<const uint4*>(x + off);
        for (long long v = lane; v < hw / 8; v += TPP) {
          float fg[8], fy[8], fx[8];
          unpack8(__ldg(dv + v), fg);
          unpack8(__ldg(yv + v), fy);
          unpack8(__ldg(xv + v), fx);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float dz = bn_dz(fg[k], fy[k], slope, relu);
            s1 = __fadd_rn(s1, dz);
            s2 = __fadd_rn(s2, __fmul_rn(dz, __fmul_rn(__fsub_rn(fx[k], mc), is)));
          }
        }
      } else {
        for (long long i = lane; i < hw; i += TPP) {
          const float dz = bn_dz(bf2f(dy[off + i]), bf2f(y[off + i]), slope, relu);
          s1 = __fadd_rn(s1, dz);
          s2 = __fadd_rn(s2, __fmul_rn(dz, __fmul_rn(__fsub_rn(bf2f(x[off + i]), mc), is)));
        }
      }
    }
    s1 = group_sum<TPP>(s1, red);
    s2 = group_sum<TPP>(s2, red);
    if (live && lane == 0) {
      ps[pl] = s1;
      pt[pl] = s2;
    }
  }
}

// One thread per channel: double sums over the N planes in order; db, dw and
// the two means the dx pass needs (k[c] = db/M, k[C + c] = dw/M).
__global__ void bn_bwd_channel_kernel(const float* __restrict__ ps, const float* __restrict__ pt,
                                      long long N, long long C, long long hw, uint16_t* dw,
                                      uint16_t* db, float* __restrict__ k) {
  const long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  double a = 0.0, bs = 0.0;
  for (long long n = 0; n < N; ++n) {
    a += double(ps[n * C + c]);
    bs += double(pt[n * C + c]);
  }
  if (db) db[c] = f2bf(float(a));
  if (dw) dw[c] = f2bf(float(bs));
  const double M = double(N) * double(hw);
  k[c] = float(a / M);
  k[C + c] = float(bs / M);
}

__device__ __forceinline__ float bn_dx(float g, float yv, float xv, float mc, float is, float ws,
                                       float k1, float k2, float slope, int relu) {
  const float dz = bn_dz(g, yv, slope, relu);
  const float xhat = __fmul_rn(__fsub_rn(xv, mc), is);
  return __fmul_rn(ws, __fsub_rn(__fsub_rn(dz, k1), __fmul_rn(xhat, k2)));
}

template <bool VEC>
__global__ void __launch_bounds__(kBnThreads) bn_bwd_dx_kernel(
    const uint16_t* __restrict__ dy, const uint16_t* __restrict__ y, const uint16_t* __restrict__ x,
    const uint16_t* __restrict__ w, const float* __restrict__ mean, const float* __restrict__ invstd,
    const float* __restrict__ k, uint16_t* __restrict__ dx, long long units, long long units_per_plane,
    long long C, float slope, int relu) {
  for (long long u = (long long)blockIdx.x * kBnThreads + threadIdx.x; u < units;
       u += (long long)gridDim.x * kBnThreads) {
    const long long c = (u / units_per_plane) % C;
    const float mc = __ldg(mean + c), is = __ldg(invstd + c);
    const float ws = __fmul_rn(w ? bf2f(__ldg(w + c)) : 1.0f, is);
    const float k1 = __ldg(k + c), k2 = __ldg(k + C + c);
    if constexpr (VEC) {
      float fg[8], fy[8], fx[8], r[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(dy) + u), fg);
      unpack8(__ldg(reinterpret_cast<const uint4*>(y) + u), fy);
      unpack8(__ldg(reinterpret_cast<const uint4*>(x) + u), fx);
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = bn_dx(fg[e], fy[e], fx[e], mc, is, ws, k1, k2, slope, relu);
      uint4 o;
      o.x = pack_bf2(r[0], r[1]);
      o.y = pack_bf2(r[2], r[3]);
      o.z = pack_bf2(r[4], r[5]);
      o.w = pack_bf2(r[6], r[7]);
      reinterpret_cast<uint4*>(dx)[u] = o;
    } else {
      dx[u] = f2bf(bn_dx(bf2f(dy[u]), bf2f(y[u]), bf2f(x[u]), mc, is, ws, k1, k2, slope, relu));
    }
  }
}

// Warp-per-plane when there are enough planes to fill the GPU with warps,
// else block-per-plane.
bool warp_per_plane(long long planes, int sms) { return planes >= (long long)sms * 32; }

int stats_grid(long long planes, bool warp, int sms) {
  const long long groups = warp ? (planes + kBnThreads / 32 - 1) / (kBnThreads / 32) : planes;
  return int(std::max<long long>(1, std::min<long long>(groups, (long long)sms * 8)));
}

int elem_grid(long long units, int sms) {
  const long long b = (units + kBnThreads - 1) / kBnThreads;
  return int(std::max<long long>(1, std::min<long long>(b, (long long)sms * 16)));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

b2_status bn_check(int64_t N, int64_t C, int64_t HW, const void* ws, size_t ws_bytes, const char* who) {
  if (N < 0 || C < 0 || HW < 0) return set_error(B2_ERR_INVALID, "%s: negative size", who);
  if (ws_bytes < b2_region_bn_workspace_bytes(N, C) || (N * C > 0 && !ws) || !aligned16(ws))
    return set_error(B2_ERR_WORKSPACE, "%s: workspace too small or misaligned", who);
  return B2_OK;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

size_t b2_region_bn_workspace_bytes(int64_t N, int64_t C) {
  if (N <= 0 || C <= 0) return 0;
  // two fp32 per plane, then two fp32 per channel, each array 16-byte aligned
  const size_t planes = size_t(N) * size_t(C);
  return ((2 * planes * sizeof(float) + 15) & ~size_t(15)) + ((2 * size_t(C) * sizeof(float) + 15) & ~size_t(15));
}

b2_status b2_region_bn_fwd_bf16(const void* x, const void* w, const void* b, void* rm, void* rv,
                                void* y, float* mean_out, float* invstd_out, int64_t N, int64_t C,
                                int64_t HW, float eps, float slope, float factor, int update,
                                void* workspace, size_t workspace_bytes, void* stream) {
  B2_TRY(bn_check(N, C, HW, workspace, workspace_bytes, "b2_region_bn_fwd_bf16"));
  if (N * C == 0) return B2_OK;
  if (HW == 0) return set_error(B2_ERR_INVALID, "b2_region_bn_fwd_bf16: empty planes");
  if (!x || !y || !mean_out || !invstd_out || (update && (!rm || !rv)))
    return set_error(B2_ERR_INVALID, "b2_region_bn_fwd_bf16: null pointer");
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const int sms = sm_count(dev);
  auto st = static_cast<cudaStream_t>(stream);
  const long long planes = N * C;
  float* pm = static_cast<float*>(workspace);
  float* pq = pm + planes;
  const bool vec = HW % 8 == 0 && aligned16(x) && aligned16(y);
  const bool warp = warp_per_plane(planes, sms);
  const int sg = stats_grid(planes, warp, sms);
  auto xs = static_cast<const uint16_t*>(x);
  if (warp && vec) bn_plane_stats_kernel<32, true><<<sg, kBnThreads, 0, st>>>(xs, planes, HW, pm, pq);
  else if (warp) bn_plane_stats_kernel<32, false><<<sg, kBnThreads, 0, st>>>(xs, planes, HW, pm, pq);
  else if (vec) bn_plane_stats_kernel<kBnThreads, true><<<sg, kBnThreads, 0, st>>>(xs, planes, HW, pm, pq);
  else bn_plane_stats_kernel<kBnThreads, false><<<sg, kBnThreads, 0, st>>>(xs, planes, HW, pm, pq);
  B2_TRY(check_cuda(cudaGetLastError(), "bn stats launch"));
  bn_channel_stats_kernel<<<int((C + 127) / 128), 128, 0, st>>>(
      pm, pq, N, C, HW, eps, factor, update, static_cast<uint16_t*>(rm), static_cast<uint16_t*>(rv),
      mean_out, invstd_out);
  B2_TRY(check_cuda(cudaGetLastError(), "bn channel launch"));
  auto wp = static_cast<const uint16_t*>(w);
  auto bp = static_cast<const uint16_t*>(b);
  auto yp = static_cast<uint16_t*>(y);
  if (vec) {
    const long long units = planes * (HW / 8);
    bn_apply_kernel<true><<<elem_grid(units, sms), kBnThreads, 0, st>>>(xs, wp, bp, mean_out, invstd_out, yp,
                                                                       units, HW / 8, C, slope);
  } else {
    const long long units = planes * HW;
    bn_apply_kernel<false><<<elem_grid(units, sms), kBnThreads, 0, st>>>(xs, wp, bp, mean_out, invstd_out, yp,
                                                                        units, HW, C, slope);
  }
  return check_cuda(cudaGetLastError(), "bn apply launch");
}

b2_status b2_region_bn_bwd_bf16(const void* dy, const void* y, const void* x, const void* w,
                                const float* mean, const float* invstd, void* dx, void* dw, void* db,
                                int64_t N, int64_t C, int64_t HW, float slope, int relu, void* workspace,
                                size_t workspace_bytes, void* stream) {
  B2_TRY(bn_check(N, C, HW, workspace, workspace_bytes, "b2_region_bn_bwd_bf16"));
  if (N * C == 0) return B2_OK;
  if (HW == 0) return set_error(B2_ERR_INVALID, "b2_region_bn_bwd_bf16: empty planes");
  if (!dy || !y || !x || !mean || !invstd)
    return set_error(B2_ERR_INVALID, "b2_region_bn_bwd_bf16: null pointer");
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const int sms = sm_count(dev);
  auto st = static_cast<cudaStream_t>(stream);
  const long long planes = N * C;
  float* ps = static_cast<float*>(workspace);
  float* pt = ps + planes;
  float* k = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                      ((2 * size_t(planes) * sizeof(float) + 15) & ~size_t(15)));
  const bool vec = HW % 8 == 0 && aligned16(dy) && aligned16(y) && aligned16(x) && (!dx || aligned16(dx));
  const bool warp = warp_per_plane(planes, sms);
  const int sg = stats_grid(planes, warp, sms);
  auto g = static_cast<const uint16_t*>(dy);
  auto yy = static_cast<const uint16_t*>(y);
  auto xx = static_cast<const uint16_t*>(x);
  if (warp && vec)
    bn_bwd_plane_kernel<32, true><<<sg, kBnThreads, 0, st>>>(g, yy, xx, mean, invstd, planes, C, HW, slope, relu, ps, pt);
  else if (warp)
    bn_bwd_plane_kernel<32, false><<<sg, kBnThreads, 0, st>>>(g, yy, xx, mean, invstd, planes, C, HW, slope, relu, ps, pt);
  else if (vec)
    bn_bwd_plane_kernel<kBnThreads, true><<<sg, kBnThreads, 0, st>>>(g, yy, xx, mean, invstd, planes, C, HW, slope,
                                                                     relu, ps, pt);
  else
    bn_bwd_plane_kernel<kBnThreads, false><<<sg, kBnThreads, 0, st>>>(g, yy, xx, mean, invstd, planes, C, HW, slope,
                                                                      relu, ps, pt);
  B2_TRY(check_cuda(cudaGetLastError(), "bn bwd plane launch"));
  bn_bwd_channel_kernel<<<int((C + 127) / 128), 128, 0, st>>>(ps, pt, N, C, HW, static_cast<uint16_t*>(dw),
                                                              static_cast<uint16_t*>(db), k);
  B2_TRY(check_cuda(cudaGetLastError(), "bn bwd channel launch"));
  if (!dx) return B2_OK;
  auto wp = static_cast<const uint16_t*>(w);
  auto out = static_cast<uint16_t*>(dx);
  if (vec) {
    const long long units = planes * (HW / 8);
    bn_bwd_dx_kernel<true><<<elem_grid(units, sms), kBnThreads, 0, st>>>(g, yy, xx, wp, mean, invstd, k, out, units,
                                                                        HW / 8, C, slope, relu);
  } else {
    const long long units = planes * HW;
    bn_bwd_dx_kernel<false><<<elem_grid(units, sms), kBnThreads, 0, st>>>(g, yy, xx, wp, mean, invstd, k, out, units,
                                                                         HW, C, slope, relu);
  }
  return check_cuda(cudaGetLastError(), "bn dx launch");
}

}  // extern "C"
