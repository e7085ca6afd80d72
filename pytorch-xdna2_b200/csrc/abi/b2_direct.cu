// Direct convolution on the CUDA cores for layers with a handful of output
// channels (an RGB output layer, 9x9 32->3), forward and input gradient.  The
// reference runs every convolution outside its 3x3 fast path on its CPU path
// (torch_xdna_device.cpp:4578-4605, 4828-4878); on B200 the tensor-core
// formulations waste almost all of an MMA tile on such layers, and ATen's
// library falls back to a direct kernel that takes ~0.5 ms for the 9x9 32->3
// input gradient of a B40 36x36 batch.
//
//   out[b][o][y][x] = bias[o] + sum_{i, ky, kx} in[b][i][y*sy - py + ky*dy][x*sx - px + kx*dx] * wt[i][ky][kx][o]
//
// in fp32, summed in (i, ky, kx) order, rounded once to bf16.  The forward is
// this with wt[ci][ky][kx][co] = W[co][ci][ky][kx]; the input gradient of a
// stride-1 convolution is this over dY with wt[co][ky][kx][ci] =
// W[co][ci][kh-1-ky][kw-1-kx] and padding (k-1)*d - p.
//
// A CTA computes a TH x TW tile of output pixels of one image, a thread per
// pixel with NOUT fp32 accumulators; the input tile (with its halo, zero
// outside the image) and all weights sit in shared memory, weights as fp32
// with the output channel fastest so that a thread reads four of them per
// 16-byte broadcast load.
#include <algorithm>

#include "b2_common.cuh"

namespace b2 {
namespace {

struct DirectGeom {
  int B, NIN, Hin, Win, NOUTr, Ho, Wo;  // NOUTr: real output channels
  int kh, kw, sy, sx, py, px, dy, dx;
  long long is[4], os[4];
  int TH, TW, IH, IW, tiles_x, tiles_y;
};

// KW > 0: the kernel width is a compile-time constant and the tap loop
// unrolls, so a thread issues all of a row's loads back to back.
template <int NOUT, int KW>
__global__ void direct_conv_kernel(const uint16_t* __restrict__ in, const float* __restrict__ wt,
                                   const uint16_t* __restrict__ bias, DirectGeom g, uint16_t* __restrict__ out) {
  extern __shared__ float sm[];
  float* ws = sm;                                                      // [NIN][kh][kw][NOUT]
  const int nw = g.NIN * g.kh * g.kw * NOUT;
  uint16_t* xs = reinterpret_cast<uint16_t*>(sm + nw);                 // [NIN][IH][IW]
  const int tile = blockIdx.x % (g.tiles_x * g.tiles_y);
  const int b = blockIdx.x / (g.tiles_x * g.tiles_y);
  const int oy0 = (tile / g.tiles_x) * g.TH, ox0 = (tile % g.tiles_x) * g.TW;
  const int iy0 = oy0 * g.sy - g.py, ix0 = ox0 * g.sx - g.px;
  const int nthr = blockDim.x;
  for (int e = threadIdx.x; e < nw; e += nthr) ws[e] = wt[e];
  const int plane = g.IH * g.IW;
  for (int e = threadIdx.x; e < g.NIN * plane; e += nthr) {
    const int i = e / plane, r = e - i * plane;
    const int yy = r / g.IW, xx = r - yy * g.IW;
    const int iy = iy0 + yy, ix = ix0 + xx;
    uint16_t v = 0;
    if (iy >= 0 && iy < g.Hin && ix >= 0 && ix < g.Win)
      v = in[b * g.is[0] + i * g.is[1] + (long long)iy * g.is[2] + (long long)ix * g.is[3]];
    xs[e] = v;
  }
  __syncthreads();
  const int ty = threadIdx.x / g.TW, tx = threadIdx.x - ty * g.TW;
  const int oy = oy0 + ty, ox = ox0 + tx;
  if (ty >= g.TH || oy >= g.Ho || ox >= g.Wo) return;
  float acc[NOUT];
#pragma unroll
  for (int o = 0; o < NOUT; ++o) acc[o] = (bias && o < g.NOUTr) ? bf2f(bias[o]) : 0.f;
  const int by = ty * g.sy, bx = tx * g.sx;
  for (int i = 0; i < g.NIN; ++i) {
    const uint16_t* xi = xs + i * plane;
    const float* wi = ws + i * g.kh * g.kw * NOUT;
    for (int ky = 0; ky < g.kh; ++ky) {
      const uint16_t* xr = xi + (by + ky * g.dy) * g.IW + bx;
      const float* wr = wi + ky * g.kw * NOUT;
      auto tap = [&](int kx) {
        const float v = bf2f(xr[kx * g.dx]);
        const float4* w4 = reinterpret_cast<const float4*>(wr + kx * NOUT);
#pragma unroll
        for (int q = 0; q < NOUT / 4; ++q) {
          const float4 w = w4[q];
          acc[4 * q + 0] = fmaf(v, w.x, acc[4 * q + 0]);
          acc[4 * q + 1] = fmaf(v, w.y, acc[4 * q + 1]);
          acc[4 * q + 2] = fmaf(v, w.z, acc[4 * q + 2]);
          acc[4 * q + 3] = fmaf(v, w.w, acc[4 * q + 3]);
        }
      };
      if constexpr (KW > 0) {
#pragma unroll
        for (int kx = 0; kx < KW; ++kx) tap(kx);
      } else {
        for (int kx = 0; kx < g.kw; ++kx) tap(kx);
      }
    }
  }
  uint16_t* op = out + b * g.os[0] + (long long)oy * g.os[2] + (long long)ox * g.os[3];
#pragma unroll
  for (int o = 0; o < NOUT; ++o)
    if (o < g.NOUTr) op[o * g.os[1]] = f2bf(acc[o]);
}

// wt[i][ky][kx][o] (o padded to noutp with zeros) from OIHW bf16 weights
__global__ void direct_weight_kernel(const uint16_t* __restrict__ w, int Cout, int Cin, int kh, int kw, int dgrad,
                                     int noutp, float* __restrict__ wt) {
  const int nin = dgrad ? Cout : Cin, nout = dgrad ? Cin : Cout;
  const int total = nin * kh * kw * noutp;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int o = e % noutp;
    int r = e / noutp;
    const int kx = r % kw;
    r /= kw;
    const int ky = r % kh;
    const int i = r / kh;
    float v = 0.f;
    if (o < nout) {
      if (dgrad)  // i = co, o = ci, taps flipped
        v = bf2f(w[((long long)(i * Cin + o) * kh + (kh - 1 - ky)) * kw + (kw - 1 - kx)]);
      else  // i = ci, o = co
        v = bf2f(w[((long long)(o * Cin + i) * kh + ky) * kw + kx]);
    }
    wt[e] = v;
  }
}

constexpr int kDirectMaxSmem = 200 * 1024;

int pad_out(int n) { return n <= 4 ? 4 : n <= 8 ? 8 : n <= 16 ? 16 : n <= 32 ? 32 : n <= 64 ? 64 : 0; }

size_t direct_smem(const DirectGeom& g, int noutp) {
  return size_t(g.NIN) * g.kh * g.kw * noutp * 4 + size_t(g.NIN) * g.IH * g.IW * 2;
}

// Tile of at most `threads` threads whose sides split the output evenly.
void direct_tile(DirectGeom& g, int threads) {
  const int nx = (g.Wo + 31) / 32;
  g.TW = (g.Wo + nx - 1) / nx;
  int th = std::max(1, std::min(g.Ho, threads / g.TW));
  const int ny = (g.Ho + th - 1) / th;
  g.TH = (g.Ho + ny - 1) / ny;
  g.tiles_x = (g.Wo + g.TW - 1) / g.TW;
  g.tiles_y = (g.Ho + g.TH - 1) / g.TH;
  g.IH = (g.TH - 1) * g.sy + (g.kh - 1) * g.dy + 1;
  g.IW = (g.TW - 1) * g.sx + (g.kw - 1) * g.dx + 1;
}

template <int NOUT, int KW>
b2_status launch_direct_kw(const uint16_t* in, const float* wt, const uint16_t* bias, const DirectGeom& g,
                           uint16_t* out, cudaStream_t st) {
  const size_t smem = direct_smem(g, NOUT);
  auto kern = direct_conv_kernel<NOUT, KW>;
  // once per device, at the largest size accepted (no attribute calls per
  // launch: they must not run inside a CUDA graph capture)
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  if (!configured[dev]) {
    B2_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDirectMaxSmem),
                      "cudaFuncSetAttribute(direct conv smem)"));
    configured[dev] = true;
  }
  const long long blocks = (long long)g.B * g.tiles_x * g.tiles_y;
  kern<<<unsigned(blocks), g.TH * g.TW, smem, st>>>(in, wt, bias, g, out);
  return check_cuda(cudaGetLastError(), "direct conv launch");
}

template <int NOUT>
b2_status launch_direct(const uint16_t* in, const float* wt, const uint16_t* bias, const DirectGeom& g, uint16_t* out,
                        cudaStream_t st) {
  switch (g.kw) {
    case 3: return launch_direct_kw<NOUT, 3>(in, wt, bias, g, out, st);
    case 5: return launch_direct_kw<NOUT, 5>(in, wt, bias, g, out, st);
    case 7: return launch_direct_kw<NOUT, 7>(in, wt, bias, g, out, st);
    case 9: return launch_direct_kw<NOUT, 9>(in, wt, bias, g, out, st);
    default: return launch_direct_kw<NOUT, 0>(in, wt, bias, g, out, st);
  }
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

size_t b2_direct_conv_weight_floats(int64_t Cout, int64_t Cin, int kh, int kw, int dgrad) {
  const int np = pad_out(int(dgrad ? Cin : Cout));
  if (np == 0 || Cout <= 0 || Cin <= 0 || kh <= 0 || kw <= 0) return 0;
  return size_t(dgrad ? Cout : Cin) * kh * kw * np;
}

b2_status b2_direct_conv_weight(const void* w, int64_t Cout, int64_t Cin, int kh, int kw, int dgrad, float* wt,
                                void* stream) {
  const size_t n = b2_direct_conv_weight_floats(Cout, Cin, kh, kw, dgrad);
  if (!w || !wt || n == 0) return set_error(B2_ERR_INVALID, "b2_direct_conv_weight: bad arguments");
  const int np = pad_out(int(dgrad ? Cin : Cout));
  const int blocks = int(std::min<size_t>((n + 255) / 256, 1024));
  direct_weight_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(w), int(Cout), int(Cin), kh, kw, dgrad, np, wt);
  return check_cuda(cudaGetLastError(), "direct conv weight launch");
}

b2_status b2_direct_conv_bf16(const void* in, const int64_t* in_strides, int64_t B, int64_t NIN, int64_t Hin,
                              int64_t Win, const float* wt, int kh, int kw, int sy, int sx, int py, int px, int dy,
                              int dx, const void* bias, void* out, const int64_t* out_strides, int64_t NOUT,
                              int64_t Ho, int64_t Wo, void* stream) {
  if (!in || !wt || !out || !in_strides || !out_strides)
    return set_error(B2_ERR_INVALID, "b2_direct_conv_bf16: null pointer");
  if (B < 0 || NIN <= 0 || Hin <= 0 || Win <= 0 || NOUT <= 0 || Ho < 0 || Wo < 0 || kh <= 0 || kw <= 0 || sy <= 0 ||
      sx <= 0 || dy <= 0 || dx <= 0 || py < 0 || px < 0)
    return set_error(B2_ERR_INVALID, "b2_direct_conv_bf16: bad geometry");
  const int np = pad_out(int(NOUT));
  if (np == 0) return set_error(B2_ERR_UNSUPPORTED, "b2_direct_conv_bf16: more than 64 output channels");
  if (B == 0 || Ho == 0 || Wo == 0) return B2_OK;
  if (B > INT32_MAX || Hin > INT32_MAX / 4 || Win > INT32_MAX / 4 || Ho > INT32_MAX / 4 || Wo > INT32_MAX / 4 ||
      NIN > 4096)
    return set_error(B2_ERR_UNSUPPORTED, "b2_direct_conv_bf16: too large");
  DirectGeom g{};
  g.B = int(B);
  g.NIN = int(NIN);
  g.Hin = int(Hin);
  g.Win = int(Win);
  g.NOUTr = int(NOUT);
  g.Ho = int(Ho);
  g.Wo = int(Wo);
  g.kh = kh;
  g.kw = kw;
  g.sy = sy;
  g.sx = sx;
  g.py = py;
  g.px = px;
  g.dy = dy;
  g.dx = dx;
  for (int k = 0; k < 4; ++k) {
    g.is[k] = in_strides[k];
    g.os[k] = out_strides[k];
  }
  // few output channels: small tiles, so that enough CTAs (and warps) are
  // resident to hide the shared-memory latency of the long reduction
  direct_tile(g, np <= 8 ? 64 : 256);
  if (direct_smem(g, np) > size_t(kDirectMaxSmem))
    return set_error(B2_ERR_UNSUPPORTED, "b2_direct_conv_bf16: %zu bytes of shared memory needed",
                     direct_smem(g, np));
  if ((long long)g.B * g.tiles_x * g.tiles_y >= (1LL << 31))
    return set_error(B2_ERR_UNSUPPORTED, "b2_direct_conv_bf16: too many tiles");
  auto* ip = static_cast<const uint16_t*>(in);
  auto* bp = static_cast<const uint16_t*>(bias);
  auto* op = static_cast<uint16_t*>(out);
  auto st = static_cast<cudaStream_t>(stream);
  switch (np) {
    case 4: return launch_direct<4>(ip, wt, bp, g, op, st);
    case 8: return launch_direct<8>(ip, wt, bp, g, op, st);
    case 16: return launch_direct<16>(ip, wt, bp, g, op, st);
    case 32: return launch_direct<32>(ip, wt, bp, g, op, st);
    default: return launch_direct<64>(ip, wt, bp, g, op, st);
  }
}

}  // extern "C"
