/*
 * CPU oracle for the offloaded BF16 training path -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * this library, and only as the checker.  The product path never calls it.
 *
 * Plain-C restatement of the reference's algorithms, each function citing the
 * reference file:line it follows (paths within mistrjirka/pytorch-XDNA2):
 *   - padded-grid row packing    xdna_train/_designs/conv3x3w_host.py:32-47
 *   - weight K order (fwd, dX)   conv3x3w_host.py:66-78, _native/conv_pack.cpp:470-519
 *   - conv as GEMM on rows       xdna_train/_designs/conv3x3w.py:10-16 (taps =
 *                                row offsets dy*(W+2)+dx), unpack conv3x3w_host.py:81-87
 *   - wgrad                      xdna_train/_designs/conv3x3w_dw.py:1-21
 *   - region kernels             xdna_train/_native/region_kernels.cpp:52-307
 *   - BatchNorm + activation     region_kernels.cpp:309-460
 * Parity pins: tests/test_oracle_golden.py checks the packers against vectors
 * generated from conv3x3w_host.py itself (tests/golden/make_golden.py) and the
 * region kernels bit-exactly against the reference's region_kernels.cpp built
 * from its own source (oracle/Makefile -> oracle/_ref); the conv/GEMM results
 * are checked against the reference's CPU path (stock PyTorch CPU kernels,
 * torch_xdna_device.cpp:4594-4603, 4862-4873).
 *
 * Accumulation is in double, so the oracle is a tighter reference than the
 * fp32-accumulating kernels it checks.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bf2f(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

/* conv3x3w_host.py:32-47 (pack_input), rows before the NPU's group split:
 * rows[(b*(H+2)+y+1)*(W+2)+x+1][c] = x[b][c][y][x]; zeros elsewhere. */
void oracle_pack_rows(const uint16_t* x, int B, int C, int H, int W, int chunks, uint16_t* rows) {
  const int wp = W + 2, cp = chunks * 64;
  const long long m_total = (long long)B * (H + 2) * wp;
  memset(rows, 0, (size_t)m_total * cp * sizeof(uint16_t));
  for (int b = 0; b < B; ++b)
    for (int c = 0; c < C; ++c)
      for (int y = 0; y < H; ++y)
        for (int xx = 0; xx < W; ++xx)
          rows[((long long)(b * (H + 2) + y + 1) * wp + xx + 1) * cp + c] =
              x[(((long long)b * C + c) * H + y) * W + xx];
}

/* conv3x3w_host.py:66-78 K order (chunk, dy, dx, c); dgrad reads
 * w'[ci][co][dy][dx] = w[co][ci][2-dy][2-dx] (conv_pack.cpp:470-473). */
void oracle_pack_weight(const uint16_t* w, int Cout, int Cin, int chunks, int dgrad, uint16_t* wk) {
  const int n_rows = dgrad ? Cin : Cout, kred = dgrad ? Cout : Cin, kt = chunks * 576;
  for (int n = 0; n < n_rows; ++n)
    for (int chunk = 0; chunk < chunks; ++chunk)
      for (int tap = 0; tap < 9; ++tap)
        for (int c = 0; c < 64; ++c) {
          const int cc = chunk * 64 + c;
          uint16_t v = 0;
          if (cc < kred)
            v = dgrad ? w[((long long)cc * Cin + n) * 9 + (8 - tap)] : w[((long long)n * Cin + cc) * 9 + tap];
          wk[(long long)n * kt + chunk * 576 + tap * 64 + c] = v;
        }
}

/* The conv3x3w computation: output row p (padded grid, top-left origin) =
 * sum over K of rows[p + dy*(W+2)+dx][chunk*64+c] * wk[co][k], then the
 * unpack of conv3x3w_host.py:81-87 keeps y < H, x < W.  Output NCHW float. */
void oracle_conv_rows(const uint16_t* rows, const uint16_t* wk, const uint16_t* bias, int B, int Cin,
                      int H, int W, int Cout, int relu, float* y) {
  const int wp = W + 2, hp = H + 2, chunks = (Cin + 63) / 64, cp = chunks * 64, kt = chunks * 576;
  const long long m_total = (long long)B * hp * wp;
  for (int b = 0; b < B; ++b)
    for (int yy = 0; yy < H; ++yy)
      for (int xx = 0; xx < W; ++xx) {
        const long long p = ((long long)b * hp + yy) * wp + xx;
        for (int co = 0; co < Cout; ++co) {
          double acc = 0.0;
          for (int chunk = 0; chunk < chunks; ++chunk)
            for (int tap = 0; tap < 9; ++tap) {
              const long long r = p + (tap / 3) * wp + (tap % 3);
              if (r >= m_total) continue;
              const uint16_t* a = rows + r * cp + chunk * 64;
              const uint16_t* bw = wk + (long long)co * kt + chunk * 576 + tap * 64;
              for (int c = 0; c < 64; ++c) acc += (double)bf2f(a[c]) * (double)bf2f(bw[c]);
            }
          if (bias) acc += bf2f(bias[co]);
          if (relu && acc < 0) acc = 0;
          y[(((long long)b * Cout + co) * H + yy) * W + xx] = (float)acc;
        }
      }
}

/* conv3x3w_dw.py:1-21: dW[co][ci][dy][dx] = sum_p dY[p][co] * X[p + dy(W+2)+dx][ci]
 * with dY in output (top-left) convention: dY row p = input-convention row
 * p + W + 3 of the packed dY.  Output OIHW float. */
void oracle_wgrad_rows(const uint16_t* dy_rows, const uint16_t* x_rows, int B, int Cin, int H, int W,
                       int Cout, float* dw) {
  const int wp = W + 2, hp = H + 2;
  const int cpo = ((Cout + 63) / 64) * 64, cpi = ((Cin + 63) / 64) * 64;
  const long long m_total = (long long)B * hp * wp;
  for (int co = 0; co < Cout; ++co)
    for (int ci = 0; ci < Cin; ++ci)
      for (int tap = 0; tap < 9; ++tap) {
        const long long off = (tap / 3) * wp + (tap % 3);
        double acc = 0.0;
        for (long long p = 0; p < m_total; ++p) {
          const long long rd = p + W + 3, rx = p + off;
          if (rd >= m_total || rx >= m_total) continue;
          const float d = bf2f(dy_rows[rd * cpo + co]);
          if (d == 0.0f) continue;
          acc += (double)d * (double)bf2f(x_rows[rx * cpi + ci]);
        }
        dw[((long long)co * Cin + ci) * 9 + tap] = (float)acc;
      }
}

/* D[m][n] = alpha * sum_k A[m][k] * B[k][n] + beta * C[m][n] (row-major, fp32 out). */
void oracle_gemm(const uint16_t* A, const uint16_t* Bm, const float* Cm, int M, int N, int K, float alpha,
                 float beta, float* D) {
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      double acc = 0.0;
      for (int k = 0; k < K; ++k) acc += (double)bf2f(A[(long long)m * K + k]) * (double)bf2f(Bm[(long long)k * N + n]);
      double v = alpha * acc;
      if (beta != 0.0f) v += (double)beta * Cm[(long long)m * N + n];
      D[(long long)m * N + n] = (float)v;
    }
}

/* ---- region kernels: region_kernels.cpp:52-307 ---------------------------- */

static int nan_or_gt(float v, float m) { return (v > m) ? 1 : (v != v); }

double oracle_sqdiff_sum(const uint16_t* a, const uint16_t* b, long long n) {
  double t = 0.0;
  for (long long i = 0; i < n; ++i) {
    const double d = (double)bf2f(a[i]) - (double)bf2f(b[i]);
    t += d * d;
  }
  return t;
}

void oracle_relu(const uint16_t* a, uint16_t* r, long long n) {
  for (long long i = 0; i < n; ++i) r[i] = (bf2f(a[i]) <= 0.0f) ? 0 : a[i];
}

void oracle_relu_maxpool2(const uint16_t* a, uint16_t* r, uint16_t* p, long long planes, long long H, long long W) {
  const long long Ho = H / 2, Wo = W / 2;
  oracle_relu(a, r, planes * H * W);
  for (long long pl = 0; pl < planes; ++pl)
    for (long long y = 0; y < Ho; ++y)
      for (long long x = 0; x < Wo; ++x) {
        const uint16_t* r0 = r + pl * H * W + (2 * y) * W + 2 * x;
        const uint16_t e00 = r0[0], e01 = r0[1], e10 = r0[W], e11 = r0[W + 1];
        uint16_t m;
        if ((W & 1) == 0) { /* vertical pairs, then horizontal: region_kernels.cpp:98-122 */
          const float f00 = bf2f(e00), f01 = bf2f(e01), f10 = bf2f(e10), f11 = bf2f(e11);
          const int s0 = nan_or_gt(f10, f00), s1 = nan_or_gt(f11, f01);
          const uint16_t m0 = s0 ? e10 : e00, m1 = s1 ? e11 : e01;
          const float v0 = s0 ? f10 : f00, v1 = s1 ? f11 : f01;
          m = nan_or_gt(v1, v0) ? m1 : m0;
        } else { /* scan order: region_kernels.cpp:169-180 */
          const uint16_t c[3] = {e01, e10, e11};
          float mv;
          m = e00;
          mv = bf2f(m);
          for (int k = 0; k < 3; ++k)
            if (nan_or_gt(bf2f(c[k]), mv)) { m = c[k]; mv = bf2f(c[k]); }
        }
        p[pl * Ho * Wo + y * Wo + x] = m;
      }
}

void oracle_addtap(const uint16_t* base, const uint16_t* a, const uint16_t* b, uint16_t* out, long long n,
                   float scale) {
  for (long long i = 0; i < n; ++i) {
    const float t = scale * (bf2f(a[i]) - bf2f(b[i]));
    out[i] = f2bf(base ? bf2f(base[i]) + t : t);
  }
}

void oracle_relu_bwd(const uint16_t* r, const uint16_t* base, const uint16_t* a, const uint16_t* b,
                     uint16_t* out, long long n, float scale) {
  for (long long i = 0; i < n; ++i) {
    float g = 0.0f;
    if (base) g = bf2f(base[i]);
    if (a) g += scale * (bf2f(a[i]) - bf2f(b[i]));
    out[i] = (bf2f(r[i]) <= 0.0f) ? 0 : f2bf(g);
  }
}

void oracle_maxpool2_bwd(const uint16_t* x, const uint16_t* g, uint16_t* out, long long planes, long long H,
                         long long W) {
  const long long Ho = H / 2, Wo = W / 2;
  memset(out, 0, (size_t)(planes * H * W) * sizeof(uint16_t));
  for (long long pl = 0; pl < planes; ++pl)
    for (long long y = 0; y < Ho; ++y)
      for (long long xo = 0; xo < Wo; ++xo) {
        const long long base = pl * H * W + (2 * y) * W + 2 * xo;
        const long long off[4] = {0, 1, W, W + 1};
        int best = 0;
        float mv = bf2f(x[base]);
        for (int k = 1; k < 4; ++k) {
          const float v = bf2f(x[base + off[k]]);
          if (nan_or_gt(v, mv)) { best = k; mv = v; }
        }
        out[base + off[best]] = g[pl * Ho * Wo + y * Wo + xo];
      }
}

/* ---- Adam / AdamW, fp32 ----------------------------------------------------
 * PyTorch's Adam/AdamW definition in the operation order of its CPU
 * _fused_adam_ kernel (the reference's path, torch_xdna_device.cpp:5196-5198):
 * m = fma(1-b1, g-m, m); v = fma((1-b2)g, g, b2 v); AdamW decay p *= 1-lr*wd;
 * coefficients formed in double, rounded to float once. */
void oracle_adam_f32(float* p, const float* g_in, float* m, float* v, float* vmax, long long n, float step,
                     float lr, float beta1, float beta2, float wd, float eps, int amsgrad, int maximize,
                     int adamw) {
  const double bc1 = 1.0 - pow((double)beta1, (double)step), bc2 = 1.0 - pow((double)beta2, (double)step);
  const float step_size = (float)((double)lr / bc1), bc2_sqrt = (float)sqrt(bc2);
  const float omb1 = (float)(1.0 - (double)beta1), omb2 = (float)(1.0 - (double)beta2);
  const float decay = (float)(1.0 - (double)lr * (double)wd);
  for (long long i = 0; i < n; ++i) {
    float g = maximize ? -g_in[i] : g_in[i];
    float pp = p[i];
    if (wd != 0.0f) {
      if (adamw) pp = pp * decay;
      else g = fmaf(wd, pp, g);
    }
    m[i] = fmaf(omb1, g - m[i], m[i]);
    {
      const float gs = omb2 * g, bv = beta2 * v[i];
      v[i] = fmaf(gs, g, bv);
    }
    float vv = v[i];
    if (amsgrad) {
      vv = vmax[i] > v[i] ? vmax[i] : v[i];
      vmax[i] = vv;
    }
    {
      const float denom = sqrtf(vv) / bc2_sqrt + eps;
      const float upd = step_size * m[i];
      pp = pp - upd / denom;
    }
    p[i] = pp;
  }
}

/* ---- training BatchNorm2d + LeakyReLU/ReLU: region_kernels.cpp:309-460 -----
 * Contiguous NCHW bf16 [N, C, HW].  Statistics over (N, HW) per channel in
 * double (two passes: mean, then squared deviations), so the oracle is tighter
 * than the reference's fp32 plane sums merged with Chan's formula; invstd =
 * 1/sqrt(var + eps); running statistics (bf16) move by `factor` towards the
 * mean and the unbiased variance.  The elementwise expressions are the
 * reference's, in fp32 with one rounding each and no contraction:
 *   y  = act(x*scale + shift), scale = w*invstd, shift = b - mean*scale,
 *        act(z) = z > 0 ? z : z*slope
 *   dz = (y > 0 or (relu and y is NaN)) ? dy : dy*slope
 *   dx = (w*invstd) * ((dz - sum(dz)/M) - xhat*(sum(dz*xhat)/M)),
 *        xhat = (x - mean)*invstd. */
#if defined(__FP_FAST_FMAF)
#error "the BN oracle needs fp32 expressions without FMA contraction"
#endif

void oracle_bn_fwd(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* rm, uint16_t* rv,
                   uint16_t* y, float* mean_out, float* invstd_out, long long N, long long C, long long HW,
                   float eps, float slope, float factor, int update) {
  const double M = (double)N * (double)HW;
  for (long long c = 0; c < C; ++c) {
    double s = 0.0;
    for (long long n = 0; n < N; ++n)
      for (long long i = 0; i < HW; ++i) s += (double)bf2f(x[(n * C + c) * HW + i]);
    const double mean = s / M;
    double q = 0.0;
    for (long long n = 0; n < N; ++n)
      for (long long i = 0; i < HW; ++i) {
        const double d = (double)bf2f(x[(n * C + c) * HW + i]) - mean;
        q += d * d;
      }
    const double var = q / M;
    mean_out[c] = (float)mean;
    invstd_out[c] = (float)(1.0 / sqrt(var + (double)eps));
    if (update) {
      const double unbiased = M > 1.0 ? var * M / (M - 1.0) : var;
      const double f = (double)factor;
      rm[c] = f2bf((float)((1.0 - f) * (double)bf2f(rm[c]) + f * mean));
      rv[c] = f2bf((float)((1.0 - f) * (double)bf2f(rv[c]) + f * unbiased));
    }
    const float scale = (w ? bf2f(w[c]) : 1.0f) * invstd_out[c];
    const float shift = (b ? bf2f(b[c]) : 0.0f) - mean_out[c] * scale;
    for (long long n = 0; n < N; ++n)
      for (long long i = 0; i < HW; ++i) {
        const long long o = (n * C + c) * HW + i;
        const float z = bf2f(x[o]) * scale + shift;
        y[o] = f2bf(z > 0.0f ? z : z * slope);
      }
  }
}

static float bn_dz(float g, float yv, float slope, int relu) {
  return ((yv > 0.0f) || (relu && yv != yv)) ? g : g * slope;
}

void oracle_bn_bwd(const uint16_t* dy, const uint16_t* y, const uint16_t* x, const uint16_t* w,
                   const float* mean, const float* invstd, uint16_t* dx, uint16_t* dw, uint16_t* db,
                   long long N, long long C, long long HW, float slope, int relu) {
  const double M = (double)N * (double)HW;
  for (long long c = 0; c < C; ++c) {
    const float mc = mean[c], is = invstd[c];
    double a = 0.0, bs = 0.0;
    for (long long n = 0; n < N; ++n)
      for (long long i = 0; i < HW; ++i) {
        const long long o = (n * C + c) * HW + i;
        const float dz = bn_dz(bf2f(dy[o]), bf2f(y[o]), slope, relu);
        const float xhat = (bf2f(x[o]) - mc) * is;
        a += (double)dz;
        bs += (double)dz * (double)xhat;
      }
    if (db) db[c] = f2bf((float)a);
    if (dw) dw[c] = f2bf((float)bs);
    if (!dx) continue;
    const float k1 = (float)(a / M), k2 = (float)(bs / M);
    const float ws = (w ? bf2f(w[c]) : 1.0f) * is;
    for (long long n = 0; n < N; ++n)
      for (long long i = 0; i < HW; ++i) {
        const long long o = (n * C + c) * HW + i;
        const float dz = bn_dz(bf2f(dy[o]), bf2f(y[o]), slope, relu);
        const float xhat = (bf2f(x[o]) - mc) * is;
        dx[o] = f2bf(ws * ((dz - k1) - xhat * k2));
      }
  }
}
