/*
 * b2.h -- C ABI of libxdna_b200.so, the sm_100a kernel library behind the
 * `xdna` PyTorch device of this package.
 *
 * Plain pointers and sizes only: no torch types, no CUDA types.  Streams are
 * passed as `void*` (a cudaStream_t; NULL is the legacy default stream).  All
 * pointers except the explicitly host-side ones are device (HBM) pointers.
 *
 * Error convention (mirrors the reference's C shims, which return NULL or
 * nonzero and keep the message in a thread-local string --
 * xdna_train/_vendor/xrt_shim/xrt_shim.h:2-3, xrt_shim.cpp:235-238):
 * every call returns B2_OK (0) or a nonzero b2_status; the message of the
 * last failure on the calling thread is b2_last_error().  Launches are
 * asynchronous: a kernel that detects a problem on the device (a pipeline
 * wait that ran out of its time limit) records a code in a per-device status
 * word read by b2_device_status().
 *
 * Layouts (the reference's conv3x3w host layouts, xdna_train/_designs/
 * conv3x3w_host.py:15-47, without the NPU's group/halo duplication):
 *   padded-grid rows  : X_rows[B*(H+2)*(W+2)][chunks*64] bf16.  Pixel (b,y,x)
 *                       is row (b*(H+2)+y+1)*(W+2)+x+1; the border rows and
 *                       the channels >= C are zero.  Output pixel (b,y,x) of a
 *                       3x3/s1/p1 conv is row p=(b*(H+2)+y)*(W+2)+x and its tap
 *                       (dy,dx) reads row p + dy*(W+2) + dx.
 *   conv weights      : Wk[Cout][chunks*9*64] bf16 with K order
 *                       (chunk, dy, dx, c) (conv3x3w_host.py:66-78); the
 *                       dgrad copy reads w'[ci][co][dy][dx] = w[co][ci][2-dy][2-dx]
 *                       (xdna_train/_native/conv_pack.cpp:470-473).
 */
#ifndef XDNA_B200_B2_H
#define XDNA_B200_B2_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int b2_status;

enum {
  B2_OK = 0,
  B2_ERR_INVALID = 1,      /* bad argument (shape, alignment, null pointer) */
  B2_ERR_CUDA = 2,         /* a CUDA runtime call failed */
  B2_ERR_UNSUPPORTED = 3,  /* valid request this library does not serve */
  B2_ERR_TIMEOUT = 4,      /* device-side wait ran out of its limit */
  B2_ERR_WORKSPACE = 5     /* workspace too small */
};

/* dtype codes used where a pointer can hold more than one element type */
enum { B2_BF16 = 0, B2_F32 = 1 };

/* ---- runtime ------------------------------------------------------------ */

/* Thread-local message of the last failed call on this thread ("" if none).
 * Replaces shim_last_error() (xdna_train/_vendor/xrt_shim/xrt_shim.h:157). */
const char* b2_last_error(void);

/* Library ABI version (increments on any signature change). */
int b2_abi_version(void);

/* Reads and clears the device-side status word of `device` (0 = no error,
 * else a b2_status recorded by a kernel).  Synchronizes the device.
 * Replaces the dispatch-deadline check of shim_run_wait
 * (xdna_train/_vendor/xrt_shim/xrt_shim.cpp:174-233). */
b2_status b2_device_status(int device, int* code);

/* ---- layout packers (replace xdna_train/_native/conv_pack.cpp) ---------- */

/* Strided bf16 activation x (element strides sn, sc, sh, sw; NCHW and NHWC
 * are both strided views) -> padded-grid rows [B*(H+2)*(W+2)][chunks*64].
 * Writes every row (borders and padded channels zero), so `rows` needs no
 * prior memset.  chunks >= ceil(C/64).
 * Replaces xdna_conv3x3w_pack_input_bf16 / _strips_range_bf16
 * (conv_pack.cpp:352-392, 632-700). */
b2_status b2_pack_rows_bf16(const void* x, int64_t sn, int64_t sc, int64_t sh,
                            int64_t sw, int B, int C, int H, int W, int chunks,
                            void* rows, void* stream);

/* b2_pack_rows_bf16 of dY that also produces the conv bias gradient
 * dbias[c] = sum over (b, y, x) of x[b][c][y][x] (dtype B2_BF16 or B2_F32),
 * taken from the tile the packer already holds (no second pass over dY on the
 * NCHW path), reduced in a fixed order: deterministic.  Workspace:
 * b2_pack_rows_dbias_workspace_bytes().  Replaces the reference's CPU dbias
 * (mask[2] of convolution_backward, torch_xdna_device.cpp:4828-4878). */
size_t b2_pack_rows_dbias_workspace_bytes(int B, int C, int H, int W);
b2_status b2_pack_rows_dbias_bf16(const void* x, int64_t sn, int64_t sc,
                                  int64_t sh, int64_t sw, int B, int C, int H,
                                  int W, int chunks, void* rows, void* dbias,
                                  int dbias_dtype, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* dbias of a channels-last dY read in place (the conv bias gradient when no
 * padded-row copy of dY is made): out[c] = sum over (b, y, x) of
 * x[b][y][x][c] (pixels dense: sh == W*sw, sn == H*sh, sw >= C), fp32 sums
 * over fixed 64-pixel groups added in group order (deterministic), rounded
 * once to out_dtype (B2_BF16 or B2_F32).  Workspace:
 * b2_channel_sum_nhwc_workspace_bytes().  Replaces the reference's CPU dbias
 * (mask[2] of convolution_backward, torch_xdna_device.cpp:4828-4878). */
size_t b2_channel_sum_nhwc_workspace_bytes(int B, int C, int H, int W);
b2_status b2_channel_sum_nhwc_bf16(const void* x, int64_t sn, int64_t sh,
                                   int64_t sw, int B, int C, int H, int W,
                                   void* out, int out_dtype, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* OIHW bf16 weight [Cout][Cin][3][3] -> Wk[Cout][chunks*9*64], K order
 * (chunk, dy, dx, c), zero for c >= Cin.  chunks >= ceil(Cin/64).
 * Replaces the K ordering of xdna_conv3x3w_pack_weights_bfp16
 * (conv_pack.cpp:398-443) without the NPU's BFP16 encode. */
b2_status b2_pack_weight_fwd_bf16(const void* w, int Cout, int Cin, int chunks,
                                  void* wk, void* stream);

/* dgrad weights: Wk'[Cin][chunks_o*9*64] with w'[ci][co][dy][dx] =
 * w[co][ci][2-dy][2-dx], chunks_o >= ceil(Cout/64).
 * Replaces xdna_conv3x3w_pack_weights_dx_bfp16 (conv_pack.cpp:474-519). */
b2_status b2_pack_weight_dgrad_bf16(const void* w, int Cout, int Cin,
                                    int chunks_o, void* wk, void* stream);

/* Either packing (dgrad != 0: the dgrad form) from a weight read through its
 * element strides {co, ci, ky, kx} -- OIHW is {9*Cin, 9, 3, 1}, a
 * channels-last OHWI weight {9*Cin, 1, 3*Cin, Cin} -- so a channels-last
 * model's weights need no contiguous copy first.  Same output as the two
 * calls above (conv_pack.cpp:398-443, 474-519). */
b2_status b2_pack_weight_strided_bf16(const void* w, const int64_t* strides,
                                      int Cout, int Cin, int chunks, int dgrad,
                                      void* wk, void* stream);

/* Dense bf16 NCHW [B][C][H*W] <-> NHWC [B][H*W][C] transposes.
 * Replace xdna_pack_conv3x3_halo_padded_bf16 / xdna_yxbc_to_channels_last_bf16
 * (conv_pack.cpp:19-112) for the channels-last boundary. */
b2_status b2_nchw_to_nhwc_bf16(const void* src, void* dst, int B, int C,
                               int HW, void* stream);
b2_status b2_nhwc_to_nchw_bf16(const void* src, void* dst, int B, int C,
                               int HW, void* stream);

/* ---- 3x3 / stride 1 / pad 1 convolution (tcgen05 implicit GEMM) ---------- */

/* y[b][co][y][x] (strided bf16, element strides ysn..ysw) =
 *   bias[co] + sum_{ci,dy,dx} x[b][ci][y+dy-1][x+dx-1] * w[co][ci][dy][dx]
 * from padded-grid rows of x (chunks = ceil(Cin/64)) and Wk from
 * b2_pack_weight_fwd_bf16.  bias may be NULL (bf16 [Cout]); relu != 0 clamps
 * at zero.  FP32 accumulation in tensor memory, one bf16 rounding.
 * Replaces XdnaConv3x3wRuntime::run (xdna_train/_native/
 * torch_xdna_device.cpp:2317-2483) and the unpack of conv_pack.cpp:447-466. */
b2_status b2_conv3x3_fwd(const void* x_rows, const void* wk, const void* bias,
                         void* y, int64_t ysn, int64_t ysc, int64_t ysh,
                         int64_t ysw, int B, int Cin, int H, int W, int Cout,
                         int relu, void* stream);

/* dgrad: dx = conv3x3(dy, w') from padded-grid rows of dy (chunks =
 * ceil(Cout/64)) and Wk' from b2_pack_weight_dgrad_bf16; dx strided bf16.
 * Replaces XdnaConv3x3wRuntime::input_grad (torch_xdna_device.cpp:2515-2522). */
b2_status b2_conv3x3_dgrad(const void* dy_rows, const void* wk_dgrad, void* dx,
                           int64_t sn, int64_t sc, int64_t sh, int64_t sw,
                           int B, int Cout, int H, int W, int Cin, void* stream);

/* Workspace bytes b2_conv3x3_wgrad needs for this shape (fp32 split-K
 * partial sums; 0 is never returned). */
size_t b2_conv3x3_wgrad_workspace_bytes(int B, int Cin, int H, int W, int Cout);

/* wgrad: dw[co][ci][dy][dx] = sum_{b,y,x} dy[b][co][y][x] *
 * x[b][ci][y+dy-1][x+dx-1], from the padded-grid rows of dy (chunks_o =
 * ceil(Cout/64)) and of x (chunks_i = ceil(Cin/64)), the same buffers the
 * forward and dgrad read.  dw is OIHW, dtype B2_BF16 or B2_F32.  FP32
 * accumulation; the split-K reduction is deterministic (fixed order).
 * Replaces XdnaConv3x3wDwRuntime::compute (torch_xdna_device.cpp:2683-2751). */
b2_status b2_conv3x3_wgrad(const void* dy_rows, const void* x_rows, void* dw,
                           int dw_dtype, int B, int Cin, int H, int W, int Cout,
                           void* workspace, size_t workspace_bytes,
                           void* stream);

/* The three directions with channels-last activations read in place: x / dy
 * are bf16 [B][H][W][C] views with channel stride 1 and element strides
 * (sn, sh, sw), C and the strides multiples of 8, 16-byte aligned base.  The
 * kernels fetch them through an im2col TMA map whose pixel box is the
 * zero-padded grid, so they read exactly the rows b2_pack_rows_bf16 would
 * have written, without that pass over the activation (same results, bit for
 * bit).  Weights and outputs as in the padded-row entry points; wgrad's
 * workspace size is b2_conv3x3_wgrad_workspace_bytes.  Replace the same
 * reference functions as b2_conv3x3_fwd / _dgrad / _wgrad together with its
 * channels-last strip packer (conv_pack.cpp:632-700). */
b2_status b2_conv3x3_fwd_nhwc(const void* x, int64_t xsn, int64_t xsh,
                              int64_t xsw, const void* wk, const void* bias,
                              void* y, int64_t ysn, int64_t ysc, int64_t ysh,
                              int64_t ysw, int B, int Cin, int H, int W,
                              int Cout, int relu, void* stream);
b2_status b2_conv3x3_dgrad_nhwc(const void* dy, int64_t dsn, int64_t dsh,
                                int64_t dsw, const void* wk_dgrad, void* dx,
                                int64_t sn, int64_t sc, int64_t sh, int64_t sw,
                                int B, int Cout, int H, int W, int Cin,
                                void* stream);
b2_status b2_conv3x3_wgrad_nhwc(const void* dy, int64_t dsn, int64_t dsh,
                                int64_t dsw, const void* x, int64_t xsn,
                                int64_t xsh, int64_t xsw, void* dw,
                                int dw_dtype, int B, int Cin, int H, int W,
                                int Cout, void* workspace,
                                size_t workspace_bytes, void* stream);

/* b2_conv3x3_wgrad_nhwc with dw written in [Cout][3][3][Cin] order, the
 * storage order of a channels-last weight (OHWI), so that a channels-last
 * model's gradient lands in its parameter's layout without a re-layout copy.
 * Same values, bit for bit.  Replaces the same reference function as
 * b2_conv3x3_wgrad (torch_xdna_device.cpp:2683-2751); the reference allocates
 * that gradient in OIHW order (torch_xdna_device.cpp:4690), which autograd
 * then copies into a channels-last parameter's layout. */
b2_status b2_conv3x3_wgrad_nhwc_ohwi(const void* dy, int64_t dsn, int64_t dsh,
                                     int64_t dsw, const void* x, int64_t xsn,
                                     int64_t xsh, int64_t xsw, void* dw,
                                     int dw_dtype, int B, int Cin, int H,
                                     int W, int Cout, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* Weight gradient that allocates nothing (no counterpart in the reference).
 * Same result as b2_conv3x3_wgrad, but the split-K partial sums live in one
 * fixed device array inside this library instead of a caller workspace, for
 * callers that cannot allocate device memory (a framework that reserved the
 * GPU's memory for its own pool, a loop that must never reach cudaMalloc).
 * The array holds b2_conv3x3_wgrad_noalloc_max_bytes() (16 MiB) on every GPU
 * that loads the library, until exit.  If the usual split plan needs more,
 * fewer splits are used; shapes with 9*Cout*Cin*4 bytes above the limit fail
 * with B2_ERR_WORKSPACE.  The first call on a device looks the array's
 * address up (make it before any stream capture); the address is kept for the
 * lifetime of that device's primary context (not valid after a
 * cudaDeviceReset in the same process).  Calls share the array:
 * calls that overlap on the GPU race and must be serialized by the caller.
 * Calls no cudaMalloc / cudaFree. */
b2_status b2_conv3x3_wgrad_noalloc(const void* dy_rows, const void* x_rows,
                                   void* dw, int dw_dtype, int B, int Cin,
                                   int H, int W, int Cout, void* stream);
size_t b2_conv3x3_wgrad_noalloc_max_bytes(void);

/* ---- dense GEMM (tcgen05) ------------------------------------------------ */

/* For each batch index i < batch:
 *   D_i[m][n] = alpha * sum_k opA(A_i)[m][k] * opB(B_i)[k][n] + beta * C_i[m][n]
 * A, B, D bf16 row-major with leading dims lda, ldb, ldd and batch strides;
 * opA(A) = A ([M][K]) if transA == 0 else A^T (A stored [K][M]); likewise B
 * ([K][N], or [N][K] when transB).  C (may be NULL when beta == 0) is read
 * through element strides c_sm, c_sn, c_sb (0 broadcasts, e.g. a bias row)
 * with dtype c_dtype.  lda/ldb (in elements) must be multiples of 8 and the
 * operand base addresses 16-byte aligned (B2_ERR_UNSUPPORTED otherwise).
 * Replaces XdnaGemmRuntime (torch_xdna_device.cpp:1320-1458), which served
 * three fixed shapes; this serves any shape. */
b2_status b2_gemm_bf16(int transA, int transB, int M, int N, int K, float alpha,
                       const void* A, int64_t lda, int64_t strideA,
                       const void* B, int64_t ldb, int64_t strideB, float beta,
                       const void* C, int c_dtype, int64_t c_sm, int64_t c_sn,
                       int64_t c_sb, void* D, int64_t ldd, int64_t strideD,
                       int batch, void* stream);

/* b2_gemm_bf16 with room for split-K partial sums: when the output has too
 * few 128-row tiles to occupy the SMs (a 512-row activation GEMM with 1024
 * output columns has 32), the reduction is split and the fp32 partials,
 * summed in split order (deterministic), get alpha and beta * C in a second
 * pass.  Workspace bytes: b2_gemm_bf16_workspace_bytes (0: no split for this
 * shape; a smaller or NULL workspace runs unsplit).  Same results as
 * b2_gemm_bf16 up to the fp32 summation order. */
size_t b2_gemm_bf16_workspace_bytes(int M, int N, int K, int batch);
b2_status b2_gemm_bf16_ws(int transA, int transB, int M, int N, int K,
                          float alpha, const void* A, int64_t lda,
                          int64_t strideA, const void* B, int64_t ldb,
                          int64_t strideB, float beta, const void* C,
                          int c_dtype, int64_t c_sm, int64_t c_sn,
                          int64_t c_sb, void* D, int64_t ldd, int64_t strideD,
                          int batch, void* workspace, size_t workspace_bytes,
                          void* stream);

/* ---- multi-tensor fused Adam / AdamW ---------------------------------- */

/* One parameter tensor of a fused step (device pointers; host struct). */
typedef struct b2_adam_tensor {
  void* param;           /* param_dtype */
  const void* grad;      /* param_dtype */
  void* exp_avg;         /* state_dtype */
  void* exp_avg_sq;      /* state_dtype */
  void* max_exp_avg_sq;  /* state_dtype, NULL unless amsgrad */
  const float* step;     /* device fp32 scalar (already incremented) */
  int64_t numel;
} b2_adam_tensor;

typedef struct b2_adam_hparams {
  double lr, beta1, beta2, weight_decay, eps;
  int amsgrad, maximize, adamw;
  int param_dtype;        /* B2_BF16 or B2_F32 */
  int state_dtype;        /* B2_BF16 or B2_F32 */
  const float* lr_tensor; /* device fp32 scalar overriding lr, or NULL */
  const float* grad_scale;/* device fp32 scalar, or NULL */
  const float* found_inf; /* device fp32 scalar, or NULL (nonzero skips) */
} b2_adam_hparams;

/* In-place fused Adam/AdamW over n tensors, one pass per element in FP32
 * (opmath) arithmetic.  Replaces the reference's CPU _fused_adam_ reached
 * through the boxed fallback (torch_xdna_device.cpp:5124-5260). */
b2_status b2_fused_adam(const b2_adam_tensor* tensors, int n,
                        const b2_adam_hparams* hp, void* stream);

/* ---- multi-tensor fused SGD ------------------------------------------- */

/* One parameter tensor of a fused SGD step (device pointers; host struct). */
typedef struct b2_sgd_tensor {
  void* param;            /* param_dtype */
  void* grad;             /* param_dtype; rewritten unscaled when grad_scale is set */
  void* momentum_buffer;  /* param_dtype; may be NULL when momentum == 0 */
  int64_t numel;
} b2_sgd_tensor;

typedef struct b2_sgd_hparams {
  double lr, weight_decay, momentum, dampening;
  int nesterov, maximize, is_first_step; /* first step: the buffer becomes the gradient */
  int param_dtype;        /* B2_BF16 or B2_F32 */
  const float* lr_tensor; /* device fp32 scalar overriding lr, or NULL */
  const float* grad_scale;/* device fp32 scalar, or NULL */
  const float* found_inf; /* device fp32 scalar, or NULL (nonzero skips) */
} b2_sgd_hparams;

/* In-place fused SGD over n tensors in one pass per element, fp32 operands
 * with the hyper-parameters in double (PyTorch's fused-SGD arithmetic):
 * g = grad [/ grad_scale] [negated if maximize] [+ wd * p]; with momentum
 * buf = first ? g : momentum * buf + (1 - dampening) * g and g = nesterov ?
 * g + momentum * buf : buf; p -= lr * g.  Replaces the reference's CPU
 * _fused_sgd_ reached through the boxed fallback and _prefer_fused_optimizer
 * (torch_xdna_device.cpp:5124-5260, xdna_train/device.py:408-436). */
b2_status b2_fused_sgd(const b2_sgd_tensor* tensors, int n,
                       const b2_sgd_hparams* hp, void* stream);

/* ---- fused region kernels (replace xdna_train/_native/region_kernels.cpp) */

/* *out (device double) = sum (a[i]-b[i])^2 over n bf16 elements.
 * region_kernels.cpp:52-71 */
b2_status b2_region_sqdiff_sum_bf16(const void* a, const void* b, int64_t n,
                                    double* out, void* stream);
/* r = relu(a), NaN kept.  region_kernels.cpp:74-87 */
b2_status b2_region_relu_bf16(const void* a, void* r, int64_t n, void* stream);
/* r = relu(a); p = 2x2/2 max-pool of r over [planes][H][W].
 * region_kernels.cpp:150-184 */
b2_status b2_region_relu_maxpool2_bf16(const void* a, void* r, void* p,
                                       int64_t planes, int64_t H, int64_t W,
                                       void* stream);
/* out = bf16(base + scale*(a-b)), base may be NULL.  region_kernels.cpp:187-205 */
b2_status b2_region_addtap_bf16(const void* base, const void* a, const void* b,
                                void* out, int64_t n, float scale, void* stream);
/* out = (r <= 0) ? 0 : bf16(base + scale*(a-b)); base, a/b may be NULL.
 * region_kernels.cpp:212-246 */
b2_status b2_region_relu_bwd_bf16(const void* r, const void* base,
                                  const void* a, const void* b, void* out,
                                  int64_t n, float scale, void* stream);
/* out[argmax of each 2x2 window of x] = g, 0 elsewhere.
 * region_kernels.cpp:248-307 */
b2_status b2_region_maxpool2_bwd_bf16(const void* x, const void* g, void* out,
                                      int64_t planes, int64_t H, int64_t W,
                                      void* stream);

/* ---- 1x1 convolutions, stride 1, no padding (the reference runs them on its
 * CPU path, torch_xdna_device.cpp:4578-4603, 4828-4878) as tcgen05 GEMMs.
 * layout 0 = contiguous NCHW [B][C][HW], 1 = channels-last NHWC [B*HW][C];
 * w = [Cout][Cin] bf16; bias bf16 [Cout] or NULL.  Cin, Cout (and HW for
 * NCHW) multiples of 8; pointers 16-byte aligned.  The weight gradient sums
 * over all B*HW pixels with split-K fp32 partials (workspace of
 * b2_conv1x1_wgrad_workspace_bytes bytes, queried with the target device
 * current) reduced in a fixed order: deterministic; dw dtype B2_BF16 or
 * B2_F32. */
b2_status b2_conv1x1_fwd(const void* x, const void* w, const void* bias,
                         void* y, int layout, int64_t B, int64_t Cin,
                         int64_t HW, int64_t Cout, void* stream);
b2_status b2_conv1x1_dgrad(const void* dy, const void* w, void* dx, int layout,
                           int64_t B, int64_t Cin, int64_t HW, int64_t Cout,
                           void* stream);
size_t b2_conv1x1_wgrad_workspace_bytes(int layout, int64_t B, int64_t Cin,
                                        int64_t HW, int64_t Cout);
b2_status b2_conv1x1_wgrad(const void* dy, const void* x, void* dw,
                           int dw_dtype, int layout, int64_t B, int64_t Cin,
                           int64_t HW, int64_t Cout, void* workspace,
                           size_t workspace_bytes, void* stream);

/* General GEMM with split-K (deterministic, fixed-order reduction):
 * D[M][N] (dtype d_dtype, row stride ldd) = op(A) . op(B), operands as in
 * b2_gemm_bf16 (transA: A stored [K][M]; transB: B stored [N][K]).  Splits fill
 * one wave of SMs; workspace: b2_gemm_splitk_workspace_bytes (0 when a dense
 * fp32 D takes the sums directly). */
size_t b2_gemm_splitk_workspace_bytes(int M, int N, int K, int d_dtype);
b2_status b2_gemm_splitk_bf16(int transA, int transB, int M, int N, int K,
                              const void* A, int64_t lda, const void* B,
                              int64_t ldb, void* D, int d_dtype, int64_t ldd,
                              void* workspace, size_t workspace_bytes,
                              void* stream);

/* ---- general convolutions (any kernel size / stride / padding / dilation,
 * groups 1; the reference's CPU path, torch_xdna_device.cpp:4578-4605,
 * 4828-4878) as GEMMs over an explicit column matrix:
 *   col[P][Kp] (P = B*Ho*Wo, column (ky*kw + kx)*C + ci, zero past K = kh*kw*C,
 *   Kp a multiple of 8 >= K), weights Wk[Cout][Kp] in the same order; the
 *   input gradient from dcol = dY . Wk (fp32) by a gather over the taps in
 *   (ky, kx) order (deterministic).  Tensors through element strides (sb, sc,
 *   sh, sw), so NCHW and channels-last work alike. */
b2_status b2_im2col_bf16(const void* x, int64_t sb, int64_t sc, int64_t sh,
                         int64_t sw, int64_t B, int64_t C, int64_t H, int64_t W,
                         int kh, int kw, int sy, int sx, int py, int px,
                         int dy, int dx, int64_t Ho, int64_t Wo, int64_t Kp,
                         void* col, void* stream);
b2_status b2_col2im_bf16(const float* dcol, int64_t Kp, int64_t B, int64_t C,
                         int64_t H, int64_t W, int kh, int kw, int sy, int sx,
                         int py, int px, int dy, int dx, int64_t Ho,
                         int64_t Wo, void* dx_out, int64_t sb, int64_t sc,
                         int64_t sh, int64_t sw, void* stream);
b2_status b2_pack_weight_khwc_bf16(const void* w, int64_t Cout, int64_t Cin,
                                   int kh, int kw, int64_t Kp, void* wk,
                                   void* stream);
b2_status b2_unpack_weight_khwc(const float* dwk, int64_t Cout, int64_t Cin,
                                int kh, int kw, int64_t Kp, void* dw,
                                int dtype, void* stream);

/* ---- direct convolutions for layers with few output channels (an RGB
 * output layer; the reference's CPU path, torch_xdna_device.cpp:4578-4605,
 * 4828-4878), on the CUDA cores:
 *   out[b][o][y][x] = bias[o] + sum_{i,ky,kx} in[b][i][y*sy-py+ky*dy][x*sx-px+kx*dx] * wt[i][ky][kx][o]
 * in fp32 in (i, ky, kx) order, rounded once to bf16; at most 64 output
 * channels.  wt comes from b2_direct_conv_weight: the forward's
 * (wt[ci][ky][kx][co] = W[co][ci][ky][kx]) or, with dgrad = 1, the input
 * gradient's of a stride-1 convolution (wt[co][ky][kx][ci] =
 * W[co][ci][kh-1-ky][kw-1-kx]; run over dY with padding (k-1)*d - p), output
 * channels padded to 4/8/16/32/64 with zeros.  Tensors through element
 * strides [n, c, h, w]; bias (bf16, NOUT values) may be null. */
size_t b2_direct_conv_weight_floats(int64_t Cout, int64_t Cin, int kh, int kw,
                                    int dgrad);
b2_status b2_direct_conv_weight(const void* w, int64_t Cout, int64_t Cin,
                                int kh, int kw, int dgrad, float* wt,
                                void* stream);
b2_status b2_direct_conv_bf16(const void* in, const int64_t* in_strides,
                              int64_t B, int64_t NIN, int64_t Hin, int64_t Win,
                              const float* wt, int kh, int kw, int sy, int sx,
                              int py, int px, int dy, int dx, const void* bias,
                              void* out, const int64_t* out_strides,
                              int64_t NOUT, int64_t Ho, int64_t Wo,
                              void* stream);

/* ---- 2-D max pooling with indices (the reference runs it on its CPU path;
 * the same results as ATen): windows scanned in (kh, kw) order, a value
 * replaces the maximum when greater or NaN, index h*W + w within the plane
 * (int64).  The backward gathers, per input element in (oh, ow) order, the
 * gradients whose saved index is its own, in fp32, rounded once.  x/dx and
 * y/indices/dy through element strides [n, c, h, w] (indices and dy share
 * y_strides); dtype B2_BF16 or B2_F32. */
b2_status b2_maxpool2d_fwd(const void* x, const int64_t* x_strides, void* y,
                           int64_t* indices, const int64_t* y_strides,
                           int dtype, int64_t N, int64_t C, int64_t H,
                           int64_t W, int64_t OH, int64_t OW, int kh, int kw,
                           int sh, int sw, int ph, int pw, int dh, int dw,
                           void* stream);
b2_status b2_maxpool2d_bwd(const void* dy, const int64_t* indices,
                           const int64_t* y_strides, void* dx,
                           const int64_t* x_strides, int dtype, int64_t N,
                           int64_t C, int64_t H, int64_t W, int64_t OH,
                           int64_t OW, int kh, int kw, int sh, int sw, int ph,
                           int pw, int dh, int dw, void* stream);
/* The same pooling with the argmax kept as one byte per output element --
 * its tap i*kw + j inside the window that starts at (oh*sh - ph, ow*sw - pw)
 * -- instead of ATen's int64 index: the forward writes y and `taps` (uint8,
 * y's element strides); b2_maxpool2d_taps_to_indices expands them to exactly
 * the int64 indices b2_maxpool2d_fwd writes; b2_maxpool2d_bwd_taps is
 * b2_maxpool2d_bwd reading the taps (same sums in the same order).  The
 * backward of a ResNet stem reads 1 byte of index per element instead of 8.
 * Channels-last bf16 (C % 8 == 0, 16-byte aligned tensors, 8-byte aligned
 * taps), 3x3 windows for the forward, windows spanning at most two strides
 * for the backward.  Replaces the reference's CPU max_pool2d_with_indices and
 * its backward (torch_xdna_device.cpp:5124-5260) like the two calls above. */
b2_status b2_maxpool2d_fwd_taps(const void* x, const int64_t* x_strides,
                                void* y, void* taps, const int64_t* y_strides,
                                int64_t N, int64_t C, int64_t H, int64_t W,
                                int64_t OH, int64_t OW, int kh, int kw, int sh,
                                int sw, int ph, int pw, int dh, int dw,
                                void* stream);
b2_status b2_maxpool2d_taps_to_indices(const void* taps,
                                       const int64_t* y_strides,
                                       int64_t* indices, int64_t N, int64_t C,
                                       int64_t H, int64_t W, int64_t OH,
                                       int64_t OW, int kh, int kw, int sh,
                                       int sw, int ph, int pw, int dh, int dw,
                                       void* stream);
b2_status b2_maxpool2d_bwd_taps(const void* dy, const void* taps,
                                const int64_t* y_strides, void* dx,
                                const int64_t* x_strides, int64_t N, int64_t C,
                                int64_t H, int64_t W, int64_t OH, int64_t OW,
                                int kh, int kw, int sh, int sw, int ph, int pw,
                                int dh, int dw, void* stream);

/* ---- layout ops (replace the reference's host cat / nearest-2x upsample,
 * torch_xdna_device.cpp:3796-4175; used by the xdna `cat`,
 * `upsample_nearest2d` and `upsample_nearest2d_backward` kernels) ---------- */

/* Concatenation of contiguous byte blocks: for every outer index o and source
 * i (in order), block_bytes[i] bytes at srcs[i] + o*block_bytes[i] go to dst +
 * o*out_block_bytes + (block_bytes[0] + ... + block_bytes[i-1]).  The blocks
 * must add up to out_block_bytes.  Any dtype; any number of sources. */
b2_status b2_cat_blocks(const void* const* srcs, const int64_t* block_bytes,
                        int n, void* dst, int64_t outer,
                        int64_t out_block_bytes, void* stream);
/* Nearest 2x upsampling [N, C, H, W] -> [N, C, 2H, 2W] (a copy).  dtype
 * B2_BF16 or B2_F32; layout 0 = contiguous NCHW, 1 = channels-last NHWC. */
b2_status b2_upsample_nearest2x(const void* in, void* out, int dtype,
                                int layout, int64_t N, int64_t C, int64_t H,
                                int64_t W, void* stream);
/* Its backward: each input gradient = the fp32 sum of its 2x2 block of output
 * gradients from +0 in raster order (ATen's CPU order, x86 NaN propagation),
 * rounded once (bf16: nearest even, NaN -> 0x7FC0). */
b2_status b2_upsample_nearest2x_backward(const void* go, void* gi, int dtype,
                                         int layout, int64_t N, int64_t C,
                                         int64_t H, int64_t W, void* stream);

/* Training-mode BatchNorm on bf16 activations [N, C, HW] (replaces the
 * reference's native_batch_norm / native_batch_norm_backward on CPU aliases,
 * torch_xdna_device.cpp:4214-4358).  layout 0 = contiguous NCHW; 1 =
 * channels-last NHWC (C % 8 == 0, C <= 2048, 16-byte aligned tensors).
 * Batch statistics as in the fused region below (NCHW: per-plane fp32, Chan
 * merge in double; NHWC: one pass of shifted fp32 sums, merged in double);
 * y = x*scale + shift.  w, b (dtype pdtype), rm, rv (dtype rdtype; updated with
 * `momentum` when both are given) may be NULL; pdtype / rdtype are B2_BF16 or
 * B2_F32.  save_mean / save_invstd: fp32 [C].  Workspace: at least
 * b2_batch_norm_workspace_bytes(N, C, HW, layout) bytes, 16-byte aligned. */
size_t b2_batch_norm_workspace_bytes(int64_t N, int64_t C, int64_t HW,
                                     int layout);
b2_status b2_batch_norm_fwd_bf16(const void* x, int layout, const void* w,
                                 const void* b, int pdtype, void* rm, void* rv,
                                 int rdtype, void* y, float* save_mean,
                                 float* save_invstd, int64_t N, int64_t C,
                                 int64_t HW, float momentum, float eps,
                                 void* workspace, size_t workspace_bytes,
                                 void* stream);

/* The forward in two calls: the statistics (save_mean / save_invstd and the
 * running statistics, as above) and the output pass, which can also run the
 * ops that followed the BatchNorm in the same pass: y = bf16(x*scale + shift),
 * then, with `residual` (bf16 in x's layout, may be NULL), y = bf16(y +
 * residual) (an fp32 add, as ATen's), then, with relu != 0, y = y > 0 ? y : 0
 * (NaN kept).  w, b as above; mean / invstd from the statistics call. */
b2_status b2_batch_norm_stats_bf16(const void* x, int layout, int pdtype,
                                   void* rm, void* rv, int rdtype,
                                   float* save_mean, float* save_invstd,
                                   int64_t N, int64_t C, int64_t HW,
                                   float momentum, float eps, void* workspace,
                                   size_t workspace_bytes, void* stream);
/* b2_batch_norm_stats_bf16 that also advances a module's step counter:
 * *count += count_inc (count: an int64 scalar in device memory, 8-byte
 * aligned) in the same launch, once.  A training BatchNorm2d runs
 * `num_batches_tracked.add_(1)` right before its forward; done here, that
 * increment costs no kernel of its own.  Replaces the pair of that add_
 * (through the CPU-alias fallback, torch_xdna_device.cpp:5124-5260) and
 * native_batch_norm_xdna's statistics (torch_xdna_device.cpp:4214-4358).
 * Empty inputs are refused (nothing would run the increment). */
b2_status b2_batch_norm_stats_count_bf16(const void* x, int layout, int pdtype,
                                         void* rm, void* rv, int rdtype,
                                         float* save_mean, float* save_invstd,
                                         int64_t N, int64_t C, int64_t HW,
                                         float momentum, float eps,
                                         int64_t* count, int64_t count_inc,
                                         void* workspace,
                                         size_t workspace_bytes, void* stream);
b2_status b2_batch_norm_apply_bf16(const void* x, int layout, const void* w,
                                   const void* b, int pdtype, const float* mean,
                                   const float* invstd, const void* residual,
                                   int relu, void* y, int64_t N, int64_t C,
                                   int64_t HW, void* stream);
/* Backward from the saved batch statistics: dx (may be NULL), dw = sum
 * dy*xhat, db = sum dy (dtype gdtype, each may be NULL). */
b2_status b2_batch_norm_bwd_bf16(const void* dy, const void* x, int layout,
                                 const void* w, int pdtype,
                                 const float* save_mean,
                                 const float* save_invstd, void* dx, void* dw,
                                 void* db, int gdtype, int64_t N, int64_t C,
                                 int64_t HW, void* workspace,
                                 size_t workspace_bytes, void* stream);
/* Backward of a BatchNorm whose output pass folded a ReLU (no residual): dy is
 * the gradient of y = relu(bf16(x*scale + shift)); the ReLU's gate (y > 0 or
 * NaN, as ATen's threshold_backward) is recomputed from x, w, b and the saved
 * statistics, so neither y nor the gated gradient is read.  Results are bit
 * for bit those of threshold_backward(dy, y, 0) followed by
 * b2_batch_norm_bwd_bf16 (replaces the reference's two CPU-alias ops,
 * threshold_backward and native_batch_norm_backward,
 * torch_xdna_device.cpp:4214-4358, 5124-5260, for this pair).  Channels-last
 * only, C a power of two in [8, 2048]; workspace as b2_batch_norm_bwd_bf16
 * (layout 1). */
b2_status b2_batch_norm_relu_bwd_bf16(const void* dy, const void* x,
                                      const void* w, const void* b, int pdtype,
                                      const float* save_mean,
                                      const float* save_invstd, void* dx,
                                      void* dw, void* db, int gdtype, int64_t N,
                                      int64_t C, int64_t HW, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* A ReLU's backward on the sum of two gradients, in one pass over n bf16
 * elements of four dense tensors with the same layout (16-byte aligned, n a
 * multiple of 8):  dz = (y > 0 or y is NaN) ? bf16(float(a) + float(b)) : +0
 * -- bit for bit ATen's in-place add a += b (fp32 add, hardware round to
 * nearest even) followed by threshold_backward(a, y, 0).  Autograd sums the
 * two gradients of a residual block's output this way before the block's
 * ReLU backward; the reference runs both ops on its CPU-alias fallback
 * (torch_xdna_device.cpp:5124-5260). */
b2_status b2_relu_bwd_sum_bf16(const void* a, const void* b, const void* y,
                               void* dz, int64_t n, void* stream);
/* The same gated sum feeding a BatchNorm's backward (the residual block's
 * last BatchNorm): dz = (y > 0 or NaN) ? bf16(a + b) : +0 is made, written to
 * dz (its other readers need it) and reduced in one pass, then dx, dw, db as
 * b2_batch_norm_bwd_bf16 from dy = dz.  Bit for bit b2_relu_bwd_sum_bf16
 * followed by b2_batch_norm_bwd_bf16 (replaces the reference's CPU add,
 * threshold_backward and native_batch_norm_backward for this chain,
 * torch_xdna_device.cpp:4214-4358, 5124-5260).  Channels-last, C a power of
 * two in [8, 2048]; x, w, statistics and workspace as b2_batch_norm_bwd_bf16
 * (layout 1); dx may be NULL. */
b2_status b2_batch_norm_bwd_relu_sum_bf16(const void* a, const void* b,
                                          const void* y, const void* x,
                                          const void* w, int pdtype,
                                          const float* save_mean,
                                          const float* save_invstd, void* dz,
                                          void* dx, void* dw, void* db,
                                          int gdtype, int64_t N, int64_t C,
                                          int64_t HW, void* workspace,
                                          size_t workspace_bytes, void* stream);

/* Training BatchNorm2d + LeakyReLU/ReLU on contiguous NCHW bf16 [N, C, HW]
 * (replaces xdna_region_bn_fwd_bf16 / xdna_region_bn_bwd_bf16,
 * region_kernels.cpp:309-460; used by regions.fuse_norm_activation,
 * regions.py:426-548).  Statistics: each (n, c) plane reduced in fp32 (mean,
 * then the sum of squared deviations), the N planes of a channel merged in
 * double in plane order with Chan's formula.  Workspace: at least
 * b2_region_bn_workspace_bytes(N, C) bytes of device memory, 16-byte aligned.
 *
 * Forward: w, b may be NULL (affine=False); if update != 0 the bf16 running
 * statistics rm, rv move by `factor` towards the batch mean and the unbiased
 * batch variance.  mean_out / invstd_out: fp32 [C].  y = act(x*scale + shift)
 * with scale = w*invstd, shift = b - mean*scale, act(z) = z > 0 ? z : z*slope,
 * rounded once to bf16. */
size_t b2_region_bn_workspace_bytes(int64_t N, int64_t C);
b2_status b2_region_bn_fwd_bf16(const void* x, const void* w, const void* b,
                                void* rm, void* rv, void* y, float* mean_out,
                                float* invstd_out, int64_t N, int64_t C,
                                int64_t HW, float eps, float slope, float factor,
                                int update, void* workspace,
                                size_t workspace_bytes, void* stream);
/* Backward: dz = (y > 0 or (relu and y is NaN)) ? dy : dy*slope; dw, db (bf16
 * [C], each may be NULL) get sum(dz*xhat) and sum(dz); dx (may be NULL) gets
 * w*invstd*(dz - mean(dz) - xhat*mean(dz*xhat)). */
b2_status b2_region_bn_bwd_bf16(const void* dy, const void* y, const void* x,
                                const void* w, const float* mean,
                                const float* invstd, void* dx, void* dw,
                                void* db, int64_t N, int64_t C, int64_t HW,
                                float slope, int relu, void* workspace,
                                size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XDNA_B200_B2_H */
