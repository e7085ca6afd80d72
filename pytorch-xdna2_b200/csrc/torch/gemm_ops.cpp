// aten::mm / addmm / bmm (and their out= forms) on xdna.
//
// Replaces mm_xdna, addmm_out_xdna and bmm_out_xdna (torch_xdna_device.cpp:
// 4387-4417, 3740-3790) and the fixed-shape XdnaGemmRuntime (:1320-1458): the
// reference served three contiguous BF16 shapes on the NPU and everything else
// on the CPU; here every BF16 product whose operands are row- or column-major
// (any transpose view, e.g. nn.Linear's W.t()) runs the tcgen05 GEMM, with
// addmm's beta*self + alpha*(A@B) fused into the epilogue.  Other dtypes and
// layouts that break TMA's 16-byte row alignment take ATen's CUDA kernels on
// aliases.
#include <ATen/ops/addmm.h>
#include <ATen/ops/bmm.h>
#include <ATen/ops/mm.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "xdna.h"

namespace xdna {
namespace {

// A 2-D (or per-batch) operand as the kernel sees it.
struct Operand {
  const void* ptr = nullptr;
  int trans = 0;     // 0: rows contiguous (row-major); 1: columns contiguous
  int64_t ld = 0;
  int64_t bstride = 0;
  bool ok = false;
};

bool aligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// t: [rows][cols] (dim offset `d0`), possibly batched in dim 0.
Operand describe(const at::Tensor& t, int d0) {
  Operand o;
  const int64_t rows = t.size(d0), cols = t.size(d0 + 1);
  const int64_t s0 = t.stride(d0), s1 = t.stride(d0 + 1);
  if (s1 == 1 && (s0 >= cols || rows == 1)) {
    o.trans = 0;
    o.ld = rows == 1 ? std::max<int64_t>(s0, cols) : s0;
  } else if (s0 == 1 && (s1 >= rows || cols == 1)) {
    o.trans = 1;
    o.ld = cols == 1 ? std::max<int64_t>(s1, rows) : s1;
  } else {
    return o;
  }
  o.ptr = t.data_ptr();
  o.bstride = d0 == 1 ? t.stride(0) : 0;
  o.ok = aligned(o.ptr) && o.ld % 8 == 0 && (d0 == 0 || o.bstride % 8 == 0 || t.size(0) == 1);
  return o;
}

bool eligible(const at::Tensor& a, const at::Tensor& b) {
  return g_mode.load() > 0 && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 &&
         a.device().type() == kXdna && b.device().type() == kXdna;
}

// out[b] = alpha * A[b] @ B[b] + beta * C[b]; returns false if the operands do
// not fit the kernel (caller falls back).
bool run_gemm(const at::Tensor& A, const at::Tensor& Bm, const at::Tensor& out, float alpha, float beta,
              const at::Tensor& C, bool batched) {
  const int d0 = batched ? 1 : 0;
  const int64_t M = A.size(d0), K = A.size(d0 + 1), N = Bm.size(d0 + 1);
  const int64_t batch = batched ? A.size(0) : 1;
  if (M == 0 || N == 0 || batch == 0) return true;
  if (K == 0) return false;
  if (!out.is_contiguous() || out.scalar_type() != at::kBFloat16) return false;
  materialize(A);
  materialize(Bm);
  Operand a = describe(A, d0), b = describe(Bm, d0);
  if (!a.ok || !b.ok) return false;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || batch > INT32_MAX) return false;
  int c_dtype = B2_BF16;
  const void* cptr = nullptr;
  int64_t c_sm = 0, c_sn = 0, c_sb = 0;
  at::Tensor Ce;
  if (beta != 0.f && C.defined()) {
    materialize(C);
    if (C.scalar_type() != at::kBFloat16 && C.scalar_type() != at::kFloat) return false;
    c_dtype = C.scalar_type() == at::kFloat ? B2_F32 : B2_BF16;
    Ce = batched ? C.expand({batch, M, N}) : C.expand({M, N});
    cptr = Ce.data_ptr();
    c_sm = Ce.stride(d0);
    c_sn = Ce.stride(d0 + 1);
    c_sb = batched ? Ce.stride(0) : 0;
  } else {
    beta = 0.f;
  }
  const c10::DeviceIndex dev = out.device().index();
  // split-K room for GEMMs with too few output tiles (from the caching allocator)
  const size_t ws_bytes = b2_gemm_bf16_workspace_bytes(int(M), int(N), int(K), int(batch));
  at::Tensor ws;
  if (ws_bytes) ws = empty({int64_t((ws_bytes + 15) / 16) * 4}, at::kFloat, dev);
  KernelTimer kt("gemm", 2.0 * double(M) * double(N) * double(K) * double(batch), stream(dev));
  XDNA_B2(b2_gemm_bf16_ws(a.trans, b.trans, int(M), int(N), int(K), alpha, a.ptr, a.ld, a.bstride, b.ptr, b.ld,
                          b.bstride, beta, cptr, c_dtype, c_sm, c_sn, c_sb, out.data_ptr(), N, M * N, int(batch),
                          ws_bytes ? ws.data_ptr() : nullptr, ws_bytes ? size_t(ws.numel()) * 4 : 0, stream(dev)));
  count_launch("gemm");
  return true;
}

at::Tensor mm(const at::Tensor& self, const at::Tensor& mat2) {
  c10::cuda::CUDAGuard g(self.device().index());
  if (eligible(self, mat2) && self.dim() == 2 && mat2.dim() == 2) {
    at::Tensor out = empty({self.size(0), mat2.size(1)}, at::kBFloat16, self.device().index());
    if (self.size(1) == 0) return adopt(to_cuda(out).zero_());
    if (run_gemm(self, mat2, out, 1.f, 0.f, at::Tensor(), false)) return out;
  }
  count_fallback("mm");
  return adopt(at::mm(to_cuda(self), to_cuda(mat2)));
}

at::Tensor& mm_out(const at::Tensor& self, const at::Tensor& mat2, at::Tensor& out) {
  before_write(out);
  note_write(out);
  c10::cuda::CUDAGuard g(self.device().index());
  if (eligible(self, mat2) && self.dim() == 2 && mat2.dim() == 2 && self.size(1) > 0) {
    materialize(out);
    std::vector<c10::SymInt> sz{c10::SymInt(self.size(0)), c10::SymInt(mat2.size(1))};
    if (out.sizes() != at::IntArrayRef{self.size(0), mat2.size(1)}) out.resize_({self.size(0), mat2.size(1)});
    if (run_gemm(self, mat2, out, 1.f, 0.f, at::Tensor(), false)) return out;
  }
  count_fallback("mm.out");
  at::Tensor r = at::mm(to_cuda(self), to_cuda(mat2));
  if (out.sizes() != r.sizes()) out.resize_(r.sizes());
  to_cuda(out).copy_(r);
  return out;
}

at::Tensor addmm(const at::Tensor& self, const at::Tensor& mat1, const at::Tensor& mat2, const at::Scalar& beta,
                 const at::Scalar& alpha) {
  c10::cuda::CUDAGuard g(mat1.device().index());
  if (eligible(mat1, mat2) && mat1.dim() == 2 && mat2.dim() == 2 && mat1.size(1) > 0) {
    at::Tensor out = empty({mat1.size(0), mat2.size(1)}, at::kBFloat16, mat1.device().index());
    if (run_gemm(mat1, mat2, out, alpha.toFloat(), beta.toFloat(), self, false)) return out;
  }
  count_fallback("addmm");
  return adopt(at::addmm(to_cuda(self), to_cuda(mat1), to_cuda(mat2), beta, alpha));
}

at::Tensor& addmm_out(const at::Tensor& self, const at::Tensor& mat1, const at::Tensor& mat2, const at::Scalar& beta,
                      const at::Scalar& alpha, at::Tensor& out) {
  before_write(out);
  note_write(out);
  c10::cuda::CUDAGuard g(mat1.device().index());
  if (eligible(mat1, mat2) && mat1.dim() == 2 && mat2.dim() == 2 && mat1.size(1) > 0 && !out.is_same(self)) {
    materialize(out);
    if (out.sizes() != at::IntArrayRef{mat1.size(0), mat2.size(1)}) out.resize_({mat1.size(0), mat2.size(1)});
    if (run_gemm(mat1, mat2, out, alpha.toFloat(), beta.toFloat(), self, false)) return out;
  }
  count_fallback("addmm.out");
  at::Tensor r = at::addmm(to_cuda(self), to_cuda(mat1), to_cuda(mat2), beta, alpha);
  if (out.sizes() != r.sizes()) out.resize_(r.sizes());
  to_cuda(out).copy_(r);
  return out;
}

at::Tensor bmm(const at::Tensor& self, const at::Tensor& mat2) {
  c10::cuda::CUDAGuard g(self.device().index());
  if (eligible(self, mat2) && self.dim() == 3 && mat2.dim() == 3 && self.size(2) > 0) {
    at::Tensor out = empty({self.size(0), self.size(1), mat2.size(2)}, at::kBFloat16, self.device().index());
    if (run_gemm(self, mat2, out, 1.f, 0.f, at::Tensor(), true)) return out;
  }
  count_fallback("bmm");
  return adopt(at::bmm(to_cuda(self), to_cuda(mat2)));
}

at::Tensor& bmm_out(const at::Tensor& self, const at::Tensor& mat2, at::Tensor& out) {
  before_write(out);
  note_write(out);
  c10::cuda::CUDAGuard g(self.device().index());
  if (eligible(self, mat2) && self.dim() == 3 && mat2.dim() == 3 && self.size(2) > 0) {
    materialize(out);
    if (out.sizes() != at::IntArrayRef{self.size(0), self.size(1), mat2.size(2)})
      out.resize_({self.size(0), self.size(1), mat2.size(2)});
    if (run_gemm(self, mat2, out, 1.f, 0.f, at::Tensor(), true)) return out;
  }
  count_fallback("bmm.out");
  at::Tensor r = at::bmm(to_cuda(self), to_cuda(mat2));
  if (out.sizes() != r.sizes()) out.resize_(r.sizes());
  to_cuda(out).copy_(r);
  return out;
}

}  // namespace

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("mm", mm);
  m.impl("mm.out", mm_out);
  m.impl("addmm", addmm);
  m.impl("addmm.out", addmm_out);
  m.impl("bmm", bmm);
  m.impl("bmm.out", bmm_out);
}

}  // namespace xdna
