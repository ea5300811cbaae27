// Thin PyTorch binding over the C ABI in include/ashqk_b200.h.
//
// Registers torch.ops.ashqk.* for the CUDA dispatch key only: a CPU tensor gets
// PyTorch's "could not run ... with arguments from the CPU backend" error, so
// there is no silent host fallback. The binding owns the split-K workspace: one
// zero-initialised byte buffer per (device, stream), grown on demand and left
// zeroed by every kernel -- the role of the reference's _workspace caches
// (ashqk/kernels/w4a16_gemv.py:110-120, ashqk/kernels/w4a16_gemm_v3.py:108-119).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <utility>

#include "ashqk_b200.h"

namespace {

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == ASHQK_OK, "ashqk.", what, ": ", ashqk_status_string(rc), " (status ", rc, ")");
}

std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, at::Tensor> g_ws;

// Zeroed workspace of at least `bytes` for the current stream of `dev`.
at::Tensor workspace_for(const at::Device& dev, size_t bytes) {
  if (bytes == 0) return at::Tensor();
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  std::lock_guard<std::mutex> lock(g_ws_mu);
  at::Tensor& t = g_ws[{dev.index(), stream}];
  if (!t.defined() || static_cast<size_t>(t.numel()) < bytes) {
    const int64_t rounded = static_cast<int64_t>((bytes + (1u << 20) - 1) >> 20 << 20);
    t = at::zeros({rounded}, at::TensorOptions().dtype(at::kByte).device(dev));
  }
  return t;
}

struct Problem {
  int64_t M, N, K, G;
};

// Shape / dtype / device checks shared by the linear ops. Returns x with a unit
// column stride (a copy only when the caller's x has another inner stride).
Problem check_linear(const at::Tensor& x, const at::Tensor& qw, const at::Tensor& qz, const at::Tensor& s) {
  TORCH_CHECK(x.is_cuda(), "ashqk: x must be a CUDA tensor");
  TORCH_CHECK(x.scalar_type() == at::kHalf && x.dim() == 2, "ashqk: x must be a 2-D float16 tensor");
  TORCH_CHECK(qw.scalar_type() == at::kInt && qw.dim() == 2, "ashqk: qweight must be a 2-D int32 tensor");
  TORCH_CHECK(qz.scalar_type() == at::kInt && qz.dim() == 2, "ashqk: qzeros must be a 2-D int32 tensor");
  TORCH_CHECK(s.scalar_type() == at::kHalf && s.dim() == 2, "ashqk: scales must be a 2-D float16 tensor");
  TORCH_CHECK(qw.device() == x.device() && qz.device() == x.device() && s.device() == x.device(),
              "ashqk: all tensors must be on the same device");
  Problem p;
  p.M = x.size(0);
  p.K = x.size(1);
  p.N = qw.size(1) * 8;
  TORCH_CHECK(s.size(0) > 0 && p.K % s.size(0) == 0, "ashqk: K must be a multiple of scales.shape[0]");
  p.G = p.K / s.size(0);
  TORCH_CHECK(qw.size(0) == p.K, "ashqk: qweight must be [K, N/8]");
  TORCH_CHECK(qz.size(0) == p.K / p.G && qz.size(1) == p.N / 8, "ashqk: qzeros must be [K/G, N/8]");
  TORCH_CHECK(s.size(1) == p.N, "ashqk: scales must be [K/G, N]");
  return p;
}

at::Tensor unit_inner(const at::Tensor& t) { return t.stride(1) == 1 ? t : t.contiguous(); }

enum class Path { kGemv, kGemm, kLinear };

at::Tensor run_linear(Path path, const at::Tensor& x_in, const at::Tensor& qw_in, const at::Tensor& qz_in,
                      const at::Tensor& s_in, int64_t split_k, c10::optional<at::Tensor> out) {
  Problem p = check_linear(x_in, qw_in, qz_in, s_in);
  c10::cuda::CUDAGuard guard(x_in.device());
  at::Tensor x = unit_inner(x_in), qw = unit_inner(qw_in), qz = unit_inner(qz_in), s = unit_inner(s_in);
  at::Tensor y;
  if (out.has_value()) {
    y = *out;
    TORCH_CHECK(y.is_cuda() && y.device() == x.device() && y.scalar_type() == at::kHalf && y.dim() == 2 &&
                    y.size(0) == p.M && y.size(1) == p.N && y.stride(1) == 1,
                "ashqk: out must be a float16 [M, N] CUDA tensor with unit column stride");
  } else {
    y = at::empty({p.M, p.N}, x.options());
  }
  if (p.M == 0) return y;
  TORCH_CHECK(p.M <= INT32_MAX && p.N <= INT32_MAX && p.K <= INT32_MAX, "ashqk: problem too large");
  const int M = static_cast<int>(p.M), N = static_cast<int>(p.N), K = static_cast<int>(p.K),
            G = static_cast<int>(p.G);
  size_t bytes = 0;
  int rc;
  switch (path) {
    case Path::kGemv:
      rc = ashqk_gemv_workspace_size(M < 16 ? M : 16, N, K, G, static_cast<int>(split_k), &bytes);
      break;
    case Path::kGemm:
      rc = ashqk_gemm_workspace_size(M, N, K, G, &bytes);
      break;
    default:
      rc = ashqk_linear_workspace_size(M, N, K, G, &bytes);
  }
  check_rc(rc, "workspace_size");
  at::Tensor ws = workspace_for(x.device(), bytes);
  void* wsp = ws.defined() ? ws.data_ptr() : nullptr;
  const size_t wsb = ws.defined() ? static_cast<size_t>(ws.numel()) : 0;
  void* stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
  switch (path) {
    case Path::kGemv:
      rc = ashqk_w4a16_gemv(x.data_ptr(), x.stride(0), qw.data_ptr<int32_t>(), qw.stride(0),
                            qz.data_ptr<int32_t>(), qz.stride(0), s.data_ptr(), s.stride(0), y.data_ptr(),
                            y.stride(0), M, N, K, G, static_cast<int>(split_k), wsp, wsb, stream);
      break;
    case Path::kGemm:
      rc = ashqk_w4a16_gemm(x.data_ptr(), x.stride(0), qw.data_ptr<int32_t>(), qw.stride(0),
                            qz.data_ptr<int32_t>(), qz.stride(0), s.data_ptr(), s.stride(0), y.data_ptr(),
                            y.stride(0), M, N, K, G, wsp, wsb, stream);
      break;
    default:
      rc = ashqk_w4a16_linear(x.data_ptr(), x.stride(0), qw.data_ptr<int32_t>(), qw.stride(0),
                              qz.data_ptr<int32_t>(), qz.stride(0), s.data_ptr(), s.stride(0), y.data_ptr(),
                              y.stride(0), M, N, K, G, wsp, wsb, stream);
  }
  check_rc(rc, "w4a16 launch");
  return y;
}

at::Tensor w4a16_gemv(const at::Tensor& x, const at::Tensor& qw, const at::Tensor& qz, const at::Tensor& s,
                      int64_t split_k) {
  return run_linear(Path::kGemv, x, qw, qz, s, split_k, c10::nullopt);
}

at::Tensor w4a16_gemm(const at::Tensor& x, const at::Tensor& qw, const at::Tensor& qz, const at::Tensor& s) {
  return run_linear(Path::kGemm, x, qw, qz, s, 0, c10::nullopt);
}

at::Tensor w4a16_linear(const at::Tensor& x, const at::Tensor& qw, const at::Tensor& qz, const at::Tensor& s) {
  return run_linear(Path::kLinear, x, qw, qz, s, 0, c10::nullopt);
}

at::Tensor w4a16_linear_out(const at::Tensor& x, const at::Tensor& qw, const at::Tensor& qz, const at::Tensor& s,
                            at::Tensor out) {
  run_linear(Path::kLinear, x, qw, qz, s, 0, out);
  return out;
}

at::Tensor dequantize_awq(const at::Tensor& qw_in, const at::Tensor& qz_in, const at::Tensor& s_in,
                          at::ScalarType dtype) {
  TORCH_CHECK(qw_in.is_cuda(), "ashqk: qweight must be a CUDA tensor");
  TORCH_CHECK(qw_in.scalar_type() == at::kInt && qw_in.dim() == 2, "ashqk: qweight must be a 2-D int32 tensor");
  TORCH_CHECK(qz_in.scalar_type() == at::kInt && qz_in.dim() == 2, "ashqk: qzeros must be a 2-D int32 tensor");
  TORCH_CHECK(s_in.scalar_type() == at::kHalf && s_in.dim() == 2, "ashqk: scales must be a 2-D float16 tensor");
  TORCH_CHECK(dtype == at::kHalf || dtype == at::kFloat, "ashqk: dequantize_awq supports float16 and float32");
  TORCH_CHECK(qz_in.device() == qw_in.device() && s_in.device() == qw_in.device(),
              "ashqk: all tensors must be on the same device");
  c10::cuda::CUDAGuard guard(qw_in.device());
  at::Tensor qw = unit_inner(qw_in), qz = unit_inner(qz_in), s = unit_inner(s_in);
  const int64_t K = qw.size(0), N = qw.size(1) * 8;
  TORCH_CHECK(s.size(0) > 0 && K % s.size(0) == 0, "ashqk: K must be a multiple of scales.shape[0]");
  const int64_t G = K / s.size(0);
  TORCH_CHECK(qz.size(0) == K / G && qz.size(1) == N / 8 && s.size(1) == N, "ashqk: inconsistent AWQ shapes");
  at::Tensor w = at::empty({K, N}, qw.options().dtype(dtype));
  if (K == 0 || N == 0) return w;
  void* stream = c10::cuda::getCurrentCUDAStream(qw.device().index()).stream();
  int rc;
  if (dtype == at::kHalf) {
    rc = ashqk_dequantize_awq_f16(qw.data_ptr<int32_t>(), qw.stride(0), qz.data_ptr<int32_t>(), qz.stride(0),
                                  s.data_ptr(), s.stride(0), w.data_ptr(), w.stride(0), static_cast<int>(N),
                                  static_cast<int>(K), static_cast<int>(G), stream);
  } else {
    rc = ashqk_dequantize_awq_f32(qw.data_ptr<int32_t>(), qw.stride(0), qz.data_ptr<int32_t>(), qz.stride(0),
                                  s.data_ptr(), s.stride(0), w.data_ptr<float>(), w.stride(0), static_cast<int>(N),
                                  static_cast<int>(K), static_cast<int>(G), stream);
  }
  check_rc(rc, "dequantize_awq");
  return w;
}

}  // namespace

TORCH_LIBRARY(ashqk, m) {
  m.def("w4a16_gemv(Tensor x, Tensor qweight, Tensor qzeros, Tensor scales, int split_k=0) -> Tensor");
  m.def("w4a16_gemm(Tensor x, Tensor qweight, Tensor qzeros, Tensor scales) -> Tensor");
  m.def("w4a16_linear(Tensor x, Tensor qweight, Tensor qzeros, Tensor scales) -> Tensor");
  m.def("w4a16_linear_out(Tensor x, Tensor qweight, Tensor qzeros, Tensor scales, Tensor(a!) out) -> Tensor(a!)");
  m.def("dequantize_awq(Tensor qweight, Tensor qzeros, Tensor scales, ScalarType dtype) -> Tensor");
}

TORCH_LIBRARY_IMPL(ashqk, CUDA, m) {
  m.impl("w4a16_gemv", &w4a16_gemv);
  m.impl("w4a16_gemm", &w4a16_gemm);
  m.impl("w4a16_linear", &w4a16_linear);
  m.impl("w4a16_linear_out", &w4a16_linear_out);
  m.impl("dequantize_awq", &dequantize_awq);
}
