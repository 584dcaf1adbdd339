// torch_ext.cpp — the thin torch extension between the reference-compatible
// Python entry points and the C ABI of libnvfp4dg.so.
//
// The reference binds its kernel with load_inline/pybind as
// cuda_nvfp4_dual_gemm(A, B1, B2, SFA, SFB1, SFB2, C) (submission.py:17-20,
// nvfp4_dual_gemm.cu:381-446) and calls it from custom_kernel(data)
// (submission.py:1153-1157).  This module exposes the same two functions
// plus dual_gemm (flags, caller workspace).  It checks the tensors (shape,
// strides, dtype, device: the same rules and messages as the Python checks
// in api.py), takes the current CUDA stream of C's device, and calls
// nvfp4_dual_gemm_run / nvfp4_dual_gemm_run_ws.  All of that costs a few
// microseconds per call, against tens for the same checks in Python plus a
// ctypes call, which matters when a caller launches one call at a time.
// Invalid arguments raise ValueError; CUDA and device failures RuntimeError.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/csrc/autograd/python_variable.h>
#include <torch/extension.h>

#include <string>

#include "nvfp4_dual_gemm.h"

namespace {

namespace py = pybind11;

[[noreturn]] void bad(const std::string& msg) { throw py::value_error(msg); }

std::string dims(const at::Tensor& t) {
  std::string s = "(";
  for (int64_t i = 0; i < t.dim(); ++i) {
    if (i) s += ", ";
    s += std::to_string(t.size(i));
  }
  return s + (t.dim() == 1 ? ",)" : ")");
}

void check_bytes(const char* name, const at::Tensor& t) {
  if (t.element_size() != 1)
    bad(std::string(name) +
        " must hold 1-byte elements (fp4x2 / fp8 / uint8), got " +
        std::string(c10::toString(t.scalar_type())));
  if (!t.is_cuda()) bad(std::string(name) + " must be a CUDA tensor");
}

int64_t batches(const at::Tensor& t) { return t.dim() == 3 ? t.size(2) : 1; }

// [rows, row_bytes] or [rows, row_bytes, L], rows dense and K-major, a batch
// stored batch after batch (api._rows_dense).
void rows_dense(const char* name, const at::Tensor& t, int64_t rows,
                int64_t row_bytes, int64_t L) {
  if (t.dim() != 2 && t.dim() != 3)
    bad(std::string(name) + " must be [rows, K/2] or [rows, K/2, L]");
  if (batches(t) != L)
    bad(std::string(name) + " holds " + std::to_string(batches(t)) +
        " batches, A holds " + std::to_string(L));
  if (t.size(0) != rows || t.size(1) != row_bytes)
    bad(std::string(name) + " has shape " + dims(t) + ", expected [" +
        std::to_string(rows) + ", " + std::to_string(row_bytes) + "(, " +
        std::to_string(L) + ")]");
  if (rows > 1 && row_bytes > 0 && t.stride(0) != row_bytes)
    bad(std::string(name) + " rows must be dense (stride(0) == K/2)");
  if (row_bytes > 1 && t.stride(1) != 1)
    bad(std::string(name) + " must be K-major (stride(1) == 1)");
  if (L > 1 && rows * row_bytes > 0 && t.stride(2) != rows * row_bytes)
    bad(std::string(name) + ": the batches must follow one another "
        "(stride(2) == " + std::to_string(rows * row_bytes) + ")");
}

int64_t blocked_bytes(int64_t rows, int64_t k) {
  return ((rows + 127) / 128) * (k / 64) * 512;
}

bool batch_major(const at::Tensor& t, int64_t L) {
  return t.is_contiguous() ||
         (L > 1 && t.dim() >= 2 && t.size(-1) == L &&
          t.movedim(-1, 0).is_contiguous());
}

void check_blocked(const char* name, const at::Tensor& t, int64_t rows,
                   int64_t k, int64_t L) {
  check_bytes(name, t);
  const int64_t need = blocked_bytes(rows, k);
  if (!batch_major(t, L))
    bad(std::string(name) + " must be contiguous (batch after batch)");
  if (L > 1 && !t.is_contiguous() && t.numel() != L * need)
    bad(std::string(name) + " holds " + std::to_string(t.numel()) +
        " bytes, " + std::to_string(L) +
        " batches of the blocked layout need " + std::to_string(L * need));
  if (t.numel() < L * need)
    bad(std::string(name) + " holds " + std::to_string(t.numel()) +
        " bytes, the blocked layout needs " + std::to_string(L * need));
}

struct Problem {
  int64_t M, N, K, L;
};

Problem check_problem(const at::Tensor& A, const at::Tensor& B1,
                      const at::Tensor& B2, const at::Tensor& SFA,
                      const at::Tensor& SFB1, const at::Tensor& SFB2,
                      const at::Tensor& C) {
  check_bytes("A", A);
  check_bytes("B1", B1);
  check_bytes("B2", B2);
  Problem p;
  p.M = A.size(0);
  p.N = B1.size(0);
  p.K = A.dim() >= 2 ? 2 * A.size(1) : 0;
  p.L = batches(A);
  if (p.L < 1) bad("L must be >= 1");
  rows_dense("A", A, p.M, p.K / 2, p.L);
  rows_dense("B1", B1, p.N, p.K / 2, p.L);
  rows_dense("B2", B2, p.N, p.K / 2, p.L);
  if (p.N % 64 != 0)
    bad("N = " + std::to_string(p.N) + " must be a multiple of 64");
  if (p.K % 256 != 0)
    bad("K = " + std::to_string(p.K) + " must be a multiple of 256");
  check_blocked("SFA", SFA, p.M, p.K, p.L);
  check_blocked("SFB1", SFB1, p.N, p.K, p.L);
  check_blocked("SFB2", SFB2, p.N, p.K, p.L);
  if (C.scalar_type() != at::kHalf)
    bad("C must be float16, got " +
        std::string(c10::toString(C.scalar_type())));
  if (!C.is_cuda() || !batch_major(C, p.L))
    bad("C must be a contiguous CUDA tensor (batch after batch)");
  if (C.numel() != p.L * p.M * p.N || C.size(0) != p.M ||
      (C.dim() == 3 && C.size(2) != p.L))
    bad("C has shape " + dims(C) + ", expected [" + std::to_string(p.M) +
        ", " + std::to_string(p.N) + "(, " + std::to_string(p.L) + ")]");
  if (p.L > 1 && C.dim() != 3)
    bad("C must be [" + std::to_string(p.M) + ", " + std::to_string(p.N) +
        ", " + std::to_string(p.L) + "] for a batch");
  const at::Device dev = C.device();
  const char* names[6] = {"A", "B1", "B2", "SFA", "SFB1", "SFB2"};
  const at::Tensor* ts[6] = {&A, &B1, &B2, &SFA, &SFB1, &SFB2};
  for (int i = 0; i < 6; ++i)
    if (ts[i]->device() != dev)
      bad(std::string(names[i]) + " is on " + ts[i]->device().str() +
          ", C on " + dev.str());
  return p;
}

void check_status(int rc, const char* what) {
  if (rc == NVFP4DG_OK) return;
  const char* m = nvfp4_dual_gemm_last_error();
  const std::string msg = std::string(what) + " failed (status " +
                          std::to_string(rc) + "): " + (m ? m : "");
  if (rc == NVFP4DG_ERR_INVALID || rc == NVFP4DG_ERR_ALIGN ||
      rc == NVFP4DG_ERR_WORKSPACE)
    throw py::value_error(msg);
  throw std::runtime_error(msg);
}

at::Tensor run(const at::Tensor& A, const at::Tensor& B1, const at::Tensor& B2,
               const at::Tensor& SFA, const at::Tensor& SFB1,
               const at::Tensor& SFB2, const at::Tensor& C, int64_t flags,
               const at::Tensor* ws) {
  const Problem p = check_problem(A, B1, B2, SFA, SFB1, SFB2, C);
  const c10::cuda::CUDAGuard guard(C.device());
  void* stream = at::cuda::getCurrentCUDAStream(C.device().index()).stream();
  int rc;
  if (ws == nullptr) {
    rc = nvfp4_dual_gemm_run(A.data_ptr(), B1.data_ptr(), B2.data_ptr(),
                             SFA.data_ptr(), SFB1.data_ptr(), SFB2.data_ptr(),
                             C.data_ptr(), static_cast<int>(p.M),
                             static_cast<int>(p.N), static_cast<int>(p.K),
                             static_cast<int>(p.L),
                             static_cast<unsigned>(flags), stream);
  } else {
    if (ws->device() != C.device() || !ws->is_contiguous())
      bad("workspace must be a contiguous tensor on C's device");
    rc = nvfp4_dual_gemm_run_ws(
        A.data_ptr(), B1.data_ptr(), B2.data_ptr(), SFA.data_ptr(),
        SFB1.data_ptr(), SFB2.data_ptr(), C.data_ptr(), static_cast<int>(p.M),
        static_cast<int>(p.N), static_cast<int>(p.K), static_cast<int>(p.L),
        static_cast<unsigned>(flags), ws->data_ptr(),
        static_cast<size_t>(ws->numel()) * ws->element_size(), stream);
  }
  check_status(rc, "nvfp4_dual_gemm_run");
  return C;
}

// The reference's torch-extension function: packed A/B1/B2, blocked
// SFA/SFB1/SFB2, preallocated fp16 C; returns C.
at::Tensor cuda_nvfp4_dual_gemm(const at::Tensor& A, const at::Tensor& B1,
                                const at::Tensor& B2, const at::Tensor& SFA,
                                const at::Tensor& SFB1, const at::Tensor& SFB2,
                                const at::Tensor& C) {
  return run(A, B1, B2, SFA, SFB1, SFB2, C, 0, nullptr);
}

// custom_kernel(data): data = (a, b1, b2, sfa, sfb1, sfb2, sfa_blocked,
// sfb1_blocked, sfb2_blocked, c), a tuple or any sequence of 10 tensors; the
// plain scales are not read.  The tensors are taken straight from the
// sequence's items (no per-item conversion objects).
at::Tensor custom_kernel(const py::object& data) {
  PyObject* seq = PySequence_Fast(data.ptr(), "data must be a sequence");
  if (seq == nullptr) throw py::error_already_set();
  const py::object keep = py::reinterpret_steal<py::object>(seq);
  if (PySequence_Fast_GET_SIZE(seq) != 10)
    bad("data must be the 10-tuple (a, b1, b2, sfa, sfb1, sfb2, "
        "sfa_blocked, sfb1_blocked, sfb2_blocked, c)");
  PyObject** items = PySequence_Fast_ITEMS(seq);
  auto t = [&](int i) -> const at::Tensor& {
    if (!THPVariable_Check(items[i]))
      throw py::type_error("data[" + std::to_string(i) +
                           "] must be a torch.Tensor");
    return THPVariable_Unpack(items[i]);
  };
  return run(t(0), t(1), t(2), t(6), t(7), t(8), t(9), 0, nullptr);
}

at::Tensor dual_gemm(const at::Tensor& A, const at::Tensor& B1,
                     const at::Tensor& B2, const at::Tensor& SFA,
                     const at::Tensor& SFB1, const at::Tensor& SFB2,
                     const at::Tensor& C, int64_t flags,
                     const c10::optional<at::Tensor>& workspace) {
  return run(A, B1, B2, SFA, SFB1, SFB2, C, flags,
             workspace.has_value() ? &workspace.value() : nullptr);
}

}  // namespace

PYBIND11_MODULE(_C, m) {
  m.doc() = "torch binding of the NVFP4 dual GEMM C ABI (libnvfp4dg.so)";
  m.def("custom_kernel", &custom_kernel, py::arg("data"));
  m.def("cuda_nvfp4_dual_gemm", &cuda_nvfp4_dual_gemm, py::arg("A"),
        py::arg("B1"), py::arg("B2"), py::arg("SFA"), py::arg("SFB1"),
        py::arg("SFB2"), py::arg("C"));
  m.def("dual_gemm", &dual_gemm, py::arg("A"), py::arg("B1"), py::arg("B2"),
        py::arg("SFA"), py::arg("SFB1"), py::arg("SFB2"), py::arg("C"),
        py::arg("flags") = 0, py::arg("workspace") = py::none());
}
