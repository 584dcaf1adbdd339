// Python binding of the reference's own kernel, compiled from the reference
// sources where they lie (the include path points at the reference checkout;
// nothing of the reference is copied into this repository).  Test and
// benchmark infrastructure only: it serves as a second oracle on the shapes
// the reference dispatches, and as the reference arm of bench.py.
//
// The reference's nvfp4_dual_gemm.cu includes its PTX headers before the
// standard headers they rely on (uint32_t, printf), and names torch::Tensor
// with only ATen headers included; its own JIT build (load_inline) supplies
// <torch/types.h> ahead of the source, so those come first here.
#include <torch/types.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "nvfp4_dual_gemm.cu"

#include <torch/extension.h>

// Shapes outside the reference's dispatch table (nvfp4_dual_gemm.cu:403-442)
// that the benchmark configurations name: the prefill shape 4096 x 14336 x
// 4096 and the N-sharded 8192 x (28672 / world) x 8192 rank slices for world
// 1, 2, 4, 8.  Each runs the reference's own launcher template
// (launch_nvfp4_dual_gemm, nvfp4_dual_gemm.cu:319-373) with the
// configuration its table uses for its large shapes (BLOCK_M = BLOCK_N = 128,
// BLOCK_K = 256, 4 stages, accurate SiLU, row-major C, nvfp4_dual_gemm.cu:
// 419-440) and one CTA per 128 x 128 tile, the grid being a template
// argument.  Valid there because M % 128 == N % 128 == 0 and K / 256 >= 4.
torch::Tensor cuda_nvfp4_dual_gemm_generic(
    const torch::Tensor& A, const torch::Tensor& B1, const torch::Tensor& B2,
    const torch::Tensor& SFA, const torch::Tensor& SFB1,
    const torch::Tensor& SFB2, torch::Tensor& C) {
  const int M = A.size(0);
  const int N = B1.size(0);
  const int K = A.size(1) * 2;
  TORCH_CHECK(M % 128 == 0 && N % 128 == 0, "M and N must be multiples of 128");
  uint8_t* A_ptr = reinterpret_cast<uint8_t*>(A.data_ptr());
  uint8_t* B1_ptr = reinterpret_cast<uint8_t*>(B1.data_ptr());
  uint8_t* B2_ptr = reinterpret_cast<uint8_t*>(B2.data_ptr());
  uint8_t* SFA_ptr = reinterpret_cast<uint8_t*>(SFA.data_ptr());
  uint8_t* SFB1_ptr = reinterpret_cast<uint8_t*>(SFB1.data_ptr());
  uint8_t* SFB2_ptr = reinterpret_cast<uint8_t*>(SFB2.data_ptr());
  half* C_ptr = reinterpret_cast<half*>(C.data_ptr());
  const long long grid = static_cast<long long>(M / 128) * (N / 128);
  if (K == 4096 && grid == 3584) {
    LAUNCH(4096, 128, 128, 256, 4, false, false, false, 3584);
  } else if (K == 8192 && grid == 14336) {
    LAUNCH(8192, 128, 128, 256, 4, false, false, false, 14336);
  } else if (K == 8192 && grid == 7168) {
    LAUNCH(8192, 128, 128, 256, 4, false, false, false, 7168);
  } else if (K == 8192 && grid == 3584) {
    LAUNCH(8192, 128, 128, 256, 4, false, false, false, 3584);
  } else if (K == 8192 && grid == 1792) {
    LAUNCH(8192, 128, 128, 256, 4, false, false, false, 1792);
  } else {
    TORCH_CHECK(false, "shape ", M, "x", N, "x", K,
                " has no instantiation of the reference launcher");
  }
  return C;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("cuda_nvfp4_dual_gemm", &cuda_nvfp4_dual_gemm,
        "reference NVFP4 dual GEMM (13 hard-coded shapes)");
  m.def("cuda_nvfp4_dual_gemm_generic", &cuda_nvfp4_dual_gemm_generic,
        "the reference's launcher template instantiated for the benchmark "
        "shapes outside its table (4096x14336x4096, 8192x(28672/w)x8192)");
}
