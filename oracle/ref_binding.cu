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

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("cuda_nvfp4_dual_gemm", &cuda_nvfp4_dual_gemm,
        "reference NVFP4 dual GEMM (13 hard-coded shapes)");
}
