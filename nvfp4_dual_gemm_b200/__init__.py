"""B200-native (sm_100a) NVFP4 dual GEMM: C = silu(A B1^T) * (A B2^T).

Drop-in for the reference's ``custom_kernel(data)`` path; the compute runs in
the in-tree CUDA library ``libnvfp4dg.so`` behind the C ABI declared in
``include/nvfp4_dual_gemm.h``.
"""
from .api import (  # noqa: F401
    cuda_nvfp4_dual_gemm,
    custom_kernel,
    dual_gemm,
    dual_gemm_grouped,
    dual_gemm_host,
    dual_gemm_nvfp4,
    generate_input,
    group_offsets,
    grouped_workspace_size,
    host_staging_size,
    plan,
    plan_work,
    quantize_nvfp4,
    scales_from_blocked,
    scales_to_blocked,
    workspace_size,
)
from .shard import (  # noqa: F401
    ShardSpec,
    gather_columns,
    shard_spec,
    shard_weights,
    sharded_dual_gemm,
)
from ._lib import (  # noqa: F401
    FLAG_BN64,
    FLAG_BN128,
    FLAG_FORCE_STREAMK,
    FLAG_NO_PAIR,
    FLAG_NO_PDL,
    FLAG_NO_SPLITK,
    FLAG_NO_STREAMK,
    FLAG_PAIR,
    FLAG_SPLITK,
    FLAG_STATIC_WEIGHTS,
    FLAG_SYNC_CHECK,
    NativeLibraryError,
)

__version__ = "1.1.0"
