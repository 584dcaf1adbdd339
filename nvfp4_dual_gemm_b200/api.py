"""Python host API mirroring the reference's operator interface.

* :func:`custom_kernel` — same name, argument and return contract as the
  reference's entry point (submission.py:1153-1157): ``data`` is the 10-tuple
  ``(a, b1, b2, sfa, sfb1, sfb2, sfa_blocked, sfb1_blocked, sfb2_blocked, c)``;
  the plain scales are ignored, the blocked ones are used, ``c`` is filled and
  returned.
* :func:`cuda_nvfp4_dual_gemm` — the reference's torch-extension function
  (nvfp4_dual_gemm.cu:381-446, declared submission.py:17-20): M = A.size(0),
  N = B1.size(0), K = 2 * A.size(1).

Both call the C ABI (``nvfp4_dual_gemm_run``) on the current torch stream
through the in-tree torch binding ``_C`` (csrc/torch_ext.cpp), which checks
the tensors and launches in a few microseconds of host time.
Error behaviour differs from the reference on purpose: the reference accepts
only 13 hard-coded shapes and silently returns ``c`` untouched for any other
(nvfp4_dual_gemm.cu:443-444); here every shape that meets the preconditions
(N % 64 == 0, K % 256 == 0, L >= 1) is computed and anything else raises
``ValueError``.  The reference returns a transposed view for one shape
(nvfp4_dual_gemm.cu:413-415); here ``c`` itself, row-major, is always returned.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

__all__ = [
    "custom_kernel",
    "cuda_nvfp4_dual_gemm",
    "dual_gemm",
    "dual_gemm_host",
    "host_staging_size",
    "quantize_nvfp4",
    "scales_to_blocked",
    "scales_from_blocked",
    "generate_input",
    "workspace_size",
    "plan",
]


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check_bytes(name: str, t: torch.Tensor, cuda: bool = True) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.element_size() != 1:
        raise ValueError(f"{name} must hold 1-byte elements "
                         f"(fp4x2 / fp8 / uint8), got {t.dtype}")
    placed = t.is_cuda if cuda else t.device.type == "cpu"
    if not placed:
        raise ValueError(f"{name} must be a {'CUDA' if cuda else 'CPU'} "
                         "tensor")


def _batches(t: torch.Tensor) -> int:
    """L of a [rows, cols] or [rows, cols, L] operand."""
    return t.size(2) if t.dim() == 3 else 1


def _rows_dense(name: str, t: torch.Tensor, rows: int, row_bytes: int,
                L: int = 1) -> None:
    """[rows, row_bytes] or [rows, row_bytes, L]: rows dense and K-major; a
    batch (L > 1) stored batch after batch (``t.movedim(-1, 0)`` contiguous,
    the layout of a [L, rows, row_bytes] tensor viewed through
    ``permute(1, 2, 0)``, as the reference's harness builds its tensors)."""
    if t.dim() not in (2, 3):
        raise ValueError(f"{name} must be [rows, K/2] or [rows, K/2, L]")
    if _batches(t) != L:
        raise ValueError(f"{name} holds {_batches(t)} batches, A holds {L}")
    if t.size(0) != rows or t.size(1) != row_bytes:
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected "
                         f"[{rows}, {row_bytes}(, {L})]")
    if rows > 1 and row_bytes > 0 and t.stride(0) != row_bytes:
        raise ValueError(f"{name} rows must be dense (stride(0) == K/2)")
    if row_bytes > 1 and t.stride(1) != 1:
        raise ValueError(f"{name} must be K-major (stride(1) == 1)")
    if L > 1 and rows * row_bytes > 0 and t.stride(2) != rows * row_bytes:
        raise ValueError(f"{name}: the batches must follow one another "
                         f"(stride(2) == {rows * row_bytes})")


def _blocked_bytes(rows: int, k: int) -> int:
    return ((rows + 127) // 128) * (k // 64) * 512


def _check_blocked(name: str, t: torch.Tensor, rows: int, k: int,
                   cuda: bool = True, L: int = 1) -> None:
    """Blocked scales: contiguous bytes, or for a batch (L > 1) a tensor whose
    last dimension is the batch, stored batch after batch; each batch holds
    the blocked layout of its rows."""
    _check_bytes(name, t, cuda)
    need = _blocked_bytes(rows, k)
    dense = t.is_contiguous() or (
        L > 1 and t.dim() >= 2 and t.size(-1) == L and
        t.movedim(-1, 0).is_contiguous())
    if not dense:
        raise ValueError(f"{name} must be contiguous (batch after batch)")
    if L > 1 and not t.is_contiguous() and t.numel() != L * need:
        raise ValueError(f"{name} holds {t.numel()} bytes, {L} batches of the "
                         f"blocked layout need {L * need}")
    if t.numel() < L * need:
        raise ValueError(f"{name} holds {t.numel()} bytes, the blocked layout "
                         f"needs {L * need}")


def _check_problem(A, B1, B2, SFA, SFB1, SFB2, C, cuda: bool):
    """Shape, dtype and placement checks shared by both entry points;
    returns (M, N, K)."""
    M, N, K, L = _check_inputs(A, B1, B2, SFA, SFB1, SFB2, cuda)
    if C.dtype != torch.float16:
        raise ValueError(f"C must be float16, got {C.dtype}")
    where = "CUDA" if cuda else "CPU"
    placed = C.is_cuda if cuda else C.device.type == "cpu"
    batch_major = C.is_contiguous() or (
        L > 1 and C.dim() == 3 and C.movedim(-1, 0).is_contiguous())
    if not placed or not batch_major:
        raise ValueError(f"C must be a contiguous {where} tensor "
                         "(batch after batch)")
    if C.numel() != L * M * N or C.size(0) != M or \
            (C.dim() == 3 and C.size(2) != L):
        raise ValueError(f"C has shape {tuple(C.shape)}, expected "
                         f"[{M}, {N}(, {L})]")
    if L > 1 and C.dim() != 3:
        raise ValueError(f"C must be [{M}, {N}, {L}] for a batch")
    return M, N, K, L


def _check_inputs(A, B1, B2, SFA, SFB1, SFB2, cuda: bool):
    for name, t in (("A", A), ("B1", B1), ("B2", B2)):
        _check_bytes(name, t, cuda)
    M = A.size(0)
    N = B1.size(0)
    K = 2 * A.size(1) if A.dim() >= 2 else 0
    L = _batches(A)
    if L < 1:
        raise ValueError("L must be >= 1")
    _rows_dense("A", A, M, K // 2, L)
    _rows_dense("B1", B1, N, K // 2, L)
    _rows_dense("B2", B2, N, K // 2, L)
    if N % 64 != 0:
        raise ValueError(f"N = {N} must be a multiple of 64")
    if K % 256 != 0:
        raise ValueError(f"K = {K} must be a multiple of 256")
    _check_blocked("SFA", SFA, M, K, cuda, L)
    _check_blocked("SFB1", SFB1, N, K, cuda, L)
    _check_blocked("SFB2", SFB2, N, K, cuda, L)
    return M, N, K, L


def dual_gemm(A, B1, B2, SFA, SFB1, SFB2, C, *, flags: int = 0,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """C = silu(A B1^T) * (A B2^T) on the current stream; returns C.

    ``flags`` are the NVFP4DG_FLAG_* bits of the C ABI (0 = automatic).  With
    ``workspace`` (a zero-initialised uint8 CUDA tensor of at least
    :func:`workspace_size` bytes) the caller owns the split-K scratch;
    otherwise the library keeps one per (device, stream).  The checks (the
    same rules as :func:`dual_gemm_host`'s) and the call of
    ``nvfp4_dual_gemm_run`` / ``_run_ws`` run in the torch binding ``_C``."""
    return _lib.ext().dual_gemm(A, B1, B2, SFA, SFB1, SFB2, C, flags,
                                workspace)


def dual_gemm_nvfp4(A, B1, B2, SFA, SFB1, SFB2, Cq=None, SFC=None, *,
                    flags: int = 0):
    """The dual GEMM with its result in NVFP4, for the next GEMM of an FFN:
    returns (Cq, SFC), the e2m1 codes [M, N/2] (uint8, element 2i in the low
    nibble) and the blocked e4m3 scales of h = fp16(silu(A B1^T) * (A B2^T)),
    equal bit for bit to ``quantize_nvfp4`` of :func:`dual_gemm`'s C.  The
    fp16 C is never written (``nvfp4_dual_gemm_run_nvfp4_out``).  ``Cq`` /
    ``SFC`` are allocated on A's device when not given.  For a batch (A of
    shape [M, K/2, L]) Cq is [M, N/2, L] stored batch after batch and SFC
    holds L blocked layouts one after another."""
    M, N, K, L = _check_inputs(A, B1, B2, SFA, SFB1, SFB2, cuda=True)
    dev = A.device
    if Cq is None:
        Cq = (torch.empty((M, N // 2), dtype=torch.uint8, device=dev)
              if L == 1 else
              torch.empty((L, M, N // 2), dtype=torch.uint8,
                          device=dev).permute(1, 2, 0))
    if SFC is None:
        SFC = torch.empty(max(L * _blocked_bytes(M, N), 1), dtype=torch.uint8,
                          device=dev)
    _check_bytes("Cq", Cq, True)
    _rows_dense("Cq", Cq, M, N // 2, L)
    _check_blocked("SFC", SFC, M, N, True, L)
    for name, t in (("B1", B1), ("B2", B2), ("SFA", SFA), ("SFB1", SFB1),
                    ("SFB2", SFB2), ("Cq", Cq), ("SFC", SFC)):
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, A on {dev}")
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.nvfp4_dual_gemm_run_nvfp4_out(
            _ptr(A), _ptr(B1), _ptr(B2), _ptr(SFA), _ptr(SFB1), _ptr(SFB2),
            _ptr(Cq), _ptr(SFC), M, N, K, L, flags, _stream(dev))
    _lib.check(rc, "nvfp4_dual_gemm_run_nvfp4_out")
    return Cq, SFC


def group_offsets(group_rows) -> list[int]:
    """Default first rows of the groups: each group's rows rounded up to 128,
    one group after another."""
    out, r = [], 0
    for n in group_rows:
        out.append(r)
        r += (int(n) + 127) // 128 * 128
    return out


def grouped_workspace_size(group_rows, N: int, K: int,
                           flags: int = 0) -> int:
    """Bytes of caller-owned workspace :func:`dual_gemm_grouped` needs."""
    rows = [int(n) for n in group_rows]
    lib = _lib.load()
    return int(lib.nvfp4_dual_gemm_grouped_workspace_size(
        (ctypes.c_int * len(rows))(*rows), len(rows), N, K, flags))


def dual_gemm_grouped(A, B1, B2, SFA, SFB1, SFB2, C, group_rows,
                      group_row0=None, *, flags: int = 0,
                      workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Grouped dual GEMM (a mixture-of-experts FFN) in one launch: group g
    computes rows [row0[g], row0[g] + group_rows[g]) of C from the same rows
    of A / SFA and expert g's weights (batch g of B1, B2 [N, K/2, G] and of
    SFB1 / SFB2, G blocked layouts one after another).  ``group_row0``
    (multiples of 128, increasing, non-overlapping once each group's rows are
    rounded up to 128) defaults to :func:`group_offsets`.  A is [R, K/2], SFA
    the blocked layout of R rows and C [R, N] with R = max(row0 + rows); rows
    outside the groups are not written (``nvfp4_dual_gemm_run_grouped``).
    ``workspace`` (zero-initialised uint8 CUDA tensor of at least
    :func:`grouped_workspace_size` bytes) makes the call allocation-free,
    e.g. for CUDA graph capture; otherwise the library keeps one."""
    rows = [int(n) for n in group_rows]
    G = len(rows)
    row0 = group_offsets(rows) if group_row0 is None else \
        [int(r) for r in group_row0]
    if len(row0) != G:
        raise ValueError("group_row0 needs one entry per group")
    R = max([r + n for r, n in zip(row0, rows) if n > 0], default=0)
    for name, t in (("A", A), ("B1", B1), ("B2", B2)):
        _check_bytes(name, t, True)
    N = B1.size(0)
    K = 2 * B1.size(1) if B1.dim() >= 2 else 0
    _rows_dense("A", A, A.size(0), K // 2)
    if A.size(0) < R:
        raise ValueError(f"A has {A.size(0)} rows, the groups need {R}")
    _rows_dense("B1", B1, N, K // 2, G)
    _rows_dense("B2", B2, N, K // 2, G)
    _check_blocked("SFA", SFA, A.size(0), K, True)
    _check_blocked("SFB1", SFB1, N, K, True, G)
    _check_blocked("SFB2", SFB2, N, K, True, G)
    if (C.dtype != torch.float16 or not C.is_cuda or not C.is_contiguous()
            or C.dim() != 2 or C.size(1) != N or C.size(0) < R):
        raise ValueError(f"C must be a contiguous CUDA float16 [>= {R}, {N}] "
                         "tensor")
    dev = C.device
    for name, t in (("A", A), ("B1", B1), ("B2", B2), ("SFA", SFA),
                    ("SFB1", SFB1), ("SFB2", SFB2)):
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, C on {dev}")
    arr = ctypes.c_int * G
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.nvfp4_dual_gemm_run_grouped(
            _ptr(A), _ptr(B1), _ptr(B2), _ptr(SFA), _ptr(SFB1), _ptr(SFB2),
            _ptr(C), arr(*rows), arr(*row0), G, N, K, flags,
            None if workspace is None else _ptr(workspace),
            0 if workspace is None else workspace.numel(), _stream(dev))
    _lib.check(rc, "nvfp4_dual_gemm_run_grouped")
    return C


def host_staging_size(M: int, N: int, K: int) -> int:
    """Bytes of device staging :func:`dual_gemm_host` needs (host-only)."""
    lib = _lib.load()
    n = lib.nvfp4_dual_gemm_host_staging_size(M, N, K, 1)
    msg = _lib.last_error()
    if n == 0 and msg:
        raise ValueError(msg)
    return int(n)


# Staging buffers dual_gemm_host keeps per (device, stream): calls on one
# stream are ordered, so they may share one.
_staging: dict[tuple[int, int], torch.Tensor] = {}


def dual_gemm_host(A, B1, B2, SFA, SFB1, SFB2, C, *, flags: int = 0,
                   slabs: int = 0, device: torch.device | int | None = None,
                   staging: torch.Tensor | None = None) -> torch.Tensor:
    """The same product with every tensor in HOST memory (page-locked, e.g.
    ``tensor.pin_memory()``, for the copies to overlap).

    Uploads the inputs to ``device`` (default: the current CUDA device),
    computes and downloads C, overlapping the weight upload, the kernels and
    the download slab by slab (``nvfp4_dual_gemm_run_host``).  Work is queued
    on the device's current stream; C is complete once that stream is
    (``torch.cuda.current_stream(device).synchronize()``).  ``staging``, a
    uint8 CUDA tensor of at least :func:`host_staging_size` bytes, is the
    device buffer the inputs go through; by default the library keeps one per
    (device, stream)."""
    M, N, K, L = _check_problem(A, B1, B2, SFA, SFB1, SFB2, C, cuda=False)
    if L != 1:
        raise ValueError("dual_gemm_host takes unbatched problems (L = 1)")
    dev = torch.device("cuda", torch.cuda.current_device()
                       if device is None else torch.device(device).index or 0)
    lib = _lib.load()
    need = host_staging_size(M, N, K)
    with torch.cuda.device(dev):
        stream = _stream(dev)
        if staging is None:
            key = (dev.index, stream)
            buf = _staging.get(key)
            if buf is None or buf.numel() < need:
                buf = torch.empty(max(need, 1), dtype=torch.uint8,
                                  device=dev)
                _staging[key] = buf
        else:
            if (not staging.is_cuda or staging.device != dev or
                    not staging.is_contiguous()):
                raise ValueError("staging must be a contiguous CUDA tensor on "
                                 f"{dev}")
            buf = staging
        rc = lib.nvfp4_dual_gemm_run_host(
            _ptr(A), _ptr(B1), _ptr(B2), _ptr(SFA), _ptr(SFB1), _ptr(SFB2),
            _ptr(C), M, N, K, 1, flags, slabs, _ptr(buf),
            buf.numel() * buf.element_size(), stream)
    _lib.check(rc, "nvfp4_dual_gemm_run_host")
    return C


def cuda_nvfp4_dual_gemm(A, B1, B2, SFA, SFB1, SFB2, C) -> torch.Tensor:
    """Drop-in for the reference's ``cuda_nvfp4_dual_gemm`` (same arguments:
    packed A/B1/B2, blocked SFA/SFB1/SFB2, preallocated fp16 C)."""
    return _lib.ext().cuda_nvfp4_dual_gemm(A, B1, B2, SFA, SFB1, SFB2, C)


def custom_kernel(data):
    """Drop-in for the reference's ``custom_kernel(data)``: ``data`` is
    ``(a, b1, b2, sfa, sfb1, sfb2, sfa_blocked, sfb1_blocked, sfb2_blocked,
    c)``; unpacked, checked and launched in the torch binding (a few
    microseconds of host time per call)."""
    return _lib.ext().custom_kernel(data)


def workspace_size(M: int, N: int, K: int, flags: int = 0,
                   device: torch.device | int | None = None,
                   L: int = 1) -> int:
    """Bytes of caller-owned workspace :func:`dual_gemm` needs (0 = none)
    for L problems of shape M x N x K."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()
                       if device is None else torch.device(device).index or 0)
    with torch.cuda.device(dev):
        n = lib.nvfp4_dual_gemm_workspace_size(M, N, K, L, flags)
    msg = _lib.last_error()
    if n == 0 and msg:
        raise RuntimeError(msg)
    return int(n)


def plan(M: int, N: int, K: int, flags: int = 0, num_sms: int = 148) -> dict:
    """The schedule the library would use (host-only; needs no GPU)."""
    lib = _lib.load()
    bn, ctas, grid, dp, sk, split = (ctypes.c_int() for _ in range(6))
    rc = lib.nvfp4_dual_gemm_plan(M, N, K, flags, num_sms, ctypes.byref(bn),
                                  ctypes.byref(ctas), ctypes.byref(grid),
                                  ctypes.byref(dp), ctypes.byref(sk),
                                  ctypes.byref(split))
    _lib.check(rc, "nvfp4_dual_gemm_plan")
    return {"bn": bn.value, "ctas": ctas.value, "grid": grid.value,
            "dp_tiles": dp.value, "sk_tiles": sk.value,
            "split": split.value}


def plan_work(M: int, N: int, K: int, cta: int, flags: int = 0,
              num_sms: int = 148) -> list[tuple[int, int, int, int]]:
    """Work records (tile, kb_begin, kb_end, slot) of one work unit (a CTA or
    a 2-SM CTA pair; host-only)."""
    lib = _lib.load()
    n = lib.nvfp4_dual_gemm_plan_work(M, N, K, flags, num_sms, cta, None, 0)
    if n < 0:
        raise ValueError(_lib.last_error())
    buf = (ctypes.c_int * (4 * max(n, 1)))()
    lib.nvfp4_dual_gemm_plan_work(M, N, K, flags, num_sms, cta, buf, n)
    return [tuple(buf[4 * i:4 * i + 4]) for i in range(n)]


_QUANT_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16,
                 torch.bfloat16: _lib.DTYPE_BF16}


def quantize_nvfp4(x: torch.Tensor, plain: bool = True):
    """Activation quantiser: a [rows, K] CUDA tensor of float32, float16 or
    bfloat16 (rows may be strided: stride(1) == 1, the row pitch a multiple
    of 16 bytes) -> (codes [rows, K/2] uint8, plain scales [rows, K/16]
    float8_e4m3fn or None when ``plain`` is False, blocked scales uint8), by
    the library's quantiser kernel on the current stream."""
    if x.dtype not in _QUANT_DTYPES or not x.is_cuda or x.dim() != 2:
        raise ValueError("x must be a 2-D float32 / float16 / bfloat16 CUDA "
                         "tensor")
    if x.stride(1) != 1 or (x.stride(0) * x.element_size()) % 16 != 0:
        x = x.contiguous()
    rows, k = x.shape
    if k % 64 != 0:
        raise ValueError("K must be a multiple of 64")
    codes = torch.empty((rows, k // 2), dtype=torch.uint8, device=x.device)
    sf = (torch.empty((rows, k // 16), dtype=torch.uint8, device=x.device)
          if plain else None)
    blk = torch.empty((_blocked_bytes(rows, k),), dtype=torch.uint8,
                      device=x.device)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.nvfp4_quantize_rows(
            _ptr(x), _QUANT_DTYPES[x.dtype], rows, k, max(x.stride(0), k),
            _ptr(codes), None if sf is None else _ptr(sf), _ptr(blk),
            _stream(x.device))
    _lib.check(rc, "nvfp4_quantize_rows")
    return codes, (None if sf is None else sf.view(torch.float8_e4m3fn)), blk


def _byte_view(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.element_size() == 1 else t


def scales_to_blocked(sf: torch.Tensor) -> torch.Tensor:
    """Plain scales [rows, K/16] (1-byte CUDA tensor, rows may be strided:
    stride(1) == 1, row pitch a multiple of 4 bytes) -> the blocked layout
    the dual GEMM reads (uint8, padding rows zero), on the current stream."""
    if not sf.is_cuda or sf.dim() != 2 or sf.element_size() != 1:
        raise ValueError("sf must be a 2-D 1-byte CUDA tensor")
    sf = _byte_view(sf)
    if sf.stride(1) != 1 or sf.stride(0) % 4 != 0:
        sf = sf.contiguous()
    rows, kb = sf.shape
    k = kb * 16
    if k % 64 != 0:
        raise ValueError("K / 16 must be a multiple of 4")
    out = torch.empty((_blocked_bytes(rows, k),), dtype=torch.uint8,
                      device=sf.device)
    lib = _lib.load()
    with torch.cuda.device(sf.device):
        rc = lib.nvfp4_scales_to_blocked(_ptr(sf), rows, k,
                                         max(sf.stride(0), kb), _ptr(out),
                                         _stream(sf.device))
    _lib.check(rc, "nvfp4_scales_to_blocked")
    return out


def scales_from_blocked(blocked: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """Blocked scales (1-byte CUDA tensor) -> plain [rows, K/16] uint8, on
    the current stream."""
    if not blocked.is_cuda or blocked.element_size() != 1:
        raise ValueError("blocked must be a 1-byte CUDA tensor")
    blocked = _byte_view(blocked).contiguous()
    if k % 64 != 0:
        raise ValueError("K must be a multiple of 64")
    if blocked.numel() < _blocked_bytes(rows, k):
        raise ValueError("blocked holds fewer bytes than the layout needs")
    out = torch.empty((rows, k // 16), dtype=torch.uint8, device=blocked.device)
    lib = _lib.load()
    with torch.cuda.device(blocked.device):
        rc = lib.nvfp4_scales_from_blocked(_ptr(blocked), rows, k, _ptr(out),
                                           k // 16, _stream(blocked.device))
    _lib.check(rc, "nvfp4_scales_from_blocked")
    return out


def generate_input(m: int, n: int, k: int, l: int = 1, seed: int = 0,
                   a_scale: float = 1.0, w_scale: float = 1.0,
                   device="cuda"):
    """Seeded synthetic ``data`` tuple for :func:`custom_kernel`: randn fp32
    activations / weights (times a_scale / w_scale) quantised to NVFP4 on the
    GPU.  Tensors: a/b1/b2 float4_e2m1fn_x2 [rows, K/2, l], plain scales
    float8_e4m3fn [rows, K/16, l], blocked scales float8_e4m3fn (flat, l
    blocked layouts one after another), c float16 [m, n, l]; for l > 1 each
    [rows, cols, l] tensor is a [l, rows, cols] tensor viewed through
    ``permute(1, 2, 0)`` (batch after batch in memory).  Batch 0 is the same
    for every l."""
    if l < 1:
        raise ValueError("l must be >= 1")
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    out = []
    plain = []
    blocked = []
    for idx, (rows, scale) in enumerate(((m, a_scale), (n, w_scale),
                                         (n, w_scale))):
        codes_l, sf_l, blk_l = [], [], []
        for b in range(l):
            gen.manual_seed(seed * 1000003 + idx + 7919 * b)
            x = torch.randn((rows, k), generator=gen, device=dev,
                            dtype=torch.float32)
            if scale != 1.0:
                x.mul_(scale)
            codes, sf, blk = quantize_nvfp4(x)
            del x
            codes_l.append(codes)
            sf_l.append(sf)
            blk_l.append(blk)
        codes = torch.stack(codes_l).permute(1, 2, 0)
        out.append(codes.view(torch.float4_e2m1fn_x2))
        plain.append(torch.stack(sf_l).permute(1, 2, 0))
        blocked.append(torch.cat(blk_l).view(torch.float8_e4m3fn))
    c = torch.empty((l, m, n), dtype=torch.float16,
                    device=dev).permute(1, 2, 0)
    return (out[0], out[1], out[2], plain[0], plain[1], plain[2],
            blocked[0], blocked[1], blocked[2], c)
