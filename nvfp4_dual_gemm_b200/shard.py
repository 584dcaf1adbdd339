"""N-sharding of the dual GEMM over ranks (one process per GPU).

C = silu(A B1^T) * (A B2^T) splits along N with no exchange: rank r of w owns
rows [r N/w, (r+1) N/w) of B1 and B2 and of their blocked scales, A and SFA
are replicated, and the rank computes its own column slice C_r [M, N/w] with
the single-GPU kernel.  In the blocked scale layout (one 512-byte atom per
128 rows x 64 K, atoms ordered row block-major; the reference addresses them
as ``SF + (rowblk * K/64 + k) * 512``, nvfp4_dual_gemm.cu:226-243) the scales
of rows [n0, n1) are the single byte range
[n0/128 * K/64 * 512, n1/128 * K/64 * 512) whenever n0 and n1 are multiples of
128, so a shard is a set of views, never a copy.

:func:`gather_columns` assembles the full C from the slices with one
all-gather; it is a separate collective after the kernels, for callers that
need the whole matrix (the reference has no multi-GPU path).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

ROW_BLOCK = 128   # rows per scale atom
K_ATOM = 64       # K columns per scale atom
ATOM_BYTES = 512  # one 128 x 4 atom of e4m3 scales


@dataclass(frozen=True)
class ShardSpec:
    """Rows [n0, n1) of B1/B2 owned by `rank` of `world`."""
    world: int
    rank: int
    N: int
    K: int
    n0: int
    n1: int

    @property
    def rows(self) -> int:
        return self.n1 - self.n0

    @property
    def scale_bytes(self) -> tuple[int, int]:
        """Byte range of this shard's rows in a blocked scale tensor."""
        per_block = (self.K // K_ATOM) * ATOM_BYTES
        return (self.n0 // ROW_BLOCK * per_block,
                self.n1 // ROW_BLOCK * per_block)


def shard_spec(N: int, K: int, world: int, rank: int) -> ShardSpec:
    """Even split of N over `world` ranks; each slice a multiple of 128 rows
    (so its blocked scales are one contiguous range)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    if K % 256:
        raise ValueError(f"K = {K} must be a multiple of 256")
    if N % (world * ROW_BLOCK):
        raise ValueError(
            f"N = {N} does not split into {world} slices of a multiple of "
            f"{ROW_BLOCK} rows")
    rows = N // world
    return ShardSpec(world, rank, N, K, rank * rows, (rank + 1) * rows)


def _flat_bytes(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.reshape(-1).view(torch.uint8)


def shard_weights(spec: ShardSpec, B1: torch.Tensor, B2: torch.Tensor,
                  SFB1: torch.Tensor, SFB2: torch.Tensor):
    """Views of this rank's rows of B1, B2 ([N, K/2] packed codes) and of the
    matching blocked scales SFB1, SFB2 (N*K/16 bytes).  Returns
    (B1_r, B2_r, SFB1_r, SFB2_r); no data moves."""
    out = []
    for name, b in (("B1", B1), ("B2", B2)):
        if b.size(0) != spec.N or b.size(1) * 2 != spec.K:
            raise ValueError(f"{name} has shape {tuple(b.shape)}, expected "
                             f"[{spec.N}, {spec.K // 2}]")
        out.append(b[spec.n0:spec.n1])
    lo, hi = spec.scale_bytes
    for name, sf in (("SFB1", SFB1), ("SFB2", SFB2)):
        flat = _flat_bytes(sf, name)
        if flat.numel() != spec.N * spec.K // 16:
            raise ValueError(f"{name} holds {flat.numel()} bytes, expected "
                             f"{spec.N * spec.K // 16}")
        out.append(flat[lo:hi].view(sf.dtype))
    return tuple(out)


def sharded_dual_gemm(spec: ShardSpec, A, B1, B2, SFA, SFB1, SFB2,
                      C_local: torch.Tensor | None = None, **kw):
    """This rank's slice C_r = silu(A B1_r^T) * (A B2_r^T), [M, N/w] fp16,
    through the single-GPU kernel.  B1/B2/SFB1/SFB2 are the full tensors."""
    from .api import dual_gemm

    b1, b2, s1, s2 = shard_weights(spec, B1, B2, SFB1, SFB2)
    if C_local is None:
        C_local = torch.empty(A.size(0), spec.rows, dtype=torch.float16,
                              device=A.device)
    return dual_gemm(A, b1, b2, SFA, s1, s2, C_local, **kw)


def gather_columns(C_local: torch.Tensor, spec: ShardSpec, group=None):
    """All-gather the [M, N/w] slices of every rank into the full [M, N]
    (rank r's slice lands in columns [n0_r, n1_r))."""
    import torch.distributed as dist

    M = C_local.size(0)
    if C_local.shape != (M, spec.rows):
        raise ValueError(f"C_local has shape {tuple(C_local.shape)}, expected "
                         f"[M, {spec.rows}]")
    parts = [torch.empty_like(C_local) for _ in range(spec.world)]
    dist.all_gather(parts, C_local.contiguous(), group=group)
    return torch.cat(parts, dim=1)


def max_over_ranks(value: float, device="cpu", group=None) -> float:
    """Max of a per-rank scalar (a device-timed duration) over the group;
    `device` is where the collective's buffer lives ("cuda" for NCCL)."""
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
