"""Multi-GPU column sharding of the quantized matmul (one process per GPU).

The reference has no tensor parallelism (its only multi-device code is a
layer partition helper, crates/opencuda-multidev/src/lib.rs:28-83).  For the
large-N INT4 GEMMs this module splits W^T [N][K] (as the reference
quantizes it) by output rows across the ranks of a torch.distributed group:
rank r owns rows [r*N/g, (r+1)*N/g) -- its packed INT4 bytes and group
scales are a contiguous slice, because every row is a whole number of
groups.  Activations are replicated.  Each rank computes its [M][N/g] block
with the CUDA library and one all-gather (NCCL over NVLink on GPUs, gloo on
CPU) brings the blocks to every rank, where oc_gather_columns (GPU) or a
permute (CPU) lays them out as [M][N].  There is no other exchange.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ColumnShard:
    """Partition of N output columns over `world` ranks."""

    n: int
    world: int

    def __post_init__(self):
        if self.world < 1 or self.n % self.world:
            raise ValueError(f"N={self.n} is not divisible by {self.world} ranks")

    @property
    def cols(self) -> int:
        return self.n // self.world

    def rows(self, rank: int) -> tuple[int, int]:
        """Rows of W^T (output columns) owned by `rank`: [start, end)."""
        if not 0 <= rank < self.world:
            raise ValueError(f"rank {rank} out of range for {self.world} ranks")
        return rank * self.cols, (rank + 1) * self.cols

    def w4_slices(self, rank: int, k: int, group: int):
        """Byte range of the packed INT4 W^T and range of its group scales."""
        if k % group or k % 2:
            raise ValueError("k must be even and a multiple of the group size")
        r0, r1 = self.rows(rank)
        return (r0 * k // 2, r1 * k // 2), (r0 * (k // group), r1 * (k // group))

    def w8_slices(self, rank: int, k: int):
        r0, r1 = self.rows(rank)
        return (r0 * k, r1 * k), (r0, r1)


def gather_columns(local, plan: ColumnShard, group=None):
    """All-gathers each rank's [M][N/g] block and returns the full [M][N]."""
    import torch
    import torch.distributed as dist

    m = local.shape[0]
    flat = torch.empty(plan.world * local.numel(), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(flat, local.contiguous().view(-1), group=group)
    if local.is_cuda:
        import opencuda_cuda as oc

        out = torch.empty(m, plan.n, dtype=local.dtype, device=local.device)
        oc.check(oc.lib().oc_gather_columns(flat.data_ptr(), out.data_ptr(), plan.world, m, plan.cols,
                                            torch.cuda.current_stream().cuda_stream))
        return out
    return flat.view(plan.world, m, plan.cols).permute(1, 0, 2).reshape(m, plan.n)


def sharded_qgemm_w4a8(A, wq_full, ws_full, group: int, bias_full, plan: ColumnShard, rank: int, pg=None):
    """Y = A . dequant(W4)^T + bias with this rank's column block computed
    locally and the rest gathered.  wq_full / ws_full / bias_full may be the
    full tensors (sliced here) or already this rank's slices."""
    import opencuda_cuda as oc

    k = A.shape[1]
    (b0, b1), (s0, s1) = plan.w4_slices(rank, k, group)
    r0, r1 = plan.rows(rank)
    wq = wq_full[b0:b1] if wq_full.numel() * 2 // k == plan.n else wq_full
    ws = ws_full[s0:s1] if ws_full.numel() * group // k == plan.n else ws_full
    bias = None if bias_full is None else (bias_full[r0:r1] if bias_full.numel() == plan.n else bias_full)
    local = oc.qgemm_w4a8(A, wq, ws, group, bias)
    return gather_columns(local, plan, pg)


def sharded_qgemm_w4(A, wq_full, ws_full, group: int, bias_full, plan: ColumnShard, rank: int, pg=None):
    """Weight-only INT4 (f32 activations, oc_qgemm_w4) with this rank's column
    block computed locally and the rest gathered; arguments as
    sharded_qgemm_w4a8."""
    import opencuda_cuda as oc

    k = A.shape[1]
    (b0, b1), (s0, s1) = plan.w4_slices(rank, k, group)
    r0, r1 = plan.rows(rank)
    wq = wq_full[b0:b1] if wq_full.numel() * 2 // k == plan.n else wq_full
    ws = ws_full[s0:s1] if ws_full.numel() * group // k == plan.n else ws_full
    bias = None if bias_full is None else (bias_full[r0:r1] if bias_full.numel() == plan.n else bias_full)
    local = oc.qgemm_w4(A, wq, ws, group, bias=bias)
    return gather_columns(local, plan, pg)
