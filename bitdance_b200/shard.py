"""N-sharded (column-parallel) W4A6 GEMM across the GPUs of one node.

Each rank holds rows [r*N/w, (r+1)*N/w) of the NVFP4 weight matrix (its own packed shard,
the fp32 tensor scale replicated) and the full MXFP6 activations, and computes
C[:, shard] with no communication. Only when the caller asks for the full C are the shards
all-gathered over NCCL (NVLink / NVSwitch) and reassembled as (M, N).

The reference is single-GPU (HIP_VISIBLE_DEVICES pinned, REPRODUCE.md:70-72); this module
is the scale-out this build adds for the 70B-shaped config.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import ops


def shard_rows(N: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of an N-row weight matrix owned by `rank` of `world`. Every shard must
    be a whole number of 128-row tiles."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if N % (128 * world):
        raise ValueError(f"N={N} does not split into {world} shards of whole 128-row tiles")
    per = N // world
    return rank * per, (rank + 1) * per


def shard_weights(codes: torch.Tensor, scales16: torch.Tensor, tensor_scale: float, rank: int,
                  world: int, stream=None) -> ops.PackedWeights:
    """This rank's shard of natural-layout NVFP4 weights ((N, K/2) codes, (N, K/16) scales),
    packed for the GEMM on this rank's device."""
    lo, hi = shard_rows(codes.shape[0], world, rank)
    return ops.pack_weights(codes[lo:hi].contiguous(), scales16[lo:hi].contiguous(),
                            tensor_scale, stream=stream)


def assemble(gathered: torch.Tensor) -> torch.Tensor:
    """(world, M, N/world) shard outputs -> (M, N) with shard r in columns r*N/w.."""
    w, M, n = gathered.shape
    return gathered.permute(1, 0, 2).reshape(M, w * n)


def sharded_gemm(acts: ops.PackedActivations, shard: ops.PackedWeights, gather: bool = False,
                 group: Optional[dist.ProcessGroup] = None, out: Optional[torch.Tensor] = None,
                 workspace=None, **kw) -> torch.Tensor:
    """C_shard = A . B_shard^T on this rank; with gather=True the full (M, N) C on every rank
    (NCCL all-gather of the bf16 shards, then reassembly)."""
    C = ops.w4a6_gemm(acts, shard, out=out, workspace=workspace, **kw)
    if not gather:
        return C
    world = dist.get_world_size(group)
    M, n = C.shape
    buf = torch.empty((world * M, n), dtype=C.dtype, device=C.device)
    dist.all_gather_into_tensor(buf, C.contiguous(), group=group)
    return assemble(buf.view(world, M, n))
