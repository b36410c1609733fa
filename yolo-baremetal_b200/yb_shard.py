"""Image sharding across processes (one per GPU) and the host-side gather.

YOLO26 inference shards by image: rank g of G runs images [g*B/G, (g+1)*B/G)
on its own device replica, with no collective on the data path; only the
detections [B_g, max_det, 6] come back.  The same split is used by the
in-process multi-GPU entry yb_cuda_forward_sharded (include/yb_cuda.h).
gather_detections() collects every rank's rows on every rank (all_gather over
whatever process group is initialised: gloo on CPU, nccl on GPUs), and fails
with the group's timeout when a rank never arrives.
"""
from __future__ import annotations

import numpy as np


def shard_bounds(B: int, world: int, rank: int) -> tuple[int, int]:
    """Half-open image range of `rank`: [rank*B//world, (rank+1)*B//world)."""
    if world < 1 or not 0 <= rank < world or B < 0:
        raise ValueError("bad shard geometry")
    return rank * B // world, (rank + 1) * B // world


def gather_detections(local: np.ndarray, B: int, max_det: int = 300) -> np.ndarray:
    """All-gathers per-rank detections [B_rank, max_det, 6] into [B, max_det, 6]
    ordered by image.  Ranks hold different counts; rows are padded to the
    largest shard for the collective and trimmed after."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size()
    rank = dist.get_rank()
    b0, b1 = shard_bounds(B, world, rank)
    if local.shape != (b1 - b0, max_det, 6):
        raise ValueError(f"rank {rank}: expected {(b1 - b0, max_det, 6)}, got {local.shape}")
    cap = max(shard_bounds(B, world, r)[1] - shard_bounds(B, world, r)[0] for r in range(world))
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    buf = torch.zeros((cap, max_det, 6), dtype=torch.float32, device=device)
    buf[: b1 - b0] = torch.from_numpy(np.ascontiguousarray(local)).to(device)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    out = np.empty((B, max_det, 6), dtype=np.float32)
    for r in range(world):
        s0, s1 = shard_bounds(B, world, r)
        out[s0:s1] = parts[r][: s1 - s0].cpu().numpy()
    return out
