"""Multi-GPU plumbing for data-parallel decoding: one process per GPU, each decoding its own
utterances with no collective on the decode path; codes are gathered to rank 0 afterwards.

Works with any torch.distributed backend (NCCL over NVLink on the GPU box, gloo on CPU tests)."""
from __future__ import annotations

import torch
import torch.distributed as dist


def _device_for(backend: str) -> torch.device:
    return torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")


def max_over_ranks(x: float) -> float:
    """Max of a scalar over all ranks (timing rule: a multi-GPU step takes as long as the
    slowest rank)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=_device_for(dist.get_backend()))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_codes(codes: torch.Tensor, dst: int = 0):
    """Gather every rank's int32 codes [n_frames, 16] (n_frames may differ per rank) to rank
    ``dst``. Returns the list of per-rank tensors on ``dst`` and None elsewhere. Implemented as
    an all-gather of the lengths plus an all-gather of padded buffers (collectives every backend
    supports)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [codes]
    dev = _device_for(dist.get_backend())
    world = dist.get_world_size()
    codes = codes.to(dev, torch.int32).contiguous()
    n = torch.tensor([codes.shape[0]], dtype=torch.int64, device=dev)
    lens = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(lens, n)
    lens = [int(x.item()) for x in lens]
    width = codes.shape[1]
    pad = torch.zeros(max(lens), width, dtype=torch.int32, device=dev)
    pad[: codes.shape[0]] = codes
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad)
    if dist.get_rank() != dst:
        return None
    return [b[:l].cpu() for b, l in zip(bufs, lens)]
