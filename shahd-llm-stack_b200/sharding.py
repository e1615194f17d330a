"""Sequence sharding across GPUs (one process per GPU, no collective on the hot path).

Each rank owns a contiguous block of `workload.seqs` sequences with global indices
rank * seqs .. rank * seqs + seqs - 1; a sequence's prompt is drawn from SeededRng(1000 + global index)
(floor(NextFloat() * vocab), Brain/Random/SeededRng.ts:32-40, as Scripts/Bench.ts:41-42 draws prompt
ids), so every sequence decodes the same way whatever the number of GPUs. After the job the ranks
gather their generated ids (a fixed-size int tensor per rank) for checking.
"""
from __future__ import annotations

import numpy as np

PROMPT_SEED_BASE = 1000


def uniform_ids(count: int, vocab: int, seed: int) -> np.ndarray:
    """floor(NextFloat() * vocab) drawn `count` times from SeededRng(seed)."""
    st = seed & 0xFFFFFFFF
    out = np.empty(count, dtype=np.int32)
    for i in range(count):
        st = (st * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = int(st / 4294967296.0 * vocab)
    return out


def global_indices(rank: int, seqs_per_rank: int) -> range:
    return range(rank * seqs_per_rank, (rank + 1) * seqs_per_rank)


def shard_prompts(workload, rank: int) -> np.ndarray:
    """The prompts [seqs, prompt_len] of `rank`'s block of sequences."""
    return np.stack([uniform_ids(workload.prompt_len, workload.model.vocab_size, PROMPT_SEED_BASE + g)
                     for g in global_indices(rank, workload.seqs)])


def gather_ids(ids: np.ndarray, dist) -> np.ndarray:
    """All ranks' generated ids [world * seqs, new] in global sequence order (torch.distributed)."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int64))
    if dist is None or not dist.is_initialized():
        return t.numpy()
    backend = dist.get_backend()
    if backend == "nccl":
        t = t.cuda()
    parts = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return torch.cat(parts).cpu().numpy()
