"""Sequence sharding over ranks (one process per GPU, no collective on the hot path), checked on CPU with
two gloo ranks: the ids every rank generates for its block of sequences, gathered, equal one process
decoding all of them. The per-rank decoder here is the oracle (no GPU on this host); the sharding,
seeding by global index and the gather are the bench's own code.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch.multiprocessing as mp

from tests.helpers import ARCHS, O, oracle_shape, pkg

NEW = 5


def _workload(seqs):
    return pkg.configs.Workload("tiny", pkg.ModelConfig(**ARCHS[3][1]), weight_seed=5, seqs=seqs, prompt_len=6,
                                new_tokens=NEW)


def _decode(w, prompts):
    p = pkg.init_params(w.model, w.weight_seed)
    model = O.Model(oracle_shape(w.model, "F32"), p.astype(np.float64))
    return model.cached_generate_batch(prompts, NEW)[:, -NEW:]


def _rank(rank, world, port, out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        w = _workload(3)
        ids = _decode(w, pkg.sharding.shard_prompts(w, rank))
        everything = pkg.sharding.gather_ids(ids, dist)
        if rank == 0:
            np.save(out, everything)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_decode_like_one_process(tmp_path):
    out = str(tmp_path / "ids.npy")
    mp.spawn(_rank, args=(2, _free_port(), out), nprocs=2, join=True)
    gathered = np.load(out)
    alone = _decode(_workload(6), pkg.sharding.shard_prompts(_workload(6), 0))
    assert gathered.shape == (6, NEW)
    assert np.array_equal(gathered, alone)


def test_shard_prompts_follow_global_index():
    w = _workload(4)
    assert np.array_equal(pkg.sharding.shard_prompts(w, 1)[2], pkg.sharding.uniform_ids(6, 12, 1000 + 6))
    assert np.array_equal(pkg.sharding.uniform_ids(6, 12, 1000 + 6), O.uniform_ids(6, 12, seed=1006))
