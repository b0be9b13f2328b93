"""Batch x head sharding and the gather to rank 0 (apex_attn/shard.py) on CPU ranks.

Two gloo ranks in child processes (spawned, 127.0.0.1 rendezvous) each compute the
oracle on their slice of the flattened b*h axis; rank 0 gathers and compares with the
unsharded oracle. This is the host-side logic of the multi-GPU path with no GPU.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from apex_attn.shard import shard_heads


def test_shard_heads_partitions_exactly():
    for total in (1, 7, 8, 512, 513):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_heads(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (s0, e0), (s1, _) in zip(spans, spans[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_heads(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, B, H, N, D, result_path):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "apex-tune-results_b200")]
    import datetime

    import torch.distributed as dist
    from apex_attn.shard import gather_to_rank0, shard_heads
    from oracle.attention_oracle import attention_np, make_inputs, to_np32

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v = (to_np32(t).reshape(B * H, 1, N, D) for t in make_inputs(B, H, N, D, seed=13))
        h0, h1 = shard_heads(B * H, world, rank)
        o, _ = attention_np(q[h0:h1], k[h0:h1], v[h0:h1])
        full = gather_to_rank0(torch.from_numpy(o[:, 0]), B * H, world, rank)
        if rank == 0:
            np.save(result_path, full.numpy())
        else:
            assert full is None
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gather_to_rank0_matches_unsharded(tmp_path, world):
    from oracle.attention_oracle import attention_np, make_inputs, to_np32
    B, H, N, D = 1, 5, 40, 64  # 5 heads over 2 ranks: uneven shards (3 + 2)
    out = str(tmp_path / "gathered.npy")
    mp.start_processes(_worker, args=(world, _free_port(), B, H, N, D, out), nprocs=world,
                       join=True, start_method="spawn")
    got = np.load(out)
    q, k, v = (to_np32(t) for t in make_inputs(B, H, N, D, seed=13))
    ref, _ = attention_np(q, k, v)
    np.testing.assert_array_equal(got, ref.reshape(B * H, N, D))
