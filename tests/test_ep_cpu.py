"""Expert parallelism, host side, on CPU with world-size-2 gloo groups: the
expert shards, the communicator-id exchange, and the cross-rank combine of
per-slot outputs (zero outside a rank's experts, summed over ranks) being
bit-identical to one process holding every expert."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from midge_b200 import ep


def test_expert_range_partitions():
    for E, G in [(8, 1), (8, 2), (128, 8), (32, 4), (128, 2)]:
        seen = []
        for r in range(G):
            a, b = ep.expert_range(E, G, r)
            seen.extend(range(a, b))
            assert all(ep.owner(e, E, G) == r for e in range(a, b))
        assert seen == list(range(E))
    with pytest.raises(ValueError):
        ep.expert_range(10, 4, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import datetime

    import torch

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        uid = ep.exchange_id(rank, world, make_id=lambda: bytes(np.random.default_rng(5).integers(0, 256, 128,
                                                                                                    dtype=np.uint8)))
        # the same seeded routing and expert outputs on every rank; each keeps
        # only the slots of its own experts and the ranks sum
        rng = np.random.default_rng(1)
        E, k, n, H = 8, 2, 5, 16
        sel = np.stack([rng.permutation(E)[:k] for _ in range(n)]).astype(np.int32)
        w = rng.random((n, k)).astype(np.float32)
        yfull = rng.standard_normal((n * k, H)).astype(np.float32)
        a, b = ep.expert_range(E, world, rank)
        mine = ((sel.reshape(-1) >= a) & (sel.reshape(-1) < b))[:, None]
        part = torch.from_numpy(np.where(mine, yfull, np.float32(0)))
        dist.all_reduce(part)
        _, got = ep.combine_slots([part.numpy()], sel, w, E)
        _, want = ep.combine_slots([yfull], sel, w, E)
        out[rank] = (uid, bool(np.array_equal(part.numpy(), yfull)), bool(np.array_equal(got, want)))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_exchange_and_combine():
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    assert out[0][0] == out[1][0] and len(out[0][0]) == 128
    for r in range(world):
        assert out[r][1] and out[r][2]
