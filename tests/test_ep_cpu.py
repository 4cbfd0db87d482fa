"""Expert parallelism, host side, on CPU: the expert and sequence shards,
the communicator-id exchange, the token-exchange bookkeeping of
mg_ep_xchg.cu (stated in numpy by midge_b200.ep) run across gloo ranks with
all-to-all transfers and checked bit for bit against one process holding
every expert, and the watchdog that aborts a communicator whose peers do not
answer (its loop run against fakes)."""
import ctypes as C
import datetime
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from midge_b200 import abi
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


def test_sequence_split():
    for n, G in [(8, 1), (8, 2), (8, 8), (3, 2), (5, 4), (2, 4)]:
        parts = [ep.sequence_split(n, G, r) for r in range(G)]
        assert sum(parts, []) == list(range(n))
        assert max(map(len, parts)) - min(map(len, parts)) <= 1


def test_plan_numbering_by_hand():
    # 4 experts over 2 ranks (per 2); 3 tokens, top-2
    sel = np.array([[0, 3], [1, 0], [2, 3]])
    counts, send_row, ret_pos = ep.plan(sel, world=2, per=2, n_experts=4)
    # tokens to rank 0: t0, t1; to rank 1: t0, t2.  Slots to rank 0: (0,0) (1,0) (1,1); to rank 1: (0,1) (2,0) (2,1)
    assert list(counts) == [2, 2, 3, 3]
    assert send_row.tolist() == [[0, 2], [1, -1], [-1, 3]]
    assert ret_pos.tolist() == [[0, 3], [1, 2], [4, 5]]
    # the expert side numbers the received local slots in received order
    assert ep.retplan(np.array([[0, 3], [1, 0]]), 0, 2).tolist() == [[0, -1], [1, 2]]
    assert ep.retplan(np.array([[0, 3], [2, 3]]), 2, 2).tolist() == [[-1, 0], [1, 2]]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _expert_out(e, rows):
    """A stand-in expert: any function of (expert, row) exercises the routing."""
    return (rows * np.float32(1.0 + e / 16.0) + np.float32(e)).astype(np.float32)


def _case(world, seed=3):
    rng = np.random.default_rng(seed)
    E, k, H = 8 * world, 3, 12
    ns = [0] + [int(v) for v in rng.integers(3, 9, world - 1)]  # rank 0 has no tokens but still serves its experts
    data = []
    for r in range(world):
        sel = np.stack([rng.permutation(E)[:k] for _ in range(ns[r])]).astype(np.int32) if ns[r] else \
            np.zeros((0, k), np.int32)
        if ns[r]:
            sel[0, 1] = -1  # an id out of range takes no part
        data.append((sel, rng.standard_normal((ns[r], H)).astype(np.float32),
                     rng.random((ns[r], k)).astype(np.float32), rng.standard_normal((ns[r], H)).astype(np.float32)))
    return E, k, H, data


def _single_process(E, k, H, sel, xb, w, x):
    Y = np.zeros((len(sel) * k, H), np.float32)
    for t in range(len(sel)):
        for i in range(k):
            if 0 <= sel[t, i] < E:
                Y[t * k + i] = _expert_out(int(sel[t, i]), xb[t])
    return ep.combine(x, sel, w, Y, None, E)


def _a2a(torch, send, send_counts, recv_counts, width):
    out = torch.empty((int(sum(recv_counts)), width), dtype=torch.float32)
    dist.all_to_all_single(out, torch.from_numpy(np.ascontiguousarray(send, np.float32)).reshape(-1, width),
                           [int(c) for c in recv_counts], [int(c) for c in send_counts])
    return out.numpy()


def _worker(rank, world, port, out):
    import torch

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        uid = ep.exchange_id(rank, world, make_id=lambda: bytes(np.random.default_rng(5).integers(0, 256, 128,
                                                                                                    dtype=np.uint8)))
        E, k, H, data = _case(world)
        sel, xb, w, x = data[rank]
        per = E // world
        e0 = rank * per
        counts, send_row, ret_pos = ep.plan(sel, world, per, E)
        allc = [torch.zeros(2 * world, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(allc, torch.from_numpy(counts.astype(np.int64)))
        A = np.stack([a.numpy() for a in allc])  # A[r, d] tokens r -> d; A[r, G + d] slots r -> d
        rowf = H + k
        send = np.zeros((int(counts[:world].sum()), rowf), np.float32)
        for t in range(len(sel)):
            for d in range(world):
                if send_row[t, d] >= 0:
                    send[send_row[t, d], :H] = xb[t]
                    send[send_row[t, d], H:] = sel[t]
        recv = _a2a(torch, send, A[rank, :world], A[:, rank], rowf)
        sel_recv = recv[:, H:].astype(np.int32)
        ret_row = ep.retplan(sel_recv, e0, per)
        ret_send = np.zeros((int(A[:, world + rank].sum()), H), np.float32)
        for j in range(len(recv)):
            for i in range(k):
                if ret_row[j, i] >= 0:
                    ret_send[ret_row[j, i]] = _expert_out(int(sel_recv[j, i]), recv[j, :H])
        ret_recv = _a2a(torch, ret_send, A[:, world + rank], A[rank, world:], H)
        got = ep.combine(x, sel, w, ret_recv, ret_pos, E)
        want = _single_process(E, k, H, sel, xb, w, x)
        out[rank] = (uid, len(sel), bool(np.array_equal(got.view(np.uint32), want.view(np.uint32))), int(len(recv)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_dispatch_and_combine_match_one_process(world):
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    assert len({out[r][0] for r in range(world)}) == 1 and len(out[0][0]) == 128
    assert out[0][1] == 0  # rank 0 had no tokens of its own ...
    assert out[0][3] > 0   # ... and still served its experts
    for r in range(world):
        assert out[r][2], r


@pytest.mark.parametrize("scenario,rc,aborts", [(0, abi.MG_OK, 0), (1, abi.MG_ERR_COMM, 1), (2, abi.MG_ERR_COMM, 1),
                                                (3, abi.MG_ERR_CUDA, 1)])
def test_watchdog_aborts_on_timeout_and_errors(scenario, rc, aborts):
    """The loop that watches every blocking wait of an expert-parallel model:
    a wait that completes returns OK; one that never completes is ended by
    the timeout, and an asynchronous communicator error or a device error
    ends it at once -- each of those aborts the communicator exactly once."""
    n = C.c_int(-1)
    got = abi.lib.mg_ep_watchdog_selftest(scenario, 0.2, C.byref(n))
    assert got == rc
    assert n.value == aborts
    if scenario == 1:
        assert b"exceeded" in abi.lib.mg_last_error()
