"""Expert parallelism on the host side: which experts a rank holds and how
the ranks of one box agree on the NCCL communicator of the C library.

Every rank runs the same model calls with the same inputs (tokens,
attention, KV cache, router and trunk are replicated); only the routed
experts are sharded, contiguously: rank r of G holds experts
[r*E/G, (r+1)*E/G).  The library sums each layer's per-slot expert outputs
over the ranks, so every rank ends each layer with identical state.
"""
from __future__ import annotations


def expert_range(n_experts: int, world: int, rank: int) -> tuple[int, int]:
    """[first, end) of the experts rank `rank` holds."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per


def owner(expert: int, n_experts: int, world: int) -> int:
    """The rank holding `expert`."""
    return expert // (n_experts // world)


def exchange_id(rank: int, world: int, group=None, make_id=None) -> bytes:
    """The communicator id, made on rank 0 and broadcast over the existing
    torch.distributed process group (any backend; gloo on CPU).  make_id()
    returns the id bytes; by default the C library's mg_ep_unique_id."""
    import torch.distributed as dist

    if world == 1:
        return b"\0" * 128
    if make_id is None:
        from midge_b200 import abi
        import ctypes as C

        def make_id():
            buf = C.create_string_buffer(abi.EP_ID_BYTES)
            abi.check(abi.lib.mg_ep_unique_id(buf))
            return buf.raw

    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def combine_slots(partials, sel, weights, n_experts: int):
    """Reference for the cross-rank combine (numpy): partials[r] holds rank
    r's per-slot outputs [n_tok*top_k x hidden], zero for slots whose expert
    it does not hold; their sum is the exact per-slot output, which is then
    combined in top-k rank order (engine/midge.c:544-548).  Used by the
    host-side tests of the sharding."""
    import numpy as np

    y = np.zeros_like(partials[0])
    for p in partials:
        y = y + p
    n_tok, k = sel.shape
    out = np.zeros((n_tok, y.shape[1]), np.float32)
    for t in range(n_tok):
        for i in range(k):
            e = int(sel[t, i])
            if 0 <= e < n_experts:
                out[t] = out[t] + np.float32(weights[t, i]) * y[t * k + i]
    return y, out
