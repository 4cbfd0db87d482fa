"""Expert parallelism on the host side: which experts and sequences a rank
holds, how the ranks of one box agree on the NCCL communicator of the C
library, and a numpy statement of the token-exchange bookkeeping the device
kernels perform (mg_ep_xchg.cu), used by the CPU tests.

Experts shard contiguously: rank r of G holds experts [r*E/G, (r+1)*E/G).
Every rank owns whole sequences (attention, KV cache, router and lm_head of
its own tokens); the trunk weights are replicated.  Per MoE layer each
token's normed row travels once to every rank that holds one of its routed
experts, and each (token, slot) output travels back to the token's owner,
which adds them to the residual in the reference's order.  The collective
model calls (prefill, decode) are made by every rank together.
"""
from __future__ import annotations

import numpy as np


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


def sequence_split(n_seqs: int, world: int, rank: int) -> list[int]:
    """The global sequence ids rank `rank` owns: contiguous blocks, the first
    n_seqs % world ranks taking one more."""
    base, extra = divmod(n_seqs, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


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


# ------------------------------------------------- exchange bookkeeping
def plan(sel: np.ndarray, world: int, per: int, n_experts: int):
    """The owner's side of one layer's exchange (k_ep_pf_plan).

    sel [n x k] global expert ids.  Returns
      counts [2G]: tokens, then slots, this rank sends to each destination;
      send_row [n x G]: row of (token, destination) in the destination-major
        send buffer (tokens in token order), -1 when the token has no expert
        on that destination;
      ret_pos [n x k]: row of each slot's output in the destination-major
        return buffer (per destination: tokens in order, then top-k rank
        order), -1 for an id out of range."""
    sel = np.asarray(sel)
    n, k = sel.shape
    valid = (sel >= 0) & (sel < n_experts)
    dest = np.where(valid, sel // per, -1)
    c = np.stack([(dest == d).sum(1) for d in range(world)], 1) if n else np.zeros((0, world), int)
    tok = c > 0
    tok_cnt, slot_cnt = tok.sum(0).astype(np.int64), c.sum(0).astype(np.int64)
    tok_off = np.concatenate([[0], np.cumsum(tok_cnt)[:-1]])
    slot_off = np.concatenate([[0], np.cumsum(slot_cnt)[:-1]])
    send_row = np.full((n, world), -1, np.int64)
    ret_pos = np.full((n, k), -1, np.int64)
    for d in range(world):
        idx = np.cumsum(tok[:, d]) - 1
        send_row[:, d] = np.where(tok[:, d], tok_off[d] + idx, -1)
        base = np.cumsum(c[:, d]) - c[:, d]  # slots to d of the tokens before
        seen = np.zeros(n, np.int64)
        for i in range(k):
            hit = dest[:, i] == d
            ret_pos[hit, i] = slot_off[d] + base[hit] + seen[hit]
            seen += hit
    return np.concatenate([tok_cnt, slot_cnt]), send_row, ret_pos


def retplan(sel_recv: np.ndarray, e0: int, n_local: int) -> np.ndarray:
    """The expert side (k_ep_pf_retplan): each received slot whose expert is
    local gets the next return row, in received order; -1 otherwise."""
    local = ((sel_recv >= e0) & (sel_recv < e0 + n_local)).reshape(-1)
    return np.where(local, np.cumsum(local) - 1, -1).reshape(np.shape(sel_recv))


def combine(x: np.ndarray, sel: np.ndarray, w: np.ndarray, Y: np.ndarray, slot_row, n_experts: int) -> np.ndarray:
    """x[t] += w * Y[row] per routed expert in ascending expert id (the
    prefill combine, engine/midge.c:595-611); row = slot_row[t, i] or the
    slot-major t*k + i."""
    out = np.array(x, np.float32, copy=True)
    n, k = sel.shape
    for t in range(n):
        order = sorted((int(sel[t, i]), i) for i in range(k) if 0 <= sel[t, i] < n_experts)
        for _, i in order:
            row = int(slot_row[t, i]) if slot_row is not None else t * k + i
            out[t] = out[t] + np.float32(w[t, i]) * Y[row]
    return out
