"""Expert parallelism on 2 GPUs through the C ABI: each rank holds half of
the experts and owns its own sequences (rank 0: sequences 0 and 1, rank 1:
sequence 2); every MoE layer sends the routed tokens to the expert holders and
the slot outputs back (mg_ep_xchg.cu).  Prefill logits (every position),
device-fed greedy decode, per-step decode, a step in which rank 0 has no
sequence of its own (it only serves its experts) and the usage counters summed
over the ranks must be bit-identical to one GPU holding every expert and
every sequence.  Skipped with fewer than 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

OWN = {0: [0, 1], 1: [2]}  # global sequence ids per rank


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model(case, ctx, max_seqs, device, ep_arg=None):
    from midge_b200 import abi
    from midge_b200 import container as ct

    if case == "c1":
        spec, edt = ct.config_spec("c1_tiny")
        seed = 31
    else:  # the gpt-oss-20b layer shape (32 MXFP4 experts of width 2880), 2 layers
        spec, edt = ct.config_spec("c3_20b", 2)
        seed = 37
    rng = np.random.default_rng(seed)
    dense = list(ct.dense_tensors(spec, rng))
    lay = ct.ExpertLayout(edt, spec["hidden"], spec["moe"]["ffn"], spec["moe"]["experts"], spec["n_layers"])
    blob = ct.expert_blob(lay, rng)
    return abi.Model.from_arrays(spec, dense, edt, blob, ctx=ctx, max_seqs=max_seqs, device=device, ep=ep_arg), spec


def _prompts(case, vocab):
    rng = np.random.default_rng(32)
    lens = (40, 17, 70) if case == "c1" else (300, 25, 140)
    return [rng.integers(0, vocab, n).astype(np.int32) for n in lens]


def _run(m, prompts, seqs_local, n_gen, subset_local):
    """The same call sequence on one GPU (seqs_local = every sequence) and on
    each rank (its own sequences; every rank makes every call)."""
    lg = {}
    rounds = max(len(v) for v in OWN.values())
    for r in range(rounds):  # prefill: one sequence per rank per round (n = 0 when a rank has none left)
        if r < len(seqs_local):
            g = seqs_local[r]
            lg[g] = m.forward_batch(r, prompts[g], logits_mode=2).copy()
        else:
            m.forward_batch(0, np.zeros(0, np.int32), logits_mode=0)
    first = np.array([int(np.argmax(lg[g][-1])) for g in seqs_local], np.int32)
    local_ids = np.arange(len(seqs_local), dtype=np.int32)
    toks = m.decode_greedy(local_ids, first, n_gen)  # collective: every rank calls, with 0 sequences too
    cur = toks[-1]
    steps = []
    for _ in range(3):
        _, cur = m.decode_step(local_ids, cur)
        steps.append(np.asarray(cur).copy())
    sub_ids = np.array([seqs_local.index(g) for g in subset_local], np.int32)
    sub_tok = np.array([steps[-1][i] for i in sub_ids], np.int32)
    sub_lg, _ = m.decode_step(sub_ids, sub_tok, want_logits=True)
    return lg, toks, np.stack(steps, 1), sub_lg, m.usage()


def _worker(rank, world, port, case, ctx, n_gen, outdir):
    import torch
    import torch.distributed as dist

    from midge_b200 import ep

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
    try:
        uid = ep.exchange_id(rank, world)
        m, spec = _model(case, ctx, max_seqs=len(OWN[rank]), device=rank, ep_arg=(rank, world, uid))
        prompts = _prompts(case, spec["vocab"])
        own = OWN[rank]
        lg, toks, steps, sub_lg, usage = _run(m, prompts, own, n_gen, [g for g in own if g == 2])
        m.close()
        np.savez(os.path.join(outdir, f"r{rank}.npz"), toks=toks, steps=steps, usage=usage,
                 sub_lg=sub_lg if sub_lg is not None else np.zeros(0, np.float32),
                 **{f"lg{g}": lg[g] for g in own})
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["c1", "c3_width"])
def test_two_gpu_expert_parallel_bit_identical(torch_cuda, tmp_path, case):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx, n_gen = (128, 12) if case == "c1" else (400, 6)
    m, spec = _model(case, ctx, max_seqs=3, device=0)
    prompts = _prompts(case, spec["vocab"])
    lg1 = {g: m.forward_batch(g, prompts[g], logits_mode=2).copy() for g in range(3)}
    first = np.array([int(np.argmax(lg1[g][-1])) for g in range(3)], np.int32)
    toks1 = m.decode_greedy(np.arange(3, dtype=np.int32), first, n_gen)
    cur = toks1[-1]
    steps1 = []
    for _ in range(3):
        _, cur = m.decode_step(np.arange(3, dtype=np.int32), cur)
        steps1.append(np.asarray(cur).copy())
    steps1 = np.stack(steps1, 1)
    sub_lg1, _ = m.decode_step(np.array([2], np.int32), np.array([steps1[2, -1]], np.int32), want_logits=True)
    usage1 = m.usage()
    m.close()
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), case, ctx, n_gen, str(tmp_path)), nprocs=world, join=True)
    usage = 0
    for r in range(world):
        z = np.load(os.path.join(tmp_path, f"r{r}.npz"))
        own = OWN[r]
        for i, g in enumerate(own):
            assert np.array_equal(z[f"lg{g}"].view(np.uint32), lg1[g].view(np.uint32)), (r, g)
            assert np.array_equal(z["toks"][:, i], toks1[:, g]), (r, g)
            assert np.array_equal(z["steps"][i], steps1[g]), (r, g)
        usage = usage + z["usage"]
        if r == 1:  # the step in which only sequence 2 decodes (rank 0 served its experts only)
            assert np.array_equal(z["sub_lg"].view(np.uint32), sub_lg1.view(np.uint32))
    assert np.array_equal(usage, usage1)
