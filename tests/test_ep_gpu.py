"""Expert parallelism on 2 GPUs through the C ABI: each rank holds half of
the experts, tokens and trunk are replicated, and each layer's per-slot
expert outputs are summed over the ranks with NCCL.  Prefill logits (every
position), greedy decode tokens of concurrent sequences and usage counters
must be bit-identical to one GPU holding every expert.  Skipped with fewer
than 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(md, ctx, prompts, n_gen, ep_arg=None, device=0):
    from midge_b200 import abi

    m = abi.Model.from_dir(md, ctx=ctx, max_seqs=len(prompts), device=device, ep=ep_arg)
    try:
        lg = [m.forward_batch(i, p, logits_mode=2) for i, p in enumerate(prompts)]
        first = np.array([int(np.argmax(l[-1])) for l in lg], np.int32)
        toks = m.decode_greedy(np.arange(len(prompts), dtype=np.int32), first, n_gen)
        steps = []
        cur = toks[-1]
        for _ in range(3):  # the per-step API continues the same sequences
            _, cur = m.decode_step(np.arange(len(prompts), dtype=np.int32), cur)
            steps.append(np.asarray(cur).copy())
        return [l.copy() for l in lg], toks, np.stack(steps), m.usage()
    finally:
        m.close()


def _worker(rank, world, port, md, ctx, prompts, n_gen, outdir):
    import torch
    import torch.distributed as dist

    from midge_b200 import ep

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        uid = ep.exchange_id(rank, world)
        lg, toks, steps, usage = _run(md, ctx, prompts, n_gen, ep_arg=(rank, world, uid), device=rank)
        np.savez(os.path.join(outdir, f"r{rank}.npz"), toks=toks, steps=steps, usage=usage,
                 **{f"lg{i}": l for i, l in enumerate(lg)})
    finally:
        dist.destroy_process_group()


def test_two_gpu_expert_parallel_bit_identical(torch_cuda, tmp_path):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from midge_b200 import container as ct

    spec, edt = ct.config_spec("c1_tiny")
    md = ct.write_synthetic_model(str(tmp_path / "m"), spec, edt, seed=31)
    rng = np.random.default_rng(32)
    prompts = [rng.integers(0, 1024, n).astype(np.int32) for n in (40, 17, 70)]
    ctx, n_gen = 128, 12
    lg1, toks1, steps1, usage1 = _run(md, ctx, prompts, n_gen)
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), md, ctx, prompts, n_gen, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        z = np.load(os.path.join(tmp_path, f"r{r}.npz"))
        for i in range(len(prompts)):
            assert np.array_equal(z[f"lg{i}"].view(np.uint32), lg1[i].view(np.uint32)), (r, i)
        assert np.array_equal(z["toks"], toks1)
        assert np.array_equal(z["steps"], steps1)
        assert np.array_equal(z["usage"], usage1)
