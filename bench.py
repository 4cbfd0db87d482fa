"""bench.py -- decode / prefill throughput of the gpt-oss-120b-shaped MoE on B200.

Workload ("C4"): a random-init gpt-oss-120b-shaped
model (36 layers, d_model 2880, 64 q / 8 kv heads of dim 64, sliding-128 /
full layers, YaRN, 128 MXFP4 experts top-4 of width 2880, int8 trunk, vocab
201088) serving 8 concurrent sequences: a prompt per sequence, then greedy
decode steps of all 8 at once.  The trunk is generated on the host with the
config's distributions and uploaded through the C ABI; the 64.7 GB expert
blob is generated in HBM with the same distributions (the file would not fit
the box's disk).  Inputs: seeded synthetic token ids.

One bench "step" = 64 decode steps of the 8 sequences (512 tokens), so
--warmup 3 --steps 5 covers the workload's 512 decode tokens per sequence.
  value  = decode tokens/s of greedy decode with the argmax fed back on the
           device (mg_decode_greedy), device-timed (CUDA events on the
           model's stream)
  e2e    = decode tokens/s through mg_decode_step with host buffers (token ids
           in, argmax ids out, copies inside the timed region), the same
           number of steps continuing the same sequences
  prefill_tok_s = the prompts' prefill through mg_forward_batch (device-timed)
The decode working set (~15 GB of weights per step) is far larger than L2,
so no flush is needed between steps.

--gpus N (torchrun, one rank per GPU): expert parallel -- every rank holds
1/N of the experts and owns 8/N of the sequences (their attention, KV cache,
router and lm_head; trunk weights replicated); each MoE layer sends the
routed tokens to the expert holders and the slot outputs back.  value is the
8 sequences' tokens/s over the max of the ranks' times ("scaling": "strong":
the total work is the same 8 sequences at every N).

--impl reference times the reference engine (oracle/_ref/midged, built from
the reference sources with AVX2 + OpenMP) on the host cores: its per-token
decode on 1- and 3-layer slices of the same shape (fastest of several runs
each), extrapolated to 36 layers.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MEASURED = os.path.join(ROOT, "MEASURED_PEAKS.json")
# DRAM bytes (read + write) per routed expert of one launch of the
# block-scaled decode MoE (gate/up and down in one kernel), from an ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum) of the 45 launches of
# moe_kernel_roofline at 8 tokens, divided by the experts each launch routes
# (its seeded routing replayed on the host): 1.012 x the algorithmic
# 13,253,760 B; per-launch traffic = experts routed x this figure
TRAFFIC_PER_EXPERT = 13418000
DECODE_PER_STEP = 64
N_SEQ = 8


def sustained_tflops():
    try:
        with open(MEASURED) as f:
            return float(json.load(f)["bf16_tflops_sustained"])
    except Exception:
        return 1400.0


def peaks():
    try:
        with open(MEASURED) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, index=0):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                self.samples.append([v.strip() for v in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 3 + i and s[3 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons}


def build_model(torch, spec, edt, ctx, max_seqs, device=0, seed=0, ep=None):
    from midge_b200 import abi
    from midge_b200 import container as ct

    m = abi.Model(spec, ctx=ctx, max_seqs=max_seqs, device=device, ep=ep)
    rng = np.random.default_rng(seed)
    for (n, dt, shape, d, s) in ct.dense_tensors(spec, rng):
        rows = shape[0]
        cols = shape[1] if len(shape) > 1 else 0
        m.set_dense(n, dt, rows, cols, np.frombuffer(d, np.uint8), np.frombuffer(s, np.uint8) if s else None)
    m.synth_experts(edt, seed + 1)
    m.ready()
    return m


def moe_kernel_roofline(torch, m, spec, hbm_peak, reps=40, rank=0, world=1):
    """Time the dominant kernel pair of the decode step live: the streamed
    routed-expert FFN (gate/up + clamped SwiGLU, then down) that the decode
    graph runs, on the resident 120b experts with decode routing of 8 tokens
    (mg_model_moe_stream on the model's stream, CUDA events on that stream).
    Algorithmic bytes per launch: every distinct routed expert's three
    matrices once (nibbles + one ue8m0 scale byte per 32 values + f32 bias),
    plus the activations read and written."""
    from midge_b200 import abi

    H, F, E, k = spec["hidden"], spec["moe"]["ffn"], spec["moe"]["experts"], spec["moe"]["top_k"]
    rng = np.random.default_rng(7)
    layers = spec["n_layers"]
    stream = torch.cuda.ExternalStream(m.stream())
    sels, nbytes, nexp = [], [], []
    per_mat = lambda rows, cols: rows * cols // 2 + rows * cols // 32 + rows * 4
    for _ in range(reps):
        sel = np.stack([rng.permutation(E)[:k] for _ in range(N_SEQ)]).astype(np.int32)
        sels.append(torch.from_numpy(sel).cuda())
        per = E // world  # this rank's experts (expert parallel): only they are read
        d = len([e for e in np.unique(sel) if rank * per <= e < (rank + 1) * per])
        nexp.append(d)
        nbytes.append(d * (2 * per_mat(F, H) + per_mat(H, F)) + N_SEQ * H * 4 + N_SEQ * k * F * 4 * 2
                      + 2 * N_SEQ * k * H * 4)
    torch.cuda.synchronize()

    def launch(i):
        abi.check(abi.lib.mg_model_moe_stream(m.h, i % layers, N_SEQ, sels[i].data_ptr()))

    for i in range(5):
        launch(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps):
        launch(i)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    by = float(np.mean(nbytes))
    ach = by / (ms * 1e-3) / 1e9
    kind = os.environ.get("MIDGE_MOE_KERNELS", "")
    if kind == "mma":
        kname = "k_stream<PolMoeGateUp> + k_stream<PolMoeDown> (mma.sync)"
    else:
        kname = "k_bs_limbs + k_bsmoe gate/up + k_bsmoe down (tcgen05 kind::mxf4 block-scaled)"
    return {"kernel": kname + ", 8 tokens, top-4 of 128 experts", "ms": ms,
            "bytes": by, "experts": float(np.mean(nexp)), "achieved_gbs": ach, "frac": ach / hbm_peak}


def prefill_flops_per_token(spec, prompt_len):
    """Algorithmic FLOPs per prompt token of the prefill (2 per multiply-add):
    routed experts (top_k x 3 matrices of hidden x ffn), q/k/v/o, the router,
    causal attention (QK^T and PV over min(position + 1, window) keys per head,
    averaged over the prompt) and the last position's lm_head spread over the
    prompt."""
    H, F, k = spec["hidden"], spec["moe"]["ffn"], spec["moe"]["top_k"]
    nh, nkv, hd, E = spec["n_heads"], spec["n_kv_heads"], spec["head_dim"], spec["moe"]["experts"]
    win = spec["attn"].get("sliding_window", 0)
    per_layer = 2 * 3 * H * F * k + 2 * (nh * hd * H * 2 + 2 * nkv * hd * H) + 2 * E * H
    flops = 0.0
    for lt in spec["attn"]["layer_types"]:
        if "sliding" in lt and win:
            ctx_avg = float(np.mean(np.minimum(np.arange(1, prompt_len + 1), win)))
        else:
            ctx_avg = (prompt_len + 1) / 2.0
        flops += per_layer + 4.0 * nh * hd * ctx_avg
    flops += 2.0 * spec["vocab"] * H / prompt_len
    return flops


def gemv_microbench(device, hbm_peak, seconds=0.25):
    """BASELINE configs[1] (C2): the MXFP4 dequant-GEMV of the gpt-oss expert
    shapes, gate_up [5760 x 2880] and down [2880 x 2880], at token batches 1,
    4, 16, 64 and 256 (mg_bench_gemv: seeded weights, ue8m0 scales, enough
    copies to exceed L2, CUDA-graph replays timed by events).  GB/s counts the
    bytes the device reads per call once (nibbles + one ue8m0 byte per 32
    values); ref_gib_s counts them as run_bench does (f16 scales, GiB)."""
    import ctypes as C

    from midge_b200 import abi

    out = []
    for name, rows, cols in (("gate_up", 5760, 2880), ("down", 2880, 2880)):
        db = rows * cols // 2
        dev_bytes, file_bytes = db + rows * cols // 32, db + rows * cols // 16
        for t in (1, 4, 16, 64, 256):
            gib = C.c_double(0.0)
            abi.check(abi.lib.mg_bench_gemv(abi.MG_MXFP4, rows, cols, t, seconds, device, C.byref(gib)))
            sec_per_call = file_bytes / (gib.value * 2 ** 30)
            gbs = dev_bytes / sec_per_call / 1e9
            out.append({"matrix": name, "rows": rows, "cols": cols, "tokens": t, "gb_s": round(gbs, 1),
                        "frac": round(gbs / hbm_peak, 4), "us_per_call": round(sec_per_call * 1e6, 2),
                        "tflop_s": round(2.0 * rows * cols * t / sec_per_call / 1e12, 2),
                        "ref_gib_s": round(gib.value, 1)})
    return out


def cpu_reference(spec_name="c4_120b", seconds_budget=20.0, gen=8, reps=5, warmup=1, deep=3):
    """The reference engine on this host: decode seconds per token on 1- and
    `deep`-layer slices of the config (all experts), extrapolated linearly to
    the full depth.  Each slice's per-token time is the fastest of `reps` runs
    of `gen` tokens in one process, after `warmup` untimed runs: the lm_head
    dominates every slice, so the per-layer slope is a small difference of two
    times (one layer is ~2 ms against ~20 ms per token), and single runs of a
    1- and a 2-layer slice moved the estimate by 4x between two back-to-back
    calls on one host; three runs of this form stayed within +-13%.  Returns
    (tok_s, cores, sample description)."""
    from midge_b200 import container as ct
    from oracle import oracle as orc

    if not os.path.exists(orc.REF_MIDGED):
        return None
    cores = os.cpu_count() or 1
    spec_full, edt = ct.config_spec(spec_name)
    times = {}
    tmp = tempfile.mkdtemp(prefix="midge_cpu_")
    try:
        for nl in (1, deep):
            spec, _ = ct.config_spec(spec_name, nl)
            md = ct.write_synthetic_model(os.path.join(tmp, f"l{nl}"), spec, edt, seed=3)
            env = dict(os.environ, OMP_NUM_THREADS=str(cores))
            ctx = max(256, 16 + (warmup + reps) * gen)  # the 8-token prompt and every run's tokens
            p = subprocess.Popen([orc.REF_MIDGED, md, "--ctx", str(ctx), "--temp", "0"], stdin=subprocess.PIPE,
                                 stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, env=env)
            while p.stdout.readline().strip() != "READY":
                pass
            p.stdin.write("ids: 1 2 3 4 5 6 7 8\n")
            p.stdin.flush()
            p.stdout.readline()
            best = None
            for r in range(warmup + reps):
                p.stdin.write(f"gen: {gen}\n")
                p.stdin.flush()
                while True:
                    ln = p.stdout.readline()
                    if ln.startswith("DONE"):
                        t = float(ln.split()[3]) / gen
                        if r >= warmup:
                            best = t if best is None else min(best, t)
                        break
            times[nl] = best
            p.stdin.write("quit\n")
            p.stdin.flush()
            p.wait(timeout=120)
            shutil.rmtree(md, ignore_errors=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    per_layer = max((times[deep] - times[1]) / (deep - 1), 1e-9)
    t_full = times[1] + (spec_full["n_layers"] - 1) * per_layer
    sample = (f"reference midged (AVX2+OpenMP, {cores} threads) greedy decode on 1- and {deep}-layer slices of the "
              f"{spec_name} shape (all experts), fastest of {reps} runs of {gen} tokens each after {warmup} untimed, "
              f"extrapolated to {spec_full['n_layers']} layers; one sequence at a time (the reference is "
              f"single-context)")
    return 1.0 / t_full, cores, sample


def run_ours(args):
    import torch

    from midge_b200 import abi  # fails loudly without the CUDA library
    from midge_b200 import container as ct

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    spec, edt = ct.config_spec(args.config, args.layers)
    prompt_len = args.prompt
    ctx = prompt_len + DECODE_PER_STEP * (args.warmup + 2 * args.steps) + 8  # value run, then the e2e run
    hbm_peak, tc_peak, peak_kind = peaks()
    t0 = time.time()
    ep_arg = None
    if world > 1:  # expert parallel: the same model and inputs on every rank, experts sharded
        from midge_b200 import ep as mep

        ep_arg = (rank, world, mep.exchange_id(rank, world))
    from midge_b200 import ep as mep

    if world > 1:
        os.environ.setdefault("MIDGE_EP_STATS", "1")  # per-phase timing of the expert-parallel prefill
    own = mep.sequence_split(N_SEQ, world, rank)  # this rank's sequences (global ids)
    rounds = -(-N_SEQ // world)
    m = build_model(torch, spec, edt, ctx, max(1, len(own)), device=local, seed=0, ep=ep_arg)
    load_s = time.time() - t0
    stream = torch.cuda.ExternalStream(m.stream())
    rng = np.random.default_rng(100)
    prompts = [rng.integers(0, spec["vocab"], prompt_len).astype(np.int32) for _ in range(N_SEQ)]

    # prefill of the 8 prompts (device-timed on the model stream); expert
    # parallel: every rank prefills one of its own sequences per round
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    t_pf = time.time()
    last = []
    for r in range(rounds):
        if r < len(own):
            last.append(m.forward_batch(r, prompts[own[r]], logits_mode=1))
        else:
            m.forward_batch(0, np.zeros(0, np.int32), logits_mode=0)
    e1.record(stream)
    e1.synchronize()
    pf_wall = time.time() - t_pf
    pf_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([pf_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pf_ms = float(t[0])
    prefill_tok_s = N_SEQ * prompt_len / (pf_ms / 1e3)
    ep_phases = None
    if world > 1:
        import ctypes as C

        ph = (C.c_double * 4)()
        abi.check(abi.lib.mg_model_ep_stats(m.h, ph))
        ep_phases = {"plan_agree_ms": round(ph[0], 2), "dispatch_ms": round(ph[1], 2),
                     "experts_ms": round(ph[2], 2), "return_combine_ms": round(ph[3], 2)}
    toks = np.array([int(np.argmax(l)) for l in last], np.int32)
    seqs = np.arange(len(own), dtype=np.int32)

    # value: greedy decode fed back on the device (mg_decode_greedy), inputs
    # resident, no host round trip inside the timed region
    cur = m.decode_greedy(seqs, toks, args.warmup * DECODE_PER_STEP)[-1]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    k0 = m.kernel_launches()
    with ClockSampler(local) as clk:
        e0.record(stream)
        out = m.decode_greedy(seqs, cur, args.steps * DECODE_PER_STEP)
        e1.record(stream)
        e1.synchronize()
    launches = m.kernel_launches() - k0
    dev_ms = e0.elapsed_time(e1)
    cur = out[-1]
    # e2e: the same decode through mg_decode_step with host buffers: token
    # ids copied in and argmax ids read back every step
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    tw = time.time()
    for _ in range(args.steps * DECODE_PER_STEP):
        _, cur = m.decode_step(seqs, cur)
    wall = time.time() - tw
    if dist:
        t = torch.tensor([dev_ms, wall * 1e3], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, wall = float(t[0]), float(t[1]) / 1e3
    ntok = N_SEQ * DECODE_PER_STEP * args.steps  # the 8 sequences, over all ranks
    value = ntok / (dev_ms / 1e3)
    e2e = ntok / wall
    roof = moe_kernel_roofline(torch, m, spec, hbm_peak, rank=rank, world=world)
    cpu = cpu_reference(args.config) if (rank == 0 and world == 1 and not args.no_cpu) else None
    m.close()
    gemv = gemv_microbench(local, hbm_peak) if (rank == 0 and not args.no_gemv) else None
    tc_sustained = sustained_tflops()
    pf_flops = prefill_flops_per_token(spec, prompt_len) * N_SEQ * prompt_len
    pf_tflops = pf_flops / (pf_ms * 1e-3) / 1e12
    tc_job = tc_sustained * world  # whole-job tensor peak: every rank's
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    line = {
        "metric": "decode tok/s (gpt-oss-120b shape, 8 concurrent sequences, greedy)",
        "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "mxfp4/int8 weights, fp32 accumulate",
        "data": "synthetic (seeded random-init weights and token ids)",
        "config": {"workload": f"{args.config}{'' if args.layers is None else f' ({args.layers} layers)'}: 8 sequences x {prompt_len}-token prompt, "
                               f"{DECODE_PER_STEP} decode steps per bench step",
                   "parallelism": (f"expert-parallel ep{world}: experts and sequences sharded, trunk weights "
                                   f"replicated, token dispatch/combine over NVLink peer memory per MoE layer (NCCL for "
                                   f"control only)") if world > 1 else "single GPU",
                   "l2": "working set (~15 GB/step) >> L2, no flush"},
        "prefill_tok_s": round(prefill_tok_s, 1), "prefill_wall_s": round(pf_wall, 3),
        "prefill": {"tok_s": round(prefill_tok_s, 1), "ms": round(pf_ms, 2),
                    "roofline": {"bound": "tensor", "achieved": round(pf_tflops, 1), "peak": round(tc_job, 1),
                                 "unit": "TFLOP/s", "frac": round(pf_tflops / tc_job, 4),
                                 "flops_per_token": round(pf_flops / (N_SEQ * prompt_len), 0),
                                 "peak_kind": peak_kind + " (bf16_tflops_sustained, cuBLAS, x n_gpus)",
                                 "note": "useful FLOPs (experts, q/k/v/o, router, causal attention, lm_head of "
                                         "the last position); the kernels run fp32-exact products as f16 hi/lo "
                                         "pairs, two tensor-core MMAs per useful one"}},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s",
                # token id, position and sequence id in; argmax key out (+ the
                # error word, and expert parallel the 3-int step agreement per rank)
                "h2d_bytes_per_step": (N_SEQ * 12 + (world * 12 if world > 1 else 0)) * DECODE_PER_STEP,
                "d2h_bytes_per_step": (N_SEQ * 8 + world * 4 + (world * 12 if world > 1 else 0)) * DECODE_PER_STEP},
        "roofline": {"bound": "hbm", "achieved": round(roof["achieved_gbs"], 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(roof["frac"], 4),
                     "traffic": round(roof["experts"] * TRAFFIC_PER_EXPERT, 0) if TRAFFIC_PER_EXPERT else None,
                     "kernel": roof["kernel"], "bytes_per_launch": round(roof["bytes"], 0),
                     "ms_per_launch": round(roof["ms"], 4), "peak_kind": peak_kind + " (hbm_gbs burst copy)"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "load_s": round(load_s, 1),
    }
    if ep_phases:
        line["prefill"]["ep_moe_phases_rank0"] = ep_phases
    if gemv:
        line["gemv"] = {"config": "C2: MXFP4 gate_up [5760x2880] and down [2880x2880], fp32 activations",
                        "peak_gb_s": hbm_peak, "kernel": "k_gemv (mg_gemv: 16 tokens per weight pass)",
                        "results": gemv}
    if cpu:
        line["cpu_baseline"] = {"value": round(cpu[0], 4), "unit": "tok/s", "cores": cpu[1], "kind": "reference",
                                "sample": cpu[2]}
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # K timed runs (at least 5: the fastest is kept) after W untimed ones, per slice
    r = cpu_reference(args.config, reps=max(5, args.steps), warmup=args.warmup)
    if r is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/midged was not built (reference tree absent "
                                                               "when the repository was built)"}))
        return
    tok_s, cores, sample = r
    print(json.dumps({
        "impl": "reference", "metric": "decode tok/s (gpt-oss-120b shape, 8 concurrent sequences, greedy)",
        "value": round(tok_s, 4), "unit": "tok/s", "n_gpus": 0, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "config": {"workload": f"{args.config} (reference CPU engine)"},
        "cpu_baseline": {"value": round(tok_s, 4), "unit": "tok/s", "cores": cores, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(tok_s, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main():
    global DECODE_PER_STEP
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c4_120b")
    ap.add_argument("--prompt", type=int, default=4096)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-gemv", action="store_true", help="skip the C2 GEMV microbench block")
    ap.add_argument("--layers", type=int, default=None,
                    help="depth-reduced slice of the config (profiling captures); default: the full depth")
    ap.add_argument("--decode-per-step", type=int, default=DECODE_PER_STEP,
                    help="decode steps per bench step (64: the workload's 512 tokens over --steps 5 --warmup 3)")
    args = ap.parse_args()
    DECODE_PER_STEP = max(1, args.decode_per_step)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
