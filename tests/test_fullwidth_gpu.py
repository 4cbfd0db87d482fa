"""Model-level parity at the widths the bench runs: depth-reduced (2-layer)
slices of the BASELINE configs at full width, on the default kernels, against
the CPU oracle on the same in-memory weights.

  C4 slice  gpt-oss-120b layer shape: d2880, 64 q / 8 kv heads of dim 64,
            sliding-128 + full layers, 128 MXFP4 experts top-4 of width 2880,
            int8 trunk, vocab 201088
  C3 slice  the same with 32 experts (gpt-oss-20b), 1024-token prompt: experts
            take more than one 128-slot prefill tile
  C5 slice  Qwen3-MoE: d2048, 32 q / 4 kv heads of dim 128, QK-norm, 128 int8
            experts top-8 of width 768, plain SwiGLU, router_norm 0, vocab 151936

At hidden 2880 the block-scaled decode kernels run 12 K stages per unit
(11 full 256-value stages + one 64-value stage whose 1440-byte row ends are
zero-filled by the TMA bounds), their 9-stage ring wraps inside every unit,
the down pass is K-split over several 128-row tiles, the lm_head argmax
reduces 201,088 rows, and the 8:1 GQA decode attention walks a sliding ring
that has wrapped (prompt > 128).

Each slice: 8 sequences prefilled (one prompt >= 512 tokens), last-position
logits against the oracle's 64-token-chunk prefill; decode steps of the 8
sequences and of subsets (1 and 3 sequences) against the oracle's per-token
forward; then device-fed greedy decode (mg_decode_greedy) against the
oracle's greedy tokens; usage counters equal.
Bar: logits within max relative error 1e-3 of the
oracle (bit-exact with the reference engine), greedy tokens identical.
"""
import numpy as np
import pytest

from midge_b200 import abi
from midge_b200 import container as ct
from oracle import oracle as orc
from tests.helpers import max_rel

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


def _slice(config, n_layers, seed, experts=None):
    spec, edt = ct.config_spec(config, n_layers)
    if experts is not None:
        spec["moe"]["experts"] = experts
    rng = np.random.default_rng(seed)
    dense = list(ct.dense_tensors(spec, rng))
    lay = ct.ExpertLayout(edt, spec["hidden"], spec["moe"]["ffn"], spec["moe"]["experts"], n_layers)
    blob = ct.expert_blob(lay, rng)
    return spec, edt, dense, blob, rng


def _check_slice(config, n_layers, seed, prompt_lens, plan, greedy_steps, experts=None):
    spec, edt, dense, blob, rng = _slice(config, n_layers, seed, experts)
    V = spec["vocab"]
    n = len(prompt_lens)
    prompts = [rng.integers(0, V, k).astype(np.int32) for k in prompt_lens]
    ctx = max(prompt_lens) + len(plan) + greedy_steps + 8
    m = abi.Model.from_arrays(spec, dense, edt, blob, ctx=ctx, max_seqs=n)
    oms = [orc.OracleModel.from_arrays(spec, dense, edt, blob, ctx) for _ in range(n)]
    try:
        cur = np.zeros(n, np.int32)
        for s, p in enumerate(prompts):
            lg = m.forward_batch(s, p, logits_mode=1)
            want = oms[s].prefill(list(p))
            assert max_rel(want, lg) < LOGIT_TOL, (config, "prefill", s, max_rel(want, lg))
            assert int(np.argmax(lg)) == int(np.argmax(want)), (config, "prefill argmax", s)
            cur[s] = int(np.argmax(want))
        for step, subset in enumerate(plan):
            subset = np.asarray(subset, np.int32)
            lg, am = m.decode_step(subset, cur[subset], want_logits=True)
            for i, s in enumerate(subset):
                want = oms[s].forward(int(cur[s]))
                assert max_rel(want, lg[i]) < LOGIT_TOL, (config, "decode", step, int(s), max_rel(want, lg[i]))
                assert int(am[i]) == int(np.argmax(want)), (config, "decode argmax", step, int(s))
                cur[s] = int(am[i])
        seqs = np.arange(n, dtype=np.int32)
        got = m.decode_greedy(seqs, cur, greedy_steps)
        for s in range(n):
            tok = int(cur[s])
            for k in range(greedy_steps):
                tok = int(np.argmax(oms[s].forward(tok)))
                assert int(got[k, s]) == tok, (config, "greedy", s, k)
        assert np.array_equal(m.usage(), sum(om.usage() for om in oms))
    finally:
        m.close()
        for om in oms:
            om.close()


ALL8 = list(range(8))


def test_c4_slice_default_kernels_vs_oracle(torch_cuda):
    """120b layer shape: one 520-token prompt (sliding ring wrapped four
    times), seven short ones; decode of 8, 3 and 1 sequences."""
    _check_slice("c4_120b", 2, seed=101, prompt_lens=[520, 3, 7, 12, 20, 31, 45, 64],
                 plan=[ALL8, [0, 4, 7], [1], ALL8], greedy_steps=3)


def test_c3_slice_default_kernels_vs_oracle(torch_cuda):
    """20b layer shape (32 experts): a 1024-token prompt gives ~128 slots
    per expert in prefill (several experts take two 128-slot tiles); eight
    decoding sequences put 32 slots on 32 experts, so experts take token
    groups of two."""
    _check_slice("c3_20b", 2, seed=202, prompt_lens=[1024, 5, 9, 16, 2, 40, 23, 11],
                 plan=[ALL8, [2, 3, 5], ALL8], greedy_steps=3)


def test_c5_slice_default_kernels_vs_oracle(torch_cuda):
    """Qwen3-MoE layer shape: int8 experts (streamed mma.sync decode MoE),
    head_dim 128, QK-norm, top-8 with full-softmax weights."""
    _check_slice("c5_qwen3", 2, seed=303, prompt_lens=[600, 4, 10, 18, 27, 6, 50, 33],
                 plan=[ALL8, [6], [0, 1, 2], ALL8], greedy_steps=3)
