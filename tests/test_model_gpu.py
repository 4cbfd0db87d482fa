"""Model-level parity through the C ABI (host buffers in, host buffers out):
the GPU engine against the reference midged's golden outputs and the CPU
oracle.  Bar: logits within max relative error 1e-3
(the reference's own measure, tools/validate.py:133) and greedy tokens
identical."""
import os

import numpy as np
import pytest

from midge_b200 import abi
from midge_b200 import container as ct
from oracle import oracle as orc
from tests.helpers import GOLDEN, VALIDATE_CASES, load_validate_case, max_rel

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


@pytest.fixture(scope="module")
def c1_dir(tmp_path_factory):
    spec, edt = ct.config_spec("c1_tiny")
    return ct.write_synthetic_model(str(tmp_path_factory.mktemp("c1")), spec, edt, seed=0)


@pytest.mark.parametrize("case", VALIDATE_CASES)
def test_validate_cases(torch_cuda, case, tmp_path):
    """tools/validate.py's seven cases: tfall logits at 12 positions (the
    ctx-64 sliding ring of 8 wraps) and 24 greedy tokens."""
    md, g = load_validate_case(case, str(tmp_path / "m"))
    m = abi.Model.from_dir(md, ctx=int(g["ctx"]))
    lg = m.forward_batch(0, g["ids"], logits_mode=2)
    worst = max(max_rel(g["tfall"][i], lg[i]) for i in range(len(g["ids"])))
    assert worst < LOGIT_TOL, worst
    assert np.allclose(g["tfall"], lg, rtol=2e-3, atol=2e-3)
    toks = []
    cur = int(np.argmax(lg[-1]))
    for _ in range(len(g["gen"])):
        toks.append(cur)
        _, cur = m.forward(0, cur, want_logits=False)
    assert toks == list(g["gen"]), (toks, list(g["gen"]))
    m.close()


def test_c1_tfall_and_greedy_vs_reference(torch_cuda, c1_dir):
    z = np.load(os.path.join(GOLDEN, "c1_tiny.npz"))
    ctx = int(z["ctx"])
    m = abi.Model.from_dir(c1_dir, ctx=ctx)
    lg = m.forward_batch(0, z["prompt"], logits_mode=2)
    worst = max(max_rel(z["tfall"][i], lg[i]) for i in range(len(z["prompt"])))
    assert worst < LOGIT_TOL, worst
    m.close()
    m = abi.Model.from_dir(c1_dir, ctx=ctx)
    last = m.forward_batch(0, z["prompt"], logits_mode=1)
    cur = int(np.argmax(last))
    toks = []
    for _ in range(len(z["gen"])):
        toks.append(cur)
        _, cur = m.forward(0, cur, want_logits=False)
    assert toks == list(z["gen"])
    m.close()


def test_c1_decode_path_vs_oracle(torch_cuda, c1_dir):
    """Per-token forward (the MIDGE_NO_BATCH path) against the oracle at
    every position, plus the usage histogram."""
    m = abi.Model.from_dir(c1_dir, ctx=64)
    om = orc.OracleModel(c1_dir, 64)
    rng = np.random.default_rng(9)
    for t in rng.integers(0, 1024, 40):
        lg, am = m.forward(0, int(t))
        want = om.forward(int(t))
        assert max_rel(want, lg) < LOGIT_TOL
        assert am == int(np.argmax(lg))
    assert np.array_equal(m.usage(), om.usage())
    assert m.expert_loads() == 40 * 2 * 2
    m.close()
    om.close()


def test_concurrent_sequences_match_single(torch_cuda, c1_dir):
    """Decoding 4 sequences in one step gives the same logits, bit for bit,
    as decoding each alone (every token is its own MMA column)."""
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 1024, n) for n in (5, 9, 3, 12)]
    multi = abi.Model.from_dir(c1_dir, ctx=64, max_seqs=4)
    for i, p in enumerate(prompts):
        multi.forward_batch(i, p, logits_mode=0)
    toks = [int(p[-1]) for p in prompts]
    lg_multi, am_multi = multi.decode_step([0, 1, 2, 3], toks, want_logits=True)
    for i, p in enumerate(prompts):
        single = abi.Model.from_dir(c1_dir, ctx=64)
        single.forward_batch(0, p, logits_mode=0)
        lg, am = single.forward(0, toks[i])
        assert np.array_equal(lg.view(np.uint32), lg_multi[i].view(np.uint32))
        assert am == am_multi[i]
        single.close()
    multi.close()


def test_prefill_chunking_and_long_context(torch_cuda, tmp_path, monkeypatch):
    """A prompt longer than the prefill chunk and the sliding window (ring
    wrap inside and across chunks) against the oracle's 64-token chunking."""
    monkeypatch.setenv("MIDGE_PREFILL_CHUNK", "128")
    spec, edt = ct.config_spec("c1_tiny")
    spec["attn"]["sliding_window"] = 40
    md = ct.write_synthetic_model(str(tmp_path / "m"), spec, edt, seed=4)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, 1024, 300)
    m = abi.Model.from_dir(md, ctx=400)
    lg = m.forward_batch(0, prompt, logits_mode=1)
    om = orc.OracleModel(md, 400)
    want = om.prefill(list(prompt))
    assert max_rel(want, lg) < LOGIT_TOL
    for t in rng.integers(0, 1024, 10):
        a, _ = m.forward(0, int(t))
        b = om.forward(int(t))
        assert max_rel(b, a) < LOGIT_TOL
    m.close()
    om.close()


def test_errors_are_status_codes(torch_cuda, c1_dir):
    m = abi.Model.from_dir(c1_dir, ctx=8)
    with pytest.raises(abi.MidgeError) as e:
        m.forward(0, 5000)
    assert e.value.code == abi.MG_ERR_RANGE
    m.forward_batch(0, list(range(8)), logits_mode=0)
    with pytest.raises(abi.MidgeError) as e:
        m.forward(0, 1)
    assert e.value.code == abi.MG_ERR_RANGE and b"context full" in abi.lib.mg_last_error()
    m.reset(0)
    m.forward(0, 1)
    m.close()


@pytest.mark.parametrize("kernels", ["stream", "tile"])
def test_decode_greedy_matches_step_loop(torch_cuda, c1_dir, monkeypatch, kernels):
    """mg_decode_greedy (argmax fed back on the device) gives exactly the
    tokens of the host loop over mg_decode_step, for concurrent sequences."""
    if kernels == "tile":
        monkeypatch.setenv("MIDGE_DECODE_KERNELS", "tile")
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, 1024, 10 + 3 * i) for i in range(5)]
    seqs = np.arange(5, dtype=np.int32)

    def prefilled():
        m = abi.Model.from_dir(c1_dir, ctx=96, max_seqs=5)
        first = [int(np.argmax(m.forward_batch(i, p, logits_mode=1))) for i, p in enumerate(prompts)]
        return m, np.array(first, np.int32)

    a, toks = prefilled()
    want = []
    cur = toks.copy()
    for _ in range(24):
        _, cur = a.decode_step(seqs, cur)
        want.append(np.asarray(cur, np.int32).copy())
    u_loop = a.usage()
    a.close()
    b, toks_b = prefilled()
    assert np.array_equal(toks, toks_b)
    got = b.decode_greedy(seqs, toks_b, 24)
    assert np.array_equal(np.stack(want), got)
    assert np.array_equal(b.usage(), u_loop)
    assert b.kernel_launches() > 0
    # the sequences continue where the greedy run left them
    _, nxt = b.decode_step(seqs, got[-1])
    b.close()
    a, _ = prefilled()
    cur = toks.copy()
    for _ in range(25):
        _, cur = a.decode_step(seqs, cur)
    assert np.array_equal(np.asarray(cur), np.asarray(nxt))
    a.close()


@pytest.mark.parametrize("moe", ["bs", "mma"])
def test_decode_moe_kernels_vs_oracle(torch_cuda, c1_dir, monkeypatch, moe):
    """Both decode expert kernels (block-scaled tcgen05, the default for
    MXFP4; the mma.sync streamed kernels) against the oracle, 8 concurrent
    sequences."""
    if moe == "bs":
        monkeypatch.delenv("MIDGE_MOE_KERNELS", raising=False)
    else:
        monkeypatch.setenv("MIDGE_MOE_KERNELS", moe)
    rng = np.random.default_rng(41)
    prompts = [rng.integers(0, 1024, 6 + i).astype(np.int32) for i in range(8)]
    m = abi.Model.from_dir(c1_dir, ctx=64, max_seqs=8)
    first = np.array([int(np.argmax(m.forward_batch(i, p, logits_mode=1))) for i, p in enumerate(prompts)], np.int32)
    seqs = np.arange(8, dtype=np.int32)
    lg, nxt = m.decode_step(seqs, first, want_logits=True)
    for i, p in enumerate(prompts):
        om = orc.OracleModel(c1_dir, 64)
        om.prefill(list(p))
        want = om.forward(int(first[i]))
        om.close()
        assert max_rel(want, lg[i]) < LOGIT_TOL
    m.close()


def test_decode_trunk_kernels_vs_oracle(torch_cuda, c1_dir):
    """The decode kernels of the int8 trunk (q, k, v, o: the mma.sync
    streamed GEMV), 8 concurrent sequences against the oracle, two steps."""
    rng = np.random.default_rng(47)
    prompts = [rng.integers(0, 1024, 4 + i).astype(np.int32) for i in range(8)]
    m = abi.Model.from_dir(c1_dir, ctx=64, max_seqs=8)
    first = np.array([int(np.argmax(m.forward_batch(i, p, logits_mode=1))) for i, p in enumerate(prompts)], np.int32)
    seqs = np.arange(8, dtype=np.int32)
    _, nxt = m.decode_step(seqs, first)
    lg, _ = m.decode_step(seqs, nxt, want_logits=True)
    for i, p in enumerate(prompts):
        om = orc.OracleModel(c1_dir, 64)
        om.prefill(list(p))
        om.forward(int(first[i]))
        want = om.forward(int(nxt[i]))
        om.close()
        assert max_rel(want, lg[i]) < LOGIT_TOL
    m.close()


def test_decode_block_scaled_token_groups_vs_oracle(torch_cuda, tmp_path, monkeypatch):
    """Block-scaled decode experts when every expert takes all 8 tokens: each
    expert's slots form four token groups of two, each group's tiles spread
    over several CTAs (the groups must be the same in every CTA).  Two decode
    steps of 8 sequences against the oracle."""
    monkeypatch.delenv("MIDGE_MOE_KERNELS", raising=False)
    spec, edt = ct.config_spec("c1_tiny")
    spec["moe"]["experts"] = 4
    spec["moe"]["top_k"] = 4
    md = ct.write_synthetic_model(str(tmp_path / "m"), spec, edt, seed=5)
    rng = np.random.default_rng(43)
    prompts = [rng.integers(0, 1024, 5 + i).astype(np.int32) for i in range(8)]
    m = abi.Model.from_dir(md, ctx=64, max_seqs=8)
    first = np.array([int(np.argmax(m.forward_batch(i, p, logits_mode=1))) for i, p in enumerate(prompts)], np.int32)
    seqs = np.arange(8, dtype=np.int32)
    lg1, nxt = m.decode_step(seqs, first, want_logits=True)
    lg2, _ = m.decode_step(seqs, nxt, want_logits=True)
    for i, p in enumerate(prompts):
        om = orc.OracleModel(md, 64)
        om.prefill(list(p))
        assert max_rel(om.forward(int(first[i])), lg1[i]) < LOGIT_TOL
        assert max_rel(om.forward(int(nxt[i])), lg2[i]) < LOGIT_TOL
        om.close()
    m.close()


@pytest.mark.parametrize("experts,n_seqs", [(322, 8), (128, 5)])
def test_decode_router_widths_vs_oracle(torch_cuda, tmp_path, experts, n_seqs):
    """The decode router away from the default shape: 322 experts (the last
    logits block holds 2 of its 4 expert rows; the top-k scans 11 logits per
    lane) and 5 sequences (a partly filled token group).  Two decode steps
    against the oracle; greedy tokens and usage counters equal."""
    spec, edt = ct.config_spec("c1_tiny")
    spec["moe"]["experts"] = experts
    md = ct.write_synthetic_model(str(tmp_path / "m"), spec, edt, seed=11)
    rng = np.random.default_rng(53)
    prompts = [rng.integers(0, 1024, 4 + i).astype(np.int32) for i in range(n_seqs)]
    m = abi.Model.from_dir(md, ctx=64, max_seqs=n_seqs)
    first = np.array([int(np.argmax(m.forward_batch(i, p, logits_mode=1))) for i, p in enumerate(prompts)], np.int32)
    seqs = np.arange(n_seqs, dtype=np.int32)
    u0 = np.asarray(m.usage()).copy()
    lg1, nxt = m.decode_step(seqs, first, want_logits=True)
    lg2, nxt2 = m.decode_step(seqs, nxt, want_logits=True)
    du = np.asarray(m.usage()) - u0
    want_usage = np.zeros_like(du)
    for i, p in enumerate(prompts):
        om = orc.OracleModel(md, 64)
        om.prefill(list(p))
        ou0 = np.asarray(om.usage()).copy()
        w1 = om.forward(int(first[i]))
        assert max_rel(w1, lg1[i]) < LOGIT_TOL
        assert int(nxt[i]) == int(np.argmax(w1))
        w2 = om.forward(int(nxt[i]))
        assert max_rel(w2, lg2[i]) < LOGIT_TOL
        assert int(nxt2[i]) == int(np.argmax(w2))
        want_usage += np.asarray(om.usage()) - ou0
        om.close()
    assert np.array_equal(du, want_usage)
    m.close()


@pytest.mark.parametrize("split", ["128", "192"])
def test_decode_attention_multi_tile_splits_vs_oracle(torch_cuda, c1_dir, monkeypatch, split):
    """Decode attention with splits of several 64-position tiles
    (MIDGE_ATTN_SPLIT): the tensor-core kernel's double-buffered tile loop
    with the running-maximum rescale, a ragged last tile and a partial last
    split on the full-attention layer (~330-420 positions), and the wrapped
    128-slot ring of the sliding layer in one split.  Two decode steps of 3
    sequences against the oracle."""
    monkeypatch.setenv("MIDGE_ATTN_SPLIT", split)
    rng = np.random.default_rng(59)
    prompts = [rng.integers(0, 1024, n).astype(np.int32) for n in (330, 377, 419)]
    m = abi.Model.from_dir(c1_dir, ctx=512, max_seqs=3)
    first = np.array([int(np.argmax(m.forward_batch(i, p, logits_mode=1))) for i, p in enumerate(prompts)], np.int32)
    seqs = np.arange(3, dtype=np.int32)
    lg1, nxt = m.decode_step(seqs, first, want_logits=True)
    lg2, nxt2 = m.decode_step(seqs, nxt, want_logits=True)
    for i, p in enumerate(prompts):
        om = orc.OracleModel(c1_dir, 512)
        om.prefill(list(p))
        w1 = om.forward(int(first[i]))
        assert max_rel(w1, lg1[i]) < LOGIT_TOL
        assert int(nxt[i]) == int(np.argmax(w1))
        w2 = om.forward(int(nxt[i]))
        assert max_rel(w2, lg2[i]) < LOGIT_TOL
        assert int(nxt2[i]) == int(np.argmax(w2))
        om.close()
    m.close()


def test_ue8m0_container_bit_identical(torch_cuda, c1_dir, tmp_path):
    """An experts.midge rewritten as dtype mxfp4e8 (ue8m0 scales on disk,
    midge_b200.convert_ue8m0) loads without re-expression and gives the same
    logits and greedy tokens, bit for bit, as the original f16-scale file."""
    from midge_b200 import convert_ue8m0 as cv

    e8 = cv.convert(c1_dir, str(tmp_path / "e8"))
    prompt = np.random.default_rng(8).integers(0, 1024, 40)
    out = []
    for md in (c1_dir, e8):
        m = abi.Model.from_dir(md, ctx=96)
        lg = m.forward_batch(0, prompt, logits_mode=2)
        toks = m.decode_greedy(np.zeros(1, np.int32), np.array([int(np.argmax(lg[-1]))], np.int32), 12)
        m.close()
        out.append((lg, toks))
    assert np.array_equal(out[0][0].view(np.uint32), out[1][0].view(np.uint32))
    assert np.array_equal(out[0][1], out[1][1])


def test_bounded_wait_runs_out_and_context_survives(torch_cuda, c1_dir):
    """A device wait that nothing satisfies runs out after its poll budget:
    the kernel records the timeout, drains its own copy, frees its tensor
    memory and exits; the host gets MG_ERR_TIMEOUT (not a hang, not a fault)
    and the next model call on the same context is exact."""
    import ctypes as C

    m = abi.Model.from_dir(c1_dir, ctx=64)
    prompt = np.random.default_rng(2).integers(0, 1024, 12)
    want = m.forward_batch(0, prompt, logits_mode=2)
    m.reset(0)
    for polls in (1, 1000):
        d = C.c_int(0)
        assert abi.lib.mg_wait_selftest(polls, C.byref(d)) == abi.MG_ERR_TIMEOUT
        assert d.value == 43  # the copy issued before the wait landed before the CTA exited
    got = m.forward_batch(0, prompt, logits_mode=2)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    m.close()
