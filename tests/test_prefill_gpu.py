"""Tensor-core prefill of the routed experts (expert-major grouped tcgen05
GEMM, engine/midge.c:576-622) against the CPU oracle and against the tile
kernels (MIDGE_PREFILL_KERNELS=tile).  Shapes are chosen so that experts
get more than one 128-token tile and the weight matrices more than one
128-row tile.  Bar: logits within max relative error 1e-3, usage identical."""
import numpy as np
import pytest

from midge_b200 import abi
from midge_b200 import container as ct
from oracle import oracle as orc
from tests.helpers import max_rel

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


def _spec(kind):
    if kind == "gpt-oss":
        return ct.gpt_oss_spec(hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, vocab=1024, experts=8,
                               top_k=2, ffn=512)
    return ct.qwen3_spec(hidden=320, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, vocab=1024, experts=6,
                         top_k=3, ffn=192)


@pytest.mark.parametrize("kind,edt", [("gpt-oss", "mxfp4"), ("qwen3", "q8r")])
def test_tc_prefill_vs_oracle_and_tile(torch_cuda, tmp_path, monkeypatch, kind, edt):
    md = ct.write_synthetic_model(str(tmp_path / "m"), _spec(kind), edt, seed=11)
    rng = np.random.default_rng(12)
    prompt = rng.integers(0, 1024, 700)
    ctx = 800
    m = abi.Model.from_dir(md, ctx=ctx)
    lg = m.forward_batch(0, prompt, logits_mode=2)
    om = orc.OracleModel(md, ctx)
    want = om.prefill(list(prompt), tfall=True)
    worst = max(max_rel(want[i], lg[i]) for i in range(0, len(prompt), 7))
    assert worst < LOGIT_TOL, worst
    assert np.array_equal(m.usage(), om.usage())
    # decode continues from the prefilled cache
    for t in rng.integers(0, 1024, 4):
        a, _ = m.forward(0, int(t))
        b = om.forward(int(t))
        assert max_rel(b, a) < LOGIT_TOL
    m.close()
    om.close()
    monkeypatch.setenv("MIDGE_PREFILL_KERNELS", "tile")
    mt = abi.Model.from_dir(md, ctx=ctx)
    lt = mt.forward_batch(0, prompt, logits_mode=2)
    mt.close()
    assert max(max_rel(lt[i], lg[i]) for i in range(0, len(prompt), 7)) < LOGIT_TOL


def test_tc_prefill_chunks(torch_cuda, tmp_path, monkeypatch):
    """Chunks of 64 tokens (the reference's prefill batch) give the same
    logits as one chunk."""
    spec = _spec("gpt-oss")
    md = ct.write_synthetic_model(str(tmp_path / "m"), spec, "mxfp4", seed=13)
    prompt = np.random.default_rng(14).integers(0, 1024, 200)
    m = abi.Model.from_dir(md, ctx=256)
    one = m.forward_batch(0, prompt, logits_mode=2)
    m.close()
    monkeypatch.setenv("MIDGE_PREFILL_CHUNK", "64")
    m = abi.Model.from_dir(md, ctx=256)
    chunked = m.forward_batch(0, prompt, logits_mode=2)
    m.close()
    assert np.array_equal(one.view(np.uint32), chunked.view(np.uint32))


@pytest.mark.parametrize("window", [0, 40])
def test_tc_attention_matches_scalar(torch_cuda, tmp_path, monkeypatch, window):
    """Prefill attention on the tensor cores (Q and P split into f16 hi/lo)
    against the fp32 kernel and the oracle: long prompt over several chunks,
    full and sliding-window layers."""
    spec, edt = ct.config_spec("c1_tiny")
    spec["attn"]["sliding_window"] = window
    if window:
        spec["attn"]["layer_types"] = ["sliding_attention", "full_attention"]
    md = ct.write_synthetic_model(str(tmp_path / "m"), spec, edt, seed=17)
    prompt = np.random.default_rng(18).integers(0, 1024, 333)
    monkeypatch.setenv("MIDGE_PREFILL_CHUNK", "128")
    nxt = np.random.default_rng(19).integers(0, 1024, 6)

    def run():
        m = abi.Model.from_dir(md, ctx=400)
        lg = m.forward_batch(0, prompt, logits_mode=2)
        dec = [m.forward(0, int(t))[0] for t in nxt]  # decode attention over the long context
        m.close()
        return lg, dec

    tc, tc_dec = run()
    monkeypatch.setenv("MIDGE_ATTN_KERNELS", "scalar")
    sc, sc_dec = run()
    assert max(max_rel(sc[i], tc[i]) for i in range(0, len(prompt), 5)) < 1e-4
    assert max(max_rel(a, b) for a, b in zip(sc_dec, tc_dec)) < 1e-4
    om = orc.OracleModel(md, 400)
    want = om.prefill(list(prompt))
    om.close()
    assert max_rel(want, tc[-1]) < LOGIT_TOL
