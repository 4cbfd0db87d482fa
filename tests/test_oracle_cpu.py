"""The CPU oracle (oracle/oracle.c) pinned against the reference: bit-exact
against the reference engine compiled from its own sources (oracle/_ref)
where that build exists, and against the reference midged's golden outputs
stored in tests/golden/ everywhere."""
import os
import tempfile

import numpy as np
import pytest

from oracle import oracle as orc
from midge_b200 import container as ct
from tests.helpers import VALIDATE_CASES, load_validate_case, max_rel

needs_ref = pytest.mark.skipif(not orc.ref_available(), reason="oracle/_ref not built (reference tree absent)")


@pytest.mark.parametrize("dt", [0, 1, 2, 3])
@pytest.mark.parametrize("shape", [(37, 64), (64, 2880), (16, 100)])
@needs_ref
def test_matvec_bit_exact_vs_reference(dt, shape):
    rows, cols = shape
    if dt in (2, 3) and cols % 32:
        pytest.skip("4-bit needs cols % 32 == 0")
    rng = np.random.default_rng(dt * 100 + cols)
    d, s = ct.synth_matrix(rng, ct.DT_NAMES[dt], rows, cols)
    d = np.frombuffer(d, np.uint8).copy()
    s = np.frombuffer(s, np.uint8).copy() if s else None
    x = rng.standard_normal(cols).astype(np.float32)
    ref = orc.RefLib().matvec(dt, d, s, rows, cols, x)
    got = orc.matvec(dt, d, s, rows, cols, x)
    assert np.array_equal(ref.view(np.uint32), got.view(np.uint32))


@needs_ref
def test_rmsnorm_and_f16_bit_exact_vs_reference():
    rng = np.random.default_rng(3)
    rl = orc.RefLib()
    for n in (7, 64, 2880):
        x = rng.standard_normal(n).astype(np.float32) * 3
        w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        assert np.array_equal(rl.rmsnorm(x, w, 1e-5), orc.rmsnorm(x, w, 1e-5))
    v = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 2000),
                        np.array([6.1e-5, 6.09e-5, 65504, 65519, 65520, 1e9, -0.0, 2 ** -14, 2 ** -15], np.float32)])
    assert np.array_equal(rl.to_f16(v), orc.f32_to_f16_ftz(v))


@needs_ref
@pytest.mark.parametrize("case", ["c1", "bf16_q8r", "mxfp4_blocks", "qwen3moe_q4g32", "bf16_f32"])
def test_model_bit_exact_vs_reference(case, tmp_path):
    if case == "c1":
        spec, edt = ct.config_spec("c1_tiny")
        md = ct.write_synthetic_model(str(tmp_path / "m"), spec, edt, seed=0)
    else:
        md, _ = load_validate_case(case, str(tmp_path / "m"))
    rl = orc.RefLib()
    ids = [1, 17, 42, 5, 99, 3, 77, 12]
    # per-token forward (MIDGE_NO_BATCH path)
    ref, om = orc.RefModel(rl, md, 64), orc.OracleModel(md, 64)
    for t in ids:
        assert np.array_equal(ref.forward(t), om.forward(t))
    ref.close(), om.close()
    # expert-major batch
    ref, om = orc.RefModel(rl, md, 64), orc.OracleModel(md, 64)
    assert np.array_equal(ref.forward_batch(ids), om.forward_batch(ids, False))
    ref.close(), om.close()


@pytest.mark.parametrize("case", VALIDATE_CASES)
def test_oracle_matches_reference_golden(case, tmp_path):
    """tools/validate.py's cases: oracle vs the reference midged's stored
    tfall logits (7 printed digits) and its 24 greedy tokens."""
    md, g = load_validate_case(case, str(tmp_path / "m"))
    om = orc.OracleModel(md, int(g["ctx"]))
    lg = om.prefill(list(g["ids"]), tfall=True)
    assert max_rel(g["tfall"], lg) < 1e-6
    toks = []
    cur = lg[-1]
    for _ in range(len(g["gen"])):
        t = orc.sample(cur, 0.0, 0.9, 1)[0]
        toks.append(t)
        cur = om.forward(t)
    assert toks == list(g["gen"])
    om.close()


def test_oracle_matches_reference_golden_c1(tmp_path):
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "c1_tiny.npz"))
    spec, edt = ct.config_spec("c1_tiny")
    md = ct.write_synthetic_model(str(tmp_path / "m"), spec, edt, seed=0)
    import hashlib
    assert hashlib.sha256(open(os.path.join(md, "dense.midge"), "rb").read()).hexdigest() == str(z["sha_dense"])
    assert hashlib.sha256(open(os.path.join(md, "experts.midge"), "rb").read()).hexdigest() == str(z["sha_experts"])
    ctx = int(z["ctx"])
    om = orc.OracleModel(md, ctx)
    lg = om.prefill(list(z["prompt"]), tfall=True)
    assert max_rel(z["tfall"], lg) < 1e-6
    om.close()
    om = orc.OracleModel(md, ctx)
    cur = om.prefill(list(z["prompt"]))
    toks = []
    for _ in range(len(z["gen"])):
        t = int(np.argmax(cur))
        toks.append(t)
        cur = om.forward(t)
    assert toks == list(z["gen"])
    om.close()


def test_container_writer_matches_reference_writer(tmp_path):
    """midge_b200.container writes byte-identical files to the reference's
    tools/midgepack.py writers (checked only where the reference tree exists)."""
    ref = orc.reference_dir()
    ref_tools = os.path.join(ref, "tools") if ref else ""
    if not ref or not os.path.exists(os.path.join(ref_tools, "midgepack.py")):
        pytest.skip("reference tools absent")
    import importlib.util
    spec_ = importlib.util.spec_from_file_location("midgepack", os.path.join(ref_tools, "midgepack.py"))
    wp = importlib.util.module_from_spec(spec_)
    spec_.loader.exec_module(wp)
    rng = np.random.default_rng(5)
    spec, _ = ct.config_spec("c1_tiny")
    w = rng.standard_normal((64, 96)).astype(np.float32)
    v = rng.standard_normal(96).astype(np.float32)
    dw = wp.DenseWriter(str(tmp_path / "a.midge"), spec)
    dw.add("w", w, "q8r")
    dw.add("v", v)
    dw.close()
    d, s = wp.q8r_encode(w)
    ct.write_dense(str(tmp_path / "b.midge"), spec,
                   [("w", "q8r", [64, 96], d, s), ("v", "f32", [96], v.tobytes(), b"")])
    assert open(tmp_path / "a.midge", "rb").read() == open(tmp_path / "b.midge", "rb").read()
    a = wp.ExpertLayout("mxfp4", 2880, 2880, 128, 36)
    b = ct.ExpertLayout("mxfp4", 2880, 2880, 128, 36)
    assert (a.expert_stride, a.total) == (b.expert_stride, b.total) == (14031360, 36 * 128 * 14031360)
