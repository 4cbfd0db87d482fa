"""Kernel-level parity: each CUDA entry point of libmidgecuda.so against the
CPU oracle (oracle/oracle.c, itself bit-exact with the reference engine) on
the same seeded inputs.

Tolerances: dequantised values, f16 conversions, ue8m0 scales, router logits
and selected experts are compared bit for bit.  Matvec outputs differ from
the reference only by fp32 summation order (and the exact f16 hi/lo split of
the activations, ~2^-22 relative per element), so they are bounded by
TOL_DOT * sum_c |w_rc| |x_c| per output row.
"""
import ctypes as C
import zlib

import numpy as np
import pytest

from midge_b200 import abi
from midge_b200 import container as ct
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL_DOT = 2e-6


def _mat(rng, dt, rows, cols):
    d, s = ct.synth_matrix(rng, dt, rows, cols)
    return np.frombuffer(d, np.uint8).copy(), (np.frombuffer(s, np.uint8).copy() if s else None)


def _to_ue8m0(torch, s_np):
    s_dev = torch.from_numpy(s_np).cuda()
    out = torch.zeros(s_np.size // 2, dtype=torch.uint8, device="cuda")
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    abi.check(abi.lib.mg_scales_to_ue8m0(s_dev.data_ptr(), out.data_ptr(), s_np.size // 2, bad.data_ptr(), None))
    torch.cuda.synchronize()
    assert int(bad.item()) == 0
    return out


GEMV_SHAPES = [(256, 256), (2880, 2880), (5760, 2880), (2880, 768), (100, 64), (48, 128), (33, 320)]


@pytest.mark.parametrize("dt", ["mxfp4", "q4g32", "q8r", "f32"])
@pytest.mark.parametrize("shape", GEMV_SHAPES)
@pytest.mark.parametrize("n_tok", [1, 3, 4, 8, 16])
def test_gemv_matches_oracle(torch_cuda, dt, shape, n_tok):
    torch = torch_cuda
    rows, cols = shape
    if dt in ("mxfp4", "q4g32") and cols % 32:
        pytest.skip("4-bit needs cols % 32")
    rng = np.random.default_rng(zlib.crc32(f"{dt}-{rows}-{cols}-{n_tok}".encode()))
    d, s = _mat(rng, dt, rows, cols)
    x = rng.standard_normal((n_tok, cols)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(rows)).astype(np.float32)
    dtc = ct.DT_CODES[dt]
    fmts = [abi.MG_SCALE_F16] + ([abi.MG_SCALE_UE8M0] if dt == "mxfp4" else [])
    for fmt in fmts:
        d_dev = torch.from_numpy(d).cuda()
        s_dev = None
        if s is not None:
            s_dev = _to_ue8m0(torch, s) if fmt == abi.MG_SCALE_UE8M0 else torch.from_numpy(s).cuda()
        x_dev = torch.from_numpy(x).cuda()
        b_dev = torch.from_numpy(bias).cuda()
        y_dev = torch.full((n_tok, rows), 0.5, dtype=torch.float32, device="cuda")
        prev = None
        for accumulate in (0, 1):
            abi.check(abi.lib.mg_gemv(dtc, fmt, d_dev.data_ptr(), None if s_dev is None else s_dev.data_ptr(), rows,
                                      cols, x_dev.data_ptr(), cols, n_tok, b_dev.data_ptr(), accumulate,
                                      y_dev.data_ptr(), rows, None))
            torch.cuda.synchronize()
            got = y_dev.cpu().numpy()
            for t in range(n_tok):
                ref = orc.matvec(dtc, d, s, rows, cols, x[t]) + bias
                mag = orc.matvec_abs(dtc, d, s, rows, cols, x[t])
                want = ref.astype(np.float64)
                if accumulate:
                    want = want + prev[t]
                err = np.abs(got[t].astype(np.float64) - want)
                bound = TOL_DOT * mag + 1e-6 * (1 + np.abs(want))
                assert np.all(err <= bound), (fmt, accumulate, t, float((err / (mag + 1e-30)).max()))
            prev = got.copy()


@pytest.mark.parametrize("dt", ["mxfp4", "q8r"])
@pytest.mark.parametrize("shape", [(5760, 2880), (2880, 2880)])
@pytest.mark.parametrize("n_tok", [64, 256])
def test_gemv_wide_batches_c2(torch_cuda, dt, shape, n_tok):
    """The C2 microbench shapes (gpt-oss gate_up [5760 x 2880] and down
    [2880 x 2880]) at token batches 64 and 256, every output row of every
    token against the oracle (16-token groups, each a full weight pass)."""
    torch = torch_cuda
    rows, cols = shape
    rng = np.random.default_rng(zlib.crc32(f"wide-{dt}-{rows}-{n_tok}".encode()))
    d, s = _mat(rng, dt, rows, cols)
    x = rng.standard_normal((n_tok, cols)).astype(np.float32)
    dtc = ct.DT_CODES[dt]
    fmt = abi.MG_SCALE_UE8M0 if dt == "mxfp4" else abi.MG_SCALE_F16
    d_dev = torch.from_numpy(d).cuda()
    s_dev = _to_ue8m0(torch, s) if dt == "mxfp4" else torch.from_numpy(s).cuda()
    x_dev = torch.from_numpy(x).cuda()
    y_dev = torch.empty((n_tok, rows), dtype=torch.float32, device="cuda")
    abi.check(abi.lib.mg_gemv(dtc, fmt, d_dev.data_ptr(), s_dev.data_ptr(), rows, cols, x_dev.data_ptr(), cols, n_tok,
                              None, 0, y_dev.data_ptr(), rows, None))
    torch.cuda.synchronize()
    got = y_dev.cpu().numpy()
    for t in range(n_tok):
        want = orc.matvec(dtc, d, s, rows, cols, x[t]).astype(np.float64)
        mag = orc.matvec_abs(dtc, d, s, rows, cols, x[t])
        err = np.abs(got[t].astype(np.float64) - want)
        assert np.all(err <= TOL_DOT * mag + 1e-6 * (1 + np.abs(want))), (t, float((err / (mag + 1e-30)).max()))


@pytest.mark.parametrize("dt", ["mxfp4", "q4g32", "q8r", "f32"])
def test_dequant_rows_bit_exact(torch_cuda, dt):
    torch = torch_cuda
    rng = np.random.default_rng(11)
    rows, cols = 300, 256
    d, s = _mat(rng, dt, rows, cols)
    ids = np.array([0, 5, 299, 17, 5, 150], np.int32)
    want = orc.dequant_rows(ct.DT_CODES[dt], d, s, cols, ids)
    fmts = [abi.MG_SCALE_F16] + ([abi.MG_SCALE_UE8M0] if dt == "mxfp4" else [])
    for fmt in fmts:
        s_dev = None
        if s is not None:
            s_dev = _to_ue8m0(torch, s) if fmt == abi.MG_SCALE_UE8M0 else torch.from_numpy(s).cuda()
        out = torch.empty((len(ids), cols), dtype=torch.float32, device="cuda")
        d_dev, ids_dev = torch.from_numpy(d).cuda(), torch.from_numpy(ids).cuda()  # alive across the call
        abi.check(abi.lib.mg_dequant_rows(ct.DT_CODES[dt], fmt, d_dev.data_ptr(),
                                          None if s_dev is None else s_dev.data_ptr(), rows, cols,
                                          ids_dev.data_ptr(), len(ids), out.data_ptr(), None))
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_ue8m0_reexpression_exact(torch_cuda):
    torch = torch_cuda
    e = np.arange(-24, 16)
    f16 = np.exp2(e).astype(np.float16)
    extra = np.array([0.0, 3.0, -2.0, np.inf, 0.75, 2.0 ** -24 * 3], np.float16)
    allv = np.concatenate([f16, extra]).view(np.uint16)
    out = torch.zeros(len(allv), dtype=torch.uint8, device="cuda")
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    src = torch.from_numpy(allv.copy()).cuda()
    abi.check(abi.lib.mg_scales_to_ue8m0(src.data_ptr(), out.data_ptr(), len(allv), bad.data_ptr(), None))
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    assert list(o[:len(e)]) == list(e + 127)
    assert o[len(e)] == 0                      # zero scale -> reserved code 0
    assert int(bad.item()) == 5                 # 3, -2, inf, 0.75, 3*2^-24 are not powers of two


def test_f16_ftz_bit_exact(torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(2)
    v = np.concatenate([
        (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32),
        np.array([6.1e-5, 6.09e-5, 6.103515625e-05, 6.1035153e-05, 65504, 65519, 65520, 1e9, -0.0, 0.0,
                  np.inf, -np.inf, np.nan, 2 ** -14, 2 ** -15, -2 ** -14], np.float32)])
    out = torch.zeros(len(v), dtype=torch.int16, device="cuda")
    src = torch.from_numpy(v).cuda()
    abi.check(abi.lib.mg_to_f16_ftz(src.data_ptr(), out.data_ptr(), len(v), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    assert np.array_equal(got, orc.f32_to_f16_ftz(v))


@pytest.mark.parametrize("n", [64, 2880, 2048, 100])
def test_rmsnorm_close(torch_cuda, n):
    torch = torch_cuda
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((5, n)) * 4).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    out = torch.empty((5, n), dtype=torch.float32, device="cuda")
    x_dev, w_dev = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    abi.check(abi.lib.mg_rmsnorm(x_dev.data_ptr(), w_dev.data_ptr(), out.data_ptr(), n, 5, 1e-5, None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for r in range(5):
        want = orc.rmsnorm(x[r], w, 1e-5)
        assert np.max(np.abs(got[r] - want) / (np.abs(want) + 1e-6)) < 4e-6


@pytest.mark.parametrize("E,k", [(128, 4), (32, 4), (8, 2), (4, 2), (128, 8), (5, 5)])
@pytest.mark.parametrize("H", [2880, 2048, 64, 100])
@pytest.mark.parametrize("router_norm", [1, 0])
@pytest.mark.parametrize("variant", [0, 1])
def test_router_bit_exact(torch_cuda, E, k, H, router_norm, variant):
    """Router logits and top-k ids are bit-identical to the reference's AVX2
    path for the same normed input; weights differ only by expf ulps."""
    torch = torch_cuda
    rng = np.random.default_rng(E * 7 + H)
    n = 9
    xb = rng.standard_normal((n, H)).astype(np.float32)
    rw = (rng.standard_normal((E, H)) / np.sqrt(H)).astype(np.float32)
    rb = (0.1 * rng.standard_normal(E)).astype(np.float32)
    # planted ties: token 0 gets equal logits on two experts through equal rows
    rw[3] = rw[1]
    rb[3] = rb[1]
    lg_w, sel_w, w_w = orc.route(xb, rw, rb, k, router_norm, prefill=bool(variant))
    lg = torch.empty((n, E), dtype=torch.float32, device="cuda")
    sel = torch.empty((n, k), dtype=torch.int32, device="cuda")
    wt = torch.empty((n, k), dtype=torch.float32, device="cuda")
    xb_d, rw_d, rb_d = (torch.from_numpy(a).cuda() for a in (xb, rw, rb))
    abi.check(abi.lib.mg_router_topk(xb_d.data_ptr(), n, rw_d.data_ptr(), rb_d.data_ptr(), E, H, k, router_norm,
                                     variant, lg.data_ptr(), sel.data_ptr(), wt.data_ptr(), None))
    torch.cuda.synchronize()
    assert np.array_equal(lg.cpu().numpy().view(np.uint32), lg_w.view(np.uint32))
    assert np.array_equal(sel.cpu().numpy(), sel_w)
    assert np.allclose(wt.cpu().numpy(), w_w, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("dt", ["mxfp4", "q4g32", "q8r", "f32"])
@pytest.mark.parametrize("n_tok,top_k,E", [(1, 4, 16), (3, 2, 4), (8, 4, 32), (16, 4, 8), (5, 8, 16)])
def test_moe_ffn_matches_oracle(torch_cuda, dt, n_tok, top_k, E):
    torch = torch_cuda
    H, F = (256, 192) if dt != "q8r" else (256, 128)
    rng = np.random.default_rng(n_tok * 31 + top_k + E)
    lay = ct.ExpertLayout(dt, H, F, E, 2)
    blob = ct.expert_blob(lay, rng)
    layer = 1
    xb = rng.standard_normal((n_tok, H)).astype(np.float32)
    x0 = rng.standard_normal((n_tok, H)).astype(np.float32)
    sel = np.stack([rng.permutation(E)[:top_k] for _ in range(n_tok)]).astype(np.int32)
    w = rng.dirichlet(np.ones(top_k), n_tok).astype(np.float32)
    act_plain, alpha, limit = (1, 1.702, 7.0) if dt == "q8r" else (0, 1.702, 7.0)
    dtc = ct.DT_CODES[dt]

    def expert_mat(e, m):
        r, c = lay.rows[m], lay.cols[m]
        db, sb = ct.blob_sizes(dt, r, c)
        o = lay.offset(layer, e, m, "data")
        d = blob[o:o + db]
        so = lay.offset(layer, e, m, "scales")
        s = blob[so:so + sb] if sb else None
        bo = lay.offset(layer, e, m, "bias")
        return d, s, blob[bo:bo + 4 * r].view(np.float32), r, c

    want = x0.copy().astype(np.float64)
    mags = np.zeros((n_tok, H))
    for t in range(n_tok):
        moe = np.zeros(H, np.float32)
        for i in range(top_k):
            e = int(sel[t, i])
            dg, sg, bg, r, c = expert_mat(e, "gate")
            du, su, bu, _, _ = expert_mat(e, "up")
            g = orc.matvec(dtc, dg, sg, r, c, xb[t]) + bg
            u = orc.matvec(dtc, du, su, r, c, xb[t]) + bu
            h = g.copy()
            orc.lib.or_swiglu(h.ctypes.data, u.ctypes.data, r, act_plain, alpha, limit)
            dd, sd, bd, r2, c2 = expert_mat(e, "down")
            y = orc.matvec(dtc, dd, sd, r2, c2, h) + bd
            moe += w[t, i] * y
            mags[t] += np.abs(w[t, i]) * (orc.matvec_abs(dtc, dd, sd, r2, c2, h) + np.abs(bd))
        want[t] += moe
    L = abi.MgExpertLayout()
    abi.check(abi.lib.mg_expert_layout_init(C.byref(L), dtc, H, F, E))
    blob_dev = torch.from_numpy(blob).cuda()
    x_dev = torch.from_numpy(x0).cuda()
    hbuf = torch.empty(n_tok * top_k * F, dtype=torch.float32, device="cuda")
    xb_d, sel_d, w_d = (torch.from_numpy(a).cuda() for a in (xb, sel, w))
    abi.check(abi.lib.mg_moe_ffn(C.byref(L), blob_dev.data_ptr(), layer, E, xb_d.data_ptr(), n_tok, top_k,
                                 sel_d.data_ptr(), w_d.data_ptr(), act_plain, alpha, limit, hbuf.data_ptr(),
                                 x_dev.data_ptr(), None))
    torch.cuda.synchronize()
    got = x_dev.cpu().numpy()
    # the gate/up error passes through the activation (slope <= ~1.1 * (limit+1))
    bound = 3e-5 * (mags + np.abs(x0)) + 1e-5
    err = np.abs(got - want)
    assert np.all(err <= bound), float((err / (mags + 1e-9)).max())
