"""CPU-side checks of the C ABI: the library loads, exports every function
include/midgecuda.h declares, and its host-only logic agrees with the
container format.  No compute call is made (there is no GPU here)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from midge_b200 import abi
from midge_b200 import container as ct

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    txt = open(os.path.join(ROOT, "include", "midgecuda.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(mg_[a-z0-9_]+)\s*\(", txt)))


def test_header_functions_exported():
    names = declared_functions()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", abi.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (mg_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        getattr(abi.lib, n)


@pytest.mark.parametrize("dt", ["f32", "q8r", "q4g32", "mxfp4"])
@pytest.mark.parametrize("dims", [(64, 64, 4), (2880, 2880, 128), (2048, 768, 128), (256, 256, 8)])
def test_expert_layout_matches_container(dt, dims):
    h, f, e = dims
    L = abi.MgExpertLayout()
    abi.check(abi.lib.mg_expert_layout_init(C.byref(L), ct.DT_CODES[dt], h, f, e))
    ref = ct.ExpertLayout(dt, h, f, e, 1)
    assert L.expert_stride == ref.expert_stride and L.layer_stride == ref.layer_stride
    for mi, m in enumerate(ct.ExpertLayout.MATS):
        for pi, p in enumerate(("data", "scales", "bias")):
            assert L.off[mi][pi] == ref.off[(m, p)]


def test_bad_layout_rejected():
    L = abi.MgExpertLayout()
    assert abi.lib.mg_expert_layout_init(C.byref(L), 3, 100, 64, 4) == abi.MG_ERR_SPEC
    assert b"32" in abi.lib.mg_last_error()


def test_spec_struct_roundtrip():
    spec, _ = ct.config_spec("c4_120b")
    s, arr = abi.make_spec(spec)
    assert s.n_experts == 128 and s.top_k == 4 and s.hidden == 2880
    assert [arr[i] for i in range(4)] == [1, 0, 1, 0]
    assert abs(s.attn_scale - 0.125) < 1e-7 and s.yarn == 1 and abs(s.yarn_factor - 32) < 1e-6


def test_ue8m0_container_converter(tmp_path):
    """midge_b200.convert_ue8m0 rewrites experts.midge as dtype mxfp4e8: the
    same nibbles and biases, one ue8m0 byte per group scale at the offsets of
    the C layout for MG_MXFP4_E8, exactly the f16 scales again when read
    back; a scale that is not a power of two stops the conversion."""
    from midge_b200 import convert_ue8m0 as cv

    spec, edt = ct.config_spec("c1_tiny")
    src = ct.write_synthetic_model(str(tmp_path / "src"), spec, edt, seed=0)
    dst = cv.convert(src, str(tmp_path / "dst"))
    a, b = ct.ModelDir(src), ct.ModelDir(dst)
    assert b.expert_dt == "mxfp4e8"
    L = abi.MgExpertLayout()
    abi.check(abi.lib.mg_expert_layout_init(C.byref(L), 4, 256, 256, 8))
    assert L.dt == abi.MG_MXFP4 and L.scale_fmt == abi.MG_SCALE_UE8M0
    assert L.expert_stride == b.layout.expert_stride
    for mi, m in enumerate(ct.ExpertLayout.MATS):
        assert [L.off[mi][j] for j in range(3)] == [b.layout.off[(m, p)] for p in ("data", "scales", "bias")]
    ab, bb = a.expert_blob(), b.expert_blob()
    for layer in range(2):
        for e in range(8):
            for m in ct.ExpertLayout.MATS:
                r, c = a.layout.rows[m], a.layout.cols[m]
                nd, ns = r * c // 2, r * (c // 32)
                oa, ob = a.layout.offset(layer, e, m, "data"), b.layout.offset(layer, e, m, "data")
                assert np.array_equal(ab[oa:oa + nd], bb[ob:ob + nd])
                oa, ob = a.layout.offset(layer, e, m, "scales"), b.layout.offset(layer, e, m, "scales")
                s16 = ab[oa:oa + 2 * ns].view(np.uint16)
                back = np.exp2(bb[ob:ob + ns].astype(np.float64) - 127).astype(np.float16).view(np.uint16)
                assert np.array_equal(back, s16)
    a.close()
    b.close()
    with pytest.raises(ValueError):
        cv.f16_to_ue8m0(np.array([0x3C00, 0x3E00], np.uint16))  # 1.0 ok, 1.5 is not a power of two
