"""mg_moe_ffn_noalloc (no counterpart in the reference): the routed-expert FFN
with its gate/up scratch in the library's fixed device array, called through
the C ABI, against mg_moe_ffn with a caller buffer on the same inputs, twice
in a row (the second call reuses the array set up by the first).  Kept in a
file collected last so that it also runs after every other GPU test."""
import ctypes as C

import numpy as np
import pytest

from midge_b200 import abi
from midge_b200 import container as ct

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt,n_tok,top_k,E", [("mxfp4", 8, 4, 32), ("q8r", 3, 2, 8), ("mxfp4", 1, 4, 16)])
def test_noalloc_matches_moe_ffn(torch_cuda, dt, n_tok, top_k, E):
    torch = torch_cuda
    H, F = 256, 192 if dt != "q8r" else 128
    rng = np.random.default_rng(7 * n_tok + E)
    lay = ct.ExpertLayout(dt, H, F, E, 2)
    blob = ct.expert_blob(lay, rng)
    layer = 1
    xb = rng.standard_normal((n_tok, H)).astype(np.float32)
    x0 = rng.standard_normal((n_tok, H)).astype(np.float32)
    sel = np.stack([rng.permutation(E)[:top_k] for _ in range(n_tok)]).astype(np.int32)
    w = rng.dirichlet(np.ones(top_k), n_tok).astype(np.float32)
    L = abi.MgExpertLayout()
    abi.check(abi.lib.mg_expert_layout_init(C.byref(L), ct.DT_CODES[dt], H, F, E))
    blob_d = torch.from_numpy(np.frombuffer(blob, np.uint8).copy()).cuda()
    xb_d, sel_d, w_d = (torch.from_numpy(a).cuda() for a in (xb, sel, w))
    act_plain, alpha, limit = (1, 1.702, 7.0) if dt == "q8r" else (0, 1.702, 7.0)

    x_ref = torch.from_numpy(x0).cuda()
    hbuf = torch.empty(n_tok * top_k * F, dtype=torch.float32, device="cuda")
    abi.check(abi.lib.mg_moe_ffn(C.byref(L), blob_d.data_ptr(), layer, E, xb_d.data_ptr(), n_tok, top_k,
                                 sel_d.data_ptr(), w_d.data_ptr(), act_plain, alpha, limit, hbuf.data_ptr(),
                                 x_ref.data_ptr(), None))
    torch.cuda.synchronize()
    want = x_ref.cpu().numpy()
    for _ in range(2):
        x_na = torch.from_numpy(x0).cuda()
        abi.check(abi.lib.mg_moe_ffn_noalloc(C.byref(L), blob_d.data_ptr(), layer, E, xb_d.data_ptr(), n_tok, top_k,
                                             sel_d.data_ptr(), w_d.data_ptr(), act_plain, alpha, limit,
                                             x_na.data_ptr(), None))
        torch.cuda.synchronize()
        got = x_na.cpu().numpy()
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)


def test_noalloc_rejects_oversize(torch_cuda):
    """Both limits are checked before any launch: more than 16 tokens is a
    bad argument (as for mg_moe_ffn); 16 tokens whose gate/up activations
    exceed the fixed array are a range error."""
    L = abi.MgExpertLayout()
    abi.check(abi.lib.mg_expert_layout_init(C.byref(L), ct.DT_CODES["mxfp4"], 2880, 2880, 128))
    rc = abi.lib.mg_moe_ffn_noalloc(C.byref(L), 16, 0, 128, 16, 17, 4, 16, 16, 0, 1.702, 7.0, 16, None)
    assert rc == abi.MG_ERR_ARG
    assert b"tokens per call" in abi.lib.mg_last_error()
    abi.check(abi.lib.mg_expert_layout_init(C.byref(L), ct.DT_CODES["mxfp4"], 2880, 8192, 128))
    # 16 tokens x top-16 x 8192 = 2,097,152 floats > the fixed scratch
    rc = abi.lib.mg_moe_ffn_noalloc(C.byref(L), 16, 0, 128, 16, 16, 16, 16, 16, 0, 1.702, 7.0, 16, None)
    assert rc == abi.MG_ERR_RANGE
    assert b"fixed scratch" in abi.lib.mg_last_error()
