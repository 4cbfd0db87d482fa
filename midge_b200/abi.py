"""ctypes binding of libmidgecuda.so (include/midgecuda.h).

The library is loaded from the package directory; if it is missing the import
fails loudly -- there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .container import DT_CODES, ModelDir, spec_fields

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libmidgecuda.so")

MG_F32, MG_Q8R, MG_Q4G32, MG_MXFP4 = 0, 1, 2, 3
MG_SCALE_F16, MG_SCALE_UE8M0 = 0, 1
MG_OK, MG_ERR_ARG, MG_ERR_CUDA, MG_ERR_OOM, MG_ERR_STATE, MG_ERR_RANGE, MG_ERR_SPEC = 0, -1, -2, -3, -4, -5, -6
MG_ERR_TIMEOUT, MG_ERR_COMM = -8, -9
EP_ID_BYTES = 128

i64, i32, f32, vp = C.c_int64, C.c_int, C.c_float, C.c_void_p


class MgSpec(C.Structure):
    _fields_ = [
        ("hidden", i64), ("vocab", i64), ("ffn", i64),
        ("n_layers", i32), ("n_heads", i32), ("n_kv_heads", i32), ("head_dim", i32),
        ("n_experts", i32), ("top_k", i32),
        ("alpha", f32), ("limit", f32),
        ("act_plain", i32), ("router_norm", i32), ("qk_norm", i32),
        ("sliding_window", i32), ("sinks", i32),
        ("norm_eps", f32), ("rope_theta", f32),
        ("yarn", i32),
        ("yarn_factor", f32), ("yarn_beta_fast", f32), ("yarn_beta_slow", f32),
        ("yarn_orig_ctx", i32), ("yarn_truncate", i32),
        ("attn_scale", f32),
        ("layer_sliding", C.POINTER(i32)),
    ]


class MgExpertLayout(C.Structure):
    _fields_ = [("dt", i32), ("scale_fmt", i32), ("hidden", i64), ("ffn", i64),
                ("off", (i64 * 3) * 3), ("expert_stride", i64), ("layer_stride", i64)]


class MidgeError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"midgecuda error {code}: {msg}")
        self.code = code


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built (run python -m midge_b200.build); "
                          "the midge_b200 hot path has no CPU fallback")
    lib = C.CDLL(LIB_PATH)
    sig = {
        "mg_last_error": (C.c_char_p, []),
        "mg_version": (i32, []),
        "mg_gemv": (i32, [i32, i32, vp, vp, i64, i64, vp, i64, i32, vp, i32, vp, i64, vp]),
        "mg_dequant_rows": (i32, [i32, i32, vp, vp, i64, i64, vp, i32, vp, vp]),
        "mg_scales_to_ue8m0": (i32, [vp, vp, i64, vp, vp]),
        "mg_rmsnorm": (i32, [vp, vp, vp, i64, i32, f32, vp]),
        "mg_to_f16_ftz": (i32, [vp, vp, i64, vp]),
        "mg_router_topk": (i32, [vp, i32, vp, vp, i32, i64, i32, i32, i32, vp, vp, vp, vp]),
        "mg_expert_layout_init": (i32, [C.POINTER(MgExpertLayout), i32, i64, i64, i64]),
        "mg_moe_ffn": (i32, [C.POINTER(MgExpertLayout), vp, i32, i32, vp, i32, i32, vp, vp, i32, f32, f32, vp, vp,
                             vp]),
        "mg_moe_ffn_noalloc": (i32, [C.POINTER(MgExpertLayout), vp, i32, i32, vp, i32, i32, vp, vp, i32, f32, f32,
                                     vp, vp]),
        "mg_model_create": (i32, [C.POINTER(MgSpec), i32, i32, i32, C.POINTER(vp)]),
        "mg_model_set_dense": (i32, [vp, C.c_char_p, i32, i64, i64, vp, vp]),
        "mg_model_set_experts": (i32, [vp, i32, vp, C.c_uint64]),
        "mg_model_synth_experts": (i32, [vp, i32, C.c_uint64]),
        "mg_model_ready": (i32, [vp]),
        "mg_model_reset": (i32, [vp, i32]),
        "mg_model_pos": (i32, [vp, i32]),
        "mg_forward": (i32, [vp, i32, i32, vp, vp]),
        "mg_forward_batch": (i32, [vp, i32, vp, i32, i32, vp]),
        "mg_decode_step": (i32, [vp, i32, vp, vp, vp, vp]),
        "mg_model_get_usage": (i32, [vp, vp]),
        "mg_model_set_usage": (i32, [vp, vp]),
        "mg_model_expert_loads": (C.c_uint64, [vp]),
        "mg_decode_greedy": (i32, [vp, i32, vp, vp, i32, vp]),
        "mg_model_kernel_launches": (C.c_uint64, [vp]),
        "mg_model_moe_stream": (i32, [vp, i32, i32, vp]),
        "mg_ep_unique_id": (i32, [vp]),
        "mg_model_set_ep": (i32, [vp, i32, i32, vp]),
        "mg_ep_watchdog_selftest": (i32, [i32, C.c_double, C.POINTER(i32)]),
        "mg_model_experts_device": (vp, [vp, C.POINTER(MgExpertLayout)]),
        "mg_model_stream": (vp, [vp]),
        "mg_model_free": (i32, [vp]),
        "mg_model_logits": (i32, [vp, i32, vp]),
        "mg_bench_gemv": (i32, [i32, i64, i64, i32, C.c_double, i32, C.POINTER(C.c_double)]),
        "mg_sample_topp": (i32, [vp, i64, i64, i32, f32, f32, vp, vp, vp, vp]),
        "mg_model_sample": (i32, [vp, i32, f32, f32, vp, vp]),
        "mg_model_put_logits": (i32, [vp, i32, vp]),
        "mg_wait_selftest": (i32, [i32, C.POINTER(i32)]),
        "mg_model_ep_stats": (i32, [vp, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()

# every entry point include/midgecuda.h declares (checked by the CPU tests)
EXPORTS = [n for n in dir(lib) if n.startswith("mg_")]


def check(rc):
    if rc != MG_OK:
        raise MidgeError(rc, (lib.mg_last_error() or b"").decode())
    return rc


def make_spec(spec: dict):
    """An MgSpec (and the int array it points at, which must stay alive)."""
    f = spec_fields(spec)
    arr = (i32 * f["n_layers"])(*f.pop("layer_sliding"))
    s = MgSpec(**f)
    s.layer_sliding = C.cast(arr, C.POINTER(i32))
    return s, arr


def ptr(a):
    """Host address of a numpy array (or None)."""
    if a is None:
        return None
    return a.ctypes.data


class Model:
    """A model resident on one GPU, driven through the C ABI with host buffers."""

    def __init__(self, spec: dict, ctx: int, max_seqs: int = 1, device: int = 0, ep=None):
        """ep: (rank, world, id bytes) for expert parallelism (midge_b200.ep)."""
        self.spec = spec
        self._cspec, self._arr = make_spec(spec)
        h = vp()
        check(lib.mg_model_create(C.byref(self._cspec), ctx, max_seqs, device, C.byref(h)))
        self.h = h
        self.vocab = int(spec["vocab"])
        self.ctx = ctx
        if ep is not None:
            rank, world, uid = ep
            buf = C.create_string_buffer(bytes(uid), EP_ID_BYTES)
            check(lib.mg_model_set_ep(self.h, int(rank), int(world), buf))

    @classmethod
    def from_dir(cls, path: str, ctx: int, max_seqs: int = 1, device: int = 0, ep=None):
        md = ModelDir(path)
        m = cls(md.spec, ctx, max_seqs, device, ep=ep)
        try:
            for name, dt, rows, cols, d, s in md.tensors():
                m.set_dense(name, dt, rows, cols, d, s)
            blob = md.expert_blob()
            check(lib.mg_model_set_experts(m.h, DT_CODES[md.expert_dt], blob.ctypes.data, blob.nbytes))
        finally:
            md.close()
        check(lib.mg_model_ready(m.h))
        return m

    @classmethod
    def from_arrays(cls, spec: dict, dense, expert_dt: str, blob, ctx: int, max_seqs: int = 1, device: int = 0,
                    ep=None):
        """A model from in-memory tensors: dense = [(name, dt, shape, data, scales)]
        as container.dense_tensors yields them, blob = the experts.midge data
        region (container.expert_blob)."""
        m = cls(spec, ctx, max_seqs, device, ep=ep)
        for name, dt, shape, d, s in dense:
            rows = int(shape[0])
            cols = int(shape[1]) if len(shape) > 1 else 0
            m.set_dense(name, dt, rows, cols, d, s if s is not None and len(s) else None)
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        check(lib.mg_model_set_experts(m.h, DT_CODES[expert_dt], blob.ctypes.data, blob.nbytes))
        check(lib.mg_model_ready(m.h))
        return m

    def set_dense(self, name, dt, rows, cols, data, scales=None):
        data = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray)) else data)
        if scales is not None and not isinstance(scales, np.ndarray):
            scales = np.frombuffer(scales, np.uint8) if len(scales) else None
        check(lib.mg_model_set_dense(self.h, name.encode(), DT_CODES[dt] if isinstance(dt, str) else dt, rows, cols,
                                     data.ctypes.data, None if scales is None else np.ascontiguousarray(scales).ctypes.data))

    def synth_experts(self, dt: str, seed: int):
        check(lib.mg_model_synth_experts(self.h, DT_CODES[dt], seed))

    def ready(self):
        check(lib.mg_model_ready(self.h))

    def forward(self, seq: int, token: int, want_logits=True):
        lg = np.empty(self.vocab, np.float32) if want_logits else None
        am = np.zeros(1, np.int32)
        check(lib.mg_forward(self.h, seq, int(token), ptr(lg), ptr(am)))
        return lg, int(am[0])

    def forward_batch(self, seq: int, toks, logits_mode: int = 1):
        t = np.ascontiguousarray(toks, dtype=np.int32)
        n = len(t)
        lg = None
        if logits_mode == 1:
            lg = np.empty(self.vocab, np.float32)
        elif logits_mode == 2:
            lg = np.empty((n, self.vocab), np.float32)
        check(lib.mg_forward_batch(self.h, seq, ptr(t), n, logits_mode, ptr(lg)))
        return lg

    def decode_step(self, seq_ids, toks, want_logits=False):
        s = np.ascontiguousarray(seq_ids, dtype=np.int32)
        t = np.ascontiguousarray(toks, dtype=np.int32)
        n = len(t)
        lg = np.empty((n, self.vocab), np.float32) if want_logits else None
        am = np.zeros(n, np.int32)
        check(lib.mg_decode_step(self.h, n, ptr(s), ptr(t), ptr(lg), ptr(am)))
        return lg, am

    def pos(self, seq=0):
        return lib.mg_model_pos(self.h, seq)

    def reset(self, seq=0):
        check(lib.mg_model_reset(self.h, seq))

    def usage(self):
        u = np.zeros((self.spec["n_layers"], self.spec["moe"]["experts"]), np.uint32)
        check(lib.mg_model_get_usage(self.h, ptr(u)))
        return u

    def expert_loads(self):
        return int(lib.mg_model_expert_loads(self.h))

    def decode_greedy(self, seqs, toks, n_steps):
        """n_steps greedy tokens for each sequence, fed back on the device:
        returns int32 [n_steps x len(seqs)]."""
        s = np.ascontiguousarray(seqs, dtype=np.int32)
        t = np.ascontiguousarray(toks, dtype=np.int32)
        out = np.zeros((n_steps, len(s)), np.int32)
        check(lib.mg_decode_greedy(self.h, len(s), ptr(s), ptr(t), n_steps, ptr(out)))
        return out

    def sample(self, n_rows, temp, topp, rng_states):
        """Next tokens of the first n_rows rows of the last logits, sampled on
        the device; rng_states (uint64 array, n_rows) advance in place."""
        out = np.zeros(n_rows, np.int32)
        rng = np.ascontiguousarray(rng_states, dtype=np.uint64)
        check(lib.mg_model_sample(self.h, n_rows, float(temp), float(topp), ptr(rng), ptr(out)))
        if rng is not rng_states:
            rng_states[:] = rng
        return out

    def kernel_launches(self):
        return int(lib.mg_model_kernel_launches(self.h))

    def experts_device(self):
        L = MgExpertLayout()
        p = lib.mg_model_experts_device(self.h, C.byref(L))
        return p, L

    def stream(self):
        return lib.mg_model_stream(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib.mg_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
