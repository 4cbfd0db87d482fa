"""ctypes wrapper of the CPU checker (oracle/oracle.c) and of the reference
engine compiled as a library (oracle/_ref/libmidgeref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py, always as the checker, never as the thing measured.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libmidgeref.so")
REF_MIDGED = os.path.join(HERE, "_ref", "midged")

i64, i32, f32, vp = C.c_int64, C.c_int, C.c_float, C.c_void_p


def reference_dir():
    """The reference source tree, read-only: $MIDGE_REFERENCE, else the
    reference_path that BASELINE.json at the repository root names; None when
    neither names an existing directory (e.g. on a GPU box, which only uses
    the prebuilt oracle/_ref)."""
    cand = os.environ.get("MIDGE_REFERENCE")
    if not cand:
        try:
            import json

            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                cand = json.load(f).get("reference_path")
        except (OSError, ValueError):
            cand = None
    return cand if cand and os.path.isdir(cand) else None


def build():
    """Compile liboracle.so (always) and the reference build (when the
    reference tree is present)."""
    cmd = ["make", "-s", "-f", os.path.join(HERE, "Makefile")]
    ref = reference_dir()
    if ref:
        cmd.append(f"REF={ref}")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)


class OrSpec(C.Structure):
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


def _load():
    if not os.path.exists(LIB):
        build()
    lib = C.CDLL(LIB)
    sig = {
        "or_f16_to_f32": (f32, [C.c_uint16]),
        "or_f32_to_f16_ftz": (C.c_uint16, [f32]),
        "or_dequant_row": (None, [i32, vp, vp, i64, i64, vp]),
        "or_matvec": (None, [i32, vp, vp, i64, i64, vp, vp]),
        "or_matvec_abs": (None, [i32, vp, vp, i64, i64, vp, vp]),
        "or_rmsnorm": (None, [vp, vp, vp, i64, f32]),
        "or_route": (None, [vp, i32, vp, vp, i32, i64, i32, i32, i32, vp, vp, vp]),
        "or_swiglu": (None, [vp, vp, i64, i32, f32, f32]),
        "or_model_new": (vp, [C.POINTER(OrSpec), i32, i32, vp]),
        "or_model_set": (i32, [vp, C.c_char_p, i32, i64, i64, vp, vp]),
        "or_forward": (i32, [vp, i32, vp, vp, vp]),
        "or_forward_batch": (i32, [vp, vp, i32, i32, i32, vp]),
        "or_model_pos": (i32, [vp]),
        "or_model_usage": (C.POINTER(C.c_uint32), [vp]),
        "or_model_expert_loads": (C.c_uint64, [vp]),
        "or_model_free": (None, [vp]),
        "or_sample": (i32, [vp, i64, f32, f32, C.POINTER(C.c_uint64)]),
        "or_expert_layout": (None, [i32, i64, i64, i64, vp, vp, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def p(a):
    return None if a is None else a.ctypes.data


# ------------------------------------------------------------ kernel pieces
def matvec(dt: int, data: np.ndarray, scales, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(rows, np.float32)
    lib.or_matvec(dt, p(data), p(scales), rows, cols, p(x), p(y))
    return y


def matvec_abs(dt, data, scales, rows, cols, x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(rows, np.float64)
    lib.or_matvec_abs(dt, p(data), p(scales), rows, cols, p(x), p(y))
    return y


def dequant_rows(dt, data, scales, cols, ids) -> np.ndarray:
    out = np.empty((len(ids), cols), np.float32)
    for i, r in enumerate(ids):
        lib.or_dequant_row(dt, p(data), p(scales), cols, int(r), out[i].ctypes.data)
    return out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib.or_rmsnorm(p(x), p(np.ascontiguousarray(w, np.float32)), p(out), x.shape[-1], eps)
    return out


def route(xb: np.ndarray, rw: np.ndarray, rb: np.ndarray, top_k: int, router_norm: int, prefill: bool):
    xb = np.ascontiguousarray(xb, np.float32)
    n, H = xb.shape
    E = rw.shape[0]
    logits = np.empty((n, E), np.float32)
    sel = np.empty((n, top_k), np.int32)
    w = np.empty((n, top_k), np.float32)
    lib.or_route(p(xb), n, p(np.ascontiguousarray(rw, np.float32)), p(np.ascontiguousarray(rb, np.float32)), E, H,
                 top_k, router_norm, 1 if prefill else 0, p(logits), p(sel), p(w))
    return logits, sel, w


def f32_to_f16_ftz(x: np.ndarray) -> np.ndarray:
    return np.array([lib.or_f32_to_f16_ftz(float(v)) for v in np.asarray(x, np.float32).ravel()], np.uint16)


def sample(logits: np.ndarray, temp: float, topp: float, state: int):
    st = C.c_uint64(state)
    lg = np.ascontiguousarray(logits, np.float32)
    tok = lib.or_sample(p(lg), len(lg), temp, topp, C.byref(st))
    return tok, st.value


# ------------------------------------------------------------------- model
class OracleModel:
    """The whole reference forward on the CPU, over a converted model dir."""

    def __init__(self, model_dir: str | None, ctx: int, arrays=None):
        """model_dir: a converted model directory; or arrays = (spec, dense,
        expert_dt, blob) held in memory (see from_arrays)."""
        import sys
        sys.path.insert(0, os.path.dirname(HERE))
        from midge_b200.container import DT_CODES, ModelDir, spec_fields

        if arrays is None:
            self.md = ModelDir(model_dir)
            spec, expert_dt, blob = self.md.spec, self.md.expert_dt, self.md.expert_blob()
            tensors = list(self.md.tensors())
        else:
            self.md = None
            spec, dense, expert_dt, blob = arrays
            tensors = [(n, dt, int(sh[0]), int(sh[1]) if len(sh) > 1 else 0, np.frombuffer(d, np.uint8),
                        None if s is None or not len(s) else np.frombuffer(s, np.uint8)) for n, dt, sh, d, s in dense]
        f = spec_fields(spec)
        self._sl = (i32 * f["n_layers"])(*f.pop("layer_sliding"))
        self.spec = OrSpec(**f)
        self.spec.layer_sliding = C.cast(self._sl, C.POINTER(i32))
        self.vocab = f["vocab"]
        self.top_k = f["top_k"]
        self.n_layers = f["n_layers"]
        self.n_experts = f["n_experts"]
        self._blob = np.ascontiguousarray(blob, dtype=np.uint8)
        self.h = lib.or_model_new(C.byref(self.spec), ctx, DT_CODES[expert_dt], self._blob.ctypes.data)
        self._keep = []
        for name, dt, rows, cols, d, s in tensors:
            self._keep.append((d, s))
            rc = lib.or_model_set(self.h, name.encode(), DT_CODES[dt], rows, cols, d.ctypes.data,
                                  None if s is None else s.ctypes.data)
            if rc != 0:
                pass  # tensors the engine does not use

    @classmethod
    def from_arrays(cls, spec: dict, dense, expert_dt: str, blob, ctx: int):
        """The oracle over in-memory tensors (the same arrays a GPU model was
        built from): dense = [(name, dt, shape, data, scales)], blob = the
        experts.midge data region.  The arrays must outlive the model."""
        return cls(None, ctx, arrays=(spec, dense, expert_dt, blob))

    def forward(self, tok: int, trace=False):
        lg = np.empty(self.vocab, np.float32)
        sel = np.empty((self.n_layers, self.top_k), np.int32) if trace else None
        w = np.empty((self.n_layers, self.top_k), np.float32) if trace else None
        rc = lib.or_forward(self.h, int(tok), p(lg), p(sel), p(w))
        if rc:
            raise RuntimeError(f"oracle forward rc={rc}")
        return (lg, sel, w) if trace else lg

    def forward_batch(self, toks, tfall: bool):
        t = np.ascontiguousarray(toks, np.int32)
        out = np.empty((len(t) if tfall else 1, self.vocab), np.float32)
        rc = lib.or_forward_batch(self.h, p(t), len(t), 1 if tfall else 0, 1, p(out))
        if rc:
            raise RuntimeError(f"oracle forward_batch rc={rc}")
        return out if tfall else out[0]

    def prefill(self, toks, tfall=False):
        """midged's ids:/tf:/tfall: path: 64-token chunks through forward_batch
        (engine/midge.c:796-800)."""
        outs = []
        for o in range(0, len(toks), 64):
            chunk = toks[o:o + 64]
            r = self.forward_batch(chunk, tfall)
            outs.append(r if tfall else r[None])
        return np.concatenate(outs) if tfall else outs[-1][0]

    def pos(self):
        return lib.or_model_pos(self.h)

    def usage(self):
        u = lib.or_model_usage(self.h)
        return np.ctypeslib.as_array(u, shape=(self.n_layers * self.n_experts,)).reshape(self.n_layers,
                                                                                      self.n_experts).copy()

    def close(self):
        if self.h:
            lib.or_model_free(self.h)
            self.h = None
        self._keep, self._blob = [], None
        if self.md is not None:
            self.md.close()


# ------------------------------------------------------- the reference itself
def ref_available() -> bool:
    return os.path.exists(REF_LIB)


class RefLib:
    """oracle/_ref/libmidgeref.so: the reference's own functions."""

    def __init__(self):
        self.lib = C.CDLL(REF_LIB)
        L = self.lib
        L.ref_matvec.argtypes = [i32, vp, vp, i64, i64, vp, vp]
        L.ref_row.argtypes = [i32, vp, vp, i64, i64, i64, vp]
        L.ref_rmsnorm.argtypes = [vp, vp, vp, i64, f32]
        L.ref_to_f16.argtypes = [f32]
        L.ref_to_f16.restype = C.c_uint16
        L.ref_model_load.argtypes = [C.c_char_p, i32]
        L.ref_model_load.restype = vp
        L.ref_forward.argtypes = [vp, i32, vp]
        L.ref_forward_batch.argtypes = [vp, vp, i32, vp]
        L.ref_vocab.argtypes = [vp]
        L.ref_model_free.argtypes = [vp]
        L.ref_usage.argtypes = [vp]
        L.ref_usage.restype = C.POINTER(C.c_uint32)

    def matvec(self, dt, data, scales, rows, cols, x):
        y = np.empty(rows, np.float32)
        self.lib.ref_matvec(dt, p(data), p(scales), rows, cols, p(np.ascontiguousarray(x, np.float32)), p(y))
        return y

    def rmsnorm(self, x, w, eps):
        out = np.empty_like(x)
        self.lib.ref_rmsnorm(p(x), p(w), p(out), x.shape[-1], eps)
        return out

    def to_f16(self, x):
        return np.array([self.lib.ref_to_f16(float(v)) for v in np.asarray(x, np.float32).ravel()], np.uint16)

    def row(self, dt, data, scales, rows, cols, r):
        out = np.empty(cols, np.float32)
        self.lib.ref_row(dt, p(data), p(scales), rows, cols, r, p(out))
        return out


class RefModel:
    def __init__(self, rl: RefLib, model_dir: str, ctx: int):
        self.rl = rl
        self.h = rl.lib.ref_model_load(model_dir.encode(), ctx)
        self.vocab = rl.lib.ref_vocab(self.h)

    def forward(self, tok):
        lg = np.empty(self.vocab, np.float32)
        self.rl.lib.ref_forward(self.h, int(tok), p(lg))
        return lg

    def forward_batch(self, toks):
        t = np.ascontiguousarray(toks, np.int32)
        lg = np.empty(self.vocab, np.float32)
        self.rl.lib.ref_forward_batch(self.h, p(t), len(t), p(lg))
        return lg

    def close(self):
        if self.h:
            self.rl.lib.ref_model_free(self.h)
            self.h = None
