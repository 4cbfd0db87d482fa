"""The midge container format (v1), read and written without the reference tools.

Layout (engine/mten.h:1-31, docs/DESIGN.md:32-51 of the reference):
    [u64 LE header_len][JSON header][zero pad to 64][data]
dense.midge's header holds the model spec and a tensor index
{name: {dt, shape, off, soff}} (offsets relative to the 64-aligned data
start); experts.midge's header is {"midge":1,"kind":"experts","dt":...} and
its blobs sit at the deterministic offsets of ExpertLayout.

This module is host-side plumbing for the tests and the bench: reading a
converted model to hand its tensors to the C ABI, and writing seeded
synthetic models with the value distributions of the benchmark configs.
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import numpy as np

ALIGN = 64
# engine/mten.h:42, plus "mxfp4e8": MXFP4 with one ue8m0 byte per 32 columns
# (an opt-in expert dtype of this implementation, see convert_ue8m0.py)
DT_CODES = {"f32": 0, "q8r": 1, "q4g32": 2, "mxfp4": 3, "mxfp4e8": 4}
DT_NAMES = {v: k for k, v in DT_CODES.items()}


def align64(x: int) -> int:
    return (x + ALIGN - 1) & ~(ALIGN - 1)


def blob_sizes(dt: str, rows: int, cols: int):
    """(data bytes, scale bytes) of a [rows x cols] matrix; engine/mten.h:101-109."""
    if dt == "f32":
        return rows * cols * 4, 0
    if dt == "q8r":
        return rows * cols, rows * 4
    if dt in ("q4g32", "mxfp4"):
        return rows * cols // 2, rows * (cols // 32) * 2
    if dt == "mxfp4e8":
        return rows * cols // 2, rows * (cols // 32)
    raise ValueError(dt)


class ExpertLayout:
    """Deterministic expert offsets; engine/mten.h:136-150 (wt_expert_layout).
    Per layer, per expert, for gate, up, down: data, scales, f32 bias, each
    64-byte aligned; the expert stride is the aligned end."""

    MATS = ("gate", "up", "down")

    def __init__(self, dt: str, hidden: int, ffn: int, n_experts: int, n_layers: int):
        self.dt, self.hidden, self.ffn = dt, hidden, ffn
        self.n_experts, self.n_layers = n_experts, n_layers
        self.rows = {"gate": ffn, "up": ffn, "down": hidden}
        self.cols = {"gate": hidden, "up": hidden, "down": ffn}
        o = 0
        self.off = {}
        for m in self.MATS:
            db, sb = blob_sizes(dt, self.rows[m], self.cols[m])
            self.off[(m, "data")] = o
            o = align64(o + db)
            self.off[(m, "scales")] = o
            o = align64(o + sb)
            self.off[(m, "bias")] = o
            o = align64(o + self.rows[m] * 4)
        self.expert_stride = align64(o)
        self.layer_stride = self.expert_stride * n_experts
        self.total = self.layer_stride * n_layers

    def offset(self, layer: int, expert: int, mat: str, part: str) -> int:
        return layer * self.layer_stride + expert * self.expert_stride + self.off[(mat, part)]


# ------------------------------------------------------------------ reading
def _read_header(mm):
    (hl,) = struct.unpack_from("<Q", mm, 0)
    hdr = json.loads(bytes(mm[8:8 + hl]))
    return hdr, align64(8 + hl)


class Container:
    """A memory-mapped .midge file: header dict and the data region."""

    def __init__(self, path: str):
        self.path = path
        self.f = open(path, "rb")
        self.mm = mmap.mmap(self.f.fileno(), 0, access=mmap.ACCESS_READ)
        self.hdr, self.base = _read_header(self.mm)
        self.data = np.frombuffer(self.mm, dtype=np.uint8, offset=self.base)

    def close(self):
        self.data = None
        try:
            self.mm.close()
        except BufferError:  # views still alive elsewhere: the map goes with them
            pass
        self.f.close()


class ModelDir:
    """A converted model directory: dense.midge + experts.midge."""

    def __init__(self, path: str):
        self.path = path
        self.dense = Container(os.path.join(path, "dense.midge"))
        self.experts = Container(os.path.join(path, "experts.midge"))
        self.spec = self.dense.hdr["spec"]
        self.expert_dt = self.experts.hdr["dt"]
        s = self.spec
        self.layout = ExpertLayout(self.expert_dt, s["hidden"], s["moe"]["ffn"], s["moe"]["experts"], s["n_layers"])

    def tensors(self):
        """Yield (name, dt, rows, cols, data ndarray(u8), scales ndarray(u8) or None)."""
        for name, e in self.dense.hdr["tensors"].items():
            shape = e["shape"]
            dt = e.get("dt", "f32")
            rows = int(shape[0])
            cols = int(shape[1]) if len(shape) > 1 else 0
            if cols == 0:
                db, sb = rows * 4, 0
            else:
                db, sb = blob_sizes(dt, rows, cols)
            d = self.dense.data[e["off"]:e["off"] + db]
            s_ = self.dense.data[e["soff"]:e["soff"] + sb] if (sb and "soff" in e) else None
            yield name, dt, rows, cols, d, s_

    def expert_blob(self):
        return self.experts.data[: self.layout.total]

    def close(self):
        self.dense.close()
        self.experts.close()


def spec_fields(spec: dict) -> dict:
    """The spec fields the engine reads, with the reference's defaults
    (engine/midge.c:95-138)."""
    moe = spec.get("moe", {})
    attn = spec.get("attn", {})
    rope = spec.get("rope", {})
    y = rope.get("yarn")
    hd = int(spec.get("head_dim", 64))
    n_layers = int(spec["n_layers"])
    lt = attn.get("layer_types", [])
    sliding = [1 if (i < len(lt) and isinstance(lt[i], str) and "sliding" in lt[i]) else 0 for i in range(n_layers)]
    f = dict(
        hidden=int(spec["hidden"]), vocab=int(spec["vocab"]), ffn=int(moe["ffn"]),
        n_layers=n_layers, n_heads=int(spec["n_heads"]), n_kv_heads=int(spec["n_kv_heads"]), head_dim=hd,
        n_experts=int(moe["experts"]), top_k=int(moe["top_k"]),
        alpha=float(moe.get("alpha", 1.702)), limit=float(moe.get("limit", 7.0)),
        act_plain=1 if moe.get("act", "swiglu_clamp") == "swiglu" else 0,
        router_norm=int(moe.get("router_norm", 1)), qk_norm=int(bool(attn.get("qk_norm", 0))),
        sliding_window=int(attn.get("sliding_window", 0)), sinks=int(bool(attn.get("sinks", 0))),
        norm_eps=float(spec.get("norm_eps", 1e-5)), rope_theta=float(rope.get("theta", 10000.0)),
        yarn=1 if isinstance(y, dict) else 0,
        yarn_factor=float(y.get("factor", 1.0)) if isinstance(y, dict) else 0.0,
        yarn_beta_fast=float(y.get("beta_fast", 32.0)) if isinstance(y, dict) else 0.0,
        yarn_beta_slow=float(y.get("beta_slow", 1.0)) if isinstance(y, dict) else 0.0,
        yarn_orig_ctx=int(y.get("orig_ctx", 4096)) if isinstance(y, dict) else 0,
        yarn_truncate=int(bool(y.get("truncate", 0))) if isinstance(y, dict) else 0,
        attn_scale=float(attn.get("scale", 1.0 / np.sqrt(hd))),
        layer_sliding=sliding,
    )
    return f


# ------------------------------------------------------------------ writing
def _write_header(f, hdr: dict) -> int:
    blob = json.dumps(hdr).encode()
    f.write(struct.pack("<Q", len(blob)))
    f.write(blob)
    end = align64(8 + len(blob))
    f.write(b"\0" * (end - 8 - len(blob)))
    return end


def write_dense(path: str, spec: dict, tensors):
    """tensors: iterable of (name, dt, shape, data bytes, scale bytes)."""
    index, chunks, off = {}, [], 0
    for name, dt, shape, data, scales in tensors:
        e = {"dt": dt, "shape": list(shape), "off": off}
        chunks.append(data)
        chunks.append(b"\0" * (align64(len(data)) - len(data)))
        off = align64(off + len(data))
        if scales:
            e["soff"] = off
            chunks.append(scales)
            chunks.append(b"\0" * (align64(len(scales)) - len(scales)))
            off = align64(off + len(scales))
        index[name] = e
    with open(path, "wb") as f:
        _write_header(f, {"midge": 1, "kind": "dense", "spec": spec, "tensors": index})
        for c in chunks:
            f.write(c)


def write_experts(path: str, layout: ExpertLayout, blob: np.ndarray):
    with open(path, "wb") as f:
        _write_header(f, {"midge": 1, "kind": "experts", "dt": layout.dt})
        f.write(memoryview(np.ascontiguousarray(blob, dtype=np.uint8)))


# ---------------------------------------------------- synthetic model weights
def _pow2_scale(cols: int) -> float:
    """A power of two near 1/(127*sqrt(cols)): int8 rows of unit-ish gain."""
    return float(2.0 ** np.round(np.log2(1.0 / (127.0 * np.sqrt(cols)))))


def synth_q8r(rng, rows: int, cols: int):
    q = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
    s = np.full(rows, _pow2_scale(cols), dtype=np.float32)
    return q.tobytes(), s.tobytes()


def synth_g32(rng, rows: int, cols: int, dt: str):
    """4-bit data uniform over all 16 codes; mxfp4 scales 2^k with k uniform
    in [-8, -4] (f16 0x1C00..0x2C00); q4g32 scales uniform-ish f16 near 2^-6."""
    data = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    if dt == "mxfp4":
        k = rng.integers(-8, -3, size=(rows, cols // 32))
        sc = np.exp2(k).astype(np.float16)
    else:
        sc = (rng.uniform(0.5, 1.5, size=(rows, cols // 32)) * 2.0 ** -6).astype(np.float16)
    return data.tobytes(), sc.tobytes()


def synth_matrix(rng, dt: str, rows: int, cols: int):
    if dt == "q8r":
        return synth_q8r(rng, rows, cols)
    if dt in ("mxfp4", "q4g32"):
        return synth_g32(rng, rows, cols, dt)
    if dt == "f32":
        return (rng.standard_normal((rows, cols)) / np.sqrt(cols)).astype(np.float32).tobytes(), b""
    raise ValueError(dt)


def gpt_oss_spec(hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab, experts, top_k, ffn, window=128,
                 yarn_factor=32.0, orig_ctx=4096, theta=150000.0):
    """A gpt-oss-architecture spec (the shape of specs/gpt-oss-*.json)."""
    return {
        "arch": "gpt-oss", "hidden": hidden, "n_layers": n_layers, "n_heads": n_heads, "n_kv_heads": n_kv_heads,
        "head_dim": head_dim, "vocab": vocab, "norm_eps": 1e-05,
        "moe": {"experts": experts, "top_k": top_k, "ffn": ffn, "act": "swiglu_clamp", "alpha": 1.702,
                "limit": 7.0},
        "attn": {"layer_types": ["sliding_attention" if i % 2 == 0 else "full_attention" for i in range(n_layers)],
                 "sliding_window": window, "sinks": True, "scale": 1.0 / float(np.sqrt(head_dim))},
        "rope": {"theta": theta, "yarn": {"factor": yarn_factor, "beta_fast": 32.0, "beta_slow": 1.0,
                                          "orig_ctx": orig_ctx, "truncate": False}},
    }


def qwen3_spec(hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab, experts, top_k, ffn, theta=1e6):
    return {
        "arch": "qwen3-moe", "hidden": hidden, "n_layers": n_layers, "n_heads": n_heads, "n_kv_heads": n_kv_heads,
        "head_dim": head_dim, "vocab": vocab, "norm_eps": 1e-06,
        "moe": {"experts": experts, "top_k": top_k, "ffn": ffn, "act": "swiglu", "router_norm": 0},
        "attn": {"layer_types": ["full_attention"] * n_layers, "sliding_window": 0, "sinks": False,
                 "qk_norm": True, "scale": 1.0 / float(np.sqrt(head_dim))},
        "rope": {"theta": theta},
    }


# The benchmark configs ([2], [3], [4]) as specs.
CONFIGS = {
    "c1_tiny": dict(kind="gpt-oss", hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, vocab=1024,
                    experts=8, top_k=2, ffn=256, expert_dt="mxfp4"),
    "c3_20b": dict(kind="gpt-oss", hidden=2880, n_layers=24, n_heads=64, n_kv_heads=8, head_dim=64, vocab=201088,
                   experts=32, top_k=4, ffn=2880, expert_dt="mxfp4"),
    "c4_120b": dict(kind="gpt-oss", hidden=2880, n_layers=36, n_heads=64, n_kv_heads=8, head_dim=64, vocab=201088,
                    experts=128, top_k=4, ffn=2880, expert_dt="mxfp4"),
    "c5_qwen3": dict(kind="qwen3", hidden=2048, n_layers=48, n_heads=32, n_kv_heads=4, head_dim=128, vocab=151936,
                     experts=128, top_k=8, ffn=768, expert_dt="q8r"),
}


def config_spec(name: str, n_layers: int | None = None) -> tuple[dict, str]:
    c = dict(CONFIGS[name])
    if n_layers is not None:
        c["n_layers"] = n_layers
    kind, edt = c.pop("kind"), c.pop("expert_dt")
    spec = gpt_oss_spec(**c) if kind == "gpt-oss" else qwen3_spec(**c)
    return spec, edt


def dense_tensors(spec: dict, rng, dense_dt: str = "q8r"):
    """Yield (name, dt, shape, data, scales) for a random trunk of `spec`, in
    the order and with the names of docs/ADDING_MODELS.md."""
    H, V = spec["hidden"], spec["vocab"]
    nh, nkv, hd = spec["n_heads"], spec["n_kv_heads"], spec["head_dim"]
    E = spec["moe"]["experts"]

    def vec(name, n, kind):
        if kind == "norm":
            v = 1.0 + 0.1 * rng.standard_normal(n)
        elif kind == "sink":
            v = rng.standard_normal(n)
        else:
            v = 0.1 * rng.standard_normal(n)
        return (name, "f32", [n], v.astype(np.float32).tobytes(), b"")

    def mat(name, rows, cols, dt=dense_dt):
        d, s = synth_matrix(rng, dt, rows, cols)
        return (name, dt, [rows, cols], d, s)

    yield mat("embed", V, H)
    yield mat("lm_head", V, H)
    yield vec("final_norm", H, "norm")
    for i in range(spec["n_layers"]):
        p = f"L{i}."
        yield vec(p + "attn.norm", H, "norm")
        yield vec(p + "mlp.norm", H, "norm")
        yield mat(p + "attn.q", nh * hd, H)
        yield vec(p + "attn.q_b", nh * hd, "bias")
        yield mat(p + "attn.k", nkv * hd, H)
        yield vec(p + "attn.k_b", nkv * hd, "bias")
        yield mat(p + "attn.v", nkv * hd, H)
        yield vec(p + "attn.v_b", nkv * hd, "bias")
        yield mat(p + "attn.o", H, nh * hd)
        yield vec(p + "attn.o_b", H, "bias")
        if spec["attn"].get("sinks"):
            yield vec(p + "attn.sinks", nh, "sink")
        if spec["attn"].get("qk_norm"):
            yield vec(p + "attn.q_norm", hd, "norm")
            yield vec(p + "attn.k_norm", hd, "norm")
        rw = (rng.standard_normal((E, H)) / np.sqrt(H)).astype(np.float32)
        yield (p + "router.w", "f32", [E, H], rw.tobytes(), b"")
        yield vec(p + "router.b", E, "bias")


def expert_blob(layout: ExpertLayout, rng) -> np.ndarray:
    """Random experts in the deterministic layout (biases N(0, 0.1))."""
    blob = np.zeros(layout.total, dtype=np.uint8)
    for layer in range(layout.n_layers):
        for e in range(layout.n_experts):
            for m in ExpertLayout.MATS:
                r, c = layout.rows[m], layout.cols[m]
                d, s = synth_matrix(rng, layout.dt, r, c)
                o = layout.offset(layer, e, m, "data")
                blob[o:o + len(d)] = np.frombuffer(d, np.uint8)
                if s:
                    o = layout.offset(layer, e, m, "scales")
                    blob[o:o + len(s)] = np.frombuffer(s, np.uint8)
                b = (0.1 * rng.standard_normal(r)).astype(np.float32).tobytes()
                o = layout.offset(layer, e, m, "bias")
                blob[o:o + len(b)] = np.frombuffer(b, np.uint8)
    return blob


def write_synthetic_model(outdir: str, spec: dict, expert_dt: str, seed: int = 0, dense_dt: str = "q8r"):
    """Write dense.midge + experts.midge of a seeded random model."""
    os.makedirs(outdir, exist_ok=True)
    rng = np.random.default_rng(seed)
    write_dense(os.path.join(outdir, "dense.midge"), spec, list(dense_tensors(spec, rng, dense_dt)))
    lay = ExpertLayout(expert_dt, spec["hidden"], spec["moe"]["ffn"], spec["moe"]["experts"], spec["n_layers"])
    write_experts(os.path.join(outdir, "experts.midge"), lay, expert_blob(lay, rng))
    with open(os.path.join(outdir, "spec.json"), "w") as f:
        json.dump(spec, f, indent=2)
    return outdir
