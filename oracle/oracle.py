"""Test infrastructure only: ctypes bindings for the CPU oracle and the reference harness.

* ``Oracle`` wraps ``oracle/_build/libgtenoracle.so``, the C restatement of the reference's gten
  compute path (``oracle/gten_oracle.c``; each function cites the reference file:line it
  restates).
* ``Reference`` wraps ``oracle/_ref/libgtenref.so``: the UNMODIFIED reference sources
  (iangitonga/nanochatllms.cpp ``src/gten`` and model files) compiled with
  ``oracle/ref_harness.cpp`` by ``oracle/build_ref.sh``.

Only tests, ``__graft_entry__.smoke()`` and bench.py's cpu-baseline / reference arms use this
module, and only as the checker or the timed CPU baseline; the product never imports it.

Both expose the same op-level calls on numpy buffers, so a test can run one case through either.
dtype codes follow gten::Dtype (src/gten/gten_types.h:20-26): 0 Int32, 1 Float16, 2 Float32,
3 Qint8, 4 Qint4.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
I32, F16, F32, Q8, Q4 = 0, 1, 2, 3, 4
QBLK = 32


def row_bytes(dt: int, n: int) -> int:
    if dt == Q8:
        return (n + QBLK - 1) // QBLK * 34
    if dt == Q4:
        return n // QBLK * 18
    if dt == F16:
        return 2 * n
    return 4 * n


def reference_dir() -> str | None:
    """The reference checkout to build or read from: $GTEN_REFERENCE_DIR, else the
    ``reference_path`` that BASELINE.json (repository root) records; None when neither names an
    existing checkout (e.g. on a GPU box, which only uses the prebuilt oracle/_ref library)."""
    d = os.environ.get("GTEN_REFERENCE_DIR")
    if not d:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                d = json.load(f).get("reference_path")
        except (OSError, ValueError):
            d = None
    return d if d and os.path.isdir(os.path.join(d, "src", "gten")) else None


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class _Lib:
    prefix = ""

    def __init__(self, path: str):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)

    def f(self, name):
        return getattr(self.lib, self.prefix + name)

    # ---- op-level (same argument order in both libraries) ----
    def q8_quantize_row(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(row_bytes(Q8, x.size), np.uint8)
        self.f("q8_quantize_row")(_p(x), _p(out), C.c_int(x.size))
        return out

    def matmul_2d(self, x, xdt, n_ctx, n_embd, w, wdt, n_out, odt, start_pos=0, out_1d=False, **kw):
        out = np.zeros(row_bytes(odt, n_out) * (1 if out_1d else n_ctx), np.uint8)
        args = [_p(x), C.c_int(xdt), C.c_int(n_ctx), C.c_int(n_embd), _p(w), C.c_int(wdt), C.c_int(n_out),
                _p(out), C.c_int(odt), C.c_int(start_pos), C.c_int(int(out_1d))]
        if self.prefix == "or_":
            args.append(C.c_int(kw.get("order", 0)))
        self.f("matmul_2d")(*args)
        return out

    def rms_norm(self, x, dt, n_ctx, n_embd, w, start_pos=0):
        out = np.zeros(row_bytes(dt, n_embd) * n_ctx, np.uint8)
        self.f("rms_norm")(_p(x), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_embd), _p(w), _p(out), C.c_int(start_pos))
        return out

    def rms_norm_3d(self, x, dt, n_ctx, n_heads, d_head, w, start_pos=0):
        out = np.zeros(row_bytes(dt, n_heads * d_head) * n_ctx, np.uint8)
        self.f("rms_norm_3d")(_p(x), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_heads), C.c_int(d_head), _p(w),
                              _p(out), C.c_int(start_pos))
        return out

    def layer_norm(self, x, dt, n_ctx, n_embd, w, b, start_pos=0):
        out = np.zeros(row_bytes(dt, n_embd) * n_ctx, np.uint8)
        self.f("layer_norm")(_p(x), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_embd), _p(w), _p(b), _p(out),
                             C.c_int(start_pos))
        return out

    def rotary_emb(self, x, dt, n_ctx, n_embd, d_head, rope_pct, start_pos=0):
        inp = np.array(x, copy=True)
        out = np.array(x, copy=True)
        self.f("rotary_emb")(_p(inp), _p(out), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_embd), C.c_int(d_head),
                             C.c_float(rope_pct), C.c_int(start_pos))
        return out

    def silu(self, x, dt, n_ctx, n_embd, start_pos=0):
        out = np.array(x, copy=True)
        self.f("silu")(_p(x), _p(out), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_embd), C.c_int(start_pos))
        return out

    def multiply(self, a, b, dt, n_ctx, n_embd, start_pos=0):
        out = np.array(a, copy=True)
        self.f("multiply")(_p(a), _p(b), _p(out), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_embd), C.c_int(start_pos))
        return out

    def add(self, a, b, dt, n_ctx, n_embd, start_pos=0):
        out = np.array(a, copy=True)
        self.f("add")(_p(a), _p(b), _p(out), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_embd), C.c_int(start_pos))
        return out

    def scale(self, x, dt, n_ctx, n_embd, s, start_pos=0):
        out = np.array(x, copy=True)
        self.f("scale")(_p(out), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_embd), C.c_float(s), C.c_int(start_pos))
        return out

    def bias_add_inplace(self, x, dt, n_ctx, n_embd, bias, start_pos=0):
        out = np.array(x, copy=True)
        self.f("bias_add_inplace")(_p(out), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_embd), _p(bias),
                                   C.c_int(start_pos))
        return out

    def token_embed(self, w, wdt, n_vocab, n_embd, tokens, odt, start_pos=0):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(row_bytes(odt, n_embd) * tokens.size, np.uint8)
        self.f("token_embed")(_p(w), C.c_int(wdt), C.c_int(n_vocab), C.c_int(n_embd), _p(tokens),
                              C.c_int(tokens.size), _p(out), C.c_int(odt), C.c_int(start_pos))
        return out


class Oracle(_Lib):
    prefix = "or_"

    def __init__(self, path: str | None = None):
        super().__init__(path or os.path.join(HERE, "_build", "libgtenoracle.so"))
        L = self.lib
        L.or_fp32_to_fp16.restype = C.c_uint16
        L.or_fp16_to_fp32.restype = C.c_float
        L.or_vec_dot.restype = C.c_float
        L.or_model_new.restype = C.c_void_p
        L.or_model_free.argtypes = [C.c_void_p]
        L.or_model_load.argtypes = [C.c_void_p, C.c_void_p, C.c_long]
        L.or_model_logits.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.or_model_greedy.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.or_model_n_vocab.argtypes = [C.c_void_p]

    def pack_q8(self, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        out = np.zeros(rows * row_bytes(Q8, cols), np.uint8)
        self.lib.or_pack_q8(_p(w), C.c_int(rows), C.c_int(cols), _p(out))
        return out

    def pack_q4(self, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        out = np.zeros(rows * row_bytes(Q4, cols), np.uint8)
        self.lib.or_pack_q4(_p(w), C.c_int(rows), C.c_int(cols), _p(out))
        return out

    def read_row(self, row: np.ndarray, dt: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        self.lib.or_read_row(_p(np.ascontiguousarray(row)), C.c_int(dt), _p(out), C.c_int(n))
        return out

    def dequant(self, buf: np.ndarray, dt: int, rows: int, n: int) -> np.ndarray:
        rb = row_bytes(dt, n)
        return np.stack([self.read_row(buf[r * rb:(r + 1) * rb], dt, n) for r in range(rows)])

    def qkv_attn(self, q, k, v, dt, n_ctx, n_head, q_dim, kv_dim, start_pos=0, **_):
        out = np.zeros(row_bytes(dt, q_dim) * n_ctx, np.uint8)
        self.lib.or_qkv_attn(_p(q), _p(k), _p(v), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_head), C.c_int(q_dim),
                             C.c_int(kv_dim), _p(out), C.c_int(start_pos))
        return out

    def argmax(self, x: np.ndarray) -> int:
        x = np.ascontiguousarray(x, dtype=np.float32)
        return self.lib.or_argmax(_p(x), C.c_int(x.size))


class OracleModel:
    """The oracle's model wiring; ``image`` is a complete .gten file as bytes/uint8 array."""

    def __init__(self, orc: Oracle, kind: int, wdt: int, n_ctx: int, image, dims=None):
        self.o = orc
        self.dims = np.zeros(7, np.int32) if dims is None else np.asarray(dims, np.int32)
        self.h = orc.lib.or_model_new(C.c_int(kind), C.c_int(wdt), C.c_int(n_ctx), _p(self.dims))
        self.image = np.frombuffer(image, np.uint8) if not isinstance(image, np.ndarray) else image
        rc = orc.lib.or_model_load(self.h, _p(self.image), C.c_long(self.image.size))
        if rc != 0:
            raise ValueError(f"or_model_load failed: {rc}")
        self.n_vocab = orc.lib.or_model_n_vocab(self.h)

    def logits(self, tokens, start_pos):
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.n_vocab, np.float32)
        self.o.lib.or_model_logits(self.h, _p(t), C.c_int(t.size), C.c_int(start_pos), _p(out))
        return out

    def greedy(self, prompt, n_gen):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen, np.int32)
        rc = self.o.lib.or_model_greedy(self.h, _p(p), C.c_int(p.size), C.c_int(n_gen), _p(out))
        if rc != 0:
            raise RuntimeError("or_model_greedy failed")
        return out

    def __del__(self):
        try:
            self.o.lib.or_model_free(self.h)
        except Exception:
            pass


class Reference(_Lib):
    prefix = "ref_"

    def __init__(self, path: str | None = None):
        super().__init__(path or os.path.join(HERE, "_ref", "libgtenref.so"))
        L = self.lib
        L.ref_fp32_to_fp16.restype = C.c_uint16
        L.ref_fp16_to_fp32.restype = C.c_float
        L.ref_model_new.restype = C.c_void_p
        L.ref_model_free.argtypes = [C.c_void_p]
        L.ref_model_load.argtypes = [C.c_void_p, C.c_char_p]
        L.ref_model_logits.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.ref_model_greedy.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]

    def qkv_attn(self, q, k, v, dt, n_ctx, n_head, q_dim, kv_dim, start_pos=0, max_ctx=None):
        out = np.zeros(row_bytes(dt, q_dim) * n_ctx, np.uint8)
        max_ctx = max_ctx or max(2 * n_ctx, 64)
        self.lib.ref_qkv_attn(_p(q), _p(k), _p(v), C.c_int(dt), C.c_int(n_ctx), C.c_int(n_head), C.c_int(q_dim),
                              C.c_int(kv_dim), C.c_int(max_ctx), _p(out), C.c_int(start_pos))
        return out


class SamplerOracle(_Lib):
    """oracle/sampler_oracle.cpp: the reference's top-k sampling step with std::mt19937(seed)."""

    def __init__(self, path: str | None = None):
        super().__init__(path or os.path.join(HERE, "_build", "libsampleroracle.so"))
        self.lib.or_topk_sample.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_uint32, C.c_int,
                                            C.c_void_p]

    def topk_sample(self, logits: np.ndarray, temp: float, top_k: int, seed: int) -> np.ndarray:
        """logits [draws, n] fp32: one draw per row, one generator for all rows."""
        x = np.ascontiguousarray(np.atleast_2d(logits), np.float32)
        out = np.zeros(x.shape[0], np.int32)
        rc = self.lib.or_topk_sample(_p(x), x.shape[1], C.c_float(temp), top_k, C.c_uint32(seed), x.shape[0], _p(out))
        if rc != 0:
            raise ValueError("or_topk_sample: bad arguments")
        return out

    def generator(self, seed: int) -> "OracleSampler":
        return OracleSampler(self, seed)


class OracleSampler:
    """One std::mt19937(seed) that persists across topk_sample steps (a decode loop)."""

    def __init__(self, so: SamplerOracle, seed: int):
        self.lib = so.lib
        self.lib.or_sampler_new.restype = C.c_void_p
        self.lib.or_sampler_new.argtypes = [C.c_uint32]
        self.lib.or_sampler_step.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_int]
        self.lib.or_sampler_free.argtypes = [C.c_void_p]
        self.h = self.lib.or_sampler_new(C.c_uint32(seed))

    def step(self, logits: np.ndarray, temp: float, top_k: int) -> int:
        x = np.ascontiguousarray(logits, np.float32).ravel()
        r = self.lib.or_sampler_step(self.h, _p(x), x.size, C.c_float(temp), top_k)
        if r < 0:
            raise ValueError("or_sampler_step: bad arguments")
        return int(r)

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.or_sampler_free(self.h)
            self.h = None


class ReferenceModel:
    def __init__(self, ref: Reference, kind: int, wdt: int, n_ctx: int, path: str, n_vocab: int):
        self.r = ref
        self.h = ref.lib.ref_model_new(C.c_int(kind), C.c_int(wdt), C.c_int(n_ctx))
        if ref.lib.ref_model_load(self.h, path.encode()) != 0:
            raise FileNotFoundError(path)
        self.n_vocab = n_vocab

    def logits(self, tokens, start_pos):
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.n_vocab, np.float32)
        self.r.lib.ref_model_logits(self.h, _p(t), C.c_int(t.size), C.c_int(start_pos), _p(out))
        return out

    def greedy(self, prompt, n_gen, margins=False):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen, np.int32)
        mg = np.zeros(n_gen, np.float32) if margins else None
        self.r.lib.ref_model_greedy(self.h, _p(p), C.c_int(p.size), C.c_int(n_gen), _p(out), _p(mg))
        return (out, mg) if margins else out

    def __del__(self):
        try:
            self.r.lib.ref_model_free(self.h)
        except Exception:
            pass
