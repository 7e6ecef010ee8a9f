"""Python binding of the gten B200 library (lib/libgten_b200.so) through its C ABI.

The entry points mirror the reference's operator API (namespace gten::ops, src/gten/ops.h) and
its model / greedy-sampler interface (src/gten/abc.h, src/gten/sampler.cpp), with the same
argument meaning: every op computes rows [start_pos, n_ctx) into a caller-owned output.

Tensors are ``GT`` values: a device buffer (a torch CUDA tensor, or a raw device pointer) plus a
gten dtype and a logical shape in elements. Quantized tensors use the reference block layout
(Q8: 34-byte blocks of fp16 delta + 32 int8; Q4: 18-byte blocks), stored in uint8 buffers.

Errors: a non-zero status from the library raises ``GtenError`` with the library's message (the
reference prints and exits instead). The library must be built (``build.py``); there is no CPU
fallback, and using this module without the built library raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "lib", "libgten_b200.so")

I32, F16, F32, Q8, Q4 = 0, 1, 2, 3, 4
QBLK = 32

TINYLLAMA, ZEPHYR, MINICPM, OPENELM_SM, OPENELM_MD, OPENELM_LG, CUSTOM = range(7)


class GtenError(RuntimeError):
    pass


class gtn_tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_int32), ("ndim", C.c_int32),
                ("shape", C.c_int32 * 3), ("strides", C.c_int32 * 3)]


_lib = None


def lib() -> C.CDLL:
    """Loads lib/libgten_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise GtenError(f"{LIB_PATH} is missing: build it with nanochatllms.cpp_b200/build.py")
        L = C.CDLL(LIB_PATH)
        L.gtn_last_error.restype = C.c_char_p
        L.gtn_kernel_launches.restype = C.c_ulonglong
        L.gtn_model_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]
        L.gtn_model_free.argtypes = [C.c_void_p]
        L.gtn_model_n_vocab.argtypes = [C.c_void_p]
        L.gtn_model_load.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
        L.gtn_model_load_file.argtypes = [C.c_void_p, C.c_char_p]
        L.gtn_slot_start.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int32)]
        L.gtn_slots_step.argtypes = [C.c_void_p, C.c_void_p]
        L.gtn_slot_finish.argtypes = [C.c_void_p, C.c_int]
        L.gtn_model_logits.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.gtn_model_generate.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.gtn_model_generate_device.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.gtn_model_generate_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.gtn_model_stream.argtypes = [C.c_void_p]
        L.gtn_model_stream.restype = C.c_void_p
        L.gtn_model_check.argtypes = [C.c_void_p]
        for name in ("gtn_pack_q8", "gtn_pack_q4", "gtn_quantize_q8_rows"):
            getattr(L, name).argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p]
        L.gtn_argmax.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.gtn_rng_create.argtypes = [C.c_uint32, C.POINTER(C.c_void_p)]
        L.gtn_rng_free.argtypes = [C.c_void_p]
        L.gtn_sample_topk.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.gtn_model_generate_topk.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_int,
                                              C.c_void_p, C.c_void_p]
        _lib = L
    return _lib


def kernel_launches() -> int:
    """Kernels launched by the library so far in this process."""
    return int(lib().gtn_kernel_launches())


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().gtn_last_error().decode(errors="replace")
        raise GtenError(f"{what} failed (status {rc}): {msg}")


def row_bytes(dt: int, n: int) -> int:
    if dt == Q8:
        return (n + QBLK - 1) // QBLK * 34
    if dt == Q4:
        return n // QBLK * 18
    if dt == F16:
        return 2 * n
    return 4 * n


def nbytes(dt: int, shape: Sequence[int]) -> int:
    rows = 1
    for s in shape[:-1]:
        rows *= s
    return rows * row_bytes(dt, shape[-1])


def _ptr(buf) -> int:
    if hasattr(buf, "data_ptr"):
        return buf.data_ptr()
    return int(buf)


def _stream(stream):
    if stream is not None:
        if hasattr(stream, "cuda_stream"):
            return C.c_void_p(stream.cuda_stream)
        return C.c_void_p(int(stream))
    try:
        import torch
        if torch.cuda.is_available():
            return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    except Exception:
        pass
    return C.c_void_p(0)


@dataclass
class GT:
    """A gten tensor view: device buffer + dtype + logical shape (elements), contiguous rows."""
    buf: object
    dtype: int
    shape: tuple

    def desc(self) -> gtn_tensor:
        t = gtn_tensor()
        t.data = _ptr(self.buf)
        t.dtype = self.dtype
        t.ndim = len(self.shape)
        st = [1] * len(self.shape)
        for i in range(len(self.shape) - 2, -1, -1):
            st[i] = st[i + 1] * self.shape[i + 1]
        for i, s in enumerate(self.shape):
            t.shape[i] = s
            t.strides[i] = st[i]
        return t


def _d(t):
    return None if t is None else C.byref(t.desc())


# ---- gten::ops (src/gten/ops.h) -------------------------------------------------------------
def matmul_2d(x: GT, w: GT, out: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_matmul_2d(_d(x), _d(w), _d(out), start_pos, _stream(stream)), "matmul_2d")


def qkv_attn(q: GT, k: GT, v: GT, qk, qkv: GT, max_ctx: int, start_pos: int = 0, stream=None):
    _check(lib().gtn_qkv_attn(_d(q), _d(k), _d(v), _d(qk), _d(qkv), max_ctx, start_pos, _stream(stream)), "qkv_attn")


def rms_norm(inp: GT, weight: GT, out: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_rms_norm(_d(inp), _d(weight), _d(out), start_pos, _stream(stream)), "rms_norm")


def layer_norm(inp: GT, weight: GT, bias: GT, out: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_layer_norm(_d(inp), _d(weight), _d(bias), _d(out), start_pos, _stream(stream)), "layer_norm")


def rotary_emb(inp: GT, out: GT, d_head: int, rope_pct: float, start_pos: int = 0, stream=None):
    _check(lib().gtn_rotary_emb(_d(inp), _d(out), d_head, C.c_float(rope_pct), start_pos, _stream(stream)),
           "rotary_emb")


def silu(inp: GT, out: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_silu(_d(inp), _d(out), start_pos, _stream(stream)), "silu")


def silu_inplace(inp: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_silu_inplace(_d(inp), start_pos, _stream(stream)), "silu_inplace")


def multiply(a: GT, b: GT, out: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_multiply(_d(a), _d(b), _d(out), start_pos, _stream(stream)), "multiply")


def multiply_inplace(a: GT, b: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_multiply_inplace(_d(a), _d(b), start_pos, _stream(stream)), "multiply_inplace")


def add(a: GT, b: GT, out: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_add(_d(a), _d(b), _d(out), start_pos, _stream(stream)), "add")


def scale(inp: GT, scaler: float, start_pos: int = 0, stream=None):
    _check(lib().gtn_scale(_d(inp), C.c_float(scaler), start_pos, _stream(stream)), "scale")


def bias_add_inplace(inp: GT, bias: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_bias_add_inplace(_d(inp), _d(bias), start_pos, _stream(stream)), "bias_add_inplace")


def token_embed(weight: GT, tokens: GT, out: GT, start_pos: int = 0, stream=None):
    _check(lib().gtn_token_embed(_d(weight), _d(tokens), _d(out), start_pos, _stream(stream)), "token_embed")


# ---- quantization -------------------------------------------------------------------------
def pack_q8(w, out, stream=None):
    """w: device fp32 [rows, cols]; out: device uint8 buffer of rows*cols/32*34 bytes."""
    rows, cols = w.shape
    _check(lib().gtn_pack_q8(_ptr(w), rows, cols, _ptr(out), _stream(stream)), "pack_q8")


def pack_q4(w, out, stream=None):
    rows, cols = w.shape
    _check(lib().gtn_pack_q4(_ptr(w), rows, cols, _ptr(out), _stream(stream)), "pack_q4")


def quantize_q8_rows(x, out, stream=None):
    rows, cols = x.shape
    _check(lib().gtn_quantize_q8_rows(_ptr(x), rows, cols, _ptr(out), _stream(stream)), "quantize_q8_rows")


def argmax(logits, out_index, stream=None):
    _check(lib().gtn_argmax(_ptr(logits), logits.numel(), _ptr(out_index), _stream(stream)), "argmax")


class Rng:
    """std::mt19937(seed) state on the current CUDA device, for sample_topk (the reference seeds from
    std::random_device, sampler.cpp:70-71)."""

    def __init__(self, seed: int):
        self._h = C.c_void_p()
        _check(lib().gtn_rng_create(C.c_uint32(seed & 0xFFFFFFFF), C.byref(self._h)), "rng_create")

    def close(self):
        if self._h:
            lib().gtn_rng_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sample_topk(logits, temp: float, top_k: int, rng: Rng, out_index, stream=None):
    """One top-k / temperature draw of topk_sample (sampler.cpp:90-128) from device fp32 logits into
    a device int32 tensor; advances rng."""
    _check(lib().gtn_sample_topk(_ptr(logits), logits.numel(), C.c_float(temp), top_k, rng._h, _ptr(out_index),
                                 _stream(stream)), "sample_topk")


# ---- models (src/gten/abc.h) ----------------------------------------------------------------
class Model:
    """A model of one of the reference's families on the current CUDA device.

    ``Model(kind, wdtype, max_ctx)`` mirrors the reference constructors (e.g. TinyLLama(n_ctx,
    dtype), tinyllama.h:52); ``load(image)`` is load_from_ckpt on a .gten byte image;
    ``logits`` is Model::logits; ``generate`` is greedy_sample without tokenization."""

    def __init__(self, kind: int, wdtype: int, max_ctx: int, max_batch: int = 1, dims=None):
        self._h = C.c_void_p()
        arr = None
        if dims is not None:
            arr = (C.c_int32 * 7)(*dims)
        _check(lib().gtn_model_create(kind, wdtype, max_ctx, max_batch, arr, C.byref(self._h)), "model_create")
        self.max_batch = max_batch
        self.max_ctx = max_ctx
        self.n_vocab = lib().gtn_model_n_vocab(self._h)

    def load(self, image) -> None:
        """image: the .gten file as bytes or a uint8 numpy array (host memory)."""
        import numpy as np
        arr = np.frombuffer(image, np.uint8) if isinstance(image, (bytes, bytearray, memoryview)) else image
        arr = np.ascontiguousarray(arr, np.uint8)
        _check(lib().gtn_model_load(self._h, arr.ctypes.data, arr.size), "model_load")

    def load_file(self, path: str) -> None:
        """load_from_ckpt from a .gten file path."""
        _check(lib().gtn_model_load_file(self._h, os.fsencode(path)), "model_load_file")

    def logits(self, tokens, start_pos: int):
        import numpy as np
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.n_vocab, np.float32)
        _check(lib().gtn_model_logits(self._h, t.ctypes.data, t.size, start_pos, out.ctypes.data), "model_logits")
        return out

    def generate(self, prompt, n_gen: int):
        import numpy as np
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen, np.int32)
        _check(lib().gtn_model_generate(self._h, p.ctypes.data, p.size, n_gen, out.ctypes.data), "model_generate")
        return out

    def generate_topk(self, prompt, n_gen: int, temp: float, top_k: int, rng: "Rng"):
        """topk_sample (sampler.cpp:63-143) without tokenization: n_gen ids drawn with rng."""
        import numpy as np
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen, np.int32)
        _check(lib().gtn_model_generate_topk(self._h, p.ctypes.data, p.size, n_gen, C.c_float(temp), top_k, rng._h,
                                             out.ctypes.data), "model_generate_topk")
        return out

    # ---- continuous batching (gtn_slot_*)
    def slot_start(self, prompt):
        """Prefills prompt into a free slot; returns (slot, first greedy id)."""
        import numpy as np
        p = np.ascontiguousarray(prompt, np.int32)
        slot, first = C.c_int(), C.c_int32()
        _check(lib().gtn_slot_start(self._h, p.ctypes.data, p.size, C.byref(slot), C.byref(first)), "slot_start")
        return slot.value, first.value

    def slots_step(self):
        """One decode step of every busy slot; returns max_batch ids (-1 for idle slots)."""
        import numpy as np
        out = np.empty(self.max_batch, np.int32)
        _check(lib().gtn_slots_step(self._h, out.ctypes.data), "slots_step")
        return out

    def slot_finish(self, slot: int) -> None:
        _check(lib().gtn_slot_finish(self._h, slot), "slot_finish")

    def generate_batch(self, prompts, n_gen: int):
        """prompts: [batch, n_prompt] int32 (host); returns [batch, n_gen] greedy ids."""
        import numpy as np
        p = np.ascontiguousarray(prompts, np.int32)
        out = np.zeros((p.shape[0], n_gen), np.int32)
        _check(lib().gtn_model_generate_batch(self._h, p.ctypes.data, p.shape[0], p.shape[1], n_gen, out.ctypes.data),
               "model_generate_batch")
        return out

    def generate_device(self, prompt_dev, n_gen: int, out_dev) -> None:
        """Greedy decode with device int32 tensors; asynchronous on ``self.stream_ptr``."""
        _check(lib().gtn_model_generate_device(self._h, _ptr(prompt_dev), prompt_dev.numel(), n_gen, _ptr(out_dev)),
               "model_generate_device")

    @property
    def stream_ptr(self) -> int:
        return lib().gtn_model_stream(self._h) or 0

    def check(self) -> None:
        _check(lib().gtn_model_check(self._h), "model_check")

    def close(self):
        if self._h:
            lib().gtn_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
