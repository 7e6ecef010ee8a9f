"""The .gten checkpoint format and seeded synthetic checkpoints.

Format (the reference's converters write it, src/tinyllama/tinyllama_to_gten.py:94-148 and
siblings; the model files read it, src/gten/utils.cpp:29-61): int64 magic 0x454c49464e455447,
then per tensor: int32 name length + name, int32 name length + name again, int32 payload size,
payload (fp16 values, or Q8/Q4 blocks row-major). Records follow each model's load order
(tinyllama.cpp:195-251, zephyr.cpp:79-150, minicpm.cpp:113-166, openelm.cpp:201-262).

Synthetic checkpoints: matrices are N(0, 0.02) fp32 from ``torch.Generator().manual_seed(seed +
record_index)``, packed by a caller-supplied packer (the CUDA packer or a CPU one; both are
bit-exact with the reference's Python q8_quantize / q4_quantize); norm gains are 1 and biases 0.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import Callable, List, Optional

import numpy as np

from . import F16, Q4, Q8, row_bytes

MAGIC = 0x454C49464E455447

ELM = {
    3: dict(d=1280, qh=[12, 12, 12, 12, 12, 16, 16, 16, 16, 16, 16, 16, 20, 20, 20, 20],
            kv=[3, 3, 3, 3, 3, 4, 4, 4, 4, 4, 4, 4, 5, 5, 5, 5],
            ff=[768, 1024, 1280, 1536, 1792, 2048, 2560, 2816, 3072, 3328, 3584, 3840, 4352, 4608, 4864, 5120]),
    4: dict(d=1536, qh=[12, 12, 12, 16, 16, 16, 16, 16, 16, 16, 20, 20, 20, 20, 20, 20, 24, 24, 24, 24],
            kv=[3, 3, 3, 4, 4, 4, 4, 4, 4, 4, 5, 5, 5, 5, 5, 5, 6, 6, 6, 6],
            ff=[768, 1024, 1280, 1536, 1792, 2304, 2560, 2816, 3072, 3328, 3584, 3840, 4096, 4352, 4608, 5120,
                5376, 5632, 5888, 6144]),
    5: dict(d=2048, qh=[16, 16, 16, 20, 20, 20, 20, 20, 20, 20, 24, 24, 24, 24, 24, 24, 24, 24, 28, 28, 28, 28, 28,
                        28, 32, 32, 32, 32],
            kv=[4, 4, 4, 5, 5, 5, 5, 5, 5, 5, 6, 6, 6, 6, 6, 6, 6, 6, 7, 7, 7, 7, 7, 7, 8, 8, 8, 8],
            ff=[1024, 1280, 1536, 1792, 2048, 2304, 2560, 2816, 3072, 3328, 3584, 3840, 4096, 4608, 4608, 5120, 5376,
                5632, 5888, 6144, 6400, 6656, 6912, 7168, 7424, 7680, 7936, 8192]),
}


@dataclass
class Arch:
    family: int  # 0 tinyllama-like, 1 zephyr-like, 2 minicpm-like, 3 openelm
    n_vocab: int
    d: int
    layers: List[tuple]  # per layer (q_heads, kv_heads, ffn)
    d_head: int = 64


def arch(kind: int, dims: Optional[List[int]] = None) -> Arch:
    """Architectures of tinyllama.h:12-24, zephyr.h:10-23, minicpm.h:9-24, openelm.h:26-51."""
    if kind == 0:
        return Arch(0, 32003, 2048, [(32, 4, 5632)] * 22)
    if kind == 1:
        return Arch(1, 100352, 2048, [(32, 32, 5632)] * 24)
    if kind == 2:
        return Arch(2, 122753, 2304, [(36, 36, 5760)] * 40)
    if kind in ELM:
        e = ELM[kind]
        return Arch(3, 32000, e["d"], list(zip(e["qh"], e["kv"], e["ff"])))
    v, d, nl, nh, nkv, nff, fam = dims
    return Arch(fam, v, d, [(nh, nkv, nff)] * nl)


def records(a: Arch):
    """Yields (name, kind, shape) in load order; kind is 'w' (packed matrix), 'g' (norm gain) or
    'b' (bias)."""
    d, dh = a.d, a.d_head
    yield "model.embed_tokens.weight", "w", (a.n_vocab, d)
    for i, (qh, kv, ff) in enumerate(a.layers):
        p = f"model.layers.{i}"
        qd, kvd = qh * dh, kv * dh
        yield f"{p}.self_attn.q_proj.weight", "w", (qd, d)
        if a.family == 1:
            yield f"{p}.self_attn.q_proj.bias", "b", (qd,)
        yield f"{p}.self_attn.k_proj.weight", "w", (kvd, d)
        if a.family == 1:
            yield f"{p}.self_attn.k_proj.bias", "b", (kvd,)
        yield f"{p}.self_attn.v_proj.weight", "w", (kvd, d)
        if a.family == 1:
            yield f"{p}.self_attn.v_proj.bias", "b", (kvd,)
        yield f"{p}.self_attn.o_proj.weight", "w", (d, qd)
        yield f"{p}.mlp.gate_proj.weight", "w", (ff, d)
        yield f"{p}.mlp.up_proj.weight", "w", (ff, d)
        yield f"{p}.mlp.down_proj.weight", "w", (d, ff)
        if a.family == 3:
            yield f"{p}.attn.q_norm.weight", "g", (dh,)
            yield f"{p}.attn.k_norm.weight", "g", (dh,)
        yield f"{p}.input_layernorm.weight", "g", (d,)
        if a.family == 1:
            yield f"{p}.input_layernorm.bias", "b", (d,)
        yield f"{p}.post_attention_layernorm.weight", "g", (d,)
        if a.family == 1:
            yield f"{p}.post_attention_layernorm.bias", "b", (d,)
    yield "model.norm.weight", "g", (d,)
    if a.family == 1:
        yield "model.norm.bias", "b", (d,)
    if a.family in (0, 1):
        yield "lm_head.weight", "w", (a.n_vocab, d)


def _header(name: str, payload: int) -> bytes:
    nb = name.encode()
    return struct.pack("<i", len(nb)) + nb + struct.pack("<i", len(nb)) + nb + struct.pack("<i", payload)


def synthetic_image(kind: int, wdtype: int, seed: int, pack: Callable, dims=None, std: float = 0.02,
                    gain_std: float = 0.0) -> np.ndarray:
    """Builds a complete .gten image (uint8 array). ``pack(w_fp32_torch_cpu, wdtype)`` returns the
    packed bytes (numpy uint8) of a 2-D fp32 matrix; wdtype F16 packs as fp16 here. gain_std > 0
    draws norm gains as 1 + N(0, gain_std) and biases as N(0, gain_std) (for op coverage tests)."""
    import torch

    a = arch(kind, dims)
    parts = [struct.pack("<q", MAGIC)]
    for idx, (name, k, shape) in enumerate(records(a)):
        g = torch.Generator().manual_seed(seed + idx)
        if k == "w":
            w = torch.randn(shape, generator=g, dtype=torch.float32) * std
            if wdtype == F16:
                payload = w.to(torch.float16).numpy().tobytes()
            else:
                payload = np.asarray(pack(w, wdtype), np.uint8).tobytes()
                assert len(payload) == shape[0] * row_bytes(wdtype, shape[1])
        else:
            base = 1.0 if k == "g" else 0.0
            if gain_std > 0:
                v = base + torch.randn(shape, generator=g, dtype=torch.float32) * gain_std
            else:
                v = torch.full(shape, base, dtype=torch.float32)
            payload = v.to(torch.float16).numpy().tobytes()
        parts.append(_header(name, len(payload)))
        parts.append(payload)
    return np.frombuffer(b"".join(parts), np.uint8)


def synthetic_image_device(kind: int, wdtype: int, seed: int, dims=None, std: float = 0.02,
                           device: str = "cuda") -> np.ndarray:
    """Like synthetic_image, but the N(0, std) matrices are drawn by a CUDA generator (much faster
    for multi-GB checkpoints; the values differ from the CPU-seeded ones) and packed by the
    library's CUDA packer."""
    import torch

    from . import pack_q4, pack_q8

    a = arch(kind, dims)
    parts = [struct.pack("<q", MAGIC)]
    gen = torch.Generator(device=device)
    for idx, (name, k, shape) in enumerate(records(a)):
        if k == "w":
            gen.manual_seed(seed + idx)
            w = torch.randn(shape, generator=gen, dtype=torch.float32, device=device) * std
            if wdtype == F16:
                payload = w.to(torch.float16).cpu().numpy().tobytes()
            else:
                out = torch.empty(shape[0] * row_bytes(wdtype, shape[1]), dtype=torch.uint8, device=device)
                (pack_q8 if wdtype == Q8 else pack_q4)(w, out)
                payload = out.cpu().numpy().tobytes()
            del w
        else:
            payload = np.full(shape, 1.0 if k == "g" else 0.0, np.float16).tobytes()
        parts.append(_header(name, len(payload)))
        parts.append(payload)
    return np.frombuffer(b"".join(parts), np.uint8)


def cuda_packer(device: str = "cuda"):
    """A packer running the library's CUDA kernels (gtn_pack_q8 / gtn_pack_q4)."""
    import torch

    from . import pack_q4, pack_q8

    def pack(w, wdtype):
        wd = w.to(device).contiguous()
        out = torch.empty(w.shape[0] * row_bytes(wdtype, w.shape[1]), dtype=torch.uint8, device=device)
        (pack_q8 if wdtype == Q8 else pack_q4)(wd, out)
        return out.cpu().numpy()

    return pack
