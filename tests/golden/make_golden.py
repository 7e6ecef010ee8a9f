"""Generates the committed golden vectors from the REFERENCE itself (run in the build container,
where the reference checkout exists; the GPU box only reads the outputs).

* pack.npz: seeded fp32 matrices (with all-zero blocks and exact .5 ties) and the bytes produced
  by the reference converter's own q8_quantize / q4_quantize / write_layer
  (src/tinyllama/tinyllama_to_gten.py:24-148, executed from its source text up to its argparse
  section, which would otherwise run at import).
* ops.npz: small seeded cases run through the compiled reference ops (oracle/_ref/libgtenref.so,
  built from src/gten by oracle/build_ref.sh): inputs and outputs.
* greedy_tokens.json: full-size TinyLlama (Q8, Q4, F16) with seeded N(0, 0.02) weights (packed by
  the oracle's packer, which pack.npz pins to the reference packer), a seeded 64-token prompt and
  the first 64 greedy token ids of the compiled reference (ref_model_greedy = sampler.cpp:11-53
  without the EOS stop), with each step's top-2 logit margin.
* sampled_tokens.json: the same TinyLlama Q8 model and prompt decoded by the reference's top-k loop
  (sampler.cpp:63-143 without tokenization or the EOS stop): each step's logits from the compiled
  reference's Model::logits, each draw by oracle/sampler_oracle.cpp (the loop body with the same
  libstdc++ calls) from one std::mt19937(seed) in place of std::random_device; with each step's gap
  between the k-th and (k+1)-th largest logit (a tie there would make the pick library-specific).

* model_tokens.json: the other BASELINE architectures at full size, each with seeded N(0, 0.02)
  weights packed by the oracle's packer and a seeded uniform-random prompt: the compiled reference's
  first 64 greedy ids (same harness as greedy_tokens.json) with each step's top-2 margin.
  StableLM-2-Zephyr-1.6B Q4 (512-token prompt), MiniCPM-2B Q8 and Q4 (128-token prompt) and
  OpenELM-1.1B (openelm_lg_cfg) fp16 (1024-token prompt; the reference runs OpenELM in fp16 only).
  n_ctx = 2 x (prompt + 64) keeps the reference's attention-probability rows apart
  (ops.cpp:1033-1034 offsets them by element counts used as byte counts).

The reference checkout is named by the first non-option argument, GTEN_REFERENCE_DIR or
BASELINE.json's reference_path (the packer goldens need it; the model goldens only need oracle/_ref/libgtenref.so, which
oracle/build_ref.sh builds from the same checkout).

Usage: python tests/golden/make_golden.py <reference_dir>
       python tests/golden/make_golden.py --sampled     (sampled_tokens.json only)
       python tests/golden/make_golden.py --models [name ...]   (model_tokens.json; default all)
"""
import hashlib
import io
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "nanochatllms.cpp_b200"))

from oracle.oracle import F16, F32, Q4, Q8, Oracle, Reference, ReferenceModel, SamplerOracle, row_bytes  # noqa: E402


def reference_packer(ref_dir):
    """q8_quantize / q4_quantize / write_layer from the reference converter's source text."""
    path = os.path.join(ref_dir, "src", "tinyllama", "tinyllama_to_gten.py")
    src = open(path).read()
    src = src[: src.index("parser = argparse")]
    ns = {}
    exec(compile(src, path, "exec"), ns)
    return ns


def pack_cases():
    rng = np.random.default_rng(20241201)
    w = (rng.standard_normal((24, 256)) * 0.02).astype(np.float32)
    w[0, :32] = 0.0  # zero block -> delta 0
    w[1, :32] = 0.0
    w[1, 5] = 1e-3  # single non-zero
    # ties after scaling: values at exact multiples of delta/2 for both packers
    w[2, :32] = np.float32(0.25) * np.tile([-1, 0, 1, 2], 8).astype(np.float32)
    w[3, :32] = np.float32(7.0) * np.linspace(-1, 1, 32).astype(np.float32)
    w[4, :] = np.float32(1e-6) * rng.standard_normal(256).astype(np.float32)  # fp16 subnormal deltas
    w[5, :] = np.float32(30000.0) * rng.standard_normal(256).astype(np.float32)  # large values
    return w


def reference_dir():
    from oracle.oracle import reference_dir as configured
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    d = args[0] if args else configured()
    if not d or not os.path.isdir(os.path.join(d, "src")):
        sys.exit("make_golden.py: name the reference checkout (argument, GTEN_REFERENCE_DIR or BASELINE.json "
                 "reference_path)")
    return d


def main():
    ref_dir = reference_dir()
    import torch

    ns = reference_packer(ref_dir)
    w = pack_cases()
    out = {"w": w}
    for name, dt in (("q8", "q8"), ("q4", "q4")):
        buf = io.BytesIO()
        ns["write_layer"](buf, "t", torch.from_numpy(w.copy()), dt)
        raw = buf.getvalue()
        # record: int32 len + name, int32 len + name, int32 size, payload
        hdr = 4 + 1 + 4 + 1 + 4
        out[name] = np.frombuffer(raw[hdr:], np.uint8)
    np.savez_compressed(os.path.join(HERE, "pack.npz"), **out)

    orc = Oracle()
    ref = Reference()
    rng = np.random.default_rng(7)
    ops = {}

    def q8(M, K, s=1.0):
        x = (rng.standard_normal((M, K)) * s).astype(np.float32)
        return np.concatenate([ref.q8_quantize_row(x[i]) for i in range(M)])

    def f16(M, K, s=1.0):
        return (rng.standard_normal((M, K)) * s).astype(np.float16).view(np.uint8).ravel().copy()

    for wdt, wname in ((Q8, "q8"), (Q4, "q4"), (F16, "f16")):
        xdt = F16 if wdt == F16 else Q8
        M, K, N = 3, 256, 64
        x = f16(M, K) if xdt == F16 else q8(M, K)
        wf = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        wb = orc.pack_q8(wf) if wdt == Q8 else (orc.pack_q4(wf) if wdt == Q4 else
                                                wf.astype(np.float16).view(np.uint8).ravel().copy())
        ops[f"mm_{wname}_x"] = x
        ops[f"mm_{wname}_w"] = wb
        ops[f"mm_{wname}_out"] = ref.matmul_2d(x, xdt, M, K, wb, wdt, N, xdt, start_pos=0)
        ops[f"mm_{wname}_out32"] = ref.matmul_2d(x, xdt, M, K, wb, wdt, N, F32, start_pos=0)
    for dt, dname in ((Q8, "q8"), (F16, "f16")):
        M, D = 4, 256
        x = q8(M, D, 2.0) if dt == Q8 else f16(M, D, 2.0)
        y = q8(M, D) if dt == Q8 else f16(M, D)
        g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16).view(np.uint16).copy()
        b = (0.1 * rng.standard_normal(D)).astype(np.float16).view(np.uint16).copy()
        ops[f"{dname}_x"], ops[f"{dname}_y"], ops[f"{dname}_g"], ops[f"{dname}_b"] = x, y, g, b
        ops[f"{dname}_rms"] = ref.rms_norm(x, dt, M, D, g, 0)
        ops[f"{dname}_ln"] = ref.layer_norm(x, dt, M, D, g, b, 0)
        ops[f"{dname}_rope"] = ref.rotary_emb(x, dt, M, D, 64, 1.0, 0)
        ops[f"{dname}_rope25"] = ref.rotary_emb(x, dt, M, D, 64, 0.25, 0)
        ops[f"{dname}_silu"] = ref.silu(x, dt, M, D, 0)
        ops[f"{dname}_mul"] = ref.multiply(x, y, dt, M, D)
        ops[f"{dname}_add"] = ref.add(x, y, dt, M, D)
        ops[f"{dname}_scale"] = ref.scale(x, dt, M, D, 12.0)
        ops[f"{dname}_bias"] = ref.bias_add_inplace(x, dt, M, D, b)
        n, H, KVH = 37, 4, 2
        q, k, v = (q8(n, H * 64), q8(n, KVH * 64), q8(n, KVH * 64)) if dt == Q8 else \
            (f16(n, H * 64), f16(n, KVH * 64), f16(n, KVH * 64))
        ops[f"{dname}_q"], ops[f"{dname}_k"], ops[f"{dname}_v"] = q, k, v
        ops[f"{dname}_attn"] = ref.qkv_attn(q, k, v, dt, n, H, H * 64, KVH * 64, 0, max_ctx=4 * n)
        ops[f"{dname}_attn_dec"] = ref.qkv_attn(q, k, v, dt, n, H, H * 64, KVH * 64, n - 1, max_ctx=4 * n)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **ops)

    from gten_b200 import gtenfile

    def pack(wt, dt):
        return orc.pack_q8(wt.numpy()) if dt == Q8 else orc.pack_q4(wt.numpy())

    gold = {}
    for wdt, n_ctx in ((Q8, 128), (Q4, 128), (F16, 128)):
        seed = 1234
        img = gtenfile.synthetic_image(0, wdt, seed, pack)
        path = f"/tmp/golden_tinyllama_{wdt}.gten"
        img.tofile(path)
        prompt = np.random.default_rng(42).integers(0, 32000, 64).astype(np.int32)
        rm = ReferenceModel(ref, 0, wdt, n_ctx, path, 32003)
        toks, margins = rm.greedy(prompt, 64, margins=True)
        del rm
        os.remove(path)
        gold[f"tinyllama_w{wdt}"] = {"seed": seed, "n_ctx": n_ctx, "prompt": prompt.tolist(),
                                     "tokens": toks.tolist(), "margins": [float(x) for x in margins]}
        print(wdt, toks[:16].tolist(), "min margin", float(margins.min()))
    with open(os.path.join(HERE, "greedy_tokens.json"), "w") as f:
        json.dump(gold, f)


def sampled():
    from gten_b200 import gtenfile
    orc, ref = Oracle(), Reference()

    def pack(wt, dt):
        return orc.pack_q8(wt.numpy()) if dt == Q8 else orc.pack_q4(wt.numpy())

    gold = {}
    for wdt, temp, top_k, rng_seed in ((Q8, 0.9, 40, 20240607), (Q4, 1.7, 200, 7)):
        seed, n_ctx, n_gen = 1234, 128, 48
        img = gtenfile.synthetic_image(0, wdt, seed, pack)
        path = f"/tmp/golden_tinyllama_sampled_{wdt}.gten"
        img.tofile(path)
        prompt = np.random.default_rng(42).integers(0, 32000, 64).astype(np.int32)
        rm = ReferenceModel(ref, 0, wdt, n_ctx, path, 32003)
        gen = SamplerOracle().generator(rng_seed)
        toks, out, gaps = list(prompt), [], []
        for i in range(n_gen):
            lg = rm.logits(np.array(toks, np.int32), 0 if i == 0 else len(toks) - 1)
            top = np.sort(lg)[::-1]
            gaps.append(float(top[min(top_k, 1000) - 1] - top[min(top_k, 1000)]))
            t = gen.step(lg, temp, top_k)
            out.append(t)
            toks.append(t)
        del rm
        os.remove(path)
        gold[f"tinyllama_w{wdt}"] = {"seed": seed, "n_ctx": n_ctx, "prompt": prompt.tolist(), "temp": temp,
                                     "top_k": top_k, "rng_seed": rng_seed, "tokens": out, "kth_gaps": gaps}
        print(wdt, out[:16], "min k-th gap", min(gaps))
    with open(os.path.join(HERE, "sampled_tokens.json"), "w") as f:
        json.dump(gold, f)


# name -> (gtenfile kind, weight dtype, prompt tokens); BASELINE configs[2], [3], [4]
MODEL_CASES = {
    "zephyr_w4": (1, Q4, 512),
    "minicpm_w3": (2, Q8, 128),
    "minicpm_w4": (2, Q4, 128),
    "openelm_lg_w1": (5, F16, 1024),
}
MODEL_VOCAB = {0: 32003, 1: 100352, 2: 122753, 5: 32000}


def models(names):
    """model_tokens.json: the compiled reference's first 64 greedy ids on full-size models."""
    import time

    from gten_b200 import gtenfile
    orc, ref = Oracle(), Reference()

    def pack(wt, dt):
        return orc.pack_q8(wt.numpy()) if dt == Q8 else orc.pack_q4(wt.numpy())

    path_json = os.path.join(HERE, "model_tokens.json")
    gold = json.load(open(path_json)) if os.path.exists(path_json) else {}
    for name in names:
        kind, wdt, n_prompt = MODEL_CASES[name]
        seed, n_gen = 1234, 64
        n_ctx = 2 * (n_prompt + n_gen)
        t0 = time.time()
        img = gtenfile.synthetic_image(kind, wdt, seed, pack)
        path = f"/tmp/golden_{name}.gten"
        img.tofile(path)
        del img
        prompt = np.random.default_rng(42).integers(0, 32000, n_prompt).astype(np.int32)
        rm = ReferenceModel(ref, kind, wdt, n_ctx, path, MODEL_VOCAB[kind])
        # the greedy loop of ref_model_greedy (sampler.cpp:11-53), step by step so that the logits
        # of the prefill and of two decode steps are recorded as SHA-256 digests of their fp32 bytes
        toks, ids, margins, digests = [int(t) for t in prompt], [], [], {}
        for i in range(n_gen):
            lg = rm.logits(np.array(toks, np.int32), 0 if i == 0 else len(toks) - 1)
            t = int(np.argmax(lg))  # the first maximum, as the reference's strict '>' scan
            top = np.sort(lg)[::-1]
            margins.append(float(top[0] - top[1]))
            if i in (0, 1, n_gen - 1):
                digests[str(i)] = hashlib.sha256(lg.astype(np.float32).tobytes()).hexdigest()
            ids.append(t)
            toks.append(t)
        del rm
        os.remove(path)
        gold[name] = {"kind": kind, "wdtype": wdt, "seed": seed, "n_ctx": n_ctx, "prompt": prompt.tolist(),
                      "tokens": ids, "margins": margins, "logits_sha256": digests}
        print(name, ids[:16], "distinct", len(set(ids)), "min margin", min(margins), f"{time.time() - t0:.0f} s",
              flush=True)
        with open(path_json, "w") as f:
            json.dump(gold, f)


if __name__ == "__main__":
    if "--models" in sys.argv:
        names = [a for a in sys.argv[sys.argv.index("--models") + 1:] if not a.startswith("--")]
        models(names or list(MODEL_CASES))
    elif "--sampled" in sys.argv:
        sampled()
    else:
        main()
        sampled()
