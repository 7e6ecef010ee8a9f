"""Benchmark of the gten B200 path on BASELINE.json's headline workload.

Workload: TinyLlama-1.1B architecture, Q8 weights (reference block
layout) from seeded N(0, 0.02) values, batch 1, a 64-token uniform-random prompt and 256 greedy
decode tokens. One step = one such request (prefill + 256 decode steps, each ending in the fused
argmax). Metric: decode tok/s = generated tokens / request time (the reference's own throughput
definition divides by the whole inference time, tinyllama.cpp:176-178).

* value: device-timed (CUDA events on the model's stream) with prompt and output ids resident in
  HBM; the 1.17 GB of weights are far larger than L2 (126 MB), so every step streams from HBM.
* e2e: the same request through the public C ABI call gtn_model_generate with host buffers (prompt
  from pinned memory -> HBM, ids -> host) inside the timed region.
* roofline: the dominant kernel, the exact Q8 GEMV (k_gemv3), timed live with CUDA events on the
  launching stream over the model's weight shapes (rotating weight copies > L2 between launches,
  launches replayed from a CUDA graph); achieved = weight bytes per launch / mean launch time;
  traffic = DRAM bytes read + written per launch of the same kernel and shape from one ncu capture
  (profiles/k_gemv3_gate_up_q8.md).
* cpu_baseline: the compiled reference (oracle/_ref/libgtenref.so) on this host's cores, a bounded
  sample (prefill + 16 decode steps) extrapolated to the 256-token request.
* --impl reference: the reference arm, same config and metric, on rank 0.
* --gpus N (torchrun): N independent replicas (a batch-1 request does not shard), value summed.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "nanochatllms.cpp_b200"))

N_PROMPT, N_GEN, SEED = 64, 256, 1234
# dram__bytes_read.sum + dram__bytes_write.sum of one k_gemv3 launch on gate_up 11264x2048 (Q8), from
# `ncu --set full --clock-control none -k regex:k_gemv3 -s 3 -c 1 python bench.py --gemv-only
# --gemv-shape gate_up` (profiles/k_gemv3_gate_up_q8.md)
GATE_UP_TRAFFIC_BYTES = 24_539_648
WEIGHT_GB = {1: 2.07, 3: 1.10, 4: 0.58}  # TinyLlama weight bytes streamed per token
WDT_NAMES = {3: "q8", 4: "q4", 1: "f16"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""

    def __init__(self, index: int):
        self.path = f"/tmp/gten_clocks_{os.getpid()}.csv"
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
                for n, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        except Exception:
            return None
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_init():
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


class RefRequestTimer:
    """Times the compiled reference on the host for one batch-1 request (64-token prompt, 256 greedy
    tokens) on the given .gten image. The prompt's prefill is timed as is; the decode steps are
    timed at contexts spread over the request, because the reference's per-token cost grows with the
    context (it re-reads and transposes the whole V prefix every call, ops.cpp:1091-1132). The cache
    is filled once with a prefill of all 319 positions; a decode step at context n is then
    Model::logits(tokens[:n], n - 1), which recomputes only row n - 1 over the cached rows below it
    (the work of that step of the request; rows below n - 1 are not touched). A least-squares line
    t(n) = a + b*n through the samples, summed over n = 65..319, gives the request's decode time."""

    CTX = (65, 128, 192, 256, 319)

    def __init__(self, image, wdt: int, prompt):
        import numpy as np
        from oracle.oracle import Reference, ReferenceModel
        self.path = f"/tmp/gten_bench_{os.getpid()}.gten"
        image.tofile(self.path)
        # max_ctx 2 x 320 keeps the reference's probability rows apart (ops.cpp:1033-1034)
        self.rm = ReferenceModel(Reference(), 0, wdt, 2 * (N_PROMPT + N_GEN), self.path, 32003)
        self.toks = np.concatenate([prompt, np.random.default_rng(5).integers(0, 32000, N_GEN - 1)]).astype(np.int32)
        self.rm.logits(self.toks, 0)  # fills the cache rows 0..318 (untimed)

    def sample(self, reps: int = 2):
        """Returns (tok/s of one request, details)."""
        import numpy as np
        t0 = time.perf_counter()
        self.rm.logits(self.toks[:N_PROMPT], 0)
        t_prefill = time.perf_counter() - t0
        xs, ys = [], []
        for _ in range(reps):
            for n in self.CTX:
                t0 = time.perf_counter()
                self.rm.logits(self.toks[:n], n - 1)
                ys.append(time.perf_counter() - t0)
                xs.append(n)
        b, a = np.polyfit(np.array(xs, float), np.array(ys, float), 1)
        t_dec = float(sum(a + b * n for n in range(N_PROMPT + 1, N_PROMPT + N_GEN)))
        return N_GEN / (t_prefill + t_dec), {"prefill_s": t_prefill, "decode_ms_at_65": (a + b * 65) * 1e3,
                                              "decode_ms_at_319": (a + b * 319) * 1e3, "decode_s": t_dec}

    def close(self):
        del self.rm
        os.remove(self.path)


def ref_sample_text(det) -> str:
    return (f"compiled reference on the same .gten bytes: the 64-token prefill ({det['prefill_s']:.2f} s) and decode "
            f"steps timed at contexts 65-319 ({det['decode_ms_at_65']:.1f} -> {det['decode_ms_at_319']:.1f} ms/token, "
            f"a linear fit summed over the 255 steps)")


def gemv_roofline(G, torch, wdt: int, device, hbm_peak: float, only: str | None = None):
    """Live timing of the exact quantized GEMV on TinyLlama's weight shapes (M = 1)."""
    from gten_b200 import row_bytes
    shapes = [(2560, 2048, "qkv"), (2048, 2048, "o"), (11264, 2048, "gate_up"), (2048, 5632, "down"),
              (32003, 2048, "lm_head")]
    if only:
        shapes = [s for s in shapes if s[2] == only]
    out = {}
    dom = None
    stream = torch.cuda.current_stream()
    for N, K, name in shapes:
        wb = N * row_bytes(wdt, K)
        ncopy = max(2, int(300e6 // wb) + 1)  # rotate through > L2 worth of weights
        ws = [torch.randint(0, 255, (wb,), dtype=torch.uint8, device=device) for _ in range(ncopy)]
        # valid fp16 deltas: overwrite each block's delta with 1/1024
        bb = 34 if wdt == 3 else 18
        for w in ws:
            w.view(-1, bb)[:, 0] = 0x00
            w.view(-1, bb)[:, 1] = 0x14
        xq = torch.zeros(row_bytes(3, K), dtype=torch.uint8, device=device)
        y = torch.empty(N, dtype=torch.float32, device=device)
        X = G.GT(xq, 3, (1, K))
        Y = G.GT(y, 2, (1, N))
        for i in range(3):
            G.matmul_2d(X, G.GT(ws[i % ncopy], wdt, (N, K)), Y)
        reps = 3 * ncopy
        torch.cuda.synchronize()
        # the launches are captured once into a CUDA graph, so the timing sees the kernels only
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(reps):
                G.matmul_2d(X, G.GT(ws[i % ncopy], wdt, (N, K)), Y)
        graph.replay()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
        del graph
        t = ev0.elapsed_time(ev1) / reps * 1e-3
        gbs = wb / t / 1e9
        out[name] = {"N": N, "K": K, "bytes": wb, "us": round(t * 1e6, 2), "GB_s": round(gbs, 1),
                     "frac": round(gbs / hbm_peak, 3)}
        if name == "gate_up" or only:
            dom = out[name]
        del ws
    torch.cuda.empty_cache()
    return dom, out


def gemm_sweep(G, torch, wdt: int, device, M: int, only: str | None = None):
    """Live timing of the exact quantized GEMM with M activation rows on TinyLlama's weight shapes:
    gtn_matmul_2d (the tcgen05 kernel from 32 rows on) and, for comparison, gtn_matmul_2d_noalloc,
    which has no scratch for the activation image and so runs the CUDA-core GEMM. Rotating weight
    copies larger than L2. cells = M*N*K/8 lane sums; the CUDA-core bound of the exact epilogue is
    SMs x 128 lanes x the SM clock / 3 ordered fp32 operations per lane sum. With fp16 weights
    (--wdtype 1) the exact fp16 GEMM (k_gemm_f16) is timed against SMs x 128 lanes x the clock
    fused multiply-adds per second."""
    import ctypes as C
    from gten_b200 import row_bytes
    shapes = [(2560, 2048, "qkv"), (2048, 2048, "o"), (11264, 2048, "gate_up"), (2048, 5632, "down")]
    if only:
        shapes = [s for s in shapes if s[2] == only]
    props = torch.cuda.get_device_properties(device)
    bound = props.multi_processor_count * 128 * 1.965e9 / 3
    stream = torch.cuda.current_stream()
    out = {}
    xdt = 1 if wdt == 1 else 3  # fp16 weights take fp16 activations, Q8 / Q4 weights Q8 ones
    for N, K, name in shapes:
        wb = N * row_bytes(wdt, K)
        ncopy = max(2, int(300e6 // wb) + 1)
        if wdt == 1:  # N(0, 0.02) fp16 weights, N(0, 1) fp16 activations
            ws = [(torch.randn(N * K, device=device) * 0.02).half().view(torch.uint8) for _ in range(ncopy)]
            xq = torch.randn(M * K, device=device).half().view(torch.uint8)
        else:
            ws = [torch.randint(0, 255, (wb,), dtype=torch.uint8, device=device) for _ in range(ncopy)]
            bb = 34 if wdt == 3 else 18
            for w in ws:  # valid fp16 deltas (1/1024) in every block
                w.view(-1, bb)[:, 0] = 0x00
                w.view(-1, bb)[:, 1] = 0x14
            xq = torch.randint(0, 255, (M * row_bytes(3, K),), dtype=torch.uint8, device=device)
            xq.view(-1, 34)[:, 0] = 0x00
            xq.view(-1, 34)[:, 1] = 0x14
        y = torch.empty(M * N, dtype=torch.float32, device=device)
        X, Y = G.GT(xq, xdt, (M, K)), G.GT(y, 2, (M, N))

        def tc(i):
            G.matmul_2d(X, G.GT(ws[i % ncopy], wdt, (N, K)), Y)

        def cc(i):
            rc = G.lib().gtn_matmul_2d_noalloc(C.byref(X.desc()), C.byref(G.GT(ws[i % ncopy], wdt, (N, K)).desc()),
                                               C.byref(Y.desc()), 0,
                                               C.c_void_p(torch.cuda.current_stream().cuda_stream))
            assert rc == 0, G.lib().gtn_last_error()

        res = {"N": N, "K": K, "M": M, "timing": "graph"}
        for key, fn in ((("k_gemm_f16", tc),) if wdt == 1 else (("tc", tc), ("cuda_cores", cc))):
            for i in range(3):
                fn(i)
            reps = 2 * ncopy
            torch.cuda.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            try:
                # the calls replayed from one CUDA graph: device time only, no host work between launches
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for i in range(reps):
                        fn(i)
                graph.replay()
                torch.cuda.synchronize()
                ev0.record(stream)
                graph.replay()
                ev1.record(stream)
                torch.cuda.synchronize()
                del graph
            except Exception:  # not capturable: back-to-back calls (host work can show in the time)
                res["timing"] = "loop"
                torch.cuda.synchronize()
                ev0.record(stream)
                for i in range(reps):
                    fn(i)
                ev1.record(stream)
                torch.cuda.synchronize()
            t = ev0.elapsed_time(ev1) / reps * 1e-3
            if wdt == 1:  # products: one fused multiply-add each on 128 lanes per SM
                macs = M * N * K
                res[key] = {"us": round(t * 1e6, 2), "T_mac_s": round(macs / t / 1e12, 3),
                            "frac_of_fma_bound": round(macs / t / (bound * 3), 3)}
            else:
                cells = M * N * K / 8
                res[key] = {"us": round(t * 1e6, 2), "T_cells_s": round(cells / t / 1e12, 3),
                            "frac_of_epilogue_bound": round(cells / t / bound, 3)}
        out[name] = res
        del ws
    torch.cuda.empty_cache()
    return out


def run_tokenizers(assets: str) -> dict:
    """Host tokenizers: encode() of one seeded ~16 KB text (words, digits, punctuation, whitespace
    runs, multi-byte UTF-8) per model configuration; the reference's own tokenizer (compiled from
    src/gten/tokenizer.cpp into oracle/_ref) is the baseline leg, and its ids must equal ours."""
    import random

    from gten_b200 import tokenizer as T
    rng = random.Random(11)
    alphabet = ([bytes([c]) for c in b"abcdefghijklmnopqrstuvwxyz ABCXYZ0123456789.,;:!?'-\n\t"] +
                [w.encode() for w in ("the ", "and ", "é", "中文", "の", "🙂", "  ", "'s ", "'ll ")])
    text = b"".join(rng.choice(alphabet) for _ in range(12000))[:16384]
    ref_lib = os.path.join(ROOT, "oracle", "_ref", "libgtenref.so")
    out = {"metric": "tokenizer encode ms", "text_bytes": len(text), "models": {}}
    for name in ("tinyllama", "zephyr", "minicpm", "openelm"):
        tok = T.for_model(name, assets)
        t0 = time.perf_counter()
        ids = tok.encode(text)
        ours = time.perf_counter() - t0
        rec = {"ours_ms": round(ours * 1e3, 3), "ids": len(ids)}
        if os.path.exists(ref_lib):
            from oracle.tokenizer_oracle import ReferenceTokenizer, for_model
            ref = ReferenceTokenizer(ref_lib, for_model(name, assets))
            t0 = time.perf_counter()
            rids = ref.encode(text)
            rec["reference_ms"] = round((time.perf_counter() - t0) * 1e3, 1)
            rec["same_ids"] = rids == ids
            ref.close()
        tok.close()
        out["models"][name] = rec
    return out


def weight_bytes(kind: int, wdt: int) -> int:
    """Algorithmic weight bytes one decode token streams: every projection matrix and the lm_head
    (the embedding contributes one row), in the reference's block format."""
    from gten_b200 import gtenfile, row_bytes
    a = gtenfile.arch(kind)
    tot = 0
    for qh, kv, ff in a.layers:
        qd, kvd = qh * 64, kv * 64
        tot += (qd + 2 * kvd) * row_bytes(wdt, a.d) + a.d * row_bytes(wdt, qd)
        tot += 2 * ff * row_bytes(wdt, a.d) + a.d * row_bytes(wdt, ff)
    return tot + a.n_vocab * row_bytes(wdt, a.d)


def kv_bytes_per_ctx(kind: int, wdt: int) -> int:
    """K and V bytes one decode step reads per token of context (all layers, activation dtype)."""
    from gten_b200 import gtenfile, row_bytes
    adt = 1 if wdt == 1 else 3
    return sum(2 * kv * row_bytes(adt, 64) for _, kv, _ in gtenfile.arch(kind).layers)


def time_request(G, torch, wdt, prompt, device, steps, warmup, hbm, image=None, clocks_index=None):
    """One batch-1 TinyLlama request (64-token prompt, 256 greedy tokens) on the device: CUDA events
    on the model's stream over `steps` requests with the prompt and ids in HBM; also the prompt's
    prefill + first id alone, so that the decode steps' time per token is the difference / 255.
    Returns (model, image, dict)."""
    from gten_b200 import gtenfile
    if image is None:  # the bytes the reference arm loads: CPU-seeded values, packed bit-exactly on the GPU
        image = gtenfile.synthetic_image(G.TINYLLAMA, wdt, SEED, gtenfile.cuda_packer(str(device)))
    m = G.Model(G.TINYLLAMA, wdt, N_PROMPT + N_GEN)
    m.load(image)
    st = torch.cuda.ExternalStream(m.stream_ptr, device=device)
    p_dev = torch.from_numpy(prompt).to(device)
    o_dev = torch.empty(N_GEN, dtype=torch.int32, device=device)
    for _ in range(warmup):
        m.generate_device(p_dev, N_GEN, o_dev)
        m.generate_device(p_dev, 1, o_dev)
    m.check()
    torch.cuda.synchronize()
    res = {}
    clocks = Clocks(clocks_index) if clocks_index is not None else None
    for key, n in (("request", N_GEN), ("prefill", 1)):
        launches0 = G.kernel_launches()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            m.generate_device(p_dev, n, o_dev)
        e1.record(st)
        torch.cuda.synchronize()
        res[key] = e0.elapsed_time(e1) * 1e-3 / steps
        if key == "request":
            res["launches"] = G.kernel_launches() - launches0
    res["clocks"] = clocks.stop() if clocks else None
    m.check()
    dec = (res["request"] - res["prefill"]) / (N_GEN - 1)
    # bytes per decode token: the weights plus the K/V rows of the mean context of the decode steps
    mean_ctx = N_PROMPT + N_GEN / 2
    byt = weight_bytes(G.TINYLLAMA, wdt) + kv_bytes_per_ctx(G.TINYLLAMA, wdt) * mean_ctx
    res["decode_s_per_token"] = dec
    res["step_roofline"] = {"bound": "hbm", "bytes_per_token": int(byt), "achieved": round(byt / dec / 1e9, 1),
                            "peak": hbm, "unit": "GB/s", "frac": round(byt / dec / 1e9 / hbm, 4)}
    return m, image, res


def run_ours(args, rank, world, local):
    import numpy as np
    import torch

    import gten_b200 as G
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    hbm, peak_kind = peaks()
    wdt = args.wdtype
    prompt = np.random.default_rng(42).integers(0, 32000, N_PROMPT).astype(np.int32)
    barrier(world)
    torch.cuda.synchronize()
    m, image, req = time_request(G, torch, wdt, prompt, device, args.steps, args.warmup, hbm, clocks_index=local)
    launches, clk = req["launches"], req["clocks"]
    barrier(world)
    t = max_over_ranks(req["request"] * args.steps, world)
    value = world * args.steps * N_GEN / t

    # end to end through the public API with host buffers (pinned prompt, ids read back)
    pin_p = torch.from_numpy(prompt).pin_memory()
    pin_o = torch.empty(N_GEN, dtype=torch.int32).pin_memory()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = m.generate(pin_p.numpy(), N_GEN)
        pin_o.numpy()[:] = out
    t_e2e = max_over_ranks(time.perf_counter() - t0, world)
    e2e = world * args.steps * N_GEN / t_e2e
    m.close()

    # the north-star configuration: the same request with Q4 weights (BASELINE target: >= 0.70 of
    # the HBM roofline per decode token)
    q4 = None
    if wdt != 4:
        mq, _, rq = time_request(G, torch, 4, prompt, device, args.steps, args.warmup, hbm)
        mq.close()
        q4 = {"value": round(N_GEN / rq["request"], 2), "unit": "tok/s",
              "ms_per_step": round(rq["request"] * 1e3, 3),
              "decode_ms_per_token": round(rq["decode_s_per_token"] * 1e3, 4),
              "step_roofline": rq["step_roofline"], "target_frac": 0.70}

    dom, sweep = gemv_roofline(G, torch, wdt, device, hbm)
    result = None
    if rank == 0:
        cpu = None
        if world == 1:
            try:
                rt = RefRequestTimer(image, wdt, prompt)
                tps, det = rt.sample()
                rt.close()
                cpu = {"value": round(tps, 3), "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
                       "sample": ref_sample_text(det)}
            except Exception as ex:  # reference library missing on this machine
                cpu = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
                       "sample": f"unavailable: {ex}"}
        result = {
            "metric": "decode tok/s",
            "value": round(value, 2),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(t / args.steps * 1e3, 3),
            "ms_per_token": round(t / args.steps / N_GEN * 1e3, 4),
            "decode_ms_per_token": round(req["decode_s_per_token"] * 1e3, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int8-blocks/fp32-accum (Q8 weights, Q8 activations)" if wdt == 3 else WDT_NAMES[wdt],
            "data": "synthetic: seeded N(0,0.02) weights (CPU generator, the reference arm's bytes), uniform-random "
                    "prompt ids",
            "config": {"workload": f"TinyLlama-1.1B {WDT_NAMES[wdt].upper()} batch-1, 64-token prompt + 256 greedy "
                                   f"decode tokens per request (BASELINE configs[0])",
                       "model": "tinyllama-1.1b", "global_batch": world, "seq_len": N_PROMPT + N_GEN,
                       "parallelism": f"replicas x{world} (a batch-1 request does not shard)",
                       "l2": f"weights {WEIGHT_GB[wdt]} GB > 126 MB L2; no flush needed"},
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": N_PROMPT * 4,
                    "d2h_bytes_per_step": N_GEN * 4},
            "step_roofline": req["step_roofline"],
            "q4_bs1": q4,
            "roofline": {"bound": "hbm", "kernel": f"k_gemv3 (exact {WDT_NAMES[wdt].upper()} GEMV, gate_up 11264x2048)",
                         "achieved": dom["GB_s"], "peak": hbm, "unit": "GB/s",
                         "frac": round(dom["GB_s"] / hbm, 3), "peak_kind": peak_kind,
                         "traffic": GATE_UP_TRAFFIC_BYTES if wdt == 3 else None,
                         "per_launch_bytes": dom["bytes"], "gemv_sweep": sweep},
            "gpu_launches": int(launches),
            "cpu_baseline": cpu,
        }
        if clk:
            result["clocks"] = clk
    return result


BATCH_MODELS = {"tinyllama": ("TinyLlama-1.1B", 0), "zephyr": ("StableLM-2-Zephyr-1.6B", 1),
                "minicpm": ("MiniCPM-2B", 2), "openelm": ("OpenELM-1.1B", 5)}
# BASELINE configs[0], [2], [3], [4]: prompt tokens and greedy tokens per sequence
BATCH_PROMPT = {"tinyllama": N_PROMPT, "zephyr": 512, "minicpm": 128, "openelm": 1024}
BATCH_GEN = {"tinyllama": N_GEN, "zephyr": N_GEN, "minicpm": N_GEN, "openelm": 512}


def run_batch(args, rank, world, local):
    """--batch B: a global batch of B independent sequences sharded by sequence over the ranks
    (gten_b200.shard): each rank decodes its shard with its own replica in one fused batched step;
    value = B * generated tokens / (max over ranks of the device time of the shard); e2e = the same
    through generate_sharded (host prompts, ids gathered to rank 0), wall clock."""
    import numpy as np
    import torch

    import gten_b200 as G
    from gten_b200 import gtenfile
    from gten_b200.shard import generate_sharded, shard_range
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    name, kind = BATCH_MODELS[args.model]
    n_prompt, n_gen = BATCH_PROMPT[args.model], BATCH_GEN[args.model]
    start, count = shard_range(args.batch, world, rank)
    m = G.Model(kind, args.wdtype, n_prompt + n_gen, max(1, count))
    m.load(gtenfile.synthetic_image_device(kind, args.wdtype, SEED))
    prompts = np.random.default_rng(42).integers(0, 32000, (args.batch, n_prompt)).astype(np.int32)
    mine = prompts[start:start + count]
    st = torch.cuda.ExternalStream(m.stream_ptr, device=device)
    for _ in range(args.warmup):
        if count:
            m.generate_batch(mine, n_gen)
    torch.cuda.synchronize()
    barrier(world)
    clocks = Clocks(local)
    launches0 = G.kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        if count:
            m.generate_batch(mine, n_gen)
    e1.record(st)
    torch.cuda.synchronize()
    launches = G.kernel_launches() - launches0
    clk = clocks.stop()
    t = max_over_ranks(e0.elapsed_time(e1) * 1e-3, world)
    if world > 1:
        # the ids' gather is the process's first point-to-point exchange: set it up (NCCL creates
        # its communicators lazily, which took ~1 s at 4 ranks) before the end-to-end clock starts
        import torch.distributed as dist
        parts = [None] * world if rank == 0 else None
        dist.gather_object((0, np.zeros((0, n_gen), np.int32)), parts, dst=0)
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = generate_sharded(m, prompts, n_gen) if world > 1 else m.generate_batch(prompts, n_gen)
    t_e2e = max_over_ranks(time.perf_counter() - t0, world)
    m.close()
    if rank != 0:
        return None
    tot = args.batch * n_gen * args.steps
    res = {
        "metric": "decode tok/s", "value": round(tot / t, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8-blocks/fp32-accum (Q8 weights, Q8 activations)" if args.wdtype == 3 else WDT_NAMES[args.wdtype],
        "data": "synthetic: seeded N(0,0.02) weights (CUDA generator), uniform-random prompt ids",
        "config": {"workload": f"{name} {WDT_NAMES[args.wdtype].upper()} batch {args.batch} sharded by sequence over "
                               f"{world} GPU(s), {n_prompt}-token prompts + {n_gen} greedy tokens",
                   "model": args.model, "global_batch": args.batch, "seq_len": n_prompt + n_gen,
                   "parallelism": f"sequence shards x{world} (no collective on the data path)"},
        "e2e": {"value": round(tot / t_e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": args.batch * n_prompt * 4,
                "d2h_bytes_per_step": args.batch * n_gen * 4},
        "gpu_launches": int(launches),
        "first_ids": [int(x) for x in out[0, :4]],
    }
    if clk:
        res["clocks"] = clk
    return res


def run_serve(args):
    """Continuous batching on TinyLlama: R requests, prompt lengths uniform in [16, 128] and new
    tokens uniform in [32, 256] (seeded), through --slots slots (gten_b200.serve); then the same
    requests one after another through gtn_model_generate (the reference's one-sequence loop).
    Wall-clock over each whole run (both synchronous), generated tokens / s."""
    import numpy as np
    import torch

    import gten_b200 as G
    from gten_b200 import gtenfile
    from gten_b200.serve import ContinuousBatcher
    rng = np.random.default_rng(7)
    reqs = [(rng.integers(0, 32000, int(rng.integers(16, 129))).astype(np.int32), int(rng.integers(32, 257)))
            for _ in range(args.serve)]
    max_ctx = 128 + 256
    m = G.Model(G.TINYLLAMA, args.wdtype, max_ctx, max_batch=args.slots)
    m.load(gtenfile.synthetic_image_device(G.TINYLLAMA, args.wdtype, SEED))
    # warm-up: capture the slot step and the single-sequence step
    b = ContinuousBatcher(m)
    for i in range(min(args.slots, len(reqs))):
        b.submit(i, reqs[i][0], 8)
    b.run()
    m.generate(reqs[0][0], 8)
    torch.cuda.synchronize()
    total = sum(n for _, n in reqs)
    b = ContinuousBatcher(m)
    for i, (p, n) in enumerate(reqs):
        b.submit(i, p, n)
    t0 = time.perf_counter()
    res = b.run()
    t_cb = time.perf_counter() - t0
    t0 = time.perf_counter()
    same = 0
    for i, (p, n) in enumerate(reqs):
        same += int(np.array_equal(m.generate(p, n), res[i]))
    t_seq = time.perf_counter() - t0
    m.close()
    return {"metric": "served tok/s (continuous batching)", "value": round(total / t_cb, 1), "unit": "tok/s",
            "requests": len(reqs), "slots": args.slots, "generated_tokens": total,
            "steps": b.steps, "mean_busy_slots": round(b.busy_slot_steps / max(b.steps, 1), 2),
            "wall_s": round(t_cb, 3),
            "sequential": {"value": round(total / t_seq, 1), "unit": "tok/s", "wall_s": round(t_seq, 3)},
            "ids_equal_to_sequential": same,
            "config": {"workload": f"TinyLlama-1.1B {WDT_NAMES[args.wdtype].upper()}, prompts U[16,128], "
                                   f"new tokens U[32,256], greedy", "data": "synthetic"}}


def run_load(args):
    """Model upload throughput: a TinyLlama image (host memory) through gtn_model_load, and the same
    bytes from a file (written first, so it is in the page cache) through gtn_model_load_file."""
    import tempfile

    import torch

    import gten_b200 as G
    from gten_b200 import gtenfile
    img = gtenfile.synthetic_image_device(G.TINYLLAMA, args.wdtype, SEED)
    m = G.Model(G.TINYLLAMA, args.wdtype, N_PROMPT + N_GEN)
    m.load(img)  # first load: the arena and the pinned upload buffers are allocated
    res = {"metric": "model upload GB/s", "unit": "GB/s", "bytes": int(img.size),
           "config": {"workload": f"TinyLlama-1.1B {WDT_NAMES[args.wdtype].upper()} .gten image"}}
    for key, fn in (("host_image", lambda: m.load(img)), ("file", None)):
        if fn is None:
            d = "/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir()
            path = os.path.join(d, f"bench_load_{os.getpid()}.gten")
            img.tofile(path)
            fn = (lambda p: (lambda: m.load_file(p)))(path)
        ts = []
        for _ in range(max(args.steps, 3)):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize()
            ts.append(time.perf_counter() - t0)
        res[key] = {"GB_s": round(img.size / min(ts) / 1e9, 2), "ms_best": round(min(ts) * 1e3, 2),
                    "ms_median": round(sorted(ts)[len(ts) // 2] * 1e3, 2)}
        if key == "file":
            os.remove(path)
    res["value"] = res["host_image"]["GB_s"]
    m.close()
    return res


def run_reference(args, rank, world):
    """The reference arm: the compiled reference CPU path on this host (rank 0 only)."""
    if rank != 0:
        return None
    import numpy as np
    import torch

    from gten_b200 import gtenfile
    ref_lib = os.path.join(ROOT, "oracle", "_ref", "libgtenref.so")
    if not os.path.exists(ref_lib):
        return {"impl": "reference", "unavailable": "oracle/_ref/libgtenref.so was not built (needs the reference "
                                                    "checkout at build time)"}
    from oracle.oracle import Oracle
    orc = Oracle()

    def pack(w, dt):
        return orc.pack_q8(w.numpy()) if dt == 3 else orc.pack_q4(w.numpy())

    # CPU-seeded weights packed by the oracle packer (bit-exact with the reference converter)
    image = gtenfile.synthetic_image(0, args.wdtype, SEED, pack)
    prompt = np.random.default_rng(42).integers(0, 32000, N_PROMPT).astype(np.int32)
    rt = RefRequestTimer(image, args.wdtype, prompt)
    vals = []
    for i in range(args.warmup + args.steps):
        tps, det = rt.sample(reps=1)
        if i >= args.warmup:
            vals.append(tps)
    rt.close()
    v = statistics.mean(vals)
    wdt = args.wdtype
    return {
        "impl": "reference", "metric": "decode tok/s", "value": round(v, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": WDT_NAMES[wdt], "data": "synthetic (seeded CPU generator)",
        "config": {"workload": f"TinyLlama-1.1B {WDT_NAMES[wdt].upper()} batch-1, 64-token prompt + 256 greedy "
                               f"decode tokens per request (BASELINE configs[0])", "model": "tinyllama-1.1b",
                   "global_batch": 1, "seq_len": N_PROMPT + N_GEN, "parallelism": "cpu (OpenMP, all cores)"},
        "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
                         "sample": "per step: " + ref_sample_text(det)},
        "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--wdtype", type=int, default=3, choices=[1, 3, 4], help="1 fp16, 3 q8, 4 q4")
    ap.add_argument("--gemm-only", action="store_true",
                    help="only time the exact GEMM (tensor cores vs CUDA cores) on TinyLlama shapes")
    ap.add_argument("--gemm-m", type=int, default=128, help="with --gemm-only: activation rows")
    ap.add_argument("--gemv-only", action="store_true",
                    help="only the exact GEMV sweep on TinyLlama's shapes (M=1), e.g. for profiling")
    ap.add_argument("--gemv-shape", default=None, choices=["qkv", "o", "gate_up", "down", "lm_head"],
                    help="with --gemv-only: one shape only")
    ap.add_argument("--batch", type=int, default=1,
                    help="global batch of sequences sharded over the ranks (default 1: the headline bs1 request)")
    ap.add_argument("--model", default="tinyllama", choices=sorted(BATCH_MODELS), help="with --batch > 1")
    ap.add_argument("--serve", type=int, default=0, metavar="R",
                    help="continuous batching: R requests of mixed prompt / generation lengths through "
                         "--slots slots, against the same requests one at a time")
    ap.add_argument("--slots", type=int, default=16, help="with --serve: decode slots (max_batch)")
    ap.add_argument("--load", action="store_true",
                    help="only time the model upload (gtn_model_load from host memory, gtn_model_load_file "
                         "from a file in the page cache)")
    ap.add_argument("--decode-only", type=int, default=0, metavar="T",
                    help="only load the model and run one request of T generated tokens (for a launch list); "
                         "with --batch B > 1: one warm generate_batch of B sequences of --model, then the measured "
                         "one of T tokens inside the NVTX range 'gen' (ncu --nvtx --nvtx-include gen/)")
    ap.add_argument("--tokenizers", default=None, metavar="DIR",
                    help="only time encode() of a seeded 16 KB text with each model's tokenizer, from the "
                         "vocabulary files in DIR (the reference's assets/tokenizers), against the reference's "
                         "own tokenizer (oracle/_ref) where it was built")
    ap.add_argument("--topk", type=int, default=0, metavar="K",
                    help="with --decode-only: draw with top-k sampling (temperature 0.9, seed 7) instead of greedy")
    args = ap.parse_args()
    if args.tokenizers:
        print(json.dumps(run_tokenizers(args.tokenizers)), flush=True)
        return
    if args.decode_only and args.batch > 1:
        import numpy as np
        import torch

        import gten_b200 as G
        from gten_b200 import gtenfile
        _, kind = BATCH_MODELS[args.model]
        n_prompt = BATCH_PROMPT[args.model]
        m = G.Model(kind, args.wdtype, n_prompt + BATCH_GEN[args.model], args.batch)
        m.load(gtenfile.synthetic_image_device(kind, args.wdtype, SEED))
        prompts = np.random.default_rng(42).integers(0, 32000, (args.batch, n_prompt)).astype(np.int32)
        m.generate_batch(prompts, 2)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("gen")
        out = m.generate_batch(prompts, args.decode_only)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        m.check()
        m.close()
        print(json.dumps({"decode_only": args.decode_only, "batch": args.batch, "model": args.model,
                          "first_ids": [int(x) for x in out[0, :8]]}), flush=True)
        return
    if args.decode_only:
        import numpy as np
        import torch

        import gten_b200 as G
        from gten_b200 import gtenfile
        m = G.Model(G.TINYLLAMA, args.wdtype, N_PROMPT + N_GEN)
        m.load(gtenfile.synthetic_image_device(G.TINYLLAMA, args.wdtype, SEED))
        prompt = np.random.default_rng(42).integers(0, 32000, N_PROMPT).astype(np.int32)
        if args.topk:
            rng = G.Rng(7)
            out = m.generate_topk(prompt, args.decode_only, 0.9, args.topk, rng)
            rng.close()
        else:
            out = m.generate(prompt, args.decode_only)
        m.check()
        m.close()
        print(json.dumps({"decode_only": args.decode_only, "first_ids": [int(x) for x in out[:8]]}), flush=True)
        return
    if args.load:
        print(json.dumps(run_load(args)), flush=True)
        return
    if args.serve:
        print(json.dumps(run_serve(args)), flush=True)
        return
    if args.gemm_only:
        import torch

        import gten_b200 as G
        sweep = gemm_sweep(G, torch, args.wdtype, torch.device("cuda", 0), args.gemm_m, args.gemv_shape)
        print(json.dumps({"gemm_sweep": sweep, "wdtype": WDT_NAMES[args.wdtype]}), flush=True)
        return
    if args.gemv_only:
        import torch

        import gten_b200 as G
        hbm, _ = peaks()
        _, sweep = gemv_roofline(G, torch, args.wdtype, torch.device("cuda", 0), hbm, args.gemv_shape)
        print(json.dumps({"gemv_sweep": sweep, "wdtype": WDT_NAMES[args.wdtype]}), flush=True)
        return
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        res = run_reference(args, rank, world)
    else:
        rank, world, local = dist_init()
        res = run_batch(args, rank, world, local) if args.batch > 1 else run_ours(args, rank, world, local)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
