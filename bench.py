"""Benchmark of the BASELINE headline: q4 decode tokens/s at batch 1 and 4K context (config 2),
one independent replica per GPU (weak scaling), plus the HBM roofline of the dominant kernel and
the CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Side modes (one GPU, one JSON line each): --micro (config 1, per-shape dequant-GEMV GB/s),
--prefill (config 3, multimodal prefill through the tensor-core path, TFLOP/s against the
measured GEMM peak), --batched (config 4, 64 sessions decoded together, HBM roofline).

A step is one greedy decode token (28 layers + lm_head + on-device argmax) of a session whose KV
cache was pre-filled with 4096 positions of N(0,1) bf16 values; the context grows by one per step.
Weights are seeded N(0,0.02) (torch CUDA generator), q4s decoder matrices and q8 lm_head.  The
weights streamed per step (1.12 GB) and the KV (0.47 GB) are far larger than L2, so no flush is
needed between steps.
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

CTX = 4096
SETTLE_STEPS = 512
PROFILE_STEPS = 32
SEED = 0
METRIC = "q4 decode tokens/s (batch 1, 4K ctx)"
WORKLOAD = "config 2: batch-1 q4 decode, KV pre-filled to 4096 positions, CUDA graph of 8 steps"
H, FF, V, NL = 2048, 6144, 151936, 28
Q4_LAYER_BYTES = (4096 * 2048 + 2048 * 2048 + 12288 * 2048 + 2048 * 6144) * 9 // 16  # 0.5625 B / weight
Q8_HEAD_BYTES = V * 2048 * 17 // 16                                                  # 1.0625 B / weight
NORM_BYTES = (NL * (2 * 2048 + 2 * 128) + 2048) * 4
KV_BYTES_PER_POS = NL * 8 * 128 * 2 * 2


def step_bytes(ctx: int) -> int:
    """Algorithmic HBM bytes of one decode token at context ctx (weights + norms + KV read)."""
    return NL * Q4_LAYER_BYTES + Q8_HEAD_BYTES + NORM_BYTES + KV_BYTES_PER_POS * ctx


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = [r.split(", ") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        load = sorted(sm)[len(sm) // 2:] if sm else []
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def model_source_key() -> str:
    """Hash of the sources that decide the bytes of the bench model file (seeded generator, file
    writer, quantizers), so a cached file is never reused after any of them changes."""
    import hashlib

    h = hashlib.sha256()
    for rel in ("instantcua_b200/model.py", "instantcua_b200/_lib.py", "instantcua_b200/csrc/pack.cpp"):
        with open(os.path.join(ROOT, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def model_file(rank_local: int, group, device: int) -> str:
    """Generates the seeded q4s model once per box (local rank 0) into /tmp and reuses it while the
    sources that produce it are unchanged."""
    path = f"/tmp/icua_bench_seed{SEED}_q4s_{model_source_key()}.icua"
    if rank_local == 0 and not os.path.exists(path):
        from instantcua_b200 import model

        tensors = model.quantize_stream(model.synthetic_fp32_fast(seed=SEED, device=device))
        tmp = path + f".{os.getpid()}.tmp"
        model.write_icua(tmp, tensors)
        os.replace(tmp, path)
    if group is not None:
        group.barrier()
    return path


def replica_group(backend: str = "nccl"):
    """The replicas of this launch (one process per GPU under torchrun): the product's ReplicaGroup,
    whose process group carries only barriers and the end-of-run gather of counts and times."""
    from instantcua_b200.replicas import ReplicaGroup

    return ReplicaGroup(backend)


def run_ours(args):
    import numpy as np
    import torch

    from instantcua_b200.replicas import aggregate_rate

    group = replica_group("nccl")
    world, rank, local = group.world, group.rank, group.local
    torch.cuda.set_device(local)
    from instantcua_b200 import Engine
    from instantcua_b200 import _lib as L

    path = model_file(local, group, local)
    K, W = args.steps, args.warmup
    # S more warm-up steps run while the clock sampler starts (about half a second of decoding), so
    # the sampler's start-up never overlaps the timed steps; the cache is pre-filled so that the
    # timed region starts at context CTX exactly.
    S = SETTLE_STEPS
    n_inject = CTX - 1 - W - S
    eng = Engine(path, max_context=CTX + K + 2 * 64 + 64 + PROFILE_STEPS, max_pass=16,
                 max_steps=W + S + K + 128 + PROFILE_STEPS, kv_dtype="bf16",
                 steps_per_graph=8, device=local)
    eng.stop_on_eos = False
    eng.inject_kv_random(n_inject, seed=2 + rank)
    tok = int(np.random.default_rng(rank).integers(0, 151643))
    tok = eng.decode_step(tok)  # primes the session
    eng.decode(W)  # warm-up steps (graphs instantiated, clocks up)

    group.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        eng.decode(S)
        torch.cuda.synchronize()
        ctx0 = eng.position()
        group.barrier()
        eng.decode(K)
        ms = eng.last_timing.decode_ms
    torch.cuda.synchronize()
    ms = group.max_over_ranks(ms)
    group.barrier()
    ms_step = ms / K
    value = aggregate_rate(K, world, ms / 1e3)

    # e2e through the public host API: one decode step per call, token in from host, token out
    # to host, synchronised each call (inputs and results cross PCIe every step).
    KE = min(K, 64)
    cur = eng.decode(1)[-1]
    group.barrier()
    t0 = time.perf_counter()
    for _ in range(KE):
        cur = eng.decode_step(cur)
    e2e_s = group.max_over_ranks(time.perf_counter() - t0)
    e2e = aggregate_rate(KE, world, e2e_s)

    # Per-kernel rooflines: PROFILE_STEPS more steps with CUDA events (engine stream) around each
    # step's decoder layers (on q4s engines one persistent kernel) and around its lm_head + commit.
    peak, peak_kind = peaks()
    ctx_p = eng.position()
    lay_ms, head_ms = eng.profile_decode(PROFILE_STEPS)
    kps = eng.kernels_per_step
    attn_o = eng.attn_o_cluster
    dev_bytes = eng.device_bytes
    roof = None
    if rank == 0:
        roof = lm_head_roofline(torch, L, peak)
    eng.close()
    lay_ms /= PROFILE_STEPS
    head_ms /= PROFILE_STEPS
    lay_bytes = NL * Q4_LAYER_BYTES + NORM_BYTES - 2048 * 4 + KV_BYTES_PER_POS * int(ctx_p + PROFILE_STEPS / 2)
    lay_ach = lay_bytes / (lay_ms / 1e3) / 1e9
    head_bytes = Q8_HEAD_BYTES + 2048 * 4
    head_ach = head_bytes / (head_ms / 1e3) / 1e9

    ctx_mid = ctx0 + K / 2
    out = None
    if rank == 0:
        sb = step_bytes(int(ctx_mid))
        achieved_step = sb / (ms_step / 1e3) / 1e9
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4s/q8 weights, fp32 math, bf16 KV", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) KV)",
            "config": {"workload": WORKLOAD,
                       "model": "Qwen3-VL-2B text decoder (28 layers, random init)", "global_batch": world,
                       "seq_len": CTX, "context_range": [ctx0, ctx0 + K], "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2 (1.59 GB streamed per step)"},
            "roofline": {"kernel": ("decode_mk_kernel: all 28 decoder layers of a token in one cooperative launch"
                                    if kps == 3 else
                                    f"decoder layers: {(kps - 2) // NL} x {NL} PDL-chained launches"
                                    + (f" (o-proj folded into the attention, clusters of {attn_o})" if attn_o else "")),
                         "bound": "hbm", "achieved": round(lay_ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(lay_ach / peak, 4),
                         "traffic": profile_traffic("decode_mk_layers_config2.md") if kps == 3 else None,
                         "algorithmic_bytes": int(lay_bytes), "ms_per_launch": round(lay_ms, 5),
                         "note": f"q4s layer weights + norms + KV at ctx {int(ctx_p + PROFILE_STEPS / 2)}, CUDA events "
                                 f"around the layers of each of {PROFILE_STEPS} steps; peak {peak_kind}"},
            "step_roofline": {"bound": "hbm", "achieved": round(achieved_step, 1), "peak": peak, "unit": "GB/s",
                              "frac": round(achieved_step / peak, 4), "bytes_per_step": sb, "ms_per_step": round(ms_step, 5),
                              "note": f"whole token (layers + lm_head + commit) at ctx {int(ctx_mid)}, CUDA events "
                                      f"over the timed graph launches; peak {peak_kind}"},
            "head_roofline": {"kernel": "lm_head GEMV (q8 151936x2048) + commit, in the step", "bound": "hbm",
                              "achieved": round(head_ach, 1), "peak": peak, "unit": "GB/s",
                              "frac": round(head_ach / peak, 4), "ms_per_step": round(head_ms, 5)},
            "lm_head_roofline": roof,
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": 24, "d2h_bytes_per_step": 4,
                    "api": "icua_decode_step (host token in, host token out, synchronised per step)", "steps": KE},
            "gpu_launches": K * kps,
            "engine_device_bytes": dev_bytes,
            "clocks": clk.summary(),
        }
    group.close()
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        out["cpu_baseline"] = cpu_baseline(path)
    if rank == 0:
        print(json.dumps(out))


def fill_units(torch, w, fmt):
    """Random codes with valid fp16 scales (0x1419, about 1.06e-3) in every unit's scale block, so
    the arithmetic is representative."""
    ub, wb = (1088, 1024) if fmt == 1 else (576, 512)
    units = w.view(-1, ub)
    units[:, wb:] = torch.tensor([0x1419], dtype=torch.int16, device=w.device).view(torch.uint8).repeat(32)


def time_gemv(torch, L, fmt, n, k, x_dtype=0, reps=50, min_bytes=0):
    """Times icua_gemv with CUDA events: `reps` launches captured back to back in one CUDA graph
    (so the host's launch rate is not what is measured), replayed 5 times.  When min_bytes > 0
    the weights are replicated until the copies exceed it and the launches rotate through them
    (L2 defeated).  Returns (ms per launch, algorithmic bytes per launch, copies)."""
    import ctypes as C

    nbytes = L.lib().icua_packed_bytes(fmt, n, k)
    copies = max(1, -(-min_bytes // nbytes)) if min_bytes else 1
    w = torch.randint(0, 255, (copies * nbytes,), dtype=torch.uint8, device="cuda")
    fill_units(torch, w, fmt)
    x = torch.randn(k, device="cuda", dtype=torch.bfloat16 if x_dtype == 1 else torch.float32)
    y = torch.empty(n, device="cuda")
    base = w.data_ptr()

    def run(i):
        s = torch.cuda.current_stream()
        L.check(L.lib().icua_gemv(fmt, n, k, C.c_void_p(base + (i % copies) * nbytes), C.c_void_p(x.data_ptr()),
                                  x_dtype, C.c_void_p(y.data_ptr()), C.c_void_p(s.cuda_stream)))

    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        for i in range(max(5, copies)):
            run(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            run(i)
    g.replay()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for _ in range(5):
        g.replay()
    b.record(s)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (5 * reps)
    alg = nbytes + k * x.element_size() + n * 4
    return ms, alg, copies


def profile_traffic(name):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) recorded in a committed
    ncu summary under profiles/, or None when that summary is absent."""
    import re

    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*(\d+)", open(p).read())
    return int(m.group(1)) if m else None


def lm_head_roofline(torch, L, peak):
    n, k = V, 2048
    ms, alg, _ = time_gemv(torch, L, 1, n, k)
    ach = alg / (ms / 1e3) / 1e9
    return {"kernel": "gemv_kernel<q8,store> lm_head 151936x2048", "bound": "hbm", "achieved": round(ach, 1),
            "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
            "traffic": profile_traffic("gemv_q8_lm_head_151936x2048.md"),
            "algorithmic_bytes": alg, "ms_per_launch": round(ms, 5)}


MICRO_SHAPES = (("q/o 2048x2048", 3, 2048, 2048), ("k/v 2048x1024", 3, 1024, 2048),
                ("gate+up 2048x12288", 3, 12288, 2048), ("down 6144x2048", 3, 2048, 6144),
                ("lm_head q8 2048x151936", 1, V, 2048))


def run_micro(args):
    """Config 1: isolated batch-1 dequant-GEMV per decoder shape (K x N), bf16 activations N(0,1),
    weights rotated over copies totalling more than twice the 126 MB L2."""
    import torch

    from instantcua_b200 import _lib as L

    peak, peak_kind = peaks()
    rows = []
    for name, fmt, n, k in MICRO_SHAPES:
        if args.micro_shape and args.micro_shape not in name:
            continue
        ms, alg, copies = time_gemv(torch, L, fmt, n, k, x_dtype=1, reps=max(args.steps, 20), min_bytes=256 << 20)
        gbs = alg / (ms / 1e3) / 1e9
        rows.append({"shape": name, "fmt": "q8" if fmt == 1 else "q4s", "n_rows": n, "k": k, "us": round(ms * 1e3, 2),
                     "GB/s": round(gbs, 1), "frac": round(gbs / peak, 4), "algorithmic_bytes": alg,
                     "copies_rotated": copies})
    tot_b = sum(r["algorithmic_bytes"] for r in rows)
    tot_us = sum(r["us"] for r in rows)
    print(json.dumps({"metric": "q4/q8 dequant-GEMV GB/s (batch 1, config 1)", "value": round(tot_b / tot_us / 1e3, 1),
                      "unit": "GB/s", "n_gpus": 1, "steps": max(args.steps, 20), "higher_is_better": True,
                      "dtype": "q4s/q8 weights, bf16 x, fp32 accumulate", "data": "synthetic random codes",
                      "config": {"workload": "config 1: GEMV microbench", "l2": "weights rotated over > 256 MB"},
                      "peak": peak, "peak_kind": peak_kind, "shapes": rows}))


def cpu_baseline(path, steps: int = 3):
    """The numpy oracle (fp32, all host threads) decoding at 4K context on the same model file."""
    t0 = time.perf_counter()
    w, model = oracle_model_from_file(path)
    sample_ctx = CTX
    import numpy as np

    rng = np.random.default_rng(5)
    kc = [rng.standard_normal((sample_ctx, 8, 128), dtype=np.float32) for _ in range(NL)]
    vc = [rng.standard_normal((sample_ctx, 8, 128), dtype=np.float32) for _ in range(NL)]
    model.inject_kv(kc, vc)
    limiter, cores = host_blas_threads()
    with limiter:
        model.decode_step(1)  # warm-up
        t1 = time.perf_counter()
        for i in range(steps):
            model.decode_step(100 + i)
        dt = time.perf_counter() - t1
    return {"value": round(steps / dt, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{steps} decode tokens at context {sample_ctx}, numpy fp32 oracle on dequantized weights "
                      f"(setup {t1 - t0:.0f}s untimed)"}


def oracle_model_from_file(path):
    """Dequantized fp32 weights for the oracle, read from the bench's .icua file."""
    import struct

    import numpy as np

    from oracle import qwen3vl_oracle as O
    from instantcua_b200 import _lib as LB
    from instantcua_b200.model import layer_tid

    raw = open(path, "rb").read()

    def get(tid):
        off, size = struct.unpack_from("<QQ", raw, 16 + 16 * tid)
        return np.frombuffer(raw, np.uint8, size, off)

    w = {"embed": O.dequant_q8(get(LB.TID_EMBED).view(np.int8).reshape(V, H),
                               get(LB.TID_EMBED_SB).view(np.float16).reshape(V, H // 32)),
         "final_norm": get(LB.TID_FINAL_NORM).view(np.float32)}
    shapes = {"wqkv": (4096, 2048), "wo": (2048, 2048), "wgu": (12288, 2048), "wd": (2048, 6144)}
    for l in range(NL):
        for nm in ("attn_norm", "q_norm", "k_norm", "mlp_norm"):
            w[f"l{l}.{nm}"] = get(layer_tid(l, nm)).view(np.float32)
        for nm, (r, c) in shapes.items():
            w[f"l{l}.{nm}"] = O.dequant_q4s(get(layer_tid(l, nm)).reshape(r, c // 2),
                                            get(layer_tid(l, nm + "_sb")).view(np.float16).reshape(r, c // 32))
    del raw
    return w, O.TextModel(w)


GEMM_SHAPES = (("qkv", 4096, 2048), ("o", 2048, 2048), ("gate+up", 12288, 2048), ("down", 2048, 6144))


def run_gemm(args):
    """The prefill GEMMs alone (config 3 shapes, 1255 prompt rows): icua_gemm_f16 (the prefill
    route: fp16 weights by TMA) per layer matrix, back to back in a CUDA graph; TFLOP/s against
    the measured bf16 GEMM peak."""
    import ctypes as C

    import torch

    from instantcua_b200 import _lib as L

    torch.cuda.set_device(0)
    m = N_VIS + N_TEXT - 1
    peaks_d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    tpk = float(peaks_d.get("bf16_tflops", 1590.0))
    rows = []
    reps = max(args.steps, 10)
    for name, n, k in GEMM_SHAPES:
        w = (torch.randn(n, k, device="cuda") * 0.02).half()
        x = torch.randn(m, k, device="cuda").half()
        y = torch.empty(m, n, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")

        def run():
            s = torch.cuda.current_stream()
            L.check(L.lib().icua_gemm_f16(n, k, m, C.c_void_p(w.data_ptr()), C.c_void_p(x.data_ptr()),
                                          C.c_void_p(y.data_ptr()), C.c_void_p(err.data_ptr()),
                                          C.c_void_p(s.cuda_stream)))

        side = torch.cuda.Stream()
        with torch.cuda.stream(side):
            for _ in range(3):
                run()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                run()
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / reps
        tf = 2.0 * m * n * k / (us * 1e-6) / 1e12
        assert int(err.item()) == 0
        rows.append({"gemm": name, "m": m, "n": n, "k": k, "us": round(us, 2), "TFLOP/s": round(tf, 1),
                     "frac": round(tf / tpk, 4)})
    tot_f = sum(2.0 * r["m"] * r["n"] * r["k"] for r in rows)
    tot_us = sum(r["us"] for r in rows)
    print(json.dumps({"metric": "prefill GEMM TFLOP/s (config 3 shapes, fp16 operands)",
                      "value": round(tot_f / (tot_us * 1e-6) / 1e12, 1), "unit": "TFLOP/s", "n_gpus": 1,
                      "steps": reps, "peak": tpk, "peak_kind": "measured burst bf16", "shapes": rows}))


N_VIS, LLM_H, LLM_W, N_TEXT, PREFILL_DECODE = 1000, 25, 40, 256, 32
VIS_H, VIS_W = LLM_H * 32, LLM_W * 32  # the config-3 image: 800 x 1280 pixels, 50 x 80 patches


def vision_flops(n_patch: int) -> int:
    """Algorithmic FLOPs of one encode: 24 blocks of QKV / projection / MLP GEMMs (2 x 12.58 M
    weights per patch) and bidirectional attention (QK^T and PV: 4 n^2 x 1024), the patch
    embedding, and the four mergers (2 x 25.2 M weights per merged row)."""
    nv = n_patch // 4
    blocks = 24 * (2 * (3072 * 1024 + 1024 * 1024 + 4096 * 1024 + 1024 * 4096) * n_patch + 4 * n_patch * n_patch * 1024)
    return blocks + 2 * n_patch * 1024 * 768 + 4 * nv * 2 * (4096 * 4096 + 2048 * 4096)


def run_vision(args):
    """The vision encoder + mergers on a config-3 sized image (800 x 1280, 4000 patches, 1000 visual
    tokens) with seeded synthetic fp16 weights: value = patches per second of device time
    (CUDA events around the encode), roofline = algorithmic TFLOP/s against the measured
    sustained bf16 peak; e2e = icua_encode_vision from host RGB to host pooler / DeepStack rows."""
    import numpy as np
    import torch

    from instantcua_b200 import Engine, model

    torch.cuda.set_device(0)
    eng = Engine(max_context=64, max_pass=N_VIS, max_steps=8, kv_dtype="bf16")
    eng.set_tensors(model.synthetic_vision_fast(seed=7), ready=False)
    rgb = np.random.default_rng(5).integers(0, 256, (VIS_H, VIS_W, 3), dtype=np.uint8)
    K, W = args.steps, args.warmup
    for _ in range(max(W, 1)):
        eng.encode_vision(rgb)
    dev_ms, wall_ms = [], []
    with Clocks(0) as clk:
        for _ in range(K):
            t0 = time.perf_counter()
            pooler, ds = eng.encode_vision(rgb)
            wall_ms.append((time.perf_counter() - t0) * 1e3)
            dev_ms.append(eng.last_timing.vision_ms)
    eng.close()
    n_patch = (VIS_H // 16) * (VIS_W // 16)
    med = statistics.median(dev_ms)
    fl = vision_flops(n_patch)
    peaks_d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    tpk = float(peaks_d.get("bf16_tflops_sustained", 1400.0))
    ach = fl / (med / 1e3) / 1e12
    print(json.dumps({
        "metric": "vision encoder patches/s (config 3 image, 800x1280)", "value": round(n_patch / (med / 1e3), 1),
        "unit": "patches/s", "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": round(med, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 operands, fp32 accumulate (fp16 q/k/v, probabilities, GEMM inputs)",
        "data": "synthetic (seeded fp16 weights, uniform RGB8 image)",
        "config": {"workload": f"vision encoder + 3 DeepStack mergers + final merger, {n_patch} patches -> "
                               f"{n_patch // 4} visual rows", "image": [VIS_H, VIS_W]},
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": tpk, "unit": "TFLOP/s",
                     "frac": round(ach / tpk, 4), "traffic": None,
                     "note": f"{fl / 1e12:.3f} TFLOP per encode (GEMMs + attention + mergers); peak: measured sustained bf16"},
        "e2e": {"value": round(statistics.median(wall_ms), 2), "unit": "ms per image",
                "h2d_bytes_per_step": int(VIS_H * VIS_W * 3), "d2h_bytes_per_step": int(4 * pooler.size + 4 * ds.size),
                "api": "icua_encode_vision (host RGB8 in, host pooler + DeepStack rows out)"},
        "clocks": clk.summary(),
    }))
LAYER_PARAMS = {"qkv": 4096 * 2048, "o": 2048 * 2048, "gu": 12288 * 2048, "d": 2048 * 6144}


def prefill_flops(n: int) -> int:
    """Linear-layer FLOPs of the tensor-core prefill of an n-token prompt: rows 0..n-2 through all
    layers, except that the last layer only projects K/V (QKV GEMM); the last row runs as a
    decode step and is not counted."""
    rows = n - 1
    per_row = NL * LAYER_PARAMS["qkv"] + (NL - 1) * (LAYER_PARAMS["o"] + LAYER_PARAMS["gu"] + LAYER_PARAMS["d"])
    return 2 * rows * per_row


def config3_inputs(seed: int = 3):
    """1000 visual rows (pooler + 3 DeepStack tensors, N(0,1) rounded to bf16 values) on a 25 x 40
    merged grid at the start of the prompt, then 256 uniform text ids."""
    import numpy as np
    import torch

    rng = np.random.default_rng(seed)

    def bf16(a):
        return torch.from_numpy(a).to(torch.bfloat16).float().numpy()

    pooler = bf16(rng.standard_normal((N_VIS, H), dtype=np.float32))
    ds = [bf16(rng.standard_normal((N_VIS, H), dtype=np.float32)) for _ in range(3)]
    tokens = np.concatenate([np.full(N_VIS, 151655, np.int32), rng.integers(0, 151643, N_TEXT).astype(np.int32)])
    return tokens, pooler, ds


def run_prefill(args):
    """Config 3: multimodal prefill (1000 visual + 256 text rows, DeepStack at layers 0-2) through
    the tcgen05 dequant-GEMM path, then 32 greedy decode steps.  value = prefill tokens/s (device
    time of the prefill call); roofline = linear-layer TFLOP/s against the measured bf16 GEMM peak."""
    import torch

    from instantcua_b200 import Engine

    torch.cuda.set_device(0)
    path = model_file(0, None, 0)
    tokens, pooler, ds = config3_inputs()
    n = len(tokens)
    eng = Engine(path, max_context=n + PREFILL_DECODE + 64, max_pass=n, max_steps=PREFILL_DECODE + 8,
                 kv_dtype="f16", steps_per_graph=8)  # the reference's KV type
    eng.stop_on_eos = False
    K, W = args.steps, args.warmup
    for _ in range(W):
        eng.generate_vision(tokens, PREFILL_DECODE, pooler=pooler, deepstack=ds, grid=(LLM_H, LLM_W))
    pre_ms, dec_ms, wall_ms = [], [], []
    with Clocks(0) as clk:
        for _ in range(K):
            t0 = time.perf_counter()
            out = eng.generate_vision(tokens, PREFILL_DECODE, pooler=pooler, deepstack=ds, grid=(LLM_H, LLM_W))
            wall_ms.append((time.perf_counter() - t0) * 1e3)
            t = eng.last_timing
            pre_ms.append(t.prefill_ms)
            dec_ms.append(t.decode_ms)
    eng.close()
    pm = statistics.median(pre_ms)
    fl = prefill_flops(n)
    peaks_d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    tpk = float(peaks_d.get("bf16_tflops_sustained", 1400.0))
    ach = fl / (pm / 1e3) / 1e12
    print(json.dumps({
        "metric": "multimodal prefill tokens/s (config 3)", "value": round(n / (pm / 1e3), 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": round(pm, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 operands (q4s weights dequantised), fp32 accumulate",
        "data": "synthetic (seeded weights; N(0,1) bf16-valued visual rows)",
        "config": {"workload": f"config 3: {N_VIS} visual ({LLM_H}x{LLM_W}) + {N_TEXT} text rows, DeepStack, then "
                               f"{PREFILL_DECODE} greedy steps", "prompt_tokens": n},
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": tpk, "unit": "TFLOP/s",
                     "frac": round(ach / tpk, 4), "traffic": None,
                     "note": f"{fl / 1e12:.3f} TFLOP of linear layers per prefill over the whole prefill call "
                             "(GEMMs, attention, norms, and the last row's decode step); peak: measured sustained bf16"},
        "decode_ms_per_token": round(statistics.median(dec_ms) / PREFILL_DECODE, 4),
        "e2e": {"value": round(statistics.median(wall_ms), 2), "unit": "ms per request",
                "h2d_bytes_per_step": int(4 * N_VIS * H * 4 + n * 4), "d2h_bytes_per_step": 4 * PREFILL_DECODE,
                "api": "icua_generate (host pooler/DeepStack/tokens in, host tokens out)"},
        "generated": len(out), "clocks": clk.summary(),
    }))


BATCH_SESSIONS, BATCH_CTX, BATCH_STEPS = 64, 2048, 128


def run_batched(args):
    """Config 4: 64 concurrent sessions per GPU (2048-position random KV each), greedy decode of all
    of them together through the batched step (tensor-core GEMMs over the session rows,
    per-session attention, per-row argmax).  Under torchrun the job's 64 x N sessions are sharded
    round-robin over the N replicas (instantcua_b200.replicas: one engine per GPU, no collective
    while decoding, the counts and device times gathered at the end); value = tokens/s of the whole
    job over the slowest replica's time; roofline = HBM bytes of one replica's step (weights once +
    its sessions' KV) per second."""
    import numpy as np
    import torch

    from instantcua_b200 import Engine
    from instantcua_b200.replicas import decode_shard, local_sessions

    group = replica_group("nccl")
    world, rank, local = group.world, group.rank, group.local
    torch.cuda.set_device(local)
    path = model_file(local, group, local)
    n, K, W = BATCH_SESSIONS, args.steps, args.warmup
    ctx = args.batch_ctx  # config 4: 2048; smaller for profiler captures of the same GEMM shapes
    job = list(range(n * world))
    mine = local_sessions(job, group)
    eng = Engine(path, max_context=ctx + K + W + 64, max_pass=n, max_steps=K + W + 16, kv_dtype="bf16",
                 steps_per_graph=8, max_sessions=n, device=local)
    eng.stop_on_eos = False
    for g, s in mine.items():
        eng.inject_kv_random(ctx, seed=100 + g, session=s)
    toks = {g: int(t) for g, t in zip(job, np.random.default_rng(4).integers(0, 151643, len(job)))}
    decode_shard(eng, group, job, max(W, 1), in_tokens=toks)  # warm-up (graphs built, clocks up)
    ctx0 = eng.position(0)
    torch.cuda.synchronize()
    group.barrier()
    with Clocks(local) as clk:
        _, total, job_s = decode_shard(eng, group, job, K)
        ms = eng.last_timing.decode_ms
    eng.close()
    ms_step = ms / K
    ctx_mid = ctx0 + K / 2
    step_b = NL * Q4_LAYER_BYTES + Q8_HEAD_BYTES + NORM_BYTES + n * KV_BYTES_PER_POS * ctx_mid
    peak, peak_kind = peaks()
    ach = step_b / (ms_step / 1e3) / 1e9
    group.close()
    if rank != 0:
        return
    print(json.dumps({
        "metric": "batched decode tokens/s (config 4, 64 sessions x 2K ctx per GPU)", "value": round(total / job_s, 1),
        "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(job_s * 1e3 / K, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q4s/q8 weights as fp16 operands, fp32 accumulate, bf16 KV", "data": "synthetic (seeded weights, N(0,1) KV)",
        "config": {"workload": f"config 4: {n} sessions per GPU, KV pre-filled to {ctx} positions, {K} batched greedy steps",
                   "sessions": len(job), "context_range": [ctx0, ctx0 + K],
                   "parallelism": f"replicas x{world}, sessions sharded round-robin"},
        "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                     "traffic": None, "bytes_per_step": int(step_b),
                     "note": f"rank 0: weights once + {n} sessions' KV at ctx {int(ctx_mid)} per step; peak {peak_kind}"},
        "tokens_checked": int(total), "clocks": clk.summary(),
    }))


def run_probe(args):
    """A small decode run for profiler captures of the decode kernels (not a bench line of the
    headline): a synthetic model with --probe-layers decoder layers and --probe-vocab rows of tied
    embedding (default 16384: a smaller lm_head than the bench's), KV pre-filled to --probe-ctx bf16
    positions, then
    warm-up steps and --steps steps through the CUDA-graph path.  Prints the per-step time."""
    import torch

    from instantcua_b200 import Engine, model

    torch.cuda.set_device(0)
    nl, ctx, K, voc = args.probe_layers, args.probe_ctx, args.steps, args.probe_vocab
    t = model.quantize_stream(model.synthetic_fp32_fast(seed=SEED, n_layers=nl, vocab=voc))
    eng = Engine(tensors=t, n_layers=nl, vocab=voc, max_context=ctx + K + args.warmup + 64, max_pass=16,
                 max_steps=K + args.warmup + 16, kv_dtype="bf16", steps_per_graph=8)
    eng.stop_on_eos = False
    eng.inject_kv_random(ctx, seed=2)
    tok = eng.decode_step(5)
    eng.decode(max(args.warmup, 1))
    eng.decode(K)
    ms = eng.last_timing.decode_ms
    print(json.dumps({"probe": f"{nl} layers, ctx {ctx}, {K} steps", "ms_per_step": round(ms / K, 5),
                      "kernels_per_step": eng.kernels_per_step, "first_token": tok}))
    eng.close()


def host_blas_threads():
    """All host cores for the numpy oracle's BLAS, whatever OMP_NUM_THREADS torchrun exported."""
    from threadpoolctl import threadpool_limits

    cores = len(os.sched_getaffinity(0))
    return threadpool_limits(limits=cores), cores


def run_reference(args):
    """The reference's own CPU path (the numpy port of tools/reference/qwen3vl_ref.py): each step
    decodes one token at 4K context through a 4-of-28-layer sample plus 1/7 of the lm_head rows,
    so a token costs 7 steps; value = tokens/s."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    from oracle import qwen3vl_oracle as O

    rng = np.random.default_rng(0)
    n_layers = 4
    w = {k: v for k, v in O.generate_fp32_weights(seed=0, n_layers=n_layers, vocab=V // 7 // 16 * 16)}
    model = O.TextModel(w)
    kc = [rng.standard_normal((CTX, 8, 128), dtype=np.float32) for _ in range(n_layers)]
    vc = [rng.standard_normal((CTX, 8, 128), dtype=np.float32) for _ in range(n_layers)]
    model.inject_kv(kc, vc)
    limiter, cores = host_blas_threads()
    with limiter:
        for i in range(args.warmup):
            model.decode_step(i)
        t0 = time.perf_counter()
        for i in range(args.steps):
            model.decode_step(i)
        dt = time.perf_counter() - t0
    tok_s = args.steps / 7 / dt
    sample = (f"each step: 1 decode token through 4 of 28 layers + 1/7 of the lm_head rows at context {CTX}; "
              f"7 steps = 1 token; numpy fp32 oracle, BLAS on {cores} threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(tok_s, 4), "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) KV)",
        "config": {"workload": WORKLOAD, "model": "Qwen3-VL-2B text decoder (28 layers, random init)",
                   "seq_len": CTX, "parallelism": "the reference's CPU path on the host cores of rank 0",
                   "l2": "n/a (host run)"},
        "cpu_baseline": {"value": round(tok_s, 4), "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(tok_s, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--micro", action="store_true", help="config 1: per-shape GEMV microbench")
    ap.add_argument("--micro-shape", default="", help="run only the microbench shapes whose name contains this")
    ap.add_argument("--prefill", action="store_true", help="config 3: multimodal prefill through the GEMM path")
    ap.add_argument("--batched", action="store_true", help="config 4: 64 sessions decoded together")
    ap.add_argument("--gemm", action="store_true", help="the prefill GEMMs alone (config 3 shapes)")
    ap.add_argument("--vision", action="store_true", help="the vision encoder on a config-3 sized image")
    ap.add_argument("--probe", action="store_true", help="small decode run for profiler captures")
    ap.add_argument("--probe-layers", type=int, default=4)
    ap.add_argument("--probe-ctx", type=int, default=4096)
    ap.add_argument("--probe-vocab", type=int, default=16384)
    ap.add_argument("--batch-ctx", type=int, default=BATCH_CTX,
                    help="--batched: KV positions per session (config 4: 2048; smaller for ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3 and not (args.prefill or args.batched or args.micro or args.gemm or args.vision or args.probe):
        args.warmup = 3  # the headline bench always warms up; the side modes allow short profiling runs
    if args.impl == "reference":
        run_reference(args)
    elif args.micro:
        run_micro(args)
    elif args.prefill:
        run_prefill(args)
    elif args.batched:
        run_batched(args)
    elif args.gemm:
        run_gemm(args)
    elif args.vision:
        run_vision(args)
    elif args.probe:
        run_probe(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
