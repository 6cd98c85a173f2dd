"""Benchmark of the BASELINE headline: q4 decode tokens/s at batch 1 and 4K context (config 2),
one independent replica per GPU (weak scaling), plus the HBM roofline of the dominant kernel and
the CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

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
SEED = 0
METRIC = "q4 decode tokens/s (batch 1, 4K ctx)"
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


def model_file(rank_local: int, dist, device: int) -> str:
    """Generates the seeded q4s model once per box (local rank 0) into /tmp and reuses it."""
    path = f"/tmp/icua_bench_seed{SEED}_q4s_v1.icua"
    if rank_local == 0 and not os.path.exists(path):
        from instantcua_b200 import model

        tensors = model.quantize_stream(model.synthetic_fp32_fast(seed=SEED, device=device))
        tmp = path + f".{os.getpid()}.tmp"
        model.write_icua(tmp, tensors)
        os.replace(tmp, path)
    if dist is not None:
        dist.barrier()
    return path


def run_ours(args):
    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
        dist = tdist
    torch.cuda.set_device(local)
    from instantcua_b200 import Engine
    from instantcua_b200 import _lib as L

    path = model_file(local, dist, local)
    K, W = args.steps, args.warmup
    eng = Engine(path, max_context=CTX + W + K + 2 * 64 + 64, max_pass=16, max_steps=W + K + 64, kv_dtype="bf16",
                 steps_per_graph=8, device=local)
    eng.stop_on_eos = False
    eng.inject_kv_random(CTX, seed=2 + rank)
    tok = int(np.random.default_rng(rank).integers(0, 151643))
    tok = eng.decode_step(tok)  # primes the session; position CTX + 1
    eng.decode(W)  # warm-up steps (graphs instantiated, clocks up)
    ctx0 = eng.position()

    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        eng.decode(K)
        ms = eng.last_timing.decode_ms
    torch.cuda.synchronize()
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_step = ms / K
    value = world * K / (ms / 1e3)

    # e2e through the public host API: one decode step per call, token in from host, token out
    # to host, synchronised each call (inputs and results cross PCIe every step).
    KE = min(K, 64)
    cur = eng.decode(1)[-1]
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(KE):
        cur = eng.decode_step(cur)
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * KE / e2e_s

    # roofline of the dominant kernel: the q8 lm_head dequant-GEMV (largest single stream, 330.6 MB),
    # timed alone with CUDA events on the launching stream; and the whole step for context.
    peak, peak_kind = peaks()
    roof = None
    if rank == 0:
        roof = lm_head_roofline(torch, L, peak)
    eng.close()

    ctx_mid = ctx0 + K / 2
    out = None
    if rank == 0:
        sb = step_bytes(int(ctx_mid))
        achieved_step = sb / (ms_step / 1e3) / 1e9
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4s/q8 weights, fp32 math, bf16 KV", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) KV)",
            "config": {"workload": "config 2: batch-1 q4 decode, KV pre-filled to 4096 positions, CUDA graph of 8 steps",
                       "model": "Qwen3-VL-2B text decoder (28 layers, random init)", "global_batch": world,
                       "seq_len": CTX, "context_range": [ctx0, ctx0 + K], "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2 (1.59 GB streamed per step)"},
            "roofline": roof,
            "step_roofline": {"bound": "hbm", "achieved": round(achieved_step, 1), "peak": peak, "unit": "GB/s",
                              "frac": round(achieved_step / peak, 4), "bytes_per_step": sb,
                              "note": f"whole decode token: weights + norms + KV at ctx {int(ctx_mid)}; peak {peak_kind}"},
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": 24, "d2h_bytes_per_step": 4,
                    "api": "icua_decode_step (host token in, host token out, synchronised per step)", "steps": KE},
            "gpu_launches": K * (5 * NL + 2),
            "clocks": clk.summary(),
        }
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        out["cpu_baseline"] = cpu_baseline(path)
    if rank == 0:
        print(json.dumps(out))


def lm_head_roofline(torch, L, peak):
    import ctypes as C

    import numpy as np

    n, k = V, 2048
    nbytes = L.lib().icua_packed_bytes(L.FMT_Q8, n, k)
    w = torch.randint(0, 255, (nbytes,), dtype=torch.uint8, device="cuda")
    # valid fp16 scales (1e-3) in every unit's scale block so the arithmetic is representative
    units = w.view(-1, 1088)
    units[:, 1024:] = torch.tensor([0x1419], dtype=torch.int16, device="cuda").view(torch.uint8).repeat(32)
    x = torch.randn(k, device="cuda")
    y = torch.empty(n, device="cuda")
    s = torch.cuda.current_stream()

    def run():
        L.check(L.lib().icua_gemv(L.FMT_Q8, n, k, C.c_void_p(w.data_ptr()), C.c_void_p(x.data_ptr()), 0,
                                  C.c_void_p(y.data_ptr()), C.c_void_p(s.cuda_stream)))

    for _ in range(5):
        run()
    reps = 50
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(s)
    for _ in range(reps):
        run()
    b.record(s)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    alg = nbytes + k * 4 + n * 4
    ach = alg / (ms / 1e3) / 1e9
    return {"kernel": "gemv_kernel<q8,store> lm_head 151936x2048", "bound": "hbm", "achieved": round(ach, 1),
            "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4), "traffic": None,
            "algorithmic_bytes": alg, "ms_per_launch": round(ms, 5)}


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
    model.decode_step(1)  # warm-up
    t1 = time.perf_counter()
    for i in range(steps):
        model.decode_step(100 + i)
    dt = time.perf_counter() - t1
    return {"value": round(steps / dt, 4), "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)), "kind": "port",
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
    for i in range(args.warmup):
        model.decode_step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        model.decode_step(i)
    dt = time.perf_counter() - t0
    tok_s = args.steps / 7 / dt
    cores = len(os.sched_getaffinity(0))
    sample = (f"each step: 1 decode token through 4 of 28 layers + 1/7 of the lm_head rows at context {CTX}; "
              f"7 steps = 1 token; numpy fp32 oracle, BLAS on {cores} threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(tok_s, 4), "unit": "tokens/s", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) KV)",
        "config": {"workload": "config 2: batch-1 decode at 4K context (CPU reference path)", "seq_len": CTX},
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
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
