#!/usr/bin/env python3
"""Benchmark: batch-1 greedy decode (tok/s, % of HBM roofline) and 512-token
prefill of the Qwen2.5-3B-shaped synthetic Q4_K/Q6_K model on B200.

Workload (one "step"): prefill a 512-token seeded random prompt, then 256
greedy decode steps, batch 1 - the 3B configuration of the benchmark contract
(hidden 2048, 36 layers, 16/2 heads, FFN 11008, vocab 151936, tied Q6_K head).
Weights are generated from a fixed seed (no checkpoints or datasets exist on
the machine) and are 2.03 GB, far larger than L2, so every token streams them
from HBM.

  value      decode tok/s from CUDA events on the library's stream (device time
             of the generate calls), inputs resident on the GPU
  e2e        the same metric through the public C API with host buffers:
             host wall time around atlas_rt_prefill / atlas_rt_generate, which
             copy token ids in and picked ids (or logits) out every call
  roofline   algorithmic bytes of one decode step (all weights + the KV cache
             read at that position) / device time per token, against the
             measured HBM copy bandwidth in MEASURED_PEAKS.json
  cpu_baseline  the reference's own CPU runtime (src/brain_runtime.c compiled
             in place as oracle/_ref) on a bounded sample of the same workload

--impl reference runs only that CPU reference (all host cores it may use, the
reference caps its GEMV workers at 16) and prints its own JSON line.
Multi-GPU (torchrun, --gpus N): this model has 2 KV heads, so ranks run
independent replicas ("replicas only"): value = N * tokens / max-over-ranks time.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "-1.7-atlas---apollo_b200", "python"))

CFG = dict(hidden=2048, layers=36, q_heads=16, kv_heads=2, ffn=11008, vocab=151936, head_dim=128,
           context_length=32768, seed=1, tied=True)
PROMPT, GEN = 512, 256
METRIC = "decode tok/s (batch 1) & % HBM roofline; prefill tok/s at 512-token prompt"
Q4K, Q6K = 144.0 / 256.0, 210.0 / 256.0


def weight_bytes(c):
    H, qd, kvd, F, L, V = c["hidden"], c["q_heads"] * 128, c["kv_heads"] * 128, c["ffn"], c["layers"], c["vocab"]
    per_layer = (qd * H * Q4K + kvd * H * Q4K + kvd * H * Q6K + H * qd * Q4K + 2 * F * H * Q4K + H * F * Q6K
                 + 4 * (2 * H + qd + 2 * kvd))
    return L * per_layer + V * H * Q6K + 4 * H


def kv_bytes_per_position(c, kv_elem_bytes=4):
    return 2 * c["layers"] * c["kv_heads"] * 128 * kv_elem_bytes


def prefill_flops(c, T):
    """Algorithmic flops of a T-token prefill: linear layers 2T(2 q_dim H + 2 kv_dim H + 3 F H) per layer plus
    causal attention 4 n_q 128 T^2 / 2 per layer (the last token's head GEMV is a GEMV, not counted)."""
    H, qd, kvd, F, L = c["hidden"], c["q_heads"] * 128, c["kv_heads"] * 128, c["ffn"], c["layers"]
    return L * (2.0 * T * (2 * qd * H + 2 * kvd * H + 3 * F * H) + 4.0 * c["q_heads"] * 128 * T * T / 2.0)


def tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def model_path(rank):
    d = os.environ.get("ATLAS_BENCH_DIR", tempfile.gettempdir())
    return os.path.join(d, "atlas_bench_qwen25_3b_seed1.gguf")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    def __init__(self, gpu):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows if len(r) >= 9 for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


def cpu_reference_sample(path, n_decode=4, n_prompt=2):
    """The reference's own forward_token (oracle/_ref) on the host cores: a
    bounded sample of the workload (n_prompt prompt tokens, then n_decode
    greedy decode tokens); returns (decode tok/s, cores)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import numpy as np
    import oracle_bind
    cores = min(16, os.cpu_count() or 1)
    os.environ["ATLAS_REF_THREADS"] = str(cores)
    ref = oracle_bind.Reference.load()
    if ref is None:
        return None, cores, "oracle/_ref/libbrainref.so not built"
    r = ref.open(path)
    prompt = np.random.default_rng(0).integers(0, CFG["vocab"], n_prompt)
    lg = None
    for i, t in enumerate(prompt):
        lg = r.forward(int(t), i, i + 1 == n_prompt)
    nxt = r.greedy(lg)
    t0 = time.perf_counter()
    for s in range(n_decode):
        lg = r.forward(nxt, n_prompt + s)
        nxt = r.greedy(lg)
    dt = time.perf_counter() - t0
    r.close()
    return n_decode / dt, cores, f"{n_prompt} prompt tokens then {n_decode} greedy decode tokens of the 3B model"


def dist_setup(n_gpus):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        pg = dist
    return ws, rank, local, pg


def barrier(pg):
    if pg:
        pg.barrier()


def allmax(pg, v):
    if not pg:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def ensure_model(rank, pg):
    import atlas_cuda
    path = model_path(rank)
    if rank == 0 and not os.path.exists(path):
        tmp = path + ".tmp"
        atlas_cuda.write_synthetic_gguf(tmp, **CFG)
        os.replace(tmp, path)
    barrier(pg)
    return path


def run_reference(args):
    ws, rank, local, pg = dist_setup(args.gpus)
    path = ensure_model(rank, pg)
    if rank != 0:
        barrier(pg)
        return
    steps = []
    for i in range(args.warmup + args.steps):
        tps, cores, sample = cpu_reference_sample(path, n_decode=2, n_prompt=1)
        if tps is None:
            print(json.dumps({"impl": "reference", "unavailable": sample}))
            barrier(pg)
            return
        if i >= args.warmup:
            steps.append(tps)
    v = statistics.mean(steps)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(2000.0 / v, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random Q4_K/Q6_K weights)",
            "config": {"workload": "Qwen2.5-3B-shaped Q4_K/Q6_K, batch-1 greedy decode (CPU sample)"},
            "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": cores, "kind": "reference",
                             "sample": "per step: 1 prompt token then 2 greedy decode tokens of the 3B model"},
            "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    barrier(pg)


def run_ours(args):
    import numpy as np
    import atlas_cuda
    ws, rank, local, pg = dist_setup(args.gpus)
    path = ensure_model(rank, pg)
    rt = atlas_cuda.Runtime(path, device=local, max_context=PROMPT + GEN + 16, max_prefill=PROMPT)
    prompt = np.random.default_rng(1234).integers(0, CFG["vocab"], PROMPT).astype(np.uint32)

    def step():
        d0 = rt.stats()[2]
        t0 = time.perf_counter()
        _, first = rt.prefill(prompt, 0, want_logits=False)
        t1 = time.perf_counter()
        d1 = rt.stats()[2]
        ids = rt.generate(first, PROMPT, GEN)
        t2 = time.perf_counter()
        d2 = rt.stats()[2]
        return dict(prefill_dev=(d1 - d0) / 1e3, gen_dev=(d2 - d1) / 1e3, prefill_wall=t1 - t0, gen_wall=t2 - t1,
                    ids=ids)

    for _ in range(args.warmup):
        ref_ids = step()["ids"]
    barrier(pg)
    launches0 = rt.stats()[0]
    res = []
    with Clocks(local) as clk:
        barrier(pg)
        for _ in range(args.steps):
            r = step()
            assert np.array_equal(r["ids"], ref_ids), "greedy output changed between steps"
            res.append(r)
        barrier(pg)
    launches = rt.stats()[0] - launches0
    gen_dev = allmax(pg, sum(r["gen_dev"] for r in res))
    pre_dev = allmax(pg, sum(r["prefill_dev"] for r in res))
    gen_wall = allmax(pg, sum(r["gen_wall"] for r in res))
    pre_wall = allmax(pg, sum(r["prefill_wall"] for r in res))
    decode_tps = ws * args.steps * GEN / gen_dev
    prefill_tps = ws * args.steps * PROMPT / pre_dev
    e2e_decode = ws * args.steps * GEN / gen_wall
    # roofline of the decode step (a chain of HBM-bound kernels replayed as one graph per token)
    wb = weight_bytes(CFG)
    kv_avg = kv_bytes_per_position(CFG) * (PROMPT + GEN / 2.0)
    bytes_per_token = wb + kv_avg
    per_token_s = gen_dev / (args.steps * GEN)
    achieved = bytes_per_token / per_token_s / 1e9
    peak, peak_kind = peaks()
    tpeak, tpeak_kind = tensor_peak()
    pf_flops = prefill_flops(CFG, PROMPT)
    pf_tflops = pf_flops / (pre_dev / (ws * args.steps)) / 1e12
    traffic = None
    tf = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if os.path.exists(tf):
        try:
            traffic = json.load(open(tf)).get("dram_bytes_per_token")
        except Exception:
            traffic = None
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        tps, cores, sample = cpu_reference_sample(path)
        if tps is not None:
            cpu = {"value": round(tps, 4), "unit": "tok/s", "cores": cores, "kind": "reference", "sample": sample}
    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": round(decode_tps, 2), "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * (gen_dev + pre_dev) / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random Q4_K/Q6_K weights, random prompt ids)",
            "config": {"workload": "Qwen2.5-3B-shaped Q4_K/Q6_K (hidden 2048, 36 layers, 16/2 heads, FFN 11008, "
                                   "vocab 151936, tied Q6_K head): 512-token prefill + 256 greedy decode, batch 1",
                       "parallelism": f"replicas x{ws}" if ws > 1 else "1 GPU",
                       "l2": "inputs larger than L2 (2.03 GB of weights streamed per token)",
                       "kv_cache": "fp32"},
            "prefill_tok_s": round(prefill_tps, 2),
            "prefill_roofline": {"bound": "tensor", "achieved": round(pf_tflops, 1), "peak": tpeak, "unit": "TFLOP/s",
                                 "frac": round(pf_tflops / tpeak, 4), "peak_kind": tpeak_kind,
                                 "flops_per_prefill": pf_flops,
                                 "note": "algorithmic flops; the contraction computes hi.hi + lo.hi + hi.lo binary16 "
                                         "products (3x the tensor work) for fp32-level accuracy"},
            "decode_ms_per_token": round(1e3 * per_token_s, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "bytes_per_token": int(bytes_per_token),
                         "kernel": "decode step: CUDA graph of PDL-chained kernels (mv_kernel dequant-GEMVs, "
                                   "attn_kernel, embed, argmax); achieved = weight + KV bytes per token / device "
                                   "time per token"},
            "e2e": {"value": round(e2e_decode, 2), "unit": "tok/s", "h2d_bytes_per_step": PROMPT * 4 + 64,
                    "d2h_bytes_per_step": GEN * 4 + 64,
                    "prefill_tok_s": round(ws * args.steps * PROMPT / pre_wall, 2)},
            "gpu_launches": int(launches),
            "cpu_baseline": cpu,
            "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
        }
        print(json.dumps(line), flush=True)
    rt.close()
    barrier(pg)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
