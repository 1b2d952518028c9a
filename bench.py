#!/usr/bin/env python3
"""Benchmark: batch-1 greedy decode (tok/s, fraction of the HBM roofline) and
512-token batched prefill (tok/s, fraction of the bf16 tensor roofline) of the
Qwen2.5-7B-shaped synthetic Q4_K/Q6_K model on B200.

Workload (one "step"): prefill a 512-token seeded random prompt, then 256
greedy decode steps at batch 1 (hidden 3584, 28 layers, 28 query / 4 KV
heads, FFN 18944, vocab 152064, untied Q6_K head, fp32 KV cache). Weights are
generated from a fixed seed (no checkpoints or datasets exist on the machine):
4.62 GB, far larger than L2, so every token streams them from HBM.

  value      decode tok/s from CUDA events on the library's stream (device time
             of the generate calls), inputs resident on the GPU
  e2e        the same metric through the public C API with host buffers: host
             wall time around atlas_rt_prefill / atlas_rt_generate, which copy
             the token ids in and the picked ids out on every call
  roofline   algorithmic bytes of one decode step (all weights + the KV cache
             read at that position) / device time per token, against the
             measured HBM copy bandwidth (MEASURED_PEAKS.json)
  parity     the first 32 greedy picks against the reference's own run of the
             same prompt (tests/golden/cfg2.npz, made by the reference itself)
  cpu_baseline  the reference's own CPU runtime (src/brain_runtime.c compiled in
             place as oracle/_ref) on the box's host cores: decode at the same
             positions as the GPU arm (512 onwards) and prompt tokens, on a
             bounded sample

Multi-GPU (torchrun, --gpus N): the 7B model is tensor-parallel over its 4 KV
heads. N = 2 and 4 run one tensor-parallel group of N ranks; N = 8 runs two
groups of 4 (each decodes its own copy of the workload). value = groups x
tokens / max-over-ranks device time.

--shape 14b: the long-context workload instead (Qwen2.5-14B shape, 48 layers,
40 / 8 heads, FFN 13824: an 8192-token prompt, then 512 greedy decode steps),
tensor-parallel over up to 8 GPUs (its 8 KV heads).

--impl reference runs only the CPU reference (rank 0; other ranks exit) and
prints its own JSON line; it never loads libatlas_cuda.so (its model file
comes from the writer built into oracle/liboracle.so).
"""
import argparse
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
sys.path.insert(0, os.path.join(ROOT, "tests"))

CFG2 = dict(hidden=3584, layers=28, q_heads=28, kv_heads=4, ffn=18944, vocab=152064, context_length=32768, seed=2,
            tied=False)
CFG1 = dict(hidden=2048, layers=36, q_heads=16, kv_heads=2, ffn=11008, vocab=151936, context_length=32768, seed=1,
            tied=True)
WORKLOAD = {
    "cfg2": "Qwen2.5-7B-shaped Q4_K/Q6_K (hidden 3584, 28 layers, 28/4 heads, FFN 18944, vocab 152064, untied Q6_K "
            "head): 512-token prefill + 256 greedy decode, batch 1",
    "cfg1": "Qwen2.5-3B-shaped Q4_K/Q6_K (hidden 2048, 36 layers, 16/2 heads, FFN 11008, vocab 151936, tied Q6_K "
            "head): 512-token prefill + 256 greedy decode, batch 1",
}
# The long-context workload (--shape 14b): Qwen2.5-14B shape, an 8192-token prompt through the batched
# prefill, then 512 greedy decode steps; tensor-parallel over up to 8 GPUs (8 KV heads).
CFG3 = dict(hidden=5120, layers=48, q_heads=40, kv_heads=8, ffn=13824, vocab=152064, context_length=32768, seed=3,
            tied=False)
WORKLOAD["cfg3"] = ("Qwen2.5-14B-shaped Q4_K/Q6_K (hidden 5120, 48 layers, 40/8 heads, FFN 13824, vocab 152064, untied "
                    "Q6_K head): 8192-token prefill + 512 greedy decode over a binary16 KV cache, batch 1")
# the workloads whose KV cache is binary16 (the long-context one stresses split-K decode over a full fp16 cache)
FP16_CACHE = {"cfg3"}
LONG_PROMPT, LONG_GEN = 8192, 512
# The 8-sequence workload (--workload 32b-batch8): Qwen2.5-32B shape, 8 independent sequences, each a
# 2048-token prompt prefilled batched, then 256 decode steps at batch 8 (all sequences in one step).
CFG4 = dict(hidden=5120, layers=64, q_heads=40, kv_heads=8, ffn=27648, vocab=152064, context_length=32768, seed=4,
            tied=False)
WORKLOAD["cfg4"] = ("Qwen2.5-32B-shaped Q4_K/Q6_K (hidden 5120, 64 layers, 40/8 heads, FFN 27648, vocab 152064, untied "
                    "Q6_K head): 8 independent sequences, each a 2048-token prefill, then 256 decode steps at batch 8")
B8_SEQ, B8_PROMPT, B8_GEN = 8, 2048, 256
PROMPT, GEN, PROMPT_SEED = 512, 256, 1234
METRIC = "decode tok/s (batch 1) & % HBM roofline; prefill tok/s at 512-token prompt"
Q4K, Q6K = 144.0 / 256.0, 210.0 / 256.0


def weight_bytes(c, sl=None):
    """Algorithmic weight bytes of one decode step (of one tensor-parallel rank when sl is its slice)."""
    H, L, V = c["hidden"], c["layers"], c["vocab"]
    qd, kvd, F = c["q_heads"] * 128, c["kv_heads"] * 128, c["ffn"]
    if sl is None:
        per_layer = (qd * H * Q4K + kvd * H * Q4K + kvd * H * Q6K + H * qd * Q4K + 2 * F * H * Q4K + H * F * Q6K
                     + 4 * (2 * H + qd + 2 * kvd))
        return L * per_layer + V * H * Q6K + 4 * H
    lq, lkv = sl["q_heads"] * 128, sl["kv_heads"] * 128
    per_layer = ((lq + lkv) * H * Q4K + lkv * H * Q6K + H * sl["o_blocks"] * 256 * Q4K + 2 * sl["ffn_rows"] * H * Q4K
                 + H * sl["ffn_rows"] * Q6K + 4 * (2 * H + lq + 2 * lkv))
    return L * per_layer + sl["vocab_rows"] * H * Q6K + 4 * H


def kv_bytes_per_position(c, kv_heads=None, elem=4):
    return 2 * c["layers"] * (kv_heads or c["kv_heads"]) * 128 * elem


def prefill_flops(c, T):
    """Algorithmic flops of a T-token prefill: linear layers 2T(2 q_dim H + 2 kv_dim H + 3 F H) per layer plus
    causal attention 4 n_q 128 T^2 / 2 per layer (the last token's head GEMV is a GEMV, not counted)."""
    H, qd, kvd, F, L = c["hidden"], c["q_heads"] * 128, c["kv_heads"] * 128, c["ffn"], c["layers"]
    return L * (2.0 * T * (2 * qd * H + 2 * kvd * H + 3 * F * H) + 4.0 * c["q_heads"] * 128 * T * T / 2.0)


def measured(key, fallback):
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)[key]), "measured"
    except Exception:
        return fallback, "fallback"


def model_path(name):
    d = os.environ.get("ATLAS_BENCH_DIR", tempfile.gettempdir())
    return os.path.join(d, f"atlas_bench_{name}.gguf")


def prompt_ids(cfg):
    import numpy as np
    return np.random.default_rng(PROMPT_SEED).integers(0, cfg["vocab"], PROMPT).astype(np.uint32)


def golden_picks(name, cfg):
    """The reference's 32 greedy picks after this prompt, if the fixture exists and matches the model."""
    import numpy as np
    p = os.path.join(ROOT, "tests", "golden", f"{name}.npz")
    if not os.path.exists(p):
        return None
    g = np.load(p)
    same = all(int(g[f"cfg_{k}"]) == int(v) for k, v in cfg.items() if f"cfg_{k}" in g.files)
    if not same or int(g["tied"]) != int(cfg["tied"]) or not np.array_equal(g["prompt"], prompt_ids(cfg)):
        return None
    return g["picks"]


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


# ------------------------------------------------------------------ CPU side --

def ref_threads():
    """All host threads; the reference itself caps its GEMV workers at 16 (src/brain_runtime.c:1172)."""
    n = os.cpu_count() or 1
    return n, min(16, n)


def cpu_reference_sample(path, cfg, n_decode, n_prompt, pos=None):
    """The reference's own forward_token (oracle/_ref) on the host cores.
    Prompt rate: n_prompt tokens without logits, as the reference's own prompt
    loop runs them (src/brain_runtime.c:2025-2028). Decode rate: the cache is
    filled to PROMPT positions by repeating those rows (the work of a decode
    step does not depend on the cached values), then n_decode greedy steps at
    positions PROMPT.. as the GPU arm decodes them. Returns a dict or None."""
    import numpy as np
    import oracle_bind
    host, used = ref_threads()
    os.environ["ATLAS_REF_THREADS"] = str(host)
    ref = oracle_bind.Reference.load()
    if ref is None:
        return None
    pos = PROMPT if pos is None else pos
    r = ref.open(path)
    prompt = prompt_ids(cfg)[:n_prompt]
    t0 = time.perf_counter()
    for i, t in enumerate(prompt):
        r.forward(int(t), i, False)
    t_prompt = time.perf_counter() - t0
    r.fill_cache(n_prompt, pos)
    nxt = int(prompt[-1])
    t0 = time.perf_counter()
    for s in range(n_decode):
        lg = r.forward(nxt, pos + s, True)
        nxt = r.greedy(lg)
    t_dec = time.perf_counter() - t0
    r.close()
    return {"decode_tok_s": n_decode / t_dec, "prefill_tok_s": n_prompt / t_prompt, "host_cores": host,
            "gemv_threads": used}


def ensure_model_oracle_writer(name, cfg):
    import oracle_bind
    path = model_path(name)
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        oracle_bind.write_synthetic_gguf(tmp, **cfg)
        os.replace(tmp, path)
    return path


SHAPES = {"3b": ("cfg1", CFG1), "7b": ("cfg2", CFG2), "14b": ("cfg3", CFG3)}


def run_reference(args):
    """CPU reference arm: rank 0 only; other ranks exit at once without work. The workload of --shape, decoded at
    the positions the GPU arm decodes (after a PROMPT-position cache)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    name, cfg = SHAPES[args.shape]
    path = ensure_model_oracle_writer(name, cfg)
    dec, pre = [], []
    smp = None
    for i in range(args.warmup + args.steps):
        smp = cpu_reference_sample(path, cfg, n_decode=2, n_prompt=2)
        if smp is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libbrainref.so was not built "
                                                                  "(the reference sources were absent at build time)"}))
            return
        if i >= args.warmup:
            dec.append(smp["decode_tok_s"])
            pre.append(smp["prefill_tok_s"])
    v = statistics.mean(dec)
    sample = (f"per step: 2 prompt tokens (token at a time, no logits), then 2 greedy decode tokens at positions "
              f"{PROMPT}-{PROMPT + 1} over a {PROMPT}-position cache, {args.shape.upper()} shape; "
              f"{smp['host_cores']} host threads, {smp['gemv_threads']} GEMV workers (the reference's cap)")
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(2000.0 / v + 2000.0 / statistics.mean(pre), 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random Q4_K/Q6_K weights, random prompt ids)",
            "config": {"workload": WORKLOAD[name] + " (CPU: bounded sample)", "parallelism": "CPU threads",
                       "kv_cache": "fp32"},
            "prefill_tok_s": round(statistics.mean(pre), 4),
            "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": smp["gemv_threads"],
                             "host_cores": smp["host_cores"], "kind": "reference", "sample": sample,
                             "prefill_tok_s": round(statistics.mean(pre), 4)},
            "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU side --

def dist_setup():
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


def tp_layout(ws, kv_heads=4):
    """(tensor-parallel size, groups) for N ranks: one group over up to kv_heads ranks (the 7B model's 4, the
    14B's 8), else groups of kv_heads ranks that each decode their own copy of the workload."""
    if ws <= kv_heads:
        return ws, 1
    if ws % kv_heads:
        raise SystemExit(f"--gpus {ws}: the model is tensor-parallel over up to {kv_heads} ranks; use a divisor "
                         f"or a multiple of {kv_heads}")
    return kv_heads, ws // kv_heads


def run_model(name, cfg, rt, steps, warmup, pg, clocks_gpu=None):
    """Times `steps` workload steps (prefill + GEN decode) after `warmup`; returns per-rank sums."""
    import numpy as np
    prompt = prompt_ids(cfg)

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
                    ids=np.concatenate([[first], ids]).astype(np.uint32))

    ref_ids = None
    for _ in range(warmup):
        ref_ids = step()["ids"]
    barrier(pg)
    launches0 = rt.stats()[0]
    res = []
    clk = Clocks(clocks_gpu) if clocks_gpu is not None else None
    if clk:
        clk.__enter__()
    try:
        barrier(pg)
        for _ in range(steps):
            r = step()
            if ref_ids is not None and not np.array_equal(r["ids"], ref_ids):
                raise AssertionError(f"{name}: greedy output changed between steps")
            ref_ids = r["ids"]
            res.append(r)
        barrier(pg)
    finally:
        if clk:
            clk.__exit__(None, None, None)
    out = {k: sum(r[k] for r in res) for k in ("gen_dev", "prefill_dev", "gen_wall", "prefill_wall")}
    out["launches"] = rt.stats()[0] - launches0
    out["ids"] = ref_ids
    out["clocks"] = clk.summary() if clk else None
    return out


def summarize(name, cfg, r, steps, pg, groups, sl=None, tp=1):
    """Whole-job rates (max over ranks) and the roofline of the decode step."""
    gen_dev, pre_dev = allmax(pg, r["gen_dev"]), allmax(pg, r["prefill_dev"])
    gen_wall, pre_wall = allmax(pg, r["gen_wall"]), allmax(pg, r["prefill_wall"])
    decode_tps = groups * steps * GEN / gen_dev
    per_token_s = gen_dev / (steps * GEN)
    kv_heads = sl["kv_heads"] if sl else cfg["kv_heads"]
    elem = 2 if name.split("_")[0] in FP16_CACHE else 4
    kv_avg = kv_bytes_per_position(cfg, kv_heads, elem) * (PROMPT + GEN / 2.0)
    rank_bytes = weight_bytes(cfg, sl) + kv_avg             # one rank's algorithmic bytes per token
    total_bytes = weight_bytes(cfg) + kv_bytes_per_position(cfg, None, elem) * (PROMPT + GEN / 2.0)
    hbm, hbm_kind = measured("hbm_gbs", 6650.0)
    tpk, tpk_kind = measured("bf16_tflops", 1590.0)
    rank_gbs = rank_bytes / per_token_s / 1e9
    pf_tflops = prefill_flops(cfg, PROMPT) / (pre_dev / steps) / 1e12 / tp   # per GPU of a group
    golden = golden_picks(name, cfg)
    parity = None
    if golden is not None and r["ids"] is not None:
        n = min(len(golden), len(r["ids"]))
        parity = {"picks_checked": int(n), "picks_match_reference": bool((r["ids"][:n] == golden[:n]).all()),
                  "fixture": f"tests/golden/{name}.npz"}
    return {
        "decode_tok_s": decode_tps, "prefill_tok_s": groups * steps * PROMPT / pre_dev,
        "decode_ms_per_token": 1e3 * per_token_s, "ms_per_step": 1e3 * (gen_dev + pre_dev) / steps,
        "e2e_decode_tok_s": groups * steps * GEN / gen_wall, "e2e_prefill_tok_s": groups * steps * PROMPT / pre_wall,
        "roofline": {"bound": "hbm", "achieved": round(rank_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(rank_gbs / hbm, 4), "peak_kind": hbm_kind,
                     "bytes_per_token": int(rank_bytes), "traffic": None,
                     "traffic_note": "not re-measured in the timed run; ncu captures of one 7B-shape layer's "
                                     "GEMV launches read within 1 % of their algorithmic bytes "
                                     "(profiles/mv4_kernel_qkv_o_gateup_down_7b_shape_two_layers.md)",
                     "kernel": "decode step: CUDA graph of PDL-chained kernels (mv4_kernel dequant-GEMVs, attention, "
                               "embed, argmax); achieved = one GPU's weight + KV bytes per token / device time per "
                               "token"},
        "prefill_roofline": {"bound": "tensor", "achieved": round(pf_tflops, 1), "peak": tpk, "unit": "TFLOP/s",
                             "frac": round(pf_tflops / tpk, 4), "peak_kind": tpk_kind,
                             "flops_per_prefill": prefill_flops(cfg, PROMPT),
                             "note": "algorithmic flops per GPU; the contraction computes hi.hi + lo.hi + hi.lo "
                                     "binary16 products (3x the tensor work) for fp32-level accuracy"},
        "total_bytes_per_token": int(total_bytes),
        "parity": parity,
    }


def ensure_model_product_writer(name, cfg, rank, pg):
    import atlas_cuda
    path = model_path(name)
    if rank == 0 and not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        atlas_cuda.write_synthetic_gguf(tmp, **cfg)
        os.replace(tmp, path)
    barrier(pg)
    return path


def run_ours(args):
    import atlas_cuda
    ws, rank, local, pg = dist_setup()
    name, cfg = SHAPES[args.shape]
    if args.layers:
        # profiles on a small case: the same launch shapes, fewer layers (no reference fixture applies)
        name, cfg = f"{name}_l{args.layers}", dict(cfg, layers=args.layers)
        WORKLOAD[name] = WORKLOAD[name.split("_")[0]] + f" (cut to {args.layers} layers)"
    tp, groups = tp_layout(ws, cfg["kv_heads"])
    group_id, tp_rank = rank // tp, rank % tp
    tp_group = None
    if pg and groups > 1:
        subgroups = [pg.new_group(list(range(g * tp, (g + 1) * tp))) for g in range(groups)]
        tp_group = subgroups[group_id]
    path = ensure_model_product_writer(name, cfg, rank, pg)
    fp16 = name.split("_")[0] in FP16_CACHE
    rt = atlas_cuda.Runtime(path, device=local, max_context=PROMPT + GEN + 16, max_prefill=PROMPT,
                            tp_rank=tp_rank, tp_size=tp, kv_fp16=fp16)
    if tp > 1:
        atlas_cuda.connect_tp(rt, group=tp_group)
    barrier(pg)
    sl = rt.tp_slice().as_dict() if tp > 1 else None
    r = run_model(name, cfg, rt, args.steps, args.warmup, pg, clocks_gpu=local if rank == 0 else None)
    s = summarize(name, cfg, r, args.steps, pg, groups, sl, tp)
    rt.close()
    barrier(pg)
    if ws == 1 and s["parity"] is not None and not s["parity"]["picks_match_reference"]:
        raise SystemExit(f"greedy picks differ from the reference's (tests/golden/{name}.npz): {list(r['ids'][:32])}")
    secondary, cpu = None, None
    if ws == 1 and not args.no_secondary and name == "cfg2":
        p1 = ensure_model_product_writer("cfg1", CFG1, rank, pg)
        with atlas_cuda.Runtime(p1, device=local, max_context=PROMPT + GEN + 16, max_prefill=PROMPT) as rt1:
            r1 = run_model("cfg1", CFG1, rt1, args.steps, args.warmup, pg)
            s1 = summarize("cfg1", CFG1, r1, args.steps, pg, 1)
        if s1["parity"] is not None and not s1["parity"]["picks_match_reference"]:
            raise SystemExit(f"greedy picks differ from the reference's (tests/golden/cfg1.npz): {list(r1['ids'][:32])}")
        secondary = {"workload": WORKLOAD["cfg1"], "decode_tok_s": round(s1["decode_tok_s"], 2),
                     "decode_ms_per_token": round(s1["decode_ms_per_token"], 4),
                     "prefill_tok_s": round(s1["prefill_tok_s"], 1), "roofline_frac": s1["roofline"]["frac"],
                     "prefill_roofline_frac": s1["prefill_roofline"]["frac"],
                     "e2e_decode_tok_s": round(s1["e2e_decode_tok_s"], 2), "parity": s1["parity"],
                     "gpu_launches": int(r1["launches"])}
    if ws == 1 and not args.no_cpu_baseline:
        c = cpu_reference_sample(model_path(name), cfg, n_decode=3, n_prompt=3)
        if c is not None:
            cpu = {"value": round(c["decode_tok_s"], 4), "unit": "tok/s", "cores": c["gemv_threads"],
                   "host_cores": c["host_cores"], "kind": "reference",
                   "prefill_tok_s": round(c["prefill_tok_s"], 4),
                   "sample": f"3 prompt tokens (token at a time, no logits), then 3 greedy decode tokens at positions "
                             f"{PROMPT}-{PROMPT + 2} over a {PROMPT}-position cache, {args.shape.upper()} shape"}
    if rank == 0:
        clocks = r["clocks"] or {}
        par = f"tp{tp}" if groups == 1 else f"tp{tp} x {groups} groups"
        line = {
            "metric": METRIC, "value": round(s["decode_tok_s"], 2), "unit": "tok/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(s["ms_per_step"], 3),
            "higher_is_better": True, "scaling": "strong" if groups == 1 and ws > 1 else "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random Q4_K/Q6_K weights, random prompt ids)",
            "config": {"workload": WORKLOAD[name], "parallelism": par if ws > 1 else "1 GPU",
                       "l2": f"inputs larger than L2 ({weight_bytes(cfg) / 1e9:.2f} GB of weights streamed per token)",
                       "kv_cache": "fp16" if fp16 else "fp32"},
            "decode_ms_per_token": round(s["decode_ms_per_token"], 4),
            "prefill_tok_s": round(s["prefill_tok_s"], 1),
            "roofline": s["roofline"],
            "prefill_roofline": s["prefill_roofline"],
            "e2e": {"value": round(s["e2e_decode_tok_s"], 2), "unit": "tok/s", "h2d_bytes_per_step": PROMPT * 4 + 4,
                    "d2h_bytes_per_step": GEN * 4 + 4, "prefill_tok_s": round(s["e2e_prefill_tok_s"], 1)},
            "parity": s["parity"],
            "gpu_launches": int(r["launches"]),
            "cpu_baseline": cpu,
            "secondary": secondary,
            "clocks": {k: clocks.get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons")},
        }
        if tp > 1:
            line["tensor_parallel"] = {"tp": tp, "groups": groups, "rank0_slice": sl,
                                       "per_gpu_gbs": s["roofline"]["achieved"],
                                       "aggregate_gbs": round(s["roofline"]["achieved"] * ws, 1)}
        print(json.dumps(line), flush=True)
    barrier(pg)
    if pg:
        pg.destroy_process_group()


def run_batch8(args):
    """The 32B-shaped 8-sequence workload on one GPU: every sequence's prompt through the batched prefill
    (atlas_cuda_prefill_seq), then B8_GEN steps of all 8 sequences at once (atlas_cuda_generate_batch). value =
    aggregate decode tok/s (8 tokens per step). Consistency: sequence 0's batch-8 picks equal its batch-1 picks
    from the same prefill."""
    import numpy as np
    import atlas_cuda
    cfg4 = dict(CFG4, layers=args.layers) if args.layers else CFG4
    name4 = "cfg4" if not args.layers else f"cfg4_l{args.layers}"
    path = ensure_model_product_writer(name4, cfg4, 0, None)
    V = cfg4["vocab"]
    prompts = [np.random.default_rng(PROMPT_SEED + s).integers(0, V, B8_PROMPT).astype(np.uint32)
               for s in range(B8_SEQ)]
    with atlas_cuda.Runtime(path, max_context=B8_PROMPT + B8_GEN + 16, max_prefill=B8_PROMPT,
                            max_batch=B8_SEQ) as rt:
        def step():
            d0, t0 = rt.stats()[2], time.perf_counter()
            first = [rt.prefill_seq(s, prompts[s], 0, want_logits=False)[1] for s in range(B8_SEQ)]
            d1, t1 = rt.stats()[2], time.perf_counter()
            ids = rt.generate_batch(first, [B8_PROMPT] * B8_SEQ, B8_GEN)
            d2, t2 = rt.stats()[2], time.perf_counter()
            return dict(pre_dev=(d1 - d0) / 1e3, gen_dev=(d2 - d1) / 1e3, pre_wall=t1 - t0, gen_wall=t2 - t1,
                        first=first, ids=ids)
        ref = None
        for _ in range(args.warmup):
            ref = step()
        launches0 = rt.stats()[0]
        res = []
        with Clocks(0) as clk:
            for _ in range(args.steps):
                r = step()
                if ref is not None and not np.array_equal(r["ids"], ref["ids"]):
                    raise AssertionError("32b-batch8: greedy output changed between steps")
                ref = r
                res.append(r)
        launches = rt.stats()[0] - launches0
        # sequence 0 alone at batch 1 from the same prompt
        _, f0 = rt.prefill_seq(0, prompts[0], 0, want_logits=False)
        nchk = min(32, B8_GEN)
        single = rt.generate(f0, B8_PROMPT, nchk)
        consistent = bool(f0 == ref["first"][0] and np.array_equal(single, ref["ids"][0][:nchk]))
    gen_dev = sum(r["gen_dev"] for r in res)
    pre_dev = sum(r["pre_dev"] for r in res)
    gen_wall = sum(r["gen_wall"] for r in res)
    pre_wall = sum(r["pre_wall"] for r in res)
    steps_s = gen_dev / (args.steps * B8_GEN)
    kv_step = kv_bytes_per_position(cfg4) * (B8_PROMPT + B8_GEN / 2.0) * B8_SEQ
    step_bytes = weight_bytes(cfg4) + kv_step
    hbm, hbm_kind = measured("hbm_gbs", 6650.0)
    tpk, tpk_kind = measured("bf16_tflops", 1590.0)
    gbs = step_bytes / steps_s / 1e9
    pf_tflops = prefill_flops(cfg4, B8_PROMPT) * B8_SEQ * args.steps / pre_dev / 1e12
    c = clk.summary()
    cpu = None
    if not args.no_cpu_baseline:
        smp = cpu_reference_sample(path, cfg4, n_decode=2, n_prompt=1, pos=B8_PROMPT)
        if smp is not None:
            cpu = {"value": round(smp["decode_tok_s"], 4), "unit": "tok/s", "cores": smp["gemv_threads"],
                   "host_cores": smp["host_cores"], "kind": "reference",
                   "sample": f"one sequence (the reference decodes one per process): 1 prompt token, then 2 greedy "
                             f"decode tokens at positions {B8_PROMPT}-{B8_PROMPT + 1} over a {B8_PROMPT}-position "
                             f"cache, 32B shape"}
    line = {
        "metric": "aggregate decode tok/s at batch 8 (8 sequences per step) & % HBM roofline; prefill tok/s",
        "value": round(args.steps * B8_GEN * B8_SEQ / gen_dev, 2), "unit": "tok/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * (gen_dev + pre_dev) / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random Q4_K/Q6_K weights, random prompt ids)",
        "config": {"workload": WORKLOAD["cfg4"] + (f" ({args.layers} layers)" if args.layers else ""),
                   "parallelism": "1 GPU",
                   "l2": f"inputs larger than L2 ({weight_bytes(cfg4) / 1e9:.2f} GB of weights per step)",
                   "kv_cache": "fp32"},
        "decode_ms_per_step": round(1e3 * steps_s, 4),
        "prefill_tok_s": round(args.steps * B8_SEQ * B8_PROMPT / pre_dev, 1),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4),
                     "peak_kind": hbm_kind, "bytes_per_step": int(step_bytes), "traffic": None,
                     "kernel": "batched decode step: CUDA graph of mvb_kernel GEMVs (8 sequence columns), reduce, "
                               "residual and attention kernels; achieved = weights + 8 sequences' KV bytes per step / "
                               "device time per step"},
        "prefill_roofline": {"bound": "tensor", "achieved": round(pf_tflops, 1), "peak": tpk, "unit": "TFLOP/s",
                             "frac": round(pf_tflops / tpk, 4), "peak_kind": tpk_kind},
        "e2e": {"value": round(args.steps * B8_GEN * B8_SEQ / gen_wall, 2), "unit": "tok/s",
                "h2d_bytes_per_step": B8_SEQ * (B8_PROMPT * 4 + 8), "d2h_bytes_per_step": B8_SEQ * (B8_GEN * 4 + 4),
                "prefill_tok_s": round(args.steps * B8_SEQ * B8_PROMPT / pre_wall, 1)},
        "consistency": {"sequence0_batch8_equals_batch1_picks": consistent, "picks_checked": nchk},
        "gpu_launches": int(launches),
        "cpu_baseline": cpu,
        "clocks": {k: c.get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons")},
    }
    print(json.dumps(line), flush=True)
    if not consistent:
        raise SystemExit("32b-batch8: sequence 0's batch-8 picks differ from its batch-1 picks")


def main():
    global GEN, PROMPT
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the 3B workload at N=1")
    ap.add_argument("--shape", default="7b", choices=["7b", "3b", "14b"],
                    help="the headline workload's model shape (3b: the secondary workload alone, e.g. for profiles; "
                         "14b: the long-context workload, an 8192-token prompt and 512 decode steps)")
    ap.add_argument("--gen", type=int, default=None, help="greedy decode steps per workload step (profiles: fewer)")
    ap.add_argument("--workload", default="default", choices=["default", "32b-batch8"],
                    help="32b-batch8: the 8-sequence 32B-shaped workload (one GPU)")
    ap.add_argument("--layers", type=int, default=0, help="fewer layers (profiles on a small case)")
    args = ap.parse_args()
    if args.shape == "14b":
        PROMPT, GEN = LONG_PROMPT, LONG_GEN
    if args.gen is not None:
        GEN = args.gen
    if args.workload == "32b-batch8":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "32b-batch8: the reference decodes one sequence "
                              "per process; its 32B CPU run takes hours (time the default workload instead)"}))
            return
        global B8_GEN
        B8_GEN = args.gen if args.gen is not None else B8_GEN
        run_batch8(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
