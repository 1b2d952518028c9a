"""Kernel-level timing of libatlas_cuda's C ABI entry points on seeded synthetic data.

    python -m atlas_kernels gemv --type 14 --rows 151936 --cols 2048 [--reps 20]
    python -m atlas_kernels trace --hidden 2048 --layers 36 --q-heads 16 --kv-heads 2 --ffn 11008 --pos 600
    python -m atlas_kernels gemm --type 12 --rows 22016 --cols 2048 --tokens 512
    python -m atlas_kernels prefill --tokens 512

`gemv` times atlas_cuda_gemv with CUDA events (with --reps 1 it runs one warm-up
and one launch, the shape an ncu capture wants); `trace` runs one decode step
with device-side timestamps (atlas_cuda_trace_step) and prints the time per
phase kind; `gemm` times atlas_cuda_gemm (per-call scratch allocation
included); `prefill` times a whole batched prefill of a synthetic model
(device time of the call, best of --reps). Device buffers come from torch;
every kernel is this library's.
"""
import argparse
import os
import sys
import tempfile

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import atlas_cuda  # noqa: E402

KIND = {0: "embed", 16: "gemv_store", 17: "gemv_resid_add", 18: "gemv_swiglu", 19: "gemv_logits", 32: "attention",
        48: "argmax"}


def cmd_gemv(a):
    import torch
    nb = a.rows * a.cols // 256
    w = atlas_cuda.synth_blocks(a.type, nb, seed=1)
    d_w = torch.from_numpy(w).cuda()
    d_x = torch.randn(a.cols, device="cuda")
    d_y = torch.empty(a.rows, device="cuda")
    atlas_cuda.gemv(a.type, d_w, a.rows, a.cols, d_x, d_y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        atlas_cuda.gemv(a.type, d_w, a.rows, a.cols, d_x, d_y)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.reps
    print(f"gemv type {a.type} {a.rows}x{a.cols}: {w.nbytes / 1e6:.1f} MB, {ms * 1e3:.1f} us, "
          f"{w.nbytes / ms / 1e6:.0f} GB/s")


def cmd_trace(a):
    tag = "u" if a.untied else "t"
    path = os.path.join(tempfile.gettempdir(),
                        f"atlas_trace_{a.hidden}_{a.layers}_{a.q_heads}_{a.kv_heads}_{a.ffn}_{a.vocab}{tag}.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, hidden=a.hidden, layers=a.layers, q_heads=a.q_heads,
                                        kv_heads=a.kv_heads, ffn=a.ffn, vocab=a.vocab, seed=1,
                                        tied=not a.untied)
    with atlas_cuda.Runtime(path, max_context=a.pos + 16) as rt:
        rt.prefill(np.arange(1, a.pos + 1, dtype=np.uint32) % a.vocab, 0, want_logits=False)
        tr, ext, kinds = rt.trace_step(7, a.pos)
    tr, ext = tr.astype(np.int64), ext.astype(np.int64)
    t0 = tr[tr > 0].min()
    tr = np.where(tr > 0, tr - t0, -1)
    ext = np.where(ext > 0, ext - t0, -1)
    end = tr[:, :, 2].max()
    print(f"decode step at position {a.pos}: {end / 1e3:.1f} us over {len(kinds)} phases")
    agg, prev = {}, 0
    for p, k in enumerate(kinds):
        done = tr[:, p, 2].max()
        busy = tr[:, p, 1] >= 0
        start = tr[:, p, 1][busy].min() if busy.any() else prev
        # inner stamps of the slowest CTA, relative to its wait end
        slow = int(np.argmax(tr[:, p, 2]))
        inner = [(ext[slow, p, i] - tr[slow, p, 1]) for i in range(8) if ext[slow, p, i] >= 0]
        s = agg.setdefault(KIND.get(int(k), str(k)), [0, 0, 0, [0.0] * 8, 0])
        s[0] += done - prev
        s[1] += start - prev
        s[2] += 1
        for i, v in enumerate(inner):
            s[3][i] += v
        s[4] = max(s[4], len(inner))
        prev = done
    for name, (tot, gap, n, inner, ni) in agg.items():
        stamps = " ".join(f"{v / n / 1e3:.2f}" for v in inner[:ni])
        print(f"  {name:16s} x{n:3d}  {tot / 1e3:9.1f} us total  {tot / n / 1e3:7.2f} us each  "
              f"(barrier gap {gap / n / 1e3:5.2f} us; slowest CTA stamps {stamps} us)")


def cmd_gemm(a):
    import torch
    nb = a.rows * a.cols // 256
    w = atlas_cuda.synth_blocks(a.type, nb, seed=1)
    d_w = torch.from_numpy(w).cuda()
    d_x = torch.randn(a.tokens, a.cols, device="cuda")
    d_y = torch.empty(a.tokens, a.rows, device="cuda")
    atlas_cuda.gemm(a.type, d_w, a.rows, a.cols, d_x, a.tokens, d_y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        atlas_cuda.gemm(a.type, d_w, a.rows, a.cols, d_x, a.tokens, d_y)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.reps
    flops = 2.0 * a.rows * a.cols * a.tokens
    print(f"gemm type {a.type} {a.rows}x{a.cols} x {a.tokens} tokens: {ms * 1e3:.1f} us per call "
          f"(scratch allocation and split included), {flops / ms / 1e9:.1f} TFLOP/s algorithmic")


def cmd_prefill(a):
    tag = "u" if a.untied else "t"
    path = os.path.join(tempfile.gettempdir(),
                        f"atlas_trace_{a.hidden}_{a.layers}_{a.q_heads}_{a.kv_heads}_{a.ffn}_{a.vocab}{tag}.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, hidden=a.hidden, layers=a.layers, q_heads=a.q_heads,
                                        kv_heads=a.kv_heads, ffn=a.ffn, vocab=a.vocab, seed=1,
                                        tied=not a.untied)
    ids = (np.arange(1, a.tokens + 1, dtype=np.uint32) * 7919) % a.vocab
    with atlas_cuda.Runtime(path, max_context=a.tokens + 16, max_prefill=a.tokens) as rt:
        rt.prefill(ids, 0, want_logits=False)
        best = None
        for _ in range(a.reps):
            rt.prefill(ids, 0, want_logits=False)
            _, ms, _ = rt.stats()
            best = ms if best is None else min(best, ms)
    h, f, q, kv, L = a.hidden, a.ffn, a.q_heads * 128, a.kv_heads * 128, a.layers
    flops = 2.0 * a.tokens * L * (2 * q * h + 2 * kv * h + 3 * f * h)
    print(f"prefill {a.tokens} tokens: {best:.2f} ms device time, {a.tokens / best * 1e3:.0f} tok/s, "
          f"{flops / best / 1e9:.1f} TFLOP/s of linear-layer work")


def cmd_decode(a):
    """Prefill a random prompt, then `steps` greedy decode steps through the
    graph decode step; prints the device time per token of a 64-step run
    unless --steps-only (then only the `steps` steps run: a capture target)."""
    tag = "u" if a.untied else "t"
    path = os.path.join(tempfile.gettempdir(),
                        f"atlas_trace_{a.hidden}_{a.layers}_{a.q_heads}_{a.kv_heads}_{a.ffn}_{a.vocab}{tag}.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, hidden=a.hidden, layers=a.layers, q_heads=a.q_heads,
                                        kv_heads=a.kv_heads, ffn=a.ffn, vocab=a.vocab, seed=1,
                                        tied=not a.untied)
    ids = np.random.default_rng(1).integers(0, a.vocab, a.prompt).astype(np.uint32)
    with atlas_cuda.Runtime(path, max_context=a.prompt + a.steps + 80, max_prefill=min(a.prompt, a.chunk),
                            kv_fp16=a.kv_fp16) as rt:
        _, first = rt.prefill(ids, 0, want_logits=False)
        pre_ms = rt.stats()[1]
        rt.generate(first, a.prompt, a.steps)
        if a.steps_only:
            return
        d0 = rt.stats()[2]
        rt.generate(first, a.prompt, 64)
        ms = (rt.stats()[2] - d0) / 64
    print(f"prefill {a.prompt} tokens: {pre_ms:.2f} ms ({a.prompt / pre_ms * 1e3:.0f} tok/s)")
    print(f"decode at position {a.prompt}: {ms:.4f} ms per token, {1e3 / ms:.1f} tok/s")


def cmd_tp(a):
    """Tensor-parallel decode, one rank per process (launch under
    torch.distributed.run): prefill a random prompt through the TP prompt mode,
    then time `steps` greedy decode steps; rank 0 prints each rank's device
    time per token and the per-GPU HBM rate of the rank's share."""
    import datetime
    import torch.distributed as dist
    if "RANK" not in os.environ:   # one rank without a launcher
        import socket
        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            port = sk.getsockname()[1]
        os.environ.update(RANK="0", WORLD_SIZE="1", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    path = os.path.join(tempfile.gettempdir(),
                        f"atlas_trace_{a.hidden}_{a.layers}_{a.q_heads}_{a.kv_heads}_{a.ffn}_{a.vocab}u.gguf")
    if rank == 0 and not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, hidden=a.hidden, layers=a.layers, q_heads=a.q_heads,
                                        kv_heads=a.kv_heads, ffn=a.ffn, vocab=a.vocab, seed=1, tied=False)
    dist.barrier()
    ids = np.random.default_rng(1).integers(0, a.vocab, a.prompt).astype(np.uint32)
    rt = atlas_cuda.Runtime(path, device=int(os.environ.get("LOCAL_RANK", rank)),
                            max_context=a.prompt + 2 * a.steps + 8, tp_rank=rank, tp_size=world)
    if world > 1:
        atlas_cuda.connect_tp(rt)
    dist.barrier()
    _, first = rt.prefill(ids, 0, want_logits=False)
    prompt_ms = rt.stats()[1]
    picks = rt.generate(first, a.prompt, a.steps)           # warm-up
    rt.generate(int(picks[-1]), a.prompt + a.steps, a.steps)
    ms = rt.stats()[1] / a.steps
    sl = rt.tp_slice()
    h, f, q, kv, L = a.hidden, a.ffn, a.q_heads * 128, a.kv_heads * 128, a.layers
    q4, q6 = 144 / 256, 210 / 256
    # this rank's weight bytes per token (o and down: its blocks) + its KV read at the mean position
    lq, lkv = sl.q_heads * 128, sl.kv_heads * 128
    layer = (lq + lkv) * h * q4 + lkv * h * q6 + h * sl.o_blocks * 256 * q4 + 2 * sl.ffn_rows * h * q4 + \
        h * sl.ffn_rows * q6
    pos = a.prompt + 1.5 * a.steps
    rank_bytes = L * layer + sl.vocab_rows * h * q6 + L * 2 * lkv * 4 * pos
    got = [None] * world
    dist.all_gather_object(got, (ms, rank_bytes, prompt_ms))
    dist.barrier()
    rt.close()
    if rank == 0:
        worst = max(g[0] for g in got)
        print(f"tp {world}: {h}x{L} layers, q/kv heads {a.q_heads}/{kv // 128}, ffn {f}, vocab {a.vocab}")
        for r, (m, b, pm) in enumerate(got):
            print(f"  rank {r}: {m:.4f} ms per token, {b / 1e9:.3f} GB per token -> {b / m / 1e6:.0f} GB/s "
                  f"(prompt {a.prompt} tokens {pm:.1f} ms)")
        print(f"decode {1e3 / worst:.1f} tok/s (slowest rank {worst:.4f} ms per token)")
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    m = sub.add_parser("gemm")
    m.add_argument("--type", type=int, default=12)
    m.add_argument("--rows", type=int, default=22016)
    m.add_argument("--cols", type=int, default=2048)
    m.add_argument("--tokens", type=int, default=512)
    m.add_argument("--reps", type=int, default=10)
    p = sub.add_parser("prefill")
    p.add_argument("--hidden", type=int, default=2048)
    p.add_argument("--layers", type=int, default=36)
    p.add_argument("--q-heads", type=int, default=16)
    p.add_argument("--kv-heads", type=int, default=2)
    p.add_argument("--ffn", type=int, default=11008)
    p.add_argument("--vocab", type=int, default=151936)
    p.add_argument("--tokens", type=int, default=512)
    p.add_argument("--reps", type=int, default=5)
    p.add_argument("--untied", action="store_true", help="separate Q6_K output head")
    g = sub.add_parser("gemv")
    g.add_argument("--type", type=int, default=14)
    g.add_argument("--rows", type=int, default=151936)
    g.add_argument("--cols", type=int, default=2048)
    g.add_argument("--reps", type=int, default=20)
    t = sub.add_parser("trace")
    t.add_argument("--hidden", type=int, default=2048)
    t.add_argument("--layers", type=int, default=36)
    t.add_argument("--q-heads", type=int, default=16)
    t.add_argument("--kv-heads", type=int, default=2)
    t.add_argument("--ffn", type=int, default=11008)
    t.add_argument("--vocab", type=int, default=151936)
    t.add_argument("--pos", type=int, default=600)
    t.add_argument("--untied", action="store_true", help="separate Q6_K output head")
    dcd = sub.add_parser("decode")
    dcd.add_argument("--hidden", type=int, default=2048)
    dcd.add_argument("--layers", type=int, default=36)
    dcd.add_argument("--q-heads", type=int, default=16)
    dcd.add_argument("--kv-heads", type=int, default=2)
    dcd.add_argument("--ffn", type=int, default=11008)
    dcd.add_argument("--vocab", type=int, default=151936)
    dcd.add_argument("--prompt", type=int, default=512)
    dcd.add_argument("--steps", type=int, default=3)
    dcd.add_argument("--steps-only", action="store_true")
    dcd.add_argument("--untied", action="store_true", help="separate Q6_K output head")
    dcd.add_argument("--kv-fp16", action="store_true", help="fp16 KV cache")
    dcd.add_argument("--chunk", type=int, default=512, help="prefill chunk (max_prefill)")
    tpp = sub.add_parser("tp")
    tpp.add_argument("--hidden", type=int, default=3584)
    tpp.add_argument("--layers", type=int, default=28)
    tpp.add_argument("--q-heads", type=int, default=28)
    tpp.add_argument("--kv-heads", type=int, default=4)
    tpp.add_argument("--ffn", type=int, default=18944)
    tpp.add_argument("--vocab", type=int, default=152064)
    tpp.add_argument("--prompt", type=int, default=512)
    tpp.add_argument("--steps", type=int, default=64)
    a = ap.parse_args()
    {"gemv": cmd_gemv, "trace": cmd_trace, "gemm": cmd_gemm, "prefill": cmd_prefill, "decode": cmd_decode,
     "tp": cmd_tp}[a.cmd](a)


if __name__ == "__main__":
    main()
