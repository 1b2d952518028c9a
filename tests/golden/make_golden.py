"""Regenerates the golden fixtures in this directory from the REFERENCE itself.

Run here, where the reference sources exist and oracle/_ref/libbrainref.so has
been built from them (oracle/Makefile):  python tests/golden/make_golden.py

Fixtures (all produced by the reference's own code, src/brain_runtime.c):
  dequant.npz   per block type: input block bytes (random bytes and blocks with
                the synthetic distributions) and dequant_block's output bits
  tiny.npz      a 2-layer synthetic model (regenerated from its seed by the
                repository's GGUF writer; its SHA-256 is stored): logits of a
                12-token prompt at every position and the 32 greedy picks after it
  cfg0.npz      the Qwen2-1.5B-shaped synthetic model (hidden 1536, 28 layers,
                12/2 heads, FFN 8960, vocab 151936, tied Q6_K head, seed 0):
                a 32-token uniform-random prompt, the 32 greedy picks, and the
                logits (fp16) after the prompt and after the first pick
  cfg1.npz      the same for the Qwen2.5-3B shape (hidden 2048, 36 layers,
                16/2 heads, FFN 11008, vocab 151936, tied head, seed 1) with
                the 512-token prompt the benchmark decodes after
  cfg2.npz      the same for the Qwen2.5-7B shape (hidden 3584, 28 layers,
                28/4 heads, FFN 18944, vocab 152064, untied Q6_K head, seed 2),
                512-token prompt

The reference runs the prompt token by token (src/brain_runtime.c:2025-2028),
so cfg1/cfg2 take tens of minutes on a few cores. Usage:
  python tests/golden/make_golden.py            # dequant, tiny, cfg0
  python tests/golden/make_golden.py cfg1 cfg2  # the large shapes
"""
import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "-1.7-atlas---apollo_b200", "python"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import atlas_cuda  # noqa: E402
import oracle_bind  # noqa: E402

TINY = dict(hidden=512, layers=2, q_heads=4, kv_heads=2, ffn=768, vocab=1024, context_length=512, seed=1234)
CFG0 = dict(hidden=1536, layers=28, q_heads=12, kv_heads=2, ffn=8960, vocab=151936, context_length=32768, seed=0)
# large shapes: (model, tied, prompt seed, prompt length)
LARGE = {
    "cfg1": (dict(hidden=2048, layers=36, q_heads=16, kv_heads=2, ffn=11008, vocab=151936, context_length=32768,
                  seed=1), True, 1234, 512),
    "cfg2": (dict(hidden=3584, layers=28, q_heads=28, kv_heads=4, ffn=18944, vocab=152064, context_length=32768,
                  seed=2), False, 1234, 512),
}


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def greedy_run(ref, prompt, steps):
    """Prompt token by token, then `steps` greedy picks (src/brain_runtime.c:2025-2048)."""
    logits = []
    for i, t in enumerate(prompt):
        lg = ref.forward(int(t), i, i + 1 == len(prompt))
        if lg is not None:
            logits.append(lg)
    picks = []
    lg = logits[-1]
    for s in range(steps):
        nxt = ref.greedy(lg)
        picks.append(nxt)
        if s + 1 < steps:
            lg = ref.forward(nxt, len(prompt) + s, True)
            if s == 0:
                logits.append(lg)
    return np.array(picks, np.uint32), logits


def make_large(ref, name, workdir):
    cfg, tied, pseed, plen = LARGE[name]
    p = os.path.join(workdir, f"{name}.gguf")
    atlas_cuda.write_synthetic_gguf(p, tied=tied, **cfg)
    r = ref.open(p)
    prompt = np.random.default_rng(pseed).integers(0, cfg["vocab"], plen).astype(np.uint32)
    picks, logits = greedy_run(r, prompt, 32)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), sha256=sha256(p), prompt=prompt, picks=picks,
                        tied=np.int32(tied), logits_prompt=logits[0].astype(np.float16),
                        logits_step1=logits[1].astype(np.float16),
                        max_abs_prompt=np.float32(np.abs(logits[0]).max()),
                        max_abs_step1=np.float32(np.abs(logits[1]).max()),
                        **{f"cfg_{k}": v for k, v in cfg.items()})
    r.close()
    os.remove(p)


def main():
    ref = oracle_bind.Reference.load()
    assert ref is not None, "build oracle/_ref first (make -C oracle ref)"
    large = [a for a in sys.argv[1:] if a in LARGE]
    if large:
        with tempfile.TemporaryDirectory(dir=os.environ.get("ATLAS_GOLDEN_TMP")) as td:
            for name in large:
                make_large(ref, name, td)
                print("golden fixture written:", name, flush=True)
        return
    ref = oracle_bind.Reference.load()
    assert ref is not None, "build oracle/_ref first (make -C oracle ref)"
    rng = np.random.default_rng(20261201)
    out = {}
    for t in (atlas_cuda.TYPE_Q4_K, atlas_cuda.TYPE_Q6_K, atlas_cuda.TYPE_Q5_K, atlas_cuda.TYPE_Q5_0,
              atlas_cuda.TYPE_Q5_1, atlas_cuda.TYPE_Q8_0, atlas_cuda.TYPE_F16):
        bb, be = atlas_cuda.BLOCK_BYTES[t], atlas_cuda.BLOCK_ELEMS[t]
        raw = rng.integers(0, 256, 48 * bb, dtype=np.uint8)
        if t in (atlas_cuda.TYPE_Q4_K, atlas_cuda.TYPE_Q6_K):
            raw = np.concatenate([raw, atlas_cuda.synth_blocks(t, 48, seed=7, stream=t)])
        n = raw.size // bb
        out[f"in_{t}"] = raw
        out[f"out_{t}"] = ref.dequant(t, raw, n, be).view(np.uint32)
    np.savez_compressed(os.path.join(HERE, "dequant.npz"), **out)

    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "tiny.gguf")
        atlas_cuda.write_synthetic_gguf(p, tied=True, **TINY)
        r = ref.open(p)
        prompt = np.array([5, 77, 300, 1000, 3, 9, 400, 256, 512, 18, 700, 1020], np.uint32)
        all_logits = np.stack([r.forward(int(t), i) for i, t in enumerate(prompt)])
        lg = all_logits[-1]
        picks = []
        for s in range(32):
            nxt = r.greedy(lg)
            picks.append(nxt)
            lg = r.forward(nxt, len(prompt) + s)
        np.savez_compressed(os.path.join(HERE, "tiny.npz"), sha256=sha256(p), prompt=prompt, logits=all_logits,
                            picks=np.array(picks, np.uint32), **{f"cfg_{k}": v for k, v in TINY.items()})
        r.close()

        p = os.path.join(td, "cfg0.gguf")
        atlas_cuda.write_synthetic_gguf(p, tied=True, **CFG0)
        r = ref.open(p)
        prompt = np.random.default_rng(0).integers(0, CFG0["vocab"], 32).astype(np.uint32)
        picks, logits = greedy_run(r, prompt, 32)
        np.savez_compressed(os.path.join(HERE, "cfg0.npz"), sha256=sha256(p), prompt=prompt, picks=picks,
                            logits_prompt=logits[0].astype(np.float16), logits_step1=logits[1].astype(np.float16),
                            max_abs_prompt=np.float32(np.abs(logits[0]).max()),
                            max_abs_step1=np.float32(np.abs(logits[1]).max()),
                            **{f"cfg_{k}": v for k, v in CFG0.items()})
        r.close()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
