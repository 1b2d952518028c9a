"""GPU: end-to-end parity of the decode engine against the reference.

Bar (the contract for this path): final logits within
max|dlogit| <= 2e-2 * max|logit| of the reference CPU path, and identical greedy
tokens for the first 32 steps. fp32 activations and fp32 KV cache (the default; the fp16 cache is an option
whose parity these random-weight models do not support, see atlas_cuda.h)."""
import os

import numpy as np
import pytest

import atlas_cuda

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 2e-2


def _close(got, want, tol=TOL):
    err = np.abs(got.astype(np.float64) - want).max()
    bound = tol * np.abs(want).max()
    assert err <= bound, f"max|dlogit| {err} > {bound}"
    return err / np.abs(want).max()


def test_tiny_matches_golden(torch_cuda, tiny_model):
    g = np.load(os.path.join(GOLDEN, "tiny.npz"))
    with atlas_cuda.Runtime(tiny_model, max_context=256) as rt:
        prompt = g["prompt"]
        for i, t in enumerate(prompt):
            lg, am = rt.forward(int(t), i)
            rel = _close(lg, g["logits"][i])
            assert rel < 1e-3
        picks = rt.generate(int(g["picks"][0]), len(prompt), 32)
        # generate() returns the pick after each forward: picks[1:] of the reference
        np.testing.assert_array_equal(picks[:31], g["picks"][1:32])
        assert am == int(g["picks"][0])


def test_tiny_untied_matches_oracle(torch_cuda, oracle, tiny_untied_model):
    m = oracle.open(tiny_untied_model)
    m.begin(128)
    with atlas_cuda.Runtime(tiny_untied_model, max_context=128) as rt:
        for pos, tok in enumerate([1, 900, 44, 1000, 2, 17, 17, 17]):
            want = m.forward(tok, pos)
            got, am = rt.forward(tok, pos)
            _close(got, want, 1e-3)
            assert am == m.argmax(want)


@pytest.mark.parametrize("ranges", ["auto", "tiles", "shares"])
def test_small_prefill_generate_matches_oracle(torch_cuda, oracle, small_model, monkeypatch, ranges):
    """Prompt logits and 32 greedy steps against the oracle, with the decode
    GEMVs' CTA ranges as the planner picks them, in whole row tiles
    (ATLAS_MV_TILE_RANGES=1), and as equal task shares with the row tiles cut
    between CTAs finished by the last CTA to arrive (=0)."""
    if ranges != "auto":
        monkeypatch.setenv("ATLAS_MV_TILE_RANGES", "1" if ranges == "tiles" else "0")
    m = oracle.open(small_model)
    m.begin(128)
    prompt = np.random.default_rng(1).integers(0, 4096, 40).astype(np.uint32)
    for i, t in enumerate(prompt):
        want = m.forward(int(t), i, i + 1 == len(prompt))
    want_picks = []
    lg = want
    for s in range(32):
        nxt = m.argmax(lg)
        want_picks.append(nxt)
        lg = m.forward(nxt, len(prompt) + s)
    with atlas_cuda.Runtime(small_model, max_context=128) as rt:
        got, am = rt.prefill(prompt)
        _close(got, want, 1e-3)
        assert am == want_picks[0]
        picks = rt.generate(am, len(prompt), 31)
        np.testing.assert_array_equal(picks, np.array(want_picks[1:], np.uint32))


@pytest.mark.parametrize("case", __import__("conftest").OTHER_TYPES, ids=lambda c: c[0])
def test_other_block_types_match_oracle(torch_cuda, oracle, model_dir, case):
    """Files with the reference's other block types in the projections and the
    head, and with types that change across layers: the prompt (replayed
    through the decode step for the other types, batched for Q4_K / Q6_K) and
    24 greedy steps against the oracle."""
    from conftest import other_type_model
    path = other_type_model(model_dir, case)
    m = oracle.open(path)
    m.begin(128)
    prompt = np.random.default_rng(5).integers(0, 2048, 20).astype(np.uint32)
    for i, t in enumerate(prompt):
        want = m.forward(int(t), i, i + 1 == len(prompt))
    want_picks, lg = [], want
    for s in range(24):
        want_picks.append(m.argmax(lg))
        lg = m.forward(want_picks[-1], len(prompt) + s)
    with atlas_cuda.Runtime(path, max_context=128) as rt:
        got, am = rt.prefill(prompt)
        _close(got, want, 1e-3)
        assert am == want_picks[0]
        picks = rt.generate(am, len(prompt), 23)
        np.testing.assert_array_equal(picks, np.array(want_picks[1:], np.uint32))
        got2, _ = rt.forward(int(want_picks[0]), len(prompt))
        w2 = m.forward(int(want_picks[0]), len(prompt))   # the oracle's cache is rewritten at this position too
        _close(got2, w2, 1e-3)


LONG = dict(hidden=256, layers=2, q_heads=2, kv_heads=1, ffn=512, vocab=1024, context_length=8448, seed=8191)
LONG_PROMPT = 8176   # positions up to 8,191 after the 16 greedy steps (the 14B shape's 8,192-token prompt length)
_long_want = {}


def _long_oracle(oracle, path):
    """The oracle over the long prompt and 16 greedy steps (computed once)."""
    if path not in _long_want:
        m = oracle.open(path)
        m.begin(LONG_PROMPT + 32)
        prompt = np.random.default_rng(81).integers(0, LONG["vocab"], LONG_PROMPT).astype(np.uint32)
        for i, t in enumerate(prompt):
            lg = m.forward(int(t), i, i + 1 == len(prompt))
        first = lg
        picks = []
        for s in range(16):
            picks.append(m.argmax(lg))
            lg = m.forward(picks[-1], LONG_PROMPT + s)
        _long_want[path] = (prompt, first, picks, lg)
    return _long_want[path]


@pytest.mark.slow
@pytest.mark.parametrize("kv_fp16", [False, True])
def test_long_context_matches_oracle(torch_cuda, oracle, model_dir, kv_fp16):
    """An 8,176-token batched prefill and 16 greedy steps (positions up to
    8,191) against the oracle. fp32 cache: logits within 1e-3 max|logit| and
    every pick; fp16 cache (the 14B shape's cache): within the 2e-2 bound."""
    path = os.path.join(str(model_dir), "long.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, tied=True, **LONG)
    prompt, first, picks, last = _long_oracle(oracle, path)
    with atlas_cuda.Runtime(path, max_context=LONG_PROMPT + 32, max_prefill=512, kv_fp16=kv_fp16) as rt:
        got, am = rt.prefill(prompt)
        rel = _close(got, first, 2e-2 if kv_fp16 else 1e-3)
        if not kv_fp16:
            assert am == picks[0]
            got_picks = rt.generate(am, LONG_PROMPT, 15)
            np.testing.assert_array_equal(got_picks, np.array(picks[1:], np.uint32))
            lg, _ = rt.forward(int(picks[-1]), LONG_PROMPT + 15)
            _close(lg, last, 1e-3)
        print(f"long context, fp16 cache {kv_fp16}: max|dlogit|/max|logit| {rel:.3g}")


def test_generate_equals_forward_loop(torch_cuda, small_model):
    with atlas_cuda.Runtime(small_model, max_context=64) as rt:
        _, am = rt.prefill(np.arange(10, 30, dtype=np.uint32))
        a = rt.generate(am, 20, 12)
        _, am2 = rt.prefill(np.arange(10, 30, dtype=np.uint32))
        b = [am2]
        for s in range(12):
            _, nxt = rt.forward(b[-1], 20 + s)
            b.append(nxt)
        np.testing.assert_array_equal(a, np.array(b[1:], np.uint32))


def test_range_errors(torch_cuda, tiny_model):
    with atlas_cuda.Runtime(tiny_model, max_context=32) as rt:
        with pytest.raises(atlas_cuda.AtlasError):
            rt.forward(5, 32)                       # position beyond the KV cache
        with pytest.raises(atlas_cuda.AtlasError):
            rt.forward(1024, 0)                     # token >= vocab
        with pytest.raises(atlas_cuda.AtlasError):
            rt.prefill(np.zeros(0, np.uint32))      # empty prefill
        rt.forward(5, 0)                            # the handle still works


@pytest.mark.slow
def test_cfg0_full_size_matches_reference(torch_cuda, model_dir):
    """Qwen2-1.5B shape, 32-token prompt + 32 greedy steps vs the reference's own run."""
    g = np.load(os.path.join(GOLDEN, "cfg0.npz"))
    cfg = {k[4:]: int(g[k]) for k in g.files if k.startswith("cfg_")}
    p = os.path.join(str(model_dir), "cfg0.gguf")
    if not os.path.exists(p):
        atlas_cuda.write_synthetic_gguf(p, tied=True, **cfg)
    with atlas_cuda.Runtime(p, max_context=512) as rt:
        prompt = g["prompt"]
        lg, am = rt.prefill(prompt)
        _close(lg, g["logits_prompt"].astype(np.float32))
        assert am == int(g["picks"][0])
        lg1, am1 = rt.forward(am, len(prompt))
        _close(lg1, g["logits_step1"].astype(np.float32))
        picks = rt.generate(am1, len(prompt) + 1, 30)
        got = np.concatenate([[am, am1], picks]).astype(np.uint32)
        np.testing.assert_array_equal(got, g["picks"])


WIDE = {
    # Qwen2.5-7B and -14B layer widths (2 of their 28 / 48 layers), untied Q6_K head
    "7b_width": dict(hidden=3584, layers=2, q_heads=28, kv_heads=4, ffn=18944, vocab=152064,
                     context_length=1024, seed=77),
    "14b_width": dict(hidden=5120, layers=2, q_heads=40, kv_heads=8, ffn=13824, vocab=152064,
                      context_length=1024, seed=78),
}


@pytest.mark.slow
@pytest.mark.parametrize("name", sorted(WIDE))
def test_wide_shapes_match_oracle(torch_cuda, oracle, model_dir, name):
    """Full-width layers of the 7B / 14B shapes (rows longer than 8 blocks on every
    projection, 7 and 5 query heads per KV head, vocab 152064): prompt logits and
    32 greedy steps against the oracle."""
    cfg = WIDE[name]
    p = os.path.join(str(model_dir), f"{name}.gguf")
    if not os.path.exists(p):
        atlas_cuda.write_synthetic_gguf(p, tied=False, **cfg)
    m = oracle.open(p)
    m.begin(128)
    prompt = np.random.default_rng(cfg["seed"]).integers(0, cfg["vocab"], 12).astype(np.uint32)
    for i, t in enumerate(prompt):
        want = m.forward(int(t), i, i + 1 == len(prompt))
    want_picks, lg = [], want
    for s in range(32):
        want_picks.append(m.argmax(lg))
        if s < 31:
            lg = m.forward(want_picks[-1], len(prompt) + s)
    with atlas_cuda.Runtime(p, max_context=128) as rt:
        got, am = rt.prefill(prompt)
        _close(got, want, 1e-3)
        assert am == want_picks[0]
        picks = rt.generate(am, len(prompt), 31)
        np.testing.assert_array_equal(picks, np.array(want_picks[1:], np.uint32))


@pytest.mark.parametrize("kparts,layers", [(2, 3), (3, 4)])
def test_down_k_parts_match_oracle(torch_cuda, oracle, model_dir, monkeypatch, kparts, layers):
    """The one-GPU down projection in K parts (ATLAS_DOWN_KPARTS; chosen by
    itself for long FFN rows such as the 7B's 18944): each part stores partial
    rows, the next layer's q/k/v staging (or the head's) adds them to the
    residual in part order, and the residual alternates between two buffers.
    Odd and even layer counts (the head reads either buffer); odd layers keep
    ffn_down in Q4_K (a Q4_K_M file's mix). Prompt logits and 16 greedy steps
    against the oracle, and against one part."""
    monkeypatch.setenv("ATLAS_DOWN_KPARTS", str(kparts))
    p = os.path.join(str(model_dir), f"kparts_{layers}.gguf")
    if not os.path.exists(p):
        atlas_cuda.write_synthetic_gguf(p, hidden=1024, layers=layers, q_heads=8, kv_heads=2, ffn=3072, vocab=4096,
                                        context_length=256, tied=False, layer_mix=True, seed=90 + layers)
    m = oracle.open(p)
    m.begin(64)
    prompt = np.random.default_rng(layers).integers(0, 4096, 20).astype(np.uint32)
    for i, t in enumerate(prompt):
        want = m.forward(int(t), i, i + 1 == len(prompt))
    want_picks, logits, lg = [], [], want
    for s in range(16):
        want_picks.append(m.argmax(lg))
        lg = m.forward(want_picks[-1], len(prompt) + s)
        logits.append(lg)
    with atlas_cuda.Runtime(p, max_context=64) as rt:
        got, am = rt.prefill(prompt)
        _close(got, want, 1e-3)
        assert am == want_picks[0]
        picks = rt.generate(am, len(prompt), 15)
        np.testing.assert_array_equal(picks, np.array(want_picks[1:], np.uint32))
        lg16, _ = rt.forward(int(want_picks[15]), len(prompt) + 15)
        _close(lg16, logits[15], 1e-3)
    monkeypatch.setenv("ATLAS_DOWN_KPARTS", "1")
    with atlas_cuda.Runtime(p, max_context=64) as rt:
        got1, _ = rt.prefill(prompt)
        _close(got1, got.astype(np.float64), 1e-4)


@pytest.mark.slow
@pytest.mark.parametrize("min_span", ["192", "8"])
def test_long_splits_match_oracle(torch_cuda, oracle, tiny_model, monkeypatch, min_span):
    """Decode attention over a 1400-token prompt, then 8 greedy steps, against
    the oracle: splits of >= 192 positions (one cluster of 8 splits, 6 K/V
    tiles each: the double-buffered tile loop) and of >= 8 positions (18
    clusters: the merge of cluster records in global memory)."""
    monkeypatch.setenv("ATLAS_ATTN_MIN_SPAN", min_span)
    prompt = np.random.default_rng(11).integers(0, 1024, 1400).astype(np.uint32)
    m = oracle.open(tiny_model)
    m.begin(1500)
    for i, t in enumerate(prompt):
        want = m.forward(int(t), i, i + 1 == len(prompt))
    want_picks, lg = [], want
    for s in range(8):
        want_picks.append(m.argmax(lg))
        if s < 7:
            lg = m.forward(want_picks[-1], len(prompt) + s)
    with atlas_cuda.Runtime(tiny_model, max_context=1500) as rt:
        got, am = rt.prefill(prompt)
        _close(got, want, 1e-3)
        assert am == want_picks[0]
        _, am1 = rt.forward(am, len(prompt))
        picks = rt.generate(am1, len(prompt) + 1, 6)
        np.testing.assert_array_equal(np.concatenate([[am, am1], picks]).astype(np.uint32),
                                      np.array(want_picks, np.uint32))


def test_qwen3_qk_norm_matches_oracle(torch_cuda, oracle, tiny_qwen3_model):
    """qwen3 (per-head q/k RMSNorm before RoPE, src/brain_runtime.c:1727-1737):
    token-by-token decode logits, a chunked batched prefill and 32 greedy
    steps against the oracle (itself pinned to the reference for qwen3)."""
    m = oracle.open(tiny_qwen3_model)
    m.begin(128)
    prompt = np.random.default_rng(21).integers(0, 1024, 40).astype(np.uint32)
    with atlas_cuda.Runtime(tiny_qwen3_model, max_context=128) as rt:
        for pos, tok in enumerate(prompt[:6]):
            got, am = rt.forward(int(tok), pos)
            want = m.forward(int(tok), pos)
            _close(got, want, 1e-3)
            assert am == m.argmax(want)
    m.begin(128)
    for i, t in enumerate(prompt):
        want = m.forward(int(t), i, i + 1 == len(prompt))
    want_picks, lg = [], want
    for s in range(32):
        want_picks.append(m.argmax(lg))
        if s < 31:
            lg = m.forward(want_picks[-1], len(prompt) + s)
    with atlas_cuda.Runtime(tiny_qwen3_model, max_context=128, max_prefill=16) as rt:
        got, am = rt.prefill(prompt)
        _close(got, want, 1e-3)
        assert am == want_picks[0]
        picks = rt.generate(am, len(prompt), 31)
        np.testing.assert_array_equal(picks, np.array(want_picks[1:], np.uint32))


@pytest.mark.slow
@pytest.mark.parametrize("min_span", ["96", "8"])
def test_fp16_cache_tensor_core_attention_matches_cuda_cores(torch_cuda, small_model, monkeypatch, min_span):
    """fp16 KV cache: the tensor-core decode attention (binary16 pairs of q and
    of the softmax weights against the cache's binary16 K and V) against the
    CUDA-core kernel over the same cache, 600 cached positions, with one
    cluster of splits and with 10 clusters (their records merged in global
    memory): logits of a decode step within 1e-4 of the largest, and 16 greedy
    picks identical."""
    monkeypatch.setenv("ATLAS_ATTN_MIN_SPAN", min_span)
    prompt = np.random.default_rng(17).integers(0, 4096, 600).astype(np.uint32)
    runs = []
    for tc in ("1", "0"):
        monkeypatch.setenv("ATLAS_ATTN_TC", tc)
        with atlas_cuda.Runtime(small_model, max_context=700, max_prefill=128, kv_fp16=True) as rt:
            _, am = rt.prefill(prompt)
            lg, am1 = rt.forward(am, len(prompt))
            picks = rt.generate(am1, len(prompt) + 1, 16)
        runs.append((lg, am, am1, picks))
    (lg_tc, am_tc, am1_tc, picks_tc), (lg_cc, am_cc, am1_cc, picks_cc) = runs
    _close(lg_tc, lg_cc.astype(np.float64), 1e-4)
    assert (am_tc, am1_tc) == (am_cc, am1_cc)
    np.testing.assert_array_equal(picks_tc, picks_cc)


def test_fp16_cache_tensor_core_attention_qwen3(torch_cuda, tiny_qwen3_model, monkeypatch):
    """The tensor-core decode attention of fp16 caches on a qwen3 model (q and
    the new k normalised per head before RoPE): decode logits within 1e-4 of
    the CUDA-core kernel's over the same cache, 8 greedy picks identical."""
    prompt = np.random.default_rng(23).integers(0, 1024, 90).astype(np.uint32)
    runs = []
    for tc in ("1", "0"):
        monkeypatch.setenv("ATLAS_ATTN_TC", tc)
        with atlas_cuda.Runtime(tiny_qwen3_model, max_context=128, max_prefill=32, kv_fp16=True) as rt:
            _, am = rt.prefill(prompt)
            lg, am1 = rt.forward(am, len(prompt))
            picks = rt.generate(am1, len(prompt) + 1, 8)
        runs.append((lg, am, am1, picks))
    (lg_tc, am_tc, am1_tc, picks_tc), (lg_cc, am_cc, am1_cc, picks_cc) = runs
    _close(lg_tc, lg_cc.astype(np.float64), 1e-4)
    assert (am_tc, am1_tc) == (am_cc, am1_cc)
    np.testing.assert_array_equal(picks_tc, picks_cc)


def _sha256(path):
    import hashlib
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def _large(model_dir, name):
    p = os.path.join(GOLDEN, f"{name}.npz")
    if not os.path.exists(p):
        pytest.skip(f"{name}.npz not generated (tests/golden/make_golden.py {name})")
    g = np.load(p)
    cfg = {k[4:]: int(g[k]) for k in g.files if k.startswith("cfg_")}
    path = os.path.join(str(model_dir), f"{name}.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, tied=bool(int(g["tied"])), **cfg)
        assert _sha256(path) == str(g["sha256"]), "the model file differs from the one the fixture was made from"
    return g, path


def _run_512(g, path, kv_fp16):
    """The benchmark's workload shape against the reference's own run: the
    512-token prompt through the batched prefill, the first pick through one
    forward, 30 more through the decode graph (src/brain_runtime.c:2025-2048)."""
    prompt = g["prompt"]
    with atlas_cuda.Runtime(path, max_context=len(prompt) + 64, max_prefill=len(prompt), kv_fp16=kv_fp16) as rt:
        lg, am = rt.prefill(prompt)
        lg1, am1 = rt.forward(am, len(prompt))
        picks = rt.generate(am1, len(prompt) + 1, 30)
    got = np.concatenate([[am, am1], picks]).astype(np.uint32)
    rel = [np.abs(lg.astype(np.float64) - g["logits_prompt"].astype(np.float64)).max() / float(g["max_abs_prompt"]),
           np.abs(lg1.astype(np.float64) - g["logits_step1"].astype(np.float64)).max() / float(g["max_abs_step1"])]
    return rel, got


@pytest.mark.slow
@pytest.mark.parametrize("name", ["cfg1", "cfg2"])
def test_full_depth_512_token_prompt_matches_reference(torch_cuda, model_dir, name):
    """Qwen2.5-3B (36 layers) and -7B (28 layers, untied head) shapes at full
    depth, fp32 KV cache: logits after the 512-token prompt and after the first
    pick within 2e-2 of the largest reference logit (the fixture stores them
    as fp16, whose rounding is ~5e-4 of the largest), and the 32 greedy picks
    identical to the reference's."""
    g, path = _large(model_dir, name)
    rel, got = _run_512(g, path, kv_fp16=False)
    print(f"{name} fp32 cache: max|dlogit|/max|logit| after prompt {rel[0]:.2e}, after pick 1 {rel[1]:.2e}")
    assert max(rel) <= TOL, rel
    np.testing.assert_array_equal(got, g["picks"])


@pytest.mark.slow
@pytest.mark.parametrize("name", ["cfg1", "cfg2"])
def test_full_depth_fp16_cache_against_reference(torch_cuda, model_dir, name):
    """The fp16 KV cache (binary16 K and V, read by the tensor-core decode
    attention and the prefill) against the reference's fp32 run of the same
    512-token prompt, held to the same contract: logits within 2e-2 of the
    largest and 32 identical greedy picks."""
    g, path = _large(model_dir, name)
    rel, got = _run_512(g, path, kv_fp16=True)
    agree = int((got == g["picks"]).sum())
    first_diff = int(np.argmax(got != g["picks"])) if agree < len(got) else -1
    print(f"{name} fp16 cache: max|dlogit|/max|logit| after prompt {rel[0]:.2e}, after pick 1 {rel[1]:.2e}; "
          f"greedy picks equal {agree}/32 (first difference at {first_diff})")
    assert max(rel) <= TOL, rel
    np.testing.assert_array_equal(got, g["picks"])
