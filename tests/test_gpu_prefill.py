"""GPU: the batched prefill path against the oracle.

The contraction kernel (tcgen05, binary16 hi/lo operand splits, fp32
accumulation in tensor memory) is compared with the oracle's bit-exact
dequantized weights times fp32 activations summed in float64. Each element must
be within 3e-5 of sum_k |x_k w_k|: the three-product split carries ~22
significant bits per product, so this is the bar of an fp32 dot product of the
same length, not of a binary16 one (a single hi.hi product fails it by an order
of magnitude).

Whole prompts go through embedding, the contractions with their fused epilogues
(bias + RoPE + KV-cache store, residual add, SwiGLU), the prompt attention and
the head, and must meet the path's bar against the oracle's token-at-a-time
forward: max|dlogit| <= 2e-2 * max|logit| (the tests ask for 1e-3) and the same
greedy tokens."""
import numpy as np
import pytest

import atlas_cuda

pytestmark = pytest.mark.gpu


def _close(got, want, tol):
    err = np.abs(got.astype(np.float64) - want).max()
    bound = tol * np.abs(want).max()
    assert err <= bound, f"max|dlogit| {err} > {bound}"


Q4, Q6 = atlas_cuda.TYPE_Q4_K, atlas_cuda.TYPE_Q6_K
GEMM_CASES = [(Q4, 256, 256, 1), (Q6, 300, 512, 7), (Q4, 2560, 2048, 130), (Q6, 2048, 11008, 64),
              (Q4, 1024, 1024, 300), (Q6, 256, 2048, 512), (Q4, 22016, 2048, 128)]


@pytest.mark.parametrize("t,rows,cols,tokens", GEMM_CASES)
def test_gemm_matches_oracle(torch_cuda, oracle, t, rows, cols, tokens):
    torch = torch_cuda
    rng = np.random.default_rng(rows + cols + tokens)
    nb = rows * cols // 256
    w = atlas_cuda.synth_blocks(t, nb, seed=rows * 3 + cols, stream=t)
    W = oracle.dequant(t, w, nb, 256).reshape(rows, cols).astype(np.float64)
    X = rng.standard_normal((tokens, cols)).astype(np.float32)
    X *= (2.0 ** rng.integers(-8, 9, (tokens, 1))).astype(np.float32)   # rows over many binades
    want = X.astype(np.float64) @ W.T
    bound = 3e-5 * (np.abs(X).astype(np.float64) @ np.abs(W).T)
    d_w = torch.from_numpy(w).cuda()
    d_x = torch.from_numpy(X).cuda()
    d_y = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
    atlas_cuda.gemm(t, d_w, rows, cols, d_x, tokens, d_y)
    torch.cuda.synchronize()
    got = d_y.cpu().numpy().astype(np.float64)
    err = np.abs(got - want)
    bad = ~(err <= bound)
    assert not bad.any(), (f"{bad.sum()} of {bad.size} outside the bound; worst rel "
                           f"{(err / np.maximum(bound, 1e-30)).max():.3g} at {np.unravel_index(np.argmax(err / np.maximum(bound, 1e-30)), err.shape)}")


def test_gemm_rejects_bad_arguments(torch_cuda):
    torch = torch_cuda
    d = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    x = torch.zeros(256, dtype=torch.float32, device="cuda")
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.gemm(Q4, d, 1, 300, x, 1, x)      # cols not a multiple of 256
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.gemm(Q4, d, 1, 256, x, 0, x)      # no tokens
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.gemm(8, d, 1, 256, x, 1, x)       # type without a tensor-core path


def _oracle_prompt(m, prompt, pos0=0):
    want = None
    for i, t in enumerate(prompt):
        want = m.forward(int(t), pos0 + i, i + 1 == len(prompt))
    return want


def _oracle_greedy(m, first, pos, steps):
    picks, tok = [], first
    for s in range(steps):
        lg = m.forward(tok, pos + s)
        tok = m.argmax(lg)
        picks.append(tok)
    return np.array(picks, np.uint32)


def test_prefill_token_tile_boundaries(torch_cuda, oracle, tiny_model):
    """1, 128, 129 and 255 tokens: one partial, one full, a full + 1-token and
    a full + partial token tile; each prompt restarts at position 0."""
    m = oracle.open(tiny_model)
    m.begin(300)
    rng = np.random.default_rng(5)
    with atlas_cuda.Runtime(tiny_model, max_context=300) as rt:
        for n in (1, 128, 129, 255):
            prompt = rng.integers(0, 1024, n).astype(np.uint32)
            want = _oracle_prompt(m, prompt)
            got, am = rt.prefill(prompt)
            _close(got, want, 1e-3)
            assert am == m.argmax(want)


def test_prefill_chunked_then_decode_then_continued(torch_cuda, oracle, small_model):
    """max_prefill 64: a 150-token prompt runs as chunks of 64, 64 and 22
    tokens; 10 greedy steps follow; a second prompt of 30 tokens then
    continues at position 160 over the cache both wrote."""
    m = oracle.open(small_model)
    m.begin(256)
    rng = np.random.default_rng(11)
    p1 = rng.integers(0, 4096, 150).astype(np.uint32)
    p2 = rng.integers(0, 4096, 30).astype(np.uint32)
    want1 = _oracle_prompt(m, p1)
    first = m.argmax(want1)
    want_picks = _oracle_greedy(m, first, 150, 10)
    want2 = _oracle_prompt(m, p2, 160)
    with atlas_cuda.Runtime(small_model, max_context=256, max_prefill=64) as rt:
        got1, am = rt.prefill(p1)
        _close(got1, want1, 1e-3)
        assert am == first
        picks = rt.generate(am, 150, 10)
        np.testing.assert_array_equal(picks, want_picks)
        got2, am2 = rt.prefill(p2, pos0=160)
        _close(got2, want2, 1e-3)
        assert am2 == m.argmax(want2)


def test_prefill_rejects_out_of_vocab(torch_cuda, tiny_model):
    with atlas_cuda.Runtime(tiny_model, max_context=64) as rt:
        with pytest.raises(atlas_cuda.AtlasError):
            rt.prefill(np.array([1, 2, 1024], np.uint32))
        rt.prefill(np.array([1, 2, 3], np.uint32))   # the handle still works


def test_gemm_rows_near_fp32_underflow(torch_cuda, oracle):
    """Rows whose largest value is tiny (a SwiGLU output with every gate far
    below zero reaches ~1e-35, subnormals included) or zero: the per-row scale
    must stay finite and the rows contribute ~0, as they do in fp32."""
    torch = torch_cuda
    t, rows, cols = Q6, 512, 11008
    nb = rows * cols // 256
    w = atlas_cuda.synth_blocks(t, nb, seed=5, stream=t)
    W = oracle.dequant(t, w, nb, 256).reshape(rows, cols).astype(np.float64)
    rng = np.random.default_rng(3)
    X = rng.standard_normal((6, cols)).astype(np.float32)
    X[0] *= np.float32(8.3e-35 / np.abs(X[0]).max())          # max just below 2^-113
    X[1] *= np.float32(1e-39)                                   # subnormal
    X[2] = 0.0
    X[3] *= np.float32(1e-30)
    want = X.astype(np.float64) @ W.T
    bound = 3e-5 * (np.abs(X).astype(np.float64) @ np.abs(W).T) + 1e-30
    d_w = torch.from_numpy(w).cuda()
    d_x = torch.from_numpy(X).cuda()
    d_y = torch.full((6, rows), float("nan"), dtype=torch.float32, device="cuda")
    atlas_cuda.gemm(t, d_w, rows, cols, d_x, 6, d_y)
    torch.cuda.synchronize()
    got = d_y.cpu().numpy().astype(np.float64)
    assert np.isfinite(got).all()
    assert (np.abs(got - want) <= bound).all()


def test_gemv_input_near_fp32_underflow(torch_cuda, oracle):
    torch = torch_cuda
    t, rows, cols = Q6, 256, 11008
    w = atlas_cuda.synth_blocks(t, rows * cols // 256, seed=6, stream=t)
    d_w = torch.from_numpy(w).cuda()
    for scale in (8.3e-35, 1e-39, 0.0):
        x = (np.random.default_rng(4).standard_normal(cols) * scale).astype(np.float32)
        want = oracle.matvec_raw(t, w, rows, cols, x)
        d_x = torch.from_numpy(x).cuda()
        d_y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        atlas_cuda.gemv(t, d_w, rows, cols, d_x, d_y)
        torch.cuda.synchronize()
        got = d_y.cpu().numpy()
        assert np.isfinite(got).all()
        assert np.abs(got.astype(np.float64) - want).max() <= 1e-4 * np.abs(want).max() + 1e-30


def test_prefill_fp16_kv_cache_matches_decode_loop(torch_cuda, small_model):
    """fp16 KV cache: the batched prefill (K/V stored as binary16 by the
    contraction epilogue, read back as binary16 by the prompt attention, in
    chunks that straddle the cache) matches a token-by-token decode loop over
    the same fp16 cache, and generation continues from either identically."""
    prompt = np.random.default_rng(3).integers(0, 4096, 150).astype(np.uint32)
    with atlas_cuda.Runtime(small_model, max_context=256, max_prefill=64, kv_fp16=True) as rt:
        lg, am = rt.prefill(prompt)
        a = rt.generate(am, len(prompt), 8)
    with atlas_cuda.Runtime(small_model, max_context=256, max_prefill=64, kv_fp16=True) as rt:
        for i, t in enumerate(prompt):
            want, am2 = rt.forward(int(t), i, i + 1 == len(prompt))
        b = rt.generate(am2, len(prompt), 8)
    err = np.abs(lg.astype(np.float64) - want).max()
    assert err <= 1e-3 * np.abs(want).max(), f"max|dlogit| {err}"
    assert am == am2
    np.testing.assert_array_equal(a, b)
