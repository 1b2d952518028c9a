"""GPU: several independent sequences per decode step (atlas_cuda_prefill_seq,
atlas_cuda_generate_batch, atlas_cuda_decode_batch).

The reference decodes one sequence per process (forward_token,
src/brain_runtime.c:1698); each sequence of a batched step must give what the
oracle gives for that sequence alone: logits within 1e-3 max|logit| and the
same greedy picks."""
import os

import numpy as np
import pytest

import atlas_cuda

pytestmark = pytest.mark.gpu
BATCH = dict(hidden=1024, layers=4, q_heads=8, kv_heads=2, ffn=2816, vocab=4096, context_length=1024, seed=515)


def _close(got, want, tol=1e-3):
    err = np.abs(got.astype(np.float64) - want).max()
    assert err <= tol * np.abs(want).max(), (err, np.abs(want).max())


@pytest.fixture(scope="module", params=[False, True], ids=["uniform", "layer_mix"])
def batch_model(request, model_dir):
    path = os.path.join(str(model_dir), f"batch_{request.param}.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, tied=not request.param, layer_mix=request.param, **BATCH)
    return path


def _oracle_run(oracle, path, prompt, steps):
    m = oracle.open(path)
    m.begin(len(prompt) + steps + 2)
    for i, t in enumerate(prompt):
        lg = m.forward(int(t), i, i + 1 == len(prompt))
    picks, logits = [], [lg]
    for s in range(steps):
        picks.append(m.argmax(lg))
        lg = m.forward(picks[-1], len(prompt) + s)
        logits.append(lg)
    return picks, logits


@pytest.mark.parametrize("nseq", [8, 3])
def test_batched_steps_match_single_sequences(torch_cuda, oracle, batch_model, nseq):
    rng = np.random.default_rng(60 + nseq)
    prompts = [rng.integers(0, BATCH["vocab"], int(rng.integers(5, 48))).astype(np.uint32) for _ in range(nseq)]
    steps = 16
    want = [_oracle_run(oracle, batch_model, p, steps) for p in prompts]
    with atlas_cuda.Runtime(batch_model, max_context=128, max_batch=8) as rt:
        first = []
        for s, p in enumerate(prompts):
            lg, am = rt.prefill_seq(s, p)
            _close(lg, want[s][1][0])
            assert am == want[s][0][0], s
            first.append(am)
        pos0 = [len(p) for p in prompts]
        got = rt.generate_batch(first, pos0, steps - 1)
        for s in range(nseq):
            np.testing.assert_array_equal(got[s], np.array(want[s][0][1:], np.uint32), err_msg=f"sequence {s}")
        # one more step through decode_batch: the logits of each sequence
        ids = [want[s][0][steps - 1] for s in range(nseq)]
        pos = [pos0[s] + steps - 1 for s in range(nseq)]
        logits, am = rt.decode_batch(ids, pos)
        for s in range(nseq):
            _close(logits[s], want[s][1][steps])
            assert am[s] == int(np.argmax(want[s][1][steps])), s


def test_batched_step_errors(torch_cuda, batch_model, model_dir):
    with atlas_cuda.Runtime(batch_model, max_context=64, max_batch=2) as rt:
        with pytest.raises(atlas_cuda.AtlasError):
            rt.generate_batch([1, 2, 3], [0, 0, 0], 2)          # more sequences than max_batch
        with pytest.raises(atlas_cuda.AtlasError):
            rt.prefill_seq(2, np.arange(4, dtype=np.uint32))     # sequence >= max_batch
        with pytest.raises(atlas_cuda.AtlasError):
            rt.generate_batch([1, 5000], [0, 0], 2)             # token >= vocab
        rt.prefill_seq(1, np.arange(1, 9, dtype=np.uint32))
        out = rt.generate_batch([3, 4], [0, 8], 4)               # the handle still works
        assert out.shape == (2, 4)
    path = os.path.join(str(model_dir), "batch_q8.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, tied=False, alt_type=8, hidden=512, layers=2, q_heads=4, kv_heads=2,
                                        ffn=768, vocab=2048, context_length=256, seed=3)
    with atlas_cuda.Runtime(path, max_context=64, max_batch=2) as rt:
        with pytest.raises(atlas_cuda.AtlasError):
            rt.generate_batch([1, 2], [0, 0], 2)                # other block types: one sequence per step
