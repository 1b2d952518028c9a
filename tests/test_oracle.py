"""CPU: the oracle (C restatement, oracle/atlas_oracle.c) is pinned to the
reference's own outputs - the golden fixtures made by tests/golden/make_golden.py
from the reference compiled in place, and, where it is built, that compiled
reference itself."""
import hashlib
import os

import numpy as np
import pytest

import atlas_cuda

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TYPES = [atlas_cuda.TYPE_Q4_K, atlas_cuda.TYPE_Q6_K, atlas_cuda.TYPE_Q5_K, atlas_cuda.TYPE_Q5_0,
         atlas_cuda.TYPE_Q5_1, atlas_cuda.TYPE_Q8_0, atlas_cuda.TYPE_F16]


def _sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


@pytest.mark.parametrize("t", TYPES)
def test_oracle_dequant_matches_golden(oracle, t):
    g = np.load(os.path.join(GOLDEN, "dequant.npz"))
    raw, want = g[f"in_{t}"], g[f"out_{t}"]
    n = raw.size // atlas_cuda.BLOCK_BYTES[t]
    got = oracle.dequant(t, raw, n, atlas_cuda.BLOCK_ELEMS[t]).view(np.uint32)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("t", TYPES)
def test_oracle_dequant_matches_reference_random(oracle, ref, t):
    rng = np.random.default_rng(t)
    bb, be = atlas_cuda.BLOCK_BYTES[t], atlas_cuda.BLOCK_ELEMS[t]
    raw = rng.integers(0, 256, 2000 * bb, dtype=np.uint8)
    a = oracle.dequant(t, raw, 2000, be).view(np.uint32)
    b = ref.dequant(t, raw, 2000, be).view(np.uint32)
    np.testing.assert_array_equal(a, b)


def test_generator_matches_fixture(tiny_model):
    g = np.load(os.path.join(GOLDEN, "tiny.npz"))
    assert _sha256(tiny_model) == str(g["sha256"]), "synthetic GGUF bytes changed"


def test_oracle_forward_matches_golden_tiny(oracle, tiny_model):
    g = np.load(os.path.join(GOLDEN, "tiny.npz"))
    m = oracle.open(tiny_model)
    m.begin(64)
    prompt = g["prompt"]
    for i, t in enumerate(prompt):
        lg = m.forward(int(t), i)
        np.testing.assert_array_equal(lg, g["logits"][i])
    picks = []
    for s in range(32):
        nxt = m.argmax(lg)
        picks.append(nxt)
        lg = m.forward(nxt, len(prompt) + s)
    np.testing.assert_array_equal(np.array(picks, np.uint32), g["picks"])


def test_oracle_matvec_matches_reference(oracle, ref, tiny_untied_model):
    m = oracle.open(tiny_untied_model)
    r = ref.open(tiny_untied_model)
    rng = np.random.default_rng(3)
    for name in ("blk.0.attn_q.weight", "blk.1.attn_v.weight", "blk.0.ffn_down.weight", "output.weight"):
        t, (cols, rows), _ = m.tensor(name)
        x = rng.standard_normal(cols).astype(np.float32)
        np.testing.assert_array_equal(m.matvec(name, x), r.matvec(name, x, rows))
    r.close()


def test_oracle_forward_matches_reference_untied(oracle, ref, tiny_untied_model):
    m = oracle.open(tiny_untied_model)
    m.begin(64)
    r = ref.open(tiny_untied_model)
    for pos, tok in enumerate([1, 900, 44, 1000, 2]):
        np.testing.assert_array_equal(m.forward(tok, pos), r.forward(tok, pos))
    r.close()


def test_oracle_forward_matches_reference_qwen3(oracle, ref, tiny_qwen3_model):
    """qwen3 per-head q/k RMSNorm (src/brain_runtime.c:1727-1737): the oracle's
    logits equal the reference's bit for bit."""
    m = oracle.open(tiny_qwen3_model)
    assert m.qk_norm == 1
    m.begin(64)
    r = ref.open(tiny_qwen3_model)
    for pos, tok in enumerate([1, 900, 44, 1000, 2, 17]):
        np.testing.assert_array_equal(m.forward(tok, pos), r.forward(tok, pos))
    r.close()


@pytest.mark.slow
def test_oracle_cfg0_prompt_logits(oracle, model_dir):
    """Full-size Qwen2-1.5B shape: the oracle reproduces the reference's logits."""
    g = np.load(os.path.join(GOLDEN, "cfg0.npz"))
    cfg = {k[4:]: int(g[k]) for k in g.files if k.startswith("cfg_")}
    p = os.path.join(str(model_dir), "cfg0.gguf")
    if not os.path.exists(p):
        atlas_cuda.write_synthetic_gguf(p, tied=True, **cfg)
    assert _sha256(p) == str(g["sha256"])
    m = oracle.open(p)
    m.begin(80)
    prompt = g["prompt"]
    for i, t in enumerate(prompt):
        lg = m.forward(int(t), i, i + 1 == len(prompt))
    np.testing.assert_array_equal(lg.astype(np.float16), g["logits_prompt"])
    assert m.argmax(lg) == int(g["picks"][0])


@pytest.mark.parametrize("tied", [True, False])
def test_oracle_writer_bytes_equal_product_writer(model_dir, tied):
    """The CPU reference arm of the benchmark writes its model file with the
    writer built into liboracle.so (it never loads libatlas_cuda.so); the file
    must be byte-identical to the product library's."""
    import oracle_bind
    cfg = dict(hidden=768, layers=2, q_heads=6, kv_heads=2, ffn=1280, vocab=2048, context_length=4096,
               seed=42 + int(tied))
    a = os.path.join(str(model_dir), f"writer_product_{tied}.gguf")
    b = os.path.join(str(model_dir), f"writer_oracle_{tied}.gguf")
    atlas_cuda.write_synthetic_gguf(a, tied=tied, **cfg)
    oracle_bind.write_synthetic_gguf(b, tied=tied, **cfg)
    assert os.path.getsize(a) == os.path.getsize(b)
    assert _sha256(a) == _sha256(b)


def test_large_goldens_pin_their_model_files():
    """cfg1.npz / cfg2.npz (512-token prompts, made by the reference itself) name
    the sha256 of the model file they were made from and carry the prompt the
    benchmark decodes after."""
    for name, vocab in (("cfg1", 151936), ("cfg2", 152064)):
        p = os.path.join(GOLDEN, f"{name}.npz")
        if not os.path.exists(p):
            pytest.skip(f"{name}.npz not generated")
        g = np.load(p)
        assert len(str(g["sha256"])) == 64
        assert g["prompt"].shape == (512,) and int(g["prompt"].max()) < vocab
        assert g["picks"].shape == (32,) and int(g["picks"].max()) < vocab
        assert np.isfinite(g["logits_prompt"].astype(np.float32)).all()
        want = np.random.default_rng(1234).integers(0, vocab, 512).astype(np.uint32)
        np.testing.assert_array_equal(g["prompt"], want)


@pytest.mark.parametrize("case", __import__("conftest").OTHER_TYPES, ids=lambda c: c[0])
def test_oracle_forward_matches_reference_other_types(oracle, ref, model_dir, case):
    """Files whose projections and head use F16 / Q5_0 / Q5_1 / Q8_0 / Q5_K
    (dequant_block, src/brain_runtime.c:1017-1121), and types that change
    across layers: the oracle's logits equal the reference's bit for bit."""
    from conftest import other_type_model
    path = other_type_model(model_dir, case)
    m = oracle.open(path)
    m.begin(64)
    r = ref.open(path)
    for pos, tok in enumerate([1, 900, 44, 2000, 2, 17]):
        np.testing.assert_array_equal(m.forward(tok, pos), r.forward(tok, pos))
    r.close()
