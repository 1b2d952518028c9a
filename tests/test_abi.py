"""CPU: the C-ABI library loads, exports every function the public headers
declare, parses GGUF files like the reference, and the seeded model writer is
deterministic. No device compute is called here."""
import ctypes
import glob
import os
import re

import numpy as np
import pytest

import atlas_cuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M):
            if m.group(1) not in ("if", "while", "for", "return", "sizeof"):
                names.add(m.group(1))
    return sorted(names)


def test_library_exports_every_declared_function(lib):
    declared = _declared_functions()
    assert len(declared) >= 30
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared) == set(atlas_cuda.EXPORTS)


def test_runtime_parses_like_reference(oracle, tiny_model):
    rt = atlas_cuda.Runtime(tiny_model, no_device=True)
    m = oracle.open(tiny_model)
    s = rt.shape
    assert (s.hidden_size, s.q_dim, s.kv_dim, s.q_heads, s.kv_heads, s.head_dim, s.ffn_size, s.layers,
            s.vocab_size) == (m.hidden, m.q_dim, m.kv_dim, m.q_heads, m.kv_heads, m.head_dim, m.ffn, m.layers,
                              m.vocab)
    assert s.architecture == b"qwen2" and abs(s.rope_base - 1e6) < 1
    t = rt.tensor("blk.1.ffn_down.weight")
    assert t is not None and t.type == 14 and (t.dims[0], t.dims[1]) == (768, 512)
    assert rt.tensor("no.such.tensor") is None
    rt.close()


def test_runtime_tied_output_and_context_cap(model_dir):
    p = os.path.join(str(model_dir), "ctx.gguf")
    atlas_cuda.write_synthetic_gguf(p, hidden=256, layers=1, q_heads=2, kv_heads=1, ffn=256, vocab=512,
                                    context_length=20000, seed=5)
    rt = atlas_cuda.Runtime(p, no_device=True)
    # the reference caps at 8192 (src/brain_runtime.c:549); this runtime does not
    assert rt.shape.max_context == 20000
    rt.close()


def test_runtime_rejects_bad_files(model_dir):
    bad = os.path.join(str(model_dir), "bad.gguf")
    with open(bad, "wb") as f:
        f.write(b"NOPE" + b"\0" * 64)
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.Runtime(bad, no_device=True)
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.Runtime(os.path.join(str(model_dir), "missing.gguf"), no_device=True)
    # truncated directory
    good = os.path.join(str(model_dir), "trunc_src.gguf")
    atlas_cuda.write_synthetic_gguf(good, hidden=256, layers=1, q_heads=2, kv_heads=1, ffn=256, vocab=512, seed=1)
    data = open(good, "rb").read()
    trunc = os.path.join(str(model_dir), "trunc.gguf")
    with open(trunc, "wb") as f:
        f.write(data[:4096])
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.Runtime(trunc, no_device=True)


def test_synth_deterministic_across_threads(model_dir):
    a, b = (os.path.join(str(model_dir), n) for n in ("d1.gguf", "d2.gguf"))
    kw = dict(hidden=512, layers=1, q_heads=4, kv_heads=2, ffn=512, vocab=600, seed=11)
    atlas_cuda.write_synthetic_gguf(a, threads=1, **kw)
    atlas_cuda.write_synthetic_gguf(b, threads=3, **kw)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_synth_block_distributions(oracle):
    q4 = atlas_cuda.synth_blocks(atlas_cuda.TYPE_Q4_K, 4096, seed=1).reshape(4096, 144)
    d = q4[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    dmin = q4[:, 2:4].copy().view(np.float16).astype(np.float32).ravel()
    for v in (d, dmin):
        assert v.min() >= 0.99e-4 and v.max() <= 2.001e-3
    q6 = atlas_cuda.synth_blocks(atlas_cuda.TYPE_Q6_K, 4096, seed=2).reshape(4096, 210)
    sc = q6[:, 192:208].view(np.int8)
    assert sc.min() == -32 and sc.max() == 31
    d6 = q6[:, 208:210].copy().view(np.float16).astype(np.float32).ravel()
    assert d6.min() >= 0.99e-4 and d6.max() <= 2.001e-3
    # dequantized values are finite and in the expected range
    w = oracle.dequant(atlas_cuda.TYPE_Q6_K, q6.ravel(), 4096, 256)
    assert np.isfinite(w).all() and np.abs(w).max() < 2.2e-3 * 32 * 32


def test_no_gpu_calls_fail_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    sm = ctypes.c_int()
    assert lib.atlas_cuda_device_info(0, ctypes.byref(sm), None, None) == -2
    assert lib.brain_gpu_init(None, 0) == 0
