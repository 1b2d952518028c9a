"""Shared fixtures. `-m gpu` tests need a B200; everything else runs on CPU.

The oracle libraries (oracle/liboracle.so: this repository's C restatement of
the reference path; oracle/_ref/libbrainref.so: the reference's own
src/brain_runtime.c compiled in place) are test infrastructure: they are only
ever used here as the checker.
"""
import ctypes
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "-1.7-atlas---apollo_b200")
sys.path.insert(0, os.path.join(PKG, "python"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import atlas_cuda  # noqa: E402
import oracle_bind  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: full-size model case (tens of seconds)")


@pytest.fixture(scope="session")
def lib():
    return atlas_cuda.lib()


@pytest.fixture(scope="session")
def oracle():
    return oracle_bind.Oracle()


@pytest.fixture(scope="session")
def ref():
    r = oracle_bind.Reference.load()
    if r is None:
        pytest.skip("oracle/_ref (the reference compiled in place) is not built")
    return r


TINY = dict(hidden=512, layers=2, q_heads=4, kv_heads=2, ffn=768, vocab=1024, context_length=512, seed=1234)
SMALL = dict(hidden=1024, layers=4, q_heads=8, kv_heads=2, ffn=2816, vocab=4096, context_length=1024, seed=99)


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


def _model(model_dir, name, cfg, tied=True):
    path = os.path.join(str(model_dir), f"{name}.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, tied=tied, **cfg)
    return path


# Models with the reference's other block types (F16, Q5_0, Q5_1, Q8_0, Q5_K)
# in attn_q, ffn_gate/up/down and the head; odd layers' attn_v / ffn_down Q4_K
# where layer_mix is set. (name, alt_type, tied, layer_mix)
OTHER_TYPES = [("f16", 1, True, False), ("q5_0", 6, False, True), ("q5_1", 7, True, True),
               ("q8_0", 8, False, False), ("q5_k", 13, False, True), ("q4q6_mix", 0, True, True)]
OTHER = dict(hidden=512, layers=3, q_heads=4, kv_heads=2, ffn=768, vocab=2048, context_length=512, seed=777)


def other_type_model(model_dir, case):
    name, alt, tied, mix = case
    path = os.path.join(str(model_dir), f"types_{name}.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, tied=tied, alt_type=alt, layer_mix=mix, **OTHER)
    return path


@pytest.fixture(scope="session")
def tiny_model(model_dir):
    return _model(model_dir, "tiny", TINY)


@pytest.fixture(scope="session")
def tiny_untied_model(model_dir):
    return _model(model_dir, "tiny_untied", dict(TINY, seed=4321), tied=False)


@pytest.fixture(scope="session")
def tiny_qwen3_model(model_dir):
    """qwen3: per-head q/k RMSNorm, no q/k/v bias."""
    path = os.path.join(str(model_dir), "tiny_qwen3.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, tied=True, qkv_bias=False, qk_norm=True, **dict(TINY, seed=2468))
    return path


@pytest.fixture(scope="session")
def small_model(model_dir):
    return _model(model_dir, "small", SMALL)


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
