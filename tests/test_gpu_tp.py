"""GPU: tensor-parallel decode (2 / 4 / 8 ranks, one process per GPU) against the oracle.

The 7B and 14B layer widths (2 layers, untied Q6_K head) split by KV head:
the prompt's last logits (all ranks' vocab slices) within the contract's
2e-2 * max|logit| (held here to 1e-3) and 32 greedy tokens identical to the
oracle's, on every rank. Skipped when the box has fewer GPUs than ranks."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import atlas_cuda
from test_gpu_model import WIDE

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
N_PROMPT, STEPS = 12, 32


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.slow
@pytest.mark.parametrize("name,tp", [("7b_width", 2), ("14b_width", 2), ("7b_width", 4), ("14b_width", 8)])
def test_tp_matches_oracle(torch_cuda, oracle, model_dir, tmp_path, name, tp):
    if _gpus() < tp:
        pytest.skip(f"{tp} GPUs needed")
    cfg = WIDE[name]
    p = os.path.join(str(model_dir), f"{name}.gguf")
    if not os.path.exists(p):
        atlas_cuda.write_synthetic_gguf(p, tied=False, **cfg)
    out = str(tmp_path / "tp.npz")
    seed = cfg["seed"]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_worker.py"), p, out, str(N_PROMPT), str(STEPS), str(seed)]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    got = np.load(out)

    m = oracle.open(p)
    m.begin(64)
    prompt = got["prompt"]
    np.testing.assert_array_equal(prompt, np.random.default_rng(seed).integers(0, cfg["vocab"], N_PROMPT))
    for i, t in enumerate(prompt):
        want = m.forward(int(t), i, i + 1 == len(prompt))
    err = np.abs(got["logits"].astype(np.float64) - want).max()
    assert err <= 1e-3 * np.abs(want).max(), f"max|dlogit| {err}"
    want_picks, lg = [], want
    for s in range(STEPS):
        want_picks.append(m.argmax(lg))
        if s + 1 < STEPS:
            lg = m.forward(want_picks[-1], N_PROMPT + s)
    for rank_picks in got["picks"]:
        np.testing.assert_array_equal(rank_picks, np.array(want_picks, np.uint32))


@pytest.mark.slow
@pytest.mark.parametrize("tp", [2, 4])
def test_tp_fp16_cache_matches_one_gpu(torch_cuda, model_dir, tmp_path, tp):
    """A binary16 KV cache under tensor parallelism (the 14B long-context
    workload's cache): every rank keeps its KV heads' cache in binary16 and
    runs the tensor-core decode attention over it. Against the same model on
    one GPU with the same cache (the cache rounds alike; only the partial-row
    sums of o and down are grouped by rank): the prompt's last logits within
    1e-3 * max|logit| and 32 greedy tokens identical on every rank."""
    if _gpus() < tp:
        pytest.skip(f"{tp} GPUs needed")
    cfg = WIDE["14b_width"]
    p = os.path.join(str(model_dir), "14b_width.gguf")
    if not os.path.exists(p):
        atlas_cuda.write_synthetic_gguf(p, tied=False, **cfg)
    out = str(tmp_path / "tp16.npz")
    seed = cfg["seed"]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_worker.py"), p, out, str(N_PROMPT), str(STEPS), str(seed), "fp16"]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    got = np.load(out)
    with atlas_cuda.Runtime(p, max_context=N_PROMPT + STEPS + 8, kv_fp16=True) as rt:
        want, first = rt.prefill(got["prompt"])
        want_picks = np.concatenate([[first], rt.generate(first, N_PROMPT, STEPS - 1)]).astype(np.uint32)
    err = np.abs(got["logits"].astype(np.float64) - want).max()
    assert err <= 1e-3 * np.abs(want).max(), f"max|dlogit| {err}"
    for rank_picks in got["picks"]:
        np.testing.assert_array_equal(rank_picks, want_picks)
