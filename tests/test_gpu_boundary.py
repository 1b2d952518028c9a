"""GPU: the reference's own runtime (src/brain_runtime.c, compiled in place as
oracle/_ref/libbrainref_gpu.so) with its device plugin (src/gpu_matvec.h)
taken from libatlas_cuda.so instead of the Direct3D 12 file - the drop-in the
plugin ABI exists for:
  * its `model.gguf --gpu-check` self-test (src/brain_runtime.c:1958-1984)
    passes by the reference's own criterion;
  * forward_token with the plugin on (every GEMV on the GPU) and with
    BRAIN_HYBRID=1 (rows split between the GPU and CPU threads,
    src/brain_runtime.c:1202-1244) gives the CPU runtime's logits and picks."""
import ctypes
import os

import numpy as np
import pytest

import atlas_cuda
import oracle_bind

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "oracle", "_ref", "libbrainref_gpu.so")
# vocab >= 8192 rows: the hybrid path splits the output head between GPU and CPU
BOUNDARY = dict(hidden=512, layers=2, q_heads=4, kv_heads=2, ffn=768, vocab=16384, context_length=512, seed=4242)


class RefGpu(oracle_bind.Reference):
    PATH = LIB

    def __init__(self):
        super().__init__()
        self.L.ref_gpu_init.argtypes = [ctypes.c_int]
        self.L.ref_main.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p)]


@pytest.fixture(scope="module")
def refgpu(torch_cuda):
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libbrainref_gpu.so is not built (make -C oracle ref-gpu)")
    return RefGpu()


@pytest.fixture(scope="module")
def boundary_model(model_dir):
    path = os.path.join(str(model_dir), "boundary.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, tied=False, **BOUNDARY)
    return path


def test_reference_gpu_check_passes_on_b200(refgpu, small_model, capfd):
    argv = (ctypes.c_char_p * 3)(b"atlas_dynamic_infer", small_model.encode(), b"--gpu-check")
    rc = refgpu.L.ref_main(3, argv)
    ctypes.CDLL(None).fflush(None)
    out = capfd.readouterr().out
    assert rc == 0, out
    assert out.count("GPU/CPU PASS") == 2, out


@pytest.mark.parametrize("hybrid", [0, 1])
def test_reference_forward_with_b200_plugin(refgpu, ref, boundary_model, hybrid):
    tokens = [5, 900, 77, 3000, 12000, 16383, 1]
    ref.open(boundary_model)
    want = [ref.forward(t, p) for p, t in enumerate(tokens)]
    ref.close()
    refgpu.open(boundary_model)
    try:
        assert refgpu.L.ref_gpu_init(hybrid) == 1, "brain_gpu_init failed"
        assert refgpu.L.ref_session_begin()
        got = [refgpu.forward(t, p) for p, t in enumerate(tokens)]
    finally:
        refgpu.L.ref_gpu_shutdown()
        refgpu.close()
    for p, (g, w) in enumerate(zip(got, want)):
        err = np.abs(g.astype(np.float64) - w).max()
        assert err <= 1e-3 * np.abs(w).max(), (p, err)
        assert int(np.argmax(g)) == int(np.argmax(w)), p


CLI_GPU = os.path.join(ROOT, "oracle", "_ref", "atlas_dynamic_infer")
CLI_CPU = os.path.join(ROOT, "oracle", "_ref", "atlas_dynamic_infer_cpu")


def _cli(exe, *args):
    import subprocess
    env = dict(os.environ, ATLAS_REF_THREADS="8")
    return subprocess.run(["timeout", "300", exe, *args], capture_output=True, env=env)


def test_reference_cli_drop_in_matches_cpu(torch_cuda, small_model):
    """The reference's own atlas_dynamic_infer (argv, chat template,
    tokenizer, greedy sampling, stop tokens, stdout text), linked against
    libatlas_cuda.so as its device plugin, prints exactly what its CPU build
    prints for the same prompt, and keeps the exit codes."""
    if not (os.path.exists(CLI_GPU) and os.path.exists(CLI_CPU)):
        pytest.skip("oracle/_ref/atlas_dynamic_infer is not built (make -C oracle ref-gpu)")
    prompt = "Hello there, how are you?"
    gpu = _cli(CLI_GPU, small_model, prompt, "16")
    cpu = _cli(CLI_CPU, small_model, prompt, "16")
    assert gpu.returncode == 0 and cpu.returncode == 0, (gpu.stderr[-2000:], cpu.stderr[-2000:])
    assert b"Direct3D 12 GPU" in gpu.stderr          # the plugin came up (the reference's own device message)
    assert b"CPU fallback" in cpu.stderr
    assert gpu.stdout == cpu.stdout and len(gpu.stdout) > 1
    check = _cli(CLI_GPU, small_model, "--gpu-check")
    assert check.returncode == 0 and check.stdout.count(b"GPU/CPU PASS") == 2, check.stdout
    assert _cli(CLI_GPU, small_model, prompt, "0").returncode == 2      # max_new_tokens out of range


NATIVE = os.path.join(ROOT, "-1.7-atlas---apollo_b200", "atlas_dynamic_infer")


def test_native_cli_matches_reference_cli(torch_cuda, small_model):
    """The native atlas_dynamic_infer (host/cli.c over the library's batched
    prefill and graph decode) prints what the reference's CPU build prints for
    greedy prompts, with the same exit codes, self-test and confidence line."""
    if not (os.path.exists(NATIVE) and os.path.exists(CLI_CPU)):
        pytest.skip("atlas_dynamic_infer (make -C -1.7-atlas---apollo_b200) or the reference CLI is not built")
    for prompt, n in (("Hello there, how are you?", "24"), ("Don't stop: 1234 + 5678 = ?", "40"),
                      ("<|im_start|>user\nplain template<|im_end|>\n<|im_start|>assistant\n", "16")):
        got = _cli(NATIVE, small_model, prompt, n)
        want = _cli(CLI_CPU, small_model, prompt, n)
        assert got.returncode == 0 and want.returncode == 0, (got.stderr[-2000:], want.stderr[-2000:])
        assert got.stdout == want.stdout and len(got.stdout) > 1, (prompt, got.stdout, want.stdout)
    conf = _cli(NATIVE, small_model, "Explain why", "8", "0", "--confidence")
    assert conf.returncode == 0
    line = conf.stdout.split(b"\n")[-2]
    assert line.startswith(b"\x1eATLAS_CONFIDENCE=") and line.endswith(b"\x1e"), conf.stdout
    check = _cli(NATIVE, small_model, "--gpu-check")
    assert check.returncode == 0 and check.stdout.count(b"GPU/CPU PASS") == 2, check.stdout
    assert _cli(NATIVE, small_model, "x", "0").returncode == 2       # max_new_tokens out of range
    assert _cli(NATIVE, small_model, "x", "769").returncode == 2
    assert _cli(NATIVE, small_model, "x", "4", "5").returncode == 2  # min_new > max_new
    assert _cli(NATIVE, small_model).returncode == 2                 # usage
    sampled = _cli(NATIVE, small_model, "Hello", "12", "3")          # top-k sampling, at least 3 tokens
    assert sampled.returncode == 0 and len(sampled.stdout) > 1
