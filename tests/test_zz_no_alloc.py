"""GPU: atlas_cuda_gemv_noalloc, the GEMV entry point for callers that cannot
allocate device memory (a host that owns all of HBM, or a path that cannot
absorb cudaMalloc's device synchronisation). Its launch scratch is a static
device array of the library; this file checks that two calls in a row give
the oracle's result and the same result as atlas_cuda_gemv.

Collected last on purpose (file name), and safe in a fresh process: its first
call on the device does the one-time set-up."""
import numpy as np
import pytest

import atlas_cuda

pytestmark = pytest.mark.gpu


def _case(torch, t, rows, cols, seed):
    w = atlas_cuda.synth_blocks(t, rows * cols // 256, seed=seed, stream=t)
    x = np.random.default_rng(seed).standard_normal(cols).astype(np.float32)
    return w, x, torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()


def test_noalloc_gemv_matches_oracle_and_gemv_two_calls(torch_cuda, oracle):
    torch = torch_cuda
    cases = [(atlas_cuda.TYPE_Q4_K, 2048, 2048, 11), (atlas_cuda.TYPE_Q6_K, 1536, 8960, 12)]
    for t, rows, cols, seed in cases:
        w, x, d_w, d_x = _case(torch, t, rows, cols, seed)
        want = oracle.matvec_raw(t, w, rows, cols, x)
        ref = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        atlas_cuda.gemv(t, d_w, rows, cols, d_x, ref)
        torch.cuda.synchronize()
        a = ref.cpu().numpy()
        bound = 1e-4 * np.abs(want).max() + 1e-5   # the GEMV parity tests' bound (tests/test_gpu_kernels.py)
        for call in range(2):
            got = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
            atlas_cuda.gemv_noalloc(t, d_w, rows, cols, d_x, got)   # returns once y is complete
            b = got.cpu().numpy()
            assert np.isfinite(b).all(), call
            assert np.abs(b - want).max() <= bound, (call, np.abs(b - want).max(), bound)
            assert np.abs(b - a).max() <= bound, (call, np.abs(b - a).max(), bound)


def test_noalloc_gemv_rejects_oversized_input(torch_cuda):
    torch = torch_cuda
    d = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    x = torch.zeros(1 << 17, dtype=torch.float32, device="cuda")
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.gemv_noalloc(atlas_cuda.TYPE_Q4_K, d, 1, 1 << 17, x, x)
