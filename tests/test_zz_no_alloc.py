"""GPU: atlas_cuda_gemv_noalloc, the GEMV entry point for callers that cannot
allocate device memory (its launch scratch is a static device array), gives
the same result as atlas_cuda_gemv on two calls in a row.

Collected last on purpose (file name), and safe in a fresh process: its first
call on the device does the one-time set-up."""
import numpy as np
import pytest

import atlas_cuda

pytestmark = pytest.mark.gpu


def _case(torch, t, rows, cols, seed):
    w = atlas_cuda.synth_blocks(t, rows * cols // 256, seed=seed, stream=t)
    x = np.random.default_rng(seed).standard_normal(cols).astype(np.float32)
    return torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()


def test_noalloc_gemv_matches_gemv_two_calls(torch_cuda):
    torch = torch_cuda
    cases = [(atlas_cuda.TYPE_Q4_K, 2048, 2048, 11), (atlas_cuda.TYPE_Q6_K, 1536, 8960, 12)]
    for t, rows, cols, seed in cases:
        d_w, d_x = _case(torch, t, rows, cols, seed)
        want = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        got = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        atlas_cuda.gemv(t, d_w, rows, cols, d_x, want)
        atlas_cuda.gemv_noalloc(t, d_w, rows, cols, d_x, got)
        torch.cuda.synchronize()
        a, b = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(b).all()
        # same tolerance as the GEMV parity tests (tests/test_gpu_kernels.py)
        assert np.abs(a - b).max() <= 1e-4 * np.abs(a).max() + 1e-5


def test_noalloc_gemv_rejects_oversized_input(torch_cuda):
    torch = torch_cuda
    d = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    x = torch.zeros(1 << 17, dtype=torch.float32, device="cuda")
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.gemv_noalloc(atlas_cuda.TYPE_Q4_K, d, 1, 1 << 17, x, x)
