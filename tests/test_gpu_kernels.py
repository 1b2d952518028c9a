"""GPU: kernel-level parity through the C ABI against the oracle.

Dequantization is bit-exact against the reference's own outputs. Random
bytes make some fp16 scales Inf/NaN; where the reference's value is a NaN the
GPU value must be a NaN too, but the payload is not compared: x86 SSE
propagates an input NaN's payload while the GPU returns the canonical NaN, and
IEEE 754 leaves NaN payloads unspecified. Every other value (Inf, -0.0,
subnormals) is compared bit for bit. The decode GEMV engine is compared with the
oracle's restatement of matvec_rows (src/brain_runtime.c:1133); its fp32
accumulation order differs from the reference's single sequential sum, so the
bar is max|dy| <= 1e-4 * max|y| + 1e-5, far inside the reference's own GPU
self-check bound 0.005 * max|y| + 0.002 (src/brain_runtime.c:1976)."""
import ctypes
import os

import numpy as np
import pytest

import atlas_cuda

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TYPES = [atlas_cuda.TYPE_Q4_K, atlas_cuda.TYPE_Q6_K, atlas_cuda.TYPE_Q5_K, atlas_cuda.TYPE_Q5_0,
         atlas_cuda.TYPE_Q5_1, atlas_cuda.TYPE_Q8_0, atlas_cuda.TYPE_F16]


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_bits_equal(got_bits, want_bits):
    got, want = got_bits.view(np.float32), want_bits.view(np.float32)
    nan = np.isnan(want)
    np.testing.assert_array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got_bits[~nan], want_bits[~nan])


@pytest.mark.parametrize("t", TYPES)
def test_dequant_bit_exact_golden(torch_cuda, t):
    torch = torch_cuda
    g = np.load(os.path.join(GOLDEN, "dequant.npz"))
    raw, want = g[f"in_{t}"], g[f"out_{t}"]
    n = raw.size // atlas_cuda.BLOCK_BYTES[t]
    d_in = _dev(torch, raw)
    d_out = torch.empty(n * atlas_cuda.BLOCK_ELEMS[t], dtype=torch.float32, device="cuda")
    atlas_cuda.dequant(t, d_in, n, d_out)
    torch.cuda.synchronize()
    assert_bits_equal(d_out.cpu().numpy().view(np.uint32), want)


@pytest.mark.parametrize("t", [atlas_cuda.TYPE_Q4_K, atlas_cuda.TYPE_Q6_K])
def test_dequant_bit_exact_large(torch_cuda, oracle, t):
    torch = torch_cuda
    n = 200_000
    rng = np.random.default_rng(t)
    raw = np.concatenate([rng.integers(0, 256, (n // 2) * atlas_cuda.BLOCK_BYTES[t], dtype=np.uint8),
                          atlas_cuda.synth_blocks(t, n - n // 2, seed=3)])
    want = oracle.dequant(t, raw, n, 256).view(np.uint32)
    d_in = _dev(torch, raw)
    d_out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
    atlas_cuda.dequant(t, d_in, n, d_out)
    torch.cuda.synchronize()
    got = d_out.cpu().numpy().view(np.uint32)
    assert_bits_equal(got, want)
    # the synthetic-distribution half has no NaN at all and is fully bit-exact
    np.testing.assert_array_equal(got[(n // 2) * 256:], want[(n // 2) * 256:])


SHAPES = [(1, 256), (7, 512), (256, 1536), (2048, 2048), (513, 3584), (1536, 8960), (2048, 11008), (300, 13824),
          (96, 18944), (64, 27648), (4000, 5120)]


@pytest.mark.parametrize("t", [atlas_cuda.TYPE_Q4_K, atlas_cuda.TYPE_Q6_K])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_matches_oracle(torch_cuda, oracle, t, rows, cols):
    torch = torch_cuda
    nb = rows * cols // 256
    w = atlas_cuda.synth_blocks(t, nb, seed=rows * 7 + cols, stream=t)
    x = np.random.default_rng(rows + cols).standard_normal(cols).astype(np.float32)
    want = oracle.matvec_raw(t, w, rows, cols, x)
    # a 2-byte offset exercises Q6_K rows that start off 4-byte alignment
    off = 2 if t == atlas_cuda.TYPE_Q6_K else 0
    buf = torch.zeros(w.size + 64, dtype=torch.uint8, device="cuda")
    buf[off:off + w.size] = _dev(torch, w)
    d_w = buf[off:]
    d_x, d_y = _dev(torch, x), torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    atlas_cuda.gemv(t, d_w, rows, cols, d_x, d_y)
    torch.cuda.synchronize()
    got = d_y.cpu().numpy()
    err = np.abs(got - want).max()
    assert err <= 1e-4 * np.abs(want).max() + 1e-5, (err, np.abs(want).max())


def test_gemv_repeated_calls_and_streams(torch_cuda, oracle):
    torch = torch_cuda
    t, rows, cols = atlas_cuda.TYPE_Q4_K, 1024, 2048
    w = atlas_cuda.synth_blocks(t, rows * cols // 256, seed=5)
    d_w = _dev(torch, w)
    s = torch.cuda.Stream()
    for i in range(5):
        x = np.random.default_rng(i).standard_normal(cols).astype(np.float32)
        d_x, d_y = _dev(torch, x), torch.empty(rows, dtype=torch.float32, device="cuda")
        with torch.cuda.stream(s):
            atlas_cuda.gemv(t, d_w, rows, cols, d_x, d_y, stream=s.cuda_stream)
        s.synchronize()
        want = oracle.matvec_raw(t, w, rows, cols, x)
        assert np.abs(d_y.cpu().numpy() - want).max() <= 1e-4 * np.abs(want).max() + 1e-5


def test_gemv_rejects_bad_arguments(torch_cuda):
    torch = torch_cuda
    d = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.gemv(atlas_cuda.TYPE_Q4_K, d, 1, 100, d, d)            # cols not a multiple of 256
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.gemv(99, d, 1, 256, d, d)                               # unknown type
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.gemv(atlas_cuda.TYPE_Q4_K, d[1:], 1, 256, d, d)         # misaligned Q4_K


def test_brain_gpu_plugin_gpu_check(torch_cuda, oracle, tiny_untied_model):
    """The reference's --gpu-check (src/brain_runtime.c:1958-1984) against this plugin."""
    L = atlas_cuda.lib()
    data = np.fromfile(tiny_untied_model, dtype=np.uint8)
    data = np.concatenate([data, np.zeros((-data.size) % 4, np.uint8)])
    assert L.brain_gpu_init(data.ctypes.data_as(ctypes.c_void_p), data.size) == 1
    m = oracle.open(tiny_untied_model)
    rt = atlas_cuda.Runtime(tiny_untied_model, no_device=True)
    try:
        for name in ("blk.0.attn_q.weight", "blk.0.attn_v.weight", "blk.1.ffn_down.weight", "output.weight"):
            ti = rt.tensor(name)
            cols, rows = ti.dims[0], ti.dims[1]
            x = (np.sin(np.arange(cols, dtype=np.float32) * np.float32(0.0137)) * np.float32(0.25)).astype(np.float32)
            out = np.zeros(rows, np.float32)
            ok = L.brain_gpu_matvec(rt.data_base + ti.offset, ti.type, rows, cols,
                                    x.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p))
            assert ok == 1
            cpu = m.matvec(name, x)
            err = np.abs(out.astype(np.float64) - cpu).max()
            assert err <= np.abs(cpu).max() * 0.005 + 0.002, (name, err)
            assert err <= 1e-4 * np.abs(cpu).max() + 1e-5, (name, err)
        # batch of three sharing one input, as tensor_matvec_batch issues them
        ops = (atlas_cuda.BrainGpuMatvec * 3)()
        outs = []
        x = np.random.default_rng(0).standard_normal(512).astype(np.float32)
        for i, name in enumerate(("blk.1.attn_q.weight", "blk.1.attn_k.weight", "blk.1.attn_v.weight")):
            ti = rt.tensor(name)
            o = np.zeros(ti.dims[1], np.float32)
            outs.append((name, o))
            ops[i] = atlas_cuda.BrainGpuMatvec(rt.data_base + ti.offset, ti.dims[1], ti.dims[0], ti.type,
                                               x.ctypes.data_as(ctypes.c_void_p).value,
                                               o.ctypes.data_as(ctypes.c_void_p).value)
        assert L.brain_gpu_matvec_batch(ops, 3) == 1
        for name, o in outs:
            cpu = m.matvec(name, x)
            assert np.abs(o - cpu).max() <= 1e-4 * np.abs(cpu).max() + 1e-5
        assert L.brain_gpu_matvec_batch(ops, 4) == 0      # more than 3 ops is refused (src/gpu_matvec.c:218)
    finally:
        L.brain_gpu_shutdown()
        rt.close()


def test_plugin_generic_types(torch_cuda, oracle):
    """Q5_0 / Q5_1 / Q8_0 / Q5_K rows through the plugin's generic kernel."""
    L = atlas_cuda.lib()
    rng = np.random.default_rng(9)
    for t in (atlas_cuda.TYPE_Q8_0, atlas_cuda.TYPE_Q5_0, atlas_cuda.TYPE_Q5_1, atlas_cuda.TYPE_Q5_K):
        rows, cols = 64, 512
        be, bb = atlas_cuda.BLOCK_ELEMS[t], atlas_cuda.BLOCK_BYTES[t]
        w = rng.integers(0, 256, rows * cols // be * bb, dtype=np.uint8)
        # finite scales: clear the fp16 exponent's top bits of d (and of m for Q5_1)
        blk = w.reshape(-1, bb)
        blk[:, 1] &= 0x3b
        if t in (atlas_cuda.TYPE_Q5_1, atlas_cuda.TYPE_Q5_K):
            blk[:, 3] &= 0x3b
        img = np.concatenate([np.zeros(64, np.uint8), w, np.zeros((-w.size) % 4, np.uint8)])
        assert L.brain_gpu_init(img.ctypes.data_as(ctypes.c_void_p), img.size) == 1
        x = rng.standard_normal(cols).astype(np.float32)
        out = np.zeros(rows, np.float32)
        assert L.brain_gpu_matvec(64, t, rows, cols, x.ctypes.data_as(ctypes.c_void_p),
                                  out.ctypes.data_as(ctypes.c_void_p)) == 1
        want = oracle.matvec_raw(t, w, rows, cols, x)
        assert np.abs(out - want).max() <= 1e-4 * np.abs(want).max() + 1e-5
        L.brain_gpu_shutdown()
