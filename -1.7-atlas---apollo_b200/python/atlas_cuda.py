"""ctypes binding of libatlas_cuda's C ABI (include/atlas_cuda.h, include/atlas_runtime.h,
include/gpu_matvec.h, include/atlas_synth.h).

The library is the in-tree ``libatlas_cuda.so`` next to this package's ``csrc/``.
Loading fails loudly when it is missing: there is no Python or CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libatlas_cuda.so")

ATLAS_OK = 0
ERRORS = {
    -1: "EINVAL", -2: "ENODEV", -3: "ENOMEM", -4: "ECUDA", -5: "ETIMEOUT", -6: "ENCCL", -7: "ERANGE",
}
TYPE_F32, TYPE_F16, TYPE_Q5_0, TYPE_Q5_1, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 0, 1, 6, 7, 8, 12, 13, 14
BLOCK_BYTES = {TYPE_F16: 2, TYPE_Q5_0: 22, TYPE_Q5_1: 24, TYPE_Q8_0: 34, TYPE_Q4_K: 144, TYPE_Q5_K: 176,
               TYPE_Q6_K: 210}
BLOCK_ELEMS = {TYPE_F16: 1, TYPE_Q5_0: 32, TYPE_Q5_1: 32, TYPE_Q8_0: 32, TYPE_Q4_K: 256, TYPE_Q5_K: 256,
               TYPE_Q6_K: 256}

# Every symbol the public headers declare (checked by the CPU test suite).
EXPORTS = [
    "atlas_cuda_create", "atlas_cuda_destroy", "atlas_cuda_last_error", "atlas_cuda_prefill",
    "atlas_cuda_decode", "atlas_cuda_generate", "atlas_cuda_stats", "atlas_cuda_dequant",
    "atlas_cuda_gemv", "atlas_cuda_gemm", "atlas_cuda_device_info", "atlas_cuda_trace_step",
    "atlas_cuda_device_ms", "atlas_cuda_trace_graph", "atlas_cuda_gemv_noalloc", "atlas_cuda_tp_slice", "atlas_cuda_tp_handle",
    "atlas_cuda_tp_connect", "atlas_cuda_prefill_seq", "atlas_cuda_generate_batch", "atlas_cuda_decode_batch",
    "brain_gpu_init", "brain_gpu_matvec_batch", "brain_gpu_matvec", "brain_gpu_shutdown",
    "atlas_rt_open", "atlas_rt_close", "atlas_rt_error", "atlas_rt_shape", "atlas_rt_data_base",
    "atlas_rt_find_tensor", "atlas_rt_file_bytes", "atlas_rt_device", "atlas_rt_forward_token",
    "atlas_rt_prefill", "atlas_rt_generate",
    "atlas_synth_write_gguf", "atlas_synth_q4k_blocks", "atlas_synth_q6k_blocks", "atlas_synth_file_size",
]


class AtlasError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class SynthConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("hidden", "layers", "q_heads", "kv_heads", "head_dim", "ffn", "vocab", "context_length")] + [
        ("rope_base", ctypes.c_float), ("tied", ctypes.c_int32), ("qkv_bias", ctypes.c_int32),
        ("threads", ctypes.c_int32), ("seed", ctypes.c_uint64), ("qk_norm", ctypes.c_int32),
        ("alt_type", ctypes.c_int32), ("layer_mix", ctypes.c_int32)]


class Shape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("hidden_size", "q_dim", "kv_dim", "q_heads", "kv_heads", "head_dim", "ffn_size", "layers",
                 "max_context", "vocab_size")] + [
        ("rope_base", ctypes.c_float), ("has_qk_norm", ctypes.c_int32), ("architecture", ctypes.c_char * 64)]


class TensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("n_dims", ctypes.c_uint32), ("dims", ctypes.c_uint64 * 4),
                ("type", ctypes.c_uint32), ("offset", ctypes.c_uint64)]


class RtOptions(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("max_context", ctypes.c_uint32), ("max_prefill", ctypes.c_uint32),
                ("kv_fp16", ctypes.c_int32), ("no_device", ctypes.c_int32), ("tp_rank", ctypes.c_int32),
                ("tp_size", ctypes.c_int32), ("max_batch", ctypes.c_uint32)]


class ModelDesc(ctypes.Structure):
    """AtlasModelDesc (include/atlas_cuda.h)."""
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("hidden", "q_dim", "kv_dim", "q_heads", "kv_heads", "head_dim", "ffn", "layers", "vocab",
                 "max_context", "max_prefill")] + [
        ("rope_base", ctypes.c_float), ("rms_eps", ctypes.c_float)] + [
        (n, ctypes.c_int32) for n in ("has_qk_norm", "kv_fp16", "device", "tp_rank", "tp_size")] + [
        ("max_batch", ctypes.c_uint32)]


class TpSlice(ctypes.Structure):
    """AtlasTpSlice: one tensor-parallel rank's share of the model."""
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("q_head0", "q_heads", "kv_head0", "kv_heads", "o_block0", "o_blocks", "o_lo", "o_hi",
                 "ffn_row0", "ffn_rows", "vocab_row0", "vocab_rows")]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


TP_HANDLE_BYTES = 64


class BrainGpuMatvec(ctypes.Structure):
    _fields_ = [("offset", ctypes.c_uint64), ("rows", ctypes.c_uint64), ("cols", ctypes.c_uint64),
                ("type", ctypes.c_uint32), ("input", ctypes.c_void_p), ("output", ctypes.c_void_p)]


_LIB = None


def lib() -> ctypes.CDLL:
    """Load the in-tree library (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        P, U32, U64, I32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
        L.atlas_cuda_last_error.restype = ctypes.c_char_p
        L.atlas_cuda_last_error.argtypes = [P]
        L.atlas_cuda_dequant.argtypes = [U32, P, U64, P, P]
        L.atlas_cuda_gemv.argtypes = [U32, P, U64, U64, P, P, P]
        L.atlas_cuda_gemv_noalloc.argtypes = [U32, P, U64, U64, P, P, P]
        L.atlas_cuda_gemm.argtypes = [U32, P, U64, U64, P, U64, P, P]
        L.atlas_cuda_device_info.argtypes = [I32, P, P, P]
        L.atlas_cuda_decode.argtypes = [P, U32, U32, P, P]
        L.atlas_cuda_prefill.argtypes = [P, P, U32, U32, P, P]
        L.atlas_cuda_generate.argtypes = [P, U32, U32, U32, P]
        L.atlas_cuda_stats.argtypes = [P, P, P]
        L.atlas_cuda_device_ms.argtypes = [P, P]
        L.atlas_cuda_trace_step.argtypes = [P, U32, U32, P, ctypes.c_size_t, P, P, P]
        L.atlas_cuda_trace_graph.argtypes = [P, U32, U32, P, ctypes.c_size_t, P, P, P]
        L.atlas_cuda_tp_slice.argtypes = [P, I32, I32, P]
        L.atlas_cuda_tp_handle.argtypes = [P, P]
        L.atlas_cuda_tp_connect.argtypes = [P, P]
        L.atlas_rt_open.argtypes = [ctypes.c_char_p, P, P]
        L.atlas_rt_close.argtypes = [P]
        L.atlas_rt_error.restype = ctypes.c_char_p
        L.atlas_rt_error.argtypes = [P]
        L.atlas_rt_shape.argtypes = [P, P]
        L.atlas_rt_data_base.restype = U64
        L.atlas_rt_data_base.argtypes = [P]
        L.atlas_rt_find_tensor.argtypes = [P, ctypes.c_char_p, P]
        L.atlas_rt_file_bytes.restype = P
        L.atlas_rt_file_bytes.argtypes = [P, P]
        L.atlas_rt_device.restype = P
        L.atlas_rt_device.argtypes = [P]
        L.atlas_rt_forward_token.argtypes = [P, U32, U32, P, P]
        L.atlas_rt_prefill.argtypes = [P, P, U32, U32, P, P]
        L.atlas_rt_generate.argtypes = [P, U32, U32, U32, P]
        L.atlas_cuda_prefill_seq.argtypes = [P, U32, P, U32, U32, P, P]
        L.atlas_cuda_generate_batch.argtypes = [P, U32, P, P, U32, P]
        L.atlas_cuda_decode_batch.argtypes = [P, U32, P, P, P, P]
        L.atlas_synth_write_gguf.argtypes = [P, ctypes.c_char_p]
        L.atlas_synth_q4k_blocks.argtypes = [U64, U64, P, U64]
        L.atlas_synth_q6k_blocks.argtypes = [U64, U64, P, U64]
        L.atlas_synth_file_size.restype = U64
        L.atlas_synth_file_size.argtypes = [P]
        L.brain_gpu_init.argtypes = [P, ctypes.c_size_t]
        L.brain_gpu_matvec_batch.argtypes = [P, ctypes.c_size_t]
        L.brain_gpu_matvec.argtypes = [U64, U32, U64, U64, P, P]
        _LIB = L
    return _LIB


def check(rc: int, where: str = "", handle=None) -> None:
    if rc != ATLAS_OK:
        msg = lib().atlas_cuda_last_error(handle)
        raise AtlasError(rc, f"{where}: {msg.decode() if msg else ''}")


def _ptr(a) -> ctypes.c_void_p:
    """Host numpy array or device torch tensor -> void*."""
    if a is None:
        return ctypes.c_void_p(0)
    if hasattr(a, "data_ptr"):
        return ctypes.c_void_p(a.data_ptr())
    return a.ctypes.data_as(ctypes.c_void_p)


def write_synthetic_gguf(path: str, *, hidden: int, layers: int, q_heads: int, kv_heads: int, ffn: int, vocab: int,
                         head_dim: int = 128, context_length: int = 32768, rope_base: float = 1e6,
                         tied: bool = True, qkv_bias: bool = True, seed: int = 0, threads: int = 0,
                         qk_norm: bool = False, alt_type: int = 0, layer_mix: bool = False) -> int:
    """qk_norm: a qwen3 file (per-head q/k RMSNorm weights). alt_type: another
    block type (F16, Q5_0, Q5_1, Q8_0, Q5_K) for attn_q, ffn_gate, ffn_up,
    ffn_down and the head. layer_mix: odd layers' attn_v and ffn_down are Q4_K."""
    cfg = SynthConfig(hidden, layers, q_heads, kv_heads, head_dim, ffn, vocab, context_length, rope_base,
                      int(tied), int(qkv_bias), threads, seed, int(qk_norm), int(alt_type), int(layer_mix))
    rc = lib().atlas_synth_write_gguf(ctypes.byref(cfg), path.encode())
    if rc != 0:
        raise RuntimeError(f"synthetic GGUF write failed: {path}")
    return lib().atlas_synth_file_size(ctypes.byref(cfg))


def synth_blocks(type_id: int, n: int, seed: int = 0, stream: int = 0):
    import numpy as np
    out = np.zeros(n * BLOCK_BYTES[type_id], np.uint8)
    fn = lib().atlas_synth_q4k_blocks if type_id == TYPE_Q4_K else lib().atlas_synth_q6k_blocks
    fn(seed, stream, _ptr(out), n)
    return out


class Runtime:
    """Reference-shaped model API: open a GGUF, forward tokens, prefill, generate."""

    def __init__(self, path: str, *, device: int = 0, max_context: int = 0, max_prefill: int = 0,
                 kv_fp16: bool = False, no_device: bool = False, tp_rank: int = 0, tp_size: int = 1,
                 max_batch: int = 1):
        self._h = ctypes.c_void_p()
        opt = RtOptions(device, max_context, max_prefill, int(kv_fp16), int(no_device), tp_rank, tp_size, max_batch)
        self.tp_rank, self.tp_size = tp_rank, tp_size
        rc = lib().atlas_rt_open(path.encode(), ctypes.byref(opt), ctypes.byref(self._h))
        if rc != ATLAS_OK:
            msg = lib().atlas_rt_error(self._h).decode()
            lib().atlas_rt_close(self._h)
            self._h = None
            raise AtlasError(rc, f"atlas_rt_open({path}): {msg}")
        s = Shape()
        lib().atlas_rt_shape(self._h, ctypes.byref(s))
        self.shape = s
        self.vocab = s.vocab_size

    def _check(self, rc: int, where: str) -> None:
        if rc != ATLAS_OK:
            raise AtlasError(rc, f"{where}: {lib().atlas_rt_error(self._h).decode()}")

    def tensor(self, name: str) -> TensorInfo | None:
        t = TensorInfo()
        return t if lib().atlas_rt_find_tensor(self._h, name.encode(), ctypes.byref(t)) else None

    @property
    def data_base(self) -> int:
        return lib().atlas_rt_data_base(self._h)

    def forward(self, token: int, pos: int, want_logits: bool = True):
        import numpy as np
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        am = ctypes.c_uint32()
        self._check(lib().atlas_rt_forward_token(self._h, token, pos, _ptr(logits), ctypes.byref(am)), "forward")
        return logits, am.value

    def prefill(self, ids, pos0: int = 0, want_logits: bool = True):
        import numpy as np
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        am = ctypes.c_uint32()
        self._check(lib().atlas_rt_prefill(self._h, _ptr(ids), len(ids), pos0, _ptr(logits), ctypes.byref(am)),
                    "prefill")
        return logits, am.value

    def generate(self, first: int, pos0: int, steps: int):
        import numpy as np
        out = np.zeros(steps, np.uint32)
        self._check(lib().atlas_rt_generate(self._h, first, pos0, steps, _ptr(out)), "generate")
        return out

    def prefill_seq(self, seq: int, ids, pos0: int = 0, want_logits: bool = True):
        """atlas_cuda_prefill into sequence seq's KV cache (open with max_batch > seq)."""
        import numpy as np
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        am = ctypes.c_uint32()
        dev = lib().atlas_rt_device(self._h)
        check(lib().atlas_cuda_prefill_seq(dev, seq, _ptr(ids), len(ids), pos0, _ptr(logits), ctypes.byref(am)),
              "prefill_seq", dev)
        return logits, am.value

    def generate_batch(self, first, pos0, steps: int):
        """Greedy steps of len(first) sequences at once: array [nseq, steps] of picks."""
        import numpy as np
        first = np.ascontiguousarray(first, dtype=np.uint32)
        pos0 = np.ascontiguousarray(pos0, dtype=np.uint32)
        out = np.zeros((len(first), steps), np.uint32)
        dev = lib().atlas_rt_device(self._h)
        check(lib().atlas_cuda_generate_batch(dev, len(first), _ptr(first), _ptr(pos0), steps, _ptr(out)),
              "generate_batch", dev)
        return out

    def decode_batch(self, ids, pos, want_logits: bool = True):
        """One step of len(ids) sequences: (logits [nseq, vocab] or None, picks [nseq])."""
        import numpy as np
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        pos = np.ascontiguousarray(pos, dtype=np.uint32)
        logits = np.zeros((len(ids), self.vocab), np.float32) if want_logits else None
        am = np.zeros(len(ids), np.uint32)
        dev = lib().atlas_rt_device(self._h)
        check(lib().atlas_cuda_decode_batch(dev, len(ids), _ptr(ids), _ptr(pos), _ptr(logits), _ptr(am)),
              "decode_batch", dev)
        return logits, am

    def trace_step(self, token: int, pos: int):
        """One traced decode step: (stamps[cta, phase, 4], inner stamps[cta, phase, 8], phase kind codes)."""
        import numpy as np
        dev = lib().atlas_rt_device(self._h)
        nc, nph = ctypes.c_uint32(), ctypes.c_uint32()
        lib().atlas_cuda_trace_step(dev, token, pos, None, 0, ctypes.byref(nc), ctypes.byref(nph), None)
        per = nc.value * nph.value
        buf = np.zeros(per * 12, np.uint64)
        kinds = np.zeros(nph.value, np.uint32)
        check(lib().atlas_cuda_trace_step(dev, token, pos, _ptr(buf), buf.size, ctypes.byref(nc), ctypes.byref(nph),
                                          _ptr(kinds)), "trace_step", dev)
        return buf[:per * 4].reshape(nc.value, nph.value, 4), buf[per * 4:].reshape(nc.value, nph.value, 8), kinds

    def trace_graph(self, token: int, pos: int):
        """One decode step of the graph engine with device timestamps:
        array [launch, cta, word] of globaltimer ns (0 = not recorded); word 0
        start, 1 inputs ready, 2 + w warp w done (atlas_cuda_trace_graph)."""
        import numpy as np
        dev = lib().atlas_rt_device(self._h)
        nl, nc, nw = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
        check(lib().atlas_cuda_trace_graph(dev, token, pos, None, 0, ctypes.byref(nl), ctypes.byref(nc),
                                           ctypes.byref(nw)), "trace_graph", dev)
        buf = np.zeros(nl.value * nc.value * nw.value, np.uint64)
        check(lib().atlas_cuda_trace_graph(dev, token, pos, _ptr(buf), buf.size, None, None, None), "trace_graph", dev)
        return buf.reshape(nl.value, nc.value, nw.value)

    def tp_slice(self) -> TpSlice:
        """This rank's share of the model (the whole model without tensor parallelism)."""
        s = self.shape
        return tp_slice(dict(hidden=s.hidden_size, q_heads=s.q_heads, kv_heads=s.kv_heads, ffn=s.ffn_size,
                             vocab=s.vocab_size), self.tp_rank, self.tp_size)

    def tp_handle(self) -> bytes:
        """The exchange area of this rank, to hand to every other rank."""
        buf = ctypes.create_string_buffer(TP_HANDLE_BYTES)
        dev = lib().atlas_rt_device(self._h)
        check(lib().atlas_cuda_tp_handle(dev, buf), "atlas_cuda_tp_handle", dev)
        return buf.raw

    def tp_connect(self, handles) -> None:
        """handles: every rank's tp_handle() in rank order; builds the decode step."""
        if len(handles) != self.tp_size or any(len(b) != TP_HANDLE_BYTES for b in handles):
            raise ValueError("tp_connect needs tp_size handles of TP_HANDLE_BYTES bytes")
        buf = ctypes.create_string_buffer(b"".join(handles), TP_HANDLE_BYTES * self.tp_size)
        dev = lib().atlas_rt_device(self._h)
        check(lib().atlas_cuda_tp_connect(dev, buf), "atlas_cuda_tp_connect", dev)

    def stats(self):
        """(kernel launches since creation, device ms of the last call, device ms of all calls)."""
        n = ctypes.c_uint64()
        ms = ctypes.c_double()
        tot = ctypes.c_double()
        dev = lib().atlas_rt_device(self._h)
        lib().atlas_cuda_stats(dev, ctypes.byref(n), ctypes.byref(ms))
        lib().atlas_cuda_device_ms(dev, ctypes.byref(tot))
        return n.value, ms.value, tot.value

    def close(self) -> None:
        if self._h:
            lib().atlas_rt_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_slice(shape: dict, rank: int, size: int) -> TpSlice:
    """atlas_cuda_tp_slice for a shape given as hidden / q_heads / kv_heads / ffn / vocab."""
    d = ModelDesc()
    d.hidden, d.q_heads, d.kv_heads, d.ffn, d.vocab = (shape[k] for k in ("hidden", "q_heads", "kv_heads", "ffn",
                                                                           "vocab"))
    d.head_dim, d.q_dim, d.kv_dim = 128, 128 * d.q_heads, 128 * d.kv_heads
    out = TpSlice()
    check(lib().atlas_cuda_tp_slice(ctypes.byref(d), rank, size, ctypes.byref(out)), "atlas_cuda_tp_slice")
    return out


def connect_tp(rt: "Runtime", group=None) -> None:
    """Exchange the ranks' handles through torch.distributed (any backend:
    the handles are 64 host bytes each) and connect this rank's runtime."""
    import torch.distributed as dist
    handles = [None] * rt.tp_size
    dist.all_gather_object(handles, rt.tp_handle(), group=group)
    rt.tp_connect(handles)


def dequant(type_id: int, d_blocks, nblocks: int, d_out, stream: int = 0) -> None:
    check(lib().atlas_cuda_dequant(type_id, _ptr(d_blocks), nblocks, _ptr(d_out), ctypes.c_void_p(stream)),
          "atlas_cuda_dequant")


def gemv(type_id: int, d_w, rows: int, cols: int, d_x, d_y, stream: int = 0) -> None:
    check(lib().atlas_cuda_gemv(type_id, _ptr(d_w), rows, cols, _ptr(d_x), _ptr(d_y), ctypes.c_void_p(stream)),
          "atlas_cuda_gemv")


def gemv_noalloc(type_id: int, d_w, rows: int, cols: int, d_x, d_y, stream: int = 0) -> None:
    check(lib().atlas_cuda_gemv_noalloc(type_id, _ptr(d_w), rows, cols, _ptr(d_x), _ptr(d_y),
                                        ctypes.c_void_p(stream)), "atlas_cuda_gemv_noalloc")


def gemm(type_id: int, d_w, rows: int, cols: int, d_x, tokens: int, d_y, stream: int = 0) -> None:
    check(lib().atlas_cuda_gemm(type_id, _ptr(d_w), rows, cols, _ptr(d_x), tokens, _ptr(d_y),
                                ctypes.c_void_p(stream)), "atlas_cuda_gemm")
