"""ctypes bindings of the ORACLE libraries (test infrastructure only).

Oracle:    oracle/liboracle.so, this repository's C restatement of the
           reference path (oracle/atlas_oracle.c).
Reference: oracle/_ref/libbrainref.so, the reference's own src/brain_runtime.c
           compiled in place by oracle/Makefile (present where it was built).
"""
import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
P, U32, U64 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64


def _p(a):
    return ctypes.c_void_p(0) if a is None else a.ctypes.data_as(ctypes.c_void_p)


def write_synthetic_gguf(path, *, hidden, layers, q_heads, kv_heads, ffn, vocab, head_dim=128, context_length=32768,
                         rope_base=1e6, tied=True, qkv_bias=True, seed=0, threads=0, qk_norm=False, alt_type=0,
                         layer_mix=False):
    """The seeded synthetic GGUF writer as built into liboracle.so (the same
    writer source as the product library's atlas_synth_write_gguf; a CPU test
    checks that both produce identical bytes). Lets the CPU reference arm make
    its model file without loading libatlas_cuda.so."""
    from atlas_cuda import SynthConfig
    L = ctypes.CDLL(Oracle.PATH)
    L.atlas_synth_write_gguf.argtypes = [P, ctypes.c_char_p]
    cfg = SynthConfig(hidden, layers, q_heads, kv_heads, head_dim, ffn, vocab, context_length, rope_base, int(tied),
                      int(qkv_bias), threads, seed, int(qk_norm), int(alt_type), int(layer_mix))
    if L.atlas_synth_write_gguf(ctypes.byref(cfg), path.encode()) != 0:
        raise RuntimeError(f"synthetic GGUF write failed: {path}")


class Oracle:
    PATH = os.path.join(ROOT, "oracle", "liboracle.so")

    def __init__(self):
        L = ctypes.CDLL(self.PATH)
        L.oracle_half_to_float.restype = ctypes.c_float
        L.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        L.oracle_dequant.argtypes = [U32, P, P, U64]
        L.oracle_matvec_raw.argtypes = [U32, P, U64, U64, P, P]
        L.oracle_open.restype = P
        L.oracle_open.argtypes = [ctypes.c_char_p]
        L.oracle_close.argtypes = [P]
        L.oracle_shape.argtypes = [P, P, P]
        L.oracle_tensor.argtypes = [P, ctypes.c_char_p, P, P, P]
        L.oracle_matvec.argtypes = [P, ctypes.c_char_p, P, P]
        L.oracle_session_begin.argtypes = [P, U32]
        L.oracle_forward.argtypes = [P, U32, U64, ctypes.c_int, P]
        L.oracle_argmax.restype = U32
        L.oracle_argmax.argtypes = [P, U64]
        L.oracle_last_hidden.argtypes = [P, P]
        L.oracle_kv_row.argtypes = [P, U32, U64, P, P]
        L.oracle_rope_table.argtypes = [ctypes.c_int, ctypes.c_float, ctypes.c_int, P, P]
        self.L = L

    def dequant(self, type_id, blocks, nblocks, elems_per_block):
        out = np.zeros(nblocks * elems_per_block, np.float32)
        assert self.L.oracle_dequant(type_id, _p(blocks), _p(out), nblocks)
        return out

    def matvec_raw(self, type_id, w, rows, cols, x):
        y = np.zeros(rows, np.float32)
        assert self.L.oracle_matvec_raw(type_id, _p(w), rows, cols, _p(np.ascontiguousarray(x, np.float32)), _p(y))
        return y

    def open(self, path):
        return OracleModel(self, path)


class OracleModel:
    def __init__(self, o, path):
        self.o, self.L = o, o.L
        self.h = self.L.oracle_open(path.encode())
        assert self.h, f"oracle could not open {path}"
        sh = (U32 * 11)()
        rb = ctypes.c_float()
        self.L.oracle_shape(self.h, sh, ctypes.byref(rb))
        (self.hidden, self.q_dim, self.kv_dim, self.q_heads, self.kv_heads, self.head_dim, self.ffn, self.layers,
         self.max_context, self.vocab, self.qk_norm) = list(sh)
        self.rope_base = rb.value

    def tensor(self, name):
        t = U32()
        dims = (U64 * 2)()
        ptr = ctypes.c_void_p()
        if not self.L.oracle_tensor(self.h, name.encode(), ctypes.byref(t), dims, ctypes.byref(ptr)):
            return None
        return t.value, (dims[0], dims[1]), ptr.value

    def tensor_bytes(self, name):
        t, (cols, rows), ptr = self.tensor(name)
        from atlas_cuda import BLOCK_BYTES, BLOCK_ELEMS
        n = rows * cols // BLOCK_ELEMS[t] * BLOCK_BYTES[t] if t != 0 else rows * cols * 4
        return t, cols, rows, np.ctypeslib.as_array((ctypes.c_uint8 * n).from_address(ptr))

    def matvec(self, name, x):
        t, (cols, rows), _ = self.tensor(name)
        y = np.zeros(rows, np.float32)
        assert self.L.oracle_matvec(self.h, name.encode(), _p(np.ascontiguousarray(x, np.float32)), _p(y))
        return y

    def begin(self, max_positions):
        assert self.L.oracle_session_begin(self.h, max_positions)

    def forward(self, token, pos, want_logits=True):
        lg = np.zeros(self.vocab, np.float32) if want_logits else None
        assert self.L.oracle_forward(self.h, token, pos, int(want_logits), _p(lg))
        return lg

    def argmax(self, logits):
        return int(self.L.oracle_argmax(_p(logits), len(logits)))

    def close(self):
        if self.h:
            self.L.oracle_close(self.h)
            self.h = None

    def __del__(self):
        self.close()


class Reference:
    PATH = os.path.join(ROOT, "oracle", "_ref", "libbrainref.so")

    @classmethod
    def load(cls):
        return cls() if os.path.exists(cls.PATH) else None

    def __init__(self):
        L = ctypes.CDLL(self.PATH)
        L.ref_open.argtypes = [ctypes.c_char_p]
        L.ref_half_to_float.restype = ctypes.c_float
        L.ref_half_to_float.argtypes = [ctypes.c_uint16]
        L.ref_dequant_blocks.argtypes = [U32, P, P, ctypes.c_size_t]
        L.ref_matvec.argtypes = [ctypes.c_char_p, P, P]
        L.ref_forward.argtypes = [U32, U64, ctypes.c_int, P]
        L.ref_sample_greedy.restype = U32
        L.ref_sample_greedy.argtypes = [P, U64]
        L.ref_shape.argtypes = [P, P]
        L.ref_data_base.restype = U64
        L.ref_kv_row.argtypes = [U32, U64, P, P]
        L.ref_last_hidden.argtypes = [P]
        L.ref_fill_cache.argtypes = [U64, U64]
        self.L = L
        self.vocab = None

    def dequant(self, type_id, blocks, nblocks, elems_per_block):
        out = np.zeros(nblocks * elems_per_block, np.float32)
        self.L.ref_dequant_blocks(type_id, _p(blocks), _p(out), nblocks)
        return out

    def open(self, path):
        assert self.L.ref_open(path.encode()), f"reference could not open {path}"
        sh = (U32 * 11)()
        rb = ctypes.c_float()
        self.L.ref_shape(sh, ctypes.byref(rb))
        self.vocab = sh[9]
        self.hidden = sh[0]
        assert self.L.ref_session_begin()
        return self

    def forward(self, token, pos, want_logits=True):
        lg = np.zeros(self.vocab, np.float32) if want_logits else None
        assert self.L.ref_forward(token, pos, int(want_logits), _p(lg))
        return lg

    def matvec(self, name, x, rows):
        y = np.zeros(rows, np.float32)
        assert self.L.ref_matvec(name.encode(), _p(np.ascontiguousarray(x, np.float32)), _p(y))
        return y

    def greedy(self, logits):
        return int(self.L.ref_sample_greedy(_p(logits), len(logits)))

    def fill_cache(self, filled, upto):
        """Cache positions [filled, upto) repeat rows [0, filled) (benchmark helper)."""
        assert self.L.ref_fill_cache(filled, upto)

    def close(self):
        self.L.ref_close()
