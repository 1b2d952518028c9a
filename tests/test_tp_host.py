"""CPU: tensor-parallel host logic - the rank slices (atlas_cuda_tp_slice) and
the handle exchange over torch.distributed (gloo, world size 2)."""
import os
import socket

import numpy as np
import pytest

import atlas_cuda

SHAPES = {
    "7b": dict(hidden=3584, q_heads=28, kv_heads=4, ffn=18944, vocab=152064),
    "14b": dict(hidden=5120, q_heads=40, kv_heads=8, ffn=13824, vocab=152064),
    "32b": dict(hidden=5120, q_heads=40, kv_heads=8, ffn=27648, vocab=152064),
    "3b": dict(hidden=2048, q_heads=16, kv_heads=2, ffn=11008, vocab=151936),
}


@pytest.mark.parametrize("name", sorted(SHAPES))
@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_slices_tile_the_model(name, size):
    sh = SHAPES[name]
    if sh["kv_heads"] % size:
        with pytest.raises(atlas_cuda.AtlasError):
            atlas_cuda.tp_slice(sh, 0, size)
        return
    q_dim = sh["q_heads"] * 128
    sl = [atlas_cuda.tp_slice(sh, r, size) for r in range(size)]
    # heads, KV heads, FFN rows and vocab rows: contiguous, disjoint, complete
    for f0, fn, total in (("q_head0", "q_heads", sh["q_heads"]), ("kv_head0", "kv_heads", sh["kv_heads"]),
                          ("ffn_row0", "ffn_rows", sh["ffn"]), ("vocab_row0", "vocab_rows", sh["vocab"])):
        at = 0
        for s in sl:
            assert getattr(s, f0) == at and getattr(s, fn) > 0
            at += getattr(s, fn)
        assert at == total
    covered = np.zeros(q_dim, np.int32)
    for s in sl:
        assert s.q_heads == s.kv_heads * (sh["q_heads"] // sh["kv_heads"])   # query heads stay with their KV head
        assert s.ffn_row0 % 256 == 0 and s.ffn_rows % 256 == 0               # ffn_down column blocks
        assert s.vocab_row0 % 16 == 0 and s.vocab_rows % 16 == 0             # whole 16-row tiles
        # the o blocks hold exactly the rank's attention-output elements
        e0 = 256 * s.o_block0
        assert e0 + s.o_lo == 128 * s.q_head0 and s.o_hi - s.o_lo == 128 * s.q_heads
        assert 0 <= s.o_lo < 256 and s.o_hi <= 256 * s.o_blocks and 256 * (s.o_block0 + s.o_blocks) <= q_dim
        assert s.o_hi > 256 * (s.o_blocks - 1)
        covered[e0 + s.o_lo:e0 + s.o_hi] += 1
    assert (covered == 1).all()


def test_slice_rejects_bad_sizes():
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.tp_slice(SHAPES["7b"], 0, 3)
    with pytest.raises(atlas_cuda.AtlasError):
        atlas_cuda.tp_slice(SHAPES["7b"], 2, 2)


class _FakeRuntime:
    """Stands in for a device runtime: a rank-specific handle, records what connect gets."""

    def __init__(self, rank, size):
        self.tp_rank, self.tp_size = rank, size
        self.got = None

    def tp_handle(self):
        return bytes([self.tp_rank + 1]) * atlas_cuda.TP_HANDLE_BYTES

    def tp_connect(self, handles):
        self.got = handles


def _exchange_worker(rank, size, port, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=size)
    rt = _FakeRuntime(rank, size)
    atlas_cuda.connect_tp(rt)
    q.put((rank, rt.got))
    dist.destroy_process_group()


def test_connect_tp_exchanges_handles_in_rank_order():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    q = ctx.Queue()
    ps = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [bytes([r + 1]) * atlas_cuda.TP_HANDLE_BYTES for r in range(2)]
    assert got[0] == want and got[1] == want
