"""CPU: the arithmetic and layout facts the batched GEMV (csrc/batch.cu) rests on.

* The staged-input swizzle: quad e4 of sequence s sits at 16-byte unit
  e4 * 8 + xcol(e4, s); the 8 lanes of every quarter warp of every k step's
  B-operand load must fall in 8 distinct bank groups, for the Q4_K word order
  (quads base + 2t) and the Q6_K one (base + t), and xcol must be a bijection
  of the 8 sequences for every quad (the in-place staging writes every slot
  once).
* The Q4_K scale folding: the binary16 1024 + q (or 1024 + 16 q) times sc
  (or sc / 16) plus -1024 sc (or -64 sc), rounded once (fma.rn.f16x2), is
  q sc exactly for every 4-bit q and 6-bit sc."""
import numpy as np


def xcol(e4, s, q4):
    """The column function of csrc/batch.cu (xcol)."""
    return s ^ ((((e4 >> 1) & 3) if q4 else (e4 & 3)) << 1)


def test_staging_swizzle_is_conflict_free_per_quarter_warp():
    q4_steps = [16 * c + 8 * hn + s for c in range(4) for hn in range(2) for s in range(2)]
    q6_steps = [32 * h + 8 * k + 4 * l16 for h in range(2) for k in range(4) for l16 in range(2)]
    for q4, steps, mul in ((True, q4_steps, 2), (False, q6_steps, 1)):
        for base in steps:
            for phase in range(4):
                groups = set()
                for lane in range(8 * phase, 8 * phase + 8):
                    g, t = lane >> 2, lane & 3
                    e4 = base + mul * t
                    groups.add((e4 * 8 + xcol(e4, g, q4)) % 8)
                assert len(groups) == 8, (q4, base, phase)
        for e4 in range(64):
            assert sorted(xcol(e4, s, q4) for s in range(8)) == list(range(8))


def _f16(x):
    return np.float64(np.float16(x))


def test_q4k_scale_folding_is_exact():
    for sc in range(64):
        for q in range(16):
            lo = np.float16(_f16(1024 + q) * _f16(sc) + _f16(-1024.0 * sc))        # one rounding
            hi = np.float16(_f16(1024 + 16 * q) * _f16(sc / 16.0) + _f16(-64.0 * sc))
            assert float(lo) == q * sc and float(hi) == q * sc, (q, sc)
    # the exponent-byte construction and the constants the kernel uses
    as_f16 = lambda bits: float(np.frombuffer(np.uint16(bits).tobytes(), np.float16)[0])
    for q in range(16):
        assert as_f16(0x6400 | q) == 1024 + q and as_f16(0x6400 | (16 * q)) == 1024 + 16 * q
    assert (as_f16(0xE400), as_f16(0xD400), as_f16(0x2C00)) == (-1024.0, -64.0, 0.0625)
