"""CPU: the integer-MMA decode GEMV tasks (csrc/decode2.cu: m4_stage_x<W,
true>, m4_bsel, q4k_task8, q6k_task8), emulated lane by lane.

The emulation follows the kernel's register-level steps - the staged int8
planes and their chunk layout, every lane's A words (raw quant words masked /
merged exactly as the kernel does, including the 2-byte-misaligned Q6_K loads
through aligned words and funnel shifts), its B operand address, the
m16n8k32 fragment layout of PTX's mma.sync (A u8 16x32 row-major, B s8 32x8
column-major, s32 accumulators), the integer scale application and the fp32
finish - and compares the 16 row sums of a task with the float64 product of
the oracle's dequantized rows. It also checks that the B loads of every MMA
are conflict-free per half warp and that the integer sums cannot overflow."""
import numpy as np
import pytest

import atlas_cuda

F32 = np.float32


# ---------------------------------------------------------------- staging ----

def stage_block(x):
    """m4_stage_x<W, true> for one 256-element block: (1024-byte area, the 16
    sums of e, 1 / 2^k)."""
    x = np.asarray(x, F32)
    m = F32(np.fmax.reduce(np.abs(x)))   # fmaxf: a NaN operand is skipped
    k = 0
    if m > 0 and np.isfinite(m):
        k = 6 - int(np.floor(np.log2(np.float64(m))))
        if k > 126:
            k = 126
        elif F32(m * F32(2.0 ** k)) >= F32(127.5):
            k -= 1
    sc = F32(2.0 ** k)
    with np.errstate(invalid="ignore"):   # inf - inf in a non-finite block, as on the GPU
        e = (x * sc).astype(F32)
        hi = np.rint(e).astype(F32)
        r1 = ((e - hi).astype(F32) * F32(128)).astype(F32)
        mid = np.rint(r1).astype(F32)
        lo = np.rint(((r1 - mid).astype(F32) * F32(128)).astype(F32)).astype(F32)
    nonfinite = not np.isfinite(x).all()
    planes = [cvt_s32(hi), cvt_s32(mid), cvt_s32(lo)]
    if not nonfinite:
        assert planes[0].min() >= -127 and planes[0].max() <= 127
        assert all(p.min() >= -64 and p.max() <= 64 for p in planes[1:])
    area = np.zeros(1024, np.uint8)
    for ei in range(256):
        for pl in range(3):
            area[(ei >> 3) * 32 + pl * 8 + (ei & 7)] = planes[pl][ei] & 0xFF
    # 16-element sums in the kernel's order: lanes hold 4 elements, (e0 + e1) + (e2 + e3),
    # then adds across lanes xor 1 and xor 2
    s4 = ((e[0::4] + e[1::4]).astype(F32) + (e[2::4] + e[3::4]).astype(F32)).astype(F32)
    s8 = (s4 + s4.reshape(-1, 2)[:, ::-1].reshape(-1)).astype(F32)
    s16 = (s8[0::4] + s8[2::4]).astype(F32)
    return area, s16, (F32(np.nan) if nonfinite else F32(2.0 ** -k))


def cvt_s32(f):
    """The GPU's float -> int32 conversion: NaN -> 0, saturating at the int32 range."""
    f = np.asarray(f, np.float64)
    return np.where(np.isnan(f), 0, np.clip(np.nan_to_num(f, posinf=2.0 ** 31 - 1, neginf=-2.0 ** 31),
                                            -2.0 ** 31, 2.0 ** 31 - 1)).astype(np.int64)


# ------------------------------------------------------- register helpers ----

def u32(b, off):
    return int.from_bytes(bytes(b[off:off + 4]), "little")


def funnel_r(lo, hi, sh):
    return ((hi << 32 | lo) >> sh) & 0xFFFFFFFF


def ld8_u2(buf, addr):
    a = addr & ~3
    sh = (addr & 3) * 8
    v = [u32(buf, a + 4 * i) for i in range(3)]
    return funnel_r(v[0], v[1], sh), funnel_r(v[1], v[2], sh)


def ld16_u2(buf, addr):
    a = addr & ~3
    sh = (addr & 3) * 8
    v = [u32(buf, a + 4 * i) for i in range(5)]
    return [funnel_r(v[i], v[i + 1], sh) for i in range(4)]


def s32(v):
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v & 0x80000000 else v


def prmt_sx(x, sel):
    """prmt.b32 default mode with b = 0."""
    src = x.to_bytes(4, "little") + bytes(4)
    out = 0
    for i in range(4):
        n = (sel >> (4 * i)) & 0xF
        byte = src[n & 7]
        if n & 8:
            byte = 0xFF if byte & 0x80 else 0
        out |= byte << (8 * i)
    return out


def sx_sel(k):
    return k | ((k | 8) * 0x1110)


def h2f(bits):
    return np.float64(np.frombuffer(np.uint16(bits).tobytes(), np.float16)[0]).astype(F32)


def bsel(lane, q6):
    """m4_bsel."""
    g, t = lane >> 2, lane & 3
    act = (g >> 2) == (t >> 1) and (g & 3) < 3
    if q6:
        return 32 * t + 8 * ((g & 3) if act else 3)
    return 512 * (t >> 1) + 64 * (t & 1) + 8 * (g & 3) if act else 512 * (g >> 2) + 24


def mma(regs):
    """regs[lane] = (a0, a1, a2, a3, b0, b1) -> per lane (d0, d1, d2, d3), D = A B."""
    A = np.zeros((16, 32), np.int64)
    B = np.zeros((32, 8), np.int64)
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        a0, a1, a2, a3, b0, b1 = regs[lane]
        for i in range(4):
            A[g, 4 * t + i] = (a0 >> (8 * i)) & 0xFF
            A[g + 8, 4 * t + i] = (a1 >> (8 * i)) & 0xFF
            A[g, 16 + 4 * t + i] = (a2 >> (8 * i)) & 0xFF
            A[g + 8, 16 + 4 * t + i] = (a3 >> (8 * i)) & 0xFF
            bb0, bb1 = (b0 >> (8 * i)) & 0xFF, (b1 >> (8 * i)) & 0xFF
            B[4 * t + i, g] = bb0 - 256 if bb0 & 0x80 else bb0
            B[16 + 4 * t + i, g] = bb1 - 256 if bb1 & 0x80 else bb1
    D = A @ B
    out = []
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        out.append((D[g, 2 * t], D[g, 2 * t + 1], D[g + 8, 2 * t], D[g + 8, 2 * t + 1]))
    return out


def rows_of(o):
    """m4_rows: lanes t of row group g summed -> rows g, g + 8."""
    y = np.zeros(16, F32)
    for g in range(8):
        y[g] = (F32(o[4 * g][0] + o[4 * g + 1][0]) + F32(o[4 * g + 2][0] + o[4 * g + 3][0]))
        y[g + 8] = (F32(o[4 * g][1] + o[4 * g + 1][1]) + F32(o[4 * g + 2][1] + o[4 * g + 3][1]))
    return y


# ------------------------------------------------------------------ tasks ----

def q4k_task8(rows, area, xs):
    """rows: 16 Q4_K blocks (144 bytes each, 16-byte aligned slot rows)."""
    o = []
    st = []
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        H = [[u32(rows[r], 4 * i) for i in range(4)] for r in (g, g + 8)]
        SC, MN = [], []
        for Hr in H:
            sc03, m03 = Hr[1] & 0x3F3F3F3F, Hr[2] & 0x3F3F3F3F
            sc47 = (Hr[3] & 0x0F0F0F0F) | ((Hr[1] >> 2) & 0x30303030)
            m47 = ((Hr[3] >> 4) & 0x0F0F0F0F) | ((Hr[2] >> 2) & 0x30303030)
            SC.append(sc47 if t >= 2 else sc03)
            MN.append(m47 if t >= 2 else m03)
        st.append(dict(H=H, SC=SC, MN=MN, T=[0, 0, 0, 0], M=[F32(0), F32(0)], off=16 + 64 * (t >> 1) + 16 * (t & 1)))
    for pi in range(2):
        for nu in range(2):
            k = 0xF0F0F0F0 if nu else 0x0F0F0F0F
            D = [(0, 0, 0, 0)] * 32
            for h in range(2):
                regs = []
                for lane in range(32):
                    g, t = lane >> 2, lane & 3
                    s = st[lane]
                    W0 = [u32(rows[g], s["off"] + 32 * pi + 4 * i) for i in range(4)]
                    W1 = [u32(rows[g + 8], s["off"] + 32 * pi + 4 * i) for i in range(4)]
                    xp = bsel(lane, False) + 256 * pi + 128 * nu + 32 * h
                    regs.append((W0[2 * h] & k, W1[2 * h] & k, W0[2 * h + 1] & k, W1[2 * h + 1] & k,
                                 u32(area, xp), u32(area, xp + 4)))
                Dh = mma(regs)
                D = [tuple(D[l][i] + Dh[l][i] for i in range(4)) for l in range(32)]
            for lane in range(32):
                t = lane & 3
                s = st[lane]
                sh = 8 * (2 * pi + nu)
                s0 = ((s["SC"][0] >> sh) & 63) << (0 if nu else 4)
                s1 = ((s["SC"][1] >> sh) & 63) << (0 if nu else 4)
                for i, sv in ((0, s0), (1, s0), (2, s1), (3, s1)):
                    s["T"][i] += sv * D[lane][i]
                j = 2 * pi + 4 * (t >> 1) + nu
                xj = F32(xs[2 * j] + xs[2 * j + 1])
                s["M"][0] = F32(s["M"][0] + F32((s["MN"][0] >> sh) & 63) * xj)
                s["M"][1] = F32(s["M"][1] + F32((s["MN"][1] >> sh) & 63) * xj)
    for lane in range(32):
        t = lane & 3
        s = st[lane]
        assert all(abs(v) < 2 ** 31 for v in s["T"])
        odd = t & 1
        u0 = F32(1 / (16384 * 16)) if odd else F32(1 / 16)
        u1 = F32(0) if odd else F32(1 / (128 * 16))
        mo = F32(0) if odd else F32(1)
        res = []
        for r, (ta, tb) in enumerate(((0, 1), (2, 3))):
            d, dm = h2f(s["H"][r][0] & 0xFFFF), h2f(s["H"][r][0] >> 16)
            res.append(F32(d * F32(F32(F32(s["T"][ta]) * u0) + F32(F32(s["T"][tb]) * u1)) - dm * F32(mo * s["M"][r])))
        o.append(res)
    return rows_of(o)


def q6k_task8(win, offs, area, xs):
    """win: 16 slot rows (240 bytes each) holding 224-byte windows; offs: the
    block's even offset in each window."""
    o = []
    for lane in range(32):
        o.append(None)
    st = []
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        r0, r1 = 240 * g + offs[g], 240 * (g + 8) + offs[g + 8]
        st.append(dict(r=(r0, r1), S=(ld16_u2(win, r0 + 192), ld16_u2(win, r1 + 192)), T=[0, 0, 0, 0],
                       F=[F32(0), F32(0)]))
    for q in range(2):
        lanes = []
        for lane in range(32):
            t = lane & 3
            r0, r1 = st[lane]["r"]
            l0, h0 = ld8_u2(win, r0 + 64 * q + 8 * t), ld8_u2(win, r0 + 64 * q + 32 + 8 * t)
            l1, h1 = ld8_u2(win, r1 + 64 * q + 8 * t), ld8_u2(win, r1 + 64 * q + 32 + 8 * t)
            b0, b1 = ld8_u2(win, r0 + 128 + 32 * q + 8 * t), ld8_u2(win, r1 + 128 + 32 * q + 8 * t)
            m02 = [b0[0] & 0x33333333, b0[1] & 0x33333333, b1[0] & 0x33333333, b1[1] & 0x33333333]
            m13 = [b0[0] & 0xCCCCCCCC, b0[1] & 0xCCCCCCCC, b1[0] & 0xCCCCCCCC, b1[1] & 0xCCCCCCCC]
            lanes.append((l0, h0, l1, h1, m02, m13))

        def quant(c, ql_lo, ql_hi, a02, a13):
            low = 0x0F0F0F0F
            if c == 0:
                return (ql_lo & low) | ((a02 << 4) & 0xF0F0F0F0)
            if c == 1:
                return (ql_hi & low) | ((a13 << 2) & 0xF0F0F0F0)
            if c == 2:
                return ((ql_lo >> 4) & low) | (a02 & 0xF0F0F0F0)
            return ((ql_hi >> 4) & low) | ((a13 >> 2) & 0xF0F0F0F0)

        for c in range(4):
            regs = []
            for lane in range(32):
                l0, h0, l1, h1, m02, m13 = lanes[lane]
                xp = bsel(lane, True) + 512 * q + 128 * c
                regs.append((quant(c, l0[0], h0[0], m02[0], m13[0]) & 0xFFFFFFFF,
                             quant(c, l1[0], h1[0], m02[2], m13[2]) & 0xFFFFFFFF,
                             quant(c, l0[1], h0[1], m02[1], m13[1]) & 0xFFFFFFFF,
                             quant(c, l1[1], h1[1], m02[3], m13[3]) & 0xFFFFFFFF,
                             u32(area, xp), u32(area, xp + 4)))
            D = mma(regs)
            for lane in range(32):
                t = lane & 3
                s = st[lane]
                sel = sx_sel(2 + (t >> 1)) if c & 1 else sx_sel(t >> 1)
                s0 = s32(prmt_sx(s["S"][0][2 * q + (c >> 1)], sel))
                s1 = s32(prmt_sx(s["S"][1][2 * q + (c >> 1)], sel))
                for i, sv in ((0, s0), (1, s0), (2, s1), (3, s1)):
                    s["T"][i] += sv * D[lane][i]
                xg = xs[8 * q + 2 * c + (t >> 1)]
                s["F"][0] = F32(s["F"][0] + F32(s0) * xg)
                s["F"][1] = F32(s["F"][1] + F32(s1) * xg)
    for lane in range(32):
        t = lane & 3
        s = st[lane]
        assert all(abs(v) < 2 ** 31 for v in s["T"])
        odd = t & 1
        u0 = F32(1 / 16384) if odd else F32(1)
        u1 = F32(0) if odd else F32(1 / 128)
        fo = F32(0) if odd else F32(32)
        res = []
        for r, (ta, tb) in enumerate(((0, 1), (2, 3))):
            d = h2f(int(win[s["r"][r] + 208]) | int(win[s["r"][r] + 209]) << 8)
            res.append(F32(d * F32(F32(F32(s["T"][ta]) * u0) + F32(F32(s["T"][tb]) * u1) - F32(fo * s["F"][r]))))
        o[lane] = res
    return rows_of(o)


# ------------------------------------------------------------------ tests ----

def _x(rng, kind):
    if kind == "normal":
        return rng.standard_normal(256).astype(F32)
    if kind == "outlier":
        x = rng.standard_normal(256).astype(F32) * F32(1e-3)
        x[rng.integers(256)] = F32(37.5)
        return x
    if kind == "tiny":
        return (rng.standard_normal(256) * 1e-30).astype(F32)
    if kind == "half":   # many exact half-integers after scaling
        return (rng.integers(-254, 255, 256) / 2.0).astype(F32)
    return np.zeros(256, F32)


def _check(y, w, x, isb):
    want = w.astype(np.float64) @ x.astype(np.float64)
    got = y.astype(np.float64) * np.float64(isb)
    bound = 1e-6 * np.abs(x).max() * np.abs(w).sum(axis=1) + 1e-6 * np.abs(w * x).sum(axis=1) + 1e-30
    assert (np.abs(got - want) <= bound).all(), (np.abs(got - want) / bound).max()


@pytest.mark.parametrize("kind", ["normal", "outlier", "tiny", "half", "zero"])
def test_q4k_task8_matches_dequantized_rows(oracle, kind):
    rng = np.random.default_rng(hash(kind) % 1000)
    for src in ("synth", "random"):
        blocks = (atlas_cuda.synth_blocks(atlas_cuda.TYPE_Q4_K, 16, seed=5) if src == "synth"
                  else rng.integers(0, 256, 16 * 144).astype(np.uint8))
        if src == "random":   # finite scales: d, dmin as small positive fp16
            v = blocks.reshape(16, 144)
            v[:, 0:4] = np.frombuffer(rng.uniform(1e-4, 2e-3, 32).astype(np.float16).tobytes(), np.uint8).reshape(16, 4)
        w = oracle.dequant(atlas_cuda.TYPE_Q4_K, blocks, 16, 256).reshape(16, 256)
        x = _x(rng, kind)
        area, xs, isb = stage_block(x)
        y = q4k_task8([blocks[144 * r:144 * r + 144] for r in range(16)], area, xs)
        _check(y, w, x, isb)


@pytest.mark.parametrize("kind", ["normal", "outlier", "tiny", "half", "zero"])
def test_q6k_task8_matches_dequantized_rows(oracle, kind):
    rng = np.random.default_rng(7 + hash(kind) % 1000)
    for src in ("synth", "random"):
        blocks = (atlas_cuda.synth_blocks(atlas_cuda.TYPE_Q6_K, 16, seed=9) if src == "synth"
                  else rng.integers(0, 256, 16 * 210).astype(np.uint8))
        if src == "random":
            v = blocks.reshape(16, 210)
            v[:, 208:210] = np.frombuffer(rng.uniform(1e-4, 2e-3, 16).astype(np.float16).tobytes(), np.uint8).reshape(16, 2)
        w = oracle.dequant(atlas_cuda.TYPE_Q6_K, blocks, 16, 256).reshape(16, 256)
        x = _x(rng, kind)
        area, xs, isb = stage_block(x)
        win = np.zeros(16 * 240, np.uint8)
        offs = [2 * int(rng.integers(0, 8)) for _ in range(16)]   # every even offset the 224-byte window allows
        offs[0], offs[1] = 0, 14
        for r in range(16):
            win[240 * r + offs[r]:240 * r + offs[r] + 210] = blocks[210 * r:210 * r + 210]
        y = q6k_task8(win, offs, area, xs)
        _check(y, w, x, isb)


def test_q6k_task8_reads_stay_inside_the_window():
    # farthest reads: the scales' 5 aligned words and the qh runs' 3 words, at the largest offset
    for off in range(0, 16, 2):
        r = off
        assert (r + 192) // 4 * 4 + 20 <= 224
        assert (r + 128 + 32 + 24) // 4 * 4 + 12 <= 224
        assert (r + 64 + 32 + 24) // 4 * 4 + 12 <= 224


def test_b_operand_loads_conflict_free_per_half_warp():
    for q6, offsets in ((True, [512 * q + 128 * c for q in range(2) for c in range(4)]),
                        (False, [256 * p + 128 * n + 32 * h for p in range(2) for n in range(2) for h in range(2)])):
        for off in offsets:
            for half in range(2):
                seen = {}
                for lane in range(16 * half, 16 * half + 16):
                    a = bsel(lane, q6) + off
                    assert a % 8 == 0 and a + 8 <= 1024
                    for bank in ((a // 4) % 32, (a // 4 + 1) % 32):
                        assert seen.setdefault(bank, a) == a, (q6, off, lane)


def test_b_operand_holds_each_group_once():
    # every (column, k slot) of B is read by exactly the lane that the fragment layout names,
    # and nonzero planes reach only the k slots of the column's own group
    for q6 in (True, False):
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            pl = (bsel(lane, q6) % 32) // 8
            assert (pl < 3) == ((g >> 2) == (t >> 1) and (g & 3) < 3)


def q4_slot_row(m):
    """q4_slot_row (csrc/decode2.cu)."""
    return m ^ 3 if (m + 1) & 2 else m


def test_q4k_quant_loads_conflict_free_per_quarter_warp():
    # slot rows 144 bytes apart; lane (g, t) loads 16 bytes at 16 + 64 (t >> 1) + 16 (t & 1) + 32 pi of
    # rows g and g + 8; a 16-byte load is served a quarter warp at a time
    assert sorted(q4_slot_row(m) for m in range(16)) == list(range(16))
    for pi in range(2):
        for rbase in (0, 8):
            for quarter in range(4):
                groups = set()
                for lane in range(8 * quarter, 8 * quarter + 8):
                    g, t = lane >> 2, lane & 3
                    a = 144 * q4_slot_row(g + rbase) + 16 + 64 * (t >> 1) + 16 * (t & 1) + 32 * pi
                    groups.add((a // 16) % 8)
                assert len(groups) == 8, (pi, rbase, quarter)
        # the header loads: one row per lane group of 4, two rows per quarter warp
        for quarter in range(4):
            assert len({(144 * q4_slot_row(g)) // 16 % 8 for g in (2 * quarter, 2 * quarter + 1)}) == 2


def test_q6k_copy_table_encoding():
    # slot offset in the low 16 bits, the chunk's offset inside the window in the high 16 bits
    for idx in range(224):
        r, p = idx // 14, idx % 14
        y = (r * 240 + 16 * p) | (16 * p) << 16
        assert y & 0xFFFF == r * 240 + 16 * p and y >> 16 == 16 * p


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_nonfinite_input_gives_nan_rows(oracle, bad):
    # the staged factor of a block holding NaN or inf is NaN: every row sum over it is NaN
    rng = np.random.default_rng(3)
    x = rng.standard_normal(256).astype(F32)
    x[77] = F32(bad)
    area, xs, isb = stage_block(x)
    assert np.isnan(isb)
    blocks = atlas_cuda.synth_blocks(atlas_cuda.TYPE_Q4_K, 16, seed=5)
    with np.errstate(invalid="ignore", over="ignore"):
        y = q4k_task8([blocks[144 * r:144 * r + 144] for r in range(16)], area, xs).astype(np.float64) * isb
    assert np.isnan(y).all()
    # and a finite block's factor is the plain 1 / 2^k
    assert np.isfinite(stage_block(rng.standard_normal(256))[2])
