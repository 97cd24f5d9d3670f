"""CPU emulation of the integer tensor-core operand layouts of the decode
GEMV kernels (go-infer_b200/csrc/gemv.cu): the int32 products the MMAs form
and the way the kernels combine them reproduce the exact block dot products.

* Activations: four balanced base-256 limbs of round(x * 2^e) per 256
  columns, limb bytes = (v + 0x80808080) ^ 0x80808080.
* Q4_K (two MMAs per 64-column chunk): B carries the low nibbles'
  sub-block limbs in columns 0-3 and the high nibbles' in columns 4-7; MMA
  L takes the masked low nibbles, MMA F the whole bytes; columns 0-3 of L
  and columns 4-7 of (F - L) / 16 are the two sub-blocks' limb dots.
* Q8_0 (one MMA per block): the block's 32 quants are read as eight aligned
  words in a block-dependent order (odd blocks natural, even blocks quants
  2..29 then 0, 1, 30, 31); the staged activation uses the same order.
"""
import numpy as np


def limbs_of(x, e):
    v = np.rint(x.astype(np.float64) * 2.0 ** e).astype(np.int64) & 0xFFFFFFFF
    u = ((v + 0x80808080) & 0xFFFFFFFF) ^ 0x80808080
    out = np.zeros((4, x.size), np.int64)
    for n in range(4):
        b = (u >> (8 * (3 - n))) & 0xFF
        out[n] = np.where(b >= 128, b - 256, b)
    return out


def exponent(x):
    m = float(np.abs(x).max())
    return 29 - int(np.floor(np.log2(m))) if m > 0 else 0


def test_limbs_are_exact_fixed_point():
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, 256).astype(np.float32)
    e = exponent(x)
    L = limbs_of(x, e)
    assert np.all(np.abs(L) <= 128)
    X = sum(L[n] * 256 ** (3 - n) for n in range(4))
    assert np.all(X == np.rint(x.astype(np.float64) * 2.0 ** e))


def test_q4k_two_mma_column_layout():
    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, 256).astype(np.float32)
    e = exponent(x)
    L = limbs_of(x, e)
    for _ in range(20):
        packed = rng.integers(0, 256, (16, 4, 32), dtype=np.int64)  # [row][chunk c][byte l]
        sc = rng.integers(0, 64, (16, 8), dtype=np.int64)          # 6-bit sub-block scales
        lo, hi = packed & 0x0F, packed >> 4
        acc = np.zeros(16, np.float64)
        for c in range(4):
            xl, xh = L[:, 64 * c:64 * c + 32], L[:, 64 * c + 32:64 * c + 64]  # sub-blocks 2c, 2c+1
            B = np.concatenate([xl.T, xh.T], axis=1)  # [k][8 columns]
            Dl = lo[:, c, :] @ B        # MMA L: masked low nibbles
            Df = packed[:, c, :] @ B    # MMA F: whole bytes q_lo + 16 q_hi
            assert np.abs(Df).max() < 2 ** 31
            low = Dl[:, 0:4]
            high16 = (Df - Dl)[:, 4:8]
            assert np.array_equal(low, lo[:, c, :] @ xl.T)
            assert np.array_equal(high16, 16 * (hi[:, c, :] @ xh.T))
            w = np.array([256.0 ** (3 - n) for n in range(4)])
            acc += sc[:, 2 * c] * (low @ w) + sc[:, 2 * c + 1] * (high16 @ w) / 16
        want = np.zeros(16, np.float64)
        X = sum(L[n] * 256 ** (3 - n) for n in range(4)).astype(np.float64)
        for c in range(4):
            want += sc[:, 2 * c] * (lo[:, c, :] @ X[64 * c:64 * c + 32])
            want += sc[:, 2 * c + 1] * (hi[:, c, :] @ X[64 * c + 32:64 * c + 64])
        assert np.array_equal(acc, want)


def kslot(b, i, j):
    """Element of Q8_0 block b carried by byte j of slot word i."""
    if b % 2 == 1:
        return 4 * i + j
    if i < 7:
        return 2 + 4 * i + j
    return (0, 1, 30, 31)[j]


def slot_word(row, b, i):
    """Slot word i of block b of a 272-byte row unit, from aligned loads."""
    o = 34 * b + 2
    if b % 2 == 1:
        assert o % 4 == 0
        return row[o + 4 * i:o + 4 * i + 4]
    base = o - 2
    assert base % 4 == 0
    if i < 7:
        return row[base + 4 * (i + 1):base + 4 * (i + 2)]
    u0, u8 = row[base:base + 4], row[base + 32:base + 36]
    return np.array([u0[2], u0[3], u8[0], u8[1]], np.uint8)  # prmt(u0, u8, 0x5432)


def test_q8_0_slot_order_is_a_permutation_of_each_block():
    for b in range(8):
        ks = sorted(kslot(b, i, j) for i in range(8) for j in range(4))
        assert ks == list(range(32))


def test_q8_0_aligned_words_give_exact_block_dots():
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, 256).astype(np.float32)
    e = exponent(x)
    L = limbs_of(x, e)
    for _ in range(10):
        unit = rng.integers(0, 256, (16, 272), dtype=np.uint8)  # 16 rows x 8 blocks of 34 bytes
        for r in range(16):
            for b in range(8):
                q = unit[r, 34 * b + 2:34 * b + 34].view(np.int8).astype(np.int64)
                D = np.zeros(4, np.int64)
                for i in range(8):
                    w = slot_word(unit[r], b, i).view(np.int8).astype(np.int64)
                    for j in range(4):
                        k = kslot(b, i, j)
                        assert w[j] == q[k]
                        D += w[j] * L[:, 32 * b + k]
                v01, v23 = D[0] * 256 + D[1], D[2] * 256 + D[3]  # lanes 0 and 1, exact in int32
                assert max(abs(v01), abs(v23)) < 2 ** 31
                X = sum(L[n, 32 * b:32 * b + 32] * 256 ** (3 - n) for n in range(4))
                assert v01 * 65536 + v23 == int(q @ X)


def test_q4k_stage_swizzle_and_ldmatrix_fragments():
    """The Q4_K kernel's stage as its cp.async requests fill it (16-byte
    piece q of row r at slot q ^ (r & 7)), read back by ldmatrix.x4 at each
    lane's lofs ^ 32c, against activations staged in B-fragment k order: the
    two MMAs per chunk give the exact sub-block limb dots, every address is a
    16-byte-aligned offset inside the 2304-byte stage, and each ldmatrix
    phase (eight rows of one matrix) touches eight distinct bank groups."""
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 256).astype(np.float32)
    e = exponent(x)
    L = limbs_of(x, e)
    # staged activations: stage_x / stage_unit, lane (j, q) -> positions 8q..8q+7
    xs = np.zeros((8, 4, 32), np.int64)  # [sub-block j][limb n][position]
    for lane in range(32):
        j, q = lane >> 2, lane & 3
        offA = 64 * (j >> 1) + 32 * (j & 1) + 4 * q
        offB = offA + 16
        for n in range(4):
            xs[j, n, 8 * q:8 * q + 4] = L[n, offA:offA + 4]
            xs[j, n, 8 * q + 4:8 * q + 8] = L[n, offB:offB + 4]
    xflat = xs.reshape(-1)
    for _ in range(5):
        unit = rng.integers(0, 256, (16, 144), dtype=np.int64)  # 16 rows of one Q4_K super-block
        stage = np.full(2304, -1, np.int64)
        for lane in range(32):  # request(): the cp.async destinations
            g, t = lane >> 2, lane & 3
            dst0 = g * 128 + 16 * ((2 * t) ^ g)
            dst1 = g * 128 + 16 * ((2 * t + 1) ^ g)
            for d, row, src in ((dst0, g, 16 + 32 * t), (dst1, g, 32 + 32 * t),
                                (dst0 + 1024, g + 8, 16 + 32 * t), (dst1 + 1024, g + 8, 32 + 32 * t)):
                assert d % 16 == 0 and 0 <= d and d + 16 <= 2048
                stage[d:d + 16] = unit[row, src:src + 16]
            if t < 2:
                dh = 2048 + (g + 8 * (t & 1)) * 16
                stage[dh:dh + 16] = unit[g + 8 * t, 0:16]
        assert (stage >= 0).all()
        for c in range(4):
            # ldmatrix.x4: lanes 8i..8i+7 give the rows of matrix i
            addr = []
            for lane in range(32):
                lrow = (lane & 7) + 8 * ((lane >> 3) & 1)
                lofs = lrow * 128 + 16 * ((lane >> 4) ^ (lrow & 7))
                a = lofs ^ (32 * c)
                assert a % 16 == 0 and 0 <= a and a + 16 <= 2048
                addr.append(a)
            for i in range(4):
                banks = {(addr[8 * i + r] % 128) // 16 for r in range(8)}
                assert len(banks) == 8
            A = np.zeros((16, 32), np.int64)
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                for i in range(4):
                    row16 = stage[addr[8 * i + g]:addr[8 * i + g] + 16]
                    word = row16[4 * t:4 * t + 4]                 # register i of this lane
                    r = g + (8 if i in (1, 3) else 0)              # a0, a2: row g; a1, a3: row g + 8
                    k0 = 4 * t + (16 if i >= 2 else 0)             # a0, a1: k 4t..; a2, a3: k 16+4t..
                    A[r, k0:k0 + 4] = word
            assert np.array_equal(A, unit[:, 16 + 32 * c:16 + 32 * c + 32])  # qs bytes of chunk c
            B = np.zeros((32, 8), np.int64)
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                xl = (g & 3) * 32 + 8 * t + (128 if g >= 4 else 0) + 256 * c
                v = xflat[xl:xl + 8]
                B[4 * t:4 * t + 4, g] = v[:4]        # b0: k 4t..4t+3, column g
                B[16 + 4 * t:20 + 4 * t, g] = v[4:]  # b1: k 16+4t..
            lo, whole = A & 0x0F, A
            Dl, Df = lo @ B, whole @ B
            xlo = L[:, 64 * c:64 * c + 32]
            xhi = L[:, 64 * c + 32:64 * c + 64]
            assert np.array_equal(Dl[:, 0:4], lo @ xlo.T)
            assert np.array_equal((Df - Dl)[:, 4:8], 16 * ((A >> 4) @ xhi.T))


# ---- Q6_K on the int8 tensor cores (gemv.cu, namespace q6m) ----------------

def q6m_ldw(slot, a):
    """ldw<Odd>: the word at byte a of a row slot (a even); a % 4 == 2 reads
    the aligned words at a - 2 and a + 2 and joins them (funnel shift 16)."""
    def word(o):
        assert o % 4 == 0 and 0 <= o and o + 4 <= slot.size
        return int.from_bytes(bytes(slot[o:o + 4].astype(np.uint8)), "little")
    if a % 4 == 0:
        return word(a)
    assert a % 4 == 2
    return ((word(a - 2) >> 16) | (word(a + 2) << 16)) & 0xFFFFFFFF


def q6m_stage_x(L):
    """stage_unit: [chunk][limb][32 bytes, element order] and, per chunk and
    lane t, the pair (-32 x limb sum) of columns 2t, 2t+1."""
    xs = np.zeros((8, 4, 32), np.int64)
    cs = np.zeros((8, 4, 2), np.int64)
    for c in range(8):
        e0 = 128 * (c >> 2) + 32 * (c & 3)
        xs[c] = L[:, e0:e0 + 32]
        sa = L[:, e0:e0 + 16].sum(axis=1)
        sb = L[:, e0 + 16:e0 + 32].sum(axis=1)
        for t in range(4):
            src = sa if t < 2 else sb
            n0 = 2 * (t & 1)
            cs[c, t] = (-32 * src[n0], -32 * src[n0 + 1])
    return xs, cs


def test_q6k_mma_fragments_give_exact_sub_block_dots():
    """The Q6_K tensor-core kernel's unit as its cp.async requests stage it
    (the 14 aligned chunks that cover each row's block, the block at byte
    (2b) % 16 of a 224-byte slot), its A fragments built from (funnel-shifted)
    ql / qh words, B from the staged limbs, the accumulator started at -32 x
    the limb sums and the per-lane int8 scales: the lanes' integer sums give
    sum_sub-blocks sc * sum (q - 32) * X exactly, with q as the oracle's
    DequantizeQ6_K decodes it (quant.go:256-291), for both block parities."""
    import oracle as O
    rng = np.random.default_rng(6)
    x = rng.normal(0, 1, 256).astype(np.float32)
    e = exponent(x)
    L = limbs_of(x, e)
    X = sum(L[n] * 256 ** (3 - n) for n in range(4))
    xs, cs = q6m_stage_x(L)
    for b in range(16):  # column block: the parity and the offset in the slot
        s = (2 * b) % 16
        blocks = rng.integers(0, 256, (16, 210), dtype=np.int64)
        blocks[:, 208:210] = (0x00, 0x3C)  # d = 1.0: the oracle then gives sc * (q - 32)
        slots = rng.integers(0, 256, (16, 224), dtype=np.int64)  # bytes around the block: garbage
        slots[:, s:s + 210] = blocks
        # the oracle's decode of each row: integer sc * (q - 32)
        want_w = np.stack([O.dequantize(O.GGML_Q6_K, blocks[r].astype(np.uint8), 256) for r in range(16)])
        assert np.array_equal(want_w, np.rint(want_w))
        want = want_w.astype(np.int64) @ X
        got = np.zeros(16, np.int64)
        # per lane: its words, fragments and accumulators
        lanes = {}
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            rows = (g, g + 8)
            w = {}
            for r in rows:
                sl = slots[r]
                for n in range(2):
                    for name, off in (("L0", 64 * n), ("L1", 64 * n + 32), ("Q", 128 + 32 * n)):
                        w[r, n, name, 0] = q6m_ldw(sl, s + off + 4 * t)
                        w[r, n, name, 1] = q6m_ldw(sl, s + off + 16 + 4 * t)
                w[r, "sc"] = [q6m_ldw(sl, s + 192 + 4 * i) for i in range(4)]
            lanes[lane] = w
        acc = {lane: [0, 0, 0, 0] for lane in range(32)}
        for n in range(2):
            for j in range(4):
                c = 4 * n + j
                A = np.zeros((16, 32), np.int64)
                B = np.zeros((32, 8), np.int64)
                for lane in range(32):
                    g, t = lane >> 2, lane & 3
                    w = lanes[lane]
                    for reg, (r, half) in enumerate(((g, 0), (g + 8, 0), (g, 1), (g + 8, 1))):
                        Lw = w[r, n, "L1" if j & 1 else "L0", half]
                        Qw = w[r, n, "Q", half]
                        lo = (Lw >> 4) & 0x0F0F0F0F if j >> 1 else Lw & 0x0F0F0F0F
                        a = lo | (((Qw >> (2 * j)) << 4) & 0x30303030)
                        k0 = 4 * t + 16 * half
                        A[r, k0:k0 + 4] = [(a >> (8 * i)) & 0xFF for i in range(4)]
                    xw = xs[c, g & 3, (0 if g < 4 else 16) + 4 * t:(0 if g < 4 else 16) + 4 * t + 4]
                    if g < 4:
                        B[4 * t:4 * t + 4, g] = xw      # b0
                    else:
                        B[16 + 4 * t:20 + 4 * t, g] = xw  # b1
                assert A.max() < 64 and A.min() >= 0
                C = np.zeros((16, 8), np.int64)
                for lane in range(32):
                    g, t = lane >> 2, lane & 3
                    C[g, 2 * t:2 * t + 2] = cs[c, t]
                    C[g + 8, 2 * t:2 * t + 2] = cs[c, t]
                D = A @ B + C
                assert np.abs(D).max() < 2 ** 31
                for lane in range(32):
                    g, t = lane >> 2, lane & 3
                    sbk = 2 * j + (1 if t >= 2 else 0)
                    for idx, r in ((0, g), (2, g + 8)):
                        word = lanes[lane][r, "sc"][2 * n + (sbk >> 2)]
                        byte = (word >> (8 * (sbk & 3))) & 0xFF
                        sc = byte - 256 if byte >= 128 else byte
                        acc[lane][idx] += int(D[r, 2 * t]) * sc
                        acc[lane][idx + 1] += int(D[r, 2 * t + 1]) * sc
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            W0, W1 = (256, 1) if t & 1 else (2 ** 24, 2 ** 16)
            assert max(abs(v) for v in acc[lane]) < 2 ** 31
            got[g] += acc[lane][0] * W0 + acc[lane][1] * W1
            got[g + 8] += acc[lane][2] * W0 + acc[lane][3] * W1
        assert np.array_equal(got, want), b


def test_q6k_mma_request_covers_each_block():
    """The cursor's source offsets: row start + ((210 b) & ~15) + 16 i for the
    14 chunks covers block b and ends inside the row when the row holds whole
    2048-column groups (the last block ends exactly at the row's end)."""
    for nsb in (8, 16, 32, 112):
        rowb = 210 * nsb
        assert rowb % 16 == 0
        for b in range(nsb):
            start = (210 * b) & ~15
            assert start <= 210 * b and start + 224 >= 210 * b + 210
            assert start + 224 <= rowb
            assert (210 * b) - start == (2 * b) % 16
