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
