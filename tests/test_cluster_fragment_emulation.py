"""Lane-level emulation of the cluster-split decode GEMV's consumer (``csrc/gemv_cluster.cu``).

Builds the shared-memory bytes of a warp's 128-row block the way the tensor-memory-access (TMA)
copies leave them -- the packed weights of a 256-column box as [rows][128 bytes] with the 128-byte
swizzle (16-byte chunk c of row r stored at chunk c ^ (r % 8)), the warp's 64-column strip being
chunks 2 (strip % 4) and +1 of each row, x token-interleaved as [8 pairs of 16 k][M tokens][16 values]
with the 32-byte swizzle (the two chunks of a 32-byte row swapped on rows 4-7 of every 8) -- and replays
what each of the warp's 32 lanes does: the ldmatrix row addresses, the ldmatrix / ldmatrix.trans
register distribution of the PTX ISA (thread i of an 8x8 b16 matrix gets row i/4, columns
2(i%4), 2(i%4)+1; transposed: rows 2(i%4), 2(i%4)+1 of column i/4), the nibble masks that turn
a register into (1024 + q) / (1024 + 16 q) pairs, the m16n8k16 fragment layouts, the ones-mma
for the group's sum of x, and the per-group correction with the lane's scale and zero constants.
The per-lane accumulators are mapped back to output columns exactly as the kernel's ``deposit``
does and compared with the oracle's fp64 product. A planted error (wrong swizzle, wrong nibble
order) must fail.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import awq_oracle as O

ROWS = 128          # k rows of a warp's block per stage
WORDS = 8           # packed words per strip row (64 columns)
BOX_WORDS = 32      # packed words per 128-byte box row (4 strips)
KLO, KHI, MAGIC = 0x000F000F, 0x00F000F0, 0x64006400


def h2f(u16: int) -> float:
    return float(np.array([u16 & 0xFFFF], dtype=np.uint16).view(np.float16)[0])


def halves(u32: int):
    return h2f(u32 & 0xFFFF), h2f(u32 >> 16)


def swz32(off: int) -> int:
    """32-byte TMA swizzle of a byte offset inside a 256-byte-aligned region."""
    return off ^ (((off >> 7) & 1) << 4)


def swz128(off: int) -> int:
    """128-byte TMA swizzle of a byte offset inside a 1024-byte-aligned region."""
    return off ^ (((off >> 7) & 7) << 4)


class Stage:
    def __init__(self, words, x_bits, M, strip=1, swizzle=True):
        self.M = M
        self.strip = strip  # the warp's strip: words 8 (strip % 4) .. of each 128-byte box row
        self.w = bytearray(ROWS * 128)
        for r in range(ROWS):
            for c in range(WORDS):
                off = r * 128 + 4 * (WORDS * (strip % 4) + c)
                dst = swz128(off) if swizzle else off
                self.w[dst:dst + 4] = int(words[r, c]).to_bytes(4, "little")
        # x: [8 pairs][M][16 halves]
        self.x = bytearray(8 * M * 32)
        for p in range(8):
            for m in range(M):
                for i in range(16):
                    off = (p * M + m) * 32 + 2 * i
                    dst = swz32(off) if swizzle else off
                    self.x[dst:dst + 2] = int(x_bits[m, 16 * p + i]).to_bytes(2, "little")

    def row16(self, buf, addr):
        """8 b16 elements of the 16-byte row at addr."""
        return [int.from_bytes(buf[addr + 2 * e: addr + 2 * e + 2], "little") for e in range(8)]


def ldsm_x4(rows_per_matrix, trans):
    """rows_per_matrix[q][r] = 8 b16 values; returns regs[lane][q] (32-bit)."""
    regs = [[0] * 4 for _ in range(32)]
    for lane in range(32):
        for q in range(4):
            mat = rows_per_matrix[q]
            if trans:
                lo, hi = mat[2 * (lane % 4)][lane // 4], mat[2 * (lane % 4) + 1][lane // 4]
            else:
                lo, hi = mat[lane // 4][2 * (lane % 4)], mat[lane // 4][2 * (lane % 4) + 1]
            regs[lane][q] = lo | (hi << 16)
    return regs


def emulate_strip(words, qz_row_words, scales, x, G, nibble_shift_bug=False, swizzle_reads=True):
    """One warp consuming every stage of one strip; returns y [M][64] (fp64 accumulation)."""
    K = words.shape[0]
    M = x.shape[0]
    x_bits = x.astype(np.float16).view(np.uint16)
    acc = np.zeros((32, 4, 4))      # lane, j, d-register (MT = 1 or 2 handled by token tiles below)
    MT = 2 if M > 8 else 1
    acc = np.zeros((MT, 32, 4, 4))
    for k0 in range(0, K, ROWS):
        st = Stage(words[k0:k0 + ROWS], x_bits[:, k0:k0 + ROWS], M, swizzle=True)
        steps = min(ROWS, K - k0) // 16
        part = np.zeros((MT, 32, 4, 4))
        psx = np.zeros((MT, 32, 4))
        cur_grp = -1
        for s in range(steps):
            k = k0 + 16 * s
            if k // G != cur_grp:
                if cur_grp >= 0:
                    acc += flush(part, psx, consts, M)
                    part[:] = 0
                    psx[:] = 0
                cur_grp = k // G
                consts = lane_consts(qz_row_words[cur_grp], scales[cur_grp])
            # weights: matrix q rows = k rows 8(q//2)+r, chunk 2 (strip % 4) + q%2 of the 128-byte row
            mats = []
            for q in range(4):
                rows = []
                for r in range(8):
                    krow = 16 * s + 8 * (q >> 1) + r
                    chunk = 2 * (st.strip % 4) + (q & 1)
                    lane_off = krow * 128 + 16 * ((chunk ^ r) if swizzle_reads else chunk)
                    rows.append(st.row16(st.w, lane_off))
                mats.append(rows)
            R = ldsm_x4(mats, trans=True)
            # x: matrix q = pair s + ... only pair s here (half q % 2); token rows
            for mt in range(MT):
                xm = []
                for q in range(2):
                    rows = []
                    for r in range(8):
                        tok = 8 * mt + r
                        tok = tok if tok < M else 0
                        row = s * M + tok
                        addr = row * 32 + 16 * (q ^ ((row >> 2) & 1))
                        rows.append(st.row16(st.x, addr))
                    xm.append(rows)
                xm += xm  # registers 2, 3 unused in this emulation
                Bx = ldsm_x4(xm, trans=False)
                for j in range(4):
                    A = np.zeros((16, 16))
                    B = np.zeros((16, 8))
                    for lane in range(32):
                        g, t = lane >> 2, lane & 3
                        for i in range(4):
                            v = R[lane][i] >> (8 if j >= 2 else 0)
                            if nibble_shift_bug and j == 1:
                                v = R[lane][i] >> 4
                            bits = (v & (KHI if j & 1 else KLO)) | MAGIC
                            lo, hi = halves(bits)
                            row = g + 8 * (i & 1)
                            kc = 2 * t + 8 * (i >> 1)
                            A[row, kc], A[row, kc + 1] = lo, hi
                        b0, b1 = Bx[lane][0], Bx[lane][1]
                        B[2 * t, g], B[2 * t + 1, g] = halves(b0)
                        B[2 * t + 8, g], B[2 * t + 9, g] = halves(b1)
                    D = A @ B
                    ones = np.ones((16, 16)) @ B
                    for lane in range(32):
                        g, t = lane >> 2, lane & 3
                        part[mt, lane, j] += [D[g, 2 * t], D[g, 2 * t + 1], D[g + 8, 2 * t], D[g + 8, 2 * t + 1]]
                        if j == 0:
                            psx[mt, lane] += [ones[g, 2 * t], ones[g, 2 * t + 1], ones[g + 8, 2 * t],
                                              ones[g + 8, 2 * t + 1]]
        acc += flush(part, psx, consts, M)
    # deposit
    y = np.zeros((M, 64))
    for mt in range(MT):
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            wA, hA = g >> 1, g & 1
            for j in range(4):
                cA = 8 * wA + 2 * j + hA
                for d, (m, c) in enumerate([(8 * mt + 2 * t, cA), (8 * mt + 2 * t + 1, cA),
                                            (8 * mt + 2 * t, cA + 32), (8 * mt + 2 * t + 1, cA + 32)]):
                    if m < M:
                        y[m, c] = acc[mt, lane, j, d]
    return y


def lane_consts(zwords, srow):
    """ca, cb [32 lanes][8]: A-rows g (0..3) and g + 8 (4..7) per nibble j."""
    ca = np.zeros((32, 8))
    cb = np.zeros((32, 8))
    for lane in range(32):
        g = lane >> 2
        wA, hA = g >> 1, g & 1
        for j in range(4):
            f, c = (1.0 / 16, 64.0) if j & 1 else (1.0, 1024.0)
            for half, w in ((0, wA), (1, 4 + wA)):
                col = 8 * w + 2 * j + hA
                s = float(srow[col])
                z = (int(zwords[w]) >> (16 * hA + 4 * j)) & 15
                ca[lane, 4 * half + j] = s * f
                cb[lane, 4 * half + j] = -s * (c + z)
    return ca, cb


def flush(part, psx, consts, M):
    ca, cb = consts
    out = np.zeros_like(part)
    for j in range(4):
        out[:, :, j, 0] = ca[None, :, j] * part[:, :, j, 0] + cb[None, :, j] * psx[:, :, 0]
        out[:, :, j, 1] = ca[None, :, j] * part[:, :, j, 1] + cb[None, :, j] * psx[:, :, 1]
        out[:, :, j, 2] = ca[None, :, 4 + j] * part[:, :, j, 2] + cb[None, :, 4 + j] * psx[:, :, 0]
        out[:, :, j, 3] = ca[None, :, 4 + j] * part[:, :, j, 3] + cb[None, :, 4 + j] * psx[:, :, 1]
    return out


def strip_problem(M, K, G, seed):
    rng = np.random.default_rng(seed)
    qw = rng.integers(0, 2 ** 32, size=(K, 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    qz = rng.integers(0, 2 ** 32, size=(K // G, 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    s = rng.uniform(0.002, 0.02, size=(K // G, 64)).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float16)
    return x, qw, qz, s


@pytest.mark.parametrize("M,K,G", [(1, 256, 128), (3, 384, 64), (8, 256, 32), (12, 128, 128), (16, 512, 256)])
def test_consumer_lane_math_matches_oracle(M, K, G):
    x, qw, qz, s = strip_problem(M, K, G, seed=M * 7 + K)
    w = O.dequantize_awq(qw, qz, s, np.float32).astype(np.float64)
    y_true = x.astype(np.float64) @ w
    y = emulate_strip(qw.view(np.uint32), qz.view(np.uint32), s, x, G)
    assert np.allclose(y, y_true, rtol=1e-9, atol=1e-9 * np.abs(y_true).max()), np.abs(y - y_true).max()


def test_planted_errors_are_caught():
    x, qw, qz, s = strip_problem(2, 256, 128, seed=5)
    y_true = x.astype(np.float64) @ O.dequantize_awq(qw, qz, s, np.float32).astype(np.float64)
    for kw in ({"nibble_shift_bug": True}, {"swizzle_reads": False}):
        y = emulate_strip(qw.view(np.uint32), qz.view(np.uint32), s, x, 128, **kw)
        assert not np.allclose(y, y_true, rtol=1e-3), kw


def emulate_block_sums(x, half_bug=False):
    """The one-token kernel's sum of x over a 128-row block: one ldmatrix.x2 of the block's 8 x rows
    (lanes 0-7 give the rows of matrix 0 = k 0-7, lanes 8-15 those of matrix 1 = k 8-15, the 32-byte
    swizzle applied), one mma against ones (B column n = step n), then the kernel's lane shuffles.
    Returns each lane's value."""
    st = Stage(np.zeros((ROWS, WORDS), dtype=np.uint32), x.astype(np.float16).view(np.uint16)[:, :ROWS], 1)
    mats = []
    for q in range(2):  # lane 8 q + r gives row r of matrix q
        half = 0 if half_bug else q
        mats.append([st.row16(st.x, r * 32 + 16 * (half ^ ((r >> 2) & 1))) for r in range(8)])
    regs = ldsm_x4(mats + mats, trans=False)
    B = np.zeros((16, 8))
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        B[2 * t, g], B[2 * t + 1, g] = halves(regs[lane][0])
        B[2 * t + 8, g], B[2 * t + 9, g] = halves(regs[lane][1])
    D = np.ones((16, 16)) @ B
    v = np.array([D[lane >> 2, 2 * (lane & 3)] + D[lane >> 2, 2 * (lane & 3) + 1] for lane in range(32)])
    for mask in (1, 2):
        v = v + v[[lane ^ mask for lane in range(32)]]
    return v


def test_block_sum_of_x():
    """Every lane ends with the block's sum of x; a planted error (matrix 1 reading k 0-7) fails."""
    x = np.random.default_rng(3).standard_normal((1, ROWS)).astype(np.float16)
    want = float(x.astype(np.float64).sum())
    assert np.allclose(emulate_block_sums(x), want, rtol=0, atol=1e-9)
    assert not np.allclose(emulate_block_sums(x, half_bug=True), want, rtol=1e-3)
