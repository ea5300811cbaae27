"""Lane-level emulation of one 16-row step of the column-strip GEMV consumer (``csrc/gemv_strip.cu``).

Emulates, on the bytes of a shared-memory stage, exactly what each of a warp's 32 lanes loads and
computes: the weight-row offsets, the byte permutes (``prmt``) and nibble masks that build the
mma.sync A fragments and the x loads that build the B fragments. The fragments of all lanes are then assembled into the m16n8k16 A (16 x 16) and B (16 x 8)
matrices following the PTX fragment layout, multiplied, and compared with the dot products the
kernel's epilogue assumes: row r of mma j is column j (r < 8) or j + 4 (r >= 8) of word r % 8,
column n is token 8 * mt + n. The fragments are checked on the magic-number halves (1024 + q for
columns 0, 1, 4, 5 of a word, 1024 + 16 q for 2, 3, 6, 7) before the kernel subtracts the zero point,
so the nibble selection is what is tested.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import awq_oracle as O

X_ROW_BYTES = 512  # one token's 256 fp16 x values per stage


def prmt(a: int, b: int, sel: int) -> int:
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    return sum(src[(sel >> (4 * i)) & 7] << (8 * i) for i in range(4))


def lop3_and_or(v: int, mask: int, magic: int) -> int:
    return (v & mask) | magic


def magic_halves(T: int):
    T8 = T >> 8
    return [lop3_and_or(T, 0x000F000F, 0x64006400), lop3_and_or(T, 0x00F000F0, 0x64006400),
            lop3_and_or(T8, 0x000F000F, 0x64006400), lop3_and_or(T8, 0x00F000F0, 0x64006400)]


def halves(u32: int):
    lo, hi = np.array([u32 & 0xFFFF, u32 >> 16], dtype=np.uint16).view(np.float16)
    return float(lo), float(hi)


class Stage:
    """Shared memory of one stage: weights [256 rows][8 words], then x [M][256] fp16."""

    def __init__(self, words: np.ndarray, x: np.ndarray):
        self.words = words.astype(np.uint32)            # [256, 8]
        self.x = x.astype(np.float16).view(np.uint16)   # [M, 256] bit patterns
        self.M = x.shape[0]

    def w_at(self, byte_off: int) -> int:
        return int(self.words.reshape(-1)[byte_off // 4])

    def x_u32(self, byte_off: int) -> int:
        flat = self.x.reshape(-1)
        i = byte_off // 2
        return int(flat[i]) | (int(flat[i + 1]) << 16)


def emulate_step(stage: Stage, s: int, mt_count: int):
    """Assemble, for every mma j and token tile mt, the A and B matrices the warp feeds mma.sync."""
    A = np.full((4, 16, 16), np.nan)
    B = np.full((mt_count, 16, 8), np.nan)
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        roff = [(2 * t + (q & 1) + 8 * (q >> 1)) * 32 + 4 * g for q in range(4)]
        w = [stage.w_at(s * 16 * 32 + r) for r in roff]
        oa, ob = magic_halves(prmt(w[0], w[1], 0x6420)), magic_halves(prmt(w[0], w[1], 0x7531))
        oc, od = magic_halves(prmt(w[2], w[3], 0x6420)), magic_halves(prmt(w[2], w[3], 0x7531))
        for j in range(4):
            sl = ((j & 1) << 1) | (j >> 1)
            regs = [oa[sl], ob[sl], oc[sl], od[sl]]
            for reg, (row, kb) in zip(regs, [(g, 2 * t), (g + 8, 2 * t), (g, 2 * t + 8), (g + 8, 2 * t + 8)]):
                assert np.isnan(A[j, row, kb]) and np.isnan(A[j, row, kb + 1])
                A[j, row, kb], A[j, row, kb + 1] = halves(reg)
        for mt in range(mt_count):
            tok = 8 * mt + g
            b0 = b1 = 0
            if tok < stage.M:
                xrow = tok * X_ROW_BYTES + 4 * t
                b0 = stage.x_u32(xrow + s * 32)
                b1 = stage.x_u32(xrow + s * 32 + 16)
            for reg, kb in ((b0, 2 * t), (b1, 2 * t + 8)):
                assert np.isnan(B[mt, kb, g])
                B[mt, kb, g], B[mt, kb + 1, g] = halves(reg)
    assert not np.isnan(A).any() and not np.isnan(B).any()
    return A, B


@pytest.mark.parametrize("m", [1, 4, 9, 16])
def test_fragments_compute_the_strip_dot_products(m):
    rng = np.random.default_rng(1000 * m)
    k0, n_words = 0, 8
    q = rng.integers(0, 16, (256, 8 * n_words))
    words = O.pack_awq(q.astype(np.int32)).view(np.uint32)      # [256, 8]: the stage's weight box
    x = rng.standard_normal((m, 256)).astype(np.float16)
    stage = Stage(words, x)
    mt_count = 2 if m > 8 else 1
    low = np.array([c % 4 < 2 for c in range(8)])
    magic = np.where(np.tile(low, n_words), 1024 + q, 1024 + 16 * q).astype(np.float64)  # [256, 64]
    xf = x.astype(np.float64)
    for s in range(16):
        A, B = emulate_step(stage, s, mt_count)
        for j in range(4):
            for mt in range(mt_count):
                C = A[j] @ B[mt]                                  # [16 mma rows, 8 tokens]
                for r in range(16):
                    col = 8 * (r % 8) + j + (4 if r >= 8 else 0)
                    for n in range(8):
                        tok = 8 * mt + n
                        want = 0.0 if tok >= m else float(magic[k0 + 16 * s:k0 + 16 * s + 16, col]
                                                            @ xf[tok, 16 * s:16 * s + 16])
                        assert C[r, n] == pytest.approx(want, rel=1e-12, abs=1e-9), (s, j, mt, r, n)


def _consumer_strip(x, q, z, s_scales, g_size):
    """The consumer warp's whole K loop for one 64-column strip, lane by lane: per 16-row step the
    warp-wide mma on the assembled fragments (fp32 accumulation into the lanes' partials), a flush
    at every quantization-group change, and the final per-lane
    accumulators mapped back to y[token, column] as the kernel's reduction stores them."""
    m, k = x.shape
    mt_count = 2 if m > 8 else 1
    words = O.pack_awq(q.astype(np.int32)).view(np.uint32)          # [K, 8]
    low = np.array([c % 4 < 2 for c in range(8)])
    acc = np.zeros((32, mt_count, 4, 4), np.float32)
    part = np.zeros_like(acc)
    cur = -1
    for k0 in range(0, k, 256):
        stage = Stage(words[k0:k0 + 256], x[:, k0:k0 + 256])
        for s in range(min(256, k - k0) // 16):
            grp = (k0 + 16 * s) // g_size
            if grp != cur:
                if cur >= 0:
                    _flush(acc, part, s_scales[cur])
                cur = grp
            A, B = emulate_step(stage, s, mt_count)
            zc = z[cur]  # the kernel feeds (q - z): rebuild A from the magic values
            for j in range(4):
                for r in range(16):
                    col = 8 * (r % 8) + j + (4 if r >= 8 else 0)
                    A[j, r] = (A[j, r] - 1024) / (1 if low[col % 8] else 16) - zc[col]
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                for mt in range(mt_count):
                    for j in range(4):
                        C = (A[j].astype(np.float64) @ B[mt].astype(np.float64)).astype(np.float32)
                        part[lane, mt, j] += np.array([C[g, 2 * t], C[g, 2 * t + 1], C[g + 8, 2 * t],
                                                       C[g + 8, 2 * t + 1]], np.float32)
    _flush(acc, part, s_scales[cur])
    y = np.zeros((m, 64), np.float32)
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        for mt in range(mt_count):
            for j in range(4):
                for e, (dc, dt) in enumerate([(0, 0), (0, 1), (4, 0), (4, 1)]):
                    tok = 8 * mt + 2 * t + dt
                    if tok < m:
                        y[tok, 8 * g + j + dc] = acc[lane, mt, j, e]
    return y


def _flush(acc, part, srow):
    for lane in range(32):
        g = lane >> 2
        sc = srow[8 * g:8 * g + 8].astype(np.float32)
        for mt in range(part.shape[1]):
            for j in range(4):
                acc[lane, mt, j] += np.array([sc[j], sc[j], sc[4 + j], sc[4 + j]], np.float32) * part[lane, mt, j]
                part[lane, mt, j] = 0


@pytest.mark.parametrize("g_size", [32, 64, 128])
@pytest.mark.parametrize("m", [1, 9])
def test_consumer_loop_matches_the_oracle(g_size, m):
    """The strip consumer's K loop (two stages, several quantization groups) gives
    y within the reference's parity criterion of the oracle's fp64 truth, on one 64-column strip."""
    rng = np.random.default_rng(g_size + 7 * m)
    k = 512
    q = rng.integers(0, 16, (k, 64))
    z = rng.integers(0, 16, (k // g_size, 64))
    s_scales = (rng.random((k // g_size, 64)) * 0.018 + 0.002).astype(np.float16)
    x = rng.standard_normal((m, k)).astype(np.float16)
    qw, qz = O.pack_awq(q.astype(np.int32)), O.pack_awq(z.astype(np.int32))
    y_true = O.w4a16_gemm_fp64(x, qw, qz, s_scales)
    w16 = O.dequantize_awq(qw, qz, s_scales, np.float16)
    e_fp16 = O.rel_err((x.astype(np.float32) @ w16.astype(np.float32)).astype(np.float16).astype(np.float32),
                       y_true)
    y = _consumer_strip(x, q, z, s_scales, g_size).astype(np.float16).astype(np.float32)
    assert O.rel_err(y, y_true) <= 2 * e_fp16 + 1e-5, (O.rel_err(y, y_true), e_fp16)
