"""numpy emulation of the decode kernel's integer-MMA scheme (test helper).

Reproduces, lane by lane, what k_gemv2b_imma does for one 16-row tile at batch 1:
the fixed-point activation table, the masked code words used as the u8 A fragment,
the s8 limb B fragment selected per lane, mma.sync m16n8k32 semantics, and the flush
arithmetic.  Used by tests/test_imma_scheme.py to check the scheme against the oracle
on the CPU.
"""
import numpy as np


def fixed_point_exp(maxabs: float) -> int:
    if not maxabs > 0:
        return 0
    _, e = np.frexp(np.float32(maxabs))
    return 14 - int(e)


def split_limbs(X: np.ndarray):
    hi = (X + 128) >> 8
    return hi, X - 256 * hi


def build_table(x16, mask16, K, W, cb):
    """Per block of 16W codes: entries[blk, limb, w, j] = 8 bytes (4 l-slot limbs, 4 h-slot limbs)."""
    BLK = 16 * W
    nblk = K // BLK
    xt = x16.astype(np.float16)
    if mask16 is not None:
        xt = (xt * mask16.astype(np.float16)).astype(np.float16)
    xt = xt.astype(np.float32)
    c0, c1, c2, _ = [np.float32(c) for c in cb]
    bl, bh = np.float32(c1 - c0), np.float32(np.float32(0.5) * np.float32(c2 - c0))
    cmax = max(abs(bl), abs(bh))
    ent = np.zeros((nblk, 2, W, 4, 8), dtype=np.int8)
    F = np.zeros(nblk, dtype=np.float32)
    T = np.zeros(nblk, dtype=np.float32)
    S = np.zeros(nblk, dtype=np.float32)
    for b in range(nblk):
        xb = xt[b * BLK:(b + 1) * BLK]
        E = fixed_point_exp(float(np.max(np.abs(xb))) * float(cmax))
        sc = np.float32(2.0 ** E)
        Xl = np.rint((xb * bl) * sc).astype(np.int64)
        Xh = np.rint((xb * bh) * sc).astype(np.int64)
        for limb in range(2):
            for w in range(W):
                for j in range(4):
                    for i in range(4):
                        k = 16 * w + 4 * i + j
                        hl, ll = split_limbs(Xl[k])
                        hh, lh = split_limbs(Xh[k])
                        ent[b, limb, w, j, i] = hl if limb == 0 else ll
                        ent[b, limb, w, j, 4 + i] = hh if limb == 0 else lh
        F[b] = np.float32(2.0 ** -E) / np.float32(64.0)
        S[b] = np.float32(np.sum(xb, dtype=np.float32))
        T[b] = np.float32(c0) * S[b]
    return ent, F, T, S


def mma_m16n8k32(a_regs, b_regs):
    """a_regs[lane][4] u8x4 words, b_regs[lane][2] s8x4 words -> C[16][8] int64 (mma.sync semantics)."""
    A = np.zeros((16, 32), dtype=np.int64)
    B = np.zeros((32, 8), dtype=np.int64)
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        for r in range(4):
            row = g + (8 if r & 1 else 0)
            kb = 4 * t + (16 if r & 2 else 0)
            for i in range(4):
                A[row, kb + i] = (int(a_regs[lane][r]) >> (8 * i)) & 0xFF          # u8
        for r in range(2):
            kb = 4 * t + (16 if r else 0)
            for i in range(4):
                v = (int(b_regs[lane][r]) >> (8 * i)) & 0xFF
                B[kb + i, g] = v - 256 if v >= 128 else v                          # s8
    return A @ B


def c_frag(C, lane):
    g, t = lane >> 2, lane & 3
    return [C[g, 2 * t], C[g, 2 * t + 1], C[g + 8, 2 * t], C[g + 8, 2 * t + 1]]


def words_of(row_bytes: np.ndarray, blk: int, W: int):
    seg = row_bytes[blk * 4 * W:(blk + 1) * 4 * W]
    return [int(np.frombuffer(seg[4 * w:4 * w + 4].tobytes(), dtype="<u4")[0]) for w in range(W)]


def tile_gemv(x16, packed, scales, G, cb, mask16=None, zeros=None, W=4, rows=range(16)):
    """Return fp32 y for the 16 rows of one tile (rows beyond N produce 0), without outliers/bias."""
    N, Kq = packed.shape
    K = 4 * Kq
    BLK = 16 * W
    nblk = K // BLK
    ent, F, T, S = build_table(x16, mask16, K, W, cb)
    acc = np.zeros(16, dtype=np.float64)
    rows = list(rows)
    for c in range((nblk + 3) // 4):
        a_w = {}
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            blk = 4 * c + t
            for half, gr in ((0, g), (1, g + 8)):
                r = rows[gr] if gr < len(rows) else None
                ok = r is not None and r < N and blk < nblk
                a_w[(lane, half)] = words_of(packed[r], blk, W) if ok else [0] * W
        C = [np.zeros((16, 8), dtype=np.int64) for _ in range(4)]
        for w in range(W):
            for j in range(4):
                ml, mh = 0x01010101 << (2 * j), 0x02020202 << (2 * j)
                a_regs, b_regs = [], []
                for lane in range(32):
                    g, t = lane >> 2, lane & 3
                    wg, wg8 = a_w[(lane, 0)][w], a_w[(lane, 1)][w]
                    a_regs.append([wg & ml, wg8 & ml, wg & mh, wg8 & mh])
                    bblk = 4 * c + (g >> 1)
                    if (g >> 1) == t and bblk < nblk:
                        e = ent[bblk, g & 1, w, j].view(np.uint8)
                        b_regs.append([int(np.frombuffer(e[:4].tobytes(), "<u4")[0]),
                                       int(np.frombuffer(e[4:].tobytes(), "<u4")[0])])
                    else:
                        b_regs.append([0, 0])
                C[j] += mma_m16n8k32(a_regs, b_regs)
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            blk = 4 * c + t
            if blk >= nblk:
                continue
            fr = [c_frag(C[j], lane) for j in range(4)]
            v = [64 * fr[0][f] + 16 * fr[1][f] + 4 * fr[2][f] + fr[3][f] for f in range(4)]
            grp = blk * BLK // G
            for half, gr, vh, vl in ((0, g, v[0], v[1]), (1, g + 8, v[2], v[3])):
                r = rows[gr] if gr < len(rows) else None
                if r is None or r >= N:
                    continue
                d = float(np.float32(256 * vh + vl)) * float(F[blk]) + float(T[blk])
                acc[gr] += float(scales[r, grp]) * d
                if zeros is not None:
                    acc[gr] += float(zeros[r, grp]) * float(S[blk])
    return acc
