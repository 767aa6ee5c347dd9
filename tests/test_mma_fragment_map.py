"""Lane-level model of the warp-MMA expert GEMM's fragment maps
(``mma_consume`` in ``csrc/qgemm_mma.cu``, 4-bit codes), run on the CPU.

One warp, one 16-row weight tile, one 128-wide K chunk (two 64-wide groups)
and 16 tokens (two n-tiles of 8).  Restated here: the 64B swizzle of the
TMA-staged code rows, the 32-bit word each lane reads (word c of 16-byte
chunk j ^ swizzle, for rows r and r+8), the unpack of a word into four bf16
A registers (``(w >> s) & 0x000F000F | 0x43004300`` = 128 + nibble), the
pairing of the token fragments from one 16-byte read of a token row, the
``mma.m16n8k16`` fragment layouts, the all-ones MMA giving sum(x), and the
per-group fold ``y += s*T + (b - 128 s)*X``.  The model's result must equal
the direct ``s*sum(q x) + b*sum(x)``, and every shared-memory read of the
warp must touch distinct banks.  The GPU parity tests check the kernel itself.
"""

import numpy as np

ROWS, K, TOK = 16, 128, 16
XS = 320  # bytes between staged token rows


def _a_matrix(frag):
    a = np.zeros((16, 16))
    for lane, regs in enumerate(frag):
        g, c = lane >> 2, lane & 3
        a[g, 2 * c:2 * c + 2] = regs[0]
        a[g + 8, 2 * c:2 * c + 2] = regs[1]
        a[g, 2 * c + 8:2 * c + 10] = regs[2]
        a[g + 8, 2 * c + 8:2 * c + 10] = regs[3]
    return a


def _b_matrix(frag):
    b = np.zeros((16, 8))
    for lane, regs in enumerate(frag):
        g, c = lane >> 2, lane & 3
        b[2 * c:2 * c + 2, g] = regs[0]
        b[2 * c + 8:2 * c + 10, g] = regs[1]
    return b


def _c_frags(cm):
    return np.array([[cm[l >> 2, 2 * (l & 3)], cm[l >> 2, 2 * (l & 3) + 1],
                      cm[(l >> 2) + 8, 2 * (l & 3)], cm[(l >> 2) + 8, 2 * (l & 3) + 1]] for l in range(32)])


def _swizzle_64b(rows):
    """Code rows of 64 bytes as the TMA 64B swizzle stores them."""
    out = np.zeros(rows.shape[0] * 64, np.uint8)
    for r in range(rows.shape[0]):
        for byte in range(64):
            out[r * 64 + (((byte >> 4) ^ ((r >> 1) & 3)) << 4) + (byte & 15)] = rows[r, byte]
    return out


def _word(buf, off):
    return int(buf[off]) | int(buf[off + 1]) << 8 | int(buf[off + 2]) << 16 | int(buf[off + 3]) << 24


def _unpack(w, s):
    v = ((w >> s) & 0x000F000F) | 0x43004300  # two bf16: 0x43 0x00 | nibble = 128 + nibble
    return (128 + (v & 0xF), 128 + ((v >> 16) & 0xF))


def _wword_offset(lane, j):
    r, c = lane >> 2, lane & 3
    sw = (r >> 1) & 3
    return r * 64 + ((j ^ sw) << 4) + 4 * c


def _banks_distinct(addrs, width):
    per_pass = 128 // width
    for p0 in range(0, 32, per_pass):
        seen = set()
        for a in addrs[p0:p0 + per_pass]:
            for k in range(0, width, 4):
                bank = ((a + k) // 4) % 32
                if bank in seen:
                    return False
                seen.add(bank)
    return True


def test_shared_memory_reads_are_bank_conflict_free():
    for j in range(4):
        for h in (0, 8 * 64):  # rows r and r+8
            assert _banks_distinct([h + _wword_offset(lane, j) for lane in range(32)], 4)
        for nt in range(2):
            assert _banks_distinct([(8 * nt + (lane >> 2)) * XS + 16 * (lane & 3) + 64 * j for lane in range(32)], 16)


def test_fragment_maps_reproduce_group_affine_matmul():
    rng = np.random.default_rng(3)
    q = rng.integers(0, 16, (ROWS, K))
    # MLX packing: element k of a row is nibble k % 8 (LSB first) of word k // 8
    codes = np.zeros((ROWS, 64), np.uint8)
    for k in range(0, K, 2):
        codes[:, k // 2] = q[:, k] | (q[:, k + 1] << 4)
    wsm = _swizzle_64b(codes)
    x = rng.standard_normal((TOK, K)).astype(np.float32).astype(np.float64)
    s = rng.uniform(0.001, 0.01, (ROWS, 2))
    b = rng.uniform(-0.05, 0.05, (ROWS, 2))

    acc = np.zeros((32, 2, 4))  # [lane][n-tile][c0..c3]
    for grp in range(2):
        t = np.zeros((2, 16, 8))
        xs = np.zeros((2, 16, 8))
        for jj in range(2):
            j = 2 * grp + jj
            a0, a1 = [], []
            for lane in range(32):
                wl = _word(wsm, _wword_offset(lane, j))
                wh = _word(wsm, 8 * 64 + _wword_offset(lane, j))
                a0.append([_unpack(wl, 0), _unpack(wh, 0), _unpack(wl, 4), _unpack(wh, 4)])
                a1.append([_unpack(wl, 8), _unpack(wh, 8), _unpack(wl, 12), _unpack(wh, 12)])
            for nt in range(2):
                b0, b1 = [], []
                for lane in range(32):
                    r, c = lane >> 2, lane & 3
                    u = x[8 * nt + r, 32 * j + 8 * c: 32 * j + 8 * c + 8]
                    b0.append([(u[0], u[4]), (u[1], u[5])])
                    b1.append([(u[2], u[6]), (u[3], u[7])])
                bm0, bm1 = _b_matrix(b0), _b_matrix(b1)
                t[nt] += _a_matrix(a0) @ bm0 + _a_matrix(a1) @ bm1
                xs[nt] += np.ones((16, 16)) @ bm0 + np.ones((16, 16)) @ bm1
        for nt in range(2):
            tf, xf = _c_frags(t[nt]), _c_frags(xs[nt])
            for lane in range(32):
                r = lane >> 2
                for e in range(4):
                    row = r + 8 * (e >> 1)
                    cc = b[row, grp] - 128 * s[row, grp]
                    acc[lane, nt, e] += s[row, grp] * tf[lane, e] + cc * xf[lane, e]

    got = np.zeros((ROWS, TOK))
    for lane in range(32):
        r, c = lane >> 2, lane & 3
        for nt in range(2):
            for e in range(4):
                got[r + 8 * (e >> 1), 8 * nt + 2 * c + (e & 1)] = acc[lane, nt, e]
    want = np.zeros((ROWS, TOK))
    for grp in range(2):
        ks = slice(64 * grp, 64 * grp + 64)
        want += s[:, grp:grp + 1] * (q[:, ks] @ x[:, ks].T) + b[:, grp:grp + 1] * x[:, ks].sum(1)[None, :]
    np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-9)
