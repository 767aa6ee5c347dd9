"""Lane-level model of the token-row decode-attention kernel's fragment maps
(``qkv_decode_attn_t8_kernel`` in ``csrc/qkv_attn.cu``), run on the CPU.

The kernel's correctness and its bank-conflict freedom rest on a few integer
maps: the token order sigma inside each 8-token half, the dims each lane's V
fragment covers, the 128B-swizzled byte offsets of the K/V reads, and the
PTX fragment layouts of ``mma.m16n8k16`` and ``movmatrix.m8n8.trans``.  This
test restates those maps, runs one warp over one 64-token page in numpy
(fp16 operands, fp32-like accumulation in float64) and compares the result
with a direct computation of the same attention; it also checks that every
K (16-byte) and V (8-byte) fragment read of the warp touches 32 distinct
banks.  The GPU parity tests check the kernel itself against the oracle.
"""

import numpy as np

PS, D, RB, G = 64, 128, 128, 8
KOFF = 1024.0 + 127.0
SIGMA = 0x35247160  # nibble i = page row (mod 8) of MMA row i


def _f16(x):
    return np.float16(x).astype(np.float64)


def _lane_consts(lane):
    g, c = lane >> 2, lane & 3
    sg = (SIGMA >> (4 * g)) & 7
    sv0 = (SIGMA >> (8 * c)) & 7
    sv1 = (SIGMA >> (8 * c + 4)) & 7
    vdim = 32 * ((g >> 1) & 1) + 16 * (g >> 2) + 8 * (g & 1)
    kcol = [(((4 * grp) | c) ^ sg) << 4 for grp in range(2)]
    vcol0 = [(((64 * grp + vdim) >> 4 ^ sv0) << 4) + 8 * (g & 1) for grp in range(2)]
    vcol1 = [(((64 * grp + vdim) >> 4 ^ sv1) << 4) + 8 * (g & 1) for grp in range(2)]
    return dict(g=g, c=c, sg=sg, sv0=sv0, sv1=sv1, vdim=vdim, kcol=kcol, vcol0=vcol0, vcol1=vcol1)


LANES = [_lane_consts(lane) for lane in range(32)]


def _swizzle_128b(rows):
    """Page tile as the TMA 128B swizzle stores it: 16-byte chunk ^= row % 8."""
    out = np.zeros(rows.shape[0] * RB, np.uint8)
    for r in range(rows.shape[0]):
        for byte in range(RB):
            out[r * RB + (((byte >> 4) ^ (r & 7)) << 4) + (byte & 15)] = rows[r, byte]
    return out


# ---- PTX fragment layouts (lane = 4*g + c) ----------------------------------
def _a_matrix(frag):  # 16x16 A from per-lane registers (lo, hi)
    a = np.zeros((16, 16))
    for lane, regs in enumerate(frag):
        g, c = lane >> 2, lane & 3
        a[g, 2 * c:2 * c + 2] = regs[0]
        a[g + 8, 2 * c:2 * c + 2] = regs[1]
        a[g, 2 * c + 8:2 * c + 10] = regs[2]
        a[g + 8, 2 * c + 8:2 * c + 10] = regs[3]
    return a


def _b_matrix(frag):  # 16x8 B
    b = np.zeros((16, 8))
    for lane, regs in enumerate(frag):
        g, c = lane >> 2, lane & 3
        b[2 * c:2 * c + 2, g] = regs[0]
        b[2 * c + 8:2 * c + 10, g] = regs[1]
    return b


def _c_frags(cm):  # 16x8 accumulator -> per-lane (c0, c1, c2, c3)
    return np.array([[cm[l >> 2, 2 * (l & 3)], cm[l >> 2, 2 * (l & 3) + 1],
                      cm[(l >> 2) + 8, 2 * (l & 3)], cm[(l >> 2) + 8, 2 * (l & 3) + 1]] for l in range(32)])


def _movmatrix_trans(frag):  # 8x8 b16: lane holds (row g, cols 2c, 2c+1)
    m = np.zeros((8, 8))
    for lane, pair in enumerate(frag):
        m[lane >> 2, 2 * (lane & 3):2 * (lane & 3) + 2] = pair
    t = m.T
    return [(t[l >> 2, 2 * (l & 3)], t[l >> 2, 2 * (l & 3) + 1]) for l in range(32)]


def _banks_distinct(addrs, width):
    lanes_per_pass = 128 // width
    for p0 in range(0, 32, lanes_per_pass):
        seen = set()
        for a in addrs[p0:p0 + lanes_per_pass]:
            for k in range(0, width, 4):
                bank = ((a + k) // 4) % 32
                if bank in seen:
                    return False
                seen.add(bank)
    return True


def test_fragment_reads_are_bank_conflict_free():
    for lr in (0, 16, 32, 48):
        for grp in range(2):
            for h in range(2):
                assert _banks_distinct([(lr + 8 * h + L["sg"]) * RB + L["kcol"][grp] for L in LANES], 16)
                assert _banks_distinct([(lr + 8 * h + L["sv0"]) * RB + L["vcol0"][grp] for L in LANES], 8)
                assert _banks_distinct([(lr + 8 * h + L["sv1"]) * RB + L["vcol1"][grp] for L in LANES], 8)


def test_token_row_maps_reproduce_attention():
    rng = np.random.default_rng(7)
    kc = rng.integers(0, 255, (PS, D)).astype(np.uint8)
    vc = rng.integers(0, 255, (PS, D)).astype(np.uint8)
    ks = rng.uniform(0.01, 0.05, (PS, 2))
    vs = rng.uniform(0.01, 0.05, (PS, 2))
    q = _f16(rng.standard_normal((G, D)) * 0.3)
    length = 50  # the last tile is partly past the sequence end
    ksm, vsm = _swizzle_128b(kc), _swizzle_128b(vc)

    qsum = np.array([[q[h, 64 * grp:64 * grp + 64].sum() for grp in range(2)] for h in range(G)])
    qb = [{grp * 4 + st: [(q[L["g"], 64 * grp + 16 * L["c"] + 4 * st], q[L["g"], 64 * grp + 16 * L["c"] + 4 * st + 1]),
                          (q[L["g"], 64 * grp + 16 * L["c"] + 4 * st + 2], q[L["g"], 64 * grp + 16 * L["c"] + 4 * st + 3])]
           for grp in range(2) for st in range(4)} for L in LANES]
    kq = [[[KOFF * qsum[2 * L["c"] + e, grp] for grp in range(2)] for e in range(2)] for L in LANES]

    oacc = np.zeros((32, 8, 4))
    oone = np.zeros((32, 2, 4))
    m_run = np.full((32, 2), -np.inf)
    l_run = np.zeros((32, 2))
    for lr in (0, 16, 32, 48):
        kw = [[[ksm[(lr + 8 * h + L["sg"]) * RB + L["kcol"][grp]:][:16] for grp in range(2)] for h in range(2)]
              for L in LANES]
        vw = [[[vsm[(lr + r) * RB + col[grp]:][:8] for grp in range(2)]
               for r, col in ((L["sv0"], L["vcol0"]), (L["sv1"], L["vcol1"]),
                              (8 + L["sv0"], L["vcol0"]), (8 + L["sv1"], L["vcol1"]))] for L in LANES]
        valid = np.array([[lr + 8 * h + L["sg"] < length for h in range(2)] for L in LANES])
        ksc = np.array([[ks[lr + 8 * h + L["sg"]] for h in range(2)] for L in LANES])
        vsc = np.array([[vs[lr + 8 * h + L["sg"]] if valid[i, h] else (0.0, 0.0) for h in range(2)]
                        for i, L in enumerate(LANES)])
        # S^T = K.Q^T per 64-wide group
        sacc = np.zeros((32, 2, 4))
        for grp in range(2):
            cm = np.zeros((16, 8))
            for st in range(4):
                frag = []
                for lane in range(32):
                    k0 = kw[lane][0][grp][4 * st:4 * st + 4].astype(np.float64) + 1024
                    k1 = kw[lane][1][grp][4 * st:4 * st + 4].astype(np.float64) + 1024
                    frag.append([(k0[0], k0[1]), (k1[0], k1[1]), (k0[2], k0[3]), (k1[2], k1[3])])
                cm += _a_matrix(frag) @ _b_matrix([qb[lane][grp * 4 + st] for lane in range(32)])
            sacc[:, grp] = _c_frags(cm)
        s = np.full((32, 4), -np.inf)
        for lane in range(32):
            for i in range(4):
                h, e = i >> 1, i & 1
                if valid[lane, h]:
                    s[lane, i] = sum(ksc[lane, h, grp] * (sacc[lane, grp, i] - kq[lane][e][grp]) for grp in range(2))
        # online softmax per head column (lanes sharing c)
        pr = np.zeros((32, 4))
        for e in range(2):
            mt = np.maximum(s[:, e], s[:, 2 + e])
            for off in (4, 8, 16):
                mt = np.maximum(mt, mt[np.arange(32) ^ off])
            mnew = np.maximum(m_run[:, e], mt)
            none = mnew == -np.inf
            with np.errstate(invalid="ignore"):
                alpha = np.where(none, 1.0, np.exp2(m_run[:, e] - mnew))
                pr[:, e] = np.where(none, 0.0, np.exp2(s[:, e] - mnew))
                pr[:, 2 + e] = np.where(none, 0.0, np.exp2(s[:, 2 + e] - mnew))
            l_run[:, e] = l_run[:, e] * alpha + pr[:, e] + pr[:, 2 + e]
            m_run[:, e] = mnew
            oacc[:, :, e] *= alpha[:, None]
            oacc[:, :, 2 + e] *= alpha[:, None]
            oone[:, :, e] *= alpha[:, None]
            oone[:, :, 2 + e] *= alpha[:, None]
        # O^T += V^T.P'^T, P' moved into the B layout by the 8x8 transposes
        for grp in range(2):
            lo = [(_f16(pr[lane, 0] * vsc[lane, 0, grp]), _f16(pr[lane, 1] * vsc[lane, 0, grp])) for lane in range(32)]
            hi = [(_f16(pr[lane, 2] * vsc[lane, 1, grp]), _f16(pr[lane, 3] * vsc[lane, 1, grp])) for lane in range(32)]
            tlo, thi = _movmatrix_trans(lo), _movmatrix_trans(hi)
            bm = _b_matrix([[tlo[lane], thi[lane]] for lane in range(32)])
            oone[:, grp] += _c_frags(np.ones((16, 16)) @ bm)
            for jl in range(4):
                bs, wi = 2 * (jl & 1), jl >> 1
                frag = []
                for lane in range(32):
                    w = [vw[lane][t][grp][4 * wi:4 * wi + 4].astype(np.float64) + 1024 for t in range(4)]
                    frag.append([(w[0][bs], w[1][bs]), (w[0][bs + 1], w[1][bs + 1]),
                                 (w[2][bs], w[3][bs]), (w[2][bs + 1], w[3][bs + 1])])
                oacc[:, grp * 4 + jl] += _c_frags(_a_matrix(frag) @ bm)

    out = np.zeros((G, D))
    lsum = np.zeros(G)
    for lane, L in enumerate(LANES):
        for e in range(2):
            head = 2 * L["c"] + e
            if L["g"] == 0:
                lsum[head] = sum(l_run[(lane & 3) + 4 * gg, e] for gg in range(8))
            for j in range(8):
                grp, jl = j >> 2, j & 3
                for h in range(2):
                    out[head, 64 * grp + L["vdim"] + 2 * jl + h] = (oacc[lane, j, 2 * h + e]
                                                                    - KOFF * oone[lane, grp, 2 * h + e])
    out /= lsum[:, None]

    kd = (kc.astype(np.float64) - 127) * np.repeat(ks, 64, axis=1)
    vd = (vc.astype(np.float64) - 127) * np.repeat(vs, 64, axis=1)
    sc = q @ kd[:length].T
    p = np.exp2(sc - sc.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    want = p @ vd[:length]
    # fp16 rounding of P*vscale is the only approximation in the model
    np.testing.assert_allclose(out, want, rtol=1e-2, atol=2e-2)
    assert np.abs(out - want).max() < 5e-3
