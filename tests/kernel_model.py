"""Numpy model of the GEMV kernels' index arithmetic (test infrastructure).

Restates, element by element, what gemv.cu / weights.cu do with the device
row layout: the within-block permutations of the repack, the x-image
positions, the words each lane loads, the DP4A products and the lane
reductions; and the integer decompositions of the batched GEMV
(gemv_batch.cu): Q4_K's scale split into two 3-bit digits folded into A,
Q6_K's digit planes w = 128 w1 + w0. Tests compare this model with the oracle on CPU, so a wrong
permutation or lane mapping is caught before anything runs on a GPU.
"""
from __future__ import annotations

import numpy as np


def q4_xpos(e):
    e = np.asarray(e)
    p, half, r = e >> 6, (e >> 5) & 1, e & 31
    return 128 * half + 32 * p + 4 * (r & 7) + (r >> 3)


def q6_pic(ipos):
    ipos = np.asarray(ipos)
    return 4 * ((ipos & 7) >> 1) + 2 * (ipos & 1) + (ipos >> 3)


def q6_xpos(e):
    e = np.asarray(e)
    h, pos = e >> 7, e & 127
    hi, c = pos >> 6, pos & 63
    u = c >> 4
    return 128 * hi + 16 * (4 * h + u) + q6_pic(c & 15)


# ---- repack of one GGUF block (weights.cu repack_q4k / repack_q6k) ----------

def repack_q4k_block(blk: np.ndarray):
    hdr = blk[:16].copy()
    qs = np.zeros(128, np.uint8)
    o = np.arange(128)
    p, rr = o >> 5, o & 31
    qs[32 * p + 4 * (rr & 7) + (rr >> 3)] = blk[16 + o]
    return hdr, qs


def repack_q6k_block(blk: np.ndarray):
    """repack_q6k (weights.cu): ql and qh permuted within 16-byte chunks, qh
    stored with the top bit of every 2-bit field flipped (^ 0xAA)."""
    ql = np.zeros(128, np.uint8)
    qh = np.zeros(64, np.uint8)
    o = np.arange(128)
    ql[16 * (o >> 4) + q6_pic(o & 15)] = blk[o]
    o = np.arange(64)
    qh[16 * (o >> 4) + q6_pic(o & 15)] = blk[128 + o] ^ 0xAA
    return ql, qh, blk[192:208].view(np.int8).astype(np.int64), blk[208:210].view(np.float16)[0]


def q6_a4_bytes(wl: np.ndarray, wh: np.ndarray, sl: int, hh: int) -> np.ndarray:
    """Bytes of q6_a4_lo (hh = 0) / q6_a4_hi (hh = 1) from device ql / qh
    bytes, as signed values: no sign flip of their own (the stored qh carries
    it)."""
    wl, wh = wl.astype(np.int64), wh.astype(np.int64)
    if hh == 0:
        b = ((wl << 2) & 0x3C) | ((wh << (6 - sl)) & 0xC0)
    else:
        b = ((wl >> 2) & 0x3C) | ((wh << (2 - sl)) & 0xC0)
    b &= 0xFF
    return np.where(b >= 128, b - 256, b)


def _bytes(words_u8: np.ndarray) -> np.ndarray:
    return words_u8.astype(np.int64)


def q4_scales(hdr: np.ndarray, p: int):
    s = hdr[4:16].astype(np.int64)
    out = []
    for g in (2 * p, 2 * p + 1):
        if g < 4:
            out.append((s[g] & 63, s[g + 4] & 63))
        else:
            out.append(((s[g + 4] & 0xF) | ((s[g - 4] >> 6) << 4), (s[g + 4] >> 4) | ((s[g] >> 6) << 4)))
    return out  # [(sc_lo, m_lo), (sc_hi, m_hi)]


# ---- Q8_K exact: per-block integer lane sums -------------------------------------

def q4k_q8k_xpos(e):
    e = np.asarray(e)
    g = e >> 5
    return 128 * (g >> 2) + 16 * (e & 7) + 4 * (g & 3) + ((e >> 3) & 3)


def q4k_block_sumi_model(blk: np.ndarray, q8: np.ndarray):
    """Per-class sums sumi[k] and minsum of one block, via the kernel's lanes:
    lane j owns class j (its qs words at 32p + 4j, its q8 words at 16j and
    128 + 16j of the class-major image) and group j's min term."""
    hdr, qs = repack_q4k_block(blk)
    img = np.zeros(256, np.int64)
    img[q4k_q8k_xpos(np.arange(256))] = q8
    bs = q8.astype(np.int64).reshape(8, 32).sum(1)
    sumi = np.zeros(8, np.int64)
    msum = 0
    for j in range(8):
        xg = np.concatenate([img[16 * j: 16 * j + 16], img[128 + 16 * j: 128 + 16 * j + 16]]).reshape(8, 4)
        for p in range(4):
            (sc_lo, _), (sc_hi, _) = q4_scales(hdr, p)
            w = _bytes(qs[32 * p + 4 * j: 32 * p + 4 * j + 4])
            sumi[j] += sc_lo * int(((w & 0xF) * xg[2 * p]).sum()) + sc_hi * int(((w >> 4) * xg[2 * p + 1]).sum())
        m_j = q4_scales(hdr, j >> 1)[j & 1][1]  # group j's min, taken by lane j
        msum += m_j * int(bs[j])
    return sumi, msum


def q4k_block_sumi_reference(blk: np.ndarray, q8: np.ndarray):
    """quants.rs:328-351 directly."""
    s = blk[4:16].astype(np.int64)
    sc, m = [], []
    for g in range(8):
        if g < 4:
            sc.append(s[g] & 63)
            m.append(s[g + 4] & 63)
        else:
            sc.append((s[g + 4] & 0xF) | ((s[g - 4] >> 6) << 4))
            m.append((s[g + 4] >> 4) | ((s[g] >> 6) << 4))
    qs = blk[16:].astype(np.int64)
    sumi = np.zeros(8, np.int64)
    for e in range(256):
        pos = e % 64
        byte = qs[32 * (e // 64) + pos % 32]
        a = byte & 0xF if pos < 32 else byte >> 4
        sumi[e % 8] += sc[e // 32] * a * int(q8[e])
    bsums = q8.astype(np.int64).reshape(16, 16).sum(1)
    minsum = int(sum(bsums[g] * m[g // 2] for g in range(16)))
    return sumi, minsum


def q6k_block_sumi_model(blk: np.ndarray, q8: np.ndarray):
    ql, qh, sc, _ = repack_q6k_block(blk)
    # x image: masked A/B words per (lane, half, word)
    A = np.zeros((8, 2, 4, 4), np.int64)
    B = np.zeros((8, 2, 4, 4), np.int64)
    for e in range(256):
        h, pos = e >> 7, e & 127
        hh, c = pos >> 6, pos & 63
        u, ipos = c >> 4, c & 15
        j = 4 * h + u
        pic = int(q6_pic(ipos))
        w, bpos = pic >> 2, pic & 3
        (A if bpos < 2 else B)[j, hh, w, bpos] = int(q8[e])
    P = np.zeros((8, 8), np.int64)  # [lane, class] partial 4*sumi
    for j in range(8):
        h, u = j >> 2, j & 3
        sl = 2 * (u >> 1)
        wl = _bytes(ql[16 * j: 16 * j + 16]).reshape(4, 4)
        wh = _bytes(qh[16 * (2 * h + (u & 1)): 16 * (2 * h + (u & 1)) + 16]).reshape(4, 4)
        sc_lo, sc_hi = sc[8 * h + u], sc[8 * h + 4 + u]
        for t in range(4):
            whr = wh[t] ^ 0xAA  # the stored qh is flipped
            raw_lo = (wl[t] & 0xF) | (((whr >> sl) & 3) << 4)
            raw_hi = (wl[t] >> 4) | (((whr >> (sl + 4)) & 3) << 4)
            a_lo, a_hi = 4 * (raw_lo - 32), 4 * (raw_hi - 32)
            assert np.array_equal(a_lo, q6_a4_bytes(wl[t], wh[t], sl, 0))
            assert np.array_equal(a_hi, q6_a4_bytes(wl[t], wh[t], sl, 1))
            P[j, 2 * t] += sc_lo * int((a_lo * A[j, 0, t]).sum()) + sc_hi * int((a_hi * A[j, 1, t]).sum())
            P[j, 2 * t + 1] += sc_lo * int((a_lo * B[j, 0, t]).sum()) + sc_hi * int((a_hi * B[j, 1, t]).sum())
    tot = P.sum(0)
    assert np.all(tot % 4 == 0)
    return tot >> 2


def q6_q8k_byte(j, hh, w, ab, bpos):
    return 128 * (2 * hh + (w >> 1)) + 16 * j + 4 * (2 * (w & 1) + ab) + bpos


def q6k_q8k_image(q8: np.ndarray) -> np.ndarray:
    """The 512 masked-word bytes of the Q6_K Q8_K x image (q8k_span_write)."""
    im = np.zeros(512, np.int64)
    for e in range(256):
        h, pos = e >> 7, e & 127
        hh, c = pos >> 6, pos & 63
        u, ipos = c >> 4, c & 15
        j = 4 * h + u
        pic = int(q6_pic(ipos))
        w, bpos = pic >> 2, pic & 3
        own = 0 if bpos < 2 else 1
        im[q6_q8k_byte(j, hh, w, own, bpos)] = int(q8[e])
        im[q6_q8k_byte(j, hh, w, 1 - own, bpos)] = 0
    return im


def q6k_rows_mma_model(blks: list, q8: np.ndarray) -> np.ndarray:
    """sumi[row][class] of one block for 16 rows, through the fragments of
    q6k_q8k_mma_item: per (chunk j, half hh) an m16n8k16 MMA with A[r][4t+i]
    = byte i of 4 (raw6 - 32) built from word t of row r's ql/qh chunk, and
    B[4t+i][n] = byte i of lane (gid n, tig t)'s XBlock6 word b[2j+hh]; then
    the per-row int8 scales and the final division by 4."""
    assert len(blks) == 16
    im = q6k_q8k_image(q8)
    rows = [repack_q6k_block(b) for b in blks]
    # XBlock6 of every lane (gid, tig)
    breg = np.zeros((8, 4, 16, 4), np.int64)  # [gid, tig, 2j+hh, byte]
    for gid in range(8):
        for tig in range(4):
            own, ab = (gid >> 1) == tig, gid & 1
            for j in range(8):
                for hh in range(2):
                    if own:
                        o = q6_q8k_byte(j, hh, tig, ab, 0)
                        breg[gid, tig, 2 * j + hh] = im[o:o + 4]
    acc = np.zeros((16, 8), np.int64)
    for j in range(8):
        h, u = j >> 2, j & 3
        sl, c = 2 * (u >> 1), 2 * h + (u & 1)
        for hh in range(2):
            s_idx = 8 * h + u + 4 * hh
            A = np.zeros((16, 16), np.int64)
            for r, (ql, qh, sc, _) in enumerate(rows):
                for t in range(4):
                    wl = ql[16 * j + 4 * t: 16 * j + 4 * t + 4].astype(np.int64)
                    wh = qh[16 * c + 4 * t: 16 * c + 4 * t + 4].astype(np.int64)
                    A[r, 4 * t: 4 * t + 4] = q6_a4_bytes(wl, wh, sl, hh)
            B = np.zeros((16, 8), np.int64)
            for n in range(8):
                for t in range(4):
                    B[4 * t: 4 * t + 4, n] = breg[n, t, 2 * j + hh]
            D = A @ B
            for r, (ql, qh, sc, _) in enumerate(rows):
                acc[r] += sc[s_idx] * D[r]
    assert np.all(acc % 4 == 0) and np.all(np.abs(acc) < 2**31)
    return acc >> 2


def q6k_block_sumi_reference(blk: np.ndarray, q8: np.ndarray):
    ql, qh = blk[:128].astype(np.int64), blk[128:192].astype(np.int64)
    sc = blk[192:208].view(np.int8).astype(np.int64)
    sumi = np.zeros(8, np.int64)
    for e in range(256):
        pos = e % 128
        byte = ql[64 * (e // 128) + pos % 64]
        nib = byte & 0xF if pos < 64 else byte >> 4
        hi2 = (qh[32 * (e // 128) + pos % 32] >> (2 * (pos // 32))) & 3
        a = (nib | (hi2 << 4)) - 32
        sumi[e % 8] += sc[e // 16] * a * int(q8[e])
    return sumi


# ---- F32X: 22-bit fixed-point limbs, exact integer dots ---------------------------

def f32x_limbs(x: np.ndarray):
    """prep_f32x for one 256-span: (xint, xs) with x ~= xint * xs."""
    amax = float(np.max(np.abs(x)))
    if amax == 0.0:
        return np.zeros(256, np.int64), 0.0
    _, ex = np.frexp(np.float32(amax))
    xi = np.rint(np.ldexp(x.astype(np.float64), 22 - int(ex))).astype(np.int64)
    return xi, float(np.ldexp(1.0, int(ex) - 22))


def q4k_block_f32x_model(blk: np.ndarray, x: np.ndarray) -> float:
    """F32X block contribution via lanes: exact ints, combined in float64 here."""
    hdr, qs = repack_q4k_block(blk)
    xi, xs = f32x_limbs(x)
    img = np.zeros(256, np.int64)
    img[q4_xpos(np.arange(256))] = xi
    hi_l, mid_l, lo_l = img >> 16, (img >> 8) & 255, img & 255
    assert np.all(hi_l * 65536 + mid_l * 256 + lo_l == img) and np.all(np.abs(hi_l) <= 64)
    d = float(hdr[0:2].view(np.float16)[0])
    dmin = float(hdr[2:4].view(np.float16)[0])
    tot = 0.0
    for j in range(8):
        p, kh = j >> 1, j & 1
        (sc_lo, m_lo), (sc_hi, m_hi) = q4_scales(hdr, p)
        w = _bytes(qs[32 * p + 16 * kh: 32 * p + 16 * kh + 16])
        o_lo, o_hi = 16 * j, 128 + 16 * j
        lo, hi = w & 0xF, w >> 4
        A = [sc_lo * int((lo * L[o_lo:o_lo + 16]).sum()) + sc_hi * int((hi * L[o_hi:o_hi + 16]).sum())
             for L in (hi_l, mid_l, lo_l)]
        F = A[0] * 65536.0 + A[1] * 256.0 + A[2]
        xsl = float(img[o_lo:o_lo + 16].sum()) * xs
        xsh = float(img[o_hi:o_hi + 16].sum()) * xs
        tot += d * xs * F - dmin * (m_lo * xsl + m_hi * xsh)
    return tot


def q4k_minsum_mma_model(hdrs: list, q8: np.ndarray) -> np.ndarray:
    """minsum of 16 Q4_K rows (one block each) through the fragments of the
    min-term MMA in q4k_q8k_mma_item: m16n8k16 int8, A[r][4t+i] = byte i of
    lane (r, t)'s A word (tig 0: mins of groups 0..3 = hdr bytes 8..11 & 63;
    tig 1: groups 4..7 from the packed high bits; tig 2, 3: zero), B[4t+i][n]
    = byte i of lane (n, t)'s XBlock::bm (n = 0: balanced low bytes, n = 1:
    high bytes of the eight group sums); minsum = D[r][0] + 256 D[r][1]."""
    gs = q8.astype(np.int64).reshape(8, 32).sum(1)
    lo = ((gs + 128) & 255) - 128
    hi = (gs - lo) >> 8
    assert np.all(np.abs(hi) < 128)
    B = np.zeros((16, 8), np.int64)
    for t in range(2):
        for i in range(4):
            B[4 * t + i, 0] = lo[4 * t + i]
            B[4 * t + i, 1] = hi[4 * t + i]
    A = np.zeros((16, 16), np.int64)
    for r, hdr in enumerate(hdrs):
        w = hdr.astype(np.uint32)
        z = int(w[8]) | int(w[9]) << 8 | int(w[10]) << 16 | int(w[11]) << 24   # header word .z
        ww = int(w[12]) | int(w[13]) << 8 | int(w[14]) << 16 | int(w[15]) << 24  # header word .w
        ma = z & 0x3F3F3F3F
        mb = ((ww >> 4) & 0x0F0F0F0F) | ((z >> 2) & 0x30303030)
        for i in range(4):
            A[r, i] = (ma >> (8 * i)) & 0xFF
            A[r, 4 + i] = (mb >> (8 * i)) & 0xFF
    D = A @ B
    return D[:, 0] + 256 * D[:, 1]


# ---- batched decode (design model): scales folded into the A operand -------

def q4k_sumi_scale_split_batched(blks: list, q8s: np.ndarray) -> np.ndarray:
    """sumi[r][b][k] of rows `blks` (one Q4_K block each) against B Q8_K
    blocks `q8s` [B, 256], as two integer matrix products over the whole
    block (K = 256) instead of one product per scale group.

    A row's 6-bit group scale is split as sc = 8 * sc_hi + sc_lo (3 bits
    each), so both A operands sc_lo * a and sc_hi * a (a = the 4-bit quant)
    lie in [0, 105] and fit the u8 operand of an int8 MMA; B holds, per
    sequence b and lane class k, the q8 values of the elements e with
    e % 8 == k (zero elsewhere), i.e. N = 8 * B columns. Then
    sumi = 8 * (A_hi @ B) + (A_lo @ B), every partial exact in int32
    (|A_lo @ B| <= 256 * 105 * 127 < 2^23)."""
    R, B = len(blks), q8s.shape[0]
    a_lo = np.zeros((R, 256), np.int64)
    a_hi = np.zeros((R, 256), np.int64)
    e = np.arange(256)
    pos = e % 64
    for r, blk in enumerate(blks):
        s = blk[4:16].astype(np.int64)
        sc = [(s[g] & 63) if g < 4 else ((s[g + 4] & 0xF) | ((s[g - 4] >> 6) << 4)) for g in range(8)]
        qs = blk[16:].astype(np.int64)
        byte = qs[32 * (e // 64) + pos % 32]
        a = np.where(pos < 32, byte & 0xF, byte >> 4)
        scv = np.array(sc, np.int64)[e // 32]
        a_lo[r] = (scv & 7) * a
        a_hi[r] = (scv >> 3) * a
    bmat = np.zeros((256, B * 8), np.int64)
    for b in range(B):
        for k in range(8):
            sel = e % 8 == k
            bmat[sel, 8 * b + k] = q8s[b, sel]
    assert a_lo.max() <= 105 and a_hi.max() <= 105
    d_lo, d_hi = a_lo @ bmat, a_hi @ bmat
    assert np.abs(d_lo).max() < 2 ** 31 and np.abs(d_hi).max() < 2 ** 31
    return (8 * d_hi + d_lo).reshape(R, B, 8)


def q4k_gemv_q8k_batched_model(wb: np.ndarray, dim_in: int, dim_out: int, q8_d: np.ndarray,
                               q8_qs: np.ndarray) -> np.ndarray:
    """y[b][r] = dot_q4_k_q8_k of row r with Q8_K vector b (quants.rs:312-360),
    for B vectors at once: the integer sums of every (row, sequence) from
    q4k_sumi_scale_split_batched, the min term as an (8 x B) integer product,
    then the reference's f32 epilogue per (row, sequence) in its order
    (d = q8.d * f16(d); sums[k] += d * sumi[k]; sumf -= (f16(dmin) * q8.d) *
    minsum; s = sumf + sums[0] + ... + sums[7]), every operation rounded
    separately in f32. q8_d: [B, nb] f32; q8_qs: [B, nb, 256] int."""
    nb = dim_in // 256
    B = q8_qs.shape[0]
    f32 = np.float32
    rows = wb.reshape(dim_out, nb, 144)
    y = np.zeros((B, dim_out), f32)
    bsums = q8_qs.astype(np.int64).reshape(B, nb, 16, 16).sum(3)  # [B, nb, 16]
    for r in range(dim_out):
        sums = np.zeros((B, 8), f32)
        sumf = np.zeros(B, f32)
        for i in range(nb):
            blk = rows[r, i]
            sumi = q4k_sumi_scale_split_batched([blk], q8_qs[:, i, :])[0]  # [B, 8]
            s = blk[4:16].astype(np.int64)
            m = [(s[g + 4] & 63) if g < 4 else ((s[g + 4] >> 4) | ((s[g] >> 6) << 4)) for g in range(8)]
            m16 = np.repeat(np.array(m, np.int64), 2)  # bsums group g pairs with m[g // 2]
            minsum = bsums[:, i, :] @ m16  # [B]
            dd = blk[0:2].view(np.float16).astype(f32)[0]
            dmin = blk[2:4].view(np.float16).astype(f32)[0]
            d = (q8_d[:, i].astype(f32) * dd).astype(f32)
            sums = (sums + (d[:, None] * sumi.astype(f32)).astype(f32)).astype(f32)
            sumf = (sumf - ((dmin * q8_d[:, i].astype(f32)).astype(f32) * minsum.astype(f32)).astype(f32)).astype(f32)
        out = sumf
        for k in range(8):
            out = (out + sums[:, k]).astype(f32)
        y[:, r] = out
    return y


def q6k_gemv_q8k_batched_model(wb: np.ndarray, dim_in: int, dim_out: int, q8_d: np.ndarray,
                               q8_qs: np.ndarray) -> np.ndarray:
    """y[b][r] = dot_q6_k_q8_k of row r with Q8_K vector b (quants.rs:371-412)
    for B vectors at once. The scaled quant w = sc * (raw6 - 32) lies in
    [-4064, 4096]; it enters the int8 MMA as two operands w = 128 * w1 + w0,
    w0 = w & 127 in [0, 127], w1 = w >> 7 in [-32, 32], so per block
    sumi = 128 * (W1 @ Bq) + (W0 @ Bq) with the class-masked q8 columns Bq of
    q4k_sumi_scale_split_batched (|W0 @ Bq| <= 256 * 127 * 127 < 2^23). The
    f32 epilogue follows the reference per (row, sequence): d = q8.d * f16(d),
    sums[k] += d * sumi[k], s = sums[0] + ... + sums[7] from 0."""
    nb = dim_in // 256
    B = q8_qs.shape[0]
    f32 = np.float32
    rows = wb.reshape(dim_out, nb, 210)
    e = np.arange(256)
    pos = e % 128
    bq = np.zeros((nb, 256, B * 8), np.int64)
    for b in range(B):
        for k in range(8):
            sel = e % 8 == k
            bq[:, sel, 8 * b + k] = q8_qs[b][:, sel]
    y = np.zeros((B, dim_out), f32)
    for r in range(dim_out):
        sums = np.zeros((B, 8), f32)
        for i in range(nb):
            blk = rows[r, i]
            ql, qh = blk[:128].astype(np.int64), blk[128:192].astype(np.int64)
            sc = blk[192:208].view(np.int8).astype(np.int64)
            byte = ql[64 * (e // 128) + pos % 64]
            nib = np.where(pos < 64, byte & 0xF, byte >> 4)
            hi2 = (qh[32 * (e // 128) + pos % 32] >> (2 * (pos // 32))) & 3
            w = sc[e // 16] * ((nib | (hi2 << 4)) - 32)
            w0, w1 = w & 127, w >> 7
            assert w0.min() >= 0 and w0.max() <= 127 and w1.min() >= -32 and w1.max() <= 32
            sumi = (128 * (w1 @ bq[i]) + (w0 @ bq[i])).reshape(B, 8)
            dd = blk[208:210].view(np.float16).astype(f32)[0]
            d = (q8_d[:, i].astype(f32) * dd).astype(f32)
            sums = (sums + (d[:, None] * sumi.astype(f32)).astype(f32)).astype(f32)
        out = np.zeros(B, f32)
        for k in range(8):
            out = (out + sums[:, k]).astype(f32)
        y[:, r] = out
    return y
