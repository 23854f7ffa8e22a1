"""Q5_K blocks for the tests (the reference's tests hold none): hand-built
blocks whose values are written out from the format, and the scale packing
(llambda.lisp L4316-4336, L4387-4441, L6861-6917).

Block (176 bytes): fp16 d @0, fp16 dmin @2, 12 packed 6-bit scale/min bytes
@4, qh[32] @16, qs[128] @48.  Value l (l < 32) of sub-block pair g is the low
nibble of qs[32g + l] plus 16 if bit 2g of qh[l] is set, scaled by sub-block
2g; value 32 + l is the high nibble plus 16 if bit 2g + 1 is set, scaled by
sub-block 2g + 1."""
import numpy as np

Q5_K = 13


def pack_scales(sc, mn) -> bytes:
    """The 12 bytes from which get-scale-min-k4 reads (sc[j], mn[j]), j < 8,
    each a 6-bit value: j < 4 in the low 6 bits of bytes j and j + 4; j >= 4
    as a low nibble in byte j + 4 (scale low, min high) with the two high bits
    in the top bits of bytes j - 4 (scale) and j (min)."""
    b = [0] * 12
    for j in range(4):
        b[j] = sc[j] & 63
        b[j + 4] = mn[j] & 63
    for j in range(4, 8):
        b[j + 4] = (sc[j] & 15) | ((mn[j] & 15) << 4)
        b[j - 4] |= (sc[j] >> 4) << 6
        b[j] |= (mn[j] >> 4) << 6
    return bytes(b)


def hand_q5k():
    """One block with d = 0.5, dmin = 0.25, scales / mins covering the full
    6-bit range, every qh bit pattern, and its 256 values computed the way the
    reference does: delta = d*sc and offset = dmin*m in single float, then
    (delta * q) - offset."""
    sc = [1, 2, 63, 17, 33, 47, 50, 63]
    mn = [0, 5, 9, 63, 16, 31, 48, 1]
    qh = bytes((l * 37 + 11) & 0xFF for l in range(32))
    qs = bytes(((i * 7) & 15) | (((i * 5 + 3) & 15) << 4) for i in range(128))
    d, dmin = np.float32(0.5), np.float32(0.25)
    blk = (np.array([d, dmin], np.float16).tobytes() + pack_scales(sc, mn) + qh + qs)
    vals = np.zeros(256, np.float32)
    for g in range(4):
        for half in range(2):
            s = 2 * g + half
            delta = np.float32(d * np.float32(sc[s]))
            offset = np.float32(dmin * np.float32(mn[s]))
            for l in range(32):
                nib = (qs[32 * g + l] >> (4 * half)) & 15
                q = nib + (16 if (qh[l] >> s) & 1 else 0)
                vals[64 * g + 32 * half + l] = np.float32(np.float32(delta * np.float32(q)) - offset)
    return np.frombuffer(blk, np.uint8).copy(), vals


def dot_in_order(blk_row: np.ndarray, x: np.ndarray) -> np.float32:
    """dot-product-with-q5-k-tensor-data's own summation order in float32:
    one running sum, per sub-block pair and lane the low value's product then
    the high value's, every operation rounded."""
    s = np.float32(0)
    nb = blk_row.size // 176
    for b in range(nb):
        blk = blk_row[b * 176:(b + 1) * 176]
        d = np.frombuffer(blk[0:2].tobytes(), np.float16)[0].astype(np.float32)
        dmin = np.frombuffer(blk[2:4].tobytes(), np.float16)[0].astype(np.float32)
        sc12, qh, qs = blk[4:16], blk[16:48], blk[48:176]

        def scale_min(j):
            if j < 4:
                return sc12[j] & 63, sc12[j + 4] & 63
            return ((sc12[j + 4] & 15) | ((sc12[j - 4] >> 6) << 4),
                    (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4))

        for g in range(4):
            s0, m0 = scale_min(2 * g)
            s1, m1 = scale_min(2 * g + 1)
            dl0, of0 = np.float32(d * np.float32(s0)), np.float32(dmin * np.float32(m0))
            dl1, of1 = np.float32(d * np.float32(s1)), np.float32(dmin * np.float32(m1))
            for l in range(32):
                q0 = (int(qs[32 * g + l]) & 15) + (16 if (qh[l] >> (2 * g)) & 1 else 0)
                q1 = (int(qs[32 * g + l]) >> 4) + (16 if (qh[l] >> (2 * g + 1)) & 1 else 0)
                w0 = np.float32(np.float32(dl0 * np.float32(q0)) - of0)
                w1 = np.float32(np.float32(dl1 * np.float32(q1)) - of1)
                s = np.float32(s + np.float32(x[b * 256 + 64 * g + l] * w0))
                s = np.float32(s + np.float32(x[b * 256 + 64 * g + 32 + l] * w1))
    return s
