"""Q5_0 / Q8_0 blocks for the tests (the reference's tests hold none): seeded
random blocks, and hand-built blocks whose dequantized values are written out
from the format (llambda.lisp L3965-4009)."""
import numpy as np

Q5_0, Q8_0 = 6, 8


def fp16_bytes(v: float) -> bytes:
    return np.array([v], np.float16).tobytes()


def random_blocks(type_tag: int, n_blocks: int, seed: int, dscale: float = 0.02) -> np.ndarray:
    """n_blocks random blocks: d = fp16(|N(0,1)| * dscale), values uniform."""
    rng = np.random.default_rng(seed)
    d = (np.abs(rng.standard_normal(n_blocks)) * dscale).astype(np.float16).view(np.uint8)
    d = d.reshape(n_blocks, 2)
    if type_tag == Q8_0:
        qs = rng.integers(0, 256, (n_blocks, 32), dtype=np.uint8)
        return np.ascontiguousarray(np.concatenate([d, qs], axis=1)).reshape(-1)
    qh = rng.integers(0, 256, (n_blocks, 4), dtype=np.uint8)
    qs = rng.integers(0, 256, (n_blocks, 16), dtype=np.uint8)
    return np.ascontiguousarray(np.concatenate([d, qh, qs], axis=1)).reshape(-1)


def hand_q5_0():
    """One Q5_0 block (d = 0.5) and its 32 values: value j = d * (q - 16) with
    q = (low nibble of qs[j] | bit j of qh << 4) for j < 16, (high nibble of
    qs[j-16] | bit j of qh << 4) otherwise."""
    qh = 0b1010_0000_0000_0001_1000_0000_0000_0011  # bits 0, 1, 15, 16, 29, 31
    qs = bytes(((15 - j) << 4) | j for j in range(16))  # low nibble j, high 15 - j
    blk = fp16_bytes(0.5) + qh.to_bytes(4, "little") + qs
    vals = []
    for j in range(32):
        nib = (j if j < 16 else 15 - (j - 16))
        q = nib | (((qh >> j) & 1) << 4)
        vals.append(0.5 * (q - 16))
    return np.frombuffer(blk, np.uint8).copy(), np.array(vals, np.float32)


def hand_q8_0():
    """One Q8_0 block (d = 0.25) holding -128..127 spread out, and its values."""
    q = np.array([-128, -127, -64, -1, 0, 1, 2, 63, 64, 127] + list(range(-11, 11)), np.int8)
    blk = fp16_bytes(0.25) + q.tobytes()
    return np.frombuffer(blk, np.uint8).copy(), (0.25 * q.astype(np.float32))
