"""CPU oracle against the reference's own known-answer tests (tests.lisp) and
self-consistency checks of the restated algorithm."""
import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")))


def _slices(checks, arr):
    for key, want in checks.items():
        if ":" in key:
            a, b = map(int, key.split(":"))
            assert np.all(arr[a:b] == np.float32(want)), key
        else:
            assert arr[int(key)] == np.float32(want), key


def test_dequantize_q4_k_known_answer():  # tests.lisp T2386-2416, T2324-2367
    blk = np.array(GOLD["q4k_block"], np.uint8)
    out = O.dequantize(O.TYPE_Q4_K, blk, 256)
    for checks in GOLD["q4k_dequant_checks"].values():
        _slices(checks, out)
    assert np.array_equal(out, np.array(GOLD["q4k_dequant"], np.float32))


def test_dequantize_q6_k_known_answer():  # tests.lisp T2418-2450, T2324-2367
    blk = np.array(GOLD["q6k_block"], np.uint8)
    out = O.dequantize(O.TYPE_Q6_K, blk, 256)
    for checks in GOLD["q6k_dequant_checks"].values():
        _slices(checks, out)
    assert np.array_equal(out, np.array(GOLD["q6k_dequant"], np.float32))


@pytest.mark.parametrize("kind", ["q4k", "q6k"])
def test_fused_dot_matches_dequant_dot(kind):  # tests.lisp T2257-2288, T2290-2322
    tag = O.TYPE_Q4_K if kind == "q4k" else O.TYPE_Q6_K
    blk = np.array(GOLD[f"{kind}_block"], np.uint8)
    x = np.array(GOLD[f"{kind}_dot_x"], np.float32)
    expected = O.lib().or_dot_product(O._fptr(O.dequantize(tag, blk, 256)), O._fptr(x), 256)
    assert abs(O.dot_row(tag, blk, x) - expected) < GOLD["dot_tolerance"]


def test_silu_known_answer():  # tests.lisp T298-344
    assert abs(O.silu(2.0) - GOLD["silu_2"]) < GOLD["silu_tolerance"]
    assert O.silu(0.0) == 0.0
    assert O.sigmoid(0.0) == 0.5
    assert O.relu_squared(-3.0) == 0.0 and O.relu_squared(3.0) == 9.0


def test_fp16_decode_semantics():  # fp16-to-single-float, L716-733
    assert O.fp16_to_f32(0x3C00) == 1.0
    assert O.fp16_to_f32(0x0001) == 2.0 ** -24          # smallest subnormal
    assert O.fp16_to_f32(0x03FF) == 1023 * 2.0 ** -24   # largest subnormal
    assert O.fp16_to_f32(0x7BFF) == 65504.0
    assert math.copysign(1.0, O.fp16_to_f32(0x8000)) == -1.0
    for bad in (0x7C00, 0xFC00, 0x7E00):
        with pytest.raises(O.OracleError):
            O.fp16_to_f32(bad)
    for bits in range(0, 0x7C00, 7):
        assert O.fp16_to_f32(bits) == np.array([bits], np.uint16).view(np.float16).astype(np.float32)[0]


def test_fp16_special_in_block_is_an_error():
    blk = np.array(GOLD["q4k_block"], np.uint8)
    blk[1] = 0x7C  # d = +Inf
    with pytest.raises(O.OracleError):
        O.dot_row(O.TYPE_Q4_K, blk, np.ones(256, np.float32))


def test_scale_min_unpack_roundtrip():  # get-scale-min-k4-at, L4316-4336
    rng = np.random.default_rng(3)
    for _ in range(200):
        sc = rng.integers(0, 64, 8)
        mn = rng.integers(0, 64, 8)
        b = np.zeros(12, np.uint8)
        for j in range(4):
            b[j] = sc[j] | ((sc[j + 4] >> 4) << 6)
            b[j + 4] = mn[j] | ((mn[j + 4] >> 4) << 6)
            b[j + 8] = (sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4)
        for j in range(8):
            s, m = O.C.c_int(), O.C.c_int()
            O.lib().or_get_scale_min_k4(b.ctypes.data, j, O.C.byref(s), O.C.byref(m))
            assert (s.value, m.value) == (sc[j], mn[j])


def test_f16_encoder_is_round_to_nearest_even():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(0.001),
        rng.standard_normal(20000).astype(np.float32) * np.float32(100),
        (rng.random(5000).astype(np.float32) * np.float32(2.0 ** -14)),
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, 2.0 ** -25, 3 * 2.0 ** -26,
                  2.0 ** -24, 1.5 * 2.0 ** -24], np.float32)])
    want = vals.astype(np.float16).view(np.uint16)
    got = np.array([O.f32_to_f16(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, want)


def test_synthetic_distributions():
    blocks = O.synth_q4k(0, 5, 0, 4096, 0.02).reshape(-1, 144)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    assert np.all(d >= 0) and 0.012 < d.mean() < 0.02  # |N|*0.02 has mean 0.016
    nib = np.concatenate([blocks[:, 16:] & 15, blocks[:, 16:] >> 4]).ravel()
    assert abs(nib.mean() - 7.5) < 0.05
    q6 = O.synth_q6k(0, 7, 0, 4096, 0.001).reshape(-1, 210)
    d6 = q6[:, 208:210].copy().view(np.uint16).ravel()
    assert np.any((d6 & 0x7C00) == 0) and np.any(d6 != 0)  # some subnormal d
    x = O.synth_f32(0, 1, 0, 1 << 16, 1.0)
    assert abs(x.mean()) < 0.02 and abs(x.std() - 1.0) < 0.02
    # deterministic and position-addressable
    assert np.array_equal(O.synth_q4k(0, 5, 100, 3, 0.02), blocks[100:103].ravel())


def test_top_k_ties_keep_lower_index():  # select-top-k-logits-into, L5265-5292
    logits = np.array([1.0, 3.0, 3.0, 2.0, 3.0, -1.0], np.float32)
    idx, vals = O.select_top_k(logits, 4)
    assert idx.tolist() == [1, 2, 4, 3]
    assert vals.tolist() == [3.0, 3.0, 3.0, 2.0]


def _dequant_matrix(tag, data, ne0, rows):
    return O.dequantize(tag, data, ne0 * rows).reshape(rows, ne0).astype(np.float64)


def _np_moe(arch, H, x, router, bias, shg, gate, up, down, sh, k, scale, norm):
    """float64 restatement on dequantized weights (independent of the C dot order)."""
    logits = router @ x
    if bias is not None:
        logits = logits + bias
    order = np.argsort(-logits.astype(np.float32), kind="stable")[:k]
    w = 1.0 / (1.0 + np.exp(-logits[order]))
    if arch == 0 or norm:
        w = w / w.sum()
    if arch == 1:
        w = w * scale
    out = np.zeros(H)
    for e, wi in zip(order, w):
        if arch == 0:
            g = gate[e] @ x
            u = up[e] @ x
            h = g / (1 + np.exp(-g)) * u
        else:
            u = up[e] @ np.pad(x, (0, up[e].shape[1] - H))
            h = np.maximum(u, 0) ** 2
        out += wi * (down[e] @ np.pad(h, (0, down[e].shape[1] - h.size)))
    if arch == 0:
        g, u, d = sh
        sw = 1.0 / (1.0 + np.exp(-(shg @ x)))
        out += sw * (d @ ((g @ x) / (1 + np.exp(-(g @ x))) * (u @ x)))
    else:
        u, d = sh
        hh = np.maximum(u @ np.pad(x, (0, u.shape[1] - H)), 0) ** 2
        out += d @ np.pad(hh, (0, d.shape[1] - hh.size))
    return out, order


@pytest.mark.parametrize("arch", [0, 1])
@pytest.mark.parametrize("norm", [0, 1])
def test_moe_forward_matches_dequantized_float64(arch, norm):
    if arch == 0 and norm == 0:
        pytest.skip("qwen3next always normalises")
    seed, E, k = 11, 8, 3
    H = 256 if arch == 0 else 200          # nemotron hidden padded to 256 for K-quants
    HP = 256
    I = 256 if arch == 0 else 160          # intermediate; padded to 256 for the down rows
    IP = 256
    x = O.synth_f32(seed, 1, 0, H * 2, 1.0)
    router = O.synth_f32(seed, 2, 0, E * H, 0.02)
    bias = O.synth_f32(seed, 3, 0, E, 0.01) if arch == 1 else None
    shg = O.synth_f32(seed, 4, 0, H, 0.02)
    nb_in = HP // 256
    gate = O.synth_q4k(seed, 5, 0, E * I * nb_in, 0.02)
    up = O.synth_q4k(seed, 6, 0, E * I * nb_in, 0.02)
    down = O.synth_q6k(seed, 7, 0, E * H * (IP // 256), 0.001)
    sg = O.synth_q4k(seed, 8, 0, I * nb_in, 0.02)
    su = O.synth_q4k(seed, 9, 0, I * nb_in, 0.02)
    sd = O.synth_q6k(seed, 10, 0, H * (IP // 256), 0.001)
    L = O.MoeLayer()
    L.arch, L.hidden, L.top_k, L.weight_scale, L.weights_norm = arch, H, k, 1.0, norm
    L.router = O.make_tensor(O.TYPE_F32, router, H, E)
    L.router_bias = bias.ctypes.data if bias is not None else None
    L.shared_gate_inp = shg.ctypes.data
    L.gate_exps = O.make_tensor(O.TYPE_Q4_K, gate, HP, I, E)
    L.up_exps = O.make_tensor(O.TYPE_Q4_K, up, HP, I, E)
    L.down_exps = O.make_tensor(O.TYPE_Q6_K, down, IP, H, E)
    L.gate_shexp = O.make_tensor(O.TYPE_Q4_K, sg, HP, I)
    L.up_shexp = O.make_tensor(O.TYPE_Q4_K, su, HP, I)
    L.down_shexp = O.make_tensor(O.TYPE_Q6_K, sd, IP, H)
    out, sel, w = O.moe_forward(L, x, 2, k)
    R = router.reshape(E, H).astype(np.float64)
    G = _dequant_matrix(O.TYPE_Q4_K, gate, HP, E * I).reshape(E, I, HP)[:, :, :H]
    U = _dequant_matrix(O.TYPE_Q4_K, up, HP, E * I).reshape(E, I, HP)
    D = _dequant_matrix(O.TYPE_Q6_K, down, IP, E * H).reshape(E, H, IP)
    SG = _dequant_matrix(O.TYPE_Q4_K, sg, HP, I)[:, :H]
    SU = _dequant_matrix(O.TYPE_Q4_K, su, HP, I)
    SD = _dequant_matrix(O.TYPE_Q6_K, sd, IP, H)
    for t in range(2):
        xt = x[t * H:(t + 1) * H].astype(np.float64)
        if arch == 0:
            ref, order = _np_moe(0, H, xt, R, None, shg.astype(np.float64), G,
                                 U[:, :, :H], D, (SG, SU[:, :H], SD), k, 1.0, 1)
        else:
            ref, order = _np_moe(1, H, xt, R, bias.astype(np.float64), None, None,
                                 U, D, (SU, SD), k, 1.0, norm)
        assert sel[t].tolist() == order.tolist()
        err = np.max(np.abs(out[t * H:(t + 1) * H] - ref)) / np.max(np.abs(ref))
        assert err < 1e-5, err


def test_gemv_is_worker_count_independent():
    rows, K = 200, 512
    w = O.synth_q6k(1, 11, 0, rows * K // 256, 0.001)
    x = O.synth_f32(1, 1, 0, K, 1.0)
    O.set_workers(1)
    a = O.gemv(O.TYPE_Q6_K, w, K, rows, x)
    O.set_workers(7)
    b = O.gemv(O.TYPE_Q6_K, w, K, rows, x)
    O.set_workers(24)
    assert np.array_equal(a, b)
    # row-by-row equals the whole GEMV
    assert np.array_equal(a[5], np.float32(O.dot_row(O.TYPE_Q6_K, w[5 * 420:6 * 420], x)))


@pytest.mark.parametrize("kind", ["q5_0", "q8_0"])
def test_block32_dequantize_hand_blocks(kind):  # dequantize-q5-0 / -q8-0, L3965-4009
    from tests import block32 as B
    blk, want = B.hand_q5_0() if kind == "q5_0" else B.hand_q8_0()
    t = O.TYPE_Q5_0 if kind == "q5_0" else O.TYPE_Q8_0
    assert np.array_equal(O.dequantize(t, blk, 32), want)


@pytest.mark.parametrize("kind", ["q5_0", "q8_0"])
def test_block32_dot_matches_dequant_dot(kind):  # L4037-4094 against L3965-4009
    from tests import block32 as B
    t = O.TYPE_Q5_0 if kind == "q5_0" else O.TYPE_Q8_0
    blocks = B.random_blocks(t, 64, seed=3)
    x = np.random.default_rng(4).standard_normal(64 * 32).astype(np.float32)
    deq = O.dequantize(t, blocks, 64 * 32).astype(np.float64)
    ref = float(np.dot(deq, x))
    got = O.dot_row(t, blocks, x)
    assert abs(got - ref) <= 1e-4 * max(1.0, abs(ref))
    # rows of a tensor through the GEMV (sequential rows, L4582-4593)
    y = O.gemv(t, blocks, 1024, 2, x[:1024])
    assert abs(float(y[1]) - O.dot_row(t, blocks[(len(blocks) // 2):], x[:1024])) == 0.0


def test_block32_fp16_special_is_an_error():
    from tests import block32 as B
    blk, _ = B.hand_q8_0()
    blk[0:2] = np.frombuffer(np.array([np.inf], np.float16).tobytes(), np.uint8)
    with pytest.raises(O.OracleError):
        O.dequantize(O.TYPE_Q8_0, blk, 32)
