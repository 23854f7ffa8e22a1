"""CPU oracle: the Q5_K row dot and dequantizer (dot-product-with-q5-k-
tensor-data L4387-4441, dequantize-q5-k L6861-6917) and nemotron's latent
projections (nemotron-h-moe-ffn-into L5845-5855, L5883-5887, L5933-5938).
The reference's tests hold no Q5_K blocks and no latent layer, so the oracle
is pinned by hand-built blocks written out from the format, by the
reference's own summation order restated independently in numpy, and by a
float64 restatement of the latent block on dequantized weights."""
import numpy as np
import pytest

from oracle import oracle as O
from oracle.layers import random_q5k
from tests import kquant5 as K5


def test_q5k_dequantize_hand_block():
    blk, want = K5.hand_q5k()
    assert np.array_equal(O.dequantize(O.TYPE_Q5_K, blk, 256), want)


def test_q5k_dot_follows_the_reference_order():
    blocks = random_q5k(4, seed=5, stream=1, dscale=0.02)
    x = np.random.default_rng(6).standard_normal(4 * 256).astype(np.float32)
    assert np.float32(O.dot_row(O.TYPE_Q5_K, blocks, x)) == K5.dot_in_order(blocks, x)


def test_q5k_dot_matches_dequant_dot():  # as tests.lisp T2257-2322 do for Q4_K / Q6_K
    blocks = random_q5k(16, seed=7, stream=2, dscale=0.02)
    x = np.random.default_rng(8).standard_normal(16 * 256).astype(np.float32)
    ref = float(np.dot(O.dequantize(O.TYPE_Q5_K, blocks, 16 * 256).astype(np.float64), x))
    assert abs(O.dot_row(O.TYPE_Q5_K, blocks, x) - ref) <= 1e-4 * max(1.0, abs(ref))


def test_q5k_gemv_rows_split_over_workers():
    rows, K = 130, 512
    w = random_q5k(rows * K // 256, seed=9, stream=3, dscale=0.02)
    x = O.synth_f32(2, 1, 0, K, 1.0)
    O.set_workers(1)
    a = O.gemv(O.TYPE_Q5_K, w, K, rows, x)
    O.set_workers(5)
    b = O.gemv(O.TYPE_Q5_K, w, K, rows, x)
    assert np.array_equal(a, b)
    assert a[7] == np.float32(O.dot_row(O.TYPE_Q5_K, w[7 * 352:8 * 352], x))


def test_q5k_fp16_special_is_an_error():
    blk, _ = K5.hand_q5k()
    blk[2:4] = np.frombuffer(np.array([np.nan], np.float16).tobytes(), np.uint8)
    with pytest.raises(O.OracleError):
        O.dequantize(O.TYPE_Q5_K, blk, 256)


def _deq(tag, data, ne0, rows):
    if tag == O.TYPE_F32:
        return np.asarray(data, np.float64).reshape(rows, ne0)
    return O.dequantize(tag, data, ne0 * rows).reshape(rows, ne0).astype(np.float64)


@pytest.mark.parametrize("lat_type", [O.TYPE_Q4_K, O.TYPE_Q5_K, O.TYPE_Q6_K, O.TYPE_F32])
def test_latent_moe_matches_dequantized_float64(lat_type):
    seed, E, k, H, HP, L, I, IP, Ish = 5, 8, 3, 200, 256, 256, 160, 256, 300
    ISP = 512
    rng_x = O.synth_f32(seed, 1, 0, H * 2, 1.0)
    router = O.synth_f32(seed, 2, 0, E * H, 0.02)
    bias = O.synth_f32(seed, 3, 0, E, 0.01)
    up = O.synth_q4k(seed, 6, 0, E * I, 0.02)            # [E][I][L]
    down = O.synth_q6k(seed, 7, 0, E * L * (IP // 256), 0.001)  # [E][L][IP]
    su = O.synth_q4k(seed, 9, 0, Ish * (HP // 256), 0.02)
    sd = O.synth_q6k(seed, 10, 0, H * (ISP // 256), 0.001)
    ld_w = H if lat_type == O.TYPE_F32 else HP
    if lat_type == O.TYPE_F32:
        ld = O.synth_f32(seed, 12, 0, L * H, 0.05)
        lu = O.synth_f32(seed, 13, 0, H * L, 0.05)
    elif lat_type == O.TYPE_Q5_K:
        ld = random_q5k(L * HP // 256, seed, 12, 0.02)
        lu = random_q5k(H * L // 256, seed, 13, 0.02)
    else:
        syn = O.synth_q4k if lat_type == O.TYPE_Q4_K else O.synth_q6k
        ds = 0.02 if lat_type == O.TYPE_Q4_K else 0.001
        ld = syn(seed, 12, 0, L * HP // 256, ds)
        lu = syn(seed, 13, 0, H * L // 256, ds)
    Lyr = O.MoeLayer()
    Lyr.arch, Lyr.hidden, Lyr.top_k, Lyr.weight_scale, Lyr.weights_norm = 1, H, k, 2.5, 1
    Lyr.router = O.make_tensor(O.TYPE_F32, router, H, E)
    Lyr.router_bias = bias.ctypes.data
    Lyr.up_exps = O.make_tensor(O.TYPE_Q4_K, up, L, I, E)
    Lyr.down_exps = O.make_tensor(O.TYPE_Q6_K, down, IP, L, E)
    Lyr.up_shexp = O.make_tensor(O.TYPE_Q4_K, su, HP, Ish)
    Lyr.down_shexp = O.make_tensor(O.TYPE_Q6_K, sd, ISP, H)
    Lyr.latent_down = O.make_tensor(lat_type, ld, ld_w, L)
    Lyr.latent_up = O.make_tensor(lat_type, lu, L, H)
    out, sel, w = O.moe_forward(Lyr, rng_x, 2, k)
    R = router.reshape(E, H).astype(np.float64)
    U = _deq(O.TYPE_Q4_K, up, L, E * I).reshape(E, I, L)
    D = _deq(O.TYPE_Q6_K, down, IP, E * L).reshape(E, L, IP)
    SU = _deq(O.TYPE_Q4_K, su, HP, Ish)
    SD = _deq(O.TYPE_Q6_K, sd, ISP, H)
    LDm = _deq(lat_type, ld, ld_w, L)[:, :H]
    LUm = _deq(lat_type, lu, L, H)
    for t in range(2):
        x = rng_x[t * H:(t + 1) * H].astype(np.float64)
        logits = R @ x + bias
        order = np.argsort(-logits.astype(np.float32), kind="stable")[:k]
        wt = 1.0 / (1.0 + np.exp(-logits[order]))
        wt = wt / wt.sum() * 2.5
        xl = LDm @ x
        mo = np.zeros(L)
        for e, wi in zip(order, wt):
            h = np.maximum(U[e] @ xl, 0) ** 2
            mo += wi * (D[e] @ np.pad(h, (0, IP - I)))
        hh = np.maximum(SU @ np.pad(x, (0, HP - H)), 0) ** 2
        ref = LUm @ mo + SD @ np.pad(hh, (0, ISP - Ish))
        assert sel[t].tolist() == order.tolist()
        err = np.max(np.abs(out[t * H:(t + 1) * H] - ref)) / np.max(np.abs(ref))
        assert err < 1e-5, err
