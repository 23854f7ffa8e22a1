"""GPU parity of the dense dequant-GEMV kernels against the CPU oracle, on the
same seeded GGUF blocks, through the C ABI."""
import json
import os

import numpy as np
import pytest

import llambda_b200 as LB
from llambda_b200 import configs as CF
from oracle import oracle as O
from tests.helpers import MAX_REL, host_tensor, max_rel

pytestmark = pytest.mark.gpu

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")))


def _oracle_gemv(t, data, ne0, ne1, x):
    x = np.asarray(x, np.float32).reshape(-1, ne0)
    return np.stack([O.gemv(t, data, ne0, ne1, xi) for xi in x])


@pytest.mark.parametrize("kind", ["q4k", "q6k"])
def test_known_answer_blocks(kind):  # tests.lisp T2257-2322
    t = LB.TYPE_Q4_K if kind == "q4k" else LB.TYPE_Q6_K
    blk = np.array(GOLD[f"{kind}_block"], np.uint8)
    x = np.array(GOLD[f"{kind}_dot_x"], np.float32)
    s = LB.ProjectionSession.from_tensor(t, 256, 1, blk)
    y = s.run(x)
    deq = np.array(GOLD[f"{kind}_dequant"], np.float32)
    assert abs(y[0] - float(np.dot(deq.astype(np.float64), x))) < GOLD["dot_tolerance"]
    assert abs(y[0] - O.dot_row(t, blk, x)) < GOLD["dot_tolerance"]
    # dequantized weights through the GEMV: unit vectors pick single weights
    eye = np.eye(256, dtype=np.float32)[[0, 31, 32, 63, 64, 96, 200, 255]]
    got = s.run_batch(eye)[:, 0]
    assert np.array_equal(got, deq[[0, 31, 32, 63, 64, 96, 200, 255]])


@pytest.mark.parametrize("type_tag,K,rows", [
    (LB.TYPE_Q4_K, 256, 7), (LB.TYPE_Q4_K, 512, 33), (LB.TYPE_Q4_K, 2048, 512),
    (LB.TYPE_Q4_K, 2816, 100), (LB.TYPE_Q4_K, 4096, 300),
    (LB.TYPE_Q6_K, 256, 5), (LB.TYPE_Q6_K, 512, 2048), (LB.TYPE_Q6_K, 768, 77),
    (LB.TYPE_Q6_K, 2048, 129), (LB.TYPE_Q6_K, 3840, 64), (LB.TYPE_Q6_K, 4096, 300),
    (LB.TYPE_Q6_K, 2048, 160), (LB.TYPE_Q6_K, 4096, 96),  # K slices of 8 super-blocks
])
@pytest.mark.parametrize("tokens", [1, 2, 3, 8, 11])
def test_gemv_matches_oracle(type_tag, K, rows, tokens):
    dscale = CF.Q4K_DSCALE if type_tag == LB.TYPE_Q4_K else CF.Q6K_DSCALE
    w = host_tensor(type_tag, K, rows, 1, 7 + K, 11, dscale)
    x = O.synth_f32(3, 1, 0, tokens * K, 1.0).reshape(tokens, K)
    s = LB.ProjectionSession.from_tensor(type_tag, K, rows, w)
    y = s.run_batch(x)
    r = _oracle_gemv(type_tag, w, K, rows, x)
    assert max_rel(y, r) < MAX_REL
    assert max_rel(y, r) < 1e-5  # what the kernels actually achieve
    if tokens == 1:
        assert np.array_equal(s.run(x[0]), y[0])


def test_f32_gemv_matches_oracle():
    K, rows = 2048, 513
    w = O.synth_f32(1, 2, 0, K * rows, 0.02)
    x = O.synth_f32(1, 1, 0, 3 * K, 1.0).reshape(3, K)
    s = LB.ProjectionSession.from_tensor(LB.TYPE_F32, K, rows, w)
    y = s.run_batch(x)
    r = np.stack([O.gemv(O.TYPE_F32, w, K, rows, xi) for xi in x])
    assert max_rel(y, r) < 1e-5


def test_expert_rows_match_oracle():
    # gguf-model-expert-matrix-vector-multiply-into, L4951-4971
    K, rows, E = 512, 64, 5
    w = host_tensor(LB.TYPE_Q6_K, K, rows, E, 5, 7, CF.Q6K_DSCALE)
    x = O.synth_f32(5, 1, 0, K, 1.0)
    s = LB.ProjectionSession.from_tensor(LB.TYPE_Q6_K, K, rows, w, ne2=E)
    for e in (0, 3, 4):
        r = O.gemv(O.TYPE_Q6_K, w, K, rows * E, x, start_row=e * rows, row_count=rows)
        assert max_rel(s.run_expert(e, x), r) < 1e-5
    with pytest.raises(LB.LlambdaCudaError, match="out of range"):
        s.run_expert(E, x)


def test_count_mismatch_and_bad_scales_are_errors():
    blk = np.array(GOLD["q4k_block"], np.uint8)
    s = LB.ProjectionSession.from_tensor(LB.TYPE_Q4_K, 256, 1, blk)
    with pytest.raises(LB.LlambdaCudaError, match="element count"):
        s.run_into(np.empty(2, np.float32), np.ones(256, np.float32))
    bad = blk.copy()
    bad[3] = 0x7C  # dmin = +Inf: fp16-to-single-float rejects it (L727-728)
    with pytest.raises(LB.LlambdaCudaError, match="fp16"):
        LB.ProjectionSession.from_tensor(LB.TYPE_Q4_K, 256, 1, bad)
    with pytest.raises(LB.LlambdaCudaError, match="multiple of 256"):
        LB.ProjectionSession.from_tensor(LB.TYPE_Q4_K, 200, 1, blk)


def test_device_generator_matches_host_generator():
    import torch
    for t, first, n, scale in [(LB.TYPE_Q4_K, 12345, 1000, 0.02), (LB.TYPE_Q6_K, 777, 1001, 0.001),
                               (LB.TYPE_F32, 99, 4097, 0.02)]:
        nbytes = n * {LB.TYPE_Q4_K: 144, LB.TYPE_Q6_K: 210, LB.TYPE_F32: 4}[t]
        dev = torch.empty(nbytes + 256, dtype=torch.uint8, device="cuda")
        LB.synth_fill_device(t, 42, 6, first, n, scale, dev)
        torch.cuda.synchronize()
        got = dev[:nbytes].cpu().numpy()
        if t == LB.TYPE_Q4_K:
            want = O.synth_q4k(42, 6, first, n, scale)
        elif t == LB.TYPE_Q6_K:
            want = O.synth_q6k(42, 6, first, n, scale)
        else:
            want = O.synth_f32(42, 6, first, n, scale).view(np.uint8)
        assert np.array_equal(got, want)


def test_export_file_session(tmp_path):
    from llambda_b200.accelerator import write_projection_file
    K, rows = 512, 40
    w = host_tensor(LB.TYPE_Q4_K, K, rows, 1, 9, 5, CF.Q4K_DSCALE)
    path = str(tmp_path / "proj.llbcuda")
    write_projection_file(path, LB.TYPE_Q4_K, K, rows, 1, w)
    s = LB.ProjectionSession.from_file(path)
    assert (s.input_element_count, s.output_element_count) == (K, rows)
    x = O.synth_f32(9, 1, 0, K, 1.0)
    assert max_rel(s.run(x), O.gemv(O.TYPE_Q4_K, w, K, rows, x)) < 1e-5


@pytest.mark.parametrize("tokens", [1, 8])
def test_config1_full_size(tokens):
    c = CF.CONFIG1
    w = host_tensor(c.type, c.cols, c.rows, 1, 0, CF.S_DENSE, c.dscale)
    x = O.synth_f32(0, CF.S_ACT, 0, tokens * c.cols, 1.0).reshape(tokens, c.cols)
    s = LB.ProjectionSession.from_tensor(c.type, c.cols, c.rows, w)
    y = s.run_batch(x)
    assert max_rel(y, _oracle_gemv(c.type, w, c.cols, c.rows, x)) < 1e-5


@pytest.mark.parametrize("tokens", [1, 8])
def test_config2_full_size(tokens):
    c = CF.CONFIG2
    w = host_tensor(c.type, c.cols, c.rows, 1, 0, CF.S_DENSE, c.dscale)
    x = O.synth_f32(0, CF.S_ACT, 0, tokens * c.cols, 1.0).reshape(tokens, c.cols)
    s = LB.ProjectionSession.from_tensor(c.type, c.cols, c.rows, w)
    y = s.run_batch(x)
    rows = np.arange(0, c.rows, 97)  # oracle on a row sample keeps the test short
    r = np.stack([[O.dot_row(c.type, w[i * 3360:(i + 1) * 3360], xi) for i in rows] for xi in x])
    assert max_rel(y[:, rows], r) < 1e-5


@pytest.mark.parametrize("kind", ["q5_0", "q8_0"])
@pytest.mark.parametrize("K,rows,tokens", [(32, 5, 1), (1856, 300, 1), (2688, 129, 3),
                                           (3712, 64, 9), (6144, 40, 2)])
def test_block32_gemv_matches_oracle(kind, K, rows, tokens):
    """Q5_0 / Q8_0 projection sessions (dot-product-with-q5-0/-q8-0-tensor-data,
    L4037-4094) against the oracle: Nemotron-H widths that are not multiples
    of 256, a single block, and more tokens than one launch takes."""
    from tests import block32 as B
    t = LB.TYPE_Q5_0 if kind == "q5_0" else LB.TYPE_Q8_0
    blocks = B.random_blocks(t, rows * K // 32, seed=K + rows)
    x = np.random.default_rng(K).standard_normal((tokens, K)).astype(np.float32)
    s = LB.ProjectionSession.from_tensor(t, K, rows, blocks)
    y = s.run_batch(x) if tokens > 1 else s.run(x[0])[None]
    ref = _oracle_gemv(t, blocks, K, rows, x)
    assert max_rel(y, ref) < MAX_REL
    assert max_rel(y, ref) < 1e-5


@pytest.mark.parametrize("kind", ["q5_0", "q8_0"])
def test_block32_hand_blocks_through_the_gemv(kind):
    from tests import block32 as B
    t = LB.TYPE_Q5_0 if kind == "q5_0" else LB.TYPE_Q8_0
    blk, want = B.hand_q5_0() if kind == "q5_0" else B.hand_q8_0()
    s = LB.ProjectionSession.from_tensor(t, 32, 1, blk)
    got = s.run_batch(np.eye(32, dtype=np.float32))[:, 0]  # unit vectors pick the weights
    assert np.array_equal(got, want)


def test_block32_rejects_fp16_specials():
    from tests import block32 as B
    blk, _ = B.hand_q8_0()
    blk[0:2] = np.frombuffer(np.array([np.nan], np.float16).tobytes(), np.uint8)
    with pytest.raises(LB.LlambdaCudaError, match="Inf/NaN"):
        LB.ProjectionSession.from_tensor(LB.TYPE_Q8_0, 32, 1, blk)


def test_page_locked_buffers_match_pageable():
    """Page-locked input/output buffers are copied by DMA without staging;
    results equal the pageable path's."""
    import torch
    t, K, rows = LB.TYPE_Q4_K, 2048, 96
    w = host_tensor(t, K, rows, 1, 3, 11, CF.Q4K_DSCALE)
    x = np.random.default_rng(3).standard_normal((3, K)).astype(np.float32)
    s = LB.ProjectionSession.from_tensor(t, K, rows, w)
    want = s.run_batch(x)
    xp = torch.from_numpy(x.copy()).pin_memory()
    out = torch.empty((3, rows), dtype=torch.float32, pin_memory=True)
    LB._native._check(LB.lib().llambda_cuda_session_run_batch(
        s._h, LB._native._fptr(xp.numpy()), 3, LB._native._fptr(out.numpy())))
    assert np.array_equal(out.numpy(), want)
