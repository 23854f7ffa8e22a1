"""GPU parity of the MoE feed-forward layer (qwen3next-moe-into, L5321-5426;
nemotron-h-moe-ffn-into, L5827-5949) against the CPU oracle on identical
seeded tensors, through the C ABI."""
import dataclasses

import numpy as np
import pytest

import llambda_b200 as LB
from llambda_b200 import configs as CF
from oracle import oracle as O
from tests.helpers import MAX_REL, gpu_tensors, host_layer, max_rel, oracle_layer

pytestmark = pytest.mark.gpu

SMALL_QWEN = dataclasses.replace(CF.CONFIG3, name="small_qwen", hidden=512, experts=24, top_k=5,
                                 inter=256, inter_sh=512)
SMALL_NEMO = dataclasses.replace(CF.CONFIG4, name="small_nemo", hidden=400, experts=16, top_k=3,
                                 inter=200, inter_sh=300)


def _session(cfg, tensors, max_tokens, **kw):
    return LB.MoeSession.create(cfg.arch, cfg.hidden, cfg.top_k, gpu_tensors(tensors),
                                weight_scale=cfg.weight_scale, weights_norm=cfg.weights_norm,
                                max_tokens=max_tokens, **kw)


def _check_selection(cfg, tensors, x, sel_gpu, sel_ref):
    """Selected experts must be identical wherever the k-th/(k+1)-th score
    margin exceeds 1e-6."""
    t, ne0, ne1, _, router = tensors["ffn_gate_inp"]
    bias = tensors["exp_probs_b.bias"][4] if "exp_probs_b.bias" in tensors else None
    checked = 0
    for i, xi in enumerate(x):
        logits = O.gemv(O.TYPE_F32, router, ne0, ne1, xi)
        if bias is not None:
            logits = logits + bias
        srt = np.sort(logits)[::-1]
        k = cfg.top_k
        if k < srt.size and srt[k - 1] - srt[k] <= 1e-6:
            continue
        assert set(sel_gpu[i].tolist()) == set(sel_ref[i].tolist())
        gaps = -np.diff(srt[:k])
        if np.all(gaps > 1e-6):
            assert sel_gpu[i].tolist() == sel_ref[i].tolist()
        checked += 1
    assert checked >= max(1, len(x) // 2)


@pytest.mark.parametrize("cfg", [SMALL_QWEN, SMALL_NEMO], ids=lambda c: c.name)
@pytest.mark.parametrize("tokens", [1, 3, 9, 33])
def test_small_layer_matches_oracle(cfg, tokens):
    tensors = host_layer(cfg, seed=5)
    x = O.synth_f32(5, CF.S_ACT, 0, tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)
    ref, sel_ref, w_ref = O.moe_forward(oracle_layer(cfg, tensors), x, tokens, cfg.top_k)
    s = _session(cfg, tensors, max_tokens=64)
    out, sel, w = s.run(x, with_routing=True)
    _check_selection(cfg, tensors, x, sel, sel_ref)
    same = np.all(sel == sel_ref, axis=1)
    assert same.mean() > 0.5
    assert max_rel(out[same], ref[same]) < MAX_REL
    assert max_rel(out[same], ref[same]) < 1e-5
    assert max_rel(w[same], w_ref[same]) < 1e-6


@pytest.mark.parametrize("cfg", [SMALL_QWEN, SMALL_NEMO], ids=lambda c: c.name)
def test_topk_ties_take_lower_index(cfg):
    """Equal scores rank by lower expert index, as the reference's repeated
    strict-> scan (select-top-k-logits-into, L5265-5292) finds them: experts
    2j and 2j+1 get identical router rows, and a block of experts gets zero
    rows (scores +0.0 / -0.0, which compare equal)."""
    cfg = dataclasses.replace(cfg, experts=32, top_k=6)
    tensors = host_layer(cfg, seed=11)
    t, ne0, ne1, ne2, router = tensors["ffn_gate_inp"]
    r = router.reshape(ne1, ne0).copy()
    r[1::2] = r[0::2]
    r[20:26] = 0.0
    tensors["ffn_gate_inp"] = (t, ne0, ne1, ne2, np.ascontiguousarray(r.reshape(-1)))
    if "exp_probs_b.bias" in tensors:  # keep the pairs tied after the bias
        tb, b0, b1, b2, bias = tensors["exp_probs_b.bias"]
        b = bias.copy()
        b[1::2] = b[0::2]
        b[20:26] = 0.0
        tensors["exp_probs_b.bias"] = (tb, b0, b1, b2, b)
    tokens = 12
    x = O.synth_f32(11, CF.S_ACT, 0, tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)
    ref, sel_ref, w_ref = O.moe_forward(oracle_layer(cfg, tensors), x, tokens, cfg.top_k)
    _, sel, w = _session(cfg, tensors, max_tokens=16).run(x, with_routing=True)
    bias = tensors["exp_probs_b.bias"][4] if "exp_probs_b.bias" in tensors else 0.0
    checked = 0
    for i in range(tokens):
        scores = O.gemv(O.TYPE_F32, tensors["ffn_gate_inp"][4], ne0, ne1, x[i]) + bias
        uniq = np.unique(scores)[::-1][: cfg.top_k + 2]
        if uniq.size > 1 and np.min(-np.diff(uniq)) <= 1e-5:
            continue  # distinct scores too close for an exact order
        assert sel[i].tolist() == sel_ref[i].tolist()
        for j in range(cfg.top_k - 1):  # tied neighbours in index order
            if scores[sel[i][j]] == scores[sel[i][j + 1]]:
                assert sel[i][j] < sel[i][j + 1]
        checked += 1
    assert checked >= tokens // 2


@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("scale", [1.0, 2.5])
def test_nemotron_weight_policy(norm, scale):
    cfg = dataclasses.replace(SMALL_NEMO, weights_norm=norm, weight_scale=scale)
    tensors = host_layer(cfg, seed=8)
    x = O.synth_f32(8, CF.S_ACT, 0, 4 * cfg.hidden, 1.0).reshape(4, cfg.hidden)
    ref, sel_ref, w_ref = O.moe_forward(oracle_layer(cfg, tensors), x, 4, cfg.top_k)
    out, sel, w = _session(cfg, tensors, 8).run(x, with_routing=True)
    same = np.all(sel == sel_ref, axis=1)
    assert same.all()
    assert max_rel(w, w_ref) < 1e-6
    assert max_rel(out, ref) < 1e-5


def test_norm_and_residual():
    cfg = SMALL_QWEN
    tensors = host_layer(cfg, seed=3)
    nw = O.synth_f32(3, 30, 0, cfg.hidden, 1.0)
    x = O.synth_f32(3, CF.S_ACT, 0, 5 * cfg.hidden, 3.0).reshape(5, cfg.hidden)
    ref, sel_ref, _ = O.moe_forward(oracle_layer(cfg, tensors, input_norm=nw, eps=1e-6,
                                                 residual=True), x, 5, cfg.top_k)
    out, sel, _ = _session(cfg, tensors, 8, input_norm=nw, norm_epsilon=1e-6,
                           add_residual=True).run(x, with_routing=True)
    same = np.all(sel == sel_ref, axis=1)
    assert same.mean() > 0.5
    assert max_rel(out[same], ref[same]) < 1e-5


def test_repeated_host_calls_replay_one_graph():
    """Host-buffer calls of one token count run eagerly once, are then captured
    into a CUDA graph and replayed: every call must see its own input."""
    cfg = SMALL_QWEN
    tensors = host_layer(cfg, seed=5)
    xs = [O.synth_f32(5, CF.S_ACT, i, 6 * cfg.hidden, 1.0).reshape(6, cfg.hidden)
          for i in range(3)]
    refs = [O.moe_forward(oracle_layer(cfg, tensors), x, 6, cfg.top_k)[0] for x in xs]
    s = _session(cfg, tensors, 8)
    try:
        for i in (0, 1, 1, 2, 0, 2):  # eager, capture, replays with new inputs
            out = s.run(xs[i])
            assert max_rel(out, refs[i]) < 1e-5, i
        out3 = s.run(xs[0][:3])  # another token count: eager, then its own graph
        assert max_rel(out3, O.moe_forward(oracle_layer(cfg, tensors), xs[0][:3], 3,
                                           cfg.top_k)[0]) < 1e-5
        assert max_rel(s.run(xs[1]), refs[1]) < 1e-5
        dest = np.empty_like(xs[2])  # the run-into form writes the caller's buffer
        assert s.run_into(dest, xs[2]) is dest
        assert max_rel(dest, refs[2]) < 1e-5
    finally:
        s.close()


def test_expert_parallel_split_sums_to_full():
    """Expert-parallel shards (owned expert ranges, shared expert on one
    shard) add up to the whole layer."""
    cfg = SMALL_QWEN
    tensors = host_layer(cfg, seed=4)
    x = O.synth_f32(4, CF.S_ACT, 0, 7 * cfg.hidden, 1.0).reshape(7, cfg.hidden)
    full = _session(cfg, tensors, 8).run(x)
    parts = [_session(cfg, tensors, 8, expert_range=(a, b), shared_here=(a == 0)).run(x)
             for a, b in ((0, 10), (10, 17), (17, cfg.experts))]
    assert max_rel(sum(parts), full) < 1e-5


def test_non_positive_weight_sum_is_an_error():
    # nemotron with norm on and a weight scale; all-zero router with a bias of
    # -inf-like values makes every sigmoid 0 -> the reference errors (L5903-5905)
    cfg = dataclasses.replace(SMALL_NEMO, weights_norm=True)
    tensors = host_layer(cfg, seed=2)
    t = list(tensors["exp_probs_b.bias"])
    t[4] = np.full(cfg.experts, -1e30, np.float32)
    tensors["exp_probs_b.bias"] = tuple(t)
    x = O.synth_f32(2, CF.S_ACT, 0, cfg.hidden, 1.0)
    with pytest.raises(O.OracleError):
        O.moe_forward(oracle_layer(cfg, tensors), x, 1, cfg.top_k)
    with pytest.raises(LB.LlambdaCudaError, match="non-positive"):
        _session(cfg, tensors, 2).run(x)


@pytest.fixture
def decode_kernels_only():
    """Every batch through the fp32 decode kernels (no bf16 prefill path)."""
    old = LB.prefill_min_tokens()
    LB.set_prefill_min_tokens(1 << 30)
    yield
    LB.set_prefill_min_tokens(old)


@pytest.mark.parametrize("tokens", [1, 16, 512])  # decode and a prefill batch (config 3)
def test_config3_full_layer(tokens, decode_kernels_only):
    cfg = CF.CONFIG3
    tensors = host_layer(cfg, seed=0)
    x = O.synth_f32(0, CF.S_ACT, 0, tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)
    ref, sel_ref, w_ref = O.moe_forward(oracle_layer(cfg, tensors), x, tokens, cfg.top_k)
    out, sel, w = _session(cfg, tensors, max(64, tokens)).run(x, with_routing=True)
    _check_selection(cfg, tensors, x, sel, sel_ref)
    same = np.all(sel == sel_ref, axis=1)
    assert max_rel(out[same], ref[same]) < MAX_REL
    assert max_rel(out[same], ref[same]) < 1e-5


@pytest.mark.parametrize("tokens", [1, 64, 1024])  # decode and a prefill batch (config 4)
def test_config4_full_layer(tokens, decode_kernels_only):
    cfg = CF.CONFIG4
    tensors = host_layer(cfg, seed=0)
    x = O.synth_f32(0, CF.S_ACT, 0, tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)
    ref, sel_ref, w_ref = O.moe_forward(oracle_layer(cfg, tensors), x, tokens, cfg.top_k)
    out, sel, w = _session(cfg, tensors, max(64, tokens)).run(x, with_routing=True)
    _check_selection(cfg, tensors, x, sel, sel_ref)
    same = np.all(sel == sel_ref, axis=1)
    assert max_rel(out[same], ref[same]) < MAX_REL
    assert max_rel(out[same], ref[same]) < 1e-5


def test_page_locked_host_buffers_are_copied_directly():
    """Page-locked caller buffers skip the staging copies (DMA straight from
    and into them); the bytes equal those of pageable buffers, on repeated
    calls (the second one replays a captured graph) and alternating outputs."""
    import torch
    cfg = SMALL_QWEN
    tensors = host_layer(cfg, seed=9)
    x = O.synth_f32(9, CF.S_ACT, 0, 7 * cfg.hidden, 1.0).reshape(7, cfg.hidden)
    s = _session(cfg, tensors, max_tokens=8)
    want = s.run(x)
    xp = torch.from_numpy(x.copy()).pin_memory()
    outs = [torch.empty(x.shape, dtype=torch.float32, pin_memory=True) for _ in range(2)]
    for i in range(4):
        got = s.run_into(outs[i % 2].numpy(), xp.numpy())
        assert np.array_equal(got, want)
    assert s.status() == 0
    s.close()


@pytest.mark.parametrize("arch", [0, 1], ids=["qwen3next_dense", "nemotron_dense"])
@pytest.mark.parametrize("tokens", [1, 5, 130])
def test_dense_ffn_as_one_expert(arch, tokens):
    """A dense FFN (qwen3next-dense-ffn-into, L5294-5319: down(silu(gate x) * up x);
    nemotron: down(relu(up x)^2)) through the MoE session as one expert with top-1:
    its routing weight normalises to exactly 1 (sigmoid(l) / sigmoid(l)), so the
    layer output is the dense FFN.  fp32 path up to 129 tokens; 130 tokens take
    the bf16 prefill path (tolerance 2e-2)."""
    H, I = 1024, 512
    rng_seed = 40 + arch
    tensors = {
        "ffn_gate_inp": (O.TYPE_F32, H, 1, 1, O.synth_f32(rng_seed, 1, 0, H, 0.02)),
        "ffn_up_exps": (LB.TYPE_Q4_K, H, I, 1, O.synth_q4k(rng_seed, 2, 0, H * I // 256, CF.Q4K_DSCALE)),
        "ffn_down_exps": (LB.TYPE_Q6_K, I, H, 1, O.synth_q6k(rng_seed, 3, 0, I * H // 256, CF.Q6K_DSCALE)),
    }
    if arch == 0:
        tensors["ffn_gate_exps"] = (LB.TYPE_Q4_K, H, I, 1,
                                    O.synth_q4k(rng_seed, 4, 0, H * I // 256, CF.Q4K_DSCALE))
    x = O.synth_f32(rng_seed, CF.S_ACT, 0, tokens * H, 1.0).reshape(tokens, H)
    ref = np.empty_like(x)
    for t in range(tokens):
        up = O.gemv(LB.TYPE_Q4_K, tensors["ffn_up_exps"][4], H, I, x[t])
        if arch == 0:
            gate = O.gemv(LB.TYPE_Q4_K, tensors["ffn_gate_exps"][4], H, I, x[t])
            h = np.array([np.float32(O.silu(float(g))) * np.float32(u) for g, u in zip(gate, up)],
                         np.float32)
        else:
            h = np.array([O.relu_squared(float(u)) for u in up], np.float32)
        ref[t] = O.gemv(LB.TYPE_Q6_K, tensors["ffn_down_exps"][4], I, H, h)
    s = LB.MoeSession.create(arch, H, 1, gpu_tensors(tensors), weights_norm=True,
                             max_tokens=max(64, tokens))
    out = s.run(x)
    assert s.status() == 0
    s.close()
    tol = 2e-2 if tokens >= LB.prefill_min_tokens() else 1e-5
    assert max_rel(out, ref) < tol
