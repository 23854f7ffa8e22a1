"""GPU parity of the prefill path: MoE batches of at least
prefill_min_tokens() tokens run their expert products as bf16 grouped GEMMs
on the tcgen05 tensor cores (weights decoded once per 128-row block and 64
tokens).  Checked against the CPU oracle (qwen3next-moe-into, L5321-5426;
nemotron-h-moe-ffn-into, L5827-5949) on identical seeded tensors, through the
C ABI, with the bf16 tolerance of 2e-2 relative; the routing is unchanged and
must select the same experts as the oracle."""
import dataclasses

import numpy as np
import pytest

import llambda_b200 as LB
from llambda_b200 import configs as CF
from oracle import oracle as O
from tests.helpers import gpu_tensors, host_layer, max_rel, oracle_layer
from tests.test_gpu_moe import _check_selection

pytestmark = pytest.mark.gpu

PREFILL_MAX_REL = 2e-2  # bf16 operands, fp32 sums

# Odd shapes: hidden 400 -> k_in 512 (zero padding), inter 200 -> down K 256
# (half of the last row block invalid), H = 400 = 3 x 128 + 16 (a partial down
# row block), Q6_K rows of 210 / 420 bytes (2-byte-aligned super-blocks).
SMALL_QWEN = dataclasses.replace(CF.CONFIG3, name="pf_qwen", hidden=512, experts=24, top_k=5,
                                 inter=256, inter_sh=512)
SMALL_NEMO = dataclasses.replace(CF.CONFIG4, name="pf_nemo", hidden=400, experts=16, top_k=3,
                                 inter=200, inter_sh=300)


@pytest.fixture
def prefill_from(request):
    old = LB.prefill_min_tokens()
    yield LB.set_prefill_min_tokens
    LB.set_prefill_min_tokens(old)


def _run(cfg, tensors, x, max_tokens, **kw):
    s = LB.MoeSession.create(cfg.arch, cfg.hidden, cfg.top_k, gpu_tensors(tensors),
                             weight_scale=cfg.weight_scale, weights_norm=cfg.weights_norm,
                             max_tokens=max_tokens, **kw)
    out, sel, w = s.run(x, with_routing=True)
    assert s.status() == 0
    return s, out, sel, w


@pytest.mark.parametrize("cfg", [SMALL_QWEN, SMALL_NEMO], ids=lambda c: c.name)
@pytest.mark.parametrize("tokens", [64, 130, 300])
def test_small_prefill_matches_oracle(cfg, tokens, prefill_from):
    prefill_from(64)
    tensors = host_layer(cfg, seed=7)
    x = O.synth_f32(7, CF.S_ACT, 0, tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)
    ref, sel_ref, _ = O.moe_forward(oracle_layer(cfg, tensors), x, tokens, cfg.top_k)
    s, out, sel, _ = _run(cfg, tensors, x, max_tokens=tokens)
    s.close()
    _check_selection(cfg, tensors, x, sel, sel_ref)
    same = np.all(sel == sel_ref, axis=1)
    assert same.mean() > 0.5
    assert np.isfinite(out).all()
    assert max_rel(out[same], ref[same]) < PREFILL_MAX_REL


# config 3 at T=2048 is the config-5 prefill batch: the largest workspace
# (T*k = 20480 grouped rows), tile lists and router slices the bench reaches
@pytest.mark.parametrize("cfg,tokens", [(CF.CONFIG3, 512), (CF.CONFIG4, 1024),
                                        (CF.CONFIG3, 2048)],
                         ids=["config3_T512", "config4_T1024", "config3_T2048"])
def test_prefill_full_layer(cfg, tokens, prefill_from):
    prefill_from(128)
    tensors = host_layer(cfg, seed=0)
    x = O.synth_f32(0, CF.S_ACT, 0, tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)
    ref, sel_ref, _ = O.moe_forward(oracle_layer(cfg, tensors), x, tokens, cfg.top_k)
    s, out, sel, _ = _run(cfg, tensors, x, max_tokens=tokens)
    _check_selection(cfg, tensors, x, sel, sel_ref)
    same = np.all(sel == sel_ref, axis=1)
    assert max_rel(out[same], ref[same]) < PREFILL_MAX_REL
    # repeated host calls (the second is captured into a graph) give the same bytes
    again = s.run(x)
    third = s.run(x)
    assert s.status() == 0
    s.close()
    assert np.array_equal(again, out) and np.array_equal(third, out)


def test_prefill_and_decode_paths_agree_with_norm_and_residual(prefill_from):
    cfg = SMALL_QWEN
    tokens = 200
    tensors = host_layer(cfg, seed=11)
    norm = O.synth_f32(11, 30, 0, cfg.hidden, 1.0)
    x = O.synth_f32(11, CF.S_ACT, 0, tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)
    ref, sel_ref, _ = O.moe_forward(oracle_layer(cfg, tensors, input_norm=norm, residual=True),
                                    x, tokens, cfg.top_k)
    kw = dict(input_norm=norm, norm_epsilon=1e-6, add_residual=True)
    prefill_from(64)
    s, pf, sel, _ = _run(cfg, tensors, x, max_tokens=tokens, **kw)
    s.close()
    prefill_from(1 << 30)
    s, dec, sel2, _ = _run(cfg, tensors, x, max_tokens=tokens, **kw)
    s.close()
    assert np.array_equal(sel, sel2)
    same = np.all(sel == sel_ref, axis=1)
    assert max_rel(dec[same], ref[same]) < 1e-5
    assert max_rel(pf[same], ref[same]) < PREFILL_MAX_REL
    assert max_rel(pf, dec) < PREFILL_MAX_REL
