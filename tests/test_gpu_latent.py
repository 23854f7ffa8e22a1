"""GPU parity of the Q5_K dequant-GEMV (dot-product-with-q5-k-tensor-data,
L4387-4441) and of nemotron's latent projections (nemotron-h-moe-ffn-into
L5845-5855, L5883-5887, L5933-5938) against the CPU oracle, on the same
blocks, through the C ABI."""
import ctypes as C
import dataclasses

import numpy as np
import pytest

import llambda_b200 as LB
from llambda_b200 import _native as N
from llambda_b200 import configs as CF
from oracle import oracle as O
from oracle.layers import random_q5k
from tests import block32 as B32
from tests import kquant5 as K5
from tests.helpers import MAX_REL, gpu_tensors, host_layer, max_rel, oracle_layer
from tests.test_gpu_moe import _check_selection

pytestmark = pytest.mark.gpu

PREFILL_MAX_REL = 2e-2  # bf16 expert products of the prefill path


def _oracle_gemv(t, data, ne0, ne1, x):
    return np.stack([O.gemv(t, data, ne0, ne1, xi) for xi in np.asarray(x).reshape(-1, ne0)])


def test_q5k_hand_block_reads_back_through_unit_vectors():
    blk, want = K5.hand_q5k()
    s = LB.ProjectionSession.from_tensor(LB.TYPE_Q5_K, 256, 1, blk)
    eye = np.eye(256, dtype=np.float32)
    got = s.run_batch(eye)[:, 0]
    s.close()
    # d*sc*q is exact in fp32 and the kernel forms (d*sc)*q - dmin*m with one
    # rounding, so every weight comes back bit for bit
    assert np.array_equal(got, want)


@pytest.mark.parametrize("K,rows", [(256, 1), (512, 37), (2816, 300), (4096, 1000)])
@pytest.mark.parametrize("tokens", [1, 3, 8, 11])
def test_q5k_gemv_matches_oracle(K, rows, tokens):
    w = random_q5k(rows * K // 256, seed=K, stream=rows, dscale=0.02)
    x = O.synth_f32(4, 1, 0, tokens * K, 1.0).reshape(tokens, K)
    s = LB.ProjectionSession.from_tensor(LB.TYPE_Q5_K, K, rows, w)
    y = s.run_batch(x)
    s.close()
    r = _oracle_gemv(O.TYPE_Q5_K, w, K, rows, x)
    assert max_rel(y, r) < MAX_REL
    assert max_rel(y, r) < 1e-5


def test_q5k_rejects_fp16_specials():
    blk, _ = K5.hand_q5k()
    blk[0:2] = np.frombuffer(np.array([np.inf], np.float16).tobytes(), np.uint8)
    with pytest.raises(LB.LlambdaCudaError, match="Inf/NaN"):
        LB.ProjectionSession.from_tensor(LB.TYPE_Q5_K, 256, 1, blk)


LATENT = dataclasses.replace(CF.CONFIG4, name="latent_nemo", hidden=400, experts=16, top_k=3,
                             inter=200, inter_sh=300, latent=256, weight_scale=2.5)


def _latent_layer(lat_type, seed):
    cfg = dataclasses.replace(LATENT, latent_type=lat_type if lat_type != O.TYPE_Q8_0
                              else LB.TYPE_Q4_K)
    tensors = host_layer(cfg, seed)
    if lat_type == O.TYPE_Q8_0:  # 32-value blocks: rows of 400 values padded to 416
        H, L, HP = cfg.hidden, cfg.latent, (cfg.hidden + 31) // 32 * 32
        tensors["ffn_latent_down"] = (8, HP, L, 1, B32.random_blocks(8, L * HP // 32, seed))
        tensors["ffn_latent_up"] = (8, L, H, 1, B32.random_blocks(8, H * L // 32, seed + 1))
    return cfg, tensors


@pytest.mark.parametrize("lat_type", [LB.TYPE_Q4_K, LB.TYPE_Q5_K, LB.TYPE_Q6_K, LB.TYPE_F32,
                                      O.TYPE_Q8_0], ids=["q4k", "q5k", "q6k", "f32", "q8_0"])
@pytest.mark.parametrize("tokens", [1, 5, 64, 130])
def test_latent_layer_matches_oracle(lat_type, tokens):
    cfg, tensors = _latent_layer(lat_type, 17)
    norm = O.synth_f32(17, 30, 0, cfg.hidden, 1.0)
    x = O.synth_f32(17, CF.S_ACT, 0, tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)
    ref, sel_ref, _ = O.moe_forward(oracle_layer(cfg, tensors, input_norm=norm, residual=True),
                                    x, tokens, cfg.top_k)
    s = LB.MoeSession.create(cfg.arch, cfg.hidden, cfg.top_k, gpu_tensors(tensors),
                             weight_scale=cfg.weight_scale, weights_norm=cfg.weights_norm,
                             max_tokens=tokens, input_norm=norm, norm_epsilon=1e-6,
                             add_residual=True)
    out, sel, _ = s.run(x, with_routing=True)
    again = s.run(x)  # a second call (the host-buffer graph) gives the same bytes
    assert s.status() == 0
    s.close()
    assert np.array_equal(again, out)
    _check_selection(cfg, tensors, x, sel, sel_ref)
    same = np.all(sel == sel_ref, axis=1)
    assert np.isfinite(out).all()
    # fp32 decode kernels and projections: well inside the 1e-3 bar; prefill
    # batches (bf16 expert products): the 2e-2 bar
    bar = PREFILL_MAX_REL if tokens >= LB.prefill_min_tokens() else MAX_REL / 10
    assert max_rel(out[same], ref[same]) < bar


def test_latent_descriptors_are_checked():
    cfg, tensors = _latent_layer(LB.TYPE_Q4_K, 3)
    t = gpu_tensors(tensors)
    one = dict(t)
    del one["ffn_latent_up"]
    with pytest.raises(LB.LlambdaCudaError, match="together"):
        LB.MoeSession.create(cfg.arch, cfg.hidden, cfg.top_k, one, max_tokens=4)
    bad = dict(t)
    typ, ne0, ne1, ne2, arr = bad["ffn_latent_up"]
    bad["ffn_latent_up"] = (typ, ne0, ne1 - 16, ne2, arr[: arr.size * (ne1 - 16) // ne1])
    with pytest.raises(LB.LlambdaCudaError, match="ffn_latent_up"):
        LB.MoeSession.create(cfg.arch, cfg.hidden, cfg.top_k, bad, max_tokens=4)
    # qwen3next has no latent projections
    q = dataclasses.replace(CF.CONFIG3, hidden=512, experts=8, top_k=2, inter=256, inter_sh=256)
    qt = gpu_tensors(host_layer(q, 4))
    qt["ffn_latent_down"], qt["ffn_latent_up"] = t["ffn_latent_down"], t["ffn_latent_up"]
    with pytest.raises(LB.LlambdaCudaError, match="nemotron_h_moe"):
        LB.MoeSession.create(q.arch, q.hidden, q.top_k, qt, max_tokens=4)
    # a latent layer runs on one device: no peer reduction
    s = LB.MoeSession.create(cfg.arch, cfg.hidden, cfg.top_k, t, max_tokens=4)
    with pytest.raises(LB.LlambdaCudaError, match="one device"):
        s.attach_peers(0, 2, [0, 0], 1 << 30)
    s.close()


def test_static_scratch_refuses_latent_layers():
    import torch
    cfg, tensors = _latent_layer(LB.TYPE_Q4_K, 6)
    dev = {}
    for name, v in tensors.items():
        if isinstance(v, tuple):
            t, ne0, ne1, ne2, arr = v
            dev[name] = (t, ne0, ne1, ne2,
                         torch.from_numpy(np.ascontiguousarray(arr).view(np.uint8).copy()).cuda())
        else:
            dev[name] = torch.from_numpy(np.ascontiguousarray(v).view(np.uint8).copy()).cuda()
    s = LB.MoeSession.create(cfg.arch, cfg.hidden, cfg.top_k, gpu_tensors(dev), on_device=True,
                             max_tokens=2)
    d = s.desc
    x = torch.zeros(1, cfg.hidden, device="cuda")
    out = torch.empty_like(x)
    rc = LB.lib().llambda_cuda_moe_forward_static_scratch(C.byref(d), x.data_ptr(), 1,
                                                          out.data_ptr(), None)
    s.close()
    assert rc == -1 and "MoE session" in N.last_error()
