"""The allocation-free MoE entry point (llambda_cuda_moe_forward_static_scratch).

Some callers cannot call cudaMalloc: their own pooling allocator already owns
the device memory, or their decode loop must not pay for an allocation and
the synchronisation it can bring.  For them the library runs a MoE layer out
of one static device array and the caller's own device tensors.  These tests
call that entry point through the C ABI and compare it with the session entry
point (llambda_cuda_moe_session_run_device) on the same device tensors, on
several calls in a row of different sizes and shapes (decode sizes and
prefill-sized batches of 64 to 130 tokens), since the static array keeps the
previous call's contents.

This file is named to be collected last, and it builds everything it needs
itself, so it passes alone in a fresh process and after the rest of the suite.
"""
import ctypes as C
import dataclasses

import numpy as np
import pytest

import llambda_b200 as LB
from llambda_b200 import _native as N
from llambda_b200 import configs as CF
from oracle import oracle as O
from tests.helpers import host_layer, max_rel

pytestmark = pytest.mark.gpu

QWEN = dataclasses.replace(CF.CONFIG3, name="static_qwen", hidden=512, experts=32, top_k=6,
                           inter=256, inter_sh=512)
NEMO = dataclasses.replace(CF.CONFIG4, name="static_nemo", hidden=400, experts=16, top_k=3,
                           inter=200, inter_sh=300)


def _device_layer(cfg, seed, torch):
    """Every tensor of a layer in device memory (the caller owns them)."""
    host = host_layer(cfg, seed)
    dev = {}
    for name, (t, ne0, ne1, ne2, arr) in host.items():
        d = torch.from_numpy(np.ascontiguousarray(arr).view(np.uint8).copy()).cuda()
        dev[name] = d if name in ("exp_probs_b.bias", "ffn_gate_inp_shexp") else (t, ne0, ne1, ne2, d)
    return dev


def _desc(cfg, dev, norm_w=None, residual=False, expert_range=(0, 0), shared_here=True):
    def T(name):
        if name not in dev:
            return N.Tensor(0, 0, 0, 0, None)
        t, ne0, ne1, ne2, d = dev[name]
        return N.Tensor(t, ne0, ne1, ne2, d.data_ptr())

    d = N.MoeDesc()
    d.arch, d.hidden, d.top_k = cfg.arch, cfg.hidden, cfg.top_k
    d.weight_scale, d.weights_norm, d.data_on_device = cfg.weight_scale, int(cfg.weights_norm), 1
    d.router = T("ffn_gate_inp")
    d.router_bias = dev["exp_probs_b.bias"].data_ptr() if "exp_probs_b.bias" in dev else None
    d.shared_gate_inp = dev["ffn_gate_inp_shexp"].data_ptr() if "ffn_gate_inp_shexp" in dev else None
    d.gate_exps, d.up_exps, d.down_exps = T("ffn_gate_exps"), T("ffn_up_exps"), T("ffn_down_exps")
    d.gate_shexp, d.up_shexp, d.down_shexp = T("ffn_gate_shexp"), T("ffn_up_shexp"), T("ffn_down_shexp")
    d.expert_begin, d.expert_end = expert_range
    d.shared_here = int(shared_here)
    d.max_tokens = 256
    d.input_norm = norm_w.data_ptr() if norm_w is not None else None
    d.norm_epsilon = 1e-6
    d.add_residual = int(residual)
    return d


def _static_call(desc, x, out, tokens, stream):
    rc = LB.lib().llambda_cuda_moe_forward_static_scratch(C.byref(desc), x.data_ptr(), tokens,
                                                          out.data_ptr(), stream.cuda_stream)
    if rc != 0:
        raise LB.LlambdaCudaError(N.last_error())


# Token counts of the calls in a row: decode sizes, then batches at and past
# the prefill threshold (128: the bf16 tcgen05 path, whose buffers are carved
# into the array from 64 tokens on), then smaller ones again over the stale
# prefill contents.
DECODE_CALLS = ((5, 1), (17, 2))
PREFILL_CALLS = ((5, 1), (128, 4), (64, 5), (130, 6), (17, 2))


def _tol(tokens):
    # both entry points run the same kernels on the same bytes; prefill-sized
    # batches compute in bf16 (bar 2e-2), the decode kernels in fp32
    return 2e-2 if tokens >= LB.prefill_min_tokens() else 1e-5


@pytest.mark.parametrize("cfg,extra,calls", [
    (QWEN, {}, DECODE_CALLS), (NEMO, {}, DECODE_CALLS),
    (QWEN, {"norm": True, "residual": True}, DECODE_CALLS),
    (QWEN, {"expert_range": (8, 20), "shared_here": False}, DECODE_CALLS),
    (QWEN, {}, PREFILL_CALLS), (NEMO, {"norm": True, "residual": True}, PREFILL_CALLS)],
    ids=["qwen", "nemotron", "qwen_norm_residual", "qwen_expert_shard", "qwen_prefill_sizes",
         "nemotron_prefill_sizes_after_qwen"])
def test_static_scratch_matches_session_on_calls_in_a_row(cfg, extra, calls):
    import torch
    dev = _device_layer(cfg, 21, torch)
    norm_w = torch.from_numpy(O.synth_f32(21, 30, 0, cfg.hidden, 1.0)).cuda() \
        if extra.get("norm") else None
    desc = _desc(cfg, dev, norm_w, extra.get("residual", False),
                 extra.get("expert_range", (0, 0)), extra.get("shared_here", True))
    stream = torch.cuda.current_stream()
    for tokens, seed in calls:  # calls in a row, different sizes
        x = torch.from_numpy(O.synth_f32(seed, CF.S_ACT, 0, tokens * cfg.hidden, 1.0)).cuda()
        want = torch.empty_like(x)
        got = torch.full_like(x, float("nan"))
        # the existing entry point, on the very same device tensors
        sess_tensors = {k: v for k, v in dev.items()}
        s = LB.MoeSession.create(cfg.arch, cfg.hidden, cfg.top_k, sess_tensors,
                                 weight_scale=cfg.weight_scale, weights_norm=cfg.weights_norm,
                                 on_device=True, max_tokens=max(t for t, _ in calls),
                                 expert_range=extra.get("expert_range", (0, 0)),
                                 shared_here=extra.get("shared_here", True),
                                 input_norm=norm_w, norm_epsilon=1e-6,
                                 add_residual=extra.get("residual", False))
        s.run_device(x, want, tokens, stream=stream)
        _static_call(desc, x, got, tokens, stream)
        torch.cuda.synchronize()
        assert s.status() == 0
        s.close()
        w, g = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(g).all()
        assert max_rel(g, w) < _tol(tokens), (tokens, max_rel(g, w))


def test_static_scratch_rejects_oversized_calls():
    import torch
    cfg = dataclasses.replace(CF.CONFIG4, name="static_big", hidden=2048, experts=8, top_k=8,
                              inter=3840, inter_sh=3840)
    dev = _device_layer(cfg, 3, torch)
    desc = _desc(cfg, dev)
    tokens = 200  # (200*8 + 200) intermediates of 3840 floats alone exceed 16 MiB
    x = torch.zeros(tokens, cfg.hidden, device="cuda")
    out = torch.empty_like(x)
    with pytest.raises(LB.LlambdaCudaError, match="static scratch holds"):
        _static_call(desc, x, out, tokens, torch.cuda.current_stream())
    # a host-memory descriptor is refused: nothing may be uploaded
    desc.data_on_device = 0
    with pytest.raises(LB.LlambdaCudaError, match="data_on_device"):
        _static_call(desc, x, out, 1, torch.cuda.current_stream())


def test_static_scratch_reports_non_positive_weight_sum():
    import torch
    cfg = dataclasses.replace(NEMO, weights_norm=True)
    dev = _device_layer(cfg, 2, torch)
    dev["exp_probs_b.bias"] = torch.full((cfg.experts,), -1e30, device="cuda")
    desc = _desc(cfg, dev)
    x = torch.from_numpy(O.synth_f32(2, CF.S_ACT, 0, cfg.hidden, 1.0)).cuda()
    out = torch.empty_like(x)
    with pytest.raises(LB.LlambdaCudaError, match="non-positive"):
        _static_call(desc, x, out, 1, torch.cuda.current_stream())
    # the status word starts at zero again on the next call
    dev2 = _device_layer(NEMO, 2, torch)
    x2 = torch.from_numpy(O.synth_f32(3, CF.S_ACT, 0, 2 * NEMO.hidden, 1.0)).cuda()
    out2 = torch.empty_like(x2)
    _static_call(_desc(NEMO, dev2), x2, out2, 2, torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert np.isfinite(out2.cpu().numpy()).all()
