"""A MoE layer and a projection loaded from a GGUF file into a device arena
(llambda_cuda_gguf_upload) and run through device-pointer sessions, against
the oracle on the same bytes."""
import dataclasses

import numpy as np
import pytest

import llambda_b200 as LB
from llambda_b200 import configs as CF
from oracle import oracle as O
from tests import gguf_writer as W
from tests.helpers import MAX_REL, host_layer, max_rel, oracle_layer

pytestmark = pytest.mark.gpu

CFG = dataclasses.replace(CF.CONFIG3, name="gguf_qwen", hidden=512, experts=16, top_k=4,
                          inter=256, inter_sh=256)


def test_moe_layer_and_projection_from_gguf(tmp_path):
    tensors = host_layer(CFG, seed=13)
    names = list(tensors)
    path = tmp_path / "layer.gguf"
    W.write(path, [("general.architecture", W.STR, "qwen3next")],
            [(f"blk.0.{n}.weight", [d for d in (ne0, ne1, ne2) if d != 1] or [1], t,
              np.ascontiguousarray(arr).view(np.uint8).reshape(-1))
             for n, (t, ne0, ne1, ne2, arr) in tensors.items()])
    g = LB.GgufFile(str(path))
    idx = [g.find(f"blk.0.{n}.weight") for n in names]
    assert min(idx) >= 0
    arena, ptrs = g.upload(idx)
    try:
        dev = {}
        for n, p in zip(names, ptrs):
            t, ne0, ne1, ne2, _ = tensors[n]
            dev[n] = p if n in ("exp_probs_b.bias", "ffn_gate_inp_shexp") else (t, ne0, ne1, ne2, p)
        x = O.synth_f32(13, CF.S_ACT, 0, 3 * CFG.hidden, 1.0).reshape(3, CFG.hidden)
        ref, sel_ref, _ = O.moe_forward(oracle_layer(CFG, tensors), x, 3, CFG.top_k)
        s = LB.MoeSession.create(CFG.arch, CFG.hidden, CFG.top_k, dev, on_device=True, max_tokens=4)
        out, sel, _ = s.run(x, with_routing=True)
        s.close()
        same = np.all(sel == sel_ref, axis=1)
        assert same.mean() > 0.5
        assert max_rel(out[same], ref[same]) < MAX_REL
        # one expert's up rows as a projection session over the arena
        t, ne0, ne1, ne2, arr = tensors["ffn_up_exps"]
        p = LB.ProjectionSession.from_device(t, ne0, ne1, ptrs[names.index("ffn_up_exps")], ne2)
        xi = O.synth_f32(14, 1, 0, ne0, 1.0)
        y = p.run(xi)
        p.close()
        assert max_rel(y, O.gemv(t, arr, ne0, ne1, xi)) < MAX_REL
    finally:
        LB.device_free(arena)
        g.close()
