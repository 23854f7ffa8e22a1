"""TEST INFRASTRUCTURE ONLY: seeded host-side MoE layers for the CPU oracle.

The synthetic tensors of a layer are made on the host by the oracle's copy of
the generator (byte-identical to the device generator), and an oracle layer
descriptor points at them.  Only the test suite, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg use this module, as the checker or the
timed CPU reference.
"""
from __future__ import annotations

import numpy as np

from llambda_b200 import configs as CF
from llambda_b200._native import TYPE_F32, TYPE_Q4_K

from . import oracle as O


def max_rel(y: np.ndarray, r: np.ndarray) -> float:
    """max|y - r| / max|r| (the parity measure of the fp32 and bf16 paths)."""
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    den = np.max(np.abs(r))
    return float(np.max(np.abs(y - r)) / den) if den > 0 else float(np.max(np.abs(y - r)))


def random_q5k(blocks: int, seed: int, stream: int, dscale: float) -> np.ndarray:
    """Q5_K blocks (176 bytes) from numpy's seeded generator: d, dmin =
    fp16(|N(0,1)| * dscale), the 12 packed scale bytes, qh and qs uniform.
    The device generator has no Q5_K form; these blocks are uploaded."""
    rng = np.random.default_rng([seed, stream, 13])
    dm = (np.abs(rng.standard_normal((blocks, 2))) * dscale).astype(np.float16)
    rest = rng.integers(0, 256, (blocks, 172), dtype=np.uint8)
    return np.ascontiguousarray(np.concatenate([dm.view(np.uint8), rest], axis=1)).reshape(-1)


def host_tensor(type_tag: int, ne0: int, ne1: int, ne2: int, seed: int, stream: int,
                scale: float) -> np.ndarray:
    units = CF.tensor_units(type_tag, ne0, ne1, ne2)
    if type_tag == TYPE_F32:
        return O.synth_f32(seed, stream, 0, units, scale)
    if type_tag == TYPE_Q4_K:
        return O.synth_q4k(seed, stream, 0, units, scale)
    if type_tag == O.TYPE_Q5_K:
        return random_q5k(units, seed, stream, scale)
    return O.synth_q6k(seed, stream, 0, units, scale)


def host_layer(cfg: CF.MoeConfig, seed: int) -> dict:
    """name -> (type, ne0, ne1, ne2, numpy array) for every tensor of a layer."""
    out = {}
    for name, t, ne0, ne1, ne2, stream, scale in CF.moe_tensor_specs(cfg):
        arr = host_tensor(t, ne0, ne1, ne2, seed, stream, scale)
        out[name] = (t, ne0, ne1, ne2, arr)
    return out


def oracle_layer(cfg: CF.MoeConfig, tensors: dict, input_norm=None, eps=1e-6,
                 residual=False) -> O.MoeLayer:
    L = O.MoeLayer()
    L.arch, L.hidden, L.top_k = cfg.arch, cfg.hidden, cfg.top_k
    L.weight_scale, L.weights_norm = cfg.weight_scale, int(cfg.weights_norm)

    def T(name):
        if name not in tensors:
            return O.make_tensor(0, None, 0, 0, 0)
        t, ne0, ne1, ne2, arr = tensors[name]
        return O.make_tensor(t, arr, ne0, ne1, ne2)

    L.router = T("ffn_gate_inp")
    L.router_bias = tensors["exp_probs_b.bias"][4].ctypes.data if "exp_probs_b.bias" in tensors else None
    L.shared_gate_inp = (tensors["ffn_gate_inp_shexp"][4].ctypes.data
                         if "ffn_gate_inp_shexp" in tensors else None)
    L.gate_exps, L.up_exps, L.down_exps = T("ffn_gate_exps"), T("ffn_up_exps"), T("ffn_down_exps")
    L.gate_shexp, L.up_shexp, L.down_shexp = T("ffn_gate_shexp"), T("ffn_up_shexp"), T("ffn_down_shexp")
    L._keep = input_norm
    L.input_norm = input_norm.ctypes.data if input_norm is not None else None
    L.norm_epsilon = eps
    L.add_residual = int(residual)
    L.latent_down, L.latent_up = T("ffn_latent_down"), T("ffn_latent_up")
    return L
