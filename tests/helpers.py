"""Shared test helpers: host-side seeded layers (through the oracle's copy of
the generator, oracle/layers.py) and the parity measure."""
from __future__ import annotations

import numpy as np

from llambda_b200 import configs as CF  # noqa: F401  (re-exported for the tests)
from oracle import oracle as O  # noqa: F401
from oracle.layers import host_layer, host_tensor, max_rel, oracle_layer  # noqa: F401

# Tolerance of the fp32 paths: max|y - r| / max|r| (north-star parity bar).
MAX_REL = 1e-3


def gpu_tensors(tensors: dict) -> dict:
    """Drops the bias / shared-gate vectors into the shape MoeSession.create wants."""
    out = {}
    for name, v in tensors.items():
        if name in ("exp_probs_b.bias", "ffn_gate_inp_shexp"):
            out[name] = v[4]
        else:
            out[name] = v
    return out


def topk_margin_ok(logits_sorted_desc: np.ndarray, k: int, margin: float = 1e-6) -> bool:
    return logits_sorted_desc.size <= k or (logits_sorted_desc[k - 1] - logits_sorted_desc[k]) > margin
