"""The benchmark configurations of the quantized-FFN path, as data.

Shapes and value distributions follow the five workloads the path is measured
on (dense Q4_K GEMV, dense Q6_K lm-head GEMV, a qwen3next-shaped MoE layer, a
nemotron_h_moe-shaped MoE layer, and a 48-layer stack of the qwen3next layer).
Inputs are synthetic (seeded, llambda_b200/csrc/synth.h); there is no model
file.  Nemotron widths that are not multiples of 256 (2688, 1856, 3712) are
zero-padded to K-quant rows (2816, 2048, 3840): the padded columns meet
zero activations, so the result is the unpadded product, and bytes are
counted as stored.
"""
from __future__ import annotations

from dataclasses import dataclass, field

from ._native import ARCH_NEMOTRON_H_MOE, ARCH_QWEN3NEXT, TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, row_bytes

# generator stream ids (synth.h)
S_ACT, S_ROUTER, S_BIAS, S_SHGATE = 1, 2, 3, 4
S_GATE, S_UP, S_DOWN, S_GATE_SH, S_UP_SH, S_DOWN_SH, S_DENSE = 5, 6, 7, 8, 9, 10, 11
S_LAT_DOWN, S_LAT_UP = 12, 13

Q4K_DSCALE = 0.02    # fp16 d, dmin = |N(0,1)| * 0.02
Q6K_DSCALE = 0.001   # fp16 d = |N(0,1)| * 0.001
ROUTER_SIGMA = 0.02
BIAS_SIGMA = 0.01


def pad256(n: int) -> int:
    return (n + 255) // 256 * 256


@dataclass(frozen=True)
class DenseConfig:
    name: str
    type: int
    rows: int
    cols: int
    dscale: float

    @property
    def weight_bytes(self) -> int:
        return row_bytes(self.type, self.cols) * self.rows

    def algorithmic_bytes(self, tokens: int) -> int:
        return self.weight_bytes + 4 * tokens * (self.cols + self.rows)


CONFIG1 = DenseConfig("config1_q4k_gemv_14336x4096", TYPE_Q4_K, 14336, 4096, Q4K_DSCALE)
CONFIG2 = DenseConfig("config2_q6k_lmhead_128256x4096", TYPE_Q6_K, 128256, 4096, Q6K_DSCALE)
# 32-value-block GEMVs at a Nemotron-H width that is not a multiple of 256
# (hidden 2688), rows enough to exceed L2; random blocks, d = |N(0,1)| * 0.02
DENSE_Q8_0 = DenseConfig("q8_0_gemv_65536x2688", 8, 65536, 2688, 0.02)
DENSE_Q5_0 = DenseConfig("q5_0_gemv_65536x2688", 6, 65536, 2688, 0.02)


@dataclass(frozen=True)
class MoeConfig:
    name: str
    arch: int
    hidden: int
    experts: int
    top_k: int
    inter: int
    inter_sh: int
    gate_type: int = TYPE_Q4_K
    up_type: int = TYPE_Q4_K
    down_type: int = TYPE_Q6_K
    weights_norm: bool = True
    weight_scale: float = 1.0
    has_bias: bool = False
    tokens: tuple = field(default=(1,))
    # nemotron latent projections (0: none): the routed experts work at this
    # width, between ffn_latent_down and ffn_latent_up
    latent: int = 0
    latent_type: int = TYPE_Q4_K

    @property
    def expert_width(self) -> int:
        """Input and output width of the routed experts."""
        return self.latent or self.hidden

    @property
    def k_in(self) -> int:
        return pad256(self.expert_width)

    @property
    def k_in_sh(self) -> int:
        return pad256(self.hidden)

    @property
    def k_down(self) -> int:
        return pad256(self.inter)

    @property
    def k_down_sh(self) -> int:
        return pad256(self.inter_sh)

    @property
    def has_gate(self) -> bool:
        return self.arch == ARCH_QWEN3NEXT

    def expert_bytes(self) -> int:
        up = row_bytes(self.up_type, self.k_in) * self.inter
        gate = up if self.has_gate else 0
        down = row_bytes(self.down_type, self.k_down) * self.expert_width
        return gate + up + down

    def gate_up_bytes(self) -> int:
        up = row_bytes(self.up_type, self.k_in) * self.inter
        return up * (2 if self.has_gate else 1)

    def down_bytes(self) -> int:
        return row_bytes(self.down_type, self.k_down) * self.expert_width

    def shared_gate_up_bytes(self) -> int:
        up = row_bytes(self.up_type, self.k_in_sh) * self.inter_sh
        return up * (2 if self.has_gate else 1)

    def shared_bytes(self) -> int:
        up = row_bytes(self.up_type, self.k_in_sh) * self.inter_sh
        gate = up if self.has_gate else 0
        down = row_bytes(self.down_type, self.k_down_sh) * self.hidden
        return gate + up + down

    def router_bytes(self) -> int:
        b = self.experts * self.hidden * 4
        if self.arch == ARCH_QWEN3NEXT:
            b += self.hidden * 4          # ffn_gate_inp_shexp
        if self.has_bias:
            b += self.experts * 4
        return b

    def algorithmic_bytes(self, tokens: int, distinct_experts: int) -> int:
        """Weights that one layer call must stream (router, shared expert and
        every distinct routed expert once) plus activations in and out."""
        return (self.router_bytes() + self.shared_bytes() + distinct_experts * self.expert_bytes()
                + 2 * 4 * tokens * self.hidden)

    def flops(self, tokens: int) -> int:
        per_expert = (3 if self.has_gate else 2) * 2 * self.hidden * self.inter
        shared = (3 if self.has_gate else 2) * 2 * self.hidden * self.inter_sh
        return tokens * (2 * self.experts * self.hidden + self.top_k * per_expert + shared)


CONFIG3 = MoeConfig("config3_qwen3next_moe", ARCH_QWEN3NEXT, 2048, 512, 10, 512, 512,
                    tokens=(1, 16, 512))
CONFIG4 = MoeConfig("config4_nemotron_h_moe", ARCH_NEMOTRON_H_MOE, 2688, 128, 6, 1856, 3712,
                    has_bias=True, tokens=(1, 64, 1024))
CONFIG5_LAYERS = 48


def layer_seed(base_seed: int, layer: int) -> int:
    """Independent seeds per stacked layer."""
    return base_seed * 1000003 + layer


def moe_tensor_specs(cfg: MoeConfig):
    """(gguf name, type, ne0, ne1, ne2, stream id, scale) of every layer tensor."""
    specs = [("ffn_gate_inp", TYPE_F32, cfg.hidden, cfg.experts, 1, S_ROUTER, ROUTER_SIGMA)]
    if cfg.has_bias:
        specs.append(("exp_probs_b.bias", TYPE_F32, cfg.experts, 1, 1, S_BIAS, BIAS_SIGMA))
    if cfg.arch == ARCH_QWEN3NEXT:
        specs.append(("ffn_gate_inp_shexp", TYPE_F32, cfg.hidden, 1, 1, S_SHGATE, ROUTER_SIGMA))
        specs.append(("ffn_gate_exps", cfg.gate_type, cfg.k_in, cfg.inter, cfg.experts, S_GATE,
                      Q4K_DSCALE))
    specs.append(("ffn_up_exps", cfg.up_type, cfg.k_in, cfg.inter, cfg.experts, S_UP, Q4K_DSCALE))
    specs.append(("ffn_down_exps", cfg.down_type, cfg.k_down, cfg.expert_width, cfg.experts,
                  S_DOWN, Q6K_DSCALE))
    if cfg.latent:
        lt = cfg.latent_type
        ds = Q6K_DSCALE if lt == TYPE_Q6_K else (ROUTER_SIGMA if lt == TYPE_F32 else Q4K_DSCALE)
        specs.append(("ffn_latent_down", lt, cfg.k_in_sh if lt != TYPE_F32 else cfg.hidden,
                      cfg.latent, 1, S_LAT_DOWN, ds))
        specs.append(("ffn_latent_up", lt, pad256(cfg.latent) if lt != TYPE_F32 else cfg.latent,
                      cfg.hidden, 1, S_LAT_UP, ds))
    if cfg.inter_sh:
        if cfg.arch == ARCH_QWEN3NEXT:
            specs.append(("ffn_gate_shexp", cfg.gate_type, cfg.k_in_sh, cfg.inter_sh, 1, S_GATE_SH,
                          Q4K_DSCALE))
        specs.append(("ffn_up_shexp", cfg.up_type, cfg.k_in_sh, cfg.inter_sh, 1, S_UP_SH,
                      Q4K_DSCALE))
        specs.append(("ffn_down_shexp", cfg.down_type, cfg.k_down_sh, cfg.hidden, 1, S_DOWN_SH,
                      Q6K_DSCALE))
    return specs


def tensor_units(type_tag: int, ne0: int, ne1: int, ne2: int) -> int:
    """Generator units: super-blocks for K-quants, floats for F32."""
    n = ne0 * ne1 * ne2
    return n if type_tag == TYPE_F32 else n // 256
