"""llambda_b200: a B200-native (sm_100a) backend for llambda's quantized
feed-forward path — Q4_K/Q6_K dequant-fused GEMV and the routed-MoE blocks of
qwen3next and nemotron_h_moe — behind llambda's accelerator-backend protocol.

The compute lives in libllambda_cuda.so (CUDA kernels plus a C ABI declared in
include/llambda_cuda.h); this package holds the Python side of that ABI and a
mirror of llambda's accelerator-backend descriptor protocol.
"""
from ._native import (ARCH_NEMOTRON_H_MOE, ARCH_QWEN3NEXT, TYPE_F32, TYPE_Q4_K,  # noqa: F401
                      TYPE_Q5_0, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_0, LlambdaCudaError, MoeSession,
                      GgufFile, ProjectionSession, bridge_version, device_free,
                      lib, prefill_min_tokens, probe, row_bytes, runtime_version,
                      set_prefill_min_tokens, sha256, synth_fill_device)

__all__ = ["ARCH_NEMOTRON_H_MOE", "ARCH_QWEN3NEXT", "TYPE_F32", "TYPE_Q4_K", "TYPE_Q5_0",
           "TYPE_Q5_K", "TYPE_Q6_K", "TYPE_Q8_0",
           "GgufFile", "LlambdaCudaError", "MoeSession", "ProjectionSession", "bridge_version",
           "device_free", "lib",
           "prefill_min_tokens", "set_prefill_min_tokens",
           "probe", "row_bytes", "runtime_version", "sha256", "synth_fill_device"]
