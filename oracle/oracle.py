"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the CPU oracle.

The oracle (oracle/llambda_oracle.c) restates llambda's quantized FFN CPU path
(jrm-code-project/llambda, llambda.lisp L4109-4658 and L5265-5949).  Only the
test suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use
this module, and only as the checker or the timed CPU reference; the shipped
library never calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

TYPE_F32, TYPE_F16, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 0, 1, 12, 13, 14
TYPE_Q5_0, TYPE_Q8_0 = 6, 8
Q4K_BLOCK, Q5K_BLOCK, Q6K_BLOCK, QK_K = 144, 176, 210, 256

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


class Tensor(C.Structure):
    _fields_ = [("type", C.c_int), ("data", C.c_void_p),
                ("ne0", C.c_size_t), ("ne1", C.c_size_t), ("ne2", C.c_size_t)]


class MoeLayer(C.Structure):
    _fields_ = [("arch", C.c_int), ("hidden", C.c_size_t), ("top_k", C.c_int),
                ("weight_scale", C.c_float), ("weights_norm", C.c_int),
                ("router", Tensor), ("router_bias", C.c_void_p),
                ("shared_gate_inp", C.c_void_p),
                ("gate_exps", Tensor), ("up_exps", Tensor), ("down_exps", Tensor),
                ("gate_shexp", Tensor), ("up_shexp", Tensor), ("down_shexp", Tensor),
                ("input_norm", C.c_void_p), ("norm_epsilon", C.c_float),
                ("add_residual", C.c_int),
                ("latent_down", Tensor), ("latent_up", Tensor)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        fp, u8p, i32p = C.POINTER(C.c_float), C.c_void_p, C.POINTER(C.c_int32)
        L.or_last_error.restype = C.c_char_p
        L.or_fp16_to_f32.argtypes = [C.c_uint16, C.POINTER(C.c_int)]
        L.or_fp16_to_f32.restype = C.c_float
        L.or_get_scale_min_k4.argtypes = [u8p, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        for name in ("or_dequantize_q4_k", "or_dequantize_q6_k", "or_dequantize_q5_0",
                     "or_dequantize_q8_0", "or_dequantize_q5_k"):
            getattr(L, name).argtypes = [u8p, C.c_size_t, fp]
            getattr(L, name).restype = C.c_int
        for name in ("or_dot_q4_k", "or_dot_q6_k", "or_dot_q5_0", "or_dot_q8_0", "or_dot_q5_k"):
            getattr(L, name).argtypes = [u8p, fp, C.c_size_t, fp]
            getattr(L, name).restype = C.c_int
        for name in ("or_dot_f32", "or_dot_product"):
            getattr(L, name).argtypes = [fp, fp, C.c_size_t]
            getattr(L, name).restype = C.c_float
        L.or_row_bytes.argtypes = [C.c_int, C.c_size_t]
        L.or_row_bytes.restype = C.c_size_t
        L.or_gemv.argtypes = [C.POINTER(Tensor), C.c_size_t, C.c_size_t, fp, fp]
        L.or_gemv.restype = C.c_int
        L.or_select_top_k.argtypes = [fp, C.c_size_t, C.c_int, i32p, fp]
        for name in ("or_sigmoid", "or_silu", "or_relu_squared"):
            getattr(L, name).argtypes = [C.c_float]
            getattr(L, name).restype = C.c_float
        L.or_moe_forward.argtypes = [C.POINTER(MoeLayer), fp, C.c_size_t, fp, i32p, fp]
        L.or_moe_forward.restype = C.c_int
        for name in ("or_synth_q4k", "or_synth_q6k"):
            getattr(L, name).argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_size_t,
                                         C.c_float, u8p]
        L.or_synth_f32.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_size_t,
                                   C.c_float, fp]
        L.or_rms_norm.argtypes = [fp, fp, C.c_size_t, C.c_float, fp]
        L.or_f32_to_f16.argtypes = [C.c_float]
        L.or_f32_to_f16.restype = C.c_uint16
        L.or_set_workers.argtypes = [C.c_int]
        L.or_get_workers.restype = C.c_int
        _lib = L
    return _lib


class OracleError(RuntimeError):
    pass


def _fptr(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _check(rc):
    if rc != 0:
        raise OracleError(lib().or_last_error().decode())


def set_workers(n: int) -> None:
    lib().or_set_workers(int(n))


def fp16_to_f32(bits: int) -> float:
    err = C.c_int(0)
    v = lib().or_fp16_to_f32(bits, C.byref(err))
    if err.value:
        raise OracleError(lib().or_last_error().decode())
    return v


def dequantize(type_tag: int, blocks: np.ndarray, count: int) -> np.ndarray:
    out = np.empty(count, np.float32)
    fn = {TYPE_Q4_K: lib().or_dequantize_q4_k, TYPE_Q6_K: lib().or_dequantize_q6_k,
          TYPE_Q5_0: lib().or_dequantize_q5_0, TYPE_Q8_0: lib().or_dequantize_q8_0,
          TYPE_Q5_K: lib().or_dequantize_q5_k}[type_tag]
    _check(fn(blocks.ctypes.data, count, _fptr(out)))
    return out


def dot_row(type_tag: int, row: np.ndarray, x: np.ndarray) -> float:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(1, np.float32)
    if type_tag == TYPE_F32:
        return lib().or_dot_f32(_fptr(np.ascontiguousarray(row, np.float32)), _fptr(x), x.size)
    fn = {TYPE_Q4_K: lib().or_dot_q4_k, TYPE_Q6_K: lib().or_dot_q6_k,
          TYPE_Q5_0: lib().or_dot_q5_0, TYPE_Q8_0: lib().or_dot_q8_0,
          TYPE_Q5_K: lib().or_dot_q5_k}[type_tag]
    _check(fn(row.ctypes.data, _fptr(x), x.size, _fptr(out)))
    return float(out[0])


def make_tensor(type_tag: int, data: np.ndarray | None, ne0: int, ne1: int, ne2: int = 1) -> Tensor:
    return Tensor(type_tag, 0 if data is None else data.ctypes.data, ne0, ne1, ne2)


def gemv(type_tag: int, data: np.ndarray, ne0: int, ne1: int, x: np.ndarray,
         start_row: int = 0, row_count: int | None = None) -> np.ndarray:
    """%gguf-model-matrix-vector-multiply-into over rows [start, start+count)."""
    row_count = ne1 - start_row if row_count is None else row_count
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(row_count, np.float32)
    flat = ne1
    t = make_tensor(type_tag, data, ne0, flat, 1)
    _check(lib().or_gemv(C.byref(t), start_row, row_count, _fptr(x), _fptr(y)))
    return y


def select_top_k(logits: np.ndarray, k: int):
    logits = np.ascontiguousarray(logits, np.float32)
    idx = np.empty(k, np.int32)
    vals = np.empty(k, np.float32)
    lib().or_select_top_k(_fptr(logits), logits.size, k,
                          idx.ctypes.data_as(C.POINTER(C.c_int32)), _fptr(vals))
    return idx, vals


def sigmoid(v: float) -> float:
    return lib().or_sigmoid(v)


def silu(v: float) -> float:
    return lib().or_silu(v)


def relu_squared(v: float) -> float:
    return lib().or_relu_squared(v)


def moe_forward(layer: MoeLayer, x: np.ndarray, tokens: int, top_k: int):
    """qwen3next-moe-into / nemotron-h-moe-ffn-into over `tokens` rows of x."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    sel = np.empty((tokens, top_k), np.int32)
    w = np.empty((tokens, top_k), np.float32)
    _check(lib().or_moe_forward(C.byref(layer), _fptr(x), tokens, _fptr(out),
                                sel.ctypes.data_as(C.POINTER(C.c_int32)), _fptr(w)))
    return out, sel, w


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().or_rms_norm(_fptr(x), _fptr(w), x.size, eps, _fptr(out))
    return out


def synth_q4k(seed: int, stream: int, first_block: int, blocks: int, dscale: float) -> np.ndarray:
    out = np.empty(blocks * Q4K_BLOCK, np.uint8)
    lib().or_synth_q4k(seed, stream, first_block, blocks, dscale, out.ctypes.data)
    return out


def synth_q6k(seed: int, stream: int, first_block: int, blocks: int, dscale: float) -> np.ndarray:
    out = np.empty(blocks * Q6K_BLOCK, np.uint8)
    lib().or_synth_q6k(seed, stream, first_block, blocks, dscale, out.ctypes.data)
    return out


def synth_f32(seed: int, stream: int, first: int, count: int, sigma: float) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().or_synth_f32(seed, stream, first, count, sigma, _fptr(out))
    return out


def f32_to_f16(v: float) -> int:
    return lib().or_f32_to_f16(v)
