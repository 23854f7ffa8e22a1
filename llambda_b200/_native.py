"""ctypes bindings of libllambda_cuda.so (the C ABI in include/llambda_cuda.h).

There is deliberately no CPU fallback here: if the library cannot be loaded,
or a call fails, a LlambdaCudaError carries the library's own message, and the
caller's fallback logic (the accelerator protocol in accelerator.py) decides
what happens, as llambda's call-with-accelerator-runtime-fallback does
(llambda.lisp L4660-4676).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libllambda_cuda.so")

TYPE_F32, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 0, 12, 13, 14
TYPE_Q5_0, TYPE_Q8_0 = 6, 8  # 32-value blocks: projection sessions only
ARCH_QWEN3NEXT, ARCH_NEMOTRON_H_MOE = 0, 1
BLOCK_BYTES = {TYPE_Q4_K: 144, TYPE_Q5_K: 176, TYPE_Q6_K: 210}
BLOCK32_BYTES = {TYPE_Q5_0: 22, TYPE_Q8_0: 34}


class LlambdaCudaError(RuntimeError):
    """A failed call into the CUDA backend (status -1 plus last_error)."""


def row_bytes(type_tag: int, ne0: int) -> int:
    if type_tag == TYPE_F32:
        return ne0 * 4
    if type_tag in BLOCK_BYTES:
        if ne0 % 256:
            raise ValueError(f"K-quant rows need a multiple of 256 columns, got {ne0}")
        return ne0 // 256 * BLOCK_BYTES[type_tag]
    if type_tag in BLOCK32_BYTES:
        if ne0 % 32:
            raise ValueError(f"Q5_0/Q8_0 rows need a multiple of 32 columns, got {ne0}")
        return ne0 // 32 * BLOCK32_BYTES[type_tag]
    raise ValueError(f"unsupported GGML type tag {type_tag}")


class Tensor(C.Structure):
    _fields_ = [("type", C.c_int), ("ne0", C.c_uint64), ("ne1", C.c_uint64),
                ("ne2", C.c_uint64), ("data", C.c_void_p)]


class MoeDesc(C.Structure):
    _fields_ = [("arch", C.c_int), ("hidden", C.c_uint64), ("top_k", C.c_int),
                ("weight_scale", C.c_float), ("weights_norm", C.c_int),
                ("data_on_device", C.c_int),
                ("router", Tensor), ("router_bias", C.c_void_p),
                ("shared_gate_inp", C.c_void_p),
                ("gate_exps", Tensor), ("up_exps", Tensor), ("down_exps", Tensor),
                ("gate_shexp", Tensor), ("up_shexp", Tensor), ("down_shexp", Tensor),
                ("expert_begin", C.c_int), ("expert_end", C.c_int),
                ("shared_here", C.c_int), ("max_tokens", C.c_int),
                ("input_norm", C.c_void_p), ("norm_epsilon", C.c_float),
                ("add_residual", C.c_int),
                ("latent_down", Tensor), ("latent_up", Tensor)]


# name -> (restype, argtypes); every symbol the public header declares.
_vp, _sz, _u64, _fp, _i32p = C.c_void_p, C.c_size_t, C.c_uint64, C.POINTER(C.c_float), C.POINTER(C.c_int32)
SIGNATURES = {
    "llambda_cuda_probe": (C.c_int, []),
    "llambda_cuda_bridge_version": (C.c_char_p, []),
    "llambda_cuda_runtime_version": (C.c_char_p, []),
    "llambda_cuda_last_error": (C.c_char_p, []),
    "llambda_cuda_sha256": (C.c_int, [_vp, _sz, C.c_char_p, _sz]),
    "llambda_cuda_session_create": (C.c_int, [C.c_char_p, C.POINTER(_vp)]),
    "llambda_cuda_session_create_from_tensor": (C.c_int, [C.c_int, _u64, _u64, _u64, _vp, _sz,
                                                          C.POINTER(_vp)]),
    "llambda_cuda_session_create_device": (C.c_int, [C.c_int, _u64, _u64, _u64, _vp,
                                                     C.POINTER(_vp)]),
    "llambda_cuda_session_destroy": (None, [_vp]),
    "llambda_cuda_session_input_element_count": (_sz, [_vp]),
    "llambda_cuda_session_output_element_count": (_sz, [_vp]),
    "llambda_cuda_session_run": (C.c_int, [_vp, _fp, _sz, _fp, _sz]),
    "llambda_cuda_session_run_batch": (C.c_int, [_vp, _fp, _sz, _fp]),
    "llambda_cuda_session_run_expert": (C.c_int, [_vp, C.c_int, _fp, _sz, _fp, _sz]),
    "llambda_cuda_session_run_device": (C.c_int, [_vp, _vp, _sz, _vp, _vp]),
    "llambda_cuda_moe_session_create": (C.c_int, [C.POINTER(MoeDesc), C.POINTER(_vp)]),
    "llambda_cuda_moe_session_destroy": (None, [_vp]),
    "llambda_cuda_moe_session_hidden": (_sz, [_vp]),
    "llambda_cuda_moe_session_run": (C.c_int, [_vp, _fp, _sz, _fp, _i32p, _fp]),
    "llambda_cuda_moe_session_run_device": (C.c_int, [_vp, _vp, _sz, _vp, _vp, _vp, _vp]),
    "llambda_cuda_moe_session_status": (C.c_int, [_vp]),
    "llambda_cuda_moe_session_time_kernels": (C.c_int, [_vp, C.c_int]),
    "llambda_cuda_moe_session_kernel_breakdown": (C.c_int, [_vp, C.POINTER(C.c_float), C.c_int]),
    "llambda_cuda_moe_dispatch_bytes": (_sz, [_vp, C.c_int, C.c_int]),
    "llambda_cuda_moe_session_attach_dispatch": (C.c_int, [_vp, C.c_int, C.c_int, C.POINTER(_vp),
                                                           _sz, C.c_int]),
    "llambda_cuda_moe_session_kernel_ms": (C.c_int, [_vp, C.POINTER(C.c_float),
                                                      C.POINTER(C.c_float)]),
    "llambda_cuda_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(_vp)]),
    "llambda_cuda_gguf_close": (None, [_vp]),
    "llambda_cuda_gguf_tensor_count": (_u64, [_vp]),
    "llambda_cuda_gguf_find": (C.c_int64, [_vp, C.c_char_p]),
    "llambda_cuda_gguf_tensor_info": (C.c_int, [_vp, _u64, C.c_char_p, _sz, C.POINTER(C.c_int),
                                               C.POINTER(C.c_uint32), C.POINTER(_u64),
                                               C.POINTER(_u64), C.POINTER(_vp)]),
    "llambda_cuda_gguf_upload": (C.c_int, [_vp, C.POINTER(_u64), _sz, C.POINTER(_vp),
                                          C.POINTER(_vp)]),
    "llambda_cuda_device_free": (C.c_int, [_vp]),
    "llambda_cuda_set_prefill_min_tokens": (C.c_int, [C.c_int]),
    "llambda_cuda_prefill_min_tokens": (C.c_int, []),
    "llambda_cuda_moe_peer_bytes": (_sz, [_vp, C.c_int]),
    "llambda_cuda_moe_session_attach_peers": (C.c_int, [_vp, C.c_int, C.c_int,
                                                        C.POINTER(_vp), _sz]),
    "llambda_cuda_moe_forward_static_scratch": (C.c_int, [C.POINTER(MoeDesc), _vp, _sz, _vp, _vp]),
    "llambda_cuda_synth_fill_device": (C.c_int, [C.c_int, _u64, _u64, _u64, _sz, C.c_float, _vp,
                                                 _vp]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """Loads the library, building it first if the sources are newer."""
    global _lib
    with _lock:
        if _lib is None:
            from . import build as _build
            if _build.needs_build():
                _build.build()
            if not os.path.exists(LIB_PATH):
                raise LlambdaCudaError(f"{LIB_PATH} is missing and could not be built")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    return (lib().llambda_cuda_last_error() or b"").decode()


def _check(rc: int) -> int:
    if rc != 0:
        raise LlambdaCudaError(last_error() or f"llambda_cuda call failed ({rc})")
    return rc


def _f32(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def probe() -> int:
    return lib().llambda_cuda_probe()


def bridge_version() -> str:
    return lib().llambda_cuda_bridge_version().decode()


def runtime_version() -> str:
    v = lib().llambda_cuda_runtime_version()
    if v is None:
        raise LlambdaCudaError(last_error())
    return v.decode()


def sha256(data: bytes | np.ndarray) -> str:
    buf = np.frombuffer(bytes(data), np.uint8) if isinstance(data, (bytes, bytearray)) else \
        np.ascontiguousarray(data).view(np.uint8).ravel()
    out = C.create_string_buffer(65)
    _check(lib().llambda_cuda_sha256(buf.ctypes.data if buf.size else None, buf.size, out, 65))
    return out.value.decode()


def _dev_ptr(t) -> int:
    """Device pointer of a CUDA torch tensor (torch is only plumbing here), or
    a device address given as an int (e.g. from GgufFile.upload)."""
    return int(t) if isinstance(t, int) else int(t.data_ptr())


def _stream_ptr(stream) -> int | None:
    if stream is None:
        return None
    return int(getattr(stream, "cuda_stream", stream))


class ProjectionSession:
    """One GGUF tensor resident on the GPU (a projection of llambda's store)."""

    def __init__(self, handle: int, type_tag: int, ne0: int, ne1: int, ne2: int, keep=None):
        self._h = C.c_void_p(handle)
        self.type, self.ne0, self.ne1, self.ne2 = type_tag, ne0, ne1, ne2
        self._keep = keep

    @classmethod
    def from_tensor(cls, type_tag: int, ne0: int, ne1: int, data: np.ndarray, ne2: int = 1):
        data = np.ascontiguousarray(data).view(np.uint8).ravel()
        h = C.c_void_p()
        _check(lib().llambda_cuda_session_create_from_tensor(type_tag, ne0, ne1, ne2,
                                                             data.ctypes.data, data.size,
                                                             C.byref(h)))
        return cls(h.value, type_tag, ne0, ne1, ne2)

    @classmethod
    def from_file(cls, path: str):
        h = C.c_void_p()
        _check(lib().llambda_cuda_session_create(path.encode(), C.byref(h)))
        ne0 = lib().llambda_cuda_session_input_element_count(h)
        ne1 = lib().llambda_cuda_session_output_element_count(h)
        return cls(h.value, -1, ne0, ne1, 1)

    @classmethod
    def from_device(cls, type_tag: int, ne0: int, ne1: int, device_tensor, ne2: int = 1):
        """Borrows device memory (a torch CUDA tensor kept alive by the session)."""
        h = C.c_void_p()
        _check(lib().llambda_cuda_session_create_device(type_tag, ne0, ne1, ne2,
                                                        _dev_ptr(device_tensor), C.byref(h)))
        return cls(h.value, type_tag, ne0, ne1, ne2, keep=device_tensor)

    @property
    def input_element_count(self) -> int:
        return lib().llambda_cuda_session_input_element_count(self._h)

    @property
    def output_element_count(self) -> int:
        return lib().llambda_cuda_session_output_element_count(self._h)

    def run_into(self, dest: np.ndarray, x: np.ndarray) -> np.ndarray:
        x = _f32(x)
        if dest.dtype != np.float32 or not dest.flags.c_contiguous:
            raise ValueError("dest must be a contiguous float32 array")
        _check(lib().llambda_cuda_session_run(self._h, _fptr(x), x.size, _fptr(dest), dest.size))
        return dest

    def run(self, x: np.ndarray) -> np.ndarray:
        return self.run_into(np.empty(self.ne1, np.float32), x)

    def run_batch(self, x: np.ndarray) -> np.ndarray:
        x = _f32(x).reshape(-1, self.ne0)
        out = np.empty((x.shape[0], self.ne1), np.float32)
        _check(lib().llambda_cuda_session_run_batch(self._h, _fptr(x), x.shape[0], _fptr(out)))
        return out

    def run_expert(self, expert: int, x: np.ndarray) -> np.ndarray:
        x = _f32(x)
        out = np.empty(self.ne1, np.float32)
        _check(lib().llambda_cuda_session_run_expert(self._h, expert, _fptr(x), x.size,
                                                     _fptr(out), out.size))
        return out

    def run_device(self, x_dev, out_dev, tokens: int, stream=None) -> None:
        _check(lib().llambda_cuda_session_run_device(self._h, _dev_ptr(x_dev), tokens,
                                                     _dev_ptr(out_dev), _stream_ptr(stream)))

    def close(self) -> None:
        if self._h:
            lib().llambda_cuda_session_destroy(self._h)
            self._h = C.c_void_p()
        self._keep = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _tensor(type_tag, ne0, ne1, ne2, ptr) -> Tensor:
    return Tensor(type_tag, ne0, ne1, ne2, ptr or None)


class MoeSession:
    """One routed feed-forward layer (qwen3next-moe-into / nemotron-h-moe-ffn-into)."""

    def __init__(self, desc: MoeDesc, keep=()):
        self._keep = list(keep)
        self.desc = desc
        h = C.c_void_p()
        _check(lib().llambda_cuda_moe_session_create(C.byref(desc), C.byref(h)))
        self._h = h
        self.hidden = int(desc.hidden)
        self.top_k = min(int(desc.top_k), int(desc.router.ne1))

    @classmethod
    def create(cls, arch: int, hidden: int, top_k: int, tensors: dict, *, weight_scale=1.0,
               weights_norm=False, on_device=False, expert_range=(0, 0), shared_here=True,
               max_tokens=64, input_norm=None, norm_epsilon=1e-6, add_residual=False):
        """tensors: name -> (type, ne0, ne1, ne2, array); names follow GGUF:
        ffn_gate_inp, exp_probs_b.bias, ffn_gate_inp_shexp, ffn_{gate,up,down}_exps,
        ffn_{gate,up,down}_shexp, ffn_latent_{down,up} (nemotron, optional).
        Arrays are numpy (host) or CUDA torch tensors (on_device=True)."""
        keep = []

        def ptr(a):
            if a is None:
                return None
            if on_device:
                keep.append(a)
                return _dev_ptr(a)
            a = np.ascontiguousarray(a)
            keep.append(a)
            return a.ctypes.data

        def T(name):
            if name not in tensors or tensors[name] is None:
                return _tensor(0, 0, 0, 0, None)
            t, ne0, ne1, ne2, arr = tensors[name]
            return _tensor(t, ne0, ne1, ne2, ptr(arr))

        def V(name):
            v = tensors.get(name)
            return ptr(v) if v is not None else None

        d = MoeDesc()
        d.arch, d.hidden, d.top_k = arch, hidden, top_k
        d.weight_scale, d.weights_norm = weight_scale, int(bool(weights_norm))
        d.data_on_device = int(bool(on_device))
        d.router = T("ffn_gate_inp")
        d.router_bias = V("exp_probs_b.bias")
        d.shared_gate_inp = V("ffn_gate_inp_shexp")
        d.gate_exps, d.up_exps, d.down_exps = T("ffn_gate_exps"), T("ffn_up_exps"), T("ffn_down_exps")
        d.gate_shexp, d.up_shexp, d.down_shexp = T("ffn_gate_shexp"), T("ffn_up_shexp"), T("ffn_down_shexp")
        d.expert_begin, d.expert_end = expert_range
        d.shared_here = int(bool(shared_here))
        d.max_tokens = max_tokens
        d.input_norm = ptr(input_norm) if input_norm is not None else None
        d.norm_epsilon = norm_epsilon
        d.add_residual = int(bool(add_residual))
        d.latent_down, d.latent_up = T("ffn_latent_down"), T("ffn_latent_up")
        return cls(d, keep)

    def run_into(self, dest: np.ndarray, x: np.ndarray) -> np.ndarray:
        """The layer output of x written into dest (a C-contiguous float32
        array of x's shape), as the reference's run-into functions do."""
        x = _f32(x).reshape(-1, self.hidden)
        if dest.dtype != np.float32 or not dest.flags.c_contiguous or dest.size != x.size:
            raise ValueError("dest must be a C-contiguous float32 array of x's size")
        _check(lib().llambda_cuda_moe_session_run(self._h, _fptr(x), x.shape[0], _fptr(dest),
                                                  None, None))
        return dest

    def run(self, x: np.ndarray, with_routing: bool = False):
        x = _f32(x).reshape(-1, self.hidden)
        T = x.shape[0]
        out = np.empty_like(x)
        sel = np.empty((T, self.top_k), np.int32) if with_routing else None
        w = np.empty((T, self.top_k), np.float32) if with_routing else None
        _check(lib().llambda_cuda_moe_session_run(
            self._h, _fptr(x), T, _fptr(out),
            sel.ctypes.data_as(C.POINTER(C.c_int32)) if sel is not None else None,
            _fptr(w) if w is not None else None))
        return (out, sel, w) if with_routing else out

    def run_device(self, x_dev, out_dev, tokens: int, sel_dev=None, w_dev=None, stream=None):
        _check(lib().llambda_cuda_moe_session_run_device(
            self._h, _dev_ptr(x_dev), tokens, _dev_ptr(out_dev),
            _dev_ptr(sel_dev) if sel_dev is not None else None,
            _dev_ptr(w_dev) if w_dev is not None else None, _stream_ptr(stream)))

    def peer_bytes(self, world: int) -> int:
        """Bytes of the symmetric buffer `world` expert-parallel ranks need."""
        return int(lib().llambda_cuda_moe_peer_bytes(self._h, world))

    def attach_peers(self, rank: int, world: int, peer_ptrs, nbytes: int) -> None:
        """Sum every rank's partial output inside each run, over peer memory:
        peer_ptrs[r] is rank r's copy of one zero-filled symmetric buffer."""
        arr = (_vp * world)(*[int(p) for p in peer_ptrs])
        _check(lib().llambda_cuda_moe_session_attach_peers(self._h, rank, world, arr, nbytes))

    def dispatch_bytes(self, world: int, max_local_tokens: int) -> int:
        return int(lib().llambda_cuda_moe_dispatch_bytes(self._h, world, max_local_tokens))

    def attach_dispatch(self, rank: int, world: int, peer_ptrs, nbytes: int,
                        max_local_tokens: int) -> None:
        """Prefill-sized runs route this rank's own tokens to the experts'
        owners over peer memory (see llambda_cuda_moe_session_attach_dispatch)."""
        arr = (_vp * world)(*[int(p) for p in peer_ptrs])
        _check(lib().llambda_cuda_moe_session_attach_dispatch(self._h, rank, world, arr, nbytes,
                                                              max_local_tokens))

    def time_kernels(self, enable: bool = True) -> None:
        """Record CUDA events around the gate/up and routed down passes of
        every later run (a measurement aid)."""
        _check(lib().llambda_cuda_moe_session_time_kernels(self._h, int(bool(enable))))

    def kernel_ms(self) -> tuple[float, float]:
        """(gate/up, routed down) milliseconds of the last run (timing on)."""
        a, b = C.c_float(), C.c_float()
        _check(lib().llambda_cuda_moe_session_kernel_ms(self._h, C.byref(a), C.byref(b)))
        return float(a.value), float(b.value)

    def kernel_breakdown(self) -> dict:
        """Stage durations (ms) of the last timed run: router (with the
        rms-norm and the prepared gate/up input), top-k with the routing,
        gate/up pass, routed down pass, shared down pass, combine; with the
        expert-parallel reduction also the combine's phases (its first CTA):
        pushing the partial, waiting for every rank, summing."""
        a = (C.c_float * 9)()
        n = lib().llambda_cuda_moe_session_kernel_breakdown(self._h, a, 9)
        if n < 0:
            raise LlambdaCudaError(last_error())
        names = ("router", "topk", "gate_up", "down", "shared_down", "combine",
                 "combine_push", "combine_wait", "combine_sum")
        return {names[i]: float(a[i]) for i in range(n)}

    def status(self) -> int:
        rc = lib().llambda_cuda_moe_session_status(self._h)
        if rc < 0:
            raise LlambdaCudaError(last_error())
        return rc

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().llambda_cuda_moe_session_destroy(self._h)
            self._h = C.c_void_p()
        self._keep = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def synth_fill_device(type_tag: int, seed: int, stream_id: int, first: int, count: int,
                      scale: float, out_dev, stream=None) -> None:
    _check(lib().llambda_cuda_synth_fill_device(type_tag, seed, stream_id, first, count, scale,
                                                _dev_ptr(out_dev), _stream_ptr(stream)))


def set_prefill_min_tokens(tokens: int) -> None:
    """MoE runs of at least `tokens` tokens take the bf16 tensor-core prefill
    path (process-wide; values below 64 act as 64)."""
    _check(lib().llambda_cuda_set_prefill_min_tokens(int(tokens)))


def prefill_min_tokens() -> int:
    return int(lib().llambda_cuda_prefill_min_tokens())


class GgufFile:
    """A mapped, parsed GGUF file (llambda_cuda_gguf_open): tensor infos by
    name, host views of their raw bytes, and upload into a device arena."""

    def __init__(self, path: str):
        h = _vp()
        _check(lib().llambda_cuda_gguf_open(os.fsencode(path), C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib().llambda_cuda_gguf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return int(lib().llambda_cuda_gguf_tensor_count(self._h))

    def find(self, name: str) -> int:
        return int(lib().llambda_cuda_gguf_find(self._h, name.encode()))

    def info(self, index: int) -> dict:
        name = C.create_string_buffer(4096)
        t, nd = C.c_int(), C.c_uint32()
        ne = (_u64 * 4)()
        nb = _u64()
        ptr = _vp()
        _check(lib().llambda_cuda_gguf_tensor_info(self._h, index, name, 4096, C.byref(t),
                                                   C.byref(nd), ne, C.byref(nb), C.byref(ptr)))
        return {"name": name.value.decode(), "type": t.value, "dims": list(ne)[: nd.value],
                "ne": list(ne), "byte_size": nb.value, "host_ptr": ptr.value}

    def host_bytes(self, index: int) -> np.ndarray:
        """The tensor's raw bytes (a copy out of the mapping)."""
        i = self.info(index)
        buf = (C.c_uint8 * i["byte_size"]).from_address(i["host_ptr"])
        return np.frombuffer(buf, np.uint8).copy()

    def upload(self, indices) -> tuple[int, list[int]]:
        """(device arena, device pointer of each tensor); free the arena with
        device_free once no session uses it."""
        idx = (_u64 * len(indices))(*indices)
        ptrs = (_vp * len(indices))()
        arena = _vp()
        _check(lib().llambda_cuda_gguf_upload(self._h, idx, len(indices), C.byref(arena), ptrs))
        return arena.value, [p or 0 for p in ptrs]


def device_free(ptr: int) -> None:
    _check(lib().llambda_cuda_device_free(_vp(ptr)))
