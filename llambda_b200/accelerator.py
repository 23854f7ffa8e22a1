"""llambda's accelerator-backend protocol, restated on the host side, with the
B200 CUDA backend registered in it.

llambda (Common Lisp) selects per-tensor projection backends through immutable
descriptors (accelerator.lisp:3-129), keeps bindings per tensor sorted by
priority (register-model-accelerator-projection, llambda.lisp L2672-2741) and
runs them with a soft fallback: a backend error accepted by the descriptor's
error predicate unregisters that binding, warns, and moves on to the next
binding or the CPU (call-with-accelerator-runtime-fallback, L4660-4676;
gguf-model-matrix-vector-multiply-into, L4688-4741).  SBCL is not available
here, so the same protocol is mirrored in Python over the same C ABI the Lisp
descriptor file binds through CFFI (include/llambda_cuda.h); names, argument
meaning and error behaviour follow the Lisp.  The CPU path itself is not part
of this package: callers pass it in (cpu_gemv / cpu_moe), as the Lisp model
does with its own CPU kernels.

Routed experts bypass llambda's projection store today
(gguf-model-expert-matrix-vector-multiply-into, L4951-4971), so the
descriptor gains optional MoE slots (make_moe_session_function,
run_moe_function, close_moe_session_function; default None) and the model a
per-layer MoE binding table consulted at the top of the MoE blocks.
"""
from __future__ import annotations

import dataclasses
import os
import struct
import threading
import warnings
from typing import Any, Callable, Optional

import numpy as np

from . import _native as N


class AcceleratorBackendError(RuntimeError):
    """Base condition of accelerator backends (llambda's gpu-backend-error)."""


class CudaBackendError(AcceleratorBackendError):
    """The CUDA backend's condition type."""


@dataclasses.dataclass(frozen=True)
class AcceleratorBackend:
    """Immutable descriptor; every slot of accelerator.lisp:3-91 is required."""
    name: str
    display_name: str
    priority: float
    initialization_priority: float
    load_function: Callable
    available_p_function: Callable
    runtime_version_function: Callable
    bridge_version_function: Callable
    make_session_function: Callable
    close_session_function: Callable
    run_session_function: Callable
    session_input_element_count_function: Callable
    session_output_element_count_function: Callable
    error_p_function: Callable
    signal_error_function: Callable
    default_cache_directory_function: Callable
    export_projection_function: Callable
    weight_format: str
    foreign_data_sha256_function: Callable
    byte_vector_sha256_function: Callable
    # Optional MoE extension (absent from the Lisp struct; default: none).
    make_moe_session_function: Optional[Callable] = None
    run_moe_function: Optional[Callable] = None
    close_moe_session_function: Optional[Callable] = None

    def __post_init__(self):
        for f in dataclasses.fields(self):
            if f.default is dataclasses.MISSING and getattr(self, f.name) is None:
                raise TypeError(f"Accelerator backend {f.name.replace('_', ' ')} is required.")
        if not isinstance(self.priority, (int, float)):
            raise TypeError("Accelerator backend priority must be a real number.")


_backends: dict = {}
_backends_lock = threading.Lock()


def register_accelerator_backend(backend: AcceleratorBackend, replace: bool = False):
    """register-accelerator-backend, accelerator.lisp:95-104."""
    if not isinstance(backend, AcceleratorBackend):
        raise TypeError(f"Expected an accelerator backend descriptor, got {backend!r}.")
    with _backends_lock:
        if backend.name in _backends and not replace:
            raise ValueError(f"Accelerator backend {backend.name!r} is already registered.")
        _backends[backend.name] = backend
    return backend


def unregister_accelerator_backend(name: str) -> None:
    with _backends_lock:
        _backends.pop(name, None)


def find_accelerator_backend(name, required: bool = False):
    """find-accelerator-backend, accelerator.lisp:106-113."""
    b = _backends.get(name) if name is not None else None
    if required and b is None:
        raise KeyError(f"Unknown accelerator backend {name!r}. Registered backends: "
                       f"{', '.join(repr(x.name) for x in ordered_accelerator_backends())}.")
    return b


def ordered_accelerator_backends():
    """ordered-accelerator-backends, accelerator.lisp:115-120 (lower priority first)."""
    return sorted(_backends.values(), key=lambda b: b.priority)


def resolve_accelerator_backend(backend):
    return backend if isinstance(backend, AcceleratorBackend) else find_accelerator_backend(backend, True)


def accelerator_backend_error_p(backend, condition) -> bool:
    return bool(resolve_accelerator_backend(backend).error_p_function(condition))


def signal_accelerator_backend_error(backend, fmt: str, *args):
    return resolve_accelerator_backend(backend).signal_error_function(fmt, *args)


# ------------------------------------------------------------------ CUDA backend

PROJECTION_MAGIC = b"LLBCUDA1"
PROJECTION_HEADER = struct.Struct("<8sIIQQQQQ")  # 56 bytes


def write_projection_file(path: str, type_tag: int, ne0: int, ne1: int, ne2: int,
                          data: np.ndarray) -> str:
    """Writes the file llambda_cuda_session_create opens: header + raw GGUF
    tensor bytes (what export-projection-function produces for this backend,
    in place of an ONNX graph)."""
    data = np.ascontiguousarray(data).view(np.uint8).ravel()
    expect = N.row_bytes(type_tag, ne0) * ne1 * max(ne2, 1)
    if data.size != expect:
        raise ValueError(f"tensor data is {data.size} bytes, expected {expect}")
    offset = 64
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(PROJECTION_HEADER.pack(PROJECTION_MAGIC, 1, type_tag, ne0, ne1, ne2, data.size, offset))
        f.write(b"\0" * (offset - PROJECTION_HEADER.size))
        f.write(data.tobytes())
    os.replace(tmp, path)  # atomic, as the Lisp exporter's MoveFileExW (L391-400)
    return path


def _cuda_signal(fmt: str, *args):
    raise CudaBackendError(fmt % args if args else fmt)


def _cuda_make_session(model_path: str, cache_directory=None, cache_key=None):
    try:
        return N.ProjectionSession.from_file(model_path)
    except N.LlambdaCudaError as e:
        raise CudaBackendError(str(e)) from e


def _cuda_run_session(dest: np.ndarray, session, vector: np.ndarray):
    try:
        return session.run_into(dest, vector)
    except N.LlambdaCudaError as e:
        raise CudaBackendError(str(e)) from e


def _cuda_available() -> bool:
    try:
        return N.probe() == 1
    except Exception:
        return False


def _cuda_load() -> bool:
    try:
        N.lib()
        return True
    except Exception as e:  # library missing: setup fails softly (L3144-3152)
        warnings.warn(f"CUDA backend library could not be loaded: {e}")
        return False


def _cuda_export(model, tensor_name: str, path: str, python_command=None, generator_path=None):
    info = model.tensor_info(tensor_name, required=True)
    return write_projection_file(path, info.type, info.ne0, info.ne1, info.ne2, info.data)


def _cuda_sha256_bytes(data) -> str:
    return N.sha256(data)


def _cuda_make_moe_session(model, layer_index: int, max_tokens: int = 64, **kw):
    try:
        return model.make_moe_session(layer_index, max_tokens=max_tokens, **kw)
    except N.LlambdaCudaError as e:
        raise CudaBackendError(str(e)) from e


def _cuda_run_moe(dest: np.ndarray, session, inputs: np.ndarray):
    try:
        dest[...] = session.run(inputs).reshape(dest.shape)
        return dest
    except N.LlambdaCudaError as e:
        raise CudaBackendError(str(e)) from e


CUDA_BACKEND = AcceleratorBackend(
    name="cuda",
    display_name="CUDA (B200)",
    priority=5,                      # ahead of :gpu (10) and :npu (20)
    initialization_priority=30,
    load_function=_cuda_load,
    available_p_function=_cuda_available,
    runtime_version_function=lambda: N.runtime_version(),
    bridge_version_function=lambda: N.bridge_version(),
    make_session_function=_cuda_make_session,
    close_session_function=lambda s: s.close(),
    run_session_function=_cuda_run_session,
    session_input_element_count_function=lambda s: s.input_element_count,
    session_output_element_count_function=lambda s: s.output_element_count,
    error_p_function=lambda c: isinstance(c, CudaBackendError),
    signal_error_function=_cuda_signal,
    default_cache_directory_function=lambda: os.path.join(
        os.environ.get("XDG_CACHE_HOME", os.path.expanduser("~/.cache")), "llambda", "cuda"),
    export_projection_function=_cuda_export,
    weight_format="gguf-raw",
    foreign_data_sha256_function=lambda ptr, size: N.sha256(np.ctypeslib.as_array(ptr, (size,))),
    byte_vector_sha256_function=_cuda_sha256_bytes,
    make_moe_session_function=_cuda_make_moe_session,
    run_moe_function=_cuda_run_moe,
    close_moe_session_function=lambda s: s.close(),
)


# ------------------------------------------------------------------ model side

@dataclasses.dataclass
class TensorInfo:
    name: str
    type: int
    ne0: int
    ne1: int
    ne2: int
    data: np.ndarray


@dataclasses.dataclass(frozen=True)
class AcceleratorProjection:
    """accelerator-projection, llambda.lisp L2356-2364."""
    backend: AcceleratorBackend
    session: Any
    run_mutex: threading.Lock = dataclasses.field(default_factory=threading.Lock)


@dataclasses.dataclass(frozen=True)
class MoeBinding(AcceleratorProjection):
    """A layer's MoE block bound to a backend with the optional MoE slots
    (closed through close_moe_session_function)."""


class GgufModel:
    """The parts of gguf-model (L2366-2394) the projection and MoE paths use."""

    def __init__(self, tensors: dict, cpu_gemv: Callable, cpu_moe: Optional[Callable] = None,
                 kv: Optional[dict] = None):
        self.tensors = tensors
        self.cpu_gemv = cpu_gemv      # (dest, info, vector, start_row, row_count) -> dest
        self.cpu_moe = cpu_moe        # (dest, model, layer_index, inputs) -> dest
        self.kv = kv or {}
        self.accelerator_projections: dict = {}
        self.moe_bindings: dict = {}
        self.runtime_mutex = threading.Lock()
        # inference contexts in use, and the bindings unregistered while any
        # was: closed when the count drops to zero (L2517-2549, L2662-2670)
        self.active_inference_count = 0
        self.retired_bindings: list = []
        self.closed = False

    def tensor_info(self, name: str, required: bool = False) -> Optional[TensorInfo]:
        info = self.tensors.get(name)
        if required and info is None:
            raise KeyError(f"Model is missing required tensor {name!r}.")
        return info

    # -- MoE layer description from GGUF tensor names (blk.N.*)
    def make_moe_session(self, layer_index: int, max_tokens: int = 64, **kw):
        p = f"blk.{layer_index}."

        def T(name):
            i = self.tensor_info(p + name)
            return None if i is None else (i.type, i.ne0, i.ne1, i.ne2, i.data)

        def V(name):
            i = self.tensor_info(p + name)
            return None if i is None else i.data

        router = self.tensor_info(p + "ffn_gate_inp", required=True)
        arch = N.ARCH_QWEN3NEXT if self.kv.get("general.architecture", "qwen3next") == "qwen3next" \
            else N.ARCH_NEMOTRON_H_MOE
        if arch == N.ARCH_QWEN3NEXT:
            top_k = int(self.kv.get("qwen3next.expert_used_count", 10))
            scale, norm = 1.0, True
        else:
            top_k = int(self.kv["nemotron_h_moe.expert_used_count"])
            scale = float(self.kv.get("nemotron_h_moe.expert_weights_scale", 1.0))
            norm = bool(self.kv.get("nemotron_h_moe.expert_weights_norm", False))
        tensors = {"ffn_gate_inp": T("ffn_gate_inp"), "exp_probs_b.bias": V("exp_probs_b.bias"),
                   "ffn_gate_inp_shexp": V("ffn_gate_inp_shexp"),
                   "ffn_gate_exps": T("ffn_gate_exps"), "ffn_up_exps": T("ffn_up_exps"),
                   "ffn_down_exps": T("ffn_down_exps"), "ffn_gate_shexp": T("ffn_gate_shexp"),
                   "ffn_up_shexp": T("ffn_up_shexp"), "ffn_down_shexp": T("ffn_down_shexp")}
        return N.MoeSession.create(arch, router.ne0, top_k, tensors, weight_scale=scale,
                                   weights_norm=norm, max_tokens=max_tokens, **kw)


def register_model_accelerator_projection(model: GgufModel, backend, tensor_name: str,
                                          model_path: str, cache_directory=None, cache_key=None):
    """register-model-accelerator-projection, L2672-2741: make the session,
    check its element counts against the tensor, insert sorted by priority
    (copy-on-write); close the session on any failure."""
    b = resolve_accelerator_backend(backend)
    info = model.tensor_info(tensor_name, required=True)
    session = b.make_session_function(model_path, cache_directory=cache_directory,
                                      cache_key=cache_key)
    try:
        if b.session_input_element_count_function(session) != info.ne0:
            raise ValueError(f"{b.display_name} input size does not match tensor {tensor_name!r}.")
        if b.session_output_element_count_function(session) != info.ne1:
            raise ValueError(f"{b.display_name} output size does not match tensor {tensor_name!r}.")
        with model.runtime_mutex:
            cur = model.accelerator_projections.get(tensor_name, ())
            if any(p.backend.name == b.name for p in cur):
                raise ValueError(f"Tensor {tensor_name!r} already has a {b.display_name} projection.")
            table = dict(model.accelerator_projections)
            table[tensor_name] = tuple(sorted(cur + (AcceleratorProjection(b, session),),
                                              key=lambda p: p.backend.priority))
            model.accelerator_projections = table
        session = None
    finally:
        if session is not None:
            b.close_session_function(session)
    return model


def _close_retired(bindings) -> None:
    """close-retired-accelerator-projections, L2517-2530: close every
    session, then re-raise the first close error."""
    first = None
    for p in bindings:
        try:
            with p.run_mutex:
                if isinstance(p, MoeBinding):
                    p.backend.close_moe_session_function(p.session)
                else:
                    p.backend.close_session_function(p.session)
        except Exception as e:  # noqa: BLE001
            first = first or e
    if first is not None:
        raise first


def _defer_or_collect(model: "GgufModel", bindings: list) -> list:
    """defer-or-collect-accelerator-projections, L2662-2670: with inference
    contexts active the removed bindings wait on the model (closed by the
    last release); otherwise they are returned for closing now.  Called with
    the model's runtime mutex held."""
    if model.active_inference_count > 0:
        model.retired_bindings = bindings + model.retired_bindings
        return []
    return bindings


def model_accelerator_projection(model: GgufModel, backend, tensor_name: str):
    """model-accelerator-projection, L2636-2645: the tensor's binding to the
    backend, or None."""
    name = resolve_accelerator_backend(backend).name
    for p in model.accelerator_projections.get(tensor_name, ()):
        if p.backend.name == name:
            return p
    return None


def unregister_model_accelerator_projection(model: GgufModel, backend, tensor_name: str) -> bool:
    """unregister-model-accelerator-projection, L2742-2789 (close deferred
    while inference contexts are active)."""
    b = resolve_accelerator_backend(backend)
    with model.runtime_mutex:
        cur = model.accelerator_projections.get(tensor_name, ())
        keep = tuple(p for p in cur if p.backend.name != b.name)
        gone = [p for p in cur if p.backend.name == b.name]
        if gone:
            table = dict(model.accelerator_projections)
            if keep:
                table[tensor_name] = keep
            else:
                table.pop(tensor_name, None)
            model.accelerator_projections = table
        to_close = _defer_or_collect(model, gone)
    _close_retired(to_close)
    return bool(gone)


def clear_model_accelerator_projections(model: GgufModel, backend=None) -> GgufModel:
    """clear-model-accelerator-projections, L2791-2827: every binding, or
    those of one backend."""
    b = resolve_accelerator_backend(backend) if backend is not None else None
    with model.runtime_mutex:
        table, removed = {}, []
        for name, bindings in model.accelerator_projections.items():
            keep = tuple(p for p in bindings if b is not None and p.backend.name != b.name)
            removed += [p for p in bindings if p not in keep]
            if keep:
                table[name] = keep
        model.accelerator_projections = table
        to_close = _defer_or_collect(model, removed)
    _close_retired(to_close)
    return model


class InferenceContext:
    """The part of llambda's inference context (L2415-2600) the accelerator
    protocol depends on: while a context is in use, the model's unregistered
    bindings are not closed."""

    def __init__(self, model: GgufModel):
        self.model = model
        self.in_use = False
        self.closed = False
        self._mutex = threading.Lock()

    def close(self) -> None:
        """close-inference-context, L2591-2600."""
        with self._mutex:
            if self.in_use:
                raise RuntimeError("Cannot close an inference context while it is in use.")
            self.closed = True


def make_inference_context(model: GgufModel) -> InferenceContext:
    return InferenceContext(model)


def acquire_model_inference_use(model: GgufModel) -> GgufModel:
    """acquire-model-inference-use, L2532-2536."""
    with model.runtime_mutex:
        if model.closed:
            raise RuntimeError("The model is closed.")
        model.active_inference_count += 1
    return model


def release_model_inference_use(model: GgufModel) -> GgufModel:
    """release-model-inference-use, L2538-2549: the last release closes the
    bindings retired meanwhile."""
    retired = []
    with model.runtime_mutex:
        model.active_inference_count -= 1
        if model.active_inference_count < 0:
            raise RuntimeError("Model inference use count became negative.")
        if model.active_inference_count == 0:
            retired, model.retired_bindings = model.retired_bindings, []
    _close_retired(retired)
    return model


def call_with_inference_context(context: InferenceContext, function: Callable):
    """call-with-inference-context, L2551-2581."""
    with context._mutex:
        if context.closed:
            raise RuntimeError("The inference context is closed.")
        if context.in_use:
            raise RuntimeError("Inference context is already in use.")
        context.in_use = True
    acquired = False
    try:
        acquire_model_inference_use(context.model)
        acquired = True
        return function(context)
    finally:
        try:
            if acquired:
                release_model_inference_use(context.model)
        finally:
            with context._mutex:
                context.in_use = False


def close_model(model: GgufModel) -> None:
    """close-model, L2849-2880: refuses while inference contexts are active,
    then closes every projection and MoE session the model holds."""
    with model.runtime_mutex:
        if model.closed:
            return
        if model.active_inference_count > 0:
            raise RuntimeError(f"Cannot close a model while {model.active_inference_count} "
                               f"inference context(s) are active.")
        bindings = [p for ps in model.accelerator_projections.values() for p in ps]
        bindings += [p for ps in model.moe_bindings.values() for p in ps]
        bindings += model.retired_bindings
        model.accelerator_projections, model.moe_bindings, model.retired_bindings = {}, {}, []
        model.closed = True
    _close_retired(bindings)


def _cache_component(text) -> str:
    """accelerator-cache-component, L2963-2971: alphanumerics, '-' and '.'
    kept, anything else becomes '-'."""
    return "".join(c if c.isalnum() or c in "-." else "-" for c in str(text))


def model_accelerator_projection_cache_key(model: GgufModel, backend, info: TensorInfo) -> str:
    """model-accelerator-projection-cache-key, L2976-2993: bridge version,
    runtime version, weight format, type tag, dimensions and a SHA-256 of the
    tensor bytes (there is no ONNX generator script for this backend)."""
    b = resolve_accelerator_backend(backend)
    data = np.ascontiguousarray(info.data).view(np.uint8).ravel()
    return "bridge-{}-runtime-{}-weights-{}-ggml-{}-{}-{}-{}-{}".format(
        _cache_component(b.bridge_version_function()),
        _cache_component(b.runtime_version_function()),
        _cache_component(b.weight_format).lower(), info.type, info.ne0, info.ne1, info.ne2,
        b.byte_vector_sha256_function(data))


def ensure_model_accelerator_projection(model: GgufModel, backend, tensor_name: str,
                                        cache_directory: Optional[str] = None):
    """ensure-model-accelerator-projection, L3039-3066: (model, path,
    reused_p); exports the projection file into the cache unless it is
    there, then registers it.  An existing binding returns (model, None,
    True)."""
    b = resolve_accelerator_backend(backend)
    if model_accelerator_projection(model, b, tensor_name) is not None:
        return model, None, True
    info = model.tensor_info(tensor_name, required=True)
    key = model_accelerator_projection_cache_key(model, b, info)
    root = cache_directory or b.default_cache_directory_function()
    path = os.path.join(root, key, "projection.llbcuda")
    reused = os.path.exists(path)
    if not reused:
        os.makedirs(os.path.dirname(path), exist_ok=True)
        b.export_projection_function(model, tensor_name, path)
    register_model_accelerator_projection(model, b, tensor_name, path,
                                          cache_directory=root, cache_key=key)
    return model, path, reused


def enable_model_accelerator_projections(model: GgufModel, backend, tensor_names,
                                         cache_directory: Optional[str] = None) -> GgufModel:
    """enable-model-accelerator-projections, L3068-3091: all or nothing (the
    tensors added by this call are unregistered again on failure)."""
    b = resolve_accelerator_backend(backend)
    added, done = [], False
    try:
        for name in tensor_names:
            if model_accelerator_projection(model, b, name) is None:
                ensure_model_accelerator_projection(model, b, name, cache_directory)
                added.append(name)
        done = True
        return model
    finally:
        if not done:
            for name in added:
                unregister_model_accelerator_projection(model, b, name)


def call_with_accelerator_setup_fallback(backend, setup_function: Callable):
    """call-with-accelerator-setup-fallback, L3144-3152: any error during
    set-up warns and returns None (the model keeps running on what it has)."""
    b = resolve_accelerator_backend(backend)
    try:
        return setup_function()
    except Exception as condition:  # noqa: BLE001 - mirrors handler-case error
        warnings.warn(f"{b.display_name} setup failed; continuing with the next available "
                      f"backend: {condition}")
        return None


def try_enable_model_accelerator_projections(model: GgufModel, backend, tensor_names,
                                             cache_directory: Optional[str] = None):
    """try-enable-model-accelerator-projections, L3160-3208: True when every
    named projection is bound, None (with a warning) when the backend cannot
    load, is unavailable, no projection was named, or set-up fails."""
    b = resolve_accelerator_backend(backend)

    def setup():
        names = list(dict.fromkeys(tensor_names or ()))
        if not names:
            b.signal_error_function("%s acceleration was requested without any projections.",
                                    b.display_name)
        if not b.load_function():
            b.signal_error_function("%s backend library could not be loaded.", b.display_name)
        if not b.available_p_function():
            b.signal_error_function("%s acceleration is unavailable.", b.display_name)
        enable_model_accelerator_projections(model, b, names, cache_directory)
        return True

    return call_with_accelerator_setup_fallback(b, setup)


def call_with_accelerator_runtime_fallback(backend, accelerator_function, fallback_function,
                                           disable_function, tensor_name):
    """call-with-accelerator-runtime-fallback, L4660-4676."""
    b = resolve_accelerator_backend(backend)
    try:
        return accelerator_function()
    except Exception as condition:  # noqa: BLE001 - mirrors handler-case error
        if accelerator_backend_error_p(b, condition):
            disable_function()
            warnings.warn(f"{b.display_name} projection {tensor_name!r} failed and was disabled; "
                          f"using the next available backend: {condition}")
            return fallback_function()
        raise


def gguf_model_matrix_vector_multiply_into(dest: np.ndarray, model: GgufModel, tensor_name: str,
                                           vector: np.ndarray) -> np.ndarray:
    """gguf-model-matrix-vector-multiply-into, L4688-4741."""
    projections = model.accelerator_projections.get(tensor_name)

    def run_on_cpu():
        info = model.tensor_info(tensor_name, required=True)
        return model.cpu_gemv(dest, info, vector, 0, info.ne1)

    if not projections:
        return run_on_cpu()

    def run_projection_or_cpu(index):
        if index >= len(projections):
            return run_on_cpu()
        p = projections[index]

        def accel():
            with p.run_mutex:
                return p.backend.run_session_function(dest, p.session, vector)

        return call_with_accelerator_runtime_fallback(
            p.backend, accel, lambda: run_projection_or_cpu(index + 1),
            lambda: unregister_model_accelerator_projection(model, p.backend, tensor_name),
            tensor_name)

    return run_projection_or_cpu(0)


def register_model_moe_binding(model: GgufModel, backend, layer_index: int, **kw):
    """Binds a layer's MoE block to a backend that has the optional MoE slots."""
    b = resolve_accelerator_backend(backend)
    if b.make_moe_session_function is None:
        raise ValueError(f"{b.display_name} has no MoE session support.")
    session = b.make_moe_session_function(model, layer_index, **kw)
    with model.runtime_mutex:
        cur = model.moe_bindings.get(layer_index, ())
        table = dict(model.moe_bindings)
        if any(p.backend.name == b.name for p in cur):
            b.close_moe_session_function(session)
            raise ValueError(f"Layer {layer_index} already has a {b.display_name} MoE binding.")
        table[layer_index] = tuple(sorted(cur + (MoeBinding(b, session),),
                                          key=lambda p: p.backend.priority))
        model.moe_bindings = table
    return model


def unregister_model_moe_binding(model: GgufModel, backend, layer_index: int) -> None:
    b = resolve_accelerator_backend(backend)
    with model.runtime_mutex:
        cur = model.moe_bindings.get(layer_index, ())
        gone = [p for p in cur if p.backend.name == b.name]
        table = dict(model.moe_bindings)
        keep = tuple(p for p in cur if p.backend.name != b.name)
        if keep:
            table[layer_index] = keep
        else:
            table.pop(layer_index, None)
        model.moe_bindings = table
        to_close = _defer_or_collect(model, gone)
    _close_retired(to_close)


def gguf_model_moe_into(dest: np.ndarray, model: GgufModel, layer_index: int,
                        inputs: np.ndarray) -> np.ndarray:
    """The lookup added at the top of qwen3next-moe-into / nemotron-h-moe-ffn-into:
    a bound MoE session runs the layer, with the same soft fallback as
    projections, else the model's CPU MoE block."""
    bindings = model.moe_bindings.get(layer_index)

    def run_on_cpu():
        if model.cpu_moe is None:
            raise RuntimeError("no CPU MoE path was supplied to the model")
        return model.cpu_moe(dest, model, layer_index, inputs)

    if not bindings:
        return run_on_cpu()

    def attempt(index):
        if index >= len(bindings):
            return run_on_cpu()
        p = bindings[index]

        def accel():
            with p.run_mutex:
                return p.backend.run_moe_function(dest, p.session, inputs)

        return call_with_accelerator_runtime_fallback(
            p.backend, accel, lambda: attempt(index + 1),
            lambda: unregister_model_moe_binding(model, p.backend, layer_index),
            f"blk.{layer_index}.ffn")

    return attempt(0)


# Loading the backend file registers its descriptor, as accelerators/*.lisp do
# with (register-accelerator-backend ... :replace t).
register_accelerator_backend(CUDA_BACKEND, replace=True)
