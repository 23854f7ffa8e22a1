"""The accelerator-backend protocol restated in llambda_b200/accelerator.py,
tested with fake backends on the CPU the way the reference tests it:

  * accelerator-backend-protocol (tests.lisp:543-715): registration and
    priority order, projection bindings sorted by priority, a backend error
    disabling its binding (session closed, warning) and falling through to the
    next binding and then the CPU, cache-keyed ensure, closing deferred while
    inference contexts are active, set-up of an unavailable backend returning
    None;
  * accelerator-session-runs-are-serialized (tests.lisp:717-803): two threads
    on one binding never run it at the same time;
  * npu-soft-fallback / gpu-priority-and-soft-fallback (tests.lisp:1137-1220):
    the runtime and set-up fallbacks on their own.

The optional MoE slots (the per-layer MoE bindings consulted at the top of the
MoE blocks) get the same treatment.  No GPU is used: the CUDA descriptor is
only checked for its slots and its behaviour without a device.
"""
import threading
import time
import warnings

import numpy as np
import pytest

from llambda_b200 import accelerator as A


class FakeAcceleratorError(A.AcceleratorBackendError):
    pass


def fake_backend(name, priority, run, close, available=lambda: True, moe=None):
    """make-fake-accelerator-backend (tests.lisp:133-180)."""
    def signal(fmt, *args):
        raise FakeAcceleratorError(fmt % args if args else fmt)

    def unused(*a, **k):
        raise AssertionError("this fake backend's slot is not expected to run")

    run = run or unused
    close = close or unused
    kw = {}
    if moe is not None:
        kw = dict(make_moe_session_function=lambda model, layer, **k: (name, layer),
                  run_moe_function=moe, close_moe_session_function=close)
    return A.AcceleratorBackend(
        name=name, display_name=name.upper(), priority=priority,
        initialization_priority=priority, load_function=lambda: True,
        available_p_function=available, runtime_version_function=lambda: "test-runtime",
        bridge_version_function=lambda: "test-bridge",
        make_session_function=lambda path, cache_directory=None, cache_key=None: name,
        close_session_function=close, run_session_function=run,
        session_input_element_count_function=lambda s: 1,
        session_output_element_count_function=lambda s: 1,
        error_p_function=lambda c: isinstance(c, FakeAcceleratorError),
        signal_error_function=signal,
        default_cache_directory_function=lambda: "/nonexistent",
        export_projection_function=lambda model, tensor, path, **k: open(path, "wb").close(),
        weight_format="float32",
        foreign_data_sha256_function=lambda ptr, size: "fake-foreign-sha256",
        byte_vector_sha256_function=lambda data: "fake-sha256", **kw)


def cpu_gemv(dest, info, vector, start_row, row_count):
    w = np.asarray(info.data, np.float32).reshape(info.ne1, info.ne0)
    dest[:] = w @ np.asarray(vector, np.float32)
    return dest


def one_weight_model(cpu_moe=None):
    t = A.TensorInfo("test.weight", 0, 1, 1, 1, np.array([3.0], np.float32))
    return A.GgufModel({"test.weight": t}, cpu_gemv, cpu_moe)


@pytest.fixture
def registry():
    names = []

    def reg(b, replace=False):
        A.register_accelerator_backend(b, replace=replace)
        names.append(b.name)
        return b

    yield reg
    for n in names:
        A.unregister_accelerator_backend(n)


def test_accelerator_backend_protocol(registry, tmp_path):
    state = dict(gpu_fails=False, npu_fails=False, available=True, gpu_runs=0, npu_runs=0)
    closed = []

    def run_gpu(dest, session, x):
        state["gpu_runs"] += 1
        if state["gpu_fails"]:
            raise FakeAcceleratorError("simulated GPU failure")
        dest[0] = 10.0
        return dest

    def run_npu(dest, session, x):
        state["npu_runs"] += 1
        if state["npu_fails"]:
            raise FakeAcceleratorError("simulated NPU failure")
        dest[0] = 20.0
        return dest

    gpu = fake_backend("fake-gpu", 1, run_gpu, closed.append,
                       available=lambda: state["available"])
    npu = fake_backend("fake-npu", 2, run_npu, closed.append)
    registry(gpu)
    registry(npu)
    order = [b.name for b in A.ordered_accelerator_backends() if b.name.startswith("fake-")]
    assert order == ["fake-gpu", "fake-npu"]
    with pytest.raises(ValueError):
        A.register_accelerator_backend(gpu)  # already registered
    model = one_weight_model()
    x = np.array([2.0], np.float32)
    out = np.zeros(1, np.float32)
    A.register_model_accelerator_projection(model, npu, "test.weight", "fake-npu.bin")
    A.register_model_accelerator_projection(model, gpu, "test.weight", "fake-gpu.bin")
    # a replaced descriptor of the same name still finds the binding
    registry(fake_backend("fake-gpu", 1, run_gpu, closed.append), replace=True)
    assert A.model_accelerator_projection(model, "fake-gpu", "test.weight") is not None
    bindings = model.accelerator_projections["test.weight"]
    assert [p.backend for p in bindings] == [gpu, npu]  # priority order, not registration

    A.gguf_model_matrix_vector_multiply_into(out, model, "test.weight", x)
    assert out[0] == 10.0 and state["gpu_runs"] == 1 and state["npu_runs"] == 0

    state["gpu_fails"] = True
    with pytest.warns(UserWarning, match="failed and was disabled"):
        A.gguf_model_matrix_vector_multiply_into(out, model, "test.weight", x)
    assert out[0] == 20.0 and state["gpu_runs"] == 2 and state["npu_runs"] == 1
    assert "fake-gpu" in closed
    assert A.model_accelerator_projection(model, gpu, "test.weight") is None

    state["npu_fails"] = True
    with pytest.warns(UserWarning):
        A.gguf_model_matrix_vector_multiply_into(out, model, "test.weight", x)
    assert out[0] == 6.0 and state["npu_runs"] == 2  # the CPU: 3 * 2
    assert "fake-npu" in closed
    assert model.accelerator_projections == {}

    ensured, path, reused = A.ensure_model_accelerator_projection(model, gpu, "test.weight",
                                                                  str(tmp_path))
    assert ensured is model and path is not None and not reused
    assert A.model_accelerator_projection(model, "fake-gpu", "test.weight") is not None
    assert A.ensure_model_accelerator_projection(model, gpu, "test.weight",
                                                 str(tmp_path)) == (model, None, True)

    # closing is deferred while inference contexts are active
    left, right = A.make_inference_context(model), A.make_inference_context(model)
    before = closed.count("fake-gpu")

    def inner(_):
        assert model.active_inference_count == 2
        A.unregister_model_accelerator_projection(model, "fake-gpu", "test.weight")
        assert closed.count("fake-gpu") == before

    def outer(_):
        A.call_with_inference_context(right, inner)
        assert closed.count("fake-gpu") == before

    A.call_with_inference_context(left, outer)
    assert closed.count("fake-gpu") == before + 1
    left.close()
    right.close()

    # the exported file is reused: same cache key, no second export
    _, path2, reused2 = A.ensure_model_accelerator_projection(model, gpu, "test.weight",
                                                              str(tmp_path))
    assert reused2 and path2 == path
    A.unregister_model_accelerator_projection(model, gpu, "test.weight")

    state["available"] = False
    with pytest.warns(UserWarning, match="unavailable"):
        assert A.try_enable_model_accelerator_projections(model, gpu, ["test.weight"]) is None
    assert A.clear_model_accelerator_projections(model) is model
    A.close_model(model)


def test_cache_key_follows_the_tensor_bytes():
    import hashlib
    b = fake_backend("fake-key", 1, None, None)
    b = A.AcceleratorBackend(**{**b.__dict__, "byte_vector_sha256_function":
                               lambda d: hashlib.sha256(d.tobytes()).hexdigest()})
    model = one_weight_model()
    k1 = A.model_accelerator_projection_cache_key(model, b, model.tensors["test.weight"])
    model.tensors["test.weight"] = A.TensorInfo("test.weight", 0, 1, 1, 1,
                                                np.array([4.0], np.float32))
    k2 = A.model_accelerator_projection_cache_key(model, b, model.tensors["test.weight"])
    assert k1 != k2 and "bridge-test-bridge" in k1 and "weights-float32-ggml-0-1-1-1" in k1


def test_enable_rolls_back_on_failure(registry, tmp_path):
    closed = []
    b = registry(fake_backend("fake-roll", 1, lambda d, s, x: d, closed.append))
    model = one_weight_model()
    with pytest.raises(KeyError):  # the second tensor does not exist
        A.enable_model_accelerator_projections(model, b, ["test.weight", "missing.weight"],
                                               str(tmp_path))
    assert model.accelerator_projections == {} and closed == ["fake-roll"]
    with pytest.warns(UserWarning, match="without any projections"):
        assert A.try_enable_model_accelerator_projections(model, b, []) is None
    assert A.try_enable_model_accelerator_projections(model, b, ["test.weight"],
                                                      str(tmp_path)) is True
    A.close_model(model)
    assert closed == ["fake-roll", "fake-roll"]


def test_session_runs_are_serialized(registry):
    active = [0]
    peak = [0]
    runs = [0]
    closes = [0]
    lock = threading.Lock()

    def run(dest, session, x):
        with lock:
            active[0] += 1
            peak[0] = max(peak[0], active[0])
        try:
            time.sleep(0.02)
            runs[0] += 1
            dest[0] = 7.0
            return dest
        finally:
            with lock:
                active[0] -= 1

    b = registry(fake_backend("serialized", 1, run, lambda s: closes.__setitem__(0, closes[0] + 1)))
    model = one_weight_model()
    A.register_model_accelerator_projection(model, b, "test.weight", "serialized.bin")
    ready, start = threading.Barrier(3), threading.Event()
    results = [None, None]

    def worker(i):
        ready.wait()
        start.wait()
        try:
            results[i] = A.gguf_model_matrix_vector_multiply_into(
                np.zeros(1, np.float32), model, "test.weight", np.array([2.0], np.float32))
        except Exception as e:  # noqa: BLE001
            results[i] = e

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    ready.wait()
    start.set()
    for t in threads:
        t.join()
    assert [float(r[0]) for r in results] == [7.0, 7.0]
    assert runs[0] == 2 and peak[0] == 1
    A.close_model(model)
    assert closes[0] == 1


def test_runtime_and_setup_fallbacks(registry):
    gpu = registry(fake_backend("fake-gpu2", 10, None, None))
    npu = registry(fake_backend("fake-npu2", 20, None, None))
    flags = dict(gpu_disabled=False, npu_disabled=False, npu_called=False, cpu_called=False)

    def set_(k):
        return lambda: flags.__setitem__(k, True)

    def raise_(msg):
        def f():
            raise FakeAcceleratorError(msg)
        return f

    assert A.call_with_accelerator_runtime_fallback(
        gpu, lambda: "gpu", lambda: (set_("npu_called")(), "npu")[1], set_("gpu_disabled"),
        "test.weight") == "gpu"
    assert not flags["npu_called"] and not flags["gpu_disabled"]

    def npu_then_cpu(npu_fn):
        return lambda: A.call_with_accelerator_runtime_fallback(
            npu, npu_fn, lambda: (set_("cpu_called")(), "cpu")[1], set_("npu_disabled"),
            "test.weight")

    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        assert A.call_with_accelerator_runtime_fallback(
            gpu, raise_("simulated GPU failure"), npu_then_cpu(lambda: "npu"),
            set_("gpu_disabled"), "test.weight") == "npu"
        assert flags["gpu_disabled"] and not flags["npu_disabled"] and not flags["cpu_called"]
        flags.update(gpu_disabled=False, npu_disabled=False)
        assert A.call_with_accelerator_runtime_fallback(
            gpu, raise_("simulated GPU failure"), npu_then_cpu(raise_("simulated NPU failure")),
            set_("gpu_disabled"), "test.weight") == "cpu"
        assert flags["gpu_disabled"] and flags["npu_disabled"] and flags["cpu_called"]
        # set-up failures of any kind return None
        assert A.call_with_accelerator_setup_fallback(
            gpu, lambda: (_ for _ in ()).throw(RuntimeError("simulated missing bridge"))) is None

    # an error the backend does not claim is not a fallback case: it propagates
    flags["gpu_disabled"] = False
    with pytest.raises(ZeroDivisionError):
        A.call_with_accelerator_runtime_fallback(gpu, lambda: 1 / 0, lambda: "npu",
                                                 set_("gpu_disabled"), "test.weight")
    assert not flags["gpu_disabled"]


def test_moe_binding_falls_back_to_the_next_binding_and_the_cpu(registry):
    state = dict(a_fails=False, b_fails=False)
    closed = []

    def moe_run(tag, key):
        def run(dest, session, inputs):
            if state[key]:
                raise FakeAcceleratorError(f"simulated {tag} failure")
            dest[...] = {"a": 1.0, "b": 2.0}[tag]
            return dest
        return run

    a = registry(fake_backend("moe-a", 1, None, closed.append, moe=moe_run("a", "a_fails")))
    b = registry(fake_backend("moe-b", 2, None, closed.append, moe=moe_run("b", "b_fails")))
    plain = registry(fake_backend("moe-none", 3, None, closed.append))

    def cpu_moe(dest, model, layer, inputs):
        dest[...] = -1.0
        return dest

    model = one_weight_model(cpu_moe)
    x = np.zeros((2, 4), np.float32)
    out = np.zeros((2, 4), np.float32)
    assert A.gguf_model_moe_into(out, model, 0, x)[0, 0] == -1.0  # no binding: the CPU block
    with pytest.raises(ValueError, match="no MoE session support"):
        A.register_model_moe_binding(model, plain, 0)
    A.register_model_moe_binding(model, b, 0)
    A.register_model_moe_binding(model, a, 0)
    with pytest.raises(ValueError, match="already has"):
        A.register_model_moe_binding(model, a, 0)
    assert [p.backend.name for p in model.moe_bindings[0]] == ["moe-a", "moe-b"]
    assert A.gguf_model_moe_into(out, model, 0, x)[0, 0] == 1.0
    assert A.gguf_model_moe_into(out, model, 1, x)[0, 0] == -1.0  # other layers: CPU
    state["a_fails"] = True
    with pytest.warns(UserWarning, match="disabled"):
        assert A.gguf_model_moe_into(out, model, 0, x)[0, 0] == 2.0
    assert ("moe-a", 0) in closed
    assert [p.backend.name for p in model.moe_bindings[0]] == ["moe-b"]
    state["b_fails"] = True
    with pytest.warns(UserWarning):
        assert A.gguf_model_moe_into(out, model, 0, x)[0, 0] == -1.0
    assert ("moe-b", 0) in closed and model.moe_bindings == {}

    # a binding retired while an inference context is active closes on release
    A.register_model_moe_binding(model, a, 0)
    ctx = A.make_inference_context(model)
    before = closed.count(("moe-a", 0))

    def body(_):
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            A.gguf_model_moe_into(out, model, 0, x)  # moe-a still fails: retired
        assert closed.count(("moe-a", 0)) == before
    A.call_with_inference_context(ctx, body)
    assert closed.count(("moe-a", 0)) == before + 1
    with pytest.raises(RuntimeError, match="already in use"):
        A.call_with_inference_context(ctx, lambda c: A.call_with_inference_context(c, None))
    A.close_model(model)


def test_close_model_refuses_while_a_context_is_active(registry):
    b = registry(fake_backend("fake-close", 1, lambda d, s, x: d, lambda s: None))
    model = one_weight_model()
    A.register_model_accelerator_projection(model, b, "test.weight", "p.bin")
    ctx = A.make_inference_context(model)

    def body(_):
        with pytest.raises(RuntimeError, match="Cannot close a model"):
            A.close_model(model)
    A.call_with_inference_context(ctx, body)
    A.close_model(model)
    with pytest.raises(RuntimeError, match="closed"):
        A.acquire_model_inference_use(model)


def test_cuda_descriptor_is_registered_with_every_slot():
    b = A.find_accelerator_backend("cuda", required=True)
    assert b is A.CUDA_BACKEND
    assert b.priority < 10  # ahead of llambda's :gpu (10) and :npu (20)
    assert b.make_moe_session_function and b.run_moe_function and b.close_moe_session_function
    assert b.error_p_function(A.CudaBackendError("x")) and not b.error_p_function(ValueError())
    with pytest.raises(A.CudaBackendError, match="unavailable 3"):
        b.signal_error_function("unavailable %d", 3)


def test_cuda_setup_without_a_device_falls_back(tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    model = one_weight_model()
    with pytest.warns(UserWarning, match="unavailable"):
        assert A.try_enable_model_accelerator_projections(model, "cuda", ["test.weight"],
                                                          str(tmp_path)) is None
    assert model.accelerator_projections == {}
