// C ABI of the llambda B200 backend (declarations and contract in
// include/llambda_cuda.h).  Host-side session management: uploads raw GGUF
// tensors once, keeps one CUDA stream and pinned bounce buffers per session,
// serialises calls per session, and reports failures through a status int
// plus a thread-local message, as llambda's ONNX bridge does
// (native/llambda_npu.cpp:24, 43-49).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/llambda_cuda.h"
#include "kernels.h"

extern "C" void lb_sha256_hex(const void* data, size_t n, char out[65]);

namespace {

thread_local std::string g_last_error;

struct Failure : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void set_error(const std::string& m) { g_last_error = m; }

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear a sticky launch error where possible
    throw Failure(std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                  cudaGetErrorString(e) + ")");
  }
}

size_t row_bytes(int type, uint64_t ne0) {
  switch (type) {
    case LLAMBDA_CUDA_TYPE_F32: return ne0 * 4;
    case LLAMBDA_CUDA_TYPE_Q4_K: return ne0 % 256 ? 0 : ne0 / 256 * 144;
    case LLAMBDA_CUDA_TYPE_Q6_K: return ne0 % 256 ? 0 : ne0 / 256 * 210;
    case LLAMBDA_CUDA_TYPE_Q5_K: return ne0 % 256 ? 0 : ne0 / 256 * 176;
    case LLAMBDA_CUDA_TYPE_Q5_0: return ne0 % 32 ? 0 : ne0 / 32 * 22;
    case LLAMBDA_CUDA_TYPE_Q8_0: return ne0 % 32 ? 0 : ne0 / 32 * 34;
    default: return 0;
  }
}

const char* type_name(int type) {
  switch (type) {
    case LLAMBDA_CUDA_TYPE_F32: return "F32";
    case LLAMBDA_CUDA_TYPE_Q4_K: return "Q4_K";
    case LLAMBDA_CUDA_TYPE_Q6_K: return "Q6_K";
    case LLAMBDA_CUDA_TYPE_Q5_K: return "Q5_K";
    case LLAMBDA_CUDA_TYPE_Q5_0: return "Q5_0";
    case LLAMBDA_CUDA_TYPE_Q8_0: return "Q8_0";
    default: return "unsupported";
  }
}

bool block32(int type) {
  return type == LLAMBDA_CUDA_TYPE_Q5_0 || type == LLAMBDA_CUDA_TYPE_Q8_0;
}

// Types of the MoE layer's tensors (the K-quants and the F32 router); a
// projection session (and a latent projection of a MoE layer) also takes
// Q5_K, Q5_0 and Q8_0 rows (projection = true).
void require_rows(int type, uint64_t ne0, const char* what, bool projection = false) {
  if (type != LLAMBDA_CUDA_TYPE_F32 && type != LLAMBDA_CUDA_TYPE_Q4_K &&
      type != LLAMBDA_CUDA_TYPE_Q6_K &&
      !(projection && (block32(type) || type == LLAMBDA_CUDA_TYPE_Q5_K)))
    throw Failure(std::string(what) + ": unsupported GGML type tag " + std::to_string(type));
  if (!row_bytes(type, ne0))
    throw Failure(std::string(what) + ": " + type_name(type) + " rows need a multiple of " +
                  (block32(type) ? "32" : "256") + " columns, got " + std::to_string(ne0));
}

int current_device() {
  int d = 0;
  cuda_check(cudaGetDevice(&d), "cudaGetDevice");
  return d;
}

void require_b200(int dev) {
  cudaDeviceProp p;
  cuda_check(cudaGetDeviceProperties(&p, dev), "cudaGetDeviceProperties");
  if (p.major != 10 || p.minor != 0)
    throw Failure(std::string("device ") + p.name + " is sm_" + std::to_string(p.major) +
                  std::to_string(p.minor) + "; this library is built for sm_100a (B200)");
}

// Device allocation with 256 bytes of slack: the Q6_K loaders read up to
// 4 bytes past a 16-byte chunk inside a block, never past the tensor, but the
// slack keeps every read of a tensor's last block inside the allocation.
void* dev_alloc(size_t bytes) {
  void* p = nullptr;
  cuda_check(cudaMalloc(&p, bytes + 256), "cudaMalloc");
  return p;
}

void validate_scales(int type, const void* dev, size_t bytes, cudaStream_t s, const char* what) {
  if (type != LLAMBDA_CUDA_TYPE_Q4_K && type != LLAMBDA_CUDA_TYPE_Q6_K &&
      type != LLAMBDA_CUDA_TYPE_Q5_K && !block32(type))
    return;
  const size_t blocks =
      bytes / (type == LLAMBDA_CUDA_TYPE_Q4_K   ? 144
               : type == LLAMBDA_CUDA_TYPE_Q6_K ? 210
               : type == LLAMBDA_CUDA_TYPE_Q5_K ? 176
               : type == LLAMBDA_CUDA_TYPE_Q5_0 ? 22
                                                : 34);
  unsigned* bad = nullptr;
  cuda_check(cudaMalloc(&bad, sizeof(unsigned)), "cudaMalloc");
  unsigned host = 0;
  cudaError_t e = cudaMemsetAsync(bad, 0, sizeof(unsigned), s);
  if (e == cudaSuccess) e = lb::check_fp16_scales(type, dev, blocks, bad, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&host, bad, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(bad);
  cuda_check(e, "fp16 scale check");
  if (host)
    throw Failure(std::string(what) + ": " + std::to_string(host) +
                  " block(s) have an Inf/NaN fp16 scale (unsupported fp16 special value)");
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cuda_check(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// Pinned host bounce buffer, grown on demand.
// [p, p + bytes) lies in page-locked host memory (cudaHostAlloc'd or
// registered), so the GPU can copy it by DMA without staging.
bool page_locked(const void* p, size_t bytes) {
  auto locked = [](const void* q) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
      cudaGetLastError();  // clear the sticky-free error of an unknown pointer
      return false;
    }
    return a.type == cudaMemoryTypeHost;
  };
  return bytes && locked(p) && locked(static_cast<const char*>(p) + bytes - 1);
}

struct Pinned {
  void* p = nullptr;
  size_t n = 0;
  void* get(size_t bytes) {
    if (bytes > n) {
      if (p) cudaFreeHost(p);
      p = nullptr;
      n = 0;
      cuda_check(cudaMallocHost(&p, bytes), "cudaMallocHost");
      n = bytes;
    }
    return p;
  }
  ~Pinned() {
    if (p) cudaFreeHost(p);
  }
};

struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  void* get(size_t bytes) {
    if (bytes > n) {
      if (p) cudaFree(p);
      p = nullptr;
      n = 0;
      cuda_check(cudaMalloc(&p, bytes), "cudaMalloc");
      n = bytes;
    }
    return p;
  }
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

template <typename F>
int guarded(F&& f) {
  try {
    g_last_error.clear();
    return f();
  } catch (const std::exception& e) {
    set_error(e.what());
    return -1;
  } catch (...) {
    set_error("unknown error");
    return -1;
  }
}

}  // namespace

struct llambda_cuda_session {
  int type = 0;
  uint64_t ne0 = 0, ne1 = 0, ne2 = 1;
  size_t rb = 0;
  int device = 0;
  void* weights = nullptr;
  bool owned = false;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  Pinned hin, hout;
  DevBuf din, dout, dxp;
  int* status = nullptr;  // device status word of the GEMV kernels
  ~llambda_cuda_session() {
    if (stream) cudaStreamDestroy(stream);
    if (owned && weights) cudaFree(weights);
    if (status) cudaFree(status);
  }
};

namespace {

// The GEMV of `tokens` device vectors through the session's scratch.
void session_launch(llambda_cuda_session* s, const uint8_t* W, const float* din, size_t tokens,
                    float* dout, cudaStream_t st) {
  const int K = (int)s->ne0;
  float* xp = nullptr;
  if (s->type == LLAMBDA_CUDA_TYPE_Q4_K || s->type == LLAMBDA_CUDA_TYPE_Q6_K)
    xp = static_cast<float*>(s->dxp.get(lb::xprep_floats(K, (int)tokens) * 4));
  cuda_check(lb::launch_projection(s->type, W, s->rb, (int)s->ne1, K, din, (long)K, K,
                                   (int)tokens, dout, (long)s->ne1, xp, s->status, st),
             "GEMV launch");
}

void require_aligned16(const void* p, const char* what) {
  if (reinterpret_cast<uintptr_t>(p) & 15)
    throw Failure(std::string(what) + ": device pointers must be 16-byte aligned.");
}

}  // namespace

struct llambda_cuda_moe_session {
  lb::MoeDevice m{};
  lb::MoeWork w{};
  lb::SlabMaps maps{};  // tensor maps of the gate/up matrices, built once
  int device = 0;
  int max_tokens = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  std::vector<void*> owned;
  void* work = nullptr;
  Pinned hx, hout, hsel, hw;
  DevBuf dx, dout, dsel, dw;
  // kernel timing, when enabled (launch_moe's six marks)
  cudaEvent_t marks[7] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  unsigned long long* ep_stamps = nullptr;  // combine phase stamps (timing, expert parallel)
  bool timing = false;
  // The host-buffer call (copies in, the layer's kernels, copies out, status)
  // as one CUDA graph, captured for one token count and replayed while the
  // staging buffers stay where they are.
  Pinned hstatus;
  cudaGraphExec_t graph = nullptr;
  int graph_tokens = 0;
  int eager_tokens = 0;  // the first call of a token count runs eagerly (fills the caches)
  const void* graph_key[2] = {nullptr, nullptr};
  int graph_prefill_min = 0;  // the prefill threshold the graph was captured under
  void drop_graph() {
    if (graph) cudaGraphExecDestroy(graph);
    graph = nullptr;
    graph_tokens = 0;
  }
  ~llambda_cuda_moe_session() {
    drop_graph();
    for (cudaEvent_t e : marks)
      if (e) cudaEventDestroy(e);
    if (stream) cudaStreamDestroy(stream);
    for (void* p : owned) cudaFree(p);
    if (work) cudaFree(work);
  }
};

extern "C" {

int llambda_cuda_probe(void) {
  try {
    g_last_error.clear();
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver || n == 0) {
      cudaGetLastError();
      set_error(std::string("No usable CUDA device: ") + cudaGetErrorString(e));
      return 0;
    }
    cuda_check(e, "cudaGetDeviceCount");
    try {
      require_b200(current_device());
    } catch (const Failure& f) {
      set_error(f.what());
      return 0;
    }
    return 1;
  } catch (const std::exception& e) {
    set_error(e.what());
    return -1;
  }
}

const char* llambda_cuda_bridge_version(void) { return "cuda-sm100a-1"; }

const char* llambda_cuda_runtime_version(void) {
  try {
    g_last_error.clear();
    thread_local std::string v;
    int rt = 0, drv = 0;
    cuda_check(cudaRuntimeGetVersion(&rt), "cudaRuntimeGetVersion");
    cuda_check(cudaDriverGetVersion(&drv), "cudaDriverGetVersion");
    char buf[256];
    std::snprintf(buf, sizeof(buf), "CUDA runtime %d.%d, driver %d.%d", rt / 1000, (rt % 1000) / 10,
                  drv / 1000, (drv % 1000) / 10);
    v = buf;
    int n = 0;
    if (cudaGetDeviceCount(&n) == cudaSuccess && n > 0) {
      cudaDeviceProp p;
      if (cudaGetDeviceProperties(&p, current_device()) == cudaSuccess)
        v += std::string(", ") + p.name + " sm_" + std::to_string(p.major) + std::to_string(p.minor);
    } else {
      cudaGetLastError();
    }
    return v.c_str();
  } catch (const std::exception& e) {
    set_error(e.what());
    return nullptr;
  }
}

const char* llambda_cuda_last_error(void) { return g_last_error.c_str(); }

int llambda_cuda_sha256(const void* data, size_t data_size, char* output, size_t output_size) {
  if ((!data && data_size != 0) || !output || output_size < 65) {
    set_error("SHA-256 requires input data and a 65-byte output buffer.");
    return -1;
  }
  g_last_error.clear();
  lb_sha256_hex(data, data_size, output);
  return 0;
}

static int session_make(int type, uint64_t ne0, uint64_t ne1, uint64_t ne2, const void* data,
                        size_t data_size, bool on_device, llambda_cuda_session** result) {
  if (!result) {
    set_error("A result pointer is required.");
    return -1;
  }
  *result = nullptr;
  return guarded([&] {
    if (!data) throw Failure("Tensor data is required.");
    if (ne0 == 0 || ne1 == 0) throw Failure("Tensor dimensions must be positive.");
    if (ne2 == 0) ne2 = 1;
    require_rows(type, ne0, "projection tensor", true);
    const size_t rb = row_bytes(type, ne0);
    const size_t bytes = rb * ne1 * ne2;
    if (!on_device && data_size != bytes)
      throw Failure("Tensor data size " + std::to_string(data_size) + " does not match " +
                    std::to_string(bytes) + " bytes of " + type_name(type) + " data.");
    if (ne1 > 0x7fffffffull || ne0 > 0x7fffffffull) throw Failure("Tensor too large.");
    auto s = new llambda_cuda_session();
    try {
      s->type = type;
      s->ne0 = ne0;
      s->ne1 = ne1;
      s->ne2 = ne2;
      s->rb = rb;
      s->device = current_device();
      require_b200(s->device);
      cuda_check(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate");
      cuda_check(cudaMalloc(&s->status, sizeof(int)), "cudaMalloc");
      cuda_check(cudaMemsetAsync(s->status, 0, sizeof(int), s->stream), "memset");
      if (on_device) {
        require_aligned16(data, "projection tensor");
        s->weights = const_cast<void*>(data);
        s->owned = false;
      } else {
        s->weights = dev_alloc(bytes);
        s->owned = true;
        cuda_check(cudaMemcpyAsync(s->weights, data, bytes, cudaMemcpyHostToDevice, s->stream),
                   "upload tensor");
      }
      validate_scales(type, s->weights, bytes, s->stream, "projection tensor");
    } catch (...) {
      delete s;
      throw;
    }
    *result = s;
    return 0;
  });
}

int llambda_cuda_session_create_from_tensor(int type, uint64_t ne0, uint64_t ne1, uint64_t ne2,
                                            const void* data, size_t data_size,
                                            llambda_cuda_session** result) {
  return session_make(type, ne0, ne1, ne2, data, data_size, false, result);
}

int llambda_cuda_session_create_device(int type, uint64_t ne0, uint64_t ne1, uint64_t ne2,
                                       const void* device_data, llambda_cuda_session** result) {
  return session_make(type, ne0, ne1, ne2, device_data, 0, true, result);
}

int llambda_cuda_session_create(const char* model_path, llambda_cuda_session** result) {
  if (!model_path || !result) {
    set_error("Model path and result pointer are required.");
    return -1;
  }
  *result = nullptr;
  std::vector<unsigned char> data;
  uint32_t type = 0;
  uint64_t ne0 = 0, ne1 = 0, ne2 = 0;
  int rc = guarded([&] {
    FILE* f = std::fopen(model_path, "rb");
    if (!f) throw Failure(std::string("Cannot open projection file ") + model_path);
    struct Closer {
      FILE* f;
      ~Closer() { std::fclose(f); }
    } closer{f};
    unsigned char hdr[56];
    if (std::fread(hdr, 1, sizeof(hdr), f) != sizeof(hdr) || std::memcmp(hdr, "LLBCUDA1", 8) != 0)
      throw Failure(std::string("Not a llambda CUDA projection file: ") + model_path);
    auto u32 = [&](int o) {
      uint32_t v;
      std::memcpy(&v, hdr + o, 4);
      return v;
    };
    auto u64 = [&](int o) {
      uint64_t v;
      std::memcpy(&v, hdr + o, 8);
      return v;
    };
    if (u32(8) != 1) throw Failure("Unsupported projection file version.");
    type = u32(12);
    ne0 = u64(16);
    ne1 = u64(24);
    ne2 = u64(32);
    const uint64_t nbytes = u64(40), offset = u64(48);
    require_rows((int)type, ne0, "projection file", true);
    if (nbytes != row_bytes((int)type, ne0) * ne1 * (ne2 ? ne2 : 1))
      throw Failure("Projection file data size does not match its dimensions.");
    if (offset < sizeof(hdr) || std::fseek(f, (long)offset, SEEK_SET) != 0)
      throw Failure("Projection file data offset is invalid.");
    data.resize(nbytes);
    if (std::fread(data.data(), 1, nbytes, f) != nbytes)
      throw Failure("Projection file is truncated.");
    return 0;
  });
  if (rc) return rc;
  return session_make((int)type, ne0, ne1, ne2, data.data(), data.size(), false, result);
}

void llambda_cuda_session_destroy(llambda_cuda_session* session) {
  if (!session) return;
  try {
    DeviceGuard g(session->device);
    if (session->stream) cudaStreamSynchronize(session->stream);
    delete session;
  } catch (...) {
    delete session;
  }
}

size_t llambda_cuda_session_input_element_count(const llambda_cuda_session* s) {
  return s ? s->ne0 : 0;
}

size_t llambda_cuda_session_output_element_count(const llambda_cuda_session* s) {
  return s ? s->ne1 : 0;
}

static int session_run_rows(llambda_cuda_session* s, int expert, const float* input, size_t tokens,
                            float* output) {
  return guarded([&] {
    std::lock_guard<std::mutex> lock(s->mu);
    DeviceGuard g(s->device);
    if (expert < 0 || (uint64_t)expert >= s->ne2)
      throw Failure("Expert index " + std::to_string(expert) + " is out of range for a tensor with " +
                    std::to_string(s->ne2) + " experts.");
    const size_t in_bytes = tokens * s->ne0 * 4, out_bytes = tokens * s->ne1 * 4;
    // page-locked caller buffers are copied directly, pageable ones staged
    const bool direct_in = page_locked(input, in_bytes), direct_out = page_locked(output, out_bytes);
    float* hin = direct_in ? nullptr : static_cast<float*>(s->hin.get(in_bytes));
    float* hout = direct_out ? output : static_cast<float*>(s->hout.get(out_bytes));
    float* din = static_cast<float*>(s->din.get(in_bytes));
    float* dout = static_cast<float*>(s->dout.get(out_bytes));
    if (!direct_in) std::memcpy(hin, input, in_bytes);
    cuda_check(cudaMemcpyAsync(din, direct_in ? input : hin, in_bytes, cudaMemcpyHostToDevice,
                               s->stream),
               "input copy");
    const uint8_t* W = static_cast<const uint8_t*>(s->weights) + (size_t)expert * s->ne1 * s->rb;
    session_launch(s, W, din, tokens, dout, s->stream);
    int status = 0;
    cuda_check(cudaMemcpyAsync(hout, dout, out_bytes, cudaMemcpyDeviceToHost, s->stream), "output copy");
    cuda_check(cudaMemcpyAsync(&status, s->status, sizeof(int), cudaMemcpyDeviceToHost, s->stream),
               "status copy");
    cuda_check(cudaStreamSynchronize(s->stream), "GEMV");
    if (status) {
      cudaMemsetAsync(s->status, 0, sizeof(int), s->stream);
      throw Failure("A GEMV shared-memory stage wait timed out (device status " +
                    std::to_string(status) + ").");
    }
    if (!direct_out) std::memcpy(output, hout, out_bytes);
    return 0;
  });
}

int llambda_cuda_session_run(llambda_cuda_session* session, const float* input,
                             size_t input_element_count, float* output,
                             size_t output_element_count) {
  if (!session || !input || !output) {
    set_error("Session, input, and output are required.");
    return -1;
  }
  if (input_element_count != session->ne0 || output_element_count != session->ne1) {
    set_error("Input or output element count does not match the projection tensor.");
    return -1;
  }
  return session_run_rows(session, 0, input, 1, output);
}

int llambda_cuda_session_run_batch(llambda_cuda_session* session, const float* input,
                                   size_t tokens, float* output) {
  if (!session || !input || !output || tokens == 0) {
    set_error("Session, input, output and a positive token count are required.");
    return -1;
  }
  return session_run_rows(session, 0, input, tokens, output);
}

int llambda_cuda_session_run_expert(llambda_cuda_session* session, int expert, const float* input,
                                    size_t input_element_count, float* output,
                                    size_t output_element_count) {
  if (!session || !input || !output) {
    set_error("Session, input, and output are required.");
    return -1;
  }
  if (input_element_count != session->ne0 || output_element_count != session->ne1) {
    set_error("Input or output element count does not match the expert tensor.");
    return -1;
  }
  return session_run_rows(session, expert, input, 1, output);
}

int llambda_cuda_session_run_device(llambda_cuda_session* s, const float* device_input,
                                    size_t tokens, float* device_output, void* cuda_stream) {
  if (!s || !device_input || !device_output || tokens == 0) {
    set_error("Session, device input/output and a positive token count are required.");
    return -1;
  }
  return guarded([&] {
    DeviceGuard g(s->device);
    std::lock_guard<std::mutex> lock(s->mu);
    session_launch(s, static_cast<const uint8_t*>(s->weights), device_input, tokens,
                   device_output, static_cast<cudaStream_t>(cuda_stream));
    return 0;
  });
}

// ------------------------------------------------------------------ MoE

static void check_tensor(const llambda_cuda_tensor& t, const char* what, bool required) {
  if (!t.data) {
    if (required) throw Failure(std::string("MoE tensor ") + what + " is required.");
    return;
  }
  require_rows(t.type, t.ne0, what);
  if (t.type == LLAMBDA_CUDA_TYPE_F32 && std::strcmp(what, "ffn_gate_inp") != 0)
    throw Failure(std::string("MoE tensor ") + what + " must be Q4_K or Q6_K.");
}

int llambda_cuda_moe_session_create(const llambda_cuda_moe_desc* d,
                                    llambda_cuda_moe_session** result) {
  if (!result) {
    set_error("A result pointer is required.");
    return -1;
  }
  *result = nullptr;
  if (!d) {
    set_error("A MoE descriptor is required.");
    return -1;
  }
  return guarded([&] {
    if (d->arch != LLAMBDA_CUDA_ARCH_QWEN3NEXT && d->arch != LLAMBDA_CUDA_ARCH_NEMOTRON_H_MOE)
      throw Failure("Unknown MoE architecture " + std::to_string(d->arch));
    const bool qwen = d->arch == LLAMBDA_CUDA_ARCH_QWEN3NEXT;
    const uint64_t H = d->hidden;
    if (!H || H > (1u << 20)) throw Failure("MoE hidden size must be positive.");
    if (!d->router.data || d->router.type != LLAMBDA_CUDA_TYPE_F32)
      throw Failure("MoE router ffn_gate_inp must be an F32 tensor.");
    if (d->router.ne0 != H) throw Failure("Router row width does not match the hidden size.");
    const uint64_t E = d->router.ne1;
    if (E == 0 || E > 1024) throw Failure("MoE expert count must be in 1..1024.");
    check_tensor(d->up_exps, "ffn_up_exps", true);
    check_tensor(d->down_exps, "ffn_down_exps", true);
    check_tensor(d->gate_exps, "ffn_gate_exps", qwen);
    const bool shared = d->up_shexp.data != nullptr;
    if (shared) {
      check_tensor(d->up_shexp, "ffn_up_shexp", true);
      check_tensor(d->down_shexp, "ffn_down_shexp", true);
      check_tensor(d->gate_shexp, "ffn_gate_shexp", qwen);
      if (qwen && !d->shared_gate_inp) throw Failure("ffn_gate_inp_shexp is required.");
    }
    const uint64_t I = d->up_exps.ne1;
    auto dims = [&](const llambda_cuda_tensor& t, uint64_t min_ne0, uint64_t ne1, uint64_t ne2,
                    const char* what) {
      if (t.ne0 < min_ne0 || t.ne1 != ne1 || (ne2 && (t.ne2 ? t.ne2 : 1) != ne2))
        throw Failure(std::string("MoE tensor ") + what + " has unexpected dimensions.");
    };
    // latent projections: the experts' input and output width is L
    const bool latent = d->latent_down.data || d->latent_up.data;
    uint64_t XW = H;  // width of the routed experts' input and output
    if (latent) {
      if (qwen) throw Failure("Latent projections are only defined for nemotron_h_moe.");
      if (!d->latent_down.data || !d->latent_up.data)
        throw Failure("ffn_latent_down and ffn_latent_up must be given together.");
      require_rows(d->latent_down.type, d->latent_down.ne0, "ffn_latent_down", true);
      require_rows(d->latent_up.type, d->latent_up.ne0, "ffn_latent_up", true);
      XW = d->latent_down.ne1;
      if (!XW || XW > (1u << 20)) throw Failure("ffn_latent_down has no rows.");
      dims(d->latent_down, H, XW, 1, "ffn_latent_down");
      dims(d->latent_up, XW, H, 1, "ffn_latent_up");
      if ((d->latent_down.type == LLAMBDA_CUDA_TYPE_F32 && d->latent_down.ne0 != H) ||
          (d->latent_up.type == LLAMBDA_CUDA_TYPE_F32 && d->latent_up.ne0 != XW))
        throw Failure("F32 latent projections must have exactly the input's width.");
    }
    dims(d->up_exps, XW, I, E, "ffn_up_exps");
    if (qwen) {
      dims(d->gate_exps, H, I, E, "ffn_gate_exps");
      if (d->gate_exps.ne0 != d->up_exps.ne0 || d->gate_exps.type != d->up_exps.type)
        throw Failure("ffn_gate_exps and ffn_up_exps must share type and width.");
    }
    dims(d->down_exps, I, XW, E, "ffn_down_exps");
    uint64_t Ish = 0;
    if (shared) {
      Ish = d->up_shexp.ne1;
      dims(d->up_shexp, H, Ish, 0, "ffn_up_shexp");
      dims(d->down_shexp, Ish, H, 0, "ffn_down_shexp");
      if (qwen) {
        dims(d->gate_shexp, H, Ish, 0, "ffn_gate_shexp");
        if (d->gate_shexp.type != d->up_shexp.type || d->gate_shexp.ne0 != d->up_shexp.ne0)
          throw Failure("ffn_gate_shexp and ffn_up_shexp must share type and width.");
      }
      if (d->up_shexp.type != d->up_exps.type || d->down_shexp.type != d->down_exps.type)
        throw Failure("Shared and routed expert tensors must share their types.");
    }
    const int top_k = (int)std::min<uint64_t>((uint64_t)std::max(d->top_k, 1), E);
    if (d->top_k < 1 || top_k > 32) throw Failure("top_k must be in 1..32.");
    int eb = d->expert_begin, ee = d->expert_end;
    if (eb == 0 && ee == 0) ee = (int)E;
    if (eb < 0 || ee > (int)E || eb >= ee) throw Failure("Invalid owned expert range.");
    if (d->max_tokens < 1 || (int64_t)d->max_tokens * top_k > 65536)
      throw Failure("max_tokens must be positive and max_tokens * top_k at most 65536.");

    auto s = new llambda_cuda_moe_session();
    try {
      s->device = current_device();
      require_b200(s->device);
      cuda_check(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate");
      const cudaMemcpyKind kind =
          d->data_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
      auto upload = [&](const void* src, size_t bytes) -> void* {
        void* p = dev_alloc(bytes);
        s->owned.push_back(p);
        cuda_check(cudaMemcpyAsync(p, src, bytes, kind, s->stream), "upload");
        return p;
      };
      // Expert tensors: only the owned experts [eb, ee) are kept on this device.
      auto experts = [&](const llambda_cuda_tensor& t, const char* what) -> const uint8_t* {
        if (!t.data) return nullptr;
        const size_t per = row_bytes(t.type, t.ne0) * t.ne1;
        const size_t bytes = per * (size_t)(ee - eb);
        const uint8_t* src = static_cast<const uint8_t*>(t.data) + per * (size_t)eb;
        const uint8_t* p;
        if (d->data_on_device) {
          require_aligned16(t.data, what);
          p = src;  // borrowed
        } else {
          p = static_cast<const uint8_t*>(upload(src, bytes));
        }
        validate_scales(t.type, p, bytes, s->stream, what);
        return p - per * (size_t)eb;  // indexable by global expert id in [eb, ee)
      };
      auto plain = [&](const llambda_cuda_tensor& t, const char* what) -> const uint8_t* {
        if (!t.data) return nullptr;
        const size_t bytes = row_bytes(t.type, t.ne0) * t.ne1;
        if (d->data_on_device) require_aligned16(t.data, what);
        const uint8_t* p = d->data_on_device ? static_cast<const uint8_t*>(t.data)
                                             : static_cast<const uint8_t*>(upload(t.data, bytes));
        validate_scales(t.type, p, bytes, s->stream, what);
        return p;
      };
      lb::MoeDevice& m = s->m;
      m.arch = d->arch;
      m.hidden = (int)H;
      m.experts = (int)E;
      m.top_k = top_k;
      m.weights_norm = d->weights_norm ? 1 : 0;
      m.weight_scale = d->weight_scale;
      m.inter = (int)I;
      m.inter_sh = (int)Ish;
      m.k_in = (int)d->up_exps.ne0;
      m.k_down = (int)d->down_exps.ne0;
      m.k_in_sh = shared ? (int)d->up_shexp.ne0 : 0;
      m.k_down_sh = shared ? (int)d->down_shexp.ne0 : 0;
      m.gate_type = qwen ? d->gate_exps.type : d->up_exps.type;
      m.up_type = d->up_exps.type;
      m.down_type = d->down_exps.type;
      m.gate_sh_type = qwen && shared ? d->gate_shexp.type : m.gate_type;
      m.up_sh_type = shared ? d->up_shexp.type : m.up_type;
      m.down_sh_type = shared ? d->down_shexp.type : m.down_type;
      // Router, with the qwen3next shared-expert gate vector appended as row E.
      {
        const size_t rbytes = (size_t)E * H * 4;
        float* r = static_cast<float*>(dev_alloc(rbytes + H * 4));
        s->owned.push_back(r);
        cuda_check(cudaMemcpyAsync(r, d->router.data, rbytes, kind, s->stream), "upload router");
        if (qwen && shared)
          cuda_check(cudaMemcpyAsync(r + E * H, d->shared_gate_inp, H * 4, kind, s->stream),
                     "upload shared gate");
        else
          cuda_check(cudaMemsetAsync(r + E * H, 0, H * 4, s->stream), "memset");
        m.router = r;
        m.router_rows = E + 1;
      }
      if (d->router_bias) {
        if (qwen) throw Failure("A router bias is only defined for nemotron_h_moe.");
        m.router_bias = static_cast<const float*>(upload(d->router_bias, E * 4));
      }
      m.gate_exps = qwen ? experts(d->gate_exps, "ffn_gate_exps") : nullptr;
      m.up_exps = experts(d->up_exps, "ffn_up_exps");
      m.down_exps = experts(d->down_exps, "ffn_down_exps");
      m.gate_rb = qwen ? row_bytes(d->gate_exps.type, d->gate_exps.ne0) : 0;
      m.up_rb = row_bytes(d->up_exps.type, d->up_exps.ne0);
      m.down_rb = row_bytes(d->down_exps.type, d->down_exps.ne0);
      m.shared_here = shared && d->shared_here ? 1 : 0;
      if (m.shared_here) {
        m.gate_sh = qwen ? plain(d->gate_shexp, "ffn_gate_shexp") : nullptr;
        m.up_sh = plain(d->up_shexp, "ffn_up_shexp");
        m.down_sh = plain(d->down_shexp, "ffn_down_shexp");
        m.gate_sh_rb = qwen ? row_bytes(d->gate_shexp.type, d->gate_shexp.ne0) : 0;
        m.up_sh_rb = row_bytes(d->up_shexp.type, d->up_shexp.ne0);
        m.down_sh_rb = row_bytes(d->down_shexp.type, d->down_shexp.ne0);
      } else {
        m.inter_sh = 0;
      }
      m.expert_begin = eb;
      m.expert_end = ee;
      if (latent) {
        m.latent_dim = (int)XW;
        m.lat_down_type = d->latent_down.type;
        m.lat_up_type = d->latent_up.type;
        m.k_lat_down = (int)d->latent_down.ne0;
        m.k_lat_up = (int)d->latent_up.ne0;
        m.lat_down = plain(d->latent_down, "ffn_latent_down");
        m.lat_up = plain(d->latent_up, "ffn_latent_up");
        m.lat_down_rb = row_bytes(d->latent_down.type, d->latent_down.ne0);
        m.lat_up_rb = row_bytes(d->latent_up.type, d->latent_up.ne0);
        if (m.shared_here &&
            ((m.up_sh_type == LLAMBDA_CUDA_TYPE_F32 && m.k_in_sh != (int)H) ||
             (m.down_sh_type == LLAMBDA_CUDA_TYPE_F32 && m.k_down_sh != m.inter_sh)))
          throw Failure("F32 shared expert rows must have exactly the input's width.");
      }
      if (d->input_norm) m.input_norm = static_cast<const float*>(upload(d->input_norm, H * 4));
      m.norm_epsilon = d->norm_epsilon;
      m.add_residual = d->add_residual ? 1 : 0;
      s->max_tokens = d->max_tokens;
      const size_t wb = lb::moe_work_bytes(m, d->max_tokens);
      cuda_check(cudaMalloc(&s->work, wb), "cudaMalloc workspace");
      cuda_check(cudaMemsetAsync(s->work, 0, wb, s->stream), "memset workspace");
      lb::moe_work_carve(m, d->max_tokens, s->work, &s->w);
      cuda_check(lb::moe_maps_build(m, &s->maps), "tensor maps");
      cuda_check(cudaStreamSynchronize(s->stream), "MoE session upload");
    } catch (...) {
      delete s;
      throw;
    }
    *result = s;
    return 0;
  });
}

void llambda_cuda_moe_session_destroy(llambda_cuda_moe_session* session) {
  if (!session) return;
  try {
    DeviceGuard g(session->device);
    if (session->stream) cudaStreamSynchronize(session->stream);
    delete session;
  } catch (...) {
    delete session;
  }
}

size_t llambda_cuda_moe_session_hidden(const llambda_cuda_moe_session* s) {
  return s ? (size_t)s->m.hidden : 0;
}

int llambda_cuda_moe_session_run(llambda_cuda_moe_session* s, const float* x, size_t tokens,
                                 float* out, int32_t* selected, float* weights) {
  if (!s || !x || !out || tokens == 0) {
    set_error("Session, input, output and a positive token count are required.");
    return -1;
  }
  return guarded([&] {
    std::lock_guard<std::mutex> lock(s->mu);
    DeviceGuard g(s->device);
    if ((int64_t)tokens > s->max_tokens)
      throw Failure("Token count " + std::to_string(tokens) + " exceeds the session's max_tokens " +
                    std::to_string(s->max_tokens) + ".");
    const int T = (int)tokens, k = s->m.top_k;
    const size_t xb = tokens * s->m.hidden * 4, sb = tokens * k * 4;
    float* hx = static_cast<float*>(s->hx.get(xb));
    float* hout = static_cast<float*>(s->hout.get(xb));
    float* dx = static_cast<float*>(s->dx.get(xb));
    float* dout = static_cast<float*>(s->dout.get(xb));
    int* hstatus = static_cast<int*>(s->hstatus.get(4));
    // Page-locked caller buffers are copied to and from directly (DMA, no
    // staging memcpy), outside the cached graph, which then holds the
    // layer's kernels only; pageable ones go through the session's staging.
    const bool direct = page_locked(x, xb) && page_locked(out, xb);
    if (!direct) std::memcpy(hx, x, xb);
    auto enqueue = [&]() {
      cuda_check(cudaMemsetAsync(s->w.status, 0, 4, s->stream), "memset");
      if (!direct)
        cuda_check(cudaMemcpyAsync(dx, hx, xb, cudaMemcpyHostToDevice, s->stream), "input copy");
      cuda_check(lb::launch_moe(s->m, s->w, dx, T, dout, &s->maps, s->stream,
                                s->timing ? s->marks : nullptr),
                 "MoE launch");
      if (!direct)
        cuda_check(cudaMemcpyAsync(hout, dout, xb, cudaMemcpyDeviceToHost, s->stream),
                   "output copy");
      cuda_check(cudaMemcpyAsync(hstatus, s->w.status, 4, cudaMemcpyDeviceToHost, s->stream),
                 "copy");
    };
    // graph key: the staging buffers, or a tag for the kernels-only graph
    static const char kDirectTag = 0;
    const void* key0 = direct ? static_cast<const void*>(&kDirectTag) : hx;
    const void* key1 = direct ? static_cast<const void*>(&kDirectTag) : hout;
    if (direct)
      cuda_check(cudaMemcpyAsync(dx, x, xb, cudaMemcpyHostToDevice, s->stream), "input copy");
    const bool same = s->graph && s->graph_tokens == T && s->graph_key[0] == key0 &&
                      s->graph_key[1] == key1 && s->graph_prefill_min == lb::prefill_min_tokens();
    if (s->timing || selected || weights || (!same && s->eager_tokens != T)) {
      enqueue();  // timed or checked calls, and a new token count's first call
      s->eager_tokens = T;
    } else {
      if (!same) {
        s->drop_graph();
        cudaGraph_t g = nullptr;
        cuda_check(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal),
                   "begin capture");
        try {
          enqueue();
        } catch (...) {
          cudaStreamEndCapture(s->stream, &g);
          if (g) cudaGraphDestroy(g);
          throw;
        }
        cuda_check(cudaStreamEndCapture(s->stream, &g), "end capture");
        const cudaError_t ie = cudaGraphInstantiate(&s->graph, g, 0);
        cudaGraphDestroy(g);
        cuda_check(ie, "graph instantiate");
        s->graph_tokens = T;
        s->graph_key[0] = key0;
        s->graph_key[1] = key1;
        s->graph_prefill_min = lb::prefill_min_tokens();
      }
      cuda_check(cudaGraphLaunch(s->graph, s->stream), "graph launch");
    }
    if (direct)
      cuda_check(cudaMemcpyAsync(out, dout, xb, cudaMemcpyDeviceToHost, s->stream),
                 "output copy");
    int32_t* hsel = selected ? static_cast<int32_t*>(s->hsel.get(sb)) : nullptr;
    float* hw = weights ? static_cast<float*>(s->hw.get(sb)) : nullptr;
    if (hsel)
      cuda_check(cudaMemcpyAsync(hsel, s->w.sel, sb, cudaMemcpyDeviceToHost, s->stream), "copy");
    if (hw) cuda_check(cudaMemcpyAsync(hw, s->w.wts, sb, cudaMemcpyDeviceToHost, s->stream), "copy");
    cuda_check(cudaStreamSynchronize(s->stream), "MoE layer");
    if (*hstatus)
      throw Failure("MoE router produced non-positive top-k weight sum.");
    if (!direct) std::memcpy(out, hout, xb);
    if (hsel) std::memcpy(selected, hsel, sb);
    if (hw) std::memcpy(weights, hw, sb);
    return 0;
  });
}

int llambda_cuda_moe_session_run_device(llambda_cuda_moe_session* s, const float* device_x,
                                        size_t tokens, float* device_out,
                                        int32_t* device_selected, float* device_weights,
                                        void* cuda_stream) {
  if (!s || !device_x || !device_out || tokens == 0) {
    set_error("Session, device input/output and a positive token count are required.");
    return -1;
  }
  return guarded([&] {
    DeviceGuard g(s->device);
    if ((int64_t)tokens > s->max_tokens) throw Failure("Token count exceeds max_tokens.");
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    cuda_check(lb::launch_moe(s->m, s->w, device_x, (int)tokens, device_out, &s->maps, st,
                              s->timing ? s->marks : nullptr),
               "MoE launch");
    const size_t sb = tokens * s->m.top_k * 4;
    if (device_selected)
      cuda_check(cudaMemcpyAsync(device_selected, s->w.sel, sb, cudaMemcpyDeviceToDevice, st), "copy");
    if (device_weights)
      cuda_check(cudaMemcpyAsync(device_weights, s->w.wts, sb, cudaMemcpyDeviceToDevice, st), "copy");
    return 0;
  });
}

int llambda_cuda_set_prefill_min_tokens(int tokens) {
  if (tokens < 1) {
    set_error("The prefill threshold must be positive.");
    return -1;
  }
  lb::set_prefill_min_tokens(tokens);
  return 0;
}

int llambda_cuda_prefill_min_tokens(void) { return lb::prefill_min_tokens(); }

int llambda_cuda_moe_session_time_kernels(llambda_cuda_moe_session* s, int enable) {
  if (!s) {
    set_error("A session is required.");
    return -1;
  }
  return guarded([&] {
    std::lock_guard<std::mutex> lock(s->mu);
    DeviceGuard g(s->device);
    if (enable)
      for (cudaEvent_t& e : s->marks)
        if (!e) cuda_check(cudaEventCreate(&e), "create timing event");
    if (enable && s->m.ep_world > 1 && !s->ep_stamps) {
      void* p = nullptr;
      cuda_check(cudaMalloc(&p, 8 * sizeof(unsigned long long)), "cudaMalloc");
      cuda_check(cudaMemset(p, 0, 8 * sizeof(unsigned long long)), "memset");
      s->owned.push_back(p);
      s->ep_stamps = static_cast<unsigned long long*>(p);
    }
    s->m.ep_stamps = enable ? s->ep_stamps : nullptr;
    s->timing = enable != 0;
    return 0;
  });
}

int llambda_cuda_moe_session_kernel_ms(llambda_cuda_moe_session* s, float* gate_up_ms,
                                       float* down_ms) {
  if (!s || !gate_up_ms || !down_ms) {
    set_error("A session and two outputs are required.");
    return -1;
  }
  return guarded([&] {
    std::lock_guard<std::mutex> lock(s->mu);
    DeviceGuard g(s->device);
    if (!s->timing) throw Failure("Kernel timing is not enabled on this session.");
    cuda_check(cudaEventSynchronize(s->marks[2]), "timing events");
    cuda_check(cudaEventElapsedTime(gate_up_ms, s->marks[0], s->marks[1]), "gate/up time");
    cuda_check(cudaEventElapsedTime(down_ms, s->marks[1], s->marks[2]), "down time");
    return 0;
  });
}

int llambda_cuda_moe_session_kernel_breakdown(llambda_cuda_moe_session* s, float* ms, int n) {
  if (!s || !ms || n < 1) {
    set_error("A session and an output array are required.");
    return -1;
  }
  return guarded([&] {
    std::lock_guard<std::mutex> lock(s->mu);
    DeviceGuard g(s->device);
    if (!s->timing) throw Failure("Kernel timing is not enabled on this session.");
    cuda_check(cudaEventSynchronize(s->marks[5]), "timing events");
    // marks: 3 layer start, 6 router end, 0 gate/up start, 1 gate/up end,
    // 2 routed down end, 4 combine start, 5 layer end
    const int order[7] = {3, 6, 0, 1, 2, 4, 5};
    const int parts = std::min(n, 6);
    for (int i = 0; i < parts; ++i)
      cuda_check(cudaEventElapsedTime(&ms[i], s->marks[order[i]], s->marks[order[i + 1]]),
                 "stage time");
    if (n < 9 || !s->m.ep_stamps) return parts;
    // the expert-parallel combine's phases (its CTA 0): pushing its partial
    // to every rank, waiting for every rank's, summing
    unsigned long long st[4];
    cuda_check(cudaMemcpy(st, s->m.ep_stamps, sizeof(st), cudaMemcpyDeviceToHost), "stamps");
    for (int i = 0; i < 3; ++i) ms[6 + i] = (float)((double)(st[i + 1] - st[i]) * 1e-6);
    return 9;
  });
}

int llambda_cuda_moe_session_status(llambda_cuda_moe_session* s) {
  if (!s) {
    set_error("A session is required.");
    return -1;
  }
  return guarded([&] {
    std::lock_guard<std::mutex> lock(s->mu);
    DeviceGuard g(s->device);
    int status = 0;
    cuda_check(cudaMemcpy(&status, s->w.status, 4, cudaMemcpyDeviceToHost), "status copy");
    cuda_check(cudaMemset(s->w.status, 0, 4), "status clear");
    return status;
  });
}

size_t llambda_cuda_moe_peer_bytes(const llambda_cuda_moe_session* s, int world) {
  if (!s || world < 1 || world > lb::kEpMaxWorld) return 0;
  return lb::ep_buffer_bytes(world, s->max_tokens, s->m.hidden);
}

size_t llambda_cuda_moe_dispatch_bytes(const llambda_cuda_moe_session* s, int world,
                                       int max_local_tokens) {
  if (!s || world < 2 || world > lb::kEpMaxWorld || max_local_tokens < 1) return 0;
  return lb::dx_layout(world, max_local_tokens, s->m.top_k, s->m.k_in, s->m.hidden).bytes;
}

int llambda_cuda_moe_session_attach_dispatch(llambda_cuda_moe_session* s, int rank, int world,
                                             void* const* peer_buffers, size_t bytes,
                                             int max_local_tokens) {
  if (!s || !peer_buffers) {
    set_error("A session and the peer buffer pointers are required.");
    return -1;
  }
  return guarded([&] {
    std::lock_guard<std::mutex> lock(s->mu);
    DeviceGuard g(s->device);
    s->drop_graph();
    s->eager_tokens = 0;
    const lb::MoeDevice& m = s->m;
    if (world < 2 || world > lb::kEpMaxWorld || rank < 0 || rank >= world)
      throw Failure("world must be 2.." + std::to_string(lb::kEpMaxWorld) +
                    " and 0 <= rank < world.");
    if (m.latent_dim > 0)
      throw Failure("A layer with latent projections runs on one device (no token dispatch).");
    if (m.expert_begin != (int)((long)rank * m.experts / world) ||
        m.expert_end != (int)((long)(rank + 1) * m.experts / world))
      throw Failure("The token dispatch needs rank r to own experts [r*E/world, (r+1)*E/world).");
    if (m.inter_sh && !m.shared_here)
      throw Failure("Every rank computes the shared expert of its own tokens: shared_here = 1.");
    if (max_local_tokens < 1 || (long)world * max_local_tokens > s->max_tokens ||
        s->max_tokens < 64)
      throw Failure("world * max_local_tokens must be at most the session's max_tokens "
                    "(and max_tokens at least 64).");
    const lb::DxLayout L = lb::dx_layout(world, max_local_tokens, m.top_k, m.k_in, m.hidden);
    if (bytes < L.bytes) throw Failure("The peer buffer is smaller than llambda_cuda_moe_dispatch_bytes.");
    for (int r = 0; r < world; ++r)
      if (reinterpret_cast<uintptr_t>(peer_buffers[r]) & 255)
        throw Failure("Token dispatch buffers must be 256-byte aligned.");
    std::vector<void*> table(2 * world);
    for (int r = 0; r < world; ++r) {
      table[r] = peer_buffers[r];
      table[world + r] = static_cast<char*>(peer_buffers[r]) + L.partial;
    }
    void* dev = nullptr;
    cuda_check(cudaMalloc(&dev, sizeof(void*) * 2 * world), "cudaMalloc dispatch table");
    s->owned.push_back(dev);
    cuda_check(cudaMemcpy(dev, table.data(), sizeof(void*) * 2 * world, cudaMemcpyHostToDevice),
               "dispatch table copy");
    s->m.dx_peers = static_cast<void* const*>(dev);
    s->m.dx_partials = reinterpret_cast<float* const*>(static_cast<void**>(dev) + world);
    s->m.dx_partial_local = static_cast<float*>(table[world + rank]);
    s->m.dx_rank = rank;
    s->m.dx_world = world;
    s->m.dx_cap = max_local_tokens;
    return 0;
  });
}

int llambda_cuda_moe_session_attach_peers(llambda_cuda_moe_session* s, int rank, int world,
                                          void* const* peer_buffers, size_t bytes) {
  if (!s || !peer_buffers) {
    set_error("A session and the peer buffer pointers are required.");
    return -1;
  }
  return guarded([&] {
    std::lock_guard<std::mutex> lock(s->mu);
    DeviceGuard g(s->device);
    s->drop_graph();  // the layer's launches change with the reduction
    s->eager_tokens = 0;
    if (world < 2 || world > lb::kEpMaxWorld || rank < 0 || rank >= world)
      throw Failure("world must be 2.." + std::to_string(lb::kEpMaxWorld) +
                    " and 0 <= rank < world.");
    if (s->m.hidden % 4) throw Failure("The peer-memory reduction needs hidden % 4 == 0.");
    if (s->m.latent_dim > 0)
      throw Failure("A layer with latent projections runs on one device (no peer reduction).");
    if (bytes < lb::ep_buffer_bytes(world, s->max_tokens, s->m.hidden))
      throw Failure("The peer buffer is smaller than llambda_cuda_moe_peer_bytes.");
    for (int r = 0; r < world; ++r) require_aligned16(peer_buffers[r], "peer buffer");
    void* dev = nullptr;
    cuda_check(cudaMalloc(&dev, sizeof(void*) * world), "cudaMalloc peer table");
    s->owned.push_back(dev);
    cuda_check(cudaMemcpy(dev, peer_buffers, sizeof(void*) * world, cudaMemcpyHostToDevice),
               "peer table copy");
    s->m.ep_peers = static_cast<void* const*>(dev);
    s->m.ep_rank = rank;
    s->m.ep_world = world;
    s->m.ep_max_tokens = s->max_tokens;
    // every rank holding the shared expert computes it for its part of the tokens
    s->m.sh_part = rank;
    s->m.sh_parts = world;
    return 0;
  });
}

}  // extern "C"

// ------------------------------------------------- MoE layer, no allocation
//
// For callers that cannot allocate device memory (their allocator owns the
// device, or their decode loop must not pay for cudaMalloc and its implicit
// synchronisation): the layer's working memory is this one static array, and
// every tensor is the caller's device memory.  The array exists on every GPU
// that loads the library, for the life of the process.

namespace {

static __device__ __align__(256) unsigned char g_moe_static_scratch[LLAMBDA_CUDA_STATIC_SCRATCH_BYTES];

constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxScratchDevices] = {};

// Device address of the static array on the current device, looked up once
// per device with that device current.  The name g_moe_static_scratch in
// host code is only a host-side handle; kernels must get this address.
void* static_scratch_address(int dev) {
  if (dev < 0 || dev >= kMaxScratchDevices) throw Failure("device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    // the first call on a device: refuse anything but sm_100 with the
    // library's own message, before any launch
    require_b200(dev);
    void* p = nullptr;
    cuda_check(cudaGetSymbolAddress(&p, g_moe_static_scratch), "cudaGetSymbolAddress");
    if (!p) throw Failure("cudaGetSymbolAddress returned a null scratch address");
    g_scratch_addr[dev] = p;
  }
  return g_scratch_addr[dev];
}

// The layer description of a device-resident desc, without uploads.
lb::MoeDevice static_layer(const llambda_cuda_moe_desc* d) {
  if (!d->data_on_device) throw Failure("The static-scratch MoE call needs data_on_device = 1.");
  if (d->latent_down.data || d->latent_up.data)
    throw Failure("Latent projections need a MoE session (llambda_cuda_moe_session_create).");
  if (d->arch != LLAMBDA_CUDA_ARCH_QWEN3NEXT && d->arch != LLAMBDA_CUDA_ARCH_NEMOTRON_H_MOE)
    throw Failure("Unknown MoE architecture " + std::to_string(d->arch));
  const bool qwen = d->arch == LLAMBDA_CUDA_ARCH_QWEN3NEXT;
  const uint64_t H = d->hidden;
  if (!H || H > (1u << 20)) throw Failure("MoE hidden size must be positive.");
  if (!d->router.data || d->router.type != LLAMBDA_CUDA_TYPE_F32 || d->router.ne0 != H)
    throw Failure("MoE router ffn_gate_inp must be an F32 tensor of row width hidden.");
  const uint64_t E = d->router.ne1;
  if (E == 0 || E > 1024) throw Failure("MoE expert count must be in 1..1024.");
  check_tensor(d->up_exps, "ffn_up_exps", true);
  check_tensor(d->down_exps, "ffn_down_exps", true);
  check_tensor(d->gate_exps, "ffn_gate_exps", qwen);
  const bool shared = d->up_shexp.data != nullptr;
  if (shared) {
    check_tensor(d->up_shexp, "ffn_up_shexp", true);
    check_tensor(d->down_shexp, "ffn_down_shexp", true);
    check_tensor(d->gate_shexp, "ffn_gate_shexp", qwen);
    if (qwen && !d->shared_gate_inp) throw Failure("ffn_gate_inp_shexp is required.");
  }
  const uint64_t I = d->up_exps.ne1, Ish = shared ? d->up_shexp.ne1 : 0;
  auto dims = [&](const llambda_cuda_tensor& t, uint64_t min_ne0, uint64_t ne1, uint64_t ne2,
                  const char* what) {
    if (t.ne0 < min_ne0 || t.ne1 != ne1 || (ne2 && (t.ne2 ? t.ne2 : 1) != ne2))
      throw Failure(std::string("MoE tensor ") + what + " has unexpected dimensions.");
  };
  dims(d->up_exps, H, I, E, "ffn_up_exps");
  dims(d->down_exps, I, H, E, "ffn_down_exps");
  if (qwen) {
    dims(d->gate_exps, H, I, E, "ffn_gate_exps");
    if (d->gate_exps.ne0 != d->up_exps.ne0 || d->gate_exps.type != d->up_exps.type)
      throw Failure("ffn_gate_exps and ffn_up_exps must share type and width.");
  }
  if (shared) {
    dims(d->up_shexp, H, Ish, 0, "ffn_up_shexp");
    dims(d->down_shexp, Ish, H, 0, "ffn_down_shexp");
    if (qwen) {
      dims(d->gate_shexp, H, Ish, 0, "ffn_gate_shexp");
      if (d->gate_shexp.type != d->up_shexp.type || d->gate_shexp.ne0 != d->up_shexp.ne0)
        throw Failure("ffn_gate_shexp and ffn_up_shexp must share type and width.");
    }
    if (d->up_shexp.type != d->up_exps.type || d->down_shexp.type != d->down_exps.type)
      throw Failure("Shared and routed expert tensors must share their types.");
  }
  if (d->router_bias && qwen) throw Failure("A router bias is only defined for nemotron_h_moe.");
  const int top_k = (int)std::min<uint64_t>((uint64_t)std::max(d->top_k, 1), E);
  if (d->top_k < 1 || top_k > 32) throw Failure("top_k must be in 1..32.");
  int eb = d->expert_begin, ee = d->expert_end;
  if (eb == 0 && ee == 0) ee = (int)E;
  if (eb < 0 || ee > (int)E || eb >= ee) throw Failure("Invalid owned expert range.");
  lb::MoeDevice m{};
  m.arch = d->arch;
  m.hidden = (int)H;
  m.experts = (int)E;
  m.top_k = top_k;
  m.weights_norm = d->weights_norm ? 1 : 0;
  m.weight_scale = d->weight_scale;
  m.inter = (int)I;
  m.k_in = (int)d->up_exps.ne0;
  m.k_down = (int)d->down_exps.ne0;
  m.gate_type = qwen ? d->gate_exps.type : d->up_exps.type;
  m.up_type = d->up_exps.type;
  m.down_type = d->down_exps.type;
  for (const llambda_cuda_tensor* t : {&d->gate_exps, &d->up_exps, &d->down_exps, &d->gate_shexp,
                                       &d->up_shexp, &d->down_shexp})
    if (t->data) require_aligned16(t->data, "MoE tensor");
  m.router = static_cast<const float*>(d->router.data);
  m.router_rows = (int)E;
  m.router_extra_row = qwen && shared ? d->shared_gate_inp : nullptr;
  m.router_bias = d->router_bias;
  m.gate_exps = qwen ? static_cast<const uint8_t*>(d->gate_exps.data) : nullptr;
  m.up_exps = static_cast<const uint8_t*>(d->up_exps.data);
  m.down_exps = static_cast<const uint8_t*>(d->down_exps.data);
  m.gate_rb = qwen ? row_bytes(d->gate_exps.type, d->gate_exps.ne0) : 0;
  m.up_rb = row_bytes(d->up_exps.type, d->up_exps.ne0);
  m.down_rb = row_bytes(d->down_exps.type, d->down_exps.ne0);
  m.shared_here = shared && d->shared_here ? 1 : 0;
  if (m.shared_here) {
    m.inter_sh = (int)Ish;
    m.k_in_sh = (int)d->up_shexp.ne0;
    m.k_down_sh = (int)d->down_shexp.ne0;
    m.gate_sh_type = qwen ? d->gate_shexp.type : m.gate_type;
    m.up_sh_type = d->up_shexp.type;
    m.down_sh_type = d->down_shexp.type;
    m.gate_sh = qwen ? static_cast<const uint8_t*>(d->gate_shexp.data) : nullptr;
    m.up_sh = static_cast<const uint8_t*>(d->up_shexp.data);
    m.down_sh = static_cast<const uint8_t*>(d->down_shexp.data);
    m.gate_sh_rb = qwen ? row_bytes(d->gate_shexp.type, d->gate_shexp.ne0) : 0;
    m.up_sh_rb = row_bytes(d->up_shexp.type, d->up_shexp.ne0);
    m.down_sh_rb = row_bytes(d->down_shexp.type, d->down_shexp.ne0);
  } else {
    m.gate_sh_type = m.gate_type;
    m.up_sh_type = m.up_type;
    m.down_sh_type = m.down_type;
  }
  m.expert_begin = eb;
  m.expert_end = ee;
  m.input_norm = d->input_norm;
  m.norm_epsilon = d->norm_epsilon;
  m.add_residual = d->add_residual ? 1 : 0;
  return m;
}

}  // namespace

extern "C" {

int llambda_cuda_moe_forward_static_scratch(const llambda_cuda_moe_desc* desc,
                                            const float* device_x, size_t tokens,
                                            float* device_out, void* cuda_stream) {
  if (!desc || !device_x || !device_out || tokens == 0) {
    set_error("A descriptor, device input/output and a positive token count are required.");
    return -1;
  }
  return guarded([&] {
    const lb::MoeDevice m = static_layer(desc);
    // bound checked in unsigned arithmetic before any narrowing (top_k >= 1)
    if (tokens > 65536u / (size_t)m.top_k)
      throw Failure("tokens * top_k must be at most 65536.");
    const int T = (int)tokens;
    const size_t need = lb::moe_work_bytes(m, T);
    if (need > LLAMBDA_CUDA_STATIC_SCRATCH_BYTES)
      throw Failure("This layer call needs " + std::to_string(need) +
                    " bytes of working memory; the static scratch holds " +
                    std::to_string((size_t)LLAMBDA_CUDA_STATIC_SCRATCH_BYTES) +
                    " bytes (use fewer tokens per call or a MoE session).");
    void* base = static_scratch_address(current_device());
    lb::MoeWork w{};
    lb::moe_work_carve(m, T, base, &w);
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    int status = 0;
    // A launch that fails part-way leaves earlier kernels of this call
    // writing the shared array: wait for them before reporting, so that the
    // caller's next call (on any stream) does not race with them.
    auto drained = [&](cudaError_t e, const char* what) {
      if (e != cudaSuccess) cudaStreamSynchronize(st);
      cuda_check(e, what);
    };
    drained(cudaMemsetAsync(w.status, 0, 2 * sizeof(int), st), "clear status and ticket");
    drained(lb::launch_moe(m, w, device_x, T, device_out, nullptr, st), "MoE launch");
    drained(cudaMemcpyAsync(&status, w.status, sizeof(int), cudaMemcpyDeviceToHost, st),
            "status copy");
    cuda_check(cudaStreamSynchronize(st), "MoE layer");
    if (status) throw Failure("MoE router produced non-positive top-k weight sum.");
    return 0;
  });
}

int llambda_cuda_synth_fill_device(int type, uint64_t seed, uint64_t stream_id, uint64_t first,
                                   size_t count, float scale, void* device_out, void* cuda_stream) {
  if (!device_out) {
    set_error("An output buffer is required.");
    return -1;
  }
  return guarded([&] {
    cuda_check(lb::synth_fill(type, seed, stream_id, first, count, scale, device_out,
                              static_cast<cudaStream_t>(cuda_stream)),
               "synthetic fill");
    return 0;
  });
}

}  // extern "C"

// The GGUF loader (gguf.cu) reports through the same thread-local last error.
void llambda_cuda_set_last_error(const std::string& message) { set_error(message); }
