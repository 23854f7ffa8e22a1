// GGUF files: mapped and parsed on the host, chosen tensors uploaded raw into
// one device arena (the weights stay GGUF blocks in device memory; sessions
// and MoE descriptors then point into the arena with data_on_device = 1).
//
// The parse follows the reference loader (llambda.lisp): header
// (read-gguf-header, L2049-2062: "GGUF" magic, version, tensor count,
// metadata count), metadata section (read-gguf-metadata-section,
// L2064-2084, values read by type as read-gguf-value, L1984-2047, nested
// arrays rejected), tensor infos (read-gguf-tensor-infos, L2157-2238: 1..4
// positive dimensions, type tag, offset), the data start aligned to
// general.alignment (default 32, a power of two; L2089-2101), byte sizes by
// type (ggml-tensor-byte-size, L2126-2155; unsupported types get no size),
// and every tensor's byte range checked against the file.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <stdint.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/llambda_cuda.h"

namespace {

struct GgufTensor {
  std::string name;
  uint32_t n_dims = 0;
  uint64_t ne[4] = {1, 1, 1, 1};
  int type = 0;
  uint64_t offset = 0;     // from the data start
  uint64_t byte_size = 0;  // 0: type without a size here
};

// Block size and block bytes of the types the reference sizes (L2104-2144).
bool type_layout(int t, uint64_t* block, uint64_t* bytes) {
  switch (t) {
    case 0: *block = 1; *bytes = 4; return true;      // F32
    case 1: *block = 1; *bytes = 2; return true;      // F16
    case 30: *block = 1; *bytes = 2; return true;     // BF16
    case 6: *block = 32; *bytes = 22; return true;    // Q5_0
    case 8: *block = 32; *bytes = 34; return true;    // Q8_0
    case 12: *block = 256; *bytes = 144; return true; // Q4_K
    case 13: *block = 256; *bytes = 176; return true; // Q5_K
    case 14: *block = 256; *bytes = 210; return true; // Q6_K
    default: return false;
  }
}

struct Reader {
  const uint8_t* p;
  uint64_t size;
  uint64_t at = 0;
  void need(uint64_t n, const char* what) {
    if (n > size || at > size - n)
      throw std::runtime_error(std::string("GGUF file ends inside ") + what + ".");
  }
  uint64_t u(int bytes, const char* what) {
    need((uint64_t)bytes, what);
    uint64_t v = 0;
    for (int i = 0; i < bytes; ++i) v |= (uint64_t)p[at + i] << (8 * i);
    at += bytes;
    return v;
  }
  std::string str(const char* what) {
    const uint64_t n = u(8, what);
    need(n, what);
    std::string s(reinterpret_cast<const char*>(p + at), n);
    at += n;
    return s;
  }
  // One metadata value of type t; the alignment key's integer value is kept.
  uint64_t value(uint32_t t, bool top) {
    switch (t) {
      case 0: case 1: case 7: return u(1, "a GGUF metadata value");
      case 2: case 3: return u(2, "a GGUF metadata value");
      case 4: case 5: case 6: return u(4, "a GGUF metadata value");
      case 10: case 11: case 12: return u(8, "a GGUF metadata value");
      case 8: str("a GGUF metadata string"); return 0;
      case 9: {
        if (!top) throw std::runtime_error("Nested GGUF metadata arrays are unsupported.");
        const uint32_t et = (uint32_t)u(4, "a GGUF metadata array element type");
        const uint64_t n = u(8, "a GGUF metadata array length");
        if (et == 9) throw std::runtime_error("Nested GGUF metadata arrays are unsupported.");
        for (uint64_t i = 0; i < n; ++i) value(et, false);
        return 0;
      }
      default:
        throw std::runtime_error("Unsupported GGUF metadata value type: " + std::to_string(t) +
                                 ".");
    }
  }
};

}  // namespace

struct llambda_cuda_gguf {
  int fd = -1;
  void* map = nullptr;
  uint64_t size = 0;
  uint32_t version = 0;
  uint64_t alignment = 32;
  uint64_t data_start = 0;
  std::vector<GgufTensor> tensors;
  std::unordered_map<std::string, uint64_t> by_name;
  ~llambda_cuda_gguf() {
    if (map && map != MAP_FAILED) munmap(map, size);
    if (fd >= 0) close(fd);
  }
};

// Defined in capi.cu: thread-local last error and the guarded-call wrapper.
void llambda_cuda_set_last_error(const std::string& message);

namespace {

template <typename F>
int guard(F&& f) {
  try {
    return f();
  } catch (const std::exception& e) {
    llambda_cuda_set_last_error(e.what());
    return -1;
  }
}

void parse(llambda_cuda_gguf* g) {
  Reader r{static_cast<const uint8_t*>(g->map), g->size};
  r.need(4, "the GGUF magic");
  if (memcmp(r.p, "GGUF", 4) != 0) throw std::runtime_error("Invalid GGUF magic.");
  r.at = 4;
  g->version = (uint32_t)r.u(4, "the GGUF version");
  const uint64_t tensor_count = r.u(8, "the GGUF tensor count");
  const uint64_t kv_count = r.u(8, "the GGUF metadata count");
  // every entry takes at least 13 (metadata) or 24 (tensor info) bytes
  if (kv_count > g->size / 13 || tensor_count > g->size / 24)
    throw std::runtime_error("GGUF counts exceed the file size.");
  bool have_alignment = false;
  for (uint64_t i = 0; i < kv_count; ++i) {
    const std::string key = r.str("a GGUF metadata key");
    const uint32_t t = (uint32_t)r.u(4, "a GGUF metadata value type");
    const uint64_t v = r.value(t, true);
    if (key == "general.alignment") {
      if (t > 5 && t != 10 && t != 11) throw std::runtime_error("general.alignment is not an integer.");
      g->alignment = v;
      have_alignment = true;
    }
  }
  if (have_alignment && (g->alignment == 0 || (g->alignment & (g->alignment - 1))))
    throw std::runtime_error("GGUF alignment must be a positive power of two, got " +
                             std::to_string(g->alignment) + ".");
  g->tensors.resize(tensor_count);
  for (uint64_t i = 0; i < tensor_count; ++i) {
    GgufTensor& t = g->tensors[i];
    t.name = r.str("a GGUF tensor name");
    t.n_dims = (uint32_t)r.u(4, "a GGUF tensor dimension count");
    if (t.n_dims < 1 || t.n_dims > 4)
      throw std::runtime_error("Tensor \"" + t.name + "\" has invalid dimension count " +
                               std::to_string(t.n_dims) + "; GGUF permits 1 through 4.");
    uint64_t elements = 1;
    for (uint32_t d = 0; d < t.n_dims; ++d) {
      t.ne[d] = r.u(8, "a GGUF tensor dimension");
      if (t.ne[d] == 0)
        throw std::runtime_error("Tensor \"" + t.name + "\" has non-positive dimensions.");
      if (elements > UINT64_MAX / t.ne[d])
        throw std::runtime_error("Tensor \"" + t.name + "\" is too large.");
      elements *= t.ne[d];
    }
    t.type = (int)r.u(4, "a GGUF tensor type");
    t.offset = r.u(8, "a GGUF tensor offset");
    uint64_t block, bytes;
    if (type_layout(t.type, &block, &bytes)) {
      if (elements % block)
        throw std::runtime_error("Tensor \"" + t.name + "\" element count " +
                                 std::to_string(elements) + " is not a multiple of block size " +
                                 std::to_string(block) + ".");
      t.byte_size = elements / block * bytes;
    }
    g->by_name[t.name] = i;
  }
  g->data_start = (r.at + g->alignment - 1) / g->alignment * g->alignment;
  for (const GgufTensor& t : g->tensors) {
    if (g->data_start > g->size || t.offset > g->size - g->data_start ||
        t.byte_size > g->size - g->data_start - t.offset)
      throw std::runtime_error("GGUF tensor \"" + t.name + "\" lies past the end of the file.");
  }
}

}  // namespace

extern "C" {

int llambda_cuda_gguf_open(const char* path, llambda_cuda_gguf** out) {
  if (out) *out = nullptr;
  if (!path || !out) {
    llambda_cuda_set_last_error("A path and an output handle are required.");
    return -1;
  }
  return guard([&] {
    auto* g = new llambda_cuda_gguf();
    try {
      g->fd = open(path, O_RDONLY);
      if (g->fd < 0) throw std::runtime_error(std::string("Cannot open GGUF file ") + path + ".");
      struct stat st;
      if (fstat(g->fd, &st) != 0) throw std::runtime_error("Cannot stat the GGUF file.");
      g->size = (uint64_t)st.st_size;
      if (g->size < 24) throw std::runtime_error("GGUF file ends inside the header.");
      g->map = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
      if (g->map == MAP_FAILED) throw std::runtime_error("Cannot map the GGUF file.");
      parse(g);
    } catch (...) {
      delete g;
      throw;
    }
    *out = g;
    return 0;
  });
}

void llambda_cuda_gguf_close(llambda_cuda_gguf* g) { delete g; }

uint64_t llambda_cuda_gguf_tensor_count(const llambda_cuda_gguf* g) {
  return g ? g->tensors.size() : 0;
}

int64_t llambda_cuda_gguf_find(const llambda_cuda_gguf* g, const char* name) {
  if (!g || !name) return -1;
  const auto it = g->by_name.find(name);
  return it == g->by_name.end() ? -1 : (int64_t)it->second;
}

int llambda_cuda_gguf_tensor_info(const llambda_cuda_gguf* g, uint64_t index, char* name_out,
                                  size_t name_capacity, int* type, uint32_t* n_dims,
                                  uint64_t* ne, uint64_t* byte_size, const void** host_data) {
  if (!g || index >= g->tensors.size()) {
    llambda_cuda_set_last_error("A GGUF handle and a tensor index in range are required.");
    return -1;
  }
  const GgufTensor& t = g->tensors[index];
  if (name_out && name_capacity) {
    const size_t n = std::min(name_capacity - 1, t.name.size());
    memcpy(name_out, t.name.data(), n);
    name_out[n] = 0;
  }
  if (type) *type = t.type;
  if (n_dims) *n_dims = t.n_dims;
  if (ne)
    for (int d = 0; d < 4; ++d) ne[d] = t.ne[d];
  if (byte_size) *byte_size = t.byte_size;
  if (host_data)
    *host_data = static_cast<const uint8_t*>(g->map) + g->data_start + t.offset;
  return 0;
}

int llambda_cuda_gguf_upload(const llambda_cuda_gguf* g, const uint64_t* indices, size_t count,
                             void** device_arena, void** device_ptrs) {
  if (device_arena) *device_arena = nullptr;
  if (!g || !indices || !count || !device_arena || !device_ptrs) {
    llambda_cuda_set_last_error("A GGUF handle, tensor indices and outputs are required.");
    return -1;
  }
  return guard([&] {
    std::vector<uint64_t> at(count);
    uint64_t total = 0;
    for (size_t i = 0; i < count; ++i) {
      if (indices[i] >= g->tensors.size()) throw std::runtime_error("Tensor index out of range.");
      const GgufTensor& t = g->tensors[indices[i]];
      if (!t.byte_size)
        throw std::runtime_error("Tensor \"" + t.name + "\" has a type this loader does not size.");
      at[i] = total;
      total += (t.byte_size + 255) / 256 * 256;  // every tensor 256-byte aligned
    }
    void* arena = nullptr;
    // 256 bytes of slack past the last tensor, as the sessions' own uploads
    cudaError_t e = cudaMalloc(&arena, total + 256);
    if (e != cudaSuccess)
      throw std::runtime_error(std::string("cudaMalloc: ") + cudaGetErrorString(e));
    for (size_t i = 0; i < count && e == cudaSuccess; ++i) {
      const GgufTensor& t = g->tensors[indices[i]];
      e = cudaMemcpy(static_cast<uint8_t*>(arena) + at[i],
                     static_cast<const uint8_t*>(g->map) + g->data_start + t.offset, t.byte_size,
                     cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
      cudaFree(arena);
      throw std::runtime_error(std::string("GGUF upload: ") + cudaGetErrorString(e));
    }
    for (size_t i = 0; i < count; ++i) device_ptrs[i] = static_cast<uint8_t*>(arena) + at[i];
    *device_arena = arena;
    return 0;
  });
}

int llambda_cuda_device_free(void* device_ptr) {
  const cudaError_t e = cudaFree(device_ptr);
  if (e != cudaSuccess) {
    llambda_cuda_set_last_error(std::string("cudaFree: ") + cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

}  // extern "C"
