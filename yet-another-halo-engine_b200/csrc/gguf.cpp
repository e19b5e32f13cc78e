// GGUF reader and device weight chunks behind the C ABI (include/yah_qgemm.h, "GGUF files").
//
// Reference counterparts: core::Gguf (engine/core/gguf.hpp:74-105, engine/core/gguf.cpp: header, metadata and
// tensor table, data region aligned to general.alignment), the GGML block table (gguf.hpp:49-50, gguf.cpp:27-35,
// BlockElements / BlockBytes), model::TensorRef (engine/model/weights.hpp:15-25: ne0 = row length, ne1 = rows) and
// LoomWeights (engine/model/loom_runtime.hpp:487-516: the tensor-data region copied to device buffers of about
// 1 GiB cut at tensor boundaries, a tensor bound as (buffer, offset), no repacking).
//
// The file is mapped read-only; the tensor table is parsed once with every read bounds-checked against the file
// size, so a truncated or corrupt file is refused with YAH_ERR_IO instead of read out of range. Host code only.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/yah_qgemm.h"
#include "kernels.h"

namespace {

using yah::set_error;

// GGML block geometry: (elements per block, bytes per block) by type id; {0, 0} for ids this reader does not know.
struct BlockGeom {
  uint32_t elements, bytes;
};

BlockGeom geom_of(uint32_t type) {
  switch (type) {
    case 0: return {1, 4};        // F32
    case 1: return {1, 2};        // F16
    case 2: return {32, 18};      // Q4_0
    case 3: return {32, 20};      // Q4_1
    case 6: return {32, 22};      // Q5_0
    case 7: return {32, 24};      // Q5_1
    case 8: return {32, 34};      // Q8_0
    case 9: return {32, 36};      // Q8_1
    case 10: return {256, 84};    // Q2_K
    case 11: return {256, 110};   // Q3_K
    case 12: return {256, 144};   // Q4_K
    case 13: return {256, 176};   // Q5_K
    case 14: return {256, 210};   // Q6_K
    case 15: return {256, 292};   // Q8_K
    case 16: return {256, 66};    // IQ2_XXS
    case 17: return {256, 74};    // IQ2_XS
    case 18: return {256, 98};    // IQ3_XXS
    case 19: return {256, 50};    // IQ1_S
    case 20: return {32, 18};     // IQ4_NL
    case 21: return {256, 110};   // IQ3_S
    case 22: return {256, 82};    // IQ2_S
    case 23: return {256, 136};   // IQ4_XS
    case 24: return {1, 1};       // I8
    case 25: return {1, 2};       // I16
    case 26: return {1, 4};       // I32
    case 27: return {1, 8};       // I64
    case 28: return {1, 8};       // F64
    case 29: return {256, 56};    // IQ1_M
    case 30: return {1, 2};       // BF16
    default: return {0, 0};
  }
}

// Metadata value kinds of the GGUF format.
enum : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kString = 8, kArray = 9, kU64 = 10,
  kI64 = 11, kF64 = 12
};

struct Meta {
  uint32_t kind = 0;
  uint64_t u = 0;  // unsigned and bool values; signed ones as two's complement
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  uint32_t elem_kind = 0;  // arrays: element kind and count (the elements are not kept)
  uint64_t count = 0;
};

// Bounds-checked little-endian reads over the mapping.
struct Cursor {
  const uint8_t* p;
  uint64_t size, pos = 0;
  bool ok = true;

  bool take(void* dst, uint64_t n) {
    if (!ok || n > size - pos) return ok = false;
    std::memcpy(dst, p + pos, n);
    pos += n;
    return true;
  }
  bool skip(uint64_t n) {
    if (!ok || n > size - pos) return ok = false;
    pos += n;
    return true;
  }
  template <class T>
  T get() {
    T v{};
    take(&v, sizeof v);
    return v;
  }
  bool str(std::string* out, uint64_t max_len) {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > max_len || n > size - pos) return ok = false;
    if (out) out->assign(reinterpret_cast<const char*>(p + pos), n);
    pos += n;
    return true;
  }
};

uint64_t scalar_bytes(uint32_t kind) {
  switch (kind) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
  }
}

bool read_scalar(Cursor& c, uint32_t kind, Meta* m) {
  switch (kind) {
    case kU8: m->u = c.get<uint8_t>(); m->i = (int64_t)m->u; break;
    case kI8: m->i = c.get<int8_t>(); m->u = (uint64_t)m->i; break;
    case kU16: m->u = c.get<uint16_t>(); m->i = (int64_t)m->u; break;
    case kI16: m->i = c.get<int16_t>(); m->u = (uint64_t)m->i; break;
    case kU32: m->u = c.get<uint32_t>(); m->i = (int64_t)m->u; break;
    case kI32: m->i = c.get<int32_t>(); m->u = (uint64_t)m->i; break;
    case kU64: m->u = c.get<uint64_t>(); m->i = (int64_t)m->u; break;
    case kI64: m->i = c.get<int64_t>(); m->u = (uint64_t)m->i; break;
    case kBool: m->u = c.get<uint8_t>() ? 1 : 0; m->i = (int64_t)m->u; break;
    case kF32: m->f = c.get<float>(); break;
    case kF64: m->f = c.get<double>(); break;
    default: return c.ok = false;
  }
  if (kind != kF32 && kind != kF64) m->f = kind == kI8 || kind == kI16 || kind == kI32 || kind == kI64
                                               ? (double)m->i : (double)m->u;
  return c.ok;
}

constexpr uint64_t kMaxString = 1 << 20;   // longest key or string value accepted
constexpr uint64_t kMaxName = 127;          // tensor names (yah_gguf_tensor.name holds 127 bytes and a NUL)
constexpr uint32_t kMaxDims = 4;

}  // namespace

struct yah_gguf {
  int fd = -1;
  const uint8_t* base = nullptr;
  uint64_t size = 0;
  uint32_t version = 0;
  uint64_t alignment = 32;
  uint64_t data_offset = 0;
  std::vector<yah_gguf_tensor> tensors;
  std::unordered_map<std::string, int64_t> by_name;
  std::unordered_map<std::string, Meta> meta;

  ~yah_gguf() {
    if (base) munmap(const_cast<uint8_t*>(base), size);
    if (fd >= 0) close(fd);
  }
};

namespace {

int parse(yah_gguf* g, const std::string& path) {
  Cursor c{g->base, g->size};
  const uint32_t magic = c.get<uint32_t>();
  if (!c.ok || magic != 0x46554747u) return set_error(YAH_ERR_IO, "gguf: " + path + " is not a GGUF file");
  g->version = c.get<uint32_t>();
  if (!c.ok || (g->version != 2 && g->version != 3))
    return set_error(YAH_ERR_IO, "gguf: " + path + ": version " + std::to_string(g->version) + " (2 and 3 are read)");
  const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
  if (!c.ok || n_tensors > g->size / 24 || n_kv > g->size / 13)
    return set_error(YAH_ERR_IO, "gguf: " + path + ": header counts exceed the file");
  for (uint64_t k = 0; k < n_kv; ++k) {
    std::string key;
    if (!c.str(&key, kMaxString)) break;
    Meta m;
    m.kind = c.get<uint32_t>();
    if (m.kind == kString) {
      c.str(&m.s, kMaxString);
    } else if (m.kind == kArray) {
      m.elem_kind = c.get<uint32_t>();
      m.count = c.get<uint64_t>();
      if (!c.ok) break;
      if (m.elem_kind == kString) {
        for (uint64_t e = 0; e < m.count && c.ok; ++e) c.str(nullptr, kMaxString);
      } else {
        const uint64_t eb = scalar_bytes(m.elem_kind);
        if (!eb || m.count > (c.size - c.pos) / eb) c.ok = false;
        else c.skip(m.count * eb);
      }
    } else {
      read_scalar(c, m.kind, &m);
    }
    if (!c.ok) break;
    g->meta[key] = std::move(m);
  }
  if (!c.ok) return set_error(YAH_ERR_IO, "gguf: " + path + ": metadata truncated or malformed");
  auto al = g->meta.find("general.alignment");
  if (al != g->meta.end()) {
    const Meta& m = al->second;
    if (m.kind == kString || m.kind == kArray || m.kind == kF32 || m.kind == kF64 || m.u == 0 || (m.u & (m.u - 1)))
      return set_error(YAH_ERR_IO, "gguf: " + path + ": general.alignment is not a power of two");
    g->alignment = m.u;
  }
  g->tensors.reserve(n_tensors);
  for (uint64_t t = 0; t < n_tensors; ++t) {
    yah_gguf_tensor ti{};
    std::string name;
    if (!c.str(&name, kMaxName)) break;  // truncated, or a name longer than kMaxName
    std::memcpy(ti.name, name.data(), name.size());
    const uint32_t nd = c.get<uint32_t>();
    if (!c.ok) break;
    if (nd < 1 || nd > kMaxDims)
      return set_error(YAH_ERR_IO, "gguf: " + path + ": tensor " + name + " has " + std::to_string(nd) + " dims");
    ti.n_dims = (int)nd;
    uint64_t elements = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      const uint64_t v = c.get<uint64_t>();
      if (!c.ok) break;
      if (v == 0 || v > (1ull << 40) || elements > (1ull << 50) / v)
        return set_error(YAH_ERR_IO, "gguf: " + path + ": tensor " + name + " has a bad shape");
      ti.dims[d] = (int64_t)v;
      elements *= v;
    }
    if (!c.ok) break;
    for (uint32_t d = nd; d < kMaxDims; ++d) ti.dims[d] = 1;
    const uint32_t type = c.get<uint32_t>();
    ti.offset = c.get<uint64_t>();
    if (!c.ok) break;
    const BlockGeom bg = geom_of(type);
    if (!bg.elements)
      return set_error(YAH_ERR_UNSUPPORTED, "gguf: " + path + ": tensor " + name + " has GGML type " +
                                                std::to_string(type) + ", whose block size this reader does not know");
    if (ti.dims[0] % bg.elements)
      return set_error(YAH_ERR_IO, "gguf: " + path + ": tensor " + name + " rows are not whole blocks");
    ti.ggml_type = (int)type;
    ti.bytes = elements / bg.elements * bg.bytes;
    if (g->by_name.count(name)) return set_error(YAH_ERR_IO, "gguf: " + path + ": duplicate tensor " + name);
    g->by_name[name] = (int64_t)t;
    g->tensors.push_back(ti);
  }
  if (!c.ok || g->tensors.size() != n_tensors)
    return set_error(YAH_ERR_IO, "gguf: " + path + ": tensor table truncated or malformed");
  const uint64_t a = g->alignment;
  g->data_offset = (c.pos + a - 1) / a * a;
  if (g->data_offset > g->size) return set_error(YAH_ERR_IO, "gguf: " + path + ": no tensor-data region");
  const uint64_t data_bytes = g->size - g->data_offset;
  for (const yah_gguf_tensor& t : g->tensors) {
    if (t.offset % a)
      return set_error(YAH_ERR_IO, "gguf: " + path + ": tensor " + t.name + " is not aligned to " + std::to_string(a));
    if (t.offset > data_bytes || t.bytes > data_bytes - t.offset)
      return set_error(YAH_ERR_IO, "gguf: " + path + ": tensor " + t.name + " lies beyond the end of the file");
  }
  return YAH_OK;
}

const Meta* find_meta(const yah_gguf* g, const char* key) {
  if (!g || !key) return nullptr;
  auto it = g->meta.find(key);
  return it == g->meta.end() ? nullptr : &it->second;
}

int cuda_err(cudaError_t e, const char* what) {
  return set_error(YAH_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

int yah_gguf_open(const char* path, yah_gguf** out) {
  if (!path || !out) return set_error(YAH_ERR_ARG, "gguf: null path or handle");
  *out = nullptr;
  auto* g = new yah_gguf;
  g->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (g->fd < 0) {
    delete g;
    return set_error(YAH_ERR_IO, std::string("gguf: cannot open ") + path + ": " + strerror(errno));
  }
  struct stat st;
  if (fstat(g->fd, &st) != 0 || st.st_size < 24) {
    delete g;
    return set_error(YAH_ERR_IO, std::string("gguf: ") + path + " is too short for a GGUF header");
  }
  g->size = (uint64_t)st.st_size;
  void* m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
  if (m == MAP_FAILED) {
    delete g;
    return set_error(YAH_ERR_IO, std::string("gguf: cannot map ") + path + ": " + strerror(errno));
  }
  g->base = static_cast<const uint8_t*>(m);
  const int rc = parse(g, path);
  if (rc) {
    delete g;
    return rc;
  }
  *out = g;
  return YAH_OK;
}

int yah_gguf_close(yah_gguf* g) {
  delete g;
  return YAH_OK;
}

int yah_gguf_version(const yah_gguf* g, uint32_t* version) {
  if (!g || !version) return set_error(YAH_ERR_ARG, "gguf: null argument");
  *version = g->version;
  return YAH_OK;
}

int yah_gguf_tensor_count(const yah_gguf* g, int64_t* n) {
  if (!g || !n) return set_error(YAH_ERR_ARG, "gguf: null argument");
  *n = (int64_t)g->tensors.size();
  return YAH_OK;
}

int yah_gguf_tensor_info(const yah_gguf* g, int64_t index, yah_gguf_tensor* out) {
  if (!g || !out) return set_error(YAH_ERR_ARG, "gguf: null argument");
  if (index < 0 || index >= (int64_t)g->tensors.size())
    return set_error(YAH_ERR_ARG, "gguf: tensor index " + std::to_string(index) + " out of range");
  *out = g->tensors[(size_t)index];
  return YAH_OK;
}

int yah_gguf_find(const yah_gguf* g, const char* name, int64_t* index) {
  if (!g || !name || !index) return set_error(YAH_ERR_ARG, "gguf: null argument");
  auto it = g->by_name.find(name);
  *index = it == g->by_name.end() ? -1 : it->second;
  if (*index < 0) return set_error(YAH_ERR_ARG, std::string("gguf: no tensor named ") + name);
  return YAH_OK;
}

int yah_gguf_data(const yah_gguf* g, const void** base, uint64_t* bytes) {
  if (!g || !base || !bytes) return set_error(YAH_ERR_ARG, "gguf: null argument");
  *base = g->base + g->data_offset;
  *bytes = g->size - g->data_offset;
  return YAH_OK;
}

int yah_gguf_meta_kind(const yah_gguf* g, const char* key, int* kind, uint64_t* count) {
  const Meta* m = find_meta(g, key);
  if (!kind || !m) return set_error(YAH_ERR_ARG, std::string("gguf: no metadata key ") + (key ? key : "(null)"));
  *kind = (int)m->kind;
  if (count) *count = m->kind == kArray ? m->count : 1;
  return YAH_OK;
}

int yah_gguf_meta_int(const yah_gguf* g, const char* key, int64_t* value) {
  const Meta* m = find_meta(g, key);
  if (!value || !m) return set_error(YAH_ERR_ARG, std::string("gguf: no metadata key ") + (key ? key : "(null)"));
  if (m->kind == kString || m->kind == kArray || m->kind == kF32 || m->kind == kF64)
    return set_error(YAH_ERR_ARG, std::string("gguf: metadata key ") + key + " is not an integer or bool");
  *value = m->i;
  return YAH_OK;
}

int yah_gguf_meta_float(const yah_gguf* g, const char* key, double* value) {
  const Meta* m = find_meta(g, key);
  if (!value || !m) return set_error(YAH_ERR_ARG, std::string("gguf: no metadata key ") + (key ? key : "(null)"));
  if (m->kind == kString || m->kind == kArray)
    return set_error(YAH_ERR_ARG, std::string("gguf: metadata key ") + key + " is not a number");
  *value = m->f;
  return YAH_OK;
}

int yah_gguf_meta_string(const yah_gguf* g, const char* key, char* buf, int64_t cap, int64_t* len) {
  const Meta* m = find_meta(g, key);
  if (!m) return set_error(YAH_ERR_ARG, std::string("gguf: no metadata key ") + (key ? key : "(null)"));
  if (m->kind != kString) return set_error(YAH_ERR_ARG, std::string("gguf: metadata key ") + key + " is not a string");
  if (len) *len = (int64_t)m->s.size();
  if (buf && cap > 0) {
    const size_t n = std::min<size_t>((size_t)cap - 1, m->s.size());
    std::memcpy(buf, m->s.data(), n);
    buf[n] = 0;
  }
  return YAH_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------ device chunks
struct yah_weights {
  struct Chunk {
    uint64_t begin, end;  // [begin, end) of the tensor-data region held
    uint8_t* dev;
  };
  std::vector<Chunk> chunks;
  int device = 0;

  ~yah_weights() {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    for (Chunk& c : chunks) cudaFree(c.dev);
    cudaSetDevice(cur);
  }
};

extern "C" {

int yah_weights_upload(const yah_gguf* g, uint64_t chunk_bytes, void* stream, yah_weights** out) {
  if (!g || !out) return set_error(YAH_ERR_ARG, "weights: null argument");
  *out = nullptr;
  if (chunk_bytes == 0) chunk_bytes = 1ull << 30;
  constexpr uint64_t kPad = 64 << 10;  // a kernel's over-read past a chunk's last tensor stays in the allocation
  std::vector<std::pair<uint64_t, uint64_t>> spans;
  for (const yah_gguf_tensor& t : g->tensors) spans.emplace_back(t.offset, t.offset + t.bytes);
  std::sort(spans.begin(), spans.end());
  auto* w = new yah_weights;
  if (cudaGetDevice(&w->device) != cudaSuccess) {
    delete w;
    return set_error(YAH_ERR_CUDA, "weights: no current device");
  }
  const uint8_t* src = g->base + g->data_offset;
  for (size_t i = 0; i < spans.size();) {
    const uint64_t begin = spans[i].first;
    uint64_t end = spans[i].second;
    for (++i; i < spans.size() && spans[i].second - begin <= chunk_bytes; ++i) end = std::max(end, spans[i].second);
    yah_weights::Chunk c{begin, end, nullptr};
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&c.dev), end - begin + kPad);
    if (e == cudaSuccess) e = cudaMemsetAsync(c.dev + (end - begin), 0, kPad, (cudaStream_t)stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(c.dev, src + begin, end - begin, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e != cudaSuccess) {
      if (c.dev) cudaFree(c.dev);
      delete w;
      return cuda_err(e, "weights: chunk upload");
    }
    w->chunks.push_back(c);
  }
  const cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);  // the mapping may be closed after return
  if (e != cudaSuccess) {
    delete w;
    return cuda_err(e, "weights: upload");
  }
  *out = w;
  return YAH_OK;
}

int yah_weights_ref(const yah_weights* w, uint64_t offset, uint64_t bytes, const void** dev) {
  if (!w || !dev) return set_error(YAH_ERR_ARG, "weights: null argument");
  *dev = nullptr;
  auto it = std::upper_bound(w->chunks.begin(), w->chunks.end(), offset,
                             [](uint64_t o, const yah_weights::Chunk& c) { return o < c.begin; });
  if (it == w->chunks.begin()) return set_error(YAH_ERR_ARG, "weights: offset before the first tensor");
  --it;
  if (offset > it->end || bytes > it->end - offset)
    return set_error(YAH_ERR_ARG, "weights: [" + std::to_string(offset) + ", +" + std::to_string(bytes) +
                                      ") is not inside one uploaded chunk");
  *dev = it->dev + (offset - it->begin);
  return YAH_OK;
}

int yah_weights_chunk_count(const yah_weights* w, int64_t* n) {
  if (!w || !n) return set_error(YAH_ERR_ARG, "weights: null argument");
  *n = (int64_t)w->chunks.size();
  return YAH_OK;
}

int yah_weights_free(yah_weights* w) {
  delete w;
  return YAH_OK;
}

}  // extern "C"
