// Safetensors reader behind the C ABI (host code; no device calls).
//
// Same format, limits and errors as the reference's SafetensorsFile
// (nnmetal/src/safetensors.zig): an 8-byte little-endian header length, a
// JSON header of tensor descriptors {"dtype", "shape", "data_offsets"}
// ("__metadata__" skipped), then the tensor bytes; the file is memory-mapped
// and descriptors point into the mapping.  Limits: header <= 16 MiB and
// inside the file, <= 1024 tensors, names <= 256 bytes, <= 4 dimensions,
// dtypes U8 / U32 / F16 / F32 / BF16, offsets ordered and inside the data
// region.  One check beyond the reference, which leaves it to its loader: a
// tensor's byte range must equal its element count times the dtype size.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "../../include/nnz_b200.h"
#include "json_reader.h"

namespace nnz {
void set_last_error(const std::string& msg);   // nnz_last_error() text (engine.cu)
}

namespace {

using nnz_json::JsonReader;
using nnz_json::JVal;

// Limits of safetensors.zig:28-39.
constexpr uint32_t kMaxTensors = 1024;
constexpr uint32_t kMaxDims = 4;
constexpr uint64_t kMaxHeaderBytes = 16ull * 1024 * 1024;
constexpr size_t kMaxNameLength = 256;

int fail(int code, const std::string& msg) {
  nnz::set_last_error(msg);
  return code;
}

// No C++ exception crosses the C ABI: a failed host allocation becomes
// NNZ_ENOMEM.
template <typename F>
int host_guard(F&& f) {
  try {
    return f();
  } catch (const std::bad_alloc&) {
    return fail(NNZ_ENOMEM, "OutOfMemory: host allocation failed");
  } catch (const std::exception& e) {
    return fail(NNZ_EINVAL, std::string("host error: ") + e.what());
  }
}

// Dtype.fromString / sizeBytes (safetensors.zig:45-78).
bool dtype_of(const std::string& s, int* code, uint32_t* size) {
  if (s == "U8") { *code = NNZ_DT_U8; *size = 1; return true; }
  if (s == "U32") { *code = NNZ_DT_U32; *size = 4; return true; }
  if (s == "F16") { *code = NNZ_DT_F16; *size = 2; return true; }
  if (s == "F32") { *code = NNZ_DT_F32; *size = 4; return true; }
  if (s == "BF16") { *code = NNZ_DT_BF16; *size = 2; return true; }
  return false;
}

struct Tensor {
  std::string name;
  int dtype;
  uint32_t rank;
  uint32_t dims[kMaxDims];
  uint64_t offset;   // into the data region
  uint64_t nbytes;
};

}  // namespace

struct nnz_safetensors {
  const uint8_t* base = nullptr;   // whole file (mapped or caller-owned)
  size_t size = 0;
  bool mapped = false;
  const uint8_t* data = nullptr;   // data region
  std::vector<Tensor> tensors;

  ~nnz_safetensors() {
    if (mapped && base) munmap(const_cast<uint8_t*>(base), size);
  }

  // parseHeaderFromSlice / parseJsonHeader / parseTensorEntry
  // (safetensors.zig:227-521)
  int parse() {
    if (size < 10) return fail(NNZ_EINVAL, "InvalidHeader: file shorter than 10 bytes");
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | base[i];
    if (hlen > kMaxHeaderBytes)
      return fail(NNZ_EINVAL, "InvalidHeader: header length " + std::to_string(hlen) + " exceeds 16 MiB");
    if (8 + hlen > size)
      return fail(NNZ_EINVAL, "InvalidHeader: header length (" + std::to_string(hlen) + ") exceeds file size (" +
                                  std::to_string(size) + ")");
    data = base + 8 + hlen;
    const uint64_t data_size = size - 8 - hlen;
    JVal root;
    std::string err;
    if (hlen == 0 || !JsonReader(reinterpret_cast<const char*>(base + 8), hlen).parse(root, err))
      return fail(NNZ_EINVAL, "InvalidJson: " + (hlen == 0 ? std::string("empty header") : err));
    if (root.kind != JVal::OBJ) return fail(NNZ_EINVAL, "InvalidJson: header is not an object");
    for (const auto& [name, v] : root.obj) {
      if (name == "__metadata__") continue;
      if (tensors.size() >= kMaxTensors) return fail(NNZ_EINVAL, "TooManyTensors: more than 1024");
      if (name.empty() || name.size() > kMaxNameLength)
        return fail(NNZ_EINVAL, "InvalidTensorEntry: tensor name empty or longer than 256 bytes");
      if (v.kind != JVal::OBJ) return fail(NNZ_EINVAL, "InvalidTensorEntry: '" + name + "'");
      Tensor t{};
      t.name = name;
      const JVal* dt = v.get("dtype");
      if (!dt) return fail(NNZ_EINVAL, "MissingDtype: '" + name + "'");
      if (dt->kind != JVal::STR) return fail(NNZ_EINVAL, "InvalidDtype: '" + name + "'");
      uint32_t esize = 0;
      if (!dtype_of(dt->s, &t.dtype, &esize))
        return fail(NNZ_EINVAL, "UnsupportedDtype: '" + name + "' has " + dt->s);
      const JVal* sh = v.get("shape");
      if (!sh) return fail(NNZ_EINVAL, "MissingShape: '" + name + "'");
      if (sh->kind != JVal::ARR) return fail(NNZ_EINVAL, "InvalidShape: '" + name + "'");
      if (sh->arr.size() > kMaxDims)
        return fail(NNZ_EINVAL, "TooManyDimensions: '" + name + "' has " + std::to_string(sh->arr.size()));
      t.rank = (uint32_t)sh->arr.size();
      uint64_t count = 1;
      for (uint32_t i = 0; i < t.rank; ++i) {
        const JVal& d = sh->arr[i];
        if (d.kind != JVal::INT || d.i < 0 || d.i > 0xFFFFFFFFll)
          return fail(NNZ_EINVAL, "InvalidShape: '" + name + "'");
        t.dims[i] = (uint32_t)d.i;
        // checked product: a wrapped element count must not pass the size check
        if (t.dims[i] && count > UINT64_MAX / t.dims[i])
          return fail(NNZ_EINVAL, "InvalidShape: '" + name + "' element count overflows");
        count *= t.dims[i];
      }
      if (esize && count > UINT64_MAX / esize)
        return fail(NNZ_EINVAL, "InvalidShape: '" + name + "' byte size overflows");
      const JVal* off = v.get("data_offsets");
      if (!off) return fail(NNZ_EINVAL, "MissingDataOffsets: '" + name + "'");
      if (off->kind != JVal::ARR || off->arr.size() != 2 || off->arr[0].kind != JVal::INT ||
          off->arr[1].kind != JVal::INT || off->arr[0].i < 0 || off->arr[1].i < 0)
        return fail(NNZ_EINVAL, "InvalidDataOffsets: '" + name + "'");
      const uint64_t s0 = (uint64_t)off->arr[0].i, s1 = (uint64_t)off->arr[1].i;
      if (s1 < s0) return fail(NNZ_EINVAL, "InvalidDataOffsets: '" + name + "'");
      if (s1 > data_size)
        return fail(NNZ_EINVAL, "DataOffsetOutOfBounds: '" + name + "' ends at " + std::to_string(s1) + " of " +
                                    std::to_string(data_size));
      if (s1 - s0 != count * esize)
        return fail(NNZ_EINVAL, "InvalidDataOffsets: '" + name + "' holds " + std::to_string(s1 - s0) +
                                    " bytes, shape needs " + std::to_string(count * esize));
      t.offset = s0;
      t.nbytes = s1 - s0;
      tensors.push_back(std::move(t));
    }
    return NNZ_OK;
  }

  void describe(const Tensor& t, nnz_tensor_desc* d) const {
    d->name = t.name.c_str();
    d->dtype = t.dtype;
    d->rank = t.rank;
    for (uint32_t i = 0; i < kMaxDims; ++i) d->dims[i] = i < t.rank ? t.dims[i] : 0;
    d->data = data + t.offset;
    d->nbytes = (size_t)t.nbytes;
  }
};

extern "C" {

static int safetensors_open_impl(const char* path, nnz_safetensors** out) {
  if (!path || !*path || !out) return fail(NNZ_EINVAL, "nnz_safetensors_open: null or empty path");
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(NNZ_ENOTFOUND, std::string("FileNotFound: cannot open ") + path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    return fail(NNZ_EINVAL, std::string("InvalidHeader: cannot stat ") + path);
  }
  auto f = std::make_unique<nnz_safetensors>();
  f->size = (size_t)st.st_size;
  if (f->size >= 10) {
    void* p = mmap(nullptr, f->size, PROT_READ, MAP_SHARED, fd, 0);
    if (p == MAP_FAILED) {
      close(fd);
      return fail(NNZ_EINVAL, std::string("InvalidHeader: cannot map ") + path);
    }
    f->base = static_cast<const uint8_t*>(p);
    f->mapped = true;
  }
  close(fd);   // the mapping stays valid
  const int rc = f->parse();
  if (rc != NNZ_OK) return rc;
  *out = f.release();
  return NNZ_OK;
}

int nnz_safetensors_open(const char* path, nnz_safetensors** out) {
  return host_guard([&] { return safetensors_open_impl(path, out); });
}

static int safetensors_from_bytes_impl(const void* bytes, size_t len, nnz_safetensors** out) {
  if (!out || (!bytes && len)) return fail(NNZ_EINVAL, "nnz_safetensors_from_bytes: null argument");
  *out = nullptr;
  auto f = std::make_unique<nnz_safetensors>();
  f->base = static_cast<const uint8_t*>(bytes);
  f->size = len;
  const int rc = f->parse();
  if (rc != NNZ_OK) return rc;
  *out = f.release();
  return NNZ_OK;
}

int nnz_safetensors_from_bytes(const void* bytes, size_t len, nnz_safetensors** out) {
  return host_guard([&] { return safetensors_from_bytes_impl(bytes, len, out); });
}

static int safetensors_close_impl(nnz_safetensors* f) {
  delete f;
  return NNZ_OK;
}

int nnz_safetensors_close(nnz_safetensors* f) {
  return host_guard([&] { return safetensors_close_impl(f); });
}

uint32_t nnz_safetensors_count(const nnz_safetensors* f) { return f ? (uint32_t)f->tensors.size() : 0; }

static int safetensors_tensor_impl(const nnz_safetensors* f, uint32_t index, nnz_tensor_desc* desc) {
  if (!f || !desc) return fail(NNZ_EINVAL, "nnz_safetensors_tensor: null argument");
  if (index >= f->tensors.size()) return fail(NNZ_EINVAL, "nnz_safetensors_tensor: index out of range");
  f->describe(f->tensors[index], desc);
  return NNZ_OK;
}

int nnz_safetensors_tensor(const nnz_safetensors* f, uint32_t index, nnz_tensor_desc* desc) {
  return host_guard([&] { return safetensors_tensor_impl(f, index, desc); });
}

static int safetensors_find_impl(const nnz_safetensors* f, const char* name, nnz_tensor_desc* desc) {
  if (!f || !name || !desc) return fail(NNZ_EINVAL, "nnz_safetensors_find: null argument");
  for (const Tensor& t : f->tensors)
    if (t.name == name) {
      f->describe(t, desc);
      return NNZ_OK;
    }
  return fail(NNZ_ENOTFOUND, std::string("TensorNotFound: ") + name);
}

int nnz_safetensors_find(const nnz_safetensors* f, const char* name, nnz_tensor_desc* desc) {
  return host_guard([&] { return safetensors_find_impl(f, name, desc); });
}

}  // extern "C"
