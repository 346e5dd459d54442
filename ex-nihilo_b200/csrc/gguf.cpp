// gguf.cpp -- a reader for the GGUF files the DiT comes in: the header, the
// metadata (only general.architecture is kept), the tensor directory, and the
// tensor data by mmap.  Format version 2 and 3, little endian.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace exn {

namespace {

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (end - p < static_cast<long>(sizeof(T))) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || static_cast<uint64_t>(end - p) < n) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
  void skip(uint64_t n) {
    if (static_cast<uint64_t>(end - p) < n) {
      ok = false;
      return;
    }
    p += n;
  }
};

// GGUF metadata value types
enum { T_U8 = 0, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 };

size_t scalar_size(uint32_t t) {
  switch (t) {
    case T_U8: case T_I8: case T_BOOL: return 1;
    case T_U16: case T_I16: return 2;
    case T_U32: case T_I32: case T_F32: return 4;
    case T_U64: case T_I64: case T_F64: return 8;
  }
  return 0;
}

void skip_value(Cursor& c, uint32_t t, int depth = 0) {
  if (depth > 4) {
    c.ok = false;
    return;
  }
  if (t == T_STR) {
    c.str();
  } else if (t == T_ARR) {
    const uint32_t et = c.get<uint32_t>();
    const uint64_t n = c.get<uint64_t>();
    if (et == T_STR || et == T_ARR) {
      for (uint64_t i = 0; i < n && c.ok; ++i) skip_value(c, et, depth + 1);
    } else {
      const size_t s = scalar_size(et);
      if (!s) c.ok = false;
      else c.skip(n * s);
    }
  } else {
    const size_t s = scalar_size(t);
    if (!s) c.ok = false;
    else c.skip(s);
  }
}

}  // namespace

size_t ggml_nbytes(int type, const std::vector<int64_t>& dims) {
  int64_t n = 1;
  for (int64_t d : dims) n *= d;
  switch (type) {
    case GGML_F32: return static_cast<size_t>(n) * 4;
    case GGML_F16: case GGML_BF16: return static_cast<size_t>(n) * 2;
    case GGML_Q8_0: return (dims.empty() || dims[0] % 32) ? 0 : static_cast<size_t>(n / 32) * 34;
  }
  return 0;
}

GgufFile::~GgufFile() {
  if (map_) munmap(const_cast<uint8_t*>(map_), size_);
  if (fd_ >= 0) close(fd_);
}

bool GgufFile::open(const char* path, std::string& err) {
  fd_ = ::open(path, O_RDONLY);
  if (fd_ < 0) {
    err = std::string(path) + ": cannot open";
    return false;
  }
  struct stat st;
  if (fstat(fd_, &st) != 0 || st.st_size < 24) {
    err = std::string(path) + ": not a GGUF file";
    return false;
  }
  size_ = static_cast<size_t>(st.st_size);
  void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (m == MAP_FAILED) {
    err = std::string(path) + ": mmap failed";
    return false;
  }
  map_ = static_cast<const uint8_t*>(m);
  Cursor c{map_, map_ + size_};
  if (std::memcmp(map_, "GGUF", 4) != 0) {
    err = std::string(path) + ": not a GGUF file";
    return false;
  }
  c.skip(4);
  const uint32_t version = c.get<uint32_t>();
  if (version < 2 || version > 3) {
    err = std::string(path) + ": GGUF version " + std::to_string(version);
    return false;
  }
  const uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < nkv && c.ok; ++i) {
    const std::string key = c.str();
    const uint32_t t = c.get<uint32_t>();
    if (key == "general.architecture" && t == T_STR) {
      arch = c.str();
    } else if (key == "general.alignment" && t == T_U32) {
      alignment = c.get<uint32_t>();
    } else {
      skip_value(c, t);
    }
  }
  for (uint64_t i = 0; i < nt && c.ok; ++i) {
    GgufTensor ti;
    ti.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    if (nd > 4) {
      c.ok = false;
      break;
    }
    for (uint32_t d = 0; d < nd; ++d) ti.dims.push_back(static_cast<int64_t>(c.get<uint64_t>()));
    ti.type = static_cast<int>(c.get<uint32_t>());
    ti.offset = c.get<uint64_t>();
    ti.nbytes = ggml_nbytes(ti.type, ti.dims);
    tensors.push_back(std::move(ti));
  }
  if (!c.ok || alignment == 0) {
    err = std::string(path) + ": truncated or malformed GGUF header";
    return false;
  }
  const uint64_t hdr = static_cast<uint64_t>(c.p - map_);
  data_start = (hdr + alignment - 1) / alignment * alignment;
  for (const auto& t : tensors) {
    if (t.nbytes && data_start + t.offset + t.nbytes > size_) {
      err = std::string(path) + ": tensor " + t.name + " runs past the end of the file";
      return false;
    }
  }
  return true;
}

const uint8_t* GgufFile::data(const GgufTensor& t) const { return map_ + data_start + t.offset; }

}  // namespace exn
