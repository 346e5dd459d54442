// gguf.h -- the GGUF reader used by exn_load_gguf.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace exn {

enum { GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8, GGML_BF16 = 30 };

struct GgufTensor {
  std::string name;
  std::vector<int64_t> dims;  // ggml order: contiguous axis first
  int type = -1;
  uint64_t offset = 0;
  size_t nbytes = 0;          // 0: a type this reader does not size
};

class GgufFile {
 public:
  ~GgufFile();
  bool open(const char* path, std::string& err);
  const uint8_t* data(const GgufTensor& t) const;
  std::string arch;
  std::vector<GgufTensor> tensors;
  uint64_t data_start = 0;

 private:
  int fd_ = -1;
  const uint8_t* map_ = nullptr;
  size_t size_ = 0;
};

size_t ggml_nbytes(int type, const std::vector<int64_t>& dims);

}  // namespace exn
