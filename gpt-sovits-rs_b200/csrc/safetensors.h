// safetensors.h -- minimal reader of the safetensors container (mmap + JSON
// header), the on-disk format the reference loads with
// `load_safetensors` (src/utils/weights.rs:116-162) and writes with
// gpt-sovits-convert (src/bin/gpt-sovits-convert.rs:282-309).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace gsv {

struct StEntry {
  std::string name;
  std::string dtype;  // "F32", "F16", "BF16", "I64", ...
  std::vector<int64_t> shape;
  const void* data = nullptr;
  size_t nbytes = 0;
};

class StFile {
 public:
  StFile() = default;
  ~StFile();
  StFile(const StFile&) = delete;
  StFile& operator=(const StFile&) = delete;
  // Maps `path` and parses its header.  Returns false with `err` set on failure.
  bool open(const char* path, std::string& err);
  const std::vector<StEntry>& entries() const { return entries_; }

 private:
  void* map_ = nullptr;
  size_t size_ = 0;
  std::vector<StEntry> entries_;
};

// Parses a safetensors header (the JSON text) against a data region of
// `data_len` bytes starting at `data`.  Exposed for tests of the parser.
bool parse_st_header(const char* json, size_t len, const uint8_t* data, size_t data_len,
                     std::vector<StEntry>& out, std::string& err);

}  // namespace gsv
