// safetensors.cpp -- mmap-based safetensors reader (see safetensors.h).
//
// Layout: u64 little-endian header length n, n bytes of UTF-8 JSON mapping
// each tensor name to {"dtype", "shape", "data_offsets": [begin, end]}
// (offsets relative to the byte after the header), plus an optional
// "__metadata__" object of strings.  The file is mapped read-only and the
// tensors are returned as views into the mapping.
#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace gsv {

namespace {

struct Json {
  const char* p;
  const char* end;
  std::string err;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool expect(char c) {
    ws();
    if (p >= end || *p != c) {
      err = std::string("expected '") + c + "'";
      return false;
    }
    ++p;
    return true;
  }
  bool string(std::string& out) {
    ws();
    if (p >= end || *p != '"') { err = "expected a string"; return false; }
    ++p;
    out.clear();
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) break;
        switch (*p) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (end - p < 5) { err = "bad \\u escape"; return false; }
            unsigned v = 0;
            for (int i = 1; i <= 4; ++i) {
              char c = p[i];
              v <<= 4;
              if (c >= '0' && c <= '9') v |= c - '0';
              else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
              else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
              else { err = "bad \\u escape"; return false; }
            }
            if (v < 0x80) out += (char)v;
            else if (v < 0x800) { out += (char)(0xC0 | (v >> 6)); out += (char)(0x80 | (v & 63)); }
            else { out += (char)(0xE0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 63)); out += (char)(0x80 | (v & 63)); }
            p += 4;
            break;
          }
          default: out += *p;
        }
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= end) { err = "unterminated string"; return false; }
    ++p;
    return true;
  }
  bool integer(int64_t& v) {
    ws();
    bool neg = false;
    if (p < end && *p == '-') { neg = true; ++p; }
    if (p >= end || *p < '0' || *p > '9') { err = "expected an integer"; return false; }
    v = 0;
    while (p < end && *p >= '0' && *p <= '9') {
      if (v > (INT64_MAX - 9) / 10) { err = "integer overflow"; return false; }
      v = v * 10 + (*p++ - '0');
    }
    if (neg) v = -v;
    return true;
  }
  bool int_array(std::vector<int64_t>& out) {
    out.clear();
    if (!expect('[')) return false;
    ws();
    if (p < end && *p == ']') { ++p; return true; }
    for (;;) {
      int64_t v;
      if (!integer(v)) return false;
      out.push_back(v);
      ws();
      if (p < end && *p == ',') { ++p; continue; }
      return expect(']');
    }
  }
  // Skips any JSON value (used for __metadata__ and unknown fields).
  bool skip() {
    ws();
    if (p >= end) { err = "unexpected end"; return false; }
    if (*p == '"') { std::string s; return string(s); }
    if (*p == '{' || *p == '[') {
      const char open = *p, close = open == '{' ? '}' : ']';
      ++p;
      ws();
      if (p < end && *p == close) { ++p; return true; }
      for (;;) {
        if (open == '{') {
          std::string k;
          if (!string(k) || !expect(':')) return false;
        }
        if (!skip()) return false;
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        return expect(close);
      }
    }
    while (p < end && *p != ',' && *p != '}' && *p != ']') ++p;  // number / literal
    return true;
  }
};

size_t dtype_size(const std::string& d) {
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  return 0;
}

}  // namespace

bool parse_st_header(const char* json, size_t len, const uint8_t* data, size_t data_len,
                     std::vector<StEntry>& out, std::string& err) {
  Json j{json, json + len, {}};
  out.clear();
  if (!j.expect('{')) { err = j.err; return false; }
  j.ws();
  if (j.p < j.end && *j.p == '}') return true;
  for (;;) {
    std::string name;
    if (!j.string(name) || !j.expect(':')) { err = j.err; return false; }
    if (name == "__metadata__") {
      if (!j.skip()) { err = j.err; return false; }
    } else {
      StEntry e;
      e.name = name;
      int64_t b = -1, en = -1;
      bool have_off = false;
      if (!j.expect('{')) { err = j.err; return false; }
      for (;;) {
        std::string key;
        if (!j.string(key) || !j.expect(':')) { err = j.err; return false; }
        if (key == "dtype") {
          if (!j.string(e.dtype)) { err = j.err; return false; }
        } else if (key == "shape") {
          if (!j.int_array(e.shape)) { err = j.err; return false; }
        } else if (key == "data_offsets") {
          std::vector<int64_t> o;
          if (!j.int_array(o) || o.size() != 2) { err = "bad data_offsets for " + name; return false; }
          b = o[0]; en = o[1]; have_off = true;
        } else if (!j.skip()) {
          err = j.err;
          return false;
        }
        j.ws();
        if (j.p < j.end && *j.p == ',') { ++j.p; continue; }
        if (!j.expect('}')) { err = j.err; return false; }
        break;
      }
      const size_t es = dtype_size(e.dtype);
      if (!es) { err = "unknown dtype " + e.dtype + " for " + name; return false; }
      if (!have_off || b < 0 || en < b || (uint64_t)en > data_len) {
        err = "data_offsets out of range for " + name;
        return false;
      }
      int64_t n = 1;
      for (int64_t d : e.shape) {
        if (d < 0) { err = "negative dimension in " + name; return false; }
        n *= d;
      }
      if ((uint64_t)(en - b) != (uint64_t)n * es) { err = "size mismatch for " + name; return false; }
      e.data = data + b;
      e.nbytes = (size_t)(en - b);
      out.push_back(std::move(e));
    }
    j.ws();
    if (j.p < j.end && *j.p == ',') { ++j.p; continue; }
    if (!j.expect('}')) { err = j.err; return false; }
    return true;
  }
}

StFile::~StFile() {
  if (map_) munmap(map_, size_);
}

bool StFile::open(const char* path, std::string& err) {
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) { err = std::string("Failed to open file: ") + path; return false; }
  struct stat stt;
  if (fstat(fd, &stt) != 0 || stt.st_size < 8) {
    ::close(fd);
    err = "Failed to read file: too short";
    return false;
  }
  size_ = (size_t)stt.st_size;
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) { map_ = nullptr; err = "mmap failed"; return false; }
  const uint8_t* base = static_cast<const uint8_t*>(map_);
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | base[i];
  if (n > size_ - 8) { err = "Failed to parse safetensors: header length out of range"; return false; }
  if (!parse_st_header(reinterpret_cast<const char*>(base + 8), (size_t)n, base + 8 + n,
                       size_ - 8 - (size_t)n, entries_, err)) {
    err = "Failed to parse safetensors: " + err;
    return false;
  }
  return true;
}

}  // namespace gsv
