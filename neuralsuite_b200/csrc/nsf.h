// NSF weight files (the reference's checkpoint format, include/serialization.h:17-29):
//
//   magic "NSFMT001" | version u32 = 1 | n_meta u32, then (key, value) strings |
//   n_tensors u32, then per tensor: name string, dtype u32 (0 = float32),
//   rank u32, dims i32[rank], n_bytes u64, data | checksum u32
//
// strings are u32 length + bytes, integers little-endian, and the checksum is
// 32-bit FNV-1a over every byte before it.  Metadata are written in key
// order (the reference keeps them in a std::map).  The format has to match
// byte for byte so that files move between the reference and this library;
// the code is this library's own (host side; the device copy happens in the
// callers).
#pragma once

#include <cstdint>
#include <cstdio>
#include <map>
#include <string>
#include <vector>

namespace nsb {
namespace nsf {

// One tensor of a file: name, shape, and its floats in host memory.
struct Entry {
  std::string name;
  std::vector<int> dims;
  const float* data = nullptr;  // write: source; read: filled by Read into `out`
  float* out = nullptr;
  uint64_t numel() const {
    uint64_t n = 1;
    for (int d : dims) n *= (uint64_t)d;
    return dims.empty() ? 0 : n;
  }
};

// Writes `entries` and `meta` to `path`.  Returns "" or the reason it failed.
std::string Write(const std::string& path, const std::map<std::string, std::string>& meta,
                  const std::vector<Entry>& entries);

// Reads `path`, checking magic, version, every expected metadata value, the
// tensor count, each tensor's name, dtype, shape and byte count, and the
// checksum; the floats go to entries[i].out.  All checks run before the
// caller sees any data: on failure the outputs may hold a partial read and
// must be discarded.  Returns "" or the reason.  `meta_out` (optional)
// receives every metadata entry of the file.
std::string Read(const std::string& path, const std::map<std::string, std::string>& expected,
                 const std::vector<Entry>& entries,
                 std::map<std::string, std::string>* meta_out = nullptr);

}  // namespace nsf
}  // namespace nsb
