// NSF weight files: writer and checked reader (format in nsf.h).
#include "nsf.h"

#include <cstring>
#include <memory>

namespace nsb {
namespace nsf {
namespace {

constexpr char kMagic[8] = {'N', 'S', 'F', 'M', 'T', '0', '0', '1'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kFloat32 = 0;
constexpr uint32_t kMaxString = 1u << 20;

// 32-bit FNV-1a (offset basis 2166136261, prime 16777619): a serial chain
// over the bytes, so it runs on the host next to the file I/O.
struct Fnv1a {
  uint32_t h = 2166136261u;
  void update(const void* p, size_t n) {
    const unsigned char* b = static_cast<const unsigned char*>(p);
    uint32_t x = h;
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
      x = (x ^ b[i]) * 16777619u;
      x = (x ^ b[i + 1]) * 16777619u;
      x = (x ^ b[i + 2]) * 16777619u;
      x = (x ^ b[i + 3]) * 16777619u;
      x = (x ^ b[i + 4]) * 16777619u;
      x = (x ^ b[i + 5]) * 16777619u;
      x = (x ^ b[i + 6]) * 16777619u;
      x = (x ^ b[i + 7]) * 16777619u;
    }
    for (; i < n; ++i) x = (x ^ b[i]) * 16777619u;
    h = x;
  }
};

struct FileCloser {
  void operator()(FILE* f) const {
    if (f) std::fclose(f);
  }
};
using File = std::unique_ptr<FILE, FileCloser>;

class Out {
 public:
  explicit Out(FILE* f) : f_(f) {}
  void bytes(const void* p, size_t n) {
    if (n && std::fwrite(p, 1, n, f_) != n) ok_ = false;
    sum_.update(p, n);
  }
  template <typename T>
  void pod(T v) {
    bytes(&v, sizeof(T));
  }
  void str(const std::string& s) {
    pod<uint32_t>((uint32_t)s.size());
    bytes(s.data(), s.size());
  }
  bool ok() const { return ok_; }
  uint32_t sum() const { return sum_.h; }

 private:
  FILE* f_;
  Fnv1a sum_;
  bool ok_ = true;
};

class In {
 public:
  explicit In(FILE* f) : f_(f) {}
  bool bytes(void* p, size_t n) {
    if (n && std::fread(p, 1, n, f_) != n) return false;
    sum_.update(p, n);
    return true;
  }
  template <typename T>
  bool pod(T* v) {
    return bytes(v, sizeof(T));
  }
  bool str(std::string* s) {
    uint32_t n = 0;
    if (!pod(&n) || n > kMaxString) return false;
    s->assign(n, '\0');
    return bytes(n ? &(*s)[0] : nullptr, n);
  }
  uint32_t sum() const { return sum_.h; }

 private:
  FILE* f_;
  Fnv1a sum_;
};

}  // namespace

std::string Write(const std::string& path, const std::map<std::string, std::string>& meta,
                  const std::vector<Entry>& entries) {
  File f(std::fopen(path.c_str(), "wb"));
  if (!f) return "cannot open for writing: " + path;
  std::setvbuf(f.get(), nullptr, _IOFBF, 8 << 20);
  Out o(f.get());
  o.bytes(kMagic, sizeof(kMagic));
  o.pod<uint32_t>(kVersion);
  o.pod<uint32_t>((uint32_t)meta.size());
  for (const auto& kv : meta) {
    o.str(kv.first);
    o.str(kv.second);
  }
  o.pod<uint32_t>((uint32_t)entries.size());
  for (const Entry& e : entries) {
    o.str(e.name);
    o.pod<uint32_t>(kFloat32);
    o.pod<uint32_t>((uint32_t)e.dims.size());
    for (int d : e.dims) o.pod<int32_t>(d);
    const uint64_t nb = e.numel() * sizeof(float);
    o.pod<uint64_t>(nb);
    o.bytes(e.data, (size_t)nb);
  }
  const uint32_t sum = o.sum();
  if (std::fwrite(&sum, 1, sizeof(sum), f.get()) != sizeof(sum) || !o.ok())
    return "write error: " + path;
  if (std::fflush(f.get()) != 0) return "write error: " + path;
  return "";
}

std::string Read(const std::string& path, const std::map<std::string, std::string>& expected,
                 const std::vector<Entry>& entries, std::map<std::string, std::string>* meta_out) {
  File f(std::fopen(path.c_str(), "rb"));
  if (!f) return "cannot open for reading: " + path;
  std::setvbuf(f.get(), nullptr, _IOFBF, 8 << 20);
  In in(f.get());
  char magic[8];
  if (!in.bytes(magic, sizeof(magic)) || std::memcmp(magic, kMagic, sizeof(magic)) != 0)
    return path + ": not an NSF file (no NSFMT001 header)";
  uint32_t version = 0;
  if (!in.pod(&version)) return path + ": truncated header";
  if (version != kVersion)
    return path + ": format version " + std::to_string(version) + ", this build reads version " +
           std::to_string(kVersion);
  uint32_t n_meta = 0;
  if (!in.pod(&n_meta)) return path + ": truncated metadata";
  std::map<std::string, std::string> meta;
  for (uint32_t i = 0; i < n_meta; ++i) {
    std::string k, v;
    if (!in.str(&k) || !in.str(&v)) return path + ": truncated metadata";
    meta[k] = v;
  }
  for (const auto& kv : expected) {
    auto it = meta.find(kv.first);
    if (it == meta.end()) return path + ": the file does not declare '" + kv.first + "'";
    if (it->second != kv.second)
      return path + ": " + kv.first + " is " + it->second + " in the file and " + kv.second +
             " in the model";
  }
  uint32_t n = 0;
  if (!in.pod(&n)) return path + ": truncated tensor table";
  if (n != entries.size())
    return path + ": " + std::to_string(n) + " tensors in the file, " +
           std::to_string(entries.size()) + " in the model";
  for (uint32_t i = 0; i < n; ++i) {
    const Entry& e = entries[i];
    std::string name;
    uint32_t dtype = 0, rank = 0;
    if (!in.str(&name) || !in.pod(&dtype) || !in.pod(&rank))
      return path + ": tensor " + std::to_string(i) + " truncated";
    if (name != e.name)
      return path + ": tensor " + std::to_string(i) + " is '" + name + "', the model expects '" +
             e.name + "'";
    if (dtype != kFloat32) return path + ": '" + name + "' is not float32";
    if (rank > 8) return path + ": '" + name + "' has rank " + std::to_string(rank);
    std::vector<int> dims(rank);
    for (uint32_t d = 0; d < rank; ++d) {
      int32_t v = 0;
      if (!in.pod(&v)) return path + ": truncated shape";
      dims[d] = v;
    }
    if (dims != e.dims) return path + ": '" + name + "' has a different shape from the model's";
    uint64_t nb = 0;
    if (!in.pod(&nb)) return path + ": truncated length";
    if (nb != e.numel() * sizeof(float))
      return path + ": '" + name + "' declares " + std::to_string(nb) + " bytes, expected " +
             std::to_string(e.numel() * sizeof(float));
    if (!in.bytes(e.out, (size_t)nb)) return path + ": data of '" + name + "' truncated";
  }
  uint32_t stored = 0;
  if (std::fread(&stored, 1, sizeof(stored), f.get()) != sizeof(stored))
    return path + ": checksum missing";
  if (stored != in.sum()) return path + ": checksum mismatch; the file is corrupt";
  if (meta_out) *meta_out = meta;
  return "";
}

}  // namespace nsf
}  // namespace nsb
