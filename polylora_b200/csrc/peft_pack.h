// Host side of the GPU slot refills: packs a PEFT adapter's safetensors file
// into a slot image (the plora_slot_fill layout) in one pass, without Python.
//
// The CPU tier (polylora_b200/store.py) calls this from its prefetch workers
// through ctypes, which releases the interpreter lock for the call, so files
// are parsed in parallel with the serving thread.  It handles the common case
// only -- every LoRA tensor present, 2-D, of the image's element type, ranks
// consistent, all LoRA keys inside the configured modules -- and answers
// PLORA_ERR_UNSUPPORTED otherwise, so that the Python loader (which raises the
// reference's exact errors) takes over.  Key matching is the reference's
// (src/polylora/store.py: a module's weight is the first key, in data-offset
// order (the order safetensors' load_file returns the keys in),
// ending in "<module>.<lora_A|lora_B>[.<adapter name>].weight").
//
// safetensors layout: 8-byte little-endian header length n, n bytes of JSON
// ({"<name>": {"dtype", "shape", "data_offsets": [begin, end]}, ...,
// optional "__metadata__"}), then the data section the offsets index.
#pragma once

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <string_view>
#include <unordered_set>
#include <utility>
#include <vector>

#include "../../include/polylora_b200.h"

namespace plora {
namespace peft {

// ------------------------------------------------------------------ JSON
struct JVal {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  double num = 0;
  bool int_lit = false;  // the number was written as plain decimal digits
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;  // insertion (file) order
};

class JParser {
 public:
  JParser(const char* p, size_t n) : p_(p), end_(p + n) {}
  bool parse(JVal& v) {
    ws();
    if (!value(v, 0)) return false;
    ws();
    return p_ == end_;
  }

 private:
  const char* p_;
  const char* end_;

  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if ((size_t)(end_ - p_) < n || memcmp(p_, s, n) != 0) return false;
    p_ += n;
    return true;
  }
  bool hex4(uint32_t& cp) {
    if (end_ - p_ < 4) return false;
    cp = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      cp <<= 4;
      if (c >= '0' && c <= '9') cp |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') cp |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') cp |= (uint32_t)(c - 'A' + 10);
      else return false;
    }
    return true;
  }
  static void utf8(uint32_t cp, std::string& out) {
    if (cp < 0x80) {
      out += (char)cp;
    } else if (cp < 0x800) {
      out += (char)(0xC0 | (cp >> 6));
      out += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += (char)(0xE0 | (cp >> 12));
      out += (char)(0x80 | ((cp >> 6) & 0x3F));
      out += (char)(0x80 | (cp & 0x3F));
    } else {
      out += (char)(0xF0 | (cp >> 18));
      out += (char)(0x80 | ((cp >> 12) & 0x3F));
      out += (char)(0x80 | ((cp >> 6) & 0x3F));
      out += (char)(0x80 | (cp & 0x3F));
    }
  }
  bool string(std::string& out) {
    if (p_ >= end_ || *p_ != '"') return false;
    ++p_;
    while (p_ < end_ && *p_ != '"') {
      const char c = *p_++;
      if (c != '\\') {
        out += c;
        continue;
      }
      if (p_ >= end_) return false;
      const char e = *p_++;
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp;
          if (!hex4(cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            uint32_t lo;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return false;
            p_ += 2;
            if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(cp, out);
          break;
        }
        default:
          return false;
      }
    }
    if (p_ >= end_) return false;
    ++p_;
    return true;
  }
  bool number(double& out, bool& int_lit) {
    const char* s = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                         *p_ == '+' || *p_ == '-'))
      ++p_;
    if (p_ == s || p_ - s > 64) return false;
    char buf[72];
    memcpy(buf, s, (size_t)(p_ - s));
    buf[p_ - s] = 0;
    char* stop = nullptr;
    out = strtod(buf, &stop);
    int_lit = true;
    for (const char* q = s; q < p_; ++q) int_lit = int_lit && *q >= '0' && *q <= '9';
    return stop == buf + (p_ - s);
  }
  bool value(JVal& v, int depth) {
    if (depth > 64 || p_ >= end_) return false;
    ws();
    if (p_ >= end_) return false;
    const char c = *p_;
    if (c == '{') {
      v.kind = JVal::kObj;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      for (;;) {
        ws();
        std::string key;
        if (!string(key)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return false;
        ++p_;
        v.obj.emplace_back(std::move(key), JVal());
        if (!value(v.obj.back().second, depth + 1)) return false;
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '[') {
      v.kind = JVal::kArr;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      for (;;) {
        v.arr.emplace_back();
        if (!value(v.arr.back(), depth + 1)) return false;
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '"') {
      v.kind = JVal::kStr;
      return string(v.str);
    }
    if (lit("true") || lit("false")) {
      v.kind = JVal::kBool;
      return true;
    }
    if (lit("null")) return true;
    v.kind = JVal::kNum;
    return number(v.num, v.int_lit);
  }
};

// ------------------------------------------------------------------ packing
struct TensorInfo {
  std::string name, dtype;
  std::vector<int64_t> shape;
  bool has_shape = false;
  int64_t begin = -1, end = -1;
};

// Element bytes of the safetensors dtypes this packer checks (0: any other,
// which the Python loader then judges).
inline int64_t dtype_bytes(const std::string& d) {
  if (d == "BOOL" || d == "U8" || d == "I8" || d == "F8_E5M2" || d == "F8_E4M3") return 1;
  if (d == "I16" || d == "U16" || d == "F16" || d == "BF16") return 2;
  if (d == "I32" || d == "U32" || d == "F32") return 4;
  if (d == "I64" || d == "U64" || d == "F64") return 8;
  return 0;
}

// Header size limit of the safetensors format's loader.
constexpr uint64_t kMaxHeaderBytes = 100000000;

// A file opened for positioned reads (closed on destruction).  Tensors are
// read with pread straight into the image: one kernel copy per tensor, no
// page faults on a mapping.
struct InputFile {
  int fd = -1;
  uint64_t size = 0;
  explicit InputFile(const char* path) {
    fd = open(path, O_RDONLY | O_CLOEXEC);
    struct stat st;
    if (fd >= 0 && (fstat(fd, &st) != 0 || st.st_size <= 8)) {
      close(fd);
      fd = -1;
    }
    if (fd >= 0) size = (uint64_t)st.st_size;
  }
  ~InputFile() {
    if (fd >= 0) close(fd);
  }
  InputFile(const InputFile&) = delete;
  InputFile& operator=(const InputFile&) = delete;
  bool read_at(void* dst, size_t n, uint64_t offset) const {
    uint8_t* p = static_cast<uint8_t*>(dst);
    while (n > 0) {
      const ssize_t got = pread(fd, p, n, (off_t)offset);
      if (got <= 0) return false;
      p += got;
      n -= (size_t)got;
      offset += (uint64_t)got;
    }
    return true;
  }
};

inline bool ends_with(const std::string& s, const std::string& suffix) {
  return s.size() >= suffix.size() && memcmp(s.data() + s.size() - suffix.size(), suffix.data(), suffix.size()) == 0;
}

inline int64_t align256(int64_t n) { return (n + 255) / 256 * 256; }

inline bool is_int(double d) { return d >= 0 && d == (double)(int64_t)d && d < 9.0e15; }

}  // namespace peft
}  // namespace plora

extern "C" int plora_peft_pack(const char* path, const char* const* modules, int32_t num_modules,
                               const char* adapter_name, int32_t dtype, double lora_alpha, void* image,
                               size_t capacity, size_t* image_bytes, int64_t* dims) {
  using namespace plora::peft;
  if (!path || !modules || num_modules < 1 || !adapter_name || !image_bytes || !dims)
    return PLORA_ERR_INVALID_ARGUMENT;
  const char* code = dtype == PLORA_DTYPE_BF16 ? "BF16" : dtype == PLORA_DTYPE_F16 ? "F16"
                     : dtype == PLORA_DTYPE_F32 ? "F32" : nullptr;
  if (!code) return PLORA_ERR_INVALID_ARGUMENT;
  const int64_t esize = dtype == PLORA_DTYPE_F32 ? 4 : 2;
  InputFile file(path);
  if (file.fd < 0) return PLORA_ERR_INVALID_ARGUMENT;
  uint8_t head[8];
  if (!file.read_at(head, 8, 0)) return PLORA_ERR_INVALID_ARGUMENT;
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | head[i];
  if (hlen > file.size - 8 || hlen > kMaxHeaderBytes) return PLORA_ERR_UNSUPPORTED;
  std::string header((size_t)hlen, '\0');
  if (!file.read_at(&header[0], (size_t)hlen, 8)) return PLORA_ERR_INVALID_ARGUMENT;
  JVal root;
  if (!JParser(header.data(), header.size()).parse(root) || root.kind != JVal::kObj) return PLORA_ERR_UNSUPPORTED;
  const uint64_t data_start = 8 + hlen;
  const int64_t data_len = (int64_t)(file.size - data_start);

  std::vector<TensorInfo> tensors;
  tensors.reserve(root.obj.size());
  std::unordered_set<std::string> seen;
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") {  // a map of strings, or the format's loader refuses the file
      if (kv.second.kind != JVal::kObj) return PLORA_ERR_UNSUPPORTED;
      for (auto& m : kv.second.obj)
        if (m.second.kind != JVal::kStr) return PLORA_ERR_UNSUPPORTED;
      continue;
    }
    if (!seen.insert(kv.first).second) return PLORA_ERR_UNSUPPORTED;  // duplicate names
    const JVal& t = kv.second;
    if (t.kind != JVal::kObj) return PLORA_ERR_UNSUPPORTED;
    TensorInfo info;
    info.name = kv.first;
    for (auto& f : t.obj) {
      if (f.first == "dtype" && f.second.kind == JVal::kStr) {
        info.dtype = f.second.str;
      } else if (f.first == "shape" && f.second.kind == JVal::kArr) {
        info.has_shape = true;
        for (auto& d : f.second.arr) {
          if (d.kind != JVal::kNum || !d.int_lit || !is_int(d.num)) return PLORA_ERR_UNSUPPORTED;
          info.shape.push_back((int64_t)d.num);
        }
      } else if (f.first == "data_offsets" && f.second.kind == JVal::kArr && f.second.arr.size() == 2) {
        if (f.second.arr[0].kind != JVal::kNum || f.second.arr[1].kind != JVal::kNum ||
            !f.second.arr[0].int_lit || !f.second.arr[1].int_lit || !is_int(f.second.arr[0].num) ||
            !is_int(f.second.arr[1].num))
          return PLORA_ERR_UNSUPPORTED;
        info.begin = (int64_t)f.second.arr[0].num;
        info.end = (int64_t)f.second.arr[1].num;
      }
    }
    tensors.push_back(std::move(info));
  }
  // The checks the safetensors loader makes on every tensor, which the Python
  // path runs and raises on: a known dtype, a shape whose bytes are the
  // tensor's, and data blocks that tile the data section from 0 to its end.
  // Files failing them, and files with empty tensors, are left to that path.
  for (auto& t : tensors) {
    const int64_t esz = dtype_bytes(t.dtype);
    if (esz == 0 || !t.has_shape || t.begin < 0 || t.end <= t.begin) return PLORA_ERR_UNSUPPORTED;
    int64_t n = 1;
    for (int64_t d : t.shape) {
      if (d <= 0 || d > INT32_MAX || n > (INT64_MAX / esz) / d) return PLORA_ERR_UNSUPPORTED;
      n *= d;
    }
    if (n * esz != t.end - t.begin) return PLORA_ERR_UNSUPPORTED;
  }
  // data-offset order: the order safetensors' load_file returns the keys in,
  // which decides the reference's first matching key
  std::sort(tensors.begin(), tensors.end(),
            [](const TensorInfo& a, const TensorInfo& b) { return a.begin < b.begin; });
  int64_t expect = 0;
  for (auto& t : tensors) {
    if (t.begin != expect) return PLORA_ERR_UNSUPPORTED;
    expect = t.end;
  }
  if (expect != data_len) return PLORA_ERR_UNSUPPORTED;

  std::vector<std::string> names(modules, modules + num_modules);
  const std::unordered_set<std::string_view> wanted(names.begin(), names.end());
  // every LoRA key must belong to a configured module (else: the Python loader raises)
  static const char* kMarkers[] = {".lora_A.", ".lora_B.", ".lora_A.weight", ".lora_B.weight"};
  for (auto& t : tensors) {
    for (const char* marker : kMarkers) {
      const size_t pos = t.name.find(marker);
      if (pos == std::string::npos) continue;
      const std::string mod = t.name.substr(0, pos);
      bool inside = false;
      for (auto& a : names)
        if (mod == a || ends_with(mod, "." + a)) {
          inside = true;
          break;
        }
      if (!inside) return PLORA_ERR_UNSUPPORTED;
      break;
    }
  }
  // (module, side) -> first tensor, in data-offset order, whose prefix ends with the module name
  const std::string name(adapter_name);
  std::map<std::pair<std::string, int>, int> index;
  for (int k = 0; k < (int)tensors.size(); ++k) {
    const std::string& key = tensors[k].name;
    for (int side = 0; side < 2; ++side) {
      const std::string s = side == 0 ? "lora_A" : "lora_B";
      const std::string sfx1 = "." + s + "." + name + ".weight", sfx2 = "." + s + ".weight";
      size_t plen;
      if (ends_with(key, sfx1)) plen = key.size() - sfx1.size();
      else if (ends_with(key, sfx2)) plen = key.size() - sfx2.size();
      else continue;
      const std::string_view prefix(key.data(), plen);
      for (size_t i = 0; i < plen; ++i) {
        const std::string_view tail = prefix.substr(i);
        if (wanted.count(tail)) index.emplace(std::make_pair(std::string(tail), side), k);
      }
    }
  }
  // check what the packing uses, lay out the image
  auto usable = [&](const TensorInfo& t) {
    if (t.dtype != code || t.shape.size() != 2) return false;
    // dims below 2^31, so that their product cannot overflow (the header is untrusted input)
    if (t.shape[0] < 0 || t.shape[1] < 0 || t.shape[0] > INT32_MAX || t.shape[1] > INT32_MAX) return false;
    if (t.begin < 0 || t.end < t.begin || t.end > data_len) return false;
    const int64_t n = t.shape[0] * t.shape[1];
    return n <= (t.end - t.begin) / esize && n * esize == t.end - t.begin;
  };
  int64_t offset = align256((int64_t)num_modules * (int64_t)sizeof(plora_slot_record));
  std::vector<plora_slot_record> recs((size_t)num_modules);
  std::vector<std::pair<int, int64_t>> places;  // (tensor, image offset)
  for (int i = 0; i < num_modules; ++i) {
    auto ia = index.find(std::make_pair(names[i], 0));
    auto ib = index.find(std::make_pair(names[i], 1));
    memset(&recs[i], 0, sizeof(plora_slot_record));
    dims[3 * i] = dims[3 * i + 1] = dims[3 * i + 2] = 0;
    if (ia == index.end() && ib == index.end()) continue;  // absent: rank 0
    if (ia == index.end() || ib == index.end()) return PLORA_ERR_UNSUPPORTED;
    const TensorInfo& A = tensors[ia->second];
    const TensorInfo& B = tensors[ib->second];
    if (!usable(A) || !usable(B)) return PLORA_ERR_UNSUPPORTED;
    const int64_t rank = A.shape[0];
    if (rank <= 0 || B.shape[1] != rank) return PLORA_ERR_UNSUPPORTED;
    recs[i].a_offset = offset;
    places.emplace_back(ia->second, offset);
    offset = align256(offset + A.shape[0] * A.shape[1] * esize);
    recs[i].b_offset = offset;
    places.emplace_back(ib->second, offset);
    offset = align256(offset + B.shape[0] * B.shape[1] * esize);
    recs[i].rank = (int32_t)rank;
    recs[i].scale = (float)(lora_alpha / (double)rank);
    dims[3 * i] = rank;
    dims[3 * i + 1] = A.shape[1];  // in_features
    dims[3 * i + 2] = B.shape[0];  // out_features
  }
  *image_bytes = (size_t)offset;
  if (!image || (size_t)offset > capacity) return PLORA_ERR_WORKSPACE;
  uint8_t* out = static_cast<uint8_t*>(image);
  const int64_t head_bytes = (int64_t)(recs.size() * sizeof(plora_slot_record));
  memcpy(out, recs.data(), (size_t)head_bytes);
  int64_t filled = head_bytes;  // zero each gap before the next block, then read the block
  for (auto& pl : places) {
    const TensorInfo& t = tensors[pl.first];
    memset(out + filled, 0, (size_t)(pl.second - filled));
    if (!file.read_at(out + pl.second, (size_t)(t.end - t.begin), data_start + (uint64_t)t.begin))
      return PLORA_ERR_INVALID_ARGUMENT;
    filled = pl.second + (t.end - t.begin);
  }
  memset(out + filled, 0, (size_t)(offset - filled));
  return PLORA_OK;
}
