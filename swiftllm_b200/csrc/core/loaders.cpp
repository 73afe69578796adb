#include "loaders.h"

#include <fcntl.h>
#include <pybind11/numpy.h>
#include <pybind11/stl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace swift {

// ------------------------------------------------------------------ mapping
struct Mapping {
  void* base = nullptr;
  size_t size = 0;
  explicit Mapping(const std::string& path) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("cannot open " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) {
      ::close(fd);
      throw std::runtime_error("cannot stat " + path);
    }
    size = static_cast<size_t>(st.st_size);
    if (size) {
      base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
      if (base == MAP_FAILED) {
        ::close(fd);
        throw std::runtime_error("mmap failed for " + path);
      }
    }
    ::close(fd);
  }
  ~Mapping() {
    if (base && size) munmap(base, size);
  }
  const uint8_t* data() const { return static_cast<const uint8_t*>(base); }
};

// ------------------------------------------------------------- tiny JSON
// Only what the safetensors header needs: objects, arrays, strings, numbers.
struct JVal {
  enum Kind { NUL, NUM, STR, ARR, OBJ, BOOL } kind = NUL;
  double num = 0;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

class JParser {
 public:
  JParser(const char* s, size_t n) : s_(s), n_(n) {}
  JVal parse() {
    JVal v = value();
    return v;
  }

 private:
  void ws() {
    while (i_ < n_ && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\t' || s_[i_] == '\r')) ++i_;
  }
  char peek() {
    ws();
    if (i_ >= n_) throw std::runtime_error("truncated JSON header");
    return s_[i_];
  }
  void expect(char c) {
    if (peek() != c) throw std::runtime_error(std::string("bad JSON header: expected ") + c);
    ++i_;
  }
  std::string string() {
    expect('"');
    std::string out;
    while (i_ < n_ && s_[i_] != '"') {
      if (s_[i_] == '\\' && i_ + 1 < n_) {
        char e = s_[++i_];
        if (e == 'n') out += '\n';
        else if (e == 't') out += '\t';
        else if (e == 'u' && i_ + 4 < n_) {  // keep ASCII range only
          unsigned cp = std::stoul(std::string(s_ + i_ + 1, 4), nullptr, 16);
          out += cp < 128 ? static_cast<char>(cp) : '?';
          i_ += 4;
        } else out += e;
        ++i_;
      } else {
        out += s_[i_++];
      }
    }
    ++i_;
    return out;
  }
  JVal value() {
    char c = peek();
    JVal v;
    if (c == '{') {
      v.kind = JVal::OBJ;
      ++i_;
      if (peek() == '}') { ++i_; return v; }
      for (;;) {
        std::string k = string();
        expect(':');
        v.obj.emplace_back(k, value());
        char d = peek();
        ++i_;
        if (d == '}') break;
        if (d != ',') throw std::runtime_error("bad JSON object");
      }
    } else if (c == '[') {
      v.kind = JVal::ARR;
      ++i_;
      if (peek() == ']') { ++i_; return v; }
      for (;;) {
        v.arr.push_back(value());
        char d = peek();
        ++i_;
        if (d == ']') break;
        if (d != ',') throw std::runtime_error("bad JSON array");
      }
    } else if (c == '"') {
      v.kind = JVal::STR;
      v.str = string();
    } else if (c == 't' || c == 'f') {
      v.kind = JVal::BOOL;
      v.num = c == 't';
      i_ += c == 't' ? 4 : 5;
    } else if (c == 'n') {
      i_ += 4;
    } else {
      v.kind = JVal::NUM;
      size_t j = i_;
      while (j < n_ && (isdigit(s_[j]) || s_[j] == '-' || s_[j] == '+' || s_[j] == '.' ||
                        s_[j] == 'e' || s_[j] == 'E'))
        ++j;
      v.num = std::stod(std::string(s_ + i_, j - i_));
      i_ = j;
    }
    return v;
  }
  const char* s_;
  size_t n_;
  size_t i_ = 0;
};

// ---------------------------------------------------------- safetensors
struct StInfo {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin, end;
};

class SafeTensorsFile {
 public:
  explicit SafeTensorsFile(const std::string& path) : path_(path), map_(std::make_shared<Mapping>(path)) {
    if (map_->size < 8) throw std::runtime_error(path + ": not a safetensors file");
    uint64_t hlen;
    std::memcpy(&hlen, map_->data(), 8);
    if (hlen + 8 > map_->size) throw std::runtime_error(path + ": header length out of range");
    data_off_ = 8 + hlen;
    JParser p(reinterpret_cast<const char*>(map_->data() + 8), hlen);
    JVal root = p.parse();
    for (auto& kv : root.obj) {
      if (kv.first == "__metadata__") {
        for (auto& m : kv.second.obj)
          if (m.second.kind == JVal::STR) meta_[m.first] = m.second.str;
        continue;
      }
      StInfo t;
      const JVal* dt = kv.second.get("dtype");
      const JVal* sh = kv.second.get("shape");
      const JVal* off = kv.second.get("data_offsets");
      if (!dt || !sh || !off || off->arr.size() != 2)
        throw std::runtime_error(path + ": malformed entry " + kv.first);
      t.dtype = dt->str;
      for (auto& d : sh->arr) t.shape.push_back(static_cast<int64_t>(d.num));
      t.begin = static_cast<uint64_t>(off->arr[0].num);
      t.end = static_cast<uint64_t>(off->arr[1].num);
      if (data_off_ + t.end > map_->size || t.begin > t.end)
        throw std::runtime_error(path + ": tensor " + kv.first + " out of range");
      order_.push_back(kv.first);
      infos_[kv.first] = t;
    }
  }
  std::vector<std::string> keys() const { return order_; }
  std::map<std::string, std::string> metadata() const { return meta_; }
  const StInfo& info(const std::string& k) const {
    auto it = infos_.find(k);
    if (it == infos_.end()) throw py::key_error(k);
    return it->second;
  }
  // Raw bytes as a uint8 numpy view that keeps the mapping alive.
  py::array raw(const std::string& k) const {
    const StInfo& t = info(k);
    auto holder = new std::shared_ptr<Mapping>(map_);
    py::capsule cap(holder, [](void* p) { delete static_cast<std::shared_ptr<Mapping>*>(p); });
    return py::array(py::dtype("uint8"), {static_cast<py::ssize_t>(t.end - t.begin)}, {1},
                     map_->data() + data_off_ + t.begin, cap);
  }

 private:
  std::string path_;
  std::shared_ptr<Mapping> map_;
  uint64_t data_off_ = 0;
  std::vector<std::string> order_;
  std::map<std::string, StInfo> infos_;
  std::map<std::string, std::string> meta_;
};

// ----------------------------------------------------------------- GGUF
enum GgmlType : uint32_t {
  G_F32 = 0, G_F16 = 1, G_Q4_0 = 2, G_Q4_1 = 3, G_Q5_0 = 6, G_Q5_1 = 7, G_Q8_0 = 8,
  G_Q8_1 = 9, G_Q2_K = 10, G_Q3_K = 11, G_Q4_K = 12, G_Q5_K = 13, G_Q6_K = 14, G_Q8_K = 15,
  G_I8 = 24, G_I16 = 25, G_I32 = 26, G_I64 = 27, G_F64 = 28, G_BF16 = 30,
};

static void type_geom(uint32_t t, int* block, int* bytes) {
  switch (t) {
    case G_F32: *block = 1; *bytes = 4; return;
    case G_F16: case G_BF16: *block = 1; *bytes = 2; return;
    case G_Q4_0: *block = 32; *bytes = 18; return;
    case G_Q4_1: *block = 32; *bytes = 20; return;
    case G_Q5_0: *block = 32; *bytes = 22; return;
    case G_Q5_1: *block = 32; *bytes = 24; return;
    case G_Q8_0: *block = 32; *bytes = 34; return;
    case G_Q8_1: *block = 32; *bytes = 36; return;
    case G_Q2_K: *block = 256; *bytes = 84; return;
    case G_Q3_K: *block = 256; *bytes = 110; return;
    case G_Q4_K: *block = 256; *bytes = 144; return;
    case G_Q5_K: *block = 256; *bytes = 176; return;
    case G_Q6_K: *block = 256; *bytes = 210; return;
    case G_Q8_K: *block = 256; *bytes = 292; return;
    case G_I8: *block = 1; *bytes = 1; return;
    case G_I16: *block = 1; *bytes = 2; return;
    case G_I32: *block = 1; *bytes = 4; return;
    case G_I64: case G_F64: *block = 1; *bytes = 8; return;
  }
  throw std::runtime_error("unsupported GGUF tensor type " + std::to_string(t));
}

static float half_to_float(uint16_t h) {
  uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
  float v;
  if (exp == 0) v = std::ldexp(static_cast<float>(man), -24);
  else if (exp == 31) v = man ? NAN : INFINITY;
  else v = std::ldexp(static_cast<float>(man | 0x400), static_cast<int>(exp) - 25);
  return sign ? -v : v;
}
static float bf16_to_float(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t rd16(const uint8_t* p) { uint16_t v; std::memcpy(&v, p, 2); return v; }

// Dequantise `n` elements of type `t` from `src` to fp32.
void dequantize(uint32_t t, const uint8_t* src, int64_t n, float* dst) {
  int blk, bytes;
  type_geom(t, &blk, &bytes);
  if (n % blk) throw std::runtime_error("element count not a multiple of the block size");
  int64_t nb = n / blk;
  switch (t) {
    case G_F32: std::memcpy(dst, src, n * 4); return;
    case G_F16: for (int64_t i = 0; i < n; ++i) dst[i] = half_to_float(rd16(src + 2 * i)); return;
    case G_BF16: for (int64_t i = 0; i < n; ++i) dst[i] = bf16_to_float(rd16(src + 2 * i)); return;
    case G_Q4_0:
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* p = src + b * 18;
        float d = half_to_float(rd16(p));
        for (int j = 0; j < 16; ++j) {
          dst[b * 32 + j] = (static_cast<int>(p[2 + j] & 0xF) - 8) * d;
          dst[b * 32 + j + 16] = (static_cast<int>(p[2 + j] >> 4) - 8) * d;
        }
      }
      return;
    case G_Q4_1:
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* p = src + b * 20;
        float d = half_to_float(rd16(p)), mn = half_to_float(rd16(p + 2));
        for (int j = 0; j < 16; ++j) {
          dst[b * 32 + j] = (p[4 + j] & 0xF) * d + mn;
          dst[b * 32 + j + 16] = (p[4 + j] >> 4) * d + mn;
        }
      }
      return;
    case G_Q8_0:
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* p = src + b * 34;
        float d = half_to_float(rd16(p));
        for (int j = 0; j < 32; ++j) dst[b * 32 + j] = static_cast<int8_t>(p[2 + j]) * d;
      }
      return;
    case G_Q4_K:
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* p = src + b * 144;
        float d = half_to_float(rd16(p)), dmin = half_to_float(rd16(p + 2));
        const uint8_t* sc = p + 4;
        const uint8_t* q = p + 16;
        float* y = dst + b * 256;
        auto scale_min = [&](int j, uint8_t* s, uint8_t* m) {
          if (j < 4) {
            *s = sc[j] & 63;
            *m = sc[j + 4] & 63;
          } else {
            *s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
            *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
          }
        };
        for (int c = 0, is = 0; c < 4; ++c, is += 2) {
          uint8_t s1, m1, s2, m2;
          scale_min(is, &s1, &m1);
          scale_min(is + 1, &s2, &m2);
          for (int l = 0; l < 32; ++l) y[c * 64 + l] = d * s1 * (q[c * 32 + l] & 0xF) - dmin * m1;
          for (int l = 0; l < 32; ++l) y[c * 64 + 32 + l] = d * s2 * (q[c * 32 + l] >> 4) - dmin * m2;
        }
      }
      return;
    case G_Q6_K:
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* p = src + b * 210;
        const uint8_t* ql = p;
        const uint8_t* qh = p + 128;
        const int8_t* sc = reinterpret_cast<const int8_t*>(p + 192);
        float d = half_to_float(rd16(p + 208));
        float* y = dst + b * 256;
        for (int half = 0; half < 2; ++half) {
          for (int l = 0; l < 32; ++l) {
            int is = l / 16;
            int q1 = static_cast<int>((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
            int q2 = static_cast<int>((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = static_cast<int>((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = static_cast<int>((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            y[l] = d * sc[is] * q1;
            y[l + 32] = d * sc[is + 2] * q2;
            y[l + 64] = d * sc[is + 4] * q3;
            y[l + 96] = d * sc[is + 6] * q4;
          }
          y += 128;
          ql += 64;
          qh += 32;
          sc += 8;
        }
      }
      return;
  }
  throw std::runtime_error("no dequantiser for GGUF type " + std::to_string(t));
}

struct GgufTensor {
  std::string name;
  std::vector<int64_t> dims;  // ne[0] innermost
  uint32_t type;
  uint64_t offset;            // relative to data start
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
  uint64_t nbytes() const {
    int blk, bytes;
    type_geom(type, &blk, &bytes);
    return static_cast<uint64_t>(numel() / blk) * bytes;
  }
};

class GgufFile {
 public:
  explicit GgufFile(const std::string& path) : map_(std::make_shared<Mapping>(path)) {
    const uint8_t* p = map_->data();
    size_t n = map_->size;
    size_t off = 0;
    auto need = [&](size_t k) {
      if (off + k > n) throw std::runtime_error(path + ": truncated GGUF");
    };
    auto u32 = [&]() { need(4); uint32_t v; std::memcpy(&v, p + off, 4); off += 4; return v; };
    auto u64 = [&]() { need(8); uint64_t v; std::memcpy(&v, p + off, 8); off += 8; return v; };
    if (u32() != 0x46554747u) throw std::runtime_error(path + ": bad GGUF magic");
    version_ = u32();
    if (version_ < 1 || version_ > 3) throw std::runtime_error("unsupported GGUF version");
    auto count = [&]() -> uint64_t { return version_ == 1 ? u32() : u64(); };
    uint64_t n_tensors = count(), n_kv = count();
    auto str = [&]() {
      uint64_t len = count();
      need(len);
      std::string s(reinterpret_cast<const char*>(p + off), len);
      off += len;
      return s;
    };
    std::function<py::object(uint32_t)> value = [&](uint32_t t) -> py::object {
      switch (t) {
        case 0: { need(1); uint8_t v = p[off]; off += 1; return py::int_(v); }
        case 1: { need(1); int8_t v = static_cast<int8_t>(p[off]); off += 1; return py::int_(v); }
        case 2: { need(2); uint16_t v; std::memcpy(&v, p + off, 2); off += 2; return py::int_(v); }
        case 3: { need(2); int16_t v; std::memcpy(&v, p + off, 2); off += 2; return py::int_(v); }
        case 4: return py::int_(u32());
        case 5: { uint32_t v = u32(); return py::int_(static_cast<int32_t>(v)); }
        case 6: { uint32_t v = u32(); float f; std::memcpy(&f, &v, 4); return py::float_(f); }
        case 7: { need(1); bool v = p[off] != 0; off += 1; return py::bool_(v); }
        case 8: return py::str(str());
        case 9: {
          uint32_t et = u32();
          uint64_t cnt = count();
          py::list l;
          for (uint64_t i = 0; i < cnt; ++i) l.append(value(et));
          return l;
        }
        case 10: return py::int_(u64());
        case 11: { uint64_t v = u64(); return py::int_(static_cast<int64_t>(v)); }
        case 12: { uint64_t v = u64(); double d; std::memcpy(&d, &v, 8); return py::float_(d); }
      }
      throw std::runtime_error("bad GGUF metadata type " + std::to_string(t));
    };
    for (uint64_t i = 0; i < n_kv; ++i) {
      std::string k = str();
      uint32_t t = u32();
      meta_[py::str(k)] = value(t);
    }
    for (uint64_t i = 0; i < n_tensors; ++i) {
      GgufTensor t;
      t.name = str();
      uint32_t nd = u32();
      for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(static_cast<int64_t>(count()));
      t.type = u32();
      t.offset = u64();
      tensors_.push_back(t);
    }
    uint64_t align = 32;
    if (meta_.contains("general.alignment")) align = meta_["general.alignment"].cast<uint64_t>();
    data_off_ = (off + align - 1) / align * align;
    for (auto& t : tensors_) {
      if (data_off_ + t.offset + t.nbytes() > n)
        throw std::runtime_error(path + ": tensor " + t.name + " out of range");
    }
  }
  uint32_t version() const { return version_; }
  py::dict metadata() const { return meta_; }
  py::list tensor_infos() const {
    py::list l;
    for (auto& t : tensors_) {
      py::dict d;
      d["name"] = t.name;
      d["dims"] = t.dims;
      d["type"] = t.type;
      d["offset"] = t.offset;
      d["nbytes"] = t.nbytes();
      l.append(d);
    }
    return l;
  }
  const GgufTensor& find(const std::string& name) const {
    for (auto& t : tensors_)
      if (t.name == name) return t;
    throw py::key_error(name);
  }
  py::array raw(const std::string& name) const {
    const GgufTensor& t = find(name);
    auto holder = new std::shared_ptr<Mapping>(map_);
    py::capsule cap(holder, [](void* q) { delete static_cast<std::shared_ptr<Mapping>*>(q); });
    return py::array(py::dtype("uint8"), {static_cast<py::ssize_t>(t.nbytes())}, {1},
                     map_->data() + data_off_ + t.offset, cap);
  }
  // fp32 array with numpy shape reversed from GGUF dims ([..., ne1, ne0]).
  py::array_t<float> dequant(const std::string& name) const {
    const GgufTensor& t = find(name);
    std::vector<py::ssize_t> shape(t.dims.rbegin(), t.dims.rend());
    py::array_t<float> out(shape);
    const uint8_t* src = map_->data() + data_off_ + t.offset;
    {
      py::gil_scoped_release nogil;
      dequantize(t.type, src, t.numel(), out.mutable_data());
    }
    return out;
  }

 private:
  std::shared_ptr<Mapping> map_;
  uint32_t version_ = 0;
  py::dict meta_;
  std::vector<GgufTensor> tensors_;
  uint64_t data_off_ = 0;
};

}  // namespace swift

void bind_loaders(py::module_& m) {
  using namespace swift;
  py::class_<SafeTensorsFile>(m, "SafeTensorsFile")
      .def(py::init<const std::string&>())
      .def("keys", &SafeTensorsFile::keys)
      .def("metadata", &SafeTensorsFile::metadata)
      .def("dtype", [](const SafeTensorsFile& f, const std::string& k) { return f.info(k).dtype; })
      .def("shape", [](const SafeTensorsFile& f, const std::string& k) { return f.info(k).shape; })
      .def("raw", &SafeTensorsFile::raw);
  py::class_<GgufFile>(m, "GgufFile")
      .def(py::init<const std::string&>())
      .def_property_readonly("version", &GgufFile::version)
      .def("metadata", &GgufFile::metadata)
      .def("tensor_infos", &GgufFile::tensor_infos)
      .def("raw", &GgufFile::raw)
      .def("dequant", &GgufFile::dequant);
  m.def("gguf_dequantize",
        [](uint32_t type, py::array_t<uint8_t, py::array::c_style> src, int64_t n) {
          py::array_t<float> out(n);
          int blk, bytes;
          type_geom(type, &blk, &bytes);
          if (static_cast<int64_t>(src.size()) < n / blk * bytes)
            throw std::invalid_argument("source buffer too small");
          dequantize(type, src.data(), n, out.mutable_data());
          return out;
        });
}
