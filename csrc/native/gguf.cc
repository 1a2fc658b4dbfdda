// GGUF v2/v3 reader (mmap) and CPU dequantisation.
//
// Replaces the reference's own GGUF parser (src/gguf/parser.rs:15-215: magic 0x46554747,
// metadata KV types, tensor infos, alignment 32 by default) and its ggml-quants CPU
// dequantisation (src/quantization/mod.rs:158-255: Q4_0 / Q4_K / Q8_0).  Block layouts are
// the published GGUF/ggml formats; this file also dequantises Q6_K (common for output
// layers of Q4_K_M files), F16 and BF16.  The dequantiser doubles as the oracle for the
// GPU dequant-fused GEMMs.
#include <fcntl.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <torch/extension.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace lbn {

enum GgmlType : uint32_t {
  GGML_F32 = 0, GGML_F16 = 1, GGML_Q4_0 = 2, GGML_Q4_1 = 3, GGML_Q5_0 = 6, GGML_Q5_1 = 7,
  GGML_Q8_0 = 8, GGML_Q8_1 = 9, GGML_Q2_K = 10, GGML_Q3_K = 11, GGML_Q4_K = 12, GGML_Q5_K = 13,
  GGML_Q6_K = 14, GGML_Q8_K = 15, GGML_BF16 = 30,
};

// (elements per block, bytes per block)
static std::pair<int, int> type_geometry(uint32_t t) {
  switch (t) {
    case GGML_F32: return {1, 4};
    case GGML_F16: return {1, 2};
    case GGML_BF16: return {1, 2};
    case GGML_Q4_0: return {32, 18};
    case GGML_Q4_1: return {32, 20};
    case GGML_Q5_0: return {32, 22};
    case GGML_Q5_1: return {32, 24};
    case GGML_Q8_0: return {32, 34};
    case GGML_Q8_1: return {32, 36};
    case GGML_Q2_K: return {256, 84};
    case GGML_Q3_K: return {256, 110};
    case GGML_Q4_K: return {256, 144};
    case GGML_Q5_K: return {256, 176};
    case GGML_Q6_K: return {256, 210};
    case GGML_Q8_K: return {256, 292};
    default: throw std::runtime_error("unknown ggml type " + std::to_string(t));
  }
}

static inline float half_to_float(uint16_t h) {
  const uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1f, mant = h & 0x3ff;
  uint32_t f;
  if (exp == 0) {
    if (mant == 0) {
      f = sign << 31;
    } else {  // subnormal
      int e = -1;
      uint32_t m = mant;
      do {
        e++;
        m <<= 1;
      } while ((m & 0x400) == 0);
      f = (sign << 31) | ((127 - 15 - e) << 23) | ((m & 0x3ff) << 13);
    }
  } else if (exp == 31) {
    f = (sign << 31) | 0x7f800000u | (mant << 13);
  } else {
    f = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float out;
  std::memcpy(&out, &f, 4);
  return out;
}

static inline uint16_t rd16(const uint8_t* p) { uint16_t v; std::memcpy(&v, p, 2); return v; }

// Q4_K / Q5_K packed 6-bit scale and min of sub-block j (0..7) from the 12-byte array.
static inline void scale_min_k4(int j, const uint8_t* q, uint8_t* sc, uint8_t* mn) {
  if (j < 4) {
    *sc = q[j] & 63;
    *mn = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

void dequantize_row(uint32_t type, const uint8_t* src, float* dst, int64_t n) {
  auto geo = type_geometry(type);
  const int64_t nb = n / geo.first;
  switch (type) {
    case GGML_F32: std::memcpy(dst, src, n * 4); return;
    case GGML_F16:
      for (int64_t i = 0; i < n; ++i) dst[i] = half_to_float(rd16(src + 2 * i));
      return;
    case GGML_BF16:
      for (int64_t i = 0; i < n; ++i) {
        uint32_t f = static_cast<uint32_t>(rd16(src + 2 * i)) << 16;
        std::memcpy(&dst[i], &f, 4);
      }
      return;
    case GGML_Q4_0:
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = src + b * 18;
        const float d = half_to_float(rd16(blk));
        const uint8_t* qs = blk + 2;
        float* y = dst + b * 32;
        for (int j = 0; j < 16; ++j) {
          y[j] = d * (static_cast<int>(qs[j] & 0xF) - 8);
          y[j + 16] = d * (static_cast<int>(qs[j] >> 4) - 8);
        }
      }
      return;
    case GGML_Q8_0:
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = src + b * 34;
        const float d = half_to_float(rd16(blk));
        const int8_t* qs = reinterpret_cast<const int8_t*>(blk + 2);
        float* y = dst + b * 32;
        for (int j = 0; j < 32; ++j) y[j] = d * qs[j];
      }
      return;
    case GGML_Q4_K:
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = src + b * 144;
        const float d = half_to_float(rd16(blk));
        const float dmin = half_to_float(rd16(blk + 2));
        const uint8_t* scales = blk + 4;
        const uint8_t* q = blk + 16;
        float* y = dst + b * 256;
        for (int j = 0; j < 4; ++j) {  // pairs of 32-element sub-blocks
          uint8_t sc1, m1, sc2, m2;
          scale_min_k4(2 * j, scales, &sc1, &m1);
          scale_min_k4(2 * j + 1, scales, &sc2, &m2);
          const float d1 = d * sc1, mm1 = dmin * m1, d2 = d * sc2, mm2 = dmin * m2;
          for (int l = 0; l < 32; ++l) y[l] = d1 * (q[l] & 0xF) - mm1;
          for (int l = 0; l < 32; ++l) y[32 + l] = d2 * (q[l] >> 4) - mm2;
          q += 32;
          y += 64;
        }
      }
      return;
    case GGML_Q6_K:
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = src + b * 210;
        const uint8_t* ql = blk;
        const uint8_t* qh = blk + 128;
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
        const float d = half_to_float(rd16(blk + 208));
        float* y = dst + b * 256;
        for (int half = 0; half < 2; ++half) {
          for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q1 = static_cast<int>((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
            const int q2 = static_cast<int>((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = static_cast<int>((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = static_cast<int>((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
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
    default:
      throw std::runtime_error("dequantize: unsupported ggml type " + std::to_string(type));
  }
}

struct TensorInfo {
  std::string name;
  std::vector<int64_t> dims;  // ggml order: dims[0] is the contiguous dimension
  uint32_t type;
  uint64_t offset;  // relative to data section
  int64_t numel;
  int64_t nbytes;
};

class GGUFFile {
 public:
  explicit GGUFFile(const std::string& path) : path_(path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("cannot open " + path);
    struct stat st;
    if (fstat(fd_, &st) != 0) throw std::runtime_error("stat failed");
    size_ = st.st_size;
    if (size_ < 24) throw std::runtime_error("gguf: file too small");
    base_ = static_cast<uint8_t*>(mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0));
    if (base_ == MAP_FAILED) throw std::runtime_error("mmap failed");
    parse();
  }
  ~GGUFFile() {
    if (base_ && base_ != MAP_FAILED) munmap(base_, size_);
    if (fd_ >= 0) ::close(fd_);
  }

  uint32_t version() const { return version_; }
  uint64_t alignment() const { return alignment_; }
  uint64_t data_offset() const { return data_off_; }
  py::dict metadata() const { return meta_; }

  std::vector<py::tuple> tensors() const {
    std::vector<py::tuple> out;
    for (auto& t : infos_)
      out.push_back(py::make_tuple(t.name, t.dims, t.type, t.offset, t.nbytes));
    return out;
  }

  const TensorInfo& info(const std::string& name) const {
    for (auto& t : infos_)
      if (t.name == name) return t;
    throw std::runtime_error("gguf: no tensor " + name);
  }

  torch::Tensor raw(const std::string& name) const {
    const auto& t = info(name);
    auto out = torch::empty({t.nbytes}, torch::kUInt8);
    std::memcpy(out.data_ptr(), base_ + data_off_ + t.offset, t.nbytes);
    return out;
  }

  // Dequantised tensor in torch (row-major) order: shape = reversed ggml dims.
  torch::Tensor dequantize(const std::string& name) const {
    const auto& t = info(name);
    std::vector<int64_t> shape(t.dims.rbegin(), t.dims.rend());
    auto out = torch::empty(shape, torch::kFloat32);
    const int64_t row = t.dims[0];
    const int64_t nrows = t.numel / row;
    auto geo = type_geometry(t.type);
    const int64_t row_bytes = row / geo.first * geo.second;
    const uint8_t* src = base_ + data_off_ + t.offset;
    float* dst = out.data_ptr<float>();
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < nrows; ++r) dequantize_row(t.type, src + r * row_bytes, dst + r * row, row);
    return out;
  }

 private:
  template <typename T>
  T rd() {
    if (pos_ + sizeof(T) > size_) throw std::runtime_error("gguf: truncated file");
    T v;
    std::memcpy(&v, base_ + pos_, sizeof(T));
    pos_ += sizeof(T);
    return v;
  }
  std::string rd_str() {
    const uint64_t n = rd<uint64_t>();
    if (n > (1ull << 30) || pos_ + n > size_) throw std::runtime_error("gguf: bad string length");
    std::string s(reinterpret_cast<const char*>(base_ + pos_), n);
    pos_ += n;
    return s;
  }
  py::object rd_value(uint32_t type, int depth = 0) {
    if (depth > 4) throw std::runtime_error("gguf: nested arrays too deep");
    switch (type) {
      case 0: return py::int_(rd<uint8_t>());
      case 1: return py::int_(rd<int8_t>());
      case 2: return py::int_(rd<uint16_t>());
      case 3: return py::int_(rd<int16_t>());
      case 4: return py::int_(rd<uint32_t>());
      case 5: return py::int_(rd<int32_t>());
      case 6: return py::float_(rd<float>());
      case 7: return py::bool_(rd<uint8_t>() != 0);
      case 8: return py::str(rd_str());
      case 9: {
        const uint32_t et = rd<uint32_t>();
        const uint64_t n = rd<uint64_t>();
        if (n > (1ull << 28)) throw std::runtime_error("gguf: array too long");
        py::list l;
        for (uint64_t i = 0; i < n; ++i) l.append(rd_value(et, depth + 1));
        return l;
      }
      case 10: return py::int_(rd<uint64_t>());
      case 11: return py::int_(rd<int64_t>());
      case 12: return py::float_(rd<double>());
      default: throw std::runtime_error("gguf: bad metadata type " + std::to_string(type));
    }
  }

  void parse() {
    const uint32_t magic = rd<uint32_t>();
    if (magic != 0x46554747u) throw std::runtime_error("gguf: bad magic");
    version_ = rd<uint32_t>();
    if (version_ < 2 || version_ > 3) throw std::runtime_error("gguf: unsupported version");
    const uint64_t n_tensors = rd<uint64_t>();
    const uint64_t n_kv = rd<uint64_t>();
    if (n_tensors > (1u << 24) || n_kv > (1u << 24)) throw std::runtime_error("gguf: bad counts");
    for (uint64_t i = 0; i < n_kv; ++i) {
      std::string key = rd_str();
      const uint32_t t = rd<uint32_t>();
      meta_[py::str(key)] = rd_value(t);
      if (key == "general.alignment") alignment_ = py::cast<uint64_t>(meta_[py::str(key)]);
    }
    if (alignment_ == 0 || (alignment_ & (alignment_ - 1)))
      throw std::runtime_error("gguf: alignment must be a power of two");
    for (uint64_t i = 0; i < n_tensors; ++i) {
      TensorInfo ti;
      ti.name = rd_str();
      const uint32_t nd = rd<uint32_t>();
      if (nd > 4) throw std::runtime_error("gguf: too many dims");
      ti.numel = 1;
      for (uint32_t d = 0; d < nd; ++d) {
        ti.dims.push_back(static_cast<int64_t>(rd<uint64_t>()));
        ti.numel *= ti.dims.back();
      }
      ti.type = rd<uint32_t>();
      ti.offset = rd<uint64_t>();
      auto geo = type_geometry(ti.type);
      if (ti.dims.empty() || ti.dims[0] % geo.first) throw std::runtime_error("gguf: bad row size");
      ti.nbytes = ti.numel / geo.first * geo.second;
      infos_.push_back(ti);
    }
    data_off_ = (pos_ + alignment_ - 1) / alignment_ * alignment_;
    for (auto& t : infos_) {
      if (t.offset % alignment_ != 0) throw std::runtime_error("gguf: unaligned tensor " + t.name);
      if (data_off_ + t.offset + t.nbytes > size_)
        throw std::runtime_error("gguf: tensor out of file bounds: " + t.name);
    }
  }

  std::string path_;
  int fd_ = -1;
  uint8_t* base_ = nullptr;
  size_t size_ = 0, pos_ = 0;
  uint32_t version_ = 0;
  uint64_t alignment_ = 32, data_off_ = 0;
  py::dict meta_;
  std::vector<TensorInfo> infos_;
};

torch::Tensor dequantize_buffer(uint32_t type, torch::Tensor raw, int64_t numel) {
  TORCH_CHECK(raw.scalar_type() == torch::kUInt8 && raw.is_contiguous(), "raw bytes");
  auto geo = type_geometry(type);
  TORCH_CHECK(numel % geo.first == 0, "numel not a multiple of the block");
  TORCH_CHECK(raw.numel() >= numel / geo.first * geo.second, "raw buffer too small");
  auto out = torch::empty({numel}, torch::kFloat32);
  dequantize_row(type, raw.data_ptr<uint8_t>(), out.data_ptr<float>(), numel);
  return out;
}

}  // namespace lbn

void register_gguf(py::module_& m) {
  using lbn::GGUFFile;
  py::class_<GGUFFile>(m, "GGUFFile")
      .def(py::init<const std::string&>())
      .def_property_readonly("version", &GGUFFile::version)
      .def_property_readonly("alignment", &GGUFFile::alignment)
      .def_property_readonly("data_offset", &GGUFFile::data_offset)
      .def("metadata", &GGUFFile::metadata)
      .def("tensors", &GGUFFile::tensors)
      .def("raw", &GGUFFile::raw)
      .def("dequantize", &GGUFFile::dequantize);
  m.def("dequantize", &lbn::dequantize_buffer, "dequantize a raw ggml buffer to f32");
  m.def("ggml_type_geometry", &lbn::type_geometry);
}
