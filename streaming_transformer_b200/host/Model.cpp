// Model.cpp -- checkpoint loader of the Stream API (include/Model.hpp).
//
// The checkpoint format and its acceptance rules are the reference's
// (reference src/runtime/Model.cpp:15-145), so its checkpoints and fixtures
// load unchanged: manifest version 1, little endian, out_in orientation,
// whole-file and per-tensor SHA-256, tensors contiguous in manifest order,
// exact shapes, storage widened to float; bf16 tensors ("bfloat16", mode
// "bf16") are accepted in addition to float32 / float16. The error messages
// are the reference's too, since callers match on them.
//
// The loader itself is organised differently: tensors.bin is mapped read
// only, the manifest is turned into a table of tensor descriptors that is
// validated in one pass before any tensor is decoded, hashing goes through
// OpenSSL's EVP interface, and the shape contract is a table of (name,
// dimension expressions) rows.
#include "Model.hpp"

#include <bit>
#include <cmath>
#include <cstring>
#include <fstream>
#include <stdexcept>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <openssl/evp.h>

namespace Stream {

namespace {

[[noreturn]] void reject(const std::string& message) { throw std::runtime_error(message); }

// A read-only view of a whole file, unmapped (and closed) on scope exit.
class MappedFile {
 public:
  explicit MappedFile(const std::filesystem::path& path) {
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    struct stat st {};
    if (fd_ < 0 || ::fstat(fd_, &st) != 0) {
      if (fd_ >= 0) ::close(fd_);
      reject("Cannot read " + path.string());
    }
    size_ = static_cast<std::size_t>(st.st_size);
    if (size_ > 0) {
      void* p = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
      if (p == MAP_FAILED) {
        ::close(fd_);
        reject("Cannot read " + path.string());
      }
      data_ = static_cast<const unsigned char*>(p);
    }
  }
  ~MappedFile() {
    if (data_) ::munmap(const_cast<unsigned char*>(data_), size_);
    if (fd_ >= 0) ::close(fd_);
  }
  MappedFile(const MappedFile&) = delete;
  MappedFile& operator=(const MappedFile&) = delete;
  const unsigned char* data() const { return data_; }
  std::size_t size() const { return size_; }

 private:
  int fd_ = -1;
  const unsigned char* data_ = nullptr;
  std::size_t size_ = 0;
};

// One manifest entry, as read, before validation.
struct TensorDesc {
  std::string name, dtype, digest;
  std::vector<int> shape;
  std::size_t offset = 0, nbytes = 0;
  std::size_t elements = 0, width = 0;  // filled by validation
};

std::size_t dtype_width(const std::string& dtype) {
  if (dtype == "float32") return 4;
  if (dtype == "float16" || dtype == "bfloat16") return 2;
  return 0;
}

// The descriptor table: every bound, size and order rule checked before any
// tensor is decoded.
std::vector<TensorDesc> describe(const Json& entries, std::size_t file_bytes) {
  std::vector<TensorDesc> table;
  std::size_t next = 0;
  for (const auto& item : entries) {
    TensorDesc t;
    t.name = item.at("name").get<std::string>();
    t.dtype = item.at("dtype").get<std::string>();
    t.digest = item.at("sha256").get<std::string>();
    t.shape = item.at("shape").get<std::vector<int>>();
    t.offset = item.at("offset").get<std::size_t>();
    t.nbytes = item.at("nbytes").get<std::size_t>();
    t.elements = 1;
    for (const int dim : t.shape) {
      // a product that could exceed the file is invalid before it overflows
      if (dim <= 0 || t.elements > file_bytes / static_cast<std::size_t>(dim)) reject("Invalid tensor dimensions");
      t.elements *= static_cast<std::size_t>(dim);
    }
    t.width = dtype_width(t.dtype);
    const bool inside = t.offset <= file_bytes && t.nbytes <= file_bytes - t.offset;
    if (t.width == 0 || t.offset != next || t.nbytes != t.elements * t.width || !inside)
      reject("Invalid tensor bounds");
    next = t.offset + t.nbytes;
    table.push_back(std::move(t));
  }
  if (next != file_bytes) reject("Trailing tensor bytes");
  return table;
}

float binary16_to_float(std::uint16_t h) {
  const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16;
  const std::uint32_t exponent = (h >> 10) & 0x1fu, mantissa = h & 0x3ffu;
  if (exponent == 0) {  // zero or subnormal: mantissa * 2^-24
    const float magnitude = std::ldexp(static_cast<float>(mantissa), -24);
    return std::bit_cast<float>(std::bit_cast<std::uint32_t>(magnitude) | sign);
  }
  const std::uint32_t bits = exponent == 31 ? (sign | 0x7f800000u | (mantissa << 13))
                                            : (sign | ((exponent + 112u) << 23) | (mantissa << 13));
  return std::bit_cast<float>(bits);
}

// Decode one validated tensor into floats.
void widen(const TensorDesc& t, const unsigned char* src, std::vector<float>& out) {
  out.resize(t.elements);
  if (t.width == 4) {
    std::memcpy(out.data(), src, t.nbytes);
    return;
  }
  const bool brain = t.dtype == "bfloat16";
  for (std::size_t i = 0; i < t.elements; ++i) {
    std::uint16_t bits;
    std::memcpy(&bits, src + 2 * i, 2);
    out[i] = brain ? std::bit_cast<float>(static_cast<std::uint32_t>(bits) << 16) : binary16_to_float(bits);
  }
}

Json load_manifest(const std::filesystem::path& path) {
  std::ifstream in(path);
  if (!in) reject("Cannot read " + path.string());
  Json manifest;
  in >> manifest;
  return manifest;
}

}  // namespace

ModelConfig ModelConfig::fromJson(const Json& j) {
  ModelConfig c{j.at("layers").get<int>(), j.at("width").get<int>(), j.at("heads").get<int>(),
                j.at("ffn").get<int>(), j.at("window").get<int>(), j.at("features").get<int>(),
                j.at("epsilon").get<float>()};
  c.validate();
  return c;
}

// The reference's dimension limits (reference src/runtime/Model.cpp:22-29).
void ModelConfig::validate() const {
  const bool ok = layers >= 1 && layers <= 16 && width >= 1 && width <= 1024 && heads >= 1 && width % heads == 0 &&
                  (width / heads) % 2 == 0 && ffn >= 1 && ffn <= 4096 && window >= 1 && window <= 4096 &&
                  features >= 1 && features <= 1024 && std::isfinite(epsilon) && epsilon > 0;
  if (!ok) reject("Invalid or unsupported model dimensions");
}

std::size_t ModelConfig::cacheElements() const {
  return static_cast<std::size_t>(layers) * static_cast<std::size_t>(width) * static_cast<std::size_t>(window);
}

std::vector<char> readBytes(const std::filesystem::path& path) {
  const MappedFile file(path);
  const char* begin = reinterpret_cast<const char*>(file.data());
  return std::vector<char>(begin, begin + file.size());
}

std::string sha256(const void* data, std::size_t bytes) {
  unsigned char digest[EVP_MAX_MD_SIZE];
  unsigned int length = 0;
  if (EVP_Digest(data, bytes, digest, &length, EVP_sha256(), nullptr) != 1) reject("SHA-256 failed");
  static const char kHex[] = "0123456789abcdef";
  std::string text(2 * length, '0');
  for (unsigned int i = 0; i < length; ++i) {
    text[2 * i] = kHex[digest[i] >> 4];
    text[2 * i + 1] = kHex[digest[i] & 15];
  }
  return text;
}

// IEEE-754 binary16 round-to-nearest-even, widened back to float.
float roundHalf(float value) {
  const std::uint32_t bits = std::bit_cast<std::uint32_t>(value);
  const std::uint32_t sign = bits & 0x80000000u, magnitude = bits & 0x7fffffffu;
  if (magnitude >= 0x7f800000u) return value;                                     // inf, nan
  if (magnitude >= 0x477ff000u) return std::bit_cast<float>(sign | 0x7f800000u);  // rounds past 65504
  if (magnitude < 0x38800000u) {  // binary16 subnormal range: a multiple of 2^-24
    const float q = std::ldexp(std::nearbyint(std::ldexp(std::fabs(value), 24)), -24);
    return std::bit_cast<float>(std::bit_cast<std::uint32_t>(q) | sign);
  }
  // keep 10 mantissa bits, ties to even
  const std::uint32_t kept = (magnitude + 0x0fffu + ((magnitude >> 13) & 1u)) & ~0x1fffu;
  return std::bit_cast<float>(sign | kept);
}

Model::Model(const std::filesystem::path& path) {
  manifest = load_manifest(path / "manifest.json");
  const bool format_ok = manifest.at("version").get<int>() == 1 &&
                         manifest.at("byte_order").get<std::string>() == "little" &&
                         manifest.at("orientation").get<std::string>() == "out_in" &&
                         std::endian::native == std::endian::little;
  if (!format_ok) reject("Unsupported tensor format");
  config = ModelConfig::fromJson(manifest.at("config"));
  mode = manifest.at("mode").get<std::string>();
  if (mode != "fp32" && mode != "mixed" && mode != "bf16") reject("Unknown numerical mode");
  mixed = mode != "fp32";

  const MappedFile blob(path / "tensors.bin");
  if (sha256(blob.data(), blob.size()) != manifest.at("sha256").get<std::string>()) reject("Checkpoint hash mismatch");
  const std::vector<TensorDesc> table = describe(manifest.at("tensors"), blob.size());
  for (const TensorDesc& t : table) {
    const unsigned char* src = blob.data() + t.offset;
    if (sha256(src, t.nbytes) != t.digest) reject("Tensor hash mismatch");
    Tensor tensor;
    tensor.shape = t.shape;
    widen(t, src, tensor.data);
    if (!mTensors.emplace(t.name, std::move(tensor)).second) reject("Duplicate tensor");
  }

  // The shape contract: every tensor the step reads, with its exact shape.
  const int d = config.width, f = config.ffn;
  struct Contract {
    const char* name;
    std::vector<int> shape;
  };
  const Contract model_wide[] = {{"input", {d, config.features}}, {"final_norm", {d}}, {"score", {1, d}}};
  const Contract per_layer[] = {{"norm1", {d}}, {"norm2", {d}}, {"q", {d, d}},    {"k", {d, d}},   {"v", {d, d}},
                                {"out", {d, d}}, {"gate", {f, d}}, {"up", {f, d}}, {"down", {d, f}}};
  auto require = [&](const std::string& name, const std::vector<int>& shape) {
    if (get(name).shape != shape) reject("Shape mismatch: " + name);
  };
  for (const Contract& c : model_wide) require(c.name, c.shape);
  for (int l = 0; l < config.layers; ++l)
    for (const Contract& c : per_layer) require("layers." + std::to_string(l) + "." + c.name, c.shape);
}

const Tensor& Model::get(const std::string& name) const {
  const auto found = mTensors.find(name);
  if (found == mTensors.end()) reject("Unknown tensor " + name);
  return found->second;
}

}  // namespace Stream
