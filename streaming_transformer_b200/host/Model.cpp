// Model.cpp -- checkpoint loader of the Stream API (include/Model.hpp).
//
// Same format and checks as the reference loader (reference
// src/runtime/Model.cpp:15-145): manifest version 1, little endian, out_in
// orientation, whole-file and per-tensor SHA-256 (OpenSSL), contiguous tensors
// in manifest order, exact shapes, storage widened to float. bf16 tensors
// ("bfloat16", mode "bf16") are accepted in addition to float32 / float16.
#include "Model.hpp"

#include <bit>
#include <cmath>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <sstream>
#include <stdexcept>

#include <openssl/sha.h>

namespace Stream {

ModelConfig ModelConfig::fromJson(const Json& j) {
  ModelConfig c{j.at("layers").get<int>(), j.at("width").get<int>(), j.at("heads").get<int>(),
                j.at("ffn").get<int>(), j.at("window").get<int>(), j.at("features").get<int>(),
                j.at("epsilon").get<float>()};
  c.validate();
  return c;
}

// reference src/runtime/Model.cpp:22-29
void ModelConfig::validate() const {
  if (layers < 1 || layers > 16 || width < 1 || width > 1024 || heads < 1 || width % heads ||
      (width / heads) % 2 || ffn < 1 || ffn > 4096 || window < 1 || window > 4096 || features < 1 ||
      features > 1024 || !std::isfinite(epsilon) || epsilon <= 0) {
    throw std::runtime_error("Invalid or unsupported model dimensions");
  }
}

std::size_t ModelConfig::cacheElements() const { return std::size_t(layers) * width * window; }

std::vector<char> readBytes(const std::filesystem::path& path) {
  std::ifstream file(path, std::ios::binary | std::ios::ate);
  if (!file) throw std::runtime_error("Cannot read " + path.string());
  const auto length = file.tellg();
  std::vector<char> bytes(static_cast<std::size_t>(length));
  file.seekg(0);
  if (!file.read(bytes.data(), (std::streamsize)bytes.size())) throw std::runtime_error("Short read " + path.string());
  return bytes;
}

std::string sha256(const void* data, std::size_t bytes) {
  unsigned char hash[SHA256_DIGEST_LENGTH];
  SHA256(static_cast<const unsigned char*>(data), bytes, hash);
  std::ostringstream out;
  for (auto byte : hash) out << std::hex << std::setw(2) << std::setfill('0') << int(byte);
  return out.str();
}

// IEEE-754 binary16 round-to-nearest-even, widened back to float.
float roundHalf(float value) {
  std::uint32_t u;
  std::memcpy(&u, &value, 4);
  const std::uint32_t sign = u & 0x80000000u, mag = u & 0x7fffffffu;
  std::uint32_t r;
  if (mag >= 0x7f800000u) {
    r = u;
  } else if (mag >= 0x477ff000u) {
    r = sign | 0x7f800000u;
  } else if (mag < 0x38800000u) {
    float scaled = std::fabs(value) * 16777216.0f;
    float q = std::nearbyint(scaled) / 16777216.0f;
    std::memcpy(&r, &q, 4);
    r |= sign;
  } else {
    r = sign | ((mag + 0x0fffu + ((mag >> 13) & 1u)) & ~0x1fffu);
  }
  float out;
  std::memcpy(&out, &r, 4);
  return out;
}

namespace {
float half_to_float(std::uint16_t h) {
  const std::uint32_t sign = (std::uint32_t)(h & 0x8000u) << 16;
  const std::uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  std::uint32_t bits;
  if (exp == 0) {
    float v = (float)man * (1.0f / 16777216.0f);
    std::memcpy(&bits, &v, 4);
    bits |= sign;
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}
}  // namespace

// reference src/runtime/Model.cpp:63-140
Model::Model(const std::filesystem::path& path) {
  std::ifstream file(path / "manifest.json");
  if (!file) throw std::runtime_error("Cannot read " + (path / "manifest.json").string());
  file >> manifest;
  if (manifest.at("version").get<int>() != 1 || manifest.at("byte_order").get<std::string>() != "little" ||
      manifest.at("orientation").get<std::string>() != "out_in" || std::endian::native != std::endian::little) {
    throw std::runtime_error("Unsupported tensor format");
  }
  config = ModelConfig::fromJson(manifest.at("config"));
  mode = manifest.at("mode").get<std::string>();
  if (mode != "fp32" && mode != "mixed" && mode != "bf16") throw std::runtime_error("Unknown numerical mode");
  mixed = mode != "fp32";
  auto bytes = readBytes(path / "tensors.bin");
  if (sha256(bytes.data(), bytes.size()) != manifest.at("sha256").get<std::string>())
    throw std::runtime_error("Checkpoint hash mismatch");
  std::size_t end = 0;
  for (const auto& item : manifest.at("tensors")) {
    Tensor tensor;
    tensor.shape = item.at("shape").get<std::vector<int>>();
    std::size_t count = 1;
    for (int dim : tensor.shape) {
      if (dim <= 0 || count > bytes.size() / std::size_t(dim)) throw std::runtime_error("Invalid tensor dimensions");
      count *= dim;
    }
    const auto dtype = item.at("dtype").get<std::string>();
    const std::size_t size = dtype == "float32" ? 4 : (dtype == "float16" || dtype == "bfloat16") ? 2 : 0;
    const std::size_t offset = item.at("offset").get<std::size_t>(), nbytes = item.at("nbytes").get<std::size_t>();
    if (!size || offset != end || nbytes != count * size || offset > bytes.size() || nbytes > bytes.size() - offset)
      throw std::runtime_error("Invalid tensor bounds");
    if (sha256(bytes.data() + offset, nbytes) != item.at("sha256").get<std::string>())
      throw std::runtime_error("Tensor hash mismatch");
    tensor.data.resize(count);
    if (size == 4) {
      std::memcpy(tensor.data.data(), bytes.data() + offset, nbytes);
    } else {
      for (std::size_t i = 0; i < count; i++) {
        std::uint16_t h;
        std::memcpy(&h, bytes.data() + offset + 2 * i, 2);
        if (dtype == "float16") {
          tensor.data[i] = half_to_float(h);
        } else {
          const std::uint32_t bits = (std::uint32_t)h << 16;
          std::memcpy(&tensor.data[i], &bits, 4);
        }
      }
    }
    const auto name = item.at("name").get<std::string>();
    if (!mTensors.emplace(name, std::move(tensor)).second) throw std::runtime_error("Duplicate tensor");
    end += nbytes;
  }
  if (end != bytes.size()) throw std::runtime_error("Trailing tensor bytes");
  auto check = [&](const std::string& name, std::vector<int> shape) {
    if (get(name).shape != shape) throw std::runtime_error("Shape mismatch: " + name);
  };
  check("input", {config.width, config.features});
  check("final_norm", {config.width});
  check("score", {1, config.width});
  for (int l = 0; l < config.layers; l++) {
    const auto p = "layers." + std::to_string(l) + ".";
    for (auto name : {"norm1", "norm2"}) check(p + name, {config.width});
    for (auto name : {"q", "k", "v", "out"}) check(p + name, {config.width, config.width});
    for (auto name : {"gate", "up"}) check(p + name, {config.ffn, config.width});
    check(p + "down", {config.width, config.ffn});
  }
}

const Tensor& Model::get(const std::string& name) const {
  auto it = mTensors.find(name);
  if (it == mTensors.end()) throw std::runtime_error("Unknown tensor " + name);
  return it->second;
}

}  // namespace Stream
