// Runtime.cpp -- Stream::Runtime (include/Runtime.hpp) over the C ABI.
//
// This is the reference's Runtime::Impl (reference src/cuda/Runtime.cu:164-665)
// reduced to argument marshalling: every device resource, kernel and
// protocol lives behind include/streaming_b200.h. Non-zero C status codes
// become std::runtime_error carrying st_last_error(), as the reference raised
// std::runtime_error for the same conditions.
#include "Runtime.hpp"

#include <fstream>
#include <stdexcept>
#include <string>

#include "streaming_b200.h"

namespace Stream {

namespace {
void check(int status, const st_runtime* rt) {
  if (status != ST_OK) throw std::runtime_error(st_last_error(rt));
}

int mode_code(const Model& m) {
  if (m.mode == "mixed") return ST_MODE_FP16;
  if (m.mode == "bf16") return ST_MODE_BF16;
  return ST_MODE_FP32;
}

Json json_call(int status, const std::string& text, const st_runtime* rt) {
  check(status, rt);
  return Json::parse(text);
}
}  // namespace

class Runtime::Impl {
 public:
  Impl(const Model& model, RuntimeOptions options) : mModel(model), mOptions(options) {
    const auto& c = model.config;
    st_model_desc desc{c.layers, c.width, c.heads, c.ffn, c.window, c.features, c.epsilon, mode_code(model), 1};
    st_options o;
    st_default_options(&o);
    o.backend = static_cast<int>(options.backend);
    o.blocks = options.blocks;
    o.backoff = options.backoff;
    o.mapped = options.mapped;
    o.vector_matvec = options.vectorMatvec;
    o.fused_attention = options.fusedAttention;
    o.max_events = options.maxEvents;
    o.initial_sequence = options.initialSequence;
    o.idle_seconds = options.idleSeconds;
    check(st_create(&desc, &o, &mRt), nullptr);
    try {
      auto upload = [&](const std::string& name) {
        const auto& t = model.get(name);
        check(st_set_tensor(mRt, name.c_str(), t.data.data(), t.data.size()), mRt);
      };
      upload("input");
      upload("final_norm");
      upload("score");
      for (int l = 0; l < c.layers; l++) {
        const auto p = "layers." + std::to_string(l) + ".";
        for (auto n : {"norm1", "norm2", "q", "k", "v", "out", "gate", "up", "down"}) upload(p + n);
      }
      check(st_start(mRt), mRt);
    } catch (...) {
      st_destroy(mRt);
      throw;
    }
  }
  ~Impl() { st_destroy(mRt); }

  float step(const float* input) {
    float score = 0;
    check(st_step(mRt, input, &score), mRt);
    return score;
  }
  void reset() { check(st_reset(mRt), mRt); }
  void stop() { check(st_stop(mRt), mRt); }
  Snapshot snapshot() {
    Snapshot s;
    const auto cache = mModel.config.cacheElements();
    s.keys.resize(cache);
    s.values.resize(cache);
    s.hidden.resize(std::size_t(mModel.config.layers) * mModel.config.width);
    std::uint64_t position = 0;
    check(st_snapshot(mRt, 0, &position, s.keys.data(), s.values.data(), s.hidden.data()), mRt);
    s.position = position;
    return s;
  }
  std::map<std::string, std::vector<float>> traceStep(const float* input) {
    std::map<std::string, std::vector<float>> trace;
    float score = 0;
    auto capture = [](void* user, const char* name, const float* data, size_t count) {
      (*static_cast<std::map<std::string, std::vector<float>>*>(user))[name].assign(data, data + count);
    };
    check(st_trace_step(mRt, input, &score, capture, &trace), mRt);
    return trace;
  }
  Json info() const {
    size_t needed = 0;
    check(st_info(mRt, nullptr, 0, &needed), mRt);
    std::string text(needed, '\0');
    const int status = st_info(mRt, text.data(), text.size(), &needed);
    text.resize(needed ? needed - 1 : 0);
    return json_call(status, text, mRt);
  }
  double deviceTrace(const float* inputs, std::size_t count) {
    double us = 0;
    check(st_device_trace(mRt, inputs, count, nullptr, &us), mRt);
    return us;
  }

 private:
  const Model& mModel;
  RuntimeOptions mOptions;
  st_runtime* mRt = nullptr;
};

Runtime::Runtime(const Model& model, RuntimeOptions options) : mImpl(std::make_unique<Impl>(model, options)) {}
Runtime::~Runtime() = default;
float Runtime::step(const float* input) { return mImpl->step(input); }
void Runtime::reset() { mImpl->reset(); }
void Runtime::stop() { mImpl->stop(); }
Snapshot Runtime::snapshot() { return mImpl->snapshot(); }
std::map<std::string, std::vector<float>> Runtime::traceStep(const float* input) { return mImpl->traceStep(input); }
Json Runtime::info() const { return mImpl->info(); }
double Runtime::deviceTrace(const float* inputs, std::size_t count) { return mImpl->deviceTrace(inputs, count); }

Json probe() {
  size_t needed = 0;
  int status = st_probe(0, nullptr, 0, &needed);
  if (status != ST_OK) throw std::runtime_error(st_last_error(nullptr));
  std::string text(needed, '\0');
  status = st_probe(0, text.data(), text.size(), &needed);
  text.resize(needed ? needed - 1 : 0);
  if (status != ST_OK) throw std::runtime_error(st_last_error(nullptr));
  return Json::parse(text);
}

// reference src/cuda/Runtime.cu:706-814; `output` + ".csv" receives the samples
// and `output` + ".json" the report, as in the reference bench.
Json transportBench(const std::string& mode, std::size_t count, bool backoff, const std::string& output) {
  std::string text(1 << 16, '\0');
  size_t needed = 0;
  const std::string csv = output.empty() ? std::string() : output + ".csv";
  const int status = st_transport_bench(0, mode.c_str(), count, backoff, csv.empty() ? nullptr : csv.c_str(),
                                        text.data(), text.size(), &needed);
  if (status != ST_OK) throw std::runtime_error(st_transport_error());
  text.resize(needed ? needed - 1 : 0);
  Json report = Json::parse(text);
  if (!output.empty()) std::ofstream(output + ".json") << report.dump(2) << '\n';
  return report;
}

}  // namespace Stream
