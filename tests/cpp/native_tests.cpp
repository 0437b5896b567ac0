// native_tests.cpp -- the C++ drop-in API exercised the way the reference's
// own C++ tests exercise it (reference tests/Native.cpp:10-74,
// tests/Lifecycle.cu:17-137). The CPU oracle (oracle/st_oracle.h) stands in
// for the reference's Eigen Stream::Cpu as the comparison.
//
//   native_tests <repo-root> cpu   checks that need no GPU
//   native_tests <repo-root> gpu   checks that run the B200 runtime
// Exit status = number of failed checks.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <functional>
#include <limits>
#include <string>
#include <thread>
#include <vector>

#include "Model.hpp"
#include "Runtime.hpp"
#include "st_oracle.h"

namespace {
int g_failures = 0;
std::string g_test;

#define EXPECT(cond)                                                                     \
  do {                                                                                   \
    if (!(cond)) {                                                                       \
      ++g_failures;                                                                      \
      std::fprintf(stderr, "FAIL %s: %s (%s:%d)\n", g_test.c_str(), #cond, __FILE__, __LINE__); \
    }                                                                                    \
  } while (0)
#define EXPECT_THROW(stmt)                         \
  do {                                             \
    bool thrown = false;                           \
    try { stmt; } catch (const std::exception&) { thrown = true; } \
    EXPECT(thrown && #stmt);                       \
  } while (0)

void run(const std::string& name, const std::function<void()>& fn) {
  g_test = name;
  const int before = g_failures;
  try {
    fn();
  } catch (const std::exception& e) {
    ++g_failures;
    std::fprintf(stderr, "FAIL %s: exception %s\n", name.c_str(), e.what());
  }
  std::printf("%s %s\n", g_failures == before ? "PASS" : "FAIL", name.c_str());
}

std::filesystem::path g_root;

std::filesystem::path fixture(const std::string& name) { return g_root / "tests" / "golden" / name; }

// The oracle as the CPU comparison (reference Stream::Cpu).
struct CpuOracle {
  st_oracle* o = nullptr;
  explicit CpuOracle(const Stream::Model& m) {
    st_oracle_config c{m.config.layers, m.config.width, m.config.heads, m.config.ffn, m.config.window,
                       m.config.features, m.config.epsilon, m.mode == "mixed" ? 1 : m.mode == "bf16" ? 2 : 0};
    o = st_oracle_create(&c, 1);
    auto set = [&](const std::string& n) {
      const auto& t = m.get(n);
      st_oracle_set_tensor(o, n.c_str(), t.data.data(), t.data.size());
    };
    set("input");
    set("final_norm");
    set("score");
    for (int l = 0; l < m.config.layers; ++l)
      for (auto n : {"norm1", "norm2", "q", "k", "v", "out", "gate", "up", "down"})
        set("layers." + std::to_string(l) + "." + n);
  }
  ~CpuOracle() { st_oracle_destroy(o); }
  float step(const float* e) { return st_oracle_step(o, e); }
  void reset() { st_oracle_reset(o); }
  std::uint64_t position() const { return st_oracle_position(o); }
};

std::vector<float> trace_events(const std::filesystem::path& dir, const Stream::Model& m) {
  auto bytes = Stream::readBytes(dir / "trace.bin");
  std::vector<float> events(bytes.size() / sizeof(float));
  std::memcpy(events.data(), bytes.data(), bytes.size());
  return events;
}

bool close(float a, float b, bool mixed) {
  return std::fabs(a - b) <= (mixed ? 2e-3 : 1e-5) + (mixed ? 2e-2 : 1e-4) * std::fabs(b);
}

void cpu_tests() {
  run("Config.RejectInvalid", [] {
    auto c = Stream::ModelConfig::fromJson(Stream::Json{{"layers", 1}, {"width", 64}, {"heads", 4}, {"ffn", 128},
                                                        {"window", 64}, {"features", 32}, {"epsilon", 1e-5}});
    EXPECT(c.cacheElements() == 4096u);
    c.heads = 3;
    EXPECT_THROW(c.validate());
  });
  run("Format.HashAndHalf", [] {
    EXPECT(Stream::sha256("abc", 3) == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad");
    EXPECT(Stream::roundHalf(1.0001f) == 1.0f);
    EXPECT(std::isinf(Stream::roundHalf(1e10f)));
  });
  run("Model.LoadsGoldenCheckpoints", [] {
    for (auto name : {"ref-small-fp32", "ref-small-mixed", "ref-main-fp32", "ref-main-mixed"}) {
      Stream::Model m(fixture(name));
      EXPECT(m.mixed == (m.mode == "mixed"));
      EXPECT(m.get("input").shape == (std::vector<int>{m.config.width, m.config.features}));
    }
    EXPECT_THROW(Stream::Model(fixture("does-not-exist")));
  });
  run("Json.RoundTrip", [] {
    auto j = Stream::Json::parse(R"({"a": [1, 2.5, "x", true, null], "b": {"c": -3}})");
    EXPECT(j.at("a").size() == 5 && j.at("a").at(1).get<double>() == 2.5);
    EXPECT(j.at("b").at("c").get<int>() == -3);
    EXPECT(Stream::Json::parse(j.dump()) == j);
    EXPECT(Stream::Json::parse(j.dump(2)) == j);
  });
  run("Runtime.RejectsCublasBeforeTouchingTheDevice", [] {
    Stream::Model m(fixture("ref-small-fp32"));
    Stream::RuntimeOptions o;
    o.backend = Stream::Backend::CUBLAS;
    EXPECT_THROW({ Stream::Runtime r(m, o); });
    o.backend = Stream::Backend::GRAPH;
    o.idleSeconds = 0;
    EXPECT_THROW({ Stream::Runtime r(m, o); });
  });
}

void gpu_tests() {
  run("Backends.MatchTheCpuOracle", [] {
    for (auto name : {"ref-small-fp32", "ref-main-mixed"}) {
      Stream::Model m(fixture(name));
      auto events = trace_events(fixture(name), m);
      for (auto b : {Stream::Backend::CUDA, Stream::Backend::GRAPH, Stream::Backend::FUSED, Stream::Backend::PERSISTENT}) {
        Stream::RuntimeOptions o;
        o.backend = b;
        o.blocks = 0;
        Stream::Runtime rt(m, o);
        CpuOracle cpu(m);
        for (int i = 0; i < 40; ++i) {
          const float* e = events.data() + (size_t)i * m.config.features;
          EXPECT(close(rt.step(e), cpu.step(e), m.mixed));
        }
        EXPECT(rt.snapshot().position == 40u);
      }
    }
  });
  // reference tests/Lifecycle.cu:17-48
  run("Persistent.ResetRepeatedScoresAndRestart", [] {
    for (const std::string mode : {"fp32", "mixed"}) {
      Stream::Model model(fixture("ref-small-" + mode));
      for (int blocks : {1, 4}) {
        Stream::RuntimeOptions options;
        options.backend = Stream::Backend::PERSISTENT;
        options.blocks = blocks;
        for (int restart = 0; restart < 2; restart++) {
          Stream::Runtime runtime(model, options);
          CpuOracle cpu(model);
          std::vector<float> event(model.config.features, 0);
          for (int i = 0; i < 3 * model.config.window + 9; i++) {
            if (i == 1 || i == model.config.window || i == 2 * model.config.window + 3) {
              runtime.reset();
              runtime.reset();
              cpu.reset();
              EXPECT(runtime.snapshot().position == 0u);
            }
            EXPECT(std::fabs(runtime.step(event.data()) - cpu.step(event.data())) <= 1e-6);
            EXPECT(runtime.snapshot().position == cpu.position());
          }
          runtime.stop();
          runtime.stop();
          EXPECT_THROW(runtime.step(event.data()));
          EXPECT_THROW(runtime.reset());
        }
      }
    }
  });
  // reference tests/Lifecycle.cu:50-73
  run("Persistent.FiniteAndIdleExit", [] {
    Stream::Model model(fixture("ref-small-fp32"));
    std::vector<float> event(model.config.features, 0);
    for (int blocks : {1, 4}) {
      Stream::RuntimeOptions options;
      options.backend = Stream::Backend::PERSISTENT;
      options.blocks = blocks;
      options.maxEvents = 2;
      Stream::Runtime runtime(model, options);
      EXPECT(runtime.step(event.data()) == 0.0f);
      runtime.reset();
      EXPECT(runtime.step(event.data()) == 0.0f);
      EXPECT_THROW(runtime.step(event.data()));
      runtime.stop();
    }
    Stream::RuntimeOptions idle;
    idle.backend = Stream::Backend::PERSISTENT;
    idle.idleSeconds = .001;
    Stream::Runtime runtime(model, idle);
    std::this_thread::sleep_for(std::chrono::milliseconds(100));
    EXPECT_THROW(runtime.step(event.data()));
    runtime.stop();
  });
  // reference tests/Lifecycle.cu:75-91
  run("Persistent.SequenceExhaustionStillAllowsStop", [] {
    Stream::Model model(fixture("ref-small-fp32"));
    std::vector<float> event(model.config.features, 0);
    for (int blocks : {1, 4}) {
      Stream::RuntimeOptions options;
      options.backend = Stream::Backend::PERSISTENT;
      options.blocks = blocks;
      options.initialSequence = std::numeric_limits<std::uint64_t>::max() - 2;
      Stream::Runtime runtime(model, options);
      EXPECT(runtime.step(event.data()) == 0.0f);
      EXPECT_THROW(runtime.step(event.data()));
      EXPECT_THROW(runtime.reset());
      runtime.stop();
      runtime.stop();
    }
  });
  // reference tests/Lifecycle.cu:108-137
  run("Diagnostic.CudaSnapshotsPreserveExecution", [] {
    Stream::Model model(fixture("ref-main-mixed"));
    Stream::RuntimeOptions options;
    options.backend = Stream::Backend::CUDA;
    options.blocks = 4;
    Stream::Runtime runtime(model, options);
    auto events = trace_events(fixture("ref-main-mixed"), model);
    std::vector<float> scores;
    for (int i = 0; i < 12; i++) scores.push_back(runtime.step(events.data() + (size_t)i * model.config.features));
    auto state = runtime.snapshot();
    runtime.reset();
    for (int i = 0; i < 12; i++) {
      auto trace = runtime.traceStep(events.data() + (size_t)i * model.config.features);
      EXPECT(trace.at("layers.0.attention").size() == (size_t)model.config.width);
      EXPECT(scores[i] == trace.at("score.linear")[0]);
    }
    auto traced = runtime.snapshot();
    EXPECT(state.position == traced.position);
    EXPECT(state.keys == traced.keys);
    EXPECT(state.values == traced.values);
    EXPECT(state.hidden == traced.hidden);
  });
  run("Runtime.InfoProbeAndDeviceTrace", [] {
    auto p = Stream::probe();
    EXPECT(p.at("compute_major").get<int>() == 10);
    Stream::Model model(fixture("ref-small-fp32"));
    Stream::RuntimeOptions options;
    options.backend = Stream::Backend::FUSED;
    options.blocks = 0;
    Stream::Runtime runtime(model, options);
    auto info = runtime.info();
    EXPECT(info.at("threads").get<int>() == 512);
    EXPECT(info.at("backend").get<std::string>() == "fused");
    auto events = trace_events(fixture("ref-small-fp32"), model);
    EXPECT(runtime.deviceTrace(events.data(), 20) > 0.0);
    EXPECT(runtime.snapshot().position == 20u);
  });
  run("Transport.CopyAndGridBarrier", [] {
    auto copy = Stream::transportBench("copy", 200, false, "");
    EXPECT(copy.at("failed").get<int>() == 0 && copy.at("p50_us").get<double>() > 0);
    auto barrier = Stream::transportBench("grid-barrier", 1000, false, "");
    EXPECT(barrier.at("ns_per_barrier").get<double>() > 0);
  });
}
}  // namespace

int main(int argc, char** argv) {
  if (argc < 3) {
    std::fprintf(stderr, "usage: native_tests <repo-root> cpu|gpu\n");
    return 2;
  }
  g_root = argv[1];
  const std::string group = argv[2];
  if (group == "cpu") cpu_tests();
  else if (group == "gpu") gpu_tests();
  else return 2;
  std::printf("%d failed\n", g_failures);
  return g_failures;
}
