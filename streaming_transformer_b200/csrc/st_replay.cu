// st_replay.cu -- scheduled-arrival replay of an event trace (host only).
//
// The service-level benchmark of the reference (reference bench/Main.cpp:
// 282-343, statistics 416-447): a producer thread lets event i "arrive" at
// its scheduled time -- i / rate seconds after the start, or in groups of 16
// arriving together when bursty -- and appends it to a bounded single-producer
// single-consumer queue (an arrival that finds the queue full is dropped);
// the calling thread takes events from the queue in order and steps them.
// Every event gets four timestamps on one steady clock: intended arrival,
// enqueue, submit (taken off the queue) and completion. Reported: injection
// (enqueue - intended), queueing (submit - enqueue), service (complete -
// submit) and arrival-to-completion (complete - intended) distributions,
// deadline misses, drops and the service rate.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include <pthread.h>
#include <sched.h>

#include "../../include/streaming_b200.h"

namespace {

thread_local std::string g_replay_error;

double now_ns() {
  return (double)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

void pin(int core) {
  if (core < 0) return;
  cpu_set_t set;
  CPU_ZERO(&set);
  CPU_SET(core, &set);
  pthread_setaffinity_np(pthread_self(), sizeof set, &set);
}

// Nearest-rank percentiles (sorted[ceil(q n) - 1]), as the reference's bench.
std::string distribution(std::vector<double> v) {
  if (v.empty()) return "{}";
  std::sort(v.begin(), v.end());
  auto rank = [&](double q) {
    size_t i = (size_t)std::ceil(q * (double)v.size());
    return v[i == 0 ? 0 : i - 1];
  };
  std::ostringstream o;
  o.precision(17);
  o << "{\"p50_us\":" << rank(0.5) << ",\"p95_us\":" << rank(0.95) << ",\"p99_us\":" << rank(0.99)
    << ",\"p999_us\":" << rank(0.999) << ",\"worst_us\":" << v.back() << "}";
  return o.str();
}

int fail(int code, const std::string& msg) {
  g_replay_error = msg;
  return code;
}

}  // namespace

extern "C" {

int st_replay_scheduled_with(st_step_fn step, void* user, const float* inputs, size_t count, size_t features,
                             const st_schedule* schedule, double* samples, float* scores, char* json,
                             size_t capacity, size_t* needed) {
  if (!step || !inputs || !schedule || count == 0 || features == 0) return fail(ST_ERR_INVALID, "null argument");
  const st_schedule sc = *schedule;
  if (!(sc.rate > 0) || !std::isfinite(sc.rate) || sc.queue == 0 || !(sc.deadline_us >= 0))
    return fail(ST_ERR_INVALID, "Invalid rate, queue capacity or deadline");
  struct Sample {
    double intended = 0, enqueue = 0, submit = 0, complete = 0;
    float score = NAN;
    bool dropped = false;
  };
  std::vector<Sample> s(count);
  std::vector<double> when(count);
  for (size_t i = 0; i < count; ++i) when[i] = (double)(sc.bursty ? (i / 16) * 16 : i) * 1e9 / sc.rate;
  std::vector<size_t> queue(sc.queue);
  std::atomic<size_t> head{0}, tail{0};
  std::atomic<bool> done{false};
  size_t dropped = 0;
  const double epoch = now_ns() + 1e8;  // the first arrival 100 ms from now
  std::thread producer([&] {
    pin(sc.producer_core);
    for (size_t i = 0; i < count; ++i) {
      s[i].intended = epoch + when[i];
      while (now_ns() < s[i].intended) std::this_thread::yield();
      s[i].enqueue = now_ns();
      const size_t write = tail.load(std::memory_order_relaxed);
      if (write - head.load(std::memory_order_acquire) == sc.queue) {
        s[i].dropped = true;
        ++dropped;
      } else {
        queue[write % sc.queue] = i;
        tail.store(write + 1, std::memory_order_release);
      }
    }
    done.store(true, std::memory_order_release);
  });
  int status = ST_OK;
  const double start = now_ns();
  while (true) {
    const size_t read = head.load(std::memory_order_relaxed);
    if (read == tail.load(std::memory_order_acquire)) {
      // re-read the tail after seeing `done`, so the last queued event is not lost
      if (done.load(std::memory_order_acquire) && read == tail.load(std::memory_order_acquire)) break;
      std::this_thread::yield();
      continue;
    }
    const size_t i = queue[read % sc.queue];
    head.store(read + 1, std::memory_order_release);
    s[i].submit = now_ns();
    float score = NAN;
    const int st = step(user, inputs + i * features, &score);
    s[i].complete = now_ns();
    s[i].score = score;
    if (st != ST_OK) {
      status = st;
      break;  // the producer finishes its schedule; the rest stays unserved
    }
  }
  producer.join();
  const double wall = (now_ns() - start) / 1e9;
  std::vector<double> service, arrival, queueing, injection;
  size_t misses = 0, completed = 0;
  for (size_t i = 0; i < count; ++i) {
    const Sample& x = s[i];
    injection.push_back((x.enqueue - x.intended) / 1000.0);
    if (!x.dropped && x.complete > 0) {
      ++completed;
      service.push_back((x.complete - x.submit) / 1000.0);
      arrival.push_back((x.complete - x.intended) / 1000.0);
      queueing.push_back((x.submit - x.enqueue) / 1000.0);
      if (arrival.back() > sc.deadline_us) ++misses;
    }
    if (samples) {
      samples[4 * i] = x.intended;
      samples[4 * i + 1] = x.enqueue;
      samples[4 * i + 2] = x.dropped ? 0 : x.submit;
      samples[4 * i + 3] = x.dropped ? 0 : x.complete;
    }
    if (scores) scores[i] = x.dropped ? NAN : x.score;
  }
  std::ostringstream o;
  o.precision(17);
  o << "{\"mode\":\"scheduled\",\"events\":" << count << ",\"completed\":" << completed << ",\"dropped\":" << dropped
    << ",\"rate_per_second\":" << sc.rate << ",\"bursty\":" << (sc.bursty ? "true" : "false")
    << ",\"queue_capacity\":" << sc.queue << ",\"wall_seconds\":" << wall
    << ",\"service_rate_per_second\":" << (wall > 0 ? (double)completed / wall : 0.0)
    << ",\"deadline_us\":" << sc.deadline_us << ",\"deadline_misses\":" << misses
    << ",\"service\":" << distribution(service) << ",\"arrival\":" << distribution(arrival)
    << ",\"queueing\":" << distribution(queueing) << ",\"injection\":" << distribution(injection)
    << ",\"timing_clock\":\"std::chrono::steady_clock; all timestamps share this clock\"}";
  const std::string out = o.str();
  if (needed) *needed = out.size() + 1;
  if (json && capacity) {
    const size_t n = std::min(capacity - 1, out.size());
    std::memcpy(json, out.data(), n);
    json[n] = '\0';
  }
  if (status != ST_OK) g_replay_error = "a step failed during the replay";
  return status;
}

static int runtime_step(void* user, const float* input, float* score) {
  return st_step(static_cast<st_runtime*>(user), input, score);
}

int st_replay_scheduled(st_runtime* rt, const float* inputs, size_t count, const st_schedule* schedule,
                        double* samples, float* scores, char* json, size_t capacity, size_t* needed) {
  if (!rt) return fail(ST_ERR_INVALID, "null runtime");
  // the feature count comes from the runtime's own description
  size_t need = 0;
  int st = st_info(rt, nullptr, 0, &need);
  if (st != ST_OK) return fail(st, "st_info failed");
  std::vector<char> info(need + 1, '\0');
  st = st_info(rt, info.data(), info.size(), &need);
  if (st != ST_OK) return fail(st, "st_info failed");
  const char* key = std::strstr(info.data(), "\"features\":");
  const size_t features = key ? (size_t)std::strtoul(key + 11, nullptr, 10) : 0;
  if (features == 0) return fail(ST_ERR_STATE, "runtime did not report its feature count");
  return st_replay_scheduled_with(runtime_step, rt, inputs, count, features, schedule, samples, scores, json,
                                  capacity, needed);
}

const char* st_replay_error(void) { return g_replay_error.c_str(); }

}  // extern "C"
