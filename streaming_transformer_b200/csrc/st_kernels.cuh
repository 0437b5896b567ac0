// st_kernels.cuh -- kernel entry points of the streaming step.
//
//   per-op (CUDA / GRAPH backends)   k_input, k_qkv, k_attention, k_out,
//                                    k_ffn_in, k_ffn_out, k_final, k_reset
//   FUSED                            k_fused: one cooperative launch per step
//   device trace                     k_trace: a preloaded trace in one launch
//   PERSISTENT                       k_persistent: resident, mapped mailbox
// They replace the reference's stage/input/norm/score/advance/reset kernels,
// fused_kernel, trace_kernel and persistent_kernel (reference
// src/cuda/Runtime.cu:16-132).
#pragma once

#include "st_device.cuh"

namespace st {

// Host-visible request/completion words, each on its own 64-byte line, in
// cudaHostAllocMapped memory. Host and device only load and store them (no
// read-modify-write across the bus), release/acquire as in the reference
// protocol (reference docs/transport.md:7-18, src/cuda/Primitives.cuh:14-24).
struct alignas(64) Mailbox {
  alignas(64) unsigned long long request;
  alignas(64) unsigned long long completion;
  alignas(64) unsigned long long exited;
  alignas(64) int command;
  int arg;                       // RESET: stream index, or -1 for all streams
  unsigned long long checksum;   // PING reply
  alignas(64) int error;         // mirror of the device error word
};

// Coordinator decision broadcast to every CTA through device memory.
struct Control {
  unsigned long long sequence;
  int command;
  int arg;
  int exit;
};

struct PersistArgs {
  Mailbox* mailbox;                 // device alias of the mapped mailbox
  unsigned long long max_events;    // 0 = unbounded
  unsigned long long initial_sequence;
  unsigned long long idle_ns;       // coordinator idle budget
  unsigned long long dispatch_timeout_ns;
  Control* control;
  int backoff;
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_input(StepArgs a) {
  __shared__ Smem sm;
  phase_input<T>(a, a.input, sm);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_qkv(StepArgs a, int l) {
  __shared__ Smem sm;
  phase_qkv<T>(a, l, sm);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_attention(StepArgs a, int l) {
  phase_attention<T>(a, l);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_out(StepArgs a, int l) {
  __shared__ Smem sm;
  phase_out<T>(a, l, sm);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_ffn_in(StepArgs a, int l) {
  __shared__ Smem sm;
  phase_ffn_in<T>(a, l, sm);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_ffn_out(StepArgs a, int l) {
  __shared__ Smem sm;
  phase_ffn_out<T>(a, l, sm);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_final(StepArgs a) {
  __shared__ Smem sm;
  phase_final<T>(a, sm);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_reset(StepArgs a, int s0, int s1) {
  reset_streams<T>(a, s0, s1);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_fused(StepArgs a, unsigned long long base) {
  __shared__ Smem sm;
  GridSync gs{base, 0};
  forward<T>(a, a.input, gs, sm);
}

// Steps `count` preloaded events ([count][S][features], device memory) in one
// launch. scores ([count][S]) may be null. One extra barrier per event keeps
// the next input projection from overwriting x while CTA 0 still reads it.
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_trace(StepArgs a, const float* inputs, unsigned long long count,
                                                      float* scores, unsigned long long base) {
  __shared__ Smem sm;
  GridSync gs{base, 0};
  const size_t stride = (size_t)a.streams * a.features;
  for (unsigned long long e = 0; e < count; ++e) {
    if (!forward<T>(a, inputs + e * stride, gs, sm)) return;
    if (scores && blockIdx.x == 0)
      for (int s = threadIdx.x; s < a.streams; s += kThreads) scores[e * a.streams + s] = a.score[s];
    if (!gs.sync(a, a.bar_timeout_ns)) return;
  }
}

template <typename T>
__device__ void persistent_exit(const StepArgs& a, const PersistArgs& p) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const int err = ld_volatile_int(a.error);
    if (err) *reinterpret_cast<volatile int*>(&p.mailbox->error) = err;
    __threadfence_system();
    st_release_sys(&p.mailbox->exited, 1ull);
  }
}

// Resident worker (reference src/cuda/Runtime.cu:58-122): CTA 0 thread 0 polls
// the mailbox within the idle budget and broadcasts the command; every CTA runs
// it; CTA 0 publishes the score and the completion ID with release ordering.
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_persistent(StepArgs a, PersistArgs p, unsigned long long base) {
  __shared__ Smem sm;
  __shared__ Control local;
  GridSync gs{base, 0};
  unsigned long long previous = p.initial_sequence, processed = 0;
  while (true) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      const unsigned long long start = globaltimer();
      unsigned long long seq;
      int exit = 0;
      while ((seq = ld_acquire_sys(&p.mailbox->request)) == previous) {
        if (globaltimer() - start >= p.idle_ns) { exit = 1; break; }
        if (p.backoff) __nanosleep(128);
      }
      volatile Control* c = p.control;
      c->exit = exit;
      if (!exit) {
        c->sequence = seq;
        c->command = *reinterpret_cast<volatile int*>(&p.mailbox->command);
        c->arg = *reinterpret_cast<volatile int*>(&p.mailbox->arg);
      }
    }
    if (!gs.sync(a, p.dispatch_timeout_ns)) { persistent_exit<T>(a, p); return; }
    if (threadIdx.x == 0) {
      const volatile Control* c = p.control;
      local.exit = c->exit;
      local.command = c->command;
      local.arg = c->arg;
      local.sequence = c->sequence;
    }
    __syncthreads();
    if (local.exit) break;
    const int command = local.command;
    const unsigned long long seq = local.sequence;
    if (command == kRun) {
      if (!forward<T>(a, a.input, gs, sm)) { persistent_exit<T>(a, p); return; }
    } else if (command == kReset) {
      const int s0 = local.arg < 0 ? 0 : local.arg;
      const int s1 = local.arg < 0 ? a.streams : local.arg + 1;
      reset_streams<T>(a, s0, s1);
      if (!gs.sync(a, a.bar_timeout_ns)) { persistent_exit<T>(a, p); return; }
    } else {
      if (command == kPing && blockIdx.x == 0 && threadIdx.x == 0) {
        unsigned long long checksum = 0;
        for (int i = 0; i < a.features; ++i) checksum += __float_as_uint(__ldcv(a.input + i));
        *reinterpret_cast<volatile unsigned long long*>(&p.mailbox->checksum) = checksum;
      }
      // No CTA may see the next command before every CTA has read this one.
      if (!gs.sync(a, a.bar_timeout_ns)) { persistent_exit<T>(a, p); return; }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      __threadfence_system();
      st_release_sys(&p.mailbox->completion, seq);
    }
    previous = seq;
    if (command == kRun) ++processed;
    if (command == kStop || (p.max_events && processed >= p.max_events)) break;
  }
  gs.sync(a, a.bar_timeout_ns);
  persistent_exit<T>(a, p);
}

}  // namespace st
