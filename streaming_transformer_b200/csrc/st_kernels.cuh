// st_kernels.cuh -- kernel entry points of the streaming step.
//
//   per-op (CUDA / GRAPH backends)   k2_input, k2_attention, k2_ffn (cluster
//                                    launches), k2_final, k_reset
//   FUSED                            k2_fused: one cooperative cluster launch per step
//   device trace                     k2_trace: a preloaded trace in one launch
//   PERSISTENT                       k2_persistent: resident, mapped mailbox
// They replace the reference's stage/input/norm/score/advance/reset kernels,
// fused_kernel, trace_kernel and persistent_kernel (reference
// src/cuda/Runtime.cu:16-132).
#pragma once

#include "st_batch.cuh"
#include "st_step.cuh"

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

#define ST_SMEM2 \
  extern __shared__ __align__(128) unsigned char st_smem_raw[]; \
  Smem2& sm = *reinterpret_cast<Smem2*>(st_smem_raw); \
  RingSmem& rs = *reinterpret_cast<RingSmem*>(st_smem_raw + sizeof(Smem2)); \
  unsigned char* ring_buf = st_smem_raw + kRingOffset; \
  (void)rs; \
  (void)ring_buf; \
  for (int i_ = threadIdx.x; i_ < a.head_dim / 2; i_ += kThreads) sm.rope[i_] = a.rope_freq[i_]; \
  __syncthreads()

// Ring setup shared by the step kernels (kRing variants only; the host chose
// them after ring_supported). `steps` bounds the chunks issued: steps x
// streams x chunks per step (0: unbounded, resident kernel). Returns false, with the error word set, when the chunk
// table could not be built -- the whole grid then leaves before any barrier.
template <typename T, bool kRing>
__device__ bool ring_setup(const StepArgs& a, Ring& rg, RingSmem& rs, unsigned char* buf, unsigned long long steps) {
  rg.enabled = false;
  rg.consumed = 0;
  if constexpr (!kRing) return true;
  const ClusterPos cp = ClusterPos::get();
  const Where w{(int)cp.rank, (int)cp.size, (int)cp.id, (int)cp.count};
  // every stream of every step walks the chunk list once
  const unsigned long long limit =
      steps ? steps * (unsigned long long)a.streams * chunks_per_step(a, w, sizeof(T)) : ~0ull;
  ring_begin(a, rg, rs, buf, kRingCapacity, w, sizeof(T), limit, true);
  if (!rg.enabled && threadIdx.x == 0) set_error(a, kRingTable);
  return rg.enabled;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k2_input(StepArgs a) {
  ST_SMEM2;
  if (!cluster_shape_ok(a)) return;
  op_input<T>(a, sm, rs);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k2_attention(StepArgs a, int l) {
  ST_SMEM2;
  if (!cluster_shape_ok(a)) return;
  op_attention<T>(a, l, sm, rs);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k2_ffn(StepArgs a, int l) {
  ST_SMEM2;
  if (!cluster_shape_ok(a)) return;
  op_ffn<T>(a, l, sm, rs);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k2_final(StepArgs a, int nclusters) {
  ST_SMEM2;
  op_final<T>(a, nclusters, sm);
}
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_reset(StepArgs a, int s0, int s1) {
  reset_streams<T>(a, s0, s1);
}

template <typename T, bool kRing>
__global__ void __launch_bounds__(kThreads, 1) k2_fused(StepArgs a, unsigned long long base) {
  ST_SMEM2;
  if (!cluster_shape_ok(a)) return;
  ClusterGridSync gs{base, 0};
  Ring rg;
  if (!ring_setup<T, kRing>(a, rg, rs, ring_buf, 1)) return;
  forward2<T, StepCfg<kRing, false>>(a, a.input, gs, sm, rg, rs);
  ring_drain(a, rg, rs);
}

// Steps `count` preloaded events ([count][S][features], device memory) in one
// launch; the kDiag variant also records the phase timeline. scores
// ([count][S]) may be null.
template <typename T, bool kRing, bool kDiag>
__global__ void __launch_bounds__(kThreads, 1) k2_trace(StepArgs a, const float* inputs, unsigned long long count,
                                                       float* scores, unsigned long long base) {
  ST_SMEM2;
  if (!cluster_shape_ok(a)) return;
  ClusterGridSync gs{base, 0};
  if (threadIdx.x < kWarps) sm.tl_nw[threadIdx.x] = 0;
  __syncthreads();
  Ring rg;
  if (!ring_setup<T, kRing>(a, rg, rs, ring_buf, count)) return;
  const size_t stride = (size_t)a.streams * a.features;
  bool ok = true;
  for (unsigned long long e = 0; e < count && ok; ++e)
    ok = forward2<T, StepCfg<kRing, kDiag>>(a, inputs + e * stride, gs, sm, rg, rs, e,
                                            scores ? scores + e * a.streams : nullptr, false);
  // Every CTA derived its positions from the stored ones plus the event index,
  // so they are stored once, after the last event (whose reads of them all
  // precede its grid syncs).
  if (ok && is_score_cta())
    for (int s = threadIdx.x; s < a.streams; s += kThreads) a.position[s] = ld_cg_u64(a.position + s) + count;
  ring_drain(a, rg, rs);
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
// the mailbox within the idle budget; on RUN, CTA 0 stages the mapped event
// into device memory before the dispatch barrier (one PCIe read per value, by
// one CTA); every CTA runs the command; CTA 0 publishes the score and the
// completion ID with release ordering.
template <typename T, bool kRing>
__global__ void __launch_bounds__(kThreads, 1) k2_persistent(StepArgs a, PersistArgs p, const float* mapped_input,
                                                            unsigned long long base) {
  ST_SMEM2;
  __shared__ Control local;
  if (!cluster_shape_ok(a)) { persistent_exit<T>(a, p); return; }
  ClusterGridSync gs{base, 0};
  Ring rg;
  if (!ring_setup<T, kRing>(a, rg, rs, ring_buf, 0)) { persistent_exit<T>(a, p); return; }
  unsigned long long previous = p.initial_sequence, processed = 0;
  const int nin = a.streams * a.features;
  while (true) {
    if (blockIdx.x == 0) {
      if (threadIdx.x == 0) {
        const unsigned long long start = globaltimer();
        unsigned long long seq;
        int exit = 0;
        while ((seq = ld_acquire_sys(&p.mailbox->request)) == previous) {
          if (globaltimer() - start >= p.idle_ns) { exit = 1; break; }
          if (p.backoff) __nanosleep(128);
        }
        volatile Control* c = p.control;
        c->exit = exit;
        local.exit = exit;
        if (!exit) {
          local.command = *reinterpret_cast<volatile int*>(&p.mailbox->command);
          c->sequence = seq;
          c->command = local.command;
          c->arg = *reinterpret_cast<volatile int*>(&p.mailbox->arg);
        }
      }
      __syncthreads();
      if (!local.exit && local.command == kRun)
        for (int i = threadIdx.x; i < nin; i += kThreads) const_cast<float*>(a.input)[i] = __ldcv(mapped_input + i);
    }
    if (!gs.sync(a, p.dispatch_timeout_ns, &sm.sync_ok, nullptr, kRing ? &rg : nullptr, &rs)) {
      ring_drain(a, rg, rs);
      persistent_exit<T>(a, p);
      return;
    }
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
      if (!forward2<T, StepCfg<kRing, false>>(a, a.input, gs, sm, rg, rs)) {
        ring_drain(a, rg, rs);
        persistent_exit<T>(a, p);
        return;
      }
    } else if (command == kReset) {
      const int s0 = local.arg < 0 ? 0 : local.arg;
      const int s1 = local.arg < 0 ? a.streams : local.arg + 1;
      reset_streams<T>(a, s0, s1);
      if (!gs.sync(a, a.bar_timeout_ns, &sm.sync_ok)) { ring_drain(a, rg, rs); persistent_exit<T>(a, p); return; }
    } else {
      if (command == kPing && blockIdx.x == 0 && threadIdx.x == 0) {
        unsigned long long checksum = 0;
        for (int i = 0; i < a.features; ++i) checksum += __float_as_uint(__ldcv(mapped_input + i));
        *reinterpret_cast<volatile unsigned long long*>(&p.mailbox->checksum) = checksum;
      }
      // No CTA may see the next command before every CTA has read this one.
      if (!gs.sync(a, a.bar_timeout_ns, &sm.sync_ok)) { ring_drain(a, rg, rs); persistent_exit<T>(a, p); return; }
    }
    // A step's score, hidden state and position come from the score CTA, so it
    // publishes RUN completions; other commands end with a grid sync.
    if ((command == kRun ? is_score_cta() : blockIdx.x == 0) && threadIdx.x == 0) {
      __threadfence_system();
      st_release_sys(&p.mailbox->completion, seq);
    }
    previous = seq;
    if (command == kRun) ++processed;
    if (command == kStop || (p.max_events && processed >= p.max_events)) break;
  }
  gs.sync(a, a.bar_timeout_ns, &sm.sync_ok);
  ring_drain(a, rg, rs);
  persistent_exit<T>(a, p);
}

// Batched rounds (st_batch.cuh): one CTA per SM, no clusters, `count` events
// of every stream, inputs [count][S][features] in device memory, scores
// [count][S] when given; kTc runs the GEMM phases on the tensor cores (16-bit
// modes). Steps of a batched runtime launch it with count 1.
template <typename T, bool kTc>
__global__ void __launch_bounds__(kThreads, 1) k3_rounds(StepArgs a, const float* inputs, unsigned long long count,
                                                        float* scores, unsigned long long base) {
  batched_rounds<T, kTc>(a, inputs, count, scores, base);
}

}  // namespace st
