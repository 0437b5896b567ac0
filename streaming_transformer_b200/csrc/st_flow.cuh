// st_flow.cuh -- the single-stream step at the benchmark shapes, with no grid
// barrier on the step path.
//
// Shapes: width D in {256, 512, 1024} (a template parameter), head_dim 64,
// 32 features, one stream; the host picks this kernel when the model has them
// (flow_supported) and the generic kernels of st_step.cuh otherwise. The
// arithmetic and cast points are the reference step's (reference
// src/cpu/Cpu.cpp:59-141); only the association of the fp32 sums differs.
//
// Grid: NC clusters of CS CTAs (CS = 8, or 4 when 8-CTA clusters are fewer
// than the heads), 512 threads, one CTA per SM, all co-resident. Cluster c
// owns heads c, c + NC, ...; rank r of every cluster owns segment r of the
// width, [r n, (r + 1) n) with n = D / CS. Per layer:
//
//   attention (clusters that own a head; per head h)
//     z = norm1(x)                    every CTA, the gain from the ring
//     q, k, v rows of head h          row pairs split over the cluster, RoPE and
//                                     casts in the warp epilogue, broadcast into
//                                     every rank (st.async); k, v to slot t % W
//     receive (the site's mbarrier)
//     attention over [0, valid)       slots split over the cluster, an online
//                                     softmax per warp, warps merged per CTA, the
//                                     CTA partial sent into every rank (st.async)
//     receive; merge -> o_h (cast)
//     out-projection rows of segment r (K-split by head): P[h][seg r] published
//   exchange 1 (every CTA)            every CTA gathers P[*] of every head for the
//                                     whole width, x' = cast(x + cast(sum_h P[h])) and
//                                     its sum of squares, no cluster handoff
//   FFN (every CTA)                   z = norm2(x'); gate/up row pairs of this CTA's
//                                     ffn slice -> SwiGLU; down-projection K-split
//                                     over the slice -> partial d-vector;
//                                     reduce-scatter in the cluster (DSMEM, barrier);
//                                     rank r publishes D[c][seg r]
//   exchange 2 (every CTA)            rank r gathers D[*][seg r] of every cluster,
//                                     x[seg r] = cast(x' + cast(sum_c D[c])),
//                                     published into every rank (st.async) with its
//                                     sum of squares and the rank's verdict
//
// Publishing is by tagged records: an 8-byte store of {fp32 value, 32-bit tag}
// (single-copy atomic), the tag unique to (step, layer). A consumer polls the
// records of its segment until every tag matches, so the wait and the data
// arrive in one L2 round trip instead of a grid barrier followed by a read.
// The record buffers alternate by layer parity; no CTA can lag a producer by
// two layers (every exchange needs every cluster's previous contribution), so
// a record is never overwritten before all its readers have read it. Tags
// continue across launches from a device word (flow_epoch), so records left
// by an earlier launch or step never match.
//
// Weights: every CTA streams its fixed per-step span sequence (st_ring.cuh's
// span_of assignment: IN, then per layer NORM1 and QKV/OUT of each owned head,
// NORM2, GATEUP, DOWN) through a shared-memory ring of chunks of at most
// 64 KB, copied by cp.async.bulk (global -> this CTA's shared memory, no
// multicast) with mbarrier completion. One issuer thread (lane 0 of warp 15)
// issues whenever released bytes allow, including while its CTA polls records.
// A chunk is shared by all 16 warps: warp passes are dealt round robin, every
// warp arrives on the chunk's empty mbarrier when done (or at once when it has
// no pass in it). The first l2_keep_layers layers are copied with an
// L2::evict_last policy, the rest evict_first.
//
// Every wait is bounded (bar_timeout_ns) and sets the device error word.
// Verdicts are made cluster-uniform at each exchange (every rank broadcasts
// its own), so a failing cluster leaves together after a cluster barrier and
// no CTA exits while a peer may still write into its shared memory.
#pragma once

#include "st_kernels.cuh"

namespace st {

constexpr int kFlowHd = 64;
constexpr int kFlowFeatures = 32;
constexpr int kFlowMaxCluster = 8;
constexpr int kFlowSlots = 8;                  // ring chunks in flight (one mbarrier pair each)
constexpr unsigned kFlowChunkMax = 64u * 1024u;
constexpr int kFlowMaxChunks = 320;            // chunks per step one CTA may consume
constexpr int kFlowKvBytes = 16 * 1024;        // K and V rows one CTA prefetches per head
constexpr int kFlowMaxD = 1024;
constexpr int kFlowMaxAct = 512;               // SwiGLU outputs per CTA
constexpr int kFlowThreads = kThreads + 32;    // 16 compute warps and the producer warp
constexpr int kFlowProducer = kThreads;        // lane 0 of the producer warp

enum FlowMode : int { kFlowTrace = 0, kFlowPersistent = 1 };
enum FlowCommand : int { kFlowExit = 15 };

// Launch parameters of k4_flow beyond StepArgs.
struct FlowLaunch {
  int mode;                         // kFlowTrace or kFlowPersistent
  const float* inputs;              // trace: [count][features] (device)
  unsigned long long count;         // trace: events
  float* scores;                    // trace: [count] or null
  PersistArgs p;                    // persistent: mailbox protocol
  const float* mapped_input;        // persistent: device alias of the mapped event
  unsigned long long bar_base;      // value of a.bar_counter at launch
};

// ---------------------------------------------------------------- chunking
// Rows one warp pass covers for a span: U rows per epilogue group (2 for the
// q/k/v, out and gate/up spans, whose epilogues take row pairs) times the
// groups a warp covers at once when a row is shorter than 32 vectors. Norm
// and down spans are read by the whole CTA, row by row.
__host__ __device__ inline int flow_pass_rows(int kind, int row_bytes) {
  if (kind == kSpanNorm1 || kind == kSpanNorm2 || kind == kSpanDown) return 1;
  const int u = (kind == kSpanQkv || kind == kSpanGateUp || kind == kSpanOut) ? 2 : 1;
  const int nv = row_bytes / 16;
  const int lpr = nv < 32 ? nv : 32;
  return u * (32 / lpr);
}

struct FlowSplit {
  int chunks, rows_per_chunk;
};

// A span is cut into the fewest chunks of at most kFlowChunkMax bytes whose
// row counts are whole warp passes and as equal as possible.
__host__ __device__ inline FlowSplit flow_split(const Span& s, int kind) {
  if (s.rows <= 0) return {0, 0};
  const int pr = flow_pass_rows(kind, s.row_bytes);
  const int units = (s.rows + pr - 1) / pr;
  int per = (int)(kFlowChunkMax / (unsigned)(pr * s.row_bytes));
  if (per < 1) per = 1;
  const int chunks = (units + per - 1) / per;
  const int upc = (units + chunks - 1) / chunks;
  return {chunks, upc * pr};
}

// Chunks one step consumes for CTA position w (the issuer's table order).
__host__ __device__ inline int flow_chunks_per_step(const StepArgs& a, const Where& w, size_t elem) {
  int n = 0;
  auto count = [&](int kind, int l, int h) { n += flow_split(span_of(a, w, kind, l, h, elem), kind).chunks; };
  count(kSpanIn, -1, 0);
  const int hl = a.heads / a.tp_size, hb = a.tp_rank * hl;
  for (int l = 0; l < a.layers; ++l) {
    if (w.id < hl) {
      count(kSpanNorm1, l, 0);
      for (int h = hb + w.id; h < hb + hl; h += w.count) {
        count(kSpanQkv, l, h);
        count(kSpanOut, l, h);
      }
    }
    count(kSpanNorm2, l, 0);
    count(kSpanGateUp, l, 0);
    count(kSpanDown, l, 0);
  }
  return n;
}

// Rows, chunk count and rows per chunk of one span of this CTA. The same for
// every layer and head, so computed once per launch (flow_plan) and read from
// shared memory by the phases (the span arithmetic divides by runtime values).
struct FlowSpan {
  int rows, chunks, rpc;
};
struct FlowPlan {
  FlowSpan in, qkv, out, gateup, down;
  int qkv_lo;   // first q/k/v row pair of this rank within the head
};
__device__ inline FlowSpan flow_span(const StepArgs& a, const Where& w, int kind, size_t elem) {
  const int hl = a.heads / a.tp_size;
  const Span s = span_of(a, w, kind, 0, a.tp_rank * hl + (w.id < hl ? w.id : 0), elem);
  const FlowSplit sp = flow_split(s, kind);
  return {s.rows, sp.chunks, sp.rows_per_chunk};
}

// ---------------------------------------------------------------- shared memory
enum FlowMark : int {
  kFmStep = 1, kFmIn, kFmNorm1, kFmQkv, kFmQkvSync, kFmAttn, kFmPartSync, kFmMerge, kFmOut, kFmGather1,
  kFmPub2, kFmNorm2, kFmGateUp, kFmDown, kFmDredSync, kFmDpub, kFmGather2, kFmPub1, kFmScore,
  kFmKvIssue = 20, kFmNormScale = 21, kFmNormGain = 22,  // parts of the first head's norm1
  kFmAcqWait = 24  // not a phase: cycles spent waiting for ring chunks, inside the phases above
};
constexpr int kFlowTags = 32;
constexpr int kFlowFullGather2 = 16384;  // records per CTA up to which exchange 2 gathers the whole width

struct FlowChunk {
  const char* src;
  unsigned bytes;
  unsigned keep;  // 1: L2 evict_last, 0: evict_first
};

struct alignas(128) FlowRing {
  unsigned long long full[kFlowSlots];   // completion of chunk c at c % kFlowSlots
  unsigned long long empty[kFlowSlots];  // release of chunk c (one arrival per warp)
  unsigned off[kFlowSlots];              // buffer offset of that chunk
  unsigned long long end[kFlowSlots];    // allocation position just past it
  unsigned long long head, tail, issued, released, limit;
  unsigned long long keep_policy, stream_policy;
  unsigned char* buf;
  unsigned capacity, head_off;
  int next, nchunks, failed, ok;
  int stop;                              // the compute warps have left; the producer stops issuing
  long long tlast;                       // diagnostics: clock64() of the previous phase mark
  unsigned long long tsum[kFlowTags];    // diagnostics: cycles per phase tag, tsum[0] = steps
  FlowChunk table[kFlowMaxChunks];
};

// Every DSMEM target sits at the same offset in every CTA of the cluster.
// Exchange sites: data every rank of the cluster writes into its peers' shared
// memory with st.async, each store completing its byte count on the
// receiver's mbarrier for the site (no cluster barrier). Every site is double
// buffered by the parity of its exchange count: a sender reaches exchange
// k + 2 of a site only after every receiver has sent its part of exchange
// k + 1, which each does after its last read of exchange k's buffer.
enum FlowSite : int { kSiteX = 0, kSiteQkv = 1, kSiteAtt = 2, kSiteDred = 3, kSites = 4 };

struct alignas(128) FlowSmem {
  unsigned long long sbar[kSites][2];    // receive mbarriers per site and parity
  float x[2][kFlowMaxD];                 // residual entering the layer (site X)
  float x2[kFlowMaxD];                   // residual after attention (every CTA computes all of it)
  float z[kFlowMaxD];                    // norm output, GEMV input
  float dred[2][kFlowMaxD];              // down partials from every rank, [CS][n] (site DRED)
  float seg[kFlowMaxD];                  // this rank's segment values before publishing
  float fnorm[kFlowMaxD];                // final norm gain (score CTA)
  float fscore[kFlowMaxD];               // score weights (score CTA)
  float qkv[2][3 * kFlowHd];             // q, k, v of the current head (site QKV)
  float apart[2][kFlowMaxCluster][kFlowHd + 2];  // CTA attention partials per rank (site ATT)
  float wpart[kWarps][kFlowHd + 2];      // warp attention partials
  float o[kFlowHd];                      // merged attention output (cast)
  float act[kFlowMaxAct];                // this CTA's SwiGLU slice
  float ssx[2][kFlowMaxCluster][8];      // sum of squares of x per rank and warp (site X)
  int okx[2][kFlowMaxCluster];           // verdict per rank (site X)
  int oksetup[kFlowMaxCluster];          // launch setup verdict per rank
  float2 rope_cs[kFlowHd / 2];           // cos, sin of t * frequency
  float rope[kFlowHd / 2];               // frequencies 10000^(-2i/hd)
  float ev[kFlowFeatures];               // the event
  float warp_scratch[kWarps];
  unsigned long long cmd;                // persistent: the dispatched command
  FlowPlan plan;                         // this CTA's span geometry
  union {
    alignas(16) unsigned char kv[kFlowKvBytes];   // K rows then V rows of this CTA's slots
    float red[kFlowKvBytes / 4];                   // gather / down group partials
  } u;
};

// ---------------------------------------------------------------- timeline
// Phase marks of the diagnostic instantiations (kDiag) only: thread 0 of every
// CTA adds the clock64() cycles since its previous mark to fr.tsum[tag], in
// shared memory (tens of cycles per mark), and at the end of every step stores
// the running sums to a.timeline[cta * kFlowTags + tag] (tsum[0] counts the
// steps). The production instantiations contain none of this code.

// Everything off the hot path (error reporting, slow waits) lives in
// functions of its own, called with scalars (a call that took the kernel
// parameters by reference would copy them to local memory).

template <bool kDiag>
__device__ __forceinline__ void fmark(const StepArgs& a, FlowRing& fr, int tag) {
  if constexpr (kDiag) {
    if (threadIdx.x == 0) {
      const long long now = clock64();
      fr.tsum[tag] += (unsigned long long)(now - fr.tlast);
      fr.tlast = now;
      if (tag == kFmScore && a.timeline) {
        fr.tsum[0] += 1;
        for (int i = 0; i < kFlowTags; ++i) a.timeline[blockIdx.x * kFlowTags + i] = (long long)fr.tsum[i];
      }
    }
  }
}

// First error wins; mirrored to the host (set_error with scalars).
static __device__ __noinline__ void flow_error(int* error, int* host_error, int code) {
  if (atomicCAS(error, 0, code) == 0 && host_error) {
    *reinterpret_cast<volatile int*>(host_error) = code;
    __threadfence_system();
  }
}

constexpr size_t kFlowRingOffset = (sizeof(FlowSmem) + sizeof(FlowRing) + 127) / 128 * 128;
constexpr size_t kFlowSmemBytes = kSmemLimit - kStaticSmemReserve;
constexpr unsigned kFlowRingCapacity = (unsigned)((kFlowSmemBytes - kFlowRingOffset) / 128 * 128);
static_assert(kFlowRingCapacity >= 2 * kFlowChunkMax, "the flow ring needs room for two chunks");

// ---------------------------------------------------------------- tagged records
__device__ __forceinline__ unsigned long long ll_pack(float v, unsigned tag) {
  return ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
}
__device__ __forceinline__ void ll_store2(unsigned long long* p, float v0, float v1, unsigned tag) {
  asm volatile("st.relaxed.gpu.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(ll_pack(v0, tag)), "l"(ll_pack(v1, tag))
               : "memory");
}
// Records that cross GPUs (tensor parallelism): system scope, stored through
// the peer's mapping over NVLink; each 8-byte record is single-copy atomic.
__device__ __forceinline__ void ll_store2_sys(unsigned long long* p, float v0, float v1, unsigned tag) {
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(ll_pack(v0, tag)), "l"(ll_pack(v1, tag))
               : "memory");
}
__device__ __forceinline__ void ll_load2(const unsigned long long* p, unsigned long long& r0, unsigned long long& r1) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(r0), "=l"(r1) : "l"(p) : "memory");
}
__device__ __forceinline__ unsigned ll_tag(unsigned long long r) { return (unsigned)(r >> 32); }
__device__ __forceinline__ float ll_value(unsigned long long r) { return __uint_as_float((unsigned)r); }

__device__ __forceinline__ void dsmem_store2(float* local, unsigned rank, float v0, float v1) {
  const unsigned addr = (unsigned)__cvta_generic_to_shared(local);
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(remote), "f"(v0), "f"(v1) : "memory");
}
__device__ __forceinline__ void dsmem_store4(float* local, unsigned rank, float4 v) {
  const unsigned addr = (unsigned)__cvta_generic_to_shared(local);
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// st.async: a store into CTA `rank`'s shared memory at the offset of `local`,
// completing its bytes on that CTA's mbarrier at the offset of `bar`.
__device__ __forceinline__ unsigned flow_remote(const void* local, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"((unsigned)__cvta_generic_to_shared(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_async1(const float* dst, const unsigned long long* bar, unsigned rank, float v) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];"
               ::"r"(flow_remote(dst, rank)), "f"(v), "r"(flow_remote(bar, rank)) : "memory");
}
__device__ __forceinline__ void st_async1i(const int* dst, const unsigned long long* bar, unsigned rank, int v) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
               ::"r"(flow_remote(dst, rank)), "r"(v), "r"(flow_remote(bar, rank)) : "memory");
}
__device__ __forceinline__ void st_async2(const float* dst, const unsigned long long* bar, unsigned rank, float v0,
                                          float v1) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];"
               ::"r"(flow_remote(dst, rank)), "f"(v0), "f"(v1), "r"(flow_remote(bar, rank)) : "memory");
}
__device__ __forceinline__ void st_async4(const float* dst, const unsigned long long* bar, unsigned rank, float4 v) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
               ::"r"(flow_remote(dst, rank)), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(flow_remote(bar, rank))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"((unsigned)__cvta_generic_to_shared(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// ---------------------------------------------------------------- ring
// Compute threads (warps 0-15) meet at named barrier 1; the producer warp
// (warp 16) never joins it, so issuing never holds up a compute phase. The
// non-aligned barrier forms: a warp may reach them diverged (one lane still
// polling while the others wait), which the .aligned forms (bar.sync,
// bar.red) do not allow.
__device__ __forceinline__ void flow_bar() { asm volatile("barrier.sync 1, %0;" ::"n"(kThreads) : "memory"); }
__device__ __forceinline__ bool flow_bar_and(bool p) {
  int r;
  asm volatile(
      "{\n\t.reg .pred a, r;\n\t"
      "setp.ne.u32 a, %1, 0;\n\t"
      "barrier.red.and.pred r, 1, %2, a;\n\t"
      "selp.u32 %0, 1, 0, r;\n\t}"
      : "=r"(r) : "r"((unsigned)p), "n"(kThreads) : "memory");
  return r != 0;
}
__device__ __forceinline__ void flow_bsync(FlowRing&) { flow_bar(); }

// The producer: reclaim the bytes of chunks every compute warp has released,
// then issue the next chunk of the table (cp.async.bulk global -> this CTA's
// shared memory, completion on its full mbarrier, no multicast) as soon as a
// slot and its bytes are free. Leaves when the launch's chunks are issued or
// the compute warps set fr.stop, after waiting for the copies in flight;
// every wait is bounded by wait_ns without progress.
__device__ inline void flow_produce(const StepArgs& a, FlowRing& fr, unsigned long long wait_ns) {
  unsigned long long since = globaltimer();
  while (fr.issued < fr.limit) {
    while (fr.released < fr.issued &&
           mbar_test_wait(&fr.empty[fr.released % kFlowSlots], (unsigned)((fr.released / kFlowSlots) & 1ull))) {
      fr.tail = fr.end[fr.released % kFlowSlots];
      fr.released += 1;
    }
    bool issued = false;
    if (fr.issued < fr.released + kFlowSlots) {
      const FlowChunk c = fr.table[fr.next];
      const unsigned alloc = (c.bytes + 127u) & ~127u;
      unsigned long long pos = fr.head;
      unsigned off = fr.head_off;
      if (off + alloc > fr.capacity) {  // never split a chunk across the end
        pos += fr.capacity - off;
        off = 0;
      }
      if (pos + alloc - fr.tail <= fr.capacity) {
        const int slot = (int)(fr.issued % kFlowSlots);
        fr.off[slot] = off;
        fr.end[slot] = pos + alloc;
        fr.head = pos + alloc;
        fr.head_off = off + alloc == fr.capacity ? 0u : off + alloc;
        mbar_expect_tx(&fr.full[slot], c.bytes);
        bulk_copy(fr.buf + off, c.src, c.bytes, &fr.full[slot], c.keep ? fr.keep_policy : fr.stream_policy);
        fr.next = fr.next + 1 == fr.nchunks ? 0 : fr.next + 1;
        fr.issued += 1;
        issued = true;
      }
    }
    if (issued) {
      since = globaltimer();
      continue;
    }
    if (*reinterpret_cast<volatile int*>(&fr.stop)) break;
    // sleep until the oldest outstanding chunk is released
    mbar_try_wait_for(&fr.empty[fr.released % kFlowSlots], (unsigned)((fr.released / kFlowSlots) & 1ull), 2000u);
    if (globaltimer() - since > wait_ns) {
      flow_error(a.error, a.host_error, kBarrierTimeout);
      break;
    }
  }
  // copies still in flight land before the CTA may leave
  for (unsigned long long c = fr.released; c < fr.issued; ++c) {
    const int slot = (int)(c % kFlowSlots);
    const unsigned parity = (unsigned)((c / kFlowSlots) & 1ull);
    const unsigned long long start = globaltimer();
    while (!mbar_try_wait(&fr.full[slot], parity))
      if (globaltimer() - start > a.bar_timeout_ns) break;
  }
}

// Per-thread consumer position (uniform across the compute warps).
struct FlowCur {
  unsigned long long consumed;
};

static __device__ __noinline__ bool flow_wait_slow(FlowRing& fr, int slot, unsigned parity,
                                                   unsigned long long timeout_ns) {
  const unsigned long long start = globaltimer();
  while (true) {
    if (mbar_try_wait_for(&fr.full[slot], parity, 20000u)) return true;
    if (globaltimer() - start > timeout_ns) return false;
  }
}

// Wait (bounded) for the next chunk; returns its bytes. After a failed wait
// the ring is marked failed and every later acquire returns the start of the
// buffer without waiting (the error word ends the launch at its next exchange).
__device__ __forceinline__ const unsigned char* flow_acquire_plain(const StepArgs& a, FlowRing& fr, const FlowCur& cur) {
  const int slot = (int)(cur.consumed % kFlowSlots);
  const unsigned parity = (unsigned)((cur.consumed / kFlowSlots) & 1ull);
  if (!mbar_try_wait(&fr.full[slot], parity) && !*reinterpret_cast<volatile int*>(&fr.failed) &&
      !flow_wait_slow(fr, slot, parity, a.bar_timeout_ns)) {
    fr.failed = 1;
    flow_error(a.error, a.host_error, kBarrierTimeout);
  }
  return fr.buf + (*reinterpret_cast<volatile int*>(&fr.failed) ? 0u : fr.off[slot]);
}
template <bool kDiag = false>
__device__ __forceinline__ const unsigned char* flow_acquire(const StepArgs& a, FlowRing& fr, const FlowCur& cur) {
  long long t0 = 0;
  if constexpr (kDiag) t0 = clock64();
  const unsigned char* p = flow_acquire_plain(a, fr, cur);
  if constexpr (kDiag)
    if (threadIdx.x == 0) fr.tsum[kFmAcqWait] += (unsigned long long)(clock64() - t0);
  return p;
}

// Every thread of a compute warp, after the warp's last read of the chunk (or
// without reading it): one arrival per warp on its empty mbarrier.
__device__ __forceinline__ void flow_release(FlowRing& fr, FlowCur& cur) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&fr.empty[cur.consumed % kFlowSlots]);
  cur.consumed += 1;
}

// Every thread: the chunk table and mbarriers (built by the producer lane).
// `steps` bounds the chunks issued (0: unbounded). Returns false when the
// table does not fit (the host checks this before choosing the kernel).
__device__ inline bool flow_ring_begin(const StepArgs& a, FlowRing& fr, unsigned char* buf, const Where& w,
                                       size_t elem, unsigned long long steps, unsigned capacity) {
  if (threadIdx.x == kFlowProducer) {
    fr.head = fr.tail = fr.issued = fr.released = 0;
    fr.head_off = 0;
    fr.failed = 0;
    fr.stop = 0;
    fr.keep_policy = policy_evict_last();
    fr.stream_policy = policy_evict_first();
    fr.buf = buf;
    fr.capacity = capacity;
    fr.next = 0;
    int n = 0;
    bool ok = true;
    unsigned keep = 1u;
    auto add = [&](int kind, int l, int h) {
      const Span s = span_of(a, w, kind, l, h, elem);
      const FlowSplit sp = flow_split(s, kind);
      for (int c = 0; c < sp.chunks; ++c) {
        if (n >= kFlowMaxChunks) { ok = false; return; }
        const int r0 = c * sp.rows_per_chunk;
        const int rows = min(sp.rows_per_chunk, s.rows - r0);
        fr.table[n++] = FlowChunk{s.base + (size_t)r0 * s.row_bytes, (unsigned)(rows * s.row_bytes), keep};
      }
    };
    add(kSpanIn, -1, 0);
    const int hl = a.heads / a.tp_size, hb = a.tp_rank * hl;
    for (int l = 0; l < a.layers; ++l) {
      keep = l < a.l2_keep_layers ? 1u : 0u;
      if (w.id < hl) {
        add(kSpanNorm1, l, 0);
        for (int h = hb + w.id; h < hb + hl; h += w.count) {
          add(kSpanQkv, l, h);
          add(kSpanOut, l, h);
        }
      }
      add(kSpanNorm2, l, 0);
      add(kSpanGateUp, l, 0);
      add(kSpanDown, l, 0);
    }
    fr.nchunks = n;
    fr.limit = steps ? steps * (unsigned long long)n : ~0ull;
    fr.ok = ok && n > 0;
    if (fr.ok) {
      for (int i = 0; i < kFlowSlots; ++i) {
        mbar_init(&fr.full[i], 1);
        mbar_init(&fr.empty[i], kWarps);
      }
      fence_mbar_init();
    }
  }
  __syncthreads();
  return fr.ok != 0;
}

// ---------------------------------------------------------------- warp GEMV
// Geometry of rows of K elements of T: 16-byte vectors, LPR lanes per row,
// VPL vectors per lane, RPP row groups per warp pass.
template <typename T, int K>
struct FlowRow {
  static constexpr int V = Storage<T>::kVec;
  static constexpr int NV = K / V;
  static constexpr int LPR = NV < 32 ? NV : 32;
  static constexpr int VPL = NV / LPR;
  static constexpr int RPP = 32 / LPR;
  static_assert(K % V == 0 && (NV & (NV - 1)) == 0 && NV >= 2, "rows must be a power-of-two number of vectors");
};

// The lane's share of a GEMV input vector (shared memory), in registers.
template <typename T, int K>
struct FlowX {
  using R = FlowRow<T, K>;
  float v[R::VPL * R::V];
  __device__ __forceinline__ void load(const float* xs) {
    const int sl = (threadIdx.x & 31) % R::LPR;
#pragma unroll
    for (int k = 0; k < R::VPL; ++k)
#pragma unroll
      for (int e = 0; e < R::V; e += 4) {
        const float4 q = *reinterpret_cast<const float4*>(xs + (sl + R::LPR * k) * R::V + e);
        v[k * R::V + e] = q.x;
        v[k * R::V + e + 1] = q.y;
        v[k * R::V + e + 2] = q.z;
        v[k * R::V + e + 3] = q.w;
      }
  }
};

// Per-lane partial dot products of U consecutive rows (stride K) with x.
template <typename T, int K, int U>
__device__ __forceinline__ void flow_dot(const T* row, int sl, const FlowX<T, K>& x, float (&acc)[U]) {
  using R = FlowRow<T, K>;
  constexpr int B = 4;  // vectors per row in flight
#pragma unroll
  for (int u = 0; u < U; ++u) acc[u] = 0.f;
#pragma unroll
  for (int k0 = 0; k0 < R::VPL; k0 += B) {
    uint4 w[U][B];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int b = 0; b < B; ++b)
        if (k0 + b < R::VPL) w[u][b] = ld_shared_v4(row + (size_t)u * K + (size_t)(sl + R::LPR * (k0 + b)) * R::V);
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int b = 0; b < B; ++b)
        if (k0 + b < R::VPL) acc[u] += dot_regs<T>(w[u][b], x.v + (k0 + b) * R::V);
  }
}

// Rows of span s from the ring, U rows per group; epi(row, v[U]) runs on lane
// 0 of each valid group (row relative to the span). Passes of RPP groups are
// dealt to warps round robin across the span's chunks; a warp without a pass
// in a chunk releases it without waiting.
template <typename T, int K, int U, bool kDiag, class Epi>
__device__ __forceinline__ void flow_rows(const StepArgs& a, FlowRing& fr, FlowCur& cur, const FlowSpan sp,
                                          const FlowX<T, K>& x, Epi&& epi) {
  using R = FlowRow<T, K>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / R::LPR, sl = lane - sub * R::LPR;
  constexpr int pr = U * R::RPP;
  int pass0 = 0;
  for (int c = 0; c < sp.chunks; ++c) {
    const int r0 = c * sp.rpc;
    const int n = min(sp.rpc, sp.rows - r0);
    const int passes = (n + pr - 1) / pr;
    const int first = (warp - pass0 % kWarps + kWarps) % kWarps;
    if (first < passes) {
      const T* base = (const T*)flow_acquire<kDiag>(a, fr, cur);
      for (int p = first; p < passes; p += kWarps) {
        const int row = p * pr + sub * U;
        const bool valid = row < n;
        float acc[U];
        flow_dot<T, K, U>(base + (size_t)(valid ? row : 0) * K, sl, x, acc);
        if constexpr (U == 2) {
          // Halve the shuffles: the upper half-group keeps row 1, the lower row 0.
          constexpr int H = R::LPR / 2;
          const bool hi = (sl & H) != 0;
          const float send = hi ? acc[0] : acc[1];
          float r = (hi ? acc[1] : acc[0]) + __shfl_xor_sync(0xffffffffu, send, H);
#pragma unroll
          for (int o = H / 2; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
          const float r1 = __shfl_down_sync(0xffffffffu, r, H);
          if (valid && sl == 0) {
            const float v[2] = {r, r1};
            epi(r0 + row, v);
          }
        } else {
          float r = acc[0];
#pragma unroll
          for (int o = R::LPR / 2; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
          if (valid && sl == 0) {
            const float v[1] = {r};
            epi(r0 + row, v);
          }
        }
      }
    }
    flow_release(fr, cur);
    pass0 += passes;
  }
}

// A one-row span (a norm gain) read by every thread: g(i) for i < D.
template <typename T, bool kDiag, class Fn>
__device__ __forceinline__ void flow_gain(const StepArgs& a, FlowRing& fr, FlowCur& cur, Fn&& fn) {
  const T* g = (const T*)flow_acquire<kDiag>(a, fr, cur);
  fn(g);
  flow_release(fr, cur);
}

// ---------------------------------------------------------------- exchanges
// Sum over sources src < nsrc of the records rec[src * D + seg0 + i], i < n,
// into sm.seg[i] (threads i < n after the final barrier), sources added in
// index order. Thread t polls element pair t % (n/2) for sources congruent to
// t / (n/2) modulo G = 1024 / n, eight sources per round trip. Returns false
// (error word set) when a wait ran out or another CTA failed.
// Inlined at its two call sites: an out-of-line copy (divergent polling, then
// the named-barrier reductions inside the call) gave nondeterministic results
// on B200, while the inlined form is bit-stable run to run.
__device__ __forceinline__ bool flow_gather_impl(const unsigned long long* rec, int stride, int nsrc, int seg0,
                                                     int n, unsigned tag, float* red, float* seg, int* error,
                                                     int* host_error, unsigned long long timeout_ns) {
  // n is a power of two (D / CS), so the thread split is by shifts.
  const int np = n >> 1, lg = 31 - __clz(np), G = kThreads >> lg;
  const int e = (int)threadIdx.x & (np - 1), g = (int)threadIdx.x >> lg;
  float s0 = 0.f, s1 = 0.f;
  bool ok = true;
  unsigned long long start = 0;
  unsigned polls = 0;
  for (int src0 = g; src0 < nsrc && ok; src0 += 8 * G) {
    unsigned long long r[8][2];
    while (true) {
      bool ready = true;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int src = src0 + k * G;
        if (src < nsrc) {
          ll_load2(rec + (size_t)src * stride + seg0 + 2 * e, r[k][0], r[k][1]);
        } else {
          r[k][0] = r[k][1] = ll_pack(0.f, tag);
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) ready = ready && ll_tag(r[k][0]) == tag && ll_tag(r[k][1]) == tag;
      if (ready) break;
      if ((++polls & 31u) == 0) {
        if (ld_volatile_int(error) != 0) { ok = false; break; }
        const unsigned long long now = globaltimer();
        if (start == 0) start = now;
        else if (now - start > timeout_ns) { flow_error(error, host_error, kBarrierTimeout); ok = false; break; }
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      s0 += ll_value(r[k][0]);
      s1 += ll_value(r[k][1]);
    }
  }
  red[g * n + 2 * e] = s0;
  red[g * n + 2 * e + 1] = s1;
  ok = flow_bar_and(ok);
  if ((int)threadIdx.x < n) {
    float t = 0.f;
    for (int k = 0; k < G; ++k) t += red[k * n + threadIdx.x];
    seg[threadIdx.x] = t;
  }
  flow_bar();
  return ok;
}
template <int D>
__device__ __forceinline__ bool flow_gather(const StepArgs& a, FlowRing&, const unsigned long long* rec, int nsrc,
                                            int seg0, int n, unsigned tag, FlowSmem& sm) {
  return flow_gather_impl(rec, D, nsrc, seg0, n, tag, sm.u.red, sm.seg, a.error, a.host_error, a.bar_timeout_ns);
}

// Every element of x' = cast(x + cast(sum_h P[h])) for the whole width, into
// x2 (local), with sum(x'^2) returned through *ss; heads summed in a fixed
// order. Thread t polls element pair t % (D/2) for heads congruent to t / (D/2).
template <typename T, int D>
__device__ __forceinline__ bool flow_gather_full(const unsigned long long* rec, int nsrc, unsigned tag,
                                                 const float* x, float* x2, float* red, float* scratch, float* ss,
                                                 int* error, int* host_error, unsigned long long timeout_ns) {
  constexpr int np = D / 2, G = kThreads / np;
  const int e = (int)threadIdx.x % np, g = (int)threadIdx.x / np;
  float s0 = 0.f, s1 = 0.f;
  bool ok = true;
  unsigned long long start = 0;
  unsigned polls = 0;
  for (int src0 = g; src0 < nsrc && ok; src0 += 8 * G) {
    unsigned long long r[8][2];
    while (true) {
      bool ready = true;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int src = src0 + k * G;
        if (src < nsrc) ll_load2(rec + (size_t)src * D + 2 * e, r[k][0], r[k][1]);
        else r[k][0] = r[k][1] = ll_pack(0.f, tag);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) ready = ready && ll_tag(r[k][0]) == tag && ll_tag(r[k][1]) == tag;
      if (ready) break;

      if ((++polls & 31u) == 0) {
        if (ld_volatile_int(error) != 0) { ok = false; break; }
        const unsigned long long now = globaltimer();
        if (start == 0) start = now;
        else if (now - start > timeout_ns) { flow_error(error, host_error, kBarrierTimeout); ok = false; break; }
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) { s0 += ll_value(r[k][0]); s1 += ll_value(r[k][1]); }
  }
  red[g * D + 2 * e] = s0;
  red[g * D + 2 * e + 1] = s1;
  ok = flow_bar_and(ok);
  float q = 0.f;
  for (int i = threadIdx.x; i < D; i += kThreads) {
    float t = 0.f;
    for (int k = 0; k < G; ++k) t += red[k * D + i];
    const float v = Storage<T>::round(x[i] + Storage<T>::round(t));
    x2[i] = v;
    q = fmaf(v, v, q);
  }
  q = warp_sum(q);
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = q;
  flow_bar();
  float total = 0.f;
  for (int w = 0; w < kWarps; ++w) total += scratch[w];
  *ss = total;
  return ok;
}

// ---------------------------------------------------------------- step context
struct FlowCtx {
  unsigned rank, cs, id, nc;
  int n, seg0;
  int slot, valid;           // t % W and the retained slot count of the current step
  bool heads_here, score_cluster;
  unsigned long long epoch;  // tag base of this launch
  unsigned long long steps;  // steps this launch has run
  unsigned k[kSites];        // exchanges so far per site (selects buffer and mbarrier phase)
  unsigned bx;               // buffer holding the current x
  float xss;                 // sum(x^2) of the current x when this CTA computed it whole (-1: from the publish)
};

// Bounded wait for an exchange phase that had not completed at the first try.
static __device__ __noinline__ bool flow_receive_slow(unsigned long long* bar, unsigned parity, int* error,
                                                      int* host_error, unsigned long long timeout_ns) {
  const unsigned long long start = globaltimer();
  unsigned polls = 0;
  while (!mbar_try_wait_cluster(bar, parity)) {
    if ((++polls & 63u) == 0 && globaltimer() - start > timeout_ns) {
      flow_error(error, host_error, kBarrierTimeout);
      return false;
    }
  }
  return true;
}

// Receive exchange k of a site: thread 0 arms the site's mbarrier with the
// bytes every rank sends (one arrival), every thread waits for the phase to
// complete (bounded). False when the wait ran out.
__device__ __forceinline__ bool flow_receive_at(unsigned long long* bar, unsigned k, unsigned bytes, int* error,
                                                int* host_error, unsigned long long timeout_ns) {
  const unsigned parity = (k >> 1) & 1u;
  if (threadIdx.x == 0) mbar_expect_tx(bar, bytes);
  return mbar_try_wait_cluster(bar, parity) || flow_receive_slow(bar, parity, error, host_error, timeout_ns);
}
template <class Sm>
__device__ __forceinline__ bool flow_receive(const StepArgs& a, FlowRing& fr, Sm& sm, int site, unsigned k,
                                             unsigned bytes) {
  const bool ok = flow_receive_at(&sm.sbar[site][k & 1u], k, bytes, a.error, a.host_error, a.bar_timeout_ns);
  return ok;
}

// Publish this rank's segment (seg[i], i < n) into dst of every rank, with the
// segment's per-warp sums of squares (ss, [rank][warp]) and this CTA's verdict
// (okv[rank]), then receive every rank's part; returns the cluster's verdict
// (every CTA of the cluster sees the same flags).
static __device__ __noinline__ bool flow_publish_impl(const float* seg, float* dst, float* ss, int* okv,
                                                      unsigned long long* bar, unsigned k, unsigned rank, unsigned cs,
                                                      int seg0, int n, bool ok, int* error, int* host_error,
                                                      unsigned long long timeout_ns) {
  const int np = n >> 1, nw = (np + 31) >> 5, t = (int)threadIdx.x;
  float q = 0.f;
  if (t < np) {
    const float v0 = seg[2 * t], v1 = seg[2 * t + 1];
    for (unsigned r = 0; r < cs; ++r) st_async2(dst + seg0 + 2 * t, bar, r, v0, v1);
    q = v0 * v0 + v1 * v1;
  }
  if (t < nw * 32) {
    q = warp_sum(q);
    if ((t & 31) == 0)
      for (unsigned r = 0; r < cs; ++r) st_async1(&ss[rank * 8 + (t >> 5)], bar, r, q);
  }
  if (t < (int)cs) st_async1i(&okv[rank], bar, (unsigned)t, ok ? 1 : 0);
  bool all = flow_receive_at(bar, k, cs * (unsigned)(4 * n + 4 * nw + 4), error, host_error, timeout_ns);
  for (unsigned r = 0; r < cs; ++r) all = all && (*reinterpret_cast<volatile int*>(&okv[r]) != 0);
  return all;
}

// Publish x (site X) into the site's next buffer, then make it current.
template <class Sm>
__device__ __forceinline__ bool flow_publish(const StepArgs& a, FlowRing& fr, Sm& sm, FlowCtx& cx, bool ok) {
  const unsigned k = cx.k[kSiteX]++;
  const unsigned b = k & 1u;
  const bool all = flow_publish_impl(sm.seg, sm.x[b], &sm.ssx[b][0][0], sm.okx[b], &sm.sbar[kSiteX][b], k, cx.rank,
                                     cx.cs, cx.seg0, cx.n, ok, a.error, a.host_error, a.bar_timeout_ns);
  cx.bx = b;
  return all;
}

// 1 / sqrt(mean(x^2) + eps) from the published per-rank, per-warp sums.
__device__ __forceinline__ float flow_norm_scale(const float (*ss)[8], unsigned cs, int n, int d, float eps) {
  const int nw = ((n >> 1) + 31) >> 5;
  float t = 0.f;
  for (unsigned r = 0; r < cs; ++r)
    for (int w = 0; w < nw; ++w) t += ss[r][w];
  return rsqrtf(t * (1.0f / (float)d) + eps);
}

// ---------------------------------------------------------------- attention
// One head h of layer l: q/k/v rows, attention over the retained slots and
// the out-projection rows of this rank's segment, published as P[h].
// Returns false when a wait ran out (the error word is set; the next
// exchange's verdict ends the launch).
template <typename T, int D, bool kDiag>
__device__ __forceinline__ bool flow_head(const StepArgs& a, FlowRing& fr, FlowCur& cur, FlowSmem& sm,
                                          FlowCtx& cx, int l, int h, unsigned long long t, unsigned tag,
                                          bool first_head) {
  constexpr int hd = kFlowHd;
  const int W = a.window;
  const int slot = cx.slot, valid = cx.valid;
  const size_t head_base = (((size_t)l * a.heads + h) * (size_t)W) * hd;
  T* keys = (T*)a.keys + head_base;
  T* values = (T*)a.values + head_base;
  int j0, j1;
  split(valid, (int)cx.rank, (int)cx.cs, j0, j1);
  // K and V rows of this CTA's slots into shared memory (the slot this step
  // overwrites comes from sm.qkv instead).
  const int nj = j1 - j0;
  const bool kv_smem = 2 * nj * hd * (int)sizeof(T) <= kFlowKvBytes;
  if (kv_smem) {
    constexpr int vpr = hd * (int)sizeof(T) / 16;
    const int vecs = nj * vpr;
    for (int i = threadIdx.x; i < 2 * vecs; i += kThreads) {
      const bool is_v = i >= vecs;
      const int k = is_v ? i - vecs : i;
      if (j0 + k / vpr == slot) continue;
      const char* src = (const char*)(is_v ? values : keys) + (size_t)j0 * hd * sizeof(T) + (size_t)k * 16;
      cp_async16(sm.u.kv + (size_t)i * 16, src);
    }
    cp_async_commit();
  }
  fmark<kDiag>(a, fr, kFmKvIssue);
  if (first_head) {
    const float scale = cx.xss >= 0.f ? rsqrtf(cx.xss * (1.0f / (float)D) + a.epsilon)
                                      : flow_norm_scale(sm.ssx[cx.bx], cx.cs, cx.n, D, a.epsilon);
    const float* x = sm.x[cx.bx];
    fmark<kDiag>(a, fr, kFmNormScale);
    flow_gain<T, kDiag>(a, fr, cur, [&](const T* g) {
      for (int i = threadIdx.x; i < D; i += kThreads) sm.z[i] = Storage<T>::round(x[i] * scale * Storage<T>::load(g, i));
    });
    fmark<kDiag>(a, fr, kFmNormGain);
    flow_bsync(fr);
    fmark<kDiag>(a, fr, kFmNorm1);
  }
  // q, k, v row pairs of this rank, sent into every rank's q/k/v buffer
  const unsigned kq = cx.k[kSiteQkv]++, bq = kq & 1u;
  float* qkv = sm.qkv[bq];
  {
    const unsigned long long* qbar = &sm.sbar[kSiteQkv][bq];
    const int lo = sm.plan.qkv_lo;
    FlowX<T, D> xr;
    xr.load(sm.z);
    flow_rows<T, D, 2, kDiag>(a, fr, cur, sm.plan.qkv, xr,
                       [&](int r, const float (&v)[2]) {
                         const int row = 2 * lo + r;
                         const int which = row / hd, dim = row - which * hd;
                         float v0 = Storage<T>::round(v[0]);
                         float v1 = Storage<T>::round(v[1]);
                         if (which < 2) {
                           const float2 c = sm.rope_cs[dim >> 1];
                           const float r0v = v0 * c.x - v1 * c.y;
                           const float r1v = v0 * c.y + v1 * c.x;
                           v0 = Storage<T>::round(r0v);
                           v1 = Storage<T>::round(r1v);
                         }
                         for (unsigned k = 0; k < cx.cs; ++k) st_async2(&qkv[row], qbar, k, v0, v1);
                         if (which > 0) {
                           T* ring = which == 1 ? keys : values;
                           const size_t at = (size_t)slot * hd + dim;
                           Storage<T>::store(ring, at, v0);
                           Storage<T>::store(ring, at + 1, v1);
                         }
                       });
  }
  fmark<kDiag>(a, fr, kFmQkv);
  // this CTA's K/V copies, then every rank's q/k/v rows
  if (kv_smem) cp_async_wait_all();
  flow_bar();
  bool ok = flow_receive(a, fr, sm, kSiteQkv, kq, 3u * hd * 4u);
  fmark<kDiag>(a, fr, kFmQkvSync);
  // attention over this CTA's slots: an online softmax per warp
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const T* Ks = reinterpret_cast<const T*>(sm.u.kv);
    const T* Vs = Ks + (size_t)nj * hd;
    const float2 q = *reinterpret_cast<const float2*>(&qkv[2 * lane]);
    const float rroot = 1.0f / 8.0f;  // 1 / sqrt(head_dim 64), exact
    float m = -INFINITY, lsum = 0.f, acc0 = 0.f, acc1 = 0.f;
    for (int j = j0 + warp; j < j1; j += kWarps) {
      float k0, k1, v0, v1;
      if (j == slot) {
        k0 = qkv[hd + 2 * lane];
        k1 = qkv[hd + 2 * lane + 1];
        v0 = qkv[2 * hd + 2 * lane];
        v1 = qkv[2 * hd + 2 * lane + 1];
      } else if (kv_smem) {
        k0 = Storage<T>::load(Ks + (size_t)(j - j0) * hd, 2 * lane);
        k1 = Storage<T>::load(Ks + (size_t)(j - j0) * hd, 2 * lane + 1);
        v0 = Storage<T>::load(Vs + (size_t)(j - j0) * hd, 2 * lane);
        v1 = Storage<T>::load(Vs + (size_t)(j - j0) * hd, 2 * lane + 1);
      } else {
        k0 = Storage<T>::load_cg(keys + (size_t)j * hd, 2 * lane);
        k1 = Storage<T>::load_cg(keys + (size_t)j * hd, 2 * lane + 1);
        v0 = Storage<T>::load_cg(values + (size_t)j * hd, 2 * lane);
        v1 = Storage<T>::load_cg(values + (size_t)j * hd, 2 * lane + 1);
      }
      const float s = warp_sum(fmaf(q.y, k1, q.x * k0)) * rroot;
      const float mn = fmaxf(m, s);
      const float c = expf(m - mn);
      const float p = expf(s - mn);
      lsum = fmaf(lsum, c, p);
      acc0 = fmaf(acc0, c, p * v0);
      acc1 = fmaf(acc1, c, p * v1);
      m = mn;
    }
    sm.wpart[warp][2 + 2 * lane] = acc0;
    sm.wpart[warp][3 + 2 * lane] = acc1;
    if (lane == 0) {
      sm.wpart[warp][0] = m;
      sm.wpart[warp][1] = lsum;
    }
  }
  flow_bsync(fr);
  fmark<kDiag>(a, fr, kFmAttn);
  const unsigned ka = cx.k[kSiteAtt]++, ba = ka & 1u;
  float(*apart)[kFlowHd + 2] = sm.apart[ba];
  if (threadIdx.x < 64) {
    // warps 0 and 1: this CTA's partial (M, L, A[dim]) from the 16 warp partials
    const int lane = threadIdx.x & 31, dim = threadIdx.x;
    const float mk = lane < kWarps ? sm.wpart[lane][0] : -INFINITY;
    const float lk = lane < kWarps ? sm.wpart[lane][1] : 0.f;
    const float M = warp_max(lk > 0.f ? mk : -INFINITY);
    const float sk = lk > 0.f ? expf(mk - M) : 0.f;
    const float L = warp_sum(lk * sk);
    float A = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) A = fmaf(sm.wpart[k][2 + dim], __shfl_sync(0xffffffffu, sk, k), A);
    const unsigned long long* abar = &sm.sbar[kSiteAtt][ba];
    for (unsigned r = 0; r < cx.cs; ++r) st_async1(&apart[cx.rank][2 + dim], abar, r, A);
    if (threadIdx.x < cx.cs) st_async2(&apart[cx.rank][0], abar, threadIdx.x, M, L);
  }
  ok = flow_receive(a, fr, sm, kSiteAtt, ka, cx.cs * (unsigned)(4 * hd + 8)) && ok;
  fmark<kDiag>(a, fr, kFmPartSync);
  if (threadIdx.x < 64) {
    // merge the cluster's partials in rank order -> o (cast)
    const int lane = threadIdx.x & 31, dim = threadIdx.x;
    const float mr = lane < (int)cx.cs ? apart[lane][0] : -INFINITY;
    const float lr = lane < (int)cx.cs ? apart[lane][1] : 0.f;
    const float M = warp_max(lr > 0.f ? mr : -INFINITY);
    const float sr = lr > 0.f ? expf(mr - M) : 0.f;
    const float L = warp_sum(lr * sr);
    float A = 0.f;
    for (unsigned r = 0; r < cx.cs; ++r) A = fmaf(apart[r][2 + dim], __shfl_sync(0xffffffffu, sr, r), A);
    sm.o[dim] = Storage<T>::round(__fdividef(A, L));
  }
  flow_bsync(fr);
  fmark<kDiag>(a, fr, kFmMerge);
  // out-projection rows of this rank's segment, published as P[h]
  {
    FlowX<T, hd> xr;
    xr.load(sm.o);
    const size_t at = ((size_t)(tag & 1u) * a.heads + h) * D + cx.seg0;
    // (a failure-path test may withhold this CTA's first layer-0 records)
    const bool drop = (int)blockIdx.x == a.test_drop_cta && l == 0 && cx.steps == 0;
    flow_rows<T, hd, 2, kDiag>(a, fr, cur, sm.plan.out, xr, [&](int r, const float (&v)[2]) {
      if (drop) return;
      if (a.tp_size == 1) {
        ll_store2(a.ll_heads + at + r, v[0], v[1], tag);
      } else {
        // every GPU gathers every head: the record into each GPU's buffer
        for (int g = 0; g < a.tp_size; ++g) ll_store2_sys(a.ll_heads_peer[g] + at + r, v[0], v[1], tag);
      }
    });
  }
  fmark<kDiag>(a, fr, kFmOut);
  return ok;
}

// ---------------------------------------------------------------- one step
// One event through every layer; the score CTA writes the score to score_dst
// (and score_copy when given). Returns the cluster-uniform verdict.
template <typename T, int D, bool kDiag>
__device__ __forceinline__ bool flow_step(const StepArgs& a, FlowRing& fr, FlowCur& cur, FlowSmem& sm, FlowCtx& cx,
                          const float* event, unsigned long long t, float* score_dst, float* score_copy) {
  const int n = cx.n, seg0 = cx.seg0;
  fmark<kDiag>(a, fr, kFmStep);
  cx.slot = (int)(t % (unsigned long long)a.window);
  cx.valid = t + 1 < (unsigned long long)a.window ? (int)(t + 1) : a.window;
  if (threadIdx.x < kFlowFeatures) sm.ev[threadIdx.x] = __ldcv(event + threadIdx.x);
  if (threadIdx.x < kFlowHd / 2) {
    const float angle = (float)t * sm.rope[threadIdx.x];
    sm.rope_cs[threadIdx.x] = make_float2(cosf(angle), sinf(angle));
  }
  flow_bsync(fr);
  // x[seg] = cast(W_in[seg] e)
  {
    FlowX<T, kFlowFeatures> xr;
    xr.load(sm.ev);
    flow_rows<T, kFlowFeatures, 1, kDiag>(a, fr, cur, sm.plan.in, xr,
                                   [&](int r, const float (&v)[1]) { sm.seg[r] = Storage<T>::round(v[0]); });
    flow_bsync(fr);
    if (!flow_publish(a, fr, sm, cx, !fr.failed)) return false;
    cx.xss = -1.f;
    fmark<kDiag>(a, fr, kFmIn);
  }
  for (int l = 0; l < a.layers; ++l) {
    const unsigned tag = (unsigned)(cx.epoch + cx.steps * (unsigned long long)a.layers + (unsigned long long)l + 1ull);
    bool hok = true;
    if (cx.heads_here) {
      const int hl = a.heads / a.tp_size, hb = a.tp_rank * hl;
      for (int h = hb + (int)cx.id; h < hb + hl; h += (int)cx.nc)
        hok = flow_head<T, D, kDiag>(a, fr, cur, sm, cx, l, h, t, tag, h == hb + (int)cx.id) && hok;
    }
    // exchange 1 (whole width, no cluster handoff): x' = cast(x + cast(sum_h P[h]))
    float ssq = 0.f;
    bool ok1;
    {
      const unsigned long long* P = a.ll_heads + (size_t)(tag & 1u) * a.heads * D;
      ok1 = flow_gather_full<T, D>(P, a.heads, tag, sm.x[cx.bx], sm.x2, sm.u.red, sm.warp_scratch, &ssq, a.error,
                                   a.host_error, a.bar_timeout_ns) && hok && !fr.failed;
      fmark<kDiag>(a, fr, kFmGather1);
    }
    // FFN: norm2, gate/up -> SwiGLU, down partial
    bool dok = true;
    {
      const float scale = rsqrtf(ssq * (1.0f / (float)D) + a.epsilon);
      const float* x2 = sm.x2;
      flow_gain<T, kDiag>(a, fr, cur, [&](const T* g) {
        for (int i = threadIdx.x; i < D; i += kThreads)
          sm.z[i] = Storage<T>::round(x2[i] * scale * Storage<T>::load(g, i));
      });
      flow_bsync(fr);
      fmark<kDiag>(a, fr, kFmNorm2);
      FlowX<T, D> xr;
      xr.load(sm.z);
      flow_rows<T, D, 2, kDiag>(a, fr, cur, sm.plan.gateup, xr,
                         [&](int r, const float (&v)[2]) {
                           const float gt = Storage<T>::round(v[0]);
                           const float up = Storage<T>::round(v[1]);
                           sm.act[r >> 1] = Storage<T>::round(__fdividef(gt, 1.0f + expf(-gt)) * up);
                         });
      flow_bsync(fr);
      fmark<kDiag>(a, fr, kFmGateUp);
      // partial[col] = sum_f act[f] W_down^T[f][col]: thread t owns 16-byte
      // column vector t % NVd and rows f = g, g + G2, ... of the slice.
      using R = FlowRow<T, D>;
      constexpr int NVd = R::NV, G2 = kThreads / NVd, V = R::V;
      const int cv = (int)threadIdx.x % NVd, g = (int)threadIdx.x / NVd;
      float acc[V];
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] = 0.f;
      const FlowSpan sp = sm.plan.down;
      for (int c = 0; c < sp.chunks; ++c) {
        const int r0 = c * sp.rpc;
        const int rows = min(sp.rpc, sp.rows - r0);
        const T* base = (const T*)flow_acquire<kDiag>(a, fr, cur);
        int f = ((g - r0) % G2 + G2) % G2;
        for (; f < rows; f += G2) {
          const float av = sm.act[r0 + f];
          float w[V];
          Storage<T>::unpack(ld_shared_v4(base + (size_t)f * D + (size_t)cv * V), w);
#pragma unroll
          for (int k = 0; k < V; ++k) acc[k] = fmaf(w[k], av, acc[k]);
        }
        flow_release(fr, cur);
      }
      fmark<kDiag>(a, fr, kFmDown);
      // sm.u.red was last read by exchange 1, before its publish.
#pragma unroll
      for (int k = 0; k < V; k += 4)
        *reinterpret_cast<float4*>(&sm.u.red[g * D + cv * V + k]) = make_float4(acc[k], acc[k + 1], acc[k + 2], acc[k + 3]);
      flow_bsync(fr);
      // column sums in group order, sent in float4s to the rank owning them
      const unsigned kd = cx.k[kSiteDred]++, bd = kd & 1u;
      float* dred = sm.dred[bd];
      const unsigned long long* dbar = &sm.sbar[kSiteDred][bd];
      for (int c4 = threadIdx.x; c4 < D / 4; c4 += kThreads) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < G2; ++k) {
          const float4 q = *reinterpret_cast<const float4*>(&sm.u.red[k * D + 4 * c4]);
          s.x += q.x; s.y += q.y; s.z += q.z; s.w += q.w;
        }
        const int col = 4 * c4, owner = col / n;
        st_async4(&dred[cx.rank * n + (col - owner * n)], dbar, (unsigned)owner, s);
      }
      dok = flow_receive(a, fr, sm, kSiteDred, kd, cx.cs * (unsigned)n * 4u);
      fmark<kDiag>(a, fr, kFmDredSync);
      // this rank's segment of the cluster partial, ranks added in order
      unsigned long long* Dp = a.ll_clusters + ((size_t)(tag & 1u) * cx.nc + cx.id) * D + seg0;
      if ((int)threadIdx.x < (n >> 1)) {
        const int i = 2 * threadIdx.x;
        float s0 = 0.f, s1 = 0.f;
        for (unsigned r = 0; r < cx.cs; ++r) {
          s0 += dred[r * n + i];
          s1 += dred[r * n + i + 1];
        }
        ll_store2(Dp + i, s0, s1, tag);
      }
      fmark<kDiag>(a, fr, kFmDpub);
    }
    // exchange 2 on one GPU at the Main/Small widths (whole width, no cluster
    // handoff): x = cast(x' + cast(sum_c D[c])) in every CTA, with its sum of
    // squares. Measured on B200: C2 102.6 -> 95.6 us per step; at the Large width
    // (33 clusters x 1024 columns of records per CTA) the segment gather and the
    // cluster publish below stay faster (356 against 370 us).
    if (a.tp_size == 1 && (int)cx.nc * D <= kFlowFullGather2) {
      const unsigned long long* Dq = a.ll_clusters + (size_t)(tag & 1u) * cx.nc * D;
      const unsigned nb = cx.bx ^ 1u;  // the previous layer's x buffer: free in this layer
      float ssn = 0.f;
      const bool ok = flow_gather_full<T, D>(Dq, (int)cx.nc, tag, sm.x2, sm.x[nb], sm.u.red, sm.warp_scratch, &ssn,
                                             a.error, a.host_error, a.bar_timeout_ns) && dok && ok1 && !fr.failed;
      fmark<kDiag>(a, fr, kFmGather2);
      if (cx.score_cluster && (int)threadIdx.x < n) a.hidden[(size_t)l * D + seg0 + threadIdx.x] = sm.x[nb][seg0 + threadIdx.x];
      cx.bx = nb;
      cx.xss = ssn;
      // A CTA whose wait ran out leaves the step here; its cluster peers find out
      // at their next exchange with it (bounded) and every CTA meets at the
      // cluster barrier before the kernel ends.
      if (!ok) return false;
      fmark<kDiag>(a, fr, kFmPub1);
    } else {
      // exchange 2 over several GPUs: x[seg] = cast(x'[seg] + cast(sum_c D[c][seg]))
      const unsigned long long* Dq = a.ll_clusters + (size_t)(tag & 1u) * cx.nc * D;
      bool ok = flow_gather<D>(a, fr, Dq, (int)cx.nc, seg0, n, tag, sm) && dok && ok1;
      if (a.tp_size > 1) {
        // sm.seg holds this GPU's ffn share of the segment; cluster 0 sends it to
        // every GPU, and every rank sums the GPUs' shares in GPU order
        const size_t at = ((size_t)(tag & 1u) * a.tp_size + a.tp_rank) * D + seg0;
        if (cx.id == 0)
          for (int i = 2 * (int)threadIdx.x; i < n; i += 2 * kThreads)
            for (int g = 0; g < a.tp_size; ++g)
              ll_store2_sys(a.ll_xd_peer[g] + at + i, sm.seg[i], sm.seg[i + 1], tag);
        flow_bsync(fr);  // sm.seg is read above before the gather overwrites it
        const unsigned long long* X = a.ll_xd + (size_t)(tag & 1u) * a.tp_size * D;
        ok = flow_gather<D>(a, fr, X, a.tp_size, seg0, n, tag, sm) && ok;
      }
      fmark<kDiag>(a, fr, kFmGather2);
      const float* x2 = sm.x2;
      if ((int)threadIdx.x < n) {
        const float v = Storage<T>::round(x2[seg0 + threadIdx.x] + Storage<T>::round(sm.seg[threadIdx.x]));
        sm.seg[threadIdx.x] = v;
        if (cx.score_cluster) a.hidden[(size_t)l * D + seg0 + threadIdx.x] = v;
      }
      flow_bsync(fr);
      if (!flow_publish(a, fr, sm, cx, ok && !fr.failed)) return false;
      cx.xss = -1.f;
      fmark<kDiag>(a, fr, kFmPub1);
    }
  }
  // final RMSNorm and score head (no cast), by the score CTA
  if (cx.score_cluster && cx.rank == 0) {
    const float scale = cx.xss >= 0.f ? rsqrtf(cx.xss * (1.0f / (float)D) + a.epsilon)
                                      : flow_norm_scale(sm.ssx[cx.bx], cx.cs, n, D, a.epsilon);
    const float* x = sm.x[cx.bx];
    float acc = 0.f;
    for (int i = threadIdx.x; i < D; i += kThreads)
      acc = fmaf(sm.fscore[i], Storage<T>::round(x[i] * scale * sm.fnorm[i]), acc);
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) sm.warp_scratch[threadIdx.x >> 5] = acc;
    flow_bar();
    float total = 0.f;
    for (int w = 0; w < kWarps; ++w) total += sm.warp_scratch[w];
    if (threadIdx.x == 0) {
      *score_dst = total;
      if (score_copy) *score_copy = total;
    }
  }
  fmark<kDiag>(a, fr, kFmScore);
  cx.steps += 1;
  return true;
}

// ---------------------------------------------------------------- kernel
// Trace mode: `count` events from f.inputs, positions derived from the stored
// one plus the event index and stored once at the end. Persistent mode: the
// mailbox worker of k2_persistent (reference src/cuda/Runtime.cu:58-122):
// CTA 0 polls the mapped mailbox, stages the event and publishes each command
// on a tagged control word every CTA polls; the score CTA publishes RUN
// completions; RESET ends with a count of CTAs on the barrier counter.
// The body of the single-stream step kernel: Sm is its shared-memory struct
// (the ring bookkeeping follows it, the ring buffer starts at ring_offset),
// step(a, fr, cur, sm, cx, event, t, score_dst, score_copy) runs one event.
template <typename T, int D, class Sm, class Step>
__device__ __forceinline__ void flow_run(const StepArgs& a, const FlowLaunch& f, unsigned char* flow_raw,
                                         size_t ring_offset, unsigned ring_capacity, Step&& step) {
  Sm& sm = *reinterpret_cast<Sm*>(flow_raw);
  FlowRing& fr = *reinterpret_cast<FlowRing*>(flow_raw + sizeof(Sm));
  if (!cluster_shape_ok(a)) {
    if (f.mode == kFlowPersistent && blockIdx.x == 0) persistent_exit<T>(a, f.p);
    return;
  }
  FlowCtx cx;
  cx.rank = cluster_rank();
  cx.cs = cluster_size();
  cx.id = cluster_id();
  cx.nc = cluster_count();
  cx.n = D / (int)cx.cs;
  cx.seg0 = (int)cx.rank * cx.n;
  cx.heads_here = (int)cx.id < a.heads / a.tp_size;
  cx.score_cluster = cx.id == cx.nc - 1;
  cx.xss = -1.f;
  cx.epoch = ld_cg_u64(a.flow_epoch);
  cx.steps = 0;
  for (int i = 0; i < kSites; ++i) cx.k[i] = 0;
  cx.bx = 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kFlowTags; ++i) fr.tsum[i] = 0;
    fr.tlast = clock64();
  }
  const unsigned long long t0 = ld_cg_u64(a.position);
  for (int i = threadIdx.x; i < kFlowHd / 2; i += kThreads) sm.rope[i] = a.rope_freq[i];
  if (cx.score_cluster && cx.rank == 0)
    for (int i = threadIdx.x; i < D; i += kThreads) {
      sm.fnorm[i] = Storage<T>::load((const T*)a.final_norm, i);
      sm.fscore[i] = Storage<T>::load((const T*)a.score_w, i);
    }
  FlowCur cur{0};
  const Where wh{(int)cx.rank, (int)cx.cs, (int)cx.id, (int)cx.nc};
  if (threadIdx.x == 0) {
    FlowPlan pl;
    pl.in = flow_span(a, wh, kSpanIn, sizeof(T));
    pl.qkv = flow_span(a, wh, kSpanQkv, sizeof(T));
    pl.out = flow_span(a, wh, kSpanOut, sizeof(T));
    pl.gateup = flow_span(a, wh, kSpanGateUp, sizeof(T));
    pl.down = flow_span(a, wh, kSpanDown, sizeof(T));
    int lo, hi;
    split_range(3 * kFlowHd / 2, wh.rank, wh.size, lo, hi);
    pl.qkv_lo = lo;
    sm.plan = pl;
    // one arrival (the receiver's expect_tx) per phase; the peers' st.async
    // stores complete the transaction bytes
    for (int i = 0; i < kSites; ++i) {
      mbar_init(&sm.sbar[i][0], 1);
      mbar_init(&sm.sbar[i][1], 1);
    }
    fence_mbar_init();
  }
  const bool ring_ok = flow_ring_begin(a, fr, flow_raw + ring_offset, wh, sizeof(T),
                                       f.mode == kFlowTrace ? f.count : 0ull, ring_capacity);
  if (!ring_ok && threadIdx.x == 0) flow_error(a.error, a.host_error, kRingTable);
  // every CTA of the cluster learns every rank's setup verdict
  // (the barrier also orders the mbarrier initialisation before any peer's st.async)
  if (threadIdx.x < cx.cs) dsmem_store_u32(&sm.oksetup[cx.rank], threadIdx.x, ring_ok ? 1 : 0);
  cluster_sync();
  bool ok = true;
  for (unsigned k = 0; k < cx.cs; ++k) ok = ok && (*reinterpret_cast<volatile int*>(&sm.oksetup[k]) != 0);
  if (!ok) {  // nothing issued or sent yet
    if (f.mode == kFlowPersistent && blockIdx.x == 0 && threadIdx.x < kThreads) persistent_exit<T>(a, f.p);
    return;
  }

  // One command loop for both modes, so the step is inlined at a single call
  // site (a call that takes the kernel parameters by reference would copy them
  // to local memory). Trace mode: RUN for each of f.count events. Persistent
  // mode: CTA 0 polls the mailbox and publishes each command on the tagged
  // control word.
  const bool trace = f.mode == kFlowTrace;
  const PersistArgs& p = f.p;
  unsigned long long previous = p.initial_sequence, dispatched = 0, processed = 0, counts = 0;
  if (threadIdx.x >= kThreads) {
    // the producer warp: lane 0 streams the weights until the compute warps leave
    if (threadIdx.x == kFlowProducer)
      flow_produce(a, fr, trace ? a.bar_timeout_ns : p.idle_ns + p.dispatch_timeout_ns + a.bar_timeout_ns);
    __syncwarp();
  }
  bool exit_loop = threadIdx.x >= kThreads;
  while (!exit_loop) {
    int command, arg = -1;
    if (trace) {
      command = processed < f.count ? kRun : kFlowExit;
    } else {
      if (blockIdx.x == 0 && threadIdx.x < 32) {
        // warp 0 of CTA 0: lane 0 polls the mailbox, the warp stages the event
        // (one mapped read per lane, in parallel), lane 0 publishes the command
        const int lane = threadIdx.x;
        unsigned long long seq = 0;
        int cmd = 0, carg = 0;
        if (lane == 0) {
          const unsigned long long start = globaltimer();
          while ((seq = ld_acquire_sys(&p.mailbox->request)) == previous) {
            if (globaltimer() - start >= p.idle_ns) { cmd = kFlowExit; break; }
            if (p.backoff) __nanosleep(128);
          }
        }
        cmd = __shfl_sync(0xffffffffu, cmd, 0);
        if (cmd == 0) {
          // a request arrived: its input (one float per lane), command and
          // argument are read together, one round trip over the host link
          static_assert(kFlowFeatures == 32, "one input feature per lane");
          const float v = __ldcv(f.mapped_input + lane);
          if (lane == 0) {
            cmd = *reinterpret_cast<volatile int*>(&p.mailbox->command);
            carg = *reinterpret_cast<volatile int*>(&p.mailbox->arg);
          }
          cmd = __shfl_sync(0xffffffffu, cmd, 0);
          if (cmd == kRun) const_cast<float*>(a.input)[lane] = v;
        }
        __syncwarp();
        if (lane == 0) {
          if (cmd != kFlowExit) {
            *a.flow_seq = seq;
            previous = seq;
          }
          const unsigned long long word = ((dispatched + 1ull) << 32) |
                                          ((unsigned long long)(unsigned)(carg + 1) << 8) | (unsigned long long)cmd;
          __threadfence();
          asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(a.flow_ctl), "l"(word) : "memory");
        }
      }
      if (threadIdx.x == 0) {
        const unsigned long long want = dispatched + 1ull;
        const unsigned long long start = globaltimer();
        unsigned long long w;
        unsigned polls = 0;
        while (((w = ld_acquire_gpu(a.flow_ctl)) >> 32) != (want & 0xffffffffull)) {
          if ((++polls & 63u) == 0) {
            if (ld_volatile_int(a.error) != 0) { w = kFlowExit; break; }
            if (globaltimer() - start > p.dispatch_timeout_ns) {
              flow_error(a.error, a.host_error, kBarrierTimeout);
              w = kFlowExit;
              break;
            }
          }
        }
        sm.cmd = w;
      }
      flow_bar();
      const unsigned long long word = *reinterpret_cast<volatile unsigned long long*>(&sm.cmd);
      command = (int)(word & 0xffull);
      arg = (int)((word >> 8) & 0xffffffull) - 1;
      dispatched += 1;
    }
    if (command == kRun) {
      const unsigned long long t = trace ? t0 + processed : ld_cg_u64(a.position);
      const float* event = trace ? f.inputs + processed * kFlowFeatures : a.input;
      float* copy = trace && f.scores ? f.scores + processed : nullptr;
      if (!step(a, fr, cur, sm, cx, event, t, a.score, copy)) {
        ok = false;
        break;
      }
      processed += 1;
      if (!trace) {
        if (cx.score_cluster && cx.rank == 0 && threadIdx.x == 0) {
          a.position[0] = t + 1;
          const unsigned long long seq = ld_cg_u64(a.flow_seq);
          __threadfence_system();
          st_release_sys(&p.mailbox->completion, seq);
        }
        if (p.max_events && processed >= p.max_events) exit_loop = true;
      }
    } else if (command == kReset || command == kPing) {
      // Every CTA takes the command before CTA 0 completes it, so the control
      // word is not rewritten while a CTA has yet to read it.
      if (command == kReset) reset_streams<T>(a, 0, 1);  // one stream: arg -1 and 0 both reset it
      (void)arg;
      flow_bar();
      counts += 1;
      if (threadIdx.x == 0) {
        __threadfence();
        red_release_gpu_add(a.bar_counter, 1ull);
      }
      if (blockIdx.x == 0 && threadIdx.x == 0) {
        const unsigned long long target = f.bar_base + counts * gridDim.x;
        const unsigned long long start = globaltimer();
        bool good = true;
        while (ld_acquire_gpu(a.bar_counter) < target)
          if (globaltimer() - start > a.bar_timeout_ns) { flow_error(a.error, a.host_error, kBarrierTimeout); good = false; break; }
        if (good) {
          if (command == kPing) {
            unsigned long long checksum = 0;
            for (int i = 0; i < a.features; ++i) checksum += __float_as_uint(__ldcv(f.mapped_input + i));
            *reinterpret_cast<volatile unsigned long long*>(&p.mailbox->checksum) = checksum;
          }
          const unsigned long long seq = ld_cg_u64(a.flow_seq);
          __threadfence_system();
          st_release_sys(&p.mailbox->completion, seq);
        }
      }
    } else if (command == kStop) {
      if (blockIdx.x == 0 && threadIdx.x == 0) {
        const unsigned long long seq = ld_cg_u64(a.flow_seq);
        __threadfence_system();
        st_release_sys(&p.mailbox->completion, seq);
      }
      exit_loop = true;
    } else {
      exit_loop = true;  // end of the trace, idle budget, error or an unknown command
    }
  }
  if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(&fr.stop) = 1;
  // No CTA leaves while a peer may still store into its shared memory, or
  // before its producer has seen its copies land (the cluster barrier is the
  // aligned form: every warp reconverges first).
  __syncwarp();
  cluster_sync();
  if (threadIdx.x >= kThreads) return;
  if (trace) {
    if (ok && cx.score_cluster && cx.rank == 0 && threadIdx.x == 0) {
      a.position[0] = t0 + f.count;
      *a.flow_epoch = cx.epoch + f.count * (unsigned long long)a.layers;
    }
    return;
  }
  // Persistent: every CTA counts itself out; CTA 0 then stores the tag base
  // for the next launch and tells the host.
  if (threadIdx.x == 0) {
    __threadfence();
    red_release_gpu_add(a.bar_counter, 1ull);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const unsigned long long target = f.bar_base + (counts + 1ull) * gridDim.x;
    const unsigned long long start = globaltimer();
    while (ld_acquire_gpu(a.bar_counter) < target)
      if (globaltimer() - start > a.bar_timeout_ns) { flow_error(a.error, a.host_error, kBarrierTimeout); break; }
    *a.flow_epoch = cx.epoch + processed * (unsigned long long)a.layers;
  }
  if (blockIdx.x == 0) persistent_exit<T>(a, p);
}

template <typename T, int D, bool kDiag>
__global__ void __launch_bounds__(kFlowThreads, 1) k4_flow(StepArgs a, FlowLaunch f) {
  extern __shared__ __align__(128) unsigned char flow_raw[];
  flow_run<T, D, FlowSmem>(a, f, flow_raw, kFlowRingOffset, kFlowRingCapacity,
                           [](const StepArgs& a, FlowRing& fr, FlowCur& cur, FlowSmem& sm, FlowCtx& cx,
                              const float* event, unsigned long long t, float* dst, float* copy) {
                             return flow_step<T, D, kDiag>(a, fr, cur, sm, cx, event, t, dst, copy);
                           });
}

}  // namespace st
