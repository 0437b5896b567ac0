// st_ring.cuh -- weight streaming through a shared-memory ring fed by bulk copies.
//
// Every weight byte a CTA needs in a step is one of a fixed sequence of spans
// (contiguous row ranges of the slab), identical every step:
//   IN      this CTA's share of W_in rows (its cluster splits the rows)
//   per layer l:
//     NORM1(l)                      only in clusters that own a head
//     QKV(l, h), OUT(l, h)          for each head h the cluster owns
//     NORM2(l), GATEUP(l), DOWN(l)  this CTA's ffn slice
// Spans are cut into chunks of whole rows (at most kChunkBytes each) and the
// per-step chunk list is tabulated once per launch. The ring is a byte buffer:
// chunks are packed back to back (128-byte aligned, never split across the
// end), so a 2 KB norm vector occupies 2 KB, and up to kRingChunks chunks are
// in flight. One thread (the issuer) issues chunk c with cp.async.bulk (global
// -> this CTA's shared memory, completion on mbarrier c % kRingChunks; no
// multicast) as soon as both an mbarrier and enough free bytes are available,
// so while the CTA works or waits at a grid barrier the next chunks, up to the
// ring's capacity, are landing. Consumers walk the same sequence: every warp
// waits on the chunk's full mbarrier (bounded), computes its share from shared
// memory and arrives on the chunk's empty mbarrier (one arrival per warp), so
// warps move from chunk to chunk without a CTA-wide barrier. The issuer
// reclaims the bytes of chunks whose empty phase has completed whenever it
// issues.
//
// Every step reads every weight once, and the fp32 models are about as large
// as L2, so plain copies would flush L2 each step (code and the K/V cache
// included). Chunks of the first a.l2_keep_layers layers are copied with an
// L2 evict_last policy and stay resident from step to step; the rest use
// evict_first and pass through without displacing them.
//
// The issuer is lane 0 of the CTA's last warp (kIssuer). A launch issues at
// most `limit` chunks (fused and trace kernels: exactly
// the chunks their steps consume; the resident kernel keeps prefetching the
// next step) and drains every outstanding copy before any exit, so no bulk
// copy can land after its CTA has left.
#pragma once

#include "st_device.cuh"

namespace st {

constexpr int kRingChunks = 16;            // chunks in flight at most (one mbarrier each)
constexpr int kChunkBytes = 32 * 1024;     // largest chunk
constexpr int kMaxRingChunkTable = 512;    // chunks per step one CTA may consume
// The issuing thread: lane 0 of the last warp. GEMV chunks hand row groups to
// the low warps first, so the issuer's warp is the one most often idle.
constexpr int kIssuer = kThreads - 32;

__device__ __forceinline__ unsigned smem_addr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Same, with a bound (ns) on how long the thread may be suspended waiting.
__device__ __forceinline__ bool mbar_try_wait_for(unsigned long long* bar, unsigned parity, unsigned suspend_ns) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity), "r"(suspend_ns) : "memory");
  return ok != 0;
}
// Bulk copy global -> this CTA's shared memory with an L2 eviction policy
// (from createpolicy); completion on `bar`. No multicast.
__device__ __forceinline__ void bulk_copy(void* dst_smem, const void* src, unsigned bytes, unsigned long long* bar,
                                          unsigned long long policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      :: "r"(smem_addr(dst_smem)), "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy) : "memory");
}
// L2 policies for weight chunks: layers that should stay resident across
// steps, and the rest, streamed once per step without displacing them.
__device__ __forceinline__ unsigned long long policy_evict_last() {
  unsigned long long p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ unsigned long long policy_evict_first() {
  unsigned long long p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_addr(bar)) : "memory");
}
// Non-blocking test of phase completion.
__device__ __forceinline__ bool mbar_test_wait(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
  return ok != 0;
}

enum SpanKind : int { kSpanIn = 0, kSpanNorm1, kSpanQkv, kSpanOut, kSpanNorm2, kSpanGateUp, kSpanDown, kSpanEnd };

struct Span {
  const char* base;   // first byte of row 0 of the span
  int rows;
  int row_bytes;
  int unit;           // rows per epilogue group (chunks hold whole groups)
};

// Position of this CTA in the grid, for span arithmetic.
struct Where {
  int rank, size, id, count;
};

__host__ __device__ __forceinline__ void split_range(int units, int part, int parts, int& lo, int& hi) {
  lo = (int)(((long long)units * part) / parts);
  hi = (int)(((long long)units * (part + 1)) / parts);
}

// Rows of a chunk: as many as fit kChunkBytes, a multiple of `unit` (2 for
// the QKV and gate/up spans, whose epilogues take row pairs).
__host__ __device__ __forceinline__ int rows_per_chunk(int row_bytes, int unit) {
  return row_bytes * unit > kChunkBytes ? 0 : kChunkBytes / row_bytes / unit * unit;
}
__host__ __device__ __forceinline__ int span_unit(int kind) { return kind == kSpanQkv || kind == kSpanGateUp ? 2 : 1; }

// Span `kind` of layer l (see header); `head` selects the head of QKV/OUT.
__host__ __device__ inline Span span_of(const StepArgs& a, const Where& w, int kind, int l, int head, size_t elem) {
  const int d = a.width, hd = a.head_dim, F = a.ffn;
  const LayerPtrs& L = a.layer[l < 0 ? 0 : l];
  Span s{nullptr, 0, 0, span_unit(kind)};
  int lo, hi;
  switch (kind) {
    case kSpanIn:
      split_range(d, w.rank, w.size, lo, hi);
      s.row_bytes = (int)(a.features * elem);
      s.base = (const char*)a.input_w + (size_t)lo * s.row_bytes;
      s.rows = hi - lo;
      break;
    case kSpanNorm1:
      s = {(const char*)L.norm1, 1, (int)(d * elem), 1};
      break;
    case kSpanNorm2:
      s = {(const char*)L.norm2, 1, (int)(d * elem), 1};
      break;
    case kSpanQkv:
      split_range(3 * hd / 2, w.rank, w.size, lo, hi);
      s.row_bytes = (int)(d * elem);
      s.base = (const char*)L.qkv + ((size_t)head * 3 * hd + 2 * (size_t)lo) * s.row_bytes;
      s.rows = 2 * (hi - lo);
      break;
    case kSpanOut:
      split_range(d, w.rank, w.size, lo, hi);
      s.row_bytes = (int)(hd * elem);
      s.base = (const char*)L.out + ((size_t)head * d + lo) * s.row_bytes;
      s.rows = hi - lo;
      break;
    case kSpanGateUp: {
      // this GPU's ffn shard (all of F without tensor parallelism), split over its CTAs
      const int tps = a.tp_size > 0 ? a.tp_size : 1, fl = F / tps, fb = a.tp_rank * fl;
      split_range(fl, w.id * w.size + w.rank, w.count * w.size, lo, hi);
      lo += fb;
      hi += fb;
      s.row_bytes = (int)(d * elem);
      s.base = (const char*)L.gateup + 2 * (size_t)lo * s.row_bytes;
      s.rows = 2 * (hi - lo);
    }
      break;
    case kSpanDown: {
      // this GPU's ffn shard (all of F without tensor parallelism), split over its CTAs
      const int tps = a.tp_size > 0 ? a.tp_size : 1, fl = F / tps, fb = a.tp_rank * fl;
      split_range(fl, w.id * w.size + w.rank, w.count * w.size, lo, hi);
      lo += fb;
      hi += fb;
      s.row_bytes = (int)(d * elem);
      s.base = (const char*)L.down + (size_t)lo * s.row_bytes;
      s.rows = hi - lo;
    }
      break;
    default:
      break;
  }
  return s;
}


// Chunks one step consumes for CTA position w.
__host__ __device__ inline unsigned long long chunks_per_step(const StepArgs& a, const Where& w, size_t elem) {
  unsigned long long n = 0;
  auto count = [&](const Span& s) {
    if (s.rows <= 0) return;
    const int rpc = rows_per_chunk(s.row_bytes, s.unit);
    n += (unsigned long long)((s.rows + rpc - 1) / rpc);
  };
  count(span_of(a, w, kSpanIn, -1, 0, elem));
  for (int l = 0; l < a.layers; ++l) {
    if (w.id < a.heads) {
      count(span_of(a, w, kSpanNorm1, l, 0, elem));
      for (int h = w.id; h < a.heads; h += w.count) {
        count(span_of(a, w, kSpanQkv, l, h, elem));
        count(span_of(a, w, kSpanOut, l, h, elem));
      }
    }
    count(span_of(a, w, kSpanNorm2, l, 0, elem));
    count(span_of(a, w, kSpanGateUp, l, 0, elem));
    count(span_of(a, w, kSpanDown, l, 0, elem));
  }
  return n;
}

// True when every span of this configuration can be moved by bulk copies
// (16-byte aligned rows, a row pair fits a chunk) and every CTA's chunk list
// fits the table, for a grid of `clusters` clusters of `cluster_size` CTAs.
// The host decides with this before choosing the ring kernels.
__host__ __device__ inline bool ring_supported(const StepArgs& a, size_t elem, int cluster_size, int clusters) {
  const size_t rb[3] = {a.width * elem, a.features * elem, a.head_dim * elem};
  for (size_t b : rb)
    if (b % 16 != 0 || 2 * b > (size_t)kChunkBytes) return false;
  for (int id = 0; id < clusters; ++id)
    for (int rank = 0; rank < cluster_size; ++rank)
      if (chunks_per_step(a, Where{rank, cluster_size, id, clusters}, elem) > (unsigned long long)kMaxRingChunkTable)
        return false;
  return true;
}

struct RingChunk {
  const char* src;
  unsigned bytes;
  unsigned keep;  // 1: L2 evict_last (the layer stays resident), 0: evict_first
};

// Per-thread ring state (uniform across the CTA).
struct Ring {
  bool enabled;
  unsigned long long consumed;  // chunks consumed
  __device__ void set_enabled(bool e) { enabled = e; }
};

// Shared-memory header of the ring; the byte buffer lies elsewhere in the
// CTA's shared memory (`buf`). Apart from the mbarriers and `off`, which every
// thread reads, the fields are the issuer's.
struct alignas(128) RingSmem {
  unsigned long long full[kRingChunks];  // completion mbarrier of chunk c at c % kRingChunks
  unsigned long long empty[kRingChunks]; // release mbarrier of chunk c (kWarps arrivals)
  unsigned off[kRingChunks];             // buffer offset of that chunk's bytes
  unsigned long long end[kRingChunks];   // allocation position just past that chunk
  long long issued_at[kRingChunks];      // clock64() when the chunk was issued (diagnostics)
  unsigned long long head;               // bytes allocated so far (monotonic, includes wrap padding)
  unsigned long long tail;               // bytes released so far
  unsigned long long issued;             // chunks issued
  unsigned long long released;           // chunks whose bytes have been reclaimed
  unsigned long long limit;              // chunks this launch may issue
  unsigned char* buf;                    // the ring bytes (128-byte aligned)
  unsigned long long keep_policy;        // createpolicy L2::evict_last
  unsigned long long stream_policy;      // createpolicy L2::evict_first
  unsigned capacity;                     // ring bytes
  unsigned head_off;                     // head % capacity
  int failed;                            // a wait timed out; acquires no longer wait
  int nchunks;                           // chunks per step in `table`
  int next;                              // table index of the next chunk to issue
  RingChunk table[kMaxRingChunkTable];
};

// The issuer: the step's chunks in consumption order (empty spans dropped).
// Returns false when the table would overflow (the ring then stays off).
__device__ inline bool build_chunk_table(const StepArgs& a, const Where& w, size_t elem, RingSmem& rs) {
  int n = 0;
  bool ok = true;
  unsigned keep = 1u;
  auto add = [&](const Span& s) {
    if (s.rows <= 0) return;
    const int rpc = rows_per_chunk(s.row_bytes, s.unit);
    for (int r = 0; r < s.rows; r += rpc) {
      if (n >= kMaxRingChunkTable) { ok = false; return; }
      const int rows = min(rpc, s.rows - r);
      rs.table[n++] = RingChunk{s.base + (size_t)r * s.row_bytes, (unsigned)(rows * s.row_bytes), keep};
    }
  };
  add(span_of(a, w, kSpanIn, -1, 0, elem));
  for (int l = 0; l < a.layers; ++l) {
    keep = l < a.l2_keep_layers ? 1u : 0u;
    if (w.id < a.heads) {
      add(span_of(a, w, kSpanNorm1, l, 0, elem));
      for (int h = w.id; h < a.heads; h += w.count) {
        add(span_of(a, w, kSpanQkv, l, h, elem));
        add(span_of(a, w, kSpanOut, l, h, elem));
      }
    }
    add(span_of(a, w, kSpanNorm2, l, 0, elem));
    add(span_of(a, w, kSpanGateUp, l, 0, elem));
    add(span_of(a, w, kSpanDown, l, 0, elem));
  }
  rs.nchunks = n;
  return ok && n > 0;
}

// The issuer: reclaim the bytes of chunks every warp has released, then issue
// chunks while an mbarrier pair and enough free bytes are available and the
// launch limit allows. Every warp read its share of a released chunk before
// arriving on its empty mbarrier (release semantics), and the test below
// observes that arrival (acquire), so a copy into those bytes cannot race a
// reader.
static __device__ __noinline__ void ring_fill_slow(Ring& r, RingSmem& rs, int max_issue) {
  while (rs.released < rs.issued &&
         mbar_test_wait(&rs.empty[rs.released % kRingChunks], (unsigned)((rs.released / kRingChunks) & 1ull))) {
    rs.tail = rs.end[rs.released % kRingChunks];
    rs.released += 1;
  }
  for (int n = 0; n < max_issue && rs.issued < rs.limit && rs.issued < rs.released + kRingChunks; ++n) {
    const RingChunk c = rs.table[rs.next];
    const unsigned alloc = (c.bytes + 127u) & ~127u;
    unsigned long long pos = rs.head;
    unsigned off = rs.head_off;  // == head % capacity, tracked to avoid a 64-bit modulo
    if (off + alloc > rs.capacity) {  // never split a chunk across the end
      pos += rs.capacity - off;
      off = 0;
    }
    if (pos + alloc - rs.tail > rs.capacity) return;  // not enough free bytes yet
    const int slot = (int)(rs.issued % kRingChunks);
    rs.off[slot] = off;
    rs.end[slot] = pos + alloc;
    rs.head = pos + alloc;
    rs.head_off = off + alloc == rs.capacity ? 0u : off + alloc;
    rs.issued_at[slot] = clock64();
    mbar_expect_tx(&rs.full[slot], c.bytes);
    bulk_copy(rs.buf + off, c.src, c.bytes, &rs.full[slot], c.keep ? rs.keep_policy : rs.stream_policy);
    rs.next = rs.next + 1 == rs.nchunks ? 0 : rs.next + 1;  // the next step repeats the table
    rs.issued += 1;
  }
}

// Out of line: only the issuer runs it. `max_issue` bounds the copies issued
// in one call: one where the issuer's warp has work waiting (a release), all
// that fit where the CTA is idle anyway (a grid barrier).
__device__ __forceinline__ void ring_fill(Ring& r, RingSmem& rs, int max_issue = 1) {
  if (threadIdx.x == kIssuer && r.enabled) ring_fill_slow(r, rs, max_issue);
}
constexpr int kFillAll = kRingChunks;

// All threads: set up (mbarriers, chunk table, first issues). `buf` holds
// `capacity` bytes (a multiple of 128, at least two chunks, so a chunk that
// wraps always fits once the ring has drained); `limit` bounds the chunks
// issued.
__device__ inline void ring_begin(const StepArgs& a, Ring& r, RingSmem& rs, unsigned char* buf, unsigned capacity,
                                  const Where& w, size_t elem, unsigned long long limit, bool enabled) {
  r.consumed = 0;
  __shared__ int table_ok;
  if (threadIdx.x == kIssuer) {
    rs.head = rs.tail = rs.issued = rs.released = 0;
    rs.head_off = 0;
    rs.failed = 0;
    rs.keep_policy = policy_evict_last();
    rs.stream_policy = policy_evict_first();
    rs.limit = limit;
    rs.buf = buf;
    rs.capacity = capacity;
    rs.next = 0;
    for (int i = 0; i < kRingChunks; ++i) rs.off[i] = 0;
    table_ok = enabled && capacity >= 2u * kChunkBytes && build_chunk_table(a, w, elem, rs);
    if (table_ok) {
      for (int i = 0; i < kRingChunks; ++i) {
        mbar_init(&rs.full[i], 1);
        mbar_init(&rs.empty[i], kWarps);
      }
      fence_mbar_init();
    }
  }
  __syncthreads();
  r.set_enabled(table_ok != 0);
  ring_fill(r, rs, kFillAll);
}

// Wait (bounded) until the next chunk has landed; returns its bytes. The
// issuer keeps issuing while it waits (the chunk may not have had room yet)
// and so sleeps only briefly; other threads sleep until the copy completes.
// Out of line (scalars only, so the kernel parameters keep no address): the
// bounded wait of ring_acquire. Returns false when the bound ran out.
static __device__ __noinline__ bool ring_wait_slow(Ring& r, RingSmem& rs, int slot, unsigned parity,
                                            unsigned long long timeout_ns) {
  const bool issuer = threadIdx.x == kIssuer;
  const unsigned long long start = globaltimer();
  while (true) {
    ring_fill(r, rs);
    if (mbar_try_wait_for(&rs.full[slot], parity, issuer ? 200u : 20000u)) return true;
    if (globaltimer() - start > timeout_ns) return false;
  }
}

// After a timed-out wait the slot may never have been issued in this launch
// (its offset is whatever the previous use left), so the ring is marked
// failed (later acquires stop waiting; the error word ends the launch at its
// next grid barrier) and every acquire from then on returns the start of the
// ring, which holds a full chunk. A completed wait returns the offset the
// issuer stored for the chunk, which never crosses the end of the ring.
__device__ __forceinline__ const unsigned char* ring_acquire(const StepArgs& a, Ring& r, RingSmem& rs) {
  const int slot = (int)(r.consumed % kRingChunks);
  const unsigned parity = (unsigned)((r.consumed / kRingChunks) & 1ull);
  if (!mbar_try_wait(&rs.full[slot], parity) && !*reinterpret_cast<volatile int*>(&rs.failed) &&
      !ring_wait_slow(r, rs, slot, parity, a.bar_timeout_ns)) {
    rs.failed = 1;
    if (threadIdx.x == kIssuer) set_error(a, kBarrierTimeout);
  }
  return rs.buf + (*reinterpret_cast<volatile int*>(&rs.failed) ? 0u : rs.off[slot]);
}

// Every thread of a warp, after the warp's last read of the chunk: one
// arrival per warp on the chunk's empty mbarrier.
__device__ inline void ring_release(Ring& r, RingSmem& rs) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&rs.empty[r.consumed % kRingChunks]);
  r.consumed += 1;
  ring_fill(r, rs);
}

// Wait for every issued copy (bounded); call before any exit of the kernel.
__device__ inline void ring_drain(const StepArgs& a, Ring& r, RingSmem& rs) {
  if (!r.enabled) return;
  if (threadIdx.x == kIssuer) {
    for (unsigned long long c = r.consumed; c < rs.issued; ++c) {
      const int slot = (int)(c % kRingChunks);
      const unsigned parity = (unsigned)((c / kRingChunks) & 1ull);
      const unsigned long long start = globaltimer();
      while (!mbar_try_wait(&rs.full[slot], parity))
        if (globaltimer() - start > a.bar_timeout_ns) break;
    }
  }
  __syncthreads();
}

}  // namespace st
