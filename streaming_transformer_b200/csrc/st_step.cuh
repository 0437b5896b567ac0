// st_step.cuh -- the streaming step, organised around thread-block clusters.
//
// Measured on B200: a grid-wide barrier costs ~1.3 us, a hardware cluster
// barrier ~0.24 us and a 512-thread __syncthreads ~0.06 us, so a step is built
// from two grid-wide dependencies per layer, cheap cluster-local exchanges
// (DSMEM) and as few CTA barriers as the data flow allows. The grid is NC
// clusters of CS CTAs (CS = 8 at full size). Per layer:
//
//  attention block (cluster c owns heads c, c + NC, ...; other clusters idle)
//    z = norm1(x)                      every CTA, from its shared-memory copy of x
//    q,k,v rows of head h              row pairs split over the cluster's CTAs, one
//                                      warp per pair; RoPE + cast in the warp's
//                                      epilogue; values broadcast to every CTA of the
//                                      cluster through DSMEM; k, v stored to slot t % W
//    cluster barrier
//    attention over [0, valid)         slots split over the cluster; every warp keeps
//                                      an online-softmax partial (m, l, acc) over its
//                                      slots (K, V rows prefetched into shared memory
//                                      with cp.async while the projections run); the
//                                      CTA merges its warps and broadcasts (m, l, acc)
//    cluster barrier
//    merge -> attn_h (cast); out-projection K-split by head: P[h] = W_out[:, h] attn_h,
//                                      output rows split over the cluster -> global
//  grid sync A
//  FFN block (every CTA)
//    x' = cast(x + cast(sum_h P[h]))   redundantly, heads summed in a fixed order
//    z = norm2(x'); gate/up row pairs of this CTA's ffn slice -> act = cast(silu(g) u)
//    down-projection K-split over the slice (W_down stored transposed, [F][d]):
//                                      partial d-vector, reduce-scattered inside the
//                                      cluster through DSMEM -> D[cluster] -> global
//  grid sync B
//    x = cast(x' + cast(sum_c D[c]))   redundantly, clusters summed in a fixed order
//
// GEMVs: one warp (or a power-of-two lane group for short rows) computes a row
// or a row pair completely -- lanes over 16-byte vectors, a butterfly over the
// group -- so the epilogue runs in the same warp with no CTA barrier. With the
// weight ring (kRing) the rows come from shared-memory chunks that warps
// consume and release independently; otherwise straight from HBM. Both give
// bit-identical sums, so every backend produces the same bits.
//
// The input projection is computed by every cluster (rows split over its CTAs),
// and CTA 0 runs the final norm and score head. The per-op and graph backends
// run the same block functions as separate kernels, where a kernel boundary
// replaces each grid sync and the residual crosses kernels through global
// buffers written by CTA 0. Cast points and op order follow the reference step
// (reference src/cpu/Cpu.cpp:59-141); the sums are reassociated (per-lane
// partials, per-head and per-slice partials, per-warp softmax partials), which
// the fp32 1e-5 tolerance absorbs.
#pragma once

#include "st_device.cuh"
#include "st_ring.cuh"

namespace st {

constexpr int kMaxCluster = 8;
constexpr int kMaxWidth = 1024;
constexpr int kMaxHeadDim = 1024;
constexpr int kMaxWindow = 4096;
constexpr int kMaxFfn = 4096;
constexpr int kKvBytes = 16 * 1024;           // K and V rows one CTA prefetches per head

// Shared scratch of one step CTA (~110 KB; the weight ring takes the rest of
// the CTA's shared memory). The attention buffers and the FFN buffers are
// never live together (a grid sync separates them) and share one union; every
// DSMEM target sits at the same offset in every CTA.
struct alignas(128) Smem2 {
  Smem g;                                        // GEMV input (event, attn_h) / reductions
  float xres[kMaxWidth];                         // residual entering the block
  float x2res[kMaxWidth];                        // residual after attention
  float qkv[3 * kMaxHeadDim];                    // q, k, v of the current head (DSMEM target)
  union {
    struct {
      float apart[kMaxCluster * (kMaxHeadDim + 2)];  // CTA attention partials per rank (DSMEM target)
      float logits[kMaxWindow];                      // this CTA's logits, then softmax weights
      alignas(16) unsigned char kv[kKvBytes];        // this CTA's K rows, then V rows
    } at;
    struct {
      float act[kMaxFfn];                            // this CTA's SwiGLU slice
      float dred[2 * kMaxWidth];                     // down partial rows per rank (DSMEM target)
    } ff;
  } u;
  float gpart[2 * kMaxWidth];                    // down-projection group partials
  float z[kMaxWidth];                            // norm output (GEMV input of QKV and gate/up)
  float rope[kMaxHeadDim / 2];                   // RoPE frequencies, loaded once per launch
  float2 rope_cs[kMaxHeadDim / 2];               // cos, sin of t * frequency for the current stream
  unsigned long long t;                          // position of the stream being stepped
  int slot, valid;                               // t % window and the retained slot count
  float att[2];                                  // max logit and softmax sum of this CTA's slots
  float rscale[kMaxCluster];                     // merge weight of each rank's attention partial
  int sync_ok;                                   // verdict of the last grid sync (DSMEM target)
  int tl_nw[kWarps];                             // timeline entries written by each warp
};

// Dynamic shared memory of the step kernels: Smem2, the ring header, then the
// ring bytes up to the per-block opt-in limit (227 KB on sm_100, 1 KB of it
// left for the kernels' static shared variables).
constexpr size_t kSmemLimit = 227 * 1024;
constexpr size_t kStaticSmemReserve = 1024;
constexpr size_t kRingOffset = (sizeof(Smem2) + sizeof(RingSmem) + 127) / 128 * 128;
constexpr size_t kStepSmemBytes = kSmemLimit - kStaticSmemReserve;
constexpr unsigned kRingCapacity = (unsigned)((kStepSmemBytes - kRingOffset) / 128 * 128);
static_assert(kRingCapacity >= 2 * kChunkBytes, "the weight ring needs room for two chunks");

// Timeline mark tags: the interval since the previous mark is charged to the
// tag of the mark that ends it.
enum TimelineTag : int {
  kTlStepStart = 1, kTlInput, kTlNorm1, kTlRingWait, kTlGemv, kTlQkvRows, kTlQkvShared, kTlKvWait, kTlMerge,
  kTlPv, kTlAttention, kTlPartialsShared, kTlOutProj, kTlSyncArrive, kTlSyncWait, kTlResidualHeads, kTlNorm2,
  kTlGateUp, kTlDownPartial, kTlClusterReduce, kTlResidualClusters, kTlStepEnd, kTlRingFill, kTlIssueAt
};

// Phase-boundary mark, clock64() << 8 | tag, by lane 0 of every warp of CTA
// a.timeline_cta when a timeline buffer is given; warp w fills its own
// region [w * capacity / kWarps, (w + 1) * capacity / kWarps). Compiled only
// into the diagnostic kernel variants.
__device__ __forceinline__ void tl_put(const StepArgs& a, Smem2& sm, long long value) {
  if (a.timeline && blockIdx.x == a.timeline_cta && (threadIdx.x & 31) == 0) {
    const int w = threadIdx.x >> 5, per_warp = a.timeline_capacity / kWarps;
    if (sm.tl_nw[w] < per_warp) a.timeline[(size_t)w * per_warp + sm.tl_nw[w]++] = value;
  }
}
template <bool kDiag = true>
__device__ __forceinline__ void tl_mark(const StepArgs& a, Smem2& sm, int tag) {
  if constexpr (kDiag) tl_put(a, sm, (long long)((clock64() << 8) | (long long)tag));
}

// Diagnostics: the issue time of the chunk just acquired, as a mark tagged
// kTlIssueAt (not an interval; the host pairs it with the next mark).
__device__ __forceinline__ void tl_mark_issue(const StepArgs& a, Smem2& sm, const RingSmem& rs, const Ring& rg) {
  tl_put(a, sm, (long long)((rs.issued_at[(rg.consumed) % kRingChunks] << 8) | (long long)kTlIssueAt));
}

// Compile-time shape of a step kernel: weights through the shared-memory ring
// (kRing) or straight from HBM; diagnostics (timeline marks, trace buffers)
// compiled in (kDiag) or not. The hot kernels carry no diagnostic code, which
// keeps the per-layer instruction footprint small.
template <bool R, bool D>
struct StepCfg {
  static constexpr bool kRing = R;
  static constexpr bool kDiag = D;
};

// ---------------------------------------------------------------- cluster helpers
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ unsigned cluster_size() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ unsigned cluster_id() {
  unsigned r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ unsigned cluster_count() {
  unsigned r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// All threads of every CTA in the cluster; release/acquire at cluster scope.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store v at the same shared-memory offset as `local` in CTA `rank` of the cluster.
__device__ __forceinline__ void dsmem_store(float* local, unsigned rank, float v) {
  const unsigned addr = (unsigned)__cvta_generic_to_shared(local);
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" :: "r"(remote), "f"(v) : "memory");
}

__device__ __forceinline__ void dsmem_store_u32(int* local, unsigned rank, int v) {
  const unsigned addr = (unsigned)__cvta_generic_to_shared(local);
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
  asm volatile("st.shared::cluster.u32 [%0], %1;" :: "r"(remote), "r"(v) : "memory");
}

// 16-byte global -> shared copy through L2 (generic proxy), and its waits.
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_addr(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Waits until at most n of this thread's committed cp.async groups are pending
// (n in [0, 7]; the instruction takes an immediate).
__device__ __forceinline__ void cp_async_wait_pending(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
  }
}

struct ClusterPos {
  unsigned rank, size, id, count;
  __device__ static ClusterPos get() { return {cluster_rank(), cluster_size(), cluster_id(), cluster_count()}; }
};

// Grid-wide barrier in cluster units. The cluster first meets at a hardware
// barrier, then one thread of its rank-0 CTA (the ring issuer, which keeps
// issuing weight chunks while it polls) alone arrives on the global counter and waits
// (bounded, with the error word checked) and writes its verdict into every
// CTA of the cluster through DSMEM before a second cluster barrier. Every CTA
// of a cluster therefore returns the same verdict, so a failed wait can never
// leave a peer stranded at a later cluster barrier. The counter rises by one
// per cluster per barrier; `base` is its value when the launch started.
struct ClusterGridSync {
  unsigned long long base;
  unsigned long long epoch;
  // The cluster barrier (release/acquire at cluster scope) orders every
  // thread's earlier writes before the arriving thread's gpu-scope release,
  // so only that thread fences.
  // With a ring, thread 0 of every CTA issues weight chunks once the whole
  // CTA has arrived (every earlier chunk released), and the waiting thread
  // keeps issuing while it polls, so the next phases' weights land during the
  // wait.
  __device__ bool sync(const StepArgs& a, unsigned long long timeout_ns, int* ok_slot, Smem2* tl = nullptr,
                       Ring* rg = nullptr, RingSmem* rs = nullptr) {
    cluster_sync();
    if (tl) tl_mark(a, *tl, kTlSyncArrive);
    if (rg) ring_fill(*rg, *rs, kFillAll);
    const unsigned rank = cluster_rank();
    if (rank == 0 && threadIdx.x == kIssuer) {
      epoch += 1;
      const unsigned long long target = base + epoch * cluster_count();
      int good = ld_volatile_int(a.error) == 0;
      if (good) {
        __threadfence();
        red_release_gpu_add(a.bar_counter, 1ull);
        unsigned long long start = 0;
        unsigned int polls = 0;
        while (ld_acquire_gpu(a.bar_counter) < target) {
          if ((++polls & 63u) == 0) {
            if (rg) ring_fill(*rg, *rs, kFillAll);
            if (ld_volatile_int(a.error) != 0) { good = 0; break; }
            const unsigned long long now = globaltimer();
            if (start == 0) start = now;
            else if (now - start > timeout_ns) { set_error(a, kBarrierTimeout); good = 0; break; }
          }
        }
      }
      const unsigned n = cluster_size();
      for (unsigned k = 0; k < n; ++k) dsmem_store_u32(ok_slot, k, good);
    }
    cluster_sync();
    if (tl) tl_mark(a, *tl, kTlSyncWait);
    return *reinterpret_cast<volatile int*>(ok_slot) != 0;
  }
};

// Every step kernel starts here: a launch whose cluster shape differs from the
// one the buffers were sized for would write past dpart and mistime the grid
// syncs, so the whole grid returns at once (no barrier executed yet) with the
// error word set.
__device__ __forceinline__ bool cluster_shape_ok(const StepArgs& a) {
  if ((int)cluster_size() == a.cluster_size && (int)cluster_count() == a.clusters) return true;
  if (threadIdx.x == 0) set_error(a, kClusterShape);
  return false;
}

// Contiguous share [lo, hi) of `units` for part `part` of `parts`. Model and
// grid limits (units <= 4096, parts <= 1024) keep units * parts in 32 bits,
// so this stays a 32-bit division (a 64-bit one is a long software routine).
__device__ __forceinline__ void split(int units, int part, int parts, int& lo, int& hi) {
  lo = (int)(((unsigned)units * (unsigned)part) / (unsigned)parts);
  hi = (int)(((unsigned)units * (unsigned)(part + 1)) / (unsigned)parts);
}

__device__ __forceinline__ int valid_length(unsigned long long t, int window) {
  return t + 1 < (unsigned long long)window ? (int)(t + 1) : window;
}

// ---------------------------------------------------------------- warp GEMV
// Geometry of a GEMV over rows of `cols` elements of type T. Aligned rows
// (cols a multiple of the 16-byte vector) are split over a power-of-two group
// of `lpr` lanes, each lane taking vectors sl, sl + lpr, ...; unaligned rows
// fall back to one warp per row with scalar loads.
template <typename T>
struct RowGeom {
  int cols, units, lpr, rpw;
  bool vec;
  __device__ RowGeom(int c, int u, int l, int r, bool v) : cols(c), units(u), lpr(l), rpw(r), vec(v) {}
  __device__ explicit RowGeom(int c) : cols(c) {
    constexpr int V = Storage<T>::kVec;
    vec = (c % V) == 0;
    units = vec ? c / V : c;
    int p = 1;
    while (p < units && p < 32) p <<= 1;
    lpr = vec ? p : 32;
    rpw = 32 / lpr;
  }
};

// The lane's share of a GEMV input vector xs, held in registers for a whole
// phase: the V floats of each vector sl + lpr * k, k < kN, that its rows meet
// (zeros past the row). Every row the warp computes reuses them, so shared
// memory carries the weights only.
template <typename T>
struct XRegs {
  static constexpr int V = Storage<T>::kVec;
  static constexpr int kN = kMaxCols / V / 32;  // vectors per lane at most
  float x[kN * V];
  __device__ __forceinline__ void load(const float* xs, const RowGeom<T>& g, int sl) {
#pragma unroll
    for (int k = 0; k < kN; ++k) {
      const int v = sl + g.lpr * k;
#pragma unroll
      for (int e = 0; e < V; e += 4) {
        const float4 q = g.vec && v < g.units ? *reinterpret_cast<const float4*>(xs + v * V + e)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
        x[k * V + e] = q.x;
        x[k * V + e + 1] = q.y;
        x[k * V + e + 2] = q.z;
        x[k * V + e + 3] = q.w;
      }
    }
  }
};

__device__ __forceinline__ uint4 ld_shared_v4(const void* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(smem_addr(p)));
  return r;
}

// Sum over one 16-byte weight vector times V register floats, in element order.
template <typename T>
__device__ __forceinline__ float dot_regs(const uint4& w, const float* x) {
  constexpr int V = Storage<T>::kVec;
  float f[V];
  Storage<T>::unpack(w, f);
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < V; ++k) acc = fmaf(f[k], x[k], acc);
  return acc;
}

// U dot products of consecutive rows (row stride `cols`) by the lpr lanes of
// one group; every lane of the group returns the full sums. Lanes of an
// invalid group compute zeros but still take part in the shuffles. Aligned
// rows use the register copy xr; unaligned rows read xs.
template <typename T, int U, bool kShared>
__device__ __forceinline__ void dot_rows(const T* row, const RowGeom<T>& g, int sl, const XRegs<T>& xr,
                                         const float* xs, bool valid, float (&out)[U]) {
  constexpr int V = Storage<T>::kVec;
  constexpr int kN = XRegs<T>::kN;
  constexpr int kB = 4;  // vectors per lane in flight per row
#pragma unroll
  for (int u = 0; u < U; ++u) out[u] = 0.f;
  if (g.vec) {
#pragma unroll
    for (int k0 = 0; k0 < kN; k0 += kB) {
      if (sl + g.lpr * k0 >= g.units) break;
      uint4 w[U][kB];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          const int v = sl + g.lpr * (k0 + b);
          const T* p = row + (size_t)u * g.cols + (size_t)v * V;
          if (valid && v < g.units) {
            if constexpr (kShared) w[u][b] = ld_shared_v4(p);
            else w[u][b] = ld_stream(p);
          } else {
            w[u][b] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int b = 0; b < kB; ++b)
          if (sl + g.lpr * (k0 + b) < g.units) out[u] += dot_regs<T>(w[u][b], xr.x + (k0 + b) * V);
    }
  } else if (valid) {
    for (int e = sl; e < g.cols; e += 32)
#pragma unroll
      for (int u = 0; u < U; ++u) out[u] = fmaf(Storage<T>::load(row + (size_t)u * g.cols, e), xs[e], out[u]);
  }
#pragma unroll
  for (int u = 0; u < U; ++u)
    for (int o = g.lpr >> 1; o > 0; o >>= 1) out[u] += __shfl_xor_sync(0xffffffffu, out[u], o);
}

// Rows [0, n) of W (n a multiple of U) against the input vector (xr in
// registers, xs in shared memory), in groups of U rows spread over the warps;
// epi(row, v[U], sl) runs on every lane of the group that computed rows
// row .. row+U-1 (sl = lane within the group). No CTA barrier.
// Groups are dealt to warps by their index within the whole span (g0 = index
// of this block's first group), so consecutive chunks of one span go to
// different warps and are computed concurrently.
template <typename T, int U, bool kShared, typename Epi>
__device__ __forceinline__ void warp_rows_x(const T* W, int n, const RowGeom<T>& g, const XRegs<T>& xr,
                                            const float* xs, Epi&& epi, int g0 = 0) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Rows from the ring skip the issuer's warp, whose copies would hold up the
  // barrier that ends the phase.
  constexpr int kW = kShared ? kWarps - 1 : kWarps;
  if (warp >= kW) return;
  const int sub = lane / g.lpr, sl = lane - sub * g.lpr;
  const int groups = n / U, per_pass = kW * g.rpw;
  const int first = ((warp * g.rpw - g0) % per_pass + per_pass) % per_pass;
  for (int base = first; base < groups; base += per_pass) {
    const int gi = base + sub;
    const bool valid = gi < groups;
    float v[U];
    dot_rows<T, U, kShared>(W + (size_t)(valid ? gi : 0) * U * g.cols, g, sl, xr, xs, valid, v);
    if (valid) epi(gi * U, v, sl);
  }
}

// Same, loading the register copy of xs first.
template <typename T, int U, bool kShared, typename Epi>
__device__ __forceinline__ void warp_rows(const T* W, int n, const RowGeom<T>& g, const float* xs, Epi&& epi) {
  XRegs<T> xr;
  xr.load(xs, g, (threadIdx.x & 31) % g.lpr);
  warp_rows_x<T, U, kShared>(W, n, g, xr, xs, epi);
}

// The next `rows` rows of the ring's current span (groups of U rows, as the
// chunk table was cut), chunk by chunk; epi gets rows relative to the span.
template <typename T, int U, class Cfg, typename Epi>
__device__ __forceinline__ void ring_rows(const StepArgs& a, Ring& rg, RingSmem& rs, Smem2& sm, int rows,
                                          const RowGeom<T>& g, const float* xs, Epi&& epi) {
  const int rpc = rows_per_chunk(g.cols * (int)sizeof(T), U);
  XRegs<T> xr;
  xr.load(xs, g, (threadIdx.x & 31) % g.lpr);
  for (int c0 = 0; c0 < rows; c0 += rpc) {
    const int n = min(rpc, rows - c0);
    const T* p = (const T*)ring_acquire(a, rg, rs);
    tl_mark<Cfg::kDiag>(a, sm, kTlRingWait);
    if constexpr (Cfg::kDiag) tl_mark_issue(a, sm, rs, rg);
    warp_rows_x<T, U, true>(p, n, g, xr, xs, [&](int r, const float (&v)[U], int sl) { epi(c0 + r, v, sl); }, c0 / U);
    tl_mark<Cfg::kDiag>(a, sm, kTlGemv);
    ring_release(rg, rs);
    tl_mark<Cfg::kDiag>(a, sm, kTlRingFill);
  }
}

// The issuer reclaims released chunks and issues more (kRing only); called
// right after barriers, when every warp has released what it consumed.
template <class Cfg>
__device__ __forceinline__ void ring_poll(Ring& rg, RingSmem& rs) {
  if constexpr (Cfg::kRing) ring_fill(rg, rs, 2);
}

// Rows [0, rows) of a weight matrix: from the ring (kRing) or straight from
// global memory at W.
template <typename T, int U, class Cfg, typename Epi>
__device__ __forceinline__ void gemv_rows(const StepArgs& a, Ring& rg, RingSmem& rs, Smem2& sm, const T* W, int rows,
                                          const RowGeom<T>& g, const float* xs, Epi&& epi) {
  if constexpr (Cfg::kRing) ring_rows<T, U, Cfg>(a, rg, rs, sm, rows, g, xs, epi);
  else warp_rows<T, U, false>(W, rows, g, xs, epi);
}

// ---------------------------------------------------------------- norms and residuals
// RMSNorm of x into out, cast to storage precision (reference
// src/cpu/Cpu.cpp:43-57: scale = 1/sqrt(mean(x^2)+eps), out = x*scale*g).
// Thread i reads x[i], x[i + kThreads], ...: callers that just wrote x with
// the same mapping need no barrier first. Ends with a barrier (out complete).
template <typename T>
__device__ __forceinline__ void norm_vec(const float* x, const T* gain, int width, float eps, Smem2& sm, float* out) {
  float s = 0.f;
#pragma unroll 1
  for (int i = threadIdx.x; i < width; i += kThreads) s += x[i] * x[i];
  const float total = block_sum(s, sm.g);
  const float scale = 1.0f / sqrtf(total / (float)width + eps);
#pragma unroll 1
  for (int i = threadIdx.x; i < width; i += kThreads) out[i] = Storage<T>::round(x[i] * scale * Storage<T>::load(gain, i));
  __syncthreads();
}

// The norm with its gain vector from the ring (kRing) or from `gain`.
template <typename T, class Cfg>
__device__ __forceinline__ void norm_block(const StepArgs& a, Ring& rg, RingSmem& rs, Smem2& sm, const float* x,
                                           const T* gain, float* out) {
  if constexpr (Cfg::kRing) {
    const T* g = (const T*)ring_acquire(a, rg, rs);
    norm_vec<T>(x, g, a.width, a.epsilon, sm, out);
    ring_release(rg, rs);
  } else {
    norm_vec<T>(x, gain, a.width, a.epsilon, sm, out);
  }
}

// p[0] + p[stride] + ... + p[(n-1) stride], added in index order, with the
// L2 loads issued 16 at a time ahead of the adds (the partials were written
// by other CTAs of this launch, so they are read with ld.global.cg).
__device__ __forceinline__ float sum_rows(const float* p, int stride, int n) {
  float acc = 0.f;
#pragma unroll 1
  for (int k0 = 0; k0 < n; k0 += 16) {
    float v[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) v[u] = k0 + u < n ? ld_cg(p + (size_t)(k0 + u) * stride) : 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u)
      if (k0 + u < n) acc += v[u];
  }
  return acc;
}

// x' = cast(x + cast(sum_h P[h])) from sm.xres into sm.x2res (thread i writes
// element i, i + kThreads, ...; no barrier).
template <typename T>
__device__ __forceinline__ void residual_from_heads(const StepArgs& a, int s, Smem2& sm) {
  const int d = a.width;
  const float* P = a.pout + (size_t)s * a.heads * d;
#pragma unroll 1
  for (int i = threadIdx.x; i < d; i += kThreads)
    sm.x2res[i] = Storage<T>::round(sm.xres[i] + Storage<T>::round(sum_rows(P + i, d, a.heads)));
}

// x = cast(x' + cast(sum_c D[c])) from sm.x2res into sm.xres (same mapping; no barrier).
template <typename T>
__device__ __forceinline__ void residual_from_clusters(const StepArgs& a, int s, int nclusters, Smem2& sm) {
  const int d = a.width;
  const float* D = a.dpart + (size_t)s * nclusters * d;
#pragma unroll 1
  for (int i = threadIdx.x; i < d; i += kThreads)
    sm.xres[i] = Storage<T>::round(sm.x2res[i] + Storage<T>::round(sum_rows(D + i, d, nclusters)));
}

// ---------------------------------------------------------------- blocks
// Position of stream s into sm.t (read by other threads after the next
// barrier): the stored position plus `event`, the events this launch has
// already stepped without storing their positions.
__device__ __forceinline__ void load_position(const StepArgs& a, int s, Smem2& sm, unsigned long long event = 0) {
  if (threadIdx.x == 0) {
    const unsigned long long t = ld_cg_u64(a.position + s) + event;
    sm.t = t;
    sm.slot = (int)(t % (unsigned long long)a.window);
    sm.valid = valid_length(t, a.window);
  }
}

// RoPE rotation of the current position, angle = float(t) * frequency
// (reference src/cpu/Cpu.cpp:81-89), for every dim pair; needs sm.t visible,
// and is read after the caller's next barrier.
__device__ __forceinline__ void rope_table(const StepArgs& a, Smem2& sm) {
  const float tf = (float)sm.t;
  for (int i = threadIdx.x; i < a.head_dim / 2; i += kThreads) {
    const float angle = tf * sm.rope[i];
    sm.rope_cs[i] = make_float2(cosf(angle), sinf(angle));
  }
}

// x = cast(W_in input) for stream s into sm.xres. With the ring the cluster
// splits the rows and broadcasts them into every member through DSMEM;
// otherwise this CTA computes every row. Ends after a barrier.
template <typename T, class Cfg>
__device__ void step_input(const StepArgs& a, int s, const float* input, const ClusterPos& cp, Smem2& sm, Ring& rg,
                           RingSmem& rs) {
  for (int i = threadIdx.x; i < a.features; i += kThreads) sm.g.xs[i] = __ldcv(input + (size_t)s * a.features + i);
  __syncthreads();
  rope_table(a, sm);  // sm.t was written before the barrier; published by the barrier below
  const RowGeom<T> g(a.features);
  if constexpr (Cfg::kRing) {
    int lo, hi;
    split(a.width, (int)cp.rank, (int)cp.size, lo, hi);
    ring_rows<T, 1, Cfg>(a, rg, rs, sm, hi - lo, g, sm.g.xs, [&](int r, const float (&v)[1], int sl) {
      const float x = Storage<T>::round(v[0]);
      for (unsigned k = (unsigned)sl; k < cp.size; k += (unsigned)g.lpr) dsmem_store(&sm.xres[lo + r], k, x);
    });
    cluster_sync();
  } else {
    warp_rows<T, 1, false>((const T*)a.input_w, a.width, g, sm.g.xs, [&](int r, const float (&v)[1], int sl) {
      if (sl == 0) sm.xres[r] = Storage<T>::round(v[0]);
    });
    __syncthreads();
  }
}

// Issue cp.async copies of this CTA's K and V rows [j0, j1) of one head into
// sm.u.at.kv (K rows, then V rows), skipping the slot this step overwrites.
// Returns false (nothing issued) when they do not fit or are not 16-byte rows.
template <typename T>
__device__ __forceinline__ bool kv_prefetch(const T* keys, const T* values, int j0, int j1, int slot, int hd,
                                            Smem2& sm) {
  const int row_bytes = hd * (int)sizeof(T);
  const int n = j1 - j0;
  if (row_bytes % 16 != 0 || 2 * n * row_bytes > kKvBytes) return false;
  const int vpr = row_bytes / 16, vecs = n * vpr;
  for (int i = threadIdx.x; i < 2 * vecs; i += kThreads) {
    const bool is_v = i >= vecs;
    const int k = is_v ? i - vecs : i;
    const int j = j0 + k / vpr;
    if (j == slot) continue;
    const char* src = (const char*)(is_v ? values : keys) + (size_t)j0 * row_bytes + (size_t)k * 16;
    cp_async16(sm.u.at.kv + (size_t)i * 16, src);
  }
  cp_async_commit();
  return true;
}

// Attention of head h over this CTA's slots [j0, j1) (reference
// src/cpu/Cpu.cpp:97-110: logits q.k / sqrt(hd), softmax over the retained
// slots, sum p v): warps compute the logits (one slot per warp at a time),
// warp 0 turns them into softmax weights against this CTA's max, and every
// thread then computes one (rank, dim) value of the partial (m, l, acc),
// storing it straight into apart[rank] of that rank's CTA. The partial is
// computed once per destination rank, which costs a few FMAs and saves a
// barrier.
template <typename T, class Cfg>
__device__ void attention_share(const StepArgs& a, int l, int s, int h, int j0, int j1, int slot, bool kv_smem,
                                const ClusterPos& cp, Smem2& sm) {
  const int hd = a.head_dim, W = a.window, n = j1 - j0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const size_t head_base = ((((size_t)s * a.layers + l) * a.heads + h) * (size_t)W) * hd;
  const T* Kg = (const T*)a.keys + head_base;
  const T* Vg = (const T*)a.values + head_base;
  const T* Ks = reinterpret_cast<const T*>(sm.u.at.kv);
  const T* Vs = Ks + (size_t)n * hd;
  const float* q = sm.qkv;
  const float* kcur = sm.qkv + hd;
  const float* vcur = sm.qkv + 2 * hd;
  const float root = sqrtf((float)hd);
  float* logits = sm.u.at.logits;
  for (int j = j0 + warp; j < j1; j += kWarps) {
    const T* krow = kv_smem ? Ks + (size_t)(j - j0) * hd : Kg + (size_t)j * hd;
    float dot = 0.f;
    if (j == slot) {
      for (int i = lane; i < hd; i += 32) dot = fmaf(q[i], kcur[i], dot);
    } else if (kv_smem) {
      for (int i = lane; i < hd; i += 32) dot = fmaf(q[i], Storage<T>::load(krow, i), dot);
    } else {
      for (int i = lane; i < hd; i += 32) dot = fmaf(q[i], Storage<T>::load_cg(krow, i), dot);
    }
    dot = warp_sum(dot);
    if (lane == 0) logits[j - j0] = dot / root;
  }
  __syncthreads();
  if (warp == 0) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, logits[j]);
    m = warp_max(m);
    float sum = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float p = expf(logits[j] - m);
      logits[j] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      sm.att[0] = n > 0 ? m : -INFINITY;
      sm.att[1] = n > 0 ? sum : 0.f;
    }
  }
  __syncthreads();
  tl_mark<Cfg::kDiag>(a, sm, kTlPv);
  float* mine = sm.u.at.apart + (size_t)cp.rank * (hd + 2);
  const int vals = hd + 2, items = vals * (int)cp.size;
  for (int it = threadIdx.x; it < items; it += kThreads) {
    const int k = it / vals, i = it - k * vals;
    float v;
    if (i < 2) {
      v = sm.att[i];
    } else {
      const int dd = i - 2;
      v = 0.f;
      for (int j = j0; j < j1; ++j) {
        const float x = j == slot ? vcur[dd]
                        : kv_smem ? Storage<T>::load(Vs + (size_t)(j - j0) * hd, dd)
                                  : Storage<T>::load_cg(Vg + (size_t)j * hd, dd);
        v = fmaf(logits[j - j0], x, v);
      }
    }
    dsmem_store(mine + i, (unsigned)k, v);
  }
}

// One head h of one stream, run by the CTAs of one cluster; z (norm1 output)
// is in sm.z. Leaves P[h] rows of this CTA in global memory.
template <typename T, class Cfg>
__device__ void attention_head(const StepArgs& a, int l, int s, int h, const ClusterPos& cp, Smem2& sm, Ring& rg,
                               RingSmem& rs) {
  const int d = a.width, hd = a.head_dim, W = a.window;
  const LayerPtrs& w = a.layer[l];
  const int slot = sm.slot, valid = sm.valid;
  T* keys = (T*)a.keys + ((((size_t)s * a.layers + l) * a.heads + h) * (size_t)W) * hd;
  T* values = (T*)a.values + ((((size_t)s * a.layers + l) * a.heads + h) * (size_t)W) * hd;
  int j0, j1;
  split(valid, (int)cp.rank, (int)cp.size, j0, j1);
  const bool kv_smem = kv_prefetch<T>(keys, values, j0, j1, slot, hd, sm);
  // q, k, v rows of head h (head-major [H][3 hd][d]); pairs split over the cluster.
  int lo, hi;
  split(3 * hd / 2, (int)cp.rank, (int)cp.size, lo, hi);
  const RowGeom<T> gd(d);
  auto qkv_epi = [&](int r, const float (&v)[2], int sl) {
    const int row = 2 * lo + r;
    const int which = row / hd, dim = row - which * hd;
    float v0 = Storage<T>::round(v[0]);
    float v1 = Storage<T>::round(v[1]);
    if (which < 2) {
      const float2 cs = sm.rope_cs[dim >> 1];
      const float r0v = v0 * cs.x - v1 * cs.y;
      const float r1v = v0 * cs.y + v1 * cs.x;
      v0 = Storage<T>::round(r0v);
      v1 = Storage<T>::round(r1v);
    }
    for (unsigned k = (unsigned)sl; k < cp.size; k += (unsigned)gd.lpr) {
      dsmem_store(&sm.qkv[row], k, v0);
      dsmem_store(&sm.qkv[row + 1], k, v1);
    }
    if (which > 0 && sl == gd.lpr - 1) {
      T* ring = which == 1 ? keys : values;
      const size_t at = (size_t)slot * hd + dim;
      Storage<T>::store(ring, at, v0);
      Storage<T>::store(ring, at + 1, v1);
    }
  };
  gemv_rows<T, 2, Cfg>(a, rg, rs, sm, (const T*)w.qkv + ((size_t)h * 3 * hd + 2 * (size_t)lo) * d, 2 * (hi - lo),
                         gd, sm.z, qkv_epi);
  if (kv_smem) cp_async_wait_all();
  tl_mark<Cfg::kDiag>(a, sm, kTlQkvRows);
  cluster_sync();
  ring_poll<Cfg>(rg, rs);
  tl_mark<Cfg::kDiag>(a, sm, kTlQkvShared);
  if constexpr (Cfg::kDiag)
    if (a.trace_qkv && cp.rank == 0)
      for (int i = threadIdx.x; i < 3 * hd; i += kThreads)
        a.trace_qkv[(size_t)s * 3 * d + (size_t)(i / hd) * d + (size_t)h * hd + i % hd] = sm.qkv[i];
  attention_share<T, Cfg>(a, l, s, h, j0, j1, slot, kv_smem, cp, sm);
  tl_mark<Cfg::kDiag>(a, sm, kTlAttention);
  cluster_sync();
  tl_mark<Cfg::kDiag>(a, sm, kTlPartialsShared);
  // merge the cluster's partials in rank order -> attn_h (cast) in sm.g.xs[0..hd):
  // the first warp computes each rank's weight exp(m_k - M) (0 for an empty
  // share) once, then every dim folds the ranks in order.
  if (threadIdx.x < 32) {
    float M = -INFINITY;
    for (unsigned k = 0; k < cp.size; ++k) {
      const float* pk = sm.u.at.apart + (size_t)k * (hd + 2);
      if (pk[1] > 0.f) M = fmaxf(M, pk[0]);
    }
    if (threadIdx.x < cp.size) {
      const float* pk = sm.u.at.apart + (size_t)threadIdx.x * (hd + 2);
      sm.rscale[threadIdx.x] = pk[1] > 0.f ? expf(pk[0] - M) : 0.f;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < hd; i += kThreads) {
    float L = 0.f, acc = 0.f;
    for (unsigned k = 0; k < cp.size; ++k) {
      const float* pk = sm.u.at.apart + (size_t)k * (hd + 2);
      const float scale = sm.rscale[k];
      L = fmaf(pk[1], scale, L);
      acc = fmaf(pk[2 + i], scale, acc);
    }
    sm.g.xs[i] = Storage<T>::round(acc / L);
    if constexpr (Cfg::kDiag)
      if (a.trace_attention && cp.rank == 0) a.trace_attention[(size_t)s * d + (size_t)h * hd + i] = sm.g.xs[i];
  }
  __syncthreads();
  tl_mark<Cfg::kDiag>(a, sm, kTlMerge);
  // out-projection partial of this head: rows split over the cluster ([H][d][hd] layout)
  split(d, (int)cp.rank, (int)cp.size, lo, hi);
  float* P = a.pout + ((size_t)s * a.heads + h) * d + lo;
  const RowGeom<T> gh(hd);
  gemv_rows<T, 1, Cfg>(a, rg, rs, sm, (const T*)w.out + ((size_t)h * d + lo) * hd, hi - lo, gh, sm.g.xs,
                         [&](int r, const float (&v)[1], int sl) {
                           if (sl == 0) P[r] = v[0];
                         });
  tl_mark<Cfg::kDiag>(a, sm, kTlOutProj);
}

// FFN block for stream s: needs sm.x2res (x', written with the norm's thread
// mapping); leaves D[cluster] in global memory.
template <typename T, class Cfg>
__device__ void block_ffn(const StepArgs& a, int l, int s, const ClusterPos& cp, Smem2& sm, Ring& rg, RingSmem& rs) {
  const int d = a.width, F = a.ffn;
  const LayerPtrs& w = a.layer[l];
  norm_block<T, Cfg>(a, rg, rs, sm, sm.x2res, (const T*)w.norm2, sm.z);
  tl_mark<Cfg::kDiag>(a, sm, kTlNorm2);
  const int G = (int)(cp.count * cp.size), gi = (int)(cp.id * cp.size + cp.rank);
  int lo, hi;
  split(F, gi, G, lo, hi);
  float* act_trace = Cfg::kDiag && a.trace_act ? a.trace_act + (size_t)s * F : nullptr;
  const RowGeom<T> gd(d);
  gemv_rows<T, 2, Cfg>(a, rg, rs, sm, (const T*)w.gateup + 2 * (size_t)lo * d, 2 * (hi - lo), gd, sm.z,
                         [&](int r, const float (&v)[2], int sl) {
                           if (sl != 0) return;
                           const float gt = Storage<T>::round(v[0]);
                           const float up = Storage<T>::round(v[1]);
                           const int f = lo + (r >> 1);
                           const float x = Storage<T>::round((gt / (1.0f + expf(-gt))) * up);
                           sm.u.ff.act[f - lo] = x;
                           if (Cfg::kDiag && act_trace) act_trace[f] = x;
                         });
  __syncthreads();
  ring_poll<Cfg>(rg, rs);
  tl_mark<Cfg::kDiag>(a, sm, kTlGateUp);
  // partial[row] = sum_{f in slice} W_down^T[f][row] act[f]. With d < kThreads
  // the CTA splits into `groups` thread groups over rows, group g taking
  // f = lo+g, lo+g+groups, ...; each thread accumulates f in ascending order.
  constexpr int kCols = kMaxWidth / kThreads;  // columns per thread at most
  const int groups = d >= kThreads ? 1 : kThreads / d;
  const int tpg = d >= kThreads ? kThreads : d;  // threads per group
  const int g = (int)threadIdx.x / tpg, c0 = (int)threadIdx.x - g * tpg;
  const bool active = g < groups;
  float acc[kCols];
#pragma unroll
  for (int k = 0; k < kCols; ++k) acc[k] = 0.f;
  auto rows_from = [&](const T* rows, int f_begin, int f_end) {
    // `rows` holds W_down^T rows f_begin .. f_end-1 (row stride d)
    if (!active) return;
    int f = f_begin + ((g - (f_begin - lo)) % groups + groups) % groups;
    for (; f < f_end; f += groups) {
      const float av = sm.u.ff.act[f - lo];
      const T* wrow = rows + (size_t)(f - f_begin) * d;
#pragma unroll
      for (int k = 0; k < kCols; ++k) {
        const int c = c0 + k * tpg;
        if (c < d && (k == 0 || tpg == kThreads)) acc[k] = fmaf(Storage<T>::load(wrow, c), av, acc[k]);
      }
    }
  };
  if constexpr (Cfg::kRing) {
    const int rpc = rows_per_chunk(d * (int)sizeof(T), 1);
    for (int f0 = lo; f0 < hi; f0 += rpc) {
      const int n = min(rpc, hi - f0);
      const T* p = (const T*)ring_acquire(a, rg, rs);
      tl_mark<Cfg::kDiag>(a, sm, kTlRingWait);
      rows_from(p, f0, f0 + n);
      ring_release(rg, rs);
    }
  } else {
    rows_from((const T*)w.down + (size_t)lo * d, lo, hi);  // W_down^T, [F][d]
  }
  float* part = sm.gpart;  // [groups][d]
  if (groups > 1) {
    if (active) part[g * d + c0] = acc[0];
    __syncthreads();
  }
  // sum groups in order, then reduce-scatter to the owning rank of each row segment
  const int seg = (d + (int)cp.size - 1) / (int)cp.size;
#pragma unroll
  for (int k = 0; k < kCols; ++k) {
    const int row = (int)threadIdx.x + k * kThreads;
    if (row >= d) continue;
    float v = acc[k];
    if (groups > 1) {
      v = 0.f;
      for (int gg = 0; gg < groups; ++gg) v += part[gg * d + row];
    }
    const unsigned owner = (unsigned)(row / seg);
    dsmem_store(&sm.u.ff.dred[cp.rank * seg + (row - (int)owner * seg)], owner, v);
  }
  tl_mark<Cfg::kDiag>(a, sm, kTlDownPartial);
  cluster_sync();
  ring_poll<Cfg>(rg, rs);
  const int r_lo = (int)cp.rank * seg, r_hi = min(d, r_lo + seg);
  float* D = a.dpart + ((size_t)s * cp.count + cp.id) * d;
  for (int row = r_lo + threadIdx.x; row < r_hi; row += kThreads) {
    float v = 0.f;
    for (unsigned k = 0; k < cp.size; ++k) v += sm.u.ff.dred[k * seg + (row - r_lo)];
    D[row] = v;
  }
  tl_mark<Cfg::kDiag>(a, sm, kTlClusterReduce);
}

// Final RMSNorm + score head (no cast) for stream s from sm.xres, into
// a.score[s] and, when given, score_out[s]; one CTA.
template <typename T>
__device__ void block_score(const StepArgs& a, int s, Smem2& sm, float* score_out = nullptr) {
  norm_vec<T>(sm.xres, (const T*)a.final_norm, a.width, a.epsilon, sm, sm.g.xs);
  float acc = 0.f;
  for (int i = threadIdx.x; i < a.width; i += kThreads)
    acc = fmaf(Storage<T>::load((const T*)a.score_w, i), sm.g.xs[i], acc);
  const float total = block_sum(acc, sm.g);
  if (threadIdx.x == 0) {
    a.score[s] = total;
    if (score_out) score_out[s] = total;
  }
  __syncthreads();
}

// The CTA that writes hidden state, scores and positions in the device-loop
// kernels: the last one, whose cluster has no attention head at full size and
// so has slack while the attention clusters work.
__device__ __forceinline__ bool is_score_cta() { return blockIdx.x == gridDim.x - 1; }

// hidden[s][l] and the residual buffer a.x from x (thread i writes element i,
// i + kThreads, ...).
__device__ __forceinline__ void write_hidden(const StepArgs& a, int s, int l, const float* x) {
  float* hidden = a.hidden + ((size_t)s * a.layers + l) * a.width;
  float* xg = a.x + (size_t)s * a.width;
  for (int i = threadIdx.x; i < a.width; i += kThreads) {
    hidden[i] = x[i];
    xg[i] = x[i];
  }
}

// Whole step inside one cluster launch; `input` is [S][features]. Every CTA
// keeps x and x' in shared memory; streams run one after another. `event`
// counts the events this launch stepped before (their positions are not yet
// stored); `score_out` ([S], may be null) receives the scores too; with
// `advance` the positions are stored incremented.
template <typename T, class Cfg>
__device__ bool forward2(const StepArgs& a, const float* input, ClusterGridSync& gs, Smem2& sm, Ring& rg,
                         RingSmem& rs, unsigned long long event = 0, float* score_out = nullptr,
                         bool advance = true) {
  const ClusterPos cp = ClusterPos::get();
  for (int s = 0; s < a.streams; ++s) {
    // The score CTA may still read its x for the previous stream or event
    // while the next input projection writes x through DSMEM.
    if (s > 0 || event > 0) cluster_sync();
    tl_mark<Cfg::kDiag>(a, sm, kTlStepStart);
    load_position(a, s, sm, event);
    step_input<T, Cfg>(a, s, input, cp, sm, rg, rs);
    tl_mark<Cfg::kDiag>(a, sm, kTlInput);
    for (int l = 0; l < a.layers; ++l) {
      if ((int)cp.id < a.heads) {
        norm_block<T, Cfg>(a, rg, rs, sm, sm.xres, (const T*)a.layer[l].norm1, sm.z);
        tl_mark<Cfg::kDiag>(a, sm, kTlNorm1);
        for (int h = (int)cp.id; h < a.heads; h += (int)cp.count) {
          attention_head<T, Cfg>(a, l, s, h, cp, sm, rg, rs);
          if (h + (int)cp.count < a.heads) cluster_sync();
        }
      }
      if (!gs.sync(a, a.bar_timeout_ns, &sm.sync_ok, Cfg::kDiag ? &sm : nullptr, Cfg::kRing ? &rg : nullptr, &rs)) return false;
      residual_from_heads<T>(a, s, sm);
      tl_mark<Cfg::kDiag>(a, sm, kTlResidualHeads);
      block_ffn<T, Cfg>(a, l, s, cp, sm, rg, rs);
      if (!gs.sync(a, a.bar_timeout_ns, &sm.sync_ok, Cfg::kDiag ? &sm : nullptr, Cfg::kRing ? &rg : nullptr, &rs)) return false;
      residual_from_clusters<T>(a, s, (int)cp.count, sm);
      tl_mark<Cfg::kDiag>(a, sm, kTlResidualClusters);
      if (is_score_cta()) write_hidden(a, s, l, sm.xres);
    }
    if (is_score_cta()) block_score<T>(a, s, sm, score_out);
  }
  if (advance && is_score_cta())
    for (int s = threadIdx.x; s < a.streams; s += kThreads) a.position[s] = ld_cg_u64(a.position + s) + 1;
  return true;
}

__host__ __device__ inline int forward2_barriers(int layers, int streams) { return 2 * layers * streams; }

// ---------------------------------------------------------------- per-op kernels' bodies
// The per-op kernels also serve st_trace_step, so they carry the trace hooks.
using OpCfg = StepCfg<false, true>;

// Residual state crosses kernels through a.x (x entering the layer / after it)
// and a.x2 (x' after attention), written by CTA 0. They run the direct-load
// block functions, which give the same bits as the ring ones.
template <typename T>
__device__ void op_input(const StepArgs& a, Smem2& sm, RingSmem& rs) {
  const ClusterPos cp = ClusterPos::get();
  Ring off{};
  for (int s = 0; s < a.streams; ++s) {
    step_input<T, OpCfg>(a, s, a.input, cp, sm, off, rs);
    if (blockIdx.x == 0) {
      float* xg = a.x + (size_t)s * a.width;
      for (int i = threadIdx.x; i < a.width; i += kThreads) xg[i] = sm.xres[i];
    }
    __syncthreads();
  }
}

// Layer l's attention block; for l > 0 it first completes layer l-1's residual
// from a.x2 and the down partials.
template <typename T>
__device__ void op_attention(const StepArgs& a, int l, Smem2& sm, RingSmem& rs) {
  const ClusterPos cp = ClusterPos::get();
  Ring off{};
  for (int s = 0; s < a.streams; ++s) {
    load_position(a, s, sm);
    if (l == 0) {
      for (int i = threadIdx.x; i < a.width; i += kThreads) sm.xres[i] = ld_cg(a.x + (size_t)s * a.width + i);
    } else {
      for (int i = threadIdx.x; i < a.width; i += kThreads) sm.x2res[i] = ld_cg(a.x2 + (size_t)s * a.width + i);
      residual_from_clusters<T>(a, s, (int)cp.count, sm);
      if (blockIdx.x == 0) write_hidden(a, s, l - 1, sm.xres);
    }
    norm_block<T, OpCfg>(a, off, rs, sm, sm.xres, (const T*)a.layer[l].norm1, sm.z);
    rope_table(a, sm);
    __syncthreads();
    for (int h = (int)cp.id; h < a.heads; h += (int)cp.count) {
      attention_head<T, OpCfg>(a, l, s, h, cp, sm, off, rs);
      if (h + (int)cp.count < a.heads) cluster_sync();
    }
    cluster_sync();  // sm.t, z and the attention buffers are reused by the next stream
  }
}

template <typename T>
__device__ void op_ffn(const StepArgs& a, int l, Smem2& sm, RingSmem& rs) {
  const ClusterPos cp = ClusterPos::get();
  Ring off{};
  for (int s = 0; s < a.streams; ++s) {
    for (int i = threadIdx.x; i < a.width; i += kThreads) sm.xres[i] = ld_cg(a.x + (size_t)s * a.width + i);
    residual_from_heads<T>(a, s, sm);
    if (blockIdx.x == 0) {
      float* x2 = a.x2 + (size_t)s * a.width;
      for (int i = threadIdx.x; i < a.width; i += kThreads) x2[i] = sm.x2res[i];
    }
    block_ffn<T, OpCfg>(a, l, s, cp, sm, off, rs);
    cluster_sync();  // the FFN buffers are reused by the next stream
  }
}

// Completes the last layer, the score and position++ (CTA 0 of cluster 0 only).
template <typename T>
__device__ void op_final(const StepArgs& a, int nclusters, Smem2& sm) {
  if (blockIdx.x != 0) return;
  for (int s = 0; s < a.streams; ++s) {
    for (int i = threadIdx.x; i < a.width; i += kThreads) sm.x2res[i] = ld_cg(a.x2 + (size_t)s * a.width + i);
    residual_from_clusters<T>(a, s, nclusters, sm);
    write_hidden(a, s, a.layers - 1, sm.xres);
    block_score<T>(a, s, sm);
  }
  for (int s = threadIdx.x; s < a.streams; s += kThreads) a.position[s] = ld_cg_u64(a.position + s) + 1;
}

}  // namespace st
