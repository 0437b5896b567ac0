// st_chain.cuh -- the single-stream step at the benchmark shapes with a small
// instruction footprint (k5_chain).
//
// Same work split, exchange protocol, weight ring and arithmetic as k4_flow
// (st_flow.cuh): NC clusters of CS CTAs, cluster c owns heads c, c + NC, ...,
// rank r owns segment r of the width; tagged records {fp32, tag} carry the
// head partials (exchange 1) and the cluster down partials (exchange 2)
// through L2; st.async stores completing on the receiver's mbarrier carry
// q/k/v, the attention partials, the down reduce-scatter and x inside a
// cluster; a producer warp streams every CTA's fixed chunk table into a
// shared-memory ring with cp.async.bulk. The cast points are the reference
// step's (reference src/cpu/Cpu.cpp:59-141).
//
// Why a second kernel: the step is a serial chain of short phases, and each
// phase runs once per layer, so its instructions are fetched again every
// layer unless the whole per-layer body stays in the SM's instruction caches.
// Measured on B200 (a straight-line probe): about 1.2 cycles per instruction
// from the first-level cache (<= 8 KB), 2.7 from the second (<= 32 KB) and
// 5.9 beyond it; k4_flow's per-layer code is ~78 KB, and its device time per
// step moved by ~1 us per KB removed. This kernel keeps the per-layer code
// small by construction:
//   - two GEMV routines (rows spanning the warp for K = D; short rows for the
//     32 features and head_dim), each holding every epilogue it serves behind
//     a switch, so the q/k/v and gate/up spans share one copy of the loop and
//     the input and out-projection spans another;
//   - epilogues spread over lanes (every lane of a row group holds the sums;
//     lane r stores into cluster rank r), not loops over ranks;
//   - one merge routine for the warp and the cluster softmax partials, one
//     gather routine for both tagged-record exchanges, a compact publish;
//   - remote shared-memory addresses mapped once per head, reciprocal square
//     root and fast division (a few ulp in fp32, within the fp32 1e-5 relative
//     bound), 32-bit index arithmetic, and the phase timeline compiled into a
//     separate diagnostic instantiation only.
#pragma once

#include "st_flow.cuh"

namespace st {

// Phase marks only in the diagnostic instantiation (kDiag).
template <bool kDiag>
__device__ __forceinline__ void cmark(const StepArgs& a, FlowRing& fr, int tag) {
  if constexpr (kDiag) fmark(a, fr, tag);
}

// Epilogues of the GEMV routines.
enum ChainEpi : int { kEpiQkv = 0, kEpiGateUp = 1, kEpiIn = 2, kEpiOut = 3 };

// Per-span epilogue parameters, in shared memory (set before the span).
struct ChainEpiArgs {
  unsigned qkv_remote[kFlowMaxCluster];   // q/k/v receive buffer in each cluster rank (shared::cluster)
  unsigned qbar_remote[kFlowMaxCluster];  // its mbarrier in each rank
  void* kslot;                            // this step's ring row of the head: keys (global)
  void* vslot;                            // values
  unsigned long long* P;                  // out-projection records of this head, at this rank's segment
  unsigned tag;
  int lo;                                 // first q/k/v row pair of this rank within the head
  int cs;
};

struct alignas(128) ChainSmem {
  unsigned long long sbar[kSites][2];    // receive mbarriers per site and parity
  float x[2][kFlowMaxD];                 // residual entering the layer (site X)
  float x2[kFlowMaxD];                   // residual after attention (whole width)
  float z[kFlowMaxD];                    // norm output, GEMV input
  float dred[2][kFlowMaxD];              // down partials from every rank, [CS][n] (site DRED)
  float seg[kFlowMaxD];                  // this rank's segment values before publishing
  float fnorm[kFlowMaxD];                // final norm gain (score CTA)
  float fscore[kFlowMaxD];               // score weights (score CTA)
  float qkv[2][3 * kFlowHd];             // q, k, v of the current head (site QKV)
  float apart[2][kFlowMaxCluster][kFlowHd + 2];  // CTA attention partials per rank (site ATT)
  float wpart[kWarps][kFlowHd + 2];      // warp attention partials (m, l, acc)
  alignas(16) float o[kFlowHd];          // merged attention output (cast)
  float act[kFlowMaxAct];                // this CTA's SwiGLU slice
  float ssx[2][kFlowMaxCluster][8];      // sum of squares of x per rank and warp (site X)
  int okx[2][kFlowMaxCluster];           // verdict per rank (site X)
  int oksetup[kFlowMaxCluster];          // launch setup verdict per rank
  float2 rope_cs[kFlowHd / 2];           // cos, sin of t * frequency
  float rope[kFlowHd / 2];               // frequencies 10000^(-2i/hd)
  alignas(16) float ev[kFlowFeatures];   // the event
  float warp_scratch[kWarps];
  unsigned long long cmd;                // persistent: the dispatched command
  FlowPlan plan;                         // this CTA's span geometry
  ChainEpiArgs ep;                       // epilogue parameters of the current span
  union {
    alignas(16) unsigned char kv[kFlowKvBytes];   // K rows then V rows of this CTA's slots
    float red[kFlowKvBytes / 4];                   // gather / down group partials
  } u;
};

constexpr size_t kChainRingOffset = (sizeof(ChainSmem) + sizeof(FlowRing) + 127) / 128 * 128;
constexpr unsigned kChainRingCapacity = (unsigned)((kFlowSmemBytes - kChainRingOffset) / 128 * 128);
static_assert(kChainRingCapacity >= 2 * kFlowChunkMax, "the chain ring needs room for two chunks");

// st.async of two floats to a remote shared::cluster address, completing 8
// bytes on the remote mbarrier.
__device__ __forceinline__ void st_async2_at(unsigned remote, unsigned remote_bar, float v0, float v1) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];"
               ::"r"(remote), "f"(v0), "f"(v1), "r"(remote_bar) : "memory");
}
__device__ __forceinline__ void ll_store1(unsigned long long* p, float v, unsigned tag) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(ll_pack(v, tag)) : "memory");
}

// ---------------------------------------------------------------- GEMV routines
// Rows [0, nrows) of a ring chunk (row stride D, rows in pairs), two rows per
// warp pass, passes dealt to warps from pass0; x (shared memory) in registers
// for the call. Every lane ends a pass with both sums, and the epilogue `kind`
// consumes them (row r0 + r of the span):
//   kEpiQkv     RoPE on q/k rows, casts, the pair into every rank's q/k/v
//               buffer (lane r -> rank r), k/v into the ring slot (lane 31)
//   kEpiGateUp  act[pair] = cast(silu(cast(gate)) * cast(up))  (lane 0)
// Compute warps only; no barrier inside.
template <typename T, int D>
static __device__ __noinline__ void chain_rows(int kind, const T* rows, int nrows, int r0, int pass0, const float* xs,
                                               ChainSmem* smp) {
  using R = FlowRow<T, D>;
  static_assert(R::LPR == 32, "wide rows span the warp");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  FlowX<T, D> x;
  x.load(xs);
  const int passes = (nrows + 1) >> 1;
#pragma unroll 1
  for (int p = (warp - pass0 % kWarps + kWarps) % kWarps; p < passes; p += kWarps) {
    const int r = 2 * p;
    const T* p0 = rows + r * D + lane * R::V;
    const T* p1 = r + 1 < nrows ? p0 + D : p0;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int k = 0; k < R::VPL; ++k) {
      const uint4 w0 = ld_shared_v4(p0 + k * 32 * R::V);
      const uint4 w1 = ld_shared_v4(p1 + k * 32 * R::V);
      a0 += dot_regs<T>(w0, x.v + k * R::V);
      a1 += dot_regs<T>(w1, x.v + k * R::V);
    }
    // the upper half-warp keeps row 1, the lower row 0; then every lane takes both
    const bool hi = (lane & 16) != 0;
    float s = (hi ? a1 : a0) + __shfl_xor_sync(0xffffffffu, hi ? a0 : a1, 16);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float v0 = __shfl_sync(0xffffffffu, s, 0), v1 = __shfl_sync(0xffffffffu, s, 16);
    const int row = r0 + r;
    if (kind == kEpiQkv) {
      const ChainEpiArgs& e = smp->ep;
      const int grow = 2 * e.lo + row;
      const int which = grow >> 6, dim = grow & (kFlowHd - 1);
      float q0 = Storage<T>::round(v0), q1 = Storage<T>::round(v1);
      if (which < 2) {
        const float2 c = smp->rope_cs[dim >> 1];
        const float r0v = q0 * c.x - q1 * c.y;
        const float r1v = q0 * c.y + q1 * c.x;
        q0 = Storage<T>::round(r0v);
        q1 = Storage<T>::round(r1v);
      }
      if (lane < e.cs) st_async2_at(e.qkv_remote[lane] + 4u * grow, e.qbar_remote[lane], q0, q1);
      if (which > 0 && lane == 31) {
        T* ring = (T*)(which == 1 ? e.kslot : e.vslot);
        Storage<T>::store(ring, dim, q0);
        Storage<T>::store(ring, dim + 1, q1);
      }
    } else if (lane == 0) {
      const float gt = Storage<T>::round(v0), up = Storage<T>::round(v1);
      smp->act[row >> 1] = Storage<T>::round(__fdividef(gt, 1.0f + expf(-gt)) * up);
    }
  }
}

// Short rows (K = V * nv elements, nv a power of two <= 32 vectors: the 32
// features of the input projection, head_dim of the out-projection), 32 / nv
// rows per warp pass, one 16-byte vector per lane. Epilogues (lane 0 of the
// row's lanes): kEpiIn seg[row] = cast(sum); kEpiOut the tagged record
// P[row] = {sum, tag}.
template <typename T>
static __device__ __noinline__ void chain_rows_short(int kind, const T* rows, int nrows, int K, int r0, int pass0,
                                                     const float* xs, ChainSmem* smp) {
  constexpr int V = Storage<T>::kVec;
  const int nv = K / V, rpw = 32 / nv;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / nv, sl = lane - sub * nv;
  float xv[V];
#pragma unroll
  for (int e = 0; e < V; e += 4) {
    const float4 q = *reinterpret_cast<const float4*>(xs + sl * V + e);
    xv[e] = q.x;
    xv[e + 1] = q.y;
    xv[e + 2] = q.z;
    xv[e + 3] = q.w;
  }
  const int passes = (nrows + rpw - 1) / rpw;
#pragma unroll 1
  for (int p = (warp - pass0 % kWarps + kWarps) % kWarps; p < passes; p += kWarps) {
    const int r = p * rpw + sub;
    const bool valid = r < nrows;
    float acc = dot_regs<T>(ld_shared_v4(rows + (valid ? r : 0) * K + sl * V), xv);
#pragma unroll 1
    for (int o = nv >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (valid && sl == 0) {
      if (kind == kEpiIn) smp->seg[r0 + r] = Storage<T>::round(acc);
      else ll_store1(smp->ep.P + r0 + r, acc, smp->ep.tag);
    }
  }
}

// ---------------------------------------------------------------- softmax partials
struct ChainMLA {
  float m, l, a;
};
// Merge of n partials (m, l, acc[hd]) of stride `stride` floats into (M, L,
// A[dim]); partials with l = 0 are empty. Called by the thread owning `dim`.
static __device__ __noinline__ ChainMLA chain_merge(const float* st, int n, int stride, int dim) {
  float M = -INFINITY;
#pragma unroll 1
  for (int k = 0; k < n; ++k)
    if (st[k * stride + 1] > 0.f) M = fmaxf(M, st[k * stride]);
  float L = 0.f, A = 0.f;
#pragma unroll 1
  for (int k = 0; k < n; ++k) {
    const float l = st[k * stride + 1];
    if (l > 0.f) {
      const float s = expf(st[k * stride] - M);
      L = fmaf(l, s, L);
      A = fmaf(st[k * stride + 2 + dim], s, A);
    }
  }
  return {M, L, A};
}

// ---------------------------------------------------------------- waits
// The next ring chunk (bounded wait); after a failed wait the ring is marked
// failed and every later acquire returns the buffer start at once (the error
// word ends the launch at its next exchange).
static __device__ __noinline__ const unsigned char* chain_acquire(FlowRing& fr, unsigned long long consumed,
                                                                  int* error, int* host_error,
                                                                  unsigned long long timeout_ns) {
  const int slot = (int)(consumed % kFlowSlots);
  const unsigned parity = (unsigned)((consumed / kFlowSlots) & 1ull);
  if (!mbar_try_wait(&fr.full[slot], parity) && !*reinterpret_cast<volatile int*>(&fr.failed) &&
      !flow_wait_slow(fr, slot, parity, timeout_ns)) {
    fr.failed = 1;
    flow_error(error, host_error, kBarrierTimeout);
  }
  return fr.buf + (*reinterpret_cast<volatile int*>(&fr.failed) ? 0u : fr.off[slot]);
}

// Receive exchange k of a site (thread 0 arms the mbarrier with the bytes
// every rank sends; every thread waits, bounded).
static __device__ __noinline__ bool chain_receive(unsigned long long* bar, unsigned k, unsigned bytes, int* error,
                                                  int* host_error, unsigned long long timeout_ns) {
  const unsigned parity = (k >> 1) & 1u;
  if (threadIdx.x == 0) mbar_expect_tx(bar, bytes);
  return mbar_try_wait_cluster(bar, parity) || flow_receive_slow(bar, parity, error, host_error, timeout_ns);
}
__device__ __forceinline__ bool chain_recv(const StepArgs& a, ChainSmem& sm, int site, unsigned k, unsigned bytes) {
  return chain_receive(&sm.sbar[site][k & 1u], k, bytes, a.error, a.host_error, a.bar_timeout_ns);
}

// Sum over sources src < nsrc of the tagged records rec[src * stride + e0 + i],
// i < n (n / 2 a power of two <= kThreads), into out[i], sources added in index
// order: thread t polls element pair t % (n / 2) for the sources congruent to
// t / (n / 2) (four per round trip), partial sums meet in red. False (error
// word set) when a wait ran out or another CTA failed. Every compute thread;
// ends with a compute-thread barrier.
static __device__ __noinline__ bool chain_gather(const unsigned long long* rec, int stride, int nsrc, int e0, int n,
                                                 unsigned tag, float* red, float* out, int* error, int* host_error,
                                                 unsigned long long timeout_ns) {
  const int np = n >> 1, lg = 31 - __clz(np), G = kThreads >> lg;
  const int e = (int)threadIdx.x & (np - 1), g = (int)threadIdx.x >> lg;
  float s0 = 0.f, s1 = 0.f;
  bool ok = true;
  unsigned long long start = 0;
  unsigned polls = 0;
#pragma unroll 1
  for (int src0 = g; src0 < nsrc && ok; src0 += 4 * G) {
    unsigned long long r[4][2];
#pragma unroll 1
    while (true) {
      bool ready = true;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int src = src0 + k * G;
        if (src < nsrc) {
          ll_load2(rec + src * stride + e0 + 2 * e, r[k][0], r[k][1]);
          ready = ready && ll_tag(r[k][0]) == tag && ll_tag(r[k][1]) == tag;
        } else {
          r[k][0] = r[k][1] = 0ull;
        }
      }
      if (ready) break;
      if ((++polls & 31u) == 0) {
        if (ld_volatile_int(error) != 0) { ok = false; break; }
        const unsigned long long now = globaltimer();
        if (start == 0) start = now;
        else if (now - start > timeout_ns) { flow_error(error, host_error, kBarrierTimeout); ok = false; break; }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s0 += ll_value(r[k][0]);
      s1 += ll_value(r[k][1]);
    }
  }
  red[g * n + 2 * e] = s0;
  red[g * n + 2 * e + 1] = s1;
  ok = flow_bar_and(ok);
#pragma unroll 1
  for (int i = threadIdx.x; i < n; i += kThreads) {
    float t = 0.f;
#pragma unroll 1
    for (int k = 0; k < G; ++k) t += red[k * n + i];
    out[i] = t;
  }
  flow_bar();
  return ok;
}

// Publish this rank's segment seg[i], i < n, into dst of every rank (thread
// (r, e) sends pair e to rank r), with the segment's per-warp sums of squares
// ss[rank][w] (lane r of warp w sends to rank r) and this CTA's verdict
// okv[rank]; then receive every rank's part. Returns the cluster's verdict.
static __device__ __noinline__ bool chain_publish(const float* seg, float* dst, float* ss, int* okv,
                                                  unsigned long long* bar, unsigned k, unsigned rank, unsigned cs,
                                                  int seg0, int n, bool ok, int* error, int* host_error,
                                                  unsigned long long timeout_ns) {
  const int np = n >> 1, nw = (np + 31) >> 5, t = (int)threadIdx.x;
  if (t < (int)cs * np) {
    const unsigned r = (unsigned)t / (unsigned)np;
    const int e = t - (int)r * np;
    st_async2(dst + seg0 + 2 * e, bar, r, seg[2 * e], seg[2 * e + 1]);
  }
  if (t < nw * 32) {
    float q = 0.f;
    if (t < np) q = seg[2 * t] * seg[2 * t] + seg[2 * t + 1] * seg[2 * t + 1];
    q = warp_sum(q);
    const int lane = t & 31;
    if (lane < (int)cs) st_async1(&ss[rank * 8 + (t >> 5)], bar, (unsigned)lane, q);
  }
  if (t < (int)cs) st_async1i(&okv[rank], bar, (unsigned)t, ok ? 1 : 0);
  bool all = chain_receive(bar, k, cs * (unsigned)(4 * n + 4 * nw + 4), error, host_error, timeout_ns);
#pragma unroll 1
  for (unsigned r = 0; r < cs; ++r) all = all && (*reinterpret_cast<volatile int*>(&okv[r]) != 0);
  return all;
}
__device__ __forceinline__ bool chain_publish_x(const StepArgs& a, ChainSmem& sm, FlowCtx& cx, bool ok) {
  const unsigned k = cx.k[kSiteX]++;
  const unsigned b = k & 1u;
  const bool all = chain_publish(sm.seg, sm.x[b], &sm.ssx[b][0][0], sm.okx[b], &sm.sbar[kSiteX][b], k, cx.rank, cx.cs,
                                 cx.seg0, cx.n, ok, a.error, a.host_error, a.bar_timeout_ns);
  cx.bx = b;
  return all;
}

// 1 / sqrt(mean(x^2) + eps) from the published per-rank, per-warp sums.
__device__ __forceinline__ float chain_norm_scale(const float (*ss)[8], unsigned cs, int n, int d, float eps) {
  const int nw = ((n >> 1) + 31) >> 5;
  float t = 0.f;
#pragma unroll 1
  for (unsigned r = 0; r < cs; ++r)
#pragma unroll 1
    for (int w = 0; w < nw; ++w) t += ss[r][w];
  return rsqrtf(t * (1.0f / (float)d) + eps);
}

// ---------------------------------------------------------------- ring spans
// Every chunk of span sp acquired, passed to fn(base, r0, rows, pass0) and
// released; pr rows per warp pass (the routine's pass dealing continues across
// chunks).
template <typename Fn>
__device__ __forceinline__ void chain_span(const StepArgs& a, FlowRing& fr, FlowCur& cur, const FlowSpan sp, int pr,
                                           Fn&& fn) {
  int pass0 = 0;
#pragma unroll 1
  for (int c = 0; c < sp.chunks; ++c) {
    const int r0 = c * sp.rpc;
    const int n = min(sp.rpc, sp.rows - r0);
    fn(chain_acquire(fr, cur.consumed, a.error, a.host_error, a.bar_timeout_ns), r0, n, pass0);
    flow_release(fr, cur);
    pass0 += (n + pr - 1) / pr;
  }
}

// A norm gain (one-row span): z[i] = cast(x[i] * scale * g[i]), then a barrier.
template <typename T, int D>
__device__ __forceinline__ void chain_norm(const StepArgs& a, FlowRing& fr, FlowCur& cur, const float* x, float scale,
                                           float* z) {
  const T* g = (const T*)chain_acquire(fr, cur.consumed, a.error, a.host_error, a.bar_timeout_ns);
#pragma unroll 1
  for (int i = threadIdx.x; i < D; i += kThreads) z[i] = Storage<T>::round(x[i] * scale * Storage<T>::load(g, i));
  flow_release(fr, cur);
  flow_bar();
}

// ---------------------------------------------------------------- attention per head
// One head h of layer l: q/k/v rows, attention over this CTA's slots, the
// out-projection rows of this rank's segment published as P[h]. False when a
// wait ran out (the error word is set; the next exchange ends the launch).
template <typename T, int D, bool kDiag>
__device__ __forceinline__ bool chain_head(const StepArgs& a, FlowRing& fr, FlowCur& cur, ChainSmem& sm,
                                           FlowCtx& cx, int l, int h, unsigned tag, bool first_head) {
  constexpr int hd = kFlowHd;
  const int W = a.window, slot = cx.slot;
  T* keys = (T*)a.keys + ((unsigned)(l * a.heads + h) * (unsigned)W) * (size_t)hd;
  T* values = (T*)a.values + ((unsigned)(l * a.heads + h) * (unsigned)W) * (size_t)hd;
  int j0, j1;
  split(cx.valid, (int)cx.rank, (int)cx.cs, j0, j1);
  // K and V rows of this CTA's slots into shared memory (the slot this step
  // overwrites comes from the q/k/v exchange instead)
  const int nj = j1 - j0;
  const bool kv_smem = 2 * nj * hd * (int)sizeof(T) <= kFlowKvBytes;
  if (kv_smem) {
    constexpr int vpr = hd * (int)sizeof(T) / 16;
    const int vecs = nj * vpr;
#pragma unroll 1
    for (int i = threadIdx.x; i < 2 * vecs; i += kThreads) {
      const bool is_v = i >= vecs;
      const int k = is_v ? i - vecs : i;
      if (j0 + k / vpr == slot) continue;
      cp_async16(sm.u.kv + i * 16, (const char*)(is_v ? values : keys) + (j0 * hd * (int)sizeof(T) + k * 16));
    }
    cp_async_commit();
  }
  // epilogue parameters of the q/k/v span
  const unsigned kq = cx.k[kSiteQkv]++, bq = kq & 1u;
  if (threadIdx.x < cx.cs) {
    sm.ep.qkv_remote[threadIdx.x] = flow_remote(&sm.qkv[bq][0], threadIdx.x);
    sm.ep.qbar_remote[threadIdx.x] = flow_remote(&sm.sbar[kSiteQkv][bq], threadIdx.x);
  }
  if (threadIdx.x == 0) {
    sm.ep.kslot = keys + slot * hd;
    sm.ep.vslot = values + slot * hd;
    sm.ep.lo = sm.plan.qkv_lo;
    sm.ep.cs = (int)cx.cs;
  }
  if (first_head) chain_norm<T, D>(a, fr, cur, sm.x[cx.bx], chain_norm_scale(sm.ssx[cx.bx], cx.cs, cx.n, D, a.epsilon),
                                   sm.z);
  else flow_bar();
  cmark<kDiag>(a, fr, kFmNorm1);
  chain_span(a, fr, cur, sm.plan.qkv, 2, [&](const unsigned char* base, int r0, int n, int pass0) {
    chain_rows<T, D>(kEpiQkv, (const T*)base, n, r0, pass0, sm.z, &sm);
  });
  cmark<kDiag>(a, fr, kFmQkv);
  // this CTA's K/V copies, then every rank's q/k/v rows
  if (kv_smem) cp_async_wait_all();
  flow_bar();
  const float* qkv = sm.qkv[bq];
  bool ok = chain_recv(a, sm, kSiteQkv, kq, 3u * hd * 4u);
  cmark<kDiag>(a, fr, kFmQkvSync);
  // attention over this CTA's slots: an online softmax per warp
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const T* Ks = reinterpret_cast<const T*>(sm.u.kv);
    const T* Vs = Ks + nj * hd;
    const float2 q = *reinterpret_cast<const float2*>(&qkv[2 * lane]);
    float m = -INFINITY, lsum = 0.f, acc0 = 0.f, acc1 = 0.f;
#pragma unroll 1
    for (int j = j0 + warp; j < j1; j += kWarps) {
      float k0, k1, v0, v1;
      if (j == slot) {
        k0 = qkv[hd + 2 * lane];
        k1 = qkv[hd + 2 * lane + 1];
        v0 = qkv[2 * hd + 2 * lane];
        v1 = qkv[2 * hd + 2 * lane + 1];
      } else if (kv_smem) {
        k0 = Storage<T>::load(Ks + (j - j0) * hd, 2 * lane);
        k1 = Storage<T>::load(Ks + (j - j0) * hd, 2 * lane + 1);
        v0 = Storage<T>::load(Vs + (j - j0) * hd, 2 * lane);
        v1 = Storage<T>::load(Vs + (j - j0) * hd, 2 * lane + 1);
      } else {
        k0 = Storage<T>::load_cg(keys + j * hd, 2 * lane);
        k1 = Storage<T>::load_cg(keys + j * hd, 2 * lane + 1);
        v0 = Storage<T>::load_cg(values + j * hd, 2 * lane);
        v1 = Storage<T>::load_cg(values + j * hd, 2 * lane + 1);
      }
      const float s = warp_sum(fmaf(q.y, k1, q.x * k0)) * (1.0f / 8.0f);  // 1 / sqrt(head_dim 64), exact
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
  flow_bar();
  cmark<kDiag>(a, fr, kFmAttn);
  // this CTA's partial (M, L, A[dim]) from the warp partials, into every rank
  const unsigned ka = cx.k[kSiteAtt]++, ba = ka & 1u;
  float(*apart)[kFlowHd + 2] = sm.apart[ba];
  if (threadIdx.x < hd) {
    const ChainMLA r = chain_merge(&sm.wpart[0][0], kWarps, hd + 2, threadIdx.x);
    const unsigned long long* abar = &sm.sbar[kSiteAtt][ba];
#pragma unroll 1
    for (unsigned k = 0; k < cx.cs; ++k) st_async1(&apart[cx.rank][2 + threadIdx.x], abar, k, r.a);
    if (threadIdx.x < cx.cs) st_async2(&apart[cx.rank][0], abar, threadIdx.x, r.m, r.l);
  }
  ok = chain_recv(a, sm, kSiteAtt, ka, cx.cs * (unsigned)(4 * hd + 8)) && ok;
  cmark<kDiag>(a, fr, kFmPartSync);
  // merge the cluster's partials in rank order -> o (cast); out-projection
  // parameters for the span that follows
  if (threadIdx.x < hd) {
    const ChainMLA r = chain_merge(&apart[0][0], (int)cx.cs, hd + 2, threadIdx.x);
    sm.o[threadIdx.x] = Storage<T>::round(__fdividef(r.a, r.l));
  }
  if (threadIdx.x == 0) {
    sm.ep.P = a.ll_heads + ((unsigned)((tag & 1u) * a.heads + h) * (unsigned)D + cx.seg0);
    sm.ep.tag = tag;
  }
  flow_bar();
  cmark<kDiag>(a, fr, kFmMerge);
  // out-projection rows of this rank's segment (K-split by head) -> P[h][seg]
  chain_span(a, fr, cur, sm.plan.out, 32 / (hd / Storage<T>::kVec),
             [&](const unsigned char* base, int r0, int n, int pass0) {
               chain_rows_short<T>(kEpiOut, (const T*)base, n, hd, r0, pass0, sm.o, &sm);
             });
  cmark<kDiag>(a, fr, kFmOut);
  return ok;
}

// ---------------------------------------------------------------- one step
template <typename T, int D, bool kDiag>
__device__ __forceinline__ bool chain_step(const StepArgs& a, FlowRing& fr, FlowCur& cur, ChainSmem& sm, FlowCtx& cx,
                                           const float* event, unsigned long long t, float* score_dst,
                                           float* score_copy) {
  const int n = cx.n, seg0 = cx.seg0;
  cmark<kDiag>(a, fr, kFmStep);
  cx.slot = t < 0xffffffffull ? (int)((unsigned)t % (unsigned)a.window) : (int)(t % (unsigned long long)a.window);
  cx.valid = t + 1 < (unsigned long long)a.window ? (int)(t + 1) : a.window;
  if (threadIdx.x < kFlowFeatures) sm.ev[threadIdx.x] = __ldcv(event + threadIdx.x);
  if (threadIdx.x < kFlowHd / 2) {
    float sn, cs;
    sincosf((float)t * sm.rope[threadIdx.x], &sn, &cs);
    sm.rope_cs[threadIdx.x] = make_float2(cs, sn);
  }
  flow_bar();
  // x[seg] = cast(W_in[seg] e)
  chain_span(a, fr, cur, sm.plan.in, 32 / (kFlowFeatures / Storage<T>::kVec),
             [&](const unsigned char* base, int r0, int rows, int pass0) {
               chain_rows_short<T>(kEpiIn, (const T*)base, rows, kFlowFeatures, r0, pass0, sm.ev, &sm);
             });
  flow_bar();
  if (!chain_publish_x(a, sm, cx, !fr.failed)) return false;
  cmark<kDiag>(a, fr, kFmIn);
#pragma unroll 1
  for (int l = 0; l < a.layers; ++l) {
    const unsigned tag = (unsigned)(cx.epoch + cx.steps * (unsigned long long)a.layers + (unsigned long long)l + 1ull);
    bool hok = true;
    if (cx.heads_here)
#pragma unroll 1
      for (int h = (int)cx.id; h < a.heads; h += (int)cx.nc)
        hok = chain_head<T, D, kDiag>(a, fr, cur, sm, cx, l, h, tag, h == (int)cx.id) && hok;
    // exchange 1 (whole width): x' = cast(x + cast(sum_h P[h])), and sum(x'^2)
    float ssq = 0.f;
    const bool ok1 = chain_gather(a.ll_heads + (tag & 1u) * (unsigned)(a.heads * D), D, a.heads, 0, D, tag, sm.u.red,
                                  sm.x2, a.error, a.host_error, a.bar_timeout_ns) && hok && !fr.failed;
    {
      const float* x = sm.x[cx.bx];
      float q = 0.f;
#pragma unroll 1
      for (int i = threadIdx.x; i < D; i += kThreads) {
        const float v = Storage<T>::round(x[i] + Storage<T>::round(sm.x2[i]));
        sm.x2[i] = v;
        q = fmaf(v, v, q);
      }
      q = warp_sum(q);
      if ((threadIdx.x & 31) == 0) sm.warp_scratch[threadIdx.x >> 5] = q;
      flow_bar();
#pragma unroll 1
      for (int w = 0; w < kWarps; ++w) ssq += sm.warp_scratch[w];
      cmark<kDiag>(a, fr, kFmGather1);
    }
    // FFN: norm2, gate/up -> SwiGLU, down partial
    chain_norm<T, D>(a, fr, cur, sm.x2, rsqrtf(ssq * (1.0f / (float)D) + a.epsilon), sm.z);
    cmark<kDiag>(a, fr, kFmNorm2);
    chain_span(a, fr, cur, sm.plan.gateup, 2, [&](const unsigned char* base, int r0, int rows, int pass0) {
      chain_rows<T, D>(kEpiGateUp, (const T*)base, rows, r0, pass0, sm.z, &sm);
    });
    flow_bar();
    cmark<kDiag>(a, fr, kFmGateUp);
    bool dok;
    {
      // partial[col] = sum_f act[f] W_down^T[f][col]: thread t owns 16-byte
      // column vector t % NVd and rows f = g, g + G2, ... of the slice.
      using R = FlowRow<T, D>;
      constexpr int NVd = R::NV, G2 = kThreads / NVd, V = R::V;
      const int cv = (int)threadIdx.x % NVd, g = (int)threadIdx.x / NVd;
      float acc[V];
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] = 0.f;
      const FlowSpan sp = sm.plan.down;
#pragma unroll 1
      for (int c = 0; c < sp.chunks; ++c) {
        const int r0 = c * sp.rpc;
        const int rows = min(sp.rpc, sp.rows - r0);
        const T* base = (const T*)chain_acquire(fr, cur.consumed, a.error, a.host_error, a.bar_timeout_ns);
#pragma unroll 1
        for (int f = ((g - r0) % G2 + G2) % G2; f < rows; f += G2) {
          const float av = sm.act[r0 + f];
          float w[V];
          Storage<T>::unpack(ld_shared_v4(base + f * D + cv * V), w);
#pragma unroll
          for (int k = 0; k < V; ++k) acc[k] = fmaf(w[k], av, acc[k]);
        }
        flow_release(fr, cur);
      }
      cmark<kDiag>(a, fr, kFmDown);
      // sm.u.red was last read by exchange 1, before its barrier.
#pragma unroll
      for (int k = 0; k < V; k += 4)
        *reinterpret_cast<float4*>(&sm.u.red[g * D + cv * V + k]) = make_float4(acc[k], acc[k + 1], acc[k + 2], acc[k + 3]);
      flow_bar();
      // column sums in group order, sent in float4s to the rank owning them
      const unsigned kd = cx.k[kSiteDred]++, bd = kd & 1u;
      float* dred = sm.dred[bd];
      const unsigned long long* dbar = &sm.sbar[kSiteDred][bd];
#pragma unroll 1
      for (int c4 = threadIdx.x; c4 < D / 4; c4 += kThreads) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
        for (int k = 0; k < G2; ++k) {
          const float4 q = *reinterpret_cast<const float4*>(&sm.u.red[k * D + 4 * c4]);
          s.x += q.x; s.y += q.y; s.z += q.z; s.w += q.w;
        }
        const int col = 4 * c4, owner = col / n;
        st_async4(&dred[cx.rank * n + (col - owner * n)], dbar, (unsigned)owner, s);
      }
      dok = chain_recv(a, sm, kSiteDred, kd, cx.cs * (unsigned)n * 4u);
      cmark<kDiag>(a, fr, kFmDredSync);
      // this rank's segment of the cluster partial, ranks added in order
      unsigned long long* Dp = a.ll_clusters + ((tag & 1u) * cx.nc + cx.id) * (unsigned)D + seg0;
#pragma unroll 1
      for (int i = 2 * threadIdx.x; i < n; i += 2 * kThreads) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll 1
        for (unsigned r = 0; r < cx.cs; ++r) {
          s0 += dred[r * n + i];
          s1 += dred[r * n + i + 1];
        }
        ll_store2(Dp + i, s0, s1, tag);
      }
      cmark<kDiag>(a, fr, kFmDpub);
    }
    // exchange 2: x[seg] = cast(x'[seg] + cast(sum_c D[c][seg]))
    {
      const bool ok = chain_gather(a.ll_clusters + (tag & 1u) * cx.nc * (unsigned)D, D, (int)cx.nc, seg0, n, tag,
                                   sm.u.red, sm.seg, a.error, a.host_error, a.bar_timeout_ns) && dok && ok1;
      cmark<kDiag>(a, fr, kFmGather2);
#pragma unroll 1
      for (int i = threadIdx.x; i < n; i += kThreads) {
        const float v = Storage<T>::round(sm.x2[seg0 + i] + Storage<T>::round(sm.seg[i]));
        sm.seg[i] = v;
        if (cx.score_cluster) a.hidden[l * D + seg0 + i] = v;
      }
      flow_bar();
      if (!chain_publish_x(a, sm, cx, ok && !fr.failed)) return false;
      cmark<kDiag>(a, fr, kFmPub1);
    }
  }
  // final RMSNorm and score head (no cast), by the score CTA
  if (cx.score_cluster && cx.rank == 0) {
    const float scale = chain_norm_scale(sm.ssx[cx.bx], cx.cs, n, D, a.epsilon);
    const float* x = sm.x[cx.bx];
    float acc = 0.f;
#pragma unroll 1
    for (int i = threadIdx.x; i < D; i += kThreads)
      acc = fmaf(sm.fscore[i], Storage<T>::round(x[i] * scale * sm.fnorm[i]), acc);
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) sm.warp_scratch[threadIdx.x >> 5] = acc;
    flow_bar();
    float total = 0.f;
#pragma unroll 1
    for (int w = 0; w < kWarps; ++w) total += sm.warp_scratch[w];
    if (threadIdx.x == 0) {
      *score_dst = total;
      if (score_copy) *score_copy = total;
    }
  }
  cmark<kDiag>(a, fr, kFmScore);
  cx.steps += 1;
  return true;
}

// ---------------------------------------------------------------- kernel
// Trace mode and persistent mailbox mode exactly as k4_flow (flow_run); kDiag
// records the phase timeline (st_device_timeline_cta).
template <typename T, int D, bool kDiag>
__global__ void __launch_bounds__(kFlowThreads, 1) k5_chain(StepArgs a, FlowLaunch f) {
  extern __shared__ __align__(128) unsigned char chain_raw[];
  flow_run<T, D, ChainSmem>(a, f, chain_raw, kChainRingOffset, kChainRingCapacity,
                            [](const StepArgs& a, FlowRing& fr, FlowCur& cur, ChainSmem& sm, FlowCtx& cx,
                               const float* event, unsigned long long t, float* dst, float* copy) {
                              return chain_step<T, D, kDiag>(a, fr, cur, sm, cx, event, t, dst, copy);
                            });
}

}  // namespace st
