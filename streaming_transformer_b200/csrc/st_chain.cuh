// st_chain.cuh -- the single-stream step at the benchmark shapes, built to keep
// its per-layer chain of dependent phases short (k5_chain).
//
// Same work split, exchange protocol and weight ring as k4_flow (st_flow.cuh):
// NC clusters of CS CTAs, cluster c owns heads c, c + NC, ..., rank r owns
// segment r of the width; tagged records {fp32, tag} carry the head partials
// (exchange 1) and the cluster down partials (exchange 2) through L2; st.async
// stores completing on the receiver's mbarrier carry q/k/v, the attention
// partials, the down reduce-scatter and x inside a cluster; a producer warp
// streams every CTA's fixed chunk table into a shared-memory ring with
// cp.async.bulk. The arithmetic and cast points are the reference step's
// (reference src/cpu/Cpu.cpp:59-141).
//
// What differs is the shape of the code. Every layer runs the same few phases,
// and a phase's first execution in a layer used to pay for fetching its
// instructions again (the k4_flow step was ~145 KB of code, more than the SM
// keeps, so each layer refetched it). Here the heavy pieces -- the GEMV over a
// ring chunk, the short-row GEMV, the down-projection accumulation, the
// attention over staged slots and the tagged-record gather -- are single
// out-of-line routines taking scalars and pointers, every GEMV writes its dot
// products to shared memory, and a short epilogue loop per phase consumes
// them. The kernel stays small enough that its code remains resident from one
// layer to the next.
//
// Attention: each CTA stages the K and V rows of its share of the window into
// shared memory (cp.async, issued before the q/k/v GEMV so the copies overlap
// it; windows larger than the staging buffer go in batches); after the q/k/v
// exchange the rank that owns this step's slot writes the new k/v row into
// the staged copy. One warp scores 16 slots at once (a lane pair per slot,
// 32 dimensions per lane), takes their softmax and value sum, and merges the
// result into its running (m, l, acc); the warps' states are merged per CTA,
// and the CTA partials per cluster.
#pragma once

#include "st_flow.cuh"

namespace st {

constexpr int kChainDots = 1024;        // GEMV outputs of one span (rows of this CTA)
constexpr int kChainSlotsPerWarp = 16;  // attention slots one warp scores at once

struct alignas(128) ChainSmem {
  unsigned long long sbar[kSites][2];    // receive mbarriers per site and parity
  float x[2][kFlowMaxD];                 // residual entering the layer (site X)
  float x2[kFlowMaxD];                   // residual after attention (whole width)
  float z[kFlowMaxD];                    // norm output, GEMV input
  float dred[2][kFlowMaxD];              // down partials from every rank, [CS][n] (site DRED)
  float seg[kFlowMaxD];                  // this rank's segment values before publishing
  float fnorm[kFlowMaxD];                // final norm gain (score CTA)
  float fscore[kFlowMaxD];               // score weights (score CTA)
  float dots[kChainDots];                // GEMV outputs of the current span
  float qkv[2][3 * kFlowHd];             // q, k, v of the current head (site QKV)
  float apart[2][kFlowMaxCluster][kFlowHd + 2];  // CTA attention partials per rank (site ATT)
  float wst[kWarps][kFlowHd + 2];        // per-warp attention state (m, l, acc)
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
    alignas(16) unsigned char kv[kFlowKvBytes];   // staged K rows then V rows of a batch of slots
    float red[kFlowKvBytes / 4];                   // gather / down group partials
  } u;
};

constexpr size_t kChainRingOffset = (sizeof(ChainSmem) + sizeof(FlowRing) + 127) / 128 * 128;
constexpr unsigned kChainRingCapacity = (unsigned)((kFlowSmemBytes - kChainRingOffset) / 128 * 128);
static_assert(kChainRingCapacity >= 2 * kFlowChunkMax, "the chain ring needs room for two chunks");

// ---------------------------------------------------------------- GEMV routines
// Rows [0, nrows) of a chunk in shared memory (row stride D): dots[r] = row r . x.
// Two rows per warp pass (all 32 lanes on a row: D / V >= 32 vectors), passes
// dealt to warps round robin starting at `pass0`. x (shared memory) is held in
// registers for the call. Compute warps only; no barrier inside.
template <typename T, int D>
static __device__ __noinline__ void chain_gemv(const T* rows, int nrows, int pass0, const float* xs, float* dots) {
  using R = FlowRow<T, D>;
  static_assert(R::LPR == 32, "rows of the wide GEMV span the whole warp");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  FlowX<T, D> x;
  x.load(xs);
  const int passes = (nrows + 1) >> 1;
#pragma unroll 1
  for (int p = (warp - pass0 % kWarps + kWarps) % kWarps; p < passes; p += kWarps) {
    const int r = 2 * p;
    const bool two = r + 1 < nrows;
    // a single last row reads itself twice (its pair's sum is dropped)
    const T* p0 = rows + (size_t)r * D + (size_t)lane * R::V;
    const T* p1 = rows + (size_t)(two ? r + 1 : r) * D + (size_t)lane * R::V;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int k = 0; k < R::VPL; ++k) {
      const uint4 w0 = ld_shared_v4(p0 + (size_t)k * 32 * R::V);
      const uint4 w1 = ld_shared_v4(p1 + (size_t)k * 32 * R::V);
      a0 += dot_regs<T>(w0, x.v + k * R::V);
      a1 += dot_regs<T>(w1, x.v + k * R::V);
    }
    // the upper half-warp keeps row 1, the lower row 0: 5 shuffles for 2 rows
    const bool hi = (lane & 16) != 0;
    float s = (hi ? a1 : a0) + __shfl_xor_sync(0xffffffffu, hi ? a0 : a1, 16);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) dots[r] = s;
    if (lane == 16 && two) dots[r + 1] = s;
  }
}

// Short rows (K = V * nv elements, nv a power of two <= 32 vectors: the 32
// features of the input projection, head_dim of the out-projection): 32 / nv
// rows per warp pass, one 16-byte vector per lane.
template <typename T>
static __device__ __noinline__ void chain_gemv_short(const T* rows, int nrows, int K, int pass0, const float* xs,
                                                     float* dots) {
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
    float acc = dot_regs<T>(ld_shared_v4(rows + (size_t)(valid ? r : 0) * K + (size_t)sl * V), xv);
#pragma unroll 1
    for (int o = nv >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (valid && sl == 0) dots[r] = acc;
  }
}

// Down-projection partial over one chunk of this CTA's ffn rows (W_down
// transposed: row f has D elements): thread t owns the 16-byte column vector
// t % (D / V) and the rows f with (r0 + f) = t / (D / V) modulo G rows, so the
// sum order does not depend on how the span is cut into chunks. Accumulates
// into red[g * D + col] (first: starts from zero).
template <typename T, int D>
static __device__ __noinline__ void chain_down(const T* rows, int nrows, int r0, const float* act, float* red,
                                               bool first) {
  constexpr int V = Storage<T>::kVec, NVd = D / V, G = kThreads / NVd;
  const int cv = (int)threadIdx.x % NVd, g = (int)threadIdx.x / NVd;
  float* mine = red + g * D + cv * V;
  float acc[V];
#pragma unroll
  for (int k = 0; k < V; k += 4) {
    const float4 q = first ? make_float4(0.f, 0.f, 0.f, 0.f) : *reinterpret_cast<const float4*>(mine + k);
    acc[k] = q.x;
    acc[k + 1] = q.y;
    acc[k + 2] = q.z;
    acc[k + 3] = q.w;
  }
#pragma unroll 1
  for (int f = ((g - r0) % G + G) % G; f < nrows; f += G) {
    const float av = act[r0 + f];
    float w[V];
    Storage<T>::unpack(ld_shared_v4(rows + (size_t)f * D + (size_t)cv * V), w);
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] = fmaf(w[k], av, acc[k]);
  }
#pragma unroll
  for (int k = 0; k < V; k += 4)
    *reinterpret_cast<float4*>(mine + k) = make_float4(acc[k], acc[k + 1], acc[k + 2], acc[k + 3]);
}

// ---------------------------------------------------------------- attention
// One batch of nb staged slots (K rows at ks, V rows at vs, slot i at i * hd):
// warp w scores slots [16 w, 16 w + 16) at once -- lane L takes slot 16 w +
// L / 2 and dimensions [32 (L & 1), +32) of it -- takes their softmax and the
// value sum (lane L: dimensions 2L, 2L + 1) and merges them into its state
// wst[w] = (m, l, acc[hd]). first: the warp's state starts empty.
template <typename T>
static __device__ __noinline__ void chain_attend(const float* q, const T* ks, const T* vs, int nb, float* wst,
                                                 bool first) {
  constexpr int hd = kFlowHd, V = Storage<T>::kVec;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int s0 = warp * kChainSlotsPerWarp;
  float* st = wst + warp * (hd + 2);
  if (s0 >= nb) {
    if (first && lane == 0) {
      st[0] = -INFINITY;
      st[1] = 0.f;
    }
    if (first) {
      st[2 + 2 * lane] = 0.f;
      st[3 + 2 * lane] = 0.f;
    }
    return;
  }
  const int slot = s0 + (lane >> 1), half = lane & 1;
  const bool valid = slot < nb;
  float dot = 0.f;
  {
    const T* krow = ks + (size_t)(valid ? slot : s0) * hd + half * 32;
    const float* qh = q + half * 32;
#pragma unroll
    for (int v = 0; v < 32 / V; ++v) {
      float kf[V];
      Storage<T>::unpack(ld_shared_v4(krow + v * V), kf);
#pragma unroll
      for (int e = 0; e < V; ++e) dot = fmaf(qh[v * V + e], kf[e], dot);
    }
  }
  dot += __shfl_xor_sync(0xffffffffu, dot, 1);
  const float score = valid ? dot / sqrtf((float)hd) : -INFINITY;
  const float mb = warp_max(score);
  const float p = valid ? expf(score - mb) : 0.f;
  const float lb = warp_sum(half == 0 ? p : 0.f);
  float a0 = 0.f, a1 = 0.f;
  const int n = min(kChainSlotsPerWarp, nb - s0);
#pragma unroll 1
  for (int i = 0; i < n; ++i) {
    const float pi = __shfl_sync(0xffffffffu, p, 2 * i);
    const T* vrow = vs + (size_t)(s0 + i) * hd;
    a0 = fmaf(pi, Storage<T>::load(vrow, 2 * lane), a0);
    a1 = fmaf(pi, Storage<T>::load(vrow, 2 * lane + 1), a1);
  }
  if (first) {
    st[2 + 2 * lane] = a0;
    st[3 + 2 * lane] = a1;
    if (lane == 0) {
      st[0] = mb;
      st[1] = lb;
    }
  } else {
    const float mo = st[0], lo = st[1];
    const float m = fmaxf(mo, mb);
    const float co = lo > 0.f ? expf(mo - m) : 0.f, cb = expf(mb - m);
    st[2 + 2 * lane] = st[2 + 2 * lane] * co + a0 * cb;
    st[3 + 2 * lane] = st[3 + 2 * lane] * co + a1 * cb;
    __syncwarp();
    if (lane == 0) {
      st[0] = m;
      st[1] = lo * co + lb * cb;
    }
  }
  __syncwarp();
}

// Merge of nst (m, l, acc[hd]) states of stride hd + 2 into (M, L, A[dim]) by
// the 64 threads of warps 0 and 1 (dim = threadIdx.x); states with l = 0 are
// empty. Returns A for this thread's dim and M, L through the pointers.
__device__ __forceinline__ float chain_merge(const float* states, int nst, float* M_out, float* L_out) {
  const int lane = threadIdx.x & 31, dim = threadIdx.x;
  const float mk = lane < nst ? states[lane * (kFlowHd + 2)] : -INFINITY;
  const float lk = lane < nst ? states[lane * (kFlowHd + 2) + 1] : 0.f;
  const float M = warp_max(lk > 0.f ? mk : -INFINITY);
  const float sk = lk > 0.f ? expf(mk - M) : 0.f;
  const float L = warp_sum(lk * sk);
  float A = 0.f;
#pragma unroll 1
  for (int k = 0; k < nst; ++k) A = fmaf(states[k * (kFlowHd + 2) + 2 + dim], __shfl_sync(0xffffffffu, sk, k), A);
  *M_out = M;
  *L_out = L;
  return A;
}

// ---------------------------------------------------------------- gather
// Sum over sources src < nsrc of the tagged records rec[src * stride + e0 + i],
// i < n (n even, n / 2 a power of two <= kThreads), into out[i], sources added
// in index order. Thread t polls element pair t % (n / 2) for the sources
// congruent to t / (n / 2); partial sums meet in red. False (error word set)
// when a wait ran out or another CTA failed. Every compute thread calls; ends
// with a compute-thread barrier.
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
          ll_load2(rec + (size_t)src * stride + e0 + 2 * e, r[k][0], r[k][1]);
          ready = ready && ll_tag(r[k][0]) == tag && ll_tag(r[k][1]) == tag;
        } else {
          r[k][0] = r[k][1] = 0ull;
        }
      }
      if (ready) break;
      __nanosleep(32);
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
    for (int k = 0; k < G; ++k) t += red[k * n + i];
    out[i] = t;
  }
  flow_bar();
  return ok;
}

// ---------------------------------------------------------------- ring spans
// A span of this CTA's chunk table through a GEMV routine: every chunk is
// acquired, read by the warps that have passes in it and released by every
// warp. `rows` rows of `pr`-row passes; r0 of chunk c is c * rpc.
template <typename Fn>
__device__ __forceinline__ void chain_span(const StepArgs& a, FlowRing& fr, FlowCur& cur, const FlowSpan sp, int pr,
                                           Fn&& fn) {
  int pass0 = 0;
#pragma unroll 1
  for (int c = 0; c < sp.chunks; ++c) {
    const int r0 = c * sp.rpc;
    const int n = min(sp.rpc, sp.rows - r0);
    const unsigned char* base = flow_acquire(a, fr, cur);
    fn(base, r0, n, pass0);
    flow_release(fr, cur);
    pass0 += (n + pr - 1) / pr;
  }
}

// ---------------------------------------------------------------- attention per head
// K and V rows of slots [b0, b1) of this head's ring into u.kv (K rows, then
// V rows), skipping `skip` (the slot this step overwrites; its row comes from
// the q/k/v exchange). Committed as one cp.async group.
template <typename T>
__device__ __forceinline__ void chain_stage(const T* keys, const T* values, int b0, int b1, int skip,
                                            unsigned char* kv) {
  constexpr int vpr = kFlowHd * (int)sizeof(T) / 16;
  const int vecs = (b1 - b0) * vpr;
#pragma unroll 1
  for (int i = threadIdx.x; i < 2 * vecs; i += kThreads) {
    const bool is_v = i >= vecs;
    const int k = is_v ? i - vecs : i;
    if (b0 + k / vpr == skip) continue;
    const char* src = (const char*)(is_v ? values : keys) + (size_t)b0 * kFlowHd * sizeof(T) + (size_t)k * 16;
    cp_async16(kv + (size_t)i * 16, src);
  }
  cp_async_commit();
}

// One head h of layer l: q/k/v rows, attention over this CTA's slots, the
// out-projection rows of this rank's segment published as P[h]. False when a
// wait ran out (the error word is set; the next exchange ends the launch).
template <typename T, int D>
__device__ __forceinline__ bool chain_head(const StepArgs& a, FlowRing& fr, FlowCur& cur, ChainSmem& sm,
                                           FlowCtx& cx, int l, int h, unsigned tag, bool first_head) {
  constexpr int hd = kFlowHd;
  const int W = a.window, slot = cx.slot, valid = cx.valid;
  const size_t head_base = (((size_t)l * a.heads + h) * (size_t)W) * hd;
  T* keys = (T*)a.keys + head_base;
  T* values = (T*)a.values + head_base;
  int j0, j1;
  split(valid, (int)cx.rank, (int)cx.cs, j0, j1);
  // slots per staging batch: K and V rows of `per` slots fill u.kv at most
  const int per = kFlowKvBytes / (2 * hd * (int)sizeof(T));
  int b1 = min(j1, j0 + per);
  chain_stage<T>(keys, values, j0, b1, slot, sm.u.kv);
  if (first_head) {
    const float scale = flow_norm_scale(sm.ssx[cx.bx], cx.cs, cx.n, D, a.epsilon);
    const float* x = sm.x[cx.bx];
    flow_gain<T>(a, fr, cur, [&](const T* g) {
      for (int i = threadIdx.x; i < D; i += kThreads) sm.z[i] = Storage<T>::round(x[i] * scale * Storage<T>::load(g, i));
    });
    flow_bar();
    fmark(a, fr, kFmNorm1);
  }
  // q, k, v row pairs of this rank -> dots
  chain_span(a, fr, cur, sm.plan.qkv, 2, [&](const unsigned char* base, int r0, int n, int pass0) {
    chain_gemv<T, D>((const T*)base, n, pass0, sm.z, sm.dots + r0);
  });
  flow_bar();
  // epilogue: RoPE and casts, broadcast into every rank, k/v into slot t % W
  const unsigned kq = cx.k[kSiteQkv]++, bq = kq & 1u;
  float* qkv = sm.qkv[bq];
  {
    const unsigned long long* qbar = &sm.sbar[kSiteQkv][bq];
    const int lo = sm.plan.qkv_lo, pairs = sm.plan.qkv.rows >> 1;
    for (int i = threadIdx.x; i < pairs; i += kThreads) {
      const int row = 2 * (lo + i);
      const int which = row / hd, dim = row - which * hd;
      float v0 = Storage<T>::round(sm.dots[2 * i]);
      float v1 = Storage<T>::round(sm.dots[2 * i + 1]);
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
    }
  }
  fmark(a, fr, kFmQkv);
  bool ok = flow_receive(a, fr, sm, kSiteQkv, kq, 3u * hd * 4u);
  fmark(a, fr, kFmQkvSync);
  // attention over [j0, j1) in batches of `per` staged slots
  bool first = true;
#pragma unroll 1
  for (int b0 = j0; b0 < j1 || first; b0 = b1, b1 = min(j1, b0 + per)) {
    const T* Ks = reinterpret_cast<const T*>(sm.u.kv);
    const T* Vs = Ks + (size_t)(b1 - b0) * hd;
    cp_async_wait_all();
    if (slot >= b0 && slot < b1)
      for (int i = threadIdx.x; i < 2 * hd; i += kThreads) {
        const int which = i / hd, dim = i - which * hd;
        Storage<T>::store(const_cast<T*>(which ? Vs : Ks), (size_t)(slot - b0) * hd + dim, qkv[(1 + which) * hd + dim]);
      }
    flow_bar();
    chain_attend<T>(qkv, Ks, Vs, b1 - b0, &sm.wst[0][0], first);
    first = false;
    if (b1 < j1) {
      flow_bar();
      chain_stage<T>(keys, values, b1, min(j1, b1 + per), slot, sm.u.kv);
    }
  }
  flow_bar();
  fmark(a, fr, kFmAttn);
  // this CTA's partial from the warp states, sent into every rank
  const unsigned ka = cx.k[kSiteAtt]++, ba = ka & 1u;
  float(*apart)[kFlowHd + 2] = sm.apart[ba];
  if (threadIdx.x < hd) {
    float M, L;
    const float A = chain_merge(&sm.wst[0][0], kWarps, &M, &L);
    const unsigned long long* abar = &sm.sbar[kSiteAtt][ba];
    for (unsigned r = 0; r < cx.cs; ++r) st_async1(&apart[cx.rank][2 + threadIdx.x], abar, r, A);
    if (threadIdx.x < cx.cs) st_async2(&apart[cx.rank][0], abar, threadIdx.x, M, L);
  }
  ok = flow_receive(a, fr, sm, kSiteAtt, ka, cx.cs * (unsigned)(4 * hd + 8)) && ok;
  fmark(a, fr, kFmPartSync);
  // merge the cluster's partials in rank order -> o (cast)
  if (threadIdx.x < hd) {
    float M, L;
    const float A = chain_merge(&apart[0][0], (int)cx.cs, &M, &L);
    sm.o[threadIdx.x] = Storage<T>::round(A / L);
  }
  flow_bar();
  fmark(a, fr, kFmMerge);
  // out-projection rows of this rank's segment (K-split by head) -> P[h][seg]
  chain_span(a, fr, cur, sm.plan.out, 32 / (hd / Storage<T>::kVec), [&](const unsigned char* base, int r0, int n,
                                                                          int pass0) {
    chain_gemv_short<T>((const T*)base, n, hd, pass0, sm.o, sm.dots + r0);
  });
  flow_bar();
  {
    unsigned long long* P = a.ll_heads + ((size_t)(tag & 1u) * a.heads + h) * D + cx.seg0;
    for (int i = threadIdx.x; i < (cx.n >> 1); i += kThreads) ll_store2(P + 2 * i, sm.dots[2 * i], sm.dots[2 * i + 1], tag);
  }
  fmark(a, fr, kFmOut);
  return ok;
}

// ---------------------------------------------------------------- one step
template <typename T, int D>
__device__ __forceinline__ bool chain_step(const StepArgs& a, FlowRing& fr, FlowCur& cur, ChainSmem& sm, FlowCtx& cx,
                                           const float* event, unsigned long long t, float* score_dst,
                                           float* score_copy) {
  const int n = cx.n, seg0 = cx.seg0;
  fmark(a, fr, kFmStep);
  cx.slot = (int)(t % (unsigned long long)a.window);
  cx.valid = t + 1 < (unsigned long long)a.window ? (int)(t + 1) : a.window;
  if (threadIdx.x < kFlowFeatures) sm.ev[threadIdx.x] = __ldcv(event + threadIdx.x);
  if (threadIdx.x < kFlowHd / 2) {
    const float angle = (float)t * sm.rope[threadIdx.x];
    sm.rope_cs[threadIdx.x] = make_float2(cosf(angle), sinf(angle));
  }
  flow_bar();
  // x[seg] = cast(W_in[seg] e)
  chain_span(a, fr, cur, sm.plan.in, 32 / (kFlowFeatures / Storage<T>::kVec),
             [&](const unsigned char* base, int r0, int rows, int pass0) {
               chain_gemv_short<T>((const T*)base, rows, kFlowFeatures, pass0, sm.ev, sm.dots + r0);
             });
  flow_bar();
  for (int i = threadIdx.x; i < n; i += kThreads) sm.seg[i] = Storage<T>::round(sm.dots[i]);
  flow_bar();
  if (!flow_publish(a, fr, sm, cx, !fr.failed)) return false;
  fmark(a, fr, kFmIn);
#pragma unroll 1
  for (int l = 0; l < a.layers; ++l) {
    const unsigned tag = (unsigned)(cx.epoch + cx.steps * (unsigned long long)a.layers + (unsigned long long)l + 1ull);
    bool hok = true;
    if (cx.heads_here)
      for (int h = (int)cx.id; h < a.heads; h += (int)cx.nc)
        hok = chain_head<T, D>(a, fr, cur, sm, cx, l, h, tag, h == (int)cx.id) && hok;
    // exchange 1 (whole width): x' = cast(x + cast(sum_h P[h])), and sum(x'^2)
    bool ok1;
    float ssq = 0.f;
    {
      const unsigned long long* P = a.ll_heads + (size_t)(tag & 1u) * a.heads * D;
      ok1 = chain_gather(P, D, a.heads, 0, D, tag, sm.u.red, sm.x2, a.error, a.host_error, a.bar_timeout_ns) && hok &&
            !fr.failed;
      const float* x = sm.x[cx.bx];
      float q = 0.f;
      for (int i = threadIdx.x; i < D; i += kThreads) {
        const float v = Storage<T>::round(x[i] + Storage<T>::round(sm.x2[i]));
        sm.x2[i] = v;
        q = fmaf(v, v, q);
      }
      q = warp_sum(q);
      if ((threadIdx.x & 31) == 0) sm.warp_scratch[threadIdx.x >> 5] = q;
      flow_bar();
      for (int w = 0; w < kWarps; ++w) ssq += sm.warp_scratch[w];
      fmark(a, fr, kFmGather1);
    }
    // FFN: norm2, gate/up -> SwiGLU, down partial
    bool dok;
    {
      const float scale = 1.0f / sqrtf(ssq / (float)D + a.epsilon);
      flow_gain<T>(a, fr, cur, [&](const T* g) {
        for (int i = threadIdx.x; i < D; i += kThreads)
          sm.z[i] = Storage<T>::round(sm.x2[i] * scale * Storage<T>::load(g, i));
      });
      flow_bar();
      fmark(a, fr, kFmNorm2);
      chain_span(a, fr, cur, sm.plan.gateup, 2, [&](const unsigned char* base, int r0, int rows, int pass0) {
        chain_gemv<T, D>((const T*)base, rows, pass0, sm.z, sm.dots + r0);
      });
      flow_bar();
      for (int i = threadIdx.x; i < (sm.plan.gateup.rows >> 1); i += kThreads) {
        const float gt = Storage<T>::round(sm.dots[2 * i]);
        const float up = Storage<T>::round(sm.dots[2 * i + 1]);
        sm.act[i] = Storage<T>::round((gt / (1.0f + expf(-gt))) * up);
      }
      flow_bar();
      fmark(a, fr, kFmGateUp);
      {
        const FlowSpan sp = sm.plan.down;
        int c = 0;
        chain_span(a, fr, cur, sp, 1, [&](const unsigned char* base, int r0, int rows, int) {
          chain_down<T, D>((const T*)base, rows, r0, sm.act, sm.u.red, c++ == 0);
        });
        if (sp.chunks == 0) {
          // no ffn rows here: a zero partial
          for (int i = threadIdx.x; i < (kThreads / (D / Storage<T>::kVec)) * D; i += kThreads) sm.u.red[i] = 0.f;
        }
      }
      fmark(a, fr, kFmDown);
      flow_bar();
      // column sums in group order, sent in float4s to the rank owning them
      const unsigned kd = cx.k[kSiteDred]++, bd = kd & 1u;
      float* dred = sm.dred[bd];
      const unsigned long long* dbar = &sm.sbar[kSiteDred][bd];
      constexpr int G2 = kThreads / (D / Storage<T>::kVec);
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
      fmark(a, fr, kFmDredSync);
      // this rank's segment of the cluster partial, ranks added in order
      unsigned long long* Dp = a.ll_clusters + ((size_t)(tag & 1u) * cx.nc + cx.id) * D + seg0;
      for (int i = 2 * threadIdx.x; i < n; i += 2 * kThreads) {
        float s0 = 0.f, s1 = 0.f;
        for (unsigned r = 0; r < cx.cs; ++r) {
          s0 += dred[r * n + i];
          s1 += dred[r * n + i + 1];
        }
        ll_store2(Dp + i, s0, s1, tag);
      }
      fmark(a, fr, kFmDpub);
    }
    // exchange 2: x[seg] = cast(x'[seg] + cast(sum_c D[c][seg]))
    {
      const unsigned long long* Dq = a.ll_clusters + (size_t)(tag & 1u) * cx.nc * D;
      const bool ok = chain_gather(Dq, D, (int)cx.nc, seg0, n, tag, sm.u.red, sm.seg, a.error, a.host_error,
                                   a.bar_timeout_ns) && dok && ok1;
      fmark(a, fr, kFmGather2);
      for (int i = threadIdx.x; i < n; i += kThreads) {
        const float v = Storage<T>::round(sm.x2[seg0 + i] + Storage<T>::round(sm.seg[i]));
        sm.seg[i] = v;
        if (cx.score_cluster) a.hidden[(size_t)l * D + seg0 + i] = v;
      }
      flow_bar();
      if (!flow_publish(a, fr, sm, cx, ok && !fr.failed)) return false;
      fmark(a, fr, kFmPub1);
    }
  }
  // final RMSNorm and score head (no cast), by the score CTA
  if (cx.score_cluster && cx.rank == 0) {
    const float scale = flow_norm_scale(sm.ssx[cx.bx], cx.cs, n, D, a.epsilon);
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
  fmark(a, fr, kFmScore);
  cx.steps += 1;
  return true;
}

// ---------------------------------------------------------------- kernel
// Trace mode and persistent mailbox mode exactly as k4_flow (flow_run).
template <typename T, int D>
__global__ void __launch_bounds__(kFlowThreads, 1) k5_chain(StepArgs a, FlowLaunch f) {
  extern __shared__ __align__(128) unsigned char chain_raw[];
  flow_run<T, D, ChainSmem>(a, f, chain_raw, kChainRingOffset, kChainRingCapacity,
                            [](const StepArgs& a, FlowRing& fr, FlowCur& cur, ChainSmem& sm, FlowCtx& cx,
                               const float* event, unsigned long long t, float* dst, float* copy) {
                              return chain_step<T, D>(a, fr, cur, sm, cx, event, t, dst, copy);
                            });
}

}  // namespace st
