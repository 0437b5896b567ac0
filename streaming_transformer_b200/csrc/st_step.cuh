// st_step.cuh -- the streaming step, organised around thread-block clusters.
//
// Measured on B200: a grid-wide barrier costs ~1.3 us and a hardware cluster
// barrier ~0.24 us, so a step is built from two grid-wide dependencies per
// layer and cheap cluster-local exchanges (DSMEM) for everything else. The
// grid is NC clusters of CS CTAs (CS = 8 at full size). Per layer:
//
//  attention block (cluster c owns heads c, c + NC, ...; other clusters idle)
//    z = norm1(x)                      every CTA, from its shared-memory copy of x
//    q,k,v rows of head h              split over the cluster's CTAs; RoPE + cast in
//                                      the epilogue; values broadcast to every CTA of
//                                      the cluster through distributed shared memory;
//                                      k, v stored to ring slot t % W
//    cluster barrier
//    attention over [0, valid)         slots split over the cluster; (m, l, acc)
//                                      partials broadcast through DSMEM
//    cluster barrier
//    merge -> attn_h (cast); out-projection K-split by head: P[h] = W_out[:, h] attn_h,
//                                      output rows split over the cluster -> global
//  grid sync A
//  FFN block (every CTA)
//    x' = cast(x + cast(sum_h P[h]))   redundantly, heads summed in a fixed order
//    z = norm2(x'); gate/up rows of this CTA's ffn slice -> act = cast(silu(g) u)
//    down-projection K-split over the slice (W_down stored transposed, [F][d]):
//                                      partial d-vector, reduce-scattered inside the
//                                      cluster through DSMEM -> D[cluster] -> global
//  grid sync B
//    x = cast(x' + cast(sum_c D[c]))   redundantly, clusters summed in a fixed order
//
// The input projection is computed redundantly by every CTA (no grid sync), and
// CTA 0 runs the final norm and score head. The same block functions run as
// separate kernels for the per-op and graph backends, where a kernel boundary
// replaces each grid sync and the residual crosses kernels through global
// buffers written by CTA 0. Cast points and op order follow the reference step
// (reference src/cpu/Cpu.cpp:59-141); the GEMV sums are reassociated (per-head
// and per-slice partials), which the fp32 1e-5 tolerance absorbs.
#pragma once

#include "st_device.cuh"

namespace st {

constexpr int kMaxCluster = 8;
constexpr int kMaxWidth = 1024;
constexpr int kMaxHeadDim = 1024;
constexpr int kMaxWindow = 4096;
constexpr int kMaxFfn = 4096;

// Dynamic shared memory of one CTA (~125 KB).
struct alignas(16) Smem2 {
  Smem g;                                        // GEMV input / reductions
  float xres[kMaxWidth];                         // residual entering the block
  float x2res[kMaxWidth];                        // residual after attention
  float qkv[3 * kMaxHeadDim];                    // q, k, v of the current head (DSMEM target)
  float apart[kMaxCluster * (kMaxHeadDim + 2)];  // attention partials per rank (DSMEM target)
  float dred[2 * kMaxWidth];                     // down partial rows per rank (DSMEM target)
  float act[kMaxFfn];                            // this CTA's SwiGLU slice
  float logits[kMaxWindow];
  float gpart[2 * kMaxWidth];                    // per-group attention accumulators
  float head[2];                                 // m, l of this CTA's attention partial
  int sync_ok;                                   // verdict of the last grid sync (DSMEM target)
  int tl_n;                                      // timeline entries written by this CTA
};

// Phase-boundary timestamp (CTA 0, thread 0) when a timeline buffer is given.
__device__ __forceinline__ void tl_mark(const StepArgs& a, Smem2& sm) {
  if (a.timeline && blockIdx.x == 0 && threadIdx.x == 0 && sm.tl_n < a.timeline_capacity)
    a.timeline[sm.tl_n++] = clock64();
}

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

struct ClusterPos {
  unsigned rank, size, id, count;
  __device__ static ClusterPos get() { return {cluster_rank(), cluster_size(), cluster_id(), cluster_count()}; }
};

// Grid-wide barrier in cluster units. The cluster first meets at a hardware
// barrier, then its rank-0 CTA alone arrives on the global counter and waits
// (bounded, with the error word checked) and writes its verdict into every
// CTA of the cluster through DSMEM before a second cluster barrier. Every CTA
// of a cluster therefore returns the same verdict, so a failed wait can never
// leave a peer stranded at a later cluster barrier. The counter rises by one
// per cluster per barrier; `base` is its value when the launch started.
struct ClusterGridSync {
  unsigned long long base;
  unsigned long long epoch;
  __device__ bool sync(const StepArgs& a, unsigned long long timeout_ns, int* ok_slot) {
    __threadfence();  // this thread's global writes, visible GPU-wide before the release below
    cluster_sync();
    const unsigned rank = cluster_rank();
    if (rank == 0 && threadIdx.x == 0) {
      epoch += 1;
      const unsigned long long target = base + epoch * cluster_count();
      int good = ld_volatile_int(a.error) == 0;
      if (good) {
        red_release_gpu_add(a.bar_counter, 1ull);
        unsigned long long start = 0;
        unsigned int polls = 0;
        while (ld_acquire_gpu(a.bar_counter) < target) {
          if ((++polls & 63u) == 0) {
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

__device__ __forceinline__ void split(int units, int part, int parts, int& lo, int& hi) {
  lo = (int)(((long long)units * part) / parts);
  hi = (int)(((long long)units * (part + 1)) / parts);
}

// GEMV over rows [r_begin, r_end) of W (row-major, `cols`) against sm.g.xs, in
// tiles; epi(r0, n) consumes sm.g.rowsum[0..n).
template <typename T, typename Epi>
__device__ void rows_gemv(const T* W, int r_begin, int r_end, int cols, Smem& sm, Epi epi) {
  for (int r0 = r_begin; r0 < r_end; r0 += kRowTile) {
    const int n = min(kRowTile, r_end - r0);
    gemv_tile<T>(W, r0, n, cols, sm);
    epi(r0, n);
    __syncthreads();
  }
}

// RMSNorm of a shared-memory vector into sm.g.xs (reference src/cpu/Cpu.cpp:43-57).
template <typename T>
__device__ void norm_smem(const float* x, const T* gain, int width, float eps, Smem2& sm) {
  float s = 0.f;
  for (int i = threadIdx.x; i < width; i += kThreads) s += x[i] * x[i];
  const float total = block_sum(s, sm.g);
  const float scale = 1.0f / sqrtf(total / (float)width + eps);
  for (int i = threadIdx.x; i < width; i += kThreads)
    sm.g.xs[i] = Storage<T>::round(x[i] * scale * Storage<T>::load(gain, i));
  __syncthreads();
}

__device__ __forceinline__ int valid_length(unsigned long long t, int window) {
  return t + 1 < (unsigned long long)window ? (int)(t + 1) : window;
}

// ---------------------------------------------------------------- blocks
// x = cast(W_in input) for stream s into `dst` (shared memory), all rows, this CTA.
template <typename T>
__device__ void block_input(const StepArgs& a, int s, const float* input, float* dst, Smem2& sm) {
  for (int i = threadIdx.x; i < a.features; i += kThreads) sm.g.xs[i] = __ldcv(input + (size_t)s * a.features + i);
  __syncthreads();
  rows_gemv<T>((const T*)a.input_w, 0, a.width, a.features, sm.g, [&](int r0, int n) {
    for (int i = threadIdx.x; i < n; i += kThreads) dst[r0 + i] = Storage<T>::round(sm.g.rowsum[i]);
  });
}

// Attention for head h of stream s over this CTA's share of [0, valid): logits,
// local softmax statistics and sum p V; the current slot's k, v come from the
// cluster-shared sm.qkv, older slots from the ring. Leaves (m, l) in sm.head and
// acc in sm.gpart[0..hd).
template <typename T>
__device__ void attention_share(const StepArgs& a, int l, int s, int h, int j0, int j1, int slot, Smem2& sm) {
  const int hd = a.head_dim, W = a.window, H = a.heads;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const size_t head_base = ((((size_t)s * a.layers + l) * H + h) * (size_t)W) * hd;
  const T* K = (const T*)a.keys + head_base;
  const T* V = (const T*)a.values + head_base;
  const float* q = sm.qkv;
  const float* kcur = sm.qkv + hd;
  const float* vcur = sm.qkv + 2 * hd;
  const int n = j1 - j0;
  const float inv = sqrtf((float)hd);
  // logits: warp per slot, lanes over dims
  for (int j = j0 + warp; j < j1; j += kWarps) {
    float dot = 0.f;
    if (j == slot) {
      for (int i = lane; i < hd; i += 32) dot = fmaf(q[i], kcur[i], dot);
    } else {
      const T* krow = K + (size_t)j * hd;
      for (int i = lane; i < hd; i += 32) dot = fmaf(q[i], Storage<T>::load_cg(krow, i), dot);
    }
    dot = warp_sum(dot);
    if (lane == 0) sm.logits[j - j0] = dot / inv;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int j = threadIdx.x; j < n; j += kThreads) m = fmaxf(m, sm.logits[j]);
  // block max
  m = warp_max(m);
  if (lane == 0) sm.g.warp_scratch[warp] = m;
  __syncthreads();
  if (warp == 0) {
    float t = lane < kWarps ? sm.g.warp_scratch[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) sm.g.scalar[1] = t;
  }
  __syncthreads();
  m = sm.g.scalar[1];
  float psum = 0.f;
  for (int j = threadIdx.x; j < n; j += kThreads) {
    const float p = expf(sm.logits[j] - m);
    sm.logits[j] = p;
    psum += p;
  }
  const float lsum = block_sum(psum, sm.g);
  // acc[d] = sum_j p_j V[j][d]. With hd < kThreads the CTA splits into
  // `groups` thread groups over dims, group g taking slots j0+g, j0+g+groups, ...;
  // the group sums are then added in group order.
  if (hd < kThreads) {
    const int groups = kThreads / hd;
    const int g = threadIdx.x / hd, dd = threadIdx.x - g * hd;
    if (g < groups) {
      float acc = 0.f;
      for (int j = j0 + g; j < j1; j += groups) {
        const float v = j == slot ? vcur[dd] : Storage<T>::load_cg(V + (size_t)j * hd, dd);
        acc = fmaf(sm.logits[j - j0], v, acc);
      }
      sm.gpart[g * hd + dd] = acc;
    }
    __syncthreads();
    float total = 0.f;
    if (threadIdx.x < hd)
      for (int gg = 0; gg < groups; ++gg) total += sm.gpart[gg * hd + threadIdx.x];
    __syncthreads();
    if (threadIdx.x < hd) sm.gpart[threadIdx.x] = total;
  } else {
    for (int dd = threadIdx.x; dd < hd; dd += kThreads) {
      float acc = 0.f;
      for (int j = j0; j < j1; ++j) {
        const float v = j == slot ? vcur[dd] : Storage<T>::load_cg(V + (size_t)j * hd, dd);
        acc = fmaf(sm.logits[j - j0], v, acc);
      }
      sm.gpart[dd] = acc;
    }
  }
  if (threadIdx.x == 0) {
    sm.head[0] = n > 0 ? m : -INFINITY;
    sm.head[1] = n > 0 ? lsum : 0.f;
  }
  __syncthreads();
}

// One head h of one stream, run by the CTAs of one cluster.
template <typename T>
__device__ void attention_head(const StepArgs& a, int l, int s, int h, const ClusterPos& cp, Smem2& sm) {
  const int d = a.width, hd = a.head_dim, W = a.window;
  const LayerPtrs& w = a.layer[l];
  const unsigned long long t = ld_cg_u64(a.position + s);
  const int slot = (int)(t % (unsigned long long)W);
  const int valid = valid_length(t, W);
  T* keys = (T*)a.keys + ((((size_t)s * a.layers + l) * a.heads + h) * (size_t)W) * hd;
  T* values = (T*)a.values + ((((size_t)s * a.layers + l) * a.heads + h) * (size_t)W) * hd;
  // q, k, v rows of head h (head-major [H][3 hd][d]); pairs split over the cluster.
  const T* Wh = (const T*)w.qkv + (size_t)h * 3 * hd * d;
  int lo, hi;
  split(3 * hd / 2, cp.rank, cp.size, lo, hi);
  const float tf = (float)t;
  rows_gemv<T>(Wh, 2 * lo, 2 * hi, d, sm.g, [&](int r0, int n) {
    for (int p = threadIdx.x; p < n / 2; p += kThreads) {
      const int row = r0 + 2 * p;
      const int which = row / hd, dim = row - which * hd;
      float v0 = Storage<T>::round(sm.g.rowsum[2 * p]);
      float v1 = Storage<T>::round(sm.g.rowsum[2 * p + 1]);
      if (which < 2) {
        const float angle = tf * a.rope_freq[dim >> 1];
        const float co = cosf(angle), si = sinf(angle);
        const float r0v = v0 * co - v1 * si;
        const float r1v = v0 * si + v1 * co;
        v0 = Storage<T>::round(r0v);
        v1 = Storage<T>::round(r1v);
      }
      for (unsigned k = 0; k < cp.size; ++k) {
        dsmem_store(&sm.qkv[row], k, v0);
        dsmem_store(&sm.qkv[row + 1], k, v1);
      }
      if (which > 0) {
        T* ring = which == 1 ? keys : values;
        const size_t at = (size_t)slot * hd + dim;
        Storage<T>::store(ring, at, v0);
        Storage<T>::store(ring, at + 1, v1);
      }
    }
  });
  tl_mark(a, sm);  // qkv rows done
  cluster_sync();
  tl_mark(a, sm);  // q, k, v shared
  if (a.trace_qkv && cp.rank == 0)
    for (int i = threadIdx.x; i < 3 * hd; i += kThreads)
      a.trace_qkv[(size_t)s * 3 * d + (size_t)(i / hd) * d + (size_t)h * hd + i % hd] = sm.qkv[i];
  // this CTA's share of the retained slots
  int j0, j1;
  split(valid, cp.rank, cp.size, j0, j1);
  attention_share<T>(a, l, s, h, j0, j1, slot, sm);
  tl_mark(a, sm);  // attention share done
  float* mine = sm.apart + (size_t)cp.rank * (hd + 2);
  for (int i = threadIdx.x; i < hd + 2; i += kThreads) {
    const float v = i == 0 ? sm.head[0] : i == 1 ? sm.head[1] : sm.gpart[i - 2];
    for (unsigned k = 0; k < cp.size; ++k) dsmem_store(mine + i, k, v);
  }
  cluster_sync();
  tl_mark(a, sm);  // partials shared
  // merge the cluster's partials in rank order -> attn_h (cast) in sm.g.xs[0..hd)
  for (int i = threadIdx.x; i < hd; i += kThreads) {
    float M = -INFINITY;
    for (unsigned k = 0; k < cp.size; ++k) {
      const float* pk = sm.apart + (size_t)k * (hd + 2);
      if (pk[1] > 0.f) M = fmaxf(M, pk[0]);
    }
    float L = 0.f, acc = 0.f;
    for (unsigned k = 0; k < cp.size; ++k) {
      const float* pk = sm.apart + (size_t)k * (hd + 2);
      if (pk[1] > 0.f) {
        const float scale = expf(pk[0] - M);
        L = fmaf(pk[1], scale, L);
        acc = fmaf(pk[2 + i], scale, acc);
      }
    }
    sm.g.xs[i] = Storage<T>::round(acc / L);
    if (a.trace_attention && cp.rank == 0) a.trace_attention[(size_t)s * d + (size_t)h * hd + i] = sm.g.xs[i];
  }
  __syncthreads();
  // out-projection partial of this head: rows split over the cluster ([H][d][hd] layout)
  const T* Wo = (const T*)w.out + (size_t)h * d * hd;
  split(d, cp.rank, cp.size, lo, hi);
  float* P = a.pout + ((size_t)s * a.heads + h) * d;
  rows_gemv<T>(Wo, lo, hi, hd, sm.g, [&](int r0, int n) {
    for (int i = threadIdx.x; i < n; i += kThreads) P[r0 + i] = sm.g.rowsum[i];
  });
  tl_mark(a, sm);  // merge + out-projection partial done
}

// x' = cast(x + cast(sum_h P[h])) from sm.xres into sm.x2res.
template <typename T>
__device__ void residual_from_heads(const StepArgs& a, int s, Smem2& sm) {
  const int d = a.width;
  const float* P = a.pout + (size_t)s * a.heads * d;
  for (int i = threadIdx.x; i < d; i += kThreads) {
    float acc = 0.f;
    for (int h = 0; h < a.heads; ++h) acc += ld_cg(P + (size_t)h * d + i);
    sm.x2res[i] = Storage<T>::round(sm.xres[i] + Storage<T>::round(acc));
  }
  __syncthreads();
}

// x = cast(x' + cast(sum_c D[c])) from sm.x2res into sm.xres.
template <typename T>
__device__ void residual_from_clusters(const StepArgs& a, int s, int nclusters, Smem2& sm) {
  const int d = a.width;
  const float* D = a.dpart + (size_t)s * nclusters * d;
  for (int i = threadIdx.x; i < d; i += kThreads) {
    float acc = 0.f;
    for (int c = 0; c < nclusters; ++c) acc += ld_cg(D + (size_t)c * d + i);
    sm.xres[i] = Storage<T>::round(sm.x2res[i] + Storage<T>::round(acc));
  }
  __syncthreads();
}

// FFN block for stream s: needs sm.x2res (x'); leaves D[cluster] in global memory.
template <typename T>
__device__ void block_ffn(const StepArgs& a, int l, int s, const ClusterPos& cp, Smem2& sm) {
  const int d = a.width, F = a.ffn;
  const LayerPtrs& w = a.layer[l];
  norm_smem<T>(sm.x2res, (const T*)w.norm2, d, a.epsilon, sm);
  tl_mark(a, sm);  // norm2 done
  const int G = (int)(cp.count * cp.size), gi = (int)(cp.id * cp.size + cp.rank);
  int lo, hi;
  split(F, gi, G, lo, hi);
  float* act_trace = a.trace_act ? a.trace_act + (size_t)s * F : nullptr;
  rows_gemv<T>((const T*)w.gateup, 2 * lo, 2 * hi, d, sm.g, [&](int r0, int n) {
    for (int p = threadIdx.x; p < n / 2; p += kThreads) {
      const float g = Storage<T>::round(sm.g.rowsum[2 * p]);
      const float u = Storage<T>::round(sm.g.rowsum[2 * p + 1]);
      const int f = (r0 >> 1) + p;
      const float v = Storage<T>::round((g / (1.0f + expf(-g))) * u);
      sm.act[f - lo] = v;
      if (act_trace) act_trace[f] = v;
    }
  });
  tl_mark(a, sm);  // gate/up + SwiGLU done
  // partial[row] = sum_{f in slice} W_down^T[f][row] act[f]. With d < kThreads
  // the CTA splits into `groups` thread groups over rows, group g taking
  // f = lo+g, lo+g+groups, ...; loads are issued 8 at a time before use.
  const T* WdT = (const T*)w.down;  // [F][d]
  const int groups = d >= kThreads ? 1 : kThreads / d;
  const int seg = (d + (int)cp.size - 1) / (int)cp.size;
  float* part = sm.gpart;  // [groups][d], groups * d <= max(kThreads, d)
  {
    const int g = d >= kThreads ? 0 : (int)threadIdx.x / d;
    if (g < groups) {
      for (int row = (d >= kThreads ? (int)threadIdx.x : (int)threadIdx.x - g * d); row < d; row += (d >= kThreads ? kThreads : d)) {
        float acc = 0.f;
        for (int f0 = lo + g; f0 < hi; f0 += 8 * groups) {
          float wv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int f = f0 + u * groups;
            wv[u] = f < hi ? Storage<T>::load(WdT, (size_t)f * d + row) : 0.f;
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int f = f0 + u * groups;
            if (f < hi) acc = fmaf(wv[u], sm.act[f - lo], acc);
          }
        }
        part[g * d + row] = acc;
      }
    }
  }
  __syncthreads();
  // sum groups in order, then reduce-scatter to the owning rank of each row segment
  for (int row = threadIdx.x; row < d; row += kThreads) {
    float acc = 0.f;
    for (int gg = 0; gg < groups; ++gg) acc += part[gg * d + row];
    const unsigned owner = (unsigned)(row / seg);
    dsmem_store(&sm.dred[cp.rank * seg + (row - (int)owner * seg)], owner, acc);
  }
  tl_mark(a, sm);  // down partial done
  cluster_sync();
  const int r_lo = (int)cp.rank * seg, r_hi = min(d, r_lo + seg);
  float* D = a.dpart + ((size_t)s * cp.count + cp.id) * d;
  for (int row = r_lo + threadIdx.x; row < r_hi; row += kThreads) {
    float acc = 0.f;
    for (unsigned k = 0; k < cp.size; ++k) acc += sm.dred[k * seg + (row - r_lo)];
    D[row] = acc;
  }
  __syncthreads();
  tl_mark(a, sm);  // cluster reduce done
}

// Final RMSNorm + score head (no cast) for stream s from sm.xres; CTA 0 only.
template <typename T>
__device__ void block_score(const StepArgs& a, int s, Smem2& sm) {
  norm_smem<T>(sm.xres, (const T*)a.final_norm, a.width, a.epsilon, sm);
  float acc = 0.f;
  for (int i = threadIdx.x; i < a.width; i += kThreads)
    acc = fmaf(Storage<T>::load((const T*)a.score_w, i), sm.g.xs[i], acc);
  const float total = block_sum(acc, sm.g);
  if (threadIdx.x == 0) a.score[s] = total;
  __syncthreads();
}

__device__ __forceinline__ void write_hidden(const StepArgs& a, int s, int l, const float* x) {
  float* hidden = a.hidden + ((size_t)s * a.layers + l) * a.width;
  float* xg = a.x + (size_t)s * a.width;
  for (int i = threadIdx.x; i < a.width; i += kThreads) {
    hidden[i] = x[i];
    xg[i] = x[i];
  }
}

// Whole step inside one cooperative cluster launch; `input` is [S][features].
// Every CTA keeps x and x' in shared memory. Streams run one after another.
template <typename T>
__device__ bool forward2(const StepArgs& a, const float* input, ClusterGridSync& gs, Smem2& sm) {
  const ClusterPos cp = ClusterPos::get();
  for (int s = 0; s < a.streams; ++s) {
    tl_mark(a, sm);  // step start
    block_input<T>(a, s, input, sm.xres, sm);
    tl_mark(a, sm);  // input projection done
    for (int l = 0; l < a.layers; ++l) {
      for (int h = (int)cp.id; h < a.heads; h += (int)cp.count) {
        norm_smem<T>(sm.xres, (const T*)a.layer[l].norm1, a.width, a.epsilon, sm);
        tl_mark(a, sm);  // norm1 done
        attention_head<T>(a, l, s, h, cp, sm);
        if (h + (int)cp.count < a.heads) cluster_sync();
      }
      if (!gs.sync(a, a.bar_timeout_ns, &sm.sync_ok)) return false;
      tl_mark(a, sm);  // grid sync A done
      residual_from_heads<T>(a, s, sm);
      tl_mark(a, sm);  // x' done
      block_ffn<T>(a, l, s, cp, sm);
      if (!gs.sync(a, a.bar_timeout_ns, &sm.sync_ok)) return false;
      tl_mark(a, sm);  // grid sync B done
      residual_from_clusters<T>(a, s, (int)cp.count, sm);
      tl_mark(a, sm);  // x done
      if (blockIdx.x == 0) write_hidden(a, s, l, sm.xres);
    }
    if (blockIdx.x == 0) block_score<T>(a, s, sm);
  }
  if (blockIdx.x == 0)
    for (int s = threadIdx.x; s < a.streams; s += kThreads) a.position[s] = ld_cg_u64(a.position + s) + 1;
  return true;
}

__host__ __device__ inline int forward2_barriers(int layers, int streams) { return 2 * layers * streams; }

// ---------------------------------------------------------------- per-op kernels' bodies
// Residual state crosses kernels through a.x (x entering the layer / after it)
// and a.x2 (x' after attention), written by CTA 0.
template <typename T>
__device__ void op_input(const StepArgs& a, Smem2& sm) {
  for (int s = 0; s < a.streams; ++s) {
    block_input<T>(a, s, a.input, sm.xres, sm);
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
__device__ void op_attention(const StepArgs& a, int l, Smem2& sm) {
  const ClusterPos cp = ClusterPos::get();
  for (int s = 0; s < a.streams; ++s) {
    if (l == 0) {
      for (int i = threadIdx.x; i < a.width; i += kThreads) sm.xres[i] = ld_cg(a.x + (size_t)s * a.width + i);
      __syncthreads();
    } else {
      for (int i = threadIdx.x; i < a.width; i += kThreads) sm.x2res[i] = ld_cg(a.x2 + (size_t)s * a.width + i);
      __syncthreads();
      residual_from_clusters<T>(a, s, (int)cp.count, sm);
      if (blockIdx.x == 0) write_hidden(a, s, l - 1, sm.xres);
      __syncthreads();
    }
    for (int h = (int)cp.id; h < a.heads; h += (int)cp.count) {
      norm_smem<T>(sm.xres, (const T*)a.layer[l].norm1, a.width, a.epsilon, sm);
      attention_head<T>(a, l, s, h, cp, sm);
      if (h + (int)cp.count < a.heads) cluster_sync();
    }
  }
}

template <typename T>
__device__ void op_ffn(const StepArgs& a, int l, Smem2& sm) {
  const ClusterPos cp = ClusterPos::get();
  for (int s = 0; s < a.streams; ++s) {
    for (int i = threadIdx.x; i < a.width; i += kThreads) sm.xres[i] = ld_cg(a.x + (size_t)s * a.width + i);
    __syncthreads();
    residual_from_heads<T>(a, s, sm);
    if (blockIdx.x == 0) {
      float* x2 = a.x2 + (size_t)s * a.width;
      for (int i = threadIdx.x; i < a.width; i += kThreads) x2[i] = sm.x2res[i];
    }
    block_ffn<T>(a, l, s, cp, sm);
  }
}

// Completes the last layer, the score and position++ (CTA 0 of cluster 0 only).
template <typename T>
__device__ void op_final(const StepArgs& a, int nclusters, Smem2& sm) {
  if (blockIdx.x != 0) return;
  for (int s = 0; s < a.streams; ++s) {
    for (int i = threadIdx.x; i < a.width; i += kThreads) sm.x2res[i] = ld_cg(a.x2 + (size_t)s * a.width + i);
    __syncthreads();
    residual_from_clusters<T>(a, s, nclusters, sm);
    write_hidden(a, s, a.layers - 1, sm.xres);
    __syncthreads();
    block_score<T>(a, s, sm);
  }
  for (int s = threadIdx.x; s < a.streams; s += kThreads) a.position[s] = ld_cg_u64(a.position + s) + 1;
}

}  // namespace st
