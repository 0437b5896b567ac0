// st_device.cuh -- device side of the B200 streaming step (sm_100a).
//
// One event per stream flows through input projection, per layer
// [RMSNorm, QKV + RoPE + ring insert, split-window attention, out-projection +
// residual, RMSNorm, gate/up + SwiGLU, down-projection + residual], final
// RMSNorm and a 1-row score head (reference src/cuda/Primitives.cuh:137-278,
// src/cpu/Cpu.cpp:59-141). Cast points and op order follow the reference; see
// each phase below.
//
// Work split: every phase spreads its rows over all CTAs (contiguous row
// ranges, so a CTA's weight slice is one contiguous span of HBM) and each CTA
// streams its span with 16-byte non-temporal loads, many in flight per thread.
// Phases are separated by a grid barrier (fused / persistent kernels) or a
// kernel boundary (per-op and graph backends). Six phases per layer replace the
// reference's 17 stages: RoPE and ring insert run in the QKV epilogue, SwiGLU in
// the gate/up epilogue, residuals in the projection epilogues, and RMSNorm is
// recomputed redundantly by every CTA from the 2-4 KB residual vector.
//
// Coherence: weights are the only data read through the non-coherent path
// (they never change while a kernel runs). Activations, ring slots, partials
// and positions are written by other CTAs inside the same kernel, so they are
// read with ld.global.cg (L2 only); the event input may be mapped host memory
// rewritten between steps and is read with ld.global.cv.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace st {

constexpr int kThreads = 512;               // threads per CTA in every kernel
constexpr int kWarps = kThreads / 32;
constexpr int kRowTile = 64;                // GEMV rows per shared-memory tile
constexpr int kMaxCols = 1024;              // max(width, features, head_dim): GEMV input length
constexpr int kMaxBlocksPerRow = kMaxCols / 4 / 32;  // fp32: 16-byte vectors / 32 lanes
constexpr int kAttChunk = 32;               // ring slots per attention work item
constexpr int kMaxLayers = 16;
constexpr int kUnroll = 8;                  // 16-byte loads in flight per lane
constexpr int kMaxTp = 8;                   // GPUs one tensor-parallel stream may span

enum ErrorCode : int { kOk = 0, kBarrierTimeout = 1, kAborted = 2, kClusterShape = 3, kRingTable = 4 };
enum Command : int { kRun = 1, kReset = 2, kStop = 3, kPing = 4 };

struct LayerPtrs {
  const void* norm1;
  const void* norm2;
  const void* qkv;     // [H][3][hd][d]: per head its q rows, k rows, v rows
  const void* out;     // [H][d][hd]: per head the out-projection columns it feeds
  const void* gateup;  // [2F, d]: row 2i = gate_i, row 2i+1 = up_i
  const void* down;    // [F][d]: W_down transposed
};

// Everything a step needs; passed by value to every kernel.
struct StepArgs {
  int layers, width, heads, ffn, window, features, head_dim, streams;
  float epsilon;
  int nchunks_max;                    // ceil(window / kAttChunk)
  const void* input_w;                // [d, features]
  const void* final_norm;             // [d]
  const void* score_w;                // [1, d]
  LayerPtrs layer[kMaxLayers];
  const float* rope_freq;             // [head_dim / 2]: 10000^(-i/head_dim), host powf
  void* keys;                         // [S][L][H][W][hd] storage type
  void* values;
  float* hidden;                      // [S][L][d]
  unsigned long long* position;       // [S]
  const float* input;                 // [S][features] (device or mapped host)
  float* x;                           // [S][d] residual entering / leaving a layer (per-op backends)
  float* x2;                          // [S][d] residual after attention (per-op backends)
  float* q;                           // [S][d] rotated, cast query (op-level attention)
  float* part;                        // [S][H][nchunks_max][hd + 2] op-level attention partials
  float* act;                         // unused by the step kernels
  float* score;                       // [S]
  unsigned long long* bar_counter;    // grid barrier arrivals (monotonic)
  int* error;                         // first error code, 0 = none (device memory)
  int* host_error;                    // mapped host mirror of the error word (may be null)
  unsigned long long bar_timeout_ns;  // bound on any single barrier wait
  float* pout;                        // [S][H][d] out-projection partial per head
  float* dpart;                       // [S][clusters][d] down-projection partial per cluster
  float* trace_attention;             // [S][d] merged attention, diagnostics only (null in timed paths)
  float* trace_qkv;                   // [S][3][d] rotated q, k and v, diagnostics only
  float* trace_act;                   // [S][F] SwiGLU output, diagnostics only
  long long* timeline;                // clock64() of one CTA at phase boundaries, diagnostics only
  int timeline_capacity;
  int timeline_cta;                   // the CTA that records the timeline
  int l2_keep_layers;                 // layers whose weights are kept L2-resident (weight ring)
  // tensor parallelism of one stream over tp_size GPUs (single-stream kernel):
  // this GPU owns heads [tp_rank H / tp_size, +H / tp_size) and ffn rows
  // [tp_rank F / tp_size, +F / tp_size); record buffers of every GPU (this
  // one at tp_rank), mapped into this GPU's address space
  int tp_rank, tp_size;
  unsigned long long* ll_heads_peer[kMaxTp];  // [2][H][d] out-projection records on each GPU
  unsigned long long* ll_xd_peer[kMaxTp];     // [2][tp_size][d] GPU-local down sums on each GPU
  unsigned long long* ll_xd;                  // this GPU's [2][tp_size][d] down-sum records
  int test_drop_cta;                  // failure-path test only (-1 off): this CTA of the single-stream
                                      // kernel withholds its layer-0 out-projection records, so every
                                      // exchange-1 wait runs out its bound
  int cluster_size;                   // CTAs per cluster the buffers were sized for
  int clusters;                       // clusters in the grid (sizes dpart)
  // single-stream flow kernel (st_flow.cuh)
  unsigned long long* ll_heads;       // [2][H][d] tagged out-projection partials per head
  unsigned long long* ll_clusters;    // [2][clusters][d] tagged down-projection partials per cluster
  unsigned long long* flow_epoch;     // tag base for the next launch
  unsigned long long* flow_ctl;       // persistent: tagged command word
  unsigned long long* flow_seq;       // persistent: mailbox sequence of the command
  // batched round (all streams per pass over the weights)
  float* bx;                          // [S][d] residual x
  float* bx2;                         // [S][d] residual x'
  float* bz;                          // [S][K] input of the next GEMM phase (K = d or F)
  float* bpart;                       // [split][S][rows] K-split partials of the last GEMM phase
  int bsplit[4];                      // K-splits of the q/k/v, out, gate/up and down GEMMs
  int tc_n[4];                        // streams per tensor-core unit (MMA N) of the same GEMMs
  // batched round on the tensor cores (16-bit modes)
  const void* tqkv[kMaxLayers];       // weights pre-tiled for the MMA (128-row x 64-column core-matrix tiles)
  const void* tout[kMaxLayers];
  const void* tgateup[kMaxLayers];
  const void* tdown[kMaxLayers];
  void* bz16;                         // next GEMM input, storage type, tiled [K/64][spad/8][8][8][8]
  void* bz16_act;                     // the down GEMM's input (SwiGLU output) when the gate/up epilogue makes it
  int fuse_swiglu;                    // gate/up GEMM without K-split computes SwiGLU in its epilogue
  int spad;                           // streams rounded up to 16 (MMA N granularity)
  int tc_stages;                      // shared-memory stages of the MMA pipeline
  unsigned tc_stage_bytes;            // bytes per stage: A tile 16 KB + B tile (<= 256 streams x 128 B)
  unsigned tc_ncols;                  // tensor-memory columns allocated (power of two >= 32)
  unsigned att_buf_bytes;             // staged batched attention: bytes per warp stage, K then V (0: direct loads)
  int att_chunk;                      // ring slots per stage (a power of two <= 16)
  int att_stages;                     // stages per warp
  unsigned att_table_bytes;           // the q/k/v table ahead of the stages in dynamic shared memory
  int att_hd64;                       // staged attention by the head-dim-64 phase (q table in static memory)
};

// ---------------------------------------------------------------- storage types
template <typename T> struct Storage;
template <> struct Storage<float> {
  static constexpr int kVec = 4;
  __device__ static float load(const float* p, size_t i) { return p[i]; }
  __device__ static float load_cg(const float* p, size_t i) { return __ldcg(p + i); }
  __device__ static float round(float v) { return v; }
  __device__ static void store(float* p, size_t i, float v) { p[i] = v; }
  __device__ static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
};
template <> struct Storage<__half> {
  static constexpr int kVec = 8;
  __device__ static float load(const __half* p, size_t i) { return __half2float(p[i]); }
  __device__ static float load_cg(const __half* p, size_t i) { return __half2float(__ldcg(p + i)); }
  __device__ static float round(float v) { return __half2float(__float2half_rn(v)); }
  __device__ static void store(__half* p, size_t i, float v) { p[i] = __float2half_rn(v); }
  __device__ static void unpack(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
      float2 t = __half22float2(h);
      f[2 * k] = t.x; f[2 * k + 1] = t.y;
    }
  }
};
template <> struct Storage<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ static float load(const __nv_bfloat16* p, size_t i) { return __bfloat162float(p[i]); }
  __device__ static float load_cg(const __nv_bfloat16* p, size_t i) { return __bfloat162float(__ldcg(p + i)); }
  __device__ static float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
  __device__ static void store(__nv_bfloat16* p, size_t i, float v) { p[i] = __float2bfloat16_rn(v); }
  __device__ static void unpack(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      f[2 * k] = __uint_as_float(w[k] << 16);
      f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  }
};

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  // Weights are read once per step: skip L1, default L2 policy.
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ unsigned long long ld_cg_u64(const unsigned long long* p) { return __ldcg(p); }
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile_int(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void set_error(const StepArgs& a, int code) {
  if (atomicCAS(a.error, 0, code) == 0 && a.host_error) {
    *reinterpret_cast<volatile int*>(a.host_error) = code;
    __threadfence_system();
  }
}

// Grid barrier on a monotonically increasing arrival counter. Every CTA keeps
// the same local epoch count; `base` is the counter value when the launch
// started. Returns false (and records the error) when the wait exceeds the
// bound or another CTA already failed; callers then leave the kernel.
struct GridSync {
  unsigned long long base;
  unsigned long long epoch;
  __device__ bool sync(const StepArgs& a, unsigned long long timeout_ns) {
    __syncthreads();
    __shared__ int ok;
    if (threadIdx.x == 0) {
      epoch += 1;
      const unsigned long long target = base + epoch * gridDim.x;
      red_release_gpu_add(a.bar_counter, 1ull);
      int good = 1;
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
      ok = good;
    }
    __syncthreads();
    return ok != 0;
  }
};

// ---------------------------------------------------------------- shared scratch
struct alignas(16) Smem {
  float xs[kMaxCols];                        // GEMV input vector (one stream)
  float red[kRowTile * kMaxBlocksPerRow];    // per-(row, 32-vector block) partials
  float rowsum[kRowTile];
  float warp_scratch[kWarps];                // block_sum slot (16-byte aligned)
  float max_scratch[kWarps];                 // block_max slot
  float scalar[4];
};
static_assert(kWarps % 4 == 0, "block reductions read the warp totals as float4");

// Block-wide reductions in one barrier: each warp reduces its lanes, lane 0
// posts the warp total into `slot` (kWarps floats, 16-byte aligned), and after
// the barrier every thread combines the kWarps totals in the same fixed order.
// Two uses of one slot must be separated by a __syncthreads; every caller
// below reaches one (a GEMV tile, a norm's final barrier) before its next use.
__device__ __forceinline__ float block_reduce_sum(float v, float* slot) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) slot[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; w += 4) {
    const float4 q = *reinterpret_cast<const float4*>(slot + w);
    t += (q.x + q.y) + (q.z + q.w);
  }
  return t;
}

__device__ __forceinline__ float block_reduce_max(float v, float* slot) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) slot[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = -INFINITY;
#pragma unroll
  for (int w = 0; w < kWarps; w += 4) {
    const float4 q = *reinterpret_cast<const float4*>(slot + w);
    t = fmaxf(t, fmaxf(fmaxf(q.x, q.y), fmaxf(q.z, q.w)));
  }
  return t;
}

__device__ __forceinline__ float block_sum(float v, Smem& sm) { return block_reduce_sum(v, sm.warp_scratch); }
__device__ __forceinline__ float block_max(float v, Smem& sm) { return block_reduce_max(v, sm.max_scratch); }

// RMSNorm of a residual vector into sm.xs, cast to storage precision
// (reference src/cpu/Cpu.cpp:43-57: scale = 1/sqrt(mean(x^2)+eps), out = x*scale*g).
template <typename T>
__device__ void norm_to_smem(const float* x, const T* gain, int width, float eps, Smem& sm) {
  float s = 0.f;
  for (int i = threadIdx.x; i < width; i += kThreads) {
    const float v = ld_cg(x + i);
    sm.xs[i] = v;
    s += v * v;
  }
  const float total = block_sum(s, sm);
  const float scale = 1.0f / sqrtf(total / (float)width + eps);
  for (int i = threadIdx.x; i < width; i += kThreads)
    sm.xs[i] = Storage<T>::round(sm.xs[i] * scale * Storage<T>::load(gain, i));
  __syncthreads();
}

template <typename T>
__device__ __forceinline__ float dot_vec(const uint4& w, const float* x) {
  constexpr int V = Storage<T>::kVec;
  float f[V];
  Storage<T>::unpack(w, f);
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < V; k += 4) {
    const float4 xv = *reinterpret_cast<const float4*>(x + k);
    acc = fmaf(f[k], xv.x, acc);
    acc = fmaf(f[k + 1], xv.y, acc);
    acc = fmaf(f[k + 2], xv.z, acc);
    acc = fmaf(f[k + 3], xv.w, acc);
  }
  return acc;
}

// rowsum[i] = sum_c W[row0 + i, c] * xs[c] for i < nrows (nrows <= kRowTile),
// fp32 accumulation in a fixed order (bit-stable run to run). All threads call.
template <bool kShared>
__device__ __forceinline__ uint4 ld_weights(const void* p) {
  if constexpr (kShared) return *reinterpret_cast<const uint4*>(p);
  else return ld_stream(p);
}

// kShared: W points at rows staged in this CTA's shared memory (same
// arithmetic, so both sources give bit-identical sums).
template <typename T, bool kShared = false>
__device__ void gemv_tile(const T* __restrict__ W, int row0, int nrows, int cols, Smem& sm) {
  constexpr int V = Storage<T>::kVec;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const T* base = W + (size_t)row0 * cols;
  const bool vec_ok = (cols % V) == 0;
  const int vpr = cols / V;
  if (vec_ok && (vpr & 31) == 0) {
    // 32 consecutive 16-byte vectors of one row per warp block.
    const int bpr = vpr >> 5;
    const int nblk = nrows * bpr;
    for (int b0 = warp; b0 < nblk; b0 += kWarps * kUnroll) {
      uint4 w[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int blk = b0 + u * kWarps;
        if (blk < nblk) {
          const int r = blk / bpr, cb = blk - r * bpr;
          w[u] = ld_weights<kShared>(base + (size_t)r * cols + (size_t)((cb << 5) + lane) * V);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int blk = b0 + u * kWarps;
        if (blk < nblk) {
          const int r = blk / bpr, cb = blk - r * bpr;
          float acc = dot_vec<T>(w[u], sm.xs + ((cb << 5) + lane) * V);
          acc = warp_sum(acc);
          if (lane == 0) sm.red[blk] = acc;
          (void)r;
        }
      }
    }
    __syncthreads();
    for (int r = threadIdx.x; r < nrows; r += kThreads) {
      float s = 0.f;
      for (int k = 0; k < bpr; ++k) s += sm.red[r * bpr + k];
      sm.rowsum[r] = s;
    }
  } else if (vec_ok && (32 % vpr) == 0) {
    // Short rows: 32 / vpr rows per warp, one vector per lane.
    const int rpw = 32 / vpr;
    const int sub = lane / vpr, c = lane - sub * vpr;
    for (int r0 = warp * rpw; r0 < nrows; r0 += kWarps * rpw) {
      const int r = r0 + sub;
      float acc = 0.f;
      if (r < nrows) acc = dot_vec<T>(ld_weights<kShared>(base + (size_t)r * cols + (size_t)c * V), sm.xs + c * V);
      for (int o = vpr >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (c == 0 && r < nrows) sm.rowsum[r] = acc;
    }
  } else if (vec_ok) {
    for (int r = warp; r < nrows; r += kWarps) {
      float acc = 0.f;
      for (int c = lane; c < vpr; c += 32)
        acc += dot_vec<T>(ld_weights<kShared>(base + (size_t)r * cols + (size_t)c * V), sm.xs + c * V);
      acc = warp_sum(acc);
      if (lane == 0) sm.rowsum[r] = acc;
    }
  } else {
    // Unaligned rows: scalar loads.
    for (int r = warp; r < nrows; r += kWarps) {
      float acc = 0.f;
      for (int c = lane; c < cols; c += 32) acc = fmaf(Storage<T>::load(base, (size_t)r * cols + c), sm.xs[c], acc);
      acc = warp_sum(acc);
      if (lane == 0) sm.rowsum[r] = acc;
    }
  }
  __syncthreads();
}

// Contiguous share [lo, hi) of `units` for this CTA.
__device__ __forceinline__ void cta_range(int units, int& lo, int& hi) {
  lo = (int)(((long long)units * blockIdx.x) / gridDim.x);
  hi = (int)(((long long)units * (blockIdx.x + 1)) / gridDim.x);
}

// Runs gemv over this CTA's rows [lo*unit, hi*unit) in tiles and calls
// epi(row, sum) for each row (all threads participate; epi is called by the
// thread that owns the row within the tile, possibly in pairs).
template <typename T, typename Epi>
__device__ void cta_gemv(const T* W, int rows, int cols, int unit, Smem& sm, Epi epi) {
  int lo, hi;
  cta_range(rows / unit, lo, hi);
  const int r_begin = lo * unit, r_end = hi * unit;
  for (int r0 = r_begin; r0 < r_end; r0 += kRowTile) {
    const int n = min(kRowTile, r_end - r0);
    gemv_tile<T>(W, r0, n, cols, sm);
    epi(r0, n);
    __syncthreads();
  }
}

// ---------------------------------------------------------------- phases

// One (stream, head, chunk of <= 32 ring slots) work item per warp, used by the
// op-level attention entry point (st_static.cu).
// q.K/sqrt(hd), chunk max, exp, sum and sum p*V -> partial (m, l, acc[hd]).
// Physical ring slots [0, valid) are the retained history; softmax does not
// depend on their order (reference src/cpu/Cpu.cpp:97-110).
template <typename T, int DPL>
__device__ void attention_item(const StepArgs& a, int l, int s, int h, int c, int valid) {
  const int lane = threadIdx.x & 31;
  const int hd = a.head_dim, W = a.window, H = a.heads;
  const int j0 = c * kAttChunk;
  const int nj = min(kAttChunk, valid - j0);
  const size_t head_base = ((((size_t)s * a.layers + l) * H + h) * (size_t)W) * hd;
  const T* K = (const T*)a.keys + head_base;
  const T* Vv = (const T*)a.values + head_base;
  const float* q = a.q + (size_t)s * a.width + (size_t)h * hd;
  float score = -INFINITY;
  if (lane < nj) {
    const T* krow = K + (size_t)(j0 + lane) * hd;
    float dot = 0.f;
    for (int i = 0; i < hd; ++i) dot = fmaf(ld_cg(q + i), Storage<T>::load_cg(krow, i), dot);
    score = dot / sqrtf((float)hd);
  }
  const float m = warp_max(score);
  const float p = lane < nj ? expf(score - m) : 0.f;
  const float lsum = warp_sum(p);
  float acc[DPL];
#pragma unroll
  for (int k = 0; k < DPL; ++k) acc[k] = 0.f;
  for (int j = 0; j < nj; ++j) {
    const float pj = __shfl_sync(0xffffffffu, p, j);
    const T* vrow = Vv + (size_t)(j0 + j) * hd;
#pragma unroll
    for (int k = 0; k < DPL; ++k) {
      const int dd = lane + 32 * k;
      if (dd < hd) acc[k] = fmaf(pj, Storage<T>::load_cg(vrow, dd), acc[k]);
    }
  }
  float* out = a.part + ((((size_t)s * H + h) * a.nchunks_max + c) * (size_t)(hd + 2));
  if (lane == 0) { out[0] = m; out[1] = lsum; }
#pragma unroll
  for (int k = 0; k < DPL; ++k) {
    const int dd = lane + 32 * k;
    if (dd < hd) out[2 + dd] = acc[k];
  }
}

// Zero K/V/hidden and position for streams [s0, s1) (reference
// src/cuda/Primitives.cuh:280-292), grid-stride over all CTAs.
template <typename T>
__device__ void reset_streams(const StepArgs& a, int s0, int s1) {
  const size_t per_stream = (size_t)a.layers * a.width * a.window;
  const size_t begin = (size_t)s0 * per_stream, end = (size_t)s1 * per_stream;
  const size_t stride = (size_t)gridDim.x * kThreads;
  for (size_t i = begin + (size_t)blockIdx.x * kThreads + threadIdx.x; i < end; i += stride) {
    Storage<T>::store((T*)a.keys, i, 0.f);
    Storage<T>::store((T*)a.values, i, 0.f);
  }
  const size_t hb = (size_t)s0 * a.layers * a.width, he = (size_t)s1 * a.layers * a.width;
  for (size_t i = hb + (size_t)blockIdx.x * kThreads + threadIdx.x; i < he; i += stride) a.hidden[i] = 0.f;
  if (blockIdx.x == 0)
    for (int s = s0 + threadIdx.x; s < s1; s += kThreads) a.position[s] = 0ull;
}

}  // namespace st
