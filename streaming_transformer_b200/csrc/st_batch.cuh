// st_batch.cuh -- the batched round: one step of every stream in one pass over
// the weights.
//
// With S independent streams the per-stream GEMVs of the step become skinny
// GEMMs (rows = weight rows, columns = streams), so every weight byte is read
// once per round instead of once per stream. A round is a sequence of phases
// over the whole grid (one CTA per SM, 512 threads), separated by grid
// barriers:
//
//   P0   per stream: x = cast(W_in e), z = norm1_0(x)               (CTA per stream)
//   per layer l:
//   G1   Pq[k][s][m]  = sum_{k-split} Wqkv[m] . z[s]                (warp units)
//   A    per (stream, head): q, k, v = cast(sum_k Pq), RoPE, cast, K/V slot
//        insert, window attention (each warp a slice of the slots, online
//        softmax, merged in warp order), a = cast(out)               (CTA per unit)
//   G2   Po = W_out . a                                             (warp units)
//   R2   per stream: x' = cast(x + cast(sum_k Po)), z = norm2(x')    (CTA per stream)
//   G3   Pg = W_gateup . z                                          (warp units)
//   R3   act = cast(silu(cast(sum_k Pg[2f])) cast(sum_k Pg[2f+1]))  (elementwise)
//   G4   Pd = W_down . act                                          (warp units)
//   R1   per stream: x = cast(x' + cast(sum_k Pd)), hidden[l] = x, then norm1
//        of layer l+1 or, after the last layer, the final norm and score
//
// The math and cast points are the reference step's (reference
// src/cpu/Cpu.cpp:59-141); only the summation order of the dot products
// differs from the one-stream path. Every K-split partial is written to its
// own slot and summed in split order, so a round is deterministic.
//
// GEMM warp unit: 64 weight rows (two per lane) x 32 streams over one K
// range; the lane keeps its two rows' weights in registers for 8 columns at a
// time and the streams' inputs arrive as uniform (broadcast) 16-byte loads,
// so each weight element feeds 32 FMAs. Data written inside the launch by
// other CTAs (inputs, partials, residuals) is read through L2 (ld.cg); only
// weights take the read-only path.
#pragma once

#include "st_step.cuh"
#include "st_umma.cuh"

namespace st {

constexpr int kBatchStreams = 32;     // streams per GEMM warp unit
constexpr int kBatchRows = 64;        // weight rows per GEMM warp unit (two per lane)
constexpr int kBatchMaxHeadDim = 256; // attention unit: head_dim <= 256 (4 dim pairs per lane)

// How the GEMM reads W[m][k] from the weight slab.
enum BatchView : int {
  kViewRows = 0,      // W[m * K + k] (q/k/v fused [3d, d], gate/up interleaved [2F, d])
  kViewOutHeads = 1,  // out projection stored per head [H][d][hd]: W[(k / hd) * d * hd + m * hd + k % hd]
  kViewColumns = 2    // W_down stored transposed [F][d]: W[k * M + m]
};

// Attention units run four at a time per CTA, one per group of four warps.
constexpr int kAttGroups = 4;
constexpr int kAttWarps = kWarps / kAttGroups;
constexpr int kAttThreads = kAttWarps * 32;

struct AttSmem {
  float q[kBatchMaxHeadDim];                      // rotated, cast q, k, v of the unit
  float k[kBatchMaxHeadDim];
  float v[kBatchMaxHeadDim];
  float part_m[kAttWarps];                        // per-warp softmax partials
  float part_l[kAttWarps];
  float part_acc[kAttWarps][kBatchMaxHeadDim];
};

// Staged attention (attention_phase_staged): each warp walks whole (stream,
// head) units through its own ring of K/V stages in dynamic shared memory.
constexpr int kAttMaxStages = 8;                  // stages per warp at most (cp.async groups pending <= 7)
constexpr int kAttMaxChunk = 16;                  // ring slots per stage at most

// Bytes of the staged attention's q/k/v table for `units` units of head_dim
// hd: the final q, k, v rows (fp32), then each unit's {slot, valid}; the
// stages start at the next 128-byte boundary (host and device).
__host__ __device__ inline unsigned att_table_bytes(int units, int hd) {
  const unsigned rows = ((unsigned)units * 3u * (unsigned)hd * 4u + 15u) / 16u * 16u;
  return (rows + (unsigned)units * 8u + 127u) / 128u * 128u;
}

struct BatchSmem {
  float red[kWarps];                              // block reductions (16-byte aligned)
  union __align__(16) {
    AttSmem att[kAttGroups];                      // attention phase (direct loads)
    float zt[kWarps][kBatchStreams * 8];          // GEMM phases: each warp's stream-input tile
    float xs[kMaxCols];                           // row phases: per-stream input vector
  } u;
  int tl_n;                                       // timeline marks recorded (diagnostics)
  // tensor-core GEMM pipeline (kTc rounds)
  unsigned long long tc_full[8];                  // stage landed (bulk-copy bytes)
  unsigned long long tc_empty[8];                 // stage consumed (MMA commit)
  unsigned long long tc_tfull;                    // unit's accumulator complete (MMA commit)
  unsigned long long tc_tempty;                   // unit's accumulator read (4 epilogue warps)
  unsigned long long tc_done;                     // every MMA issued has completed (teardown)
  unsigned tc_tmem;                               // tensor-memory base address
};
constexpr int kTcMaxStages = 8;
constexpr int kTcProducer = kThreads - 32;        // lane 0 of the last warp: bulk copies
constexpr int kTcIssuer = kThreads - 64;          // lane 0 of the next-to-last warp: MMAs
constexpr unsigned kTcTileBytes = kUmmaM * kTileK * 2;  // one 128 x 64 16-bit A tile
constexpr int kTcMaxN = 256;                      // streams per MMA (N)

// Diagnostics: thread 0 of the timeline CTA records clock64() << 8 | tag at
// every phase end and barrier exit (warp 0's row of the timeline buffer).
enum BatchTag : int {
  kBtlInput = 40, kBtlQkv = 41, kBtlAttention = 42, kBtlOut = 43, kBtlResidual2 = 44, kBtlGateUp = 45,
  kBtlSwiglu = 46, kBtlDown = 47, kBtlResidual1 = 48, kBtlSync = 49,
  kBtlAttPrepare = 50
};
__device__ __forceinline__ void btl(const StepArgs& a, BatchSmem& sm, int tag) {
  if (a.timeline && blockIdx.x == a.timeline_cta && threadIdx.x == 0 && sm.tl_n < a.timeline_capacity / kWarps)
    a.timeline[sm.tl_n++] = (long long)((clock64() << 8) | (long long)tag);
}

// Round barriers per launch step: one after P0, eight per layer (seven when
// the gate/up epilogue computes SwiGLU), none after the last R1 (the next
// round's P0 of a stream runs on the CTA that did its R1).
__host__ __device__ inline int round_barriers(int layers, bool fused_swiglu) {
  return (fused_swiglu ? 7 : 8) * layers;
}

// True when the batched round supports this model (host and device).
__host__ __device__ inline bool batch_supported(int width, int heads, int ffn, int features) {
  const int hd = heads > 0 ? width / heads : 0;
  return width <= kMaxCols && features <= kMaxCols && hd % 8 == 0 && hd >= 8 && hd <= kBatchMaxHeadDim &&
         width % 8 == 0 && ffn % 8 == 0;
}

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// Stores element (stream s, column k) of the next GEMM's input: fp32 [S][K]
// for the CUDA-core GEMM, or the storage type in the MMA's tiled B layout
// for the tensor cores: one tile of all `spad` streams x 64 columns per K
// chunk, so the B operand of streams [s0, s0 + N) in chunk c is one contiguous
// run of N x 128 bytes. fp32 on the tensor cores: tf32 hi and lo planes of 32
// columns per chunk, the lo plane spad x K floats after the hi plane.
template <typename T, bool kTc>
__device__ __forceinline__ void put_z_at(const StepArgs& a, void* dst, int s, int k, int K, float v) {
  if constexpr (kTc && std::is_same<T, float>::value) {
    float* z = (float*)dst;
    const unsigned at = z_tile_offset32((unsigned)s, (unsigned)k, (unsigned)a.spad);
    const float hi = to_tf32(v);
    z[at] = hi;
    z[(size_t)a.spad * K + at] = to_tf32(v - hi);
  } else if constexpr (kTc) {
    Storage<T>::store((T*)dst, z_tile_offset((unsigned)s, (unsigned)k, (unsigned)a.spad), v);
  } else {
    a.bz[(size_t)s * K + k] = v;
  }
}
template <typename T, bool kTc>
__device__ __forceinline__ void put_z(const StepArgs& a, int s, int k, int K, float v) {
  put_z_at<T, kTc>(a, a.bz16, s, k, K, v);
}

// Two consecutive cache elements (K/V rows are 16-byte aligned, dim even).
template <typename T> __device__ __forceinline__ float2 load2_shared(const T* p);
template <> __device__ __forceinline__ float2 load2_shared<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <> __device__ __forceinline__ float2 load2_shared<__half>(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
template <> __device__ __forceinline__ float2 load2_shared<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
template <typename T> __device__ __forceinline__ float2 load2_cg(const T* p);
template <> __device__ __forceinline__ float2 load2_cg<float>(const float* p) {
  return __ldcg(reinterpret_cast<const float2*>(p));
}
template <> __device__ __forceinline__ float2 load2_cg<__half>(const __half* p) {
  const unsigned u = __ldcg(reinterpret_cast<const unsigned*>(p));
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
template <> __device__ __forceinline__ float2 load2_cg<__nv_bfloat16>(const __nv_bfloat16* p) {
  const unsigned u = __ldcg(reinterpret_cast<const unsigned*>(p));
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

// Raw (not yet widened) weights of a lane's two rows for 8 columns. (Loading
// them a step ahead as well spills at 128 registers; the warps of the SM hide
// their latency instead.)
template <typename T> struct RawBits { using U = unsigned short; };
template <> struct RawBits<float> { using U = float; };
__device__ __forceinline__ float widen(float v, float*) { return v; }
__device__ __forceinline__ float widen(unsigned short v, __nv_bfloat16*) { return __uint_as_float((unsigned)v << 16); }
__device__ __forceinline__ float widen(unsigned short v, __half*) { return __half2float(__ushort_as_half(v)); }

template <typename T, int kView>
struct WeightPair {
  static constexpr int kVecs = sizeof(T) == 4 ? 2 : 1;  // 16-byte vectors per 8 columns
  uint4 vec[2][kVecs];                                // kViewRows / kViewOutHeads
  typename RawBits<T>::U col[2][8];                   // kViewColumns

  __device__ __forceinline__ const T* row_ptr(const T* W, int M, int K, int hd, int m, int k) const {
    return kView == kViewRows ? W + (size_t)m * K + k : W + ((size_t)(k / hd) * M + m) * hd + (k % hd);
  }
  __device__ __forceinline__ void load(const T* W, int M, int K, int hd, const int (&m)[2], int k,
                                       const bool (&ok)[2]) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if constexpr (kView == kViewColumns) {
        const typename RawBits<T>::U* p = reinterpret_cast<const typename RawBits<T>::U*>(W) + (size_t)k * M + m[r];
#pragma unroll
        for (int u = 0; u < 8; ++u) col[r][u] = ok[r] ? __ldg(p + (size_t)u * M) : (typename RawBits<T>::U)0;
      } else {
        const uint4* p = reinterpret_cast<const uint4*>(row_ptr(W, M, K, hd, m[r], k));
#pragma unroll
        for (int v = 0; v < kVecs; ++v) vec[r][v] = ok[r] ? __ldg(p + v) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
  __device__ __forceinline__ void widen_to(float (&w)[2][8]) const {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if constexpr (kView == kViewColumns) {
#pragma unroll
        for (int u = 0; u < 8; ++u) w[r][u] = widen(col[r][u], (T*)nullptr);
      } else {
#pragma unroll
        for (int v = 0; v < kVecs; ++v) Storage<T>::unpack(vec[r][v], w[r] + v * Storage<T>::kVec);
      }
    }
  }
};

// One warp unit: rows [m0, m0 + 64) x streams [s0, s0 + 32) over K range
// [k0, k1) into P[ks][s][m] (P holds S x M floats per split). Lane i loads
// stream s0+i's 8 inputs one step ahead (one coalesced load per step) and
// stores them into the warp's shared tile; the FMAs read the tile with
// broadcast loads.
template <typename T, int kView>
__device__ __forceinline__ void gemm_unit(const T* W, int M, int K, int hd, const float* Z, int S, float* P,
                                          int m0, int k0, int k1, int s0, int ks, float* zt) {
  const int lane = threadIdx.x & 31;
  const int m[2] = {m0 + lane, m0 + 32 + lane};
  const bool ok[2] = {m[0] < M, m[1] < M};
  const int ns = min(kBatchStreams, S - s0);
  const bool zl = lane < ns;
  const float* zrow = Z + (size_t)(s0 + (zl ? lane : 0)) * K;
  float acc0[kBatchStreams], acc1[kBatchStreams];
#pragma unroll
  for (int s = 0; s < kBatchStreams; ++s) acc0[s] = acc1[s] = 0.f;
  float4 za = make_float4(0.f, 0.f, 0.f, 0.f), zc = za;
  if (zl) {
    za = ldcg4(zrow + k0);
    zc = ldcg4(zrow + k0 + 4);
  }
  WeightPair<T, kView> wp;
#pragma unroll 1
  for (int k = k0; k < k1; k += 8) {
    __syncwarp();  // every lane has finished reading the previous tile
    reinterpret_cast<float4*>(zt + lane * 8)[0] = za;
    reinterpret_cast<float4*>(zt + lane * 8)[1] = zc;
    float w[2][8];
    wp.load(W, M, K, hd, m, k, ok);
    wp.widen_to(w);
    __syncwarp();
    if (k + 8 < k1 && zl) {
      za = ldcg4(zrow + k + 8);
      zc = ldcg4(zrow + k + 12);
    }
#pragma unroll
    for (int s = 0; s < kBatchStreams; ++s) {
      if (s < ns) {
        const float4 a = reinterpret_cast<const float4*>(zt + s * 8)[0];
        const float4 b = reinterpret_cast<const float4*>(zt + s * 8)[1];
        const float zz[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          acc0[s] = fmaf(w[0][u], zz[u], acc0[s]);
          acc1[s] = fmaf(w[1][u], zz[u], acc1[s]);
        }
      }
    }
  }
  float* out = P + ((size_t)ks * S + s0) * M;
#pragma unroll
  for (int s = 0; s < kBatchStreams; ++s) {
    if (s < ns) {
      if (ok[0]) out[(size_t)s * M + m[0]] = acc0[s];
      if (ok[1]) out[(size_t)s * M + m[1]] = acc1[s];
    }
  }
}

// P[ks][s][m] = sum over split ks's K range of W[m][k] Z[s][k], every unit
// dealt to the grid's warps in turn.
template <typename T, int kView>
__device__ void gemm_phase(const StepArgs& a, BatchSmem& sm, const T* W, int M, int K, int ksplit, const float* Z,
                           float* P) {
  const int S = a.streams;
  const int mblocks = (M + kBatchRows - 1) / kBatchRows, sgroups = (S + kBatchStreams - 1) / kBatchStreams;
  const int kchunks = K / 8;
  const int units = mblocks * ksplit * sgroups;
  const int nwarps = (int)gridDim.x * kWarps;
  for (int u = (int)blockIdx.x * kWarps + (int)(threadIdx.x >> 5); u < units; u += nwarps) {
    const int mb = u % mblocks, rest = u / mblocks;
    const int ks = rest % ksplit, sg = rest / ksplit;
    int c0, c1;
    split(kchunks, ks, ksplit, c0, c1);
    gemm_unit<T, kView>(W, M, K, a.head_dim, Z, S, P, mb * kBatchRows, c0 * 8, c1 * 8, sg * kBatchStreams, ks,
                        sm.u.zt[threadIdx.x >> 5]);
  }
}

// Sum of the K-split partials of one output in split order; the loads of a
// group of eight are issued together so they overlap in flight.
__device__ __forceinline__ float sum_splits(const float* P, int ksplit, size_t stride) {
  float v = 0.f;
  for (int k0 = 0; k0 < ksplit; k0 += 8) {
    float t[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) t[u] = k0 + u < ksplit ? __ldcg(P + (size_t)(k0 + u) * stride) : 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (k0 + u < ksplit) v += t[u];
  }
  return v;
}

// Thread i of the CTA handles elements i and i + kThreads of a d-vector.
constexpr int kRowPer = kMaxCols / kThreads;

// RMSNorm of the CTA's row values xv of stream s (reference
// src/cpu/Cpu.cpp:43-57) into the next GEMM input (cast), or, with `score_w`,
// the final norm followed by the score head (no cast). Ends with a barrier.
template <typename T, bool kTc>
__device__ __forceinline__ void row_norm(const StepArgs& a, BatchSmem& sm, int s, const float (&xv)[kRowPer],
                                         float ss, const T* gain, const T* score_w, float* score, float* score_out) {
  const int d = a.width;
  const float total = block_reduce_sum(ss, sm.red);
  const float scale = 1.0f / sqrtf(total / (float)d + a.epsilon);
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < kRowPer; ++c) {
    const int i = (int)threadIdx.x + c * kThreads;
    if (i < d) {
      const float zi = Storage<T>::round(xv[c] * scale * Storage<T>::load(gain, i));
      if (score_w) acc = fmaf(Storage<T>::load(score_w, i), zi, acc);
      else put_z<T, kTc>(a, s, i, d, zi);
    }
  }
  __syncthreads();  // the reduction slot is reused below and by the next unit
  if (score_w) {
    const float total_score = block_reduce_sum(acc, sm.red);
    if (threadIdx.x == 0) {
      *score = total_score;
      if (score_out) *score_out = total_score;
    }
    __syncthreads();
  }
}

// P0: x = cast(W_in e) for stream s (reference src/cpu/Cpu.cpp:64-66), then norm1 of layer 0.
template <typename T, bool kTc>
__device__ void row_input(const StepArgs& a, BatchSmem& sm, int s, const float* input) {
  const int d = a.width, nf = a.features;
  for (int i = threadIdx.x; i < nf; i += kThreads) sm.u.xs[i] = __ldcv(input + (size_t)s * nf + i);
  __syncthreads();
  const T* Win = (const T*)a.input_w;
  float xv[kRowPer];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kRowPer; ++c) {
    const int i = (int)threadIdx.x + c * kThreads;
    xv[c] = 0.f;
    if (i < d) {
      float acc = 0.f;
      for (int f = 0; f < nf; ++f) acc = fmaf(Storage<T>::load(Win, (size_t)i * nf + f), sm.u.xs[f], acc);
      const float x = Storage<T>::round(acc);
      a.bx[(size_t)s * d + i] = x;
      xv[c] = x;
      ss += x * x;
    }
  }
  row_norm<T, kTc>(a, sm, s, xv, ss, (const T*)a.layer[0].norm1, nullptr, nullptr, nullptr);
}

// R1 / R2: out = cast(base + cast(sum_k P)) for stream s, then the next norm
// (gain) into z, or the final norm and score when `final_`.
template <typename T, bool kTc>
__device__ void row_residual(const StepArgs& a, BatchSmem& sm, int s, const float* base, float* out, const float* P,
                             int ksplit, float* hidden, const T* gain, bool final_, float* score_out) {
  const int d = a.width;
  const size_t stride = (size_t)a.streams * d;
  float xv[kRowPer];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kRowPer; ++c) {
    const int i = (int)threadIdx.x + c * kThreads;
    xv[c] = 0.f;
    if (i < d) {
      const float t = Storage<T>::round(sum_splits(P + (size_t)s * d + i, ksplit, stride));
      const float x = Storage<T>::round(__ldcg(base + (size_t)s * d + i) + t);
      out[(size_t)s * d + i] = x;
      if (hidden) hidden[i] = x;
      xv[c] = x;
      ss += x * x;
    }
  }
  if (final_)
    row_norm<T, kTc>(a, sm, s, xv, ss, (const T*)a.final_norm, (const T*)a.score_w, a.score + s, score_out);
  else
    row_norm<T, kTc>(a, sm, s, xv, ss, gain, nullptr, nullptr, nullptr);
}

// R3: act[s][f] = cast(silu(g) u) with g, u the cast gate/up sums
// (reference src/cpu/Cpu.cpp:121-127), every element of every stream.
template <typename T, bool kTc>
__device__ void swiglu_phase(const StepArgs& a, int ksplit) {
  const int F = a.ffn, S = a.streams;
  const size_t n = (size_t)S * F, stride = (size_t)S * 2 * F;
  for (size_t e = (size_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += (size_t)gridDim.x * kThreads) {
    const size_t s = e / F, f = e - s * F;
    const float* P = a.bpart + s * 2 * F + 2 * f;
    const float g = Storage<T>::round(sum_splits(P, ksplit, stride));
    const float u = Storage<T>::round(sum_splits(P + 1, ksplit, stride));
    put_z<T, kTc>(a, (int)s, (int)f, F, Storage<T>::round((g / (1.0f + expf(-g))) * u));
  }
}

// q . K_j over head_dim, K row from the cache (16-byte loads through L2).
template <typename T>
__device__ __forceinline__ float dot_cache_row(const T* krow, const float* q, int hd) {
  constexpr int V = Storage<T>::kVec;
  float acc = 0.f;
  for (int e = 0; e < hd; e += V) {
    float f[V];
    Storage<T>::unpack(__ldcg(reinterpret_cast<const uint4*>(krow + e)), f);
#pragma unroll
    for (int u = 0; u < V; ++u) acc = fmaf(q[e + u], f[u], acc);
  }
  return acc;
}

// Barrier of one attention group (named barrier 1 + group, kAttThreads threads).
__device__ __forceinline__ void group_sync(int group) {
  asm volatile("bar.sync %0, %1;" ::"r"(group + 1), "r"(kAttThreads) : "memory");
}

// A: stream s, head h of layer l (reference src/cpu/Cpu.cpp:72-111), run by
// one group of kAttWarps warps (`gt` = thread index within the group).
template <typename T, bool kTc>
__device__ void attention_unit(const StepArgs& a, AttSmem& sm, int group, int l, int s, int h,
                               unsigned long long event, int ksplit) {
  const int hd = a.head_dim, W = a.window, d = a.width, M = 3 * d, S = a.streams;
  const int gt = (int)threadIdx.x - group * kAttThreads;
  const int lane = gt & 31, warp = gt >> 5;
  const unsigned long long t = __ldcg(a.position + s) + event;
  const int slot = (int)(t % (unsigned long long)W);
  const int valid = valid_length(t, W);
  const size_t head_base = ((((size_t)s * a.layers + l) * a.heads + h) * (size_t)W) * hd;
  T* keys = (T*)a.keys + head_base;
  T* values = (T*)a.values + head_base;
  // q, k, v of head h: sums of the split partials, cast, RoPE on q and k in
  // adjacent pairs with angle float(t) * 10000^(-i/hd), cast (reference
  // src/cpu/Cpu.cpp:76-89), and the K/V insert at slot t % W.
  const float* P = a.bpart + (size_t)s * M + (size_t)h * 3 * hd;
  const size_t stride = (size_t)S * M;
  const float tf = (float)t;
  for (int p = gt; p < 3 * hd / 2; p += kAttThreads) {
    const int row = 2 * p, which = row / hd, dim = row - which * hd;
    float v0 = Storage<T>::round(sum_splits(P + row, ksplit, stride));
    float v1 = Storage<T>::round(sum_splits(P + row + 1, ksplit, stride));
    if (which < 2) {
      const float angle = tf * a.rope_freq[dim >> 1];
      const float c = cosf(angle), sn = sinf(angle);
      const float r0 = v0 * c - v1 * sn;
      const float r1 = v0 * sn + v1 * c;
      v0 = Storage<T>::round(r0);
      v1 = Storage<T>::round(r1);
    }
    float* dst = which == 0 ? sm.q : which == 1 ? sm.k : sm.v;
    dst[dim] = v0;
    dst[dim + 1] = v1;
    if (which > 0) {
      T* ring = which == 1 ? keys : values;
      Storage<T>::store(ring, (size_t)slot * hd + dim, v0);
      Storage<T>::store(ring, (size_t)slot * hd + dim + 1, v1);
    }
  }
  group_sync(group);
  // Each warp: slots [j0, j1), one slot per lane per pass, online softmax;
  // the current slot's key and value come from shared memory.
  int j0, j1;
  split(valid, warp, kAttWarps, j0, j1);
  const float root = sqrtf((float)hd);
  const int pairs = hd / 2;
  constexpr int kPairRegs = kBatchMaxHeadDim / 64;
  float m = -INFINITY, lsum = 0.f;
  float acc[kPairRegs][2];
#pragma unroll
  for (int c = 0; c < kPairRegs; ++c) acc[c][0] = acc[c][1] = 0.f;
  for (int c0 = j0; c0 < j1; c0 += 32) {
    const int j = c0 + lane;
    float lg = -INFINITY;
    if (j < j1) {
      float dot = 0.f;
      if (j == slot) {
        for (int i = 0; i < hd; ++i) dot = fmaf(sm.q[i], sm.k[i], dot);
      } else {
        dot = dot_cache_row<T>(keys + (size_t)j * hd, sm.q, hd);
      }
      lg = dot / root;
    }
    const float mn = fmaxf(m, warp_max(lg));
    const float sc = expf(m - mn);
    const float p = j < j1 ? expf(lg - mn) : 0.f;
    lsum = lsum * sc + warp_sum(p);
#pragma unroll
    for (int c = 0; c < kPairRegs; ++c) {
      acc[c][0] *= sc;
      acc[c][1] *= sc;
    }
    const int n = min(32, j1 - c0);
#pragma unroll 8
    for (int jj = 0; jj < n; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
      const int row = c0 + jj;
#pragma unroll
      for (int c = 0; c < kPairRegs; ++c) {
        const int pi = lane + 32 * c;
        if (pi < pairs) {
          const float2 v = row == slot ? make_float2(sm.v[2 * pi], sm.v[2 * pi + 1])
                                       : load2_cg<T>(values + (size_t)row * hd + 2 * pi);
          acc[c][0] = fmaf(pj, v.x, acc[c][0]);
          acc[c][1] = fmaf(pj, v.y, acc[c][1]);
        }
      }
    }
    m = mn;
  }
  if (lane == 0) {
    sm.part_m[warp] = m;
    sm.part_l[warp] = lsum;
  }
#pragma unroll
  for (int c = 0; c < kPairRegs; ++c) {
    const int pi = lane + 32 * c;
    if (pi < pairs) {
      sm.part_acc[warp][2 * pi] = acc[c][0];
      sm.part_acc[warp][2 * pi + 1] = acc[c][1];
    }
  }
  group_sync(group);
  // merge the warps' partials in warp order, cast (reference src/cpu/Cpu.cpp:105-111)
  for (int i = gt; i < hd; i += kAttThreads) {
    float mx = -INFINITY;
    for (int w = 0; w < kAttWarps; ++w)
      if (sm.part_l[w] > 0.f) mx = fmaxf(mx, sm.part_m[w]);
    float L = 0.f, o = 0.f;
    for (int w = 0; w < kAttWarps; ++w) {
      if (sm.part_l[w] > 0.f) {
        const float e = expf(sm.part_m[w] - mx);
        L = fmaf(sm.part_l[w], e, L);
        o = fmaf(sm.part_acc[w][i], e, o);
      }
    }
    put_z<T, kTc>(a, s, h * hd + i, d, Storage<T>::round(o / L));
  }
  group_sync(group);  // the next unit of this group overwrites q, k, v and the partials
}

// The attention phase: units (stream, head) dealt to the grid's groups in turn.
template <typename T, bool kTc>
__device__ void attention_phase(const StepArgs& a, BatchSmem& sm, int l, unsigned long long event) {
  const int group = (int)threadIdx.x / kAttThreads;
  const int units = a.streams * a.heads;
  for (int u = (int)blockIdx.x * kAttGroups + group; u < units; u += (int)gridDim.x * kAttGroups)
    attention_unit<T, kTc>(a, sm.u.att[group], group, l, u / a.heads, u % a.heads, event, a.bsplit[0]);
}

// The attention phase with K/V staged in shared memory, one warp per unit.
// The CTA owns a contiguous range of (stream, head) units u = lo + k
// (k < mine; consecutive units are adjacent K/V regions, so a CTA's reads stay
// within a few pages); warp w takes k = w, w + kWarps, ... and walks each unit's ring
// in chunks of C = a.att_chunk slots through its own a.att_stages stages.
//  * The warp's lanes copy a chunk's K rows and V rows into its next stage
//    with 16-byte cp.async (one commit group per chunk), a.att_stages - 1
//    chunks ahead of the compute; a chunk is read after its group completes
//    and a warp barrier. (One bulk copy per chunk would cost the copy engine
//    a request per 1-2 KB: measured slower at these chunk sizes.) Every chunk
//    of the window is copied; chunks past the retained slots are skipped.
//  * First, all threads finish every owned unit's q, k, v at once: sums of the
//    K-split partials, cast, RoPE on q and k (adjacent pairs, angle float(t) *
//    10000^(-i/hd)), cast, K/V insert at slot t % W (reference
//    src/cpu/Cpu.cpp:76-89), into a shared-memory table with each unit's
//    {slot, valid}.
//  * Per chunk, G = 32 / C lanes take each slot: a lane's dimension pairs are
//    rotated by its slot so the row reads hit distinct banks; the key dot sums
//    over the slot's lanes; the warp's online softmax takes the chunk; the
//    value rows accumulate with lanes over dimension pairs. After the unit's
//    last chunk, out = cast(value sum / sum) (reference src/cpu/Cpu.cpp:97-111).
// The slot this step writes comes from the unit's own k and v in the table,
// whatever its staged copy holds. No block barrier inside the unit loop.
template <typename T, bool kTc>
__device__ void attention_phase_staged(const StepArgs& a, BatchSmem& sm, unsigned char* dyn, int l,
                                       unsigned long long event) {
  const int hd = a.head_dim, W = a.window, H = a.heads, S = a.streams, d = a.width, M = 3 * d;
  const int C = a.att_chunk, NB = a.att_stages, nch = (W + C - 1) / C;
  int lo, hi;
  split(S * H, (int)blockIdx.x, (int)gridDim.x, lo, hi);
  const int mine = hi - lo;
  if (mine <= 0) return;
  if (att_table_bytes(mine, hd) > a.att_table_bytes) {  // the host sized the table for this grid
    if (threadIdx.x == 0) set_error(a, kClusterShape);
    return;
  }
  const int warp = (int)threadIdx.x >> 5, lane = (int)threadIdx.x & 31;
  const int rowf = 3 * hd;
  float* table = reinterpret_cast<float*>(dyn);
  int2* meta = reinterpret_cast<int2*>(dyn + ((unsigned)mine * (unsigned)rowf * 4u + 15u) / 16u * 16u);
  unsigned char* stages = dyn + a.att_table_bytes;
  const unsigned sbytes = a.att_buf_bytes, half = sbytes / 2;
  const int nu = mine > warp ? (mine - 1 - warp) / kWarps + 1 : 0;
  const int total = nu * nch;
  auto unit_of = [&](int k) { return lo + k; };
  auto issue = [&](int i) {  // every lane: its 16-byte pieces of chunk i into stage i % NB, one group
    if (i < total) {
      const int u = unit_of(warp + (i / nch) * kWarps), c = i % nch;
      const int su = u / H, hu = u - su * H;
      const size_t head_base = ((((size_t)su * a.layers + l) * H + hu) * (size_t)W) * hd;
      const int c0 = c * C, n = min(C, W - c0);
      unsigned char* dst = stages + (size_t)(warp * NB + i % NB) * sbytes;
      const unsigned char* ks = reinterpret_cast<const unsigned char*>((const T*)a.keys + head_base + (size_t)c0 * hd);
      const unsigned char* vs = reinterpret_cast<const unsigned char*>((const T*)a.values + head_base + (size_t)c0 * hd);
      const unsigned bytes = (unsigned)(n * hd * (int)sizeof(T));
      for (unsigned o = (unsigned)lane * 16u; o < bytes; o += 512u) {
        cp_async16(dst + o, ks + o);
        cp_async16(dst + half + o, vs + o);
      }
    }
    cp_async_commit();  // empty past the last chunk: the group count stays uniform
  };
  for (int i = 0; i < NB - 1; ++i) issue(i);
  // every owned unit's final q, k, v (and the K/V insert), all units at once
  const int per_unit = 3 * hd / 2;
  for (int x = threadIdx.x; x < mine * per_unit; x += kThreads) {
    const int k = x / per_unit, p = x - k * per_unit;
    const int u = unit_of(k), su = u / H, hu = u - su * H;
    const unsigned long long t = __ldcg(a.position + su) + event;
    const int row = 2 * p, which = row / hd, dim = row - which * hd;
    const float* P = a.bpart + (size_t)su * M + (size_t)hu * 3 * hd + row;
    float v0 = Storage<T>::round(sum_splits(P, a.bsplit[0], (size_t)S * M));
    float v1 = Storage<T>::round(sum_splits(P + 1, a.bsplit[0], (size_t)S * M));
    if (which < 2) {
      const float angle = (float)t * a.rope_freq[dim >> 1];
      const float co = cosf(angle), sn = sinf(angle);
      const float r0 = v0 * co - v1 * sn;
      const float r1 = v0 * sn + v1 * co;
      v0 = Storage<T>::round(r0);
      v1 = Storage<T>::round(r1);
    }
    table[(size_t)k * rowf + row] = v0;
    table[(size_t)k * rowf + row + 1] = v1;
    const int slot = (int)(t % (unsigned long long)W);
    if (p == 0) meta[k] = make_int2(slot, valid_length(t, W));
    if (which > 0) {
      const size_t head_base = ((((size_t)su * a.layers + l) * H + hu) * (size_t)W) * hd;
      T* ring = (T*)(which == 1 ? a.keys : a.values) + head_base;
      Storage<T>::store(ring, (size_t)slot * hd + dim, v0);
      Storage<T>::store(ring, (size_t)slot * hd + dim + 1, v1);
    }
  }
  __syncthreads();
  btl(a, sm, kBtlAttPrepare);
  const int pairs = hd / 2;
  constexpr int kPairRegs = kBatchMaxHeadDim / 64;
  const float rroot = 1.0f / sqrtf((float)hd);
  const int G = 32 / C;                      // lanes per slot (C is a power of two <= 16)
  const int nq = (pairs + G - 1) / G;        // dimension pairs per lane in the key dot
  const int g = lane / G, r = lane - g * G;  // this lane's slot in the chunk and its part
  const int rot = g % nq;                    // the slot's first dimension pair (bank rotation)
  int s = 0, h = 0, slot = 0, valid = 0;
  const float* qrow = table;
  float m = -INFINITY, lsum = 0.f;
  float acc[kPairRegs][2];
  for (int i = 0; i < total; ++i) {
    const int c = i % nch, k = warp + (i / nch) * kWarps;
    if (c == 0) {
      const int u = unit_of(k);
      s = u / H;
      h = u - s * H;
      const int2 mt = meta[k];
      slot = mt.x;
      valid = mt.y;
      qrow = table + (size_t)k * rowf;
      m = -INFINITY;
      lsum = 0.f;
#pragma unroll
      for (int e = 0; e < kPairRegs; ++e) acc[e][0] = acc[e][1] = 0.f;
    }
    issue(i + NB - 1);  // into the stage chunk i - 1 used (read before the warp barrier below)
    cp_async_wait_pending(NB - 1);  // chunk i's group is complete
    __syncwarp();
    const int b = i % NB;
    const T* Kc = reinterpret_cast<const T*>(stages + (size_t)(warp * NB + b) * sbytes);
    const T* Vc = reinterpret_cast<const T*>(stages + (size_t)(warp * NB + b) * sbytes + half);
    const int c0 = c * C, n = min(min(C, W - c0), valid - c0);  // retained slots of this chunk
    if (n > 0) {
      const bool ok = g < n;
      float dot = 0.f;
      if (ok) {
        const bool own = c0 + g == slot;
        const T* krow = Kc + (size_t)g * hd;
        const float* kown = qrow + hd;
        for (int e = 0; e < nq; ++e) {
          int qq = e + rot;
          qq -= (qq >= nq) ? nq : 0;
          const int p = r + G * qq;
          if (p < pairs) {
            const float2 kv = own ? *reinterpret_cast<const float2*>(kown + 2 * p) : load2_shared<T>(krow + 2 * p);
            const float2 qv = *reinterpret_cast<const float2*>(qrow + 2 * p);
            dot = fmaf(qv.x, kv.x, dot);
            dot = fmaf(qv.y, kv.y, dot);
          }
        }
      }
      for (int o = 1; o < G; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      const float lg = ok ? dot * rroot : -INFINITY;
      float mx = lg;
      for (int o = G; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m, mx);  // finite: the chunk's first slot is retained
      const float sc = expf(m - mn);
      const float pj = ok ? expf(lg - mn) : 0.f;
      float ps = pj;
      for (int o = G; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      lsum = fmaf(lsum, sc, ps);
      const float* vown = qrow + 2 * hd;
#pragma unroll
      for (int e = 0; e < kPairRegs; ++e) {
        acc[e][0] *= sc;
        acc[e][1] *= sc;
      }
#pragma unroll 4
      for (int x = 0; x < n; ++x) {
        const float px = __shfl_sync(0xffffffffu, pj, x * G);
        const bool own = c0 + x == slot;
        const T* vrow = Vc + (size_t)x * hd;
#pragma unroll
        for (int e = 0; e < kPairRegs; ++e) {
          const int pi = lane + 32 * e;
          if (pi < pairs) {
            const float2 vv = own ? *reinterpret_cast<const float2*>(vown + 2 * pi) : load2_shared<T>(vrow + 2 * pi);
            acc[e][0] = fmaf(px, vv.x, acc[e][0]);
            acc[e][1] = fmaf(px, vv.y, acc[e][1]);
          }
        }
      }
      m = mn;
    }
    __syncwarp();  // the stage is read: the next issue may refill it
    if (c == nch - 1) {
#pragma unroll
      for (int e = 0; e < kPairRegs; ++e) {
        const int pi = lane + 32 * e;
        if (pi < pairs) {
          put_z<T, kTc>(a, s, h * hd + 2 * pi, d, Storage<T>::round(acc[e][0] / lsum));
          put_z<T, kTc>(a, s, h * hd + 2 * pi + 1, d, Storage<T>::round(acc[e][1] / lsum));
        }
      }
    }
  }
  // every chunk's group was waited for above; later groups are empty
}

// Head dimension 64 (every benchmark shape): the same per-warp walk as
// attention_phase_staged, with 16-byte shared-memory reads throughout.
//  * A row is kNch 16-byte pieces (8 for 16-bit storage, 16 for fp32). A
//    chunk (one stage, 4 KB of K and V) holds kC slots and is computed in two
//    passes of kP = 32 / kG slots; kG lanes take each slot's key dot, two
//    pieces per lane, with this lane's q pieces held in registers.
//  * 16-bit rows are stored with piece p of row j at p ^ (4 (j & 1)), so the
//    8 lanes of a quarter-warp (two slots, pieces 0-3 or 4-7) read 8 distinct
//    bank groups; fp32 quarter-warps read one row's 8 consecutive pieces.
//  * Value rows: lane (y, c) accumulates piece c of slots y, y + kY, ... into
//    kVec partial sums; the kY slot groups are summed once per unit.
//  * The q of the CTA's units (and their retained-slot counts) sit in the
//    static shared-memory union, idle in this phase, so the dynamic shared
//    memory holds only the stages (kWarps x a.att_stages x 4 KB).
//  * The chunk copies start after the q/k/v inserts and a block barrier
//    (cp.async reads are ordered after it), so the staged rows include the
//    slot this step writes.
template <typename T>
struct Att64 {
  static constexpr int kVec = Storage<T>::kVec;       // elements per 16-byte piece
  static constexpr int kNch = 64 / kVec;              // pieces per row
  static constexpr int kG = sizeof(T) == 2 ? 4 : 8;   // lanes per slot in the key dot
  static constexpr int kP = 32 / kG;                  // slots per pass
  static constexpr int kC = 2 * kP;                   // slots per chunk (stage)
  static constexpr int kY = 32 / kNch;                // slot groups in the value sums
  static constexpr unsigned kRowBytes = 64u * sizeof(T);
  __device__ static int swz(int row) { return sizeof(T) == 2 ? ((row & 1) << 2) : 0; }
};

// Bytes of the head-dim-64 phase's q table for `units` units (q in fp32, then
// each unit's retained-slot count); it must fit the static union.
__host__ __device__ inline unsigned att64_table_bytes(int units) {
  return (unsigned)units * (64u * 4u + 4u);
}

template <typename T, bool kTc>
__device__ void attention_phase_hd64(const StepArgs& a, BatchSmem& sm, unsigned char* dyn, int l,
                                     unsigned long long event) {
  using A = Att64<T>;
  constexpr int E = A::kVec, NCH = A::kNch, G = A::kG, P = A::kP, C = A::kC, Y = A::kY;
  const int W = a.window, H = a.heads, S = a.streams, d = a.width, M = 3 * d;
  const int NB = a.att_stages, nch = (W + C - 1) / C;
  int lo, hi;
  split(S * H, (int)blockIdx.x, (int)gridDim.x, lo, hi);
  const int mine = hi - lo;
  if (mine <= 0) return;
  if (att64_table_bytes(mine) > sizeof(sm.u) || a.att_chunk != C || a.att_buf_bytes != 4096u) {  // host-sized
    if (threadIdx.x == 0) set_error(a, kClusterShape);
    return;
  }
  const int warp = (int)threadIdx.x >> 5, lane = (int)threadIdx.x & 31;
  float* qtab = reinterpret_cast<float*>(&sm.u);                  // [mine][64]
  int* vtab = reinterpret_cast<int*>(qtab + (size_t)mine * 64);  // [mine] retained slots
  unsigned char* stages = dyn + (size_t)warp * NB * 4096u;        // this warp's stages
  constexpr unsigned kHalf = (unsigned)C * A::kRowBytes;          // K, then V
  const int nu = mine > warp ? (mine - 1 - warp) / kWarps + 1 : 0;
  const int total = nu * nch;
  const size_t head_stride = (size_t)W * 64;  // elements per (stream, layer, head) ring
  auto ring_base = [&](int k) {               // element offset of owned unit k's ring in layer l
    const int u = lo + k, su = u / H, hu = u - su * H;
    return (((size_t)su * a.layers + l) * H + hu) * head_stride;
  };
  // issue state: the next chunk to copy (unit k_i of this warp's list, chunk c_i, stage s_i)
  int ik = warp, ic = 0, is = 0, issued = 0;
  const T* ikeys = (const T*)a.keys + (nu > 0 ? ring_base(warp) : 0);
  const T* ivals = (const T*)a.values + (ikeys - (const T*)a.keys);
  auto issue = [&]() {  // every lane: its pieces of the next chunk into its stage, one group
    if (issued < total) {
      unsigned char* dst = stages + (unsigned)is * 4096u;
      const int c0 = ic * C, n = min(C, W - c0);
      const unsigned char* ks = reinterpret_cast<const unsigned char*>(ikeys + (size_t)c0 * 64);
      const unsigned char* vs = reinterpret_cast<const unsigned char*>(ivals + (size_t)c0 * 64);
#pragma unroll 4
      for (int q = lane; q < n * NCH; q += 32) {
        const int row = q / NCH, pc = q - row * NCH;
        const unsigned so = (unsigned)row * A::kRowBytes + (unsigned)pc * 16u;
        const unsigned dp = (unsigned)row * A::kRowBytes + (unsigned)(pc ^ A::swz(row)) * 16u;
        cp_async16(dst + dp, ks + so);
        cp_async16(dst + kHalf + dp, vs + so);
      }
      ++issued;
      is = is + 1 == NB ? 0 : is + 1;
      if (++ic == nch) {
        ic = 0;
        ik += kWarps;
        if (ik < mine) {
          ikeys = (const T*)a.keys + ring_base(ik);
          ivals = (const T*)a.values + (ikeys - (const T*)a.keys);
        }
      }
    }
    cp_async_commit();  // empty past the last chunk: the group count stays uniform
  };
  // every owned unit's final q, k, v (the K/V insert into the ring, q into the table)
  constexpr int per_unit = 3 * 64 / 2;
  for (int x = threadIdx.x; x < mine * per_unit; x += kThreads) {
    const int k = x / per_unit, p = x - k * per_unit;
    const int u = lo + k, su = u / H, hu = u - su * H;
    const unsigned long long t = __ldcg(a.position + su) + event;
    const int row = 2 * p, which = row >> 6, dim = row & 63;
    const float* Pp = a.bpart + (size_t)su * M + (size_t)hu * 192 + row;
    float v0 = Storage<T>::round(sum_splits(Pp, a.bsplit[0], (size_t)S * M));
    float v1 = Storage<T>::round(sum_splits(Pp + 1, a.bsplit[0], (size_t)S * M));
    if (which < 2) {
      const float angle = (float)t * a.rope_freq[dim >> 1];
      const float co = cosf(angle), sn = sinf(angle);
      const float r0 = v0 * co - v1 * sn;
      const float r1 = v0 * sn + v1 * co;
      v0 = Storage<T>::round(r0);
      v1 = Storage<T>::round(r1);
    }
    if (which == 0) {
      qtab[(size_t)k * 64 + dim] = v0;
      qtab[(size_t)k * 64 + dim + 1] = v1;
      if (dim == 0) vtab[k] = valid_length(t, W);
    } else {
      const int slot = (int)(t % (unsigned long long)W);
      T* ring = (T*)(which == 1 ? a.keys : a.values) + ring_base(k);
      Storage<T>::store(ring, (size_t)slot * 64 + dim, v0);
      Storage<T>::store(ring, (size_t)slot * 64 + dim + 1, v1);
    }
  }
  __syncthreads();  // the inserts are in the ring before any chunk is copied
  btl(a, sm, kBtlAttPrepare);
  for (int i = 0; i < NB - 1; ++i) issue();
  const float rroot = 0.125f;                 // 1 / sqrt(64)
  const int g = lane / G, r = lane - g * G;   // key dot: slot g of a pass, pieces r and r + G
  const int vy = lane / NCH, vc = lane - vy * NCH;  // value sums: slot group vy, piece vc
  int k = warp, c = 0, cs = 0, s = 0, h = 0, valid = 0;
  float qv[2][E];
  float m = -INFINITY, lsum = 0.f;
  float acc[E];
  for (int i = 0; i < total; ++i) {
    if (c == 0) {
      const int u = lo + k;
      s = u / H;
      h = u - s * H;
      valid = vtab[k];
      const float* qrow = qtab + (size_t)k * 64;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < E; e += 4) {
          const float4 f = *reinterpret_cast<const float4*>(qrow + (r + G * j) * E + e);
          qv[j][e] = f.x;
          qv[j][e + 1] = f.y;
          qv[j][e + 2] = f.z;
          qv[j][e + 3] = f.w;
        }
      m = -INFINITY;
      lsum = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] = 0.f;
    }
    issue();                        // into the stage chunk i - 1 used (read before the warp barrier below)
    cp_async_wait_pending(NB - 1);  // chunk i's group is complete
    __syncwarp();
    const unsigned char* Kc = stages + (unsigned)cs * 4096u;
    const unsigned char* Vc = Kc + kHalf;
    const int c0 = c * C, n = min(min(C, W - c0), valid - c0);  // retained slots of this chunk
#pragma unroll
    for (int po = 0; po < C; po += P) {
      const int np = n - po;  // retained slots from this pass on (warp-uniform)
      if (np > 0) {
        const bool ok = g < np;
        float dot = 0.f;
        if (ok) {
          const int row = po + g;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int pc = r + G * j;
            float kf[E];
            const uint4 w = *reinterpret_cast<const uint4*>(Kc + (unsigned)row * A::kRowBytes +
                                                            (unsigned)(pc ^ A::swz(row)) * 16u);
            Storage<T>::unpack(w, kf);
#pragma unroll
            for (int e = 0; e < E; ++e) dot = fmaf(qv[j][e], kf[e], dot);
          }
        }
#pragma unroll
        for (int o = 1; o < G; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float lg = ok ? dot * rroot : -INFINITY;
        float mx = lg;
#pragma unroll
        for (int o = G; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mn = fmaxf(m, mx);  // finite: the pass's first slot is retained
        const float sc = expf(m - mn);
        const float pj = ok ? expf(lg - mn) : 0.f;
        float ps = pj;
#pragma unroll
        for (int o = G; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        lsum = fmaf(lsum, sc, ps);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] *= sc;
#pragma unroll
        for (int x0 = 0; x0 < P; x0 += Y) {
          const int x = x0 + vy;
          const float px = __shfl_sync(0xffffffffu, pj, x * G);  // 0 past the retained slots
          if (x < np) {
            const int row = po + x;
            float vf[E];
            const uint4 w = *reinterpret_cast<const uint4*>(Vc + (unsigned)row * A::kRowBytes +
                                                            (unsigned)(vc ^ A::swz(row)) * 16u);
            Storage<T>::unpack(w, vf);
#pragma unroll
            for (int e = 0; e < E; ++e) acc[e] = fmaf(px, vf[e], acc[e]);
          }
        }
        m = mn;
      }
    }
    __syncwarp();  // the stage is read: the next issue may refill it
    cs = cs + 1 == NB ? 0 : cs + 1;
    if (++c == nch) {
      // the unit's value sums over the slot groups, in a fixed order
#pragma unroll
      for (int o = NCH; o < 32; o <<= 1)
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
      if (vy == 0) {
#pragma unroll
        for (int e = 0; e < E; ++e) put_z<T, kTc>(a, s, h * 64 + vc * E + e, d, Storage<T>::round(acc[e] / lsum));
      }
      c = 0;
      k += kWarps;
    }
  }
  // every chunk's group was waited for above; later groups are empty
}

// ---------------------------------------------------------------- tensor-core GEMM phase
// Per-thread pipeline counters of the roles below; they persist across the
// GEMM phases, layers and rounds of one launch (every role thread walks the
// same unit sequence).
struct TcRoles {
  unsigned long long issued = 0;    // producer: chunks issued
  unsigned long long consumed = 0;  // MMA issuer: chunks consumed
  unsigned long long units = 0;     // every thread: units walked
  bool failed = false;
};

// P[ks][s][m] = sum over split ks's K chunks of W[m][k] z[s][k] on the tensor
// cores. A unit is (128-row tile, K split, group of nu <= 256 streams): the
// producer thread copies each 64-column chunk's A tile (16 KB of pre-tiled
// weights) and B tile (the streams' inputs, N x 128 bytes) into a stage with
// one mbarrier completion; the issuer thread runs four 128 x N x 16 MMAs per
// chunk into the unit's tensor-memory accumulator and frees the stage with a
// commit; warps 0-3 read the accumulator (32 rows each) and store the
// partials. Every wait is bounded; a timeout sets the error word. fp32: a
// chunk is 32 columns, its stage holds the hi and lo tiles of A and B, and
// the issuer runs Ahi Bhi, Ahi Blo and Alo Bhi (three 128 x N x 8 tf32 MMAs)
// per 8 columns: Ahi Bhi into the unit's accumulator, the two corrections into
// a second one (columns kTcMaxN on), summed once in the epilogue. (Adding the
// small correction products into the large accumulator, MMA after MMA, lost
// more than fp32 accuracy: measured on B200 as a 1.2e-5 error against the
// oracle where the CUDA-core fp32 round stays within the policy.)
template <typename T>
__device__ void tc_gemm_phase(const StepArgs& a, BatchSmem& sm, unsigned char* stages, TcRoles& tr, const T* Wt,
                              int M, int K, int ksplit, int nu, float* P, const void* Bsrc, bool swiglu) {
  constexpr bool kX3 = std::is_same<T, float>::value;  // fp32 as three tf32 products
  constexpr int kK = kX3 ? kTileK32 : kTileK;           // K elements per 128-byte chunk row
  const int S = a.streams, spad = a.spad;
  const int mtiles = (M + kUmmaM - 1) / kUmmaM, kchunks = K / kK;
  const int sgroups = (spad + nu - 1) / nu;  // nu: streams per unit (MMA N), a multiple of 16
  const int units = mtiles * ksplit * sgroups;
  const int warp = (int)threadIdx.x >> 5, lane = (int)threadIdx.x & 31;
  const T* Bt = (const T*)Bsrc;
  // tf32 lo planes: weights after the padded hi matrix, inputs after the hi plane
  const size_t wlo = (size_t)mtiles * kUmmaM * K, blo = (size_t)spad * K;
  const unsigned long long tmo = a.bar_timeout_ns;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int mt = u % mtiles, rest = u / mtiles, ks = rest % ksplit, sg = rest / ksplit;
    int c0, c1;
    split(kchunks, ks, ksplit, c0, c1);
    const int s0 = sg * nu, n = min(nu, spad - s0);
    if (threadIdx.x == kTcProducer) {
      const unsigned long long wpol = policy_evict_first(), zpol = policy_evict_last();
      for (int kc = c0; kc < c1 && !tr.failed; ++kc) {
        const int st = (int)(tr.issued % (unsigned long long)a.tc_stages);
        const unsigned long long r = tr.issued / (unsigned long long)a.tc_stages;
        if (r > 0 && !mbar_wait_bounded(&sm.tc_empty[st], (unsigned)((r - 1) & 1ull), tmo)) {
          tr.failed = true;
          set_error(a, kBarrierTimeout);
          break;
        }
        unsigned char* sa = stages + (size_t)st * a.tc_stage_bytes;
        const T* wsrc = Wt + ((size_t)mt * kchunks + kc) * (kUmmaM * kK);
        const T* bsrc = Bt + ((size_t)kc * spad + s0) * kK;
        const unsigned bbytes = (unsigned)n * kCoreBytes;
        if constexpr (kX3) {  // stage: A hi, A lo, B hi, B lo
          mbar_expect_tx(&sm.tc_full[st], 2 * kTcTileBytes + 2 * bbytes);
          bulk_copy(sa, wsrc, kTcTileBytes, &sm.tc_full[st], wpol);
          bulk_copy(sa + kTcTileBytes, wsrc + wlo, kTcTileBytes, &sm.tc_full[st], wpol);
          bulk_copy(sa + 2 * kTcTileBytes, bsrc, bbytes, &sm.tc_full[st], zpol);
          bulk_copy(sa + 2 * kTcTileBytes + bbytes, bsrc + blo, bbytes, &sm.tc_full[st], zpol);
        } else {
          mbar_expect_tx(&sm.tc_full[st], kTcTileBytes + bbytes);
          bulk_copy(sa, wsrc, kTcTileBytes, &sm.tc_full[st], wpol);
          bulk_copy(sa + kTcTileBytes, bsrc, bbytes, &sm.tc_full[st], zpol);
        }
        tr.issued += 1;
      }
    } else if (threadIdx.x == kTcIssuer) {
      if (!tr.failed && tr.units > 0 && !mbar_wait_bounded(&sm.tc_tempty, (unsigned)((tr.units - 1) & 1ull), tmo)) {
        tr.failed = true;
        set_error(a, kBarrierTimeout);
      }
      tc_fence_after();
      const unsigned idesc = umma_idesc<T>(kUmmaM, n);
      for (int kc = c0; kc < c1 && !tr.failed; ++kc) {
        const int st = (int)(tr.consumed % (unsigned long long)a.tc_stages);
        const unsigned long long r = tr.consumed / (unsigned long long)a.tc_stages;
        if (!mbar_wait_bounded(&sm.tc_full[st], (unsigned)(r & 1ull), tmo)) {
          tr.failed = true;
          set_error(a, kBarrierTimeout);
          break;
        }
        tc_fence_after();
        const unsigned char* sa = stages + (size_t)st * a.tc_stage_bytes;
        if constexpr (kX3) {
          const unsigned bbytes = (unsigned)n * kCoreBytes;
          const unsigned char* ahi = sa;
          const unsigned char* alo = sa + kTcTileBytes;
          const unsigned char* bhi = sa + 2 * kTcTileBytes;
          const unsigned char* blo_s = bhi + bbytes;
          const unsigned corr = sm.tc_tmem + (unsigned)kTcMaxN;  // the correction accumulator's columns
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const unsigned o = kk * 2 * kCoreBytes;
            const unsigned acc = (kc > c0 || kk > 0) ? 1u : 0u;
            umma_tf32(sm.tc_tmem, umma_desc(ahi + o), umma_desc(bhi + o), idesc, acc);
            umma_tf32(corr, umma_desc(ahi + o), umma_desc(blo_s + o), idesc, acc);
            umma_tf32(corr, umma_desc(alo + o), umma_desc(bhi + o), idesc, 1u);
          }
        } else {
#pragma unroll
          for (int kk = 0; kk < kTileK / kUmmaK; ++kk)
            umma_f16(sm.tc_tmem, umma_desc(sa + kk * 2 * kCoreBytes), umma_desc(sa + kTcTileBytes + kk * 2 * kCoreBytes),
                     idesc, (kc > c0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&sm.tc_empty[st]);
        tr.consumed += 1;
      }
      umma_commit(&sm.tc_tfull);
    } else if (warp < 4) {
      bool ok = !tr.failed && mbar_wait_bounded(&sm.tc_tfull, (unsigned)(tr.units & 1ull), tmo);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const int m = mt * kUmmaM + warp * 32 + lane;
        float* out = P + ((size_t)ks * S + s0) * M;
        const int live = min(n, S - s0);
        for (int c = 0; c < n; c += 16) {
          float v[16];
          tmem_ld16(sm.tc_tmem + ((unsigned)(warp * 32) << 16) + (unsigned)c, v);
          if constexpr (kX3) {  // main + corrections, added once in fp32
            float w[16];
            tmem_ld16(sm.tc_tmem + ((unsigned)(warp * 32) << 16) + (unsigned)(kTcMaxN + c), w);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += w[j];
          }
          if (!kX3 && swiglu) {  // 16-bit only (fp32 keeps its K-split and the SwiGLU phase)
            // rows 2i (gate) and 2i + 1 (up) are lanes 2i, 2i + 1 of this warp:
            // act[s][i] = cast(silu(cast(g)) cast(u)) (reference src/cpu/Cpu.cpp:121-127);
            // the even lane takes columns 0-7 of the 16, the odd lane 8-15
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = __shfl_xor_sync(0xffffffffu, v[j], 1);
            const bool odd = (lane & 1) != 0;
            if (m < M) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int jj = odd ? j + 8 : j;
                const float gv = odd ? o[jj] : v[jj], uv = odd ? v[jj] : o[jj];
                if (c + jj < live) {
                  const float g = Storage<T>::round(gv), u = Storage<T>::round(uv);
                  put_z_at<T, true>(a, a.bz16_act, s0 + c + jj, m >> 1, M >> 1,
                                    Storage<T>::round((g / (1.0f + expf(-g))) * u));
                }
              }
            }
          } else if (m < M) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (c + j < live) out[(size_t)(c + j) * M + m] = v[j];
          }
        }
        tc_fence_before();
      } else if (lane == 0 && !tr.failed) {
        set_error(a, kBarrierTimeout);
      }
      if (!ok) tr.failed = true;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.tc_tempty);
    }
    tr.units += 1;
  }
}

// Kernel start (kTc): mbarriers, tensor-memory allocation (warp 0).
__device__ inline void tc_setup(const StepArgs& a, BatchSmem& sm) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.tc_stages; ++i) {
      mbar_init(&sm.tc_full[i], 1);
      mbar_init(&sm.tc_empty[i], 1);
    }
    mbar_init(&sm.tc_tfull, 1);
    mbar_init(&sm.tc_tempty, 4);
    mbar_init(&sm.tc_done, 1);
    fence_mbar_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(&sm.tc_tmem, a.tc_ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// Kernel end (kTc), reached on every path: every MMA issued has completed,
// every bulk copy issued has landed, then warp 0 frees the tensor memory.
__device__ inline void tc_teardown(const StepArgs& a, BatchSmem& sm, const TcRoles& tr) {
  __syncthreads();
  if (threadIdx.x == kTcIssuer) {
    umma_commit(&sm.tc_done);
    if (!mbar_wait_bounded(&sm.tc_done, 0u, a.bar_timeout_ns)) set_error(a, kBarrierTimeout);
  }
  if (threadIdx.x == kTcProducer) {
    const unsigned long long n = tr.issued, stages = (unsigned long long)a.tc_stages;
    for (unsigned long long c = n > stages ? n - stages : 0; c < n; ++c)
      if (!mbar_wait_bounded(&sm.tc_full[c % stages], (unsigned)((c / stages) & 1ull), a.bar_timeout_ns)) {
        set_error(a, kBarrierTimeout);
        break;
      }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(sm.tc_tmem, a.tc_ncols);
}

// One GEMM phase on the CUDA cores or the tensor cores.
template <typename T, bool kTc, int kView>
__device__ __forceinline__ void gemm_any(const StepArgs& a, BatchSmem& sm, unsigned char* stages, TcRoles& tr,
                                         const void* W, const void* Wt, int M, int K, int ksplit, int nu,
                                         const void* Bsrc = nullptr, bool swiglu = false) {
  if constexpr (kTc)
    tc_gemm_phase<T>(a, sm, stages, tr, (const T*)Wt, M, K, ksplit, nu, a.bpart, Bsrc ? Bsrc : a.bz16, swiglu);
  else gemm_phase<T, kView>(a, sm, (const T*)W, M, K, ksplit, a.bz, a.bpart);
}

// One round (event `event` of this launch) for every stream. `input` is
// [S][features]; scores go to a.score and, when given, score_out[S].
template <typename T, bool kTc>
__device__ bool round_batched(const StepArgs& a, BatchSmem& sm, unsigned char* stages, TcRoles& tr, GridSync& gs,
                              const float* input, unsigned long long event, float* score_out) {
  const int S = a.streams, d = a.width, F = a.ffn, L = a.layers;
  auto sync = [&](int tag) {
    btl(a, sm, tag);
    const bool ok = gs.sync(a, a.bar_timeout_ns);
    btl(a, sm, kBtlSync);
    return ok;
  };
  for (int s = blockIdx.x; s < S; s += gridDim.x) row_input<T, kTc>(a, sm, s, input);
  if (!sync(kBtlInput)) return false;
  for (int l = 0; l < L; ++l) {
    const LayerPtrs& w = a.layer[l];
    gemm_any<T, kTc, kViewRows>(a, sm, stages, tr, w.qkv, a.tqkv[l], 3 * d, d, a.bsplit[0], a.tc_n[0]);
    if (!sync(kBtlQkv)) return false;
    if (a.att_hd64) attention_phase_hd64<T, kTc>(a, sm, stages, l, event);
    else if (a.att_buf_bytes) attention_phase_staged<T, kTc>(a, sm, stages, l, event);
    else attention_phase<T, kTc>(a, sm, l, event);
    if (!sync(kBtlAttention)) return false;
    gemm_any<T, kTc, kViewOutHeads>(a, sm, stages, tr, w.out, a.tout[l], d, d, a.bsplit[1], a.tc_n[1]);
    if (!sync(kBtlOut)) return false;
    for (int s = blockIdx.x; s < S; s += gridDim.x)
      row_residual<T, kTc>(a, sm, s, a.bx, a.bx2, a.bpart, a.bsplit[1], nullptr, (const T*)w.norm2, false, nullptr);
    if (!sync(kBtlResidual2)) return false;
    // SwiGLU in the 16-bit gate/up epilogue (no K-split there)
    const bool fused = kTc && !std::is_same<T, float>::value && a.fuse_swiglu;
    gemm_any<T, kTc, kViewRows>(a, sm, stages, tr, w.gateup, a.tgateup[l], 2 * F, d, a.bsplit[2], a.tc_n[2],
                                nullptr, fused);
    if (!sync(kBtlGateUp)) return false;
    if (!fused) {
      swiglu_phase<T, kTc>(a, a.bsplit[2]);
      if (!sync(kBtlSwiglu)) return false;
    }
    gemm_any<T, kTc, kViewColumns>(a, sm, stages, tr, w.down, a.tdown[l], d, F, a.bsplit[3], a.tc_n[3],
                                   fused ? a.bz16_act : nullptr);
    if (!sync(kBtlDown)) return false;
    const bool last = l + 1 == L;
    for (int s = blockIdx.x; s < S; s += gridDim.x)
      row_residual<T, kTc>(a, sm, s, a.bx2, a.bx, a.bpart, a.bsplit[3], a.hidden + ((size_t)s * L + l) * d,
                           last ? nullptr : (const T*)a.layer[l + 1].norm1, last, score_out ? score_out + s : nullptr);
    if (last) btl(a, sm, kBtlResidual1);
    else if (!sync(kBtlResidual1)) return false;
  }
  return true;
}

// `count` rounds over inputs [count][S][features] (scores [count][S] when
// given); positions advance by `count` at the end, each stream's by the CTA
// that ran its last R1. kTc: the GEMM phases run on the tensor cores, with
// the pipeline stages in dynamic shared memory.
template <typename T, bool kTc>
__device__ void batched_rounds(const StepArgs& a, const float* inputs, unsigned long long count, float* scores,
                               unsigned long long base) {
  __shared__ BatchSmem sm;
  extern __shared__ __align__(1024) unsigned char tc_stage_smem[];
  if (threadIdx.x == 0) sm.tl_n = 0;
  __syncthreads();
  TcRoles tr;
  if constexpr (kTc) tc_setup(a, sm);
  GridSync gs{base, 0};
  const size_t stride = (size_t)a.streams * a.features;
  bool ok = true;
  for (unsigned long long e = 0; e < count && ok; ++e)
    ok = round_batched<T, kTc>(a, sm, tc_stage_smem, tr, gs, inputs + e * stride, e,
                               scores ? scores + e * a.streams : nullptr);
  if (ok && threadIdx.x == 0)
    for (int s = blockIdx.x; s < a.streams; s += gridDim.x) a.position[s] = __ldcg(a.position + s) + count;
  if constexpr (kTc) tc_teardown(a, sm, tr);
}

}  // namespace st
