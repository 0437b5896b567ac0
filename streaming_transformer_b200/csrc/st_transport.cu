// st_transport.cu -- transport and synchronization calibration.
//
// Restates the reference's transport micro-benchmark (reference
// src/cuda/Runtime.cu:667-814, docs/transport.md:20-24) with its modes
//   empty         empty kernel launch + stream synchronize
//   empty-graph   one-node graph launch + stream synchronize
//   copy          128 B pinned H2D, echo kernel, 128 B D2H, synchronize; payload checked
//   ping-pong     host-initiated mapped-mailbox round trip to a resident 1-thread kernel
//   gpu-ping      GPU-initiated round trip: the GPU publishes, the host acknowledges
// and adds one mode of its own:
//   grid-barrier  device time of one grid-wide barrier of the step kernels
//                 (one 512-thread CTA per SM, cooperative launch), CUDA events
//   ll-exchange   device time of one all-to-all exchange of a 512-float vector
//                 in tagged 8-byte records (value | epoch), each CTA writing its
//                 slice and polling every record until its tag matches
//   cluster-barrier  device time of one hardware cluster barrier, clusters of 8
//   bulk-stream / load-stream  every CTA (one per SM) streams its own 1 MiB of
//                 HBM `count` times, either through a 4 x 32 KiB shared-memory
//                 ring fed by cp.async.bulk (thread 0 issuing, all threads
//                 waiting on the slot mbarriers) or with 16-byte vector loads;
//                 reports GB/s and thread 0's cycles inside the issue
//   icache        cycles per pass over 8-64 KB of straight-line code (512
//                 threads per SM), and cycles per call over 8-128 distinct
//                 ~1 KB out-of-line functions: instruction fetch cost and the
//                 instruction cache capacity the step's per-layer code must fit
//   primitives    SM cycles per call of the step's building blocks, every CTA
//                 (one per SM) calling each one `count` times back to back:
//                 __syncthreads, block_sum, gemv_tile on 16 x 512 and 64 x 64
//                 fp32 tiles read from shared or global memory, and the step's
//                 warp-per-row GEMV (warp_rows) on the same shared tiles
// Every device wait is bounded (30 s budget, globaltimer) and every host wait
// gives up after 60 s.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../../include/streaming_b200.h"
#include "st_device.cuh"
#include "st_ring.cuh"
#include "st_step.cuh"

using namespace st;

namespace {

thread_local std::string g_transport_error;

struct alignas(64) PingBox {
  alignas(64) unsigned long long request;
  alignas(64) unsigned long long completion;
  alignas(64) unsigned long long exited;
  alignas(64) unsigned long long checksum;
};

__global__ void k_empty() {}

__global__ void k_echo(const float* in, float* out, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = in[i];
}

// Resident single-thread partner of the ping-pong / gpu-ping modes.
__global__ void k_ping(PingBox* box, const float* input, unsigned long long count, int backoff,
                       unsigned long long budget_ns, int gpu_initiated, unsigned long long* cycles, int* errors) {
  if (threadIdx.x || blockIdx.x) return;
  for (unsigned long long seq = 1; seq <= count; ++seq) {
    const long long c0 = clock64();
    const unsigned long long t0 = globaltimer();
    if (gpu_initiated) {
      *reinterpret_cast<volatile unsigned long long*>(&box->checksum) = seq * 2654435761ull;
      st_release_sys(&box->request, seq);
      while (ld_acquire_sys(&box->completion) != seq) {
        if (globaltimer() - t0 > budget_ns) { st_release_sys(&box->exited, 1ull); return; }
        if (backoff) __nanosleep(128);
      }
      if (*reinterpret_cast<volatile unsigned long long*>(&box->checksum) != ((seq * 2654435761ull) ^ 0xabcdefull))
        atomicAdd(errors, 1);
    } else {
      while (ld_acquire_sys(&box->request) != seq) {
        if (globaltimer() - t0 > budget_ns) { st_release_sys(&box->exited, 1ull); return; }
        if (backoff) __nanosleep(128);
      }
      unsigned long long sum = 0;
      for (int i = 0; i < 32; ++i) sum += __float_as_uint(__ldcv(input + i));
      *reinterpret_cast<volatile unsigned long long*>(&box->checksum) = sum;
      __threadfence_system();
      st_release_sys(&box->completion, seq);
    }
    cycles[seq - 1] = (unsigned long long)(clock64() - c0);
  }
  st_release_sys(&box->exited, 1ull);
}

__device__ __forceinline__ void st_release_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

// All-to-all exchange of n floats per round: CTA b owns records [b*n/G, (b+1)*n/G).
// Two record buffers alternate by epoch parity, so no CTA can overwrite a record
// another CTA has not read yet (writing round r+2 needs every CTA's round r+1
// slice, written only after that CTA read all of round r).
__global__ void __launch_bounds__(kThreads, 1) k_ll_exchange(unsigned long long* buffers, int n, unsigned long long rounds,
                                                             unsigned int epoch0, int* error) {
  const int lo = (int)((long long)n * blockIdx.x / gridDim.x), hi = (int)((long long)n * (blockIdx.x + 1) / gridDim.x);
  float carry = 0.f;
  for (unsigned long long r = 0; r < rounds; ++r) {
    const unsigned int tag = epoch0 + (unsigned int)r;
    unsigned long long* records = buffers + (size_t)(tag & 1u) * n;
    for (int i = lo + threadIdx.x; i < hi; i += kThreads) {
      const float v = carry + (float)i;
      st_release_gpu_u64(records + i, ((unsigned long long)tag << 32) | __float_as_uint(v));
    }
    float acc = 0.f;
    for (int i = threadIdx.x; i < n; i += kThreads) {
      unsigned long long rec;
      const unsigned long long t0 = globaltimer();
      while ((unsigned int)((rec = ld_acquire_gpu(records + i)) >> 32) != tag) {
        if (globaltimer() - t0 > 2000000000ull) { atomicExch(error, 1); return; }
      }
      acc += __uint_as_float((unsigned int)rec);
    }
    carry = acc * 0.f;  // keep the reads live without changing the values
    // Every thread of this CTA must finish reading round r before any of them
    // publishes round r+1 (that is what keeps round r+2 off an unread buffer).
    __syncthreads();
  }
}

__global__ void __cluster_dims__(8, 1, 1) __launch_bounds__(kThreads, 1) k_cluster_barriers(unsigned long long rounds) {
  for (unsigned long long r = 0; r < rounds; ++r) {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
}

// Streams `bytes_per_cta` from src + blockIdx.x * bytes_per_cta, `rounds` times,
// through kStreamSlots fixed slots of kStreamSlotBytes.
constexpr int kStreamSlots = 4;
constexpr int kStreamSlotBytes = 32 * 1024;
struct alignas(128) StreamRing {
  unsigned char slot[kStreamSlots][kStreamSlotBytes];
  unsigned long long full[kStreamSlots];
};

__global__ void __launch_bounds__(kThreads, 1) k_bulk_stream(const char* src, size_t bytes_per_cta, int rounds,
                                                             unsigned long long* issue_cycles, float* sink) {
  extern __shared__ __align__(128) unsigned char raw[];
  StreamRing& rs = *reinterpret_cast<StreamRing*>(raw);
  const char* base = src + (size_t)blockIdx.x * bytes_per_cta;
  const unsigned long long total = (unsigned long long)rounds * (bytes_per_cta / kStreamSlotBytes);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStreamSlots; ++i) mbar_init(&rs.full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  unsigned long long issued = 0, spent = 0;
  const size_t chunks = bytes_per_cta / kStreamSlotBytes;
  const unsigned long long policy = policy_evict_first();
  auto issue = [&]() {
    const int slot = (int)(issued % kStreamSlots);
    const long long c0 = clock64();
    mbar_expect_tx(&rs.full[slot], kStreamSlotBytes);
    bulk_copy(rs.slot[slot], base + (issued % chunks) * kStreamSlotBytes, kStreamSlotBytes, &rs.full[slot], policy);
    spent += (unsigned long long)(clock64() - c0);
    ++issued;
  };
  if (threadIdx.x == 0)
    while (issued < total && issued < kStreamSlots) issue();
  float acc = 0.f;
  for (unsigned long long c = 0; c < total; ++c) {
    const int slot = (int)(c % kStreamSlots);
    const unsigned parity = (unsigned)((c / kStreamSlots) & 1ull);
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(&rs.full[slot], parity))
      if (globaltimer() - t0 > 2000000000ull) break;
    const float4* p = reinterpret_cast<const float4*>(rs.slot[slot]);
    for (int i = threadIdx.x; i < kStreamSlotBytes / 16; i += kThreads) {
      const float4 v = p[i];
      acc += v.x + v.y + v.z + v.w;
    }
    __syncthreads();
    if (threadIdx.x == 0 && issued < total) issue();
  }
  if (threadIdx.x == 0) issue_cycles[blockIdx.x] = spent / (issued ? issued : 1);
  if (acc == 12345.f) sink[blockIdx.x] = acc;
}

__global__ void __launch_bounds__(kThreads, 1) k_load_stream(const char* src, size_t bytes_per_cta, int rounds, float* sink) {
  const uint4* base = reinterpret_cast<const uint4*>(src + (size_t)blockIdx.x * bytes_per_cta);
  const size_t n = bytes_per_cta / 16;
  float acc = 0.f;
  for (int r = 0; r < rounds; ++r) {
    for (size_t i = threadIdx.x; i < n; i += (size_t)kThreads * 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const size_t j = i + (size_t)u * kThreads;
        v[u] = j < n ? ld_stream(base + j) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) acc += __uint_as_float(v[u].x);
    }
  }
  if (acc == 12345.f) sink[blockIdx.x] = acc;
}

// Straight-line code of N independent-chain FMAs per warp (asm, so none is
// folded), looped `reps` times: cycles per pass against the code size show
// the instruction cache capacity the step kernels must fit in.
template <int N>
__device__ __forceinline__ void fma_block(float& a, float& b, float& c, float& d) {
#pragma unroll
  for (int i = 0; i < N; i += 4) {
    asm volatile("fma.rn.f32 %0, %0, 0f3F800054, 0f3F000000;" : "+f"(a));
    asm volatile("fma.rn.f32 %0, %0, 0f3F800054, 0f3F000000;" : "+f"(b));
    asm volatile("fma.rn.f32 %0, %0, 0f3F800054, 0f3F000000;" : "+f"(c));
    asm volatile("fma.rn.f32 %0, %0, 0f3F800054, 0f3F000000;" : "+f"(d));
  }
}

template <int N>
__global__ void __launch_bounds__(kThreads, 1) k_icache(int reps, unsigned long long* out, float* sink) {
  float a = threadIdx.x, b = a + 1.f, c = a + 2.f, d = a + 3.f;
  __syncthreads();
  const long long c0 = clock64();
  for (int r = 0; r < reps; ++r) fma_block<N>(a, b, c, d);
  __syncthreads();
  const long long c1 = clock64();
  if (threadIdx.x == 0) out[blockIdx.x] = (unsigned long long)((c1 - c0) / reps);
  if (a + b + c + d == 12345.f) sink[threadIdx.x] = a;
}

// Capacity probe: a pass calls N distinct out-of-line functions of ~64
// instructions each (non-sequential code, so prefetching cannot hide misses);
// the cycles per call against N (x ~1 KB) show when the code stops fitting.
template <int K>
__device__ __noinline__ float icache_fn(float x) {
#pragma unroll
  for (int i = 0; i < 60; ++i) asm volatile("fma.rn.f32 %0, %0, 0f3F800054, 0f3F000000;" : "+f"(x));
  return x + (float)K;
}

// Calls in a scrambled order (37 K mod N), so consecutive calls land far apart.
template <int N, int... K>
__device__ __forceinline__ float icache_calls(float x, std::integer_sequence<int, K...>) {
  ((x = icache_fn<(K * 37) % N>(x)), ...);
  return x;
}

template <int N>
__global__ void __launch_bounds__(kThreads, 1) k_icache_calls(int reps, unsigned long long* out, float* sink) {
  float x = threadIdx.x;
  __syncthreads();
  const long long c0 = clock64();
  for (int r = 0; r < reps; ++r) x = icache_calls<N>(x, std::make_integer_sequence<int, N>{});
  __syncthreads();
  const long long c1 = clock64();
  if (threadIdx.x == 0) out[blockIdx.x] = (unsigned long long)((c1 - c0) / reps / N);
  if (x == 12345.f) sink[threadIdx.x] = x;
}

constexpr int kPrimitives = 10;

__global__ void __launch_bounds__(kThreads, 1) k_primitives(const float* wglobal, int reps, unsigned long long* out) {
  extern __shared__ __align__(128) unsigned char raw[];
  Smem& sm = *reinterpret_cast<Smem*>(raw);
  float* tile = reinterpret_cast<float*>(raw + ((sizeof(Smem) + 127) / 128) * 128);
  for (int i = threadIdx.x; i < 16 * 512; i += kThreads) tile[i] = wglobal[i];
  for (int i = threadIdx.x; i < kMaxCols; i += kThreads) sm.xs[i] = 0.001f * (float)i;
  __syncthreads();
  float sink = 0.f;
  for (int prim = 0; prim < kPrimitives; ++prim) {
    __syncthreads();
    const long long c0 = clock64();
    for (int r = 0; r < reps; ++r) {
      switch (prim) {
        case 0: __syncthreads(); break;
        case 1: sink += block_sum((float)threadIdx.x, sm); __syncthreads(); break;
        case 2: gemv_tile<float, true>(tile, 0, 16, 512, sm); sink += sm.rowsum[threadIdx.x & 15]; break;
        case 3: gemv_tile<float, false>(wglobal, 0, 16, 512, sm); sink += sm.rowsum[threadIdx.x & 15]; break;
        case 4: gemv_tile<float, true>(tile, 0, 64, 64, sm); sink += sm.rowsum[threadIdx.x & 63]; break;
        case 5: gemv_tile<float, false>(wglobal, 0, 64, 64, sm); sink += sm.rowsum[threadIdx.x & 63]; break;
        case 6:
          warp_rows<float, 2, true>(tile, 16, RowGeom<float>(512), sm.xs, [&](int row, const float (&v)[2], int sl) {
            if (sl == 0) { sm.rowsum[row] = v[0]; sm.rowsum[row + 1] = v[1]; }
          });
          __syncthreads();
          sink += sm.rowsum[threadIdx.x & 15];
          break;
        case 7:
          warp_rows<float, 2, true>(tile, 16, RowGeom<float>(512), sm.xs, [&](int row, const float (&v)[2], int sl) {
            if (sl == 0) sink += v[0] + v[1];
          });
          break;
        case 9:
          warp_rows<float, 2, false>(wglobal, 16, RowGeom<float>(512), sm.xs, [&](int row, const float (&v)[2], int sl) {
            if (sl == 0) { sm.rowsum[row] = v[0]; sm.rowsum[row + 1] = v[1]; }
          });
          __syncthreads();
          sink += sm.rowsum[threadIdx.x & 15];
          break;
        default:
          warp_rows<float, 1, true>(tile, 64, RowGeom<float>(64), sm.xs, [&](int row, const float (&v)[1], int sl) {
            if (sl == 0) sm.rowsum[row] = v[0];
          });
          __syncthreads();
          sink += sm.rowsum[threadIdx.x & 63];
          break;
      }
    }
    __syncthreads();
    const long long c1 = clock64();
    if (threadIdx.x == 0) out[(size_t)prim * gridDim.x + blockIdx.x] = (unsigned long long)((c1 - c0) / reps);
  }
  if (sink == 12345.f) out[0] = 0;
}

__global__ void __launch_bounds__(kThreads, 1) k_barriers(StepArgs a, unsigned long long count, unsigned long long base) {
  GridSync gs{base, 0};
  for (unsigned long long i = 0; i < count; ++i)
    if (!gs.sync(a, a.bar_timeout_ns)) return;
}

double pct(std::vector<double> v, double q) {
  if (v.empty()) return 0;
  std::sort(v.begin(), v.end());
  size_t i = (size_t)std::ceil(q * v.size());
  return v[i ? i - 1 : 0];
}

#define TB_CUDA(expr)                                                                   \
  do {                                                                                  \
    cudaError_t _e = (expr);                                                            \
    if (_e != cudaSuccess) {                                                            \
      g_transport_error = std::string(#expr) + ": " + cudaGetErrorString(_e);           \
      return ST_ERR_CUDA;                                                               \
    }                                                                                   \
  } while (0)

struct Resources {
  cudaStream_t stream = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  PingBox* box_h = nullptr;
  PingBox* box_d = nullptr;
  float* in_h = nullptr;
  float* in_d = nullptr;
  float* out_h = nullptr;
  float* dev_in = nullptr;
  float* dev_out = nullptr;
  unsigned long long* cycles = nullptr;
  int* errors = nullptr;
  unsigned long long* counter = nullptr;
  int* error_word = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  ~Resources() {
    if (stream) cudaStreamSynchronize(stream);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (stream) cudaStreamDestroy(stream);
    if (box_h) cudaFreeHost(box_h);
    if (in_h) cudaFreeHost(in_h);
    if (out_h) cudaFreeHost(out_h);
    cudaFree(dev_in);
    cudaFree(dev_out);
    cudaFree(cycles);
    cudaFree(errors);
    cudaFree(counter);
    cudaFree(error_word);
  }
};

int run_bench(int device, const std::string& mode, size_t count, int backoff, const char* csv_path, std::string* json) {
  const bool interactive = mode == "ping-pong" || mode == "gpu-ping";
  if (mode != "empty" && mode != "empty-graph" && mode != "copy" && !interactive && mode != "grid-barrier" &&
      mode != "ll-exchange" && mode != "cluster-barrier" && mode != "bulk-stream" && mode != "load-stream" &&
      mode != "primitives" && mode != "icache") {
    g_transport_error = "Unknown transport mode " + mode;
    return ST_ERR_INVALID;
  }
  if (count == 0 || count > 100000000) {
    g_transport_error = "Invalid event count";
    return ST_ERR_INVALID;
  }
  TB_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop{};
  TB_CUDA(cudaGetDeviceProperties(&prop, device));
  int watchdog = 0;
  cudaDeviceGetAttribute(&watchdog, cudaDevAttrKernelExecTimeout, device);
  if (interactive && watchdog) {
    g_transport_error = "Host-fed ping-pong refused with active watchdog";
    return ST_ERR_UNSUPPORTED;
  }
  Resources r;
  TB_CUDA(cudaStreamCreateWithFlags(&r.stream, cudaStreamNonBlocking));
  TB_CUDA(cudaEventCreate(&r.e0));
  TB_CUDA(cudaEventCreate(&r.e1));
  std::ostringstream o;
  o.precision(9);
  if (mode == "icache") {
    const int grid = prop.multiProcessorCount;
    unsigned long long* out = nullptr;
    float* sink = nullptr;
    TB_CUDA(cudaMalloc(&out, grid * sizeof(unsigned long long)));
    TB_CUDA(cudaMalloc(&sink, kThreads * sizeof(float)));
    const int reps = (int)std::min<size_t>(std::max<size_t>(count, 1), 10000);
    o << "{\"mode\":\"icache\",\"ctas\":" << grid << ",\"threads\":" << kThreads << ",\"reps\":" << reps
      << ",\"cycles_per_pass\":{";
    auto run = [&](auto kernel, int n, bool first) -> int {
      kernel<<<grid, kThreads, 0, r.stream>>>(reps, out, sink);
      if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(r.stream) != cudaSuccess) return -1;
      std::vector<unsigned long long> v(grid);
      if (cudaMemcpy(v.data(), out, grid * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
      std::sort(v.begin(), v.end());
      o << (first ? "" : ",") << "\"" << n * 16 / 1024 << "KB\":" << v[grid / 2];
      return 0;
    };
    int bad = 0;
    bad |= run(k_icache<512>, 512, true);
    bad |= run(k_icache<1024>, 1024, false);
    bad |= run(k_icache<2048>, 2048, false);
    bad |= run(k_icache<4096>, 4096, false);
    o << "},\"cycles_per_call\":{";
    auto run_calls = [&](auto kernel, int n, bool first) -> int {
      kernel<<<grid, kThreads, 0, r.stream>>>(reps, out, sink);
      if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(r.stream) != cudaSuccess) return -1;
      std::vector<unsigned long long> v(grid);
      if (cudaMemcpy(v.data(), out, grid * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
      std::sort(v.begin(), v.end());
      o << (first ? "" : ",") << "\"" << n << "fn\":" << v[grid / 2];
      return 0;
    };
    bad |= run_calls(k_icache_calls<8>, 8, true);
    bad |= run_calls(k_icache_calls<16>, 16, false);
    bad |= run_calls(k_icache_calls<32>, 32, false);
    bad |= run_calls(k_icache_calls<64>, 64, false);
    bad |= run_calls(k_icache_calls<128>, 128, false);
    bad |= run_calls(k_icache_calls<256>, 256, false);
    cudaFree(out);
    cudaFree(sink);
    if (bad) {
      g_transport_error = "icache kernel failed";
      return ST_ERR_CUDA;
    }
    o << "}}";
    *json = o.str();
    return ST_OK;
  }
  if (mode == "primitives") {
    const int grid = prop.multiProcessorCount;
    float* w = nullptr;
    unsigned long long* out = nullptr;
    TB_CUDA(cudaMalloc(&w, 16 * 512 * sizeof(float)));
    TB_CUDA(cudaMalloc(&out, (size_t)kPrimitives * grid * sizeof(unsigned long long)));
    TB_CUDA(cudaMemsetAsync(w, 0, 16 * 512 * sizeof(float), r.stream));
    const size_t smem = ((sizeof(Smem) + 127) / 128) * 128 + 16 * 512 * sizeof(float);
    TB_CUDA(cudaFuncSetAttribute(k_primitives, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int reps = (int)std::min<size_t>(std::max<size_t>(count, 1), 100000);
    k_primitives<<<grid, kThreads, smem, r.stream>>>(w, reps, out);
    TB_CUDA(cudaGetLastError());
    TB_CUDA(cudaStreamSynchronize(r.stream));
    std::vector<unsigned long long> v((size_t)kPrimitives * grid);
    TB_CUDA(cudaMemcpy(v.data(), out, v.size() * 8, cudaMemcpyDeviceToHost));
    cudaFree(w);
    cudaFree(out);
    static const char* names[kPrimitives] = {"syncthreads", "block_sum", "gemv_smem_16x512", "gemv_global_16x512",
                                             "gemv_smem_64x64", "gemv_global_64x64", "warp_rows_pairs_16x512",
                                             "warp_rows_pairs_16x512_no_barrier", "warp_rows_64x64",
                                             "warp_rows_pairs_16x512_global"};
    o << "{\"mode\":\"primitives\",\"ctas\":" << grid << ",\"threads\":" << kThreads << ",\"reps\":" << reps
      << ",\"cycles_median\":{";
    for (int p = 0; p < kPrimitives; ++p) {
      std::vector<unsigned long long> s(v.begin() + (size_t)p * grid, v.begin() + (size_t)(p + 1) * grid);
      std::sort(s.begin(), s.end());
      o << (p ? "," : "") << "\"" << names[p] << "\":" << s[grid / 2];
    }
    o << "}}";
    *json = o.str();
    return ST_OK;
  }
  if (mode == "bulk-stream" || mode == "load-stream") {
    const int grid = prop.multiProcessorCount;
    const size_t per = 1u << 20;
    char* src = nullptr;
    unsigned long long* cyc = nullptr;
    float* sink = nullptr;
    TB_CUDA(cudaMalloc(&src, per * grid));
    TB_CUDA(cudaMalloc(&cyc, grid * sizeof(unsigned long long)));
    TB_CUDA(cudaMalloc(&sink, grid * sizeof(float)));
    TB_CUDA(cudaMemsetAsync(src, 1, per * grid, r.stream));
    const int rounds = (int)std::min<size_t>(count, 1000);
    const size_t smem = sizeof(StreamRing);
    if (mode == "bulk-stream")
      TB_CUDA(cudaFuncSetAttribute(k_bulk_stream, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    auto launch = [&](int rr) {
      if (mode == "bulk-stream") k_bulk_stream<<<grid, kThreads, smem, r.stream>>>(src, per, rr, cyc, sink);
      else k_load_stream<<<grid, kThreads, 0, r.stream>>>(src, per, rr, sink);
    };
    launch(1);
    TB_CUDA(cudaGetLastError());
    TB_CUDA(cudaEventRecord(r.e0, r.stream));
    launch(rounds);
    TB_CUDA(cudaEventRecord(r.e1, r.stream));
    TB_CUDA(cudaEventSynchronize(r.e1));
    TB_CUDA(cudaGetLastError());
    float ms = 0;
    TB_CUDA(cudaEventElapsedTime(&ms, r.e0, r.e1));
    std::vector<unsigned long long> cycles(grid, 0);
    if (mode == "bulk-stream") TB_CUDA(cudaMemcpy(cycles.data(), cyc, grid * 8, cudaMemcpyDeviceToHost));
    cudaFree(src);
    cudaFree(cyc);
    cudaFree(sink);
    std::sort(cycles.begin(), cycles.end());
    const double bytes = (double)per * grid * rounds;
    o << "{\"mode\":\"" << mode << "\",\"ctas\":" << grid << ",\"mib_per_cta\":1,\"rounds\":" << rounds
      << ",\"gb_per_s\":" << bytes / (ms * 1e-3) / 1e9 << ",\"issue_cycles_median\":" << cycles[grid / 2]
      << ",\"issue_cycles_max\":" << cycles[grid - 1] << "}";
    *json = o.str();
    return ST_OK;
  }
  if (mode == "ll-exchange" || mode == "cluster-barrier") {
    const int grid = mode == "ll-exchange" ? prop.multiProcessorCount : prop.multiProcessorCount / 8 * 8;
    float ms = 0;
    int err = 0;
    if (mode == "ll-exchange") {
      const int n = 512;
      TB_CUDA(cudaMalloc(&r.counter, 2 * n * sizeof(unsigned long long)));
      TB_CUDA(cudaMalloc(&r.error_word, sizeof(int)));
      TB_CUDA(cudaMemsetAsync(r.counter, 0, 2 * n * sizeof(unsigned long long), r.stream));
      TB_CUDA(cudaMemsetAsync(r.error_word, 0, sizeof(int), r.stream));
      int per_sm = 0;
      TB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_ll_exchange, kThreads, 0));
      if (per_sm < 1) { g_transport_error = "exchange kernel cannot be resident"; return ST_ERR_CUDA; }
      unsigned long long warm = 16, cnt = count;
      unsigned int e0 = 1, e1 = 1 + 16;
      int nn = n;
      void* wp[] = {&r.counter, &nn, &warm, &e0, &r.error_word};
      TB_CUDA(cudaLaunchCooperativeKernel((const void*)k_ll_exchange, grid, kThreads, wp, 0, r.stream));
      void* pp[] = {&r.counter, &nn, &cnt, &e1, &r.error_word};
      TB_CUDA(cudaEventRecord(r.e0, r.stream));
      TB_CUDA(cudaLaunchCooperativeKernel((const void*)k_ll_exchange, grid, kThreads, pp, 0, r.stream));
      TB_CUDA(cudaEventRecord(r.e1, r.stream));
      TB_CUDA(cudaEventSynchronize(r.e1));
      TB_CUDA(cudaMemcpy(&err, r.error_word, sizeof err, cudaMemcpyDeviceToHost));
    } else {
      unsigned long long warm = 16, cnt = count;
      k_cluster_barriers<<<grid, kThreads, 0, r.stream>>>(warm);
      TB_CUDA(cudaGetLastError());
      TB_CUDA(cudaEventRecord(r.e0, r.stream));
      k_cluster_barriers<<<grid, kThreads, 0, r.stream>>>(cnt);
      TB_CUDA(cudaEventRecord(r.e1, r.stream));
      TB_CUDA(cudaEventSynchronize(r.e1));
      TB_CUDA(cudaGetLastError());
    }
    TB_CUDA(cudaEventElapsedTime(&ms, r.e0, r.e1));
    o << "{\"mode\":\"" << mode << "\",\"events\":" << count << ",\"ctas\":" << grid << ",\"threads\":" << kThreads
      << ",\"ns_per_round\":" << (ms * 1e6 / (double)count) << ",\"failed\":" << (err ? count : 0) << "}";
    *json = o.str();
    if (err) { g_transport_error = "exchange wait exceeded its bound"; return ST_ERR_DEVICE_TIMEOUT; }
    return ST_OK;
  }
  if (mode == "grid-barrier") {
    TB_CUDA(cudaMalloc(&r.counter, sizeof(unsigned long long)));
    TB_CUDA(cudaMalloc(&r.error_word, sizeof(int)));
    TB_CUDA(cudaMemsetAsync(r.counter, 0, sizeof(unsigned long long), r.stream));
    TB_CUDA(cudaMemsetAsync(r.error_word, 0, sizeof(int), r.stream));
    StepArgs a{};
    a.bar_counter = r.counter;
    a.error = r.error_word;
    a.bar_timeout_ns = 2ull * 1000000000ull;
    int per_sm = 0;
    TB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_barriers, kThreads, 0));
    const int grid = prop.multiProcessorCount;
    if (per_sm < 1) { g_transport_error = "barrier kernel cannot be resident"; return ST_ERR_CUDA; }
    unsigned long long n = 16, base = 0;
    void* warm[] = {&a, &n, &base};
    TB_CUDA(cudaLaunchCooperativeKernel((const void*)k_barriers, grid, kThreads, warm, 0, r.stream));
    base += n * grid;
    unsigned long long cnt = count;
    void* params[] = {&a, &cnt, &base};
    TB_CUDA(cudaEventRecord(r.e0, r.stream));
    TB_CUDA(cudaLaunchCooperativeKernel((const void*)k_barriers, grid, kThreads, params, 0, r.stream));
    TB_CUDA(cudaEventRecord(r.e1, r.stream));
    TB_CUDA(cudaEventSynchronize(r.e1));
    int err = 0;
    TB_CUDA(cudaMemcpy(&err, r.error_word, sizeof err, cudaMemcpyDeviceToHost));
    float ms = 0;
    TB_CUDA(cudaEventElapsedTime(&ms, r.e0, r.e1));
    o << "{\"mode\":\"grid-barrier\",\"events\":" << count << ",\"ctas\":" << grid << ",\"threads\":" << kThreads
      << ",\"ns_per_barrier\":" << (ms * 1e6 / (double)count) << ",\"failed\":" << (err ? count : 0)
      << ",\"boundary\":\"device time of back-to-back grid barriers (CUDA events), one launch\"}";
    *json = o.str();
    if (err) { g_transport_error = "barrier wait exceeded its bound"; return ST_ERR_DEVICE_TIMEOUT; }
    return ST_OK;
  }
  void* hp = nullptr;
  TB_CUDA(cudaHostAlloc(&hp, sizeof(PingBox), cudaHostAllocMapped));
  r.box_h = (PingBox*)hp;
  std::memset(hp, 0, sizeof(PingBox));
  TB_CUDA(cudaHostGetDevicePointer((void**)&r.box_d, hp, 0));
  TB_CUDA(cudaHostAlloc(&hp, 32 * sizeof(float), cudaHostAllocMapped));
  r.in_h = (float*)hp;
  TB_CUDA(cudaHostGetDevicePointer((void**)&r.in_d, hp, 0));
  TB_CUDA(cudaHostAlloc(&hp, 32 * sizeof(float), cudaHostAllocDefault));
  r.out_h = (float*)hp;
  TB_CUDA(cudaMalloc(&r.dev_in, 32 * sizeof(float)));
  TB_CUDA(cudaMalloc(&r.dev_out, 32 * sizeof(float)));
  TB_CUDA(cudaMalloc(&r.cycles, count * sizeof(unsigned long long)));
  TB_CUDA(cudaMalloc(&r.errors, sizeof(int)));
  TB_CUDA(cudaMemsetAsync(r.errors, 0, sizeof(int), r.stream));
  TB_CUDA(cudaMemsetAsync(r.cycles, 0, count * sizeof(unsigned long long), r.stream));
  TB_CUDA(cudaStreamSynchronize(r.stream));
  if (mode == "empty-graph") {
    TB_CUDA(cudaStreamBeginCapture(r.stream, cudaStreamCaptureModeThreadLocal));
    k_empty<<<1, 1, 0, r.stream>>>();
    TB_CUDA(cudaStreamEndCapture(r.stream, &r.graph));
    TB_CUDA(cudaGraphInstantiate(&r.exec, r.graph, 0));
  }
  if (interactive) {
    k_ping<<<1, 1, 0, r.stream>>>(r.box_d, r.in_d, count, backoff, 30ull * 1000000000ull, mode == "gpu-ping",
                                  r.cycles, r.errors);
    TB_CUDA(cudaGetLastError());
  }
  std::vector<double> samples(count);
  unsigned long long failed = 0;
  auto wait = [&](unsigned long long* word, unsigned long long seq) -> int {
    const auto start = std::chrono::steady_clock::now();
    size_t polls = 0;
    while (__atomic_load_n(word, __ATOMIC_ACQUIRE) != seq) {
      if (backoff) std::this_thread::yield();
      if ((++polls & 0xffff) == 0) {
        if (__atomic_load_n(&r.box_h->exited, __ATOMIC_ACQUIRE)) {
          g_transport_error = "Ping-pong kernel exited before request/acknowledgement";
          return ST_ERR_WORKER_EXITED;
        }
        if (std::chrono::steady_clock::now() - start > std::chrono::seconds(60)) {
          g_transport_error = "Ping-pong host timeout";
          return ST_ERR_HOST_TIMEOUT;
        }
      }
    }
    return ST_OK;
  };
  const auto begin = std::chrono::steady_clock::now();
  for (unsigned long long seq = 1; seq <= count; ++seq) {
    unsigned long long checksum = 0;
    for (int i = 0; i < 32; ++i) {
      r.in_h[i] = float(seq % 1024 + i);
      uint32_t bits;
      std::memcpy(&bits, r.in_h + i, 4);
      checksum += bits;
    }
    const auto t0 = std::chrono::steady_clock::now();
    if (mode == "gpu-ping") {
      int st = wait(&r.box_h->request, seq);
      if (st != ST_OK) return st;
      if (r.box_h->checksum != seq * 2654435761ull) ++failed;
      r.box_h->checksum ^= 0xabcdefull;
      __atomic_store_n(&r.box_h->completion, seq, __ATOMIC_RELEASE);
    } else if (mode == "ping-pong") {
      __atomic_store_n(&r.box_h->request, seq, __ATOMIC_RELEASE);
      int st = wait(&r.box_h->completion, seq);
      if (st != ST_OK) return st;
      if (r.box_h->checksum != checksum) ++failed;
    } else {
      if (mode == "empty") {
        k_empty<<<1, 1, 0, r.stream>>>();
      } else if (mode == "empty-graph") {
        TB_CUDA(cudaGraphLaunch(r.exec, r.stream));
      } else {
        TB_CUDA(cudaMemcpyAsync(r.dev_in, r.in_h, 128, cudaMemcpyHostToDevice, r.stream));
        k_echo<<<1, 32, 0, r.stream>>>(r.dev_in, r.dev_out, 32);
        TB_CUDA(cudaMemcpyAsync(r.out_h, r.dev_out, 128, cudaMemcpyDeviceToHost, r.stream));
      }
      TB_CUDA(cudaGetLastError());
      TB_CUDA(cudaStreamSynchronize(r.stream));
      if (mode == "copy" && std::memcmp(r.out_h, r.in_h, 128)) ++failed;
    }
    samples[seq - 1] = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
  }
  const double wall = std::chrono::duration<double>(std::chrono::steady_clock::now() - begin).count();
  TB_CUDA(cudaStreamSynchronize(r.stream));
  std::vector<unsigned long long> cycles(count, 0);
  if (interactive) {
    TB_CUDA(cudaMemcpy(cycles.data(), r.cycles, count * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    int dev_errors = 0;
    TB_CUDA(cudaMemcpy(&dev_errors, r.errors, sizeof(int), cudaMemcpyDeviceToHost));
    failed += dev_errors;
  }
  if (csv_path && *csv_path) {
    std::ofstream csv(csv_path);
    csv << "sequence,host_observation_us,device_round_trip_or_wait_cycles\n";
    csv.precision(17);
    for (size_t i = 0; i < count; ++i) csv << i + 1 << ',' << samples[i] << ',' << cycles[i] << '\n';
  }
  o << "{\"mode\":\"" << mode << "\",\"events\":" << count << ",\"failed\":" << failed
    << ",\"poll_policy\":\"" << (backoff ? "device-nanosleep-128-host-yield" : "tight") << "\""
    << ",\"wall_seconds\":" << wall << ",\"p50_us\":" << pct(samples, 0.5) << ",\"p99_us\":" << pct(samples, 0.99)
    << ",\"worst_us\":" << pct(samples, 1.0) << ",\"boundary\":\""
    << (mode == "gpu-ping" ? "host wait+ack service observation; GPU round trip in device cycles"
                           : "host submission through host-visible completion")
    << "\"}";
  *json = o.str();
  if (failed) {
    g_transport_error = "Transport checksum failure";
    return ST_ERR_CUDA;
  }
  return ST_OK;
}

}  // namespace

extern "C" int st_transport_bench(int device, const char* mode, size_t count, int backoff, const char* csv_path,
                                  char* json, size_t capacity, size_t* needed) {
  if (!mode) return ST_ERR_INVALID;
  std::string out;
  const int st = run_bench(device, mode, count, backoff, csv_path, &out);
  if (needed) *needed = out.size() + 1;
  if (json && capacity) {
    const size_t n = std::min(capacity - 1, out.size());
    std::memcpy(json, out.data(), n);
    json[n] = '\0';
  }
  return st;
}

extern "C" const char* st_transport_error(void) { return g_transport_error.c_str(); }
