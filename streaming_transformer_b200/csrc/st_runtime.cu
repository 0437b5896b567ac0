// st_runtime.cu -- host runtime behind the C ABI (include/streaming_b200.h).
//
// Owns every device and pinned buffer of one runtime and drives the kernels of
// st_kernels.cuh for the five backends. It takes the place of the reference's
// Runtime::Impl (reference src/cuda/Runtime.cu:164-665) behind a plain C ABI.
//
// Device layout (one runtime, S streams):
//   weights slab   every tensor 256-byte aligned, in storage precision; per
//                  layer q/k/v are fused into one [3d, d] matrix and gate/up are
//                  interleaved row by row into [2F, d] so each CTA's row range
//                  is one contiguous span and pairs (RoPE, SwiGLU) stay together
//   state          K, V [S][L][H][W][hd] storage precision; hidden [S][L][d]
//                  fp32; position u64 [S]
//   scratch        fp32 activations, attention partials, barrier counter,
//                  error word, RoPE frequency table
//   mapped pinned  mailbox (request/completion/exited on separate 64-byte
//                  lines), input [S][features], scores [S]
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <map>
#include <sstream>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "../../include/streaming_b200.h"
#include "st_flow.cuh"
#include "st_flow_host.h"

using namespace st;

namespace {

thread_local std::string g_create_error;

// Where element (r, c) of a checkpoint tensor [rows, cols] lands in its region.
enum LayoutKind : int {
  kPlain = 0,      // dst row = r * p0 + p1 (p0 = 2 interleaves gate/up)
  kQkvHead = 1,    // q/k/v [d, d] -> [H][3][hd][d]; p0 = which (0 q, 1 k, 2 v), p1 = hd
  kOutHead = 2,    // out [d, d] -> [H][d][hd]; p1 = hd
  kTranspose = 3   // down [d, F] -> [F][d]
};

struct TensorSlot {
  size_t offset;      // bytes into the weights slab (region start)
  int rows, cols;     // logical tensor shape (1-D tensors: rows = 1)
  int kind, p0, p1;   // LayoutKind and its parameters
  int index;          // presence flag index
  // Tensor-core copy (batched round, 16-bit modes): the GEMM matrix this
  // tensor belongs to, pre-tiled for the MMA; tiled_rows = 0 when none.
  size_t tiled_offset = 0;
  int tiled_rows = 0, tiled_cols = 0;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Exact widening of binary16 / bfloat16 bit patterns for snapshots.
float half_bits_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: value = man * 2^-24
      float v = (float)man * (1.0f / 16777216.0f);
      std::memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}
float bf16_bits_to_float(uint16_t h) {
  uint32_t bits = (uint32_t)h << 16;
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

template <typename T>
__global__ void k_convert(const float* src, T* dst, int rows, int cols, int kind, int p0, int p1) {
  const size_t n = (size_t)rows * cols;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / cols, c = i - r * cols;
    size_t at;
    if (kind == kQkvHead) {
      const size_t h = r / p1, dim = r % p1;
      at = ((h * 3 + p0) * p1 + dim) * cols + c;
    } else if (kind == kOutHead) {
      const size_t h = c / p1, e = c % p1;
      at = (h * rows + r) * p1 + e;
    } else if (kind == kTranspose) {
      at = c * rows + r;
    } else {
      at = (r * p0 + p1) * cols + c;
    }
    Storage<T>::store(dst, at, src[i]);
  }
}

// The tensor-core copy of one checkpoint tensor: element (r, c) goes to row m,
// column k of its GEMM matrix (q/k/v fused head-major [3d, d], out [d, d],
// gate/up interleaved [2F, d], down [d, F]) in the MMA's tiled layout
// (umma_tile_offset, 128-row tiles). fp32: tf32 hi at the tiled offset
// (umma_tile_offset32) and tf32 lo `lo` floats further (the padded matrix size).
template <typename T>
__global__ void k_convert_tiled(const float* src, T* dst, int rows, int cols, int kind, int p0, int p1, int gemm_cols,
                                size_t lo) {
  const size_t n = (size_t)rows * cols;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / cols, c = i - r * cols;
    size_t m = r;
    if (kind == kQkvHead) m = ((r / p1) * 3 + p0) * p1 + r % p1;
    else if (kind == kPlain) m = r * p0 + p1;
    if constexpr (std::is_same<T, float>::value) {
      const size_t at = umma_tile_offset32(m, c, kUmmaM, (size_t)gemm_cols / kTileK32);
      const float hi = to_tf32(src[i]);
      dst[at] = hi;
      dst[lo + at] = to_tf32(src[i] - hi);
    } else {
      Storage<T>::store(dst, umma_tile_offset(m, c, kUmmaM, (size_t)gemm_cols / kTileK), src[i]);
    }
  }
}

}  // namespace

struct st_runtime {
  st_model_desc desc{};
  st_options opt{};
  int device = 0;
  int sms = 0;
  int grid = 1;
  int cluster = 1;        // CTAs per cluster
  int nclusters = 1;
  int legal_blocks = 1;
  // Step kernels are plain cluster launches. A cooperative launch would add the
  // co-residency guarantee, but a profiler replays it without its runtime
  // cluster shape; the grid is instead sized from cudaOccupancyMaxActiveClusters
  // (all clusters fit at once) and every grid-sync wait is bounded.
  bool coop_clusters = false;
  // Device-loop kernels stream their weights through the shared-memory ring
  // (st_ring.cuh) when the configuration allows it (ring_supported); the
  // environment variable ST_WEIGHT_RING=0 selects the direct-load variants.
  bool ring = false;
  // Several streams step together through the batched round (st_batch.cuh):
  // one CTA per SM, every weight read once per round for all streams. Chosen
  // for 4 or more streams when the model allows it; ST_BATCHED=0/1 overrides.
  bool batched = false;
  bool tc = false;        // batched GEMM phases on the tensor cores (fp32 as three tf32 products)
  // One stream at the benchmark shapes: the device-loop backends (FUSED,
  // PERSISTENT, device traces) run the flow kernel (st_flow.cuh) on its own
  // cluster shape; ST_FLOW=0 selects the generic kernels.
  bool flow = false;
  const void* flow_fn = nullptr;
  // tensor parallelism of the one stream over tp_size GPUs (st_create_tp)
  int tp_rank = 0, tp_size = 1;
  size_t llh_at = 0, llx_at = 0;          // record buffers' offsets in the scratch allocation
  char* tp_peer_base[kMaxTp] = {};        // peers' scratch allocations opened through IPC
  const void* flow_diag_fn = nullptr;  // the same kernel with per-phase cycle sums (timelines)
  int fcluster = 0, fnclusters = 0, fgrid = 0;
  int bgrid = 0;
  int bsplit[4] = {1, 1, 1, 1};
  int tcn[4] = {0, 0, 0, 0};  // streams per tensor-core GEMM unit
  size_t tc_smem = 0;     // dynamic shared memory of the tensor-core rounds kernel
  char* tweights = nullptr;
  size_t tweights_bytes = 0;
  size_t elem = 4;
  cudaStream_t stream = nullptr;
  cudaStream_t aux = nullptr;
  cudaEvent_t ev_start = nullptr, ev_stop = nullptr;

  char* weights = nullptr;
  size_t weights_bytes = 0;
  std::map<std::string, TensorSlot> slots;
  std::vector<char> have;

  char* state = nullptr;
  size_t state_bytes = 0;
  char* scratch = nullptr;
  size_t scratch_bytes = 0;
  size_t kv_bytes_per_tensor = 0;

  Mailbox* mb_h = nullptr;
  Mailbox* mb_d = nullptr;
  float* in_h = nullptr;
  float* in_d = nullptr;   // device alias of in_h
  float* out_h = nullptr;
  float* out_d = nullptr;  // device alias of out_h
  float* dev_input = nullptr;
  float* dev_score = nullptr;
  Control* control = nullptr;

  StepArgs args{};
  unsigned long long bar_base = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t graph_exec = nullptr;

  bool started = false;
  bool running = false;  // persistent worker resident
  bool failed = false;
  uint64_t sequence = 0;
  uint64_t launches = 0;
  std::string error;

  int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    error = buf;
    if (code == ST_ERR_CUDA || code == ST_ERR_DEVICE_TIMEOUT) failed = true;
    return code;
  }
  int cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return ST_OK;
    return fail(ST_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  }
};

#define ST_TRY(expr)                                  \
  do {                                                \
    int _st = (expr);                                 \
    if (_st != ST_OK) return _st;                     \
  } while (0)
#define ST_CUDA(rt, expr) ST_TRY((rt)->cuda((expr), #expr))

namespace {

int forward_barrier_count(const st_runtime* rt) { return forward2_barriers(rt->desc.layers, rt->desc.streams); }

constexpr size_t kSmem2 = kStepSmemBytes;

template <typename T>
struct Kernels {
  static const void* input() { return (const void*)k2_input<T>; }
  static const void* attention() { return (const void*)k2_attention<T>; }
  static const void* ffn() { return (const void*)k2_ffn<T>; }
  static const void* final_() { return (const void*)k2_final<T>; }
  static const void* reset() { return (const void*)k_reset<T>; }
  static const void* fused(bool ring) { return ring ? (const void*)k2_fused<T, true> : (const void*)k2_fused<T, false>; }
  static const void* trace(bool ring, bool diag = false) {
    if (diag) return ring ? (const void*)k2_trace<T, true, true> : (const void*)k2_trace<T, false, true>;
    return ring ? (const void*)k2_trace<T, true, false> : (const void*)k2_trace<T, false, false>;
  }
  static const void* persistent(bool ring) {
    return ring ? (const void*)k2_persistent<T, true> : (const void*)k2_persistent<T, false>;
  }
  static const void* convert() { return (const void*)k_convert<T>; }
  static const void* rounds(bool tc) { return tc ? (const void*)k3_rounds<T, true> : (const void*)k3_rounds<T, false>; }
};

#define ST_KERNEL(rt, name) \
  ((rt)->desc.mode == ST_MODE_FP16 ? Kernels<__half>::name() \
   : (rt)->desc.mode == ST_MODE_BF16 ? Kernels<__nv_bfloat16>::name() : Kernels<float>::name())
// The device-loop kernels in the weight-ring or direct-load variant the runtime chose.
#define ST_LOOP_KERNEL(rt, name) \
  ((rt)->desc.mode == ST_MODE_FP16 ? Kernels<__half>::name((rt)->ring) \
   : (rt)->desc.mode == ST_MODE_BF16 ? Kernels<__nv_bfloat16>::name((rt)->ring) : Kernels<float>::name((rt)->ring))
// The trace kernel with the phase timeline compiled in.
#define ST_TIMELINE_KERNEL(rt) \
  ((rt)->desc.mode == ST_MODE_FP16 ? Kernels<__half>::trace((rt)->ring, true) \
   : (rt)->desc.mode == ST_MODE_BF16 ? Kernels<__nv_bfloat16>::trace((rt)->ring, true) \
                                     : Kernels<float>::trace((rt)->ring, true))

const void* persistent_fn(const st_runtime* rt) { return ST_LOOP_KERNEL(rt, persistent); }
const void* rounds_fn(const st_runtime* rt) {
  if (rt->desc.mode == ST_MODE_FP16) return Kernels<__half>::rounds(rt->tc);
  if (rt->desc.mode == ST_MODE_BF16) return Kernels<__nv_bfloat16>::rounds(rt->tc);
  return Kernels<float>::rounds(rt->tc);
}

// Launch with this runtime's cluster shape. `cooperative` requests the
// co-residency guarantee when coop_clusters is set (off: see st_runtime).
int launch_ex(st_runtime* rt, const void* fn, int grid, int cluster, bool cooperative, void** params) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem2;
  cfg.stream = rt->stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  attrs[n].id = cudaLaunchAttributeClusterDimension;
  attrs[n].val.clusterDim.x = cluster;
  attrs[n].val.clusterDim.y = 1;
  attrs[n].val.clusterDim.z = 1;
  ++n;
  if (cooperative && rt->coop_clusters) {
    attrs[n].id = cudaLaunchAttributeCooperative;
    attrs[n].val.cooperative = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelExC(&cfg, fn, params);
  if (e != cudaSuccess && cooperative && rt->coop_clusters) {
    (void)cudaGetLastError();
    rt->coop_clusters = false;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelExC(&cfg, fn, params);
  }
  rt->launches += 1;
  return rt->cuda(e, "cluster launch");
}

int launch_sequence(st_runtime* rt, const StepArgs& a0) {
  StepArgs a = a0;
  const void* kin = ST_KERNEL(rt, input);
  const void* kat = ST_KERNEL(rt, attention);
  const void* kff = ST_KERNEL(rt, ffn);
  const void* kfi = ST_KERNEL(rt, final_);
  void* p0[] = {&a};
  ST_TRY(launch_ex(rt, kin, rt->grid, rt->cluster, false, p0));
  for (int l = 0; l < rt->desc.layers; ++l) {
    void* p1[] = {&a, &l};
    ST_TRY(launch_ex(rt, kat, rt->grid, rt->cluster, false, p1));
    ST_TRY(launch_ex(rt, kff, rt->grid, rt->cluster, false, p1));
  }
  int nc = rt->nclusters;
  void* p2[] = {&a, &nc};
  ST_TRY(launch_ex(rt, kfi, 1, 1, false, p2));
  return ST_OK;
}

int sequence_launches(const st_runtime* rt) { return 2 + 2 * rt->desc.layers; }

int launch_reset(st_runtime* rt, int s0, int s1) {
  StepArgs a = rt->args;
  void* p[] = {&a, &s0, &s1};
  return launch_ex(rt, ST_KERNEL(rt, reset), rt->grid, rt->cluster, false, p);
}

// The flow kernel's arguments: its own cluster shape in place of the generic one.
StepArgs flow_args(const st_runtime* rt, const StepArgs& a0) {
  StepArgs a = a0;
  a.cluster_size = rt->fcluster;
  a.clusters = rt->fnclusters;
  return a;
}

int launch_flow(st_runtime* rt, const StepArgs& a0, const FlowLaunch& f) {
  const void* fn = a0.timeline ? rt->flow_diag_fn : rt->flow_fn;
  const cudaError_t e = flow_launch(fn, rt->fgrid, rt->fcluster, rt->stream, flow_args(rt, a0), f);
  rt->launches += 1;
  return rt->cuda(e, "flow cluster launch");
}

int launch_flow_trace(st_runtime* rt, const StepArgs& a, const float* inputs, unsigned long long count, float* scores) {
  FlowLaunch f{};
  f.mode = kFlowTrace;
  f.inputs = inputs;
  f.count = count;
  f.scores = scores;
  f.bar_base = rt->bar_base;
  return launch_flow(rt, a, f);
}

int launch_fused(st_runtime* rt, const StepArgs& a0) {
  if (rt->flow) return launch_flow_trace(rt, a0, a0.input, 1, nullptr);
  StepArgs a = a0;
  unsigned long long base = rt->bar_base;
  void* params[] = {&a, &base};
  ST_TRY(launch_ex(rt, ST_LOOP_KERNEL(rt, fused), rt->grid, rt->cluster, true, params));
  rt->bar_base += (unsigned long long)forward_barrier_count(rt) * rt->nclusters;
  return ST_OK;
}

int launch_trace(st_runtime* rt, const StepArgs& a0, const float* inputs, unsigned long long count, float* scores,
                 bool timeline = false) {
  if (rt->flow) return launch_flow_trace(rt, a0, inputs, count, scores);
  StepArgs a = a0;
  unsigned long long base = rt->bar_base;
  void* params[] = {&a, &inputs, &count, &scores, &base};
  ST_TRY(launch_ex(rt, timeline ? ST_TIMELINE_KERNEL(rt) : ST_LOOP_KERNEL(rt, trace), rt->grid, rt->cluster, true,
                   params));
  rt->bar_base += count * (unsigned long long)forward_barrier_count(rt) * rt->nclusters;
  return ST_OK;
}

// `count` batched rounds over inputs [count][S][features] (device memory);
// scores [count][S] may be null (a.score always holds the last round's).
int launch_rounds(st_runtime* rt, const StepArgs& a0, const float* inputs, unsigned long long count, float* scores) {
  StepArgs a = a0;
  unsigned long long base = rt->bar_base;
  void* params[] = {&a, &inputs, &count, &scores, &base};
  ST_CUDA(rt, cudaLaunchKernel(rounds_fn(rt), dim3(rt->bgrid), dim3(kThreads), params, rt->tc_smem, rt->stream));
  rt->launches += 1;
  rt->bar_base += count * (unsigned long long)round_barriers(rt->desc.layers, rt->args.fuse_swiglu != 0) * (unsigned long long)rt->bgrid;
  return ST_OK;
}

// Host-side check of the error word mirrored into mapped memory.
int check_device_error(st_runtime* rt) {
  const int e = __atomic_load_n(&rt->mb_h->error, __ATOMIC_ACQUIRE);
  if (e == kBarrierTimeout) return rt->fail(ST_ERR_DEVICE_TIMEOUT, "device grid barrier wait exceeded its bound");
  if (e == kClusterShape) return rt->fail(ST_ERR_CUDA, "kernel launched with a cluster shape other than the runtime's");
  if (e == kRingTable) return rt->fail(ST_ERR_STATE, "weight ring chunk table does not fit this configuration");
  if (e != 0) return rt->fail(ST_ERR_DEVICE_TIMEOUT, "device error code %d", e);
  return ST_OK;
}

// Load every kernel of this mode before a resident worker starts: lazy module
// loading of a cold kernel can synchronize the context, which would wait for a
// worker that is itself waiting for the host (reference src/cuda/Runtime.cu:288-290).
int preload(st_runtime* rt) {
  const void* fns[] = {ST_KERNEL(rt, input), ST_KERNEL(rt, attention), ST_KERNEL(rt, ffn), ST_KERNEL(rt, final_),
                       ST_KERNEL(rt, reset), ST_LOOP_KERNEL(rt, fused), ST_LOOP_KERNEL(rt, trace), ST_LOOP_KERNEL(rt, persistent),
                       ST_TIMELINE_KERNEL(rt), ST_KERNEL(rt, convert), rounds_fn(rt),
                       rt->flow ? rt->flow_fn : ST_KERNEL(rt, input), rt->flow ? rt->flow_diag_fn : ST_KERNEL(rt, input)};
  for (const void* f : fns) {
    cudaFuncAttributes fa{};
    ST_CUDA(rt, cudaFuncGetAttributes(&fa, f));
  }
  return ST_OK;
}

int start_persistent(st_runtime* rt) {
  ST_CUDA(rt, cudaMemsetAsync(rt->control, 0, sizeof(Control), rt->stream));
  std::memset((void*)rt->mb_h, 0, sizeof(Mailbox));
  rt->sequence = rt->opt.initial_sequence;
  __atomic_store_n(&rt->mb_h->request, rt->sequence, __ATOMIC_RELEASE);
  __atomic_store_n(&rt->mb_h->completion, rt->sequence, __ATOMIC_RELEASE);
  PersistArgs p{};
  p.mailbox = rt->mb_d;
  p.max_events = rt->opt.max_events;
  p.initial_sequence = rt->opt.initial_sequence;
  p.idle_ns = (unsigned long long)(rt->opt.idle_seconds * 1e9);
  p.dispatch_timeout_ns = p.idle_ns + 10ull * 1000000000ull;
  p.control = rt->control;
  p.backoff = rt->opt.backoff;
  StepArgs a = rt->args;
  a.input = rt->dev_input;
  a.score = rt->out_d;
  const float* mapped = rt->in_d;
  unsigned long long base = rt->bar_base;
  if (rt->flow) {
    FlowLaunch f{};
    f.mode = kFlowPersistent;
    f.p = p;
    f.mapped_input = mapped;
    f.bar_base = base;
    ST_CUDA(rt, cudaMemsetAsync(rt->args.flow_ctl, 0, sizeof(unsigned long long), rt->stream));
    ST_TRY(launch_flow(rt, a, f));
    rt->running = true;
    return ST_OK;
  }
  void* params[] = {&a, &p, &mapped, &base};
  ST_TRY(launch_ex(rt, persistent_fn(rt), rt->grid, rt->cluster, true, params));
  rt->running = true;
  return ST_OK;
}

// After the resident worker has left: join it and restart barrier accounting.
int join_persistent(st_runtime* rt) {
  rt->running = false;
  ST_CUDA(rt, cudaStreamSynchronize(rt->stream));
  ST_CUDA(rt, cudaMemsetAsync(rt->args.bar_counter, 0, sizeof(unsigned long long), rt->stream));
  ST_CUDA(rt, cudaStreamSynchronize(rt->stream));
  rt->bar_base = 0;
  return check_device_error(rt);
}

// reference src/cuda/Runtime.cu:398-428
int command(st_runtime* rt, int cmd, int arg) {
  if (!rt->running) return rt->fail(ST_ERR_STOPPED, "Persistent runtime is stopped");
  const uint64_t maximum = std::numeric_limits<uint64_t>::max();
  if (rt->sequence == maximum || (rt->sequence == maximum - 1 && cmd != kStop))
    return rt->fail(ST_ERR_EXHAUSTED, "Sequence exhausted; create a new runtime before wraparound");
  if (__atomic_load_n(&rt->mb_h->exited, __ATOMIC_ACQUIRE)) {
    int st = join_persistent(rt);
    if (st != ST_OK) return st;
    return rt->fail(ST_ERR_WORKER_EXITED, "Persistent worker exited: finite-event or idle budget reached");
  }
  rt->mb_h->command = cmd;
  rt->mb_h->arg = arg;
  // Input and command are written before the request is published.
  __atomic_store_n(&rt->mb_h->request, ++rt->sequence, __ATOMIC_RELEASE);
  const auto start = std::chrono::steady_clock::now();
  uint64_t polls = 0;
  while (__atomic_load_n(&rt->mb_h->completion, __ATOMIC_ACQUIRE) != rt->sequence) {
    if (rt->opt.backoff) std::this_thread::yield();
    if ((++polls & 0xffff) == 0) {
      if (__atomic_load_n(&rt->mb_h->exited, __ATOMIC_ACQUIRE) || cudaStreamQuery(rt->stream) != cudaErrorNotReady) {
        int st = join_persistent(rt);
        if (st != ST_OK) return st;
        return rt->fail(ST_ERR_WORKER_EXITED, "Persistent worker exited before completion");
      }
      const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
      if (waited > rt->opt.idle_seconds + 30)
        return rt->fail(ST_ERR_HOST_TIMEOUT, "Persistent response timeout");
    }
  }
  return ST_OK;
}

int validate_desc(const st_model_desc* m) {
  // reference src/runtime/Model.cpp:22-29 plus the stream count and mode.
  if (m->layers < 1 || m->layers > 16 || m->width < 1 || m->width > 1024 || m->heads < 1 ||
      m->width % m->heads || (m->width / m->heads) % 2 || m->ffn < 1 || m->ffn > 4096 ||
      m->window < 1 || m->window > 4096 || m->features < 1 || m->features > 1024 ||
      !std::isfinite(m->epsilon) || m->epsilon <= 0)
    return 0;
  if (m->mode < ST_MODE_FP32 || m->mode > ST_MODE_BF16) return 0;
  if (m->streams < 1) return 0;
  return 1;
}

int graph_capture(st_runtime* rt) {
  ST_CUDA(rt, cudaStreamBeginCapture(rt->stream, cudaStreamCaptureModeThreadLocal));
  const uint64_t before = rt->launches;
  int st = launch_sequence(rt, rt->args);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(rt->stream, &g);
  if (st != ST_OK) return st;
  ST_TRY(rt->cuda(e, "cudaStreamEndCapture"));
  rt->graph = g;
  ST_CUDA(rt, cudaGraphInstantiate(&rt->graph_exec, g, 0));
  rt->launches = before;  // captured launches are counted when the graph runs
  return ST_OK;
}

int run_step_nonpersistent(st_runtime* rt) {
  const size_t in_bytes = (size_t)rt->desc.streams * rt->desc.features * sizeof(float);
  const size_t out_bytes = (size_t)rt->desc.streams * sizeof(float);
  if (!rt->opt.mapped)
    ST_CUDA(rt, cudaMemcpyAsync(rt->dev_input, rt->in_h, in_bytes, cudaMemcpyHostToDevice, rt->stream));
  if (rt->batched) {
    ST_TRY(launch_rounds(rt, rt->args, rt->args.input, 1, nullptr));
  } else if (rt->opt.backend == ST_BACKEND_GRAPH) {
    ST_CUDA(rt, cudaGraphLaunch(rt->graph_exec, rt->stream));
    rt->launches += sequence_launches(rt);
  } else if (rt->opt.backend == ST_BACKEND_FUSED) {
    ST_TRY(launch_fused(rt, rt->args));
  } else {
    ST_TRY(launch_sequence(rt, rt->args));
  }
  if (!rt->opt.mapped)
    ST_CUDA(rt, cudaMemcpyAsync(rt->out_h, rt->dev_score, out_bytes, cudaMemcpyDeviceToHost, rt->stream));
  ST_CUDA(rt, cudaStreamSynchronize(rt->stream));
  return check_device_error(rt);
}

std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') { o += '\\'; o += c; }
    else if ((unsigned char)c < 0x20) { char b[8]; snprintf(b, sizeof b, "\\u%04x", c); o += b; }
    else o += c;
  }
  return o;
}

int copy_json(const std::string& s, char* json, size_t capacity, size_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (json && capacity) {
    const size_t n = std::min(capacity - 1, s.size());
    std::memcpy(json, s.data(), n);
    json[n] = '\0';
  }
  return ST_OK;
}

std::string probe_json(int device, int* status) {
  *status = ST_OK;
  cudaDeviceProp p{};
  int driver = 0, runtime = 0;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess || cudaDriverGetVersion(&driver) != cudaSuccess ||
      cudaRuntimeGetVersion(&runtime) != cudaSuccess) {
    *status = ST_ERR_CUDA;
    return "{}";
  }
  auto attr = [&](cudaDeviceAttr a) {
    int v = 0;
    cudaDeviceGetAttribute(&v, a, device);
    return v;
  };
  char bus[32] = {0};
  cudaDeviceGetPCIBusId(bus, sizeof bus, device);
  std::ostringstream o;
  o << "{\"gpu\":\"" << json_escape(p.name) << "\",\"device\":" << device << ",\"compute_major\":" << p.major
    << ",\"compute_minor\":" << p.minor << ",\"sm_count\":" << p.multiProcessorCount
    << ",\"registers_per_sm\":" << p.regsPerMultiprocessor << ",\"shared_bytes_per_sm\":" << p.sharedMemPerMultiprocessor
    << ",\"shared_bytes_per_block\":" << p.sharedMemPerBlock << ",\"global_bytes\":" << p.totalGlobalMem
    << ",\"l2_bytes\":" << p.l2CacheSize << ",\"pci_bus\":\"" << bus << "\""
    << ",\"clock_khz\":" << attr(cudaDevAttrClockRate) << ",\"memory_clock_khz\":" << attr(cudaDevAttrMemoryClockRate)
    << ",\"driver_version\":" << driver << ",\"runtime_version\":" << runtime
    << ",\"nvcc\":" << (__CUDACC_VER_MAJOR__ * 1000 + __CUDACC_VER_MINOR__ * 10 + __CUDACC_VER_BUILD__)
    << ",\"build_cuda_architectures\":\"100a\""
    << ",\"kernel_timeout\":" << attr(cudaDevAttrKernelExecTimeout)
    << ",\"cooperative_launch\":" << attr(cudaDevAttrCooperativeLaunch)
    << ",\"can_map_host\":" << attr(cudaDevAttrCanMapHostMemory)
    << ",\"unified_addressing\":" << attr(cudaDevAttrUnifiedAddressing)
    << ",\"host_native_atomic_supported\":" << attr(cudaDevAttrHostNativeAtomicSupported)
    << ",\"cpu_logical_count\":" << std::thread::hardware_concurrency() << ",\"os\":\"Linux\"}";
  return o.str();
}

}  // namespace

extern "C" {

int st_abi_version(void) { return ST_ABI_VERSION; }

void st_default_options(st_options* o) {
  if (!o) return;
  std::memset(o, 0, sizeof *o);
  o->backend = ST_BACKEND_GRAPH;
  o->blocks = 1;
  o->idle_seconds = 30;
}

const char* st_last_error(const st_runtime* rt) { return rt ? rt->error.c_str() : g_create_error.c_str(); }

uint64_t st_kernel_launches(const st_runtime* rt) { return rt ? rt->launches : 0; }

static int create_impl(const st_model_desc* model, const st_options* options, int tp_rank, int tp_size,
                       st_runtime** out);

int st_create(const st_model_desc* model, const st_options* options, st_runtime** out) {
  return create_impl(model, options, 0, 1, out);
}

int st_create_tp(const st_model_desc* model, const st_options* options, int tp_rank, int tp_size,
                 st_runtime** out) {
  if (!model || !options || !out) { g_create_error = "null argument"; return ST_ERR_INVALID; }
  if (tp_size < 1 || tp_size > kMaxTp || tp_rank < 0 || tp_rank >= tp_size) {
    g_create_error = "tensor-parallel rank or size out of range (1..8 GPUs)";
    return ST_ERR_INVALID;
  }
  if (model->streams != 1 || model->heads % tp_size || model->ffn % tp_size) {
    g_create_error = "tensor parallelism needs one stream and heads and ffn divisible by the GPU count";
    return ST_ERR_INVALID;
  }
  if (options->backend != ST_BACKEND_FUSED && options->backend != ST_BACKEND_PERSISTENT) {
    g_create_error = "tensor parallelism runs the single-stream device loop: FUSED or PERSISTENT backend";
    return ST_ERR_UNSUPPORTED;
  }
  return create_impl(model, options, tp_rank, tp_size, out);
}

static int create_impl(const st_model_desc* model, const st_options* options, int tp_rank, int tp_size,
                       st_runtime** out) {
  if (!model || !options || !out) { g_create_error = "null argument"; return ST_ERR_INVALID; }
  *out = nullptr;
  if (!validate_desc(model)) { g_create_error = "Invalid or unsupported model dimensions"; return ST_ERR_INVALID; }
  const st_options& o = *options;
  if (o.backend < ST_BACKEND_CUDA || o.backend > ST_BACKEND_PERSISTENT) { g_create_error = "Unknown backend"; return ST_ERR_INVALID; }
  if (o.backend == ST_BACKEND_CUBLAS || o.backend == ST_BACKEND_CUBLAS_GRAPH) {
    g_create_error = "cuBLAS backends are not provided by the B200 runtime";
    return ST_ERR_UNSUPPORTED;
  }
  // reference src/cuda/Runtime.cu:178-183
  if (o.blocks < 0 || !(o.idle_seconds > 0) || o.idle_seconds > 3600) {
    g_create_error = "Invalid blocks or idle budget";
    return ST_ERR_INVALID;
  }
  if (o.initial_sequence >= std::numeric_limits<uint64_t>::max() - 1) {
    g_create_error = "Initial sequence must leave room for RUN and STOP";
    return ST_ERR_INVALID;
  }
  auto* rt = new st_runtime();
  rt->desc = *model;
  rt->opt = o;
  rt->device = o.device;
  rt->tp_rank = tp_rank;
  rt->tp_size = tp_size;
  auto bail = [&](int code) {
    g_create_error = rt->error;
    st_destroy(rt);
    return code;
  };
  if (rt->cuda(cudaSetDevice(rt->device), "cudaSetDevice") != ST_OK) return bail(ST_ERR_CUDA);
  cudaDeviceProp prop{};
  if (rt->cuda(cudaGetDeviceProperties(&prop, rt->device), "cudaGetDeviceProperties") != ST_OK) return bail(ST_ERR_CUDA);
  if (prop.major != 10) {
    rt->fail(ST_ERR_UNSUPPORTED, "This build targets sm_100a (B200); device is compute %d.%d", prop.major, prop.minor);
    return bail(ST_ERR_UNSUPPORTED);
  }
  int can_map = 0, uva = 0, coop = 0;
  cudaDeviceGetAttribute(&can_map, cudaDevAttrCanMapHostMemory, rt->device);
  cudaDeviceGetAttribute(&uva, cudaDevAttrUnifiedAddressing, rt->device);
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, rt->device);
  if (!can_map || !uva) {
    rt->fail(ST_ERR_UNSUPPORTED, "Mapped communication requires mapped host memory and UVA");
    return bail(ST_ERR_UNSUPPORTED);
  }
  rt->sms = prop.multiProcessorCount;
  const st_model_desc& m = rt->desc;
  rt->elem = m.mode == ST_MODE_FP32 ? 4 : 2;
  // Every step kernel takes the same dynamic shared memory.
  {
    const void* fns[] = {ST_KERNEL(rt, input), ST_KERNEL(rt, attention), ST_KERNEL(rt, ffn), ST_KERNEL(rt, final_),
                         ST_KERNEL(rt, reset), nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                         nullptr, nullptr};
    for (int r = 0; r < 2; ++r) {
      rt->ring = r == 1;
      fns[5 + 3 * r] = ST_LOOP_KERNEL(rt, fused);
      fns[6 + 3 * r] = ST_LOOP_KERNEL(rt, trace);
      fns[7 + 3 * r] = ST_LOOP_KERNEL(rt, persistent);
      fns[11 + r] = ST_TIMELINE_KERNEL(rt);
    }
    rt->ring = false;
    for (const void* f : fns)
      if (rt->cuda(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem2),
                   "cudaFuncSetAttribute") != ST_OK)
        return bail(ST_ERR_CUDA);
  }
  // Cluster shape: 8 CTAs per cluster at full size; an explicit `blocks` takes
  // its largest divisor <= 8. The cooperative limit is the number of co-resident
  // clusters of the compiled kernels (reference src/cuda/Runtime.cu:306-314).
  int cluster = 8;
  if (o.blocks > 0) {
    cluster = 1;
    for (int c = std::min(8, o.blocks); c >= 1; --c)
      if (o.blocks % c == 0) { cluster = c; break; }
  }
  int max_clusters = 1 << 30;
  {
    const void* fns[8];
    for (int r = 0; r < 2; ++r) {
      rt->ring = r == 1;
      fns[4 * r] = ST_LOOP_KERNEL(rt, fused);
      fns[4 * r + 1] = ST_LOOP_KERNEL(rt, trace);
      fns[4 * r + 2] = ST_LOOP_KERNEL(rt, persistent);
      fns[4 * r + 3] = ST_TIMELINE_KERNEL(rt);
    }
    rt->ring = false;
    for (const void* f : fns) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(cluster);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kSmem2;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = cluster;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (rt->cuda(cudaOccupancyMaxActiveClusters(&n, f, &cfg), "cudaOccupancyMaxActiveClusters") != ST_OK)
        return bail(ST_ERR_CUDA);
      max_clusters = std::min(max_clusters, n);
    }
  }
  if (!coop) max_clusters = 1;
  rt->legal_blocks = max_clusters * cluster;
  rt->cluster = cluster;
  if (o.blocks == 0) {
    const int nc = std::max(1, std::min(max_clusters, rt->sms / cluster));
    rt->grid = nc * cluster;
  } else {
    rt->grid = o.blocks;
  }
  rt->nclusters = rt->grid / rt->cluster;
  const bool cooperative = o.backend == ST_BACKEND_FUSED || o.backend == ST_BACKEND_PERSISTENT;
  if (cooperative && rt->grid > rt->legal_blocks) {
    rt->fail(ST_ERR_INVALID, "Requested cooperative grid exceeds actual occupancy limit %d", rt->legal_blocks);
    return bail(ST_ERR_INVALID);
  }
  if (rt->cuda(cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking), "stream") != ST_OK ||
      rt->cuda(cudaStreamCreateWithFlags(&rt->aux, cudaStreamNonBlocking), "stream") != ST_OK ||
      rt->cuda(cudaEventCreate(&rt->ev_start), "event") != ST_OK ||
      rt->cuda(cudaEventCreate(&rt->ev_stop), "event") != ST_OK)
    return bail(ST_ERR_CUDA);

  // ---- weights slab layout
  const int d = m.width, F = m.ffn, L = m.layers, hd = m.width / m.heads;
  size_t off = 0;
  int index = 0;
  auto region = [&](size_t rows, size_t cols) {
    const size_t at = off;
    off = align_up(off + rows * cols * rt->elem, 256);
    return at;
  };
  auto slot = [&](const std::string& name, size_t at, int rows, int cols, int kind, int p0, int p1) {
    rt->slots[name] = TensorSlot{at, rows, cols, kind, p0, p1, index++};
  };
  slot("input", region(d, m.features), d, m.features, kPlain, 1, 0);
  slot("final_norm", region(1, d), 1, d, kPlain, 1, 0);
  slot("score", region(1, d), 1, d, kPlain, 1, 0);
  std::vector<size_t> qkv_at(L), gu_at(L), out_at(L), down_at(L), n1_at(L), n2_at(L);
  for (int l = 0; l < L; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    n1_at[l] = region(1, d);
    n2_at[l] = region(1, d);
    qkv_at[l] = region(3 * (size_t)d, d);
    out_at[l] = region(d, d);
    gu_at[l] = region(2 * (size_t)F, d);
    down_at[l] = region(d, F);
    slot(p + "norm1", n1_at[l], 1, d, kPlain, 1, 0);
    slot(p + "norm2", n2_at[l], 1, d, kPlain, 1, 0);
    slot(p + "q", qkv_at[l], d, d, kQkvHead, 0, hd);
    slot(p + "k", qkv_at[l], d, d, kQkvHead, 1, hd);
    slot(p + "v", qkv_at[l], d, d, kQkvHead, 2, hd);
    slot(p + "out", out_at[l], d, d, kOutHead, 0, hd);
    slot(p + "gate", gu_at[l], F, d, kPlain, 2, 0);
    slot(p + "up", gu_at[l], F, d, kPlain, 2, 1);
    slot(p + "down", down_at[l], d, F, kTranspose, 0, 0);
  }
  rt->have.assign(index, 0);
  rt->weights_bytes = off;
  if (rt->cuda(cudaMalloc(&rt->weights, off), "cudaMalloc weights") != ST_OK) return bail(ST_ERR_CUDA);

  // ---- state
  const size_t S = m.streams;
  rt->kv_bytes_per_tensor = S * L * (size_t)d * m.window * rt->elem;
  const size_t kv_at = 0;
  size_t so = align_up(rt->kv_bytes_per_tensor, 256) * 2;
  const size_t hidden_at = so;
  so = align_up(so + S * L * d * sizeof(float), 256);
  const size_t pos_at = so;
  so = align_up(so + S * sizeof(unsigned long long), 256);
  rt->state_bytes = so;
  if (rt->cuda(cudaMalloc(&rt->state, so), "cudaMalloc state") != ST_OK) return bail(ST_ERR_CUDA);
  if (rt->cuda(cudaMemsetAsync(rt->state, 0, so, rt->stream), "cudaMemset state") != ST_OK) return bail(ST_ERR_CUDA);

  // ---- scratch
  const int nch = (m.window + kAttChunk - 1) / kAttChunk;
  size_t co = 0;
  auto take = [&](size_t bytes) { const size_t at = co; co = align_up(co + bytes, 256); return at; };
  const size_t x_at = take(S * d * 4), x2_at = take(S * d * 4), q_at = take(S * d * 4);
  const size_t part_at = take(S * m.heads * (size_t)nch * (hd + 2) * 4);
  const size_t act_at = take(S * F * 4), score_at = take(S * 4), input_at = take(S * m.features * 4);
  const size_t pout_at = take(S * m.heads * (size_t)d * 4), dpart_at = take(S * (size_t)rt->nclusters * d * 4);
  // batched round: selection, grid (one CTA per SM) and K-splits. On the
  // tensor cores (d and F multiples of 64; fp32 as 3xTF32; ST_TC=0 disables) a
  // GEMM unit is a 128-row tile x K split x up to 256 streams, and each phase
  // gets at most one unit per CTA. On the CUDA cores a unit is 64 rows x 32
  // streams, about one per warp, with at most 16 splits. Splits never exceed
  // one per 64 columns, and partials stay within 64 MB.
  {
    const char* env = std::getenv("ST_BATCHED");
    bool want = S >= 4;
    if (env && env[0] == '0') want = false;
    if (env && env[0] == '1') want = true;
    rt->batched = want && S >= 2 && batch_supported(d, m.heads, F, m.features);
    const char* tenv = std::getenv("ST_TC");
    rt->tc = rt->batched && d % kTileK == 0 && F % kTileK == 0 && !(tenv && tenv[0] == '0');
  }
  const size_t spad = (S + 15) / 16 * 16;
  size_t bpart_floats = 0;
  if (rt->batched) {
    rt->bgrid = rt->sms;
    const size_t nmax = std::min<size_t>(spad, kTcMaxN);
    if (rt->tc) {
      // a stage: the A tile and the B tile of one chunk (fp32: hi and lo of each)
      const size_t planes = m.mode == ST_MODE_FP32 ? 2 : 1;
      const size_t stage = planes * (kTcTileBytes + nmax * kCoreBytes);
      const int stages = (int)std::min<size_t>(kTcMaxStages, ((size_t)192 << 10) / stage);
      rt->args.tc_stages = stages;
      rt->args.tc_stage_bytes = (unsigned)stage;
      rt->tc_smem = (size_t)stages * stage;
      unsigned ncols = 32;
      while (ncols < nmax) ncols *= 2;
      if (m.mode == ST_MODE_FP32) ncols = 2 * kTcMaxN;  // fp32: main and correction accumulators
      rt->args.tc_ncols = ncols;
      if (rt->cuda(cudaFuncSetAttribute(rounds_fn(rt), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rt->tc_smem),
                   "cudaFuncSetAttribute rounds") != ST_OK)
        return bail(ST_ERR_CUDA);
    }
    // Staged attention: per warp, a ring of K/V stages in the round's dynamic
    // shared memory behind the q/k/v table of the CTA's units -- the largest
    // dynamic allocation the kernel takes beside its static shared memory
    // (the tensor-core GEMM stages reuse the same bytes). C ring slots per
    // stage (a power of two <= 16): the largest C that leaves at least 4
    // stages per warp, else 2 (more stages keep more bytes in flight). At
    // head_dim 64, when the CTA's q table fits the static union, the chunk is
    // fixed by the storage type (16 slots of 16-bit rows, 8 of fp32: 4 KB) and
    // the dynamic memory holds stages only. ST_ATT_STAGE=0 selects the
    // direct-load attention phase.
    {
      const char* aenv = std::getenv("ST_ATT_STAGE");
      cudaFuncAttributes fa{};
      int optin = 0;
      if (rt->cuda(cudaFuncGetAttributes(&fa, rounds_fn(rt)), "cudaFuncGetAttributes rounds") != ST_OK ||
          rt->cuda(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, rt->device),
                   "cudaDeviceGetAttribute smem") != ST_OK)
        return bail(ST_ERR_CUDA);
      const size_t dyn = (size_t)optin > fa.sharedSizeBytes ? ((size_t)optin - fa.sharedSizeBytes) / 1024 * 1024 : 0;
      const int mine = (int)((S * (size_t)m.heads + (size_t)rt->bgrid - 1) / (size_t)rt->bgrid);
      unsigned table = att_table_bytes(mine, hd);
      int chunk = 0, nb = 0;
      bool hd64 = false;
      if (hd == 64 && att64_table_bytes(mine) <= sizeof(BatchSmem::u)) {
        // the head-dim-64 phase: q table in the static union, 4 KB stages of 16
        // 16-bit or 8 fp32 slots, as many as fit (>= 2)
        const size_t fit = dyn / ((size_t)kWarps * 4096u);
        if (fit >= 2) {
          chunk = rt->elem == 2 ? 16 : 8;
          nb = (int)std::min<size_t>(fit, kAttMaxStages);
          table = 0;
          hd64 = true;
        }
      }
      for (int want = 4; want >= 2 && !chunk; want -= 2)
        for (int c = kAttMaxChunk; c >= 1 && !chunk; c /= 2) {
          const size_t stage = 2ull * (size_t)c * (size_t)hd * (size_t)rt->elem;
          const size_t fit = dyn > table ? (dyn - table) / ((size_t)kWarps * stage) : 0;
          if (fit >= (size_t)want) {
            chunk = c;
            nb = (int)std::min<size_t>(fit, kAttMaxStages);
          }
        }
      if (chunk && !(aenv && aenv[0] == '0')) {
        const unsigned stage = 2u * (unsigned)chunk * (unsigned)hd * (unsigned)rt->elem;
        rt->args.att_chunk = chunk;
        rt->args.att_stages = nb;
        rt->args.att_buf_bytes = stage;
        rt->args.att_table_bytes = table;
        rt->args.att_hd64 = hd64 ? 1 : 0;
        rt->tc_smem = std::max(rt->tc_smem, (size_t)table + (size_t)kWarps * nb * stage);
        if (rt->cuda(cudaFuncSetAttribute(rounds_fn(rt), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rt->tc_smem),
                     "cudaFuncSetAttribute rounds") != ST_OK)
          return bail(ST_ERR_CUDA);
      }
    }
    int occ = 0;
    if (rt->cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, rounds_fn(rt), kThreads, rt->tc_smem),
                 "cudaOccupancyMaxActiveBlocksPerMultiprocessor") != ST_OK)
      return bail(ST_ERR_CUDA);
    if (occ < 1) {
      rt->fail(ST_ERR_UNSUPPORTED, "batched round kernel does not fit on an SM");
      return bail(ST_ERR_UNSUPPORTED);
    }
    // Tensor cores: per GEMM, the streams per unit (MMA N: 256, 128 or 64) and
    // the K-split that minimise (waves of units over the grid) x (bytes one unit
    // moves: its chunks' A and B tiles plus its partial store), plus the
    // partials' share per CTA. CUDA cores: about one unit per warp.
    // ST_TC_N forces N.
    const char* nenv = std::getenv("ST_TC_N");
    const size_t planes = m.mode == ST_MODE_FP32 ? 2 : 1;  // tf32 hi and lo
    const size_t kk = m.mode == ST_MODE_FP32 ? kTileK32 : kTileK;
    auto pick = [&](size_t M, size_t K, int which) {
      size_t best_ks = 1;
      if (rt->tc) {
        const size_t mt = (M + kUmmaM - 1) / kUmmaM, kch = K / kk;
        double best = 1e300;
        size_t best_n = kTcMaxN;
        for (size_t n = std::min<size_t>(spad, kTcMaxN); n >= 16; n /= 2) {
          if (n % 16 || (nenv && (size_t)std::atoi(nenv) != n)) {
            if (n < 64) break;
            continue;
          }
          const size_t sg = (spad + n - 1) / n;
          // 16-bit gate/up: no K-split, so its epilogue can compute SwiGLU (one
          // phase and one grid barrier per layer less). fp32 (3xTF32): at most
          // 512 columns, 64 MMAs, per accumulator: the tensor core's
          // accumulation of longer runs missed the fp32 bound on B200
          // (1.2e-5 on one key element at C5-A).
          const size_t ks_min = planes == 2 ? std::max<size_t>(1, K / 512) : 1;
          const size_t ks_max = which == 2 && planes == 1 ? 1 : std::min(K / 64, (size_t)16);
          for (size_t ks = ks_min; ks <= ks_max; ++ks) {
            if (ks > 1 && ks * S * M * 4 > ((size_t)64 << 20)) break;
            const size_t units = mt * sg * ks, waves = (units + rt->bgrid - 1) / rt->bgrid;
            const size_t chunks = (kch + ks - 1) / ks;
            const double unit_bytes = (double)chunks * planes * (kTcTileBytes + n * kCoreBytes) + 512.0 * n;
            const double part = 0.5 * (double)(ks * S * M * 8) / (double)rt->bgrid;
            const double cost = (double)waves * unit_bytes + part;
            if (cost < best) {
              best = cost;
              best_ks = ks;
              best_n = n;
            }
          }
          if (n <= 64) break;
        }
        rt->tcn[which] = (int)best_n;
      } else {
        const size_t units1 = ((M + kBatchRows - 1) / kBatchRows) * ((S + kBatchStreams - 1) / kBatchStreams);
        const size_t target = (size_t)rt->bgrid * kWarps;
        best_ks = (target + units1 - 1) / units1;
        best_ks = std::min(best_ks, std::min(K / 64, (size_t)16));
        while (best_ks > 1 && best_ks * S * M * 4 > ((size_t)64 << 20)) --best_ks;
        best_ks = std::max(best_ks, (size_t)1);
      }
      bpart_floats = std::max(bpart_floats, best_ks * S * M);
      return (int)best_ks;
    };
    rt->bsplit[0] = pick(3 * (size_t)d, d, 0);
    rt->bsplit[1] = pick(d, d, 1);
    rt->bsplit[2] = pick(2 * (size_t)F, d, 2);
    rt->bsplit[3] = pick(d, F, 3);
  }
  const size_t bx_at = take(rt->batched ? S * d * 4 : 0), bx2_at = take(rt->batched ? S * d * 4 : 0);
  const size_t bz_at = take(rt->batched && !rt->tc ? S * (size_t)std::max(d, F) * 4 : 0), bpart_at = take(bpart_floats * 4);
  // the tensor cores' tiled input: storage type, or tf32 hi and lo planes for fp32
  const size_t bz16_at = take(rt->tc ? spad * (size_t)std::max(d, F) * (m.mode == ST_MODE_FP32 ? 8 : 2) : 0);
  const size_t bzact_at = take(rt->tc ? spad * (size_t)F * (m.mode == ST_MODE_FP32 ? 8 : 2) : 0);
  const size_t bar_at = take(sizeof(unsigned long long)), err_at = take(sizeof(int));
  const size_t rope_at = take((hd / 2) * sizeof(float)), ctl_at = take(sizeof(Control));
  // flow kernel: choose it and its cluster shape (largest cluster whose
  // co-resident count still gives every head its own cluster).
  {
    const char* env = std::getenv("ST_FLOW");
    const int mode_index = m.mode == ST_MODE_FP16 ? 1 : m.mode == ST_MODE_BF16 ? 2 : 0;
    rt->flow_fn = flow_kernel(mode_index, d, false);
    rt->flow_diag_fn = flow_kernel(mode_index, d, true);
    const bool want = rt->flow_fn && S == 1 && hd == kFlowHd && m.features == kFlowFeatures && o.blocks == 0 &&
                      !rt->batched && coop && !(env && env[0] == '0');
    if (want) {
      if (rt->cuda(cudaFuncSetAttribute(rt->flow_fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)flow_smem_bytes()), "cudaFuncSetAttribute flow") != ST_OK ||
          rt->cuda(cudaFuncSetAttribute(rt->flow_diag_fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)flow_smem_bytes()), "cudaFuncSetAttribute flow") != ST_OK)
        return bail(ST_ERR_CUDA);
      int best_cs = 0, best_nc = 0;
      // ST_FLOW_CLUSTER=2/4/8 forces the cluster size (tuning).
      const char* cenv = std::getenv("ST_FLOW_CLUSTER");
      const int forced = cenv ? std::atoi(cenv) : 0;
      for (int cs : {8, 4, 2}) {
        if (forced ? cs != forced : cs == 2) continue;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(cs);
        cfg.blockDim = dim3(flow_threads());
        cfg.dynamicSmemBytes = flow_smem_bytes();
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = cs;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int nmax = 0;
        if (rt->cuda(cudaOccupancyMaxActiveClusters(&nmax, rt->flow_fn, &cfg), "cudaOccupancyMaxActiveClusters flow") != ST_OK)
          return bail(ST_ERR_CUDA);
        const int nc = std::min(nmax, rt->sms / cs);
        if (nc < 1) continue;
        const int local_heads = m.heads / tp_size;
        if (best_cs == 0 || (best_nc < local_heads && nc >= local_heads)) {
          best_cs = cs;
          best_nc = nc;
        }
        if (best_nc >= local_heads) break;
      }
      if (best_cs > 0) {
        rt->flow = true;
        rt->fcluster = best_cs;
        rt->fnclusters = best_nc;
        rt->fgrid = best_cs * best_nc;
      }
    }
  }
  if (tp_size > 1 && !rt->flow) {
    rt->fail(ST_ERR_UNSUPPORTED, "tensor parallelism needs the single-stream kernel's shapes (head_dim 64, 32 "
                                 "features, width 256/512/1024, blocks 0)");
    return bail(ST_ERR_UNSUPPORTED);
  }
  const size_t llh_at = take(rt->flow ? 2 * (size_t)m.heads * d * 8 : 0);
  const size_t llx_at = take(tp_size > 1 ? 2 * (size_t)tp_size * d * 8 : 0);
  rt->llh_at = llh_at;
  rt->llx_at = llx_at;
  const size_t llc_at = take(rt->flow ? 2 * (size_t)rt->fnclusters * d * 8 : 0);
  const size_t fwords_at = take(3 * sizeof(unsigned long long));
  rt->scratch_bytes = co;
  if (rt->cuda(cudaMalloc(&rt->scratch, co), "cudaMalloc scratch") != ST_OK) return bail(ST_ERR_CUDA);
  if (rt->cuda(cudaMemsetAsync(rt->scratch, 0, co, rt->stream), "cudaMemset scratch") != ST_OK) return bail(ST_ERR_CUDA);
  std::vector<float> freq(hd / 2);
  for (int i = 0; i < hd; i += 2) freq[i / 2] = powf(10000.0f, -(float)i / (float)hd);
  if (rt->cuda(cudaMemcpyAsync(rt->scratch + rope_at, freq.data(), freq.size() * 4, cudaMemcpyHostToDevice, rt->stream),
               "rope table") != ST_OK ||
      rt->cuda(cudaStreamSynchronize(rt->stream), "rope table") != ST_OK)
    return bail(ST_ERR_CUDA);

  // ---- mapped pinned memory
  void* hp = nullptr;
  if (rt->cuda(cudaHostAlloc(&hp, sizeof(Mailbox), cudaHostAllocMapped), "cudaHostAlloc mailbox") != ST_OK) return bail(ST_ERR_CUDA);
  rt->mb_h = (Mailbox*)hp;
  std::memset(hp, 0, sizeof(Mailbox));
  if (rt->cuda(cudaHostGetDevicePointer((void**)&rt->mb_d, hp, 0), "mailbox alias") != ST_OK) return bail(ST_ERR_CUDA);
  if (rt->cuda(cudaHostAlloc(&hp, S * m.features * 4, cudaHostAllocMapped), "cudaHostAlloc input") != ST_OK) return bail(ST_ERR_CUDA);
  rt->in_h = (float*)hp;
  std::memset(hp, 0, S * m.features * 4);
  if (rt->cuda(cudaHostGetDevicePointer((void**)&rt->in_d, hp, 0), "input alias") != ST_OK) return bail(ST_ERR_CUDA);
  if (rt->cuda(cudaHostAlloc(&hp, S * 4, cudaHostAllocMapped), "cudaHostAlloc output") != ST_OK) return bail(ST_ERR_CUDA);
  rt->out_h = (float*)hp;
  std::memset(hp, 0, S * 4);
  if (rt->cuda(cudaHostGetDevicePointer((void**)&rt->out_d, hp, 0), "output alias") != ST_OK) return bail(ST_ERR_CUDA);

  // ---- step arguments
  StepArgs& a = rt->args;
  a.layers = L; a.width = d; a.heads = m.heads; a.ffn = F; a.window = m.window; a.features = m.features;
  a.head_dim = hd; a.streams = (int)S; a.epsilon = m.epsilon; a.nchunks_max = nch;
  a.input_w = rt->weights + rt->slots["input"].offset;
  a.final_norm = rt->weights + rt->slots["final_norm"].offset;
  a.score_w = rt->weights + rt->slots["score"].offset;
  for (int l = 0; l < L; ++l) {
    a.layer[l].norm1 = rt->weights + n1_at[l];
    a.layer[l].norm2 = rt->weights + n2_at[l];
    a.layer[l].qkv = rt->weights + qkv_at[l];
    a.layer[l].out = rt->weights + out_at[l];
    a.layer[l].gateup = rt->weights + gu_at[l];
    a.layer[l].down = rt->weights + down_at[l];
  }
  a.rope_freq = (const float*)(rt->scratch + rope_at);
  a.keys = rt->state + kv_at;
  a.values = rt->state + kv_at + align_up(rt->kv_bytes_per_tensor, 256);
  a.hidden = (float*)(rt->state + hidden_at);
  a.position = (unsigned long long*)(rt->state + pos_at);
  rt->dev_input = (float*)(rt->scratch + input_at);
  rt->dev_score = (float*)(rt->scratch + score_at);
  a.input = o.mapped ? rt->in_d : rt->dev_input;
  a.score = o.mapped ? rt->out_d : rt->dev_score;
  a.x = (float*)(rt->scratch + x_at);
  a.x2 = (float*)(rt->scratch + x2_at);
  a.q = (float*)(rt->scratch + q_at);
  a.part = (float*)(rt->scratch + part_at);
  a.act = (float*)(rt->scratch + act_at);
  a.pout = (float*)(rt->scratch + pout_at);
  a.dpart = (float*)(rt->scratch + dpart_at);
  a.bar_counter = (unsigned long long*)(rt->scratch + bar_at);
  a.error = (int*)(rt->scratch + err_at);
  a.host_error = &rt->mb_d->error;
  // Bound on any single device-side wait. ST_DEVICE_TIMEOUT_MS shortens it
  // and ST_TEST_DROP_RECORD=<cta> makes that CTA of the single-stream kernel
  // withhold one exchange record: the failure-path test of the bounded waits
  // (a flag nothing sets, no fault), which must end in ST_ERR_DEVICE_TIMEOUT.
  a.bar_timeout_ns = 2ull * 1000000000ull;
  if (const char* env = std::getenv("ST_DEVICE_TIMEOUT_MS"))
    a.bar_timeout_ns = (unsigned long long)std::max(1, std::atoi(env)) * 1000000ull;
  a.test_drop_cta = -1;
  if (const char* env = std::getenv("ST_TEST_DROP_RECORD")) a.test_drop_cta = std::atoi(env);
  a.cluster_size = rt->cluster;
  a.clusters = rt->nclusters;
  if (rt->batched) {
    a.bx = (float*)(rt->scratch + bx_at);
    a.bx2 = (float*)(rt->scratch + bx2_at);
    a.bz = (float*)(rt->scratch + bz_at);
    a.bpart = (float*)(rt->scratch + bpart_at);
    for (int i = 0; i < 4; ++i) {
      a.bsplit[i] = rt->bsplit[i];
      a.tc_n[i] = rt->tcn[i];
    }
    a.spad = (int)spad;
  }
  if (rt->tc) {
    // The tensor-core copy of the layer matrices, rows padded to 128 (zeros).
    a.bz16 = rt->scratch + bz16_at;
    a.bz16_act = rt->scratch + bzact_at;
    a.fuse_swiglu = rt->bsplit[2] == 1 && m.mode != ST_MODE_FP32 ? 1 : 0;
    auto pad = [](size_t rows) { return (rows + kUmmaM - 1) / kUmmaM * kUmmaM; };
    size_t to = 0;
    const size_t tbytes = m.mode == ST_MODE_FP32 ? 8 : 2;  // fp32: tf32 hi and lo planes
    auto matrix = [&](size_t rows, size_t cols) {
      const size_t at = to;
      to = align_up(to + pad(rows) * cols * tbytes, 256);
      return at;
    };
    std::vector<size_t> tq(L), tout(L), tgu(L), tdn(L);
    for (int l = 0; l < L; ++l) {
      tq[l] = matrix(3 * (size_t)d, d);
      tout[l] = matrix(d, d);
      tgu[l] = matrix(2 * (size_t)F, d);
      tdn[l] = matrix(d, F);
    }
    rt->tweights_bytes = to;
    if (rt->cuda(cudaMalloc(&rt->tweights, to), "cudaMalloc tiled weights") != ST_OK ||
        rt->cuda(cudaMemsetAsync(rt->tweights, 0, to, rt->stream), "cudaMemset tiled weights") != ST_OK)
      return bail(ST_ERR_CUDA);
    for (int l = 0; l < L; ++l) {
      a.tqkv[l] = rt->tweights + tq[l];
      a.tout[l] = rt->tweights + tout[l];
      a.tgateup[l] = rt->tweights + tgu[l];
      a.tdown[l] = rt->tweights + tdn[l];
      const std::string p = "layers." + std::to_string(l) + ".";
      auto set = [&](const char* name, size_t at, int rows, int cols) {
        TensorSlot& ts = rt->slots[p + name];
        ts.tiled_offset = at;
        ts.tiled_rows = rows;
        ts.tiled_cols = cols;
      };
      for (const char* n : {"q", "k", "v"}) set(n, tq[l], 3 * d, d);
      set("out", tout[l], d, d);
      set("gate", tgu[l], 2 * F, d);
      set("up", tgu[l], 2 * F, d);
      set("down", tdn[l], d, F);
    }
  }
  {
    // Keep as many whole layers L2-resident as fit in 70% of L2 (the rest holds
    // the K/V cache, activations and code); ST_L2_KEEP_LAYERS overrides.
    const size_t dd = (size_t)m.width, ff = (size_t)m.ffn;
    const size_t per_layer = (2 * dd + 4 * dd * dd + 3 * ff * dd) * rt->elem;
    int keep = per_layer ? (int)std::min<size_t>(L, (size_t)(0.7 * (double)prop.l2CacheSize) / per_layer) : 0;
    if (const char* env = std::getenv("ST_L2_KEEP_LAYERS")) keep = std::max(0, std::min(L, std::atoi(env)));
    a.l2_keep_layers = keep;
  }
  {
    const char* env = std::getenv("ST_WEIGHT_RING");
    rt->ring = ring_supported(a, rt->elem, rt->cluster, rt->nclusters) && !(env && env[0] == '0');
  }
  rt->control = (Control*)(rt->scratch + ctl_at);
  a.ll_heads = (unsigned long long*)(rt->scratch + llh_at);
  a.ll_clusters = (unsigned long long*)(rt->scratch + llc_at);
  a.tp_rank = tp_rank;
  a.tp_size = tp_size;
  a.ll_xd = (unsigned long long*)(rt->scratch + llx_at);
  a.ll_heads_peer[tp_rank] = a.ll_heads;  // peers' entries arrive with st_tp_connect
  a.ll_xd_peer[tp_rank] = a.ll_xd;
  a.flow_epoch = (unsigned long long*)(rt->scratch + fwords_at);
  a.flow_ctl = a.flow_epoch + 1;
  a.flow_seq = a.flow_epoch + 2;
  if (rt->flow && !flow_shape_ok(a, rt->elem, rt->fcluster, rt->fnclusters)) rt->flow = false;
  *out = rt;
  return ST_OK;
}

int st_set_tensor(st_runtime* rt, const char* name, const float* data, size_t count) {
  if (!rt || !name || !data) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (rt->started) return rt->fail(ST_ERR_STATE, "tensors are fixed once the runtime has started");
  auto it = rt->slots.find(name);
  if (it == rt->slots.end()) return rt->fail(ST_ERR_INVALID, "Unknown tensor %s", name);
  const TensorSlot& s = it->second;
  if (count != (size_t)s.rows * s.cols) return rt->fail(ST_ERR_INVALID, "Shape mismatch: %s", name);
  float* tmp = nullptr;
  ST_CUDA(rt, cudaMalloc(&tmp, count * sizeof(float)));
  // Stream-ordered: a pageable cudaMemcpy may return before its DMA lands, and
  // the non-blocking stream is not ordered after the legacy stream.
  int st = rt->cuda(cudaMemcpyAsync(tmp, data, count * sizeof(float), cudaMemcpyHostToDevice, rt->stream), "tensor upload");
  if (st == ST_OK) {
    const int blocks = (int)std::min<size_t>((count + 255) / 256, 4096);
    void* dst = rt->weights + s.offset;
    if (rt->desc.mode == ST_MODE_FP16) k_convert<__half><<<blocks, 256, 0, rt->stream>>>(tmp, (__half*)dst, s.rows, s.cols, s.kind, s.p0, s.p1);
    else if (rt->desc.mode == ST_MODE_BF16) k_convert<__nv_bfloat16><<<blocks, 256, 0, rt->stream>>>(tmp, (__nv_bfloat16*)dst, s.rows, s.cols, s.kind, s.p0, s.p1);
    else k_convert<float><<<blocks, 256, 0, rt->stream>>>(tmp, (float*)dst, s.rows, s.cols, s.kind, s.p0, s.p1);
    if (rt->tc && s.tiled_rows) {
      void* tdst = rt->tweights + s.tiled_offset;
      const size_t lo = (size_t)(s.tiled_rows + kUmmaM - 1) / kUmmaM * kUmmaM * (size_t)s.tiled_cols;
      if (rt->desc.mode == ST_MODE_FP16)
        k_convert_tiled<__half><<<blocks, 256, 0, rt->stream>>>(tmp, (__half*)tdst, s.rows, s.cols, s.kind, s.p0, s.p1, s.tiled_cols, lo);
      else if (rt->desc.mode == ST_MODE_BF16)
        k_convert_tiled<__nv_bfloat16><<<blocks, 256, 0, rt->stream>>>(tmp, (__nv_bfloat16*)tdst, s.rows, s.cols, s.kind, s.p0, s.p1, s.tiled_cols, lo);
      else
        k_convert_tiled<float><<<blocks, 256, 0, rt->stream>>>(tmp, (float*)tdst, s.rows, s.cols, s.kind, s.p0, s.p1, s.tiled_cols, lo);
    }
    st = rt->cuda(cudaGetLastError(), "convert launch");
    if (st == ST_OK) st = rt->cuda(cudaStreamSynchronize(rt->stream), "convert");
  }
  cudaFree(tmp);
  if (st == ST_OK) rt->have[s.index] = 1;
  return st;
}

int st_start(st_runtime* rt) {
  if (!rt) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (rt->started) return rt->fail(ST_ERR_STATE, "runtime already started");
  for (const auto& kv : rt->slots)
    if (!rt->have[kv.second.index]) return rt->fail(ST_ERR_INVALID, "Missing tensor %s", kv.first.c_str());
  for (int g = 0; g < rt->tp_size; ++g)
    if (!rt->args.ll_heads_peer[g] || !rt->args.ll_xd_peer[g])
      return rt->fail(ST_ERR_STATE, "tensor-parallel GPU %d is not connected (st_tp_connect)", g);
  ST_CUDA(rt, cudaSetDevice(rt->device));
  ST_TRY(preload(rt));
  // Warm every kernel once (lazy module loading), then restore the initial state.
  if (rt->opt.backend != ST_BACKEND_PERSISTENT) {
    // (a tensor-parallel stream runs only the sharded single-stream kernel;
    // its warm-up step is collective: every GPU of the stream takes it)
    if (rt->tp_size == 1) ST_TRY(launch_sequence(rt, rt->args));
    if (rt->opt.backend == ST_BACKEND_FUSED) ST_TRY(launch_fused(rt, rt->args));
  }
  ST_TRY(launch_reset(rt, 0, rt->desc.streams));
  ST_CUDA(rt, cudaStreamSynchronize(rt->stream));
  ST_TRY(check_device_error(rt));
  if (rt->opt.backend == ST_BACKEND_GRAPH) ST_TRY(graph_capture(rt));
  rt->started = true;
  if (rt->opt.backend == ST_BACKEND_PERSISTENT) ST_TRY(start_persistent(rt));
  return ST_OK;
}

static int step_common(st_runtime* rt, const float* inputs, float* scores) {
  if (!rt || !inputs || !scores) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (!rt->started) return rt->fail(ST_ERR_STATE, "st_start has not been called");
  const size_t n = (size_t)rt->desc.streams * rt->desc.features;
  if (rt->opt.backend == ST_BACKEND_PERSISTENT) {
    if (!rt->running) return rt->fail(ST_ERR_STOPPED, "Persistent runtime is stopped");
    std::memcpy(rt->in_h, inputs, n * sizeof(float));
    ST_TRY(command(rt, kRun, -1));
  } else {
    std::memcpy(rt->in_h, inputs, n * sizeof(float));
    ST_TRY(run_step_nonpersistent(rt));
  }
  std::memcpy(scores, rt->out_h, (size_t)rt->desc.streams * sizeof(float));
  return ST_OK;
}

int st_step(st_runtime* rt, const float* input, float* score) {
  if (rt && rt->desc.streams != 1) return rt->fail(ST_ERR_INVALID, "st_step needs streams == 1; use st_step_batch");
  return step_common(rt, input, score);
}

int st_step_batch(st_runtime* rt, const float* inputs, float* scores) { return step_common(rt, inputs, scores); }

int st_reset_stream(st_runtime* rt, int stream) {
  if (!rt) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (!rt->started) return rt->fail(ST_ERR_STATE, "st_start has not been called");
  if (stream < -1 || stream >= rt->desc.streams) return rt->fail(ST_ERR_INVALID, "stream index out of range");
  if (rt->opt.backend == ST_BACKEND_PERSISTENT) return command(rt, kReset, stream);
  const int s0 = stream < 0 ? 0 : stream, s1 = stream < 0 ? rt->desc.streams : stream + 1;
  ST_TRY(launch_reset(rt, s0, s1));
  ST_CUDA(rt, cudaStreamSynchronize(rt->stream));
  return check_device_error(rt);
}

int st_reset(st_runtime* rt) { return st_reset_stream(rt, -1); }

int st_stop(st_runtime* rt) {
  if (!rt) return ST_ERR_INVALID;
  if (rt->running) {
    if (!__atomic_load_n(&rt->mb_h->exited, __ATOMIC_ACQUIRE)) {
      int st = command(rt, kStop, -1);
      if (st != ST_OK && st != ST_ERR_WORKER_EXITED) return st;
    }
    if (rt->running) ST_TRY(join_persistent(rt));
  }
  return ST_OK;
}

int st_resume(st_runtime* rt) {
  if (!rt) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (!rt->started) return rt->fail(ST_ERR_STATE, "st_start has not been called");
  if (rt->opt.backend != ST_BACKEND_PERSISTENT || rt->running) return ST_OK;
  return start_persistent(rt);
}

int st_snapshot(st_runtime* rt, int stream, uint64_t* position, float* keys, float* values, float* hidden) {
  if (!rt) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (stream < 0 || stream >= rt->desc.streams) return rt->fail(ST_ERR_INVALID, "stream index out of range");
  const st_model_desc& m = rt->desc;
  const size_t cache = (size_t)m.layers * m.width * m.window;
  cudaStream_t s = rt->aux;
  if (position) {
    unsigned long long p = 0;
    ST_CUDA(rt, cudaMemcpyAsync(&p, rt->args.position + stream, sizeof p, cudaMemcpyDeviceToHost, s));
    ST_CUDA(rt, cudaStreamSynchronize(s));
    *position = p;
  }
  auto download = [&](const void* base, float* dst) -> int {
    if (!dst) return ST_OK;
    const char* src = (const char*)base + (size_t)stream * cache * rt->elem;
    if (m.mode == ST_MODE_FP32) {
      ST_CUDA(rt, cudaMemcpyAsync(dst, src, cache * 4, cudaMemcpyDeviceToHost, s));
      ST_CUDA(rt, cudaStreamSynchronize(s));
      return ST_OK;
    }
    std::vector<uint16_t> raw(cache);
    ST_CUDA(rt, cudaMemcpyAsync(raw.data(), src, cache * 2, cudaMemcpyDeviceToHost, s));
    ST_CUDA(rt, cudaStreamSynchronize(s));
    for (size_t i = 0; i < cache; ++i)
      dst[i] = m.mode == ST_MODE_FP16 ? half_bits_to_float(raw[i]) : bf16_bits_to_float(raw[i]);
    return ST_OK;
  };
  ST_TRY(download(rt->args.keys, keys));
  ST_TRY(download(rt->args.values, values));
  if (hidden) {
    const size_t n = (size_t)m.layers * m.width;
    ST_CUDA(rt, cudaMemcpyAsync(hidden, rt->args.hidden + (size_t)stream * n, n * 4, cudaMemcpyDeviceToHost, s));
    ST_CUDA(rt, cudaStreamSynchronize(s));
  }
  return ST_OK;
}

// What one GPU of a tensor-parallel stream tells the others: the layout it was
// built with (which must match theirs) and the IPC handle of the allocation
// holding its record buffers.
struct TpBlob {
  unsigned long long magic;
  int tp_rank, tp_size, heads, width, clusters, pad;
  unsigned long long scratch_bytes, llh_at, llx_at;
  cudaIpcMemHandle_t handle;
};
constexpr unsigned long long kTpMagic = 0x7374747062303031ull;

int st_tp_handle(st_runtime* rt, void* blob, size_t capacity, size_t* needed) {
  if (!rt) return ST_ERR_INVALID;
  if (needed) *needed = sizeof(TpBlob);
  if (!blob || capacity < sizeof(TpBlob)) return rt->fail(ST_ERR_INVALID, "handle buffer smaller than %zu bytes", sizeof(TpBlob));
  TpBlob b{};
  b.magic = kTpMagic;
  b.tp_rank = rt->tp_rank;
  b.tp_size = rt->tp_size;
  b.heads = rt->desc.heads;
  b.width = rt->desc.width;
  b.clusters = rt->fnclusters;
  b.scratch_bytes = rt->scratch_bytes;
  b.llh_at = rt->llh_at;
  b.llx_at = rt->llx_at;
  ST_CUDA(rt, cudaSetDevice(rt->device));
  ST_CUDA(rt, cudaIpcGetMemHandle(&b.handle, rt->scratch));
  std::memcpy(blob, &b, sizeof b);
  return ST_OK;
}

int st_tp_connect(st_runtime* rt, const void* blobs, size_t count) {
  if (!rt || !blobs) return ST_ERR_INVALID;
  if (rt->started) return rt->fail(ST_ERR_STATE, "connect the tensor-parallel GPUs before st_start");
  if ((int)count != rt->tp_size) return rt->fail(ST_ERR_INVALID, "expected %d handles, got %zu", rt->tp_size, count);
  ST_CUDA(rt, cudaSetDevice(rt->device));
  const TpBlob* all = static_cast<const TpBlob*>(blobs);
  for (int g = 0; g < rt->tp_size; ++g) {
    const TpBlob& b = all[g];
    if (b.magic != kTpMagic || b.tp_rank != g || b.tp_size != rt->tp_size || b.heads != rt->desc.heads ||
        b.width != rt->desc.width || b.clusters != rt->fnclusters || b.scratch_bytes != rt->scratch_bytes ||
        b.llh_at != rt->llh_at || b.llx_at != rt->llx_at)
      return rt->fail(ST_ERR_INVALID, "tensor-parallel GPU %d was built with another layout", g);
    if (g == rt->tp_rank) continue;
    void* base = nullptr;
    ST_CUDA(rt, cudaIpcOpenMemHandle(&base, b.handle, cudaIpcMemLazyEnablePeerAccess));
    rt->tp_peer_base[g] = static_cast<char*>(base);
    rt->args.ll_heads_peer[g] = reinterpret_cast<unsigned long long*>(rt->tp_peer_base[g] + b.llh_at);
    rt->args.ll_xd_peer[g] = reinterpret_cast<unsigned long long*>(rt->tp_peer_base[g] + b.llx_at);
  }
  return ST_OK;
}

int st_load_state(st_runtime* rt, int stream, uint64_t position, const float* keys, const float* values,
                  const float* hidden) {
  if (!rt || !keys || !values || !hidden) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (!rt->started) return rt->fail(ST_ERR_STATE, "st_start has not been called");
  if (rt->running) return rt->fail(ST_ERR_STATE, "stop the persistent worker before loading state");
  if (stream < 0 || stream >= rt->desc.streams) return rt->fail(ST_ERR_INVALID, "stream index out of range");
  const st_model_desc& m = rt->desc;
  const size_t cache = (size_t)m.layers * m.width * m.window;
  const int hd = m.width / m.heads;
  float* tmp = nullptr;
  ST_CUDA(rt, cudaMalloc(&tmp, cache * sizeof(float)));
  int st = ST_OK;
  for (int which = 0; which < 2 && st == ST_OK; ++which) {
    const float* src = which == 0 ? keys : values;
    char* base = (char*)(which == 0 ? rt->args.keys : rt->args.values) + (size_t)stream * cache * rt->elem;
    st = rt->cuda(cudaMemcpyAsync(tmp, src, cache * sizeof(float), cudaMemcpyHostToDevice, rt->stream), "state upload");
    if (st != ST_OK) break;
    const int rows = (int)(cache / hd), blocks = (int)std::min<size_t>((cache + 255) / 256, 4096);
    if (m.mode == ST_MODE_FP16) k_convert<__half><<<blocks, 256, 0, rt->stream>>>(tmp, (__half*)base, rows, hd, kPlain, 1, 0);
    else if (m.mode == ST_MODE_BF16) k_convert<__nv_bfloat16><<<blocks, 256, 0, rt->stream>>>(tmp, (__nv_bfloat16*)base, rows, hd, kPlain, 1, 0);
    else k_convert<float><<<blocks, 256, 0, rt->stream>>>(tmp, (float*)base, rows, hd, kPlain, 1, 0);
    st = rt->cuda(cudaGetLastError(), "state convert");
    if (st == ST_OK) st = rt->cuda(cudaStreamSynchronize(rt->stream), "state convert");
  }
  cudaFree(tmp);
  ST_TRY(st);
  const size_t n = (size_t)m.layers * m.width;
  unsigned long long p = position;
  ST_CUDA(rt, cudaMemcpyAsync(rt->args.hidden + (size_t)stream * n, hidden, n * 4, cudaMemcpyHostToDevice, rt->stream));
  ST_CUDA(rt, cudaMemcpyAsync(rt->args.position + stream, &p, sizeof p, cudaMemcpyHostToDevice, rt->stream));
  ST_CUDA(rt, cudaStreamSynchronize(rt->stream));
  return ST_OK;
}

}  // extern "C"

static int trace_step_impl(st_runtime* rt, st_trace_fn fn, void* user) {
  const st_model_desc& m = rt->desc;
  const int d = m.width, F = m.ffn;
  StepArgs a = rt->args;
  float* dbg = nullptr;
  ST_CUDA(rt, cudaMalloc(&dbg, (size_t)(5 * d + F) * sizeof(float)));
  a.trace_qkv = dbg;
  a.trace_attention = dbg + 3 * d;
  a.trace_act = dbg + 4 * d;
  std::vector<float> buf(std::max(3 * d, F));
  auto emit = [&](const std::string& name, const float* dev, int count) -> int {
    ST_CUDA(rt, cudaStreamSynchronize(rt->stream));
    ST_CUDA(rt, cudaMemcpy(buf.data(), dev, count * sizeof(float), cudaMemcpyDeviceToHost));
    fn(user, name.c_str(), buf.data(), (size_t)count);
    return ST_OK;
  };
  auto run = [&]() -> int {
    void* p0[] = {&a};
    ST_TRY(launch_ex(rt, ST_KERNEL(rt, input), rt->grid, rt->cluster, false, p0));
    ST_TRY(emit("input", a.x, d));
    for (int l = 0; l < m.layers; ++l) {
      const std::string p = "layers." + std::to_string(l) + ".";
      void* p1[] = {&a, &l};
      ST_TRY(launch_ex(rt, ST_KERNEL(rt, attention), rt->grid, rt->cluster, false, p1));
      if (l > 0) ST_TRY(emit("layers." + std::to_string(l - 1) + ".hidden", a.hidden + (size_t)(l - 1) * d, d));
      ST_TRY(emit(p + "q", a.trace_qkv, d));
      ST_TRY(emit(p + "k", a.trace_qkv + d, d));
      ST_TRY(emit(p + "v", a.trace_qkv + 2 * d, d));
      ST_TRY(emit(p + "attention", a.trace_attention, d));
      ST_TRY(launch_ex(rt, ST_KERNEL(rt, ffn), rt->grid, rt->cluster, false, p1));
      ST_TRY(emit(p + "attention_residual", a.x2, d));
      ST_TRY(emit(p + "activation", a.trace_act, F));
    }
    int nc = rt->nclusters;
    void* p2[] = {&a, &nc};
    ST_TRY(launch_ex(rt, ST_KERNEL(rt, final_), 1, 1, false, p2));
    ST_TRY(emit("layers." + std::to_string(m.layers - 1) + ".hidden", a.hidden + (size_t)(m.layers - 1) * d, d));
    ST_TRY(emit("score.linear", a.score, 1));
    return ST_OK;
  };
  const int st = run();
  cudaFree(dbg);
  return st;
}

extern "C" {

int st_trace_step(st_runtime* rt, const float* input, float* score, st_trace_fn fn, void* user) {
  if (!rt || !input || !fn) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (!rt->started) return rt->fail(ST_ERR_STATE, "st_start has not been called");
  if (rt->opt.backend != ST_BACKEND_CUDA) return rt->fail(ST_ERR_INVALID, "traceStep requires conventional custom CUDA");
  if (rt->desc.streams != 1) return rt->fail(ST_ERR_INVALID, "traceStep supports one stream");
  const size_t n = (size_t)rt->desc.features;
  std::memcpy(rt->in_h, input, n * sizeof(float));
  if (!rt->opt.mapped)
    ST_CUDA(rt, cudaMemcpyAsync(rt->dev_input, rt->in_h, n * 4, cudaMemcpyHostToDevice, rt->stream));
  ST_TRY(trace_step_impl(rt, fn, user));
  ST_CUDA(rt, cudaStreamSynchronize(rt->stream));
  ST_TRY(check_device_error(rt));
  if (score) {
    float v = 0;
    if (rt->opt.mapped) v = rt->out_h[0];
    else ST_CUDA(rt, cudaMemcpy(&v, rt->dev_score, 4, cudaMemcpyDeviceToHost));
    *score = v;
  }
  return ST_OK;
}

static int device_trace_impl(st_runtime* rt, const float* dev_inputs, size_t count, float* dev_scores,
                             double* us_per_step, bool reset = true) {
  const int S = rt->desc.streams;
  const size_t stride = (size_t)S * rt->desc.features;
  StepArgs a = rt->args;
  a.input = rt->dev_input;
  a.score = rt->dev_score;
  if (reset) ST_TRY(launch_reset(rt, 0, S));
  ST_CUDA(rt, cudaEventRecord(rt->ev_start, rt->stream));
  if (rt->batched) {
    ST_TRY(launch_rounds(rt, a, dev_inputs, count, dev_scores));
  } else if (rt->opt.backend == ST_BACKEND_FUSED || rt->opt.backend == ST_BACKEND_PERSISTENT) {
    ST_TRY(launch_trace(rt, a, dev_inputs, count, dev_scores));
  } else {
    const bool graph = rt->opt.backend == ST_BACKEND_GRAPH && !rt->opt.mapped;
    for (size_t e = 0; e < count; ++e) {
      ST_CUDA(rt, cudaMemcpyAsync(rt->dev_input, dev_inputs + e * stride, stride * 4, cudaMemcpyDeviceToDevice, rt->stream));
      if (graph) {
        ST_CUDA(rt, cudaGraphLaunch(rt->graph_exec, rt->stream));
        rt->launches += sequence_launches(rt);
      } else {
        ST_TRY(launch_sequence(rt, a));
      }
      if (dev_scores)
        ST_CUDA(rt, cudaMemcpyAsync(dev_scores + e * S, rt->dev_score, S * 4, cudaMemcpyDeviceToDevice, rt->stream));
    }
  }
  ST_CUDA(rt, cudaEventRecord(rt->ev_stop, rt->stream));
  ST_CUDA(rt, cudaEventSynchronize(rt->ev_stop));
  ST_TRY(check_device_error(rt));
  float ms = 0;
  ST_CUDA(rt, cudaEventElapsedTime(&ms, rt->ev_start, rt->ev_stop));
  if (us_per_step) *us_per_step = count ? ms * 1000.0 / (double)count : 0.0;
  return ST_OK;
}

int st_device_trace(st_runtime* rt, const float* inputs, size_t count, float* scores, double* us_per_step) {
  if (!rt || !inputs || count == 0) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (!rt->started) return rt->fail(ST_ERR_STATE, "st_start has not been called");
  if (rt->opt.backend == ST_BACKEND_PERSISTENT) ST_TRY(st_stop(rt));
  const int S = rt->desc.streams;
  const size_t n = count * (size_t)S * rt->desc.features;
  float* dev = nullptr;
  float* dev_scores = nullptr;
  ST_CUDA(rt, cudaMalloc(&dev, n * 4));
  int st = rt->cuda(cudaMalloc(&dev_scores, count * (size_t)S * 4), "cudaMalloc scores");
  if (st == ST_OK) st = rt->cuda(cudaMemcpyAsync(dev, inputs, n * 4, cudaMemcpyHostToDevice, rt->stream), "trace upload");
  if (st == ST_OK) st = device_trace_impl(rt, dev, count, dev_scores, us_per_step);
  if (st == ST_OK && scores)
    st = rt->cuda(cudaMemcpyAsync(scores, dev_scores, count * (size_t)S * 4, cudaMemcpyDeviceToHost, rt->stream), "scores download");
  if (st == ST_OK) st = rt->cuda(cudaStreamSynchronize(rt->stream), "scores download");
  cudaFree(dev);
  cudaFree(dev_scores);
  return st;
}

int st_device_timeline(st_runtime* rt, const float* inputs, size_t count, long long* marks, size_t capacity,
                       size_t* used) {
  return st_device_timeline_cta(rt, inputs, count, 0, marks, capacity, used);
}

int st_device_timeline_cta(st_runtime* rt, const float* inputs, size_t count, int cta, long long* marks,
                           size_t capacity, size_t* used) {
  if (!rt || !inputs || !marks || count == 0 || capacity == 0) return ST_ERR_INVALID;
  const int grid = rt->batched ? rt->bgrid : rt->flow ? rt->fgrid : rt->grid;
  // The single-stream kernels record per-phase cycle sums of every CTA
  // (cta -1, marks[cta * 32 + tag]); the others one CTA's clock marks.
  if (rt->flow && !rt->batched) {
    if (cta != -1 || capacity < (size_t)grid * kFlowTags)
      return rt->fail(ST_ERR_INVALID, "the single-stream kernel records per-CTA phase sums: cta -1, capacity >= %d",
                      grid * kFlowTags);
  } else if (cta < 0 || cta >= grid) {
    return rt->fail(ST_ERR_INVALID, "timeline CTA %d outside the grid of %d", cta, grid);
  }
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (!rt->started) return rt->fail(ST_ERR_STATE, "st_start has not been called");
  if (rt->opt.backend == ST_BACKEND_PERSISTENT) ST_TRY(st_stop(rt));
  const size_t n = count * (size_t)rt->desc.streams * rt->desc.features;
  float* dev = nullptr;
  long long* tl = nullptr;
  ST_CUDA(rt, cudaMalloc(&dev, n * 4));
  int st = rt->cuda(cudaMalloc(&tl, capacity * sizeof(long long)), "cudaMalloc timeline");
  if (st == ST_OK) st = rt->cuda(cudaMemsetAsync(tl, 0, capacity * sizeof(long long), rt->stream), "timeline clear");
  if (st == ST_OK) st = rt->cuda(cudaMemcpyAsync(dev, inputs, n * 4, cudaMemcpyHostToDevice, rt->stream), "trace upload");
  if (st == ST_OK) st = launch_reset(rt, 0, rt->desc.streams);
  if (st == ST_OK) {
    StepArgs a = rt->args;
    a.input = rt->dev_input;
    a.score = rt->dev_score;
    a.timeline = tl;
    a.timeline_capacity = (int)std::min<size_t>(capacity, 1u << 30);
    a.timeline_cta = cta;
    st = rt->batched ? launch_rounds(rt, a, dev, count, nullptr) : launch_trace(rt, a, dev, count, nullptr, true);
  }
  if (st == ST_OK) st = rt->cuda(cudaStreamSynchronize(rt->stream), "timeline run");
  if (st == ST_OK) st = check_device_error(rt);
  if (st == ST_OK) st = rt->cuda(cudaMemcpy(marks, tl, capacity * sizeof(long long), cudaMemcpyDeviceToHost), "timeline download");
  if (st == ST_OK && used && rt->flow && !rt->batched) {
    *used = (size_t)grid * kFlowTags;
  } else if (st == ST_OK && used) {  // warp 0's entries
    const size_t per_warp = capacity / kWarps;
    size_t u = 0;
    while (u < per_warp && marks[u] != 0) ++u;
    *used = u;
  }
  cudaFree(dev);
  cudaFree(tl);
  return st;
}

int st_device_trace_resident(st_runtime* rt, const float* device_inputs, size_t count, double* us_per_step,
                             uint64_t* kernel_launches) {
  if (!rt || !device_inputs || count == 0) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (!rt->started) return rt->fail(ST_ERR_STATE, "st_start has not been called");
  if (rt->opt.backend == ST_BACKEND_PERSISTENT) ST_TRY(st_stop(rt));
  const uint64_t before = rt->launches;
  ST_TRY(device_trace_impl(rt, device_inputs, count, nullptr, us_per_step));
  // The reset that precedes the timed region is not counted.
  if (kernel_launches) *kernel_launches = rt->launches - before - 1;
  return ST_OK;
}

int st_device_trace_continue(st_runtime* rt, const float* device_inputs, size_t count, double* us_per_step,
                             uint64_t* kernel_launches) {
  if (!rt || !device_inputs || count == 0) return ST_ERR_INVALID;
  if (rt->failed) return rt->fail(ST_ERR_STATE, "runtime failed earlier: %s", rt->error.c_str());
  if (!rt->started) return rt->fail(ST_ERR_STATE, "st_start has not been called");
  if (rt->opt.backend == ST_BACKEND_PERSISTENT) ST_TRY(st_stop(rt));
  const uint64_t before = rt->launches;
  ST_TRY(device_trace_impl(rt, device_inputs, count, nullptr, us_per_step, false));
  if (kernel_launches) *kernel_launches = rt->launches - before;
  return ST_OK;
}

int st_info(st_runtime* rt, char* json, size_t capacity, size_t* needed) {
  if (!rt) return ST_ERR_INVALID;
  cudaFuncAttributes fa{};
  const void* kernel = persistent_fn(rt);
  std::string name = "k2_persistent";
  if (rt->opt.backend == ST_BACKEND_FUSED) {
    kernel = ST_LOOP_KERNEL(rt, fused);
    name = "k2_fused";
  } else if (rt->opt.backend == ST_BACKEND_CUDA || rt->opt.backend == ST_BACKEND_GRAPH) {
    kernel = ST_KERNEL(rt, ffn);
    name = "k2_ffn (per-op block kernels)";
  }
  const bool flow_loop = rt->flow && (rt->opt.backend == ST_BACKEND_FUSED || rt->opt.backend == ST_BACKEND_PERSISTENT);
  if (flow_loop) {
    kernel = rt->flow_fn;
    name = "k4_flow";
  }
  cudaFuncGetAttributes(&fa, kernel);
  static const char* backends[] = {"cuda", "graph", "cublas", "cublas-graph", "fused", "persistent"};
  static const char* modes[] = {"fp32", "fp16", "bf16"};
  int pst = ST_OK;
  std::ostringstream o;
  o << "{\"environment\":" << probe_json(rt->device, &pst) << ",\"backend\":\"" << backends[rt->opt.backend]
    << "\",\"blocks\":" << rt->grid << ",\"legal_cooperative_blocks\":" << rt->legal_blocks
    << ",\"threads\":" << (flow_loop ? flow_threads() : kThreads) << ",\"resource_kernel\":\"" << name << "\""
    << ",\"registers_per_thread\":" << fa.numRegs << ",\"local_bytes\":" << fa.localSizeBytes
    << ",\"shared_bytes\":" << fa.sharedSizeBytes << ",\"dynamic_shared_bytes\":" << (flow_loop ? flow_smem_bytes() : kSmem2)
    << ",\"cluster\":" << (flow_loop ? rt->fcluster : rt->cluster) << ",\"clusters\":" << (flow_loop ? rt->fnclusters : rt->nclusters)
    << ",\"flow\":" << (rt->flow ? "true" : "false") << ",\"flow_grid\":" << rt->fgrid
    << ",\"cooperative_clusters\":" << (rt->coop_clusters ? "true" : "false")
    << ",\"weight_ring\":" << (rt->ring ? "true" : "false") << ",\"l2_keep_layers\":" << rt->args.l2_keep_layers
    << ",\"attention_implementation\":\"one cluster per head, window split over the cluster, partials merged through DSMEM\""
    << ",\"matvec_implementation\":\"16-byte non-temporal loads; out- and down-projections K-split (per head, per ffn slice)\""
    << ",\"barriers_per_step\":" << (flow_loop ? 0 : forward_barrier_count(rt))
    << ",\"transport\":\"" << (rt->opt.backend == ST_BACKEND_PERSISTENT ? "mapped-system-load-store" : rt->opt.mapped ? "mapped-stream-sync" : "pinned-copy-stream-sync") << "\""
    << ",\"poll_policy\":\"" << (rt->opt.backoff ? "bounded-device-backoff-host-yield" : "tight") << "\""
    << ",\"workspace_storage\":\"FP32 with explicit rounding to the storage type\""
    << ",\"weights_and_kv_storage\":\"" << modes[rt->desc.mode] << "\""
    << ",\"layers\":" << rt->desc.layers << ",\"width\":" << rt->desc.width << ",\"heads\":" << rt->desc.heads
    << ",\"ffn\":" << rt->desc.ffn << ",\"window\":" << rt->desc.window << ",\"features\":" << rt->desc.features
    << ",\"tp_rank\":" << rt->tp_rank << ",\"tp_size\":" << rt->tp_size
    << ",\"streams\":" << rt->desc.streams << ",\"batched\":" << (rt->batched ? "true" : "false")
    << ",\"batched_tensor_cores\":" << (rt->tc ? "true" : "false") << ",\"tc_stages\":" << rt->args.tc_stages
    << ",\"tc_stage_bytes\":" << rt->args.tc_stage_bytes << ",\"tc_tmem_columns\":" << rt->args.tc_ncols
    << ",\"attention_stage_bytes\":" << rt->args.att_buf_bytes << ",\"attention_stage_slots\":" << rt->args.att_chunk << ",\"attention_stages_per_warp\":" << rt->args.att_stages << ",\"attention_hd64\":" << rt->args.att_hd64
    << ",\"tiled_weights_bytes\":" << rt->tweights_bytes
    << ",\"batched_grid\":" << rt->bgrid << ",\"batched_splits\":[" << rt->bsplit[0] << "," << rt->bsplit[1] << ","
    << rt->bsplit[2] << "," << rt->bsplit[3] << "],\"batched_tc_streams_per_unit\":[" << rt->tcn[0] << ","
    << rt->tcn[1] << "," << rt->tcn[2] << "," << rt->tcn[3] << "],\"batched_barriers_per_round\":"
    << (rt->batched ? round_barriers(rt->desc.layers, rt->args.fuse_swiglu != 0) : 0) << ",\"weights_bytes\":" << rt->weights_bytes
    << ",\"state_bytes\":" << rt->state_bytes << ",\"scratch_bytes\":" << rt->scratch_bytes << "}";
  return copy_json(o.str(), json, capacity, needed);
}

int st_probe(int device, char* json, size_t capacity, size_t* needed) {
  int st = ST_OK;
  std::string s = probe_json(device, &st);
  if (st != ST_OK) { g_create_error = "device probe failed"; return st; }
  return copy_json(s, json, capacity, needed);
}

void st_destroy(st_runtime* rt) {
  if (!rt) return;
  if (rt->running && !rt->failed) {
    if (st_stop(rt) != ST_OK && rt->stream) cudaStreamSynchronize(rt->stream);
  } else if (rt->stream) {
    cudaStreamSynchronize(rt->stream);
  }
  for (int g = 0; g < kMaxTp; ++g)
    if (rt->tp_peer_base[g]) cudaIpcCloseMemHandle(rt->tp_peer_base[g]);
  if (rt->graph_exec) cudaGraphExecDestroy(rt->graph_exec);
  if (rt->graph) cudaGraphDestroy(rt->graph);
  if (rt->ev_start) cudaEventDestroy(rt->ev_start);
  if (rt->ev_stop) cudaEventDestroy(rt->ev_stop);
  if (rt->stream) cudaStreamDestroy(rt->stream);
  if (rt->aux) cudaStreamDestroy(rt->aux);
  cudaFree(rt->weights);
  cudaFree(rt->tweights);
  cudaFree(rt->state);
  cudaFree(rt->scratch);
  if (rt->mb_h) cudaFreeHost(rt->mb_h);
  if (rt->in_h) cudaFreeHost(rt->in_h);
  if (rt->out_h) cudaFreeHost(rt->out_h);
  delete rt;
}

}  // extern "C"
