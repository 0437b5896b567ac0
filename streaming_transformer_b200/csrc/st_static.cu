// st_static.cu -- split-window attention that allocates nothing.
//
// Some callers cannot call cudaMalloc: code running where device allocation is
// forbidden or unsafe (inside a host callback of a stream, in a process whose
// memory pool is owned by another framework and must not fragment, or in a
// hard-real-time loop that may not take the allocator's locks). For them,
// st_attention_static computes the same split-window attention as the step
// kernels' attention phase over one layer's K/V ring, keeping its chunk
// partials in a fixed file-scope device array instead of allocated scratch.
// The caller still provides q, the ring and the output in its own memory.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "../../include/streaming_b200.h"
#include "st_device.cuh"

using namespace st;

namespace {

// Partials [heads][ceil(window / 32)][head_dim + 2] of one call. Every GPU
// that loads this library holds this array until the process exits.
static __device__ __align__(256) float g_attention_scratch[ST_ATTENTION_STATIC_MAX_FLOATS];

// Dimension limits of the entry point, and proof that every shape they admit
// fits the array: heads * head_dim <= 1024 with head_dim >= 2 gives at most
// 512 heads of (2 + 2) floats per chunk, and a window of 4096 slots 128 chunks.
constexpr int kStaticMaxWidth = 1024, kStaticMaxWindow = 4096;
static_assert((long long)(kStaticMaxWidth / 2) * ((kStaticMaxWindow + kAttChunk - 1) / kAttChunk) * (2 + 2) <=
                  ST_ATTENTION_STATIC_MAX_FLOATS,
              "the largest admitted attention shape must fit the static scratch array");

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
float* g_scratch_address[kMaxDevices] = {};
thread_local std::string g_static_error;

int fail(int code, const std::string& msg) {
  g_static_error = msg;
  return code;
}

// Device address of the scratch array on `device` (which must be current).
// The host-side symbol is only a stand-in and must never reach a kernel.
int scratch_address(int device, float** out) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_scratch_address[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (e != cudaSuccess) return fail(ST_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_scratch_address[device] = static_cast<float*>(p);
  }
  *out = g_scratch_address[device];
  return ST_OK;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) k_attention_static(StepArgs a, int valid) {
  const int warp = threadIdx.x >> 5;
  const int item = blockIdx.x * kWarps + warp;
  const int c = item % a.nchunks_max, h = item / a.nchunks_max;
  if (h >= a.heads || c * kAttChunk >= valid) return;
  const int dpl = (a.head_dim + 31) / 32;
  if (dpl <= 1) attention_item<T, 1>(a, 0, 0, h, c, valid);
  else if (dpl <= 2) attention_item<T, 2>(a, 0, 0, h, c, valid);
  else if (dpl <= 4) attention_item<T, 4>(a, 0, 0, h, c, valid);
  else if (dpl <= 8) attention_item<T, 8>(a, 0, 0, h, c, valid);
  else attention_item<T, 32>(a, 0, 0, h, c, valid);
}

// out[e] = round(sum_c acc_c[e] exp(m_c - M) / sum_c l_c exp(m_c - M)), the
// same merge the step applies before its out-projection.
template <typename T>
__global__ void __launch_bounds__(kThreads) k_merge_static(StepArgs a, int valid, float* out) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= a.width) return;
  const int hd = a.head_dim, C = a.nchunks_max;
  const int nc = (valid + kAttChunk - 1) / kAttChunk;
  const int h = e / hd, dd = e - h * hd;
  const float* ph = a.part + (size_t)h * C * (hd + 2);
  float M = -INFINITY;
  for (int c = 0; c < nc; ++c) M = fmaxf(M, ld_cg(ph + (size_t)c * (hd + 2)));
  float L = 0.f, acc = 0.f;
  for (int c = 0; c < nc; ++c) {
    const float* pc = ph + (size_t)c * (hd + 2);
    const float scale = expf(ld_cg(pc) - M);
    L = fmaf(ld_cg(pc + 1), scale, L);
    acc = fmaf(ld_cg(pc + 2 + dd), scale, acc);
  }
  out[e] = Storage<T>::round(acc / L);
}

template <typename T>
int launch(const StepArgs& a, int valid, float* out, cudaStream_t stream) {
  // An error left by an earlier launch on this thread belongs to its caller:
  // report it without clearing it rather than take it for this call's own.
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess)
    return fail(ST_ERR_CUDA, std::string("an earlier CUDA error is pending: ") + cudaGetErrorString(e));
  const int items = a.heads * a.nchunks_max;
  k_attention_static<T><<<(items + kWarps - 1) / kWarps, kThreads, 0, stream>>>(a, valid);
  if ((e = cudaGetLastError()) != cudaSuccess)
    return fail(ST_ERR_CUDA, std::string("attention launch: ") + cudaGetErrorString(e));
  k_merge_static<T><<<(a.width + kThreads - 1) / kThreads, kThreads, 0, stream>>>(a, valid, out);
  if ((e = cudaGetLastError()) != cudaSuccess)
    return fail(ST_ERR_CUDA, std::string("attention merge launch: ") + cudaGetErrorString(e));
  return ST_OK;
}

}  // namespace

extern "C" {

int st_attention_static(int device, int mode, int heads, int head_dim, int window, uint64_t position,
                        const float* q, const void* keys, const void* values, float* out, void* stream) {
  if (!q || !keys || !values || !out) return fail(ST_ERR_INVALID, "null pointer");
  if (device < 0 || device >= kMaxDevices) return fail(ST_ERR_INVALID, "device ordinal out of range");
  if (mode < ST_MODE_FP32 || mode > ST_MODE_BF16) return fail(ST_ERR_INVALID, "unknown storage mode");
  if (heads < 1 || head_dim < 2 || head_dim % 2 || (long long)heads * head_dim > kStaticMaxWidth || window < 1 ||
      window > kStaticMaxWindow)
    return fail(ST_ERR_INVALID, "Invalid or unsupported attention dimensions");
  const int nchunks = (window + kAttChunk - 1) / kAttChunk;
  const long long need = (long long)heads * nchunks * (head_dim + 2);
  // A guard only: the static_assert above shows the dimension limits keep
  // every admitted shape within the array.
  if (need > ST_ATTENTION_STATIC_MAX_FLOATS)
    return fail(ST_ERR_INVALID, "attention partials need " + std::to_string(need) +
                                    " floats, above the static scratch of " +
                                    std::to_string(ST_ATTENTION_STATIC_MAX_FLOATS));
  int previous = 0;
  cudaError_t e = cudaGetDevice(&previous);
  if (e != cudaSuccess) return fail(ST_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (previous != device && (e = cudaSetDevice(device)) != cudaSuccess)
    return fail(ST_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  float* scratch = nullptr;
  int st = scratch_address(device, &scratch);
  if (st == ST_OK) {
    StepArgs a{};
    a.layers = 1;
    a.streams = 1;
    a.heads = heads;
    a.head_dim = head_dim;
    a.width = heads * head_dim;
    a.window = window;
    a.nchunks_max = nchunks;
    a.q = const_cast<float*>(q);
    a.keys = const_cast<void*>(keys);
    a.values = const_cast<void*>(values);
    a.part = scratch;
    // retained slots: position + 1 until the ring is full (no overflow at the
    // largest position)
    const int valid = position >= (uint64_t)window - 1 ? window : (int)(position + 1);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (mode == ST_MODE_FP16) st = launch<__half>(a, valid, out, s);
    else if (mode == ST_MODE_BF16) st = launch<__nv_bfloat16>(a, valid, out, s);
    else st = launch<float>(a, valid, out, s);
  }
  if (previous != device) cudaSetDevice(previous);
  return st;
}

const char* st_attention_static_error(void) { return g_static_error.c_str(); }

}  // extern "C"
