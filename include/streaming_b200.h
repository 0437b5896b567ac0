/*
 * streaming_b200.h -- C ABI of the B200 streaming-step runtime.
 *
 * This is the drop-in boundary for the reference's per-event hot path,
 * Stream::Runtime (reference include/Runtime.hpp:7-46, src/cuda/Runtime.cu:164-665).
 * The reference has no FFI: its C++ Runtime::Impl drives CUDA directly. Here the
 * C++ Runtime (include/Runtime.hpp in this repo) and any other host language call
 * these functions instead; every argument is a plain pointer, size or struct.
 *
 * Conventions
 *   - Every function returns ST_OK (0) or a negative ST_ERR_* code; the message
 *     is then available from st_last_error(handle) (or st_last_error(NULL) for
 *     a failed st_create). The reference raised std::runtime_error for the same
 *     conditions (src/cuda/Resources.cuh:9-20, src/cuda/Runtime.cu:178-194, 399-425).
 *   - One outstanding command per runtime, one submitting thread; not thread
 *     safe (reference docs/transport.md:14).
 *   - After a device-side error (ST_ERR_DEVICE_TIMEOUT, ST_ERR_CUDA) the runtime
 *     only accepts st_destroy.
 */
#ifndef STREAMING_B200_H
#define STREAMING_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ST_ABI_VERSION 1

enum st_status {
  ST_OK = 0,
  ST_ERR_INVALID = -1,         /* bad argument, option or model dimension */
  ST_ERR_UNSUPPORTED = -2,     /* valid in the reference but not provided (cuBLAS backends) */
  ST_ERR_CUDA = -3,            /* a CUDA runtime call failed */
  ST_ERR_STOPPED = -4,         /* persistent worker stopped or never started */
  ST_ERR_EXHAUSTED = -5,       /* mailbox sequence exhausted (last ID reserved for STOP) */
  ST_ERR_WORKER_EXITED = -6,   /* persistent worker left: max_events or idle budget */
  ST_ERR_DEVICE_TIMEOUT = -7,  /* a bounded device-side wait gave up */
  ST_ERR_HOST_TIMEOUT = -8,    /* the host gave up waiting for a completion */
  ST_ERR_STATE = -9            /* call out of order (e.g. step before st_start) */
};

/* reference include/Runtime.hpp:7 (Backend). Values match the enum order there. */
enum st_backend {
  ST_BACKEND_CUDA = 0,         /* per-phase kernel sequence */
  ST_BACKEND_GRAPH = 1,        /* the same sequence captured once as a CUDA graph */
  ST_BACKEND_CUBLAS = 2,       /* rejected: cuBLAS comparator is not provided */
  ST_BACKEND_CUBLAS_GRAPH = 3, /* rejected */
  ST_BACKEND_FUSED = 4,        /* one cooperative launch per step */
  ST_BACKEND_PERSISTENT = 5    /* one resident kernel driven by a mapped host mailbox */
};

/* Storage precision. 1 is the reference "mixed" mode (fp16 storage,
 * reference reference/model.py:3-5); 2 is the bf16 variant. Accumulation,
 * norms and softmax are fp32 in every mode. */
enum st_mode { ST_MODE_FP32 = 0, ST_MODE_FP16 = 1, ST_MODE_BF16 = 2 };

/* reference include/Model.hpp:12-18 (ModelConfig) + numeric mode + stream count. */
typedef struct {
  int layers, width, heads, ffn, window, features;
  float epsilon;
  int mode;    /* st_mode */
  int streams; /* independent streams advanced together by one step; 1 = reference */
} st_model_desc;

/* reference include/Runtime.hpp:8-19 (RuntimeOptions), same field meaning.
 * blocks: CTAs in every launch; 0 selects one CTA per SM. vector_matvec and
 * fused_attention are accepted for compatibility: the kernels here always use
 * 16-byte weight loads and split-window attention. */
typedef struct {
  int backend;                /* st_backend */
  int blocks;
  int backoff;                /* device nanosleep / host yield while polling */
  int mapped;                 /* mapped pinned staging for CUDA/GRAPH backends */
  int vector_matvec;
  int fused_attention;
  uint64_t max_events;        /* persistent: exit after this many RUNs (0 = unbounded) */
  uint64_t initial_sequence;  /* persistent: first mailbox sequence number */
  double idle_seconds;        /* persistent: idle budget, (0, 3600] */
  int device;                 /* CUDA device ordinal */
} st_options;

typedef struct st_runtime st_runtime;

/* Fills *options with the reference defaults (backend GRAPH, blocks 1,
 * idle 30 s; reference include/Runtime.hpp:8-19). */
void st_default_options(st_options* options);

/* Replaces the reference Runtime::Impl constructor's validation and allocation
 * (reference src/cuda/Runtime.cu:169-271). Allocates all device state, zeroed;
 * weights follow with st_set_tensor, then st_start. */
int st_create(const st_model_desc* model, const st_options* options, st_runtime** out);

/* Uploads one checkpoint tensor, float32 values already representable in the
 * storage type (reference src/cuda/Runtime.cu:231-256 upload). Names as in the
 * manifest: "input", "final_norm", "score", "layers.<l>.<norm1|norm2|q|k|v|out|gate|up|down>".
 * count must equal the tensor's element count. */
int st_set_tensor(st_runtime* rt, const char* name, const float* data, size_t count);

/* Tensor parallelism of one stream over tp_size GPUs of one node (1..8), one
 * runtime per GPU in its own process: GPU tp_rank owns heads
 * [tp_rank H/tp_size, +H/tp_size) and ffn rows [tp_rank F/tp_size, +F/tp_size)
 * of every layer, and the single-stream kernels of all GPUs exchange the
 * out-projection partials and the down-projection sums through each other's
 * memory over NVLink (plain stores into the peers' record buffers, polled
 * locally, every wait bounded). Needs the single-stream kernel's shapes,
 * streams == 1, heads and ffn divisible by tp_size, and the FUSED or PERSISTENT
 * backend. New; the reference runs one GPU per stream.
 * Sequence: st_create_tp on every GPU; st_tp_handle on every GPU; give every
 * GPU all tp_size handles in rank order with st_tp_connect; upload the tensors
 * (every GPU keeps the full weights and reads its shard); st_start on all GPUs
 * together. Every later call that runs the model (st_step, st_reset,
 * st_device_trace*) is collective: all GPUs of the stream make it with the
 * same inputs, in the same order, within the device wait bound (2 s).
 * st_snapshot of a GPU returns its own heads' K/V (zeros elsewhere) and the
 * full hidden state. */
int st_create_tp(const st_model_desc* model, const st_options* options, int tp_rank, int tp_size,
                 st_runtime** out);
/* This GPU's connection handle (an opaque blob of at most 256 bytes; *needed
 * receives its size). */
int st_tp_handle(st_runtime* rt, void* blob, size_t capacity, size_t* needed);
/* All tp_size handles, concatenated in rank order (this GPU's included). */
int st_tp_connect(st_runtime* rt, const void* blobs, size_t count);

/* Checks that every tensor is present, warms up, captures the graph (GRAPH) or
 * starts the resident worker (PERSISTENT) (reference src/cuda/Runtime.cu:263-291). */
int st_start(st_runtime* rt);

/* One event -> one score (reference Runtime::step, src/cuda/Runtime.cu:430-455).
 * input: features floats in host memory. For streams > 1 use st_step_batch. */
int st_step(st_runtime* rt, const float* input, float* score);

/* All streams advance by one event: inputs [streams][features], scores [streams],
 * both host memory. New; the reference runs one stream per runtime. */
int st_step_batch(st_runtime* rt, const float* inputs, float* scores);

/* Zero every stream's K/V/hidden and position (reference Runtime::reset,
 * src/cuda/Runtime.cu:457-464). */
int st_reset(st_runtime* rt);

/* Zero one stream's state only (new; needed once several streams share a step). */
int st_reset_stream(st_runtime* rt, int stream);

/* STOP the resident worker and join it; idempotent (reference Runtime::stop,
 * src/cuda/Runtime.cu:466-474). No-op for the other backends. */
int st_stop(st_runtime* rt);

/* Start a new resident worker after st_stop (PERSISTENT backend; a no-op
 * otherwise or while one runs). New: with st_load_state it hands a state to
 * the persistent backend; the reference's stop is final. Collective for a
 * tensor-parallel stream. */
int st_resume(st_runtime* rt);

/* Copy stream `stream`'s state to host: position, keys and values
 * [layers][heads][window][head_dim] widened to float, hidden [layers][width]
 * (reference Runtime::snapshot, src/cuda/Runtime.cu:548-568). Any output
 * pointer may be NULL. */
int st_snapshot(st_runtime* rt, int stream, uint64_t* position, float* keys,
                float* values, float* hidden);

/* Replace stream `stream`'s state: position, keys, values ([layers][heads]
 * [window][head_dim] floats, rounded to the storage type) and hidden
 * ([layers][width]). New: the reference can only read state. Used for sampled
 * checking of long runs by state hand-off and for testing far positions. */
int st_load_state(st_runtime* rt, int stream, uint64_t position, const float* keys,
                  const float* values, const float* hidden);

/* Per-op snapshot callback: name as in the reference trace ("input",
 * "layers.<l>.q", "layers.<l>.k", "layers.<l>.v", "layers.<l>.attention",
 * "layers.<l>.attention_residual", "layers.<l>.activation", "layers.<l>.hidden",
 * "score.linear"), values widened to float. */
typedef void (*st_trace_fn)(void* user, const char* name, const float* data, size_t count);

/* One step of stream 0 with a synchronizing snapshot after every phase kernel
 * (reference Runtime::traceStep, src/cuda/Runtime.cu:476-546). CUDA backend and
 * streams == 1 only, as in the reference. State advances exactly as st_step. */
int st_trace_step(st_runtime* rt, const float* input, float* score, st_trace_fn fn, void* user);

/* Device-only timing over a preloaded host trace of `count` events
 * ([count][streams][features]): resets, then steps every event on the device
 * and reports microseconds per step from CUDA events (reference
 * Runtime::deviceTrace, src/cuda/Runtime.cu:596-630). scores ([count][streams])
 * may be NULL. Stops a PERSISTENT worker first, as the reference does. */
int st_device_trace(st_runtime* rt, const float* inputs, size_t count, float* scores,
                    double* us_per_step);

/* Diagnostic device timeline: like st_device_trace (FUSED/PERSISTENT device
 * loop), with every warp of CTA 0 recording clock64() << 8 | tag at every phase
 * boundary of every step; warp w (of 16) fills marks[w * capacity / 16 ..
 * (w + 1) * capacity / 16) and unused entries stay 0. *used receives the number
 * warp 0 wrote. New; the reference exposes no intra-step timing. */
int st_device_timeline(st_runtime* rt, const float* inputs, size_t count, long long* marks, size_t capacity,
                       size_t* used);

/* Same, recorded by CTA `cta` of the grid (0 <= cta < blocks in st_info, or
 * < batched_grid when st_info reports "batched": then thread 0 of that CTA
 * records the end of every phase of the batched round, tags 40-48, and every
 * grid-barrier exit, tag 49, in warp 0's row). For the single-stream step
 * kernel ("flow" in st_info) pass cta = -1 and capacity >= flow_grid * 32:
 * marks[c * 32 + tag] receives CTA c's clock64() cycles spent in the phase
 * ending at each tag, summed over the steps, and marks[c * 32] the steps. */
int st_device_timeline_cta(st_runtime* rt, const float* inputs, size_t count, int cta, long long* marks,
                           size_t capacity, size_t* used);

/* Same, but `inputs` is a device pointer already resident in HBM and no score is
 * copied back; *kernel_launches receives the number of kernels launched. */
int st_device_trace_resident(st_runtime* rt, const float* device_inputs, size_t count,
                             double* us_per_step, uint64_t* kernel_launches);

/* Same as st_device_trace_resident, but from the current state: no reset
 * before the timed region, so positions continue where the previous step,
 * trace or st_load_state left them (steady-state timing with a full window).
 * *kernel_launches counts every kernel of the timed region. New; the
 * reference's deviceTrace always starts from reset. */
int st_device_trace_continue(st_runtime* rt, const float* device_inputs, size_t count,
                             double* us_per_step, uint64_t* kernel_launches);

/* Allocation-free attention. No counterpart in the reference.
 *
 * Split-window attention over one layer's K/V ring, as the step computes it,
 * for callers that cannot allocate device memory: code that runs where
 * cudaMalloc is not allowed or not safe (a stream host callback, a process
 * whose device memory pool belongs to another framework, a real-time loop
 * that may not take the allocator's locks). Its chunk partials live in a fixed
 * device array of ST_ATTENTION_STATIC_MAX_FLOATS floats (1 MiB) compiled into
 * this library, which every GPU that loads the library keeps until the process
 * exits. The call allocates and frees nothing.
 *
 *   q       [heads * head_dim] float, device memory, already rotated
 *   keys    [heads][window][head_dim] storage type of `mode`, device memory
 *   values  same layout as keys
 *   out     [heads * head_dim] float, device memory; rounded to the storage
 *           precision like the step's attention output
 * position is the absolute position of the current event: ring slots
 * 0 .. min(position + 1, window) - 1 are attended. Work is queued on `stream`
 * (a cudaStream_t, NULL for the legacy stream); the call returns without
 * waiting. The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture. Every call shares the one array and overwrites
 * the previous call's partials, so calls that may overlap on the GPU (other
 * streams, other host threads) race and must be serialized by the caller.
 * Dimensions beyond heads * head_dim <= 1024 or a window above 4096 are
 * rejected with ST_ERR_INVALID (every admitted shape fits the array; the
 * library checks that at compile time); the message is in
 * st_attention_static_error(). A CUDA error already pending on the calling
 * thread is reported as ST_ERR_CUDA and left pending. */
#define ST_ATTENTION_STATIC_MAX_FLOATS 262144
int st_attention_static(int device, int mode, int heads, int head_dim, int window, uint64_t position,
                        const float* q, const void* keys, const void* values, float* out, void* stream);
const char* st_attention_static_error(void);

/* Scheduled-arrival replay (reference bench/Main.cpp:282-343, statistics
 * 416-447): event i of `inputs` ([count][features]) arrives at
 * i / rate seconds after the start (bursty: in groups of 16 arriving at the
 * group's first time) and is appended by a producer thread to a queue of
 * `queue` events, or dropped when the queue is full; the calling thread takes
 * events off the queue in order and steps them. */
typedef struct {
  double rate;          /* arrivals per second, > 0 */
  int bursty;           /* 1: arrivals in groups of 16 */
  size_t queue;         /* queue capacity, >= 1 */
  double deadline_us;   /* an arrival-to-completion time above it counts as a miss */
  int producer_core;    /* CPU the producer thread is pinned to, -1 for none */
} st_schedule;
/* One step: score the event `input`; returns ST_OK or an error code. */
typedef int (*st_step_fn)(void* user, const float* input, float* score);
/* The replay through any step function. samples ([count][4], may be NULL)
 * receive each event's intended, enqueue, submit and completion times in
 * steady-clock nanoseconds (submit and completion 0 when dropped); scores
 * ([count], may be NULL) the scores (NaN when dropped); json the report:
 * completed, dropped, service rate, deadline misses and the service,
 * arrival-to-completion, queueing and injection distributions. A failing step
 * ends the replay with its code; st_replay_error() has the message. */
int st_replay_scheduled_with(st_step_fn step, void* user, const float* inputs, size_t count, size_t features,
                             const st_schedule* schedule, double* samples, float* scores, char* json,
                             size_t capacity, size_t* needed);
/* The same through st_step of a one-stream runtime. */
int st_replay_scheduled(st_runtime* rt, const float* inputs, size_t count, const st_schedule* schedule,
                        double* samples, float* scores, char* json, size_t capacity, size_t* needed);
const char* st_replay_error(void);

/* JSON description of the runtime: options, grid, kernel resources, layout
 * (reference Runtime::info, src/cuda/Runtime.cu:570-594). Writes at most
 * capacity bytes including the terminator; *needed gets the full length. */
int st_info(st_runtime* rt, char* json, size_t capacity, size_t* needed);

/* JSON device probe (reference deviceProbe/probe(), src/cuda/Runtime.cu:134-161). */
int st_probe(int device, char* json, size_t capacity, size_t* needed);

/* Transport and synchronization calibration (reference transportBench,
 * src/cuda/Runtime.cu:706-814): mode "empty", "empty-graph", "copy",
 * "ping-pong", "gpu-ping", or "grid-barrier" (device ns per grid barrier of the
 * step kernels, one 512-thread CTA per SM). Writes a JSON report; csv_path
 * (may be NULL) receives per-event samples. On error see st_transport_error(). */
int st_transport_bench(int device, const char* mode, size_t count, int backoff, const char* csv_path,
                       char* json, size_t capacity, size_t* needed);
const char* st_transport_error(void);

/* Kernels launched by this runtime since creation (for launch-count reporting). */
uint64_t st_kernel_launches(const st_runtime* rt);

const char* st_last_error(const st_runtime* rt);

/* Stops the worker, synchronizes and frees everything (reference
 * src/cuda/Runtime.cu:294-299). NULL is ignored. */
void st_destroy(st_runtime* rt);

int st_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif
