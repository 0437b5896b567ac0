/*
 * st_oracle.h -- CPU restatement of the reference streaming step.
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity checker for the CUDA runtime,
 * not part of the product. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference legs may load it. The product library never links it.
 *
 * It restates Stream::Cpu (reference include/Cpu.hpp:11-34, src/cpu/Cpu.cpp:8-154)
 * in plain C without Eigen: same op order, same cast points, physical-ring
 * attention, float32 accumulation. The numeric mode selects the cast applied at
 * the reference's cast points: 0 = fp32 (no cast), 1 = fp16 round-to-nearest-even
 * (the reference "mixed" mode, Eigen::half), 2 = bf16 round-to-nearest-even
 * (the bf16 variant requested for the B200 configs).
 */
#ifndef ST_ORACLE_H
#define ST_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct st_oracle st_oracle;

typedef struct {
  int layers, width, heads, ffn, window, features;
  float epsilon;
  int mode; /* 0 fp32, 1 fp16 ("mixed"), 2 bf16 */
} st_oracle_config;

/* Per-op capture hook (reference CpuTrace, src/cpu/Cpu.cpp:29-57). Called with a
 * name such as "layers.0.q.pre_cast" and the values; may be NULL. */
typedef void (*st_oracle_trace_fn)(void* user, const char* name, const float* data, int count);

/* Returns NULL on an invalid configuration (reference ModelConfig::validate,
 * src/runtime/Model.cpp:22-29). threads > 1 splits GEMV rows across OpenMP
 * threads; each row keeps the same fixed summation order, so results do not
 * depend on the thread count. */
st_oracle* st_oracle_create(const st_oracle_config* config, int threads);
void st_oracle_destroy(st_oracle* o);

/* Tensor names follow the checkpoint manifest (reference reference/model.py:35-46):
 * "input", "final_norm", "score", "layers.<l>.{norm1,norm2,q,k,v,out,gate,up,down}".
 * Data are float32 values (already representable in the storage type).
 * Returns 0 on success, -1 for an unknown name or wrong element count. */
int st_oracle_set_tensor(st_oracle* o, const char* name, const float* data, size_t count);
/* Non-zero when every tensor has been set. */
int st_oracle_ready(const st_oracle* o);

/* One event (features floats) -> one score. Advances the position. */
float st_oracle_step(st_oracle* o, const float* input);
/* Same, calling trace(user, name, ...) at the reference's capture points. */
float st_oracle_step_traced(st_oracle* o, const float* input, st_oracle_trace_fn trace, void* user);
void st_oracle_reset(st_oracle* o);

uint64_t st_oracle_position(const st_oracle* o);
/* [layers, heads, window, head_dim] float32 views of the ring and [layers, width] hidden. */
const float* st_oracle_keys(const st_oracle* o);
const float* st_oracle_values(const st_oracle* o);
const float* st_oracle_hidden(const st_oracle* o);
size_t st_oracle_cache_elements(const st_oracle* o);

/* State hand-off for sampled checking of long runs: replaces position, ring
 * and hidden state (sizes as above). */
void st_oracle_load_state(st_oracle* o, uint64_t position, const float* keys,
                          const float* values, const float* hidden);

/* IEEE-754 round-to-nearest-even narrowing, widened back to float. */
float st_oracle_round_half(float value);
float st_oracle_round_bf16(float value);

/* Run `count` events back to back from a [count, features] array, writing
 * scores; used to time the CPU baseline. */
void st_oracle_run(st_oracle* o, const float* inputs, size_t count, float* scores);

#ifdef __cplusplus
}
#endif
#endif
