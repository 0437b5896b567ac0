/*
 * st_oracle.c -- CPU restatement of the reference streaming step (TEST INFRASTRUCTURE).
 *
 * This file is the parity checker and the CPU baseline, never the product path.
 * Each function names the reference code it restates:
 *   reference src/cpu/Cpu.cpp:21-27    cast           -> oracle_cast
 *   reference src/cpu/Cpu.cpp:29-41    linear         -> oracle_linear
 *   reference src/cpu/Cpu.cpp:43-57    norm           -> oracle_norm
 *   reference src/cpu/Cpu.cpp:59-141   step           -> st_oracle_step_traced
 *   reference src/cpu/Cpu.cpp:143-148  reset          -> st_oracle_reset
 *   reference src/runtime/Model.cpp:22-29 validate    -> config_valid
 *   reference src/runtime/Model.cpp:59-61 roundHalf   -> st_oracle_round_half
 * Eigen's GEMV summation order is unspecified, so the dot products here use a
 * fixed order of their own (eight interleaved float partial sums combined
 * pairwise); parity with the reference is tolerance based for that reason.
 * Built with -ffp-contract=off so no multiply-add is fused.
 */
#include "st_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
  float *norm1, *norm2, *q, *k, *v, *out, *gate, *up, *down;
} oracle_layer;

struct st_oracle {
  st_oracle_config c;
  int threads;
  uint64_t position;
  float *input_w, *final_norm, *score_w;
  oracle_layer* layers;
  unsigned char* have; /* one flag per tensor */
  int tensor_count;
  float *keys, *values, *hidden;
  float *x, *norm, *q, *k, *v, *attention, *temp, *gate, *up, *logits;
};

static uint32_t float_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float bits_float(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE-754 binary16 round-to-nearest-even (reference uses Eigen::half, Cpu.cpp:24). */
float st_oracle_round_half(float value) {
  uint32_t u = float_bits(value);
  uint32_t sign = u & 0x80000000u, mag = u & 0x7fffffffu;
  if (mag >= 0x7f800000u) return value;                 /* inf / NaN unchanged */
  if (mag >= 0x477ff000u) return bits_float(sign | 0x7f800000u); /* >= 65520 -> inf */
  if (mag < 0x38800000u) {                              /* below 2^-14: subnormal half */
    /* quantum is 2^-24: scale (exact), round to an integer with ties to even, unscale */
    float scaled = fabsf(value) * 16777216.0f;
    float r = rintf(scaled);                            /* default mode: nearest-even */
    return bits_float(sign | float_bits(r / 16777216.0f));
  }
  /* normal half: keep 10 of float's 23 mantissa bits */
  uint32_t lsb = (mag >> 13) & 1u;
  uint32_t rounded = (mag + 0x0fffu + lsb) & ~0x1fffu;
  return bits_float(sign | rounded);
}

/* bfloat16 round-to-nearest-even: keep the top 16 bits of the float. */
float st_oracle_round_bf16(float value) {
  uint32_t u = float_bits(value);
  if ((u & 0x7fffffffu) > 0x7f800000u) return value;   /* NaN unchanged */
  uint32_t lsb = (u >> 16) & 1u;
  u = (u + 0x7fffu + lsb) & 0xffff0000u;
  return bits_float(u);
}

static float oracle_round(int mode, float v) {
  if (mode == 1) return st_oracle_round_half(v);
  if (mode == 2) return st_oracle_round_bf16(v);
  return v;
}

/* reference Cpu.cpp:21-27 */
static void oracle_cast(const st_oracle* o, float* data, int size) {
  if (o->c.mode == 0) return;
  for (int i = 0; i < size; i++) data[i] = oracle_round(o->c.mode, data[i]);
}

/* Fixed-order float dot product: 8 interleaved partial sums, combined pairwise. */
static float dot(const float* w, const float* x, int n) {
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int i = 0;
  for (; i + 8 <= n; i += 8) {
    s[0] += w[i + 0] * x[i + 0];
    s[1] += w[i + 1] * x[i + 1];
    s[2] += w[i + 2] * x[i + 2];
    s[3] += w[i + 3] * x[i + 3];
    s[4] += w[i + 4] * x[i + 4];
    s[5] += w[i + 5] * x[i + 5];
    s[6] += w[i + 6] * x[i + 6];
    s[7] += w[i + 7] * x[i + 7];
  }
  for (int j = 0; i < n; i++, j++) s[j] += w[i] * x[i];
  return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

static void emit(st_oracle_trace_fn trace, void* user, const char* a, const char* b,
                 const float* data, int count) {
  if (!trace) return;
  char name[128];
  snprintf(name, sizeof name, "%s%s", a, b);
  trace(user, name, data, count);
}

/* reference Cpu.cpp:29-41: output = W * input (row-major [rows, cols]); cast unless final. */
static void oracle_linear(st_oracle* o, const float* input, const float* w, int rows, int cols,
                          float* output, int final, const char* name,
                          st_oracle_trace_fn trace, void* user) {
  emit(trace, user, name, ".operand", input, cols);
#ifdef _OPENMP
#pragma omp parallel for num_threads(o->threads) schedule(static) if (o->threads > 1 && rows >= 64)
#endif
  for (int r = 0; r < rows; r++) output[r] = dot(w + (size_t)r * cols, input, cols);
  emit(trace, user, name, ".pre_cast", output, rows);
  if (!final) oracle_cast(o, output, rows);
  emit(trace, user, name, ".linear", output, rows);
}

/* reference Cpu.cpp:43-57 */
static void oracle_norm(st_oracle* o, const float* input, const float* weight, float* output,
                        const char* name, st_oracle_trace_fn trace, void* user) {
  int width = o->c.width;
  emit(trace, user, name, ".operand", input, width);
  float sum = 0;
  for (int i = 0; i < width; i++) sum += input[i] * input[i];
  float scale = 1.0f / sqrtf(sum / (float)width + o->c.epsilon);
  for (int i = 0; i < width; i++) output[i] = input[i] * scale * weight[i];
  emit(trace, user, name, ".pre_cast", output, width);
  oracle_cast(o, output, width);
  emit(trace, user, name, ".norm", output, width);
}

/* reference src/runtime/Model.cpp:22-29 */
static int config_valid(const st_oracle_config* c) {
  if (c->layers < 1 || c->layers > 16 || c->width < 1 || c->width > 1024 || c->heads < 1) return 0;
  if (c->width % c->heads || (c->width / c->heads) % 2) return 0;
  if (c->ffn < 1 || c->ffn > 4096 || c->window < 1 || c->window > 4096) return 0;
  if (c->features < 1 || c->features > 1024) return 0;
  if (!isfinite(c->epsilon) || c->epsilon <= 0) return 0;
  if (c->mode < 0 || c->mode > 2) return 0;
  return 1;
}

static float* alloc_floats(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

st_oracle* st_oracle_create(const st_oracle_config* config, int threads) {
  if (!config || !config_valid(config)) return NULL;
  st_oracle* o = (st_oracle*)calloc(1, sizeof(st_oracle));
  if (!o) return NULL;
  o->c = *config;
  o->threads = threads < 1 ? 1 : threads;
  const st_oracle_config* c = &o->c;
  size_t d = (size_t)c->width, f = (size_t)c->ffn;
  o->input_w = alloc_floats(d * c->features);
  o->final_norm = alloc_floats(d);
  o->score_w = alloc_floats(d);
  o->layers = (oracle_layer*)calloc((size_t)c->layers, sizeof(oracle_layer));
  for (int l = 0; l < c->layers; l++) {
    oracle_layer* L = &o->layers[l];
    L->norm1 = alloc_floats(d); L->norm2 = alloc_floats(d);
    L->q = alloc_floats(d * d); L->k = alloc_floats(d * d);
    L->v = alloc_floats(d * d); L->out = alloc_floats(d * d);
    L->gate = alloc_floats(f * d); L->up = alloc_floats(f * d);
    L->down = alloc_floats(d * f);
  }
  o->tensor_count = 3 + 9 * c->layers;
  o->have = (unsigned char*)calloc((size_t)o->tensor_count, 1);
  size_t cache = (size_t)c->layers * d * c->window;
  o->keys = alloc_floats(cache);
  o->values = alloc_floats(cache);
  o->hidden = alloc_floats((size_t)c->layers * d);
  o->x = alloc_floats(d); o->norm = alloc_floats(d); o->q = alloc_floats(d);
  o->k = alloc_floats(d); o->v = alloc_floats(d); o->attention = alloc_floats(d);
  o->temp = alloc_floats(d); o->gate = alloc_floats(f); o->up = alloc_floats(f);
  o->logits = alloc_floats((size_t)c->window);
  return o;
}

void st_oracle_destroy(st_oracle* o) {
  if (!o) return;
  free(o->input_w); free(o->final_norm); free(o->score_w);
  for (int l = 0; l < o->c.layers; l++) {
    oracle_layer* L = &o->layers[l];
    free(L->norm1); free(L->norm2); free(L->q); free(L->k); free(L->v);
    free(L->out); free(L->gate); free(L->up); free(L->down);
  }
  free(o->layers); free(o->have);
  free(o->keys); free(o->values); free(o->hidden);
  free(o->x); free(o->norm); free(o->q); free(o->k); free(o->v); free(o->attention);
  free(o->temp); free(o->gate); free(o->up); free(o->logits);
  free(o);
}

int st_oracle_set_tensor(st_oracle* o, const char* name, const float* data, size_t count) {
  size_t d = (size_t)o->c.width, f = (size_t)o->c.ffn;
  float* target = NULL;
  size_t expect = 0;
  int index = -1;
  if (!strcmp(name, "input")) { target = o->input_w; expect = d * o->c.features; index = 0; }
  else if (!strcmp(name, "final_norm")) { target = o->final_norm; expect = d; index = 1; }
  else if (!strcmp(name, "score")) { target = o->score_w; expect = d; index = 2; }
  else {
    int l = -1;
    char part[32];
    if (sscanf(name, "layers.%d.%31s", &l, part) != 2 || l < 0 || l >= o->c.layers) return -1;
    oracle_layer* L = &o->layers[l];
    static const char* names[9] = {"norm1", "norm2", "q", "k", "v", "out", "gate", "up", "down"};
    float* slots[9] = {L->norm1, L->norm2, L->q, L->k, L->v, L->out, L->gate, L->up, L->down};
    size_t sizes[9] = {d, d, d * d, d * d, d * d, d * d, f * d, f * d, d * f};
    for (int i = 0; i < 9; i++) {
      if (!strcmp(part, names[i])) { target = slots[i]; expect = sizes[i]; index = 3 + 9 * l + i; }
    }
  }
  if (!target || count != expect) return -1;
  memcpy(target, data, count * sizeof(float));
  o->have[index] = 1;
  return 0;
}

int st_oracle_ready(const st_oracle* o) {
  for (int i = 0; i < o->tensor_count; i++) if (!o->have[i]) return 0;
  return 1;
}

/* reference Cpu.cpp:59-141 */
float st_oracle_step_traced(st_oracle* o, const float* input, st_oracle_trace_fn trace, void* user) {
  const st_oracle_config* c = &o->c;
  int d = c->width / c->heads;
  int slot = (int)(o->position % (uint64_t)c->window);
  int valid = o->position + 1 < (uint64_t)c->window ? (int)(o->position + 1) : c->window;
  char p[48];
  oracle_linear(o, input, o->input_w, c->width, c->features, o->x, 0, "input", trace, user);
  emit(trace, user, "input", "", o->x, c->width);
  for (int l = 0; l < c->layers; l++) {
    oracle_layer* L = &o->layers[l];
    char n[64];
    snprintf(p, sizeof p, "layers.%d.", l);
    snprintf(n, sizeof n, "%snorm1", p);
    oracle_norm(o, o->x, L->norm1, o->norm, n, trace, user);
    snprintf(n, sizeof n, "%sq", p);
    oracle_linear(o, o->norm, L->q, c->width, c->width, o->q, 0, n, trace, user);
    snprintf(n, sizeof n, "%sk", p);
    oracle_linear(o, o->norm, L->k, c->width, c->width, o->k, 0, n, trace, user);
    snprintf(n, sizeof n, "%sv", p);
    oracle_linear(o, o->norm, L->v, c->width, c->width, o->v, 0, n, trace, user);
    /* RoPE on adjacent pairs, angle = t * 10000^(-i/d) in float (Cpu.cpp:73-83) */
    for (int h = 0; h < c->heads; h++) {
      for (int i = 0; i < d; i += 2) {
        float angle = (float)o->position * powf(10000.0f, -(float)i / (float)d);
        float co = cosf(angle), si = sinf(angle);
        float* vectors[2] = {o->q, o->k};
        for (int s = 0; s < 2; s++) {
          float* vec = vectors[s];
          float a = vec[h * d + i], b = vec[h * d + i + 1];
          vec[h * d + i] = a * co - b * si;
          vec[h * d + i + 1] = a * si + b * co;
        }
      }
    }
    oracle_cast(o, o->q, c->width);
    oracle_cast(o, o->k, c->width);
    emit(trace, user, p, "q", o->q, c->width);
    emit(trace, user, p, "k", o->k, c->width);
    emit(trace, user, p, "v", o->v, c->width);
    float sqrt_d = sqrtf((float)d);
    for (int h = 0; h < c->heads; h++) {
      size_t base = ((size_t)l * c->heads + h) * (size_t)c->window * d;
      for (int i = 0; i < d; i++) {
        o->keys[base + (size_t)slot * d + i] = o->k[h * d + i];
        o->values[base + (size_t)slot * d + i] = o->v[h * d + i];
      }
      /* physical ring order: slots 0..valid-1 (Cpu.cpp:97-110) */
      const float* qh = o->q + h * d;
      for (int j = 0; j < valid; j++) o->logits[j] = dot(o->keys + base + (size_t)j * d, qh, d);
      for (int j = 0; j < valid; j++) o->logits[j] /= sqrt_d;
      float maximum = o->logits[0];
      for (int j = 1; j < valid; j++) if (o->logits[j] > maximum) maximum = o->logits[j];
      float total = 0;
      for (int j = 0; j < valid; j++) { o->logits[j] = expf(o->logits[j] - maximum); total += o->logits[j]; }
      for (int j = 0; j < valid; j++) o->logits[j] /= total;
      float* out = o->attention + h * d;
      for (int i = 0; i < d; i++) out[i] = 0;
      for (int j = 0; j < valid; j++) {
        const float* vrow = o->values + base + (size_t)j * d;
        float pj = o->logits[j];
        for (int i = 0; i < d; i++) out[i] += pj * vrow[i];
      }
    }
    oracle_cast(o, o->attention, c->width);
    emit(trace, user, p, "attention", o->attention, c->width);
    snprintf(n, sizeof n, "%sout", p);
    oracle_linear(o, o->attention, L->out, c->width, c->width, o->temp, 0, n, trace, user);
    for (int i = 0; i < c->width; i++) o->x[i] += o->temp[i];
    oracle_cast(o, o->x, c->width);
    emit(trace, user, p, "attention_residual", o->x, c->width);
    snprintf(n, sizeof n, "%snorm2", p);
    oracle_norm(o, o->x, L->norm2, o->norm, n, trace, user);
    snprintf(n, sizeof n, "%sgate", p);
    oracle_linear(o, o->norm, L->gate, c->ffn, c->width, o->gate, 0, n, trace, user);
    snprintf(n, sizeof n, "%sup", p);
    oracle_linear(o, o->norm, L->up, c->ffn, c->width, o->up, 0, n, trace, user);
    for (int i = 0; i < c->ffn; i++) o->gate[i] = (o->gate[i] / (1.0f + expf(-o->gate[i]))) * o->up[i];
    oracle_cast(o, o->gate, c->ffn);
    emit(trace, user, p, "activation", o->gate, c->ffn);
    snprintf(n, sizeof n, "%sdown", p);
    oracle_linear(o, o->gate, L->down, c->width, c->ffn, o->temp, 0, n, trace, user);
    for (int i = 0; i < c->width; i++) o->x[i] += o->temp[i];
    oracle_cast(o, o->x, c->width);
    emit(trace, user, p, "hidden", o->x, c->width);
    memcpy(o->hidden + (size_t)l * c->width, o->x, (size_t)c->width * sizeof(float));
  }
  oracle_norm(o, o->x, o->final_norm, o->norm, "final_norm", trace, user);
  float score;
  oracle_linear(o, o->norm, o->score_w, 1, c->width, &score, 1, "score", trace, user);
  o->position++;
  return score;
}

float st_oracle_step(st_oracle* o, const float* input) {
  return st_oracle_step_traced(o, input, NULL, NULL);
}

void st_oracle_run(st_oracle* o, const float* inputs, size_t count, float* scores) {
  for (size_t i = 0; i < count; i++) scores[i] = st_oracle_step(o, inputs + i * (size_t)o->c.features);
}

/* reference Cpu.cpp:143-148 */
void st_oracle_reset(st_oracle* o) {
  size_t cache = st_oracle_cache_elements(o);
  o->position = 0;
  memset(o->keys, 0, cache * sizeof(float));
  memset(o->values, 0, cache * sizeof(float));
  memset(o->hidden, 0, (size_t)o->c.layers * o->c.width * sizeof(float));
}

uint64_t st_oracle_position(const st_oracle* o) { return o->position; }
const float* st_oracle_keys(const st_oracle* o) { return o->keys; }
const float* st_oracle_values(const st_oracle* o) { return o->values; }
const float* st_oracle_hidden(const st_oracle* o) { return o->hidden; }
size_t st_oracle_cache_elements(const st_oracle* o) {
  return (size_t)o->c.layers * o->c.width * o->c.window;
}

void st_oracle_load_state(st_oracle* o, uint64_t position, const float* keys,
                          const float* values, const float* hidden) {
  size_t cache = st_oracle_cache_elements(o);
  o->position = position;
  memcpy(o->keys, keys, cache * sizeof(float));
  memcpy(o->values, values, cache * sizeof(float));
  memcpy(o->hidden, hidden, (size_t)o->c.layers * o->c.width * sizeof(float));
}
