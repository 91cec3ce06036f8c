/*
 * tq_oracle.h — declarations shared by the oracle's translation units
 * (test infrastructure only; see tq_oracle.c).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#define TQO_EXPORT __attribute__((visibility("default")))

uint64_t tqo_synth_key(uint64_t seed, uint64_t stream);
void tqo_pool_run(void (*fn)(void *arg, int idx), void *arg, int ntasks);
int tqo_get_threads(void);
void tqo_synth_fill(float *out, size_t n, uint64_t seed, uint64_t stream, float sigma);
void tqo_quantize8(const float *w, int rows, int cols, int8_t *q, float *scale);
int tqo_quantize4(const float *w, int rows, int cols, uint8_t *q, float *scale);
void tqo_q8_matmul(const int8_t *q, const float *scale, int rows, int cols, const float *x, float *out, int m,
                   int variant);
void tqo_q4_matmul(const uint8_t *q, const float *scale, int rows, int cols, const float *x, float *out, int m,
                   int variant);
