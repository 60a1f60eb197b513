/* Helpers shared by the two oracle translation units (mamba_oracle.c, rwkv7_oracle.c).
 * TEST INFRASTRUCTURE ONLY; see mamba_oracle.c for the reference citations. */
#ifndef ORACLE_INTERNAL_H
#define ORACLE_INTERNAL_H
#include <stddef.h>

typedef void (*par_fn)(void* ctx, long begin, long end);

float orc_expf(float x);                  /* portable_expf, tensor.rs:765-794 */
float orc_lnf(float x);                   /* portable_lnf, tensor.rs:799-837 */
float orc_lane_sigmoidf(float x);         /* lane_sigmoidf, tensor.rs:881-885 */
float lane_expf(float x);                 /* lane_expf, tensor.rs:877-879 */
float portable_sigmoidf(float x);         /* portable_sigmoidf, tensor.rs:841-843 */
float dot_ref(const float* w, const float* v, size_t n);   /* dot_avx2_order, tensor.rs:1680-1693 */
void layer_norm_into(float* out, const float* x, const float* w, const float* b, size_t n, float eps);
void par_for(long n, long work, par_fn fn, void* ctx);     /* row partition over the pool */
int use_avx2(void);                                        /* REDUKT_NO_SIMD=1 or orc_set_simd(0) turn it off */
#endif
