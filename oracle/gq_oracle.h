/*
 * gq_oracle.h — CPU restatement of the reference engine's quantized-weight path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA kernels are
 * compared against (tests/, __graft_entry__.smoke(), and the cpu_baseline /
 * --impl reference legs of bench.py). Nothing in the product library (libgq.so)
 * links, loads or calls it.
 *
 * It restates, function by function, the Rust CPU backend of
 * Dhruba531/gemma-4-webgpu-kernels (paths are relative to that project):
 *   rust/src/backend.rs:16-56     QuantWeight {per_byte,row_bytes,scale_stride,deq}
 *   rust/src/dequant.rs:16-82     unpack_int / pack_int / pack_unsigned / dequantize
 *   rust/src/backend_cpu.rs:55-58 gelu_tanh_scalar
 *   rust/src/backend_cpu.rs:70-91 par_ranges (GEMMA_CPU_THREADS row split)
 *   rust/src/backend_cpu.rs:127-145 embed_rows
 *   rust/src/backend_cpu.rs:174-222 linear (dequantize the row once, then a
 *                                   sequential f32 dot, k ascending)
 *   rust/src/backend_cpu.rs:239-244 geglu / softcap
 *   rust/src/backend.rs:155-167   linear_geglu / linear_gelu_mul_cols compositions
 *   rust/src/backend_cpu.rs:149-172, 224-235, 248-336 rms_norm, add/mul/scale, rope,
 *                                 attention; rust/src/backend.rs:137-154 add_rms_norm,
 *                                 head_norm_rope (the support ops of a decode step)
 *   rust/src/sampler.rs:5-190     Rng, top_k_desc, softmax_over, sample_all, sample
 *
 * Arithmetic order follows the Rust code exactly (no FMA contraction: the build
 * uses -ffp-contract=off), so results are bit-identical to the reference CPU
 * backend wherever libm's tanhf agrees with Rust's f32::tanh (both call the
 * platform libm on Linux).
 *
 * Pinning: the known-answer tests of rust/tests/weights.rs:32-52 are re-run
 * against this library in tests/test_oracle.py.
 */
#ifndef GQ_ORACLE_H
#define GQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors rust/src/backend.rs:16-24 (QuantWeight). Host memory only. */
typedef struct gqo_qweight {
  const uint8_t *qbytes;
  const float *scales;
  int64_t n;          /* shape[0]: output rows */
  int64_t k;          /* shape[1]: logical columns */
  int32_t bits;       /* 2, 4 or 8 */
  int32_t signed_i8;  /* 1: native two's-complement I8 payload */
  int64_t group_size; /* columns per scale entry */
} gqo_qweight;

/* rust/src/backend.rs:28-41 */
int64_t gqo_per_byte(const gqo_qweight *w);
int64_t gqo_row_bytes(const gqo_qweight *w);
int64_t gqo_scale_stride(const gqo_qweight *w);
/* The integer code of element [n,k] (the part of deq before the scale). */
int32_t gqo_code(const gqo_qweight *w, int64_t n, int64_t k);
/* rust/src/backend.rs:45-56: q * scale[n*scale_stride + k/group_size]. */
float gqo_deq(const gqo_qweight *w, int64_t n, int64_t k);

/* rust/src/dequant.rs:16-33 */
void gqo_unpack_int(const uint8_t *bytes, int32_t bits, size_t count, int32_t *out);
/* rust/src/dequant.rs:37-50; returns bytes written (ceil(count/per_byte)) */
size_t gqo_pack_int(const int32_t *values, size_t count, int32_t bits, uint8_t *out);
/* rust/src/dequant.rs:53-62 */
size_t gqo_pack_unsigned(const uint32_t *values, size_t count, int32_t bits, uint8_t *out);
/* rust/src/dequant.rs:65-75 */
void gqo_dequantize(const int32_t *q, const float *scales, size_t rows, size_t cols,
                    size_t group_size, float *out);

/* Thread count with the GEMMA_CPU_THREADS semantics of backend_cpu.rs:72-78. */
int32_t gqo_default_threads(void);

/* rust/src/backend_cpu.rs:174-222. x [t,k] f32, y [t,n] f32.
 * threads <= 0 selects gqo_default_threads(). Returns 0, or -1 on bad shape. */
int32_t gqo_linear(const float *x, int64_t t, int64_t k, const gqo_qweight *w, float *y,
                   int32_t threads);
/* Plain f32 weight [n,k] (the CpuBackend non-quant branch of linear). */
int32_t gqo_linear_f32(const float *x, int64_t t, int64_t k, const float *w, int64_t n,
                       float *y, int32_t threads);

/* rust/src/backend_cpu.rs:127-137. Returns 0, or -1 if an id is out of range
 * (where the Rust code would panic on the slice index). */
int32_t gqo_embed_rows(const gqo_qweight *table, const uint32_t *ids, int64_t t, float scale,
                       float *out);

/* rust/src/backend_cpu.rs:55-58 */
float gqo_gelu_tanh(float v);
/* rust/src/backend_cpu.rs:239-241: gelu(gate) * up, elementwise */
void gqo_geglu(const float *gate, const float *up, size_t n, float *out);
/* rust/src/backend_cpu.rs:242-244: cap * tanh(v / cap) */
void gqo_softcap(const float *x, size_t n, float cap, float *out);
/* rust/src/backend_cpu.rs:343-350: [:, offset:offset+width] of [rows, stride] */
void gqo_slice_cols(const float *x, int64_t rows, int64_t stride, int64_t offset, int64_t width,
                    float *out);

/* rust/src/backend.rs:156-160: geglu(linear(x, wg), linear(x, wu)) */
int32_t gqo_linear_geglu(const float *x, int64_t t, int64_t k, const gqo_qweight *wg,
                         const gqo_qweight *wu, float *y, int32_t threads);
/* rust/src/backend.rs:163-167: geglu(linear(x, w), b[:, offset:offset+n]) */
int32_t gqo_linear_gelu_mul_cols(const float *x, int64_t t, int64_t k, const gqo_qweight *w,
                                 const float *b, int64_t b_stride, int64_t offset, float *y,
                                 int32_t threads);


/* ---- support ops of the decode step ---------------------------------------
 * rust/src/backend_cpu.rs:149-172 rms_norm (w NULL: unweighted) */
void gqo_rms_norm(const float *x, int64_t rows, int64_t d, const float *w, float eps, float *out);
/* rust/src/backend_cpu.rs:224-235 add / mul / scale */
void gqo_add(const float *a, const float *b, size_t n, float *out);
void gqo_mul(const float *a, const float *b, size_t n, float *out);
void gqo_scale(const float *a, size_t n, float s, float *out);
/* rust/src/backend.rs:137-144: (residual + rms_norm(x, w)) * scale_by[0] (scale_by may be NULL) */
void gqo_add_rms_norm(const float *residual, const float *x, int64_t rows, int64_t d, const float *w,
                      float eps, const float *scale_by, float *out);
/* rust/src/backend_cpu.rs:248-268: half-split partial RoPE on [t, heads, head_dim] */
void gqo_rope(const float *x, int64_t t, int64_t heads, int64_t head_dim, const uint32_t *positions,
              float theta, int64_t rotary_dim, float *out);
/* rust/src/backend.rs:148-154: per-head weighted RMSNorm then rope */
void gqo_head_norm_rope(const float *x, int64_t t, int64_t heads, int64_t head_dim, const float *w,
                        float eps, const uint32_t *positions, float theta, int64_t rotary_dim,
                        float *out);
/* rust/src/backend_cpu.rs:270-336: causal (+ sliding window) grouped-query
 * attention. q [t, hq, dh], k [s, hkv, dh], v [s, hkv, dv] -> out [t, hq*dv]. */
int32_t gqo_attention(const float *q, int64_t t, int64_t hq, int64_t dh, const float *k, const float *v,
                      int64_t s, int64_t hkv, int64_t dv, const uint32_t *q_pos, const uint32_t *k_pos,
                      float scale, uint32_t sliding_window, float attn_softcap, float *out,
                      int32_t threads);

/* ---- sampling: rust/src/sampler.rs ------------------------------------------------
 * Rng (sampler.rs:5-27): splitmix64; next_u64 advances *state, next_f64 is
 * (next_u64 >> 11) / 2^53. */
uint64_t gqo_rng_next_u64(uint64_t *state);
double gqo_rng_next_f64(uint64_t *state);
/* sample (sampler.rs:116-190) of one logits row: repetition penalty on a copy (each
 * distinct recent token < vocab once), greedy when temperature <= 0, else one draw
 * u in [0, 1) (the caller's rng()) through sample_all (no top-k, top-p >= 1) or the
 * candidate path: top_k_desc (the bounded min-heap of sampler.rs:67-113, then a
 * stable descending sort) or a stable sort of the whole row, the top-p cut over
 * softmax_over, and the draw over the kept candidates. Returns the token id, or -1
 * for a bad argument. */
int32_t gqo_sample(const float *logits, int64_t vocab, float temperature, int64_t top_k, float top_p,
                   float repetition_penalty, const uint32_t *recent, int64_t n_recent, double u);

#ifdef __cplusplus
}
#endif
#endif /* GQ_ORACLE_H */
