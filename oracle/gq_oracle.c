/*
 * gq_oracle.c — CPU restatement of the reference's quantized-weight path.
 * TEST INFRASTRUCTURE ONLY (see gq_oracle.h): the checker, never the product.
 *
 * Every function cites the Rust function it restates (paths relative to
 * Dhruba531/gemma-4-webgpu-kernels). Compiled with -ffp-contract=off so each
 * `a * b` and `+` rounds separately, as the Rust code does.
 */
#include "gq_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* rust/src/backend.rs:28-30 */
int64_t gqo_per_byte(const gqo_qweight *w) { return w->signed_i8 ? 1 : (8 / w->bits); }

/* rust/src/backend.rs:33-36 */
int64_t gqo_row_bytes(const gqo_qweight *w) {
  return w->signed_i8 ? w->k : w->k / gqo_per_byte(w);
}

/* rust/src/backend.rs:39-41 (div_ceil) */
int64_t gqo_scale_stride(const gqo_qweight *w) {
  return (w->k + w->group_size - 1) / w->group_size;
}

/* rust/src/backend.rs:46-54: the integer part of deq. Sub-byte and unsigned
 * 8-bit codes are offset binary (raw - 2^(bits-1)); I8 is two's complement. */
int32_t gqo_code(const gqo_qweight *w, int64_t n, int64_t k) {
  if (w->signed_i8) {
    return (int32_t)(int8_t)w->qbytes[n * gqo_row_bytes(w) + k];
  }
  int64_t per_byte = gqo_per_byte(w);
  uint32_t b = w->qbytes[n * gqo_row_bytes(w) + k / per_byte];
  uint32_t shift = (uint32_t)(k % per_byte) * (uint32_t)w->bits;
  return (int32_t)((b >> shift) & ((1u << w->bits) - 1u)) - (1 << (w->bits - 1));
}

/* rust/src/backend.rs:45-56 */
float gqo_deq(const gqo_qweight *w, int64_t n, int64_t k) {
  return (float)gqo_code(w, n, k) * w->scales[n * gqo_scale_stride(w) + k / w->group_size];
}

/* rust/src/dequant.rs:16-33 */
void gqo_unpack_int(const uint8_t *bytes, int32_t bits, size_t count, int32_t *out) {
  if (bits == 8) {
    for (size_t i = 0; i < count; i++) out[i] = (int32_t)(int8_t)bytes[i];
    return;
  }
  size_t per_byte = (size_t)(8 / bits);
  uint32_t mask = (1u << bits) - 1u;
  int32_t zp = 1 << (bits - 1);
  for (size_t i = 0; i < count; i++) {
    uint32_t byte = bytes[i / per_byte];
    uint32_t shift = (uint32_t)(i % per_byte) * (uint32_t)bits;
    out[i] = (int32_t)((byte >> shift) & mask) - zp;
  }
}

/* rust/src/dequant.rs:37-50 */
size_t gqo_pack_int(const int32_t *values, size_t count, int32_t bits, uint8_t *out) {
  if (bits == 8) {
    for (size_t i = 0; i < count; i++) out[i] = (uint8_t)values[i];
    return count;
  }
  size_t per_byte = (size_t)(8 / bits);
  int32_t mask = (1 << bits) - 1;
  int32_t zp = 1 << (bits - 1);
  size_t nb = (count + per_byte - 1) / per_byte;
  memset(out, 0, nb);
  for (size_t i = 0; i < count; i++) {
    uint32_t shift = (uint32_t)(i % per_byte) * (uint32_t)bits;
    out[i / per_byte] |= (uint8_t)(((values[i] + zp) & mask) << shift);
  }
  return nb;
}

/* rust/src/dequant.rs:53-62 */
size_t gqo_pack_unsigned(const uint32_t *values, size_t count, int32_t bits, uint8_t *out) {
  size_t per_byte = (size_t)(8 / bits);
  uint32_t mask = (1u << bits) - 1u;
  size_t nb = (count + per_byte - 1) / per_byte;
  memset(out, 0, nb);
  for (size_t i = 0; i < count; i++) {
    uint32_t shift = (uint32_t)(i % per_byte) * (uint32_t)bits;
    out[i / per_byte] |= (uint8_t)((values[i] & mask) << shift);
  }
  return nb;
}

/* rust/src/dequant.rs:65-75 */
void gqo_dequantize(const int32_t *q, const float *scales, size_t rows, size_t cols,
                    size_t group_size, float *out) {
  size_t groups_per_row = (cols + group_size - 1) / group_size;
  for (size_t r = 0; r < rows; r++)
    for (size_t c = 0; c < cols; c++)
      out[r * cols + c] = (float)q[r * cols + c] * scales[r * groups_per_row + c / group_size];
}

/* rust/src/backend_cpu.rs:72-78: GEMMA_CPU_THREADS, else the core count. */
int32_t gqo_default_threads(void) {
  const char *e = getenv("GEMMA_CPU_THREADS");
  if (e && *e) {
    char *end = NULL;
    long v = strtol(e, &end, 10);
    if (end && *end == '\0' && v >= 1) return (int32_t)v;
  }
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n >= 1 ? (int32_t)n : 1;
}

/* ---- par_ranges: rust/src/backend_cpu.rs:63-91 ------------------------- */

#define PAR_MIN_WORK (1u << 14)

typedef void (*range_fn)(void *ctx, int64_t start, int64_t end);
typedef struct {
  range_fn f;
  void *ctx;
  int64_t start, end;
} range_job;

static void *range_thread(void *p) {
  range_job *j = (range_job *)p;
  j->f(j->ctx, j->start, j->end);
  return NULL;
}

/* Contiguous chunks of ceil(n/threads) rows, one scoped thread each. Each chunk
 * owns disjoint output rows, so results do not depend on the thread count. */
static void par_ranges(int64_t n, uint64_t work, int32_t threads, range_fn f, void *ctx) {
  if (threads <= 0) threads = gqo_default_threads();
  if (threads > n) threads = (int32_t)n;
  if (threads < 1) threads = 1;
  if (threads == 1 || work < PAR_MIN_WORK) {
    f(ctx, 0, n);
    return;
  }
  int64_t chunk = (n + threads - 1) / threads;
  int64_t njobs = (n + chunk - 1) / chunk;
  pthread_t *tid = (pthread_t *)calloc((size_t)njobs, sizeof(pthread_t));
  range_job *jobs = (range_job *)calloc((size_t)njobs, sizeof(range_job));
  int *started = (int *)calloc((size_t)njobs, sizeof(int));
  for (int64_t i = 0; i < njobs; i++) {
    jobs[i].f = f;
    jobs[i].ctx = ctx;
    jobs[i].start = i * chunk;
    jobs[i].end = (i + 1) * chunk < n ? (i + 1) * chunk : n;
    started[i] = pthread_create(&tid[i], NULL, range_thread, &jobs[i]) == 0;
    if (!started[i]) range_thread(&jobs[i]); /* no thread: run inline */
  }
  for (int64_t i = 0; i < njobs; i++)
    if (started[i]) pthread_join(tid[i], NULL);
  free(started);
  free(jobs);
  free(tid);
}

/* ---- linear: rust/src/backend_cpu.rs:174-222 ---------------------------- */

typedef struct {
  const float *x;
  int64_t t, k;
  const gqo_qweight *w; /* NULL for the f32 branch */
  const float *wf;      /* f32 weight [n,k] */
  float *out_t;         /* [n, t] transposed result */
} linear_ctx;

static void linear_rows(void *p, int64_t start, int64_t end) {
  linear_ctx *c = (linear_ctx *)p;
  const int64_t k = c->k, tt = c->t;
  float *row = (float *)malloc((size_t)(k > 0 ? k : 1) * sizeof(float));
  for (int64_t nn = start; nn < end; nn++) {
    const float *wb;
    if (c->w) {
      /* dequantize the weight row once, reuse for every input row */
      for (int64_t kk = 0; kk < k; kk++) row[kk] = gqo_deq(c->w, nn, kk);
      wb = row;
    } else {
      wb = c->wf + nn * k;
    }
    for (int64_t i = 0; i < tt; i++) {
      const float *xb = c->x + i * k;
      float acc = 0.0f;
      for (int64_t kk = 0; kk < k; kk++) acc += xb[kk] * wb[kk];
      c->out_t[nn * tt + i] = acc;
    }
  }
  free(row);
}

static int32_t linear_impl(const float *x, int64_t t, int64_t k, const gqo_qweight *w,
                           const float *wf, int64_t n, float *y, int32_t threads) {
  if (t < 0 || k < 0 || n < 0) return -1;
  if (t == 0 || n == 0) return 0;
  float *out_t = (t == 1) ? y : (float *)malloc((size_t)(n * t) * sizeof(float));
  linear_ctx c = {x, t, k, w, wf, out_t};
  par_ranges(n, (uint64_t)n * (uint64_t)k * (uint64_t)t, threads, linear_rows, &c);
  if (t != 1) {
    for (int64_t nn = 0; nn < n; nn++)
      for (int64_t i = 0; i < t; i++) y[i * n + nn] = out_t[nn * t + i];
    free(out_t);
  }
  return 0;
}

int32_t gqo_linear(const float *x, int64_t t, int64_t k, const gqo_qweight *w, float *y,
                   int32_t threads) {
  if (!w || w->k != k) return -1;
  return linear_impl(x, t, k, w, NULL, w->n, y, threads);
}

int32_t gqo_linear_f32(const float *x, int64_t t, int64_t k, const float *w, int64_t n,
                       float *y, int32_t threads) {
  return linear_impl(x, t, k, NULL, w, n, y, threads);
}

/* ---- embed_rows: rust/src/backend_cpu.rs:127-137 ------------------------ */
int32_t gqo_embed_rows(const gqo_qweight *table, const uint32_t *ids, int64_t t, float scale,
                       float *out) {
  const int64_t d = table->k;
  for (int64_t i = 0; i < t; i++)
    if ((int64_t)ids[i] >= table->n) return -1;
  for (int64_t i = 0; i < t; i++)
    for (int64_t dd = 0; dd < d; dd++)
      out[i * d + dd] = gqo_deq(table, (int64_t)ids[i], dd) * scale;
  return 0;
}

/* ---- elementwise: rust/src/backend_cpu.rs:55-58, 239-244, 343-350 ------- */
float gqo_gelu_tanh(float v) {
  const float c = sqrtf(2.0f / (float)M_PI);
  return 0.5f * v * (1.0f + tanhf(c * (v + 0.044715f * v * v * v)));
}

void gqo_geglu(const float *gate, const float *up, size_t n, float *out) {
  for (size_t i = 0; i < n; i++) out[i] = gqo_gelu_tanh(gate[i]) * up[i];
}

void gqo_softcap(const float *x, size_t n, float cap, float *out) {
  for (size_t i = 0; i < n; i++) out[i] = cap * tanhf(x[i] / cap);
}

void gqo_slice_cols(const float *x, int64_t rows, int64_t stride, int64_t offset, int64_t width,
                    float *out) {
  for (int64_t r = 0; r < rows; r++)
    memcpy(out + r * width, x + r * stride + offset, (size_t)width * sizeof(float));
}

/* ---- fused-op compositions: rust/src/backend.rs:155-167 ------------------ */
int32_t gqo_linear_geglu(const float *x, int64_t t, int64_t k, const gqo_qweight *wg,
                         const gqo_qweight *wu, float *y, int32_t threads) {
  if (!wg || !wu || wg->n != wu->n) return -1;
  size_t cnt = (size_t)(t * wg->n);
  float *g = (float *)malloc((cnt ? cnt : 1) * sizeof(float));
  float *u = (float *)malloc((cnt ? cnt : 1) * sizeof(float));
  int32_t rc = gqo_linear(x, t, k, wg, g, threads);
  if (rc == 0) rc = gqo_linear(x, t, k, wu, u, threads);
  if (rc == 0) gqo_geglu(g, u, cnt, y);
  free(g);
  free(u);
  return rc;
}

int32_t gqo_linear_gelu_mul_cols(const float *x, int64_t t, int64_t k, const gqo_qweight *w,
                                 const float *b, int64_t b_stride, int64_t offset, float *y,
                                 int32_t threads) {
  if (!w || offset < 0 || offset + w->n > b_stride) return -1;
  size_t cnt = (size_t)(t * w->n);
  float *g = (float *)malloc((cnt ? cnt : 1) * sizeof(float));
  float *s = (float *)malloc((cnt ? cnt : 1) * sizeof(float));
  int32_t rc = gqo_linear(x, t, k, w, g, threads);
  if (rc == 0) {
    gqo_slice_cols(b, t, b_stride, offset, w->n, s);
    gqo_geglu(g, s, cnt, y);
  }
  free(g);
  free(s);
  return rc;
}

/* ---- support ops of the decode step (norms, rope, attention, elementwise) --- */

/* rust/src/backend_cpu.rs:149-172: y = x / sqrt(mean(x^2) + eps) * w per row of
 * d values (w NULL: unweighted). Sequential f32 sum of squares. */
void gqo_rms_norm(const float *x, int64_t rows, int64_t d, const float *w, float eps, float *out) {
  for (int64_t i = 0; i < rows; i++) {
    const float *xr = x + i * d;
    float *o = out + i * d;
    float ss = 0.0f;
    for (int64_t dd = 0; dd < d; dd++) ss += xr[dd] * xr[dd];
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    if (w) {
      for (int64_t dd = 0; dd < d; dd++) o[dd] = xr[dd] * inv * w[dd];
    } else {
      for (int64_t dd = 0; dd < d; dd++) o[dd] = xr[dd] * inv;
    }
  }
}

/* rust/src/backend_cpu.rs:224-235 */
void gqo_add(const float *a, const float *b, size_t n, float *out) {
  for (size_t i = 0; i < n; i++) out[i] = a[i] + b[i];
}
void gqo_mul(const float *a, const float *b, size_t n, float *out) {
  for (size_t i = 0; i < n; i++) out[i] = a[i] * b[i];
}
void gqo_scale(const float *a, size_t n, float s, float *out) {
  for (size_t i = 0; i < n; i++) out[i] = a[i] * s;
}

/* rust/src/backend.rs:137-144: (residual + rms_norm(x, w)) * scale_by[0]. */
void gqo_add_rms_norm(const float *residual, const float *x, int64_t rows, int64_t d, const float *w,
                      float eps, const float *scale_by, float *out) {
  const size_t n = (size_t)(rows * d);
  float *t = (float *)malloc((n ? n : 1) * sizeof(float));
  gqo_rms_norm(x, rows, d, w, eps, t);
  gqo_add(residual, t, n, out);
  if (scale_by) gqo_scale(out, n, scale_by[0], out);
  free(t);
}

/* rust/src/backend_cpu.rs:248-268: half-split partial RoPE on [t, heads, head_dim];
 * the first rotary_dim values of every head rotate, the rest pass through. */
void gqo_rope(const float *x, int64_t t, int64_t heads, int64_t head_dim, const uint32_t *positions,
              float theta, int64_t rotary_dim, float *out) {
  const size_t n = (size_t)(t * heads * head_dim);
  if (out != x) memcpy(out, x, n * sizeof(float));
  const int64_t half = rotary_dim / 2;
  for (int64_t i = 0; i < t; i++) {
    const float pos = (float)positions[i];
    for (int64_t h = 0; h < heads; h++) {
      const int64_t base = (i * heads + h) * head_dim;
      for (int64_t j = 0; j < half; j++) {
        const float freq = powf(theta, -(2.0f * (float)j) / (float)rotary_dim);
        const float ang = pos * freq;
        const float s = sinf(ang), c = cosf(ang);
        const float a = x[base + j], b = x[base + j + half];
        out[base + j] = a * c - b * s;
        out[base + j + half] = b * c + a * s;
      }
    }
  }
}

/* rust/src/backend.rs:148-154: per-head weighted RMSNorm, then rope. */
void gqo_head_norm_rope(const float *x, int64_t t, int64_t heads, int64_t head_dim, const float *w,
                        float eps, const uint32_t *positions, float theta, int64_t rotary_dim,
                        float *out) {
  const size_t n = (size_t)(t * heads * head_dim);
  float *normed = (float *)malloc((n ? n : 1) * sizeof(float));
  gqo_rms_norm(x, t * heads, head_dim, w, eps, normed);
  gqo_rope(normed, t, heads, head_dim, positions, theta, rotary_dim, out);
  free(normed);
}

/* ---- attention: rust/src/backend_cpu.rs:270-336 -------------------------- */

typedef struct {
  const float *q, *k, *v;
  int64_t tt, hq, dh, s, hkv, dv;
  const uint32_t *q_pos, *k_pos;
  float scale;
  uint32_t window;
  float softcap;
  float *out;
} attn_ctx;

static void attn_rows(void *p, int64_t start, int64_t end) {
  attn_ctx *c = (attn_ctx *)p;
  const int64_t s = c->s, hq = c->hq, dh = c->dh, dv = c->dv, hkv = c->hkv, group = hq / hkv;
  float *scores = (float *)malloc((size_t)(s > 0 ? s : 1) * sizeof(float));
  for (int64_t r = start; r < end; r++) {
    const int64_t i = r / hq, h = r % hq;
    const uint32_t qpos = c->q_pos[i];
    const int64_t kvh = h / group;
    const int64_t qb = (i * hq + h) * dh;
    float maxv = -INFINITY;
    for (int64_t j = 0; j < s; j++) {
      const uint32_t kpos = c->k_pos[j];
      /* causal + optional sliding-window mask */
      if (kpos > qpos || (c->window > 0 && qpos - kpos >= c->window)) {
        scores[j] = -INFINITY;
        continue;
      }
      const int64_t kb = (j * hkv + kvh) * dh;
      float dot = 0.0f;
      for (int64_t d = 0; d < dh; d++) dot += c->q[qb + d] * c->k[kb + d];
      dot *= c->scale;
      if (c->softcap > 0.0f) dot = c->softcap * tanhf(dot / c->softcap);
      scores[j] = dot;
      if (dot > maxv) maxv = dot;
    }
    float sum = 0.0f;
    for (int64_t j = 0; j < s; j++) {
      if (scores[j] == -INFINITY) {
        scores[j] = 0.0f;
      } else {
        const float e = expf(scores[j] - maxv);
        scores[j] = e;
        sum += e;
      }
    }
    const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
    float *o = c->out + r * dv;
    for (int64_t d = 0; d < dv; d++) o[d] = 0.0f;
    for (int64_t j = 0; j < s; j++) {
      const float wgt = scores[j] * inv;
      if (wgt == 0.0f) continue;
      const int64_t vb = (j * hkv + kvh) * dv;
      for (int64_t d = 0; d < dv; d++) o[d] += wgt * c->v[vb + d];
    }
  }
  free(scores);
}

int32_t gqo_attention(const float *q, int64_t t, int64_t hq, int64_t dh, const float *k, const float *v,
                      int64_t s, int64_t hkv, int64_t dv, const uint32_t *q_pos, const uint32_t *k_pos,
                      float scale, uint32_t sliding_window, float attn_softcap, float *out,
                      int32_t threads) {
  if (t < 0 || s < 0 || hq <= 0 || hkv <= 0 || hq % hkv != 0) return -1;
  attn_ctx c = {q, k, v, t, hq, dh, s, hkv, dv, q_pos, k_pos, scale, sliding_window, attn_softcap, out};
  if (t == 0) return 0;
  par_ranges(t * hq, (uint64_t)(t * hq) * (uint64_t)s * (uint64_t)(dh + dv), threads, attn_rows, &c);
  return 0;
}

/* ---- sampling (rust/src/sampler.rs) --------------------------------------------- */

/* Rng::next_u64 / next_f64 (sampler.rs:13-26) */
uint64_t gqo_rng_next_u64(uint64_t *state) {
  *state += 0x9e3779b97f4a7c15ull;
  uint64_t z = *state;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

double gqo_rng_next_f64(uint64_t *state) {
  return (double)(gqo_rng_next_u64(state) >> 11) / (double)(1ull << 53);
}

/* softmax_over (sampler.rs:46-54): max by f32::max (NaN ignored), exp((l - max) * inv_t),
 * sequential f32 sum, then each divided by the sum. */
static void softmax_over(const float *l, const int64_t *idx, int64_t n, float inv_t, float *probs) {
  float mx = -INFINITY;
  for (int64_t i = 0; i < n; i++) mx = fmaxf(mx, l[idx[i]]);
  float sum = 0.0f;
  for (int64_t i = 0; i < n; i++) {
    probs[i] = expf((l[idx[i]] - mx) * inv_t);
    sum += probs[i];
  }
  for (int64_t i = 0; i < n; i++) probs[i] /= sum;
}

/* sample_all (sampler.rs:58-69) */
static int32_t sample_all(const float *l, int64_t vocab, float inv_t, double u) {
  float mx = -INFINITY;
  for (int64_t i = 0; i < vocab; i++) mx = fmaxf(mx, l[i]);
  float sum = 0.0f;
  for (int64_t i = 0; i < vocab; i++) sum += expf((l[i] - mx) * inv_t);
  float r = (float)u * sum;
  for (int64_t i = 0; i < vocab; i++) {
    r -= expf((l[i] - mx) * inv_t);
    if (r <= 0.0f) return (int32_t)i;
  }
  return (int32_t)(vocab - 1);
}

/* values[b].partial_cmp(&values[a]) of the descending sorts: Greater / Less / Equal
 * (unordered counts as Equal), as -1 when a goes first. */
static int desc_cmp(const float *v, int64_t a, int64_t b) {
  if (v[a] > v[b]) return -1;
  if (v[a] < v[b]) return 1;
  return 0;
}

/* stable merge sort of idx[0..n) by desc_cmp (Rust's sort_by is stable) */
static void stable_sort_desc(const float *v, int64_t *idx, int64_t n, int64_t *tmp) {
  for (int64_t width = 1; width < n; width *= 2) {
    for (int64_t lo = 0; lo < n; lo += 2 * width) {
      int64_t mid = lo + width < n ? lo + width : n;
      int64_t hi = lo + 2 * width < n ? lo + 2 * width : n;
      int64_t i = lo, j = mid, o = lo;
      while (i < mid && j < hi) tmp[o++] = desc_cmp(v, idx[j], idx[i]) < 0 ? idx[j++] : idx[i++];
      while (i < mid) tmp[o++] = idx[i++];
      while (j < hi) tmp[o++] = idx[j++];
    }
    memcpy(idx, tmp, (size_t)n * sizeof(int64_t));
  }
}

/* top_k_desc (sampler.rs:73-113): a bounded min-heap (heap[0] the smallest), then the
 * stable descending sort of the heap's contents in heap order. Returns k. */
static int64_t top_k_desc(const float *v, int64_t vocab, int64_t k, int64_t *heap, int64_t *tmp) {
  int64_t len = 0;
  for (int64_t i = 0; i < vocab; i++) {
    if (len < k) {
      heap[len++] = i;
      int64_t c = len - 1;
      while (c > 0) { /* sift_up */
        const int64_t parent = (c - 1) / 2;
        if (v[heap[c]] >= v[heap[parent]]) break;
        const int64_t t = heap[c]; heap[c] = heap[parent]; heap[parent] = t;
        c = parent;
      }
    } else if (v[i] > v[heap[0]]) {
      heap[0] = i;
      int64_t c = 0;
      for (;;) { /* sift_down */
        const int64_t l = 2 * c + 1, r = 2 * c + 2;
        int64_t m = c;
        if (l < len && v[heap[l]] < v[heap[m]]) m = l;
        if (r < len && v[heap[r]] < v[heap[m]]) m = r;
        if (m == c) break;
        const int64_t t = heap[c]; heap[c] = heap[m]; heap[m] = t;
        c = m;
      }
    }
  }
  stable_sort_desc(v, heap, len, tmp);
  return len;
}

int32_t gqo_sample(const float *logits, int64_t vocab, float temperature, int64_t top_k, float top_p,
                   float repetition_penalty, const uint32_t *recent, int64_t n_recent, double u) {
  if (!logits || vocab <= 0 || top_k < 0 || n_recent < 0 || (n_recent > 0 && !recent)) return -1;
  float *l = (float *)malloc((size_t)vocab * sizeof(float));
  int64_t *idx = (int64_t *)malloc((size_t)vocab * sizeof(int64_t));
  int64_t *tmp = (int64_t *)malloc((size_t)vocab * sizeof(int64_t));
  float *probs = (float *)malloc((size_t)vocab * sizeof(float));
  int32_t out = -1;
  if (!l || !idx || !tmp || !probs) goto done;
  memcpy(l, logits, (size_t)vocab * sizeof(float));
  /* repetition penalty on the copy, each vocabulary item once (sampler.rs:120-133) */
  if (repetition_penalty != 1.0f && n_recent > 0) {
    for (int64_t j = 0; j < n_recent; j++) {
      const uint32_t tok = recent[j];
      if ((int64_t)tok >= vocab) continue;
      int seen = 0;
      for (int64_t i = 0; i < j && !seen; i++) seen = recent[i] == tok;
      if (seen) continue;
      const float x = l[tok];
      l[tok] = x > 0.0f ? x / repetition_penalty : x * repetition_penalty;
    }
  }
  if (temperature <= 0.0f) { /* greedy (sampler.rs:135-145) */
    int64_t best = 0;
    float bv = -INFINITY;
    for (int64_t i = 0; i < vocab; i++)
      if (l[i] > bv) {
        bv = l[i];
        best = i;
      }
    out = (int32_t)best;
    goto done;
  }
  {
    const float inv_t = 1.0f / temperature;
    if (top_k == 0 && top_p >= 1.0f) {
      out = sample_all(l, vocab, inv_t, u);
      goto done;
    }
    int64_t n;
    if (top_k > 0) {
      n = top_k_desc(l, vocab, top_k < vocab ? top_k : vocab, idx, tmp);
    } else {
      for (int64_t i = 0; i < vocab; i++) idx[i] = i;
      stable_sort_desc(l, idx, vocab, tmp);
      n = vocab;
    }
    if (top_p < 1.0f) {
      softmax_over(l, idx, n, inv_t, probs);
      float cum = 0.0f;
      int64_t keep = 0;
      for (int64_t i = 0; i < n; i++) {
        keep = i + 1;
        cum += probs[i];
        if (cum >= top_p) break;
      }
      n = keep;
    }
    softmax_over(l, idx, n, inv_t, probs);
    float r = (float)u;
    for (int64_t i = 0; i < n; i++) {
      r -= probs[i];
      if (r <= 0.0f) {
        out = (int32_t)idx[i];
        goto done;
      }
    }
    out = (int32_t)idx[n - 1];
  }
done:
  free(l);
  free(idx);
  free(tmp);
  free(probs);
  return out;
}
