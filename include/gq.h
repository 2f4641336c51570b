/*
 * gq.h — C ABI of the B200 quantized-weight backend (libgq.so).
 *
 * This is the drop-in boundary for the quantized-weight hot path of the Gemma-4
 * engine in Dhruba531/gemma-4-webgpu-kernels. Each entry point replaces one
 * method of the Rust `Backend` trait (rust/src/backend.rs:88-180) for quantized
 * tensors; a Rust `CudaBackend` binds these symbols through `extern "C"` (an
 * `extern "C"` block mirroring the declarations below, built by build.rs) and
 * maps a non-zero status to `panic!`, which is what the trait's infallible
 * signatures do today.
 *
 * Conventions
 *  - Every function returns an int status (GQ_OK == 0). Nothing aborts or traps.
 *  - Activation/output pointers are DEVICE pointers owned by the caller. A
 *    gq_qweight owns its device copy of the packed bytes and scales until
 *    gq_qweight_free (the reference's ownership rule, backend_wgpu.rs:25-35).
 *  - All work is enqueued on the context's stream and returns immediately, like
 *    the reference's recorded dispatches; gq_sync / gq_readback block
 *    (backend.rs:169-173).
 *  - One host thread per context (the reference backend is !Sync).
 *  - f32 tensors are dense row-major. Outputs are fully overwritten; nothing
 *    relies on zeroed buffers (backend_wgpu.rs:380-383).
 *  - Kernel-detected errors (an embedding id >= rows, a pipeline wait that
 *    timed out) set a device status word; the next gq_sync returns
 *    GQ_ERR_DEVICE and gq_last_error says which.
 */
#ifndef GQ_H
#define GQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GQ_ABI_VERSION 1

typedef enum gq_status {
  GQ_OK = 0,
  GQ_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape, K mismatch, bad offset */
  GQ_ERR_UNSUPPORTED = 2,      /* bits not in {2,4,8}, K not a multiple of values/byte */
  GQ_ERR_CUDA = 3,             /* CUDA runtime error; text in gq_last_error */
  GQ_ERR_OUT_OF_MEMORY = 4,
  GQ_ERR_DEVICE = 5            /* a kernel reported an error (see gq_last_error) */
} gq_status;

/* Device status bits reported through GQ_ERR_DEVICE. */
#define GQ_DEVERR_BAD_ID 0x1u       /* embed id >= table rows (output row zeroed) */
#define GQ_DEVERR_WAIT_TIMEOUT 0x2u /* a bounded pipeline wait gave up */
#define GQ_DEVERR_SAMPLE_CAP 0x4u   /* a top-p nucleus exceeded the device sampler's candidates */

typedef struct gq_ctx gq_ctx;         /* device + stream + error word + workspace */
typedef struct gq_qweight gq_qweight; /* packed weight resident on the device */
typedef struct gq_graph gq_graph;     /* a recorded, replayable sequence of ops */

int gq_abi_version(void);
const char *gq_status_string(int status);

/* ---- context: replaces WgpuBackend::create (rust/src/backend_wgpu.rs:239-300) */
int gq_ctx_create(int device, gq_ctx **out);
int gq_ctx_destroy(gq_ctx *ctx);
/* Use the caller's cudaStream_t (e.g. torch's current stream); NULL restores the
 * context's own (non-blocking) stream. To run on the legacy default stream pass
 * cudaStreamLegacy ((void*)0x1). */
int gq_ctx_set_stream(gq_ctx *ctx, void *cuda_stream);
void *gq_ctx_get_stream(gq_ctx *ctx);
/* Number of SMs of the context's device (grid sizing; reported by bench tools). */
int gq_ctx_num_sms(gq_ctx *ctx);
const char *gq_last_error(gq_ctx *ctx);

/* ---- sync / memory: replaces Backend::{tensor, zeros, readback, flush,
 *      free_tensor} (rust/src/backend.rs:94-96, :169-179) */
int gq_sync(gq_ctx *ctx);
int gq_alloc(gq_ctx *ctx, size_t bytes, void **dptr);
int gq_free(gq_ctx *ctx, void *dptr);
int gq_memcpy_h2d(gq_ctx *ctx, void *dst_dev, const void *src_host, size_t bytes);
int gq_memcpy_d2h(gq_ctx *ctx, void *dst_host, const void *src_dev, size_t bytes);
int gq_memset(gq_ctx *ctx, void *dst_dev, int value, size_t bytes);
/* Blocking f32 read (Backend::readback, rust/src/backend.rs:171). */
int gq_readback(gq_ctx *ctx, float *dst_host, const float *src_dev, size_t count);

/* ---- weights: replaces Backend::quant_tensor (rust/src/backend.rs:95;
 *      wgpu upload at rust/src/backend_wgpu.rs:442-456). Arguments mirror
 *      QuantWeight (rust/src/backend.rs:16-24): qbytes are the raw payload
 *      (U8 sub-byte packed LSB-first offset-binary, or native I8), scales are
 *      one f32 per (row, group), shape [n, k]. Host pointers; copied. */
int gq_qweight_upload(gq_ctx *ctx, const uint8_t *qbytes, size_t nbytes, const float *scales,
                      size_t nscales, int64_t n, int64_t k, int32_t bits, int32_t signed_i8,
                      int64_t group_size, gq_qweight **out);
/* Same, with the packed bytes already in DEVICE memory (copied device to
 * device; scales are host f32) — WgpuBackend::quant_tensor_from_gpu
 * (rust/src/backend_wgpu.rs:447-456), used when the payload was streamed to the
 * GPU by another path. */
int gq_qweight_upload_device(gq_ctx *ctx, const uint8_t *qbytes_dev, size_t nbytes,
                             const float *scales, size_t nscales, int64_t n, int64_t k,
                             int32_t bits, int32_t signed_i8, int64_t group_size,
                             gq_qweight **out);
int gq_qweight_free(gq_qweight *w);
/* Shape/format of an uploaded weight (any out pointer may be NULL). */
int gq_qweight_info(const gq_qweight *w, int64_t *n, int64_t *k, int32_t *bits,
                    int32_t *signed_i8, int64_t *group_size);

/* ---- record / replay: the reference records every op of a forward pass into
 *      one command encoder and submits it at flush (rust/src/backend_wgpu.rs:
 *      11-15, :562-594). Here the ops issued between gq_graph_begin and
 *      gq_graph_end are captured from the context's stream into a CUDA graph
 *      that gq_graph_launch replays with one call. The context's stream must be
 *      a non-default stream while recording (the context's own stream is). No
 *      synchronising call (gq_sync, gq_readback, uploads) may be made while
 *      recording. */
int gq_graph_begin(gq_ctx *ctx);
int gq_graph_end(gq_ctx *ctx, gq_graph **out);
int gq_graph_launch(gq_ctx *ctx, gq_graph *graph);
int gq_graph_destroy(gq_graph *graph);

/* ---- ops. x is [m, k] f32, y is [m, w.n] f32, all device pointers. */

/* Backend::linear (rust/src/backend.rs:105-106): y = x · deq(W)ᵀ. The wgpu
 * backend dispatches MATMUL_Q / MATMUL_Q_TILED / MATMUL_Q_SCALAR here
 * (rust/src/backend_wgpu.rs:768-806). */
int gq_linear(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w,
              float *y);

/* Backend::linear_geglu (rust/src/backend.rs:155-160; MODE 1 at
 * rust/src/backend_wgpu.rs:808-821): y = gelu_tanh(x·Wgᵀ) * (x·Wuᵀ). */
int gq_linear_geglu(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *wg,
                    const gq_qweight *wu, float *y);

/* Backend::linear_gelu_mul_cols (rust/src/backend.rs:161-167; MODE 2 at
 * rust/src/backend_wgpu.rs:823-835): y = gelu_tanh(x·Wᵀ) * b[:, off:off+n],
 * b is [m, b_stride] f32. */
int gq_linear_gelu_mul_cols(gq_ctx *ctx, const float *x, int64_t m, int64_t k,
                            const gq_qweight *w, const float *b, int64_t b_stride,
                            int64_t b_offset, float *y);

/* lm_head with the final logit soft-cap fused: the composition
 * softcap(linear(x, lm_head), cap) of rust/src/model.rs:192 and
 * Backend::softcap (rust/src/backend.rs:116). cap <= 0 means no cap. The
 * output row stride is ldy floats and the n results of each row are written at
 * column y_col0 (a vocab shard writing into its slice of the full logits). */
int gq_linear_softcap(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w,
                      float cap, float *y, int64_t ldy, int64_t y_col0);

/* The lm_head of a vocab-sharded model with its all-gather fused in: the same
 * output as gq_linear_softcap (rows of w = this rank's vocab shard, written at
 * columns y_col0 .. y_col0 + N of the [m, ldy] logits), and every element is also
 * stored at the same offset of each peer_y[i] — other GPUs' logits buffers mapped
 * into this device (gq_ipc_open) — by the GEMV epilogue itself, over NVLink.
 * After the call, a stream-ordered collective on every rank (any NCCL op) makes
 * the full logits complete on all of them. 0 <= npeers <= 8; M < 128 and shapes
 * served by the GEMV kernels only (GQ_ERR_UNSUPPORTED otherwise). No counterpart
 * in the reference (its lm_head runs on one device); replaces the NCCL all-gather
 * of vocab sharding (rust/src/model.rs:192 is the op itself). */
int gq_linear_softcap_peers(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w, float cap,
                            float *y, int64_t ldy, int64_t y_col0, float *const *peer_y, int32_t npeers);

/* The same call with the completion barrier fused in as well: flags[0] is this
 * rank's array of `world` uint32 flags and flags[1 + i] the array of the rank
 * that owns peer_y[i] (gq_ipc_open'd); sync is a zeroed pair of uint32 on this
 * device {CTA counter, epoch}. The last CTA of the GEMV (after every CTA's peer
 * stores and a system fence) increments the epoch and stores it at element
 * `rank` of every rank's flag array; gq_peer_wait then holds the stream
 * (bounded) until all of this rank's flags have reached the epoch, so no NCCL
 * call is needed. The epoch is device-resident: the pair of calls can be
 * captured in a graph and replayed. After a device error the flags and sync
 * words must be re-zeroed on every rank. No counterpart in the reference (see
 * gq_linear_softcap_peers). */
int gq_linear_softcap_peers_signal(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w,
                                   float cap, float *y, int64_t ldy, int64_t y_col0, float *const *peer_y,
                                   int32_t npeers, uint32_t *const *flags, uint32_t *sync, int32_t rank);

/* gq_linear_softcap_peers_signal with the completion wait folded into the same
 * launch: after publishing the epoch, the GEMV's last CTA waits (acquire, system
 * scope, bounded by the context's wait limit -> GQ_DEVERR_WAIT_TIMEOUT) until every
 * rank's flag in flags[0] has reached it, so the kernel completes only when the
 * full logits are on this rank and no gq_peer_wait launch follows. Same arguments
 * and set-up. No counterpart in the reference. */
int gq_linear_softcap_peers_sync(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w,
                                 float cap, float *y, int64_t ldy, int64_t y_col0, float *const *peer_y,
                                 int32_t npeers, uint32_t *const *flags, uint32_t *sync, int32_t rank);

/* Stream-ordered wait until flags[0 .. world) have all reached the epoch in
 * sync[1] (acquire, system scope). A wait that runs past the context's wait
 * limit (2 s unless gq_ctx_set_wait_limit changed it) sets
 * GQ_DEVERR_WAIT_TIMEOUT in the context's device error word (read by the next
 * gq_sync) and returns; the context stays usable. */
int gq_peer_wait(gq_ctx *ctx, const uint32_t *flags, int32_t world, const uint32_t *sync);

/* Bound of the cross-GPU waits of this context (gq_peer_wait) and of the
 * inter-CTA waits of a decode chain (gq_chain_run), in nanoseconds, 1 ms .. 60 s;
 * applies to waits enqueued afterwards (a captured graph keeps the bound it was
 * recorded with). The failure detector of a multi-GPU caller: a rank that dies
 * or stalls makes its peers' waits end with GQ_DEVERR_WAIT_TIMEOUT after this
 * long instead of hanging their GPUs. No counterpart in the reference (single
 * device). */
int gq_ctx_set_wait_limit(gq_ctx *ctx, uint64_t limit_ns);

/* ---- decode chains: consecutive one-row MATMUL_Q calls in one launch.
 * The reference records each call as its own dispatch in one compute pass
 * (rust/src/backend_wgpu.rs:311-367, :768-835); a chain gives the results of
 * issuing its ops one after another on the context's stream (each op may read
 * what the ops before it wrote), from a single persistent kernel that streams
 * the weights of later ops while earlier ones wait for their inputs. Every op
 * has ONE activation row (m = 1): x is [k] and y is [w.n], device pointers fixed
 * when the chain is created (bind the decode step's buffers once). Modes:
 *   0  gq_linear                       y = x · deq(W)ᵀ
 *   1  gq_linear_geglu                 y = gelu_tanh(x·Wᵀ) * (x·W2ᵀ)   (w2 = up)
 *   2  gq_linear_gelu_mul_cols         y = gelu_tanh(x·Wᵀ) * b[b_offset + j]
 *   3  gq_linear_softcap               y = cap·tanh((x·Wᵀ)/cap), cap <= 0: none
 * Requirements (GQ_ERR_UNSUPPORTED otherwise): one scale per weight row
 * (group_size = k), rows a whole number of 16 bytes, k a multiple of 4, x 16-byte
 * aligned, a row that fits the kernel's 24 KB ring slot. y must not overlap the
 * op's x or b (GQ_ERR_INVALID_ARGUMENT). Results agree with the single calls to
 * the GEMV tolerance (the same dequantising arithmetic; sums grouped per CTA).
 * One chain runs at a time per stream; all of its CTAs are resident at once (a
 * cooperative launch of one CTA per SM). Waits between CTAs are bounded by the
 * context's wait limit: a timeout reports GQ_DEVERR_WAIT_TIMEOUT at the next
 * gq_sync, and the chain then needs gq_chain_reset before it runs again. A chain
 * may be captured by gq_graph_begin/end; destroy it only after the last graph
 * that holds it. No counterpart in the reference. */
typedef struct gq_chain gq_chain;
typedef struct gq_chain_op {
  int32_t mode;
  const gq_qweight *w;
  const gq_qweight *w2; /* mode 1: the up weight (same shape and format as w) */
  const float *x;       /* [w.k] */
  float *y;             /* [w.n] */
  const float *b;       /* mode 2: the columns b[b_offset .. b_offset + w.n) */
  int64_t b_offset;
  float cap;            /* mode 3 */
} gq_chain_op;
int gq_chain_create(gq_ctx *ctx, const gq_chain_op *ops, int32_t n_ops, gq_chain **out);
int gq_chain_run(gq_chain *chain);
int gq_chain_reset(gq_chain *chain);
int gq_chain_destroy(gq_chain *chain);

/* Greedy decoding over a vocab shard: for each of the m rows of x (row stride
 * ldx floats, 0 = n) the largest of its n values and the first column holding it
 * (NaN ranks above every number, -0 equals +0: numpy.argmax), written as val[row]
 * and idx[row] = idx_base + column. With idx_base = the shard's first vocab row,
 * the best of the ranks' (val, idx) pairs (ties to the smaller index) is the
 * argmax of the full logits, so a vocab-sharded lm_head exchanges m pairs per
 * rank instead of its logits. Uses the context workspace (m * 8 bytes). No
 * counterpart in the reference (its sampler reads the whole logits row,
 * rust/src/sampler.rs). */
int gq_argmax_rows(gq_ctx *ctx, const float *x, int64_t m, int64_t n, int64_t ldx, int64_t idx_base, float *val,
                   int64_t *idx);

/* ---- sampling: the reference's sampler (rust/src/sampler.rs:116-190) on the
 *      device, so a decode step reads back token ids, not logits rows. */
/* SampleOpts (rust/src/sampler.rs:29-39): temperature <= 0 is greedy; top_k = 0
 * disables top-k (1..256 on the device); top_p >= 1 disables top-p;
 * repetition_penalty = 1 disables the penalty. */
typedef struct gq_sample_opts {
  float temperature;
  int32_t top_k;
  float top_p;
  float repetition_penalty;
} gq_sample_opts;

/* sample() for each of the m rows of logits [m, vocab] (row stride ld floats, 0 =
 * vocab): the repetition penalty over recent[row * recent_stride .. + n_recent)
 * (device u32 ids; 0 <= n_recent <= 4096; ids >= vocab ignored; each distinct id
 * once; the logits are not modified), then greedy, sample_all, or top-k / top-p
 * over the sorted candidates (ties to the smaller id), the draw being
 * Rng::next_f64 of rng_state[row] (device u64 splitmix64 states, advanced in place
 * by every non-greedy row, as the reference's Rng). tokens[row] (device int32)
 * receives the id. top_k = 0 with top_p < 1 keeps the 256 largest as candidates
 * (with the whole row's softmax denominator): a row whose nucleus needs more gets
 * -1 and raises GQ_DEVERR_SAMPLE_CAP at the next gq_sync. Sums over a whole row are
 * chunked (a draw within f32 rounding of a token boundary may pick its
 * neighbour); the candidate arithmetic is the reference's sequential f32 order.
 * Uses the context workspace. No counterpart in the reference's backend (its
 * sampler reads the logits back, rust/src/engine.rs:207-215). */
int gq_sample_rows(gq_ctx *ctx, const float *logits, int64_t m, int64_t vocab, int64_t ld,
                   const gq_sample_opts *opts, const uint32_t *recent, int64_t n_recent,
                   int64_t recent_stride, uint64_t *rng_state, int32_t *tokens);

/* The k largest (1 <= k <= 256) of each row of a vocab shard's logits [m, n] (row
 * stride ld, 0 = n), after the repetition penalty (ids relative to the whole
 * vocabulary: column c is id idx_base + c), sorted by value, ties to the smaller id:
 * val [m, k] f32 and idx [m, k] int64 (device; -inf / -1 past the row's end). The
 * union of every shard's top k holds the whole vocabulary's top k, so a
 * vocab-sharded lm_head exchanges G * k pairs per row (any all-gather) and samples
 * them with gq_sample_candidates. Uses the context workspace. No counterpart in the
 * reference. */
int gq_topk_rows(gq_ctx *ctx, const float *logits, int64_t m, int64_t n, int64_t ld, int64_t idx_base,
                 int32_t k, float repetition_penalty, const uint32_t *recent, int64_t n_recent,
                 int64_t recent_stride, float *val, int64_t *idx);

/* Greedy or top-k (+ top-p) sampling of rows given as candidate pairs val/idx
 * [m, ncand] (device; idx -1 = none; 1 <= ncand <= 4096), e.g. every rank's
 * gq_topk_rows output gathered: the candidates are sorted (value, then smaller
 * id) and sampled as gq_sample_rows does with the same options (penalty already
 * applied by gq_topk_rows). Modes that need the whole row's softmax (top_k = 0
 * with temperature > 0) return GQ_ERR_UNSUPPORTED. No counterpart in the
 * reference. */
int gq_sample_candidates(gq_ctx *ctx, const float *val, const int64_t *idx, int64_t m, int64_t ncand,
                         const gq_sample_opts *opts, uint64_t *rng_state, int32_t *tokens);

/* CUDA IPC for the peer buffers above: the 64-byte handle of a gq_alloc'd device
 * buffer, the mapping of a peer's handle into this context's device (peer access
 * enabled), and its release. */
int gq_ipc_get_handle(gq_ctx *ctx, void *dptr, uint8_t *handle64);
int gq_ipc_open(gq_ctx *ctx, const uint8_t *handle64, void **dptr);
int gq_ipc_close(gq_ctx *ctx, void *dptr);

/* ---- checkpoint loading: the reference's safetensors reader and quantized-weight
 *      construction (rust/src/safetensors.rs, rust/src/weights.rs:37-118), on the
 *      host side of this library, so a caller without the Rust loader (C, Python)
 *      reads the real QAT checkpoint layout straight into gq_qweight objects. */
typedef struct gq_st_file gq_st_file; /* a parsed safetensors file */

/* Memory-map a safetensors file read-only and parse its header (parse_header,
 * rust/src/safetensors.rs:52-72: [u64 LE header length][JSON header][payload];
 * __metadata__ skipped). Tensor bytes are read only when used. */
int gq_st_open(const char *path, gq_st_file **out);
/* Same over a caller-owned blob in host memory (kept referenced until gq_st_close). */
int gq_st_open_memory(const uint8_t *bytes, size_t nbytes, gq_st_file **out);
int gq_st_close(gq_st_file *f);
/* Tensor count and the i-th name (names sorted; the pointer lives as long as f). */
int64_t gq_st_count(const gq_st_file *f);
const char *gq_st_name(const gq_st_file *f, int64_t i);
/* dtype (NUL-terminated, 16 bytes), shape (up to 8 dims), the payload slice inside the
 * mapping and its size (offsets checked against the file: raw_bytes,
 * rust/src/safetensors.rs:154-163). Any out pointer may be NULL. */
int gq_st_info(const gq_st_file *f, const char *name, char *dtype16, int64_t *shape8, int32_t *ndim,
               const uint8_t **data, size_t *nbytes);
/* decode_to_f32 (rust/src/safetensors.rs:98-105) of an F32 / F16 / BF16 tensor of
 * exactly `count` elements into host memory. */
int gq_st_read_f32(const gq_st_file *f, const char *name, float *dst_host, size_t count);
/* Gemma4Config::bits_for (rust/src/config.rs:161-169): the bits of the first pattern
 * (ECMAScript regex, searched anywhere in name) that matches, 16 when none does, -1
 * for a bad pattern or argument. */
int32_t gq_bits_for(const char *name, const char *const *patterns, const int32_t *bits, int32_t nrules);
/* resolve_tensor_names (rust/src/weights.rs:37-48): the on-disk weight, scale and bare
 * names (256-byte buffers; bare is "" when there is none) of a logical weight name. */
int gq_st_resolve(const char *logical, char *weight256, char *scale256, char *bare256);
/* ModelWeights::load for a quantized tensor (rust/src/weights.rs:86-110): the U8 / I8
 * payload of `logical` (resolved as above, falling back to the bare name) and its F32
 * / F16 / BF16 scale become a weight with bits = 8 for I8 else bits_u8 (the caller's
 * gq_bits_for of the logical name without ".weight"), K = stored columns x values per
 * byte and group_size = K / scale columns, uploaded with gq_qweight_upload. */
int gq_st_upload_quant(gq_ctx *ctx, const gq_st_file *f, const char *logical, int32_t bits_u8, gq_qweight **out);

/* Backend::embed_rows for a quantized table (rust/src/backend.rs:101-102;
 * CPU rust/src/backend_cpu.rs:127-137, wgpu EMBED_Q at
 * rust/src/backend_wgpu.rs:734-754): out[i, d] = deq(table, ids[i], d) * scale.
 * ids is a DEVICE array of t u32. An id >= table rows zeroes that output row
 * and raises GQ_DEVERR_BAD_ID at the next gq_sync. */
int gq_embed_rows(gq_ctx *ctx, const gq_qweight *table, const uint32_t *ids, int64_t t,
                  float scale, float *out);

/* Allocation-free prefill linear. No counterpart in the reference: it exists for
 * callers that cannot allocate device memory when they call (a serving process
 * that reserves all of its HBM at start-up and must not cudaMalloc afterwards,
 * or an embedder whose buffers all come from its own arena), and who therefore
 * cannot create a gq_ctx either. y[m, n] = x' · deq(W)ᵀ, x' = x rounded to f16
 * after a power-of-two scaling per row (undone exactly), with the same
 * tensor-core kernel as gq_linear uses for m >= 128 (any m >= 1 is accepted).
 * Weights are caller device pointers in the upload layout: qbytes [n, row_bytes]
 * (16-byte aligned), one f32 scale per row. Requires k % 64 == 0,
 * m * k <= 4,194,304 (GQ_ERR_INVALID_ARGUMENT beyond) and n <= 8,388,480
 * (GQ_ERR_UNSUPPORTED beyond): the f16 copy of x goes to a file-scope 8 MiB device
 * array (plus 256 KB of row exponents) that every GPU loading the library holds
 * until exit. Nothing is allocated by the call.
 * Set-up: the first call on a device looks up the arrays' device addresses
 * (cudaGetSymbolAddress, once per device, thread-safe). Under CUDA's lazy module
 * loading (the default) that first call is also when the arrays and the kernels
 * are placed in device memory, so make it at start-up — a small valid call, e.g.
 * m = 1 — before reserving the rest of HBM and before any stream capture, or run
 * with CUDA_MODULE_LOADING=EAGER.
 * All calls share the arrays and each leaves its scratch behind: calls that
 * overlap on the GPU (different streams, concurrent) race on them. Work is
 * enqueued on cuda_stream (NULL = legacy default stream) of the current device.
 * A pipeline wait that gave up (bounded at 2 s) leaves y incomplete and sets
 * GQ_DEVERR_WAIT_TIMEOUT in a device status word that
 * gq_linear_prefill_static_status reports. */
int gq_linear_prefill_static(void *cuda_stream, const float *x, int64_t m, int64_t k,
                             const uint8_t *qbytes, const float *scales, int64_t n, int32_t bits,
                             int32_t signed_i8, float *y);
/* Status of the allocation-free calls on the current device: synchronises
 * cuda_stream, stores the GQ_DEVERR_* bits raised since the last read in
 * *status_bits, clears them, and returns GQ_ERR_DEVICE when any was set
 * (GQ_OK otherwise). Allocates nothing. No counterpart in the reference. */
int gq_linear_prefill_static_status(void *cuda_stream, uint32_t *status_bits);

/* Backend::softcap / geglu / gelu_tanh (rust/src/backend.rs:112-116) on n
 * f32 elements. */
int gq_softcap(gq_ctx *ctx, const float *x, int64_t n, float cap, float *y);
int gq_geglu(gq_ctx *ctx, const float *gate, const float *up, int64_t n, float *y);

/* ---- support ops of a decode step ----------------------------------------------
 * The non-quantized methods of the Backend trait that a Gemma-4 decode step runs
 * between the MATMUL_Q calls (rust/src/backend.rs:103-154; CPU semantics in
 * rust/src/backend_cpu.rs:149-336). All pointers are device pointers; f32
 * tensors are dense row-major unless a stride says otherwise. */

/* Backend::rms_norm (rust/src/backend.rs:103-104; CPU rust/src/backend_cpu.rs:149-172):
 * y = x / sqrt(mean(x^2) + eps) * w per row of d values; w NULL is the unweighted
 * variant. Output row r starts at y + r * y_stride (0 = d), which lets a value row
 * land directly in its KV-cache slot. */
int gq_rms_norm(gq_ctx *ctx, const float *x, int64_t rows, int64_t d, const float *w, float eps, float *y,
                int64_t y_stride);

/* Backend::add_rms_norm (rust/src/backend.rs:137-144): y = (residual + rms_norm(x, w))
 * * scale_by[0]; scale_by is a device scalar or NULL. */
int gq_add_rms_norm(gq_ctx *ctx, const float *residual, const float *x, int64_t rows, int64_t d, const float *w,
                    float eps, const float *scale_by, float *y);

/* add_rms_norm followed by rms_norm of its result (the post-norm + residual of one
 * block and the input norm of the next: rust/src/model.rs:219 then :223, and :236
 * then the next layer's :214), in one pass: h = (residual + rms_norm(x, w1)) * scale_by[0],
 * xn = rms_norm(h, w2). Results equal the two calls exactly. h may alias residual. */
int gq_add_rms_norm_norm(gq_ctx *ctx, const float *residual, const float *x, int64_t rows, int64_t d, const float *w1,
                         float eps, const float *scale_by, const float *w2, float *h, float *xn);

/* One decode row (m = 1): the residual add + RMSNorm that precedes a projection
 * (rust/src/model.rs:219+223 before the MLP, :233 before the per-layer-input
 * gate, :236 + the next layer's :214 before its q/k/v), fused into that
 * projection's launch. h_out = (residual + rms_norm(x, w_norm)) * scale_by[0]
 * (scale_by may be NULL), the row the projection reads is
 * w_norm2 ? rms_norm(h_out, w_norm2) : h_out, and y = that row times w in
 * `mode` 0 (gq_linear), 1 (gq_linear_geglu, w_up = up) or 2
 * (gq_linear_gelu_mul_cols on b's columns from b_offset). h_out and the row
 * equal gq_add_rms_norm / gq_add_rms_norm_norm bit for bit (k a multiple of 4,
 * 16-byte aligned rows); y equals the CUDA-core GEMV's gq_linear of that row. Every
 * CTA of the GEMV makes the row itself, so the separate norm launch goes away.
 * Where that path does not apply (k not a multiple of 4 or above 4096, unaligned
 * rows, a weight the streaming GEMV does not serve) the call runs the norm and
 * the projection as their own calls, with the same results. k must equal w.k;
 * h_out and y must not overlap x or residual (GQ_ERR_INVALID_ARGUMENT). */
int gq_add_norm_linear(gq_ctx *ctx, int32_t mode, const float *x, const float *residual, int64_t k,
                       const float *w_norm, float eps, const float *scale_by, const float *w_norm2, float *h_out,
                       const gq_qweight *w, const gq_qweight *w_up, const float *b, int64_t b_offset, float *y);

/* Backend::head_norm_rope (rust/src/backend.rs:148-154) and Backend::rope
 * (rust/src/backend.rs:118-119; CPU rust/src/backend_cpu.rs:248-268) on x [t, heads,
 * head_dim]: per-head weighted RMSNorm (head_norm_rope only), then the half-split
 * rotation of the first rotary_dim values at positions[t] (device u32). Token i's
 * heads are written at y + i * y_tok_stride (0 = heads * head_dim), so a key row can
 * be written straight into a KV cache. rotary_dim must be even and <= 512. */
int gq_head_norm_rope(gq_ctx *ctx, const float *x, int64_t t, int64_t heads, int64_t head_dim, const float *w,
                      float eps, const uint32_t *positions, float theta, int64_t rotary_dim, float *y,
                      int64_t y_tok_stride);
/* The attention inputs of a KV layer in one launch, on the stacked q|k|v
 * projection output qkv [t, (hq + 2 hkv) * head_dim] (token stride qkv_tok_stride,
 * 0 = packed): q = head_norm_rope(q rows, q_w), k = head_norm_rope(k rows, k_w) and
 * v = rms_norm(v rows, no weight) per head, the composition of
 * rust/src/model.rs:258-273 (the three Backend::head_norm_rope / rms_norm calls).
 * Each output token i is written at out + i * out_tok_stride (0 = packed), so the
 * key and value rows can go straight into a KV cache. Same arithmetic as the
 * separate calls (bit-identical). head_dim a multiple of 4 up to 512. */
int gq_qkv_norm_rope(gq_ctx *ctx, const float *qkv, int64_t t, int64_t qkv_tok_stride, int64_t hq, int64_t hkv,
                     int64_t head_dim, const float *q_w, const float *k_w, float eps, const uint32_t *positions,
                     float theta, int64_t rotary_dim, float *q_out, int64_t q_tok_stride, float *k_out,
                     int64_t k_tok_stride, float *v_out, int64_t v_tok_stride);
int gq_rope(gq_ctx *ctx, const float *x, int64_t t, int64_t heads, int64_t head_dim, const uint32_t *positions,
            float theta, int64_t rotary_dim, float *y, int64_t y_tok_stride);

/* Key positions are strictly ascending (a KV cache's are): the causal and sliding-window
 * bounds are then found by binary search and masked keys are never read. */
#define GQ_ATTN_KPOS_ASCENDING 0x1u
/* Key j is at position j (k_pos may be NULL): a KV cache indexed by position. The
 * visible range is then computed without reading k_pos. Implies ascending. */
#define GQ_ATTN_KPOS_IDENTITY 0x2u

/* Backend::attention (rust/src/backend.rs:120-121; CPU rust/src/backend_cpu.rs:270-336),
 * over `batch` independent sequences: q [batch, t, hq, head_dim], k and v of sequence b
 * at k + b * kv_batch_stride as [s, hkv, head_dim], q_pos [batch * t], k_pos of
 * sequence b at k_pos + b * kpos_batch_stride ([s]). Causal + optional sliding window
 * (a key is visible when kpos <= qpos and qpos - kpos < window), scores * scale,
 * optional tanh soft-cap, softmax, weighted sum of v -> out [batch * t, hq * head_dim].
 * A query with no visible key gets zeros. batch = 1, kv_batch_stride = 0 is the
 * trait's call. Requires hq / hkv <= 8, head_dim % 4 == 0 and <= 1024, 16-byte
 * aligned q/k/v/out and kv_batch_stride % 4 == 0. Long key ranges are split over
 * several CTAs whose partial results live in the context workspace. */
int gq_attention(gq_ctx *ctx, const float *q, int64_t batch, int64_t t, int64_t hq, int64_t head_dim, const float *k,
                 const float *v, int64_t s, int64_t hkv, int64_t kv_batch_stride, const uint32_t *q_pos,
                 const uint32_t *k_pos, int64_t kpos_batch_stride, float scale, uint32_t sliding_window,
                 float attn_softcap, uint32_t flags, float *out);

/* Backend::linear with a plain weight (the CpuBackend non-quant branch of
 * rust/src/backend_cpu.rs:174-222), weight stored as bf16 [n, k]: exact for weights
 * that are bf16 on disk (Gemma-4's per_layer_model_projection, rust/src/weights.rs:11-14).
 * y [m, n] = x [m, k] . w^T in f32. */
int gq_linear_bf16(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const uint16_t *w, int64_t n, float *y);

/* Backend::add / mul / scale / scale_by_tensor (rust/src/backend.rs:107-111; CPU
 * rust/src/backend_cpu.rs:224-235) on n elements; s of scale_by_tensor is a device scalar. */
int gq_add(gq_ctx *ctx, const float *a, const float *b, int64_t n, float *y);
int gq_mul(gq_ctx *ctx, const float *a, const float *b, int64_t n, float *y);
int gq_scale(gq_ctx *ctx, const float *a, int64_t n, float s, float *y);
int gq_scale_by_tensor(gq_ctx *ctx, const float *a, int64_t n, const float *s, float *y);

/* Strided row copy dst[r * dst_stride + c] = src[r * src_stride + c]: slice_rows,
 * slice_cols, concat_rows and kv_append of rust/src/backend.rs:122-130. */
int gq_copy_rows(gq_ctx *ctx, const float *src, int64_t rows, int64_t cols, int64_t src_stride, float *dst,
                 int64_t dst_stride);

#ifdef __cplusplus
}
#endif
#endif /* GQ_H */
