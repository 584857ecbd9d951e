/*
 * indecis_b200 — C ABI of the B200 (sm_100a) int8 ModernBERT encoder.
 *
 * This is the drop-in boundary for the int8 inference path of
 * github.com/bornholm/indecis (paths relative to that module). The seam is
 * internal/modernbert/infer.go:304 `func (m *Model) run(seqs [][]int32,
 * done func(xn []float32, offs []int)) error`, the single place where the
 * int8 forward runs; a cgo file under the build tag indecisgpu
 * (go/internal/modernbert/infer_gpu.go in this repository) gives it a device
 * branch that calls ig_encode. Plain pointers and sizes only; no allocation is
 * handed to the caller. All entry points are reentrant: a model is read-only after
 * creation and every call takes its own workspace and stream.
 *
 * Status codes: 0 on success, otherwise an IG_ERR_* value; ig_last_error()
 * gives the message of the calling thread's last failure.
 */
#ifndef INDECIS_B200_H
#define INDECIS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define IG_API __attribute__((visibility("default")))
#else
#define IG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define IG_OK 0
#define IG_ERR_BAD_ARG 1      /* inconsistent sizes or pointers (the reference panics or errors) */
#define IG_ERR_OUT_OF_VOCAB 2 /* "modernbert: id %d out of vocabulary" (infer.go:310-312) */
#define IG_ERR_CUDA 3         /* a CUDA call failed */
#define IG_ERR_TIMEOUT 4      /* a kernel's bounded wait ran out */
#define IG_ERR_UNSUPPORTED 5  /* a shape this build does not handle */
#define IG_ERR_NO_DEVICE 6    /* no usable sm_100 device */

#define IG_MODE_POOLED 0 /* EncodeSeqs: [nseq][hidden], mean or first token */
#define IG_MODE_TOKENS 1 /* EncodeTokens: [sum of lengths][hidden] */

#define IG_POOL_MEAN 0
#define IG_POOL_CLS 1

/* modernbert.Config (internal/modernbert/model.go:25-49), the fields that
 * determine the computation. Biases are not supported, as in validate()
 * (model.go:64-80). simd_lanes is the float32 lane count whose summation
 * order LayerNorm and ExpShift reproduce (8: the reference on AVX2). */
typedef struct ig_config {
  int32_t vocab, hidden, layers, heads, intermediate;
  int32_t global_every;    /* global_attn_every_n_layers */
  int32_t local_attention; /* total window width; half-window = local_attention / 2 */
  int32_t pooling;         /* IG_POOL_MEAN or IG_POOL_CLS */
  double norm_eps, global_theta, local_theta;
  int32_t simd_lanes;
} ig_config;

/* Float32 host views in transformers layouts (FromTensors, model.go:179-234).
 * Per-layer arrays have `layers` entries; attn_norm[0] is ignored (layer 0
 * has no attention norm). Weights are copied; the views are not retained. */
typedef struct ig_weights {
  const float *tok_embeddings; /* [vocab][hidden] embeddings.tok_embeddings.weight, or NULL when
                                  ig_model_set_embeddings supplies the table */
  const float *emb_norm;       /* [hidden] embeddings.norm.weight */
  const float *final_norm;     /* [hidden] final_norm.weight */
  const float *const *attn_norm; /* [hidden] layers.%d.attn_norm.weight */
  const float *const *wqkv;      /* [3*hidden][hidden] layers.%d.attn.Wqkv.weight */
  const float *const *wo;        /* [hidden][hidden] layers.%d.attn.Wo.weight */
  const float *const *mlp_norm;  /* [hidden] layers.%d.mlp_norm.weight */
  const float *const *wi;        /* [2*intermediate][hidden] layers.%d.mlp.Wi.weight (input, then gate) */
  const float *const *wo_mlp;    /* [hidden][intermediate] layers.%d.mlp.Wo.weight */
} ig_weights;

/* A decision head (heads.go:19-27): `rows` logits z = W.x + b over the pooled
 * vector, or over every token state when per_token (Spans). */
typedef struct ig_head {
  int32_t rows;
  int32_t per_token;
  const float *w; /* [rows][hidden] */
  const float *b; /* [rows] */
} ig_head;

typedef struct ig_model ig_model;

/* Embedding table formats (embeddings.go:9-68). */
#define IG_EMB_F32 0  /* float32 [vocab][hidden] */
#define IG_EMB_BF16 1 /* bf16 [vocab][hidden] (value = bits << 16), with float32 rows for some ids */
#define IG_EMB_INT8 2 /* int8 [vocab][hidden] times a float32 scale per row */

/* An embedding table as the reference's mappedEmbeddings holds it
 * (newMappedEmbeddings, newInt8Embeddings: embeddings.go:24-47). Only the
 * fields of `format` are read. */
typedef struct ig_embedding_table {
  int32_t format;
  const float *f32;         /* IG_EMB_F32: [vocab][hidden] */
  const uint16_t *bf16;     /* IG_EMB_BF16: [vocab][hidden] bf16 bits */
  int32_t n_exact;          /* IG_EMB_BF16: rows kept in float32 */
  const int32_t *exact_ids; /* [n_exact] token ids, each in [0, vocab) */
  const float *exact_rows;  /* [n_exact][hidden] */
  const int8_t *i8;         /* IG_EMB_INT8: [vocab][hidden] */
  const float *scale;       /* IG_EMB_INT8: [vocab] */
} ig_embedding_table;

/* Replaces modernbert.FromTensors + SetInt8(true) + the first-use packing
 * (infer.go:119-135, :184-219): validates the config, uploads the weights to
 * `device` and quantizes each layer matrix per output channel (PackB8,
 * linalg/int8.go:36-77) on the device. */
IG_API int ig_model_create(const ig_config *cfg, const ig_weights *w, int32_t device, ig_model **out);

/* Tensor dtypes as a safetensors file stores them (safetensors.go:200-245). */
#define IG_DT_F32 0
#define IG_DT_BF16 1 /* value = bits << 16 */
#define IG_DT_F16 2  /* IEEE binary16, widened exactly */
#define IG_DT_I8 3   /* the integer's value */

/* A host tensor in its stored dtype. */
typedef struct ig_tensor {
  int32_t dtype; /* IG_DT_* */
  const void *data;
} ig_tensor;

/* The layer tensors of a model as its file stores them (Load reads every
 * tensor but the embedding table decoded to float32, model.go:661-735, and
 * the layer matrices lazily through SetCompact). Shapes as ig_weights;
 * attn_norm[0] is ignored. The embedding table comes separately, as stored,
 * through ig_model_set_embeddings (required before encoding). */
typedef struct ig_stored_weights {
  ig_tensor emb_norm, final_norm;
  const ig_tensor *attn_norm, *wqkv, *wo, *mlp_norm, *wi, *wo_mlp; /* [layers] */
} ig_stored_weights;

/* ig_model_create from tensors as stored: each is copied to the device in
 * its own dtype (half the bytes of float32 for bf16 checkpoints) and decoded
 * there exactly as the reference's safetensors reader decodes it (decode,
 * safetensors.go:218-245) before PackB8; the result is bit-identical to
 * ig_model_create on the decoded float32 tensors. Errors: IG_ERR_BAD_ARG for
 * a missing tensor or an unknown dtype. */
IG_API int ig_model_create_stored(const ig_config *cfg, const ig_stored_weights *w, int32_t device, ig_model **out);

/* ig_model_create on several GPUs of this process: one replica of the
 * weights per listed device. The host entry points (ig_encode, ig_logits,
 * ig_window_logits, ig_infer_windows, the batcher) split each call's
 * sequences into contiguous ranges balanced by cost (GEMM work ~ n,
 * attention ~ n x keys per query), encode every range on its own GPU from
 * its own host thread, and write each range's rows into its slice of the
 * caller's output: no collective, no peer memory. Calls under 8192 rows per
 * GPU use fewer GPUs, those with the fewest calls in flight. Results are
 * bit-identical to one device's (sequences are independent:
 * linalg/int8_test.go:149, concurrency_test.go:51-60). This is the batch
 * sharding across the GPUs of one box that EncodeSeqs' callers
 * (model.go:391-426, batch.go:24-81) reach with no change. One device listed:
 * the same as ig_model_create. The device-buffer entry points
 * (ig_encode_device, ig_logits_device) take a replica (ig_model_replica). */
IG_API int ig_model_create_multi(const ig_config *cfg, const ig_weights *w, const int32_t *devices, int32_t ndevices,
                                 ig_model **out);
/* ig_model_create_stored on several GPUs, as ig_model_create_multi. */
IG_API int ig_model_create_stored_multi(const ig_config *cfg, const ig_stored_weights *w, const int32_t *devices,
                                        int32_t ndevices, ig_model **out);
/* Replica `index` of a model and its device (the model itself, index 0, for
 * a single-device model); borrowed: destroyed with the model. */
IG_API int ig_model_replica(ig_model *m, int32_t index, ig_model **replica, int32_t *device);
/* Number of devices a model runs on. */
IG_API int ig_model_device_count(ig_model *m, int32_t *n);
/* Number of sm_100 devices this process can use (0 without a driver or GPU). */
IG_API int ig_device_count(int32_t *n);

/* Releases the model's device memory. Replaces Invalidate (infer.go:95-100)
 * for the device copy: a changed model is destroyed and created again. */
IG_API void ig_model_destroy(ig_model *m);

/* Replaces SetEmbeddingTable (internal/modernbert/infer.go:20-25) with a
 * table uploaded in its stored format and read row by row in the embedding
 * gather (Row, embeddings.go:49-68): bf16 rows widen exactly (bits << 16), an
 * id listed in exact_ids takes its float32 row, int8 rows are
 * float32(int8) * scale[id]. Copied; replaces the table given at creation.
 * Must not run concurrently with an encode on the same model. Errors:
 * IG_ERR_BAD_ARG ("indecis: exact row %d out of vocabulary", a missing array). */
IG_API int ig_model_set_embeddings(ig_model *m, const ig_embedding_table *t);

/* Replaces the heads of Model (heads.go:29-48, model.go:312-341); copied. */
IG_API int ig_model_set_heads(ig_model *m, int32_t nheads, const ig_head *heads);

/* Replaces EncodeSeqs (infer.go:261, mode IG_MODE_POOLED, out [nseq][hidden])
 * and EncodeTokens (infer.go:293, mode IG_MODE_TOKENS, out [offs[nseq]][hidden]).
 * ids are the concatenated sequences, offs[nseq+1] their starts (offs[0] = 0).
 * Host buffers; the call returns when out is written. An id outside
 * [0, vocab) fails with IG_ERR_OUT_OF_VOCAB before any device work. */
IG_API int ig_encode(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, int32_t mode, float *out,
              size_t out_len);

/* ig_encode on device buffers (d_ids [offs[nseq]], d_out) enqueued on
 * `stream` (a cudaStream_t; NULL: the legacy default stream). offs stays a
 * host array: it sizes the launches. Returns once the work is enqueued;
 * an out-of-vocabulary id is reported by ig_device_error() after the stream
 * completes (its row reads embedding row 0). */
IG_API int ig_encode_device(ig_model *m, const int32_t *d_ids, const int64_t *offs, int32_t nseq, int32_t mode,
                     float *d_out, void *stream);

/* Replaces the logits half of DecideInputs (spans.go:369-461 then
 * heads.go:62-74 per head): float64 logits of every pooled head for each
 * sequence, concatenated in head order ([nseq][sum of pooled rows]), and,
 * when token_logits is not NULL, of every per-token head for each token
 * ([offs[nseq]][sum of per-token rows]). The answers (sigmoid, softmax,
 * ordinal distribution, heads.go:124-187) stay with the caller. */
IG_API int ig_logits(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, double *logits,
              size_t logits_len, double *token_logits, size_t token_len);

/* ig_logits on device buffers, enqueued on `stream` like ig_encode_device:
 * d_logits [nseq][sum of pooled rows], d_token_logits [offs[nseq]][sum of
 * per-token rows] (either may be NULL). */
IG_API int ig_logits_device(ig_model *m, const int32_t *d_ids, const int64_t *offs, int32_t nseq, double *d_logits,
                            double *d_token_logits, void *stream);

/* Kernel profiling. ig_profile(1) clears the records and brackets every
 * encoder launch with CUDA events on its stream (outside stream capture);
 * ig_profile(0) stops. ig_profile_report synchronizes the device and writes
 * a JSON summary {"launches": total kernel launches since ig_profile(1),
 * "graphs_recorded", "graph_runs": CUDA graphs recorded and launched by host
 * calls since the library loaded (a host call of at most 16384 tokens whose
 * offsets, mode and outputs repeat the previous call's on the same workspace
 * replays its kernels as one graph; none while profiling),
 * "kernels": [{name, launches, ms, bytes, ops}]} where bytes and ops are the
 * launches' algorithmic memory traffic and arithmetic; returns its length. */
IG_API int ig_profile(int32_t enable);
IG_API int64_t ig_profile_report(char *buf, size_t len);
/* Restricts the events of ig_profile to the launches recorded under `name`
 * (a "kernels" name of the report; NULL or "": every launch), so that a timed
 * run carries events around one kernel only. Call it between runs. */
IG_API int ig_profile_only(const char *name);

/* Message of the calling thread's last failure ("" if none). */
IG_API const char *ig_last_error(void);

/* First error code a kernel recorded on the current device since the last
 * reset (one value per device, shared by every model and call on it): 1, 2, 3
 * a bounded wait gave up (a TMA stage, a stage release, an accumulator), 4 a
 * bad shape, 5 an id outside the vocabulary in ig_encode_device; 0 none.
 * Host calls (ig_encode, ig_logits, ...) return IG_ERR_CUDA while it holds
 * 1-3. reset != 0 clears it. Synchronizes the device. */
IG_API int32_t ig_device_error(int32_t reset);

/* Self-check of the bounded waits (no counterpart in the reference, which
 * runs on the CPU). Every mbarrier wait in the kernels gives
 * up after a limit (2 s), records its code (1-3) in ig_device_error() and
 * lets the kernel wind down instead of hanging the GPU. This runs one such
 * wait on a barrier that nothing completes, with a limit of limit_ns
 * (0 < limit_ns <= 2 s): *timed_out = 1 when it gave up, *waited_ns
 * (optional) = the time it waited. It leaves code 1 in ig_device_error();
 * the device stays usable. Synchronizes the device. */
IG_API int ig_check_wait_timeout(int64_t limit_ns, int32_t *timed_out, int64_t *waited_ns);

/* Self-check of the GELU vector body's division shortcut (an FMA-refined
 * reciprocal in place of the IEEE division of geluMulAVX2's VDIVPS,
 * linalg/gelu_amd64.s:165-225): over every float t in [-4, 4] on the current
 * device, mismatches[0] = quotients that differ from the IEEE quotient and
 * mismatches[1] = values of 1 + quotient that differ (the GELU uses the
 * quotient only through 1 + erf; 0 required); first_bad_bits (optional) = the
 * smallest |t| bits of the latter; histogram (optional, [2][256]) = both
 * counts by the biased exponent of t. Synchronizes the device. */
IG_API int ig_check_gelu_division(int64_t *mismatches, uint32_t *first_bad_bits, int64_t *histogram);

/* ---- per-operation entry points (device pointers, enqueued on stream) ---- */

/* MatMul8N's integer product and dequantization (linalg/int8.go:88-155):
 * acc = A . B^T with A uint8 [M][lda] (q + 128) and B int8 [N][ldb] (K bytes
 * used per row; lda, ldb multiples of 16);
 * C[i][j] (+)= ((float(acc) - zc[j]) * sb[j]) * sa[i] with row stride ldc.
 * acc_out (optional, [M][ldc] int32) receives the accumulators instead of C. */
IG_API int ig_gemm_u8s8(const uint8_t *A, int32_t lda, const int8_t *B, int32_t ldb, int32_t M, int32_t N, int32_t K,
                 const float *sa, const float *sb, const float *zc, float *C, int32_t ldc, int32_t accumulate,
                 int32_t *acc_out, void *stream);

/* The encoder's Wi product with its GeGLU epilogue and the output rows
 * quantized in the same kernel (MatMul8N + GeluMul + quantizeA of
 * internal/modernbert/infer.go:416-423, linalg/int8.go:157-191): B holds the
 * 2I weight rows interleaved per 128 (the GELU inputs of GeGLU columns
 * 128t..128t+127, then their gates), sa/sb/zc as ig_gemm_u8s8; out q [M][ldq]
 * uint8 (q + 128) and sa_out [M]. I a multiple of 128, at most 1024. */
IG_API int ig_gemm_geglu_quant(const uint8_t *A, int32_t lda, const int8_t *B, int32_t ldb, int32_t M, int32_t I,
                               int32_t K, const float *sa, const float *sb, const float *zc, uint8_t *q, int32_t ldq,
                               float *sa_out, void *stream);

/* quantizeA (linalg/int8.go:157-191): per row s = max|x|/127,
 * q = rne(x * (1/s)) + 128 (all 128 and s = 0 for a zero row). */
IG_API int ig_quantize_rows(const float *x, int32_t ldx, int32_t M, int32_t K, uint8_t *q, int32_t ldq, float *sa,
                     void *stream);

/* LayerNormRow (linalg/vec_simd.go:281-327) of each row, optional f32
 * output xn, and the quantized rows as ig_quantize_rows (q may be NULL). */
IG_API int ig_layernorm_quant(const float *x, const float *gamma, int32_t M, int32_t H, double eps, int32_t simd_lanes,
                       float *xn, uint8_t *q, int32_t ldq, float *sa, void *stream);

/* PackB8 with transB (linalg/int8.go:36-77): w [n][k] f32 -> q int8 [n][ldq]
 * (zero padded), scale [n], zc [n] = 128 * colsum, colsum [n] (optional). */
IG_API int ig_pack_b8(const float *w, int32_t n, int32_t k, int8_t *q, int32_t ldq, float *scale, float *zc,
               int32_t *colsum, void *stream);

/* attention8 (infer.go:484-518; linalg/attention8.go): qkv [N][3*hidden]
 * rows after RoPE, sequences at host offsets offs[nseq+1]; window < 0 for a
 * global layer, else the half-window; ctx [N][hidden]. Work buffers are
 * allocated for the call (a test entry point; ig_encode uses its workspace).
 * A (sequence, head) whose Q or K values are NaN, infinite or large enough
 * for a score to overflow is recomputed with the reference's float->int
 * conversions and NaN flow, so it too gets the reference's bits. */
IG_API int ig_attention(const float *qkv, int32_t hidden, int32_t heads, const int64_t *offs, int32_t nseq,
                 int32_t window, int32_t simd_lanes, float *ctx, void *stream);

/* ig_attention for callers that cannot allocate device memory (processes that
 * reserve all device memory up front, latency-critical paths that must not
 * synchronize the device through cudaMalloc/cudaFree). No counterpart in the
 * reference: its attention buffers are Go slices. Same arguments and result as
 * ig_attention, but the work buffers come from one array of 32 MiB built into
 * the library, held on every GPU that loads it until the process exits; inputs
 * needing more scratch fail with IG_ERR_BAD_ARG, sequences longer than 10240
 * tokens with IG_ERR_UNSUPPORTED, both before any GPU work. The first call on
 * a device looks up the array's address (make it before any stream capture).
 * The offsets are read from host memory during the call. All calls share the
 * array: calls that overlap on the GPU race. Asynchronous on `stream`. */
IG_API int ig_attention_noalloc(const float *qkv, int32_t hidden, int32_t heads, const int64_t *offs, int32_t nseq,
                                int32_t window, int32_t simd_lanes, float *ctx, void *stream);

/* Per-layer intermediates of one ig_encode call, copied to host buffers for
 * parity checks (NULL fields are skipped). Layouts as the oracle's. */
typedef struct ig_dump {
  int32_t layer;
  uint8_t *xq;  float *xq_s;  /* QKV input quantized [N][hidden], [N] */
  float *qkv;                 /* [N][3*hidden] QKV projection (RoPE is applied in the attention) */
  float *ctx;                 /* [N][hidden] */
  uint8_t *cq;  float *cq_s;  /* Wo input quantized */
  float *x_attn;              /* residual after attention */
  uint8_t *hq;  float *hq_s;  /* Wi input quantized */
  float *g;                   /* [N][intermediate] GeGLU output */
  uint8_t *gq;  float *gq_s;  /* WoMLP input quantized [N][intermediate] */
  float *x_mlp;               /* residual after the MLP */
  float *emb_ln;              /* [N][hidden] embedding after its norm */
} ig_dump;

IG_API int ig_encode_dump(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, int32_t mode, float *out,
                   size_t out_len, ig_dump *dump);

/* ---- Spans questions (spans.go): long texts read in windows, per-token BIO
 * tags decoded into passages. The window planning, log-softmax and Viterbi
 * decoding are host code (no device, callable without a GPU); the encoder
 * and the per-token heads of ig_infer_windows run on the device. ---- */

/* A slice [start, end) of a text's tokens read in one encoder pass; the
 * tokens [keep_from, keep_to) take their tags from it (window, spans.go:314). */
typedef struct ig_window {
  int32_t start, end, keep_from, keep_to;
} ig_window;

/* planWindows (spans.go:322-334): cuts n tokens into windows of at most
 * `size` tokens, each reading up to `margin` tokens (at most (size-1)/4) of
 * context beside the slice it keeps. *count receives the number of windows;
 * out (may be NULL) receives them when cap allows, else IG_ERR_BAD_ARG. */
IG_API int ig_plan_windows(int32_t n, int32_t size, int32_t margin, ig_window *out, int32_t cap, int32_t *count);

/* logSoftmax (spans.go:293-311): out = z/T - log sum exp(z/T), T <= 0 read as 1. */
IG_API int ig_log_softmax(const double *z, int32_t n, double temperature, double *out);

/* A passage found by a Spans question (Span, spans.go:43-50): bytes
 * [start, end) of the text, `type` the index of its option. */
typedef struct ig_span {
  int32_t type, start, end;
  double confidence; /* mean probability of the passage's tags */
} ig_span;

/* decodeSpans (spans.go:172-246): the most probable consistent BIO tag
 * sequence of logp [ntok][ntags] (log-probabilities; tag 0 outside, 1+2k
 * begins a passage of type k, 2+2k continues it; bias added to every tag
 * but outside), then its passages: from the first token's core (its leading
 * spaces skipped) to the last token's end, edge punctuation trimmed.
 * offsets [ntok][2] are the tokens' byte ranges in text. *nspans receives
 * the number of passages (at most ntok); out receives them when cap allows,
 * else IG_ERR_BAD_ARG. tags (optional, [ntok]) receives the decoded tags. */
IG_API int ig_decode_spans(const double *logp, int32_t ntok, int32_t ntags, double bias, const char *text,
                           int64_t text_len, const int32_t *offsets, int32_t *tags, ig_span *out, int32_t cap,
                           int32_t *nspans);

/* answerSpans (spans.go:479-491): ig_log_softmax of each token's logits
 * (z [ntok][ldz], the first ntags used) at `temperature`, then
 * ig_decode_spans. */
IG_API int ig_answer_spans(const double *z, int32_t ntok, int32_t ldz, int32_t ntags, double temperature, double bias,
                           const char *text, int64_t text_len, const int32_t *offsets, ig_span *out, int32_t cap,
                           int32_t *nspans);

/* The tags ig_answer_spans decodes, for many texts at once on the device
 * (the log-softmax and the Viterbi pass; one warp per text): d_z device
 * logits [offs[ntexts]][ldz] (the first ntags used), texts at host offsets
 * offs[ntexts+1], d_tags [offs[ntexts]] (device). At most 32 tags
 * (IG_ERR_UNSUPPORTED beyond). exp and log are the device's double-precision
 * functions: scores tied to the last bit may decide differently from the
 * host's. Enqueued on `stream`. */
IG_API int ig_spans_tags_device(const double *d_z, int64_t ldz, const int64_t *offs, int32_t ntexts, int32_t ntags,
                                double temperature, double bias, int32_t *d_tags, void *stream);
/* ig_spans_tags_device on host buffers, on `device` (synchronous). */
IG_API int ig_spans_tags(const double *z, int64_t ldz, const int64_t *offs, int32_t ntexts, int32_t ntags,
                         double temperature, double bias, int32_t *tags, int32_t device);
/* The passages of one text's tag sequence (decodeSpans' extraction,
 * spans.go:222-245), confidences from the tempered log-softmax of z. */
IG_API int ig_spans_from_tags(const double *z, int32_t ntok, int32_t ldz, int32_t ntags, double temperature,
                              const int32_t *tags, const char *text, int64_t text_len, const int32_t *offsets,
                              ig_span *out, int32_t cap, int32_t *nspans);

/* ig_logits with every sequence pooled by the mean of its rows whatever the
 * config's pooling (meanRows, spans.go:464-477): the pooled heads of a
 * model with Spans questions read that mean. */
IG_API int ig_window_logits(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, double *logits,
                            size_t logits_len, double *token_logits, size_t token_len);

/* The Spans branch of infer (spans.go:385-461) for ninputs tokenized texts:
 * ids the texts' tokens end to end (no special tokens), offs[ninputs+1]
 * their starts. Each text is cut by ig_plan_windows into windows of
 * max(max_len - nprefix - nsuffix, 1) tokens with a margin of a sixteenth
 * of that; each window is framed by prefix and suffix and encoded, up to
 * batch_size windows per device pass (<= 0: all in one). logits
 * [ninputs][sum of pooled rows] receives the pooled heads of each text's
 * first window, token_logits [offs[ninputs]][sum of per-token rows] the
 * per-token heads of each text token, from the window that keeps it. */
IG_API int ig_infer_windows(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t ninputs,
                            const int32_t *prefix, int32_t nprefix, const int32_t *suffix, int32_t nsuffix,
                            int32_t max_len, int32_t batch_size, double *logits, size_t logits_len,
                            double *token_logits, size_t token_len);

/* Rows of the heads set by ig_model_set_heads: *pooled_rows and
 * *token_rows receive the sums over pooled and per-token heads. */
IG_API int ig_model_head_rows(ig_model *m, int32_t *pooled_rows, int32_t *token_rows);

/* SetInt8 (infer.go:115-135): on != 0 (the state after ig_model_create)
 * computes the layers in int8; 0 switches the model to the reference's
 * float32 path (float products in its FMA-chain order, RoPE in place,
 * attendBlocks' blocked softmax, the erf GELU x gate: infer.go:304-430,
 * :590-650), from float32 copies of the weights kept at creation. Must not
 * run concurrently with an encode on the same model. The per-layer dump
 * (ig_encode_dump) is of the int8 path only. */
IG_API int ig_model_set_int8(ig_model *m, int32_t on);

/* Vocabulary size and hidden width of a model. */
IG_API int ig_model_dims(ig_model *m, int32_t *vocab, int32_t *hidden);

/* ---- Batching front end (WithBatching, model.go:137-160; batch.go) ----
 * Concurrent callers' EncodeSeqs requests are coalesced into device
 * batches: a worker takes the first pending request, then those already
 * queued while the batch holds fewer than max_rows positions (<= 0: 512),
 * encodes them in one pass and returns each caller its rows. Workers of
 * every model (one per GPU) share one queue; max_wait_us > 0 lets a worker
 * wait that long for more requests while its batch is short (0: the
 * reference's behaviour, never wait). A request whose ids fail is answered
 * alone, with its own error. */
typedef struct ig_batcher ig_batcher;
/* The encoder a batcher drives: pooled [nseq][hidden] of the sequences at
 * offs (0 or an IG_ERR_* status). */
typedef int (*ig_batch_encode_fn)(void *user, const int32_t *ids, const int64_t *offs, int32_t nseq, float *pooled);
IG_API int ig_batcher_create(ig_model *const *models, int32_t nmodels, int32_t workers_per_model, int32_t max_rows,
                             int32_t max_wait_us, ig_batcher **out);
/* The same over any encoder (one `users` entry per device). */
IG_API int ig_batcher_create_fn(ig_batch_encode_fn fn, void *const *users, int32_t nusers, int32_t hidden,
                                int32_t workers_per_user, int32_t max_rows, int32_t max_wait_us, ig_batcher **out);
/* Finishes the queued requests, then stops the workers. */
IG_API void ig_batcher_destroy(ig_batcher *b);
/* EncodeSeqs through the batcher (blocking, thread-safe): pooled [nseq][hidden]. */
IG_API int ig_batcher_encode(ig_batcher *b, const int32_t *ids, const int64_t *offs, int32_t nseq, float *pooled,
                             size_t pooled_len);
/* Requests taken, device passes run and positions encoded so far. */
IG_API int ig_batcher_stats(ig_batcher *b, int64_t *requests, int64_t *batches, int64_t *rows);

/* ---- SigLIP vision tower (internal/siglip): int8 layers, float32 patch
 * embedding, attention and pooling head, as the reference computes them.
 * The seam is Vision.forward (internal/siglip/vision.go:101-141), reached by
 * Embed and Forward (vision.go:85-99); one call takes a batch of images. ---- */

/* Dimensions (Config, siglip.go:26-33 with ReadConfig's defaults applied). */
typedef struct ig_vision_config {
  int32_t hidden, layers, heads, mlp, image_size, patch_size;
  double eps;
  int32_t simd_lanes; /* float32 lanes of LayerNorm/ExpShift/GeluTanh sums (8: AVX2) */
} ig_vision_config;

/* Float32 weights in transformers layouts ([out][in] matrices), as
 * loadVision reads them (vision.go:30-80); q, k, v stacked into wqkv. */
typedef struct ig_vision_weights {
  const float *patch_w, *patch_b; /* [H][3*P*P] conv weight in (channel, y, x) order, [H] */
  const float *pos;               /* [T][H], T = (image_size/patch_size)^2 */
  const float *const *ln1_g, *const *ln1_b, *const *ln2_g, *const *ln2_b; /* [layers] of [H] */
  const float *const *wqkv, *const *bqkv; /* [layers] of [3H][H], [3H] */
  const float *const *wo, *const *bo;     /* [layers] of [H][H], [H] */
  const float *const *w1, *const *b1;     /* [layers] of [mlp][H], [mlp] */
  const float *const *w2, *const *b2;     /* [layers] of [H][mlp], [H] */
  const float *post_g, *post_b;           /* [H] */
  const float *probe;                     /* [H] */
  const float *in_w, *in_b;               /* [3H][H], [3H] pooling attention in_proj */
  const float *hout_w, *hout_b;           /* [H][H], [H] */
  const float *hln_g, *hln_b;             /* [H] */
  const float *hfc1_w, *hfc1_b;           /* [mlp][H], [mlp] */
  const float *hfc2_w, *hfc2_b;           /* [H][mlp], [H] */
} ig_vision_weights;

typedef struct ig_vision ig_vision;

/* loadVision with int8 layers (vision.go:30-80, encoder.go:95-156): weights
 * copied to `device`, each layer matrix quantized per output channel there,
 * the probe's query computed once. head_dim must be 64 and the patches at
 * most 256 in this build (IG_ERR_UNSUPPORTED otherwise). */
IG_API int ig_vision_create(const ig_vision_config *cfg, const ig_vision_weights *w, int32_t device,
                            ig_vision **out);
IG_API void ig_vision_destroy(ig_vision *v);

/* Vision.forward on n images of normalized pixels [n][3][S][S] (host
 * buffers): layer 0 runs every layer; layer > 0 stops after that many layers
 * unless pooled is wanted. patches (may be NULL) receives [n][T][H] — the
 * states after `layer` layers, or the final ones (after post_layernorm) for
 * layer 0; pooled (may be NULL) the embeddings [n][H] (Embed). Errors:
 * IG_ERR_BAD_ARG "siglip: layer %d, the tower has %d". */
IG_API int ig_vision_forward(ig_vision *v, const float *pixels, int32_t n, int32_t layer, float *patches,
                             size_t patches_len, float *pooled, size_t pooled_len);

/* ig_vision_forward on device buffers, enqueued on `stream` (NULL: legacy
 * default stream). Calls on one ig_vision are serialized. */
IG_API int ig_vision_forward_device(ig_vision *v, const float *d_pixels, int32_t n, int32_t layer,
                                    float *d_patches, float *d_pooled, void *stream);

/* Intermediates of one layer for parity checks (NULL fields skipped); rows
 * are images x patches. */
typedef struct ig_vision_dump {
  int32_t layer;
  float *x_embed;               /* [n*T][H] patch embedding + positions */
  uint8_t *h1q; float *h1q_s;   /* LN1 output quantized [n*T][H], [n*T] */
  float *qkv;                   /* [n*T][3H] with bias */
  float *attn;                  /* [n*T][H] attention output */
  float *x_attn;                /* [n*T][H] residual after attention */
  uint8_t *h2q; float *h2q_s;   /* LN2 output quantized */
  float *mlp;                   /* [n*T][mlp] GeluTanh(fc1) */
  int32_t *outliers;            /* [n][32] fc2 input channels computed in float32, in order */
  int32_t *noutliers;           /* [n] */
  uint8_t *mq; float *mq_s;     /* fc2 input quantized, those channels zeroed */
  float *x_mlp;                 /* [n*T][H] residual after the MLP */
} ig_vision_dump;

IG_API int ig_vision_dump_layer(ig_vision *v, const float *pixels, int32_t n, ig_vision_dump *dump, float *pooled,
                                size_t pooled_len);

#ifdef __cplusplus
}
#endif

#endif /* INDECIS_B200_H */
