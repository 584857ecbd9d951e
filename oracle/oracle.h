/*
 * CPU oracle for the int8 ModernBERT encoder path of Bornholm/indecis.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against, and the CPU baseline that bench.py times beside it. Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU legs load it. The product
 * (indecis_b200, libindecis_b200.so) never links, loads or calls it.
 *
 * It restates, in scalar C++, the arithmetic of the reference's int8 inference
 * path (Go module github.com/bornholm/indecis; file:line citations are relative
 * to that module's root):
 *   internal/modernbert/infer.go:304-430   run(): layer order, residuals, pooling
 *   linalg/int8.go:38-77,160-191,207       PackB8, quantizeA, roundHalfEven
 *   linalg/kernel_vnni_amd64.s:144-234     dequant order ((acc - zc)*sb)*sa [+c]
 *   linalg/quant_amd64.s:17-156            quantRowAVX2 / quantColsAVX2
 *   linalg/attention8.go:203-376           Attn8.prepareAVX2 / Attend
 *   linalg/vec_simd.go:220-425             ExpShift, LayerNormRow, MaxOf, Rope
 *   linalg/gelu_amd64.s:165-225            geluMulAVX2 (FMA polynomial order)
 *   linalg/fastmath.go:9-51                erf32, exp32 (scalar tails)
 *   internal/modernbert/model.go:256-277   RoPE cos/sin table
 *   heads.go:63-74                         head.logits (float64)
 *   internal/siglip/encoder.go, vision.go  SigLIP vision tower (siglip.cpp)
 *   linalg/gemm.go:65-240                  float32 products (chain per 256-deep block)
 *   linalg/int8.go:281-349                 MatMul8Outliers
 *   linalg/vec_simd.go:166-202             GeluTanh
 *
 * Parity status (stated here because it bounds what the oracle proves):
 *   - The reference cannot run in this environment (it is Go 1.27 with
 *     GOEXPERIMENT=simd; no Go toolchain exists here or on the GPU hosts) and
 *     ships no int8 golden vectors. The composite encoder is therefore
 *     "parity unpinned" against a reference run.
 *   - Its elementary operations are pinned by the reference's own known-answer
 *     data and exactness properties (tests/test_oracle_pins.py): the
 *     roundHalfEven cases of linalg/int8_test.go:88-94, the GELU constants as
 *     the hex words of linalg/gelu_amd64.s, the properties of
 *     linalg/vec_test.go:9, linalg/int8_test.go:36,149 and
 *     linalg/attention8_test.go:50,87.
 *   - Machine-dependent choices are fixed and recorded: vector width V = 8
 *     float32 lanes (AVX2, the width of all of the reference's assembly),
 *     GOAMD64=v1 (the Go compiler does not contract scalar a*b+c into FMA),
 *     and FMA exactly where the reference writes MulAdd or VFMADD.
 *
 * Compile with -ffp-contract=off: every a*b+c below is two roundings unless it
 * is spelled std::fma.
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- elementary operations ------------------------------------------------ */
float or_round_half_even(float v);
float or_exp32(float x);
float or_erf32(float x);
float or_exp_shift(float *x, int n, float m, int V);
void or_gelu_mul(float *o, const float *a, const float *b, int n);
void or_layernorm_row(float *o, const float *x, const float *gamma, int n, double eps, int V);
void or_rope(float *x, const float *cos_, const float *sin_, int half);
void or_rope_table(double theta, int D, int npos, float *cos_, float *sin_);
/* quantRowAVX2: c = x - mean; returns scale (0: all zero, dst untouched). */
float or_quant_row(int8_t *dst, const float *x, const float *mean, int n, int flip, int32_t *sum);

/* ---- int8 GEMM -------------------------------------------------------------- */
/* PackB8 (per output channel). q is [n][k] row-major (k contiguous). */
void or_pack_b8(const float *b, int k, int n, int transB, int8_t *q, float *scale, int32_t *colsum,
                float *zc);
/* quantizeA: q[i][j] = rne(a*inv)+128 as uint8, sa[i] = max|a_i|/127 (0: row of 128). */
void or_quantize_a(const float *a, int m, int k, uint8_t *q, float *sa);
/* acc[i][j] = sum_k A[i][k] * B[j][k]: uint8 A times int8 B, exact int32. */
void or_gemm_u8s8(const uint8_t *A, int lda, const int8_t *B, int ldb, int M, int N, int K, int32_t *acc);
/* C[i][j] (+)= ((float(acc) - zc[j]) * sb[j]) * sa[i]. */
void or_dequant(const int32_t *acc, int M, int N, const float *sa, const float *sb, const float *zc, float *C,
                int accumulate);
/* MatMul8N: quantize a, multiply by the packed weights, dequantize. */
void or_matmul8(float *c, const float *a, int m, const int8_t *q, const float *scale, const float *zc, int k,
                int n, int accumulate);

/* ---- attention (Attn8.Prepare + Attend over all queries) -------------------- */
typedef struct {
  uint8_t *qa;  /* [n][D]  uint8 Q (q+128) */
  float *sq;    /* [n]     Q row scale times the score scale */
  int8_t *kq;   /* [n][D]  centred K, int8 */
  float *ks;    /* [n] */
  float *kzc;   /* [n]     128*sum(kq) */
  int8_t *vq;   /* [n][D]  V per column, int8 */
  float *vs;    /* [D] */
  float *kmean; /* [D] */
  uint8_t *p;   /* [n][n]  quantized softmax weights (0 outside the window) */
  float *sp;    /* [n] */
  int32_t *sacc;/* [n][n]  score accumulators sum(qa*kq) */
  int32_t *oacc;/* [n][D]  P.V accumulators */
} or_attn_dbg;
void or_attn8(const float *q, const float *k, const float *v, int ld, int n, int D, int window, float scale,
              float *o, int ldo, or_attn_dbg *dbg);

/* ---- encoder ----------------------------------------------------------------- */
typedef struct {
  int vocab, hidden, layers, heads, intermediate;
  int global_every, local_attention; /* local_attention: total window width */
  int cls;                           /* pooling: 0 mean, 1 first token */
  double norm_eps, global_theta, local_theta;
  int V; /* float32 lanes of the reference's portable SIMD (8 = AVX2) */
} or_config;

typedef struct {
  const float *emb;        /* [V][H] */
  const float *emb_norm;   /* [H] */
  const float *final_norm; /* [H] */
  const float *const *attn_norm; /* [L] of [H]; entry 0 unused (layer 0 has none) */
  const float *const *wqkv;      /* [L] of [3H][H] */
  const float *const *wo;        /* [L] of [H][H] */
  const float *const *mlp_norm;  /* [L] of [H] */
  const float *const *wi;        /* [L] of [2I][H] (input then gate) */
  const float *const *wo_mlp;    /* [L] of [H][I] */
} or_weights;

typedef struct or_model or_model;

/* Intermediate values of one layer, for per-op parity (NULL: not wanted). */
typedef struct {
  int layer;
  uint8_t *xq;      float *xq_s;   /* QKV input, quantized [N][H], [N] */
  int32_t *qkv_acc;                /* [N][3H] */
  float *qkv;                      /* [N][3H] QKV projection, before RoPE */
  float *ctx;                      /* [N][H] attention output */
  uint8_t *cq;      float *cq_s;   /* Wo input quantized */
  float *x_attn;                   /* [N][H] residual after attention */
  uint8_t *hq;      float *hq_s;   /* Wi input quantized (LN mlp) */
  float *z;                        /* [N][2I] Wi output */
  uint8_t *gq;      float *gq_s;   /* WoMLP input quantized */
  float *x_mlp;                    /* [N][H] residual after the MLP */
  float *emb_ln;                   /* [N][H] x after the embedding norm (layer-independent) */
} or_dump;

or_model *or_model_create(const or_config *cfg, const or_weights *w);
void or_model_destroy(or_model *m);
/* Packed weights of layer l, matrix which (0 qkv, 1 o, 2 i, 3 o_mlp). */
void or_model_packed(const or_model *m, int l, int which, const int8_t **q, const float **scale,
                     const float **zc, int *k, int *n);

/* mode: 0 pooled (mean or CLS per config) [nseq][H]; 1 token states [N][H].
 * Returns 0, 1 with *bad_id set when an id is out of the vocabulary, or 2 for
 * offsets that do not start at 0 or decrease.
 * threads <= 1: scalar reference loops. threads > 1 or fast != 0: the CPU
 * baseline (cpu_baseline.cpp), bitwise equal to the scalar loops. */
int or_encode(const or_model *m, const int32_t *ids, const int64_t *offs, int nseq, int mode, float *out,
              int threads, int fast, or_dump *dump, int32_t *bad_id);

/* The encoder without SetInt8 (float32 products as linalg/gemm.go, RoPE in
 * place, attendBlocks' blocked softmax, infer.go:304-430, :590-650); same
 * arguments and return values as or_encode. */
int or_encode_f32(const or_model *m, const int32_t *ids, const int64_t *offs, int nseq, int mode, float *out,
                  int threads, int32_t *bad_id);

/* head.logits: z[r] = sum_i double(w[r][i])*double(x[i]) + double(b[r]). */
void or_head_logits(const float *w, const float *b, int rows, int H, const float *x, int nx, double *z);

/* ---- SigLIP vision tower (internal/siglip) ----------------------------------- */
typedef struct {
  int hidden, layers, heads, mlp, image_size, patch_size;
  double eps;
  int V; /* float32 lanes of the reference's portable SIMD (8 = AVX2) */
} or_siglip_config;

/* Float32 weights in transformers layouts ([out][in] matrices). */
typedef struct {
  const float *patch_w, *patch_b; /* [H][3*P*P] (channel, y, x), [H] */
  const float *pos;               /* [T][H] */
  const float *const *ln1_g, *const *ln1_b, *const *ln2_g, *const *ln2_b; /* [L] of [H] */
  const float *const *wqkv, *const *bqkv; /* [L] of [3H][H] (q, k, v stacked), [3H] */
  const float *const *wo, *const *bo;     /* [L] of [H][H], [H] */
  const float *const *w1, *const *b1;     /* [L] of [M][H], [M] */
  const float *const *w2, *const *b2;     /* [L] of [H][M], [H] */
  const float *post_g, *post_b;           /* [H] */
  const float *probe;                     /* [H] */
  const float *in_w, *in_b;               /* [3H][H], [3H]: pooling attention projections */
  const float *hout_w, *hout_b;           /* [H][H], [H] */
  const float *hln_g, *hln_b;             /* [H] */
  const float *hfc1_w, *hfc1_b;           /* [M][H], [M] */
  const float *hfc2_w, *hfc2_b;           /* [H][M], [H] */
} or_siglip_weights;

/* Intermediate values of one layer for one call (NULL: not wanted). Rows are
 * images x patches. */
typedef struct {
  int layer;
  float *x_embed;            /* [n*T][H] patch embedding + positions */
  uint8_t *h1q; float *h1q_s;/* LN1 output quantized */
  float *qkv;                /* [n*T][3H] (with bias) */
  float *attn;               /* [n*T][H] attention output */
  float *x_attn;             /* [n*T][H] residual after attention */
  uint8_t *h2q; float *h2q_s;/* LN2 output quantized */
  float *mlp;                /* [n*T][M] GELU(fc1) */
  int32_t *outliers;         /* [n][32] fc2 input channels computed in float32 */
  int32_t *noutliers;        /* [n] */
  uint8_t *mq; float *mq_s;  /* fc2 input quantized, outlier channels zeroed */
  float *x_mlp;              /* [n*T][H] residual after the MLP */
} or_siglip_dump;

typedef struct or_siglip or_siglip;
or_siglip *or_siglip_create(const or_siglip_config *cfg, const or_siglip_weights *w);
void or_siglip_destroy(or_siglip *m);
/* Vision.forward (internal/siglip/vision.go:101-141) on n images of
 * normalized pixels [n][3][S][S]. layer 0 runs every layer; layer > 0 stops
 * after that many layers unless pooled is wanted, and patches then hold the
 * states after that layer. patches [n][T][H] and pooled [n][H] may be NULL.
 * threads > 1 spreads the images over threads; fast != 0 uses the VNNI
 * integer products (same integers). Returns 0, or 1 for a bad layer. */
int or_siglip_forward(const or_siglip *m, const float *pixels, int n, int layer, float *patches, float *pooled,
                      int threads, int fast, or_siglip_dump *dump);
/* The float32 products of linalg/gemm.go (MatMulPackedN + AddTo): dst[r][o] =
 * the sum over k of x[r][k]*W[o][k] as one FMA chain per 256-deep block,
 * blocks added in order, then + b[o] (b may be NULL). */
void or_linear_f32(float *dst, const float *x, int rows, const float *W, const float *b, int in, int out);
/* linalg.GeluTanh over n values (V-lane vector body, scalar tail). */
void or_gelu_tanh(float *o, const float *a, int n, int V);
/* internal/siglip/encoder.go:236-251 softmax(s*scale) in place. */
void or_siglip_softmax(float *s, int n, float scale, int V);
/* linalg.MatMul8Outliers (linalg/int8.go:281-349) with the packed weights of
 * or_pack_b8; out receives the chosen channels in the order they are added. */
void or_matmul8_outliers(float *c, const float *a, int m, const int8_t *q, const float *scale, const float *zc, int k,
                         int n, float ratio, int32_t *out, int32_t *nout);

/* CPU features used by the baseline (bit 0: AVX-VNNI, bit 1: AVX512-VNNI). */
int or_cpu_features(void);
/* Wall seconds of or_encode's phases summed since the last reset: [0] norms,
   QKV and RoPE, [1] attention, [2] output projection, norm and MLP. */
void or_phase_seconds(double *out, int reset);

#ifdef __cplusplus
}
#endif
