// Declarations shared by the CUDA translation units of libindecis_b200.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/indecis_b200.h"

namespace ig {

enum Epilogue : int {
  kEpiF32 = 0,
  kEpiI32 = 1,
  kEpiGeglu = 3,
  kEpiF32Bias = 4,   // C (+)= dequant + bias[j]   (MatMul8N then AddTo(bias), accumulate: AddTo(x, .))
  kEpiGeluTanh = 5,  // C = GeluTanh(dequant + bias[j])
  kEpiOutlierRes = 6,  // C += (dequant + outlier terms in order) + bias[j]  (MatMul8Outliers, then AddTo twice)
  kEpiGegluQ = 7,      // kEpiGeglu, then the output row quantized (quantizeA) into q_out + sa_out: a cluster per
                       // row block, its CTAs (one per 256-column tile) exchanging the row maxima
};

struct GemmArgs {
  const uint8_t *A;  // [M][lda] uint8 activations (q + 128)
  const int8_t *B;   // [N][ldb] int8 weights, output channel rows
  int M, N, K;
  int lda, ldb;      // row strides in bytes, multiples of 16
  int bn;            // 128 or 256 (0: choose)
};

struct GemmEpilogue {
  const float *sa;  // [M] row scales
  const float *sb;  // [N] column scales
  const float *zc;  // [N] 128 * column sums
  float *C;         // f32 output, row stride ldc (elements)
  int32_t *acc_out; // int32 output (kEpiI32)
  int ldc;
  int accumulate;   // C = dequant + C
  // kEpiGeglu, kEpiGegluQ
  int geglu_n;  // GeGLU output width (intermediate size)
  // kEpiGegluQ: the quantized GeGLU rows (uint8 q + 128, row stride ldq) and
  // their scales; neither may alias the A operand or sa.
  uint8_t *q_out;
  int ldq;
  float *sa_out;
  // kEpiF32Bias, kEpiGeluTanh
  const float *bias;  // [N], 16-byte aligned
  int seg_rows;       // kEpiGeluTanh: rows per GeluTanh call (its vector/tail split), >= 1;
                      // kEpiOutlierRes: rows per image
  int V;              // float32 lanes of that split
  // kEpiOutlierRes: per image its outlier count, the rows' set-aside values
  // [M][32] and the dequantized weight rows [images][32][N] of those channels.
  const int32_t *nout;
  const float *outv;
  const float *outw;
};

int gemm_u8s8(const GemmArgs &g, const GemmEpilogue &ep, int epi, cudaStream_t st);
// Whether the GeGLU GEMM can quantize its output rows itself (kEpiGegluQ).
bool gemm_geglu_q_fits(int N, const GemmEpilogue &ep);

// ---- row kernels (rows.cu) ----
// x (f32 [M][H]) -> LayerNorm (gamma) -> optional xn out -> per-row quantized
// uint8 q [M][ldq] + sa. gamma == nullptr: no norm, quantize x itself.
int launch_ln_quant(const float *x, const float *gamma, int M, int H, double eps, int V, float *xn, uint8_t *q,
                    int ldq, float *sa, cudaStream_t st);
// LayerNorm with a bias (LayerNormRow then AddTo(beta): the SigLIP norms),
// optional f32 output (may be x itself) and optional quantized copy.
int launch_ln_beta(const float *x, const float *gamma, const float *beta, int M, int H, double eps, int V, float *xout,
                   uint8_t *q, int ldq, float *sa, cudaStream_t st);
// An embedding table on the device in its stored format (Row,
// embeddings.go:49-68): f32 rows; bf16 rows widened exactly, with float32
// rows for the ids whose exact_idx >= 0; or int8 rows times a row scale.
struct EmbTable {
  int fmt;  // IG_EMB_F32 / IG_EMB_BF16 / IG_EMB_INT8
  const float *f32;
  const uint16_t *bf16;
  const int32_t *exact_idx;  // [vocab] -> row of exact_rows, or -1
  const float *exact_rows;
  const int8_t *i8;
  const float *scale;
};
// Element j of row id (id in range).
__device__ __forceinline__ float emb_elem(const EmbTable &t, int id, int j, int H) {
  if (t.fmt == IG_EMB_BF16) {
    const int e = __ldg(t.exact_idx + id);
    if (e >= 0) return __ldg(t.exact_rows + (size_t)e * H + j);
    return __uint_as_float((uint32_t)__ldg(t.bf16 + (size_t)id * H + j) << 16);
  }
  if (t.fmt == IG_EMB_INT8) return __fmul_rn((float)__ldg(t.i8 + (size_t)id * H + j), __ldg(t.scale + id));
  return __ldg(t.f32 + (size_t)id * H + j);
}
// Embedding gather then LayerNorm: x = LN(emb[ids]) (f32), and its quantized copy.
int launch_embed_checked(const int32_t *ids, int vocab, const EmbTable &emb, const float *gamma, int M, int H,
                         double eps, int V, float *x, uint8_t *q, int ldq, float *sa, cudaStream_t st);
// Per-row quantization of f32 rows (ld elements apart).
int launch_quant_rows(const float *x, int ldx, int M, int K, uint8_t *q, int ldq, float *sa, cudaStream_t st);
// Mean (float64, token order) or first-token pooling.
// Row -> sequence and position within it of every row of a batch, from its
// int32 offsets (one CTA per sequence).
int launch_fill_rows(const int32_t *offs, int nseq, int32_t *row_seq, int32_t *pos, cudaStream_t st);
// max_len, nrows: the batch's longest sequence and total rows (long
// sequences take the TMA-streamed kernel).
int launch_pool(const float *xn, const int32_t *offs, int nseq, int H, int cls, float *out, cudaStream_t st,
                int max_len, int nrows);
// Head logits in float64: z[t][r] = sum_i w[r][i] x[t][i] + b[r] (heads.go:62-74).
int launch_head_logits(const float *w, const float *b, int rows, int H, const float *x, int nx, double *z,
                       int ldz, cudaStream_t st);
// Weight quantization per output channel (PackB8, linalg/int8.go:36-77):
// w f32 [n][k] -> q int8 [n][ldq], scale, zc. Rows of `perm` (optional)
// choose the source channel of each packed row (-1: zero row).
int launch_pack_b8(const float *w, int n, int k, const int32_t *perm, int n_out, int8_t *q, int ldq, float *scale,
                   float *zc, int32_t *colsum, cudaStream_t st);

// ---- attention (attention.cu) ----
struct AttnArgs {
  const float *qkv;     // [N][3H] q, k, v rows
  int H, nh, D;
  const int32_t *offs;  // [nseq+1] row offsets (device)
  int nseq;
  int max_len;          // longest sequence
  int window;           // half window, < 0: global
  float scale;          // 1/sqrt(D)
  // RoPE (Rope, linalg/vec_simd.go:404-425) of q and k at each row's position
  // in its sequence, applied while preparing; null when qkv is already rotated.
  const float *rope_cos, *rope_sin;  // [positions][D/2]
  int V;                // lanes of ExpShift
  // work buffers (device)
  uint8_t *qa;          // [nh][N][D]
  float *sq;            // [nh][N]
  int8_t *kq;           // [nh][N][D]
  float *ks, *kzc;      // [nh][N]
  int8_t *vq;           // [nh][N][D]
  float *kmean;         // [nseq][nh][D]
  float *vs, *vinv;     // [nseq][nh][D]
  const int32_t *row_seq;  // [N] sequence of each row
  int N;
  // Optional: (sequence, first row) of every 64-row tile of every sequence
  // (device), for the tiled rotation and quantization of long sequences.
  const int2 *row_tiles = nullptr;
  int nrow_tiles = 0;
  float *ctx;           // [N][H] output
  // Optional (the fused short-sequence kernel, nh <= 8): instead of ctx, its
  // per-row int8 quantization (quant_rows over all heads of a row: bytes
  // q + 128 into xq with row pitch ldq, scales into sa).
  uint8_t *xq = nullptr;
  int ldq = 0;
  float *sa = nullptr;
  // Optional (the fused short-sequence kernel with the QKV projection in
  // front, qkv unused): the normalized rows quantized (uint8 q + 128, row
  // pitch lda, scales xa_s) and the QKV weights (int8 [3H][ldw] output
  // channel rows, scales wsb, 128 * column sums wzc).
  const uint8_t *xa = nullptr;
  int lda = 0;
  const float *xa_s = nullptr;
  const int8_t *wqkv = nullptr;
  int ldw = 0;
  const float *wsb = nullptr, *wzc = nullptr;
};
// Whether launch_attn_short can quantize ctx itself (AttnArgs::xq).
bool attn_short_quantizes(const AttnArgs &a);
int launch_attention(const AttnArgs &a, cudaStream_t st);
int launch_attn_exact(const AttnArgs &a, cudaStream_t st);
int launch_attend(const AttnArgs &a, const int2 *d_blocks, int nblocks, cudaStream_t st);
int attn_query_block();
// Tensor-core attention (attention_tc.cu): 128-query blocks whose keys span
// at most 256 columns.
int attn_tc_fits(int n, int i0, int window, int *c0_out, int *nkt_out);
int attn_tc_query_block();
int launch_attend_tc(const AttnArgs &a, const int4 *d_blocks, int nshort, int nlong, cudaStream_t st);
// Prepare + attend in one kernel (attention_short.cu): D = 64, sequences of at
// most 128 tokens, H a multiple of 4; RoPE applied when rope_cos is set.
bool attn_short_fits(const AttnArgs &a);
int launch_attn_short(const AttnArgs &a, cudaStream_t st);
// Whether the short-sequence kernel can also compute the QKV projection
// (AttnArgs::xa, ::wqkv; ctx quantized into xq): H = nh * 64 of 128 or 256.
bool attn_short_projects(const AttnArgs &a);

// Device error flag (kernels' bounded waits).
int read_device_error(int reset);

// ---- SigLIP pieces (siglip.cu) ----
// C[r][c] = chain(A[r] . W[c]) (+ bias[c]) (-> GeluTanh) (+ add[..][c]): the
// float32 product of linalg/gemm.go, one FMA chain per 256-deep block.
struct F32Gemm {
  const float *A;      // [M][lda] rows, or nullptr with pix
  int lda;
  const float *pix;    // patch rows read from pixels [n][3][S][S] (T patches per image)
  int S, P, T;
  const float *W;      // [N][ldw]
  int ldw;
  int M, N, K;
  const float *bias;   // [N] or nullptr
  int gelu_seg_rows;   // > 0: GeluTanh after the bias, calls of that many rows
  int V;
  const float *add;    // nullptr, or + add[(add_mod ? r % add_mod : r) * ldadd + c] last
  int ldadd, add_mod;
  float *C;
  int ldc;
  bool accumulate;     // C += each block's chain (MatMulPackedN with accumulate); no bias/GELU/add then
  bool vec_a, vec_w;   // set by the launcher
};
int launch_f32_gemm(const F32Gemm &p, cudaStream_t st);

// ---- the float32 encoder path (encoder_f32.cu) ----
// Rope (vec_simd.go:408-425) in place on the q and k heads of qkv rows
// [N][3H], positions pos[N], tables [npos][D/2].
int launch_rope_f32(float *qkv, const int32_t *pos, int N, int H, int nh, const float *cos_, const float *sin_,
                    cudaStream_t st);
// GeluMul (vec_simd.go:121-160) of each row: g[r] = gelu(z[r][:I]) * z[r][I:].
int launch_gelu_mul_rows(const float *z, int N, int I, float *g, cudaStream_t st);
// attendBlocks (internal/modernbert/infer.go:590-650) for every (sequence,
// head, block of 64 queries): tasks [ntasks] = (sequence, first query).
int launch_attend_blocks_f32(const float *qkv, const int32_t *seq_off, const int2 *tasks, int ntasks, int H, int nh,
                             int window, float scale, int V, float *ctx, cudaStream_t st);
// Float attention of the vision layers over the qkv rows [n*T][3H] -> ctx [n*T][H].
int launch_attn_f32(const float *qkv, int nimg, int T, int H, int nh, float scale, int V, float *ctx,
                    cudaStream_t st);
// Attention pooling: the probe's query over the K|V rows [n*T][2H] -> att [n][H].
int launch_pool_attn(const float *kv, const float *probe_q, int nimg, int T, int H, int nh, float scale, int V,
                     float *att, cudaStream_t st);
// MatMul8Outliers, before the int8 product: per image the outlier channels
// of x [n*T][K] (out [n][32], nout [n]), their values moved to outv
// [n*T][32] and zeroed in x. colmax [n][K] and cand [n][K] are scratch.
int launch_outliers_select(const float *x, int nimg, int T, int K, float ratio, float *colmax, int32_t *cand,
                           int32_t *out, int32_t *nout, float *outv, cudaStream_t st);
// After it: x += (c + the outlier terms in order) + bias, c the int8 product
// [n*T][N], q/scale the packed weights; w [n][32][N] is scratch for the
// dequantized weight rows of the outlier channels.
int launch_outliers_fixup(const float *c, int nimg, int T, int N, const int32_t *out, const int32_t *nout,
                          const float *outv, const int8_t *q, int ldq, const float *scale, const float *bias, float *w,
                          float *x, cudaStream_t st);

}  // namespace ig
