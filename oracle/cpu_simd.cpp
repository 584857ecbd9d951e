// CPU baseline, vector forms (test/bench infrastructure): the elementwise,
// normalisation and attention steps of the oracle's encoder in AVX2 with
// V = 8 float32 lanes, and attention's integer products on the VNNI units in
// the reference's 6 x 16 tiles. Lane k of a 256-bit register is the
// reference's lane k, every float operation is the scalar restatement's
// operation in the same order (FMA exactly where it has one), so the results
// equal the scalar oracle's bit for bit (tests/test_oracle_pins.py checks
// the encoder both ways). Where a row holds values the scalar code orders
// differently under NaN (maxima), the row is handed to the scalar function.
//
// Follows:
//   layernorm_row8   linalg/vec_simd.go:281-327 LayerNormRow (AVX2 branch)
//   quant_row8       linalg/quant_amd64.s:17-121 quantRowAVX2
//   exp_shift8       linalg/vec_simd.go:216-264 ExpShift
//   gelu_mul8        linalg/gelu_amd64.s:165-225 geluMulAVX2 (+ scalar tail)
//   rope8            linalg/vec_simd.go:404-425 Rope
//   dequant_row8     linalg/vec_simd.go:93-119 Dequantize
//   attn_prepare8    linalg/attention8.go:203-294 Prepare
//   attend8          linalg/attention8.go:298-376 Attend (VNNI tiles for
//                    S = Q.K^T and O = P.V, microKernel8Deq)
#include <immintrin.h>

#include <cmath>
#include <cstring>
#include <vector>

#include "oracle_internal.h"

namespace orc {

#define ORC_AVX2 __attribute__((target("avx2,fma")))

bool simd8_ok() {
  static const bool ok = [] {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && (cpu_features() & 3) != 0;
  }();
  return ok;
}

namespace {

ORC_AVX2 inline float hmax8(__m256 v) {
  alignas(32) float t[8];
  _mm256_store_ps(t, v);
  float m = t[0];
  for (int k = 1; k < 8; k++) m = std::max(m, t[k]);
  return m;
}

ORC_AVX2 inline int32_t hsum8i(__m256i v) {
  alignas(32) int32_t t[8];
  _mm256_store_si256((__m256i *)t, v);
  uint32_t s = 0;
  for (int k = 0; k < 8; k++) s += (uint32_t)t[k];
  return (int32_t)s;
}

// Eight int32 values clamped to int8 (VPACKSSDW + VPACKSSWB saturation), in
// order, as the low 8 bytes of the result.
ORC_AVX2 inline uint64_t pack8_s8(__m256i q) {
  const __m128i lo = _mm256_castsi256_si128(q), hi = _mm256_extracti128_si256(q, 1);
  const __m128i w = _mm_packs_epi32(lo, hi);
  const __m128i b = _mm_packs_epi16(w, w);
  return (uint64_t)_mm_cvtsi128_si64(b);
}

ORC_AVX2 inline bool all_finite(const float *x, int n) {
  const __m256 inf = _mm256_set1_ps(INFINITY), sign = _mm256_set1_ps(-0.0f);
  __m256 bad = _mm256_setzero_ps();
  int i = 0;
  for (; i + 8 <= n; i += 8) bad = _mm256_or_ps(bad, _mm256_cmp_ps(_mm256_andnot_ps(sign, _mm256_loadu_ps(x + i)), inf, _CMP_NLT_UQ));
  if (_mm256_movemask_ps(bad)) return false;
  for (; i < n; i++)
    if (!std::isfinite(x[i])) return false;
  return true;
}

// The vector body of exp_body for 8 lanes (v = x - m already formed).
ORC_AVX2 inline __m256 exp_body8(__m256 v) {
  const __m256 under = _mm256_cmp_ps(v, _mm256_set1_ps(-87.3f), _CMP_LT_OQ);
  // std::max(v, -87.3f) keeps a NaN v, as MAXPS does with v second.
  v = _mm256_max_ps(_mm256_set1_ps(-87.3f), v);
  v = _mm256_min_ps(_mm256_set1_ps(88.7f), v);
  const __m256 magic = _mm256_set1_ps(12582912.0f);
  const __m256 n = _mm256_sub_ps(_mm256_fmadd_ps(v, _mm256_set1_ps(1.44269504088896341f), magic), magic);
  __m256 r = _mm256_fmadd_ps(n, _mm256_set1_ps(-0.693359375f), v);
  r = _mm256_fmadd_ps(n, _mm256_set1_ps(2.12194440e-4f), r);
  __m256 p = _mm256_fmadd_ps(r, _mm256_set1_ps(1.9875691500e-4f), _mm256_set1_ps(1.3981999507e-3f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(8.3334519073e-3f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(4.1665795894e-2f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(1.6666665459e-1f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(5.0000001201e-1f));
  const __m256 y = _mm256_add_ps(_mm256_fmadd_ps(_mm256_mul_ps(p, r), r, r), _mm256_set1_ps(1.0f));
  const __m256i ni = _mm256_cvtps_epi32(n);
  const __m256 pw = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_add_epi32(ni, _mm256_set1_epi32(127)), 23));
  return _mm256_andnot_ps(under, _mm256_mul_ps(y, pw));
}

}  // namespace

// layernorm_row with V = 8.
ORC_AVX2 void layernorm_row8(float *o, const float *x, const float *gamma, int n, double eps) {
  __m256 lanes = _mm256_setzero_ps();
  int i = 0;
  for (; i + 8 <= n; i += 8) lanes = _mm256_add_ps(lanes, _mm256_loadu_ps(x + i));
  alignas(32) float t[8];
  _mm256_store_ps(t, lanes);
  double sum = 0.0;
  for (int k = 0; k < 8; k++) sum += (double)t[k];
  for (; i < n; i++) sum += (double)x[i];
  const float mean = (float)(sum / (double)n);
  const __m256 mv = _mm256_set1_ps(mean);
  __m256 sq = _mm256_setzero_ps();
  i = 0;
  for (; i + 8 <= n; i += 8) {
    const __m256 d = _mm256_sub_ps(_mm256_loadu_ps(x + i), mv);
    sq = _mm256_fmadd_ps(d, d, sq);
  }
  _mm256_store_ps(t, sq);
  double var = 0.0;
  for (int k = 0; k < 8; k++) var += (double)t[k];
  for (; i < n; i++) {
    const double d = (double)(x[i] - mean);
    var += d * d;
  }
  const float rstd = (float)(1.0 / std::sqrt(var / (double)n + eps));
  const __m256 rv = _mm256_set1_ps(rstd);
  int j = 0;
  for (; j + 8 <= n; j += 8)
    _mm256_storeu_ps(o + j, _mm256_mul_ps(_mm256_mul_ps(_mm256_sub_ps(_mm256_loadu_ps(x + j), mv), rv),
                                          _mm256_loadu_ps(gamma + j)));
  for (; j < n; j++) o[j] = ((x[j] - mean) * rstd) * gamma[j];
}

// quant_row (n a multiple of 8, finite inputs; otherwise the scalar form).
ORC_AVX2 float quant_row8(int8_t *dst, const float *x, const float *mean, int n, bool flip, int32_t *sum) {
  if ((n & 7) != 0) return quant_row(dst, x, mean, n, flip, sum);
  // One pass for the maximum and for values that are not finite (inputs,
  // means or differences), whose rows take the scalar form.
  const __m256 sign = _mm256_set1_ps(-0.0f), inf = _mm256_set1_ps(INFINITY);
  __m256 mx = _mm256_setzero_ps(), bad = _mm256_setzero_ps();
  for (int i = 0; i < n; i += 8) {
    __m256 c = _mm256_loadu_ps(x + i);
    if (mean) {
      const __m256 mv = _mm256_loadu_ps(mean + i);
      bad = _mm256_or_ps(bad, _mm256_cmp_ps(_mm256_andnot_ps(sign, c), inf, _CMP_NLT_UQ));
      bad = _mm256_or_ps(bad, _mm256_cmp_ps(_mm256_andnot_ps(sign, mv), inf, _CMP_NLT_UQ));
      c = _mm256_sub_ps(c, mv);
    }
    const __m256 a = _mm256_andnot_ps(sign, c);
    bad = _mm256_or_ps(bad, _mm256_cmp_ps(a, inf, _CMP_NLT_UQ));
    mx = _mm256_max_ps(a, mx);
  }
  if (_mm256_movemask_ps(bad)) return quant_row(dst, x, mean, n, flip, sum);
  const float m = hmax8(mx);
  if (m == 0.0f) {
    if (sum) *sum = 0;
    return 0.0f;
  }
  const float scale = m / 127.0f;
  const float inv = 1.0f / scale;
  const __m256 iv = _mm256_set1_ps(inv);
  __m256i s = _mm256_setzero_si256();
  const uint64_t fl = flip ? 0x8080808080808080ull : 0ull;
  for (int i = 0; i < n; i += 8) {
    __m256 c = _mm256_loadu_ps(x + i);
    if (mean) c = _mm256_sub_ps(c, _mm256_loadu_ps(mean + i));
    const __m256i q = _mm256_cvtps_epi32(_mm256_mul_ps(c, iv));
    s = _mm256_add_epi32(s, q);
    const uint64_t b = pack8_s8(q) ^ fl;
    std::memcpy(dst + i, &b, 8);
  }
  if (sum) *sum = hsum8i(s);
  return scale;
}

void quantize_a_row8(const float *x, int k, uint8_t *q, float *sa) {
  const float s = quant_row8(reinterpret_cast<int8_t *>(q), x, nullptr, k, true, nullptr);
  if (s == 0.0f) std::memset(q, 128, k);
  *sa = s;
}

// dequant of one row: ((float(acc) - zc) * sb) * sa (+ c).
ORC_AVX2 void dequant_row8(const int32_t *acc, int N, float sa, const float *sb, const float *zc, float *c,
                           bool accumulate) {
  const __m256 av = _mm256_set1_ps(sa);
  int j = 0;
  for (; j + 8 <= N; j += 8) {
    __m256 v = _mm256_sub_ps(_mm256_cvtepi32_ps(_mm256_loadu_si256((const __m256i *)(acc + j))), _mm256_loadu_ps(zc + j));
    v = _mm256_mul_ps(_mm256_mul_ps(v, _mm256_loadu_ps(sb + j)), av);
    if (accumulate) v = _mm256_add_ps(v, _mm256_loadu_ps(c + j));
    _mm256_storeu_ps(c + j, v);
  }
  for (; j < N; j++) {
    const float v = dequant1(acc[j], zc[j], sb[j], sa);
    c[j] = accumulate ? v + c[j] : v;
  }
}

// exp_shift with V = 8: the FMA body over whole 8-lane blocks from x[0], the
// eight lane sums added in lane order, then the exp32 tail.
ORC_AVX2 float exp_shift8(float *x, int n, float m) {
  const __m256 mv = _mm256_set1_ps(m);
  __m256 lanes = _mm256_setzero_ps();
  int i = 0;
  for (; i + 8 <= n; i += 8) {
    const __m256 e = exp_body8(_mm256_sub_ps(_mm256_loadu_ps(x + i), mv));
    _mm256_storeu_ps(x + i, e);
    lanes = _mm256_add_ps(lanes, e);
  }
  alignas(32) float t[8];
  _mm256_store_ps(t, lanes);
  float sum = 0.0f;
  for (int k = 0; k < 8; k++) sum += t[k];
  for (; i < n; i++) {
    const float e = exp32(x[i] - m);
    x[i] = e;
    sum += e;
  }
  return sum;
}

// gelu_mul: the FMA form over n &~ 15, the scalar form after.
ORC_AVX2 void gelu_mul8(float *o, const float *a, const float *b, int n) {
  const int nf = n & ~15;
  for (int i = 0; i < nf; i += 8) {
    const __m256 x = _mm256_loadu_ps(a + i);
    __m256 t = _mm256_mul_ps(x, _mm256_set1_ps(0.7071067811865476f));
    t = _mm256_max_ps(_mm256_set1_ps(-4.0f), t);
    t = _mm256_min_ps(_mm256_set1_ps(4.0f), t);
    const __m256 t2 = _mm256_mul_ps(t, t);
    __m256 p = _mm256_fmadd_ps(t2, _mm256_set1_ps(-2.72614225801306e-10f), _mm256_set1_ps(2.77068142495902e-08f));
    p = _mm256_fmadd_ps(t2, p, _mm256_set1_ps(-2.10102402082508e-06f));
    p = _mm256_fmadd_ps(t2, p, _mm256_set1_ps(-5.69250639462346e-05f));
    p = _mm256_fmadd_ps(t2, p, _mm256_set1_ps(-7.34990630326855e-04f));
    p = _mm256_fmadd_ps(t2, p, _mm256_set1_ps(-2.95459980854025e-03f));
    p = _mm256_fmadd_ps(t2, p, _mm256_set1_ps(-1.60960333262415e-02f));
    p = _mm256_mul_ps(p, t);
    __m256 q = _mm256_fmadd_ps(t2, _mm256_set1_ps(-1.45660718464996e-05f), _mm256_set1_ps(-2.13374055278905e-04f));
    q = _mm256_fmadd_ps(t2, q, _mm256_set1_ps(-1.68282697438203e-03f));
    q = _mm256_fmadd_ps(t2, q, _mm256_set1_ps(-7.37332916720468e-03f));
    q = _mm256_fmadd_ps(t2, q, _mm256_set1_ps(-1.42647390514189e-02f));
    const __m256 r = _mm256_add_ps(_mm256_div_ps(p, q), _mm256_set1_ps(1.0f));
    const __m256 h = _mm256_mul_ps(x, _mm256_set1_ps(0.5f));
    _mm256_storeu_ps(o + i, _mm256_mul_ps(_mm256_mul_ps(r, h), _mm256_loadu_ps(b + i)));
  }
  for (int i = nf; i < n; i++) o[i] = gelu_mul_scalar(a[i], b[i]);
}

// rope (rotate_half; separate roundings).
ORC_AVX2 void rope8(float *x, const float *c, const float *s, int half) {
  int i = 0;
  for (; i + 8 <= half; i += 8) {
    const __m256 a = _mm256_loadu_ps(x + i), b = _mm256_loadu_ps(x + half + i);
    const __m256 cv = _mm256_loadu_ps(c + i), sv = _mm256_loadu_ps(s + i);
    _mm256_storeu_ps(x + i, _mm256_sub_ps(_mm256_mul_ps(a, cv), _mm256_mul_ps(b, sv)));
    _mm256_storeu_ps(x + half + i, _mm256_add_ps(_mm256_mul_ps(b, cv), _mm256_mul_ps(a, sv)));
  }
  for (; i < half; i++) {
    const float a = x[i], b = x[half + i];
    x[i] = a * c[i] - b * s[i];
    x[half + i] = b * c[i] + a * s[i];
  }
}

// ---------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------

namespace {

// acc[r][c] = sum_q A[r][4q..4q+3] . B[q][c][0..3] for a 6 x 16 tile: all six
// rows of A are read (callers pad A to whole tiles), `rows` of them stored;
// the twelve accumulators stay in registers, as in the reference's kernel.
#define ORC_TILE_BODY(DPBUSD)                                                              \
  __m256i c[6][2];                                                                         \
  _Pragma("GCC unroll 6") for (int r = 0; r < 6; r++) c[r][0] = c[r][1] = _mm256_setzero_si256(); \
  for (int q = 0; q < kq; q++) {                                                           \
    const __m256i b0 = _mm256_loadu_si256((const __m256i *)(bp + q * 64));                 \
    const __m256i b1 = _mm256_loadu_si256((const __m256i *)(bp + q * 64 + 32));            \
    _Pragma("GCC unroll 6") for (int r = 0; r < 6; r++) {                                  \
      int32_t w;                                                                           \
      std::memcpy(&w, a + (size_t)r * lda + q * 4, 4);                                     \
      const __m256i av = _mm256_set1_epi32(w);                                             \
      c[r][0] = DPBUSD(c[r][0], av, b0);                                                   \
      c[r][1] = DPBUSD(c[r][1], av, b1);                                                   \
    }                                                                                      \
  }                                                                                        \
  _Pragma("GCC unroll 6") for (int r = 0; r < 6; r++) {                                    \
    _mm256_storeu_si256((__m256i *)(out + r * 16), c[r][0]);                               \
    _mm256_storeu_si256((__m256i *)(out + r * 16 + 8), c[r][1]);                           \
  }                                                                                        \
  (void)rows;

__attribute__((target("avxvnni,avx2"))) void tile_vnni(const uint8_t *a, int lda, int rows, const int8_t *bp,
                                                        int kq, int32_t *out) {
  ORC_TILE_BODY(_mm256_dpbusd_avx_epi32)
}
__attribute__((target("avx512vnni,avx512vl,avx2"))) void tile_vnni512(const uint8_t *a, int lda, int rows,
                                                                      const int8_t *bp, int kq, int32_t *out) {
  ORC_TILE_BODY(_mm256_dpbusd_epi32)
}

// The tile dequantized on the way out (microKernel8Deq): row r, column c
// ((float(acc) - zc[c]) * sb[c]) * sa[r], `cols` columns of `rows` rows
// stored at o + r * ldo.
#define ORC_TILE_DEQ_BODY(DPBUSD)                                                                    \
  __m256i c[6][2];                                                                                   \
  _Pragma("GCC unroll 6") for (int r = 0; r < 6; r++) c[r][0] = c[r][1] = _mm256_setzero_si256();    \
  for (int q = 0; q < kq; q++) {                                                                     \
    const __m256i b0 = _mm256_loadu_si256((const __m256i *)(bp + q * 64));                           \
    const __m256i b1 = _mm256_loadu_si256((const __m256i *)(bp + q * 64 + 32));                      \
    _Pragma("GCC unroll 6") for (int r = 0; r < 6; r++) {                                            \
      int32_t w;                                                                                     \
      std::memcpy(&w, a + (size_t)r * lda + q * 4, 4);                                               \
      const __m256i av = _mm256_set1_epi32(w);                                                       \
      c[r][0] = DPBUSD(c[r][0], av, b0);                                                             \
      c[r][1] = DPBUSD(c[r][1], av, b1);                                                             \
    }                                                                                                \
  }                                                                                                  \
  const __m256 z0 = _mm256_loadu_ps(zc), z1 = _mm256_loadu_ps(zc + 8);                               \
  const __m256 s0 = _mm256_loadu_ps(sb), s1 = _mm256_loadu_ps(sb + 8);                               \
  alignas(32) float t[6][16];                                                                        \
  _Pragma("GCC unroll 6") for (int r = 0; r < 6; r++) {                                              \
    const __m256 av = _mm256_set1_ps(sa[r]);                                                         \
    _mm256_store_ps(t[r], _mm256_mul_ps(_mm256_mul_ps(_mm256_sub_ps(_mm256_cvtepi32_ps(c[r][0]), z0), s0), av)); \
    _mm256_store_ps(t[r] + 8, _mm256_mul_ps(_mm256_mul_ps(_mm256_sub_ps(_mm256_cvtepi32_ps(c[r][1]), z1), s1), av)); \
  }                                                                                                  \
  for (int r = 0; r < rows; r++) std::memcpy(o + (size_t)r * ldo, t[r], sizeof(float) * cols);

__attribute__((target("avxvnni,avx2"))) void tile_deq_vnni(const uint8_t *a, int lda, int rows, const int8_t *bp,
                                                            int kq, const float *sb, const float *zc,
                                                            const float *sa, float *o, int ldo, int cols) {
  ORC_TILE_DEQ_BODY(_mm256_dpbusd_avx_epi32)
}
__attribute__((target("avx512vnni,avx512vl,avx2"))) void tile_deq_vnni512(const uint8_t *a, int lda, int rows,
                                                                          const int8_t *bp, int kq, const float *sb,
                                                                          const float *zc, const float *sa, float *o,
                                                                          int ldo, int cols) {
  ORC_TILE_DEQ_BODY(_mm256_dpbusd_epi32)
}

inline void tile6x16_deq(const uint8_t *a, int lda, int rows, const int8_t *bp, int kq, const float *sb,
                         const float *zc, const float *sa, float *o, int ldo, int cols) {
  static const int feat = cpu_features();
  if (feat & 1)
    tile_deq_vnni(a, lda, rows, bp, kq, sb, zc, sa, o, ldo, cols);
  else
    tile_deq_vnni512(a, lda, rows, bp, kq, sb, zc, sa, o, ldo, cols);
}

inline void tile6x16(const uint8_t *a, int lda, int rows, const int8_t *bp, int kq, int32_t *out) {
  static const int feat = cpu_features();
  if (feat & 1)
    tile_vnni(a, lda, rows, bp, kq, out);
  else
    tile_vnni512(a, lda, rows, bp, kq, out);
}

}  // namespace

// attn_prepare in vector form, plus the VNNI panels of K (keys as columns)
// and V (dimensions as columns, keys as depth), keys padded to 16.
ORC_AVX2 void attn_prepare8(const float *q, const float *k, const float *v, int ld, int n, int D, float scale,
                            AttnPrep8 &P) {
  if ((D & 15) != 0 || D > 512) {  // the vector forms take whole 16-column panels
    attn_prepare(q, k, v, ld, n, D, scale, P.base);
    return;
  }
  {
    AttnPrep &B = P.base;
    B.n = n;
    B.D = D;
    B.qa.assign((size_t)n * D, 128);
    B.sq.assign(n, 0.0f);
    B.kq.assign((size_t)n * D, 0);
    B.ks.assign(n, 0.0f);
    B.kzc.assign(n, 0.0f);
    B.vq.assign((size_t)n * D, 0);
    B.vs.assign(D, 0.0f);
    B.kmean.assign(D, 0.0f);
    for (int i = 0; i < n; i++) {
      int8_t *dst = reinterpret_cast<int8_t *>(B.qa.data() + (size_t)i * D);
      const float s = quant_row8(dst, q + (size_t)i * ld, nullptr, D, true, nullptr);
      if (s != 0.0f)
        B.sq[i] = s * scale;
      else
        std::memset(B.qa.data() + (size_t)i * D, 128, D);
    }
    // K mean: keys added in order, every column its own chain.
    for (int j = 0; j < n; j++)
      for (int d = 0; d < D; d += 8)
        _mm256_storeu_ps(&B.kmean[d], _mm256_add_ps(_mm256_loadu_ps(&B.kmean[d]), _mm256_loadu_ps(k + (size_t)j * ld + d)));
    const float invn = 1.0f / (float)n;
    for (int d = 0; d < D; d += 8) _mm256_storeu_ps(&B.kmean[d], _mm256_mul_ps(_mm256_loadu_ps(&B.kmean[d]), _mm256_set1_ps(invn)));
    for (int j = 0; j < n; j++) {
      int32_t sum = 0;
      int8_t kb[512];
      const float s = quant_row8(kb, k + (size_t)j * ld, B.kmean.data(), D, false, &sum);
      if (s == 0.0f) continue;
      B.ks[j] = s;
      B.kzc[j] = 128.0f * (float)sum;
      std::memcpy(B.kq.data() + (size_t)j * D, kb, D);
    }
    // V per column: maxima (NaN-ignoring, as std::max with the maximum first).
    bool finite = true;
    for (int j = 0; j < n && finite; j++) finite = all_finite(v + (size_t)j * ld, D);
    if (!finite) {
      AttnPrep tmp;
      attn_prepare(q, k, v, ld, n, D, scale, tmp);
      B.vq = tmp.vq;
      B.vs = tmp.vs;
    } else {
      const __m256 sign = _mm256_set1_ps(-0.0f);
      for (int j = 0; j < n; j++)
        for (int d = 0; d < D; d += 8)
          _mm256_storeu_ps(&B.vs[d], _mm256_max_ps(_mm256_andnot_ps(sign, _mm256_loadu_ps(v + (size_t)j * ld + d)),
                                                   _mm256_loadu_ps(&B.vs[d])));
      std::vector<float> vinv(D, 0.0f);
      for (int d = 0; d < D; d++)
        if (B.vs[d] > 0.0f) {
          B.vs[d] /= 127.0f;
          vinv[d] = 1.0f / B.vs[d];
        }
      for (int j = 0; j < n; j++)
        for (int d = 0; d < D; d += 8) {
          const __m256i qv = _mm256_cvtps_epi32(_mm256_mul_ps(_mm256_loadu_ps(v + (size_t)j * ld + d), _mm256_loadu_ps(&vinv[d])));
          const uint64_t b = pack8_s8(qv);
          std::memcpy(B.vq.data() + (size_t)j * D + d, &b, 8);
        }
    }
  }
  // Panels: K [n16/16][D/4][16][4], V [D/16][n16/4][16][4] (padding zero).
  const int n16 = (n + 15) / 16 * 16, kqd = D / 4, D16 = (D + 15) / 16 * 16;
  P.n16 = n16;
  P.kp.assign((size_t)n16 * ((D + 3) / 4 * 4), 0);
  P.vp.assign((size_t)D16 * n16, 0);
  const AttnPrep &B = P.base;
  for (int j = 0; j < n; j++)
    for (int d = 0; d < D; d++) P.kp[(size_t)(j / 16) * kqd * 64 + (d / 4) * 64 + (j % 16) * 4 + d % 4] = B.kq[(size_t)j * D + d];
  for (int j = 0; j < n; j++)
    for (int d = 0; d < D; d++)
      P.vp[(size_t)(d / 16) * (n16 / 4) * 64 + (j / 4) * 64 + (d % 16) * 4 + j % 4] = B.vq[(size_t)j * D + d];
  P.qpad.assign((size_t)(n + 6) * D, 128);
  std::memcpy(P.qpad.data(), B.qa.data(), (size_t)n * D);
  P.ks16.assign(n16, 0.0f);
  P.kzc16.assign(n16, 0.0f);
  P.sq6.assign(n + 6, 0.0f);
  std::memcpy(P.ks16.data(), B.ks.data(), sizeof(float) * n);
  std::memcpy(P.kzc16.data(), B.kzc.data(), sizeof(float) * n);
  std::memcpy(P.sq6.data(), B.sq.data(), sizeof(float) * n);
}

// Attend for the queries [i0, i1) (i1 - i0 <= kAttnBlock8) with output row i
// at o + (i - i0) * ldo: the block's keys in whole 16-key panels, S by VNNI
// tiles and dequantized per element, the softmax per row, P = rne(e * 255),
// O = P.V by VNNI tiles over the block's key panels.
ORC_AVX2 void attend8(const AttnPrep8 &P, int i0, int i1, int window, float *o, int ldo, AttnScratch8 &sc) {
  const AttnPrep &B = P.base;
  const int n = B.n, D = B.D, n16 = P.n16;
  if ((D & 15) != 0 || D > 512 || i0 >= i1) {  // whole dimension panels only
    std::vector<float> srow(n);
    std::vector<uint8_t> prow(n);
    for (int i = i0; i < i1; i++) attn_row(B, i, window, 8, o + (size_t)(i - i0) * ldo, srow.data(), prow.data(), nullptr, nullptr, nullptr);
    return;
  }
  int c0 = 0, c1 = n16;
  if (window >= 0) {
    c0 = std::max(0, i0 - window) / 16 * 16;
    c1 = std::min(n16, (i1 - 1 + window + 1 + 15) / 16 * 16);
  }
  const int W = c1 - c0, rows = i1 - i0, kqd = D / 4;
  sc.s.resize((size_t)kAttnBlock8 * W);
  sc.p.assign((size_t)(kAttnBlock8 + 6) * W, 0);
  sc.sp.assign(kAttnBlock8 + 6, 0.0f);
  for (int r0 = 0; r0 < rows; r0 += 6) {
    const int rr = std::min(6, rows - r0);
    for (int p = c0 / 16; p < c1 / 16; p++)
      tile6x16_deq(P.qpad.data() + (size_t)(i0 + r0) * D, D, rr, P.kp.data() + (size_t)p * kqd * 64, kqd,
                   P.ks16.data() + p * 16, P.kzc16.data() + p * 16, P.sq6.data() + i0 + r0,
                   &sc.s[(size_t)r0 * W + p * 16 - c0], W, std::min(16, n - p * 16));
  }
  for (int r = 0; r < rows; r++) {
    const int i = i0 + r;
    float *row = &sc.s[(size_t)r * W];
    uint8_t *prow = &sc.p[(size_t)r * W];
    int cs = 0, ce = std::min(n, c1) - c0;
    if (window >= 0) cs = std::max(0, i - window - c0), ce = std::min(n, i + window + 1) - c0;
    const int len = ce - cs;
    float *valid = row + cs;
    // MaxOf (NaN-ignoring as std::max with the maximum first); a row with a
    // non-finite score goes through the scalar softmax.
    if (!all_finite(valid, len)) {
      float mx = -INFINITY;
      for (int j = 0; j < len; j++) mx = std::max(mx, valid[j]);
      exp_shift(valid, len, mx, 8);
      int32_t qsum = 0;
      for (int j = 0; j < len; j++) {
        const int32_t qi = (int32_t)round_half_even(valid[j] * 255.0f);
        prow[cs + j] = (uint8_t)qi;
        qsum += qi;
      }
      sc.sp[r] = 1.0f / (float)qsum;
      continue;
    }
    __m256 mv = _mm256_set1_ps(-INFINITY);
    int j = 0;
    for (; j + 8 <= len; j += 8) mv = _mm256_max_ps(_mm256_loadu_ps(valid + j), mv);
    float mx = hmax8(mv);
    for (; j < len; j++) mx = std::max(mx, valid[j]);
    exp_shift8(valid, len, mx);
    // QuantizeRowU8(prow, valid, 255): e in [0, 1], e * 255 rounded to even.
    __m256i qs = _mm256_setzero_si256();
    j = 0;
    for (; j + 8 <= len; j += 8) {
      const __m256i qi = _mm256_cvtps_epi32(_mm256_mul_ps(_mm256_loadu_ps(valid + j), _mm256_set1_ps(255.0f)));
      qs = _mm256_add_epi32(qs, qi);
      const __m128i w = _mm_packs_epi32(_mm256_castsi256_si128(qi), _mm256_extracti128_si256(qi, 1));
      const uint64_t b = (uint64_t)_mm_cvtsi128_si64(_mm_packus_epi16(w, w));
      std::memcpy(prow + cs + j, &b, 8);
    }
    int32_t qsum = hsum8i(qs);
    for (; j < len; j++) {
      const int32_t qi = (int32_t)round_half_even(valid[j] * 255.0f);
      prow[cs + j] = (uint8_t)qi;
      qsum += qi;
    }
    sc.sp[r] = 1.0f / (float)qsum;
  }
  // O = P.V over the block's key panels, depth W (a multiple of 16).
  static const float zeros[16] = {0};
  for (int r0 = 0; r0 < rows; r0 += 6) {
    const int rr = std::min(6, rows - r0);
    for (int p = 0; p < D / 16; p++)
      tile6x16_deq(&sc.p[(size_t)r0 * W], W, rr, P.vp.data() + (size_t)p * (n16 / 4) * 64 + (c0 / 4) * 64, W / 4,
                   B.vs.data() + p * 16, zeros, sc.sp.data() + r0, o + (size_t)r0 * ldo + p * 16, ldo, 16);
  }
}

}  // namespace orc
