// CPU oracle (test infrastructure): scalar restatement of the reference's int8
// encoder arithmetic. See oracle.h for scope, citations and parity status.
// Build: oracle/Makefile (-O2 -ffp-contract=off).
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "oracle_internal.h"

namespace orc {

// ---------------------------------------------------------------------------
// Elementary operations
// ---------------------------------------------------------------------------

// linalg/int8.go:205-210 roundHalfEven: (v + 1.5*2^23) - 1.5*2^23, two roundings.
float round_half_even(float v) {
  const float magic = 12582912.0f;
  float t = v + magic;
  return t - magic;
}

float abs32(float v) { return std::fabs(v); }

// linalg/fastmath.go:35-51 exp32 (scalar, no FMA: GOAMD64=v1 does not contract).
float exp32(float x) {
  if (x < -87.3f) return 0.0f;
  x = std::min(x, 88.7f);
  float n = round_half_even(x * 1.44269504088896341f);
  float r = x - n * 0.693359375f;
  r = r - n * -2.12194440e-4f;
  float p = 1.9875691500e-4f;
  p = p * r + 1.3981999507e-3f;
  p = p * r + 8.3334519073e-3f;
  p = p * r + 4.1665795894e-2f;
  p = p * r + 1.6666665459e-1f;
  p = p * r + 5.0000001201e-1f;
  float y = p * r * r + r + 1.0f;
  uint32_t bits = (uint32_t)((int32_t)n + 127) << 23;
  float pw;
  std::memcpy(&pw, &bits, 4);
  return y * pw;
}

// The vector body of linalg/vec_simd.go:234-250 ExpShift for one lane
// (v = x - m already formed): MulAdd is a fused multiply-add.
float exp_body(float v) {
  const bool under = v < -87.3f;
  v = std::min(std::max(v, -87.3f), 88.7f);
  float n = std::fma(v, 1.44269504088896341f, 12582912.0f) - 12582912.0f;
  float r = std::fma(n, -0.693359375f, v);
  r = std::fma(n, 2.12194440e-4f, r);  // ln2lo.Neg() with ln2lo = -2.12194440e-4
  float p = std::fma(r, 1.9875691500e-4f, 1.3981999507e-3f);
  p = std::fma(r, p, 8.3334519073e-3f);
  p = std::fma(r, p, 4.1665795894e-2f);
  p = std::fma(r, p, 1.6666665459e-1f);
  p = std::fma(r, p, 5.0000001201e-1f);
  float y = std::fma(p * r, r, r) + 1.0f;
  int32_t ni = (int32_t)std::nearbyint(n);  // VCVTPS2DQ; n is integral
  uint32_t bits = (uint32_t)(ni + 127) << 23;
  float pw;
  std::memcpy(&pw, &bits, 4);
  return under ? 0.0f : y * pw;
}

// The widest SIMD width a configuration may name (simd_lanes in [1, 32]).
constexpr int kMaxLanes = 32;

// linalg/vec_simd.go:216-264 ExpShift: x[i] = exp(x[i]-m); lanes in V-wide
// blocks use the FMA body, the tail (n mod V) uses exp32. Returns the sum.
float exp_shift(float *x, int n, float m, int V) {
  float lanes[kMaxLanes] = {0};
  int i = 0;
  for (; i + V <= n; i += V) {
    for (int k = 0; k < V; k++) {
      float e = exp_body(x[i + k] - m);
      x[i + k] = e;
      lanes[k] += e;
    }
  }
  float sum = 0.0f;
  for (int k = 0; k < V; k++) sum += lanes[k];
  for (; i < n; i++) {
    float e = exp32(x[i] - m);
    x[i] = e;
    sum += e;
  }
  return sum;
}

// linalg/fastmath.go:7-24 erf32 (scalar; no FMA).
float erf32(float x) {
  x = std::min(std::max(x, -4.0f), 4.0f);
  float x2 = x * x;
  float p = x2 * -2.72614225801306e-10f + 2.77068142495902e-08f;
  p = x2 * p + -2.10102402082508e-06f;
  p = x2 * p + -5.69250639462346e-05f;
  p = x2 * p + -7.34990630326855e-04f;
  p = x2 * p + -2.95459980854025e-03f;
  p = x2 * p + -1.60960333262415e-02f;
  p *= x;
  float q = x2 * -1.45660718464996e-05f + -2.13374055278905e-04f;
  q = x2 * q + -1.68282697438203e-03f;
  q = x2 * q + -7.37332916720468e-03f;
  q = x2 * q + -1.42647390514189e-02f;
  return p / q;
}

// linalg/gelu_amd64.s:165-225 geluMulAVX2 for one element: FMA polynomial
// (VFMADD213PS), then ((p/q + 1) * (x*0.5)) * gate.
float gelu_mul_fma(float x, float gate) {
  float t = x * 0.7071067811865476f;
  t = std::max(t, -4.0f);
  t = std::min(t, 4.0f);
  float t2 = t * t;
  float p = std::fma(t2, -2.72614225801306e-10f, 2.77068142495902e-08f);
  p = std::fma(t2, p, -2.10102402082508e-06f);
  p = std::fma(t2, p, -5.69250639462346e-05f);
  p = std::fma(t2, p, -7.34990630326855e-04f);
  p = std::fma(t2, p, -2.95459980854025e-03f);
  p = std::fma(t2, p, -1.60960333262415e-02f);
  p = p * t;
  float q = std::fma(t2, -1.45660718464996e-05f, -2.13374055278905e-04f);
  q = std::fma(t2, q, -1.68282697438203e-03f);
  q = std::fma(t2, q, -7.37332916720468e-03f);
  q = std::fma(t2, q, -1.42647390514189e-02f);
  float r = p / q;
  r = r + 1.0f;
  float h = x * 0.5f;
  float g = r * h;
  return g * gate;
}

// linalg/fastmath.go:26 geluScalar(x) * b (the tail of GeluMul, vec_simd.go:157-159).
float gelu_mul_scalar(float x, float gate) {
  float g = 0.5f * x * (1.0f + erf32(x * 0.7071067811865476f));
  return g * gate;
}

// linalg/vec_simd.go:121-160 GeluMul on amd64: geluMulFast covers n &^ 15
// (kernel_amd64.go:279-290), the rest is scalar.
void gelu_mul(float *o, const float *a, const float *b, int n) {
  int nf = n & ~15;
  for (int i = 0; i < nf; i++) o[i] = gelu_mul_fma(a[i], b[i]);
  for (int i = nf; i < n; i++) o[i] = gelu_mul_scalar(a[i], b[i]);
}

// linalg/vec_simd.go:281-327 LayerNormRow with V float32 lanes.
void layernorm_row(float *o, const float *x, const float *gamma, int n, double eps, int V) {
  float lanes[kMaxLanes] = {0};
  int i = 0;
  for (; i + V <= n; i += V)
    for (int k = 0; k < V; k++) lanes[k] += x[i + k];
  double sum = 0.0;
  for (int k = 0; k < V; k++) sum += (double)lanes[k];
  for (; i < n; i++) sum += (double)x[i];
  const float mean = (float)(sum / (double)n);
  float sq[kMaxLanes] = {0};
  i = 0;
  for (; i + V <= n; i += V)
    for (int k = 0; k < V; k++) {
      float d = x[i + k] - mean;
      sq[k] = std::fma(d, d, sq[k]);
    }
  double var = 0.0;
  for (int k = 0; k < V; k++) var += (double)sq[k];
  for (; i < n; i++) {
    double d = (double)(x[i] - mean);
    var += d * d;
  }
  const float rstd = (float)(1.0 / std::sqrt(var / (double)n + eps));
  for (int j = 0; j < n; j++) o[j] = ((x[j] - mean) * rstd) * gamma[j];
}

// linalg/vec_simd.go:404-425 Rope (rotate_half, no FMA).
void rope(float *x, const float *c, const float *s, int half) {
  for (int i = 0; i < half; i++) {
    float a = x[i], b = x[half + i];
    x[i] = a * c[i] - b * s[i];
    x[half + i] = b * c[i] + a * s[i];
  }
}

// internal/modernbert/model.go:255-277 ropeFor: float64 pow/cos/sin, float32
// frequencies and positions.
void rope_table(double theta, int D, int npos, float *cs, float *sn) {
  int half = D / 2;
  for (int i = 0; i < half; i++) {
    float inv = (float)(1.0 / std::pow(theta, (double)(2 * i) / (double)D));
    for (int p = 0; p < npos; p++) {
      double f = (double)((float)p * inv);
      cs[p * half + i] = (float)std::cos(f);
      sn[p * half + i] = (float)std::sin(f);
    }
  }
}

// linalg/quant_amd64.s:17-121 quantRowAVX2: c = x - mean, scale = max|c|/127,
// q = rne(c * (1/scale)), optional top-bit flip; sum of the int8 values.
float quant_row(int8_t *dst, const float *x, const float *mean, int n, bool flip, int32_t *sum) {
  float mx = 0.0f;
  for (int i = 0; i < n; i++) mx = std::max(mx, abs32(x[i] - (mean ? mean[i] : 0.0f)));
  if (mx == 0.0f) {
    if (sum) *sum = 0;
    return 0.0f;
  }
  const float scale = mx / 127.0f;
  const float inv = 1.0f / scale;
  int32_t s = 0;
  for (int i = 0; i < n; i++) {
    float c = x[i] - (mean ? mean[i] : 0.0f);
    int32_t q = (int32_t)std::nearbyint(c * inv);  // VCVTPS2DQ: round to nearest even
    s += q;                                          // VPADDD before narrowing
    q = std::min(127, std::max(-128, q));            // VPACKSS saturation
    dst[i] = (int8_t)(flip ? (q ^ 0x80) : q);
  }
  if (sum) *sum = s;
  return scale;
}

// ---------------------------------------------------------------------------
// int8 GEMM
// ---------------------------------------------------------------------------

// linalg/int8.go:36-77 PackB8: per output channel j, s = max|w|/127 (float32),
// q = int8(math.Round(float64(w/s))) (half away from zero), colsum, zc = 128*colsum.
void pack_b8(const float *b, int k, int n, bool transB, int8_t *q, float *scale, int32_t *colsum, float *zc) {
  for (int j = 0; j < n; j++) {
    auto at = [&](int d) { return transB ? b[(size_t)j * k + d] : b[(size_t)d * n + j]; };
    float mx = 0.0f;
    for (int d = 0; d < k; d++) mx = std::max(mx, abs32(at(d)));
    scale[j] = 0.0f;
    colsum[j] = 0;
    std::memset(q + (size_t)j * k, 0, k);
    if (mx == 0.0f) {
      zc[j] = 0.0f;
      continue;
    }
    const float s = mx / 127.0f;
    scale[j] = s;
    int32_t cs = 0;
    for (int d = 0; d < k; d++) {
      float qf = at(d) / s;
      int8_t v = (int8_t)std::round((double)qf);
      q[(size_t)j * k + d] = v;
      cs += v;
    }
    colsum[j] = cs;
    zc[j] = 128.0f * (float)cs;
  }
}

// linalg/int8.go:157-191 quantizeA (both its AVX2 and Go branches compute
// s = max/127, q = rne(x * (1/s)) + 128).
void quantize_a_row(const float *x, int k, uint8_t *q, float *sa) {
  float s = quant_row(reinterpret_cast<int8_t *>(q), x, nullptr, k, true, nullptr);
  if (s == 0.0f) std::memset(q, 128, k);
  *sa = s;
}

void gemm_u8s8(const uint8_t *A, int lda, const int8_t *B, int ldb, int M, int N, int K, int32_t *acc) {
  for (int i = 0; i < M; i++)
    for (int j = 0; j < N; j++) {
      int32_t s = 0;
      const uint8_t *a = A + (size_t)i * lda;
      const int8_t *w = B + (size_t)j * ldb;
      for (int d = 0; d < K; d++) s += (int32_t)a[d] * (int32_t)w[d];
      acc[(size_t)i * N + j] = s;
    }
}

// linalg/kernel_vnni_amd64.s:144-234 (and Dequantize, vec_simd.go:93-119):
// ((float(acc) - zc) * sb) * sa, then + c_old when accumulating.
float dequant1(int32_t acc, float zc, float sb, float sa) {
  float v = (float)acc - zc;
  v = v * sb;
  return v * sa;
}

void dequant(const int32_t *acc, int M, int N, const float *sa, const float *sb, const float *zc, float *C,
             bool accumulate) {
  for (int i = 0; i < M; i++)
    for (int j = 0; j < N; j++) {
      float v = dequant1(acc[(size_t)i * N + j], zc[j], sb[j], sa[i]);
      float *c = C + (size_t)i * N + j;
      *c = accumulate ? v + *c : v;
    }
}

// linalg/int8.go:88-155 MatMul8N (its tiles and edges all compute the same
// per-element arithmetic, int8_test.go:146-171).
void matmul8(float *c, const float *a, int m, const int8_t *q, const float *scale, const float *zc, int k, int n,
             bool accumulate, std::vector<uint8_t> &abuf, std::vector<float> &sbuf, std::vector<int32_t> &accbuf,
             int32_t *acc_dump, uint8_t *aq_dump, float *sa_dump) {
  abuf.resize((size_t)m * k);
  sbuf.resize(m);
  accbuf.resize((size_t)m * n);
  for (int i = 0; i < m; i++) quantize_a_row(a + (size_t)i * k, k, abuf.data() + (size_t)i * k, &sbuf[i]);
  gemm_u8s8(abuf.data(), k, q, k, m, n, k, accbuf.data());
  dequant(accbuf.data(), m, n, sbuf.data(), scale, zc, c, accumulate);
  if (acc_dump) std::memcpy(acc_dump, accbuf.data(), sizeof(int32_t) * m * n);
  if (aq_dump) std::memcpy(aq_dump, abuf.data(), (size_t)m * k);
  if (sa_dump) std::memcpy(sa_dump, sbuf.data(), sizeof(float) * m);
}

// ---------------------------------------------------------------------------
// Attention (linalg/attention8.go:203-376, AVX2 branch: D % 32 == 0 there;
// the same arithmetic is used for every D here)
// ---------------------------------------------------------------------------

void attn_prepare(const float *q, const float *k, const float *v, int ld, int n, int D, float scale, AttnPrep &P) {
  P.n = n;
  P.D = D;
  P.qa.assign((size_t)n * D, 128);
  P.sq.assign(n, 0.0f);
  P.kq.assign((size_t)n * D, 0);
  P.ks.assign(n, 0.0f);
  P.kzc.assign(n, 0.0f);
  P.vq.assign((size_t)n * D, 0);
  P.vs.assign(D, 0.0f);
  P.kmean.assign(D, 0.0f);
  std::vector<float> vinv(D, 0.0f);
  // Q per row, the score scale folded into its scale (attention8.go:210-220).
  for (int i = 0; i < n; i++) {
    int8_t *dst = reinterpret_cast<int8_t *>(P.qa.data() + (size_t)i * D);
    float s = quant_row(dst, q + (size_t)i * ld, nullptr, D, true, nullptr);
    if (s != 0.0f)
      P.sq[i] = s * scale;
    else
      std::memset(P.qa.data() + (size_t)i * D, 128, D);
  }
  // K mean: AddTo over keys in order, then Scale by 1/float32(n) (attention8.go:224-229).
  for (int j = 0; j < n; j++)
    for (int d = 0; d < D; d++) P.kmean[d] += k[(size_t)j * ld + d];
  const float invn = 1.0f / (float)n;
  for (int d = 0; d < D; d++) P.kmean[d] *= invn;
  // Centred K per key (attention8.go:240-251).
  for (int j = 0; j < n; j++) {
    int32_t sum = 0;
    std::vector<int8_t> kb(D);
    float s = quant_row(kb.data(), k + (size_t)j * ld, P.kmean.data(), D, false, &sum);
    if (s == 0.0f) continue;
    P.ks[j] = s;
    P.kzc[j] = 128.0f * (float)sum;
    std::memcpy(P.kq.data() + (size_t)j * D, kb.data(), D);
  }
  // V per column (attention8.go:255-279).
  for (int j = 0; j < n; j++)
    for (int d = 0; d < D; d++) P.vs[d] = std::max(P.vs[d], abs32(v[(size_t)j * ld + d]));
  for (int d = 0; d < D; d++) {
    vinv[d] = 0.0f;
    if (P.vs[d] > 0.0f) {
      P.vs[d] /= 127.0f;
      vinv[d] = 1.0f / P.vs[d];
    }
  }
  for (int j = 0; j < n; j++)
    for (int d = 0; d < D; d++) {
      int32_t qv = (int32_t)std::nearbyint(v[(size_t)j * ld + d] * vinv[d]);
      qv = std::min(127, std::max(-128, qv));
      P.vq[(size_t)j * D + d] = (int8_t)qv;
    }
}

// One query row of Attend (attention8.go:335-374). s_row, p_row: scratch [n].
void attn_row(const AttnPrep &P, int i, int window, int V, float *o, float *s_row, uint8_t *p_row, float *sp_out,
              int32_t *sacc_row, int32_t *oacc_row) {
  const int n = P.n, D = P.D;
  int js = 0, je = n;
  if (window >= 0) {
    js = std::max(0, i - window);
    je = std::min(n, i + window + 1);
  }
  const uint8_t *qa = P.qa.data() + (size_t)i * D;
  for (int j = js; j < je; j++) {
    const int8_t *kq = P.kq.data() + (size_t)j * D;
    int32_t acc = 0;
    for (int d = 0; d < D; d++) acc += (int32_t)qa[d] * (int32_t)kq[d];
    if (sacc_row) sacc_row[j] = acc;
    s_row[j] = dequant1(acc, P.kzc[j], P.ks[j], P.sq[i]);
  }
  const int len = je - js;
  float mx = -INFINITY;
  for (int j = js; j < je; j++) mx = std::max(mx, s_row[j]);
  exp_shift(s_row + js, len, mx, V);
  // QuantizeRowU8(prow, valid, 255): q = rne(e*255), sum of q (vec_simd.go:59-91).
  std::memset(p_row, 0, n);
  int32_t qsum = 0;
  for (int j = js; j < je; j++) {
    float t = round_half_even(s_row[j] * 255.0f);
    int32_t qi = (int32_t)t;
    p_row[j] = (uint8_t)qi;
    qsum += qi;
  }
  const float sp = 1.0f / (float)qsum;
  if (sp_out) *sp_out = sp;
  for (int d = 0; d < D; d++) {
    int32_t acc = 0;
    for (int j = js; j < je; j++) acc += (int32_t)p_row[j] * (int32_t)P.vq[(size_t)j * D + d];
    if (oacc_row) oacc_row[d] = acc;
    o[d] = dequant1(acc, 0.0f, P.vs[d], sp);
  }
}

}  // namespace orc

using namespace orc;

extern "C" {

float or_round_half_even(float v) { return round_half_even(v); }
float or_exp32(float x) { return exp32(x); }
float or_erf32(float x) { return erf32(x); }
float or_exp_shift(float *x, int n, float m, int V) { return exp_shift(x, n, m, V); }
void or_gelu_mul(float *o, const float *a, const float *b, int n) { gelu_mul(o, a, b, n); }
void or_layernorm_row(float *o, const float *x, const float *gamma, int n, double eps, int V) {
  layernorm_row(o, x, gamma, n, eps, V);
}
void or_rope(float *x, const float *c, const float *s, int half) { rope(x, c, s, half); }
void or_rope_table(double theta, int D, int npos, float *c, float *s) { rope_table(theta, D, npos, c, s); }
float or_quant_row(int8_t *dst, const float *x, const float *mean, int n, int flip, int32_t *sum) {
  return quant_row(dst, x, mean, n, flip != 0, sum);
}
void or_pack_b8(const float *b, int k, int n, int transB, int8_t *q, float *scale, int32_t *colsum, float *zc) {
  pack_b8(b, k, n, transB != 0, q, scale, colsum, zc);
}
void or_quantize_a(const float *a, int m, int k, uint8_t *q, float *sa) {
  for (int i = 0; i < m; i++) quantize_a_row(a + (size_t)i * k, k, q + (size_t)i * k, sa + i);
}
void or_gemm_u8s8(const uint8_t *A, int lda, const int8_t *B, int ldb, int M, int N, int K, int32_t *acc) {
  gemm_u8s8(A, lda, B, ldb, M, N, K, acc);
}
void or_dequant(const int32_t *acc, int M, int N, const float *sa, const float *sb, const float *zc, float *C,
                int accumulate) {
  dequant(acc, M, N, sa, sb, zc, C, accumulate != 0);
}
void or_matmul8(float *c, const float *a, int m, const int8_t *q, const float *scale, const float *zc, int k,
                int n, int accumulate) {
  std::vector<uint8_t> ab;
  std::vector<float> sb;
  std::vector<int32_t> acc;
  matmul8(c, a, m, q, scale, zc, k, n, accumulate != 0, ab, sb, acc, nullptr, nullptr, nullptr);
}

void or_attn8(const float *q, const float *k, const float *v, int ld, int n, int D, int window, float scale,
              float *o, int ldo, or_attn_dbg *dbg) {
  if (n <= 0) return;
  AttnPrep P;
  attn_prepare(q, k, v, ld, n, D, scale, P);
  std::vector<float> srow(n);
  std::vector<uint8_t> prow(n);
  for (int i = 0; i < n; i++) {
    float sp;
    attn_row(P, i, window, 8, o + (size_t)i * ldo, srow.data(), prow.data(), &sp,
             dbg && dbg->sacc ? dbg->sacc + (size_t)i * n : nullptr, dbg && dbg->oacc ? dbg->oacc + (size_t)i * D : nullptr);
    if (dbg) {
      if (dbg->p) std::memcpy(dbg->p + (size_t)i * n, prow.data(), n);
      if (dbg->sp) dbg->sp[i] = sp;
    }
  }
  if (dbg) {
    if (dbg->qa) std::memcpy(dbg->qa, P.qa.data(), (size_t)n * D);
    if (dbg->sq) std::memcpy(dbg->sq, P.sq.data(), sizeof(float) * n);
    if (dbg->kq) std::memcpy(dbg->kq, P.kq.data(), (size_t)n * D);
    if (dbg->ks) std::memcpy(dbg->ks, P.ks.data(), sizeof(float) * n);
    if (dbg->kzc) std::memcpy(dbg->kzc, P.kzc.data(), sizeof(float) * n);
    if (dbg->vq) std::memcpy(dbg->vq, P.vq.data(), (size_t)n * D);
    if (dbg->vs) std::memcpy(dbg->vs, P.vs.data(), sizeof(float) * D);
    if (dbg->kmean) std::memcpy(dbg->kmean, P.kmean.data(), sizeof(float) * D);
  }
}

void or_head_logits(const float *w, const float *b, int rows, int H, const float *x, int nx, double *z) {
  // heads.go:62-74: sequential float64 dot product, then + float64(b).
  for (int t = 0; t < nx; t++)
    for (int r = 0; r < rows; r++) {
      double s = 0.0;
      for (int i = 0; i < H; i++) s += (double)w[(size_t)r * H + i] * (double)x[(size_t)t * H + i];
      z[(size_t)t * rows + r] = s + (double)b[r];
    }
}

}  // extern "C"
