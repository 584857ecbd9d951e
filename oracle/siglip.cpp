// CPU oracle (test infrastructure): the int8 SigLIP vision tower of
// internal/siglip (encoder.go, vision.go) with its float32 pieces — the
// patch embedding, the attention, the pooling head — in the arithmetic of
// linalg/gemm.go (one FMA chain per 256-deep block of the product, blocks
// added in order), linalg/vec_simd.go (LayerNormRow, ExpShift, GeluTanh with
// V float32 lanes) and linalg/int8.go (MatMul8N, MatMul8Outliers). Scalar
// loops; images may be spread over threads, and fast != 0 takes the VNNI
// integer products of cpu_baseline.cpp (same integers).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "oracle.h"
#include "oracle_internal.h"

using namespace orc;

namespace {

constexpr int kKc = 256;                // depth of a k block, linalg/gemm.go:26
constexpr int kMaxOutliers = 32;        // linalg/int8.go:276
constexpr float kOutlierRatio = 6.0f;   // internal/siglip/encoder.go:165

float bits_float(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// linalg/gemm.go:65-240 for one output: the micro-kernel's FMA chain over
// each 256-deep block from zero (kernel_amd64.s: VXORPS then VFMADD231PS in
// depth order), the first block stored, the next ones added.
float dot_chain(const float *x, const float *w, int k) {
  float total = 0.0f;
  for (int pc = 0; pc < k; pc += kKc) {
    const int kb = std::min(kKc, k - pc);
    float acc = 0.0f;
    for (int q = 0; q < kb; q++) acc = std::fma(x[pc + q], w[pc + q], acc);
    total = pc == 0 ? acc : total + acc;
  }
  return total;
}

// The vector body of linalg.GeluTanh (vec_simd.go:166-197), one lane.
float gelu_tanh_vec(float x) {
  const float k = -1.5957691216057308f;  // -2*sqrt(2/pi) rounded once, as Go's constant
  float v = x * x;
  v = std::fma(v, 0.044715f, 1.0f);
  v = v * x;
  v = v * k;
  v = std::min(std::max(v, -87.3f), 88.7f);
  const float n = std::fma(v, 1.44269504088896341f, 12582912.0f) - 12582912.0f;
  float r = std::fma(n, -0.693359375f, v);
  r = std::fma(n, 2.12194440e-4f, r);
  float p = std::fma(r, 1.9875691500e-4f, 1.3981999507e-3f);
  p = std::fma(r, p, 8.3334519073e-3f);
  p = std::fma(r, p, 4.1665795894e-2f);
  p = std::fma(r, p, 1.6666665459e-1f);
  p = std::fma(r, p, 5.0000001201e-1f);
  const float y = std::fma(p * r, r, r) + 1.0f;
  const int32_t ni = (int32_t)std::nearbyint(n);
  const float pw = bits_float((uint32_t)(ni + 127) << 23);
  return x / (1.0f + y * pw);
}

// geluTanhScalar (linalg/fastmath.go:28-32): separate roundings.
float gelu_tanh_scalar(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return x / (1.0f + exp32(-2.0f * u));
}

// MaxOf (vec_simd.go:332-345): the maximum, -Inf for none.
float max_of(const float *x, int n) {
  float m = -INFINITY;
  for (int i = 0; i < n; i++) m = std::max(m, x[i]);
  return m;
}

// softmax (internal/siglip/encoder.go:246-251): Scale, ExpShift from the
// maximum, Scale by 1/sum.
void softmax_scaled(float *s, int n, float scale, int V) {
  for (int i = 0; i < n; i++) s[i] = s[i] * scale;
  const float sum = exp_shift(s, n, max_of(s, n), V);
  const float inv = 1.0f / sum;
  for (int i = 0; i < n; i++) s[i] = s[i] * inv;
}

void layer_norm_beta(float *o, const float *x, const float *g, const float *b, int H, double eps, int V) {
  layernorm_row(o, x, g, H, eps, V);
  for (int i = 0; i < H; i++) o[i] = o[i] + b[i];
}

// MatMul8Outliers (linalg/int8.go:281-349): the channels of a whose maximum
// magnitude exceeds ratio times the mean of the channel maxima (32 at
// most: the largest, in the order a partial selection sort leaves them) go
// through float32 with the dequantized weight rows; the rest through int8.
void matmul8_outliers(float *c, const float *a, int m, const PackedMat &W, float ratio, bool fast, GemmScratch &gs,
                      int32_t *out_dump, int32_t *nout_dump, uint8_t *aq_dump, float *sa_dump) {
  const int k = W.k, n = W.n;
  std::vector<float> colmax(k, 0.0f);
  for (int i = 0; i < m; i++)
    for (int j = 0; j < k; j++) colmax[j] = std::max(colmax[j], std::fabs(a[(size_t)i * k + j]));
  float mean = 0.0f;
  for (int j = 0; j < k; j++) mean += colmax[j];
  mean /= (float)k;
  std::vector<int> out;
  for (int j = 0; j < k; j++)
    if (colmax[j] > ratio * mean) out.push_back(j);
  if (out.size() > (size_t)kMaxOutliers) {
    for (int i = 0; i < kMaxOutliers; i++) {
      int best = i;
      for (int x = i + 1; x < (int)out.size(); x++)
        if (colmax[out[x]] > colmax[out[best]]) best = x;
      std::swap(out[i], out[best]);
    }
    out.resize(kMaxOutliers);
  }
  if (nout_dump) *nout_dump = (int32_t)out.size();
  if (out_dump)
    for (size_t i = 0; i < out.size(); i++) out_dump[i] = out[i];
  if (out.empty()) {
    matmul_rows(W, a, c, m, false, fast, gs, aq_dump, sa_dump, nullptr);
    return;
  }
  std::vector<float> rest(a, a + (size_t)m * k);
  for (int i = 0; i < m; i++)
    for (int j : out) rest[(size_t)i * k + j] = 0.0f;
  matmul_rows(W, rest.data(), c, m, false, fast, gs, aq_dump, sa_dump, nullptr);
  std::vector<float> w(n);
  for (int j : out) {
    for (int col = 0; col < n; col++) w[col] = (float)W.q[(size_t)col * k + j] * W.scale[col];
    for (int i = 0; i < m; i++) {
      const float x = a[(size_t)i * k + j];
      float *ci = c + (size_t)i * n;
      for (int col = 0; col < n; col++) ci[col] = ci[col] + x * w[col];
    }
  }
}

void linear_f32(float *dst, const float *x, int rows, const std::vector<float> &W, const std::vector<float> &b, int in,
                int out) {
  for (int r = 0; r < rows; r++)
    for (int o = 0; o < out; o++) {
      float v = dot_chain(x + (size_t)r * in, W.data() + (size_t)o * in, in);
      if (!b.empty()) v = v + b[o];
      dst[(size_t)r * out + o] = v;
    }
}

void gelu_tanh(float *o, const float *a, int n, int V) {
  const int nv = n - n % V;
  for (int i = 0; i < nv; i++) o[i] = gelu_tanh_vec(a[i]);
  for (int i = nv; i < n; i++) o[i] = gelu_tanh_scalar(a[i]);
}

}  // namespace

struct SigLayer {
  std::vector<float> ln1g, ln1b, ln2g, ln2b, bqkv, bo, b1, b2;
  PackedMat qkv, o, fc1, fc2;
};

struct or_siglip {
  or_siglip_config cfg;
  std::vector<float> patch_w, patch_b, pos, post_g, post_b;
  std::vector<SigLayer> layers;
  std::vector<float> probe_q, hk_w, hk_b, hv_w, hv_b, hout_w, hout_b, hln_g, hln_b, hfc1_w, hfc1_b, hfc2_w, hfc2_b;
};

namespace {

std::vector<float> vec(const float *p, size_t n) { return std::vector<float>(p, p + n); }

// Vision.forward for one image (internal/siglip/vision.go:101-141).
void forward_image(const or_siglip *m, const float *pixels, int layer, float *patches, float *pooled, bool fast,
                   or_siglip_dump *dump, int img) {
  const or_siglip_config &c = m->cfg;
  const int H = c.hidden, M = c.mlp, S = c.image_size, P = c.patch_size, g = S / P, T = g * g, V = c.V;
  const int d = H / c.heads, K0 = 3 * P * P;
  // patchify (vision.go:145-160): a row per patch in raster order, (channel, y, x).
  std::vector<float> rows((size_t)T * K0);
  size_t i = 0;
  for (int py = 0; py < g; py++)
    for (int px = 0; px < g; px++)
      for (int ch = 0; ch < 3; ch++)
        for (int y = 0; y < P; y++) {
          std::memcpy(&rows[i], pixels + (size_t)ch * S * S + (size_t)(py * P + y) * S + px * P, P * sizeof(float));
          i += P;
        }
  std::vector<float> x((size_t)T * H), h((size_t)T * H), qkv((size_t)T * 3 * H), attn((size_t)T * H),
      tmp((size_t)T * H), mlp((size_t)T * M);
  linear_f32(x.data(), rows.data(), T, m->patch_w, m->patch_b, K0, H);
  for (size_t e = 0; e < x.size(); e++) x[e] = x[e] + m->pos[e];
  const size_t ro = (size_t)img * T;  // first dump row of this image
  if (dump && dump->x_embed) std::memcpy(dump->x_embed + ro * H, x.data(), x.size() * 4);
  const int n = (layer > 0 && !pooled) ? layer : c.layers;
  GemmScratch gs;
  const float scale = (float)(1 / std::sqrt((double)d));
  std::vector<float> q((size_t)T * d), k((size_t)T * d), v((size_t)T * d), s((size_t)T * T), o((size_t)T * d);
  for (int l = 0; l < n; l++) {
    const SigLayer &L = m->layers[l];
    const bool dl = dump && dump->layer == l;
    for (int t = 0; t < T; t++)
      layer_norm_beta(&h[(size_t)t * H], &x[(size_t)t * H], L.ln1g.data(), L.ln1b.data(), H, c.eps, V);
    matmul_rows(L.qkv, h.data(), qkv.data(), T, false, fast, gs, dl && dump->h1q ? dump->h1q + ro * H : nullptr,
                dl && dump->h1q_s ? dump->h1q_s + ro : nullptr, nullptr);
    for (int t = 0; t < T; t++)
      for (int j = 0; j < 3 * H; j++) qkv[(size_t)t * 3 * H + j] = qkv[(size_t)t * 3 * H + j] + L.bqkv[j];
    if (dl && dump->qkv) std::memcpy(dump->qkv + ro * 3 * H, qkv.data(), qkv.size() * 4);
    // attention (encoder.go:219-243), head by head.
    for (int hh = 0; hh < c.heads; hh++) {
      for (int t = 0; t < T; t++) {
        const float *row = &qkv[(size_t)t * 3 * H];
        std::memcpy(&q[(size_t)t * d], row + hh * d, d * 4);
        std::memcpy(&k[(size_t)t * d], row + H + hh * d, d * 4);
        std::memcpy(&v[(size_t)t * d], row + 2 * H + hh * d, d * 4);
      }
      for (int t = 0; t < T; t++)
        for (int u = 0; u < T; u++) s[(size_t)t * T + u] = dot_chain(&q[(size_t)t * d], &k[(size_t)u * d], d);
      for (int t = 0; t < T; t++) softmax_scaled(&s[(size_t)t * T], T, scale, V);
      std::vector<float> col(T);
      for (int t = 0; t < T; t++)
        for (int j = 0; j < d; j++) {
          for (int u = 0; u < T; u++) col[u] = v[(size_t)u * d + j];
          o[(size_t)t * d + j] = dot_chain(&s[(size_t)t * T], col.data(), T);
        }
      for (int t = 0; t < T; t++) std::memcpy(&attn[(size_t)t * H + hh * d], &o[(size_t)t * d], d * 4);
    }
    if (dl && dump->attn) std::memcpy(dump->attn + ro * H, attn.data(), attn.size() * 4);
    matmul_rows(L.o, attn.data(), tmp.data(), T, false, fast, gs, nullptr, nullptr, nullptr);
    for (int t = 0; t < T; t++)
      for (int j = 0; j < H; j++) {
        const size_t e = (size_t)t * H + j;
        x[e] = x[e] + (tmp[e] + L.bo[j]);
      }
    if (dl && dump->x_attn) std::memcpy(dump->x_attn + ro * H, x.data(), x.size() * 4);
    for (int t = 0; t < T; t++)
      layer_norm_beta(&h[(size_t)t * H], &x[(size_t)t * H], L.ln2g.data(), L.ln2b.data(), H, c.eps, V);
    matmul_rows(L.fc1, h.data(), mlp.data(), T, false, fast, gs, dl && dump->h2q ? dump->h2q + ro * H : nullptr,
                dl && dump->h2q_s ? dump->h2q_s + ro : nullptr, nullptr);
    for (int t = 0; t < T; t++)
      for (int j = 0; j < M; j++) mlp[(size_t)t * M + j] = mlp[(size_t)t * M + j] + L.b1[j];
    gelu_tanh(mlp.data(), mlp.data(), T * M, V);
    if (dl && dump->mlp) std::memcpy(dump->mlp + ro * M, mlp.data(), mlp.size() * 4);
    matmul8_outliers(tmp.data(), mlp.data(), T, L.fc2, kOutlierRatio, fast, gs,
                     dl && dump->outliers ? dump->outliers + (size_t)img * kMaxOutliers : nullptr,
                     dl && dump->noutliers ? dump->noutliers + img : nullptr,
                     dl && dump->mq ? dump->mq + ro * M : nullptr, dl && dump->mq_s ? dump->mq_s + ro : nullptr);
    for (int t = 0; t < T; t++)
      for (int j = 0; j < H; j++) {
        const size_t e = (size_t)t * H + j;
        x[e] = x[e] + (tmp[e] + L.b2[j]);
      }
    if (dl && dump->x_mlp) std::memcpy(dump->x_mlp + ro * H, x.data(), x.size() * 4);
    if (l + 1 == layer && patches) std::memcpy(patches, x.data(), x.size() * 4);
  }
  if (n < c.layers) return;
  for (int t = 0; t < T; t++)
    layer_norm_beta(&x[(size_t)t * H], &x[(size_t)t * H], m->post_g.data(), m->post_b.data(), H, c.eps, V);
  if (layer == 0 && patches) std::memcpy(patches, x.data(), x.size() * 4);
  if (!pooled) return;
  // Attention pooling (vision.go:164-194): the probe's query attends to the
  // patches; float32 throughout.
  std::vector<float> kk((size_t)T * H), vv((size_t)T * H), att(H, 0.0f), sc(T);
  linear_f32(kk.data(), x.data(), T, m->hk_w, m->hk_b, H, H);
  linear_f32(vv.data(), x.data(), T, m->hv_w, m->hv_b, H, H);
  for (int hh = 0; hh < c.heads; hh++) {
    const float *qh = &m->probe_q[(size_t)hh * d];
    for (int t = 0; t < T; t++) {
      float dot = 0.0f;
      const float *kt = &kk[(size_t)t * H + hh * d];
      for (int j = 0; j < d; j++) dot = dot + qh[j] * kt[j];
      sc[t] = dot;
    }
    softmax_scaled(sc.data(), T, scale, V);
    float *oh = &att[(size_t)hh * d];
    for (int t = 0; t < T; t++) {
      const float *vt = &vv[(size_t)t * H + hh * d];
      for (int j = 0; j < d; j++) oh[j] = oh[j] + sc[t] * vt[j];
    }
  }
  std::vector<float> out(H), nrm(H), mm(M);
  linear_f32(out.data(), att.data(), 1, m->hout_w, m->hout_b, H, H);
  layer_norm_beta(nrm.data(), out.data(), m->hln_g.data(), m->hln_b.data(), H, c.eps, V);
  linear_f32(mm.data(), nrm.data(), 1, m->hfc1_w, m->hfc1_b, H, M);
  gelu_tanh(mm.data(), mm.data(), M, V);
  linear_f32(nrm.data(), mm.data(), 1, m->hfc2_w, m->hfc2_b, M, H);
  for (int j = 0; j < H; j++) pooled[j] = out[j] + nrm[j];
}

}  // namespace

extern "C" {

or_siglip *or_siglip_create(const or_siglip_config *cfg, const or_siglip_weights *w) {
  auto *m = new or_siglip();
  m->cfg = *cfg;
  const int H = cfg->hidden, M = cfg->mlp, L = cfg->layers, P = cfg->patch_size, g = cfg->image_size / P;
  const int T = g * g;
  m->patch_w = vec(w->patch_w, (size_t)H * 3 * P * P);
  m->patch_b = vec(w->patch_b, H);
  m->pos = vec(w->pos, (size_t)T * H);
  m->post_g = vec(w->post_g, H);
  m->post_b = vec(w->post_b, H);
  m->layers.resize(L);
  for (int l = 0; l < L; l++) {
    SigLayer &y = m->layers[l];
    y.ln1g = vec(w->ln1_g[l], H), y.ln1b = vec(w->ln1_b[l], H);
    y.ln2g = vec(w->ln2_g[l], H), y.ln2b = vec(w->ln2_b[l], H);
    y.bqkv = vec(w->bqkv[l], 3 * H), y.bo = vec(w->bo[l], H), y.b1 = vec(w->b1[l], M), y.b2 = vec(w->b2[l], H);
    pack(y.qkv, w->wqkv[l], H, 3 * H);
    pack(y.o, w->wo[l], H, H);
    pack(y.fc1, w->w1[l], H, M);
    pack(y.fc2, w->w2[l], M, H);
  }
  // The probe's query, once (vision.go:62-66).
  const std::vector<float> qw = vec(w->in_w, (size_t)H * H), qb = vec(w->in_b, H);
  m->probe_q.resize(H);
  linear_f32(m->probe_q.data(), w->probe, 1, qw, qb, H, H);
  m->hk_w = vec(w->in_w + (size_t)H * H, (size_t)H * H), m->hk_b = vec(w->in_b + H, H);
  m->hv_w = vec(w->in_w + (size_t)2 * H * H, (size_t)H * H), m->hv_b = vec(w->in_b + 2 * H, H);
  m->hout_w = vec(w->hout_w, (size_t)H * H), m->hout_b = vec(w->hout_b, H);
  m->hln_g = vec(w->hln_g, H), m->hln_b = vec(w->hln_b, H);
  m->hfc1_w = vec(w->hfc1_w, (size_t)M * H), m->hfc1_b = vec(w->hfc1_b, M);
  m->hfc2_w = vec(w->hfc2_w, (size_t)H * M), m->hfc2_b = vec(w->hfc2_b, H);
  return m;
}

void or_siglip_destroy(or_siglip *m) { delete m; }

int or_siglip_forward(const or_siglip *m, const float *pixels, int n, int layer, float *patches, float *pooled,
                      int threads, int fast, or_siglip_dump *dump) {
  const or_siglip_config &c = m->cfg;
  if (layer < 0 || layer > c.layers) return 1;
  const int S = c.image_size, g = S / c.patch_size, T = g * g, H = c.hidden;
  parallel_n(threads, n, 1, [&](int lo, int hi) {
    for (int i = lo; i < hi; i++)
      forward_image(m, pixels + (size_t)i * 3 * S * S, layer, patches ? patches + (size_t)i * T * H : nullptr,
                    pooled ? pooled + (size_t)i * H : nullptr, fast != 0, dump, i);
  });
  return 0;
}

void or_linear_f32(float *dst, const float *x, int rows, const float *W, const float *b, int in, int out) {
  linear_f32(dst, x, rows, vec(W, (size_t)in * out), b ? vec(b, out) : std::vector<float>(), in, out);
}

void or_gelu_tanh(float *o, const float *a, int n, int V) { gelu_tanh(o, a, n, V); }

void or_siglip_softmax(float *s, int n, float scale, int V) { softmax_scaled(s, n, scale, V); }

void or_matmul8_outliers(float *c, const float *a, int m, const int8_t *q, const float *scale, const float *zc, int k,
                         int n, float ratio, int32_t *out, int32_t *nout) {
  PackedMat W;
  W.k = k, W.n = n;
  W.q.assign(q, q + (size_t)n * k);
  W.scale.assign(scale, scale + n);
  W.zc.assign(zc, zc + n);
  GemmScratch gs;
  matmul8_outliers(c, a, m, W, ratio, false, gs, out, nout, nullptr, nullptr);
}

}  // extern "C"
