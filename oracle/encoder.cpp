// CPU oracle (test infrastructure): the int8 encoder forward of
// internal/modernbert/infer.go:304-430 (run) and its pooling (:261-289),
// assembled from the elementary restatements in oracle.cpp. With threads > 1
// or fast != 0 it is also the CPU baseline bench.py times: the same
// arithmetic, rows sliced over threads as linalg/parallel.go:38-72 does and
// the integer products on AVX-VNNI (cpu_baseline.cpp).
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <mutex>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "oracle.h"
#include "oracle_internal.h"

using namespace orc;

namespace {
// Wall time of the encoder's phases summed over calls (the CPU baseline's
// per-phase split): 0 norms + QKV + RoPE, 1 attention, 2 output projection,
// norm and MLP.
std::mutex g_phase_mu;
double g_phase_s[3] = {0, 0, 0};
struct PhaseClock {
  int phase;
  std::chrono::steady_clock::time_point t0 = std::chrono::steady_clock::now();
  explicit PhaseClock(int p) : phase(p) {}
  ~PhaseClock() {
    const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::lock_guard<std::mutex> lk(g_phase_mu);
    g_phase_s[phase] += s;
  }
};
}  // namespace

struct or_model {
  or_config cfg;
  std::vector<float> emb, emb_norm, final_norm;
  std::vector<std::vector<float>> attn_norm, mlp_norm;
  std::vector<PackedMat> qkv, o, wi, womlp;
  // float32 copies for the path without SetInt8 (or_encode_f32)
  std::vector<std::vector<float>> fqkv, fo, fwi, fwomlp;
};

extern "C" {

or_model *or_model_create(const or_config *cfg, const or_weights *w) {
  auto *m = new or_model();
  m->cfg = *cfg;
  const int H = cfg->hidden, I = cfg->intermediate, L = cfg->layers, V = cfg->vocab;
  m->emb.assign(w->emb, w->emb + (size_t)V * H);
  m->emb_norm.assign(w->emb_norm, w->emb_norm + H);
  m->final_norm.assign(w->final_norm, w->final_norm + H);
  m->attn_norm.resize(L);
  m->mlp_norm.resize(L);
  m->qkv.resize(L);
  m->o.resize(L);
  m->wi.resize(L);
  m->womlp.resize(L);
  for (int l = 0; l < L; l++) {
    if (l > 0) m->attn_norm[l].assign(w->attn_norm[l], w->attn_norm[l] + H);
    m->mlp_norm[l].assign(w->mlp_norm[l], w->mlp_norm[l] + H);
    pack(m->qkv[l], w->wqkv[l], H, 3 * H);
    pack(m->o[l], w->wo[l], H, H);
    pack(m->wi[l], w->wi[l], H, 2 * I);
    pack(m->womlp[l], w->wo_mlp[l], I, H);
  }
  m->fqkv.resize(L), m->fo.resize(L), m->fwi.resize(L), m->fwomlp.resize(L);
  for (int l = 0; l < L; l++) {
    m->fqkv[l].assign(w->wqkv[l], w->wqkv[l] + (size_t)3 * H * H);
    m->fo[l].assign(w->wo[l], w->wo[l] + (size_t)H * H);
    m->fwi[l].assign(w->wi[l], w->wi[l] + (size_t)2 * I * H);
    m->fwomlp[l].assign(w->wo_mlp[l], w->wo_mlp[l] + (size_t)H * I);
  }
  return m;
}

void or_model_destroy(or_model *m) { delete m; }

void or_model_packed(const or_model *m, int l, int which, const int8_t **q, const float **scale, const float **zc,
                     int *k, int *n) {
  const PackedMat *p = which == 0 ? &m->qkv[l] : which == 1 ? &m->o[l] : which == 2 ? &m->wi[l] : &m->womlp[l];
  *q = p->q.data();
  *scale = p->scale.data();
  *zc = p->zc.data();
  *k = p->k;
  *n = p->n;
}

int or_encode(const or_model *m, const int32_t *ids, const int64_t *offs, int nseq, int mode, float *out,
              int threads, int fast, or_dump *dump, int32_t *bad_id) {
  const or_config &cfg = m->cfg;
  const int H = cfg.hidden, I = cfg.intermediate, nh = cfg.heads, D = H / nh, half = D / 2, VL = cfg.V;
  // infer.go:245-247: a consistent batch (offsets from 0, non-decreasing).
  if (nseq < 0 || offs[0] != 0) return 2;
  for (int i = 0; i < nseq; i++)
    if (offs[i + 1] < offs[i]) return 2;
  const int64_t N = offs[nseq];
  // infer.go:307-315: every id in [0, vocab).
  for (int64_t t = 0; t < N; t++)
    if (ids[t] < 0 || ids[t] >= cfg.vocab) {
      if (bad_id) *bad_id = ids[t];
      return 1;
    }
  if (mode == 0) std::memset(out, 0, sizeof(float) * (size_t)nseq * H);
  if (N == 0) return 0;
  const bool use_fast = fast != 0 || threads > 1;
  // The CPU baseline's vector forms (AVX2, V = 8, VNNI attention tiles): the
  // same bits as the scalar loops.
  const bool simd = use_fast && VL == 8 && simd8_ok();
  auto norm = [&](float *o, const float *xr, const float *gamma) {
    if (simd)
      layernorm_row8(o, xr, gamma, H, cfg.norm_eps);
    else
      layernorm_row(o, xr, gamma, H, cfg.norm_eps, VL);
  };
  const int workers = std::max(1, threads);
  std::vector<float> x((size_t)N * H), xn((size_t)N * H), qkv((size_t)N * 3 * H), ctx((size_t)N * H);
  std::vector<int32_t> pos(N);
  int T = 0;
  for (int i = 0; i < nseq; i++) {
    T = std::max<int>(T, (int)(offs[i + 1] - offs[i]));
    for (int64_t t = offs[i]; t < offs[i + 1]; t++) pos[t] = (int32_t)(t - offs[i]);
  }
  for (int64_t r = 0; r < N; r++) std::memcpy(&xn[r * H], &m->emb[(size_t)ids[r] * H], sizeof(float) * H);
  for (int64_t r = 0; r < N; r++) norm(&x[r * H], &xn[r * H], m->emb_norm.data());
  if (dump && dump->emb_ln) std::memcpy(dump->emb_ln, x.data(), sizeof(float) * N * H);

  // infer.go:570-572 sliceRows.
  const int slice = std::min(24, std::max(6, (int)((N / 8 + 3) / 6 * 6)));
  const int npos = std::max(T, 512);
  std::vector<float> rc((size_t)npos * half), rs((size_t)npos * half);
  double theta_cached = -1;

  for (int l = 0; l < cfg.layers; l++) {
    const bool global = l % cfg.global_every == 0;
    const double theta = global ? cfg.global_theta : cfg.local_theta;
    if (theta != theta_cached) {
      rope_table(theta, D, npos, rc.data(), rs.data());
      theta_cached = theta;
    }
    const bool dl = dump && dump->layer == l;
    // Norm, QKV projection, RoPE (infer.go:382-400).
    std::unique_ptr<PhaseClock> clock(new PhaseClock(0));
    parallel_n(workers, (int)N, slice, [&](int lo, int hi) {
      GemmScratch s;
      const float *in = &x[(size_t)lo * H];
      if (l > 0) {
        for (int r = lo; r < hi; r++) norm(&xn[(size_t)r * H], &x[(size_t)r * H], m->attn_norm[l].data());
        in = &xn[(size_t)lo * H];
      }
      matmul_rows(m->qkv[l], in, &qkv[(size_t)lo * 3 * H], hi - lo, false, use_fast, s,
                  dl && dump->xq ? dump->xq + (size_t)lo * H : nullptr, dl && dump->xq_s ? dump->xq_s + lo : nullptr,
                  dl && dump->qkv_acc ? dump->qkv_acc + (size_t)lo * 3 * H : nullptr);
      if (dl && dump->qkv)
        std::memcpy(dump->qkv + (size_t)lo * 3 * H, &qkv[(size_t)lo * 3 * H], sizeof(float) * (hi - lo) * 3 * H);
      for (int r = lo; r < hi; r++) {
        const int t = pos[r];
        float *row = &qkv[(size_t)r * 3 * H];
        for (int h = 0; h < 2 * nh; h++)
          (simd ? rope8 : rope)(row + h * D, &rc[(size_t)t * half], &rs[(size_t)t * half], half);
      }
    });

    // attention8 (infer.go:484-518): prepare per (sequence, head), attend per
    // block of queries.
    const int window = global ? -1 : cfg.local_attention / 2;
    const float scale = (float)(1.0 / std::sqrt((double)D));
    clock.reset(new PhaseClock(1));
    if (simd) {
      // The CPU baseline: prepare per (sequence, head), then the blocks of
      // queries, S and O on VNNI tiles (linalg/attention8.go:298-376).
      std::vector<AttnPrep8> prep8((size_t)nseq * nh);
      parallel_n(workers, nseq * nh, 1, [&](int lo, int hi) {
        for (int task = lo; task < hi; task++) {
          const int bi = task / nh, h = task % nh;
          const int64_t off = offs[bi];
          const int n = (int)(offs[bi + 1] - off);
          if (n == 0) continue;
          const float *rows = &qkv[(size_t)off * 3 * H];
          attn_prepare8(rows + h * D, rows + H + h * D, rows + 2 * H + h * D, 3 * H, n, D, scale, prep8[task]);
        }
      });
      struct Blk8 {
        int task, i0;
      };
      std::vector<Blk8> blocks8;
      for (int bi = 0; bi < nseq; bi++)
        for (int h = 0; h < nh; h++)
          for (int i0 = 0; i0 < offs[bi + 1] - offs[bi]; i0 += kAttnBlock8) blocks8.push_back({bi * nh + h, i0});
      parallel_n(workers, (int)blocks8.size(), 1, [&](int lo, int hi) {
        AttnScratch8 sc;
        for (int b = lo; b < hi; b++) {
          const int bi = blocks8[b].task / nh, h = blocks8[b].task % nh;
          const int64_t off = offs[bi];
          const int n = (int)(offs[bi + 1] - off);
          attend8(prep8[blocks8[b].task], blocks8[b].i0, std::min(n, blocks8[b].i0 + kAttnBlock8), window,
                  &ctx[(size_t)(off + blocks8[b].i0) * H + h * D], H, sc);
        }
      });
    }
    std::vector<AttnPrep> prep(simd ? 0 : (size_t)nseq * nh);
    if (!simd) parallel_n(workers, nseq * nh, 1, [&](int lo, int hi) {
      for (int task = lo; task < hi; task++) {
        const int bi = task / nh, h = task % nh;
        const int64_t off = offs[bi];
        const int n = (int)(offs[bi + 1] - off);
        if (n == 0) continue;
        const float *rows = &qkv[(size_t)off * 3 * H];
        attn_prepare(rows + h * D, rows + H + h * D, rows + 2 * H + h * D, 3 * H, n, D, scale, prep[task]);
      }
    });
    struct Blk {
      int task, i0;
    };
    std::vector<Blk> blocks;
    const int AttnBlock = 48;
    for (int bi = 0; bi < nseq && !simd; bi++)
      for (int h = 0; h < nh; h++)
        for (int i0 = 0; i0 < offs[bi + 1] - offs[bi]; i0 += AttnBlock) blocks.push_back({bi * nh + h, i0});
    parallel_n(workers, (int)blocks.size(), 1, [&](int lo, int hi) {
      std::vector<float> srow(T);
      std::vector<uint8_t> prow(T);
      for (int b = lo; b < hi; b++) {
        const int bi = blocks[b].task / nh, h = blocks[b].task % nh;
        const int64_t off = offs[bi];
        const int n = (int)(offs[bi + 1] - off);
        const AttnPrep &P = prep[blocks[b].task];
        for (int i = blocks[b].i0; i < std::min(n, blocks[b].i0 + AttnBlock); i++)
          attn_row(P, i, window, VL, &ctx[(size_t)(off + i) * H + h * D], srow.data(), prow.data(), nullptr, nullptr,
                   nullptr);
      }
    });
    if (dl && dump->ctx) std::memcpy(dump->ctx, ctx.data(), sizeof(float) * N * H);

    // Output projection, norm, MLP (infer.go:402-425).
    clock.reset(new PhaseClock(2));
    std::vector<float> xa;
    if (dl && dump->x_attn) xa.resize((size_t)N * H);
    parallel_n(workers, (int)N, slice, [&](int lo, int hi) {
      GemmScratch s;
      const int rows = hi - lo;
      matmul_rows(m->o[l], &ctx[(size_t)lo * H], &x[(size_t)lo * H], rows, true, use_fast, s,
                  dl && dump->cq ? dump->cq + (size_t)lo * H : nullptr, dl && dump->cq_s ? dump->cq_s + lo : nullptr,
                  nullptr);
      if (!xa.empty()) std::memcpy(&xa[(size_t)lo * H], &x[(size_t)lo * H], sizeof(float) * rows * H);
      for (int r = lo; r < hi; r++) norm(&xn[(size_t)r * H], &x[(size_t)r * H], m->mlp_norm[l].data());
      std::vector<float> z((size_t)rows * 2 * I), g((size_t)rows * I);
      matmul_rows(m->wi[l], &xn[(size_t)lo * H], z.data(), rows, false, use_fast, s,
                  dl && dump->hq ? dump->hq + (size_t)lo * H : nullptr, dl && dump->hq_s ? dump->hq_s + lo : nullptr,
                  nullptr);
      if (dl && dump->z) std::memcpy(dump->z + (size_t)lo * 2 * I, z.data(), sizeof(float) * rows * 2 * I);
      for (int r = 0; r < rows; r++)
        (simd ? gelu_mul8 : gelu_mul)(&g[(size_t)r * I], &z[(size_t)r * 2 * I], &z[(size_t)r * 2 * I + I], I);
      matmul_rows(m->womlp[l], g.data(), &x[(size_t)lo * H], rows, true, use_fast, s,
                  dl && dump->gq ? dump->gq + (size_t)lo * I : nullptr, dl && dump->gq_s ? dump->gq_s + lo : nullptr,
                  nullptr);
    });
    if (!xa.empty()) std::memcpy(dump->x_attn, xa.data(), sizeof(float) * N * H);
    if (dl && dump->x_mlp) std::memcpy(dump->x_mlp, x.data(), sizeof(float) * N * H);
  }
  // Final norm (infer.go:427) then pooling (infer.go:261-289).
  for (int64_t r = 0; r < N; r++) norm(&xn[r * H], &x[r * H], m->final_norm.data());
  if (mode == 1) {
    std::memcpy(out, xn.data(), sizeof(float) * N * H);
    return 0;
  }
  for (int i = 0; i < nseq; i++) {
    const int64_t n = offs[i + 1] - offs[i];
    if (n == 0) continue;
    if (cfg.cls) {
      std::memcpy(out + (size_t)i * H, &xn[(size_t)offs[i] * H], sizeof(float) * H);
      continue;
    }
    for (int k = 0; k < H; k++) {
      double acc = 0.0;
      for (int64_t t = offs[i]; t < offs[i + 1]; t++) acc += (double)xn[(size_t)t * H + k];
      out[(size_t)i * H + k] = (float)(acc / (double)n);
    }
  }
  return 0;
}

int or_cpu_features(void) { return cpu_features(); }

void or_phase_seconds(double *out, int reset) {
  std::lock_guard<std::mutex> lk(g_phase_mu);
  for (int i = 0; i < 3; i++) {
    out[i] = g_phase_s[i];
    if (reset) g_phase_s[i] = 0;
  }
}

}  // extern "C"


// ---------------------------------------------------------------------------
// The float32 path (the encoder without SetInt8): run (infer.go:304-430) with
// packedMat.mul in float32 (linalg/gemm.go) and attentionInfer's attendBlocks
// (infer.go:437-476, :590-650).
// ---------------------------------------------------------------------------

namespace {

constexpr int kF32Kc = 256;  // linalg/gemm.go:26
constexpr int kQBlock = 64, kKBlock = 128;  // infer.go:537-538

// c[r][o] (+)= x[r] . W[o] as linalg/gemm.go computes it: one FMA chain per
// 256-deep block from zero; without accumulate the first block is stored
// and the next added, with accumulate every block is added to c.
void f32_product(float *c, const float *x, int rows, const float *W, int in, int out, bool accumulate) {
  for (int r = 0; r < rows; r++)
    for (int o = 0; o < out; o++) {
      float total = accumulate ? c[(size_t)r * out + o] : 0.0f;
      for (int pc = 0; pc < in; pc += kF32Kc) {
        const int kb = std::min(kF32Kc, in - pc);
        float acc = 0.0f;
        const float *xr = x + (size_t)r * in + pc, *wr = W + (size_t)o * in + pc;
        for (int q = 0; q < kb; q++) acc = std::fma(xr[q], wr[q], acc);
        total = (!accumulate && pc == 0) ? acc : total + acc;
      }
      c[(size_t)r * out + o] = total;
    }
}

// Go's built-in max on float32 (NaN wins, +0 over -0).
float go_max32(float a, float b) {
  if (a != a || b != b) return NAN;
  if (a == b) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}

float max_of32(const float *x, int n) {
  float m = -INFINITY;
  for (int i = 0; i < n; i++) m = go_max32(m, x[i]);
  return m;
}

// attendBlocks (infer.go:590-650): key blocks of 128 outside, query blocks of
// 64 inside, the softmax maximum and sum kept per row and the output rescaled
// when the maximum grows.
void attend_blocks(float *o, float *q, const float *k, const float *v, int n, int D, int window, float scale, int V) {
  for (int i = 0; i < n * D; i++) q[i] = q[i] * scale;
  std::fill(o, o + (size_t)n * D, 0.0f);
  std::vector<float> mx(n, -INFINITY), sum(n, 0.0f), sc((size_t)kQBlock * kKBlock);
  for (int jb = 0; jb < n; jb += kKBlock) {
    const int je = std::min(n, jb + kKBlock), cols = je - jb;
    int q0 = 0, q1 = n;
    if (window >= 0) q0 = std::max(0, jb - window), q1 = std::min(n, je + window);
    q0 = q0 / kQBlock * kQBlock;
    for (int i0 = q0; i0 < q1; i0 += kQBlock) {
      const int i1 = std::min(n, i0 + kQBlock), rows = i1 - i0;
      f32_product(sc.data(), q + (size_t)i0 * D, rows, k + (size_t)jb * D, D, cols, false);
      for (int r = 0; r < rows; r++) {
        const int i = i0 + r;
        float *row = &sc[(size_t)r * cols];
        int cs = 0, ce = cols;
        if (window >= 0) cs = std::max(0, i - window - jb), ce = std::min(cols, i + window + 1 - jb);
        if (cs >= ce) {
          std::fill(row, row + cols, 0.0f);
          continue;
        }
        const float m = go_max32(mx[i], max_of32(row + cs, ce - cs));
        const float corr = exp32(mx[i] - m);
        if (corr != 1.0f) {
          sum[i] = sum[i] * corr;
          for (int d = 0; d < D; d++) o[(size_t)i * D + d] = o[(size_t)i * D + d] * corr;
        }
        mx[i] = m;
        sum[i] = sum[i] + exp_shift(row + cs, ce - cs, m, V);
        std::fill(row, row + cs, 0.0f);
        std::fill(row + ce, row + cols, 0.0f);
      }
      // o += P V of the block (one chain over the block's keys per output).
      std::vector<float> vt((size_t)D * cols);
      for (int u = 0; u < cols; u++)
        for (int d = 0; d < D; d++) vt[(size_t)d * cols + u] = v[(size_t)(jb + u) * D + d];
      f32_product(o + (size_t)i0 * D, sc.data(), rows, vt.data(), cols, D, true);
    }
  }
  for (int i = 0; i < n; i++) {
    const float inv = 1.0f / sum[i];
    for (int d = 0; d < D; d++) o[(size_t)i * D + d] = o[(size_t)i * D + d] * inv;
  }
}

}  // namespace

extern "C" int or_encode_f32(const or_model *m, const int32_t *ids, const int64_t *offs, int nseq, int mode,
                             float *out, int threads, int32_t *bad_id) {
  const or_config &cfg = m->cfg;
  const int H = cfg.hidden, I = cfg.intermediate, nh = cfg.heads, D = H / nh, half = D / 2, VL = cfg.V;
  if (nseq < 0 || offs[0] != 0) return 2;
  for (int i = 0; i < nseq; i++)
    if (offs[i + 1] < offs[i]) return 2;
  const int64_t N = offs[nseq];
  for (int64_t t = 0; t < N; t++)
    if (ids[t] < 0 || ids[t] >= cfg.vocab) {
      if (bad_id) *bad_id = ids[t];
      return 1;
    }
  if (mode == 0) std::memset(out, 0, sizeof(float) * (size_t)nseq * H);
  if (N == 0) return 0;
  const int workers = std::max(1, threads);
  std::vector<float> x((size_t)N * H), xn((size_t)N * H), qkv((size_t)N * 3 * H), ctx((size_t)N * H);
  std::vector<int32_t> pos(N);
  int T = 0;
  for (int i = 0; i < nseq; i++) {
    T = std::max<int>(T, (int)(offs[i + 1] - offs[i]));
    for (int64_t t = offs[i]; t < offs[i + 1]; t++) pos[t] = (int32_t)(t - offs[i]);
  }
  for (int64_t r = 0; r < N; r++) std::memcpy(&xn[r * H], &m->emb[(size_t)ids[r] * H], sizeof(float) * H);
  for (int64_t r = 0; r < N; r++) layernorm_row(&x[r * H], &xn[r * H], m->emb_norm.data(), H, cfg.norm_eps, VL);
  const int npos = std::max(T, 512);
  std::vector<float> rc((size_t)npos * half), rs((size_t)npos * half);
  double theta_cached = -1;
  for (int l = 0; l < cfg.layers; l++) {
    const bool global = l % cfg.global_every == 0;
    const double theta = global ? cfg.global_theta : cfg.local_theta;
    if (theta != theta_cached) {
      rope_table(theta, D, npos, rc.data(), rs.data());
      theta_cached = theta;
    }
    parallel_n(workers, (int)N, 24, [&](int lo, int hi) {
      const float *in = &x[(size_t)lo * H];
      if (l > 0) {
        for (int r = lo; r < hi; r++)
          layernorm_row(&xn[(size_t)r * H], &x[(size_t)r * H], m->attn_norm[l].data(), H, cfg.norm_eps, VL);
        in = &xn[(size_t)lo * H];
      }
      f32_product(&qkv[(size_t)lo * 3 * H], in, hi - lo, m->fqkv[l].data(), H, 3 * H, false);
      for (int r = lo; r < hi; r++) {
        const int t = pos[r];
        float *row = &qkv[(size_t)r * 3 * H];
        for (int h = 0; h < 2 * nh; h++) rope(row + h * D, &rc[(size_t)t * half], &rs[(size_t)t * half], half);
      }
    });
    const int window = global ? -1 : cfg.local_attention / 2;
    const float scale = (float)(1.0 / std::sqrt((double)D));
    parallel_n(workers, nseq * nh, 1, [&](int lo, int hi) {
      std::vector<float> q, k, v, o;
      for (int task = lo; task < hi; task++) {
        const int bi = task / nh, h = task % nh;
        const int64_t off = offs[bi];
        const int n = (int)(offs[bi + 1] - off);
        if (n == 0) continue;
        q.resize((size_t)n * D), k.resize((size_t)n * D), v.resize((size_t)n * D), o.resize((size_t)n * D);
        for (int t = 0; t < n; t++) {
          const float *row = &qkv[(size_t)(off + t) * 3 * H];
          std::memcpy(&q[(size_t)t * D], row + h * D, D * 4);
          std::memcpy(&k[(size_t)t * D], row + H + h * D, D * 4);
          std::memcpy(&v[(size_t)t * D], row + 2 * H + h * D, D * 4);
        }
        attend_blocks(o.data(), q.data(), k.data(), v.data(), n, D, window, scale, VL);
        for (int t = 0; t < n; t++) std::memcpy(&ctx[(size_t)(off + t) * H + h * D], &o[(size_t)t * D], D * 4);
      }
    });
    parallel_n(workers, (int)N, 24, [&](int lo, int hi) {
      f32_product(&x[(size_t)lo * H], &ctx[(size_t)lo * H], hi - lo, m->fo[l].data(), H, H, true);
      for (int r = lo; r < hi; r++)
        layernorm_row(&xn[(size_t)r * H], &x[(size_t)r * H], m->mlp_norm[l].data(), H, cfg.norm_eps, VL);
      std::vector<float> z((size_t)(hi - lo) * 2 * I), g((size_t)(hi - lo) * I);
      f32_product(z.data(), &xn[(size_t)lo * H], hi - lo, m->fwi[l].data(), H, 2 * I, false);
      for (int r = 0; r < hi - lo; r++) gelu_mul(&g[(size_t)r * I], &z[(size_t)r * 2 * I], &z[(size_t)r * 2 * I + I], I);
      f32_product(&x[(size_t)lo * H], g.data(), hi - lo, m->fwomlp[l].data(), I, H, true);
    });
  }
  for (int64_t r = 0; r < N; r++) layernorm_row(&xn[r * H], &x[r * H], m->final_norm.data(), H, cfg.norm_eps, VL);
  if (mode == 1) {
    std::memcpy(out, xn.data(), sizeof(float) * N * H);
    return 0;
  }
  for (int i = 0; i < nseq; i++) {
    const int64_t n = offs[i + 1] - offs[i];
    if (n == 0) continue;
    if (cfg.cls) {
      std::memcpy(out + (size_t)i * H, &xn[(size_t)offs[i] * H], sizeof(float) * H);
      continue;
    }
    for (int k = 0; k < H; k++) {
      double acc = 0;
      for (int64_t t = offs[i]; t < offs[i + 1]; t++) acc += (double)xn[(size_t)t * H + k];
      out[(size_t)i * H + k] = (float)(acc / (double)n);
    }
  }
  return 0;
}
