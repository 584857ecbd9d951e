// Internal declarations shared by the oracle's translation units (test
// infrastructure; see oracle.h).
#pragma once
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <thread>
#include <vector>

namespace orc {

float round_half_even(float v);
float abs32(float v);
float exp32(float x);
float exp_body(float v);
float exp_shift(float *x, int n, float m, int V);
float erf32(float x);
float gelu_mul_fma(float x, float gate);
float gelu_mul_scalar(float x, float gate);
void gelu_mul(float *o, const float *a, const float *b, int n);
void layernorm_row(float *o, const float *x, const float *gamma, int n, double eps, int V);
void rope(float *x, const float *c, const float *s, int half);
void rope_table(double theta, int D, int npos, float *cs, float *sn);
float quant_row(int8_t *dst, const float *x, const float *mean, int n, bool flip, int32_t *sum);
void pack_b8(const float *b, int k, int n, bool transB, int8_t *q, float *scale, int32_t *colsum, float *zc);
void quantize_a_row(const float *x, int k, uint8_t *q, float *sa);
void gemm_u8s8(const uint8_t *A, int lda, const int8_t *B, int ldb, int M, int N, int K, int32_t *acc);
float dequant1(int32_t acc, float zc, float sb, float sa);
void dequant(const int32_t *acc, int M, int N, const float *sa, const float *sb, const float *zc, float *C,
             bool accumulate);

struct AttnPrep {
  int n = 0, D = 0;
  std::vector<uint8_t> qa;
  std::vector<float> sq;
  std::vector<int8_t> kq;
  std::vector<float> ks, kzc;
  std::vector<int8_t> vq;
  std::vector<float> vs, kmean;
};
void attn_prepare(const float *q, const float *k, const float *v, int ld, int n, int D, float scale, AttnPrep &P);
void attn_row(const AttnPrep &P, int i, int window, int V, float *o, float *s_row, uint8_t *p_row, float *sp_out,
              int32_t *sacc_row, int32_t *oacc_row);

// CPU baseline GEMM (cpu_baseline.cpp): same integers as gemm_u8s8, VNNI when
// the host has it; rows [r0, r1) of acc.
void gemm_u8s8_fast(const uint8_t *A, const int8_t *Bpanels, int M, int N, int K, int r0, int r1, int32_t *acc);
// Panels of 16 output channels, 4 depths per 32-bit word (linalg/int8.go:25-34).
void pack_panels(const int8_t *q, int N, int K, std::vector<int8_t> &out);
int cpu_features();

struct PackedMat {
  int k = 0, n = 0;
  std::vector<int8_t> q;       // [n][k]
  std::vector<int8_t> panels;  // [n/16][k/4][16][4] for the fast GEMM
  std::vector<float> scale, zc;
  std::vector<int32_t> colsum;
};


void pack(PackedMat &p, const float *w, int k, int n);

// linalg/parallel.go:38-72 ParallelN: about four slices per worker, each a
// multiple of grain, taken with an atomic counter.
template <class F>
inline void parallel_n(int workers, int n, int grain, F fn) {
  if (n <= 0) return;
  grain = std::max(1, grain);
  if (workers <= 1 || n <= grain) {
    fn(0, n);
    return;
  }
  int step = ((n + 4 * workers - 1) / (4 * workers) + grain - 1) / grain * grain;
  workers = std::min(workers, (n + step - 1) / step);
  std::atomic<int> next(0);
  auto run = [&]() {
    for (;;) {
      int lo = next.fetch_add(1) * step;
      if (lo >= n) return;
      fn(lo, std::min(lo + step, n));
    }
  };
  std::vector<std::thread> ts;
  for (int w = 1; w < workers; w++) ts.emplace_back(run);
  run();
  for (auto &t : ts) t.join();
}

// One MatMul8N call on rows [lo, hi): c (+)= dequant(quant(a) . W^T).
struct GemmScratch {
  std::vector<uint8_t> aq;
  std::vector<float> sa;
  std::vector<int32_t> acc;
};

void matmul_rows(const PackedMat &W, const float *a, float *c, int rows, bool accumulate, bool fast,
                 GemmScratch &s, uint8_t *aq_dump, float *sa_dump, int32_t *acc_dump);

// Vector forms of the CPU baseline (cpu_simd.cpp): AVX2 with V = 8 lanes and
// VNNI attention tiles, bit-equal to the scalar functions above.
bool simd8_ok();  // AVX2 + FMA + a VNNI form on this host
void layernorm_row8(float *o, const float *x, const float *gamma, int n, double eps);
float quant_row8(int8_t *dst, const float *x, const float *mean, int n, bool flip, int32_t *sum);
void quantize_a_row8(const float *x, int k, uint8_t *q, float *sa);
void dequant_row8(const int32_t *acc, int N, float sa, const float *sb, const float *zc, float *c, bool accumulate);
float exp_shift8(float *x, int n, float m);
void gelu_mul8(float *o, const float *a, const float *b, int n);
void rope8(float *x, const float *c, const float *s, int half);

constexpr int kAttnBlock8 = 48;  // queries scored at a time (linalg/attention8.go:26, 8 x 6)
struct AttnPrep8 {
  AttnPrep base;
  int n16 = 0;                // keys padded to whole 16-key panels
  std::vector<uint8_t> qpad;  // qa plus 6 padding rows
  std::vector<int8_t> kp, vp;  // K [n16/16][D/4][16][4]; V [D/16][n16/4][16][4]
  std::vector<float> ks16, kzc16, sq6;  // key scales and sums padded to n16, query scales to n + 6
};
struct AttnScratch8 {
  std::vector<float> s;
  std::vector<uint8_t> p;
  std::vector<float> sp;
};
void attn_prepare8(const float *q, const float *k, const float *v, int ld, int n, int D, float scale, AttnPrep8 &P);
void attend8(const AttnPrep8 &P, int i0, int i1, int window, float *o, int ldo, AttnScratch8 &sc);


}  // namespace orc
