// Shared pieces of the oracle's encoders (test infrastructure): weight
// packing for the int8 products and one MatMul8N call on a slice of rows.
#include <cstring>

#include "oracle.h"
#include "oracle_internal.h"

namespace orc {

void pack(PackedMat &p, const float *w, int k, int n) {
  p.k = k;
  p.n = n;
  p.q.resize((size_t)n * k);
  p.scale.resize(n);
  p.zc.resize(n);
  p.colsum.resize(n);
  pack_b8(w, k, n, true, p.q.data(), p.scale.data(), p.colsum.data(), p.zc.data());
  pack_panels(p.q.data(), n, k, p.panels);
}

void matmul_rows(const PackedMat &W, const float *a, float *c, int rows, bool accumulate, bool fast,
                        GemmScratch &s, uint8_t *aq_dump, float *sa_dump, int32_t *acc_dump) {
  const int k = W.k, n = W.n;
  const int kp = (k + 3) / 4 * 4;
  const int rp = (rows + 5) / 6 * 6;
  s.aq.assign((size_t)rp * kp, 128);
  s.sa.assign(rp, 0.0f);
  s.acc.resize((size_t)rows * n);
  // The fast path (the CPU baseline) also quantizes and dequantizes in AVX2:
  // the same bits.
  const bool simd = fast && simd8_ok();
  for (int i = 0; i < rows; i++)
    (simd ? quantize_a_row8 : quantize_a_row)(a + (size_t)i * k, k, s.aq.data() + (size_t)i * kp, &s.sa[i]);
  if (fast)
    gemm_u8s8_fast(s.aq.data(), W.panels.data(), rp, n, kp, 0, rows, s.acc.data());
  else
    gemm_u8s8(s.aq.data(), kp, W.q.data(), k, rows, n, k, s.acc.data());
  if (simd)
    for (int i = 0; i < rows; i++)
      dequant_row8(s.acc.data() + (size_t)i * n, n, s.sa[i], W.scale.data(), W.zc.data(), c + (size_t)i * n,
                   accumulate);
  else
    dequant(s.acc.data(), rows, n, s.sa.data(), W.scale.data(), W.zc.data(), c, accumulate);
  if (aq_dump)
    for (int i = 0; i < rows; i++) std::memcpy(aq_dump + (size_t)i * k, s.aq.data() + (size_t)i * kp, k);
  if (sa_dump) std::memcpy(sa_dump, s.sa.data(), sizeof(float) * rows);
  if (acc_dump) std::memcpy(acc_dump, s.acc.data(), sizeof(int32_t) * rows * n);
}

}  // namespace orc
