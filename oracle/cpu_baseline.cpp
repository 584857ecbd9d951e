// CPU baseline (test/bench infrastructure): the integer products of the
// oracle's encoder on the host's VNNI units, in the reference's own tile shape
// (6 rows x 16 output channels, 4 depths per 32-bit word,
// linalg/kernel_vnni_amd64.s:13-79 and linalg/int8.go:25-34). The integers are
// exact, so the results equal the scalar oracle's bit for bit; tests check it.
#include <immintrin.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "oracle_internal.h"

namespace orc {

int cpu_features() {
  int f = 0;
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avxvnni")) f |= 1;
  if (__builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512vl")) f |= 2;
  return f;
}

void pack_panels(const int8_t *q, int N, int K, std::vector<int8_t> &out) {
  const int kq = (K + 3) / 4, panels = (N + 15) / 16;
  out.assign((size_t)panels * kq * 64, 0);
  for (int j = 0; j < N; j++)
    for (int d = 0; d < K; d++) out[(size_t)(j / 16) * kq * 64 + (d / 4) * 64 + (j % 16) * 4 + d % 4] = q[(size_t)j * K + d];
}

// 6x16 tile: acc[r][c] = sum_q A[r][4q..4q+3] . B[q][c][0..3]. DPBUSD names the
// VEX (AVX-VNNI) or EVEX (AVX512-VNNI, 256-bit) form of the same instruction.
#define ORC_GEMM_BODY(DPBUSD)                                                                         \
  const int kq = K / 4;                                                                               \
  for (int i0 = r0; i0 < r1; i0 += 6)                                                                 \
    for (int p = 0; p < (N + 15) / 16; p++) {                                                         \
      const uint8_t *a = A + (size_t)i0 * K;                                                          \
      const int8_t *bp = Bp + (size_t)p * kq * 64;                                                    \
      __m256i c[6][2];                                                                                \
      _Pragma("GCC unroll 6") for (int r = 0; r < 6; r++) c[r][0] = c[r][1] = _mm256_setzero_si256();  \
      for (int q = 0; q < kq; q++) {                                                                  \
        __m256i b0 = _mm256_loadu_si256((const __m256i *)(bp + q * 64));                              \
        __m256i b1 = _mm256_loadu_si256((const __m256i *)(bp + q * 64 + 32));                         \
        _Pragma("GCC unroll 6") for (int r = 0; r < 6; r++) {                                         \
          int32_t w;                                                                                  \
          std::memcpy(&w, a + (size_t)r * K + q * 4, 4);                                              \
          __m256i av = _mm256_set1_epi32(w);                                                          \
          c[r][0] = DPBUSD(c[r][0], av, b0);                                                          \
          c[r][1] = DPBUSD(c[r][1], av, b1);                                                          \
        }                                                                                             \
      }                                                                                               \
      alignas(32) int32_t t[6][16];                                                                   \
      _Pragma("GCC unroll 6") for (int r = 0; r < 6; r++) {                                           \
        _mm256_store_si256((__m256i *)&t[r][0], c[r][0]);                                             \
        _mm256_store_si256((__m256i *)&t[r][8], c[r][1]);                                             \
      }                                                                                               \
      const int rows = std::min(6, r1 - i0), cols = std::min(16, N - p * 16);                         \
      for (int r = 0; r < rows; r++)                                                                  \
        std::memcpy(acc + (size_t)(i0 + r) * N + p * 16, t[r], sizeof(int32_t) * cols);               \
    }

__attribute__((target("avxvnni,avx2"))) static void gemm_vnni(const uint8_t *A, const int8_t *Bp, int N, int K,
                                                             int r0, int r1, int32_t *acc) {
  ORC_GEMM_BODY(_mm256_dpbusd_avx_epi32)
}

__attribute__((target("avx512vnni,avx512vl,avx2"))) static void gemm_vnni512(const uint8_t *A, const int8_t *Bp,
                                                                             int N, int K, int r0, int r1,
                                                                             int32_t *acc) {
  ORC_GEMM_BODY(_mm256_dpbusd_epi32)
}

// A: rows padded to a multiple of 6 with K (a multiple of 4) bytes each;
// padding depths hold 128 and the panels hold 0 there.
void gemm_u8s8_fast(const uint8_t *A, const int8_t *Bp, int M, int N, int K, int r0, int r1, int32_t *acc) {
  (void)M;
  static const int feat = cpu_features();
  if (feat & 1) return gemm_vnni(A, Bp, N, K, r0, r1, acc);
  if (feat & 2) return gemm_vnni512(A, Bp, N, K, r0, r1, acc);
  // No VNNI: portable loop over the panels (same integers).
  const int kq = K / 4;
  for (int i = r0; i < r1; i++)
    for (int j = 0; j < N; j++) {
      int32_t s = 0;
      const int8_t *b = Bp + (size_t)(j / 16) * kq * 64 + (j % 16) * 4;
      for (int q = 0; q < kq; q++)
        for (int t = 0; t < 4; t++) s += (int32_t)A[(size_t)i * K + q * 4 + t] * (int32_t)b[q * 64 + t];
      acc[(size_t)i * N + j] = s;
    }
}

}  // namespace orc
