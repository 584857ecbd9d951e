// Exhaustive device self-checks of exact-arithmetic shortcuts.
//
// div_erf / div_erf2 (exactmath.cuh) replace an IEEE division in the GELU
// vector body; their argument is a function of the clamped t alone, so
// comparing them with the IEEE quotient for every float t in [-4, 4]
// (2 x 1,082,130,433 values) proves them equal on every input the GeGLU
// epilogue can see.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "exactmath.cuh"

namespace ig {

// [0]: quotients that differ from the IEEE quotient; [1]: values of 1 +
// quotient that differ (the GELU uses the quotient only through 1 + erf).
// Per kind, a histogram over the biased exponent of t.
__device__ unsigned long long g_div_check_bad[2][256];
__device__ unsigned int g_div_check_first = 0xFFFFFFFFu;

__device__ __forceinline__ void div_check_one(uint32_t bits, float fast, float ieee) {
  const uint32_t ex = (bits >> 23) & 255u;
  if (__float_as_uint(fast) != __float_as_uint(ieee)) atomicAdd(&g_div_check_bad[0][ex], 1ull);
  if (__float_as_uint(__fadd_rn(fast, 1.0f)) != __float_as_uint(__fadd_rn(ieee, 1.0f))) {
    atomicAdd(&g_div_check_bad[1][ex], 1ull);
    atomicMin(&g_div_check_first, bits & 0x7FFFFFFFu);
  }
}

// Bits 0 .. 0x40800000 (0 .. 4.0f) and the same values negated; the scalar
// form runs on both, the packed form on the pair (t, -t).
__global__ void gelu_div_check_kernel(uint32_t npos) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < npos; i += stride) {
    const float t = __uint_as_float((uint32_t)i);
    float p, q, pn, qn;
    erf_pq_fma(t, p, q);
    erf_pq_fma(-t, pn, qn);
    const float ip = __fdiv_rn(p, q), in = __fdiv_rn(pn, qn);
    const float2 v2 = div_erf2(make_float2(p, pn), make_float2(q, qn));
    div_check_one((uint32_t)i, div_erf(p, q), ip);
    div_check_one((uint32_t)i | 0x80000000u, div_erf(pn, qn), in);
    div_check_one((uint32_t)i, v2.x, ip);
    div_check_one((uint32_t)i | 0x80000000u, v2.y, in);
  }
}

// The bounded wait every kernel's mbarrier waits go through, made to run out:
// one thread waits on a barrier that no thread and no copy will ever
// complete, with a limit of limit_ns. The wait gives up, records
// kDevTimeoutFull in g_device_error and returns false; the kernel then
// stores the outcome and the time waited and exits, leaving the context
// usable. out[0] = 1 if the wait returned false, out[1] = ns waited.
__global__ void wait_timeout_check_kernel(uint64_t limit_ns, long long *out) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  const uint64_t t0 = globaltimer();
  const bool ok = mbar_wait_limit(&bar, 0, kDevTimeoutFull, limit_ns);
  out[0] = ok ? 0 : 1;
  out[1] = (long long)(globaltimer() - t0);
}

}  // namespace ig

extern "C" int ig_check_wait_timeout(int64_t limit_ns, int32_t *timed_out, int64_t *waited_ns) {
  using namespace ig;
  if (!timed_out || limit_ns <= 0 || limit_ns > 2000000000ll) return IG_ERR_BAD_ARG;
  long long *d = nullptr;
  if (cudaMalloc(&d, 2 * sizeof(long long)) != cudaSuccess) return IG_ERR_CUDA;
  wait_timeout_check_kernel<<<1, 1>>>((uint64_t)limit_ns, d);
  long long h[2] = {0, 0};
  const bool good = cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess &&
                    cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost) == cudaSuccess;
  cudaFree(d);
  if (!good) return IG_ERR_CUDA;
  *timed_out = (int32_t)h[0];
  if (waited_ns) *waited_ns = h[1];
  return 0;
}

extern "C" int ig_check_gelu_division(int64_t *mismatches, uint32_t *first_bad_bits, int64_t *histogram) {
  using namespace ig;
  if (!mismatches) return IG_ERR_BAD_ARG;
  static unsigned long long h[2][256];
  memset(h, 0, sizeof(h));
  unsigned int f = 0xFFFFFFFFu;
  if (cudaMemcpyToSymbol(g_div_check_bad, h, sizeof(h)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_div_check_first, &f, sizeof(f)) != cudaSuccess)
    return IG_ERR_CUDA;
  gelu_div_check_kernel<<<148 * 8, 256>>>(0x40800000u + 1u);
  if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return IG_ERR_CUDA;
  if (cudaMemcpyFromSymbol(h, g_div_check_bad, sizeof(h)) != cudaSuccess ||
      cudaMemcpyFromSymbol(&f, g_div_check_first, sizeof(f)) != cudaSuccess)
    return IG_ERR_CUDA;
  int64_t tot[2] = {0, 0};
  for (int k = 0; k < 2; k++)
    for (int e = 0; e < 256; e++) {
      tot[k] += (int64_t)h[k][e];
      if (histogram) histogram[k * 256 + e] = (int64_t)h[k][e];
    }
  mismatches[0] = tot[0];
  mismatches[1] = tot[1];
  if (first_bad_bits) *first_bad_bits = f;
  return 0;
}
