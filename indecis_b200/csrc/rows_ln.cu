// LayerNorm (+ per-row int8 quantization) with several rows per warp.
//
// Same arithmetic as layernorm_warp / quant_row_warp (rows.cu), which restate
// linalg/vec_simd.go:281-327 and linalg/int8.go:157-191; this version only
// maps it better onto a warp: with V float32 lanes in the reference, a warp
// takes 32/V rows and lane (r, k) = r*V + k runs the reference's lane-k
// chain of row r in registers, so no lane idles during the ordered sums.
// Rows are staged in shared memory with a pitch that is V mod 32, which puts
// the lanes of one chain step in distinct banks. The float64 combine of the
// V partial sums happens in each lane of the group through shuffles, in lane
// order; outputs are then written by the whole warp with 16-byte stores.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"

namespace ig {

template <bool EMBED>
__global__ void ln_group_kernel(const float *__restrict__ x, const int32_t *__restrict__ ids, int vocab,
                                const EmbTable emb, const float *__restrict__ gamma, const float *__restrict__ beta,
                                int M, int H,
                                double eps, int V, int P, int wpb, float *__restrict__ xout, uint8_t *__restrict__ q,
                                int ldq, float *__restrict__ sa) {
  extern __shared__ float s_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rpw = 32 / V;
  const int row0 = (blockIdx.x * wpb + warp) * rpw;
  if (row0 >= M) return;
  float *s = s_all + (size_t)warp * rpw * P;
  for (int r = 0; r < rpw && row0 + r < M; r++) {
    const int row = row0 + r;
    const float *src;
    float *dst = s + r * P;
    if constexpr (EMBED) {
      int id = ids[row];
      if (id < 0 || id >= vocab) {
        if (lane == 0) set_device_error(kDevBadId);
        id = 0;
      }
      if (emb.fmt != IG_EMB_F32) {  // rows widened element by element
        for (int i = lane; i < H; i += 32) dst[i] = emb_elem(emb, id, i, H);
        continue;
      }
      src = emb.f32 + (size_t)id * H;
    } else {
      src = x + (size_t)row * H;
    }
    if ((H & 3) == 0 && (P & 3) == 0) {
      for (int i = lane * 4; i < H; i += 128)
        *reinterpret_cast<float4 *>(dst + i) = __ldg(reinterpret_cast<const float4 *>(src + i));
    } else {
      for (int i = lane; i < H; i += 32) dst[i] = __ldg(src + i);
    }
  }
  __syncwarp();
  const int r = lane / V, k = lane % V;
  const int row = row0 + r;
  const bool rv = row < M;
  float *sr = s + r * P;
  float mx = 0.0f;
  if (gamma) {
    const int nb = H / V;
    float ls = 0.0f;
    for (int b = 0; b < nb; b++) ls = __fadd_rn(ls, sr[b * V + k]);
    double sum = 0.0;
    for (int kk = 0; kk < V; kk++) sum = __dadd_rn(sum, (double)__shfl_sync(0xffffffffu, ls, r * V + kk));
    for (int i = nb * V; i < H; i++) sum = __dadd_rn(sum, (double)sr[i]);
    const float mean = __double2float_rn(__ddiv_rn(sum, (double)H));
    float lq = 0.0f;
    for (int b = 0; b < nb; b++) {
      const float d = __fsub_rn(sr[b * V + k], mean);
      lq = __fmaf_rn(d, d, lq);
    }
    double var = 0.0;
    for (int kk = 0; kk < V; kk++) var = __dadd_rn(var, (double)__shfl_sync(0xffffffffu, lq, r * V + kk));
    for (int i = nb * V; i < H; i++) {
      const double d = (double)__fsub_rn(sr[i], mean);
      var = __dadd_rn(var, __dmul_rn(d, d));
    }
    const float rstd = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(var, (double)H), eps))));
    __syncwarp();
    for (int i = k; i < H; i += V) {
      float o = __fmul_rn(__fmul_rn(__fsub_rn(sr[i], mean), rstd), __ldg(gamma + i));
      if (beta) o = __fadd_rn(o, __ldg(beta + i));  // AddTo(o, beta) after LayerNormRow
      sr[i] = o;
      mx = fmaxf(mx, fabsf(o));
    }
  } else {
    for (int i = k; i < H; i += V) mx = fmaxf(mx, fabsf(sr[i]));
  }
  for (int off = V >> 1; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  float scale = 0.0f, inv = 0.0f;
  if (mx > 0.0f) {
    scale = __fdiv_rn(mx, 127.0f);
    inv = __fdiv_rn(1.0f, scale);
  }
  if (q && k == 0 && rv) sa[row] = scale;
  __syncwarp();
  for (int rr = 0; rr < rpw && row0 + rr < M; rr++) {
    const int rowr = row0 + rr;
    const float invr = __shfl_sync(0xffffffffu, inv, rr * V);
    const float scaler = __shfl_sync(0xffffffffu, scale, rr * V);
    const float *srr = s + rr * P;
    if (xout) {
      float *dst = xout + (size_t)rowr * H;
      if ((H & 3) == 0 && (P & 3) == 0) {
        for (int i = lane * 4; i < H; i += 128)
          *reinterpret_cast<float4 *>(dst + i) = *reinterpret_cast<const float4 *>(srr + i);
      } else {
        for (int i = lane; i < H; i += 32) dst[i] = srr[i];
      }
    }
    if (q) {
      uint8_t *dq = q + (size_t)rowr * ldq;
      auto qv = [&](float v) -> uint32_t {
        if (scaler == 0.0f) return 128u;  // a zero row
        const int t = max(-128, min(127, rne_int(__fmul_rn(v, invr))));
        return (uint32_t)(t + 128);
      };
      if ((H & 3) == 0 && (ldq & 3) == 0) {
        for (int i = lane * 4; i < H; i += 128) {
          const uint32_t w = qv(srr[i]) | (qv(srr[i + 1]) << 8) | (qv(srr[i + 2]) << 16) | (qv(srr[i + 3]) << 24);
          *reinterpret_cast<uint32_t *>(dq + i) = w;
        }
      } else {
        for (int i = lane; i < H; i += 32) dq[i] = (uint8_t)qv(srr[i]);
      }
    }
  }
}

// Launch geometry of ln_group_kernel for H values and V lanes; false when
// the grouped kernel does not apply (V not dividing 32, rows too wide).
static bool ln_group_geometry(int H, int V, int *P, int *wpb, size_t *smem) {
  if (V < 1 || V > 32 || (32 % V) != 0 || H <= 0) return false;
  const int rpw = 32 / V;
  int p = (H + 31) / 32 * 32 + V;
  if (V < 4) p = (H + 31) / 32 * 32 + 4;
  const size_t per_warp = (size_t)rpw * p * sizeof(float);
  if (per_warp > 96 * 1024) return false;
  int w = (int)((48 * 1024) / per_warp);
  w = w < 1 ? 1 : (w > 8 ? 8 : w);
  *P = p;
  *wpb = w;
  *smem = per_warp * w;
  return true;
}

template <bool EMBED>
static int launch_ln_group(const float *x, const int32_t *ids, int vocab, const EmbTable &emb, const float *gamma,
                           const float *beta, int M, int H, double eps, int V, float *xout, uint8_t *q, int ldq,
                           float *sa, cudaStream_t st) {
  int P = 0, wpb = 0;
  size_t smem = 0;
  if (!ln_group_geometry(H, V, &P, &wpb, &smem)) return -1;
  static SmemOptIn attr;
  if (smem > 48 * 1024 && attr.ensure((const void *)ln_group_kernel<EMBED>, (int)smem) != cudaSuccess)
    return IG_ERR_CUDA;
  const int rows_per_block = wpb * (32 / V);
  const int blocks = (M + rows_per_block - 1) / rows_per_block;
  ln_group_kernel<EMBED><<<blocks, 32 * wpb, smem, st>>>(x, ids, vocab, emb, gamma, beta, M, H, eps, V, P, wpb, xout,
                                                          q, ldq, sa);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig
