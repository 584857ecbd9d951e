// Kernels of the SigLIP vision tower (internal/siglip) beyond the int8
// products: its float32 pieces and the outlier split of fc2.
//
// The reference computes these in float32 on the CPU, and the device
// reproduces its roundings:
//  * products (linalg/gemm.go:65-240): each output is one fused multiply-add
//    chain per 256-deep block of the inner dimension, from zero, in depth
//    order (kernel_amd64.s), the first block stored and the next ones added.
//    f32_chain_gemm_kernel runs these chains on the CUDA cores — tensor cores
//    round differently — with 8 x 8 outputs per thread;
//  * attention (internal/siglip/encoder.go:219-251): S = QK^T by chains of
//    head-dim length, softmax(S * scale) with ExpShift's V-lane sums, O = PV
//    by chains over the keys; one CTA per (image, head) keeps K, V and a block
//    of scores in shared memory;
//  * attention pooling (vision.go:164-194): plain multiply-then-add loops;
//  * MatMul8Outliers (linalg/int8.go:281-349): per image, the fc2 input
//    channels whose maximum exceeds six times the mean channel maximum (at
//    most 32) are set aside before the int8 product and added back in
//    float32, in the order the reference adds them.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "exactmath.cuh"
#include "internal.h"

namespace ig {

// ---- float32 products with the reference's chains ----------------------------

constexpr int kFB = 128;  // tile rows and columns
constexpr int kFK = 16;   // depth per shared-memory stage
constexpr int kKc = 256;  // depth of a chain block (linalg/gemm.go:26)

// Eight consecutive elements [k, k+8) of row r of a row-major matrix, zero
// outside [0, rows) x [0, K).
__device__ __forceinline__ void load8_rows(const float *__restrict__ base, int ld, int rows, int K, int r, int k,
                                           bool vec, float (&o)[8]) {
  if (r < rows && vec && k + 8 <= K) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(base + (size_t)r * ld + k));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(base + (size_t)r * ld + k + 4));
    o[0] = a.x, o[1] = a.y, o[2] = a.z, o[3] = a.w, o[4] = b.x, o[5] = b.y, o[6] = b.z, o[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) o[i] = (r < rows && k + i < K) ? __ldg(base + (size_t)r * ld + k + i) : 0.0f;
  }
}

// Elements [k, k+8) of patch row r (image r / T, patch r % T in raster
// order), flattened in (channel, y, x) order as patchify does
// (vision.go:145-160), read straight from the pixels [n][3][S][S].
__device__ __forceinline__ void load8_patch(const F32Gemm &p, int r, int k, float (&o)[8]) {
  const int PP = p.P * p.P, g = p.S / p.P;
  if (r < p.M && p.vec_a && k + 8 <= p.K) {  // P % 8 == 0: one pixel row
    const int img = r / p.T, pt = r % p.T;
    const int c = k / PP, rem = k % PP, y = rem / p.P, x = rem % p.P;
    const float *src =
        p.pix + (((size_t)img * 3 + c) * p.S + (size_t)(pt / g) * p.P + y) * p.S + (size_t)(pt % g) * p.P + x;
    const float4 a = __ldg(reinterpret_cast<const float4 *>(src));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(src + 4));
    o[0] = a.x, o[1] = a.y, o[2] = a.z, o[3] = a.w, o[4] = b.x, o[5] = b.y, o[6] = b.z, o[7] = b.w;
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int kk = k + i;
    float v = 0.0f;
    if (r < p.M && kk < p.K) {
      const int img = r / p.T, pt = r % p.T;
      const int c = kk / PP, rem = kk % PP, y = rem / p.P, x = rem % p.P;
      v = __ldg(p.pix + (((size_t)img * 3 + c) * p.S + (size_t)(pt / g) * p.P + y) * p.S + (size_t)(pt % g) * p.P +
                x);
    }
    o[i] = v;
  }
}

template <bool PATCH>
__global__ void __launch_bounds__(256) f32_chain_gemm_kernel(const F32Gemm p) {
  __shared__ __align__(16) float As[2][kFK][kFB + 4];
  __shared__ __align__(16) float Ws[2][kFK][kFB + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * kFB, n0 = blockIdx.x * kFB;
  const int lr = tid >> 1, kh = (tid & 1) * 8;  // loader: one row, half a stage
  float ra[8], rw[8];
  auto load = [&](int k0) {
    if constexpr (PATCH)
      load8_patch(p, m0 + lr, k0 + kh, ra);
    else
      load8_rows(p.A, p.lda, p.M, p.K, m0 + lr, k0 + kh, p.vec_a, ra);
    load8_rows(p.W, p.ldw, p.N, p.K, n0 + lr, k0 + kh, p.vec_w, rw);
  };
  auto store = [&](int b) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
      As[b][kh + i][lr] = ra[i];
      Ws[b][kh + i][lr] = rw[i];
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
  // Output (row, col) of acc[i][j].
  auto orow = [&](int i) { return m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4); };
  auto ocol = [&](int j) { return n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4); };
  const int nk = (p.K + kFK - 1) / kFK;
  load(0);
  store(0);
  __syncthreads();
  for (int kt = 0; kt < nk; kt++) {
    const int b = kt & 1;
    if (kt + 1 < nk) load((kt + 1) * kFK);
#pragma unroll
    for (int kk = 0; kk < kFK; kk++) {
      const float4 a0 = *reinterpret_cast<const float4 *>(&As[b][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&As[b][kk][64 + ty * 4]);
      const float4 w0 = *reinterpret_cast<const float4 *>(&Ws[b][kk][tx * 4]);
      const float4 w1 = *reinterpret_cast<const float4 *>(&Ws[b][kk][64 + tx * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = __fmaf_rn(a[i], w[j], acc[i][j]);
    }
    // A 256-deep block that is not the last ends: as the reference, the
    // first is stored into C and the next ones added to it.
    const int kend = (kt + 1) * kFK;
    if (kend % kKc == 0 && kt + 1 < nk) {
      const bool first = kend <= kKc;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int r = orow(i);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int c = ocol(j);
          if (r < p.M && c < p.N) {
            float *o = p.C + (size_t)r * p.ldc + c;
            *o = first ? acc[i][j] : __fadd_rn(*o, acc[i][j]);
          }
          acc[i][j] = 0.0f;
        }
      }
    }
    if (kt + 1 < nk) store(b ^ 1);
    __syncthreads();
  }
  const long long seg_len = (long long)p.gelu_seg_rows * p.N;
  const bool one_block = p.K <= kKc;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int r = orow(i);
    if (r >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int c = ocol(j);
      if (c >= p.N) continue;
      float v = one_block ? acc[i][j] : __fadd_rn(p.C[(size_t)r * p.ldc + c], acc[i][j]);
      if (p.bias) v = __fadd_rn(v, __ldg(p.bias + c));
      if (p.gelu_seg_rows > 0) v = gelu_tanh_at(v, (long long)(r % p.gelu_seg_rows) * p.N + c, seg_len, p.V);
      if (p.add) v = __fadd_rn(__ldg(p.add + (size_t)(p.add_mod ? r % p.add_mod : r) * p.ldadd + c), v);
      p.C[(size_t)r * p.ldc + c] = v;
    }
  }
}

int launch_f32_gemm(const F32Gemm &p0, cudaStream_t st) {
  if (p0.M <= 0 || p0.N <= 0) return 0;
  if (p0.K <= 0 || !p0.W || !p0.C || (!p0.A && !p0.pix)) return IG_ERR_BAD_ARG;
  F32Gemm p = p0;
  auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  p.vec_w = al16(p.W) && p.ldw % 4 == 0;
  if (p.pix)
    p.vec_a = al16(p.pix) && p.P % 8 == 0 && p.S % 4 == 0;
  else
    p.vec_a = al16(p.A) && p.lda % 4 == 0;
  const dim3 grid((p.N + kFB - 1) / kFB, (p.M + kFB - 1) / kFB);
  if (grid.y > 65535) return IG_ERR_UNSUPPORTED;
  if (p.pix)
    f32_chain_gemm_kernel<true><<<grid, 256, 0, st>>>(p);
  else
    f32_chain_gemm_kernel<false><<<grid, 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

// ---- attention: one CTA per (image, head) --------------------------------------

constexpr int kAttMaxT = 256;   // patches held in shared memory
constexpr int kAttD = 64;       // head dimension
constexpr int kAttQB = 64;      // queries per block
constexpr int kAttKP = kAttMaxT + 4;  // pitch of K^T rows
constexpr int kAttSP = kAttQB + 4;    // pitch of score rows (one key per row)
struct AttF32Smem {
  static constexpr int kKt = 0;                                  // [64][kAttKP]  K^T
  static constexpr int kV = kKt + kAttD * kAttKP * 4;            // [256][64]     V
  static constexpr int kQt = kV + kAttMaxT * kAttD * 4;          // [64][kAttSP]  Q^T of the block
  static constexpr int kSt = kQt + kAttD * kAttSP * 4;           // [256][kAttSP] scores, key-major
  static constexpr int kTotal = kSt + kAttMaxT * kAttSP * 4;
  static_assert(kTotal <= 227 * 1024, "shared memory");
};

__global__ void __launch_bounds__(256, 1)
    attn_f32_kernel(const float *__restrict__ qkv, int T, int H, int nh, float scale, float *__restrict__ ctx) {
  extern __shared__ __align__(16) uint8_t sm[];
  float *Kt = reinterpret_cast<float *>(sm + AttF32Smem::kKt);
  float *Vs = reinterpret_cast<float *>(sm + AttF32Smem::kV);
  float *Qt = reinterpret_cast<float *>(sm + AttF32Smem::kQt);
  float *St = reinterpret_cast<float *>(sm + AttF32Smem::kSt);
  const int img = blockIdx.x / nh, h = blockIdx.x % nh;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const size_t row0 = (size_t)img * T;
  const size_t ld = (size_t)3 * H;
  const int TP = (T + 63) & ~63;  // keys padded to whole groups of 64 (zeros)
  for (int idx = tid; idx < TP * 16; idx += 256) {
    const int u = idx >> 4, j4 = (idx & 15) * 4;
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
    if (u < T) {
      const float *src = qkv + (row0 + u) * ld + h * kAttD + j4;
      kv = __ldg(reinterpret_cast<const float4 *>(src + H));
      vv = __ldg(reinterpret_cast<const float4 *>(src + 2 * H));
    }
    Kt[(j4 + 0) * kAttKP + u] = kv.x;
    Kt[(j4 + 1) * kAttKP + u] = kv.y;
    Kt[(j4 + 2) * kAttKP + u] = kv.z;
    Kt[(j4 + 3) * kAttKP + u] = kv.w;
    *reinterpret_cast<float4 *>(Vs + u * kAttD + j4) = vv;
  }
  const int nb = TP / 64;  // key groups of 64
  const int nv = T - T % 8;  // ExpShift's vector part (V = 8 lanes)
  for (int q0 = 0; q0 < T; q0 += kAttQB) {
    for (int idx = tid; idx < kAttQB * 16; idx += 256) {
      const int qq = idx >> 4, j4 = (idx & 15) * 4;
      float4 qv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q0 + qq < T) qv = __ldg(reinterpret_cast<const float4 *>(qkv + (row0 + q0 + qq) * ld + h * kAttD + j4));
      Qt[(j4 + 0) * kAttSP + qq] = qv.x;
      Qt[(j4 + 1) * kAttSP + qq] = qv.y;
      Qt[(j4 + 2) * kAttSP + qq] = qv.z;
      Qt[(j4 + 3) * kAttSP + qq] = qv.w;
    }
    __syncthreads();
    // S = Q K^T: queries ty*4.., keys tx*4 + 64b.., one chain over the head
    // dimension each (the whole dimension is one 256-deep block).
    {
      float s[4][16];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int c = 0; c < 16; c++) s[i][c] = 0.0f;
#pragma unroll 4
      for (int j = 0; j < kAttD; j++) {
        const float4 a = *reinterpret_cast<const float4 *>(Qt + j * kAttSP + ty * 4);
        const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int b = 0; b < 4; b++) {
          if (b < nb) {
            const float4 k = *reinterpret_cast<const float4 *>(Kt + j * kAttKP + tx * 4 + 64 * b);
            const float kv[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
              for (int c = 0; c < 4; c++) s[i][4 * b + c] = __fmaf_rn(av[i], kv[c], s[i][4 * b + c]);
          }
        }
      }
      // Scale(s, scale), stored key-major.
#pragma unroll
      for (int b = 0; b < 4; b++)
        if (b < nb)
#pragma unroll
          for (int c = 0; c < 4; c++)
#pragma unroll
            for (int i = 0; i < 4; i++) St[(tx * 4 + 64 * b + c) * kAttSP + ty * 4 + i] = __fmul_rn(s[i][4 * b + c], scale);
    }
    __syncthreads();
    // softmax of each query row: four threads per row, each running two of
    // ExpShift's eight lane sums in order; the first combines them, adds the
    // scalar tail and takes 1/sum.
    {
      const int row = tid >> 2, part = tid & 3;
      float mx = -INFINITY;
      for (int u = part; u < T; u += 4) mx = fmaxf(mx, St[u * kAttSP + row]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float la = 0.0f, lb = 0.0f;
      const int ea = 2 * part, eb = 2 * part + 1;
      for (int u0 = 0; u0 < nv; u0 += 8) {
        float *pa = St + (u0 + ea) * kAttSP + row, *pb = St + (u0 + eb) * kAttSP + row;
        const float xa = exp_body(__fsub_rn(*pa, mx)), xb = exp_body(__fsub_rn(*pb, mx));
        *pa = xa, *pb = xb;
        la = __fadd_rn(la, xa);
        lb = __fadd_rn(lb, xb);
      }
      const int base = threadIdx.x & ~3 & 31;
      float lanes[8];
#pragma unroll
      for (int p = 0; p < 4; p++) {
        lanes[2 * p] = __shfl_sync(0xffffffffu, la, base + p);
        lanes[2 * p + 1] = __shfl_sync(0xffffffffu, lb, base + p);
      }
      float inv = 0.0f;
      if (part == 0) {
        float sum = 0.0f;
#pragma unroll
        for (int l = 0; l < 8; l++) sum = __fadd_rn(sum, lanes[l]);
        for (int u = nv; u < T; u++) {
          const float e = exp_tail(__fsub_rn(St[u * kAttSP + row], mx));
          St[u * kAttSP + row] = e;
          sum = __fadd_rn(sum, e);
        }
        inv = __fdiv_rn(1.0f, sum);
      }
      __syncwarp();
      inv = __shfl_sync(0xffffffffu, inv, base);
      for (int u = part; u < T; u += 4) St[u * kAttSP + row] = __fmul_rn(St[u * kAttSP + row], inv);
    }
    __syncthreads();
    // O = P V: queries ty*4.., dimensions tx*4.., one chain over the keys.
    {
      float o[4][4];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int c = 0; c < 4; c++) o[i][c] = 0.0f;
#pragma unroll 4
      for (int u = 0; u < T; u++) {
        const float4 pv = *reinterpret_cast<const float4 *>(St + u * kAttSP + ty * 4);
        const float4 vv = *reinterpret_cast<const float4 *>(Vs + u * kAttD + tx * 4);
        const float pa[4] = {pv.x, pv.y, pv.z, pv.w}, va[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int c = 0; c < 4; c++) o[i][c] = __fmaf_rn(pa[i], va[c], o[i][c]);
      }
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int q = q0 + ty * 4 + i;
        if (q < T)
          *reinterpret_cast<float4 *>(ctx + (row0 + q) * H + h * kAttD + tx * 4) =
              make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
      }
    }
    __syncthreads();
  }
}

int launch_attn_f32(const float *qkv, int nimg, int T, int H, int nh, float scale, int V, float *ctx,
                    cudaStream_t st) {
  if (nimg <= 0) return 0;
  if (H != nh * kAttD || T < 1 || T > kAttMaxT || V != 8) return IG_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(ctx)) & 15) return IG_ERR_BAD_ARG;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AttF32Smem::kTotal) !=
        cudaSuccess)
      return IG_ERR_CUDA;
    attr = true;
  }
  attn_f32_kernel<<<nimg * nh, 256, AttF32Smem::kTotal, st>>>(qkv, T, H, nh, scale, ctx);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

// ---- attention pooling (vision.go:164-194): one CTA per (image, head) ----------

// softmax(s * scale) over n values in shared memory (encoder.go:246-251),
// the whole block taking part; V = 8 lanes for ExpShift's sums.
__device__ void block_softmax(float *s, int n, float scale, float *red) {
  const int tid = threadIdx.x;
  for (int u = tid; u < n; u += blockDim.x) s[u] = __fmul_rn(s[u], scale);
  __syncthreads();
  float mx = -INFINITY;
  for (int u = tid; u < n; u += blockDim.x) mx = fmaxf(mx, s[u]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) m = fmaxf(m, red[w]);
    red[32] = m;
  }
  __syncthreads();
  mx = red[32];
  const int nv = n - n % 8;
  if (tid < 8) {
    float l = 0.0f;
    for (int u = tid; u < nv; u += 8) {
      const float e = exp_body(__fsub_rn(s[u], mx));
      s[u] = e;
      l = __fadd_rn(l, e);
    }
    red[40 + tid] = l;
  }
  __syncthreads();
  if (tid == 0) {
    float sum = 0.0f;
    for (int l = 0; l < 8; l++) sum = __fadd_rn(sum, red[40 + l]);
    for (int u = nv; u < n; u++) {
      const float e = exp_tail(__fsub_rn(s[u], mx));
      s[u] = e;
      sum = __fadd_rn(sum, e);
    }
    red[33] = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = red[33];
  for (int u = tid; u < n; u += blockDim.x) s[u] = __fmul_rn(s[u], inv);
  __syncthreads();
}

__global__ void __launch_bounds__(256) pool_attn_kernel(const float *__restrict__ kv, const float *__restrict__ probe_q,
                                                        int T, int H, int nh, float scale, float *__restrict__ att) {
  __shared__ float s[kAttMaxT];
  __shared__ float red[64];
  const int img = blockIdx.x / nh, h = blockIdx.x % nh;
  const int tid = threadIdx.x;
  const size_t row0 = (size_t)img * T;
  const float *q = probe_q + h * kAttD;
  for (int t = tid; t < T; t += blockDim.x) {
    const float *k = kv + (row0 + t) * 2 * H + h * kAttD;
    float dot = 0.0f;
    for (int j = 0; j < kAttD; j++) dot = __fadd_rn(dot, __fmul_rn(__ldg(q + j), __ldg(k + j)));
    s[t] = dot;
  }
  __syncthreads();
  block_softmax(s, T, scale, red);
  if (tid < kAttD) {
    float o = 0.0f;
    for (int t = 0; t < T; t++) o = __fadd_rn(o, __fmul_rn(s[t], __ldg(kv + (row0 + t) * 2 * H + H + h * kAttD + tid)));
    att[(size_t)img * H + h * kAttD + tid] = o;
  }
}

int launch_pool_attn(const float *kv, const float *probe_q, int nimg, int T, int H, int nh, float scale, int V,
                     float *att, cudaStream_t st) {
  if (nimg <= 0) return 0;
  if (H != nh * kAttD || T < 1 || T > kAttMaxT || V != 8) return IG_ERR_UNSUPPORTED;
  pool_attn_kernel<<<nimg * nh, 256, 0, st>>>(kv, probe_q, T, H, nh, scale, att);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

// ---- MatMul8Outliers for fc2 --------------------------------------------------

// colmax[img][j] = max over the image's T rows of |x[row][j]|.
__global__ void __launch_bounds__(256) colmax_kernel(const float *__restrict__ x, int T, int K,
                                                     float *__restrict__ colmax) {
  const int img = blockIdx.y;
  const int j = blockIdx.x * 256 + threadIdx.x;
  if (j >= K) return;
  const float *p = x + (size_t)img * T * K + j;
  float m = 0.0f;
  for (int t = 0; t < T; t++) m = fmaxf(m, fabsf(__ldg(p + (size_t)t * K)));
  colmax[(size_t)img * K + j] = m;
}

// One warp per image: the mean of the channel maxima (float32 sum in channel
// order, then / K), the channels above ratio * mean in ascending order and,
// when more than 32, the reference's partial selection sort down to 32.
__global__ void outlier_select_kernel(const float *__restrict__ colmax, int K, float ratio, int32_t *__restrict__ cand,
                                      int32_t *__restrict__ out, int32_t *__restrict__ nout) {
  const int img = blockIdx.x, lane = threadIdx.x;
  const float *cm = colmax + (size_t)img * K;
  int32_t *cd = cand + (size_t)img * K;
  float mean = 0.0f;
  if (lane == 0) {
    for (int j = 0; j < K; j++) mean = __fadd_rn(mean, cm[j]);
    mean = __fdiv_rn(mean, (float)K);
  }
  const float thr = __fmul_rn(ratio, __shfl_sync(0xffffffffu, mean, 0));
  int cnt = 0;
  for (int j0 = 0; j0 < K; j0 += 32) {
    const int j = j0 + lane;
    const bool hit = j < K && cm[j] > thr;
    const unsigned bal = __ballot_sync(0xffffffffu, hit);
    if (hit) cd[cnt + __popc(bal & ((1u << lane) - 1))] = j;
    cnt += __popc(bal);
  }
  __syncwarp();
  for (int i = 0; i < 32 && cnt > 32; i++) {
    // best = the first position x >= i holding the largest maximum
    float bv = -1.0f;
    int bx = 0x7fffffff;
    for (int x = i + lane; x < cnt; x += 32) {
      const float v = cm[cd[x]];
      if (v > bv) bv = v, bx = x;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int ox = __shfl_xor_sync(0xffffffffu, bx, o);
      if (ov > bv || (ov == bv && ox < bx)) bv = ov, bx = ox;
    }
    if (lane == 0) {
      const int t = cd[i];
      cd[i] = cd[bx];
      cd[bx] = t;
    }
    __syncwarp();
  }
  const int n = cnt < 32 ? cnt : 32;
  if (lane < n) out[img * 32 + lane] = cd[lane];
  if (lane == 0) nout[img] = n;
}

// Each row keeps the values of its image's outlier channels (in their
// order) and has them zeroed for the int8 product.
__global__ void outlier_gather_kernel(float *__restrict__ x, int M, int T, int K, const int32_t *__restrict__ out,
                                      const int32_t *__restrict__ nout, float *__restrict__ outv) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), k = threadIdx.x & 31;
  if (row >= M) return;
  const int img = row / T;
  if (k < nout[img]) {
    float *p = x + (size_t)row * K + out[img * 32 + k];
    outv[(size_t)row * 32 + k] = *p;
    *p = 0.0f;
  }
}

// x[row][col] += ((c + sum_k outv[k] * w_k[col]) + bias[col]), c the int8
// product, the outlier terms added in order, w_k = float(q[col][j_k]) * scale.
__global__ void __launch_bounds__(128) outlier_fixup_kernel(const float *__restrict__ c, int T, int N,
                                                            const int32_t *__restrict__ out,
                                                            const int32_t *__restrict__ nout,
                                                            const float *__restrict__ outv, const int8_t *__restrict__ q,
                                                            int ldq, const float *__restrict__ scale,
                                                            const float *__restrict__ bias, float *__restrict__ x) {
  __shared__ float w[32][128];
  const int img = blockIdx.y, col = blockIdx.x * 128 + threadIdx.x;
  const int n = nout[img];
  const bool ok = col < N;
  for (int k = 0; k < n; k++)
    w[k][threadIdx.x] = ok ? __fmul_rn((float)q[(size_t)col * ldq + out[img * 32 + k]], __ldg(scale + col)) : 0.0f;
  if (!ok) return;
  const float b = __ldg(bias + col);
  for (int t = 0; t < T; t++) {
    const size_t row = (size_t)img * T + t;
    float v = c[row * N + col];
    for (int k = 0; k < n; k++) v = __fadd_rn(v, __fmul_rn(__ldg(outv + row * 32 + k), w[k][threadIdx.x]));
    v = __fadd_rn(v, b);
    x[row * N + col] = __fadd_rn(x[row * N + col], v);
  }
}

int launch_outliers_select(const float *x, int nimg, int T, int K, float ratio, float *colmax, int32_t *cand,
                           int32_t *out, int32_t *nout, float *outv, cudaStream_t st) {
  if (nimg <= 0) return 0;
  colmax_kernel<<<dim3((K + 255) / 256, nimg), 256, 0, st>>>(x, T, K, colmax);
  outlier_select_kernel<<<nimg, 32, 0, st>>>(colmax, K, ratio, cand, out, nout);
  const int M = nimg * T;
  outlier_gather_kernel<<<(M + 7) / 8, 256, 0, st>>>(const_cast<float *>(x), M, T, K, out, nout, outv);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

int launch_outliers_fixup(const float *c, int nimg, int T, int N, const int32_t *out, const int32_t *nout,
                          const float *outv, const int8_t *q, int ldq, const float *scale, const float *bias, float *x,
                          cudaStream_t st) {
  if (nimg <= 0) return 0;
  outlier_fixup_kernel<<<dim3((N + 127) / 128, nimg), 128, 0, st>>>(c, T, N, out, nout, outv, q, ldq, scale, bias, x);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig
