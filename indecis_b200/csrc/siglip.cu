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
__global__ void __launch_bounds__(256, 2) f32_chain_gemm_kernel(const F32Gemm p) {
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
      const bool first = kend <= kKc && !p.accumulate;
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
  const bool one_block = p.K <= kKc && !p.accumulate;
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
  if (p0.accumulate && (p0.bias || p0.gelu_seg_rows > 0 || p0.add)) return IG_ERR_BAD_ARG;
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

constexpr int kAttMaxT = 256;         // patches held in shared memory
constexpr int kAttD = 64;             // head dimension
constexpr int kAttQB = 32;            // queries per block
constexpr int kAttKP = kAttMaxT + 4;  // pitch of K^T rows
constexpr int kAttSP = kAttQB + 4;    // pitch of score rows (one key per row) and of Q^T rows
constexpr int kAttThreads = 512;      // 8 producer warps + 8 consumer warps
struct AttF32Smem {
  static constexpr int kKt = 0;                                   // [64][kAttKP]     K^T
  static constexpr int kV = kKt + kAttD * kAttKP * 4;             // [256][64]        V
  static constexpr int kQt = kV + kAttMaxT * kAttD * 4;           // [2][64][kAttSP]  Q^T of a block
  static constexpr int kSt = kQt + 2 * kAttD * kAttSP * 4;        // [2][256][kAttSP] scores, key-major
  static constexpr int kInv = kSt + 2 * kAttMaxT * kAttSP * 4;    // [2][32] 1/sum of each row
  static constexpr int kTotal = kInv + 2 * kAttQB * 4;
  static_assert(kTotal <= 227 * 1024, "shared memory");
};
// Named barriers (0 is __syncthreads): block b's scores ready / its buffer free.
constexpr int kBarFull = 1, kBarEmpty = 3, kBarProd = 5;

// Warp-specialized: warps 0-7 (producer) load a block of 32 queries,
// compute its scores S = QK^T (4 queries x 7 key groups per thread, keys
// lane + 32m, the query values broadcast) and its softmax into one of two
// score buffers; warps 8-15 (consumer) compute O = PV of the block before
// (4 queries x 2 dimensions per thread). Every output keeps the reference's
// chain: S over the head dimension, O over the keys, in order; chains that
// share an operand run in pairs (f32x2: each lane one fused multiply-add).
__global__ void __launch_bounds__(kAttThreads, 1)
    attn_f32_kernel(const float *__restrict__ qkv, int T, int H, int nh, float scale, float *__restrict__ ctx) {
  extern __shared__ __align__(16) uint8_t sm[];
  float *Kt = reinterpret_cast<float *>(sm + AttF32Smem::kKt);
  float *Vs = reinterpret_cast<float *>(sm + AttF32Smem::kV);
  const int img = blockIdx.x / nh, h = blockIdx.x % nh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t row0 = (size_t)img * T;
  const size_t ld = (size_t)3 * H;
  const int T4 = (T + 3) & ~3;  // keys in whole groups of four (zeros past T)
  // K^T: lanes run along the keys, so the scalar stores hit distinct banks.
  for (int idx = tid; idx < T4 * 16; idx += kAttThreads) {
    const int u = idx % T4, j4 = (idx / T4) * 4;
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (u < T) kv = __ldg(reinterpret_cast<const float4 *>(qkv + (row0 + u) * ld + H + h * kAttD + j4));
    Kt[(j4 + 0) * kAttKP + u] = kv.x;
    Kt[(j4 + 1) * kAttKP + u] = kv.y;
    Kt[(j4 + 2) * kAttKP + u] = kv.z;
    Kt[(j4 + 3) * kAttKP + u] = kv.w;
  }
  for (int idx = tid; idx < T * 16; idx += kAttThreads) {
    const int u = idx >> 4, j4 = (idx & 15) * 4;
    *reinterpret_cast<float4 *>(Vs + u * kAttD + j4) =
        __ldg(reinterpret_cast<const float4 *>(qkv + (row0 + u) * ld + 2 * H + h * kAttD + j4));
  }
  __syncthreads();
  const int nb = (T + kAttQB - 1) / kAttQB;
  if (warp < 8) {
    // ---- producer ----
    const int pt = tid;                    // 0..255
    const int nv = T - T % 8;              // ExpShift's vector part (V = 8 lanes)
    const int nkg = (T4 + 31) >> 5;        // key groups of 32
    const int sq = warp * 4;               // this warp's four queries
    for (int b = 0; b < nb; b++) {
      const int q0 = b * kAttQB, buf = b & 1;
      float *Qt = reinterpret_cast<float *>(sm + AttF32Smem::kQt) + buf * kAttD * kAttSP;
      float *St = reinterpret_cast<float *>(sm + AttF32Smem::kSt) + buf * kAttMaxT * kAttSP;
      if (b >= 2) named_barrier_sync(kBarEmpty + buf, kAttThreads);  // the consumer is done with this buffer
      for (int idx = pt; idx < kAttQB * 16; idx += 256) {
        const int qq = idx & 31, j4 = (idx >> 5) * 4;
        float4 qv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + qq < T) qv = __ldg(reinterpret_cast<const float4 *>(qkv + (row0 + q0 + qq) * ld + h * kAttD + j4));
        Qt[(j4 + 0) * kAttSP + qq] = qv.x;
        Qt[(j4 + 1) * kAttSP + qq] = qv.y;
        Qt[(j4 + 2) * kAttSP + qq] = qv.z;
        Qt[(j4 + 3) * kAttSP + qq] = qv.w;
      }
      named_barrier_sync(kBarProd, 256);
      // S = Q K^T (one 256-deep block), Scale(s, scale), stored key-major.
      if (q0 + sq < T) {
        float2 acc[4][4];  // [query][group pair]: .x group 2p, .y group 2p + 1
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int g = 0; g < 4; g++) acc[i][g] = make_float2(0.0f, 0.0f);
        const float *kr = Kt + lane;
#pragma unroll 4
        for (int j = 0; j < kAttD; j++) {
          const float4 a = *reinterpret_cast<const float4 *>(Qt + j * kAttSP + sq);
          const float av[4] = {a.x, a.y, a.z, a.w};
          const float *kj = kr + j * kAttKP;
#pragma unroll
          for (int g = 0; g < 4; g++) {
            if (2 * g < nkg) {
              const float2 kk = make_float2(kj[64 * g], kj[64 * g + 32]);
#pragma unroll
              for (int i = 0; i < 4; i++) acc[i][g] = __ffma2_rn(make_float2(av[i], av[i]), kk, acc[i][g]);
            }
          }
        }
#pragma unroll
        for (int m = 0; m < 8; m++) {
          const int u = lane + 32 * m;
          if (m < nkg && u < T4) {
            float sv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) sv[i] = __fmul_rn((m & 1) ? acc[i][m >> 1].y : acc[i][m >> 1].x, scale);
            *reinterpret_cast<float4 *>(St + u * kAttSP + sq) = make_float4(sv[0], sv[1], sv[2], sv[3]);
          }
        }
      }
      named_barrier_sync(kBarProd, 256);
      // softmax of each query row: eight threads per row, thread p running
      // ExpShift's lane p in order (two exponentials at a time, summed in
      // order); the first combines the lane sums, adds the scalar tail and
      // takes 1/sum.
      if (q0 + (warp << 2) < T) {
        const int row = pt >> 3, part = pt & 7;
        float mx = -INFINITY;
        for (int u = part; u < T; u += 8) mx = fmaxf(mx, St[u * kAttSP + row]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        float l = 0.0f;
        int u = part;
        for (; u + 8 < nv; u += 16) {
          float *p0 = St + u * kAttSP + row, *p1 = p0 + 8 * kAttSP;
          const float2 e = exp_body2(make_float2(__fsub_rn(*p0, mx), __fsub_rn(*p1, mx)));
          *p0 = e.x, *p1 = e.y;
          l = __fadd_rn(__fadd_rn(l, e.x), e.y);
        }
        if (u < nv) {
          float *p0 = St + u * kAttSP + row;
          const float e = exp_body(__fsub_rn(*p0, mx));
          *p0 = e;
          l = __fadd_rn(l, e);
        }
        const int base = lane & ~7;
        float inv = 0.0f;
        float lanes[8];
#pragma unroll
        for (int k = 0; k < 8; k++) lanes[k] = __shfl_sync(0xffffffffu, l, base + k);
        if (part == 0) {
          float sum = 0.0f;
#pragma unroll
          for (int k = 0; k < 8; k++) sum = __fadd_rn(sum, lanes[k]);
          for (int t = nv; t < T; t++) {
            const float e = exp_tail(__fsub_rn(St[t * kAttSP + row], mx));
            St[t * kAttSP + row] = e;
            sum = __fadd_rn(sum, e);
          }
          inv = __fdiv_rn(1.0f, sum);
        }
        // Scale(s, 1/sum) is left to the consumer, which multiplies each
        // weight as it reads it (the same single rounding).
        if (part == 0) reinterpret_cast<float *>(sm + AttF32Smem::kInv)[buf * kAttQB + row] = inv;
      }
      named_barrier_arrive(kBarFull + buf, kAttThreads);  // block b's exponentials and 1/sum are ready
    }
  } else {
    // ---- consumer: O = P V, one chain over the keys each ----
    const int cw = warp - 8;
    const int oq = (cw & 1) * 16 + (lane & 3) * 4, od = (cw >> 1) * 16 + (lane >> 2) * 2;
    for (int b = 0; b < nb; b++) {
      const int q0 = b * kAttQB, buf = b & 1;
      const float *St = reinterpret_cast<const float *>(sm + AttF32Smem::kSt) + buf * kAttMaxT * kAttSP;
      named_barrier_sync(kBarFull + buf, kAttThreads);
      if (q0 + (cw & 1) * 16 < T) {
        const float4 iv = *reinterpret_cast<const float4 *>(sm + AttF32Smem::kInv + (buf * kAttQB + oq) * 4);
        const float2 i01 = make_float2(iv.x, iv.y), i23 = make_float2(iv.z, iv.w);
        float2 o[4];
#pragma unroll
        for (int i = 0; i < 4; i++) o[i] = make_float2(0.0f, 0.0f);
#pragma unroll 4
        for (int t = 0; t < T; t++) {
          const float4 ev = *reinterpret_cast<const float4 *>(St + t * kAttSP + oq);
          const float2 p01 = __fmul2_rn(make_float2(ev.x, ev.y), i01), p23 = __fmul2_rn(make_float2(ev.z, ev.w), i23);
          const float4 pv = make_float4(p01.x, p01.y, p23.x, p23.y);
          const float2 vv = *reinterpret_cast<const float2 *>(Vs + t * kAttD + od);
          o[0] = __ffma2_rn(make_float2(pv.x, pv.x), vv, o[0]);
          o[1] = __ffma2_rn(make_float2(pv.y, pv.y), vv, o[1]);
          o[2] = __ffma2_rn(make_float2(pv.z, pv.z), vv, o[2]);
          o[3] = __ffma2_rn(make_float2(pv.w, pv.w), vv, o[3]);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int q = q0 + oq + i;
          if (q < T) *reinterpret_cast<float2 *>(ctx + (row0 + q) * H + h * kAttD + od) = o[i];
        }
      }
      if (b + 2 < nb) named_barrier_arrive(kBarEmpty + buf, kAttThreads);  // the producer may refill it
    }
  }
}

int launch_attn_f32(const float *qkv, int nimg, int T, int H, int nh, float scale, int V, float *ctx,
                    cudaStream_t st) {
  if (nimg <= 0) return 0;
  if (H != nh * kAttD || T < 1 || T > kAttMaxT || V != 8) return IG_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(ctx)) & 15) return IG_ERR_BAD_ARG;
  static SmemOptIn attr;
  if (attr.ensure((const void *)attn_f32_kernel, AttF32Smem::kTotal) != cudaSuccess) return IG_ERR_CUDA;
  attn_f32_kernel<<<nimg * nh, kAttThreads, AttF32Smem::kTotal, st>>>(qkv, T, H, nh, scale, ctx);
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

// The dequantized weight rows of each image's outlier channels:
// w[img][k][col] = float(q[col][j_k]) * scale[col] (MatMul8Outliers' w).
__global__ void __launch_bounds__(256) outlier_weights_kernel(const int32_t *__restrict__ out,
                                                              const int32_t *__restrict__ nout, int N,
                                                              const int8_t *__restrict__ q, int ldq,
                                                              const float *__restrict__ scale, float *__restrict__ w) {
  const int img = blockIdx.y, k = blockIdx.z;
  if (k >= __ldg(nout + img)) return;
  const int jk = __ldg(out + img * 32 + k);
  for (int col = blockIdx.x * 256 + threadIdx.x; col < N; col += gridDim.x * 256)
    w[((size_t)img * 32 + k) * N + col] = __fmul_rn((float)__ldg(q + (size_t)col * ldq + jk), __ldg(scale + col));
}

// x[row][col] += ((c + sum_k outv[k] * w_k[col]) + bias[col]), c the int8
// product, the outlier terms added in order. One thread per (row, 4 columns).
__global__ void __launch_bounds__(256) outlier_fixup_kernel(const float *__restrict__ c, int M, int T, int N,
                                                            const int32_t *__restrict__ nout,
                                                            const float *__restrict__ outv,
                                                            const float *__restrict__ w,
                                                            const float *__restrict__ bias, float *__restrict__ x) {
  const int n4 = N >> 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)M * n4) return;
  const int row = (int)(idx / n4), col = (int)(idx % n4) * 4;
  const int img = row / T, cnt = __ldg(nout + img);
  const size_t e = (size_t)row * N + col;
  const float4 cv = __ldg(reinterpret_cast<const float4 *>(c + e));
  float v[4] = {cv.x, cv.y, cv.z, cv.w};
  for (int k = 0; k < cnt; k++) {
    const float xv = __ldg(outv + (size_t)row * 32 + k);
    const float4 wk = __ldg(reinterpret_cast<const float4 *>(w + ((size_t)img * 32 + k) * N + col));
    v[0] = __fadd_rn(v[0], __fmul_rn(xv, wk.x));
    v[1] = __fadd_rn(v[1], __fmul_rn(xv, wk.y));
    v[2] = __fadd_rn(v[2], __fmul_rn(xv, wk.z));
    v[3] = __fadd_rn(v[3], __fmul_rn(xv, wk.w));
  }
  const float4 b = __ldg(reinterpret_cast<const float4 *>(bias + col));
  float4 xv = *reinterpret_cast<const float4 *>(x + e);
  xv.x = __fadd_rn(xv.x, __fadd_rn(v[0], b.x));
  xv.y = __fadd_rn(xv.y, __fadd_rn(v[1], b.y));
  xv.z = __fadd_rn(xv.z, __fadd_rn(v[2], b.z));
  xv.w = __fadd_rn(xv.w, __fadd_rn(v[3], b.w));
  *reinterpret_cast<float4 *>(x + e) = xv;
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
                          const float *outv, const int8_t *q, int ldq, const float *scale, const float *bias, float *w,
                          float *x, cudaStream_t st) {
  if (nimg <= 0) return 0;
  if (N % 4 || ((reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(bias) |
                 reinterpret_cast<uintptr_t>(w)) & 15))
    return IG_ERR_BAD_ARG;  // (c may be null: then only the weight rows)
  outlier_weights_kernel<<<dim3((N + 255) / 256, nimg, 32), 256, 0, st>>>(out, nout, N, q, ldq, scale, w);
  if (!c) return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;  // the GEMM epilogue adds them
  const long long total = (long long)nimg * T * (N / 4);
  outlier_fixup_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(c, nimg * T, T, N, nout, outv, w, bias, x);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig
