// Kernels of the encoder's float32 path, the one the reference runs without
// SetInt8 (internal/modernbert/infer.go:304-430): RoPE applied in place to
// the projected queries and keys, the erf GELU x gate of the MLP, and
// attendBlocks' blocked softmax attention (infer.go:590-650). The float32
// products are f32_chain_gemm_kernel's (siglip.cu), in the reference's FMA-
// chain order; every other operation keeps its rounding as written.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "exactmath.cuh"
#include "internal.h"

namespace ig {

// Rope (vec_simd.go:408-425): x1' = a*cos - b*sin, x2' = b*cos + a*sin, each
// product rounded (no FMA). One thread per (row, head, pair).
__global__ void rope_f32_kernel(float *__restrict__ qkv, const int32_t *__restrict__ pos, int N, int H, int nh,
                                const float *__restrict__ cs, const float *__restrict__ sn) {
  const int D = H / nh, half = D / 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long per_row = 2LL * nh * half;
  if (idx >= (long long)N * per_row) return;
  const int r = (int)(idx / per_row), rem = (int)(idx % per_row), h = rem / half, i = rem % half;
  const int t = pos[r];
  float *x = qkv + (size_t)r * 3 * H + h * D;
  const float a = x[i], b = x[half + i], c = __ldg(cs + (size_t)t * half + i), s = __ldg(sn + (size_t)t * half + i);
  x[i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  x[half + i] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

int launch_rope_f32(float *qkv, const int32_t *pos, int N, int H, int nh, const float *cos_, const float *sin_,
                    cudaStream_t st) {
  if (N <= 0) return 0;
  const long long total = (long long)N * nh * (H / nh);  // 2 * nh * half per row
  rope_f32_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(qkv, pos, N, H, nh, cos_, sin_);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

// GeluMul (vec_simd.go:121-160) of each row of I values: the first I &^ 15
// through the FMA body (gelu_amd64.s), the rest through the scalar form.
__global__ void gelu_mul_rows_kernel(const float *__restrict__ z, int N, int I, float *__restrict__ g) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)N * I) return;
  const int r = (int)(idx / I), i = (int)(idx % I);
  const float *zr = z + (size_t)r * 2 * I;
  g[idx] = gelu_mul_at(__ldg(zr + i), __ldg(zr + I + i), i, I);
}

int launch_gelu_mul_rows(const float *z, int N, int I, float *g, cudaStream_t st) {
  if (N <= 0) return 0;
  const long long total = (long long)N * I;
  gelu_mul_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(z, N, I, g);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

// ---- attendBlocks: one CTA per (sequence, head, block of 64 queries) -------------

constexpr int kAbQ = 64;     // qBlock (infer.go:537)
constexpr int kAbK = 128;    // kBlock (infer.go:538)
constexpr int kAbD = 64;     // head dimension
constexpr int kAbSP = kAbK + 4;  // pitch of a score row (query-major)
struct AbSmem {
  // K^T [64][128] of the key block, then its V [128][64] in the same place:
  // V is copied in (cp.async) while the softmax runs, once S is computed.
  static constexpr int kKt = 0;
  static constexpr int kV = 0;
  static constexpr int kQt = kKt + kAbD * kAbK * 4;       // [64][64]    scaled Q^T of this query block
  static constexpr int kS = kQt + kAbD * kAbQ * 4;        // [64][132]   scores / weights, query-major
  static constexpr int kRow = kS + kAbQ * kAbSP * 4;      // mx[64], sum[64], corr[64]
  static constexpr int kTotal = kRow + 3 * kAbQ * 4;
};

// Go's built-in max on float32: NaN wins, +0 over -0.
__device__ __forceinline__ float go_max_f(float a, float b) {
  if (a != a || b != b) return __int_as_float(0x7fc00000);
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}

// The rows of the block keep the reference's per-row state: the running
// maximum and sum, and the output rescaled by exp32(old max - new max)
// before each key block's P V is added (one chain over the block's keys,
// then added: MatMulPackedN with accumulate). ExpShift runs over each row's
// window slice of the block, its eight lanes counted from the slice start.
__global__ void __launch_bounds__(256, 2) attend_blocks_f32_kernel(const float *__restrict__ qkv,
                                                                const int32_t *__restrict__ seq_off,
                                                                const int2 *__restrict__ tasks, int H, int nh,
                                                                int window, float scale, float *__restrict__ ctx) {
  extern __shared__ __align__(16) uint8_t sm[];
  float *Kt = reinterpret_cast<float *>(sm + AbSmem::kKt);
  float *Vs = reinterpret_cast<float *>(sm + AbSmem::kV);
  float *Qt = reinterpret_cast<float *>(sm + AbSmem::kQt);
  float *S = reinterpret_cast<float *>(sm + AbSmem::kS);
  float *s_mx = reinterpret_cast<float *>(sm + AbSmem::kRow), *s_sum = s_mx + kAbQ, *s_corr = s_sum + kAbQ;
  const int2 task = tasks[blockIdx.x];
  const int h = blockIdx.y;
  const int off = seq_off[task.x], n = seq_off[task.x + 1] - off, i0 = task.y;
  const int rows = min(kAbQ, n - i0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t ld = (size_t)3 * H;
  // Scale(q, scale): the scores are of the scaled queries.
  for (int idx = tid; idx < kAbQ * 16; idx += 256) {
    const int qq = idx & 63, j4 = (idx >> 6) * 4;
    float4 qv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (qq < rows) qv = __ldg(reinterpret_cast<const float4 *>(qkv + (size_t)(off + i0 + qq) * ld + h * kAbD + j4));
    Qt[(j4 + 0) * kAbQ + qq] = __fmul_rn(qv.x, scale);
    Qt[(j4 + 1) * kAbQ + qq] = __fmul_rn(qv.y, scale);
    Qt[(j4 + 2) * kAbQ + qq] = __fmul_rn(qv.z, scale);
    Qt[(j4 + 3) * kAbQ + qq] = __fmul_rn(qv.w, scale);
  }
  if (tid < kAbQ) s_mx[tid] = -INFINITY, s_sum[tid] = 0.0f;
  // P V tile of this thread: queries 4qg..4qg+3, dimensions 4dq..4dq+3.
  const int qg = tid >> 4, dq = tid & 15;
  float o[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int c = 0; c < 4; c++) o[i][c] = 0.0f;
  for (int jb = 0; jb < n; jb += kAbK) {
    const int je = min(n, jb + kAbK), cols = je - jb;
    // The query blocks the reference visits for this key block (infer.go:609-614).
    int q0 = 0, q1 = n;
    if (window >= 0) q0 = max(0, jb - window), q1 = min(n, je + window);
    q0 = q0 / kAbQ * kAbQ;
    if (i0 < q0 || i0 >= q1) continue;
    __syncthreads();  // the previous block's weights and K, V are consumed
    for (int idx = tid; idx < kAbK * 16; idx += 256) {
      const int u = idx & 127, j4 = (idx >> 7) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (u < cols) kv = __ldg(reinterpret_cast<const float4 *>(qkv + (size_t)(off + jb + u) * ld + H + h * kAbD + j4));
      Kt[(j4 + 0) * kAbK + u] = kv.x;
      Kt[(j4 + 1) * kAbK + u] = kv.y;
      Kt[(j4 + 2) * kAbK + u] = kv.z;
      Kt[(j4 + 3) * kAbK + u] = kv.w;
    }
    __syncthreads();
    // S = (scaled Q) K^T: warp w takes queries 8w.., lane the keys 4 lane..4 lane + 3.
    {
      float acc[8][4];
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int m = 0; m < 4; m++) acc[i][m] = 0.0f;
#pragma unroll 4
      for (int j = 0; j < kAbD; j++) {
        const float4 a0 = *reinterpret_cast<const float4 *>(Qt + j * kAbQ + warp * 8);
        const float4 a1 = *reinterpret_cast<const float4 *>(Qt + j * kAbQ + warp * 8 + 4);
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float4 k4 = *reinterpret_cast<const float4 *>(Kt + j * kAbK + 4 * lane);
        const float kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
          for (int m = 0; m < 4; m++) acc[i][m] = __fmaf_rn(av[i], kv[m], acc[i][m]);
      }
#pragma unroll
      for (int i = 0; i < 8; i++)
        *reinterpret_cast<float4 *>(S + (warp * 8 + i) * kAbSP + 4 * lane) =
            make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
    __syncthreads();
    // K^T is consumed: V of the block comes into its place during the softmax
    // (the rows past the block's keys are never read).
    for (int idx = tid; idx < cols * 16; idx += 256) {
      const int u = idx >> 4, j4 = (idx & 15) * 4;
      cp_async16(Vs + u * kAbD + j4, qkv + (size_t)(off + jb + u) * ld + 2 * H + h * kAbD + j4);
    }
    // The softmax update of each row: four threads per row, thread p running
    // ExpShift's lanes 2p and 2p + 1 over the row's window slice.
    {
      const int row = tid >> 2, part = tid & 3, i = i0 + row;
      float *sr = S + row * kAbSP;
      int cs = 0, ce = cols;
      if (window >= 0) cs = max(0, i - window - jb), ce = min(cols, i + window + 1 - jb);
      const bool live = row < rows && cs < ce;
      float bm = -INFINITY;
      if (live)
        for (int u = cs + part; u < ce; u += 4) bm = go_max_f(bm, sr[u]);
      bm = go_max_f(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
      bm = go_max_f(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
      const float mold = s_mx[row];
      const float m = go_max_f(mold, bm);
      const int nval = ce - cs, nvv = nval - nval % 8;
      float la = 0.0f, lb = 0.0f;
      if (live) {
        for (int k = 0; k < nvv; k += 8) {
          float *pa = sr + cs + k + 2 * part, *pb = pa + 1;
          const float ea = exp_body(__fsub_rn(*pa, m)), eb = exp_body(__fsub_rn(*pb, m));
          *pa = ea, *pb = eb;
          la = __fadd_rn(la, ea);
          lb = __fadd_rn(lb, eb);
        }
      }
      const int base = lane & ~3;
      float lanes[8];
#pragma unroll
      for (int p = 0; p < 4; p++) {
        lanes[2 * p] = __shfl_sync(0xffffffffu, la, base + p);
        lanes[2 * p + 1] = __shfl_sync(0xffffffffu, lb, base + p);
      }
      if (part == 0) {
        float corr = 1.0f;
        if (live) {
          float es = 0.0f;
#pragma unroll
          for (int k = 0; k < 8; k++) es = __fadd_rn(es, lanes[k]);
          for (int u = cs + nvv; u < ce; u++) {
            const float e = exp_tail(__fsub_rn(sr[u], m));
            sr[u] = e;
            es = __fadd_rn(es, e);
          }
          corr = exp_tail(__fsub_rn(mold, m));
          float sum = s_sum[row];
          if (corr != 1.0f) sum = __fmul_rn(sum, corr);
          s_sum[row] = __fadd_rn(sum, es);
          s_mx[row] = m;
        }
        s_corr[row] = corr;
      }
      __syncwarp();
      // clear(row[:cs]), clear(row[ce:]); a row without a key of the block is cleared whole.
      if (row < rows)
        for (int u = part; u < cols; u += 4)
          if (!live || u < cs || u >= ce) sr[u] = 0.0f;
    }
    cp_async_wait_all();
    __syncthreads();
    // o = o * corr, then o += (one chain over the block's keys, in key
    // order: four keys' weights of a query come in one 16-byte read).
    if (4 * qg < rows) {
      float acc[4][4];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int c = 0; c < 4; c++) acc[i][c] = 0.0f;
      const float *pr = S + 4 * qg * kAbSP;
      const float *vc = Vs + 4 * dq;
      const int cols4 = cols & ~3;
      for (int u = 0; u < cols4; u += 4) {
        float pv[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float4 p4 = *reinterpret_cast<const float4 *>(pr + i * kAbSP + u);
          pv[i][0] = p4.x, pv[i][1] = p4.y, pv[i][2] = p4.z, pv[i][3] = p4.w;
        }
#pragma unroll
        for (int t = 0; t < 4; t++) {
          const float4 v4 = *reinterpret_cast<const float4 *>(vc + (u + t) * kAbD);
#pragma unroll
          for (int i = 0; i < 4; i++) {
            acc[i][0] = __fmaf_rn(pv[i][t], v4.x, acc[i][0]);
            acc[i][1] = __fmaf_rn(pv[i][t], v4.y, acc[i][1]);
            acc[i][2] = __fmaf_rn(pv[i][t], v4.z, acc[i][2]);
            acc[i][3] = __fmaf_rn(pv[i][t], v4.w, acc[i][3]);
          }
        }
      }
      for (int u = cols4; u < cols; u++) {
        const float4 v4 = *reinterpret_cast<const float4 *>(vc + u * kAbD);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float p = pr[i * kAbSP + u];
          acc[i][0] = __fmaf_rn(p, v4.x, acc[i][0]);
          acc[i][1] = __fmaf_rn(p, v4.y, acc[i][1]);
          acc[i][2] = __fmaf_rn(p, v4.z, acc[i][2]);
          acc[i][3] = __fmaf_rn(p, v4.w, acc[i][3]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float c = s_corr[4 * qg + i];
#pragma unroll
        for (int d = 0; d < 4; d++) {
          if (c != 1.0f) o[i][d] = __fmul_rn(o[i][d], c);
          o[i][d] = __fadd_rn(o[i][d], acc[i][d]);
        }
      }
    }
  }
  __syncthreads();
  // Scale(o, 1/sum).
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int q = 4 * qg + i;
    if (q < rows) {
      const float inv = __fdiv_rn(1.0f, s_sum[q]);
      *reinterpret_cast<float4 *>(ctx + (size_t)(off + i0 + q) * H + h * kAbD + 4 * dq) =
          make_float4(__fmul_rn(o[i][0], inv), __fmul_rn(o[i][1], inv), __fmul_rn(o[i][2], inv),
                      __fmul_rn(o[i][3], inv));
    }
  }
}

int launch_attend_blocks_f32(const float *qkv, const int32_t *seq_off, const int2 *tasks, int ntasks, int H, int nh,
                             int window, float scale, int V, float *ctx, cudaStream_t st) {
  if (ntasks <= 0) return 0;
  if (H != nh * kAbD || V != 8) return IG_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(ctx)) & 15) return IG_ERR_BAD_ARG;
  static SmemOptIn attr;
  if (attr.ensure((const void *)attend_blocks_f32_kernel, AbSmem::kTotal) != cudaSuccess) return IG_ERR_CUDA;
  attend_blocks_f32_kernel<<<dim3(ntasks, nh), 256, AbSmem::kTotal, st>>>(qkv, seq_off, tasks, H, nh, window, scale,
                                                                           ctx);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig
