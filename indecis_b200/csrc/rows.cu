// Row kernels of the encoder: embedding gather, LayerNorm with the fused
// per-row int8 quantization of the next GEMM's input, plain quantization,
// pooling, float64 head logits and the one-time weight quantization.
//
// LayerNorm restates linalg/vec_simd.go:281-327 (LayerNormRow): sums in V
// float32 lanes, lane k adding x[k], x[k+V], ... in order, the lanes then
// summed in float64; the variance lanes use a fused multiply-add; rstd is
// computed in float64. A row is one warp: the row is staged in shared memory,
// V lanes run the ordered float32 chains, lane 0 the float64 reductions, and
// all 32 lanes do the elementwise output and quantization.
//
// Quantization restates linalg/int8.go:157-191 (quantizeA) and
// linalg/quant_amd64.s:17-121: s = max|x|/127, q = rne(x * (1/s)) + 128.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"

namespace ig {

constexpr int kRowWarps = 8;

// Several rows per warp (rows_ln.cu); -1 when it does not apply.
template <bool EMBED>
static int launch_ln_group(const float *x, const int32_t *ids, int vocab, const EmbTable &emb, const float *gamma,
                           const float *beta, int M, int H, double eps, int V, float *xout, uint8_t *q, int ldq,
                           float *sa, cudaStream_t st);

// Per-row quantization of the n values in s_row (shared), by one warp.
__device__ __forceinline__ void quant_row_warp(const float *s_row, int n, uint8_t *q, float *sa, int lane) {
  float mx = 0.0f;
  for (int i = lane; i < n; i += 32) mx = fmaxf(mx, fabsf(s_row[i]));
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (mx == 0.0f) {
    for (int i = lane; i < n; i += 32) q[i] = 128;
    if (lane == 0) *sa = 0.0f;
    return;
  }
  const float s = __fdiv_rn(mx, 127.0f);
  const float inv = __fdiv_rn(1.0f, s);
  for (int i = lane; i < n; i += 32) {
    int v = rne_int(__fmul_rn(s_row[i], inv));
    v = max(-128, min(127, v));
    q[i] = (uint8_t)(v + 128);
  }
  if (lane == 0) *sa = s;
}

// LayerNormRow over s_x (shared, n values), result back into s_x.
__device__ __forceinline__ void layernorm_warp(float *s_x, const float *gamma, int n, double eps, int V, int lane) {
  const int nb = n / V;
  float lane_sum = 0.0f;
  if (lane < V)
    for (int b = 0; b < nb; b++) lane_sum = __fadd_rn(lane_sum, s_x[b * V + lane]);
  double sum = 0.0;
  for (int k = 0; k < V; k++) sum = __dadd_rn(sum, (double)__shfl_sync(0xffffffffu, lane_sum, k));
  for (int i = nb * V; i < n; i++) sum = __dadd_rn(sum, (double)s_x[i]);
  const float mean = __double2float_rn(__ddiv_rn(sum, (double)n));
  float lane_sq = 0.0f;
  if (lane < V)
    for (int b = 0; b < nb; b++) {
      const float d = __fsub_rn(s_x[b * V + lane], mean);
      lane_sq = __fmaf_rn(d, d, lane_sq);
    }
  double var = 0.0;
  for (int k = 0; k < V; k++) var = __dadd_rn(var, (double)__shfl_sync(0xffffffffu, lane_sq, k));
  for (int i = nb * V; i < n; i++) {
    const double d = (double)__fsub_rn(s_x[i], mean);
    var = __dadd_rn(var, __dmul_rn(d, d));
  }
  const float rstd = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(var, (double)n), eps))));
  __syncwarp();
  for (int i = lane; i < n; i += 32)
    s_x[i] = __fmul_rn(__fmul_rn(__fsub_rn(s_x[i], mean), rstd), __ldg(gamma + i));
  __syncwarp();
}

__global__ void ln_quant_kernel(const float *__restrict__ x, const float *__restrict__ gamma, int M, int H,
                                double eps, int V, float *__restrict__ xn, uint8_t *__restrict__ q, int ldq,
                                float *__restrict__ sa) {
  extern __shared__ float s_rows[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= M) return;
  float *s_x = s_rows + warp * H;
  const float *src = x + (size_t)row * H;
  if ((H & 3) == 0) {
    for (int i = lane * 4; i < H; i += 128) *reinterpret_cast<float4 *>(s_x + i) = __ldg(reinterpret_cast<const float4 *>(src + i));
  } else {
    for (int i = lane; i < H; i += 32) s_x[i] = src[i];
  }
  __syncwarp();
  if (gamma) layernorm_warp(s_x, gamma, H, eps, V, lane);
  if (xn) {
    float *dst = xn + (size_t)row * H;
    for (int i = lane; i < H; i += 32) dst[i] = s_x[i];
  }
  if (q) quant_row_warp(s_x, H, q + (size_t)row * ldq, sa + row, lane);
}

// Embedding gather (infer.go:361-367) + LayerNorm(emb_norm) (:368). An id
// outside [0, vocab) is recorded in g_device_error and reads row 0.
__global__ void embed_ln_quant_kernel(const int32_t *__restrict__ ids, int vocab, const EmbTable emb,
                                      const float *__restrict__ gamma, int M, int H, double eps, int V,
                                      float *__restrict__ x, uint8_t *__restrict__ q, int ldq, float *__restrict__ sa) {
  extern __shared__ float s_rows[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= M) return;
  float *s_x = s_rows + warp * H;
  int id = ids[row];
  if (id < 0 || id >= vocab) {
    if (lane == 0) set_device_error(kDevBadId);
    id = 0;
  }
  for (int i = lane; i < H; i += 32) s_x[i] = emb_elem(emb, id, i, H);
  __syncwarp();
  layernorm_warp(s_x, gamma, H, eps, V, lane);
  float *dst = x + (size_t)row * H;
  for (int i = lane; i < H; i += 32) dst[i] = s_x[i];
  if (q) quant_row_warp(s_x, H, q + (size_t)row * ldq, sa + row, lane);
}

__global__ void quant_rows_kernel(const float *__restrict__ x, int ldx, int M, int K, uint8_t *__restrict__ q,
                                  int ldq, float *__restrict__ sa) {
  extern __shared__ float s_rows[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= M) return;
  float *s_x = s_rows + warp * K;
  const float *src = x + (size_t)row * ldx;
  for (int i = lane; i < K; i += 32) s_x[i] = src[i];
  __syncwarp();
  quant_row_warp(s_x, K, q + (size_t)row * ldq, sa + row, lane);
}

// infer.go:261-289: mean over the sequence's tokens in float64, token order.
__global__ void pool_kernel(const float *__restrict__ xn, const int32_t *__restrict__ offs, int H, int cls,
                            float *__restrict__ out) {
  const int s = blockIdx.x;
  dep_wait();
  dep_trigger();
  const int t0 = offs[s], t1 = offs[s + 1];
  const int n = t1 - t0;
  for (int d = threadIdx.x; d < H; d += blockDim.x) {
    float v = 0.0f;
    if (n > 0) {
      if (cls) {
        v = xn[(size_t)t0 * H + d];
      } else {
        // Token order; eight rows' loads are issued ahead of their additions.
        double acc = 0.0;
        int t = t0;
        for (; t + 8 <= t1; t += 8) {
          float f[8];
#pragma unroll
          for (int u = 0; u < 8; u++) f[u] = __ldg(xn + (size_t)(t + u) * H + d);
#pragma unroll
          for (int u = 0; u < 8; u++) acc = __dadd_rn(acc, (double)f[u]);
        }
        for (; t < t1; t++) acc = __dadd_rn(acc, (double)__ldg(xn + (size_t)t * H + d));
        v = __double2float_rn(__ddiv_rn(acc, (double)n));
      }
    }
    out[(size_t)s * H + d] = v;
  }
}

// pool_kernel's mean for long sequences: the sequence's rows streamed by TMA
// (per stage 64 rows x 32 columns, kPlStages stages in flight) so that one
// CTA per (sequence, 32 columns) reads at the rate its float64 chains
// consume; lane d of warp 0 runs column d's chain in token order (the same
// additions as pool_kernel), warp 1 issues the copies.
constexpr int kPlRows = 64, kPlStages = 8;
__global__ void __launch_bounds__(64) pool_long_kernel(const __grid_constant__ CUtensorMap mx,
                                                       const int32_t *__restrict__ offs, int H,
                                                       float *__restrict__ out) {
  extern __shared__ __align__(128) uint8_t pl_smem[];
  float *stages = reinterpret_cast<float *>(pl_smem);
  uint64_t *full = reinterpret_cast<uint64_t *>(pl_smem + kPlStages * kPlRows * 128);
  uint64_t *empty = full + kPlStages;
  const int s = blockIdx.x, c0 = blockIdx.y * 32, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  dep_wait();
  const int t0 = offs[s], n = offs[s + 1] - t0;
  const int nchunks = (n + kPlRows - 1) / kPlRows;
  if (threadIdx.x == 32) {
    for (int k = 0; k < kPlStages; k++) {
      mbar_init(&full[k], 1);
      mbar_init(&empty[k], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) {
      prefetch_tensormap(&mx);
      for (int c = 0; c < nchunks; c++) {
        const int k = c % kPlStages;
        if (c >= kPlStages && !mbar_wait(&empty[k], ((c / kPlStages) - 1) & 1, kDevTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full[k], kPlRows * 128);
        tma_load_2d(&mx, stages + k * kPlRows * 32, &full[k], c0, t0 + c * kPlRows);
      }
    }
    return;  // exits count as the trigger
  }
  double acc = 0.0;
  for (int c = 0; c < nchunks; c++) {
    const int k = c % kPlStages;
    if (!mbar_wait(&full[k], (c / kPlStages) & 1, kDevTimeoutFull)) break;
    const float *st = stages + k * kPlRows * 32 + lane;
    const int rows = min(kPlRows, n - c * kPlRows);
    if (rows == kPlRows) {
#pragma unroll 16
      for (int r = 0; r < kPlRows; r++) acc = __dadd_rn(acc, (double)st[r * 32]);
    } else {
      for (int r = 0; r < rows; r++) acc = __dadd_rn(acc, (double)st[r * 32]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[k]);
  }
  out[(size_t)s * H + c0 + lane] = n > 0 ? __double2float_rn(__ddiv_rn(acc, (double)n)) : 0.0f;
  dep_trigger();  // one wave of long-lived CTAs: the next kernel is let in at the end
}

__global__ void head_logits_kernel(const float *__restrict__ w, const float *__restrict__ b, int rows, int H,
                                   const float *__restrict__ x, int nx, double *__restrict__ z, int ldz) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  dep_wait();
  dep_trigger();
  if (idx >= nx * rows) return;
  const int t = idx / rows, r = idx % rows;
  const float *wr = w + (size_t)r * H;
  const float *xt = x + (size_t)t * H;
  double s = 0.0;
  for (int i = 0; i < H; i++) s = __dadd_rn(s, __dmul_rn((double)__ldg(wr + i), (double)__ldg(xt + i)));
  z[(size_t)t * ldz + r] = __dadd_rn(s, (double)b[r]);
}

// Every row of a head for one token per thread: the rows' sequential float64
// sums run side by side (heads.go:62-74, same order per row), and the token's
// x[i] is read once for all rows.
__global__ void head_logits_rows_kernel(const float *__restrict__ w, const float *__restrict__ b, int rows, int H,
                                        const float *__restrict__ x, int nx, double *__restrict__ z, int ldz) {
  constexpr int kMaxRows = 16;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  dep_wait();
  dep_trigger();
  if (t >= nx) return;
  const float *xt = x + (size_t)t * H;
  double s[kMaxRows];
#pragma unroll
  for (int r = 0; r < kMaxRows; r++) s[r] = 0.0;
  for (int i = 0; i < H; i++) {
    const double xi = (double)__ldg(xt + i);
#pragma unroll
    for (int r = 0; r < kMaxRows; r++)
      if (r < rows) s[r] = __dadd_rn(s[r], __dmul_rn((double)__ldg(w + (size_t)r * H + i), xi));
  }
#pragma unroll
  for (int r = 0; r < kMaxRows; r++)
    if (r < rows) z[(size_t)t * ldz + r] = __dadd_rn(s[r], (double)b[r]);
}

// PackB8 for one packed row per warp.
__global__ void pack_b8_kernel(const float *__restrict__ w, int n, int k, const int32_t *__restrict__ perm,
                               int n_out, int8_t *__restrict__ q, int ldq, float *__restrict__ scale,
                               float *__restrict__ zc, int32_t *__restrict__ colsum) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= n_out) return;
  const int src = perm ? perm[warp] : warp;
  int8_t *dst = q + (size_t)warp * ldq;
  if (src < 0 || src >= n) {
    for (int i = lane; i < ldq; i += 32) dst[i] = 0;
    if (lane == 0) {
      scale[warp] = 0.0f;
      zc[warp] = 0.0f;
      if (colsum) colsum[warp] = 0;
    }
    return;
  }
  const float *row = w + (size_t)src * k;
  float mx = 0.0f;
  for (int i = lane; i < k; i += 32) mx = fmaxf(mx, fabsf(row[i]));
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  int cs = 0;
  if (mx == 0.0f) {
    for (int i = lane; i < ldq; i += 32) dst[i] = 0;
  } else {
    const float s = __fdiv_rn(mx, 127.0f);
    for (int i = lane; i < ldq; i += 32) {
      int v = 0;
      if (i < k) v = (int)round((double)__fdiv_rn(row[i], s));  // math.Round: half away from zero
      dst[i] = (int8_t)v;
      cs += v;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
  if (lane == 0) {
    const float s = mx == 0.0f ? 0.0f : __fdiv_rn(mx, 127.0f);
    scale[warp] = s;
    zc[warp] = mx == 0.0f ? 0.0f : __fmul_rn(128.0f, (float)cs);
    if (colsum) colsum[warp] = mx == 0.0f ? 0 : cs;
  }
}

static inline int row_blocks(int M) { return (M + kRowWarps - 1) / kRowWarps; }

static int smem_rows_ok(int H) { return H > 0 && (size_t)H * kRowWarps * sizeof(float) <= 200 * 1024; }

static int set_rows_smem(SmemOptIn &attr, const void *fn, int H) {
  const int bytes = H * kRowWarps * (int)sizeof(float);
  if (bytes > 48 * 1024 && attr.ensure(fn, bytes) != cudaSuccess) return IG_ERR_CUDA;
  return 0;
}

int launch_ln_quant(const float *x, const float *gamma, int M, int H, double eps, int V, float *xn, uint8_t *q,
                    int ldq, float *sa, cudaStream_t st) {
  if (M <= 0) return 0;
  if (gamma) {
    int rc = launch_ln8<false>(x, nullptr, 0, EmbTable{}, gamma, nullptr, M, H, eps, V, xn, q, ldq, sa, st);
    if (rc != -1) return rc;
    rc = launch_ln_group<false>(x, nullptr, 0, EmbTable{}, gamma, nullptr, M, H, eps, V, xn, q, ldq, sa, st);
    if (rc != -1) return rc;
  }
  if (!smem_rows_ok(H) || V < 1 || V > 32) return IG_ERR_BAD_ARG;
  static SmemOptIn attr;
  if (set_rows_smem(attr, (const void *)ln_quant_kernel, H)) return IG_ERR_CUDA;
  ln_quant_kernel<<<row_blocks(M), 32 * kRowWarps, H * kRowWarps * sizeof(float), st>>>(x, gamma, M, H, eps, V, xn,
                                                                                          q, ldq, sa);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

int launch_ln_beta(const float *x, const float *gamma, const float *beta, int M, int H, double eps, int V, float *xout,
                   uint8_t *q, int ldq, float *sa, cudaStream_t st) {
  if (M <= 0) return 0;
  if (!gamma || !beta) return IG_ERR_BAD_ARG;
  int rc = launch_ln8<false>(x, nullptr, 0, EmbTable{}, gamma, beta, M, H, eps, V, xout, q, ldq, sa, st);
  if (rc != -1) return rc;
  rc = launch_ln_group<false>(x, nullptr, 0, EmbTable{}, gamma, beta, M, H, eps, V, xout, q, ldq, sa, st);
  return rc == -1 ? IG_ERR_UNSUPPORTED : rc;
}

int launch_embed_checked(const int32_t *ids, int vocab, const EmbTable &emb, const float *gamma, int M, int H,
                         double eps, int V, float *x, uint8_t *q, int ldq, float *sa, cudaStream_t st) {
  if (M <= 0) return 0;
  {
    int rc = launch_ln8<true>(nullptr, ids, vocab, emb, gamma, nullptr, M, H, eps, V, x, q, ldq, sa, st);
    if (rc != -1) return rc;
    rc = launch_ln_group<true>(nullptr, ids, vocab, emb, gamma, nullptr, M, H, eps, V, x, q, ldq, sa, st);
    if (rc != -1) return rc;
  }
  if (!smem_rows_ok(H) || V < 1 || V > 32) return IG_ERR_BAD_ARG;
  static SmemOptIn attr;
  if (set_rows_smem(attr, (const void *)embed_ln_quant_kernel, H)) return IG_ERR_CUDA;
  embed_ln_quant_kernel<<<row_blocks(M), 32 * kRowWarps, H * kRowWarps * sizeof(float), st>>>(
      ids, vocab, emb, gamma, M, H, eps, V, x, q, ldq, sa);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

int launch_quant_rows(const float *x, int ldx, int M, int K, uint8_t *q, int ldq, float *sa, cudaStream_t st) {
  if (M <= 0) return 0;
  {
    const int rc = launch_quant_rows4(x, ldx, M, K, q, ldq, sa, st);
    if (rc != -1) return rc;
  }
  if (!smem_rows_ok(K)) return IG_ERR_BAD_ARG;
  static SmemOptIn attr;
  if (set_rows_smem(attr, (const void *)quant_rows_kernel, K)) return IG_ERR_CUDA;
  quant_rows_kernel<<<row_blocks(M), 32 * kRowWarps, K * kRowWarps * sizeof(float), st>>>(x, ldx, M, K, q, ldq, sa);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

__global__ void fill_rows_kernel(const int32_t *__restrict__ offs, int32_t *__restrict__ row_seq,
                                 int32_t *__restrict__ pos) {
  dep_wait();
  dep_trigger();
  const int s = blockIdx.x, t0 = offs[s], n = offs[s + 1] - t0;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    row_seq[t0 + t] = s;
    pos[t0 + t] = t;
  }
}

int launch_fill_rows(const int32_t *offs, int nseq, int32_t *row_seq, int32_t *pos, cudaStream_t st) {
  if (nseq <= 0) return 0;
  launch_dep(fill_rows_kernel, nseq, 128, 0, st, offs, row_seq, pos);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

int launch_pool(const float *xn, const int32_t *offs, int nseq, int H, int cls, float *out, cudaStream_t st,
                int max_len, int nrows) {
  if (nseq <= 0) return 0;
  if (!cls && max_len >= 1024 && H % 32 == 0 && nrows > 0 && !(reinterpret_cast<uintptr_t>(xn) & 15)) {
    // Long sequences: a CTA per (sequence, 32 columns), rows streamed by TMA.
    auto enc = get_encode_fn();
    if (!enc) return IG_ERR_CUDA;
    CUtensorMap map;
    cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)nrows};
    cuuint64_t strides[1] = {(cuuint64_t)H * sizeof(float)};
    cuuint32_t box[2] = {32, (cuuint32_t)kPlRows};
    cuuint32_t estr[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(xn), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return IG_ERR_CUDA;
    const int smem = kPlStages * kPlRows * 128 + 16 * kPlStages;
    static SmemOptIn attr;
    if (attr.ensure((const void *)pool_long_kernel, smem) != cudaSuccess) return IG_ERR_CUDA;
    launch_dep(pool_long_kernel, dim3(nseq, H / 32), 64, smem, st, map, offs, H, out);
    return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
  }
  launch_dep(pool_kernel, nseq, 256, 0, st, xn, offs, H, cls, out);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

int launch_head_logits(const float *w, const float *b, int rows, int H, const float *x, int nx, double *z, int ldz,
                       cudaStream_t st) {
  if (nx <= 0 || rows <= 0) return 0;
  {
    // Any token count: the weights staged in shared memory once per block
    // beat per-thread global loads in the sequential chains even for the 32
    // pooled vectors of one batch (18 us -> a few us per head).
    const int rc = launch_head_logits_tok(w, b, rows, H, x, nx, z, ldz, st);
    if (rc != -1) return rc;
  }
  if (rows <= 16 && nx >= 1024) {
    launch_dep(head_logits_rows_kernel, (nx + 127) / 128, 128, 0, st, w, b, rows, H, x, nx, z, ldz);
    return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
  }
  const int total = nx * rows;
  launch_dep(head_logits_kernel, (total + 127) / 128, 128, 0, st, w, b, rows, H, x, nx, z, ldz);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

int launch_pack_b8(const float *w, int n, int k, const int32_t *perm, int n_out, int8_t *q, int ldq, float *scale,
                   float *zc, int32_t *colsum, cudaStream_t st) {
  if (n_out <= 0) return 0;
  if (ldq < k) return IG_ERR_BAD_ARG;
  const int threads = 256;
  const int blocks = (n_out * 32 + threads - 1) / threads;
  pack_b8_kernel<<<blocks, threads, 0, st>>>(w, n, k, perm, n_out, q, ldq, scale, zc, colsum);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig
