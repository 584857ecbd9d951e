// int8 attention over unpadded variable-length sequences, local (|i-j| <=
// window) or global, restating linalg/attention8.go (Attn8.prepareAVX2 and
// Attend) as three kernels:
//
//   attn_stats   per (sequence, head, dimension): the mean of K over the
//                sequence (float32, keys in order, then times 1/float32(n):
//                AddTo + Scale, attention8.go:224-229) and the V column
//                scale max|v|/127 with its inverse (attention8.go:255-269).
//   attn_quant   per (row, head), one warp: Q per row (uint8, q+128; scale
//                times the score scale), K centred per key (int8, scale,
//                128*sum), V per column (int8) (quant_amd64.s:17-156).
//   attn_attend  per (sequence, head, block of queries), one warp per query:
//                scores ((acc - kzc)*ks)*sq over the query's valid keys,
//                ExpShift (vector body / scalar tail split by position),
//                P = rne(e*255) as uint8 with sp = 1/float32(sum P), then
//                O = (float(sum P*V) * vs) * sp (attention8.go:298-376).
//
// All products are exact integer dot products (dp4a), so the scores and
// outputs are the reference's bits whatever the tiling.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "exactmath.cuh"
#include "internal.h"

namespace ig {

constexpr int kAttnWarps = 4;
constexpr int kAttnQPerWarp = 4;
constexpr int kAttnQBlock = kAttnWarps * kAttnQPerWarp;

__global__ void attn_stats_kernel(const float *__restrict__ qkv, const int32_t *__restrict__ offs, int H, int nh,
                                  int D, float *__restrict__ kmean, float *__restrict__ vs,
                                  float *__restrict__ vinv) {
  const int s = blockIdx.x, h = blockIdx.y;
  const int t0 = offs[s], t1 = offs[s + 1];
  const int n = t1 - t0;
  const size_t ld = 3 * (size_t)H;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float sum = 0.0f, mx = 0.0f;
    const float *kc = qkv + (size_t)t0 * ld + H + h * D + d;
    const float *vc = qkv + (size_t)t0 * ld + 2 * H + h * D + d;
    int j = 0;
    for (; j + 4 <= n; j += 4) {
      const float k0 = kc[(j + 0) * ld], k1 = kc[(j + 1) * ld], k2 = kc[(j + 2) * ld], k3 = kc[(j + 3) * ld];
      const float v0 = vc[(j + 0) * ld], v1 = vc[(j + 1) * ld], v2 = vc[(j + 2) * ld], v3 = vc[(j + 3) * ld];
      sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, k0), k1), k2), k3);
      mx = fmaxf(fmaxf(fmaxf(fmaxf(mx, fabsf(v0)), fabsf(v1)), fabsf(v2)), fabsf(v3));
    }
    for (; j < n; j++) {
      sum = __fadd_rn(sum, kc[j * ld]);
      mx = fmaxf(mx, fabsf(vc[j * ld]));
    }
    const size_t o = ((size_t)s * nh + h) * D + d;
    kmean[o] = n > 0 ? __fmul_rn(sum, __fdiv_rn(1.0f, (float)n)) : 0.0f;
    const float sc = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 0.0f;
    vs[o] = sc;
    vinv[o] = mx > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
  }
}

// attn_stats_kernel for D = 64 with the (sequence, head) slices of K and V
// (and, with ROPE, the rows' cos/sin factors) staged in shared memory by
// cp.async, 32 rows per stage, STAGES stages in flight. Threads 0-63 run the
// ordered float32 sums (thread d: dimension d of K, rotated at each row's
// position when ROPE), reading a stage whose keys the other 192 threads
// rotated in place while the sums walked the previous stage; those threads
// also take the V column maxima over interleaved rows (maxima combine in any
// order). So the sums' chain holds only a shared-memory read and the add per
// row. The same values as attn_stats_kernel / attn_prep_kernel.
constexpr int kStRows = 32;
constexpr int kStStageFloats = 2 * kStRows * 64 + 2 * kStRows * 32;  // K, V, cos, sin

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_pending() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int STAGES, bool ROPE>
__global__ void __launch_bounds__(256)
    attn_stats64_kernel(const float *__restrict__ qkv, const int32_t *__restrict__ offs, int H, int nh,
                        const float *__restrict__ rope_cos, const float *__restrict__ rope_sin,
                        float *__restrict__ kmean, float *__restrict__ vs, float *__restrict__ vinv) {
  static_assert(STAGES >= 3, "one stage summed, one rotated, one in flight");
  extern __shared__ __align__(16) float st_smem[];  // [stages][K 32x64, V 32x64, cos 32x32, sin 32x32]
  __shared__ float s_vmax[3][64];
  const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  dep_wait();
  dep_trigger();
  const int t0 = offs[s], n = offs[s + 1] - t0;
  const size_t ld = 3 * (size_t)H;
  const float *kbase = qkv + (size_t)t0 * ld + H + h * 64;
  const int nchunks = (n + kStRows - 1) / kStRows;
  // Stage chunk c: 32 rows x 16 float4 of K and of V (four 16-byte copies a
  // thread), and 32 rows x 8 float4 of cos and of sin (one each). Always one
  // commit group per call (empty past the last chunk).
  auto stage = [&](int c) {
    if (c < nchunks) {
      float *dst = st_smem + (size_t)(c % STAGES) * kStStageFloats;
#pragma unroll
      for (int e = tid; e < 2 * kStRows * 16; e += 256) {
        const int kv = e >> 9, r = (e >> 4) & 31, q4 = e & 15;
        const int row = c * kStRows + r;
        if (row < n) cp_async16(dst + (kv * kStRows + r) * 64 + q4 * 4, kbase + (size_t)row * ld + kv * H + q4 * 4);
      }
      if (ROPE) {
        const int tab = tid >> 7, r = (tid >> 3) & 15, q4 = tid & 7;  // 2 tables x 16 rows x 8 float4, twice
#pragma unroll
        for (int half = 0; half < 2; half++) {
          const int row = c * kStRows + half * 16 + r;
          if (row < n)
            cp_async16(dst + 2 * kStRows * 64 + (tab * kStRows + half * 16 + r) * 32 + q4 * 4,
                       (tab ? rope_sin : rope_cos) + (size_t)row * 32 + q4 * 4);
        }
      }
    }
    cp_async_commit();
  };
  // Threads 64-255 on chunk c: K rotated in place (pair i, i + 32 of a row by
  // one thread, rotate_half without FMA), then the V maxima.
  float vmax = 0.0f;
  const int vd = (tid - 64) & 63, vsub = (tid - 64) >> 6;
  auto prep = [&](int c) {
    if (c >= nchunks) return;
    float *kc = st_smem + (size_t)(c % STAGES) * kStStageFloats;
    const float *vc = kc + kStRows * 64, *cc = kc + 2 * kStRows * 64, *sc = cc + kStRows * 32;
    const int rows = min(kStRows, n - c * kStRows);
    if constexpr (ROPE) {
      for (int e = tid - 64; e < rows * 32; e += 192) {
        const int r = e >> 5, i = e & 31;
        const float x1 = kc[r * 64 + i], x2 = kc[r * 64 + i + 32], cs = cc[r * 32 + i], sn = sc[r * 32 + i];
        kc[r * 64 + i] = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
        kc[r * 64 + i + 32] = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
      }
    }
    for (int r = vsub; r < rows; r += 3) vmax = fmaxf(vmax, fabsf(vc[r * 64 + vd]));
  };
  for (int c = 0; c < STAGES - 1; c++) stage(c);
  cp_async_wait_pending<STAGES - 2>();  // chunk 0 has landed
  __syncthreads();
  if (tid >= 64) prep(0);
  float acc = 0.0f;  // K sum (tid < 64)
  for (int c = 0; c < nchunks; c++) {
    cp_async_wait_pending<STAGES - 3>();  // chunk c + 1 has landed
    __syncthreads();  // chunk c rotated, chunk c - 1's slot free
    stage(c + STAGES - 1);
    if (tid < 64) {
      const float *kc = st_smem + (size_t)(c % STAGES) * kStStageFloats + tid;
      const int rows = min(kStRows, n - c * kStRows);
      if (rows == kStRows) {
#pragma unroll
        for (int r = 0; r < kStRows; r++) acc = __fadd_rn(acc, kc[r * 64]);
      } else {
        for (int r = 0; r < rows; r++) acc = __fadd_rn(acc, kc[r * 64]);
      }
    } else {
      prep(c + 1);
    }
  }
  cp_async_wait_pending<0>();
  if (tid >= 64) s_vmax[vsub][vd] = vmax;
  __syncthreads();
  if (tid < 64) {
    const size_t o = ((size_t)s * nh + h) * 64 + tid;
    kmean[o] = n > 0 ? __fmul_rn(acc, __fdiv_rn(1.0f, (float)n)) : 0.0f;
    const float mx = fmaxf(fmaxf(s_vmax[0][tid], s_vmax[1][tid]), s_vmax[2][tid]);
    const float scv = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 0.0f;
    vs[o] = scv;
    vinv[o] = mx > 0.0f ? __fdiv_rn(1.0f, scv) : 0.0f;
  }
}

// The statistics of attn_stats64_kernel with each (sequence, head) split by
// RoPE pair over 32 / P CTAs: CTA (s, h, pg) takes the pairs i in
// [pg P, pg P + P), dimensions i and 32 + i, over all the sequence's rows in
// order. A dimension's ordered K sum is one chain in one thread, so no CTA
// waits for another; the rows stream through a ring of STAGES stages of SR
// rows, each six TMA boxes [SR rows][P floats] (K and V lower and upper
// halves, cos, sin; no multicast).
//   warp 0     lane 0 issues the loads.
//   warp 1     lanes 0..2P-1: the ordered K sums, one dimension each, over
//              the rotated keys of each stage as it comes.
//   warps 2-5  rotate the stage's keys in place (rotate_half without FMA)
//              and take the V column maxima of its rows (any order).
// Per stage a full barrier (the loads), a rotated barrier (the four warps)
// and an empty barrier (the sums); every wait is bounded.
constexpr int kPgRotWarps = 4;
constexpr int kPgThreads = 64 + 32 * kPgRotWarps;

template <int P, int SR>
struct PgLayout {
  static constexpr int kBox = SR * P;          // floats per box
  static constexpr int kPitch = kBox + 32;     // box stride (128-byte aligned starts)
  static constexpr int kStage = 6 * kPitch;    // K lo, K hi, V lo, V hi, cos, sin
  static int bytes(int stages) { return stages * kStage * 4 + stages * 3 * 8 + kPgRotWarps * 2 * P * 4 + 16; }
};

template <int P, int SR, int STAGES, bool ROPE>
__global__ void __launch_bounds__(kPgThreads)
    attn_stats_pg_kernel(const __grid_constant__ CUtensorMap mqkv, const __grid_constant__ CUtensorMap mcos,
                         const __grid_constant__ CUtensorMap msin, const int32_t *__restrict__ offs, int H, int nh,
                         float *__restrict__ kmean, float *__restrict__ vs, float *__restrict__ vinv) {
  static_assert(P % 4 == 0 && 2 * P <= 32 && (32 * kPgRotWarps) % P == 0, "pair groups");
  using L = PgLayout<P, SR>;
  extern __shared__ __align__(128) float pg_smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(pg_smem + STAGES * L::kStage);
  uint64_t *rotd = full + STAGES;
  uint64_t *empty = rotd + STAGES;
  float *vred = reinterpret_cast<float *>(empty + STAGES);  // [kPgRotWarps][2P]
  const int s = blockIdx.x, h = blockIdx.y, pg = blockIdx.z;
  dep_wait();
  const int t0 = offs[s], n = offs[s + 1] - t0;
  const int nst = (n + SR - 1) / SR;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int b = 0; b < STAGES; b++) {
      mbar_init(&full[b], 1);
      mbar_init(&rotd[b], kPgRotWarps);
      mbar_init(&empty[b], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&mqkv);
      if (ROPE) {
        prefetch_tensormap(&mcos);
        prefetch_tensormap(&msin);
      }
      const int xk = H + h * 64 + pg * P, xv = 2 * H + h * 64 + pg * P;
      for (int c = 0; c < nst; c++) {
        const int b = c % STAGES;
        if (c >= STAGES && !mbar_wait(&empty[b], (uint32_t)(c / STAGES - 1) & 1, kDevTimeoutEmpty)) break;
        float *stg = pg_smem + b * L::kStage;
        mbar_arrive_expect_tx(&full[b], (ROPE ? 6 : 4) * L::kBox * 4);
        const int y = t0 + c * SR;
        tma_load_2d(&mqkv, stg, &full[b], xk, y);
        tma_load_2d(&mqkv, stg + L::kPitch, &full[b], xk + 32, y);
        tma_load_2d(&mqkv, stg + 2 * L::kPitch, &full[b], xv, y);
        tma_load_2d(&mqkv, stg + 3 * L::kPitch, &full[b], xv + 32, y);
        if (ROPE) {
          tma_load_2d(&mcos, stg + 4 * L::kPitch, &full[b], pg * P, c * SR);
          tma_load_2d(&msin, stg + 5 * L::kPitch, &full[b], pg * P, c * SR);
        }
      }
    }
  } else if (warp == 1) {
    // Lane l < P: dimension pg P + l (the K lower box), lane P + l:
    // 32 + pg P + l (the upper box).
    const bool act = lane < 2 * P;
    const int off = lane < P ? lane : L::kPitch + lane - P;
    float acc = 0.0f;
    bool ok = true;
    for (int c = 0; c < nst; c++) {
      const int b = c % STAGES;
      ok = ok && mbar_wait(&rotd[b], (uint32_t)(c / STAGES) & 1, kDevTimeoutFull);
      const float *kc = pg_smem + b * L::kStage + off;
      const int rows = min(SR, n - c * SR);
      if (act && ok) {
        if (rows == SR) {
          // Whole stage unrolled: the loads run ahead of the add chain.
#pragma unroll
          for (int r = 0; r < SR; r++) acc = __fadd_rn(acc, kc[r * P]);
        } else {
          for (int r = 0; r < rows; r++) acc = __fadd_rn(acc, kc[r * P]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[b]);
    }
    if (act) {
      const int d = lane < P ? pg * P + lane : 32 + pg * P + lane - P;
      kmean[((size_t)s * nh + h) * 64 + d] = n > 0 ? __fmul_rn(acc, __fdiv_rn(1.0f, (float)n)) : 0.0f;
    }
  } else {
    // Thread tr keeps pair i = tr % P over rows tr / P, + 128 / P, ...
    constexpr int kStep = 32 * kPgRotWarps / P;
    const int tr = threadIdx.x - 64;
    const int i = tr % P, rb = tr / P;
    float vlo = 0.0f, vhi = 0.0f;
    bool ok = true;
    for (int c = 0; c < nst; c++) {
      const int b = c % STAGES;
      ok = ok && mbar_wait(&full[b], (uint32_t)(c / STAGES) & 1, kDevTimeoutFull);
      float *stg = pg_smem + b * L::kStage;
      const int rows = ok ? min(SR, n - c * SR) : 0;
#pragma unroll 4
      for (int r = rb; r < rows; r += kStep) {
        const int o = r * P + i;
        if (ROPE) {
          const float x1 = stg[o], x2 = stg[L::kPitch + o];
          const float cs = stg[4 * L::kPitch + o], sn = stg[5 * L::kPitch + o];
          stg[o] = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
          stg[L::kPitch + o] = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
        }
        vlo = fmaxf(vlo, fabsf(stg[2 * L::kPitch + o]));
        vhi = fmaxf(vhi, fabsf(stg[3 * L::kPitch + o]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rotd[b]);
    }
    // Maxima of the lanes holding the same pair, then over the four warps.
#pragma unroll
    for (int o = P; o < 32; o <<= 1) {
      vlo = fmaxf(vlo, __shfl_xor_sync(0xffffffffu, vlo, o));
      vhi = fmaxf(vhi, __shfl_xor_sync(0xffffffffu, vhi, o));
    }
    if (lane < P) {
      vred[(warp - 2) * 2 * P + lane] = vlo;
      vred[(warp - 2) * 2 * P + P + lane] = vhi;
    }
    named_barrier_sync(1, 32 * kPgRotWarps);
    if (tr < 2 * P) {
      float mx = 0.0f;
#pragma unroll
      for (int w = 0; w < kPgRotWarps; w++) mx = fmaxf(mx, vred[w * 2 * P + tr]);
      const int d = tr < P ? pg * P + tr : 32 + pg * P + tr - P;
      const size_t o = ((size_t)s * nh + h) * 64 + d;
      const float scv = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 0.0f;
      vs[o] = scv;
      vinv[o] = mx > 0.0f ? __fdiv_rn(1.0f, scv) : 0.0f;
    }
  }
  dep_trigger();  // one wave of long-lived CTAs: the next kernel is let in at the end
}

// attn_quant_kernel for D = 64 with one warp per row over all its heads: the
// row's sequence, position and RoPE factors are read once, and successive
// heads' loads are independent. Lane l holds dimensions l and l + 32 (a
// rotate_half pair); the bytes are gathered by shuffles so that each plane's
// 64-byte row leaves in 16-bit stores. The same arithmetic as
// attn_quant_kernel / attn_prep_kernel.
__global__ void __launch_bounds__(256)
    attn_quant64_kernel(const float *__restrict__ qkv, const int32_t *__restrict__ row_seq,
                        const int32_t *__restrict__ offs, int N, int H, int nh, float scale,
                        const float *__restrict__ rope_cos, const float *__restrict__ rope_sin,
                        const float *__restrict__ kmean, const float *__restrict__ vinv, uint8_t *__restrict__ qa,
                        float *__restrict__ sq, int8_t *__restrict__ kq, float *__restrict__ ks,
                        float *__restrict__ kzc, int8_t *__restrict__ vq) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  dep_wait();
  dep_trigger();
  if (row >= N) return;
  const int s = row_seq[row];
  float c = 1.0f, sn = 0.0f;
  if (rope_cos) {
    const int pos = row - offs[s];
    c = __ldg(rope_cos + (size_t)pos * 32 + lane);
    sn = __ldg(rope_sin + (size_t)pos * 32 + lane);
  }
  const float *base = qkv + (size_t)row * 3 * H;
  // Lane m < 16 stores dimensions 2m, 2m+1; lane 16 + m dimensions 32+2m, 33+2m.
  const bool hi_half = lane >= 16;
  const int src = (2 * lane) & 31;
  const uint32_t pick = hi_half ? 0x0062u : 0x0040u;
  const int off = hi_half ? 32 + 2 * (lane - 16) : 2 * lane;
#pragma unroll 2
  for (int h = 0; h < nh; h++) {
    const float *b = base + h * 64;
    const float *km = kmean + ((size_t)s * nh + h) * 64;
    const float *vi = vinv + ((size_t)s * nh + h) * 64;
    float q1 = b[lane], q2 = b[lane + 32], k1 = b[H + lane], k2 = b[H + lane + 32];
    const float v1 = b[2 * H + lane], v2 = b[2 * H + lane + 32];
    if (rope_cos) {  // Rope (linalg/vec_simd.go:404-425): separate roundings, no FMA
      const float qa_ = q1, qb_ = q2, ka_ = k1, kb_ = k2;
      q1 = __fsub_rn(__fmul_rn(qa_, c), __fmul_rn(qb_, sn));
      q2 = __fadd_rn(__fmul_rn(qb_, c), __fmul_rn(qa_, sn));
      k1 = __fsub_rn(__fmul_rn(ka_, c), __fmul_rn(kb_, sn));
      k2 = __fadd_rn(__fmul_rn(kb_, c), __fmul_rn(ka_, sn));
    }
    k1 = __fsub_rn(k1, __ldg(km + lane));
    k2 = __fsub_rn(k2, __ldg(km + lane + 32));
    float qmx = fmaxf(fmaxf(0.0f, fabsf(q1)), fabsf(q2));
    float kmx = fmaxf(fmaxf(0.0f, fabsf(k1)), fabsf(k2));
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      qmx = fmaxf(qmx, __shfl_xor_sync(0xffffffffu, qmx, o));
      kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
    }
    // Q (attention8.go:210-220): uint8 with the 128 offset.
    const float qs = qmx > 0.0f ? __fdiv_rn(qmx, 127.0f) : 0.0f;
    const float qinv = qmx > 0.0f ? __fdiv_rn(1.0f, qs) : 0.0f;
    // K (attention8.go:240-251): centred, int8, scale and 128*sum.
    const float kss = kmx > 0.0f ? __fdiv_rn(kmx, 127.0f) : 0.0f;
    const float kinv = kmx > 0.0f ? __fdiv_rn(1.0f, kss) : 0.0f;
    int qa1 = qmx > 0.0f ? rne_int(__fmul_rn(q1, qinv)) : 0, qa2 = qmx > 0.0f ? rne_int(__fmul_rn(q2, qinv)) : 0;
    qa1 = max(-128, min(127, qa1)) + 128;
    qa2 = max(-128, min(127, qa2)) + 128;
    int kb1 = 0, kb2 = 0, ksum = 0;
    if (kmx > 0.0f) {
      kb1 = rne_int(__fmul_rn(k1, kinv));
      kb2 = rne_int(__fmul_rn(k2, kinv));
      ksum = kb1 + kb2;
      kb1 = max(-128, min(127, kb1));
      kb2 = max(-128, min(127, kb2));
    }
    const int vb1 = max(-128, min(127, rne_int(__fmul_rn(v1, __ldg(vi + lane))))),
              vb2 = max(-128, min(127, rne_int(__fmul_rn(v2, __ldg(vi + lane + 32)))));
#pragma unroll
    for (int o = 16; o; o >>= 1) ksum += __shfl_xor_sync(0xffffffffu, ksum, o);
    // Byte 0: dimension lane, byte 2: dimension lane + 32.
    const uint32_t wq = (uint32_t)qa1 | ((uint32_t)qa2 << 16);
    const uint32_t wk = ((uint32_t)kb1 & 0xFFu) | (((uint32_t)kb2 & 0xFFu) << 16);
    const uint32_t wv = ((uint32_t)vb1 & 0xFFu) | (((uint32_t)vb2 & 0xFFu) << 16);
    const uint32_t q_lo = __shfl_sync(0xffffffffu, wq, src), q_hi = __shfl_sync(0xffffffffu, wq, src + 1);
    const uint32_t k_lo = __shfl_sync(0xffffffffu, wk, src), k_hi = __shfl_sync(0xffffffffu, wk, src + 1);
    const uint32_t v_lo = __shfl_sync(0xffffffffu, wv, src), v_hi = __shfl_sync(0xffffffffu, wv, src + 1);
    const size_t plane = (size_t)h * N + row;
    *reinterpret_cast<uint16_t *>(qa + plane * 64 + off) = (uint16_t)__byte_perm(q_lo, q_hi, pick);
    *reinterpret_cast<uint16_t *>(kq + plane * 64 + off) = (uint16_t)__byte_perm(k_lo, k_hi, pick);
    *reinterpret_cast<uint16_t *>(vq + plane * 64 + off) = (uint16_t)__byte_perm(v_lo, v_hi, pick);
    if (lane == 0) {
      sq[plane] = qmx > 0.0f ? __fmul_rn(qs, scale) : 0.0f;
      ks[plane] = kss;
      kzc[plane] = kmx > 0.0f ? __fmul_rn(128.0f, (float)ksum) : 0.0f;
    }
  }
}

// attn_quant64_kernel's bytes and scales for a tile of 64 rows of one
// sequence and one head, two threads per row: the tile's Q, K and V halves
// ([64 rows][32 floats] each) and the rows' RoPE factors (positions i0..,
// contiguous within the sequence) come in by TMA, SWIZZLE_128B (no
// multicast); thread (rr, hh) holds dimensions 16hh.. and 32 + 16hh.. of row
// rr (both halves of its rotate_half pairs), so a row maximum or key sum is
// the thread's and its neighbour's (one shuffle) instead of a 32-lane
// reduction per head. Q and K take the fast byte conversion where the
// attention short kernel does (no NaN, normal scale), V the generic one, as
// attn_quant64_kernel: the same bits.
constexpr int kQtRows = 64;

template <bool ROPE>
__global__ void __launch_bounds__(2 * kQtRows)
    attn_quant_tile_kernel(const __grid_constant__ CUtensorMap mqkv, const __grid_constant__ CUtensorMap mcos,
                           const __grid_constant__ CUtensorMap msin, const int2 *__restrict__ tiles,
                           const int32_t *__restrict__ offs, int N, int H, int nh, float scale,
                           const float *__restrict__ kmean, const float *__restrict__ vinv, uint8_t *__restrict__ qa,
                           float *__restrict__ sq, int8_t *__restrict__ kq, float *__restrict__ ks,
                           float *__restrict__ kzc, int8_t *__restrict__ vq) {
  constexpr int kBox = kQtRows * 128;  // bytes of one [64 rows][32 floats] box
  extern __shared__ uint8_t qt_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(qt_raw) + 1023) & ~uintptr_t(1023));
  // Boxes: Q lo, Q hi, K lo, K hi, V lo, V hi, cos, sin.
  float *s_km = reinterpret_cast<float *>(sm + 8 * kBox);  // [64] K column means
  float *s_vi = s_km + 64;                                  // [64] V inverse scales
  uint64_t *bar = reinterpret_cast<uint64_t *>(s_vi + 64);
  dep_wait();
  dep_trigger();
  const int2 tile = tiles[blockIdx.x];
  const int s = tile.x, i0 = tile.y, h = blockIdx.y;
  const int t0 = offs[s], n = offs[s + 1] - t0;
  const int tid = threadIdx.x, rr = tid >> 1, hh = tid & 1;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (tid < 64) {
    s_km[tid] = __ldg(kmean + ((size_t)s * nh + h) * 64 + tid);
  } else {
    s_vi[tid - 64] = __ldg(vinv + ((size_t)s * nh + h) * 64 + tid - 64);
  }
  __syncthreads();
  if (tid == 0) {
    prefetch_tensormap(&mqkv);
    mbar_arrive_expect_tx(bar, (ROPE ? 8 : 6) * kBox);
    const int y = t0 + i0;
#pragma unroll
    for (int p = 0; p < 3; p++) {
      tma_load_2d(&mqkv, sm + (2 * p) * kBox, bar, p * H + h * 64, y);
      tma_load_2d(&mqkv, sm + (2 * p + 1) * kBox, bar, p * H + h * 64 + 32, y);
    }
    if (ROPE) {
      tma_load_2d(&mcos, sm + 6 * kBox, bar, 0, i0);
      tma_load_2d(&msin, sm + 7 * kBox, bar, 0, i0);
    }
  }
  const bool ok = mbar_wait(bar, 0, kDevTimeoutFull);
  const bool valid = ok && i0 + rr < n;
  // Chunk c (dimensions 4c..4c+3 of a half) of row rr in box b.
  auto chunk = [&](int b, int c) {
    return *reinterpret_cast<const float4 *>(sm + b * kBox + rr * 128 + (((c ^ (rr & 7))) << 4));
  };
  // v[0..15]: dimensions 16hh.., v[16..31]: 32 + 16hh.. of box pair p.
  auto load_pair = [&](int p, float (&v)[32]) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float4 lo = chunk(2 * p, 4 * hh + k), hi = chunk(2 * p + 1, 4 * hh + k);
      v[4 * k] = lo.x, v[4 * k + 1] = lo.y, v[4 * k + 2] = lo.z, v[4 * k + 3] = lo.w;
      v[16 + 4 * k] = hi.x, v[17 + 4 * k] = hi.y, v[18 + 4 * k] = hi.z, v[19 + 4 * k] = hi.w;
    }
  };
  auto rotate = [&](float (&v)[32]) {  // Rope (linalg/vec_simd.go:404-425): separate roundings, no FMA
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float4 c = chunk(6, 4 * hh + k), sn = chunk(7, 4 * hh + k);
      const float c4[4] = {c.x, c.y, c.z, c.w}, s4[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float a = v[4 * k + u], b = v[16 + 4 * k + u];
        v[4 * k + u] = __fsub_rn(__fmul_rn(a, c4[u]), __fmul_rn(b, s4[u]));
        v[16 + 4 * k + u] = __fadd_rn(__fmul_rn(b, c4[u]), __fmul_rn(a, s4[u]));
      }
    }
  };
  const size_t plane = (size_t)h * N + t0 + i0 + rr;
  // Q (attention8.go:210-220): uint8 q + 128, scale times the score scale.
  {
    float v[32];
    load_pair(0, v);
    if (ROPE) rotate(v);
    float m = absmax32<true>(v);  // NaN-propagating first: a NaN row takes the generic path
    m = fmax_nan(m, __shfl_xor_sync(0xffffffffu, m, 1));
    const bool nan = m != m;
    if (nan) {
      m = absmax32<false>(v);
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    }
    const float qs = m > 0.0f ? __fdiv_rn(m, 127.0f) : 0.0f;
    const float inv = m > 0.0f ? __fdiv_rn(1.0f, qs) : 0.0f;
    uint32_t w[8];
    if (m == 0.0f) {
#pragma unroll
      for (int k = 0; k < 8; k++) w[k] = 0x80808080u;
    } else if (!nan && scale_is_normal(qs)) {
#pragma unroll
      for (int k = 0; k < 8; k++) w[k] = quant4_fast(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3], f2(inv), f2(inv));
    } else {
#pragma unroll
      for (int k = 0; k < 8; k++) {
        uint32_t b[4];
#pragma unroll
        for (int u = 0; u < 4; u++) b[u] = quant_bits(__fmul_rn(v[4 * k + u], inv)) + 128u;
        w[k] = pack_low_bytes(b[0], b[1], b[2], b[3]);
      }
    }
    if (valid) {
      *reinterpret_cast<uint4 *>(qa + plane * 64 + 16 * hh) = make_uint4(w[0], w[1], w[2], w[3]);
      *reinterpret_cast<uint4 *>(qa + plane * 64 + 32 + 16 * hh) = make_uint4(w[4], w[5], w[6], w[7]);
      if (hh == 0) sq[plane] = m > 0.0f ? __fmul_rn(qs, scale) : 0.0f;
    }
  }
  // K (attention8.go:240-251): centred, int8, scale and 128 * sum of the
  // unclamped bytes; a zero row is zero bytes, scale and sum.
  {
    float v[32];
    load_pair(1, v);
    if (ROPE) rotate(v);
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const int d = 16 * hh + k;
      v[k] = __fsub_rn(v[k], s_km[d]);
      v[16 + k] = __fsub_rn(v[16 + k], s_km[32 + d]);
    }
    float m = absmax32<true>(v);
    m = fmax_nan(m, __shfl_xor_sync(0xffffffffu, m, 1));
    const bool nan = m != m;
    if (nan) {
      m = absmax32<false>(v);
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    }
    const float kss = m > 0.0f ? __fdiv_rn(m, 127.0f) : 0.0f;
    const float inv = m > 0.0f ? __fdiv_rn(1.0f, kss) : 0.0f;
    uint32_t w[8];
    int sum = 0;
    if (m == 0.0f) {
#pragma unroll
      for (int k = 0; k < 8; k++) w[k] = 0u;
    } else if (!nan && scale_is_normal(kss)) {  // bytes are q itself: summed as signed bytes
#pragma unroll
      for (int k = 0; k < 8; k++) {
        w[k] = quant4_fast_s8(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3], f2(inv), f2(inv));
        sum = dp4a_ss(w[k], 0x01010101u, sum);
      }
    } else {  // the reference's conversion (NaN -> INT_MIN, summed before the clamp)
#pragma unroll
      for (int k = 0; k < 8; k++) {
        uint32_t b[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int x = rne_int(__fmul_rn(v[4 * k + u], inv));
          sum += x;
          b[u] = (uint32_t)max(-128, min(127, x));
        }
        w[k] = pack_low_bytes(b[0], b[1], b[2], b[3]);
      }
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    if (valid) {
      *reinterpret_cast<uint4 *>(kq + plane * 64 + 16 * hh) = make_uint4(w[0], w[1], w[2], w[3]);
      *reinterpret_cast<uint4 *>(kq + plane * 64 + 32 + 16 * hh) = make_uint4(w[4], w[5], w[6], w[7]);
      if (hh == 0) {
        ks[plane] = kss;
        kzc[plane] = m > 0.0f ? __fmul_rn(128.0f, (float)sum) : 0.0f;
      }
    }
  }
  // V (attention8.go:255-269): int8 per column.
  {
    float v[32];
    load_pair(2, v);
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      uint32_t b[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int j = 4 * k + u, d = j < 16 ? 16 * hh + j : 32 + 16 * hh + j - 16;
        b[u] = quant_bits(__fmul_rn(v[j], s_vi[d]));
      }
      w[k] = pack_low_bytes(b[0], b[1], b[2], b[3]);
    }
    if (valid) {
      *reinterpret_cast<uint4 *>(vq + plane * 64 + 16 * hh) = make_uint4(w[0], w[1], w[2], w[3]);
      *reinterpret_cast<uint4 *>(vq + plane * 64 + 32 + 16 * hh) = make_uint4(w[4], w[5], w[6], w[7]);
    }
  }
}

// One warp per (row, head); D <= 128 (each lane holds D/32 values).
// With rope_cos (D = 64: lane l holds dimensions l and l + 32, a rotate_half
// pair) q and k are rotated at the row's position in its sequence first, as
// attn_prep_kernel does.
__global__ void attn_quant_kernel(const float *__restrict__ qkv, const int32_t *__restrict__ row_seq,
                                  const int32_t *__restrict__ offs, int N, int H, int nh, int D, float scale,
                                  const float *__restrict__ rope_cos, const float *__restrict__ rope_sin,
                                  const float *__restrict__ kmean, const float *__restrict__ vinv,
                                  uint8_t *__restrict__ qa, float *__restrict__ sq, int8_t *__restrict__ kq,
                                  float *__restrict__ ks, float *__restrict__ kzc, int8_t *__restrict__ vq) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (gw >= N * nh) return;
  const int row = gw / nh, h = gw % nh;
  const int s = row_seq[row];
  const float *base = qkv + (size_t)row * 3 * H + h * D;
  const size_t plane = (size_t)h * N + row;
  const float *km = kmean + ((size_t)s * nh + h) * D;
  const float *vi = vinv + ((size_t)s * nh + h) * D;
  constexpr int kMax = 4;  // D <= 128
  float qv[kMax], kv[kMax], vv[kMax];
  float qmx = 0.0f, kmx = 0.0f;
#pragma unroll
  for (int u = 0; u < kMax; u++) {
    const int d = lane + 32 * u;
    qv[u] = kv[u] = vv[u] = 0.0f;
    if (d < D) {
      qv[u] = base[d];
      kv[u] = base[H + d];
      vv[u] = base[2 * H + d];
    }
  }
  if (rope_cos) {  // Rope (linalg/vec_simd.go:404-425): separate roundings, no FMA
    const int pos = row - offs[s];
    const float c = __ldg(rope_cos + (size_t)pos * 32 + lane), sn = __ldg(rope_sin + (size_t)pos * 32 + lane);
    const float q1 = qv[0], q2 = qv[1], k1 = kv[0], k2 = kv[1];
    qv[0] = __fsub_rn(__fmul_rn(q1, c), __fmul_rn(q2, sn));
    qv[1] = __fadd_rn(__fmul_rn(q2, c), __fmul_rn(q1, sn));
    kv[0] = __fsub_rn(__fmul_rn(k1, c), __fmul_rn(k2, sn));
    kv[1] = __fadd_rn(__fmul_rn(k2, c), __fmul_rn(k1, sn));
  }
#pragma unroll
  for (int u = 0; u < kMax; u++) {
    const int d = lane + 32 * u;
    if (d < D) {
      kv[u] = __fsub_rn(kv[u], km[d]);
      qmx = fmaxf(qmx, fabsf(qv[u]));
      kmx = fmaxf(kmx, fabsf(kv[u]));
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    qmx = fmaxf(qmx, __shfl_xor_sync(0xffffffffu, qmx, o));
    kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
  }
  // Q (attention8.go:210-220): uint8 with the 128 offset.
  const float qs = qmx > 0.0f ? __fdiv_rn(qmx, 127.0f) : 0.0f;
  const float qinv = qmx > 0.0f ? __fdiv_rn(1.0f, qs) : 0.0f;
  // K (attention8.go:240-251): centred, int8, scale and 128*sum.
  const float kss = kmx > 0.0f ? __fdiv_rn(kmx, 127.0f) : 0.0f;
  const float kinv = kmx > 0.0f ? __fdiv_rn(1.0f, kss) : 0.0f;
  int ksum = 0;
#pragma unroll
  for (int u = 0; u < kMax; u++) {
    const int d = lane + 32 * u;
    if (d < D) {
      int a = qmx > 0.0f ? rne_int(__fmul_rn(qv[u], qinv)) : 0;
      a = max(-128, min(127, a));
      qa[plane * D + d] = (uint8_t)(a + 128);
      int b = 0;
      if (kmx > 0.0f) {
        b = rne_int(__fmul_rn(kv[u], kinv));
        ksum += b;
        b = max(-128, min(127, b));
      }
      kq[plane * D + d] = (int8_t)b;
      int c = rne_int(__fmul_rn(vv[u], vi[d]));
      vq[plane * D + d] = (int8_t)max(-128, min(127, c));
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ksum += __shfl_xor_sync(0xffffffffu, ksum, o);
  if (lane == 0) {
    sq[plane] = qmx > 0.0f ? __fmul_rn(qs, scale) : 0.0f;
    ks[plane] = kss;
    kzc[plane] = kmx > 0.0f ? __fmul_rn(128.0f, (float)ksum) : 0.0f;
  }
}

// Block table entry: (sequence, first query).
__global__ void __launch_bounds__(32 * kAttnWarps)
    attn_attend_kernel(const int2 *__restrict__ blocks, const int32_t *__restrict__ offs, int N, int H, int nh,
                       int D, int window, int V, int max_len, const uint8_t *__restrict__ qa,
                       const float *__restrict__ sq, const int8_t *__restrict__ kq, const float *__restrict__ ks,
                       const float *__restrict__ kzc, const int8_t *__restrict__ vq, const float *__restrict__ vs,
                       float *__restrict__ ctx) {
  extern __shared__ uint8_t attn_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int2 blk = blocks[blockIdx.x];
  const int s = blk.x, h = blockIdx.y;
  const int t0 = offs[s];
  const int n = offs[s + 1] - t0;
  float *s_buf = reinterpret_cast<float *>(attn_smem) + (size_t)warp * max_len;
  uint8_t *p_buf = attn_smem + (size_t)kAttnWarps * max_len * sizeof(float) + (size_t)warp * max_len;
  const int DW = D / 4;  // 32-bit words per row
  const size_t hbase = (size_t)h * N;
  const float *vsc = vs + ((size_t)s * nh + h) * D;

  for (int qi = 0; qi < kAttnQPerWarp; qi++) {
    const int i = blk.y + warp * kAttnQPerWarp + qi;
    if (i >= n) break;
    const size_t qrow = hbase + t0 + i;
    int js = 0, je = n;
    if (window >= 0) {
      js = max(0, i - window);
      je = min(n, i + window + 1);
    }
    const int len = je - js;
    // Scores of the valid keys, and their maximum (MaxOf).
    uint32_t qw[32];
    const uint32_t *qsrc = reinterpret_cast<const uint32_t *>(qa + qrow * D);
#pragma unroll
    for (int w = 0; w < 32; w++) qw[w] = w < DW ? __ldg(qsrc + w) : 0u;
    const float sqi = sq[qrow];
    float mx = -INFINITY;
    for (int j = js + lane; j < je; j += 32) {
      const size_t krow = hbase + t0 + j;
      const uint32_t *ksrc = reinterpret_cast<const uint32_t *>(kq + krow * D);
      int acc = 0;
#pragma unroll
      for (int w = 0; w < 32; w++)
        if (w < DW) acc = dp4a_us(qw[w], __ldg(ksrc + w), acc);
      const float sc = dequant1(acc, kzc[krow], ks[krow], sqi);
      s_buf[j] = sc;
      mx = fmaxf(mx, sc);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // exp, uint8 P and its sum (QuantizeRowU8).
    int psum = 0;
    for (int j = js + lane; j < je; j += 32) {
      const float e = exp_shift_at(s_buf[j], mx, j - js, len, V);
      const int p = rne_int(__fmul_rn(e, 255.0f));
      p_buf[j] = (uint8_t)p;
      psum += p;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    const float sp = __fdiv_rn(1.0f, (float)psum);
    __syncwarp();
    // O = P.V over the valid keys, lane d handles dimensions d, d+32, ...
    int acc[4] = {0, 0, 0, 0};
    for (int j = js; j < je; j++) {
      const int p = p_buf[j];
      const int8_t *vr = vq + (hbase + t0 + j) * D;
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int d = lane + 32 * u;
        if (d < D) acc[u] += p * (int)vr[d];
      }
    }
    __syncwarp();
    float *o = ctx + (size_t)(t0 + i) * H + h * D;
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int d = lane + 32 * u;
      if (d < D) o[d] = dequant1(acc[u], 0.0f, vsc[d], sp);
    }
  }
}

int launch_attention_two_pass(const AttnArgs &a, cudaStream_t st);

// attn_stats followed by attn_quant for one (sequence, head) in one CTA: the
// statistics pass reads the sequence's K and V columns, the quantization pass
// re-reads its Q, K and V rows while they are still in L2 (same results).
// With rope tables, q and k are first rotated (rotate_half, no FMA) at the
// row's position within its sequence, as run() does after the QKV product
// (internal/modernbert/infer.go:391-399); the K statistics use rotated keys.
__global__ void __launch_bounds__(256)
    attn_prep_kernel(const float *__restrict__ qkv, const int32_t *__restrict__ offs, int N, int H, int nh, int D,
                     float scale, const float *__restrict__ rope_cos, const float *__restrict__ rope_sin,
                     float *__restrict__ vs_out, uint8_t *__restrict__ qa, float *__restrict__ sq,
                     int8_t *__restrict__ kq, float *__restrict__ ks, float *__restrict__ kzc,
                     int8_t *__restrict__ vq) {
  __shared__ float s_mean[128], s_vinv[128];
  const int s = blockIdx.x, h = blockIdx.y;
  const int t0 = offs[s], n = offs[s + 1] - t0;
  const size_t ld = 3 * (size_t)H;
  const int tid = threadIdx.x;
  if (rope_cos) {
    // D = 64. Chunks of 64 keys: every thread loads (and rotates) K and V
    // values into shared memory, then thread d < 64 continues the ordered
    // float32 sum of dimension d and thread 64 + d the max of |v[., d]|.
    __shared__ float s_k[64][64], s_v[64][64];
    float acc = 0.0f;
    const float *kbase = qkv + (size_t)t0 * ld + H + h * 64;
    for (int c0 = 0; c0 < n; c0 += 64) {
      const int rows = min(64, n - c0);
#pragma unroll 4
      for (int e = tid; e < 64 * 64; e += 256) {
        const int r = e >> 6, d = e & 63;
        if (r < rows) {
          const float *kr = kbase + (size_t)(c0 + r) * ld;
          const int i = d & 31;
          const float a = kr[d], b = kr[d ^ 32];
          const float c = __ldg(rope_cos + (size_t)(c0 + r) * 32 + i), sn = __ldg(rope_sin + (size_t)(c0 + r) * 32 + i);
          s_k[r][d] = d < 32 ? __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn)) : __fadd_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
          s_v[r][d] = kr[H + d];
        }
      }
      __syncthreads();
      if (tid < 64) {
        for (int r = 0; r < rows; r++) acc = __fadd_rn(acc, s_k[r][tid]);
      } else if (tid < 128) {
        for (int r = 0; r < rows; r++) acc = fmaxf(acc, fabsf(s_v[r][tid - 64]));
      }
      __syncthreads();
    }
    if (tid < 64) {
      s_mean[tid] = n > 0 ? __fmul_rn(acc, __fdiv_rn(1.0f, (float)n)) : 0.0f;
    } else if (tid < 128) {
      const int d = tid - 64;
      const float sc = acc > 0.0f ? __fdiv_rn(acc, 127.0f) : 0.0f;
      vs_out[((size_t)s * nh + h) * 64 + d] = sc;
      s_vinv[d] = acc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
    }
  } else if (tid < 2 * D) {
    const bool is_k = tid < D;
    const int d = is_k ? tid : tid - D;
    const float *col = qkv + (size_t)t0 * ld + (is_k ? H : 2 * H) + h * D + d;
    float acc = 0.0f;
    int j = 0;
    if (is_k) {
      for (; j + 4 <= n; j += 4) {
        const float k0 = col[(j + 0) * ld], k1 = col[(j + 1) * ld], k2 = col[(j + 2) * ld], k3 = col[(j + 3) * ld];
        acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, k0), k1), k2), k3);
      }
      for (; j < n; j++) acc = __fadd_rn(acc, col[j * ld]);
      s_mean[d] = n > 0 ? __fmul_rn(acc, __fdiv_rn(1.0f, (float)n)) : 0.0f;
    } else {
      for (; j + 4 <= n; j += 4) {
        const float v0 = col[(j + 0) * ld], v1 = col[(j + 1) * ld], v2 = col[(j + 2) * ld], v3 = col[(j + 3) * ld];
        acc = fmaxf(fmaxf(fmaxf(fmaxf(acc, fabsf(v0)), fabsf(v1)), fabsf(v2)), fabsf(v3));
      }
      for (; j < n; j++) acc = fmaxf(acc, fabsf(col[j * ld]));
      const float sc = acc > 0.0f ? __fdiv_rn(acc, 127.0f) : 0.0f;
      vs_out[((size_t)s * nh + h) * D + d] = sc;
      s_vinv[d] = acc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
    }
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  for (int j = warp; j < n; j += 8) {
    const int row = t0 + j;
    const float *base = qkv + (size_t)row * ld + h * D;
    const size_t plane = (size_t)h * N + row;
    float qv[4], kv[4], vv[4];
    float qmx = 0.0f, kmx = 0.0f;
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int d = lane + 32 * u;
      qv[u] = kv[u] = vv[u] = 0.0f;
      if (d < D) {
        qv[u] = base[d];
        kv[u] = base[H + d];
        vv[u] = base[2 * H + d];
      }
    }
    if (rope_cos) {
      // D = 64: lane l holds dimensions l and l + 32, a rotate_half pair.
      const float c = __ldg(rope_cos + (size_t)j * 32 + lane), sn = __ldg(rope_sin + (size_t)j * 32 + lane);
      const float q1 = qv[0], q2 = qv[1], k1 = kv[0], k2 = kv[1];
      qv[0] = __fsub_rn(__fmul_rn(q1, c), __fmul_rn(q2, sn));
      qv[1] = __fadd_rn(__fmul_rn(q2, c), __fmul_rn(q1, sn));
      kv[0] = __fsub_rn(__fmul_rn(k1, c), __fmul_rn(k2, sn));
      kv[1] = __fadd_rn(__fmul_rn(k2, c), __fmul_rn(k1, sn));
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int d = lane + 32 * u;
      if (d < D) {
        kv[u] = __fsub_rn(kv[u], s_mean[d]);
        qmx = fmaxf(qmx, fabsf(qv[u]));
        kmx = fmaxf(kmx, fabsf(kv[u]));
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      qmx = fmaxf(qmx, __shfl_xor_sync(0xffffffffu, qmx, o));
      kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
    }
    const float qs = qmx > 0.0f ? __fdiv_rn(qmx, 127.0f) : 0.0f;
    const float qinv = qmx > 0.0f ? __fdiv_rn(1.0f, qs) : 0.0f;
    const float kss = kmx > 0.0f ? __fdiv_rn(kmx, 127.0f) : 0.0f;
    const float kinv = kmx > 0.0f ? __fdiv_rn(1.0f, kss) : 0.0f;
    int ksum = 0;
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int d = lane + 32 * u;
      if (d < D) {
        int a = qmx > 0.0f ? rne_int(__fmul_rn(qv[u], qinv)) : 0;
        a = max(-128, min(127, a));
        qa[plane * D + d] = (uint8_t)(a + 128);
        int b = 0;
        if (kmx > 0.0f) {
          b = rne_int(__fmul_rn(kv[u], kinv));
          ksum += b;
          b = max(-128, min(127, b));
        }
        kq[plane * D + d] = (int8_t)b;
        const int c = rne_int(__fmul_rn(vv[u], s_vinv[d]));
        vq[plane * D + d] = (int8_t)max(-128, min(127, c));
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ksum += __shfl_xor_sync(0xffffffffu, ksum, o);
    if (lane == 0) {
      sq[plane] = qmx > 0.0f ? __fmul_rn(qs, scale) : 0.0f;
      ks[plane] = kss;
      kzc[plane] = kmx > 0.0f ? __fmul_rn(128.0f, (float)ksum) : 0.0f;
    }
  }
}

// attn_prep_kernel for sequences of at most kShortSeq tokens and D = 64 with
// RoPE: the (sequence, head) slices of Q, K and V are staged once in shared
// memory with 16-byte loads, Q and K rotated there, the ordered K sum and V
// maxima read from there, and each row quantized from there (one warp per
// row). Same arithmetic, one pass over qkv.
constexpr int kShortSeq = 128;

__global__ void __launch_bounds__(256)
    attn_prep_short_kernel(const float *__restrict__ qkv, const int32_t *__restrict__ offs, int N, int H, int nh,
                           float scale, const float *__restrict__ rope_cos, const float *__restrict__ rope_sin,
                           float *__restrict__ vs_out, uint8_t *__restrict__ qa, float *__restrict__ sq,
                           int8_t *__restrict__ kq, float *__restrict__ ks, float *__restrict__ kzc,
                           int8_t *__restrict__ vq) {
  extern __shared__ float s_rows[];
  float(*s_q)[64] = reinterpret_cast<float(*)[64]>(s_rows);
  float(*s_k)[64] = reinterpret_cast<float(*)[64]>(s_rows + kShortSeq * 64);
  float(*s_v)[64] = reinterpret_cast<float(*)[64]>(s_rows + 2 * kShortSeq * 64);
  __shared__ float s_mean[64], s_vinv[64];
  const int s = blockIdx.x, h = blockIdx.y;
  const int t0 = offs[s], n = offs[s + 1] - t0;
  const size_t ld = 3 * (size_t)H;
  const int tid = threadIdx.x;
  const float *base = qkv + (size_t)t0 * ld + h * 64;
  for (int e = tid; e < n * 16; e += 256) {
    const int r = e >> 4, c = (e & 15) * 4;
    const float *row = base + (size_t)r * ld + c;
    *reinterpret_cast<float4 *>(&s_q[r][c]) = __ldg(reinterpret_cast<const float4 *>(row));
    *reinterpret_cast<float4 *>(&s_k[r][c]) = __ldg(reinterpret_cast<const float4 *>(row + H));
    *reinterpret_cast<float4 *>(&s_v[r][c]) = __ldg(reinterpret_cast<const float4 *>(row + 2 * H));
  }
  __syncthreads();
  for (int e = tid; e < n * 32; e += 256) {
    const int r = e >> 5, i = e & 31;
    const float c = __ldg(rope_cos + (size_t)r * 32 + i), sn = __ldg(rope_sin + (size_t)r * 32 + i);
    const float q1 = s_q[r][i], q2 = s_q[r][i + 32], k1 = s_k[r][i], k2 = s_k[r][i + 32];
    s_q[r][i] = __fsub_rn(__fmul_rn(q1, c), __fmul_rn(q2, sn));
    s_q[r][i + 32] = __fadd_rn(__fmul_rn(q2, c), __fmul_rn(q1, sn));
    s_k[r][i] = __fsub_rn(__fmul_rn(k1, c), __fmul_rn(k2, sn));
    s_k[r][i + 32] = __fadd_rn(__fmul_rn(k2, c), __fmul_rn(k1, sn));
  }
  __syncthreads();
  if (tid < 64) {
    // Ordered float32 sum over the keys; loads run ahead of the adds.
    float acc = 0.0f;
    int r = 0;
    for (; r + 8 <= n; r += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = s_k[r + u][tid];
#pragma unroll
      for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, v[u]);
    }
    for (; r < n; r++) acc = __fadd_rn(acc, s_k[r][tid]);
    s_mean[tid] = n > 0 ? __fmul_rn(acc, __fdiv_rn(1.0f, (float)n)) : 0.0f;
  } else if (tid < 128) {
    const int d = tid - 64;
    float mx = 0.0f;
    for (int r = 0; r < n; r++) mx = fmaxf(mx, fabsf(s_v[r][d]));
    const float sc = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 0.0f;
    vs_out[((size_t)s * nh + h) * 64 + d] = sc;
    s_vinv[d] = mx > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
  }
  __syncthreads();
  // Four rows per warp: lanes 8g..8g+7 take row j + g, eight dimensions each.
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 3, d0 = (lane & 7) * 8;
  for (int j0 = warp * 4; j0 < n; j0 += 32) {
    const int j = j0 + g;
    const bool ok = j < n;
    const int jr = ok ? j : 0;
    float qv[8], kv[8], vv[8];
    *reinterpret_cast<float4 *>(qv) = *reinterpret_cast<const float4 *>(&s_q[jr][d0]);
    *reinterpret_cast<float4 *>(qv + 4) = *reinterpret_cast<const float4 *>(&s_q[jr][d0 + 4]);
    *reinterpret_cast<float4 *>(kv) = *reinterpret_cast<const float4 *>(&s_k[jr][d0]);
    *reinterpret_cast<float4 *>(kv + 4) = *reinterpret_cast<const float4 *>(&s_k[jr][d0 + 4]);
    *reinterpret_cast<float4 *>(vv) = *reinterpret_cast<const float4 *>(&s_v[jr][d0]);
    *reinterpret_cast<float4 *>(vv + 4) = *reinterpret_cast<const float4 *>(&s_v[jr][d0 + 4]);
    float qmx = 0.0f, kmx = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; u++) {
      kv[u] = __fsub_rn(kv[u], s_mean[d0 + u]);
      qmx = fmaxf(qmx, fabsf(qv[u]));
      kmx = fmaxf(kmx, fabsf(kv[u]));
    }
#pragma unroll
    for (int o = 4; o; o >>= 1) {
      qmx = fmaxf(qmx, __shfl_xor_sync(0xffffffffu, qmx, o));
      kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
    }
    const float qs = qmx > 0.0f ? __fdiv_rn(qmx, 127.0f) : 0.0f;
    const float qinv = qmx > 0.0f ? __fdiv_rn(1.0f, qs) : 0.0f;
    const float kss = kmx > 0.0f ? __fdiv_rn(kmx, 127.0f) : 0.0f;
    const float kinv = kmx > 0.0f ? __fdiv_rn(1.0f, kss) : 0.0f;
    uint32_t qw[2] = {0, 0}, kw[2] = {0, 0}, vw[2] = {0, 0};
    int ksum = 0;
#pragma unroll
    for (int u = 0; u < 8; u++) {
      int a = 0, b = 0;
      if (qmx > 0.0f) a = max(-128, min(127, rne_int(__fmul_rn(qv[u], qinv))));
      if (kmx > 0.0f) {
        b = rne_int(__fmul_rn(kv[u], kinv));
        ksum += b;
        b = max(-128, min(127, b));
      }
      const int c = max(-128, min(127, rne_int(__fmul_rn(vv[u], s_vinv[d0 + u]))));
      qw[u >> 2] |= (uint32_t)(a + 128) << (8 * (u & 3));
      kw[u >> 2] |= (uint32_t)(b & 0xff) << (8 * (u & 3));
      vw[u >> 2] |= (uint32_t)(c & 0xff) << (8 * (u & 3));
    }
#pragma unroll
    for (int o = 4; o; o >>= 1) ksum += __shfl_xor_sync(0xffffffffu, ksum, o);
    if (ok) {
      const size_t plane = (size_t)h * N + t0 + j;
      *reinterpret_cast<uint2 *>(qa + plane * 64 + d0) = make_uint2(qw[0], qw[1]);
      *reinterpret_cast<uint2 *>(kq + plane * 64 + d0) = make_uint2(kw[0], kw[1]);
      *reinterpret_cast<uint2 *>(vq + plane * 64 + d0) = make_uint2(vw[0], vw[1]);
      if ((lane & 7) == 0) {
        sq[plane] = qmx > 0.0f ? __fmul_rn(qs, scale) : 0.0f;
        ks[plane] = kss;
        kzc[plane] = kmx > 0.0f ? __fmul_rn(128.0f, (float)ksum) : 0.0f;
      }
    }
  }
}

// IG_ATTN_PG_STATS=0 keeps one CTA per (sequence, head) for the statistics of
// long sequences (the same bits; for comparisons).
static bool pg_stats_enabled() {
  static const bool on = [] {
    const char *s = getenv("IG_ATTN_PG_STATS");
    return !(s && s[0] == '0');
  }();
  return on;
}

// attn_stats_pg_kernel over every (sequence, head, pair group) of a: eight
// pairs per CTA, 128-row stages, six in flight.
static int launch_stats_pg(const AttnArgs &a, cudaStream_t st) {
  constexpr int P = 8, SR = 128, STAGES = 6;
  auto enc = get_encode_fn();
  if (!enc) return IG_ERR_CUDA;
  CUtensorMap mq, mc, ms;
  cuuint32_t estr[2] = {1, 1};
  {
    cuuint64_t dims[2] = {(cuuint64_t)(3 * a.H), (cuuint64_t)a.N};
    cuuint64_t strides[1] = {(cuuint64_t)(3 * a.H) * sizeof(float)};
    cuuint32_t box[2] = {(cuuint32_t)P, (cuuint32_t)SR};
    if (enc(&mq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.qkv), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return IG_ERR_CUDA;
  }
  mc = mq;
  ms = mq;
  if (a.rope_cos) {
    // The factor tables [positions][32]; positions past max_len are never read.
    cuuint64_t dims[2] = {32, (cuuint64_t)a.max_len};
    cuuint64_t strides[1] = {32 * sizeof(float)};
    cuuint32_t box[2] = {(cuuint32_t)P, (cuuint32_t)SR};
    if (enc(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.rope_cos), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.rope_sin), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return IG_ERR_CUDA;
  }
  const int smem = PgLayout<P, SR>::bytes(STAGES);
  static SmemOptIn at_r, at_n;
  auto kern = a.rope_cos ? attn_stats_pg_kernel<P, SR, STAGES, true> : attn_stats_pg_kernel<P, SR, STAGES, false>;
  if ((a.rope_cos ? at_r : at_n).ensure((const void *)kern, smem) != cudaSuccess) return IG_ERR_CUDA;
  return launch_dep(kern, dim3(a.nseq, a.nh, 32 / P), kPgThreads, smem, st, mq, mc, ms, a.offs, a.H, a.nh, a.kmean,
                    a.vs, a.vinv) == cudaSuccess
             ? 0
             : IG_ERR_CUDA;
}

// IG_ATTN_QUANT_TILE=0 keeps the warp-per-row quantization (the same bits;
// for comparisons).
static bool quant_tile_enabled() {
  static const bool on = [] {
    const char *s = getenv("IG_ATTN_QUANT_TILE");
    return !(s && s[0] == '0');
  }();
  return on;
}

// Q, K, V rotation and quantization of every row of a (D = 64): by 64-row
// tiles when the plan's tiles are given and qkv suits TMA, else a warp per row.
static int launch_quant64(const AttnArgs &a, cudaStream_t st) {
  if (a.row_tiles && a.nrow_tiles > 0 && quant_tile_enabled()) {
    auto enc = get_encode_fn();
    if (!enc) return IG_ERR_CUDA;
    CUtensorMap mq, mc, ms;
    cuuint32_t estr[2] = {1, 1};
    cuuint32_t box[2] = {32, (cuuint32_t)kQtRows};
    {
      cuuint64_t dims[2] = {(cuuint64_t)(3 * a.H), (cuuint64_t)a.N};
      cuuint64_t strides[1] = {(cuuint64_t)(3 * a.H) * sizeof(float)};
      if (enc(&mq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.qkv), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return IG_ERR_CUDA;
    }
    mc = mq;
    ms = mq;
    if (a.rope_cos) {
      cuuint64_t dims[2] = {32, (cuuint64_t)a.max_len};
      cuuint64_t strides[1] = {32 * sizeof(float)};
      if (enc(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.rope_cos), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
          enc(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.rope_sin), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return IG_ERR_CUDA;
    }
    const int smem = 1024 + 8 * kQtRows * 128 + 2 * 64 * 4 + 16;
    static SmemOptIn at_r, at_n;
    auto kern = a.rope_cos ? attn_quant_tile_kernel<true> : attn_quant_tile_kernel<false>;
    if ((a.rope_cos ? at_r : at_n).ensure((const void *)kern, smem) != cudaSuccess) return IG_ERR_CUDA;
    return launch_dep(kern, dim3(a.nrow_tiles, a.nh), 2 * kQtRows, smem, st, mq, mc, ms, a.row_tiles, a.offs, a.N,
                      a.H, a.nh, a.scale, a.kmean, a.vinv, a.qa, a.sq, a.kq, a.ks, a.kzc, a.vq) == cudaSuccess
               ? 0
               : IG_ERR_CUDA;
  }
  return launch_dep(attn_quant64_kernel, (unsigned)(((long long)a.N * 32 + 255) / 256), 256, 0, st, a.qkv, a.row_seq,
                    a.offs, a.N, a.H, a.nh, a.scale, a.rope_cos, a.rope_sin, a.kmean, a.vinv, a.qa, a.sq, a.kq, a.ks,
                    a.kzc, a.vq) == cudaSuccess
             ? 0
             : IG_ERR_CUDA;
}

// ---- exact recomputation for inputs outside the fast kernels' range ----------
//
// The tensor-core attend kernels assume what finite inputs of moderate size
// guarantee: score corrections 128*sum(kq) below 2^22 (the TMEM preset
// shortcut), finite scores, and no NaN reaching ExpShift. A NaN or an infinity
// in a Q or K row, or values so large that a score overflows, breaks those,
// and the reference then does things the fast kernels do not follow: its
// float->int conversions (VCVTPS2DQ) turn NaN and out-of-range values into
// INT_MIN, which enters the key's byte sum and the row's P sum; its clamps
// (VMAXPS/VMINPS with the value second) let NaN through ExpShift; and the row
// scale 1/qsum has no guard. ig_attention runs this kernel after the fast
// ones: one CTA per (sequence, head) scans that head's Q and K values, and
// only where they are outside the range recomputes the head's prepare
// (attention8.go:203-294) and attend (attention8.go:298-376) row by row on the
// CUDA cores with the reference's conversions and orders, overwriting its ctx
// columns and quantized operands. Clean heads return after the scan.
constexpr int kExThreads = 128;

// x86 semantics of the steps that differ from CUDA's defaults: comparisons
// as clamps (NaN passes through), conversions with NaN/out of range ->
// INT_MIN, integer sums that wrap.
__device__ __forceinline__ float x86_max(float a, float b) { return a < b ? b : a; }   // std::max(a, b)
__device__ __forceinline__ float x86_min(float a, float b) { return b < a ? b : a; }   // std::min(a, b)
__device__ __forceinline__ int32_t wrap_add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }

// ExpShift's vector body (vec_simd.go:235-248) with the reference's NaN flow.
__device__ __forceinline__ float exp_body_x86(float v) {
  const bool under = v < -87.3f;
  v = x86_min(x86_max(v, -87.3f), 88.7f);
  const float n = __fsub_rn(__fmaf_rn(v, 1.44269504088896341f, 12582912.0f), 12582912.0f);
  float r = __fmaf_rn(n, -0.693359375f, v);
  r = __fmaf_rn(n, 2.12194440e-4f, r);
  float p = __fmaf_rn(r, 1.9875691500e-4f, 1.3981999507e-3f);
  p = __fmaf_rn(r, p, 8.3334519073e-3f);
  p = __fmaf_rn(r, p, 4.1665795894e-2f);
  p = __fmaf_rn(r, p, 1.6666665459e-1f);
  p = __fmaf_rn(r, p, 5.0000001201e-1f);
  const float y = __fadd_rn(__fmaf_rn(__fmul_rn(p, r), r, r), 1.0f);
  const float pw = __uint_as_float((uint32_t)wrap_add(rne_int(n), 127) << 23);
  return under ? 0.0f : __fmul_rn(y, pw);
}

// exp32 (fastmath.go:35-51) with the reference's NaN flow.
__device__ __forceinline__ float exp32_x86(float x) {
  if (x < -87.3f) return 0.0f;
  x = x86_min(x, 88.7f);
  const float n = __fsub_rn(__fadd_rn(__fmul_rn(x, 1.44269504088896341f), 12582912.0f), 12582912.0f);
  float r = __fsub_rn(x, __fmul_rn(n, 0.693359375f));
  r = __fsub_rn(r, __fmul_rn(n, -2.12194440e-4f));
  float p = 1.9875691500e-4f;
  p = __fadd_rn(__fmul_rn(p, r), 1.3981999507e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 8.3334519073e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 4.1665795894e-2f);
  p = __fadd_rn(__fmul_rn(p, r), 1.6666665459e-1f);
  p = __fadd_rn(__fmul_rn(p, r), 5.0000001201e-1f);
  const float y = __fadd_rn(__fadd_rn(__fmul_rn(__fmul_rn(p, r), r), r), 1.0f);
  return __fmul_rn(y, __uint_as_float((uint32_t)wrap_add(rne_int(n), 127) << 23));
}

// The reference's row quantization (attention8.go:210-251 through
// quantizeRow): maximum of |x - mean| skipping NaN, scale max/127, bytes
// rne(c * inv) summed before the int8 clamp. Writes D bytes (q + 128 when
// flip) unless the maximum is 0; returns the scale (0 for a zero row).
__device__ float quant_row_x86(const float *x, const float *mean, int8_t *dst, bool flip, int32_t *sum) {
  float mx = 0.0f;
  for (int d = 0; d < 64; d++) mx = x86_max(mx, fabsf(mean ? __fsub_rn(x[d], mean[d]) : x[d]));
  if (mx == 0.0f) {
    *sum = 0;
    return 0.0f;
  }
  const float scale = __fdiv_rn(mx, 127.0f), inv = __fdiv_rn(1.0f, scale);
  int32_t s = 0;
  for (int d = 0; d < 64; d++) {
    const float c = mean ? __fsub_rn(x[d], mean[d]) : x[d];
    const int32_t q = rne_int(__fmul_rn(c, inv));
    s = wrap_add(s, q);
    const int32_t qc = max(-128, min(127, q));
    dst[d] = (int8_t)(flip ? (qc ^ 0x80) : qc);
  }
  *sum = s;
  return scale;
}

__global__ void __launch_bounds__(kExThreads)
    attn_exact_kernel(const float *__restrict__ qkv, const int32_t *__restrict__ offs, int N, int H, int nh,
                      int window, int V, float scale, uint8_t *__restrict__ qa, float *__restrict__ sq,
                      int8_t *__restrict__ kq, float *__restrict__ ks, float *__restrict__ kzc,
                      int8_t *__restrict__ vq, float *__restrict__ ctx) {
  __shared__ float s_mean[64], s_vs[64], s_vinv[64], s_qmax[kExThreads / 32], s_kmax[kExThreads / 32];
  __shared__ int s_bad;
  const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = offs[s], n = offs[s + 1] - t0;
  if (n <= 0) return;
  const size_t ld = 3 * (size_t)H;
  const float *qb = qkv + (size_t)t0 * ld + h * 64, *kb = qb + H, *vb = qb + 2 * H;
  // 1. The scan: non-finite Q or K values, and the largest magnitudes.
  bool bad = false;
  float qm = 0.0f, km = 0.0f;
  for (int e = tid; e < n * 64; e += kExThreads) {
    const size_t o = (size_t)(e >> 6) * ld + (e & 63);
    const float q = qb[o], k = kb[o];
    bad |= !isfinite(q) || !isfinite(k);
    qm = fmaxf(qm, fabsf(q));
    km = fmaxf(km, fabsf(k));
  }
  for (int o = 16; o; o >>= 1) {
    qm = fmaxf(qm, __shfl_xor_sync(0xffffffffu, qm, o));
    km = fmaxf(km, __shfl_xor_sync(0xffffffffu, km, o));
  }
  bad = __any_sync(0xffffffffu, bad);
  if (tid == 0) s_bad = 0;
  __syncthreads();
  if (lane == 0) {
    s_qmax[warp] = qm;
    s_kmax[warp] = km;
    if (bad) s_bad = 1;
  }
  __syncthreads();
  if (tid == 0 && !s_bad) {
    float q = 0.0f, k = 0.0f;
    for (int w = 0; w < kExThreads / 32; w++) {
      q = fmaxf(q, s_qmax[w]);
      k = fmaxf(k, s_kmax[w]);
    }
    // |score| <= 64*128*127 * (2k/127) * (q/127) * scale; the K sum <= n*k.
    if ((double)q * (double)k * (double)scale * 130.0 >= 1e30 || (double)k * n >= 1e38) s_bad = 1;
  }
  __syncthreads();
  if (!s_bad) return;

  // 2. Prepare (attention8.go:203-294): K column means (AddTo in row order,
  // then Scale by 1/n), V column scales.
  if (tid < 64) {
    float acc = 0.0f;
    for (int r = 0; r < n; r++) acc = __fadd_rn(acc, kb[(size_t)r * ld + tid]);
    s_mean[tid] = __fmul_rn(acc, __fdiv_rn(1.0f, (float)n));
  } else {
    const int d = tid - 64;
    float m = 0.0f;
    for (int r = 0; r < n; r++) m = x86_max(m, fabsf(vb[(size_t)r * ld + d]));
    float sc = m, inv = 0.0f;
    if (m > 0.0f) {
      sc = __fdiv_rn(m, 127.0f);
      inv = __fdiv_rn(1.0f, sc);
    }
    s_vs[d] = sc;
    s_vinv[d] = inv;
  }
  __syncthreads();
  for (int r = tid; r < n; r += kExThreads) {
    const size_t plane = (size_t)h * N + t0 + r, o = (size_t)r * ld;
    int32_t sum = 0;
    int8_t *qd = reinterpret_cast<int8_t *>(qa + plane * 64);
    const float qs = quant_row_x86(qb + o, nullptr, qd, true, &sum);
    if (qs != 0.0f) {
      sq[plane] = __fmul_rn(qs, scale);
    } else {
      sq[plane] = 0.0f;
      for (int d = 0; d < 64; d++) qa[plane * 64 + d] = 128;
    }
    int8_t *kd = kq + plane * 64;
    const float kss = quant_row_x86(kb + o, s_mean, kd, false, &sum);
    if (kss != 0.0f) {
      ks[plane] = kss;
      kzc[plane] = __fmul_rn(128.0f, (float)sum);
    } else {
      ks[plane] = 0.0f;
      kzc[plane] = 0.0f;
      for (int d = 0; d < 64; d++) kd[d] = 0;
    }
    for (int d = 0; d < 64; d++)
      vq[plane * 64 + d] = (int8_t)max(-128, min(127, rne_int(__fmul_rn(vb[o + d], s_vinv[d]))));
  }
  __syncthreads();

  // 3. Attend (attention8.go:335-374), a row a thread: scores, their maximum,
  // ExpShift (V-lane body, exp32 tail), P = rne(e * 255) with its int32 sum,
  // O = P . V dequantized with 1 / qsum.
  const size_t pl0 = (size_t)h * N + t0;
  for (int i = tid; i < n; i += kExThreads) {
    int js = 0, je = n;
    if (window >= 0) {
      js = max(0, i - window);
      je = min(n, i + window + 1);
    }
    const int len = je - js, body = (len / V) * V;
    const uint32_t *qrow = reinterpret_cast<const uint32_t *>(qa + (pl0 + i) * 64);
    const float sqi = sq[pl0 + i];
    auto score = [&](int j) {
      const uint32_t *krow = reinterpret_cast<const uint32_t *>(kq + (pl0 + j) * 64);
      int32_t acc = 0;
      for (int w = 0; w < 16; w++) acc = dp4a_us(qrow[w], krow[w], acc);  // u8 x s8
      return dequant1(acc, kzc[pl0 + j], ks[pl0 + j], sqi);
    };
    float mx = -INFINITY;
    for (int j = js; j < je; j++) mx = x86_max(mx, score(j));
    int32_t oacc[64];
    for (int d = 0; d < 64; d++) oacc[d] = 0;
    int32_t qsum = 0;
    for (int j = js; j < je; j++) {
      const float v = __fsub_rn(score(j), mx);
      const float e = j - js < body ? exp_body_x86(v) : exp32_x86(v);
      const int32_t pq = rne_int(__fsub_rn(__fadd_rn(__fmul_rn(e, 255.0f), 12582912.0f), 12582912.0f));
      qsum = wrap_add(qsum, pq);
      const int32_t pb = (int32_t)(uint8_t)pq;
      const int8_t *vr = vq + (pl0 + j) * 64;
      for (int d = 0; d < 64; d++) oacc[d] += pb * (int32_t)vr[d];
    }
    const float sp = __fdiv_rn(1.0f, (float)qsum);
    float *out = ctx + (size_t)(t0 + i) * H + h * 64;
    for (int d = 0; d < 64; d++) out[d] = dequant1(oacc[d], 0.0f, s_vs[d], sp);
  }
}

int launch_attn_exact(const AttnArgs &a, cudaStream_t st) {
  if (a.nseq <= 0 || a.N <= 0) return 0;
  if (a.D != 64 || a.rope_cos || a.V < 1) return IG_ERR_UNSUPPORTED;
  attn_exact_kernel<<<dim3(a.nseq, a.nh), kExThreads, 0, st>>>(a.qkv, a.offs, a.N, a.H, a.nh, a.window, a.V,
                                                               a.scale, a.qa, a.sq, a.kq, a.ks, a.kzc, a.vq,
                                                               a.ctx);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

int launch_attention(const AttnArgs &a, cudaStream_t st) {
  if (a.rope_cos && a.D != 64) return IG_ERR_UNSUPPORTED;
  if (a.rope_cos && a.nseq > 0 && a.N > 0 && a.max_len <= kShortSeq && (a.H % 4) == 0) {
    const int smem = 3 * kShortSeq * 64 * (int)sizeof(float);
    static SmemOptIn attr;
    if (attr.ensure((const void *)attn_prep_short_kernel, smem) != cudaSuccess) return IG_ERR_CUDA;
    attn_prep_short_kernel<<<dim3(a.nseq, a.nh), 256, smem, st>>>(a.qkv, a.offs, a.N, a.H, a.nh, a.scale,
                                                                   a.rope_cos, a.rope_sin, a.vs, a.qa, a.sq, a.kq,
                                                                   a.ks, a.kzc, a.vq);
    return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
  }
  if (a.nseq > 0 && a.N > 0 && a.D == 64 && a.V >= 1 && a.max_len > kShortSeq && (a.H % 4) == 0 && a.row_seq &&
      !(reinterpret_cast<uintptr_t>(a.qkv) & 15)) {
    // Long sequences: the statistics, then the rotation and quantization.
    // From 2048 tokens the statistics of a (sequence, head) are split over
    // four CTAs by RoPE pair (few long sequences would leave most SMs idle).
    if (a.max_len >= 2048 && pg_stats_enabled()) {
      const int rc = launch_stats_pg(a, st);
      if (rc) return rc;
      return launch_quant64(a, st);
    }
    // Otherwise one CTA per (sequence, head): eight stages in flight for
    // sequences of 1024 tokens or more (one CTA per SM), three below.
    static SmemOptIn attr[4];
    const bool deep = a.max_len >= 1024;
    const int smem = (deep ? 8 : 3) * kStStageFloats * (int)sizeof(float);
    auto kern = deep ? (a.rope_cos ? attn_stats64_kernel<8, true> : attn_stats64_kernel<8, false>)
                     : (a.rope_cos ? attn_stats64_kernel<3, true> : attn_stats64_kernel<3, false>);
    if (attr[(deep ? 2 : 0) + (a.rope_cos ? 1 : 0)].ensure((const void *)kern, smem) != cudaSuccess)
      return IG_ERR_CUDA;
    if (launch_dep(kern, dim3(a.nseq, a.nh), 256, smem, st, a.qkv, a.offs, a.H, a.nh, a.rope_cos, a.rope_sin, a.kmean,
                   a.vs, a.vinv) != cudaSuccess)
      return IG_ERR_CUDA;
    return launch_quant64(a, st);
  }
  if (a.nseq > 0 && a.N > 0 && a.D <= 128 && (a.D % 4) == 0 && a.V >= 1) {
    attn_prep_kernel<<<dim3(a.nseq, a.nh), 256, 0, st>>>(a.qkv, a.offs, a.N, a.H, a.nh, a.D, a.scale, a.rope_cos,
                                                          a.rope_sin, a.vs, a.qa, a.sq, a.kq, a.ks, a.kzc, a.vq);
    return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
  }
  if (a.rope_cos) return IG_ERR_UNSUPPORTED;
  return launch_attention_two_pass(a, st);
}

int launch_attention_two_pass(const AttnArgs &a, cudaStream_t st) {
  if (a.nseq <= 0 || a.N <= 0) return 0;
  if (a.D > 128 || (a.D % 4) || a.max_len <= 0 || a.V < 1) return IG_ERR_BAD_ARG;
  const int sthreads = a.D <= 128 ? 128 : 256;
  attn_stats_kernel<<<dim3(a.nseq, a.nh), sthreads, 0, st>>>(a.qkv, a.offs, a.H, a.nh, a.D, a.kmean, a.vs, a.vinv);
  if (cudaGetLastError() != cudaSuccess) return IG_ERR_CUDA;
  const int warps = a.N * a.nh;
  attn_quant_kernel<<<(warps * 32 + 255) / 256, 256, 0, st>>>(a.qkv, a.row_seq, a.offs, a.N, a.H, a.nh, a.D,
                                                             a.scale, nullptr, nullptr, a.kmean, a.vinv, a.qa, a.sq,
                                                             a.kq, a.ks, a.kzc, a.vq);
  if (cudaGetLastError() != cudaSuccess) return IG_ERR_CUDA;
  return 0;
}

// Second half: the attend kernel over a host-built block table.
int launch_attend(const AttnArgs &a, const int2 *d_blocks, int nblocks, cudaStream_t st) {
  if (nblocks <= 0) return 0;
  const size_t smem = (size_t)kAttnWarps * a.max_len * (sizeof(float) + 1);
  if (smem > 200 * 1024) return IG_ERR_UNSUPPORTED;
  static SmemOptIn attr;
  if (smem > 48 * 1024 && attr.ensure((const void *)attn_attend_kernel, (int)smem) != cudaSuccess) return IG_ERR_CUDA;
  attn_attend_kernel<<<dim3(nblocks, a.nh), 32 * kAttnWarps, smem, st>>>(
      d_blocks, a.offs, a.N, a.H, a.nh, a.D, a.window, a.V, a.max_len, a.qa, a.sq, a.kq, a.ks, a.kzc, a.vq, a.vs,
      a.ctx);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

int attn_query_block() { return kAttnQBlock; }

}  // namespace ig
