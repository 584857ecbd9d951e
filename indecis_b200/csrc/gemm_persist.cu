// Persistent int8 GEMM: the same arithmetic as gemm_u8s8_kernel (gemm_i8.cu),
// organised so that memory traffic and tensor-core work overlap:
//
//   * one CTA per SM walks the output tiles (tile t, t + gridDim.x, ...);
//   * the smem ring of A/B K-blocks runs continuously across tiles;
//   * two TMEM accumulators (2 x BN columns): the MMA warp fills one while
//     the epilogue warps drain the other;
//   * the epilogue writes each warp's 32 rows x 32 columns of f32 into a
//     128-byte-swizzled staging buffer and hands it to a TMA bulk store
//     (cp.async.bulk.tensor ... bulk_group) — or a TMA reduce-add for the
//     residual stream x += dequant (the reference's accumulate store,
//     linalg/kernel_vnni_amd64.s:201-234; float addition commutes, so
//     x + v is the reference's v + x bit for bit). Double-buffered staging
//     per warp, recycled with cp.async.bulk.wait_group.read.
// Requirements (checked by the launcher): C 16-byte aligned with a row stride
// that is a multiple of 4 elements.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "exactmath.cuh"
#include "internal.h"

namespace ig {

// Epilogue warps per TMEM lane quarter: four for the GeGLU epilogue, whose
// arithmetic needs warps enough to cover its latencies; two for the plain
// stores, which are bound by the TMA store stream.
template <int EPI>
struct PEpi {
  static constexpr int kWarps = (EPI == kEpiGeglu || EPI == kEpiGegluQ || EPI == kEpiGeluTanh) ? 16 : 8;
  static constexpr int kGroups = kWarps / 4;  // warps per lane quarter
  static constexpr int kThreads = 64 + 32 * kWarps;
};

template <int BN, int EPI>
struct PGemmSmem {
  static constexpr int kEpiWarps = PEpi<EPI>::kWarps;
  // Two staging buffers per epilogue warp. The plain epilogue holds the
  // column scales in shared memory (when N <= kMaxCols); the GeGLU one, with
  // twice the warps, reads them from global memory.
  static constexpr int kStageBufs = 2;
  static constexpr int kMaxCols = (EPI == kEpiF32 || EPI == kEpiI32) ? 1024 : 0;
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // kEpiGegluQ stores its int8 rows directly (no staging) and keeps the row
  // maxima exchange: [4 warps per lane quarter][128 rows] partial maxima and
  // [2 parities][8 cluster CTAs][128 rows] pushed by the cluster's CTAs.
  static constexpr bool kQ = EPI == kEpiGegluQ;
  static constexpr int kStagingBytes = kQ ? 0 : kEpiWarps * kStageBufs * 4096;
  static constexpr int kXchBytes = kQ ? (4 * 128 + 2 * 8 * 128) * 4 + 16 : 0;
  // K is a few 128-byte blocks per tile here (hidden sizes of a few hundred),
  // so two to four stages keep the tensor cores fed.
  static constexpr int kStagesRaw = (224 * 1024 - kStagingBytes - 8 * kMaxCols - kXchBytes) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 4 ? 4 : kStagesRaw;
  static constexpr int kStaging = kStages * kStageBytes;  // per epilogue warp kStageBufs x [32 rows][128 B]
  static constexpr int kCols = kStaging + kStagingBytes;  // sb[kMaxCols], zc[kMaxCols]
  static constexpr int kXPart = kCols + 8 * kMaxCols;     // kEpiGegluQ exchange (float [4][128])
  static constexpr int kXBuf = kXPart + 4 * 128 * 4;      // float [2][8][128]
  static constexpr int kXFlag = kXBuf + 2 * 8 * 128 * 4;  // abort flag
  static constexpr int kBar = kCols + 8 * kMaxCols + kXchBytes;
  static constexpr int kTmemSlot = kBar + 8 * (2 * kStages + 6);
  static constexpr int kTotal = kTmemSlot + 16 + 1024;
  static_assert(kStages >= 2, "two stages at least");
  static_assert(kTotal <= 227 * 1024, "shared memory");
};

// Dequantized accumulators of columns j0..j0+15, the column scales read four
// at a time (sb, zc 16-byte aligned, in shared or global memory; columns past
// N read column N-1 and are clipped by the store).
__device__ __forceinline__ void dequant16(const uint32_t (&r)[16], const float *__restrict__ sb,
                                          const float *__restrict__ zc, int j0, int N, float sa, float (&o)[16]) {
  if (j0 + 16 <= N) {
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
      const float4 b = *reinterpret_cast<const float4 *>(sb + j0 + k);
      const float4 z = *reinterpret_cast<const float4 *>(zc + j0 + k);
      const float2 lo = dequant2((int32_t)r[k], (int32_t)r[k + 1], make_float2(z.x, z.y), make_float2(b.x, b.y), sa);
      const float2 hi =
          dequant2((int32_t)r[k + 2], (int32_t)r[k + 3], make_float2(z.z, z.w), make_float2(b.z, b.w), sa);
      o[k] = lo.x;
      o[k + 1] = lo.y;
      o[k + 2] = hi.x;
      o[k + 3] = hi.y;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const int j = min(j0 + k, N - 1);
      o[k] = dequant1((int32_t)r[k], zc[j], sb[j], sa);
    }
  }
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *smem_src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One warp's 32 x 32 float sub-tile: thread = row; writes the row into the
// 128-byte-swizzled staging buffer, then lane 0 issues the bulk store.
template <int NBUF>
struct StageWriter {
  uint8_t *bufs;  // NBUF 4 KB buffers, used in turn
  int count = 0;
  // The next buffer, once the bulk store that last used it has read it.
  __device__ __forceinline__ uint8_t *begin(int lane) {
    uint8_t *b = bufs + (count % NBUF) * 4096;
    if (lane == 0) bulk_wait_read<NBUF - 1>();
    __syncwarp();
    return b;
  }
  // Columns [16*half, 16*half+16) of the warp's 32-column row.
  __device__ __forceinline__ static void put_half(uint8_t *b, int lane, int half, const float (&v)[16]) {
    uint8_t *row = b + lane * 128;
#pragma unroll
    for (int j = 0; j < 4; j++)
      *reinterpret_cast<float4 *>(row + (((half * 4 + j) ^ (lane & 7)) << 4)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  __device__ __forceinline__ static void put_row(uint8_t *b, int lane, const float (&v)[32]) {
    uint8_t *row = b + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; j++)
      *reinterpret_cast<float4 *>(row + ((j ^ (lane & 7)) << 4)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  __device__ __forceinline__ void finish(const CUtensorMap *map, uint8_t *b, int lane, int col, int row0,
                                         bool reduce_add) {
    fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) {
      if (reduce_add)
        tma_reduce_add_2d(map, b, col, row0);
      else
        tma_store_2d(map, b, col, row0);
      bulk_commit();
    }
    count++;
  }
  __device__ __forceinline__ static void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
};

// v[k] + bias[j0 + k] for the 16 columns j0.. (AddTo after MatMul8N); columns
// past N read column N-1 and are clipped by the store.
__device__ __forceinline__ void add_bias16(float (&v)[16], const float *__restrict__ bias, int j0, int N) {
  if (j0 + 16 <= N) {
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
      const float4 b = __ldg(reinterpret_cast<const float4 *>(bias + j0 + k));
      v[k] = __fadd_rn(v[k], b.x);
      v[k + 1] = __fadd_rn(v[k + 1], b.y);
      v[k + 2] = __fadd_rn(v[k + 2], b.z);
      v[k + 3] = __fadd_rn(v[k + 3], b.w);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 16; k++) v[k] = __fadd_rn(v[k], __ldg(bias + min(j0 + k, N - 1)));
  }
}

// One output tile's epilogue for one warp: TMEM lane quarter at tbase (row0 its
// first row, sa the thread's row scale), column chunks g, g + GROUPS, ...
template <int BN, int EPI, int GROUPS, int NBUF>
__device__ __forceinline__ void epilogue_tile(uint32_t tbase, int n0, int N, int row0, float sa, int g, int lane,
                                              StageWriter<NBUF> &sw, const CUtensorMap *mapC, const GemmEpilogue &ep,
                                              int ep_rows) {
  constexpr int kPGroups = GROUPS;
  if constexpr (EPI == kEpiF32 || EPI == kEpiI32) {
#pragma unroll 1
    for (int c = g * 32; c < BN; c += 32 * kPGroups) {
      if (n0 + c >= N) continue;
      uint8_t *buf = sw.begin(lane);
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tbase + c + 16 * h, r);
        tmem_ld_wait();
        float v[16];
        if constexpr (EPI == kEpiI32) {
#pragma unroll
          for (int k = 0; k < 16; k++) v[k] = __int_as_float((int)r[k]);
        } else {
          dequant16(r, ep.sb, ep.zc, n0 + c + 16 * h, N, sa, v);
        }
        StageWriter<NBUF>::put_half(buf, lane, h, v);
      }
      sw.finish(mapC, buf, lane, n0 + c, row0, EPI == kEpiF32 && ep.accumulate);
    }
  } else if constexpr (EPI == kEpiF32Bias || EPI == kEpiGeluTanh) {
    // GeluTanh runs over each segment of seg_rows rows as one call: its
    // element index decides the vector body or the scalar tail.
    const long long seg_len = (long long)ep.seg_rows * N;
    const long long seg_row = (long long)((row0 + lane) % ep.seg_rows) * N;
    const long long body_end = seg_len - seg_len % ep.V;
#pragma unroll 1
    for (int c = g * 32; c < BN; c += 32 * kPGroups) {
      if (n0 + c >= N) continue;
      uint8_t *buf = sw.begin(lane);
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tbase + c + 16 * h, r);
        tmem_ld_wait();
        float v[16];
        const int j0 = n0 + c + 16 * h;
        dequant16(r, ep.sb, ep.zc, j0, N, sa, v);
        add_bias16(v, ep.bias, j0, N);
        if constexpr (EPI == kEpiGeluTanh) {
          if (seg_row + j0 + 16 <= body_end) {
#pragma unroll
            for (int k = 0; k < 16; k += 2) {
              const float2 o2 = gelu_tanh_body2(make_float2(v[k], v[k + 1]));
              v[k] = o2.x;
              v[k + 1] = o2.y;
            }
          } else {
#pragma unroll
            for (int k = 0; k < 16; k++) v[k] = gelu_tanh_at(v[k], seg_row + j0 + k, seg_len, ep.V);
          }
        }
        StageWriter<NBUF>::put_half(buf, lane, h, v);
      }
      sw.finish(mapC, buf, lane, n0 + c, row0, EPI == kEpiF32Bias && ep.accumulate);
    }
  } else if constexpr (EPI == kEpiOutlierRes) {
    // The int8 product of the rest, then this row's image's outlier terms in
    // order, then the bias; added into C (the residual) by the TMA reduce.
    const int row = row0 + lane;
    const int img = row / ep.seg_rows;
    const bool row_ok = row < ep_rows;
    const int cnt = row_ok ? __ldg(ep.nout + img) : 0;
    const float *ov = ep.outv + (size_t)row * 32;
    const float *ow = ep.outw + (size_t)img * 32 * N;
#pragma unroll 1
    for (int c = g * 32; c < BN; c += 32 * kPGroups) {
      if (n0 + c >= N) continue;
      uint8_t *buf = sw.begin(lane);
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tbase + c + 16 * h, r);
        tmem_ld_wait();
        float v[16];
        const int j0 = n0 + c + 16 * h;
        dequant16(r, ep.sb, ep.zc, j0, N, sa, v);
        for (int k = 0; k < cnt; k++) {
          const float xv = __ldg(ov + k);
          const float *wk = ow + (size_t)k * N;
          if (j0 + 16 <= N) {
#pragma unroll
            for (int t = 0; t < 16; t += 4) {
              const float4 w4 = __ldg(reinterpret_cast<const float4 *>(wk + j0 + t));
              v[t] = __fadd_rn(v[t], __fmul_rn(xv, w4.x));
              v[t + 1] = __fadd_rn(v[t + 1], __fmul_rn(xv, w4.y));
              v[t + 2] = __fadd_rn(v[t + 2], __fmul_rn(xv, w4.z));
              v[t + 3] = __fadd_rn(v[t + 3], __fmul_rn(xv, w4.w));
            }
          } else {
#pragma unroll
            for (int t = 0; t < 16; t++) v[t] = __fadd_rn(v[t], __fmul_rn(xv, __ldg(wk + min(j0 + t, N - 1))));
          }
        }
        add_bias16(v, ep.bias, j0, N);
        StageWriter<NBUF>::put_half(buf, lane, h, v);
      }
      sw.finish(mapC, buf, lane, n0 + c, row0, true);
    }
  } else if constexpr (EPI == kEpiGeglu) {
    // Tile columns [0, BN/2) are GELU inputs, [BN/2, BN) their gates.
    constexpr int H2 = BN / 2;
    const int g0 = n0 / 2;
#pragma unroll 1
    for (int c = g * 32; c < H2; c += 32 * kPGroups) {
      if (g0 + c >= ep.geglu_n) continue;
      uint8_t *buf = sw.begin(lane);
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t ra[16], rg[16];
        tmem_ld_32x32b_x16(tbase + c + 16 * h, ra);
        tmem_ld_32x32b_x16(tbase + H2 + c + 16 * h, rg);
        tmem_ld_wait();
        float a[16], gt[16];
        dequant16(ra, ep.sb, ep.zc, n0 + c + 16 * h, N, sa, a);
        dequant16(rg, ep.sb, ep.zc, n0 + H2 + c + 16 * h, N, sa, gt);
        const int i0 = g0 + c + 16 * h;  // GeGLU column of a[0]
        if (i0 + 16 <= (ep.geglu_n & ~15)) {
#pragma unroll
          for (int k = 0; k < 16; k += 2) {
            const float2 o2 = gelu_mul_fma2(make_float2(a[k], a[k + 1]), make_float2(gt[k], gt[k + 1]));
            a[k] = o2.x;
            a[k + 1] = o2.y;
          }
        } else {
#pragma unroll
          for (int k = 0; k < 16; k++) a[k] = gelu_mul_at(a[k], gt[k], i0 + k, ep.geglu_n);
        }
        StageWriter<NBUF>::put_half(buf, lane, h, a);
      }
      sw.finish(mapC, buf, lane, g0 + c, row0, false);
    }
  }
}

// kEpiGegluQ, one output tile for one epilogue warp (lane quarter q, column
// group g of four): the 32 GeGLU values of its row (as kEpiGeglu computes
// them), then the row quantized over all geglu_n columns as
// quant_rows4_kernel does (linalg/int8.go:157-191 quantizeA). The row's
// maximum is formed in three steps: each thread's |maximum| over its 32
// values (NaN-ignoring, the sign bit set when a NaN was seen: the
// NaN-propagating maximum is NaN exactly then), the four column groups of
// this CTA through shared memory, and the cluster's CTAs (one per 256-column
// tile of the same 128-row block) by asynchronous stores (st.async) into
// every CTA's exchange buffer, counted as transaction bytes on its barrier,
// which one thread of the receiving CTA arms for the tile. The TMEM
// accumulator is handed back as soon as the values are in registers.
// Returns false when a wait ran out (the caller then stops waiting).
template <int BN>
__device__ __forceinline__ bool epilogue_geglu_q(uint32_t tbase, int n0, int m0, int M, float sa, int q, int g, int lane,
                                                 const GemmEpilogue &ep, uint64_t *acce_b, float *xpart, float *xbuf,
                                                 uint64_t *xfull, int it, int csize, uint32_t rank, bool ok) {
  constexpr int H2 = BN / 2;
  const int g0 = n0 / 2, c = g * 32;
  const int r = q * 32 + lane, row = m0 + r;
  const int par = it & 1;
  // One thread arms this tile's phase for every CTA's 128 row maxima.
  if (g == 0 && q == 2 && lane == 0) mbar_arrive_expect_tx(&xfull[par], 128 * 4 * csize);
  float v[32];
#pragma unroll
  for (int h = 0; h < 2; h++) {
    uint32_t ra[16], rg[16];
    tmem_ld_32x32b_x16(tbase + c + 16 * h, ra);
    tmem_ld_32x32b_x16(tbase + H2 + c + 16 * h, rg);
    tmem_ld_wait();
    float a[16], gt[16];
    dequant16(ra, ep.sb, ep.zc, n0 + c + 16 * h, 1 << 30, sa, a);
    dequant16(rg, ep.sb, ep.zc, n0 + H2 + c + 16 * h, 1 << 30, sa, gt);
#pragma unroll
    for (int k = 0; k < 16; k += 2) {
      const float2 o2 = gelu_mul_fma2(make_float2(a[k], a[k + 1]), make_float2(gt[k], gt[k + 1]));
      v[16 * h + k] = o2.x;
      v[16 * h + k + 1] = o2.y;
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(acce_b);
  float m = 0.0f;
  bool nan = false;
#pragma unroll
  for (int k = 0; k < 32; k++) {
    m = fmaxf(m, fabsf(v[k]));
    nan |= v[k] != v[k];
  }
  xpart[g * 128 + r] = nan ? -m : m;  // -0.0 keeps the sign bit for a zero maximum
  named_barrier_sync(3, 512);
  if (g == 0) {
    float e = 0.0f;
    bool en = false;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float x = xpart[k * 128 + r];
      e = fmaxf(e, fabsf(x));
      en |= signbit(x);
    }
    e = en ? -e : e;
    float *slot = xbuf + (par * 8 + (int)rank) * 128 + r;
    for (int cr = 0; cr < csize; cr++) st_async_f32(slot, (uint32_t)cr, e, &xfull[par]);
  }
  ok = ok && mbar_wait(&xfull[par], (uint32_t)(it >> 1) & 1u, kDevTimeoutAccum);
  float mx = 0.0f;
  bool has_nan = false;
  for (int cr = 0; cr < csize; cr++) {
    const float x = xbuf[(par * 8 + cr) * 128 + r];
    mx = fmaxf(mx, fabsf(x));
    has_nan |= signbit(x);
  }
  float qs = 0.0f, qinv = 0.0f;
  if (mx > 0.0f) {
    qs = __fdiv_rn(mx, 127.0f);
    qinv = __fdiv_rn(1.0f, qs);
  }
  const bool fast = !has_nan && row_scale_normal(qs);
  uint32_t w[8];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const float *x4 = v + 4 * k;
    if (mx == 0.0f) {
      w[k] = 0x80808080u;
    } else if (fast) {
      const float2 p0 = __fmul2_rn(make_float2(x4[0], x4[1]), f2(qinv));
      const float2 p1 = __fmul2_rn(make_float2(x4[2], x4[3]), f2(qinv));
      const uint32_t b0 = __float_as_uint(__fadd_rn(p0.x, kMagic + 128.0f));
      const uint32_t b1 = __float_as_uint(__fadd_rn(p0.y, kMagic + 128.0f));
      const uint32_t b2 = __float_as_uint(__fadd_rn(p1.x, kMagic + 128.0f));
      const uint32_t b3 = __float_as_uint(__fadd_rn(p1.y, kMagic + 128.0f));
      w[k] = __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
    } else {
      w[k] = quant_byte_slow(x4[0], qinv) | (quant_byte_slow(x4[1], qinv) << 8) |
             (quant_byte_slow(x4[2], qinv) << 16) | (quant_byte_slow(x4[3], qinv) << 24);
    }
  }
  if (ok && row < M) {
    uint4 *dst = reinterpret_cast<uint4 *>(ep.q_out + (size_t)row * ep.ldq + g0 + c);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    if (rank == 0 && g == 0) ep.sa_out[row] = qs;
  }
  return ok;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(PEpi<EPI>::kThreads, 1)
    gemm_persist_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                        const __grid_constant__ CUtensorMap mapC, int M, int N, int K, GemmEpilogue ep) {
  using S = PGemmSmem<BN, EPI>;
  constexpr int kStages = S::kStages;
  constexpr int kPGroups = PEpi<EPI>::kGroups;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::kBar);
  uint64_t *empty = full + kStages;
  uint64_t *accf = empty + kStages;
  uint64_t *acce = accf + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + S::kTmemSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = (N + BN - 1) / BN;
  const int ntiles = ((M + kBM - 1) / kBM) * tiles_n;
  const int num_kb = (K + kBK - 1) / kBK;

  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&mapA);
    prefetch_tensormap(&mapB);
    prefetch_tensormap(&mapC);
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], PEpi<EPI>::kWarps);
    }
    if constexpr (S::kQ) {
      // Each phase of a row-maximum exchange barrier completes when this
      // CTA has armed it and the 128 row maxima of every CTA of the cluster
      // (one per column tile) have landed.
      for (int b = 0; b < 2; b++) mbar_init(&acce[2 + b], 1);
      *reinterpret_cast<volatile int *>(smem + S::kXFlag) = 0;
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // The cluster's barriers are initialised before any CTA arrives on them.
  if constexpr (S::kQ) cluster_sync_all();
  const uint32_t tmem = *tmem_slot;
  // Everything above touches no global memory an earlier kernel writes.
  dep_wait();

  if (warp == 0) {
    if (lane == 0) {
      int kbg = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int m0 = (t / tiles_n) * kBM, n0 = (t % tiles_n) * BN;
        for (int kb = 0; kb < num_kb; kb++, kbg++) {
          const int s = kbg % kStages;
          const uint32_t ph = (kbg / kStages) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t *a = smem + s * S::kStageBytes;
          mbar_arrive_expect_tx(&full[s], S::kStageBytes);
          tma_load_2d(&mapA, a, &full[s], kb * kBK, m0);
          tma_load_2d(&mapB, a + S::kABytes, &full[s], kb * kBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_u8s8(kBM, BN);
      int kbg = 0, it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, it++) {
        const int b = it & 1;
        const uint32_t u = (uint32_t)(it >> 1);
        if (!mbar_wait(&acce[b], (u & 1) ^ 1, kDevTimeoutEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * BN;
        for (int kb = 0; kb < num_kb; kb++, kbg++) {
          const int s = kbg % kStages;
          const uint32_t ph = (kbg / kStages) & 1;
          if (!mbar_wait(&full[s], ph, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * S::kStageBytes);
          const uint32_t b_base = a_base + S::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 32; kk++)
            mma_u8s8(d, smem_desc_k_sw128(a_base + kk * 32), smem_desc_k_sw128(b_base + kk * 32), idesc,
                     (kb | kk) != 0);
          mma_commit(&empty[s]);
        }
        mma_commit(&accf[b]);
      }
    }
  } else {
    const int q = warp & 3;            // TMEM lane quarter
    const int e = warp - 2;            // epilogue warp 0..7
    const int g = e >> 2;              // column chunks g, g + kPGroups, ...
    StageWriter<S::kStageBufs> sw{smem + S::kStaging + e * S::kStageBufs * 4096};
    // The column scales in shared memory, once per CTA.
    GemmEpilogue eps = ep;
    if (N <= S::kMaxCols && EPI == kEpiF32) {
      float *s_sb = reinterpret_cast<float *>(smem + S::kCols), *s_zc = s_sb + S::kMaxCols;
      for (int j = threadIdx.x - 64; j < N; j += 32 * PEpi<EPI>::kWarps) {
        s_sb[j] = __ldg(ep.sb + j);
        s_zc[j] = __ldg(ep.zc + j);
      }
      named_barrier_sync(2, 32 * PEpi<EPI>::kWarps);
      eps.sb = s_sb;
      eps.zc = s_zc;
    }
    int it = 0;
    if constexpr (S::kQ) {
      // Every epilogue warp takes part in every tile's exchange (named
      // barrier, cluster barrier phases) whatever happens, so a wait that ran
      // out only sets the abort flag: later tiles skip their waits.
      volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + S::kXFlag);
      float *xpart = reinterpret_cast<float *>(smem + S::kXPart);
      float *xbuf = reinterpret_cast<float *>(smem + S::kXBuf);
      const uint32_t rank = cluster_ctarank();
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, it++) {
        const int m0 = (t / tiles_n) * kBM, n0 = (t % tiles_n) * BN;
        const int b = it & 1;
        const uint32_t u = (uint32_t)(it >> 1);
        bool ok = *abort_flag == 0 && mbar_wait(&accf[b], u & 1, kDevTimeoutAccum);
        tc_fence_after();
        const int row = m0 + q * 32 + lane;
        const float sa = row < M ? __ldg(ep.sa + row) : 0.0f;
        const uint32_t tbase = tmem + b * BN + ((uint32_t)(q * 32) << 16);
        ok = epilogue_geglu_q<BN>(tbase, n0, m0, M, sa, q, g, lane, ep, &acce[b], xpart, xbuf, acce + 2, it, tiles_n,
                                  rank, ok);
        if (!ok) *abort_flag = 1;
      }
    }
    for (int t = blockIdx.x; t < ntiles && !S::kQ; t += gridDim.x, it++) {
      const int m0 = (t / tiles_n) * kBM, n0 = (t % tiles_n) * BN;
      const int b = it & 1;
      const uint32_t u = (uint32_t)(it >> 1);
      if (!mbar_wait(&accf[b], u & 1, kDevTimeoutAccum)) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < M;
      const int row0 = m0 + q * 32;
      const uint32_t tbase = tmem + b * BN + ((uint32_t)(q * 32) << 16);
      const float sa = (EPI != kEpiI32 && row_ok) ? __ldg(ep.sa + row) : 0.0f;
      epilogue_tile<BN, EPI, kPGroups, S::kStageBufs>(tbase, n0, N, row0, sa, g, lane, sw, &mapC, eps, M);
      // This accumulator buffer is drained: hand it back to the MMA warp.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  // The next kernel is scheduled once every CTA is here: a persistent grid
  // that let it in at its start would have it wait on the SMs all along.
  dep_trigger();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
  // No CTA leaves while another may still write its exchange buffer.
  if constexpr (S::kQ) cluster_sync_all();
}

// f32 (or int32) output [rows][cols] with row stride ld elements: TMA boxes of
// 32 rows x 32 columns (128-byte rows, 128-byte swizzle).
static int make_map_out32(CUtensorMap *map, const void *base, int rows, int cols, int ld, bool is_int) {
  auto enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, is_int ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

static int num_sms() {
  static PerDevice sms;
  return sms.get([] {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  });
}

template <int BN, int EPI>
static cudaError_t launch_persist(const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &mc, int M, int N,
                                  int K, const GemmEpilogue &ep, cudaStream_t st) {
  using S = PGemmSmem<BN, EPI>;
  static SmemOptIn attr;
  cudaError_t e = attr.ensure((const void *)gemm_persist_kernel<BN, EPI>, S::kTotal);
  if (e != cudaSuccess) return e;
  const int tiles_n = (N + BN - 1) / BN, mblocks = (M + kBM - 1) / kBM;
  const int ntiles = mblocks * tiles_n;
  if constexpr (S::kQ) {
    // One cluster of tiles_n CTAs per 128-row block at a time: the grid is a
    // whole number of clusters, so CTA rank r always takes column tile r. A
    // persistent grid must be resident all at once: clusters of one-CTA-per-SM
    // blocks fit the GPCs only so many times (SMs left over in a GPC take
    // none), so the cluster count comes from the occupancy query.
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(PEpi<EPI>::kThreads);
    cfg.dynamicSmemBytes = S::kTotal;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = tiles_n;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(tiles_n * (num_sms() / tiles_n));
    static PerDevice resident_by_size[9];
    const int resident = resident_by_size[tiles_n].get([&] {
      int r = 0;
      if (cudaOccupancyMaxActiveClusters(&r, (const void *)gemm_persist_kernel<BN, EPI>, &cfg) != cudaSuccess ||
          r < 1) {
        cudaGetLastError();
        r = num_sms() / tiles_n / 2;
      }
      return r;
    });
    int clusters = resident < mblocks ? resident : mblocks;
    if (clusters < 1) clusters = 1;
    cfg.gridDim = dim3(clusters * tiles_n);
    add_dep_attr(at, cfg.numAttrs);
    return cudaLaunchKernelEx(&cfg, gemm_persist_kernel<BN, EPI>, ma, mb, mc, M, N, K, ep);
  }
  const int grid = ntiles < num_sms() ? ntiles : num_sms();
  return launch_dep(gemm_persist_kernel<BN, EPI>, grid, PEpi<EPI>::kThreads, S::kTotal, st, ma, mb, mc, M, N, K, ep);
}

// kEpiGegluQ needs whole 128-column GeGLU tiles (so each CTA's columns are
// all valid), at most 8 tiles (a portable cluster), and 16-byte row pieces.
bool gemm_geglu_q_fits(int N, const GemmEpilogue &ep) {
  return ep.geglu_n > 0 && ep.geglu_n % 128 == 0 && N == 2 * ep.geglu_n && N / 256 <= 8 && ep.q_out &&
         ep.sa_out && ep.ldq >= ep.geglu_n && ep.ldq % 16 == 0 && (reinterpret_cast<uintptr_t>(ep.q_out) & 15) == 0;
}

// The CTA-pair kernel (gemm_pair.cu) for deep products with 256-column
// tiles; -1 when it is not taken.
static int gemm_pair_try(const GemmArgs &g, const GemmEpilogue &ep, int epi, const CUtensorMap &ma,
                         const CUtensorMap &mc, cudaStream_t st);

// Persistent path when the output suits TMA stores; returns -1 to ask the
// caller for the plain kernel.
static int gemm_persist_try(const GemmArgs &g, const GemmEpilogue &ep, int epi, int bn, const CUtensorMap &ma,
                            const CUtensorMap &mb, cudaStream_t st) {
  if (epi == kEpiGegluQ) {
    // No float output: the quantized rows are stored by the epilogue itself.
    if (bn != 256 || !gemm_geglu_q_fits(g.N, ep) ||
        ((reinterpret_cast<uintptr_t>(ep.sb) | reinterpret_cast<uintptr_t>(ep.zc)) & 15))
      return IG_ERR_UNSUPPORTED;
    const cudaError_t e = launch_persist<256, kEpiGegluQ>(ma, mb, mb, g.M, g.N, g.K, ep, st);
    return e == cudaSuccess ? 0 : IG_ERR_CUDA;
  }
  void *out = epi == kEpiI32 ? (void *)ep.acc_out : (void *)ep.C;
  if (!out || (reinterpret_cast<uintptr_t>(out) & 15) || (ep.ldc & 3)) return -1;
  if (epi != kEpiI32 && ((reinterpret_cast<uintptr_t>(ep.sb) | reinterpret_cast<uintptr_t>(ep.zc)) & 15)) return -1;
  if (epi == kEpiF32Bias || epi == kEpiGeluTanh || epi == kEpiOutlierRes) {
    if (!ep.bias || (reinterpret_cast<uintptr_t>(ep.bias) & 15)) return IG_ERR_BAD_ARG;
    if (epi == kEpiGeluTanh && (ep.seg_rows < 1 || ep.V < 1)) return IG_ERR_BAD_ARG;
    if (epi == kEpiOutlierRes &&
        (ep.seg_rows < 1 || !ep.nout || !ep.outv || !ep.outw || (reinterpret_cast<uintptr_t>(ep.outw) & 15) ||
         (g.N & 3)))
      return IG_ERR_BAD_ARG;
  }
  const int out_cols = epi == kEpiGeglu ? ep.geglu_n : g.N;
  CUtensorMap mc;
  if (make_map_out32(&mc, out, g.M, out_cols, ep.ldc, epi == kEpiI32)) return IG_ERR_CUDA;
  if (bn == 256) {
    const int prc = gemm_pair_try(g, ep, epi, ma, mc, st);
    if (prc != -1) return prc;
  }
  cudaError_t e;
#define IG_PCASE(E)                                                                         \
  case E:                                                                                   \
    e = bn == 256 ? launch_persist<256, E>(ma, mb, mc, g.M, g.N, g.K, ep, st)               \
                  : launch_persist<128, E>(ma, mb, mc, g.M, g.N, g.K, ep, st);              \
    break;
  switch (epi) {
    IG_PCASE(kEpiF32)
    IG_PCASE(kEpiI32)
    IG_PCASE(kEpiF32Bias)
    IG_PCASE(kEpiGeluTanh)
    IG_PCASE(kEpiOutlierRes)
    case kEpiGeglu:
      e = launch_persist<256, kEpiGeglu>(ma, mb, mc, g.M, g.N, g.K, ep, st);
      break;
    default:
      return IG_ERR_BAD_ARG;
  }
#undef IG_PCASE
  return e == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig
