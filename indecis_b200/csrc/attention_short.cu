// Prepare + attend in one kernel for sequences of at most 128 tokens (D = 64):
// the whole of linalg/attention8.go (Prepare, then Attend over every query)
// for one (sequence, head) per CTA, with the quantized operands built
// directly in shared memory in the tensor cores' layouts instead of a global
// round trip.
//
//   1. one thread copies the (sequence, head) slices of Q, K and V (f32) into
//      shared memory by TMA as six [128 rows][32 floats] SWIZZLE_128B boxes
//      (rows past the sequence come along and are never used) while the
//      row threads load the RoPE factors of their row;
//   A. threads 0-255, two per row (16+16 dimensions each, the halves of
//      every rotate_half pair): K rotated in place; Q rotated in registers
//      and quantized per row (uint8, q+128) into its [128][64 B] SWIZZLE_64B
//      tile over the f32 Q rows, with scale times the score scale;
//      threads 256-319: V column maxima (attention8.go:224-269);
//   B. threads 0-63: ordered float32 K column sums (the mean); threads
//      64-319: V quantized per column into its tile;
//   C. threads 0-255: K rows centred and quantized per key into its tile,
//      with the per-key scale and 128*sum(kq); rows past n are zeros;
//   D. warp 1 issues S = Q.K^T (M=128, N=128, K=64) into TMEM; warps 2-9 run
//      the softmax (MaxOf, ExpShift vector body, P = rne(e*255), the scalar-
//      tail keys recomputed by tail_fixup, sp) into P beside the Q tile; warp
//      1 issues O = P.V (V as an MN-major operand) over S's columns; warps
//      2-9 stage ctx = (float(acc)*vs)*sp in shared memory and store it with
//      row-contiguous 16-byte writes.
// Every float operation is the one attn_prep_* and attn_tc_kernel perform, in
// the same order, so the results are the same bits.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "exactmath.cuh"
#include "internal.h"

namespace ig {

constexpr int kShortN = 128;  // longest sequence this kernel takes

// Once a region's f32 rows have been read, it holds the quantized tile made
// from them; the Q region also holds P, and after O = P.V the ctx staging.
struct AttnShortSmem {
  static constexpr int kHalf = 16384;      // one [128][32 f32] SWIZZLE_128B box
  static constexpr int kQf = 0;            // f32 Q (dims 0-31, then 32-63)
  static constexpr int kKf = 32768;        // f32 K
  static constexpr int kVf = 65536;        // f32 V
  static constexpr int kQt = kQf;          // Q tile [128][64 B] SW64, uint8
  static constexpr int kP = kQf + 8192;    // P [128][128 B] SW128 (1024-aligned)
  static constexpr int kKt = kKf;          // K tile [128][64 B] SW64, int8
  static constexpr int kVt = kVf;          // V tile [128][64 B] SW64 (MN-major B operand)
  static constexpr int kO = 0;             // ctx staging [128][kOPitch] f32
  static constexpr int kOPitch = 68;       // floats; 16-byte row writes hit distinct banks
  static constexpr int kKs = 98304;        // 128 key scales
  static constexpr int kKzc = kKs + 512;   // 128 x (128*sum(kq) + 1.5*2^23)
  static constexpr int kSq = kKzc + 512;   // 128 query scales
  static constexpr int kMean = kSq + 512;  // 64
  static constexpr int kVs = kMean + 256;  // 64
  static constexpr int kVinv = kVs + 256;  // 64
  static constexpr int kRed = kVinv + 256; // 2 x 128 exchange (max, then P sums)
  static constexpr int kBar = kRed + 1024; // 4 mbarriers
  static constexpr int kTmem = kBar + 32;
  static constexpr int kTotal = kTmem + 16 + 1024;
  static_assert(kO + kShortN * kOPitch * 4 <= kKs, "ctx staging overlaps the scales");
};

// Chunk c (16 bytes: dimensions 4c..4c+3, c in 0..15) of row r of an f32
// slice staged as two SWIZZLE_128B boxes: in a 128-byte row, chunk c & 7 is
// stored at position (c & 7) ^ (r & 7).
__device__ __forceinline__ float4 *f32_chunk(uint8_t *base, int r, int c) {
  return reinterpret_cast<float4 *>(base + (c >> 3) * AttnShortSmem::kHalf + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}
__device__ __forceinline__ float f32_at(const uint8_t *base, int r, int d) {
  return *reinterpret_cast<const float *>(base + (d >> 5) * AttnShortSmem::kHalf + r * 128 +
                                          ((((d >> 2) & 7) ^ (r & 7)) << 4) + (d & 3) * 4);
}
// 16-byte chunk c (dimensions 16c..16c+15) of row r of a [rows][64 B]
// SWIZZLE_64B tile.
__device__ __forceinline__ uint4 *tile_chunk(uint8_t *base, int r, int c) {
  return reinterpret_cast<uint4 *>(base + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// rotate_half RoPE of the pair (x1, x2) = (x[i], x[i+32]) (linalg/vec_simd.go
// Rope: separate roundings, no FMA).
__device__ __forceinline__ void rope1(float &x1, float &x2, float c, float s) {
  const float a = x1, b = x2;
  x1 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  x2 = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}
__device__ __forceinline__ void rope4(float4 &lo, float4 &hi, float4 c, float4 s) {
  rope1(lo.x, hi.x, c.x, s.x);
  rope1(lo.y, hi.y, c.y, s.y);
  rope1(lo.z, hi.z, c.z, s.z);
  rope1(lo.w, hi.w, c.w, s.w);
}

// ((float(acc) - 0) * vs) * sp of an O accumulator: |acc| <= 128 keys x 255 x
// 128 < 2^22, so float(acc) comes from the 1.5*2^23 bit trick exactly.
__device__ __forceinline__ float dequant_o(uint32_t acc, float vs, float sp) {
  return __fmul_rn(__fmul_rn(__fsub_rn(magic_float((int32_t)acc), kMagic), vs), sp);
}

// The low bytes of four words as one word (byte k from word k).
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Byte of clamp(rne(x)) (two's complement) in the low byte of the result.
__device__ __forceinline__ uint32_t quant_bits(float x) {
  return __float_as_uint(__fadd_rn(fminf(fmaxf(x, -128.0f), 127.0f), kMagic));
}

__global__ void __launch_bounds__(kAtThreads, 2)
    attn_short_kernel(const __grid_constant__ CUtensorMap mqkv, const int32_t *__restrict__ offs, int H, int nh,
                      int window, int V, float scale, const float *__restrict__ rope_cos,
                      const float *__restrict__ rope_sin, float *__restrict__ ctx) {
  using S = AttnShortSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *qf = smem + S::kQf;
  uint8_t *kf = smem + S::kKf;
  uint8_t *vf = smem + S::kVf;
  float *s_ks = reinterpret_cast<float *>(smem + S::kKs);
  float *s_kzc = reinterpret_cast<float *>(smem + S::kKzc);
  float *s_sq = reinterpret_cast<float *>(smem + S::kSq);
  float *s_mean = reinterpret_cast<float *>(smem + S::kMean);
  float *s_vs = reinterpret_cast<float *>(smem + S::kVs);
  float *s_vinv = reinterpret_cast<float *>(smem + S::kVinv);
  uint64_t *bar_load = reinterpret_cast<uint64_t *>(smem + S::kBar);
  uint64_t *bar_s = bar_load + 1;
  uint64_t *bar_p = bar_load + 2;
  uint64_t *bar_o = bar_load + 3;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + S::kTmem);

  const int s = blockIdx.x, h = blockIdx.y;
  const int t0 = offs[s];
  const int n = offs[s + 1] - t0;
  if (n <= 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // 1. Slices by TMA; RoPE factors of this thread's row and dimensions.
  if (tid == 0) {
    prefetch_tensormap(&mqkv);
    mbar_init(bar_load, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_p, 32 * kAtSoftWarps);
    mbar_init(bar_o, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(bar_load, 6 * S::kHalf);
#pragma unroll
    for (int x = 0; x < 3; x++)
#pragma unroll
      for (int half = 0; half < 2; half++)
        tma_load_2d(&mqkv, smem + x * 32768 + half * S::kHalf, bar_load, x * H + h * 64 + half * 32, t0);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 128);
  // Row threads: row rr, dimension half hh = chunks 4hh..4hh+3 of each
  // 32-dimension half (dimensions 16hh..16hh+15 and 32+16hh..32+16hh+15).
  const int rr = (tid >> 1) & 127, hh = tid & 1;
  const bool rope = rope_cos != nullptr;
  float4 rc[4], rs[4];
  if (rope && tid < 256 && rr < n) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
      rc[k] = __ldg(reinterpret_cast<const float4 *>(rope_cos + (size_t)rr * 32 + 16 * hh + 4 * k));
      rs[k] = __ldg(reinterpret_cast<const float4 *>(rope_sin + (size_t)rr * 32 + 16 * hh + 4 * k));
    }
  }
  __syncthreads();  // barriers initialised
  bool ok = mbar_wait(bar_load, 0, kDevTimeoutFull);

  // A. K rotated in place; Q rotated and quantized; V column maxima.
  if (tid < 256) {
    float qv[32];  // [0,16): dimensions 16hh.., [16,32): 32+16hh..
    if (rr < n) {
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int c = 4 * hh + k;
        float4 lo = *f32_chunk(qf, rr, c), hi = *f32_chunk(qf, rr, 8 + c);
        if (rope) {
          float4 klo = *f32_chunk(kf, rr, c), khi = *f32_chunk(kf, rr, 8 + c);
          rope4(lo, hi, rc[k], rs[k]);
          rope4(klo, khi, rc[k], rs[k]);
          *f32_chunk(kf, rr, c) = klo;
          *f32_chunk(kf, rr, 8 + c) = khi;
        }
        qv[4 * k] = lo.x, qv[4 * k + 1] = lo.y, qv[4 * k + 2] = lo.z, qv[4 * k + 3] = lo.w;
        qv[16 + 4 * k] = hi.x, qv[17 + 4 * k] = hi.y, qv[18 + 4 * k] = hi.z, qv[19 + 4 * k] = hi.w;
      }
    } else {
#pragma unroll
      for (int u = 0; u < 32; u++) qv[u] = 0.0f;
    }
    float qmx = 0.0f;
#pragma unroll
    for (int u = 0; u < 32; u++) qmx = fmaxf(qmx, fabsf(qv[u]));
    qmx = fmaxf(qmx, __shfl_xor_sync(0xffffffffu, qmx, 1));
    const float qs = qmx > 0.0f ? __fdiv_rn(qmx, 127.0f) : 0.0f;
    const float qinv = qmx > 0.0f ? __fdiv_rn(1.0f, qs) : 0.0f;
    // Byte q + 128, q = clamp(rne(x * qinv)) (a zero row gives q = 0).
    uint32_t qw[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      uint32_t b[4];
#pragma unroll
      for (int u = 0; u < 4; u++) b[u] = quant_bits(__fmul_rn(qv[4 * k + u], qinv)) + 128u;
      qw[k] = pack_low_bytes(b[0], b[1], b[2], b[3]);
    }
    named_barrier_sync(2, 256);  // every f32 Q row has been read
    *tile_chunk(smem + S::kQt, rr, hh) = make_uint4(qw[0], qw[1], qw[2], qw[3]);
    *tile_chunk(smem + S::kQt, rr, 2 + hh) = make_uint4(qw[4], qw[5], qw[6], qw[7]);
    if (hh == 0) s_sq[rr] = qmx > 0.0f ? __fmul_rn(qs, scale) : 0.0f;
  } else {
    const int d = tid - 256;
    float m[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int r = 0;
    for (; r + 4 <= n; r += 4) {
#pragma unroll
      for (int u = 0; u < 4; u++) m[u] = fmaxf(m[u], fabsf(f32_at(vf, r + u, d)));
    }
    for (; r < n; r++) m[0] = fmaxf(m[0], fabsf(f32_at(vf, r, d)));
    const float mx = fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
    const float sc = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 0.0f;
    s_vs[d] = sc;
    s_vinv[d] = mx > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
  }
  __syncthreads();

  // B. K column means (ordered float32 sums over the rotated keys); V rows.
  if (tid < 64) {
    float acc = 0.0f;
    int r = 0;
    for (; r + 8 <= n; r += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = f32_at(kf, r + u, tid);
#pragma unroll
      for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, v[u]);
    }
    for (; r < n; r++) acc = __fadd_rn(acc, f32_at(kf, r, tid));
    s_mean[tid] = __fmul_rn(acc, __fdiv_rn(1.0f, (float)n));
  } else {
    const int vr = (tid - 64) >> 1, vh = tid & 1;
    uint32_t vw[8];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int c = 4 * vh + k;
      float4 lo = make_float4(0.0f, 0.0f, 0.0f, 0.0f), hi = lo;
      if (vr < n) {
        lo = *f32_chunk(vf, vr, c);
        hi = *f32_chunk(vf, vr, 8 + c);
      }
      const float4 il = *reinterpret_cast<const float4 *>(s_vinv + 4 * c);
      const float4 ih = *reinterpret_cast<const float4 *>(s_vinv + 32 + 4 * c);
      vw[k] = pack_low_bytes(quant_bits(__fmul_rn(lo.x, il.x)), quant_bits(__fmul_rn(lo.y, il.y)),
                             quant_bits(__fmul_rn(lo.z, il.z)), quant_bits(__fmul_rn(lo.w, il.w)));
      vw[4 + k] = pack_low_bytes(quant_bits(__fmul_rn(hi.x, ih.x)), quant_bits(__fmul_rn(hi.y, ih.y)),
                                 quant_bits(__fmul_rn(hi.z, ih.z)), quant_bits(__fmul_rn(hi.w, ih.w)));
    }
    named_barrier_sync(2, 256);  // every f32 V row has been read
    *tile_chunk(smem + S::kVt, vr, vh) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
    *tile_chunk(smem + S::kVt, vr, 2 + vh) = make_uint4(vw[4], vw[5], vw[6], vw[7]);
  }
  __syncthreads();

  // C. K rows: centred, x = rne(kv * kinv) (the key's sum takes x before the
  // int8 clamp; a zero row gives kinv = 0, so x = 0).
  if (tid < 256) {
    float kv[32];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int c = 4 * hh + k;
      float4 lo = make_float4(0.0f, 0.0f, 0.0f, 0.0f), hi = lo;
      if (rr < n) {
        const float4 ml = *reinterpret_cast<const float4 *>(s_mean + 4 * c);
        const float4 mh = *reinterpret_cast<const float4 *>(s_mean + 32 + 4 * c);
        lo = *f32_chunk(kf, rr, c);
        hi = *f32_chunk(kf, rr, 8 + c);
        lo = make_float4(__fsub_rn(lo.x, ml.x), __fsub_rn(lo.y, ml.y), __fsub_rn(lo.z, ml.z), __fsub_rn(lo.w, ml.w));
        hi = make_float4(__fsub_rn(hi.x, mh.x), __fsub_rn(hi.y, mh.y), __fsub_rn(hi.z, mh.z), __fsub_rn(hi.w, mh.w));
      }
      kv[4 * k] = lo.x, kv[4 * k + 1] = lo.y, kv[4 * k + 2] = lo.z, kv[4 * k + 3] = lo.w;
      kv[16 + 4 * k] = hi.x, kv[17 + 4 * k] = hi.y, kv[18 + 4 * k] = hi.z, kv[19 + 4 * k] = hi.w;
    }
    float kmx = 0.0f;
#pragma unroll
    for (int u = 0; u < 32; u++) kmx = fmaxf(kmx, fabsf(kv[u]));
    kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, 1));
    const float kss = kmx > 0.0f ? __fdiv_rn(kmx, 127.0f) : 0.0f;
    const float kinv = kmx > 0.0f ? __fdiv_rn(1.0f, kss) : 0.0f;
    uint32_t kw[8];
    int ksum = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      uint32_t b[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int x = magic_rne(__fmul_rn(kv[4 * k + u], kinv));
        ksum += x;
        b[u] = (uint32_t)max(-128, min(127, x));
      }
      kw[k] = pack_low_bytes(b[0], b[1], b[2], b[3]);
    }
    ksum += __shfl_xor_sync(0xffffffffu, ksum, 1);
    named_barrier_sync(2, 256);  // every f32 K row has been read
    *tile_chunk(smem + S::kKt, rr, hh) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
    *tile_chunk(smem + S::kKt, rr, 2 + hh) = make_uint4(kw[4], kw[5], kw[6], kw[7]);
    if (hh == 0) {
      s_ks[rr] = kss;
      s_kzc[rr] = __fadd_rn(kmx > 0.0f ? __fmul_rn(128.0f, (float)ksum) : 0.0f, kMagic);  // zcm for dequant2m
    }
  }
  fence_proxy_async_smem();  // the tiles are read by the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // D. Attend.
  if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_u8s8(128, 128);
      constexpr uint32_t idesc_o = idesc_u8s8(128, 64) | (1u << 16);  // B (V) MN-major
      const uint32_t q_base = smem_u32(smem + S::kQt), k_base = smem_u32(smem + S::kKt);
#pragma unroll
      for (int kk = 0; kk < 2; kk++)
        mma_u8s8(tmem, smem_desc_k_sw64(q_base + kk * 32), smem_desc_k_sw64(k_base + kk * 32), idesc_s, kk);
      mma_commit(bar_s);
      if (mbar_wait(bar_p, 0, kDevTimeoutEmpty)) {
        tc_fence_after();
        const uint32_t p_base = smem_u32(smem + S::kP), v_base = smem_u32(smem + S::kVt);
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
          mma_u8s8(tmem, smem_desc_k_sw128(p_base + kk * 32), smem_desc_mn_sw64(v_base + kk * 32 * 64), idesc_o,
                   kk != 0);
      }
      mma_commit(bar_o);
    }
  } else if (warp >= 2) {
    const int q = warp & 3;         // TMEM lane quarter: rows [32q, 32q+32)
    const int g = (warp - 2) >> 2;  // 16-key chunks with parity g
    const int r = q * 32 + lane;
    const bool valid = r < n;
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
    int js = 0, je = n;
    if (window >= 0) {
      js = max(0, r - window);
      je = min(n, r + window + 1);
    }
    const int len = je - js;
    const int body_end = js + (len / V) * V;
    ScoreRow w;
    w.a = valid ? js : 1 << 30;
    w.b = valid ? je : 0;
    w.t0 = valid ? body_end : 0;
    w.t1 = valid ? je : 0;
    w.sq = s_sq[r];
    const int wa = __reduce_min_sync(0xffffffffu, w.a), wb = __reduce_max_sync(0xffffffffu, w.b);
    const int ch0 = wb > 0 ? wa / 16 : 0, ch1 = wb > 0 ? (wb + 15) / 16 : 0;
    float *red = reinterpret_cast<float *>(smem + S::kRed);
    uint8_t *prow_smem = smem + S::kP + r * 128;
    ok = ok && mbar_wait(bar_s, 0, kDevTimeoutAccum);
    ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
    tc_fence_after();
    float mx = -INFINITY;
    if (ok) {
      for (int ch = ch0 + ((ch0 ^ g) & 1); ch < ch1; ch += 2) mx = chunk_max(tbase + ch * 16, ch * 16, s_kzc, s_ks, w, mx);
    }
    red[g * 128 + r] = mx;
    named_barrier_sync(1, 32 * kAtSoftWarps);
    mx = fmaxf(red[r], red[128 + r]);
    int psum = 0;
    for (int ch = g; ch < 8; ch += 2) {
      uint4 pw = make_uint4(0, 0, 0, 0);
      if (ok && ch >= ch0 && ch < ch1) pw = chunk_p(tbase + ch * 16, ch * 16, s_kzc, s_ks, w, mx, psum);
      *reinterpret_cast<uint4 *>(prow_smem + ((ch ^ (r & 7)) << 4)) = pw;
    }
    if (ok && w.t0 < w.t1)
      psum += tail_fixup(smem + S::kQt, smem + S::kKt, 8192, smem + S::kP, r, g, w.t0, w.t1, s_kzc, s_ks, w.sq, mx);
    tc_fence_before();
    fence_proxy_async_smem();
    mbar_arrive(bar_p);
    named_barrier_sync(1, 32 * kAtSoftWarps);  // every thread has read red[] (max)
    reinterpret_cast<int *>(red)[g * 128 + r] = psum;
    named_barrier_sync(1, 32 * kAtSoftWarps);
    psum = reinterpret_cast<int *>(red)[r] + reinterpret_cast<int *>(red)[128 + r];
    const float sp = psum > 0 ? __fdiv_rn(1.0f, (float)psum) : 0.0f;
    if (ok) ok = mbar_wait(bar_o, 0, kDevTimeoutAccum);
    tc_fence_after();
    uint32_t o[32];
    tmem_ld_32x32b_x32(tbase + 32 * g, o);
    tmem_ld_wait();
    // Stage the row's 32 dimensions, then copy the valid rows out with each
    // row's 256 bytes written contiguously.
    float *ostage = reinterpret_cast<float *>(smem + S::kO);
    float *orow = ostage + r * S::kOPitch + 32 * g;
    const float *vsc = s_vs + 32 * g;
#pragma unroll
    for (int d = 0; d < 32; d += 4)
      *reinterpret_cast<float4 *>(orow + d) =
          make_float4(dequant_o(o[d], vsc[d], sp), dequant_o(o[d + 1], vsc[d + 1], sp),
                      dequant_o(o[d + 2], vsc[d + 2], sp), dequant_o(o[d + 3], vsc[d + 3], sp));
    named_barrier_sync(1, 32 * kAtSoftWarps);
    if (ok) {
      for (int e = tid - 64; e < n * 16; e += 32 * kAtSoftWarps) {
        const int row = e >> 4, c4 = (e & 15) * 4;
        *reinterpret_cast<float4 *>(ctx + (size_t)(t0 + row) * H + h * 64 + c4) =
            *reinterpret_cast<const float4 *>(ostage + row * S::kOPitch + c4);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// The 16-byte row loads and stores need H a multiple of 4 and 16-byte
// aligned qkv and ctx.
bool attn_short_fits(const AttnArgs &a) {
  return a.D == 64 && a.max_len <= kShortN && (a.H % 4) == 0 && a.V >= 1 &&
         (reinterpret_cast<uintptr_t>(a.qkv) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.ctx) & 15) == 0;
}

int launch_attn_short(const AttnArgs &a, cudaStream_t st) {
  if (a.nseq <= 0 || a.N <= 0) return 0;
  if (!attn_short_fits(a)) return IG_ERR_UNSUPPORTED;
  // qkv as a [N][3H] f32 plane, copied in 32-float x 128-row SWIZZLE_128B boxes.
  auto enc = get_encode_fn();
  if (!enc) return IG_ERR_CUDA;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)3 * a.H, (cuuint64_t)a.N};
  cuuint64_t strides[1] = {(cuuint64_t)3 * a.H * sizeof(float)};
  cuuint32_t box[2] = {32, (cuuint32_t)kShortN};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.qkv), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return IG_ERR_CUDA;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnShortSmem::kTotal) !=
        cudaSuccess)
      return IG_ERR_CUDA;
    attr = true;
  }
  attn_short_kernel<<<dim3(a.nseq, a.nh), kAtThreads, AttnShortSmem::kTotal, st>>>(
      map, a.offs, a.H, a.nh, a.window, a.V, a.scale, a.rope_cos, a.rope_sin, a.ctx);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig
