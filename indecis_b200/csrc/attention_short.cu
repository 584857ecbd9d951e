// Prepare + attend in one kernel for sequences of at most 128 tokens (D = 64):
// the whole of linalg/attention8.go (Prepare, then Attend over every query)
// for one (sequence, head) per CTA, with the quantized operands built
// directly in shared memory in the tensor cores' layouts instead of a global
// round trip. 8 warps and 73 KB of shared memory, so three CTAs share an SM
// and one CTA's waits are covered by the others' work. The variant that also
// computes the QKV projection (QKV below) stages the cos/sin rows of
// positions 0..127 as well (105 KB, two CTAs per SM with up to 128 registers
// a thread): per-row RoPE loads from L2, which the 28 KB of L1 left beside
// three CTAs could not hold, cost it 17% of its time.
//
// Threads work on rows in pairs: row rr = tid/2, and thread tid&1 takes
// dimensions 16hh..16hh+15 and 32+16hh..32+16hh+15 (hh = tid&1), so both
// halves of every rotate_half pair are in one thread.
//   1. one thread copies the (sequence, head) slices of K and V (f32) into
//      shared memory by TMA as four [128 rows][32 floats] SWIZZLE_128B boxes
//      (rows past the sequence come along and are never used); every thread
//      loads its Q row half and RoPE factors from global memory, rotates and
//      quantizes Q per row (uint8, q+128; scale times the score scale kept);
//   A. K rotated in place;
//   B. warps 0-1: ordered float32 K column sums (the mean); warps 2-3: V
//      column maxima (attention8.go:224-269), after which warps 4-7 quantize
//      V per column, a row each, while the K sums run;
//   C. K rows centred and quantized per key (scale, 128*sum(kq)); the K, Q
//      and V tiles ([128][64 B] SWIZZLE_64B; rows past n: zeros, Q 128s) are
//      written over the f32 rows once all have been read;
//   D. warp 0 issues S = Q.K^T (M=128, N=128, K=64) into TMEM; all 8 warps
//      run the softmax (MaxOf, ExpShift vector body, P = rne(e*255), the
//      scalar-tail keys recomputed by tail_fixup, sp) into P; warp 0 issues
//      O = P.V (V as an MN-major operand) over S's columns; the warps stage
//      ctx = (float(acc)*vs)*sp in shared memory and store it with
//      row-contiguous 16-byte writes; or, launched as one cluster per
//      sequence, quantize ctx per row over the cluster's heads (row maxima
//      pushed to every CTA of the cluster through shared memory) and store the int8 row
//      pieces and the row scales instead.
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

constexpr int kShortThreads = 256;
// CTAs per SM: three for the plain kernel; two for the projecting one, whose
// shared memory also holds the RoPE rows (and whose threads may then hold 128
// registers).
constexpr int kShortCtasPerSm = 3;
constexpr int kShortProjCtasPerSm = 2;

// Once a region's f32 rows have been read it holds the quantized tiles; after
// O = P.V the K region and the start of the V region hold the ctx staging.
struct AttnShortSmem {
  static constexpr int kHalf = 16384;       // one [128][32 f32] SWIZZLE_128B box
  static constexpr int kKf = 0;             // f32 K (dims 0-31, then 32-63)
  static constexpr int kVf = 32768;         // f32 V
  static constexpr int kKt = kKf;           // K tile [128][64 B] SW64, int8
  static constexpr int kQt = kKf + 8192;    // Q tile [128][64 B] SW64, uint8
  static constexpr int kP = kKf + 16384;    // P [128][128 B] SW128 (1024-aligned)
  static constexpr int kVt = kVf;           // V tile [128][64 B] SW64 (MN-major B operand)
  static constexpr int kRed = kVf + 8192;   // 2 x 128 exchange (max, then P sums)
  static constexpr int kO = 0;              // ctx staging [128][kOPitch] f32
  static constexpr int kOPitch = 68;        // floats; 16-byte row writes hit distinct banks
  static constexpr int kKs = 65536;         // 128 key scales
  static constexpr int kKzc = kKs + 512;    // 128 x (128*sum(kq) + 1.5*2^23)
  static constexpr int kSq = kKzc + 512;    // 128 query scales
  static constexpr int kMean = kSq + 512;   // 64
  static constexpr int kVs = kMean + 256;   // 64
  static constexpr int kVinv = kVs + 256;   // 64
  static constexpr int kBar = kVinv + 256;  // 6 mbarriers
  static constexpr int kTmem = kBar + 48;   // TMEM base address; V fast-path flag at +4
  static constexpr int kXch = kTmem + 16;   // [8][128] row maxima of the cluster's CTAs (ctx quantization)
  // Fused projection: the head's 192 column scales and zero corrections
  // (Q, K, V columns), staged once; the Q row half-maxima [2][128] use the
  // key scale region, which is written only later.
  static constexpr int kWsb = kXch + 8 * 128 * 4;
  static constexpr int kWzc = kWsb + 192 * 4;
  static constexpr int kQx = kKs;
  static constexpr int kTotal = kWzc + 192 * 4 + 1024;
  // The projecting kernel: the cos and sin rows of positions 0..127
  // ([128][32 f32] each, SWIZZLE_128B), read by the Q and K rotations.
  static constexpr int kRope = ((kWzc + 192 * 4 + 1023) / 1024) * 1024;
  static constexpr int kTotalProj = kRope + 2 * 16384 + 1024;
  static_assert(kKs + 1024 <= kSq, "Q half-maxima overlap the query scales");
  // Fused projection: the operands of the Q product (A = the sequence's
  // quantized rows, [128][128 B] SWIZZLE_128B per 128-byte K block; B = the
  // head's 64 Q weight rows) and then of the K|V product (B = its 64 K and
  // 64 V weight rows, [128][128 B] per K block, over the Q weights) lie where
  // the f32 K and V slices go once the products have read them.
  static constexpr int kA = 0;
  static constexpr int kB = 32768;
  static_assert(kO + 128 * kOPitch * 4 <= kRed, "ctx staging overlaps the exchange");
  static_assert(kShortCtasPerSm * (kTotal + 1024) <= 228 * 1024, "three CTAs per SM");
  static_assert(kShortProjCtasPerSm * (kTotalProj + 1024) <= 228 * 1024, "two CTAs per SM");
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


// The rare branches of the row quantizations (a NaN in the row, or a scale
// that is not a normal float) out of line, so that the kernel's hot code
// stays small: the reference's conversion, byte by byte.
struct Words8 {
  uint32_t w[8];
  int sum;  // quant32_s8_slow: the running sum
};
struct Vals32 {
  float4 v[8];
};
// Bytes q + 128 of 32 values.
__device__ __noinline__ Words8 quant32_u8_slow(Vals32 x, float inv) {
  Words8 r;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const float4 a = x.v[k];
    r.w[k] = pack_low_bytes(quant_bits(__fmul_rn(a.x, inv)) + 128u, quant_bits(__fmul_rn(a.y, inv)) + 128u,
                            quant_bits(__fmul_rn(a.z, inv)) + 128u, quant_bits(__fmul_rn(a.w, inv)) + 128u);
  }
  return r;
}
// int8 bytes of 32 values and sum plus their unclamped conversions.
__device__ __noinline__ Words8 quant32_s8_slow(Vals32 x, float inv, int sum) {
  Words8 r;
  int s = sum;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const float4 a = x.v[k];
    const float e[4] = {a.x, a.y, a.z, a.w};
    uint32_t b[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int q = rne_int(__fmul_rn(e[u], inv));
      s += q;
      b[u] = (uint32_t)max(-128, min(127, q));
    }
    r.w[k] = pack_low_bytes(b[0], b[1], b[2], b[3]);
  }
  r.sum = s;
  return r;
}
// int8 bytes of 32 values with a scale per value (V's column scales).
__device__ __noinline__ Words8 quant32_s8_cols_slow(Vals32 x, Vals32 inv) {
  Words8 r;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const float4 a = x.v[k], i = inv.v[k];
    r.w[k] = pack_low_bytes(quant_bits(__fmul_rn(a.x, i.x)), quant_bits(__fmul_rn(a.y, i.y)),
                            quant_bits(__fmul_rn(a.z, i.z)), quant_bits(__fmul_rn(a.w, i.w)));
  }
  r.sum = 0;
  return r;
}
__device__ __forceinline__ Vals32 vals32(const float (&v)[32]) {
  Vals32 x;
#pragma unroll
  for (int k = 0; k < 8; k++) x.v[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  return x;
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

// Presets 16 TMEM columns of a projection accumulator (this thread's lane) to
// the bits 2 * 0x4B400000 - bits(zc + 1.5*2^23) = 0x4B400000 - zc (zc is
// 128 * a column sum, an integer below 2^22 in magnitude), so that after the
// products the accumulator holds the float 1.5*2^23 + (acc - zc):
// |acc - zc| = |sum (x_q) w| <= 128 * 127 * H < 2^22 for H <= 256.
__device__ __forceinline__ void tmem_preset_zc16(uint32_t taddr, const float *zc) {
  uint32_t v[16];
#pragma unroll
  for (int k = 0; k < 16; k += 4) {
    const float4 z = *reinterpret_cast<const float4 *>(zc + k);
    v[k] = 2u * (uint32_t)kMagicBits - __float_as_uint(__fadd_rn(z.x, kMagic));
    v[k + 1] = 2u * (uint32_t)kMagicBits - __float_as_uint(__fadd_rn(z.y, kMagic));
    v[k + 2] = 2u * (uint32_t)kMagicBits - __float_as_uint(__fadd_rn(z.z, kMagic));
    v[k + 3] = 2u * (uint32_t)kMagicBits - __float_as_uint(__fadd_rn(z.w, kMagic));
  }
  tmem_st_32x32b_x16(taddr, v);
}

// ((float(acc) - zc) * sb) * sa of four accumulators preset by
// tmem_preset_zc16: the subtraction of 1.5*2^23 recovers acc - zc exactly (as
// float(acc) - zc is exact: both are integers below 2^24), then the two
// products of the QKV GEMM's epilogue.
__device__ __forceinline__ float4 dequant_preset4(const uint32_t *a, const float *sb, float sa) {
  const float4 b = *reinterpret_cast<const float4 *>(sb);
  float2 lo = __fadd2_rn(make_float2(__uint_as_float(a[0]), __uint_as_float(a[1])), f2(-kMagic));
  float2 hi = __fadd2_rn(make_float2(__uint_as_float(a[2]), __uint_as_float(a[3])), f2(-kMagic));
  lo = __fmul2_rn(__fmul2_rn(lo, make_float2(b.x, b.y)), f2(sa));
  hi = __fmul2_rn(__fmul2_rn(hi, make_float2(b.z, b.w)), f2(sa));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

// QKV: the kernel also computes the (sequence, head) slices of the QKV
// projection (internal/modernbert/infer.go:388-390, MatMul8N with the
// quantized normalized rows) on the tensor cores: mqkv then maps the
// quantized rows [N][H] (uint8), mw the QKV weights [3H][H] (int8); xa_s,
// wsb, wzc are the row scales, column scales and 128 * column sums.
template <bool QKV>
__global__ void __launch_bounds__(kShortThreads, QKV ? kShortProjCtasPerSm : kShortCtasPerSm)
    attn_short_kernel(const __grid_constant__ CUtensorMap mqkv, const __grid_constant__ CUtensorMap mw,
                      const __grid_constant__ CUtensorMap mcos, const __grid_constant__ CUtensorMap msin,
                      const float *__restrict__ qkv, const int32_t *__restrict__ offs, int H, int nh, int window,
                      int V, float scale, const float *__restrict__ rope_cos, const float *__restrict__ rope_sin,
                      float *__restrict__ ctx, uint8_t *__restrict__ xq, int ldq, float *__restrict__ sa,
                      const float *__restrict__ xa_s, const float *__restrict__ wsb, const float *__restrict__ wzc) {
  using S = AttnShortSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
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
  uint64_t *bar_b = bar_load + 4;  // fused projection: the K|V weight rows have landed
  uint64_t *bar_m = bar_load + 5;  // fused projection: a product is complete (Q, then K|V)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + S::kTmem);
  volatile int *s_vfast = reinterpret_cast<volatile int *>(smem + S::kTmem + 4);

  const int s = blockIdx.x, h = blockIdx.y;
  // The offsets are copied from the host ahead of every kernel of the
  // stream, not written by one: they may be read before dep_wait().
  const int t0 = offs[s];
  const int n = offs[s + 1] - t0;
  if (n <= 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rr = tid >> 1, hh = tid & 1;
  const bool rope = rope_cos != nullptr;

  uint32_t qw[8];  // this thread's half of its Q row, quantized (bytes q + 128)
  int qr = rr, qh = hh;  // that row and half
  bool ok;
  if constexpr (QKV) {
    // 1'. The projection: Q = A . Wq^T (N = 64) into TMEM, the Q rows
    // dequantized, rotated and quantized in registers; then K|V = A . Wkv^T
    // (N = 128) over the same columns, K rotated into the f32 K slice and V
    // into the f32 V slice. Thread (lane quarter q4, half hq) takes row
    // r = 32 q4 + lane (its TMEM lane) and dimensions 16hq.., 32+16hq..
    const int nkb = H >> 7;  // 128-byte K blocks of the projection
    if (tid == 0) {
      *s_vfast = 1;
      prefetch_tensormap(&mqkv);
      prefetch_tensormap(&mw);
      mbar_init(bar_load, 1);
      mbar_init(bar_s, 1);
      mbar_init(bar_p, kShortThreads);
      mbar_init(bar_o, 1);
      mbar_init(bar_b, 1);
      mbar_init(bar_m, 1);
      fence_barrier_init();
      // A: 128 rows from the sequence's first (rows past it are never used);
      // B: the head's 64 Q weight rows. The weights and the RoPE rows are
      // fetched while the previous kernel finishes, A after dep_wait().
      mbar_arrive_expect_tx(bar_load, nkb * (16384 + 8192) + (rope ? 32768 : 0));
      for (int kb = 0; kb < nkb; kb++) tma_load_2d(&mw, smem + S::kB + kb * 8192, bar_load, kb * 128, h * 64);
      if (rope) {
        tma_load_2d(&mcos, smem + S::kRope, bar_load, 0, 0);
        tma_load_2d(&msin, smem + S::kRope + 16384, bar_load, 0, 0);
      }
    }
    if (warp == 1) tmem_alloc(tmem_slot, 128);
    dep_wait();
    if (tid == 0)
      for (int kb = 0; kb < nkb; kb++) tma_load_2d(&mqkv, smem + S::kA + kb * 16384, bar_load, kb * 128, t0);
    const int q4 = warp & 3, hq = warp >> 2, r = q4 * 32 + lane;
    qr = r;
    qh = hq;
    tc_fence_before();
    __syncthreads();  // barriers initialised, TMEM allocated
    tc_fence_after();
    dep_trigger();
    const uint32_t tm = *tmem_slot;
    const uint32_t trow = tm + ((uint32_t)(q4 * 32) << 16);
    const uint32_t a_base = smem_u32(smem + S::kA), b_base = smem_u32(smem + S::kB);
    // The head's column scales and zero corrections: column j of part p
    // (0 Q, 1 K, 2 V) at p * 64 + j.
    float *s_wsb = reinterpret_cast<float *>(smem + S::kWsb), *s_wzc = reinterpret_cast<float *>(smem + S::kWzc);
    if (tid < 192) {
      const int col = (tid >> 6) * H + h * 64 + (tid & 63);
      s_wsb[tid] = __ldg(wsb + col);
      s_wzc[tid] = __ldg(wzc + col);
    }
    __syncthreads();
    tmem_preset_zc16(trow + 16 * hq, s_wzc + 16 * hq);
    tmem_preset_zc16(trow + 32 + 16 * hq, s_wzc + 32 + 16 * hq);
    tmem_st_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const bool okl = mbar_wait(bar_load, 0, kDevTimeoutFull);
      tc_fence_after();
      if (okl)
        for (int kb = 0; kb < nkb; kb++)
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            mma_u8s8(tm, smem_desc_k_sw128(a_base + kb * 16384 + kk * 32),
                     smem_desc_k_sw128(b_base + kb * 8192 + kk * 32), idesc_u8s8(128, 64), 1);
      mma_commit(bar_m);
      // The Q weights' region takes the K and V weight rows once the products
      // have read it.
      if (okl && mbar_wait(bar_m, 0, kDevTimeoutAccum)) {
        mbar_arrive_expect_tx(bar_b, nkb * 16384);
        for (int kb = 0; kb < nkb; kb++) {
          tma_load_2d(&mw, smem + S::kB + kb * 16384, bar_b, kb * 128, H + h * 64);
          tma_load_2d(&mw, smem + S::kB + kb * 16384 + 8192, bar_b, kb * 128, 2 * H + h * 64);
        }
      }
    }
    __syncwarp();
    // The row's RoPE factors come from the cos/sin rows staged with the
    // operands (positions 0..127; shared memory, not a global load per row).
    const bool rot = rope && r < n;
    const float sar = r < n ? __ldg(xa_s + t0 + r) : 0.0f;
    ok = mbar_wait(bar_m, 0, kDevTimeoutAccum);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    float qv[32];
    {
      uint32_t a0[16], a1[16];
      tmem_ld_32x32b_x16(trow + 16 * hq, a0);
      tmem_ld_32x32b_x16(trow + 32 + 16 * hq, a1);
      tmem_ld_wait();
      const float *qb_lo = s_wsb + 16 * hq, *qb_hi = qb_lo + 32;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float4 lo = dequant_preset4(a0 + 4 * k, qb_lo + 4 * k, sar);
        const float4 hi = dequant_preset4(a1 + 4 * k, qb_hi + 4 * k, sar);
        qv[4 * k] = lo.x, qv[4 * k + 1] = lo.y, qv[4 * k + 2] = lo.z, qv[4 * k + 3] = lo.w;
        qv[16 + 4 * k] = hi.x, qv[17 + 4 * k] = hi.y, qv[18 + 4 * k] = hi.z, qv[19 + 4 * k] = hi.w;
      }
    }
    if (r < n) {
      if (rot) {
        mbar_wait(bar_load, 0, kDevTimeoutFull);  // the RoPE rows have landed
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const float4 rc = *reinterpret_cast<const float4 *>(smem + S::kRope + r * 128 + (((4 * hq + k) ^ (r & 7)) << 4));
          const float4 rs = *reinterpret_cast<const float4 *>(smem + S::kRope + 16384 + r * 128 + (((4 * hq + k) ^ (r & 7)) << 4));
          const float c4[4] = {rc.x, rc.y, rc.z, rc.w}, s4[4] = {rs.x, rs.y, rs.z, rs.w};
#pragma unroll
          for (int u = 0; u < 4; u++) rope1(qv[4 * k + u], qv[16 + 4 * k + u], c4[u], s4[u]);
        }
      }
    } else {
#pragma unroll
      for (int u = 0; u < 32; u++) qv[u] = 0.0f;
    }
    // The row's maximum over both halves (the other half is another warp's):
    // |maximum| over the non-NaN values, the sign bit set where a NaN was seen.
    float *s_qx = reinterpret_cast<float *>(smem + S::kQx);
    const float qm = absmax32<false>(qv);
    bool qn = false;
#pragma unroll
    for (int u = 0; u < 32; u++) qn |= qv[u] != qv[u];
    s_qx[hq * 128 + r] = qn ? neg_bits(qm) : qm;
    tc_fence_before();
    __syncthreads();  // the Q accumulators are read, the half maxima written
    tc_fence_after();
    const float qo = s_qx[(hq ^ 1) * 128 + r];
    const float qmx = fmaxf(qm, fabsf(qo));
    const bool qnan = qn || signbit(qo);
    const float qs = qmx > 0.0f ? __fdiv_rn(qmx, 127.0f) : 0.0f;
    const float qinv = qmx > 0.0f ? __fdiv_rn(1.0f, qs) : 0.0f;
    if (qmx == 0.0f) {
#pragma unroll
      for (int k = 0; k < 8; k++) qw[k] = 0x80808080u;
    } else if (!qnan && scale_is_normal(qs)) {
#pragma unroll
      for (int k = 0; k < 8; k++)
        qw[k] = quant4_fast(qv[4 * k], qv[4 * k + 1], qv[4 * k + 2], qv[4 * k + 3], f2(qinv), f2(qinv));
    } else {
      const Words8 r8 = quant32_u8_slow(vals32(qv), qinv);
#pragma unroll
      for (int k = 0; k < 8; k++) qw[k] = r8.w[k];
    }
    if (hq == 0) s_sq[r] = qmx > 0.0f ? __fmul_rn(qs, scale) : 0.0f;
    // K|V: columns 0-63 K, 64-127 V.
    tmem_preset_zc16(trow + 16 * hq, s_wzc + 64 + 16 * hq);
    tmem_preset_zc16(trow + 32 + 16 * hq, s_wzc + 96 + 16 * hq);
    tmem_preset_zc16(trow + 64 + 16 * hq, s_wzc + 128 + 16 * hq);
    tmem_preset_zc16(trow + 96 + 16 * hq, s_wzc + 160 + 16 * hq);
    tmem_st_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const bool okb = ok && mbar_wait(bar_b, 0, kDevTimeoutFull);
      tc_fence_after();
      if (okb)
        for (int kb = 0; kb < nkb; kb++)
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            mma_u8s8(tm, smem_desc_k_sw128(a_base + kb * 16384 + kk * 32),
                     smem_desc_k_sw128(b_base + kb * 16384 + kk * 32), idesc_u8s8(128, 128), 1);
      mma_commit(bar_m);
    }
    __syncwarp();
    // K is rotated with the same staged factors as Q (same position and pairs).
    ok = ok && mbar_wait(bar_m, 1, kDevTimeoutAccum);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    // The products have read the operand tiles: K and V (f32) go over them.
    {
      uint32_t a0[16], a1[16];
      tmem_ld_32x32b_x16(trow + 16 * hq, a0);
      tmem_ld_32x32b_x16(trow + 32 + 16 * hq, a1);
      tmem_ld_wait();
      const float *kb_lo = s_wsb + 64 + 16 * hq, *kb_hi = kb_lo + 32;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        float4 lo = dequant_preset4(a0 + 4 * k, kb_lo + 4 * k, sar);
        float4 hi = dequant_preset4(a1 + 4 * k, kb_hi + 4 * k, sar);
        if (rot) {
          const float4 rc = *reinterpret_cast<const float4 *>(smem + S::kRope + r * 128 + (((4 * hq + k) ^ (r & 7)) << 4));
          const float4 rs = *reinterpret_cast<const float4 *>(smem + S::kRope + 16384 + r * 128 + (((4 * hq + k) ^ (r & 7)) << 4));
          rope4(lo, hi, rc, rs);
        }
        *f32_chunk(kf, r, 4 * hq + k) = lo;
        *f32_chunk(kf, r, 8 + 4 * hq + k) = hi;
      }
      tmem_ld_32x32b_x16(trow + 64 + 16 * hq, a0);
      tmem_ld_32x32b_x16(trow + 96 + 16 * hq, a1);
      tmem_ld_wait();
      const float *vb_lo = s_wsb + 128 + 16 * hq, *vb_hi = vb_lo + 32;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        *f32_chunk(vf, r, 4 * hq + k) = dequant_preset4(a0 + 4 * k, vb_lo + 4 * k, sar);
        *f32_chunk(vf, r, 8 + 4 * hq + k) = dequant_preset4(a1 + 4 * k, vb_hi + 4 * k, sar);
      }
    }
    tc_fence_before();
    __syncthreads();
  } else {
    dep_wait();
    // 1. K and V by TMA; Q and the RoPE factors straight into registers.
    if (tid == 0) {
      *s_vfast = 1;
      prefetch_tensormap(&mqkv);
      mbar_init(bar_load, 1);
      mbar_init(bar_s, 1);
      mbar_init(bar_p, kShortThreads);
      mbar_init(bar_o, 1);
      fence_barrier_init();
      mbar_arrive_expect_tx(bar_load, 4 * S::kHalf);
  #pragma unroll
      for (int x = 0; x < 2; x++)
  #pragma unroll
        for (int half = 0; half < 2; half++)
          tma_load_2d(&mqkv, smem + x * 32768 + half * S::kHalf, bar_load, (x + 1) * H + h * 64 + half * 32, t0);
    }
    if (warp == 1) tmem_alloc(tmem_slot, 128);
    float qv[32];  // [0,16): dimensions 16hh.., [16,32): 32+16hh..
    if (rr < n) {
      const float *qrow = qkv + (size_t)(t0 + rr) * 3 * H + h * 64 + 16 * hh;
  #pragma unroll
      for (int k = 0; k < 4; k++) {
        const float4 lo = __ldg(reinterpret_cast<const float4 *>(qrow + 4 * k));
        const float4 hi = __ldg(reinterpret_cast<const float4 *>(qrow + 32 + 4 * k));
        qv[4 * k] = lo.x, qv[4 * k + 1] = lo.y, qv[4 * k + 2] = lo.z, qv[4 * k + 3] = lo.w;
        qv[16 + 4 * k] = hi.x, qv[17 + 4 * k] = hi.y, qv[18 + 4 * k] = hi.z, qv[19 + 4 * k] = hi.w;
      }
      if (rope) {
  #pragma unroll
        for (int k = 0; k < 4; k++) {
          const float4 rc = __ldg(reinterpret_cast<const float4 *>(rope_cos + (size_t)rr * 32 + 16 * hh + 4 * k));
          const float4 rs = __ldg(reinterpret_cast<const float4 *>(rope_sin + (size_t)rr * 32 + 16 * hh + 4 * k));
          const float c4[4] = {rc.x, rc.y, rc.z, rc.w}, s4[4] = {rs.x, rs.y, rs.z, rs.w};
  #pragma unroll
          for (int u = 0; u < 4; u++) rope1(qv[4 * k + u], qv[16 + 4 * k + u], c4[u], s4[u]);
        }
      }
    } else {
  #pragma unroll
      for (int u = 0; u < 32; u++) qv[u] = 0.0f;
    }
    {
      // Row maximum, NaN-propagating first: a row holding a NaN takes the
      // clamped path (with the NaN-ignoring maximum, as the reference's).
      float qmx = absmax32<true>(qv);
      qmx = fmax_nan(qmx, __shfl_xor_sync(0xffffffffu, qmx, 1));
      const bool qnan = qmx != qmx;
      if (__any_sync(0xffffffffu, qnan)) {
        qmx = absmax32<false>(qv);
        qmx = fmaxf(qmx, __shfl_xor_sync(0xffffffffu, qmx, 1));
      }
      const float qs = qmx > 0.0f ? __fdiv_rn(qmx, 127.0f) : 0.0f;
      const float qinv = qmx > 0.0f ? __fdiv_rn(1.0f, qs) : 0.0f;
      // Byte q + 128, q = clamp(rne(x * qinv)); a row whose maximum is 0 is all
      // 128 (attention8.go:210-220).
      if (qmx == 0.0f) {
  #pragma unroll
        for (int k = 0; k < 8; k++) qw[k] = 0x80808080u;
      } else if (!qnan && scale_is_normal(qs)) {
  #pragma unroll
        for (int k = 0; k < 8; k++)
          qw[k] = quant4_fast(qv[4 * k], qv[4 * k + 1], qv[4 * k + 2], qv[4 * k + 3], f2(qinv), f2(qinv));
      } else {
        const Words8 r8 = quant32_u8_slow(vals32(qv), qinv);
  #pragma unroll
        for (int k = 0; k < 8; k++) qw[k] = r8.w[k];
      }
      if (hh == 0) s_sq[rr] = qmx > 0.0f ? __fmul_rn(qs, scale) : 0.0f;
    }
    __syncthreads();  // barriers initialised
    dep_trigger();
    ok = mbar_wait(bar_load, 0, kDevTimeoutFull);

    // A. K rotated in place (the RoPE factors are read again; they are cached).
    if (rope && rr < n) {
  #pragma unroll
      for (int k = 0; k < 4; k++) {
        const int c = 4 * hh + k;
        const float4 rc = __ldg(reinterpret_cast<const float4 *>(rope_cos + (size_t)rr * 32 + 16 * hh + 4 * k));
        const float4 rs = __ldg(reinterpret_cast<const float4 *>(rope_sin + (size_t)rr * 32 + 16 * hh + 4 * k));
        float4 lo = *f32_chunk(kf, rr, c), hi = *f32_chunk(kf, rr, 8 + c);
        rope4(lo, hi, rc, rs);
        *f32_chunk(kf, rr, c) = lo;
        *f32_chunk(kf, rr, 8 + c) = hi;
      }
    }
    __syncthreads();
  }

  // B. Warps 0-1: K column means (ordered float32 sums over the rotated
  // keys). Warps 2-3: V column maxima; then warps 4-7 quantize V per column,
  // one row each, into its tile (over the f32 V rows once all are read).
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
  } else if (tid < 128) {
    const int d = tid - 64;
    float m[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // NaN-ignoring maxima
    bool nan = false;                       // a NaN in the column
    int r = 0;
    for (; r + 4 <= n; r += 4) {
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float a = fabsf(f32_at(vf, r + u, d));
        m[u] = fmaxf(m[u], a);
        nan |= a != a;
      }
    }
    for (; r < n; r++) {
      const float a = fabsf(f32_at(vf, r, d));
      m[0] = fmaxf(m[0], a);
      nan |= a != a;
    }
    const float mx = fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
    const float sc = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 0.0f;
    s_vs[d] = sc;
    s_vinv[d] = mx > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
    // vinv = 0 (a zero column): every byte is rne(v * 0).
    if (nan || !(mx == 0.0f || scale_is_normal(sc))) *s_vfast = 0;
    named_barrier_sync(2, 192);  // the V scales are in shared memory
  } else {
    named_barrier_sync(2, 192);
    const int vr = tid - 128;
    const bool vfast = *s_vfast != 0;
    uint32_t vw[16];
    if (vfast) {
#pragma unroll
      for (int c = 0; c < 8; c++) {
        float4 lo = make_float4(0.0f, 0.0f, 0.0f, 0.0f), hi = lo;
        if (vr < n) {
          lo = *f32_chunk(vf, vr, c);
          hi = *f32_chunk(vf, vr, 8 + c);
        }
        const float4 il = *reinterpret_cast<const float4 *>(s_vinv + 4 * c);
        const float4 ih = *reinterpret_cast<const float4 *>(s_vinv + 32 + 4 * c);
        vw[c] = quant4_fast_s8(lo.x, lo.y, lo.z, lo.w, make_float2(il.x, il.y), make_float2(il.z, il.w));
        vw[8 + c] = quant4_fast_s8(hi.x, hi.y, hi.z, hi.w, make_float2(ih.x, ih.y), make_float2(ih.z, ih.w));
      }
    } else {  // dimensions 0-31, then 32-63, each with its column's scale
#pragma unroll
      for (int half = 0; half < 2; half++) {
        Vals32 x, inv;
#pragma unroll
        for (int c = 0; c < 8; c++) {
          x.v[c] = vr < n ? *f32_chunk(vf, vr, 8 * half + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          inv.v[c] = *reinterpret_cast<const float4 *>(s_vinv + 32 * half + 4 * c);
        }
        const Words8 r8 = quant32_s8_cols_slow(x, inv);
#pragma unroll
        for (int c = 0; c < 8; c++) vw[8 * half + c] = r8.w[c];
      }
    }
    named_barrier_sync(3, 128);  // every f32 V row has been read
    // Tile chunk t holds dimensions 16t..16t+15: f32 chunks 4t..4t+3.
    *tile_chunk(smem + S::kVt, vr, 0) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
    *tile_chunk(smem + S::kVt, vr, 1) = make_uint4(vw[4], vw[5], vw[6], vw[7]);
    *tile_chunk(smem + S::kVt, vr, 2) = make_uint4(vw[8], vw[9], vw[10], vw[11]);
    *tile_chunk(smem + S::kVt, vr, 3) = make_uint4(vw[12], vw[13], vw[14], vw[15]);
  }
  __syncthreads();

  // C. K rows: centred, x = rne(kv * kinv) (the key's sum takes x before the
  // int8 clamp; a zero row gives kinv = 0, so x = 0).
  uint32_t kw[8];
  {
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
    float kmx = absmax32<true>(kv);
    kmx = fmax_nan(kmx, __shfl_xor_sync(0xffffffffu, kmx, 1));
    const bool knan = kmx != kmx;
    if (__any_sync(0xffffffffu, knan)) {
      kmx = absmax32<false>(kv);
      kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, 1));
    }
    const float kss = kmx > 0.0f ? __fdiv_rn(kmx, 127.0f) : 0.0f;
    const float kinv = kmx > 0.0f ? __fdiv_rn(1.0f, kss) : 0.0f;
    int ksum = 0;
    const bool slow = kmx > 0.0f && (knan || !scale_is_normal(kss));
    if (kmx == 0.0f) {  // a zero key: zero bytes, scale and sum (attention8.go:240-251)
#pragma unroll
      for (int k = 0; k < 8; k++) kw[k] = 0u;
    } else if (!slow) {  // bytes are x itself: sum them as signed bytes (two exact integer chains)
      int ks2 = 0;
#pragma unroll
      for (int k = 0; k < 8; k++) {
        kw[k] = quant4_fast_s8(kv[4 * k], kv[4 * k + 1], kv[4 * k + 2], kv[4 * k + 3], f2(kinv), f2(kinv));
        if (k & 1)
          ks2 = dp4a_ss(kw[k], 0x01010101u, ks2);
        else
          ksum = dp4a_ss(kw[k], 0x01010101u, ksum);
      }
      ksum += ks2;
    } else {  // the reference's conversion (NaN -> INT_MIN, summed before the clamp)
      const Words8 r8 = quant32_s8_slow(vals32(kv), kinv, ksum);
#pragma unroll
      for (int k = 0; k < 8; k++) kw[k] = r8.w[k];
      ksum = r8.sum;
    }
    ksum += __shfl_xor_sync(0xffffffffu, ksum, 1);
    if (hh == 0) {
      s_ks[rr] = kss;
      s_kzc[rr] = __fadd_rn(kmx > 0.0f ? __fmul_rn(128.0f, (float)ksum) : 0.0f, kMagic);  // zcm for dequant2m
    }
  }
  __syncthreads();  // every f32 K row has been read
  *tile_chunk(smem + S::kKt, rr, hh) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
  *tile_chunk(smem + S::kKt, rr, 2 + hh) = make_uint4(kw[4], kw[5], kw[6], kw[7]);
  *tile_chunk(smem + S::kQt, qr, qh) = make_uint4(qw[0], qw[1], qw[2], qw[3]);
  *tile_chunk(smem + S::kQt, qr, 2 + qh) = make_uint4(qw[4], qw[5], qw[6], qw[7]);
  fence_proxy_async_smem();  // the tiles are read by the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // D. Attend.
  const int q = warp & 3;   // TMEM lane quarter: rows [32q, 32q+32)
  const int g = warp >> 2;  // 16-key chunks with parity g
  const int r = q * 32 + lane;
  const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
  // Every row's score accumulator of key j starts at 0x4B400000 - 128*sum(kq_j)
  // (the bits of 1.5*2^23 + (acc - zc) once the products are added).
#pragma unroll
  for (int c16 = 0; c16 < 4; c16++) {
    uint32_t init[16];
#pragma unroll
    for (int u = 0; u < 16; u++) init[u] = 2u * (uint32_t)kMagicBits - __float_as_uint(s_kzc[64 * g + 16 * c16 + u]);
    tmem_st_32x32b_x16(tbase + 64 * g + 16 * c16, init);
  }
  tmem_st_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    constexpr uint32_t idesc_s = idesc_u8s8(128, 128);
    const uint32_t q_base = smem_u32(smem + S::kQt), k_base = smem_u32(smem + S::kKt);
#pragma unroll
    for (int kk = 0; kk < 2; kk++)
      mma_u8s8(tmem, smem_desc_k_sw64(q_base + kk * 32), smem_desc_k_sw64(k_base + kk * 32), idesc_s, 1);
    mma_commit(bar_s);
  }
  __syncwarp();
  const bool valid = r < n;
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
  float mx = -INFINITY;  // of (acc - zc) * ks; times sq below
  if (ok) {
    for (int ch = ch0 + ((ch0 ^ g) & 1); ch < ch1; ch += 2)
      mx = chunk_max<true>(tbase + ch * 16, ch * 16, s_kzc, s_ks, w, mx);
  }
  red[g * 128 + r] = mx;
  __syncthreads();
  mx = __fmul_rn(fmaxf(red[r], red[128 + r]), w.sq);
  int psum = 0;
  for (int ch = g; ch < 8; ch += 2) {
    uint4 pw = make_uint4(0, 0, 0, 0);
    if (ok && ch >= ch0 && ch < ch1) pw = chunk_p<true>(tbase + ch * 16, ch * 16, s_kzc, s_ks, w, mx, psum);
    *reinterpret_cast<uint4 *>(prow_smem + ((ch ^ (r & 7)) << 4)) = pw;
  }
  if (ok && w.t0 < w.t1)
    psum += tail_fixup(smem + S::kQt, smem + S::kKt, 8192, smem + S::kP, r, g, w.t0, w.t1, s_kzc, s_ks, w.sq, mx);
  tc_fence_before();
  fence_proxy_async_smem();
  mbar_arrive(bar_p);
  if (warp == 0) {
    if (lane == 0) {
      constexpr uint32_t idesc_o = idesc_u8s8(128, 64) | (1u << 16);  // B (V) MN-major
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
    __syncwarp();
  }
  __syncthreads();  // every thread has read red[] (max)
  reinterpret_cast<int *>(red)[g * 128 + r] = psum;
  __syncthreads();
  psum = reinterpret_cast<int *>(red)[r] + reinterpret_cast<int *>(red)[128 + r];
  const float sp = psum > 0 ? __fdiv_rn(1.0f, (float)psum) : 0.0f;
  if (ok) ok = mbar_wait(bar_o, 0, kDevTimeoutAccum);
  ok = __all_sync(0xffffffffu, ok);
  tc_fence_after();
  uint32_t o[32];
  tmem_ld_32x32b_x32(tbase + 32 * g, o);
  tmem_ld_wait();
  if (xq != nullptr) {
    // ctx quantized per row over all heads (the launch's cluster holds the
    // sequence's nh heads, one CTA each): quant_rows4_kernel's arithmetic on
    // the row maximum, each CTA's part pushed to every CTA of the cluster
    // through distributed shared memory.
    const float *vsc = s_vs + 32 * g;
    // Row maxima travel as |maximum| over the non-NaN values with the sign
    // bit set where a NaN was seen: the NaN-propagating maximum is NaN
    // exactly then, and otherwise equals the other.
    float v[32], pi = 0.0f;
    bool pnan = false;
#pragma unroll
    for (int d = 0; d < 32; d++) {
      v[d] = dequant_o(o[d], vsc[d], sp);
      pi = fmaxf(pi, fabsf(v[d]));
      pnan |= v[d] != v[d];
    }
    float *xh = reinterpret_cast<float *>(smem + S::kO);  // [2][128] per half row
    float *gx = reinterpret_cast<float *>(smem + S::kXch);  // [8][128] per cluster CTA, pushed by it
    xh[g * 128 + r] = pnan ? neg_bits(pi) : pi;
    __syncthreads();
    if (tid < 128) {
      const float a = xh[tid], b = xh[128 + tid];
      const float m = fmaxf(fabsf(a), fabsf(b));
      const float e = (signbit(a) || signbit(b)) ? neg_bits(m) : m;
      const uint32_t me = cluster_ctarank();
      for (int c = 0; c < nh; c++) st_dsmem_f32(gx + me * 128 + tid, (uint32_t)c, e);
    }
    // The exchange region is used by nothing else, and after this every CTA
    // reads only its own shared memory, so none waits for the others to leave.
    cluster_sync_all();
    float mx = 0.0f;
    bool has_nan = false;
    for (int c = 0; c < nh; c++) {
      const float e = gx[c * 128 + r];
      mx = fmaxf(mx, fabsf(e));
      has_nan |= signbit(e);
    }
    float qs = 0.0f, qinv = 0.0f;
    if (mx > 0.0f) {
      qs = __fdiv_rn(mx, 127.0f);
      qinv = __fdiv_rn(1.0f, qs);
    }
    const bool fast = !has_nan && row_scale_normal(qs), store = ok && valid;
    uint4 *dst = reinterpret_cast<uint4 *>(xq + (size_t)(t0 + r) * ldq + h * 64 + 32 * g);
    uint32_t wv[8];
    if (mx == 0.0f) {
#pragma unroll
      for (int k = 0; k < 8; k++) wv[k] = 0x80808080u;
    } else if (fast) {
#pragma unroll
      for (int k = 0; k < 8; k++) wv[k] = quant4_fast(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3], f2(qinv), f2(qinv));
    } else {
      const Words8 r8 = quant32_u8_slow(vals32(v), qinv);
#pragma unroll
      for (int k = 0; k < 8; k++) wv[k] = r8.w[k];
    }
    if (store) {
      dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
    }
    if (store && h == 0 && g == 0) sa[t0 + r] = qs;
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, 128);
    }
    return;
  }
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
  tc_fence_before();
  __syncthreads();
  if (ok) {
    for (int e = tid; e < n * 16; e += kShortThreads) {
      const int row = e >> 4, c4 = (e & 15) * 4;
      *reinterpret_cast<float4 *>(ctx + (size_t)(t0 + row) * H + h * 64 + c4) =
          *reinterpret_cast<const float4 *>(ostage + row * S::kOPitch + c4);
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// The 16-byte row loads and stores need H a multiple of 4 and 16-byte
// aligned qkv and ctx (the fused projection reads no qkv).
bool attn_short_fits(const AttnArgs &a) {
  if (a.D != 64 || a.max_len > kShortN || (a.H % 4) != 0 || a.V < 1) return false;
  if (a.xa) return attn_short_projects(a);
  return (reinterpret_cast<uintptr_t>(a.qkv) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.ctx) & 15) == 0;
}

// The fused projection: H = nh * 64 in {128, 256} (one or two 128-byte K
// blocks; |acc - zc| < 2^22 for the preset accumulators), rows and weights
// with 16-byte aligned pitches, ctx quantized in the kernel.
bool attn_short_projects(const AttnArgs &a) {
  return a.xa && a.wqkv && a.xa_s && a.wsb && a.wzc && a.D == 64 && a.max_len <= kShortN && a.V >= 1 &&
         (a.H == 128 || a.H == 256) && a.H == a.nh * 64 && a.lda >= a.H && a.lda % 16 == 0 && a.ldw >= a.H &&
         a.ldw % 16 == 0 && ((reinterpret_cast<uintptr_t>(a.xa) | reinterpret_cast<uintptr_t>(a.wqkv)) & 15) == 0 &&
         ((reinterpret_cast<uintptr_t>(a.wsb) | reinterpret_cast<uintptr_t>(a.wzc)) & 15) == 0 && a.xq && a.sa &&
         a.nh <= 8 && (a.ldq % 16) == 0 && (reinterpret_cast<uintptr_t>(a.xq) & 15) == 0;
}

static int map_u8_rows(CUtensorMap *map, const void *base, int rows, int cols, int ld, int box_rows) {
  auto enc = get_encode_fn();
  if (!enc) return IG_ERR_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0
             : IG_ERR_CUDA;
}

int launch_attn_short(const AttnArgs &a, cudaStream_t st) {
  if (a.nseq <= 0 || a.N <= 0) return 0;
  if (!attn_short_fits(a)) return IG_ERR_UNSUPPORTED;
  const bool proj = a.xa != nullptr;
  CUtensorMap map, mapw;
  if (proj) {
    // The quantized rows [N][H] in [128 rows][128 B] boxes; the QKV weights
    // [3H][H] in [64 rows][128 B] boxes; both SWIZZLE_128B (UMMA K-major).
    if (map_u8_rows(&map, a.xa, a.N, a.H, a.lda, 128) || map_u8_rows(&mapw, a.wqkv, 3 * a.H, a.H, a.ldw, 64))
      return IG_ERR_CUDA;
  } else {
    // qkv as a [N][3H] f32 plane, copied in 32-float x 128-row SWIZZLE_128B boxes.
    auto enc = get_encode_fn();
    if (!enc) return IG_ERR_CUDA;
    cuuint64_t dims[2] = {(cuuint64_t)3 * a.H, (cuuint64_t)a.N};
    cuuint64_t strides[1] = {(cuuint64_t)3 * a.H * sizeof(float)};
    cuuint32_t box[2] = {32, (cuuint32_t)kShortN};
    cuuint32_t estr[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.qkv), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return IG_ERR_CUDA;
    mapw = map;
  }
  // The RoPE factor rows of positions 0..127 ([rows][32] f32, SWIZZLE_128B),
  // staged by the projecting kernel.
  CUtensorMap mcos = map, msin = map;
  if (proj && a.rope_cos) {
    auto enc = get_encode_fn();
    if (!enc) return IG_ERR_CUDA;
    cuuint64_t dims[2] = {32, (cuuint64_t)a.max_len};
    cuuint64_t strides[1] = {32 * sizeof(float)};
    cuuint32_t box[2] = {32, (cuuint32_t)kShortN};
    cuuint32_t estr[2] = {1, 1};
    if (enc(&mcos, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.rope_cos), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&msin, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.rope_sin), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return IG_ERR_CUDA;
  }
  auto kern = proj ? attn_short_kernel<true> : attn_short_kernel<false>;
  static SmemOptIn attr_plain, attr_proj;
  const int smem = proj ? AttnShortSmem::kTotalProj : AttnShortSmem::kTotal;
  if ((proj ? attr_proj : attr_plain).ensure((const void *)kern, smem) != cudaSuccess)
    return IG_ERR_CUDA;
  if (a.xq) {
    if (!attn_short_quantizes(a)) return IG_ERR_UNSUPPORTED;
    // One cluster per sequence: its nh head CTAs share the row maxima.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.nseq, a.nh);
    cfg.blockDim = dim3(kShortThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = a.nh;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    add_dep_attr(at, cfg.numAttrs);
    if (cudaLaunchKernelEx(&cfg, kern, map, mapw, mcos, msin, a.qkv, a.offs, a.H, a.nh, a.window, a.V, a.scale, a.rope_cos,
                           a.rope_sin, a.ctx, a.xq, a.ldq, a.sa, a.xa_s, a.wsb, a.wzc) != cudaSuccess)
      return IG_ERR_CUDA;
    return 0;
  }
  if (proj) return IG_ERR_UNSUPPORTED;
  return launch_dep(attn_short_kernel<false>, dim3(a.nseq, a.nh), kShortThreads, AttnShortSmem::kTotal, st, map,
                    mapw, map, map, a.qkv, a.offs, a.H, a.nh, a.window, a.V, a.scale, a.rope_cos, a.rope_sin, a.ctx,
                    nullptr, 0, nullptr, nullptr, nullptr, nullptr) == cudaSuccess
             ? 0
             : IG_ERR_CUDA;
}

// The row quantization needs the whole row in one cluster (nh <= 8 CTAs, a
// portable cluster size), H = nh * 64, and 16-byte aligned row pieces.
bool attn_short_quantizes(const AttnArgs &a) {
  return attn_short_fits(a) && a.nh >= 1 && a.nh <= 8 && a.H == a.nh * 64 && a.xq && a.sa && (a.ldq % 16) == 0 &&
         (reinterpret_cast<uintptr_t>(a.xq) & 15) == 0;
}

}  // namespace ig
