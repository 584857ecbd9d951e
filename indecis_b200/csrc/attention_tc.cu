// int8 attention on the tensor cores: the Attend half of linalg/attention8.go
// (:298-376) for a block of 128 queries of one (sequence, head) whose keys
// fit in 256 columns (every local layer with a half-window up to 64, and
// global layers up to 256 tokens). Longer key ranges go through
// attn_attend_kernel (attention.cu), which computes the same bits.
//
// One CTA, 10 warps:
//   warp 0     TMA: Q tile [128 rows][64 B], K and V tiles [128 keys][64 B]
//              per 128 keys, all SWIZZLE_64B (no multicast).
//   warp 1     TMEM (256 columns) and the MMAs:
//                S = Q . K^T     M=128 queries, N=128 keys per tile, K=64
//                                (kind::i8, Q uint8 q+128, K int8, K-major)
//                O = P . V       M=128, N=64 dims, K=keys; P uint8 from shared
//                                memory (K-major, SWIZZLE_128B), V int8 read
//                                in its natural [keys][dims] layout as an
//                                MN-major operand. O overwrites S's columns.
//   warps 2-9  two warps per query row quarter (TMEM lanes), each taking
//              alternate 16-key chunks: dequantize the row's scores, MaxOf
//              over the valid keys (the two halves combined through shared
//              memory), ExpShift (vector-body / scalar-tail split by position),
//              P = rne(e*255) into shared memory, sp = 1/float32(sum P); then
//              O = (float(acc)*vs[d])*sp, each warp 32 of the 64 dimensions.
// Every wait is bounded (mbar_wait), so a lost arrival ends the kernel with
// an error code instead of a hang.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "exactmath.cuh"
#include "internal.h"

namespace ig {

constexpr int kAtQ = 128;       // queries per CTA
constexpr int kAtKT = 128;      // keys per S tile
constexpr int kAtSoftWarps = 8;  // two per TMEM lane quarter, alternate 16-key chunks
constexpr int kAtThreads = 64 + 32 * kAtSoftWarps;

struct AttnTcSmem {
  static constexpr int kQ = 0;                  // [128][64 B] SW64
  static constexpr int kK = kQ + 8192;          // 2 x [128][64 B] SW64
  static constexpr int kV = kK + 16384;         // 2 x [128][64 B] SW64 (MN-major B operand)
  static constexpr int kP = kV + 16384;         // 2 x [128][128 B] SW128 (1024-aligned)
  static constexpr int kKs = kP + 32768;        // 256 key scales
  static constexpr int kKzc = kKs + 1024;       // 256 key zero corrections
  static constexpr int kRed = kKzc + 1024;      // row max / P-sum exchange: 2 groups x 128 rows x 8 B
  static constexpr int kBar = kRed + 2048;      // 4 mbarriers
  static constexpr int kTmem = kBar + 64;
  // Requested size: padded so that at most two CTAs share an SM (two x 256
  // TMEM columns fill the SM's 512).
  static constexpr int kTotal = 100 * 1024;
};

// K-major operand with 64-byte rows (SWIZZLE_64B): 8-row groups 512 B apart.
__device__ __forceinline__ uint64_t smem_desc_k_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;  // SWIZZLE_64B
  return d;
}

// MN-major operand whose MN extent is one 64-byte swizzle row (64 int8 values):
// rows along K are 64 B apart, 8-row groups 512 B apart (SBO). The leading
// offset (between 64-byte MN atoms) is unused at N = 64; it is set to the
// V tile size so that it would stay inside the CTA's shared memory.
__device__ __forceinline__ uint64_t smem_desc_mn_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(16384 >> 4) << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;
  return d;
}



// One query row's view of a tile of scores: valid key columns [a, b) and the
// columns [t0, t1) that take the scalar-tail exp (ExpShift's last len % V
// keys), all relative to the tile's first key; sq is the row's scale.
struct ScoreRow {
  int a, b, t0, t1;
  float sq;
};

// Scores (acc - zc) * ks [* sq] of two keys. PRE: the accumulators started
// from 0x4B400000 - 128*sum(kq) (written into TMEM before the MMA), so their
// bits are the float 1.5*2^23 + (acc - zc) and one subtraction recovers
// acc - zc exactly; otherwise zcm holds 128*sum(kq) + 1.5*2^23 (dequant2m).
template <bool PRE>
__device__ __forceinline__ float2 score2(uint32_t a0, uint32_t a1, float2 zcm, float2 ks, float sq, bool with_sq) {
  if constexpr (PRE) {
    const float2 u = __fmul2_rn(__fadd2_rn(make_float2(__uint_as_float(a0), __uint_as_float(a1)), f2(-kMagic)), ks);
    return with_sq ? __fmul2_rn(u, f2(sq)) : u;
  } else {
    return dequant2m((int32_t)a0, (int32_t)a1, zcm, ks, sq);
  }
}

// MaxOf over the valid columns of the 16-key chunk at TMEM column tcol.
// PRE: the maximum of (acc - zc) * ks, before the row's sq (x -> x * sq is
// non-decreasing for sq >= 0, so the row maximum is that maximum times sq).
// MASK: some column of the chunk may lie outside a row's [a, b) (false when
// every lane's row takes all 16: no per-column tests).
template <bool PRE, bool MASK>
__device__ __forceinline__ float chunk_max_acc(const uint32_t (&acc)[16], int c, const float *zcm, const float *ks,
                                               const ScoreRow &w, float mx) {
#pragma unroll
  for (int v = 0; v < 16; v += 4) {
    const float4 z = PRE ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : *reinterpret_cast<const float4 *>(zcm + c + v);
    const float4 k = *reinterpret_cast<const float4 *>(ks + c + v);
    const float2 s0 = score2<PRE>(acc[v], acc[v + 1], make_float2(z.x, z.y), make_float2(k.x, k.y), w.sq, false);
    const float2 s1 = score2<PRE>(acc[v + 2], acc[v + 3], make_float2(z.z, z.w), make_float2(k.z, k.w), w.sq, false);
    if (!MASK) {
      mx = fmaxf(mx, fmaxf(fmaxf(s0.x, s0.y), fmaxf(s1.x, s1.y)));
    } else {
      const int col = c + v;
      if (col >= w.a && col < w.b) mx = fmaxf(mx, s0.x);
      if (col + 1 >= w.a && col + 1 < w.b) mx = fmaxf(mx, s0.y);
      if (col + 2 >= w.a && col + 2 < w.b) mx = fmaxf(mx, s1.x);
      if (col + 3 >= w.a && col + 3 < w.b) mx = fmaxf(mx, s1.y);
    }
  }
  return mx;
}

// The quantized softmax weights P = rne(exp(score - mx) * 255) of the 16-key
// chunk at TMEM column tcol as 16 bytes (0 outside the row's valid keys), all
// with ExpShift's vector-body exp (tail_fixup then rewrites the row's
// scalar-tail keys); the sum of the 16 is added to psum. The subtraction is
// scalar: with a packed add here (after the packed products of dequant2m or
// score2) one row in a few thousand came out different, every run.
template <bool PRE, bool MASK>
__device__ __forceinline__ uint4 chunk_p_acc(const uint32_t (&acc)[16], int c, const float *zcm, const float *ks,
                                            const ScoreRow &w, float mx, int &psum) {
  uint32_t bits[16];  // 0x4B400000 + P (low byte P)
#pragma unroll
  for (int v = 0; v < 16; v += 4) {
    const float4 z = PRE ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : *reinterpret_cast<const float4 *>(zcm + c + v);
    const float4 k = *reinterpret_cast<const float4 *>(ks + c + v);
#pragma unroll
    for (int h = 0; h < 4; h += 2) {
      const float2 sc = score2<PRE>(acc[v + h], acc[v + h + 1], h ? make_float2(z.z, z.w) : make_float2(z.x, z.y),
                                    h ? make_float2(k.z, k.w) : make_float2(k.x, k.y), w.sq, true);
      const uint2 b = exp_p_bits2(make_float2(__fsub_rn(sc.x, mx), __fsub_rn(sc.y, mx)));
      bits[v + h] = b.x;
      bits[v + h + 1] = b.y;
      if (MASK) {
        const int col = c + v + h;
        if (!(col >= w.a && col < w.b)) bits[v + h] = (uint32_t)kMagicBits;
        if (!(col + 1 >= w.a && col + 1 < w.b)) bits[v + h + 1] = (uint32_t)kMagicBits;
      }
    }
  }
  uint32_t word[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    word[k] = __byte_perm(__byte_perm(bits[4 * k], bits[4 * k + 1], 0x0040),
                          __byte_perm(bits[4 * k + 2], bits[4 * k + 3], 0x0040), 0x5410);
    psum = dp4a_us(word[k], 0x01010101u, psum);
  }
  return make_uint4(word[0], word[1], word[2], word[3]);
}

// Whether every row of the warp takes all 16 keys of the chunk at column c.
__device__ __forceinline__ bool chunk_inner(int c, const ScoreRow &w) {
  return __all_sync(0xffffffffu, c >= w.a && c + 16 <= w.b);
}

template <bool PRE>
__device__ __forceinline__ float chunk_max(uint32_t tcol, int c, const float *zcm, const float *ks,
                                           const ScoreRow &w, float mx) {
  uint32_t acc[16];
  tmem_ld_32x32b_x16(tcol, acc);
  tmem_ld_wait();
  if (chunk_inner(c, w)) return chunk_max_acc<PRE, false>(acc, c, zcm, ks, w, mx);
  return chunk_max_acc<PRE, true>(acc, c, zcm, ks, w, mx);
}

template <bool PRE>
__device__ __forceinline__ uint4 chunk_p(uint32_t tcol, int c, const float *zcm, const float *ks, const ScoreRow &w,
                                        float mx, int &psum) {
  uint32_t acc[16];
  tmem_ld_32x32b_x16(tcol, acc);
  tmem_ld_wait();
  if (chunk_inner(c, w)) return chunk_p_acc<PRE, false>(acc, c, zcm, ks, w, mx, psum);
  return chunk_p_acc<PRE, true>(acc, c, zcm, ks, w, mx, psum);
}

// ExpShift's scalar-tail keys [t0, t1) of query row r (its last len % V
// keys; at most V - 1) that lie in this thread's 16-key chunks (parity g):
// the int32 score is recomputed on the CUDA cores from the quantized Q and K
// rows in shared memory (the same dot product the tensor cores formed; both
// tiles [rows][64 B] SWIZZLE_64B, key tiles ktile_bytes apart), dequantized
// as in chunk_p, and P = rne(exp32(score - mx) * 255) replaces the byte the
// chunk pass wrote into P ([128 rows][128 B] SWIZZLE_128B per 128 keys).
// Returns the change of the row's P sum.
__device__ __forceinline__ int tail_fixup(const uint8_t *qtile, const uint8_t *ktile, int ktile_bytes, uint8_t *ptile,
                                       int r, int g, int t0, int t1, const float *zcm, const float *ks, float sq,
                                       float mx) {
  int dsum = 0;  // change of the row's P sum
  if (t0 >= t1) return 0;
  uint4 qa4[4];
  const uint8_t *qrow = qtile + r * 64;
#pragma unroll
  for (int ch = 0; ch < 4; ch++) qa4[ch] = *reinterpret_cast<const uint4 *>(qrow + ((ch ^ ((r >> 1) & 3)) << 4));
  // The tail keys in this thread's 16-key chunks (parity g), chunk by chunk.
  int ck = t0 >> 4;
  ck += (ck & 1) != g;
  for (int c = max(t0, 16 * ck); c < t1; c = (c & 15) == 15 ? c + 17 : c + 1) {
    const int kt = c >> 7, kr = c & 127;
    const uint8_t *krow = ktile + kt * ktile_bytes + kr * 64;
    int part[4] = {0, 0, 0, 0};  // four exact integer chains, summed after
#pragma unroll
    for (int ch = 0; ch < 4; ch++) {
      const uint4 qa = qa4[ch];
      const uint4 kb = *reinterpret_cast<const uint4 *>(krow + ((ch ^ ((kr >> 1) & 3)) << 4));
      part[ch] = dp4a_us(qa.x, kb.x, part[ch]);
      part[ch] = dp4a_us(qa.y, kb.y, part[ch]);
      part[ch] = dp4a_us(qa.z, kb.z, part[ch]);
      part[ch] = dp4a_us(qa.w, kb.w, part[ch]);
    }
    const int acc = (part[0] + part[1]) + (part[2] + part[3]);
    const float sc = __fmul_rn(__fmul_rn(__fsub_rn(magic_float(acc), zcm[c]), ks[c]), sq);
    const int p = __float2int_rn(__fmul_rn(exp_tail(__fsub_rn(sc, mx)), 255.0f));
    uint8_t *pb = ptile + kt * 16384 + r * 128 + ((((c & 127) >> 4) ^ (r & 7)) << 4) + (c & 15);
    dsum += p - (int)*pb;
    *pb = (uint8_t)p;
  }
  return dsum;
}

// Block entry: x sequence, y first query, z first key c0 (a multiple of 16),
// w number of 128-key tiles (1 or 2).
__global__ void __launch_bounds__(kAtThreads, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                   const __grid_constant__ CUtensorMap mv, const int4 *__restrict__ blocks,
                   const int32_t *__restrict__ offs, int N, int H, int nh, int window, int V,
                   const float *__restrict__ sq, const float *__restrict__ ks, const float *__restrict__ kzc,
                   const float *__restrict__ vs, float *__restrict__ ctx) {
  using S = AttnTcSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *s_ks = reinterpret_cast<float *>(smem + S::kKs);
  float *s_kzc = reinterpret_cast<float *>(smem + S::kKzc);
  uint64_t *bar_load = reinterpret_cast<uint64_t *>(smem + S::kBar);
  uint64_t *bar_s = bar_load + 1;
  uint64_t *bar_p = bar_load + 2;
  uint64_t *bar_o = bar_load + 3;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + S::kTmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  dep_wait();
  const int4 blk = blocks[blockIdx.x];
  if (blk.w > 2) return;  // a longer key range: attn_tc_long_kernel
  const int s = blk.x, i0 = blk.y, c0 = blk.z, nkt = blk.w;
  const int h = blockIdx.y;
  const int t0 = offs[s];
  const int n = offs[s + 1] - t0;
  const int prow = h * N + t0;  // first row of this sequence in the head plane

  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&mq);
    prefetch_tensormap(&mk);
    prefetch_tensormap(&mv);
    mbar_init(bar_load, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_p, 32 * kAtSoftWarps);
    mbar_init(bar_o, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 256);
  if (warp >= 2) {
    for (int c = threadIdx.x - 64; c < nkt * kAtKT; c += 32 * kAtSoftWarps) {
      const int j = c0 + c;
      s_ks[c] = j < n ? ks[prow + j] : 0.0f;
      s_kzc[c] = __fadd_rn(j < n ? kzc[prow + j] : 0.0f, kMagic);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  dep_trigger();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(bar_load, 8192 + nkt * 16384);
      tma_load_2d(&mq, smem + S::kQ, bar_load, 0, prow + i0);
      for (int kt = 0; kt < nkt; kt++) {
        tma_load_2d(&mk, smem + S::kK + kt * 8192, bar_load, 0, prow + c0 + kt * kAtKT);
        tma_load_2d(&mv, smem + S::kV + kt * 8192, bar_load, 0, prow + c0 + kt * kAtKT);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_u8s8(kAtQ, kAtKT);
      constexpr uint32_t idesc_o = idesc_u8s8(kAtQ, 64) | (1u << 16);  // B (V) MN-major
      if (mbar_wait(bar_load, 0, kDevTimeoutFull)) {
        tc_fence_after();
        const uint32_t q_base = smem_u32(smem + S::kQ);
        for (int kt = 0; kt < nkt; kt++) {
          const uint32_t k_base = smem_u32(smem + S::kK + kt * 8192);
#pragma unroll
          for (int kk = 0; kk < 2; kk++)
            mma_u8s8(tmem + kt * kAtKT, smem_desc_k_sw64(q_base + kk * 32), smem_desc_k_sw64(k_base + kk * 32),
                     idesc_s, kk);
        }
        mma_commit(bar_s);
        if (mbar_wait(bar_p, 0, kDevTimeoutEmpty)) {
          tc_fence_after();
          const uint32_t p_base = smem_u32(smem + S::kP);
          const uint32_t v_base = smem_u32(smem + S::kV);
          for (int kt = 0; kt < nkt; kt++) {
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
              mma_u8s8(tmem, smem_desc_k_sw128(p_base + kt * 16384 + kk * 32),
                       smem_desc_mn_sw64(v_base + (kt * kAtKT + kk * 32) * 64), idesc_o, (kt | kk) != 0);
          }
        }
        mma_commit(bar_o);
      } else {
        mma_commit(bar_s);
        mma_commit(bar_o);
      }
    }
  } else {
    const int q = warp & 3;                // TMEM lane quarter: rows [32q, 32q+32)
    const int g = (warp - 2) >> 2;         // 16-key chunks with parity g
    const int r = q * 32 + lane;
    const int i = i0 + r;
    const bool valid = i < n;
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
    int js = 0, je = n;
    if (window >= 0) {
      js = max(0, i - window);
      je = min(n, i + window + 1);
    }
    const int len = je - js;
    const int body_end = js + (len / V) * V;  // ExpShift: vector body before, exp32 tail after
    ScoreRow w;
    w.a = valid ? js - c0 : 1 << 30;  // valid columns [a, b)
    w.b = valid ? je - c0 : 0;
    w.t0 = valid ? body_end - c0 : 0;
    w.t1 = valid ? je - c0 : 0;
    w.sq = valid ? sq[prow + i] : 0.0f;
    // Columns any row of this warp needs, in 16-key chunks [ch0, ch1).
    const int wa = __reduce_min_sync(0xffffffffu, w.a), wb = __reduce_max_sync(0xffffffffu, w.b);
    const int ch0 = wb > 0 ? wa / 16 : 0, ch1 = wb > 0 ? (wb + 15) / 16 : 0;
    const int nch = nkt * (kAtKT / 16);
    float *red = reinterpret_cast<float *>(smem + S::kRed);  // [2][128] max, then [2][128] P sums
    uint8_t *prow_smem = smem + S::kP + r * 128;
    bool ok = mbar_wait(bar_s, 0, kDevTimeoutAccum);
    ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
    tc_fence_after();
    float mx = -INFINITY;
    if (ok) {
      for (int ch = ch0 + ((ch0 ^ g) & 1); ch < ch1; ch += 2)
        mx = chunk_max<false>(tbase + ch * 16, ch * 16, s_kzc, s_ks, w, mx);
    }
    red[g * 128 + r] = mx;
    named_barrier_sync(1, 32 * kAtSoftWarps);
    mx = fmaxf(red[r], red[128 + r]);
    int psum = 0;
    if (ok) {
      for (int ch = g; ch < nch; ch += 2) {
        uint4 pw = make_uint4(0, 0, 0, 0);
        if (ch >= ch0 && ch < ch1) pw = chunk_p<false>(tbase + ch * 16, ch * 16, s_kzc, s_ks, w, mx, psum);
        // 16 keys = one 16-byte piece of the row's 128-byte swizzle row.
        const int kc = ch >> 3, piece = ch & 7;
        *reinterpret_cast<uint4 *>(prow_smem + kc * 16384 + ((piece ^ (r & 7)) << 4)) = pw;
      }
      if (w.t0 < w.t1)
        psum += tail_fixup(smem + S::kQ, smem + S::kK, 8192, smem + S::kP, r, g, w.t0, w.t1, s_kzc, s_ks, w.sq, mx);
    }
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
    // Output dimensions [32g, 32g+32) of the row.
    uint32_t o[32];
    tmem_ld_32x32b_x32(tbase + 32 * g, o);
    tmem_ld_wait();
    if (ok && valid) {
      const float *vsc = vs + ((size_t)s * nh + h) * 64 + 32 * g;
      float *out = ctx + (size_t)(t0 + i) * H + h * 64 + 32 * g;
#pragma unroll
      for (int d = 0; d < 32; d += 4) {
        const float4 sv = __ldg(reinterpret_cast<const float4 *>(vsc + d));
        *reinterpret_cast<float4 *>(out + d) =
            make_float4(dequant1((int32_t)o[d], 0.0f, sv.x, sp), dequant1((int32_t)o[d + 1], 0.0f, sv.y, sp),
                        dequant1((int32_t)o[d + 2], 0.0f, sv.z, sp), dequant1((int32_t)o[d + 3], 0.0f, sv.w, sp));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}


// ---- key ranges beyond 256 columns: two passes over 128-key tiles --------------
//
// attn_tc_long_kernel handles a 128-query block whose keys span more than two
// tiles (global layers over sequences longer than 256 tokens). The score
// tile S = Q.K^T is computed twice per key tile: a first pass takes MaxOf over
// every valid key of each row, a second recomputes S (the same integer
// accumulators), forms P = rne(exp(s - max) * 255) with ExpShift's
// body/tail split by key position, and accumulates O += P.V in TMEM. P's sum
// and O are integer sums, exact in any order, so the result is the
// single-pass kernel's (and attention8.go's) bit for bit.
//
// One CTA, 10 warps, 256 TMEM columns (S: 0-127, O: 128-191), two CTAs per SM:
//   warp 0     TMA: Q once; per step K (pass 1) or K and V (pass 2) of one
//              key tile into a 3-stage ring.
//   warp 1     MMAs: S per step (after the softmax warps released the
//              previous S), O += P.V per pass-2 step; commits release the
//              ring stages and the P buffers.
//   warps 2-9  as attn_tc_kernel, per tile; P double-buffered in shared memory.
//              After reading a 16-key chunk of S they write the next tile's
//              accumulator presets (0x4B400000 - zc) into it, so the scores
//              come out of TMEM as 1.5*2^23 + (acc - zc) and each needs one
//              subtraction instead of an integer add and a subtraction.
constexpr int kAlStages = 3;

struct AttnLongSmem {
  static constexpr int kQ = 0;                             // [128][64 B] SW64
  static constexpr int kKV = 8192;                         // kAlStages x (K, V) [128][64 B] SW64
  static constexpr int kP = kKV + kAlStages * 16384;       // 2 x [128][128 B] SW128 (1024-aligned)
  static constexpr int kKs = kP + 32768;                   // 3 slots x 128 key scales
  static constexpr int kKzc = kKs + 1536;                  // 3 slots x 128 (kzc + 1.5*2^23)
  static constexpr int kKpre = kKzc + 1536;                // 3 slots x 128 S presets 0x4B400000 - kzc
  static constexpr int kRed = kKpre + 1536;                // [2][128] row maxima, then [2][128] P sums
  static constexpr int kBar = kRed + 2048;                 // 13 mbarriers
  static constexpr int kTmem = kBar + 128;
  static constexpr int kTotal = 100 * 1024;
  static_assert(kP % 1024 == 0, "SW128 P tiles");
  static_assert(kTmem + 16 + 1024 <= kTotal, "shared memory");
};

__global__ void __launch_bounds__(kAtThreads, 2)
    attn_tc_long_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                        const __grid_constant__ CUtensorMap mv, const int4 *__restrict__ blocks,
                        const int32_t *__restrict__ offs, int N, int H, int nh, int window, int V,
                        const float *__restrict__ sq, const float *__restrict__ ks, const float *__restrict__ kzc,
                        const float *__restrict__ vs, float *__restrict__ ctx) {
  using S = AttnLongSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  dep_wait();
  const int4 blk = blocks[blockIdx.x];
  if (blk.w <= 2) return;  // attn_tc_kernel's block
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + S::kBar);
  uint64_t *qfull = bar;               // Q landed
  uint64_t *kfull = bar + 1;           // [kAlStages] stage landed
  uint64_t *kempty = bar + 4;          // [kAlStages] stage released by the MMAs
  uint64_t *sfull = bar + 7;           // S computed
  uint64_t *sfree = bar + 8;           // S read by all softmax warps
  uint64_t *pfull = bar + 9;           // [2] P buffer written
  uint64_t *pfree = bar + 11;          // [2] P buffer read by its P.V
  uint64_t *ofull = bar + 13;          // all P.V done
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + S::kTmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = blk.x, i0 = blk.y, c0 = blk.z, nkt = blk.w;
  const int h = blockIdx.y;
  const int t0 = offs[s];
  const int n = offs[s + 1] - t0;
  const int prow = h * N + t0;  // first row of this sequence in the head plane
  const int steps = 2 * nkt;    // pass 1: tiles 0..nkt-1, pass 2: again

  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&mq);
    prefetch_tensormap(&mk);
    prefetch_tensormap(&mv);
    mbar_init(qfull, 1);
    for (int i = 0; i < kAlStages; i++) {
      mbar_init(&kfull[i], 1);
      mbar_init(&kempty[i], 1);
    }
    mbar_init(sfull, 1);
    mbar_init(sfree, kAtSoftWarps);
    for (int i = 0; i < 2; i++) {
      mbar_init(&pfull[i], kAtSoftWarps);
      mbar_init(&pfree[i], 1);
    }
    mbar_init(ofull, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  dep_trigger();

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(qfull, 8192);
      tma_load_2d(&mq, smem + S::kQ, qfull, 0, prow + i0);
      for (int j = 0; j < steps; j++) {
        const int st = j % kAlStages;
        const uint32_t ph = (uint32_t)(j / kAlStages) & 1;
        if (!mbar_wait(&kempty[st], ph ^ 1, kDevTimeoutEmpty)) break;
        const bool pass2 = j >= nkt;
        const int kt = pass2 ? j - nkt : j;
        uint8_t *stage = smem + S::kKV + st * 16384;
        mbar_arrive_expect_tx(&kfull[st], pass2 ? 16384 : 8192);
        tma_load_2d(&mk, stage, &kfull[st], 0, prow + c0 + kt * kAtKT);
        if (pass2) tma_load_2d(&mv, stage + 8192, &kfull[st], 0, prow + c0 + kt * kAtKT);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_u8s8(kAtQ, kAtKT);
      constexpr uint32_t idesc_o = idesc_u8s8(kAtQ, 64) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(qfull, 0, kDevTimeoutFull);
      const uint32_t q_base = smem_u32(smem + S::kQ);
      const uint32_t p_base = smem_u32(smem + S::kP);
      for (int j = 0; j < steps && ok; j++) {
        const int st = j % kAlStages;
        const uint32_t ph = (uint32_t)(j / kAlStages) & 1;
        const bool pass2 = j >= nkt;
        const int kt = pass2 ? j - nkt : j;
        ok = mbar_wait(&kfull[st], ph, kDevTimeoutFull);
        if (ok) ok = mbar_wait(sfree, (uint32_t)j & 1, kDevTimeoutEmpty);  // S read, next presets in
        if (!ok) break;
        tc_fence_after();
        const uint32_t k_base = smem_u32(smem + S::kKV + st * 16384);
#pragma unroll
        for (int kk = 0; kk < 2; kk++)  // onto the presets
          mma_u8s8(tmem, smem_desc_k_sw64(q_base + kk * 32), smem_desc_k_sw64(k_base + kk * 32), idesc_s, 1);
        mma_commit(sfull);
        if (pass2) {
          const int pb = kt & 1;
          ok = mbar_wait(&pfull[pb], (uint32_t)(kt >> 1) & 1, kDevTimeoutEmpty);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            mma_u8s8(tmem + 128, smem_desc_k_sw128(p_base + pb * 16384 + kk * 32),
                     smem_desc_mn_sw64(k_base + 8192 + kk * 32 * 64), idesc_o, (kt | kk) != 0);
          mma_commit(&pfree[pb]);
        }
        mma_commit(&kempty[st]);
      }
      mma_commit(ofull);
    }
  } else {
    const int q = warp & 3;         // TMEM lane quarter: rows [32q, 32q+32)
    const int g = (warp - 2) >> 2;  // 16-key chunks with parity g
    const int r = q * 32 + lane;
    const int i = i0 + r;
    const bool valid = i < n;
    const int tid = threadIdx.x - 64;  // 0..255
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
    int js = 0, je = n;
    if (window >= 0) {
      js = max(0, i - window);
      je = min(n, i + window + 1);
    }
    const int len = je - js;
    const int body_end = js + (len / V) * V;  // ExpShift: vector body before, exp32 tail after
    const float sqr = valid ? sq[prow + i] : 0.0f;
    float *red = reinterpret_cast<float *>(smem + S::kRed);
    float *ks_slots = reinterpret_cast<float *>(smem + S::kKs);
    float *zcm_slots = reinterpret_cast<float *>(smem + S::kKzc);
    uint32_t *pre_slots = reinterpret_cast<uint32_t *>(smem + S::kKpre);
    // Step j's key terms live in slot j % 3: slot j + 1 is written at the top
    // of step j while other threads may still read slot j - 1 in step j - 1.
    // This thread's key scale (tid < 128) or zero correction of step j's
    // tile, fetched one step ahead so that no step waits on the global load.
    auto key_term = [&](int j) {
      const int kt = j >= nkt ? j - nkt : j;
      const int key = c0 + kt * kAtKT + (tid & 127);
      if (tid < 128) return key < n ? ks[prow + key] : 0.0f;
      return key < n ? kzc[prow + key] : 0.0f;
    };
    auto put_term = [&](int j, float v) {
      const int o = (j % 3) * 128 + (tid & 127);
      if (tid < 128) {
        ks_slots[o] = v;
      } else {
        const float zm = __fadd_rn(v, kMagic);  // zc + 1.5*2^23 for tail_fixup
        zcm_slots[o] = zm;
        pre_slots[o] = 2u * (uint32_t)kMagicBits - __float_as_uint(zm);  // 0x4B400000 - zc
      }
    };
    // Every row's score accumulator of key c starts at 0x4B400000 - zc_c, so
    // that after the MMA it holds the float 1.5*2^23 + (acc - zc) (chunk_max
    // and chunk_p with PRE). The softmax warps write the next tile's presets
    // into each 16-key chunk right after reading it.
    auto preset_chunk = [&](int ch, const uint32_t *pre) {
      uint32_t v[16];
#pragma unroll
      for (int k = 0; k < 16; k += 4) {
        const uint4 u = *reinterpret_cast<const uint4 *>(pre + ch * 16 + k);
        v[k] = u.x, v[k + 1] = u.y, v[k + 2] = u.z, v[k + 3] = u.w;
      }
      tmem_st_32x32b_x16(tbase + ch * 16, v);
    };
    auto release_s = [&]() {  // S read (and the next tile preset) by this warp
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sfree);
    };
    put_term(0, key_term(0));
    float next_term = steps > 1 ? key_term(1) : 0.0f;
    named_barrier_sync(1, 32 * kAtSoftWarps);
    for (int ch = g; ch < kAtKT / 16; ch += 2) preset_chunk(ch, pre_slots);
    release_s();  // sfree phase 0: the first tile's presets
    bool ok = mbar_wait(qfull, 0, kDevTimeoutFull);  // Q in shared memory for tail_fixup
    float mx = -INFINITY;  // pass 1: of (acc - zc) * ks; times sq at its end
    int psum = 0;
    for (int j = 0; j < steps; j++) {
      const bool pass2 = j >= nkt;
      const int kt = pass2 ? j - nkt : j;
      const int st = j % kAlStages;
      const int tb = c0 + kt * kAtKT;  // first key of the tile
      const bool more = j + 1 < steps;
      if (more) {
        put_term(j + 1, next_term);
        if (j + 2 < steps) next_term = key_term(j + 2);
      }
      named_barrier_sync(1, 32 * kAtSoftWarps);
      const float *s_ks = ks_slots + (j % 3) * 128;
      const float *s_kzc = zcm_slots + (j % 3) * 128;
      const uint32_t *pre_next = pre_slots + ((j + 1) % 3) * 128;
      ScoreRow w;
      w.a = valid ? js - tb : 1 << 30;
      w.b = valid ? je - tb : 0;
      w.t0 = valid ? body_end - tb : 0;
      w.t1 = valid ? je - tb : 0;
      w.sq = sqr;
      const int wa = __reduce_min_sync(0xffffffffu, max(w.a, 0)),
                wb = __reduce_max_sync(0xffffffffu, min(w.b, kAtKT));
      const int ch0 = wb > wa ? wa / 16 : 0, ch1 = wb > wa ? (wb + 15) / 16 : 0;
      if (ok) ok = mbar_wait(sfull, (uint32_t)j & 1, kDevTimeoutAccum);
      ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
      tc_fence_after();
      if (!pass2) {
        for (int ch = g; ch < kAtKT / 16; ch += 2) {
          if (ok && ch >= ch0 && ch < ch1) mx = chunk_max<true>(tbase + ch * 16, ch * 16, s_kzc, s_ks, w, mx);
          if (more) preset_chunk(ch, pre_next);
        }
        release_s();
        if (kt == nkt - 1) {  // the row maximum over both parities
          red[g * 128 + r] = mx;
          named_barrier_sync(1, 32 * kAtSoftWarps);
          mx = __fmul_rn(fmaxf(red[r], red[128 + r]), w.sq);
        }
      } else {
        const int pb = kt & 1;
        if (kt >= 2 && ok) ok = mbar_wait(&pfree[pb], (uint32_t)((kt >> 1) & 1) ^ 1, kDevTimeoutEmpty);
        ok = __all_sync(0xffffffffu, ok);
        uint8_t *ptile = smem + S::kP + pb * 16384;
        uint8_t *prow_smem = ptile + r * 128;
        for (int ch = g; ch < kAtKT / 16; ch += 2) {
          uint4 pw = make_uint4(0, 0, 0, 0);
          if (ok && ch >= ch0 && ch < ch1) pw = chunk_p<true>(tbase + ch * 16, ch * 16, s_kzc, s_ks, w, mx, psum);
          *reinterpret_cast<uint4 *>(prow_smem + (((ch & 7) ^ (r & 7)) << 4)) = pw;
          if (more) preset_chunk(ch, pre_next);
        }
        release_s();
        const int ta = max(w.t0, 0), tz = min(w.t1, kAtKT);
        if (ok && ta < tz)
          psum += tail_fixup(smem + S::kQ, smem + S::kKV + st * 16384, 8192, ptile, r, g, ta, tz, s_kzc, s_ks, w.sq,
                             mx);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pfull[pb]);
      }
    }
    int *ired = reinterpret_cast<int *>(red) + 256;
    ired[g * 128 + r] = psum;
    named_barrier_sync(1, 32 * kAtSoftWarps);
    psum = ired[r] + ired[128 + r];
    const float sp = psum > 0 ? __fdiv_rn(1.0f, (float)psum) : 0.0f;
    if (ok) ok = mbar_wait(ofull, 0, kDevTimeoutAccum);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    // Output dimensions [32g, 32g+32) of the row.
    uint32_t o[32];
    tmem_ld_32x32b_x32(tbase + 128 + 32 * g, o);
    tmem_ld_wait();
    if (ok && valid) {
      const float *vsc = vs + ((size_t)s * nh + h) * 64 + 32 * g;
      float *out = ctx + (size_t)(t0 + i) * H + h * 64 + 32 * g;
#pragma unroll
      for (int d = 0; d < 32; d += 4) {
        const float4 sv = __ldg(reinterpret_cast<const float4 *>(vsc + d));
        *reinterpret_cast<float4 *>(out + d) =
            make_float4(dequant1((int32_t)o[d], 0.0f, sv.x, sp), dequant1((int32_t)o[d + 1], 0.0f, sv.y, sp),
                        dequant1((int32_t)o[d + 2], 0.0f, sv.z, sp), dequant1((int32_t)o[d + 3], 0.0f, sv.w, sp));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// A [rows][64 B] plane as TMA tiles of box_rows x 64 B, SWIZZLE_64B.
static int make_map_rows64(CUtensorMap *map, const void *base, int rows, int box_rows) {
  auto enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {64, (cuuint64_t)rows};
  cuuint64_t strides[1] = {64};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

int attn_tc_fits(int n, int i0, int window, int *c0_out, int *nkt_out) {
  int c0 = 0, c1 = n;
  if (window >= 0) {
    c0 = max(0, i0 - window) & ~15;
    c1 = min(n, i0 + kAtQ + window);
  }
  const int width = c1 - c0;
  *c0_out = c0;
  *nkt_out = (width + kAtKT - 1) / kAtKT;  // more than 2: attn_tc_long_kernel
  return 1;
}

int attn_tc_query_block() { return kAtQ; }

// d_blocks: nshort blocks of at most two key tiles (attn_tc_kernel), then
// nlong longer ones (attn_tc_long_kernel).
int launch_attend_tc(const AttnArgs &a, const int4 *d_blocks, int nshort, int nlong, cudaStream_t st) {
  if (nshort + nlong <= 0) return 0;
  if (a.D != 64) return IG_ERR_UNSUPPORTED;
  const int rows = a.nh * a.N;
  CUtensorMap mq, mk, mv;
  if (make_map_rows64(&mq, a.qa, rows, kAtQ) || make_map_rows64(&mk, a.kq, rows, kAtKT) ||
      make_map_rows64(&mv, a.vq, rows, kAtKT))
    return IG_ERR_CUDA;
  static SmemOptIn attr_tc, attr_long;
  if (attr_tc.ensure((const void *)attn_tc_kernel, AttnTcSmem::kTotal) != cudaSuccess ||
      attr_long.ensure((const void *)attn_tc_long_kernel, AttnLongSmem::kTotal) != cudaSuccess)
    return IG_ERR_CUDA;
  if (nshort > 0) {
    if (launch_dep(attn_tc_kernel, dim3(nshort, a.nh), kAtThreads, AttnTcSmem::kTotal, st, mq, mk, mv, d_blocks,
                   a.offs, a.N, a.H, a.nh, a.window, a.V, a.sq, a.ks, a.kzc, a.vs, a.ctx) != cudaSuccess)
      return IG_ERR_CUDA;
  }
  if (nlong > 0) {
    if (launch_dep(attn_tc_long_kernel, dim3(nlong, a.nh), kAtThreads, AttnLongSmem::kTotal, st, mq, mk, mv,
                   d_blocks + nshort, a.offs, a.N, a.H, a.nh, a.window, a.V, a.sq, a.ks, a.kzc, a.vs, a.ctx) !=
        cudaSuccess)
      return IG_ERR_CUDA;
  }
  return 0;
}

}  // namespace ig
