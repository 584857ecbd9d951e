// int8 x int8 -> int32 GEMM on the 5th-generation tensor cores (sm_100a),
// replacing the reference's MatMul8N tile loop (linalg/int8.go:88-155 and the
// VPDPBUSD micro-kernels of linalg/kernel_vnni_amd64.s).
//
//   C[i][j] (+)= ((float(acc[i][j]) - zc[j]) * sb[j]) * sa[i]
//   acc[i][j]  = sum_k A[i][k] * B[j][k]      A uint8 (q + 128), B int8
//
// The tensor cores multiply unsigned A by signed B directly (tcgen05
// kind::i8 with A unsigned, B signed), so acc is the reference's own
// offset accumulator and float(acc) rounds exactly as VCVTDQ2PS does.
//
// Structure: one CTA per 128 x BN output tile, 6 warps.
//   warp 0     TMA producer: A and B K-blocks of 128 bytes into a STAGES-deep
//              ring of SWIZZLE_128B shared-memory tiles (no multicast).
//   warp 1     allocates BN TMEM columns; one lane issues tcgen05.mma
//              (M=128, N=BN, K=32) four times per K-block and commits each
//              stage back to the producer.
//   warps 2-5  epilogue: tcgen05.ld 32 lanes x 32 columns per warp quarter
//              (thread = output row), dequantize in the reference's order and
//              apply the fused tail (residual add, RoPE, GeGLU, int32 dump).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "exactmath.cuh"
#include "internal.h"

namespace ig {

constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes of K per stage (one 128-byte swizzle row)
constexpr int kGemmThreads = 192;

template <int BN>
struct GemmSmem {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTiles = kStages * kStageBytes;
  // barriers + tmem slot + per-column scales
  static constexpr int kBarOff = kTiles;
  static constexpr int kMisc = 8 * (2 * kStages + 1) + 16 + 2 * 4 * BN;
  static constexpr int kTotal = kTiles + kMisc + 1024;  // + alignment slack
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_u8s8_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, int M,
                     int N, int K, GemmEpilogue ep) {
  using S = GemmSmem<BN>;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::kBarOff);
  uint64_t *empty = full + kStages;
  uint64_t *accum = empty + kStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
  float *s_sb = reinterpret_cast<float *>(smem + S::kBarOff + 8 * (2 * kStages + 1) + 16);
  float *s_zc = s_sb + BN;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM;
  const int n0 = blockIdx.x * BN;
  const int num_kb = (K + kBK - 1) / kBK;

  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&mapA);
    prefetch_tensormap(&mapB);
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, BN);
  if (EPI != kEpiI32 && warp >= 2) {
    // Column scales of this tile, read once by the epilogue (the int32
    // output has none).
    for (int c = threadIdx.x - 64; c < BN; c += 128) {
      const int j = n0 + c;
      s_sb[c] = j < N ? ep.sb[j] : 0.0f;
      s_zc[c] = j < N ? ep.zc[j] : 0.0f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < num_kb; kb++) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, kDevTimeoutEmpty)) break;
        uint8_t *sa_tile = smem + s * S::kStageBytes;
        uint8_t *sb_tile = sa_tile + S::kABytes;
        mbar_arrive_expect_tx(&full[s], S::kStageBytes);
        tma_load_2d(&mapA, sa_tile, &full[s], kb * kBK, m0);
        tma_load_2d(&mapB, sb_tile, &full[s], kb * kBK, n0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_u8s8(kBM, BN);
      bool ok = true;
      for (int kb = 0; kb < num_kb && ok; kb++) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        if (!mbar_wait(&full[s], ph, kDevTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + s * S::kStageBytes);
        const uint32_t b_base = a_base + S::kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 32; kk++) {
          mma_u8s8(tmem, smem_desc_k_sw128(a_base + kk * 32), smem_desc_k_sw128(b_base + kk * 32), idesc,
                   (kb | kk) != 0);
        }
        mma_commit(&empty[s]);
      }
      mma_commit(accum);
    }
  } else {
    // Epilogue: warp quarter q owns TMEM lanes [32q, 32q+32) = tile rows.
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    const bool vec_ok = (ep.ldc & 3) == 0;  // 16-byte aligned row segments
    const bool row_ok = row < M;
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
    if (mbar_wait(accum, 0, kDevTimeoutAccum)) {
      tc_fence_after();
      const float sa = (EPI != kEpiI32 && row_ok) ? ep.sa[row] : 0.0f;
      if constexpr (EPI == kEpiI32 || EPI == kEpiF32) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          if (!row_ok) continue;
          const int j0 = n0 + c;
          if constexpr (EPI == kEpiI32) {
            int32_t *dst = ep.acc_out + (size_t)row * ep.ldc + j0;
            if (vec_ok && j0 + 32 <= N) {
#pragma unroll
              for (int v = 0; v < 32; v += 4)
                *reinterpret_cast<int4 *>(dst + v) = make_int4(r[v], r[v + 1], r[v + 2], r[v + 3]);
            } else {
#pragma unroll
              for (int v = 0; v < 32; v++)
                if (j0 + v < N) dst[v] = (int32_t)r[v];
            }
          } else {
            float out[32];
#pragma unroll
            for (int v = 0; v < 32; v++) out[v] = dequant1((int32_t)r[v], s_zc[c + v], s_sb[c + v], sa);
            float *dst = ep.C + (size_t)row * ep.ldc + j0;
            if (vec_ok && j0 + 32 <= N) {
#pragma unroll
              for (int v = 0; v < 32; v += 4) {
                float4 o = make_float4(out[v], out[v + 1], out[v + 2], out[v + 3]);
                if (ep.accumulate) {
                  const float4 old = *reinterpret_cast<const float4 *>(dst + v);
                  o.x = __fadd_rn(o.x, old.x);
                  o.y = __fadd_rn(o.y, old.y);
                  o.z = __fadd_rn(o.z, old.z);
                  o.w = __fadd_rn(o.w, old.w);
                }
                *reinterpret_cast<float4 *>(dst + v) = o;
              }
            } else {
#pragma unroll
              for (int v = 0; v < 32; v++)
                if (j0 + v < N) dst[v] = ep.accumulate ? __fadd_rn(out[v], dst[v]) : out[v];
            }
          }
        }
      } else if constexpr (EPI == kEpiGeglu) {
        // Tile columns [0, BN/2) hold GELU inputs, [BN/2, BN) the matching
        // gates (weights interleaved at pack time); output columns
        // [n0/2, n0/2 + BN/2) of a row of ep.geglu_n values (GeluMul,
        // linalg/vec_simd.go:121-160).
        constexpr int H2 = BN / 2;
        const int g0 = n0 / 2;
#pragma unroll 1
        for (int c = 0; c < H2; c += 32) {
          uint32_t ra[32], rg[32];
          tmem_ld_32x32b_x32(tbase + c, ra);
          tmem_ld_32x32b_x32(tbase + H2 + c, rg);
          tmem_ld_wait();
          if (!row_ok) continue;
          float out[32];
#pragma unroll
          for (int v = 0; v < 32; v++) {
            const float a = dequant1((int32_t)ra[v], s_zc[c + v], s_sb[c + v], sa);
            const float g = dequant1((int32_t)rg[v], s_zc[H2 + c + v], s_sb[H2 + c + v], sa);
            out[v] = gelu_mul_at(a, g, g0 + c + v, ep.geglu_n);
          }
          float *dst = ep.C + (size_t)row * ep.ldc + g0 + c;
          if (vec_ok && g0 + c + 32 <= ep.geglu_n) {
#pragma unroll
            for (int v = 0; v < 32; v += 4)
              *reinterpret_cast<float4 *>(dst + v) = make_float4(out[v], out[v + 1], out[v + 2], out[v + 3]);
          } else {
#pragma unroll
            for (int v = 0; v < 32; v++)
              if (g0 + c + v < ep.geglu_n) dst[v] = out[v];
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

// ---- host side ----------------------------------------------------------------

// cuTensorMapEncodeTiled, resolved through the runtime (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// A 2D byte matrix [rows][cols] with row stride ld bytes, tiles of
// box_rows x 128 bytes, 128-byte swizzle, zero fill outside.
static int make_map_u8(CUtensorMap *map, const void *base, int rows, int cols, int ld, int box_rows) {
  auto enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

template <int BN, int EPI>
static cudaError_t launch_bn(const CUtensorMap &ma, const CUtensorMap &mb, int M, int N, int K,
                             const GemmEpilogue &ep, cudaStream_t st) {
  using S = GemmSmem<BN>;
  static SmemOptIn attr;
  cudaError_t e = attr.ensure((const void *)gemm_u8s8_kernel<BN, EPI>, S::kTotal);
  if (e != cudaSuccess) return e;
  dim3 grid((N + BN - 1) / BN, (M + kBM - 1) / kBM);
  gemm_u8s8_kernel<BN, EPI><<<grid, kGemmThreads, S::kTotal, st>>>(ma, mb, M, N, K, ep);
  return cudaGetLastError();
}

// The persistent TMA-store kernel (gemm_persist.cu); -1 when the output does
// not suit it.
static int gemm_persist_try(const GemmArgs &g, const GemmEpilogue &ep, int epi, int bn, const CUtensorMap &ma,
                            const CUtensorMap &mb, cudaStream_t st);

// IG_GEMM_SMALL_TILES=0 keeps 256-column tiles for small products (the same
// bits; for comparisons).
static bool small_m_tiles_enabled() {
  static const bool on = [] {
    const char *s = getenv("IG_GEMM_SMALL_TILES");
    return !(s && s[0] == '0');
  }();
  return on;
}

static int sm_count() {
  static PerDevice sms;
  return sms.get([] {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  });
}

int gemm_u8s8(const GemmArgs &g, const GemmEpilogue &ep, int epi, cudaStream_t st) {
  if (g.M <= 0 || g.N <= 0) return 0;
  if (g.K <= 0 || (g.lda % 16) || (g.ldb % 16) || g.lda < g.K || g.ldb < g.K) return IG_ERR_BAD_ARG;
  if ((reinterpret_cast<uintptr_t>(g.A) | reinterpret_cast<uintptr_t>(g.B)) & 15) return IG_ERR_BAD_ARG;
  int bn = g.bn;
  if (bn != 128 && bn != 256) bn = g.N > 128 ? 256 : 128;
  // Small products (a batch of a few thousand rows): 128-column tiles when
  // 256-column ones would leave SMs without a tile, so every SM shares the
  // epilogue work that bounds such launches.
  if (bn == 256 && small_m_tiles_enabled() && (long long)((g.M + kBM - 1) / kBM) * ((g.N + 255) / 256) < sm_count())
    bn = 128;
  if (epi == kEpiGeglu || epi == kEpiGegluQ) bn = 256;
  CUtensorMap ma, mb;
  if (make_map_u8(&ma, g.A, g.M, g.K, g.lda, kBM) || make_map_u8(&mb, g.B, g.N, g.K, g.ldb, bn))
    return IG_ERR_CUDA;
  const int prc = gemm_persist_try(g, ep, epi, bn, ma, mb, st);
  if (prc != -1) return prc;
  cudaError_t e;
#define IG_GEMM_CASE(E)                                                    \
  case E:                                                                  \
    e = bn == 256 ? launch_bn<256, E>(ma, mb, g.M, g.N, g.K, ep, st)       \
                  : launch_bn<128, E>(ma, mb, g.M, g.N, g.K, ep, st);      \
    break;
  switch (epi) {
    IG_GEMM_CASE(kEpiF32)
    IG_GEMM_CASE(kEpiI32)
    case kEpiGeglu:
      e = launch_bn<256, kEpiGeglu>(ma, mb, g.M, g.N, g.K, ep, st);
      break;
    default:
      return IG_ERR_BAD_ARG;
  }
#undef IG_GEMM_CASE
  return e == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig
