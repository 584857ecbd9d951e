// Persistent int8 GEMM on CTA pairs (tcgen05 cta_group::2): the arithmetic of
// gemm_persist_kernel, with each output tile of 256 rows x 256 columns
// computed by two CTAs of a cluster on two SMs.
//
// One M = 256 MMA reads A from both CTAs (rows 0-127 from the even CTA,
// 128-255 from the odd one) and B from both (columns 0-127 and 128-255), and
// leaves the 128 x 256 int32 accumulator of its own rows in each CTA's TMEM.
// Per SM and per 128 x 256 x 32 MMA step, shared memory then holds 8 KB of
// operands instead of 12 KB (B is split across the pair), which cuts the
// shared-memory fill traffic that limits the single-CTA kernel on deep K.
//
//   * both CTAs' producers load their halves with TMA (no multicast); every
//     load completes on the even CTA's stage barrier, which expects both
//     halves' bytes;
//   * the even CTA's MMA warp issues the pair MMAs and commits each stage's
//     release and each accumulator's completion to both CTAs' barriers;
//   * each CTA's epilogue warps drain its own TMEM rows exactly as the
//     single-CTA kernel does (epilogue_tile), then arrive on the even CTA's
//     accumulator-empty barrier.
// Every wait is bounded (mbar_wait); the CTAs meet at a cluster barrier
// before the TMEM is released.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"

namespace ig {

// ---- pair helpers (tcgen05 cta_group::2, cluster addressing) -----------------

// The shared::cluster address of p's counterpart in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void *p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}

// Arrive on an mbarrier of another CTA of the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is counted on a
// barrier of either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap *map, void *smem_dst, uint32_t cluster_bar, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void mma_u8s8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on the barrier at cluster address `bar` once every pair MMA this
// thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}

// ---- shared memory -------------------------------------------------------------

template <int EPI>
struct PairSmem {
  static constexpr int kBN = 256;  // tile columns (each CTA holds half of B)
  static constexpr int kEpiWarps = PEpi<EPI>::kWarps;
  static constexpr int kStageBufs = 2;
  static constexpr int kMaxCols = (EPI == kEpiF32 || EPI == kEpiI32) ? 1024 : 0;
  static constexpr int kABytes = kBM * kBK;          // this CTA's 128 rows of A
  static constexpr int kBBytes = (kBN / 2) * kBK;    // this CTA's 128 columns of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagingBytes = kEpiWarps * kStageBufs * 4096;
  static constexpr int kStagesRaw = (224 * 1024 - kStagingBytes - 8 * kMaxCols) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 6 ? 6 : kStagesRaw;
  static constexpr int kStaging = kStages * kStageBytes;
  static constexpr int kCols = kStaging + kStagingBytes;
  static constexpr int kBar = kCols + 8 * kMaxCols;
  static constexpr int kTmemSlot = kBar + 8 * (2 * kStages + 4);
  static constexpr int kTotal = kTmemSlot + 16 + 1024;
  static_assert(kStages >= 2, "two stages at least");
  static_assert(kTotal <= 227 * 1024, "shared memory");
};

template <int EPI>
__global__ void __launch_bounds__(PEpi<EPI>::kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                     const __grid_constant__ CUtensorMap mapC, int M, int N, int K, GemmEpilogue ep) {
  using S = PairSmem<EPI>;
  constexpr int BN = S::kBN;
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
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_n = (N + BN - 1) / BN;
  const int ntiles = ((M + 2 * kBM - 1) / (2 * kBM)) * tiles_n;
  const int num_kb = (K + kBK - 1) / kBK;

  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&mapA);
    prefetch_tensormap(&mapB);
    prefetch_tensormap(&mapC);
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);   // the even CTA's expect_tx; both halves' bytes
      mbar_init(&empty[s], 1);  // one pair commit
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 2 * PEpi<EPI>::kWarps);  // both CTAs' epilogue warps (used on the even CTA)
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, 2 * BN);
  tc_fence_before();
  cluster_sync_all();  // barriers and TMEM of both CTAs exist before any remote use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Everything above touches no global memory an earlier kernel writes.
  dep_wait();

  if (warp == 0) {
    if (lane == 0) {
      int kbg = 0;
      bool ok = true;
      for (int t = pair; t < ntiles && ok; t += npairs) {
        const int m0 = (t / tiles_n) * 2 * kBM + (int)rank * kBM;
        const int n0 = (t % tiles_n) * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < num_kb; kb++, kbg++) {
          const int s = kbg % kStages;
          const uint32_t ph = (kbg / kStages) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t *a = smem + s * S::kStageBytes;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * S::kStageBytes);
          const uint32_t fb = cluster_addr(&full[s], 0);
          tma_load_2d_pair(&mapA, a, fb, kb * kBK, m0);
          tma_load_2d_pair(&mapB, a + S::kABytes, fb, kb * kBK, n0);
        }
      }
      // Wait for the release of every stage in use, so that no commit from
      // the even CTA is still on its way to this CTA's barriers at exit.
      for (int i = 0; i < kStages && ok; i++, kbg++) {
        const int s = kbg % kStages;
        const uint32_t ph = (kbg / kStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, kDevTimeoutEmpty)) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_u8s8(2 * kBM, BN);
      int kbg = 0, it = 0;
      bool ok = true;
      for (int t = pair; t < ntiles && ok; t += npairs, it++) {
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
            mma_u8s8_pair(d, smem_desc_k_sw128(a_base + kk * 32), smem_desc_k_sw128(b_base + kk * 32), idesc,
                          (kb | kk) != 0);
          mma_commit_pair(cluster_addr(&empty[s], 0));
          mma_commit_pair(cluster_addr(&empty[s], 1));
        }
        mma_commit_pair(cluster_addr(&accf[b], 0));
        mma_commit_pair(cluster_addr(&accf[b], 1));
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter
    const int e = warp - 2;  // epilogue warp
    const int g = e >> 2;    // column chunks g, g + kPGroups, ...
    StageWriter<S::kStageBufs> sw{smem + S::kStaging + e * S::kStageBufs * 4096};
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
    for (int t = pair; t < ntiles; t += npairs, it++) {
      const int m0 = (t / tiles_n) * 2 * kBM + (int)rank * kBM, n0 = (t % tiles_n) * BN;
      const int b = it & 1;
      const uint32_t u = (uint32_t)(it >> 1);
      if (!mbar_wait(&accf[b], u & 1, kDevTimeoutAccum)) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < M;
      const int row0 = m0 + q * 32;
      const uint32_t tbase = tmem + b * BN + ((uint32_t)(q * 32) << 16);
      const float sa = (EPI != kEpiI32 && row_ok) ? __ldg(ep.sa + row) : 0.0f;
      // Rows past M (the odd CTA's half of the last tile) hold zeros and are
      // clipped by the TMA store.
      epilogue_tile<BN, EPI, kPGroups, S::kStageBufs>(tbase, n0, N, row0, sa, g, lane, sw, &mapC, eps, M);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&acce[b]);
        else
          mbar_arrive_cluster(cluster_addr(&acce[b], 0));
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  // The next kernel is scheduled once every CTA is here: a persistent grid
  // that let it in at its start would have it wait on the SMs all along.
  dep_trigger();
  cluster_sync_all();  // no remote arrival or MMA write is still on its way
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * BN);
  }
}

// Clusters of two that can be resident at once for this kernel (0: none).
template <int EPI>
static int pair_max_clusters() {
  static PerDevice clusters;
  return clusters.get([] {
    using S = PairSmem<EPI>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(PEpi<EPI>::kThreads, 1, 1);
    cfg.dynamicSmemBytes = S::kTotal;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, gemm_pair_kernel<EPI>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      c = 0;
    }
    return c;
  });
}

template <int EPI>
static cudaError_t launch_pair(const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &mc, int M, int N,
                               int K, const GemmEpilogue &ep, cudaStream_t st, bool *launched) {
  using S = PairSmem<EPI>;
  *launched = false;
  static SmemOptIn smem_attr;
  const cudaError_t se = smem_attr.ensure((const void *)gemm_pair_kernel<EPI>, S::kTotal);
  if (se != cudaSuccess) return se;
  const int maxc = pair_max_clusters<EPI>();
  if (maxc <= 0) return cudaSuccess;  // not launched: the caller takes the single-CTA kernel
  const int ntiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + S::kBN - 1) / S::kBN);
  const int npairs = ntiles < maxc ? ntiles : maxc;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * npairs, 1, 1);
  cfg.blockDim = dim3(PEpi<EPI>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = S::kTotal;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  add_dep_attr(attr, cfg.numAttrs);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_pair_kernel<EPI>, ma, mb, mc, M, N, K, ep);
  if (e == cudaSuccess) *launched = true;
  return e;
}

}  // namespace ig

namespace ig {

// IG_GEMM_PAIR selects the kernel for products with 256-column tiles: "0"
// never the pair kernel, "1" always (tests), unset: deep products (K >= 1024)
// with enough rows to give every SM pair tiles. Measured on B200 with f32
// output: K = 3072 (768 columns) 8% faster than the single-CTA kernel, K =
// 1152 3% faster, K = 768 with 2304-3072 columns 10% slower (there the f32
// store stream bounds both kernels, and the pair couples two SMs' epilogues).
static bool pair_wanted(const GemmArgs &g) {
  const char *s = getenv("IG_GEMM_PAIR");
  if (s && s[0] == '0') return false;
  if (s && s[0] == '1') return true;
  return g.K >= 1024 && g.N >= 256 && g.M >= 8192;
}

// The pair kernel for this product, or -1 when it is not taken (then the
// single-CTA persistent kernel runs).
static int gemm_pair_try(const GemmArgs &g, const GemmEpilogue &ep, int epi, const CUtensorMap &ma,
                         const CUtensorMap &mc, cudaStream_t st) {
  if (!pair_wanted(g)) return -1;
  CUtensorMap mb;
  if (make_map_u8(&mb, g.B, g.N, g.K, g.ldb, kBM)) return IG_ERR_CUDA;
  bool launched = false;
  cudaError_t e;
  switch (epi) {
    case kEpiF32: e = launch_pair<kEpiF32>(ma, mb, mc, g.M, g.N, g.K, ep, st, &launched); break;
    case kEpiI32: e = launch_pair<kEpiI32>(ma, mb, mc, g.M, g.N, g.K, ep, st, &launched); break;
    case kEpiF32Bias: e = launch_pair<kEpiF32Bias>(ma, mb, mc, g.M, g.N, g.K, ep, st, &launched); break;
    case kEpiGeluTanh: e = launch_pair<kEpiGeluTanh>(ma, mb, mc, g.M, g.N, g.K, ep, st, &launched); break;
    case kEpiOutlierRes: e = launch_pair<kEpiOutlierRes>(ma, mb, mc, g.M, g.N, g.K, ep, st, &launched); break;
    case kEpiGeglu: e = launch_pair<kEpiGeglu>(ma, mb, mc, g.M, g.N, g.K, ep, st, &launched); break;
    default: return -1;
  }
  if (e != cudaSuccess) return IG_ERR_CUDA;
  return launched ? 0 : -1;
}

}  // namespace ig
