// Device helpers shared by the sm_100a kernels: mbarriers with bounded waits,
// TMA tile loads (no multicast), tcgen05 (TMEM allocation, int8 MMA, commit,
// loads) and the exact float/int conversions the reference's arithmetic needs.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <atomic>
#include <mutex>
#include <utility>

namespace ig {

// Error codes a kernel can leave in g_device_error (first one wins).
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutFull = 1,   // waited too long for a TMA stage
  kDevTimeoutEmpty = 2,  // waited too long for the MMA to release a stage
  kDevTimeoutAccum = 3,  // waited too long for the accumulator
  kDevBadShape = 4,
  kDevBadId = 5,         // an id outside the vocabulary (ig_encode_device)
};

__device__ int g_device_error = 0;  // single translation unit (libindecis_b200.cu)

__device__ __forceinline__ void set_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ----------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Thread-block clusters: all threads of every CTA of the cluster arrive, then
// wait (release / acquire: shared-memory writes before it are visible to the
// cluster's loads after it).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Stores v into CTA `rank`'s shared memory at the offset of p in this CTA's.
__device__ __forceinline__ void st_dsmem_f32(void *p, uint32_t rank, float v) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
// Arrives on the mbarrier at the offset of bar in CTA `rank`'s shared memory,
// releasing this thread's earlier writes (st.shared::cluster included) to
// the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t *bar, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(bar)), "r"(rank));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(a) : "memory");
}
// Asynchronous 4-byte store into CTA `rank`'s shared memory at the offset of
// p, counted as 4 transaction bytes on that CTA's mbarrier at the offset of
// bar (which the receiver arms with arrive.expect_tx): no release fence, so
// the thread's earlier global stores are not waited for.
__device__ __forceinline__ void st_async_f32(float *p, uint32_t rank, float v, uint64_t *bar) {
  uint32_t a, b;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(b) : "r"(smem_u32(bar)), "r"(rank));
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(a),
               "r"(__float_as_uint(v)), "r"(b)
               : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with cluster-scope acquire: the phase's arrivals came from other
// CTAs of the cluster (mbar_arrive_cluster), whose writes become visible.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to ns nanoseconds (or until
// the phase completes) instead of returning at once.
__device__ __forceinline__ bool mbar_try_wait_for(uint64_t *bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up after
// limit_ns (a wait that long means a lost arrival): records `code` in
// g_device_error and returns false so the caller can wind down.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t *bar, uint32_t parity, int code, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
    if (mbar_try_wait_for(bar, parity, 1000000u)) return true;
    if (globaltimer() - t0 > limit_ns) {
      set_device_error(code);
      return false;
    }
  }
}

// The kernels' waits: two seconds.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int code) {
  return mbar_wait_limit(bar, parity, code, 2000000000ull);
}

// mbar_wait for a barrier that other CTAs of the cluster arrive on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 255u) == 0 && globaltimer() - t0 > 2000000000ull) {
      set_device_error(code);
      return false;
    }
  }
}

// ---- TMA ---------------------------------------------------------------------

// 2D tiled load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(const CUtensorMap *map, void *smem_dst, uint64_t *bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 -----------------------------------------------------------------

// Allocates ncols TMEM columns (power of two >= 32); one full warp calls it.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (the layout a SWIZZLE_128B TMA load writes).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                     // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset
  d |= (uint64_t)1 << 46;                     // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                     // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::i8: D int32, A unsigned 8-bit, B signed
// 8-bit, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_u8s8(int M, int N) {
  return (2u << 4)                      // D format: S32
         | (0u << 7)                    // A: unsigned 8-bit
         | (1u << 10)                   // B: signed 8-bit
         | ((uint32_t)(N >> 3) << 17)   // N / 8
         | ((uint32_t)(M >> 4) << 24);  // M / 16
}

// D[tmem] (+)= A[smem] . B[smem]^T, one elected thread issues it.
__device__ __forceinline__ void mma_u8s8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once all previously issued MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM words: thread t gets lane (base + t),
// columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 columns of 32-bit TMEM words.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Generic-proxy shared-memory writes made visible to the async proxy (TMA,
// tensor cores).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 16-byte asynchronous global -> shared copy (cp.async.cg, L2 only), and the
// wait for all of this thread's outstanding copies.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void named_barrier_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Warp stores 32 lanes x 16 columns (32-bit) into TMEM: lane i writes row
// (taddr lane + i), columns [taddr column, +16).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---- exact arithmetic helpers ------------------------------------------------

// Round to nearest even, as VCVTPS2DQ and linalg/int8.go:205-210 roundHalfEven.
// Float -> int32 as VCVTPS2DQ converts under round-to-nearest-even, the
// conversion of the reference's quantRowAVX2 / quantColsAVX2: NaN and values
// outside the int32 range give INT_MIN ("integer indefinite"), where
// __float2int_rn alone would saturate (and give 0 for NaN).
__device__ __forceinline__ int rne_int(float v) {
  return fabsf(v) < 2147483648.0f ? __float2int_rn(v) : (int)0x80000000u;
}

// ((float(acc) - zc) * sb) * sa: the reference's dequant order, no FMA
// (linalg/kernel_vnni_amd64.s:144-200).
__device__ __forceinline__ float dequant1(int32_t acc, float zc, float sb, float sa) {
  float v = __fsub_rn(__int2float_rn(acc), zc);
  v = __fmul_rn(v, sb);
  return __fmul_rn(v, sa);
}

// mixed-sign 4-way byte dot product: a unsigned bytes, b signed bytes.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ---- host: per-device launch settings ------------------------------------------

constexpr int kMaxDevices = 64;

// A kernel's opt-in to more than 48 KB of dynamic shared memory. The attribute
// set by cudaFuncSetAttribute belongs to the current device, so the limit
// already raised is remembered per device ordinal: a process that drives
// several GPUs raises it on each of them. The limit only grows (a launch that
// needs less never lowers it under a concurrent launch that needs more), and
// the raise happens under a lock, so concurrent callers see it done before
// they launch. One static instance per kernel.
struct SmemOptIn {
  std::atomic<int> bytes[kMaxDevices];
  std::mutex mu;
  cudaError_t ensure(const void *fn, int want) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (bytes[dev].load(std::memory_order_acquire) >= want) return cudaSuccess;
    std::lock_guard<std::mutex> lk(mu);
    if (bytes[dev].load(std::memory_order_relaxed) >= want) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
    if (e == cudaSuccess) bytes[dev].store(want, std::memory_order_release);
    return e;
  }
};

// A per-device integer computed once on first use (SM counts, occupancy
// figures); get() runs fn() with the device current. 0 is stored as "unknown".
struct PerDevice {
  std::atomic<int> v[kMaxDevices];
  template <typename F>
  int get(F fn) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return fn();
    int x = v[dev].load(std::memory_order_acquire);
    if (x) return x - 1;
    x = fn();
    v[dev].store(x + 1, std::memory_order_release);
    return x;
  }
};

// ---- programmatic dependent launch ----------------------------------------------
// A kernel launched by launch_dep() may be scheduled while the kernel before it
// in the stream is still running: its CTAs take their SM slots during that
// kernel's last wave and run up to dep_wait(), which returns once that kernel
// has completed and its writes are visible. So the launch latency and the
// ramp of one kernel hide behind the tail of the previous one. Every kernel
// launched this way calls dep_wait() before it reads anything an earlier
// kernel of the stream wrote or writes anything one reads, and calls
// dep_trigger() (after which the next kernel may be scheduled) only after its
// dep_wait() and after it holds its tensor memory: a CTA of the next kernel
// that allocates before its own dep_wait() can then only wait for columns this
// kernel frees, never take ones a CTA of this kernel still has to allocate.
// Without the launch attribute both are no-ops.
__device__ __forceinline__ void dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dep_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// IG_PDL=0 launches every kernel with plain stream order (default: on).
// DepLaunchOff turns it off for the launches of the current thread while it
// lives (stretches that record events between kernels for another stream).
inline thread_local int t_dep_off = 0;
inline bool dep_launch_enabled() {
  static const bool on = [] {
    const char *s = getenv("IG_PDL");
    return !(s && s[0] == '0');
  }();
  return on && t_dep_off == 0;
}
struct DepLaunchOff {
  explicit DepLaunchOff(bool off = true) : on(off) { t_dep_off += on; }
  ~DepLaunchOff() { t_dep_off -= on; }
  DepLaunchOff(const DepLaunchOff &) = delete;
  DepLaunchOff &operator=(const DepLaunchOff &) = delete;
  int on;
};

// The launch attribute that lets the kernel start before its predecessor in
// the stream completes (appended to a launch's attribute list).
inline void add_dep_attr(cudaLaunchAttribute *attrs, unsigned &n) {
  if (!dep_launch_enabled()) return;
  attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[n].val.programmaticStreamSerializationAllowed = 1;
  n++;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_dep(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[1];
  unsigned n = 0;
  add_dep_attr(attrs, n);
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace ig
