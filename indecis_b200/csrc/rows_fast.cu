// Row kernels with the row width fixed at compile time: LayerNorm (+ int8
// quantization) for the reference's V = 8 float32 lanes, and per-row
// quantization of float4-aligned rows. Same arithmetic, in the same order, as
// ln_group_kernel (rows_ln.cu) and quant_row_warp (rows.cu), which restate
// linalg/vec_simd.go:281-327 and linalg/int8.go:157-191.
//
// LayerNorm: a warp takes 4 rows; lane (r, k) = 8r + k holds elements
// k, k+8, ..., k+8(NB-1) of row r in registers, which is exactly the
// reference's lane-k chain, so the ordered sums run without shared memory.
// The 8 partial sums are combined in float64 in lane order through shuffles.
// Quantized bytes go through a small shared buffer so that each row leaves
// in 16-byte stores.
//
// Quantization: for a normal scale s = max/127 (max > 0), |x / s| stays
// below 127 + 2^-20, so rne(x * inv) never needs the int8 clamp and is the
// low byte of RN(x * inv) + (1.5*2^23 + 128) (q + 128). Rows holding a NaN
// (found by a NaN-propagating maximum) and other scales take the clamped
// path, whose conversion follows the reference's (NaN -> INT_MIN).
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "exactmath.cuh"
#include "internal.h"

namespace ig {

// 16-byte-granular bulk copy global -> this CTA's shared memory, completing
// on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// gamma[k + 8b] read through the read-only cache.
struct GammaLdg {
  const float *p;
  __device__ __forceinline__ float operator()(int b) const { return __ldg(p + b * 8); }
};

// The rest of LayerNormRow (+ quantizeA) for the row whose lane-k chain
// values v[b] = x[k + 8b] this lane holds (lane (r, k) of the warp): the
// float64 combines, mean, variance, rstd, gamma (gam(b) = gamma[k + 8b]),
// optional beta and f32 output, and the quantized bytes through the warp's
// shared row buffer sq_row (H + 8 bytes). Every lane of the warp calls it.
template <int NB, class Gamma>
__device__ __forceinline__ void ln8_row_finish(float (&v)[NB], const Gamma &gam, const float *__restrict__ beta,
                                               int r, int k, int row, bool rv, double eps, float *__restrict__ xout,
                                               uint8_t *__restrict__ q, int ldq, float *__restrict__ sa,
                                               uint8_t *sq_row) {
  constexpr int H = 8 * NB;
  float ls = 0.0f;
#pragma unroll
  for (int b = 0; b < NB; b++) ls = __fadd_rn(ls, v[b]);
  double sum = 0.0;
#pragma unroll
  for (int kk = 0; kk < 8; kk++) sum = __dadd_rn(sum, (double)__shfl_sync(0xffffffffu, ls, (r << 3) | kk));
  const float mean = __double2float_rn(__ddiv_rn(sum, (double)H));
  float lq = 0.0f;
#pragma unroll
  for (int b = 0; b < NB; b++) {
    v[b] = __fsub_rn(v[b], mean);
    lq = __fmaf_rn(v[b], v[b], lq);
  }
  double var = 0.0;
#pragma unroll
  for (int kk = 0; kk < 8; kk++) var = __dadd_rn(var, (double)__shfl_sync(0xffffffffu, lq, (r << 3) | kk));
  const float rstd = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(var, (double)H), eps))));
  float mx = 0.0f;  // NaN-propagating here; the NaN-ignoring maximum is taken again below if needed
#pragma unroll
  for (int b = 0; b < NB; b++) {
    v[b] = __fmul_rn(__fmul_rn(v[b], rstd), gam(b));
    if (beta) v[b] = __fadd_rn(v[b], __ldg(beta + k + 8 * b));  // AddTo(o, beta) (SigLIP norms)
    mx = fmax_nan(mx, fabsf(v[b]));
  }
  if (xout && rv) {
    float *dst = xout + (size_t)row * H + k;
#pragma unroll
    for (int b = 0; b < NB; b++) dst[8 * b] = v[b];
  }
  if (!q) return;
  mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
  const bool has_nan = mx != mx;
  if (__any_sync(0xffffffffu, has_nan)) {  // the maximum over the non-NaN values (rows without NaN: the same)
    mx = 0.0f;
#pragma unroll
    for (int b = 0; b < NB; b++) mx = fmaxf(mx, fabsf(v[b]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
  }
  float scale = 0.0f, inv = 0.0f;
  if (mx > 0.0f) {
    scale = __fdiv_rn(mx, 127.0f);
    inv = __fdiv_rn(1.0f, scale);
  }
  if (k == 0 && rv) sa[row] = scale;
  uint8_t *sq = sq_row;
  if (mx == 0.0f) {  // a zero row quantizes to 128s (linalg/int8.go:157-191)
#pragma unroll
    for (int b = 0; b < NB; b++) sq[k + 8 * b] = 128;
  } else if (!has_nan && row_scale_normal(scale)) {
#pragma unroll
    for (int b = 0; b < NB; b++) sq[k + 8 * b] = (uint8_t)__float_as_uint(__fadd_rn(__fmul_rn(v[b], inv), kMagic + 128.0f));
  } else {
#pragma unroll
    for (int b = 0; b < NB; b++) sq[k + 8 * b] = (uint8_t)quant_byte_slow(v[b], inv);
  }
  __syncwarp();
  if (rv) {
    uint8_t *dq = q + (size_t)row * ldq;
    for (int c = k; c < H / 8; c += 8)
      *reinterpret_cast<uint2 *>(dq + 8 * c) = *reinterpret_cast<const uint2 *>(sq + 8 * c);
  }
}

template <int NB, bool EMBED>
__global__ void __launch_bounds__(256) ln8_kernel(const float *__restrict__ x, const int32_t *__restrict__ ids,
                                                  int vocab, const EmbTable emb,
                                                  const float *__restrict__ gamma,
                                                  const float *__restrict__ beta, int M, double eps,
                                                  float *__restrict__ xout, uint8_t *__restrict__ q, int ldq,
                                                  float *__restrict__ sa) {
  constexpr int H = 8 * NB;
  constexpr int QP = H + 8;  // byte pitch: the 4 rows' bytes of one step land in distinct banks
  __shared__ __align__(16) uint8_t s_q[8][4][QP];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 3, k = lane & 7;
  const int row = (blockIdx.x * 8 + warp) * 4 + r;
  const bool rv = row < M;
  dep_wait();
  dep_trigger();
  float v[NB];
  if constexpr (EMBED) {
    int id = rv ? ids[row] : 0;
    if (id < 0 || id >= vocab) {
      set_device_error(kDevBadId);
      id = 0;
    }
    if (emb.fmt == IG_EMB_F32) {
      const float *src = emb.f32 + (size_t)id * H;
#pragma unroll
      for (int b = 0; b < NB; b++) v[b] = rv ? __ldg(src + k + 8 * b) : 0.0f;
    } else {
#pragma unroll
      for (int b = 0; b < NB; b++) v[b] = rv ? emb_elem(emb, id, k + 8 * b, H) : 0.0f;
    }
  } else {
    const float *src = x + (size_t)(rv ? row : 0) * H;
#pragma unroll
    for (int b = 0; b < NB; b++) v[b] = rv ? __ldg(src + k + 8 * b) : 0.0f;
  }
  ln8_row_finish<NB>(v, GammaLdg{gamma + k}, beta, r, k, row, rv, eps, xout, q, ldq, sa, s_q[warp][r]);
}

// ln8_kernel for wide rows (H = 8 NB, NB even), with each lane chain held by
// two threads: lane (r, hf, k) of the warp (two rows a warp, sixteen lanes a
// row) holds x[k + 8b] for b in [hf NB/2, (hf + 1) NB/2). The first half of
// chain k is summed by its hf = 0 thread, which hands the partial sum to the
// hf = 1 thread by a shuffle; that one adds its half in order. So every sum
// is the reference's lane-k chain (linalg/vec_simd.go:281-327), while a
// thread holds half as many values as in ln8_kernel: at H = 768 that is 48
// registers of row data instead of 96, and three times the warps per SM.
// The float64 combines, gamma, the maximum and the bytes follow
// ln8_row_finish. BULK: 4 warps a block, each warp's two rows fetched into
// shared memory by bulk copies, half a row a copy (as ln8_bulk_kernel; the
// halves sit 8 floats apart and the rows 16 floats off a bank multiple, so the
// warp's 32 chain reads hit distinct banks), instead of stride-8 lane loads.
template <int NB, bool BULK>
__global__ void __launch_bounds__(BULK ? 128 : 256) ln8h_kernel(const float *__restrict__ x,
                                                                const float *__restrict__ gamma, int M, double eps,
                                                                float *__restrict__ xout, uint8_t *__restrict__ q,
                                                                int ldq, float *__restrict__ sa) {
  static_assert(NB % 2 == 0, "even chain length");
  constexpr int H = 8 * NB, NH = NB / 2;
  constexpr int QP = H + 8;
  constexpr int kWarps = BULK ? 4 : 8;
  constexpr int HP = H / 2 + 8;  // BULK: float offset of a staged row's second half
  constexpr int RP = 2 * HP;     // BULK: float pitch of the staged rows (16 mod 32)
  static_assert(RP % 32 == 16 && (HP * 4) % 16 == 0, "bank layout, 16-byte copies");
  __shared__ __align__(16) uint8_t s_q[kWarps][2][QP];
  __shared__ __align__(16) float s_x[BULK ? kWarps : 1][BULK ? 2 * RP : 1];
  __shared__ __align__(8) uint64_t s_bar[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 4, hf = (lane >> 3) & 1, k = lane & 7;
  const int row0 = (blockIdx.x * kWarps + warp) * 2, row = row0 + r;
  bool rv = row < M;
  const int b0 = hf * NH;
  if constexpr (BULK) {
    if (lane == 0) {
      mbar_init(&s_bar[warp], 1);
      fence_barrier_init();
    }
    __syncthreads();
  }
  dep_wait();
  dep_trigger();
  float v[NH];
  if constexpr (BULK) {
    const int nr = min(2, M - row0);
    bool ok = true;
    if (nr > 0) {
      if (lane == 0) mbar_arrive_expect_tx(&s_bar[warp], (uint32_t)(nr * H * 4));
      __syncwarp();
      if (lane < 2 * nr)  // lane 2r' + h copies half h of row r'
        bulk_g2s(&s_x[warp][(lane >> 1) * RP + (lane & 1) * HP], x + (size_t)(row0 + (lane >> 1)) * H + (lane & 1) * (H / 2),
                 H * 2, &s_bar[warp]);
      ok = mbar_wait(&s_bar[warp], 0, kDevTimeoutFull);
    }
    rv = rv && ok;
    const float *src = &s_x[warp][r * RP + hf * HP + k];
#pragma unroll
    for (int b = 0; b < NH; b++) v[b] = rv ? src[8 * b] : 0.0f;
  } else {
    const float *src = x + (size_t)(rv ? row : 0) * H + k + 8 * b0;
#pragma unroll
    for (int b = 0; b < NH; b++) v[b] = rv ? __ldg(src + 8 * b) : 0.0f;
  }
  const unsigned full = 0xffffffffu;
  // Lane sums: chain k over b = 0 .. NB-1, its two halves in turn.
  float ls = 0.0f;
  if (hf == 0) {
#pragma unroll
    for (int b = 0; b < NH; b++) ls = __fadd_rn(ls, v[b]);
  }
  const float ls_first = __shfl_sync(full, ls, lane ^ 8);
  if (hf == 1) {
    ls = ls_first;
#pragma unroll
    for (int b = 0; b < NH; b++) ls = __fadd_rn(ls, v[b]);
  }
  double sum = 0.0;
#pragma unroll
  for (int kk = 0; kk < 8; kk++) sum = __dadd_rn(sum, (double)__shfl_sync(full, ls, (r << 4) | 8 | kk));
  const float mean = __double2float_rn(__ddiv_rn(sum, (double)H));
#pragma unroll
  for (int b = 0; b < NH; b++) v[b] = __fsub_rn(v[b], mean);
  float lq = 0.0f;
  if (hf == 0) {
#pragma unroll
    for (int b = 0; b < NH; b++) lq = __fmaf_rn(v[b], v[b], lq);
  }
  const float lq_first = __shfl_sync(full, lq, lane ^ 8);
  if (hf == 1) {
    lq = lq_first;
#pragma unroll
    for (int b = 0; b < NH; b++) lq = __fmaf_rn(v[b], v[b], lq);
  }
  double var = 0.0;
#pragma unroll
  for (int kk = 0; kk < 8; kk++) var = __dadd_rn(var, (double)__shfl_sync(full, lq, (r << 4) | 8 | kk));
  const float rstd = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(var, (double)H), eps))));
  float mx = 0.0f;  // NaN-propagating; the NaN-ignoring maximum is taken again below if needed
#pragma unroll
  for (int b = 0; b < NH; b++) {
    v[b] = __fmul_rn(__fmul_rn(v[b], rstd), __ldg(gamma + k + 8 * (b0 + b)));
    mx = fmax_nan(mx, fabsf(v[b]));
  }
  if (xout && rv) {
    float *dst = xout + (size_t)row * H + k + 8 * b0;
#pragma unroll
    for (int b = 0; b < NH; b++) dst[8 * b] = v[b];
  }
  if (!q) return;
#pragma unroll
  for (int o = 1; o <= 8; o <<= 1) mx = fmax_nan(mx, __shfl_xor_sync(full, mx, o));
  const bool has_nan = mx != mx;
  if (__any_sync(full, has_nan)) {  // the maximum over the non-NaN values (rows without NaN: the same)
    mx = 0.0f;
#pragma unroll
    for (int b = 0; b < NH; b++) mx = fmaxf(mx, fabsf(v[b]));
#pragma unroll
    for (int o = 1; o <= 8; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(full, mx, o));
  }
  float scale = 0.0f, inv = 0.0f;
  if (mx > 0.0f) {
    scale = __fdiv_rn(mx, 127.0f);
    inv = __fdiv_rn(1.0f, scale);
  }
  if (k == 0 && hf == 0 && rv) sa[row] = scale;
  uint8_t *sq = s_q[warp][r] + k + 8 * b0;
  if (mx == 0.0f) {
#pragma unroll
    for (int b = 0; b < NH; b++) sq[8 * b] = 128;
  } else if (!has_nan && row_scale_normal(scale)) {
#pragma unroll
    for (int b = 0; b < NH; b++) sq[8 * b] = (uint8_t)__float_as_uint(__fadd_rn(__fmul_rn(v[b], inv), kMagic + 128.0f));
  } else {
#pragma unroll
    for (int b = 0; b < NH; b++) sq[8 * b] = (uint8_t)quant_byte_slow(v[b], inv);
  }
  __syncwarp();
  if (rv) {
    uint8_t *dq = q + (size_t)row * ldq;
    const uint8_t *sr = s_q[warp][r];
    for (int c = hf * 8 + k; c < H / 8; c += 16)
      *reinterpret_cast<uint2 *>(dq + 8 * c) = *reinterpret_cast<const uint2 *>(sr + 8 * c);
  }
}

// gamma[k + 8b] held in registers for the whole kernel.
template <int NB>
struct GammaRegs {
  float g[NB];
  __device__ __forceinline__ float operator()(int b) const { return g[b]; }
};

// ln8_kernel for row-contiguous f32 rows, persistent: groups of 32 rows are
// staged in shared memory by bulk copies (one per row, a padded row pitch so
// that the lanes' stride-8 chain reads hit distinct banks), three groups in
// flight per CTA, gamma in registers. The same arithmetic as ln8_kernel
// (ln8_row_finish); the global traffic is the rows' bytes, read once, in
// 1 KB copies instead of 32-byte-per-row lane loads.
template <int NB>
struct Ln8Staged {
  static constexpr int H = 8 * NB;
  static constexpr int kRows = 32;
  static constexpr int kStages = 3;
  static constexpr int kPitch = H + 8;  // floats
  static constexpr int kQP = H + 8;     // bytes
  static constexpr int kRowBytes = kStages * kRows * kPitch * 4;
  static constexpr int kQBytes = 8 * 4 * kQP;
  static constexpr int kBar = (kRowBytes + kQBytes + 15) & ~15;
  static constexpr int kTotal = kBar + 8 * kStages;
};

template <int NB>
__global__ void __launch_bounds__(256, 2) ln8_staged_kernel(const float *__restrict__ x,
                                                            const float *__restrict__ gamma,
                                                            const float *__restrict__ beta, int M, double eps,
                                                            float *__restrict__ xout, uint8_t *__restrict__ q,
                                                            int ldq, float *__restrict__ sa) {
  using S = Ln8Staged<NB>;
  constexpr int H = S::H;
  extern __shared__ __align__(128) uint8_t ln_smem[];
  float *rows = reinterpret_cast<float *>(ln_smem);
  uint8_t *s_q = ln_smem + S::kRowBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(ln_smem + S::kBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 3, k = lane & 7;
  const int ngroups = (M + S::kRows - 1) / S::kRows;

  GammaRegs<NB> gam;
#pragma unroll
  for (int b = 0; b < NB; b++) gam.g[b] = __ldg(gamma + k + 8 * b);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; s++) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  dep_wait();

  // Warp 0 stages group grp into stage s: lane i copies row i.
  auto stage = [&](int grp, int s) {
    const int r0 = grp * S::kRows;
    const int nr = min(S::kRows, M - r0);
    if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(nr * H * 4));
    __syncwarp();
    if (lane < nr)
      bulk_g2s(rows + (size_t)(s * S::kRows + lane) * S::kPitch, x + (size_t)(r0 + lane) * H, H * 4, &full[s]);
  };
  if (warp == 0)
    for (int i = 0; i < S::kStages; i++) {
      const int grp = blockIdx.x + i * gridDim.x;
      if (grp < ngroups) stage(grp, i);
    }

  int it = 0;
  for (int grp = blockIdx.x; grp < ngroups; grp += gridDim.x, it++) {
    const int s = it % S::kStages;
    const bool ok = mbar_wait(&full[s], (uint32_t)(it / S::kStages) & 1, kDevTimeoutFull);
    if (!__syncthreads_and(ok)) break;
    const int rl = warp * 4 + r;
    const int row = grp * S::kRows + rl;
    const bool rv = row < M;
    const float *src = rows + (size_t)(s * S::kRows + rl) * S::kPitch + k;
    float v[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) v[b] = rv ? src[8 * b] : 0.0f;
    ln8_row_finish<NB>(v, gam, beta, r, k, row, rv, eps, xout, q, ldq, sa, s_q + (warp * 4 + r) * S::kQP);
    __syncthreads();  // stage s has been read by every warp
    if (warp == 0) {
      const int nxt = grp + S::kStages * gridDim.x;
      if (nxt < ngroups) stage(nxt, s);
    }
  }
  dep_trigger();  // a persistent grid: the next kernel is let in at its end
}

// ln8_kernel with each warp's four rows fetched by bulk copies (one 1 KB copy
// a row into the warp's shared buffer, completing on the warp's mbarrier)
// instead of the lanes' stride-8 loads: those move 32 bytes of a row per
// instruction, four L1 wavefronts for 128 bytes, and kept the L1 at 81% of its
// throughput; the chain reads from shared memory take one wavefront each (row
// pitch H + 8 floats: the four rows' lanes hit distinct banks). The
// arithmetic is ln8_kernel's (ln8_row_finish). EMBED: the rows are float32
// embedding rows gathered by id (an id outside the vocabulary is recorded in
// g_device_error and reads row 0, as ln8_kernel does).
template <int NB, bool EMBED>
__global__ void __launch_bounds__(256) ln8_bulk_kernel(const float *__restrict__ x, const int32_t *__restrict__ ids,
                                                       int vocab, const float *__restrict__ emb,
                                                       const float *__restrict__ gamma,
                                                       const float *__restrict__ beta, int M, double eps,
                                                       float *__restrict__ xout, uint8_t *__restrict__ q, int ldq,
                                                       float *__restrict__ sa) {
  constexpr int H = 8 * NB;
  constexpr int P = H + 8;   // float pitch of the staged rows
  constexpr int QP = H + 8;  // byte pitch of the quantized rows
  __shared__ __align__(16) float s_x[8][4][P];
  __shared__ __align__(16) uint8_t s_q[8][4][QP];
  __shared__ __align__(8) uint64_t s_bar[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 3, k = lane & 7;
  const int row0 = (blockIdx.x * 8 + warp) * 4, row = row0 + r;
  const int nr = min(4, M - row0);  // this warp's rows (<= 0 past the end)
  const bool rv = row < M;
  if (lane == 0) {
    mbar_init(&s_bar[warp], 1);
    fence_barrier_init();
  }
  __syncthreads();
  dep_wait();
  dep_trigger();
  bool ok = true;
  if (nr > 0) {
    if (lane == 0) mbar_arrive_expect_tx(&s_bar[warp], (uint32_t)(nr * H * 4));
    __syncwarp();
    if (lane < nr) {
      const float *src;
      if constexpr (EMBED) {
        int id = ids[row0 + lane];
        if (id < 0 || id >= vocab) {
          set_device_error(kDevBadId);
          id = 0;
        }
        src = emb + (size_t)id * H;
      } else {
        src = x + (size_t)(row0 + lane) * H;
      }
      bulk_g2s(&s_x[warp][lane][0], src, H * 4, &s_bar[warp]);
    }
    ok = mbar_wait(&s_bar[warp], 0, kDevTimeoutFull);
  }
  float v[NB];
#pragma unroll
  for (int b = 0; b < NB; b++) v[b] = rv && ok ? s_x[warp][r][k + 8 * b] : 0.0f;
  ln8_row_finish<NB>(v, GammaLdg{gamma + k}, beta, r, k, row, rv && ok, eps, xout, q, ldq, sa, s_q[warp][r]);
}

static bool ln_bulk_enabled() {
  static const bool on = [] {
    const char *s = getenv("IG_LN_BULK");
    return !(s && s[0] == '0');
  }();
  return on;
}

// One warp per row; lane takes float4 chunks lane, lane + 32, ... (K % 4 == 0).
template <int NJ>
__global__ void __launch_bounds__(256) quant_rows4_kernel(const float *__restrict__ x, int ldx, int M, int K,
                                                          uint8_t *__restrict__ q, int ldq, float *__restrict__ sa) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  dep_wait();
  dep_trigger();
  if (row >= M) return;
  const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)row * ldx);
  const int nq = K >> 2;
  float4 v[NJ];
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int c = lane + 32 * j;
    v[j] = c < nq ? __ldg(src + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
#pragma unroll
  for (int j = 0; j < NJ; j++)
    mx = fmax_nan(fmax_nan(mx, fmax_nan(fabsf(v[j].x), fabsf(v[j].y))), fmax_nan(fabsf(v[j].z), fabsf(v[j].w)));
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const bool has_nan = mx != mx;
  if (has_nan) {  // the maximum over the non-NaN values
    mx = 0.0f;
#pragma unroll
    for (int j = 0; j < NJ; j++)
      mx = fmaxf(fmaxf(mx, fmaxf(fabsf(v[j].x), fabsf(v[j].y))), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  float scale = 0.0f, inv = 0.0f;
  if (mx > 0.0f) {
    scale = __fdiv_rn(mx, 127.0f);
    inv = __fdiv_rn(1.0f, scale);
  }
  const bool zero = mx == 0.0f, fast = !has_nan && row_scale_normal(scale);
  uint8_t *dq = q + (size_t)row * ldq;
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int c = lane + 32 * j;
    if (c >= nq) continue;
    uint32_t w;
    if (zero) {
      w = 0x80808080u;
    } else if (fast) {
      const float2 p0 = __fmul2_rn(make_float2(v[j].x, v[j].y), f2(inv));
      const float2 p1 = __fmul2_rn(make_float2(v[j].z, v[j].w), f2(inv));
      const uint32_t b0 = __float_as_uint(__fadd_rn(p0.x, kMagic + 128.0f));
      const uint32_t b1 = __float_as_uint(__fadd_rn(p0.y, kMagic + 128.0f));
      const uint32_t b2 = __float_as_uint(__fadd_rn(p1.x, kMagic + 128.0f));
      const uint32_t b3 = __float_as_uint(__fadd_rn(p1.y, kMagic + 128.0f));
      w = __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
    } else {
      w = quant_byte_slow(v[j].x, inv) | (quant_byte_slow(v[j].y, inv) << 8) | (quant_byte_slow(v[j].z, inv) << 16) |
          (quant_byte_slow(v[j].w, inv) << 24);
    }
    *reinterpret_cast<uint32_t *>(dq + 4 * c) = w;
  }
  if (lane == 0) sa[row] = scale;
}

// head.logits (heads.go:62-74) for many tokens: z[t][r] = sum_i double(w[r][i])
// * double(x[t][i]) in order, + double(b[r]). One token per thread, its R
// rows side by side. The product of two floats is exact in float64, so the
// fused multiply-add gives the bits of the reference's separate multiply and
// add. The weights are widened to float64 once per block, in shared memory
// ([H][R], read as broadcasts).
template <int R>
__global__ void __launch_bounds__(128) head_logits_tok_kernel(const float *__restrict__ w, const float *__restrict__ b,
                                                              int H, const float *__restrict__ x, int nx,
                                                              double *__restrict__ z, int ldz) {
  extern __shared__ double s_w[];
  dep_wait();
  dep_trigger();
  for (int e = threadIdx.x; e < H * R; e += blockDim.x) {
    const int i = e / R, r = e - i * R;
    s_w[e] = (double)__ldg(w + (size_t)r * H + i);
  }
  __syncthreads();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= nx) return;
  const float4 *xt = reinterpret_cast<const float4 *>(x + (size_t)t * H);
  double s[R];
#pragma unroll
  for (int r = 0; r < R; r++) s[r] = 0.0;
  for (int i4 = 0; i4 < H / 4; i4++) {
    const float4 xv = __ldg(xt + i4);
    const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const double xd = (double)xs[u];
      const double *wr = s_w + (size_t)(4 * i4 + u) * R;
#pragma unroll
      for (int r = 0; r < R; r++) s[r] = __fma_rn(wr[r], xd, s[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) z[(size_t)t * ldz + r] = __dadd_rn(s[r], (double)__ldg(b + r));
}

static int launch_head_logits_tok(const float *w, const float *b, int rows, int H, const float *x, int nx, double *z,
                                  int ldz, cudaStream_t st) {
  if (rows < 1 || rows > 16 || (H & 3) || (reinterpret_cast<uintptr_t>(x) & 15)) return -1;
  const size_t smem = (size_t)H * rows * sizeof(double);
  if (smem > 48 * 1024) return -1;
  // One token a thread, 128 a block (blocks of 32 for small batches, more
  // SMs but four times the weight staging, measured slower: 21 against 17 us
  // a head at 32 sequences).
  const int tpb = 128;
  const int blocks = (nx + tpb - 1) / tpb;
  switch (rows) {
#define IG_HT(R)                                                                                      \
  case R:                                                                                            \
    launch_dep(head_logits_tok_kernel<R>, blocks, tpb, smem, st, w, b, H, x, nx, z, ldz);            \
    break;
    IG_HT(1) IG_HT(2) IG_HT(3) IG_HT(4) IG_HT(5) IG_HT(6) IG_HT(7) IG_HT(8)
    IG_HT(9) IG_HT(10) IG_HT(11) IG_HT(12) IG_HT(13) IG_HT(14) IG_HT(15) IG_HT(16)
#undef IG_HT
  }
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

// LayerNorm (+ quantization) for V = 8 and H in {64, 128, 256}; -1 when this
// path does not apply.
// IG_LN_SPLIT=0 keeps ln8_kernel for H = 768 (the same bits; for comparisons).
static bool ln_split_enabled() {
  static const bool on = [] {
    const char *s = getenv("IG_LN_SPLIT");
    return !(s && s[0] == '0');
  }();
  return on;
}

template <bool EMBED>
static int launch_ln8(const float *x, const int32_t *ids, int vocab, const EmbTable &emb, const float *gamma,
                      const float *beta, int M, int H, double eps, int V, float *xout, uint8_t *q, int ldq, float *sa,
                      cudaStream_t st) {
  if (V != 8 || !gamma) return -1;
  if (q && ((ldq & 7) || (reinterpret_cast<uintptr_t>(q) & 7))) return -1;
  // The staged kernel for the f32-output norm (the final norm): measured at
  // C1 (262,144 rows) 90 us against 108 us for ln8_kernel. With quantized
  // output it ran slower (92 against 82 us: 16 warps per SM, limited by
  // registers and shared memory, hide the row's float64 chain less well than
  // ln8_kernel's 32), so the quantizing norms keep ln8_kernel.
  if (!EMBED && H == 256 && !q && !(reinterpret_cast<uintptr_t>(x) & 15)) {
    using S = Ln8Staged<32>;
    static SmemOptIn attr;
    if (attr.ensure((const void *)ln8_staged_kernel<32>, S::kTotal) != cudaSuccess) return IG_ERR_CUDA;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int groups = (M + S::kRows - 1) / S::kRows;
    const int grid = groups < 2 * sms ? groups : 2 * sms;
    launch_dep(ln8_staged_kernel<32>, grid, 256, S::kTotal, st, x, gamma, beta, M, eps, xout, q, ldq, sa);
    return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
  }
  // The quantizing norms at H = 256 (attn_norm, mlp_norm, and the embedding
  // norm over a float32 table): rows fetched by bulk copies.
  if (H == 256 && q && ln_bulk_enabled() &&
      (EMBED ? emb.fmt == IG_EMB_F32 && !(reinterpret_cast<uintptr_t>(emb.f32) & 15)
             : !(reinterpret_cast<uintptr_t>(x) & 15))) {
    return launch_dep(ln8_bulk_kernel<32, EMBED>, (M + 31) / 32, 256, 0, st, x, ids, vocab, emb.f32, gamma, beta, M,
                      eps, xout, q, ldq, sa) == cudaSuccess
               ? 0
               : IG_ERR_CUDA;
  }
  // Wide rows (H = 768, C4): the split-chain kernel (three times the warps
  // per SM of ln8_kernel<96>, whose 130 registers leave one block per SM).
  if (!EMBED && H == 768 && !beta && ln_split_enabled()) {
    if (ln_bulk_enabled() && !(reinterpret_cast<uintptr_t>(x) & 15))
      launch_dep(ln8h_kernel<96, true>, (M + 7) / 8, 128, 0, st, x, gamma, M, eps, xout, q, ldq, sa);
    else
      launch_dep(ln8h_kernel<96, false>, (M + 15) / 16, 256, 0, st, x, gamma, M, eps, xout, q, ldq, sa);
    return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
  }
  const int blocks = (M + 31) / 32;
#define IG_LN8(NB)                                                                                                 \
  case 8 * NB:                                                                                                     \
    launch_dep(ln8_kernel<NB, EMBED>, blocks, 256, 0, st, x, ids, vocab, emb, gamma, beta, M, eps, xout, q, ldq, \
               sa);                                                                                                \
    break;
  switch (H) {
    IG_LN8(8)
    IG_LN8(16)
    IG_LN8(32)
    IG_LN8(96)
    default:
      return -1;
  }
#undef IG_LN8
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

// Row quantization for K % 4 == 0, K <= 1024, aligned rows; -1 otherwise.
static int launch_quant_rows4(const float *x, int ldx, int M, int K, uint8_t *q, int ldq, float *sa, cudaStream_t st) {
  if ((K & 3) || (ldx & 3) || (ldq & 3) || K > 3072 || K <= 0) return -1;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 3)) return -1;
  const int nj = (K / 4 + 31) / 32;
  const int blocks = (M + 7) / 8;
  switch (nj) {
    case 1: launch_dep(quant_rows4_kernel<1>, blocks, 256, 0, st, x, ldx, M, K, q, ldq, sa); break;
    case 2: launch_dep(quant_rows4_kernel<2>, blocks, 256, 0, st, x, ldx, M, K, q, ldq, sa); break;
    case 3: launch_dep(quant_rows4_kernel<3>, blocks, 256, 0, st, x, ldx, M, K, q, ldq, sa); break;
    case 4: launch_dep(quant_rows4_kernel<4>, blocks, 256, 0, st, x, ldx, M, K, q, ldq, sa); break;
    case 5:
    case 6: launch_dep(quant_rows4_kernel<6>, blocks, 256, 0, st, x, ldx, M, K, q, ldq, sa); break;
    case 7:
    case 8: launch_dep(quant_rows4_kernel<8>, blocks, 256, 0, st, x, ldx, M, K, q, ldq, sa); break;
    default:
      if (nj <= 12)
        launch_dep(quant_rows4_kernel<12>, blocks, 256, 0, st, x, ldx, M, K, q, ldq, sa);
      else if (nj <= 16)
        launch_dep(quant_rows4_kernel<16>, blocks, 256, 0, st, x, ldx, M, K, q, ldq, sa);
      else
        launch_dep(quant_rows4_kernel<24>, blocks, 256, 0, st, x, ldx, M, K, q, ldq, sa);
      break;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig
