// ig_attention_noalloc: the attention entry point for callers that cannot
// allocate device memory.
//
// ig_attention obtains its work buffers (quantized Q/K/V, their scales, the
// per-sequence statistics and the query-block table) with cudaMalloc on every
// call. Some callers cannot do that: serving processes that reserve all
// device memory when they start and forbid allocations afterwards (a later
// cudaMalloc fails or fragments their pool), and latency-critical paths where
// cudaMalloc/cudaFree would synchronize the device and stall every other
// stream. This variant computes the same result with its work buffers carved
// out of one fixed array compiled into the library:
//
//   * size: kNoAllocScratchBytes (32 MiB) per GPU. The array is part of the
//     library's device image, so every GPU on which the library's kernels are
//     loaded holds it until the process exits. Inputs needing more are
//     rejected with IG_ERR_BAD_ARG before anything is enqueued.
//   * length: the attend kernel keeps each warp's score row in shared
//     memory, so a sequence may hold at most kNoAllocMaxLen (10240) tokens;
//     longer ones are rejected with IG_ERR_UNSUPPORTED before anything is
//     enqueued (ig_attention takes them through its tensor-core kernels).
//   * set-up: the first call on a device, with that device current, looks up
//     the array's device address (cudaGetSymbolAddress) and caches it. Make
//     that first call before any stream capture that contains the entry point.
//   * sharing: every call uses the same array, which keeps the contents the
//     last call left. Every byte a call reads is written by that call first
//     (offsets and block table by the plan kernel, statistics and quantized
//     operands by the prepare kernels), so nothing has to start at zero. Calls
//     whose work overlaps on the GPU (different streams, or different host
//     threads without ordering) race on the array; serialize them on one
//     stream or guard them.
//   * no allocation: no cudaMalloc, cudaFree, pinned or heap allocation; the
//     host work is scalar loops over the offsets and one cudaMemcpyAsync of
//     the offsets (host memory) into the array, which has taken its copy of
//     them when the call returns.
// The call is asynchronous on `stream`: ctx is complete when the stream is.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace ig {

constexpr size_t kNoAllocScratchBytes = 32u << 20;
// The attend kernel's shared memory is kAttnWarps score rows of max_len
// floats plus max_len bytes each, at most 200 KB.
constexpr int kNoAllocMaxLen = 200 * 1024 / (kAttnWarps * 5);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// int64 offsets -> int32 offsets, row -> sequence, and the query-block table
// (the same blocks ig_attention plans on the host). One CTA.
__global__ void noalloc_plan_kernel(const int64_t *__restrict__ offs64, int nseq, int qb, int32_t *__restrict__ offs32,
                                    int32_t *__restrict__ block_start, int32_t *__restrict__ row_seq,
                                    int2 *__restrict__ blocks) {
  if (threadIdx.x == 0) {
    int nb = 0;
    for (int s = 0; s < nseq; s++) {
      offs32[s] = (int32_t)offs64[s];
      block_start[s] = nb;
      nb += (int)((offs64[s + 1] - offs64[s] + qb - 1) / qb);
    }
    offs32[nseq] = (int32_t)offs64[nseq];
  }
  __syncthreads();
  for (int s = threadIdx.x; s < nseq; s += blockDim.x) {
    const int t0 = offs32[s], n = offs32[s + 1] - t0;
    for (int t = 0; t < n; t++) row_seq[t0 + t] = s;
    for (int q0 = 0, b = block_start[s]; q0 < n; q0 += qb, b++) blocks[b] = make_int2(s, q0);
  }
}

static std::mutex g_noalloc_mu;
static void *g_noalloc_base[64];

// The device address of the scratch array on the current device, looked up
// once per device.
static int noalloc_base(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return IG_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_base[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return IG_ERR_CUDA;
    g_noalloc_base[dev] = p;
  }
  *out = g_noalloc_base[dev];
  return 0;
}

}  // namespace ig

extern "C" int ig_attention_noalloc(const float *qkv, int32_t hidden, int32_t heads, const int64_t *offs,
                                    int32_t nseq, int32_t window, int32_t simd_lanes, float *ctx, void *stream) {
  using namespace ig;
  t_last_error.clear();
  if (!qkv || !ctx || !offs || nseq < 0 || heads <= 0 || hidden <= 0 || hidden % heads)
    return fail(IG_ERR_BAD_ARG, "ig_attention_noalloc: bad argument");
  if (offs[0] != 0) return fail(IG_ERR_BAD_ARG, "ig_attention_noalloc: offs[0] must be 0");
  const int qb = attn_query_block();
  long long nblocks = 0;
  int max_len = 0;
  for (int s = 0; s < nseq; s++) {
    const int64_t n = offs[s + 1] - offs[s];
    if (n < 0) return fail(IG_ERR_BAD_ARG, "ig_attention_noalloc: decreasing offsets");
    if (n > max_len) max_len = (int)std::min<int64_t>(n, INT32_MAX);
    nblocks += (n + qb - 1) / qb;
  }
  const int64_t N = offs[nseq];
  if (N == 0) return 0;
  if (max_len > kNoAllocMaxLen)
    return fail(IG_ERR_UNSUPPORTED, "ig_attention_noalloc: a sequence of " + std::to_string(max_len) +
                                        " tokens is longer than the " + std::to_string(kNoAllocMaxLen) +
                                        " this entry point takes; use ig_attention");
  const size_t nh = heads, D = hidden / heads;
  // Carve the scratch: each buffer starts on a 256-byte boundary.
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = (off + 255) / 256 * 256;
    off = o + bytes;
    return o;
  };
  const size_t o_offs64 = take(8 * ((size_t)nseq + 1)), o_offs32 = take(4 * ((size_t)nseq + 1)),
               o_bstart = take(4 * (size_t)nseq), o_rowseq = take(4 * (size_t)N),
               o_blocks = take(sizeof(int2) * (size_t)nblocks), o_qa = take((size_t)N * nh * D),
               o_kq = take((size_t)N * nh * D), o_vq = take((size_t)N * nh * D), o_sq = take(4 * (size_t)N * nh),
               o_ks = take(4 * (size_t)N * nh), o_kzc = take(4 * (size_t)N * nh),
               o_kmean = take(4 * (size_t)nseq * nh * D), o_vs = take(4 * (size_t)nseq * nh * D),
               o_vinv = take(4 * (size_t)nseq * nh * D);
  if (off > kNoAllocScratchBytes)
    return fail(IG_ERR_BAD_ARG, "ig_attention_noalloc: these sequences need " + std::to_string(off) +
                                    " bytes of scratch, more than the " + std::to_string(kNoAllocScratchBytes) +
                                    " built into the library; use ig_attention or split the batch");
  void *base = nullptr;
  if (int rc = noalloc_base(&base)) return fail(rc, "ig_attention_noalloc: cannot locate the scratch array");
  char *b = static_cast<char *>(base);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(b + o_offs64, offs, 8 * ((size_t)nseq + 1), cudaMemcpyHostToDevice, st) != cudaSuccess)
    return fail(IG_ERR_CUDA, "ig_attention_noalloc: copy of the offsets");
  noalloc_plan_kernel<<<1, 256, 0, st>>>(reinterpret_cast<const int64_t *>(b + o_offs64), nseq, qb,
                                         reinterpret_cast<int32_t *>(b + o_offs32),
                                         reinterpret_cast<int32_t *>(b + o_bstart),
                                         reinterpret_cast<int32_t *>(b + o_rowseq),
                                         reinterpret_cast<int2 *>(b + o_blocks));
  if (cudaGetLastError() != cudaSuccess) return fail(IG_ERR_CUDA, "ig_attention_noalloc: plan launch");
  AttnArgs a{};
  a.qkv = qkv;
  a.H = hidden;
  a.nh = heads;
  a.D = (int)D;
  a.offs = reinterpret_cast<const int32_t *>(b + o_offs32);
  a.nseq = nseq;
  a.max_len = max_len;
  a.window = window;
  a.scale = (float)(1.0 / std::sqrt((double)D));
  a.V = simd_lanes;
  a.qa = reinterpret_cast<uint8_t *>(b + o_qa);
  a.sq = reinterpret_cast<float *>(b + o_sq);
  a.kq = reinterpret_cast<int8_t *>(b + o_kq);
  a.ks = reinterpret_cast<float *>(b + o_ks);
  a.kzc = reinterpret_cast<float *>(b + o_kzc);
  a.vq = reinterpret_cast<int8_t *>(b + o_vq);
  a.kmean = reinterpret_cast<float *>(b + o_kmean);
  a.vs = reinterpret_cast<float *>(b + o_vs);
  a.vinv = reinterpret_cast<float *>(b + o_vinv);
  a.row_seq = reinterpret_cast<const int32_t *>(b + o_rowseq);
  a.N = (int)N;
  a.ctx = ctx;
  int rc = launch_attention(a, st);
  if (!rc) rc = launch_attend(a, reinterpret_cast<const int2 *>(b + o_blocks), (int)nblocks, st);
  // As ig_attention: heads with non-finite or overflow-sized Q/K recomputed
  // with the reference's conversions (in the same scratch, nothing allocated).
  if (!rc && a.D == 64) rc = launch_attn_exact(a, st);
  if (rc) return fail(rc, "ig_attention_noalloc: launch failed");
  return 0;
}
