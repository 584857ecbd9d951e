// The BIO decoding of Spans questions on the device (answerSpans then the
// Viterbi pass of decodeSpans, spans.go:172-220 and :293-311, :479-491):
// one warp per text, lane c holding tag c (up to 32 tags: 15 types). For
// each token the warp forms the tempered log-softmax of the tag logits (the
// maximum over the tags, the sum of exponentials in tag order, log), then
// the Viterbi step: every tag takes the best allowed predecessor (the lowest
// tag on ties, as the reference's strict comparison keeps the first), its
// back pointer going to global memory; lane 0 walks the pointers back.
// Passage extraction (byte offsets, punctuation) stays on the host
// (ig_decode_spans / spans.cpp), fed with these tags.
//
// exp and log are CUDA's double-precision functions; they may differ from
// the host's libm (and from Go's math.Exp/Log) in the last bit, so two tag
// sequences whose scores tie to within that would be decided differently.

namespace ig {

__device__ __forceinline__ bool span_inside(int tag) { return tag > 0 && (tag & 1) == 0; }
__device__ __forceinline__ int span_type(int tag) { return (tag - 1) / 2; }

// Go's built-in max on float64 (NaN wins, +0 over -0), for the softmax maximum.
__device__ __forceinline__ double go_max_d(double a, double b) {
  if (a != a || b != b) return __longlong_as_double(0x7ff8000000000000ll);
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}

__global__ void spans_viterbi_kernel(const double *__restrict__ z, long long ldz, const int64_t *__restrict__ offs,
                                     int ntexts, int C, double temperature, double bias, int16_t *__restrict__ back,
                                     int32_t *__restrict__ tags) {
  const int text = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (text >= ntexts) return;
  const long long t0 = offs[text], n = offs[text + 1] - t0;
  if (n <= 0) return;
  const double ninf = -__longlong_as_double(0x7ff0000000000000ll);
  const bool on = lane < C;
  if (temperature <= 0) temperature = 1;
  double cur = ninf;
  for (long long t = 0; t < n; t++) {
    const double v = on ? z[(t0 + t) * ldz + lane] / temperature : ninf;
    // logSoftmax: the maximum (order-free), then the exponentials summed in tag order.
    double mx = ninf;
    for (int c = 0; c < C; c++) mx = go_max_d(mx, __shfl_sync(0xffffffffu, v, c));
    const double e = on ? exp(v - mx) : 0.0;
    double sum = 0.0;
    for (int c = 0; c < C; c++) sum += __shfl_sync(0xffffffffu, e, c);
    const double lse = mx + log(sum);
    const double lp = v - lse;
    const double score = lane > 0 ? lp + bias : lp;
    if (t == 0) {
      cur = (on && !span_inside(lane)) ? score : ninf;
      continue;
    }
    double best = ninf;
    int arg = 0;
    for (int p = 0; p < C; p++) {
      const double cp = __shfl_sync(0xffffffffu, cur, p);
      const bool allowed = !span_inside(lane) || (p > 0 && span_type(p) == span_type(lane));
      if (allowed && cp > best) best = cp, arg = p;
    }
    if (on) back[(t0 + t) * 32 + lane] = (int16_t)arg;
    cur = on ? best + score : ninf;
  }
  // The best final tag (the first of equal scores), then the back pointers.
  int last = 0;
  double bv = __shfl_sync(0xffffffffu, cur, 0);
  for (int c = 1; c < C; c++) {
    const double cv = __shfl_sync(0xffffffffu, cur, c);
    if (cv > bv) bv = cv, last = c;
  }
  __syncwarp();
  if (lane == 0) {
    int tag = last;
    tags[t0 + n - 1] = tag;
    for (long long t = n - 1; t > 0; t--) {
      tag = back[(t0 + t) * 32 + tag];
      tags[t0 + t - 1] = tag;
    }
  }
}

int launch_spans_viterbi(const double *z, long long ldz, const int64_t *d_offs, int ntexts, int C, double temperature,
                         double bias, int16_t *back, int32_t *tags, cudaStream_t st) {
  if (ntexts <= 0) return 0;
  if (C < 1 || C > 32) return IG_ERR_UNSUPPORTED;
  const int warps = 4;
  spans_viterbi_kernel<<<(ntexts + warps - 1) / warps, 32 * warps, 0, st>>>(z, ldz, d_offs, ntexts, C, temperature,
                                                                           bias, back, tags);
  return cudaGetLastError() == cudaSuccess ? 0 : IG_ERR_CUDA;
}

}  // namespace ig

extern "C" {

int ig_spans_tags_device(const double *d_z, int64_t ldz, const int64_t *offs, int32_t ntexts, int32_t ntags,
                         double temperature, double bias, int32_t *d_tags, void *stream) {
  using namespace ig;
  t_last_error.clear();
  if (ntexts < 0 || (ntexts > 0 && (!offs || !d_z || !d_tags)) || ldz < ntags)
    return fail(IG_ERR_BAD_ARG, "indecis: bad span tag arguments");
  if (ntags < 1 || ntags > 32) return fail(IG_ERR_UNSUPPORTED, "indecis: at most 32 tags on the device");
  if (ntexts == 0) return 0;
  if (offs[0] != 0) return fail(IG_ERR_BAD_ARG, "modernbert: inconsistent batch");
  for (int i = 0; i < ntexts; i++)
    if (offs[i + 1] < offs[i]) return fail(IG_ERR_BAD_ARG, "modernbert: inconsistent batch");
  const int64_t ntok = offs[ntexts];
  if (ntok == 0) return 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int64_t *d_offs = nullptr;
  int16_t *back = nullptr;
  IG_CU(cudaMallocAsync(&d_offs, sizeof(int64_t) * (ntexts + 1), st));
  IG_CU(cudaMallocAsync(&back, sizeof(int16_t) * 32 * ntok, st));
  int rc = cudaMemcpyAsync(d_offs, offs, sizeof(int64_t) * (ntexts + 1), cudaMemcpyHostToDevice, st) ? IG_ERR_CUDA : 0;
  if (!rc) rc = launch_spans_viterbi(d_z, ldz, d_offs, ntexts, ntags, temperature, bias, back, d_tags, st);
  cudaFreeAsync(back, st);
  cudaFreeAsync(d_offs, st);
  if (rc) return fail(rc, "indecis: span tag kernel");
  return 0;
}

int ig_spans_tags(const double *z, int64_t ldz, const int64_t *offs, int32_t ntexts, int32_t ntags, double temperature,
                  double bias, int32_t *tags, int32_t device) {
  using namespace ig;
  t_last_error.clear();
  if (ntexts < 0 || (ntexts > 0 && (!offs || !z || !tags))) return fail(IG_ERR_BAD_ARG, "null argument");
  if (ntexts == 0 || offs[ntexts] == 0) return 0;
  DeviceGuard dg(device);
  const int64_t ntok = offs[ntexts];
  cudaStream_t st = nullptr;
  IG_CU(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  double *d_z = nullptr;
  int32_t *d_tags = nullptr;
  int rc = 0;
  if (cudaMallocAsync(&d_z, sizeof(double) * ldz * ntok, st) || cudaMallocAsync(&d_tags, sizeof(int32_t) * ntok, st))
    rc = fail(IG_ERR_CUDA, "indecis: span tag buffers");
  if (!rc && cudaMemcpyAsync(d_z, z, sizeof(double) * ldz * ntok, cudaMemcpyHostToDevice, st))
    rc = fail(IG_ERR_CUDA, "indecis: span logits copy");
  if (!rc) rc = ig_spans_tags_device(d_z, ldz, offs, ntexts, ntags, temperature, bias, d_tags, st);
  if (!rc && cudaMemcpyAsync(tags, d_tags, sizeof(int32_t) * ntok, cudaMemcpyDeviceToHost, st))
    rc = fail(IG_ERR_CUDA, "indecis: span tags copy");
  if (d_z) cudaFreeAsync(d_z, st);
  if (d_tags) cudaFreeAsync(d_tags, st);
  const cudaError_t se = cudaStreamSynchronize(st);
  cudaStreamDestroy(st);
  if (rc) return rc;
  if (se != cudaSuccess) return fail(IG_ERR_CUDA, std::string("indecis: ") + cudaGetErrorString(se));
  return 0;
}

}  // extern "C"
