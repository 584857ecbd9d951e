// Host runtime behind include/indecis_b200.h: model creation (upload and
// on-device weight quantization), a per-device workspace pool, and the
// encoder's launch sequence, which replaces internal/modernbert/infer.go:304-430
// (run) layer for layer:
//
//   embed + LN(emb_norm) + quant           infer.go:361-368
//   per layer l:
//     [l > 0] LN(attn_norm) + quant        infer.go:384-389
//     QKV GEMM, RoPE fused in the epilogue infer.go:390-399
//     attention (stats, quant, attend)     infer.go:401, :484-518
//     quant(ctx); Wo GEMM, x += fused      infer.go:403
//     LN(mlp_norm) + quant                 infer.go:404-406
//     Wi GEMM, GeGLU fused in the epilogue infer.go:416-419
//     quant(g); WoMLP GEMM, x += fused     infer.go:423
//   LN(final_norm), pooling                infer.go:427, :261-289
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <deque>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace ig {


static thread_local std::string t_last_error;

static int fail(int code, const std::string &msg) {
  t_last_error = msg;
  return code;
}

// Error reporting for the host-only entry points built in their own object
// (spans.cpp): one last-error slot per thread for the whole library.
int report_error(int code, const std::string &msg) { return fail(code, msg); }
void clear_error() { t_last_error.clear(); }

// Pooled by the mean of each sequence's rows whatever the config's pooling
// (meanRows, spans.go:464-477); internal to ig_window_logits.
constexpr int kModeMeanRows = 2;

#define IG_CU(x)                                                                         \
  do {                                                                                   \
    cudaError_t e_ = (x);                                                                \
    if (e_ != cudaSuccess) return fail(IG_ERR_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

#define IG_TRY(x)                                                                \
  do {                                                                           \
    int r_ = (x);                                                                \
    if (r_) {                                                                    \
      if (t_last_error.empty()) t_last_error = std::string("failed: ") + #x;     \
      return r_;                                                                 \
    }                                                                            \
  } while (0)

static inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---- kernel profiling (ig_profile / ig_profile_report) ----------------------
// When enabled, every launch site of the encoder brackets its kernels with a
// pair of CUDA events on the launching stream and records the algorithmic
// bytes and integer/float operations of the launch (computed from its
// shapes), so a caller can derive achieved bandwidth or throughput per kernel.
struct ProfRec {
  const char *name;
  cudaEvent_t a, b;
  double bytes, ops;
  int launches;
};

struct Profiler {
  std::mutex mu;
  bool on = false;
  std::string only;  // when set, only launches recorded under this name get events
  std::vector<ProfRec> recs;
  std::vector<cudaEvent_t> pool;
  cudaEvent_t get() {
    std::lock_guard<std::mutex> lk(mu);
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
};
static Profiler g_prof;
static std::atomic<long long> g_launches{0};
static thread_local long long t_launches = 0;  // this thread's share of g_launches
static std::atomic<long long> g_graph_runs{0}, g_graph_records{0};  // since the library loaded

struct ProfScope {
  bool on = false;
  ProfRec r{};
  cudaStream_t st = nullptr;
  ProfScope(const char *name, double bytes, double ops, int launches, cudaStream_t s, bool capturing = false) {
    g_launches += launches;
    t_launches += launches;
    on = g_prof.on && !capturing && (g_prof.only.empty() || g_prof.only == name);
    if (!on) return;
    st = s;
    r = ProfRec{name, g_prof.get(), g_prof.get(), bytes, ops, launches};
    cudaEventRecord(r.a, st);
  }
  ~ProfScope() {
    if (!on) return;
    cudaEventRecord(r.b, st);
    std::lock_guard<std::mutex> lk(g_prof.mu);
    g_prof.recs.push_back(r);
  }
};

struct DevMat {
  int8_t *q = nullptr;
  float *scale = nullptr, *zc = nullptr;
  int n = 0, k = 0, ld = 0;
};

struct DevLayer {
  DevMat qkv, o, wi, wom;
  float *attn_norm = nullptr, *mlp_norm = nullptr;
  // float32 weights [out][in] for the path without SetInt8
  float *fqkv = nullptr, *fo = nullptr, *fwi = nullptr, *fwom = nullptr;
};

struct DevHead {
  int rows = 0, per_token = 0;
  float *w = nullptr, *b = nullptr;
};

// Host-side plan of one call: offsets, row -> sequence, positions, and for
// each attention kind (0 global, 1 local) the 128-query blocks the tensor-core
// kernel takes (x seq, y first query, z first key, w key tiles) and the
// 16-query blocks of the wider key ranges it leaves to attn_attend_kernel.
struct Plan {
  int nseq = 0, N = 0, max_len = 0;
  std::vector<int32_t> offs, row_seq, pos;
  std::vector<int4> tc[2];  // blocks of at most two key tiles first, then the longer ones, longest first
  int tc_short[2] = {0, 0};  // how many of tc[k] have at most two key tiles
  std::vector<int2> v1[2];
  std::vector<int2> fb;  // float path: (sequence, first query) of each block of 64 queries
  size_t block_bytes() const {
    return 16 * (tc[0].size() + tc[1].size()) + 8 * (v1[0].size() + v1[1].size() + fb.size());
  }
};

// Device copies of the plan's block lists (inside the workspace).
struct PlanDev {
  const int4 *tc[2] = {nullptr, nullptr};
  const int2 *v1[2] = {nullptr, nullptr};
  int ntc[2] = {0, 0}, ntc_short[2] = {0, 0}, nv1[2] = {0, 0};
  const int2 *fb = nullptr;
  int nfb = 0;
};

// Device buffers of one encode call, sized for `rows` rows and `nseq` sequences.
struct Workspace {
  int device = 0;
  size_t rows_cap = 0, seq_cap = 0, blk_cap = 0, tl_cap = 0, pl_cap = 0;
  bool f32_cap = false;  // holds the float path's MLP buffer
  float *zf = nullptr;   // float path: [rows][2I] Wi output
  void *dev = nullptr;
  void *host = nullptr;  // pinned staging
  size_t host_bytes = 0;
  void *ohost = nullptr;  // pinned staging of a host call's large outputs
  size_t ohost_bytes = 0;
  std::vector<cudaEvent_t> pev;  // one per staged piece: its device-to-host copy finished
  std::vector<cudaEvent_t> cev;  // one per output chunk: computed on own_stream
  cudaStream_t copy_stream = nullptr;  // device-to-host copies that overlap the last kernels
  cudaStream_t own_stream = nullptr;
  cudaEvent_t done = nullptr;
  int32_t *ids, *offs, *row_seq, *pos;
  char *blocks;  // PlanDev lists
  PlanDev pd;
  uint64_t gen = 0;  // bumped whenever the device buffers move
  int32_t *err_host = nullptr;  // pinned copy of the device error flag at the end of a host call
  // A host call's kernels recorded as a CUDA graph (run_graphed): the call's
  // key (offsets, mode, outputs), the model version and buffer generation it
  // was recorded with, and its kernel count; `seen` is the previous call's key.
  std::vector<int64_t> graph_key, seen;
  uint64_t graph_ver = 0, graph_gen = 0;
  long long graph_launches = 0;
  cudaGraphExec_t graph = nullptr;
  float *x, *xn, *sa, *qkv, *ctx, *g, *sq, *ks, *kzc, *kmean, *vs, *vinv, *pooled;
  float *sg;  // row scales of the quantized GeGLU output (kEpiGegluQ; its bytes go over g)
  uint8_t *xq, *qa;
  int8_t *kq, *vq;
  double *logits, *tlogits;
  ~Workspace() {
    if (err_host) cudaFreeHost(err_host);
    if (graph) cudaGraphExecDestroy(graph);
    if (dev) cudaFree(dev);
    if (host) cudaFreeHost(host);
    if (ohost) cudaFreeHost(ohost);
    for (cudaEvent_t e : pev) cudaEventDestroy(e);
    for (cudaEvent_t e : cev) cudaEventDestroy(e);
    if (copy_stream) cudaStreamDestroy(copy_stream);
    if (done) cudaEventDestroy(done);
    if (own_stream) cudaStreamDestroy(own_stream);
  }
};

// Stored elements -> float32, exactly as the reference decodes them on read
// (safetensors decode, safetensors/safetensors.go:218-245): BF16 is the
// high half of the float32 bits; F16 is IEEE binary16 widened exactly (signed
// zeros, subnormals scaled by 2^-24, infinities and NaNs with their payload
// moved to the top of the float32 mantissa); I8 is the integer's value.
__global__ void widen_kernel(const void *__restrict__ src, int dtype, size_t n, float *__restrict__ dst) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float v;
    if (dtype == IG_DT_BF16) {
      v = __uint_as_float((uint32_t)static_cast<const uint16_t *>(src)[i] << 16);
    } else if (dtype == IG_DT_F16) {
      const uint32_t h = static_cast<const uint16_t *>(src)[i];
      const uint32_t sign = (h >> 15) << 31, e = (h >> 10) & 0x1f, f = h & 0x3ff;
      if (e == 0) {
        v = __uint_as_float(sign | __float_as_uint(__fmul_rn((float)f, 0x1p-24f)));  // zero or subnormal: exact
      } else if (e == 0x1f) {
        v = __uint_as_float(sign | 0x7f800000u | (f << 13));
      } else {
        v = __uint_as_float(sign | ((e + 112) << 23) | (f << 13));
      }
    } else {
      v = (float)static_cast<const int8_t *>(src)[i];
    }
    dst[i] = v;
  }
}

}  // namespace ig

using namespace ig;

struct ig_model {
  ig_config cfg{};
  int device = 0;
  int H = 0, I = 0, nh = 0, D = 0, ldk = 0, NI = 0;
  EmbTable emb{-1, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};  // fmt -1: no table yet
  std::vector<void *> emb_allocs;  // the table's device arrays (replaced by ig_model_set_embeddings)
  float *emb_norm = nullptr, *final_norm = nullptr;
  std::vector<DevLayer> layers;
  bool f32 = false;  // SetInt8(false): the float32 path
  std::mutex mu;  // rope tables, heads, workspace pool
  int rope_npos = 0;
  float *rope_cos[2] = {nullptr, nullptr}, *rope_sin[2] = {nullptr, nullptr};
  std::vector<void *> retired;  // rope tables replaced by longer ones
  std::vector<DevHead> heads;
  std::vector<std::unique_ptr<Workspace>> pool;
  std::vector<void *> allocs;
  // A model on several GPUs (ig_model_create_multi): one replica per device,
  // owned; the group itself holds no device memory.
  std::vector<ig_model *> replicas;
  std::atomic<int> inflight{0};  // host calls running on this model (shard placement)
  // Bumped by every change a recorded graph depends on (embedding table,
  // heads, SetInt8, RoPE tables): graphs of an older version are re-recorded.
  std::atomic<uint64_t> version{0};
  ~ig_model() {
    if (!replicas.empty()) {
      for (ig_model *r : replicas) delete r;
      return;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaDeviceSynchronize();
    pool.clear();
    for (void *p : allocs) cudaFree(p);
    for (void *p : emb_allocs) cudaFree(p);
    for (void *p : retired) cudaFree(p);
    for (auto &h : heads) {
      cudaFree(h.w);
      cudaFree(h.b);
    }
    cudaSetDevice(prev);
  }
};

namespace {

struct DeviceGuard {
  int prev = 0;
  explicit DeviceGuard(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~DeviceGuard() { cudaSetDevice(prev); }
};

template <class T>
int dev_alloc(ig_model *m, T **p, size_t count) {
  void *v = nullptr;
  IG_CU(cudaMalloc(&v, std::max<size_t>(count * sizeof(T), 16)));
  m->allocs.push_back(v);
  *p = reinterpret_cast<T *>(v);
  return 0;
}

int upload(ig_model *m, float **dst, const float *src, size_t count) {
  IG_TRY(dev_alloc(m, dst, count));
  IG_CU(cudaMemcpy(*dst, src, count * sizeof(float), cudaMemcpyHostToDevice));
  return 0;
}

// Quantizes a float32 [n][k] device matrix into a DevMat with n_out packed
// rows (perm chooses their source rows).
int pack_matrix(ig_model *m, DevMat &dm, const float *d_w, int n, int k, const std::vector<int32_t> &perm,
                int32_t *d_perm) {
  const int n_out = perm.empty() ? n : (int)perm.size();
  dm.n = n_out;
  dm.k = k;
  dm.ld = (int)align_up(k, 16);
  IG_TRY(dev_alloc(m, &dm.q, (size_t)n_out * dm.ld));
  IG_TRY(dev_alloc(m, &dm.scale, n_out));
  IG_TRY(dev_alloc(m, &dm.zc, n_out));
  if (!perm.empty()) IG_CU(cudaMemcpy(d_perm, perm.data(), perm.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
  IG_TRY(launch_pack_b8(d_w, n, k, perm.empty() ? nullptr : d_perm, n_out, dm.q, dm.ld, dm.scale, dm.zc, nullptr,
                        0));
  IG_CU(cudaDeviceSynchronize());
  return 0;
}

// A host tensor as its safetensors file stores it.
struct TensorView {
  int dtype;  // IG_DT_*
  const void *data;
};

size_t dtype_size(int dtype) {
  return dtype == IG_DT_F32 ? 4 : dtype == IG_DT_I8 ? 1 : 2;
}

// Fills n float32 elements of device memory from a stored host tensor; stage
// is a device buffer of at least 2n bytes for the narrow formats.
int fetch_f32(float *dst, const TensorView &t, size_t n, void *stage) {
  if (!t.data) return fail(IG_ERR_BAD_ARG, "modernbert: tensor missing");
  if (t.dtype == IG_DT_F32) {
    IG_CU(cudaMemcpy(dst, t.data, n * sizeof(float), cudaMemcpyHostToDevice));
    return 0;
  }
  if (t.dtype != IG_DT_BF16 && t.dtype != IG_DT_F16 && t.dtype != IG_DT_I8)
    return fail(IG_ERR_BAD_ARG, "unsupported dtype " + std::to_string(t.dtype));
  IG_CU(cudaMemcpy(stage, t.data, n * dtype_size(t.dtype), cudaMemcpyHostToDevice));
  widen_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256>>>(stage, t.dtype, n, dst);
  IG_CU(cudaGetLastError());
  return 0;
}

int upload_view(ig_model *m, float **dst, const TensorView &t, size_t count, void *stage) {
  IG_TRY(dev_alloc(m, dst, count));
  return fetch_f32(*dst, t, count, stage);
}

// The weights a model is made from: every tensor as its file stores it.
struct WeightSource {
  const float *tok_embeddings;  // float32 table, or NULL
  TensorView emb_norm, final_norm;
  std::vector<TensorView> attn_norm, wqkv, wo, mlp_norm, wi, wo_mlp;
};

// RoPE cos/sin of the reference's table (internal/modernbert/model.go:255-277),
// computed on the host in float64 as there, for npos positions.
void rope_table_host(double theta, int D, int npos, std::vector<float> &cs, std::vector<float> &sn) {
  const int half = D / 2;
  cs.assign((size_t)npos * half, 0.0f);
  sn.assign((size_t)npos * half, 0.0f);
  for (int i = 0; i < half; i++) {
    const float inv = (float)(1.0 / std::pow(theta, (double)(2 * i) / (double)D));
    for (int p = 0; p < npos; p++) {
      const double f = (double)((float)p * inv);
      cs[(size_t)p * half + i] = (float)std::cos(f);
      sn[(size_t)p * half + i] = (float)std::sin(f);
    }
  }
}

int ensure_rope(ig_model *m, int npos) {
  std::lock_guard<std::mutex> lk(m->mu);
  if (m->rope_npos >= npos) return 0;
  const int n = std::max(npos, std::max(512, m->rope_npos * 2));
  const double thetas[2] = {m->cfg.global_theta, m->cfg.local_theta};
  for (int t = 0; t < 2; t++) {
    std::vector<float> cs, sn;
    rope_table_host(thetas[t], m->D, n, cs, sn);
    float *dc = nullptr, *ds = nullptr;
    IG_CU(cudaMalloc(&dc, cs.size() * sizeof(float)));
    IG_CU(cudaMalloc(&ds, sn.size() * sizeof(float)));
    IG_CU(cudaMemcpy(dc, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice));
    IG_CU(cudaMemcpy(ds, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice));
    // The old tables may still be read by enqueued work: retire, free at destroy.
    if (m->rope_cos[t]) m->retired.push_back(m->rope_cos[t]);
    if (m->rope_sin[t]) m->retired.push_back(m->rope_sin[t]);
    m->rope_cos[t] = dc;
    m->rope_sin[t] = ds;
  }
  m->rope_npos = n;
  m->version++;
  return 0;
}

// windows[k]: the half window of attention kind k (-1: global); kinds whose
// window is < -1 are not planned.
// Checks a batch's offsets (the errors of run's batch checks) and returns
// its row count and longest sequence.
int scan_offsets(const int64_t *offs, int nseq, int64_t *rows, int *max_len) {
  if (nseq < 0 || !offs) return fail(IG_ERR_BAD_ARG, "modernbert: inconsistent batch");
  if (offs[0] != 0) return fail(IG_ERR_BAD_ARG, "modernbert: offs[0] must be 0");
  const int64_t N = offs[nseq];
  if (N < 0 || N > (int64_t)INT32_MAX / 4) return fail(IG_ERR_BAD_ARG, "modernbert: batch too large");
  int64_t ml = 0;
  for (int s = 0; s < nseq; s++) {
    if (offs[s + 1] < offs[s]) return fail(IG_ERR_BAD_ARG, "modernbert: decreasing offsets");
    ml = std::max(ml, offs[s + 1] - offs[s]);
  }
  *rows = N;
  *max_len = (int)ml;
  return 0;
}

// host_rows: also the row -> sequence and position tables on the host (the
// encoder paths fill them on the device from the offsets instead).
int make_plan(const int64_t *offs, int nseq, Plan &p, const int (&windows)[2], bool host_rows = false) {
  int64_t N = 0;
  int ml = 0;
  IG_TRY(scan_offsets(offs, nseq, &N, &ml));
  p.nseq = nseq;
  p.N = (int)N;
  p.offs.resize(nseq + 1);
  p.row_seq.resize(host_rows ? N : 0);
  p.pos.resize(host_rows ? N : 0);
  for (int k = 0; k < 2; k++) {
    p.tc[k].clear();
    p.v1[k].clear();
  }
  p.fb.clear();
  p.max_len = 0;
  const int qb = attn_query_block();
  for (int s = 0; s < nseq; s++) {
    p.offs[s] = (int32_t)offs[s];
    const int n = (int)(offs[s + 1] - offs[s]);
    p.max_len = std::max(p.max_len, n);
    if (host_rows)
      for (int t = 0; t < n; t++) {
        p.row_seq[offs[s] + t] = s;
        p.pos[offs[s] + t] = t;
      }
    for (int i0 = 0; i0 < n; i0 += 64) p.fb.push_back(make_int2(s, i0));
    for (int k = 0; k < 2; k++) {
      if (windows[k] < -1) continue;
      for (int i0 = 0; i0 < n; i0 += attn_tc_query_block()) {
        int c0 = 0, nkt = 0;
        if (attn_tc_fits(n, i0, windows[k], &c0, &nkt)) {
          p.tc[k].push_back(make_int4(s, i0, c0, nkt));
        } else {
          for (int q0 = i0; q0 < std::min(n, i0 + attn_tc_query_block()); q0 += qb) p.v1[k].push_back(make_int2(s, q0));
        }
      }
    }
  }
  p.offs[nseq] = (int32_t)N;
  // attn_tc_kernel takes the first tc_short blocks and attn_tc_long_kernel the
  // rest, each with a grid of its own blocks; the long ones in decreasing key
  // tile count, so that the longest CTAs start first.
  for (int k = 0; k < 2; k++) {
    auto mid = std::stable_partition(p.tc[k].begin(), p.tc[k].end(), [](const int4 &b) { return b.w <= 2; });
    p.tc_short[k] = (int)(mid - p.tc[k].begin());
    std::stable_sort(mid, p.tc[k].end(), [](const int4 &x, const int4 &y) { return x.w > y.w; });
  }
  return 0;
}

struct Carve {
  char *base;
  size_t off = 0;
  template <class T>
  T *take(size_t count) {
    off = align_up(off, 256);
    T *p = reinterpret_cast<T *>(base ? base + off : nullptr);
    off += std::max<size_t>(count * sizeof(T), 16);
    return p;
  }
};

// IG_QKV_FUSE=0 runs the QKV projection as its own GEMM (float32 qkv in HBM)
// before the short-sequence attention kernel (the same bits; for comparisons).
static bool qkv_fuse_enabled() {
  static const bool on = [] {
    const char *s = getenv("IG_QKV_FUSE");
    return !(s && s[0] == '0');
  }();
  return on;
}

// IG_GEGLU_QUANT=1 quantizes the GeGLU output inside the Wi GEMM (a cluster
// of the row block's column tiles exchanging row maxima); by default the
// output goes through g in float32 and a separate quantization pass, which
// measured faster on B200 at C1 (Wi 156 us + quantization 82 us against
// 268 us fused per launch at 2048 sequences: the Wi epilogue is bound by the
// GeGLU arithmetic, and the cluster's per-tile exchange adds to it). The
// same bits either way.
static bool geglu_quant_enabled() {
  static const bool on = [] {
    const char *s = getenv("IG_GEGLU_QUANT");
    return s && s[0] == '1';
  }();
  return on;
}

void carve_ws(Workspace &w, const ig_model *m, char *base, size_t rows, size_t seqs, size_t blks, size_t tl,
              size_t pl, bool f32, size_t *total) {
  Carve c{base};
  const size_t H = m->H, I = m->I, nh = m->nh, D = m->D;
  w.ids = c.take<int32_t>(rows);
  w.offs = c.take<int32_t>(seqs + 1);
  w.row_seq = c.take<int32_t>(rows);
  w.pos = c.take<int32_t>(rows);
  w.blocks = c.take<char>(blks);
  w.x = c.take<float>(rows * H);
  w.xn = c.take<float>(rows * H);
  w.sa = c.take<float>(rows);
  w.xq = c.take<uint8_t>(rows * m->ldk);
  w.qkv = c.take<float>(rows * 3 * H);
  w.ctx = c.take<float>(rows * H);
  w.g = c.take<float>(rows * std::max<size_t>(I, ((size_t)m->ldk + 3) / 4));
  w.sg = c.take<float>(rows);
  w.qa = c.take<uint8_t>(rows * nh * D);
  w.kq = c.take<int8_t>(rows * nh * D);
  w.vq = c.take<int8_t>(rows * nh * D);
  w.sq = c.take<float>(rows * nh);
  w.ks = c.take<float>(rows * nh);
  w.kzc = c.take<float>(rows * nh);
  w.kmean = c.take<float>(seqs * nh * D);
  w.vs = c.take<float>(seqs * nh * D);
  w.vinv = c.take<float>(seqs * nh * D);
  w.pooled = c.take<float>(seqs * H);
  w.logits = c.take<double>(seqs * pl);
  w.tlogits = c.take<double>(rows * tl);
  w.zf = f32 ? c.take<float>(rows * 2 * I) : nullptr;
  *total = c.off;
}

// Takes a workspace with room for the plan; `st` then waits for the
// workspace's previous user.
// A workspace from the model's pool with room for `rows` rows, `seqs`
// sequences, `blks` bytes of block lists and `hb` bytes of pinned plan staging.
int acquire_ws_sized(ig_model *m, size_t rows, size_t seqs, size_t blks, size_t hb, size_t tl, size_t pl,
                     cudaStream_t st, bool capturing, Workspace **out) {
  std::unique_ptr<Workspace> w;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    if (!m->pool.empty()) {
      w = std::move(m->pool.back());
      m->pool.pop_back();
    }
  }
  if (!w) {
    w.reset(new Workspace());
    w->device = m->device;
    IG_CU(cudaEventCreateWithFlags(&w->done, cudaEventDisableTiming));
  }
  rows = std::max<size_t>(rows, 1), seqs = std::max<size_t>(seqs, 1), blks = std::max<size_t>(blks, 16);
  const bool f32 = m->f32 || w->f32_cap;
  if (rows > w->rows_cap || seqs > w->seq_cap || blks > w->blk_cap || tl > w->tl_cap || pl > w->pl_cap ||
      f32 != w->f32_cap) {
    if (capturing) return fail(IG_ERR_BAD_ARG, "workspace must be sized before stream capture");
    IG_CU(cudaEventSynchronize(w->done));
    if (w->dev) IG_CU(cudaFree(w->dev));
    w->dev = nullptr;
    const size_t r2 = std::max(rows, w->rows_cap), s2 = std::max(seqs, w->seq_cap), b2 = std::max(blks, w->blk_cap);
    const size_t t2 = std::max(tl, w->tl_cap), p2 = std::max(pl, w->pl_cap);
    size_t total = 0;
    carve_ws(*w, m, nullptr, r2, s2, b2, t2, p2, f32, &total);
    IG_CU(cudaMalloc(&w->dev, total));
    carve_ws(*w, m, reinterpret_cast<char *>(w->dev), r2, s2, b2, t2, p2, f32, &total);
    w->gen++;
    w->f32_cap = f32;
    w->rows_cap = r2;
    w->seq_cap = s2;
    w->blk_cap = b2;
    w->tl_cap = t2;
    w->pl_cap = p2;
  }
  if (hb > w->host_bytes) {
    if (capturing) return fail(IG_ERR_BAD_ARG, "workspace must be sized before stream capture");
    IG_CU(cudaEventSynchronize(w->done));
    if (w->host) IG_CU(cudaFreeHost(w->host));
    w->host = nullptr;
    IG_CU(cudaMallocHost(&w->host, hb * 2));
    w->host_bytes = hb * 2;
  }
  if (!capturing) {
    IG_CU(cudaEventSynchronize(w->done));  // staging buffer reuse
    IG_CU(cudaStreamWaitEvent(st, w->done, 0));
  }
  *out = w.release();
  return 0;
}

// Pinned staging bytes of a plan's upload (offsets, ids, block lists).
size_t plan_host_bytes(const Plan &p) {
  return sizeof(int32_t) * (p.nseq + 1 + (size_t)p.N) + p.block_bytes() + 64;
}

int acquire_ws(ig_model *m, const Plan &p, size_t tl, size_t pl, cudaStream_t st, bool capturing, Workspace **out) {
  return acquire_ws_sized(m, p.N, p.nseq, p.block_bytes(), plan_host_bytes(p), tl, pl, st, capturing, out);
}

void release_ws(ig_model *m, Workspace *w, cudaStream_t st, bool capturing) {
  if (!capturing) cudaEventRecord(w->done, st);
  std::lock_guard<std::mutex> lk(m->mu);
  m->pool.emplace_back(w);
}

// Uploads the plan's metadata (offsets, query blocks, and optionally the host
// ids) through the pinned staging, one copy per device region, and fills the
// row -> sequence and position tables on the device from the offsets.
// memcpy(dst, src, n) split over the host copy pool's threads (CopyPool).
void host_copy(char *dst, const char *src, size_t n);
bool host_copy_ids(int32_t *dst, const int32_t *src, size_t n, uint32_t vocab);
int check_ids(const ig_model *m, const int32_t *ids, int64_t N);

// With host ids, `m` given: the ids are tested against the vocabulary while
// they are staged (no separate pass over them); an id outside it fails the
// call with the first such id, before anything is enqueued.
int upload_plan(Workspace &w, const Plan &p, const int32_t *host_ids, cudaStream_t st, bool capturing = false,
                const ig_model *m = nullptr) {
  char *h = reinterpret_cast<char *>(w.host);
  size_t off = 0;
  auto put = [&](const void *src, size_t bytes) {
    if (bytes >= (512u << 10))
      host_copy(h + off, static_cast<const char *>(src), bytes);
    else
      std::memcpy(h + off, src, bytes);
    off += bytes;
  };
  put(p.offs.data(), sizeof(int32_t) * (p.nseq + 1));
  for (int k = 0; k < 2; k++) put(p.tc[k].data(), 16 * p.tc[k].size());
  for (int k = 0; k < 2; k++) put(p.v1[k].data(), 8 * p.v1[k].size());
  put(p.fb.data(), 8 * p.fb.size());
  if (host_ids && m) {
    bool bad;
    if (p.N >= (128 << 10)) {
      bad = host_copy_ids(reinterpret_cast<int32_t *>(h + off), host_ids, p.N, (uint32_t)m->cfg.vocab);
    } else {
      bad = false;
      const uint32_t vocab = (uint32_t)m->cfg.vocab;
      int32_t *dst = reinterpret_cast<int32_t *>(h + off);
      uint32_t b = 0;
      for (int64_t i = 0; i < p.N; i++) {
        dst[i] = host_ids[i];
        b |= (uint32_t)((uint32_t)host_ids[i] >= vocab);
      }
      bad = b != 0;
    }
    if (bad) return check_ids(m, host_ids, p.N);  // the first bad id's error
    off += sizeof(int32_t) * p.N;
  } else if (host_ids) {
    put(host_ids, sizeof(int32_t) * p.N);
  }
  // The device buffers are carved separately: issue one copy per region
  // from the pinned staging (small, contiguous on the host).
  size_t o = 0;
  IG_CU(cudaMemcpyAsync(w.offs, h + o, sizeof(int32_t) * (p.nseq + 1), cudaMemcpyHostToDevice, st));
  o += sizeof(int32_t) * (p.nseq + 1);
  if (p.N) {
    ProfScope ps("plan_rows", 8.0 * p.N + 4.0 * (p.nseq + 1), 0, 1, st, capturing);
    IG_TRY(launch_fill_rows(w.offs, p.nseq, w.row_seq, w.pos, st));
  }
  const size_t bb = p.block_bytes();
  if (bb) IG_CU(cudaMemcpyAsync(w.blocks, h + o, bb, cudaMemcpyHostToDevice, st));
  o += bb;
  size_t bo = 0;
  for (int k = 0; k < 2; k++) {
    w.pd.tc[k] = reinterpret_cast<const int4 *>(w.blocks + bo);
    w.pd.ntc[k] = (int)p.tc[k].size();
    w.pd.ntc_short[k] = p.tc_short[k];
    bo += 16 * p.tc[k].size();
  }
  for (int k = 0; k < 2; k++) {
    w.pd.v1[k] = reinterpret_cast<const int2 *>(w.blocks + bo);
    w.pd.nv1[k] = (int)p.v1[k].size();
    bo += 8 * p.v1[k].size();
  }
  w.pd.fb = reinterpret_cast<const int2 *>(w.blocks + bo);
  w.pd.nfb = (int)p.fb.size();
  if (host_ids && p.N) IG_CU(cudaMemcpyAsync(w.ids, h + o, sizeof(int32_t) * p.N, cudaMemcpyHostToDevice, st));
  return 0;
}

int copy_rows_d2h(void *dst, const void *src, size_t row_bytes, size_t src_pitch, size_t rows, cudaStream_t st) {
  if (!dst || rows == 0) return 0;
  IG_CU(cudaMemcpy2DAsync(dst, row_bytes, src, src_pitch, row_bytes, rows, cudaMemcpyDeviceToHost, st));
  return 0;
}

// The layer loop. d_ids: device ids; results in w.xn (tokens) / w.pooled.
// Algorithmic bytes of a GEMM launch: A (M x K u8), B (N x K s8), scales,
// and out_row_bytes of output traffic per row.
double gemm_bytes(double M, double N, double K, double out_row_bytes) {
  return M * K + N * K + 4.0 * M + 8.0 * N + M * out_row_bytes;
}

// Valid (query, key) pairs of an attention layer over the plan's sequences.
double attn_pairs(const Plan &p, int window) {
  double pairs = 0;
  for (int s = 0; s < p.nseq; s++) {
    const double n = p.offs[s + 1] - p.offs[s];
    if (window < 0 || n <= window + 1) {
      pairs += n * n;
    } else {
      const double w = window;
      pairs += n * (2 * w + 1) - w * (w + 1);  // rows near the ends see fewer keys
    }
  }
  return pairs;
}

// The float32 path (run without SetInt8, infer.go:304-430): float products
// in the reference's chain order, RoPE in place, attendBlocks, GeluMul.
int run_encoder_f32(ig_model *m, Workspace &w, const int32_t *d_ids, const Plan &p, int mode, cudaStream_t st,
                    bool capturing, bool tail) {
  const ig_config &c = m->cfg;
  const int H = m->H, I = m->I, N = p.N, V = c.simd_lanes;
  if (!w.zf) return fail(IG_ERR_BAD_ARG, "workspace without the float buffers");
  {
    ProfScope ps("f32_embed_ln", (double)N * (8 + 8.0 * H) + 4.0 * H, 0, 1, st, capturing);
    if (m->emb.fmt < 0) return fail(IG_ERR_BAD_ARG, "modernbert: no embedding table");
    IG_TRY(launch_embed_checked(d_ids, c.vocab, m->emb, m->emb_norm, N, H, c.norm_eps, V, w.x, nullptr, 0, nullptr,
                                st));
  }
  const float scale = (float)(1.0 / std::sqrt((double)m->D));
  auto product = [&](const char *name, const float *A, int K, const float *W, int Nout, float *C, bool acc) {
    F32Gemm g{};
    g.A = A, g.lda = K, g.W = W, g.ldw = K, g.M = N, g.N = Nout, g.K = K, g.C = C, g.ldc = Nout, g.accumulate = acc;
    g.V = V;
    ProfScope ps(name, 4.0 * N * K + 4.0 * Nout * K + (acc ? 8.0 : 4.0) * N * Nout, 2.0 * N * Nout * K, 1, st,
                 capturing);
    return launch_f32_gemm(g, st);
  };
  for (int l = 0; l < c.layers; l++) {
    const DevLayer &L = m->layers[l];
    const bool global = l % c.global_every == 0;
    const float *in = w.x;
    if (l > 0) {
      ProfScope ps("f32_ln", (double)N * 8.0 * H + 4.0 * H, 0, 1, st, capturing);
      IG_TRY(launch_ln_quant(w.x, L.attn_norm, N, H, c.norm_eps, V, w.xn, nullptr, 0, nullptr, st));
      in = w.xn;
    }
    IG_TRY(product("f32_gemm_qkv", in, H, L.fqkv, 3 * H, w.qkv, false));
    {
      ProfScope ps("f32_rope", (double)N * 16.0 * H, 0, 1, st, capturing);
      IG_TRY(launch_rope_f32(w.qkv, w.pos, N, H, m->nh, m->rope_cos[global ? 0 : 1], m->rope_sin[global ? 0 : 1],
                             st));
    }
    {
      const int window = global ? -1 : c.local_attention / 2;
      ProfScope ps("f32_attend_blocks", (double)N * 16.0 * H, 4.0 * attn_pairs(p, window) * m->D * m->nh, 1, st,
                   capturing);
      IG_TRY(launch_attend_blocks_f32(w.qkv, w.offs, w.pd.fb, w.pd.nfb, H, m->nh, window, scale, V, w.ctx, st));
    }
    IG_TRY(product("f32_gemm_wo", w.ctx, H, L.fo, H, w.x, true));
    {
      ProfScope ps("f32_ln", (double)N * 8.0 * H + 4.0 * H, 0, 1, st, capturing);
      IG_TRY(launch_ln_quant(w.x, L.mlp_norm, N, H, c.norm_eps, V, w.xn, nullptr, 0, nullptr, st));
    }
    IG_TRY(product("f32_gemm_wi", w.xn, H, L.fwi, 2 * I, w.zf, false));
    {
      ProfScope ps("f32_gelu_mul", (double)N * 12.0 * I, 0, 1, st, capturing);
      IG_TRY(launch_gelu_mul_rows(w.zf, N, I, w.g, st));
    }
    IG_TRY(product("f32_gemm_womlp", w.g, I, L.fwom, H, w.x, true));
  }
  if (!tail) return 0;  // the final norm and pooling are left to the caller
  {
    ProfScope ps("ln_final", (double)N * 8.0 * H + 4.0 * H, 0, 1, st, capturing);
    IG_TRY(launch_ln_quant(w.x, m->final_norm, N, H, c.norm_eps, V, w.xn, nullptr, 0, nullptr, st));
  }
  if (mode != IG_MODE_TOKENS) {
    ProfScope ps("pool", (double)N * 4.0 * H + 4.0 * p.nseq * H, 0, 1, st, capturing);
    IG_TRY(launch_pool(w.xn, w.offs, p.nseq, H, mode == IG_MODE_POOLED && c.pooling == IG_POOL_CLS, w.pooled, st,
                       p.max_len, (int)p.N));
  }
  return 0;
}

// tail = false stops before the final norm and the pooling (the caller runs
// them, e.g. in row chunks whose outputs are copied out as they finish).
int run_encoder(ig_model *m, Workspace &w, const int32_t *d_ids, const Plan &p, int mode, cudaStream_t st,
                ig_dump *dump, bool capturing = false, bool tail = true) {
  const ig_config &c = m->cfg;
  const int H = m->H, I = m->I, N = p.N;
  const int V = c.simd_lanes;
  if (N == 0) return 0;
  if (m->f32) {
    if (dump) return fail(IG_ERR_UNSUPPORTED, "the per-layer dump is of the int8 path");
    return run_encoder_f32(m, w, d_ids, p, mode, st, capturing, tail);
  }
  {
    ProfScope ps("embed_ln_quant", (double)N * (8 + 9.0 * H) + 4.0 * H, 0, 1, st, capturing);
    if (m->emb.fmt < 0) return fail(IG_ERR_BAD_ARG, "modernbert: no embedding table");
    IG_TRY(launch_embed_checked(d_ids, c.vocab, m->emb, m->emb_norm, N, H, c.norm_eps, V, w.x, w.xq, m->ldk, w.sa,
                                st));
  }
  if (dump && dump->emb_ln) IG_TRY(copy_rows_d2h(dump->emb_ln, w.x, H * 4, H * 4, N, st));
  AttnArgs at{};
  at.qkv = w.qkv;
  at.H = H;
  at.nh = m->nh;
  at.D = m->D;
  at.offs = w.offs;
  at.nseq = p.nseq;
  at.max_len = p.max_len;
  at.scale = (float)(1.0 / std::sqrt((double)m->D));
  at.V = V;
  at.qa = w.qa;
  at.sq = w.sq;
  at.kq = w.kq;
  at.ks = w.ks;
  at.kzc = w.kzc;
  at.vq = w.vq;
  at.kmean = w.kmean;
  at.vs = w.vs;
  at.vinv = w.vinv;
  at.row_seq = w.row_seq;
  at.N = N;
  at.row_tiles = w.pd.fb;
  at.nrow_tiles = w.pd.nfb;
  at.ctx = w.ctx;
  for (int l = 0; l < c.layers; l++) {
    const DevLayer &L = m->layers[l];
    const bool global = l % c.global_every == 0;
    const bool dl = dump && dump->layer == l;
    if (l > 0) {
      ProfScope ps("ln_quant", (double)N * (5.0 * H + 4) + 4.0 * H, 0, 1, st, capturing);
      IG_TRY(launch_ln_quant(w.x, L.attn_norm, N, H, c.norm_eps, V, nullptr, w.xq, m->ldk, w.sa, st));
    }
    if (dl) {
      IG_TRY(copy_rows_d2h(dump->xq, w.xq, H, m->ldk, N, st));
      IG_TRY(copy_rows_d2h(dump->xq_s, w.sa, 4, 4, N, st));
    }
    at.window = global ? -1 : c.local_attention / 2;
    at.rope_cos = m->rope_cos[global ? 0 : 1];
    at.rope_sin = m->rope_sin[global ? 0 : 1];
    at.xq = nullptr;
    at.sa = nullptr;
    // Sequences of at most 128 tokens: the QKV projection runs inside the
    // attention kernel (no float qkv in HBM) and ctx is quantized there,
    // unless this layer is dumped.
    AttnArgs ap = at;
    ap.qkv = nullptr;
    ap.xa = w.xq;
    ap.lda = m->ldk;
    ap.xa_s = w.sa;
    ap.wqkv = L.qkv.q;
    ap.ldw = L.qkv.ld;
    ap.wsb = L.qkv.scale;
    ap.wzc = L.qkv.zc;
    ap.xq = w.xq;
    ap.ldq = m->ldk;
    ap.sa = w.sa;
    if (!dl && qkv_fuse_enabled() && attn_short_fits(ap)) {
      const double pairs = attn_pairs(p, ap.window);
      ProfScope ps("attn_qkv_quant", (double)N * (H + 4) * 2 + 3.0 * H * H + 24.0 * H + 8.0 * N * 32,
                   2.0 * N * 3 * H * H + 4.0 * pairs * m->D * m->nh, 1, st, capturing);
      IG_TRY(launch_attn_short(ap, st));
    } else {
    {
      GemmArgs g{w.xq, L.qkv.q, N, L.qkv.n, H, m->ldk, L.qkv.ld, 256};
      GemmEpilogue e{};
      e.sa = w.sa;
      e.sb = L.qkv.scale;
      e.zc = L.qkv.zc;
      e.C = w.qkv;
      e.ldc = 3 * H;
      ProfScope ps("gemm_qkv", gemm_bytes(N, 3 * H, H, 4.0 * 3 * H), 2.0 * N * 3 * H * H, 1, st, capturing);
      IG_TRY(gemm_u8s8(g, e, kEpiF32, st));
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->qkv, w.qkv, 3 * H * 4, 3 * H * 4, N, st));
    // ctx quantized inside the short-sequence kernel unless this layer is dumped.
    bool ctx_quantized = false;
    if (attn_short_fits(at) && !dl) {
      AttnArgs aq = at;
      aq.xq = w.xq;
      aq.ldq = m->ldk;
      aq.sa = w.sa;
      ctx_quantized = attn_short_quantizes(aq);
      if (ctx_quantized) at = aq;
    }
    if (attn_short_fits(at)) {
      const double pairs = attn_pairs(p, at.window);
      const double out_bytes = ctx_quantized ? (double)N * H + 4.0 * N : 4.0 * N * H;
      ProfScope ps(ctx_quantized ? "attn_short_quant" : "attn_short", (double)N * H * 4 * 3 + out_bytes + 8.0 * N * 32,
                   4.0 * pairs * m->D * m->nh, 1, st, capturing);
      IG_TRY(launch_attn_short(at, st));
    } else {
      {
        ProfScope ps("attn_prep", (double)N * H * 4 * 3 + (double)N * H * 3 + 12.0 * N * m->nh + 8.0 * N * 32, 0, 1,
                     st, capturing);
        IG_TRY(launch_attention(at, st));
      }
      {
        const double pairs = attn_pairs(p, at.window);
        ProfScope ps("attn_attend", (double)N * H * 7 + 12.0 * N * m->nh, 4.0 * pairs * m->D * m->nh, 1, st,
                     capturing);
        const int kind = global ? 0 : 1;
        IG_TRY(launch_attend_tc(at, w.pd.tc[kind], w.pd.ntc_short[kind], w.pd.ntc[kind] - w.pd.ntc_short[kind], st));
        IG_TRY(launch_attend(at, w.pd.v1[kind], w.pd.nv1[kind], st));
      }
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->ctx, w.ctx, H * 4, H * 4, N, st));
    if (!ctx_quantized) {
      ProfScope ps("quant_rows", (double)N * (5.0 * H + 4), 0, 1, st, capturing);
      IG_TRY(launch_quant_rows(w.ctx, H, N, H, w.xq, m->ldk, w.sa, st));
    }
    }
    if (dl) {
      IG_TRY(copy_rows_d2h(dump->cq, w.xq, H, m->ldk, N, st));
      IG_TRY(copy_rows_d2h(dump->cq_s, w.sa, 4, 4, N, st));
    }
    {
      GemmArgs g{w.xq, L.o.q, N, L.o.n, H, m->ldk, L.o.ld, 0};
      GemmEpilogue e{};
      e.sa = w.sa;
      e.sb = L.o.scale;
      e.zc = L.o.zc;
      e.C = w.x;
      e.ldc = H;
      e.accumulate = 1;
      ProfScope ps("gemm_wo_residual", gemm_bytes(N, H, H, 8.0 * H), 2.0 * N * H * H, 1, st, capturing);
      IG_TRY(gemm_u8s8(g, e, kEpiF32, st));
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->x_attn, w.x, H * 4, H * 4, N, st));
    {
      ProfScope ps("ln_quant", (double)N * (5.0 * H + 4) + 4.0 * H, 0, 1, st, capturing);
      IG_TRY(launch_ln_quant(w.x, L.mlp_norm, N, H, c.norm_eps, V, nullptr, w.xq, m->ldk, w.sa, st));
    }
    if (dl) {
      IG_TRY(copy_rows_d2h(dump->hq, w.xq, H, m->ldk, N, st));
      IG_TRY(copy_rows_d2h(dump->hq_s, w.sa, 4, 4, N, st));
    }
    // The GeGLU output quantized in the Wi epilogue (one cluster per row
    // block; its bytes over g, its scales in sg) unless this layer is dumped,
    // or through g in float32 and a quantization pass.
    GemmEpilogue eq{};
    eq.geglu_n = I;
    eq.q_out = reinterpret_cast<uint8_t *>(w.g);
    eq.ldq = m->ldk;
    eq.sa_out = w.sg;
    const bool gq_fused = !dl && geglu_quant_enabled() && gemm_geglu_q_fits(2 * I, eq);
    {
      GemmArgs g{w.xq, L.wi.q, N, L.wi.n, H, m->ldk, L.wi.ld, 256};
      GemmEpilogue e = eq;
      e.sa = w.sa;
      e.sb = L.wi.scale;
      e.zc = L.wi.zc;
      e.C = w.g;
      e.ldc = I;
      if (gq_fused) {
        ProfScope ps("gemm_wi_geglu_quant", gemm_bytes(N, 2 * I, H, (double)I + 4.0), 2.0 * N * 2 * I * H, 1, st,
                     capturing);
        IG_TRY(gemm_u8s8(g, e, kEpiGegluQ, st));
      } else {
        ProfScope ps("gemm_wi_geglu", gemm_bytes(N, 2 * I, H, 4.0 * I), 2.0 * N * 2 * I * H, 1, st, capturing);
        IG_TRY(gemm_u8s8(g, e, kEpiGeglu, st));
      }
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->g, w.g, I * 4, I * 4, N, st));
    if (!gq_fused) {
      ProfScope ps("quant_rows", (double)N * (5.0 * I + 4), 0, 1, st, capturing);
      IG_TRY(launch_quant_rows(w.g, I, N, I, w.xq, m->ldk, w.sa, st));
    }
    if (dl) {
      IG_TRY(copy_rows_d2h(dump->gq, w.xq, I, m->ldk, N, st));
      IG_TRY(copy_rows_d2h(dump->gq_s, w.sa, 4, 4, N, st));
    }
    {
      GemmArgs g{gq_fused ? reinterpret_cast<const uint8_t *>(w.g) : w.xq, L.wom.q, N, L.wom.n, I, m->ldk, L.wom.ld, 0};
      GemmEpilogue e{};
      e.sa = gq_fused ? w.sg : w.sa;
      e.sb = L.wom.scale;
      e.zc = L.wom.zc;
      e.C = w.x;
      e.ldc = H;
      e.accumulate = 1;
      ProfScope ps("gemm_womlp_residual", gemm_bytes(N, H, I, 8.0 * H), 2.0 * N * H * I, 1, st, capturing);
      IG_TRY(gemm_u8s8(g, e, kEpiF32, st));
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->x_mlp, w.x, H * 4, H * 4, N, st));
  }
  if (!tail) return 0;  // the final norm and pooling are left to the caller
  {
    ProfScope ps("ln_final", (double)N * 8.0 * H + 4.0 * H, 0, 1, st, capturing);
    IG_TRY(launch_ln_quant(w.x, m->final_norm, N, H, c.norm_eps, V, w.xn, nullptr, 0, nullptr, st));
  }
  if (mode != IG_MODE_TOKENS) {
    ProfScope ps("pool", (double)N * 4.0 * H + 4.0 * p.nseq * H, 0, 1, st, capturing);
    IG_TRY(launch_pool(w.xn, w.offs, p.nseq, H, mode == IG_MODE_POOLED && c.pooling == IG_POOL_CLS, w.pooled, st,
                       p.max_len, (int)p.N));
  }
  return 0;
}

// Head logits (heads.go:62-74) of the pooled vectors and, for per-token
// heads, of every token state, into [nseq][pooled rows] / [N][token rows].
int run_heads(ig_model *m, Workspace &w, const Plan &p, cudaStream_t st, double *d_logits, double *d_tlogits,
              bool capturing) {
  std::vector<DevHead> hs;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    hs = m->heads;
  }
  size_t pl = 0, tl = 0;
  for (auto &h : hs) (h.per_token ? tl : pl) += h.rows;
  size_t po = 0, to = 0;
  const int H = m->H;
  for (auto &h : hs) {
    if (h.per_token) {
      if (d_tlogits && p.N) {
        ProfScope ps("head_logits", (double)p.N * (4.0 * H + 8.0 * h.rows), 2.0 * p.N * h.rows * H, 1, st, capturing);
        IG_TRY(launch_head_logits(h.w, h.b, h.rows, H, w.xn, p.N, d_tlogits + to, (int)tl, st));
      }
      to += h.rows;
    } else {
      if (d_logits && p.nseq) {
        ProfScope ps("head_logits", (double)p.nseq * (4.0 * H + 8.0 * h.rows), 2.0 * p.nseq * h.rows * H, 1, st,
                     capturing);
        IG_TRY(launch_head_logits(h.w, h.b, h.rows, H, w.pooled, p.nseq, d_logits + po, (int)pl, st));
      }
      po += h.rows;
    }
  }
  return 0;
}

int check_ids(const ig_model *m, const int32_t *ids, int64_t N) {
  // Blocks of ids tested without a branch (a vectorizable OR of unsigned
  // compares); the first bad id is looked for only in a block that has one.
  const uint32_t vocab = (uint32_t)m->cfg.vocab;
  for (int64_t t0 = 0; t0 < N; t0 += 4096) {
    const int64_t t1 = std::min<int64_t>(N, t0 + 4096);
    uint32_t bad = 0;
    for (int64_t t = t0; t < t1; t++) bad |= (uint32_t)((uint32_t)ids[t] >= vocab);
    if (bad)
      for (int64_t t = t0; t < t1; t++)
        if (ids[t] < 0 || ids[t] >= m->cfg.vocab)
          return fail(IG_ERR_OUT_OF_VOCAB, "modernbert: id " + std::to_string(ids[t]) + " out of vocabulary");
  }
  return 0;
}

// Large outputs of a host call reach the caller's (pageable) memory through
// the workspace's pinned staging: the device copies 2 MB pieces there, and as
// each piece lands the host copies it on with a few threads, while the later
// pieces are in flight. A pageable destination takes about a quarter of the
// link's rate from a single copying thread.
constexpr size_t kStageMinBytes = 2 << 20;  // smaller outputs are copied directly
constexpr size_t kStagePiece = 2 << 20;

class CopyPool {
 public:
  static CopyPool &get() {
    static CopyPool *pool = new CopyPool();  // lives until the process ends
    return *pool;
  }
  // memcpy(dst, src, n), split across the pool's threads and the caller.
  void copy(char *dst, const char *src, size_t n) { run_split(dst, src, n, 0, nullptr); }
  // The same for n int32 ids, returning whether any is outside [0, vocab).
  bool copy_checked(int32_t *dst, const int32_t *src, size_t n, uint32_t vocab) {
    std::atomic<uint32_t> bad{0};
    run_split(reinterpret_cast<char *>(dst), reinterpret_cast<const char *>(src), 4 * n, vocab, &bad);
    return bad.load() != 0;
  }
  // Copies ids, OR-ing the unsigned test id >= vocab (negative ids included)
  // without a branch, so that the loop vectorizes.
  static uint32_t copy_ids(int32_t *dst, const int32_t *src, size_t n, uint32_t vocab) {
    uint32_t bad = 0;
    for (size_t i = 0; i < n; i++) {
      const int32_t v = src[i];
      dst[i] = v;
      bad |= (uint32_t)((uint32_t)v >= vocab);
    }
    return bad;
  }

 private:
  void run_split(char *dst, const char *src, size_t n, uint32_t vocab, std::atomic<uint32_t> *bad) {
    const size_t parts = std::min<size_t>(nthreads_ + 1, std::max<size_t>(1, n / kMinPart));
    const size_t per = align_up((n + parts - 1) / parts, 64);
    Batch b;
    {
      std::lock_guard<std::mutex> lk(mu_);
      for (size_t o = per; o < n; o += per) {
        jobs_.push_back({dst + o, src + o, std::min(per, n - o), &b, vocab, bad});
        b.left++;
      }
    }
    cv_.notify_all();
    const size_t n0 = std::min(per, n);
    if (vocab)
      bad->fetch_or(copy_ids(reinterpret_cast<int32_t *>(dst), reinterpret_cast<const int32_t *>(src), n0 / 4, vocab));
    else
      std::memcpy(dst, src, n0);
    std::unique_lock<std::mutex> lk(b.mu);
    b.cv.wait(lk, [&] { return b.left == 0; });
  }
  static constexpr size_t kMinPart = 256 << 10;
  struct Batch {
    std::mutex mu;
    std::condition_variable cv;
    size_t left = 0;
  };
  struct Job {
    char *dst;
    const char *src;
    size_t n;
    Batch *b;
    uint32_t vocab;         // nonzero: int32 ids, each tested against it while copied
    std::atomic<uint32_t> *bad;
  };
  CopyPool() {
    const unsigned hc = std::thread::hardware_concurrency();
    nthreads_ = std::max(1u, std::min(7u, hc / 2));
    for (unsigned i = 0; i < nthreads_; i++) std::thread([this] { run(); }).detach();
  }
  void run() {
    for (;;) {
      Job j;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return !jobs_.empty(); });
        j = jobs_.front();
        jobs_.pop_front();
      }
      if (j.vocab)
        j.bad->fetch_or(copy_ids(reinterpret_cast<int32_t *>(j.dst), reinterpret_cast<const int32_t *>(j.src),
                                 j.n / 4, j.vocab));
      else
        std::memcpy(j.dst, j.src, j.n);
      std::lock_guard<std::mutex> lk(j.b->mu);
      if (--j.b->left == 0) j.b->cv.notify_all();
    }
  }
  unsigned nthreads_ = 1;
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<Job> jobs_;
};

void host_copy(char *dst, const char *src, size_t n) { CopyPool::get().copy(dst, src, n); }
bool host_copy_ids(int32_t *dst, const int32_t *src, size_t n, uint32_t vocab) {
  return CopyPool::get().copy_checked(dst, src, n, vocab);
}

struct OutCopy {
  const void *src;  // device
  void *dst;        // host
  size_t bytes;
};

// Copies the outputs to the host through the pinned staging (enqueued on st
// after the work that produces them) and returns once all have arrived.
int copy_out_staged(Workspace &w, cudaStream_t st, const std::vector<OutCopy> &outs) {
  size_t total = 0;
  for (auto &o : outs) total += o.bytes;
  if (total > w.ohost_bytes) {
    IG_CU(cudaStreamSynchronize(st));  // the earlier user of the staging has finished
    if (w.ohost) IG_CU(cudaFreeHost(w.ohost));
    w.ohost = nullptr;
    w.ohost_bytes = 0;
    IG_CU(cudaMallocHost(&w.ohost, total));
    w.ohost_bytes = total;
  }
  struct Piece {
    const char *src;
    char *dst;
    size_t n, at;
  };
  std::vector<Piece> ps;
  size_t at = 0;
  for (auto &o : outs)
    for (size_t k = 0; k < o.bytes; k += kStagePiece) {
      const size_t n = std::min(kStagePiece, o.bytes - k);
      ps.push_back({static_cast<const char *>(o.src) + k, static_cast<char *>(o.dst) + k, n, at});
      at += n;
    }
  while (w.pev.size() < ps.size()) {
    cudaEvent_t e;
    IG_CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    w.pev.push_back(e);
  }
  char *stage = static_cast<char *>(w.ohost);
  if (total < kStageMinBytes) {
    // Small outputs: one wait, then plain host copies on this thread (a
    // device-to-pageable copy would go through the driver's shared staging,
    // which serializes concurrent callers).
    for (auto &pc : ps) IG_CU(cudaMemcpyAsync(stage + pc.at, pc.src, pc.n, cudaMemcpyDeviceToHost, st));
    const cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail(IG_ERR_CUDA, std::string("encode: ") + cudaGetErrorString(e));
    for (auto &pc : ps) std::memcpy(pc.dst, stage + pc.at, pc.n);
    return 0;
  }
  for (size_t i = 0; i < ps.size(); i++) {
    IG_CU(cudaMemcpyAsync(stage + ps[i].at, ps[i].src, ps[i].n, cudaMemcpyDeviceToHost, st));
    IG_CU(cudaEventRecord(w.pev[i], st));
  }
  for (size_t i = 0; i < ps.size(); i++) {
    const cudaError_t e = cudaEventSynchronize(w.pev[i]);
    if (e != cudaSuccess) return fail(IG_ERR_CUDA, std::string("encode: ") + cudaGetErrorString(e));
    CopyPool::get().copy(ps[i].dst, stage + ps[i].at, ps[i].n);
  }
  return 0;
}

// The encoder's tail when per-token logits go to the host: the final norm and
// the per-token heads run in row chunks on st, and each chunk's logits are
// copied out on the workspace's copy stream as soon as they exist, so the
// copies overlap the later chunks' kernels; then the pooling, the pooled
// heads and their copy. Returns once every output is in the caller's memory.
constexpr int kTailChunks = 8;
constexpr int kTailMinRows = 16384;

int run_tail_staged(ig_model *m, Workspace &w, const Plan &p, int mode, cudaStream_t st, double *logits, double *tlog,
                    size_t pl, size_t tl) {
  const ig_config &c = m->cfg;
  const int H = m->H, N = p.N;
  std::vector<DevHead> hs;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    hs = m->heads;
  }
  const size_t tbytes = sizeof(double) * (size_t)N * tl, pbytes = logits ? sizeof(double) * (size_t)p.nseq * pl : 0;
  if (tbytes + pbytes > w.ohost_bytes) {
    IG_CU(cudaStreamSynchronize(st));
    if (w.ohost) IG_CU(cudaFreeHost(w.ohost));
    w.ohost = nullptr;
    w.ohost_bytes = 0;
    IG_CU(cudaMallocHost(&w.ohost, tbytes + pbytes));
    w.ohost_bytes = tbytes + pbytes;
  }
  if (!w.copy_stream) IG_CU(cudaStreamCreateWithFlags(&w.copy_stream, cudaStreamNonBlocking));
  while ((int)w.cev.size() < kTailChunks + 2) {
    cudaEvent_t e;
    IG_CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    w.cev.push_back(e);
  }
  while ((int)w.pev.size() < kTailChunks + 1) {
    cudaEvent_t e;
    IG_CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    w.pev.push_back(e);
  }
  char *stage = static_cast<char *>(w.ohost);
  const int per = (int)align_up((size_t)(N + kTailChunks - 1) / kTailChunks, 32);
  // Each chunk's kernels follow the event the previous chunk's copy waits
  // for: plain stream order here, so that event completes with its chunk.
  DepLaunchOff plain_order;
  struct Piece {
    void *dst;
    size_t at, bytes;
  };
  std::vector<Piece> ps;
  for (int r0 = 0; r0 < N; r0 += per) {
    const int r1 = std::min(N, r0 + per), n = r1 - r0;
    {
      ProfScope pr("ln_final", (double)n * 8.0 * H + 4.0 * H, 0, 1, st);
      IG_TRY(launch_ln_quant(w.x + (size_t)r0 * H, m->final_norm, n, H, c.norm_eps, c.simd_lanes, w.xn + (size_t)r0 * H,
                             nullptr, 0, nullptr, st));
    }
    size_t to = 0;
    for (auto &h : hs) {
      if (!h.per_token) continue;
      ProfScope pr("head_logits", (double)n * (4.0 * H + 8.0 * h.rows), 2.0 * n * h.rows * H, 1, st);
      IG_TRY(launch_head_logits(h.w, h.b, h.rows, H, w.xn + (size_t)r0 * H, n, w.tlogits + (size_t)r0 * tl + to,
                                (int)tl, st));
      to += h.rows;
    }
    const int k = (int)ps.size();
    IG_CU(cudaEventRecord(w.cev[k], st));
    IG_CU(cudaStreamWaitEvent(w.copy_stream, w.cev[k], 0));
    const size_t at = sizeof(double) * (size_t)r0 * tl, bytes = sizeof(double) * (size_t)n * tl;
    IG_CU(cudaMemcpyAsync(stage + at, w.tlogits + (size_t)r0 * tl, bytes, cudaMemcpyDeviceToHost, w.copy_stream));
    IG_CU(cudaEventRecord(w.pev[k], w.copy_stream));
    ps.push_back({reinterpret_cast<char *>(tlog) + at, at, bytes});
  }
  if (mode != IG_MODE_TOKENS) {
    ProfScope pr("pool", (double)N * 4.0 * H + 4.0 * p.nseq * H, 0, 1, st);
    IG_TRY(launch_pool(w.xn, w.offs, p.nseq, H, mode == IG_MODE_POOLED && c.pooling == IG_POOL_CLS, w.pooled, st,
                       p.max_len, (int)p.N));
  }
  if (logits && p.nseq && pl) {
    size_t po = 0;
    for (auto &h : hs) {
      if (h.per_token) continue;
      ProfScope pr("head_logits", (double)p.nseq * (4.0 * H + 8.0 * h.rows), 2.0 * p.nseq * h.rows * H, 1, st);
      IG_TRY(launch_head_logits(h.w, h.b, h.rows, H, w.pooled, p.nseq, w.logits + po, (int)pl, st));
      po += h.rows;
    }
    const int k = (int)ps.size();
    IG_CU(cudaEventRecord(w.cev[k], st));
    IG_CU(cudaStreamWaitEvent(w.copy_stream, w.cev[k], 0));
    IG_CU(cudaMemcpyAsync(stage + tbytes, w.logits, pbytes, cudaMemcpyDeviceToHost, w.copy_stream));
    IG_CU(cudaEventRecord(w.pev[k], w.copy_stream));
    ps.push_back({logits, tbytes, pbytes});
  }
  // st waits for the copies, so the workspace is reused only after them.
  IG_CU(cudaEventRecord(w.cev[kTailChunks + 1], w.copy_stream));
  IG_CU(cudaStreamWaitEvent(st, w.cev[kTailChunks + 1], 0));
  for (size_t i = 0; i < ps.size(); i++) {
    const cudaError_t e = cudaEventSynchronize(w.pev[i]);
    if (e != cudaSuccess) return fail(IG_ERR_CUDA, std::string("encode: ") + cudaGetErrorString(e));
    CopyPool::get().copy(static_cast<char *>(ps[i].dst), stage + ps[i].at, ps[i].bytes);
  }
  return 0;
}

// Host calls on a model spread over several GPUs (multi.cu).
int encode_group(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, int32_t mode, float *out,
                 size_t out_len, ig_dump *dump, double *logits, size_t logits_len, double *tlog, size_t tlog_len);

// ---- repeated small host calls as CUDA graphs ------------------------------------
// A host call of at most kGraphMaxRows tokens takes about as long to launch
// its ~50 kernels as the GPU takes to run them (a 32 x 128 batch: about
// 0.37 ms of launches). Its kernels (layers, final norm, pooling, heads) are
// therefore recorded as a CUDA graph the second time a workspace sees the
// same offsets, mode and outputs in a row, and replayed by one graph launch
// after that. The same offsets give the same plan, grids and arguments; the
// data the kernels read (ids, offsets, block lists) is uploaded into the
// same workspace buffers before every call. A graph is re-recorded when the
// model changes (model version) or the workspace's buffers move (generation).
// IG_GRAPH=0 turns this off.
constexpr int64_t kGraphMaxRows = 1 << 14;

bool graphs_enabled() {
  static const bool on = [] {
    const char *s = getenv("IG_GRAPH");
    return !(s && s[0] == '0');
  }();
  return on;
}

int run_graphed(ig_model *m, Workspace &w, const Plan &p, const int64_t *offs, int enc_mode, bool want_logits,
                bool want_tlog, cudaStream_t st) {
  auto body = [&](bool capturing) -> int {
    IG_TRY(run_encoder(m, w, w.ids, p, enc_mode, st, nullptr, capturing, true));
    if (want_logits || want_tlog)
      IG_TRY(run_heads(m, w, p, st, want_logits ? w.logits : nullptr, want_tlog ? w.tlogits : nullptr, capturing));
    return 0;
  };
  std::vector<int64_t> key(offs, offs + p.nseq + 1);
  key.push_back(enc_mode);
  key.push_back((want_logits ? 1 : 0) | (want_tlog ? 2 : 0));
  const uint64_t ver = m->version.load();
  if (w.graph && w.graph_ver == ver && w.graph_gen == w.gen && w.graph_key == key) {
    g_launches += w.graph_launches;
    t_launches += w.graph_launches;
    IG_CU(cudaGraphLaunch(w.graph, st));
    g_graph_runs++;
    return 0;
  }
  if (w.seen != key) {  // first sight of this key: run as usual
    w.seen = std::move(key);
    return body(false);
  }
  if (w.graph) {
    cudaGraphExecDestroy(w.graph);
    w.graph = nullptr;
  }
  const long long l0 = t_launches;
  IG_CU(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  const int rc = body(true);
  cudaGraph_t g = nullptr;
  cudaError_t ce = cudaStreamEndCapture(st, &g);
  const long long launches = t_launches - l0;
  g_launches -= launches;  // counted when the graph runs
  t_launches -= launches;
  cudaGraphExec_t ex = nullptr;
  if (!rc && ce == cudaSuccess && g) ce = cudaGraphInstantiate(&ex, g, 0);
  if (g) cudaGraphDestroy(g);
  if (rc || ce != cudaSuccess || !ex) {
    // Not recordable: run it as usual (an error the capture hid shows here).
    cudaGetLastError();
    w.seen.clear();
    return body(false);
  }
  w.graph = ex;
  w.graph_key = std::move(key);
  w.graph_ver = ver;
  w.graph_gen = w.gen;
  w.graph_launches = launches;
  g_launches += launches;
  t_launches += launches;
  IG_CU(cudaGraphLaunch(ex, st));
  g_graph_records++;
  g_graph_runs++;
  return 0;
}

// A host call's kernels that gave up a bounded wait leave a code in the
// device error flag; the call copies the flag after its last kernel (one
// 4-byte copy on its stream) and fails when it holds a wait code, since its
// results are then not valid. The flag is not cleared (ig_device_error(1)
// does): it is one per device, and a wait that ran out means something on it
// is wrong.
void watch_device_error(Workspace &w, cudaStream_t st) {
  if (!w.err_host && cudaMallocHost(&w.err_host, sizeof(int32_t)) != cudaSuccess) {
    w.err_host = nullptr;
    cudaGetLastError();
    return;
  }
  *w.err_host = 0;
  cudaMemcpyFromSymbolAsync(w.err_host, g_device_error, sizeof(int32_t), 0, cudaMemcpyDeviceToHost, st);
}

int device_wait_failed(const Workspace &w) {
  const int e = w.err_host ? *w.err_host : 0;
  if (e < kDevTimeoutFull || e > kDevTimeoutAccum) return 0;
  return fail(IG_ERR_CUDA, "encode: a kernel gave up a bounded wait (device error " + std::to_string(e) +
                               "); the results of this call are not valid");
}

int encode_host(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, int32_t mode, float *out,
                size_t out_len, ig_dump *dump, double *logits, size_t logits_len, double *tlog, size_t tlog_len) {
  t_last_error.clear();
  if (!m || (nseq > 0 && !offs)) return fail(IG_ERR_BAD_ARG, "null argument");
  if (!m->replicas.empty())
    return encode_group(m, ids, offs, nseq, mode, out, out_len, dump, logits, logits_len, tlog, tlog_len);
  struct InFlight {
    std::atomic<int> &n;
    explicit InFlight(std::atomic<int> &c) : n(c) { n++; }
    ~InFlight() { n--; }
  } inflight(m->inflight);
  if (mode != IG_MODE_POOLED && mode != IG_MODE_TOKENS && !(mode == kModeMeanRows && !out))
    return fail(IG_ERR_BAD_ARG, "bad mode");
  DeviceGuard dg(m->device);
  int64_t nrows = 0;
  int max_len = 0;
  IG_TRY(scan_offsets(offs, nseq, &nrows, &max_len));
  if (nrows > 0 && !ids) return fail(IG_ERR_BAD_ARG, "null ids");
  const size_t H = m->H;
  const size_t need = mode == IG_MODE_POOLED ? (size_t)nseq * H : (size_t)nrows * H;
  if (out && out_len < need) return fail(IG_ERR_BAD_ARG, "output too short");
  size_t pl = 0, tl = 0;
  if (logits || tlog) {
    std::lock_guard<std::mutex> lk(m->mu);
    for (auto &h : m->heads) (h.per_token ? tl : pl) += h.rows;
  }
  if (logits && logits_len < (size_t)nseq * pl) return fail(IG_ERR_BAD_ARG, "logits too short");
  if (tlog && tlog_len < (size_t)nrows * tl) return fail(IG_ERR_BAD_ARG, "token logits too short");
  IG_TRY(ensure_rope(m, max_len));
  const size_t out_bytes = (logits ? 8 * (size_t)nseq * pl : 0) + (tlog ? 8 * (size_t)nrows * tl : 0) +
                           (out ? sizeof(float) * need : 0);
  Plan p;
  const int win[2] = {-1, m->cfg.local_attention / 2};
  IG_TRY(make_plan(offs, nseq, p, win));
  Workspace *w = nullptr;
  cudaStream_t st = nullptr;
  IG_TRY(acquire_ws(m, p, tl, pl, nullptr, false, &w));
  if (!w->own_stream) IG_CU(cudaStreamCreateWithFlags(&w->own_stream, cudaStreamNonBlocking));
  st = w->own_stream;
  int rc = upload_plan(*w, p, ids, st, false, m);  // also the id check (reference run's first check)
  const int enc_mode = (logits || tlog) ? (mode == kModeMeanRows ? kModeMeanRows : IG_MODE_POOLED) : mode;
  // Per-token logits for the host: the tail runs in chunks whose copies
  // overlap the kernels after them.
  const bool chunked_tail = tlog && tl && !out && !dump && p.N >= kTailMinRows && out_bytes >= kStageMinBytes;
  const bool graphed = !chunked_tail && !dump && !m->f32 && !g_prof.on && p.N > 0 && p.N <= kGraphMaxRows &&
                       graphs_enabled();
  if (!rc && graphed) {
    rc = run_graphed(m, *w, p, offs, enc_mode, logits != nullptr, tlog != nullptr, st);
  } else {
    if (!rc) rc = run_encoder(m, *w, w->ids, p, enc_mode, st, dump, false, !chunked_tail);
    if (!rc && chunked_tail) {
      rc = run_tail_staged(m, *w, p, enc_mode, st, logits, tlog, pl, tl);
      if (!rc) watch_device_error(*w, st);
      if (w->copy_stream) cudaStreamSynchronize(w->copy_stream);  // also after an early error
      cudaError_t se = cudaStreamSynchronize(st);
      if (!rc && se == cudaSuccess) rc = device_wait_failed(*w);
      release_ws(m, w, st, false);
      if (rc) return rc;
      if (se != cudaSuccess) return fail(IG_ERR_CUDA, std::string("encode: ") + cudaGetErrorString(se));
      return 0;
    }
    if (!rc && (logits || tlog))
      rc = run_heads(m, *w, p, st, logits ? w->logits : nullptr, tlog ? w->tlogits : nullptr, false);
  }
  std::vector<OutCopy> outs;
  if (logits && nseq && pl) outs.push_back({w->logits, logits, sizeof(double) * nseq * pl});
  if (tlog && p.N && tl) outs.push_back({w->tlogits, tlog, sizeof(double) * p.N * tl});
  if (out && need) {
    if (mode == IG_MODE_POOLED && p.N == 0) std::memset(out, 0, need * sizeof(float));
    else outs.push_back({mode == IG_MODE_POOLED ? w->pooled : w->xn, out, need * sizeof(float)});
  }
  if (!rc) watch_device_error(*w, st);
  if (!rc && out_bytes > 0) {
    rc = copy_out_staged(*w, st, outs);
  } else {
    for (auto &o : outs)
      if (!rc && cudaMemcpyAsync(o.dst, o.src, o.bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        rc = fail(IG_ERR_CUDA, "copy of the output");
  }
  cudaError_t se = cudaStreamSynchronize(st);
  if (!rc && se == cudaSuccess) rc = device_wait_failed(*w);
  release_ws(m, w, st, false);
  if (rc) return rc;
  if (se != cudaSuccess) return fail(IG_ERR_CUDA, std::string("encode: ") + cudaGetErrorString(se));
  return 0;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

int create_model(const ig_config *cfg, const WeightSource &w, int32_t device, ig_model **out) {
  t_last_error.clear();
  if (!cfg || !out) return fail(IG_ERR_BAD_ARG, "null argument");
  *out = nullptr;
  const ig_config &c = *cfg;
  // Config.validate (internal/modernbert/model.go:64-80).
  if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.intermediate <= 0 || c.vocab <= 0)
    return fail(IG_ERR_BAD_ARG, "modernbert: invalid dimensions");
  if (c.hidden % c.heads != 0 || (c.hidden / c.heads) % 2 != 0)
    return fail(IG_ERR_BAD_ARG, "modernbert: hidden_size " + std::to_string(c.hidden) + " incompatible with " +
                                    std::to_string(c.heads) + " heads");
  if (c.global_every <= 0 || c.local_attention <= 0) return fail(IG_ERR_BAD_ARG, "modernbert: invalid attention windows");
  if (c.pooling != IG_POOL_MEAN && c.pooling != IG_POOL_CLS) return fail(IG_ERR_BAD_ARG, "modernbert: pooling not supported");
  if (c.simd_lanes < 1 || c.simd_lanes > 32) return fail(IG_ERR_BAD_ARG, "simd_lanes must be in [1, 32]");
  if (c.hidden / c.heads != 64) return fail(IG_ERR_UNSUPPORTED, "head dimension must be 64 in this build");
  if (c.hidden > 4096 || c.intermediate > 8192) return fail(IG_ERR_UNSUPPORTED, "hidden/intermediate too large");
  for (int l = 0; l < c.layers; l++)
    if (!w.wqkv[l].data || !w.wo[l].data || !w.wi[l].data || !w.wo_mlp[l].data || !w.mlp_norm[l].data ||
        (l > 0 && !w.attn_norm[l].data))
      return fail(IG_ERR_BAD_ARG, "modernbert: tensor of layer " + std::to_string(l) + " missing");
  if (!w.emb_norm.data || !w.final_norm.data) return fail(IG_ERR_BAD_ARG, "modernbert: norm tensor missing");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return fail(IG_ERR_NO_DEVICE, "no such CUDA device");
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10)
    return fail(IG_ERR_NO_DEVICE, "device is not sm_100");
  DeviceGuard dg(device);
  std::unique_ptr<ig_model> m(new ig_model());
  m->cfg = c;
  m->device = device;
  m->H = c.hidden;
  m->I = c.intermediate;
  m->nh = c.heads;
  m->D = c.hidden / c.heads;
  m->ldk = (int)align_up(std::max(c.hidden, c.intermediate), 16);
  m->NI = (c.intermediate + 127) / 128 * 256;
  const int H = m->H, I = m->I;
  if (w.tok_embeddings) {
    float *e = nullptr;
    IG_CU(cudaMalloc(&e, (size_t)c.vocab * H * sizeof(float)));
    m->emb_allocs.push_back(e);
    IG_CU(cudaMemcpy(e, w.tok_embeddings, (size_t)c.vocab * H * sizeof(float), cudaMemcpyHostToDevice));
    m->emb.fmt = IG_EMB_F32;
    m->emb.f32 = e;
  }
  void *stage = nullptr;
  int32_t *dperm = nullptr;
  const size_t stage_elems = (size_t)std::max(3 * H, 2 * I) * std::max(H, I);
  IG_CU(cudaMalloc(&stage, stage_elems * 2));
  IG_CU(cudaMalloc(&dperm, sizeof(int32_t) * m->NI));
  struct Free {
    void *a, *b;
    ~Free() {
      cudaFree(a);
      cudaFree(b);
    }
  } free_tmp{stage, dperm};
  IG_TRY(upload_view(m.get(), &m->emb_norm, w.emb_norm, H, stage));
  IG_TRY(upload_view(m.get(), &m->final_norm, w.final_norm, H, stage));
  // Wi rows interleaved per 128: [input 128t.., gate 128t..] so one 256-wide
  // tile holds matching GELU inputs and gates.
  std::vector<int32_t> wi_perm(m->NI);
  for (int p = 0; p < m->NI; p++) {
    const int t = p / 256, r = p % 256;
    const int ch = 128 * t + (r % 128);
    wi_perm[p] = ch < I ? (r < 128 ? ch : I + ch) : -1;
  }
  m->layers.resize(c.layers);
  for (int l = 0; l < c.layers; l++) {
    DevLayer &L = m->layers[l];
    if (l > 0) IG_TRY(upload_view(m.get(), &L.attn_norm, w.attn_norm[l], H, stage));
    IG_TRY(upload_view(m.get(), &L.mlp_norm, w.mlp_norm[l], H, stage));
    // The float32 matrices (kept for SetInt8(false)) are quantized from the
    // device copy (PackB8 of the decoded weights, as the reference packs them).
    IG_TRY(upload_view(m.get(), &L.fqkv, w.wqkv[l], (size_t)3 * H * H, stage));
    IG_TRY(upload_view(m.get(), &L.fo, w.wo[l], (size_t)H * H, stage));
    IG_TRY(upload_view(m.get(), &L.fwi, w.wi[l], (size_t)2 * I * H, stage));
    IG_TRY(upload_view(m.get(), &L.fwom, w.wo_mlp[l], (size_t)H * I, stage));
    IG_TRY(pack_matrix(m.get(), L.qkv, L.fqkv, 3 * H, H, {}, dperm));
    IG_TRY(pack_matrix(m.get(), L.o, L.fo, H, H, {}, dperm));
    IG_TRY(pack_matrix(m.get(), L.wi, L.fwi, 2 * I, H, wi_perm, dperm));
    IG_TRY(pack_matrix(m.get(), L.wom, L.fwom, H, I, {}, dperm));
  }
  IG_TRY(ensure_rope(m.get(), 512));
  *out = m.release();
  return 0;
}

}  // namespace

extern "C" {

int ig_model_create(const ig_config *cfg, const ig_weights *w, int32_t device, ig_model **out) {
  t_last_error.clear();
  if (!cfg || !w || !out) return fail(IG_ERR_BAD_ARG, "null argument");
  if (cfg->layers <= 0 || cfg->layers > 4096) return fail(IG_ERR_BAD_ARG, "modernbert: invalid dimensions");
  if (!w->attn_norm || !w->wqkv || !w->wo || !w->mlp_norm || !w->wi || !w->wo_mlp)
    return fail(IG_ERR_BAD_ARG, "null argument");
  WeightSource src;
  src.tok_embeddings = w->tok_embeddings;
  src.emb_norm = {IG_DT_F32, w->emb_norm};
  src.final_norm = {IG_DT_F32, w->final_norm};
  for (int l = 0; l < cfg->layers; l++) {
    src.attn_norm.push_back({IG_DT_F32, l > 0 ? w->attn_norm[l] : nullptr});
    src.wqkv.push_back({IG_DT_F32, w->wqkv[l]});
    src.wo.push_back({IG_DT_F32, w->wo[l]});
    src.mlp_norm.push_back({IG_DT_F32, w->mlp_norm[l]});
    src.wi.push_back({IG_DT_F32, w->wi[l]});
    src.wo_mlp.push_back({IG_DT_F32, w->wo_mlp[l]});
  }
  return create_model(cfg, src, device, out);
}

int ig_model_create_stored(const ig_config *cfg, const ig_stored_weights *w, int32_t device, ig_model **out) {
  t_last_error.clear();
  if (!cfg || !w || !out) return fail(IG_ERR_BAD_ARG, "null argument");
  if (cfg->layers <= 0 || cfg->layers > 4096) return fail(IG_ERR_BAD_ARG, "modernbert: invalid dimensions");
  if (!w->attn_norm || !w->wqkv || !w->wo || !w->mlp_norm || !w->wi || !w->wo_mlp)
    return fail(IG_ERR_BAD_ARG, "null argument");
  WeightSource src;
  src.tok_embeddings = nullptr;  // ig_model_set_embeddings uploads the table as stored
  auto tv = [](const ig_tensor tensor) { return TensorView{tensor.dtype, tensor.data}; };
  src.emb_norm = tv(w->emb_norm);
  src.final_norm = tv(w->final_norm);
  for (int l = 0; l < cfg->layers; l++) {
    src.attn_norm.push_back(l > 0 ? tv(w->attn_norm[l]) : TensorView{IG_DT_F32, nullptr});
    src.wqkv.push_back(tv(w->wqkv[l]));
    src.wo.push_back(tv(w->wo[l]));
    src.mlp_norm.push_back(tv(w->mlp_norm[l]));
    src.wi.push_back(tv(w->wi[l]));
    src.wo_mlp.push_back(tv(w->wo_mlp[l]));
  }
  return create_model(cfg, src, device, out);
}

void ig_model_destroy(ig_model *m) { delete m; }

int ig_model_set_embeddings(ig_model *m, const ig_embedding_table *t) {
  t_last_error.clear();
  if (!m || !t) return fail(IG_ERR_BAD_ARG, "null argument");
  for (ig_model *r : m->replicas)
    if (int rc = ig_model_set_embeddings(r, t)) return rc;
  if (!m->replicas.empty()) return 0;
  const int V = m->cfg.vocab, H = m->H;
  DeviceGuard dg(m->device);
  EmbTable e{t->format, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  std::vector<void *> allocs;
  auto put = [&](const void *src, size_t bytes) -> void * {
    void *d = nullptr;
    if (cudaMalloc(&d, std::max<size_t>(bytes, 16)) != cudaSuccess) return nullptr;
    allocs.push_back(d);
    if (bytes && cudaMemcpy(d, src, bytes, cudaMemcpyHostToDevice) != cudaSuccess) return nullptr;
    return d;
  };
  auto undo = [&](int code, const std::string &msg) {
    for (void *p : allocs) cudaFree(p);
    return fail(code, msg);
  };
  if (t->format == IG_EMB_F32) {
    if (!t->f32) return fail(IG_ERR_BAD_ARG, "indecis: float32 table missing");
    if (!(e.f32 = (const float *)put(t->f32, (size_t)V * H * 4))) return undo(IG_ERR_CUDA, "cudaMalloc failed");
  } else if (t->format == IG_EMB_BF16) {
    if (!t->bf16 || t->n_exact < 0 || (t->n_exact && (!t->exact_ids || !t->exact_rows)))
      return fail(IG_ERR_BAD_ARG, "indecis: malformed exact rows");
    // newMappedEmbeddings (embeddings.go:33-47): id -> rank, a later listing of
    // an id replacing an earlier one, as the reference's map does.
    std::vector<int32_t> idx(V, -1);
    for (int i = 0; i < t->n_exact; i++) {
      const int id = t->exact_ids[i];
      if (id < 0 || id >= V) return fail(IG_ERR_BAD_ARG, "indecis: exact row " + std::to_string(id) + " out of vocabulary");
      idx[id] = i;
    }
    if (!(e.bf16 = (const uint16_t *)put(t->bf16, (size_t)V * H * 2)) ||
        !(e.exact_idx = (const int32_t *)put(idx.data(), (size_t)V * 4)) ||
        !(e.exact_rows = (const float *)put(t->exact_rows, (size_t)t->n_exact * H * 4)))
      return undo(IG_ERR_CUDA, "cudaMalloc failed");
  } else if (t->format == IG_EMB_INT8) {
    if (!t->i8 || !t->scale) return fail(IG_ERR_BAD_ARG, "indecis: int8 table or scales missing");
    if (!(e.i8 = (const int8_t *)put(t->i8, (size_t)V * H)) || !(e.scale = (const float *)put(t->scale, (size_t)V * 4)))
      return undo(IG_ERR_CUDA, "cudaMalloc failed");
  } else {
    return fail(IG_ERR_BAD_ARG, "unknown embedding table format");
  }
  // The old table is released once no queued work can read it.
  std::lock_guard<std::mutex> lk(m->mu);
  cudaDeviceSynchronize();
  for (void *p : m->emb_allocs) cudaFree(p);
  m->emb_allocs = std::move(allocs);
  m->emb = e;
  m->version++;
  return 0;
}

int ig_model_set_heads(ig_model *m, int32_t nheads, const ig_head *heads) {
  t_last_error.clear();
  if (!m || nheads < 0 || (nheads && !heads)) return fail(IG_ERR_BAD_ARG, "null argument");
  for (ig_model *r : m->replicas)
    if (int rc = ig_model_set_heads(r, nheads, heads)) return rc;
  if (!m->replicas.empty()) return 0;
  DeviceGuard dg(m->device);
  std::vector<DevHead> hs(nheads);
  for (int i = 0; i < nheads; i++) {
    if (heads[i].rows <= 0 || !heads[i].w || !heads[i].b) return fail(IG_ERR_BAD_ARG, "bad head");
    hs[i].rows = heads[i].rows;
    hs[i].per_token = heads[i].per_token;
    const size_t nw = (size_t)heads[i].rows * m->H;
    IG_CU(cudaMalloc(&hs[i].w, nw * sizeof(float)));
    IG_CU(cudaMalloc(&hs[i].b, heads[i].rows * sizeof(float)));
    IG_CU(cudaMemcpy(hs[i].w, heads[i].w, nw * sizeof(float), cudaMemcpyHostToDevice));
    IG_CU(cudaMemcpy(hs[i].b, heads[i].b, heads[i].rows * sizeof(float), cudaMemcpyHostToDevice));
  }
  IG_CU(cudaDeviceSynchronize());
  std::lock_guard<std::mutex> lk(m->mu);
  for (auto &h : m->heads) {
    cudaFree(h.w);
    cudaFree(h.b);
  }
  m->heads = hs;
  m->version++;
  return 0;
}

int ig_encode(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, int32_t mode, float *out,
              size_t out_len) {
  if (!out) return fail(IG_ERR_BAD_ARG, "null output");
  if (mode != IG_MODE_POOLED && mode != IG_MODE_TOKENS) return fail(IG_ERR_BAD_ARG, "bad mode");
  return encode_host(m, ids, offs, nseq, mode, out, out_len, nullptr, nullptr, 0, nullptr, 0);
}

int ig_encode_dump(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, int32_t mode, float *out,
                   size_t out_len, ig_dump *dump) {
  if (mode != IG_MODE_POOLED && mode != IG_MODE_TOKENS) return fail(IG_ERR_BAD_ARG, "bad mode");
  return encode_host(m, ids, offs, nseq, mode, out, out_len, dump, nullptr, 0, nullptr, 0);
}

int ig_window_logits(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, double *logits,
                     size_t logits_len, double *token_logits, size_t token_len) {
  if (!logits && !token_logits) return fail(IG_ERR_BAD_ARG, "no output");
  return encode_host(m, ids, offs, nseq, kModeMeanRows, nullptr, 0, nullptr, logits, logits_len, token_logits,
                     token_len);
}

int ig_model_set_int8(ig_model *m, int32_t on) {
  t_last_error.clear();
  if (!m) return fail(IG_ERR_BAD_ARG, "null model");
  if (on == 0 && m->D != 64) return fail(IG_ERR_UNSUPPORTED, "the float path needs a head dimension of 64");
  if (on == 0 && m->cfg.simd_lanes != 8) return fail(IG_ERR_UNSUPPORTED, "the float path needs simd_lanes 8");
  for (ig_model *r : m->replicas)
    if (int rc = ig_model_set_int8(r, on)) return rc;
  std::lock_guard<std::mutex> lk(m->mu);
  m->f32 = on == 0;
  m->version++;
  return 0;
}

int ig_model_dims(ig_model *m, int32_t *vocab, int32_t *hidden) {
  if (!m) return fail(IG_ERR_BAD_ARG, "null model");
  if (vocab) *vocab = m->cfg.vocab;
  if (hidden) *hidden = m->H;
  return 0;
}

int ig_model_head_rows(ig_model *m, int32_t *pooled_rows, int32_t *token_rows) {
  t_last_error.clear();
  if (!m || !pooled_rows || !token_rows) return fail(IG_ERR_BAD_ARG, "null argument");
  if (!m->replicas.empty()) return ig_model_head_rows(m->replicas[0], pooled_rows, token_rows);
  int32_t pl = 0, tl = 0;
  std::lock_guard<std::mutex> lk(m->mu);
  for (auto &h : m->heads) (h.per_token ? tl : pl) += h.rows;
  *pooled_rows = pl, *token_rows = tl;
  return 0;
}

int ig_logits(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, double *logits, size_t logits_len,
              double *token_logits, size_t token_len) {
  if (!logits && !token_logits) return fail(IG_ERR_BAD_ARG, "no output");
  return encode_host(m, ids, offs, nseq, IG_MODE_POOLED, nullptr, 0, nullptr, logits, logits_len, token_logits,
                     token_len);
}

int ig_encode_device(ig_model *m, const int32_t *d_ids, const int64_t *offs, int32_t nseq, int32_t mode,
                     float *d_out, void *stream) {
  t_last_error.clear();
  if (!m || !offs || !d_out) return fail(IG_ERR_BAD_ARG, "null argument");
  if (mode != IG_MODE_POOLED && mode != IG_MODE_TOKENS) return fail(IG_ERR_BAD_ARG, "bad mode");
  if (!m->replicas.empty())
    return fail(IG_ERR_BAD_ARG, "a model on several devices takes device buffers through ig_model_replica");
  DeviceGuard dg(m->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  IG_CU(cudaStreamIsCapturing(st, &cs));
  const bool capturing = cs != cudaStreamCaptureStatusNone;
  Plan p;
  const int win[2] = {-1, m->cfg.local_attention / 2};
  IG_TRY(make_plan(offs, nseq, p, win));
  if (capturing && m->rope_npos < p.max_len) return fail(IG_ERR_BAD_ARG, "run once before capturing");
  IG_TRY(ensure_rope(m, p.max_len));
  Workspace *w = nullptr;
  IG_TRY(acquire_ws(m, p, 0, 0, st, capturing, &w));
  int rc = upload_plan(*w, p, nullptr, st, capturing);
  if (!rc) rc = run_encoder(m, *w, d_ids, p, mode, st, nullptr, capturing);
  if (!rc && p.N) {
    const size_t H = m->H;
    if (mode == IG_MODE_POOLED)
      rc = cudaMemcpyAsync(d_out, w->pooled, sizeof(float) * nseq * H, cudaMemcpyDeviceToDevice, st) ? IG_ERR_CUDA : 0;
    else
      rc = cudaMemcpyAsync(d_out, w->xn, sizeof(float) * p.N * H, cudaMemcpyDeviceToDevice, st) ? IG_ERR_CUDA : 0;
  } else if (!rc && mode == IG_MODE_POOLED && nseq) {
    rc = cudaMemsetAsync(d_out, 0, sizeof(float) * nseq * m->H, st) ? IG_ERR_CUDA : 0;
  }
  release_ws(m, w, st, capturing);
  return rc;
}

int ig_logits_device(ig_model *m, const int32_t *d_ids, const int64_t *offs, int32_t nseq, double *d_logits,
                     double *d_token_logits, void *stream) {
  t_last_error.clear();
  if (!m || !offs || (!d_logits && !d_token_logits)) return fail(IG_ERR_BAD_ARG, "null argument");
  if (!m->replicas.empty())
    return fail(IG_ERR_BAD_ARG, "a model on several devices takes device buffers through ig_model_replica");
  DeviceGuard dg(m->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  IG_CU(cudaStreamIsCapturing(st, &cs));
  const bool capturing = cs != cudaStreamCaptureStatusNone;
  Plan p;
  const int win[2] = {-1, m->cfg.local_attention / 2};
  IG_TRY(make_plan(offs, nseq, p, win));
  if (capturing && m->rope_npos < p.max_len) return fail(IG_ERR_BAD_ARG, "run once before capturing");
  IG_TRY(ensure_rope(m, p.max_len));
  Workspace *w = nullptr;
  IG_TRY(acquire_ws(m, p, 0, 0, st, capturing, &w));
  int rc = upload_plan(*w, p, nullptr, st, capturing);
  if (!rc) rc = run_encoder(m, *w, d_ids, p, IG_MODE_POOLED, st, nullptr, capturing);
  if (!rc) rc = run_heads(m, *w, p, st, d_logits, d_token_logits, capturing);
  release_ws(m, w, st, capturing);
  return rc;
}

int ig_profile(int32_t enable) {
  t_last_error.clear();
  if (enable) {
    cudaDeviceSynchronize();
    std::lock_guard<std::mutex> lk(g_prof.mu);
    for (auto &r : g_prof.recs) {
      g_prof.pool.push_back(r.a);
      g_prof.pool.push_back(r.b);
    }
    g_prof.recs.clear();
    g_launches = 0;
  }
  g_prof.on = enable != 0;
  return 0;
}

int ig_profile_only(const char *name) {
  t_last_error.clear();
  std::lock_guard<std::mutex> lk(g_prof.mu);
  g_prof.only = name ? name : "";
  return 0;
}

int64_t ig_profile_report(char *buf, size_t len) {
  cudaDeviceSynchronize();
  struct Agg {
    std::string name;
    long long launches = 0;
    double ms = 0, bytes = 0, ops = 0;
    long long records = 0;
  };
  std::vector<Agg> aggs;
  {
    std::lock_guard<std::mutex> lk(g_prof.mu);
    for (auto &r : g_prof.recs) {
      float ms = 0.0f;
      if (cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) ms = 0.0f;
      Agg *a = nullptr;
      for (auto &x : aggs)
        if (x.name == r.name) a = &x;
      if (!a) {
        aggs.push_back(Agg{r.name});
        a = &aggs.back();
      }
      a->launches += r.launches;
      a->records += 1;
      a->ms += ms;
      a->bytes += r.bytes;
      a->ops += r.ops;
    }
  }
  std::string js = "{\"launches\": " + std::to_string((long long)g_launches) +
                   ", \"graphs_recorded\": " + std::to_string((long long)g_graph_records) +
                   ", \"graph_runs\": " + std::to_string((long long)g_graph_runs) + ", \"kernels\": [";
  char tmp[512];
  for (size_t i = 0; i < aggs.size(); i++) {
    snprintf(tmp, sizeof(tmp), "%s{\"name\": \"%s\", \"launches\": %lld, \"records\": %lld, \"ms\": %.6f, "
             "\"bytes\": %.1f, \"ops\": %.1f}", i ? ", " : "", aggs[i].name.c_str(), aggs[i].launches,
             aggs[i].records, aggs[i].ms, aggs[i].bytes, aggs[i].ops);
    js += tmp;
  }
  js += "]}";
  if (buf && len) {
    const size_t n = std::min(len - 1, js.size());
    std::memcpy(buf, js.data(), n);
    buf[n] = 0;
  }
  return (int64_t)js.size();
}

const char *ig_last_error(void) { return t_last_error.c_str(); }

int32_t ig_device_error(int32_t reset) {
  cudaDeviceSynchronize();
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  }
  return v;
}

int ig_gemm_u8s8(const uint8_t *A, int32_t lda, const int8_t *B, int32_t ldb, int32_t M, int32_t N, int32_t K,
                 const float *sa, const float *sb, const float *zc, float *C, int32_t ldc, int32_t accumulate,
                 int32_t *acc_out, void *stream) {
  t_last_error.clear();
  if (M < 0 || N < 0 || K < 0) return fail(IG_ERR_BAD_ARG, "negative size");
  if (!acc_out && (!sa || !sb || !zc || !C)) return fail(IG_ERR_BAD_ARG, "null argument");
  if (ldc < N) return fail(IG_ERR_BAD_ARG, "ldc must be >= N");
  GemmArgs g{A, B, M, N, K, lda, ldb, 0};
  GemmEpilogue e{};
  e.sa = sa;
  e.sb = sb;
  e.zc = zc;
  e.C = C;
  e.ldc = ldc;
  e.accumulate = accumulate;
  e.acc_out = acc_out;
  int rc = gemm_u8s8(g, e, acc_out ? kEpiI32 : kEpiF32, reinterpret_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "ig_gemm_u8s8: bad shape, stride or alignment (lda/ldb multiples of 16, >= K)");
  return 0;
}

int ig_gemm_geglu_quant(const uint8_t *A, int32_t lda, const int8_t *B, int32_t ldb, int32_t M, int32_t I, int32_t K,
                        const float *sa, const float *sb, const float *zc, uint8_t *q, int32_t ldq, float *sa_out,
                        void *stream) {
  t_last_error.clear();
  if (M < 0 || I < 0 || K < 0) return fail(IG_ERR_BAD_ARG, "negative size");
  if (!A || !B || !sa || !sb || !zc || !q || !sa_out) return fail(IG_ERR_BAD_ARG, "null argument");
  GemmArgs g{A, B, M, 2 * I, K, lda, ldb, 256};
  GemmEpilogue e{};
  e.sa = sa;
  e.sb = sb;
  e.zc = zc;
  e.geglu_n = I;
  e.q_out = q;
  e.ldq = ldq;
  e.sa_out = sa_out;
  if (!gemm_geglu_q_fits(2 * I, e))
    return fail(IG_ERR_UNSUPPORTED, "ig_gemm_geglu_quant: I must be a multiple of 128 and at most 1024, ldq a "
                                    "multiple of 16 and >= I, q 16-byte aligned");
  int rc = gemm_u8s8(g, e, kEpiGegluQ, reinterpret_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "ig_gemm_geglu_quant: bad shape, stride or alignment");
  return 0;
}

int ig_quantize_rows(const float *x, int32_t ldx, int32_t M, int32_t K, uint8_t *q, int32_t ldq, float *sa,
                     void *stream) {
  t_last_error.clear();
  int rc = launch_quant_rows(x, ldx, M, K, q, ldq, sa, reinterpret_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "ig_quantize_rows failed") : 0;
}

int ig_layernorm_quant(const float *x, const float *gamma, int32_t M, int32_t H, double eps, int32_t simd_lanes,
                       float *xn, uint8_t *q, int32_t ldq, float *sa, void *stream) {
  t_last_error.clear();
  if (!gamma) return fail(IG_ERR_BAD_ARG, "null gamma");
  int rc = launch_ln_quant(x, gamma, M, H, eps, simd_lanes, xn, q, ldq, sa, reinterpret_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "ig_layernorm_quant failed") : 0;
}

int ig_pack_b8(const float *w, int32_t n, int32_t k, int8_t *q, int32_t ldq, float *scale, float *zc,
               int32_t *colsum, void *stream) {
  t_last_error.clear();
  int rc = launch_pack_b8(w, n, k, nullptr, n, q, ldq, scale, zc, colsum, reinterpret_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "ig_pack_b8 failed") : 0;
}

int ig_attention(const float *qkv, int32_t hidden, int32_t heads, const int64_t *offs, int32_t nseq, int32_t window,
                 int32_t simd_lanes, float *ctx, void *stream) {
  t_last_error.clear();
  if (!qkv || !ctx || !offs || heads <= 0 || hidden % heads) return fail(IG_ERR_BAD_ARG, "bad argument");
  Plan p;
  const int win[2] = {window < 0 ? -1 : window, -2};
  IG_TRY(make_plan(offs, nseq, p, win, true));
  if (p.N == 0) return 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t N = p.N, nh = heads, D = hidden / heads;
  AttnArgs a{};
  a.qkv = qkv;
  a.H = hidden;
  a.nh = heads;
  a.D = (int)D;
  a.nseq = nseq;
  a.max_len = p.max_len;
  a.window = window;
  a.scale = (float)(1.0 / std::sqrt((double)D));
  a.V = simd_lanes;
  a.N = p.N;
  a.ctx = ctx;
  std::vector<void *> bufs;
  auto take = [&](size_t bytes) {
    void *v = nullptr;
    if (cudaMalloc(&v, std::max<size_t>(bytes, 16)) != cudaSuccess) return (void *)nullptr;
    bufs.push_back(v);
    return v;
  };
  int32_t *d_offs = (int32_t *)take(4 * (nseq + 1));
  int32_t *d_rs = (int32_t *)take(4 * N);
  int4 *d_tc = (int4 *)take(16 * p.tc[0].size());
  int2 *d_v1 = (int2 *)take(8 * p.v1[0].size());
  int2 *d_fb = (int2 *)take(8 * p.fb.size());
  a.qa = (uint8_t *)take(N * nh * D);
  a.kq = (int8_t *)take(N * nh * D);
  a.vq = (int8_t *)take(N * nh * D);
  a.sq = (float *)take(4 * N * nh);
  a.ks = (float *)take(4 * N * nh);
  a.kzc = (float *)take(4 * N * nh);
  a.kmean = (float *)take(4 * nseq * nh * D);
  a.vs = (float *)take(4 * nseq * nh * D);
  a.vinv = (float *)take(4 * nseq * nh * D);
  a.offs = d_offs;
  a.row_seq = d_rs;
  int rc = 0;
  for (void *b : bufs)
    if (!b) rc = fail(IG_ERR_CUDA, "cudaMalloc failed");
  if (!rc) {
    cudaMemcpyAsync(d_offs, p.offs.data(), 4 * (nseq + 1), cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(d_rs, p.row_seq.data(), 4 * N, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(d_tc, p.tc[0].data(), 16 * p.tc[0].size(), cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(d_v1, p.v1[0].data(), 8 * p.v1[0].size(), cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(d_fb, p.fb.data(), 8 * p.fb.size(), cudaMemcpyHostToDevice, st);
    a.row_tiles = d_fb;
    a.nrow_tiles = (int)p.fb.size();
    if (attn_short_fits(a)) {
      rc = launch_attn_short(a, st);
    } else {
      rc = launch_attention(a, st);
      if (!rc) rc = launch_attend_tc(a, d_tc, p.tc_short[0], (int)p.tc[0].size() - p.tc_short[0], st);
      if (!rc) rc = launch_attend(a, d_v1, (int)p.v1[0].size(), st);
    }
    // Heads whose Q or K values are non-finite or overflow-sized: recomputed
    // with the reference's conversions (the fast kernels' results replaced).
    if (!rc && a.D == 64) rc = launch_attn_exact(a, st);
    if (rc) fail(rc, "ig_attention launch failed");
  }
  cudaStreamSynchronize(st);
  for (void *b : bufs) cudaFree(b);
  return rc;
}

}  // extern "C"
