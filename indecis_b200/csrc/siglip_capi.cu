// C ABI of the SigLIP vision tower: model creation (weights to the device,
// int8 packing there), the batched forward of Vision.forward
// (internal/siglip/vision.go:101-141) and its per-layer dump.
//
// Layer order on the device, per batch of n images (N = n*T rows):
//   patch embedding (float32 chains, patches read from the pixels) + bias + pos
//   per layer: LN1+beta -> int8 rows; qkv int8 GEMM + bias; float attention;
//              int8 rows; out GEMM + bias, added to x; LN2+beta -> int8 rows;
//              fc1 GEMM + bias + GeluTanh; outlier channels per image set
//              aside; int8 rows; fc2 GEMM; outlier terms + bias added to x
//   post LN+beta; pooling head: K|V float32 product, probe attention,
//   out-proj, LN+beta, fc1 + GeluTanh, fc2 + residual.
// Included into the library's single translation unit after capi.cu (it
// shares its error reporting, device guard and profiler).

#include <algorithm>
#include <cmath>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace ig {

struct VisMat {
  int8_t *q = nullptr;
  float *scale = nullptr, *zc = nullptr;
  int n = 0, k = 0, ld = 0;
};

struct VisLayer {
  float *ln1g = nullptr, *ln1b = nullptr, *ln2g = nullptr, *ln2b = nullptr;
  float *bqkv = nullptr, *bo = nullptr, *b1 = nullptr, *b2 = nullptr;
  VisMat qkv, o, fc1, fc2;
};

struct VisWork {
  int cap = 0;  // images
  std::vector<void *> allocs;
  float *x = nullptr, *qkv = nullptr, *ctx = nullptr, *tmp = nullptr, *mlp = nullptr, *kv = nullptr;
  uint8_t *xq = nullptr;
  float *sa = nullptr, *colmax = nullptr, *outv = nullptr, *outw = nullptr;
  int32_t *cand = nullptr, *outl = nullptr, *nout = nullptr;
  float *att = nullptr, *hout = nullptr, *hn = nullptr, *hm = nullptr, *pooled = nullptr, *pix = nullptr;
  float *patches = nullptr;  // the patch states Forward returns
  cudaStream_t own = nullptr;
  ~VisWork() {
    for (void *p : allocs) cudaFree(p);
    if (own) cudaStreamDestroy(own);
  }
};

constexpr float kVisOutlierRatio = 6.0f;  // internal/siglip/encoder.go:165

}  // namespace ig

struct ig_vision {
  ig_vision_config cfg{};
  int device = 0;
  int H = 0, M = 0, T = 0, nh = 0, ldk = 0, K0 = 0;
  std::vector<void *> allocs;
  float *patch_w = nullptr, *patch_b = nullptr, *pos = nullptr, *post_g = nullptr, *post_b = nullptr;
  float *probe_q = nullptr, *kv_w = nullptr, *kv_b = nullptr, *hout_w = nullptr, *hout_b = nullptr;
  float *hln_g = nullptr, *hln_b = nullptr, *hfc1_w = nullptr, *hfc1_b = nullptr, *hfc2_w = nullptr,
        *hfc2_b = nullptr;
  std::vector<ig::VisLayer> layers;
  std::mutex mu;  // one forward at a time: they share the workspace
  std::unique_ptr<ig::VisWork> work;
  ~ig_vision() {
    work.reset();
    for (void *p : allocs) cudaFree(p);
  }
};

namespace ig {
namespace {

template <class T>
int vis_alloc(std::vector<void *> &list, T **p, size_t count) {
  void *v = nullptr;
  IG_CU(cudaMalloc(&v, std::max<size_t>(count * sizeof(T), 16)));
  list.push_back(v);
  *p = reinterpret_cast<T *>(v);
  return 0;
}

int vis_upload(ig_vision *m, float **dst, const float *src, size_t count) {
  if (!src) return fail(IG_ERR_BAD_ARG, "siglip: a weight is missing");
  IG_TRY(vis_alloc(m->allocs, dst, count));
  IG_CU(cudaMemcpy(*dst, src, count * sizeof(float), cudaMemcpyHostToDevice));
  return 0;
}

int vis_pack(ig_vision *m, VisMat &dm, const float *w, int n, int k, float *tmp) {
  if (!w) return fail(IG_ERR_BAD_ARG, "siglip: a weight is missing");
  dm.n = n, dm.k = k, dm.ld = (int)align_up(k, 16);
  IG_TRY(vis_alloc(m->allocs, &dm.q, (size_t)n * dm.ld));
  IG_TRY(vis_alloc(m->allocs, &dm.scale, n));
  IG_TRY(vis_alloc(m->allocs, &dm.zc, n));
  IG_CU(cudaMemcpy(tmp, w, (size_t)n * k * sizeof(float), cudaMemcpyHostToDevice));
  IG_TRY(launch_pack_b8(tmp, n, k, nullptr, n, dm.q, dm.ld, dm.scale, dm.zc, nullptr, 0));
  IG_CU(cudaDeviceSynchronize());
  return 0;
}

int vis_work(ig_vision *m, int n, VisWork **out) {
  if (!m->work || m->work->cap < n) {
    // Calls on device buffers return once enqueued: let them finish before
    // the workspace they use is replaced.
    if (m->work) IG_CU(cudaDeviceSynchronize());
    auto w = std::make_unique<VisWork>();
    const size_t N = (size_t)n * m->T, H = m->H, M = m->M;
    auto &L = w->allocs;
    IG_TRY(vis_alloc(L, &w->x, N * H));
    IG_TRY(vis_alloc(L, &w->qkv, N * 3 * H));
    IG_TRY(vis_alloc(L, &w->ctx, N * H));
    IG_TRY(vis_alloc(L, &w->tmp, N * H));
    IG_TRY(vis_alloc(L, &w->mlp, N * M));
    IG_TRY(vis_alloc(L, &w->kv, N * 2 * H));
    IG_TRY(vis_alloc(L, &w->xq, N * m->ldk));
    IG_TRY(vis_alloc(L, &w->sa, N));
    IG_TRY(vis_alloc(L, &w->colmax, (size_t)n * M));
    IG_TRY(vis_alloc(L, &w->cand, (size_t)n * M));
    IG_TRY(vis_alloc(L, &w->outl, (size_t)n * 32));
    IG_TRY(vis_alloc(L, &w->nout, (size_t)n));
    IG_TRY(vis_alloc(L, &w->outv, N * 32));
    IG_TRY(vis_alloc(L, &w->outw, (size_t)n * 32 * H));
    IG_TRY(vis_alloc(L, &w->att, (size_t)n * H));
    IG_TRY(vis_alloc(L, &w->hout, (size_t)n * H));
    IG_TRY(vis_alloc(L, &w->hn, (size_t)n * H));
    IG_TRY(vis_alloc(L, &w->hm, (size_t)n * M));
    IG_TRY(vis_alloc(L, &w->pooled, (size_t)n * H));
    IG_TRY(vis_alloc(L, &w->pix, (size_t)n * 3 * m->cfg.image_size * m->cfg.image_size));
    IG_TRY(vis_alloc(L, &w->patches, N * H));
    IG_CU(cudaStreamCreateWithFlags(&w->own, cudaStreamNonBlocking));
    w->cap = n;
    m->work = std::move(w);
  }
  *out = m->work.get();
  return 0;
}

double vis_gemm_bytes(size_t rows, int n, int k, double out_row_bytes) {
  return (double)rows * k + (double)n * k + 8.0 * n + 4.0 * rows + (double)rows * out_row_bytes;
}

// The tower on device pixels; results in w.x (patch states) and w.pooled.
// layer > 0 with !pool stops after that many layers (w.x then holds them);
// d_patches (optional) receives the patch states at the point Forward
// returns them.
int vis_run(ig_vision *m, VisWork &w, const float *d_pix, int n, int layer, bool pool, float *d_patches,
            cudaStream_t st, ig_vision_dump *dump) {
  const ig_vision_config &c = m->cfg;
  const int H = m->H, M = m->M, T = m->T, V = c.simd_lanes, L = c.layers;
  const size_t N = (size_t)n * T;
  const float scale = (float)(1 / std::sqrt((double)(H / m->nh)));
  const bool dl_any = dump != nullptr;
  {
    F32Gemm p{};
    p.pix = d_pix, p.S = c.image_size, p.P = c.patch_size, p.T = T;
    p.W = m->patch_w, p.ldw = m->K0, p.M = (int)N, p.N = H, p.K = m->K0;
    p.bias = m->patch_b, p.add = m->pos, p.ldadd = H, p.add_mod = T, p.C = w.x, p.ldc = H, p.V = V;
    ProfScope ps("vis_patch_embed", 4.0 * N * m->K0 + 4.0 * H * m->K0 + 4.0 * N * H, 2.0 * N * H * m->K0, 1, st);
    IG_TRY(launch_f32_gemm(p, st));
  }
  if (dl_any && dump->x_embed) IG_TRY(copy_rows_d2h(dump->x_embed, w.x, H * 4, H * 4, N, st));
  const int nl = (layer > 0 && !pool) ? layer : L;
  for (int l = 0; l < nl; l++) {
    const VisLayer &Y = m->layers[l];
    const bool dl = dl_any && dump->layer == l;
    {
      ProfScope ps("vis_ln_quant", N * (5.0 * H + 4), 0, 1, st);
      IG_TRY(launch_ln_beta(w.x, Y.ln1g, Y.ln1b, (int)N, H, c.eps, V, nullptr, w.xq, m->ldk, w.sa, st));
    }
    if (dl) {
      IG_TRY(copy_rows_d2h(dump->h1q, w.xq, H, m->ldk, N, st));
      IG_TRY(copy_rows_d2h(dump->h1q_s, w.sa, 4, 4, N, st));
    }
    {
      GemmArgs g{w.xq, Y.qkv.q, (int)N, Y.qkv.n, H, m->ldk, Y.qkv.ld, 0};
      GemmEpilogue e{};
      e.sa = w.sa, e.sb = Y.qkv.scale, e.zc = Y.qkv.zc, e.bias = Y.bqkv, e.C = w.qkv, e.ldc = 3 * H;
      ProfScope ps("vis_gemm_qkv", vis_gemm_bytes(N, 3 * H, H, 12.0 * H), 2.0 * N * 3 * H * H, 1, st);
      IG_TRY(gemm_u8s8(g, e, kEpiF32Bias, st));
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->qkv, w.qkv, 12 * H, 12 * H, N, st));
    {
      ProfScope ps("vis_attn_f32", N * 16.0 * H, 4.0 * N * T * H, 1, st);
      IG_TRY(launch_attn_f32(w.qkv, n, T, H, m->nh, scale, V, w.ctx, st));
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->attn, w.ctx, H * 4, H * 4, N, st));
    {
      ProfScope ps("vis_quant_rows", N * (5.0 * H + 4), 0, 1, st);
      IG_TRY(launch_quant_rows(w.ctx, H, (int)N, H, w.xq, m->ldk, w.sa, st));
    }
    {
      GemmArgs g{w.xq, Y.o.q, (int)N, Y.o.n, H, m->ldk, Y.o.ld, 0};
      GemmEpilogue e{};
      e.sa = w.sa, e.sb = Y.o.scale, e.zc = Y.o.zc, e.bias = Y.bo, e.C = w.x, e.ldc = H, e.accumulate = 1;
      ProfScope ps("vis_gemm_out_residual", vis_gemm_bytes(N, H, H, 8.0 * H), 2.0 * N * H * H, 1, st);
      IG_TRY(gemm_u8s8(g, e, kEpiF32Bias, st));
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->x_attn, w.x, H * 4, H * 4, N, st));
    {
      ProfScope ps("vis_ln_quant", N * (5.0 * H + 4), 0, 1, st);
      IG_TRY(launch_ln_beta(w.x, Y.ln2g, Y.ln2b, (int)N, H, c.eps, V, nullptr, w.xq, m->ldk, w.sa, st));
    }
    if (dl) {
      IG_TRY(copy_rows_d2h(dump->h2q, w.xq, H, m->ldk, N, st));
      IG_TRY(copy_rows_d2h(dump->h2q_s, w.sa, 4, 4, N, st));
    }
    {
      GemmArgs g{w.xq, Y.fc1.q, (int)N, Y.fc1.n, H, m->ldk, Y.fc1.ld, 0};
      GemmEpilogue e{};
      e.sa = w.sa, e.sb = Y.fc1.scale, e.zc = Y.fc1.zc, e.bias = Y.b1, e.C = w.mlp, e.ldc = M;
      e.seg_rows = T, e.V = V;
      ProfScope ps("vis_gemm_fc1_gelu", vis_gemm_bytes(N, M, H, 4.0 * M), 2.0 * N * M * H, 1, st);
      IG_TRY(gemm_u8s8(g, e, kEpiGeluTanh, st));
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->mlp, w.mlp, (size_t)M * 4, (size_t)M * 4, N, st));
    {
      ProfScope ps("vis_outliers", N * 8.0 * M, 0, 3, st);
      IG_TRY(launch_outliers_select(w.mlp, n, T, M, kVisOutlierRatio, w.colmax, w.cand, w.outl, w.nout, w.outv, st));
    }
    if (dl) {
      IG_TRY(copy_rows_d2h(dump->outliers, w.outl, 32 * 4, 32 * 4, n, st));
      IG_TRY(copy_rows_d2h(dump->noutliers, w.nout, 4, 4, n, st));
    }
    {
      ProfScope ps("vis_quant_rows", N * (5.0 * M + 4), 0, 1, st);
      IG_TRY(launch_quant_rows(w.mlp, M, (int)N, M, w.xq, m->ldk, w.sa, st));
    }
    if (dl) {
      IG_TRY(copy_rows_d2h(dump->mq, w.xq, M, m->ldk, N, st));
      IG_TRY(copy_rows_d2h(dump->mq_s, w.sa, 4, 4, N, st));
    }
    {
      ProfScope ps("vis_outlier_weights", (double)n * 32 * H * 5, 0, 1, st);
      IG_TRY(launch_outliers_fixup(nullptr, n, T, H, w.outl, w.nout, w.outv, Y.fc2.q, Y.fc2.ld, Y.fc2.scale, Y.b2,
                                   w.outw, w.x, st));
    }
    {
      // fc2: the int8 product of the rest, the outlier terms, the bias, added to x.
      GemmArgs g{w.xq, Y.fc2.q, (int)N, Y.fc2.n, M, m->ldk, Y.fc2.ld, 0};
      GemmEpilogue e{};
      e.sa = w.sa, e.sb = Y.fc2.scale, e.zc = Y.fc2.zc, e.bias = Y.b2, e.C = w.x, e.ldc = H, e.accumulate = 1;
      e.seg_rows = T, e.nout = w.nout, e.outv = w.outv, e.outw = w.outw;
      ProfScope ps("vis_gemm_fc2_residual", vis_gemm_bytes(N, H, M, 8.0 * H + 16.0), 2.0 * N * H * M, 1, st);
      IG_TRY(gemm_u8s8(g, e, kEpiOutlierRes, st));
    }
    if (dl) IG_TRY(copy_rows_d2h(dump->x_mlp, w.x, H * 4, H * 4, N, st));
    if (l + 1 == layer && d_patches)
      IG_CU(cudaMemcpyAsync(d_patches, w.x, N * H * sizeof(float), cudaMemcpyDeviceToDevice, st));
  }
  if (nl < L) return 0;
  {
    ProfScope ps("vis_post_ln", N * 8.0 * H, 0, 1, st);
    IG_TRY(launch_ln_beta(w.x, m->post_g, m->post_b, (int)N, H, c.eps, V, w.x, nullptr, 0, nullptr, st));
  }
  if (layer == 0 && d_patches)
    IG_CU(cudaMemcpyAsync(d_patches, w.x, N * H * sizeof(float), cudaMemcpyDeviceToDevice, st));
  if (!pool) return 0;
  {
    F32Gemm p{};
    p.A = w.x, p.lda = H, p.W = m->kv_w, p.ldw = H, p.M = (int)N, p.N = 2 * H, p.K = H, p.bias = m->kv_b;
    p.C = w.kv, p.ldc = 2 * H, p.V = V;
    ProfScope ps("vis_head_kv", 4.0 * N * H + 8.0 * H * H + 8.0 * N * H, 4.0 * N * H * H, 1, st);
    IG_TRY(launch_f32_gemm(p, st));
  }
  {
    ProfScope ps("vis_head_attn", 8.0 * N * H, 4.0 * N * H, 1, st);
    IG_TRY(launch_pool_attn(w.kv, m->probe_q, n, T, H, m->nh, scale, V, w.att, st));
  }
  {
    ProfScope ps("vis_head_mlp", 4.0 * (2.0 * H * H + 2.0 * H * M), 2.0 * n * (H * H + 2.0 * H * M), 4, st);
    F32Gemm p{};
    p.A = w.att, p.lda = H, p.W = m->hout_w, p.ldw = H, p.M = n, p.N = H, p.K = H, p.bias = m->hout_b;
    p.C = w.hout, p.ldc = H, p.V = V;
    IG_TRY(launch_f32_gemm(p, st));
    IG_TRY(launch_ln_beta(w.hout, m->hln_g, m->hln_b, n, H, c.eps, V, w.hn, nullptr, 0, nullptr, st));
    F32Gemm f1{};
    f1.A = w.hn, f1.lda = H, f1.W = m->hfc1_w, f1.ldw = H, f1.M = n, f1.N = M, f1.K = H, f1.bias = m->hfc1_b;
    f1.gelu_seg_rows = 1, f1.V = V, f1.C = w.hm, f1.ldc = M;
    IG_TRY(launch_f32_gemm(f1, st));
    F32Gemm f2{};
    f2.A = w.hm, f2.lda = M, f2.W = m->hfc2_w, f2.ldw = M, f2.M = n, f2.N = H, f2.K = M, f2.bias = m->hfc2_b;
    f2.add = w.hout, f2.ldadd = H, f2.V = V, f2.C = w.pooled, f2.ldc = H;
    IG_TRY(launch_f32_gemm(f2, st));
  }
  return 0;
}

int vis_check_layer(const ig_vision *m, int layer) {
  if (layer < 0 || layer > m->cfg.layers)
    return fail(IG_ERR_BAD_ARG,
                "siglip: layer " + std::to_string(layer) + ", the tower has " + std::to_string(m->cfg.layers));
  return 0;
}

int vis_forward_host(ig_vision *m, const float *pixels, int n, int layer, float *patches, size_t patches_len,
                     float *pooled, size_t pooled_len, ig_vision_dump *dump) {
  t_last_error.clear();
  if (!m || n < 0 || (n > 0 && !pixels)) return fail(IG_ERR_BAD_ARG, "null argument");
  IG_TRY(vis_check_layer(m, layer));
  const size_t N = (size_t)n * m->T, H = m->H, S = m->cfg.image_size;
  if (patches && patches_len < N * H) return fail(IG_ERR_BAD_ARG, "patches too short");
  if (pooled && pooled_len < (size_t)n * H) return fail(IG_ERR_BAD_ARG, "pooled too short");
  if (n == 0) return 0;
  DeviceGuard dg(m->device);
  std::lock_guard<std::mutex> lk(m->mu);
  VisWork *w = nullptr;
  IG_TRY(vis_work(m, n, &w));
  cudaStream_t st = w->own;
  IG_CU(cudaMemcpyAsync(w->pix, pixels, (size_t)n * 3 * S * S * sizeof(float), cudaMemcpyHostToDevice, st));
  const bool pool = pooled != nullptr;
  int rc = vis_run(m, *w, w->pix, n, layer, pool, patches ? w->patches : nullptr, st, dump);
  if (!rc && patches)
    rc = cudaMemcpyAsync(patches, w->patches, N * H * sizeof(float), cudaMemcpyDeviceToHost, st) ? IG_ERR_CUDA : 0;
  if (!rc && pooled)
    rc = cudaMemcpyAsync(pooled, w->pooled, (size_t)n * H * sizeof(float), cudaMemcpyDeviceToHost, st) ? IG_ERR_CUDA
                                                                                                         : 0;
  const cudaError_t se = cudaStreamSynchronize(st);
  if (rc) return rc;
  if (se != cudaSuccess) return fail(IG_ERR_CUDA, std::string("siglip: ") + cudaGetErrorString(se));
  return 0;
}

}  // namespace
}  // namespace ig

extern "C" {

int ig_vision_create(const ig_vision_config *cfg, const ig_vision_weights *w, int32_t device, ig_vision **out) {
  using namespace ig;
  t_last_error.clear();
  if (!cfg || !w || !out) return fail(IG_ERR_BAD_ARG, "null argument");
  *out = nullptr;
  const ig_vision_config &c = *cfg;
  if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.mlp <= 0 || c.image_size <= 0 || c.patch_size <= 0)
    return fail(IG_ERR_BAD_ARG, "siglip: invalid dimensions");
  if (c.hidden % c.heads != 0 || c.image_size % c.patch_size != 0)
    return fail(IG_ERR_BAD_ARG, "siglip: inconsistent dimensions");
  const int g = c.image_size / c.patch_size, T = g * g;
  if (c.hidden / c.heads != 64) return fail(IG_ERR_UNSUPPORTED, "siglip: head dimension must be 64 in this build");
  if (T > 256) return fail(IG_ERR_UNSUPPORTED, "siglip: at most 256 patches in this build");
  if (c.simd_lanes != 8) return fail(IG_ERR_UNSUPPORTED, "siglip: simd_lanes must be 8 in this build");
  if (c.hidden % 16 || c.mlp % 16) return fail(IG_ERR_UNSUPPORTED, "siglip: hidden and mlp must be multiples of 16");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return fail(IG_ERR_NO_DEVICE, "no such CUDA device");
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10)
    return fail(IG_ERR_NO_DEVICE, "device is not sm_100");
  DeviceGuard dg(device);
  auto m = std::make_unique<ig_vision>();
  m->cfg = c;
  m->device = device;
  const int H = c.hidden, M = c.mlp, P = c.patch_size;
  m->H = H, m->M = M, m->T = T, m->nh = c.heads, m->K0 = 3 * P * P;
  m->ldk = (int)align_up(std::max(H, M), 16);
  IG_TRY(vis_upload(m.get(), &m->patch_w, w->patch_w, (size_t)H * m->K0));
  IG_TRY(vis_upload(m.get(), &m->patch_b, w->patch_b, H));
  IG_TRY(vis_upload(m.get(), &m->pos, w->pos, (size_t)T * H));
  IG_TRY(vis_upload(m.get(), &m->post_g, w->post_g, H));
  IG_TRY(vis_upload(m.get(), &m->post_b, w->post_b, H));
  if (!w->in_w || !w->in_b || !w->probe) return fail(IG_ERR_BAD_ARG, "siglip: a weight is missing");
  IG_TRY(vis_upload(m.get(), &m->kv_w, w->in_w + (size_t)H * H, (size_t)2 * H * H));
  IG_TRY(vis_upload(m.get(), &m->kv_b, w->in_b + H, (size_t)2 * H));
  IG_TRY(vis_upload(m.get(), &m->hout_w, w->hout_w, (size_t)H * H));
  IG_TRY(vis_upload(m.get(), &m->hout_b, w->hout_b, H));
  IG_TRY(vis_upload(m.get(), &m->hln_g, w->hln_g, H));
  IG_TRY(vis_upload(m.get(), &m->hln_b, w->hln_b, H));
  IG_TRY(vis_upload(m.get(), &m->hfc1_w, w->hfc1_w, (size_t)M * H));
  IG_TRY(vis_upload(m.get(), &m->hfc1_b, w->hfc1_b, M));
  IG_TRY(vis_upload(m.get(), &m->hfc2_w, w->hfc2_w, (size_t)H * M));
  IG_TRY(vis_upload(m.get(), &m->hfc2_b, w->hfc2_b, H));
  // The probe's query, once, in float32 (vision.go:62-66).
  {
    float *qw = nullptr, *qb = nullptr, *probe = nullptr;
    IG_TRY(vis_upload(m.get(), &qw, w->in_w, (size_t)H * H));
    IG_TRY(vis_upload(m.get(), &qb, w->in_b, H));
    IG_TRY(vis_upload(m.get(), &probe, w->probe, H));
    IG_TRY(vis_alloc(m->allocs, &m->probe_q, H));
    F32Gemm p{};
    p.A = probe, p.lda = H, p.W = qw, p.ldw = H, p.M = 1, p.N = H, p.K = H, p.bias = qb, p.C = m->probe_q, p.ldc = H;
    p.V = c.simd_lanes;
    IG_TRY(launch_f32_gemm(p, 0));
    IG_CU(cudaDeviceSynchronize());
  }
  float *tmp = nullptr;
  IG_CU(cudaMalloc(&tmp, (size_t)std::max(3 * H * H, M * H) * sizeof(float)));
  struct TmpFree {
    float *p;
    ~TmpFree() { cudaFree(p); }
  } tf{tmp};
  m->layers.resize(c.layers);
  for (int l = 0; l < c.layers; l++) {
    VisLayer &Y = m->layers[l];
    auto need = [&](const float *const *a) { return a && a[l]; };
    if (!need(w->ln1_g) || !need(w->ln1_b) || !need(w->ln2_g) || !need(w->ln2_b) || !need(w->wqkv) ||
        !need(w->bqkv) || !need(w->wo) || !need(w->bo) || !need(w->w1) || !need(w->b1) || !need(w->w2) ||
        !need(w->b2))
      return fail(IG_ERR_BAD_ARG, "siglip: layer " + std::to_string(l) + " weights missing");
    IG_TRY(vis_upload(m.get(), &Y.ln1g, w->ln1_g[l], H));
    IG_TRY(vis_upload(m.get(), &Y.ln1b, w->ln1_b[l], H));
    IG_TRY(vis_upload(m.get(), &Y.ln2g, w->ln2_g[l], H));
    IG_TRY(vis_upload(m.get(), &Y.ln2b, w->ln2_b[l], H));
    IG_TRY(vis_upload(m.get(), &Y.bqkv, w->bqkv[l], (size_t)3 * H));
    IG_TRY(vis_upload(m.get(), &Y.bo, w->bo[l], H));
    IG_TRY(vis_upload(m.get(), &Y.b1, w->b1[l], M));
    IG_TRY(vis_upload(m.get(), &Y.b2, w->b2[l], H));
    IG_TRY(vis_pack(m.get(), Y.qkv, w->wqkv[l], 3 * H, H, tmp));
    IG_TRY(vis_pack(m.get(), Y.o, w->wo[l], H, H, tmp));
    IG_TRY(vis_pack(m.get(), Y.fc1, w->w1[l], M, H, tmp));
    IG_TRY(vis_pack(m.get(), Y.fc2, w->w2[l], H, M, tmp));
  }
  *out = m.release();
  return 0;
}

void ig_vision_destroy(ig_vision *v) {
  if (!v) return;
  DeviceGuard dg(v->device);
  cudaDeviceSynchronize();
  delete v;
}

int ig_vision_forward(ig_vision *v, const float *pixels, int32_t n, int32_t layer, float *patches, size_t patches_len,
                      float *pooled, size_t pooled_len) {
  return ig::vis_forward_host(v, pixels, n, layer, patches, patches_len, pooled, pooled_len, nullptr);
}

int ig_vision_dump_layer(ig_vision *v, const float *pixels, int32_t n, ig_vision_dump *dump, float *pooled,
                         size_t pooled_len) {
  using namespace ig;
  if (!dump) return fail(IG_ERR_BAD_ARG, "null dump");
  if (!v || dump->layer < 0 || dump->layer >= v->cfg.layers) return fail(IG_ERR_BAD_ARG, "bad dump layer");
  return vis_forward_host(v, pixels, n, 0, nullptr, 0, pooled, pooled_len, dump);
}

int ig_vision_forward_device(ig_vision *v, const float *d_pixels, int32_t n, int32_t layer, float *d_patches,
                             float *d_pooled, void *stream) {
  using namespace ig;
  t_last_error.clear();
  if (!v || n < 0 || (n > 0 && !d_pixels)) return fail(IG_ERR_BAD_ARG, "null argument");
  IG_TRY(vis_check_layer(v, layer));
  if (n == 0) return 0;
  DeviceGuard dg(v->device);
  std::lock_guard<std::mutex> lk(v->mu);
  VisWork *w = nullptr;
  IG_TRY(vis_work(v, n, &w));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  IG_TRY(vis_run(v, *w, d_pixels, n, layer, d_pooled != nullptr, d_patches, st, nullptr));
  if (d_pooled)
    IG_CU(cudaMemcpyAsync(d_pooled, w->pooled, (size_t)n * v->H * sizeof(float), cudaMemcpyDeviceToDevice, st));
  return 0;
}

}  // extern "C"
