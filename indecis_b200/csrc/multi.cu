// A model on several GPUs of one process: the batch of sequences is sharded
// across devices with no collective.
//
// Sequences are independent in the encoder: the per-row products do not
// depend on the batch (linalg/int8_test.go:149) and attention runs per
// (sequence, head) (internal/modernbert/infer.go:490-517). So a host call on
// a multi-device model (ig_model_create_multi) cuts its sequences into
// contiguous ranges balanced by cost, encodes each range on its own GPU from
// its own host thread through that GPU's replica (the single-device path,
// unchanged), and each range writes its rows straight into its slice of the
// caller's output (the host gather). Nothing crosses between GPUs; weights are
// replicated at creation. Callers that reach the encoder through
// Model.encodeSeqs (model.go:421-426), the batcher (batch.go:24-81) or
// EncodeSeqs itself (infer.go:261) therefore use every GPU of the model with
// no change on their side.
//
// Cost of a sequence of n tokens (operations, up to a constant): the four
// products grow with n (about 12 H^2 multiply-adds per token and layer at
// I ~ 1.5 H), attention with n times the keys each query sees: n on a global
// layer, at most local_attention + 1 on a local one (Window,
// internal/modernbert/model.go:60-80).
//
// Placement: a call whose rows would give a GPU fewer than kMinShardRows is
// spread over fewer GPUs (a small shard costs its launches, not its rows),
// and the shards go to the replicas with the fewest calls in flight, so
// concurrent small calls fill different GPUs.

namespace {

constexpr int64_t kMinShardRows = 8192;

std::vector<double> seq_costs(const ig_model *m, const int64_t *offs, int nseq) {
  const ig_config &c = m->cfg;
  int n_global = 0;
  for (int l = 0; l < c.layers; l++) n_global += l % c.global_every == 0;
  const int n_local = c.layers - n_global;
  const double H = c.hidden;
  std::vector<double> cost(nseq);
  for (int s = 0; s < nseq; s++) {
    const double n = (double)(offs[s + 1] - offs[s]);
    const double gemm = 2.0 * n * 12.0 * H * H * c.layers;
    const double keys = n_global * n + n_local * std::min(n, (double)c.local_attention + 1);
    cost[s] = gemm + 4.0 * H * n * keys;
  }
  return cost;
}

// Contiguous ranges [bounds[r], bounds[r+1]), one per shard: shard r starts
// at the first sequence whose cumulative cost reaches r / shards of the total.
std::vector<int> shard_bounds(const std::vector<double> &cost, int shards) {
  const int nseq = (int)cost.size();
  std::vector<double> cum(nseq + 1, 0.0);
  for (int s = 0; s < nseq; s++) cum[s + 1] = cum[s] + cost[s];
  std::vector<int> b(1, 0);
  for (int r = 1; r < shards; r++) {
    const double t = cum[nseq] * r / shards;
    int k = (int)(std::lower_bound(cum.begin(), cum.end(), t) - cum.begin());
    b.push_back(std::min(std::max(k, b.back()), nseq));
  }
  b.push_back(nseq);
  return b;
}

int encode_group(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t nseq, int32_t mode, float *out,
                 size_t out_len, ig_dump *dump, double *logits, size_t logits_len, double *tlog, size_t tlog_len) {
  const int ndev = (int)m->replicas.size();
  int64_t nrows = 0;
  int max_len = 0;
  IG_TRY(scan_offsets(offs, nseq, &nrows, &max_len));
  if (nrows > 0 && !ids) return fail(IG_ERR_BAD_ARG, "null ids");
  // The whole batch's ids first, so the error names the batch's first bad id
  // whichever shard holds it.
  IG_TRY(check_ids(m->replicas[0], ids, nrows));
  int32_t pl = 0, tl = 0;
  IG_TRY(ig_model_head_rows(m->replicas[0], &pl, &tl));
  const size_t H = m->H;
  if (out && out_len < (mode == IG_MODE_POOLED ? (size_t)nseq * H : (size_t)nrows * H))
    return fail(IG_ERR_BAD_ARG, "output too short");
  if (logits && logits_len < (size_t)nseq * pl) return fail(IG_ERR_BAD_ARG, "logits too short");
  if (tlog && tlog_len < (size_t)nrows * tl) return fail(IG_ERR_BAD_ARG, "token logits too short");

  // Replicas by calls in flight, fewest first (ties: device order).
  std::vector<int> order(ndev);
  for (int i = 0; i < ndev; i++) order[i] = i;
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return m->replicas[a]->inflight.load() < m->replicas[b]->inflight.load(); });
  int shards = (int)std::min<int64_t>(ndev, std::max<int64_t>(1, nrows / kMinShardRows));
  if (dump || nseq < 2) shards = 1;  // a dump describes one pass
  if (shards == 1)
    return encode_host(m->replicas[order[0]], ids, offs, nseq, mode, out, out_len, dump, logits, logits_len, tlog,
                       tlog_len);

  const std::vector<int> b = shard_bounds(seq_costs(m, offs, nseq), shards);
  std::vector<int> rc(shards, 0);
  std::vector<std::string> err(shards);
  auto run = [&](int r) {
    const int s0 = b[r], s1 = b[r + 1];
    if (s1 <= s0) return;
    const int64_t t0 = offs[s0], t1 = offs[s1];
    std::vector<int64_t> lo(offs + s0, offs + s1 + 1);
    for (auto &o : lo) o -= t0;
    const int n = s1 - s0;
    float *o = nullptr;
    size_t olen = 0;
    if (out) {
      o = out + (mode == IG_MODE_POOLED ? (size_t)s0 : (size_t)t0) * H;
      olen = (mode == IG_MODE_POOLED ? (size_t)n : (size_t)(t1 - t0)) * H;
    }
    rc[r] = encode_host(m->replicas[order[r]], ids + t0, lo.data(), n, mode, o, olen, nullptr,
                        logits ? logits + (size_t)s0 * pl : nullptr, (size_t)n * pl,
                        tlog ? tlog + (size_t)t0 * tl : nullptr, (size_t)(t1 - t0) * tl);
    if (rc[r]) err[r] = t_last_error;
  };
  std::vector<std::thread> threads;
  for (int r = 1; r < shards; r++) threads.emplace_back(run, r);
  run(0);
  for (auto &t : threads) t.join();
  for (int r = 0; r < shards; r++)
    if (rc[r]) return fail(rc[r], err[r]);
  return 0;
}

// One replica per listed device, each made by create(device, &replica).
template <class Create>
int create_group(const int32_t *devices, int32_t ndevices, ig_model **out, Create create) {
  if (!devices || !out || ndevices < 1) return fail(IG_ERR_BAD_ARG, "null argument");
  if (ndevices > kMaxDevices) return fail(IG_ERR_BAD_ARG, "too many devices");
  *out = nullptr;
  for (int i = 0; i < ndevices; i++)
    for (int j = 0; j < i; j++)
      if (devices[i] == devices[j]) return fail(IG_ERR_BAD_ARG, "device " + std::to_string(devices[i]) + " listed twice");
  if (ndevices == 1) return create(devices[0], out);
  std::unique_ptr<ig_model> g(new ig_model());
  for (int i = 0; i < ndevices; i++) {
    ig_model *r = nullptr;
    if (int rc = create(devices[i], &r)) return rc;  // g's destructor frees the others
    g->replicas.push_back(r);
  }
  const ig_model *r0 = g->replicas[0];
  g->cfg = r0->cfg;
  g->device = r0->device;
  g->H = r0->H, g->I = r0->I, g->nh = r0->nh, g->D = r0->D, g->ldk = r0->ldk, g->NI = r0->NI;
  *out = g.release();
  return 0;
}

}  // namespace

extern "C" {

int ig_model_create_multi(const ig_config *cfg, const ig_weights *w, const int32_t *devices, int32_t ndevices,
                          ig_model **out) {
  t_last_error.clear();
  if (!cfg || !w) return fail(IG_ERR_BAD_ARG, "null argument");
  return create_group(devices, ndevices, out, [&](int d, ig_model **m) { return ig_model_create(cfg, w, d, m); });
}

int ig_model_create_stored_multi(const ig_config *cfg, const ig_stored_weights *w, const int32_t *devices,
                                 int32_t ndevices, ig_model **out) {
  t_last_error.clear();
  if (!cfg || !w) return fail(IG_ERR_BAD_ARG, "null argument");
  return create_group(devices, ndevices, out,
                      [&](int d, ig_model **m) { return ig_model_create_stored(cfg, w, d, m); });
}

int ig_model_replica(ig_model *m, int32_t index, ig_model **replica, int32_t *device) {
  t_last_error.clear();
  if (!m || !replica) return fail(IG_ERR_BAD_ARG, "null argument");
  const int n = m->replicas.empty() ? 1 : (int)m->replicas.size();
  if (index < 0 || index >= n) return fail(IG_ERR_BAD_ARG, "no replica " + std::to_string(index));
  *replica = m->replicas.empty() ? m : m->replicas[index];
  if (device) *device = (*replica)->device;
  return 0;
}

int ig_device_count(int32_t *n) {
  t_last_error.clear();
  if (!n) return fail(IG_ERR_BAD_ARG, "null argument");
  *n = 0;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  for (int d = 0; d < count; d++) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, d) == cudaSuccess && p.major == 10) ++*n;
  }
  return 0;
}

int ig_model_device_count(ig_model *m, int32_t *n) {
  t_last_error.clear();
  if (!m || !n) return fail(IG_ERR_BAD_ARG, "null argument");
  *n = m->replicas.empty() ? 1 : (int32_t)m->replicas.size();
  return 0;
}

}  // extern "C"
