// The batching front end (WithBatching, model.go:137-160; batcher,
// batch.go:7-81): requests of concurrent callers are coalesced into device
// batches. A worker takes the first pending request, then without waiting
// those already queued while the batch holds fewer than max_rows positions,
// encodes them in one pass (sequences end to end, no padding) and hands
// each caller its rows. On the GPU a batch costs little more than its
// largest part, so the workers of every device (one ig_model per GPU) take
// from one queue, and max_wait_us > 0 lets a worker wait that long for more
// requests while its batch is short.
//
// Differences from the reference, on purpose: a request whose ids fail is
// answered alone (after a failed batch each of its requests is encoded
// separately), so an out-of-vocabulary id in one request does not fail the
// requests that happened to share its batch; the reference's outcome there
// depends on timing.
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "indecis_b200.h"

namespace ig {
int report_error(int code, const std::string &msg);
void clear_error();
}  // namespace ig

namespace {

struct Request {
  const int32_t *ids;
  const int64_t *offs;
  int32_t nseq;
  int64_t rows;
  float *out;
  int rc = 0;
  std::string err;
  bool done = false;
};

}  // namespace

struct ig_batcher {
  ig_batch_encode_fn fn = nullptr;
  std::vector<void *> users;  // one per device (model)
  int32_t hidden = 0, max_rows = 512, max_wait_us = 0;
  std::mutex mu;
  std::condition_variable cv_work, cv_done;
  std::deque<Request *> queue;
  bool stop = false;
  std::vector<std::thread> workers;
  std::atomic<int64_t> n_requests{0}, n_batches{0}, n_rows{0};
};

namespace {

// Encodes the requests of one batch on `user`'s device and answers them.
void encode_batch(ig_batcher *b, void *user, const std::vector<Request *> &batch) {
  std::vector<int32_t> ids;
  std::vector<int64_t> offs(1, 0);
  int64_t nseq = 0;
  for (Request *r : batch) {
    for (int32_t s = 0; s < r->nseq; s++) offs.push_back(offs.back() + (r->offs[s + 1] - r->offs[s]));
    ids.insert(ids.end(), r->ids, r->ids + r->offs[r->nseq]);
    nseq += r->nseq;
  }
  std::vector<float> out((size_t)nseq * b->hidden);
  int rc = b->fn(user, ids.data(), offs.data(), (int32_t)nseq, out.data());
  b->n_batches++;
  b->n_rows += offs.back();
  if (rc == 0) {
    size_t o = 0;
    for (Request *r : batch) {
      std::memcpy(r->out, out.data() + o, sizeof(float) * r->nseq * b->hidden);
      o += (size_t)r->nseq * b->hidden;
      r->rc = 0;
    }
  } else if (batch.size() == 1) {
    batch[0]->rc = rc;
    batch[0]->err = ig_last_error();
  } else {
    // One request failed the batch: answer each alone.
    for (Request *r : batch) {
      r->rc = b->fn(user, r->ids, r->offs, r->nseq, r->out);
      if (r->rc) r->err = ig_last_error();
      b->n_batches++;
    }
  }
  {
    std::lock_guard<std::mutex> lk(b->mu);
    for (Request *r : batch) r->done = true;
  }
  b->cv_done.notify_all();
}

void worker(ig_batcher *b, void *user) {
  std::vector<Request *> batch;
  for (;;) {
    batch.clear();
    {
      std::unique_lock<std::mutex> lk(b->mu);
      b->cv_work.wait(lk, [&] { return b->stop || !b->queue.empty(); });
      if (b->queue.empty()) return;  // stopping, nothing left
      batch.push_back(b->queue.front());
      b->queue.pop_front();
      int64_t rows = batch[0]->rows;
      const auto deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(b->max_wait_us);
      for (;;) {
        while (rows < b->max_rows && !b->queue.empty()) {
          rows += b->queue.front()->rows;
          batch.push_back(b->queue.front());
          b->queue.pop_front();
        }
        if (rows >= b->max_rows || b->max_wait_us <= 0 || b->stop) break;
        if (b->cv_work.wait_until(lk, deadline, [&] { return b->stop || !b->queue.empty(); })) continue;
        break;  // the wait ran out
      }
    }
    encode_batch(b, user, batch);
  }
}

}  // namespace

extern "C" {

int ig_batcher_create_fn(ig_batch_encode_fn fn, void *const *users, int32_t nusers, int32_t hidden,
                         int32_t workers_per_user, int32_t max_rows, int32_t max_wait_us, ig_batcher **out) {
  ig::clear_error();
  if (!fn || !users || nusers < 1 || hidden < 1 || !out || max_wait_us < 0)
    return ig::report_error(IG_ERR_BAD_ARG, "indecis: bad batcher arguments");
  auto *b = new ig_batcher();
  b->fn = fn;
  b->users.assign(users, users + nusers);
  b->hidden = hidden;
  b->max_rows = max_rows > 0 ? max_rows : 512;  // WithBatching's default
  b->max_wait_us = max_wait_us;
  const int per = workers_per_user > 0 ? workers_per_user : 2;
  for (void *u : b->users)
    for (int i = 0; i < per; i++) b->workers.emplace_back(worker, b, u);
  *out = b;
  return 0;
}

static int model_encode(void *user, const int32_t *ids, const int64_t *offs, int32_t nseq, float *out) {
  ig_model *m = static_cast<ig_model *>(user);
  int32_t vocab = 0, hidden = 0;
  ig_model_dims(m, &vocab, &hidden);
  return ig_encode(m, ids, offs, nseq, IG_MODE_POOLED, out, (size_t)nseq * hidden);
}

int ig_batcher_create(ig_model *const *models, int32_t nmodels, int32_t workers_per_model, int32_t max_rows,
                      int32_t max_wait_us, ig_batcher **out) {
  ig::clear_error();
  if (!models || nmodels < 1) return ig::report_error(IG_ERR_BAD_ARG, "indecis: no model");
  int32_t vocab = 0, hidden = 0;
  for (int i = 0; i < nmodels; i++) {
    int32_t v = 0, h = 0;
    if (int rc = ig_model_dims(models[i], &v, &h)) return rc;
    if (i && (v != vocab || h != hidden)) return ig::report_error(IG_ERR_BAD_ARG, "indecis: models differ");
    vocab = v, hidden = h;
  }
  std::vector<void *> users(models, models + nmodels);
  return ig_batcher_create_fn(model_encode, users.data(), nmodels, hidden, workers_per_model, max_rows, max_wait_us,
                              out);
}

void ig_batcher_destroy(ig_batcher *b) {
  if (!b) return;
  {
    std::lock_guard<std::mutex> lk(b->mu);
    b->stop = true;
  }
  b->cv_work.notify_all();
  for (auto &t : b->workers) t.join();
  delete b;
}

int ig_batcher_encode(ig_batcher *b, const int32_t *ids, const int64_t *offs, int32_t nseq, float *pooled,
                      size_t pooled_len) {
  ig::clear_error();
  if (!b || nseq < 0 || (nseq > 0 && (!offs || !pooled))) return ig::report_error(IG_ERR_BAD_ARG, "null argument");
  if (nseq == 0) return 0;
  if (pooled_len < (size_t)nseq * b->hidden) return ig::report_error(IG_ERR_BAD_ARG, "output too short");
  if (offs[0] != 0) return ig::report_error(IG_ERR_BAD_ARG, "modernbert: inconsistent batch");
  for (int32_t s = 0; s < nseq; s++)
    if (offs[s + 1] < offs[s]) return ig::report_error(IG_ERR_BAD_ARG, "modernbert: inconsistent batch");
  if (offs[nseq] > 0 && !ids) return ig::report_error(IG_ERR_BAD_ARG, "null ids");
  Request r{ids, offs, nseq, offs[nseq], pooled};
  {
    std::lock_guard<std::mutex> lk(b->mu);
    if (b->stop) return ig::report_error(IG_ERR_BAD_ARG, "indecis: batcher closed");
    b->queue.push_back(&r);
  }
  b->n_requests++;
  b->cv_work.notify_one();
  {
    std::unique_lock<std::mutex> lk(b->mu);
    b->cv_done.wait(lk, [&] { return r.done; });
  }
  if (r.rc) return ig::report_error(r.rc, r.err);
  return 0;
}

int ig_batcher_stats(ig_batcher *b, int64_t *requests, int64_t *batches, int64_t *rows) {
  if (!b) return IG_ERR_BAD_ARG;
  if (requests) *requests = b->n_requests.load();
  if (batches) *batches = b->n_batches.load();
  if (rows) *rows = b->n_rows.load();
  return 0;
}

}  // extern "C"
