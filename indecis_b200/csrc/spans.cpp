// Spans questions (spans.go): texts longer than the model are read in
// overlapping windows, every token gets the logits of the BIO tags of each
// Spans head, and the most probable consistent tag sequence gives the
// passages. Host code: the windows are planned here, framed and sent to the
// device in batches (ig_window_logits: encoder and per-token heads on the
// GPU), and the decoding runs on the host (0.25 us per token); the tags of
// many texts at once can also come from the device (spans_device.cu), the
// passages then being extracted here (ig_spans_from_tags).
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <string>
#include <vector>

#include "indecis_b200.h"

namespace ig {
int report_error(int code, const std::string &msg);
void clear_error();
}  // namespace ig

namespace {

using ig::report_error;

// ---- tags (spans.go:123-127): 0 outside, 1+2k begins a passage of type k,
// 2+2k continues it.
inline bool is_inside(int tag) { return tag > 0 && tag % 2 == 0; }
inline int tag_type(int tag) { return (tag - 1) / 2; }

// ---- UTF-8 and character classes, as Go's unicode/utf8 and unicode
// packages define them (the reference slices Go strings, i.e. bytes).

constexpr int32_t kRuneError = 0xFFFD;

// The rune at the start of s[0:n): its code point and byte length for a
// well-formed sequence (RFC 3629, Unicode Table 3-7: no overlong forms, no
// surrogates, nothing above U+10FFFF), else (U+FFFD, 1) — utf8.DecodeRune.
int32_t decode_rune(const unsigned char *s, int64_t n, int *size) {
  if (n <= 0) return *size = 0, kRuneError;
  const unsigned c = s[0];
  if (c < 0x80) return *size = 1, (int32_t)c;
  int len;
  unsigned lo = 0x80, hi = 0xBF;  // range of the second byte
  int32_t r;
  if (c >= 0xC2 && c <= 0xDF) {
    len = 2, r = c & 0x1F;
  } else if (c >= 0xE0 && c <= 0xEF) {
    len = 3, r = c & 0x0F;
    if (c == 0xE0) lo = 0xA0;
    if (c == 0xED) hi = 0x9F;
  } else if (c >= 0xF0 && c <= 0xF4) {
    len = 4, r = c & 0x07;
    if (c == 0xF0) lo = 0x90;
    if (c == 0xF4) hi = 0x8F;
  } else {
    return *size = 1, kRuneError;
  }
  if (n < len) return *size = 1, kRuneError;
  for (int i = 1; i < len; i++) {
    const unsigned b = s[i];
    const unsigned l = i == 1 ? lo : 0x80, h = i == 1 ? hi : 0xBF;
    if (b < l || b > h) return *size = 1, kRuneError;
    r = (r << 6) | (b & 0x3F);
  }
  return *size = len, r;
}

// The rune that ends s[0:n): the last rune start within the final four
// bytes, decoded, must reach the end exactly, else (U+FFFD, 1) —
// utf8.DecodeLastRune.
int32_t decode_last_rune(const unsigned char *s, int64_t n, int *size) {
  if (n <= 0) return *size = 0, kRuneError;
  int64_t start = n - 1;
  if (s[start] < 0x80) return *size = 1, (int32_t)s[start];
  const int64_t lim = std::max<int64_t>(n - 4, 0);
  for (start--; start >= lim; start--)
    if ((s[start] & 0xC0) != 0x80) break;
  if (start < 0) start = 0;
  int sz;
  const int32_t r = decode_rune(s + start, n - start, &sz);
  if (start + sz != n) return *size = 1, kRuneError;
  return *size = sz, r;
}

// unicode.IsSpace: in Latin-1 '\t' '\n' '\v' '\f' '\r' ' ' U+0085 U+00A0,
// above it the White_Space property of the Unicode character database.
bool is_space(int32_t r) {
  if (r <= 0xFF) return r == ' ' || (r >= '\t' && r <= '\r') || r == 0x85 || r == 0xA0;
  return r == 0x1680 || (r >= 0x2000 && r <= 0x200A) || r == 0x2028 || r == 0x2029 || r == 0x202F || r == 0x205F ||
         r == 0x3000;
}

// The punctuation trimPunct removes (spans.go:286-289): opening marks before
// a passage, closing marks after it.
bool is_open_punct(int32_t r) {
  switch (r) {
    case '(': case '[': case '{': case 0xAB: case 0x2039: case 0x201C: case 0x2018: case '"': case '\'':
    case 0xBF: case 0xA1:
      return true;
  }
  return false;
}

bool is_close_punct(int32_t r) {
  switch (r) {
    case ',': case ';': case ':': case '!': case '?': case ')': case ']': case '}': case 0xBB: case 0x203A:
    case 0x201D: case 0x2019: case '"': case '\'':
      return true;
  }
  return false;
}

// The opening mark of a closing bracket (pairs, spans.go:284), 0 if none.
int32_t opening_of(int32_t closing) {
  switch (closing) {
    case ')': return '(';
    case ']': return '[';
    case '}': return '{';
    case 0xBB: return 0xAB;
    case 0x203A: return 0x2039;
    case 0x201D: return 0x201C;
  }
  return 0;
}

int encode_rune(int32_t r, unsigned char *out) {
  if (r < 0x80) return out[0] = (unsigned char)r, 1;
  if (r < 0x800) return out[0] = 0xC0 | (r >> 6), out[1] = 0x80 | (r & 0x3F), 2;
  if (r < 0x10000)
    return out[0] = 0xE0 | (r >> 12), out[1] = 0x80 | ((r >> 6) & 0x3F), out[2] = 0x80 | (r & 0x3F), 3;
  out[0] = 0xF0 | (r >> 18), out[1] = 0x80 | ((r >> 12) & 0x3F), out[2] = 0x80 | ((r >> 6) & 0x3F);
  out[3] = 0x80 | (r & 0x3F);
  return 4;
}

// Non-overlapping occurrences of rune r's encoding in s[0:n) (strings.Count).
int64_t count_rune(const unsigned char *s, int64_t n, int32_t r) {
  unsigned char pat[4];
  const int len = encode_rune(r, pat);
  int64_t c = 0;
  for (int64_t i = 0; i + len <= n;) {
    if (std::memcmp(s + i, pat, len) == 0)
      c++, i += len;
    else
      i++;
  }
  return c;
}

// paired (spans.go:276-282): a closing bracket stays when the passage opened
// more of its pairs than it closed.
bool paired(const unsigned char *s, int64_t n, int32_t closing) {
  const int32_t open = opening_of(closing);
  if (!open) return false;
  return count_rune(s, n, open) > count_rune(s, n, closing);
}

// tokenCore (spans.go:131-144): a token's span without its leading spaces;
// a token made only of spaces keeps its span.
int64_t token_core_start(const unsigned char *text, int64_t s, int64_t e) {
  const int64_t s0 = s;
  while (s < e) {
    int size;
    const int32_t r = decode_rune(text + s, e - s, &size);
    if (!is_space(r)) break;
    s += size;
  }
  return s == e ? s0 : s;
}

// trimPunct (spans.go:252-272): opening punctuation and spaces off the
// front, closing punctuation (unless it closes a pair opened inside) and
// spaces off the back; a passage made only of them is kept whole.
void trim_punct(const unsigned char *text, int64_t *start, int64_t *end) {
  int64_t s = *start, e = *end;
  while (s < e) {
    int size;
    const int32_t r = decode_rune(text + s, e - s, &size);
    if (!is_open_punct(r) && !is_space(r)) break;
    s += size;
  }
  while (s < e) {
    int size;
    const int32_t r = decode_last_rune(text + s, e - s, &size);
    if (!is_space(r) && (!is_close_punct(r) || paired(text + s, e - s - size, r))) break;
    e -= size;
  }
  if (s == e) return;
  *start = s, *end = e;
}

// Go's built-in max on float64: NaN if either operand is NaN, +0 over -0.
double go_max(double a, double b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<double>::quiet_NaN();
  if (a == b) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}

void log_softmax(const double *z, int n, double temperature, double *out) {
  if (temperature <= 0) temperature = 1;
  double mx = -std::numeric_limits<double>::infinity();
  for (int i = 0; i < n; i++) mx = go_max(mx, z[i] / temperature);
  double sum = 0;
  for (int i = 0; i < n; i++) sum += std::exp(z[i] / temperature - mx);
  const double lse = mx + std::log(sum);
  for (int i = 0; i < n; i++) out[i] = z[i] / temperature - lse;
}

// The Viterbi pass of decodeSpans (spans.go:172-220): the path is chosen on
// the biased scores; an inside tag neither starts the text nor follows a
// tag of another type or the outside tag. Ties keep the lowest tag.
void viterbi(const double *logp, int n, int C, double bias, int32_t *tags) {
  auto score = [&](int t, int c) {
    const double v = logp[(size_t)t * C + c];
    return c > 0 ? v + bias : v;
  };
  auto allowed = [](int prev, int cur) { return !is_inside(cur) || (prev > 0 && tag_type(prev) == tag_type(cur)); };
  const double ninf = -std::numeric_limits<double>::infinity();
  std::vector<double> cur(C), next(C);
  std::vector<int16_t> back((size_t)n * C, 0);
  for (int c = 0; c < C; c++) cur[c] = is_inside(c) ? ninf : score(0, c);
  for (int t = 1; t < n; t++) {
    int16_t *bt = back.data() + (size_t)t * C;
    for (int c = 0; c < C; c++) {
      double best = ninf;
      int arg = 0;
      for (int p = 0; p < C; p++)
        if (allowed(p, c) && cur[p] > best) best = cur[p], arg = p;
      next[c] = best + score(t, c);
      bt[c] = (int16_t)arg;
    }
    cur.swap(next);
  }
  int last = 0;
  for (int c = 0; c < C; c++)
    if (cur[c] > cur[last]) last = c;
  tags[n - 1] = last;
  for (int t = n - 1; t > 0; t--) tags[t - 1] = back[(size_t)t * C + tags[t]];
}

// The passages of a tag sequence (decodeSpans, spans.go:222-245): each
// starts at a beginning (or a stray inside) tag, from its token's core to
// the end of the last inside tag that follows, trimmed of edge punctuation;
// its confidence is the mean of exp(logp) of its tags.
int extract(const double *logp, int32_t ntok, int32_t ntags, const int32_t *tags, const char *text, int64_t text_len,
            const int32_t *offsets, ig_span *out, int32_t cap, int32_t *nspans);

int decode(const double *logp, int32_t ntok, int32_t ntags, double bias, const char *text, int64_t text_len,
           const int32_t *offsets, int32_t *tags_out, ig_span *out, int32_t cap, int32_t *nspans) {
  if (ntok < 0 || ntags < 1 || ntags > 32767 || !nspans || text_len < 0 ||
      (ntok > 0 && (!logp || !offsets || (text_len > 0 && !text))) || (cap > 0 && !out))
    return report_error(IG_ERR_BAD_ARG, "indecis: bad span decoding arguments");
  *nspans = 0;
  if (ntok == 0) return 0;
  std::vector<int32_t> tags(ntok);
  viterbi(logp, ntok, ntags, bias, tags.data());
  if (tags_out) std::copy(tags.begin(), tags.end(), tags_out);
  return extract(logp, ntok, ntags, tags.data(), text, text_len, offsets, out, cap, nspans);
}

int extract(const double *logp, int32_t ntok, int32_t ntags, const int32_t *tags, const char *text, int64_t text_len,
            const int32_t *offsets, ig_span *out, int32_t cap, int32_t *nspans) {
  *nspans = 0;
  const unsigned char *tb = reinterpret_cast<const unsigned char *>(text);
  auto bad_offset = [&](int t) {
    return report_error(IG_ERR_BAD_ARG, "indecis: token " + std::to_string(t) + " [" + std::to_string(offsets[2 * t]) +
                                            ", " + std::to_string(offsets[2 * t + 1]) + ") out of a text of " +
                                            std::to_string(text_len) + " bytes");
  };
  std::vector<ig_span> found;
  for (int t = 0; t < ntok;) {
    if (tags[t] == 0) {
      t++;
      continue;
    }
    const int k = tag_type(tags[t]);
    const int64_t s0 = offsets[2 * t], e0 = offsets[2 * t + 1];
    if (s0 < 0 || s0 > e0 || e0 > text_len) return bad_offset(t);
    int64_t start = token_core_start(tb, s0, e0), end = e0;
    double conf = std::exp(logp[(size_t)t * ntags + tags[t]]);
    int u = t + 1;
    for (; u < ntok && is_inside(tags[u]); u++) {
      end = offsets[2 * u + 1];
      conf += std::exp(logp[(size_t)u * ntags + tags[u]]);
    }
    if (end > text_len || end < start) return bad_offset(u - 1);
    trim_punct(tb, &start, &end);
    found.push_back(ig_span{k, (int32_t)start, (int32_t)end, conf / (double)(u - t)});
    t = u;
  }
  *nspans = (int32_t)found.size();
  if ((int64_t)found.size() > cap) return report_error(IG_ERR_BAD_ARG, "indecis: span output too short");
  std::copy(found.begin(), found.end(), out);
  return 0;
}

}  // namespace

extern "C" {

int ig_plan_windows(int32_t n, int32_t size, int32_t margin, ig_window *out, int32_t cap, int32_t *count) {
  ig::clear_error();
  if (n < 0 || size < 1 || margin < 0 || !count) return report_error(IG_ERR_BAD_ARG, "indecis: bad window plan");
  if (n <= size) {
    *count = 1;
    if (!out) return 0;
    if (cap < 1) return report_error(IG_ERR_BAD_ARG, "indecis: window output too short");
    out[0] = ig_window{0, n, 0, n};
    return 0;
  }
  margin = std::min(margin, (size - 1) / 4);  // a window keeps at least half its tokens
  const int64_t k = ((int64_t)n + size - 2 * margin - 1) / (size - 2 * margin);
  *count = (int32_t)k;
  if (!out) return 0;
  if (k > cap) return report_error(IG_ERR_BAD_ARG, "indecis: window output too short");
  for (int64_t i = 0; i < k; i++) {
    const int64_t from = i * n / k, to = (i + 1) * n / k;
    out[i] = ig_window{(int32_t)std::max<int64_t>(from - margin, 0), (int32_t)std::min<int64_t>(to + margin, n),
                       (int32_t)from, (int32_t)to};
  }
  return 0;
}

int ig_log_softmax(const double *z, int32_t n, double temperature, double *out) {
  ig::clear_error();
  if (n < 0 || (n > 0 && (!z || !out))) return report_error(IG_ERR_BAD_ARG, "indecis: bad log-softmax arguments");
  log_softmax(z, n, temperature, out);
  return 0;
}

int ig_decode_spans(const double *logp, int32_t ntok, int32_t ntags, double bias, const char *text, int64_t text_len,
                    const int32_t *offsets, int32_t *tags, ig_span *out, int32_t cap, int32_t *nspans) {
  ig::clear_error();
  return decode(logp, ntok, ntags, bias, text, text_len, offsets, tags, out, cap, nspans);
}

int ig_answer_spans(const double *z, int32_t ntok, int32_t ldz, int32_t ntags, double temperature, double bias,
                    const char *text, int64_t text_len, const int32_t *offsets, ig_span *out, int32_t cap,
                    int32_t *nspans) {
  ig::clear_error();
  if (ntok < 0 || ntags < 1 || ldz < ntags || (ntok > 0 && !z))
    return report_error(IG_ERR_BAD_ARG, "indecis: bad span logits");
  std::vector<double> logp((size_t)ntok * ntags);
  for (int t = 0; t < ntok; t++) log_softmax(z + (size_t)t * ldz, ntags, temperature, logp.data() + (size_t)t * ntags);
  return decode(logp.data(), ntok, ntags, bias, text, text_len, offsets, nullptr, out, cap, nspans);
}

int ig_spans_from_tags(const double *z, int32_t ntok, int32_t ldz, int32_t ntags, double temperature,
                       const int32_t *tags, const char *text, int64_t text_len, const int32_t *offsets, ig_span *out,
                       int32_t cap, int32_t *nspans) {
  ig::clear_error();
  if (ntok < 0 || ntags < 1 || ldz < ntags || !nspans || text_len < 0 ||
      (ntok > 0 && (!z || !tags || !offsets || (text_len > 0 && !text))) || (cap > 0 && !out))
    return report_error(IG_ERR_BAD_ARG, "indecis: bad span arguments");
  *nspans = 0;
  if (ntok == 0) return 0;
  for (int t = 0; t < ntok; t++)
    if (tags[t] < 0 || tags[t] >= ntags) return report_error(IG_ERR_BAD_ARG, "indecis: tag out of range");
  std::vector<double> logp((size_t)ntok * ntags);
  for (int t = 0; t < ntok; t++) log_softmax(z + (size_t)t * ldz, ntags, temperature, logp.data() + (size_t)t * ntags);
  return extract(logp.data(), ntok, ntags, tags, text, text_len, offsets, out, cap, nspans);
}

int ig_infer_windows(ig_model *m, const int32_t *ids, const int64_t *offs, int32_t ninputs, const int32_t *prefix,
                     int32_t nprefix, const int32_t *suffix, int32_t nsuffix, int32_t max_len, int32_t batch_size,
                     double *logits, size_t logits_len, double *token_logits, size_t token_len) {
  ig::clear_error();
  if (!m || ninputs < 0 || (ninputs > 0 && !offs) || nprefix < 0 || nsuffix < 0 || (nprefix > 0 && !prefix) ||
      (nsuffix > 0 && !suffix) || max_len < 1)
    return report_error(IG_ERR_BAD_ARG, "null or negative argument");
  int32_t pl = 0, tl = 0;
  if (int rc = ig_model_head_rows(m, &pl, &tl)) return rc;
  if (ninputs == 0) return 0;
  if (offs[0] != 0) return report_error(IG_ERR_BAD_ARG, "modernbert: inconsistent batch");
  for (int i = 0; i < ninputs; i++)
    if (offs[i + 1] < offs[i]) return report_error(IG_ERR_BAD_ARG, "modernbert: inconsistent batch");
  const int64_t ntot = offs[ninputs];
  if (ntot > 0 && !ids) return report_error(IG_ERR_BAD_ARG, "null ids");
  if (logits && logits_len < (size_t)ninputs * pl) return report_error(IG_ERR_BAD_ARG, "logits too short");
  if (token_logits && token_len < (size_t)ntot * tl) return report_error(IG_ERR_BAD_ARG, "token logits too short");
  const bool want_pooled = logits && pl > 0, want_tokens = token_logits && tl > 0;
  if (!want_pooled && !want_tokens) return 0;

  // The windows of every text (windowSize, spans.go:355-359; margin a
  // sixteenth of a window, :405).
  struct Job {
    int input;
    ig_window w;
  };
  const int32_t size = std::max(max_len - nprefix - nsuffix, 1);
  std::vector<Job> jobs;
  std::vector<ig_window> ws;
  for (int i = 0; i < ninputs; i++) {
    const int64_t n = offs[i + 1] - offs[i];
    if (n > INT32_MAX) return report_error(IG_ERR_UNSUPPORTED, "text too long");
    int32_t k = 0;
    if (int rc = ig_plan_windows((int32_t)n, size, size / 16, nullptr, 0, &k)) return rc;
    ws.resize(k);
    if (int rc = ig_plan_windows((int32_t)n, size, size / 16, ws.data(), k, &k)) return rc;
    for (auto &w : ws) jobs.push_back(Job{i, w});
  }

  const size_t group = batch_size > 0 ? (size_t)batch_size : jobs.size();
  std::vector<int32_t> gids;
  std::vector<int64_t> goffs;
  std::vector<double> glog, gtok;
  for (size_t j0 = 0; j0 < jobs.size(); j0 += group) {
    const size_t j1 = std::min(jobs.size(), j0 + group);
    gids.clear();
    goffs.assign(1, 0);
    for (size_t j = j0; j < j1; j++) {
      const Job &jb = jobs[j];
      const int32_t *src = ids + offs[jb.input];
      gids.insert(gids.end(), prefix, prefix + nprefix);
      gids.insert(gids.end(), src + jb.w.start, src + jb.w.end);
      gids.insert(gids.end(), suffix, suffix + nsuffix);
      goffs.push_back((int64_t)gids.size());
    }
    const int32_t nseq = (int32_t)(j1 - j0);
    glog.assign(want_pooled ? (size_t)nseq * pl : 0, 0.0);
    gtok.assign(want_tokens ? gids.size() * tl : 0, 0.0);
    if (int rc = ig_window_logits(m, gids.data(), goffs.data(), nseq, want_pooled ? glog.data() : nullptr, glog.size(),
                                  want_tokens ? gtok.data() : nullptr, gtok.size()))
      return rc;
    for (size_t j = j0; j < j1; j++) {
      const Job &jb = jobs[j];
      const size_t g = j - j0;
      // The pooled heads read the text's first window (spans.go:432-439).
      if (want_pooled && jb.w.start == 0)
        std::copy(glog.begin() + g * pl, glog.begin() + (g + 1) * pl, logits + (size_t)jb.input * pl);
      // Each token takes its tags from the window that keeps it (:440-442).
      if (want_tokens)
        for (int32_t t = jb.w.keep_from; t < jb.w.keep_to; t++) {
          const size_t row = (size_t)goffs[g] + nprefix + t - jb.w.start;
          std::copy(gtok.begin() + row * tl, gtok.begin() + (row + 1) * tl,
                    token_logits + (size_t)(offs[jb.input] + t) * tl);
        }
    }
  }
  return 0;
}

}  // extern "C"
