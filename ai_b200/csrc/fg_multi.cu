// (*Model).Embed over several GPUs of one process: the caller's sequences,
// sorted by length, are cut into one contiguous slice per model (one model
// per GPU, each holding a full copy of the weights), each slice embedded by
// fg_embed_many on its own host thread, and every embedding placed in the
// caller's order. Sequences never interact (models/gemma/embed.go:160-475
// has no cross-sequence term), so the slices need no exchange and no
// collective: the "gather" is each thread writing its rows into the
// caller's host buffer.
//
// Split: the sequences sorted by length as sortIndex sorts them
// (models/gemma/model.go:412, stable, ascending), then cut where the running
// estimated cost crosses k/parts of the total. The cost of a sequence of L
// tokens is L·t(L), t the measured GPU time per token of full-length
// batches of that length; contiguous runs of the sorted order keep each
// slice's batches padded little.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "fg_internal.h"

namespace fg {
namespace {

// Time per token (ns) of full-length 131 072-token batches of
// EmbeddingGemma-300m on one B200 with the default split precision
// (split-fp16 products), by sequence length, measured with CUDA events:
// short sequences pay per-sequence attention tiles and pooling, long ones
// the quadratic global layers. Only the ratios matter for the split.
constexpr double kNsPerToken[][2] = {
    {16, 827.9},   {32, 669.3},   {64, 592.9},   {128, 557.9},  {192, 594.4},
    {256, 577.5},  {384, 602.2},  {512, 615.6},  {768, 635.4},  {1024, 651.1},
    {1280, 658.6}, {1536, 667.8}, {1792, 674.7}, {2048, 686.4}};
constexpr int kTable = int(sizeof(kNsPerToken) / sizeof(kNsPerToken[0]));

double ns_per_token(double L) {
  if (L <= kNsPerToken[0][0]) return kNsPerToken[0][1];
  for (int i = 1; i < kTable; ++i) {
    if (L <= kNsPerToken[i][0]) {
      const double x0 = kNsPerToken[i - 1][0], x1 = kNsPerToken[i][0];
      const double y0 = kNsPerToken[i - 1][1], y1 = kNsPerToken[i][1];
      return y0 + (y1 - y0) * (L - x0) / (x1 - x0);
    }
  }
  return kNsPerToken[kTable - 1][1];
}

}  // namespace

double sequence_cost(int length) {
  const double L = std::max(1, length);  // a length-0 sequence runs as one token
  return L * ns_per_token(L) / ns_per_token(512.0);
}

void plan_split(const int* len, int nseq, int parts, std::vector<int>& order, std::vector<int>& bounds) {
  order.resize(size_t(nseq));
  for (int i = 0; i < nseq; ++i) order[size_t(i)] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return len[a] < len[b]; });
  std::vector<double> cum(static_cast<size_t>(nseq));
  double acc = 0;
  for (int k = 0; k < nseq; ++k) {
    acc += sequence_cost(len[order[size_t(k)]]);
    cum[size_t(k)] = acc;
  }
  bounds.assign(size_t(parts) + 1, 0);
  for (int r = 1; r < parts; ++r) {
    // first position whose prefix cost reaches r/parts of the total
    const double target = acc * r / parts;
    int c = int(std::lower_bound(cum.begin(), cum.end(), target) - cum.begin()) + 1;
    c = std::min(std::max(c, bounds[size_t(r - 1)]), nseq);
    bounds[size_t(r)] = c;
  }
  bounds[size_t(parts)] = nseq;
}

}  // namespace fg

using namespace fg;

extern "C" {

double fg_sequence_cost(int length) { return sequence_cost(length); }

int fg_plan_split(const int32_t* lengths, int nseq, int nparts, int32_t* order, int32_t* bounds) {
  clear_error();
  if (nseq < 0 || nparts < 1) return set_error(FG_EINVAL, "fg_plan_split: bad arguments");
  if (!bounds || (nseq > 0 && (!lengths || !order))) return set_error(FG_EINVAL, "fg_plan_split: null buffer");
  std::vector<int> len(static_cast<size_t>(nseq)), ord, bnd;
  for (int i = 0; i < nseq; ++i) {
    if (lengths[i] < 0) return set_error(FG_EINVAL, "fg_plan_split: negative length");
    len[size_t(i)] = lengths[i];
  }
  plan_split(len.data(), nseq, nparts, ord, bnd);
  for (int i = 0; i < nseq; ++i) order[i] = ord[size_t(i)];
  for (int r = 0; r <= nparts; ++r) bounds[r] = bnd[size_t(r)];
  return FG_OK;
}

int fg_embed_many_multi(fg_model* const* models, int nmodels, const int32_t* ids, const int64_t* offsets,
                        int nseq, int max_tokens, int64_t batch_tokens, int dim, int precision, float* out) {
  clear_error();
  if (!models || nmodels < 1) return set_error(FG_EINVAL, "fg_embed_many_multi: no models");
  for (int r = 0; r < nmodels; ++r)
    if (!models[r]) return set_error(FG_EINVAL, "fg_embed_many_multi: model %d is null", r);
  if (nseq < 0) return set_error(FG_EINVAL, "negative sequence count");
  if (nseq == 0) return FG_OK;
  if (!offsets || !out) return set_error(FG_EINVAL, "null buffer");
  // the lengths the split sees are the truncated ones fg_embed_many embeds
  const int cap = model_max_tokens(models[0]);
  const int max_t = (max_tokens > 0 && max_tokens < cap) ? max_tokens : cap;
  if (offsets[0] < 0) return set_error(FG_EINVAL, "offsets[0] = %lld < 0", (long long)offsets[0]);
  std::vector<int> len(static_cast<size_t>(nseq));
  for (int i = 0; i < nseq; ++i) {
    const int64_t n = offsets[i + 1] - offsets[i];
    if (n < 0) return set_error(FG_EINVAL, "offsets decrease at sequence %d", i);
    len[size_t(i)] = int(std::min<int64_t>(n, max_t));
  }
  std::vector<int> order, bounds;
  plan_split(len.data(), nseq, nmodels, order, bounds);

  // Each slice's ids, packed in its sorted order, and its embeddings.
  struct Part {
    std::vector<int32_t> ids;
    std::vector<int64_t> offsets;
    std::vector<float> out;
    int n = 0;
    int rc = FG_OK;
    std::string err;
  };
  std::vector<Part> parts(static_cast<size_t>(nmodels));
  for (int r = 0; r < nmodels; ++r) {
    Part& p = parts[size_t(r)];
    p.n = bounds[size_t(r) + 1] - bounds[size_t(r)];
    if (p.n == 0) continue;
    p.offsets.reserve(size_t(p.n) + 1);
    p.offsets.push_back(0);
    for (int k = bounds[size_t(r)]; k < bounds[size_t(r) + 1]; ++k) {
      const int i = order[size_t(k)];
      const int l = len[size_t(i)];
      if (l > 0 && !ids) return set_error(FG_EINVAL, "null ids");
      p.ids.insert(p.ids.end(), ids + offsets[i], ids + offsets[i] + l);
      p.offsets.push_back(int64_t(p.ids.size()));
    }
    p.out.resize(size_t(p.n) * size_t(std::max(dim, 0)));
  }
  // One host thread per slice (the model's device is made current inside
  // fg_embed_many); the calling thread takes the first slice.
  auto run = [&](int r) {
    Part& p = parts[size_t(r)];
    if (p.n == 0) return;
    p.rc = fg_embed_many(models[r], p.ids.empty() ? nullptr : p.ids.data(), p.offsets.data(), p.n, max_t,
                         batch_tokens, dim, precision, p.out.data());
    if (p.rc != FG_OK) p.err = last_error();
  };
  std::vector<std::thread> threads;
  int spawn_rc = FG_OK;
  for (int r = 1; r < nmodels && spawn_rc == FG_OK; ++r) {
    if (parts[size_t(r)].n == 0) continue;
    try {
      threads.emplace_back(run, r);
    } catch (const std::exception& e) {
      spawn_rc = set_error(FG_ENOMEM, "fg_embed_many_multi: no host thread for model %d: %s", r, e.what());
    }
  }
  if (spawn_rc == FG_OK) run(0);
  for (std::thread& t : threads) t.join();
  if (spawn_rc != FG_OK) return spawn_rc;
  for (int r = 0; r < nmodels; ++r) {
    const Part& p = parts[size_t(r)];
    if (p.rc != FG_OK) return set_error(p.rc, "fg_embed_many_multi: model %d: %s", r, p.err.c_str());
  }
  for (int r = 0; r < nmodels; ++r) {
    const Part& p = parts[size_t(r)];
    for (int j = 0; j < p.n; ++j) {
      const int i = order[size_t(bounds[size_t(r)] + j)];
      std::memcpy(out + int64_t(i) * dim, p.out.data() + size_t(j) * dim, size_t(dim) * sizeof(float));
    }
  }
  return FG_OK;
}

}  // extern "C"
