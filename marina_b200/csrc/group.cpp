// The multi-GPU evaluator of include/marina_b200.h (mrn_group_*): one context per device, each
// holding a full weight replica, and one evaluator thread per device. Every batch is cut into
// contiguous shards, one per device, evaluated at the same time and written straight into the
// caller's output arrays at the shard's offset, so the outputs come back in input order.
// Positions are independent (the forward pass has no cross-position term), so no data moves
// between GPUs and no collective is involved.
//
// A batch larger than max_batch is a sequence of max_batch chunks, each cut the same way. The
// first chunk's shards go one to each device thread; every later shard is taken from a shared
// counter by whichever thread is free, so no thread waits for the others between chunks (a GPU
// that finishes early starts on the next chunk, and two contexts on one GPU drift apart, one
// copying or launching while the other's kernels run).
//
// The reference has no multi-GPU path (its backend is built on ordinal 0, src/net/mod.rs:171-192);
// this is the sharding wrapper around `Network` that the drop-in needs for a whole box.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <condition_variable>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/marina_b200.h"

namespace {

thread_local std::string g_group_create_error;

// A failed shard: its status, the thread (context) that ran it and its positions.
struct Failure {
  int rc = MRN_OK;
  int thread = 0, begin = 0, count = 0;
};

}  // namespace

struct mrn_group {
  std::vector<mrn_ctx*> ctx;
  std::vector<int> devices;
  std::vector<std::thread> workers;  // workers[i] serves shard i + 1; the caller's thread runs shard 0
  std::mutex call_mu;                // one mrn_group_evaluate at a time

  // The batch the workers are asked to evaluate, published under `mu` with a new generation.
  std::mutex mu;
  std::condition_variable go, done;
  unsigned generation = 0;
  int pending = 0;
  bool stop = false;
  int n = 0;
  const uint8_t* boards = nullptr;
  const int32_t* legal = nullptr;
  float* priors = nullptr;
  float* wdl = nullptr;
  int max_batch = 0;
  int pieces = 0;                  // shards of the whole call: chunks x contexts
  std::atomic<int> next_piece{0};  // the next shard to take after each thread's first
  Failure failure;                 // the first failure (under `mu`)

  std::string describe;
  std::string last_error;

  int fail(int code, const char* fmt, ...) {
    char buf[768];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    last_error = buf;
    return code;
  }

  // Positions [begin, begin + count) of shard `piece`: chunk piece / k, its (piece % k)-th
  // contiguous part (part sizes differ by at most one position).
  void piece_range(int piece, int* begin, int* count) const {
    const int k = static_cast<int>(ctx.size());
    const int chunk = piece / k, part = piece % k;
    const int c0 = chunk * max_batch, cn = (n - c0 < max_batch ? n - c0 : max_batch);
    const int q = cn / k, r = cn % k;
    *begin = c0 + part * q + (part < r ? part : r);
    *count = q + (part < r ? 1 : 0);
  }

  bool evaluate_piece(int i, int piece) {
    int begin = 0, count = 0;
    piece_range(piece, &begin, &count);
    if (count == 0) return true;
    const size_t b = static_cast<size_t>(begin);
    const int rc = mrn_evaluate(ctx[i], count, boards + b * MRN_BOARD_BYTES, legal + b * MRN_MAX_LEGAL,
                                priors + b * MRN_MAX_LEGAL, wdl + b * MRN_WDL);
    if (rc == MRN_OK) return true;
    std::lock_guard<std::mutex> lock(mu);
    if (failure.rc == MRN_OK) failure = Failure{rc, i, begin, count};
    next_piece.store(pieces);  // hand out nothing more
    return false;
  }

  // Thread i's part of a call: shard i of the first chunk, then shards from the shared counter.
  void run_shard(int i) {
    if (i < pieces && !evaluate_piece(i, i)) return;
    for (int p = next_piece.fetch_add(1); p < pieces; p = next_piece.fetch_add(1))
      if (!evaluate_piece(i, p)) return;
  }

  void worker(int i) {
    unsigned seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lock(mu);
        go.wait(lock, [&] { return stop || generation != seen; });
        if (stop) return;
        seen = generation;
      }
      run_shard(i);
      std::lock_guard<std::mutex> lock(mu);
      if (--pending == 0) done.notify_one();
    }
  }

  void shutdown() {
    {
      std::lock_guard<std::mutex> lock(mu);
      stop = true;
    }
    go.notify_all();
    for (std::thread& t : workers)
      if (t.joinable()) t.join();
    workers.clear();
    for (mrn_ctx* c : ctx) mrn_destroy(c);
    ctx.clear();
  }
};

extern "C" {

MRN_API int mrn_group_create(const mrn_arch* arch, const mrn_weights* weights, const int* devices, int n_devices,
                             int max_batch, int precision, mrn_group** out) {
  if (!out) {
    g_group_create_error = "out is NULL";
    return MRN_ERR_ARGUMENT;
  }
  *out = nullptr;
  if (!devices || n_devices < 1) {
    g_group_create_error = "a group needs at least one device";
    return MRN_ERR_ARGUMENT;
  }
  if (max_batch < 1) {
    g_group_create_error = "max_batch < 1";
    return MRN_ERR_ARGUMENT;
  }
  mrn_group* g = new mrn_group();
  // Each context holds its shard of the largest batch.
  const int per_device = (max_batch + n_devices - 1) / n_devices;
  for (int i = 0; i < n_devices; ++i) {
    mrn_ctx* c = nullptr;
    const int rc = mrn_create(arch, weights, devices[i], per_device, precision, &c);
    if (rc) {
      g_group_create_error = std::string("device ") + std::to_string(devices[i]) + ": " + mrn_last_error(nullptr);
      g->shutdown();
      delete g;
      return rc;
    }
    g->ctx.push_back(c);
    g->devices.push_back(devices[i]);
  }
  g->max_batch = max_batch;
  for (int i = 1; i < n_devices; ++i) g->workers.emplace_back(&mrn_group::worker, g, i);
  g->describe = std::string(mrn_describe(g->ctx[0])) + " x " + std::to_string(n_devices) + " devices (";
  for (int i = 0; i < n_devices; ++i) g->describe += (i ? "," : "") + std::to_string(devices[i]);
  g->describe += "), one shard per device";
  *out = g;
  return MRN_OK;
}

MRN_API int mrn_group_evaluate(mrn_group* g, int n, const uint8_t* boards, const int32_t* legal, float* priors,
                               float* wdl) {
  if (!g) {
    g_group_create_error = "group is NULL";
    return MRN_ERR_ARGUMENT;
  }
  std::lock_guard<std::mutex> call(g->call_mu);
  const int k = static_cast<int>(g->ctx.size());
  if (n < 0) return g->fail(MRN_ERR_ARGUMENT, "n = %d", n);
  if (n == 0) return MRN_OK;
  if (!boards || !legal || !priors || !wdl) return g->fail(MRN_ERR_ARGUMENT, "NULL buffer");
  const int chunks = (n + g->max_batch - 1) / g->max_batch;
  {
    std::lock_guard<std::mutex> lock(g->mu);
    g->n = n, g->boards = boards, g->legal = legal, g->priors = priors, g->wdl = wdl;
    g->pieces = chunks * k;
    g->next_piece.store(k);
    g->failure = Failure{};
    g->pending = k - 1;
    ++g->generation;
  }
  g->go.notify_all();
  g->run_shard(0);
  {
    std::unique_lock<std::mutex> lock(g->mu);
    g->done.wait(lock, [&] { return g->pending == 0; });
  }
  const Failure f = g->failure;
  if (f.rc)
    return g->fail(f.rc, "device %d, positions [%d, %d): %s", g->devices[f.thread], f.begin, f.begin + f.count,
                   mrn_last_error(g->ctx[f.thread]));
  return MRN_OK;
}

MRN_API int mrn_group_size(mrn_group* g) { return g ? static_cast<int>(g->ctx.size()) : 0; }

MRN_API mrn_ctx* mrn_group_context(mrn_group* g, int i) {
  return g && i >= 0 && i < static_cast<int>(g->ctx.size()) ? g->ctx[i] : nullptr;
}

MRN_API const char* mrn_group_describe(mrn_group* g) { return g ? g->describe.c_str() : ""; }

MRN_API const char* mrn_group_last_error(mrn_group* g) {
  return g ? g->last_error.c_str() : g_group_create_error.c_str();
}

MRN_API void mrn_group_destroy(mrn_group* g) {
  if (!g) return;
  g->shutdown();
  delete g;
}

}  // extern "C"
