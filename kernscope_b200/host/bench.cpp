// bench.cpp -- CUDA-event timing loop over the C ABI runtime.
#include "bench.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <numeric>

#include "kernscope_b200.h"

namespace kernscope::bench {

double quantile(std::vector<double> s, double q) {
  if (s.empty()) return 0.0;
  std::sort(s.begin(), s.end());
  const double pos = q * double(s.size() - 1);
  const std::size_t lo = std::size_t(std::floor(pos));
  const std::size_t hi = std::min(lo + 1, s.size() - 1);
  const double f = pos - double(lo);
  return s[lo] * (1.0 - f) + s[hi] * f;
}

double median(std::vector<double> s) { return quantile(std::move(s), 0.5); }

namespace {
struct Events {
  void *a = nullptr, *b = nullptr;
  ~Events() {
    if (a) ks_gpu_event_destroy(a);
    if (b) ks_gpu_event_destroy(b);
  }
};

double rel_stdev(const std::vector<double> &s) {
  if (s.size() < 2) return 0.0;
  const double mean = std::accumulate(s.begin(), s.end(), 0.0) / double(s.size());
  double v = 0.0;
  for (double x : s) v += (x - mean) * (x - mean);
  v /= double(s.size() - 1);
  return mean > 0.0 ? std::sqrt(v) / mean : 0.0;
}
}  // namespace

Result run(const LaunchFn &launch, const Options &o, void *stream) {
  Result r;
  Events ev;
  auto fail = [&](int st, const char *what) {
    r.error = st;
    r.error_message = std::string(what) + " failed: " + ks_status_string(st);
    return r;
  };
  int st = ks_gpu_event_create(&ev.a);
  if (st == KS_OK) st = ks_gpu_event_create(&ev.b);
  if (st != KS_OK) return fail(st, "event create");

  // L2 flush buffer
  void *flush = nullptr;
  std::uint64_t flush_bytes = 0;
  if (o.l2_flush) {
    flush_bytes = o.l2_flush_bytes;
    if (flush_bytes == 0) {
      int dev = 0;
      size_t l2 = 0;
      ks_gpu_get_device(&dev);
      flush_bytes = (ks_gpu_l2_bytes(dev, &l2) == KS_OK && l2 > 0) ? 2 * l2 : (256ull << 20);
    }
    if ((st = ks_gpu_malloc(&flush, flush_bytes)) != KS_OK) return fail(st, "l2 flush malloc");
  }
  r.l2_flush_bytes_used = flush_bytes;
  struct FlushFree {
    void *p;
    ~FlushFree() {
      if (p) ks_gpu_free(p);
    }
  } ff{flush};

  auto timed_once = [&](double *ms) -> int {
    int s = KS_OK;
    if (flush) s = ks_gpu_memset(flush, 0, flush_bytes, stream);
    if (s == KS_OK) s = ks_gpu_event_record(ev.a, stream);
    if (s == KS_OK) s = launch(stream);
    if (s == KS_OK) s = ks_gpu_event_record(ev.b, stream);
    if (s == KS_OK) s = ks_gpu_event_synchronize(ev.b);
    float f = 0.f;
    if (s == KS_OK) s = ks_gpu_event_elapsed_ms(ev.a, ev.b, &f);
    *ms = f;
    return s;
  };

  // warm launch + calibration
  if ((st = launch(stream)) != KS_OK) return fail(st, "warm launch");
  if ((st = ks_gpu_stream_synchronize(stream)) != KS_OK) return fail(st, "warm launch sync");
  double est = 1e30;
  for (int i = 0; i < std::max(1, o.calibration_runs); ++i) {
    double ms = 0;
    if ((st = timed_once(&ms)) != KS_OK) return fail(st, "calibration launch");
    est = std::min(est, ms);
  }
  est = std::max(est, 1e-4);
  r.n_warmup = int(std::ceil(o.warmup_ms / est));
  const int n_repeat = std::max(1, int(std::ceil(o.rep_ms / est)));
  for (int i = 0; i < r.n_warmup; ++i)
    if ((st = launch(stream)) != KS_OK) return fail(st, "warmup launch");
  if ((st = ks_gpu_stream_synchronize(stream)) != KS_OK) return fail(st, "warmup sync");

  std::vector<double> samples;
  samples.reserve(std::min(n_repeat * 2, o.max_samples));
  const auto t0 = std::chrono::steady_clock::now();
  double timed = 0.0;
  while (true) {
    for (int i = 0; i < n_repeat && int(samples.size()) < o.max_samples; ++i) {
      double ms = 0;
      if ((st = timed_once(&ms)) != KS_OK) return fail(st, "timed launch");
      samples.push_back(ms);
      timed += ms;
    }
    const double wall =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    r.relative_stdev = rel_stdev(samples);
    r.converged = r.relative_stdev <= o.max_noise;
    if (int(samples.size()) >= o.min_samples && timed >= o.min_time_ms && r.converged) break;
    if (wall >= o.timeout_ms) {
      r.timed_out = true;
      break;
    }
    if (int(samples.size()) >= o.max_samples) break;
  }
  r.n_reps = int(samples.size());
  r.median_ms = quantile(samples, 0.5);
  r.p20_ms = quantile(samples, 0.2);
  r.p80_ms = quantile(samples, 0.8);
  r.mean_ms = std::accumulate(samples.begin(), samples.end(), 0.0) / double(samples.size());
  r.min_ms = *std::min_element(samples.begin(), samples.end());
  return r;
}

Result max_over_ranks(const std::vector<Result> &rs) {
  Result out;
  if (rs.empty()) return out;
  out = rs[0];
  for (const Result &r : rs) {
    out.median_ms = std::max(out.median_ms, r.median_ms);
    out.p20_ms = std::max(out.p20_ms, r.p20_ms);
    out.p80_ms = std::max(out.p80_ms, r.p80_ms);
    out.mean_ms = std::max(out.mean_ms, r.mean_ms);
    out.min_ms = std::max(out.min_ms, r.min_ms);
    out.relative_stdev = std::max(out.relative_stdev, r.relative_stdev);
    out.converged = out.converged && r.converged;
    out.timed_out = out.timed_out || r.timed_out;
    if (r.error != 0 && out.error == 0) {
      out.error = r.error;
      out.error_message = r.error_message;
    }
  }
  return out;
}

}  // namespace kernscope::bench
