// bench.h -- kernel timing with CUDA events through the C ABI (the
// reference's libs/bench, libs/bench/include/kernscope/bench.h:49-119):
//   * L2 flush buffer sized from the device's L2 (ks_gpu_l2_bytes), written
//     with ks_gpu_memset before every timed launch (outside the events);
//   * one warm launch, then `calibration_runs` flushed launches whose minimum
//     is the per-launch estimate;
//   * n_warmup = ceil(warmup_ms / est), n_repeat = ceil(rep_ms / est);
//   * timed launches, each bracketed by its own events, until the relative
//     standard deviation is <= max_noise with >= min_samples samples and
//     >= min_time_ms timed, or timeout_ms of wall clock passed;
//   * summary: median, p20, p80, mean, min (ms).
// A failing launch or event op stops the run with the failing op named in
// error_message (no hang: every wait is a bounded event synchronize).
#pragma once

#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace kernscope::bench {

struct Options {
  double warmup_ms = 25.0;
  double rep_ms = 100.0;
  int min_samples = 10;
  double min_time_ms = 50.0;
  double max_noise = 0.05;
  double timeout_ms = 3000.0;
  bool l2_flush = true;
  std::uint64_t l2_flush_bytes = 0;  // 0 = 2 x device L2 (256 MiB if unknown)
  int calibration_runs = 5;
  int max_samples = 10000;
};

struct Result {
  double median_ms = 0.0;
  double p20_ms = 0.0;
  double p80_ms = 0.0;
  double mean_ms = 0.0;
  double min_ms = 0.0;
  double relative_stdev = 0.0;
  int n_reps = 0;
  int n_warmup = 0;
  std::uint64_t l2_flush_bytes_used = 0;
  int error = 0;  // ks_status of the failing operation, 0 = ok
  std::string error_message;
  bool converged = false;
  bool timed_out = false;
};

// A launch on `stream` (void* cudaStream_t); returns a ks_status.
using LaunchFn = std::function<int(void *stream)>;

double quantile(std::vector<double> samples, double q);
double median(std::vector<double> samples);

Result run(const LaunchFn &launch, const Options &opts = {}, void *stream = nullptr);

// Multi-GPU: the job's time is the slowest rank's; merges per-rank results
// by taking, for each statistic, the maximum over ranks.
Result max_over_ranks(const std::vector<Result> &per_rank);

}  // namespace kernscope::bench
