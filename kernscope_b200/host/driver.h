// driver.h -- the correctness-gated tuning driver (the reference's
// tools/tune/include/kernscope/tune/driver.h:70-216), B200 edition.
//
// Pipeline per candidate config:
//   1. GPU-free pre-screen: the family's validate_config (sm_100a space,
//      shared-memory / TMEM budgets), then occupancy (0 resident CTAs =
//      infeasible; below min_occupancy = rejected);
//   2. resolve the prebuilt sm_100a instantiation (the role of the
//      reference's generate + compile: no per-variant compile on B200);
//   3. correctness gate on the GPU at the gate shape: the variant's output
//      against the CPU reference of the same seeded inputs (verdict metrics
//      of tests/golden/kernscope_golden/metrics.py plus the benchmark
//      tolerance); a failing variant is discarded and recorded;
//   4. benchmark at the tune shape (CUDA events, L2 flush, median/p20/p80);
//   5. select by median (ties: p20, p80, enumeration order), write a db
//      JSONL record per fresh measurement and the arch-keyed tunecache.
// Configs already in the tunecache (same min_occupancy) are replayed without
// touching the GPU.
#pragma once

#include <cstdint>
#include <functional>
#include <string>
#include <vector>

#include "db.h"

namespace kernscope::tune {

enum class DriverStatus : std::uint8_t { kOk = 0, kNoViableConfig, kNoLiveGpu, kUsageError, kInternalError };
const char *driver_status_name(DriverStatus s) noexcept;

struct DriverOptions {
  std::string kernel_family;        // matmul | bias_gelu | softmax | layernorm | reduction | flash_attention
  std::vector<std::int64_t> shape;  // matmul M,N,K; row ops R,C; reduction R,C or N; attention Nq,Nk,d or B,H,N,d
  std::string arch = "sm_100a";
  std::string grid_preset = "auto";  // "auto" | "full"
  std::string db_path;
  std::string cache_path;
  std::string workdir;
  double min_occupancy = 0.0;
  bool live_bench = true;
  bool use_cache = true;
  std::vector<std::int64_t> gate_shape;  // empty = the family default
  // B200 additions
  bool causal = false;        // flash_attention
  std::string gelu = "erf";   // bias_gelu: "erf" (the reference) | "tanh"
  int device = 0;
  double warmup_ms = 25.0;
  double rep_ms = 100.0;
  std::uint64_t seed = 0;
};

struct DriverHooks {
  // Test hook: return true to overwrite this config's gate output with
  // zeros before the verdict (an injected wrong result).
  std::function<bool(const DriverOptions &, const db::json::Value &config)> corrupt_gate_output;
};

struct DriverResult {
  DriverStatus status = DriverStatus::kInternalError;
  std::string message;
  std::string evidence_json;
  std::string cache_key;
  std::string shape_hash;
  int variants_total = 0;
  int prescreen_rejected = 0;
  int compile_failed = 0;   // launch rejected by the C ABI
  int golden_failed = 0;
  int bench_failed = 0;
  int benchmarked = 0;
  int cached = 0;
  int compiled = 0;         // variants resolved and run this session
  bool has_best = false;
  db::json::Value best_config;
  std::string best_symbol;
  double best_median_ms = 0.0, best_p20_ms = 0.0, best_p80_ms = 0.0;
  std::vector<double> measured_medians;
};

std::string make_shape_hash(const std::string &kernel_family, const std::vector<std::int64_t> &shape);
std::string make_cache_key(const std::string &arch, const std::string &kernel_family, const std::string &shape_hash);

DriverResult tune(const DriverOptions &opts, const DriverHooks *hooks = nullptr);

// Reproducer files for the winning config: repro.cpp (calls the C ABI),
// run.sh (compiles it against the library and runs it), README.md.
bool emit_repro(const DriverOptions &opts, const DriverResult &r, const std::string &dir, std::string *error);

inline constexpr const char *kToolVersion = "kernscope-b200-tune 1.0";

}  // namespace kernscope::tune
