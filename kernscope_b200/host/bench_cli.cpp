// bench_cli.cpp -- kernscope-bench: the roofline peaks of this B200, measured.
//
// Counterpart of the reference's tools/bench/main.cpp (peak-bw, peak-flops,
// peak-lds with the kernscope::bench methodology, results written as libs/db
// JSONL records with provenance).  Here:
//
//   kernscope-bench <peak-bw|peak-flops|peak-smem|all> [--device <n>]
//                   [--sizes <MiB,...>] [--no-flush] [--db <path>] [--json]
//                   [--version]
//
//   peak-bw     HBM: device-to-device copy (2 x bytes) and read-only sweep
//               over each size; the peak is the best over sizes of at least
//               twice the L2 (HBM-resident traffic only)
//   peak-flops  bf16 tcgen05 MMA peak (TFLOP/s, dense) and fp32 FFMA peak
//   peak-smem   shared-memory load bandwidth (GB/s, whole GPU)
//
// Timing is bench::run (CUDA events, L2 flush for the bandwidth probes,
// warm-up and repetition budgets, median / p20 / p80).  Clocks are read with
// nvidia-smi after the measurements and recorded as measured: this tool
// never sets clocks or any other GPU setting.
//
// Exit codes: 0 = measured and every sanity floor passed; 1 = measured but a
// floor failed (HBM < 3000 GB/s, bf16 < 500 TFLOP/s, fp32 < 20 TFLOP/s,
// shared memory < 10000 GB/s); 2 = usage or environment error (no device,
// not sm_100).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "bench.h"
#include "db.h"
#include "json.h"
#include "kernscope_b200.h"

namespace {

using kernscope::db::json::Value;
constexpr const char *kToolVersion = "kernscope-bench 0.1.0";

struct Args {
  std::string command;
  int device = 0;
  std::vector<long long> sizes_mib = {64, 256, 1024, 4096};
  bool flush = true;
  std::string db = "reports/peaks/sm_100a-bench.jsonl";
  bool json = false;
};

struct Measurement {
  std::string family;  // peak_bw_d2d | peak_bw_read | peak_flops_bf16 | peak_flops_fp32 | peak_smem
  std::string label;
  std::string unit;
  double work = 0.0;   // bytes or FLOPs per launch
  std::string shape;   // "size=<bytes>" or "iters=<n>"
  kernscope::bench::Result r;
  double value = 0.0;  // GB/s or TFLOP/s at the median
  bool hbm_resident = true;
};

struct Clocks {
  std::string name, sm_mhz, mem_mhz, sm_max_mhz, power_w, reasons;
};

int usage(const char *msg) {
  if (msg) std::fprintf(stderr, "kernscope-bench: %s\n", msg);
  std::fprintf(stderr,
               "usage: kernscope-bench <peak-bw|peak-flops|peak-smem|all> [--device <n>] [--sizes <MiB,...>]\n"
               "                       [--no-flush] [--db <path>] [--json] [--version]\n"
               "  clocks are recorded as measured (nvidia-smi), never set\n");
  return 2;
}

bool parse(int argc, char **argv, Args *a, int *rc) {
  for (int i = 1; i < argc; ++i) {
    const std::string s = argv[i];
    auto next = [&](const char *what) -> const char * {
      if (i + 1 >= argc) {
        *rc = usage((std::string("missing value for ") + what).c_str());
        return nullptr;
      }
      return argv[++i];
    };
    if (s == "--version") {
      std::printf("%s (ABI %d, %s)\n", kToolVersion, ks_abi_version(), ks_build_info());
      *rc = 0;
      return false;
    } else if (s == "--device") {
      const char *v = next("--device");
      if (!v) return false;
      a->device = std::atoi(v);
    } else if (s == "--sizes") {
      const char *v = next("--sizes");
      if (!v) return false;
      a->sizes_mib.clear();
      for (const char *p = v; *p;) {
        char *end = nullptr;
        const long long x = std::strtoll(p, &end, 10);
        if (end == p || x <= 0) {
          *rc = usage("--sizes takes positive MiB values separated by commas");
          return false;
        }
        a->sizes_mib.push_back(x);
        p = *end == ',' ? end + 1 : end;
      }
    } else if (s == "--no-flush") {
      a->flush = false;
    } else if (s == "--db") {
      const char *v = next("--db");
      if (!v) return false;
      a->db = v;
    } else if (s == "--json") {
      a->json = true;
    } else if (!s.empty() && s[0] != '-' && a->command.empty()) {
      a->command = s;
    } else {
      *rc = usage(("unknown argument " + s).c_str());
      return false;
    }
  }
  if (a->command != "peak-bw" && a->command != "peak-flops" && a->command != "peak-smem" && a->command != "all") {
    *rc = usage("a command is required: peak-bw, peak-flops, peak-smem or all");
    return false;
  }
  return true;
}

std::string trim(std::string s) {
  while (!s.empty() && (s.back() == '\n' || s.back() == ' ' || s.back() == '\r')) s.pop_back();
  while (!s.empty() && s.front() == ' ') s.erase(s.begin());
  return s;
}

// One nvidia-smi query (read only).
Clocks read_clocks(int device) {
  Clocks c;
  const std::string cmd = "nvidia-smi -i " + std::to_string(device) +
                          " --query-gpu=name,clocks.sm,clocks.mem,clocks.max.sm,power.draw,"
                          "clocks_event_reasons.active --format=csv,noheader,nounits 2>/dev/null";
  struct Closer {
    void operator()(FILE *f) const { pclose(f); }
  };
  std::unique_ptr<FILE, Closer> p(popen(cmd.c_str(), "r"));
  if (!p) return c;
  char line[512] = {0};
  if (!std::fgets(line, sizeof(line), p.get())) return c;
  std::vector<std::string> f;
  std::string cur;
  for (const char *q = line; *q; ++q) {
    if (*q == ',') {
      f.push_back(trim(cur));
      cur.clear();
    } else {
      cur.push_back(*q);
    }
  }
  f.push_back(trim(cur));
  if (f.size() >= 6) c = Clocks{f[0], f[1], f[2], f[3], f[4], f[5]};
  return c;
}

struct DevBuf {
  void *p = nullptr;
  ~DevBuf() {
    if (p) ks_gpu_free(p);
  }
  int alloc(size_t n) { return ks_gpu_malloc(&p, n); }
};

int measure_bw(const Args &a, size_t l2, void *sink, std::vector<Measurement> *out) {
  for (long long mib : a.sizes_mib) {
    const size_t bytes = size_t(mib) << 20;
    DevBuf src, dst;
    int s = src.alloc(bytes);
    if (s == KS_OK) s = dst.alloc(bytes);
    if (s == KS_OK) s = ks_gpu_memset(src.p, 0x5a, bytes, nullptr);
    if (s == KS_OK) s = ks_gpu_synchronize();
    if (s != KS_OK) {
      std::fprintf(stderr, "kernscope-bench: %lld MiB buffers: %s\n", mib, ks_status_string(s));
      return s;
    }
    kernscope::bench::Options o;
    o.l2_flush = a.flush;
    for (int which = 0; which < 2; ++which) {
      Measurement m;
      m.family = which == 0 ? "peak_bw_d2d" : "peak_bw_read";
      m.label = std::string(which == 0 ? "D2D copy " : "read sweep ") + std::to_string(mib) + " MiB";
      m.unit = "GB/s";
      m.work = double(bytes) * (which == 0 ? 2.0 : 1.0);
      m.shape = "size=" + std::to_string(bytes);
      m.hbm_resident = bytes >= 2 * l2;
      m.r = kernscope::bench::run(
          [&](void *st) {
            return which == 0 ? ks_peak_copy(dst.p, src.p, bytes, st) : ks_peak_read(src.p, bytes, sink, st);
          },
          o);
      if (m.r.error != 0) {
        std::fprintf(stderr, "kernscope-bench: %s: %s\n", m.label.c_str(), m.r.error_message.c_str());
        return m.r.error;
      }
      m.value = m.work / (m.r.median_ms * 1e-3) / 1e9;
      out->push_back(m);
    }
  }
  return KS_OK;
}

// Iterations for a launch of about `target_ms`, from one timed launch.
long long calibrate(int (*probe)(long long, void *, double *, void *), void *sink, double target_ms) {
  void *e0 = nullptr, *e1 = nullptr;
  if (ks_gpu_event_create(&e0) != KS_OK || ks_gpu_event_create(&e1) != KS_OK) return 0;
  long long iters = 256;
  double dummy = 0;
  float ms = 0.f;
  for (int round = 0; round < 4; ++round) {
    ks_gpu_event_record(e0, nullptr);
    if (probe(iters, sink, &dummy, nullptr) != KS_OK) break;
    ks_gpu_event_record(e1, nullptr);
    ks_gpu_event_synchronize(e1);
    ks_gpu_event_elapsed_ms(e0, e1, &ms);
    if (ms >= 0.5f * float(target_ms)) break;
    iters *= 4;
  }
  ks_gpu_event_destroy(e0);
  ks_gpu_event_destroy(e1);
  if (ms <= 0.f) return 0;
  return std::max<long long>(1, (long long)(double(iters) * target_ms / ms));
}

int measure_compute(void *sink, const char *family, const char *label, const char *unit,
                    int (*probe)(long long, void *, double *, void *), std::vector<Measurement> *out) {
  const long long iters = calibrate(probe, sink, 2.0);
  if (iters <= 0) {
    std::fprintf(stderr, "kernscope-bench: %s: calibration launch failed\n", label);
    return KS_ERR_LAUNCH;
  }
  Measurement m;
  m.family = family;
  m.label = label;
  m.unit = unit;
  m.shape = "iters=" + std::to_string(iters);
  if (int s = probe(iters, sink, &m.work, nullptr); s != KS_OK) return s;
  kernscope::bench::Options o;
  o.l2_flush = false;  // no memory traffic to speak of
  double w = 0;
  m.r = kernscope::bench::run([&](void *st) { return probe(iters, sink, &w, st); }, o);
  if (m.r.error != 0) {
    std::fprintf(stderr, "kernscope-bench: %s: %s\n", label, m.r.error_message.c_str());
    return m.r.error;
  }
  const double per_s = m.work / (m.r.median_ms * 1e-3);
  m.value = std::string(unit) == "GB/s" ? per_s / 1e9 : per_s / 1e12;
  out->push_back(m);
  return KS_OK;
}

}  // namespace

static int run_main(int argc, char **argv) {
  Args a;
  int rc = 0;
  if (!parse(argc, argv, &a, &rc)) return rc;
  int n = 0;
  char arch[32] = {0};
  if (ks_gpu_device_count(&n) != KS_OK || n <= a.device) return usage("no CUDA device (kernscope-bench measures a live B200)");
  if (ks_gpu_set_device(a.device) != KS_OK || ks_gpu_arch(a.device, arch, sizeof(arch)) != KS_OK)
    return usage("cannot select the device");
  if (std::string(arch) != "sm_100a") return usage((std::string("device is ") + arch + ", not sm_100a").c_str());
  size_t l2 = 0, sink_words = 0;
  ks_gpu_l2_bytes(a.device, &l2);
  if (ks_peak_sink_words(&sink_words) != KS_OK) return usage("ks_peak_sink_words failed");
  DevBuf sink;
  if (sink.alloc(sink_words * 4) != KS_OK) return usage("cannot allocate the sink buffer");

  std::vector<Measurement> ms;
  int s = KS_OK;
  const bool all = a.command == "all";
  if (s == KS_OK && (all || a.command == "peak-bw")) s = measure_bw(a, l2, sink.p, &ms);
  if (s == KS_OK && (all || a.command == "peak-flops")) {
    s = measure_compute(sink.p, "peak_flops_bf16", "tcgen05 bf16 MMA 128x256x16", "TFLOP/s", ks_peak_mma_bf16, &ms);
    if (s == KS_OK)
      s = measure_compute(sink.p, "peak_flops_fp32", "fp32 FFMA chains", "TFLOP/s", ks_peak_ffma_f32, &ms);
  }
  if (s == KS_OK && (all || a.command == "peak-smem"))
    s = measure_compute(sink.p, "peak_smem", "shared-memory 16-byte loads", "GB/s", ks_peak_smem, &ms);
  if (s != KS_OK) {
    std::fprintf(stderr, "kernscope-bench: measurement failed: %s\n", ks_status_string(s));
    return 2;
  }
  const Clocks clk = read_clocks(a.device);

  // peaks and sanity floors
  double hbm = 0, bf16 = 0, fp32 = 0, smem = 0;
  for (const Measurement &m : ms) {
    if ((m.family == "peak_bw_d2d" || m.family == "peak_bw_read") && m.hbm_resident) hbm = std::max(hbm, m.value);
    if (m.family == "peak_flops_bf16") bf16 = m.value;
    if (m.family == "peak_flops_fp32") fp32 = m.value;
    if (m.family == "peak_smem") smem = m.value;
  }
  bool floors_ok = true;
  if ((all || a.command == "peak-bw") && hbm < 3000.0) floors_ok = false;
  if ((all || a.command == "peak-flops") && (bf16 < 500.0 || fp32 < 20.0)) floors_ok = false;
  if ((all || a.command == "peak-smem") && smem < 10000.0) floors_ok = false;

  // db records with provenance (merged into an existing db)
  kernscope::db::Database db;
  std::vector<kernscope::db::LoadWarning> warnings;
  db.load(a.db, warnings);
  const std::string ts = kernscope::db::utc_timestamp();
  for (const Measurement &m : ms) {
    kernscope::db::Record rec;
    rec.gpu_arch = "sm_100a";
    rec.kernel_family = m.family;
    rec.shape_hash = m.shape;
    rec.config = kernscope::db::json::object({{"label", Value(m.label)},
                                              {"work", Value(m.work)},
                                              {"value", Value(m.value)},
                                              {"unit", Value(m.unit)},
                                              {"hbm_resident", Value(m.hbm_resident)},
                                              {"device_name", Value(clk.name)},
                                              {"arch", Value("sm_100a")},
                                              {"sm_mhz", Value(clk.sm_mhz)},
                                              {"mem_mhz", Value(clk.mem_mhz)},
                                              {"sm_max_mhz", Value(clk.sm_max_mhz)},
                                              {"power_w", Value(clk.power_w)},
                                              {"clock_event_reasons", Value(clk.reasons)},
                                              {"measured", Value(true)}});
    rec.timings = {m.r.median_ms, m.r.p20_ms, m.r.p80_ms};
    rec.provenance.timestamp = ts;
    rec.provenance.tool_version = kToolVersion;
    rec.provenance.mode = "measured";
    try {
      db.put(std::move(rec));
    } catch (const std::invalid_argument &e) {
      std::fprintf(stderr, "kernscope-bench: record not stored: %s\n", e.what());
    }
  }
  std::error_code ec;
  const std::filesystem::path dbp(a.db);
  if (dbp.has_parent_path()) std::filesystem::create_directories(dbp.parent_path(), ec);
  const bool saved = db.save(a.db);

  if (a.json) {
    std::vector<Value> list;
    for (const Measurement &m : ms)
      list.push_back(kernscope::db::json::object({{"family", Value(m.family)},
                                                  {"label", Value(m.label)},
                                                  {"value", Value(m.value)},
                                                  {"unit", Value(m.unit)},
                                                  {"median_ms", Value(m.r.median_ms)},
                                                  {"p20_ms", Value(m.r.p20_ms)},
                                                  {"p80_ms", Value(m.r.p80_ms)},
                                                  {"hbm_resident", Value(m.hbm_resident)}}));
    const Value out = kernscope::db::json::object(
        {{"tool", Value(kToolVersion)},
         {"device", Value(clk.name)},
         {"arch", Value("sm_100a")},
         {"peaks", kernscope::db::json::object({{"hbm_gbs", Value(hbm)},
                                                {"bf16_tflops", Value(bf16)},
                                                {"fp32_tflops", Value(fp32)},
                                                {"smem_gbs", Value(smem)}})},
         {"clocks", kernscope::db::json::object({{"sm_mhz", Value(clk.sm_mhz)},
                                                 {"mem_mhz", Value(clk.mem_mhz)},
                                                 {"sm_max_mhz", Value(clk.sm_max_mhz)},
                                                 {"power_w", Value(clk.power_w)},
                                                 {"reasons", Value(clk.reasons)}})},
         {"measurements", Value(list)},
         {"db", Value(saved ? a.db : std::string())},
         {"floors_ok", Value(floors_ok)}});
    std::printf("%s\n", out.dump().c_str());
  } else {
    for (const Measurement &m : ms)
      std::printf("%-24s %-32s %10.1f %s  (median %.4f ms, p20 %.4f, p80 %.4f)%s\n", m.family.c_str(),
                  m.label.c_str(), m.value, m.unit.c_str(), m.r.median_ms, m.r.p20_ms, m.r.p80_ms,
                  m.hbm_resident ? "" : "  [L2-resident size: not an HBM number]");
    std::printf("peaks: HBM %.1f GB/s, bf16 %.1f TFLOP/s, fp32 %.1f TFLOP/s, smem %.1f GB/s; clocks sm %s MHz (max %s)%s\n",
                hbm, bf16, fp32, smem, clk.sm_mhz.c_str(), clk.sm_max_mhz.c_str(),
                saved ? (", db " + a.db).c_str() : ", db not written");
  }
  return floors_ok ? 0 : 1;
}

// An exception from the library ends the tool with an error status and its
// message instead of std::terminate.
int main(int argc, char **argv) {
  try {
    return run_main(argc, argv);
  } catch (const std::exception &e) {
    std::fprintf(stderr, "kernscope-bench: internal error: %s\n", e.what());
  } catch (...) {
    std::fprintf(stderr, "kernscope-bench: internal error\n");
  }
  return 2;
}
