// driver.cpp -- the tuning pipeline, its tunecache and JSON evidence, and the
// C entry points that the Python binding and tests use.
#include "driver.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <tuple>

#include "bench.h"
#include "families.h"
#include "hwmodel.h"
#include "kernscope_b200.h"

namespace kernscope::tune {

using db::json::Value;
using db::json::object;

const char *driver_status_name(DriverStatus s) noexcept {
  switch (s) {
    case DriverStatus::kOk: return "ok";
    case DriverStatus::kNoViableConfig: return "no_viable_config";
    case DriverStatus::kNoLiveGpu: return "no_live_gpu";
    case DriverStatus::kUsageError: return "usage_error";
    case DriverStatus::kInternalError: return "internal_error";
  }
  return "unknown";
}

// FNV-1a 64 over "family:d0,d1,..." (driver.cpp:66-76 of the reference)
std::string make_shape_hash(const std::string &family, const std::vector<std::int64_t> &shape) {
  std::string key = family + ":";
  for (size_t i = 0; i < shape.size(); ++i) key += (i ? "," : "") + std::to_string(shape[i]);
  std::uint64_t h = 0xcbf29ce484222325ull;
  for (unsigned char c : key) {
    h ^= c;
    h *= 0x100000001b3ull;
  }
  char buf[32];
  std::snprintf(buf, sizeof(buf), "%016llx", static_cast<unsigned long long>(h));
  return std::string("fnv1a64:") + buf;
}

std::string make_cache_key(const std::string &arch, const std::string &family, const std::string &hash) {
  return arch + ":" + family + ":" + hash;
}

// ---------------------------------------------------------------------------
// Tunecache: {schema_version: 1, entries: {<arch:family:hash>: {key: {gpu_arch,
// kernel_family, shape_hash, shape}, configs: [{config, outcome: {status,
// min_occupancy, reason?, timings?, occupancy?, limiter?, gate?}}]}}}
// (the reference's schema, driver_pipeline_impl.h:229-306).
// ---------------------------------------------------------------------------
struct CachedOutcome {
  std::string status;
  std::string reason;
  bool has_timings = false;
  double median = 0, p20 = 0, p80 = 0;
  double occupancy = 0;
  std::string limiter;
  std::string gate_shape, gate_grid, gate_block, gate_symbol;
  double min_occupancy = 0;
};

class Tunecache {
 public:
  bool load(const std::string &path, std::string *warning) {
    entries_.clear();
    if (path.empty()) return true;
    std::ifstream fh(path);
    if (!fh) return true;  // no cache yet
    std::stringstream ss;
    ss << fh.rdbuf();
    Value root;
    std::string err;
    if (!Value::parse(ss.str(), &root, &err) || !root.find("entries") || !root.find("entries")->is_object()) {
      if (warning) *warning = "ignoring unreadable tunecache " + path + ": " + err;
      return false;
    }
    for (const auto &[key, entry] : root.find("entries")->as_object()) {
      const Value *cfgs = entry.find("configs");
      if (!cfgs || !cfgs->is_array()) continue;
      for (const Value &rec : cfgs->as_array()) {
        const Value *c = rec.find("config");
        const Value *o = rec.find("outcome");
        if (!c || !o) continue;
        CachedOutcome out;
        out.status = o->string_or("status", "");
        out.reason = o->string_or("reason", "");
        out.min_occupancy = o->number_or("min_occupancy", 0.0);
        out.occupancy = o->number_or("occupancy", 0.0);
        out.limiter = o->string_or("limiter", "");
        if (const Value *t = o->find("timings")) {
          out.has_timings = true;
          out.median = t->number_or("median", 0);
          out.p20 = t->number_or("p20", 0);
          out.p80 = t->number_or("p80", 0);
        }
        if (const Value *g = o->find("gate")) {
          out.gate_shape = g->string_or("shape", "");
          out.gate_grid = g->string_or("grid", "");
          out.gate_block = g->string_or("block", "");
          out.gate_symbol = g->string_or("symbol", "");
        }
        entries_[key][canonical_config(*c)] = {*c, out};
      }
    }
    return true;
  }
  bool get(const std::string &key, const std::string &canon, double floor, CachedOutcome *out) const {
    auto it = entries_.find(key);
    if (it == entries_.end()) return false;
    auto jt = it->second.find(canon);
    if (jt == it->second.end() || jt->second.second.min_occupancy != floor) return false;
    *out = jt->second.second;
    return true;
  }
  void set(const std::string &key, const Value &cfg, const std::string &canon, CachedOutcome o) {
    entries_[key][canon] = {cfg, std::move(o)};
  }
  bool save(const std::string &path, const std::string &arch, const std::string &family, const std::string &hash,
            const std::vector<std::int64_t> &shape, std::string *error) const {
    if (path.empty()) return true;
    std::vector<Value::Member> em;
    for (const auto &[key, entry] : entries_) {
      std::vector<Value> cfgs;
      for (const auto &[canon, rec] : entry) {
        const CachedOutcome &o = rec.second;
        std::vector<Value::Member> om{{"status", Value(o.status)}, {"min_occupancy", Value(o.min_occupancy)}};
        if (!o.reason.empty()) om.emplace_back("reason", Value(o.reason));
        if (o.has_timings)
          om.emplace_back("timings",
                          object({{"median", Value(o.median)}, {"p20", Value(o.p20)}, {"p80", Value(o.p80)}}));
        if (o.occupancy > 0) om.emplace_back("occupancy", Value(o.occupancy));
        if (!o.limiter.empty()) om.emplace_back("limiter", Value(o.limiter));
        if (!o.gate_shape.empty())
          om.emplace_back("gate", object({{"shape", Value(o.gate_shape)}, {"grid", Value(o.gate_grid)},
                                          {"block", Value(o.gate_block)}, {"symbol", Value(o.gate_symbol)}}));
        cfgs.push_back(object({{"config", rec.first}, {"outcome", Value(std::move(om))}}));
      }
      std::vector<Value> sh;
      for (auto d : shape) sh.emplace_back(double(d));
      em.emplace_back(key, object({{"key", object({{"gpu_arch", Value(arch)}, {"kernel_family", Value(family)},
                                                   {"shape_hash", Value(hash)}, {"shape", Value(sh)}})},
                                   {"configs", Value(std::move(cfgs))}}));
    }
    const Value root = object({{"schema_version", Value(1)}, {"entries", Value(std::move(em))}});
    std::error_code ec;
    const auto dir = std::filesystem::path(path).parent_path();
    if (!dir.empty()) std::filesystem::create_directories(dir, ec);
    std::ofstream fh(path, std::ios::trunc);
    if (!(fh << root.dump() << "\n")) {
      if (error) *error = "cannot write tunecache " + path;
      return false;
    }
    return true;
  }

 private:
  std::map<std::string, std::map<std::string, std::pair<Value, CachedOutcome>>> entries_;
};

// ---------------------------------------------------------------------------
namespace {

struct Variant {
  int index = 0;
  Value config;
  std::string symbol;
  std::string status;
  std::string reason;
  bool cached = false, best = false, prescreened = false;
  double occupancy = 0;
  int blocks_per_sm = 0;
  std::string limiter;
  bool has_timings = false;
  double median = 0, p20 = 0, p80 = 0;
  GateVerdict gate;
  bool gated = false;
  std::string gate_shape, gate_grid, gate_block;
};

std::string csv(const std::vector<std::int64_t> &s) {
  std::string o;
  for (size_t i = 0; i < s.size(); ++i) o += (i ? "," : "") + std::to_string(s[i]);
  return o;
}

std::string family_key(const DriverOptions &o) {
  if (o.kernel_family == "flash_attention" && o.causal) return "flash_attention:causal";
  if (o.kernel_family == "bias_gelu" && o.gelu == "tanh") return "bias_gelu:tanh";
  return o.kernel_family;
}

int select_best(const std::vector<Variant> &v) {
  int best = -1;
  for (size_t i = 0; i < v.size(); ++i) {
    if (!v[i].has_timings) continue;
    if (best < 0) {
      best = int(i);
      continue;
    }
    const Variant &b = v[size_t(best)];
    const Variant &c = v[i];
    if (c.median < b.median || (c.median == b.median && c.p20 < b.p20) ||
        (c.median == b.median && c.p20 == b.p20 && c.p80 < b.p80))
      best = int(i);
  }
  return best;
}

}  // namespace

DriverResult tune(const DriverOptions &opts, const DriverHooks *hooks) {
  DriverResult out;
  const Family *fam = find_family(family_key(opts));
  if (!fam) {
    out.status = DriverStatus::kUsageError;
    out.message = "unknown kernel family '" + opts.kernel_family +
                  "' (matmul | bias_gelu | softmax | layernorm | reduction | flash_attention)";
    return out;
  }
  if (!has_arch(opts.arch)) {
    out.status = DriverStatus::kUsageError;
    out.message = "unknown arch '" + opts.arch + "' (this build targets sm_100a)";
    return out;
  }
  if (opts.grid_preset != "auto" && opts.grid_preset != "full") {
    out.status = DriverStatus::kUsageError;
    out.message = "unknown grid preset '" + opts.grid_preset + "' (auto | full)";
    return out;
  }
  std::string reason;
  if (!fam->check_shape(opts.shape, &reason)) {
    out.status = DriverStatus::kUsageError;
    out.message = reason;
    return out;
  }
  const std::vector<std::int64_t> gate_shape = opts.gate_shape.empty() ? fam->gate_shape(opts.shape) : opts.gate_shape;
  if (!fam->check_shape(gate_shape, &reason)) {
    out.status = DriverStatus::kUsageError;
    out.message = "gate shape: " + reason;
    return out;
  }
  const std::string fam_name = opts.kernel_family;
  out.shape_hash = make_shape_hash(fam_name, opts.shape);
  out.cache_key = make_cache_key(opts.arch, fam_name, out.shape_hash);

  Tunecache cache;
  std::string cache_warning;
  if (opts.use_cache) cache.load(opts.cache_path, &cache_warning);

  // roofline entry for the tune shape
  roofline::MachinePeak peak;
  roofline::machine_peak(opts.arch, &peak);
  const Value sample_cfg = fam->enumerate(false, opts.shape).front();
  const std::int64_t flops = fam->flops(opts.shape, sample_cfg);
  const std::int64_t bytes = fam->bytes(opts.shape);
  roofline::RooflinePosition pos;
  roofline::KernelFamily rk;
  roofline::family_from_name(fam_name, &rk);
  const bool roofline_ok = roofline::roofline_position(rk, {}, bytes, std::max<std::int64_t>(flops, 1), opts.arch,
                                                       &pos) == roofline::ErrorCode::kNone;
  const bool tensor_bound = fam_name == "matmul" || fam_name == "flash_attention";

  // live device?
  int ndev = 0;
  char arch_buf[32] = {0};
  bool have_gpu = ks_gpu_device_count(&ndev) == KS_OK && ndev > opts.device;
  if (have_gpu) {
    have_gpu = ks_gpu_set_device(opts.device) == KS_OK && ks_gpu_arch(opts.device, arch_buf, sizeof(arch_buf)) == KS_OK &&
               std::string(arch_buf) == "sm_100a";
  }
  const bool want_live = opts.live_bench && have_gpu;

  std::unique_ptr<Session> gate_session, bench_session;
  std::string session_error;
  void *stream = nullptr;
  if (want_live) ks_gpu_stream_create(&stream);

  std::vector<Variant> variants;
  const std::vector<Value> grid = fam->enumerate(opts.grid_preset == "full", opts.shape);
  const ArchInfo &arch = get_arch(opts.arch);
  int idx = 0;
  for (const Value &cfg : grid) {
    Variant v;
    v.index = idx++;
    v.config = cfg;
    v.symbol = fam->symbol(cfg);
    const std::string canon = canonical_config(cfg);
    CachedOutcome co;
    if (opts.use_cache && cache.get(out.cache_key, canon, opts.min_occupancy, &co)) {
      v.cached = true;
      v.status = co.status;
      v.reason = co.reason;
      v.has_timings = co.has_timings;
      v.median = co.median, v.p20 = co.p20, v.p80 = co.p80;
      v.occupancy = co.occupancy;
      v.limiter = co.limiter;
      v.gate_shape = co.gate_shape, v.gate_grid = co.gate_grid, v.gate_block = co.gate_block;
      ++out.cached;
      if (v.status == "prescreen_rejected") ++out.prescreen_rejected;
      if (v.has_timings) ++out.benchmarked;
      cache.set(out.cache_key, cfg, canon, co);
      variants.push_back(std::move(v));
      continue;
    }
    auto record = [&](Variant &vv) {
      CachedOutcome c;
      c.status = vv.status;
      c.reason = vv.reason;
      c.has_timings = vv.has_timings;
      c.median = vv.median, c.p20 = vv.p20, c.p80 = vv.p80;
      c.occupancy = vv.occupancy;
      c.limiter = vv.limiter;
      c.gate_shape = vv.gate_shape, c.gate_grid = vv.gate_grid, c.gate_block = vv.gate_block;
      c.gate_symbol = vv.gated ? vv.symbol : "";
      c.min_occupancy = opts.min_occupancy;
      cache.set(out.cache_key, vv.config, canon, c);
    };
    // 1a. search space + budgets
    const ConfigVerdict cv = fam->validate(cfg, opts.shape, opts.arch);
    if (!cv.valid) {
      v.status = "prescreen_rejected";
      v.reason = cv.reason;
      ++out.prescreen_rejected;
      record(v);
      variants.push_back(std::move(v));
      continue;
    }
    // 1b. occupancy
    const Resources res = fam->resources(cfg, opts.shape);
    const auto occ = occupancy::compute_occupancy(arch, res.regs_per_thread, res.smem_bytes, res.block, res.tmem_columns);
    v.prescreened = true;
    v.occupancy = occ.occupancy;
    v.blocks_per_sm = occ.blocks_per_sm;
    v.limiter = occupancy::limiter_name(occ.limiter);
    if (occ.blocks_per_sm == 0) {
      v.status = "prescreen_rejected";
      v.reason = std::string("0 resident CTAs per SM (limiter: ") + v.limiter + ")";
      ++out.prescreen_rejected;
      record(v);
      variants.push_back(std::move(v));
      continue;
    }
    if (opts.min_occupancy > 0.0 && occ.occupancy < opts.min_occupancy) {
      char buf[160];
      std::snprintf(buf, sizeof(buf), "occupancy %.3f below the floor %.3f (limiter: %s)", occ.occupancy,
                    opts.min_occupancy, v.limiter.c_str());
      v.status = "prescreen_rejected";
      v.reason = buf;
      ++out.prescreen_rejected;
      record(v);
      variants.push_back(std::move(v));
      continue;
    }
    // 2. the prebuilt instantiation
    ++out.compiled;
    if (!want_live) {
      v.status = "compiled";
      record(v);
      variants.push_back(std::move(v));
      continue;
    }
    // 3. correctness gate
    if (!gate_session) {
      gate_session = fam->make_session(gate_shape, opts.seed, &session_error);
      if (!gate_session) break;
    }
    const LaunchGeometry gg = fam->geometry(cfg, gate_shape);
    v.gated = true;
    v.gate_shape = csv(gate_shape);
    v.gate_grid = std::to_string(gg.grid_x) + (gg.grid_y > 1 ? " x " + std::to_string(gg.grid_y) : "");
    v.gate_block = std::to_string(gg.block_x) + " x " + std::to_string(gg.block_y);
    int st = gate_session->launch(cfg, stream);
    if (st == KS_OK) st = ks_gpu_stream_synchronize(stream);
    if (st != KS_OK) {
      v.status = "compile_failed";
      v.reason = std::string("launch rejected: ") + ks_status_string(st);
      ++out.compile_failed;
      record(v);
      variants.push_back(std::move(v));
      continue;
    }
    if (hooks && hooks->corrupt_gate_output && hooks->corrupt_gate_output(opts, cfg)) {
      gate_session->corrupt_output(stream);
      ks_gpu_stream_synchronize(stream);
    }
    std::vector<float> got, ref;
    st = gate_session->output(&got);
    gate_session->reference(&ref);
    v.gate = gate_session->verdict(got, ref);
    if (st != KS_OK || !v.gate.pass) {
      char buf[256];
      std::snprintf(buf, sizeof(buf), "golden gate failed: cosine %.6f max_rel_err %.4g pcc %.6f floor %.4g norm %.4g",
                    v.gate.cosine, v.gate.max_rel_err, v.gate.pcc, v.gate.floor_rel_err, v.gate.norm_rel_err);
      v.status = "golden_gate_failed";
      v.reason = buf;
      ++out.golden_failed;
      record(v);
      variants.push_back(std::move(v));
      continue;
    }
    // 4. benchmark
    if (!bench_session) {
      bench_session = fam->make_session(opts.shape, opts.seed + 1, &session_error);
      if (!bench_session) break;
    }
    bench::Options bo;
    bo.warmup_ms = opts.warmup_ms;
    bo.rep_ms = opts.rep_ms;
    Session *bs = bench_session.get();
    const bench::Result br = bench::run([&](void *s) { return bs->launch(cfg, s); }, bo, stream);
    if (br.error != 0) {
      v.status = "bench_failed";
      v.reason = br.error_message;
      ++out.bench_failed;
      record(v);
      variants.push_back(std::move(v));
      continue;
    }
    v.status = "benchmarked";
    v.has_timings = true;
    v.median = br.median_ms, v.p20 = br.p20_ms, v.p80 = br.p80_ms;
    ++out.benchmarked;
    record(v);
    variants.push_back(std::move(v));
  }
  if (stream) ks_gpu_stream_destroy(stream);
  bench_session.reset();
  gate_session.reset();

  out.variants_total = int(variants.size());
  for (const Variant &v : variants)
    if (v.has_timings) out.measured_medians.push_back(v.median);
  const int best = select_best(variants);
  if (best >= 0) {
    Variant &b = variants[size_t(best)];
    b.best = true;
    out.has_best = true;
    out.best_config = b.config;
    out.best_symbol = b.symbol;
    out.best_median_ms = b.median, out.best_p20_ms = b.p20, out.best_p80_ms = b.p80;
  }

  // db records for fresh measurements
  int db_records = 0;
  bool db_ok = true;
  if (!opts.db_path.empty()) {
    db::Database d;
    std::vector<db::LoadWarning> w;
    d.load(opts.db_path, w);
    for (const Variant &v : variants) {
      if (!v.has_timings || v.cached) continue;
      db::Record r;
      r.gpu_arch = opts.arch;
      r.kernel_family = fam_name;
      r.shape_hash = out.shape_hash;
      r.config = v.config;
      r.timings = {v.median, v.p20, v.p80};
      r.provenance = {db::utc_timestamp(), kToolVersion, "measured"};
      try {
        d.put(std::move(r));
        ++db_records;
      } catch (const std::invalid_argument &) {
        // non-finite timings: the variant's evidence keeps them, the db does not
      }
    }
    db_ok = d.save(opts.db_path);
  }
  std::string cache_error;
  cache.save(opts.cache_path, opts.arch, fam_name, out.shape_hash, opts.shape, &cache_error);

  // status
  const bool any_viable = std::any_of(variants.begin(), variants.end(), [](const Variant &v) {
    return v.status == "compiled" || v.status == "benchmarked";
  });
  if (!session_error.empty()) {
    out.status = DriverStatus::kInternalError;
    out.message = session_error;
  } else if (out.has_best) {
    out.status = DriverStatus::kOk;
    out.message = "best " + out.best_symbol;
  } else if (!any_viable && out.prescreen_rejected + out.golden_failed + out.compile_failed + out.bench_failed ==
                                out.variants_total) {
    out.status = DriverStatus::kNoViableConfig;
    out.message = "no viable config: " + std::to_string(out.prescreen_rejected) + " pre-screen rejected, " +
                  std::to_string(out.golden_failed) + " failed the golden gate, " +
                  std::to_string(out.compile_failed + out.bench_failed) + " failed to launch/bench";
  } else if (opts.live_bench && !have_gpu) {
    out.status = DriverStatus::kNoLiveGpu;
    out.message = "the gate and benchmark need an sm_100a GPU (none found); pre-screen only";
  } else {
    out.status = DriverStatus::kOk;
    out.message = "pre-screen only (--no-bench): " + std::to_string(out.compiled) + " configs viable";
  }

  // evidence
  double baseline_median = 0;
  Value baseline_cfg;
  for (const Variant &v : variants)
    if (v.has_timings) {
      baseline_median = v.median;
      baseline_cfg = v.config;
      break;
    }
  std::vector<const Variant *> ord;
  for (const Variant &v : variants) ord.push_back(&v);
  // report order (the reference's contract): measured variants by median,
  // ties on p20 then p80, then the rest in enumeration order
  std::stable_sort(ord.begin(), ord.end(), [](const Variant *a, const Variant *b) {
    if (a->has_timings != b->has_timings) return a->has_timings;
    if (a->has_timings && a->median != b->median) return a->median < b->median;
    if (a->has_timings && a->p20 != b->p20) return a->p20 < b->p20;
    if (a->has_timings && a->p80 != b->p80) return a->p80 < b->p80;
    return a->index < b->index;
  });
  std::vector<Value> vars;
  auto achieved = [&](double ms) { return ms > 0 ? (tensor_bound ? double(flops) / (ms * 1e9) : double(bytes) / (ms * 1e6)) : 0.0; };
  const double peak_unit = tensor_bound ? peak.matrix_peak_flops / 1e12 : peak.bandwidth_bytes_per_s / 1e9;
  for (const Variant *vp : ord) {
    const Variant &v = *vp;
    std::vector<Value::Member> m{{"index", Value(v.index)}, {"config", v.config}, {"symbol", Value(v.symbol)},
                                 {"status", Value(v.status)}, {"cached", Value(v.cached)}, {"best", Value(v.best)}};
    if (!v.reason.empty()) m.emplace_back("reason", Value(v.reason));
    if (v.prescreened || v.occupancy > 0) {
      m.emplace_back("occupancy", Value(v.occupancy));
      if (!v.limiter.empty()) m.emplace_back("limiter", Value(v.limiter));
      m.emplace_back("blocks_per_sm", Value(v.blocks_per_sm));
    }
    if (v.gated)
      m.emplace_back("gate", object({{"shape", Value(v.gate_shape)}, {"grid", Value(v.gate_grid)},
                                     {"block", Value(v.gate_block)}, {"pass", Value(v.gate.pass)},
                                     {"cosine", Value(v.gate.cosine)}, {"max_rel_err", Value(v.gate.max_rel_err)},
                                     {"pcc", Value(v.gate.pcc)}, {"floor_rel_err", Value(v.gate.floor_rel_err)},
                                     {"norm_rel_err", Value(v.gate.norm_rel_err)},
                                     {"criterion", Value(v.gate.criterion)}}));
    if (v.has_timings) {
      m.emplace_back("timings", object({{"median", Value(v.median)}, {"p20", Value(v.p20)}, {"p80", Value(v.p80)}}));
      const double a = achieved(v.median);
      m.emplace_back(tensor_bound ? "achieved_tflops" : "achieved_gbps", Value(a));
      m.emplace_back("roofline_achieved", Value(peak_unit > 0 ? a / peak_unit : 0.0));
    }
    vars.push_back(Value(std::move(m)));
  }
  Value best_v;
  double best_occ = 0.0;
  std::string best_limiter;
  if (out.has_best) {
    const double a = achieved(out.best_median_ms);
    std::vector<Value::Member> bm{{"config", out.best_config}, {"symbol", Value(out.best_symbol)},
                                  {"timings", object({{"median", Value(out.best_median_ms)},
                                                      {"p20", Value(out.best_p20_ms)},
                                                      {"p80", Value(out.best_p80_ms)}})},
                                  {tensor_bound ? "achieved_tflops" : "achieved_gbps", Value(a)},
                                  {"roofline_achieved", Value(peak_unit > 0 ? a / peak_unit : 0.0)}};
    for (const Variant &v : variants)
      if (v.best) {
        best_occ = v.occupancy;
        best_limiter = v.limiter;
        if (v.gated)
          bm.emplace_back("gate", object({{"shape", Value(v.gate_shape)}, {"grid", Value(v.gate_grid)},
                                          {"block", Value(v.gate_block)}, {"symbol", Value(v.symbol)}}));
      }
    best_v = Value(std::move(bm));
  }
  std::vector<Value> sh;
  for (auto d : opts.shape) sh.emplace_back(double(d));
  std::vector<Value> gsh;
  for (auto d : gate_shape) gsh.emplace_back(double(d));
  const Value ev = object({
      {"schema_version", Value(1)},
      {"tool_version", Value(kToolVersion)},
      {"kernel_family", Value(fam_name)},
      {"gpu_arch", Value(opts.arch)},
      {"shape", Value(sh)},
      {"gate_shape", Value(gsh)},
      {"shape_hash", Value(out.shape_hash)},
      {"cache_key", Value(out.cache_key)},
      {"grid_preset", Value(opts.grid_preset)},
      {"grid_size", Value(out.variants_total)},
      {"min_occupancy", Value(opts.min_occupancy)},
      {"n_gpus", Value(1)},
      {"live", Value(want_live)},
      {"status", Value(driver_status_name(out.status))},
      {"message", Value(out.message)},
      {"summary", object({{"variants_total", Value(out.variants_total)},
                          {"prescreen_rejected", Value(out.prescreen_rejected)},
                          {"compile_failed", Value(out.compile_failed)},
                          {"golden_gate_failed", Value(out.golden_failed)},
                          {"bench_failed", Value(out.bench_failed)},
                          {"benchmarked", Value(out.benchmarked)},
                          {"cached", Value(out.cached)},
                          {"compiled", Value(out.compiled)},
                          {"verifier_gated", Value(0)}})},
      {"roofline", object({{"ok", Value(roofline_ok)},
                           {"family", Value(fam_name)},
                           {"flops", Value(double(flops))},
                           {"bytes_moved", Value(double(bytes))},
                           {"arithmetic_intensity", Value(pos.arithmetic_intensity)},
                           {"ridge_point", Value(pos.ridge_point)},
                           {"bound_class", Value(roofline::bound_class_name(pos.bound_class))},
                           {"bound", Value(roofline::bound_class_name(pos.bound_class))},
                           {"position", Value(pos.compute_bound_ceiling > 0
                                                  ? pos.attained_flops / pos.compute_bound_ceiling
                                                  : 0.0)},
                           {"compute_bound_ceiling", Value(pos.compute_bound_ceiling)},
                           {"memory_bound_ceiling", Value(pos.memory_bound_ceiling)},
                           {"attained_flops", Value(pos.attained_flops)},
                           {"peak", Value(peak_unit)},
                           {"peak_unit", Value(tensor_bound ? "TFLOP/s" : "GB/s")},
                           {"peak_provenance", Value(peak.provenance)},
                           {"projected", Value(peak.projected)}})},
      {"best", best_v},
      {"occupancy", Value(best_occ)},
      {"occupancy.limiter", Value(best_limiter)},
      {"speedup", Value(baseline_median > 0 && out.best_median_ms > 0 ? baseline_median / out.best_median_ms : 0.0)},
      {"baseline", object({{"config", baseline_cfg}, {"timings", object({{"median", Value(baseline_median)}})}})},
      {"variants", Value(std::move(vars))},
      {"db", object({{"path", Value(opts.db_path)}, {"records", Value(db_records)}, {"ok", Value(db_ok)}})},
      {"cache", object({{"path", Value(opts.cache_path)}, {"warning", Value(cache_warning)},
                        {"error", Value(cache_error)}})},
  });
  out.evidence_json = ev.dump();
  return out;
}

bool emit_repro(const DriverOptions &opts, const DriverResult &r, const std::string &dir, std::string *error) {
  if (!r.has_best) {
    if (error) *error = "no winning config to reproduce";
    return false;
  }
  const Family *fam = find_family(family_key(opts));
  std::error_code ec;
  std::filesystem::create_directories(dir, ec);
  const std::string src = fam->generate_source(r.best_config, opts.shape);
  std::ofstream(dir + "/repro.cpp") << src;
  std::ofstream sh(dir + "/run.sh");
  sh << "#!/usr/bin/env bash\n# Rebuild and run the winning " << opts.kernel_family << " config through the C ABI.\n"
     << "set -euo pipefail\nREPO=\"${KERNSCOPE_B200_ROOT:-$(cd \"$(dirname \"$0\")\" && git rev-parse --show-toplevel)}\"\n"
     << "g++ -std=c++20 -O2 -I \"$REPO/include\" \"$(dirname \"$0\")/repro.cpp\" -L \"$REPO/kernscope_b200/lib\" "
        "-lkernscope_b200 -Wl,-rpath,\"$REPO/kernscope_b200/lib\" -o \"$(dirname \"$0\")/repro\"\n"
     << "\"$(dirname \"$0\")/repro\"\n";
  sh.close();
  std::filesystem::permissions(dir + "/run.sh", std::filesystem::perms::owner_exec, std::filesystem::perm_options::add,
                               ec);
  std::ofstream(dir + "/README.md") << "# Reproducer\n\nfamily: " << opts.kernel_family << "\nshape: " << csv(opts.shape)
                                    << "\nconfig: " << r.best_config.dump() << "\nsymbol: " << r.best_symbol
                                    << "\nmedian: " << r.best_median_ms << " ms\n\n`run.sh` compiles `repro.cpp` "
                                    << "against libkernscope_b200.so and launches the config once.\n";
  return true;
}

}  // namespace kernscope::tune

// ---------------------------------------------------------------------------
// C entry points (Python binding / tests)
// ---------------------------------------------------------------------------
namespace {
using kernscope::db::json::Value;

int write_out(const std::string &s, char *out, size_t cap, size_t *needed) {
  if (needed) *needed = s.size() + 1;
  if (!out || cap < s.size() + 1) return -1;
  std::memcpy(out, s.c_str(), s.size() + 1);
  return 0;
}

std::vector<std::int64_t> shape_of(const Value *v) {
  std::vector<std::int64_t> s;
  if (v && v->is_array())
    for (const Value &x : v->as_array()) s.push_back(std::int64_t(x.as_number()));
  return s;
}

kernscope::tune::DriverOptions options_from(const Value &j) {
  kernscope::tune::DriverOptions o;
  o.kernel_family = j.string_or("kernel_family", "");
  o.shape = shape_of(j.find("shape"));
  o.gate_shape = shape_of(j.find("gate_shape"));
  o.arch = j.string_or("arch", "sm_100a");
  o.grid_preset = j.string_or("grid", "auto");
  o.db_path = j.string_or("db", "");
  o.cache_path = j.string_or("cache", "");
  o.min_occupancy = j.number_or("min_occupancy", 0.0);
  if (const Value *v = j.find("live_bench")) o.live_bench = v->as_bool();
  if (const Value *v = j.find("use_cache")) o.use_cache = v->as_bool();
  if (const Value *v = j.find("causal")) o.causal = v->as_bool();
  o.gelu = j.string_or("gelu", "erf");
  o.device = int(j.number_or("device", 0));
  o.warmup_ms = j.number_or("warmup_ms", 25.0);
  o.rep_ms = j.number_or("rep_ms", 100.0);
  o.seed = std::uint64_t(j.number_or("seed", 0));
  return o;
}

// Exceptions never cross the C ABI: report them as an internal error.
template <class F>
int guarded(char *out, size_t cap, size_t *needed, F &&f) {
  try {
    return f();
  } catch (const std::exception &e) {
    return write_out(kernscope::db::json::object({{"status", Value("internal_error")}, {"error", Value(e.what())}})
                         .dump(),
                     out, cap, needed) == 0
               ? 2
               : -1;
  } catch (...) {
    return write_out("{\"status\":\"internal_error\",\"error\":\"unknown exception\"}", out, cap, needed) == 0
               ? 2
               : -1;
  }
}

// Run the tuning pipeline: options as JSON (keys of DriverOptions plus
// "inject_gate_failure": config index whose gate output is zeroed); writes
// the evidence JSON.  Returns the CLI exit code (0 ok, 1 no viable config,
// 2 otherwise) or -1 when `out` is too small (*needed = bytes required).
int tune_run_json(const char *options_json, char *out, size_t cap, size_t *needed) {
  Value j;
  std::string err;
  if (!options_json || !Value::parse(options_json, &j, &err)) {
    write_out(kernscope::db::json::object({{"status", Value("usage_error")}, {"message", Value(err)}}).dump(), out,
              cap, needed);
    return 2;
  }
  kernscope::tune::DriverOptions o = options_from(j);
  const int inject = int(j.number_or("inject_gate_failure", -1));
  kernscope::tune::DriverHooks hooks;
  int seen = 0;
  hooks.corrupt_gate_output = [&](const kernscope::tune::DriverOptions &, const Value &) { return seen++ == inject; };
  kernscope::tune::DriverResult r = kernscope::tune::tune(o, inject >= 0 ? &hooks : nullptr);
  std::string ev = r.evidence_json.empty()
                       ? kernscope::db::json::object({{"status", Value(kernscope::tune::driver_status_name(r.status))},
                                                      {"message", Value(r.message)}})
                             .dump()
                       : r.evidence_json;
  if (write_out(ev, out, cap, needed) != 0) return -1;
  if (const Value *e = j.find("emit_repro"); e && e->is_string()) kernscope::tune::emit_repro(o, r, e->as_string(), nullptr);
  return r.status == kernscope::tune::DriverStatus::kOk ? 0
         : r.status == kernscope::tune::DriverStatus::kNoViableConfig ? 1
                                                                       : 2;
}

// Small queries of the host model for tests: {"op": ...}.
//   shape_hash {family, shape}; cache_key {arch, family, shape_hash};
//   enumerate {family, shape, full, causal?, gelu?}; validate {family, shape, config};
//   occupancy {regs, smem, block, tmem}; roofline {family, shape, causal?};
//   geometry {family, shape, config}; peaks {}; db_roundtrip {path, records[]}
int tune_query_json(const char *request_json, char *out, size_t cap, size_t *needed) {
  using namespace kernscope;
  using kernscope::db::json::object;
  Value j;
  std::string err;
  if (!request_json || !Value::parse(request_json, &j, &err))
    return write_out(object({{"error", Value(err)}}).dump(), out, cap, needed) == 0 ? 2 : -1;
  const std::string op = j.string_or("op", "");
  const std::vector<std::int64_t> shape = shape_of(j.find("shape"));
  tune::DriverOptions o = options_from(j);
  o.kernel_family = j.string_or("family", "");
  Value res;
  if (op == "shape_hash") {
    res = Value(tune::make_shape_hash(o.kernel_family, shape));
  } else if (op == "cache_key") {
    res = Value(tune::make_cache_key(j.string_or("arch", "sm_100a"), o.kernel_family, j.string_or("shape_hash", "")));
  } else if (op == "enumerate" || op == "validate" || op == "geometry") {
    std::string key = o.kernel_family;
    if (key == "flash_attention" && o.causal) key += ":causal";
    if (key == "bias_gelu" && o.gelu == "tanh") key += ":tanh";
    const tune::Family *f = tune::find_family(key);
    if (!f) return write_out(object({{"error", Value("unknown family")}}).dump(), out, cap, needed) == 0 ? 2 : -1;
    if (op == "enumerate") {
      std::vector<Value> v;
      for (const Value &c : f->enumerate(j.find("full") && j.find("full")->as_bool(), shape)) {
        const tune::ConfigVerdict cv = f->validate(c, shape, j.string_or("arch", "sm_100a"));
        v.push_back(object({{"config", c}, {"valid", Value(cv.valid)}, {"reason", Value(cv.reason)},
                            {"symbol", Value(f->symbol(c))}}));
      }
      res = Value(std::move(v));
    } else if (op == "validate") {
      const tune::ConfigVerdict cv = f->validate(*j.find("config"), shape, j.string_or("arch", "sm_100a"));
      res = object({{"valid", Value(cv.valid)}, {"reason", Value(cv.reason)}});
    } else {
      const tune::LaunchGeometry g = f->geometry(*j.find("config"), shape);
      const tune::Resources r = f->resources(*j.find("config"), shape);
      res = object({{"grid_x", Value(g.grid_x)}, {"grid_y", Value(g.grid_y)}, {"block_x", Value(g.block_x)},
                    {"block_y", Value(g.block_y)}, {"smem_bytes", Value(g.smem_bytes)},
                    {"tmem_columns", Value(g.tmem_columns)}, {"regs_per_thread", Value(r.regs_per_thread)},
                    {"gate_shape", Value([&] {
                       std::vector<Value> gs;
                       for (auto d : f->gate_shape(shape)) gs.emplace_back(double(d));
                       return gs;
                     }())},
                    {"flops", Value(double(f->flops(shape, *j.find("config"))))},
                    {"bytes", Value(double(f->bytes(shape)))},
                    {"source", Value(f->generate_source(*j.find("config"), shape))}});
    }
  } else if (op == "occupancy") {
    const auto r = occupancy::compute_occupancy(get_arch(j.string_or("arch", "sm_100a")), int(j.number_or("regs", 32)),
                                                int(j.number_or("smem", 0)), int(j.number_or("block", 128)),
                                                int(j.number_or("tmem", 0)));
    res = object({{"blocks_per_sm", Value(r.blocks_per_sm)}, {"warps_resident", Value(r.warps_resident)},
                  {"occupancy", Value(r.occupancy)}, {"limiter", Value(occupancy::limiter_name(r.limiter))}});
  } else if (op == "roofline") {
    roofline::KernelFamily k;
    if (!roofline::family_from_name(o.kernel_family, &k))
      return write_out(object({{"error", Value("unknown family")}}).dump(), out, cap, needed) == 0 ? 2 : -1;
    roofline::Shape s;
    s.m = std::int64_t(j.number_or("m", 0));
    s.n = std::int64_t(j.number_or("n", 0));
    s.k = std::int64_t(j.number_or("k", 0));
    s.d = std::int64_t(j.number_or("d", 0));
    s.dtype_bytes = int(j.number_or("dtype_bytes", 2));
    s.causal = j.find("causal") && j.find("causal")->as_bool();
    const auto fl = roofline::compute_flops(k, s);
    const auto by = roofline::compute_bytes_moved(k, s);
    roofline::RooflinePosition p;
    const auto ec = roofline::roofline_position(k, s, by, std::max<std::int64_t>(fl, 1), "sm_100a", &p);
    res = object({{"flops", Value(double(fl))}, {"bytes", Value(double(by))},
                  {"reference_model_bytes", Value(double(roofline::reference_model_bytes(k, s)))},
                  {"ai", Value(p.arithmetic_intensity)}, {"ridge", Value(p.ridge_point)},
                  {"bound", Value(roofline::bound_class_name(p.bound_class))},
                  {"projected", Value(ec == roofline::ErrorCode::kProjectedPeaks)}});
  } else if (op == "peaks") {
    roofline::MachinePeak p;
    roofline::machine_peak(j.string_or("arch", "sm_100a"), &p);
    res = object({{"hbm_gbs", Value(p.bandwidth_bytes_per_s / 1e9)}, {"bf16_tflops", Value(p.matrix_peak_flops / 1e12)},
                  {"bf16_tflops_sustained", Value(p.matrix_peak_sustained_flops / 1e12)},
                  {"projected", Value(p.projected)}, {"provenance", Value(p.provenance)}});
  } else if (op == "db_roundtrip") {
    db::Database d;
    if (const Value *rs = j.find("records"); rs && rs->is_array())
      for (const Value &rv : rs->as_array()) {
        db::Record rec;
        if (db::record_from_json(rv, &rec, &err)) {
          try {
            d.put(std::move(rec));
          } catch (const std::invalid_argument &) {
          }
        }
      }
    const std::string path = j.string_or("path", "");
    const bool saved = d.save(path);
    db::Database back;
    std::vector<db::LoadWarning> w;
    back.load(path, w);
    std::vector<Value> recs;
    for (const auto &r : back.records()) recs.push_back(db::record_to_json(r));
    Value best;
    if (const Value *q = j.find("query"); q && q->is_object()) {
      auto b = back.query_best(q->string_or("gpu_arch", ""), q->string_or("kernel_family", ""),
                               q->string_or("shape_hash", ""));
      if (b) best = db::record_to_json(*b);
    }
    res = object({{"saved", Value(saved)}, {"records", Value(std::move(recs))}, {"warnings", Value(int(w.size()))},
                  {"best", best}});
  } else if (op == "db_load") {
    // Loads one JSONL db and answers query_best for every workload key in it,
    // in first-seen order.
    db::Database d;
    std::vector<db::LoadWarning> w;
    const bool opened = d.load(j.string_or("path", ""), w);
    std::vector<Value> warn, best;
    for (const auto &lw : w) warn.push_back(Value(lw.message));
    std::set<std::tuple<std::string, std::string, std::string>> seen;
    for (const auto &r : d.records()) {
      if (!seen.insert({r.gpu_arch, r.kernel_family, r.shape_hash}).second) continue;
      if (auto b = d.query_best(r.gpu_arch, r.kernel_family, r.shape_hash))
        best.push_back(object({{"gpu_arch", Value(b->gpu_arch)}, {"kernel_family", Value(b->kernel_family)},
                               {"shape_hash", Value(b->shape_hash)}, {"config", b->config},
                               {"median", Value(b->timings.median)}}));
    }
    res = object({{"opened", Value(opened)}, {"records", Value(int(d.size()))}, {"warnings", Value(std::move(warn))},
                  {"best", Value(std::move(best))}});
  } else if (op == "golden") {
    // The gate's host half: {family, shape, seed, inputs?: {name: [bf16 bits]},
    // verdict_got?: [bf16 bits]} -> the inputs used and the reference output
    // (bf16 bits), plus the gate verdict of verdict_got against it.
    std::map<std::string, std::vector<std::uint16_t>> in, used;
    if (const Value *iv = j.find("inputs"); iv && iv->is_object())
      for (const auto &[name, arr] : iv->as_object()) {
        std::vector<std::uint16_t> bits;
        if (arr.is_array())
          for (const Value &x : arr.as_array()) bits.push_back(std::uint16_t(x.as_number()));
        in[name] = std::move(bits);
      }
    std::vector<float> expected;
    std::string gerr;
    if (!tune::golden_case(j.string_or("family", ""), shape, std::uint64_t(j.number_or("seed", 0)), in, &used,
                           &expected, &gerr))
      return write_out(object({{"error", Value(gerr)}}).dump(), out, cap, needed) == 0 ? 2 : -1;
    auto to_arr = [](const std::vector<std::uint16_t> &b) {
      std::vector<Value> v;
      v.reserve(b.size());
      for (auto x : b) v.emplace_back(double(x));
      return Value(std::move(v));
    };
    std::vector<std::uint16_t> exp_bits;
    for (float x : expected) exp_bits.push_back(tune::f32_to_bf16(x));
    std::vector<Value::Member> inputs_out;
    for (const auto &[name, b] : used) inputs_out.emplace_back(name, to_arr(b));
    std::vector<Value::Member> r{{"inputs", Value(std::move(inputs_out))}, {"expected", to_arr(exp_bits)}};
    if (const Value *g = j.find("verdict_got"); g && g->is_array()) {
      std::vector<float> got;
      for (const Value &x : g->as_array()) got.push_back(tune::bf16_to_f32(std::uint16_t(x.as_number())));
      const tune::GateVerdict gv = tune::bf16_verdict(got, expected);
      r.emplace_back("verdict", object({{"pass", Value(gv.pass)}, {"cosine", Value(gv.cosine)},
                                        {"max_rel_err", Value(gv.max_rel_err)}, {"pcc", Value(gv.pcc)}}));
    }
    res = Value(std::move(r));
  } else if (op == "quantile") {
    std::vector<double> s;
    if (const Value *v = j.find("samples"); v && v->is_array())
      for (const Value &x : v->as_array()) s.push_back(x.as_number());
    res = object({{"q", Value(bench::quantile(std::move(s), j.number_or("q", 0.5)))}});
  } else {
    return write_out(object({{"error", Value("unknown op '" + op + "'")}}).dump(), out, cap, needed) == 0 ? 2 : -1;
  }
  return write_out(object({{"result", res}}).dump(), out, cap, needed) == 0 ? 0 : -1;
}

}  // namespace

extern "C" {

int ks_tune_run_json(const char *options_json, char *out, size_t cap, size_t *needed) {
  return guarded(out, cap, needed, [&] { return tune_run_json(options_json, out, cap, needed); });
}

int ks_tune_query_json(const char *request_json, char *out, size_t cap, size_t *needed) {
  return guarded(out, cap, needed, [&] { return tune_query_json(request_json, out, cap, needed); });
}

}  // extern "C"

