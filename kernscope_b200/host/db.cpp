// db.cpp -- JSONL persistence of measured configs.
#include "db.h"

#include <algorithm>
#include <cmath>
#include <ctime>
#include <filesystem>
#include <fstream>
#include <sstream>
#include <stdexcept>

namespace kernscope::db {

json::Value record_to_json(const Record &r) {
  return json::object({
      {"schema_version", json::Value(r.schema_version)},
      {"gpu_arch", json::Value(r.gpu_arch)},
      {"kernel_family", json::Value(r.kernel_family)},
      {"shape_hash", json::Value(r.shape_hash)},
      {"config", r.config},
      {"timings", json::object({{"median", json::Value(r.timings.median)},
                                {"p20", json::Value(r.timings.p20)},
                                {"p80", json::Value(r.timings.p80)}})},
      {"provenance", json::object({{"timestamp", json::Value(r.provenance.timestamp)},
                                   {"tool_version", json::Value(r.provenance.tool_version)},
                                   {"mode", json::Value(r.provenance.mode)}})},
  });
}

bool record_from_json(const json::Value &v, Record *out, std::string *error) {
  // Every field is required and typed; provenance.mode is "measured" or
  // "projected"; schema_version is an integer no newer than this reader
  // (the reference's rules, libs/db/src/db.cpp:546-585 and :689-704).
  auto fail = [&](std::string m) {
    if (error) *error = std::move(m);
    return false;
  };
  if (!v.is_object()) return fail("line is not a JSON object");
  const json::Value *sv = v.find("schema_version");
  if (!sv || !sv->is_number()) return fail("missing or non-numeric \"schema_version\"");
  const double ver = sv->as_number();
  if (ver != std::floor(ver)) return fail("\"schema_version\" must be an integer");
  if (ver > kCurrentSchemaVersion)
    return fail("record schema_version " + std::to_string(int(ver)) + " > current " +
                std::to_string(kCurrentSchemaVersion) + " - forward-incompatible");
  auto field = [&](const json::Value &obj, const char *k, json::Value::Kind kind, const char *what)
      -> const json::Value * {
    const json::Value *x = obj.find(k);
    if (!x) {
      fail(std::string("missing required field \"") + k + "\"");
      return nullptr;
    }
    if (x->kind() != kind) {
      fail(std::string("field \"") + k + "\" is not " + what);
      return nullptr;
    }
    return x;
  };
  using K = json::Value::Kind;
  Record r;
  r.schema_version = int(ver);
  const json::Value *arch = field(v, "gpu_arch", K::String, "a string");
  if (!arch) return false;
  const json::Value *fam = field(v, "kernel_family", K::String, "a string");
  if (!fam) return false;
  const json::Value *hash = field(v, "shape_hash", K::String, "a string");
  if (!hash) return false;
  const json::Value *cfg = field(v, "config", K::Object, "an object");
  if (!cfg) return false;
  const json::Value *tim = field(v, "timings", K::Object, "an object");
  if (!tim) return false;
  const json::Value *med = field(*tim, "median", K::Number, "a number");
  if (!med) return false;
  const json::Value *p20 = field(*tim, "p20", K::Number, "a number");
  if (!p20) return false;
  const json::Value *p80 = field(*tim, "p80", K::Number, "a number");
  if (!p80) return false;
  const json::Value *prov = field(v, "provenance", K::Object, "an object");
  if (!prov) return false;
  const json::Value *ts = field(*prov, "timestamp", K::String, "a string");
  if (!ts) return false;
  const json::Value *tv = field(*prov, "tool_version", K::String, "a string");
  if (!tv) return false;
  const json::Value *mode = field(*prov, "mode", K::String, "a string");
  if (!mode) return false;
  if (mode->as_string() != "measured" && mode->as_string() != "projected")
    return fail("\"provenance.mode\" must be \"measured\" or \"projected\" (got \"" + mode->as_string() + "\")");
  r.gpu_arch = arch->as_string();
  r.kernel_family = fam->as_string();
  r.shape_hash = hash->as_string();
  r.config = *cfg;
  r.timings = {med->as_number(), p20->as_number(), p80->as_number()};
  r.provenance = {ts->as_string(), tv->as_string(), mode->as_string()};
  *out = std::move(r);
  return true;
}

namespace {

bool all_finite(const json::Value &v) {
  if (v.is_number()) return std::isfinite(v.as_number());
  if (v.is_array()) {
    for (const auto &e : v.as_array())
      if (!all_finite(e)) return false;
  } else if (v.is_object()) {
    for (const auto &m : v.as_object())
      if (!all_finite(m.second)) return false;
  }
  return true;
}

// Compact JSON with every object's members sorted by name, so configs that
// differ only in member order share one key.
void canonical_dump(const json::Value &v, std::string &out) {
  if (!v.is_object()) {
    out += v.dump();
    return;
  }
  std::vector<const json::Value::Member *> ms;
  for (const auto &m : v.as_object()) ms.push_back(&m);
  std::sort(ms.begin(), ms.end(), [](const auto *a, const auto *b) { return a->first < b->first; });
  out += '{';
  for (size_t i = 0; i < ms.size(); ++i) {
    if (i) out += ',';
    out += json::Value(ms[i]->first).dump();
    out += ':';
    canonical_dump(ms[i]->second, out);
  }
  out += '}';
}

}  // namespace

Database::Key Database::make_key(const Record &r) {
  Key k{r.gpu_arch, r.kernel_family, r.shape_hash, {}};
  canonical_dump(r.config, k.config);
  return k;
}

void Database::put(Record record) {
  if (!record.config.is_object()) throw std::invalid_argument("kernscope::db: record.config must be a JSON object");
  if (!std::isfinite(record.timings.median) || !std::isfinite(record.timings.p20) ||
      !std::isfinite(record.timings.p80))
    throw std::invalid_argument("kernscope::db: record.timings must be finite numbers");
  if (!all_finite(record.config))
    throw std::invalid_argument("kernscope::db: record.config must contain only finite numbers");
  Key key = make_key(record);
  if (auto it = index_.find(key); it != index_.end()) {
    records_[it->second] = std::move(record);  // same key: replaced in place
  } else {
    index_.emplace(std::move(key), records_.size());
    records_.push_back(std::move(record));
  }
}

std::optional<Record> Database::query_best(std::string_view gpu_arch, std::string_view kernel_family,
                                           std::string_view shape_hash) const {
  // The index is ordered by (arch, family, hash, canonical config), so the
  // matching records are one run and a tie keeps the smallest config key.
  const Key lo{std::string(gpu_arch), std::string(kernel_family), std::string(shape_hash), {}};
  const Record *best = nullptr;
  for (auto it = index_.lower_bound(lo); it != index_.end(); ++it) {
    const Key &k = it->first;
    if (k.gpu_arch != gpu_arch || k.kernel_family != kernel_family || k.shape_hash != shape_hash) break;
    const Record &r = records_[it->second];
    if (!best || r.timings.median < best->timings.median) best = &r;
  }
  if (!best) return std::nullopt;
  return *best;
}

bool Database::load(const std::string &path, std::vector<LoadWarning> &warnings) {
  std::ifstream fh(path);
  if (!fh) return false;
  std::string line;
  std::size_t n = 0;
  while (std::getline(fh, line)) {
    ++n;
    if (!line.empty() && line.back() == '\r') line.pop_back();
    if (line.find_first_not_of(" \t") == std::string::npos) continue;
    const std::string at = "line " + std::to_string(n) + ": ";
    json::Value v;
    std::string err;
    if (!json::Value::parse(line, &v, &err)) {
      warnings.push_back({n, at + "malformed JSON line skipped: " + err});
      continue;
    }
    Record r;
    if (!record_from_json(v, &r, &err)) {
      warnings.push_back({n, at + "record rejected: " + err});
      continue;
    }
    try {
      put(std::move(r));
    } catch (const std::invalid_argument &e) {
      warnings.push_back({n, at + "record rejected: " + e.what()});
    }
  }
  return true;
}

bool Database::save(const std::string &path) const {
  std::error_code ec;
  const auto dir = std::filesystem::path(path).parent_path();
  if (!dir.empty()) std::filesystem::create_directories(dir, ec);
  std::ofstream fh(path, std::ios::trunc);
  if (!fh) return false;
  for (const Record &r : records_) fh << record_to_json(r).dump() << "\n";
  return bool(fh);
}

std::string utc_timestamp() {
  const std::time_t t = std::time(nullptr);
  std::tm tm{};
  gmtime_r(&t, &tm);
  char buf[32];
  std::strftime(buf, sizeof(buf), "%Y-%m-%dT%H:%M:%SZ", &tm);
  return buf;
}

}  // namespace kernscope::db
