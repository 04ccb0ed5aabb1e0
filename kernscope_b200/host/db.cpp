// db.cpp -- JSONL persistence of measured configs.
#include "db.h"

#include <ctime>
#include <filesystem>
#include <fstream>
#include <sstream>

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
  auto need = [&](const char *k) -> const json::Value * {
    const json::Value *x = v.find(k);
    if (!x && error) *error = std::string("missing field '") + k + "'";
    return x;
  };
  if (!v.is_object()) {
    if (error) *error = "record is not an object";
    return false;
  }
  const json::Value *sv = need("schema_version"), *arch = need("gpu_arch"), *fam = need("kernel_family"),
                    *hash = need("shape_hash"), *cfg = need("config"), *tim = need("timings");
  if (!sv || !arch || !fam || !hash || !cfg || !tim) return false;
  if (!sv->is_number() || int(sv->as_number()) != kCurrentSchemaVersion) {
    if (error) *error = "unsupported schema_version";
    return false;
  }
  if (!arch->is_string() || !fam->is_string() || !hash->is_string() || !tim->is_object()) {
    if (error) *error = "wrong field types";
    return false;
  }
  Record r;
  r.gpu_arch = arch->as_string();
  r.kernel_family = fam->as_string();
  r.shape_hash = hash->as_string();
  r.config = *cfg;
  r.timings.median = tim->number_or("median", 0.0);
  r.timings.p20 = tim->number_or("p20", 0.0);
  r.timings.p80 = tim->number_or("p80", 0.0);
  if (const json::Value *p = v.find("provenance"); p && p->is_object()) {
    r.provenance.timestamp = p->string_or("timestamp", "");
    r.provenance.tool_version = p->string_or("tool_version", "");
    r.provenance.mode = p->string_or("mode", "");
  }
  *out = std::move(r);
  return true;
}

void Database::put(Record record) { records_.push_back(std::move(record)); }

std::optional<Record> Database::query_best(std::string_view gpu_arch, std::string_view kernel_family,
                                           std::string_view shape_hash) const {
  const Record *best = nullptr;
  for (const Record &r : records_) {
    if (r.gpu_arch != gpu_arch || r.kernel_family != kernel_family || r.shape_hash != shape_hash) continue;
    if (!best || r.timings.median < best->timings.median) best = &r;
  }
  if (!best) return std::nullopt;
  return *best;
}

bool Database::load(const std::string &path, std::vector<LoadWarning> &warnings) {
  std::ifstream fh(path);
  if (!fh) return !std::filesystem::exists(path);
  std::string line;
  std::size_t n = 0;
  while (std::getline(fh, line)) {
    ++n;
    if (line.find_first_not_of(" \t\r") == std::string::npos) continue;
    json::Value v;
    std::string err;
    Record r;
    if (!json::Value::parse(line, &v, &err) || !record_from_json(v, &r, &err)) {
      warnings.push_back({n, err});
      continue;
    }
    records_.push_back(std::move(r));
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
