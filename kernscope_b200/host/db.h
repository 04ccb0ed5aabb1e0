// db.h -- the JSONL record store of measured configs (the reference's libs/db,
// libs/db/include/kernscope/db.h:137-198): one JSON object per line,
//   {schema_version, gpu_arch, kernel_family, shape_hash, config,
//    timings{median,p20,p80}, provenance{timestamp,tool_version,mode}},
// keyed (gpu_arch, kernel_family, shape_hash); query_best returns the
// record with the smallest median.
#pragma once

#include <compare>
#include <map>
#include <optional>
#include <string>
#include <string_view>
#include <vector>

#include "json.h"

namespace kernscope::db {

inline constexpr int kCurrentSchemaVersion = 1;

struct Timings {
  double median = 0.0;
  double p20 = 0.0;
  double p80 = 0.0;
};

struct Provenance {
  std::string timestamp;     // ISO-8601 UTC
  std::string tool_version;  // producer tool version
  std::string mode;          // "measured" | "projected"
};

struct Record {
  int schema_version = kCurrentSchemaVersion;
  std::string gpu_arch;
  std::string kernel_family;
  std::string shape_hash;
  json::Value config;
  Timings timings;
  Provenance provenance;
};

struct LoadWarning {
  std::size_t line = 0;
  std::string message;
};

json::Value record_to_json(const Record &r);
bool record_from_json(const json::Value &v, Record *out, std::string *error);

class Database {
 public:
  // Inserts `record`, or replaces in place the record with the same
  // (gpu_arch, kernel_family, shape_hash, canonical config) key. Throws
  // std::invalid_argument for a non-object config or non-finite numbers.
  void put(Record record);
  // The record with the smallest timings.median among those sharing
  // (gpu_arch, kernel_family, shape_hash); a tie keeps the smallest
  // canonical config. std::nullopt when none match.
  std::optional<Record> query_best(std::string_view gpu_arch, std::string_view kernel_family,
                                   std::string_view shape_hash) const;
  // Merges the records of `path` through put(). Blank lines are skipped;
  // a malformed or rejected line becomes a warning naming its 1-based line
  // and is skipped. Returns false only when the file cannot be opened.
  bool load(const std::string &path, std::vector<LoadWarning> &warnings);
  bool save(const std::string &path) const;
  std::size_t size() const { return records_.size(); }
  const std::vector<Record> &records() const { return records_; }

 private:
  struct Key {
    std::string gpu_arch, kernel_family, shape_hash, config;
    auto operator<=>(const Key &) const = default;
  };
  static Key make_key(const Record &r);
  std::vector<Record> records_;        // insertion order
  std::map<Key, std::size_t> index_;   // key -> position in records_
};

// Current UTC time as ISO-8601 ("2026-12-01T20:00:00Z").
std::string utc_timestamp();

}  // namespace kernscope::db
