// Test infrastructure only: a command-line checker linked against the
// reference tuner's own host sources (compiled in place by the Makefile next
// to this file; nothing of the reference is copied here). The CPU tests run
// it beside this repository's tuner and compare the answers, which pins the
// tuner's host logic to the reference itself rather than to a restatement.
//
// Every command prints one JSON object on stdout.
//   hash <family> <d0,d1,...> [arch]   make_shape_hash + make_cache_key
//                                      (tools/tune/include/kernscope/tune/driver.h:186-193)
//   db <path.jsonl>                    Database::load + query_best for every
//                                      workload key in the file
//                                      (libs/db/include/kernscope/db.h:172-198)
//   roofline <family> m n k d bytes    compute_flops + compute_bytes_moved
//                                      (libs/roofline/include/kernscope/roofline.h:125-131)
//   occupancy <arch> regs smem block   compute_occupancy
//                                      (libs/occupancy/include/kernscope/occupancy.h:85-87)
//   quantile <q> <s0,s1,...>           bench::quantile (libs/bench/include/kernscope/bench.h:105)
//   gen <family> <arch> <shape> <out.cu|-> key=value...
//                                      validate_config + launch_geometry +
//                                      kernel_symbol + generate_to_file of the
//                                      family's generator (tools/tune/include/
//                                      kernscope/tune/*_gen.h); "-" skips the file
#include "kernscope/arch.h"
#include "kernscope/bench.h"
#include "kernscope/db.h"
#include "kernscope/occupancy.h"
#include "kernscope/roofline.h"
#include "kernscope/tune/driver.h"
#include "ref_gen.h"

#include <cstdio>
#include <cstdlib>
#include <set>
#include <sstream>
#include <string>
#include <tuple>
#include <vector>

namespace json = kernscope::db::json;

namespace {

std::vector<std::string> split(const std::string &s, char sep) {
  std::vector<std::string> out;
  std::stringstream ss(s);
  std::string item;
  while (std::getline(ss, item, sep))
    if (!item.empty()) out.push_back(item);
  return out;
}

int usage() {
  std::fprintf(stderr,
               "usage: ref_tune_check hash <family> <dims> [arch] | db <path> | "
               "roofline <family> m n k d dtype_bytes | occupancy <arch> regs smem block | "
               "quantile <q> <samples> | gen <family> <arch> <shape> <out|-> key=value...\n");
  return 2;
}

bool family_of(const std::string &name, kernscope::roofline::KernelFamily *f) {
  using K = kernscope::roofline::KernelFamily;
  const std::pair<const char *, K> table[] = {
      {"matmul", K::kGemm},       {"bias_gelu", K::kFusedBiasGelu}, {"softmax", K::kSoftmax},
      {"layernorm", K::kLayerNorm}, {"reduction", K::kReduction},    {"flash_attention", K::kFlashAttention}};
  for (const auto &[n, k] : table)
    if (name == n) {
      *f = k;
      return true;
    }
  return false;
}

int cmd_hash(int argc, char **argv) {
  if (argc < 4) return usage();
  std::vector<std::int64_t> dims;
  for (const auto &t : split(argv[3], ',')) dims.push_back(std::strtoll(t.c_str(), nullptr, 10));
  const std::string arch = argc > 4 ? argv[4] : "sm_100a";
  const std::string h = kernscope::tune::make_shape_hash(argv[2], dims);
  const json::Value v = json::object({{"shape_hash", json::Value(h)},
                                      {"cache_key", json::Value(kernscope::tune::make_cache_key(arch, argv[2], h))}});
  std::printf("%s\n", v.dump().c_str());
  return 0;
}

int cmd_db(int argc, char **argv) {
  if (argc < 3) return usage();
  kernscope::db::Database d;
  std::vector<kernscope::db::LoadWarning> warnings;
  const bool opened = d.load(argv[2], warnings);
  std::vector<json::Value> warn;
  for (const auto &w : warnings) warn.push_back(json::Value(w.message));
  std::vector<json::Value> best;
  std::set<std::tuple<std::string, std::string, std::string>> seen;
  for (const auto &r : d.records()) {
    if (!seen.insert({r.gpu_arch, r.kernel_family, r.shape_hash}).second) continue;
    const auto b = d.query_best(r.gpu_arch, r.kernel_family, r.shape_hash);
    if (!b) continue;
    best.push_back(json::object({{"gpu_arch", json::Value(b->gpu_arch)},
                                 {"kernel_family", json::Value(b->kernel_family)},
                                 {"shape_hash", json::Value(b->shape_hash)},
                                 {"config", b->config},
                                 {"median", json::Value(b->timings.median)}}));
  }
  const json::Value v = json::object({{"opened", json::Value(opened)},
                                      {"records", json::Value(static_cast<double>(d.size()))},
                                      {"warnings", json::Value(warn)},
                                      {"best", json::Value(best)}});
  std::printf("%s\n", v.dump().c_str());
  return 0;
}

int cmd_roofline(int argc, char **argv) {
  if (argc < 8) return usage();
  kernscope::roofline::KernelFamily f;
  if (!family_of(argv[2], &f)) return usage();
  kernscope::roofline::Shape s;
  s.m = std::strtoll(argv[3], nullptr, 10);
  s.n = std::strtoll(argv[4], nullptr, 10);
  s.k = std::strtoll(argv[5], nullptr, 10);
  s.d = std::strtoll(argv[6], nullptr, 10);
  s.dtype_bytes = std::atoi(argv[7]);
  const json::Value v =
      json::object({{"flops", json::Value(static_cast<double>(kernscope::roofline::compute_flops(f, s)))},
                    {"bytes", json::Value(static_cast<double>(kernscope::roofline::compute_bytes_moved(f, s)))}});
  std::printf("%s\n", v.dump().c_str());
  return 0;
}

int cmd_occupancy(int argc, char **argv) {
  if (argc < 6) return usage();
  if (!kernscope::has_arch(argv[2])) return usage();
  const auto r = kernscope::occupancy::compute_occupancy(kernscope::get_arch(argv[2]), std::atoi(argv[3]),
                                                         std::atoi(argv[4]), std::atoi(argv[5]));
  const json::Value v = json::object({{"blocks_per_sm", json::Value(r.blocks_per_sm)},
                                      {"warps_resident", json::Value(r.warps_resident)},
                                      {"occupancy", json::Value(r.occupancy)},
                                      {"limiter", json::Value(kernscope::occupancy::limiter_name(r.limiter))}});
  std::printf("%s\n", v.dump().c_str());
  return 0;
}

int cmd_quantile(int argc, char **argv) {
  if (argc < 4) return usage();
  std::vector<double> s;
  for (const auto &t : split(argv[3], ',')) s.push_back(std::strtod(t.c_str(), nullptr));
  const json::Value v = json::object({{"q", json::Value(kernscope::bench::quantile(s, std::strtod(argv[2], nullptr)))}});
  std::printf("%s\n", v.dump().c_str());
  return 0;
}

int cmd_gen(int argc, char **argv) {
  if (argc < 6) return usage();
  const std::string family = argv[2], arch = argv[3], out = std::string(argv[5]) == "-" ? "" : argv[5];
  std::vector<std::int64_t> shape;
  for (const auto &t : split(argv[4], ',')) shape.push_back(std::strtoll(t.c_str(), nullptr, 10));
  RefCfg cfg;
  for (int i = 6; i < argc; ++i) {
    const std::string kv = argv[i];
    const auto eq = kv.find('=');
    if (eq == std::string::npos) return usage();
    cfg[kv.substr(0, eq)] = kv.substr(eq + 1);
  }
  RefGen g;
  std::string err;
  bool ok;
  if (family == "matmul") ok = ref_gen_matmul(arch, shape, cfg, out, &g, &err);
  else if (family == "flash_attention") ok = ref_gen_flash(arch, shape, cfg, out, &g, &err);
  else ok = ref_gen_elem(family, arch, shape, cfg, out, &g, &err);
  if (!ok) {
    std::fprintf(stderr, "ref_tune_check gen: %s\n", err.c_str());
    return 1;
  }
  const json::Value v = json::object({{"valid", json::Value(g.valid)},
                                      {"reason", json::Value(g.reason)},
                                      {"symbol", json::Value(g.symbol)},
                                      {"grid", json::array({json::Value(g.grid_x), json::Value(g.grid_y)})},
                                      {"block", json::array({json::Value(g.block_x), json::Value(g.block_y)})},
                                      {"smem_bytes", json::Value(static_cast<double>(g.smem_bytes))}});
  std::printf("%s\n", v.dump().c_str());
  return 0;
}

}  // namespace

int main(int argc, char **argv) {
  if (argc < 2) return usage();
  const std::string cmd = argv[1];
  if (cmd == "hash") return cmd_hash(argc, argv);
  if (cmd == "db") return cmd_db(argc, argv);
  if (cmd == "roofline") return cmd_roofline(argc, argv);
  if (cmd == "occupancy") return cmd_occupancy(argc, argv);
  if (cmd == "quantile") return cmd_quantile(argc, argv);
  if (cmd == "gen") return cmd_gen(argc, argv);
  return usage();
}
