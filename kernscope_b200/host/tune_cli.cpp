// tune_cli.cpp -- kernscope-tune for B200 (the reference's
// tools/tune/src/tune_cli.cpp:66-90, 917-1166): same flags, same outputs
// (--json evidence, --text table, --html table) and exit codes (0 best
// selected, 1 no viable config, 2 usage / device / internal error).
// --arch auto resolves from the current device (compute capability 10.0 ->
// sm_100a).  The LLVM verifier gate (--verify / --inject-risky) is not part
// of this build: those flags are reported as unsupported (exit 2).
#include <cstdio>
#include <exception>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "driver.h"
#include "json.h"
#include "kernscope_b200.h"

namespace {

void usage(const char *argv0) {
  std::fprintf(stderr,
               "usage: %s --kernel <family> --shape <M,N,K|R,C|N|Nq,Nk,d|B,H,N,d>\n"
               "              [--arch <auto|sm_100a>] [--grid <auto|full>] [--gate-shape <csv>]\n"
               "              [--json|--text|--html] [--db <path>] [--cache <path>] [--workdir <dir>]\n"
               "              [--min-occupancy <f>] [--no-bench] [--no-cache|--force]\n"
               "              [--causal] [--gelu <erf|tanh>] [--device <n>] [--emit-repro <dir>] [--version]\n"
               "  family: matmul | bias_gelu | softmax | layernorm | reduction | flash_attention\n"
               "  --no-cache skips the tunecache READ but still writes the cache\n"
               "  --emit-repro <dir> writes repro.cpp + run.sh + README.md for the winning config\n",
               argv0);
}

bool parse_shape(const std::string &s, std::vector<std::int64_t> *out) {
  out->clear();
  size_t pos = 0;
  while (pos <= s.size()) {
    const size_t comma = s.find(',', pos);
    const std::string tok = s.substr(pos, comma == std::string::npos ? std::string::npos : comma - pos);
    char *end = nullptr;
    const long long v = std::strtoll(tok.c_str(), &end, 10);
    if (tok.empty() || !end || *end != '\0' || v <= 0) return false;
    out->push_back(v);
    if (comma == std::string::npos) break;
    pos = comma + 1;
  }
  return !out->empty();
}

void print_text(const kernscope::db::json::Value &ev) {
  using kernscope::db::json::Value;
  std::printf("kernscope-tune  family=%s  arch=%s  status=%s\n", ev.string_or("kernel_family", "").c_str(),
              ev.string_or("gpu_arch", "").c_str(), ev.string_or("status", "").c_str());
  std::printf("%s\n", ev.string_or("message", "").c_str());
  if (const Value *s = ev.find("summary"))
    std::printf("variants %d  prescreen-rejected %d  golden-failed %d  benchmarked %d  cached %d\n",
                int(s->number_or("variants_total", 0)), int(s->number_or("prescreen_rejected", 0)),
                int(s->number_or("golden_gate_failed", 0)), int(s->number_or("benchmarked", 0)),
                int(s->number_or("cached", 0)));
  if (const Value *vs = ev.find("variants"))
    for (const Value &v : vs->as_array()) {
      const Value *t = v.find("timings");
      std::printf("  %c %-52s %-20s %10s\n", v.find("best") && v.find("best")->as_bool() ? '*' : ' ',
                  v.string_or("symbol", "").c_str(), v.string_or("status", "").c_str(),
                  t ? (std::to_string(t->number_or("median", 0) * 1000.0).substr(0, 9) + "us").c_str() : "");
    }
}

void print_html(const kernscope::db::json::Value &ev) {
  using kernscope::db::json::Value;
  std::printf("<!doctype html><html><head><meta charset=\"utf-8\"><title>kernscope-tune %s</title></head><body>\n",
              ev.string_or("kernel_family", "").c_str());
  std::printf("<h1>kernscope-tune: %s on %s</h1><p>%s</p>\n<table border=\"1\"><tr><th>best</th><th>symbol</th>"
              "<th>status</th><th>median ms</th><th>reason</th></tr>\n",
              ev.string_or("kernel_family", "").c_str(), ev.string_or("gpu_arch", "").c_str(),
              ev.string_or("message", "").c_str());
  if (const Value *vs = ev.find("variants"))
    for (const Value &v : vs->as_array()) {
      const Value *t = v.find("timings");
      std::printf("<tr><td>%s</td><td>%s</td><td>%s</td><td>%s</td><td>%s</td></tr>\n",
                  v.find("best") && v.find("best")->as_bool() ? "*" : "", v.string_or("symbol", "").c_str(),
                  v.string_or("status", "").c_str(), t ? std::to_string(t->number_or("median", 0)).c_str() : "",
                  v.string_or("reason", "").c_str());
    }
  std::printf("</table><pre>%s</pre></body></html>\n", ev.dump().c_str());
}

}  // namespace

static int run_main(int argc, char **argv) {
  kernscope::tune::DriverOptions o;
  std::string mode = "json", repro, shape_s;
  bool have_kernel = false, have_shape = false;
  o.arch = "auto";
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto next = [&](std::string *v) {
      if (i + 1 >= argc) return false;
      *v = argv[++i];
      return true;
    };
    std::string v;
    if (a == "--kernel" && next(&v)) {
      o.kernel_family = v;
      have_kernel = true;
    } else if (a == "--shape" && next(&v)) {
      shape_s = v;
      have_shape = parse_shape(v, &o.shape);
    } else if (a == "--arch" && next(&v)) {
      o.arch = v;
    } else if (a == "--grid" && next(&v)) {
      o.grid_preset = v;
    } else if (a == "--gate-shape" && next(&v)) {
      if (!parse_shape(v, &o.gate_shape)) {
        std::fprintf(stderr, "kernscope-tune: bad --gate-shape '%s'\n", v.c_str());
        return 2;
      }
    } else if (a == "--json") {
      mode = "json";
    } else if (a == "--text") {
      mode = "text";
    } else if (a == "--html") {
      mode = "html";
    } else if (a == "--db" && next(&v)) {
      o.db_path = v;
    } else if (a == "--cache" && next(&v)) {
      o.cache_path = v;
    } else if (a == "--workdir" && next(&v)) {
      o.workdir = v;
    } else if (a == "--min-occupancy" && next(&v)) {
      char *end = nullptr;
      o.min_occupancy = std::strtod(v.c_str(), &end);
      if (!end || *end || o.min_occupancy < 0) {
        std::fprintf(stderr, "kernscope-tune: bad --min-occupancy '%s'\n", v.c_str());
        return 2;
      }
    } else if (a == "--no-bench") {
      o.live_bench = false;
    } else if (a == "--no-cache" || a == "--force") {
      o.use_cache = false;
    } else if (a == "--causal") {
      o.causal = true;
    } else if (a == "--gelu" && next(&v)) {
      o.gelu = v;
    } else if (a == "--device" && next(&v)) {
      o.device = std::atoi(v.c_str());
    } else if (a == "--emit-repro" && next(&v)) {
      repro = v;
    } else if (a == "--verify" || a == "--inject-risky") {
      std::fprintf(stderr, "kernscope-tune: %s needs the LLVM verifier, which this build does not include\n", a.c_str());
      return 2;
    } else if (a == "--version") {
      std::printf("%s (ABI %d, %s)\n", kernscope::tune::kToolVersion, ks_abi_version(), ks_build_info());
      return 0;
    } else if (a == "-h" || a == "--help") {
      usage(argv[0]);
      return 0;
    } else {
      std::fprintf(stderr, "kernscope-tune: unknown or incomplete argument '%s'\n", a.c_str());
      usage(argv[0]);
      return 2;
    }
  }
  if (!have_kernel || !have_shape) {
    usage(argv[0]);
    return 2;
  }
  if (o.arch == "auto") {
    char buf[32] = {0};
    int n = 0;
    if (ks_gpu_device_count(&n) != KS_OK || n <= o.device || ks_gpu_arch(o.device, buf, sizeof(buf)) != KS_OK) {
      std::fprintf(stderr, "kernscope-tune: --arch auto needs a visible GPU; pass --arch sm_100a for a pre-screen\n");
      return 2;
    }
    o.arch = buf;
  }
  const std::string hash = kernscope::tune::make_shape_hash(o.kernel_family, o.shape);
  if (o.db_path.empty()) o.db_path = "reports/tune/" + o.kernel_family + "-" + hash.substr(8) + ".jsonl";
  if (o.cache_path.empty()) o.cache_path = o.db_path + ".tunecache.json";

  kernscope::tune::DriverResult r = kernscope::tune::tune(o);
  kernscope::db::json::Value ev;
  if (r.evidence_json.empty() || !kernscope::db::json::Value::parse(r.evidence_json, &ev, nullptr)) {
    std::fprintf(stderr, "kernscope-tune: %s: %s\n", kernscope::tune::driver_status_name(r.status), r.message.c_str());
  } else if (mode == "html") {
    print_html(ev);
  } else if (mode == "text") {
    print_text(ev);
  } else {
    std::printf("%s\n", r.evidence_json.c_str());
  }
  if (!repro.empty()) {
    std::string err;
    if (!kernscope::tune::emit_repro(o, r, repro, &err)) std::fprintf(stderr, "kernscope-tune: %s\n", err.c_str());
  }
  switch (r.status) {
    case kernscope::tune::DriverStatus::kOk: return 0;
    case kernscope::tune::DriverStatus::kNoViableConfig: return 1;
    default: return 2;
  }
}

// An exception from the library ends the tool with an error status and its
// message instead of std::terminate.
int main(int argc, char **argv) {
  try {
    return run_main(argc, argv);
  } catch (const std::exception &e) {
    std::fprintf(stderr, "kernscope-tune: internal error: %s\n", e.what());
  } catch (...) {
    std::fprintf(stderr, "kernscope-tune: internal error\n");
  }
  return 2;
}
