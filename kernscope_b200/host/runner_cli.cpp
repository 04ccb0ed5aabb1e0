// runner_cli.cpp -- ks-template-runner: run ONE kernel of a family on raw
// host buffers (the gate runner of the reference's template flow,
// kernels/templates/tools/hip_template_runner.cpp, consumed by
// kernels/templates/tests/run_hip_gate.py).
//
//   ks-template-runner --family <f> [--kernel <symbol>] [--causal] [--gelu erf|tanh]
//       [--grid <W>[x<H>]] [--block <X>[x<Y>]]
//       [--in <raw.bin>]... --out <out.bin> --out-size <bytes> [--int <i32>]...
//
// Same flags as the reference runner with --family in place of --hsaco: on
// B200 every config is a prebuilt instantiation, so the kernel symbol (as
// kernel_symbol() names it, e.g. kernscope_b200_softmax_b256_v8_onepass)
// selects the config; without --kernel the family's default config runs.
// --grid / --block are accepted for compatibility and ignored (the launch
// geometry follows from the config).  So that the reference's gate script
// can drive this runner unchanged, --hsaco is accepted and ignored too, and
// without --family the family is read from the symbol's prefix
// (kernscope_b200_<family>_...).  Inputs and output are raw row-major
// bf16 buffers and the --int scalars come in the reference's order:
//
//   softmax    (x)            -> out   ints rows, cols
//   layernorm  (x, gamma, beta) -> out ints rows, cols     (eps 1e-5)
//   bias_gelu  (x, bias)      -> out   ints total, cols
//   reduction  (x)            -> out   ints rows, cols     (axis-0 sum, bf16)
//   matmul     (a, b)         -> out   ints m, n, k
//   attention  (q, k, v)      -> out   ints nq, nk, d      (one head)
//
// Exit codes: 0 ok; 1 the run failed (message names the failing step); 2
// usage error.  No silent skips.
#include <cstdint>
#include <cstdio>
#include <exception>
#include <cstdlib>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

#include "families.h"
#include "kernscope_b200.h"

namespace {

using kernscope::tune::json;

struct Options {
  std::string family, kernel, gelu = "erf", out;
  bool causal = false;
  std::vector<std::string> inputs;
  std::size_t out_size = 0;
  std::vector<std::int64_t> ints;
};

int usage(const char *msg) {
  if (msg) std::fprintf(stderr, "ks-template-runner: %s\n", msg);
  std::fprintf(stderr,
               "usage: ks-template-runner [--family <softmax|layernorm|bias_gelu|reduction|matmul|attention>]\n"
               "       [--kernel <symbol>] [--causal] [--gelu erf|tanh] [--grid <W[xH]>] [--block <X[xY]>]\n"
               "       [--in <bin>]... --out <bin> --out-size <bytes> [--int <i32>]...\n");
  return 2;
}

// The runner's family name for a symbol kernscope_b200_<family>_..., or "".
std::string family_of_symbol(const std::string &sym) {
  const std::string pre = "kernscope_b200_";
  if (sym.compare(0, pre.size(), pre) != 0) return "";
  const std::string rest = sym.substr(pre.size());
  static const std::pair<const char *, const char *> names[] = {
      {"flash_attention_", "attention"}, {"bias_gelu_", "bias_gelu"}, {"layernorm_", "layernorm"},
      {"softmax_", "softmax"},           {"reduction_", "reduction"}, {"matmul_", "matmul"}};
  for (const auto &[prefix, fam] : names)
    if (rest.compare(0, std::string(prefix).size(), prefix) == 0) return fam;
  return "";
}

int fail(const std::string &what, int status) {
  std::fprintf(stderr, "ks-template-runner: %s: %s\n", what.c_str(), ks_status_string(status));
  return 1;
}

bool read_file(const std::string &path, std::vector<unsigned char> *out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  out->assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  return true;
}

struct Dev {
  void *p = nullptr;
  ~Dev() {
    if (p) ks_gpu_free(p);
  }
};

int iget(const json &c, const char *k, int dflt) {
  const json *v = c.find(k);
  return v ? int(v->as_number()) : dflt;
}

int mode_of(const json &c) {
  const json *v = c.find("mode");
  if (!v) return KS_MODE_ONEPASS;
  const std::string m = v->as_string();
  return m == "twopass" ? KS_MODE_TWOPASS : m == "strided" ? KS_MODE_STRIDED : m == "tree" ? KS_MODE_TREE
       : m == "staged" ? KS_MODE_STAGED : KS_MODE_ONEPASS;
}

// The tuner's name of a family (+ variant) and its shape from the scalars.
bool tuner_view(const Options &o, std::string *fam, std::vector<std::int64_t> *shape) {
  const auto &i = o.ints;
  if (o.family == "softmax" || o.family == "layernorm" || o.family == "reduction") {
    if (i.size() != 2) return false;
    *fam = o.family;
    *shape = {i[0], i[1]};
  } else if (o.family == "bias_gelu") {
    if (i.size() != 2 || i[1] <= 0) return false;
    *fam = o.gelu == "tanh" ? "bias_gelu:tanh" : "bias_gelu";
    *shape = {(i[0] + i[1] - 1) / i[1], i[1]};
  } else if (o.family == "matmul") {
    if (i.size() != 3) return false;
    *fam = "matmul";
    *shape = {i[0], i[1], i[2]};
  } else if (o.family == "attention" || o.family == "flash_attention") {
    if (i.size() != 3) return false;
    *fam = o.causal ? "flash_attention:causal" : "flash_attention";
    *shape = {i[0], i[1], i[2]};
  } else {
    return false;
  }
  return true;
}

}  // namespace

static int run_main(int argc, char **argv) {
  Options o;
  for (int a = 1; a < argc; ++a) {
    const std::string s = argv[a];
    auto val = [&]() -> const char * { return a + 1 < argc ? argv[++a] : nullptr; };
    const char *v = nullptr;
    if (s == "--causal") {
      o.causal = true;
    } else if (s == "--family" || s == "--kernel" || s == "--gelu" || s == "--out" || s == "--in" ||
               s == "--out-size" || s == "--int" || s == "--grid" || s == "--block" || s == "--hsaco") {
      if (!(v = val())) return usage(("missing value for " + s).c_str());
      if (s == "--family") o.family = v;
      if (s == "--kernel") o.kernel = v;
      if (s == "--gelu") o.gelu = v;
      if (s == "--out") o.out = v;
      if (s == "--in") o.inputs.push_back(v);
      if (s == "--out-size") o.out_size = std::size_t(std::strtoull(v, nullptr, 10));
      if (s == "--int") o.ints.push_back(std::strtoll(v, nullptr, 10));
      // --hsaco: the HIP module path of the reference runner; nothing to load here
    } else {
      return usage(("unknown argument " + s).c_str());
    }
  }
  if (o.family.empty()) o.family = family_of_symbol(o.kernel);
  if (o.family.empty() || o.out.empty() || o.out_size == 0)
    return usage("--family (or a kernscope_b200_<family>_ --kernel symbol), --out and --out-size are required");
  if (o.gelu != "erf" && o.gelu != "tanh") return usage("--gelu must be erf or tanh");
  // the symbol names the variant of the families that have one
  if (o.kernel.find("_causal") != std::string::npos) o.causal = true;
  if (o.kernel.size() > 5 && o.kernel.compare(o.kernel.size() - 5, 5, "_tanh") == 0) o.gelu = "tanh";
  std::string fam_name;
  std::vector<std::int64_t> shape;
  if (!tuner_view(o, &fam_name, &shape)) return usage("unknown family or wrong number of --int scalars");
  const kernscope::tune::Family *fam = kernscope::tune::find_family(fam_name);
  if (!fam) return usage(("no tuner family " + fam_name).c_str());
  std::string reason;
  if (!fam->check_shape(shape, &reason)) return usage(reason.c_str());

  // the config: the one whose symbol is --kernel, else the first valid auto config
  json cfg;
  bool found = false;
  for (bool full : {false, true}) {
    for (const json &c : fam->enumerate(full, shape)) {
      if (!o.kernel.empty() ? fam->symbol(c) == o.kernel : fam->validate(c, shape, "sm_100a").valid) {
        cfg = c;
        found = true;
        break;
      }
    }
    if (found) break;
  }
  if (!found) return usage(o.kernel.empty() ? "no valid config for this shape" : ("unknown kernel symbol " + o.kernel).c_str());

  int n = 0;
  if (ks_gpu_device_count(&n) != KS_OK || n == 0) {
    std::fprintf(stderr, "ks-template-runner: no CUDA device\n");
    return 1;
  }
  // inputs to the device
  std::vector<Dev> din(o.inputs.size());
  for (std::size_t k = 0; k < o.inputs.size(); ++k) {
    std::vector<unsigned char> bytes;
    if (!read_file(o.inputs[k], &bytes) || bytes.empty()) {
      std::fprintf(stderr, "ks-template-runner: cannot read --in %s\n", o.inputs[k].c_str());
      return 1;
    }
    if (int s = ks_gpu_malloc(&din[k].p, bytes.size()); s != KS_OK) return fail("malloc", s);
    if (int s = ks_gpu_memcpy_htod(din[k].p, bytes.data(), bytes.size(), nullptr); s != KS_OK) return fail("htod", s);
  }
  Dev dout, ws;
  if (int s = ks_gpu_malloc(&dout.p, o.out_size); s != KS_OK) return fail("malloc out", s);
  auto need = [&](std::size_t k) { return din.size() == k; };
  const auto &i = o.ints;
  int st = KS_OK;
  const std::string f = o.family == "attention" ? "flash_attention" : o.family;
  if (f == "softmax") {
    if (!need(1)) return usage("softmax takes one --in (x)");
    ks_softmax_config c{iget(cfg, "block", 256), iget(cfg, "vec_width", 8), mode_of(cfg)};
    ks_softmax_args a{din[0].p, dout.p, i[0], i[1]};
    st = ks_softmax_launch(&c, &a, nullptr);
  } else if (f == "layernorm") {
    if (!need(3)) return usage("layernorm takes three --in (x, gamma, beta)");
    ks_layernorm_config c{iget(cfg, "block", 128), iget(cfg, "vec_width", 8), mode_of(cfg)};
    ks_layernorm_args a{din[0].p, din[1].p, din[2].p, dout.p, i[0], i[1], 0.f};
    st = ks_layernorm_launch(&c, &a, nullptr);
  } else if (f == "bias_gelu") {
    if (!need(2)) return usage("bias_gelu takes two --in (x, bias)");
    ks_bias_gelu_config c{iget(cfg, "block", 128), iget(cfg, "vec_width", 8),
                          o.gelu == "tanh" ? KS_GELU_TANH : KS_GELU_ERF};
    ks_bias_gelu_args a{din[0].p, din[1].p, dout.p, i[0], i[1]};
    st = ks_bias_gelu_launch(&c, &a, nullptr);
  } else if (f == "reduction") {
    if (!need(1)) return usage("reduction takes one --in (x)");
    ks_reduction_config c{iget(cfg, "block", 256), iget(cfg, "vec_width", 1), mode_of(cfg)};
    ks_reduction_args a{din[0].p, dout.p, i[0], i[1], KS_BF16, KS_BF16, 0, nullptr, 0, nullptr};
    std::size_t wsb = 0;
    if ((st = ks_reduction_workspace_bytes(&c, &a, &wsb)) != KS_OK) return fail("workspace size", st);
    if (wsb && (st = ks_gpu_malloc(&ws.p, wsb)) != KS_OK) return fail("malloc workspace", st);
    a.workspace = ws.p;
    a.workspace_bytes = wsb;
    st = ks_reduction_launch(&c, &a, nullptr);
  } else if (f == "matmul") {
    if (!need(2)) return usage("matmul takes two --in (a, b)");
    ks_matmul_config c{iget(cfg, "tile_m", 128), iget(cfg, "tile_n", 256), iget(cfg, "tile_k", 64),
                       iget(cfg, "stages", 4), iget(cfg, "acc_stages", 2), iget(cfg, "group_m", 8),
                       iget(cfg, "cta_group", 0)};
    ks_matmul_args a{din[0].p, din[1].p, dout.p, i[0], i[1], i[2]};
    st = ks_matmul_launch(&c, &a, nullptr);
  } else {
    if (!need(3)) return usage("attention takes three --in (q, k, v)");
    ks_flash_attention_config c{iget(cfg, "tile_m", 256), iget(cfg, "tile_n", 128), iget(cfg, "stages", 2),
                                o.causal ? 1 : 0};
    ks_flash_attention_args a{din[0].p, din[1].p, din[2].p, dout.p, 1, 1, i[0], i[1], i[2], 0.f};
    st = ks_flash_attention_launch(&c, &a, nullptr);
  }
  if (st != KS_OK) return fail("launch " + fam->symbol(cfg), st);
  if ((st = ks_gpu_synchronize()) != KS_OK) return fail("synchronize", st);
  int word = 0;
  if ((st = ks_device_error_take(&word)) != KS_OK || word != 0) {
    std::fprintf(stderr, "ks-template-runner: device error word %d\n", word);
    return 1;
  }
  std::vector<unsigned char> host(o.out_size);
  if ((st = ks_gpu_memcpy_dtoh(host.data(), dout.p, o.out_size, nullptr)) != KS_OK) return fail("dtoh", st);
  if ((st = ks_gpu_synchronize()) != KS_OK) return fail("synchronize", st);
  std::ofstream of(o.out, std::ios::binary);
  of.write(reinterpret_cast<const char *>(host.data()), std::streamsize(host.size()));
  if (!of) {
    std::fprintf(stderr, "ks-template-runner: cannot write --out %s\n", o.out.c_str());
    return 1;
  }
  std::printf("ran %s (%s) -> %s (%zu bytes)\n", fam->symbol(cfg).c_str(), cfg.dump().c_str(), o.out.c_str(),
              o.out_size);
  return 0;
}

// An exception from the library ends the tool with an error status and its
// message instead of std::terminate.
int main(int argc, char **argv) {
  try {
    return run_main(argc, argv);
  } catch (const std::exception &e) {
    std::fprintf(stderr, "ks-template-runner: internal error: %s\n", e.what());
  } catch (...) {
    std::fprintf(stderr, "ks-template-runner: internal error\n");
  }
  return 1;
}
