// families.cpp -- config spaces, validation, sessions and gate references of
// the six kernel families.
#include "families.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <sstream>

#include "golden.h"
#include "hwmodel.h"

namespace kernscope::tune {

// ---------------------------------------------------------------------------
// bf16, seeded inputs, device buffers
// ---------------------------------------------------------------------------
std::uint16_t f32_to_bf16(float f) { return golden::to_bf16_bits(f); }
float bf16_to_f32(std::uint16_t h) { return golden::from_bf16_bits(h); }

namespace {

// bf16 tensor with host copy (bf16 bits + fp32 view) and a device copy
struct DevBuf {
  void *p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf &) = delete;
  DevBuf &operator=(const DevBuf &) = delete;
  ~DevBuf() {
    if (p) ks_gpu_free(p);
  }
  int alloc(size_t n) {
    bytes = n;
    return ks_gpu_malloc(&p, n < 256 ? 256 : n);
  }
};

// The next n draws of the reference profile's uniform(lo, hi), rounded to
// bf16 (inputs.py:73-106 through golden::draw_bf16), with an fp32 view.
struct HostBf16 {
  std::vector<std::uint16_t> bits;
  std::vector<float> f;
  void fill_uniform(golden::Generator &g, size_t n, double lo, double hi) {
    set_bits(golden::draw_bf16(g, n, lo, hi));
  }
  void set_bits(std::vector<std::uint16_t> b) {
    bits = std::move(b);
    f.resize(bits.size());
    for (size_t i = 0; i < bits.size(); ++i) f[i] = bf16_to_f32(bits[i]);
  }
};

// A session's host inputs by the reference's names (inputs.py keys).
using NamedInputs = std::vector<std::pair<const char *, HostBf16 *>>;

int upload(DevBuf &d, const void *src, size_t bytes) {
  int s = d.alloc(bytes);
  if (s == KS_OK && bytes > 0) s = ks_gpu_memcpy_htod(d.p, src, bytes, nullptr);
  if (s == KS_OK) s = ks_gpu_synchronize();
  return s;
}

int download_bf16(const DevBuf &d, size_t n, std::vector<float> *out) {
  std::vector<std::uint16_t> h(n);
  int s = ks_gpu_memcpy_dtoh(h.data(), d.p, n * 2, nullptr);
  if (s == KS_OK) s = ks_gpu_synchronize();
  out->resize(n);
  for (size_t i = 0; i < n; ++i) (*out)[i] = bf16_to_f32(h[i]);
  return s;
}

int iget(const json &c, const char *k, int d) { return int(c.number_or(k, d)); }

// SMs of the current device, as the launches see them (ks_gpu_sm_count); the
// sm_100a model's count when no device answers (pre-screen without a GPU).
std::int64_t device_sms() {
  int dev = 0, n = 0;
  if (ks_gpu_get_device(&dev) == KS_OK && ks_gpu_sm_count(dev, &n) == KS_OK && n > 0) return n;
  return get_arch("sm_100a").sm_count;
}

std::string shape_str(const std::vector<std::int64_t> &s) {
  std::string o;
  for (size_t i = 0; i < s.size(); ++i) o += (i ? "," : "") + std::to_string(s[i]);
  return o;
}

bool valid_elem_shape(const std::vector<std::int64_t> &s, std::string *r, const char *fam) {
  if (s.size() != 2 || s[0] <= 0 || s[1] <= 0) {
    if (r) *r = std::string(fam) + " expects --shape R,C (positive)";
    return false;
  }
  return true;
}

int mode_from(const json &c, int dflt) {
  const std::string s = c.string_or("mode", "");
  if (s == "onepass") return KS_MODE_ONEPASS;
  if (s == "twopass") return KS_MODE_TWOPASS;
  if (s == "strided") return KS_MODE_STRIDED;
  if (s == "tree") return KS_MODE_TREE;
  if (s == "staged") return KS_MODE_STAGED;
  if (s == "cluster") return KS_MODE_CLUSTER;
  return dflt;
}

// CTAs a CLUSTER launch spreads one row over: the rule of the launch planner
// in rowops.cu (2 to 8 CTAs, at most 16 columns per thread while the cluster
// can grow, grown while rows x CTAs leave fewer than two per SM).
std::int64_t cluster_ctas(int block, std::int64_t rows, std::int64_t cols) {
  std::int64_t cs = 2;
  while (cs < 8 && cols > std::int64_t(block) * 16 * cs) cs <<= 1;
  const std::int64_t sms = device_sms();
  while (cs < 8 && rows * cs < 2 * sms && cols % (cs * 16) == 0 && cols / (cs * 2) >= std::int64_t(block) * 8)
    cs <<= 1;
  return cs;
}

}  // namespace

const char *elem_mode_name(ElemMode m) noexcept {
  switch (m) {
    case ElemMode::kOnePass: return "onepass";
    case ElemMode::kTwoPass: return "twopass";
    case ElemMode::kStrided: return "strided";
    case ElemMode::kTree: return "tree";
    case ElemMode::kStaged: return "staged";
    case ElemMode::kCluster: return "cluster";
  }
  return "unknown";
}

std::string canonical_config(const json &cfg) {
  if (!cfg.is_object()) return cfg.dump();
  std::vector<std::pair<std::string, std::string>> kv;
  for (const auto &[k, v] : cfg.as_object()) kv.emplace_back(k, v.dump());
  std::sort(kv.begin(), kv.end());
  std::string s = "{";
  for (size_t i = 0; i < kv.size(); ++i) s += (i ? "," : "") + kv[i].first + ":" + kv[i].second;
  return s + "}";
}

// ---------------------------------------------------------------------------
// verdicts
// ---------------------------------------------------------------------------
GateVerdict bf16_verdict(const std::vector<float> &a, const std::vector<float> &r) {
  GateVerdict v;
  const golden::Verdict rv = golden::verdict(a, r);
  v.cosine = rv.cosine;
  v.max_rel_err = rv.max_rel_err;
  v.pcc = rv.pcc;
  // diagnostics: per-element error with a 2^-8 rms floor, norm-wise error
  const size_t n = std::min(a.size(), r.size());
  double nr = 0, ss = 0, se = 0, fmax = 0;
  for (size_t i = 0; i < n; ++i) nr += double(r[i]) * r[i];
  const double rms = std::sqrt(nr / double(std::max<size_t>(n, 1)));
  for (size_t i = 0; i < n; ++i) {
    const double den = std::max(std::fabs(double(r[i])), rms * std::ldexp(1.0, -8));
    const double e = std::fabs(double(a[i]) - r[i]);
    se += e * e;
    ss += double(r[i]) * r[i];
    if (den > 0) fmax = std::max(fmax, e / den);
  }
  v.floor_rel_err = fmax;
  v.norm_rel_err = ss > 0 ? std::sqrt(se / ss) : std::sqrt(se);
  v.pass = rv.pass;
  v.criterion = "reference verdict: cosine>=0.999, max_rel_err(eps 1e-6)<=1e-2, pcc>=0.99";
  return v;
}

GateVerdict Session::verdict(const std::vector<float> &got, const std::vector<float> &ref) const {
  return bf16_verdict(got, ref);
}

// ===========================================================================
// matmul
// ===========================================================================
namespace {
ks_matmul_config to_mm(const json &c) {
  return ks_matmul_config{iget(c, "tile_m", 128), iget(c, "tile_n", 256), iget(c, "tile_k", 64),
                          iget(c, "stages", 4),   iget(c, "acc_stages", 2), iget(c, "group_m", 8),
                          iget(c, "cta_group", 0)};
}
// cta_group appears only where it is not the tile_m default, so configs
// recorded before it existed keep their keys
json mm_json(int bm, int bn, int st, int acc, int g, int cg = 0) {
  json j = db::json::object({{"tile_m", json(bm)}, {"tile_n", json(bn)}, {"tile_k", json(64)},
                             {"stages", json(st)}, {"acc_stages", json(acc)}, {"group_m", json(g)}});
  if (cg == 1) j = db::json::object({{"tile_m", json(bm)}, {"tile_n", json(bn)}, {"tile_k", json(64)},
                                      {"stages", json(st)}, {"acc_stages", json(acc)}, {"group_m", json(g)},
                                      {"cta_group", json(cg)}});
  return j;
}
int pow2_cols(int c) {
  int p = 32;
  while (p < c) p <<= 1;
  return p;
}

class MatmulSession : public Session {
 public:
  std::int64_t m, n, k;
  HostBf16 a, b;
  DevBuf da, db, dc;
  int init(std::int64_t M, std::int64_t N, std::int64_t K, std::uint64_t seed) {
    m = M, n = N, k = K;
    golden::Generator r(seed);  // inputs.py:77-80: a, then b
    a.fill_uniform(r, size_t(m * k), -1, 1);
    b.fill_uniform(r, size_t(k * n), -1, 1);
    return host_only ? KS_OK : upload_all();
  }
  bool host_only = false;  // inputs and reference only (no device buffers)
  NamedInputs named() { return {{"a", &a}, {"b", &b}}; }
  int upload_all() {
    int s = upload(da, a.bits.data(), a.bits.size() * 2);
    if (s == KS_OK) s = upload(db, b.bits.data(), b.bits.size() * 2);
    if (s == KS_OK) s = dc.alloc(size_t(m * n) * 2);
    return s;
  }
  int launch(const json &cfg, void *st) override {
    ks_matmul_config c = to_mm(cfg);
    ks_matmul_args args{da.p, db.p, dc.p, m, n, k};
    return ks_matmul_launch(&c, &args, st);
  }
  int output(std::vector<float> *o) override { return download_bf16(dc, size_t(m * n), o); }
  void reference(std::vector<float> *o) const override {  // refs.py:54-56
    o->assign(size_t(m * n), 0.f);
    golden::matmul(a.f.data(), b.f.data(), m, n, k, o->data());
  }
  int corrupt_output(void *st) override { return ks_gpu_memset(dc.p, 0, size_t(m * n) * 2, st); }
};

class MatmulFamily : public Family {
 public:
  const char *name() const override { return "matmul"; }
  bool check_shape(const std::vector<std::int64_t> &s, std::string *r) const override {
    if (s.size() != 3 || s[0] <= 0 || s[1] <= 0 || s[2] <= 0) {
      if (r) *r = "matmul expects --shape M,N,K (positive)";
      return false;
    }
    return true;
  }
  std::vector<json> enumerate(bool full, const std::vector<std::int64_t> &) const override {
    std::vector<json> v;
    // tile_m 128: one CTA per tile; tile_m 256: a CTA pair (cta_group::2)
    if (!full) {
      // group_m: M-groups of 8 or 16 tiles, or bands of 8 N-tiles with B kept in L2
      for (auto [bn, st] : {std::pair{256, 3}, {256, 4}, {128, 4}, {128, 6}})
        for (int acc : {1, 2})
          for (int g : {8, 16, -8}) v.push_back(mm_json(128, bn, st, acc, g));
      for (int st : {4, 6})
        for (int g : {8, 16}) v.push_back(mm_json(256, 256, st, 2, g));
      // 256-row tiles on one CTA (two M=128 MMAs per B tile)
      for (int g : {16, -8}) {
        v.push_back(mm_json(256, 256, 2, 1, g, 1));
        v.push_back(mm_json(256, 256, 3, 1, g, 1));
        v.push_back(mm_json(256, 128, 4, 2, g, 1));
      }
      return v;
    }
    for (int bm : {128, 256})
      for (int bn : {64, 128, 256})
        for (int st = 2; st <= 6; ++st)
          for (int acc : {1, 2})
            for (int g : {1, 4, 8, 16, 32, -8})
              if (bm == 128 || bn != 64) v.push_back(mm_json(bm, bn, st, acc, g));
    for (int bn : {128, 256})
      for (int st = 2; st <= 4; ++st)
        for (int acc : {1, 2})
          for (int g : {1, 4, 8, 16, 32, -8}) v.push_back(mm_json(256, bn, st, acc, g, 1));
    return v;
  }
  ConfigVerdict validate(const json &cfg, const std::vector<std::int64_t> &s, const std::string &arch) const override {
    MatmulConfig c{iget(cfg, "tile_m", 0), iget(cfg, "tile_n", 0), iget(cfg, "tile_k", 0), iget(cfg, "stages", 0),
                   iget(cfg, "acc_stages", 0), iget(cfg, "group_m", 0), iget(cfg, "cta_group", 0)};
    return validate_config(c, MatmulProblem{s[0], s[1], s[2], arch, 2});
  }
  Resources resources(const json &cfg, const std::vector<std::int64_t> &) const override {
    ks_matmul_config c = to_mm(cfg);
    return Resources{64, int(smem_bytes(MatmulConfig{c.tile_m, c.tile_n, c.tile_k, c.stages, c.acc_stages, c.group_m, c.cta_group})),
                     192, pow2_cols(c.acc_stages * c.tile_n * (c.tile_m == 256 && c.cta_group == 1 ? 2 : 1))};
  }
  LaunchGeometry geometry(const json &cfg, const std::vector<std::int64_t> &s) const override {
    ks_matmul_config c = to_mm(cfg);
    return launch_geometry(MatmulConfig{c.tile_m, c.tile_n, c.tile_k, c.stages, c.acc_stages, c.group_m, c.cta_group},
                           MatmulProblem{s[0], s[1], s[2], "sm_100a", 2});
  }
  std::string symbol(const json &cfg) const override {
    ks_matmul_config c = to_mm(cfg);
    return kernel_symbol(MatmulConfig{c.tile_m, c.tile_n, c.tile_k, c.stages, c.acc_stages, c.group_m, c.cta_group});
  }
  std::vector<std::int64_t> gate_shape(const std::vector<std::int64_t> &) const override { return {64, 64, 64}; }
  std::int64_t flops(const std::vector<std::int64_t> &s, const json &) const override {
    return roofline::compute_flops(roofline::KernelFamily::kGemm, {s[0], s[1], s[2], 0, 2});
  }
  std::int64_t bytes(const std::vector<std::int64_t> &s) const override {
    return roofline::compute_bytes_moved(roofline::KernelFamily::kGemm, {s[0], s[1], s[2], 0, 2});
  }
  std::unique_ptr<Session> make_session(const std::vector<std::int64_t> &s, std::uint64_t seed,
                                        std::string *err) const override {
    auto p = std::make_unique<MatmulSession>();
    const int st = p->init(s[0], s[1], s[2], seed);
    if (st != KS_OK) {
      if (err) *err = std::string("matmul session: ") + ks_status_string(st);
      return nullptr;
    }
    return p;
  }
  std::string generate_source(const json &cfg, const std::vector<std::int64_t> &s) const override {
    ks_matmul_config c = to_mm(cfg);
    std::ostringstream o;
    o << "// reproducer: " << symbol(cfg) << " at M,N,K = " << shape_str(s) << "\n"
      << "#include <kernscope_b200.h>\n#include <cstdio>\n#include <vector>\n"
      << "int main() {\n  const long long m = " << s[0] << ", n = " << s[1] << ", k = " << s[2] << ";\n"
      << "  void *a, *b, *c;\n  ks_gpu_malloc(&a, m * k * 2); ks_gpu_malloc(&b, k * n * 2); ks_gpu_malloc(&c, m * n * 2);\n"
      << "  ks_gpu_memset(a, 0, m * k * 2, nullptr); ks_gpu_memset(b, 0, k * n * 2, nullptr);\n"
      << "  ks_matmul_config cfg{" << c.tile_m << ", " << c.tile_n << ", " << c.tile_k << ", " << c.stages << ", "
      << c.acc_stages << ", " << c.group_m << ", " << c.cta_group << "};\n"
      << "  ks_matmul_args args{a, b, c, m, n, k};\n"
      << "  int st = ks_matmul_launch(&cfg, &args, nullptr);\n  if (st == 0) st = ks_gpu_synchronize();\n"
      << "  std::printf(\"%s\\n\", ks_status_string(st));\n  return st == 0 ? 0 : 1;\n}\n";
    return o.str();
  }
};

// ===========================================================================
// flash attention
// ===========================================================================
// shapes: Nq,Nk,d (one head, the reference ABI) or B,H,N,d (self-attention)
struct FaShape {
  std::int64_t bh, nq, nk, d;
};
FaShape fa_shape(const std::vector<std::int64_t> &s) {
  if (s.size() == 4) return {s[0] * s[1], s[2], s[2], s[3]};
  return {1, s[0], s[1], s[2]};
}

class FlashSession : public Session {
 public:
  FaShape sh;
  bool causal = false;
  HostBf16 q, k, v;
  DevBuf dq, dk, dv, dout;
  int init(const FaShape &s, bool c, std::uint64_t seed) {
    sh = s;
    causal = c;
    golden::Generator r(seed);
    // the reference profile (inputs.py:98-105): q, k ~ U(-1/sqrt d, 1/sqrt d),
    // v ~ U(-1, 1), each drawn for every head at once (one head = the
    // reference's single-head draws exactly)
    const double sc = 1.0 / std::sqrt(double(s.d));
    q.fill_uniform(r, size_t(s.bh * s.nq * s.d), -sc, sc);
    k.fill_uniform(r, size_t(s.bh * s.nk * s.d), -sc, sc);
    v.fill_uniform(r, size_t(s.bh * s.nk * s.d), -1, 1);
    return host_only ? KS_OK : upload_all();
  }
  bool host_only = false;  // inputs and reference only (no device buffers)
  NamedInputs named() { return {{"q", &q}, {"k", &k}, {"v", &v}}; }
  int upload_all() {
    int st = upload(dq, q.bits.data(), q.bits.size() * 2);
    if (st == KS_OK) st = upload(dk, k.bits.data(), k.bits.size() * 2);
    if (st == KS_OK) st = upload(dv, v.bits.data(), v.bits.size() * 2);
    if (st == KS_OK) st = dout.alloc(q.bits.size() * 2);
    return st;
  }
  bool tensor_path = false;  // the last launched config ran on the tcgen05 kernels
  int launch(const json &cfg, void *st) override {
    ks_flash_attention_config c{iget(cfg, "tile_m", 256), iget(cfg, "tile_n", 128), iget(cfg, "stages", 2),
                                causal ? 1 : 0};
    tensor_path = sh.d == 128 || (sh.d == 64 && c.tile_m == 256);
    ks_flash_attention_args a{dq.p, dk.p, dv.p, dout.p, 1, sh.bh, sh.nq, sh.nk, sh.d, 0.f};
    return ks_flash_attention_launch(&c, &a, st);
  }
  int output(std::vector<float> *o) override { return download_bf16(dout, size_t(sh.bh * sh.nq * sh.d), o); }
  void reference(std::vector<float> *o) const override {  // refs.py:113-142 per head
    o->assign(size_t(sh.bh * sh.nq * sh.d), 0.f);
    for (std::int64_t h = 0; h < sh.bh; ++h)
      golden::attention(&q.f[size_t(h * sh.nq * sh.d)], &k.f[size_t(h * sh.nk * sh.d)],
                        &v.f[size_t(h * sh.nk * sh.d)], sh.nq, sh.nk, sh.d, causal,
                        o->data() + h * sh.nq * sh.d);
  }
  // The CUDA-core kernel (fp32 throughout) is judged by the reference verdict
  // as it stands.  The tensor-core path rounds P to bf16 before P V (2^-9 per
  // probability), which no tensor-core attention avoids; on outputs near zero
  // that alone exceeds max_rel_err's 1e-2 with eps 1e-6, so for that path the
  // per-element term becomes |a - r| <= 1e-2 * rho, rho = softmax |V| (the
  // scale of the P rounding error), beside the reference's cosine and pcc
  // and a norm-wise error <= 1e-2.
  GateVerdict verdict(const std::vector<float> &got, const std::vector<float> &ref) const override {
    GateVerdict gv = bf16_verdict(got, ref);
    if (!tensor_path) return gv;
    double worst = 0.0;
    const float sd = float(std::sqrt(double(sh.d)));
    std::vector<float> srow(static_cast<size_t>(sh.nk));
    for (std::int64_t h = 0; h < sh.bh; ++h)
      for (std::int64_t i = 0; i < sh.nq; ++i) {
        const float *qi = &q.f[size_t((h * sh.nq + i) * sh.d)];
        float mx = -INFINITY;
        for (std::int64_t j = 0; j < sh.nk; ++j) {
          float s = -INFINITY;
          if (!(causal && j > i)) {
            const float *kj = &k.f[size_t((h * sh.nk + j) * sh.d)];
            s = 0.f;
            for (std::int64_t c = 0; c < sh.d; ++c) s += qi[c] * kj[c];
            s /= sd;
          }
          srow[size_t(j)] = s;
          mx = std::max(mx, s);
        }
        double sum = 0;
        for (auto &x : srow) {
          x = std::exp(x - mx);
          sum += x;
        }
        for (std::int64_t c = 0; c < sh.d; ++c) {
          double rho = 0;
          for (std::int64_t j = 0; j < sh.nk; ++j) rho += srow[size_t(j)] * std::fabs(v.f[size_t((h * sh.nk + j) * sh.d + c)]);
          rho /= sum;
          const size_t idx = size_t((h * sh.nq + i) * sh.d + c);
          if (rho > 0) worst = std::max(worst, std::fabs(double(got[idx]) - ref[idx]) / rho);
        }
      }
    gv.floor_rel_err = worst;
    gv.pass = gv.cosine >= 0.999 && gv.pcc >= 0.99 && worst <= 1e-2 && gv.norm_rel_err <= 1e-2;
    gv.criterion = "cosine>=0.999, pcc>=0.99, |a-r| <= 1e-2 * softmax|V|, norm rel-err<=1e-2";
    return gv;
  }
  int corrupt_output(void *st) override { return ks_gpu_memset(dout.p, 0, dout.bytes, st); }
};

// The tcgen05 kernels take d = 128 with either tile_m and d = 64 with tile_m
// 256; every other (config, d) runs on the CUDA-core kernel.
static bool fa_tensor_path(const FlashAttentionConfig &c, std::int64_t d) {
  return d == 128 || (d == 64 && c.tile_m == 256);
}

class FlashFamily : public Family {
 public:
  bool causal = false;
  const char *name() const override { return "flash_attention"; }
  bool check_shape(const std::vector<std::int64_t> &s, std::string *r) const override {
    if ((s.size() != 3 && s.size() != 4) || std::any_of(s.begin(), s.end(), [](auto x) { return x <= 0; })) {
      if (r) *r = "flash_attention expects --shape Nq,Nk,d or B,H,N,d (positive)";
      return false;
    }
    return true;
  }
  std::vector<json> enumerate(bool, const std::vector<std::int64_t> &) const override {
    // TMEM (512 columns) holds two 128x128 S tiles and two 128x128 O tiles
    // (tile_m 256: two query tiles per CTA) or two S tiles and one O tile
    // (tile_m 128: one query tile, S double-buffered); 128-key K/V tiles in a
    // 2-stage ring.
    // tile_n 64: two query tiles with S in 64-key slots (one online-softmax
    // step per 64 keys, the next Q K^T of a slot overlapping the other's softmax)
    std::vector<json> out;
    for (auto [tm, tn] : {std::pair{256, 128}, {128, 128}, {256, 64}})
      out.push_back(db::json::object({{"tile_m", json(tm)}, {"tile_n", json(tn)}, {"stages", json(2)},
                                      {"causal", json(causal)}}));
    return out;
  }
  ConfigVerdict validate(const json &cfg, const std::vector<std::int64_t> &s, const std::string &arch) const override {
    const FaShape f = fa_shape(s);
    FlashAttentionConfig c{iget(cfg, "tile_m", 0), iget(cfg, "tile_n", 0), iget(cfg, "stages", 0),
                           cfg.find("causal") && cfg.find("causal")->as_bool()};
    return validate_config(c, FlashAttentionProblem{f.nq, f.nk, f.d, f.bh, causal, arch, 2});
  }
  static FlashAttentionConfig typed(const json &cfg, bool causal) {
    return FlashAttentionConfig{iget(cfg, "tile_m", 256), iget(cfg, "tile_n", 128), iget(cfg, "stages", 2), causal};
  }
  Resources resources(const json &cfg, const std::vector<std::int64_t> &s) const override {
    const FaShape f = fa_shape(s);
    const FlashAttentionConfig c = typed(cfg, causal);
    if (!fa_tensor_path(c, f.d)) return Resources{48, 4 * 256 * 4, 128, 0};
    // tile_m 256: three warpgroups (the producer/MMA one hands registers to
    // the two softmax ones); tile_m 128: ten warps
    FlashAttentionProblem p{};
    p.d = f.d;
    return Resources{168, int(smem_bytes(c, p)), c.tile_m == 256 ? 384 : 320, 512};
  }
  LaunchGeometry geometry(const json &cfg, const std::vector<std::int64_t> &s) const override {
    const FaShape f = fa_shape(s);
    return launch_geometry(typed(cfg, causal), FlashAttentionProblem{f.nq, f.nk, f.d, f.bh, causal, "sm_100a", 2});
  }
  std::string symbol(const json &cfg) const override { return kernel_symbol(typed(cfg, causal)); }
  std::vector<std::int64_t> gate_shape(const std::vector<std::int64_t> &s) const override {
    const FaShape f = fa_shape(s);
    return {1, 2, std::min<std::int64_t>(std::max(f.nq, f.nk), 256), f.d};
  }
  std::int64_t flops(const std::vector<std::int64_t> &s, const json &) const override {
    const FaShape f = fa_shape(s);
    roofline::Shape r{f.bh, f.nq, 0, f.d, 2, causal};
    return roofline::compute_flops(roofline::KernelFamily::kFlashAttention, r);
  }
  std::int64_t bytes(const std::vector<std::int64_t> &s) const override {
    const FaShape f = fa_shape(s);
    return 2 * f.bh * (2 * f.nq + 2 * f.nk) * f.d;
  }
  std::unique_ptr<Session> make_session(const std::vector<std::int64_t> &s, std::uint64_t seed,
                                        std::string *err) const override {
    auto p = std::make_unique<FlashSession>();
    const int st = p->init(fa_shape(s), causal, seed);
    if (st != KS_OK) {
      if (err) *err = std::string("flash_attention session: ") + ks_status_string(st);
      return nullptr;
    }
    return p;
  }
  std::string generate_source(const json &cfg, const std::vector<std::int64_t> &s) const override {
    const FaShape f = fa_shape(s);
    std::ostringstream o;
    o << "// reproducer: " << symbol(cfg) << " at (B*H, Nq, Nk, d) = (" << f.bh << ", " << f.nq << ", " << f.nk
      << ", " << f.d << ")\n#include <kernscope_b200.h>\n#include <cstdio>\n"
      << "int main() {\n  const long long bh = " << f.bh << ", nq = " << f.nq << ", nk = " << f.nk << ", d = " << f.d
      << ";\n  void *q, *k, *v, *o;\n"
      << "  ks_gpu_malloc(&q, bh * nq * d * 2); ks_gpu_malloc(&k, bh * nk * d * 2); ks_gpu_malloc(&v, bh * nk * d * 2);\n"
      << "  ks_gpu_malloc(&o, bh * nq * d * 2);\n"
      << "  ks_gpu_memset(q, 0, bh * nq * d * 2, nullptr); ks_gpu_memset(k, 0, bh * nk * d * 2, nullptr);\n"
      << "  ks_gpu_memset(v, 0, bh * nk * d * 2, nullptr);\n"
      << "  ks_flash_attention_config cfg{128, 128, 2, " << (causal ? 1 : 0) << "};\n"
      << "  ks_flash_attention_args args{q, k, v, o, 1, bh, nq, nk, d, 0.f};\n"
      << "  int st = ks_flash_attention_launch(&cfg, &args, nullptr);\n  if (st == 0) st = ks_gpu_synchronize();\n"
      << "  std::printf(\"%s\\n\", ks_status_string(st));\n  return st == 0 ? 0 : 1;\n}\n";
    return o.str();
  }
};

// ===========================================================================
// row ops (softmax, layernorm, bias_gelu) and reduction
// ===========================================================================
enum class RowKind { kSoftmax, kLayerNorm, kBiasGelu, kReduction };

class RowSession : public Session {
 public:
  RowKind kind;
  std::int64_t rows = 0, cols = 0;
  int gelu = KS_GELU_ERF;
  int axis = 0;  // reduction
  HostBf16 x, p1, p2;
  std::vector<float> xf32;  // reduction full sum input
  DevBuf dx, dp1, dp2, dout, dws;
  size_t out_n = 0;

  int init(RowKind k, std::int64_t r, std::int64_t c, int g, int ax, std::uint64_t seed) {
    kind = k;
    rows = r;
    cols = c;
    gelu = g;
    axis = ax;
    golden::Generator rng(seed);
    const size_t n = size_t(r * c);
    out_n = k == RowKind::kReduction ? (axis == -1 ? 1 : size_t(c)) : n;
    // distributions of the reference profile (inputs.py:77-97)
    switch (k) {
      case RowKind::kSoftmax: x.fill_uniform(rng, n, -2, 2); break;
      case RowKind::kLayerNorm:
        x.fill_uniform(rng, n, -1, 1);
        p1.fill_uniform(rng, size_t(c), 0.5, 1.5);
        p2.fill_uniform(rng, size_t(c), -0.25, 0.25);
        break;
      case RowKind::kBiasGelu:
        x.fill_uniform(rng, n, -1, 1);
        p1.fill_uniform(rng, size_t(c), -0.25, 0.25);
        break;
      case RowKind::kReduction:
        if (axis == -1) {
          xf32.resize(n);
          for (auto &v : xf32) v = float(rng.uniform(0, 1));
        } else {
          x.fill_uniform(rng, n, -1, 1);
        }
        break;
    }
    return host_only ? KS_OK : upload_all();
  }
  bool host_only = false;  // inputs and reference only (no device buffers)
  NamedInputs named() {
    switch (kind) {
      case RowKind::kLayerNorm: return {{"x", &x}, {"gamma", &p1}, {"beta", &p2}};
      case RowKind::kBiasGelu: return {{"x", &x}, {"bias", &p1}};
      default: return {{"x", &x}};
    }
  }
  int upload_all() {
    const size_t n = size_t(rows * cols);
    int st = KS_OK;
    if (kind == RowKind::kReduction && axis == -1)
      st = upload(dx, xf32.data(), n * 4);
    else
      st = upload(dx, x.bits.data(), n * 2);
    if (st == KS_OK && !p1.bits.empty()) st = upload(dp1, p1.bits.data(), p1.bits.size() * 2);
    if (st == KS_OK && !p2.bits.empty()) st = upload(dp2, p2.bits.data(), p2.bits.size() * 2);
    const size_t out_bytes = kind == RowKind::kReduction && axis == -1 ? 4 : out_n * 2;
    if (st == KS_OK) st = dout.alloc(out_bytes);
    return st;
  }

  int launch(const json &cfg, void *st) override {
    const int block = iget(cfg, "block", 256), vec = iget(cfg, "vec_width", 8);
    switch (kind) {
      case RowKind::kSoftmax: {
        ks_softmax_config c{block, vec, mode_from(cfg, KS_MODE_ONEPASS)};
        ks_softmax_args a{dx.p, dout.p, rows, cols};
        return ks_softmax_launch(&c, &a, st);
      }
      case RowKind::kLayerNorm: {
        ks_layernorm_config c{block, vec, mode_from(cfg, KS_MODE_ONEPASS)};
        ks_layernorm_args a{dx.p, dp1.p, dp2.p, dout.p, rows, cols, 1e-5f};
        return ks_layernorm_launch(&c, &a, st);
      }
      case RowKind::kBiasGelu: {
        ks_bias_gelu_config c{block, vec, gelu};
        ks_bias_gelu_args a{dx.p, dp1.p, dout.p, rows * cols, cols};
        return ks_bias_gelu_launch(&c, &a, st);
      }
      case RowKind::kReduction: {
        ks_reduction_config c{block, vec, mode_from(cfg, KS_MODE_TREE)};
        ks_reduction_args a{dx.p,      dout.p, rows, cols, axis == -1 ? KS_F32 : KS_BF16, axis == -1 ? KS_F32 : KS_BF16,
                            axis,      nullptr, 0,    nullptr};
        size_t need = 0;
        int s = ks_reduction_workspace_bytes(&c, &a, &need);
        if (s != KS_OK) return s;
        if (need > dws.bytes) {
          if (dws.p) ks_gpu_free(dws.p);
          dws.p = nullptr;
          if ((s = dws.alloc(need)) != KS_OK) return s;
        }
        a.workspace = dws.p;
        a.workspace_bytes = dws.bytes;
        return ks_reduction_launch(&c, &a, st);
      }
    }
    return KS_ERR_OTHER;
  }

  int output(std::vector<float> *o) override {
    if (kind == RowKind::kReduction && axis == -1) {
      float v = 0;
      int s = ks_gpu_memcpy_dtoh(&v, dout.p, 4, nullptr);
      if (s == KS_OK) s = ks_gpu_synchronize();
      o->assign(1, v);
      return s;
    }
    return download_bf16(dout, out_n, o);
  }

  void reference(std::vector<float> *o) const override {
    o->assign(out_n, 0.f);
    switch (kind) {
      case RowKind::kSoftmax: golden::softmax(x.f.data(), rows, cols, o->data()); break;  // refs.py:79-84
      case RowKind::kLayerNorm:  // refs.py:87-99
        golden::layernorm(x.f.data(), p1.f.data(), p2.f.data(), rows, cols, 1e-5f, o->data());
        break;
      case RowKind::kBiasGelu:  // refs.py:59-76 (erf), or the tanh extension
        golden::bias_gelu(x.f.data(), p1.f.data(), rows, cols, gelu == KS_GELU_TANH, o->data());
        break;
      case RowKind::kReduction:
        if (axis == -1) {  // the full fp32 sum extension, judged against an fp64 sum
          double s = 0;
          for (float v : xf32) s += v;
          (*o)[0] = float(s);
        } else {  // refs.py:102-110
          golden::reduction_axis0(x.f.data(), rows, cols, o->data());
        }
        break;
    }
  }

  GateVerdict verdict(const std::vector<float> &got, const std::vector<float> &ref) const override {
    if (kind == RowKind::kReduction && axis == -1) {
      GateVerdict v;
      const double rel = std::fabs(double(got[0]) - ref[0]) / std::max(1e-30, std::fabs(double(ref[0])));
      v.cosine = v.pcc = 1.0;
      v.max_rel_err = v.floor_rel_err = v.norm_rel_err = rel;
      v.pass = rel <= 1e-5;
      v.criterion = "fp32 sum rel-err <= 1e-5 against an fp64 sum";
      return v;
    }
    return bf16_verdict(got, ref);
  }

  int corrupt_output(void *st) override { return ks_gpu_memset(dout.p, 0, dout.bytes, st); }
};

class RowFamily : public Family {
 public:
  RowKind kind;
  const char *nm;
  int gelu = KS_GELU_ERF;
  RowFamily(RowKind k, const char *n) : kind(k), nm(n) {}
  const char *name() const override { return nm; }
  bool check_shape(const std::vector<std::int64_t> &s, std::string *r) const override {
    if (kind == RowKind::kReduction && s.size() == 1 && s[0] > 0) return true;  // full fp32 sum
    return valid_elem_shape(s, r, nm);
  }
  static std::pair<std::int64_t, std::int64_t> rc(const std::vector<std::int64_t> &s) {
    return s.size() == 1 ? std::pair{std::int64_t(1), s[0]} : std::pair{s[0], s[1]};
  }
  int axis_of(const std::vector<std::int64_t> &s) const { return kind == RowKind::kReduction && s.size() == 1 ? -1 : 0; }

  std::vector<json> enumerate(bool full, const std::vector<std::int64_t> &s) const override {
    std::vector<json> v;
    // bias_gelu keeps 1024 in the bounded grid: its 8-wide erf kernel at
    // 1024 threads (a table of every bf16 code, one CTA per SM) is the fastest
    const std::vector<int> blocks = full || kind == RowKind::kBiasGelu ? std::vector<int>{128, 256, 512, 1024}
                                                                       : std::vector<int>{128, 256, 512};
    const std::vector<int> vecs = full ? std::vector<int>{1, 2, 4, 8} : std::vector<int>{4, 8};
    std::vector<std::string> modes;
    if (kind == RowKind::kSoftmax || kind == RowKind::kLayerNorm) modes = {"onepass", "twopass", "staged", "cluster"};
    if (kind == RowKind::kReduction) modes = {"strided", "tree"};
    for (int b : blocks)
      for (int vw : (axis_of(s) == -1 ? std::vector<int>{4} : vecs)) {
        if (modes.empty()) {
          v.push_back(db::json::object({{"block", json(b)}, {"vec_width", json(vw)},
                                        {"gelu", json(gelu == KS_GELU_TANH ? "tanh" : "erf")}}));
        } else {
          for (const auto &m : modes)
            v.push_back(db::json::object({{"block", json(b)}, {"vec_width", json(vw)}, {"mode", json(m)}}));
        }
      }
    return v;
  }
  ConfigVerdict validate(const json &cfg, const std::vector<std::int64_t> &s, const std::string &arch) const override {
    const auto [r, c] = rc(s);
    ElemProblem p{r, c, arch, 2, axis_of(s)};
    const int block = iget(cfg, "block", 0), vec = iget(cfg, "vec_width", 0);
    switch (kind) {
      case RowKind::kSoftmax: return validate_config(SoftmaxConfig{block, vec, ElemMode(mode_from(cfg, -1))}, p);
      case RowKind::kLayerNorm: return validate_config(LayerNormConfig{block, vec, ElemMode(mode_from(cfg, -1))}, p);
      case RowKind::kBiasGelu: return validate_config(BiasGeluConfig{block, vec, gelu}, p);
      case RowKind::kReduction: return validate_config(ReductionConfig{block, vec, ElemMode(mode_from(cfg, -1))}, p);
    }
    return {false, "unknown family"};
  }
  Resources resources(const json &cfg, const std::vector<std::int64_t> &s) const override {
    const int block = iget(cfg, "block", 256);
    const int mode = mode_from(cfg, KS_MODE_ONEPASS);
    const auto [r, c] = rc(s);
    (void)r;
    Resources res{64, 512, block, 0};
    if (kind == RowKind::kReduction) {
      res.regs_per_thread = 40;
      // axis 0 stages every thread's column partials (block x vec_width fp32)
      if (axis_of(s) == 0) res.smem_bytes = block * iget(cfg, "vec_width", 8) * 4 + 16;
    }
    if (kind == RowKind::kBiasGelu) {
      res.regs_per_thread = 61;
      // 8-wide erf: a 128 KB table of every bf16 code at 1024 threads, a
      // 6 KB table of the 3072 non-trivial codes below
      if (gelu == KS_GELU_ERF && iget(cfg, "vec_width", 8) == 8) res.smem_bytes = block == 1024 ? 131072 : 6144;
    }
    if (mode == KS_MODE_CLUSTER) {
      res.regs_per_thread = 50;  // up to four 8-wide chunks per thread
      res.smem_bytes = 288;      // warp partials and the cluster slots
    } else if (mode == KS_MODE_STAGED) {
      // 64 KB ring (plus gamma/beta for layernorm) up to 512 threads; a
      // 1024-thread CTA keeps a 200 KB ring and reads gamma/beta from L2
      const bool wide = block == 1024;
      const std::int64_t stride = (c * 2 + 127) / 128 * 128;
      const int stages = int(std::min<std::int64_t>(8, (wide ? 204800 : 65536) / std::max<std::int64_t>(stride, 1)));
      res.smem_bytes = int(stride * (stages + (kind == RowKind::kLayerNorm && !wide ? 2 : 0))) + 512;
      res.regs_per_thread = wide ? 64 : 80;
    } else if (iget(cfg, "vec_width", 8) == 8 && mode == KS_MODE_ONEPASS && c <= 1024 &&
               (kind == RowKind::kSoftmax || kind == RowKind::kLayerNorm)) {
      // one row per warp, at most 256 threads per CTA; layernorm also keeps
      // its gamma/beta chunks in registers
      res.block = std::min(block, 256);
      res.regs_per_thread = kind == RowKind::kSoftmax ? 80 : c <= 512 ? 76 : 145;
    } else if (block <= 256 && iget(cfg, "vec_width", 8) == 8 && kind != RowKind::kReduction &&
               kind != RowKind::kBiasGelu) {
      res.regs_per_thread = 80;  // the prefetching 8-wide instantiation
    }
    return res;
  }
  LaunchGeometry geometry(const json &cfg, const std::vector<std::int64_t> &s) const override {
    const auto [r, c] = rc(s);
    LaunchGeometry g;
    g.block_x = iget(cfg, "block", 256);
    const Resources res = resources(cfg, s);
    const auto occ = occupancy::compute_occupancy(get_arch("sm_100a"), res.regs_per_thread, res.smem_bytes,
                                                  g.block_x, 0);
    const std::int64_t cap = std::int64_t(std::max(1, occ.blocks_per_sm)) * device_sms();
    if (kind == RowKind::kBiasGelu) {
      const std::int64_t nvec = c / std::max(1, iget(cfg, "vec_width", 8));
      g.grid_x = int((nvec + g.block_x - 1) / g.block_x);
      g.grid_y = int((r + 31) / 32);
    } else if (mode_from(cfg, -1) == KS_MODE_CLUSTER) {
      g.grid_x = int(r * cluster_ctas(g.block_x, r, c));
    } else {
      g.grid_x = int(std::min<std::int64_t>(r, cap));
    }
    g.smem_bytes = res.smem_bytes;
    return g;
  }
  std::string symbol(const json &cfg) const override {
    const int block = iget(cfg, "block", 0), vec = iget(cfg, "vec_width", 0);
    switch (kind) {
      case RowKind::kSoftmax: return kernel_symbol(SoftmaxConfig{block, vec, ElemMode(mode_from(cfg, 0))});
      case RowKind::kLayerNorm: return kernel_symbol(LayerNormConfig{block, vec, ElemMode(mode_from(cfg, 0))});
      case RowKind::kBiasGelu: return kernel_symbol(BiasGeluConfig{block, vec, gelu});
      case RowKind::kReduction: return kernel_symbol(ReductionConfig{block, vec, ElemMode(mode_from(cfg, 3))});
    }
    return "";
  }
  std::vector<std::int64_t> gate_shape(const std::vector<std::int64_t> &s) const override {
    if (s.size() == 1) return {std::min<std::int64_t>(s[0], 1 << 22)};
    const std::int64_t rows = std::max<std::int64_t>(1, std::min<std::int64_t>(s[0], (1 << 22) / std::max<std::int64_t>(s[1], 1)));
    return {rows, s[1]};
  }
  roofline::KernelFamily rk() const {
    switch (kind) {
      case RowKind::kSoftmax: return roofline::KernelFamily::kSoftmax;
      case RowKind::kLayerNorm: return roofline::KernelFamily::kLayerNorm;
      case RowKind::kBiasGelu: return roofline::KernelFamily::kFusedBiasGelu;
      case RowKind::kReduction: return roofline::KernelFamily::kReduction;
    }
    return roofline::KernelFamily::kSoftmax;
  }
  std::int64_t flops(const std::vector<std::int64_t> &s, const json &) const override {
    const auto [r, c] = rc(s);
    return roofline::compute_flops(rk(), roofline::Shape{0, r * c, c, 0, 2});
  }
  std::int64_t bytes(const std::vector<std::int64_t> &s) const override {
    const auto [r, c] = rc(s);
    if (kind == RowKind::kReduction)
      return s.size() == 1 ? r * c * 4 + 4 : r * c * 2 + c * 2;
    return roofline::compute_bytes_moved(rk(), roofline::Shape{0, r * c, c, 0, 2});
  }
  std::unique_ptr<Session> make_session(const std::vector<std::int64_t> &s, std::uint64_t seed,
                                        std::string *err) const override {
    auto p = std::make_unique<RowSession>();
    const auto [r, c] = rc(s);
    const int st = p->init(kind, r, c, gelu, axis_of(s), seed);
    if (st != KS_OK) {
      if (err) *err = std::string(nm) + " session: " + ks_status_string(st);
      return nullptr;
    }
    return p;
  }
  std::string generate_source(const json &cfg, const std::vector<std::int64_t> &s) const override {
    const auto [r, c] = rc(s);
    const int block = iget(cfg, "block", 256), vec = iget(cfg, "vec_width", 8);
    std::ostringstream o;
    o << "// reproducer: " << symbol(cfg) << " at " << shape_str(s) << "\n#include <kernscope_b200.h>\n#include <cstdio>\n"
      << "int main() {\n  const long long rows = " << r << ", cols = " << c << ";\n  void *x, *p1, *p2, *out, *ws = nullptr;\n"
      << "  ks_gpu_malloc(&x, rows * cols * 4); ks_gpu_malloc(&p1, cols * 2); ks_gpu_malloc(&p2, cols * 2);\n"
      << "  ks_gpu_malloc(&out, rows * cols * 4); ks_gpu_memset(x, 0, rows * cols * 4, nullptr);\n"
      << "  ks_gpu_memset(p1, 0, cols * 2, nullptr); ks_gpu_memset(p2, 0, cols * 2, nullptr);\n  int st = 0;\n";
    switch (kind) {
      case RowKind::kSoftmax:
        o << "  ks_softmax_config cfg{" << block << ", " << vec << ", " << mode_from(cfg, 0) << "};\n"
          << "  ks_softmax_args a{x, out, rows, cols};\n  st = ks_softmax_launch(&cfg, &a, nullptr);\n";
        break;
      case RowKind::kLayerNorm:
        o << "  ks_layernorm_config cfg{" << block << ", " << vec << ", " << mode_from(cfg, 0) << "};\n"
          << "  ks_layernorm_args a{x, p1, p2, out, rows, cols, 1e-5f};\n  st = ks_layernorm_launch(&cfg, &a, nullptr);\n";
        break;
      case RowKind::kBiasGelu:
        o << "  ks_bias_gelu_config cfg{" << block << ", " << vec << ", " << gelu << "};\n"
          << "  ks_bias_gelu_args a{x, p1, out, rows * cols, cols};\n  st = ks_bias_gelu_launch(&cfg, &a, nullptr);\n";
        break;
      case RowKind::kReduction:
        o << "  ks_reduction_config cfg{" << block << ", " << vec << ", " << mode_from(cfg, 3) << "};\n"
          << "  ks_reduction_args a{x, out, rows, cols, " << (axis_of(s) == -1 ? "KS_F32, KS_F32, -1" : "KS_BF16, KS_BF16, 0")
          << ", nullptr, 0, nullptr};\n  size_t need = 0; ks_reduction_workspace_bytes(&cfg, &a, &need);\n"
          << "  if (need) { ks_gpu_malloc(&ws, need); a.workspace = ws; a.workspace_bytes = need; }\n"
          << "  st = ks_reduction_launch(&cfg, &a, nullptr);\n";
        break;
    }
    o << "  if (st == 0) st = ks_gpu_synchronize();\n  std::printf(\"%s\\n\", ks_status_string(st));\n"
      << "  return st == 0 ? 0 : 1;\n}\n";
    return o.str();
  }
};

}  // namespace

// ---------------------------------------------------------------------------
// typed API
// ---------------------------------------------------------------------------
static ConfigVerdict from_status(int st, const char *reason) {
  if (st == KS_OK) return {true, ""};
  return {false, reason[0] ? std::string(reason) : std::string(ks_status_string(st))};
}

static ConfigVerdict check_arch(const std::string &arch) {
  if (!has_arch(arch)) return {false, "unknown arch '" + arch + "' (sm_100a DB)"};
  return {true, ""};
}

ConfigVerdict validate_config(const MatmulConfig &c, const MatmulProblem &p) noexcept {
  if (auto a = check_arch(p.arch); !a.valid) return a;
  ks_matmul_config k{c.tile_m, c.tile_n, c.tile_k, c.stages, c.acc_stages, c.group_m, c.cta_group};
  char reason[256] = {0};
  ConfigVerdict v = from_status(ks_matmul_validate(&k, p.m, p.n, p.k, reason, sizeof(reason)), reason);
  if (!v.valid) return v;
  const ArchInfo &arch = get_arch(p.arch);
  if (smem_bytes(c) > arch.smem_per_block_max_bytes)
    return {false, "matmul: shared memory " + std::to_string(smem_bytes(c)) + " > " +
                       std::to_string(arch.smem_per_block_max_bytes) + " bytes per CTA"};
  if (pow2_cols(c.acc_stages * c.tile_n * (c.tile_m == 256 && c.cta_group == 1 ? 2 : 1)) > arch.tmem_columns_per_sm)
    return {false, "matmul: accumulators need more than 512 TMEM columns"};
  return v;
}

ConfigVerdict validate_config(const FlashAttentionConfig &c, const FlashAttentionProblem &p) noexcept {
  if (auto a = check_arch(p.arch); !a.valid) return a;
  ks_flash_attention_config k{c.tile_m, c.tile_n, c.stages, c.causal ? 1 : 0};
  ks_flash_attention_args a{nullptr, nullptr, nullptr, nullptr, 1, p.batch_heads, p.nq, p.nk, p.d, 0.f};
  char reason[256] = {0};
  return from_status(ks_flash_attention_validate(&k, &a, reason, sizeof(reason)), reason);
}

ConfigVerdict validate_config(const SoftmaxConfig &c, const ElemProblem &p) noexcept {
  if (auto a = check_arch(p.arch); !a.valid) return a;
  ks_softmax_config k{c.block, c.vec_width, int(c.mode)};
  char reason[256] = {0};
  return from_status(ks_softmax_validate(&k, p.rows, p.cols, reason, sizeof(reason)), reason);
}

ConfigVerdict validate_config(const LayerNormConfig &c, const ElemProblem &p) noexcept {
  if (auto a = check_arch(p.arch); !a.valid) return a;
  ks_layernorm_config k{c.block, c.vec_width, int(c.mode)};
  char reason[256] = {0};
  return from_status(ks_layernorm_validate(&k, p.rows, p.cols, reason, sizeof(reason)), reason);
}

ConfigVerdict validate_config(const BiasGeluConfig &c, const ElemProblem &p) noexcept {
  if (auto a = check_arch(p.arch); !a.valid) return a;
  ks_bias_gelu_config k{c.block, c.vec_width, c.gelu};
  char reason[256] = {0};
  return from_status(ks_bias_gelu_validate(&k, p.rows * p.cols, p.cols, reason, sizeof(reason)), reason);
}

ConfigVerdict validate_config(const ReductionConfig &c, const ElemProblem &p) noexcept {
  if (auto a = check_arch(p.arch); !a.valid) return a;
  ks_reduction_config k{c.block, c.vec_width, int(c.mode)};
  ks_reduction_args a{nullptr, nullptr, p.rows, p.cols, p.axis == -1 ? KS_F32 : KS_BF16,
                      p.axis == -1 ? KS_F32 : KS_BF16, p.axis, nullptr, 0, nullptr};
  char reason[256] = {0};
  return from_status(ks_reduction_validate(&k, &a, reason, sizeof(reason)), reason);
}

std::int64_t smem_bytes(const MatmulConfig &c) noexcept {
  // per CTA: A ring (128 x 64 bf16, two such boxes for a one-CTA 256-row
  // tile) + B ring (64 x tile_n bf16; half of tile_n for the CTA pair of
  // tile_m 256) + the C staging of the TMA-store epilogue (4 warps x 2 x
  // [32 x 32] bf16) + barriers + 1 KB alignment slack
  const bool pair = c.tile_m == 256 && c.cta_group != 1;
  const std::int64_t a_rows = c.tile_m == 256 && !pair ? 256 : 128;
  const std::int64_t b_cols = pair ? c.tile_n / 2 : c.tile_n;
  // barriers: full/empty per stage, tile-full per accumulator, and
  // tile-empty per accumulator (pair) or per accumulator and 128-row half
  const std::int64_t halves = pair ? 1 : a_rows / 128;
  return std::int64_t(c.stages) * (a_rows * 64 * 2 + 64 * b_cols * 2) + 16384 +
         (2 * c.stages + c.acc_stages + c.acc_stages * halves + 1) * 8 + 16 + 1024;
}

std::int64_t smem_bytes(const FlashAttentionConfig &c, const FlashAttentionProblem &p) noexcept {
  // tile_m 256: Q0, Q1 and a 2-stage K/V ring of 128 x d bf16 tiles;
  // tile_m 128: one Q tile, the K/V ring and the row-statistics exchange
  // (3 KB); plus barriers and alignment slack
  // (tile_n 64, S in 64-key slots: the same tiles, 23 barriers)
  if (c.tile_m == 128) return 5 * 32768 + 3072 + 16 * 8 + 16 + 1024;
  const std::int64_t tile = p.d == 64 ? 16384 : 32768;
  return 6 * tile + (c.tile_n == 64 ? 23 : 16) * 8 + 16 + 1024;
}

LaunchGeometry launch_geometry(const MatmulConfig &c, const MatmulProblem &p) noexcept {
  LaunchGeometry g;
  const std::int64_t tiles = ((p.m + c.tile_m - 1) / c.tile_m) * ((p.n + c.tile_n - 1) / c.tile_n);
  // persistent: one CTA per SM (the CTA pair of tile_m 256: one pair per two SMs)
  const std::int64_t sms = device_sms();
  const bool pair = c.tile_m == 256 && c.cta_group != 1;
  g.grid_x = pair ? int(2 * std::min<std::int64_t>(tiles, sms / 2)) : int(std::min<std::int64_t>(tiles, sms));
  g.block_x = 192;
  g.smem_bytes = int(smem_bytes(c));
  g.tmem_columns = pow2_cols(c.acc_stages * c.tile_n * (c.tile_m == 256 && !pair ? 2 : 1));
  return g;
}

LaunchGeometry launch_geometry(const FlashAttentionConfig &c, const FlashAttentionProblem &p) noexcept {
  LaunchGeometry g;
  g.grid_x = int((p.nq + c.tile_m - 1) / c.tile_m);
  g.grid_y = int(p.batch_heads);
  if (c.tile_m == 256) {  // persistent: one CTA per SM over the (query block, head) items
    g.grid_x = int(std::min<std::int64_t>(std::int64_t(g.grid_x) * g.grid_y, device_sms()));
    g.grid_y = 1;
  }
  const bool tc = fa_tensor_path(c, p.d);
  g.block_x = !tc ? 128 : c.tile_m == 256 ? 384 : 320;
  if (!tc) {
    g.grid_x = int((p.nq + 3) / 4);
    g.grid_y = int(p.batch_heads);
  }
  g.smem_bytes = tc ? int(smem_bytes(c, p)) : 4 * 256 * 4;
  g.tmem_columns = tc ? 512 : 0;
  return g;
}

static std::string sym(const char *fam, const void *cfg) {
  char buf[256] = {0};
  return ks_kernel_symbol(fam, cfg, buf, sizeof(buf)) == KS_OK ? std::string(buf) : std::string();
}
std::string kernel_symbol(const MatmulConfig &c) {
  ks_matmul_config k{c.tile_m, c.tile_n, c.tile_k, c.stages, c.acc_stages, c.group_m, c.cta_group};
  return sym("matmul", &k);
}
std::string kernel_symbol(const FlashAttentionConfig &c) {
  ks_flash_attention_config k{c.tile_m, c.tile_n, c.stages, c.causal ? 1 : 0};
  return sym("flash_attention", &k);
}
std::string kernel_symbol(const SoftmaxConfig &c) {
  ks_softmax_config k{c.block, c.vec_width, int(c.mode)};
  return sym("softmax", &k);
}
std::string kernel_symbol(const LayerNormConfig &c) {
  ks_layernorm_config k{c.block, c.vec_width, int(c.mode)};
  return sym("layernorm", &k);
}
std::string kernel_symbol(const BiasGeluConfig &c) {
  ks_bias_gelu_config k{c.block, c.vec_width, c.gelu};
  return sym("bias_gelu", &k);
}
std::string kernel_symbol(const ReductionConfig &c) {
  ks_reduction_config k{c.block, c.vec_width, int(c.mode)};
  return sym("reduction", &k);
}

// ---------------------------------------------------------------------------
// registry
// ---------------------------------------------------------------------------
namespace {
struct Registry {
  MatmulFamily matmul;
  FlashFamily flash, flash_causal;
  RowFamily softmax{RowKind::kSoftmax, "softmax"};
  RowFamily layernorm{RowKind::kLayerNorm, "layernorm"};
  RowFamily bias_gelu{RowKind::kBiasGelu, "bias_gelu"};
  RowFamily bias_gelu_tanh{RowKind::kBiasGelu, "bias_gelu"};
  RowFamily reduction{RowKind::kReduction, "reduction"};
  Registry() {
    flash_causal.causal = true;
    bias_gelu_tanh.gelu = KS_GELU_TANH;
  }
};
Registry &reg() {
  static Registry r;
  return r;
}
}  // namespace

const Family *find_family(const std::string &name) {
  Registry &r = reg();
  if (name == "matmul") return &r.matmul;
  if (name == "flash_attention" || name == "attention") return &r.flash;
  if (name == "flash_attention:causal") return &r.flash_causal;
  if (name == "softmax") return &r.softmax;
  if (name == "layernorm") return &r.layernorm;
  if (name == "bias_gelu") return &r.bias_gelu;
  if (name == "bias_gelu:tanh") return &r.bias_gelu_tanh;
  if (name == "reduction") return &r.reduction;
  return nullptr;
}

bool golden_case(const std::string &family, const std::vector<std::int64_t> &shape, std::uint64_t seed,
                 const std::map<std::string, std::vector<std::uint16_t>> &inputs,
                 std::map<std::string, std::vector<std::uint16_t>> *used, std::vector<float> *expected,
                 std::string *error) {
  const Family *f = find_family(family);
  if (!f || !f->check_shape(shape, error)) {
    if (error && !f) *error = "unknown family '" + family + "'";
    return false;
  }
  // the session classes with host_only set: generation and reference only
  std::unique_ptr<Session> keep;
  NamedInputs named;
  if (f == find_family("matmul")) {
    auto p = std::make_unique<MatmulSession>();
    p->host_only = true;
    p->init(shape[0], shape[1], shape[2], seed);
    named = p->named();
    keep = std::move(p);
  } else if (f == find_family("flash_attention") || f == find_family("flash_attention:causal")) {
    auto p = std::make_unique<FlashSession>();
    p->host_only = true;
    p->init(fa_shape(shape), f == find_family("flash_attention:causal"), seed);
    named = p->named();
    keep = std::move(p);
  } else {
    const auto *rf = static_cast<const RowFamily *>(f);
    if (rf->kind == RowKind::kReduction && shape.size() == 1) {
      if (error) *error = "the full fp32 sum has no bf16 golden case";
      return false;
    }
    auto p = std::make_unique<RowSession>();
    p->host_only = true;
    p->init(rf->kind, shape[0], shape[1], rf->gelu, 0, seed);
    named = p->named();
    keep = std::move(p);
  }
  for (auto &[name, buf] : named) {
    if (auto it = inputs.find(name); it != inputs.end()) {
      if (it->second.size() != buf->bits.size()) {
        if (error) *error = std::string("input '") + name + "' has " + std::to_string(it->second.size()) +
                            " elements, the shape needs " + std::to_string(buf->bits.size());
        return false;
      }
      buf->set_bits(it->second);
    }
    if (used) (*used)[name] = buf->bits;
  }
  keep->reference(expected);
  return true;
}

const std::vector<std::string> &family_names() {
  static const std::vector<std::string> n{"matmul", "bias_gelu", "softmax", "layernorm", "reduction",
                                          "flash_attention"};
  return n;
}

}  // namespace kernscope::tune
