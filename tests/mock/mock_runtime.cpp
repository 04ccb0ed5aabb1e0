// mock_runtime.cpp -- a test double of the device half of libkernscope_b200's
// C ABI, for CPU tests of the tuner host code (the role of the reference's
// MockRuntime, libs/gpuruntime/include/kernscope/gpu.h:257-330, and of the
// StubRuntime its bench tests use, libs/bench/tests/bench_test.cpp).
//
// Test infrastructure only.  It is preloaded (LD_PRELOAD) into a process
// that uses the tuner, so the tuner's calls of ks_gpu_* and ks_<family>_launch
// land here; everything else (validation, kernel symbols, status strings,
// workspace sizes) still resolves to the real library.
//
//   * one device, "sm_100a", 148 SMs, 126 MB L2;
//   * device memory is host memory; buffers above 64 MiB (the bench's L2
//     flush buffer) get no backing store and their memsets are recorded only;
//   * a launch validates its config with the real ks_<family>_validate and
//     then computes the family's result on the CPU (plain loops, fp64
//     accumulation, bf16 rounding once), so the tuner's golden gate sees
//     correct outputs;
//   * time is a fake clock: each launch advances it by the kernel's
//     duration, events read it.  KS_MOCK_TIMES="symbol=ms,..." sets the
//     duration per kernel symbol (default 1 ms);
//   * failure injection: KS_MOCK_ZERO=<symbol> makes that kernel write zeros
//     (the gate must reject it); KS_MOCK_FAIL=<symbol>:<n> makes its n-th
//     launch and every later one fail with KS_ERR_LAUNCH; KS_MOCK_DEVICES
//     sets the device count (0 = no device);
//   * KS_MOCK_LOG=<path> appends one JSON line per operation (the op log);
//   * KS_MOCK_REAL_LIB=<path> names the real libkernscope_b200.so, whose
//     validation and symbol functions the launches call (it is usually
//     loaded RTLD_LOCAL, so they are looked up through its handle).
#include <dlfcn.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "kernscope_b200.h"

namespace {

std::mutex g_mu;
std::set<void *> g_small;              // buffers with host backing
std::map<void *, size_t> g_virtual;    // large buffers without backing (fake addresses)
std::uintptr_t g_next_virtual = 0x7e0000000000ull;
double g_clock_ms = 0.0;
std::map<std::string, int> g_launches;  // per symbol
FILE *g_log = nullptr;
bool g_log_opened = false;

constexpr size_t kVirtualAbove = 64ull << 20;

void log_op(const char *op, const std::string &detail, size_t bytes = 0) {
  if (!g_log_opened) {
    g_log_opened = true;
    if (const char *p = std::getenv("KS_MOCK_LOG")) g_log = std::fopen(p, "a");
  }
  if (!g_log) return;
  std::fprintf(g_log, "{\"op\":\"%s\",\"detail\":\"%s\",\"bytes\":%zu,\"clock_ms\":%.6f}\n", op, detail.c_str(),
               bytes, g_clock_ms);
  std::fflush(g_log);
}

std::string env_str(const char *k) {
  const char *v = std::getenv(k);
  return v ? v : "";
}

double duration_ms(const std::string &symbol) {
  const std::string t = env_str("KS_MOCK_TIMES");
  size_t pos = 0;
  while (pos < t.size()) {
    size_t comma = t.find(',', pos);
    if (comma == std::string::npos) comma = t.size();
    const std::string item = t.substr(pos, comma - pos);
    const size_t eq = item.find('=');
    if (eq != std::string::npos && item.substr(0, eq) == symbol) return std::atof(item.c_str() + eq + 1);
    pos = comma + 1;
  }
  return 1.0;
}

// 0: run normally; 1: write zeros; 2: fail the launch
int injected(const std::string &symbol) {
  if (env_str("KS_MOCK_ZERO") == symbol) return 1;
  const std::string f = env_str("KS_MOCK_FAIL");
  const size_t colon = f.rfind(':');
  if (colon != std::string::npos && f.substr(0, colon) == symbol) {
    const int n = std::atoi(f.c_str() + colon + 1);
    if (g_launches[symbol] >= n) return 2;
  }
  return 0;
}

// bf16 <-> fp32, round to nearest even
float bf(uint16_t h) {
  uint32_t u = uint32_t(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
uint16_t to_bf(double d) {
  const float f = float(d);
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
// A function of the real library, looked up by name.
template <class Fn>
Fn real(const char *name) {
  static void *h = [] {
    const char *p = std::getenv("KS_MOCK_REAL_LIB");
    void *hh = p ? dlopen(p, RTLD_NOW | RTLD_LOCAL) : nullptr;
    if (!hh) {
      std::fprintf(stderr, "mock_runtime: cannot open KS_MOCK_REAL_LIB (%s)\n", p ? p : "unset");
      std::abort();
    }
    return hh;
  }();
  void *f = dlsym(h, name);
  if (!f) {
    std::fprintf(stderr, "mock_runtime: %s not found in the real library\n", name);
    std::abort();
  }
  return reinterpret_cast<Fn>(f);
}
#define REAL(name) real<decltype(&name)>(#name)

const uint16_t *H(const void *p) { return static_cast<const uint16_t *>(p); }
uint16_t *Hm(void *p) { return static_cast<uint16_t *>(p); }

// Common launch bookkeeping: the real validation result, the symbol, the
// injected behaviour and the fake clock.  Returns KS_OK to compute, 1 to
// write zeros, or a negative status.
int begin_launch(const char *family, const void *cfg, int valid_status, size_t out_bytes, void *out) {
  if (valid_status != KS_OK) return valid_status;
  char sym[256] = {0};
  REAL(ks_kernel_symbol)(family, cfg, sym, sizeof(sym));
  std::lock_guard<std::mutex> lk(g_mu);
  const std::string s(sym);
  const int inj = injected(s);
  if (inj == 2) {
    log_op("launch_failed", s);
    return KS_ERR_LAUNCH;
  }
  ++g_launches[s];
  g_clock_ms += duration_ms(s);
  log_op("launch", s);
  if (inj == 1) {
    if (out && g_small.count(out)) std::memset(out, 0, out_bytes);
    return 1;
  }
  return KS_OK;
}

}  // namespace

extern "C" {

int ks_gpu_device_count(int *count) {
  const std::string v = env_str("KS_MOCK_DEVICES");
  *count = v.empty() ? 1 : std::atoi(v.c_str());
  log_op("device_count", std::to_string(*count));
  return KS_OK;
}
int ks_gpu_set_device(int device) {
  int n = 0;
  ks_gpu_device_count(&n);
  return device < n ? KS_OK : KS_ERR_DEVICE_NOT_FOUND;
}
int ks_gpu_get_device(int *device) {
  *device = 0;
  return KS_OK;
}
int ks_gpu_arch(int device, char *buf, size_t len) {
  (void)device;
  std::snprintf(buf, len, "sm_100a");
  return KS_OK;
}
int ks_gpu_l2_bytes(int device, size_t *bytes) {
  (void)device;
  *bytes = 126ull << 20;
  return KS_OK;
}
int ks_gpu_malloc(void **ptr, size_t bytes) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (bytes > kVirtualAbove) {
    *ptr = reinterpret_cast<void *>(g_next_virtual);
    g_next_virtual += (bytes + 4095) & ~size_t(4095);
    g_virtual[*ptr] = bytes;
  } else {
    *ptr = std::calloc(1, bytes ? bytes : 1);
    if (!*ptr) return KS_ERR_MEMORY;
    g_small.insert(*ptr);
  }
  log_op("malloc", "", bytes);
  return KS_OK;
}
int ks_gpu_free(void *ptr) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_small.erase(ptr)) {
    std::free(ptr);
  } else if (!g_virtual.erase(ptr) && ptr) {
    return KS_ERR_MEMORY;
  }
  log_op("free", "");
  return KS_OK;
}
int ks_gpu_memset(void *ptr, int value, size_t bytes, void *stream) {
  (void)stream;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_small.count(ptr)) std::memset(ptr, value, bytes);
  log_op("memset", g_virtual.count(ptr) ? "virtual" : "", bytes);
  return KS_OK;
}
int ks_gpu_memcpy_htod(void *dst, const void *src, size_t bytes, void *stream) {
  (void)stream;
  std::lock_guard<std::mutex> lk(g_mu);
  std::memcpy(dst, src, bytes);
  log_op("memcpy_htod", "", bytes);
  return KS_OK;
}
int ks_gpu_memcpy_dtoh(void *dst, const void *src, size_t bytes, void *stream) {
  (void)stream;
  std::lock_guard<std::mutex> lk(g_mu);
  std::memcpy(dst, src, bytes);
  log_op("memcpy_dtoh", "", bytes);
  return KS_OK;
}
int ks_gpu_stream_create(void **stream) {
  *stream = std::malloc(1);
  log_op("stream_create", "");
  return KS_OK;
}
int ks_gpu_stream_destroy(void *stream) {
  std::free(stream);
  log_op("stream_destroy", "");
  return KS_OK;
}
int ks_gpu_stream_synchronize(void *stream) {
  (void)stream;
  log_op("stream_synchronize", "");
  return KS_OK;
}
int ks_gpu_synchronize(void) {
  log_op("synchronize", "");
  return KS_OK;
}
int ks_gpu_event_create(void **event) {
  *event = new double(0.0);
  return KS_OK;
}
int ks_gpu_event_destroy(void *event) {
  delete static_cast<double *>(event);
  return KS_OK;
}
int ks_gpu_event_record(void *event, void *stream) {
  (void)stream;
  std::lock_guard<std::mutex> lk(g_mu);
  *static_cast<double *>(event) = g_clock_ms;
  log_op("event_record", "");
  return KS_OK;
}
int ks_gpu_event_synchronize(void *event) {
  (void)event;
  return KS_OK;
}
int ks_gpu_event_elapsed_ms(void *start, void *stop, float *ms) {
  *ms = float(*static_cast<double *>(stop) - *static_cast<double *>(start));
  return KS_OK;
}

int ks_softmax_launch(const ks_softmax_config *cfg, const ks_softmax_args *a, void *stream) {
  (void)stream;
  const int64_t R = a->rows, C = a->cols;
  const int st = begin_launch("softmax", cfg, REAL(ks_softmax_validate)(cfg, R, C, nullptr, 0), size_t(R * C) * 2, a->out);
  if (st != KS_OK) return st > 0 ? KS_OK : st;
  for (int64_t r = 0; r < R; ++r) {
    const uint16_t *x = H(a->x) + r * C;
    double m = -INFINITY, s = 0.0;
    for (int64_t c = 0; c < C; ++c) m = std::fmax(m, bf(x[c]));
    for (int64_t c = 0; c < C; ++c) s += std::exp(bf(x[c]) - m);
    for (int64_t c = 0; c < C; ++c) Hm(a->out)[r * C + c] = to_bf(std::exp(bf(x[c]) - m) / s);
  }
  return KS_OK;
}

int ks_layernorm_launch(const ks_layernorm_config *cfg, const ks_layernorm_args *a, void *stream) {
  (void)stream;
  const int64_t R = a->rows, C = a->cols;
  const int st =
      begin_launch("layernorm", cfg, REAL(ks_layernorm_validate)(cfg, R, C, nullptr, 0), size_t(R * C) * 2, a->out);
  if (st != KS_OK) return st > 0 ? KS_OK : st;
  const double eps = a->eps > 0.f ? a->eps : 1e-5;
  for (int64_t r = 0; r < R; ++r) {
    const uint16_t *x = H(a->x) + r * C;
    double mean = 0.0, var = 0.0;
    for (int64_t c = 0; c < C; ++c) mean += bf(x[c]);
    mean /= double(C);
    for (int64_t c = 0; c < C; ++c) var += (bf(x[c]) - mean) * (bf(x[c]) - mean);
    var /= double(C);
    const double rstd = 1.0 / std::sqrt(var + eps);
    for (int64_t c = 0; c < C; ++c)
      Hm(a->out)[r * C + c] = to_bf((bf(x[c]) - mean) * rstd * bf(H(a->gamma)[c]) + bf(H(a->beta)[c]));
  }
  return KS_OK;
}

int ks_bias_gelu_launch(const ks_bias_gelu_config *cfg, const ks_bias_gelu_args *a, void *stream) {
  (void)stream;
  const int st = begin_launch("bias_gelu", cfg, REAL(ks_bias_gelu_validate)(cfg, a->total, a->cols, nullptr, 0),
                              size_t(a->total) * 2, a->out);
  if (st != KS_OK) return st > 0 ? KS_OK : st;
  for (int64_t i = 0; i < a->total; ++i) {
    const double t = bf(to_bf(double(bf(H(a->x)[i])) + bf(H(a->bias)[i % a->cols])));
    const double y = cfg->gelu == KS_GELU_TANH
                         ? 0.5 * t * (1.0 + std::tanh(std::sqrt(2.0 / M_PI) * (t + 0.044715 * t * t * t)))
                         : 0.5 * t * (1.0 + std::erf(t / std::sqrt(2.0)));
    Hm(a->out)[i] = to_bf(y);
  }
  return KS_OK;
}

int ks_reduction_launch(const ks_reduction_config *cfg, const ks_reduction_args *a, void *stream) {
  (void)stream;
  const bool full = a->axis != 0;
  const size_t out_bytes = full ? 4 : size_t(a->cols) * (a->out_dtype == KS_F32 ? 4 : 2);
  const int st = begin_launch("reduction", cfg, REAL(ks_reduction_validate)(cfg, a, nullptr, 0), out_bytes, a->out);
  if (st != KS_OK) return st > 0 ? KS_OK : st;
  auto in = [&](int64_t i) {
    return a->in_dtype == KS_F32 ? double(static_cast<const float *>(a->x)[i]) : double(bf(H(a->x)[i]));
  };
  if (full) {
    double s = 0.0;
    for (int64_t i = 0; i < a->rows * a->cols; ++i) s += in(i);
    *static_cast<float *>(a->out) = float(s);
    if (a->partial_f64) *a->partial_f64 = s;
    return KS_OK;
  }
  for (int64_t c = 0; c < a->cols; ++c) {
    double s = 0.0;
    for (int64_t r = 0; r < a->rows; ++r) s += in(r * a->cols + c);
    if (a->out_dtype == KS_F32) static_cast<float *>(a->out)[c] = float(s);
    else Hm(a->out)[c] = to_bf(s);
  }
  return KS_OK;
}

int ks_matmul_launch(const ks_matmul_config *cfg, const ks_matmul_args *a, void *stream) {
  (void)stream;
  const int64_t M = a->m, N = a->n, K = a->k;
  const int st =
      begin_launch("matmul", cfg, REAL(ks_matmul_validate)(cfg, M, N, K, nullptr, 0), size_t(M * N) * 2, a->out);
  if (st != KS_OK) return st > 0 ? KS_OK : st;
  std::vector<double> row(static_cast<size_t>(N));
  for (int64_t i = 0; i < M; ++i) {
    std::fill(row.begin(), row.end(), 0.0);
    for (int64_t k = 0; k < K; ++k) {
      const double av = bf(H(a->a)[i * K + k]);
      const uint16_t *b = H(a->b) + k * N;
      for (int64_t j = 0; j < N; ++j) row[size_t(j)] += av * bf(b[j]);
    }
    for (int64_t j = 0; j < N; ++j) Hm(a->out)[i * N + j] = to_bf(row[size_t(j)]);
  }
  return KS_OK;
}

int ks_flash_attention_launch(const ks_flash_attention_config *cfg, const ks_flash_attention_args *a, void *stream) {
  (void)stream;
  const int64_t BH = a->batch * a->heads, NQ = a->nq, NK = a->nk, D = a->d;
  const int st = begin_launch("flash_attention", cfg, REAL(ks_flash_attention_validate)(cfg, a, nullptr, 0),
                              size_t(BH * NQ * D) * 2, a->out);
  if (st != KS_OK) return st > 0 ? KS_OK : st;
  const double scale = a->scale > 0.f ? a->scale : 1.0 / std::sqrt(double(D));
  std::vector<double> p(static_cast<size_t>(NK));
  for (int64_t h = 0; h < BH; ++h)
    for (int64_t i = 0; i < NQ; ++i) {
      const uint16_t *q = H(a->q) + (h * NQ + i) * D;
      double m = -INFINITY, s = 0.0;
      for (int64_t j = 0; j < NK; ++j) {
        double dot = 0.0;
        const uint16_t *k = H(a->k) + (h * NK + j) * D;
        for (int64_t e = 0; e < D; ++e) dot += double(bf(q[e])) * bf(k[e]);
        p[size_t(j)] = (cfg->causal && j > i) ? -INFINITY : dot * scale;
        m = std::fmax(m, p[size_t(j)]);
      }
      for (int64_t j = 0; j < NK; ++j) s += (p[size_t(j)] = std::exp(p[size_t(j)] - m));
      for (int64_t e = 0; e < D; ++e) {
        double o = 0.0;
        for (int64_t j = 0; j < NK; ++j) o += p[size_t(j)] * bf(H(a->v)[(h * NK + j) * D + e]);
        Hm(a->out)[(h * NQ + i) * D + e] = to_bf(o / s);
      }
    }
  return KS_OK;
}

}  // extern "C"
