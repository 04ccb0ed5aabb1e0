// golden.cpp -- the reference's golden inputs, references and verdict (see
// golden.h for the algorithms and the reference lines they follow).
#include "golden.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace kernscope::tune::golden {

namespace {

// SeedSequence constants: the pool-hash and output-hash multipliers and
// their starting values, and the two-word mixing multipliers (32-bit
// arithmetic throughout, xor-shift by half a word).
constexpr std::uint32_t kPoolHashInit = 0x43b0d7e5u, kPoolHashMul = 0x931e8875u;
constexpr std::uint32_t kOutHashInit = 0x8b51f9ddu, kOutHashMul = 0x58f38dedu;
constexpr std::uint32_t kMixLeft = 0xca01f9ddu, kMixRight = 0x4973f715u;
constexpr int kPoolWords = 4;

struct PoolHash {
  std::uint32_t k = kPoolHashInit;
  std::uint32_t operator()(std::uint32_t v) {
    v ^= k;
    k *= kPoolHashMul;
    v *= k;
    return v ^ (v >> 16);
  }
};

std::uint32_t mix2(std::uint32_t x, std::uint32_t y) {
  const std::uint32_t r = kMixLeft * x - kMixRight * y;
  return r ^ (r >> 16);
}

// PCG64's LCG multiplier (128 bits).
const unsigned __int128 kPcgMul = (static_cast<unsigned __int128>(0x2360ED051FC65DA4ull) << 64) | 0x4385DF649FCCF645ull;

}  // namespace

std::vector<std::uint32_t> seed_words(std::uint64_t seed) {
  if (seed == 0) return {0u};
  std::vector<std::uint32_t> w;
  for (; seed != 0; seed >>= 32) w.push_back(std::uint32_t(seed & 0xffffffffu));
  return w;
}

Generator::Generator(std::uint64_t seed) : Generator(seed_words(seed)) {}

Generator::Generator(const std::vector<std::uint32_t> &words) {
  // 1. hash the seed words into the pool; later words mix into every slot
  std::uint32_t pool[kPoolWords];
  PoolHash h;
  for (int i = 0; i < kPoolWords; ++i) pool[i] = h(i < int(words.size()) ? words[size_t(i)] : 0u);
  for (int s = 0; s < kPoolWords; ++s)
    for (int d = 0; d < kPoolWords; ++d)
      if (s != d) pool[d] = mix2(pool[d], h(pool[s]));
  for (size_t s = kPoolWords; s < words.size(); ++s)
    for (int d = 0; d < kPoolWords; ++d) pool[d] = mix2(pool[d], h(words[s]));
  // 2. hash the pool out into four 64-bit words (pairs of 32-bit words,
  //    low word first)
  std::uint64_t st[4];
  std::uint32_t k = kOutHashInit;
  for (int i = 0; i < 8; ++i) {
    std::uint32_t v = pool[i % kPoolWords] ^ k;
    k *= kOutHashMul;
    v *= k;
    v ^= v >> 16;
    if (i % 2 == 0)
      st[i / 2] = v;
    else
      st[i / 2] |= std::uint64_t(v) << 32;
  }
  // 3. PCG64 seeding: words 0-1 are the initial state (high, low), words
  //    2-3 the stream selector; the increment is odd
  const unsigned __int128 init = (static_cast<unsigned __int128>(st[0]) << 64) | st[1];
  const unsigned __int128 seq = (static_cast<unsigned __int128>(st[2]) << 64) | st[3];
  state_ = 0;
  inc_ = (seq << 1) | 1u;
  step();
  state_ += init;
  step();
}

void Generator::step() { state_ = state_ * kPcgMul + inc_; }

std::uint64_t Generator::next_u64() {
  step();
  // XSL-RR: xor the halves, rotate right by the top six bits
  const std::uint64_t x = std::uint64_t(state_ >> 64) ^ std::uint64_t(state_);
  const unsigned r = unsigned(state_ >> 122);
  return (x >> r) | (x << ((64u - r) & 63u));
}

std::uint16_t to_bf16_bits(float f) {
  std::uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return std::uint16_t((u >> 16) | 0x40u);
  return std::uint16_t((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

float from_bf16_bits(std::uint16_t h) {
  const std::uint32_t u = std::uint32_t(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

std::vector<std::uint16_t> draw_bf16(Generator &g, std::size_t n, double lo, double hi) {
  std::vector<std::uint16_t> out(n);
  for (auto &b : out) b = to_bf16_bits(float(g.uniform(lo, hi)));
  return out;
}

float pairwise_sum(const float *a, std::int64_t n) {
  if (n < 8) {
    float r = 0.f;
    for (std::int64_t i = 0; i < n; ++i) r += a[i];
    return r;
  }
  if (n <= 128) {
    float r[8];
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    std::int64_t i = 8;
    for (; i < n - (n % 8); i += 8)
      for (int j = 0; j < 8; ++j) r[j] += a[i + j];
    float s = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) s += a[i];
    return s;
  }
  std::int64_t h = n / 2;
  h -= h % 8;
  return pairwise_sum(a, h) + pairwise_sum(a + h, n - h);
}

static float row_sum(const float *a, std::int64_t n) { return 0.f + pairwise_sum(a, n); }

void matmul(const float *a, const float *b, std::int64_t m, std::int64_t n, std::int64_t k, float *out) {
  std::vector<float> acc(static_cast<size_t>(n));
  for (std::int64_t i = 0; i < m; ++i) {
    std::fill(acc.begin(), acc.end(), 0.f);
    for (std::int64_t kk = 0; kk < k; ++kk) {
      const float av = a[i * k + kk];
      const float *brow = b + kk * n;
      for (std::int64_t j = 0; j < n; ++j) acc[size_t(j)] += av * brow[j];
    }
    for (std::int64_t j = 0; j < n; ++j) out[i * n + j] = round_bf16(acc[size_t(j)]);
  }
}

void softmax(const float *x, std::int64_t rows, std::int64_t cols, float *out) {
  std::vector<float> e(static_cast<size_t>(cols));
  for (std::int64_t r = 0; r < rows; ++r) {
    const float *xr = x + r * cols;
    float mx = -INFINITY;
    for (std::int64_t c = 0; c < cols; ++c) mx = std::max(mx, xr[c]);
    for (std::int64_t c = 0; c < cols; ++c) e[size_t(c)] = std::exp(xr[c] - mx);
    const float s = row_sum(e.data(), cols);
    for (std::int64_t c = 0; c < cols; ++c) out[r * cols + c] = round_bf16(e[size_t(c)] / s);
  }
}

void layernorm(const float *x, const float *gamma, const float *beta, std::int64_t rows, std::int64_t cols,
               float eps, float *out) {
  std::vector<float> d(static_cast<size_t>(cols));
  const float n = float(cols);
  for (std::int64_t r = 0; r < rows; ++r) {
    const float *xr = x + r * cols;
    const float mu = row_sum(xr, cols) / n;
    for (std::int64_t c = 0; c < cols; ++c) {
      const float t = xr[c] - mu;
      d[size_t(c)] = t * t;
    }
    const float var = row_sum(d.data(), cols) / n;
    const float sd = std::sqrt(var + eps);
    for (std::int64_t c = 0; c < cols; ++c) {
      const float z = (xr[c] - mu) / sd;
      const float zg = z * gamma[c];
      out[r * cols + c] = round_bf16(zg + beta[c]);
    }
  }
}

void bias_gelu(const float *x, const float *bias, std::int64_t rows, std::int64_t cols, bool tanh_form,
               float *out) {
  const float inv_sqrt2 = float(1.0 / std::sqrt(2.0));
  for (std::int64_t i = 0; i < rows * cols; ++i) {
    const float t = round_bf16(x[i] + bias[i % cols]);
    if (tanh_form) {
      const double td = t;
      const double u = std::sqrt(2.0 / M_PI) * (td + 0.044715 * td * td * td);
      out[i] = round_bf16(float(0.5 * td * (1.0 + std::tanh(u))));
    } else {
      const float arg = t * inv_sqrt2;
      const float e = float(std::erf(double(arg)));
      const float half_t = 0.5f * t;
      out[i] = round_bf16(half_t * (1.f + e));
    }
  }
}

void reduction_axis0(const float *x, std::int64_t rows, std::int64_t cols, float *out) {
  std::vector<float> acc(static_cast<size_t>(cols), 0.f);
  for (std::int64_t r = 0; r < rows; ++r)
    for (std::int64_t c = 0; c < cols; ++c) acc[size_t(c)] += x[r * cols + c];
  for (std::int64_t c = 0; c < cols; ++c) out[c] = round_bf16(acc[size_t(c)]);
}

void attention(const float *q, const float *k, const float *v, std::int64_t nq, std::int64_t nk, std::int64_t d,
               bool causal, float *out) {
  const float sd = float(std::sqrt(double(d)));
  std::vector<float> s(static_cast<size_t>(nk)), acc(static_cast<size_t>(d));
  for (std::int64_t i = 0; i < nq; ++i) {
    const float *qi = q + i * d;
    float mx = -INFINITY;
    for (std::int64_t j = 0; j < nk; ++j) {
      const float *kj = k + j * d;
      float dot = 0.f;
      for (std::int64_t c = 0; c < d; ++c) dot += qi[c] * kj[c];
      s[size_t(j)] = (causal && j > i) ? -INFINITY : dot / sd;
      mx = std::max(mx, s[size_t(j)]);
    }
    for (std::int64_t j = 0; j < nk; ++j) s[size_t(j)] = std::exp(s[size_t(j)] - mx);
    const float sum = row_sum(s.data(), nk);
    std::fill(acc.begin(), acc.end(), 0.f);
    for (std::int64_t j = 0; j < nk; ++j) {
      const float p = s[size_t(j)] / sum;
      const float *vj = v + j * d;
      for (std::int64_t c = 0; c < d; ++c) acc[size_t(c)] += p * vj[c];
    }
    for (std::int64_t c = 0; c < d; ++c) out[i * d + c] = round_bf16(acc[size_t(c)]);
  }
}

Verdict verdict(const std::vector<float> &got, const std::vector<float> &ref) {
  Verdict v;
  const size_t n = std::min(got.size(), ref.size());
  double dot = 0, na = 0, nr = 0, ma = 0, mr = 0;
  float mre = 0.f;
  bool equal = got.size() == ref.size();
  for (size_t i = 0; i < n; ++i) {
    const double a = got[i], r = ref[i];
    dot += a * r;
    na += a * a;
    nr += r * r;
    ma += a;
    mr += r;
    equal = equal && got[i] == ref[i];
    // fp32, as numpy evaluates |x - y| / (|y| + eps) on float32 views
    const float e = std::fabs(got[i] - ref[i]) / (std::fabs(ref[i]) + 1e-6f);
    mre = std::isnan(e) ? e : std::max(mre, e);
  }
  const double nx = std::sqrt(na), ny = std::sqrt(nr);
  v.cosine = nx * ny == 0.0 ? (nx == 0.0 && ny == 0.0 ? 1.0 : 0.0) : dot / (nx * ny);
  v.max_rel_err = mre;
  ma /= double(std::max<size_t>(n, 1));
  mr /= double(std::max<size_t>(n, 1));
  double sxy = 0, sxx = 0, syy = 0;
  for (size_t i = 0; i < n; ++i) {
    sxy += (got[i] - ma) * (ref[i] - mr);
    sxx += (got[i] - ma) * (got[i] - ma);
    syy += (ref[i] - mr) * (ref[i] - mr);
  }
  const double den = std::sqrt(sxx) * std::sqrt(syy);
  v.pcc = den == 0.0 ? (equal ? 1.0 : 0.0) : sxy / den;
  // inclusive thresholds (metrics.py:92-116); NaN fails every comparison
  v.pass = v.cosine >= 0.999 && v.max_rel_err <= 1e-2 && v.pcc >= 0.99;
  return v;
}

}  // namespace kernscope::tune::golden
