// golden.h -- the reference's golden gate on the host: its seeded inputs bit
// for bit, its CPU references in its operation order, and its verdict.
//
// The reference gate (tools/tune/src/driver_pipeline_impl.h:1223-1235 ->
// kernels/templates/tests/run_hip_gate.py:81-213) generates the inputs with
// tests/golden/kernscope_golden/inputs.py:73-106 (one numpy Generator,
// np.random.default_rng(seed), float64 uniform draws in a fixed order, each
// rounded to bf16 through float32), computes the expected bf16 output with
// refs.py:54-142 (fp32 arithmetic, one rounding to bf16), and judges with
// metrics.py:92-116 (cosine >= 0.999, max_rel_err <= 1e-2 with eps 1e-6,
// pcc >= 0.99, all inclusive).  The tuner's in-process gate uses this file,
// so it judges every config on the reference's own inputs and criterion.
//
// The generator restates the published algorithms numpy's default_rng is
// built from (numpy >= 1.17; checked against numpy 2.3 in the CPU tests):
//   * SeedSequence (O'Neill's seed_seq design as adopted by numpy): the seed
//     as little-endian 32-bit words is hashed into a 4-word pool, and the
//     pool is hashed out into the bit generator's initial words;
//   * PCG64 (O'Neill 2014, "PCG: A Family of Simple Fast Space-Efficient
//     Statistically Good Algorithms for Random Number Generation"): a
//     128-bit LCG with the XSL-RR 128/64 output function;
//   * uniform(lo, hi) = lo + (hi - lo) * ((x >> 11) * 2^-53).
#pragma once

#include <cstdint>
#include <vector>

namespace kernscope::tune::golden {

// numpy.random.default_rng(seed) as a stream of 64-bit outputs and uniform
// doubles.  `words` is the seed as numpy's SeedSequence sees it: a
// non-negative integer split into little-endian 32-bit words ([0] for 0), or
// the concatenation of those words for a list of integers.
class Generator {
 public:
  explicit Generator(std::uint64_t seed);
  explicit Generator(const std::vector<std::uint32_t> &words);
  std::uint64_t next_u64();
  double next_double() { return double(next_u64() >> 11) * 0x1.0p-53; }
  double uniform(double lo, double hi) { return lo + (hi - lo) * next_double(); }

 private:
  unsigned __int128 state_ = 0, inc_ = 0;
  void step();
};

// The seed of an integer as SeedSequence's 32-bit words.
std::vector<std::uint32_t> seed_words(std::uint64_t seed);

// bf16 round-to-nearest-even of a float (NaN stays NaN), and back.
std::uint16_t to_bf16_bits(float f);
float from_bf16_bits(std::uint16_t h);
inline float round_bf16(float f) { return from_bf16_bits(to_bf16_bits(f)); }

// n uniform(lo, hi) draws rounded like inputs.py's to_bf16: float64 ->
// float32 (round to nearest) -> bf16 (round to nearest even).
std::vector<std::uint16_t> draw_bf16(Generator &g, std::size_t n, double lo, double hi);

// numpy's add.reduce of a contiguous float32 row: 0 + pairwise sum (blocks
// of eight running sums up to 128 elements, halves split at a multiple of
// eight above), which is what np.sum(x, axis=-1) and x.mean(axis=-1)
// accumulate in fp32.
float pairwise_sum(const float *a, std::int64_t n);

// --- references (refs.py), fp32 inputs holding bf16 values, outputs rounded
// to bf16 once (returned as fp32 holding bf16 values) ------------------------
// refs.py:54-56; the fp32 product is accumulated in K order.
void matmul(const float *a, const float *b, std::int64_t m, std::int64_t n, std::int64_t k, float *out);
// refs.py:79-84: exp(x - max) / (pairwise) sum.
void softmax(const float *x, std::int64_t rows, std::int64_t cols, float *out);
// refs.py:87-99: mean and biased variance as fp32 pairwise means,
// (x - mu) / sqrt(var + eps) * gamma + beta.
void layernorm(const float *x, const float *gamma, const float *beta, std::int64_t rows, std::int64_t cols,
               float eps, float *out);
// refs.py:59-76: t = bf16(x + bias); 0.5 t (1 + erf(t * fp32(1/sqrt 2)))
// with erf in double cast to fp32 (tanh = true: the tanh-approximation
// extension, computed in double and rounded once).
void bias_gelu(const float *x, const float *bias, std::int64_t rows, std::int64_t cols, bool tanh_form,
               float *out);
// refs.py:102-110: column sums, rows added in order.
void reduction_axis0(const float *x, std::int64_t rows, std::int64_t cols, float *out);
// refs.py:113-142, one head: S = Q K^T / fp32(sqrt d), causal masks col >
// row, exp(S - max) / pairwise sum, O = P V.
void attention(const float *q, const float *k, const float *v, std::int64_t nq, std::int64_t nk, std::int64_t d,
               bool causal, float *out);

// metrics.py:29-116 over flattened fp32 views.
struct Verdict {
  bool pass = false;
  double cosine = 0.0, max_rel_err = 0.0, pcc = 0.0;
};
Verdict verdict(const std::vector<float> &got, const std::vector<float> &ref);

}  // namespace kernscope::tune::golden
