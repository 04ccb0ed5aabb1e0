// rowops.cu -- softmax, layernorm and bias_gelu for sm_100a.
//
// All three are HBM-bound: 2 bytes read + 2 bytes written per element (plus
// gamma/beta/bias, read once per CTA and served by L1/L2 afterwards).  The
// kernels use 128-bit vector loads/stores (vec_width 8 bf16), keep the
// working row in registers (ONEPASS) so HBM sees each byte once, reduce with
// warp shuffles plus one shared-memory exchange, and run a grid sized to the
// resident-CTA capacity of the 148 SMs with a grid-stride loop over rows.
//
// Semantics follow the reference templates / goldens:
//   softmax   y = exp(x - max) / sum(exp(x - max))           refs.py:79-84
//   layernorm y = (x - mean)/sqrt(var + eps)*gamma + beta     refs.py:87-99
//   bias_gelu y = GELU(bf16(x + bias[i % cols]))              refs.py:66-76
#include <cfloat>
#include <cmath>

#include "ks_common.cuh"

namespace {

constexpr float kLog2e = 1.4426950408889634f;

KS_DEV float ks_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- vector access of VEC consecutive bf16 (VEC in {1,2,4,8}) -------------
template <int VEC>
KS_DEV void load_bf16(const uint16_t *p, float (&v)[VEC]) {
  if constexpr (VEC == 8) {
    uint4 w = __ldcs(reinterpret_cast<const uint4 *>(p));
    v[0] = ks_bf16_lo(w.x); v[1] = ks_bf16_hi(w.x); v[2] = ks_bf16_lo(w.y); v[3] = ks_bf16_hi(w.y);
    v[4] = ks_bf16_lo(w.z); v[5] = ks_bf16_hi(w.z); v[6] = ks_bf16_lo(w.w); v[7] = ks_bf16_hi(w.w);
  } else if constexpr (VEC == 4) {
    uint2 w = __ldcs(reinterpret_cast<const uint2 *>(p));
    v[0] = ks_bf16_lo(w.x); v[1] = ks_bf16_hi(w.x); v[2] = ks_bf16_lo(w.y); v[3] = ks_bf16_hi(w.y);
  } else if constexpr (VEC == 2) {
    uint32_t w = __ldcs(reinterpret_cast<const unsigned int *>(p));
    v[0] = ks_bf16_lo(w); v[1] = ks_bf16_hi(w);
  } else {
    v[0] = ks_bf16_to_f32(__ldcs(reinterpret_cast<const unsigned short *>(p)));
  }
}
// Read-only parameter vectors (gamma/beta/bias): keep them cached.
template <int VEC>
KS_DEV void load_bf16_cached(const uint16_t *p, float (&v)[VEC]) {
  if constexpr (VEC == 8) {
    uint4 w = __ldg(reinterpret_cast<const uint4 *>(p));
    v[0] = ks_bf16_lo(w.x); v[1] = ks_bf16_hi(w.x); v[2] = ks_bf16_lo(w.y); v[3] = ks_bf16_hi(w.y);
    v[4] = ks_bf16_lo(w.z); v[5] = ks_bf16_hi(w.z); v[6] = ks_bf16_lo(w.w); v[7] = ks_bf16_hi(w.w);
  } else if constexpr (VEC == 4) {
    uint2 w = __ldg(reinterpret_cast<const uint2 *>(p));
    v[0] = ks_bf16_lo(w.x); v[1] = ks_bf16_hi(w.x); v[2] = ks_bf16_lo(w.y); v[3] = ks_bf16_hi(w.y);
  } else if constexpr (VEC == 2) {
    uint32_t w = __ldg(reinterpret_cast<const unsigned int *>(p));
    v[0] = ks_bf16_lo(w); v[1] = ks_bf16_hi(w);
  } else {
    v[0] = ks_bf16_to_f32(__ldg(reinterpret_cast<const unsigned short *>(p)));
  }
}
template <int VEC>
KS_DEV void store_bf16(uint16_t *p, const float (&v)[VEC]) {
  if constexpr (VEC == 8) {
    uint4 w;
    w.x = ks_pack_bf16x2(v[0], v[1]); w.y = ks_pack_bf16x2(v[2], v[3]);
    w.z = ks_pack_bf16x2(v[4], v[5]); w.w = ks_pack_bf16x2(v[6], v[7]);
    __stcs(reinterpret_cast<uint4 *>(p), w);
  } else if constexpr (VEC == 4) {
    uint2 w;
    w.x = ks_pack_bf16x2(v[0], v[1]); w.y = ks_pack_bf16x2(v[2], v[3]);
    __stcs(reinterpret_cast<uint2 *>(p), w);
  } else if constexpr (VEC == 2) {
    __stcs(reinterpret_cast<unsigned int *>(p), ks_pack_bf16x2(v[0], v[1]));
  } else {
    __stcs(reinterpret_cast<unsigned short *>(p), ks_f32_to_bf16(v[0]));
  }
}

// ---- block-wide combines (any blockDim.x multiple of 32, <= 1024) --------
// (max, sum-of-exp) pairs: merge(m1,s1,m2,s2) = (M, s1*e^(m1-M) + s2*e^(m2-M)).
// Values are kept pre-scaled by log2(e) so exponentials are ex2.
KS_DEV void merge_ms(float &m, float &s, float m2, float s2) {
  const float M = fmaxf(m, m2);
  const float a = (m == -INFINITY) ? 0.f : s * ks_ex2(m - M);
  const float b = (m2 == -INFINITY) ? 0.f : s2 * ks_ex2(m2 - M);
  m = M;
  s = a + b;
}
KS_DEV void block_reduce_ms(float &m, float &s, float2 *sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge_ms(m, s, m2, s2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) sh[warp] = make_float2(m, s);
  __syncthreads();
  float2 t = lane < nw ? sh[lane] : make_float2(-INFINITY, 0.f);
  m = t.x;
  s = t.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge_ms(m, s, m2, s2);
  }
  __syncthreads();  // sh is reused by the next row
}

// (count, mean, M2) triples merged with Chan et al.'s parallel update.
KS_DEV void merge_welford(float &n, float &mu, float &m2, float nb, float mub, float m2b) {
  const float nn = n + nb;
  if (nn == 0.f) return;
  const float d = mub - mu;
  const float fb = nb / nn;
  mu = mu + d * fb;
  m2 = m2 + m2b + d * d * n * fb;
  n = nn;
}
KS_DEV void block_reduce_welford(float &n, float &mu, float &m2, float4 *sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float nb = __shfl_xor_sync(0xffffffffu, n, o);
    float mb = __shfl_xor_sync(0xffffffffu, mu, o);
    float qb = __shfl_xor_sync(0xffffffffu, m2, o);
    merge_welford(n, mu, m2, nb, mb, qb);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) sh[warp] = make_float4(n, mu, m2, 0.f);
  __syncthreads();
  float4 t = lane < nw ? sh[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
  n = t.x;
  mu = t.y;
  m2 = t.z;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float nb = __shfl_xor_sync(0xffffffffu, n, o);
    float mb = __shfl_xor_sync(0xffffffffu, mu, o);
    float qb = __shfl_xor_sync(0xffffffffu, m2, o);
    merge_welford(n, mu, m2, nb, mb, qb);
  }
  __syncthreads();
}

// ===========================================================================
// softmax
// ===========================================================================
// ONEPASS: thread t owns vector chunks t, t+B, ..., t+(MAXCH-1)B of the row
// (chunk = VEC consecutive columns), held in registers across both phases.
template <int VEC, int MAXCH>
__global__ void __launch_bounds__(1024) softmax_onepass_kernel(const uint16_t *__restrict__ x,
                                                               uint16_t *__restrict__ y, int64_t rows,
                                                               int64_t cols) {
  __shared__ float2 sh[32];
  const int64_t nvec = cols / VEC;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t *xr = x + r * cols;
    uint16_t *yr = y + r * cols;
    float v[MAXCH][VEC];
#pragma unroll
    for (int i = 0; i < MAXCH; ++i) {
      const int64_t c = threadIdx.x + int64_t(i) * blockDim.x;
      if (c < nvec) {
        load_bf16<VEC>(xr + c * VEC, v[i]);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[i][j] = -INFINITY;
      }
    }
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < MAXCH; ++i)
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        v[i][j] *= kLog2e;
        m = fmaxf(m, v[i][j]);
      }
    float s = 0.f;
    if (m != -INFINITY) {
#pragma unroll
      for (int i = 0; i < MAXCH; ++i)
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          v[i][j] = ks_ex2(v[i][j] - m);
          s += v[i][j];
        }
    }
    const float m_local = m;
    block_reduce_ms(m, s, sh);
    const float scale = (m_local == -INFINITY) ? 0.f : ks_ex2(m_local - m) / s;
#pragma unroll
    for (int i = 0; i < MAXCH; ++i) {
      const int64_t c = threadIdx.x + int64_t(i) * blockDim.x;
      if (c < nvec) {
        float o[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) o[j] = v[i][j] * scale;
        store_bf16<VEC>(yr + c * VEC, o);
      }
    }
  }
}

// TWOPASS: stream the row to get (max, sum), then stream it again (the second
// read of a row just touched is served by L2) to write the output.
template <int VEC>
__global__ void __launch_bounds__(1024) softmax_twopass_kernel(const uint16_t *__restrict__ x,
                                                               uint16_t *__restrict__ y, int64_t rows,
                                                               int64_t cols) {
  __shared__ float2 sh[32];
  const int64_t nvec = cols / VEC;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t *xr = x + r * cols;
    uint16_t *yr = y + r * cols;
    float m = -INFINITY, s = 0.f;
    for (int64_t c = threadIdx.x; c < nvec; c += blockDim.x) {
      float v[VEC];
      load_bf16<VEC>(xr + c * VEC, v);
      float cm = -INFINITY;
#pragma unroll
      for (int j = 0; j < VEC; ++j) cm = fmaxf(cm, v[j] * kLog2e);
      float cs = 0.f;
#pragma unroll
      for (int j = 0; j < VEC; ++j) cs += ks_ex2(v[j] * kLog2e - cm);
      merge_ms(m, s, cm, cs);
    }
    block_reduce_ms(m, s, sh);
    const float inv = 1.f / s;
    for (int64_t c = threadIdx.x; c < nvec; c += blockDim.x) {
      float v[VEC];
      load_bf16<VEC>(xr + c * VEC, v);
#pragma unroll
      for (int j = 0; j < VEC; ++j) v[j] = ks_ex2(v[j] * kLog2e - m) * inv;
      store_bf16<VEC>(yr + c * VEC, v);
    }
  }
}

// ===========================================================================
// layernorm
// ===========================================================================
template <int VEC, int MAXCH>
__global__ void __launch_bounds__(1024) layernorm_onepass_kernel(const uint16_t *__restrict__ x,
                                                                 const uint16_t *__restrict__ gamma,
                                                                 const uint16_t *__restrict__ beta,
                                                                 uint16_t *__restrict__ y, int64_t rows,
                                                                 int64_t cols, float eps) {
  __shared__ float4 sh[32];
  const int64_t nvec = cols / VEC;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t *xr = x + r * cols;
    uint16_t *yr = y + r * cols;
    float v[MAXCH][VEC];
    float sum = 0.f, cnt = 0.f;
#pragma unroll
    for (int i = 0; i < MAXCH; ++i) {
      const int64_t c = threadIdx.x + int64_t(i) * blockDim.x;
      if (c < nvec) {
        load_bf16<VEC>(xr + c * VEC, v[i]);
#pragma unroll
        for (int j = 0; j < VEC; ++j) sum += v[i][j];
        cnt += VEC;
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[i][j] = 0.f;
      }
    }
    float mu = cnt > 0.f ? sum / cnt : 0.f;
    float m2 = 0.f;
#pragma unroll
    for (int i = 0; i < MAXCH; ++i) {
      const int64_t c = threadIdx.x + int64_t(i) * blockDim.x;
      if (c < nvec) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float d = v[i][j] - mu;
          m2 += d * d;
        }
      }
    }
    float n = cnt;
    block_reduce_welford(n, mu, m2, sh);
    const float rstd = rsqrtf(m2 / n + eps);
#pragma unroll
    for (int i = 0; i < MAXCH; ++i) {
      const int64_t c = threadIdx.x + int64_t(i) * blockDim.x;
      if (c < nvec) {
        float g[VEC], b[VEC], o[VEC];
        load_bf16_cached<VEC>(gamma + c * VEC, g);
        load_bf16_cached<VEC>(beta + c * VEC, b);
#pragma unroll
        for (int j = 0; j < VEC; ++j) o[j] = (v[i][j] - mu) * rstd * g[j] + b[j];
        store_bf16<VEC>(yr + c * VEC, o);
      }
    }
  }
}

template <int VEC>
__global__ void __launch_bounds__(1024) layernorm_twopass_kernel(const uint16_t *__restrict__ x,
                                                                 const uint16_t *__restrict__ gamma,
                                                                 const uint16_t *__restrict__ beta,
                                                                 uint16_t *__restrict__ y, int64_t rows,
                                                                 int64_t cols, float eps) {
  __shared__ float4 sh[32];
  const int64_t nvec = cols / VEC;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t *xr = x + r * cols;
    uint16_t *yr = y + r * cols;
    float n = 0.f, mu = 0.f, m2 = 0.f;
    for (int64_t c = threadIdx.x; c < nvec; c += blockDim.x) {
      float v[VEC];
      load_bf16<VEC>(xr + c * VEC, v);
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < VEC; ++j) s += v[j];
      const float cm = s / VEC;
      float q = 0.f;
#pragma unroll
      for (int j = 0; j < VEC; ++j) q += (v[j] - cm) * (v[j] - cm);
      merge_welford(n, mu, m2, float(VEC), cm, q);
    }
    block_reduce_welford(n, mu, m2, sh);
    const float rstd = rsqrtf(m2 / n + eps);
    for (int64_t c = threadIdx.x; c < nvec; c += blockDim.x) {
      float v[VEC], g[VEC], b[VEC];
      load_bf16<VEC>(xr + c * VEC, v);
      load_bf16_cached<VEC>(gamma + c * VEC, g);
      load_bf16_cached<VEC>(beta + c * VEC, b);
#pragma unroll
      for (int j = 0; j < VEC; ++j) v[j] = (v[j] - mu) * rstd * g[j] + b[j];
      store_bf16<VEC>(yr + c * VEC, v);
    }
  }
}

// ===========================================================================
// bias_gelu
// ===========================================================================
KS_DEV float gelu_erf(float t) {
  // 0.5 t (1 + erf(t/sqrt2)) written with erfc to avoid cancellation for t < 0.
  return 0.5f * t * erfcf(-t * 0.70710678118654752f);
}
KS_DEV float gelu_tanh(float t) {
  // 0.5 t (1 + tanh(u)) = t * sigmoid(2u), u = sqrt(2/pi) (t + 0.044715 t^3).
  const float u = 0.7978845608028654f * fmaf(0.044715f * t, t * t, t);
  const float e = ks_ex2(-2.f * kLog2e * u);
  return __fdividef(t, 1.f + e);
}

// Each thread owns one VEC-wide column chunk (its bias chunk is loaded once)
// and walks ROWS_PER_CTA rows, UNROLL rows at a time for memory parallelism.
// blockIdx.x covers column chunks, blockIdx.y row groups; the flat index
// (row*cols + col) is bounds-checked against `total` (ragged last row).
template <int VEC, int GELU, int UNROLL>
__global__ void __launch_bounds__(1024) bias_gelu_kernel(const uint16_t *__restrict__ x,
                                                         const uint16_t *__restrict__ bias,
                                                         uint16_t *__restrict__ y, int64_t total, int64_t cols,
                                                         int64_t rows, int rows_per_cta) {
  const int64_t nvec = cols / VEC;
  const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= nvec) return;
  float b[VEC];
  load_bf16_cached<VEC>(bias + c * VEC, b);
  const int64_t r0 = int64_t(blockIdx.y) * rows_per_cta;
  const int64_t r1 = min(rows, r0 + rows_per_cta);
  for (int64_t r = r0; r < r1; r += UNROLL) {
    float v[UNROLL][VEC];
    bool ok[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t off = (r + u) * cols + c * VEC;
      ok[u] = (r + u < r1) && (off + VEC <= total);
      if (ok[u]) load_bf16<VEC>(x + off, v[u]);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      if (!ok[u]) continue;
      float o[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        // fusion point: fp32 add of the bf16 operands, rounded to bf16
        const float t = __bfloat162float(__float2bfloat16_rn(v[u][j] + b[j]));
        o[j] = GELU == KS_GELU_TANH ? gelu_tanh(t) : gelu_erf(t);
      }
      store_bf16<VEC>(y + (r + u) * cols + c * VEC, o);
    }
  }
}

// Scalar tail kernel for a ragged last row whose length is not a multiple
// of VEC (total % cols != 0 and the tail not VEC-aligned).
template <int GELU>
__global__ void bias_gelu_tail_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ bias,
                                      uint16_t *__restrict__ y, int64_t start, int64_t total, int64_t cols) {
  const int64_t i = start + int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const float xv = ks_bf16_to_f32(x[i]);
  const float bv = ks_bf16_to_f32(bias[i % cols]);
  const float t = __bfloat162float(__float2bfloat16_rn(xv + bv));
  y[i] = ks_f32_to_bf16(GELU == KS_GELU_TANH ? gelu_tanh(t) : gelu_erf(t));
}

// ---------------------------------------------------------------------------
// Host-side dispatch helpers
// ---------------------------------------------------------------------------
constexpr int kRegElems = 32;  // per-thread register budget for a ONEPASS row

bool valid_block(int b) { return b == 128 || b == 256 || b == 512 || b == 1024; }
bool valid_vec(int v) { return v == 1 || v == 2 || v == 4 || v == 8; }

bool aligned(const void *p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

template <typename K>
int grid_for(K kernel, int block, int64_t work) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, block, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int64_t cap = int64_t(per_sm) * ks::sm_count();
  return int(work < cap ? work : cap);
}

int rowop_validate(const char *fam, int block, int vec, int mode, int64_t rows, int64_t cols, char *reason,
                   size_t len) {
  if (!valid_block(block)) {
    ks::set_reason(reason, len, "%s: block must be 128, 256, 512 or 1024 (sm_100a space)", fam);
    return KS_ERR_INVALID_CONFIG;
  }
  if (!valid_vec(vec)) {
    ks::set_reason(reason, len, "%s: vec_width must be 1, 2, 4 or 8 (sm_100a space)", fam);
    return KS_ERR_INVALID_CONFIG;
  }
  if (mode != KS_MODE_ONEPASS && mode != KS_MODE_TWOPASS) {
    ks::set_reason(reason, len, "%s: mode must be onepass or twopass", fam);
    return KS_ERR_INVALID_CONFIG;
  }
  if (rows <= 0 || cols <= 0) {
    ks::set_reason(reason, len, "%s: shape (rows, cols) must be positive (got %lld, %lld)", fam,
                   (long long)rows, (long long)cols);
    return KS_ERR_INVALID_ARGS;
  }
  if (cols % vec != 0) {
    ks::set_reason(reason, len, "%s: cols %lld not divisible by vec_width %d", fam, (long long)cols, vec);
    return KS_ERR_INVALID_CONFIG;
  }
  if (mode == KS_MODE_ONEPASS && cols > int64_t(block) * kRegElems) {
    ks::set_reason(reason, len,
                   "%s: onepass keeps the row in registers: cols %lld > block %d x %d register elements", fam,
                   (long long)cols, block, kRegElems);
    return KS_ERR_INVALID_CONFIG;
  }
  ks::set_reason(reason, len, "");
  return KS_OK;
}

template <int VEC>
int launch_softmax_vec(const ks_softmax_config &cfg, const ks_softmax_args &a, cudaStream_t st) {
  auto x = static_cast<const uint16_t *>(a.x);
  auto y = static_cast<uint16_t *>(a.out);
  if (cfg.mode == KS_MODE_TWOPASS) {
    auto k = softmax_twopass_kernel<VEC>;
    k<<<grid_for(k, cfg.block, a.rows), cfg.block, 0, st>>>(x, y, a.rows, a.cols);
  } else {
    constexpr int MAXCH = kRegElems / VEC;
    auto k = softmax_onepass_kernel<VEC, MAXCH>;
    k<<<grid_for(k, cfg.block, a.rows), cfg.block, 0, st>>>(x, y, a.rows, a.cols);
  }
  return ks::map_cuda(cudaGetLastError());
}

template <int VEC>
int launch_layernorm_vec(const ks_layernorm_config &cfg, const ks_layernorm_args &a, cudaStream_t st) {
  auto x = static_cast<const uint16_t *>(a.x);
  auto g = static_cast<const uint16_t *>(a.gamma);
  auto b = static_cast<const uint16_t *>(a.beta);
  auto y = static_cast<uint16_t *>(a.out);
  const float eps = a.eps > 0.f ? a.eps : 1e-5f;
  if (cfg.mode == KS_MODE_TWOPASS) {
    auto k = layernorm_twopass_kernel<VEC>;
    k<<<grid_for(k, cfg.block, a.rows), cfg.block, 0, st>>>(x, g, b, y, a.rows, a.cols, eps);
  } else {
    constexpr int MAXCH = kRegElems / VEC;
    auto k = layernorm_onepass_kernel<VEC, MAXCH>;
    k<<<grid_for(k, cfg.block, a.rows), cfg.block, 0, st>>>(x, g, b, y, a.rows, a.cols, eps);
  }
  return ks::map_cuda(cudaGetLastError());
}

constexpr int kBgRowsPerCta = 32;
// rows in flight per thread: 2 x 16 bytes for 8-wide vectors (register cap of
// a 1024-thread CTA), 4 for narrower vectors
template <int VEC>
constexpr int bg_unroll() { return VEC == 8 ? 2 : 4; }

template <int VEC, int GELU>
int launch_bias_gelu_vec(const ks_bias_gelu_config &cfg, const ks_bias_gelu_args &a, cudaStream_t st) {
  auto x = static_cast<const uint16_t *>(a.x);
  auto b = static_cast<const uint16_t *>(a.bias);
  auto y = static_cast<uint16_t *>(a.out);
  const int64_t rows = (a.total + a.cols - 1) / a.cols;
  const int64_t nvec = a.cols / VEC;
  dim3 grid(unsigned((nvec + cfg.block - 1) / cfg.block), unsigned((rows + kBgRowsPerCta - 1) / kBgRowsPerCta));
  bias_gelu_kernel<VEC, GELU, bg_unroll<VEC>()><<<grid, cfg.block, 0, st>>>(x, b, y, a.total, a.cols, rows, kBgRowsPerCta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return ks::map_cuda(e);
  // The vector kernel stops at the last full VEC chunk of a ragged last row.
  const int64_t last_row_start = (rows - 1) * a.cols;
  const int64_t tail_len = a.total - last_row_start;
  const int64_t vec_done = (tail_len / VEC) * VEC;
  if (vec_done < tail_len) {
    const int64_t start = last_row_start + vec_done;
    const int64_t n = a.total - start;
    bias_gelu_tail_kernel<GELU><<<unsigned((n + 255) / 256), 256, 0, st>>>(x, b, y, start, a.total, a.cols);
    e = cudaGetLastError();
  }
  return ks::map_cuda(e);
}

}  // namespace

extern "C" {

int ks_softmax_validate(const ks_softmax_config *cfg, int64_t rows, int64_t cols, char *reason, size_t len) {
  if (!cfg) return KS_ERR_INVALID_ARGS;
  return rowop_validate("softmax", cfg->block, cfg->vec_width, cfg->mode, rows, cols, reason, len);
}

int ks_softmax_launch(const ks_softmax_config *cfg, const ks_softmax_args *a, void *stream) {
  if (!cfg || !a || !a->x || !a->out) return KS_ERR_INVALID_ARGS;
  int s = ks_softmax_validate(cfg, a->rows, a->cols, nullptr, 0);
  if (s != KS_OK) return s;
  if (!aligned(a->x, 2 * cfg->vec_width) || !aligned(a->out, 2 * cfg->vec_width)) return KS_ERR_INVALID_ARGS;
  if ((s = ks::check_arch_sm100()) != KS_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (cfg->vec_width) {
    case 8: return launch_softmax_vec<8>(*cfg, *a, st);
    case 4: return launch_softmax_vec<4>(*cfg, *a, st);
    case 2: return launch_softmax_vec<2>(*cfg, *a, st);
    default: return launch_softmax_vec<1>(*cfg, *a, st);
  }
}

int ks_layernorm_validate(const ks_layernorm_config *cfg, int64_t rows, int64_t cols, char *reason, size_t len) {
  if (!cfg) return KS_ERR_INVALID_ARGS;
  return rowop_validate("layernorm", cfg->block, cfg->vec_width, cfg->mode, rows, cols, reason, len);
}

int ks_layernorm_launch(const ks_layernorm_config *cfg, const ks_layernorm_args *a, void *stream) {
  if (!cfg || !a || !a->x || !a->gamma || !a->beta || !a->out) return KS_ERR_INVALID_ARGS;
  int s = ks_layernorm_validate(cfg, a->rows, a->cols, nullptr, 0);
  if (s != KS_OK) return s;
  const int al = 2 * cfg->vec_width;
  if (!aligned(a->x, al) || !aligned(a->out, al) || !aligned(a->gamma, al) || !aligned(a->beta, al))
    return KS_ERR_INVALID_ARGS;
  if ((s = ks::check_arch_sm100()) != KS_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (cfg->vec_width) {
    case 8: return launch_layernorm_vec<8>(*cfg, *a, st);
    case 4: return launch_layernorm_vec<4>(*cfg, *a, st);
    case 2: return launch_layernorm_vec<2>(*cfg, *a, st);
    default: return launch_layernorm_vec<1>(*cfg, *a, st);
  }
}

int ks_bias_gelu_validate(const ks_bias_gelu_config *cfg, int64_t total, int64_t cols, char *reason, size_t len) {
  if (!cfg) return KS_ERR_INVALID_ARGS;
  if (!valid_block(cfg->block)) {
    ks::set_reason(reason, len, "bias_gelu: block must be 128, 256, 512 or 1024 (sm_100a space)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (!valid_vec(cfg->vec_width)) {
    ks::set_reason(reason, len, "bias_gelu: vec_width must be 1, 2, 4 or 8 (sm_100a space)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (cfg->gelu != KS_GELU_ERF && cfg->gelu != KS_GELU_TANH) {
    ks::set_reason(reason, len, "bias_gelu: gelu must be erf or tanh");
    return KS_ERR_INVALID_CONFIG;
  }
  if (total <= 0 || cols <= 0) {
    ks::set_reason(reason, len, "bias_gelu: shape (total, cols) must be positive (got %lld, %lld)",
                   (long long)total, (long long)cols);
    return KS_ERR_INVALID_ARGS;
  }
  if (cols % cfg->vec_width != 0) {
    ks::set_reason(reason, len, "bias_gelu: cols %lld not divisible by vec_width %d", (long long)cols,
                   cfg->vec_width);
    return KS_ERR_INVALID_CONFIG;
  }
  ks::set_reason(reason, len, "");
  return KS_OK;
}

int ks_bias_gelu_launch(const ks_bias_gelu_config *cfg, const ks_bias_gelu_args *a, void *stream) {
  if (!cfg || !a || !a->x || !a->bias || !a->out) return KS_ERR_INVALID_ARGS;
  int s = ks_bias_gelu_validate(cfg, a->total, a->cols, nullptr, 0);
  if (s != KS_OK) return s;
  const int al = 2 * cfg->vec_width;
  if (!aligned(a->x, al) || !aligned(a->out, al) || !aligned(a->bias, al)) return KS_ERR_INVALID_ARGS;
  if ((s = ks::check_arch_sm100()) != KS_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool th = cfg->gelu == KS_GELU_TANH;
  switch (cfg->vec_width) {
    case 8: return th ? launch_bias_gelu_vec<8, KS_GELU_TANH>(*cfg, *a, st) : launch_bias_gelu_vec<8, KS_GELU_ERF>(*cfg, *a, st);
    case 4: return th ? launch_bias_gelu_vec<4, KS_GELU_TANH>(*cfg, *a, st) : launch_bias_gelu_vec<4, KS_GELU_ERF>(*cfg, *a, st);
    case 2: return th ? launch_bias_gelu_vec<2, KS_GELU_TANH>(*cfg, *a, st) : launch_bias_gelu_vec<2, KS_GELU_ERF>(*cfg, *a, st);
    default: return th ? launch_bias_gelu_vec<1, KS_GELU_TANH>(*cfg, *a, st) : launch_bias_gelu_vec<1, KS_GELU_ERF>(*cfg, *a, st);
  }
}

}  // extern "C"
