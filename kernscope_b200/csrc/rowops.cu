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
// 8-wide fast paths (vec_width 8, 32-bit in-row indexing).  Written for the
// fewest instructions per element, since at B200 bandwidth a row op has only
// ~6-9 issue slots per element before it stops being HBM-bound:
//   * block max / sum: warp shuffles of plain max / add, one shared slot per
//     warp, every warp then reduces the <= 32 slots itself.  The two
//     reductions of a row use different slot arrays, so the next row can
//     overwrite them without a trailing barrier;
//   * the row max is taken on the packed words (bf16x2 max, exact);
//   * exp(x - m) = ex2(x*log2e - m*log2e) as one FFMA + one ex2.
// ===========================================================================
KS_DEV float block_max_fast(float v, float *sh) {
  v = ks_warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  return ks_warp_max(lane < int(blockDim.x >> 5) ? sh[lane] : -INFINITY);
}
KS_DEV float block_sum_fast(float v, float *sh) {
  v = ks_warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  return ks_warp_sum(lane < int(blockDim.x >> 5) ? sh[lane] : 0.f);
}

KS_DEV __nv_bfloat162 as_bf162(uint32_t w) { return *reinterpret_cast<__nv_bfloat162 *>(&w); }
KS_DEV uint32_t as_u32(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }

KS_DEV float max8_packed(const uint4 &w) {
  const __nv_bfloat162 a = __hmax2(as_bf162(w.x), as_bf162(w.y));
  const __nv_bfloat162 b = __hmax2(as_bf162(w.z), as_bf162(w.w));
  const uint32_t c = as_u32(__hmax2(a, b));
  return fmaxf(ks_bf16_lo(c), ks_bf16_hi(c));
}
KS_DEV void unpack8(const uint4 &w, float (&v)[8]) {
  v[0] = ks_bf16_lo(w.x); v[1] = ks_bf16_hi(w.x); v[2] = ks_bf16_lo(w.y); v[3] = ks_bf16_hi(w.y);
  v[4] = ks_bf16_lo(w.z); v[5] = ks_bf16_hi(w.z); v[6] = ks_bf16_lo(w.w); v[7] = ks_bf16_hi(w.w);
}
KS_DEV uint4 pack8(const float (&v)[8]) {
  return make_uint4(ks_pack_bf16x2(v[0], v[1]), ks_pack_bf16x2(v[2], v[3]), ks_pack_bf16x2(v[4], v[5]),
                    ks_pack_bf16x2(v[6], v[7]));
}

// Softmax of one row whose chunks (8 bf16 each) this thread holds in w[];
// chunk k of thread t is row chunk t + k*blockDim.x.  `after_max` runs on
// thread 0 right after the max reduction's barrier (every thread has then
// consumed its inputs), used by the staged kernel to refill its ring slot.
template <int MAXCH, typename AfterMax>
KS_DEV void softmax_row8(const uint4 (&w)[MAXCH], int nvec, float *sh_max, float *sh_sum, uint4 *yr,
                         AfterMax after_max) {
  const int t = threadIdx.x, nt = blockDim.x;
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < MAXCH; ++k)
    if (t + k * nt < nvec) m = fmaxf(m, max8_packed(w[k]));
  m = block_max_fast(m, sh_max);
  after_max();
  const float mL = m * kLog2e;
  float e[MAXCH][8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    if (t + k * nt < nvec) {
      unpack8(w[k], e[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        e[k][j] = ks_ex2(fmaf(e[k][j], kLog2e, -mL));
        s += e[k][j];
      }
    }
  }
  s = block_sum_fast(s, sh_sum);
  const float inv = 1.f / s;
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    if (t + k * nt < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) e[k][j] *= inv;
      __stcs(yr + t + k * nt, pack8(e[k]));
    }
  }
}

// Loads this thread's chunks of row r (chunk k = column chunk t + k*blockDim.x).
template <int MAXCH>
KS_DEV void load_row8(const uint16_t *__restrict__ x, int r, int cols, int nvec, uint4 (&w)[MAXCH]) {
  const uint4 *xr = reinterpret_cast<const uint4 *>(x + size_t(r) * cols);
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < nvec) w[k] = __ldcs(xr + c);
  }
}

// MAXB = largest block the instantiation serves.  Blocks <= 512 threads have
// the registers to prefetch the next row's packed words while the current
// row is reduced, which keeps HBM reads in flight through the barriers.
template <int MAXCH, int MAXB>
__global__ void __launch_bounds__(MAXB) softmax_onepass_v8_kernel(const uint16_t *__restrict__ x,
                                                                  uint16_t *__restrict__ y, int rows, int cols) {
  __shared__ float sh_max[32], sh_sum[32];
  const int nvec = cols >> 3;
  constexpr bool kPrefetch = MAXB <= 512;
  uint4 nxt[MAXCH];
  if (kPrefetch && int(blockIdx.x) < rows) load_row8<MAXCH>(x, blockIdx.x, cols, nvec, nxt);
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    uint4 w[MAXCH];
    if constexpr (kPrefetch) {
#pragma unroll
      for (int k = 0; k < MAXCH; ++k) w[k] = nxt[k];
      if (r + int(gridDim.x) < rows) load_row8<MAXCH>(x, r + gridDim.x, cols, nvec, nxt);
    } else {
      load_row8<MAXCH>(x, r, cols, nvec, w);
    }
    softmax_row8<MAXCH>(w, nvec, sh_max, sh_sum, reinterpret_cast<uint4 *>(y + size_t(r) * cols), [] {});
  }
}

// Layernorm of one row held as packed chunks: exact two-pass statistics from
// registers (mean, then the sum of squared deviations), each a plain sum
// reduction; y = d * (rstd * gamma) + beta with d = x - mean.
template <int MAXCH, typename AfterFirst>
KS_DEV void layernorm_row8(const uint4 (&w)[MAXCH], int nvec, float inv_cols, float eps, const uint4 *g4,
                           const uint4 *b4, float *sh_a, float *sh_b, uint4 *yr, AfterFirst after_first) {
  const int t = threadIdx.x, nt = blockDim.x;
  float v[MAXCH][8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    if (t + k * nt < nvec) {
      unpack8(w[k], v[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[k][j];
    }
  }
  const float mean = block_sum_fast(s, sh_a) * inv_cols;
  after_first();
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    if (t + k * nt < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[k][j] -= mean;
        q = fmaf(v[k][j], v[k][j], q);
      }
    }
  }
  const float rstd = rsqrtf(block_sum_fast(q, sh_b) * inv_cols + eps);
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    const int c = t + k * nt;
    if (c < nvec) {
      float g[8], b[8];
      unpack8(g4[c], g);
      unpack8(b4[c], b);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[k][j] = fmaf(v[k][j], rstd * g[j], b[j]);
      __stcs(yr + c, pack8(v[k]));
    }
  }
}

template <int MAXCH, int MAXB>
__global__ void __launch_bounds__(MAXB) layernorm_onepass_v8_kernel(const uint16_t *__restrict__ x,
                                                                    const uint16_t *__restrict__ gamma,
                                                                    const uint16_t *__restrict__ beta,
                                                                    uint16_t *__restrict__ y, int rows, int cols,
                                                                    float inv_cols, float eps) {
  __shared__ float sh_a[32], sh_b[32];
  const int nvec = cols >> 3;
  const uint4 *g4 = reinterpret_cast<const uint4 *>(gamma);
  const uint4 *b4 = reinterpret_cast<const uint4 *>(beta);
  constexpr bool kPrefetch = MAXB <= 512;
  uint4 nxt[MAXCH];
  if (kPrefetch && int(blockIdx.x) < rows) load_row8<MAXCH>(x, blockIdx.x, cols, nvec, nxt);
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    uint4 w[MAXCH];
    if constexpr (kPrefetch) {
#pragma unroll
      for (int k = 0; k < MAXCH; ++k) w[k] = nxt[k];
      if (r + int(gridDim.x) < rows) load_row8<MAXCH>(x, r + gridDim.x, cols, nvec, nxt);
    } else {
      load_row8<MAXCH>(x, r, cols, nvec, w);
    }
    layernorm_row8<MAXCH>(w, nvec, inv_cols, eps, g4, b4, sh_a, sh_b,
                          reinterpret_cast<uint4 *>(y + size_t(r) * cols), [] {});
  }
}

// ===========================================================================
// Short rows (at most 1024 columns, 8-wide vectors): one warp per row, so
// the reductions are warp shuffles with no block barrier, and a CTA of
// blockDim.x / 32 warps keeps that many rows in flight plus each warp's
// prefetched next row.  Lane l holds column chunks l, l+32, ... (WCH of
// them).  Layernorm's gamma and beta chunks are the same for every row a
// lane touches, so they stay in registers.
// ===========================================================================
template <int WCH>
KS_DEV void load_row_warp8(const uint16_t *__restrict__ x, int r, int cols, int nvec, uint4 (&w)[WCH]) {
  const uint4 *xr = reinterpret_cast<const uint4 *>(x + size_t(r) * cols);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < WCH; ++k)
    if (lane + 32 * k < nvec) w[k] = __ldcs(xr + lane + 32 * k);
}

template <int WCH>
__global__ void __launch_bounds__(256) softmax_warp_v8_kernel(const uint16_t *__restrict__ x,
                                                              uint16_t *__restrict__ y, int rows, int cols) {
  const int lane = threadIdx.x & 31, nvec = cols >> 3;
  const int wpc = blockDim.x >> 5;
  const int first = int(blockIdx.x) * wpc + (threadIdx.x >> 5), stride = int(gridDim.x) * wpc;
  uint4 nxt[WCH];
  if (first < rows) load_row_warp8<WCH>(x, first, cols, nvec, nxt);
  for (int r = first; r < rows; r += stride) {
    uint4 w[WCH];
#pragma unroll
    for (int k = 0; k < WCH; ++k) w[k] = nxt[k];
    if (r + stride < rows) load_row_warp8<WCH>(x, r + stride, cols, nvec, nxt);
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < WCH; ++k)
      if (lane + 32 * k < nvec) m = fmaxf(m, max8_packed(w[k]));
    m = ks_warp_max(m);
    const float mL = m * kLog2e;
    float e[WCH][8];
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < WCH; ++k) {
      if (lane + 32 * k < nvec) {
        unpack8(w[k], e[k]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          e[k][j] = ks_ex2(fmaf(e[k][j], kLog2e, -mL));
          sum += e[k][j];
        }
      }
    }
    const float inv = 1.f / ks_warp_sum(sum);
    uint4 *yr = reinterpret_cast<uint4 *>(y + size_t(r) * cols);
#pragma unroll
    for (int k = 0; k < WCH; ++k) {
      if (lane + 32 * k < nvec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) e[k][j] *= inv;
        __stcs(yr + lane + 32 * k, pack8(e[k]));
      }
    }
  }
}

template <int WCH>
__global__ void __launch_bounds__(256) layernorm_warp_v8_kernel(const uint16_t *__restrict__ x,
                                                                const uint16_t *__restrict__ gamma,
                                                                const uint16_t *__restrict__ beta,
                                                                uint16_t *__restrict__ y, int rows, int cols,
                                                                float inv_cols, float eps) {
  const int lane = threadIdx.x & 31, nvec = cols >> 3;
  const int wpc = blockDim.x >> 5;
  const int first = int(blockIdx.x) * wpc + (threadIdx.x >> 5), stride = int(gridDim.x) * wpc;
  uint4 gw[WCH], bw[WCH];
#pragma unroll
  for (int k = 0; k < WCH; ++k)
    if (lane + 32 * k < nvec) {
      gw[k] = __ldg(reinterpret_cast<const uint4 *>(gamma) + lane + 32 * k);
      bw[k] = __ldg(reinterpret_cast<const uint4 *>(beta) + lane + 32 * k);
    }
  uint4 nxt[WCH];
  if (first < rows) load_row_warp8<WCH>(x, first, cols, nvec, nxt);
  for (int r = first; r < rows; r += stride) {
    uint4 w[WCH];
#pragma unroll
    for (int k = 0; k < WCH; ++k) w[k] = nxt[k];
    if (r + stride < rows) load_row_warp8<WCH>(x, r + stride, cols, nvec, nxt);
    float v[WCH][8];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < WCH; ++k) {
      if (lane + 32 * k < nvec) {
        unpack8(w[k], v[k]);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += v[k][j];
      }
    }
    const float mean = ks_warp_sum(s) * inv_cols;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < WCH; ++k) {
      if (lane + 32 * k < nvec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[k][j] -= mean;
          q = fmaf(v[k][j], v[k][j], q);
        }
      }
    }
    const float rstd = rsqrtf(ks_warp_sum(q) * inv_cols + eps);
    uint4 *yr = reinterpret_cast<uint4 *>(y + size_t(r) * cols);
#pragma unroll
    for (int k = 0; k < WCH; ++k) {
      if (lane + 32 * k < nvec) {
        float g[8], b[8];
        unpack8(gw[k], g);
        unpack8(bw[k], b);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[k][j] = fmaf(v[k][j], rstd * g[j], b[j]);
        __stcs(yr + lane + 32 * k, pack8(v[k]));
      }
    }
  }
}

// ===========================================================================
// Long rows over a thread-block cluster (mode CLUSTER).  CTA rank r of a
// cluster of cs CTAs holds columns [r*seg, (r+1)*seg) of one row in
// registers (CH 8-wide chunks per thread).  The row statistics -- max and
// sum for softmax, sum and sum of squared deviations for layernorm --
// combine across the cluster through distributed shared memory between
// cluster barriers.  The row is read from HBM once however long it is, and
// a few rows still fill the 148 SMs.
// ===========================================================================
// This CTA's partial v (the same in every thread) combined over the cluster:
// publish it in `slot`, wait for every CTA, and let warp 0 gather the cs
// partials.  Each combine of a kernel uses its own slot.
KS_DEV float cluster_combine(float v, float *slot, float *bcast, bool is_max) {
  if (threadIdx.x == 0) *slot = v;
  ks_cluster_sync();
  if (threadIdx.x < 32) {
    const uint32_t cs = ks_cluster_nctarank();
    float t = is_max ? -INFINITY : 0.f;
    if (threadIdx.x < cs) t = ks_ld_shared_cluster_f32(ks_mapa(ks_smem_u32(slot), threadIdx.x));
    t = is_max ? ks_warp_max(t) : ks_warp_sum(t);
    if (threadIdx.x == 0) *bcast = t;
  }
  __syncthreads();
  return *bcast;
}

template <int CH>
__global__ void __launch_bounds__(1024) softmax_cluster_v8_kernel(const uint16_t *__restrict__ x,
                                                                  uint16_t *__restrict__ y, int64_t cols, int seg) {
  __shared__ float sh_max[32], sh_sum[32];
  __shared__ float slot_a, slot_b, bcast;
  const uint32_t cs = ks_cluster_nctarank(), rank = ks_cluster_ctarank();
  const int64_t off = int64_t(blockIdx.x / cs) * cols + int64_t(rank) * seg;
  const int t = threadIdx.x, nt = blockDim.x, nvec = seg >> 3;
  const uint4 *xs = reinterpret_cast<const uint4 *>(x + off);
  uint4 w[CH];
#pragma unroll
  for (int k = 0; k < CH; ++k)
    if (t + k * nt < nvec) w[k] = __ldcs(xs + t + k * nt);
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < CH; ++k)
    if (t + k * nt < nvec) m = fmaxf(m, max8_packed(w[k]));
  m = cluster_combine(block_max_fast(m, sh_max), &slot_a, &bcast, true);
  const float mL = m * kLog2e;
  float e[CH][8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    if (t + k * nt < nvec) {
      unpack8(w[k], e[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        e[k][j] = ks_ex2(fmaf(e[k][j], kLog2e, -mL));
        s += e[k][j];
      }
    }
  }
  const float inv = 1.f / cluster_combine(block_sum_fast(s, sh_sum), &slot_b, &bcast, false);
  uint4 *ys = reinterpret_cast<uint4 *>(y + off);
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    if (t + k * nt < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) e[k][j] *= inv;
      __stcs(ys + t + k * nt, pack8(e[k]));
    }
  }
  ks_cluster_sync();  // no CTA leaves while another may still read its slots
}

template <int CH>
__global__ void __launch_bounds__(1024) layernorm_cluster_v8_kernel(const uint16_t *__restrict__ x,
                                                                    const uint16_t *__restrict__ gamma,
                                                                    const uint16_t *__restrict__ beta,
                                                                    uint16_t *__restrict__ y, int64_t cols, int seg,
                                                                    float inv_cols, float eps) {
  __shared__ float sh_a[32], sh_b[32];
  __shared__ float slot_a, slot_b, bcast;
  const uint32_t cs = ks_cluster_nctarank(), rank = ks_cluster_ctarank();
  const int64_t off = int64_t(blockIdx.x / cs) * cols + int64_t(rank) * seg;
  const int t = threadIdx.x, nt = blockDim.x, nvec = seg >> 3;
  const uint4 *xs = reinterpret_cast<const uint4 *>(x + off);
  uint4 w[CH];
#pragma unroll
  for (int k = 0; k < CH; ++k)
    if (t + k * nt < nvec) w[k] = __ldcs(xs + t + k * nt);
  float v[CH][8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    if (t + k * nt < nvec) {
      unpack8(w[k], v[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[k][j];
    }
  }
  const float mean = cluster_combine(block_sum_fast(s, sh_a), &slot_a, &bcast, false) * inv_cols;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    if (t + k * nt < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[k][j] -= mean;
        q = fmaf(v[k][j], v[k][j], q);
      }
    }
  }
  const float rstd = rsqrtf(cluster_combine(block_sum_fast(q, sh_b), &slot_b, &bcast, false) * inv_cols + eps);
  const uint4 *g4 = reinterpret_cast<const uint4 *>(gamma + int64_t(rank) * seg);
  const uint4 *b4 = reinterpret_cast<const uint4 *>(beta + int64_t(rank) * seg);
  uint4 *ys = reinterpret_cast<uint4 *>(y + off);
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int c = t + k * nt;
    if (c < nvec) {
      float g[8], b[8];
      unpack8(__ldg(g4 + c), g);
      unpack8(__ldg(b4 + c), b);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[k][j] = fmaf(v[k][j], rstd * g[j], b[j]);
      __stcs(ys + c, pack8(v[k]));
    }
  }
  ks_cluster_sync();  // no CTA leaves while another may still read its slots
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
// ---- exact-erf GELU ---------------------------------------------------------
// The reference (refs.py:59-63, bias_gelu_gen.cpp:114-118) computes, for a
// bf16 value t,
//   x = fp32(t * fp32(1/sqrt 2)),  e = fp32(erf(double(x))),
//   y = bf16(fp32(fp32(0.5 t) * fp32(1 + e))).
// The kernels keep that operation order and replace the double erf by an
// fp32 erfc of |x| with a small relative error, so that 1 + e is formed
// from it exactly as the reference forms it:
//   w = fp32(1 - erfc|x|)  (= fp32(erf|x|)),  1 + e = fp32(1 + w) for x >= 0
//   and fp32(1 - w) for x < 0,
// which also reproduces the reference's loss of the tail (for x < -3.9,
// w rounds to 1 and y to -0).
// erfc(z) = r * 2^((P(r) - z^2) log2 e), r = 1 / (1 + 0.55 z), z = min(|x|, 4):
// the form of Press et al.'s erfcc (Numerical Recipes, section 6.2) with
// this repository's own degree-6 coefficients (fit_gelu_erfc.py beside this
// file: a least-squares fit reweighted toward minimax, relative error 3.2e-7
// in exact arithmetic).  Over the 3072 bf16 codes with 2^-9 <= |t| < 8 the
// result equals the reference bit for bit in a float32 emulation of this
// operation order, even with r and the power of two off by one and two ulps
// (rcp.approx and ex2.approx); below 2^-9, |0.5 t e| is under half a bf16 ulp
// of 0.5 t, so y = 0.5 t (taken directly: there the erfc route would round
// 1 - erfc coarsely); from 8 up (and inf, NaN) the clamp at z = 4 already
// gives t or 0.5 t * 0.  tests/test_gelu_erf_cpu.py checks the emulation and
// the closed form for all 65536 codes; the GPU tests check the kernels bit
// for bit on all of them.
constexpr float kErfcA = 0.55f;
constexpr float kErfcP0 = -1.17369068f, kErfcP1 = 1.04755867f, kErfcP2 = 0.0800859705f, kErfcP3 = 0.833066046f,
                kErfcP4 = -1.45879292f, kErfcP5 = 0.85080111f, kErfcP6 = -0.179027811f;
constexpr uint32_t kGeluSmallBits = 0x3B00u;  // bf16 bits of 2^-9

KS_DEV float ks_rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

KS_DEV float gelu_erf(float t) {
  const float x = __fmul_rn(t, 0.70710678118654752f);
  const float z = fminf(fabsf(x), 4.f);
  const float r = ks_rcp_approx(__fmaf_rn(kErfcA, z, 1.f));
  float p = kErfcP6;
  p = __fmaf_rn(p, r, kErfcP5);
  p = __fmaf_rn(p, r, kErfcP4);
  p = __fmaf_rn(p, r, kErfcP3);
  p = __fmaf_rn(p, r, kErfcP2);
  p = __fmaf_rn(p, r, kErfcP1);
  p = __fmaf_rn(p, r, kErfcP0);
  const float q = __fmul_rn(r, ks_ex2(__fmul_rn(__fmaf_rn(-z, z, p), kLog2e)));  // erfc(z)
  const float w = __fadd_rn(1.f, -q);                                          // fp32(erf z)
  const float s = __fadd_rn(1.f, x >= 0.f ? w : -w);                            // fp32(1 + e)
  const float y = __fmul_rn(__fmul_rn(0.5f, t), s);
  return (__float_as_uint(t) & 0x7fff0000u) < (kGeluSmallBits << 16) ? 0.5f * t : y;
}
// The same function as a table: for the 3072 codes with 2^-9 <= |t| < 8,
// GELU of +|t| at [i] and of -|t| at [kGeluTabN + i] (bf16 bits), i = |t|'s
// code - kGeluSmallBits; built per CTA from gelu_erf itself (3072
// evaluations, a few microseconds per launch).  A lookup costs a few integer
// operations and one shared-memory load, far less issue than the formula.
constexpr uint32_t kGeluTabHi = 0x4100u;                     // bf16 bits of 8
constexpr int kGeluTabN = int(kGeluTabHi - kGeluSmallBits);  // 1536 magnitudes

KS_DEV void gelu_erf_table_entries(uint16_t *tab, int i) {
  const float t = __uint_as_float((kGeluSmallBits + uint32_t(i)) << 16);  // +|t|
  tab[i] = ks_f32_to_bf16(gelu_erf(t));
  tab[kGeluTabN + i] = ks_f32_to_bf16(gelu_erf(-t));
}

// GELU of the bf16 code tb (low 16 bits) from the table; codes outside it
// (about 0.1 % of N(0,1) inputs) are computed out of line.  The table is
// built from gelu_erf, so both routes give the same bits.
__device__ __noinline__ uint32_t gelu_erf_edge(uint32_t tb) { return ks_f32_to_bf16(gelu_erf(__uint_as_float(tb << 16))); }
KS_DEV uint32_t gelu_erf_lookup(const uint16_t *tab, uint32_t tb) {
  const uint32_t i = (tb & 0x7fffu) - kGeluSmallBits;  // wraps below the table
  if (i < uint32_t(kGeluTabN)) return tab[i + (tb >> 15) * uint32_t(kGeluTabN)];
  return gelu_erf_edge(tb);
}

KS_DEV float gelu_tanh(float t) {
  // 0.5 t (1 + tanh(u)) = t * sigmoid(2u), u = sqrt(2/pi) (t + 0.044715 t^3).
  const float u = 0.7978845608028654f * fmaf(0.044715f * t, t * t, t);
  const float e = ks_ex2(-2.f * kLog2e * u);
  return __fdividef(t, 1.f + e);
}

// Same function with the constants folded: exp(-2u) = 2^(t * (c1 + c2 t^2)),
// c1 = -2 log2(e) sqrt(2/pi), c2 = 0.044715 c1; y = t / (1 + 2^(...)).
constexpr float kGeluC1 = -2.f * 1.4426950408889634f * 0.7978845608028654f;
constexpr float kGeluC2 = kGeluC1 * 0.044715f;
KS_DEV float gelu_tanh_fast(float t) {
  const float e = ks_ex2(t * fmaf(kGeluC2, t * t, kGeluC1));
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

// 8-wide variant: the loaded words stay packed (4 registers per 8 bf16)
// until they are used, so UNROLL rows of 16-byte loads are in flight per
// thread without spilling.
template <int GELU, int UNROLL>
__global__ void __launch_bounds__(1024) bias_gelu_v8_kernel(const uint16_t *__restrict__ x,
                                                            const uint16_t *__restrict__ bias,
                                                            uint16_t *__restrict__ y, int64_t total, int64_t cols,
                                                            int64_t rows, int rows_per_cta) {
  const int64_t nvec = cols / 8;
  const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= nvec) return;
  const uint4 bw = __ldg(reinterpret_cast<const uint4 *>(bias) + c);
  const __nv_bfloat162 bb[4] = {as_bf162(bw.x), as_bf162(bw.y), as_bf162(bw.z), as_bf162(bw.w)};
  const int64_t r0 = int64_t(blockIdx.y) * rows_per_cta;
  const int64_t r1 = min(rows, r0 + rows_per_cta);
  for (int64_t r = r0; r < r1; r += UNROLL) {
    uint4 w[UNROLL];
    bool ok[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t off = (r + u) * cols + c * 8;
      ok[u] = (r + u < r1) && (off + 8 <= total);
      if (ok[u]) w[u] = __ldcs(reinterpret_cast<const uint4 *>(x + off));
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      if (!ok[u]) continue;
      const uint32_t in[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
      uint32_t outw[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        // fusion point: bf16 + bf16 added exactly and rounded to bf16 once
        const uint32_t t2 = as_u32(__hadd2(as_bf162(in[h]), bb[h]));
        const float t0 = ks_bf16_lo(t2), t1 = ks_bf16_hi(t2);
        const float g0 = GELU == KS_GELU_TANH ? gelu_tanh_fast(t0) : gelu_erf(t0);
        const float g1 = GELU == KS_GELU_TANH ? gelu_tanh_fast(t1) : gelu_erf(t1);
        outw[h] = ks_pack_bf16x2(g0, g1);
      }
      __stcs(reinterpret_cast<uint4 *>(y + (r + u) * cols + c * 8), make_uint4(outw[0], outw[1], outw[2], outw[3]));
    }
  }
}

// Exact-erf GELU, 8-wide, for CTAs below 1024 threads (1024-thread CTAs use
// the whole-code table, bias_gelu_erf_codes_kernel).  Each CTA first builds
// the 6 KB table, then walks
// row groups of `rows_per_group` rows with a grid stride over blockIdx.y (a
// resident grid, so the table is built once per CTA; groups of 32 rows
// measured faster than groups of 4, whose last round is better balanced).
// Every element is one
// shared-memory lookup: the table answers each bf16 code with the
// reference's bits.  (Computing some pairs with gelu_erf instead, to split
// the work between the shared-memory and the FMA/MUFU pipes, measured slower
// at every split: 3.6-4.5 TB/s against 4.9 TB/s with the table alone.)
template <int UNROLL>
__global__ void __launch_bounds__(1024) bias_gelu_erf_v8_kernel(const uint16_t *__restrict__ x,
                                                                const uint16_t *__restrict__ bias,
                                                                uint16_t *__restrict__ y, int64_t total,
                                                                int64_t cols, int64_t rows, int rows_per_group) {
  __shared__ uint16_t tab[2 * kGeluTabN];
  for (int i = threadIdx.x; i < kGeluTabN; i += blockDim.x) gelu_erf_table_entries(tab, i);
  __syncthreads();
  const int64_t nvec = cols / 8;
  const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= nvec) return;
  const uint4 bw = __ldg(reinterpret_cast<const uint4 *>(bias) + c);
  const __nv_bfloat162 bb[4] = {as_bf162(bw.x), as_bf162(bw.y), as_bf162(bw.z), as_bf162(bw.w)};
  const int64_t groups = (rows + rows_per_group - 1) / rows_per_group;
  for (int64_t g = blockIdx.y; g < groups; g += gridDim.y) {
    const int64_t r0 = g * rows_per_group;
    const int64_t r1 = min(rows, r0 + rows_per_group);
    for (int64_t r = r0; r < r1; r += UNROLL) {
      uint4 w[UNROLL];
      bool ok[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int64_t off = (r + u) * cols + c * 8;
        ok[u] = (r + u < r1) && (off + 8 <= total);
        if (ok[u]) w[u] = __ldcs(reinterpret_cast<const uint4 *>(x + off));
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        if (!ok[u]) continue;
        const uint32_t in[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
        uint32_t outw[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          // t = bf16(x + bias): the bf16x2 add rounds the exact sum once
          const uint32_t t2 = as_u32(__hadd2(as_bf162(in[h]), bb[h]));
          outw[h] = __byte_perm(gelu_erf_lookup(tab, t2 & 0xffffu), gelu_erf_lookup(tab, t2 >> 16), 0x5410);
        }
        __stcs(reinterpret_cast<uint4 *>(y + (r + u) * cols + c * 8),
               make_uint4(outw[0], outw[1], outw[2], outw[3]));
      }
    }
  }
}

// Exact-erf GELU of every bf16 code, for the whole-code table below.  Codes
// take one of three routes, each giving the bits gelu_erf gives:
//   * |t| < 2^-9 (zeros and subnormals included): bf16(0.5 t), gelu_erf's
//     own small-input branch;
//   * 8 <= |t| < inf: erfc(min(|x|, 4)) is below 2^-25, so w = fp32(1 - erfc)
//     rounds to 1 and 1 + e is 2 (t >= 8) or 0 (t <= -8): y = t, or -0;
//   * everything else (2^-9 <= |t| < 8, the infinities and NaN): gelu_erf.
KS_DEV uint32_t gelu_erf_code(uint32_t code) {
  const uint32_t e = code & 0x7fffu;
  if (e < kGeluSmallBits) return ks_f32_to_bf16(0.5f * __uint_as_float(code << 16));
  if (e >= kGeluTabHi && e < 0x7f80u) return (code & 0x8000u) ? 0x8000u : code;
  return ks_f32_to_bf16(gelu_erf(__uint_as_float(code << 16)));
}
constexpr int kGeluCodeWords = 1 << 15;                            // two codes per 32-bit word
constexpr size_t kGeluCodeTableBytes = size_t(kGeluCodeWords) * 4;  // 128 KB

// Exact-erf GELU, 8-wide, from a table of all 65536 codes: an element costs
// a 16-bit extract and one shared-memory load, with no range test and no
// sign handling (the 3072-entry table above needs both, and the kernel that
// uses it is issue-bound at 75 % of the copy bandwidth).  The table takes
// 128 KB, so a CTA of 1024 threads owns an SM; it builds the table (3328
// formula evaluations, the rest closed forms) after issuing its first rows'
// loads, then walks row groups with a grid stride over blockIdx.y.
template <int UNROLL>
__global__ void __launch_bounds__(1024) bias_gelu_erf_codes_kernel(const uint16_t *__restrict__ x,
                                                                   const uint16_t *__restrict__ bias,
                                                                   uint16_t *__restrict__ y, int64_t total,
                                                                   int64_t cols, int64_t rows, int rows_per_group) {
  extern __shared__ uint32_t gelu_code_words[];  // word k: code 2k (low half), code 2k+1 (high half)
  const uint16_t *tab = reinterpret_cast<const uint16_t *>(gelu_code_words);
  const int64_t nvec = cols / 8;
  const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t groups = (rows + rows_per_group - 1) / rows_per_group;
  auto load = [&](int64_t g, int64_t r, uint4 *w) {
    const int64_t r1 = min(rows, (g + 1) * rows_per_group);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t off = (r + u) * cols + c * 8;
      if (r + u < r1 && off + 8 <= total) w[u] = __ldcs(reinterpret_cast<const uint4 *>(x + off));
    }
  };
  uint4 w[UNROLL];
  int64_t g = blockIdx.y;
  if (c < nvec && g < groups) load(g, g * rows_per_group, w);
  for (int k = threadIdx.x; k < kGeluCodeWords; k += blockDim.x)
    gelu_code_words[k] = gelu_erf_code(2u * k) | (gelu_erf_code(2u * k + 1) << 16);
  __syncthreads();
  if (c >= nvec) return;
  const uint4 bw = __ldg(reinterpret_cast<const uint4 *>(bias) + c);
  const __nv_bfloat162 bb[4] = {as_bf162(bw.x), as_bf162(bw.y), as_bf162(bw.z), as_bf162(bw.w)};
  bool loaded = true;
  for (; g < groups; g += gridDim.y) {
    const int64_t r1 = min(rows, (g + 1) * rows_per_group);
    for (int64_t r = g * rows_per_group; r < r1; r += UNROLL) {
      if (!loaded) load(g, r, w);
      loaded = false;
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int64_t off = (r + u) * cols + c * 8;
        if (!(r + u < r1 && off + 8 <= total)) continue;
        const uint32_t in[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
        uint32_t outw[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          // t = bf16(x + bias): the bf16x2 add rounds the exact sum once
          const uint32_t t2 = as_u32(__hadd2(as_bf162(in[h]), bb[h]));
          outw[h] = __byte_perm(tab[t2 & 0xffffu], tab[t2 >> 16], 0x5410);
        }
        __stcs(reinterpret_cast<uint4 *>(y + off), make_uint4(outw[0], outw[1], outw[2], outw[3]));
      }
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

// ===========================================================================
// STAGED mode (softmax, layernorm): a ring of whole rows in shared memory,
// each filled by one cp.async.bulk copy.  Thread 0 keeps `stages` rows in
// flight per CTA and refills a slot as soon as the block reduction of the
// row in it has completed (its __syncthreads proves every thread has read
// the slot into registers), so HBM reads never wait on the reductions.
// Rows need cols % 8 == 0 (16-byte copies); chunks are 8 bf16 wide.
// CTAs of up to 512 threads share an SM three ways and keep a 64 KB ring;
// a 1024-thread CTA has the SM to itself and a ring of up to 200 KB, which
// keeps two or three 64 KB rows in flight (layernorm then reads gamma and
// beta through the L2 instead of holding them in the ring).
// ===========================================================================
constexpr int kMaxStages = 8;

struct RowRing {
  uint8_t *base;
  uint32_t stride;  // slot size, rounded up to 128 bytes
  uint32_t bytes;   // row bytes copied per slot
  int stages;
  uint64_t *full;
};

// Issue the copy of local row `i` (global row blockIdx.x + i*gridDim.x) into slot i % stages.
KS_DEV void ring_issue(const RowRing &rg, const uint16_t *x, int64_t cols, int64_t i) {
  const int s = int(i % rg.stages);
  const int64_t r = blockIdx.x + i * gridDim.x;
  ks_mbar_arrive_expect_tx(rg.full + s, rg.bytes);
  ks_bulk_load(rg.base + size_t(s) * rg.stride, x + r * cols, rg.bytes, rg.full + s);
}

// Teardown after an abort at local row `i`: the copies already issued for
// rows [i, min(my_rows, i + stages)) must land before the CTA exits.
KS_DEV void ring_drain(const RowRing &rg, int64_t i, int64_t my_rows, const KsWait &w) {
  for (int64_t j = i; j < my_rows && j < i + rg.stages; ++j)
    ks_mbar_wait(rg.full + (j % rg.stages), uint32_t((j / rg.stages) & 1), nullptr, w);
}

template <int MAXCH, int MAXT>
__global__ void __launch_bounds__(MAXT) softmax_staged_kernel(const uint16_t *__restrict__ x,
                                                              uint16_t *__restrict__ y, int64_t rows,
                                                              int64_t cols, int stages, KsWait wait) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ float sh_max[32], sh_sum[32];
  __shared__ uint64_t full[kMaxStages];
  __shared__ int abort_flag;
  const int64_t my_rows = rows > blockIdx.x ? (rows - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  RowRing rg{dsm, uint32_t((cols * 2 + 127) & ~int64_t(127)), uint32_t(cols * 2), stages, full};
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) ks_mbar_init(full + s, 1);
    abort_flag = 0;
    ks_fence_mbar_init();
    for (int64_t i = 0; i < my_rows && i < stages; ++i) ring_issue(rg, x, cols, i);
  }
  __syncthreads();
  const int nvec = int(cols >> 3);
  int64_t i = 0;
  for (; i < my_rows; ++i) {
    const int s = int(i % stages);
    if (!ks_mbar_wait(full + s, uint32_t((i / stages) & 1), &abort_flag, wait)) break;
    const uint4 *row = reinterpret_cast<const uint4 *>(dsm + size_t(s) * rg.stride);
    uint4 w[MAXCH];
#pragma unroll
    for (int k = 0; k < MAXCH; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      if (c < nvec) w[k] = row[c];
    }
    const int64_t next = i + stages;
    softmax_row8<MAXCH>(w, nvec, sh_max, sh_sum, reinterpret_cast<uint4 *>(y + (blockIdx.x + i * gridDim.x) * cols),
                        [&] {
                          // every thread has read slot s: refill it
                          if (threadIdx.x == 0 && next < my_rows) {
                            ks_fence_proxy_async();
                            ring_issue(rg, x, cols, next);
                          }
                        });
  }
  if (threadIdx.x == 0 && i < my_rows) ring_drain(rg, i, my_rows, wait);
}

template <int MAXCH, int MAXT>
__global__ void __launch_bounds__(MAXT) layernorm_staged_kernel(const uint16_t *__restrict__ x,
                                                                const uint16_t *__restrict__ gamma,
                                                                const uint16_t *__restrict__ beta,
                                                                uint16_t *__restrict__ y, int64_t rows,
                                                                int64_t cols, float inv_cols, float eps, int stages,
                                                                KsWait wait) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ float sh_a[32], sh_b[32];
  __shared__ uint64_t full[kMaxStages];
  __shared__ uint64_t gb_full;
  __shared__ int abort_flag;
  const int64_t my_rows = rows > blockIdx.x ? (rows - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const uint32_t stride = uint32_t((cols * 2 + 127) & ~int64_t(127));
  // slots [0, stages) hold rows; then gamma and beta (CTAs of up to 512
  // threads) -- a 1024-thread CTA reads them from global memory
  constexpr bool kGbShared = MAXT <= 512;
  RowRing rg{dsm, stride, uint32_t(cols * 2), stages, full};
  const uint4 *g_s = kGbShared ? reinterpret_cast<const uint4 *>(dsm + size_t(stages) * stride)
                               : reinterpret_cast<const uint4 *>(gamma);
  const uint4 *b_s = kGbShared ? reinterpret_cast<const uint4 *>(dsm + size_t(stages + 1) * stride)
                               : reinterpret_cast<const uint4 *>(beta);
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) ks_mbar_init(full + s, 1);
    ks_mbar_init(&gb_full, 1);
    abort_flag = 0;
    ks_fence_mbar_init();
    if (kGbShared) {
      ks_mbar_arrive_expect_tx(&gb_full, 2 * uint32_t(cols * 2));
      ks_bulk_load(dsm + size_t(stages) * stride, gamma, uint32_t(cols * 2), &gb_full);
      ks_bulk_load(dsm + size_t(stages + 1) * stride, beta, uint32_t(cols * 2), &gb_full);
    }
    for (int64_t i = 0; i < my_rows && i < stages; ++i) ring_issue(rg, x, cols, i);
  }
  __syncthreads();
  const int nvec = int(cols >> 3);
  const bool gb_ok = kGbShared ? ks_mbar_wait(&gb_full, 0, &abort_flag, wait) : true;
  int64_t i = 0;
  for (; i < my_rows && gb_ok; ++i) {
    const int s = int(i % stages);
    if (!ks_mbar_wait(full + s, uint32_t((i / stages) & 1), &abort_flag, wait)) break;
    const uint4 *row = reinterpret_cast<const uint4 *>(dsm + size_t(s) * stride);
    uint4 w[MAXCH];
#pragma unroll
    for (int k = 0; k < MAXCH; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      if (c < nvec) w[k] = row[c];
    }
    const int64_t next = i + stages;
    layernorm_row8<MAXCH>(w, nvec, inv_cols, eps, g_s, b_s, sh_a, sh_b,
                          reinterpret_cast<uint4 *>(y + (blockIdx.x + i * gridDim.x) * cols), [&] {
                            if (threadIdx.x == 0 && next < my_rows) {
                              ks_fence_proxy_async();
                              ring_issue(rg, x, cols, next);
                            }
                          });
  }
  if (threadIdx.x == 0) {
    if (kGbShared && !gb_ok) ks_mbar_wait(&gb_full, 0, nullptr, wait);
    if (i < my_rows) ring_drain(rg, i, my_rows, wait);
  }
}

// ---------------------------------------------------------------------------
// Host-side dispatch helpers
// ---------------------------------------------------------------------------
constexpr int kRegElems = 32;  // per-thread register budget for a ONEPASS row
constexpr uint32_t kStagedRingBytes = 64 * 1024;       // row ring per CTA (3 CTAs fit an SM)
constexpr uint32_t kStagedRingBytesWide = 200 * 1024;  // 1024-thread CTAs, one per SM

int staged_stages(int64_t cols, int block) {
  const int64_t stride = (cols * 2 + 127) & ~int64_t(127);
  int64_t s = (block == 1024 ? kStagedRingBytesWide : kStagedRingBytes) / stride;
  if (s > kMaxStages) s = kMaxStages;
  return int(s);
}

bool valid_block(int b) { return b == 128 || b == 256 || b == 512 || b == 1024; }
bool valid_vec(int v) { return v == 1 || v == 2 || v == 4 || v == 8; }

bool aligned(const void *p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

template <typename K>
int grid_for(K kernel, int block, int64_t work, size_t dyn_smem = 0) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, block, dyn_smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int64_t cap = int64_t(per_sm) * ks::sm_count();
  return int(work < cap ? work : cap);
}

// ONEPASS rows of at most this many columns (8-wide vectors) run one row per
// warp (softmax_warp_v8_kernel, layernorm_warp_v8_kernel).  Longer rows
// would hold more than 4 chunks per lane and cost the occupancy that keeps
// rows in flight.
constexpr int64_t kWarpRowCols = 1024;
// The 8-wide ONEPASS kernels index rows with int and step by the resident
// grid (r + stride, stride = CTAs x rows per CTA < 2^30), so they take fewer
// than 2^30 rows; r + stride then stays below 2^31.  Larger row counts run
// the int64 generic kernels.
constexpr int64_t kIntRows = int64_t(1) << 30;
// 16-byte chunks per lane for a warp-held row: 1, 2 or 4.
int warp_chunks(int64_t cols) {
  const int64_t per_lane = (cols / 8 + 31) / 32;
  return per_lane <= 1 ? 1 : per_lane <= 2 ? 2 : 4;
}
// A resident grid of `block`-thread CTAs over rows (one row per warp).
template <typename... KArgs, typename... Args>
int launch_rows_warp(void (*k)(KArgs...), int block, int64_t rows, cudaStream_t st, Args... args) {
  const int64_t ctas = (rows + block / 32 - 1) / (block / 32);
  k<<<grid_for(k, block, ctas), block, 0, st>>>(static_cast<KArgs>(args)...);
  return ks::map_cuda(cudaGetLastError());
}

// Cluster size for mode CLUSTER, or 0 when the row cannot be spread: each
// CTA's share of the row (seg = cols / cs) is a multiple of 8 columns and
// holds at most 32 bf16 per thread (16 while the cluster can still grow);
// clusters stay within the portable 8 CTAs and grow while rows x cs leaves
// fewer than two CTAs per SM.
int cluster_plan(int block, int64_t rows, int64_t cols) {
  if (cols % 8 != 0 || block < 256) return 0;
  int cs = 2;
  while (cs < 8 && cols > int64_t(block) * 16 * cs) cs <<= 1;
  const int64_t sms = ks::sm_count();
  while (cs < 8 && rows * cs < 2 * sms && cols % (int64_t(cs) * 16) == 0 && cols / (cs * 2) >= int64_t(block) * 8)
    cs <<= 1;
  if (cols % (int64_t(cs) * 8) != 0 || cols > int64_t(block) * 32 * cs) return 0;
  return cs;
}

// One cluster of cs CTAs per row.
template <typename... KArgs, typename... Args>
int launch_cluster(void (*k)(KArgs...), int cs, int64_t rows, int block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(unsigned(rows * cs));
  c.blockDim = dim3(unsigned(block));
  c.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = unsigned(cs);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  c.attrs = at;
  c.numAttrs = 1;
  return ks::map_cuda(cudaLaunchKernelEx(&c, k, static_cast<KArgs>(args)...));
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
  if (mode != KS_MODE_ONEPASS && mode != KS_MODE_TWOPASS && mode != KS_MODE_STAGED && mode != KS_MODE_CLUSTER) {
    ks::set_reason(reason, len, "%s: mode must be onepass, twopass, staged or cluster", fam);
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
  if ((mode == KS_MODE_ONEPASS || mode == KS_MODE_STAGED) && cols > int64_t(block) * kRegElems) {
    ks::set_reason(reason, len,
                   "%s: %s keeps the row in registers: cols %lld > block %d x %d register elements", fam,
                   mode == KS_MODE_STAGED ? "staged" : "onepass", (long long)cols, block, kRegElems);
    return KS_ERR_INVALID_CONFIG;
  }
  if (mode == KS_MODE_CLUSTER && (vec != 8 || rows >= (int64_t(1) << 28) || cluster_plan(block, rows, cols) == 0)) {
    ks::set_reason(reason, len,
                   "%s: cluster spreads a row over at most 8 CTAs of 32 columns per thread: vec_width must be 8, "
                   "block >= 256, and cols %lld must split into a multiple of 8 columns per CTA within %lld",
                   fam, (long long)cols, (long long)(int64_t(block) * 32 * 8));
    return KS_ERR_INVALID_CONFIG;
  }
  if (mode == KS_MODE_STAGED && (vec != 8 || staged_stages(cols, block) < 2)) {
    ks::set_reason(reason, len,
                   "%s: staged copies whole rows with 16-byte bulk copies: vec_width must be 8 and a two-row "
                   "ring must fit %u bytes (%u at block 1024; cols %lld)",
                   fam, kStagedRingBytes, kStagedRingBytesWide, (long long)cols);
    return KS_ERR_INVALID_CONFIG;
  }
  ks::set_reason(reason, len, "");
  return KS_OK;
}

template <int VEC>
int launch_softmax_vec(const ks_softmax_config &cfg, const ks_softmax_args &a, cudaStream_t st) {
  auto x = static_cast<const uint16_t *>(a.x);
  auto y = static_cast<uint16_t *>(a.out);
  if (cfg.mode == KS_MODE_CLUSTER) {
    if constexpr (VEC == 8) {
      const int cs = cluster_plan(cfg.block, a.rows, a.cols);
      const int seg = int(a.cols / cs);
      if (seg / 8 <= cfg.block)
        return launch_cluster(softmax_cluster_v8_kernel<1>, cs, a.rows, cfg.block, st, x, y, a.cols, seg);
      if (seg / 8 <= 2 * cfg.block)
        return launch_cluster(softmax_cluster_v8_kernel<2>, cs, a.rows, cfg.block, st, x, y, a.cols, seg);
      return launch_cluster(softmax_cluster_v8_kernel<4>, cs, a.rows, cfg.block, st, x, y, a.cols, seg);
    } else {
      return KS_ERR_INVALID_CONFIG;
    }
  } else if (cfg.mode == KS_MODE_STAGED) {
    if constexpr (VEC == 8) {
      const int stages = staged_stages(a.cols, cfg.block);
      const size_t shm = size_t(stages) * size_t((a.cols * 2 + 127) & ~int64_t(127));
      auto k = cfg.block == 1024 ? softmax_staged_kernel<kRegElems / 8, 1024> : softmax_staged_kernel<kRegElems / 8, 512>;
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(shm));
      if (e != cudaSuccess) return ks::map_cuda(e);
      k<<<grid_for(k, cfg.block, a.rows, shm), cfg.block, shm, st>>>(x, y, a.rows, a.cols, stages, ks::wait_ctx());
    } else {
      return KS_ERR_INVALID_CONFIG;
    }
  } else if (cfg.mode == KS_MODE_TWOPASS) {
    auto k = softmax_twopass_kernel<VEC>;
    k<<<grid_for(k, cfg.block, a.rows), cfg.block, 0, st>>>(x, y, a.rows, a.cols);
  } else if (VEC == 8 && a.cols <= kWarpRowCols && a.rows < kIntRows) {
    const int block = cfg.block < 256 ? cfg.block : 256;
    switch (warp_chunks(a.cols)) {
      case 1: return launch_rows_warp(softmax_warp_v8_kernel<1>, block, a.rows, st, x, y, int(a.rows), int(a.cols));
      case 2: return launch_rows_warp(softmax_warp_v8_kernel<2>, block, a.rows, st, x, y, int(a.rows), int(a.cols));
      default:
        return launch_rows_warp(softmax_warp_v8_kernel<4>, block, a.rows, st, x, y, int(a.rows), int(a.cols));
    }
  } else if (VEC == 8 && a.rows < kIntRows && a.cols < (int64_t(1) << 31)) {
    auto k = cfg.block <= 256 ? softmax_onepass_v8_kernel<kRegElems / 8, 256>
                              : softmax_onepass_v8_kernel<kRegElems / 8, 1024>;
    k<<<grid_for(k, cfg.block, a.rows), cfg.block, 0, st>>>(x, y, int(a.rows), int(a.cols));
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
  if (cfg.mode == KS_MODE_CLUSTER) {
    if constexpr (VEC == 8) {
      const int cs = cluster_plan(cfg.block, a.rows, a.cols);
      const int seg = int(a.cols / cs);
      const float ic = 1.f / float(a.cols);
      if (seg / 8 <= cfg.block)
        return launch_cluster(layernorm_cluster_v8_kernel<1>, cs, a.rows, cfg.block, st, x, g, b, y, a.cols, seg,
                              ic, eps);
      if (seg / 8 <= 2 * cfg.block)
        return launch_cluster(layernorm_cluster_v8_kernel<2>, cs, a.rows, cfg.block, st, x, g, b, y, a.cols, seg,
                              ic, eps);
      return launch_cluster(layernorm_cluster_v8_kernel<4>, cs, a.rows, cfg.block, st, x, g, b, y, a.cols, seg, ic,
                            eps);
    } else {
      return KS_ERR_INVALID_CONFIG;
    }
  } else if (cfg.mode == KS_MODE_STAGED) {
    if constexpr (VEC == 8) {
      const bool wide = cfg.block == 1024;
      const int stages = staged_stages(a.cols, cfg.block);
      const size_t shm = size_t(stages + (wide ? 0 : 2)) * size_t((a.cols * 2 + 127) & ~int64_t(127));
      auto k = wide ? layernorm_staged_kernel<kRegElems / 8, 1024> : layernorm_staged_kernel<kRegElems / 8, 512>;
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(shm));
      if (e != cudaSuccess) return ks::map_cuda(e);
      k<<<grid_for(k, cfg.block, a.rows, shm), cfg.block, shm, st>>>(x, g, b, y, a.rows, a.cols,
                                                                     1.f / float(a.cols), eps, stages,
                                                                     ks::wait_ctx());
    } else {
      return KS_ERR_INVALID_CONFIG;
    }
  } else if (cfg.mode == KS_MODE_TWOPASS) {
    auto k = layernorm_twopass_kernel<VEC>;
    k<<<grid_for(k, cfg.block, a.rows), cfg.block, 0, st>>>(x, g, b, y, a.rows, a.cols, eps);
  } else if (VEC == 8 && a.cols <= kWarpRowCols && a.rows < kIntRows) {
    const int block = cfg.block < 256 ? cfg.block : 256;
    const float ic = 1.f / float(a.cols);
    switch (warp_chunks(a.cols)) {
      case 1:
        return launch_rows_warp(layernorm_warp_v8_kernel<1>, block, a.rows, st, x, g, b, y, int(a.rows), int(a.cols),
                                ic, eps);
      case 2:
        return launch_rows_warp(layernorm_warp_v8_kernel<2>, block, a.rows, st, x, g, b, y, int(a.rows), int(a.cols),
                                ic, eps);
      default:
        return launch_rows_warp(layernorm_warp_v8_kernel<4>, block, a.rows, st, x, g, b, y, int(a.rows), int(a.cols),
                                ic, eps);
    }
  } else if (VEC == 8 && a.rows < kIntRows && a.cols < (int64_t(1) << 31)) {
    auto k = cfg.block <= 256 ? layernorm_onepass_v8_kernel<kRegElems / 8, 256>
                              : layernorm_onepass_v8_kernel<kRegElems / 8, 1024>;
    k<<<grid_for(k, cfg.block, a.rows), cfg.block, 0, st>>>(x, g, b, y, int(a.rows), int(a.cols),
                                                            1.f / float(a.cols), eps);
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

// Rows per group for a resident grid of gy row-group slots: about
// kBgRowsPerCta, sized so that every slot walks the same number of groups
// (8192 rows on 74 slots: 4 groups of 28 rows each, where groups of 32 would
// leave the fourth round a third full), a multiple of the kernels' 4-row step.
inline int balanced_rows_per_group(int64_t rows, int64_t gy) {
  const int64_t rounds = std::max<int64_t>(1, (rows + gy * kBgRowsPerCta - 1) / (gy * kBgRowsPerCta));
  const int64_t rpg = (rows + gy * rounds - 1) / (gy * rounds);
  return int(std::max<int64_t>(4, (rpg + 3) / 4 * 4));
}

// The vector kernels stop at the last full VEC chunk of a ragged last row;
// the scalar tail kernel finishes it.
template <int VEC, int GELU>
int launch_bias_gelu_tail(const ks_bias_gelu_args &a, int64_t rows, cudaStream_t st) {
  const int64_t last_row_start = (rows - 1) * a.cols;
  const int64_t tail_len = a.total - last_row_start;
  const int64_t vec_done = (tail_len / VEC) * VEC;
  if (vec_done >= tail_len) return KS_OK;
  const int64_t start = last_row_start + vec_done;
  const int64_t n = a.total - start;
  bias_gelu_tail_kernel<GELU><<<unsigned((n + 255) / 256), 256, 0, st>>>(
      static_cast<const uint16_t *>(a.x), static_cast<const uint16_t *>(a.bias), static_cast<uint16_t *>(a.out),
      start, a.total, a.cols);
  return ks::map_cuda(cudaGetLastError());
}

template <int VEC, int GELU>
int launch_bias_gelu_vec(const ks_bias_gelu_config &cfg, const ks_bias_gelu_args &a, cudaStream_t st) {
  auto x = static_cast<const uint16_t *>(a.x);
  auto b = static_cast<const uint16_t *>(a.bias);
  auto y = static_cast<uint16_t *>(a.out);
  const int64_t rows = (a.total + a.cols - 1) / a.cols;
  const int64_t nvec = a.cols / VEC;
  dim3 grid(unsigned((nvec + cfg.block - 1) / cfg.block), unsigned((rows + kBgRowsPerCta - 1) / kBgRowsPerCta));
  if constexpr (VEC == 8 && GELU == KS_GELU_ERF) {
    if (cfg.block == 1024) {
      // one CTA per SM with the 128 KB table of every code, resident grid over row groups
      auto k = bias_gelu_erf_codes_kernel<4>;
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGeluCodeTableBytes));
      if (e != cudaSuccess) return ks::map_cuda(e);
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 1024, kGeluCodeTableBytes) != cudaSuccess ||
          per_sm < 1)
        per_sm = 1;
      const int64_t resident = int64_t(per_sm) * ks::sm_count();
      const int64_t gy = std::max<int64_t>(1, std::min<int64_t>(grid.y, resident / std::max<int64_t>(1, grid.x)));
      k<<<dim3(grid.x, unsigned(gy)), 1024, kGeluCodeTableBytes, st>>>(x, b, y, a.total, a.cols, rows,
                                                                      balanced_rows_per_group(rows, gy));
      e = cudaGetLastError();
      if (e != cudaSuccess) return ks::map_cuda(e);
      return launch_bias_gelu_tail<VEC, GELU>(a, rows, st);
    }
    // resident grid over row groups: the 6 KB table is built once per CTA
    constexpr int kUnroll = 4;
    auto k = bias_gelu_erf_v8_kernel<kUnroll>;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, cfg.block, 0) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    const int64_t resident = int64_t(per_sm) * ks::sm_count();
    const int64_t gy = std::max<int64_t>(1, std::min<int64_t>(grid.y, resident / std::max<int64_t>(1, grid.x)));
    k<<<dim3(grid.x, unsigned(gy)), cfg.block, 0, st>>>(x, b, y, a.total, a.cols, rows,
                                                        balanced_rows_per_group(rows, gy));
  } else if constexpr (VEC == 8)
    bias_gelu_v8_kernel<GELU, 4><<<grid, cfg.block, 0, st>>>(x, b, y, a.total, a.cols, rows, kBgRowsPerCta);
  else
    bias_gelu_kernel<VEC, GELU, bg_unroll<VEC>()><<<grid, cfg.block, 0, st>>>(x, b, y, a.total, a.cols, rows,
                                                                              kBgRowsPerCta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return ks::map_cuda(e);
  return launch_bias_gelu_tail<VEC, GELU>(a, rows, st);
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
