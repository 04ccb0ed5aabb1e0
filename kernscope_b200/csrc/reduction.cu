// reduction.cu -- the reduction family for sm_100a.
//
// axis = 0  (the reference family, refs.py:102-110, reduction_gen.cpp:127-181):
//   y[j] = sum_i x[i,j].  Thread (tx, ty) of a CTA owns one VEC-wide column
//   chunk and a strided subset of the rows; rows are also split across
//   gridDim.y CTAs so that a few columns still fill 148 SMs.  Per-CTA column
//   partials (fp32) go to the workspace; the last CTA of each column strip
//   (arrival counter) adds the partials in a fixed order and writes y, so the
//   result is deterministic run to run.
// axis = -1 (the full sum of the benchmark configuration):
//   fp32 input read with 128-bit loads, fp32 sums of 16 elements folded into
//   an fp64 per-thread accumulator, fp64 warp/CTA combine, per-CTA fp64
//   partials in the workspace, last CTA sums them in order and writes the
//   fp32 result (and the fp64 value for a cross-GPU combine).
// Both are HBM-bound: 4 (fp32) or 2 (bf16) bytes read per element.
#include <algorithm>
#include <mutex>

#include "ks_common.cuh"

namespace {

// ---------------------------------------------------------------------------
// full sum
// ---------------------------------------------------------------------------
template <int MODE>
KS_DEV double block_sum_f64(double v, double *sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  if (MODE == KS_MODE_TREE) {
    // shared-memory halving tree over every thread's value
    sh[tid] = v;
    __syncthreads();
    for (int o = blockDim.x >> 1; o > 0; o >>= 1) {
      if (tid < o) sh[tid] += sh[tid + o];
      __syncthreads();
    }
    return sh[0];
  }
  // warp shuffles, then one cross-warp exchange
  v = ks_warp_sum_f64(v);
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    double t = lane < nw ? sh[lane] : 0.0;
    t = ks_warp_sum_f64(t);
    if (lane == 0) sh[0] = t;
  }
  __syncthreads();
  return sh[0];
}

template <int MODE>
__global__ void __launch_bounds__(1024) sum_full_f32_kernel(const float *__restrict__ x, int64_t n,
                                                            float *__restrict__ out, double *__restrict__ out_f64,
                                                            double *__restrict__ partials,
                                                            unsigned int *__restrict__ counter) {
  extern __shared__ double shd[];
  __shared__ bool is_last;
  const int64_t nv4 = n / 4;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  double acc = 0.0;
  // 4 independent 16-byte loads in flight per thread per iteration
  for (; i + 3 * stride < nv4; i += 4 * stride) {
    float4 a = __ldcs(x4 + i), b = __ldcs(x4 + i + stride);
    float4 c = __ldcs(x4 + i + 2 * stride), d = __ldcs(x4 + i + 3 * stride);
    const float s = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w)) + ((c.x + c.y) + (c.z + c.w)) +
                    ((d.x + d.y) + (d.z + d.w));
    acc += double(s);
  }
  for (; i < nv4; i += stride) {
    float4 a = __ldcs(x4 + i);
    acc += double((a.x + a.y) + (a.z + a.w));
  }
  // scalar tail (n % 4) handled by the first threads of CTA 0
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) acc += double(x[nv4 * 4 + threadIdx.x]);
  const double cta = block_sum_f64<MODE>(acc, shd);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = cta;
    __threadfence();
    const unsigned int prev = atomicAdd(counter, 1u);
    is_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // fixed-order combine of the per-CTA partials
  double t = 0.0;
  for (int j = threadIdx.x; j < int(gridDim.x); j += blockDim.x) t += __ldcg(partials + j);
  const double total = block_sum_f64<MODE>(t, shd);
  if (threadIdx.x == 0) {
    *out = float(total);
    if (out_f64) *out_f64 = total;
    *counter = 0u;
  }
}

// ---------------------------------------------------------------------------
// axis 0
// ---------------------------------------------------------------------------
template <int VEC, bool BF16_IN>
KS_DEV void load_cols(const void *base, int64_t off, float (&v)[VEC]) {
  if constexpr (BF16_IN) {
    const uint16_t *p = static_cast<const uint16_t *>(base) + off;
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
  } else {
    const float *p = static_cast<const float *>(base) + off;
    if constexpr (VEC == 8) {
      float4 a = __ldcs(reinterpret_cast<const float4 *>(p)), b = __ldcs(reinterpret_cast<const float4 *>(p) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else if constexpr (VEC == 4) {
      float4 a = __ldcs(reinterpret_cast<const float4 *>(p));
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    } else if constexpr (VEC == 2) {
      float2 a = __ldcs(reinterpret_cast<const float2 *>(p));
      v[0] = a.x; v[1] = a.y;
    } else {
      v[0] = __ldcs(p);
    }
  }
}

// Block is (TX, TY) = (blockDim.x, blockDim.y).  CTA (bx, by) covers column
// chunks [bx*TX, bx*TX+TX) and rows by, by+gridDim.y, ... interleaved by TY.
template <int VEC, bool BF16_IN, bool BF16_OUT, int MODE>
__global__ void __launch_bounds__(1024) sum_axis0_kernel(const void *__restrict__ x, void *__restrict__ y,
                                                         int64_t rows, int64_t cols,
                                                         float *__restrict__ partials,
                                                         unsigned int *__restrict__ counters) {
  extern __shared__ float shf[];  // [TY][TX*VEC]
  __shared__ bool is_last;
  const int TX = blockDim.x, TY = blockDim.y, tx = threadIdx.x, ty = threadIdx.y;
  const int64_t nvec = cols / VEC;
  const int64_t cvec = int64_t(blockIdx.x) * TX + tx;
  const bool active = cvec < nvec;
  float acc[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) acc[j] = 0.f;
  if (active) {
    const int64_t rstep = int64_t(TY) * gridDim.y;
    int64_t r = int64_t(blockIdx.y) * TY + ty;
    // four rows per iteration keep four 16-byte loads per thread in flight
    for (; r + 3 * rstep < rows; r += 4 * rstep) {
      float a[VEC], b[VEC], c2[VEC], d[VEC];
      load_cols<VEC, BF16_IN>(x, r * cols + cvec * VEC, a);
      load_cols<VEC, BF16_IN>(x, (r + rstep) * cols + cvec * VEC, b);
      load_cols<VEC, BF16_IN>(x, (r + 2 * rstep) * cols + cvec * VEC, c2);
      load_cols<VEC, BF16_IN>(x, (r + 3 * rstep) * cols + cvec * VEC, d);
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[j] += (a[j] + b[j]) + (c2[j] + d[j]);
    }
    for (; r < rows; r += rstep) {
      float a[VEC];
      load_cols<VEC, BF16_IN>(x, r * cols + cvec * VEC, a);
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[j] += a[j];
    }
  }
  // combine over ty within the CTA
  const int W = TX * VEC;
#pragma unroll
  for (int j = 0; j < VEC; ++j) shf[ty * W + tx * VEC + j] = acc[j];
  __syncthreads();
  if (MODE == KS_MODE_TREE) {
    for (int o = TY >> 1; o > 0; o >>= 1) {
      if (ty < o)
        for (int j = 0; j < VEC; ++j) shf[ty * W + tx * VEC + j] += shf[(ty + o) * W + tx * VEC + j];
      __syncthreads();
    }
  } else if (ty == 0) {
    for (int k = 1; k < TY; ++k)
      for (int j = 0; j < VEC; ++j) shf[tx * VEC + j] += shf[k * W + tx * VEC + j];
  }
  __syncthreads();
  auto write_out = [&](int64_t col, float v) {
    if (BF16_OUT)
      static_cast<uint16_t *>(y)[col] = ks_f32_to_bf16(v);
    else
      static_cast<float *>(y)[col] = v;
  };
  if (gridDim.y == 1) {
    if (ty == 0 && active)
      for (int j = 0; j < VEC; ++j) write_out(cvec * VEC + j, shf[tx * VEC + j]);
    return;
  }
  // cross-CTA: partials[by][col], last arriving CTA of this strip combines
  if (ty == 0 && active)
    for (int j = 0; j < VEC; ++j) partials[int64_t(blockIdx.y) * cols + cvec * VEC + j] = shf[tx * VEC + j];
  __threadfence();
  __syncthreads();
  if (tx == 0 && ty == 0) {
    const unsigned int prev = atomicAdd(counters + blockIdx.x, 1u);
    is_last = (prev == gridDim.y - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // TX*TY threads sum the strip's W columns over gridDim.y partial rows
  const int tid = ty * TX + tx, nt = TX * TY;
  const int64_t col0 = int64_t(blockIdx.x) * W;
  for (int c = tid; c < W; c += nt) {
    const int64_t col = col0 + c;
    if (col >= nvec * VEC) continue;
    float s = 0.f;
    for (unsigned int k = 0; k < gridDim.y; ++k) s += __ldcg(partials + int64_t(k) * cols + col);
    write_out(col, s);
  }
  if (tid == 0) counters[blockIdx.x] = 0u;
}

// ---------------------------------------------------------------------------
// host planning (shared by validate / workspace sizing / launch)
// ---------------------------------------------------------------------------
// Byte offset of the partials inside an axis-0 workspace: the per-strip
// arrival counters come first, rounded up to 256 bytes.
size_t axis0_partials_offset(int64_t n_strips) { return ((size_t(n_strips) * 4 + 255) / 256) * 256; }

struct Plan {
  int64_t n_strips = 0;  // axis 0: column strips (grid.x)
  int split = 1;         // axis 0: row splits (grid.y)
  int tx = 0, ty = 0;
  int grid_full = 0;     // axis -1: CTAs
  size_t ws = 0;
};

bool valid_block(int b) { return b == 128 || b == 256 || b == 512 || b == 1024; }
bool valid_vec(int v) { return v == 1 || v == 2 || v == 4 || v == 8; }

int plan(const ks_reduction_config &c, const ks_reduction_args &a, Plan &p, char *reason, size_t len) {
  if (!valid_block(c.block)) {
    ks::set_reason(reason, len, "reduction: block must be 128, 256, 512 or 1024 (sm_100a space)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (!valid_vec(c.vec_width)) {
    ks::set_reason(reason, len, "reduction: vec_width must be 1, 2, 4 or 8 (sm_100a space)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (c.mode != KS_MODE_STRIDED && c.mode != KS_MODE_TREE) {
    ks::set_reason(reason, len, "reduction: mode must be strided or tree");
    return KS_ERR_INVALID_CONFIG;
  }
  if (a.rows <= 0 || a.cols <= 0) {
    ks::set_reason(reason, len, "reduction: shape (rows, cols) must be positive (got %lld, %lld)",
                   (long long)a.rows, (long long)a.cols);
    return KS_ERR_INVALID_ARGS;
  }
  const int sms = ks::sm_count();  // the current device's SMs (148 on a B200, and without a device)
  if (a.axis == -1) {
    if (a.in_dtype != KS_F32 || a.out_dtype != KS_F32) {
      ks::set_reason(reason, len, "reduction: the full sum (axis -1) takes fp32 in and fp32 out");
      return KS_ERR_INVALID_CONFIG;
    }
    const int64_t n = a.rows * a.cols;
    int64_t ctas = (n / 4 + c.block * 16 - 1) / (int64_t(c.block) * 16);  // >= 16 float4 per thread
    const int64_t cap = int64_t(sms) * (2048 / c.block);
    if (ctas > cap) ctas = cap;
    if (ctas < 1) ctas = 1;
    p.grid_full = int(ctas);
    p.ws = 256 + size_t(ctas) * sizeof(double);
  } else if (a.axis == 0) {
    if ((a.in_dtype != KS_BF16 && a.in_dtype != KS_F32) || (a.out_dtype != KS_BF16 && a.out_dtype != KS_F32)) {
      ks::set_reason(reason, len, "reduction: axis 0 takes bf16/fp32 in and bf16/fp32 out");
      return KS_ERR_INVALID_CONFIG;
    }
    if (a.cols % c.vec_width != 0) {
      ks::set_reason(reason, len, "reduction: cols %lld not divisible by vec_width %d", (long long)a.cols,
                     c.vec_width);
      return KS_ERR_INVALID_CONFIG;
    }
    // A strip is at most 32 vectors wide (256 columns at vec_width 8): one
    // warp spans it, or several rows of it when the rows are narrower; the
    // block's other threads take further rows of the same strip.  Rows are
    // split over gridDim.y CTAs until about 8 CTAs per SM are in flight,
    // but no further than keeps each strip's combine (split x strip width
    // fp32 partials, read by the strip's last CTA) within 128 KB.
    const int64_t nvec = a.cols / c.vec_width;
    int tx = 1;
    while (tx < 32 && tx < nvec) tx <<= 1;
    p.tx = tx;
    p.ty = c.block / tx;
    p.n_strips = (nvec + tx - 1) / tx;
    const int64_t width = std::min<int64_t>(int64_t(tx) * c.vec_width, a.cols);
    const int64_t want = (8LL * sms + p.n_strips - 1) / p.n_strips;
    const int64_t max_split = (a.rows + int64_t(p.ty) * 8 - 1) / (int64_t(p.ty) * 8);
    const int64_t combine_cap = (128 * 1024 / 4) / width;
    int64_t split = want < max_split ? want : max_split;
    if (split > combine_cap) split = combine_cap;
    if (split > 65535) split = 65535;
    if (split < 1) split = 1;
    p.split = int(split);
    p.ws = split > 1 ? axis0_partials_offset(p.n_strips) + size_t(split) * size_t(a.cols) * 4 : 0;
  } else {
    ks::set_reason(reason, len, "reduction: axis must be 0 or -1");
    return KS_ERR_INVALID_CONFIG;
  }
  ks::set_reason(reason, len, "");
  return KS_OK;
}

template <int VEC, bool BI, bool BO>
int launch_axis0_mode(const ks_reduction_config &c, const ks_reduction_args &a, const Plan &p, cudaStream_t st) {
  dim3 grid(unsigned(p.n_strips), unsigned(p.split)), block(p.tx, p.ty);
  const size_t shm = size_t(p.tx) * p.ty * VEC * sizeof(float);
  unsigned int *counters = nullptr;
  float *partials = nullptr;
  if (p.split > 1) {
    counters = reinterpret_cast<unsigned int *>(static_cast<char *>(a.workspace));
    partials = reinterpret_cast<float *>(static_cast<char *>(a.workspace) + axis0_partials_offset(p.n_strips));
    cudaError_t e = cudaMemsetAsync(counters, 0, size_t(p.n_strips) * 4, st);
    if (e != cudaSuccess) return ks::map_cuda(e);
  }
  if (c.mode == KS_MODE_TREE) {
    auto k = sum_axis0_kernel<VEC, BI, BO, KS_MODE_TREE>;
    if (shm > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(shm));
    k<<<grid, block, shm, st>>>(a.x, a.out, a.rows, a.cols, partials, counters);
  } else {
    auto k = sum_axis0_kernel<VEC, BI, BO, KS_MODE_STRIDED>;
    if (shm > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(shm));
    k<<<grid, block, shm, st>>>(a.x, a.out, a.rows, a.cols, partials, counters);
  }
  return ks::map_cuda(cudaGetLastError());
}

template <int VEC>
int launch_axis0(const ks_reduction_config &c, const ks_reduction_args &a, const Plan &p, cudaStream_t st) {
  const bool bi = a.in_dtype == KS_BF16, bo = a.out_dtype == KS_BF16;
  if (bi && bo) return launch_axis0_mode<VEC, true, true>(c, a, p, st);
  if (bi && !bo) return launch_axis0_mode<VEC, true, false>(c, a, p, st);
  if (!bi && bo) return launch_axis0_mode<VEC, false, true>(c, a, p, st);
  return launch_axis0_mode<VEC, false, false>(c, a, p, st);
}

}  // namespace

extern "C" {

int ks_reduction_validate(const ks_reduction_config *cfg, const ks_reduction_args *a, char *reason, size_t len) {
  if (!cfg || !a) return KS_ERR_INVALID_ARGS;
  Plan p;
  return plan(*cfg, *a, p, reason, len);
}

int ks_reduction_workspace_bytes(const ks_reduction_config *cfg, const ks_reduction_args *a, size_t *bytes) {
  if (!cfg || !a || !bytes) return KS_ERR_INVALID_ARGS;
  Plan p;
  int s = plan(*cfg, *a, p, nullptr, 0);
  if (s != KS_OK) return s;
  *bytes = p.ws;
  return KS_OK;
}

int ks_reduction_launch(const ks_reduction_config *cfg, const ks_reduction_args *a, void *stream) {
  if (!cfg || !a || !a->x || !a->out) return KS_ERR_INVALID_ARGS;
  Plan p;
  int s = plan(*cfg, *a, p, nullptr, 0);
  if (s != KS_OK) return s;
  size_t need = 0;
  ks_reduction_workspace_bytes(cfg, a, &need);
  if (need > 0 && (a->workspace == nullptr || a->workspace_bytes < need)) return KS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(a->workspace) % 256 != 0) return KS_ERR_WORKSPACE;
  if ((s = ks::check_arch_sm100()) != KS_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->axis == -1) {
    if (reinterpret_cast<uintptr_t>(a->x) % 16 != 0) return KS_ERR_INVALID_ARGS;
    auto counter = static_cast<unsigned int *>(a->workspace);
    auto partials = reinterpret_cast<double *>(static_cast<char *>(a->workspace) + 256);
    cudaError_t e = cudaMemsetAsync(counter, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return ks::map_cuda(e);
    const size_t shm = (cfg->mode == KS_MODE_TREE ? cfg->block : 32) * sizeof(double);
    if (cfg->mode == KS_MODE_TREE)
      sum_full_f32_kernel<KS_MODE_TREE><<<p.grid_full, cfg->block, shm, st>>>(
          static_cast<const float *>(a->x), a->rows * a->cols, static_cast<float *>(a->out), a->partial_f64,
          partials, counter);
    else
      sum_full_f32_kernel<KS_MODE_STRIDED><<<p.grid_full, cfg->block, shm, st>>>(
          static_cast<const float *>(a->x), a->rows * a->cols, static_cast<float *>(a->out), a->partial_f64,
          partials, counter);
    return ks::map_cuda(cudaGetLastError());
  }
  const int esz = a->in_dtype == KS_BF16 ? 2 : 4;
  if (reinterpret_cast<uintptr_t>(a->x) % (esz * cfg->vec_width) != 0) return KS_ERR_INVALID_ARGS;
  switch (cfg->vec_width) {
    case 8: return launch_axis0<8>(*cfg, *a, p, st);
    case 4: return launch_axis0<4>(*cfg, *a, p, st);
    case 2: return launch_axis0<2>(*cfg, *a, p, st);
    default: return launch_axis0<1>(*cfg, *a, p, st);
  }
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Reduction without caller-provided workspace.
//
// Some callers cannot call cudaMalloc: a plugin whose host framework owns all
// device memory (its allocator reserved the GPU's memory up front, so a
// direct cudaMalloc fails or competes with it), or a latency-critical path
// that cannot pay cudaMalloc's device-wide synchronisation.  They still pass
// their input and output buffers; the per-CTA partials and arrival counters
// live in the fixed scratch array below instead of a workspace.
//
// * The array is kReductionNoallocScratchBytes (1 MiB) and, like any
//   __device__ variable, is held on every GPU that loads this library until
//   the process exits.  Launches whose workspace would be larger return
//   KS_ERR_WORKSPACE.
// * Host code cannot use the array's name as a device address (it names a
//   host-side shadow).  The first call in each driver context (normally a
//   device's primary context) resolves the address with cudaGetSymbolAddress
//   while that device is current and caches it per context; make that first
//   call before any stream capture.  cudaDeviceReset destroys the context and
//   the array with it: do not call this entry point again after a reset in
//   the same process.
// * Every call shares the one array and it keeps the last call's contents;
//   the launch clears the arrival counters it needs on the stream before the
//   kernel.  Calls that overlap on the GPU (concurrent streams, several host
//   threads) race on the array and must be serialised by the caller.
// * Nothing here allocates: no cudaMalloc/cudaFree, no allocating library.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kReductionNoallocScratchBytes = size_t(1) << 20;
static_assert(kReductionNoallocScratchBytes == KS_REDUCTION_NOALLOC_SCRATCH_BYTES, "header and library disagree");

static __device__ __align__(256) unsigned char g_reduction_scratch[kReductionNoallocScratchBytes];

}  // namespace

extern "C" int ks_reduction_launch_noalloc(const ks_reduction_config *cfg, const ks_reduction_args *args,
                                           void *stream) {
  if (!cfg || !args || !args->x || !args->out) return KS_ERR_INVALID_ARGS;  // before any CUDA call
  size_t need = 0;
  int s = ks_reduction_workspace_bytes(cfg, args, &need);
  if (s != KS_OK) return s;
  if (need > kReductionNoallocScratchBytes) return KS_ERR_WORKSPACE;
  void *scratch = nullptr;
  if ((s = ks::symbol_address(reinterpret_cast<const void *>(&g_reduction_scratch), &scratch)) != KS_OK) return s;
  ks_reduction_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kReductionNoallocScratchBytes;
  return ks_reduction_launch(cfg, &a, stream);
}
