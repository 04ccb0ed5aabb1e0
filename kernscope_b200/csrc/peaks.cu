// peaks.cu -- roofline peak probes for kernscope-bench on sm_100a.
//
// The reference measures its roofline denominators with a small kernel set
// (libs/bench/kernels/peaks.hip: device-to-device copy, read-only sweep,
// FFMA chains, LDS bandwidth) driven by tools/bench/main.cpp.  The B200
// counterparts here:
//
//   * copy / read: grid-stride 16-byte vector loops over HBM-resident
//     buffers (HBM bandwidth; read+write bytes for the copy, read bytes for
//     the sweep);
//   * bf16 tensor peak: one CTA per SM issuing back-to-back tcgen05.mma
//     (kind::f16, M=128, N=256, K=16) from operands that stay in shared
//     memory, accumulating in TMEM -- the tensor pipe with no memory traffic;
//   * fp32 FFMA peak: independent FMA chains on every lane;
//   * shared-memory bandwidth: 16-byte ld.shared loops.
//
// Operand values are pseudo-random (not zero) so the tensor and FMA pipes
// toggle as they do on real data: the power draw, and so the clock the
// peak is measured at, depends on it.
#include <cmath>

#include "ks_common.cuh"

namespace {

constexpr int kReadBlocksPerSm = 8;
constexpr int kReadThreads = 512;

__global__ void __launch_bounds__(512) peak_copy_kernel(const uint4 *__restrict__ src, uint4 *__restrict__ dst,
                                                        size_t n16) {
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = __ldcs(src + i), b = __ldcs(src + i + stride), c = __ldcs(src + i + 2 * stride),
                d = __ldcs(src + i + 3 * stride);
    __stcs(dst + i, a);
    __stcs(dst + i + stride, b);
    __stcs(dst + i + 2 * stride, c);
    __stcs(dst + i + 3 * stride, d);
  }
  for (; i < n16; i += stride) __stcs(dst + i, __ldcs(src + i));
}

__global__ void __launch_bounds__(kReadThreads) peak_read_kernel(const uint4 *__restrict__ src, size_t n16,
                                                                 uint32_t *__restrict__ sink) {
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  uint32_t x = 0;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = __ldcs(src + i), b = __ldcs(src + i + stride), c = __ldcs(src + i + 2 * stride),
                d = __ldcs(src + i + 3 * stride);
    x ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
  }
  for (; i < n16; i += stride) {
    const uint4 a = __ldcs(src + i);
    x ^= a.x ^ a.y ^ a.z ^ a.w;
  }
  // one word per block keeps the loads live
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x ^= __shfl_xor_sync(0xffffffffu, x, o);
  __shared__ uint32_t w[kReadThreads / 32];
  if ((threadIdx.x & 31) == 0) w[threadIdx.x >> 5] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t y = 0;
    for (int k = 0; k < kReadThreads / 32; ++k) y ^= w[k];
    sink[blockIdx.x] = y;
  }
}

KS_DEV uint32_t mix32(uint32_t v) {
  v ^= v >> 16;
  v *= 0x7feb352du;
  v ^= v >> 15;
  v *= 0x846ca68bu;
  return v ^ (v >> 16);
}

// bf16 in [-1, 1) from a hash (sign, exponent 2^-1..2^-8, random mantissa)
KS_DEV uint16_t rand_bf16(uint32_t i) {
  const uint32_t h = mix32(i);
  return uint16_t(((h & 1u) << 15) | ((126u - ((h >> 1) & 7u)) << 7) | ((h >> 4) & 0x7fu));
}

constexpr int kMmaN = 256;
constexpr uint32_t kMmaABytes = 128 * 64 * 2;    // [128 rows x 64 K] SW128, K-major
constexpr uint32_t kMmaBBytes = 64 * kMmaN * 2;  // [64 K x 256 N] as four 64-column SW128 boxes
// More than half the SM's shared memory, so exactly one CTA (and one TMEM
// allocation) per SM.
constexpr uint32_t kMmaSmem = 120 * 1024;
static_assert(kMmaABytes + kMmaBBytes + 64 + 1024 <= kMmaSmem, "operands fit");

__global__ void __launch_bounds__(128, 1) peak_mma_kernel(long long iters, uint32_t *__restrict__ sink, KsWait wait) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ks_smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint16_t *ab = reinterpret_cast<uint16_t *>(smem);
  uint64_t *drain = reinterpret_cast<uint64_t *>(smem + kMmaABytes + kMmaBBytes);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kMmaABytes + kMmaBBytes + 8);
  // operands: any bf16 bit pattern is a valid swizzled tile; fill with data
  for (uint32_t i = threadIdx.x; i < (kMmaABytes + kMmaBBytes) / 2; i += blockDim.x)
    ab[i] = rand_bf16(i * 2654435761u + blockIdx.x);
  ks_fence_proxy_async();  // generic-proxy writes, read by the tensor core
  if (threadIdx.x == 0) {
    ks_mbar_init(drain, 1);
    ks_fence_mbar_init();
  }
  const int warp = threadIdx.x >> 5;
  if (warp == 0) {
    ks_tmem_alloc(tmem_slot, kMmaN);
    ks_tmem_relinquish();
  }
  ks_tc_fence_before();
  __syncthreads();
  ks_tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = ks_idesc_bf16_f32(128, kMmaN, false, true);
    const uint32_t a_addr = ks_smem_u32(smem), b_addr = a_addr + kMmaABytes;
    for (long long it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        ks_umma_ss(tmem, ks_umma_desc_sw128(a_addr + k * 32, 16, 1024),
                   ks_umma_desc_sw128(b_addr + k * 2048, 64 * 64 * 2, 1024), idesc, (it | k) != 0);
    }
    ks_umma_commit(drain);
    ks_mbar_wait(drain, 0, nullptr, wait);
  }
  __syncthreads();
  ks_tc_fence_after();
  // one accumulator column per lane to global: the MMAs' result is used
  uint32_t r[16];
  ks_tmem_ld16(tmem + (uint32_t(warp * 32) << 16), r);
  ks_tmem_wait_ld();
  sink[blockIdx.x * 128 + threadIdx.x] = r[0] ^ r[15];
  ks_tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ks_tc_fence_after();
    ks_tmem_dealloc(tmem, kMmaN);
  }
}

constexpr int kFmaChains = 8;

__global__ void __launch_bounds__(256) peak_ffma_kernel(long long iters, float *__restrict__ sink) {
  float x[kFmaChains];
#pragma unroll
  for (int c = 0; c < kFmaChains; ++c) x[c] = 0.001f * float(threadIdx.x + c);
  const float a = 0.9999f, b = 0.0001f;
  for (long long it = 0; it < iters; ++it) {
#pragma unroll
    for (int c = 0; c < kFmaChains; ++c) x[c] = fmaf(x[c], a, b);
  }
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kFmaChains; ++c) s += x[c];
  sink[size_t(blockIdx.x) * blockDim.x + threadIdx.x] = s;
}

// Each warp reads 512 contiguous bytes per load (four 128-byte wavefronts,
// no bank conflicts); 32 KB per block, four blocks per SM.
__global__ void __launch_bounds__(512) peak_smem_kernel(long long iters, uint32_t *__restrict__ sink) {
  __shared__ uint4 buf[2048];  // 32 KB
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) buf[i] = make_uint4(i, i * 3u, i * 5u, i * 7u);
  __syncthreads();
  uint32_t x = 0;
  int idx = threadIdx.x;
  for (long long it = 0; it < iters; ++it) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint4 v = buf[(idx + u * 512) & 2047];
      x ^= v.x ^ v.y ^ v.z ^ v.w;
    }
    idx = (idx + 32) & 2047;
  }
  sink[size_t(blockIdx.x) * blockDim.x + threadIdx.x] = x;
}

}  // namespace

extern "C" {

int ks_peak_sink_words(size_t *words) {
  if (!words) return KS_ERR_INVALID_ARGS;
  *words = size_t(ks::sm_count()) * 4 * 512;  // the largest grid x block any probe writes
  return KS_OK;
}

int ks_peak_copy(void *dst, const void *src, size_t bytes, void *stream) {
  if (!dst || !src || bytes % 16 != 0) return KS_ERR_INVALID_ARGS;
  if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) return KS_ERR_INVALID_ARGS;
  int s = ks::check_arch_sm100();
  if (s != KS_OK || bytes == 0) return s;
  const int grid = ks::sm_count() * 4;
  peak_copy_kernel<<<grid, 512, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint4 *>(src),
                                                                       static_cast<uint4 *>(dst), bytes / 16);
  return ks::map_cuda(cudaGetLastError());
}

int ks_peak_read(const void *src, size_t bytes, void *sink, void *stream) {
  if (!src || !sink || bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(src) & 15u)) return KS_ERR_INVALID_ARGS;
  int s = ks::check_arch_sm100();
  if (s != KS_OK || bytes == 0) return s;
  const int grid = ks::sm_count() * kReadBlocksPerSm / 2;  // 4 x 512 threads per SM
  peak_read_kernel<<<grid, kReadThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4 *>(src), bytes / 16, static_cast<uint32_t *>(sink));
  return ks::map_cuda(cudaGetLastError());
}

int ks_peak_mma_bf16(long long iters, void *sink, double *flops, void *stream) {
  if (!sink || iters <= 0) return KS_ERR_INVALID_ARGS;
  int s = ks::check_arch_sm100();
  if (s != KS_OK) return s;
  cudaError_t e = cudaFuncSetAttribute(peak_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMmaSmem));
  if (e != cudaSuccess) return ks::map_cuda(e);
  const int grid = ks::sm_count();
  peak_mma_kernel<<<grid, 128, kMmaSmem, static_cast<cudaStream_t>(stream)>>>(iters, static_cast<uint32_t *>(sink),
                                                                             ks::wait_ctx());
  if (flops) *flops = double(grid) * double(iters) * 4.0 * 2.0 * 128.0 * kMmaN * 16.0;
  return ks::map_cuda(cudaGetLastError());
}

int ks_peak_ffma_f32(long long iters, void *sink, double *flops, void *stream) {
  if (!sink || iters <= 0) return KS_ERR_INVALID_ARGS;
  int s = ks::check_arch_sm100();
  if (s != KS_OK) return s;
  const int grid = ks::sm_count() * 4;
  peak_ffma_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(iters, static_cast<float *>(sink));
  if (flops) *flops = double(grid) * 256.0 * double(iters) * kFmaChains * 2.0;
  return ks::map_cuda(cudaGetLastError());
}

int ks_peak_smem(long long iters, void *sink, double *bytes, void *stream) {
  if (!sink || iters <= 0) return KS_ERR_INVALID_ARGS;
  int s = ks::check_arch_sm100();
  if (s != KS_OK) return s;
  const int grid = ks::sm_count() * 4;
  peak_smem_kernel<<<grid, 512, 0, static_cast<cudaStream_t>(stream)>>>(iters, static_cast<uint32_t *>(sink));
  if (bytes) *bytes = double(grid) * 512.0 * double(iters) * 4.0 * 16.0;
  return ks::map_cuda(cudaGetLastError());
}

}  // extern "C"
