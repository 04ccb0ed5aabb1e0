/*
 * kernscope_b200.h -- C ABI of the B200 (sm_100a) kernel library that backs
 * the six kernscope-tune kernel families.
 *
 * The reference binds its kernels through a C++ runtime class
 * (libs/gpuruntime/include/kernscope/gpu.h:182-255: Module::load,
 * Kernel::create, Kernel::launch) and a raw kernel ABI of
 * `(const T* in..., T* out, int32 scalars...)` per family
 * (kernels/templates/README.md:38-48, kernels/templates/tests/
 * run_hip_gate.py:93-182).  TMA-fed kernels need host-built tensor maps, so
 * the boundary here sits one level up: one `ks_<family>_launch` per family
 * taking the reference's pointers and scalars in the reference's order (in
 * an args struct, 64-bit sizes) plus an sm_100a config struct, returning a
 * ks_status.  No exceptions cross this ABI.  Launches are asynchronous on
 * the caller's stream (a cudaStream_t passed as void*; NULL = legacy default
 * stream), allocate nothing, and are safe to call from several threads.
 *
 * All tensors are dense row-major device buffers.  bf16 is IEEE bfloat16
 * stored as 16-bit words.
 */
#ifndef KERNSCOPE_B200_H
#define KERNSCOPE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KS_ABI_VERSION 1

/* ---- status codes ------------------------------------------------------
 * 0 = success.  Negative values are errors.  -1..-11 mirror the reference's
 * GpuError enumerators numerically (libs/gpuruntime/include/kernscope/
 * gpu.h:77-90, negated); -20.. are codes of the kernel families.          */
typedef enum ks_status {
  KS_OK = 0,
  KS_ERR_NO_DEVICE = -1,          /* GpuError::kNoDevice */
  KS_ERR_NO_DRIVER = -2,          /* GpuError::kNoDriver */
  KS_ERR_MODULE_LOAD = -3,        /* GpuError::kModuleLoadFailed */
  KS_ERR_KERNEL_NOT_FOUND = -4,   /* GpuError::kKernelNotFound */
  KS_ERR_LAUNCH = -5,             /* GpuError::kLaunchFailed */
  KS_ERR_MEMORY = -6,             /* GpuError::kMemoryOpFailed */
  KS_ERR_COPY = -7,               /* GpuError::kCopyOpFailed */
  KS_ERR_EVENT = -8,              /* GpuError::kEventOpFailed */
  KS_ERR_DEVICE_NOT_FOUND = -9,   /* GpuError::kDeviceNotFound */
  KS_ERR_UNSUPPORTED = -10,       /* GpuError::kUnsupportedBackend */
  KS_ERR_OTHER = -11,             /* GpuError::kOther */
  KS_ERR_INVALID_CONFIG = -20,    /* config outside the sm_100a space */
  KS_ERR_INVALID_ARGS = -21,      /* null pointer, bad size, misalignment */
  KS_ERR_WORKSPACE = -22,         /* workspace missing or too small */
  KS_ERR_DEVICE_TIMEOUT = -23,    /* a bounded device wait gave up */
  KS_ERR_ARCH = -24               /* current device is not sm_100 */
} ks_status;

/* Stable name of a status ("ok", "invalid_config", ...). Never NULL. */
const char *ks_status_string(int status);
/* Library ABI version (KS_ABI_VERSION) and build string. */
int ks_abi_version(void);
const char *ks_build_info(void);

/* ---- runtime (replaces libs/gpuruntime's GpuRuntime, gpu.h:182-255) ---- */
int ks_gpu_device_count(int *count);
int ks_gpu_set_device(int device);
int ks_gpu_get_device(int *device);
/* "sm_100a" for compute capability 10.0; "sm_XY" otherwise. */
int ks_gpu_arch(int device, char *buf, size_t len);
int ks_gpu_sm_count(int device, int *count);
int ks_gpu_l2_bytes(int device, size_t *bytes);
int ks_gpu_malloc(void **ptr, size_t bytes);
int ks_gpu_free(void *ptr);
int ks_gpu_memset(void *ptr, int value, size_t bytes, void *stream);
int ks_gpu_memcpy_htod(void *dst, const void *src, size_t bytes, void *stream);
int ks_gpu_memcpy_dtoh(void *dst, const void *src, size_t bytes, void *stream);
int ks_gpu_host_alloc(void **ptr, size_t bytes);  /* pinned host memory */
int ks_gpu_host_free(void *ptr);
int ks_gpu_stream_create(void **stream);
int ks_gpu_stream_destroy(void *stream);
int ks_gpu_stream_synchronize(void *stream);
int ks_gpu_synchronize(void);
int ks_gpu_event_create(void **event);
int ks_gpu_event_destroy(void *event);
int ks_gpu_event_record(void *event, void *stream);
int ks_gpu_event_synchronize(void *event);
int ks_gpu_event_elapsed_ms(void *start, void *stop, float *ms);

/* Device error word written by bounded waits inside the kernels (0 = none).
 * Reads and clears it on the current device; synchronizes the device. */
int ks_device_error_take(int *word);
/* Self-test of the bounded-wait path: one CTA waits on an mbarrier that
 * nothing arrives on, gives up after `limit_ns`, records the timeout in the
 * device error word and returns normally.  Returns KS_ERR_DEVICE_TIMEOUT
 * when the timeout was recorded (the expected outcome). */
int ks_selftest_bounded_wait(uint64_t limit_ns, void *stream);
/* Bound (ns) that every spin-wait in the kernels uses; default 4e9. */
int ks_set_wait_limit_ns(uint64_t limit_ns);

/* ---- shared enums ------------------------------------------------------ */
typedef enum ks_dtype { KS_BF16 = 0, KS_F32 = 1, KS_F64 = 2 } ks_dtype;

/* Row-op strategy (ElemMode, tools/tune/include/kernscope/tune/
 * elem_common.h:49-55).  ONEPASS: the row is read from HBM once and held in
 * registers, both reductions run over registers.  TWOPASS: the row is
 * re-read for the second statistic (second read served by L2), which lifts
 * the register cap on the row length.  STAGED (softmax, layernorm): a ring
 * of whole rows in shared memory filled by bulk copies keeps several rows
 * per CTA in flight (vec_width 8, cols % 8 == 0; a 64 KB ring up to 512
 * threads, cols <= 16384; a 200 KB ring at 1024 threads, cols <= 32768). */
typedef enum ks_elem_mode {
  KS_MODE_ONEPASS = 0,
  KS_MODE_TWOPASS = 1,
  KS_MODE_STRIDED = 2,  /* reduction: warp-shuffle combine */
  KS_MODE_TREE = 3,     /* reduction: shared-memory tree combine */
  KS_MODE_STAGED = 4,
  KS_MODE_CLUSTER = 5   /* softmax, layernorm: one row over a cluster of 2-8
                           CTAs, statistics combined through distributed
                           shared memory (vec_width 8; long rows, few rows) */
} ks_elem_mode;

/* ---- softmax (tools/tune/include/kernscope/tune/softmax_gen.h:39-51) ----
 * y[r,:] = softmax(x[r,:]) over the last axis; bf16 in/out, fp32 math.
 * Reference kernel arguments: (x, out, rows, cols).
 * cfg.block: threads per row-CTA {128,256,512,1024};
 * cfg.vec_width: bf16 per vector access {1,2,4,8} (8 = 128-bit);
 * cfg.mode: KS_MODE_ONEPASS | KS_MODE_TWOPASS | KS_MODE_STAGED |
 *           KS_MODE_CLUSTER (the same modes apply to layernorm).           */
typedef struct ks_softmax_config { int block; int vec_width; int mode; } ks_softmax_config;
typedef struct ks_softmax_args {
  const void *x; void *out; int64_t rows; int64_t cols;
} ks_softmax_args;
int ks_softmax_validate(const ks_softmax_config *cfg, int64_t rows, int64_t cols,
                        char *reason, size_t reason_len);
int ks_softmax_launch(const ks_softmax_config *cfg, const ks_softmax_args *args,
                      void *stream);

/* ---- layernorm (layernorm_gen.h:45-57) ---------------------------------
 * y = (x-mean)/sqrt(var+eps)*gamma+beta over the last axis, biased
 * variance; eps <= 0 selects the reference's pinned 1e-5.
 * Reference kernel arguments: (x, gamma, beta, out, rows, cols).           */
typedef struct ks_layernorm_config { int block; int vec_width; int mode; } ks_layernorm_config;
typedef struct ks_layernorm_args {
  const void *x; const void *gamma; const void *beta; void *out;
  int64_t rows; int64_t cols; float eps;
} ks_layernorm_args;
int ks_layernorm_validate(const ks_layernorm_config *cfg, int64_t rows, int64_t cols,
                          char *reason, size_t reason_len);
int ks_layernorm_launch(const ks_layernorm_config *cfg, const ks_layernorm_args *args,
                        void *stream);

/* ---- bias_gelu (bias_gelu_gen.h:40-53) ---------------------------------
 * y[i] = GELU(bf16(x[i] + bias[i % cols])); gelu = KS_GELU_ERF is the
 * reference's exact-erf GELU (refs.py:59-76), KS_GELU_TANH the tanh
 * approximation.  Reference kernel arguments: (x, bias, out, total, cols). */
typedef enum ks_gelu_kind { KS_GELU_ERF = 0, KS_GELU_TANH = 1 } ks_gelu_kind;
typedef struct ks_bias_gelu_config { int block; int vec_width; int gelu; } ks_bias_gelu_config;
typedef struct ks_bias_gelu_args {
  const void *x; const void *bias; void *out; int64_t total; int64_t cols;
} ks_bias_gelu_args;
int ks_bias_gelu_validate(const ks_bias_gelu_config *cfg, int64_t total, int64_t cols,
                          char *reason, size_t reason_len);
int ks_bias_gelu_launch(const ks_bias_gelu_config *cfg, const ks_bias_gelu_args *args,
                        void *stream);

/* ---- reduction (reduction_gen.h:40-53) ---------------------------------
 * axis = 0 : y[j] = sum_i x[i,j] (the reference family; bf16 or fp32 in,
 *            fp32 accumulate, bf16 or fp32 out).
 * axis = -1: y[0] = sum of all rows*cols elements (fp32 in, fp64 partials,
 *            fp32 out); `partial_f64`, when non-NULL, also receives the
 *            device's fp64 sum for a cross-GPU combine.
 * Reference kernel arguments: (x, out, rows, cols).  Both axes use a
 * caller-provided workspace of ks_reduction_workspace_bytes() bytes (the
 * per-CTA partials and the arrival counter); the launch clears what it
 * needs inside the workspace itself.                                        */
typedef struct ks_reduction_config { int block; int vec_width; int mode; } ks_reduction_config;
typedef struct ks_reduction_args {
  const void *x; void *out; int64_t rows; int64_t cols;
  int in_dtype; int out_dtype; int axis;
  void *workspace; size_t workspace_bytes; double *partial_f64;
} ks_reduction_args;
int ks_reduction_validate(const ks_reduction_config *cfg, const ks_reduction_args *args,
                          char *reason, size_t reason_len);
int ks_reduction_workspace_bytes(const ks_reduction_config *cfg,
                                 const ks_reduction_args *args, size_t *bytes);
int ks_reduction_launch(const ks_reduction_config *cfg, const ks_reduction_args *args,
                        void *stream);

/* No counterpart in the reference.  ks_reduction_launch for callers that
 * cannot call cudaMalloc -- e.g. a plugin whose host framework owns all
 * device memory (its allocator reserved the GPU up front), or a
 * latency-critical path that cannot take cudaMalloc's device-wide
 * synchronisation.  Same arguments and results; args->workspace and
 * args->workspace_bytes are ignored: the partials and counters live in a
 * library-owned static device array of KS_REDUCTION_NOALLOC_SCRATCH_BYTES,
 * held on every GPU that loads the library until the process exits.
 * Returns KS_ERR_WORKSPACE when ks_reduction_workspace_bytes() for these
 * args exceeds that size.  The first call in each driver context (normally
 * a device's primary context) resolves the array's device address (do it
 * before any stream capture); cudaDeviceReset destroys the array with the
 * context, so do not call this again after a reset in the same process.  All calls
 * share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  Allocates nothing.                            */
#define KS_REDUCTION_NOALLOC_SCRATCH_BYTES (1u << 20)
int ks_reduction_launch_noalloc(const ks_reduction_config *cfg, const ks_reduction_args *args,
                                void *stream);

/* ---- matmul (matmul_gen.h:97-174) ----------------------------------------
 * C[M,N] = A[M,K] . B[K,N]; A row-major (K contiguous), B row-major
 * (N contiguous), C row-major; bf16 in/out, fp32 accumulate in TMEM.
 * Reference kernel arguments: (a, b, out, m, n, k).
 * Config (sm_100a space): tile_m 128|256; tile_n {64,128,256} (128|256 at
 * tile_m 256); tile_k 64; stages 2..6 (fewer where the ring would not fit
 * 227 KB); acc_stages 1|2 (TMEM accumulator buffers, acc_stages x tile_n x
 * tile_m/128 <= 512 columns for one-CTA tiles); group_m 1..64 (tile
 * raster: M-tiles per L2 group) or -32..-1 (bands of -group_m N-tiles whose
 * B panels are loaded evict_last; the CTA pair walks the same bands with
 * plain loads); cta_group, for tile_m 256: 2 = a CTA pair issuing
 * cta_group::2 M=256 MMAs across two SMs, 1 = one CTA issuing two M=128
 * MMAs per B tile, 0 = the default (2).  K % 8 == 0 and N % 8 == 0 (16-byte
 * TMA strides); any M; pointers 16-byte aligned.                            */
typedef struct ks_matmul_config {
  int tile_m; int tile_n; int tile_k; int stages; int acc_stages; int group_m; int cta_group;
} ks_matmul_config;
typedef struct ks_matmul_args {
  const void *a; const void *b; void *out; int64_t m; int64_t n; int64_t k;
} ks_matmul_args;
int ks_matmul_validate(const ks_matmul_config *cfg, int64_t m, int64_t n, int64_t k,
                       char *reason, size_t reason_len);
int ks_matmul_launch(const ks_matmul_config *cfg, const ks_matmul_args *args, void *stream);

/* ---- flash_attention (flash_attention_gen.h:83-168) -----------------------
 * O = softmax(Q K^T * scale [+ causal mask]) V, forward only.  Q [B,H,Nq,d],
 * K/V [B,H,Nk,d], O [B,H,Nq,d], bf16, fp32 online-softmax statistics.
 * batch = heads = 1 is the reference's single-head ABI (q, k, v, out, nq,
 * nk, d).  scale <= 0 selects 1/sqrt(d).  causal masks col > row (the
 * reference's gj > gi test).  d in 1..256: tensor cores at d = 128 (either
 * tile_m) and d = 64 (tile_m 256), CUDA cores otherwise; Nq, Nk any positive
 * value.                                                                    */
typedef struct ks_flash_attention_config {
  int tile_m; int tile_n; int stages; int causal;
} ks_flash_attention_config;
typedef struct ks_flash_attention_args {
  const void *q; const void *k; const void *v; void *out;
  int64_t batch; int64_t heads; int64_t nq; int64_t nk; int64_t d; float scale;
} ks_flash_attention_args;
int ks_flash_attention_validate(const ks_flash_attention_config *cfg,
                                const ks_flash_attention_args *args,
                                char *reason, size_t reason_len);
int ks_flash_attention_launch(const ks_flash_attention_config *cfg,
                              const ks_flash_attention_args *args, void *stream);

/* ---- roofline peak probes (libs/bench/kernels/peaks.hip, driven by
 * tools/bench/main.cpp: kernscope-bench) ------------------------------------
 * Each enqueues one kernel on `stream` and returns at once; time them with
 * events.  `sink` is a device buffer of at least ks_peak_sink_words() 32-bit
 * words (keeps the probes' results live).
 *   ks_peak_copy:     dst <- src, `bytes` (multiple of 16, 16-byte aligned);
 *                     HBM traffic = 2 * bytes.
 *   ks_peak_read:     read-only sweep of `bytes`; traffic = bytes.
 *   ks_peak_mma_bf16: one CTA per SM issuing `iters` x 4 tcgen05.mma
 *                     (bf16 -> fp32, M=128, N=256, K=16) from shared memory;
 *                     *flops = FLOPs of the launch.
 *   ks_peak_ffma_f32: fp32 FMA chains; *flops = FLOPs of the launch.
 *   ks_peak_smem:     16-byte shared-memory loads; *bytes = bytes read.     */
int ks_peak_sink_words(size_t *words);
int ks_peak_copy(void *dst, const void *src, size_t bytes, void *stream);
int ks_peak_read(const void *src, size_t bytes, void *sink, void *stream);
int ks_peak_mma_bf16(long long iters, void *sink, double *flops, void *stream);
int ks_peak_ffma_f32(long long iters, void *sink, double *flops, void *stream);
int ks_peak_smem(long long iters, void *sink, double *bytes, void *stream);

/* ---- symbols --------------------------------------------------------------
 * Stable per-config kernel symbol (kernel_symbol(), e.g. matmul_gen.h:161),
 * written into buf.  family: "matmul", "flash_attention", "softmax",
 * "layernorm", "bias_gelu", "reduction"; cfg points at that family's config. */
int ks_kernel_symbol(const char *family, const void *cfg, char *buf, size_t len);

#ifdef __cplusplus
}
#endif

#endif /* KERNSCOPE_B200_H */
