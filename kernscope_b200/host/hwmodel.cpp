// hwmodel.cpp -- arch DB, occupancy and roofline for sm_100a.
#include "hwmodel.h"

#include <dlfcn.h>

#include <algorithm>
#include <cstdlib>
#include <filesystem>
#include <fstream>
#include <sstream>
#include <stdexcept>

#include "json.h"

namespace kernscope {

namespace {
// B200: 148 SMs (2 dies x 74), 228 KB shared memory per SM (227 KB per CTA),
// 64K registers, 2048 threads / 64 warps / 32 CTAs per SM, TMEM 512 columns
// x 128 lanes x 32 bit per SM, L2 126 MB, max SM clock 1965 MHz; datasheet
// HBM3e 8 TB/s and dense bf16 2.25 PFLOP/s (projected values only).
constexpr ArchInfo kSm100a{
    .name = "sm_100a", .vendor = Vendor::kNvidia, .warp_size = 32, .max_threads_per_sm = 2048,
    .max_blocks_per_sm = 32, .smem_per_sm_bytes = 228 * 1024, .smem_per_block_max_bytes = 227 * 1024,
    .regs_per_sm = 65536, .max_regs_per_thread = 255, .reg_granule = 8, .max_warps_per_sm = 64,
    .sm_count = 148, .tmem_columns_per_sm = 512, .l2_bytes = 126LL * 1024 * 1024, .max_sm_clock_mhz = 1965.0,
    .nominal_hbm_gbs = 8000.0, .nominal_bf16_dense_tflops = 2250.0,
};
constexpr ArchInfo kSm100 = [] {
  ArchInfo a = kSm100a;
  a.name = "sm_100";
  return a;
}();
}  // namespace

const ArchInfo &get_arch(std::string_view name) {
  if (name == kSm100a.name) return kSm100a;
  if (name == kSm100.name) return kSm100;
  throw std::out_of_range("kernscope: unknown arch '" + std::string(name) + "'");
}

bool has_arch(std::string_view name) noexcept { return name == "sm_100a" || name == "sm_100"; }

namespace occupancy {

const char *limiter_name(Limiter l) noexcept {
  switch (l) {
    case Limiter::kRegisters: return "registers";
    case Limiter::kSharedMemory: return "shared";  // the reference's contract string (libs/occupancy/src/occupancy.cpp:50-62)
    case Limiter::kThreads: return "threads";
    case Limiter::kBlocks: return "blocks";
    case Limiter::kTmem: return "tmem";
  }
  return "unknown";
}

OccupancyResult compute_occupancy(const ArchInfo &a, int regs, int smem, int block, int tmem_cols) noexcept {
  OccupancyResult r;
  r.max_warps_per_sm = a.max_warps_per_sm;
  if (block <= 0 || block > 1024 || regs > a.max_regs_per_thread || smem > a.smem_per_block_max_bytes ||
      tmem_cols > a.tmem_columns_per_sm) {
    r.limiter = block <= 0 || block > 1024 ? Limiter::kThreads
                : regs > a.max_regs_per_thread ? Limiter::kRegisters
                : smem > a.smem_per_block_max_bytes ? Limiter::kSharedMemory
                                                    : Limiter::kTmem;
    return r;
  }
  const int warps = (block + a.warp_size - 1) / a.warp_size;
  struct Cand {
    int blocks;
    Limiter lim;
  };
  Cand c[5];
  int n = 0;
  // Candidates in tie-break order: on equal counts the earlier one is named
  // (registers > shared > threads > blocks, the reference's priority in
  // libs/occupancy/src/occupancy.cpp:69-93; TMEM, which it does not model,
  // last). Zero shared memory or TMEM is "not requested" and never limits.
  const int regs_rounded = ((std::max(regs, 1) + a.reg_granule - 1) / a.reg_granule) * a.reg_granule;
  c[n++] = {a.regs_per_sm / (regs_rounded * a.warp_size * warps), Limiter::kRegisters};
  if (smem > 0) c[n++] = {a.smem_per_sm_bytes / smem, Limiter::kSharedMemory};
  c[n++] = {a.max_threads_per_sm / (warps * a.warp_size), Limiter::kThreads};
  c[n++] = {a.max_blocks_per_sm, Limiter::kBlocks};
  if (tmem_cols > 0) c[n++] = {a.tmem_columns_per_sm / tmem_cols, Limiter::kTmem};
  Cand best = c[0];
  for (int i = 1; i < n; ++i)
    if (c[i].blocks < best.blocks) best = c[i];
  r.blocks_per_sm = std::max(0, best.blocks);
  r.limiter = best.lim;
  r.warps_resident = r.blocks_per_sm * warps;
  r.occupancy = double(r.warps_resident) / double(a.max_warps_per_sm);
  return r;
}

}  // namespace occupancy

namespace roofline {

const char *kernel_family_name(KernelFamily f) noexcept {
  switch (f) {
    case KernelFamily::kGemm: return "gemm";
    case KernelFamily::kFusedBiasGelu: return "bias_gelu";
    case KernelFamily::kSoftmax: return "softmax";
    case KernelFamily::kLayerNorm: return "layernorm";
    case KernelFamily::kReduction: return "reduction";
    case KernelFamily::kFlashAttention: return "flash_attention";
  }
  return "unknown";
}

bool family_from_name(std::string_view s, KernelFamily *out) noexcept {
  if (s == "gemm" || s == "matmul") *out = KernelFamily::kGemm;
  else if (s == "bias_gelu") *out = KernelFamily::kFusedBiasGelu;
  else if (s == "softmax") *out = KernelFamily::kSoftmax;
  else if (s == "layernorm") *out = KernelFamily::kLayerNorm;
  else if (s == "reduction") *out = KernelFamily::kReduction;
  else if (s == "flash_attention" || s == "attention") *out = KernelFamily::kFlashAttention;
  else return false;
  return true;
}

std::int64_t compute_flops(KernelFamily f, const Shape &s) noexcept {
  switch (f) {
    case KernelFamily::kGemm: return 2 * s.m * s.n * s.k;
    case KernelFamily::kFusedBiasGelu: return kGeluFlopsPerElement * s.n;
    case KernelFamily::kSoftmax: return kSoftmaxFlopsPerElement * s.n;
    case KernelFamily::kLayerNorm: return kLayerNormFlopsPerElement * s.n;
    case KernelFamily::kReduction: return kReductionFlopsPerElement * s.n;
    case KernelFamily::kFlashAttention: {
      const std::int64_t bh = std::max<std::int64_t>(s.m, 1);
      // S = Q K^T and O = P V, 2 N_keys d each per query row; causal rows see
      // i+1 keys: sum = N(N+1)/2
      const std::int64_t pairs = s.causal ? s.n * (s.n + 1) / 2 : s.n * s.n;
      return 4 * s.d * bh * pairs;
    }
  }
  return 0;
}

std::int64_t compute_bytes_moved(KernelFamily f, const Shape &s) noexcept {
  const std::int64_t b = s.dtype_bytes;
  switch (f) {
    case KernelFamily::kGemm: return (s.m * s.k + s.k * s.n + s.m * s.n) * b;
    case KernelFamily::kFusedBiasGelu: return 2 * s.n * b + s.k * b;
    case KernelFamily::kSoftmax: return 2 * s.n * b;
    case KernelFamily::kLayerNorm: return 2 * s.n * b + 2 * s.k * b;
    case KernelFamily::kReduction: return s.n * b + std::max<std::int64_t>(s.m, 1) * b;
    case KernelFamily::kFlashAttention: return 4 * std::max<std::int64_t>(s.m, 1) * s.n * s.d * b;
  }
  return 0;
}

std::int64_t reference_model_bytes(KernelFamily f, const Shape &s) noexcept {
  const std::int64_t b = s.dtype_bytes;
  // The reference's element model (libs/roofline/src/roofline.cpp:66-82):
  // parameter vectors and the reduction's output are not counted.
  switch (f) {
    case KernelFamily::kGemm: return compute_bytes_moved(f, s);
    case KernelFamily::kFusedBiasGelu: return 3 * s.n * b;  // x, bias (per element), y
    case KernelFamily::kSoftmax:
    case KernelFamily::kLayerNorm: return 2 * s.n * b;
    case KernelFamily::kReduction: return s.n * b;
    case KernelFamily::kFlashAttention:                     // standard attention: s(4Nd + 4N^2)
      return std::max<std::int64_t>(s.m, 1) * b * (4 * s.n * s.d + 4 * s.n * s.n);
  }
  return 0;
}

double arithmetic_intensity(KernelFamily f, const Shape &s) noexcept {
  const std::int64_t by = compute_bytes_moved(f, s);
  return by > 0 ? double(compute_flops(f, s)) / double(by) : 0.0;
}

const char *bound_class_name(BoundClass b) noexcept {
  switch (b) {
    case BoundClass::kCompute: return "compute";
    case BoundClass::kMemory: return "memory";
    case BoundClass::kLatency: return "latency";
  }
  return "unknown";
}

namespace {
std::string peaks_path() {
  if (const char *e = std::getenv("KS_MEASURED_PEAKS")) return e;
  // <repo>/kernscope_b200/lib/libkernscope_tune.so -> <repo>/MEASURED_PEAKS.json
  Dl_info info{};
  if (dladdr(reinterpret_cast<void *>(&peaks_path), &info) && info.dli_fname) {
    std::filesystem::path p(info.dli_fname);
    return (p.parent_path().parent_path().parent_path() / "MEASURED_PEAKS.json").string();
  }
  return "MEASURED_PEAKS.json";
}
}  // namespace

ErrorCode machine_peak(std::string_view arch, MachinePeak *out, std::string *err) {
  if (!has_arch(arch)) {
    if (err) *err = "unknown arch '" + std::string(arch) + "'";
    return ErrorCode::kUnknownArch;
  }
  const ArchInfo &a = get_arch(arch);
  MachinePeak p;
  p.arch = std::string(arch);
  p.gpu = "NVIDIA B200";
  p.matrix_dtype = "bf16";
  p.matrix_peak_flops = a.nominal_bf16_dense_tflops * 1e12;
  p.matrix_peak_sustained_flops = p.matrix_peak_flops;
  p.bandwidth_bytes_per_s = a.nominal_hbm_gbs * 1e9;
  p.projected = true;
  p.provenance = "datasheet (projected): 2.25 PFLOP/s dense bf16, 8 TB/s HBM3e";
  std::ifstream fh(peaks_path());
  if (fh) {
    std::stringstream ss;
    ss << fh.rdbuf();
    db::json::Value v;
    if (db::json::Value::parse(ss.str(), &v, nullptr) && v.find("hbm_gbs") && v.find("bf16_tflops")) {
      p.bandwidth_bytes_per_s = v.number_or("hbm_gbs", 0.0) * 1e9;
      p.matrix_peak_flops = v.number_or("bf16_tflops", 0.0) * 1e12;
      p.matrix_peak_sustained_flops = v.number_or("bf16_tflops_sustained", v.number_or("bf16_tflops", 0.0)) * 1e12;
      p.projected = false;
      p.provenance = "measured: " + v.string_or("how", "MEASURED_PEAKS.json") + " (" + v.string_or("when", "") + ")";
    }
  }
  *out = p;
  return ErrorCode::kNone;
}

ErrorCode roofline_position(KernelFamily f, const Shape &s, std::int64_t bytes, std::int64_t flops,
                            std::string_view arch, RooflinePosition *out, std::string *err, PeakKind kind) {
  if (bytes <= 0 || flops <= 0) {
    if (err) *err = "bytes_moved and flops must be positive";
    return ErrorCode::kInvalidInput;
  }
  MachinePeak p;
  ErrorCode ec = machine_peak(arch, &p, err);
  if (ec != ErrorCode::kNone) return ec;
  (void)f;
  (void)s;
  RooflinePosition r;
  const double peak = kind == PeakKind::kMatrixSustained ? p.matrix_peak_sustained_flops : p.matrix_peak_flops;
  r.arithmetic_intensity = double(flops) / double(bytes);
  r.ridge_point = peak / p.bandwidth_bytes_per_s;
  r.compute_bound_ceiling = peak;
  r.memory_bound_ceiling = r.arithmetic_intensity * p.bandwidth_bytes_per_s;
  r.attained_flops = std::min(r.compute_bound_ceiling, r.memory_bound_ceiling);
  // Little's law: a transfer that would finish within a few DRAM latencies at
  // full bandwidth cannot fill the memory pipeline -> latency bound.
  const double latency_bytes = p.bandwidth_bytes_per_s * kDramLatencyNs * 1e-9 * 4.0;
  if (double(bytes) < latency_bytes && r.arithmetic_intensity < r.ridge_point)
    r.bound_class = BoundClass::kLatency;
  else
    r.bound_class = r.arithmetic_intensity >= r.ridge_point ? BoundClass::kCompute : BoundClass::kMemory;
  *out = r;
  return p.projected ? ErrorCode::kProjectedPeaks : ErrorCode::kNone;
}

}  // namespace roofline
}  // namespace kernscope
