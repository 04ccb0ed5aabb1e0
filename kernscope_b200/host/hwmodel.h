// hwmodel.h -- the tuner's GPU-free hardware model for B200:
//
//   kernscope::ArchInfo / get_arch / has_arch   (libs/arch, arch.h:33-235)
//   kernscope::occupancy::compute_occupancy     (libs/occupancy, occupancy.h:85-96)
//   kernscope::roofline::{compute_flops, compute_bytes_moved, machine_peak,
//                         roofline_position}   (libs/roofline, roofline.h:74-235)
//
// The reference's sm_100 row has no SM count, TMEM or peaks
// (arch.h:143-155); the sm_100a row here carries them.  Occupancy adds the
// TMEM limiter (512 columns per SM shared by resident CTAs).  The roofline
// counts ALGORITHMIC bytes (each tensor read or written once) and the causal
// attention FLOPs; the reference's own byte model is kept beside it
// (reference_model_bytes) for comparison.  Peaks come from the measured
// MEASURED_PEAKS.json of the GPU pool when it is found, else the datasheet
// values flagged projected.
#pragma once

#include <cstdint>
#include <string>
#include <string_view>

namespace kernscope {

enum class Vendor : std::uint8_t { kNvidia, kAmd };

struct ArchInfo {
  std::string_view name;
  Vendor vendor;
  int warp_size;
  int max_threads_per_sm;
  int max_blocks_per_sm;
  int smem_per_sm_bytes;
  int smem_per_block_max_bytes;
  int regs_per_sm;
  int max_regs_per_thread;
  int reg_granule;  // per-thread allocation granule (x 32 threads per warp)
  int max_warps_per_sm;
  // sm_100a additions
  int sm_count;
  int tmem_columns_per_sm;   // 512 x 128 lanes x 32 bit = 256 KB
  std::int64_t l2_bytes;
  double max_sm_clock_mhz;
  double nominal_hbm_gbs;          // datasheet (projected) HBM bandwidth
  double nominal_bf16_dense_tflops;  // datasheet dense bf16 tensor peak
};

const ArchInfo &get_arch(std::string_view name);  // throws std::out_of_range
bool has_arch(std::string_view name) noexcept;

namespace occupancy {

enum class Limiter : std::uint8_t { kRegisters, kSharedMemory, kThreads, kBlocks, kTmem };
const char *limiter_name(Limiter l) noexcept;

struct OccupancyResult {
  int blocks_per_sm = 0;
  int warps_resident = 0;
  int max_warps_per_sm = 0;
  double occupancy = 0.0;  // warps_resident / max_warps_per_sm
  Limiter limiter = Limiter::kThreads;
};

// Min-wins resident CTAs per SM for (registers/thread, shared bytes/CTA,
// threads/CTA, TMEM columns/CTA; 0 = none).  blocks_per_sm 0 = cannot run.
OccupancyResult compute_occupancy(const ArchInfo &arch, int regs_per_thread, int smem_bytes_per_block,
                                  int block_size, int tmem_columns = 0) noexcept;

}  // namespace occupancy

namespace roofline {

enum class KernelFamily : std::uint8_t { kGemm, kFusedBiasGelu, kSoftmax, kLayerNorm, kReduction, kFlashAttention };
const char *kernel_family_name(KernelFamily family) noexcept;
bool family_from_name(std::string_view name, KernelFamily *out) noexcept;

// Problem shape.  kGemm: m, n, k.  Row ops: n = elements, k = row length
// (cols; parameter vectors gamma/beta/bias).  kReduction: n = elements,
// m = outputs.  kFlashAttention: n = sequence length, d = head dim,
// m = batch*heads, causal.
struct Shape {
  std::int64_t m = 0;
  std::int64_t n = 0;
  std::int64_t k = 0;
  std::int64_t d = 0;
  int dtype_bytes = 2;
  bool causal = false;
};

inline constexpr std::int64_t kGeluFlopsPerElement = 14;
inline constexpr std::int64_t kSoftmaxFlopsPerElement = 5;
inline constexpr std::int64_t kLayerNormFlopsPerElement = 11;
inline constexpr std::int64_t kReductionFlopsPerElement = 1;
inline constexpr double kDramLatencyNs = 600.0;

std::int64_t compute_flops(KernelFamily family, const Shape &shape) noexcept;
// Algorithmic bytes: every operand read once, every output written once.
std::int64_t compute_bytes_moved(KernelFamily family, const Shape &shape) noexcept;
// The reference's per-family byte model (roofline.cpp:42-100) for comparison.
std::int64_t reference_model_bytes(KernelFamily family, const Shape &shape) noexcept;
double arithmetic_intensity(KernelFamily family, const Shape &shape) noexcept;

enum class ErrorCode : std::uint8_t { kNone = 0, kUnknownArch, kProjectedPeaks, kNoPeaksTabulated,
                                      kNoPeakForDtype, kInvalidInput };

struct MachinePeak {
  std::string arch;
  std::string gpu;
  std::string matrix_dtype;          // "bf16"
  double matrix_peak_flops = 0.0;    // FLOP/s (burst)
  double matrix_peak_sustained_flops = 0.0;
  double bandwidth_bytes_per_s = 0.0;
  bool projected = false;            // datasheet values, not measured
  std::string provenance;
};

// Reads MEASURED_PEAKS.json from $KS_MEASURED_PEAKS, else the repository
// root next to the library; falls back to the datasheet (projected).
ErrorCode machine_peak(std::string_view arch, MachinePeak *out, std::string *error_message = nullptr);

enum class PeakKind : std::uint8_t { kMatrix, kMatrixSustained };
enum class BoundClass : std::uint8_t { kCompute, kMemory, kLatency };
const char *bound_class_name(BoundClass b) noexcept;

struct RooflinePosition {
  double arithmetic_intensity = 0.0;
  double ridge_point = 0.0;
  double compute_bound_ceiling = 0.0;  // FLOP/s
  double memory_bound_ceiling = 0.0;   // FLOP/s at this intensity
  double attained_flops = 0.0;         // min of the two ceilings
  BoundClass bound_class = BoundClass::kMemory;
};

ErrorCode roofline_position(KernelFamily family, const Shape &shape, std::int64_t bytes_moved,
                            std::int64_t flops, std::string_view arch, RooflinePosition *out,
                            std::string *error_message = nullptr, PeakKind peak_kind = PeakKind::kMatrix);

}  // namespace roofline
}  // namespace kernscope
