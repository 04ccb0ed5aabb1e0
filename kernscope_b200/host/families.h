// families.h -- the six kernel families as the tuner sees them (the
// reference's generator API, tools/tune/include/kernscope/tune/*_gen.h):
// config structs and search spaces, validate_config, launch_geometry,
// kernel_symbol, smem_bytes, generate_source / generate_to_file, plus what
// the B200 pipeline adds: resource estimates for the occupancy pre-screen,
// seeded device sessions that launch a config through the C ABI, and the
// CPU reference the correctness gate compares against.
//
// On B200 a config selects a prebuilt template instantiation in
// libkernscope_b200.so (no per-variant compile); generate_source emits a
// self-contained C++ reproducer that calls the C ABI with that config.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "json.h"
#include "kernscope_b200.h"

namespace kernscope::tune {

using json = db::json::Value;

struct ConfigVerdict {
  bool valid = true;
  std::string reason;
};

struct LaunchGeometry {
  int grid_x = 1;
  int grid_y = 1;
  int block_x = 1;
  int block_y = 1;
  int smem_bytes = 0;
  int tmem_columns = 0;
};

// --- typed configs (field names follow the C ABI structs) ------------------
struct MatmulConfig {
  int tile_m = 128, tile_n = 256, tile_k = 64, stages = 4, acc_stages = 2, group_m = 8;
  int cta_group = 0;  // tile_m 256: 2 (or 0) a CTA pair, 1 one CTA with two M=128 MMAs
};
struct MatmulProblem {
  std::int64_t m = 0, n = 0, k = 0;
  std::string arch = "sm_100a";
  int dtype_bytes = 2;
};
struct FlashAttentionConfig {
  int tile_m = 256, tile_n = 128, stages = 2;
  bool causal = false;
};
struct FlashAttentionProblem {
  std::int64_t nq = 0, nk = 0, d = 0, batch_heads = 1;
  bool causal = false;
  std::string arch = "sm_100a";
  int dtype_bytes = 2;
};
enum class ElemMode : int { kOnePass = KS_MODE_ONEPASS, kTwoPass = KS_MODE_TWOPASS, kStrided = KS_MODE_STRIDED,
                            kTree = KS_MODE_TREE, kStaged = KS_MODE_STAGED, kCluster = KS_MODE_CLUSTER };
const char *elem_mode_name(ElemMode m) noexcept;
struct ElemProblem {
  std::int64_t rows = 0, cols = 0;
  std::string arch = "sm_100a";
  int dtype_bytes = 2;
  int axis = 0;  // reduction: 0 = column sums (bf16), -1 = full fp32 sum
};
struct SoftmaxConfig {
  int block = 256, vec_width = 8;
  ElemMode mode = ElemMode::kOnePass;
};
struct LayerNormConfig {
  int block = 128, vec_width = 8;
  ElemMode mode = ElemMode::kOnePass;
};
struct BiasGeluConfig {
  int block = 128, vec_width = 8;
  int gelu = KS_GELU_ERF;
};
struct ReductionConfig {
  int block = 256, vec_width = 8;
  ElemMode mode = ElemMode::kTree;
};

ConfigVerdict validate_config(const MatmulConfig &, const MatmulProblem &) noexcept;
ConfigVerdict validate_config(const FlashAttentionConfig &, const FlashAttentionProblem &) noexcept;
ConfigVerdict validate_config(const SoftmaxConfig &, const ElemProblem &) noexcept;
ConfigVerdict validate_config(const LayerNormConfig &, const ElemProblem &) noexcept;
ConfigVerdict validate_config(const BiasGeluConfig &, const ElemProblem &) noexcept;
ConfigVerdict validate_config(const ReductionConfig &, const ElemProblem &) noexcept;
std::int64_t smem_bytes(const MatmulConfig &) noexcept;
std::int64_t smem_bytes(const FlashAttentionConfig &, const FlashAttentionProblem &) noexcept;
LaunchGeometry launch_geometry(const MatmulConfig &, const MatmulProblem &) noexcept;
LaunchGeometry launch_geometry(const FlashAttentionConfig &, const FlashAttentionProblem &) noexcept;
std::string kernel_symbol(const MatmulConfig &);
std::string kernel_symbol(const FlashAttentionConfig &);
std::string kernel_symbol(const SoftmaxConfig &);
std::string kernel_symbol(const LayerNormConfig &);
std::string kernel_symbol(const BiasGeluConfig &);
std::string kernel_symbol(const ReductionConfig &);

// --- family-generic view used by the driver ---------------------------------
struct Resources {
  int regs_per_thread = 0;  // estimate (ptxas counts of the instantiations)
  int smem_bytes = 0;
  int block = 0;
  int tmem_columns = 0;
};

class Session;  // device buffers + launches for one shape

class Family {
 public:
  virtual ~Family() = default;
  virtual const char *name() const = 0;
  // Parse / check a CLI shape ("M,N,K" ...); fills *reason when invalid.
  virtual bool check_shape(const std::vector<std::int64_t> &shape, std::string *reason) const = 0;
  // Search space: "auto" (bounded grid) or "full".
  virtual std::vector<json> enumerate(bool full, const std::vector<std::int64_t> &shape) const = 0;
  virtual ConfigVerdict validate(const json &cfg, const std::vector<std::int64_t> &shape,
                                 const std::string &arch) const = 0;
  virtual Resources resources(const json &cfg, const std::vector<std::int64_t> &shape) const = 0;
  virtual LaunchGeometry geometry(const json &cfg, const std::vector<std::int64_t> &shape) const = 0;
  virtual std::string symbol(const json &cfg) const = 0;
  // Default correctness-gate shape for a tune shape.
  virtual std::vector<std::int64_t> gate_shape(const std::vector<std::int64_t> &shape) const = 0;
  // Roofline FLOPs / algorithmic bytes of one launch at `shape`.
  virtual std::int64_t flops(const std::vector<std::int64_t> &shape, const json &cfg) const = 0;
  virtual std::int64_t bytes(const std::vector<std::int64_t> &shape) const = 0;
  // Seeded device inputs (the reference profile's distributions).
  virtual std::unique_ptr<Session> make_session(const std::vector<std::int64_t> &shape, std::uint64_t seed,
                                                std::string *error) const = 0;
  // A C++ reproducer that launches `cfg` at `shape` through the C ABI.
  virtual std::string generate_source(const json &cfg, const std::vector<std::int64_t> &shape) const = 0;
};

const Family *find_family(const std::string &name);
const std::vector<std::string> &family_names();
// Canonical config string (sorted keys) used as the tunecache config key.
std::string canonical_config(const json &cfg);

// Device-side state for one shape.  launch() runs one config on the
// session's stream; output() copies the result back as fp32; reference()
// is the CPU result of the same inputs (fp32, rounded like the reference
// goldens); verdict() compares them.
struct GateVerdict {
  bool pass = false;
  double cosine = 0.0, max_rel_err = 0.0, pcc = 0.0;   // reference verdict metrics
  double floor_rel_err = 0.0, norm_rel_err = 0.0;      // benchmark tolerance metrics
  std::string criterion;
};

class Session {
 public:
  virtual ~Session() = default;
  virtual int launch(const json &cfg, void *stream) = 0;
  virtual int output(std::vector<float> *out) = 0;
  virtual void reference(std::vector<float> *out) const = 0;
  virtual GateVerdict verdict(const std::vector<float> &got, const std::vector<float> &ref) const;
  // test hook: overwrite the device output with zeros (a wrong result)
  virtual int corrupt_output(void *stream) = 0;
};

// The reference verdict (tests/golden/kernscope_golden/metrics.py:92-116):
// bf16 outputs pass on cosine >= 0.999, max_rel_err (eps 1e-6) <= 1e-2 and
// pcc >= 0.99; the floor-guarded and norm-wise errors ride along as
// diagnostics.
GateVerdict bf16_verdict(const std::vector<float> &got, const std::vector<float> &ref);

// The host half of a gate session, for tests and tools: the reference
// profile's inputs of `family` (a find_family key) at `shape` and `seed`,
// by the reference's names (inputs.py), as bf16 bits -- with any of them
// replaced by `inputs` -- and the CPU reference output of those inputs
// (fp32 holding bf16 values).  False (and *error) on a bad family, shape or
// input size.
bool golden_case(const std::string &family, const std::vector<std::int64_t> &shape, std::uint64_t seed,
                 const std::map<std::string, std::vector<std::uint16_t>> &inputs,
                 std::map<std::string, std::vector<std::uint16_t>> *used, std::vector<float> *expected,
                 std::string *error);

// bf16 helpers shared by the sessions and references.
std::uint16_t f32_to_bf16(float f);
float bf16_to_f32(std::uint16_t h);

}  // namespace kernscope::tune
