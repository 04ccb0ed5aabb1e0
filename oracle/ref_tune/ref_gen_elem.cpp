// Test infrastructure: the reference row-family generators behind ref_gen.h.
#include "kernscope/tune/bias_gelu_gen.h"
#include "kernscope/tune/layernorm_gen.h"
#include "kernscope/tune/reduction_gen.h"
#include "kernscope/tune/softmax_gen.h"
#include "ref_gen.h"

namespace {

namespace T = kernscope::tune;

T::ElemMode mode_of(const std::string &m, T::ElemMode dflt) {
  if (m == "onepass") return T::ElemMode::kOnePass;
  if (m == "twopass") return T::ElemMode::kTwoPass;
  if (m == "strided") return T::ElemMode::kStrided;
  if (m == "tree") return T::ElemMode::kTree;
  return dflt;
}

template <class Cfg>
bool emit(const Cfg &c, const T::ElemProblem &p, const std::string &out, RefGen *g, std::string *err) {
  const T::ConfigVerdict v = T::validate_config(c, p);
  g->valid = v.valid;
  g->reason = v.reason;
  if (!v.valid) return true;
  const T::LaunchGeometry lg = T::launch_geometry(c, p);
  g->grid_x = lg.grid_x;
  g->grid_y = lg.grid_y;
  g->block_x = lg.block_x;
  g->block_y = lg.block_y;
  g->symbol = T::kernel_symbol(c);
  return out.empty() || T::generate_to_file(c, p, out, err);
}

}  // namespace

bool ref_gen_elem(const std::string &family, const std::string &arch, const std::vector<std::int64_t> &shape,
                  const RefCfg &cfg, const std::string &out, RefGen *g, std::string *err) {
  if (shape.size() != 2) {
    *err = family + " shape is rows,cols";
    return false;
  }
  T::ElemProblem p;
  p.rows = shape[0];
  p.cols = shape[1];
  p.arch = arch;
  const int block = ref_cfg_int(cfg, "block", 256), vec = ref_cfg_int(cfg, "vec_width", 1);
  const std::string mode = ref_cfg_str(cfg, "mode", "");
  if (family == "softmax") {
    T::SoftmaxConfig c;
    c.block = block;
    c.vec_width = vec;
    c.mode = mode_of(mode, c.mode);
    return emit(c, p, out, g, err);
  }
  if (family == "layernorm") {
    T::LayerNormConfig c;
    c.block = block;
    c.vec_width = vec;
    c.mode = mode_of(mode, c.mode);
    return emit(c, p, out, g, err);
  }
  if (family == "bias_gelu") {
    T::BiasGeluConfig c;
    c.block = block;
    c.vec_width = vec;
    return emit(c, p, out, g, err);
  }
  if (family == "reduction") {
    T::ReductionConfig c;
    c.block = block;
    c.vec_width = vec;
    c.mode = mode_of(mode, c.mode);
    return emit(c, p, out, g, err);
  }
  *err = "unknown family " + family;
  return false;
}
