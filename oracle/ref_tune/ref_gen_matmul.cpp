// Test infrastructure: the reference matmul generator behind ref_gen.h.
#include "kernscope/tune/matmul_gen.h"
#include "ref_gen.h"

bool ref_gen_matmul(const std::string &arch, const std::vector<std::int64_t> &shape, const RefCfg &cfg,
                    const std::string &out, RefGen *g, std::string *err) {
  namespace T = kernscope::tune;
  if (shape.size() != 3) {
    *err = "matmul shape is M,N,K";
    return false;
  }
  T::MatmulConfig c;
  c.tile_m = ref_cfg_int(cfg, "tile_m", c.tile_m);
  c.tile_n = ref_cfg_int(cfg, "tile_n", c.tile_n);
  c.tile_k = ref_cfg_int(cfg, "tile_k", c.tile_k);
  c.warps = ref_cfg_int(cfg, "warps", c.warps);
  c.stages = ref_cfg_int(cfg, "stages", c.stages);
  c.vec_width = ref_cfg_int(cfg, "vec_width", c.vec_width);
  c.unroll = ref_cfg_int(cfg, "unroll", c.unroll);
  c.smem_layout = ref_cfg_str(cfg, "smem_layout", "padding") == "xor" ? T::SmemLayout::kXorSwizzle
                                                                       : T::SmemLayout::kPadding;
  T::MatmulProblem p;
  p.m = shape[0];
  p.n = shape[1];
  p.k = shape[2];
  p.arch = arch;
  const T::ConfigVerdict v = T::validate_config(c, p);
  g->valid = v.valid;
  g->reason = v.reason;
  if (!v.valid) return true;
  const T::LaunchGeometry lg = T::launch_geometry(c, p);
  g->grid_x = lg.grid_x;
  g->grid_y = lg.grid_y;
  g->block_x = lg.block_x;
  g->block_y = lg.block_y;
  g->smem_bytes = T::smem_bytes(c);
  g->symbol = T::kernel_symbol(c);
  return out.empty() || T::generate_to_file(c, p, out, err);
}
