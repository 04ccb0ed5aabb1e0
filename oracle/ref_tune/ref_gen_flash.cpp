// Test infrastructure: the reference flash-attention generator behind ref_gen.h.
#include "kernscope/tune/flash_attention_gen.h"
#include "ref_gen.h"

bool ref_gen_flash(const std::string &arch, const std::vector<std::int64_t> &shape, const RefCfg &cfg,
                   const std::string &out, RefGen *g, std::string *err) {
  namespace T = kernscope::tune;
  if (shape.size() != 3) {
    *err = "flash_attention shape is Nq,Nk,d";
    return false;
  }
  T::FlashAttentionConfig c;
  c.tile_m = ref_cfg_int(cfg, "tile_m", c.tile_m);
  c.tile_n = ref_cfg_int(cfg, "tile_n", c.tile_n);
  c.stages = ref_cfg_int(cfg, "stages", c.stages);
  c.vec_width = ref_cfg_int(cfg, "vec_width", c.vec_width);
  c.causal = ref_cfg_int(cfg, "causal", 0) != 0;
  c.smem_layout = ref_cfg_str(cfg, "smem_layout", "padding") == "xor" ? T::SmemLayout::kXorSwizzle
                                                                       : T::SmemLayout::kPadding;
  T::FlashAttentionProblem p;
  p.nq = shape[0];
  p.nk = shape[1];
  p.d = shape[2];
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
  g->smem_bytes = T::smem_bytes(c, p);
  g->symbol = T::kernel_symbol(c);
  return out.empty() || T::generate_to_file(c, p, out, err);
}
