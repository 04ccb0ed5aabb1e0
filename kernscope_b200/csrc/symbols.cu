// symbols.cu -- stable per-config kernel symbols (the reference's
// kernel_symbol(), e.g. tools/tune/include/kernscope/tune/matmul_gen.h:158-161
// and flash_attention_gen.h:136-138), extended with the sm_100a fields.
#include <cstdio>
#include <cstring>

#include "ks_common.cuh"

namespace {
const char *mode_name(int m) {
  switch (m) {
    case KS_MODE_ONEPASS: return "onepass";
    case KS_MODE_TWOPASS: return "twopass";
    case KS_MODE_STRIDED: return "strided";
    case KS_MODE_TREE: return "tree";
    case KS_MODE_STAGED: return "staged";
    case KS_MODE_CLUSTER: return "cluster";
    default: return "unknown";
  }
}
}  // namespace

extern "C" int ks_kernel_symbol(const char *family, const void *cfg, char *buf, size_t len) {
  if (!family || !cfg || !buf || len == 0) return KS_ERR_INVALID_ARGS;
  int n = -1;
  if (!strcmp(family, "matmul")) {
    auto c = static_cast<const ks_matmul_config *>(cfg);
    // g<n>: raster groups of n M-tiles; nb<n>: bands of n N-tiles (group_m = -n);
    // _c1: a 256-row tile on one CTA (the CTA pair is tile_m 256's default)
    n = snprintf(buf, len, "kernscope_b200_matmul_m%d_n%d_k%d_s%d_a%d_%s%d%s", c->tile_m, c->tile_n, c->tile_k,
                 c->stages, c->acc_stages, c->group_m < 0 ? "nb" : "g", c->group_m < 0 ? -c->group_m : c->group_m,
                 c->tile_m == 256 && c->cta_group == 1 ? "_c1" : "");
  } else if (!strcmp(family, "flash_attention")) {
    auto c = static_cast<const ks_flash_attention_config *>(cfg);
    n = snprintf(buf, len, "kernscope_b200_flash_attention_br%d_bc%d_s%d%s", c->tile_m, c->tile_n, c->stages,
                 c->causal ? "_causal" : "");
  } else if (!strcmp(family, "softmax")) {
    auto c = static_cast<const ks_softmax_config *>(cfg);
    n = snprintf(buf, len, "kernscope_b200_softmax_b%d_v%d_%s", c->block, c->vec_width, mode_name(c->mode));
  } else if (!strcmp(family, "layernorm")) {
    auto c = static_cast<const ks_layernorm_config *>(cfg);
    n = snprintf(buf, len, "kernscope_b200_layernorm_b%d_v%d_%s", c->block, c->vec_width, mode_name(c->mode));
  } else if (!strcmp(family, "bias_gelu")) {
    auto c = static_cast<const ks_bias_gelu_config *>(cfg);
    n = snprintf(buf, len, "kernscope_b200_bias_gelu_b%d_v%d_%s", c->block, c->vec_width,
                 c->gelu == KS_GELU_TANH ? "tanh" : "erf");
  } else if (!strcmp(family, "reduction")) {
    auto c = static_cast<const ks_reduction_config *>(cfg);
    n = snprintf(buf, len, "kernscope_b200_reduction_b%d_v%d_%s", c->block, c->vec_width, mode_name(c->mode));
  } else {
    return KS_ERR_INVALID_ARGS;
  }
  return (n < 0 || size_t(n) >= len) ? KS_ERR_INVALID_ARGS : KS_OK;
}
