// flash_attention.cu -- causal / non-causal attention forward for sm_100a.
#include "ks_common.cuh"

extern "C" {

int ks_flash_attention_validate(const ks_flash_attention_config *cfg, const ks_flash_attention_args *a,
                                char *reason, size_t len) {
  if (!cfg || !a) return KS_ERR_INVALID_ARGS;
  ks::set_reason(reason, len, "flash_attention: not built yet");
  return KS_ERR_UNSUPPORTED;
}

int ks_flash_attention_launch(const ks_flash_attention_config *cfg, const ks_flash_attention_args *a,
                              void *stream) {
  (void)stream;
  if (!cfg || !a) return KS_ERR_INVALID_ARGS;
  return KS_ERR_UNSUPPORTED;
}

}  // extern "C"
