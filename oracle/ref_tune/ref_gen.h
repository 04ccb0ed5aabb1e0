// Test infrastructure: emit one of the reference generator's kernels.
//
// Each family's generator is called through the reference's own API
// (tools/tune/include/kernscope/tune/*_gen.h: validate_config,
// launch_geometry, kernel_symbol, generate_to_file) from its own
// translation unit, because matmul_gen.h and flash_attention_gen.h both
// declare kernscope::tune::SmemLayout.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

struct RefGen {
  bool valid = false;
  std::string reason;   // the reference's reject reason when !valid
  std::string symbol;   // the exported kernel symbol
  int grid_x = 1, grid_y = 1, block_x = 1, block_y = 1;
  long long smem_bytes = 0;
};

using RefCfg = std::map<std::string, std::string>;

// shape: matmul {M,N,K}; flash_attention {Nq,Nk,d}; row families {rows,cols}.
// Writes the generated source to `out` when the config is valid and `out`
// is not empty. Returns false only for an unknown family or an IO error.
bool ref_gen_matmul(const std::string &arch, const std::vector<std::int64_t> &shape, const RefCfg &cfg,
                    const std::string &out, RefGen *g, std::string *err);
bool ref_gen_flash(const std::string &arch, const std::vector<std::int64_t> &shape, const RefCfg &cfg,
                   const std::string &out, RefGen *g, std::string *err);
bool ref_gen_elem(const std::string &family, const std::string &arch, const std::vector<std::int64_t> &shape,
                  const RefCfg &cfg, const std::string &out, RefGen *g, std::string *err);

inline int ref_cfg_int(const RefCfg &c, const char *k, int dflt) {
  auto it = c.find(k);
  return it == c.end() ? dflt : std::stoi(it->second);
}
inline std::string ref_cfg_str(const RefCfg &c, const char *k, const char *dflt) {
  auto it = c.find(k);
  return it == c.end() ? dflt : it->second;
}
