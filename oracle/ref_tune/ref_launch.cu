// Test infrastructure: a launcher around one kernel emitted by the reference
// generator. Compiled once per generated source (nvcc -include <source>
// -DKS_REF_SYMBOL=<symbol>), so that each shared library holds one config.
#include <cuda_runtime.h>

extern "C" int ks_ref_launch(void **args, int grid_x, int grid_y, int block_x, int block_y, void *stream) {
  const cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void *>(&KS_REF_SYMBOL), dim3(grid_x, grid_y),
                                         dim3(block_x, block_y), args, 0, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? 0 : -static_cast<int>(e);
}
