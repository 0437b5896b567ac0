// st_chain.cu -- instantiations of the compact single-stream step kernel
// (st_chain.cuh) for the widths and storage types the runtime serves.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "st_chain.cuh"
#include "st_flow_host.h"

namespace st {

namespace {
template <typename T, bool kDiag>
const void* chain_by_width(int width) {
  switch (width) {
    case 256: return (const void*)k5_chain<T, 256, kDiag>;
    case 512: return (const void*)k5_chain<T, 512, kDiag>;
    case 1024: return (const void*)k5_chain<T, 1024, kDiag>;
    default: return nullptr;
  }
}
template <bool kDiag>
const void* chain_by_mode(int mode, int width) {
  if (mode == 1) return chain_by_width<__half, kDiag>(width);
  if (mode == 2) return chain_by_width<__nv_bfloat16, kDiag>(width);
  return chain_by_width<float, kDiag>(width);
}
}  // namespace

const void* chain_kernel(int mode, int width, bool diag) {
  return diag ? chain_by_mode<true>(mode, width) : chain_by_mode<false>(mode, width);
}

}  // namespace st
