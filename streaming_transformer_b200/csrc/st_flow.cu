// st_flow.cu -- instantiations of the single-stream flow kernel (st_flow.cuh)
// and the host helpers st_runtime.cu uses to pick and size it.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "st_flow.cuh"
#include "st_flow_host.h"

namespace st {

namespace {
template <typename T, bool kDiag>
const void* by_width(int width) {
  switch (width) {
    case 256: return (const void*)k4_flow<T, 256, kDiag>;
    case 512: return (const void*)k4_flow<T, 512, kDiag>;
    case 1024: return (const void*)k4_flow<T, 1024, kDiag>;
    default: return nullptr;
  }
}
template <bool kDiag>
const void* by_mode(int mode, int width) {
  if (mode == 1) return by_width<__half, kDiag>(width);
  if (mode == 2) return by_width<__nv_bfloat16, kDiag>(width);
  return by_width<float, kDiag>(width);
}
}  // namespace

const void* flow_kernel(int mode, int width, bool diag) {
  return diag ? by_mode<true>(mode, width) : by_mode<false>(mode, width);
}

size_t flow_smem_bytes() { return kFlowSmemBytes; }

int flow_threads() { return kFlowThreads; }

bool flow_shape_ok(const StepArgs& a, size_t elem, int cluster, int clusters) {
  if (a.streams != 1 || a.head_dim != kFlowHd || a.features != kFlowFeatures) return false;
  if (a.width != 256 && a.width != 512 && a.width != 1024) return false;
  if (cluster < 2 || cluster > kFlowMaxCluster || a.width % (2 * cluster) != 0) return false;
  const int grid = cluster * clusters, ffn = a.ffn / a.tp_size;
  if ((ffn + grid - 1) / grid > kFlowMaxAct || ffn < grid) return false;
  for (int id = 0; id < clusters; ++id)
    for (int rank = 0; rank < cluster; ++rank)
      if (flow_chunks_per_step(a, Where{rank, cluster, id, clusters}, elem) > kFlowMaxChunks) return false;
  return true;
}

cudaError_t flow_launch(const void* fn, int grid, int cluster, cudaStream_t stream, const StepArgs& a0,
                        const FlowLaunch& f0) {
  StepArgs a = a0;
  FlowLaunch f = f0;
  void* params[] = {&a, &f};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFlowThreads);
  cfg.dynamicSmemBytes = kFlowSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = cluster;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, params);
}

}  // namespace st
