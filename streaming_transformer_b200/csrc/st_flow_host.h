// st_flow_host.h -- what st_runtime.cu needs of st_flow.cu (the single-stream
// flow kernel lives in its own translation unit).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace st {

struct StepArgs;
struct FlowLaunch;

// k4_flow<T, width, diag> for mode 0 fp32, 1 fp16, 2 bf16; null for other
// widths; diag: the variant that records per-phase cycle sums.
const void* flow_kernel(int mode, int width, bool diag);
// Dynamic shared memory and threads per CTA of k4_flow.
size_t flow_smem_bytes();
int flow_threads();
// True when the flow kernel serves this model on a grid of `clusters`
// clusters of `cluster` CTAs (shapes, ffn slice, chunk tables).
bool flow_shape_ok(const StepArgs& a, size_t elem, int cluster, int clusters);
// One cluster launch of the flow kernel.
cudaError_t flow_launch(const void* fn, int grid, int cluster, cudaStream_t stream, const StepArgs& a,
                        const FlowLaunch& f);

}  // namespace st
