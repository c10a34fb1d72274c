// dn8_kernels.h -- internal launch interface between the C ABI (abi.cu) and the kernels.
#pragma once
#include <cstddef>
#include <cuda.h>
#include <cuda_runtime.h>
#include "../../include/dn8.h"

namespace dn8 {

// Launch, with programmatic stream serialization when `pdl` (see griddep_* in dn8_common.cuh):
// only for a kernel whose predecessor in the stream is one of these kernels of the same pass (an
// event wait or a copy in between would otherwise not be waited for).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// As launch_pdl, as clusters of `csize` CTAs along x (grid.x a multiple of csize).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(bool pdl, int csize, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(csize);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// As launch_pdl, as clusters of two CTAs (grid.x even).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_pairs(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args&&... args) {
    return launch_pdl_cluster(pdl, 2, kernel, grid, block, smem, st, static_cast<Args&&>(args)...);
}

__attribute__((visibility("hidden"))) void set_last_error(const char* msg);  // thread-local message (abi.cu)

cudaError_t launch_conv1(const dn8_conv1_args& a, int sms, cudaStream_t st, bool pdl = false);
void arm_wait_fault(int fault, long long wait_limit);   // test hook of the next conv1 launch
bool conv1_supported(int G);   // the layer's weights fit (resident) on single CTAs or CTA pairs
cudaError_t launch_trans(const dn8_trans_args& a, int sms, cudaStream_t st, bool pdl = false);
int trans_chunk(int cout);
cudaError_t launch_stem(const dn8_stem_args& a, int sms, cudaStream_t st);
cudaError_t launch_head(const dn8_head_args& a, cudaStream_t st, bool pdl = false);
cudaError_t launch_zoom(const dn8_zoom_args& a, int sms, cudaStream_t st);
constexpr int DN8_MAX_DEVICES = 64;
cudaError_t head_scratch_tickets(int32_t** out);

struct Conv2Plan {
    CUtensorMap map;      // bottleneck planes, built once per geometry and buffer
    int Rt;               // image rows per tile
    uint32_t stage_bytes;
    size_t smem;
};
size_t conv2_smem_bytes(int H, int W);
cudaError_t prepare_conv2(Conv2Plan* plan, const dn8_conv2_args& a);
cudaError_t launch_conv2(const Conv2Plan& plan, const dn8_conv2_args& a, int sms, cudaStream_t st, bool pdl = false);

}  // namespace dn8
