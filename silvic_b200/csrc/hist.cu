// hist.cu — the histogram as two standalone launches (see hist.cuh); the device functions are in hist_device.cuh,
// shared with the persistent tree kernel.
#include <cuda_runtime.h>

#include "hist_device.cuh"

namespace sb2 {

namespace {

__global__ void __launch_bounds__(kHistThreads) histogram_kernel(HistArgs a) {
    extern __shared__ __align__(16) int sh[];
    const HistJob job = *a.job;
    histogram_cta(a, job, blockIdx.x, sh);
}

__global__ void __launch_bounds__(256) histogram_reduce_kernel(HistArgs a) {
    const HistJob job = *a.job;
    histogram_reduce_slot(a, job, blockIdx.x * 256 + threadIdx.x);
}

}  // namespace

int histogram_threads() { return kHistThreads; }

void launch_histogram(const HistArgs& a, int grid, int smem_bytes, cudaStream_t stream) {
    histogram_kernel<<<grid, kHistThreads, smem_bytes, stream>>>(a);
}

void launch_histogram_reduce(const HistArgs& a, uint32_t total_slots, cudaStream_t stream) {
    histogram_reduce_kernel<<<static_cast<unsigned>(ceil_div(total_slots, 256)), 256, 0, stream>>>(a);
}

cudaError_t histogram_configure(int smem_bytes) {
    return cudaFuncSetAttribute(histogram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
}

cudaError_t histogram_occupancy(int smem_bytes, int* blocks_per_sm) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, histogram_kernel, kHistThreads, smem_bytes);
}

}  // namespace sb2
