// hist.cu — the histogram as two standalone launches (see hist.cuh); the device functions are in hist_device.cuh,
// shared with the persistent tree kernel.
#include <cuda_runtime.h>

#include "hist_device.cuh"

namespace sb2 {

namespace {

__global__ void __launch_bounds__(kHistThreads) histogram_kernel(HistArgs a) {
    extern __shared__ __align__(16) int sh[];
    __shared__ HistCta c;
    const HistJob job = *a.job;
    const uint32_t round_rows = packed_round_rows(*a.spec);
    if (histogram_goes_direct(job.count, round_rows)) {
        histogram_direct_cta(a, job, blockIdx.x, gridDim.x);
        return;
    }
    histogram_prepare_cta(a, blockIdx.x, sh, &c);
    histogram_cta(a, job, blockIdx.x, sh, c, round_rows);
}

__global__ void __launch_bounds__(256) histogram_reduce_kernel(HistArgs a) {
    const HistJob job = *a.job;
    if (histogram_goes_direct(job.count, packed_round_rows(*a.spec))) return;  // already in the output
    histogram_reduce_quads(a, job, blockIdx.x * 256 + threadIdx.x, gridDim.x * 256);
}

}  // namespace

int histogram_threads() { return kHistThreads; }

void launch_histogram(const HistArgs& a, int grid, int smem_bytes, cudaStream_t stream) {
    histogram_kernel<<<grid, kHistThreads, smem_bytes, stream>>>(a);
}

void launch_histogram_reduce(const HistArgs& a, cudaStream_t stream) {
    const uint64_t threads = static_cast<uint64_t>(a.num_quads) * a.quad_split;
    histogram_reduce_kernel<<<static_cast<unsigned>(ceil_div(threads, 256)), 256, 0, stream>>>(a);
}

cudaError_t histogram_configure(int smem_bytes) {
    return cudaFuncSetAttribute(histogram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
}

cudaError_t histogram_occupancy(int smem_bytes, int* blocks_per_sm) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, histogram_kernel, kHistThreads, smem_bytes);
}

}  // namespace sb2
