// partition.cu — the partition as two standalone launches (the multi-GPU path and the Backend API); the device
// functions are in partition.cuh, shared with the persistent tree kernel.
#include <cuda_runtime.h>

#include "partition.cuh"

namespace sb2 {

namespace {

__global__ void __launch_bounds__(kPartitionThreads) partition_flags_kernel(TrainArgs a) {
    __shared__ uint32_t red[kPartitionThreads / 32];
    // Zero the staging histogram (and its count slots) for this step's histogram.
    const uint32_t staging_len = 2 * a.total_bins + 2;
    for (uint32_t i = blockIdx.x * kPartitionThreads + threadIdx.x; i < staging_len; i += gridDim.x * kPartitionThreads)
        a.staging[i] = 0;
    const Step st = *a.step;
    if (!st.active || st.root) return;
    partition_flags_cta(a, st, blockIdx.x, gridDim.x, red);
}

__global__ void __launch_bounds__(kPartitionThreads) partition_scatter_kernel(TrainArgs a) {
    __shared__ uint32_t scan[2 * kPartitionThreads + 64];
    const Step st = *a.step;
    if (!st.active || st.root) return;
    const uint32_t total_left = partition_scatter_cta(a, st, blockIdx.x, gridDim.x, scan);
    if (blockIdx.x == 0 && threadIdx.x == 0) partition_publish(a, *a.step, total_left);
}

}  // namespace

void launch_partition_flags(const TrainArgs& a, int grid, cudaStream_t s) {
    partition_flags_kernel<<<grid, kPartitionThreads, 0, s>>>(a);
}

void launch_partition_scatter(const TrainArgs& a, int grid, cudaStream_t s) {
    partition_scatter_kernel<<<grid, kPartitionThreads, 0, s>>>(a);
}

}  // namespace sb2
