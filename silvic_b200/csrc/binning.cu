// binning.cu — a dense matrix's values binned into the dataset's row-major feature groups on the device
// (data::binning::bin_rows, crates/silvic-core/src/data/binning.rs:71-135, with BinMapper::value_to_bin,
// data/bin_mapper.rs:343-360).
//
// Per group, one CTA takes 128 rows: the group's upper bounds sit in shared memory (a group holds at most 8192
// bins, data/mod.rs:22, so its bounds fit), every thread bins values of the tile and writes the bytes into the
// group's rows. Row-major input: consecutive threads take consecutive features of a row (the row's values of the
// group are contiguous when its features are); column-major: consecutive rows of a feature. A value's bin is the
// number of upper bounds below it (`partition_point(bound < value)`; the last bound is +inf), NaN goes to the NaN
// bin, or to zero's bin when the feature has none. The byte-wide binary search over the feature's bounds is the
// same count as the reference's branch-free search over bounds padded to 256 with +inf (binning.rs:51-61).
#include <cuda_runtime.h>

#include <cstdint>

#include "binning.cuh"

namespace sb2 {

namespace {

constexpr uint32_t kTileRows = 128;
constexpr int kBinThreads = 256;

__device__ __forceinline__ uint32_t count_below(const double* bounds, uint32_t n, double v) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (bounds[mid] < v)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

__global__ void __launch_bounds__(kBinThreads) bin_group_kernel(BinGroupArgs a) {
    extern __shared__ double bounds[];  // the group's features' bounds, back to back (a.bound_off)
    for (uint32_t i = threadIdx.x; i < a.total_bounds; i += kBinThreads) bounds[i] = a.bounds[i];
    __syncthreads();
    const uint64_t tile0 = static_cast<uint64_t>(blockIdx.x) * kTileRows;
    const uint32_t nf = a.num_features;
    for (uint32_t e = threadIdx.x; e < kTileRows * nf; e += kBinThreads) {
        const uint32_t r = a.row_major ? e / nf : e % kTileRows;
        const uint32_t k = a.row_major ? e % nf : e / kTileRows;
        const uint64_t row = tile0 + r;  // in the chunk
        if (row >= a.chunk_rows) continue;
        const uint64_t at = a.row_major ? (a.row0 + row) * a.cols + a.feature[k]
                                        : static_cast<uint64_t>(a.feature[k]) * a.rows + a.row0 + row;
        const double v = a.f64 ? static_cast<const double*>(a.values)[at]
                               : static_cast<double>(static_cast<const float*>(a.values)[at]);
        const uint32_t off = a.bound_off[k];
        const uint32_t bin = v != v ? a.nan_bin[k] : count_below(bounds + off, a.bound_off[k + 1] - off, v);
        a.out[row * a.stride + a.column[k]] = static_cast<uint8_t>(bin);
    }
}

}  // namespace

cudaError_t launch_bin_group(const BinGroupArgs& a, cudaStream_t s) {
    if (a.chunk_rows == 0 || a.num_features == 0) return cudaSuccess;
    const size_t smem = sizeof(double) * a.total_bounds;
    cudaError_t e = cudaFuncSetAttribute(bin_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const unsigned grid = static_cast<unsigned>((a.chunk_rows + kTileRows - 1) / kTileRows);
    bin_group_kernel<<<grid, kBinThreads, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace sb2
