// binning.cu — a dense matrix's values binned into the dataset's row-major feature groups on the device
// (data::binning::bin_rows, crates/silvic-core/src/data/binning.rs:71-135, with BinMapper::value_to_bin,
// data/bin_mapper.rs:343-360).
//
// Per group, each CTA copies the group's upper bounds into shared memory once (a group holds at most 8192 bins,
// data/mod.rs:22, so its bounds fit) and bins tiles of 128 rows in turn, every thread four rows of one feature at a
// time (four searches in flight), writing the bytes into the group's rows. Row-major input: consecutive threads
// take consecutive features of the same rows (the rows' values of the group are contiguous when its features are);
// column-major: consecutive row quads of a feature. A value's bin is the number of upper bounds below it
// (`partition_point(bound < value)`; the last bound is +inf), found by binary lifting over the feature's own
// bounds: the same count as the reference's branch-free search over bounds padded to 256 with +inf
// (binning.rs:51-61). NaN goes to the NaN bin, or to zero's bin when the feature has none. A categorical feature's
// categories, ascending with their bins, take the bounds' place.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "binning.cuh"

namespace sb2 {

namespace {

constexpr uint32_t kTileRows = 128;
constexpr int kBinThreads = 256;

constexpr uint32_t kQuad = 4;  // rows of one feature a thread bins at once: four searches in flight

// Rust's `f64 as i32`: toward zero, saturating at the i32 range, NaN to 0.
__device__ __forceinline__ int32_t rust_f64_to_i32(double v) {
    if (v != v) return 0;
    if (v >= 2147483647.0) return 2147483647;
    if (v <= -2147483648.0) return static_cast<int32_t>(0x80000000u);
    return static_cast<int32_t>(v);
}

__global__ void __launch_bounds__(kBinThreads) bin_group_kernel(BinGroupArgs a) {
    extern __shared__ double bounds[];  // the group's features' bounds, back to back (a.bound_off)
    for (uint32_t i = threadIdx.x; i < a.total_bounds; i += kBinThreads) bounds[i] = a.bounds[i];
    __syncthreads();
    const uint32_t nf = a.num_features, quads = kTileRows / kQuad;
    const uint64_t tiles = (a.chunk_rows + kTileRows - 1) / kTileRows;
    // a CTA loads its group's bounds once and bins tile after tile
    for (uint64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const uint64_t tile0 = tile * kTileRows;
        for (uint32_t e = threadIdx.x; e < quads * nf; e += kBinThreads) {
            // row-major: consecutive threads take consecutive features of the same rows; column-major:
            // consecutive row quads of the same feature
            const uint32_t k = a.row_major ? e % nf : e / quads;
            const uint32_t q = a.row_major ? e / nf : e % quads;
            const uint64_t row0 = tile0 + kQuad * q;  // in the chunk
            double v[kQuad];
#pragma unroll
            for (uint32_t i = 0; i < kQuad; ++i) {
                const uint64_t row = row0 + i;
                v[i] = 0.0;
                if (row < a.chunk_rows) {
                    const uint64_t at = a.row_major ? (a.row0 + row) * a.cols + a.feature[k]
                                                    : static_cast<uint64_t>(a.feature[k]) * a.rows + a.row0 + row;
                    v[i] = a.f64 ? static_cast<const double*>(a.values)[at]
                                 : static_cast<double>(static_cast<const float*>(a.values)[at]);
                }
            }
            // The number of bounds below each value, by binary lifting over the feature's n bounds (the count is
            // built from the powers of two at or below n, largest first). A categorical feature searches its
            // ascending categories for the value truncated to i32 the same way (categorical_bin,
            // data/bin_mapper.rs:379-391: NaN and negative values are bin 0, so is a category it does not list).
            const bool cat = a.categorical[k] != 0;
            const uint32_t off = a.bound_off[k], n = (a.bound_off[k + 1] - off) >> (cat ? 1 : 0);
            const double* b = bounds + off;
            double key[kQuad];
#pragma unroll
            for (uint32_t i = 0; i < kQuad; ++i) key[i] = cat ? static_cast<double>(rust_f64_to_i32(v[i])) : v[i];
            uint32_t pos[kQuad] = {0, 0, 0, 0};
            for (uint32_t step = n ? 1u << (31 - __clz(n)) : 0u; step; step >>= 1) {
#pragma unroll
                for (uint32_t i = 0; i < kQuad; ++i)
                    if (pos[i] + step <= n && b[pos[i] + step - 1] < key[i]) pos[i] += step;
            }
#pragma unroll
            for (uint32_t i = 0; i < kQuad; ++i) {
                const uint64_t row = row0 + i;
                if (row >= a.chunk_rows) break;
                uint32_t bin;
                if (cat)
                    bin = v[i] != v[i] || key[i] < 0.0 || pos[i] >= n || b[pos[i]] != key[i]
                              ? 0u
                              : static_cast<uint32_t>(b[n + pos[i]]);
                else
                    bin = v[i] != v[i] ? a.nan_bin[k] : pos[i];
                a.out[row * a.stride + a.column[k]] = static_cast<uint8_t>(bin);
            }
        }
    }
}

}  // namespace

cudaError_t launch_bin_group(const BinGroupArgs& a, cudaStream_t s) {
    if (a.chunk_rows == 0 || a.num_features == 0) return cudaSuccess;
    const size_t smem = sizeof(double) * a.total_bounds;
    cudaError_t e = cudaFuncSetAttribute(bin_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    // enough CTAs to fill the GPU, each over many tiles (its copy of the bounds then serves many rows)
    int device = 0, sms = 0, per_sm = 0;
    e = cudaGetDevice(&device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bin_group_kernel, kBinThreads, smem);
    if (e != cudaSuccess) return e;
    const uint64_t tiles = (a.chunk_rows + kTileRows - 1) / kTileRows;
    const uint64_t want = static_cast<uint64_t>(std::max(sms, 1)) * std::max(per_sm, 1);
    const unsigned grid = static_cast<unsigned>(std::min(tiles, want));
    bin_group_kernel<<<grid, kBinThreads, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace sb2
