// binning.cuh — the device binning of a dense matrix into feature groups (binning.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace sb2 {

// One group's bins of rows row0 .. row0 + chunk_rows of a rows × cols matrix.
struct BinGroupArgs {
    const void* values;         // the whole matrix (device), f32 or f64
    uint64_t rows;              // the matrix's rows (column-major pitch)
    uint64_t row0;              // the chunk's first row
    uint64_t chunk_rows;
    uint32_t cols;              // the matrix's columns (row-major pitch)
    int32_t f64;                // values are doubles
    int32_t row_major;
    uint32_t num_features;      // the group's features
    const uint32_t* feature;    // [num_features]: matrix column (= feature index) of each
    const uint32_t* column;     // [num_features]: byte column in the group's row
    const uint32_t* bound_off;  // [num_features + 1]: each feature's bounds in `bounds`
    const uint8_t* nan_bin;     // [num_features]: the bin of NaN
    const uint8_t* categorical; // [num_features]: 1 for a categorical feature, whose `bounds` hold its n categories
                                // ascending, then their n bins (2 n entries)
    const double* bounds;       // the features' upper bounds (or categories and bins), back to back
    uint32_t total_bounds;
    uint32_t stride;            // the group's row stride
    uint8_t* out;               // the chunk's rows of the group: chunk_rows × stride bytes
};

cudaError_t launch_bin_group(const BinGroupArgs& a, cudaStream_t s);

}  // namespace sb2
