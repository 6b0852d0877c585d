// hist.cuh — the quantized leaf histogram (silvic-core CpuBackend::histogram, backend/cpu.rs:838-864 and
// histogram_quantized :479-513), as an sm_100a kernel.
//
// A CTA takes one "unit" (up to four consecutive tiles) over one chunk of the leaf's rows. Its shared memory holds
// a private histogram of the unit in 64-bit packed (h << 32) + g slots, laid out bin-major per tile
// (slot = bin * stride + lane), so lane j of a warp always hits the slot of its own feature: the 32 lanes of one row
// fall in 32 consecutive slots, a conflict-free shared atomic. 64-bit slots never overflow for any row count a GPU
// holds, so a CTA adds all its rows and flushes once, unpacking each non-zero slot into the int32 [g, h] pairs of
// the output with global reductions. Rows come from the leaf's range of the row-id buffer with their packed
// gradients from the ordered-gradient buffer (contiguous), or, for an identity partition (the root without
// bagging), straight from the row index.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace sb2 {

constexpr int kMaxUnitTiles = 4;

struct Unit {
    uint32_t first_tile;
    uint32_t num_tiles;
    uint32_t slots;  // 64-bit shared slots of the unit
    uint32_t pad_;
};

// The rows a histogram launch covers; written by the host (Backend calls) or by the partition kernel (training).
struct HistJob {
    int32_t active;    // 0: the launch does nothing
    int32_t identity;  // rows are begin .. begin + count themselves (row ids and ordered gradients not read)
    uint32_t begin;
    uint32_t count;
    uint32_t which;    // partition buffer holding the rows
    uint32_t pad_;
};

struct HistArgs {
    DevData d;
    const Unit* units;
    uint32_t num_units;
    uint32_t min_rows_per_cta;
    const HistJob* job;
    const uint32_t* rows[2];      // row-id buffers
    const int32_t* ordered[2];    // ordered packed gradients, by partition position
    const int32_t* packed;        // packed gradients by row (identity jobs)
    const uint8_t* active;        // per feature: its bins are wanted; nullptr for all
    int* out;                     // 2 * total_bins int32, accumulated into
};

void launch_histogram(const HistArgs& a, int grid, int smem_bytes, cudaStream_t stream);
cudaError_t histogram_configure(int smem_bytes);
cudaError_t histogram_occupancy(int smem_bytes, int* blocks_per_sm);
int histogram_threads();

}  // namespace sb2
