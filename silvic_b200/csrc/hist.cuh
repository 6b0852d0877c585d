// hist.cuh — the quantized leaf histogram (silvic-core CpuBackend::histogram, backend/cpu.rs:838-864 and
// histogram_quantized :479-513), as an sm_100a kernel.
//
// A CTA takes one "unit" (up to four consecutive tiles) over one chunk of the leaf's rows; units own CTA ranges in
// proportion to their features. Its shared memory holds a private histogram of the unit: per tile an int32
// gradient and an int32 hessian array, laid out bin-major (slot = bin * stride + feature lane), so a feature's bins
// all sit in one bank. int32 sums never overflow for the rows one CTA adds, so a CTA flushes once: it stores its
// shared histogram, in shared-memory order, to its own slab of a scratch buffer (coalesced stores, no atomics),
// and a reduction kernel sums the slabs of the CTAs that took part into the flat [g, h] pairs of the output, one
// writer per output value. Rows come from the leaf's range of the row-id buffer with their packed gradients from
// the ordered-gradient buffer (contiguous), or, for an identity partition (the root without bagging), straight
// from the row index.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace sb2 {

constexpr int kMaxUnitTiles = 4;
// Bytes of dynamic shared memory a histogram CTA needs beyond its unit's arrays: the kernel aligns them to this.
constexpr uint32_t kHistAlign = 128;

struct Unit {
    uint32_t first_tile;
    uint32_t num_tiles;
    uint32_t slots;      // gradient slots of the unit (as many hessian slots follow each tile's)
    uint32_t cta_begin;  // the unit's CTAs are cta_begin .. cta_begin + cta_count of the launch
    uint32_t cta_count;
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

// Four consecutive gradient slots of one tile (one bin, four feature lanes) as the reductions sum them: their
// offsets in a unit's slab region (per tile a gradient array then a hessian array) and the output pair index of
// each lane (hist_offset + bin), -1 for a lane without a feature or a bin past the feature's bins. Built at load.
struct QuadMeta {
    uint32_t unit;
    uint32_t g_off;   // ints from the unit's slab region to the gradient slot
    uint32_t h_off;   // ... to the hessian slot
    uint32_t pad_;
    int32_t out[4];
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
    const sb2_quant_spec* spec;   // the quantization of the packed gradients (bounds their per-bin sums)
    int* out;                     // 2 * total_bins int32: the wanted features' bins are overwritten
    int* slabs;                   // scratch: one slab of slab_ints per CTA of the launch
    uint32_t slab_ints;           // 2 * every unit's slots
    uint32_t num_quads;           // every unit's slots in fours
    const QuadMeta* quads;
    uint32_t quad_split;          // threads per quad in the reduction (a power of two <= 32)
    uint32_t totals;              // the tree kernel's slabs: ints before a slab's rows' totals [g, h] (0: no
                                  // tile skips its dominant bins, and no totals are kept)
};

// The CTAs a unit uses for a job of `count` rows (the histogram and its reduction agree on it).
__host__ __device__ __forceinline__ uint32_t unit_chunks(const Unit& u, uint32_t count, uint32_t min_rows) {
    uint32_t chunks = static_cast<uint32_t>(ceil_div(count, min_rows));
    chunks = chunks < 1 ? 1 : chunks;
    return chunks > u.cta_count ? u.cta_count : chunks;
}

// The histogram: each CTA's private histogram into its scratch slab, then the slabs summed into `out`.
void launch_histogram(const HistArgs& a, int grid, int smem_bytes, cudaStream_t stream);
void launch_histogram_reduce(const HistArgs& a, cudaStream_t stream);
cudaError_t histogram_configure(int smem_bytes);
cudaError_t histogram_occupancy(int smem_bytes, int* blocks_per_sm);
int histogram_threads();

}  // namespace sb2
