// partition.cu — the stable partition of a leaf's rows by a split (CpuBackend::partition and stable_partition,
// crates/silvic-core/src/backend/cpu.rs:556-599,866-884), in two launches with no inter-CTA waiting:
//  1. partition_flags: one bit per position (goes left), a left count per tile of kPartitionTile positions; it
//     also zeroes the staging histogram the step's histogram accumulates into.
//  2. partition_scatter: each tile's lefts before it come from the per-tile counts; every position moves its row id
//     and its packed gradient to the other partition buffer, lefts first, each side in its original order.
// Both children then live in the other buffer at the parent's positions, so nothing is copied back.
#include <cuda_runtime.h>

#include "train.cuh"

namespace sb2 {

namespace {

__device__ __forceinline__ bool goes_left(const uint32_t* left_bins, uint32_t bin) {
    return ((left_bins[bin >> 5] >> (bin & 31)) & 1u) != 0;
}

__global__ void __launch_bounds__(kPartitionThreads) partition_flags_kernel(TrainArgs a) {
    // Zero the staging histogram (and its count slots) for this step's histogram.
    const uint32_t staging_len = 2 * a.total_bins + 2;
    for (uint32_t i = blockIdx.x * kPartitionThreads + threadIdx.x; i < staging_len; i += gridDim.x * kPartitionThreads)
        a.staging[i] = 0;
    const Step& st = *a.step;
    if (!st.active || st.root) return;
    const uint32_t count = st.count;
    const uint32_t tiles = static_cast<uint32_t>(ceil_div(count, kPartitionTile));
    const Tile tile = a.d.tiles[st.split_tile];
    const uint8_t* column = a.d.bins + tile.base + st.split_lane;
    uint32_t left_bins[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) left_bins[k] = st.left_bins[k];
    const uint32_t* rows = a.rows[st.which & 1] + st.begin;
    __shared__ uint32_t warp_counts[kPartitionThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const uint32_t first = t * kPartitionTile;
        uint32_t mine = 0;
        // kPartitionTile / 32 words per tile, one warp-wide ballot each.
        for (uint32_t w = warp; w < kPartitionTile / 32; w += kPartitionThreads / 32) {
            const uint32_t p = first + w * 32 + lane;
            bool left = false;
            if (p < count) {
                const uint32_t row = __ldg(rows + p);
                if (st.bag)  // quantize::in_bag (quantize.rs:147-149)
                    left = static_cast<double>(uniform01(st.bag_seed, 2u, st.bag_round, st.row_offset + row)) <
                           st.bag_fraction;
                else
                    left = goes_left(left_bins, __ldg(column + static_cast<uint64_t>(row) * tile.stride));
            }
            const uint32_t word = __ballot_sync(0xffffffffu, left);
            if (lane == 0 && first + w * 32 < count) a.flags[(first >> 5) + w] = word;
            mine += __popc(word);
        }
        if (lane == 0) warp_counts[warp] = mine;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t total = 0;
            for (int k = 0; k < kPartitionThreads / 32; ++k) total += warp_counts[k];
            a.tile_left[t] = total;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kPartitionThreads) partition_scatter_kernel(TrainArgs a) {
    Step& st = *a.step;
    if (!st.active || st.root) return;
    const uint32_t count = st.count;
    const uint32_t tiles = static_cast<uint32_t>(ceil_div(count, kPartitionTile));
    __shared__ uint32_t red[kPartitionThreads / 32];
    __shared__ uint32_t word_prefix[kPartitionTile / 32];
    __shared__ uint32_t s_total, s_before;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // Total lefts over all tiles (every CTA needs it for the right side's base).
    uint32_t part = 0;
    for (uint32_t t = threadIdx.x; t < tiles; t += kPartitionThreads) part += a.tile_left[t];
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane == 0) red[warp] = part;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t total = 0;
        for (int k = 0; k < kPartitionThreads / 32; ++k) total += red[k];
        s_total = total;
    }
    __syncthreads();
    const uint32_t total_left = s_total;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        st.local_left = total_left;
        // The left count rides after the staging histogram through the step's allreduce (learner.rs:217-218).
        a.staging[2 * a.total_bins] = static_cast<int>(total_left);
        HistJob job{};
        job.active = st.may_search;
        job.identity = 0;
        job.which = (st.which & 1) ^ 1u;
        if (st.built_left) {
            job.begin = st.begin;
            job.count = total_left;
        } else {
            job.begin = st.begin + total_left;
            job.count = count - total_left;
        }
        *a.hist_job = job;
    }
    const uint32_t src = st.which & 1, dst = src ^ 1u;
    const uint32_t* rows_in = a.rows[src] + st.begin;
    const int32_t* gh_in = a.ordered[src] + st.begin;
    uint32_t* rows_out = a.rows[dst] + st.begin;
    int32_t* gh_out = a.ordered[dst] + st.begin;
    for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        // Lefts of the tiles before this one.
        uint32_t before = 0;
        for (uint32_t k = threadIdx.x; k < t; k += kPartitionThreads) before += a.tile_left[k];
        for (int o = 16; o > 0; o >>= 1) before += __shfl_xor_sync(0xffffffffu, before, o);
        __syncthreads();
        if (lane == 0) red[warp] = before;
        // Exclusive prefix of the tile's flag words (kPartitionTile / 32 = 128 words).
        const uint32_t first = t * kPartitionTile;
        const uint64_t left_words = ceil_div(count - first, 32);
        const uint32_t words = static_cast<uint32_t>(left_words < kPartitionTile / 32 ? left_words : kPartitionTile / 32);
        if (threadIdx.x < kPartitionTile / 32)
            word_prefix[threadIdx.x] = threadIdx.x < words ? __popc(a.flags[(first >> 5) + threadIdx.x]) : 0u;
        __syncthreads();
        if (warp == 0) {
            // Exclusive scan of the 128 word counts, 4 per lane.
            constexpr int kPer = kPartitionTile / 32 / 32;
            uint32_t v[kPer];
            uint32_t sum = 0;
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                v[i] = word_prefix[lane * kPer + i];
                sum += v[i];
            }
            uint32_t incl = sum;
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t up = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += up;
            }
            uint32_t run = incl - sum;
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                word_prefix[lane * kPer + i] = run;
                run += v[i];
            }
            if (lane == 0) {
                uint32_t b = 0;
                for (int k = 0; k < kPartitionThreads / 32; ++k) b += red[k];
                s_before = b;
            }
        }
        __syncthreads();
        const uint32_t lefts_before_tile = s_before;
        for (uint32_t w = warp; w < words; w += kPartitionThreads / 32) {
            const uint32_t p = first + w * 32 + lane;
            if (p >= count) continue;
            const uint32_t word = a.flags[(first >> 5) + w];
            const bool left = (word >> lane) & 1u;
            const uint32_t lefts_before = lefts_before_tile + word_prefix[w] + __popc(word & ((1u << lane) - 1u));
            const uint32_t target = left ? lefts_before : total_left + (p - lefts_before);
            rows_out[target] = __ldg(rows_in + p);
            gh_out[target] = __ldg(gh_in + p);
        }
        __syncthreads();
    }
}

}  // namespace

void launch_partition_flags(const TrainArgs& a, int grid, cudaStream_t s) {
    partition_flags_kernel<<<grid, kPartitionThreads, 0, s>>>(a);
}

void launch_partition_scatter(const TrainArgs& a, int grid, cudaStream_t s) {
    partition_scatter_kernel<<<grid, kPartitionThreads, 0, s>>>(a);
}

}  // namespace sb2
