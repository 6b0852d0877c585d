// partition.cuh — the stable partition of a leaf's rows by a split (CpuBackend::partition and stable_partition,
// crates/silvic-core/src/backend/cpu.rs:556-599,866-884), as CTA-level device functions shared by the standalone
// kernels (partition.cu) and the persistent tree kernel (grow.cu).
//
// The parent's positions are cut into 32-position words, and CTA c of G owns words [W c / G, W (c + 1) / G):
//  1. partition_flags_cta: one bit per position (goes left), kept in `flags`, and the CTA's left count.
//  2. partition_scatter_cta: the lefts of the CTAs before it (a sum over G counts) and the total; an exclusive scan
//     of the word counts in rounds of one word per thread; every position moves its row id and packed gradient to
//     the other partition buffer, lefts first, each side in its original order.
// Both children then live in the other buffer at the parent's positions, so nothing is copied back.
#pragma once

#include "train.cuh"

namespace sb2 {

__device__ __forceinline__ bool bin_goes_left(const uint32_t* left_bins, uint32_t bin) {
    return ((left_bins[bin >> 5] >> (bin & 31)) & 1u) != 0;
}

// Words of CTA `cta` of `ctas` over a parent of `count` positions.
__device__ __forceinline__ void cta_words(uint32_t count, uint32_t cta, uint32_t ctas, uint32_t& w_lo, uint32_t& w_hi) {
    const uint32_t words = static_cast<uint32_t>(ceil_div(count, 32));
    w_lo = static_cast<uint32_t>(static_cast<uint64_t>(words) * cta / ctas);
    w_hi = static_cast<uint32_t>(static_cast<uint64_t>(words) * (cta + 1) / ctas);
}

// Phase 1: flags and the CTA's left count (`cta_left[cta]`). `red` is blockDim/32 words of shared memory.
inline __device__ void partition_flags_cta(const TrainArgs& a, const Step& st, uint32_t cta, uint32_t ctas, uint32_t* red) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    uint32_t w_lo, w_hi;
    cta_words(st.count, cta, ctas, w_lo, w_hi);
    const Tile tile = a.d.tiles[st.split_tile];
    const uint8_t* column = a.d.bins + tile.base + st.split_lane;
    // the tile stores the feature's bins 0 and mfb exchanged (swap_dominant)
    const int32_t split_f = a.d.lane_feature[st.split_tile * kTileLanes + st.split_lane];
    const uint32_t mfb = split_f >= 0 ? (a.d.features[split_f].mfb & 0xFFu) : 0u;
    const uint32_t* rows = a.rows[st.which & 1] + st.begin;
    uint32_t mine = 0;
    // kBatch words per warp at a time: their row ids, then their bins, are in flight together.
    constexpr int kBatch = 4;
    for (uint32_t w0 = w_lo + warp; w0 < w_hi; w0 += kBatch * warps) {
        uint32_t row[kBatch];
        bool valid[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const uint32_t w = w0 + j * warps, p = w * 32 + lane;
            valid[j] = w < w_hi && p < st.count;
            row[j] = valid[j] ? __ldcg(rows + p) : 0u;  // written by an earlier step, maybe in the same kernel
        }
        bool left[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            left[j] = false;
            if (!valid[j]) continue;
            if (st.bag)  // quantize::in_bag (quantize.rs:147-149)
                left[j] = static_cast<double>(uniform01(st.bag_seed, 2u, st.bag_round, st.row_offset + row[j])) <
                          st.bag_fraction;
            else
                left[j] = bin_goes_left(st.left_bins,
                                        swap_dominant(__ldg(column + static_cast<uint64_t>(row[j]) * tile.pitch), mfb));
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const uint32_t w = w0 + j * warps;
            if (w >= w_hi) break;  // warp-uniform
            const uint32_t word = __ballot_sync(0xffffffffu, left[j]);
            if (lane == 0) a.flags[w] = word;
            mine += __popc(word);
        }
    }
    if (lane == 0) red[warp] = mine;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t total = 0;
        for (uint32_t k = 0; k < warps; ++k) total += red[k];
        a.tile_left[cta] = total;
    }
    __syncthreads();
}

// Phase 2: the scatter. `scan` holds 2 blockDim + 64 words of shared memory. Returns the total left count.
inline __device__ uint32_t partition_scatter_cta(const TrainArgs& a, const Step& st, uint32_t cta, uint32_t ctas, uint32_t* scan) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    uint32_t* words = scan + blockDim.x;           // the round's flag words
    uint32_t* warp_sums = scan + 2 * blockDim.x;   // 32 words
    // Lefts of the CTAs before this one, and over all of them (warp 0: G counts, four per lane in flight).
    if (warp == 0) {
        uint32_t before = 0, total = 0;
        for (uint32_t c0 = 0; c0 < ctas; c0 += 128) {
            uint32_t v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t c = c0 + 32u * j + lane;
                v[j] = c < ctas ? __ldcg(a.tile_left + c) : 0u;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                total += v[j];
                if (c0 + 32u * j + lane < cta) before += v[j];
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            before += __shfl_xor_sync(0xffffffffu, before, o);
            total += __shfl_xor_sync(0xffffffffu, total, o);
        }
        if (lane == 0) {
            warp_sums[0] = before;
            warp_sums[1] = total;
        }
    }
    __syncthreads();
    uint32_t carry = warp_sums[0];
    const uint32_t total_left = warp_sums[1];
    __syncthreads();
    uint32_t w_lo, w_hi;
    cta_words(st.count, cta, ctas, w_lo, w_hi);
    const uint32_t src = st.which & 1, dst = src ^ 1u;
    const uint32_t* rows_in = a.rows[src] + st.begin;
    const int32_t* gh_in = a.ordered[src] + st.begin;
    uint32_t* rows_out = a.rows[dst] + st.begin;
    int32_t* gh_out = a.ordered[dst] + st.begin;
    uint32_t* round_sum = warp_sums + 32;  // 1 word
    for (uint32_t r0 = w_lo; r0 < w_hi; r0 += blockDim.x) {
        // Exclusive scan of this round's word counts, one word per thread.
        const uint32_t w = r0 + threadIdx.x;
        const uint32_t word = w < w_hi ? __ldcg(a.flags + w) : 0u;
        words[threadIdx.x] = word;
        const uint32_t c = __popc(word);
        uint32_t incl = c;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t up = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= static_cast<uint32_t>(o)) incl += up;
        }
        if (lane == 31) warp_sums[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const uint32_t v = lane < warps ? warp_sums[lane] : 0u;
            uint32_t vi = v;
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t up = __shfl_up_sync(0xffffffffu, vi, o);
                if (lane >= static_cast<uint32_t>(o)) vi += up;
            }
            if (lane < warps) warp_sums[lane] = vi - v;  // exclusive warp offsets
            if (lane == 31) *round_sum = vi;             // the round's lefts
        }
        __syncthreads();
        scan[threadIdx.x] = carry + warp_sums[warp] + incl - c;  // lefts before word w over the whole parent
        const uint32_t round_total = *round_sum;
        __syncthreads();
        // Positions of the round's words, a warp per word, four words per warp in flight: coalesced row-id and
        // gradient moves.
        const uint32_t round_words = min(blockDim.x, w_hi - r0);
        constexpr int kBatch = 4;
        for (uint32_t k0 = warp; k0 < round_words; k0 += kBatch * warps) {
            uint32_t rid[kBatch];
            int32_t gh[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const uint32_t k = k0 + j * warps, p = (r0 + k) * 32 + lane;
                const bool ok = k < round_words && p < st.count;
                rid[j] = ok ? __ldcg(rows_in + p) : 0u;
                gh[j] = ok ? __ldcg(gh_in + p) : 0;
            }
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const uint32_t k = k0 + j * warps, p = (r0 + k) * 32 + lane;
                if (k >= round_words || p >= st.count) continue;
                const uint32_t bits = words[k];
                const bool left = (bits >> lane) & 1u;
                const uint32_t lefts_before = scan[k] + __popc(bits & ((1u << lane) - 1u));
                const uint32_t target = left ? lefts_before : total_left + (p - lefts_before);
                rows_out[target] = rid[j];
                gh_out[target] = gh[j];
            }
        }
        __syncthreads();
        carry += round_total;
    }
    return total_left;
}

// After the scatter: the count rides after the staging histogram (learner.rs:217-218) and the histogram job of the
// built child is written. One thread.
__device__ __forceinline__ void partition_publish(const TrainArgs& a, Step& st, uint32_t total_left) {
    st.local_left = total_left;
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
        job.count = st.count - total_left;
    }
    *a.hist_job = job;
}

}  // namespace sb2
