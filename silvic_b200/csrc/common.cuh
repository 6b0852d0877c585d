// common.cuh — device data layout and the scalar math the kernels share.
//
// Device layout of a loaded training set (one GPU's row shard):
//  - bins: the non-trivial features re-packed into tiles of at most 32 features. Tile t is row-major,
//    `rows x stride_t` bytes (stride_t = its feature count rounded up to 4), so one row of a full tile is one 32-byte
//    DRAM sector. Lane j of a warp owns the tile's feature j.
//  - partition: two u32 row-id buffers and two packed-gradient buffers ("ordered gradients"). Every leaf's rows are a
//    contiguous range of one of the two, recorded per leaf; a partition reads a leaf from one buffer and writes both
//    children to the other at the same positions.
//  - histograms: int32 [g, h] pairs per bin in the reference's flat layout (2 * total_bins), one slot per leaf plus
//    a staging buffer that every split's new histogram is accumulated (and NCCL-reduced) in.
#pragma once

#include <cstdint>

#include "../../include/silvic_b200.h"

namespace sb2 {

constexpr int kTileLanes = 32;      // features per tile
constexpr int kMaxBins = 256;       // bins per feature are bytes
constexpr int kWarp = 32;

// One tile of up to 32 features.
struct Tile {
    uint64_t base;       // byte offset of the tile's row 0 in the bins buffer
    uint32_t stride;     // bytes per row (feature count rounded up to 4)
    uint32_t nfeat;      // features in the tile
    uint32_t smem_bins;  // bins per lane kept in the histogram's shared slots (max num_bins in the tile)
    uint32_t pad_;
};

// A feature as the kernels see it.
struct DevFeature {
    int32_t tile;         // -1 for a trivial feature
    int32_t lane;
    uint32_t hist_offset;
    uint32_t num_bins;
    uint32_t nan_bin;
    uint32_t kind;
};

// The loaded training shard, passed to kernels by value.
struct DevData {
    const uint8_t* bins;
    const Tile* tiles;
    const DevFeature* features;
    const int32_t* lane_feature;  // [tile * 32 + lane] -> feature, -1 for an empty lane
    uint32_t num_tiles;
    uint32_t num_features;
    uint32_t total_bins;
    uint32_t pad_;
    uint64_t num_rows;
    uint64_t row_offset;
};

// ---- quantize.rs, shared by host and device ------------------------------------------------------------------

// lowbias32 (crates/silvic-core/src/quantize.rs:16-23)
__host__ __device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352dU;
    x ^= x >> 15;
    x *= 0x846ca68bU;
    x ^= x >> 16;
    return x;
}

// quantize.rs:27-31: 24-bit uniform in [0, 1), exact in f32.
__host__ __device__ __forceinline__ float uniform01(uint32_t seed, uint32_t stream, uint32_t iteration, uint64_t row) {
    uint32_t row_hash = mix32(static_cast<uint32_t>(row) ^ mix32(static_cast<uint32_t>(row >> 32)));
    uint32_t h = mix32(seed ^ mix32(stream ^ mix32(iteration ^ row_hash)));
    return static_cast<float>(h >> 8) * (1.0f / 16777216.0f);
}

// Rust's saturating `f32 as i32`.
__device__ __forceinline__ int32_t sat_f32_i32(float q) {
    if (q != q) return 0;
    if (q >= 2147483647.0f) return 2147483647;
    if (q <= -2147483648.0f) return static_cast<int32_t>(0x80000000u);
    return static_cast<int32_t>(q);
}

__device__ __forceinline__ int32_t clamp_i32(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

// quantize_grad / quantize_hess / quantize_row (quantize.rs:103-136): fused multiply-add as Rust's `mul_add`.
__device__ __forceinline__ int32_t quantize_row(const sb2_quant_spec& s, float grad, float hess, uint64_t row) {
    float qg;
    if (s.stochastic) {
        float u = uniform01(s.seed, 0u, s.iteration, row);
        qg = grad >= 0.0f ? truncf(__fmaf_rn(grad, s.inv_grad_scale, u)) : truncf(__fmaf_rn(grad, s.inv_grad_scale, -u));
    } else {
        qg = rintf(__fmul_rn(grad, s.inv_grad_scale));
    }
    int32_t g = clamp_i32(sat_f32_i32(qg), -s.grad_max_q, s.grad_max_q);
    int32_t h;
    if (s.constant_hessian) {
        h = 1;
    } else {
        float qh;
        if (s.stochastic) {
            float u = uniform01(s.seed, 1u, s.iteration, row);
            qh = truncf(__fmaf_rn(hess, s.inv_hess_scale, u));
        } else {
            qh = rintf(__fmul_rn(hess, s.inv_hess_scale));
        }
        h = clamp_i32(sat_f32_i32(qh), 0, s.hess_max_q);
    }
    return h * 65536 + g;
}

// unpack (quantize.rs:140-143) straight into the 64-bit (h << 32) + g the shared histograms add.
__device__ __forceinline__ long long packed_to_wide(int32_t packed) {
    int32_t g = static_cast<int16_t>(static_cast<uint16_t>(static_cast<uint32_t>(packed)));
    int32_t h = (packed - g) >> 16;
    return (static_cast<long long>(h) << 32) + static_cast<long long>(g);
}

// ---- launch helpers ------------------------------------------------------------------------------------------

__host__ __device__ __forceinline__ uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

}  // namespace sb2
