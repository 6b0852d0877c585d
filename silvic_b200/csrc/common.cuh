// common.cuh — device data layout and the scalar math the kernels share.
//
// Device layout of a loaded training set (one GPU's row shard):
//  - bins: the non-trivial features re-packed into tiles of at most 32 features. Tile t is row-major,
//    `rows x stride_t` bytes (stride_t = its feature count rounded up to 4), so one row of a full tile is one 32-byte
//    DRAM sector. Lane j of a warp owns the tile's feature j. In a tile whose features are dominated by one bin
//    each (Tile::skip, when sb2_set_dominant_share asks for it), every feature's bins 0 and mfb (its most frequent
//    bin) trade places in the tile bytes, so
//    the tree kernel's histogram skips the dominant bin with one compare against 0 and recovers it by subtraction
//    from the rows' totals (LightGBM's most_freq_bin, which the reference's hist_quant keeps in a register,
//    crates/silvic-gpu/kernels/kernels.kern:439-468). Only histograms read tile bytes; the columns stay as loaded.
//  - columns: every feature's bins again, feature-major (feature f's byte of row r at f * column_stride + r), for
//    the partition, which reads one feature of a leaf's rows: rows of a leaf sit in runs of increasing row id, so a
//    warp's 32 rows share a few sectors of a column instead of costing a 32-byte row sector each.
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
    uint32_t stride;     // the tile's bytes per row (feature count rounded up to 4)
    uint32_t nfeat;      // features in the tile
    uint32_t smem_bins;  // bins per lane kept in the histogram's shared slots (max num_bins in the tile)
    uint32_t pitch;      // bytes from one row to the next: the tiles of a histogram unit share their rows
    uint32_t skip;       // 1: the features' dominant bins are stored as 0 and the tree kernel skips stored 0s
    uint32_t pad_;
};

// DevFeature::mfb: the bin stored as 0 in the tiles (bits 0-7) and kDominantSkip when the feature's tile skips.
constexpr uint32_t kDominantSkip = 1u << 8;

// A tile byte of a feature whose bins 0 and `mfb` trade places, to its bin (and a bin to its tile byte: the
// exchange is its own inverse).
__host__ __device__ __forceinline__ uint32_t swap_dominant(uint32_t bin, uint32_t mfb) {
    return bin == 0 ? mfb : (bin == mfb ? 0u : bin);
}

// A feature as the kernels see it.
struct DevFeature {
    int32_t tile;         // -1 for a trivial feature
    int32_t lane;
    uint32_t hist_offset;
    uint32_t num_bins;
    uint32_t nan_bin;
    uint32_t kind;
    uint32_t slab_off;    // the tree kernel's slabs: this feature's packed bins start here ([g, h] pairs at twice it)
    uint32_t mfb;         // bits 0-7: the bin stored as 0 in the tiles (swap_dominant); kDominantSkip: tile skips
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
    const uint8_t* columns;  // feature-major copy (null when not built)
    uint64_t column_stride;  // bytes per column: num_rows rounded up to 128
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

// A feature flag that may sit in shared memory (the persistent kernel's copies) or in global memory written earlier
// in the same launch (read past the SM's L1).
__device__ __forceinline__ uint8_t load_flag(const uint8_t* p) { return __isShared(p) ? *p : __ldcg(p); }

// ---- correctly rounded division in pipelined FMA operations -------------------------------------------------
//
// a / b rounded to nearest even, as IEEE 754 division. The split scan divides 16 times per lane per feature; the
// library division runs those one after another at a few hundred cycles each, which made the scan a 10k-cycle
// chain. This one is straight-line FMA code, so a lane's divisions overlap. Method (Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; Cornea, Harrison, Tang,
// "Scientific Computing on Itanium-based Systems", 2002, ch. 8): a single-precision reciprocal seed refined by two
// Newton-Raphson steps y <- y + y (1 - b y); the quotient q = a y, one correction q <- q + y (a - b q), which leaves
// q within one ulp of a / b; then, since a - b q is exactly representable for such q (no underflow in the range
// below) and one FMA computes it exactly, the correctly rounded quotient is whichever of q and its neighbour toward
// a / b leaves the smaller |a - b q|, the even one on a tie. Operands outside the range where no step can overflow
// or underflow, and NaN, infinities and zero divisors, take __ddiv_rn.
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Whether div_fast is exact for a / b: no step can overflow or underflow.
__device__ __forceinline__ bool div_in_range(double a, double b) {
    const double aa = fabs(a), ab = fabs(b);
    return ab > 0x1p-120 && ab < 0x1p120 && aa < 0x1p500 && (aa > 0x1p-500 || aa == 0.0);
}

// The branch-free part of div_rn: a / b correctly rounded when div_in_range(a, b).
__device__ __forceinline__ double div_fast(double a, double b) {
    double y = static_cast<double>(rcp_approx(static_cast<float>(b)));
    double e = __fma_rn(-b, y, 1.0);
    y = __fma_rn(y, e, y);
    e = __fma_rn(-b, y, 1.0);
    y = __fma_rn(y, e, y);
    double q = __dmul_rn(a, y);
    q = __fma_rn(__fma_rn(-b, q, a), y, q);
    const double r = __fma_rn(-b, q, a);  // exact
    // a / b - q = r / b: the neighbour toward a / b is above q when r and b have the same sign; adjacent doubles of
    // one sign are adjacent bit patterns (larger magnitude, larger pattern)
    const bool up = (r > 0.0) == (b > 0.0);
    const long long qb = __double_as_longlong(q);
    const long long nb = q == 0.0 ? (up ? 1ll : static_cast<long long>(0x8000000000000001ull))
                                  : ((q > 0.0) == up ? qb + 1 : qb - 1);
    const double q2 = __longlong_as_double(nb);
    const double r2 = __fma_rn(-b, q2, a);  // exact
    const double m = fabs(r), m2 = fabs(r2);
    return m2 < m || (m2 == m && (__double_as_longlong(q2) & 1) == 0) ? q2 : q;
}

__device__ __forceinline__ double div_rn(double a, double b) { return div_in_range(a, b) ? div_fast(a, b) : __ddiv_rn(a, b); }

// N divisions issued together (their fast paths overlap), then the library division for any pair outside the range.
template <int N>
__device__ __forceinline__ void div_rn_batch(const double (&a)[N], const double (&b)[N], double (&q)[N]) {
    bool slow = false;
#pragma unroll
    for (int j = 0; j < N; ++j) {
        slow |= !div_in_range(a[j], b[j]);
        q[j] = div_fast(a[j], b[j]);
    }
    if (slow) {
#pragma unroll
        for (int j = 0; j < N; ++j)
            if (!div_in_range(a[j], b[j])) q[j] = __ddiv_rn(a[j], b[j]);
    }
}

// ---- launch helpers ------------------------------------------------------------------------------------------

__host__ __device__ __forceinline__ uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

}  // namespace sb2
