// hist_device.cuh — the histogram's CTA-level device functions (see hist.cuh), shared by the standalone kernels
// (hist.cu) and the persistent tree kernel (grow.cu).
//
// Shared memory of a CTA: for each tile of its unit, one int32 array of smem_bins * stride slots, slot = bin *
// stride + feature lane, that accumulates the rows' packed gradients h * 65536 + g as they are (quantize.rs:103-107):
// one 32-bit shared reduction per element, the shared-atomic unit's fastest operation on sm_100 (the kernel is bound
// by it). The packed sums stay exact while every bin's |sum g| <= 32767 and sum h <= 65535, so a CTA adds at most
// `round_rows` rows (packed_round_rows) before it flushes: it unpacks the slots into its slab of separate int32 g and
// h arrays (stored the first time, added afterwards) and clears them.
//
// Work per warp: a range of consecutive positions of the leaf. The unit's full tiles (32 features each, side by side
// in rows of up to 128 bytes) are read in row chunks (hist_rows): lane k loads 16 bytes of a row such that one
// 128-bit load of the warp covers whole rows, permutes them by a lane constant and walks them, so that the 32 lanes
// of every atomic hit 32 different features, i.e. 32 different banks. A partial tile (fewer than 32 features, in its
// own region) is read lane per row: lane k loads position k's row and at step i adds feature i XOR (k mod stride).
// The arrays are aligned so that an element costs one multiply-add for its address and one shared reduction. Rows
// whose packed gradient is zero add nothing and skip their loads and atomics.
#pragma once

#include "hist.cuh"

namespace sb2 {

constexpr int kHistThreads = 512;

struct LaneTile {
    const uint8_t* base;  // the tile's row 0
    uint32_t stride;      // 4, 8, 16 or 32 bytes of a row
    uint32_t bins;        // 64, 128 or 256: bin slots per feature lane
    uint32_t addr;        // shared address of the tile's packed array (aligned to 4 * stride bytes)
    uint32_t active;      // bit f: feature lane f is wanted (0: the tile is skipped)
    uint32_t stage_off;   // where a batch's rows of this tile start in a staging slot (the tree kernel's histogram)
    uint32_t pitch;       // bytes from one row to the next (Tile::pitch)
    uint32_t skip;        // Tile::skip: the tree kernel adds no stored bin 0 (each feature's dominant bin)
    uint32_t pad_;
};

// Rows whose packed gradients one packed histogram can sum exactly: every bin's |sum g| <= 32767 and sum h <=
// 65535 (h is 1 per row with a constant hessian).
__host__ __device__ __forceinline__ uint32_t packed_round_rows(const sb2_quant_spec& s) {
    const uint32_t gq = s.grad_max_q > 1 ? static_cast<uint32_t>(s.grad_max_q) : 1u;
    const uint32_t hq = s.constant_hessian ? 1u : (s.hess_max_q > 1 ? static_cast<uint32_t>(s.hess_max_q) : 1u);
    const uint32_t r = 32767u / gq < 65535u / hq ? 32767u / gq : 65535u / hq;
    return r;
}

// A packed round shorter than a batch per warp is not worth the flushes: such quantizations (more than 64
// gradient bins) histogram straight into the output instead (histogram_direct_cta).
constexpr uint32_t kMinRoundRows = kHistThreads;

// Jobs of at most kDirectRows rows skip the shared histograms too: every (row, feature) adds straight into the
// output with global reductions, so there is nothing to clear, flush or reduce, which for a small leaf costs more
// than its few atomics.
constexpr uint32_t kDirectRows = 4096;

// Whether a histogram of `count` rows goes straight into the output (histogram_direct_cta) rather than through the
// shared histograms and their slab reduction.
__host__ __device__ __forceinline__ bool histogram_goes_direct(uint32_t count, uint32_t round_rows) {
    return count <= kDirectRows || round_rows < kMinRoundRows;
}

// Permutes the `W` words of a row so that byte i becomes the row's byte i ^ k (k < 4 W): byte bits within each word
// by one byte_perm, word bits by conditional swaps.
template <int W>
__device__ __forceinline__ void xor_bytes(uint32_t (&w)[W], uint32_t k) {
    const uint32_t kb = k & 3;
    const uint32_t sel = (0u ^ kb) | ((1u ^ kb) << 4) | ((2u ^ kb) << 8) | ((3u ^ kb) << 12);
#pragma unroll
    for (int j = 0; j < W; ++j) w[j] = __byte_perm(w[j], 0u, sel);
    const uint32_t q = k >> 2;
#pragma unroll
    for (int bit = 1; bit < W; bit <<= 1) {
        const bool swap = (q & bit) != 0;
#pragma unroll
        for (int j = 0; j < W; ++j) {
            if (j & bit) continue;
            const uint32_t lo = w[j], hi = w[j | bit];
            w[j] = swap ? hi : lo;
            w[j | bit] = swap ? lo : hi;
        }
    }
}

// Adds `v` at shared address `addr` with red.shared: no return value, never the generic path. No "memory" clobber:
// the compiler may move global loads across these (the histogram is only read after a barrier).
__device__ __forceinline__ void shared_add(uint32_t addr, uint32_t v) {
    asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(addr), "r"(v));
}

// shared_add where `bin` is not 0, as one predicated instruction (no branch: lanes never diverge).
__device__ __forceinline__ void shared_add_nonzero(uint32_t addr, uint32_t v, uint32_t bin) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t@p red.shared.add.u32 [%0], %1;\n\t}" ::"r"(addr), "r"(v),
        "r"(bin));
}

// Issues the loads of one row of a tile (stride 4, 8, 16 or 32 bytes) into w[0 .. stride / 4). Streaming loads
// (evict first): a histogram reads its rows' bins once, and the leaf histograms, partition buffers and metadata the
// next phases read should stay in L2 instead.
__device__ __forceinline__ void load_row(const LaneTile& t, uint32_t row, uint32_t (&w)[8]) {
    const uint8_t* p = t.base + static_cast<uint64_t>(row) * t.pitch;
    if (t.stride == 32) {
        const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
        const uint4 b = __ldcs(reinterpret_cast<const uint4*>(p) + 1);
        w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w, w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
    } else if (t.stride == 16) {
        const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
        w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w;
    } else if (t.stride == 8) {
        const uint2 a = __ldcs(reinterpret_cast<const uint2*>(p));
        w[0] = a.x, w[1] = a.y;
    } else {
        w[0] = __ldcs(reinterpret_cast<const uint32_t*>(p));
    }
}

// Adds one loaded row of one tile of `W` words (stride S = 4 W bytes): the lane's row's packed gradient at feature
// i ^ k for i = 0 .. S-1, k = lane mod S. Slot (bin, f) is word bin * S + f, so the S lanes of every step hit S
// different features, i.e. S different banks; with the array aligned to 4 S bytes the slot's address is
// bin * 4S + (base | 4k) ^ 4i, one multiply-add per element. Every feature of the tile is added, wanted or not:
// only wanted features' bins are ever read back. With kSkip, stored bin 0 (each feature's dominant bin in a
// Tile::skip tile) adds nothing: the tree kernel recovers it from the rows' totals.
template <int W, bool kSkip = false>
__device__ __forceinline__ void add_row(const LaneTile& t, const uint32_t (&wrow)[8], uint32_t packed, uint32_t lane) {
    constexpr uint32_t kStride = 4 * W;
    uint32_t w[W];
#pragma unroll
    for (int j = 0; j < W; ++j) w[j] = wrow[j];
    const uint32_t k = lane & (kStride - 1);
    xor_bytes<W>(w, k);
    const uint32_t base = t.addr | (4 * k);
#pragma unroll
    for (int i = 0; i < static_cast<int>(kStride); ++i) {
        const uint32_t bin = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
        if (kSkip)
            shared_add_nonzero(bin * (4 * kStride) + (base ^ (4u * i)), packed, bin);
        else
            shared_add(bin * (4 * kStride) + (base ^ (4u * i)), packed);
    }
}

// Where a histogram's positions take their rows and packed gradients from: a partition buffer's row ids and
// ordered gradients at positions `begin + p`, or (`identity`) rows `begin + p` themselves with gradients by row.
struct PositionSource {
    const uint32_t* rows;
    const int32_t* gh;
    uint32_t begin;
    bool identity;
};

__device__ __forceinline__ void position_of(const PositionSource& s, uint32_t p, uint32_t& row, uint32_t& packed) {
    const uint32_t pos = s.begin + p;
    if (s.identity) {
        row = pos;
        packed = static_cast<uint32_t>(__ldcs(s.gh + pos));
    } else {
        row = __ldcg(s.rows + pos);  // written by a partition of the same stream: not through the read-only path
        packed = static_cast<uint32_t>(__ldcg(s.gh + pos));
    }
}

// The lane constants of row-chunk work over a unit's full tiles (its first F tiles: 32 features each, side by side
// in rows of 32 F bytes). A row is 2F chunks of 16 bytes, chunk c holding features 16 (c mod 2) .. of tile c / 2.
// In load g of a batch, lane k takes chunk k mod P of row g R + k / P (P = chunk_period, R = 32 / P rows a load), so
// a warp's load covers R whole rows, where a lane-per-row load of 32 scattered rows touches 32 lines for the same
// bytes. Lane k permutes its 16 bytes by r = k / 2 and at step s adds feature 16 (k mod 2) + (s ^ r) of its chunk's
// tile (chunk c has the parity of k): the 32 atomics of a step hit 32 different feature lanes, i.e. 32 banks.
struct ChunkLane {
    uint32_t r;                      // the byte permutation: lane / 2
    uint32_t addr[kMaxUnitTiles];    // per full tile: shared address of this lane's feature lane 16 (lane mod 2) + r
    uint32_t skip;                   // bit t: full tile t skips stored bin 0 (Tile::skip)
    uint32_t wanted;                 // bit t: full tile t has a wanted feature
};

// `skips`: Tile::skip tiles skip their stored bin 0 (the tree kernel, which recovers those bins from the rows'
// totals); the standalone histogram adds every stored bin and maps the exchanged bins back in its reduction.
__device__ __forceinline__ ChunkLane chunk_lane(const LaneTile* lt, uint32_t nfull, uint32_t lane, bool skips) {
    ChunkLane k;
    k.r = lane >> 1;
    k.skip = 0;
    k.wanted = 0;
    const uint32_t off = 4u * ((lane & 1u) * 16u + k.r);
#pragma unroll
    for (int t = 0; t < kMaxUnitTiles; ++t) {
        k.addr[t] = 0;
        if (t >= static_cast<int>(nfull)) continue;
        const LaneTile l = lt[t];
        k.addr[t] = l.addr | off;  // the tile's array is 128-byte aligned
        if (skips && l.skip) k.skip |= 1u << t;
        if (l.active != 0) k.wanted |= 1u << t;
    }
    return k;
}

// Adds one loaded row of a partial tile (stride 4, 8 or 16) at every feature: add_row by stride; with kSkip, a
// Tile::skip tile adds no stored bin 0.
template <bool kSkip = false>
__device__ __forceinline__ void add_partial_row(const LaneTile& l, const uint32_t (&w)[8], uint32_t packed,
                                                uint32_t lane) {
    const bool skip = kSkip && l.skip;
    switch (l.stride) {
        case 16:
            if (skip) add_row<4, true>(l, w, packed, lane); else add_row<4>(l, w, packed, lane);
            break;
        case 8:
            if (skip) add_row<2, true>(l, w, packed, lane); else add_row<2>(l, w, packed, lane);
            break;
        default:
            if (skip) add_row<1, true>(l, w, packed, lane); else add_row<1>(l, w, packed, lane);
            break;
    }
}

// When lane k's chunk c is the same in every instruction (chunk_period), its tile is fixed and every per-step
// quantity is a lane constant: the step's shared address at bin 0, the byte selector that
// extracts the step's byte (its word swapped into place once per chunk), and whether stored bin 0 adds. An element
// then costs a byte_perm, a multiply-add and the atomic.
struct FixedChunk {
    uint32_t off[16];   // step s: shared address of feature 16 (lane mod 2) + (s ^ r) of the lane's tile at bin 0
    uint32_t bsel[4];   // step s: __byte_perm selector of byte (s ^ r) mod 4 (zero-extended)
    uint32_t wq;        // r / 4: the chunk's words are swapped by it (word j to j ^ wq)
    bool skip;          // the lane's tile skips stored bin 0 (Tile::skip, tree kernel only)
    bool on;            // the lane's tile has a wanted feature
};

__device__ __forceinline__ FixedChunk fixed_chunk(const ChunkLane& k, uint32_t t) {
    FixedChunk f;
    const uint32_t base = k.addr[0] * (t == 0) + k.addr[1] * (t == 1) + k.addr[2] * (t == 2) + k.addr[3] * (t == 3);
#pragma unroll
    for (int s = 0; s < 16; ++s) f.off[s] = base ^ (4u * s);
#pragma unroll
    for (int q = 0; q < 4; ++q) f.bsel[q] = ((static_cast<uint32_t>(q) ^ k.r) & 3u) | 0x4440u;
    f.wq = k.r >> 2;
    f.skip = (k.skip >> t) & 1u;
    f.on = (k.wanted >> t) & 1u;
    return f;
}

// One lane's 16 bytes of its fixed tile added at their features; kSkip: stored bin 0 adds nothing where f.skip.
template <bool kSkip>
__device__ __forceinline__ void add_fixed(const FixedChunk& f, uint4 v, uint32_t packed) {
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
    // word j of the chunk to position j ^ wq
    {
        const bool s1 = f.wq & 1u, s2 = f.wq & 2u;
        uint32_t a = s1 ? w[1] : w[0], b = s1 ? w[0] : w[1], c = s1 ? w[3] : w[2], d = s1 ? w[2] : w[3];
        w[0] = s2 ? c : a;
        w[1] = s2 ? d : b;
        w[2] = s2 ? a : c;
        w[3] = s2 ? b : d;
    }
#pragma unroll
    for (int s = 0; s < 16; ++s) {
        const uint32_t bin = __byte_perm(w[s >> 2], 0u, f.bsel[s & 3]);
        if (kSkip && f.skip)
            shared_add_nonzero(bin * 128u + f.off[s], packed, bin);
        else
            shared_add(bin * 128u + f.off[s], packed);
    }
}

// The lanes' chunk period of F full tiles: 2F chunks a row, except F = 3, whose 6 chunks a row take 8 lanes (the
// last two idle) so that a lane's chunk, and with it its tile, is the same in every instruction.
template <int F>
__host__ __device__ constexpr uint32_t chunk_period() { return F == 3 ? 8u : 2u * F; }

// Whole warp: positions [p_lo, p_hi) of `src` into the unit's shared sums, in batches of 32 positions: the F full
// tiles in row chunks, R = 32 / P rows an instruction (P = chunk_period), lane k taking chunk k mod P of row k / P
// and adding only its own tile (FixedChunk); a partial tile `lp` (when `partial`) lane per row. Lane k loads
// position k's row and packed gradient one batch ahead; a chunk's row and gradient come from the lane that loaded
// them.
template <int F, bool kSkip = false>
__device__ __forceinline__ void hist_rows(const LaneTile* lt, bool partial, const PositionSource& src,
                                          uint32_t p_lo, uint32_t p_hi, uint32_t lane, int* tg = nullptr,
                                          int* th = nullptr) {
    constexpr uint32_t C = chunk_period<F>(), R = 32 / C;
    const ChunkLane k = chunk_lane(lt, F, lane, kSkip);
    const uint32_t c = lane % C;
    const FixedChunk f = fixed_chunk(k, c >> 1);  // with F = 3, lanes of chunks 6 and 7 are off (no tile 3)
    const LaneTile lp = lt[partial ? F : 0];
    const uint8_t* chunk = lt[0].base + 16 * c;
    const uint32_t pitch = lt[0].pitch;
    auto position = [&](uint32_t p, uint32_t& row, uint32_t& packed) {
        row = 0;
        packed = 0;
        if (p < p_hi) {
            position_of(src, p, row, packed);
            if (tg != nullptr) {  // the rows' totals (quantize.rs:140-143), for the recovery of skipped bins
                const int g = static_cast<int16_t>(packed & 0xFFFFu);
                *tg += g;
                *th += static_cast<int>((packed - static_cast<uint32_t>(g)) >> 16);
            }
        }
    };
    uint32_t next_row, next_packed;
    position(p_lo + lane, next_row, next_packed);
    for (uint32_t p0 = p_lo; p0 < p_hi; p0 += 32) {
        const uint32_t row = next_row, packed = next_packed;
        uint4 v[C];
        uint32_t pk[C];
#pragma unroll
        for (uint32_t g = 0; g < C; ++g) {
            const int src_lane = static_cast<int>(g * R + lane / C);
            const uint32_t rw = __shfl_sync(0xffffffffu, row, src_lane);
            pk[g] = __shfl_sync(0xffffffffu, packed, src_lane);
            v[g] = make_uint4(0, 0, 0, 0);
            if (pk[g] != 0 && f.on) v[g] = __ldcs(reinterpret_cast<const uint4*>(chunk + static_cast<uint64_t>(rw) * pitch));
        }
        uint32_t wp[8] = {};
        if (partial && packed != 0) load_row(lp, row, wp);
        position(p0 + 32 + lane, next_row, next_packed);
#pragma unroll
        for (uint32_t g = 0; g < C; ++g)
            if (pk[g] != 0 && f.on) add_fixed<kSkip>(f, v[g], pk[g]);
        if (partial && packed != 0) add_partial_row<kSkip>(lp, wp, packed, lane);
    }
}

// The unit of histogram CTA `cta`.
__device__ __forceinline__ uint32_t unit_of_cta(const HistArgs& a, uint32_t cta) {
    uint32_t ui = 0;
    while (ui + 1 < a.num_units && cta >= a.units[ui + 1].cta_begin) ++ui;
    return ui;
}

// The first 128-byte boundary of the dynamic shared memory `sh`: where the histogram starts (the callers reserve
// kHistAlign more bytes).
__device__ __forceinline__ uint32_t hist_shared_base(const int* sh) {
    const uint32_t raw = static_cast<uint32_t>(__cvta_generic_to_shared(sh));
    return (raw + kHistAlign - 1) & ~(kHistAlign - 1);
}

// What a histogram CTA does not relearn per job: its unit, the unit's tiles as the lanes use them (`active` 0;
// the job sets its own bits), and each tile lane's feature. Kept in shared memory; the persistent tree kernel
// fills it once per launch.
struct HistCta {
    Unit unit;
    LaneTile tiles[kMaxUnitTiles];
    int32_t lane_feature[kMaxUnitTiles][kTileLanes];
};

// Fills `c` for unit `u` (whole CTA; `sh` is the dynamic shared memory the histogram will use).
inline __device__ void histogram_prepare_unit(const HistArgs& a, uint32_t u, const int* sh, HistCta* c) {
    __syncthreads();  // every thread is done with the previous contents
    if (threadIdx.x == 0) c->unit = a.units[u];
    __syncthreads();
    const Unit unit = c->unit;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (warp < unit.num_tiles) {
        c->lane_feature[warp][lane] = a.d.lane_feature[(unit.first_tile + warp) * kTileLanes + lane];
        if (lane == 0) {
            // words before tile `warp`: every tile's array is B S words (B >= 64, so 256-word multiples)
            uint32_t slot = 0;
            for (uint32_t t = 0; t < warp; ++t) {
                const Tile prev = a.d.tiles[unit.first_tile + t];
                slot += prev.smem_bins * prev.stride;
            }
            const Tile tile = a.d.tiles[unit.first_tile + warp];
            LaneTile lt;
            lt.base = a.d.bins + tile.base;
            lt.stride = tile.stride;
            lt.bins = tile.smem_bins;
            lt.addr = hist_shared_base(sh) + 4 * slot;
            lt.active = 0;
            lt.stage_off = 0;
            lt.pitch = tile.pitch;
            lt.skip = tile.skip;
            lt.pad_ = 0;
            c->tiles[warp] = lt;
        }
    }
    __syncthreads();
}

// Fills `c` for the unit of histogram CTA `cta` (the standalone kernels: one unit per CTA).
inline __device__ void histogram_prepare_cta(const HistArgs& a, uint32_t cta, const int* sh, HistCta* c) {
    histogram_prepare_unit(a, unit_of_cta(a, cta), sh, c);
}

// Unpacks the packed shared histogram `sh` of the unit into the CTA's slab: per tile, its slots' g into the slab's
// gradient array and h into its hessian array (at twice the packed offset; see QuadMeta), stored when `first`, added
// otherwise; the shared slots are cleared for the next round when `clear`. Four slots per thread and step.
__device__ __forceinline__ void flush_packed(const HistCta& c, int4* sh, uint32_t sh_addr, int* slab, bool first,
                                             bool clear) {
    const uint32_t quads = c.unit.slots / 4;
    constexpr int kQuads = 4;  // quads per thread in flight: their slab reads overlap
    for (uint32_t i0 = threadIdx.x; i0 < quads; i0 += kQuads * kHistThreads) {
        int4 g[kQuads], h[kQuads];
        int4* gs[kQuads];
        int4* hs[kQuads];
#pragma unroll
        for (int j = 0; j < kQuads; ++j) {
            const uint32_t i = i0 + j * kHistThreads;
            gs[j] = hs[j] = nullptr;
            if (i >= quads) continue;
            // the tile of quad i, and its place in the slab
            uint32_t t = 0, s = 4 * i;
            uint32_t p = (c.tiles[0].addr - sh_addr) / 4, n = c.tiles[0].bins * c.tiles[0].stride;
            while (s >= p + n) {
                ++t;
                p = (c.tiles[t].addr - sh_addr) / 4;
                n = c.tiles[t].bins * c.tiles[t].stride;
            }
            const int4 v = sh[i];
            // unpack (quantize.rs:140-143): g is the low half sign-extended, h what remains above it
            g[j] = make_int4(static_cast<int16_t>(v.x & 0xFFFF), static_cast<int16_t>(v.y & 0xFFFF),
                             static_cast<int16_t>(v.z & 0xFFFF), static_cast<int16_t>(v.w & 0xFFFF));
            h[j] = make_int4(static_cast<int>(static_cast<uint32_t>(v.x - g[j].x) >> 16),
                             static_cast<int>(static_cast<uint32_t>(v.y - g[j].y) >> 16),
                             static_cast<int>(static_cast<uint32_t>(v.z - g[j].z) >> 16),
                             static_cast<int>(static_cast<uint32_t>(v.w - g[j].w) >> 16));
            gs[j] = reinterpret_cast<int4*>(slab + p + s);  // 2 p + (s - p): the tile's gradient array
            hs[j] = reinterpret_cast<int4*>(slab + p + n + s);
            if (clear) sh[i] = make_int4(0, 0, 0, 0);
        }
        if (!first) {
            int4 og[kQuads], oh[kQuads];
#pragma unroll
            for (int j = 0; j < kQuads; ++j) {
                og[j] = gs[j] ? __ldcg(gs[j]) : make_int4(0, 0, 0, 0);
                oh[j] = hs[j] ? __ldcg(hs[j]) : make_int4(0, 0, 0, 0);
            }
#pragma unroll
            for (int j = 0; j < kQuads; ++j) {
                g[j] = make_int4(g[j].x + og[j].x, g[j].y + og[j].y, g[j].z + og[j].z, g[j].w + og[j].w);
                h[j] = make_int4(h[j].x + oh[j].x, h[j].y + oh[j].y, h[j].z + oh[j].z, h[j].w + oh[j].w);
            }
        }
#pragma unroll
        for (int j = 0; j < kQuads; ++j) {
            if (gs[j] == nullptr) continue;
            __stcg(gs[j], g[j]);
            __stcg(hs[j], h[j]);
        }
    }
}

// CTA `cta`'s share of `job`: its unit's rows of its chunk into shared memory, then into its slab, in rounds of at
// most `round_rows` rows (packed_round_rows of the job's quantization; at least kMinRoundRows). Needs kHistThreads
// threads and the CTA's prepared `c`; returns without touching the slab when the CTA has no chunk.
inline __device__ void histogram_cta(const HistArgs& a, const HistJob& job, uint32_t cta, int* sh, const HistCta& c,
                                     uint32_t round_rows) {
    if (!job.active || job.count == 0) return;
    const Unit unit = c.unit;
    const uint32_t chunk = cta - unit.cta_begin;
    const uint32_t chunks = unit_chunks(unit, job.count, a.min_rows_per_cta);
    if (chunk >= chunks) return;
    const uint32_t lo = static_cast<uint32_t>(static_cast<uint64_t>(job.count) * chunk / chunks);
    uint32_t hi = static_cast<uint32_t>(static_cast<uint64_t>(job.count) * (chunk + 1) / chunks);

    const uint32_t sh_addr = hist_shared_base(sh);
    sh += (sh_addr - static_cast<uint32_t>(__cvta_generic_to_shared(sh))) / 4;
    {
        int4* z = reinterpret_cast<int4*>(sh);
        for (uint32_t i = threadIdx.x; i < unit.slots / 4; i += kHistThreads) z[i] = make_int4(0, 0, 0, 0);
    }
    int* slab = a.slabs + static_cast<size_t>(cta) * a.slab_ints;

    const uint32_t lane = threadIdx.x & 31;
    const uint32_t warp = threadIdx.x >> 5;
    constexpr uint32_t kWarps = kHistThreads / 32;
    // The unit's tiles with this job's wanted features (one bit per lane; warp t reads tile t's), in shared memory:
    // read per tile per batch, broadcast.
    __shared__ LaneTile s_lt[kMaxUnitTiles];
    const uint32_t num_tiles = unit.num_tiles;
    if (warp < num_tiles) {
        const int32_t f = c.lane_feature[warp][lane];
        const bool on = f >= 0 && (a.active == nullptr || __ldcg(a.active + f) != 0);
        const uint32_t bits = __ballot_sync(0xffffffffu, on);
        if (lane == 0) {
            LaneTile lt = c.tiles[warp];
            lt.active = bits;
            s_lt[warp] = lt;
        }
    }
    __syncthreads();
    uint32_t any = 0;
    for (uint32_t t = 0; t < num_tiles; ++t) any |= s_lt[t].active;
    if (any == 0) hi = lo;  // nothing wanted: one flush of zeros

    const uint32_t* rows = a.rows[job.which & 1];
    const int32_t* ordered = a.ordered[job.which & 1];
    const PositionSource src{rows, job.identity ? a.packed : ordered, job.begin, job.identity != 0};
    // The unit's leading full tiles (and a partial tile after them) go through hist_rows; a unit of one partial tile
    // through the lane-per-row loop below.
    uint32_t nfull = 0;
    while (nfull < num_tiles && s_lt[nfull].stride == 32) ++nfull;
    int4* sh4 = reinterpret_cast<int4*>(sh);
    uint32_t r0 = lo;
    do {
        const uint32_t r1 = min(hi, r0 + round_rows);
        const uint32_t span = r1 - r0;
        const uint32_t per_warp = static_cast<uint32_t>(ceil_div(ceil_div(span, kWarps), 32) * 32);
        const uint32_t w_lo = r0 + min(span, per_warp * warp);
        const uint32_t w_hi = r0 + min(span, per_warp * (warp + 1));
        // The row and packed gradient of position p (0 past the warp's range).
        auto position = [&](uint32_t p, uint32_t& row, int32_t& packed) {
            row = 0;
            packed = 0;
            if (p < w_hi) {
                uint32_t pk;
                position_of(src, p, row, pk);
                packed = static_cast<int32_t>(pk);
            }
        };
        const bool partial = nfull < num_tiles && s_lt[nfull].active != 0;
        if (w_lo < w_hi) {
            switch (nfull) {
                case 1: hist_rows<1>(s_lt, partial, src, w_lo, w_hi, lane); break;
                case 2: hist_rows<2>(s_lt, partial, src, w_lo, w_hi, lane); break;
                case 3: hist_rows<3>(s_lt, partial, src, w_lo, w_hi, lane); break;
                case 4: hist_rows<4>(s_lt, partial, src, w_lo, w_hi, lane); break;
                default: break;
            }
        }
        if (w_lo < w_hi && nfull == 0 && s_lt[0].active != 0) {
            // a unit of one partial tile (the dataset's last): lane per row
            uint32_t next_row;
            int32_t next_packed;
            position(w_lo + lane, next_row, next_packed);
            for (uint32_t p0 = w_lo; p0 < w_hi; p0 += 32) {
                const uint32_t row = next_row;
                const uint32_t packed = static_cast<uint32_t>(next_packed);
                uint32_t w[8] = {};
                if (packed != 0) load_row(s_lt[0], row, w);
                position(p0 + 32 + lane, next_row, next_packed);
                if (packed != 0) add_partial_row(s_lt[0], w, packed, lane);  // a zero row adds nothing
            }
        }
        __syncthreads();
        flush_packed(c, sh4, sh_addr, slab, r0 == lo, r1 < hi);
        __syncthreads();
        r0 = r1;
    } while (r0 < hi);
}

// The output must hold zeros in the wanted features' bins before a direct histogram (histogram_goes_direct).

__device__ __forceinline__ void global_add_pair(int* p, int32_t g, int32_t h) {
    asm volatile(
        "red.global.add.s32 [%0], %1;\n\t"
        "red.global.add.s32 [%0+4], %2;" ::"l"(p),
        "r"(g), "r"(h)
        : "memory");
}

// One loaded row of a tile of `W` words into the output: step i adds feature i ^ (lane mod S), as in add_row.
// `off_lane` is the output bin offset of feature lane `lane` (-1: not wanted) and `mfb_lane` its DevFeature::mfb
// (its tile bytes 0 and mfb trade places); rows with `add` false only take part in the shuffles.
template <int W>
__device__ __forceinline__ void direct_row(int* out, const uint32_t (&wrow)[8], int32_t off_lane, uint32_t mfb_lane,
                                           int32_t g, int32_t h, bool add, uint32_t lane) {
    constexpr uint32_t kStride = 4 * W;
    uint32_t w[W];
#pragma unroll
    for (int j = 0; j < W; ++j) w[j] = wrow[j];
    const uint32_t k = lane & (kStride - 1);
    xor_bytes<W>(w, k);
#pragma unroll
    for (int i = 0; i < static_cast<int>(kStride); ++i) {
        const int32_t off = __shfl_sync(0xffffffffu, off_lane, static_cast<int>(i ^ k));
        const uint32_t mfb = __shfl_sync(0xffffffffu, mfb_lane, static_cast<int>(i ^ k));
        const uint32_t bin = swap_dominant((w[i >> 2] >> (8 * (i & 3))) & 0xFFu, mfb);
        if (add && off >= 0) global_add_pair(out + 2 * (static_cast<uint32_t>(off) + bin), g, h);
    }
}

// CTA `cta` of `ctas`'s share of a direct job: warp items are (32-position batch, tile), the tiles of one batch on
// consecutive warps.
inline __device__ void histogram_direct_cta(const HistArgs& a, const HistJob& job, uint32_t cta, uint32_t ctas) {
    if (!job.active || job.count == 0) return;
    const uint32_t lane = threadIdx.x & 31;
    constexpr uint32_t kWarps = kHistThreads / 32;
    const uint32_t gwarp = cta * kWarps + (threadIdx.x >> 5), gwarps = ctas * kWarps;
    const uint32_t T = a.d.num_tiles;
    const uint32_t items = static_cast<uint32_t>(ceil_div(job.count, 32)) * T;
    const uint32_t* rows = a.rows[job.which & 1];
    const int32_t* ordered = a.ordered[job.which & 1];
    for (uint32_t item = gwarp; item < items; item += gwarps) {
        const uint32_t t = item % T, p = (item / T) * 32 + lane;
        uint32_t row = 0;
        int32_t packed = 0;
        if (p < job.count) {
            const uint32_t pos = job.begin + p;
            if (job.identity) {
                row = pos;
                packed = __ldg(a.packed + pos);
            } else {
                row = __ldcg(rows + pos);
                packed = __ldcg(ordered + pos);
            }
        }
        const int32_t f = a.d.lane_feature[t * kTileLanes + lane];
        int32_t off = -1;
        uint32_t mfb = 0;
        if (f >= 0 && (a.active == nullptr || __ldcg(a.active + f) != 0)) {
            off = static_cast<int32_t>(a.d.features[f].hist_offset);
            mfb = a.d.features[f].mfb & 0xFFu;
        }
        if (__ballot_sync(0xffffffffu, off >= 0) == 0) continue;  // no wanted feature in the tile
        const Tile tile = a.d.tiles[t];
        LaneTile lt;
        lt.base = a.d.bins + tile.base;
        lt.stride = tile.stride;
        lt.pitch = tile.pitch;
        uint32_t wd[8];
        load_row(lt, row, wd);  // row 0 for positions past the job: in bounds, and adds nothing
        // unpack (quantize.rs:140-143)
        const int32_t g = static_cast<int16_t>(static_cast<uint16_t>(static_cast<uint32_t>(packed)));
        const int32_t h = (packed - g) >> 16;
        const bool add = packed != 0;
        switch (tile.stride) {
            case 32:
                direct_row<8>(a.out, wd, off, mfb, g, h, add, lane);
                break;
            case 16:
                direct_row<4>(a.out, wd, off, mfb, g, h, add, lane);
                break;
            case 8:
                direct_row<2>(a.out, wd, off, mfb, g, h, add, lane);
                break;
            default:
                direct_row<1>(a.out, wd, off, mfb, g, h, add, lane);
                break;
        }
    }
}

__device__ __forceinline__ int4 add4(int4 x, int4 y) { return make_int4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w); }

__device__ __forceinline__ int4 shfl_xor4(int4 v, int o) {
    return make_int4(__shfl_xor_sync(0xffffffffu, v.x, o), __shfl_xor_sync(0xffffffffu, v.y, o),
                     __shfl_xor_sync(0xffffffffu, v.z, o), __shfl_xor_sync(0xffffffffu, v.w, o));
}

// The slab reduction, thread `thread` of `threads` (a multiple of 32): quad q's sums over the chunks of its unit
// that took part are split over a.quad_split consecutive lanes (lane j of the group adds chunks j, j + split, ...,
// with 128-bit loads, four chunks in flight), combined by shuffles, and the group's first lane writes the quad's
// four [g, h] pairs. Every feature's bins are written, wanted or not (bins of unwanted features may hold anything).
inline __device__ void histogram_reduce_quads(const HistArgs& a, const HistJob& job, uint32_t thread,
                                              uint32_t threads) {
    if (!job.active || job.count == 0) return;
    const uint32_t split = a.quad_split;
    const uint32_t j = thread & (split - 1);
    const uint32_t groups = threads / split;
    // every lane of a warp runs the same number of iterations: the shuffles need the whole warp
    const uint32_t rounds = static_cast<uint32_t>(ceil_div(a.num_quads, groups));
    for (uint32_t r = 0; r < rounds; ++r) {
        const uint32_t q = r * groups + thread / split;
        int4 g = make_int4(0, 0, 0, 0), h = g;
        QuadMeta m{};
        const bool mine = q < a.num_quads;
        if (mine) {
            m = a.quads[q];
            const Unit unit = a.units[m.unit];
            const uint32_t chunks = unit_chunks(unit, job.count, a.min_rows_per_cta);
            const int* slab0 = a.slabs + static_cast<size_t>(unit.cta_begin) * a.slab_ints;
            for (uint32_t c0 = j; c0 < chunks; c0 += 4 * split) {
                int4 vg[4], vh[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t c = c0 + k * split;
                    const int* slab = slab0 + static_cast<size_t>(c) * a.slab_ints;
                    vg[k] = c < chunks ? __ldcg(reinterpret_cast<const int4*>(slab + m.g_off)) : make_int4(0, 0, 0, 0);
                    vh[k] = c < chunks ? __ldcg(reinterpret_cast<const int4*>(slab + m.h_off)) : make_int4(0, 0, 0, 0);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    g = add4(g, vg[k]);
                    h = add4(h, vh[k]);
                }
            }
        }
        for (uint32_t o = split >> 1; o > 0; o >>= 1) {
            g = add4(g, shfl_xor4(g, static_cast<int>(o)));
            h = add4(h, shfl_xor4(h, static_cast<int>(o)));
        }
        if (mine && j == 0) {
            int2* out = reinterpret_cast<int2*>(a.out);
            if (m.out[0] >= 0) __stcg(out + m.out[0], make_int2(g.x, h.x));
            if (m.out[1] >= 0) __stcg(out + m.out[1], make_int2(g.y, h.y));
            if (m.out[2] >= 0) __stcg(out + m.out[2], make_int2(g.z, h.z));
            if (m.out[3] >= 0) __stcg(out + m.out[3], make_int2(g.w, h.w));
        }
    }
}

}  // namespace sb2
