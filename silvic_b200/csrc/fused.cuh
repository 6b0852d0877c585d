// fused.cuh — the persistent tree kernel's split step: the parent's partition and the built child's histogram as
// one phase, then the slab reduction (CpuBackend::partition_and_histogram, crates/silvic-core/src/backend/mod.rs:
// 154-168, with stable_partition, backend/cpu.rs:556-599, and the quantized histogram, :838-864).
//
// The trainer never depends on the order of rows inside a leaf: every histogram and leaf sum is an integer sum and
// every score update is per row, so any order grows the same tree. (The Backend API's sb2_partition keeps the
// reference's stable order: partition.cuh.) The kernel therefore places rows without a grid-wide prefix. Each CTA
// of the step takes a range of the parent's positions, counts its lefts and rights, reserves room for them with one
// atomic per side on the step's cursors (lefts fill the parent's range from its start, rights from its end) and
// scatters its rows into the other partition buffer; in the same pass it adds its rows that go to the built child
// into its shared histogram, unit by unit, and flushes that to its slab. The grid meets once, after which the slabs
// are reduced and the children searched.
//
// A CTA's packed shared sums are exact for at most `round_rows` rows (packed_round_rows); when its range is that
// short it flushes the packed sums as they are (half the bytes) and the reduction unpacks them, else it flushes
// unpacked sums every round.
#pragma once

#include "hist_device.cuh"
#include "partition.cuh"

namespace sb2 {

constexpr uint32_t kFusedMinRows = 1024;  // parent positions per CTA at the least: small leaves use fewer CTAs
constexpr uint32_t kFusedScanWords = kHistThreads;  // words per scatter round: one per thread of the CTA scan

// CTAs that take part in a phase over `count` positions, and CTA `cta`'s range [lo, hi) of them (whole words of
// 32 positions; every taking part CTA has at least one).
__host__ __device__ __forceinline__ uint32_t fused_chunks(uint32_t count, uint32_t ctas) {
    const uint64_t c = ceil_div(count, kFusedMinRows);
    const uint64_t words = ceil_div(count, 32);
    uint64_t n = c < 1 ? 1 : c;
    n = n > ctas ? ctas : n;
    return static_cast<uint32_t>(n > words && words > 0 ? words : n);
}

__device__ __forceinline__ void fused_range(uint32_t count, uint32_t chunks, uint32_t cta, uint32_t& lo,
                                            uint32_t& hi) {
    const uint64_t words = ceil_div(count, 32);
    lo = static_cast<uint32_t>(min(static_cast<uint64_t>(count), 32 * (words * cta / chunks)));
    hi = static_cast<uint32_t>(min(static_cast<uint64_t>(count), 32 * (words * (cta + 1) / chunks)));
}

// Whether the slabs of a phase over `count` positions hold packed sums: every CTA's range fits one packed round.
__host__ __device__ __forceinline__ bool fused_packed(uint32_t count, uint32_t chunks, uint32_t round_rows) {
    return 32 * ceil_div(ceil_div(count, 32), chunks) <= round_rows;
}

// One 32-row batch of a warp into the unit's packed shared arrays (`lt`: its tiles with the wanted bits): lane k's
// row adds `packed` (0: nothing) at every tile, each tile's bytes loaded one tile ahead.
__device__ __forceinline__ void add_batch(const LaneTile* lt, uint32_t num_tiles, uint32_t row, uint32_t packed,
                                          uint32_t lane) {
    uint32_t cur[8] = {}, nxt[8] = {};
    if (packed != 0 && lt[0].active != 0) load_row(lt[0], row, cur);
#pragma unroll
    for (int t = 0; t < kMaxUnitTiles; ++t) {
        if (t >= static_cast<int>(num_tiles)) break;
        if (packed != 0 && t + 1 < static_cast<int>(num_tiles) && lt[t + 1].active != 0) load_row(lt[t + 1], row, nxt);
        const LaneTile l = lt[t];
        if (packed != 0 && l.active != 0) {
            switch (l.stride) {
                case 32:
                    add_row<8>(l, cur, packed, lane);
                    break;
                case 16:
                    add_row<4>(l, cur, packed, lane);
                    break;
                case 8:
                    add_row<2>(l, cur, packed, lane);
                    break;
                default:
                    add_row<1>(l, cur, packed, lane);
                    break;
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
    }
}

// The unit's tiles with the wanted features' bits into `lt` (shared), its packed arrays cleared. Whole CTA; returns
// whether the unit has a wanted feature.
__device__ __forceinline__ bool fused_unit_begin(const HistCta& c, const uint8_t* active, int4* sh4, LaneTile* lt) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (uint32_t i = threadIdx.x; i < c.unit.slots / 4; i += kHistThreads) sh4[i] = make_int4(0, 0, 0, 0);
    if (warp < c.unit.num_tiles) {
        const int32_t f = c.lane_feature[warp][lane];
        const bool on = f >= 0 && (active == nullptr || load_flag(active + f) != 0);
        const uint32_t bits = __ballot_sync(0xffffffffu, on);
        if (lane == 0) {
            LaneTile l = c.tiles[warp];
            l.active = bits;
            lt[warp] = l;
        }
    }
    __syncthreads();
    uint32_t any = 0;
    for (uint32_t t = 0; t < c.unit.num_tiles; ++t) any |= lt[t].active;
    return any != 0;
}

// The unit's shared sums into the CTA's slab: packed as they are (`packed`: the slab region is one int per slot) or
// unpacked (stored when `first`, added otherwise); cleared for another round when `clear`. Whole CTA.
__device__ __forceinline__ void fused_unit_flush(const HistCta& c, int4* sh4, uint32_t sh_addr, int* slab_unit,
                                                 bool packed, bool first, bool clear) {
    __syncthreads();
    if (packed) {
        int4* dst = reinterpret_cast<int4*>(slab_unit);
        for (uint32_t i = threadIdx.x; i < c.unit.slots / 4; i += kHistThreads) __stcg(dst + i, sh4[i]);
    } else {
        flush_packed(c, sh4, sh_addr, slab_unit, first, clear);
    }
    __syncthreads();
}

// What a step's phase needs besides the kernel arguments.
struct FusedStep {
    uint32_t count;       // the parent's positions (the root: every row)
    uint32_t begin;       // the parent's first position
    uint32_t src, dst;    // partition buffers read and written
    uint32_t chunks;      // CTAs taking part
    bool root;            // identity rows, no partition: every row is built
    bool built_left;      // the histogram is of the left child
    bool histogram;       // the built child's histogram is wanted (else only the partition runs)
    bool packed;          // slabs hold packed sums
    uint32_t round_rows;  // rows per packed round
};

// CTA `cta`'s part of a step (kHistThreads threads): for a split, the partition of its range of the parent into
// the other buffer and, for every unit, its built-child rows into the unit's slab region. `scan` is 2 kHistThreads
// + 64 words of shared memory apart from the histogram's; `cursor` the step's two placement counters (zero before
// the step); `units` the prepared unit descriptions (`cached` of them; later units are prepared into `spare`).
inline __device__ void fused_step_cta(const TrainArgs& a, const HistArgs& h, const Step& st, const FusedStep& fs,
                                      uint32_t cta, int* sh, uint32_t* scan, unsigned int* cursor,
                                      const uint8_t* active, HistCta* units, uint32_t cached, HistCta* spare) {
    if (cta >= fs.chunks) return;
    uint32_t lo, hi;
    fused_range(fs.count, fs.chunks, cta, lo, hi);
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr uint32_t kWarps = kHistThreads / 32;
    const uint32_t* rows_in = a.rows[fs.src] + fs.begin;
    const int32_t* gh_in = a.ordered[fs.src] + fs.begin;
    uint32_t* rows_out = a.rows[fs.dst] + fs.begin;
    int32_t* gh_out = a.ordered[fs.dst] + fs.begin;
    uint32_t* words = scan + kHistThreads;       // a round's flag words
    uint32_t* sums = scan + 2 * kHistThreads;    // per-warp sums, then the round total
    __shared__ uint32_t s_base[2];

    // Pass 1 (splits): the flags of the CTA's words, kept in the flag buffer, and its left count.
    const uint32_t w_lo = lo / 32, w_hi = static_cast<uint32_t>(ceil_div(hi, 32));
    if (!fs.root) {
        const Tile tile = a.d.tiles[st.split_tile];
        const uint8_t* column = a.d.bins + tile.base + st.split_lane;
        uint32_t mine = 0;
        constexpr int kBatch = 4;
        for (uint32_t w0 = w_lo + warp; w0 < w_hi; w0 += kBatch * kWarps) {
            uint32_t row[kBatch];
            bool valid[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const uint32_t w = w0 + j * kWarps, p = w * 32 + lane;
                valid[j] = w < w_hi && p < hi;
                row[j] = valid[j] ? __ldcg(rows_in + p) : 0u;
            }
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const uint32_t w = w0 + j * kWarps;
                if (w >= w_hi) break;  // warp-uniform
                const bool left = valid[j] && bin_goes_left(st.left_bins, __ldg(column + static_cast<uint64_t>(row[j]) * tile.stride));
                const uint32_t word = __ballot_sync(0xffffffffu, left);
                if (lane == 0) a.flags[w] = word;
                mine += __popc(word);
            }
        }
        if (lane == 0) sums[warp] = mine;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t left = 0;
            for (uint32_t k = 0; k < kWarps; ++k) left += sums[k];
            // One atomic per side: this CTA's lefts and rights go to [base_l, base_l + left) from the parent's
            // start and to the `right` positions ending `base_r` before the parent's end.
            s_base[0] = atomicAdd(cursor, left);
            s_base[1] = atomicAdd(cursor + 1, (hi - lo) - left);
        }
        __syncthreads();
    }

    // Pass 2, per unit: the histogram of the built rows (and, with the first unit, the scatter), in rounds.
    const uint32_t sh_addr = hist_shared_base(sh);
    int4* sh4 = reinterpret_cast<int4*>(sh + (sh_addr - static_cast<uint32_t>(__cvta_generic_to_shared(sh))) / 4);
    __shared__ LaneTile s_lt[kMaxUnitTiles];
    int* slab = h.slabs + static_cast<size_t>(cta) * h.slab_ints;
    uint32_t region = 0;  // ints before this unit's slab region
    const uint32_t round_words = min(kFusedScanWords, max(1u, fs.round_rows / 32));
    for (uint32_t u = 0; u < h.num_units; ++u) {
        if (!fs.histogram && (fs.root || u > 0)) break;  // nothing more to do without the histogram
        HistCta* c = u < cached ? units + u : spare;
        if (u >= cached) histogram_prepare_unit(h, u, sh, spare);
        const bool want = fs.histogram && fused_unit_begin(*c, active, sh4, s_lt);
        const bool scatter = !fs.root && u == 0;
        const uint32_t nt = c->unit.num_tiles;
        uint32_t carry = 0;  // lefts of the CTA's earlier rounds
        for (uint32_t r0 = w_lo; r0 < w_hi || r0 == w_lo; r0 += round_words) {
            const uint32_t r1 = min(w_hi, r0 + round_words);
            const uint32_t nw = r1 > r0 ? r1 - r0 : 0;
            if (scatter) {
                // The round's word counts, scanned over the CTA (one word per thread).
                const uint32_t word = threadIdx.x < nw ? __ldcg(a.flags + r0 + threadIdx.x) : 0u;
                words[threadIdx.x] = word;
                const uint32_t cnt = __popc(word);
                uint32_t incl = cnt;
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t up = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= static_cast<uint32_t>(o)) incl += up;
                }
                if (lane == 31) sums[warp] = incl;
                __syncthreads();
                if (warp == 0) {
                    const uint32_t v = lane < kWarps ? sums[lane] : 0u;
                    uint32_t vi = v;
                    for (int o = 1; o < 32; o <<= 1) {
                        const uint32_t up = __shfl_up_sync(0xffffffffu, vi, o);
                        if (lane >= static_cast<uint32_t>(o)) vi += up;
                    }
                    if (lane < kWarps) sums[lane] = vi - v;
                    if (lane == 31) sums[32] = vi;
                }
                __syncthreads();
                scan[threadIdx.x] = carry + sums[warp] + incl - cnt;  // the CTA's lefts before this word
                __syncthreads();
            }
            if (want || scatter) {
                // A warp per word: its 32 positions' rows, targets and the built child's histogram.
                for (uint32_t k = warp; k < nw; k += kWarps) {
                    const uint32_t w = r0 + k, p = w * 32 + lane;
                    const bool valid = p < hi;
                    uint32_t row;
                    int32_t gh;
                    if (fs.root) {
                        row = fs.begin + p;
                        gh = valid ? __ldcs(h.packed + row) : 0;
                    } else {
                        row = valid ? __ldcg(rows_in + p) : 0u;
                        gh = valid ? __ldcg(gh_in + p) : 0;
                    }
                    bool built = fs.root;
                    if (!fs.root) {
                        const uint32_t bits = scatter ? words[k] : __ldcg(a.flags + w);
                        const bool left = (bits >> lane) & 1u;
                        built = left == fs.built_left;
                        if (scatter && valid) {
                            const uint32_t lefts = scan[k] + __popc(bits & ((1u << lane) - 1u));
                            const uint32_t rights = (p - lo) - lefts;
                            const uint32_t target = left ? s_base[0] + lefts : fs.count - 1 - (s_base[1] + rights);
                            rows_out[target] = row;
                            gh_out[target] = gh;
                        }
                    }
                    if (want) add_batch(s_lt, nt, row, valid && built ? static_cast<uint32_t>(gh) : 0u, lane);
                }
            }
            if (scatter) {
                carry += sums[32];
                __syncthreads();  // the round's scan and words are read
            }
            // Packed slabs: the whole range fits the packing, one flush at the end. Unpacked: a flush per round
            // (rounds hold at most round_rows positions), stored the first time and added after.
            const bool last = r1 >= w_hi;
            if (fs.histogram && (last || !fs.packed))
                fused_unit_flush(*c, sh4, sh_addr, slab + (fs.packed ? region / 2 : region), fs.packed, r0 == w_lo,
                                 !last);
            if (last) break;
        }
        region += 2 * c->unit.slots;
    }
}

// The step's slab reduction (thread `thread` of `threads`): histogram_reduce_quads over slabs that hold every unit,
// packed or not.
inline __device__ void fused_reduce(const HistArgs& a, uint32_t chunks, bool packed, uint32_t thread,
                                    uint32_t threads) {
    const uint32_t split = a.quad_split;
    const uint32_t j = thread & (split - 1);
    const uint32_t groups = threads / split;
    const uint32_t rounds = static_cast<uint32_t>(ceil_div(a.num_quads, groups));
    for (uint32_t r = 0; r < rounds; ++r) {
        const uint32_t q = r * groups + thread / split;
        int4 g = make_int4(0, 0, 0, 0), hs = g;
        QuadMeta m{};
        const bool mine = q < a.num_quads;
        if (mine) {
            m = a.quads[q];
            for (uint32_t c0 = j; c0 < chunks; c0 += 4 * split) {
                int4 v[4], w[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t c = c0 + k * split;
                    const int* slab = a.slabs + static_cast<size_t>(c) * a.slab_ints;
                    const bool in = c < chunks;
                    if (packed) {
                        v[k] = in ? __ldcg(reinterpret_cast<const int4*>(slab + m.unit_off_packed + m.p_off))
                                  : make_int4(0, 0, 0, 0);
                    } else {
                        v[k] = in ? __ldcg(reinterpret_cast<const int4*>(slab + m.unit_off + m.g_off))
                                  : make_int4(0, 0, 0, 0);
                        w[k] = in ? __ldcg(reinterpret_cast<const int4*>(slab + m.unit_off + m.h_off))
                                  : make_int4(0, 0, 0, 0);
                    }
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (packed) {
                        // unpack (quantize.rs:140-143)
                        const int4 x = v[k];
                        const int4 gx = make_int4(static_cast<int16_t>(x.x & 0xFFFF), static_cast<int16_t>(x.y & 0xFFFF),
                                                  static_cast<int16_t>(x.z & 0xFFFF), static_cast<int16_t>(x.w & 0xFFFF));
                        g = add4(g, gx);
                        hs = add4(hs, make_int4(static_cast<int>(static_cast<uint32_t>(x.x - gx.x) >> 16),
                                                static_cast<int>(static_cast<uint32_t>(x.y - gx.y) >> 16),
                                                static_cast<int>(static_cast<uint32_t>(x.z - gx.z) >> 16),
                                                static_cast<int>(static_cast<uint32_t>(x.w - gx.w) >> 16)));
                    } else {
                        g = add4(g, v[k]);
                        hs = add4(hs, w[k]);
                    }
                }
            }
        }
        for (uint32_t o = split >> 1; o > 0; o >>= 1) {
            g = add4(g, shfl_xor4(g, static_cast<int>(o)));
            hs = add4(hs, shfl_xor4(hs, static_cast<int>(o)));
        }
        if (mine && j == 0) {
            int2* out = reinterpret_cast<int2*>(a.out);
            if (m.out[0] >= 0) __stcg(out + m.out[0], make_int2(g.x, hs.x));
            if (m.out[1] >= 0) __stcg(out + m.out[1], make_int2(g.y, hs.y));
            if (m.out[2] >= 0) __stcg(out + m.out[2], make_int2(g.z, hs.z));
            if (m.out[3] >= 0) __stcg(out + m.out[3], make_int2(g.w, hs.w));
        }
    }
}

}  // namespace sb2
