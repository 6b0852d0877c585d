// fused.cuh — the persistent tree kernel's split step: the parent's partition and the built child's histogram as
// one phase, then the slab reduction (CpuBackend::partition_and_histogram, crates/silvic-core/src/backend/mod.rs:
// 154-168, with stable_partition, backend/cpu.rs:556-599, and the quantized histogram, :838-864).
//
// The trainer never depends on the order of rows inside a leaf: every histogram and leaf sum is an integer sum and
// every score update is per row, so any order grows the same tree. (The Backend API's sb2_partition keeps the
// reference's stable order: partition.cuh.) The kernel therefore places rows without a grid-wide prefix. Each CTA
// of the step takes a range of the parent's positions, counts its lefts and rights, reserves room for them with one
// atomic per side on the step's cursors (lefts fill the parent's range from its start, rights from its end) and
// scatters its rows into the other partition buffer. Its rows of the built child are then one contiguous range of
// that buffer, which the CTA histograms itself, every lane busy, and flushes to its slab. The grid meets once, after
// which the slabs are reduced and the children searched.
//
// The histogram reads its rows' bins straight into registers in row chunks (hist_rows, hist_device.cuh): a warp's
// load covers whole rows, and each warp keeps the next batch's positions in flight while it adds the current one. A
// unit of one partial tile streams its rows through shared memory with cp.async instead, `depth` batches of 32 rows
// in flight per warp.
//
// A CTA's packed shared sums are exact for at most `round_rows` rows (packed_round_rows); when its range is that
// short it flushes the packed sums as they are (half the bytes) and the reduction unpacks them, else it flushes
// unpacked sums every round.
#pragma once

#include "hist_device.cuh"
#include "partition.cuh"
#include "search.cuh"
#include "train.cuh"

namespace sb2 {

constexpr uint32_t kFusedMinRows = 512;   // parent positions per CTA at the least: small leaves use fewer CTAs
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

// Shared-memory accesses by 32-bit shared address.
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) { asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v)); }

// Whether the slabs of a phase over `count` positions hold packed sums: every CTA's range fits one packed round.
__host__ __device__ __forceinline__ bool fused_packed(uint32_t count, uint32_t chunks, uint32_t round_rows) {
    const uint32_t words = (count >> 5) + ((count & 31u) != 0);  // 32-bit: a divide per split per step
    return (words + chunks - 1) / chunks <= round_rows / 32;
}

// add_row for one tile of the tree kernel: a Tile::skip tile adds no stored bin 0 (the features' dominant bins,
// recovered from the rows' totals by recover_dominant_bins).
template <int W>
__device__ __forceinline__ void add_row_tile(const LaneTile& l, const uint32_t (&w)[8], uint32_t packed, uint32_t lane) {
    if (l.skip)
        add_row<W, true>(l, w, packed, lane);
    else
        add_row<W, false>(l, w, packed, lane);
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
                    add_row_tile<8>(l, cur, packed, lane);
                    break;
                case 16:
                    add_row_tile<4>(l, cur, packed, lane);
                    break;
                case 8:
                    add_row_tile<2>(l, cur, packed, lane);
                    break;
                default:
                    add_row_tile<1>(l, cur, packed, lane);
                    break;
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
    }
}

// The unit's tiles with the wanted features' bits into `lt` (shared). Whole CTA; returns whether the unit has a
// wanted feature. The packed arrays are zero already: cleared when the kernel starts and by every flush.
__device__ __forceinline__ bool fused_unit_begin(const HistCta& c, const uint8_t* active, LaneTile* lt) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (warp < c.unit.num_tiles) {
        const int32_t f = c.lane_feature[warp][lane];
        const bool on = f >= 0 && (active == nullptr || load_flag(active + f) != 0);
        const uint32_t bits = __ballot_sync(0xffffffffu, on);
        if (lane == 0) {
            LaneTile l = c.tiles[warp];
            l.active = bits;
            l.stage_off = 0;  // the tile's rows in a staging slot: after the earlier tiles' 32 rows each
            for (uint32_t t = 0; t < warp; ++t) l.stage_off += 32 * c.tiles[t].stride;
            lt[warp] = l;
        }
    }
    __syncthreads();
    uint32_t any = 0;
    for (uint32_t t = 0; t < c.unit.num_tiles; ++t) any |= lt[t].active;
    return any != 0;
}

// The unit's shared sums into the CTA's slab, feature-major: per tile, per lane (feature), the lane's bin slots in a
// row (DevFeature::slab_off), so the reduction reads a feature's bins contiguously. Packed (`packed`): one int per
// bin as it is; unpacked: a [g, h] pair per bin, stored when `first`, added otherwise. The shared sums are left
// cleared. Whole CTA. Per tile, through `stage` (shared, at least 32 (smem_bins + 4) words; 0 when absent): thread i
// reads bins 4q .. 4q+3 of lane i mod S (S = the tile's stride; the lanes of a warp read different banks) and
// stores them lane-major at a pitch of smem_bins + 4 words (eight lanes of a 128-bit store hit 32 banks); then the
// tile's lanes are copied out row by row with coalesced 16-byte stores. Without staging room the quads are stored
// from the first step directly.
__device__ __forceinline__ void fused_unit_flush(const HistCta& c, int* slab_packed, int* slab_pairs, bool packed,
                                                 bool first, uint32_t stage) {
    __syncthreads();
    uint32_t p = 0;  // slots of the unit's earlier tiles
    for (uint32_t t = 0; t < c.unit.num_tiles; ++t) {
        const LaneTile& tile = c.tiles[t];
        const uint32_t S = tile.stride, quads = tile.bins / 4, pitch = tile.bins + 4;
        // Stores the 4 bins of quad q of lane l (packed values v) into the slab.
        auto put = [&](uint32_t l, uint32_t q, const uint4& v) {
            const uint32_t at = p + l * tile.bins + 4 * q;  // the 4 bins' first slot in the feature-major region
            if (packed) {
                __stcg(reinterpret_cast<uint4*>(slab_packed + at), v);
                return;
            }
            // unpack (quantize.rs:140-143): g is the low half sign-extended, h what remains above it
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            int g[4], h[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                g[k] = static_cast<int16_t>(w[k] & 0xFFFFu);
                h[k] = static_cast<int>((w[k] - static_cast<uint32_t>(g[k])) >> 16);
            }
            int4* dst = reinterpret_cast<int4*>(slab_pairs + 2 * at);
            int4 x = make_int4(g[0], h[0], g[1], h[1]), y = make_int4(g[2], h[2], g[3], h[3]);
            if (!first) {
                const int4 ox = __ldcg(dst), oy = __ldcg(dst + 1);
                x = make_int4(x.x + ox.x, x.y + ox.y, x.z + ox.z, x.w + ox.w);
                y = make_int4(y.x + oy.x, y.y + oy.y, y.z + oy.z, y.w + oy.w);
            }
            __stcg(dst, x);
            __stcg(dst + 1, y);
        };
        for (uint32_t i = threadIdx.x; i < quads * S; i += kHistThreads) {
            const uint32_t l = i % S, q = i / S;
            const uint32_t a0 = tile.addr + 4 * (4 * q * S + l);  // bin 4q of lane l
            uint4 v;
            v.x = lds32(a0);
            v.y = lds32(a0 + 4 * S);
            v.z = lds32(a0 + 8 * S);
            v.w = lds32(a0 + 12 * S);
#pragma unroll
            for (int k = 0; k < 4; ++k) sts32(a0 + 4 * k * S, 0u);
            if (stage != 0)
                asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(stage + 4 * (l * pitch + 4 * q)), "r"(v.x),
                             "r"(v.y), "r"(v.z), "r"(v.w));
            else
                put(l, q, v);
        }
        if (stage != 0) {
            __syncthreads();
            for (uint32_t i = threadIdx.x; i < quads * S; i += kHistThreads) {
                const uint32_t l = i / quads, q = i % quads;
                put(l, q, lds128(stage + 4 * (l * pitch + 4 * q)));
            }
            __syncthreads();  // the staging words are free for the next tile
        }
        p += tile.bins * S;
    }
    __syncthreads();
}

// ---- staged histogram rows ---------------------------------------------------------------------------------

// An L2 policy that evicts a histogram's bin rows first: they are read once, and the partition buffers, leaf
// histograms and metadata the next phases read should stay.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, uint64_t pol) {
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint64_t pol) {
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Waits until at most `pending` of the thread's newest copy groups are outstanding (pending < kMaxStageDepth).
__device__ __forceinline__ void cp_async_wait(uint32_t pending) {
    switch (pending) {
        case 0:
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            break;
        case 1:
            asm volatile("cp.async.wait_group 1;" ::: "memory");
            break;
        case 2:
            asm volatile("cp.async.wait_group 2;" ::: "memory");
            break;
        default:
            asm volatile("cp.async.wait_group 3;" ::: "memory");
            break;
    }
}


// Staging slot of a batch (a unit of one partial tile): its 32 rows of `stride` bytes (lane k's row at k * stride),
// then the batch's 32 packed gradients.

// Lane's copies of row `row`'s bytes of partial tile `l` (stride below 32) into slot `slot`.
__device__ __forceinline__ void stage_partial(const LaneTile& l, uint32_t slot, uint32_t row, uint32_t lane,
                                              uint64_t pol) {
    const uint8_t* src = l.base + static_cast<uint64_t>(row) * l.pitch;
    const uint32_t dst = slot + l.stage_off + lane * l.stride;
    switch (l.stride) {
        case 16:
            cp_async16(dst, src, pol);
            break;
        case 8:
            cp_async8(dst, src, pol);
            break;
        default:
            cp_async4(dst, src, pol);
            break;
    }
}

// Adds the lane's staged row of the partial tile `l` (packed gradient `packed`, nonzero).
__device__ __forceinline__ void add_staged_partial(const LaneTile& l, uint32_t slot, uint32_t packed, uint32_t lane) {
    const uint32_t a = slot + l.stage_off + lane * l.stride;
    uint32_t w[8];
    switch (l.stride) {
        case 16: {
            const uint4 x = lds128(a);
            w[0] = x.x, w[1] = x.y, w[2] = x.z, w[3] = x.w;
            add_row_tile<4>(l, w, packed, lane);
            break;
        }
        case 8: {
            const uint2 x = lds64(a);
            w[0] = x.x, w[1] = x.y;
            add_row_tile<2>(l, w, packed, lane);
            break;
        }
        default:
            w[0] = lds32(a);
            add_row_tile<1>(l, w, packed, lane);
            break;
    }
}

// Where a warp's histogram rows come from: positions [b0, b1) of a partition buffer (`rows`, packed gradients `gh`),
// or, with `identity`, rows b0 .. b1 themselves (gh indexed by row).
struct RowSource {
    const uint32_t* rows;
    const int32_t* gh;
    bool identity;
};

// Whole CTA: positions [b0, b1) of `src` into the unit's packed shared arrays (`lt`, `nt` tiles). Warp w takes
// batches w, w + 16, ... of 32 positions; it keeps `depth` of them (<= kMaxStageDepth) in flight in its slots
// (`stage`: the CTA's staging area, `slot_bytes` per slot) and adds the oldest as it lands. With `depth` 0 (no room
// for staging) the lanes load their rows' bytes themselves. With `count`, each lane also adds its positions'
// unpacked gradients to (tg, th): the rows' totals, from which recover_dominant_bins restores skipped bins.
__device__ __forceinline__ void hist_stream(const LaneTile* lt, uint32_t nt, const RowSource& src, uint32_t b0,
                                            uint32_t b1, uint32_t stage, uint32_t slot_bytes, uint32_t depth,
                                            uint64_t pol, bool count, int& tg, int& th) {
    constexpr uint32_t kWarps = kHistThreads / 32;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // A unit with full tiles (and a partial tile after them): each warp a contiguous share of the positions, its
    // rows' bytes loaded straight into registers in row chunks (hist_rows), one batch of 32 positions at a time with
    // the next batch's positions in flight: no staging, so the warp never waits for a copy to land before it adds.
    uint32_t nfull = 0;
    bool skips = false;
    for (uint32_t t = 0; t < nt; ++t) skips = skips || lt[t].skip != 0;
    while (nfull < nt && lt[nfull].stride == 32) ++nfull;
    if (nfull > 0) {
        const bool partial = nfull < nt && lt[nfull].active != 0;
        const uint32_t span = b1 > b0 ? b1 - b0 : 0u;
        const uint32_t per_warp = static_cast<uint32_t>(ceil_div(ceil_div(span, kWarps), 32) * 32);
        const uint32_t w_lo = b0 + min(span, per_warp * warp), w_hi = b0 + min(span, per_warp * (warp + 1));
        if (w_lo >= w_hi) return;
        const PositionSource ps{src.rows, src.gh, 0u, src.identity};
        int* ptg = count ? &tg : nullptr;
        int* pth = count ? &th : nullptr;
        switch (nfull * 2 + (skips ? 1 : 0)) {
            case 2: hist_rows<1, false>(lt, partial, ps, w_lo, w_hi, lane, ptg, pth); break;
            case 3: hist_rows<1, true>(lt, partial, ps, w_lo, w_hi, lane, ptg, pth); break;
            case 4: hist_rows<2, false>(lt, partial, ps, w_lo, w_hi, lane, ptg, pth); break;
            case 5: hist_rows<2, true>(lt, partial, ps, w_lo, w_hi, lane, ptg, pth); break;
            case 6: hist_rows<3, false>(lt, partial, ps, w_lo, w_hi, lane, ptg, pth); break;
            case 7: hist_rows<3, true>(lt, partial, ps, w_lo, w_hi, lane, ptg, pth); break;
            case 8: hist_rows<4, false>(lt, partial, ps, w_lo, w_hi, lane, ptg, pth); break;
            case 9: hist_rows<4, true>(lt, partial, ps, w_lo, w_hi, lane, ptg, pth); break;
            default: break;
        }
        return;
    }
    // A unit of one partial tile (the dataset's last, narrower than 32 features): its rows staged lane per row.
    const uint32_t nb = b1 > b0 ? static_cast<uint32_t>(ceil_div(b1 - b0, 32)) : 0u;
    const uint32_t n = nb > warp ? (nb - warp + kWarps - 1) / kWarps : 0u;  // this warp's batches
    // The row and packed gradient of lane's position in the warp's batch i (packed 0 past the range).
    auto position = [&](uint32_t i, uint32_t& row, uint32_t& packed) {
        const uint32_t p = b0 + 32 * (warp + kWarps * i) + lane;
        row = 0;
        packed = 0;
        if (p < b1) {
            if (src.identity) {
                row = p;
                packed = static_cast<uint32_t>(__ldcs(src.gh + p));
            } else {
                row = __ldcg(src.rows + p);  // written by this step's scatter: not through the read-only path
                packed = static_cast<uint32_t>(__ldcg(src.gh + p));
            }
            if (count) {
                const int g = static_cast<int16_t>(packed & 0xFFFFu);  // quantize.rs:140-143
                tg += g;
                th += static_cast<int>((packed - static_cast<uint32_t>(g)) >> 16);
            }
        }
    };
    if (n == 0) return;
    if (depth == 0) {
        for (uint32_t i = 0; i < n; ++i) {
            uint32_t row, packed;
            position(i, row, packed);
            add_batch(lt, nt, row, packed, lane);
        }
        return;
    }
    const LaneTile& lp = lt[0];  // the unit's one tile
    const uint32_t mine = stage + warp * depth * slot_bytes;
    const uint32_t gh_off = slot_bytes - 128;  // the slot's packed gradients
    uint32_t next_row, next_packed;  // the position of batch `issued`, loaded one issue ahead
    position(0, next_row, next_packed);
    uint32_t issued = 0, issue_slot = 0, use_slot = 0;
    for (uint32_t i = 0; i < n; ++i) {
        while (issued < n && issued < i + depth) {
            const uint32_t slot = mine + issue_slot * slot_bytes;
            sts32(slot + gh_off + 4 * lane, next_packed);
            if (next_packed != 0) stage_partial(lp, slot, next_row, lane, pol);  // a zero gradient adds nothing
            cp_async_commit();
            ++issued;
            issue_slot = issue_slot + 1 == depth ? 0 : issue_slot + 1;
            if (issued < n) position(issued, next_row, next_packed);
        }
        cp_async_wait(issued - i - 1);  // batch i's copies (this lane's own row) have landed
        const uint32_t slot = mine + use_slot * slot_bytes;
        use_slot = use_slot + 1 == depth ? 0 : use_slot + 1;
        const uint32_t packed = lds32(slot + gh_off + 4 * lane);
        if (packed != 0 && lp.active != 0) add_staged_partial(lp, slot, packed, lane);
    }
}

// What a step's phase needs besides the kernel arguments.
struct FusedStep {
    uint32_t count;       // the parent's positions (the root: every row)
    uint32_t begin;       // the parent's first position
    uint32_t src, dst;    // partition buffers read and written
    uint32_t chunks;      // CTAs taking part
    bool root;            // identity rows, no partition: every row is built
    bool identity;        // the parent's rows are its positions (the root leaf's own split)
    bool built_left;      // the histogram is of the left child
    bool histogram;       // the built child's histogram is wanted (else only the partition runs)
    bool packed;          // slabs hold packed sums
    uint32_t round_rows;  // rows per packed round
    uint32_t stage;       // shared address of the CTA's staging slots
    uint32_t slot_bytes;  // bytes per staging slot
    uint32_t depth;       // staging slots per warp (0: no staging)
};

// Part `cta` (of fs.chunks) of a split (kHistThreads threads; the unit histograms' shared arrays zero on entry and
// on return): for a split, the partition of its range of the parent into the other buffer (`flags`: the split's
// flag words, one per 32 positions); then, for every unit, its built-child rows into the unit's region of slab
// `slab_index`. `scan` is 2 kHistThreads + 64 words of shared memory apart from the histogram's; `cursor` the
// split's two placement counters (8-byte aligned, zero before the step); `units` the prepared unit descriptions
// (`cached` of them; later units are prepared into `spare`).
inline __device__ void fused_step_cta(const TrainArgs& a, const HistArgs& h, const Step& st, const FusedStep& fs,
                                      uint32_t cta, uint32_t slab_index, uint32_t* flags, int* sh, uint32_t* scan,
                                      unsigned int* cursor, const uint8_t* active, HistCta* units, uint32_t cached,
                                      HistCta* spare) {
    if (cta >= fs.chunks) return;
    uint32_t lo, hi;
    fused_range(fs.count, fs.chunks, cta, lo, hi);
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr uint32_t kWarps = kHistThreads / 32;
    constexpr int kBatch = 8;  // words a warp has in flight
    const uint32_t* rows_in = a.rows[fs.src] + fs.begin;
    const int32_t* gh_in = a.ordered[fs.src] + fs.begin;
    uint32_t* rows_out = a.rows[fs.dst] + fs.begin;
    int32_t* gh_out = a.ordered[fs.dst] + fs.begin;
    uint32_t* words = scan + kHistThreads;       // a round's flag words
    uint32_t* sums = scan + 2 * kHistThreads;    // per-warp sums, then the round total
    __shared__ uint32_t s_base[3];               // the CTA's first left, first right (from the end), left count

    const uint32_t w_lo = lo / 32, w_hi = static_cast<uint32_t>(ceil_div(hi, 32));
    if (!fs.root) {
        // Pass 1: the flags of the CTA's words, kept in the flag buffer, and its left count. The split feature's
        // bins come from its feature-major column. Warp w takes kBatch consecutive words at a time, and its lanes
        // 0 .. kBatch-1 store their flag words with one instruction.
        const uint8_t* column = a.d.columns + static_cast<uint64_t>(st.info.feature) * a.d.column_stride;
        uint32_t mine = 0;
        if (fs.identity && fs.begin % 16 == 0) {
            // The parent's rows are its positions: lane k reads the bins of 16 consecutive rows with one 16-byte
            // load (a warp covers 16 words), and lanes 2i, 2i + 1 make word i's two halves. The column's stride
            // (a multiple of 128 bytes) covers the 16 bytes past any row.
            constexpr uint32_t kWords = 16;
            for (uint32_t w0 = w_lo + warp * kWords; w0 < w_hi; w0 += kWords * kWarps) {
                const uint32_t p0 = w0 * 32 + 16 * lane;
                uint32_t m = 0;
                if (p0 < hi) {
                    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(column + fs.begin + p0));
                    const uint32_t x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int k = 0; k < 16; ++k)
                        if (bin_goes_left(st.left_bins, (x[k / 4] >> (8 * (k % 4))) & 0xFFu)) m |= 1u << k;
                    if (hi - p0 < 16) m &= (1u << (hi - p0)) - 1u;
                }
                mine += __reduce_add_sync(0xffffffffu, __popc(m));  // every lane keeps the warp's count
                const uint32_t upper = __shfl_down_sync(0xffffffffu, m, 1);
                const uint32_t w = w0 + lane / 2;
                if ((lane & 1) == 0 && w < w_hi) flags[w] = m | (upper << 16);
            }
        } else {
        for (uint32_t w0 = w_lo + warp * kBatch; w0 < w_hi; w0 += kBatch * kWarps) {
            uint32_t row[kBatch];
            bool valid[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const uint32_t w = w0 + j, p = w * 32 + lane;
                valid[j] = w < w_hi && p < hi;
                row[j] = !valid[j] ? 0u : fs.identity ? fs.begin + p : __ldcg(rows_in + p);
            }
            uint32_t flag_word = 0;
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const bool left = valid[j] && bin_goes_left(st.left_bins, __ldg(column + row[j]));
                const uint32_t word = __ballot_sync(0xffffffffu, left);
                if (lane == static_cast<uint32_t>(j)) flag_word = word;
                mine += __popc(word);
            }
            if (lane < static_cast<uint32_t>(kBatch) && w0 + lane < w_hi) flags[w0 + lane] = flag_word;
        }
        }
        if (lane == 0) sums[warp] = mine;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t left = 0;
            for (uint32_t k = 0; k < kWarps; ++k) left += sums[k];
            // One 64-bit atomic for both sides (lefts in the low word, rights in the high; neither passes 2^32):
            // this CTA's lefts go to [base_l, base_l + left) from the parent's start and its rights to the `right`
            // positions ending `base_r` before the parent's end.
            const unsigned long long add = (static_cast<unsigned long long>((hi - lo) - left) << 32) | left;
            const unsigned long long old = atomicAdd(reinterpret_cast<unsigned long long*>(cursor), add);
            s_base[0] = static_cast<uint32_t>(old);
            s_base[1] = static_cast<uint32_t>(old >> 32);
            s_base[2] = left;
        }
        __syncthreads();

        // Pass 2: the scatter, in rounds of one word per thread: the round's word counts scanned over the CTA, then
        // each warp places kBatch consecutive words' positions at a time.
        uint32_t carry = 0;  // lefts of the CTA's earlier rounds
        for (uint32_t r0 = w_lo; r0 < w_hi; r0 += kFusedScanWords) {
            const uint32_t nw = min(w_hi - r0, kFusedScanWords);
            const uint32_t word = threadIdx.x < nw ? __ldcg(flags + r0 + threadIdx.x) : 0u;
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
            for (uint32_t k0 = warp * kBatch; k0 < nw; k0 += kBatch * kWarps) {
                uint32_t row[kBatch];
                int32_t gh[kBatch];
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const uint32_t k = k0 + j, p = (r0 + k) * 32 + lane;
                    const bool valid = k < nw && p < hi;
                    row[j] = !valid ? 0u : fs.identity ? fs.begin + p : __ldcg(rows_in + p);
                    gh[j] = valid ? __ldcg(gh_in + p) : 0;
                }
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const uint32_t k = k0 + j, p = (r0 + k) * 32 + lane;
                    if (k >= nw) break;  // warp-uniform
                    if (p >= hi) continue;
                    const uint32_t bits = words[k];
                    const bool left = (bits >> lane) & 1u;
                    const uint32_t lefts = scan[k] + __popc(bits & ((1u << lane) - 1u));
                    const uint32_t rights = (p - lo) - lefts;
                    const uint32_t target = left ? s_base[0] + lefts : fs.count - 1 - (s_base[1] + rights);
                    rows_out[target] = row[j];
                    gh_out[target] = gh[j];
                }
            }
            carry += sums[32];
            __syncthreads();  // the round's scan and words are read
        }
    }
    if (!fs.histogram) return;

    // Pass 3, per unit: the built child's rows of this CTA, one contiguous range, into the unit's slab region.
    RowSource src;
    uint32_t b0, b1;
    if (fs.root) {
        src = RowSource{nullptr, h.packed, true};
        b0 = lo;
        b1 = hi;
    } else {
        src = RowSource{rows_out, gh_out, false};
        const uint32_t left = s_base[2], right = (hi - lo) - left;
        b0 = fs.built_left ? s_base[0] : fs.count - s_base[1] - right;
        b1 = b0 + (fs.built_left ? left : right);
    }
    const uint64_t pol = evict_first_policy();
    __shared__ LaneTile s_lt[kMaxUnitTiles];
    int* slab = h.slabs + static_cast<size_t>(slab_index) * h.slab_ints;
    uint32_t region = 0;  // ints before this unit's slab region
    // Rows per flush: all of them when the slabs hold packed sums (the range fits a packed round), else rounds of
    // at most round_rows rows.
    const uint32_t round = fs.packed ? 0xFFFFFFFFu : max(1u, fs.round_rows);
    // With skipping tiles, the first wanted unit's pass also sums the rows' unpacked gradients (every position of
    // the range once), for the slab's totals.
    int tg = 0, th = 0;
    bool counted = h.totals == 0;
    for (uint32_t u = 0; u < h.num_units; ++u) {
        HistCta* c = u < cached ? units + u : spare;
        if (u >= cached) histogram_prepare_unit(h, u, sh, spare);
        const bool want = fused_unit_begin(*c, active, s_lt);
        const uint32_t nt = c->unit.num_tiles;
        const bool count = want && !counted;
        counted = counted || want;
        uint32_t r0 = b0;
        while (true) {
            const uint32_t r1 = want ? (b1 - r0 > round ? r0 + round : b1) : b1;
            if (want) hist_stream(s_lt, nt, src, r0, r1, fs.stage, fs.slot_bytes, fs.depth, pol, count, tg, th);
            const bool last = r1 >= b1;
            // Packed slabs: one flush at the end. Unpacked: a flush per round, stored the first time, added after.
            if (last || !fs.packed)
                fused_unit_flush(*c, slab + region / 2, slab + region, fs.packed, r0 == b0,
                                 fs.depth > 0 && fs.depth * kWarps * fs.slot_bytes >= 4 * 32 * (256 + 4) ? fs.stage : 0u);
            if (last) break;
            r0 = r1;
        }
        region += 2 * c->unit.slots;
    }
    if (h.totals != 0) {
        // The CTA's totals into the slab (zeros when no unit was wanted: then no bin is recovered from them).
        tg = __reduce_add_sync(0xffffffffu, tg);
        th = __reduce_add_sync(0xffffffffu, th);
        if (lane == 0) {
            scan[2 * warp] = static_cast<uint32_t>(tg);
            scan[2 * warp + 1] = static_cast<uint32_t>(th);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t sg = 0, sh_ = 0;
            for (uint32_t k = 0; k < kWarps; ++k) {
                sg += scan[2 * k];
                sh_ += scan[2 * k + 1];
            }
            __stcg(reinterpret_cast<int2*>(slab + h.totals), make_int2(static_cast<int>(sg), static_cast<int>(sh_)));
        }
        __syncthreads();  // the scan words are free again
    }
}

// ---- ranks: flags and sums over NVLink ------------------------------------------------------------------------


__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread: waits until a rank's `flag` reaches `epoch`, at most `limit` polls; false (error 4 recorded, or
// another CTA's error seen) when it gives up.
__device__ __forceinline__ bool wait_peer(const uint32_t* flag, uint32_t epoch, uint32_t limit, int* error) {
    for (uint32_t i = 0;; ++i) {
        if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
        if (*reinterpret_cast<volatile int*>(error) != 0) return false;
        if (i >= limit) {
            atomicCAS(error, 0, 4);
            return false;
        }
        __nanosleep(64);
    }
}

// One warp: waits, lane s for source rank s (s < world, s != `skip`), until the flag at byte `off + 4 s` of this
// rank's own exchange buffer reaches `epoch`; true when every rank's did.
__device__ __forceinline__ bool wait_ranks(const GrowExchange& x, size_t off, uint32_t epoch, int* error,
                                           int skip = -1) {
    const int lane = static_cast<int>(threadIdx.x & 31);
    bool ok = true;
    if (lane < x.world && lane != skip)
        ok = wait_peer(reinterpret_cast<const uint32_t*>(x.peers[x.rank] + off) + lane, epoch, x.spin_limit, error);
    return __all_sync(0xffffffffu, ok);
}

// Left count of split j from source rank s, in the exchange buffer's words (the step's parity).
__device__ __forceinline__ size_t exchange_left_word(const ExchangeLayout& L, uint32_t epoch, int j, int s) {
    return L.left_values / 4 + ((epoch & 1) * kSplits + static_cast<size_t>(j)) * kMaxRanks + s;
}

// CTA 0, warp 0: this rank's left counts of the step's `n` splits into every rank's buffer (lane q writes rank
// q's), each rank's followed by this rank's flag; the release store orders the counts before the flag.
__device__ __forceinline__ void publish_left(const GrowExchange& x, const ExchangeLayout& L, uint32_t epoch,
                                             const uint32_t* left, int n) {
    const int q = static_cast<int>(threadIdx.x & 31);
    if (q < x.world) {
        uint32_t* dst = reinterpret_cast<uint32_t*>(x.peers[q]);
        for (int j = 0; j < n; ++j) dst[exchange_left_word(L, epoch, j, x.rank)] = left[j];
        st_release_sys(dst + L.left_flags / 4 + x.rank, epoch);
    }
}

// Whole CTA: every rank's left counts of the step's `n` splits, summed into total[j] (shared); false when a rank
// did not answer.
__device__ __forceinline__ bool gather_left(const GrowExchange& x, const ExchangeLayout& L, uint32_t epoch, int n,
                                            int* error, int64_t* total) {
    __shared__ int s_ok;
    if (threadIdx.x < 32) {
        const bool ok = wait_ranks(x, L.left_flags, epoch, error);
        const int lane = static_cast<int>(threadIdx.x);
        const uint32_t* own = reinterpret_cast<const uint32_t*>(x.peers[x.rank]);
        for (int j = 0; j < n; ++j) {
            int64_t v = ok && lane < x.world ? static_cast<int64_t>(__ldcg(own + exchange_left_word(L, epoch, j, lane))) : 0;
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) total[j] = v;
        }
        if (lane == 0) s_ok = ok;
    }
    __syncthreads();
    const bool ok = s_ok != 0;
    __syncthreads();
    return ok;
}

__device__ __forceinline__ int owner_of(const GrowExchange& x, uint32_t f) { return static_cast<int>(f % x.world); }

// Item (j, feature f)'s word in the owner's item flags, and its bins from source s in the owner's buffer.
__device__ __forceinline__ size_t item_flags_at(const ExchangeLayout& L, const GrowExchange& x, uint32_t j, uint32_t f) {
    return L.item_flags + 4ull * (static_cast<size_t>(j) * L.owned + f / x.world) * kMaxRanks;
}
__device__ __forceinline__ size_t item_bins_at(const ExchangeLayout& L, const GrowExchange& x, int s, uint32_t j,
                                               uint32_t f) {
    return L.bins + 8ull * ((static_cast<size_t>(s) * kSplits + j) * L.owned + f / x.world) * kMaxBins;
}

// Whole CTA, at a feature this rank does not own: its built-child bins of split j (`built`, shared) written into
// the owner's buffer, then this rank's flag for the item raised there.
__device__ __forceinline__ void push_bins(const GrowExchange& x, const ExchangeLayout& L, uint32_t epoch, uint32_t j,
                                          uint32_t f, uint32_t nb, const int2* built) {
    const int owner = owner_of(x, f);
    int2* dst = reinterpret_cast<int2*>(x.peers[owner] + item_bins_at(L, x, x.rank, j, f));
    for (uint32_t t = threadIdx.x; t < nb; t += blockDim.x) dst[t] = built[t];
    __syncthreads();  // the CTA's stores are issued: the release below orders them before the flag
    if (threadIdx.x == 0)
        st_release_sys(reinterpret_cast<uint32_t*>(x.peers[owner] + item_flags_at(L, x, j, f)) + x.rank, epoch);
}

// Whole CTA, at a feature this rank owns: every other rank's built-child bins of split j added to this rank's own
// (`built`, shared); false when a rank did not answer (error recorded).
__device__ __forceinline__ bool gather_bins(const GrowExchange& x, const ExchangeLayout& L, uint32_t epoch,
                                            uint32_t j, uint32_t f, uint32_t nb, int2* built, int* error) {
    __shared__ int s_ok;
    if (threadIdx.x < 32) {
        const bool ok = wait_ranks(x, item_flags_at(L, x, j, f), epoch, error, x.rank);
        if (threadIdx.x == 0) s_ok = ok;
    }
    __syncthreads();
    const bool ok = s_ok != 0;
    if (ok) {
        for (uint32_t t = threadIdx.x; t < nb; t += blockDim.x) {
            int2 v[kMaxRanks];
#pragma unroll
            for (int q = 0; q < kMaxRanks; ++q)
                v[q] = q < x.world && q != x.rank
                           ? __ldcg(reinterpret_cast<const int2*>(x.peers[x.rank] + item_bins_at(L, x, q, j, f)) + t)
                           : make_int2(0, 0);
            int2 sum = built[t];
#pragma unroll
            for (int q = 0; q < kMaxRanks; ++q) sum = make_int2(sum.x + v[q].x, sum.y + v[q].y);
            built[t] = sum;
        }
    }
    __syncthreads();
    return ok;
}

// A search item's two candidates (rows 2 j and 2 j + 1 at feature f), written to every rank's candidate arrays (one
// rank: the local ones, as `a` holds them).
struct CandidateSink {
    FeatureCandidate* cands[kMaxRanks];
    uint8_t* flags[kMaxRanks];
    double* gains[kMaxRanks];
    int ranks;
};

// With ranks, the step's set (`parity`) of rank q's candidate arrays in its exchange buffer (ExchangeLayout).
__device__ __forceinline__ size_t candidate_set(const ExchangeLayout& L, uint32_t parity) {
    return static_cast<size_t>(parity & 1) * 2 * kSplits * L.features;
}

__device__ __forceinline__ CandidateSink candidate_sink(const TrainArgs& a, const GrowExchange& x,
                                                        const ExchangeLayout& L, uint32_t parity) {
    CandidateSink k{};
    k.ranks = x.world > 1 ? x.world : 1;
    const size_t set = candidate_set(L, parity);
    for (int q = 0; q < k.ranks; ++q) {
        if (x.world > 1) {
            k.cands[q] = reinterpret_cast<FeatureCandidate*>(x.peers[q] + L.candidates) + set;
            k.flags[q] = x.peers[q] + L.cand_flags + set;
            k.gains[q] = reinterpret_cast<double*>(x.peers[q] + L.cand_gain) + set;
        } else {
            k.cands[q] = static_cast<FeatureCandidate*>(a.candidates);
            k.flags[q] = a.cand_flags;
            k.gains[q] = a.cand_gain;
        }
    }
    return k;
}

__device__ __forceinline__ void sink_candidate(const CandidateSink& k, size_t at, const FeatureCandidate& c) {
    const uint8_t flags = static_cast<uint8_t>((c.found ? 1 : 0) | (c.splittable ? 2 : 0));
    for (int q = 0; q < k.ranks; ++q) {
        k.cands[q][at] = c;
        k.flags[q][at] = flags;
        k.gains[q][at] = c.gain;
    }
}

// CTA 0, warp 0, after the grid barrier that follows the search: this rank's step flag in every rank's buffer (every
// candidate this rank owns is written). Every CTA then waits for every rank's (wait_steps).
__device__ __forceinline__ void publish_step(const GrowExchange& x, const ExchangeLayout& L, uint32_t epoch) {
    const int q = static_cast<int>(threadIdx.x & 31);
    if (q < x.world) st_release_sys(reinterpret_cast<uint32_t*>(x.peers[q] + L.step_flags) + x.rank, epoch);
}

__device__ __forceinline__ bool wait_steps(const GrowExchange& x, const ExchangeLayout& L, uint32_t epoch, int* error) {
    __shared__ int s_ok;
    if (threadIdx.x < 32) {
        const bool ok = wait_ranks(x, L.step_flags, epoch, error);
        if (threadIdx.x == 0) s_ok = ok;
    }
    __syncthreads();
    const bool ok = s_ok != 0;
    __syncthreads();
    return ok;
}

// ---- the built child's histogram and the search, one feature per CTA ---------------------------------------

// Feature `f`'s bins of the built child summed over `chunks` slabs from slab `first` into `out` (shared, [g, h] per bin):
// thread t of the CTA takes bin t mod 256 over the chunks c = t / 256, t / 256 + 2, ... (a warp reads 32
// consecutive bins of a chunk: 128 or 256 bytes), with kLoads chunks in flight; the odd chunks' sums meet the even
// ones' through `part` (shared). Whole CTA (kHistThreads threads).
template <bool kPacked>
__device__ __forceinline__ void reduce_feature_bins_halves(const HistArgs& h, const DevFeature& feat, uint32_t first,
                                                           uint32_t chunks, int2* part, int2* out) {
    constexpr int kLoads = 16;
    const uint32_t b = threadIdx.x & 255, half = threadIdx.x >> 8;
    int sg = 0, sh = 0;
    if (b < feat.num_bins) {
        const int* base = h.slabs + static_cast<size_t>(first) * h.slab_ints + (kPacked ? feat.slab_off + b : 2 * (feat.slab_off + b));
        for (uint32_t c0 = half; c0 < chunks; c0 += 2 * kLoads) {
            uint32_t v[kLoads];
            int2 w[kLoads];
#pragma unroll
            for (int k = 0; k < kLoads; ++k) {
                const uint32_t c = c0 + 2 * k;
                const int* at = base + static_cast<size_t>(c) * h.slab_ints;
                if (kPacked)
                    v[k] = c < chunks ? static_cast<uint32_t>(__ldcg(at)) : 0u;
                else
                    w[k] = c < chunks ? __ldcg(reinterpret_cast<const int2*>(at)) : make_int2(0, 0);
            }
#pragma unroll
            for (int k = 0; k < kLoads; ++k) {
                if (kPacked) {
                    const int g = static_cast<int16_t>(v[k] & 0xFFFFu);  // quantize.rs:140-143
                    sg += g;
                    sh += static_cast<int>((v[k] - static_cast<uint32_t>(g)) >> 16);
                } else {
                    sg += w[k].x;
                    sh += w[k].y;
                }
            }
        }
        if (half == 1) part[b] = make_int2(sg, sh);
    }
    __syncthreads();
    if (half == 0 && b < feat.num_bins) out[b] = make_int2(sg + part[b].x, sh + part[b].y);
    __syncthreads();
}

// The same sum with 16-byte loads: thread (g, q) of the CTA takes bins 4q .. 4q+3 over the chunks g, g + 8, ...
// (64 threads cover a feature's 256 bins of one chunk; 8 such groups split the chunks, all of a group's loads in
// flight together), and the 8 groups' sums meet in `scratch` (shared, 8 x 64 x 32 bytes).
template <bool kPacked>
__device__ __forceinline__ void reduce_feature_bins_quads(const HistArgs& h, const DevFeature& feat, uint32_t first,
                                                          uint32_t chunks, int4* scratch, int2* out) {
    constexpr uint32_t kGroups = kHistThreads / 64, kLoads = 8;
    const uint32_t q = threadIdx.x & 63, g = threadIdx.x >> 6;
    int4 sg = make_int4(0, 0, 0, 0), sh = sg;  // bins 4q .. 4q+3: g and h sums
    if (4 * q < feat.num_bins) {
        const int* base = h.slabs + static_cast<size_t>(first) * h.slab_ints + (kPacked ? feat.slab_off + 4 * q : 2 * (feat.slab_off + 4 * q));
        for (uint32_t c0 = g; c0 < chunks; c0 += kGroups * kLoads) {
            int4 v[kLoads], w[kLoads];
#pragma unroll
            for (uint32_t k = 0; k < kLoads; ++k) {
                const uint32_t c = c0 + kGroups * k;
                const int4* at = reinterpret_cast<const int4*>(base + static_cast<size_t>(c) * h.slab_ints);
                v[k] = c < chunks ? __ldcg(at) : make_int4(0, 0, 0, 0);
                if (!kPacked) w[k] = c < chunks ? __ldcg(at + 1) : make_int4(0, 0, 0, 0);
            }
#pragma unroll
            for (uint32_t k = 0; k < kLoads; ++k) {
                if (kPacked) {
                    // unpack (quantize.rs:140-143)
                    const uint32_t x[4] = {static_cast<uint32_t>(v[k].x), static_cast<uint32_t>(v[k].y),
                                           static_cast<uint32_t>(v[k].z), static_cast<uint32_t>(v[k].w)};
                    int gx[4], hx[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        gx[j] = static_cast<int16_t>(x[j] & 0xFFFFu);
                        hx[j] = static_cast<int>((x[j] - static_cast<uint32_t>(gx[j])) >> 16);
                    }
                    sg = make_int4(sg.x + gx[0], sg.y + gx[1], sg.z + gx[2], sg.w + gx[3]);
                    sh = make_int4(sh.x + hx[0], sh.y + hx[1], sh.z + hx[2], sh.w + hx[3]);
                } else {  // [g, h] pairs: v = bins 4q, 4q+1; w = 4q+2, 4q+3
                    sg = make_int4(sg.x + v[k].x, sg.y + v[k].z, sg.z + w[k].x, sg.w + w[k].z);
                    sh = make_int4(sh.x + v[k].y, sh.y + v[k].w, sh.z + w[k].y, sh.w + w[k].w);
                }
            }
        }
    }
    scratch[2 * (g * 64 + q)] = sg;
    scratch[2 * (g * 64 + q) + 1] = sh;
    __syncthreads();
    const uint32_t b = threadIdx.x;
    if (b < feat.num_bins) {
        const int* sc = reinterpret_cast<const int*>(scratch);
        int tg = 0, th = 0;
#pragma unroll
        for (uint32_t k = 0; k < kGroups; ++k) {
            tg += sc[8 * (k * 64 + b / 4) + (b & 3)];
            th += sc[8 * (k * 64 + b / 4) + 4 + (b & 3)];
        }
        out[b] = make_int2(tg, th);
    }
    __syncthreads();
}

// A search item's slab bins copied ahead into shared memory while the CTA scans its previous item: chunk c's
// quads (int4: four packed bins, or two [g, h] pairs) at `pbuf` + 16 (c * quads + k). Whole CTA; false (nothing
// issued) when they do not fit in `cap` bytes.
__device__ __forceinline__ uint32_t slab_quads(uint32_t num_bins, bool packed) {
    return packed ? (num_bins + 3) / 4 : (num_bins + 1) / 2;
}

__device__ __forceinline__ bool prefetch_feature_bins(const HistArgs& h, const DevFeature& feat, uint32_t first,
                                                      uint32_t chunks, bool packed, uint32_t pbuf, uint32_t cap) {
    const uint32_t per = slab_quads(feat.num_bins, packed);
    if (static_cast<uint64_t>(chunks) * per * 16 > cap) return false;
    // the bins past num_bins that a quad covers lie inside the feature's smem_bins slots of the slab
    const int* base = h.slabs + static_cast<size_t>(first) * h.slab_ints + (packed ? feat.slab_off : 2 * feat.slab_off);
    const uint64_t pol = evict_first_policy();
    for (uint32_t e = threadIdx.x; e < chunks * per; e += kHistThreads) {
        const uint32_t c = e / per, k = e - c * per;
        cp_async16(pbuf + 16 * e, base + static_cast<size_t>(c) * h.slab_ints + 4 * k, pol);
    }
    cp_async_commit();
    return true;
}

// reduce_feature_bins_quads over the prefetched copy (`pbuf`, as prefetch_feature_bins laid it out).
template <bool kPacked>
__device__ __forceinline__ void reduce_feature_bins_staged(const DevFeature& feat, uint32_t chunks, uint32_t pbuf,
                                                           int4* scratch, int2* out) {
    constexpr uint32_t kGroups = kHistThreads / 64;
    const uint32_t q = threadIdx.x & 63, g = threadIdx.x >> 6;
    const uint32_t per = slab_quads(feat.num_bins, kPacked);
    int4 sg = make_int4(0, 0, 0, 0), sh = sg;
    if (4 * q < feat.num_bins) {
        for (uint32_t c = g; c < chunks; c += kGroups) {
            const uint32_t at = pbuf + 16 * (c * per + (kPacked ? q : 2 * q));
            const uint4 v = lds128(at);
            if (kPacked) {
                const uint32_t x[4] = {v.x, v.y, v.z, v.w};
                int gx[4], hx[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    gx[j] = static_cast<int16_t>(x[j] & 0xFFFFu);  // quantize.rs:140-143
                    hx[j] = static_cast<int>((x[j] - static_cast<uint32_t>(gx[j])) >> 16);
                }
                sg = make_int4(sg.x + gx[0], sg.y + gx[1], sg.z + gx[2], sg.w + gx[3]);
                sh = make_int4(sh.x + hx[0], sh.y + hx[1], sh.z + hx[2], sh.w + hx[3]);
            } else {
                const uint4 w = lds128(at + 16);
                sg = make_int4(sg.x + static_cast<int>(v.x), sg.y + static_cast<int>(v.z), sg.z + static_cast<int>(w.x),
                               sg.w + static_cast<int>(w.z));
                sh = make_int4(sh.x + static_cast<int>(v.y), sh.y + static_cast<int>(v.w), sh.z + static_cast<int>(w.y),
                               sh.w + static_cast<int>(w.w));
            }
        }
    }
    scratch[2 * (g * 64 + q)] = sg;
    scratch[2 * (g * 64 + q) + 1] = sh;
    __syncthreads();
    const uint32_t b = threadIdx.x;
    if (b < feat.num_bins) {
        const int* sc = reinterpret_cast<const int*>(scratch);
        int tg = 0, th = 0;
#pragma unroll
        for (uint32_t k = 0; k < kGroups; ++k) {
            tg += sc[8 * (k * 64 + b / 4) + (b & 3)];
            th += sc[8 * (k * 64 + b / 4) + 4 + (b & 3)];
        }
        out[b] = make_int2(tg, th);
    }
    __syncthreads();
}

// A feature of a Tile::skip tile (DevFeature::mfb): its built-child bins `bufs` (shared, [g, h] per stored bin,
// num_bins of them, as reduced from the slabs) back in bin order. Stored bin 0, its dominant bin mfb, added nothing:
// since every row adds to exactly one bin of every feature, bin mfb is the rows' totals (kept per slab, from slab
// `first` on over `chunks`) minus every other stored bin, and stored bin mfb is bin 0. Whole CTA (kHistThreads);
// bufs[kMaxBins ..] holds the warps' partial sums. Two's-complement sums: exact wherever the bin's own sum fits
// an int32, as every histogram bin must.
__device__ __forceinline__ void recover_dominant_bins(const HistArgs& h, const DevFeature& feat, uint32_t first,
                                                      uint32_t chunks, int2* bufs) {
    constexpr uint32_t kWarps = kHistThreads / 32;
    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    int2* part = bufs + kMaxBins;
    uint32_t g = 0, hh = 0;
    for (uint32_t c = t; c < chunks; c += kHistThreads) {
        const int2 v = __ldcg(reinterpret_cast<const int2*>(h.slabs + static_cast<size_t>(first + c) * h.slab_ints + h.totals));
        g += static_cast<uint32_t>(v.x);
        hh += static_cast<uint32_t>(v.y);
    }
    if (t >= 1 && t < feat.num_bins) {
        g -= static_cast<uint32_t>(bufs[t].x);
        hh -= static_cast<uint32_t>(bufs[t].y);
    }
    g = __reduce_add_sync(0xffffffffu, g);
    hh = __reduce_add_sync(0xffffffffu, hh);
    if (lane == 0) part[warp] = make_int2(static_cast<int>(g), static_cast<int>(hh));
    __syncthreads();
    if (t == 0) {
        uint32_t sg = 0, sh = 0;
        for (uint32_t k = 0; k < kWarps; ++k) {
            sg += static_cast<uint32_t>(part[k].x);
            sh += static_cast<uint32_t>(part[k].y);
        }
        const uint32_t m = feat.mfb & 0xFFu;
        if (m != 0) bufs[0] = bufs[m];
        bufs[m] = make_int2(static_cast<int>(sg), static_cast<int>(sh));
    }
    __syncthreads();
}

// What a rank does with an item's built-child bins: searches them alone (one rank), pushes them to the feature's
// owner (another rank owns it), or adds every other rank's to them (it owns the feature).
enum class BinsMode { kLocal, kPush, kGather };

// The search of split j of a step for feature `f` in one CTA, both children at once, in two parts.
// feature_bins_cta: the built child's bins reduced from the split's slabs (`chunks` of them from slab `first`,
// packed or not) into `bufs` (2 kMaxBins int2 of shared memory; `scratch`, 16 KB of shared memory or null, serves
// the 16-byte reduction), then, with ranks, pushed to the feature's owner or summed with every rank's (`mode`);
// *evaluated says whether the feature is searched at all (`evaluate`: the split's features). For a split (not the
// root) searched here, the threads of the sibling's scan group (feature_scan_cta) also load their bin of the
// parent's histogram into `parent`, so that the load overlaps the reduction. With `pbuf` (not 0) the slab bins were
// prefetched there (prefetch_feature_bins): the reduction waits for the copies and reads them from shared memory.
// False when a rank did not answer (error recorded).
__device__ bool feature_bins_cta(const TrainArgs& a, const HistArgs& h, const Step& st, uint32_t j, uint32_t f,
                                 uint32_t first, uint32_t chunks, bool packed, const uint8_t* evaluate, int2* bufs,
                                 int4* scratch, BinsMode mode, const GrowExchange& x, const ExchangeLayout& L,
                                 uint32_t epoch, bool* evaluated, int2& parent, uint32_t pbuf = 0) {
    const DevFeature feat = a.d.features[f];
    *evaluated = load_flag(evaluate + f) && feat.tile >= 0 && feat.num_bins != 0;
    if (!*evaluated) return true;
    if (mode != BinsMode::kPush) {
        const uint32_t t = threadIdx.x % kScanThreads;
        if (!st.root && threadIdx.x / kScanThreads == 1 && t < feat.num_bins)
            parent = __ldcg(reinterpret_cast<const int2*>(a.slots) +
                            static_cast<size_t>(st.leaf) * a.total_bins + feat.hist_offset + t);
    }
    if (pbuf != 0) {
        cp_async_wait(0);
        __syncthreads();  // every thread's copies have landed
        if (packed)
            reduce_feature_bins_staged<true>(feat, chunks, pbuf, scratch, bufs);
        else
            reduce_feature_bins_staged<false>(feat, chunks, pbuf, scratch, bufs);
    } else if (scratch != nullptr) {
        if (packed)
            reduce_feature_bins_quads<true>(h, feat, first, chunks, scratch, bufs);
        else
            reduce_feature_bins_quads<false>(h, feat, first, chunks, scratch, bufs);
    } else if (packed) {
        reduce_feature_bins_halves<true>(h, feat, first, chunks, bufs + kMaxBins, bufs);
    } else {
        reduce_feature_bins_halves<false>(h, feat, first, chunks, bufs + kMaxBins, bufs);
    }
    // Each rank restores its own dominant bins (its own totals and most frequent bins) before any exchange.
    if (feat.mfb & kDominantSkip) recover_dominant_bins(h, feat, first, chunks, bufs);
    if (mode == BinsMode::kPush) {
        push_bins(x, L, epoch, j, f, feat.num_bins, bufs);
        return true;
    }
    if (mode == BinsMode::kGather) return gather_bins(x, L, epoch, j, f, feat.num_bins, bufs, &a.iter->error);
    return true;
}

// The histogram slot split j of a step writes child `c`'s bins to: the child's own (learner.rs:365-367) for the
// step's first split, which always commits; a speculative split's (j >= 1) go to its leaf's prepared slots, so the
// parent's bins survive a dropped split and the children's are kept for a later commit (the finish copies them to
// the children's slots when the split commits).
__device__ __forceinline__ size_t child_slot(const TrainArgs& a, const Step& st, const SearchCtx& s, uint32_t j, int c) {
    return j > 0 ? prep_slot(a, st.leaf, c) : static_cast<size_t>(s.child[c]);
}

// feature_scan_cta: with the built child's bins in `bufs`, group 0 scans the built child and group 1 the sibling
// (parent - built, learner.rs:365-367; group 1 alone reads the parent's slot, which the built child may take over,
// and writes both children's), each with scan_feature_group, as search_item_group does for one item. The
// candidates go to rows 2 j (built) and 2 j + 1 (sibling) of F.
__device__ void feature_scan_cta(const TrainArgs& a, const Step& st, const SearchCtx& s, uint32_t j, uint32_t f,
                                 bool evaluated, const int2& parent, int2* bufs, ScanShared* scan_sh,
                                 const CandidateSink& sink) {
    const uint32_t F = a.num_features;
    const uint32_t group = threadIdx.x / kScanThreads, t = threadIdx.x % kScanThreads;
    const size_t row = static_cast<size_t>(2 * j) * F;  // candidate rows 2 j and 2 j + 1
    if (!evaluated) {
        if (threadIdx.x == 0) {
            FeatureCandidate none{};
            none.feature = static_cast<int32_t>(f);
            sink_candidate(sink, row + f, none);
            sink_candidate(sink, row + F + f, none);
        }
        return;
    }
    const DevFeature feat = a.d.features[f];
    int2* built = bufs;
    int2* other = bufs + kMaxBins;
    const size_t slot_len = 2 * static_cast<size_t>(a.total_bins);
    const size_t off = 2 * static_cast<size_t>(feat.hist_offset);
    const bool mine = t < feat.num_bins;
    const int ch = static_cast<int>(group);
    if (st.root) {
        if (group == 0 && mine) __stcg(reinterpret_cast<int2*>(a.slots + off) + t, built[t]);
    } else if (group == 1 && mine) {
        const int2 bt = built[t];
        const int2 o = make_int2(parent.x - bt.x, parent.y - bt.y);
        other[t] = o;
        __stcg(reinterpret_cast<int2*>(a.slots + child_slot(a, st, s, j, 0) * slot_len + off) + t, bt);
        __stcg(reinterpret_cast<int2*>(a.slots + child_slot(a, st, s, j, 1) * slot_len + off) + t, o);
    }
    const int bar = 1 + ch;
    if (st.root && group == 1) {
        if (t == 0) {
            FeatureCandidate none{};
            none.feature = static_cast<int32_t>(f);
            sink_candidate(sink, row + F + f, none);
        }
    } else {
        group_sync(bar);  // the group's bins are in place
        const FeatureCandidate c = scan_feature_group(ch == 0 ? built : other, feat, static_cast<int>(f), s.ctx[ch],
                                                      a.cfg, scan_sh[group], bar);
        if (t == 0) sink_candidate(sink, row + static_cast<size_t>(ch) * F + f, c);
    }
    __syncthreads();  // the buffers and the scratch are free for the CTA's next feature
}

}  // namespace sb2
