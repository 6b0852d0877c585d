// search.cuh — the split search's device functions (see split.cu for the exactness argument), shared by the
// standalone search kernel and the persistent tree kernel: sibling subtraction (learner.rs:356-371), the numerical
// scans of split::find_best_split (split.rs:919-961), the split's application to the tree (Tree::split,
// tree.rs:143-177) and the choice of the next leaf (best_leaf, learner.rs:418-429).
//
// Exactness. Histogram units are integers, so every running sum of a scan is an exact integer prefix sum whatever
// the order it is added in; each candidate's count estimate is a per-bin `round_int` summed in i64, also
// order-free. Every other value (real hessian, gain, outputs) is one IEEE operation on those exact operands, written
// with explicit round-to-nearest intrinsics so nothing is fused into a multiply-add. The only sequential parts of
// LightGBM's scan, the `break` at the first candidate whose other side is too small and the first strict maximum,
// become a warp-wide minimum over candidate indices. Across features, `better` is a total order, so any reduction
// order gives the reference's winner. The result is bit for bit the CPU search's.
#pragma once

#include "train.cuh"

namespace sb2 {

namespace {

constexpr double kEpsilon = static_cast<double>(1e-15f);  // LightGBM kEpsilon (split.rs:37)
constexpr int kPerLane = kMaxBins / 32;

__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double ddiv(double a, double b) { return div_rn(a, b); }

__device__ __forceinline__ int64_t sat_f64_i64(double q) {
    if (q != q) return 0;
    if (q >= 9223372036854775807.0) return INT64_MAX;
    if (q <= -9223372036854775808.0) return INT64_MIN;
    return static_cast<int64_t>(q);
}
// split.rs:196-198
__device__ __forceinline__ int64_t round_int(double x) { return sat_f64_i64(dadd(x, 0.5)); }
// split.rs:159-162
__device__ __forceinline__ double leaf_gain(double g, double h, double l1, double l2) {
    const double r = fmax(dsub(fabs(g), l1), 0.0);
    return ddiv(dmul(r, r), dadd(h, l2));
}
// split.rs:151-154, :145-148, :190-192
__device__ __forceinline__ double sign_of(double x) { return static_cast<double>((x > 0.0) - (x < 0.0)); }
__device__ __forceinline__ double leaf_output(double g, double h, double l1, double l2) {
    const double t = dmul(sign_of(g), fmax(dsub(fabs(g), l1), 0.0));
    return ddiv(-t, dadd(h, l2));
}

// LeafCtx (split.rs:201-233)
struct Ctx {
    bool valid;
    double units_grad, units_hess;
    int64_t num_data;
    double sum_grad, sum_hess, cnt_factor, min_gain_shift;
    double gs, hs;
};

__device__ Ctx make_ctx(const sb2_split_config& c, double gs, double hs, double ug, double uh, int64_t count) {
    Ctx x{};
    x.valid = !(uh != uh || uh <= 0.0 || count <= 0);
    x.units_grad = ug;
    x.units_hess = uh;
    x.num_data = count;
    x.gs = gs;
    x.hs = hs;
    x.sum_grad = dmul(ug, gs);
    x.sum_hess = dadd(dmul(uh, hs), 2.0 * kEpsilon);
    const double shift = leaf_gain(x.sum_grad, x.sum_hess, c.lambda_l1, c.lambda_l2);
    x.cnt_factor = ddiv(static_cast<double>(count), x.sum_hess);
    x.min_gain_shift = dadd(shift, c.min_gain_to_split);
    return x;
}

struct Grown {
    bool found;
    uint32_t bin;
    double ug, uh;
    int64_t count;
    double gain;
};

__device__ __forceinline__ int64_t shfl_up_i64(int64_t v, int o) {
    return static_cast<int64_t>(__shfl_up_sync(0xffffffffu, static_cast<unsigned long long>(v), o));
}
__device__ __forceinline__ int64_t shfl_i64(int64_t v, int src) {
    return static_cast<int64_t>(__shfl_sync(0xffffffffu, static_cast<unsigned long long>(v), src));
}

// One FindBestThresholdSequentially direction over `m` candidates: candidate k adds bin `top - k` (reverse) or bin k
// (forward). Returns ScanBuffer::best of ScanBuffer::fill + evaluate (split.rs:420-531). `hist` is the feature's
// [g, h] pairs in shared memory.
__device__ Grown warp_scan(const int2* hist, int top, bool reverse, int m, const Ctx& x, const sb2_split_config& c) {
    const int lane = threadIdx.x & 31;
    const int64_t min_count = c.min_data_in_leaf > 1 ? c.min_data_in_leaf : 1;
    int64_t G[kPerLane], H[kPerLane], C[kPerLane];
    int64_t sg = 0, sh = 0, sc = 0;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int k = lane * kPerLane + i;
        int64_t g = 0, h = 0, cnt = 0;
        if (k < m) {
            const int bin = reverse ? top - k : k;
            const int2 v = hist[bin];
            g = v.x;
            h = v.y;
            cnt = round_int(dmul(dmul(static_cast<double>(h), x.hs), x.cnt_factor));
        }
        sg += g;
        sh += h;
        sc += cnt;
        G[i] = sg;
        H[i] = sh;
        C[i] = sc;
    }
    // Exclusive prefix of the lane totals.
    int64_t ig = sg, ih = sh, ic = sc;
    for (int o = 1; o < 32; o <<= 1) {
        const int64_t ug = shfl_up_i64(ig, o), uh = shfl_up_i64(ih, o), uc = shfl_up_i64(ic, o);
        if (lane >= o) {
            ig += ug;
            ih += uh;
            ic += uc;
        }
    }
    ig -= sg;
    ih -= sh;
    ic -= sc;
    // Flags and the first break.
    int first_break = m;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        G[i] += ig;
        H[i] += ih;
        C[i] += ic;
        const int k = lane * kPerLane + i;
        if (k < m) {
            const double uh = static_cast<double>(H[i]);
            const double hh = dadd(kEpsilon, dmul(uh, x.hs));
            const bool skip = C[i] < min_count || hh < c.min_sum_hessian_in_leaf || uh <= 0.0;
            const bool other_small = x.num_data - C[i] < min_count || dsub(x.sum_hess, hh) < c.min_sum_hessian_in_leaf ||
                                     dsub(x.units_hess, uh) <= 0.0;
            if (other_small && !skip && k < first_break) first_break = k;
        }
    }
    for (int o = 16; o > 0; o >>= 1) first_break = min(first_break, __shfl_xor_sync(0xffffffffu, first_break, o));
    // Gains of the candidates before the break (ScanBuffer::evaluate): leaf_gain(sum - left) + leaf_gain(left), each
    // r^2 / (h + l2) with r = max(|g| - l1, 0), computed for every bin without branches so that the divisions of
    // four bins issue together; bins past the break or skipped keep -inf.
    double gain[kPerLane];
    double mx = -INFINITY;
#pragma unroll
    for (int i0 = 0; i0 < kPerLane; i0 += 4) {
        double num[8], den[8], q[8];
        bool use[4], window[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = i0 + j, k = lane * kPerLane + i;
            const double uh = static_cast<double>(H[i]);
            const double hh = dadd(kEpsilon, dmul(uh, x.hs));
            const bool skip = C[i] < min_count || hh < c.min_sum_hessian_in_leaf || uh <= 0.0;
            window[j] = k < first_break;
            use[j] = window[j] && !skip;
            const double g = dmul(static_cast<double>(G[i]), x.gs);
            const double rl = fmax(dsub(fabs(dsub(x.sum_grad, g)), c.lambda_l1), 0.0);
            const double rr = fmax(dsub(fabs(g), c.lambda_l1), 0.0);
            num[2 * j] = dmul(rl, rl);
            den[2 * j] = dadd(dsub(x.sum_hess, hh), c.lambda_l2);
            num[2 * j + 1] = dmul(rr, rr);
            den[2 * j + 1] = dadd(hh, c.lambda_l2);
        }
        div_rn_batch(num, den, q);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            gain[i0 + j] = use[j] ? dadd(q[2 * j], q[2 * j + 1]) : -INFINITY;
            if (window[j]) mx = fmax(mx, gain[i0 + j]);
        }
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    Grown out{};
    out.found = false;
    if (!(mx > x.min_gain_shift)) return out;
    int best_k = 1 << 30;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int k = lane * kPerLane + i;
        if (k < first_break && gain[i] == mx && k < best_k) best_k = k;
    }
    for (int o = 16; o > 0; o >>= 1) best_k = min(best_k, __shfl_xor_sync(0xffffffffu, best_k, o));
    const int owner = best_k / kPerLane, slot = best_k % kPerLane;
    int64_t g = 0, h = 0, cnt = 0;
    double gn = 0.0;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i)
        if (i == slot) {
            g = G[i];
            h = H[i];
            cnt = C[i];
            gn = gain[i];
        }
    out.found = true;
    out.bin = static_cast<uint32_t>(reverse ? top - best_k : best_k);
    out.ug = static_cast<double>(shfl_i64(g, owner));
    out.uh = static_cast<double>(shfl_i64(h, owner));
    out.count = shfl_i64(cnt, owner);
    out.gain = __shfl_sync(0xffffffffu, gn, owner);
    return out;
}

// reverse_best / forward_best (split.rs:557-580) into a FeatureCandidate (minus the gain shift).
__device__ void reverse_best(const Ctx& x, const Grown& r, FeatureCandidate& o) {
    const double right_hess = dadd(kEpsilon, dmul(r.uh, x.hs));
    o.best_gain = r.gain;
    o.threshold = r.bin - 1;
    o.left_grad = dsub(x.sum_grad, dmul(r.ug, x.gs));
    o.left_hess = dsub(x.sum_hess, right_hess);
    o.left_count = x.num_data - r.count;
    o.left_units_grad = dsub(x.units_grad, r.ug);
    o.left_units_hess = dsub(x.units_hess, r.uh);
}
__device__ void forward_best(const Ctx& x, const Grown& l, FeatureCandidate& o) {
    o.best_gain = l.gain;
    o.threshold = l.bin;
    o.left_grad = dmul(l.ug, x.gs);
    o.left_hess = dadd(kEpsilon, dmul(l.uh, x.hs));
    o.left_count = l.count;
    o.left_units_grad = l.ug;
    o.left_units_hess = l.uh;
}

// ---- categorical features (split.rs:694-845) ------------------------------------------------------------
//
// A categorical feature is scanned by one warp: the one-hot scan (at most max_cat_to_onehot bins) evaluates every
// category at once; the sorted scan ranks the categories by ctr with all-pairs comparisons, then walks both ends of
// the order in chunks of 32 steps: the left side's sums are lane prefix sums, LightGBM's sequential rules (the first
// `break`, and the min_data_per_group grouping that only resets where a candidate is evaluated) are a walk over the
// chunk's ballots, and the gains of the evaluated steps are computed in parallel. The same IEEE operations on the same
// exact integer sums as split.rs: the results are the CPU search's bit for bit.

// LeafCtx::bin_count (split.rs:236-239)
__device__ __forceinline__ int64_t bin_count(const Ctx& x, double hess_units) {
    return round_int(dmul(dmul(hess_units, x.hs), x.cnt_factor));
}

// LeafCtx::check (split.rs:241-261) of a growing side (count, real hessian, hessian units) against the shrinking
// one: 0 continue, 1 break, 2 evaluate.
__device__ __forceinline__ int side_check(const Ctx& x, const sb2_split_config& c, int64_t count, double hess,
                                          double units_hess, int64_t shrink_count, double shrink_hess) {
    if (count < c.min_data_in_leaf || count <= 0 || hess < c.min_sum_hessian_in_leaf || units_hess <= 0.0) return 0;
    if (shrink_count < c.min_data_in_leaf || shrink_count <= 0) return 1;
    if (shrink_hess < c.min_sum_hessian_in_leaf || dsub(x.units_hess, units_hess) <= 0.0) return 1;
    return 2;
}

// f64::total_cmp's key (IEEE totalOrder): every bit but the sign flipped for negative values, compared as i64.
__device__ __forceinline__ int64_t total_order_key(double v) {
    const int64_t b = __double_as_longlong(v);
    return b ^ static_cast<int64_t>(static_cast<uint64_t>(b >> 63) >> 1);
}

// The warp's best (gain, index) of the lanes that have one: the higher gain, the lower index on equal gains.
__device__ __forceinline__ void warp_best(bool& have, double& gain, int& index) {
    for (int o = 16; o > 0; o >>= 1) {
        const bool oh = __shfl_xor_sync(0xffffffffu, have, o);
        const double og = __shfl_xor_sync(0xffffffffu, gain, o);
        const int oi = __shfl_xor_sync(0xffffffffu, index, o);
        if (oh && (!have || og > gain || (og == gain && oi < index))) {
            have = true;
            gain = og;
            index = oi;
        }
    }
}

// find_onehot (split.rs:694-737): one category left, the rest right (the bin's raw hessian is tested, and kEpsilon
// comes off the other side). Whole warp; every lane gets the result.
__device__ FeatureCandidate scan_onehot(const int2* hist, const DevFeature& f, int feature, const Ctx& x,
                                        const sb2_split_config& c) {
    const int lane = threadIdx.x & 31, nb = static_cast<int>(f.num_bins);
    FeatureCandidate o{};
    o.feature = feature;
    bool have = false, splittable = false;
    double bg = 0.0;
    int bt = 0x7FFFFFFF;
    for (int t0 = 1; t0 < nb; t0 += 32) {
        const int t = t0 + lane;
        if (t >= nb) continue;
        const int2 v = hist[t];
        const double h = static_cast<double>(v.y);
        const int64_t count = bin_count(x, h);
        const double raw_hess = dmul(h, x.hs);
        const double other_hess = dsub(dsub(x.sum_hess, raw_hess), kEpsilon);
        if (side_check(x, c, count, raw_hess, h, x.num_data - count, other_hess) != 2) continue;
        const double grad = dmul(static_cast<double>(v.x), x.gs);
        const double gain = dadd(leaf_gain(dsub(x.sum_grad, grad), other_hess, c.lambda_l1, c.lambda_l2),
                                 leaf_gain(grad, dadd(raw_hess, kEpsilon), c.lambda_l1, c.lambda_l2));
        if (gain != gain || gain <= x.min_gain_shift) continue;
        splittable = true;
        if (!have || gain > bg) {
            have = true;
            bg = gain;
            bt = t;
        }
    }
    warp_best(have, bg, bt);
    o.splittable = __any_sync(0xffffffffu, splittable);
    if (have) {
        const int2 v = hist[bt];
        const double h = static_cast<double>(v.y);
        o.found = 1;
        o.kind = kCandOneHot;
        o.best_gain = bg;
        o.threshold = static_cast<uint32_t>(bt);
        o.left_grad = dmul(static_cast<double>(v.x), x.gs);
        o.left_hess = dadd(dmul(h, x.hs), kEpsilon);
        o.left_count = bin_count(x, h);
        o.left_units_grad = static_cast<double>(v.x);
        o.left_units_hess = h;
        o.cat_bins[bt >> 5] = 1u << (bt & 31);
    }
    o.gain = dsub(o.best_gain, x.min_gain_shift);
    return o;
}

// find_sorted_categorical with sorted_categories and SortedScan::run (split.rs:739-845): the categories (bins 1..)
// with at least cat_smooth estimated rows in ascending sum_g / (sum_h + cat_smooth) (total order, then the bin),
// prefixes of up to min(max_cat_threshold, ceil(used / 2)) of them from the low end, then the high end, which
// replaces the low end's best only when strictly better. Whole warp; `order` is kMaxBins u16 of the warp's shared
// memory. Every lane gets the result.
__device__ FeatureCandidate scan_sorted(const int2* hist, const DevFeature& f, int feature, const Ctx& x,
                                        const sb2_split_config& c, uint16_t* order) {
    const int lane = threadIdx.x & 31;
    const int nb = min(static_cast<int>(f.num_bins), kMaxBins);
    const int regs = (nb + 31) / 32;
    FeatureCandidate o{};
    o.feature = feature;
    // The used categories and their ctr keys: bin lane + 32 k in register k.
    int64_t key[kPerLane];
    bool used[kPerLane];
    int rank[kPerLane];
#pragma unroll
    for (int k = 0; k < kPerLane; ++k) {
        const int t = lane + 32 * k;
        used[k] = false;
        key[k] = 0;
        rank[k] = 0;
        if (t >= 1 && t < nb) {
            const int2 v = hist[t];
            const double h = static_cast<double>(v.y);
            if (static_cast<double>(bin_count(x, h)) >= c.cat_smooth) {
                used[k] = true;
                key[k] = total_order_key(ddiv(dmul(static_cast<double>(v.x), x.gs), dadd(dmul(h, x.hs), c.cat_smooth)));
            }
        }
    }
    // Each used category's rank: the used categories before it in (key, bin) order.
#pragma unroll
    for (int sk = 0; sk < kPerLane; ++sk) {
        if (sk >= regs) break;
        for (int sl = 0; sl < 32; ++sl) {
            const int64_t ok_ = shfl_i64(key[sk], sl);
            const bool ou = __shfl_sync(0xffffffffu, used[sk], sl);
            const int ot = sl + 32 * sk;
#pragma unroll
            for (int k = 0; k < kPerLane; ++k) {
                const int t = lane + 32 * k;
                if (ou && used[k] && (ok_ < key[k] || (ok_ == key[k] && ot < t))) ++rank[k];
            }
        }
    }
    int mine = 0;
#pragma unroll
    for (int k = 0; k < kPerLane; ++k) {
        if (used[k]) order[rank[k]] = static_cast<uint16_t>(lane + 32 * k);
        mine += used[k] ? 1 : 0;
    }
    __syncwarp();
    const int n_used = __reduce_add_sync(0xffffffffu, mine);
    const int max_num_cat = min(max(c.max_cat_threshold, 0), (n_used + 1) / 2);
    const int steps = min(n_used, max_num_cat);
    const double l2 = dadd(c.lambda_l2, c.cat_l2);
    bool have = false, splittable = false;
    double bg = 0.0;
    int bi = 0, bdir = 0;
    for (int dir = 0; dir < 2; ++dir) {  // 0: from the low end of the order, 1: from the high end
        int64_t carry_g = 0, carry_h = 0, carry_c = 0, last_reset = 0;
        bool dhave = false;
        double dg = 0.0;
        int di = 0;
        for (int s0 = 0; s0 < steps; s0 += 32) {
            const int s = s0 + lane;
            const bool valid = s < steps;
            int64_t g = 0, h = 0, cnt = 0;
            if (valid) {
                const int2 v = hist[order[dir == 0 ? s : n_used - 1 - s]];
                g = v.x;
                h = v.y;
                cnt = bin_count(x, static_cast<double>(h));
            }
            int64_t G = g, H = h, C = cnt;  // inclusive prefix sums over the chunk's steps
            for (int d = 1; d < 32; d <<= 1) {
                const int64_t ug = shfl_up_i64(G, d), uh = shfl_up_i64(H, d), uc = shfl_up_i64(C, d);
                if (lane >= d) {
                    G += ug;
                    H += uh;
                    C += uc;
                }
            }
            G += carry_g;
            H += carry_h;
            C += carry_c;
            const double uh = static_cast<double>(H);
            const double left_hess = dadd(kEpsilon, dmul(uh, x.hs));
            const int64_t right_count = x.num_data - C;
            const double right_hess = dsub(x.sum_hess, left_hess);
            int st = valid ? side_check(x, c, C, left_hess, uh, right_count, right_hess) : 0;
            if (st == 2 && right_count < c.min_data_per_group) st = 1;
            const uint32_t brk = __ballot_sync(0xffffffffu, valid && st == 1);
            const int first_break = brk ? __ffs(brk) - 1 : 32;
            uint32_t eval = __ballot_sync(0xffffffffu, valid && st == 2);
            if (first_break < 32) eval &= (1u << first_break) - 1u;
            // min_data_per_group: a candidate is evaluated once the rows since the last evaluated one reach it
            uint32_t resets = 0;
            for (uint32_t m = eval; m != 0; m &= m - 1u) {
                const int i = __ffs(m) - 1;
                const int64_t ci = shfl_i64(C, i);
                if (ci - last_reset >= c.min_data_per_group) {
                    resets |= 1u << i;
                    last_reset = ci;
                }
            }
            bool ok = false;
            double gain = 0.0;
            if ((resets >> lane) & 1u) {
                const double lg = dmul(static_cast<double>(G), x.gs);
                gain = dadd(leaf_gain(lg, left_hess, c.lambda_l1, l2), leaf_gain(dsub(x.sum_grad, lg), right_hess, c.lambda_l1, l2));
                ok = !(gain != gain) && gain > x.min_gain_shift;
            }
            splittable = splittable || __any_sync(0xffffffffu, ok);
            bool ch = ok;
            double cg = gain;
            int ci = s;
            warp_best(ch, cg, ci);
            if (ch && (!dhave || cg > dg)) {
                dhave = true;
                dg = cg;
                di = ci;
            }
            carry_g = shfl_i64(G, 31);
            carry_h = shfl_i64(H, 31);
            carry_c = shfl_i64(C, 31);
            if (first_break < 32) break;
        }
        if (dhave && (!have || dg > bg)) {
            have = true;
            bg = dg;
            bi = di;
            bdir = dir;
        }
    }
    o.splittable = splittable;
    if (have) {
        // the winner's left side: the first bi + 1 categories from its end
        int64_t G = 0, H = 0, C = 0;
        for (int s = lane; s <= bi; s += 32) {
            const int2 v = hist[order[bdir == 0 ? s : n_used - 1 - s]];
            G += v.x;
            H += v.y;
            C += bin_count(x, static_cast<double>(v.y));
        }
        for (int d = 16; d > 0; d >>= 1) {
            G += shfl_i64(G, lane ^ d);
            H += shfl_i64(H, lane ^ d);
            C += shfl_i64(C, lane ^ d);
        }
        uint32_t bits[8] = {};
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
            const int t = lane + 32 * k;
            if (used[k] && (bdir == 0 ? rank[k] <= bi : rank[k] >= n_used - 1 - bi)) bits[t >> 5] |= 1u << (t & 31);
        }
#pragma unroll
        for (int w = 0; w < 8; ++w) o.cat_bins[w] = __reduce_or_sync(0xffffffffu, bits[w]);
        o.found = 1;
        o.kind = bdir == 0 ? kCandSortedForward : kCandSortedReverse;
        o.best_gain = bg;
        o.threshold = static_cast<uint32_t>(bi);
        o.left_units_grad = static_cast<double>(G);
        o.left_units_hess = static_cast<double>(H);
        o.left_grad = dmul(o.left_units_grad, x.gs);
        o.left_hess = dadd(kEpsilon, dmul(o.left_units_hess, x.hs));
        o.left_count = C;
    }
    o.gain = dsub(o.best_gain, x.min_gain_shift);
    __syncwarp();  // `order` is free again
    return o;
}

// find_feature's categorical arms (split.rs:855-859). Whole warp.
__device__ FeatureCandidate scan_categorical(const int2* hist, const DevFeature& f, int feature, const Ctx& x,
                                             const sb2_split_config& c, uint16_t* order) {
    if (!x.valid) {
        FeatureCandidate o{};
        o.feature = feature;
        return o;
    }
    if (static_cast<int64_t>(f.num_bins) <= c.max_cat_to_onehot) return scan_onehot(hist, f, feature, x, c);
    return scan_sorted(hist, f, feature, x, c, order);
}

// find_feature (split.rs:848-862) for one feature: find_numerical (:584-620), or the categorical scans with
// `order` (kMaxBins u16 of the warp's shared memory). Whole warp.
__device__ FeatureCandidate scan_feature(const int2* hist, const DevFeature& f, int feature, const Ctx& x,
                                         const sb2_split_config& c, uint16_t* order) {
    if (f.kind == SB2_CATEGORICAL) return scan_categorical(hist, f, feature, x, c, order);
    FeatureCandidate o{};
    o.feature = feature;
    o.found = 0;
    o.splittable = 0;
    if (!x.valid) return o;
    const int nb = static_cast<int>(f.num_bins);
    if (f.nan_bin && nb > 2) {
        const int last = nb - 2;
        const Grown r = warp_scan(hist, last, true, last, x, c);
        const Grown fw = warp_scan(hist, 0, false, last + 1, x, c);
        double output_gain = -INFINITY;
        if (r.found) {
            reverse_best(x, r, o);
            output_gain = dsub(o.best_gain, x.min_gain_shift);
            o.default_left = 1;
            o.found = 1;
            o.splittable = 1;
        }
        if (fw.found) {
            o.splittable = 1;
            FeatureCandidate b = o;
            forward_best(x, fw, b);
            if (b.best_gain > dadd(output_gain, x.min_gain_shift)) {
                o = b;
                o.default_left = 0;
                o.found = 1;
            }
        }
    } else if (nb >= 2) {
        const Grown r = warp_scan(hist, nb - 1, true, nb - 1, x, c);
        if (r.found) {
            reverse_best(x, r, o);
            o.default_left = f.nan_bin ? 0 : 1;
            o.found = 1;
            o.splittable = 1;
        }
    }
    o.gain = dsub(o.best_gain, x.min_gain_shift);
    return o;
}

// ---- the scan over a group of warps (the persistent tree kernel) ------------------------------------------
//
// The same FindBestThresholdSequentially as warp_scan, one candidate per thread: a group of kScanWarps warps
// (kScanThreads threads) scans a feature of up to kMaxBins bins, so every thread evaluates one bin's gain (two
// divisions) instead of a lane's eight in a row, and the group meets at a named barrier for each cross-warp
// reduction (prefix totals, the first break, the best gain, its first bin). Every value is the same integer or
// IEEE operation on the same operands as warp_scan's: the results are identical.
constexpr int kScanWarps = 8;
constexpr int kScanThreads = kScanWarps * 32;

// A group's shared scratch.
struct ScanShared {
    int64_t tot[3][kScanWarps];  // warp totals of g, h and count
    int32_t imin[kScanWarps];    // warp minima: the first break, then the best candidate
    double dmax[kScanWarps];     // warp maxima of the gains
    Grown best;
    uint16_t order[kMaxBins];    // a categorical feature's sorted categories (scan_sorted)
};

__device__ __forceinline__ void group_sync(int bar) {
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "n"(kScanThreads) : "memory");
}

__device__ __forceinline__ int32_t warp_min_i32(int32_t v) {
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// warp_scan over the group: thread t (threadIdx.x mod kScanThreads) owns candidate t. `bar` is the group's named
// barrier (not 0); every thread of the group gets the result.
__device__ Grown group_scan(const int2* hist, int top, bool reverse, int m, const Ctx& x, const sb2_split_config& c,
                            ScanShared& sh, int bar) {
    const int t = static_cast<int>(threadIdx.x) % kScanThreads, lane = t & 31, w = t >> 5;
    const int64_t min_count = c.min_data_in_leaf > 1 ? c.min_data_in_leaf : 1;
    int64_t g = 0, h = 0, cnt = 0;
    if (t < m) {
        const int2 v = hist[reverse ? top - t : t];
        g = v.x;
        h = v.y;
        cnt = round_int(dmul(dmul(static_cast<double>(h), x.hs), x.cnt_factor));
    }
    // Inclusive prefix over the group: within the warp, then the earlier warps' totals.
    int64_t G = g, H = h, C = cnt;
    for (int o = 1; o < 32; o <<= 1) {
        const int64_t ug = shfl_up_i64(G, o), uh = shfl_up_i64(H, o), uc = shfl_up_i64(C, o);
        if (lane >= o) {
            G += ug;
            H += uh;
            C += uc;
        }
    }
    if (lane == 31) {
        sh.tot[0][w] = G;
        sh.tot[1][w] = H;
        sh.tot[2][w] = C;
    }
    group_sync(bar);
    for (int j = 0; j < w; ++j) {
        G += sh.tot[0][j];
        H += sh.tot[1][j];
        C += sh.tot[2][j];
    }
    // Flags and the first break.
    bool skip = true;
    double hh = 0.0;
    int32_t first_break = m;
    if (t < m) {
        const double uh = static_cast<double>(H);
        hh = dadd(kEpsilon, dmul(uh, x.hs));
        skip = C < min_count || hh < c.min_sum_hessian_in_leaf || uh <= 0.0;
        const bool other_small = x.num_data - C < min_count || dsub(x.sum_hess, hh) < c.min_sum_hessian_in_leaf ||
                                 dsub(x.units_hess, uh) <= 0.0;
        if (other_small && !skip) first_break = t;
    }
    first_break = warp_min_i32(first_break);
    if (lane == 0) sh.imin[w] = first_break;
    group_sync(bar);
    first_break = sh.imin[0];
    for (int j = 1; j < kScanWarps; ++j) first_break = min(first_break, sh.imin[j]);
    // The gain of candidate t before the break (ScanBuffer::evaluate): leaf_gain(sum - left) + leaf_gain(left).
    const bool window = t < first_break;
    double gain = -INFINITY;
    if (window && !skip) {
        const double gd = dmul(static_cast<double>(G), x.gs);
        const double rl = fmax(dsub(fabs(dsub(x.sum_grad, gd)), c.lambda_l1), 0.0);
        const double rr = fmax(dsub(fabs(gd), c.lambda_l1), 0.0);
        double num[2] = {dmul(rl, rl), dmul(rr, rr)};
        double den[2] = {dadd(dsub(x.sum_hess, hh), c.lambda_l2), dadd(hh, c.lambda_l2)};
        double q[2];
        div_rn_batch(num, den, q);
        gain = dadd(q[0], q[1]);
    }
    double mx = window ? gain : -INFINITY;
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) sh.dmax[w] = mx;
    group_sync(bar);
    mx = sh.dmax[0];
    for (int j = 1; j < kScanWarps; ++j) mx = fmax(mx, sh.dmax[j]);
    Grown out{};
    out.found = false;
    if (!(mx > x.min_gain_shift)) return out;
    int32_t best = window && gain == mx ? t : (1 << 30);
    best = warp_min_i32(best);
    if (lane == 0) sh.imin[w] = best;
    group_sync(bar);
    best = sh.imin[0];
    for (int j = 1; j < kScanWarps; ++j) best = min(best, sh.imin[j]);
    if (t == best) {
        Grown b{};
        b.found = true;
        b.bin = static_cast<uint32_t>(reverse ? top - t : t);
        b.ug = static_cast<double>(G);
        b.uh = static_cast<double>(H);
        b.count = C;
        b.gain = gain;
        sh.best = b;
    }
    group_sync(bar);
    return sh.best;
}

// scan_feature over the group (the same find_numerical, split.rs:584-620); a categorical feature is scanned by the
// group's first warp alone, whose lanes get the candidate.
__device__ FeatureCandidate scan_feature_group(const int2* hist, const DevFeature& f, int feature, const Ctx& x,
                                               const sb2_split_config& c, ScanShared& sh, int bar) {
    FeatureCandidate o{};
    o.feature = feature;
    o.found = 0;
    o.splittable = 0;
    if (f.kind == SB2_CATEGORICAL) {
        if ((threadIdx.x % kScanThreads) < 32) o = scan_categorical(hist, f, feature, x, c, sh.order);
        return o;
    }
    if (!x.valid) return o;
    const int nb = static_cast<int>(f.num_bins);
    if (f.nan_bin && nb > 2) {
        const int last = nb - 2;
        const Grown r = group_scan(hist, last, true, last, x, c, sh, bar);
        const Grown fw = group_scan(hist, 0, false, last + 1, x, c, sh, bar);
        double output_gain = -INFINITY;
        if (r.found) {
            reverse_best(x, r, o);
            output_gain = dsub(o.best_gain, x.min_gain_shift);
            o.default_left = 1;
            o.found = 1;
            o.splittable = 1;
        }
        if (fw.found) {
            o.splittable = 1;
            FeatureCandidate b = o;
            forward_best(x, fw, b);
            if (b.best_gain > dadd(output_gain, x.min_gain_shift)) {
                o = b;
                o.default_left = 0;
                o.found = 1;
            }
        }
    } else if (nb >= 2) {
        const Grown r = group_scan(hist, nb - 1, true, nb - 1, x, c, sh, bar);
        if (r.found) {
            reverse_best(x, r, o);
            o.default_left = f.nan_bin ? 0 : 1;
            o.found = 1;
            o.splittable = 1;
        }
    }
    o.gain = dsub(o.best_gain, x.min_gain_shift);
    return o;
}

// Reads a record another CTA of the same launch may have written, past this SM's L1 (which is not coherent with
// other SMs' writes): a candidate, a leaf record.
template <class T>
__device__ __forceinline__ T load_cg(const T* p) {
    static_assert(sizeof(T) % 8 == 0 && alignof(T) >= 8, "read as 64-bit words");
    T c;
    const unsigned long long* s = reinterpret_cast<const unsigned long long*>(p);
    unsigned long long* d = reinterpret_cast<unsigned long long*>(&c);
#pragma unroll
    for (int i = 0; i < static_cast<int>(sizeof(T) / 8); ++i) d[i] = __ldcg(s + i);
    return c;
}
__device__ __forceinline__ FeatureCandidate load_candidate(const FeatureCandidate* p) { return load_cg(p); }

// better (split.rs:866-873)
__device__ __forceinline__ bool better(const FeatureCandidate& a, const FeatureCandidate& b) {
    if (!a.found) return false;
    if (!b.found) return true;
    const double ga = a.gain != a.gain ? -INFINITY : a.gain;
    const double gb = b.gain != b.gain ? -INFINITY : b.gain;
    if (ga > gb) return true;
    if (ga < gb) return false;
    return a.feature < b.feature;
}

// finish (split.rs:632-651) through split_info (:654-691): a categorical split sends its candidate's bins left, and
// the sorted scan's outputs take cat_l2 too.
__device__ sb2_split_info finish(const Ctx& x, const FeatureCandidate& b, const sb2_split_config& c) {
    sb2_split_info s{};
    s.found = 1;
    s.feature = b.feature;
    s.gain = dsub(b.best_gain, x.min_gain_shift);
    s.threshold = b.kind == kCandNumerical ? b.threshold : 0u;
    s.default_left = b.default_left;
    s.categorical = b.kind != kCandNumerical;
#pragma unroll
    for (int w = 0; w < 8; ++w) s.cat_bins[w] = b.cat_bins[w];
    const double l2 = b.kind == kCandSortedForward || b.kind == kCandSortedReverse ? dadd(c.lambda_l2, c.cat_l2)
                                                                                  : c.lambda_l2;
    s.left_grad = b.left_units_grad;
    s.left_hess = b.left_units_hess;
    s.left_count = b.left_count;
    s.right_grad = dsub(x.units_grad, b.left_units_grad);
    s.right_hess = dsub(x.units_hess, b.left_units_hess);
    s.right_count = x.num_data - b.left_count;
    s.left_output = leaf_output(b.left_grad, b.left_hess, c.lambda_l1, l2);
    s.right_output = leaf_output(dsub(x.sum_grad, b.left_grad), dsub(x.sum_hess, b.left_hess), c.lambda_l1, l2);
    return s;
}

__device__ __forceinline__ bool depth_allows(const TrainArgs& a, int depth) { return a.max_depth <= 0 || depth < a.max_depth; }
// Learner::may_split (learner.rs:172-175)
__device__ __forceinline__ bool may_split(const TrainArgs& a, int depth, int64_t left, int64_t right) {
    const int64_t min_pair = 2 * a.cfg.min_data_in_leaf;
    return depth_allows(a, depth) && (left >= min_pair || right >= min_pair);
}

__device__ __forceinline__ double nan_to_zero(double v) { return v != v ? 0.0 : v; }

// The root's LeafSums units from the bins of the sums feature (LeafSums::from_feature_hist, split.rs:101-108).
__device__ void root_units(const TrainArgs& a, double& ug, double& uh) {
    if (a.root_from_rows) {
        ug = static_cast<double>(static_cast<int64_t>(__ldcg(&a.iter->root_units[0])));
        uh = static_cast<double>(static_cast<int64_t>(__ldcg(&a.iter->root_units[1])));
        return;
    }
    const int lane = threadIdx.x & 31;
    const DevFeature f = a.d.features[a.sums_feature];
    int64_t g = 0, h = 0;
    for (uint32_t b = lane; b < f.num_bins; b += 32) {
        g += __ldcg(a.staging + 2 * (f.hist_offset + b));
        h += __ldcg(a.staging + 2 * (f.hist_offset + b) + 1);
    }
    for (int o = 16; o > 0; o >>= 1) {
        g += static_cast<int64_t>(__shfl_xor_sync(0xffffffffu, static_cast<unsigned long long>(g), o));
        h += static_cast<int64_t>(__shfl_xor_sync(0xffffffffu, static_cast<unsigned long long>(h), o));
    }
    ug = static_cast<double>(g);
    uh = static_cast<double>(h);
}

// Tree::split (tree.rs:143-177) for a numerical split of `leaf` into `leaf` and the new leaf `nl` (node nl - 1),
// without the leaf count. Splits of different leaves into different new leaves may run at once: each writes only its
// own node, leaves and child pointer (a parent's left pointer is read only by the split of its left child's leaf,
// the one that may write it).
__device__ void tree_split_at(const DevTree& t, int32_t leaf, int32_t nl, const sb2_split_info& info,
                              const DevFeature& f, int64_t left_count, int64_t right_count, double hs,
                              double min_gain_to_split) {
    // Every load before the first store, so they are in flight together; through L2, since the CTA that split
    // earlier leaves may have been another one.
    const int32_t parent = __ldcg(t.leaf_parent + leaf);
    const double old_weight = __ldcg(t.leaf_weight + leaf), old_value = __ldcg(t.leaf_value + leaf);
    const int32_t depth = __ldcg(t.leaf_depth + leaf) + 1;
    const bool parent_left = parent >= 0 && __ldcg(t.left_child + parent) == ~leaf;
    const int32_t node = nl - 1;
    if (parent >= 0) {
        if (parent_left)
            t.left_child[parent] = node;
        else
            t.right_child[parent] = node;
    }
    int8_t dt = static_cast<int8_t>((f.nan_bin ? 2 : 0) << 2);
    if (info.default_left) dt |= 2;
    // Tree::split_categorical (tree.rs:125-141): the categorical mask and MissingType::NaN; the node keeps its left
    // bins, and the host numbers the tree's categorical splits in node order (their thresholds)
    if (info.categorical) dt = static_cast<int8_t>(1 | (2 << 2));
#pragma unroll
    for (int w = 0; w < 8; ++w) t.cat_bins[8 * static_cast<size_t>(node) + w] = info.categorical ? info.cat_bins[w] : 0u;
    t.split_feature[node] = info.feature;
    t.split_gain[node] = static_cast<float>(dadd(info.gain, min_gain_to_split));
    t.threshold_bin[node] = info.threshold;
    t.decision_type[node] = dt;
    t.left_child[node] = ~leaf;
    t.right_child[node] = ~nl;
    t.internal_weight[node] = old_weight;
    t.internal_value[node] = old_value;
    t.internal_count[node] = left_count + right_count;
    t.leaf_value[leaf] = nan_to_zero(info.left_output);
    t.leaf_weight[leaf] = dmul(info.left_hess, hs);
    t.leaf_count[leaf] = left_count;
    t.leaf_value[nl] = nan_to_zero(info.right_output);
    t.leaf_weight[nl] = dmul(info.right_hess, hs);
    t.leaf_count[nl] = right_count;
    t.leaf_parent[leaf] = node;
    t.leaf_parent[nl] = node;
    t.leaf_depth[leaf] = depth;
    t.leaf_depth[nl] = depth;
}

// Tree::split as one step: the new leaf is the tree's next; returns it.
__device__ int32_t tree_split(const DevTree& t, int32_t leaf, const sb2_split_info& info, const DevFeature& f,
                              int64_t left_count, int64_t right_count, double hs, double min_gain_to_split) {
    const int32_t nl = __ldcg(t.num_leaves);
    tree_split_at(t, leaf, nl, info, f, left_count, right_count, hs, min_gain_to_split);
    *t.num_leaves = nl + 1;
    return nl;
}

// Slot of child c (0: the built one) of leaf `leaf`'s speculative split in the tree kernel (TrainArgs::slots).
__device__ __forceinline__ size_t prep_slot(const TrainArgs& a, int32_t leaf, int c) {
    return static_cast<size_t>(a.max_leaves) + 2 * static_cast<size_t>(leaf) + static_cast<size_t>(c);
}

// The children of a step as the search sees them.
struct SearchCtx {
    bool searched;
    Ctx ctx[2];          // LeafCtx of [built, other]; the root has one child
    int32_t child[2];    // their leaf indices (the root: leaf 0)
    int64_t left_global, right_global;
    const uint8_t* evaluate;
};

// LeafCtx of the step's children (learner.rs:285-336), computed by a whole warp (the root's sums are a warp
// reduction); every lane gets the same values. `left_global` is the left child's rows over every rank; `evaluate`
// and `root_mask` the features the children and the root search (global or shared memory).
__device__ SearchCtx search_context(const TrainArgs& a, const Step& st, int64_t left_global, const uint8_t* evaluate,
                                    const uint8_t* root_mask) {
    const IterState& it = *a.iter;
    const double gs = it.spec.grad_scale, hs = it.spec.hess_scale;
    SearchCtx s{};
    if (st.root) {
        s.searched = a.sums_feature >= 0 && may_split(a, 0, it.root_count, 0);
        double ug = 0.0, uh = 0.0;
        if (s.searched) root_units(a, ug, uh);
        s.ctx[0] = make_ctx(a.cfg, gs, hs, ug, uh, it.root_count);
        s.child[0] = 0;
        s.child[1] = -1;
        s.evaluate = root_mask;
    } else {
        s.left_global = left_global;
        s.right_global = st.parent_count - s.left_global;
        const int depth = st.depth + 1;
        s.searched = st.may_search && s.left_global > 0 && s.right_global > 0 &&
                     may_split(a, depth, s.left_global, s.right_global);
        const Ctx lc = make_ctx(a.cfg, gs, hs, st.info.left_grad, st.info.left_hess, s.left_global);
        const Ctx rc = make_ctx(a.cfg, gs, hs, st.info.right_grad, st.info.right_hess, s.right_global);
        s.child[0] = st.built_left ? st.leaf : st.new_leaf;
        s.child[1] = st.built_left ? st.new_leaf : st.leaf;
        s.ctx[0] = st.built_left ? lc : rc;
        s.ctx[1] = st.built_left ? rc : lc;
        s.evaluate = evaluate;
    }
    return s;
}

// search_context computed once per CTA (warp 0) into shared memory `out`, with the left count and the features from
// global memory (the standalone search: the count rides after the staging histogram, reduced over ranks); every
// thread then reads `*out`.
__device__ void search_context_cta(const TrainArgs& a, const Step& st, SearchCtx* out) {
    __syncthreads();  // every thread is done with the previous context
    if ((threadIdx.x >> 5) == 0) {
        const int64_t left = st.root ? 0 : static_cast<int64_t>(static_cast<uint32_t>(__ldcg(a.staging + 2 * a.total_bins)));
        const SearchCtx s = search_context(a, st, left, a.evaluate,
                                           a.masks + static_cast<size_t>(a.iter->iteration) * a.num_features);
        if (threadIdx.x == 0) *out = s;
    }
    __syncthreads();
}


// Work items of a step's search: one per (child, feature), item = child * F + feature; the root has one child.
__device__ __forceinline__ uint32_t search_items(const TrainArgs& a, const Step& st) {
    return (st.root ? 1u : 2u) * a.num_features;
}

// One warp, one item (child `ch`, feature `f`): the child's bins into the warp's `buf` (kMaxBins int2 of shared
// memory; `order`: kMaxBins u16 for a categorical feature's scan), its scan into `cands[ch * F + f]`. Child 0 is the built one, straight from staging; child 1 is the
// sibling, parent - built (learner.rs:365-367), and its warp also writes both children's slots (it alone reads
// the parent's slot, which the built child may take over), or, at the root, child 0's warp writes the root's slot.
// Every lane loads its bins (lane, lane + 32, ...) before using any, so a warp waits on memory once.
__device__ void search_item(const TrainArgs& a, const Step& st, const SearchCtx& s, uint32_t item, int2* buf,
                            uint16_t* order) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t F = a.num_features;
    const uint32_t f = item % F, ch = item / F;
    FeatureCandidate* cands = static_cast<FeatureCandidate*>(a.candidates);
    const DevFeature feat = a.d.features[f];
    if (!load_flag(s.evaluate + f) || feat.tile < 0 || feat.num_bins == 0) {
        if (lane == 0) {
            FeatureCandidate none{};
            none.feature = static_cast<int32_t>(f);
            cands[f] = none;
            cands[F + f] = none;
            if (a.cand_flags) {
                a.cand_flags[f] = 0;
                a.cand_flags[F + f] = 0;
            }
        }
        return;
    }
    const size_t slot_len = 2 * static_cast<size_t>(a.total_bins);
    const size_t off = 2 * static_cast<size_t>(feat.hist_offset);
    const int2* staged = reinterpret_cast<const int2*>(a.staging + off);
    int2 built[kPerLane], other[kPerLane];
#pragma unroll
    for (int k = 0; k < kPerLane; ++k) {
        const uint32_t b = lane + 32u * k;
        built[k] = b < feat.num_bins ? __ldcg(staged + b) : make_int2(0, 0);
    }
    if (ch == 1) {
        const int2* parent = reinterpret_cast<const int2*>(a.slots + static_cast<size_t>(st.leaf) * slot_len + off);
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
            const uint32_t b = lane + 32u * k;
            other[k] = b < feat.num_bins ? __ldcg(parent + b) : make_int2(0, 0);
        }
        int2* built_slot = reinterpret_cast<int2*>(a.slots + static_cast<size_t>(s.child[0]) * slot_len + off);
        int2* other_slot = reinterpret_cast<int2*>(a.slots + static_cast<size_t>(s.child[1]) * slot_len + off);
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
            const uint32_t b = lane + 32u * k;
            other[k] = make_int2(other[k].x - built[k].x, other[k].y - built[k].y);
            if (b < feat.num_bins) {
                __stcg(built_slot + b, built[k]);
                __stcg(other_slot + b, other[k]);
                buf[b] = other[k];
            }
        }
    } else {
        int2* slot = st.root ? reinterpret_cast<int2*>(a.slots + off) : nullptr;
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
            const uint32_t b = lane + 32u * k;
            if (b < feat.num_bins) {
                if (slot) __stcg(slot + b, built[k]);
                buf[b] = built[k];
            }
        }
    }
    __syncwarp();
    const FeatureCandidate c = scan_feature(buf, feat, static_cast<int>(f), s.ctx[ch], a.cfg, order);
    if (lane == 0) {
        cands[static_cast<size_t>(ch) * F + f] = c;
        if (a.cand_flags) {  // what the persistent kernel's finish compares, apart from the full candidate
            a.cand_flags[static_cast<size_t>(ch) * F + f] = static_cast<uint8_t>((c.found ? 1 : 0) | (c.splittable ? 2 : 0));
            a.cand_gain[static_cast<size_t>(ch) * F + f] = c.gain;
        }
        if (st.root) {
            FeatureCandidate none{};
            none.feature = static_cast<int32_t>(f);
            cands[F + f] = none;
            if (a.cand_flags) a.cand_flags[F + f] = 0;
        }
    }
    __syncwarp();
}

// search_item for a group of kScanWarps warps (named barrier `bar`): thread t loads bin t, and the group scans the
// child's bins in `buf` (kMaxBins int2 of the group's shared memory) with scan_feature_group. The same loads, slot
// writes and candidate as search_item.
__device__ void search_item_group(const TrainArgs& a, const Step& st, const SearchCtx& s, uint32_t item, int2* buf,
                                  ScanShared& sh, int bar) {
    const uint32_t t = threadIdx.x % kScanThreads;
    const uint32_t F = a.num_features;
    const uint32_t f = item % F, ch = item / F;
    FeatureCandidate* cands = static_cast<FeatureCandidate*>(a.candidates);
    const DevFeature feat = a.d.features[f];
    if (!load_flag(s.evaluate + f) || feat.tile < 0 || feat.num_bins == 0) {
        if (t == 0) {
            FeatureCandidate none{};
            none.feature = static_cast<int32_t>(f);
            cands[f] = none;
            cands[F + f] = none;
            if (a.cand_flags) {
                a.cand_flags[f] = 0;
                a.cand_flags[F + f] = 0;
            }
        }
        return;
    }
    const size_t slot_len = 2 * static_cast<size_t>(a.total_bins);
    const size_t off = 2 * static_cast<size_t>(feat.hist_offset);
    const bool mine = t < feat.num_bins;
    const int2 built = mine ? __ldcg(reinterpret_cast<const int2*>(a.staging + off) + t) : make_int2(0, 0);
    if (ch == 1) {
        const int2* parent = reinterpret_cast<const int2*>(a.slots + static_cast<size_t>(st.leaf) * slot_len + off);
        const int2 p = mine ? __ldcg(parent + t) : make_int2(0, 0);
        if (mine) {
            const int2 other = make_int2(p.x - built.x, p.y - built.y);
            __stcg(reinterpret_cast<int2*>(a.slots + static_cast<size_t>(s.child[0]) * slot_len + off) + t, built);
            __stcg(reinterpret_cast<int2*>(a.slots + static_cast<size_t>(s.child[1]) * slot_len + off) + t, other);
            buf[t] = other;
        }
    } else if (mine) {
        if (st.root) __stcg(reinterpret_cast<int2*>(a.slots + off) + t, built);
        buf[t] = built;
    }
    group_sync(bar);
    const FeatureCandidate c = scan_feature_group(buf, feat, static_cast<int>(f), s.ctx[ch], a.cfg, sh, bar);
    if (t == 0) {
        cands[static_cast<size_t>(ch) * F + f] = c;
        if (a.cand_flags) {  // what the persistent kernel's finish compares, apart from the full candidate
            a.cand_flags[static_cast<size_t>(ch) * F + f] = static_cast<uint8_t>((c.found ? 1 : 0) | (c.splittable ? 2 : 0));
            a.cand_gain[static_cast<size_t>(ch) * F + f] = c.gain;
        }
        if (st.root) {
            FeatureCandidate none{};
            none.feature = static_cast<int32_t>(f);
            cands[F + f] = none;
            if (a.cand_flags) a.cand_flags[F + f] = 0;
        }
    }
    group_sync(bar);  // buf and the scratch are free for the group's next item
}

// The warp's best of its lanes' candidates by `better` (on found, gain and feature alone; the winner's full record
// is read back from `cands`, indexed by feature). Every lane gets it.
__device__ __forceinline__ FeatureCandidate best_of_warp(const FeatureCandidate& mine, const FeatureCandidate* cands) {
    const uint32_t lane = threadIdx.x & 31;
    FeatureCandidate best{};
    best.found = mine.found;
    best.gain = mine.gain;
    best.feature = mine.feature;
    for (int o = 16; o > 0; o >>= 1) {
        FeatureCandidate other{};
        const int src = static_cast<int>(lane) ^ o;
        other.found = __shfl_sync(0xffffffffu, best.found, src);
        other.gain = __shfl_sync(0xffffffffu, best.gain, src);
        other.feature = __shfl_sync(0xffffffffu, best.feature, src);
        if (better(other, best)) best = other;
    }
    if (!best.found) return best;
    FeatureCandidate full = load_candidate(cands + best.feature);
    full.splittable = 0;
    return full;
}

// The best candidate of child `ch` over every feature (one warp; `better` is a total order, so the reduction order
// does not matter), with the child's splittable flags written on the way.
__device__ FeatureCandidate best_candidate(const TrainArgs& a, const SearchCtx& s, int ch) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t F = a.num_features;
    const FeatureCandidate* cands = static_cast<const FeatureCandidate*>(a.candidates) + static_cast<size_t>(ch) * F;
    uint8_t* splittable = a.splittable + static_cast<size_t>(s.child[ch]) * F;
    FeatureCandidate best{};
    best.found = 0;
    // Four candidates per lane in flight at a time.
    for (uint32_t f0 = 0; f0 < F; f0 += 128) {
        FeatureCandidate c[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t f = f0 + 32u * j + lane;
            if (f < F) c[j] = load_candidate(cands + f);
            else c[j].found = 0;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t f = f0 + 32u * j + lane;
            if (f < F) {
                splittable[f] = static_cast<uint8_t>(c[j].splittable);
                if (better(c[j], best)) best = c[j];
            }
        }
    }
    return best_of_warp(best, cands);
}

// (gain, leaf) of the better of two leaves in best_leaf's order (learner.rs:418-429): the higher gain, on equal
// gains the lower index; -1 is no leaf.
__device__ __forceinline__ void prefer_leaf(double& gain, int32_t& leaf, double og, int32_t ol) {
    if (ol >= 0 && (leaf < 0 || og > gain || (og == gain && ol < leaf))) {
        leaf = ol;
        gain = og;
    }
}

// bin_split (learner.rs:432-452): bins 0..=threshold go left, and the NaN bin when missing values go left.
__device__ __forceinline__ void left_bins_of(const sb2_split_info& info, const DevFeature& f, uint32_t (&bins)[8]) {
    if (info.categorical) {  // SplitRule::Categorical: its bins
#pragma unroll
        for (int w = 0; w < 8; ++w) bins[w] = info.cat_bins[w];
        return;
    }
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const int64_t first = 32 * w, t = static_cast<int64_t>(info.threshold);
        bins[w] = t >= first + 31 ? 0xFFFFFFFFu : t >= first ? (0xFFFFFFFFu >> (31 - (t - first))) : 0u;
    }
    if (info.default_left && f.nan_bin) bins[(f.num_bins - 1) >> 5] |= 1u << ((f.num_bins - 1) & 31);
}

// The step that splits `leaf` (index `index`, its best split chosen; `f` the split's feature) into `index` and
// `num_leaves`: Learner::split_leaf's inputs (learner.rs:249-275).
__device__ Step next_step(const TrainArgs& a, const DevLeaf& leaf, int32_t index, int32_t num_leaves,
                          const DevFeature& f) {
    const sb2_split_info& info = leaf.best;
    Step n{};
    n.active = 1;
    n.root = 0;
    n.leaf = index;
    n.new_leaf = num_leaves;
    n.may_search = leaf.has_hist && num_leaves + 1 < a.max_leaves && depth_allows(a, leaf.depth + 1);
    n.built_left = info.left_count <= info.right_count;
    n.begin = leaf.begin;
    n.count = leaf.count;
    n.which = leaf.which;
    n.depth = leaf.depth;
    n.split_tile = static_cast<uint32_t>(f.tile);
    n.split_lane = static_cast<uint32_t>(f.lane);
    left_bins_of(info, f, n.left_bins);
    n.parent_count = leaf.count_global;
    n.info = info;
    return n;
}

// After every item's candidate is written: the split applied to the tree and the leaves, each child's best split,
// and the next step (learner.rs:158-163, 249-352, 418-429). One CTA of at least 128 threads. The independent parts
// run side by side so the CTA waits on memory about twice: warp 0 applies the split, warps 1-2 reduce the
// children's candidates, warp 3 finds the best of the other leaves; then warp 0 joins them and writes the step.
__device__ void search_finish(const TrainArgs& a, const Step& st, const SearchCtx& s) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t F = a.num_features;
    const IterState& it = *a.iter;
    DevLeaf* leaves = a.leaves;
    const int children = st.root ? 1 : 2;
    __shared__ DevLeaf s_child[2];           // the children's new leaf records (warp 0)
    __shared__ sb2_split_info s_best[2];     // their best splits (warps 1-2)
    __shared__ int32_t s_has_best[2];
    __shared__ double s_other_gain;          // best of the leaves that are not children (warp 3)
    __shared__ int32_t s_other_leaf;
    if (warp == 0) {
        if (lane == 0) {
            const double hs = it.spec.hess_scale;
            if (st.root) {
                DevLeaf l = load_cg(leaves);
                l.units_grad = s.ctx[0].units_grad;
                l.units_hess = s.ctx[0].units_hess;
                l.count_global = it.root_count;
                l.has_hist = s.searched;
                l.has_best = 0;
                s_child[0] = l;
            } else {
                if (s.left_global <= 0 || s.right_global <= 0) {
                    a.iter->error = 1;  // split sends every row to one side (learner.rs:295-300)
                    a.iter->error_info = st.leaf;
                }
                const DevLeaf parent = load_cg(leaves + st.leaf);
                const DevFeature f = a.d.features[st.info.feature];
                const int32_t nl = tree_split(a.tree, st.leaf, st.info, f, s.left_global, s.right_global, hs,
                                              a.cfg.min_gain_to_split);
                if (nl != st.new_leaf) {
                    a.iter->error = 2;
                    a.iter->error_info = nl;
                }
                DevLeaf l{}, r{};
                l.begin = parent.begin;
                l.count = st.local_left;
                r.begin = parent.begin + st.local_left;
                r.count = parent.count - st.local_left;
                l.which = r.which = parent.which ^ 1u;
                l.depth = r.depth = parent.depth + 1;
                l.units_grad = st.info.left_grad;
                l.units_hess = st.info.left_hess;
                l.count_global = s.left_global;
                r.units_grad = st.info.right_grad;
                r.units_hess = st.info.right_hess;
                r.count_global = s.right_global;
                l.has_hist = r.has_hist = s.searched;
                // child 0 is the built child: the left one (index st.leaf) when built_left
                s_child[st.built_left ? 0 : 1] = l;
                s_child[st.built_left ? 1 : 0] = r;
            }
        }
    } else if (warp <= 2) {
        const int ch = static_cast<int>(warp) - 1;
        if (ch < children) {
            FeatureCandidate best{};
            best.found = 0;
            if (s.searched) best = best_candidate(a, s, ch);
            if (lane == 0) {
                const bool has = best.found && s.ctx[ch].valid;
                s_has_best[ch] = has;
                s_best[ch] = has ? finish(s.ctx[ch], best, a.cfg) : sb2_split_info{};
            }
        }
    } else if (warp == 3) {
        // Leaves that existed before this step, other than the one being split.
        const int32_t before = st.root ? 0 : st.new_leaf;
        double gain = -INFINITY;
        int32_t leaf = -1;
        for (int32_t l0 = 0; l0 < before; l0 += 128) {
            int32_t has[4];
            double g[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int32_t l = l0 + 32 * j + static_cast<int32_t>(lane);
                has[j] = l < before && l != st.leaf ? __ldcg(&leaves[l].has_best) : 0;
                g[j] = has[j] ? __ldcg(&leaves[l].best.gain) : 0.0;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (has[j]) prefer_leaf(gain, leaf, g[j], l0 + 32 * j + static_cast<int32_t>(lane));
        }
        for (int o = 16; o > 0; o >>= 1)
            prefer_leaf(gain, leaf, __shfl_xor_sync(0xffffffffu, gain, o), __shfl_xor_sync(0xffffffffu, leaf, o));
        if (lane == 0) {
            s_other_gain = gain;
            s_other_leaf = leaf;
        }
    }
    __syncthreads();
    if (warp != 0) return;
    // Join: the children's records get their best splits and go out, then the best leaf over children and others.
    if (lane < static_cast<uint32_t>(children)) {
        s_child[lane].has_best = s_has_best[lane];
        if (s_has_best[lane]) s_child[lane].best = s_best[lane];
    }
    __syncwarp();
    double gain = s_other_gain;
    int32_t best_leaf = s_other_leaf;
    for (int ch = 0; ch < children; ++ch) {
        const DevLeaf& c = s_child[ch];
        if (c.has_best) prefer_leaf(gain, best_leaf, c.best.gain, s.child[ch]);
    }
    const int32_t num_leaves = st.root ? 1 : st.new_leaf + 1;
    const bool go = best_leaf >= 0 && gain > 0.0 && num_leaves < a.max_leaves;
    const int chosen = !go ? -1 : best_leaf == s.child[0] ? 0 : (children == 2 && best_leaf == s.child[1]) ? 1 : -1;
    if (lane < static_cast<uint32_t>(children)) {
        DevLeaf c = s_child[lane];
        if (static_cast<int>(lane) == chosen) c.has_best = 0;  // it is split next
        leaves[s.child[lane]] = c;
    }
    Step* next = a.step;
    if (!go) {
        if (lane == 0) next->active = 0;
        return;
    }
    DevLeaf leaf;
    if (chosen >= 0) {
        leaf = s_child[chosen];
    } else {
        leaf = load_cg(leaves + best_leaf);
        if (lane == 0) leaves[best_leaf].has_best = 0;
    }
    const sb2_split_info info = leaf.best;
    const DevFeature f = a.d.features[info.feature];
    // Features the children evaluate: the tree's mask and the parent's splittable ones (learner.rs:278-284).
    const uint8_t* mask = a.masks + static_cast<size_t>(it.iteration) * F;
    const uint8_t* split_ok = a.splittable + static_cast<size_t>(best_leaf) * F;
    for (uint32_t k0 = 0; k0 < F; k0 += 128) {
        uint8_t m[4], o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t k = k0 + 32u * j + lane;
            m[j] = k < F ? mask[k] : 0;
            o[j] = k < F ? __ldcg(split_ok + k) : 0;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t k = k0 + 32u * j + lane;
            if (k < F) a.evaluate[k] = static_cast<uint8_t>(m[j] && o[j]);
        }
    }
    if (lane == 0) *next = next_step(a, leaf, best_leaf, num_leaves, f);
}

// Whether CTA `cta` writes part `part` of a finish (CTA `part`, or CTA 0 in a grid of fewer than four).
__device__ __forceinline__ bool writes_part(uint32_t cta, uint32_t part) { return cta == (part < gridDim.x ? part : 0u); }

}  // namespace

}  // namespace sb2
