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
__device__ __forceinline__ double ddiv(double a, double b) { return __ddiv_rn(a, b); }

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
    // Gains of the candidates before the break (ScanBuffer::evaluate).
    double gain[kPerLane];
    double mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int k = lane * kPerLane + i;
        gain[i] = -INFINITY;
        if (k < first_break) {
            const double uh = static_cast<double>(H[i]);
            const double hh = dadd(kEpsilon, dmul(uh, x.hs));
            const bool skip = C[i] < min_count || hh < c.min_sum_hessian_in_leaf || uh <= 0.0;
            if (!skip) {
                const double g = dmul(static_cast<double>(G[i]), x.gs);
                gain[i] = dadd(leaf_gain(dsub(x.sum_grad, g), dsub(x.sum_hess, hh), c.lambda_l1, c.lambda_l2),
                               leaf_gain(g, hh, c.lambda_l1, c.lambda_l2));
            }
            mx = fmax(mx, gain[i]);
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

// find_numerical (split.rs:584-620) for one feature.
__device__ FeatureCandidate scan_feature(const int2* hist, const DevFeature& f, int feature, const Ctx& x,
                                         const sb2_split_config& c) {
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

// Reads a candidate another CTA wrote, past this SM's L1 (the last CTA of a launch reads every CTA's results).
__device__ FeatureCandidate load_candidate(const FeatureCandidate* p) {
    FeatureCandidate c;
    const unsigned long long* s = reinterpret_cast<const unsigned long long*>(p);
    unsigned long long* d = reinterpret_cast<unsigned long long*>(&c);
#pragma unroll
    for (int i = 0; i < static_cast<int>(sizeof(FeatureCandidate) / 8); ++i) d[i] = __ldcg(s + i);
    return c;
}

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

// finish (split.rs:632-651)
__device__ sb2_split_info finish(const Ctx& x, const FeatureCandidate& b, const sb2_split_config& c) {
    sb2_split_info s{};
    s.found = 1;
    s.feature = b.feature;
    s.gain = dsub(b.best_gain, x.min_gain_shift);
    s.threshold = b.threshold;
    s.default_left = b.default_left;
    s.left_grad = b.left_units_grad;
    s.left_hess = b.left_units_hess;
    s.left_count = b.left_count;
    s.right_grad = dsub(x.units_grad, b.left_units_grad);
    s.right_hess = dsub(x.units_hess, b.left_units_hess);
    s.right_count = x.num_data - b.left_count;
    s.left_output = leaf_output(b.left_grad, b.left_hess, c.lambda_l1, c.lambda_l2);
    s.right_output = leaf_output(dsub(x.sum_grad, b.left_grad), dsub(x.sum_hess, b.left_hess), c.lambda_l1, c.lambda_l2);
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

// Tree::split (tree.rs:143-177) for a numerical split; returns the new leaf.
__device__ int32_t tree_split(const DevTree& t, int32_t leaf, const sb2_split_info& info, const DevFeature& f,
                              int64_t left_count, int64_t right_count, double hs, double min_gain_to_split) {
    const int32_t nl = *t.num_leaves;
    const int32_t node = nl - 1;
    const int32_t parent = t.leaf_parent[leaf];
    if (parent >= 0) {
        if (t.left_child[parent] == ~leaf)
            t.left_child[parent] = node;
        else
            t.right_child[parent] = node;
    }
    int8_t dt = static_cast<int8_t>((f.nan_bin ? 2 : 0) << 2);
    if (info.default_left) dt |= 2;
    t.split_feature[node] = info.feature;
    t.split_gain[node] = static_cast<float>(dadd(info.gain, min_gain_to_split));
    t.threshold_bin[node] = info.threshold;
    t.decision_type[node] = dt;
    t.left_child[node] = ~leaf;
    t.right_child[node] = ~nl;
    t.internal_weight[node] = t.leaf_weight[leaf];
    t.internal_value[node] = t.leaf_value[leaf];
    t.internal_count[node] = left_count + right_count;
    t.leaf_value[leaf] = nan_to_zero(info.left_output);
    t.leaf_weight[leaf] = dmul(info.left_hess, hs);
    t.leaf_count[leaf] = left_count;
    t.leaf_value[nl] = nan_to_zero(info.right_output);
    t.leaf_weight[nl] = dmul(info.right_hess, hs);
    t.leaf_count[nl] = right_count;
    t.leaf_parent[leaf] = node;
    t.leaf_parent[nl] = node;
    const int32_t depth = t.leaf_depth[leaf] + 1;
    t.leaf_depth[leaf] = depth;
    t.leaf_depth[nl] = depth;
    *t.num_leaves = nl + 1;
    return nl;
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
// reduction); every lane gets the same values.
__device__ SearchCtx search_context(const TrainArgs& a, const Step& st) {
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
        s.evaluate = a.masks + static_cast<size_t>(it.iteration) * a.num_features;
    } else {
        s.left_global = static_cast<int64_t>(static_cast<uint32_t>(__ldcg(a.staging + 2 * a.total_bins)));
        s.right_global = st.parent_count - s.left_global;
        const int depth = __ldcg(&a.leaves[st.leaf].depth) + 1;
        s.searched = st.may_search && s.left_global > 0 && s.right_global > 0 &&
                     may_split(a, depth, s.left_global, s.right_global);
        const Ctx lc = make_ctx(a.cfg, gs, hs, st.info.left_grad, st.info.left_hess, s.left_global);
        const Ctx rc = make_ctx(a.cfg, gs, hs, st.info.right_grad, st.info.right_hess, s.right_global);
        s.child[0] = st.built_left ? st.leaf : st.new_leaf;
        s.child[1] = st.built_left ? st.new_leaf : st.leaf;
        s.ctx[0] = st.built_left ? lc : rc;
        s.ctx[1] = st.built_left ? rc : lc;
        s.evaluate = a.evaluate;
    }
    return s;
}

// search_context computed once per CTA (warp 0) into shared memory `out`; every thread then reads `*out`.
__device__ void search_context_cta(const TrainArgs& a, const Step& st, SearchCtx* out) {
    __syncthreads();  // every thread is done with the previous context
    if ((threadIdx.x >> 5) == 0) {
        const SearchCtx s = search_context(a, st);
        if (threadIdx.x == 0) *out = s;
    }
    __syncthreads();
}

// One warp, one feature: the built child's bins from staging, the other's as parent - built, written into both
// leaves' slots (learner.rs:365-367), then each child's scan into `cands` ([child][feature]). `buf` is the warp's
// 2 x kMaxBins int2 of shared memory.
__device__ void search_feature(const TrainArgs& a, const Step& st, const SearchCtx& s, uint32_t f, int2 (*buf)[kMaxBins]) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t F = a.num_features;
    FeatureCandidate* cands = static_cast<FeatureCandidate*>(a.candidates);
    const DevFeature feat = a.d.features[f];
    FeatureCandidate none{};
    none.feature = static_cast<int32_t>(f);
    if (!__ldcg(s.evaluate + f) || feat.tile < 0 || feat.num_bins == 0) {
        if (lane == 0) {
            cands[f] = none;
            cands[F + f] = none;
        }
        return;
    }
    const int children = st.root ? 1 : 2;
    const size_t slot_len = 2 * static_cast<size_t>(a.total_bins);
    const size_t off = 2 * static_cast<size_t>(feat.hist_offset);
    int* built_slot = a.slots + static_cast<size_t>(s.child[0]) * slot_len + off;
    int* other_slot = children == 2 ? a.slots + static_cast<size_t>(s.child[1]) * slot_len + off : nullptr;
    const int* parent_slot = a.slots + static_cast<size_t>(st.root ? 0 : st.leaf) * slot_len + off;
    for (uint32_t b = lane; b < feat.num_bins; b += 32) {
        const int sg = __ldcg(a.staging + off + 2 * b), shh = __ldcg(a.staging + off + 2 * b + 1);
        buf[0][b] = make_int2(sg, shh);
        if (children == 2) {
            const int pg = __ldcg(parent_slot + 2 * b), ph = __ldcg(parent_slot + 2 * b + 1);
            buf[1][b] = make_int2(pg - sg, ph - shh);
        }
    }
    __syncwarp();
    // Slot writes after every lane has read the parent (the built child may reuse the parent's slot).
    for (uint32_t b = lane; b < feat.num_bins; b += 32) {
        __stcg(reinterpret_cast<int2*>(built_slot) + b, buf[0][b]);
        if (children == 2) __stcg(reinterpret_cast<int2*>(other_slot) + b, buf[1][b]);
    }
    for (int ch = 0; ch < children; ++ch) {
        const FeatureCandidate c = scan_feature(buf[ch], feat, static_cast<int>(f), s.ctx[ch], a.cfg);
        if (lane == 0) cands[static_cast<size_t>(ch) * F + f] = c;
    }
    if (children == 1 && lane == 0) cands[F + f] = none;
    __syncwarp();
}

// After every feature's candidates are written: the split applied to the tree and the leaves, each child's best
// split, and the next step (learner.rs:158-163, 249-352, 418-429). One CTA of at least 64 threads.
__device__ void search_finish(const TrainArgs& a, const Step& st, const SearchCtx& s) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t F = a.num_features;
    const IterState& it = *a.iter;
    const double hs = it.spec.hess_scale;
    FeatureCandidate* cands = static_cast<FeatureCandidate*>(a.candidates);
    DevLeaf* leaves = a.leaves;
    if (threadIdx.x == 0) {
        if (st.root) {
            DevLeaf& l = leaves[0];
            l.units_grad = s.ctx[0].units_grad;
            l.units_hess = s.ctx[0].units_hess;
            l.count_global = it.root_count;
            l.has_hist = s.searched;
            l.has_best = 0;
        } else {
            if (s.left_global <= 0 || s.right_global <= 0) {
                a.iter->error = 1;  // split sends every row to one side (learner.rs:295-300)
                a.iter->error_info = st.leaf;
            }
            const DevLeaf parent = leaves[st.leaf];
            const DevFeature f = a.d.features[st.info.feature];
            const int32_t nl =
                tree_split(a.tree, st.leaf, st.info, f, s.left_global, s.right_global, hs, a.cfg.min_gain_to_split);
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
            leaves[st.leaf] = l;
            leaves[nl] = r;
        }
    }
    __syncthreads();
    if (s.searched && warp < (st.root ? 1u : 2u)) {
        // Best candidate of child `warp` over every feature.
        FeatureCandidate best{};
        best.found = 0;
        for (uint32_t f = lane; f < F; f += 32) {
            const FeatureCandidate c = load_candidate(cands + static_cast<size_t>(warp) * F + f);
            a.splittable[static_cast<size_t>(s.child[warp]) * F + f] = static_cast<uint8_t>(c.splittable);
            if (better(c, best)) best = c;
        }
        for (int o = 16; o > 0; o >>= 1) {
            FeatureCandidate other;
            const int src = lane ^ o;
            other.found = __shfl_sync(0xffffffffu, best.found, src);
            other.splittable = 0;
            other.feature = __shfl_sync(0xffffffffu, best.feature, src);
            other.default_left = __shfl_sync(0xffffffffu, best.default_left, src);
            other.gain = __shfl_sync(0xffffffffu, best.gain, src);
            other.best_gain = __shfl_sync(0xffffffffu, best.best_gain, src);
            other.threshold = __shfl_sync(0xffffffffu, best.threshold, src);
            other.left_grad = __shfl_sync(0xffffffffu, best.left_grad, src);
            other.left_hess = __shfl_sync(0xffffffffu, best.left_hess, src);
            other.left_count = shfl_i64(best.left_count, src);
            other.left_units_grad = __shfl_sync(0xffffffffu, best.left_units_grad, src);
            other.left_units_hess = __shfl_sync(0xffffffffu, best.left_units_hess, src);
            if (better(other, best)) best = other;
        }
        if (lane == 0) {
            DevLeaf& l = leaves[s.child[warp]];
            if (best.found && s.ctx[warp].valid) {
                l.best = finish(s.ctx[warp], best, a.cfg);
                l.has_best = 1;
            } else {
                l.has_best = 0;
            }
        }
    }
    __syncthreads();
    if (warp == 0) {
        // best_leaf (learner.rs:418-429): the first maximum gain over leaves with a split; continue when positive.
        const int32_t num_leaves = *a.tree.num_leaves;
        double best_gain = -INFINITY;
        int32_t best_leaf = -1;
        for (int32_t l = lane; l < num_leaves; l += 32) {
            if (leaves[l].has_best) {
                const double g = leaves[l].best.gain;
                if (best_leaf < 0 || g > best_gain) {
                    best_leaf = l;
                    best_gain = g;
                }
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const double og = __shfl_xor_sync(0xffffffffu, best_gain, o);
            const int32_t ol = __shfl_xor_sync(0xffffffffu, best_leaf, o);
            if (ol >= 0 && (best_leaf < 0 || og > best_gain || (og == best_gain && ol < best_leaf))) {
                best_leaf = ol;
                best_gain = og;
            }
        }
        Step* next = a.step;
        if (best_leaf < 0 || !(best_gain > 0.0) || num_leaves >= a.max_leaves) {
            if (lane == 0) next->active = 0;
        } else {
            const DevLeaf leaf = leaves[best_leaf];
            const sb2_split_info info = leaf.best;
            const DevFeature f = a.d.features[info.feature];
            // Features the children evaluate: the tree's mask and the parent's splittable ones (learner.rs:278-284).
            const uint8_t* mask = a.masks + static_cast<size_t>(it.iteration) * F;
            for (uint32_t k = lane; k < F; k += 32)
                a.evaluate[k] = static_cast<uint8_t>(mask[k] && a.splittable[static_cast<size_t>(best_leaf) * F + k]);
            if (lane == 0) {
                leaves[best_leaf].has_best = 0;
                Step n{};
                n.active = 1;
                n.root = 0;
                n.leaf = best_leaf;
                n.new_leaf = num_leaves;
                n.may_search = leaf.has_hist && num_leaves + 1 < a.max_leaves && depth_allows(a, leaf.depth + 1);
                n.built_left = info.left_count <= info.right_count;
                n.begin = leaf.begin;
                n.count = leaf.count;
                n.which = leaf.which;
                n.split_tile = static_cast<uint32_t>(f.tile);
                n.split_lane = static_cast<uint32_t>(f.lane);
                // bin_split (learner.rs:432-452)
                for (uint32_t b = 0; b <= info.threshold && b < 256; ++b) n.left_bins[b >> 5] |= 1u << (b & 31);
                if (info.default_left && f.nan_bin) n.left_bins[(f.num_bins - 1) >> 5] |= 1u << ((f.num_bins - 1) & 31);
                n.parent_count = leaf.count_global;
                n.info = info;
                *next = n;
            }
        }
    }
}

}  // namespace

}  // namespace sb2
