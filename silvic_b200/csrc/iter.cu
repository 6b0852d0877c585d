// iter.cu — per-iteration kernels of the boosting loop and the Backend-API kernels.
//
//  gradients        objective::gradients (objective/regression.rs:20-43, binary.rs:27-50) and the local maxima of
//                   CpuBackend::compute_gradients (backend/cpu.rs:757-780); binary gradients in f64, stored f32.
//  iteration_start  QuantSpec::new (quantize.rs:56-84) from the reduced maxima, CpuBackend::quantize
//                   (backend/cpu.rs:782-800), reset_partition(All) and the root's step.
//  leaf_sums        CpuBackend::leaf_sums (backend/cpu.rs:886-908) for every leaf of the grown tree.
//  finalize         Learner::renew_leaves (learner.rs:376-404) and Trainer::add (boosting.rs:313-324): renewal,
//                   shrinkage, the first tree's bias, and the tree's record; a tree that cannot split ends training
//                   (Trainer::single_leaf, boosting.rs:303-310).
//  add_tree         the score update: each leaf's f32 value added to its rows (the partition holds every training
//                   row in exactly one leaf without bagging), the same f32 add CpuBackend::add_tree makes.
#include <cuda_runtime.h>

#include <algorithm>

#include "iter.cuh"

namespace sb2 {

namespace {

constexpr double kZeroThreshold = static_cast<double>(1e-35f);

__device__ __forceinline__ double round_to_zero(double v) { return fabs(v) > kZeroThreshold ? v : 0.0; }

// quantize.rs:92-98
__device__ __forceinline__ double positive_or_one(double v) { return (v > 0.0 && isfinite(v)) ? v : 1.0; }

// QuantSpec::new (quantize.rs:56-84)
__device__ sb2_quant_spec make_spec(double max_abs_grad, double max_hess, const IterConsts& k, uint32_t iteration) {
    sb2_quant_spec s{};
    s.grad_max_q = k.num_grad_quant_bins / 2;
    s.hess_max_q = k.num_grad_quant_bins;
    s.grad_scale = positive_or_one(__ddiv_rn(max_abs_grad, static_cast<double>(s.grad_max_q)));
    s.hess_scale = k.constant_hessian ? 1.0 : positive_or_one(__ddiv_rn(max_hess, static_cast<double>(s.hess_max_q)));
    s.inv_grad_scale = __double2float_rn(__ddiv_rn(1.0, s.grad_scale));
    s.inv_hess_scale = __double2float_rn(__ddiv_rn(1.0, s.hess_scale));
    s.constant_hessian = k.constant_hessian;
    s.stochastic = k.stochastic;
    s.seed = k.seed;
    s.iteration = iteration;
    return s;
}

// fixed_point_scale (quantize.rs:153-159): 2^(30 - ceil(log2 max_abs)). For the f32-valued maxima it is called with,
// ceil(log2 x) is exactly the frexp exponent (less one at a power of two).
__device__ float fixed_point_scale(double max_abs) {
    if (!isfinite(max_abs) || max_abs <= 0.0) return 1.0f;
    int e;
    const double m = frexp(max_abs, &e);
    const int ceil_log2 = (m == 0.5) ? e - 1 : e;
    int exponent = 30 - ceil_log2;
    exponent = exponent < -126 ? -126 : (exponent > 127 ? 127 : exponent);
    return ldexpf(1.0f, exponent);
}

__device__ __forceinline__ int64_t to_fixed(float v, float scale) {
    const float q = rintf(__fmul_rn(v, scale));
    if (q != q) return 0;
    if (q >= 9.2233720368547758e18f) return INT64_MAX;
    if (q <= -9.2233720368547758e18f) return INT64_MIN;
    return static_cast<int64_t>(q);
}

// Gradients of one row.
__device__ __forceinline__ void row_gradient(const RowArgs& r, uint64_t row, float& g, float& h) {
    if (r.objective == SB2_REGRESSION) {
        const float residual = __fsub_rn(r.scores[row], r.label[row]);
        if (r.weight) {
            g = __fmul_rn(residual, r.weight[row]);
            h = r.weight[row];
        } else {
            g = residual;
            h = 1.0f;
        }
    } else {
        const double sign = r.label[row] > 0.0f ? 1.0 : -1.0;
        const double sigmoid = r.sigmoid;
        const double response =
            __ddiv_rn(__dmul_rn(-sign, sigmoid),
                      __dadd_rn(1.0, exp(__dmul_rn(__dmul_rn(sign, sigmoid), static_cast<double>(r.scores[row])))));
        const double abs_response = fabs(response);
        const double w = r.weight ? static_cast<double>(r.weight[row]) : 1.0;
        g = __double2float_rn(__dmul_rn(response, w));
        h = __double2float_rn(__dmul_rn(__dmul_rn(abs_response, __dsub_rn(sigmoid, abs_response)), w));
    }
}

__device__ __forceinline__ void block_max_pair(double& a, double& b) {
    __shared__ double sa[kRowThreads / 32], sb[kRowThreads / 32];
    for (int o = 16; o > 0; o >>= 1) {
        a = fmax(a, __shfl_xor_sync(0xffffffffu, a, o));
        b = fmax(b, __shfl_xor_sync(0xffffffffu, b, o));
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sa[warp] = a;
        sb[warp] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < kRowThreads / 32; ++k) {
            a = fmax(a, sa[k]);
            b = fmax(b, sb[k]);
        }
        a = fmax(a, sa[0]);
        b = fmax(b, sb[0]);
    }
}

__device__ void gradients_body(const RowArgs& r, unsigned long long* max_g, unsigned long long* max_h) {
    double mg = 0.0, mh = 0.0;
    for (uint64_t row = static_cast<uint64_t>(blockIdx.x) * kRowThreads + threadIdx.x; row < r.num_rows;
         row += static_cast<uint64_t>(gridDim.x) * kRowThreads) {
        float g, h;
        row_gradient(r, row, g, h);
        r.grad[row] = g;
        r.hess[row] = h;
        mg = fmax(mg, static_cast<double>(fabsf(g)));
        mh = fmax(mh, static_cast<double>(fabsf(h)));
    }
    block_max_pair(mg, mh);
    if (threadIdx.x == 0) {
        // Non-negative doubles order like their bit patterns.
        atomicMax(max_g, static_cast<unsigned long long>(__double_as_longlong(mg)));
        atomicMax(max_h, static_cast<unsigned long long>(__double_as_longlong(mh)));
    }
}

__global__ void __launch_bounds__(kRowThreads) gradients_kernel(IterArgs a) {
    if (a.t.iter->stopped) return;
    gradients_body(a.r, &a.t.iter->max_abs_grad_bits, &a.t.iter->max_hess_bits);
}

__device__ __forceinline__ bool may_split_root(const TrainArgs& t, int64_t count) {
    const int64_t min_pair = 2 * t.cfg.min_data_in_leaf;
    return (t.max_depth <= 0 || 0 < t.max_depth) && count >= min_pair;
}

__global__ void __launch_bounds__(kRowThreads) iteration_start_kernel(IterArgs a) {
    __shared__ sb2_quant_spec s_spec;
    IterState* it = a.t.iter;
    const bool stopped = it->stopped;
    if (threadIdx.x == 0) {
        const double mg = __longlong_as_double(static_cast<long long>(it->max_abs_grad_bits));
        const double mh = __longlong_as_double(static_cast<long long>(it->max_hess_bits));
        s_spec = make_spec(mg, mh, a.k, static_cast<uint32_t>(it->iteration));
    }
    __syncthreads();
    const uint32_t staging_len = 2 * a.t.total_bins + 2;
    for (uint32_t i = blockIdx.x * kRowThreads + threadIdx.x; i < staging_len; i += gridDim.x * kRowThreads)
        a.t.staging[i] = 0;
    if (stopped) {
        // Training ended: every later kernel of the iteration finds nothing to do.
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            a.t.step->active = 0;
            a.t.hist_job->active = 0;
        }
        return;
    }
    const sb2_quant_spec spec = s_spec;
    long long sum_g = 0, sum_h = 0;
    for (uint64_t row = static_cast<uint64_t>(blockIdx.x) * kRowThreads + threadIdx.x; row < a.r.num_rows;
         row += static_cast<uint64_t>(gridDim.x) * kRowThreads) {
        const int32_t p = quantize_row(spec, a.r.grad[row], a.r.hess[row], a.r.row_offset + row);
        a.r.packed[row] = p;
        a.t.rows[0][row] = static_cast<uint32_t>(row);
        a.t.ordered[0][row] = p;
        const int32_t g = static_cast<int16_t>(static_cast<uint16_t>(static_cast<uint32_t>(p)));  // quantize.rs:140-143
        sum_g += g;
        sum_h += (p - g) >> 16;
    }
    // The root's units: this block's sums, then one 64-bit atomic per value (two's complement adds exactly).
    for (int o = 16; o > 0; o >>= 1) {
        sum_g += __shfl_xor_sync(0xffffffffu, sum_g, o);
        sum_h += __shfl_xor_sync(0xffffffffu, sum_h, o);
    }
    __shared__ long long s_sums[2][kRowThreads / 32];
    if ((threadIdx.x & 31) == 0) {
        s_sums[0][threadIdx.x >> 5] = sum_g;
        s_sums[1][threadIdx.x >> 5] = sum_h;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < kRowThreads / 32; ++k) {
            sum_g += s_sums[0][k];
            sum_h += s_sums[1][k];
        }
        atomicAdd(&it->root_units[0], static_cast<unsigned long long>(sum_g));
        atomicAdd(&it->root_units[1], static_cast<unsigned long long>(sum_h));
    }
    if (blockIdx.x != 0) return;
    const uint32_t F = a.t.num_features;
    const uint8_t* mask = a.t.masks + static_cast<size_t>(it->iteration) * F;
    for (uint32_t f = threadIdx.x; f < F; f += kRowThreads)
        a.t.evaluate[f] = static_cast<uint8_t>(mask[f] || static_cast<int32_t>(f) == a.t.sums_feature);
    for (int32_t i = threadIdx.x; i < 2 * a.t.max_leaves; i += kRowThreads) a.leaf_sums[i] = 0;
    if (threadIdx.x == 0) {
        it->spec = spec;
        it->root_count = a.k.total_rows;
        DevLeaf root{};
        root.begin = 0;
        root.count = static_cast<uint32_t>(a.r.num_rows);
        root.which = 0;
        root.depth = 0;
        root.count_global = a.k.total_rows;
        a.t.leaves[0] = root;
        const DevTree& t = a.t.tree;
        *t.num_leaves = 1;
        t.leaf_value[0] = 0.0;
        t.leaf_weight[0] = 0.0;
        t.leaf_count[0] = 0;
        t.leaf_parent[0] = -1;
        t.leaf_depth[0] = 0;
        Step s{};
        s.active = 1;
        s.root = 1;
        *a.t.step = s;
        HistJob job{};
        job.active = a.t.sums_feature >= 0 && may_split_root(a.t, a.k.total_rows);
        job.identity = 1;
        job.begin = 0;
        job.count = static_cast<uint32_t>(a.r.num_rows);
        job.which = 0;
        *a.t.hist_job = job;
    }
}

// The leaves of the current tree (those with rows on this rank) sorted by first position, for position -> leaf
// lookups: first position, leaf index, partition buffer.
constexpr int kIndexLeaves = 1024;
struct LeafIndex {
    uint32_t begin[kIndexLeaves];
    uint16_t leaf[kIndexLeaves];
    uint8_t which[kIndexLeaves];
    int n;
};

// Whole CTA of kRowThreads threads: every leaf's record is read once (kIndexLeaves / kRowThreads leaves a thread,
// all loads in flight together), then ranked by its first position against the others in shared memory (the
// first positions of non-empty leaves are distinct).
__device__ void build_leaf_index(const TrainArgs& t, LeafIndex& li) {
    constexpr int kPer = kIndexLeaves / kRowThreads;
    const int32_t L = min(*t.tree.num_leaves, kIndexLeaves);
    uint32_t b[kPer], w[kPer];
    bool live[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        const int32_t l = static_cast<int32_t>(threadIdx.x) + q * kRowThreads;
        live[q] = false;
        b[q] = 0xFFFFFFFFu;
        w[q] = 0;
        if (l < L) {
            const DevLeaf& lf = t.leaves[l];
            const uint32_t count = lf.count;
            live[q] = count != 0;
            b[q] = live[q] ? lf.begin : 0xFFFFFFFFu;
            w[q] = lf.which & 1u;
        }
    }
    if (threadIdx.x == 0) li.n = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        const int32_t l = static_cast<int32_t>(threadIdx.x) + q * kRowThreads;
        if (l < L) li.begin[l] = b[q];  // scratch: every leaf's first position (empty: never before another)
    }
    __syncthreads();
    int rank[kPer];
    int live_here = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        rank[q] = 0;
        if (!live[q]) continue;
        ++live_here;
        for (int32_t m = 0; m < L; ++m) rank[q] += li.begin[m] < b[q];
    }
    if (live_here) atomicAdd(&li.n, live_here);
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        if (!live[q]) continue;
        li.begin[rank[q]] = b[q];
        li.leaf[rank[q]] = static_cast<uint16_t>(threadIdx.x + q * kRowThreads);
        li.which[rank[q]] = static_cast<uint8_t>(w[q]);
    }
    __syncthreads();
}

constexpr int kRowUnroll = 4;  // positions a thread has in flight in the row passes over a tree's leaves

// The index entry of position p: a binary search, or, from the entry `k` of an earlier position, a walk forward.
__device__ __forceinline__ int leaf_after(const LeafIndex& li, int k, uint32_t p) {
    while (k + 1 < li.n && li.begin[k + 1] <= p) ++k;
    return k;
}

__device__ __forceinline__ int leaf_of(const LeafIndex& li, uint32_t p) {
    int lo = 0, hi = li.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (li.begin[mid] <= p)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

// Each row's leaf in the current tree (IterArgs::leaf_of_row), from the partition: the CTA's range of positions,
// kRowUnroll a thread at a time (their row ids in flight together), each thread walking the leaf index forward.
__global__ void __launch_bounds__(kRowThreads) leaf_map_kernel(IterArgs a) {
    __shared__ LeafIndex li;
    if (a.t.iter->stopped || a.t.iter->error != 0) return;  // an error ends training at this iteration's finalize
    build_leaf_index(a.t, li);
    const uint64_t n = a.r.num_rows;
    const uint64_t lo = n * blockIdx.x / gridDim.x, hi = n * (blockIdx.x + 1) / gridDim.x;
    int walk = lo < hi ? leaf_of(li, static_cast<uint32_t>(lo)) : 0;
    for (uint64_t p0 = lo + threadIdx.x; p0 < hi; p0 += kRowUnroll * kRowThreads) {
        int kq[kRowUnroll];
#pragma unroll
        for (int q = 0; q < kRowUnroll; ++q) {
            const uint64_t p = p0 + static_cast<uint64_t>(q) * kRowThreads;
            kq[q] = -1;
            if (p < hi) {
                walk = leaf_after(li, walk, static_cast<uint32_t>(p));
                kq[q] = walk;
            }
        }
        uint32_t rq[kRowUnroll];
#pragma unroll
        for (int q = 0; q < kRowUnroll; ++q)
            rq[q] = kq[q] >= 0 ? a.t.rows[li.which[kq[q]]][p0 + static_cast<uint64_t>(q) * kRowThreads] : 0u;
#pragma unroll
        for (int q = 0; q < kRowUnroll; ++q)
            if (kq[q] >= 0) a.leaf_of_row[rq[q]] = li.leaf[kq[q]];
    }
}

// Backend::leaf_sums for every leaf of the tree (backend/cpu.rs:886-905: the fixed-point sums of the leaf's rows'
// gradients and hessians): the rows in order, four a thread at a time, each row's pair added to its leaf's sums in
// shared memory as two 32-bit halves per value (integer sums, so the order is free), then the CTA's sums added to the
// output with 64-bit atomics. A CTA takes at most kLeafSumRows rows (launch_leaf_sums sizes the grid for it): 60,000
// low halves of at most 65,535 stay below 2^32, and 60,000 high halves of magnitude below 2^15 below 2^31.
constexpr uint64_t kLeafSumRows = 60000;  // rows a leaf_sums CTA takes at most: its 32-bit halves cannot overflow

__global__ void __launch_bounds__(kRowThreads) leaf_sums_kernel(IterArgs a) {
    // Each fixed-point value (|v| < 2^31) is added as two 32-bit halves, its low 16 bits (unsigned) and the rest
    // (signed): over at most 65536 rows neither sum overflows, and 32-bit shared atomics run several times faster
    // than 64-bit ones. A value outside that range (a gradient far beyond the scale's maximum) goes straight to the
    // output with a 64-bit atomic.
    __shared__ uint32_t g_lo[kIndexLeaves], h_lo[kIndexLeaves];
    __shared__ int32_t g_hi[kIndexLeaves], h_hi[kIndexLeaves];
    if (a.t.iter->stopped || a.t.iter->error != 0) return;
    const int32_t L = min(*a.t.tree.num_leaves, kIndexLeaves);
    for (int i = threadIdx.x; i < L; i += kRowThreads) g_lo[i] = h_lo[i] = 0, g_hi[i] = h_hi[i] = 0;
    __syncthreads();
    const double mg = __longlong_as_double(static_cast<long long>(a.t.iter->max_abs_grad_bits));
    const double mh = __longlong_as_double(static_cast<long long>(a.t.iter->max_hess_bits));
    const float gs = fixed_point_scale(mg), hs = fixed_point_scale(mh);
    const uint64_t n = a.r.num_rows;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kRowThreads;
    auto add1 = [&](uint32_t leaf, int64_t v, uint32_t* lo, int32_t* hi, long long* out) {
        if (static_cast<uint64_t>(v + (1ll << 31)) < (1ull << 32)) {
            atomicAdd(lo + leaf, static_cast<uint32_t>(v) & 0xFFFFu);
            atomicAdd(hi + leaf, static_cast<int32_t>(v >> 16));
        } else {
            atomicAdd(reinterpret_cast<unsigned long long*>(out), static_cast<unsigned long long>(v));
        }
    };
    auto add = [&](uint32_t leaf, float g, float h) {
        add1(leaf, to_fixed(g, gs), g_lo, g_hi, reinterpret_cast<long long*>(a.leaf_sums) + 2 * leaf);
        add1(leaf, to_fixed(h, hs), h_lo, h_hi, reinterpret_cast<long long*>(a.leaf_sums) + 2 * leaf + 1);
    };
    for (uint64_t r0 = (static_cast<uint64_t>(blockIdx.x) * kRowThreads + threadIdx.x) * 4; r0 < n; r0 += 4 * stride) {
        if (r0 + 4 <= n) {
            const ushort4 k = *reinterpret_cast<const ushort4*>(a.leaf_of_row + r0);
            const float4 g = *reinterpret_cast<const float4*>(a.r.grad + r0);
            const float4 h = *reinterpret_cast<const float4*>(a.r.hess + r0);
            add(k.x, g.x, h.x);
            add(k.y, g.y, h.y);
            add(k.z, g.z, h.z);
            add(k.w, g.w, h.w);
        } else {
            for (uint64_t row = r0; row < n; ++row) add(a.leaf_of_row[row], a.r.grad[row], a.r.hess[row]);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < L; i += kRowThreads) {
        const long long sg = static_cast<long long>(g_hi[i]) * 65536 + g_lo[i];
        const long long sh = static_cast<long long>(h_hi[i]) * 65536 + h_lo[i];
        if (sg != 0) atomicAdd(reinterpret_cast<unsigned long long*>(&a.leaf_sums[2 * i]), static_cast<unsigned long long>(sg));
        if (sh != 0) atomicAdd(reinterpret_cast<unsigned long long*>(&a.leaf_sums[2 * i + 1]), static_cast<unsigned long long>(sh));
    }
}

// split::leaf_output (split.rs:190-192)
__device__ __forceinline__ double leaf_output(double g, double h, double l1, double l2) {
    const double sg = static_cast<double>((g > 0.0) - (g < 0.0));
    const double t = __dmul_rn(sg, fmax(__dsub_rn(fabs(g), l1), 0.0));
    return __ddiv_rn(-t, __dadd_rn(h, l2));
}

__global__ void __launch_bounds__(kRowThreads) finalize_kernel(IterArgs a) {
    IterState* it = a.t.iter;
    if (it->stopped) return;
    if (it->error != 0) {
        // The tree kernel gave up (a rank or a CTA did not answer in time): training stops here, this tree
        // unrecorded; the host reports the error.
        if (threadIdx.x == 0) it->stopped = 1;
        return;
    }
    const DevTree& t = a.t.tree;
    const int32_t L = *t.num_leaves;
    const int32_t iteration = it->iteration;
    const int32_t rec = it->trees;
    const size_t base = static_cast<size_t>(rec) * a.t.max_leaves;
    const bool first = rec == 0;
    __syncthreads();
    if (L == 1) {
        // Trainer::single_leaf: the first tree becomes the constant init score; training stops either way.
        if (threadIdx.x == 0) {
            if (first) {
                a.records[0].num_leaves = 1;
                a.records[0].iteration = iteration;
                a.records[0].shrinkage = 1.0;
                a.record_tree.leaf_value[0] = a.k.init_score;
                a.record_tree.leaf_weight[0] = 0.0;
                a.record_tree.leaf_count[0] = 0;
                it->trees = 1;
            }
            it->stopped = 1;
        }
        return;
    }
    const double mg = __longlong_as_double(static_cast<long long>(it->max_abs_grad_bits));
    const double mh = __longlong_as_double(static_cast<long long>(it->max_hess_bits));
    const float gs = fixed_point_scale(mg), hs = fixed_point_scale(mh);
    const double lr = a.k.learning_rate;
    const double bias = a.k.init_score;
    const bool add_bias = first && bias != 0.0;
    for (int32_t l = threadIdx.x; l < L; l += kRowThreads) {
        double value = t.leaf_value[l];
        double weight = t.leaf_weight[l];
        if (a.k.renew) {
            const double sg = __ddiv_rn(static_cast<double>(a.leaf_sums[2 * l]), static_cast<double>(gs));
            const double sh = __ddiv_rn(static_cast<double>(a.leaf_sums[2 * l + 1]), static_cast<double>(hs));
            value = round_to_zero(leaf_output(sg, sh, a.t.cfg.lambda_l1, a.t.cfg.lambda_l2));
            weight = sh;
        }
        value = round_to_zero(__dmul_rn(value, lr));  // Tree::shrink
        float add = __double2float_rn(value);
        if (add_bias) {
            value = round_to_zero(__dadd_rn(value, bias));  // Tree::add_bias
            add = __double2float_rn(__dsub_rn(value, bias));  // replay::leaf_values
        }
        a.leaf_values_f32[l] = add;
        a.record_tree.leaf_value[base + l] = value;
        a.record_tree.leaf_weight[base + l] = weight;
        a.record_tree.leaf_count[base + l] = t.leaf_count[l];
    }
    for (int32_t k = threadIdx.x; k + 1 < L; k += kRowThreads) {
        double iv = round_to_zero(__dmul_rn(t.internal_value[k], lr));
        if (add_bias) iv = round_to_zero(__dadd_rn(iv, bias));
        a.record_tree.internal_value[base + k] = iv;
        a.record_tree.internal_weight[base + k] = t.internal_weight[k];
        a.record_tree.internal_count[base + k] = t.internal_count[k];
        a.record_tree.split_feature[base + k] = t.split_feature[k];
        a.record_tree.split_gain[base + k] = t.split_gain[k];
        a.record_tree.threshold_bin[base + k] = t.threshold_bin[k];
        a.record_tree.decision_type[base + k] = t.decision_type[k];
        a.record_tree.left_child[base + k] = t.left_child[k];
        a.record_tree.right_child[base + k] = t.right_child[k];
#pragma unroll
        for (int w = 0; w < 8; ++w) a.record_tree.cat_bins[8 * (base + k) + w] = t.cat_bins[8 * static_cast<size_t>(k) + w];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        a.records[rec].num_leaves = L;
        a.records[rec].iteration = iteration;
        a.records[rec].shrinkage = add_bias ? 1.0 : lr;
        it->trees = rec + 1;
        // The next iteration: its draws are keyed by the new index, its maxima start from zero.
        it->iteration = iteration + 1;
        it->max_abs_grad_bits = 0ull;
        it->max_hess_bits = 0ull;
        it->root_units[0] = it->root_units[1] = 0ull;
    }
}

__global__ void __launch_bounds__(kRowThreads) add_tree_partition_kernel(IterArgs a) {
    __shared__ float values[kIndexLeaves];
    IterState* it = a.t.iter;
    // finalize has recorded the tree; a stopped run adds nothing. The iteration advances here, after every kernel
    // of this iteration has read it.
    const bool stopped = it->stopped;
    if (!stopped) {
        // Every row's leaf, as leaf_sums left it: the rows in order, four a thread at a time.
        const int32_t L = min(*a.t.tree.num_leaves, kIndexLeaves);
        for (int32_t l = threadIdx.x; l < L; l += kRowThreads) values[l] = a.leaf_values_f32[l];
        __syncthreads();
        const uint64_t n = a.r.num_rows;
        const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kRowThreads;
        for (uint64_t r0 = (static_cast<uint64_t>(blockIdx.x) * kRowThreads + threadIdx.x) * 4; r0 < n; r0 += 4 * stride) {
            if (r0 + 4 <= n) {
                const ushort4 k = *reinterpret_cast<const ushort4*>(a.leaf_of_row + r0);
                float4 s = *reinterpret_cast<const float4*>(a.r.scores + r0);
                s.x = __fadd_rn(s.x, values[k.x]);
                s.y = __fadd_rn(s.y, values[k.y]);
                s.z = __fadd_rn(s.z, values[k.z]);
                s.w = __fadd_rn(s.w, values[k.w]);
                *reinterpret_cast<float4*>(a.r.scores + r0) = s;
            } else {
                for (uint64_t row = r0; row < n; ++row) a.r.scores[row] = __fadd_rn(a.r.scores[row], values[a.leaf_of_row[row]]);
            }
        }
    }
}

// ---- Backend API kernels ------------------------------------------------------------------------------------

__global__ void __launch_bounds__(kRowThreads) api_gradients_kernel(RowArgs r, unsigned long long* bits) {
    gradients_body(r, bits, bits + 1);
}

__global__ void __launch_bounds__(kRowThreads) api_quantize_kernel(RowArgs r, sb2_quant_spec spec) {
    for (uint64_t row = static_cast<uint64_t>(blockIdx.x) * kRowThreads + threadIdx.x; row < r.num_rows;
         row += static_cast<uint64_t>(gridDim.x) * kRowThreads)
        r.packed[row] = quantize_row(spec, r.grad[row], r.hess[row], r.row_offset + row);
}

__global__ void __launch_bounds__(kRowThreads) api_iota_kernel(uint32_t* rows, int32_t* ordered, const int32_t* packed,
                                                               uint64_t n) {
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * kRowThreads + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * kRowThreads) {
        rows[i] = static_cast<uint32_t>(i);
        ordered[i] = packed[i];
    }
}

__global__ void __launch_bounds__(kRowThreads) api_leaf_sums_kernel(RowArgs r, const uint32_t* partition,
                                                                    const sb2_leaf_range* ranges, uint32_t num,
                                                                    float gs, float hs, int64_t* out) {
    __shared__ long long sg[kRowThreads / 32], sh[kRowThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (uint32_t l = 0; l < num; ++l) {
        const sb2_leaf_range rg = ranges[l];
        long long g = 0, h = 0;
        for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * kRowThreads + threadIdx.x; i < rg.count;
             i += static_cast<uint64_t>(gridDim.x) * kRowThreads) {
            const uint32_t row = partition[rg.begin + i];
            g += to_fixed(r.grad[row], gs);
            h += to_fixed(r.hess[row], hs);
        }
        for (int o = 16; o > 0; o >>= 1) {
            g += __shfl_xor_sync(0xffffffffu, g, o);
            h += __shfl_xor_sync(0xffffffffu, h, o);
        }
        if (lane == 0) {
            sg[warp] = g;
            sh[warp] = h;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            long long tg = 0, th = 0;
            for (int k = 0; k < kRowThreads / 32; ++k) {
                tg += sg[k];
                th += sh[k];
            }
            if (tg != 0) atomicAdd(reinterpret_cast<unsigned long long*>(out + 2 * l), static_cast<unsigned long long>(tg));
            if (th != 0) atomicAdd(reinterpret_cast<unsigned long long*>(out + 2 * l + 1), static_cast<unsigned long long>(th));
        }
        __syncthreads();
    }
}

// add_tree_to (backend/cpu.rs:605-695): walk each row's bins down the tree.
__global__ void __launch_bounds__(kRowThreads) api_add_tree_kernel(DevData d, RowArgs r, const TileNode* nodes,
                                                                   uint32_t num_nodes, const float* leaf_values) {
    for (uint64_t row = static_cast<uint64_t>(blockIdx.x) * kRowThreads + threadIdx.x; row < r.num_rows;
         row += static_cast<uint64_t>(gridDim.x) * kRowThreads) {
        int32_t node = num_nodes == 0 ? -1 : 0;
        while (node >= 0) {
            const TileNode& nd = nodes[node];
            const Tile tile = d.tiles[nd.tile];
            const uint32_t bin = d.bins[tile.base + row * tile.pitch + nd.lane];
            node = ((nd.left_bins[bin >> 5] >> (bin & 31)) & 1u) ? nd.left : nd.right;
        }
        r.scores[row] = __fadd_rn(r.scores[row], leaf_values[~node]);
    }
}

// A group's columns (rows of `row_stride` bytes) into the feature-major copy: one CTA per 128 rows and 64-column
// strip. The strip's bytes go to shared memory at a pitch of 65 (coalesced byte loads), then warp w writes columns
// w, w + 8, ... of the strip, lane j rows 4j .. 4j + 3 as one 32-bit store (128 bytes per warp; with the odd pitch
// the reads hit 32 different banks). `col_feature[c]` is column c's feature (-1: none or trivial), `col_bins[c]` its
// bin count: a bin past it sets `bad` (the histogram's shared slots hold exactly each feature's bins).
__global__ void group_columns_kernel(const uint8_t* src, uint64_t rows, uint32_t row_stride, const int32_t* col_feature,
                                     const uint32_t* col_bins, uint8_t* columns, uint64_t column_stride,
                                     unsigned int* bad) {
    constexpr uint32_t kRows = 128, kStrip = 64, kPitch = kStrip + 1;
    __shared__ uint8_t sh[kRows * kPitch];
    const uint64_t r0 = static_cast<uint64_t>(blockIdx.x) * kRows;
    const uint32_t c0 = blockIdx.y * kStrip;
    for (uint32_t i = threadIdx.x; i < kRows * kStrip; i += blockDim.x) {
        const uint32_t row = i / kStrip, c = i % kStrip;
        sh[row * kPitch + c] = r0 + row < rows && c0 + c < row_stride ? src[(r0 + row) * row_stride + c0 + c] : 0;
    }
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    bool out_of_range = false;
    for (uint32_t c = warp; c < kStrip && c0 + c < row_stride; c += warps) {
        const int32_t f = col_feature[c0 + c];
        if (f < 0) continue;
        const uint32_t nb = col_bins[c0 + c];
        uint32_t v = 0;
        for (int q = 0; q < 4; ++q) {
            const uint8_t bin = sh[(4 * lane + q) * kPitch + c];
            out_of_range |= r0 + 4 * lane + q < rows && bin >= nb;
            v |= static_cast<uint32_t>(bin) << (8 * q);
        }
        *reinterpret_cast<uint32_t*>(columns + static_cast<uint64_t>(f) * column_stride + r0 + 4 * lane) = v;
    }
    if (__any_sync(0xffffffffu, out_of_range) && lane == 0) atomicOr(bad, 1u);
}

// The tiles from the feature-major copy: one CTA per 128 rows of one tile. Warp w reads the columns of tile lanes
// w, w + 8, ... (128 bytes each, coalesced) into shared memory at a pitch of 132, then the CTA writes the tile's 128
// rows as 32-bit words (padding lanes 0).
__global__ void tiles_kernel(DevData d, uint8_t* bins) {
    constexpr uint32_t kRows = 128, kPitch = kRows + 4;
    __shared__ __align__(4) uint8_t sh[kTileLanes * kPitch];
    const Tile tile = d.tiles[blockIdx.y];
    const uint64_t r0 = static_cast<uint64_t>(blockIdx.x) * kRows;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    for (uint32_t l = warp; l < tile.stride; l += warps) {
        const int32_t f = l < tile.nfeat ? d.lane_feature[blockIdx.y * kTileLanes + l] : -1;
        uint32_t v = f >= 0 ? *reinterpret_cast<const uint32_t*>(d.columns + static_cast<uint64_t>(f) * d.column_stride + r0 + 4 * lane) : 0u;
        const uint32_t mfb = f >= 0 ? d.features[f].mfb : 0u;
        if (mfb & kDominantSkip) {  // the feature's bins 0 and mfb trade places (swap_dominant)
            uint32_t x = 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) x |= swap_dominant((v >> (8 * q)) & 0xFFu, mfb & 0xFFu) << (8 * q);
            v = x;
        }
        *reinterpret_cast<uint32_t*>(sh + l * kPitch + 4 * lane) = v;
    }
    __syncthreads();
    const uint32_t words = tile.stride / 4;
    for (uint32_t i = threadIdx.x; i < kRows * words; i += blockDim.x) {
        const uint32_t row = i / words, wb = i % words;
        if (r0 + row >= d.num_rows) continue;
        uint32_t v = 0;
        for (int q = 0; q < 4; ++q) v |= static_cast<uint32_t>(sh[(4 * wb + q) * kPitch + row]) << (8 * q);
        *reinterpret_cast<uint32_t*>(bins + tile.base + (r0 + row) * tile.pitch + 4 * wb) = v;
    }
}

// How many rows of column feats[k] hold each bin, added into counts[k * 256 + bin]: one CTA per kCountRows rows of
// one column (blockIdx.y + y0), each thread 16 bytes at a time; the equal bins of a warp's step are added once
// (match.any) into the CTA's shared counts, which go to `counts` at the end. The column's stride (a multiple of
// 128 bytes) covers the 16 bytes read at any row below `rows`; bytes past `rows` are not counted.
constexpr uint32_t kCountThreads = 256, kCountLoads = 8;
constexpr uint64_t kCountRows = 16ull * kCountThreads * kCountLoads;
__global__ void __launch_bounds__(kCountThreads) bin_counts_kernel(const uint8_t* columns, uint64_t column_stride,
                                                                   uint64_t rows, const int32_t* feats, uint32_t y0,
                                                                   unsigned int* counts) {
    __shared__ unsigned int sh[256];
    sh[threadIdx.x] = 0;
    __syncthreads();
    const uint32_t k = y0 + blockIdx.y, lane = threadIdx.x & 31;
    const uint8_t* col = columns + static_cast<uint64_t>(feats[k]) * column_stride;
    const uint64_t r0 = static_cast<uint64_t>(blockIdx.x) * kCountRows;
    for (uint32_t i = 0; i < kCountLoads; ++i) {
        const uint64_t r = r0 + 16ull * (i * kCountThreads + threadIdx.x);
        const bool in = r < rows;
        const uint4 v = in ? __ldcs(reinterpret_cast<const uint4*>(col + r)) : make_uint4(0, 0, 0, 0);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int b = 0; b < 16; ++b) {
            const bool valid = in && r + b < rows;
            const uint32_t bin = valid ? (w[b >> 2] >> (8 * (b & 3))) & 0xFFu : 256u;
            const uint32_t peers = __match_any_sync(0xffffffffu, bin);
            if (valid && lane == static_cast<uint32_t>(__ffs(peers) - 1)) atomicAdd(&sh[bin], __popc(peers));
        }
    }
    __syncthreads();
    if (sh[threadIdx.x] != 0) atomicAdd(&counts[static_cast<uint64_t>(k) * 256 + threadIdx.x], sh[threadIdx.x]);
}

__global__ void fill_kernel(float* out, uint64_t n, float value) {
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        out[i] = value;
}

// A double from hashed bits: sign, an exponent in [-span, span] around 0 (biased), and a mantissa that is random or
// one of the awkward patterns (all zeros, all ones, a single bit).
__device__ double division_operand(uint32_t h0, uint32_t h1, uint32_t h2, int span) {
    uint64_t mant = (static_cast<uint64_t>(h1) << 32 | h2) & ((1ull << 52) - 1);
    switch (h0 & 15) {
        case 0: mant = 0; break;
        case 1: mant = (1ull << 52) - 1; break;
        case 2: mant = 1ull << (h1 % 52); break;
        default: break;
    }
    const int exp = static_cast<int>((h0 >> 8) % static_cast<uint32_t>(2 * span + 1)) - span;
    const uint64_t bits = (static_cast<uint64_t>(h0 >> 4 & 1) << 63) | (static_cast<uint64_t>(exp + 1023) << 52) | mant;
    return __longlong_as_double(static_cast<long long>(bits));
}

// div_rn against the library's correctly rounded division on `n` hashed operand pairs: most in the range the
// split scan divides in, some wide of it (they take the library path), exact quotients and zero numerators.
__global__ void division_check_kernel(uint64_t n, uint32_t seed, unsigned long long* mismatches) {
    unsigned long long bad = 0;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t k = mix32(seed ^ mix32(static_cast<uint32_t>(i) ^ mix32(static_cast<uint32_t>(i >> 32))));
        const uint32_t h[6] = {mix32(k ^ 1u), mix32(k ^ 2u), mix32(k ^ 3u), mix32(k ^ 4u), mix32(k ^ 5u), mix32(k ^ 6u)};
        const int span_a = (k & 7) == 0 ? 700 : 80, span_b = (k & 7) == 1 ? 200 : 60;
        double b = division_operand(h[0], h[1], h[2], span_b);
        double a = division_operand(h[3], h[4], h[5], span_a);
        if ((k >> 3 & 31) == 0) a = __dmul_rn(b, static_cast<double>(h[4] & 0xFFFFF));  // exact quotients
        if ((k >> 3 & 31) == 1) a = 0.0;
        const double q = div_rn(a, b), want = __ddiv_rn(a, b);
        const bool same = __double_as_longlong(q) == __double_as_longlong(want) || (q != q && want != want);
        bad += same ? 0 : 1;
    }
    if (bad) atomicAdd(mismatches, bad);
}

}  // namespace

void launch_gradients(const IterArgs& a, int grid, cudaStream_t s) {
    if (a.r.objective == SB2_LAMBDARANK)
        launch_lambdarank(a.r, &a.t.iter->stopped, &a.t.iter->max_abs_grad_bits, &a.t.iter->max_hess_bits, s);
    else
        gradients_kernel<<<grid, kRowThreads, 0, s>>>(a);
}
void launch_iteration_start(const IterArgs& a, int grid, cudaStream_t s) {
    iteration_start_kernel<<<grid, kRowThreads, 0, s>>>(a);
}
void launch_leaf_sums(const IterArgs& a, int grid, cudaStream_t s) {
    leaf_map_kernel<<<grid, kRowThreads, 0, s>>>(a);
    // fewer CTAs than the row passes (fewer output atomics), but enough that none takes more than kLeafSumRows rows
    const uint64_t need = (a.r.num_rows + kLeafSumRows - 1025) / (kLeafSumRows - 1024);
    leaf_sums_kernel<<<static_cast<unsigned>(std::max<uint64_t>(std::max(grid / 4, 1), need)), kRowThreads, 0, s>>>(a);
}
void launch_finalize(const IterArgs& a, cudaStream_t s) { finalize_kernel<<<1, kRowThreads, 0, s>>>(a); }
void launch_add_tree_partition(const IterArgs& a, int grid, cudaStream_t s) {
    add_tree_partition_kernel<<<grid, kRowThreads, 0, s>>>(a);
}
void launch_api_gradients(const RowArgs& r, unsigned long long* bits, int grid, cudaStream_t s) {
    if (r.objective == SB2_LAMBDARANK)
        launch_lambdarank(r, nullptr, bits, bits + 1, s);
    else
        api_gradients_kernel<<<grid, kRowThreads, 0, s>>>(r, bits);
}
void launch_api_quantize(const RowArgs& r, const sb2_quant_spec& spec, int grid, cudaStream_t s) {
    api_quantize_kernel<<<grid, kRowThreads, 0, s>>>(r, spec);
}
void launch_api_iota(uint32_t* rows, int32_t* ordered, const int32_t* packed, uint64_t n, int grid, cudaStream_t s) {
    api_iota_kernel<<<grid, kRowThreads, 0, s>>>(rows, ordered, packed, n);
}
void launch_api_leaf_sums(const RowArgs& r, const uint32_t* partition, const sb2_leaf_range* ranges, uint32_t num,
                          float gs, float hs, int64_t* out, int grid, cudaStream_t s) {
    api_leaf_sums_kernel<<<grid, kRowThreads, 0, s>>>(r, partition, ranges, num, gs, hs, out);
}
void launch_api_add_tree(const DevData& d, const RowArgs& r, const TileNode* nodes, uint32_t num_nodes,
                         const float* leaf_values, int grid, cudaStream_t s) {
    api_add_tree_kernel<<<grid, kRowThreads, 0, s>>>(d, r, nodes, num_nodes, leaf_values);
}
void launch_group_columns(const uint8_t* src, uint64_t rows, uint32_t row_stride, const int32_t* col_feature,
                          const uint32_t* col_bins, uint8_t* columns, uint64_t column_stride, unsigned int* bad,
                          cudaStream_t s) {
    if (rows == 0 || row_stride == 0) return;
    const dim3 grid(static_cast<unsigned>(ceil_div(rows, 128)), static_cast<unsigned>(ceil_div(row_stride, 64)));
    group_columns_kernel<<<grid, 256, 0, s>>>(src, rows, row_stride, col_feature, col_bins, columns, column_stride, bad);
}

void launch_tiles(const DevData& d, uint8_t* bins, cudaStream_t s) {
    if (d.num_tiles == 0 || d.num_rows == 0) return;
    const dim3 grid(static_cast<unsigned>(ceil_div(d.num_rows, 128)), d.num_tiles);
    tiles_kernel<<<grid, 256, 0, s>>>(d, bins);
}

void launch_bin_counts(const uint8_t* columns, uint64_t column_stride, uint64_t rows, const int32_t* feats,
                       uint32_t num_feats, unsigned int* counts, cudaStream_t s) {
    if (rows == 0) return;
    const unsigned gx = static_cast<unsigned>(ceil_div(rows, kCountRows));
    for (uint32_t y0 = 0; y0 < num_feats; y0 += 65535) {
        const dim3 grid(gx, std::min<uint32_t>(num_feats - y0, 65535));
        bin_counts_kernel<<<grid, kCountThreads, 0, s>>>(columns, column_stride, rows, feats, y0, counts);
    }
}

void launch_fill(float* out, uint64_t n, float value, cudaStream_t s) {
    const int grid = static_cast<int>(n / 256 + 1 < 65535 ? n / 256 + 1 : 65535);
    fill_kernel<<<grid, 256, 0, s>>>(out, n, value);
}

void launch_division_check(uint64_t n, uint32_t seed, unsigned long long* mismatches, int grid, cudaStream_t s) {
    division_check_kernel<<<grid, 256, 0, s>>>(n, seed, mismatches);
}

}  // namespace sb2
