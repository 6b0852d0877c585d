// lambdarank.cu — LambdaRank gradients on the device: objective/lambdarank.rs:197-396 (LightGBM 3.3.5's
// GetGradientsForOneQuery), f64 in the reference's operation order, so every row's gradient and hessian equal the
// CPU path's bit for bit where the math library calls agree (the tables are the host's; the device computes only
// the one log2 of the normalization).
//
// A query's rows are ranked by a bitonic sort of 64-bit keys in shared memory (score descending in the high half,
// row in the low half: ties keep row order, as the reference's stable sort). The reference's pair loop visits rows
// i < truncation_level in rank order and, for each, every lower-ranked row j, adding each pair's lambda and hessian
// to i's running sums and to j's; so a row's sums are the pairs (i, row) for i = 0, 1, ... in order, then its own
// pairs (row, j) for j in order, and the loop's sum of lambdas runs over the pairs in loop order. The kernels keep
// those orders in phases, one per row i: the group's lanes evaluate every pair (i, j) at once (each pair once) and
// add it to row j's sums, writing the pair's three terms (i's lambda term, hessian term and the sum's term, or +0
// for a pair of equal labels) at j; then three lanes add the phase's terms in j order to row i's lambda, row i's
// hessian and the sum of lambdas. Adding +0 leaves a sum that started at +0 unchanged in round-to-nearest (such a
// sum is never -0), so the skipped pairs cost no branch in those chains.
//
// Two shapes: a warp per query for queries of at most kWarpQueryRows rows (every row's lambda and hessian in its
// lane's registers; 16 queries per 512-thread CTA in flight), and a CTA per query up to kMaxQueryRows rows.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "iter.cuh"

namespace sb2 {

namespace {

constexpr int kRankThreads = 512;                      // both kernels' CTAs
constexpr uint32_t kWarpQueryRows = 256;               // the warp kernel's longest query
constexpr uint32_t kWarpItems = kWarpQueryRows / 32;   // rows a lane owns
constexpr uint32_t kSharedGains = 64;                  // label gains kept in shared memory (more: read from global)

// lambdarank.rs:34: LightGBM's 0.01f added to |delta_score| when normalizing by score distance.
constexpr double kScoreDistanceEpsilon = static_cast<double>(0.01f);

// descending_key (lambdarank.rs:162-168): ascending order of the key is descending order of the score; adding 0
// folds -0 into 0, which LightGBM's comparison treats as equal.
__device__ __forceinline__ uint32_t descending_key(float score) {
    const uint32_t bits = __float_as_uint(__fadd_rn(score, 0.0f));
    const uint32_t ascending = (bits >> 31) != 0 ? ~bits : (bits | 0x80000000u);
    return ~ascending;
}

// SigmoidTable::get (lambdarank.rs:110-119): the entry at the truncated index, the ends outside the table's range.
__device__ __forceinline__ double sigmoid_at(const RankArgs& k, double delta) {
    if (delta <= k.min_input) return __ldg(k.table);
    if (delta >= k.max_input) return __ldg(k.table + kSigmoidBins - 1);
    const unsigned long long i = __double2ull_rz(__dmul_rn(__dsub_rn(delta, k.min_input), k.idx_factor));
    return __ldg(k.table + (i < kSigmoidBins - 1 ? i : kSigmoidBins - 1));
}

// What every pair of a query shares (QueryContext, lambdarank.rs:243-250).
struct PairCtx {
    double score_i, gain_i, discount_i, inverse_max_dcg;
    float label_i;
    bool by_distance;
};

// One pair (i, j) of accumulate_pairs (lambdarank.rs:369-388): j's lambda and hessian terms (added to row j's sums)
// and i's three terms (i's lambda, i's hessian, the sum of lambdas), +0 for a pair of equal labels.
struct PairTerms {
    double lambda_j, hessian_j;  // row j: lambda -= sign * p_lambda, hessian += p_hessian
    double lambda_i, hessian_i, sum;
    bool counted;
};

__device__ __forceinline__ PairTerms pair_terms(const RankArgs& k, const PairCtx& c, double score_j, double gain_j,
                                                uint32_t j, float label_j) {
    PairTerms t{0.0, 0.0, 0.0, 0.0, 0.0, false};
    if (label_j == c.label_i) return t;
    const double sign = c.label_i > label_j ? 1.0 : -1.0;
    const double delta_score = __dmul_rn(sign, __dsub_rn(c.score_i, score_j));
    const double dcg_gap = __dmul_rn(sign, __dsub_rn(c.gain_i, gain_j));
    const double paired_discount = fabs(__dsub_rn(c.discount_i, __ldg(k.discount + j)));
    double delta_pair_ndcg = __dmul_rn(__dmul_rn(dcg_gap, paired_discount), c.inverse_max_dcg);
    if (c.by_distance)
        delta_pair_ndcg = __ddiv_rn(delta_pair_ndcg, __dadd_rn(kScoreDistanceEpsilon, fabs(delta_score)));
    const double p = sigmoid_at(k, delta_score);
    const double p_lambda = __dmul_rn(p, __dmul_rn(-k.sigmoid, delta_pair_ndcg));
    const double p_hessian = __dmul_rn(__dmul_rn(p, __dsub_rn(1.0, p)), __dmul_rn(k.sigmoid_squared, delta_pair_ndcg));
    const double signed_lambda = __dmul_rn(sign, p_lambda);
    t.lambda_j = signed_lambda;
    t.hessian_j = p_hessian;
    t.lambda_i = signed_lambda;
    t.hessian_i = p_hessian;
    t.sum = -__dmul_rn(2.0, p_lambda);  // sum -= 2 p_lambda, as sum + (-(2 p_lambda)): the same IEEE operation
    t.counted = true;
    return t;
}

// Lane `lane` (0: lambda, 1: hessian, 2: the sum) adds the terms at [from, to) of its array in order to `v`.
__device__ __forceinline__ double chain(const double* terms, uint32_t from, uint32_t to, double v) {
    uint32_t j = from;
    for (; j + 4 <= to; j += 4) {
        const double a = terms[j], b = terms[j + 1], c = terms[j + 2], d = terms[j + 3];
        v = __dadd_rn(v, a);
        v = __dadd_rn(v, b);
        v = __dadd_rn(v, c);
        v = __dadd_rn(v, d);
    }
    for (; j < to; ++j) v = __dadd_rn(v, terms[j]);
    return v;
}

__device__ __forceinline__ double gain_of(const RankArgs& k, const double* s_gain, float label) {
    const uint32_t l = static_cast<uint32_t>(label);
    return l < kSharedGains ? s_gain[l] : __ldg(k.label_gain + l);
}

// Bitonic sort of `cap` keys (a power of two) ascending by `threads` threads (index `t`), with `sync` between
// stages.
template <class Sync>
__device__ __forceinline__ void bitonic_sort(unsigned long long* key, uint32_t cap, uint32_t t, uint32_t threads,
                                             Sync sync) {
    for (uint32_t size = 2; size <= cap; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t x = t; x < cap / 2; x += threads) {
                const uint32_t lo = 2 * x - (x & (stride - 1)), hi = lo + stride;
                const unsigned long long a = key[lo], b = key[hi];
                if ((a > b) == ((lo & size) == 0)) {
                    key[lo] = b;
                    key[hi] = a;
                }
            }
            sync();
        }
    }
}

__device__ __forceinline__ void block_max(double& mg, double& mh, unsigned long long* max_g, unsigned long long* max_h) {
    __shared__ double s_mg[kRankThreads / 32], s_mh[kRankThreads / 32];
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o > 0; o >>= 1) {
        mg = fmax(mg, __shfl_xor_sync(0xffffffffu, mg, o));
        mh = fmax(mh, __shfl_xor_sync(0xffffffffu, mh, o));
    }
    if (lane == 0) {
        s_mg[warp] = mg;
        s_mh[warp] = mh;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kRankThreads / 32; ++w) {
            mg = fmax(mg, s_mg[w]);
            mh = fmax(mh, s_mh[w]);
        }
        // Non-negative doubles order like their bit patterns.
        atomicMax(max_g, static_cast<unsigned long long>(__double_as_longlong(mg)));
        atomicMax(max_h, static_cast<unsigned long long>(__double_as_longlong(mh)));
    }
}

// query_gradients (lambdarank.rs:300-320) of one row: the normalization, the f32 cast, the row weight.
__device__ __forceinline__ void store_row(const RowArgs& r, uint64_t at, double lambda, double hessian, double norm,
                                          double& mg, double& mh) {
    float g = __double2float_rn(__dmul_rn(lambda, norm));
    float h = __double2float_rn(__dmul_rn(hessian, norm));
    if (r.weight != nullptr) {
        g = __fmul_rn(g, r.weight[at]);
        h = __fmul_rn(h, r.weight[at]);
    }
    r.grad[at] = g;
    r.hess[at] = h;
    mg = fmax(mg, static_cast<double>(fabsf(g)));
    mh = fmax(mh, static_cast<double>(fabsf(h)));
}

// ---- a warp per query ------------------------------------------------------------------------------------------

// Per warp: the keys (cap u64), then per rank slot the three term arrays (f64), the score and the label (f32; the
// f64 score is the f32 one converted, exactly).
constexpr size_t kWarpSlotBytes = 8 + 3 * 8 + 4 + 4;

__global__ void __launch_bounds__(kRankThreads) lambdarank_warp_kernel(RowArgs r, const uint32_t* queries,
                                                                        uint32_t num_queries, const int32_t* stopped,
                                                                        unsigned long long* max_g,
                                                                        unsigned long long* max_h) {
    if (stopped != nullptr && *stopped) return;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ double s_gain[kSharedGains];
    const RankArgs& k = r.rank;
    for (uint32_t i = threadIdx.x; i < kSharedGains; i += kRankThreads)
        s_gain[i] = i < k.num_gain ? k.label_gain[i] : 0.0;
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = kRankThreads / 32;
    unsigned char* mine = smem + static_cast<size_t>(warp) * kWarpQueryRows * kWarpSlotBytes;
    unsigned long long* key = reinterpret_cast<unsigned long long*>(mine);
    double* t_lambda = reinterpret_cast<double*>(key + kWarpQueryRows);
    double* t_hessian = t_lambda + kWarpQueryRows;
    double* t_sum = t_hessian + kWarpQueryRows;
    float* score = reinterpret_cast<float*>(t_sum + kWarpQueryRows);
    float* label = score + kWarpQueryRows;
    const auto sync = [] { __syncwarp(); };
    double mg = 0.0, mh = 0.0;
    for (uint32_t qi = blockIdx.x * warps + warp; qi < num_queries; qi += gridDim.x * warps) {
        const uint32_t q = queries[qi];
        const uint32_t b = k.bounds[q], n = k.bounds[q + 1] - b;
        if (n == 0) continue;
        uint32_t cap = 2;
        while (cap < n) cap <<= 1;
        for (uint32_t i = lane; i < cap; i += 32)
            key[i] = i < n ? (static_cast<unsigned long long>(descending_key(r.scores[b + i])) << 32) | i : ~0ull;
        __syncwarp();
        bitonic_sort(key, cap, lane, 32u, sync);
        // load_ranked (lambdarank.rs:324-341): lane owns ranks lane + 32 m (their rows, lambdas and hessians in
        // registers); `valid`: the first rank holding a -inf score (they sort last).
        uint32_t row[kWarpItems];
        double lam[kWarpItems], hes[kWarpItems];
        uint32_t valid = n;
#pragma unroll
        for (uint32_t m = 0; m < kWarpItems; ++m) {
            const uint32_t i = lane + 32 * m;
            row[m] = 0;
            lam[m] = 0.0;
            hes[m] = 0.0;
            if (i < n) {
                row[m] = static_cast<uint32_t>(key[i]);
                const float s = r.scores[b + row[m]];
                score[i] = s;
                label[i] = r.label[b + row[m]];
                if (s == -CUDART_INF_F) valid = min(valid, i);
            }
        }
        for (int o = 16; o > 0; o >>= 1) valid = min(valid, __shfl_xor_sync(0xffffffffu, valid, o));
        __syncwarp();
        uint32_t worst = n - 1;  // worst_score (lambdarank.rs:344-351): one trailing -inf skipped
        if (worst > 0 && score[worst] == -CUDART_INF_F) --worst;
        PairCtx c{};
        c.by_distance = k.norm != 0 && score[0] != score[worst];
        c.inverse_max_dcg = k.inverse_max_dcg[q];
        const uint32_t rows_i = min(k.truncation, valid > 0 ? valid - 1 : 0u);
        double total = 0.0;  // lane 2: the sum of lambdas over the pairs so far
        for (uint32_t i = 0; i < rows_i; ++i) {
            c.score_i = static_cast<double>(score[i]);
            c.label_i = label[i];
            c.gain_i = gain_of(k, s_gain, c.label_i);
            c.discount_i = __ldg(k.discount + i);
#pragma unroll
            for (uint32_t m = 0; m < kWarpItems; ++m) {
                const uint32_t j = lane + 32 * m;
                if (j > i && j < valid) {
                    const float lj = label[j];
                    const PairTerms t = pair_terms(k, c, static_cast<double>(score[j]), gain_of(k, s_gain, lj), j, lj);
                    if (t.counted) {
                        lam[m] = __dsub_rn(lam[m], t.lambda_j);
                        hes[m] = __dadd_rn(hes[m], t.hessian_j);
                    }
                    t_lambda[j] = t.lambda_i;
                    t_hessian[j] = t.hessian_i;
                    t_sum[j] = t.sum;
                }
            }
            __syncwarp();
            // Row i's sums so far, from its owner lane, then its own pairs in j order.
            const uint32_t owner = i & 31, slot = i >> 5;
            double li = 0.0, hi = 0.0;
#pragma unroll
            for (uint32_t m = 0; m < kWarpItems; ++m)
                if (m == slot) li = lam[m], hi = hes[m];
            li = __shfl_sync(0xffffffffu, li, owner);
            hi = __shfl_sync(0xffffffffu, hi, owner);
            double v = lane == 0 ? li : lane == 1 ? hi : total;
            if (lane < 3) v = chain(lane == 0 ? t_lambda : lane == 1 ? t_hessian : t_sum, i + 1, valid, v);
            const double new_li = __shfl_sync(0xffffffffu, v, 0), new_hi = __shfl_sync(0xffffffffu, v, 1);
            if (lane == 2) total = v;
            if (lane == owner) {
#pragma unroll
                for (uint32_t m = 0; m < kWarpItems; ++m)
                    if (m == slot) lam[m] = new_li, hes[m] = new_hi;
            }
            __syncwarp();  // the term arrays are read before the next phase writes them
        }
        double norm = 1.0;
        if (lane == 2 && k.norm != 0 && total > 0.0) norm = __ddiv_rn(log2(__dadd_rn(1.0, total)), total);
        norm = __shfl_sync(0xffffffffu, norm, 2);
#pragma unroll
        for (uint32_t m = 0; m < kWarpItems; ++m)
            if (lane + 32 * m < n) store_row(r, b + row[m], lam[m], hes[m], norm, mg, mh);
        __syncwarp();  // the slots are free for the warp's next query
    }
    block_max(mg, mh, max_g, max_h);
}

// ---- a CTA per query -------------------------------------------------------------------------------------------

// Per rank slot: the key (u64; after the gather, the row in its low half), lambda, hessian and the three term arrays
// (f64), the score and the label (f32): 56 bytes, so a 4096-row query fits a CTA's shared memory.
constexpr size_t kCtaSlotBytes = 8 + 5 * 8 + 4 + 4;

__global__ void __launch_bounds__(kRankThreads) lambdarank_cta_kernel(RowArgs r, const uint32_t* queries,
                                                                       uint32_t num_queries, const int32_t* stopped,
                                                                       unsigned long long* max_g,
                                                                       unsigned long long* max_h) {
    if (stopped != nullptr && *stopped) return;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ double s_gain[kSharedGains];
    __shared__ uint32_t s_valid;
    __shared__ double s_norm;
    const RankArgs& k = r.rank;
    const uint32_t cap_max = k.cap;
    unsigned long long* key = reinterpret_cast<unsigned long long*>(smem);
    double* lam = reinterpret_cast<double*>(key + cap_max);
    double* hes = lam + cap_max;
    double* t_lambda = hes + cap_max;
    double* t_hessian = t_lambda + cap_max;
    double* t_sum = t_hessian + cap_max;
    float* score = reinterpret_cast<float*>(t_sum + cap_max);
    float* label = score + cap_max;
    for (uint32_t i = threadIdx.x; i < kSharedGains; i += kRankThreads)
        s_gain[i] = i < k.num_gain ? k.label_gain[i] : 0.0;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const auto sync = [] { __syncthreads(); };
    double mg = 0.0, mh = 0.0;
    for (uint32_t qi = blockIdx.x; qi < num_queries; qi += gridDim.x) {
        const uint32_t q = queries[qi];
        const uint32_t b = k.bounds[q], n = k.bounds[q + 1] - b;
        if (n == 0) continue;
        uint32_t cap = 2;
        while (cap < n) cap <<= 1;
        for (uint32_t i = tid; i < cap; i += kRankThreads)
            key[i] = i < n ? (static_cast<unsigned long long>(descending_key(r.scores[b + i])) << 32) | i : ~0ull;
        if (tid == 0) s_valid = n;
        __syncthreads();
        bitonic_sort(key, cap, tid, static_cast<uint32_t>(kRankThreads), sync);
        for (uint32_t i = tid; i < n; i += kRankThreads) {
            const uint32_t row = static_cast<uint32_t>(key[i]);
            const float s = r.scores[b + row];
            score[i] = s;
            label[i] = r.label[b + row];
            lam[i] = 0.0;
            hes[i] = 0.0;
            if (s == -CUDART_INF_F) atomicMin(&s_valid, i);
        }
        __syncthreads();
        const uint32_t valid = s_valid;
        uint32_t worst = n - 1;
        if (worst > 0 && score[worst] == -CUDART_INF_F) --worst;
        PairCtx c{};
        c.by_distance = k.norm != 0 && score[0] != score[worst];
        c.inverse_max_dcg = k.inverse_max_dcg[q];
        const uint32_t rows_i = min(k.truncation, valid > 0 ? valid - 1 : 0u);
        double total = 0.0;  // thread 2: the sum of lambdas over the pairs so far
        for (uint32_t i = 0; i < rows_i; ++i) {
            c.score_i = static_cast<double>(score[i]);
            c.label_i = label[i];
            c.gain_i = gain_of(k, s_gain, c.label_i);
            c.discount_i = __ldg(k.discount + i);
            for (uint32_t j = i + 1 + tid; j < valid; j += kRankThreads) {
                const float lj = label[j];
                const PairTerms t = pair_terms(k, c, static_cast<double>(score[j]), gain_of(k, s_gain, lj), j, lj);
                if (t.counted) {
                    lam[j] = __dsub_rn(lam[j], t.lambda_j);
                    hes[j] = __dadd_rn(hes[j], t.hessian_j);
                }
                t_lambda[j] = t.lambda_i;
                t_hessian[j] = t.hessian_i;
                t_sum[j] = t.sum;
            }
            __syncthreads();
            if (warp == 0 && lane < 3) {
                double v = lane == 0 ? lam[i] : lane == 1 ? hes[i] : total;
                v = chain(lane == 0 ? t_lambda : lane == 1 ? t_hessian : t_sum, i + 1, valid, v);
                if (lane == 0) lam[i] = v;
                if (lane == 1) hes[i] = v;
                if (lane == 2) total = v;
            }
            __syncthreads();
        }
        if (tid == 2) s_norm = k.norm != 0 && total > 0.0 ? __ddiv_rn(log2(__dadd_rn(1.0, total)), total) : 1.0;
        __syncthreads();
        const double norm = s_norm;
        for (uint32_t i = tid; i < n; i += kRankThreads)
            store_row(r, b + static_cast<uint32_t>(key[i]), lam[i], hes[i], norm, mg, mh);
        __syncthreads();  // the slots are free for the CTA's next query
    }
    block_max(mg, mh, max_g, max_h);
}

size_t warp_kernel_smem() { return static_cast<size_t>(kRankThreads / 32) * kWarpQueryRows * kWarpSlotBytes; }

}  // namespace

size_t lambdarank_smem(uint32_t cap) { return static_cast<size_t>(cap) * kCtaSlotBytes; }

uint32_t lambdarank_warp_rows() { return kWarpQueryRows; }

cudaError_t lambdarank_configure(uint32_t cap, int* warp_blocks_per_sm, int* cta_blocks_per_sm) {
    cudaError_t e = cudaFuncSetAttribute(lambdarank_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(warp_kernel_smem()));
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(warp_blocks_per_sm, lambdarank_warp_kernel, kRankThreads,
                                                          warp_kernel_smem());
    if (e != cudaSuccess) return e;
    *cta_blocks_per_sm = 0;
    if (cap <= kWarpQueryRows) return cudaSuccess;  // no query for the CTA kernel
    const int bytes = static_cast<int>(lambdarank_smem(cap));
    e = cudaFuncSetAttribute(lambdarank_cta_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(cta_blocks_per_sm, lambdarank_cta_kernel, kRankThreads, bytes);
}

void launch_lambdarank(const RowArgs& r, const int32_t* stopped, unsigned long long* max_g, unsigned long long* max_h,
                       cudaStream_t s) {
    const RankArgs& k = r.rank;
    if (k.num_short > 0)
        lambdarank_warp_kernel<<<k.warp_grid, kRankThreads, warp_kernel_smem(), s>>>(r, k.queries, k.num_short,
                                                                                    stopped, max_g, max_h);
    if (k.num_queries > k.num_short)
        lambdarank_cta_kernel<<<k.cta_grid, kRankThreads, lambdarank_smem(k.cap), s>>>(
            r, k.queries + k.num_short, k.num_queries - k.num_short, stopped, max_g, max_h);
}

}  // namespace sb2
