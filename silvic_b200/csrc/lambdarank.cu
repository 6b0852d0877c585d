// lambdarank.cu — LambdaRank gradients on the device: objective/lambdarank.rs:197-396 (LightGBM 3.3.5's
// GetGradientsForOneQuery), f64 in the reference's operation order, so every row's gradient and hessian equal the
// CPU path's bit for bit where the math library calls agree (the tables are the host's; the device computes only
// the one log2 of the normalization).
//
// One CTA takes a query at a time (queries grid-strided over the CTAs). Its rows are ranked by a bitonic sort of
// 64-bit keys in shared memory (score descending in the high half, row in the low half: ties keep row order, as
// the reference's stable sort). The reference's pair loop visits rows i < truncation_level in rank order and, for
// each, every lower-ranked row j, adding each pair's lambda and hessian to i's running sums and to j's; a row's
// sums are therefore the pairs (i, row) for i = 0, 1, ... in order, then its own pairs (row, j) for j in order, and
// the loop's sum of lambdas runs over the pairs in loop order. The kernel keeps those orders in phases, one per row
// i: the CTA's threads evaluate every pair (i, j) at once (each pair once) and add it to row j's sums, then three
// lanes of warp 0 add the phase's pairs in j order to row i's lambda, row i's hessian and the sum of lambdas.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "iter.cuh"

namespace sb2 {

namespace {

constexpr int kRankThreads = 256;

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

// A query's rows in shared memory, `cap` slots each.
struct QuerySlots {
    unsigned long long* key;  // sort keys; after the sort, the rank-ordered rows in the low halves
    double* score;            // rank order
    double* gain;
    double* lambda;
    double* hessian;
    double* pair_lambda;      // the current phase's pairs (i, j), at j
    double* pair_hessian;
    float* label;
};

__device__ __forceinline__ QuerySlots query_slots(unsigned char* smem, uint32_t cap) {
    QuerySlots q;
    q.key = reinterpret_cast<unsigned long long*>(smem);
    q.score = reinterpret_cast<double*>(q.key + cap);
    q.gain = q.score + cap;
    q.lambda = q.gain + cap;
    q.hessian = q.lambda + cap;
    q.pair_lambda = q.hessian + cap;
    q.pair_hessian = q.pair_lambda + cap;
    q.label = reinterpret_cast<float*>(q.pair_hessian + cap);
    return q;
}

__global__ void __launch_bounds__(kRankThreads) lambdarank_kernel(RowArgs r, const int32_t* stopped,
                                                                   unsigned long long* max_g,
                                                                   unsigned long long* max_h) {
    if (stopped != nullptr && *stopped) return;
    extern __shared__ __align__(16) unsigned char smem[];
    const RankArgs& k = r.rank;
    const QuerySlots sl = query_slots(smem, k.cap);
    __shared__ uint32_t s_valid;
    __shared__ double s_norm;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    double mg = 0.0, mh = 0.0;
    for (uint32_t q = blockIdx.x; q < k.num_queries; q += gridDim.x) {
        const uint32_t b = k.bounds[q], n = k.bounds[q + 1] - b;
        if (n == 0) continue;
        uint32_t cap = 2;
        while (cap < n) cap <<= 1;
        // Rank order: keys (descending score, then row), the padding slots last.
        for (uint32_t i = tid; i < cap; i += kRankThreads)
            sl.key[i] = i < n ? (static_cast<unsigned long long>(descending_key(r.scores[b + i])) << 32) | i : ~0ull;
        if (tid == 0) s_valid = n;
        __syncthreads();
        for (uint32_t size = 2; size <= cap; size <<= 1) {
            for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
                for (uint32_t t = tid; t < cap / 2; t += kRankThreads) {
                    const uint32_t lo = 2 * t - (t & (stride - 1)), hi = lo + stride;
                    const unsigned long long x = sl.key[lo], y = sl.key[hi];
                    if ((x > y) == ((lo & size) == 0)) {
                        sl.key[lo] = y;
                        sl.key[hi] = x;
                    }
                }
                __syncthreads();
            }
        }
        // load_ranked (lambdarank.rs:324-341); `valid`: the first rank holding a -inf score (they sort last).
        for (uint32_t i = tid; i < n; i += kRankThreads) {
            const uint32_t row = static_cast<uint32_t>(sl.key[i]);
            const double score = static_cast<double>(r.scores[b + row]);
            const float label = r.label[b + row];
            sl.score[i] = score;
            sl.label[i] = label;
            sl.gain[i] = k.label_gain[static_cast<uint32_t>(label)];
            sl.lambda[i] = 0.0;
            sl.hessian[i] = 0.0;
            if (score == -CUDART_INF) atomicMin(&s_valid, i);
        }
        __syncthreads();
        const uint32_t valid = s_valid;
        // worst_score (lambdarank.rs:344-351): the lowest score, one trailing -inf skipped.
        uint32_t worst = n - 1;
        if (worst > 0 && sl.score[worst] == -CUDART_INF) --worst;
        const bool by_distance = k.norm != 0 && sl.score[0] != sl.score[worst];
        const double inverse_max_dcg = k.inverse_max_dcg[q];
        const uint32_t rows_i = min(k.truncation, valid > 0 ? valid - 1 : 0u);
        double chain_sum = 0.0;  // lane 2 of warp 0: the sum of lambdas over the pairs so far
        for (uint32_t i = 0; i < rows_i; ++i) {
            const double score_i = sl.score[i], gain_i = sl.gain[i], discount_i = __ldg(k.discount + i);
            const float label_i = sl.label[i];
            // accumulate_pairs (lambdarank.rs:353-396), the pairs (i, j) of this phase, each added to row j.
            for (uint32_t j = i + 1 + tid; j < valid; j += kRankThreads) {
                const float label_j = sl.label[j];
                if (label_j == label_i) continue;
                const double sign = label_i > label_j ? 1.0 : -1.0;
                const double delta_score = __dmul_rn(sign, __dsub_rn(score_i, sl.score[j]));
                const double dcg_gap = __dmul_rn(sign, __dsub_rn(gain_i, sl.gain[j]));
                const double paired_discount = fabs(__dsub_rn(discount_i, __ldg(k.discount + j)));
                double delta_pair_ndcg = __dmul_rn(__dmul_rn(dcg_gap, paired_discount), inverse_max_dcg);
                if (by_distance)
                    delta_pair_ndcg = __ddiv_rn(delta_pair_ndcg, __dadd_rn(kScoreDistanceEpsilon, fabs(delta_score)));
                const double p = sigmoid_at(k, delta_score);
                const double p_lambda = __dmul_rn(p, __dmul_rn(-k.sigmoid, delta_pair_ndcg));
                const double p_hessian =
                    __dmul_rn(__dmul_rn(p, __dsub_rn(1.0, p)), __dmul_rn(k.sigmoid_squared, delta_pair_ndcg));
                sl.pair_lambda[j] = p_lambda;
                sl.pair_hessian[j] = p_hessian;
                sl.lambda[j] = __dsub_rn(sl.lambda[j], __dmul_rn(sign, p_lambda));
                sl.hessian[j] = __dadd_rn(sl.hessian[j], p_hessian);
            }
            __syncthreads();
            // Row i's own pairs in j order (lane 0: lambda, lane 1: hessian) and the sum of lambdas (lane 2).
            if (warp == 0 && lane < 3) {
                double v = lane == 0 ? sl.lambda[i] : lane == 1 ? sl.hessian[i] : chain_sum;
                for (uint32_t j = i + 1; j < valid; ++j) {
                    const float label_j = sl.label[j];
                    if (label_j == label_i) continue;
                    const double pl = sl.pair_lambda[j];
                    if (lane == 0)
                        v = __dadd_rn(v, __dmul_rn(label_i > label_j ? 1.0 : -1.0, pl));
                    else if (lane == 1)
                        v = __dadd_rn(v, sl.pair_hessian[j]);
                    else
                        v = __dsub_rn(v, __dmul_rn(2.0, pl));
                }
                if (lane == 0)
                    sl.lambda[i] = v;
                else if (lane == 1)
                    sl.hessian[i] = v;
                else
                    chain_sum = v;
            }
            __syncthreads();
        }
        // query_gradients (lambdarank.rs:300-320): the normalization, the f32 cast, the row weight.
        if (tid == 2)
            s_norm = k.norm != 0 && chain_sum > 0.0 ? __ddiv_rn(log2(__dadd_rn(1.0, chain_sum)), chain_sum) : 1.0;
        __syncthreads();
        const double norm_factor = s_norm;
        for (uint32_t i = tid; i < n; i += kRankThreads) {
            const uint32_t row = static_cast<uint32_t>(sl.key[i]);
            float g = __double2float_rn(__dmul_rn(sl.lambda[i], norm_factor));
            float h = __double2float_rn(__dmul_rn(sl.hessian[i], norm_factor));
            if (r.weight != nullptr) {
                g = __fmul_rn(g, r.weight[b + row]);
                h = __fmul_rn(h, r.weight[b + row]);
            }
            r.grad[b + row] = g;
            r.hess[b + row] = h;
            mg = fmax(mg, static_cast<double>(fabsf(g)));
            mh = fmax(mh, static_cast<double>(fabsf(h)));
        }
        __syncthreads();  // the slots are free for the CTA's next query
    }
    // The CTA's maxima (CpuBackend::compute_gradients' max |grad|, max |hess|): non-negative doubles order like
    // their bit patterns.
    __shared__ double s_mg[kRankThreads / 32], s_mh[kRankThreads / 32];
    for (int o = 16; o > 0; o >>= 1) {
        mg = fmax(mg, __shfl_xor_sync(0xffffffffu, mg, o));
        mh = fmax(mh, __shfl_xor_sync(0xffffffffu, mh, o));
    }
    if (lane == 0) {
        s_mg[warp] = mg;
        s_mh[warp] = mh;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kRankThreads / 32; ++w) {
            mg = fmax(mg, s_mg[w]);
            mh = fmax(mh, s_mh[w]);
        }
        atomicMax(max_g, static_cast<unsigned long long>(__double_as_longlong(mg)));
        atomicMax(max_h, static_cast<unsigned long long>(__double_as_longlong(mh)));
    }
}

}  // namespace

size_t lambdarank_smem(uint32_t cap) { return static_cast<size_t>(cap) * (7 * sizeof(double) + sizeof(float)); }

cudaError_t lambdarank_configure(uint32_t cap, int* blocks_per_sm) {
    const int bytes = static_cast<int>(lambdarank_smem(cap));
    cudaError_t e = cudaFuncSetAttribute(lambdarank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, lambdarank_kernel, kRankThreads, bytes);
}

void launch_lambdarank(const RowArgs& r, const int32_t* stopped, unsigned long long* max_g, unsigned long long* max_h,
                       int grid, cudaStream_t s) {
    lambdarank_kernel<<<grid, kRankThreads, lambdarank_smem(r.rank.cap), s>>>(r, stopped, max_g, max_h);
}

}  // namespace sb2
