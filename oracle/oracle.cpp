// oracle.cpp — CPU restatement of silvic-core's training path. TEST INFRASTRUCTURE ONLY.
//
// This file is the checker the B200 backend is compared against. Only the tests, the smoke check and the bench's
// CPU-baseline leg load it; the product never links, imports or calls it. Each function cites the silvic-core
// source it restates (paths relative to the silvic repository). Floating-point expressions keep the reference's
// operation order; the file is compiled with -ffp-contract=off so no multiply-add is fused unless written as
// std::fma (the reference's `mul_add`).
//
// Parity pins: the quantization and split-finder semantics are pinned by porting the reference's own property
// tests (quantize.rs:167-216, split.rs:987-1507, backend/cpu.rs:945-1180, learner.rs:487-814) into tests/; the
// reference publishes no recorded trainer outputs, so whole-model parity beyond those properties is "unpinned"
// (there is no Rust toolchain to run the reference here).

#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>

#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>

namespace {

thread_local std::string g_error;

// ---- threads ----------------------------------------------------------------------------------------------------

int g_threads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));

// A pool of worker threads kept for the process: a parallel call hands every worker one job and waits for all of
// them, so a call costs two condition-variable round trips instead of creating and joining threads (the trainer makes
// thousands of calls per tree, the reference's rayon pool none of that cost either). Calls come from one thread.
class Pool {
public:
    // Runs job(k) for k in [0, t) on t threads (the caller's among them) and returns when all are done.
    void run(size_t t, const std::function<void(size_t)>& job) {
        if (t <= 1 || inside_) {  // a call from inside a job runs its parts on the calling thread
            for (size_t k = 0; k < t; ++k) job(k);
            return;
        }
        grow(t - 1);
        {
            std::lock_guard<std::mutex> g(lock_);
            job_ = &job;
            active_ = t - 1;
            pending_ = t - 1;
            ++generation_;
        }
        wake_.notify_all();
        inside_ = true;
        job(0);
        inside_ = false;
        std::unique_lock<std::mutex> g(lock_);
        done_.wait(g, [&] { return pending_ == 0; });
        job_ = nullptr;
    }
    ~Pool() {
        {
            std::lock_guard<std::mutex> g(lock_);
            stop_ = true;
        }
        wake_.notify_all();
        for (std::thread& th : workers_) th.join();
    }

private:
    void grow(size_t n) {
        while (workers_.size() < n) {
            const size_t index = workers_.size() + 1;  // job index of the worker; 0 is the caller
            workers_.emplace_back([this, index] { loop(index); });
        }
    }
    void loop(size_t index) {
        uint64_t seen = 0;
        while (true) {
            const std::function<void(size_t)>* job;
            {
                std::unique_lock<std::mutex> g(lock_);
                wake_.wait(g, [&] { return stop_ || generation_ != seen; });
                if (stop_) return;
                seen = generation_;
                if (index > active_) continue;  // this call needs fewer workers
                job = job_;
            }
            inside_ = true;
            (*job)(index);
            inside_ = false;
            std::lock_guard<std::mutex> g(lock_);
            if (--pending_ == 0) done_.notify_one();
        }
    }
    std::vector<std::thread> workers_;
    std::mutex lock_;
    std::condition_variable wake_, done_;
    const std::function<void(size_t)>* job_ = nullptr;
    size_t active_ = 0, pending_ = 0;
    uint64_t generation_ = 0;
    bool stop_ = false;
    static thread_local bool inside_;
};

thread_local bool Pool::inside_ = false;

Pool& pool() {
    static Pool p;
    return p;
}

// Runs body(i) for every i in [0, n), each thread over one contiguous range.
template <class F>
void parallel_for(size_t n, F&& body) {
    size_t t = std::min<size_t>(static_cast<size_t>(g_threads), std::max<size_t>(1, n / 2048));
    if (t <= 1) {
        for (size_t i = 0; i < n; ++i) body(i);
        return;
    }
    pool().run(t, [&](size_t k) {
        size_t b = n * k / t, e = n * (k + 1) / t;
        for (size_t i = b; i < e; ++i) body(i);
    });
}

// Runs body(i) for every i in [0, n), items claimed one at a time (uneven work).
template <class F>
void parallel_tasks(size_t n, F&& body) {
    size_t t = std::min<size_t>(static_cast<size_t>(g_threads), n);
    if (t <= 1) {
        for (size_t i = 0; i < n; ++i) body(i);
        return;
    }
    std::atomic<size_t> next{0};
    pool().run(t, [&](size_t) {
        for (size_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) body(i);
    });
}

// Sums (or otherwise combines) per-thread partial results of body(i, partial) over [0, n).
template <class T, class F, class C>
T parallel_reduce(size_t n, T init, F&& body, C&& combine) {
    size_t t = std::min<size_t>(static_cast<size_t>(g_threads), std::max<size_t>(1, n / 2048));
    std::vector<T> parts(t, init);
    pool().run(t, [&](size_t k) {
        size_t b = n * k / t, e = n * (k + 1) / t;
        for (size_t i = b; i < e; ++i) body(i, parts[k]);
    });
    T out = init;
    for (const T& p : parts) out = combine(out, p);
    return out;
}

// ---- quantize.rs -----------------------------------------------------------------------------------------------

constexpr uint32_t STREAM_GRADIENT = 0;  // quantize.rs:10
constexpr uint32_t STREAM_HESSIAN = 1;   // quantize.rs:11
constexpr uint32_t STREAM_BAGGING = 2;   // quantize.rs:12
constexpr uint32_t STREAM_FEATURE_FRACTION = 3;  // split.rs:41

// quantize.rs:16-23 (lowbias32)
inline uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352dU;
    x ^= x >> 15;
    x *= 0x846ca68bU;
    x ^= x >> 16;
    return x;
}

// quantize.rs:27-31
inline float uniform(uint32_t seed, uint32_t stream, uint32_t iteration, uint64_t row) {
    uint32_t row_hash = mix32(static_cast<uint32_t>(row) ^ mix32(static_cast<uint32_t>(row >> 32)));
    uint32_t h = mix32(seed ^ mix32(stream ^ mix32(iteration ^ row_hash)));
    return static_cast<float>(h >> 8) * (1.0f / 16777216.0f);
}

// Rust's saturating `f32 as i32` / `f64 as i64`.
inline int32_t sat_i32(float q) {
    if (std::isnan(q)) return 0;
    if (q >= 2147483647.0f) return std::numeric_limits<int32_t>::max();
    if (q <= -2147483648.0f) return std::numeric_limits<int32_t>::min();
    return static_cast<int32_t>(q);
}
inline int64_t sat_i64(double q) {
    if (std::isnan(q)) return 0;
    if (q >= 9223372036854775807.0) return std::numeric_limits<int64_t>::max();
    if (q <= -9223372036854775808.0) return std::numeric_limits<int64_t>::min();
    return static_cast<int64_t>(q);
}

inline double positive_or_one(double v) { return (v > 0.0 && std::isfinite(v)) ? v : 1.0; }  // quantize.rs:92-98

// quantize.rs:56-84
sb2_quant_spec quant_spec(double max_abs_grad, double max_hess, bool has_constant, double constant, uint32_t num_bins,
                          bool stochastic, uint32_t seed, uint32_t iteration) {
    sb2_quant_spec s{};
    s.grad_max_q = static_cast<int32_t>(num_bins / 2);
    s.hess_max_q = static_cast<int32_t>(num_bins);
    s.grad_scale = positive_or_one(max_abs_grad / static_cast<double>(s.grad_max_q));
    s.hess_scale = has_constant ? positive_or_one(constant)
                                : positive_or_one(max_hess / static_cast<double>(s.hess_max_q));
    s.inv_grad_scale = static_cast<float>(1.0 / s.grad_scale);
    s.inv_hess_scale = static_cast<float>(1.0 / s.hess_scale);
    s.constant_hessian = has_constant;
    s.stochastic = stochastic;
    s.seed = seed;
    s.iteration = iteration;
    return s;
}

// quantize.rs:110-122
inline int32_t quantize_grad(const sb2_quant_spec& s, float grad, uint64_t row) {
    float q;
    if (s.stochastic) {
        float u = uniform(s.seed, STREAM_GRADIENT, s.iteration, row);
        q = grad >= 0.0f ? std::trunc(std::fmaf(grad, s.inv_grad_scale, u))
                         : std::trunc(std::fmaf(grad, s.inv_grad_scale, -u));
    } else {
        q = std::nearbyintf(grad * s.inv_grad_scale);
    }
    return std::clamp(sat_i32(q), -s.grad_max_q, s.grad_max_q);
}

// quantize.rs:125-136
inline int32_t quantize_hess(const sb2_quant_spec& s, float hess, uint64_t row) {
    if (s.constant_hessian) return 1;
    float q;
    if (s.stochastic) {
        float u = uniform(s.seed, STREAM_HESSIAN, s.iteration, row);
        q = std::trunc(std::fmaf(hess, s.inv_hess_scale, u));
    } else {
        q = std::nearbyintf(hess * s.inv_hess_scale);
    }
    return std::clamp(sat_i32(q), 0, s.hess_max_q);
}

// quantize.rs:103-107
inline int32_t quantize_row(const sb2_quant_spec& s, float grad, float hess, uint64_t row) {
    return quantize_hess(s, hess, row) * 65536 + quantize_grad(s, grad, row);
}

// quantize.rs:140-143
inline void unpack(int32_t packed, int32_t& g, int32_t& h) {
    g = static_cast<int16_t>(static_cast<uint16_t>(static_cast<uint32_t>(packed)));
    h = (packed - g) >> 16;
}

// quantize.rs:147-149
inline bool in_bag(uint32_t seed, uint32_t round, uint64_t row, double fraction) {
    return static_cast<double>(uniform(seed, STREAM_BAGGING, round, row)) < fraction;
}

// quantize.rs:153-159
float fixed_point_scale(double max_abs) {
    if (!std::isfinite(max_abs) || max_abs <= 0.0) return 1.0f;
    int exponent = 30 - static_cast<int>(std::ceil(std::log2(max_abs)));
    exponent = std::clamp(exponent, -126, 127);
    return std::ldexp(1.0f, exponent);
}

// quantize.rs:163-165
inline int64_t to_fixed(float value, float scale) {
    return sat_i64(static_cast<double>(std::nearbyintf(value * scale)));
}

// ---- objective --------------------------------------------------------------------------------------------------

constexpr double K_EPSILON = static_cast<double>(1e-15f);  // objective/mod.rs:20, split.rs:37

// objective/regression.rs:20-43 and objective/binary.rs:27-50
void gradients(const sb2_objective& o, const float* scores, const float* label, const float* weight, size_t n,
               float* grad, float* hess) {
    if (o.kind == SB2_REGRESSION) {
        parallel_for(n, [&](size_t row) {
            float residual = scores[row] - label[row];
            if (weight) {
                grad[row] = residual * weight[row];
                hess[row] = weight[row];
            } else {
                grad[row] = residual;
                hess[row] = 1.0f;
            }
        });
    } else {
        const double sigmoid = o.sigmoid;
        parallel_for(n, [&](size_t row) {
            double sign = label[row] > 0.0f ? 1.0 : -1.0;
            double response = -sign * sigmoid / (1.0 + std::exp(sign * sigmoid * static_cast<double>(scores[row])));
            double abs_response = std::fabs(response);
            double w = weight ? static_cast<double>(weight[row]) : 1.0;
            grad[row] = static_cast<float>(response * w);
            hess[row] = static_cast<float>(abs_response * (sigmoid - abs_response) * w);
        });
    }
}

// ---- objective/lambdarank.rs ----------------------------------------------------------------------------------

constexpr size_t MAX_POSITION = 10000;             // lambdarank.rs:25
constexpr double MIN_SIGMOID_INPUT = -50.0;        // lambdarank.rs:28
constexpr size_t SIGMOID_BINS = 1024 * 1024;       // lambdarank.rs:31
constexpr double SCORE_DISTANCE_EPSILON = static_cast<double>(0.01f);  // lambdarank.rs:34

// lambdarank.rs:37-46: 1 / log2(2 + rank)
double discount(size_t rank) { return 1.0 / std::log2(2.0 + static_cast<double>(rank)); }

// config.rs:118-121
std::vector<double> default_label_gain() {
    std::vector<double> g;
    for (uint32_t i = 0; i < 31; ++i) g.push_back(static_cast<double>((1u << i) - 1u));
    return g;
}

// lambdarank.rs:122-139 (DCGCalculator::CalMaxDCGAtK)
double max_dcg_at_k(size_t k, const float* labels, size_t n, const std::vector<double>& gain) {
    std::vector<size_t> count(gain.size(), 0);
    for (size_t i = 0; i < n; ++i) ++count[static_cast<size_t>(labels[i])];
    size_t top = gain.size() - 1;
    double dcg = 0.0;
    for (size_t j = 0; j < std::min(k, n); ++j) {
        while (top > 0 && count[top] == 0) --top;
        dcg += discount(j) * gain[top];
        --count[top];  // wraps at label 0, as the reference's wrapping_sub
    }
    return dcg;
}

// ObjectiveSetup::LambdaRank (objective/mod.rs:35-65) with the sigmoid table (lambdarank.rs:51-120) of one rank.
struct LambdaRank {
    double sigmoid = 1.0;
    bool norm = true;
    size_t truncation_level = 30;
    std::vector<double> label_gain, inverse_max_dcg;
    const std::vector<double>* table = nullptr;  // shared by the setups of one sigmoid
    double min_input = 0.0, max_input = 0.0, idx_factor = 0.0;
};

bool lambdarank_setup(const sb2_params& p, const sb2_dataset& d, LambdaRank& out) {
    if (!d.query_boundaries || d.num_queries == 0 || d.query_boundaries[0] != 0 ||
        d.query_boundaries[d.num_queries] != d.num_rows) {
        g_error = "ranking tasks require query information";
        return false;
    }
    out.sigmoid = p.sigmoid;
    out.norm = p.lambdarank_norm != 0;
    out.truncation_level = p.lambdarank_truncation_level;
    out.label_gain = p.label_gain && p.num_label_gain ? std::vector<double>(p.label_gain, p.label_gain + p.num_label_gain)
                                                     : default_label_gain();
    for (size_t i = 0; i < d.num_rows; ++i) {  // check_labels (lambdarank.rs:173-195)
        const float l = d.label[i];
        if (std::fabs(static_cast<double>(l) - static_cast<double>(static_cast<int32_t>(l))) > K_EPSILON || l < 0.0f ||
            static_cast<size_t>(l) >= out.label_gain.size()) {
            g_error = "lambdarank label " + std::to_string(l) + " is not an integer below the label gains";
            return false;
        }
    }
    out.inverse_max_dcg.resize(d.num_queries);
    for (uint32_t q = 0; q < d.num_queries; ++q) {
        const uint32_t b = d.query_boundaries[q], e = d.query_boundaries[q + 1];
        const double m = max_dcg_at_k(out.truncation_level, d.label + b, e - b, out.label_gain);
        out.inverse_max_dcg[q] = m > 0.0 ? 1.0 / m : 0.0;
    }
    out.min_input = MIN_SIGMOID_INPUT / out.sigmoid / 2.0;
    out.max_input = -out.min_input;
    out.idx_factor = static_cast<double>(SIGMOID_BINS) / (out.max_input - out.min_input);
    // The table for this sigmoid, built once and kept while the sigmoid stays the same (SigmoidTable::shared).
    static double cached_sigmoid = std::numeric_limits<double>::quiet_NaN();
    static std::vector<double> cached;
    if (!(cached_sigmoid == out.sigmoid)) {
        cached.resize(SIGMOID_BINS);
        for (size_t i = 0; i < SIGMOID_BINS; ++i) {
            const double score = static_cast<double>(i) / out.idx_factor + out.min_input;
            cached[i] = 1.0 / (1.0 + std::exp(score * out.sigmoid));
        }
        cached_sigmoid = out.sigmoid;
    }
    out.table = &cached;
    return true;
}

// SigmoidTable::get (lambdarank.rs:110-119)
double sigmoid_at(const LambdaRank& lr, double delta) {
    const std::vector<double>& table = *lr.table;
    if (delta <= lr.min_input) return table[0];
    if (delta >= lr.max_input) return table[SIGMOID_BINS - 1];
    return table[std::min(static_cast<size_t>((delta - lr.min_input) * lr.idx_factor), SIGMOID_BINS - 1)];
}

// descending_key (lambdarank.rs:162-168): ascending order of the key is descending order of the score.
uint32_t descending_key(float score) {
    float v = score + 0.0f;
    uint32_t bits;
    std::memcpy(&bits, &v, 4);
    const uint32_t ascending = (bits >> 31) == 1 ? ~bits : (bits | (1u << 31));
    return ~ascending;
}

// query_gradients (lambdarank.rs:264-321) with load_ranked (:324-341), worst_score (:344-351) and accumulate_pairs
// (:353-396) for one query of n rows.
void lambdarank_query(const LambdaRank& lr, size_t query, const float* scores, const float* label, const float* weight,
                      size_t n, float* grad, float* hess) {
    if (n == 0) return;
    std::vector<uint64_t> keys(n);
    for (size_t r = 0; r < n; ++r) keys[r] = (static_cast<uint64_t>(descending_key(scores[r])) << 32) | r;
    std::sort(keys.begin(), keys.end());
    std::vector<size_t> order(n);
    std::vector<double> score(n), gain(n), disc(n), lambda(n, 0.0), hessian(n, 0.0);
    std::vector<float> lab(n);
    for (size_t k = 0; k < n; ++k) {
        order[k] = static_cast<size_t>(keys[k] & 0xFFFFFFFFull);
        score[k] = static_cast<double>(scores[order[k]]);
        lab[k] = label[order[k]];
        gain[k] = lr.label_gain[static_cast<size_t>(lab[k])];
        disc[k] = discount(k);
    }
    size_t worst = n - 1;
    if (worst > 0 && score[worst] == -std::numeric_limits<double>::infinity()) --worst;
    const bool norm_by_distance = lr.norm && score[0] != score[worst];
    const double inverse_max_dcg = lr.inverse_max_dcg[query];
    size_t valid = n;
    for (size_t k = 0; k < n; ++k)
        if (score[k] == -std::numeric_limits<double>::infinity()) {
            valid = k;
            break;
        }
    const double sigmoid_squared = lr.sigmoid * lr.sigmoid;
    double sum_lambdas = 0.0;
    const size_t rows_i = std::min(lr.truncation_level, valid > 0 ? valid - 1 : 0);
    for (size_t i = 0; i < rows_i; ++i) {
        double lambda_i = lambda[i], hessian_i = hessian[i];
        for (size_t j = i + 1; j < valid; ++j) {
            if (lab[j] == lab[i]) continue;
            const double sign = lab[i] > lab[j] ? 1.0 : -1.0;
            const double delta_score = sign * (score[i] - score[j]);
            const double dcg_gap = sign * (gain[i] - gain[j]);
            const double paired_discount = std::fabs(disc[i] - disc[j]);
            double delta_pair_ndcg = dcg_gap * paired_discount * inverse_max_dcg;
            if (norm_by_distance) delta_pair_ndcg /= SCORE_DISTANCE_EPSILON + std::fabs(delta_score);
            const double p = sigmoid_at(lr, delta_score);
            const double p_lambda = p * (-lr.sigmoid * delta_pair_ndcg);
            const double p_hessian = p * (1.0 - p) * (sigmoid_squared * delta_pair_ndcg);
            lambda_i += sign * p_lambda;
            lambda[j] -= sign * p_lambda;
            hessian_i += p_hessian;
            hessian[j] += p_hessian;
            sum_lambdas -= 2.0 * p_lambda;
        }
        lambda[i] = lambda_i;
        hessian[i] = hessian_i;
    }
    const double norm_factor = lr.norm && sum_lambdas > 0.0 ? std::log2(1.0 + sum_lambdas) / sum_lambdas : 1.0;
    for (size_t k = 0; k < n; ++k) {
        float g = static_cast<float>(lambda[k] * norm_factor);
        float h = static_cast<float>(hessian[k] * norm_factor);
        if (weight) {
            g = g * weight[order[k]];
            h = h * weight[order[k]];
        }
        grad[order[k]] = g;
        hess[order[k]] = h;
    }
}

// lambdarank::gradients (lambdarank.rs:197-240): every query of one rank, in parallel over queries.
void lambdarank_gradients(const LambdaRank& lr, const sb2_dataset& d, const float* scores, float* grad, float* hess) {
    parallel_tasks(d.num_queries, [&](size_t q) {
        const uint32_t b = d.query_boundaries[q], e = d.query_boundaries[q + 1];
        lambdarank_query(lr, q, scores + b, d.label + b, d.weight ? d.weight + b : nullptr, e - b, grad + b, hess + b);
    });
}

// objective/regression.rs:8-17 and binary.rs:8-16: [sum label * weight, sum weight] in row order.
void label_sums(int objective, const float* label, const float* weight, size_t n, double out[2]) {
    double l = 0.0, w = 0.0;
    for (size_t i = 0; i < n; ++i) {
        float y = objective == SB2_BINARY ? (label[i] > 0.0f ? 1.0f : 0.0f) : label[i];
        if (weight) {
            l += static_cast<double>(y * weight[i]);
            w += static_cast<double>(weight[i]);
        } else {
            l += static_cast<double>(y);
        }
    }
    out[0] = l;
    out[1] = weight ? w : static_cast<double>(n);
}

// objective/mod.rs:92-109; `sums` already reduced over ranks.
double init_score_from_sums(const sb2_params& p, const double sums[2]) {
    if (!p.boost_from_average || p.objective == SB2_LAMBDARANK) return 0.0;
    double score;
    if (p.objective == SB2_BINARY) {
        double prate = std::clamp(sums[0] / sums[1], K_EPSILON, 1.0 - K_EPSILON);  // binary.rs:18-21
        score = std::log(prate / (1.0 - prate)) / p.sigmoid;
    } else {
        score = sums[0] / sums[1];
    }
    return std::fabs(score) > K_EPSILON ? score : 0.0;
}

// ---- dataset helpers --------------------------------------------------------------------------------------------

inline uint8_t bin_of(const sb2_dataset& d, uint32_t feature, size_t row) {
    const sb2_feature& f = d.features[feature];
    const sb2_group& g = d.groups[f.group];
    return g.data[row * g.row_stride + f.column];
}

// GroupLayout (backend/cpu.rs:48-99, group_layout :178-223): per group, the column runs a histogram adds.
struct GroupLayout {
    size_t stride = 0, hist_offset = 0, bins = 0, width = 0;
    std::vector<int64_t> column_feature;  // -1: no feature
    std::vector<size_t> offsets;          // feature's first bin within the group; `bins` (scratch) for none
    std::vector<std::pair<uint32_t, uint32_t>> runs;
    size_t adds = 0;

    // GroupLayout::activate (backend/cpu.rs:69-98)
    void activate(const uint8_t* used, uint32_t num_features) {
        runs.clear();
        auto wanted = [&](int64_t f) {
            if (f < 0) return false;
            if (!used) return true;
            return static_cast<uint32_t>(f) < num_features ? used[f] != 0 : true;
        };
        size_t active = 0;
        for (int64_t f : column_feature)
            if (wanted(f)) ++active;
        if (active == 0) {
            adds = 0;
            return;
        }
        if (active * 4 >= width * 3) {
            runs.emplace_back(0, static_cast<uint32_t>(width));
            adds = width;
            return;
        }
        adds = active;
        int64_t start = -1;
        for (size_t c = 0; c < width; ++c) {
            bool w = wanted(column_feature[c]);
            if (w && start < 0) start = static_cast<int64_t>(c);
            if (!w && start >= 0) {
                runs.emplace_back(static_cast<uint32_t>(start), static_cast<uint32_t>(c));
                start = -1;
            }
        }
        if (start >= 0) runs.emplace_back(static_cast<uint32_t>(start), static_cast<uint32_t>(width));
    }
};

bool group_layouts(const sb2_dataset& d, std::vector<GroupLayout>& out) {
    out.clear();
    for (uint32_t gi = 0; gi < d.num_groups; ++gi) {
        const sb2_group& g = d.groups[gi];
        GroupLayout l;
        l.bins = g.total_bins;
        l.stride = g.row_stride;
        l.hist_offset = g.hist_offset;
        size_t width = 0;
        for (uint32_t k = 0; k < g.num_features; ++k)
            width = std::max<size_t>(width, d.features[g.features[k]].column + 1);
        l.width = width;
        l.column_feature.assign(width, -1);
        l.offsets.assign(width, l.bins);
        for (uint32_t k = 0; k < g.num_features; ++k) {
            uint32_t f = g.features[k];
            const sb2_feature& m = d.features[f];
            if (m.hist_offset < g.hist_offset || m.hist_offset - g.hist_offset + m.num_bins > l.bins ||
                m.column >= l.stride) {
                g_error = "feature lies outside its group's bins or row";
                return false;
            }
            l.column_feature[m.column] = f;
            l.offsets[m.column] = m.hist_offset - g.hist_offset;
        }
        l.activate(nullptr, d.num_features);
        out.push_back(std::move(l));
    }
    return true;
}

constexpr size_t MIN_ADDS_PER_BIN = 16;     // backend/cpu.rs:26
constexpr size_t MAX_BLOCKS_PER_GROUP = 64; // backend/cpu.rs:29
constexpr size_t SCRATCH_BINS = 256;        // backend/cpu.rs:31

// histogram_quantized (backend/cpu.rs:479-525 with histogram_blocks :374-415 and merge_blocks :419-463): each
// (group, row block) task adds the rows' packed (h << 32) + g into an i64 accumulator of the group's bins, flushing
// into exact (g, h) sums before the gradient half could leave i32; blocks then add in block order.
void histogram_quantized(const sb2_dataset& d, const std::vector<GroupLayout>& layout, const int32_t* packed,
                         int64_t max_quant, const uint32_t* rows, size_t n, double* out) {
    const size_t row_limit = static_cast<size_t>(static_cast<int64_t>(INT32_MAX) / std::max<int64_t>(max_quant, 1));
    std::vector<int64_t> gh(n);
    parallel_for(n, [&](size_t i) {
        int32_t g, h;
        unpack(packed[rows[i]], g, h);
        gh[i] = (static_cast<int64_t>(h) << 32) + static_cast<int64_t>(g);
    });
    struct Task {
        size_t group, start, end;
    };
    std::vector<Task> tasks;
    for (size_t gi = 0; gi < layout.size(); ++gi) {
        const GroupLayout& l = layout[gi];
        if (l.adds == 0) continue;
        size_t min_rows = (MIN_ADDS_PER_BIN * l.bins + l.adds - 1) / std::max<size_t>(l.adds, 1);
        size_t size = std::max<size_t>({min_rows, (n + MAX_BLOCKS_PER_GROUP - 1) / MAX_BLOCKS_PER_GROUP, 1});
        size_t count = std::max<size_t>((n + size - 1) / size, 1);
        for (size_t b = 0; b < count; ++b)
            tasks.push_back({gi, std::min(b * size, n), std::min((b + 1) * size, n)});
    }
    std::vector<std::vector<int64_t>> sums(tasks.size());  // per task: [g, h] per bin (+ scratch)
    parallel_tasks(tasks.size(), [&](size_t t) {
        const Task& task = tasks[t];
        const GroupLayout& l = layout[task.group];
        const uint8_t* data = d.groups[task.group].data;
        std::vector<int64_t>& s = sums[t];
        s.assign(2 * (l.bins + SCRATCH_BINS), 0);
        std::vector<int64_t> acc(l.bins + SCRATCH_BINS, 0);
        for (size_t chunk = task.start; chunk < task.end; chunk += row_limit) {
            size_t chunk_end = std::min(task.end, chunk + row_limit);
            for (size_t i = chunk; i < chunk_end; ++i) {
                const uint8_t* bins = data + static_cast<size_t>(rows[i]) * l.stride;
                int64_t v = gh[i];
                for (auto [start, end] : l.runs)
                    for (uint32_t c = start; c < end; ++c) acc[l.offsets[c] + bins[c]] += v;
            }
            // flush_packed (backend/cpu.rs:517-525)
            for (size_t b = 0; b < acc.size(); ++b) {
                int64_t g = static_cast<int32_t>(acc[b]);
                s[2 * b] += g;
                s[2 * b + 1] += (acc[b] - g) >> 32;
                acc[b] = 0;
            }
        }
    });
    const size_t total = d.total_bins;
    std::fill(out, out + 2 * total, 0.0);
    std::vector<std::vector<size_t>> by_group(layout.size());
    for (size_t t = 0; t < tasks.size(); ++t) by_group[tasks[t].group].push_back(t);
    for (size_t gi = 0; gi < layout.size(); ++gi) {
        const GroupLayout& l = layout[gi];
        const std::vector<size_t>& mine = by_group[gi];
        if (mine.empty()) continue;
        parallel_for(2 * l.bins, [&](size_t b) {
            int64_t v = 0;
            for (size_t t : mine) v += sums[t][b];
            out[2 * l.hist_offset + b] = static_cast<double>(v);
        });
    }
}

// stable_partition (backend/cpu.rs:556-599) over chunks of ROW_CHUNK rows.
uint32_t stable_partition(const sb2_dataset& d, const sb2_bin_split& split, uint32_t* rows, size_t n) {
    const sb2_group& g = d.groups[split.group];
    auto goes_left = [&](uint32_t row) {
        uint8_t bin = g.data[static_cast<size_t>(row) * g.row_stride + split.column];
        return ((split.left_bins[bin / 32] >> (bin % 32)) & 1u) == 1u;
    };
    constexpr size_t ROW_CHUNK = 8192;
    size_t chunks = (n + ROW_CHUNK - 1) / ROW_CHUNK;
    std::vector<uint32_t> scratch(n);
    std::vector<size_t> lefts(chunks);
    parallel_for(chunks, [&](size_t c) {
        size_t b = c * ROW_CHUNK, e = std::min(n, b + ROW_CHUNK);
        size_t left = b, right = e;
        for (size_t i = b; i < e; ++i) {
            if (goes_left(rows[i]))
                scratch[left++] = rows[i];
            else
                scratch[--right] = rows[i];
        }
        std::reverse(scratch.begin() + left, scratch.begin() + e);
        lefts[c] = left - b;
    });
    size_t total_left = std::accumulate(lefts.begin(), lefts.end(), size_t{0});
    std::vector<size_t> lpos(chunks), rpos(chunks);
    size_t lp = 0, rp = total_left;
    for (size_t c = 0; c < chunks; ++c) {
        size_t len = std::min(ROW_CHUNK, n - c * ROW_CHUNK);
        lpos[c] = lp;
        rpos[c] = rp;
        lp += lefts[c];
        rp += len - lefts[c];
    }
    parallel_for(chunks, [&](size_t c) {
        size_t b = c * ROW_CHUNK, e = std::min(n, b + ROW_CHUNK);
        std::copy(scratch.begin() + b, scratch.begin() + b + lefts[c], rows + lpos[c]);
        std::copy(scratch.begin() + b + lefts[c], scratch.begin() + e, rows + rpos[c]);
    });
    return static_cast<uint32_t>(total_left);
}

// add_tree_to (backend/cpu.rs:605-695): binned traversal, leaves are ~index.
bool add_tree(const sb2_dataset& d, const sb2_device_node* nodes, size_t num_nodes, const float* leaf_values,
              size_t num_leaves, float* scores) {
    if (num_leaves == 0 || num_leaves != num_nodes + 1) {
        g_error = "tree with inconsistent node and leaf counts";
        return false;
    }
    const size_t n = d.num_rows;
    if (num_nodes == 0) {
        parallel_for(n, [&](size_t r) { scores[r] += leaf_values[0]; });
        return true;
    }
    for (size_t k = 0; k < num_nodes; ++k) {
        if (nodes[k].split.group >= d.num_groups) {
            g_error = "malformed device tree";
            return false;
        }
        for (int32_t c : {nodes[k].left, nodes[k].right}) {
            bool ok = c >= 0 ? (static_cast<size_t>(c) > k && static_cast<size_t>(c) < num_nodes)
                             : (static_cast<size_t>(~c) < num_leaves);
            if (!ok) {
                g_error = "malformed device tree";
                return false;
            }
        }
    }
    parallel_for(n, [&](size_t r) {
        int32_t node = 0;
        while (node >= 0) {
            const sb2_device_node& nd = nodes[node];
            const sb2_group& g = d.groups[nd.split.group];
            uint8_t bin = g.data[r * g.row_stride + nd.split.column];
            bool left = ((nd.split.left_bins[bin >> 5] >> (bin & 31)) & 1u) != 0;
            node = left ? nd.left : nd.right;
        }
        scores[r] += leaf_values[~node];
    });
    return true;
}

// ---- split.rs ---------------------------------------------------------------------------------------------------

constexpr double MIN_SCORE = -std::numeric_limits<double>::infinity();  // split.rs:39
constexpr size_t MAX_BINS = 256;                                      // split.rs:43

struct HistScale {
    double grad, hess;
};
struct LeafSums {
    double grad = 0.0, hess = 0.0;
    int64_t count = 0;
};

inline double sign(double x) { return static_cast<double>((x > 0.0) - (x < 0.0)); }  // split.rs:151-154
inline double threshold_l1(double s, double l1) { return sign(s) * std::fmax(std::fabs(s) - l1, 0.0); }  // :145
// split.rs:159-162
inline double leaf_gain(double g, double h, double l1, double l2) {
    double r = std::fmax(std::fabs(g) - l1, 0.0);
    return r * r / (h + l2);
}
// split.rs:167-186 (scalar lanes added in lane order)
inline double split_gain(double g0, double g1, double h0, double h1, double l1, double l2) {
    return leaf_gain(g0, h0, l1, l2) + leaf_gain(g1, h1, l1, l2);
}
// split.rs:190-192
inline double leaf_output(double g, double h, double l1, double l2) { return -threshold_l1(g, l1) / (h + l2); }
// split.rs:196-198
inline int64_t round_int(double x) { return sat_i64(x + 0.5); }

// LeafCtx (split.rs:201-233)
struct LeafCtx {
    const sb2_split_config* cfg;
    HistScale scale;
    LeafSums units;
    double sum_grad, sum_hess;
    int64_t num_data;
    double cnt_factor, min_gain_shift;
};

bool leaf_ctx(const sb2_split_config* cfg, HistScale scale, LeafSums units, LeafCtx& ctx) {
    if (std::isnan(units.hess) || units.hess <= 0.0 || units.count <= 0) return false;
    ctx.cfg = cfg;
    ctx.scale = scale;
    ctx.units = units;
    ctx.sum_grad = units.grad * scale.grad;
    ctx.sum_hess = units.hess * scale.hess + 2.0 * K_EPSILON;
    double gain_shift = leaf_gain(ctx.sum_grad, ctx.sum_hess, cfg->lambda_l1, cfg->lambda_l2);
    ctx.num_data = units.count;
    ctx.cnt_factor = static_cast<double>(units.count) / ctx.sum_hess;
    ctx.min_gain_shift = gain_shift + cfg->min_gain_to_split;
    return true;
}

struct Grown {
    size_t bin;
    double units[2];
    int64_t count;
    double gain;
};

// ScanBuffer (split.rs:386-531): fill, evaluate, best.
struct ScanBuffer {
    uint16_t bin[MAX_BINS];
    double grad[MAX_BINS], hess[MAX_BINS], gain[MAX_BINS];
    int64_t count[MAX_BINS];

    // ScanBuffer::fill (split.rs:420-444); `order` lists bins in scan order.
    size_t fill(const LeafCtx& ctx, const double* hist, const uint32_t* order, size_t len_in) {
        const int64_t min_count = std::max<int64_t>(ctx.cfg->min_data_in_leaf, 1);
        const double min_hess = ctx.cfg->min_sum_hessian_in_leaf;
        double g = 0.0, uh = 0.0;
        int64_t count_acc = 0;
        size_t len = 0;
        for (size_t k = 0; k < std::min(len_in, MAX_BINS); ++k) {
            uint32_t t = order[k];
            const double* b = hist + 2 * t;
            g += b[0];
            uh += b[1];
            count_acc += round_int(b[1] * ctx.scale.hess * ctx.cnt_factor);
            double h = K_EPSILON + uh * ctx.scale.hess;
            bool skip = count_acc < min_count || h < min_hess || uh <= 0.0;
            bool other_small = ctx.num_data - count_acc < min_count || ctx.sum_hess - h < min_hess ||
                               ctx.units.hess - uh <= 0.0;
            if (other_small && !skip) break;
            bin[k] = static_cast<uint16_t>(t);
            grad[k] = g;
            hess[k] = uh;
            count[k] = count_acc;
            len = k + 1;
        }
        return len;
    }

    // ScanBuffer::evaluate (split.rs:448-462)
    void evaluate(const LeafCtx& ctx, size_t len) {
        const sb2_split_config& c = *ctx.cfg;
        const int64_t min_count = std::max<int64_t>(c.min_data_in_leaf, 1);
        for (size_t k = 0; k < len; ++k) {
            double h = K_EPSILON + hess[k] * ctx.scale.hess;
            bool skip = count[k] < min_count || h < c.min_sum_hessian_in_leaf || hess[k] <= 0.0;
            double g = grad[k] * ctx.scale.grad;
            double gn = split_gain(ctx.sum_grad - g, g, ctx.sum_hess - h, h, c.lambda_l1, c.lambda_l2);
            gain[k] = skip ? -std::numeric_limits<double>::infinity() : gn;
        }
    }

    // ScanBuffer::best (split.rs:508-531): the first strict maximum above min_gain_shift (NaN never wins).
    bool best(const LeafCtx& ctx, size_t stop, Grown& out) const {
        double mx = -std::numeric_limits<double>::infinity();
        for (size_t k = 0; k < stop; ++k) mx = std::fmax(mx, gain[k]);
        if (!(mx > ctx.min_gain_shift)) return false;
        for (size_t k = 0; k < stop; ++k) {
            if (gain[k] == mx) {
                out.bin = bin[k];
                out.units[0] = grad[k];
                out.units[1] = hess[k];
                out.count = count[k];
                out.gain = gain[k];
                return true;
            }
        }
        return false;
    }

    bool complete(const LeafCtx& ctx, size_t len, bool& splittable, Grown& out) {
        evaluate(ctx, len);
        bool found = best(ctx, len, out);
        splittable |= found;
        return found;
    }
};

struct Best {
    double gain;
    uint32_t threshold;
    double left_grad, left_hess;
    int64_t left_count;
    double left_units[2];
};

// CandidateKind (split.rs:318-327)
enum CandidateKind { kNumerical = 0, kOneHot = 1, kSortedForward = 2, kSortedReverse = 3 };

struct Candidate {
    int64_t feature;
    double gain;
    Best best;
    bool default_left;
    int kind = kNumerical;
};

// reverse_best (split.rs:557-567)
Best reverse_best(const LeafCtx& ctx, const Grown& right) {
    double right_hess = K_EPSILON + right.units[1] * ctx.scale.hess;
    Best b;
    b.gain = right.gain;
    b.threshold = static_cast<uint32_t>(right.bin - 1);
    b.left_grad = ctx.sum_grad - right.units[0] * ctx.scale.grad;
    b.left_hess = ctx.sum_hess - right_hess;
    b.left_count = ctx.num_data - right.count;
    b.left_units[0] = ctx.units.grad - right.units[0];
    b.left_units[1] = ctx.units.hess - right.units[1];
    return b;
}

// forward_best (split.rs:571-580)
Best forward_best(const LeafCtx& ctx, const Grown& left) {
    Best b;
    b.gain = left.gain;
    b.threshold = static_cast<uint32_t>(left.bin);
    b.left_grad = left.units[0] * ctx.scale.grad;
    b.left_hess = K_EPSILON + left.units[1] * ctx.scale.hess;
    b.left_count = left.count;
    b.left_units[0] = left.units[0];
    b.left_units[1] = left.units[1];
    return b;
}

// find_numerical (split.rs:584-620)
bool find_numerical(const LeafCtx& ctx, int64_t feature, const double* hist, size_t num_bins, bool nan_bin,
                    bool& splittable, Candidate& cand) {
    static thread_local ScanBuffer reverse, forward;
    uint32_t order[MAX_BINS];
    splittable = false;
    bool have = false;
    Best result{};
    bool result_default_left = false;
    Grown grown{};
    if (nan_bin && num_bins > 2) {
        size_t last = num_bins - 2;
        size_t m = 0;
        for (size_t t = last; t >= 1; --t) order[m++] = static_cast<uint32_t>(t);
        size_t reverse_len = reverse.fill(ctx, hist, order, m);
        for (size_t t = 0; t <= last; ++t) order[t] = static_cast<uint32_t>(t);
        size_t forward_len = forward.fill(ctx, hist, order, last + 1);
        double output_gain = MIN_SCORE;
        if (reverse.complete(ctx, reverse_len, splittable, grown)) {
            result = reverse_best(ctx, grown);
            output_gain = result.gain - ctx.min_gain_shift;
            result_default_left = true;
            have = true;
        }
        if (forward.complete(ctx, forward_len, splittable, grown)) {
            Best b = forward_best(ctx, grown);
            if (b.gain > output_gain + ctx.min_gain_shift) {
                result = b;
                result_default_left = false;
                have = true;
            }
        }
    } else if (num_bins >= 2) {
        size_t m = 0;
        for (size_t t = num_bins - 1; t >= 1; --t) order[m++] = static_cast<uint32_t>(t);
        size_t len = reverse.fill(ctx, hist, order, m);
        if (reverse.complete(ctx, len, splittable, grown)) {
            result = reverse_best(ctx, grown);
            result_default_left = !nan_bin;
            have = true;
        }
    }
    if (have) {
        cand.feature = feature;
        cand.gain = result.gain - ctx.min_gain_shift;
        cand.best = result;
        cand.default_left = result_default_left;
    }
    return have;
}

// LeafCtx::bin_count (split.rs:236-239)
inline int64_t bin_count(const LeafCtx& ctx, double hess_units) {
    return round_int(hess_units * ctx.scale.hess * ctx.cnt_factor);
}

// Check and LeafCtx::check (split.rs:241-261)
enum class Check { Continue, Break, Evaluate };

// Side (split.rs:269-296): the side of a scan that accumulates bins; its real hessian starts at kEpsilon.
struct Side {
    double units[2] = {0.0, 0.0};
    int64_t count = 0;
    double hess = K_EPSILON;
    void add(const LeafCtx& ctx, const double* bin) {
        units[0] += bin[0];
        units[1] += bin[1];
        count += bin_count(ctx, bin[1]);
        hess = K_EPSILON + units[1] * ctx.scale.hess;
    }
};

Check check(const LeafCtx& ctx, const Side& grow, int64_t shrink_count, double shrink_hess) {
    const sb2_split_config& c = *ctx.cfg;
    if (grow.count < c.min_data_in_leaf || grow.count <= 0 || grow.hess < c.min_sum_hessian_in_leaf ||
        grow.units[1] <= 0.0)
        return Check::Continue;
    if (shrink_count < c.min_data_in_leaf || shrink_count <= 0) return Check::Break;
    if (shrink_hess < c.min_sum_hessian_in_leaf || ctx.units.hess - grow.units[1] <= 0.0) return Check::Break;
    return Check::Evaluate;
}

// find_onehot (split.rs:694-737): one category left, the rest right.
bool find_onehot(const LeafCtx& ctx, int64_t feature, const double* hist, size_t num_bins, bool& splittable,
                 Candidate& cand) {
    const sb2_split_config& c = *ctx.cfg;
    splittable = false;
    bool have = false;
    Best best{};
    for (size_t t = 1; t < num_bins; ++t) {
        const double* bin = hist + 2 * t;
        Side left;
        left.add(ctx, bin);
        const int64_t other_count = ctx.num_data - left.count;
        // the bin's raw hessian is tested, and kEpsilon comes off the other side
        const double raw_hess = bin[1] * ctx.scale.hess;
        const double other_hess = ctx.sum_hess - raw_hess - K_EPSILON;
        Side grow = left;
        grow.hess = raw_hess;
        if (check(ctx, grow, other_count, other_hess) != Check::Evaluate) continue;
        const double grad = left.units[0] * ctx.scale.grad;
        const double gain = split_gain(ctx.sum_grad - grad, grad, other_hess, raw_hess + K_EPSILON, c.lambda_l1,
                                       c.lambda_l2);
        if (std::isnan(gain) || gain <= ctx.min_gain_shift) continue;
        splittable = true;
        if (!have || gain > best.gain) {
            best = Best{gain, static_cast<uint32_t>(t), grad, raw_hess + K_EPSILON, left.count,
                        {left.units[0], left.units[1]}};
            have = true;
        }
    }
    if (have) {
        cand.feature = feature;
        cand.gain = best.gain - ctx.min_gain_shift;
        cand.best = best;
        cand.default_left = false;
        cand.kind = kOneHot;
    }
    return have;
}

// f64::total_cmp's key: the bits with every bit but the sign flipped for negative values, compared as i64.
inline int64_t total_order_key(double v) {
    int64_t bits;
    std::memcpy(&bits, &v, sizeof(bits));
    return bits ^ static_cast<int64_t>(static_cast<uint64_t>(bits >> 63) >> 1);
}

// sorted_categories (split.rs:739-761): the categories (bins 1..) with at least cat_smooth estimated rows, sorted by
// sum_g / (sum_h + cat_smooth) (total order), equal ratios in ascending bin order; returns how many.
size_t sorted_categories(const LeafCtx& ctx, const double* hist, size_t num_bins, uint32_t* order) {
    const sb2_split_config& c = *ctx.cfg;
    const size_t nb = std::min(num_bins, MAX_BINS);
    size_t used = 0;
    for (size_t t = 1; t < nb; ++t)
        if (static_cast<double>(bin_count(ctx, hist[2 * t + 1])) >= c.cat_smooth) order[used++] = static_cast<uint32_t>(t);
    auto ctr = [&](uint32_t t) { return (hist[2 * t] * ctx.scale.grad) / (hist[2 * t + 1] * ctx.scale.hess + c.cat_smooth); };
    std::sort(order, order + used, [&](uint32_t a, uint32_t b) {
        const int64_t ka = total_order_key(ctr(a)), kb = total_order_key(ctr(b));
        return ka != kb ? ka < kb : a < b;
    });
    return used;
}

// SortedScan::run (split.rs:792-845): the best prefix of order(0 .. steps); threshold holds its length minus one.
template <class Order>
bool sorted_scan(const LeafCtx& ctx, const double* hist, double l2, size_t steps, Order order, bool& splittable,
                 Best& best) {
    const sb2_split_config& c = *ctx.cfg;
    Side left;
    int64_t cnt_cur_group = 0;
    bool have = false;
    for (size_t i = 0; i < steps; ++i) {
        const size_t t = order(i);
        const int64_t before = left.count;
        left.add(ctx, hist + 2 * t);
        cnt_cur_group += left.count - before;
        const int64_t right_count = ctx.num_data - left.count;
        const double right_hess = ctx.sum_hess - left.hess;
        const Check k = check(ctx, left, right_count, right_hess);
        if (k == Check::Continue) continue;
        if (k == Check::Break) break;
        if (right_count < c.min_data_per_group) break;
        if (cnt_cur_group < c.min_data_per_group) continue;
        cnt_cur_group = 0;
        const double left_grad = left.units[0] * ctx.scale.grad;
        const double gain = split_gain(left_grad, ctx.sum_grad - left_grad, left.hess, right_hess, c.lambda_l1, l2);
        if (std::isnan(gain) || gain <= ctx.min_gain_shift) continue;
        splittable = true;
        if (!have || gain > best.gain) {
            best = Best{gain, static_cast<uint32_t>(i), left_grad, left.hess, left.count, {left.units[0], left.units[1]}};
            have = true;
        }
    }
    return have;
}

// find_sorted_categorical (split.rs:763-788): prefixes of up to max_cat_threshold categories from either end of the
// sorted order, the low end first; the high end replaces it only when strictly better.
bool find_sorted_categorical(const LeafCtx& ctx, int64_t feature, const double* hist, size_t num_bins,
                             bool& splittable, Candidate& cand) {
    const sb2_split_config& c = *ctx.cfg;
    uint32_t sorted[MAX_BINS];
    const size_t used = sorted_categories(ctx, hist, num_bins, sorted);
    const size_t max_num_cat = std::min<size_t>(static_cast<size_t>(std::max(c.max_cat_threshold, 0)), (used + 1) / 2);
    const double l2 = c.lambda_l2 + c.cat_l2;
    splittable = false;
    bool have = false;
    Best best{};
    bool best_forward = true;
    for (bool forward : {true, false}) {
        Best b{};
        auto order = [&](size_t i) { return static_cast<size_t>(forward ? sorted[i] : sorted[used - 1 - i]); };
        if (sorted_scan(ctx, hist, l2, std::min(used, max_num_cat), order, splittable, b) && (!have || b.gain > best.gain)) {
            best = b;
            best_forward = forward;
            have = true;
        }
    }
    if (have) {
        cand.feature = feature;
        cand.gain = best.gain - ctx.min_gain_shift;
        cand.best = best;
        cand.default_left = false;
        cand.kind = best_forward ? kSortedForward : kSortedReverse;
    }
    return have;
}

// better (split.rs:866-873): higher gain (NaN as kMinScore), then the lower feature.
bool better(const Candidate& a, const Candidate& b) {
    double ga = std::isnan(a.gain) ? MIN_SCORE : a.gain;
    double gb = std::isnan(b.gain) ? MIN_SCORE : b.gain;
    if (ga > gb) return true;
    if (ga < gb) return false;
    return a.feature < b.feature;
}

// finish (split.rs:632-651) through split_info (:654-691): a categorical split's left bins are its one category or
// the first threshold + 1 categories of the sorted order from the chosen end, with the categorical l2.
sb2_split_info finish(const LeafCtx& ctx, const Candidate& c, const double* hist, size_t num_bins) {
    const Best& b = c.best;
    const double l1 = ctx.cfg->lambda_l1;
    const double l2 = c.kind == kSortedForward || c.kind == kSortedReverse ? ctx.cfg->lambda_l2 + ctx.cfg->cat_l2
                                                                          : ctx.cfg->lambda_l2;
    sb2_split_info s{};
    s.found = 1;
    s.feature = static_cast<int32_t>(c.feature);
    s.gain = b.gain - ctx.min_gain_shift;
    s.threshold = c.kind == kNumerical ? b.threshold : 0u;
    s.default_left = c.default_left;
    if (c.kind == kOneHot) {
        s.categorical = 1;
        s.cat_bins[b.threshold / 32] |= 1u << (b.threshold % 32);
    } else if (c.kind != kNumerical) {
        s.categorical = 1;
        uint32_t sorted[MAX_BINS];
        const size_t used = sorted_categories(ctx, hist, num_bins, sorted);
        for (size_t i = 0; i <= b.threshold; ++i) {
            const uint32_t bin = c.kind == kSortedForward ? sorted[i] : sorted[used - 1 - i];
            s.cat_bins[bin / 32] |= 1u << (bin % 32);
        }
    }
    s.left_grad = b.left_units[0];
    s.left_hess = b.left_units[1];
    s.left_count = b.left_count;
    s.right_grad = ctx.units.grad - b.left_units[0];
    s.right_hess = ctx.units.hess - b.left_units[1];
    s.right_count = ctx.num_data - b.left_count;
    s.left_output = leaf_output(b.left_grad, b.left_hess, l1, l2);
    s.right_output = leaf_output(ctx.sum_grad - b.left_grad, ctx.sum_hess - b.left_hess, l1, l2);
    return s;
}

// find_best_split (split.rs:919-961)
bool find_best_split(const sb2_dataset& d, const double* hist, const uint8_t* evaluate, LeafSums sums,
                     HistScale scale, const sb2_split_config* cfg, sb2_split_info& out, uint8_t* splittable) {
    std::memset(splittable, 0, d.num_features);
    out = sb2_split_info{};
    LeafCtx ctx;
    if (!leaf_ctx(cfg, scale, sums, ctx)) return true;
    const int64_t F = d.num_features;
    std::vector<Candidate> per(F);
    std::vector<char> have(F, 0);
    bool bad = false;
    std::atomic<bool> bad_flag{false};
    parallel_tasks(static_cast<size_t>(F), [&](size_t f) {
        const sb2_feature& m = d.features[f];
        if (!evaluate[f] || m.num_bins == 0 || m.kind == SB2_TRIVIAL) return;
        const double* fh = hist + 2 * static_cast<size_t>(m.hist_offset);
        bool sp = false;
        // find_feature (split.rs:848-862)
        if (m.kind == SB2_NUMERICAL)
            have[f] = find_numerical(ctx, f, fh, m.num_bins, m.nan_bin != 0, sp, per[f]);
        else if (m.kind == SB2_CATEGORICAL && static_cast<int64_t>(m.num_bins) <= cfg->max_cat_to_onehot)
            have[f] = find_onehot(ctx, f, fh, m.num_bins, sp, per[f]);
        else if (m.kind == SB2_CATEGORICAL)
            have[f] = find_sorted_categorical(ctx, f, fh, m.num_bins, sp, per[f]);
        else
            bad_flag = true;
        splittable[f] = sp;
    });
    bad = bad_flag;
    if (bad) {
        g_error = "unknown feature kind";
        return false;
    }
    const Candidate* best = nullptr;
    for (int64_t f = 0; f < F; ++f)
        if (have[f] && (!best || better(per[f], *best))) best = &per[f];
    if (best) {
        const sb2_feature& m = d.features[best->feature];
        out = finish(ctx, *best, hist + 2 * static_cast<size_t>(m.hist_offset), m.num_bins);
    }
    return true;
}

// feature_mask (split.rs:966-985)
void feature_mask(const sb2_dataset& d, double fraction, uint32_t seed, uint32_t iteration, uint8_t* mask) {
    std::vector<uint32_t> usable;
    for (uint32_t f = 0; f < d.num_features; ++f) {
        mask[f] = 0;
        if (d.features[f].num_bins != 0) usable.push_back(f);
    }
    if (fraction >= 1.0) {
        for (uint32_t f : usable) mask[f] = 1;
        return;
    }
    size_t count = std::max<size_t>(static_cast<size_t>(round_int(static_cast<double>(usable.size()) * fraction)),
                                    std::min<size_t>(usable.size(), 1));
    std::vector<std::pair<float, uint32_t>> keyed;
    for (uint32_t f : usable) keyed.emplace_back(uniform(seed, STREAM_FEATURE_FRACTION, iteration, f), f);
    std::sort(keyed.begin(), keyed.end(), [](const auto& a, const auto& b) {
        if (a.first != b.first) return a.first < b.first;
        return a.second < b.second;
    });
    for (size_t i = 0; i < std::min(count, keyed.size()); ++i) mask[keyed[i].second] = 1;
}

// ---- tree.rs ----------------------------------------------------------------------------------------------------

constexpr int8_t CATEGORICAL_MASK = 1;                         // tree.rs:10
constexpr int8_t DEFAULT_LEFT_MASK = 2;                        // tree.rs:11
constexpr double ZERO_THRESHOLD = static_cast<double>(1e-35f); // tree.rs:13

inline double nan_to_zero(double v) { return std::isnan(v) ? 0.0 : v; }                 // tree.rs:212-218
inline double round_to_zero(double v) { return std::fabs(v) > ZERO_THRESHOLD ? v : 0.0; }  // tree.rs:221-227

struct Tree {
    int32_t num_leaves = 1;
    std::vector<int32_t> split_feature;
    std::vector<float> split_gain;
    std::vector<double> threshold;
    std::vector<uint32_t> threshold_bin;
    std::vector<int8_t> decision_type;
    std::vector<int32_t> left_child, right_child;
    std::vector<double> leaf_value{0.0}, leaf_weight{0.0};
    std::vector<int64_t> leaf_count{0};
    std::vector<double> internal_value, internal_weight;
    std::vector<int64_t> internal_count;
    std::vector<uint32_t> cat_bins;  // 8 words per split: the bins a categorical split sends left (0: numerical)
    int32_t num_cat = 0;
    double shrinkage = 1.0;
    std::vector<int32_t> leaf_parent{-1}, leaf_depth{0};

    struct Children {
        double left_value, right_value;
        int64_t left_count, right_count;
        double left_weight, right_weight;
        float gain;
    };

    // Tree::split (tree.rs:143-177) through split_numerical (:108-122)
    int32_t split_numerical(int32_t leaf, int32_t feature, double thr, uint32_t thr_bin, bool default_left,
                            bool nan_missing, const Children& c) {
        int8_t dt = static_cast<int8_t>((nan_missing ? 2 : 0) << 2);
        if (default_left) dt |= DEFAULT_LEFT_MASK;
        const uint32_t none[8] = {};
        return split(leaf, feature, thr, thr_bin, dt, none, c);
    }
    // Tree::split_categorical (tree.rs:125-141): the threshold is the split's index among the tree's categorical
    // splits, MissingType::NaN; the category bitset (cat_threshold) is built from the left bins' category values
    // when the model is written, so the tree keeps the bins.
    int32_t split_categorical(int32_t leaf, int32_t feature, const uint32_t* left_bins, const Children& c) {
        const double index = static_cast<double>(num_cat++);
        return split(leaf, feature, index, 0u, static_cast<int8_t>(CATEGORICAL_MASK | (2 << 2)), left_bins, c);
    }
    int32_t split(int32_t leaf, int32_t feature, double thr, uint32_t thr_bin, int8_t dt, const uint32_t* bins,
                  const Children& c) {
        cat_bins.insert(cat_bins.end(), bins, bins + 8);
        int32_t node = num_leaves - 1, new_leaf = num_leaves;
        int32_t parent = leaf_parent[leaf];
        if (parent >= 0) {
            if (left_child[parent] == ~leaf)
                left_child[parent] = node;
            else
                right_child[parent] = node;
        }
        split_feature.push_back(feature);
        split_gain.push_back(c.gain);
        threshold.push_back(thr);
        threshold_bin.push_back(thr_bin);
        decision_type.push_back(dt);
        left_child.push_back(~leaf);
        right_child.push_back(~new_leaf);
        internal_weight.push_back(leaf_weight[leaf]);
        internal_value.push_back(leaf_value[leaf]);
        internal_count.push_back(c.left_count + c.right_count);
        leaf_value[leaf] = nan_to_zero(c.left_value);
        leaf_weight[leaf] = c.left_weight;
        leaf_count[leaf] = c.left_count;
        leaf_value.push_back(nan_to_zero(c.right_value));
        leaf_weight.push_back(c.right_weight);
        leaf_count.push_back(c.right_count);
        leaf_parent[leaf] = node;
        leaf_parent.push_back(node);
        int32_t depth = leaf_depth[leaf] + 1;
        leaf_depth[leaf] = depth;
        leaf_depth.push_back(depth);
        ++num_leaves;
        return new_leaf;
    }
    void shrink(double rate) {  // tree.rs:180-185
        for (double& v : leaf_value) v = round_to_zero(v * rate);
        for (double& v : internal_value) v = round_to_zero(v * rate);
        shrinkage *= rate;
    }
    void add_bias(double bias) {  // tree.rs:188-193
        for (double& v : leaf_value) v = round_to_zero(v + bias);
        for (double& v : internal_value) v = round_to_zero(v + bias);
        shrinkage = 1.0;
    }
    void as_constant(double value) {  // tree.rs:196-199
        *this = Tree();
        leaf_value[0] = value;
    }
};

// ---- backends: CpuBackend state per rank -------------------------------------------------------------------------

struct Rank {
    const sb2_dataset* data;
    std::vector<GroupLayout> layout;
    std::vector<float> scores, grad, hess;
    std::vector<int32_t> packed;
    std::vector<uint32_t> partition;
    int64_t max_quant = 1;
};

// The ranks of one training run; every collective is an exact sum (or max) over ranks in rank order, as
// ThreadCollective (crates/silvic-core/src/test_util.rs:13-90) does in the reference's tests.
struct World {
    std::vector<Rank> ranks;
    size_t total_bins;
};

struct LeafRangeR {
    uint32_t begin, count;
};

struct Leaf {
    std::vector<LeafRangeR> range;  // per rank
    LeafSums sums;
    std::vector<double> hist;  // empty: none
    std::vector<uint8_t> splittable;
    bool has_best = false;
    sb2_split_info best{};
};

struct ModelOut {
    std::vector<Tree> trees;
    double init_score = 0.0;
    std::vector<double> seconds;
    std::vector<double> op_seconds;  // per operation (OpTimer's order), summed over the run
};

// The per-operation split of the reference's `Timed` test backend (tests/train_cpu.rs:434-484): wall seconds spent in
// gradients, quantize, histogram, split search, partition, leaf sums and add_tree, summed over a training run.
enum { kOpGradients, kOpQuantize, kOpHistogram, kOpSearch, kOpPartition, kOpLeafSums, kOpAddTree, kOps };
double g_op_seconds[kOps];

struct OpTimer {
    int op;
    std::chrono::steady_clock::time_point t0 = std::chrono::steady_clock::now();
    explicit OpTimer(int o) : op(o) {}
    ~OpTimer() {
        g_op_seconds[op] += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    }
};

struct Learner {
    const sb2_params& p;
    World& w;
    const sb2_dataset& d0;
    sb2_split_config cfg;
    int64_t sums_feature = -1;

    Learner(const sb2_params& params, World& world) : p(params), w(world), d0(*world.ranks[0].data) {
        cfg.min_data_in_leaf = p.min_data_in_leaf;
        cfg.min_sum_hessian_in_leaf = p.min_sum_hessian_in_leaf;
        cfg.lambda_l1 = p.lambda_l1;
        cfg.lambda_l2 = p.lambda_l2;
        cfg.min_gain_to_split = p.min_gain_to_split;
        cfg.min_data_per_group = p.min_data_per_group;  // SplitConfig::new (split.rs:64-77)
        cfg.cat_l2 = p.cat_l2;
        cfg.cat_smooth = p.cat_smooth;
        cfg.max_cat_to_onehot = p.max_cat_to_onehot;
        cfg.max_cat_threshold = p.max_cat_threshold;
        for (uint32_t f = 0; f < d0.num_features; ++f)
            if (d0.features[f].num_bins != 0) {
                sums_feature = f;
                break;
            }
    }

    bool may_split(int32_t depth, int64_t left, int64_t right) const {  // learner.rs:172-175
        int64_t min_pair = 2 * cfg.min_data_in_leaf;
        return depth_allows(depth) && (left >= min_pair || right >= min_pair);
    }
    bool depth_allows(int32_t depth) const { return p.max_depth <= 0 || depth < p.max_depth; }  // :178-180

    void set_features(const uint8_t* used) {
        for (Rank& r : w.ranks)
            for (GroupLayout& l : r.layout) l.activate(used, d0.num_features);
    }

    // Learner::histogram (learner.rs:189-201): per-rank histograms summed.
    std::vector<double> histogram(const std::vector<LeafRangeR>& ranges) {
        std::vector<double> total(2 * w.total_bins, 0.0), part(2 * w.total_bins);
        for (size_t r = 0; r < w.ranks.size(); ++r) {
            Rank& rk = w.ranks[r];
            OpTimer timer(kOpHistogram);
            histogram_quantized(*rk.data, rk.layout, rk.packed.data(), rk.max_quant,
                                rk.partition.data() + ranges[r].begin, ranges[r].count, part.data());
            for (size_t i = 0; i < total.size(); ++i) total[i] += part[i];
        }
        return total;
    }

    void find_split(Leaf& leaf, std::vector<double> hist, const std::vector<uint8_t>& evaluate, HistScale scale) {
        leaf.splittable.assign(d0.num_features, 0);
        sb2_split_info info;
        OpTimer timer(kOpSearch);
        if (!find_best_split(d0, hist.data(), evaluate.data(), leaf.sums, scale, &cfg, info, leaf.splittable.data()))
            throw std::runtime_error(g_error);
        leaf.has_best = info.found != 0;
        leaf.best = info;
        leaf.hist = std::move(hist);
    }

    static sb2_bin_split bin_split(const sb2_feature& m, const sb2_split_info& info) {  // learner.rs:432-452
        sb2_bin_split s{};
        s.group = m.group;
        s.column = m.column;
        if (info.categorical) {
            std::memcpy(s.left_bins, info.cat_bins, sizeof(s.left_bins));
            return s;
        }
        for (uint32_t b = 0; b <= info.threshold; ++b) s.left_bins[b / 32] |= 1u << (b % 32);
        if (info.default_left && m.kind == SB2_NUMERICAL && m.nan_bin) {
            uint32_t b = m.num_bins - 1;
            s.left_bins[b / 32] |= 1u << (b % 32);
        }
        return s;
    }

    // Learner::grow (learner.rs:121-169)
    Tree grow(const std::vector<uint8_t>& mask, HistScale scale, const std::vector<uint32_t>& local_rows,
              int64_t root_count, std::vector<std::vector<LeafRangeR>>& leaves_out) {
        Tree tree;
        std::vector<Leaf> leaves(1);
        leaves[0].range.resize(w.ranks.size());
        for (size_t r = 0; r < w.ranks.size(); ++r) leaves[0].range[r] = {0, local_rows[r]};
        leaves[0].sums.count = root_count;
        leaves[0].splittable.assign(d0.num_features, 1);
        if (sums_feature >= 0 && may_split(0, root_count, 0)) {
            std::vector<uint8_t> root_features = mask;
            root_features[sums_feature] = 1;
            set_features(root_features.data());
            std::vector<double> hist = histogram(leaves[0].range);
            const sb2_feature& m = d0.features[sums_feature];
            double g = 0.0, h = 0.0;  // LeafSums::from_feature_hist (split.rs:101-108)
            for (uint32_t b = 0; b < m.num_bins; ++b) {
                g += hist[2 * (m.hist_offset + b)];
                h += hist[2 * (m.hist_offset + b) + 1];
            }
            leaves[0].sums.grad = g;
            leaves[0].sums.hess = h;
            find_split(leaves[0], std::move(hist), mask, scale);
        }
        while (tree.num_leaves < p.num_leaves) {
            // best_leaf (learner.rs:418-429)
            int64_t best = -1;
            double best_gain = 0.0;
            for (size_t i = 0; i < leaves.size(); ++i) {
                if (!leaves[i].has_best) continue;
                if (best < 0 || leaves[i].best.gain > best_gain) {
                    best = static_cast<int64_t>(i);
                    best_gain = leaves[i].best.gain;
                }
            }
            if (best < 0 || !(best_gain > 0.0)) break;
            split_leaf(tree, leaves, static_cast<size_t>(best), mask, scale);
        }
        leaves_out.clear();
        for (Leaf& l : leaves) leaves_out.push_back(l.range);
        return tree;
    }

    // Learner::split_leaf (learner.rs:249-352)
    void split_leaf(Tree& tree, std::vector<Leaf>& leaves, size_t index, const std::vector<uint8_t>& mask,
                    HistScale scale) {
        sb2_split_info info = leaves[index].best;
        leaves[index].has_best = false;
        const sb2_feature& meta = d0.features[info.feature];
        sb2_bin_split split = bin_split(meta, info);
        std::vector<LeafRangeR> parent_range = leaves[index].range;
        int64_t parent_count = leaves[index].sums.count;
        bool may_search = !leaves[index].hist.empty() && tree.num_leaves + 1 < p.num_leaves &&
                          depth_allows(tree.leaf_depth[index] + 1);
        bool built_left = info.left_count <= info.right_count;
        std::vector<uint8_t> evaluate(d0.num_features);
        for (uint32_t f = 0; f < d0.num_features; ++f) evaluate[f] = mask[f] && leaves[index].splittable[f];
        std::vector<uint32_t> left_local(w.ranks.size());
        int64_t left_count = 0;
        for (size_t r = 0; r < w.ranks.size(); ++r) {
            Rank& rk = w.ranks[r];
            OpTimer timer(kOpPartition);
            left_local[r] = stable_partition(*rk.data, split, rk.partition.data() + parent_range[r].begin,
                                             parent_range[r].count);
            left_count += left_local[r];
        }
        std::vector<double> built_hist;
        if (may_search) {
            set_features(evaluate.data());
            std::vector<LeafRangeR> child(w.ranks.size());
            for (size_t r = 0; r < w.ranks.size(); ++r)
                child[r] = built_left ? LeafRangeR{parent_range[r].begin, left_local[r]}
                                      : LeafRangeR{parent_range[r].begin + left_local[r],
                                                   parent_range[r].count - left_local[r]};
            built_hist = histogram(child);
        }
        int64_t right_count = parent_count - left_count;
        if (left_count <= 0 || right_count <= 0) throw std::runtime_error("split sends no rows to a side");
        Tree::Children c;
        c.left_value = info.left_output;
        c.right_value = info.right_output;
        c.left_count = left_count;
        c.right_count = right_count;
        c.left_weight = info.left_hess * scale.hess;
        c.right_weight = info.right_hess * scale.hess;
        c.gain = static_cast<float>(info.gain + cfg.min_gain_to_split);
        // apply_split (learner.rs:459-485): the threshold is the bin's upper bound, f64::MAX for +inf; a categorical
        // split keeps its left bins.
        int32_t right_index;
        if (info.categorical) {
            right_index = tree.split_categorical(static_cast<int32_t>(index), info.feature, info.cat_bins, c);
        } else {
            double bound = meta.upper_bounds[info.threshold];
            double thr = std::isfinite(bound) ? bound : std::numeric_limits<double>::max();
            right_index = tree.split_numerical(static_cast<int32_t>(index), info.feature, thr, info.threshold,
                                               info.default_left != 0, meta.nan_bin != 0, c);
        }
        if (static_cast<size_t>(right_index) != leaves.size()) throw std::runtime_error("leaf numbering");
        std::vector<double> parent_hist = std::move(leaves[index].hist);
        Leaf left, right;
        left.range.resize(w.ranks.size());
        right.range.resize(w.ranks.size());
        for (size_t r = 0; r < w.ranks.size(); ++r) {
            left.range[r] = {parent_range[r].begin, left_local[r]};
            right.range[r] = {parent_range[r].begin + left_local[r], parent_range[r].count - left_local[r]};
        }
        left.sums = {info.left_grad, info.left_hess, left_count};
        right.sums = {info.right_grad, info.right_hess, right_count};
        leaves[index] = std::move(left);
        leaves.push_back(std::move(right));
        int32_t depth = tree.leaf_depth[index];
        bool searched = may_split(depth, left_count, right_count);
        if (!parent_hist.empty() && !built_hist.empty() && searched) {
            // search_children (learner.rs:356-371)
            size_t built = built_left ? index : static_cast<size_t>(right_index);
            size_t other = built_left ? static_cast<size_t>(right_index) : index;
            for (size_t i = 0; i < parent_hist.size(); ++i) parent_hist[i] -= built_hist[i];
            find_split(leaves[built], std::move(built_hist), evaluate, scale);
            find_split(leaves[other], std::move(parent_hist), evaluate, scale);
        }
    }

    // Learner::renew_leaves (learner.rs:376-404)
    void renew_leaves(Tree& tree, const std::vector<std::vector<LeafRangeR>>& leaves, double max_abs_grad,
                      double max_hess) {
        float gs = fixed_point_scale(max_abs_grad), hs = fixed_point_scale(max_hess);
        std::vector<int64_t> flat(2 * leaves.size(), 0);
        for (size_t r = 0; r < w.ranks.size(); ++r) {
            const Rank& rk = w.ranks[r];
            std::vector<sb2_leaf_range> lr(leaves.size());
            for (size_t i = 0; i < leaves.size(); ++i) lr[i] = {leaves[i][r].begin, leaves[i][r].count};
            std::vector<int64_t> part(2 * leaves.size());
            OpTimer timer(kOpLeafSums);
            orc_leaf_sums(rk.grad.data(), rk.hess.data(), rk.partition.data(), lr.data(), lr.size(), gs, hs,
                          part.data());
            for (size_t i = 0; i < flat.size(); ++i) flat[i] += part[i];
        }
        for (size_t leaf = 0; leaf < leaves.size(); ++leaf) {
            double sg = static_cast<double>(flat[2 * leaf]) / static_cast<double>(gs);
            double sh = static_cast<double>(flat[2 * leaf + 1]) / static_cast<double>(hs);
            double output = leaf_output(sg, sh, cfg.lambda_l1, cfg.lambda_l2);
            tree.leaf_value[leaf] = round_to_zero(output);  // Tree::set_leaf_output (tree.rs:202-204)
            tree.leaf_weight[leaf] = sh;
        }
    }
};

// The device form of a grown tree (GrownTree::device_tree, learner.rs:66-84).
void device_nodes(const Tree& t, const std::vector<sb2_bin_split>& splits, std::vector<sb2_device_node>& nodes) {
    nodes.clear();
    for (size_t k = 0; k < splits.size(); ++k) nodes.push_back({splits[k], t.left_child[k], t.right_child[k]});
}

// boosting::train_from / Trainer::train_one_iter (boosting.rs:83-149,227-324) without validation sets.
ModelOut train(const sb2_dataset* shards, int num_shards, const sb2_params& p) {
    World w;
    w.total_bins = shards[0].total_bins;
    for (int r = 0; r < num_shards; ++r) {
        Rank rk;
        rk.data = &shards[r];
        if (!group_layouts(shards[r], rk.layout)) throw std::runtime_error(g_error);
        size_t n = shards[r].num_rows;
        rk.scores.assign(n, 0.0f);
        rk.grad.assign(n, 0.0f);
        rk.hess.assign(n, 0.0f);
        rk.packed.assign(n, 0);
        rk.partition.reserve(n);
        w.ranks.push_back(std::move(rk));
    }
    sb2_objective obj{};
    obj.kind = p.objective;
    obj.sigmoid = p.sigmoid;
    std::vector<LambdaRank> ranking(p.objective == SB2_LAMBDARANK ? num_shards : 0);
    for (size_t r = 0; r < ranking.size(); ++r)
        if (!lambdarank_setup(p, shards[r], ranking[r])) throw std::runtime_error(g_error);
    // init_score: per-rank label sums, allreduced in rank order.
    double sums[2] = {0.0, 0.0};
    for (int r = 0; r < num_shards; ++r) {
        double s[2];
        label_sums(p.objective, shards[r].label, shards[r].weight, shards[r].num_rows, s);
        sums[0] += s[0];
        sums[1] += s[1];
    }
    double init_score = init_score_from_sums(p, sums);
    for (Rank& rk : w.ranks) std::fill(rk.scores.begin(), rk.scores.end(), static_cast<float>(init_score));
    bool constant_hessian = p.objective == SB2_REGRESSION && shards[0].weight == nullptr;  // objective/mod.rs:84-89
    Learner learner(p, w);
    ModelOut out;
    out.init_score = init_score;
    std::fill(g_op_seconds, g_op_seconds + kOps, 0.0);
    const sb2_dataset& d0 = shards[0];
    for (int iteration = 0; iteration < p.num_iterations; ++iteration) {
        auto t0 = std::chrono::steady_clock::now();
        double maxima[2] = {0.0, 0.0};
        for (Rank& rk : w.ranks) {
            size_t n = rk.data->num_rows;
            OpTimer timer(kOpGradients);
            if (p.objective == SB2_LAMBDARANK)
                lambdarank_gradients(ranking[&rk - w.ranks.data()], *rk.data, rk.scores.data(), rk.grad.data(),
                                     rk.hess.data());
            else
                gradients(obj, rk.scores.data(), rk.data->label, rk.data->weight, n, rk.grad.data(), rk.hess.data());
            using Pair = std::pair<double, double>;
            auto [mg, mh] = parallel_reduce(
                n, Pair{0.0, 0.0},
                [&](size_t i, Pair& m) {
                    m.first = std::fmax(m.first, static_cast<double>(std::fabs(rk.grad[i])));
                    m.second = std::fmax(m.second, static_cast<double>(std::fabs(rk.hess[i])));
                },
                [](Pair a, Pair b) { return Pair{std::fmax(a.first, b.first), std::fmax(a.second, b.second)}; });
            maxima[0] = std::fmax(maxima[0], mg);
            maxima[1] = std::fmax(maxima[1], mh);
        }
        HistScale scale{1.0, 1.0};
        if (!p.use_quantized_grad) throw std::runtime_error("float histograms are not restated");
        sb2_quant_spec spec = quant_spec(maxima[0], maxima[1], constant_hessian, 1.0,
                                         static_cast<uint32_t>(p.num_grad_quant_bins), p.stochastic_rounding != 0,
                                         p.data_random_seed, static_cast<uint32_t>(iteration));
        for (Rank& rk : w.ranks) {
            size_t n = rk.data->num_rows;
            uint64_t off = rk.data->row_offset;
            OpTimer timer(kOpQuantize);
            parallel_for(n, [&](size_t i) { rk.packed[i] = quantize_row(spec, rk.grad[i], rk.hess[i], off + i); });
            rk.max_quant = std::max(spec.grad_max_q, spec.hess_max_q);
        }
        scale = {spec.grad_scale, spec.hess_scale};
        // bag (boosting.rs:288-299) and reset_partition (backend/cpu.rs:802-830)
        sb2_bag_spec bag{0, 0, 0, 0, 1.0};
        if (p.bagging_fraction < 1.0 && p.bagging_freq > 0)
            bag = {1, p.bagging_seed, static_cast<uint32_t>(iteration / p.bagging_freq), 0, p.bagging_fraction};
        std::vector<uint32_t> local_rows(w.ranks.size());
        int64_t root_count = 0;
        for (size_t r = 0; r < w.ranks.size(); ++r) {
            Rank& rk = w.ranks[r];
            rk.partition.resize(rk.data->num_rows);
            local_rows[r] = orc_reset_partition(&bag, rk.data->num_rows, rk.data->row_offset, rk.partition.data());
            rk.partition.resize(local_rows[r]);
            root_count += local_rows[r];
        }
        std::vector<uint8_t> mask(d0.num_features);
        feature_mask(d0, p.feature_fraction, p.feature_fraction_seed, static_cast<uint32_t>(iteration), mask.data());
        std::vector<std::vector<LeafRangeR>> leaf_ranges;
        Tree tree = learner.grow(mask, scale, local_rows, root_count, leaf_ranges);
        if (tree.num_leaves == 1) {
            // Trainer::single_leaf (boosting.rs:303-310)
            if (out.trees.empty()) {
                Tree t;
                t.as_constant(init_score);
                out.trees.push_back(t);
            }
            out.seconds.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
            break;
        }
        if (p.quant_train_renew_leaf) learner.renew_leaves(tree, leaf_ranges, maxima[0], maxima[1]);
        // Trainer::add (boosting.rs:313-324)
        tree.shrink(p.learning_rate);
        std::vector<float> leaf_values(tree.num_leaves);
        for (int32_t l = 0; l < tree.num_leaves; ++l) leaf_values[l] = static_cast<float>(tree.leaf_value[l]);
        if (out.trees.empty() && init_score != 0.0) {
            tree.add_bias(init_score);
            for (int32_t l = 0; l < tree.num_leaves; ++l)
                leaf_values[l] = static_cast<float>(tree.leaf_value[l] - init_score);  // replay::leaf_values
        }
        std::vector<sb2_bin_split> splits;
        for (int32_t k = 0; k + 1 < tree.num_leaves; ++k) {
            sb2_split_info info{};
            info.threshold = tree.threshold_bin[k];
            info.default_left = (tree.decision_type[k] & DEFAULT_LEFT_MASK) != 0;
            info.categorical = (tree.decision_type[k] & CATEGORICAL_MASK) != 0;
            std::memcpy(info.cat_bins, tree.cat_bins.data() + 8 * static_cast<size_t>(k), sizeof(info.cat_bins));
            splits.push_back(Learner::bin_split(d0.features[tree.split_feature[k]], info));
        }
        std::vector<sb2_device_node> nodes;
        device_nodes(tree, splits, nodes);
        for (Rank& rk : w.ranks) {
            OpTimer timer(kOpAddTree);
            if (!add_tree(*rk.data, nodes.data(), nodes.size(), leaf_values.data(), leaf_values.size(),
                          rk.scores.data()))
                throw std::runtime_error(g_error);
        }
        out.trees.push_back(std::move(tree));
        out.seconds.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
    }
    out.op_seconds.assign(g_op_seconds, g_op_seconds + kOps);
    return out;
}

}  // namespace

struct orc_model {
    ModelOut m;
};

extern "C" {

int orc_num_threads(void) { return g_threads; }
void orc_set_num_threads(int threads) { g_threads = std::max(1, threads); }
const char* orc_last_error(void) { return g_error.c_str(); }

uint32_t orc_mix32(uint32_t x) { return mix32(x); }
float orc_uniform(uint32_t seed, uint32_t stream, uint32_t iteration, uint64_t row) {
    return uniform(seed, stream, iteration, row);
}
void orc_quant_spec(double max_abs_grad, double max_hess, int has_constant_hessian, double constant_hessian,
                    uint32_t num_bins, int stochastic, uint32_t seed, uint32_t iteration, sb2_quant_spec* out) {
    *out = quant_spec(max_abs_grad, max_hess, has_constant_hessian != 0, constant_hessian, num_bins,
                      stochastic != 0, seed, iteration);
}
void orc_quantize(const sb2_quant_spec* spec, const float* grad, const float* hess, size_t n, uint64_t row_offset,
                  int32_t* out) {
    parallel_for(n, [&](size_t i) { out[i] = quantize_row(*spec, grad[i], hess[i], row_offset + i); });
}
void orc_unpack(int32_t packed, int32_t* g, int32_t* h) { unpack(packed, *g, *h); }
int orc_in_bag(uint32_t seed, uint32_t round, uint64_t row, double fraction) {
    return in_bag(seed, round, row, fraction);
}
float orc_fixed_point_scale(double max_abs) { return fixed_point_scale(max_abs); }
int64_t orc_to_fixed(float value, float scale) { return to_fixed(value, scale); }

void orc_gradients(const sb2_objective* objective, const float* scores, const float* label, const float* weight,
                   size_t n, float* grad, float* hess) {
    gradients(*objective, scores, label, weight, n, grad, hess);
}
double orc_init_score(const sb2_params* params, const float* label, const float* weight, size_t n) {
    double s[2];
    label_sums(params->objective, label, weight, n, s);
    return init_score_from_sums(*params, s);
}

int orc_histogram(const sb2_dataset* data, const int32_t* packed, int32_t max_quant, const uint32_t* rows, size_t n,
                  const uint8_t* used, double* out) {
    std::vector<GroupLayout> layout;
    if (!group_layouts(*data, layout)) return SB2_EDATA;
    for (GroupLayout& l : layout) l.activate(used, data->num_features);
    histogram_quantized(*data, layout, packed, max_quant, rows, n, out);
    return SB2_OK;
}
uint32_t orc_partition(const sb2_dataset* data, const sb2_bin_split* split, uint32_t* rows, size_t n) {
    return stable_partition(*data, *split, rows, n);
}
// CpuBackend::leaf_sums (backend/cpu.rs:886-908)
void orc_leaf_sums(const float* grad, const float* hess, const uint32_t* partition, const sb2_leaf_range* leaves,
                   size_t num_leaves, float grad_scale, float hess_scale, int64_t* out) {
    for (size_t l = 0; l < num_leaves; ++l) {
        const uint32_t* rows = partition + leaves[l].begin;
        size_t cnt = leaves[l].count;
        using Pair = std::pair<int64_t, int64_t>;
        Pair s = parallel_reduce(
            cnt, Pair{0, 0},
            [&](size_t i, Pair& p) {
                p.first += to_fixed(grad[rows[i]], grad_scale);
                p.second += to_fixed(hess[rows[i]], hess_scale);
            },
            [](Pair a, Pair b) { return Pair{a.first + b.first, a.second + b.second}; });
        out[2 * l] = s.first;
        out[2 * l + 1] = s.second;
    }
}
int orc_add_tree(const sb2_dataset* data, const sb2_device_node* nodes, size_t num_nodes, const float* leaf_values,
                 size_t num_leaves, float* scores) {
    return add_tree(*data, nodes, num_nodes, leaf_values, num_leaves, scores) ? SB2_OK : SB2_EDEVICE;
}
// BinMapper::value_to_bin for a numerical mapper (data/bin_mapper.rs:343-360): the number of upper bounds below
// the value (`partition_point(bound < value)`); NaN goes to the NaN bin, or to 0.0's bin without one.
uint32_t orc_value_to_bin(const double* ub, uint32_t n, int nan_bin, double value) {
    if (value != value) {
        if (nan_bin) return n;
        value = 0.0;
    }
    uint32_t k = 0;
    while (k < n && ub[k] < value) ++k;
    return k;
}

namespace {

// data/binning.rs:51-61: the branch-free search over the bounds padded to 256 with +inf.
uint8_t padded_numerical_bin(const double (&bounds)[256], uint8_t nan, double value) {
    if (value != value) return nan;
    size_t pos = 0;
    for (size_t step : {128, 64, 32, 16, 8, 4, 2, 1}) pos += step * static_cast<size_t>(bounds[(pos + step - 1) & 255] < value);
    return static_cast<uint8_t>(pos);
}

// categorical_bin (data/bin_mapper.rs:379-391): the value truncates to i32 (Rust's saturating `as`); NaN, negative
// and unlisted values are bin 0, category categories[i] is bin i + 1.
uint8_t categorical_bin(const int32_t* categories, uint32_t n, double value) {
    if (value != value) return 0;
    const int32_t category = value >= 2147483647.0    ? 2147483647
                             : value <= -2147483648.0 ? static_cast<int32_t>(-2147483647 - 1)
                                                      : static_cast<int32_t>(value);
    if (category < 0) return 0;
    for (uint32_t i = 0; i < n; ++i)
        if (categories[i] == category) return static_cast<uint8_t>(i + 1);
    return 0;
}

}  // namespace

// data/binning.rs:71-135 (bin_rows / bin_column / fill), one row chunk after another.
int orc_bin_rows(const void* values, int value_bytes, uint64_t rows, uint32_t cols, int row_major,
                 const sb2_feature* features, uint32_t num_features, const sb2_group* groups, uint32_t num_groups,
                 uint8_t* const* group_data) {
    if (value_bytes != 4 && value_bytes != 8) return SB2_EDATA;
    for (uint32_t g = 0; g < num_groups; ++g) {
        const sb2_group& grp = groups[g];
        std::memset(group_data[g], 0, rows * grp.row_stride);
        for (uint32_t k = 0; k < grp.num_features; ++k) {
            const uint32_t f = grp.features[k];
            if (f >= num_features || f >= cols) return SB2_EDATA;
            const sb2_feature& m = features[f];
            if (m.kind == SB2_CATEGORICAL) {
                if (!m.categories || m.num_categories == 0 || m.num_categories > 255) return SB2_EDATA;
                for (uint64_t r = 0; r < rows; ++r) {
                    const uint64_t at = row_major ? r * cols + f : static_cast<uint64_t>(f) * rows + r;
                    const double v = value_bytes == 8 ? static_cast<const double*>(values)[at]
                                                      : static_cast<double>(static_cast<const float*>(values)[at]);
                    group_data[g][r * grp.row_stride + m.column] = categorical_bin(m.categories, m.num_categories, v);
                }
                continue;
            }
            if (m.kind != SB2_NUMERICAL) return SB2_EUNSUPPORTED;
            if (m.num_upper_bounds == 0 || m.num_upper_bounds > 256) return SB2_EDATA;
            double bounds[256];
            for (size_t i = 0; i < 256; ++i)
                bounds[i] = i < m.num_upper_bounds ? m.upper_bounds[i] : std::numeric_limits<double>::infinity();
            const uint8_t nan = static_cast<uint8_t>(orc_value_to_bin(m.upper_bounds, m.num_upper_bounds, m.nan_bin,
                                                                      std::numeric_limits<double>::quiet_NaN()));
            for (uint64_t r = 0; r < rows; ++r) {
                const uint64_t at = row_major ? r * cols + f : static_cast<uint64_t>(f) * rows + r;
                const double v = value_bytes == 8 ? static_cast<const double*>(values)[at]
                                                  : static_cast<double>(static_cast<const float*>(values)[at]);
                group_data[g][r * grp.row_stride + m.column] = padded_numerical_bin(bounds, nan, v);
            }
        }
    }
    return SB2_OK;
}

uint32_t orc_reset_partition(const sb2_bag_spec* bag, uint64_t num_rows, uint64_t row_offset, uint32_t* out) {
    uint32_t k = 0;
    for (uint64_t r = 0; r < num_rows; ++r)
        if (bag->kind == 0 || in_bag(bag->seed, bag->round, row_offset + r, bag->fraction))
            out[k++] = static_cast<uint32_t>(r);
    return k;
}

int orc_find_best_split(const sb2_dataset* data, const double* hist, const uint8_t* evaluate, double sum_grad,
                        double sum_hess, int64_t count, double grad_scale, double hess_scale,
                        const sb2_split_config* cfg, sb2_split_info* out, uint8_t* splittable) {
    LeafSums sums{sum_grad, sum_hess, count};
    return find_best_split(*data, hist, evaluate, sums, HistScale{grad_scale, hess_scale}, cfg, *out, splittable)
               ? SB2_OK
               : SB2_EUNSUPPORTED;
}
void orc_feature_mask(const sb2_dataset* data, double fraction, uint32_t seed, uint32_t iteration, uint8_t* out) {
    feature_mask(*data, fraction, seed, iteration, out);
}

int orc_train(const sb2_dataset* shards, int num_shards, const sb2_params* params, orc_model** out) {
    try {
        auto* m = new orc_model;
        m->m = train(shards, num_shards, *params);
        *out = m;
        return SB2_OK;
    } catch (const std::exception& e) {
        g_error = e.what();
        return SB2_EINTERNAL;
    }
}
void orc_model_free(orc_model* m) { delete m; }
int orc_model_num_trees(const orc_model* m) { return static_cast<int>(m->m.trees.size()); }
int orc_model_tree(const orc_model* m, int index, sb2_tree_view* v) {
    if (index < 0 || static_cast<size_t>(index) >= m->m.trees.size()) return SB2_EDEVICE;
    const Tree& t = m->m.trees[index];
    v->num_leaves = t.num_leaves;
    v->shrinkage = t.shrinkage;
    v->split_feature = t.split_feature.data();
    v->split_gain = t.split_gain.data();
    v->threshold = t.threshold.data();
    v->threshold_bin = t.threshold_bin.data();
    v->decision_type = t.decision_type.data();
    v->left_child = t.left_child.data();
    v->right_child = t.right_child.data();
    v->leaf_value = t.leaf_value.data();
    v->leaf_weight = t.leaf_weight.data();
    v->leaf_count = t.leaf_count.data();
    v->internal_value = t.internal_value.data();
    v->internal_weight = t.internal_weight.data();
    v->internal_count = t.internal_count.data();
    v->cat_bins = t.cat_bins.data();
    return SB2_OK;
}
double orc_model_init_score(const orc_model* m) { return m->m.init_score; }
int orc_model_iteration_seconds(const orc_model* m, double* out, size_t len) {
    size_t k = std::min(len, m->m.seconds.size());
    std::copy(m->m.seconds.begin(), m->m.seconds.begin() + k, out);
    return static_cast<int>(m->m.seconds.size());
}
int orc_lambdarank_gradients(const sb2_params* params, const sb2_dataset* data, const float* scores, float* grad,
                             float* hess) {
    LambdaRank lr;
    if (!lambdarank_setup(*params, *data, lr)) return SB2_EDATA;
    lambdarank_gradients(lr, *data, scores, grad, hess);
    return SB2_OK;
}
double orc_lambdarank_max_dcg(size_t k, const float* labels, size_t n, const double* gain, size_t num_gain) {
    return max_dcg_at_k(k, labels, n, std::vector<double>(gain, gain + num_gain));
}
double orc_lambdarank_sigmoid(double sigmoid, double delta) {
    sb2_params p{};
    p.sigmoid = sigmoid;
    const uint32_t qb[2] = {0, 1};
    const float label = 0.0f;
    sb2_dataset d{};
    d.num_rows = 1;
    d.num_queries = 1;
    d.query_boundaries = qb;
    d.label = &label;
    LambdaRank lr;
    if (!lambdarank_setup(p, d, lr)) return std::numeric_limits<double>::quiet_NaN();
    return sigmoid_at(lr, delta);
}

int orc_model_op_seconds(const orc_model* m, double* out, size_t len) {
    const size_t k = std::min(len, m->m.op_seconds.size());
    std::copy(m->m.op_seconds.begin(), m->m.op_seconds.begin() + k, out);
    return static_cast<int>(m->m.op_seconds.size());
}

// Model::predict_raw_row (model/predict.rs:19-23) with numerical_decision (:118-141).
double orc_model_predict_raw(const orc_model* m, const sb2_dataset* data, const double* row) {
    (void)data;
    double score = 0.0;
    for (const Tree& t : m->m.trees) {
        int32_t leaf = 0;
        if (t.num_leaves > 1) {
            int32_t node = 0;
            while (node >= 0) {
                double value = row[t.split_feature[node]];
                if (std::fabs(value) <= ZERO_THRESHOLD) value = 0.0;  // read_value (predict.rs:112-116)
                int8_t dt = t.decision_type[node];
                int missing = (dt >> 2) & 3;
                if (std::isnan(value) && missing != 2) value = 0.0;
                bool is_missing = missing == 1 ? (value >= -ZERO_THRESHOLD && value <= ZERO_THRESHOLD)
                                               : (missing == 2 ? std::isnan(value) : false);
                bool left = is_missing ? (dt & DEFAULT_LEFT_MASK) != 0 : value <= t.threshold[node];
                node = left ? t.left_child[node] : t.right_child[node];
            }
            leaf = ~node;
        }
        score = score + t.leaf_value[leaf];
    }
    return score;
}

}  // extern "C"
