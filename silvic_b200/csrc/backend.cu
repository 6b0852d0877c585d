// backend.cu — the C ABI of include/silvic_b200.h: a B200 backend behind silvic's `trait Backend`
// (crates/silvic-core/src/backend/mod.rs:115-179) and the device-resident trainer.
//
// The handle owns one GPU's copy of its row shard (tiles of bins, labels, scores, gradients, the two partition
// buffers), the histogram staging and slot buffers, and the learner state the training kernels move. Every call
// enqueues on the handle's stream; calls that return data wait for it. Misuse returns SB2_EDEVICE with a message,
// as CpuBackend does (backend/cpu.rs:149-166), never a crash.
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "binning.cuh"
#include "iter.cuh"

using namespace sb2;

namespace {

thread_local std::string g_global_error;

struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    ~DeviceBuffer() {
        if (ptr) cudaFree(ptr);
    }
    cudaError_t alloc(size_t n) {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = n;
        return cudaMalloc(&ptr, n == 0 ? 16 : n);
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(ptr);
    }
};

struct HostTree {
    int32_t num_leaves = 1;
    double shrinkage = 1.0;
    std::vector<int32_t> split_feature;
    std::vector<float> split_gain;
    std::vector<double> threshold;
    std::vector<uint32_t> threshold_bin;
    std::vector<int8_t> decision_type;
    std::vector<int32_t> left_child, right_child;
    std::vector<double> leaf_value, leaf_weight;
    std::vector<int64_t> leaf_count;
    std::vector<double> internal_value, internal_weight;
    std::vector<int64_t> internal_count;
    std::vector<uint32_t> cat_bins;  // 8 words per split: a categorical split's left bins (0 for numerical)
};

}  // namespace

struct sb2_model {
    std::vector<HostTree> trees;
    std::vector<double> seconds;
    std::vector<double> tree_seconds;  // the persistent tree kernel's own time per iteration (single GPU)
};

struct sb2_backend {
    int device = 0;
    int sms = 148;
    int smem_optin = 232448;  // shared memory a CTA may hold (static and dynamic)
    cudaStream_t stream = nullptr;
    std::string error;
    std::string name;
    bool loaded = false;

    // dataset
    uint64_t num_rows = 0, row_offset = 0;
    uint64_t column_stride = 0;  // bytes per feature-major column
    uint32_t num_features = 0, total_bins = 0;
    sb2_objective objective{};
    bool weighted = false;
    std::vector<sb2_feature> features;                 // host copy (upper bounds below)
    std::vector<std::vector<double>> upper_bounds;
    std::vector<DevFeature> dev_features;
    std::vector<Tile> tiles;
    std::vector<Unit> units;
    std::vector<std::vector<int32_t>> group_column_feature;  // [group][column] -> feature
    int hist_smem = 0;
    int hist_grid = 0;
    GrowSmem grow_smem{};   // the persistent tree kernel's dynamic shared memory
    bool grow_ok = false;   // it fits one CTA per SM
    DeviceBuffer grid_barrier;
    DeviceBuffer phase_ns;  // per-phase nanoseconds of the persistent kernel (profiling runs)
    DeviceBuffer bins, d_tiles, d_features, d_lane_feature, d_units, columns;
    DeviceBuffer label, weight, scores, grad, hess, packed;
    DeviceBuffer rows[2], ordered[2], flags, tile_left;
    DeviceBuffer staging, hist_job, step, iter, api_active, candidates, cand_flags, cand_gain, counter, maxima, misc;
    // lambdarank: the queries and the host-computed tables the gradient kernel reads (RankArgs)
    DeviceBuffer rk_bounds, rk_queries, rk_imdcg, rk_gain, rk_discount, rk_table;
    RankArgs ranking{};
    std::vector<double> rank_gain;            // the loaded label gains, to check training parameters against
    DeviceBuffer api_spec;                    // the QuantSpec of the last sb2_quantize
    sb2_quant_spec api_spec_host{};
    const sb2_quant_spec* packed_spec = nullptr;  // the quantization the packed gradients now hold
    DeviceBuffer slabs;        // histogram scratch: one slab per histogram CTA
    uint32_t slab_ints = 0;    // ints per slab
    uint32_t slab_totals = 0;  // ints before a slab's rows' totals (0: none; no tile skips its dominant bins)
    double dominant_share = 2.0;  // sb2_set_dominant_share (above 1: no tile skips)
    DeviceBuffer d_quads;      // the slab reduction's QuadMeta table
    uint32_t num_quads = 0;
    uint32_t quad_split = 1;   // threads per quad
    std::vector<uint8_t> api_used;
    bool api_used_all = true;

    // multi-GPU
    ncclComm_t comm = nullptr;
    int world = 1, rank = 0;
    // The tree kernel's exchange with the other ranks (GrowExchange): this rank's buffer and every rank's mapped
    // here through CUDA IPC; set up by the first training run after the ranks joined.
    DeviceBuffer xbuf;
    void* xpeers[kMaxRanks] = {};
    size_t xbytes = 0;
    bool xready = false;
    uint32_t xepoch = 0;  // the last epoch a launch used
    int exchange_mode = SB2_EXCHANGE_AUTO;
    uint32_t peer_spins = kPeerSpins;  // polls of a rank's flag before the tree kernel gives up (error 4)
    // sb2_test_unanswered_peer: a second rank whose exchange buffer is local memory that nothing writes.
    bool fake_peer = false;
    DeviceBuffer fake_xbuf;

    // sb2_find_best_split_noalloc's scratch array on this handle's device, looked up by the handle's first such call.
    void* noalloc_scratch = nullptr;

    void close_exchange() {
        for (int r = 0; r < kMaxRanks; ++r)
            if (r != rank && xpeers[r] && !fake_peer) cudaIpcCloseMemHandle(xpeers[r]);
        for (auto& p : xpeers) p = nullptr;
        xready = false;
        xbytes = 0;
        fake_peer = false;
        peer_spins = kPeerSpins;
    }

    ~sb2_backend() {
        close_exchange();
        if (comm) ncclCommDestroy(comm);
        if (stream) cudaStreamDestroy(stream);
    }

    int fail(int code, const std::string& msg) {
        error = msg;
        return code;
    }
    int cuda(cudaError_t e, const char* what) {
        if (e == cudaSuccess) return SB2_OK;
        return fail(SB2_EDEVICE, std::string(what) + ": " + cudaGetErrorString(e));
    }

    DevData dev_data() const {
        DevData d{};
        d.bins = bins.as<uint8_t>();
        d.tiles = d_tiles.as<Tile>();
        d.features = d_features.as<DevFeature>();
        d.lane_feature = d_lane_feature.as<int32_t>();
        d.num_tiles = static_cast<uint32_t>(tiles.size());
        d.num_features = num_features;
        d.total_bins = total_bins;
        d.num_rows = num_rows;
        d.row_offset = row_offset;
        d.columns = columns.as<uint8_t>();
        d.column_stride = column_stride;
        return d;
    }

    RowArgs row_args() const {
        RowArgs r{};
        r.num_rows = num_rows;
        r.row_offset = row_offset;
        r.objective = objective.kind;
        r.sigmoid = objective.sigmoid;
        r.label = label.as<float>();
        r.weight = weighted ? weight.as<float>() : nullptr;
        r.scores = scores.as<float>();
        r.grad = grad.as<float>();
        r.hess = hess.as<float>();
        r.packed = packed.as<int32_t>();
        r.rank = ranking;
        return r;
    }

    // TrainArgs over the buffers the Backend API shares with training.
    TrainArgs api_train_args() const {
        TrainArgs a{};
        a.d = dev_data();
        a.total_bins = total_bins;
        a.num_features = num_features;
        a.step = step.as<Step>();
        a.staging = staging.as<int>();
        a.hist_job = hist_job.as<HistJob>();
        a.iter = iter.as<IterState>();
        for (int k = 0; k < 2; ++k) {
            a.rows[k] = rows[k].as<uint32_t>();
            a.ordered[k] = ordered[k].as<int32_t>();
        }
        a.flags = flags.as<uint32_t>();
        a.tile_left = tile_left.as<uint32_t>();
        a.candidates = candidates.ptr;
        a.cand_flags = cand_flags.as<uint8_t>();
        a.cand_gain = cand_gain.as<double>();
        a.done_counter = counter.as<unsigned int>();
        return a;
    }

    HistArgs hist_args(const uint8_t* active, int* out) const {
        HistArgs h{};
        h.d = dev_data();
        h.units = d_units.as<Unit>();
        h.num_units = static_cast<uint32_t>(units.size());
        h.min_rows_per_cta = 512;  // small leaves spread over many SMs; each CTA's zeroing and slab stay cheap
        h.job = hist_job.as<HistJob>();
        for (int k = 0; k < 2; ++k) {
            h.rows[k] = rows[k].as<uint32_t>();
            h.ordered[k] = ordered[k].as<int32_t>();
        }
        h.packed = packed.as<int32_t>();
        h.active = active;
        h.spec = packed_spec;
        h.out = out;
        h.slabs = slabs.as<int>();
        h.slab_ints = slab_ints;
        h.totals = slab_totals;
        h.num_quads = num_quads;
        h.quads = d_quads.as<QuadMeta>();
        h.quad_split = quad_split;
        return h;
    }

    // The histogram operation: per-CTA histograms into the slabs, then their sum into `h.out`.
    void run_hist(const HistArgs& h, cudaStream_t s) const {
        launch_histogram(h, hist_grid, hist_smem, s);
        launch_histogram_reduce(h, s);
    }

    int row_grid() const { return sms * 8; }
    int partition_grid() const { return sms * 4; }
    int search_grid() const {  // a warp per (child, feature) item, 8 warps per CTA
        int g = static_cast<int>((2 * num_features + 7) / 8);
        return std::max(1, std::min(g, sms * 4));
    }

    int check_loaded() {
        if (!loaded) return fail(SB2_EDEVICE, "b200 backend used before load");
        return SB2_OK;
    }
    int check_range(sb2_leaf_range leaf) {
        if (static_cast<uint64_t>(leaf.begin) + leaf.count > num_rows)
            return fail(SB2_EDEVICE, "leaf rows " + std::to_string(leaf.begin) + ".." +
                                         std::to_string(static_cast<uint64_t>(leaf.begin) + leaf.count) +
                                         " outside the partition of " + std::to_string(num_rows) + " rows");
        return SB2_OK;
    }
    int sync() { return cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize"); }
    // Single-GPU training grows each tree in one persistent launch; with NCCL ranks, per-step launches.
    // One launch per tree: one GPU, or ranks whose exchange is set up.
    bool persistent() const { return grow_ok && (comm == nullptr || xready); }
};

namespace {

#define SB2_TRY(expr)                        \
    do {                                     \
        int sb2_status_ = (expr);            \
        if (sb2_status_ != SB2_OK) return sb2_status_; \
    } while (0)

#define SB2_CUDA(b, expr) SB2_TRY((b)->cuda((expr), #expr))

int nccl_status(sb2_backend* b, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return SB2_OK;
    return b->fail(SB2_ECOLLECTIVE, std::string(what) + ": " + ncclGetErrorString(r));
}

void copy_string(const std::string& s, char* buf, size_t len) {
    if (!buf || len == 0) return;
    size_t n = std::min(len - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
}

// feature_mask (split.rs:966-985): the features one tree may split on.
void feature_mask(const std::vector<sb2_feature>& features, double fraction, uint32_t seed, uint32_t iteration,
                  uint8_t* mask) {
    std::vector<uint32_t> usable;
    for (uint32_t f = 0; f < features.size(); ++f) {
        mask[f] = 0;
        if (features[f].num_bins != 0) usable.push_back(f);
    }
    if (fraction >= 1.0) {
        for (uint32_t f : usable) mask[f] = 1;
        return;
    }
    double scaled = static_cast<double>(usable.size()) * fraction + 0.5;  // Common::RoundInt
    size_t count = std::max<size_t>(static_cast<size_t>(scaled), std::min<size_t>(usable.size(), 1));
    std::vector<std::pair<float, uint32_t>> keyed;
    for (uint32_t f : usable) keyed.emplace_back(uniform01(seed, 3u, iteration, f), f);
    std::sort(keyed.begin(), keyed.end(), [](const auto& x, const auto& y) {
        return x.first != y.first ? x.first < y.first : x.second < y.second;
    });
    for (size_t i = 0; i < std::min(count, keyed.size()); ++i) mask[keyed[i].second] = 1;
}

// Device form of a BinSplit: the tile and lane of its feature.
int split_feature_of(sb2_backend* b, const sb2_bin_split& s, int32_t& feature) {
    if (s.group >= b->group_column_feature.size() || s.column >= b->group_column_feature[s.group].size() ||
        b->group_column_feature[s.group][s.column] < 0)
        return b->fail(SB2_EDEVICE, "split on missing group " + std::to_string(s.group) + " column " +
                                        std::to_string(s.column));
    feature = b->group_column_feature[s.group][s.column];
    return SB2_OK;
}

// Stable partition of [begin, begin + count) of buffer 0 by `st` (a split or a bag), written back into buffer 0.
int run_partition(sb2_backend* b, Step st, uint32_t* out_left) {
    TrainArgs a = b->api_train_args();
    SB2_CUDA(b, cudaMemcpyAsync(b->step.ptr, &st, sizeof(Step), cudaMemcpyHostToDevice, b->stream));
    launch_partition_flags(a, b->partition_grid(), b->stream);
    launch_partition_scatter(a, b->partition_grid(), b->stream);
    SB2_CUDA(b, cudaGetLastError());
    const size_t off = st.begin;
    SB2_CUDA(b, cudaMemcpyAsync(b->rows[0].as<uint32_t>() + off, b->rows[1].as<uint32_t>() + off,
                                sizeof(uint32_t) * st.count, cudaMemcpyDeviceToDevice, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->ordered[0].as<int32_t>() + off, b->ordered[1].as<int32_t>() + off,
                                sizeof(int32_t) * st.count, cudaMemcpyDeviceToDevice, b->stream));
    Step back{};
    SB2_CUDA(b, cudaMemcpyAsync(&back, b->step.ptr, sizeof(Step), cudaMemcpyDeviceToHost, b->stream));
    SB2_TRY(b->sync());
    *out_left = back.local_left;
    return SB2_OK;
}

// Histogram of buffer-0 positions [begin, begin + count) into `out` (2 * total_bins doubles).
int run_histogram(sb2_backend* b, sb2_leaf_range leaf, double* out, size_t len) {
    if (len != 2ull * b->total_bins)
        return b->fail(SB2_EDEVICE, "histogram buffer of " + std::to_string(len) + " values, expected " +
                                        std::to_string(2ull * b->total_bins));
    if (b->packed_spec == nullptr) return b->fail(SB2_EDEVICE, "histogram before any quantization");
    if (b->packed_spec == b->api_spec.as<sb2_quant_spec>()) {
        // The device sums in int32: every bin's sums must fit.
        const sb2_quant_spec& q = b->api_spec_host;
        const uint64_t max_q = static_cast<uint64_t>(std::max({q.grad_max_q, q.constant_hessian ? 1 : q.hess_max_q, 1}));
        if (static_cast<uint64_t>(leaf.count) * max_q > 2147483647ull)
            return b->fail(SB2_EUNSUPPORTED, "histogram sums of " + std::to_string(leaf.count) + " rows at " +
                                                 std::to_string(max_q) + " units per row could pass int32");
    }
    SB2_CUDA(b, cudaMemsetAsync(b->staging.ptr, 0, sizeof(int) * (2ull * b->total_bins + 2), b->stream));
    HistJob job{};
    job.active = 1;
    job.identity = 0;
    job.begin = leaf.begin;
    job.count = leaf.count;
    job.which = 0;
    SB2_CUDA(b, cudaMemcpyAsync(b->hist_job.ptr, &job, sizeof(job), cudaMemcpyHostToDevice, b->stream));
    const uint8_t* active = b->api_used_all ? nullptr : b->api_active.as<uint8_t>();
    b->run_hist(b->hist_args(active, b->staging.as<int>()), b->stream);
    SB2_CUDA(b, cudaGetLastError());
    std::vector<int> host(2ull * b->total_bins);
    SB2_CUDA(b, cudaMemcpyAsync(host.data(), b->staging.ptr, sizeof(int) * host.size(), cudaMemcpyDeviceToHost,
                                b->stream));
    SB2_TRY(b->sync());
    for (size_t i = 0; i < host.size(); ++i) out[i] = static_cast<double>(host[i]);
    return SB2_OK;
}

}  // namespace

extern "C" {

int sb2_global_error(char* buf, size_t len) {
    copy_string(g_global_error, buf, len);
    return SB2_OK;
}

void sb2_default_params(sb2_params* p) {
    std::memset(p, 0, sizeof(*p));
    p->objective = SB2_REGRESSION;
    p->num_iterations = 100;
    p->learning_rate = 0.1;
    p->num_leaves = 31;
    p->max_depth = -1;
    p->min_data_in_leaf = 20;
    p->min_sum_hessian_in_leaf = 1e-3;
    p->lambda_l1 = 0.0;
    p->lambda_l2 = 0.0;
    p->min_gain_to_split = 0.0;
    p->bagging_fraction = 1.0;
    p->bagging_freq = 0;
    p->bagging_seed = 3;
    p->feature_fraction = 1.0;
    p->feature_fraction_seed = 2;
    p->data_random_seed = 1;
    p->boost_from_average = 1;
    p->use_quantized_grad = 1;
    p->sigmoid = 1.0;
    p->num_grad_quant_bins = 4;
    p->quant_train_renew_leaf = 1;
    p->stochastic_rounding = 1;
    p->lambdarank_norm = 1;                // config.rs:153-154
    p->lambdarank_truncation_level = 30;
    p->label_gain = nullptr;               // config.rs:118-121: 2^i - 1 for i < 31
    p->num_label_gain = 0;
    p->max_cat_to_onehot = 4;              // config.rs:145-149
    p->max_cat_threshold = 32;
    p->cat_l2 = 10.0;
    p->cat_smooth = 10.0;
    p->min_data_per_group = 100;
}

int sb2_create(int device, sb2_backend** out) {
    if (!out) {
        g_global_error = "sb2_create: null output";
        return SB2_EDEVICE;
    }
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        g_global_error = std::string("no CUDA device: ") + cudaGetErrorString(e);
        return SB2_EDEVICE;
    }
    if (device < 0 || device >= count) {
        g_global_error = "CUDA device " + std::to_string(device) + " of " + std::to_string(count);
        return SB2_EDEVICE;
    }
    auto b = std::make_unique<sb2_backend>();
    b->device = device;
    if ((e = cudaSetDevice(device)) != cudaSuccess || (e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking)) != cudaSuccess) {
        g_global_error = std::string("CUDA setup: ") + cudaGetErrorString(e);
        return SB2_EDEVICE;
    }
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, device);
    if (prop.major < 10) {
        g_global_error = std::string("device ") + prop.name + " is not sm_100 (Blackwell)";
        return SB2_EUNSUPPORTED;
    }
    b->sms = prop.multiProcessorCount;
    b->smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
    b->name = std::string(prop.name) + " (cuda sm_" + std::to_string(prop.major) + std::to_string(prop.minor) + ")";
    *out = b.release();
    return SB2_OK;
}

int sb2_destroy(sb2_backend* b) {
    if (!b) return SB2_OK;
    cudaSetDevice(b->device);
    delete b;
    return SB2_OK;
}

int sb2_last_error(const sb2_backend* b, char* buf, size_t len) {
    copy_string(b ? b->error : g_global_error, buf, len);
    return SB2_OK;
}

int sb2_name(const sb2_backend* b, char* buf, size_t len) {
    copy_string(b->name, buf, len);
    return SB2_OK;
}

namespace {

// LightGBM's default label gains (config.rs:118-121): 2^i - 1 for i < 31.
std::vector<double> label_gains(const double* gain, uint32_t count) {
    if (gain != nullptr && count > 0) return std::vector<double>(gain, gain + count);
    std::vector<double> g;
    for (uint32_t i = 0; i < 31; ++i) g.push_back(static_cast<double>((1u << i) - 1u));
    return g;
}

// ObjectiveSetup::LambdaRank (objective/mod.rs:35-65) for the device: the queries checked and uploaded, and the
// tables the gradient kernel reads, computed here once with the reference's own expressions and the same libm
// (lambdarank.rs:37-46 discounts, :51-72 the sigmoid table, :122-139 max DCG, :173-195 the label checks).
int load_ranking(sb2_backend* b, const sb2_dataset* d, const sb2_objective* o) {
    const uint64_t n = d->num_rows;
    const uint32_t nq = d->num_queries;
    const uint32_t* qb = d->query_boundaries;
    if (qb == nullptr || nq == 0) return b->fail(SB2_EDATA, "ranking tasks require query information");
    if (qb[0] != 0 || qb[nq] != n) return b->fail(SB2_EDATA, "query boundaries must run from row 0 to the last row");
    uint32_t longest = 0;
    for (uint32_t q = 0; q < nq; ++q) {
        if (qb[q + 1] < qb[q]) return b->fail(SB2_EDATA, "query boundaries must not decrease");
        longest = std::max(longest, qb[q + 1] - qb[q]);
    }
    if (longest > kMaxQueryRows)
        return b->fail(SB2_EUNSUPPORTED, "a query of " + std::to_string(longest) + " rows; the device takes " +
                                             std::to_string(kMaxQueryRows) + " at most");
    if (!(o->sigmoid > 0.0)) return b->fail(SB2_ECONFIG, "lambdarank needs a positive sigmoid");
    const std::vector<double> gain = label_gains(o->label_gain, o->num_label_gain);
    for (uint64_t i = 0; i < n; ++i) {
        const float l = d->label[i];
        if (std::fabs(static_cast<double>(l) - static_cast<double>(static_cast<int32_t>(l))) > static_cast<double>(1e-15f) ||
            l < 0.0f || static_cast<size_t>(l) >= gain.size())
            return b->fail(SB2_EDATA, "lambdarank label " + std::to_string(l) + " of row " + std::to_string(i) +
                                          " is not a non-negative integer below the " + std::to_string(gain.size()) +
                                          " label gains");
    }
    std::vector<double> discount(kMaxQueryRows);
    for (uint32_t i = 0; i < kMaxQueryRows; ++i) discount[i] = 1.0 / std::log2(2.0 + static_cast<double>(i));
    const size_t k = o->lambdarank_truncation_level;
    std::vector<double> inverse_max_dcg(nq);
    std::vector<size_t> count(gain.size());
    for (uint32_t q = 0; q < nq; ++q) {
        std::fill(count.begin(), count.end(), 0);
        for (uint32_t r = qb[q]; r < qb[q + 1]; ++r) ++count[static_cast<size_t>(d->label[r])];
        size_t top = gain.size() - 1;
        double dcg = 0.0;
        for (size_t j = 0; j < std::min<size_t>(k, qb[q + 1] - qb[q]); ++j) {
            while (top > 0 && count[top] == 0) --top;
            dcg += discount[j] * gain[top];
            --count[top];  // wraps at label 0, as the reference's wrapping_sub
        }
        inverse_max_dcg[q] = dcg > 0.0 ? 1.0 / dcg : 0.0;
    }
    RankArgs& a = b->ranking;
    a = RankArgs{};
    a.sigmoid = o->sigmoid;
    a.sigmoid_squared = o->sigmoid * o->sigmoid;
    a.min_input = -50.0 / o->sigmoid / 2.0;
    a.max_input = -a.min_input;
    a.idx_factor = static_cast<double>(kSigmoidBins) / (a.max_input - a.min_input);
    std::vector<double> table(kSigmoidBins);
    for (uint32_t i = 0; i < kSigmoidBins; ++i) {
        const double score = static_cast<double>(i) / a.idx_factor + a.min_input;
        table[i] = 1.0 / (1.0 + std::exp(score * o->sigmoid));
    }
    // The queries the warp kernel takes (at most lambdarank_warp_rows() rows), then the rest, each in row order.
    std::vector<uint32_t> order;
    for (uint32_t q = 0; q < nq; ++q)
        if (qb[q + 1] - qb[q] <= lambdarank_warp_rows()) order.push_back(q);
    const uint32_t num_short = static_cast<uint32_t>(order.size());
    for (uint32_t q = 0; q < nq; ++q)
        if (qb[q + 1] - qb[q] > lambdarank_warp_rows()) order.push_back(q);
    SB2_CUDA(b, b->rk_queries.alloc(sizeof(uint32_t) * nq));
    SB2_CUDA(b, cudaMemcpyAsync(b->rk_queries.ptr, order.data(), sizeof(uint32_t) * nq, cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, b->rk_bounds.alloc(sizeof(uint32_t) * (nq + 1ull)));
    SB2_CUDA(b, b->rk_imdcg.alloc(sizeof(double) * nq));
    SB2_CUDA(b, b->rk_gain.alloc(sizeof(double) * gain.size()));
    SB2_CUDA(b, b->rk_discount.alloc(sizeof(double) * discount.size()));
    SB2_CUDA(b, b->rk_table.alloc(sizeof(double) * table.size()));
    SB2_CUDA(b, cudaMemcpyAsync(b->rk_bounds.ptr, qb, sizeof(uint32_t) * (nq + 1ull), cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->rk_imdcg.ptr, inverse_max_dcg.data(), sizeof(double) * nq, cudaMemcpyHostToDevice,
                                b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->rk_gain.ptr, gain.data(), sizeof(double) * gain.size(), cudaMemcpyHostToDevice,
                                b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->rk_discount.ptr, discount.data(), sizeof(double) * discount.size(),
                                cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->rk_table.ptr, table.data(), sizeof(double) * table.size(), cudaMemcpyHostToDevice,
                                b->stream));
    SB2_TRY(b->sync());  // the host tables go out of scope
    a.bounds = b->rk_bounds.as<uint32_t>();
    a.queries = b->rk_queries.as<uint32_t>();
    a.num_short = num_short;
    a.num_gain = static_cast<uint32_t>(gain.size());
    a.inverse_max_dcg = b->rk_imdcg.as<double>();
    a.label_gain = b->rk_gain.as<double>();
    a.discount = b->rk_discount.as<double>();
    a.table = b->rk_table.as<double>();
    a.num_queries = nq;
    a.cap = 2;
    while (a.cap < longest) a.cap <<= 1;
    a.truncation = static_cast<uint32_t>(std::min<size_t>(k, 0xFFFFFFFFu));
    a.norm = o->lambdarank_norm != 0;
    int warp_per_sm = 0, cta_per_sm = 0;
    SB2_CUDA(b, lambdarank_configure(a.cap, &warp_per_sm, &cta_per_sm));
    if (warp_per_sm < 1 || (num_short < nq && cta_per_sm < 1))
        return b->fail(SB2_EUNSUPPORTED, "the lambdarank kernels do not fit this dataset's queries");
    a.warp_grid = static_cast<uint32_t>(std::max(1, b->sms * warp_per_sm));
    a.cta_grid = static_cast<uint32_t>(std::max(1, std::min<int>(static_cast<int>(nq - num_short), b->sms * cta_per_sm)));
    b->rank_gain = gain;
    return SB2_OK;
}

}  // namespace

// Backend::load
int sb2_load(sb2_backend* b, const sb2_dataset* train, const sb2_objective* objective) {
    if (!b || !train || !objective) return SB2_EDEVICE;
    SB2_CUDA(b, cudaSetDevice(b->device));
    if (train->num_rows > 0xFFFFFFFFull)
        return b->fail(SB2_EUNSUPPORTED, std::to_string(train->num_rows) + " rows on one rank; the limit is 2^32 - 1");
    if (objective->kind != SB2_REGRESSION && objective->kind != SB2_BINARY && objective->kind != SB2_LAMBDARANK)
        return b->fail(SB2_EUNSUPPORTED, "objective " + std::to_string(objective->kind) + " has no device gradients");
    b->ranking = RankArgs{};
    if (objective->kind == SB2_LAMBDARANK) SB2_TRY(load_ranking(b, train, objective));
    const uint32_t F = train->num_features;
    b->features.assign(train->features, train->features + F);
    b->upper_bounds.assign(F, {});
    b->dev_features.assign(F, DevFeature{});
    b->group_column_feature.assign(train->num_groups, {});
    for (uint32_t g = 0; g < train->num_groups; ++g) {
        const sb2_group& grp = train->groups[g];
        b->group_column_feature[g].assign(grp.row_stride, -1);
        for (uint32_t k = 0; k < grp.num_features; ++k) {
            uint32_t f = grp.features[k];
            if (f >= F) return b->fail(SB2_EDATA, "group lists a missing feature");
            const sb2_feature& m = train->features[f];
            if (m.column >= grp.row_stride || m.group != g || m.hist_offset < grp.hist_offset ||
                m.hist_offset - grp.hist_offset + m.num_bins > grp.total_bins)
                return b->fail(SB2_EDATA, "feature " + std::to_string(f) + " lies outside its group's bins or row");
            b->group_column_feature[g][m.column] = static_cast<int32_t>(f);
        }
    }
    // Tiles: the non-trivial features in order, 32 per tile.
    std::vector<uint32_t> used;
    for (uint32_t f = 0; f < F; ++f) {
        const sb2_feature& m = train->features[f];
        if (m.num_bins > 256) return b->fail(SB2_EDATA, "feature with more than 256 bins");
        if (m.kind == SB2_NUMERICAL && m.num_bins > 0) {
            size_t nb = m.num_bins - (m.nan_bin ? 1 : 0);
            if (!m.upper_bounds || m.num_upper_bounds < nb)
                return b->fail(SB2_EDATA, "numerical feature " + std::to_string(f) + " without its upper bounds");
            b->upper_bounds[f].assign(m.upper_bounds, m.upper_bounds + m.num_upper_bounds);
        }
        b->features[f].upper_bounds = nullptr;
        DevFeature& d = b->dev_features[f];
        d.tile = -1;
        d.lane = -1;
        d.hist_offset = m.hist_offset;
        d.num_bins = m.num_bins;
        d.nan_bin = m.nan_bin;
        d.kind = m.kind;
        d.slab_off = 0;
        d.mfb = 0;
        if (m.num_bins > 0 && m.kind != SB2_TRIVIAL) {
            if (m.group >= train->num_groups) return b->fail(SB2_EDATA, "feature in a missing group");
            used.push_back(f);
        }
    }
    const uint64_t n = train->num_rows;
    b->tiles.clear();
    std::vector<int32_t> lane_feature;
    for (size_t i = 0; i < used.size(); i += kTileLanes) {
        Tile t{};
        t.nfeat = static_cast<uint32_t>(std::min<size_t>(kTileLanes, used.size() - i));
        // Row bytes: 4, 8, 16 or 32, so a row is one aligned vector load.
        t.stride = 4;
        while (t.stride < t.nfeat) t.stride *= 2;
        t.base = 0;  // placed with its unit below
        t.pitch = t.stride;
        t.smem_bins = 0;
        for (uint32_t l = 0; l < kTileLanes; ++l) {
            int32_t f = l < t.nfeat ? static_cast<int32_t>(used[i + l]) : -1;
            lane_feature.push_back(f);
            if (f >= 0) {
                b->dev_features[f].tile = static_cast<int32_t>(b->tiles.size());
                b->dev_features[f].lane = static_cast<int32_t>(l);
                t.smem_bins = std::max(t.smem_bins, train->features[f].num_bins);
            }
        }
        // 64, 128 or 256 bin slots per lane: the histogram kernel's shared addressing is specialised on these.
        t.smem_bins = t.smem_bins <= 64 ? 64 : t.smem_bins <= 128 ? 128 : 256;
        b->tiles.push_back(t);
    }
    // Histogram units: consecutive tiles, up to kMaxUnitTiles within a shared-memory budget (one packed int32 array
    // of smem_bins * stride slots per tile).
#ifndef SB2_UNIT_BUDGET_KB
#define SB2_UNIT_BUDGET_KB 220  // of the 227 KB a CTA may hold, leaving room for the kernels' static shared memory
#endif
    constexpr size_t kUnitBudget = SB2_UNIT_BUDGET_KB * 1024;
    b->units.clear();
    size_t max_unit_bytes = 0;
    std::vector<uint32_t> unit_features;
    for (size_t i = 0; i < b->tiles.size();) {
        Unit u{};
        u.first_tile = static_cast<uint32_t>(i);
        size_t bytes = 0;
        uint32_t feats = 0;
        while (i < b->tiles.size() && u.num_tiles < static_cast<uint32_t>(kMaxUnitTiles)) {
            size_t tb = 4ull * b->tiles[i].smem_bins * b->tiles[i].stride;
            if (u.num_tiles > 0 && bytes + tb > kUnitBudget) break;
            bytes += tb;
            u.slots += b->tiles[i].smem_bins * b->tiles[i].stride;
            feats += b->tiles[i].nfeat;
            ++u.num_tiles;
            ++i;
        }
        max_unit_bytes = std::max(max_unit_bytes, bytes);
        b->units.push_back(u);
        unit_features.push_back(feats);
    }
    // The bins in device memory: per unit, each row's bytes of the unit's full tiles (32 features: one 32-byte
    // sector a row) side by side, so that a histogram reading a leaf's scattered rows reads one run of sectors per
    // row and unit instead of one sector in each tile's region; a partial tile (the last one) keeps its own region,
    // where its narrow rows pack whole sectors.
    uint64_t base = 0;
    for (const Unit& u : b->units) {
        uint32_t full = 0;
        for (uint32_t t = u.first_tile; t < u.first_tile + u.num_tiles; ++t) full += b->tiles[t].stride == 32;
        uint32_t k = 0;
        for (uint32_t t = u.first_tile; t < u.first_tile + u.num_tiles; ++t) {
            Tile& tile = b->tiles[t];
            if (tile.stride != 32) continue;
            tile.base = base + 32 * k++;
            tile.pitch = 32 * full;
        }
        base += (n * 32 * full + 127) / 128 * 128;
        for (uint32_t t = u.first_tile; t < u.first_tile + u.num_tiles; ++t) {
            Tile& tile = b->tiles[t];
            if (tile.stride == 32) continue;
            tile.base = base;
            tile.pitch = tile.stride;
            base += (n * tile.stride + 127) / 128 * 128;
        }
    }
    // Where each feature's bins sit in the tree kernel's slabs: feature-major inside each unit's region (the unit's
    // tiles in order, each tile's lanes in order, smem_bins slots per lane), so a feature's bins are contiguous.
    {
        uint32_t before = 0;  // slots of the earlier units
        for (const Unit& u : b->units) {
            uint32_t p = 0;  // slots of the unit's earlier tiles
            for (uint32_t t = u.first_tile; t < u.first_tile + u.num_tiles; ++t) {
                const Tile& tile = b->tiles[t];
                for (uint32_t l = 0; l < tile.nfeat; ++l) {
                    const int32_t f = lane_feature[t * kTileLanes + l];
                    if (f >= 0) b->dev_features[f].slab_off = before + p + l * tile.smem_bins;
                }
                p += tile.smem_bins * tile.stride;
            }
            before += u.slots;
        }
    }
    // The kernel aligns its histogram to kHistAlign bytes inside the dynamic shared memory.
    b->hist_smem = static_cast<int>(std::max<size_t>(max_unit_bytes, 16) + kHistAlign);
    SB2_CUDA(b, histogram_configure(b->hist_smem));
    int per_sm = 1;
    SB2_CUDA(b, histogram_occupancy(b->hist_smem, &per_sm));
    per_sm = std::max(per_sm, 1);
    // The persistent tree kernel runs every phase in the same CTAs: its shared memory also holds the partition's
    // scan and the search's bins.
    // Layout (GrowSmem): the histogram's arrays, the partition's scan words, the staging area (all three used in the
    // same phase), then the per-feature flags ((5 kSplits + 1) F bytes); the search's bins (kMaxBins [g, h] pairs per
    // group of warps, 4 KB in all) reuse the scan words. The staging area gets what is left of the CTA's shared
    // memory, up to kMaxStageDepth slots of a unit's 32 rows per warp: the histogram stages the rows of a unit of one
    // partial tile there (full tiles go straight to registers), the flush transposes the shared sums through it, and
    // the search reduces and prefetches slab bins in it.
    {
        GrowSmem& m = b->grow_smem;
        m.scan_offset = static_cast<uint32_t>((b->hist_smem + 15) / 16 * 16);
        m.stage_offset = static_cast<uint32_t>((m.scan_offset + (2ull * grow_threads() + 64) * 4 + 127) / 128 * 128);
        uint32_t slot = 0;
        for (const Unit& u : b->units) {
            uint32_t rows = 0;
            for (uint32_t t = 0; t < u.num_tiles; ++t) rows += 32 * b->tiles[u.first_tile + t].stride;
            slot = std::max(slot, rows);
        }
        m.slot_bytes = (slot + 128 + 127) / 128 * 128;  // the rows, then 32 packed gradients
        const size_t flags = ((5ull * kSplits + 1) * F + 15) / 16 * 16;
        const int stat = grow_static_smem();
        if (stat < 0) return b->fail(SB2_EDEVICE, "cudaFuncGetAttributes(grow_tree)");
        const size_t limit = static_cast<size_t>(b->smem_optin) - static_cast<size_t>(stat);
        const size_t per_depth = static_cast<size_t>(grow_threads() / 32) * m.slot_bytes;
        const size_t used = m.stage_offset + flags;
        m.stage_depth = used < limit ? static_cast<uint32_t>(std::min<size_t>((limit - used) / per_depth, kMaxStageDepth)) : 0;
        static_assert((2 * 512 + 64) * 4 >= 2 * kMaxBins * 8, "the search's bins fit the scan words");
        m.flags_offset = static_cast<uint32_t>((m.stage_offset + m.stage_depth * per_depth + 15) / 16 * 16);
        m.bytes = static_cast<int>(m.flags_offset + flags);
        // The histogram's cost per built row against the partition's per parent row: one shared atomic per bin byte
        // of the row against ~17 bytes moved; 3 at 100 features, 8 at 256, at least 1.
        uint32_t row_bytes = 0;
        for (const Tile& t : b->tiles) row_bytes += t.stride;
        m.hist_weight = std::max(1.0f, static_cast<float>(row_bytes) / 32.0f);
    }
    int grow_per_sm = 0;
    SB2_CUDA(b, grow_configure(b->grow_smem.bytes, &grow_per_sm));
    b->grow_ok = grow_per_sm >= 1;
    if (b->grow_ok) per_sm = std::min(per_sm, grow_per_sm);  // one grid for both paths: the units' CTA ranges
    // CTAs in proportion to each unit's features (its share of the atomics), at least one each.
    const int nu = static_cast<int>(b->units.size());
    const uint32_t total_ctas = static_cast<uint32_t>(std::max(nu, b->sms * per_sm));
    uint32_t all_feats = 0;
    for (uint32_t f : unit_features) all_feats += f;
    uint32_t next = 0;
    for (int u = 0; u < nu; ++u) {
        uint32_t share = all_feats ? static_cast<uint32_t>(static_cast<uint64_t>(total_ctas) * unit_features[u] / all_feats) : 1;
        b->units[u].cta_begin = next;
        b->units[u].cta_count = std::max<uint32_t>(share, 1);
        next += b->units[u].cta_count;
    }
    b->hist_grid = static_cast<int>(std::max<uint32_t>(next, 1));

    b->num_rows = n;
    b->row_offset = train->row_offset;
    b->num_features = F;
    b->total_bins = train->total_bins;
    b->objective = *objective;
    b->objective.label_gain = nullptr;  // the gains live in rank_gain; the caller's array is not kept
    b->weighted = train->weight != nullptr;

    // Device buffers.
    SB2_CUDA(b, b->bins.alloc(std::max<uint64_t>(base, 128)));
    SB2_CUDA(b, b->d_tiles.alloc(sizeof(Tile) * std::max<size_t>(b->tiles.size(), 1)));
    SB2_CUDA(b, b->d_features.alloc(sizeof(DevFeature) * std::max<size_t>(F, 1)));
    SB2_CUDA(b, b->d_lane_feature.alloc(sizeof(int32_t) * std::max<size_t>(lane_feature.size(), 1)));
    SB2_CUDA(b, b->d_units.alloc(sizeof(Unit) * std::max<size_t>(b->units.size(), 1)));
    SB2_CUDA(b, cudaMemcpyAsync(b->d_tiles.ptr, b->tiles.data(), sizeof(Tile) * b->tiles.size(), cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->d_features.ptr, b->dev_features.data(), sizeof(DevFeature) * F, cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->d_lane_feature.ptr, lane_feature.data(), sizeof(int32_t) * lane_feature.size(), cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->d_units.ptr, b->units.data(), sizeof(Unit) * b->units.size(), cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->bins.ptr, 0, b->bins.bytes, b->stream));  // tile padding past the last row
    SB2_CUDA(b, b->counter.alloc(sizeof(unsigned int)));
    SB2_CUDA(b, cudaMemsetAsync(b->counter.ptr, 0, sizeof(unsigned int), b->stream));
    // Bins: each group uploaded once (one staging buffer, in stream order) and transposed into the feature-major
    // copy the tree kernel's partition reads, every bin checked against its feature; then the tiles from the copy.
    b->column_stride = (n + 127) / 128 * 128;
    SB2_CUDA(b, b->columns.alloc(std::max<uint64_t>(static_cast<uint64_t>(F) * b->column_stride, 128)));
    {
        uint64_t max_group = 0;
        uint32_t max_stride = 1;
        for (uint32_t g = 0; g < train->num_groups; ++g) {
            max_group = std::max<uint64_t>(max_group, n * train->groups[g].row_stride);
            max_stride = std::max(max_stride, train->groups[g].row_stride);
        }
        DeviceBuffer group_buf, group_meta;
        SB2_CUDA(b, group_buf.alloc(std::max<uint64_t>(max_group, 16)));
        SB2_CUDA(b, group_meta.alloc(8ull * max_stride));
        std::vector<std::vector<int32_t>> metas(train->num_groups);  // alive until the copies are done
        for (uint32_t g = 0; g < train->num_groups && n > 0; ++g) {
            const sb2_group& grp = train->groups[g];
            std::vector<int32_t>& meta = metas[g];  // [row_stride] column -> feature, then [row_stride] bins
            meta.assign(2ull * grp.row_stride, -1);
            for (uint32_t k = 0; k < grp.num_features; ++k) {
                const uint32_t f = grp.features[k];
                const uint32_t col = train->features[f].column;
                if (col >= grp.row_stride) return b->fail(SB2_EDEVICE, "a feature's column lies outside its group's rows");
                if (b->dev_features[f].tile < 0) continue;
                meta[col] = static_cast<int32_t>(f);
                meta[grp.row_stride + col] = static_cast<int32_t>(b->dev_features[f].num_bins);
            }
            SB2_CUDA(b, cudaMemcpyAsync(group_buf.ptr, grp.data, n * grp.row_stride, cudaMemcpyHostToDevice, b->stream));
            SB2_CUDA(b, cudaMemcpyAsync(group_meta.ptr, meta.data(), sizeof(int32_t) * meta.size(), cudaMemcpyHostToDevice,
                                        b->stream));
            launch_group_columns(group_buf.as<uint8_t>(), n, grp.row_stride, group_meta.as<int32_t>(),
                                 reinterpret_cast<const uint32_t*>(group_meta.as<int32_t>() + grp.row_stride),
                                 b->columns.as<uint8_t>(), b->column_stride, b->counter.as<unsigned int>(), b->stream);
            SB2_CUDA(b, cudaGetLastError());
        }
        // Each feature's most frequent bin (LightGBM's most_freq_bin; the reference's GPU backend keeps it per
        // column, crates/silvic-gpu/src/backend.rs:336-376): a tile whose features hold at least dominant_share of
        // the rows in theirs, on average, stores each feature's bins 0 and mfb exchanged, and the tree kernel's
        // histogram skips the stored 0s (recovered from the rows' totals).
        DeviceBuffer d_used, d_counts;
        std::vector<int32_t> used_ids(used.begin(), used.end());
        std::vector<unsigned int> counts;
        if (n > 0 && !used.empty() && b->dominant_share <= 1.0) {
            SB2_CUDA(b, d_used.alloc(sizeof(int32_t) * used.size()));
            SB2_CUDA(b, d_counts.alloc(sizeof(unsigned int) * 256 * used.size()));
            SB2_CUDA(b, cudaMemcpyAsync(d_used.ptr, used_ids.data(), sizeof(int32_t) * used.size(), cudaMemcpyHostToDevice,
                                        b->stream));
            SB2_CUDA(b, cudaMemsetAsync(d_counts.ptr, 0, d_counts.bytes, b->stream));
            launch_bin_counts(b->columns.as<uint8_t>(), b->column_stride, n, d_used.as<int32_t>(),
                              static_cast<uint32_t>(used.size()), d_counts.as<unsigned int>(), b->stream);
            SB2_CUDA(b, cudaGetLastError());
            counts.resize(256 * used.size());
            SB2_CUDA(b, cudaMemcpyAsync(counts.data(), d_counts.ptr, sizeof(unsigned int) * counts.size(),
                                        cudaMemcpyDeviceToHost, b->stream));
            SB2_TRY(b->sync());
            for (size_t t = 0; t < b->tiles.size(); ++t) {
                Tile& tile = b->tiles[t];
                uint32_t mfb[kTileLanes] = {};
                double held = 0;
                for (uint32_t l = 0; l < tile.nfeat; ++l) {
                    const size_t i = t * kTileLanes + l;  // the tiles hold the used features in order
                    const unsigned int* c = counts.data() + 256 * i;
                    for (uint32_t bin = 1; bin < b->dev_features[used[i]].num_bins; ++bin)
                        if (c[bin] > c[mfb[l]]) mfb[l] = bin;
                    held += c[mfb[l]];
                }
                if (held < b->dominant_share * static_cast<double>(n) * tile.nfeat) continue;
                tile.skip = 1;
                for (uint32_t l = 0; l < tile.nfeat; ++l) b->dev_features[used[t * kTileLanes + l]].mfb = mfb[l] | kDominantSkip;
            }
            SB2_CUDA(b, cudaMemcpyAsync(b->d_tiles.ptr, b->tiles.data(), sizeof(Tile) * b->tiles.size(),
                                        cudaMemcpyHostToDevice, b->stream));
            SB2_CUDA(b, cudaMemcpyAsync(b->d_features.ptr, b->dev_features.data(), sizeof(DevFeature) * F,
                                        cudaMemcpyHostToDevice, b->stream));
        }
        launch_tiles(b->dev_data(), b->bins.as<uint8_t>(), b->stream);
        SB2_CUDA(b, cudaGetLastError());
        SB2_TRY(b->sync());  // the staging buffers go out of scope
    }
    // Rows.
    SB2_CUDA(b, b->label.alloc(sizeof(float) * n));
    SB2_CUDA(b, b->weight.alloc(sizeof(float) * (b->weighted ? n : 1)));
    SB2_CUDA(b, b->scores.alloc(sizeof(float) * n));
    SB2_CUDA(b, b->grad.alloc(sizeof(float) * n));
    SB2_CUDA(b, b->hess.alloc(sizeof(float) * n));
    SB2_CUDA(b, b->packed.alloc(sizeof(int32_t) * n));
    for (int k = 0; k < 2; ++k) {
        SB2_CUDA(b, b->rows[k].alloc(sizeof(uint32_t) * n));
        SB2_CUDA(b, b->ordered[k].alloc(sizeof(int32_t) * n));
    }
    SB2_CUDA(b, b->flags.alloc(sizeof(uint32_t) * kSplits * (n / 32 + 2)));  // the tree kernel's splits
    SB2_CUDA(b, b->tile_left.alloc(sizeof(uint32_t) * kMaxPartitionCtas));
    SB2_CUDA(b, b->staging.alloc(sizeof(int) * (2ull * b->total_bins + 2)));
    // A slab holds one unit's histogram (the standalone kernels, one unit per CTA) or every unit's (the persistent
    // tree kernel, where a CTA histograms every unit of its rows).
    b->slab_ints = 0;
    for (const Unit& u : b->units) b->slab_ints += 2 * u.slots;
    // The tree kernel's slabs end with the rows' totals [g, h] when a tile skips its dominant bins (4 ints: the
    // slabs stay 16-byte aligned).
    b->slab_totals = 0;
    for (const Tile& t : b->tiles)
        if (t.skip) b->slab_totals = b->slab_ints;
    if (b->slab_totals != 0) b->slab_ints += 4;
    // The reduction's quads: per unit, per tile, four consecutive slots (one bin, lanes l .. l + 3).
    std::vector<QuadMeta> quads;
    for (uint32_t ui = 0; ui < b->units.size(); ++ui) {
        const Unit& u = b->units[ui];
        uint32_t off = 0;
        for (uint32_t t = u.first_tile; t < u.first_tile + u.num_tiles; ++t) {
            const Tile& tile = b->tiles[t];
            const uint32_t n = tile.smem_bins * tile.stride;
            for (uint32_t s = 0; s < n; s += 4) {
                QuadMeta m{};
                m.unit = ui;
                m.g_off = off + s;
                m.h_off = off + n + s;
                const uint32_t bin = s / tile.stride, lane0 = s % tile.stride;
                for (uint32_t i = 0; i < 4; ++i) {
                    const int32_t f = lane_feature[t * kTileLanes + lane0 + i];
                    // the tiles store bins 0 and mfb exchanged: slot `bin` holds bin swap_dominant(bin, mfb)
                    m.out[i] = f >= 0 && bin < b->dev_features[f].num_bins
                                   ? static_cast<int32_t>(b->dev_features[f].hist_offset +
                                                          swap_dominant(bin, b->dev_features[f].mfb & 0xFFu))
                                   : -1;
                }
                quads.push_back(m);
            }
            off += 2 * n;
        }
    }
    b->num_quads = static_cast<uint32_t>(quads.size());
    // Threads per quad: as many as keep every thread of one histogram grid busy, up to a warp.
    const uint64_t grid_threads = static_cast<uint64_t>(b->hist_grid) * histogram_threads();
    b->quad_split = 1;
    while (b->quad_split < 32 && static_cast<uint64_t>(b->quad_split) * 2 * b->num_quads <= grid_threads)
        b->quad_split *= 2;
    SB2_CUDA(b, b->d_quads.alloc(sizeof(QuadMeta) * std::max<size_t>(quads.size(), 1)));
    if (!quads.empty())
        SB2_CUDA(b, cudaMemcpyAsync(b->d_quads.ptr, quads.data(), sizeof(QuadMeta) * quads.size(),
                                    cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, b->slabs.alloc(sizeof(int) * static_cast<size_t>(b->hist_grid) * std::max<uint32_t>(b->slab_ints, 4)));
    SB2_CUDA(b, b->hist_job.alloc(sizeof(HistJob)));
    SB2_CUDA(b, b->step.alloc(sizeof(Step)));
    SB2_CUDA(b, b->iter.alloc(sizeof(IterState)));
    SB2_CUDA(b, b->api_active.alloc(std::max<size_t>(F, 1)));
    SB2_CUDA(b, b->api_spec.alloc(sizeof(sb2_quant_spec)));
    SB2_CUDA(b, cudaMemsetAsync(b->api_spec.ptr, 0, sizeof(sb2_quant_spec), b->stream));
    b->api_spec_host = sb2_quant_spec{};
    b->packed_spec = b->api_spec.as<sb2_quant_spec>();  // the packed gradients start as zeros
    SB2_CUDA(b, b->candidates.alloc(sizeof(FeatureCandidate) * 2 * kSplits * std::max<size_t>(F, 1)));
    SB2_CUDA(b, b->cand_flags.alloc(2 * kSplits * std::max<size_t>(F, 1)));
    SB2_CUDA(b, b->cand_gain.alloc(sizeof(double) * 2 * kSplits * std::max<size_t>(F, 1)));
    SB2_CUDA(b, b->maxima.alloc(2 * sizeof(unsigned long long)));
    SB2_CUDA(b, b->grid_barrier.alloc(2 * sizeof(unsigned int)));
    SB2_CUDA(b, cudaMemsetAsync(b->grid_barrier.ptr, 0, 2 * sizeof(unsigned int), b->stream));
    unsigned int bad_bins = 0;
    SB2_CUDA(b, cudaMemcpyAsync(&bad_bins, b->counter.ptr, sizeof(unsigned int), cudaMemcpyDeviceToHost, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->counter.ptr, 0, sizeof(unsigned int), b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->iter.ptr, 0, sizeof(IterState), b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->scores.ptr, 0, sizeof(float) * n, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->grad.ptr, 0, sizeof(float) * n, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->hess.ptr, 0, sizeof(float) * n, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->packed.ptr, 0, sizeof(int32_t) * n, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->label.ptr, train->label, sizeof(float) * n, cudaMemcpyHostToDevice, b->stream));
    if (b->weighted)
        SB2_CUDA(b, cudaMemcpyAsync(b->weight.ptr, train->weight, sizeof(float) * n, cudaMemcpyHostToDevice, b->stream));
    b->api_used.assign(F, 1);
    b->api_used_all = true;
    SB2_TRY(b->sync());
    // Every bin inside its feature's bins: the histogram's shared slots rely on it.
    if (bad_bins) return b->fail(SB2_EDATA, "a bin lies outside its feature's bins");
    b->loaded = true;
    return SB2_OK;
}

int sb2_init_scores(sb2_backend* b, int dataset, double value) {
    SB2_TRY(b->check_loaded());
    if (dataset != 0) return b->fail(SB2_EDEVICE, "no dataset " + std::to_string(dataset));
    launch_fill(b->scores.as<float>(), b->num_rows, static_cast<float>(value), b->stream);
    SB2_CUDA(b, cudaGetLastError());
    return b->sync();
}

int sb2_compute_gradients(sb2_backend* b, sb2_gradient_stats* out) {
    SB2_TRY(b->check_loaded());
    SB2_CUDA(b, cudaMemsetAsync(b->maxima.ptr, 0, 2 * sizeof(unsigned long long), b->stream));
    launch_api_gradients(b->row_args(), b->maxima.as<unsigned long long>(), b->row_grid(), b->stream);
    SB2_CUDA(b, cudaGetLastError());
    unsigned long long bits[2];
    SB2_CUDA(b, cudaMemcpyAsync(bits, b->maxima.ptr, sizeof(bits), cudaMemcpyDeviceToHost, b->stream));
    SB2_TRY(b->sync());
    std::memcpy(&out->max_abs_grad, &bits[0], 8);
    std::memcpy(&out->max_hess, &bits[1], 8);
    return SB2_OK;
}

int sb2_quantize(sb2_backend* b, const sb2_quant_spec* spec) {
    SB2_TRY(b->check_loaded());
    if (!spec) return b->fail(SB2_EDEVICE, "null quantization spec");
    // The histograms bound their packed sums by the spec the packed gradients came from.
    b->api_spec_host = *spec;
    SB2_CUDA(b, cudaMemcpyAsync(b->api_spec.ptr, spec, sizeof(sb2_quant_spec), cudaMemcpyHostToDevice, b->stream));
    b->packed_spec = b->api_spec.as<sb2_quant_spec>();
    launch_api_quantize(b->row_args(), *spec, b->row_grid(), b->stream);
    SB2_CUDA(b, cudaGetLastError());
    return b->sync();
}

int sb2_reset_partition(sb2_backend* b, const sb2_bag_spec* bag, uint32_t* out_rows) {
    SB2_TRY(b->check_loaded());
    launch_api_iota(b->rows[0].as<uint32_t>(), b->ordered[0].as<int32_t>(), b->packed.as<int32_t>(), b->num_rows,
                    b->row_grid(), b->stream);
    SB2_CUDA(b, cudaGetLastError());
    if (bag->kind == 0) {
        *out_rows = static_cast<uint32_t>(b->num_rows);
        return b->sync();
    }
    Step st{};
    st.active = 1;
    st.begin = 0;
    st.count = static_cast<uint32_t>(b->num_rows);
    st.which = 0;
    st.bag = 1;
    st.bag_seed = bag->seed;
    st.bag_round = bag->round;
    st.bag_fraction = bag->fraction;
    st.row_offset = b->row_offset;
    if (b->tiles.empty()) return b->fail(SB2_EUNSUPPORTED, "bagging a dataset without features");
    return run_partition(b, st, out_rows);
}

int sb2_set_histogram_features(sb2_backend* b, const uint8_t* used, size_t num_features) {
    SB2_TRY(b->check_loaded());
    if (num_features != b->num_features) return b->fail(SB2_EDEVICE, "feature mask of the wrong length");
    b->api_used.assign(used, used + num_features);
    b->api_used_all = std::all_of(b->api_used.begin(), b->api_used.end(), [](uint8_t u) { return u != 0; });
    SB2_CUDA(b, cudaMemcpyAsync(b->api_active.ptr, b->api_used.data(), num_features, cudaMemcpyHostToDevice, b->stream));
    return b->sync();
}

int sb2_histogram(sb2_backend* b, sb2_leaf_range leaf, int quantized, double* out, size_t len) {
    SB2_TRY(b->check_loaded());
    if (!quantized) return b->fail(SB2_EUNSUPPORTED, "float histograms: the device path is quantized only");
    SB2_TRY(b->check_range(leaf));
    return run_histogram(b, leaf, out, len);
}

int sb2_partition(sb2_backend* b, sb2_leaf_range leaf, const sb2_bin_split* split, uint32_t* out_left) {
    SB2_TRY(b->check_loaded());
    SB2_TRY(b->check_range(leaf));
    int32_t f;
    SB2_TRY(split_feature_of(b, *split, f));
    Step st{};
    st.active = 1;
    st.begin = leaf.begin;
    st.count = leaf.count;
    st.which = 0;
    st.split_tile = static_cast<uint32_t>(std::max(b->dev_features[f].tile, 0));
    st.split_lane = static_cast<uint32_t>(std::max(b->dev_features[f].lane, 0));
    std::memcpy(st.left_bins, split->left_bins, sizeof(st.left_bins));
    if (leaf.count == 0) {
        *out_left = 0;
        return SB2_OK;
    }
    if (b->dev_features[f].tile < 0) return b->fail(SB2_EDEVICE, "split on a trivial feature");
    return run_partition(b, st, out_left);
}

int sb2_partition_and_histogram(sb2_backend* b, sb2_leaf_range leaf, const sb2_bin_split* split, int side,
                                int quantized, double* out, size_t len, uint32_t* out_left) {
    if (!quantized) return b->fail(SB2_EUNSUPPORTED, "float histograms: the device path is quantized only");
    SB2_TRY(sb2_partition(b, leaf, split, out_left));
    sb2_leaf_range child = side == SB2_LEFT ? sb2_leaf_range{leaf.begin, *out_left}
                                            : sb2_leaf_range{leaf.begin + *out_left, leaf.count - *out_left};
    return run_histogram(b, child, out, len);
}

int sb2_leaf_sums(sb2_backend* b, const sb2_leaf_range* leaves, size_t num_leaves, float grad_scale,
                  float hess_scale, int64_t* out) {
    SB2_TRY(b->check_loaded());
    for (size_t i = 0; i < num_leaves; ++i) SB2_TRY(b->check_range(leaves[i]));
    DeviceBuffer ranges, sums;
    SB2_CUDA(b, ranges.alloc(sizeof(sb2_leaf_range) * std::max<size_t>(num_leaves, 1)));
    SB2_CUDA(b, sums.alloc(sizeof(int64_t) * 2 * std::max<size_t>(num_leaves, 1)));
    SB2_CUDA(b, cudaMemcpyAsync(ranges.ptr, leaves, sizeof(sb2_leaf_range) * num_leaves, cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(sums.ptr, 0, sums.bytes, b->stream));
    launch_api_leaf_sums(b->row_args(), b->rows[0].as<uint32_t>(), ranges.as<sb2_leaf_range>(),
                         static_cast<uint32_t>(num_leaves), grad_scale, hess_scale, sums.as<int64_t>(), b->sms * 2,
                         b->stream);
    SB2_CUDA(b, cudaGetLastError());
    SB2_CUDA(b, cudaMemcpyAsync(out, sums.ptr, sizeof(int64_t) * 2 * num_leaves, cudaMemcpyDeviceToHost, b->stream));
    return b->sync();
}

int sb2_add_tree(sb2_backend* b, const sb2_device_node* nodes, size_t num_nodes, const float* leaf_values,
                 size_t num_leaves) {
    SB2_TRY(b->check_loaded());
    if (num_leaves == 0 || num_leaves != num_nodes + 1)
        return b->fail(SB2_EDEVICE, "tree with " + std::to_string(num_nodes) + " nodes and " +
                                        std::to_string(num_leaves) + " leaves");
    std::vector<TileNode> tn(num_nodes);
    for (size_t k = 0; k < num_nodes; ++k) {
        int32_t f;
        SB2_TRY(split_feature_of(b, nodes[k].split, f));
        if (b->dev_features[f].tile < 0) return b->fail(SB2_EDEVICE, "malformed device tree");
        for (int32_t c : {nodes[k].left, nodes[k].right}) {
            bool ok = c >= 0 ? (static_cast<size_t>(c) > k && static_cast<size_t>(c) < num_nodes)
                             : (static_cast<size_t>(~c) < num_leaves);
            if (!ok) return b->fail(SB2_EDEVICE, "malformed device tree");
        }
        tn[k].tile = static_cast<uint32_t>(b->dev_features[f].tile);
        tn[k].lane = static_cast<uint32_t>(b->dev_features[f].lane);
        std::memcpy(tn[k].left_bins, nodes[k].split.left_bins, sizeof(tn[k].left_bins));
        // The tiles store the feature's bins 0 and mfb exchanged: so do the node's bits.
        const uint32_t mfb = b->dev_features[f].mfb & 0xFFu;
        if (mfb != 0) {
            const uint32_t b0 = tn[k].left_bins[0] & 1u, bm = (tn[k].left_bins[mfb >> 5] >> (mfb & 31)) & 1u;
            tn[k].left_bins[0] = (tn[k].left_bins[0] & ~1u) | bm;
            tn[k].left_bins[mfb >> 5] = (tn[k].left_bins[mfb >> 5] & ~(1u << (mfb & 31))) | (b0 << (mfb & 31));
        }
        tn[k].left = nodes[k].left;
        tn[k].right = nodes[k].right;
    }
    DeviceBuffer dn, dv;
    SB2_CUDA(b, dn.alloc(sizeof(TileNode) * std::max<size_t>(num_nodes, 1)));
    SB2_CUDA(b, dv.alloc(sizeof(float) * num_leaves));
    SB2_CUDA(b, cudaMemcpyAsync(dn.ptr, tn.data(), sizeof(TileNode) * num_nodes, cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(dv.ptr, leaf_values, sizeof(float) * num_leaves, cudaMemcpyHostToDevice, b->stream));
    launch_api_add_tree(b->dev_data(), b->row_args(), dn.as<TileNode>(), static_cast<uint32_t>(num_nodes),
                        dv.as<float>(), b->row_grid(), b->stream);
    SB2_CUDA(b, cudaGetLastError());
    return b->sync();
}

int sb2_scores(sb2_backend* b, int dataset, float* out, size_t len) {
    SB2_TRY(b->check_loaded());
    if (dataset != 0) return b->fail(SB2_EDEVICE, "no dataset " + std::to_string(dataset));
    if (len != b->num_rows) return b->fail(SB2_EDEVICE, "scores buffer of the wrong length");
    SB2_CUDA(b, cudaMemcpyAsync(out, b->scores.ptr, sizeof(float) * len, cudaMemcpyDeviceToHost, b->stream));
    return b->sync();
}

int sb2_read_partition(sb2_backend* b, uint32_t* out, size_t len) {
    SB2_TRY(b->check_loaded());
    if (len > b->num_rows) return b->fail(SB2_EDEVICE, "partition read past its rows");
    SB2_CUDA(b, cudaMemcpyAsync(out, b->rows[0].ptr, sizeof(uint32_t) * len, cudaMemcpyDeviceToHost, b->stream));
    return b->sync();
}

int sb2_read_packed(sb2_backend* b, int32_t* out, size_t len) {
    SB2_TRY(b->check_loaded());
    if (len != b->num_rows) return b->fail(SB2_EDEVICE, "packed buffer of the wrong length");
    SB2_CUDA(b, cudaMemcpyAsync(out, b->packed.ptr, sizeof(int32_t) * len, cudaMemcpyDeviceToHost, b->stream));
    return b->sync();
}

int sb2_write_gradients(sb2_backend* b, const float* grad, const float* hess, size_t len) {
    SB2_TRY(b->check_loaded());
    if (len != b->num_rows) return b->fail(SB2_EDEVICE, "gradient buffers of the wrong length");
    SB2_CUDA(b, cudaMemcpyAsync(b->grad.ptr, grad, sizeof(float) * len, cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(b->hess.ptr, hess, sizeof(float) * len, cudaMemcpyHostToDevice, b->stream));
    return b->sync();
}

int sb2_read_gradients(sb2_backend* b, float* grad, float* hess, size_t len) {
    SB2_TRY(b->check_loaded());
    if (len != b->num_rows) return b->fail(SB2_EDEVICE, "gradient buffers of the wrong length");
    SB2_CUDA(b, cudaMemcpyAsync(grad, b->grad.ptr, sizeof(float) * len, cudaMemcpyDeviceToHost, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(hess, b->hess.ptr, sizeof(float) * len, cudaMemcpyDeviceToHost, b->stream));
    return b->sync();
}

int sb2_find_best_split(sb2_backend* b, const double* hist, size_t len, const uint8_t* evaluate, double sum_grad,
                        double sum_hess, int64_t count, double grad_scale, double hess_scale,
                        const sb2_split_config* cfg, sb2_split_info* out, uint8_t* splittable) {
    SB2_TRY(b->check_loaded());
    if (len != 2ull * b->total_bins) return b->fail(SB2_EDEVICE, "histogram of the wrong length");
    std::vector<int> ih(len);
    for (size_t i = 0; i < len; ++i) {
        if (hist[i] != std::floor(hist[i]) || std::fabs(hist[i]) > 2147483647.0)
            return b->fail(SB2_EUNSUPPORTED, "the device split search takes integer (quantized) histograms");
        ih[i] = static_cast<int>(hist[i]);
    }
    DeviceBuffer dh, de, dout, dspl;
    SB2_CUDA(b, dh.alloc(sizeof(int) * len));
    SB2_CUDA(b, de.alloc(std::max<size_t>(b->num_features, 1)));
    SB2_CUDA(b, dout.alloc(sizeof(sb2_split_info)));
    SB2_CUDA(b, dspl.alloc(std::max<size_t>(b->num_features, 1)));
    SB2_CUDA(b, cudaMemcpyAsync(dh.ptr, ih.data(), sizeof(int) * len, cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(de.ptr, evaluate, b->num_features, cudaMemcpyHostToDevice, b->stream));
    launch_api_find_split(b->dev_data(), dh.as<int>(), de.as<uint8_t>(), sum_grad, sum_hess, count, grad_scale,
                          hess_scale, *cfg, b->candidates.ptr, b->counter.as<unsigned int>(), dout.as<sb2_split_info>(),
                          dspl.as<uint8_t>(), b->search_grid(), b->stream);
    SB2_CUDA(b, cudaGetLastError());
    SB2_CUDA(b, cudaMemcpyAsync(out, dout.ptr, sizeof(sb2_split_info), cudaMemcpyDeviceToHost, b->stream));
    SB2_CUDA(b, cudaMemcpyAsync(splittable, dspl.ptr, b->num_features, cudaMemcpyDeviceToHost, b->stream));
    return b->sync();
}

}  // extern "C"

// ---- the split search without allocation ---------------------------------------------------------------------
//
// sb2_find_best_split copies its inputs into device buffers it allocates for the call. Some callers cannot let a
// call allocate: a serving or training loop whose memory belongs to another allocator (a caching allocator that
// holds nearly all of HBM, where a fresh cudaMalloc fails), a loop on other streams that cudaMalloc/cudaFree would
// stall (they synchronize the device), or code that budgets its device memory up front. For them
// sb2_find_best_split_noalloc takes device buffers the caller owns and runs the same search kernel with its scratch
// (one candidate per feature and a CTA arrival counter) in a fixed array of this library's module, sized for
// kNoAllocMaxFeatures features.
namespace {

constexpr uint32_t kNoAllocMaxFeatures = 4096;
constexpr size_t kNoAllocCounterBytes = 256;  // the arrival counter, padded so the candidates stay 256-aligned
constexpr size_t kNoAllocScratchBytes = kNoAllocCounterBytes + sizeof(FeatureCandidate) * kNoAllocMaxFeatures;
// [0, 4): the counter, which must be zero when a launch starts (each call clears it); then the candidates.
static __device__ __align__(256) unsigned char g_noalloc_split_scratch[kNoAllocScratchBytes];

// The scratch's device address on b's device, looked up with that device current by the handle's first call and kept
// in the handle: a handle made after a device reset (cudaDeviceReset ends every handle's memory) looks it up again.
int noalloc_split_scratch(sb2_backend* b, unsigned char** out) {
    if (b->noalloc_scratch == nullptr) {
        void* p = nullptr;
        SB2_CUDA(b, cudaGetSymbolAddress(&p, g_noalloc_split_scratch));
        b->noalloc_scratch = p;
    }
    *out = static_cast<unsigned char*>(b->noalloc_scratch);
    return SB2_OK;
}

// SB2_OK when `p` is memory of b's device (device or managed); what the search reads and writes must be.
int check_device_pointer(sb2_backend* b, const void* p, const char* what) {
    if (p == nullptr) return b->fail(SB2_EDEVICE, std::string("sb2_find_best_split_noalloc: null ") + what);
    cudaPointerAttributes attr{};
    cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError();  // clear it: the pointer is the caller's mistake, not a device error
        return b->fail(SB2_EDEVICE, std::string("sb2_find_best_split_noalloc: ") + what + " is not a CUDA pointer");
    }
    const bool on_device = attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
    if (!on_device || attr.device != b->device)
        return b->fail(SB2_EDEVICE, std::string("sb2_find_best_split_noalloc: ") + what + " is not memory of device " +
                                        std::to_string(b->device));
    return SB2_OK;
}

}  // namespace

extern "C" {

int sb2_find_best_split_noalloc(sb2_backend* b, const int32_t* hist, size_t len, const uint8_t* evaluate,
                                double sum_grad, double sum_hess, int64_t count, double grad_scale,
                                double hess_scale, const sb2_split_config* cfg, sb2_split_info* out,
                                uint8_t* splittable) {
    if (!b) return SB2_EDEVICE;
    SB2_TRY(b->check_loaded());
    if (!cfg) return b->fail(SB2_EDEVICE, "sb2_find_best_split_noalloc: null split config");
    if (len != 2ull * b->total_bins) return b->fail(SB2_EDEVICE, "histogram of the wrong length");
    if (b->num_features > kNoAllocMaxFeatures)
        return b->fail(SB2_EUNSUPPORTED, "sb2_find_best_split_noalloc: the dataset has " +
                                             std::to_string(b->num_features) + " features, its scratch holds " +
                                             std::to_string(kNoAllocMaxFeatures) + " (use sb2_find_best_split)");
    SB2_CUDA(b, cudaSetDevice(b->device));
    SB2_TRY(check_device_pointer(b, hist, "histogram"));
    SB2_TRY(check_device_pointer(b, evaluate, "evaluate flags"));
    SB2_TRY(check_device_pointer(b, out, "split output"));
    SB2_TRY(check_device_pointer(b, splittable, "splittable flags"));
    unsigned char* scratch = nullptr;
    SB2_TRY(noalloc_split_scratch(b, &scratch));
    unsigned int* counter = reinterpret_cast<unsigned int*>(scratch);
    SB2_CUDA(b, cudaMemsetAsync(counter, 0, sizeof(unsigned int), b->stream));
    launch_api_find_split(b->dev_data(), hist, evaluate, sum_grad, sum_hess, count, grad_scale, hess_scale, *cfg,
                          scratch + kNoAllocCounterBytes, counter, out, splittable, b->search_grid(), b->stream);
    SB2_CUDA(b, cudaGetLastError());
    return b->sync();
}

int sb2_check_division(sb2_backend* b, uint64_t count, uint32_t seed, uint64_t* mismatches) {
    if (!b || !mismatches) return SB2_EDEVICE;
    SB2_CUDA(b, cudaSetDevice(b->device));
    DeviceBuffer d;
    SB2_CUDA(b, d.alloc(sizeof(unsigned long long)));
    SB2_CUDA(b, cudaMemsetAsync(d.ptr, 0, sizeof(unsigned long long), b->stream));
    launch_division_check(count, seed, d.as<unsigned long long>(), b->sms * 8, b->stream);
    SB2_CUDA(b, cudaGetLastError());
    unsigned long long n = 0;
    SB2_CUDA(b, cudaMemcpyAsync(&n, d.ptr, sizeof(n), cudaMemcpyDeviceToHost, b->stream));
    SB2_TRY(b->sync());
    *mismatches = n;
    return SB2_OK;
}

int sb2_time_histogram(sb2_backend* b, uint64_t rows, int repeats, double* seconds) {
    SB2_TRY(b->check_loaded());
    if (repeats < 1) return b->fail(SB2_EDEVICE, "repeats must be positive");
    if (rows == 0 || rows > b->num_rows) rows = b->num_rows;
    HistJob job{};
    job.active = 1;
    job.identity = 1;
    job.begin = 0;
    job.count = static_cast<uint32_t>(rows);
    job.which = 0;
    SB2_CUDA(b, cudaMemcpyAsync(b->hist_job.ptr, &job, sizeof(job), cudaMemcpyHostToDevice, b->stream));
    const HistArgs h = b->hist_args(nullptr, b->staging.as<int>());
    const size_t staging_bytes = sizeof(int) * (2ull * b->total_bins + 2);
    std::vector<cudaEvent_t> ev(2 * repeats);
    for (auto& e : ev) SB2_CUDA(b, cudaEventCreate(&e));
    // One untimed launch, then each timed launch between its own pair of events.
    SB2_CUDA(b, cudaMemsetAsync(b->staging.ptr, 0, staging_bytes, b->stream));
    b->run_hist(h, b->stream);
    for (int i = 0; i < repeats; ++i) {
        cudaMemsetAsync(b->staging.ptr, 0, staging_bytes, b->stream);
        cudaEventRecord(ev[2 * i], b->stream);
        b->run_hist(h, b->stream);
        cudaEventRecord(ev[2 * i + 1], b->stream);
    }
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    double total = 0.0;
    for (int i = 0; i < repeats && e == cudaSuccess; ++i) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ev[2 * i], ev[2 * i + 1]);
        total += ms / 1000.0;
    }
    for (auto& x : ev) cudaEventDestroy(x);
    SB2_CUDA(b, e);
    *seconds = total / repeats;
    return SB2_OK;
}

int sb2_time_shared_adds(sb2_backend* b, int pattern, double* adds_per_second, double* adds_per_sm_clock) {
    if (!b || !adds_per_second || !adds_per_sm_clock) return SB2_EDEVICE;
    if (pattern != 0 && pattern != 1) return b->fail(SB2_EDEVICE, "sb2_time_shared_adds: pattern must be 0 or 1");
    SB2_CUDA(b, cudaSetDevice(b->device));
    double adds = 0.0, cycles = 0.0, seconds = 0.0;
    SB2_CUDA(b, time_shared_adds(pattern, b->sms, 64, b->stream, &adds, &cycles, &seconds));
    *adds_per_second = seconds > 0.0 ? adds / seconds : 0.0;
    *adds_per_sm_clock = cycles > 0.0 ? adds / cycles : 0.0;  // cycles summed over the CTAs, one CTA per SM
    return SB2_OK;
}

}  // extern "C"

namespace {
int setup_exchange(sb2_backend* b);  // below, with the trainer
}  // namespace

extern "C" {

int sb2_nccl_unique_id(uint8_t* out, size_t len) {
    if (len < sizeof(ncclUniqueId)) {
        g_global_error = "NCCL unique id buffer smaller than 128 bytes";
        return SB2_ECOLLECTIVE;
    }
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) {
        g_global_error = std::string("ncclGetUniqueId: ") + ncclGetErrorString(r);
        return SB2_ECOLLECTIVE;
    }
    std::memcpy(out, &id, sizeof(id));
    return SB2_OK;
}

int sb2_set_rank_exchange(sb2_backend* b, int mode) {
    if (!b) return SB2_EDEVICE;
    if (mode != SB2_EXCHANGE_AUTO && mode != SB2_EXCHANGE_NCCL)
        return b->fail(SB2_ECONFIG, "unknown rank exchange mode " + std::to_string(mode));
    if (b->comm) return b->fail(SB2_ECONFIG, "the rank exchange is chosen before sb2_join_ranks");
    b->exchange_mode = mode;
    return SB2_OK;
}

int sb2_set_dominant_share(sb2_backend* b, double share) {
    if (!b) return SB2_EDEVICE;
    if (!(share >= 0.0)) return b->fail(SB2_ECONFIG, "the dominant-bin share must be at least 0");
    b->dominant_share = share;
    return SB2_OK;
}

int sb2_test_unanswered_peer(sb2_backend* b, uint32_t spin_limit) {
    if (!b) return SB2_EDEVICE;
    SB2_TRY(b->check_loaded());
    SB2_CUDA(b, cudaSetDevice(b->device));
    SB2_TRY(b->sync());
    if (b->comm) return b->fail(SB2_ECONFIG, "sb2_test_unanswered_peer on a handle that joined ranks");
    b->close_exchange();
    SB2_CUDA(b, b->fake_xbuf.alloc(0));
    SB2_CUDA(b, b->xbuf.alloc(0));
    if (spin_limit == 0) return SB2_OK;  // back to one rank
    if (!b->grow_ok) return b->fail(SB2_EUNSUPPORTED, "the tree kernel does not fit this dataset");
    const size_t need = exchange_bytes(b->num_features, 2);
    SB2_CUDA(b, b->xbuf.alloc(need));
    SB2_CUDA(b, b->fake_xbuf.alloc(need));
    SB2_CUDA(b, cudaMemsetAsync(b->xbuf.ptr, 0, need, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->fake_xbuf.ptr, 0, need, b->stream));
    SB2_TRY(b->sync());
    b->xpeers[0] = b->xbuf.ptr;
    b->xpeers[1] = b->fake_xbuf.ptr;
    b->xbytes = need;
    b->xepoch = 0;
    b->fake_peer = true;
    b->peer_spins = spin_limit;
    return SB2_OK;
}

int sb2_join_ranks(sb2_backend* b, const uint8_t* unique_id, size_t len, int world, int rank) {
    if (len < sizeof(ncclUniqueId)) return b->fail(SB2_ECOLLECTIVE, "NCCL unique id shorter than 128 bytes");
    if (world < 1 || rank < 0 || rank >= world) return b->fail(SB2_ECOLLECTIVE, "bad rank or world size");
    SB2_CUDA(b, cudaSetDevice(b->device));
    if (b->comm) {
        ncclCommDestroy(b->comm);
        b->comm = nullptr;
    }
    b->close_exchange();
    b->world = world;
    b->rank = rank;
    if (world == 1) return SB2_OK;
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    SB2_TRY(nccl_status(b, ncclCommInitRank(&b->comm, world, id, rank), "ncclCommInitRank"));
    // With the training set loaded, the tree kernel's exchange (every rank's buffer mapped here) is set up now, as
    // part of joining; otherwise the first training run does it.
    return b->loaded ? setup_exchange(b) : SB2_OK;
}

}  // extern "C"

// ---- device-resident training ------------------------------------------------------------------------------

namespace {

struct TrainBuffers {
    DeviceBuffer leaves, leaf_gain, splittable, evaluate, masks, slots, tree_bufs, leaf_sums, leaf_values, records,
        record_bufs, cursors, leaf_of_row, prep, prep_split;
};

// Carves DevTree arrays for `count` trees of `L` leaves out of one buffer.
int carve_tree(sb2_backend* b, DeviceBuffer& buf, size_t count, size_t L, DevTree& t) {
    const size_t sizes[] = {4, 4, 4, 1, 4, 4, 8, 8, 8, 8, 8, 8, 4, 4, 32};  // bytes per entry of each array below
    size_t total = (sizeof(int32_t) * count + 255) / 256 * 256;
    for (size_t s : sizes) total += (s * count * L + 255) / 256 * 256;
    SB2_CUDA(b, buf.alloc(total));
    char* p = buf.as<char>();
    auto take = [&](size_t bytes) {
        char* q = p;
        p += (bytes + 255) / 256 * 256;
        return q;
    };
    const size_t n = count * L;
    t.num_leaves = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * count));
    t.split_feature = reinterpret_cast<int32_t*>(take(4 * n));
    t.split_gain = reinterpret_cast<float*>(take(4 * n));
    t.threshold_bin = reinterpret_cast<uint32_t*>(take(4 * n));
    t.decision_type = reinterpret_cast<int8_t*>(take(n));
    t.left_child = reinterpret_cast<int32_t*>(take(4 * n));
    t.right_child = reinterpret_cast<int32_t*>(take(4 * n));
    t.internal_value = reinterpret_cast<double*>(take(8 * n));
    t.internal_weight = reinterpret_cast<double*>(take(8 * n));
    t.internal_count = reinterpret_cast<int64_t*>(take(8 * n));
    t.leaf_value = reinterpret_cast<double*>(take(8 * n));
    t.leaf_weight = reinterpret_cast<double*>(take(8 * n));
    t.leaf_count = reinterpret_cast<int64_t*>(take(8 * n));
    t.leaf_parent = reinterpret_cast<int32_t*>(take(4 * n));
    t.leaf_depth = reinterpret_cast<int32_t*>(take(4 * n));
    t.cat_bins = reinterpret_cast<uint32_t*>(take(32 * n));
    if (static_cast<size_t>(p - buf.as<char>()) > buf.bytes) return b->fail(SB2_EINTERNAL, "tree buffer overrun");
    return SB2_OK;
}

template <class T>
int download(sb2_backend* b, std::vector<T>& v, const T* src, size_t n) {
    v.resize(n);
    if (n == 0) return SB2_OK;
    return b->cuda(cudaMemcpyAsync(v.data(), src, sizeof(T) * n, cudaMemcpyDeviceToHost, b->stream), "download");
}

// The operations of an iteration, as sb2_profile_train reports them (the reference's per-op `Timed` backend,
// crates/silvic-core/tests/train_cpu.rs:434-484, on the device).
enum Op { kOpGradients, kOpQuantize, kOpHistogram, kOpPartition, kOpSearch, kOpLeafSums, kOpFinalize, kOpAddTree,
          kOpCollective, kOpTree, kOpCount };

// CUDA events around each operation of one iteration (graph-free profiling runs only).
struct OpTimer {
    struct Mark {
        int op;
        cudaEvent_t start, stop;
    };
    std::vector<Mark> marks;
    void begin(int op, cudaStream_t s) {
        Mark m{op, nullptr, nullptr};
        cudaEventCreate(&m.start);
        cudaEventCreate(&m.stop);
        cudaEventRecord(m.start, s);
        marks.push_back(m);
    }
    void end(cudaStream_t s) { cudaEventRecord(marks.back().stop, s); }
    void release() {
        for (auto& m : marks) {
            cudaEventDestroy(m.start);
            cudaEventDestroy(m.stop);
        }
        marks.clear();
    }
};

// One boosting iteration's launches (the body the CUDA graph captures); `timer` brackets each operation, and
// `tree_marks` (optional) the persistent tree kernel.
int enqueue_iteration(sb2_backend* b, const IterArgs& ia, int max_leaves, OpTimer* timer,
                      const cudaEvent_t* tree_marks = nullptr) {
    cudaStream_t s = b->stream;
    const TrainArgs& t = ia.t;
    const int row_grid = b->row_grid();
    auto op = [&](int kind, auto&& launch) -> int {
        if (timer) timer->begin(kind, s);
        int st = launch();
        if (timer) timer->end(s);
        return st;
    };
    const size_t staging_len = 2ull * b->total_bins + 2;
    auto reduce_histogram = [&]() -> int {
        if (!b->comm) return SB2_OK;
        return op(kOpCollective, [&] {
            return nccl_status(b, ncclAllReduce(t.staging, t.staging, staging_len, ncclInt32, ncclSum, b->comm, s),
                               "ncclAllReduce(histogram)");
        });
    };
    HistArgs h = b->hist_args(t.evaluate, t.staging);
    h.job = t.hist_job;
    SB2_TRY(op(kOpGradients, [&] { launch_gradients(ia, row_grid, s); return SB2_OK; }));
    if (b->comm)
        SB2_TRY(op(kOpCollective, [&] {
            return nccl_status(b, ncclAllReduce(&t.iter->max_abs_grad_bits, &t.iter->max_abs_grad_bits, 2,
                                                ncclUint64, ncclMax, b->comm, s),
                               "ncclAllReduce(max)");
        }));
    SB2_TRY(op(kOpQuantize, [&] { launch_iteration_start(ia, row_grid, s); return SB2_OK; }));
    if (b->persistent()) {
        // One launch grows the whole tree (grow.cu); ranks sum the root's units first and exchange the rest inside.
        GrowExchange x{};
        x.world = b->fake_peer ? 2 : b->comm ? b->world : 1;
        x.rank = b->comm ? b->rank : 0;
        x.spin_limit = b->peer_spins;
        if (x.world > 1) {
            for (int r = 0; r < x.world; ++r) x.peers[r] = static_cast<uint8_t*>(b->xpeers[r]);
            x.epoch0 = b->xepoch;
            b->xepoch += static_cast<uint32_t>(max_leaves) + 2;
        }
        if (b->comm) {
            SB2_TRY(op(kOpCollective, [&] {
                return nccl_status(b, ncclAllReduce(t.iter->root_units, t.iter->root_units, 2, ncclUint64, ncclSum,
                                                    b->comm, s),
                                   "ncclAllReduce(root units)");
            }));
        }
        SB2_TRY(op(kOpTree, [&] {
            if (tree_marks) cudaEventRecord(tree_marks[0], s);
            const int st = b->cuda(launch_grow_tree(t, h, b->grid_barrier.as<unsigned int>(), b->hist_grid,
                                                    b->grow_smem, x, s,
                                                    timer ? b->phase_ns.as<unsigned long long>() : nullptr,
                                                    timer ? max_leaves : 0),
                                   "cudaLaunchCooperativeKernel(grow_tree)");
            if (tree_marks) cudaEventRecord(tree_marks[1], s);
            return st;
        }));
        max_leaves = 1;  // no separate split steps
    } else {
        SB2_TRY(op(kOpHistogram, [&] { b->run_hist(h, s); return SB2_OK; }));
        SB2_TRY(reduce_histogram());
        SB2_TRY(op(kOpSearch, [&] { launch_search(t, b->search_grid(), s); return SB2_OK; }));
    }
    for (int step = 0; step + 1 < max_leaves; ++step) {
        SB2_TRY(op(kOpPartition, [&] {
            launch_partition_flags(t, b->partition_grid(), s);
            launch_partition_scatter(t, b->partition_grid(), s);
            return SB2_OK;
        }));
        SB2_TRY(op(kOpHistogram, [&] { b->run_hist(h, s); return SB2_OK; }));
        SB2_TRY(reduce_histogram());
        SB2_TRY(op(kOpSearch, [&] { launch_search(t, b->search_grid(), s); return SB2_OK; }));
    }
    SB2_TRY(op(kOpLeafSums, [&] { launch_leaf_sums(ia, row_grid, s); return SB2_OK; }));
    if (b->comm)
        SB2_TRY(op(kOpCollective, [&] {
            return nccl_status(b, ncclAllReduce(ia.leaf_sums, ia.leaf_sums, 2ull * t.max_leaves, ncclInt64, ncclSum,
                                                b->comm, s),
                               "ncclAllReduce(leaf sums)");
        }));
    SB2_TRY(op(kOpFinalize, [&] { launch_finalize(ia, s); return SB2_OK; }));
    SB2_TRY(op(kOpAddTree, [&] { launch_add_tree_partition(ia, row_grid, s); return SB2_OK; }));
    return b->cuda(cudaGetLastError(), "launch");
}

}  // namespace

namespace {

// A training run's device state and launch arguments.
struct Training {
    TrainBuffers tb;
    IterArgs ia{};
    DevTree rec{};
    int L = 0;
    int iters = 0;
};

// The tree kernel's exchange with the other ranks (GrowExchange). Collective: every rank calls it, with the same
// dataset shape. A rank that cannot take part (no cooperative tree kernel, more than kMaxRanks ranks, an IPC
// mapping refused) makes every rank keep the per-step launches with NCCL.
int setup_exchange(sb2_backend* b) {
    if (!b->comm || b->world <= 1) return SB2_OK;
    const size_t need = exchange_bytes(b->num_features, static_cast<uint32_t>(b->world));
    if (b->xready && b->xbytes == need) return SB2_OK;
    b->close_exchange();
    int ok = b->grow_ok && b->world <= kMaxRanks && b->exchange_mode == SB2_EXCHANGE_AUTO ? 1 : 0;
    cudaIpcMemHandle_t mine{};
    if (ok)
        ok = b->xbuf.alloc(need) == cudaSuccess && cudaMemset(b->xbuf.ptr, 0, need) == cudaSuccess &&
             cudaIpcGetMemHandle(&mine, b->xbuf.ptr) == cudaSuccess;
    cudaGetLastError();
    // Every rank's handle (in-place all-gather), then whether every rank mapped every other rank's buffer.
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    DeviceBuffer hs;
    SB2_CUDA(b, hs.alloc(hb * b->world + sizeof(int)));
    SB2_CUDA(b, cudaMemcpyAsync(hs.as<char>() + hb * b->rank, &mine, hb, cudaMemcpyHostToDevice, b->stream));
    SB2_TRY(nccl_status(b, ncclAllGather(hs.as<char>() + hb * b->rank, hs.ptr, hb, ncclUint8, b->comm, b->stream),
                        "ncclAllGather(exchange handles)"));
    std::vector<cudaIpcMemHandle_t> handles(b->world);
    SB2_CUDA(b, cudaMemcpyAsync(handles.data(), hs.ptr, hb * b->world, cudaMemcpyDeviceToHost, b->stream));
    SB2_TRY(b->sync());
    for (int r = 0; r < b->world && ok; ++r) {
        if (r == b->rank) continue;
        if (cudaIpcOpenMemHandle(&b->xpeers[r], handles[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            b->xpeers[r] = nullptr;
            ok = 0;
            cudaGetLastError();
        }
    }
    int* agree = reinterpret_cast<int*>(hs.as<char>() + hb * b->world);
    SB2_CUDA(b, cudaMemcpyAsync(agree, &ok, sizeof(int), cudaMemcpyHostToDevice, b->stream));
    SB2_TRY(nccl_status(b, ncclAllReduce(agree, agree, 1, ncclInt32, ncclMin, b->comm, b->stream),
                        "ncclAllReduce(exchange ready)"));
    int all = 0;
    SB2_CUDA(b, cudaMemcpyAsync(&all, agree, sizeof(int), cudaMemcpyDeviceToHost, b->stream));
    SB2_TRY(b->sync());
    if (!all) {
        b->close_exchange();
        return SB2_OK;
    }
    b->xpeers[b->rank] = b->xbuf.ptr;
    b->xready = true;
    b->xbytes = need;
    b->xepoch = 0;
    return SB2_OK;
}

int setup_training(sb2_backend* b, const sb2_params* p, double init_score, Training& tr) {
    SB2_TRY(b->check_loaded());
    SB2_CUDA(b, cudaSetDevice(b->device));
    SB2_TRY(setup_exchange(b));
    if (p->objective != b->objective.kind) return b->fail(SB2_ECONFIG, "params objective differs from the loaded one");
    if (p->objective == SB2_LAMBDARANK &&
        (p->sigmoid != b->objective.sigmoid || (p->lambdarank_norm != 0) != (b->ranking.norm != 0) ||
         p->lambdarank_truncation_level != b->objective.lambdarank_truncation_level ||
         label_gains(p->label_gain, p->num_label_gain) != b->rank_gain))
        return b->fail(SB2_ECONFIG, "lambdarank parameters differ from the loaded objective's");
    if (!p->use_quantized_grad) return b->fail(SB2_EUNSUPPORTED, "the device trainer is quantized only");
    if (p->bagging_fraction < 1.0 && p->bagging_freq > 0)
        return b->fail(SB2_EUNSUPPORTED, "bagging in the device trainer");
    if (p->num_leaves < 2 || p->num_leaves > 1024)
        return b->fail(SB2_ECONFIG, "num_leaves must be in 2..=1024 on the device");
    if (p->num_grad_quant_bins < 2 || p->num_grad_quant_bins > 64)
        return b->fail(SB2_ECONFIG, "num_grad_quant_bins must be in 2..=64");
    if (p->num_iterations < 0) return b->fail(SB2_ECONFIG, "negative num_iterations");
    const uint64_t total_rows = b->num_rows;  // single rank; ranks add theirs below
    int64_t global_rows = static_cast<int64_t>(total_rows);
    const int L = p->num_leaves;
    const int iters = p->num_iterations;
    const uint32_t F = b->num_features;
    if (static_cast<double>(b->num_rows) * b->world * std::max(p->num_grad_quant_bins, 1) >= 2147483647.0)
        return b->fail(SB2_EUNSUPPORTED, "int32 histograms would overflow: rows * quant bins >= 2^31");
    tr.L = L;
    tr.iters = iters;
    // Each iteration quantizes into the iteration state's spec; the histograms bound their sums by it.
    b->packed_spec = &b->iter.as<IterState>()->spec;
    TrainBuffers& tb = tr.tb;
    SB2_CUDA(b, tb.leaves.alloc(sizeof(DevLeaf) * L));
    SB2_CUDA(b, tb.leaf_gain.alloc(sizeof(double) * L));
    SB2_CUDA(b, tb.cursors.alloc(sizeof(unsigned int) * 2 * kSplits * (static_cast<size_t>(L) + 1)));
    SB2_CUDA(b, tb.splittable.alloc(static_cast<size_t>(L) * std::max<uint32_t>(F, 1)));
    SB2_CUDA(b, tb.evaluate.alloc(std::max<uint32_t>(F, 1)));
    SB2_CUDA(b, tb.masks.alloc(static_cast<size_t>(std::max(iters, 1)) * std::max<uint32_t>(F, 1)));
    // one slot per leaf, then the tree kernel's two prepared slots per leaf, and its records of dropped splits
    SB2_CUDA(b, tb.slots.alloc(sizeof(int) * 3 * static_cast<size_t>(L) * 2 * b->total_bins));
    SB2_CUDA(b, tb.prep.alloc(sizeof(PrepSplit) * L));
    SB2_CUDA(b, tb.prep_split.alloc(2 * static_cast<size_t>(L) * std::max<uint32_t>(F, 1)));
    SB2_CUDA(b, tb.leaf_sums.alloc(sizeof(int64_t) * 2 * L));
    SB2_CUDA(b, tb.leaf_values.alloc(sizeof(float) * L));
    SB2_CUDA(b, tb.leaf_of_row.alloc(sizeof(uint16_t) * std::max<uint64_t>(b->num_rows, 1)));
    SB2_CUDA(b, tb.records.alloc(sizeof(TreeRecordHeader) * std::max(iters, 1)));
    DevTree work{};
    DevTree& rec = tr.rec;
    SB2_TRY(carve_tree(b, tb.tree_bufs, 1, L, work));
    SB2_TRY(carve_tree(b, tb.record_bufs, std::max(iters, 1), L, rec));
    std::vector<uint8_t> masks(static_cast<size_t>(std::max(iters, 1)) * F);
    for (int i = 0; i < iters; ++i)
        feature_mask(b->features, p->feature_fraction, p->feature_fraction_seed, static_cast<uint32_t>(i),
                     masks.data() + static_cast<size_t>(i) * F);
    SB2_CUDA(b, cudaMemcpyAsync(tb.masks.ptr, masks.data(), masks.size(), cudaMemcpyHostToDevice, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(tb.leaves.ptr, 0, tb.leaves.bytes, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(tb.splittable.ptr, 0, tb.splittable.bytes, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(tb.records.ptr, 0, tb.records.bytes, b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->iter.ptr, 0, sizeof(IterState), b->stream));
    SB2_CUDA(b, cudaMemsetAsync(b->counter.ptr, 0, sizeof(unsigned int), b->stream));
    if (b->comm) {
        DeviceBuffer cnt;
        SB2_CUDA(b, cnt.alloc(sizeof(int64_t)));
        SB2_CUDA(b, cudaMemcpyAsync(cnt.ptr, &global_rows, sizeof(int64_t), cudaMemcpyHostToDevice, b->stream));
        SB2_TRY(nccl_status(b, ncclAllReduce(cnt.ptr, cnt.ptr, 1, ncclInt64, ncclSum, b->comm, b->stream),
                            "ncclAllReduce(rows)"));
        SB2_CUDA(b, cudaMemcpyAsync(&global_rows, cnt.ptr, sizeof(int64_t), cudaMemcpyDeviceToHost, b->stream));
        SB2_TRY(b->sync());
    }
    // Scores start at the initial score (Backend::init_scores).
    SB2_TRY(sb2_init_scores(b, 0, init_score));

    IterArgs& ia = tr.ia;
    TrainArgs& t = ia.t;
    t = b->api_train_args();
    t.cfg.min_data_in_leaf = p->min_data_in_leaf;
    t.cfg.min_sum_hessian_in_leaf = p->min_sum_hessian_in_leaf;
    t.cfg.lambda_l1 = p->lambda_l1;
    t.cfg.lambda_l2 = p->lambda_l2;
    t.cfg.min_gain_to_split = p->min_gain_to_split;
    t.cfg.min_data_per_group = p->min_data_per_group;
    t.cfg.cat_l2 = p->cat_l2;
    t.cfg.cat_smooth = p->cat_smooth;
    t.cfg.max_cat_to_onehot = p->max_cat_to_onehot;
    t.cfg.max_cat_threshold = p->max_cat_threshold;
    t.max_leaves = L;
    t.max_depth = p->max_depth;
    t.sums_feature = -1;
    for (uint32_t f = 0; f < F; ++f)
        if (b->features[f].num_bins != 0) {
            t.sums_feature = static_cast<int32_t>(f);
            break;
        }
    t.root_from_rows = b->persistent() ? 1 : 0;  // one GPU: the root's sums straight from the rows
    t.num_iterations = iters;
    t.leaves = tb.leaves.as<DevLeaf>();
    t.leaf_gain = tb.leaf_gain.as<double>();
    t.cursors = tb.cursors.as<unsigned int>();
    t.splittable = tb.splittable.as<uint8_t>();
    t.evaluate = tb.evaluate.as<uint8_t>();
    t.masks = tb.masks.as<uint8_t>();
    t.slots = tb.slots.as<int>();
    t.prep = tb.prep.as<PrepSplit>();
    t.prep_split = tb.prep_split.as<uint8_t>();
    t.tree = work;
    ia.r = b->row_args();
    ia.k.num_grad_quant_bins = p->num_grad_quant_bins;
    ia.k.stochastic = p->stochastic_rounding;
    ia.k.seed = p->data_random_seed;
    ia.k.constant_hessian = (p->objective == SB2_REGRESSION && !b->weighted) ? 1 : 0;
    ia.k.renew = p->quant_train_renew_leaf;
    ia.k.learning_rate = p->learning_rate;
    ia.k.init_score = init_score;
    ia.k.total_rows = global_rows;
    ia.leaf_sums = tb.leaf_sums.as<int64_t>();
    ia.leaf_values_f32 = tb.leaf_values.as<float>();
    ia.leaf_of_row = tb.leaf_of_row.as<uint16_t>();
    ia.records = tb.records.as<TreeRecordHeader>();
    ia.record_tree = rec;
    return SB2_OK;
}

// The trees of a finished run, read back into a host model.
int collect_model(sb2_backend* b, Training& tr, std::unique_ptr<sb2_model>& model) {
    const int L = tr.L;
    const DevTree& rec = tr.rec;
    TrainBuffers& tb = tr.tb;
    IterState it{};
    SB2_CUDA(b, cudaMemcpy(&it, b->iter.ptr, sizeof(it), cudaMemcpyDeviceToHost));
    if (it.error == 4) return b->fail(SB2_ECOLLECTIVE, "a rank did not reach a split step's exchange in time");
    if (it.error == 3) return b->fail(SB2_EINTERNAL, "a CTA of the tree kernel did not reach a grid barrier in time");
    if (it.error) return b->fail(SB2_EINTERNAL, "internal error " + std::to_string(it.error) + " at leaf " +
                                                    std::to_string(it.error_info));
    std::vector<TreeRecordHeader> heads;
    SB2_TRY(download(b, heads, tb.records.as<TreeRecordHeader>(), static_cast<size_t>(it.trees)));
    const size_t n = static_cast<size_t>(it.trees) * L;
    std::vector<int32_t> sf, lc, rc;
    std::vector<float> sg;
    std::vector<uint32_t> tbin;
    std::vector<int8_t> dt;
    std::vector<double> iv, iw, lv, lw;
    std::vector<int64_t> ic, lcnt;
    std::vector<uint32_t> cb;
    SB2_TRY(download(b, cb, rec.cat_bins, 8 * n));
    SB2_TRY(download(b, sf, rec.split_feature, n));
    SB2_TRY(download(b, sg, rec.split_gain, n));
    SB2_TRY(download(b, tbin, rec.threshold_bin, n));
    SB2_TRY(download(b, dt, rec.decision_type, n));
    SB2_TRY(download(b, lc, rec.left_child, n));
    SB2_TRY(download(b, rc, rec.right_child, n));
    SB2_TRY(download(b, iv, rec.internal_value, n));
    SB2_TRY(download(b, iw, rec.internal_weight, n));
    SB2_TRY(download(b, ic, rec.internal_count, n));
    SB2_TRY(download(b, lv, rec.leaf_value, n));
    SB2_TRY(download(b, lw, rec.leaf_weight, n));
    SB2_TRY(download(b, lcnt, rec.leaf_count, n));
    SB2_TRY(b->sync());
    for (int k = 0; k < it.trees; ++k) {
        HostTree ht;
        const size_t o = static_cast<size_t>(k) * L;
        const int nl = heads[k].num_leaves;
        ht.num_leaves = nl;
        ht.shrinkage = heads[k].shrinkage;
        int32_t num_cat = 0;
        for (int j = 0; j + 1 < nl; ++j) {
            const int32_t f = sf[o + j];
            ht.split_feature.push_back(f);
            ht.split_gain.push_back(sg[o + j]);
            ht.threshold_bin.push_back(tbin[o + j]);
            ht.cat_bins.insert(ht.cat_bins.end(), cb.begin() + 8 * (o + j), cb.begin() + 8 * (o + j + 1));
            if (dt[o + j] & 1) {
                // Tree::split_categorical (tree.rs:125-141): the split's index among the tree's categorical splits
                ht.threshold.push_back(static_cast<double>(num_cat++));
            } else {
                // apply_split (learner.rs:470-475): the bin's upper bound, f64::MAX for the +inf bound.
                double bound = b->upper_bounds[f].at(tbin[o + j]);
                ht.threshold.push_back(std::isfinite(bound) ? bound : std::numeric_limits<double>::max());
            }
            ht.decision_type.push_back(dt[o + j]);
            ht.left_child.push_back(lc[o + j]);
            ht.right_child.push_back(rc[o + j]);
            ht.internal_value.push_back(iv[o + j]);
            ht.internal_weight.push_back(iw[o + j]);
            ht.internal_count.push_back(ic[o + j]);
        }
        for (int j = 0; j < nl; ++j) {
            ht.leaf_value.push_back(lv[o + j]);
            ht.leaf_weight.push_back(lw[o + j]);
            ht.leaf_count.push_back(lcnt[o + j]);
        }
        model->trees.push_back(std::move(ht));
    }
    return SB2_OK;
}

}  // namespace

extern "C" {

int sb2_train(sb2_backend* b, const sb2_params* p, double init_score, sb2_model** out) {
    if (!b || !p || !out) return SB2_EDEVICE;
    Training tr;
    SB2_TRY(setup_training(b, p, init_score, tr));
    const int L = tr.L, iters = tr.iters;
    // Single GPU: each iteration is a handful of launches, the tree one persistent kernel. With NCCL ranks: one
    // iteration (about four launches per split) captured as a graph and replayed. CUDA events time each iteration.
    cudaGraphExec_t exec = nullptr;
    cudaError_t ce = cudaSuccess;
    if (!b->persistent()) {
        cudaGraph_t graph = nullptr;
        SB2_CUDA(b, cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal));
        int st = enqueue_iteration(b, tr.ia, L, nullptr);
        ce = cudaStreamEndCapture(b->stream, &graph);
        if (st != SB2_OK) {
            if (graph) cudaGraphDestroy(graph);
            return st;
        }
        SB2_CUDA(b, ce);
        ce = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        SB2_CUDA(b, ce);
    }
    // events[0 .. iters]: iteration boundaries; then, single GPU, a pair per iteration around the tree kernel
    std::vector<cudaEvent_t> events(iters + 1 + (exec ? 0 : 2 * iters));
    for (auto& e : events) cudaEventCreate(&e);
    cudaEventRecord(events[0], b->stream);
    int launch_status = SB2_OK;
    for (int i = 0; i < iters; ++i) {
        if (exec) {
            ce = cudaGraphLaunch(exec, b->stream);
            if (ce != cudaSuccess) break;
        } else {
            launch_status = enqueue_iteration(b, tr.ia, L, nullptr, &events[iters + 1 + 2 * i]);
            if (launch_status != SB2_OK) break;
        }
        cudaEventRecord(events[i + 1], b->stream);
    }
    cudaError_t se = cudaStreamSynchronize(b->stream);
    if (exec) cudaGraphExecDestroy(exec);
    if (launch_status != SB2_OK) {
        for (auto& e : events) cudaEventDestroy(e);
        return launch_status;
    }
    auto model = std::make_unique<sb2_model>();
    if (ce == cudaSuccess && se == cudaSuccess) {
        for (int i = 0; i < iters; ++i) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, events[i], events[i + 1]);
            model->seconds.push_back(ms / 1000.0);
            if (!exec) {
                cudaEventElapsedTime(&ms, events[iters + 1 + 2 * i], events[iters + 2 + 2 * i]);
                model->tree_seconds.push_back(ms / 1000.0);
            }
        }
    }
    for (auto& e : events) cudaEventDestroy(e);
    SB2_CUDA(b, ce);
    SB2_CUDA(b, se);
    SB2_TRY(collect_model(b, tr, model));
    *out = model.release();
    return SB2_OK;
}

int sb2_boost_from_average(const sb2_params* p, const float* label, const float* weight, size_t n, double* out) {
    const double k_epsilon = static_cast<double>(1e-15f);
    *out = 0.0;
    if (!p->boost_from_average || p->objective == SB2_LAMBDARANK) return SB2_OK;
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(label[i])) {
            g_global_error = "label of row " + std::to_string(i) + " is not finite";
            return SB2_EDATA;
        }
    // [sum label * weight, sum weight] in row order; a binary label counts as 1 when positive.
    double l = 0.0, w = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const float y = p->objective == SB2_BINARY ? (label[i] > 0.0f ? 1.0f : 0.0f) : label[i];
        if (weight) {
            l += static_cast<double>(y * weight[i]);
            w += static_cast<double>(weight[i]);
        } else {
            l += static_cast<double>(y);
        }
    }
    if (!weight) w = static_cast<double>(n);
    double score;
    if (p->objective == SB2_BINARY) {
        double rate = std::min(std::max(l / w, k_epsilon), 1.0 - k_epsilon);
        score = std::log(rate / (1.0 - rate)) / p->sigmoid;
    } else {
        score = l / w;
    }
    // GBDT::BoostFromAverage drops an initial score indistinguishable from zero.
    *out = std::fabs(score) > k_epsilon ? score : 0.0;
    return SB2_OK;
}

}  // extern "C"

namespace {

// Training without the CUDA graph, each operation between CUDA events: `last` gets the last iteration's seconds per
// operation (kOpCount) and per phase of the tree kernel (kGrowPhases); `trace` its per-step rows (kStepTrace values,
// nanoseconds and row counts; empty when the tree kernel did not run).
int profile_run(sb2_backend* b, const sb2_params* p, double init_score, std::vector<double>& last,
                std::vector<unsigned long long>& trace, std::unique_ptr<sb2_model>& model) {
    Training tr;
    SB2_TRY(setup_training(b, p, init_score, tr));
    last.assign(kOpCount + kGrowPhases, 0.0);
    trace.clear();
    model = std::make_unique<sb2_model>();
    const size_t words = kGrowPhases + static_cast<size_t>(tr.L) * kStepTrace;
    SB2_CUDA(b, b->phase_ns.alloc(sizeof(unsigned long long) * words));
    for (int i = 0; i < tr.iters; ++i) {
        OpTimer timer;
        SB2_CUDA(b, cudaMemsetAsync(b->phase_ns.ptr, 0, b->phase_ns.bytes, b->stream));
        int st = enqueue_iteration(b, tr.ia, tr.L, &timer);
        cudaError_t se = cudaStreamSynchronize(b->stream);
        if (st == SB2_OK && se == cudaSuccess) {
            std::fill(last.begin(), last.end(), 0.0);
            double total = 0.0;
            for (auto& m : timer.marks) {
                float ms = 0.0f;
                cudaEventElapsedTime(&ms, m.start, m.stop);
                last[m.op] += ms / 1000.0;
                total += ms / 1000.0;
            }
            model->seconds.push_back(total);
            std::vector<unsigned long long> ns(words);
            SB2_CUDA(b, cudaMemcpy(ns.data(), b->phase_ns.ptr, sizeof(unsigned long long) * words,
                                   cudaMemcpyDeviceToHost));
            for (int k = 0; k < kGrowPhases; ++k) last[kOpCount + k] = ns[k] * 1e-9;
            if (b->persistent()) trace.assign(ns.begin() + kGrowPhases, ns.end());
        }
        timer.release();
        SB2_TRY(st);
        SB2_CUDA(b, se);
    }
    return collect_model(b, tr, model);
}

}  // namespace

extern "C" {

int sb2_profile_train(sb2_backend* b, const sb2_params* p, double init_score, double* seconds_by_op, size_t num_ops,
                      sb2_model** out) {
    if (!b || !p || !seconds_by_op) return SB2_EDEVICE;
    std::vector<double> last;
    std::vector<unsigned long long> trace;
    std::unique_ptr<sb2_model> model;
    SB2_TRY(profile_run(b, p, init_score, last, trace, model));
    for (size_t k = 0; k < num_ops && k < last.size(); ++k) seconds_by_op[k] = last[k];
    if (out) *out = model.release();
    return SB2_OK;
}

int sb2_profile_steps(sb2_backend* b, const sb2_params* p, double init_score, double* rows, size_t max_steps,
                      size_t* num_steps) {
    if (!b || !p || !rows || !num_steps) return SB2_EDEVICE;
    std::vector<double> last;
    std::vector<unsigned long long> trace;
    std::unique_ptr<sb2_model> model;
    SB2_TRY(profile_run(b, p, init_score, last, trace, model));
    if (trace.empty()) return b->fail(SB2_EUNSUPPORTED, "step traces come from the single-GPU tree kernel only");
    size_t steps = 0;  // the grid steps that ran: each ran at least one split
    while (steps < trace.size() / kStepTrace &&
           trace[steps * kStepTrace + kGrowPhases + 1] + trace[steps * kStepTrace + kGrowPhases + 3] > 0)
        ++steps;
    *num_steps = std::min(steps, max_steps);
    for (size_t s = 0; s < *num_steps; ++s)
        for (int k = 0; k < kStepTrace; ++k) {
            const double v = static_cast<double>(trace[s * kStepTrace + k]);
            rows[s * kStepTrace + k] = k < kGrowPhases ? v * 1e-9 : v;
        }
    return SB2_OK;
}

// data::binning::bin_rows on the device: see the header. Per chunk of rows (at most ~256 MB of values), the values
// (copied from the host when they live there) are binned group by group into a device buffer of the chunk's group
// rows, which is copied into the caller's group buffer.
int sb2_bin_dense(sb2_backend* b, const void* values, int value_bytes, uint64_t rows, uint32_t cols, int row_major,
                  const sb2_feature* features, uint32_t num_features, const sb2_group* groups, uint32_t num_groups,
                  uint8_t* const* group_data) {
    if (!b) return SB2_EDEVICE;
    SB2_CUDA(b, cudaSetDevice(b->device));
    if (value_bytes != 4 && value_bytes != 8) return b->fail(SB2_EDATA, "values must be f32 (4 bytes) or f64 (8)");
    if (rows == 0 || num_groups == 0) return SB2_OK;
    if (!values || !features || !groups || !group_data) return b->fail(SB2_EDATA, "a null buffer");
    // Per group: its features' matrix columns, byte columns, bounds and NaN bins, uploaded once.
    struct GroupPlan {
        DeviceBuffer meta, bounds, out;
        uint32_t nf = 0, total = 0;
    };
    std::vector<GroupPlan> plans(num_groups);
    for (uint32_t g = 0; g < num_groups; ++g) {
        const sb2_group& grp = groups[g];
        if (!group_data[g]) return b->fail(SB2_EDATA, "group " + std::to_string(g) + " has no output buffer");
        std::vector<uint32_t> feat, column, off{0};
        std::vector<uint8_t> nan, categorical;
        std::vector<double> bounds;
        for (uint32_t k = 0; k < grp.num_features; ++k) {
            const uint32_t f = grp.features[k];
            if (f >= num_features || f >= cols)
                return b->fail(SB2_EDATA, "group " + std::to_string(g) + " names feature " + std::to_string(f) +
                                              " beyond the matrix's columns");
            const sb2_feature& m = features[f];
            if (m.column >= grp.row_stride)
                return b->fail(SB2_EDATA, "feature " + std::to_string(f) + "'s column lies outside its group's rows");
            feat.push_back(f);
            column.push_back(m.column);
            if (m.kind == SB2_CATEGORICAL) {
                // categorical_bin (data/bin_mapper.rs:379-391): the categories ascending, then their bins
                if (!m.categories || m.num_categories == 0 || m.num_categories > 255 || m.num_bins != m.num_categories + 1)
                    return b->fail(SB2_EDATA, "categorical feature " + std::to_string(f) + " without 1..255 categories");
                std::vector<std::pair<int32_t, uint32_t>> sorted;
                for (uint32_t c = 0; c < m.num_categories; ++c) sorted.emplace_back(m.categories[c], c + 1);
                std::sort(sorted.begin(), sorted.end());
                for (size_t c = 1; c < sorted.size(); ++c)
                    if (sorted[c].first == sorted[c - 1].first)
                        return b->fail(SB2_EDATA, "categorical feature " + std::to_string(f) + " lists category " +
                                                      std::to_string(sorted[c].first) + " twice");
                for (const auto& e : sorted) bounds.push_back(static_cast<double>(e.first));
                for (const auto& e : sorted) bounds.push_back(static_cast<double>(e.second));
                off.push_back(static_cast<uint32_t>(bounds.size()));
                nan.push_back(0);
                categorical.push_back(1);
                continue;
            }
            if (m.kind != SB2_NUMERICAL || !m.upper_bounds || m.num_upper_bounds == 0 || m.num_upper_bounds > 256)
                return b->fail(SB2_EDATA, "grouped feature " + std::to_string(f) + " without 1..256 upper bounds");
            bounds.insert(bounds.end(), m.upper_bounds, m.upper_bounds + m.num_upper_bounds);
            off.push_back(static_cast<uint32_t>(bounds.size()));
            // value_to_bin(NaN) (bin_mapper.rs:347-352): the NaN bin, or the bin of 0.0
            uint32_t zero = 0;
            while (zero < m.num_upper_bounds && m.upper_bounds[zero] < 0.0) ++zero;
            nan.push_back(static_cast<uint8_t>(m.nan_bin ? m.num_upper_bounds : zero));
            categorical.push_back(0);
        }
        GroupPlan& p = plans[g];
        p.nf = static_cast<uint32_t>(feat.size());
        p.total = static_cast<uint32_t>(bounds.size());
        if (sizeof(double) * p.total > 200 * 1024)
            return b->fail(SB2_EUNSUPPORTED, "group " + std::to_string(g) + " has more bounds and categories than shared memory holds");
        // meta: feature [nf], column [nf], bound_off [nf + 1], nan [nf] (bytes), categorical [nf] (bytes)
        std::vector<uint8_t> meta(4 * (3 * p.nf + 1) + 2 * p.nf);
        std::memcpy(meta.data(), feat.data(), 4 * p.nf);
        std::memcpy(meta.data() + 4 * p.nf, column.data(), 4 * p.nf);
        std::memcpy(meta.data() + 8 * p.nf, off.data(), 4 * (p.nf + 1));
        std::memcpy(meta.data() + 4 * (3 * p.nf + 1), nan.data(), p.nf);
        std::memcpy(meta.data() + 4 * (3 * p.nf + 1) + p.nf, categorical.data(), p.nf);
        SB2_CUDA(b, p.meta.alloc(meta.size()));
        SB2_CUDA(b, p.bounds.alloc(sizeof(double) * std::max<uint32_t>(p.total, 1)));
        SB2_CUDA(b, cudaMemcpyAsync(p.meta.ptr, meta.data(), meta.size(), cudaMemcpyHostToDevice, b->stream));
        if (p.total)
            SB2_CUDA(b, cudaMemcpyAsync(p.bounds.ptr, bounds.data(), sizeof(double) * p.total, cudaMemcpyHostToDevice,
                                        b->stream));
        SB2_TRY(b->sync());  // the host vectors go out of scope
    }
    cudaPointerAttributes attr{};
    const bool on_device = cudaPointerGetAttributes(&attr, values) == cudaSuccess &&
                           (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged);
    cudaGetLastError();  // a host pointer may leave an error from the query
    // The kernels read device values in place, so they must live on the handle's own device: another GPU's memory
    // is not reachable without peer access, and is rejected before anything is launched.
    if (on_device && attr.device != b->device)
        return b->fail(SB2_EDATA, "sb2_bin_dense: the values are memory of device " + std::to_string(attr.device) +
                                      ", not of the handle's device " + std::to_string(b->device));
    const uint64_t row_bytes = static_cast<uint64_t>(cols) * value_bytes;
    uint64_t chunk = std::max<uint64_t>((256ull << 20) / std::max<uint64_t>(row_bytes, 1), 128) / 128 * 128;
    chunk = std::min(chunk, rows);
    DeviceBuffer staged;
    if (!on_device) SB2_CUDA(b, staged.alloc(chunk * row_bytes));
    for (uint32_t g = 0; g < num_groups; ++g) SB2_CUDA(b, plans[g].out.alloc(chunk * std::max<uint32_t>(groups[g].row_stride, 1)));
    for (uint64_t r0 = 0; r0 < rows; r0 += chunk) {
        const uint64_t n = std::min(chunk, rows - r0);
        BinGroupArgs a{};
        a.f64 = value_bytes == 8;
        a.row_major = row_major != 0;
        a.cols = cols;
        a.chunk_rows = n;
        if (on_device) {
            a.values = values;
            a.rows = rows;
            a.row0 = r0;
        } else {
            const uint8_t* src = static_cast<const uint8_t*>(values);
            if (row_major)
                SB2_CUDA(b, cudaMemcpyAsync(staged.ptr, src + r0 * row_bytes, n * row_bytes, cudaMemcpyHostToDevice, b->stream));
            else
                SB2_CUDA(b, cudaMemcpy2DAsync(staged.ptr, n * value_bytes, src + r0 * value_bytes, rows * value_bytes,
                                              n * value_bytes, cols, cudaMemcpyHostToDevice, b->stream));
            a.values = staged.ptr;
            a.rows = n;  // the staged column-major chunk's pitch
            a.row0 = 0;
        }
        for (uint32_t g = 0; g < num_groups; ++g) {
            GroupPlan& p = plans[g];
            const uint32_t stride = groups[g].row_stride;
            if (stride == 0) continue;
            const uint8_t* meta = p.meta.as<uint8_t>();
            a.num_features = p.nf;
            a.feature = reinterpret_cast<const uint32_t*>(meta);
            a.column = reinterpret_cast<const uint32_t*>(meta + 4 * p.nf);
            a.bound_off = reinterpret_cast<const uint32_t*>(meta + 8 * p.nf);
            a.nan_bin = meta + 4 * (3 * p.nf + 1);
            a.categorical = meta + 4 * (3 * p.nf + 1) + p.nf;
            a.bounds = p.bounds.as<double>();
            a.total_bounds = p.total;
            a.stride = stride;
            a.out = p.out.as<uint8_t>();
            SB2_CUDA(b, cudaMemsetAsync(p.out.ptr, 0, n * stride, b->stream));  // padding columns are 0
            SB2_CUDA(b, launch_bin_group(a, b->stream));
            SB2_CUDA(b, cudaMemcpyAsync(group_data[g] + r0 * stride, p.out.ptr, n * stride, cudaMemcpyDeviceToHost,
                                        b->stream));
        }
    }
    return b->sync();
}

int sb2_model_free(sb2_model* m) {
    delete m;
    return SB2_OK;
}

int sb2_model_num_trees(const sb2_model* m) { return static_cast<int>(m->trees.size()); }

int sb2_model_tree(const sb2_model* m, int index, sb2_tree_view* v) {
    if (index < 0 || static_cast<size_t>(index) >= m->trees.size()) return SB2_EDEVICE;
    const HostTree& t = m->trees[index];
    v->num_leaves = t.num_leaves;
    v->shrinkage = t.shrinkage;
    v->split_feature = t.split_feature.data();
    v->split_gain = t.split_gain.data();
    v->threshold = t.threshold.data();
    v->threshold_bin = t.threshold_bin.data();
    v->cat_bins = t.cat_bins.data();
    v->decision_type = t.decision_type.data();
    v->left_child = t.left_child.data();
    v->right_child = t.right_child.data();
    v->leaf_value = t.leaf_value.data();
    v->leaf_weight = t.leaf_weight.data();
    v->leaf_count = t.leaf_count.data();
    v->internal_value = t.internal_value.data();
    v->internal_weight = t.internal_weight.data();
    v->internal_count = t.internal_count.data();
    return SB2_OK;
}

int sb2_model_iteration_seconds(const sb2_model* m, double* out, size_t len) {
    size_t k = std::min(len, m->seconds.size());
    std::copy(m->seconds.begin(), m->seconds.begin() + k, out);
    return static_cast<int>(m->seconds.size());
}

int sb2_model_tree_seconds(const sb2_model* m, double* out, size_t len) {
    size_t k = std::min(len, m->tree_seconds.size());
    std::copy(m->tree_seconds.begin(), m->tree_seconds.begin() + k, out);
    return static_cast<int>(m->tree_seconds.size());
}

}  // extern "C"
