// ref_gpu.cu — test infrastructure, not part of the product: the reference's own GPU kernels on the same GPU. Its
// quantized histogram is the "existing GPU kernel" this build's histogram is measured against; its quantize,
// gradient, partition, bagging, leaf-sum and add-tree kernels give reference-produced outputs the CPU oracle is
// checked against.
//
// The kernel is silvic-gpu's `hist_quant` (crates/silvic-gpu/kernels/kernels.kern:473-559), compiled from the
// reference's kernel text as it lies (ref_gpu_source.sh assembles it into _ref/ref_kernels.cuh the way
// crates/silvic-gpu/src/params.rs:30-53 does for NVRTC). This file only drives it, with the reference's host-side
// set-up and launch math restated: the work units and column map (crates/silvic-gpu/src/backend.rs:376-424), the
// most frequent bin per column (:337-374), rows per block (:611-631) and the launch of `encode_histogram`
// (:901-951: the histogram zeroed, then one block of 1024 threads per row block and unit).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

#include "../include/silvic_b200.h"
#include "_ref/ref_kernels.cuh"

namespace {

constexpr uint32_t kThreads = 1024;         // HIST_THREADS (backend.rs:96)
constexpr uint32_t kTargetGroups = 1024;    // HIST_TARGET_GROUPS (backend.rs:99)
constexpr uint32_t kMinRowsPerBlock = 1024; // HIST_MIN_ROWS_PER_BLOCK (backend.rs:101)
constexpr uint32_t kMaxBins = HIST_QUANT_BINS;

std::string g_error;

struct RefHist {
    uint32_t rows = 0, total_bins = 0, units = 0, rows_per_block = 0;
    uint32_t *partition = nullptr, *bins = nullptr;
    int32_t *packed = nullptr, *col_map = nullptr, *hist = nullptr;
    uint32_t* left_total = nullptr;
    HistUnit* unit_buf = nullptr;
    ~RefHist() {
        cudaFree(partition);
        cudaFree(bins);
        cudaFree(packed);
        cudaFree(col_map);
        cudaFree(hist);
        cudaFree(left_total);
        cudaFree(unit_buf);
    }
};

int fail(const std::string& what, cudaError_t e = cudaSuccess) {
    g_error = what + (e == cudaSuccess ? "" : std::string(": ") + cudaGetErrorString(e));
    return 1;
}

}  // namespace

extern "C" {

const char* ref_gpu_last_error() { return g_error.c_str(); }

// Uploads `train` (every group's rows, as the reference stores them: 32-bit words of row-major group bytes) and the
// rows' packed gradients `packed` (num_rows values), and builds the units and column map. `rows_per_block_cap` is
// packed_block_rows of the quantization (backend.rs:622-632). Returns 0 and a handle in *out.
int ref_hist_create(const sb2_dataset* train, const int32_t* packed, uint32_t rows_per_block_cap, void** out) {
    auto h = new RefHist();
    const uint32_t n = static_cast<uint32_t>(train->num_rows);
    h->rows = n;
    h->total_bins = train->total_bins;
    std::vector<HistUnit> units;
    std::vector<int32_t> col_map;
    std::vector<uint32_t> words;
    uint64_t words_base = 0;
    for (uint32_t g = 0; g < train->num_groups; ++g) {
        const sb2_group& grp = train->groups[g];
        if (grp.row_stride % 4 != 0) {
            delete h;
            return fail("a group's row stride is not a whole number of 32-bit words");
        }
        // the most frequent bin of every column, the lowest of equally frequent ones (backend.rs:337-374)
        std::vector<uint8_t> mfb(grp.row_stride, 0);
        {
            std::vector<uint64_t> counts(static_cast<size_t>(grp.row_stride) * 256, 0);
            for (uint64_t r = 0; r < n; ++r)
                for (uint32_t c = 0; c < grp.row_stride; ++c) ++counts[c * 256 + grp.data[r * grp.row_stride + c]];
            for (uint32_t c = 0; c < grp.row_stride; ++c) {
                uint32_t best = 0;
                for (uint32_t b = 1; b < 256; ++b)
                    if (counts[c * 256 + b] > counts[c * 256 + best]) best = b;
                mfb[c] = static_cast<uint8_t>(best);
            }
        }
        // the group's features in bin order, split into runs of at most kMaxBins bins (backend.rs:378-424)
        std::vector<uint32_t> feats;
        for (uint32_t k = 0; k < grp.num_features; ++k)
            if (train->features[grp.features[k]].num_bins > 0) feats.push_back(grp.features[k]);
        std::sort(feats.begin(), feats.end(), [&](uint32_t a, uint32_t b) {
            return train->features[a].hist_offset < train->features[b].hist_offset;
        });
        for (size_t start = 0; start < feats.size();) {
            const uint32_t first = train->features[feats[start]].hist_offset;
            size_t end = start;
            uint32_t extent = 0;
            while (end < feats.size()) {
                const sb2_feature& m = train->features[feats[end]];
                const uint32_t next = m.hist_offset + m.num_bins - first;
                if (next > kMaxBins) break;
                extent = next;
                ++end;
            }
            if (end == start) {
                delete h;
                return fail("a feature has more bins than a histogram unit");
            }
            const uint32_t cols_begin = static_cast<uint32_t>(col_map.size());
            col_map.resize(cols_begin + grp.row_stride, -1);
            for (size_t i = start; i < end; ++i) {
                const sb2_feature& m = train->features[feats[i]];
                col_map[cols_begin + m.column] = static_cast<int32_t>((m.hist_offset - first) | (uint32_t(mfb[m.column]) << 16));
            }
            HistUnit u{};
            u.words_base_lo = static_cast<uint32_t>(words_base);
            u.words_base_hi = static_cast<uint32_t>(words_base >> 32);
            u.row_words = grp.row_stride / 4;
            u.bin_begin = first;
            u.num_bins = extent;
            u.cols_begin = cols_begin;
            units.push_back(u);
            start = end;
        }
        const size_t nw = static_cast<size_t>(n) * (grp.row_stride / 4);
        const size_t at = words.size();
        words.resize(at + nw);
        std::memcpy(words.data() + at, grp.data, nw * 4);
        words_base += nw;
    }
    h->units = static_cast<uint32_t>(units.size());
    // rows per block (backend.rs:617-620)
    const uint32_t blocks = (kTargetGroups + std::max(h->units, 1u) - 1) / std::max(h->units, 1u);
    h->rows_per_block = std::max(std::min(std::max((n + blocks - 1) / blocks, kMinRowsPerBlock), rows_per_block_cap), 1u);
    std::vector<uint32_t> iota(n);
    std::iota(iota.begin(), iota.end(), 0u);
    cudaError_t e = cudaSuccess;
    auto up = [&](auto** dst, const void* src, size_t bytes) {
        if (e != cudaSuccess) return;
        e = cudaMalloc(reinterpret_cast<void**>(dst), std::max<size_t>(bytes, 16));
        if (e == cudaSuccess && src) e = cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice);
    };
    up(&h->partition, iota.data(), 4ull * n);
    up(&h->packed, packed, 4ull * n);
    up(&h->bins, words.data(), 4ull * words.size());
    up(&h->col_map, col_map.data(), 4ull * col_map.size());
    up(&h->unit_buf, units.data(), sizeof(HistUnit) * units.size());
    up(&h->hist, nullptr, 8ull * h->total_bins);
    up(&h->left_total, nullptr, 16);
    if (e != cudaSuccess) {
        delete h;
        return fail("upload", e);
    }
    *out = h;
    return 0;
}

// The root histogram (every row) as the reference computes it (`encode_histogram` with side 0), `repeats` times
// after one untimed run; *seconds gets the mean of each run's CUDA-event time (zeroing + kernel), `out`
// (2 total_bins ints, may be null) the last histogram.
int ref_hist_run(void* handle, int repeats, double* seconds, int32_t* out) {
    RefHist* h = static_cast<RefHist*>(handle);
    HistParams p{};
    p.begin = 0;
    p.count = h->rows;
    p.rows_per_block = h->rows_per_block;
    p.side = 0;
    const dim3 grid((h->rows + h->rows_per_block - 1) / h->rows_per_block, h->units);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    double total = 0.0;
    for (int i = 0; i <= repeats; ++i) {
        cudaEventRecord(a);
        cudaMemsetAsync(h->hist, 0, 8ull * h->total_bins);
        hist_quant<<<grid, kThreads>>>(h->partition, h->packed, h->bins, h->unit_buf, h->col_map, h->hist,
                                       h->left_total, p);
        cudaEventRecord(b);
        cudaEventSynchronize(b);
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, a, b);
        if (i > 0) total += ms * 1e-3;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail("hist_quant", e);
    *seconds = repeats > 0 ? total / repeats : 0.0;
    if (out) {
        const cudaError_t c = cudaMemcpy(out, h->hist, 8ull * h->total_bins, cudaMemcpyDeviceToHost);
        if (c != cudaSuccess) return fail("download", c);
    }
    return 0;
}

void ref_hist_destroy(void* handle) { delete static_cast<RefHist*>(handle); }

}  // extern "C"

// ---- the reference's other training kernels -----------------------------------------------------------------
//
// Each function below uploads its inputs, launches the reference's kernel(s) with GpuBackend's launch math
// (crates/silvic-gpu/src/backend.rs) and downloads the result, so the tests can hold the CPU oracle (and this
// build's device path) against the reference's own GPU code on the same inputs.

namespace {

constexpr uint32_t kElementThreads = 256;        // ELEMENT_THREADS (backend.rs:86)
constexpr uint32_t kMaxGroups = 65535;           // MAX_GROUPS (backend.rs:84)
constexpr uint32_t kCompactChunk = 4096;         // COMPACT_CHUNK (backend.rs:91)
constexpr uint32_t kMaxCompactBlocks = 65536;    // MAX_COMPACT_BLOCKS (backend.rs:93)
constexpr uint32_t kLeafSumRows = REDUCE_THREADS * 16;  // LEAF_SUM_ROWS (backend.rs:106)

// groups_for (backend.rs:245-247)
uint32_t groups_for(uint32_t n, uint32_t threads) {
    return std::min(std::max((n + threads - 1) / threads, 1u), kMaxGroups);
}

// compact_chunk (backend.rs:611-614)
uint32_t compact_chunk(uint32_t count) {
    const uint32_t chunk = std::max((count + kMaxCompactBlocks - 1) / kMaxCompactBlocks, kCompactChunk);
    return (chunk + SCAN_THREADS - 1) / SCAN_THREADS * SCAN_THREADS;
}

// Device buffers freed on scope exit; `e` keeps the first failure.
struct Buffers {
    std::vector<void*> held;
    cudaError_t e = cudaSuccess;
    template <class T>
    T* make(size_t count, const void* src = nullptr) {
        void* p = nullptr;
        if (e == cudaSuccess) e = cudaMalloc(&p, std::max<size_t>(count * sizeof(T), 16));
        if (e == cudaSuccess) held.push_back(p);
        if (e == cudaSuccess && src) e = cudaMemcpy(p, src, count * sizeof(T), cudaMemcpyHostToDevice);
        if (e == cudaSuccess && !src) e = cudaMemset(p, 0, std::max<size_t>(count * sizeof(T), 16));
        return static_cast<T*>(p);
    }
    template <class T>
    void take(T* dst, const T* src, size_t count) {
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e == cudaSuccess && count) e = cudaMemcpy(dst, src, count * sizeof(T), cudaMemcpyDeviceToHost);
    }
    ~Buffers() {
        for (void* p : held) cudaFree(p);
    }
};

// Every group's row-major bins one after another, and their GroupLayout entries (the reference's DatasetBuffers).
void upload_bins(Buffers& bufs, const sb2_dataset* d, uint8_t** bins, GroupLayout** layouts) {
    std::vector<uint8_t> all;
    std::vector<GroupLayout> lay(d->num_groups);
    for (uint32_t g = 0; g < d->num_groups; ++g) {
        const uint64_t base = all.size();
        lay[g].base_lo = static_cast<uint32_t>(base);
        lay[g].base_hi = static_cast<uint32_t>(base >> 32);
        lay[g].row_stride = d->groups[g].row_stride;
        const size_t bytes = static_cast<size_t>(d->num_rows) * d->groups[g].row_stride;
        all.insert(all.end(), d->groups[g].data, d->groups[g].data + bytes);
    }
    *bins = bufs.make<uint8_t>(all.size(), all.data());
    *layouts = bufs.make<GroupLayout>(lay.size(), lay.data());
}

int done(Buffers& bufs, const char* what) {
    if (bufs.e == cudaSuccess) bufs.e = cudaDeviceSynchronize();
    return bufs.e == cudaSuccess ? 0 : fail(what, bufs.e);
}

}  // namespace

extern "C" {

// quantize (kernels.kern:309-319) as GpuBackend::quantize launches it (backend.rs:1170-1203).
int ref_quantize(const sb2_quant_spec* spec, const float* grad, const float* hess, uint32_t n, uint64_t row_offset,
                 int32_t* out) {
    Buffers b;
    float* dg = b.make<float>(n, grad);
    float* dh = b.make<float>(n, hess);
    int32_t* dq = b.make<int32_t>(n);
    QuantParams p{};
    p.n = n;
    p.row_offset_lo = static_cast<uint32_t>(row_offset);
    p.row_offset_hi = static_cast<uint32_t>(row_offset >> 32);
    p.inv_grad_scale = spec->inv_grad_scale;
    p.inv_hess_scale = spec->inv_hess_scale;
    p.grad_max_q = spec->grad_max_q;
    p.hess_max_q = spec->hess_max_q;
    p.constant_hessian = spec->constant_hessian ? 1u : 0u;
    p.stochastic = spec->stochastic ? 1u : 0u;
    p.seed = spec->seed;
    p.iteration = spec->iteration;
    if (b.e == cudaSuccess) quantize<<<groups_for(n, kElementThreads), kElementThreads>>>(dg, dh, dq, p);
    b.take(out, dq, n);
    return done(b, "quantize");
}

// grad_regression / grad_binary (kernels.kern:60-90) as pointwise_gradients launches them (backend.rs:668-691).
int ref_gradients(int objective, float sigmoid, const float* scores, const float* label, const float* weight,
                  uint32_t n, float* grad, float* hess) {
    Buffers b;
    float* ds = b.make<float>(n, scores);
    float* dl = b.make<float>(n, label);
    float* dw = b.make<float>(weight ? n : 1, weight);
    float* dg = b.make<float>(n);
    float* dh = b.make<float>(n);
    GradParams p{};
    p.n = n;
    p.has_weight = weight ? 1u : 0u;
    p.sigmoid = sigmoid;
    if (b.e == cudaSuccess) {
        if (objective == SB2_BINARY)
            grad_binary<<<groups_for(n, kElementThreads), kElementThreads>>>(ds, dl, dw, dg, dh, p);
        else
            grad_regression<<<groups_for(n, kElementThreads), kElementThreads>>>(ds, dl, dw, dg, dh, p);
    }
    b.take(grad, dg, n);
    b.take(hess, dh, n);
    return done(b, "gradients");
}

// The stable partition of positions [0, n) of `rows` by `split`: partition_count, scan_blocks, partition_scatter
// and copy_u32 (kernels.kern:346-435) as encode_partition launches them (backend.rs:999-1047). `out` receives the
// partitioned rows, *left the left count.
int ref_partition(const sb2_dataset* d, const uint32_t* rows, uint32_t n, const sb2_bin_split* split, uint32_t* out,
                  uint32_t* left) {
    Buffers b;
    uint8_t* bins = nullptr;
    GroupLayout* layouts = nullptr;
    upload_bins(b, d, &bins, &layouts);
    uint32_t* part = b.make<uint32_t>(n, rows);
    uint32_t* scratch = b.make<uint32_t>(n);
    uint8_t* flags = b.make<uint8_t>(n);
    uint32_t* counts = b.make<uint32_t>(kMaxCompactBlocks);
    uint32_t* total = b.make<uint32_t>(4);
    uint64_t base = 0;
    for (uint32_t g = 0; g < split->group; ++g) base += static_cast<uint64_t>(d->num_rows) * d->groups[g].row_stride;
    PartitionParams p{};
    p.begin = 0;
    p.count = n;
    p.chunk = compact_chunk(n);
    p.row_stride = d->groups[split->group].row_stride;
    p.group_base_lo = static_cast<uint32_t>(base);
    p.group_base_hi = static_cast<uint32_t>(base >> 32);
    p.column = split->column;
    std::memcpy(p.left_bins, split->left_bins, sizeof(p.left_bins));
    const uint32_t blocks = (n + p.chunk - 1) / p.chunk;
    ScanParams sp{};
    sp.n = blocks;
    CopyParams cp{};
    cp.begin = 0;
    cp.count = n;
    if (b.e == cudaSuccess && n > 0) {
        partition_count<<<blocks, SCAN_THREADS>>>(part, bins, counts, flags, p);
        scan_blocks<<<1, SCAN_THREADS>>>(counts, total, sp);
        partition_scatter<<<blocks, SCAN_THREADS>>>(part, flags, counts, total, scratch, p);
        copy_u32<<<groups_for(n, kElementThreads), kElementThreads>>>(scratch, part, cp);
    }
    b.take(out, part, n);
    b.take(left, total, 1);
    return done(b, "partition");
}

// Bernoulli bagging of n rows: bag_count, scan_blocks, bag_scatter (kernels.kern:330-389) as bernoulli_bag launches
// them (backend.rs:857-896). `out` (n rows) receives the bag, *count its size.
int ref_bag(uint32_t n, uint64_t row_offset, uint32_t seed, uint32_t round, double fraction, uint32_t* out,
            uint32_t* count) {
    Buffers b;
    uint32_t* part = b.make<uint32_t>(n);
    uint32_t* counts = b.make<uint32_t>(kMaxCompactBlocks);
    uint32_t* total = b.make<uint32_t>(4);
    BagParams p{};
    p.n = n;
    p.chunk = compact_chunk(n);
    p.row_offset_lo = static_cast<uint32_t>(row_offset);
    p.row_offset_hi = static_cast<uint32_t>(row_offset >> 32);
    p.seed = seed;
    p.round = round;
    // bag_threshold (backend.rs:1113-1123): ceil(fraction * 2^24)
    p.threshold = !(fraction > 0.0) ? 0u : fraction >= 1.0 ? 16777216u
                                                            : static_cast<uint32_t>(std::ceil(fraction * 16777216.0));
    const uint32_t blocks = (n + p.chunk - 1) / p.chunk;
    ScanParams sp{};
    sp.n = blocks;
    if (b.e == cudaSuccess && n > 0) {
        bag_count<<<blocks, SCAN_THREADS>>>(counts, p);
        scan_blocks<<<1, SCAN_THREADS>>>(counts, total, sp);
        bag_scatter<<<blocks, SCAN_THREADS>>>(counts, part, p);
    }
    b.take(count, total, 1);
    b.take(out, part, n);
    return done(b, "bag");
}

// leaf_sums (kernels.kern:660-688) with GpuBackend::leaf_sums' jobs of LEAF_SUM_ROWS positions and its host sum of
// each leaf's partials (backend.rs:1276-1330); `out` gets [g, h] per leaf.
int ref_leaf_sums(const float* grad, const float* hess, uint32_t n, const uint32_t* partition,
                  const sb2_leaf_range* leaves, uint32_t num_leaves, float grad_scale, float hess_scale, int64_t* out) {
    std::vector<uint32_t> jobs, per_leaf;
    for (uint32_t l = 0; l < num_leaves; ++l) {
        const uint32_t end = leaves[l].begin + leaves[l].count;
        uint32_t k = 0;
        for (uint32_t s = leaves[l].begin; s < end; s += kLeafSumRows, ++k) {
            jobs.push_back(s);
            jobs.push_back(std::min(s + kLeafSumRows, end));
        }
        per_leaf.push_back(k);
    }
    const uint32_t blocks = static_cast<uint32_t>(jobs.size() / 2);
    Buffers b;
    float* dg = b.make<float>(n, grad);
    float* dh = b.make<float>(n, hess);
    uint32_t* dp = b.make<uint32_t>(n, partition);
    uint32_t* dj = b.make<uint32_t>(jobs.size(), jobs.data());
    i64* partials = b.make<i64>(2ull * blocks);
    LeafSumParams p{};
    p.grad_scale = grad_scale;
    p.hess_scale = hess_scale;
    if (b.e == cudaSuccess && blocks > 0) leaf_sums<<<blocks, REDUCE_THREADS>>>(dp, dg, dh, dj, partials, p);
    std::vector<i64> host(2ull * blocks);
    b.take(host.data(), partials, host.size());
    size_t at = 0;
    for (uint32_t l = 0; l < num_leaves; ++l) {
        int64_t g = 0, h = 0;
        for (uint32_t k = 0; k < per_leaf[l]; ++k, ++at) {
            g += host[2 * at];
            h += host[2 * at + 1];
        }
        out[2 * l] = g;
        out[2 * l + 1] = h;
    }
    return done(b, "leaf_sums");
}

// add_tree (kernels.kern:693-705) as encode_add_tree launches it (backend.rs:790-811), with tree_nodes' node layout
// (:1081-1110); `scores` (num_rows) is updated in place.
int ref_add_tree(const sb2_dataset* d, const sb2_device_node* nodes, uint32_t num_nodes, const float* leaf_values,
                 uint32_t num_leaves, float* scores) {
    const uint32_t n = static_cast<uint32_t>(d->num_rows);
    std::vector<TreeNode> tn(num_nodes);
    for (uint32_t k = 0; k < num_nodes; ++k) {
        tn[k].group = nodes[k].split.group;
        tn[k].column = nodes[k].split.column;
        tn[k].left = nodes[k].left;
        tn[k].right = nodes[k].right;
        std::memcpy(tn[k].left_bins, nodes[k].split.left_bins, sizeof(tn[k].left_bins));
    }
    Buffers b;
    uint8_t* bins = nullptr;
    GroupLayout* layouts = nullptr;
    upload_bins(b, d, &bins, &layouts);
    TreeNode* dn = b.make<TreeNode>(std::max<uint32_t>(num_nodes, 1), tn.data());
    float* dv = b.make<float>(num_leaves, leaf_values);
    float* ds = b.make<float>(n, scores);
    TreeParams p{};
    p.n = n;
    p.num_nodes = num_nodes;
    if (b.e == cudaSuccess) add_tree<<<groups_for(n, kElementThreads), kElementThreads>>>(bins, layouts, dn, dv, ds, p);
    b.take(scores, ds, n);
    return done(b, "add_tree");
}

}  // extern "C"
