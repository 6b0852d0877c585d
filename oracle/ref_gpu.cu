// ref_gpu.cu — test infrastructure, not part of the product: the reference's own quantized histogram kernel on the
// same GPU, the "existing GPU kernel" this build's histogram is measured against.
//
// The kernel is silvic-gpu's `hist_quant` (crates/silvic-gpu/kernels/kernels.kern:473-559), compiled from the
// reference's kernel text as it lies (ref_gpu_source.sh assembles it into _ref/ref_kernels.cuh the way
// crates/silvic-gpu/src/params.rs:30-53 does for NVRTC). This file only drives it, with the reference's host-side
// set-up and launch math restated: the work units and column map (crates/silvic-gpu/src/backend.rs:376-424), the
// most frequent bin per column (:337-374), rows per block (:611-631) and the launch of `encode_histogram`
// (:901-951: the histogram zeroed, then one block of 1024 threads per row block and unit).
#include <cuda_runtime.h>

#include <algorithm>
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
