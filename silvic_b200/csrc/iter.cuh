// iter.cuh — per-iteration kernels of the boosting loop (boosting.rs:227-324) and the Backend-API kernels.
#pragma once

#include "train.cuh"

namespace sb2 {

// LambdaRank (objective/lambdarank.rs; ObjectiveSetup::LambdaRank, backend/mod.rs:58-71): the rank's queries and
// the tables the host computes once at load with the same libm calls as the reference (the sigmoid table's exp,
// the discounts' log2, the inverse max DCGs), so the device's pair arithmetic starts from the same values.
constexpr uint32_t kSigmoidBins = 1u << 20;   // lambdarank.rs:31
constexpr uint32_t kMaxQueryRows = 4096;      // longest query the device takes (its rows are sorted in shared memory)
struct RankArgs {
    const uint32_t* bounds;          // [num_queries + 1] row boundaries of the rank's queries
    const uint32_t* queries;         // [num_queries]: the short queries (a warp each), then the long ones (a CTA each)
    const double* inverse_max_dcg;   // [num_queries]
    const double* label_gain;        // [num_gain]
    const double* discount;          // [kMaxQueryRows]: 1 / log2(2 + rank)
    const double* table;             // [kSigmoidBins]: LightGBM's sigmoid table
    uint32_t num_queries;
    uint32_t num_short;              // queries of at most lambdarank_warp_rows() rows
    uint32_t cap;                    // a power of two >= the longest query (and >= 2): the CTA kernel's rows
    uint32_t truncation;             // lambdarank_truncation_level
    uint32_t num_gain;
    int32_t norm;                    // lambdarank_norm
    uint32_t warp_grid, cta_grid;    // CTAs of the two gradient launches
    double sigmoid, sigmoid_squared, min_input, max_input, idx_factor;
};

// The objective and the rows the gradient and score kernels read.
struct RowArgs {
    uint64_t num_rows;
    uint64_t row_offset;
    int32_t objective;   // SB2_REGRESSION / SB2_BINARY / SB2_LAMBDARANK
    int32_t pad_;
    double sigmoid;
    const float* label;
    const float* weight;  // nullptr when unweighted
    float* scores;
    float* grad;
    float* hess;
    int32_t* packed;
    RankArgs rank;        // lambdarank only
};

// Training constants of one run (Params subset) the iteration kernels need.
struct IterConsts {
    int32_t num_grad_quant_bins;
    int32_t stochastic;
    uint32_t seed;             // data_random_seed
    int32_t constant_hessian;  // objective::constant_hessian (objective/mod.rs:84-89)
    int32_t renew;             // quant_train_renew_leaf
    int32_t pad_;
    double learning_rate;
    double init_score;
    int64_t total_rows;        // rows over every rank (root count without bagging)
};

// A finished tree as the host reads it back (one per iteration).
struct TreeRecordHeader {
    int32_t num_leaves;
    int32_t iteration;
    double shrinkage;
};

struct IterArgs {
    TrainArgs t;
    RowArgs r;
    IterConsts k;
    int64_t* leaf_sums;          // [2 * max_leaves], reduced over ranks between leaf_sums and finalize
    float* leaf_values_f32;      // [max_leaves]: what add_tree adds
    uint16_t* leaf_of_row;       // [num_rows]: each row's leaf in the current tree (leaf_sums writes, add_tree reads)
    TreeRecordHeader* records;   // [num_iterations]
    DevTree record_tree;         // arrays [num_iterations * max_leaves]
};

// A device node of Backend::add_tree in tile coordinates.
struct TileNode {
    uint32_t tile, lane;
    uint32_t left_bins[8];
    int32_t left, right;
};

constexpr int kRowThreads = 256;

void launch_gradients(const IterArgs& a, int grid, cudaStream_t s);
// LambdaRank gradients of every query (lambdarank.cu) and their maxima (atomicMax of the f64 bits of |grad|, |hess|);
// nothing when `stopped` (may be null) is set. Queries of at most lambdarank_warp_rows() rows take a warp each, longer
// ones (up to kMaxQueryRows) a CTA each with lambdarank_smem(cap) bytes of dynamic shared memory.
size_t lambdarank_smem(uint32_t cap);
uint32_t lambdarank_warp_rows();
cudaError_t lambdarank_configure(uint32_t cap, int* warp_blocks_per_sm, int* cta_blocks_per_sm);
void launch_lambdarank(const RowArgs& r, const int32_t* stopped, unsigned long long* max_g, unsigned long long* max_h,
                       cudaStream_t s);
void launch_iteration_start(const IterArgs& a, int grid, cudaStream_t s);
void launch_leaf_sums(const IterArgs& a, int grid, cudaStream_t s);
void launch_finalize(const IterArgs& a, cudaStream_t s);
void launch_add_tree_partition(const IterArgs& a, int grid, cudaStream_t s);

// Backend API helpers
void launch_api_gradients(const RowArgs& r, unsigned long long* maxima_bits, int grid, cudaStream_t s);
void launch_api_quantize(const RowArgs& r, const sb2_quant_spec& spec, int grid, cudaStream_t s);
void launch_api_iota(uint32_t* rows, int32_t* ordered, const int32_t* packed, uint64_t n, int grid, cudaStream_t s);
void launch_api_leaf_sums(const RowArgs& r, const uint32_t* partition, const sb2_leaf_range* ranges, uint32_t num,
                          float gs, float hs, int64_t* out, int grid, cudaStream_t s);
void launch_api_add_tree(const DevData& d, const RowArgs& r, const TileNode* nodes, uint32_t num_nodes,
                         const float* leaf_values, int grid, cudaStream_t s);
void launch_fill(float* out, uint64_t n, float value, cudaStream_t s);
// Load: a group's columns into the feature-major copy (`col_feature`/`col_bins` per group column; a bin out of its
// feature's range sets `bad`), then, once every group is in, the tiles from the copy (whole 128-row blocks of each
// column: column_stride is the row count rounded up to 128).
void launch_group_columns(const uint8_t* src, uint64_t rows, uint32_t row_stride, const int32_t* col_feature,
                          const uint32_t* col_bins, uint8_t* columns, uint64_t column_stride, unsigned int* bad,
                          cudaStream_t s);
void launch_tiles(const DevData& d, uint8_t* bins, cudaStream_t s);
// Per column feats[k] of the feature-major copy, its rows per bin added into counts[k * 256 + bin] (zeroed first).
void launch_bin_counts(const uint8_t* columns, uint64_t column_stride, uint64_t rows, const int32_t* feats,
                       uint32_t num_feats, unsigned int* counts, cudaStream_t s);
// Counts the operand pairs where the split scan's division (div_rn) differs from CUDA's correctly rounded one.
void launch_division_check(uint64_t n, uint32_t seed, unsigned long long* mismatches, int grid, cudaStream_t s);
// diag.cu: `red.shared.add.u32` alone at the histogram's address patterns (0: every lane its own bins; 1: one bin
// per instruction), `ctas` CTAs of 512 threads; *adds lane adds made, *cycles SM clock cycles summed over the CTAs,
// *seconds the launch's duration.
cudaError_t time_shared_adds(int pattern, int ctas, uint32_t passes, cudaStream_t stream, double* adds, double* cycles,
                             double* seconds);
void launch_api_find_split(const DevData& d, const int* hist, const uint8_t* evaluate, double ug, double uh,
                           int64_t count, double gs, double hs, const sb2_split_config& cfg, void* cands,
                           unsigned int* counter, sb2_split_info* out, uint8_t* splittable, int grid, cudaStream_t s);

}  // namespace sb2
