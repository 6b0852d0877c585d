/*
 * silvic_b200.h — C ABI of the B200 (sm_100a) training backend for silvic.
 *
 * This header is the drop-in boundary. It mirrors silvic-core's device plugin API, `trait Backend`
 * (crates/silvic-core/src/backend/mod.rs:115-179), method by method, with flat C types in place of the Rust
 * structs. It also exports a device-resident trainer: the leaf-wise learner
 * (crates/silvic-core/src/learner.rs:121-404) and the boosting loop (crates/silvic-core/src/boosting.rs:227-324),
 * run on the GPU without host round trips per split.
 *
 * Conventions
 *  - Every function returns an int status: SB2_OK (0) or one of the SB2_E* codes below, which map the kinds of
 *    `SilvicError` (crates/silvic-core/src/error.rs:28-65). The message of the last failure on a handle is
 *    available through sb2_last_error(); failures without a handle (creation) through sb2_global_error().
 *  - Every pointer is a plain host pointer unless the name ends in `_dev` (device pointers, see the "kernel
 *    entry points" section).
 *  - A handle is not thread-safe: one thread at a time, as `&mut self` in Rust. Handles are independent.
 *  - Multi-GPU: one process per GPU. Each process creates its handle on its own device with the rank's
 *    contiguous row shard (`row_offset` = rows of lower ranks) and joins the ranks with sb2_join_ranks().
 *    Histogram reductions then run over NCCL inside the handle, so the caller's own Collective sees one rank.
 */
#ifndef SILVIC_B200_H
#define SILVIC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (SilvicError kinds) ---------------------------------------------------------------------- */
enum {
    SB2_OK = 0,
    SB2_ECONFIG = 1,      /* SilvicError::Config */
    SB2_EDATA = 2,        /* SilvicError::Data */
    SB2_EINTERNAL = 3,    /* SilvicError::Internal */
    SB2_EDEVICE = 4,      /* SilvicError::Device: CUDA failure, misuse, bad range or buffer length */
    SB2_ECOLLECTIVE = 5,  /* SilvicError::Collective: NCCL failure or timeout */
    SB2_EMODEL = 6,       /* SilvicError::Model */
    SB2_EUNSUPPORTED = 7, /* SilvicError::Unsupported */
};

/* ---- data types (mirrors of silvic-core structs) ----------------------------------------------------------- */

enum { SB2_NUMERICAL = 0, SB2_CATEGORICAL = 1, SB2_TRIVIAL = 2 };

/* FeatureMeta (crates/silvic-core/src/data/mod.rs:25-36) with its BinMapper (data/bin_mapper.rs:26-41). */
typedef struct sb2_feature {
    uint32_t num_bins;    /* bins in the histogram, NaN bin included; 0 for a trivial feature */
    uint32_t group;       /* the feature's group */
    uint32_t column;      /* byte offset of the feature in its group's row */
    uint32_t hist_offset; /* index of the feature's bin 0 in the flat histogram */
    uint32_t kind;        /* SB2_NUMERICAL / SB2_CATEGORICAL / SB2_TRIVIAL */
    uint32_t nan_bin;     /* numerical: the last bin holds NaN */
    const double* upper_bounds; /* numerical: ascending bin upper bounds, the last +inf */
    uint32_t num_upper_bounds;
    uint32_t pad_;
    double min_value, max_value; /* sampled min and max (feature_infos) */
    const int32_t* categories;   /* categorical: categories[b - 1] is bin b's category (bin 0: every other value);
                                    read by sb2_bin_dense only */
    uint32_t num_categories;     /* num_bins - 1 */
    uint32_t pad2_;
} sb2_feature;

/* FeatureGroup (crates/silvic-core/src/data/mod.rs:49-59): row-major bins, data[row * row_stride + column]. */
typedef struct sb2_group {
    const uint8_t* data;
    uint32_t row_stride;
    uint32_t hist_offset;
    uint32_t total_bins;
    uint32_t num_features;
    const uint32_t* features; /* indices into the feature array, in column order */
} sb2_group;

/* BinnedDataset (crates/silvic-core/src/data/mod.rs:62-74). The arrays are read during the call that takes the
 * dataset (sb2_load copies them to the device) and are not kept. */
typedef struct sb2_dataset {
    uint64_t num_rows;
    uint64_t row_offset; /* global id of local row 0 */
    uint32_t num_features;
    uint32_t num_groups;
    uint32_t total_bins;
    uint32_t num_queries;
    const sb2_feature* features;
    const sb2_group* groups;
    const float* label;
    const float* weight;              /* NULL when unweighted */
    const uint32_t* query_boundaries; /* NULL, or num_queries + 1 row boundaries */
} sb2_dataset;

/* ObjectiveSetup (crates/silvic-core/src/backend/mod.rs:58-71). Lambdarank (objective/lambdarank.rs) takes the
 * dataset's query boundaries; its per-query inverse max DCGs are computed at load from the labels. */
enum { SB2_REGRESSION = 0, SB2_BINARY = 1, SB2_LAMBDARANK = 2 };
typedef struct sb2_objective {
    int32_t kind;
    int32_t pad_;
    double sigmoid;                      /* binary and lambdarank */
    int32_t lambdarank_norm;             /* lambdarank: normalize the lambdas (LightGBM's lambdarank_norm) */
    uint32_t lambdarank_truncation_level;
    const double* label_gain;            /* lambdarank: gain per label; NULL: LightGBM's default 2^i - 1, i < 31 */
    uint32_t num_label_gain;
    uint32_t pad2_;
} sb2_objective;

/* LeafRange (crates/silvic-core/src/backend/mod.rs:17-22): partition[begin .. begin + count]. */
typedef struct sb2_leaf_range {
    uint32_t begin;
    uint32_t count;
} sb2_leaf_range;

/* BinSplit (crates/silvic-core/src/backend/mod.rs:26-38): bins set in left_bins go left. */
typedef struct sb2_bin_split {
    uint32_t group;
    uint32_t column;
    uint32_t left_bins[8];
} sb2_bin_split;

/* DeviceNode (crates/silvic-core/src/backend/mod.rs:43-47): children >= 0 are nodes, < 0 are ~leaf. */
typedef struct sb2_device_node {
    sb2_bin_split split;
    int32_t left;
    int32_t right;
} sb2_device_node;

/* QuantSpec (crates/silvic-core/src/quantize.rs:35-51). */
typedef struct sb2_quant_spec {
    float inv_grad_scale;
    float inv_hess_scale;
    double grad_scale;
    double hess_scale;
    int32_t grad_max_q;
    int32_t hess_max_q;
    int32_t constant_hessian;
    int32_t stochastic;
    uint32_t seed;
    uint32_t iteration;
} sb2_quant_spec;

/* GradientStats (crates/silvic-core/src/backend/mod.rs:75-78). */
typedef struct sb2_gradient_stats {
    double max_abs_grad;
    double max_hess;
} sb2_gradient_stats;

/* BagSpec (crates/silvic-core/src/backend/mod.rs:82-90). kind 0 = All, 1 = Bernoulli. */
typedef struct sb2_bag_spec {
    int32_t kind;
    uint32_t seed;
    uint32_t round;
    uint32_t pad_;
    double fraction;
} sb2_bag_spec;

enum { SB2_LEFT = 0, SB2_RIGHT = 1 }; /* Side (crates/silvic-core/src/backend/mod.rs:94-113) */

/* SplitConfig (crates/silvic-core/src/split.rs:50-61). The categorical fields matter only for categorical features;
 * the reference's defaults are 100, 10, 10, 4 and 32 (config.rs:145-149). */
typedef struct sb2_split_config {
    int64_t min_data_in_leaf;
    double min_sum_hessian_in_leaf;
    double lambda_l1;
    double lambda_l2;
    double min_gain_to_split;
    int64_t min_data_per_group;
    double cat_l2;
    double cat_smooth;
    int32_t max_cat_to_onehot;  /* a categorical feature of at most this many bins gets the one-hot scan */
    int32_t max_cat_threshold;  /* most categories a sorted categorical split sends left */
} sb2_split_config;

/* SplitInfo (crates/silvic-core/src/split.rs:122-132), plus LeafSplit::splittable. */
typedef struct sb2_split_info {
    int32_t found;        /* 0: the leaf has no split (LeafSplit::best == None) */
    int32_t feature;
    double gain;
    uint32_t threshold;   /* SplitRule::Numerical: bins 0..=threshold go left */
    int32_t default_left;
    double left_grad, left_hess;   /* child sums in histogram units */
    int64_t left_count;            /* estimated from hessians */
    double right_grad, right_hess;
    int64_t right_count;
    double left_output, right_output;
    int32_t categorical;           /* SplitRule::Categorical: the bins set in cat_bins go left, every other bin right */
    int32_t pad_;
    uint32_t cat_bins[8];
} sb2_split_info;

/* Training parameters (crates/silvic-core/src/config.rs:73-116, defaults :123-165), the subset this backend
 * trains with. sb2_default_params() fills the reference defaults. */
typedef struct sb2_params {
    int32_t objective;            /* SB2_REGRESSION / SB2_BINARY / SB2_LAMBDARANK */
    int32_t num_iterations;
    double learning_rate;
    int32_t num_leaves;
    int32_t max_depth;            /* <= 0: no limit */
    int64_t min_data_in_leaf;
    double min_sum_hessian_in_leaf;
    double lambda_l1;
    double lambda_l2;
    double min_gain_to_split;
    double bagging_fraction;
    int32_t bagging_freq;
    uint32_t bagging_seed;
    double feature_fraction;
    uint32_t feature_fraction_seed;
    uint32_t data_random_seed;
    int32_t boost_from_average;
    int32_t use_quantized_grad;
    double sigmoid;
    int32_t num_grad_quant_bins;
    int32_t quant_train_renew_leaf;
    int32_t stochastic_rounding;
    int32_t pad_;
    int32_t lambdarank_norm;              /* lambdarank only: as in sb2_objective */
    uint32_t lambdarank_truncation_level;
    const double* label_gain;             /* NULL: the default gains */
    uint32_t num_label_gain;
    uint32_t pad2_;
    int32_t max_cat_to_onehot;            /* categorical features: as in sb2_split_config */
    int32_t max_cat_threshold;
    double cat_l2;
    double cat_smooth;
    int64_t min_data_per_group;
} sb2_params;

/* One tree in LightGBM 3.3.5 array layout (crates/silvic-core/src/tree.rs:47-73). The arrays belong to the
 * model that returned the view and live as long as it. Internal-node arrays hold num_leaves - 1 entries. */
typedef struct sb2_tree_view {
    int32_t num_leaves;
    int32_t pad_;
    double shrinkage;
    const int32_t* split_feature;
    const float* split_gain;
    const double* threshold;
    const uint32_t* threshold_bin; /* the bin threshold of each split (bins <= threshold go left) */
    const int8_t* decision_type;
    const int32_t* left_child;
    const int32_t* right_child;
    const double* leaf_value;
    const double* leaf_weight;
    const int64_t* leaf_count;
    const double* internal_value;
    const double* internal_weight;
    const int64_t* internal_count;
    const uint32_t* cat_bins;      /* 8 words per split: the bins a categorical split sends left (0 for numerical) */
} sb2_tree_view;

typedef struct sb2_backend sb2_backend;
typedef struct sb2_model sb2_model;

/* ---- library ------------------------------------------------------------------------------------------------ */

/* The last error of a call that had no handle to record it on (sb2_create, sb2_nccl_unique_id). */
int sb2_global_error(char* buf, size_t len);

/* Reference defaults of crates/silvic-core/src/config.rs:123-165. */
void sb2_default_params(sb2_params* out);

/* ---- backend handle: trait Backend (crates/silvic-core/src/backend/mod.rs:115-179) ------------------------- */

/* A backend on CUDA device `device` (the calling process's GPU). */
int sb2_create(int device, sb2_backend** out);
int sb2_destroy(sb2_backend* b);
int sb2_last_error(const sb2_backend* b, char* buf, size_t len);
/* Backend::name */
int sb2_name(const sb2_backend* b, char* buf, size_t len);

/* Backend::load: copies the training set to the device and lays it out in 32-feature tiles. Numerical and
 * categorical features alike (the split search scans each by its kind). */
int sb2_load(sb2_backend* b, const sb2_dataset* train, const sb2_objective* objective);
/* Backend::init_scores (dataset 0, the training set) */
int sb2_init_scores(sb2_backend* b, int dataset, double value);
/* Backend::compute_gradients */
int sb2_compute_gradients(sb2_backend* b, sb2_gradient_stats* out);
/* Backend::quantize */
int sb2_quantize(sb2_backend* b, const sb2_quant_spec* spec);
/* Backend::reset_partition */
int sb2_reset_partition(sb2_backend* b, const sb2_bag_spec* bag, uint32_t* out_rows);
/* Backend::set_histogram_features: used[f] != 0 for every feature whose bins the next histograms must fill. */
int sb2_set_histogram_features(sb2_backend* b, const uint8_t* used, size_t num_features);
/* Backend::histogram (quantized mode): out holds 2 * total_bins doubles, [g, h] integer units per bin. */
int sb2_histogram(sb2_backend* b, sb2_leaf_range leaf, int quantized, double* out, size_t len);
/* Backend::partition: stable, in place; returns the left count. */
int sb2_partition(sb2_backend* b, sb2_leaf_range leaf, const sb2_bin_split* split, uint32_t* out_left);
/* Backend::partition_and_histogram: partition, then the histogram of the `side` child. */
int sb2_partition_and_histogram(sb2_backend* b, sb2_leaf_range leaf, const sb2_bin_split* split, int side,
                                int quantized, double* out, size_t len, uint32_t* out_left);
/* Backend::leaf_sums: out holds 2 * num_leaves int64, [sum rint(g*gs), sum rint(h*hs)] per leaf. */
int sb2_leaf_sums(sb2_backend* b, const sb2_leaf_range* leaves, size_t num_leaves, float grad_scale,
                  float hess_scale, int64_t* out);
/* Backend::add_tree: nodes may be empty (single leaf). */
int sb2_add_tree(sb2_backend* b, const sb2_device_node* nodes, size_t num_nodes, const float* leaf_values,
                 size_t num_leaves);
/* Backend::scores of the training set. */
int sb2_scores(sb2_backend* b, int dataset, float* out, size_t len);

/* Test access to backend state (CpuBackend's tests read the same fields). */
int sb2_read_partition(sb2_backend* b, uint32_t* out, size_t len);
int sb2_read_packed(sb2_backend* b, int32_t* out, size_t len);
int sb2_write_gradients(sb2_backend* b, const float* grad, const float* hess, size_t len);
int sb2_read_gradients(sb2_backend* b, float* grad, float* hess, size_t len);

/* ---- split search: split::find_best_split (crates/silvic-core/src/split.rs:919-961) ------------------------ */

/* The best split of a leaf from its histogram `hist` (2 * total_bins doubles in histogram units,
 * integer-valued), over the features with evaluate[f] != 0, run on the device. splittable (num_features bytes)
 * receives LeafSplit::splittable. */
int sb2_find_best_split(sb2_backend* b, const double* hist, size_t len, const uint8_t* evaluate,
                        double sum_grad, double sum_hess, int64_t count, double grad_scale, double hess_scale,
                        const sb2_split_config* cfg, sb2_split_info* out, uint8_t* splittable);

/* No counterpart in the reference: sb2_find_best_split for callers that cannot let a call allocate device memory
 * (their HBM belongs to another allocator, or a cudaMalloc/cudaFree would stall their other streams). Same search,
 * same result; every pointer is device memory of b's device that the caller owns:
 *   hist        2 * total_bins int32, [g, h] histogram units per bin (len = 2 * total_bins)
 *   evaluate    num_features bytes, nonzero = search the feature
 *   out         one sb2_split_info, written
 *   splittable  num_features bytes, written
 * The call allocates nothing: its scratch is a fixed 480 KiB array in this library's device module, enough for
 * datasets of at most 4096 features; larger ones return SB2_EUNSUPPORTED. The first call on each handle looks up
 * that array's address on the handle's device (cudaGetSymbolAddress, which may load the module) and keeps it for
 * the handle's life, so make that first call before any stream capture. A cudaDeviceReset ends the handle with
 * the rest of its device memory; a handle created afterwards looks the address up again.
 * The call runs on the handle's stream and returns once the results are written; the caller's writes to `hist`
 * and `evaluate` must be complete before it. All calls on one device share the one scratch array: calls that
 * overlap (from other threads, or other handles on the same device) race and give wrong results. */
int sb2_find_best_split_noalloc(sb2_backend* b, const int32_t* hist, size_t len, const uint8_t* evaluate,
                                double sum_grad, double sum_hess, int64_t count, double grad_scale,
                                double hess_scale, const sb2_split_config* cfg, sb2_split_info* out,
                                uint8_t* splittable);

/* No counterpart in the reference: test access to the device split search's division (a correctly rounded FMA
 * division that pipelines, where the library's runs its calls one after another). Compares it with CUDA's correctly
 * rounded division on `count` operand pairs hashed from `seed` and returns the pairs where they differ. */
int sb2_check_division(sb2_backend* b, uint64_t count, uint32_t seed, uint64_t* mismatches);

/* No counterpart in the reference: test access to the tree kernel's failure detection, the analogue of the
 * reference's hung-rank test (crates/silvic-net/tests/ring.rs:338). With `spin_limit` > 0, the single-rank handle
 * trains as rank 0 of two ranks whose other rank never answers: its exchange buffer is local memory that nothing
 * writes, so the first wait for its histogram bins gives up after `spin_limit` polls and sb2_train returns
 * SB2_ECOLLECTIVE. No GPU fault is involved: every wait is bounded and the kernel returns. `spin_limit` 0 makes the
 * handle one rank again. Not for a handle that joined ranks. */
int sb2_test_unanswered_peer(sb2_backend* b, uint32_t spin_limit);

/* ---- measurement -------------------------------------------------------------------------------------------- */

/* Times `repeats` histograms of rows 0 .. rows - 1 (all rows when `rows` is 0) with every feature, as the trainer
 * builds the root of an unbagged tree, with CUDA events on the handle's stream; *seconds gets the mean duration of
 * one histogram (its kernels, launch to completion). Uses the current packed gradients (after sb2_quantize or
 * sb2_train). */
int sb2_time_histogram(sb2_backend* b, uint64_t rows, int repeats, double* seconds);

/* No counterpart in the reference: the rate of the operation that bounds the quantized histogram, a 32-bit shared
 * memory reduction (red.shared.add.u32), measured alone on the handle's device (no dataset needed): one CTA of 512
 * threads per SM adds at the histogram's addresses (word bin * 32 + lane of a 256-bin array: 32 banks per
 * instruction) with its bins in registers, so no global memory is read. `pattern` 0: every lane its own bins (the
 * lanes' words in 32 different 128-byte rows, as in a histogram of random rows); 1: the same bin on every lane at
 * each step (one 128-byte row per instruction). *adds_per_second and *adds_per_sm_clock get lane adds per second
 * (CUDA events) and per SM clock cycle (the CTAs' clock64). */
int sb2_time_shared_adds(sb2_backend* b, int pattern, double* adds_per_second, double* adds_per_sm_clock);

/* sb2_train without the CUDA graph, each operation bracketed by CUDA events: seconds_by_op receives the device
 * time of the last iteration per operation, in the order gradients, quantize (and the iteration's start),
 * histogram, partition, split search, leaf sums, finalize (renewal and the tree record), score update, NCCL
 * collectives, and the whole tree when one persistent kernel grows it (single GPU; the histogram, partition and
 * search entries are then 0); then that kernel's phases summed over the tree's steps (device clock of its first
 * CTA): the partition with the built child's histogram, the children's search context, the slab reduction with the
 * search, finish, and the time spent in grid barriers (num_ops <= 15; fewer fills a prefix). The per-operation breakdown of the reference's `Timed` test backend
 * (crates/silvic-core/tests/train_cpu.rs:434-484). `out` (may be NULL) receives the model. */
int sb2_profile_train(sb2_backend* b, const sb2_params* params, double init_score, double* seconds_by_op,
                      size_t num_ops, sb2_model** out);
/* The same run; `rows` (max_steps rows of 9 doubles) receives one row per grid step of the last tree's kernel (row
 * 0 the root; a grid step runs up to eight splits side by side): seconds in the partitions with the built children's
 * histograms, search contexts, slab reductions with the searches, finish, grid barriers (device clock of the tree
 * kernel's first CTA), then the rows of the step's histograms, the splits it ran, the splits it committed, and the
 * splits it took ready from an earlier step that ran and dropped them (no partition, histogram or search).
 * *num_steps gets the rows written. Single GPU only (SB2_EUNSUPPORTED otherwise). */
int sb2_profile_steps(sb2_backend* b, const sb2_params* params, double init_score, double* rows, size_t max_steps,
                      size_t* num_steps);

/* ---- dataset construction -------------------------------------------------------------------------------- */

/* data::binning::bin_rows (crates/silvic-core/src/data/binning.rs:71-135) on the handle's device: the values of a
 * rows × cols matrix (`row_major`: values[row * cols + feature], else values[feature * rows + row]), f32
 * (`value_bytes` 4) or f64 (8), in host or device memory, are binned into the groups' rows by each feature's mapper
 * (BinMapper::value_to_bin, data/bin_mapper.rs:343-392): a numerical feature's bin is the number of its upper
 * bounds below the value (NaN to the NaN bin, or to 0.0's bin); a categorical feature's is the bin of the value's
 * category (the value truncated to i32), 0 for NaN, negative and unlisted values. The matrix column of feature f is
 * f. `group_data[g]` is a buffer of rows × groups[g].row_stride bytes in host memory that receives group g's rows
 * (padding columns 0); `features` and `groups` are as in sb2_dataset (each group's features, columns and row
 * stride; `data` unused). Building a large dataset in chunks of rows: call once per chunk, with the chunk's values
 * and each group_data[g] advanced by the chunk's first row × row_stride. A group whose bounds and categories
 * exceed 200 KiB returns SB2_EUNSUPPORTED. Values in device memory must be on the handle's device (else SB2_EDATA)
 * and completely written before the call: it reads them on the handle's own stream, which is not ordered after the
 * caller's streams, so the caller synchronizes the stream that produced them first. Returns when done. */
int sb2_bin_dense(sb2_backend* b, const void* values, int value_bytes, uint64_t rows, uint32_t cols, int row_major,
                  const sb2_feature* features, uint32_t num_features, const sb2_group* groups, uint32_t num_groups,
                  uint8_t* const* group_data);

/* The most-frequent-bin skip of the tree kernel's histogram (LightGBM's most_freq_bin, which the reference's GPU
 * backend keeps per column, crates/silvic-gpu/src/backend.rs:336-376 and kernels.kern:439-468): at sb2_load, a tile
 * of up to 32 features whose features hold, on average, at least `share` of the rows in their most frequent bins
 * skips those bins' shared-memory adds, and the kernel recovers them from the rows' totals. Results are identical
 * either way. Off by default (a share above 1): the histogram gives each lane of a warp a different feature, so a
 * dominant bin causes no bank conflict, and on B200 the per-element test costs more issue slots than the skipped
 * atomics save. 0: every tile skips. Takes effect at the next sb2_load. */
int sb2_set_dominant_share(sb2_backend* b, double share);

/* ---- multi-GPU --------------------------------------------------------------------------------------------- */

/* An NCCL unique id (128 bytes) for rank 0 to share with the other ranks. */
int sb2_nccl_unique_id(uint8_t* out, size_t len);
/* How the tree kernel's ranks exchange their histograms (no counterpart in the reference, whose ranks allreduce each
 * split's histogram over TCP, learner.rs:189-220): SB2_EXCHANGE_AUTO (the default) pushes each split's bins over
 * NVLink inside the tree kernel when every rank can map every other rank's buffer (CUDA IPC), else falls back to
 * SB2_EXCHANGE_NCCL: per-step launches with an ncclAllReduce of each split's histogram, in one CUDA graph per
 * iteration. Both give the same trees. Call before sb2_join_ranks, with the same mode on every rank. */
enum { SB2_EXCHANGE_AUTO = 0, SB2_EXCHANGE_NCCL = 1 };
int sb2_set_rank_exchange(sb2_backend* b, int mode);
/* Joins `world` ranks (one process per GPU) through an NCCL communicator; call after sb2_load on every rank. It also
 * maps every rank's exchange buffer (CUDA IPC) for the tree kernel's histogram exchange over NVLink. Collective. */
int sb2_join_ranks(sb2_backend* b, const uint8_t* unique_id, size_t len, int world, int rank);

/* ---- device-resident training: boosting::train (crates/silvic-core/src/boosting.rs:63-149) ------------------ */

/* Trains params->num_iterations trees on the loaded training set. Every split runs on the device: partition,
 * smaller-child histogram, (NCCL reduction), sibling subtraction, split scan and leaf choice; the host only reads
 * each finished tree. `init_score` is computed by the caller over every rank's labels in row order
 * (objective::init_score, crates/silvic-core/src/objective/mod.rs:92-109). */
int sb2_train(sb2_backend* b, const sb2_params* params, double init_score, sb2_model** out);
/* objective::init_score (crates/silvic-core/src/objective/mod.rs:92-109, regression.rs:8-17, binary.rs:8-21) over
 * `n` labels in row order: BoostFromAverage, 0 when params->boost_from_average is off. */
int sb2_boost_from_average(const sb2_params* params, const float* label, const float* weight, size_t n, double* out);
int sb2_model_free(sb2_model* m);
int sb2_model_num_trees(const sb2_model* m);
int sb2_model_tree(const sb2_model* m, int index, sb2_tree_view* out);
/* Seconds the device spent in each of the last sb2_train's iterations (CUDA events), and split steps taken. */
int sb2_model_iteration_seconds(const sb2_model* m, double* out, size_t len);
/* Seconds of each iteration's persistent tree kernel launch alone (CUDA events on the backend's stream around the
 * launch; single GPU, 0 entries otherwise); returns how many there are. No counterpart in the reference: the
 * roofline of the kernel that grows the trees. */
int sb2_model_tree_seconds(const sb2_model* m, double* out, size_t len);

#ifdef __cplusplus
}
#endif

#endif /* SILVIC_B200_H */
