/*
 * oracle.h — C API of the CPU oracle (test infrastructure, not the product).
 *
 * The oracle restates silvic-core's CPU training path in C++ so the B200 backend can be checked against it:
 * quantization (crates/silvic-core/src/quantize.rs), the CpuBackend operations
 * (crates/silvic-core/src/backend/cpu.rs), pointwise objectives (crates/silvic-core/src/objective/{regression,binary}.rs), the split
 * finder (crates/silvic-core/src/split.rs), the leaf-wise learner (crates/silvic-core/src/learner.rs) and the
 * boosting loop (crates/silvic-core/src/boosting.rs). Only tests, the smoke check and the bench's CPU baseline
 * load it. It reuses the plain data types of include/silvic_b200.h.
 */
#ifndef SILVIC_ORACLE_H
#define SILVIC_ORACLE_H

#include "../include/silvic_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_model orc_model;

int orc_num_threads(void);
void orc_set_num_threads(int threads);

/* quantize.rs */
uint32_t orc_mix32(uint32_t x);
float orc_uniform(uint32_t seed, uint32_t stream, uint32_t iteration, uint64_t row);
void orc_quant_spec(double max_abs_grad, double max_hess, int has_constant_hessian, double constant_hessian,
                    uint32_t num_bins, int stochastic, uint32_t seed, uint32_t iteration, sb2_quant_spec* out);
void orc_quantize(const sb2_quant_spec* spec, const float* grad, const float* hess, size_t n, uint64_t row_offset,
                  int32_t* out);
void orc_unpack(int32_t packed, int32_t* g, int32_t* h);
int orc_in_bag(uint32_t seed, uint32_t round, uint64_t row, double fraction);
float orc_fixed_point_scale(double max_abs);
int64_t orc_to_fixed(float value, float scale);

/* objective */
void orc_gradients(const sb2_objective* objective, const float* scores, const float* label, const float* weight,
                   size_t n, float* grad, float* hess);
double orc_init_score(const sb2_params* params, const float* label, const float* weight, size_t n);
/* objective/lambdarank.rs: every query's gradients (data: num_rows, label, weight, query boundaries) at `scores`;
 * max_dcg_at_k; the sigmoid table's entry for a score difference. SB2_EDATA for labels or queries it rejects. */
int orc_lambdarank_gradients(const sb2_params* params, const sb2_dataset* data, const float* scores, float* grad,
                             float* hess);
double orc_lambdarank_max_dcg(size_t k, const float* labels, size_t n, const double* gain, size_t num_gain);
double orc_lambdarank_sigmoid(double sigmoid, double delta);

/* CpuBackend operations on a dataset */
int orc_histogram(const sb2_dataset* data, const int32_t* packed, int32_t max_quant, const uint32_t* rows,
                  size_t n, const uint8_t* used, double* out);
uint32_t orc_partition(const sb2_dataset* data, const sb2_bin_split* split, uint32_t* rows, size_t n);
void orc_leaf_sums(const float* grad, const float* hess, const uint32_t* partition, const sb2_leaf_range* leaves,
                   size_t num_leaves, float grad_scale, float hess_scale, int64_t* out);
int orc_add_tree(const sb2_dataset* data, const sb2_device_node* nodes, size_t num_nodes, const float* leaf_values,
                 size_t num_leaves, float* scores);
uint32_t orc_reset_partition(const sb2_bag_spec* bag, uint64_t num_rows, uint64_t row_offset, uint32_t* out);

/* data/binning.rs: bin_rows over a dense f32 (value_bytes 4) or f64 (8) matrix into the groups' rows
 * (group_data[g]: rows x row_stride bytes); numerical features only (else SB2_EUNSUPPORTED). value_to_bin of one
 * value with one feature's bounds (data/bin_mapper.rs:343-360), for the tests. */
int orc_bin_rows(const void* values, int value_bytes, uint64_t rows, uint32_t cols, int row_major,
                 const sb2_feature* features, uint32_t num_features, const sb2_group* groups, uint32_t num_groups,
                 uint8_t* const* group_data);
uint32_t orc_value_to_bin(const double* upper_bounds, uint32_t num_upper_bounds, int nan_bin, double value);

/* split.rs */
int orc_find_best_split(const sb2_dataset* data, const double* hist, const uint8_t* evaluate, double sum_grad,
                        double sum_hess, int64_t count, double grad_scale, double hess_scale,
                        const sb2_split_config* cfg, sb2_split_info* out, uint8_t* splittable);
void orc_feature_mask(const sb2_dataset* data, double fraction, uint32_t seed, uint32_t iteration, uint8_t* out);

/* boosting.rs: trains on `num_shards` row shards as that many ranks (their allreduces are exact sums in rank
 * order); shard r must have row_offset = rows of shards below it. */
int orc_train(const sb2_dataset* shards, int num_shards, const sb2_params* params, orc_model** out);
void orc_model_free(orc_model* m);
int orc_model_num_trees(const orc_model* m);
int orc_model_tree(const orc_model* m, int index, sb2_tree_view* out);
double orc_model_init_score(const orc_model* m);
/* Wall seconds of each iteration of the last orc_train. */
int orc_model_iteration_seconds(const orc_model* m, double* out, size_t len);
/* Wall seconds per operation over the run, as the reference's `Timed` backend splits them
 * (crates/silvic-core/tests/train_cpu.rs:434-484): gradients, quantize, histogram, split search, partition, leaf
 * sums, add_tree. Returns how many there are (7). */
int orc_model_op_seconds(const orc_model* m, double* out, size_t len);
/* f64 prediction of one raw row (crates/silvic-core/src/model/predict.rs numerical decisions): sum of trees. */
double orc_model_predict_raw(const orc_model* m, const sb2_dataset* data, const double* row);
const char* orc_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
