// train.cuh — device-resident state of the leaf-wise learner (silvic-core learner.rs) and the kernels that move it.
//
// A tree grows as a fixed sequence of launches per split step, so the whole tree (and the whole boosting
// iteration) can be enqueued without the host waiting on the device, and captured in one CUDA graph:
//   partition_flags -> partition_scatter -> histogram (smaller child) -> [NCCL allreduce] -> search
// `search` subtracts the sibling, scans both children, applies the split to the tree arrays and chooses the next
// leaf (Learner::grow's loop, learner.rs:158-163), writing the next step. A step with nothing to split is a no-op
// for every kernel, so the host always enqueues num_leaves - 1 steps.
#pragma once

#include "common.cuh"
#include "hist.cuh"

namespace sb2 {

// A leaf being grown (learner.rs:87-94).
struct DevLeaf {
    uint32_t begin;   // this rank's rows: partition positions begin .. begin + count
    uint32_t count;
    uint32_t which;   // partition buffer holding them
    int32_t depth;
    double units_grad;  // LeafSums in histogram units, count over every rank
    double units_hess;
    int64_t count_global;
    int32_t has_hist;   // Leaf::hist is Some: its histogram slot is valid for the evaluated features
    int32_t has_best;
    sb2_split_info best;
};

// One split step: the leaf being split and everything the step's kernels need.
struct Step {
    int32_t active;      // 0: nothing to split (the tree is finished); every kernel of the step returns
    int32_t root;        // the root step: histogram of the root, no partition
    int32_t leaf;        // leaf being split; its left child keeps the index
    int32_t new_leaf;    // the right child's index
    int32_t may_search;  // the children's histograms are built (learner.rs:266-268)
    int32_t built_left;  // the histogram is built for the left child (learner.rs:271-275)
    uint32_t begin, count, which;  // the parent's rows
    int32_t depth;                 // the parent's depth
    uint32_t split_tile, split_lane;
    uint32_t left_bins[8];
    int64_t parent_count;
    sb2_split_info info;
    uint32_t local_left;  // this rank's left count, written by partition_scatter
    int32_t bag;          // the partition is a Bernoulli bag: rows with quantize::in_bag go "left"
    uint32_t bag_seed;
    uint32_t bag_round;
    double bag_fraction;
    uint64_t row_offset;
    int32_t prepared;     // the tree kernel: an earlier grid step ran this split and kept its work (PrepSplit)
    int32_t pad_;
};

// Tree arrays of one tree in LightGBM layout (tree.rs:47-73), `max_leaves` entries each.
struct DevTree {
    int32_t* num_leaves;        // [1]
    int32_t* split_feature;
    float* split_gain;
    uint32_t* threshold_bin;
    int8_t* decision_type;
    int32_t* left_child;
    int32_t* right_child;
    double* internal_value;
    double* internal_weight;
    int64_t* internal_count;
    double* leaf_value;
    double* leaf_weight;
    int64_t* leaf_count;
    int32_t* leaf_parent;
    int32_t* leaf_depth;
    uint32_t* cat_bins;         // 8 words per node: a categorical split's left bins (0 for a numerical one)
};

// Iteration state (boosting.rs:227-285).
struct IterState {
    int32_t iteration;     // global iteration index: keys quantization draws and the feature mask
    int32_t stopped;       // a tree could not split: training is over
    int32_t trees;         // trees added so far
    int32_t error;         // non-zero: an internal error (code in error_info)
    int64_t error_info;
    unsigned long long max_abs_grad_bits;  // GradientStats maxima as the bits of non-negative doubles
    unsigned long long max_hess_bits;
    sb2_quant_spec spec;
    int64_t root_count;    // bagged rows over every rank
    // This rank's sums of every row's quantized g and h (iteration start): the root's units when one GPU grows the
    // tree (every row falls in one bin of every feature, so they equal the sums over any feature's histogram).
    unsigned long long root_units[2];
};

// The tree kernel's record of a split it ran speculatively and dropped, kept until the leaf is split (learner.rs's
// split of a leaf depends on the leaf alone, so the work stays valid): the partition of the leaf's rows into the
// other buffer stays in place (only the leaf's own splits write its positions), the children's histograms sit in
// the leaf's two prepared slots, and this record holds the rest.
struct PrepSplit {
    int32_t valid;
    int32_t may_search;      // Step::may_search when it ran: the children were searched under it
    uint32_t left;           // this rank's left count
    int32_t pad_;
    DevLeaf child[2];        // the children's records, best splits included (0: the built child)
};

// Everything the training kernels read, by value.
struct TrainArgs {
    DevData d;
    sb2_split_config cfg;
    int32_t max_leaves;      // params.num_leaves
    int32_t max_depth;
    int32_t sums_feature;    // first non-trivial feature (learner.rs:115), -1 when none
    int32_t root_from_rows;  // 1: the root's units come from IterState::root_units instead of the histogram
    int32_t num_iterations;
    uint32_t total_bins;
    uint32_t num_features;
    // learner state
    DevLeaf* leaves;            // [max_leaves]
    double* leaf_gain;          // [max_leaves]: the persistent kernel's copy of each leaf's best gain (-inf: none)
    uint8_t* splittable;        // [max_leaves * num_features]
    Step* step;
    uint8_t* evaluate;          // [num_features]: the current step's evaluated features
    const uint8_t* masks;       // [num_iterations * num_features]: per-iteration feature_mask
    int* staging;               // [2 * total_bins + 2]: the step's new histogram and, after it, the left count
    int* slots;                 // [3 * max_leaves * 2 * total_bins]: one histogram per leaf, then the tree kernel's
                                // two prepared slots per leaf (prep_slot)
    PrepSplit* prep;            // [max_leaves]: the tree kernel's dropped splits, by leaf
    uint8_t* prep_split;        // [max_leaves * 2 * num_features]: their children's splittable rows
    HistJob* hist_job;
    IterState* iter;
    DevTree tree;               // the tree being grown
    // partition
    uint32_t* rows[2];
    int32_t* ordered[2];
    uint32_t* flags;            // one bit per partition position; the tree kernel: kSplits regions of
                                // num_rows / 32 + 2 words
    uint32_t* tile_left;        // left count per partition tile
    unsigned int* cursors;      // [2 kSplits (max_leaves + 1)]: the tree kernel's placement counters per split
    // per-(child, feature) scan results (the tree kernel: per split of a step, 2 kSplits rows of F) and the search
    // kernel's completion counter
    void* candidates;
    uint8_t* cand_flags;        // [2 kSplits F]: bit 0 the candidate was found, bit 1 its feature stays splittable
    double* cand_gain;          // [2 kSplits F]: its gain (what `better` compares)
    unsigned int* done_counter;
};

// The scan result of one feature for one child (split.rs:311-317 Candidate + FeatureResult::splittable).
struct FeatureCandidate {
    int32_t found;
    int32_t splittable;
    int32_t feature;
    int32_t default_left;
    double gain;        // best.gain - min_gain_shift
    double best_gain;   // best.gain
    uint32_t threshold;
    uint32_t pad_;
    double left_grad, left_hess;  // real sums as LightGBM keeps them (split.rs:300-307)
    int64_t left_count;
    double left_units_grad, left_units_hess;
    int32_t kind;                 // CandidateKind (split.rs:318-327): numerical, one-hot, sorted from either end
    int32_t pad2_;
    uint32_t cat_bins[8];         // a categorical candidate's left bins
};

// FeatureCandidate::kind
enum : int32_t { kCandNumerical = 0, kCandOneHot = 1, kCandSortedForward = 2, kCandSortedReverse = 3 };

static_assert(sizeof(FeatureCandidate) % 8 == 0, "candidates are copied as 64-bit words");

constexpr int kMaxPartitionCtas = 8192;  // CTAs a partition launch may use (one left count each)
constexpr int kPartitionThreads = 256;
constexpr int kSearchThreads = 256;   // 8 warps, one feature each

// The persistent tree kernel (grow.cu): every step of one tree in one cooperative launch.
int grow_threads();
cudaError_t grow_configure(int smem_bytes, int* blocks_per_sm);
// `phase_ns` (optional, kGrowPhases entries) receives the nanoseconds CTA 0 spent per phase: the partition with
// the built child's histogram, the children's search context, the slab reduction with the search, the finish, the
// grid barriers. With `trace_steps` > 0
// it is followed by one row of kStepTrace values per grid step (up to trace_steps): the same phase times of that
// step, then the rows of its histograms, the splits it ran, the splits it committed, and the splits it took ready
// from earlier steps (PrepSplit).
constexpr int kGrowPhases = 5;
constexpr int kStepTrace = kGrowPhases + 4;
// The layout of its dynamic shared memory (`bytes` in all): the histogram's arrays first, the partition's scan
// words (2 * 512 + 64) at `scan_offset`, the histogram's staging slots (16 warps x `stage_depth` slots of
// `slot_bytes`, 128-byte aligned) at `stage_offset`, its per-feature flags ((5 kSplits + 1) F bytes) at
// `flags_offset`. The
// search's bins (kMaxBins [g, h] pairs per group of kScanWarps warps) reuse the scan words; the histogram's arrays
// stay zero between steps.
constexpr uint32_t kMaxStageDepth = 4;  // staging slots per warp at most
struct GrowSmem {
    int bytes;
    uint32_t scan_offset;
    uint32_t stage_offset;
    uint32_t slot_bytes;
    uint32_t stage_depth;
    uint32_t flags_offset;
    // A built child's row costs a grid step's plan this many parent rows of partition: its histogram adds one
    // shared atomic per bin byte of the row, the partition moves about 17 bytes per row.
    float hist_weight;
};
// The kernel's static shared memory (bytes; -1 on error): the dynamic part has what is left of the CTA's limit.
int grow_static_smem();

// Ranks of one training run, one GPU each, every rank running the tree kernel at once. Feature f belongs to rank
// f mod world (its owner). Per grid step each rank writes its left counts into every rank's exchange buffer; per
// searched (split, feature) item every other rank reduces its own slabs of the built child's bins and writes them
// into the owner's buffer (NVLink stores through CUDA IPC mappings), raising its flag there with the step's epoch;
// the owner waits on those flags in its own memory, sums the copies with its own, searches both children and writes
// the two candidates into every rank's candidate arrays. Once every CTA of a rank has done so, the rank raises its
// step flag in every buffer; each rank's finish waits for all of them and runs on the same candidates, so every
// rank grows the same tree (split.rs:866-873 `better` is a total order: the choice does not depend on who searched).
constexpr int kMaxRanks = 8;
struct GrowExchange {
    uint8_t* peers[kMaxRanks];  // every rank's exchange buffer (this rank's own at [rank]); unused with one rank
    int32_t world, rank;
    uint32_t epoch0;            // the launch's epochs are epoch0 + 1 (the root) .. (they rise across launches)
    uint32_t spin_limit;        // polls of a rank's flag before the wait gives up (error 4)
};
constexpr uint32_t kPeerSpins = 1u << 22;  // polls of a peer's flag (a few seconds) before error 4, by default
// Splits a grid step of the tree kernel runs at most (steps.cuh).
constexpr int kSplits = 8;

// An exchange buffer, for split j of a step, source rank s and owned feature slot o = f / world (the owner's o-th
// feature): u32 flags and counts, then the arrays, each 128-byte aligned.
struct ExchangeLayout {
    size_t left_flags;    // u32 [kMaxRanks]: source s's left counts are in (the step's epoch)
    size_t left_values;   // u32 [2 parity][kSplits][kMaxRanks]
    size_t step_flags;    // u32 [kMaxRanks]: source s wrote every candidate of the step it owns
    size_t item_flags;    // u32 [kSplits][owned][kMaxRanks]: source s's bins of item (j, o) are in
    size_t bins;          // int2 [kMaxRanks][kSplits][owned][kMaxBins]: source s's built-child bins
    // The step's candidates, written by their owners, in two sets by the step's parity: an owner may write the next
    // step's candidates (those it needs no other rank for) while a slower rank still reads this step's.
    size_t candidates;    // FeatureCandidate [2 parity][2 kSplits][F]
    size_t cand_flags;    // u8 [2 parity][2 kSplits][F]
    size_t cand_gain;     // f64 [2 parity][2 kSplits][F]
    size_t bytes;
    uint32_t owned;       // feature slots a rank owns at most: ceil(F / world)
    uint32_t features;
};

__host__ __device__ inline size_t align128(size_t v) { return (v + 127) / 128 * 128; }

__host__ __device__ inline ExchangeLayout exchange_layout(uint32_t F, uint32_t world) {
    ExchangeLayout x{};
    const uint32_t w = world < 1 ? 1u : world;
    x.owned = (F + w - 1) / w;
    x.left_flags = 0;
    x.left_values = 128;
    x.step_flags = align128(x.left_values + 4ull * 2 * kSplits * kMaxRanks);
    x.item_flags = x.step_flags + 128;
    x.bins = align128(x.item_flags + 4ull * kSplits * x.owned * kMaxRanks);
    x.features = F;
    x.candidates = align128(x.bins + 8ull * kMaxRanks * kSplits * x.owned * kMaxBins);
    x.cand_flags = align128(x.candidates + sizeof(FeatureCandidate) * 2ull * 2 * kSplits * F);
    x.cand_gain = align128(x.cand_flags + 2ull * 2 * kSplits * F);
    x.bytes = align128(x.cand_gain + 8ull * 2 * 2 * kSplits * F);
    return x;
}
__host__ __device__ inline size_t exchange_bytes(uint32_t F, uint32_t world) { return exchange_layout(F, world).bytes; }

cudaError_t launch_grow_tree(const TrainArgs& t, const HistArgs& h, unsigned int* barrier, int grid,
                             const GrowSmem& smem, const GrowExchange& x, cudaStream_t s,
                             unsigned long long* phase_ns, int trace_steps);

void launch_partition_flags(const TrainArgs& a, int grid, cudaStream_t s);
void launch_partition_scatter(const TrainArgs& a, int grid, cudaStream_t s);
void launch_search(const TrainArgs& a, int grid, cudaStream_t s);

}  // namespace sb2
