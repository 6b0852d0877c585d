// steps.cuh — the persistent tree kernel's grid steps: the best leaf's split and, run beside it, the splits of the
// next kSplits - 1 leaves in the order the learner would take them, committed only as far as that order holds.
//
// The learner splits one leaf at a time, always the leaf with the best split (Learner::grow, learner.rs:158-163,
// with the ties of `prefer_leaf`). Ranked at the end of a step, the leaves X1, X2, ... by their best gains, X1 is
// split next; X2 is split after it exactly when neither child of X1 prefers over X2; X3 after that when no child of
// X1 or X2 prefers over it; and so on: every other leaf already ranks below them, and a leaf's split (its rows, its
// histogram, its children's searches) does not depend on the splits before it. A grid step therefore runs the
// splits of X1 .. Xn together (n <= kSplits, each a whole partition, histogram and search) and, at its finish,
// commits X1 and then each next Xj while the rule holds; the first Xj that a new child outranks, and all after it,
// are dropped: their leaves stay leaves, as they were, and are ranked again. The committed sequence is the
// learner's own, so the tree is identical. On the first trees of config 2 the next split is a child of the previous
// one for about 1.5% of splits, so a step commits nearly all of its splits; late in a job, with small gradients, a
// tree runs four splits for every one it commits.
//
// A dropped split's work is kept for the step that commits it (PrepSplit): its partition wrote only the other
// buffer's copy of its own positions (its leaf record still names the buffer that holds its rows, and nothing else
// writes them), its children's histograms went to its leaf's two prepared slots (copied to the children's slots only
// on commit), and the finish records its left count, its children (with their best splits) and their splittable
// rows. When the leaf is ranked into a later step, the split comes back `prepared`: no CTA partitions, histograms or
// searches it, and its finish reads the record. Its children were searched under the step's leaf count then; a
// step with fewer leaves left searches them no more (their records lose their histograms and best splits), and one
// that would search children not searched then runs the split again.
#pragma once

#include "search.cuh"
#include "train.cuh"

namespace sb2 {

// The finish's scratch (shared memory of every CTA).
struct StepsFinish {
    DevLeaf child[kSplits][2];           // the children of every split (child 0 the built one)
    double other_gain[kSplits];          // the best leaves that no split of the step touches
    int32_t other_leaf[kSplits];
    DevLeaf other[kSplits];              // their records
    DevLeaf pending[kSplits];            // the records of the step's own leaves (split j >= 1), kept if dropped
    int32_t pending_leaf[kSplits];       // their indices (-1: split 0)
    uint32_t left[kSplits];              // this rank's left count of every split
    int32_t committed;                   // splits committed by this step
    int32_t next_n;                      // splits of the next step
    Step next[kSplits];
    int32_t next_from[kSplits];          // where each next split's leaf comes from (kPool* codes)
    // The features of the best splits above, loaded ahead: the step's splits (also the pending leaves'), the
    // children's, the other leaves'.
    DevFeature split_feat[kSplits];
    DevFeature child_feat[kSplits][2];
    DevFeature other_feat[kSplits];
};

// The leaves a finish ranks, one per lane of a warp: the untouched best leaves (code k), the committed splits'
// children (kPoolChild + 2 i + c) and the dropped splits' own leaves (kPoolPending + j).
constexpr int kPoolChild = kSplits, kPoolPending = 3 * kSplits;
static_assert(4 * kSplits <= 32, "the finish ranks one leaf per lane");

// The leaf index of split `st`'s child c (0: the built one; the left child keeps the parent's index; the root's
// only child is leaf 0).
__device__ __forceinline__ int32_t child_index(const Step& st, int c) {
    if (st.root) return 0;
    return (c == 0) == (st.built_left != 0) ? st.leaf : st.new_leaf;
}

// Whether (og, ol) comes first in the learner's order over (g, l): the higher gain, then the lower index.
__device__ __forceinline__ bool ranks_before(double og, int32_t ol, double g, int32_t l) {
    return og > g || (og == g && ol < l);
}

// Warp: leaf `leaf`'s splittable row (F bytes) into `dst`, eight bytes a lane in flight.
__device__ __forceinline__ void copy_split_row(const TrainArgs& a, int32_t leaf, uint8_t* dst) {
    const uint32_t lane = threadIdx.x & 31, F = a.num_features;
    const uint8_t* row = a.splittable + static_cast<size_t>(leaf) * F;
    for (uint32_t f0 = 0; f0 < F; f0 += 32 * 8) {
        uint8_t v[8];
#pragma unroll
        for (uint32_t q = 0; q < 8; ++q) {
            const uint32_t f = f0 + 32 * q + lane;
            v[q] = f < F ? __ldcg(row + f) : 0;
        }
#pragma unroll
        for (uint32_t q = 0; q < 8; ++q) {
            const uint32_t f = f0 + 32 * q + lane;
            if (f < F) dst[f] = v[q];
        }
    }
}

// Before the step's last grid barrier completes (no candidate needed): every split's children records (warp 0);
// the kSplits best leaves no split touches, and their records and splittable rows (warp 3); the records and rows
// of the step's own speculative leaves (warp 4). `left[j]`: split j's left count on this rank.
__device__ void steps_finish_prepare(const TrainArgs& a, const Step* st, int n, const SearchCtx* sc,
                                     const uint32_t* left, uint8_t* osplit, uint8_t* psplit, StepsFinish& fs) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const IterState& it = *a.iter;
    if (warp == 0 && lane < static_cast<uint32_t>(n)) {
        const int j = static_cast<int>(lane);
        const Step& s = st[j];
        fs.left[j] = left[j];
        if (!s.root) fs.split_feat[j] = a.d.features[s.info.feature];
        if (s.prepared) {
            // Kept from the grid step that ran it; under a step whose children are no longer searched (fewer leaves
            // left), they have no histograms and no best splits.
            DevLeaf c0 = load_cg(&a.prep[s.leaf].child[0]), c1 = load_cg(&a.prep[s.leaf].child[1]);
            if (!s.may_search) c0.has_hist = c1.has_hist = c0.has_best = c1.has_best = 0;
            fs.child[j][0] = c0;
            fs.child[j][1] = c1;
        } else if (s.root) {
            DevLeaf l = load_cg(a.leaves);  // begin, count, which, depth: set before the launch
            l.units_grad = sc[j].ctx[0].units_grad;
            l.units_hess = sc[j].ctx[0].units_hess;
            l.count_global = it.root_count;
            l.has_hist = sc[j].searched;
            l.has_best = 0;
            fs.child[j][0] = l;
        } else {
            DevLeaf l{}, r{};
            l.begin = s.begin;
            l.count = left[j];
            r.begin = s.begin + left[j];
            r.count = s.count - left[j];
            l.which = r.which = s.which ^ 1u;
            l.depth = r.depth = s.depth + 1;
            l.units_grad = s.info.left_grad;
            l.units_hess = s.info.left_hess;
            l.count_global = sc[j].left_global;
            r.units_grad = s.info.right_grad;
            r.units_hess = s.info.right_hess;
            r.count_global = sc[j].right_global;
            l.has_hist = r.has_hist = sc[j].searched;
            fs.child[j][s.built_left ? 0 : 1] = l;
            fs.child[j][s.built_left ? 1 : 0] = r;
        }
    } else if (warp == 3) {
        // The leaves that existed before this step, other than the step's own: the kSplits best by their gains (as
        // the writer CTA left them in earlier steps). Each lane keeps its own best kSplits in order; the warp then
        // takes the best head kSplits times.
        const int32_t before = st[0].root ? 0 : st[0].new_leaf;
        double tg[kSplits];
        int32_t tl[kSplits];
#pragma unroll
        for (int k = 0; k < kSplits; ++k) {
            tg[k] = -INFINITY;
            tl[k] = -1;
        }
        for (int32_t l0 = 0; l0 < before; l0 += 32 * 4) {
            double g[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int32_t l = l0 + 32 * q + static_cast<int32_t>(lane);
                g[q] = l < before ? __ldcg(a.leaf_gain + l) : -INFINITY;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                int32_t l = l0 + 32 * q + static_cast<int32_t>(lane);
                bool skip = l >= before || g[q] == -INFINITY;
                for (int j = 0; j < n; ++j) skip |= l == st[j].leaf;
                if (skip) continue;
                double gv = g[q];
#pragma unroll
                for (int k = 0; k < kSplits; ++k)  // insertion: the entry carried down swaps with worse ones
                    if (tl[k] < 0 || ranks_before(gv, l, tg[k], tl[k])) {
                        const double sg = tg[k];
                        const int32_t sl = tl[k];
                        tg[k] = gv;
                        tl[k] = l;
                        gv = sg;
                        l = sl;
                        if (l < 0) break;
                    }
            }
        }
#pragma unroll
        for (int k = 0; k < kSplits; ++k) {
            double bg = tg[0];
            int32_t bl = tl[0];
            for (int o = 16; o > 0; o >>= 1)
                prefer_leaf(bg, bl, __shfl_xor_sync(0xffffffffu, bg, o), __shfl_xor_sync(0xffffffffu, bl, o));
            if (bl >= 0 && tl[0] == bl) {  // the owner pops its head
#pragma unroll
                for (int q = 0; q + 1 < kSplits; ++q) {
                    tg[q] = tg[q + 1];
                    tl[q] = tl[q + 1];
                }
                tg[kSplits - 1] = -INFINITY;
                tl[kSplits - 1] = -1;
            }
            if (lane == 0) {
                fs.other_gain[k] = bg;
                fs.other_leaf[k] = bl;
            }
        }
    } else if (warp == 4) {
        if (lane < static_cast<uint32_t>(kSplits)) fs.pending_leaf[lane] = lane >= 1 && lane < static_cast<uint32_t>(n) ? st[lane].leaf : -1;
    }
    __syncthreads();
    // The records and splittable rows of those leaves, in case they are split next, and of the step's own
    // speculative leaves, in case their splits are dropped: warp k < kSplits the k-th best other leaf's (lane 0 its
    // record and split feature), warp kSplits + j split j's leaf's.
    static_assert(2 * kSplits <= kHistThreads / 32, "a warp per prepared leaf");
    if (warp < static_cast<uint32_t>(kSplits)) {
        const int32_t leaf = fs.other_leaf[warp];
        if (leaf >= 0) {
            if (lane == 0) {
                const DevLeaf r = load_cg(a.leaves + leaf);
                fs.other[warp] = r;
                fs.other_feat[warp] = a.d.features[r.best.feature];
            }
            copy_split_row(a, leaf, osplit + static_cast<size_t>(warp) * a.num_features);
        }
    } else if (warp < static_cast<uint32_t>(2 * kSplits)) {
        const uint32_t j = warp - kSplits;
        const int32_t leaf = fs.pending_leaf[j];
        if (leaf >= 0) {
            if (lane == 0) fs.pending[j] = load_cg(a.leaves + leaf);
            copy_split_row(a, leaf, psplit + static_cast<size_t>(j) * a.num_features);
        }
    }
    __syncthreads();
}

// The step's finish, in every CTA on the same inputs: each child's best split from the compact candidates
// (`candidates`, `cand_flags`, `cand_gain`: rows 2 j + c of F; warp 2 j + c for child c of split j), the splits committed, the tree, records and slots of the committed splits (writer CTAs), and the next
// step's splits into `st` (and their features into `eval`, kSplits rows of F). `csplit` holds 2 kSplits rows of F
// (the children's splittable flags), `mask` the iteration's feature mask.
__device__ void steps_finish(const TrainArgs& a, Step* st, int& n, const SearchCtx* sc, uint8_t* eval,
                             const uint8_t* mask, uint8_t* csplit, const uint8_t* osplit, const uint8_t* psplit,
                             uint32_t cta, StepsFinish& fs, const FeatureCandidate* candidates,
                             const uint8_t* cand_flags, const double* cand_gain) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t F = a.num_features;
    const IterState& it = *a.iter;
    const int children = st[0].root ? 1 : 2;
    static_assert(2 * kSplits <= kHistThreads / 32, "a warp per child");
    if (warp < static_cast<uint32_t>(2 * n)) {
        const int j = static_cast<int>(warp) / 2, ch = static_cast<int>(warp) % 2;
        if (ch < children && st[j].prepared) {
            // The child's record came whole from the split's PrepSplit; its splittable row was kept beside it.
            uint8_t* rowc = csplit + static_cast<size_t>(2 * j + ch) * F;
            const uint8_t* kept = a.prep_split + (2 * static_cast<size_t>(st[j].leaf) + ch) * F;
            const bool has_hist = fs.child[j][ch].has_hist != 0;
            for (uint32_t f = lane; f < F; f += 32) rowc[f] = has_hist ? __ldcg(kept + f) : 0;
            if (lane == 0 && fs.child[j][ch].has_best) fs.child_feat[j][ch] = a.d.features[fs.child[j][ch].best.feature];
        } else if (ch < children) {
            // The best candidate of the child over every feature by `better` (found, then the higher gain, then the
            // lower feature), from the compact gains and flags; then the winner's full candidate.
            FeatureCandidate best{};
            best.found = 0;
            uint8_t* rowc = csplit + static_cast<size_t>(2 * j + ch) * F;
            if (sc[j].searched) {
                const uint8_t* flags = cand_flags + static_cast<size_t>(2 * j + ch) * F;
                const double* gains = cand_gain + static_cast<size_t>(2 * j + ch) * F;
                int found = 0;
                double bg = -INFINITY;
                int32_t bf = -1;
                for (uint32_t f0 = 0; f0 < F; f0 += 128) {
                    uint8_t fl[4];
                    double gn[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t f = f0 + 32u * q + lane;
                        fl[q] = f < F ? __ldcg(flags + f) : 0;
                        gn[q] = f < F ? __ldcg(gains + f) : 0.0;
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t f = f0 + 32u * q + lane;
                        if (f >= F) continue;
                        rowc[f] = static_cast<uint8_t>((fl[q] >> 1) & 1);
                        if (fl[q] & 1) {
                            const double g = gn[q] != gn[q] ? -INFINITY : gn[q];  // `better` reads NaN as -inf
                            if (!found || g > bg) {  // features rise with f: on equal gains the earlier stays
                                found = 1;
                                bg = g;
                                bf = static_cast<int32_t>(f);
                            }
                        }
                    }
                }
                for (int o = 16; o > 0; o >>= 1) {
                    const int of = __shfl_xor_sync(0xffffffffu, found, o);
                    const double og = __shfl_xor_sync(0xffffffffu, bg, o);
                    const int32_t obf = __shfl_xor_sync(0xffffffffu, bf, o);
                    if (of && (!found || og > bg || (og == bg && obf < bf))) {
                        found = 1;
                        bg = og;
                        bf = obf;
                    }
                }
                if (found && lane == 0) {
                    best = load_candidate(candidates + static_cast<size_t>(2 * j + ch) * F + bf);
                    fs.child_feat[j][ch] = a.d.features[bf];
                }
            } else {
                for (uint32_t f = lane; f < F; f += 32) rowc[f] = 0;
            }
            if (lane == 0) {
                const bool has = best.found && sc[j].ctx[ch].valid;
                fs.child[j][ch].has_best = has;
                if (has) fs.child[j][ch].best = finish(sc[j].ctx[ch], best, a.cfg);
            }
        }
    }
    __syncthreads();

    // The commit rule and the next step's splits (warp 0; every CTA takes the same decisions).
    const int32_t N = st[0].root ? 0 : st[0].new_leaf;  // leaves before the step
    if (warp == 0) {
        // Split j commits when the ones before it did and none of their children comes before its leaf: lane
        // 2 i + c tests child c of split i against every later split.
        int committed = 1;
        if (!st[0].root) {
            uint32_t beaten = 0;  // bit j: a child of an earlier split comes before split j's leaf
            if (lane < static_cast<uint32_t>(2 * n)) {
                const int i = static_cast<int>(lane) / 2, c = static_cast<int>(lane) % 2;
                if (fs.child[i][c].has_best) {
                    const double cg = fs.child[i][c].best.gain;
                    const int32_t ci = child_index(st[i], c);
                    for (int j = i + 1; j < n; ++j)
                        if (ranks_before(cg, ci, st[j].info.gain, st[j].leaf)) beaten |= 1u << j;
                }
            }
            beaten = __reduce_or_sync(0xffffffffu, beaten);
            for (int j = 1; j < n; ++j) {
                if (((beaten >> j) & 1u) || !(st[j].info.gain > 0.0) || N + j >= a.max_leaves) break;
                ++committed;
            }
        }
        // The leaves after the committed splits, one per lane (kPool* codes), ranked kSplits times.
        const int32_t leaves_after = st[0].root ? 1 : N + committed;
        double pg = -INFINITY;
        int32_t pl = -1;
        if (lane < static_cast<uint32_t>(kSplits)) {
            pg = fs.other_gain[lane];
            pl = fs.other_leaf[lane];
        } else if (lane < static_cast<uint32_t>(kPoolPending)) {
            const int i = static_cast<int>(lane - kPoolChild) / 2, c = static_cast<int>(lane - kPoolChild) % 2;
            if (i < committed && c < children && fs.child[i][c].has_best) {
                pg = fs.child[i][c].best.gain;
                pl = child_index(st[i], c);
            }
        } else if (lane < static_cast<uint32_t>(kPoolPending + kSplits)) {
            const int j = static_cast<int>(lane) - kPoolPending;
            if (j >= committed && j < n) {
                pg = st[j].info.gain;
                pl = st[j].leaf;
            }
        }
        // Each leaf's rank: the leaves that come before it (a strict order: gains are numbers or -inf, indices
        // distinct). The next step takes the first ranks while their gains are positive and leaves may be added
        // (and never more splits than the grid has CTAs: each takes at least one).
        int rank = 0;
        for (int q = 0; q < 32; ++q) {
            const double og = __shfl_sync(0xffffffffu, pg, q);
            const int32_t ol = __shfl_sync(0xffffffffu, pl, q);
            rank += ol >= 0 && ranks_before(og, ol, pg, pl);
        }
        const int positive = __popc(__ballot_sync(0xffffffffu, pl >= 0 && pg > 0.0));
        const int room = a.max_leaves - leaves_after;
        int next_n = min(min(positive, kSplits), min(room, static_cast<int>(gridDim.x)));
        next_n = max(next_n, 0);
        if (pl >= 0 && rank < next_n) {
            fs.next_from[rank] = static_cast<int32_t>(lane);
            fs.next[rank].leaf = pl;  // the rest is filled below
        }
        if (lane == 0) {
            fs.committed = committed;
            fs.next_n = next_n;
        }
    }
    __syncthreads();
    const int committed = fs.committed;
    const int32_t leaves_after = st[0].root ? 1 : N + committed;

    // Writer CTAs: the tree (a lane per committed split), the committed children's records and rows; every CTA a
    // share of the spare slots of committed speculative splits, copied into their children's slots.
    if (writes_part(cta, 0) && warp == 0 && !st[0].root) {
        if (lane < static_cast<uint32_t>(committed)) {
            const int i = static_cast<int>(lane);
            const Step& s = st[i];
            if (sc[i].left_global <= 0 || sc[i].right_global <= 0) {
                a.iter->error = 1;  // split sends every row to one side (learner.rs:295-300)
                a.iter->error_info = s.leaf;
            }
            tree_split_at(a.tree, s.leaf, N + i, s.info, fs.split_feat[i], sc[i].left_global, sc[i].right_global,
                          it.spec.hess_scale, a.cfg.min_gain_to_split);
        }
        if (lane == 0) {
            const int32_t before = __ldcg(a.tree.num_leaves);
            if (before != N) {
                a.iter->error = 2;
                a.iter->error_info = before;
            }
            *a.tree.num_leaves = N + committed;
        }
    }
    if (writes_part(cta, 1) && warp == 0 && lane < static_cast<uint32_t>(2 * committed)) {
        const int i = static_cast<int>(lane) / 2, c = static_cast<int>(lane) % 2;
        if (c < children) {
            const int32_t leaf = child_index(st[i], c);
            const DevLeaf r = fs.child[i][c];
            a.leaves[leaf] = r;
            a.leaf_gain[leaf] = r.has_best ? r.best.gain : -INFINITY;
        }
    }
    if (writes_part(cta, 2) && warp < static_cast<uint32_t>(2 * n)) {
        // warp 2 i + c: child c of split i's splittable row, into the child's row when the split commits, else
        // (a split run here and dropped) into its leaf's PrepSplit rows
        const int i = static_cast<int>(warp) / 2, c = static_cast<int>(warp) % 2;
        const uint8_t* src = csplit + static_cast<size_t>(2 * i + c) * F;
        uint8_t* row = nullptr;
        if (c < children && i < committed)
            row = a.splittable + static_cast<size_t>(child_index(st[i], c)) * F;
        else if (c < children && !st[i].prepared && !st[0].root)
            row = a.prep_split + (2 * static_cast<size_t>(st[i].leaf) + c) * F;
        if (row)
            for (uint32_t f = lane; f < F; f += 32) row[f] = src[f];
    }
    // The children's bins of each committed split that did not write them in place (a speculative split, or a
    // prepared one: child_slot), copied from its leaf's prepared slots into the children's slots by every CTA.
    {
        const size_t slot_len = a.total_bins;  // [g, h] pairs
        const size_t total = static_cast<size_t>(committed) * 2 * slot_len;
        for (size_t q = static_cast<size_t>(cta) * blockDim.x + threadIdx.x; q < total;
             q += static_cast<size_t>(gridDim.x) * blockDim.x) {
            const int i = static_cast<int>(q / (2 * slot_len)), c = static_cast<int>(q / slot_len) % 2;
            if ((i == 0 && !st[i].prepared) || st[i].root || !sc[i].searched) continue;
            const size_t e = q % slot_len;
            const int2* src = reinterpret_cast<const int2*>(a.slots) + prep_slot(a, st[i].leaf, c) * slot_len;
            int2* dst = reinterpret_cast<int2*>(a.slots) + static_cast<size_t>(child_index(st[i], c)) * slot_len;
            __stcg(dst + e, __ldcg(src + e));
        }
    }
    // PrepSplit records: a committed split's leaf has none (its index now names its left child); a split run here
    // and dropped keeps its left count, children and their rows for the step that commits it.
    if (writes_part(cta, 1) && warp == 1 && lane < static_cast<uint32_t>(n) && !st[0].root) {
        const int j = static_cast<int>(lane);
        PrepSplit* rec = a.prep + st[j].leaf;
        if (j < committed) {
            rec->valid = 0;
        } else if (!st[j].prepared) {
            rec->may_search = st[j].may_search;
            rec->left = fs.left[j];
            rec->child[0] = fs.child[j][0];
            rec->child[1] = fs.child[j][1];
            rec->valid = 1;
        }
    }


    // The next step's splits: their records, steps and features (learner.rs:249-286).
    const int next_n = fs.next_n;
    if (warp < static_cast<uint32_t>(next_n)) {
        const int k = static_cast<int>(warp);
        const int src = fs.next_from[k];
        const int32_t leaf_index = fs.next[k].leaf;
        const DevLeaf* rec;
        const DevFeature* feat;
        const uint8_t* split_ok;
        if (src < kPoolChild) {
            rec = &fs.other[src];
            feat = &fs.other_feat[src];
            split_ok = osplit + static_cast<size_t>(src) * F;
        } else if (src < kPoolPending) {
            rec = &fs.child[(src - kPoolChild) / 2][(src - kPoolChild) % 2];
            feat = &fs.child_feat[(src - kPoolChild) / 2][(src - kPoolChild) % 2];
            split_ok = csplit + static_cast<size_t>(src - kPoolChild) * F;
        } else {
            rec = &fs.pending[src - kPoolPending];
            feat = &fs.split_feat[src - kPoolPending];  // a pending leaf's best split is the step's split
            split_ok = psplit + static_cast<size_t>(src - kPoolPending) * F;
        }
        uint8_t* ev = eval + static_cast<size_t>(k) * F;
        for (uint32_t f = lane; f < F; f += 32) ev[f] = static_cast<uint8_t>(mask[f] && split_ok[f]);
        if (lane == 0) {
            Step nx = next_step(a, *rec, leaf_index, leaves_after + k, *feat);
            // Its work is kept (PrepSplit) when an earlier step ran it and dropped it, and its children were searched
            // then exactly when they are now, or then but no longer (fewer leaves left: they are searched no more).
            int kept = -1;  // the may_search it ran under, -1: not run
            if (src >= kPoolPending) {
                const Step& was = st[src - kPoolPending];
                kept = was.prepared ? __ldcg(&a.prep[leaf_index].may_search) : was.may_search;
            } else if (src < kPoolChild && __ldcg(&a.prep[leaf_index].valid)) {
                kept = __ldcg(&a.prep[leaf_index].may_search);
            }
            nx.prepared = kept >= 0 && (kept == nx.may_search || (kept != 0 && !nx.may_search));
            fs.next[k] = nx;
        }
    }
    __syncthreads();
    if (threadIdx.x < static_cast<uint32_t>(kSplits)) {
        const int k = static_cast<int>(threadIdx.x);
        if (k < next_n) {
            st[k] = fs.next[k];
        } else {
            st[k].active = 0;
        }
    }
    if (threadIdx.x == 0) n = next_n;
    __syncthreads();
}

}  // namespace sb2
