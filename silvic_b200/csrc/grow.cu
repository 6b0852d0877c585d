// grow.cu — one tree grown by one persistent kernel (Learner::grow, crates/silvic-core/src/learner.rs:121-169).
//
// A split step as separate launches costs a launch and a reload of the dataset's metadata per kernel, about 40 us
// of fixed time per split on small leaves, which dominates a 255-leaf tree. Here one cooperative launch (every CTA
// resident, one per SM) runs every step of the tree, in grid steps of up to kSplits splits (the best leaf's and,
// speculatively, the next ones', steps.cuh); a grid step's phases are separated by two grid barriers:
//   each split: partition of the parent -> histogram of the smaller child (fused.cuh), the splits side by side on
//               shares of the grid  |  the slab reductions and searches, one (split, feature) per CTA at a time
//               |  finish
// (the root: its histogram, its reduction and search, its finish). Every CTA runs the finish (commit the splits that
// hold, pick each child's best split, choose the next splits) on the same inputs and reaches the same next grid
// step in its own shared memory; three CTAs write its results for later steps and kernels. Work a CTA can do before
// the others reach a barrier (the first search item's reduction, the finish's parts without candidates) runs
// between its arrival and its wait.
//
// Every barrier wait is bounded: a CTA that waits longer than kBarrierSpins polls records an error in the
// iteration state and leaves the kernel, and every other CTA then leaves at its next barrier; the host reports the
// error. Data another CTA wrote in the same launch is read with ld.global.cg (past the SM's L1).
#include <cuda_runtime.h>

#include "fused.cuh"
#include "search.cuh"
#include "steps.cuh"

namespace sb2 {

namespace {

constexpr unsigned long long kBarrierSpins = 1ull << 26;  // ~3 s of 40 ns polls
constexpr int kGrowThreads = kHistThreads;                // 512: the histogram phase needs it

struct GrowArgs {
    TrainArgs t;
    HistArgs h;
    unsigned int* barrier;        // arrivals at grid barriers so far (zeroed before the launch)
    unsigned long long* phase_ns; // optional: nanoseconds spent per phase (kGrowPhases), summed over steps,
    int trace_steps;              // then per-step rows (kStepTrace) for this many steps
    uint32_t flags_offset;        // bytes into the dynamic shared memory of the per-feature flags ((5 kSplits + 1) F)
    uint32_t scan_offset;         // ... of the partition's scan words (2 kHistThreads + 64), past the histogram
    uint32_t stage_offset;        // ... of the histogram's staging slots (16 warps x stage_depth x slot_bytes)
    uint32_t slot_bytes;
    uint32_t stage_depth;         // 0: no staging
    float hist_weight;            // GrowSmem::hist_weight
    GrowExchange x;               // the other ranks (world 1: none)
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Phase clock of CTA 0's thread 0 (when profiling), kept in shared memory so it holds no registers across phases:
// mark(k) adds the time since the previous mark to phase k's total, and to the current step's trace row if any.
struct PhaseClock {
    unsigned long long* row;
    unsigned long long last;
};

__device__ __forceinline__ bool clock_owner(const GrowArgs& g) {
    return g.phase_ns != nullptr && blockIdx.x == 0 && threadIdx.x == 0;
}

__device__ __forceinline__ void clock_mark(const GrowArgs& g, PhaseClock& c, int k) {
    if (!clock_owner(g)) return;
    const unsigned long long now = global_ns();
    g.phase_ns[k] += now - c.last;
    if (c.row) c.row[k] += now - c.last;
    c.last = now;
}

// The trace row of step `step` (-1: the root).
__device__ __forceinline__ void clock_step(const GrowArgs& g, PhaseClock& c, int step) {
    if (!clock_owner(g)) return;
    c.row = step + 1 < g.trace_steps ? g.phase_ns + kGrowPhases + static_cast<size_t>(step + 1) * kStepTrace : nullptr;
}

// The grid step's sizes in its trace row: the rows of its histograms, the splits it runs and the ones it takes
// ready (the committed ones are added at its finish).
__device__ __forceinline__ void clock_describe(const GrowArgs& g, PhaseClock& c, uint32_t job_rows, uint32_t splits,
                                               uint32_t kept) {
    if (!clock_owner(g) || c.row == nullptr) return;
    c.row[kGrowPhases] = job_rows;
    c.row[kGrowPhases + 1] = splits;
    c.row[kGrowPhases + 3] = kept;
}

// `*p`, which another CTA may have written in this launch, copied into shared memory once per CTA (one 32-bit word
// per thread): every thread then reads the CTA's copy instead of all of them hitting the same L2 lines.
template <class T>
__device__ __forceinline__ void broadcast_cg(const T* p, T* shared_copy) {
    static_assert(sizeof(T) % 4 == 0 && sizeof(T) / 4 <= kHistThreads, "copied as 32-bit words, one per thread");
    __syncthreads();  // every thread is done with the previous copy
    if (threadIdx.x < sizeof(T) / 4)
        reinterpret_cast<unsigned int*>(shared_copy)[threadIdx.x] =
            __ldcg(reinterpret_cast<const unsigned int*>(p) + threadIdx.x);
    __syncthreads();
}

// Grid barriers count arrivals on one word that only grows during the launch (the host zeroes it before): a
// barrier is passed once the word reaches the running target, which every CTA advances identically by the grid
// size, so the last arrival itself releases the others and a barrier costs one atomic and the poll that sees it.
// The error word is polled alongside. Returns false once any CTA has recorded an error (or this one gave up).
// A barrier can be split: barrier_arrive, then CTA-local work that needs no other CTA's results (it overlaps the
// wait), then barrier_wait.
__device__ __forceinline__ void barrier_arrive(const GrowArgs& g, unsigned int& target, bool system = false) {
    target += gridDim.x;
    __syncthreads();  // the CTA's work (and its writes) are done
    // A release reduction: the CTA's writes are visible GPU-wide before its arrival is, and nothing waits for a
    // return value. `system`: the CTA also wrote other ranks' memory, which a system-scope fence orders first (the
    // rank's step flag, raised after the barrier, then covers those writes too).
    if (threadIdx.x == 0) {
        if (system) __threadfence_system();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(g.barrier) : "memory");
    }
}

__device__ bool barrier_wait(const GrowArgs& g, unsigned int target) {
    __shared__ int s_failed;
    if (threadIdx.x == 0) {
        volatile unsigned int* count = g.barrier;
        volatile int* error = &g.t.iter->error;
        unsigned long long spins = 0;
        int failed_now = 0;
        // `count - target` as a signed difference: the count never runs more than one barrier ahead of a waiter.
        while (true) {
            const unsigned int c = *count;
            failed_now = *error;
            if (failed_now != 0 || static_cast<int>(c - target) >= 0) break;
            if (++spins > kBarrierSpins) {
                atomicCAS(&g.t.iter->error, 0, 3);  // a CTA never arrived
                failed_now = 3;
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
        s_failed = failed_now;
    }
    __syncthreads();
    return !s_failed;
}

__device__ __forceinline__ bool grid_barrier(const GrowArgs& g, unsigned int& target) {
    barrier_arrive(g, target);
    return barrier_wait(g, target);
}

// How a grid step's splits share the grid in its first phase: split j takes `budget` CTAs from `base` (in
// proportion to its rows, at least one), of which `chunks` take part; its slabs hold packed sums when `packed`.
struct SplitPlan {
    uint32_t base, chunks, count;
    uint32_t packed;
};

__global__ void __launch_bounds__(kGrowThreads, 1) grow_tree_kernel(GrowArgs g) {
    extern __shared__ __align__(16) int smem[];
    const TrainArgs& a = g.t;
    const uint32_t cta = blockIdx.x, ctas = gridDim.x;
    const uint32_t warp = threadIdx.x >> 5;
    // The search's two groups of kScanWarps warps (one per child) and their scratch.
    constexpr uint32_t kGroups = kGrowThreads / kScanThreads;
    static_assert(kGroups == 2, "one scan group per child");
    __shared__ ScanShared scan_shared[kGroups];
    const uint32_t F = a.num_features;
    // Every CTA keeps the learner's control state itself: the grid step's splits and their features. The finish
    // runs in every CTA on the same inputs, so no CTA waits for another to publish the next step.
    __shared__ Step st[kSplits];
    __shared__ int s_n;  // splits of the grid step (0: the tree is done)
    __shared__ HistJob root_job;
    __shared__ SearchCtx sc[kSplits];
    __shared__ StepsFinish fs;
    __shared__ SplitPlan plan[kSplits];
    __shared__ PhaseClock clock;
    __shared__ uint32_t s_left[kSplits];          // this rank's left counts
    __shared__ int64_t s_left_global[kSplits];    // every rank's
    uint32_t* scan = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(smem) + g.scan_offset);
    uint8_t* eval = reinterpret_cast<uint8_t*>(smem) + g.flags_offset;  // kSplits rows of F: each split's features
    uint8_t* mask = eval + kSplits * F;                                  // F: the iteration's feature mask
    uint8_t* csplit = mask + F;                                          // 2 kSplits rows: the children's splittable
    uint8_t* osplit = csplit + 2 * kSplits * F;                          // kSplits rows: the best other leaves'
    uint8_t* psplit = osplit + kSplits * F;                              // kSplits rows: the split leaves'
    if (clock_owner(g)) clock = PhaseClock{nullptr, global_ns()};
    unsigned int target = 0;  // the barrier count that releases the next barrier (see grid_barrier)
    // The first units' descriptions, kept for the launch; later units are described per use.
    constexpr uint32_t kUnitCache = 2;
    __shared__ HistCta units[kUnitCache];
    __shared__ HistCta spare;
    const uint32_t cached = g.h.num_units < kUnitCache ? g.h.num_units : kUnitCache;
    for (uint32_t u = 0; u < cached; ++u) histogram_prepare_unit(g.h, u, smem, units + u);
    // The histogram's shared arrays start at zero; every flush leaves them so.
    for (uint32_t i = threadIdx.x; i < g.scan_offset / 16; i += kGrowThreads)
        reinterpret_cast<int4*>(smem)[i] = make_int4(0, 0, 0, 0);
    const uint32_t round_rows = packed_round_rows(*g.h.spec);  // the iteration's quantization, set before the launch
    const size_t flag_words = a.d.num_rows / 32 + 2;             // per split
    // The root step, its job and features, as the iteration's start left them.
    broadcast_cg(a.step, &st[0]);
    broadcast_cg(a.hist_job, &root_job);
    {
        const uint8_t* iter_mask = a.masks + static_cast<size_t>(a.iter->iteration) * F;
        for (uint32_t f = threadIdx.x; f < F; f += kGrowThreads) {
            eval[f] = a.evaluate[f];
            mask[f] = iter_mask[f];
        }
    }
    if (threadIdx.x == 0) s_n = st[0].active ? 1 : 0;
    // No leaf has a dropped split yet (the first finish that reads these records comes after two grid barriers).
    for (uint32_t l = cta * kGrowThreads + threadIdx.x; l < static_cast<uint32_t>(a.max_leaves); l += ctas * kGrowThreads)
        a.prep[l].valid = 0;
    __syncthreads();

    // Grid step gs (-1: the root) runs the splits st[0 .. n).
    for (int gs = -1; gs < a.max_leaves; ++gs) {
        clock_step(g, clock, gs);
        const int n = s_n;
        if (n == 0) break;
        // Phase A: each split's partition and built child's histogram into its slabs (the root: its histogram),
        // every CTA working on one split.
        if (warp == 0) {
            // Lane j plans split j. Its work: its partition, about one unit per parent row, and its histogram,
            // `hist_weight` units per built row (the built side's share of the split's rows, as the split's counts
            // estimate it).
            // In floats, summed in a fixed order: every CTA computes the same shares from the same steps. A prepared
            // split (its work kept from an earlier grid step) takes no CTA.
            const uint32_t lane = threadIdx.x & 31;
            const bool on = lane < static_cast<uint32_t>(n) && !st[lane].prepared;
            const uint32_t nw = __popc(__ballot_sync(0xffffffffu, on));  // the splits that work
            uint32_t count = 0;
            float w = 0.0f;
            bool hist = false;
            if (on) {
                const Step& sj = st[lane];
                count = sj.root ? root_job.count : sj.count;
                hist = sj.root ? root_job.active != 0 : sj.may_search != 0;
                const float c = static_cast<float>(count);
                const float l = sj.info.left_count > 0 ? static_cast<float>(sj.info.left_count) : 0.0f;
                const float r = sj.info.right_count > 0 ? static_cast<float>(sj.info.right_count) : 0.0f;
                w = !sj.root && sj.may_search && l + r > 0.0f ? c + g.hist_weight * c * (sj.built_left ? l : r) / (l + r) : c;
            }
            float total = w;
            for (int o = 16; o > 0; o >>= 1) total += __shfl_down_sync(0xffffffffu, total, o);
            total = __shfl_sync(0xffffffffu, total, 0);
            const float share = on && total > 0.0f ? static_cast<float>(ctas - nw) * (w / total) : 0.0f;
            const uint32_t budget = on ? 1u + min(static_cast<uint32_t>(share), ctas - nw) : 0u;
            uint32_t base = budget;  // inclusive prefix, then exclusive
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t up = __shfl_up_sync(0xffffffffu, base, o);
                if (lane >= static_cast<uint32_t>(o)) base += up;
            }
            base -= budget;
            if (on) {
                const uint32_t chunks = fused_chunks(count, budget);
                plan[lane] = SplitPlan{base, chunks, count, fused_packed(count, chunks, round_rows) ? 1u : 0u};
            } else if (lane < static_cast<uint32_t>(n)) {
                plan[lane] = SplitPlan{base, 0u, count, 0u};  // no CTA, no slab
            }
            const uint32_t hist_rows = __reduce_add_sync(0xffffffffu, hist ? count : 0u);
            if (lane == 0) clock_describe(g, clock, hist_rows, nw, static_cast<uint32_t>(n) - nw);
        }
        __syncthreads();
        int mine = -1;
        for (int j = 0; j < n; ++j)
            if (cta >= plan[j].base && cta < plan[j].base + plan[j].chunks) mine = j;
        if (mine >= 0) {
            const Step& sj = st[mine];
            FusedStep f{};
            f.root = sj.root;
            f.count = plan[mine].count;
            f.begin = sj.root ? 0u : sj.begin;
            f.src = sj.which & 1;
            f.dst = f.src ^ 1u;
            f.built_left = sj.built_left;
            f.histogram = sj.root ? root_job.active != 0 : sj.may_search != 0;
            f.chunks = plan[mine].chunks;
            f.round_rows = round_rows;
            f.packed = plan[mine].packed != 0;
            f.identity = !sj.root && sj.depth == 0;  // the root leaf's rows are still in row order
            f.stage = static_cast<uint32_t>(__cvta_generic_to_shared(smem)) + g.stage_offset;
            f.slot_bytes = g.slot_bytes;
            f.depth = g.stage_depth;
            unsigned int* cursor = a.cursors + 2 * (static_cast<size_t>(gs + 1) * kSplits + mine);
            fused_step_cta(a, g.h, sj, f, cta - plan[mine].base, cta, a.flags + mine * flag_words, smem, scan, cursor,
                           eval + static_cast<size_t>(mine) * F, units, cached, &spare);
        }
        clock_mark(g, clock, 0);
        if (!grid_barrier(g, target)) return;
        clock_mark(g, clock, 4);
        // The left counts and the splits' search contexts (every CTA: the finish is replicated), then the search:
        // items (split j, feature f) = j F + f, CTA c taking items c, c + ctas, ...: the built child's bins reduced
        // from the split's slabs and both children scanned.
        if (threadIdx.x < static_cast<uint32_t>(n)) {
            const Step& sj = st[threadIdx.x];
            s_left[threadIdx.x] = sj.root       ? 0u
                                  : sj.prepared ? __ldcg(&a.prep[sj.leaf].left)
                                                : __ldcg(a.cursors + 2 * (static_cast<size_t>(gs + 1) * kSplits + threadIdx.x));
        }
        __syncthreads();
        const uint32_t epoch = g.x.epoch0 + static_cast<uint32_t>(gs + 2);  // this grid step's, on every rank
        const bool ranks = g.x.world > 1;
        const ExchangeLayout L = exchange_layout(F, ranks ? static_cast<uint32_t>(g.x.world) : 1u);
        const CandidateSink sink = candidate_sink(a, g.x, L, epoch);
        int2* bufs = reinterpret_cast<int2*>(scan);
        // the reduction's scratch: the histogram's staging slots, free in this phase
        int4* scratch = g.stage_depth * (kGrowThreads / 32) * g.slot_bytes >= 16384
                            ? reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(smem) + g.stage_offset)
                            : nullptr;
        // While a CTA scans an item, the slab bins of its next item are copied into the staging slots past the
        // reduction's scratch (when they fit).
        const uint32_t pbuf = scratch != nullptr ? static_cast<uint32_t>(__cvta_generic_to_shared(scratch)) + 16384u : 0u;
        const uint32_t pcap = scratch != nullptr ? g.stage_depth * (kGrowThreads / 32) * g.slot_bytes - 16384u : 0u;
        if (ranks && !st[0].root && cta == 0 && threadIdx.x < 32) publish_left(g.x, L, epoch, s_left, n);
        const uint32_t items = static_cast<uint32_t>(n) * F;
        // Split j's built-child histogram was made in phase A (else there is nothing to reduce or exchange; a
        // prepared split's children were searched when it ran).
        auto built = [&](uint32_t j) {
            return st[j].root ? root_job.active != 0 : st[j].may_search != 0 && !st[j].prepared;
        };
        auto features_of = [&](uint32_t j) -> const uint8_t* { return st[j].root ? mask : eval + static_cast<size_t>(j) * F; };
        // Copies item i's slab bins ahead into pbuf (when they fit); true when it did.
        auto prefetch = [&](uint32_t i) {
            const uint32_t jn = i / F, fn = i % F;
            const DevFeature feat = a.d.features[fn];
            return pbuf != 0 && features_of(jn)[fn] && feat.tile >= 0 && feat.num_bins != 0 &&
                   prefetch_feature_bins(g.h, feat, plan[jn].base, plan[jn].chunks, plan[jn].packed != 0, pbuf, pcap);
        };
        bool have = false, evaluated = false;
        int2 parent = make_int2(0, 0);  // this thread's bin of the split's parent histogram (feature_bins_cta)
        if (ranks) {
            // Items of features another rank owns: this rank's built-child bins, reduced from its slabs, pushed to
            // the owner (they need no search context, so they run before the left counts are gathered).
            auto pushed = [&](uint32_t i) { return built(i / F) && owner_of(g.x, i % F) != g.x.rank; };
            uint32_t prefetched = 0xFFFFFFFFu;
            for (uint32_t i = cta; i < items; i += ctas) {
                if (!pushed(i)) continue;
                const uint32_t j = i / F, f = i % F;
                feature_bins_cta(a, g.h, st[j], j, f, plan[j].base, plan[j].chunks, plan[j].packed != 0, features_of(j),
                                 bufs, scratch, BinsMode::kPush, g.x, L, epoch, &evaluated, parent,
                                 prefetched == i ? pbuf : 0u);
                prefetched = 0xFFFFFFFFu;
                uint32_t next = i + ctas;
                while (next < items && !pushed(next)) next += ctas;
                if (next < items && prefetch(next)) prefetched = next;
            }
            if (prefetched != 0xFFFFFFFFu) cp_async_wait(0);  // nothing is left in flight
        } else if (cta < items) {
            // One rank: the CTA's first item's bins come before the contexts.
            const uint32_t j = cta / F, f = cta % F;
            if (built(j)) {
                feature_bins_cta(a, g.h, st[j], j, f, plan[j].base, plan[j].chunks, plan[j].packed != 0, features_of(j),
                                 bufs, scratch, BinsMode::kLocal, g.x, L, epoch, &evaluated, parent);
                have = true;
            }
        }
        // The left counts and the splits' search contexts (every CTA: the finish is replicated).
        if (ranks && !st[0].root) {
            if (!gather_left(g.x, L, epoch, n, &a.iter->error, s_left_global)) return;
        } else if (threadIdx.x < static_cast<uint32_t>(n)) {
            s_left_global[threadIdx.x] = s_left[threadIdx.x];
        }
        __syncthreads();
        if (warp < static_cast<uint32_t>(n)) {
            const SearchCtx c = search_context(a, st[warp], st[warp].root ? 0 : s_left_global[warp],
                                               eval + static_cast<size_t>(warp) * F, mask);
            if ((threadIdx.x & 31) == 0) sc[warp] = c;
        }
        __syncthreads();
        clock_mark(g, clock, 1);
        // The searches: every item (one rank) or the items of the features this rank owns, each with every rank's
        // bins added; items (split j, feature f) = j F + f, CTA c taking items c, c + ctas, ...
        auto searched = [&](uint32_t i) {
            return sc[i / F].searched && !st[i / F].prepared && (!ranks || owner_of(g.x, i % F) == g.x.rank);
        };
        const BinsMode mode = ranks ? BinsMode::kGather : BinsMode::kLocal;
        uint32_t prefetched = 0xFFFFFFFFu;  // the item whose bins are in pbuf
        for (uint32_t i = cta; i < items; i += ctas) {
            if (!searched(i)) continue;
            const uint32_t j = i / F, f = i % F;
            if (i != cta || !have) {
                if (!feature_bins_cta(a, g.h, st[j], j, f, plan[j].base, plan[j].chunks, plan[j].packed != 0,
                                      features_of(j), bufs, scratch, mode, g.x, L, epoch, &evaluated, parent,
                                      prefetched == i ? pbuf : 0u))
                    return;
            }
            prefetched = 0xFFFFFFFFu;
            uint32_t next = i + ctas;
            while (next < items && !searched(next)) next += ctas;
            if (next < items && prefetch(next)) prefetched = next;
            feature_scan_cta(a, st[j], sc[j], j, f, evaluated, parent, bufs, scan_shared, sink);
        }
        clock_mark(g, clock, 2);
        barrier_arrive(g, target, ranks);
        // While the other CTAs finish their search: the parts of the finish that need no candidates.
        steps_finish_prepare(a, st, n, sc, s_left, osplit, psplit, fs);
        if (!barrier_wait(g, target)) return;
        const FeatureCandidate* cands = static_cast<const FeatureCandidate*>(a.candidates);
        const uint8_t* cand_flags = a.cand_flags;
        const double* cand_gain = a.cand_gain;
        if (ranks) {
            // Every rank's candidates of the step are in this rank's arrays once every rank raised its step flag.
            if (cta == 0 && threadIdx.x < 32) publish_step(g.x, L, epoch);
            if (!wait_steps(g.x, L, epoch, &a.iter->error)) return;
            const uint8_t* own = g.x.peers[g.x.rank];
            const size_t set = candidate_set(L, epoch);
            cands = reinterpret_cast<const FeatureCandidate*>(own + L.candidates) + set;
            cand_flags = own + L.cand_flags + set;
            cand_gain = reinterpret_cast<const double*>(own + L.cand_gain) + set;
        }
        clock_mark(g, clock, 4);
        steps_finish(a, st, s_n, sc, eval, mask, csplit, osplit, psplit, cta, fs, cands, cand_flags, cand_gain);
        if (clock_owner(g) && clock.row) clock.row[kGrowPhases + 2] = static_cast<unsigned long long>(fs.committed);
        clock_mark(g, clock, 3);
    }
}

}  // namespace

int grow_threads() { return kGrowThreads; }

cudaError_t grow_configure(int smem_bytes, int* blocks_per_sm) {
    cudaError_t e = cudaFuncSetAttribute(grow_tree_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, grow_tree_kernel, kGrowThreads, smem_bytes);
}

int grow_static_smem() {
    cudaFuncAttributes attr{};
    if (cudaFuncGetAttributes(&attr, grow_tree_kernel) != cudaSuccess) return -1;
    return static_cast<int>(attr.sharedSizeBytes);
}

cudaError_t launch_grow_tree(const TrainArgs& t, const HistArgs& h, unsigned int* barrier, int grid,
                             const GrowSmem& smem, const GrowExchange& x, cudaStream_t s,
                             unsigned long long* phase_ns, int trace_steps) {
    GrowArgs g{};
    g.x = x;
    g.t = t;
    g.h = h;
    g.barrier = barrier;
    g.scan_offset = smem.scan_offset;
    g.stage_offset = smem.stage_offset;
    g.slot_bytes = smem.slot_bytes;
    g.stage_depth = smem.stage_depth;
    g.flags_offset = smem.flags_offset;
    g.hist_weight = smem.hist_weight;
    g.phase_ns = phase_ns;
    g.trace_steps = phase_ns ? trace_steps : 0;
    cudaError_t e = cudaMemsetAsync(barrier, 0, sizeof(unsigned int), s);  // nobody has arrived yet
    if (e != cudaSuccess) return e;
    // every split's placement cursors start at zero
    e = cudaMemsetAsync(t.cursors, 0, sizeof(unsigned int) * 2 * kSplits * (static_cast<size_t>(t.max_leaves) + 1), s);
    if (e != cudaSuccess) return e;
    void* args[] = {&g};
    return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(grow_tree_kernel), dim3(grid), dim3(kGrowThreads),
                                       args, static_cast<size_t>(smem.bytes), s);
}

}  // namespace sb2
