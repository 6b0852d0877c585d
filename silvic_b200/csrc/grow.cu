// grow.cu — one tree grown by one persistent kernel (Learner::grow, crates/silvic-core/src/learner.rs:121-169).
//
// A split step as separate launches costs a launch and a reload of the dataset's metadata per kernel, about 40 us
// of fixed time per split on small leaves, which dominates a 255-leaf tree. Here one cooperative launch (every CTA
// resident, one per SM) runs every step of the tree; its phases are separated by grid barriers:
//   root:   histogram -> [slab reduction] -> search -> finish
//   split:  partition flags -> scatter -> histogram of the smaller child -> [slab reduction] -> search -> finish
// (the slab reduction only for histograms through shared memory). Every CTA runs `finish` (apply the split, pick
// each child's best split, choose the next leaf) on the same inputs and reaches the same next step in its own
// shared memory; four CTAs write its results for later steps and kernels (search_finish_prepare). Work a CTA can do
// before the others reach a barrier (the next search's context, the finish's parts without candidates) runs between
// its arrival and its wait. The phases are the device functions of partition.cuh, hist_device.cuh and search.cuh,
// which the standalone kernels of the multi-GPU path also run.
//
// Every barrier wait is bounded: a CTA that waits longer than kBarrierSpins polls records an error in the
// iteration state and leaves the kernel, and every other CTA then leaves at its next barrier; the host reports the
// error. Data another CTA wrote in the same launch is read with ld.global.cg (past the SM's L1).
#include <cuda_runtime.h>

#include "fused.cuh"
#include "search.cuh"

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
    uint32_t flags_offset;        // bytes into the dynamic shared memory of the per-feature flags (5 F bytes)
    uint32_t scan_offset;         // ... of the partition's scan words (2 kHistThreads + 64), past the histogram
    uint32_t stage_offset;        // ... of the histogram's staging slots (16 warps x stage_depth x slot_bytes)
    uint32_t slot_bytes;
    uint32_t stage_depth;         // 0: no staging
    uint32_t pad_;
    GrowExchange x;               // the other ranks (world 1: none)
};

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31; }

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

__device__ __forceinline__ void clock_describe(const GrowArgs& g, PhaseClock& c, uint32_t job_rows, bool packed,
                                               uint32_t leaf_rows) {
    if (!clock_owner(g) || c.row == nullptr) return;
    c.row[kGrowPhases] = job_rows;
    c.row[kGrowPhases + 1] = packed;
    c.row[kGrowPhases + 2] = leaf_rows;
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
__device__ __forceinline__ void barrier_arrive(const GrowArgs& g, unsigned int& target) {
    target += gridDim.x;
    __syncthreads();  // the CTA's work (and its writes) are done
    // A release reduction: the CTA's writes are visible GPU-wide before its arrival is, and nothing waits for a
    // return value.
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(g.barrier) : "memory");
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
    // Every CTA keeps the learner's control state itself: the step, the evaluated features. The finish runs in
    // every CTA on the same inputs, so no CTA waits for another to publish the next step.
    __shared__ Step st;
    __shared__ HistJob root_job;
    __shared__ SearchCtx s;
    __shared__ FinishShared fs;
    __shared__ PhaseClock clock;
    __shared__ uint32_t s_left;
    uint32_t* scan = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(smem) + g.scan_offset);
    uint8_t* eval = reinterpret_cast<uint8_t*>(smem) + g.flags_offset;  // F: features this step searches
    uint8_t* mask = eval + F;                                            // F: the iteration's feature mask
    uint8_t* csplit = mask + F;                                          // 2 F: the children's splittable flags
    uint8_t* osplit = csplit + 2 * F;                                    // F: the best other leaf's
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
    // The root step, its job and features, as the iteration's start left them.
    broadcast_cg(a.step, &st);
    broadcast_cg(a.hist_job, &root_job);
    {
        const uint8_t* iter_mask = a.masks + static_cast<size_t>(a.iter->iteration) * F;
        for (uint32_t f = threadIdx.x; f < F; f += kGrowThreads) {
            eval[f] = a.evaluate[f];
            mask[f] = iter_mask[f];
        }
    }
    __syncthreads();

    for (int step = -1; step + 1 < a.max_leaves; ++step) {
        clock_step(g, clock, step);
        if (!st.active) break;
        // Phase A: the parent's partition and the built child's histogram into the slabs (the root: its histogram).
        FusedStep f{};
        f.root = st.root;
        f.count = st.root ? root_job.count : st.count;
        f.begin = st.root ? 0u : st.begin;
        f.src = st.which & 1;
        f.dst = f.src ^ 1u;
        f.built_left = st.built_left;
        f.histogram = st.root ? root_job.active != 0 : st.may_search != 0;
        f.chunks = fused_chunks(f.count, ctas);
        f.round_rows = round_rows;
        f.packed = fused_packed(f.count, f.chunks, round_rows);
        f.identity = !st.root && st.depth == 0;  // the root leaf's rows are still in row order
        f.stage = static_cast<uint32_t>(__cvta_generic_to_shared(smem)) + g.stage_offset;
        f.slot_bytes = g.slot_bytes;
        f.depth = g.stage_depth;
        unsigned int* cursor = a.cursors + 2 * (st.root ? 0 : st.new_leaf);
        clock_describe(g, clock, f.histogram ? f.count : 0u, f.packed, st.count);
        fused_step_cta(a, g.h, st, f, cta, smem, scan, cursor, eval, units, cached, &spare);
        clock_mark(g, clock, 0);
        if (!grid_barrier(g, target)) return;
        clock_mark(g, clock, 4);
        // The left count and the children's search context (every CTA: the finish is replicated), then the
        // search: one feature per CTA, its built child's bins reduced from the slabs and both children scanned.
        if (!st.root && threadIdx.x == 0) s_left = __ldcg(cursor);
        __syncthreads();
        const uint32_t epoch = g.x.epoch0 + static_cast<uint32_t>(step + 2);  // this step's, on every rank
        const bool ranks = g.x.world > 1;
        const uint8_t* evaluate = st.root ? mask : eval;  // the features this step searches (search_context's)
        int2* bufs = reinterpret_cast<int2*>(scan);
        // the reduction's scratch: the histogram's staging slots, free in this phase
        int4* scratch = g.stage_depth * (kGrowThreads / 32) * g.slot_bytes >= 16384
                            ? reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(smem) + g.stage_offset)
                            : nullptr;
        if (ranks && !st.root && cta == 0 && threadIdx.x < 32) publish_left(g.x, epoch, s_left);
        // With at most one feature per CTA, its bins (and their exchange) come first, so that the left counts'
        // exchange has arrived by the time the search context needs it.
        const bool early = f.histogram && F <= ctas;
        bool evaluated = false;
        if (early && cta < F &&
            !feature_bins_cta(a, g.h, cta, f.chunks, f.packed, evaluate, bufs, scratch, g.x, epoch, &evaluated))
            return;
        int64_t left_global = s_left;
        if (ranks && !st.root && !gather_left(g.x, epoch, &a.iter->error, &left_global)) return;
        if (warp == 0) {
            const SearchCtx c = search_context(a, st, st.root ? 0 : left_global, eval, mask);
            if (lane_id() == 0) s = c;
        }
        __syncthreads();
        clock_mark(g, clock, 1);
        if (s.searched) {
            if (early) {
                if (cta < F) feature_scan_cta(a, st, s, cta, evaluated, bufs, scan_shared);
            } else {
                for (uint32_t feature = cta; feature < F; feature += ctas) {
                    if (!feature_bins_cta(a, g.h, feature, f.chunks, f.packed, evaluate, bufs, scratch, g.x, epoch,
                                          &evaluated))
                        return;
                    feature_scan_cta(a, st, s, feature, evaluated, bufs, scan_shared);
                }
            }
        }
        clock_mark(g, clock, 2);
        barrier_arrive(g, target);
        // While the other CTAs finish their search: the parts of the finish that need no candidates.
        search_finish_prepare(a, st, s, st.root ? 0u : s_left, cta, osplit, fs);
        if (!barrier_wait(g, target)) return;
        clock_mark(g, clock, 4);
        search_finish_replicated(a, st, s, eval, mask, csplit, osplit, cta, fs);
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
    g.phase_ns = phase_ns;
    g.trace_steps = phase_ns ? trace_steps : 0;
    cudaError_t e = cudaMemsetAsync(barrier, 0, sizeof(unsigned int), s);  // nobody has arrived yet
    if (e != cudaSuccess) return e;
    // every step's placement cursors start at zero
    e = cudaMemsetAsync(t.cursors, 0, sizeof(unsigned int) * 2 * static_cast<size_t>(t.max_leaves), s);
    if (e != cudaSuccess) return e;
    void* args[] = {&g};
    return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(grow_tree_kernel), dim3(grid), dim3(kGrowThreads),
                                       args, static_cast<size_t>(smem.bytes), s);
}

}  // namespace sb2
