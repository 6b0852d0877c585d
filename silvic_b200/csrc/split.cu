// split.cu — the split search as a standalone launch (the multi-GPU path), and the Backend API's split search;
// the device functions, and why their results are bit for bit the CPU search's, are in search.cuh.
#include <cuda_runtime.h>

#include "search.cuh"

namespace sb2 {

namespace {

// Every feature of the step's children, a warp each; the last CTA to finish applies the split and chooses the next.
__global__ void __launch_bounds__(kSearchThreads) search_kernel(TrainArgs a) {
    __shared__ int2 sh_hist[kSearchThreads / 32][kMaxBins];
    __shared__ uint16_t sh_order[kSearchThreads / 32][kMaxBins];
    __shared__ bool s_last;
    const Step st = *a.step;
    if (!st.active) return;
    const uint32_t warp = threadIdx.x >> 5;
    __shared__ SearchCtx s;
    search_context_cta(a, st, &s);
    if (s.searched)
        for (uint32_t item = blockIdx.x * (kSearchThreads / 32) + warp; item < search_items(a, st);
             item += gridDim.x * (kSearchThreads / 32))
            search_item(a, st, s, item, sh_hist[warp], sh_order[warp]);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(a.done_counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) *a.done_counter = 0;
    search_finish(a, st, s);
}

}  // namespace

void launch_search(const TrainArgs& a, int grid, cudaStream_t s) { search_kernel<<<grid, kSearchThreads, 0, s>>>(a); }

}  // namespace sb2

namespace sb2 {

namespace {

// split::find_best_split on a given histogram (the Backend API's split search): one warp per feature, then the last
// CTA reduces the candidates with `better` and writes SplitInfo and the splittable flags.
__global__ void __launch_bounds__(kSearchThreads) api_find_split_kernel(DevData d, const int* hist,
                                                                        const uint8_t* evaluate, double ug, double uh,
                                                                        int64_t count, double gs, double hs,
                                                                        sb2_split_config cfg, FeatureCandidate* cands,
                                                                        unsigned int* counter, sb2_split_info* out,
                                                                        uint8_t* splittable) {
    __shared__ int2 sh_hist[kSearchThreads / 32][kMaxBins];
    __shared__ uint16_t sh_order[kSearchThreads / 32][kMaxBins];
    __shared__ bool s_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t F = d.num_features;
    const Ctx x = make_ctx(cfg, gs, hs, ug, uh, count);
    for (uint32_t f = blockIdx.x * (kSearchThreads / 32) + warp; f < F; f += gridDim.x * (kSearchThreads / 32)) {
        const DevFeature feat = d.features[f];
        FeatureCandidate c{};
        c.feature = static_cast<int32_t>(f);
        if (evaluate[f] && feat.tile >= 0 && feat.num_bins > 0) {
            for (uint32_t b = lane; b < feat.num_bins; b += 32)
                sh_hist[warp][b] = make_int2(hist[2 * (feat.hist_offset + b)], hist[2 * (feat.hist_offset + b) + 1]);
            __syncwarp();
            c = scan_feature(sh_hist[warp], feat, static_cast<int>(f), x, cfg, sh_order[warp]);
            __syncwarp();
        }
        if (lane == 0) cands[f] = c;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last || warp != 0) return;
    __threadfence();
    FeatureCandidate best{};
    for (uint32_t f = lane; f < F; f += 32) {
        const FeatureCandidate c = load_candidate(cands + f);
        splittable[f] = static_cast<uint8_t>(c.splittable);
        if (better(c, best)) best = c;
    }
    best = best_of_warp(best, cands);
    if (lane == 0) {
        *counter = 0;
        sb2_split_info s{};
        if (best.found && x.valid) s = finish(x, best, cfg);
        *out = s;
    }
}

}  // namespace

void launch_api_find_split(const DevData& d, const int* hist, const uint8_t* evaluate, double ug, double uh,
                           int64_t count, double gs, double hs, const sb2_split_config& cfg, void* cands,
                           unsigned int* counter, sb2_split_info* out, uint8_t* splittable, int grid, cudaStream_t s) {
    api_find_split_kernel<<<grid, kSearchThreads, 0, s>>>(d, hist, evaluate, ug, uh, count, gs, hs, cfg,
                                                          static_cast<FeatureCandidate*>(cands), counter, out,
                                                          splittable);
}

}  // namespace sb2

