// hist.cu — quantized leaf histogram kernel (see hist.cuh).
#include <cuda_runtime.h>

#include "hist.cuh"

namespace sb2 {

namespace {

constexpr int kThreads = 512;
constexpr int kUnroll = 8;  // rows whose bins are in flight per warp before their atomics

struct LaneTile {
    const uint8_t* base;  // this lane's byte of the tile's row 0
    uint32_t stride;
    uint32_t slot;        // shared slot of (bin 0, this lane)
    bool on;              // the lane holds a wanted feature of this tile
};

__global__ void __launch_bounds__(kThreads) histogram_kernel(HistArgs a) {
    extern __shared__ long long sh[];
    const HistJob job = *a.job;
    if (!job.active || job.count == 0) return;
    const uint32_t unit_index = blockIdx.x % a.num_units;
    const uint32_t chunk = blockIdx.x / a.num_units;
    const uint32_t max_chunks = gridDim.x / a.num_units;
    uint32_t chunks = static_cast<uint32_t>(ceil_div(job.count, a.min_rows_per_cta));
    chunks = chunks < 1 ? 1 : (chunks > max_chunks ? max_chunks : chunks);
    if (chunk >= chunks) return;
    const uint32_t lo = static_cast<uint32_t>(static_cast<uint64_t>(job.count) * chunk / chunks);
    const uint32_t hi = static_cast<uint32_t>(static_cast<uint64_t>(job.count) * (chunk + 1) / chunks);

    const Unit unit = a.units[unit_index];
    for (uint32_t i = threadIdx.x; i < unit.slots; i += kThreads) sh[i] = 0;

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    constexpr int kWarps = kThreads / 32;
    LaneTile lt[kMaxUnitTiles];
    bool any_on = false;
    uint32_t slot = 0;
#pragma unroll
    for (int t = 0; t < kMaxUnitTiles; ++t) {
        lt[t].on = false;
        lt[t].base = a.d.bins;
        lt[t].stride = 0;
        lt[t].slot = 0;
        if (t < static_cast<int>(unit.num_tiles)) {
            const Tile tile = a.d.tiles[unit.first_tile + t];
            const int32_t f = a.d.lane_feature[(unit.first_tile + t) * kTileLanes + lane];
            lt[t].base = a.d.bins + tile.base + lane;
            lt[t].stride = tile.stride;
            lt[t].slot = slot + lane;
            lt[t].on = lane < static_cast<int>(tile.stride) && f >= 0 && (a.active == nullptr || a.active[f] != 0);
            slot += tile.smem_bins * tile.stride;
        }
        any_on |= lt[t].on;
    }
    __syncthreads();

    // Each warp adds a contiguous share of the chunk's rows, 32 positions per batch.
    const uint32_t span = hi - lo;
    const uint32_t per_warp = static_cast<uint32_t>(ceil_div(span, kWarps));
    const uint32_t w_lo = lo + min(span, per_warp * warp);
    const uint32_t w_hi = lo + min(span, per_warp * (warp + 1));
    const uint32_t* rows = a.rows[job.which & 1];
    const int32_t* ordered = a.ordered[job.which & 1];
    const bool warp_on = __any_sync(0xffffffffu, any_on);
    if (warp_on) {
        for (uint32_t p0 = w_lo; p0 < w_hi; p0 += 32) {
            const uint32_t n = min(32u, w_hi - p0);
            uint32_t my_row = 0;
            int32_t my_gh = 0;
            if (static_cast<uint32_t>(lane) < n) {
                const uint32_t pos = job.begin + p0 + lane;
                if (job.identity) {
                    my_row = pos;
                    my_gh = __ldg(a.packed + pos);
                } else {
                    my_row = __ldg(rows + pos);
                    my_gh = __ldg(ordered + pos);
                }
            }
            for (uint32_t r0 = 0; r0 < n; r0 += kUnroll) {
                uint32_t row[kUnroll];
                int32_t gh[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    row[u] = __shfl_sync(0xffffffffu, my_row, (r0 + u) & 31);
                    gh[u] = __shfl_sync(0xffffffffu, my_gh, (r0 + u) & 31);
                }
                uint8_t bin[kUnroll][kMaxUnitTiles];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
                    for (int t = 0; t < kMaxUnitTiles; ++t) {
                        bin[u][t] = 0;
                        if (lt[t].on && r0 + u < n)
                            bin[u][t] = __ldg(lt[t].base + static_cast<uint64_t>(row[u]) * lt[t].stride);
                    }
                }
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    if (r0 + u < n) {
                        const long long v = packed_to_wide(gh[u]);
#pragma unroll
                        for (int t = 0; t < kMaxUnitTiles; ++t) {
                            if (lt[t].on)
                                atomicAdd(reinterpret_cast<unsigned long long*>(sh + lt[t].slot + bin[u][t] * lt[t].stride),
                                          static_cast<unsigned long long>(v));
                        }
                    }
                }
            }
        }
    }
    __syncthreads();

    // Flush: every non-zero slot of a wanted feature into the output's [g, h] pair.
    for (uint32_t i = threadIdx.x; i < unit.slots; i += kThreads) {
        const long long v = sh[i];
        if (v == 0) continue;
        uint32_t local = i;
        uint32_t t = 0;
        uint32_t stride = 0;
#pragma unroll
        for (int k = 0; k < kMaxUnitTiles; ++k) {
            if (k < static_cast<int>(unit.num_tiles)) {
                const Tile tile = a.d.tiles[unit.first_tile + k];
                const uint32_t size = tile.smem_bins * tile.stride;
                if (stride == 0) {
                    if (local < size) {
                        t = unit.first_tile + k;
                        stride = tile.stride;
                    } else {
                        local -= size;
                    }
                }
            }
        }
        if (stride == 0) continue;
        const uint32_t bin = local / stride;
        const uint32_t ln = local % stride;
        const int32_t f = a.d.lane_feature[t * kTileLanes + ln];
        if (f < 0) continue;
        const DevFeature feat = a.d.features[f];
        if (bin >= feat.num_bins) continue;
        if (a.active != nullptr && a.active[f] == 0) continue;
        const int32_t g = static_cast<int32_t>(static_cast<uint32_t>(static_cast<unsigned long long>(v)));
        const int32_t h = static_cast<int32_t>((v - g) >> 32);
        int* o = a.out + 2 * (static_cast<size_t>(feat.hist_offset) + bin);
        if (g != 0) atomicAdd(o, g);
        if (h != 0) atomicAdd(o + 1, h);
    }
}

}  // namespace

int histogram_threads() { return kThreads; }

void launch_histogram(const HistArgs& a, int grid, int smem_bytes, cudaStream_t stream) {
    histogram_kernel<<<grid, kThreads, smem_bytes, stream>>>(a);
}

cudaError_t histogram_configure(int smem_bytes) {
    return cudaFuncSetAttribute(histogram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
}

cudaError_t histogram_occupancy(int smem_bytes, int* blocks_per_sm) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, histogram_kernel, kThreads, smem_bytes);
}

}  // namespace sb2
