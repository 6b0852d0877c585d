// diag.cu — a measurement of the operation that bounds the histogram: `red.shared.add.u32` by a whole CTA with no
// global memory traffic, at the histogram's address patterns, so the histogram's atomic rate can be read against
// what the shared-memory atomic unit does alone.
//
// Each lane holds 64 bin bytes in registers (16 words, re-mixed every pass) and adds at word bin * 32 + lane of a
// 256-bin × 32-lane array, as a full tile of the histogram does (hist_device.cuh): 32 different banks per
// instruction. Pattern 0 gives every lane its own bins (the lanes' words sit in 32 different 128-byte rows of the
// array, as in a histogram of random rows); pattern 1 gives all lanes the same bin at each step (one 128-byte row
// per instruction). 512 threads a CTA, one CTA per SM (128 KiB of dynamic shared memory), every SM busy.
#include <cuda_runtime.h>

#include <cstdint>

namespace sb2 {

namespace {

constexpr int kDiagThreads = 512;
constexpr uint32_t kDiagArrays = 4;  // 4 arrays of 256 x 32 words: 128 KiB

__global__ void __launch_bounds__(kDiagThreads) shared_add_kernel(int pattern, uint32_t passes,
                                                                  unsigned long long* cycles, uint32_t* sink) {
    extern __shared__ __align__(128) uint32_t arr[];
    for (uint32_t i = threadIdx.x; i < kDiagArrays * 256 * 32; i += kDiagThreads) arr[i] = 0;
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // 64 bin bytes per lane: pattern 0 seeds per lane, pattern 1 the same for every lane of the CTA
    uint32_t w[16];
    uint32_t x = 0x9E3779B9u * (1u + (pattern == 0 ? threadIdx.x : warp)) + blockIdx.x;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        x ^= x << 13;
        x ^= x >> 17;
        x ^= x << 5;
        w[j] = x;
    }
    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(arr)) +
                          (warp % kDiagArrays) * (256u * 32u * 4u) + 4u * lane;
    __syncthreads();
    const long long t0 = clock64();
    for (uint32_t p = 0; p < passes; ++p) {
#pragma unroll
        for (int s = 0; s < 64; ++s) {
            const uint32_t bin = (w[s >> 2] >> (8 * (s & 3))) & 0xFFu;
            asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(base + bin * 128u), "r"(1u));
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = __funnelshift_l(w[j], w[(j + 1) & 15], 7) + 0x6D2B79F5u;
    }
    __syncthreads();
    const long long t1 = clock64();
    if (threadIdx.x == 0) atomicAdd(cycles, static_cast<unsigned long long>(t1 - t0));
    // keep the adds: one word of the array per CTA
    if (threadIdx.x == 0) sink[blockIdx.x] = arr[blockIdx.x % (kDiagArrays * 256 * 32)];
}

}  // namespace

// Runs the measurement on the current device with `ctas` CTAs; *adds = lane adds made, *cycles = SM clock cycles
// summed over the CTAs, *seconds = the launch's duration (CUDA events).
cudaError_t time_shared_adds(int pattern, int ctas, uint32_t passes, cudaStream_t stream, double* adds, double* cycles,
                             double* seconds) {
    const int smem = static_cast<int>(kDiagArrays * 256 * 32 * 4);
    cudaError_t e = cudaFuncSetAttribute(shared_add_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    unsigned long long* d_cycles = nullptr;
    uint32_t* d_sink = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    if ((e = cudaMalloc(&d_cycles, sizeof(unsigned long long))) != cudaSuccess) return e;
    if ((e = cudaMalloc(&d_sink, sizeof(uint32_t) * ctas)) != cudaSuccess) {
        cudaFree(d_cycles);
        return e;
    }
    unsigned long long h_cycles = 0;
    float ms = 0.0f;
    cudaEventCreate(&ev[0]);
    cudaEventCreate(&ev[1]);
    for (int rep = 0; rep < 2 && e == cudaSuccess; ++rep) {  // the first launch warms up
        cudaMemsetAsync(d_cycles, 0, sizeof(unsigned long long), stream);
        cudaEventRecord(ev[0], stream);
        shared_add_kernel<<<ctas, kDiagThreads, smem, stream>>>(pattern, passes, d_cycles, d_sink);
        cudaEventRecord(ev[1], stream);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaMemcpyAsync(&h_cycles, d_cycles, sizeof(h_cycles), cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, ev[0], ev[1]);
    }
    cudaEventDestroy(ev[0]);
    cudaEventDestroy(ev[1]);
    cudaFree(d_cycles);
    cudaFree(d_sink);
    *adds = static_cast<double>(ctas) * kDiagThreads * 64.0 * passes;
    *cycles = static_cast<double>(h_cycles);
    *seconds = ms / 1000.0;
    return e;
}

}  // namespace sb2
