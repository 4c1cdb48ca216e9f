// Grid size of a grid-stride kernel: `per_sm` CTAs per SM of the current device, at most `need`.
#pragma once
#include <cuda_runtime.h>
#include <atomic>

namespace {

inline int stride_grid(long long need, int per_sm)
{
    static std::atomic<int> nsm{0};
    int n = nsm.load(std::memory_order_relaxed);
    if (n == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            n <= 0)
            n = 148;
        nsm.store(n, std::memory_order_relaxed);
    }
    const long long cap = (long long)n * per_sm;
    return (int)(need < cap ? need : cap);
}

}  // namespace
