// L2 read-bandwidth probe for the roofline of the benchmark (libnavi_probe.so).
//
// The trace kernels chase pointers through node pools that mostly stay in L2, so
// their roofline is the L2 read bandwidth, which the driver's measured peaks do not
// include.  This kernel reads an L2-resident buffer again and again with 16-byte
// loads that bypass L1 (ld.global.cg), several loads in flight per thread, and
// reports the bytes read; the host times it with CUDA events.
#include <cuda_runtime.h>

#include <cstdint>

namespace {

__global__ void __launch_bounds__(512) l2_read_kernel(const uint4* __restrict__ buf, uint64_t n16, int reps,
                                                      unsigned int* __restrict__ sink)
{
    constexpr int kUnroll = 8;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    unsigned int acc = 0;
    for (int r = 0; r < reps; ++r) {
        // each repetition starts at another block offset, so a block does not re-read
        // the same lines back to back
        const uint64_t start = (tid + static_cast<uint64_t>(r) * 7919u * blockDim.x) % n16;
        uint64_t i = start;
        for (uint64_t k = 0; k < n16; k += stride * kUnroll) {
            uint4 v[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                uint64_t j = i + static_cast<uint64_t>(u) * stride;
                j = j >= n16 ? j - n16 : j;
                v[u] = __ldcg(buf + j);
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
            i += stride * kUnroll;
            while (i >= n16) i -= n16;
        }
    }
    if (acc == 0x9E3779B9u) sink[0] = acc;  // keeps the loads; the buffer never produces this value
}

}  // namespace

extern "C" {

// Reads `bytes` bytes of `buf` (device, 16-byte aligned, a multiple of 16 bytes) `reps`
// times on `stream` with `blocks` blocks of 512 threads.  Returns 0 or a cudaError_t.
int navi_probe_l2_read(const void* buf, uint64_t bytes, int reps, int blocks, void* sink, void* stream)
{
    if (!buf || !sink || bytes < 16 || bytes % 16 != 0 || reps <= 0 || blocks <= 0) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(buf) % 16 != 0) return cudaErrorInvalidValue;
    l2_read_kernel<<<blocks, 512, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(buf), bytes / 16, reps, static_cast<unsigned int*>(sink));
    return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
