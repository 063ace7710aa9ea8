// C entry point around the reference launcher, for parity tests on a B200.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/build.py together with the
// reference's own projects/torch-sdf/cpp_src/kernel.cu (unmodified, from the
// reference tree) into oracle/_ref/libref_trace.so.  The reference kernel
// copies DAG words 0..1023 into shared memory whatever the payload size
// (kernel.cu:214-220); callers must pass a buffer of at least 1024 words.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernel.cuh"

extern "C" int ref_cast_rays(int device, const uint64_t* dag, const float* origins, const float* dirs,
                             float* out_d, int32_t* out_s, int num_rays, int max_steps,
                             float max_distance, const float* bmin, const float* bmax, int resolution)
{
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return static_cast<int>(e);
    toponav::cuda::launch_sphere_trace_kernel(dag, origins, dirs, out_d, out_s, num_rays, max_steps,
                                              max_distance, bmin, bmax, resolution);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int ref_synchronize(int device)
{
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return static_cast<int>(e);
}

extern "C" int ref_set_hit_epsilon(int, float) { return -1; }  // fixed at 0.01f in this build
