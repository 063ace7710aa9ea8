// Reference kernel with its hit epsilon made a run-time value.
//
// TEST INFRASTRUCTURE ONLY.  oracle/build.py copies kernel.cu and kernel.cuh
// from the reference tree into a scratch folder under oracle/_ref/, changes the
// one line `constexpr float kHitEpsilon = 0.01f;` (kernel.cuh:7) into a
// __constant__ variable, compiles this file (which includes that kernel.cu)
// and deletes the copies.  Nothing else of the kernel changes; the benchmark
// configurations use epsilon = 1e-3 x voxel size, which the unmodified build
// cannot express.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernel.cu"

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

extern "C" int ref_set_hit_epsilon(int device, float eps)
{
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(toponav::cuda::kHitEpsilon, &eps, sizeof(float));
    return static_cast<int>(e);
}
