// Checks of tsdf::exit_quotient (exit_quotient.cuh) against the IEEE division __fdiv_rn,
// in libnavi_probe.so: exhaustive over slices of the binary32 significand pairs, and
// sampled over exponents and signs.  Both only count and report mismatches.
#include <cuda_runtime.h>

#include <cstdint>

#include "exit_quotient.cuh"

namespace {

constexpr int kPairsPerThread = 1 << 13;   // dividend significands per thread of the exhaustive check
constexpr int kDividendChunks = (1 << 23) / kPairsPerThread;

__device__ void record(unsigned long long* out, float a, float d)
{
    if (atomicAdd(&out[0], 1ull) == 0ull)
        out[1] = (static_cast<unsigned long long>(__float_as_uint(a)) << 32) | __float_as_uint(d);
}

// Thread (j, c): divisor significand d_first + j, dividends of chunk c; a, d in [1, 2).
__global__ void __launch_bounds__(256) exhaustive_kernel(uint32_t d_first, uint32_t d_count,
                                                         unsigned long long* __restrict__ out)
{
    const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (tid >= static_cast<uint64_t>(d_count) * kDividendChunks) return;
    const uint32_t j = static_cast<uint32_t>(tid / kDividendChunks);
    const uint32_t c = static_cast<uint32_t>(tid % kDividendChunks);
    const float d = __uint_as_float(0x3F800000u | (d_first + j));
    const float r = __frcp_rn(d);
    unsigned int bad = 0;
    uint32_t first = 0;
#pragma unroll 4
    for (int k = 0; k < kPairsPerThread; ++k) {
        const uint32_t m = c * kPairsPerThread + k;
        const float a = __uint_as_float(0x3F800000u | m);
        const float t = tsdf::exit_quotient(a, d, r, __fmul_rn(a, r));
        const bool miss = __float_as_uint(t) != __float_as_uint(__fdiv_rn(a, d));
        first = (miss && bad == 0) ? m : first;
        bad += miss ? 1u : 0u;
    }
    if (bad) {
        record(out, __uint_as_float(0x3F800000u | first), d);
        if (bad > 1) atomicAdd(&out[0], static_cast<unsigned long long>(bad) - 1ull);
    }
}

__device__ __forceinline__ uint64_t mix64(uint64_t x)
{
    x ^= x >> 30;
    x *= 0xBF58476D1CE4E5B9ull;
    x ^= x >> 27;
    x *= 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// The kernel's exit distance for one axis: the quotient, by the IEEE division for divisors
// of 2^126 and above, capped at 1000 by fminf (which drops a NaN from an overflowed
// approximate quotient) and floored at 1e-4.
__device__ __forceinline__ float clamped_exit(float a, float d, float r, float q0)
{
    const float t = fabsf(d) < tsdf::kQuotientMaxDivisor ? tsdf::exit_quotient(a, d, r, q0) : __fdiv_rn(a, d);
    return fmaxf(fminf(t, 1000.0f), 1e-4f);
}

// Pair i: random significands and signs, |a| = 2^[-126, 127], |d| = 2^[-13, 127] above 1e-4.
// out[0]/[1]: mismatches of the quotient where it is claimed exact (|d| < 2^126 and
// 2^-64 <= |a / d| < 2^127); out[2]/[3]: mismatches of the clamped exit distance where a
// and d have the same sign (the exit face lies ahead of the ray).
__global__ void __launch_bounds__(256) scaled_kernel(uint64_t seed, uint64_t n, unsigned long long* __restrict__ out)
{
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t h = mix64(seed ^ mix64(i));
        const uint64_t g = mix64(h + 0x9E3779B97F4A7C15ull);
        const uint32_t ea = 1u + static_cast<uint32_t>((h >> 23) % 254u);     // biased exponent 1..254
        const uint32_t ed = 114u + static_cast<uint32_t>((g >> 23) % 141u);   // 2^-13 .. 2^127
        const float a = __uint_as_float(static_cast<uint32_t>(h & 0x7FFFFFu) | (ea << 23) |
                                        (static_cast<uint32_t>(h >> 40) & 0x80000000u));
        const float d = __uint_as_float(static_cast<uint32_t>(g & 0x7FFFFFu) | (ed << 23) |
                                        (static_cast<uint32_t>(g >> 40) & 0x80000000u));
        if (!(fabsf(d) > 1e-4f)) continue;
        const float r = __frcp_rn(d);
        const float q0 = __fmul_rn(a, r);
        const float q = __fdiv_rn(a, d);
        const float aq = fabsf(q);
        if (fabsf(d) < tsdf::kQuotientMaxDivisor && aq >= 0x1p-64f && aq < 0x1p127f &&
            __float_as_uint(tsdf::exit_quotient(a, d, r, q0)) != __float_as_uint(q))
            record(out, a, d);
        if ((a < 0.0f) == (d < 0.0f) &&
            __float_as_uint(clamped_exit(a, d, r, q0)) != __float_as_uint(fmaxf(fminf(q, 1000.0f), 1e-4f)))
            record(out + 2, a, d);
    }
}

}  // namespace

extern "C" {

// Exhaustive check over divisor significands [d_first, d_first + d_count) (of 2^23) and
// all 2^23 dividend significands.  out: device, 2 words, accumulated: the mismatch count
// and the first mismatch seen (a bits << 32 | d bits).  Returns 0 or a cudaError_t.
int navi_check_exit_quotient(uint32_t d_first, uint32_t d_count, unsigned long long* out, void* stream)
{
    if (!out || d_first >= (1u << 23) || d_count == 0 || d_count > (1u << 23) - d_first) return cudaErrorInvalidValue;
    const uint64_t threads = static_cast<uint64_t>(d_count) * kDividendChunks;
    const unsigned blocks = static_cast<unsigned>((threads + 255u) / 256u);
    exhaustive_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_first, d_count, out);
    return static_cast<int>(cudaGetLastError());
}

// Sampled check over exponents and signs: n pairs from `seed`.  out: device, 4 words,
// accumulated (exact-quotient mismatches and the first; clamped-exit mismatches and the
// first).  Returns 0 or a cudaError_t.
int navi_check_exit_quotient_scaled(uint64_t seed, uint64_t n, unsigned long long* out, int blocks, void* stream)
{
    if (!out || blocks <= 0) return cudaErrorInvalidValue;
    scaled_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(seed, n, out);
    return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
