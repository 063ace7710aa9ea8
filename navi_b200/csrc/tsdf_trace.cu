// Batched sphere trace over the re-packed .gmdag node pool, sm_100a.
//
// Semantics: exactly those of the reference sphere_trace_kernel
// (projects/torch-sdf/cpp_src/kernel.cu:203-309) and its stackless descent
// (kernel.cu:88-200), per ray: the same float operations in the same order,
// the same leaf / void / depth-4 prefix caches with the same inclusive or
// strict bounds, the same 32-level descent cap.  The hit epsilon is a
// parameter (0.01 in the reference) and the number of march iterations is an
// extra output.
//
// Execution: a persistent grid (four blocks of 256 per SM).  Each lane owns one
// ray and runs a small state machine; one loop iteration performs the start of a
// march step (position, cell indices and the cache tests, which may finish the
// step), up to four levels of DAG descent (one 4-byte load each), the caching
// of the cell a descent ended in (once per iteration, not per level), the exit
// distance of a void cell, and the end of the step with up to one more step
// in place inside a cached leaf cell.  Lanes whose ray has ended are refilled,
// two at a time, at the top of a later iteration from a warp-local range of ray
// indices; the warp claims ranges of `chunk` rays from a global counter with one
// atomicAdd, so short rays never leave lanes idle while long rays march on.
// Decisions that lanes of a warp take differently are written as selects
// wherever that measured faster than branches.  Around the trace:
// the claim order of single-scene launches (order_key_kernel,
// order_scatter_kernel), the scene sort of scene tables (scene_sort_kernel;
// tables of 2-64 scenes then take one single-scene launch per scene, larger
// ones the multi-scene kernel) and the observation pass (observe_kernel).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "exit_quotient.cuh"
#include "tsdf_internal.h"

namespace {

constexpr int kThreads = 256;
constexpr unsigned kFull = 0xFFFFFFFFu;
constexpr float kOutside = 1000.0f;      // kernel.cuh:8
constexpr float kDirEps = 1e-4f;         // kernel.cuh:9
constexpr float kVoidAdvance = 1e-5f;    // kernel.cu:9
constexpr int kPrefixDepth = 4;          // kernel.cuh:11
constexpr int kMaxDepth = 32;            // kernel.cu:136
constexpr int64_t kMaxRays = (1ll << 31) - (1ll << 24);

std::atomic<int64_t> g_smem_records{0};  // top records staged per block (the L1 serves them as well on sm_100)
std::atomic<int64_t> g_chunk{0};  // 0: pick_chunk chooses
std::atomic<int64_t> g_leaf_run{1};
std::atomic<int64_t> g_order{1};  // single-scene claim order: 0 ray index, 1 longest scene-box exit first
std::atomic<int64_t> g_blocks_per_sm{0};
std::atomic<int64_t> g_descent{0};  // 0: integer grid where possible, 1: float descent only

// lane flags
constexpr uint32_t kVoidOk = 1u;
constexpr uint32_t kLeafOk = 2u;
constexpr uint32_t kPreOk = 4u;
constexpr uint32_t kInDesc = 8u;
constexpr uint32_t kUsePre = 16u;

struct TraceArgs {
    TsdfSceneDev scene;          // single-scene launches
    const TsdfSceneDev* table;   // multi-scene launches
    const float* origins;        // explicit rays [n][3]
    const float* dirs;
    const float4* poses;         // fan rays: 2 float4 per actor (tsdf_pose)
    const float* fan;            // [rays_per_actor][3]
    uint32_t rays_per_actor;
    uint32_t rpa_magic;          // r / rays_per_actor = (r * rpa_magic) >> rpa_shift for r < 2^31
    uint32_t rpa_shift;
    int use_pitch;
    uint32_t n_rays;
    int max_steps;
    float max_distance;
    uint32_t n_smem;             // records staged in shared memory
    uint32_t chunk;
    uint32_t leaf_run;           // leaf-cache steps taken in place after a step (grid kernel)
    const uint32_t* perm;        // multi-scene fan launches: actors in scene order (or null)
    const uint32_t* ray_perm;    // single-scene launches: rays in claim order (or null)
    const uint32_t* seg;         // per-scene launch of a scene table: its actors are perm[seg[0], seg[1])
                                 // (device, written by scene_sort_kernel), or null
    uint32_t n_scenes;           // multi-scene fan launches: scene table size
    float* out_d;
    int32_t* out_s;
    int32_t* out_steps;
    unsigned int* counter;
    unsigned int* err;           // bounds-checked builds: error bits (word after the counter)
};

// Bounds-checked builds (TSDF_BOUNDS_CHECK, libnavi_tsdf_debug.so): every node-pool,
// leaf-table, stack and actor-order index is checked before it is used; a failed check
// sets a bit of the error word and the access is replaced by a harmless one (an empty
// octant, leaf 0, no stack write), so the launch finishes and the host reports the
// bits.  The pools are validated when they are built, so a set bit means a bug in
// this library.  In the regular build the checks compile to nothing.
#ifdef TSDF_BOUNDS_CHECK
constexpr bool kBoundsCheck = true;
#else
constexpr bool kBoundsCheck = false;
#endif
constexpr unsigned int kErrRecord = 1u, kErrLeafTable = 2u, kErrStack = 4u, kErrActor = 8u;

__device__ __forceinline__ bool checked(unsigned int* err, bool ok, unsigned int bit)
{
    if constexpr (kBoundsCheck) {
        if (!ok) {
            atomicOr(err, bit);
            return false;
        }
    }
    return true;
}

// Quotient by rays_per_actor without a division (Granlund and Montgomery, "Division by
// invariant integers using multiplication", 1994, theorem 4.2: for N-bit dividends, with
// l = ceil(log2 d) and m = ceil(2^(N+l) / d), floor(n / d) = floor(m n / 2^(N+l)); here
// N = 31, as ray indices are below 2^31, so m < 2^32).
__device__ __forceinline__ uint32_t div_rpa(const TraceArgs& a, uint32_t r)
{
    return static_cast<uint32_t>((static_cast<uint64_t>(r) * a.rpa_magic) >> a.rpa_shift);
}

// Ray `r`: explicit origin/direction, or fan ray (actor, local direction) with the
// reference's rotation (sdfdag_backend.py:1303-1310) and the optional pitch.
template <bool kFan>
__device__ __forceinline__ void load_ray(const TraceArgs& a, uint32_t r, float3& o, float3& d, int& scene)
{
    if constexpr (kFan) {
        const uint32_t actor = div_rpa(a, r);
        const uint32_t k = r - actor * a.rays_per_actor;
        const float4 p0 = __ldg(a.poses + 2 * static_cast<size_t>(actor));
        const float4 p1 = __ldg(a.poses + 2 * static_cast<size_t>(actor) + 1);
        float bx = __ldg(a.fan + 3 * static_cast<size_t>(k));
        float by = __ldg(a.fan + 3 * static_cast<size_t>(k) + 1);
        float bz = __ldg(a.fan + 3 * static_cast<size_t>(k) + 2);
        if (a.use_pitch) {
            const float yp = __fsub_rn(__fmul_rn(by, p1.y), __fmul_rn(bz, p1.z));
            const float zp = __fadd_rn(__fmul_rn(by, p1.z), __fmul_rn(bz, p1.y));
            by = yp;
            bz = zp;
        }
        d.x = __fadd_rn(__fmul_rn(bx, p0.w), __fmul_rn(bz, p1.x));
        d.y = by;
        d.z = __fadd_rn(__fmul_rn(-bx, p1.x), __fmul_rn(bz, p0.w));
        o = make_float3(p0.x, p0.y, p0.z);
        scene = __float_as_int(p1.w);
    } else {
        const float* po = a.origins + 3 * static_cast<size_t>(r);
        const float* pd = a.dirs + 3 * static_cast<size_t>(r);
        o = make_float3(__ldg(po), __ldg(po + 1), __ldg(po + 2));
        d = make_float3(__ldg(pd), __ldg(pd + 1), __ldg(pd + 2));
        scene = 0;
    }
}

// Work item w -> output ray.  Multi-scene fan launches take actors grouped by scene
// (perm, written by scene_sort_kernel), so that the warps of a block mostly trace one
// scene and the SM's L1 holds the hot records and grid lines of fewer scenes; a
// per-scene launch takes the actors perm[seg[0], seg[1]) of its scene; single-scene
// launches take rays in claim order (ray_perm).  Outputs stay actor-major.  The traced
// values do not depend on the order.
template <bool kFan, bool kMulti>
__device__ __forceinline__ uint32_t work_ray(const TraceArgs& a, uint32_t w, uint32_t seg_base)
{
    if constexpr (kFan && !kMulti) {
        if (a.seg) {
            if (a.ray_perm) {  // claim order of the scene's rays: a work item of the scene
                w = __ldg(a.ray_perm + seg_base * a.rays_per_actor + w);
                if (!checked(a.err, w < a.n_rays, kErrActor)) w = 0;
            }
            const uint32_t slot = div_rpa(a, w);
            uint32_t actor = __ldg(a.perm + seg_base + slot);
            if (!checked(a.err, actor < a.n_rays / a.rays_per_actor, kErrActor)) actor = 0;
            return actor * a.rays_per_actor + (w - slot * a.rays_per_actor);
        }
    }
    if constexpr (!kMulti) {
        if (a.ray_perm) {
            const uint32_t r = __ldg(a.ray_perm + w);
            return checked(a.err, r < a.n_rays, kErrActor) ? r : 0u;
        }
    }
    if constexpr (kFan && kMulti) {
        if (a.perm) {
            const uint32_t slot = div_rpa(a, w);
            uint32_t actor = __ldg(a.perm + slot);
            if (!checked(a.err, actor < a.n_rays / a.rays_per_actor, kErrActor)) actor = 0;
            return actor * a.rays_per_actor + (w - slot * a.rays_per_actor);
        }
    }
    return w;
}

// Counting sort of the actors by scene index, one block: perm[i] = the i-th actor in
// scene order (scenes ascending, actors of one scene in arbitrary order; indices outside
// [0, n_scenes) last).  seg (may be null) receives the n_scenes + 2 bounds: scene b's
// actors are perm[seg[b], seg[b + 1]), those of no scene perm[seg[n_scenes], n_actors).
__global__ void __launch_bounds__(1024) scene_sort_kernel(const float4* __restrict__ poses, uint32_t n_actors,
                                                          uint32_t n_scenes, uint32_t* __restrict__ perm,
                                                          uint32_t* __restrict__ seg)
{
    extern __shared__ unsigned int bucket[];  // [n_scenes + 1]
    for (uint32_t i = threadIdx.x; i <= n_scenes; i += blockDim.x) bucket[i] = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < n_actors; i += blockDim.x) {
        const uint32_t sc = static_cast<uint32_t>(__float_as_int(__ldg(poses + 2 * static_cast<size_t>(i) + 1).w));
        atomicAdd(&bucket[sc < n_scenes ? sc : n_scenes], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned int run = 0;
        for (uint32_t b = 0; b <= n_scenes; ++b) {
            const unsigned int c = bucket[b];
            bucket[b] = run;
            if (seg) seg[b] = run;
            run += c;
        }
        if (seg) seg[n_scenes + 1] = run;
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < n_actors; i += blockDim.x) {
        const uint32_t sc = static_cast<uint32_t>(__float_as_int(__ldg(poses + 2 * static_cast<size_t>(i) + 1).w));
        perm[atomicAdd(&bucket[sc < n_scenes ? sc : n_scenes], 1u)] = i;
    }
}

// Rays of the actors whose scene index is outside the table, in a per-scene traced
// scene table: not traced (NaN distance, semantic 0, 0 steps), as the multi-scene kernel
// leaves them.  seg points at the bounds [seg[0], seg[1]) of those actors in perm.
__global__ void __launch_bounds__(256) unknown_scene_kernel(const uint32_t* __restrict__ seg,
                                                            const uint32_t* __restrict__ perm, uint32_t n_actors,
                                                            uint32_t rays_per_actor, float* __restrict__ out_d,
                                                            int32_t* __restrict__ out_s, int32_t* __restrict__ out_steps)
{
    const uint32_t lo = __ldg(seg), hi = min(__ldg(seg + 1), n_actors);
    if (lo >= hi) return;
    const uint64_t n = static_cast<uint64_t>(hi - lo) * rays_per_actor;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t actor = __ldg(perm + lo + i / rays_per_actor);
        if (actor >= n_actors) continue;
        const uint64_t ray = static_cast<uint64_t>(actor) * rays_per_actor + i % rays_per_actor;
        out_d[ray] = __int_as_float(0x7fc00000);
        out_s[ray] = 0;
        if (out_steps) out_steps[ray] = 0;
    }
}

// Epilogue of a finished ray (kernel.cu:298-308).
__device__ __forceinline__ void finish_ray(const TraceArgs& a, uint32_t ray, float dist_out, int32_t sem_out,
                                           int32_t steps)
{
    a.out_d[ray] = dist_out;
    a.out_s[ray] = sem_out;
    if (a.out_steps) a.out_steps[ray] = steps;
}

// Settings of the observation pass (tsdf_observe plus the derived constants).
struct ObserveArgs {
    uint32_t rays_per_actor;
    uint32_t el_bins;
    uint32_t az_bins;
    uint32_t fwd_half;           // forward sector: azimuth rows [0, fwd_half) and [az - fwd_half, az)
    float max_distance;
    float sat_thr;               // float32(max_distance - 1e-3)
    float band_min, band_max;
    float prox;
    float inv_log_denom;         // float32(1 / log1p(max_distance)) (reciprocal formed in double)
    float f_all, f_fwd;          // torch's mean factors: float(A) / float(A * N)
    int band_on, prox_on;
};

// The reference's post-processing of a fan cast, one block per actor over the actor's
// finished rays: clamp to [0, max], depth = clamp(log1p(d) / log1p(max), 0, 1), valid =
// isfinite (sdfdag_backend.py:436-446), the [A, 3, Az, El] stack (:1518-1525), and the
// actor's minimum distance and ratios (:366-405, :459).  The float steps are those of the
// torch ops the reference runs: clamp = min(max(v, lo), hi) with NaN passed through,
// log1pf, and a multiply by the scalar denominator's reciprocal (how torch divides by a
// host scalar); the ratios are counts times torch's mean factor.  A pass of its own
// rather than an epilogue in the trace loop: there the finishing lanes of a warp iteration
// are one or two, and the epilogue cost 8% of a config-2 launch.
__global__ void __launch_bounds__(1024) observe_kernel(const float* __restrict__ dist, const int32_t* __restrict__ sem,
                                                      float* __restrict__ obs, float* __restrict__ stats,
                                                      const ObserveArgs o)
{
    const uint32_t actor = blockIdx.x;
    const uint32_t R = o.rays_per_actor;
    const float* dd = dist + static_cast<size_t>(actor) * R;
    const int32_t* ss = sem + static_cast<size_t>(actor) * R;
    float* ob = obs + static_cast<size_t>(actor) * 3u * R;
    unsigned int nkey = 0, nan_any = 0, sat = 0, prox = 0, band = 0, fwd = 0;
    for (uint32_t k = threadIdx.x; k < R; k += blockDim.x) {
        const float d = dd[k];
        const bool valid = isfinite(d);
        const bool nan = isnan(d);
        float c = d;
        if (!nan) {
            c = (c < 0.0f) ? 0.0f : c;
            c = (o.max_distance < c) ? o.max_distance : c;
        }
        float dep = __fmul_rn(log1pf(c), o.inv_log_denom);
        if (!isnan(dep)) {
            dep = (dep < 0.0f) ? 0.0f : dep;
            dep = (1.0f < dep) ? 1.0f : dep;
        }
        ob[k] = dep;
        ob[R + k] = static_cast<float>(ss[k]);
        ob[2u * static_cast<size_t>(R) + k] = valid ? 1.0f : 0.0f;
        if (nan) {
            nan_any = 1u;
        } else {
            const unsigned int b = __float_as_uint(c);
            const unsigned int key = (b >> 31) ? ~b : (b | 0x80000000u);  // order-preserving
            nkey = max(nkey, ~key);
        }
        sat += (c >= o.sat_thr) ? 1u : 0u;
        prox += (o.prox_on && valid && c <= o.prox) ? 1u : 0u;
        if (o.band_on && valid && c >= o.band_min && c <= o.band_max) {
            ++band;
            const uint32_t az = k / o.el_bins;
            // a row in both slices is counted twice, as torch.cat does
            fwd += (az < o.fwd_half ? 1u : 0u) + (az + o.fwd_half >= o.az_bins ? 1u : 0u);
        }
    }
    for (int off = 16; off > 0; off >>= 1) {
        nkey = max(nkey, __shfl_xor_sync(kFull, nkey, off));
        nan_any |= __shfl_xor_sync(kFull, nan_any, off);
        sat += __shfl_xor_sync(kFull, sat, off);
        prox += __shfl_xor_sync(kFull, prox, off);
        band += __shfl_xor_sync(kFull, band, off);
        fwd += __shfl_xor_sync(kFull, fwd, off);
    }
    __shared__ unsigned int part[6][32];
    const unsigned int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31u) == 0) {
        part[0][w] = nkey;
        part[1][w] = nan_any;
        part[2][w] = sat;
        part[3][w] = prox;
        part[4][w] = band;
        part[5][w] = fwd;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (unsigned int i = 1; i < (blockDim.x >> 5); ++i) {
            nkey = max(nkey, part[0][i]);
            nan_any |= part[1][i];
            sat += part[2][i];
            prox += part[3][i];
            band += part[4][i];
            fwd += part[5][i];
        }
        float mn;
        if (nan_any) {
            mn = __int_as_float(0x7fc00000);
        } else {
            const unsigned int key = ~nkey;
            mn = __uint_as_float((key >> 31) ? (key & 0x7fffffffu) : ~key);
        }
        float* st = stats + static_cast<size_t>(actor) * 5u;
        st[0] = mn;
        st[1] = fminf(fmaxf(__fmul_rn(static_cast<float>(sat), o.f_all), 0.0f), 1.0f);
        st[2] = o.prox_on ? fminf(fmaxf(__fmul_rn(static_cast<float>(prox), o.f_all), 0.0f), 1.0f) : 0.0f;
        st[3] = o.band_on ? fminf(fmaxf(__fmul_rn(static_cast<float>(band), o.f_all), 0.0f), 1.0f) : 0.0f;
        st[4] = o.band_on ? fminf(fmaxf(__fmul_rn(static_cast<float>(fwd), o.f_fwd), 0.0f), 1.0f) : 0.0f;
    }
}

__device__ __forceinline__ bool in_closed(const float3 p, const float3 mn, const float3 mx)
{
    return p.x >= mn.x && p.x <= mx.x && p.y >= mn.y && p.y <= mx.y && p.z >= mn.z && p.z <= mx.z;
}

__device__ __forceinline__ bool in_open(const float3 p, const float3 mn, const float3 mx)
{
    return p.x > mn.x && p.x < mx.x && p.y > mn.y && p.y < mx.y && p.z > mn.z && p.z < mx.z;
}

// kernel.cu:54-85; divisions are IEEE round-to-nearest
__device__ __forceinline__ float exit_distance(const float3 p, const float3 d, const float3 mn,
                                               const float3 mx)
{
    float t = kOutside;
    if (d.x > kDirEps) t = fminf(t, __fdiv_rn(__fsub_rn(mx.x, p.x), d.x));
    else if (d.x < -kDirEps) t = fminf(t, __fdiv_rn(__fsub_rn(mn.x, p.x), d.x));
    if (d.y > kDirEps) t = fminf(t, __fdiv_rn(__fsub_rn(mx.y, p.y), d.y));
    else if (d.y < -kDirEps) t = fminf(t, __fdiv_rn(__fsub_rn(mn.y, p.y), d.y));
    if (d.z > kDirEps) t = fminf(t, __fdiv_rn(__fsub_rn(mx.z, p.z), d.z));
    else if (d.z < -kDirEps) t = fminf(t, __fdiv_rn(__fsub_rn(mn.z, p.z), d.z));
    return fmaxf(t, kVoidAdvance);
}

__device__ __forceinline__ float leaf_distance(uint32_t bits)
{
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits & 0xFFFFu)));
}

template <bool kFan, bool kMulti>
__global__ void __launch_bounds__(kThreads) trace_float_kernel(const TraceArgs a)
{
    extern __shared__ __align__(16) uint32_t s_recs[];
    const uint32_t n_smem = kMulti ? 0u : a.n_smem;
    if (!kMulti && n_smem) {
        const uint4* src = reinterpret_cast<const uint4*>(a.scene.recs);
        uint4* dst = reinterpret_cast<uint4*>(s_recs);
        for (uint32_t i = threadIdx.x; i < 2u * n_smem; i += blockDim.x) dst[i] = __ldg(src + i);
        __syncthreads();
    }
    // per-scene launch of a scene table: the scene's actor range, read once
    uint32_t seg_base = 0, n_work = a.n_rays;
    if constexpr (kFan && !kMulti) {
        if (a.seg) {
            seg_base = __ldg(a.seg);
            const uint32_t seg_end = __ldg(a.seg + 1);
            const bool ok = checked(a.err, seg_base <= seg_end && seg_end <= a.n_rays / a.rays_per_actor, kErrActor);
            n_work = ok ? (seg_end - seg_base) * a.rays_per_actor : 0u;
        }
    }
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t lt_mask = (1u << lane) - 1u;

    // warp-uniform work queue
    uint32_t q_next = 0, q_end = 0;
    bool exhausted = false;

    // lane state
    bool active = false;
    uint32_t ray = 0;
    float3 o = make_float3(0.f, 0.f, 0.f), d = o, p = o;
    float t = 0.f, dist = 0.f;
    int32_t sem = 0;
    int step = 0;
    uint32_t flags = 0;
    float3 vmn = o, vmx = o, lmn = o, lmx = o, pmn = o, pmx = o, cmn = o, cmx = o;
    float leaf_d = 0.f;
    int32_t leaf_s = 0;
    uint32_t pre_rec = 0, node = 0;
    int depth = 0;

    // scene of the lane's ray
    const uint32_t* recs = a.scene.recs;
    const uint64_t* ext = a.scene.ext;
    uint32_t root = a.scene.root;
    uint32_t n_recs = a.scene.n_recs, n_ext = a.scene.n_ext;
    float3 bmn = make_float3(a.scene.bmin[0], a.scene.bmin[1], a.scene.bmin[2]);
    float3 bmx = make_float3(a.scene.bmax[0], a.scene.bmax[1], a.scene.bmax[2]);
    float eps = a.scene.eps;

    for (;;) {
        // ---- refill idle lanes from the warp queue ----
        const unsigned idle = __ballot_sync(kFull, !active);
        if (idle != 0u && !exhausted) {
            const uint32_t nidle = __popc(idle);
            const uint32_t rank = __popc(idle & lt_mask);
            const uint32_t avail = q_end - q_next;
            uint32_t mine = 0xFFFFFFFFu;
            if (!active && rank < avail) mine = q_next + rank;
            const uint32_t take = min(avail, nidle);
            q_next += take;
            if (nidle > take) {
                uint32_t base = 0;
                if (lane == 0) base = atomicAdd(a.counter, a.chunk);
                base = __shfl_sync(kFull, base, 0);
                if (base >= n_work) {
                    exhausted = true;
                } else {
                    q_next = base;
                    q_end = min(base + a.chunk, n_work);
                    const uint32_t got = min(nidle - take, q_end - q_next);
                    if (!active && rank >= take && rank - take < got) mine = q_next + (rank - take);
                    q_next += got;
                }
            }
            if (mine != 0xFFFFFFFFu) {
                ray = work_ray<kFan, kMulti>(a, mine, seg_base);
                active = true;
                t = 0.f;
                dist = 0.f;
                sem = 0;
                step = 0;
                flags = 0;
                int scene = 0;
                load_ray<kFan>(a, ray, o, d, scene);
                if constexpr (kMulti) {
                    if (static_cast<uint32_t>(scene) >= a.n_scenes) {
                        // no such scene: the ray is not traced (NaN distance, semantic 0, 0 steps)
                        finish_ray(a, ray, __int_as_float(0x7fc00000), 0, 0);
                        active = false;
                    } else {
                        const TsdfSceneDev* sc = a.table + scene;
                        recs = sc->recs;
                        n_recs = sc->n_recs;
                        n_ext = sc->n_ext;
                        ext = sc->ext;
                        root = sc->root;
                        bmn = make_float3(sc->bmin[0], sc->bmin[1], sc->bmin[2]);
                        bmx = make_float3(sc->bmax[0], sc->bmax[1], sc->bmax[2]);
                        eps = sc->eps;
                    }
                }
            }
        }
        if (!__any_sync(kFull, active)) break;
        if (!active) continue;

        bool step_done = false;
        if (!(flags & kInDesc)) {
            // ---- start of a march step (kernel.cu:260-294) ----
            p.x = __fmaf_rn(t, d.x, o.x);
            p.y = __fmaf_rn(t, d.y, o.y);
            p.z = __fmaf_rn(t, d.z, o.z);
            if ((flags & kVoidOk) && in_open(p, vmn, vmx)) {
                dist = exit_distance(p, d, vmn, vmx);
                sem = 0;
                step_done = true;
            } else if (!in_closed(p, bmn, bmx)) {
                dist = kOutside;
                sem = 0;
                step_done = true;
            } else if ((flags & kLeafOk) && in_closed(p, lmn, lmx)) {
                dist = leaf_d;
                sem = leaf_s;
                step_done = true;
            } else if ((flags & kPreOk) && in_closed(p, pmn, pmx)) {
                node = pre_rec;
                depth = kPrefixDepth;
                cmn = pmn;
                cmx = pmx;
                flags |= kInDesc | kUsePre;
            } else {
                node = root;
                depth = 0;
                cmn = bmn;
                cmx = bmx;
                flags = (flags | kInDesc) & ~kUsePre;
            }
        }
        if (flags & kInDesc) {
            // ---- one descent level (kernel.cu:136-198) ----
            // `leaf` receives the low 32 bits of a leaf word (half distance, 16-bit semantic)
            uint32_t leaf = 0;
            bool is_leaf = false;
            if (node & tsdf::kSlotLeafBit) {
                leaf = node & ~tsdf::kSlotLeafBit;
                is_leaf = true;
            } else if (node & tsdf::kSlotExtBit) {
                if (checked(a.err, (node & tsdf::kSlotIndexMask) < n_ext, kErrLeafTable))
                    leaf = static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned long long*>(ext) +
                                                       (node & tsdf::kSlotIndexMask)));
                is_leaf = true;
            } else {
                if (depth == kPrefixDepth && !(flags & kUsePre)) {
                    pre_rec = node;
                    pmn = cmn;
                    pmx = cmx;
                    flags |= kPreOk;
                }
                const float mx_ = (cmn.x + cmx.x) * 0.5f;
                const float my_ = (cmn.y + cmx.y) * 0.5f;
                const float mz_ = (cmn.z + cmx.z) * 0.5f;
                const bool ux = p.x >= mx_, uy = p.y >= my_, uz = p.z >= mz_;
                const uint32_t oct = (ux ? 1u : 0u) | (uy ? 2u : 0u) | (uz ? 4u : 0u);
                if (ux) cmn.x = mx_; else cmx.x = mx_;
                if (uy) cmn.y = my_; else cmx.y = my_;
                if (uz) cmn.z = mz_; else cmx.z = mz_;
                const size_t si = static_cast<size_t>(node) * 8u + oct;
                uint32_t slot = tsdf::kSlotVoid;
                if (checked(a.err, node < n_recs, kErrRecord)) slot = (node < n_smem) ? s_recs[si] : __ldg(recs + si);
                if (slot == tsdf::kSlotVoid) {
                    vmn = cmn;
                    vmx = cmx;
                    flags |= kVoidOk;
                    dist = exit_distance(p, d, vmn, vmx);
                    sem = 0;
                    step_done = true;
                } else if (depth + 1 >= kMaxDepth) {
                    step_done = true;  // cap reached: dist / sem keep their previous values
                } else if (slot & tsdf::kSlotLeafBit) {
                    leaf = slot & ~tsdf::kSlotLeafBit;
                    is_leaf = true;
                } else {
                    node = slot;
                    ++depth;
                }
            }
            if (is_leaf) {
                lmn = cmn;
                lmx = cmx;
                leaf_d = leaf_distance(leaf);
                leaf_s = static_cast<int32_t>(leaf >> 16);
                flags |= kLeafOk;
                dist = leaf_d;
                sem = leaf_s;
                step_done = true;
            }
            if (step_done) flags &= ~kInDesc;
        }
        if (step_done) {
            // ---- end of the march step (kernel.cu:297-304) ----
            if (sem != 0 && dist < eps) {
                finish_ray(a, ray, t, sem, step + 1);
                active = false;
            } else {
                t = t + dist;
                ++step;
                if (t > a.max_distance || step >= a.max_steps) {
                    finish_ray(a, ray, t, 0, step);
                    active = false;
                }
            }
        }
    }
}


// ============================================================================
// Integer-grid kernel (main path).
//
// The float bounds the reference computes during a descent (kernel.cu:166-176)
// are a fixed set of per-axis grid lines: the root box's faces, and each cell's
// midpoint (lo + hi) * 0.5f computed once from its two faces.  With D the
// height of the record graph, the lines B[0..2^D] per axis are built once per
// block into shared memory.  Each march step converts p to doubled integer
// coordinates (X = 2k on line k, 2k + 1 strictly between lines k and k + 1),
// after which every test of the reference is an integer comparison with
// identical outcome:
//   p >= mid            <=>  X >= 2 x mid index
//   closed box test     <=>  2 lo <= X <= 2 hi
//   strict box test     <=>  2 lo < X < 2 hi
// and a descent only extracts coordinate bits.  The reference starts every
// descent at the root or at its cached depth-4 node; the path it then follows
// is a function of the coordinates alone, so the descent here resumes at the
// deepest record it shares with the lane's previous descent path (kept in
// shared memory per lane), and replays the depth-4 cache update the reference
// makes when it passes that level.
// ============================================================================

constexpr int kStackLevels = tsdf::kMaxGridDepth;
constexpr uint32_t kSvHigh = 32u;        // stack levels 0..3 not valid
constexpr uint32_t kNeedExit = 64u;      // step ended in the void cell: exit distance still to compute
constexpr uint32_t kWideRay = 128u;      // a direction component of magnitude 2^126 or more
constexpr int kSdShift = 8;              // 5 bits: number of valid stack levels

// Positions on one axis as doubled grid coordinates: X = 2k where p lies on line k
// (p == B[k]), X = 2k + 1 where it lies strictly between lines k and k + 1.  A cell of the
// finest grid's units [lo, lo + size] is then one unsigned range test per axis for both
// of the reference's box tests: the closed box B[lo] <= p <= B[lo + size] is
// X - 2 lo <u 2 size + 1, its interior B[lo] < p < B[lo + size] is X - (2 lo + 1) <u 2 size - 1.
// A cached cell keeps the base (2 lo, or 2 lo + 1 for an interior) of each axis and one span
// (its cells are cubes).
__device__ __forceinline__ bool in_span(int x, int base, int span)
{
    return static_cast<uint32_t>(x - base) < static_cast<uint32_t>(span);
}
__device__ __forceinline__ int closed_span(int shift) { return (2 << shift) + 1; }

// Per-axis grid lines: rows of line_row(n) = n + 3 floats, -inf, B[0..n], +inf; `lines`
// points at B[0] of axis 0, so line_at(axis, k) reads B[k] for k in [-1, n + 1].
__host__ __device__ constexpr int line_row(int n) { return n + 3; }

struct GridView {
    const float* lines;  // B[0] of axis 0; rows of line_row(n) floats
    int n;
};

template <bool kShared>
__device__ __forceinline__ float line_at(const GridView& g, int axis, int k)
{
    const float* ptr = g.lines + axis * line_row(g.n) + k;
    if constexpr (kShared) return *ptr;
    else return __ldg(ptr);
}

// Doubled grid coordinate of p: 2k + (p on line k ? 0 : 1) for k the last grid line <= p,
// -1 below the box, n at or above its top face (n + 1 for p = +inf); X <u 2n + 1 is the
// reference's closed domain test.  v(p) = fma(p, scale, offs), where offs carries a shift of
// half a cell, is monotone in p with floor(v(B[k])) = k - 1 at every line k (proved per
// table on the host, build_grid_lines), so e = floor(v(p)), clamped to [-1, n], is k or the
// line below it, and the line above decides.  The -inf / +inf sentinels at both ends of the
// row make the box faces need no special case; NaN gives e = -1 (fmaxf drops it), X = -1.
template <bool kShared>
__device__ __forceinline__ int grid_coord(const GridView& g, int axis, float p, float scale, float offs, int& j2)
{
    const int e = __float2int_rd(fminf(fmaxf(__fmaf_rn(p, scale, offs), -1.0f), static_cast<float>(g.n)));
    const float l0 = line_at<kShared>(g, axis, e);
    const float l1 = line_at<kShared>(g, axis, e + 1);
    const bool ge1 = p >= l1;
    const bool on = p == (ge1 ? l1 : l0);
    j2 = 2 * (e + (ge1 ? 1 : 0));
    return j2 + (on ? 0 : 1);
}

// Per-axis reciprocals of a ray's direction, correctly rounded, from which exit_quotient
// computes the exit quotients; NaN where |d| <= 1e-4, the axes kernel.cu:54-85 leaves out.
// Kept per lane in shared memory while the ray lives.
__device__ __forceinline__ float axis_reciprocal(float dv)
{
    return fabsf(dv) > kDirEps ? __frcp_rn(dv) : __int_as_float(0x7fc00000);
}

// kernel.cu:54-85 with the void cell's faces read from the grid lines: the minimum over
// the axes of the IEEE quotients (face - p) / d, each from the lane's reciprocal of d by
// exit_quotient (no division), capped at 1000 and floored at 1e-4.  rcp: the lane's
// per-axis reciprocals of d, NaN on the axes the reference skips (|d| <= 1e-4), whose
// quotients are then NaN and drop out of fminf.  wide: a component of d is 2^126 or more
// in magnitude, where exit_quotient does not apply; such rays divide.  The quotients are
// never negative: p lies in the closed cell and each face is the one d points to.
template <bool kShared>
__device__ __forceinline__ float cell_exit_distance(const GridView& g, const float3 p, const float3 d,
                                                    const float3 rcp, int bx, int by, int bz, int span, bool wide)
{
    // the cell's faces from its interior bases 2 lo + 1 and span 2 size - 1
    const int size = (span + 1) >> 1;
    const int lx = bx >> 1, ly = by >> 1, lz = bz >> 1;
    const float ax = __fsub_rn(line_at<kShared>(g, 0, d.x > 0.0f ? lx + size : lx), p.x);
    const float ay = __fsub_rn(line_at<kShared>(g, 1, d.y > 0.0f ? ly + size : ly), p.y);
    const float az = __fsub_rn(line_at<kShared>(g, 2, d.z > 0.0f ? lz + size : lz), p.z);
    float tx, ty, tz;
    if (!wide) {
        tx = tsdf::exit_quotient(ax, d.x, rcp.x, __fmul_rn(ax, rcp.x));
        ty = tsdf::exit_quotient(ay, d.y, rcp.y, __fmul_rn(ay, rcp.y));
        tz = tsdf::exit_quotient(az, d.z, rcp.z, __fmul_rn(az, rcp.z));
    } else {
        const float nan = __int_as_float(0x7fc00000);
        tx = rcp.x == rcp.x ? __fdiv_rn(ax, d.x) : nan;
        ty = rcp.y == rcp.y ? __fdiv_rn(ay, d.y) : nan;
        tz = rcp.z == rcp.z ? __fdiv_rn(az, d.z) : nan;
    }
    return fmaxf(fminf(fminf(fminf(tx, ty), tz), kOutside), kVoidAdvance);
}

// Claim rays for the idle lanes of the warp: returns this lane's new ray or ~0u.  A
// single idle lane waits for a second one (config 5: +1.3 %): the ray-loading block then
// runs for two lanes at a time instead of one, and consecutive rays start together.  No
// lane waits for long: the next lane of its warp to finish a ray joins it.
__device__ __forceinline__ uint32_t claim_ray(uint32_t& q_next, uint32_t& q_end, bool& exhausted, bool active,
                                              uint32_t lane, unsigned int* counter, uint32_t chunk, uint32_t n_rays)
{
    const unsigned idle = __ballot_sync(kFull, !active);
    uint32_t mine = 0xFFFFFFFFu;
    if (__popc(idle) < 2 || exhausted) return mine;
    const uint32_t nidle = __popc(idle);
    const uint32_t rank = __popc(idle & ((1u << lane) - 1u));
    const uint32_t avail = q_end - q_next;
    if (!active && rank < avail) mine = q_next + rank;
    const uint32_t take = min(avail, nidle);
    q_next += take;
    if (nidle > take) {
        uint32_t base = 0;
        if (lane == 0) base = atomicAdd(counter, chunk);
        base = __shfl_sync(kFull, base, 0);
        if (base >= n_rays) {
            exhausted = true;
        } else {
            q_next = base;
            q_end = min(base + chunk, n_rays);
            const uint32_t got = min(nidle - take, q_end - q_next);
            if (!active && rank >= take && rank - take < got) mine = q_next + (rank - take);
            q_next += got;
        }
    }
    return mine;
}

// Claim order of a single-scene launch.  A launch ends with its longest rays, and a ray's
// step count grows with the distance it can travel before it leaves the scene's box (rank
// correlation 0.65 on config 2): claiming rays by that distance, longest first, lets the
// long ones run while the short ones fill the GPU (config 2: 15% shorter launches).  The
// key is only a schedule; every ray is traced exactly as before.  Rays go into
// kOrderBuckets buckets of exit distance, counted, then scattered longest bucket first.
// A per-scene launch of a scene table orders its own scene's rays the same way.
constexpr int kOrderBuckets = 64;

// Work items of a claim order: the launch's rays, or for a per-scene launch the rays of
// its scene's actors perm[seg[0], seg[1]) (read on the device).  Keys and order entries
// live at [base, base + n) of their arrays; an order entry is a work item w < n.
struct OrderRange {
    uint32_t n, base, seg_base;
};

template <bool kFan>
__device__ __forceinline__ OrderRange order_range(const TraceArgs& a)
{
    OrderRange r{a.n_rays, 0u, 0u};
    if constexpr (kFan) {
        if (a.seg) {
            const uint32_t n_actors = a.n_rays / a.rays_per_actor;
            const uint32_t end = min(__ldg(a.seg + 1), n_actors);
            r.seg_base = min(__ldg(a.seg), end);
            r.n = (end - r.seg_base) * a.rays_per_actor;
            r.base = r.seg_base * a.rays_per_actor;
        }
    }
    return r;
}

// Ray of work item w < rg.n.
template <bool kFan>
__device__ __forceinline__ uint32_t order_ray(const TraceArgs& a, const OrderRange& rg, uint32_t w)
{
    if constexpr (kFan) {
        if (a.seg) {
            const uint32_t slot = div_rpa(a, w);
            const uint32_t actor = __ldg(a.perm + rg.seg_base + slot);
            return actor * a.rays_per_actor + (w - slot * a.rays_per_actor);
        }
    }
    return w;
}

template <bool kFan>
__global__ void __launch_bounds__(256) order_key_kernel(const TraceArgs a, float buckets_per_unit,
                                                        uint8_t* __restrict__ key, unsigned int* __restrict__ hist)
{
    __shared__ unsigned int h[kOrderBuckets];
    for (int i = threadIdx.x; i < kOrderBuckets; i += blockDim.x) h[i] = 0;
    __syncthreads();
    const OrderRange rg = order_range<kFan>(a);
    const float3 lo = make_float3(a.scene.bmin[0], a.scene.bmin[1], a.scene.bmin[2]);
    const float3 hi = make_float3(a.scene.bmax[0], a.scene.bmax[1], a.scene.bmax[2]);
    for (uint32_t w = blockIdx.x * blockDim.x + threadIdx.x; w < rg.n; w += gridDim.x * blockDim.x) {
        float3 o, d;
        int scene = 0;
        load_ray<kFan>(a, order_ray<kFan>(a, rg, w), o, d, scene);
        const float inf = __int_as_float(0x7f800000);
        const float tx = d.x > 0.f ? (hi.x - o.x) / d.x : (d.x < 0.f ? (lo.x - o.x) / d.x : inf);
        const float ty = d.y > 0.f ? (hi.y - o.y) / d.y : (d.y < 0.f ? (lo.y - o.y) / d.y : inf);
        const float tz = d.z > 0.f ? (hi.z - o.z) / d.z : (d.z < 0.f ? (lo.z - o.z) / d.z : inf);
        const float te = fminf(fminf(tx, ty), tz) * buckets_per_unit;
        const int b = (te >= 0.f) ? min(kOrderBuckets - 1, static_cast<int>(fminf(te, 1.0e9f))) : 0;
        const unsigned int k = static_cast<unsigned int>(kOrderBuckets - 1 - b);  // longest first
        key[rg.base + w] = static_cast<uint8_t>(k);
        atomicAdd(&h[k], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kOrderBuckets; i += blockDim.x)
        if (h[i]) atomicAdd(&hist[i], h[i]);
}

// Tiles of kOrderTile work items, looped over by a persistent grid: ranks within the tile
// from shared-memory counters, then one global reservation per bucket and tile (a global
// atomic per ray would serialise on the few buckets that hold most rays).
constexpr int kOrderPerThread = 8;
constexpr int kOrderTile = 256 * kOrderPerThread;

template <bool kFan>
__global__ void __launch_bounds__(256) order_scatter_kernel(const TraceArgs a, const uint8_t* __restrict__ key,
                                                            const unsigned int* __restrict__ hist,
                                                            unsigned int* __restrict__ cursor, uint32_t* __restrict__ perm)
{
    __shared__ unsigned int off[kOrderBuckets];
    __shared__ unsigned int cnt[kOrderBuckets];
    if (threadIdx.x == 0) {
        unsigned int run = 0;
        for (int b = 0; b < kOrderBuckets; ++b) {
            off[b] = run;
            run += hist[b];
        }
    }
    const OrderRange rg = order_range<kFan>(a);
    for (uint32_t tile = blockIdx.x * static_cast<uint32_t>(kOrderTile); tile < rg.n;
         tile += gridDim.x * static_cast<uint32_t>(kOrderTile)) {
        if (threadIdx.x < kOrderBuckets) cnt[threadIdx.x] = 0;
        __syncthreads();
        uint8_t bk[kOrderPerThread];
        unsigned int rank[kOrderPerThread];
#pragma unroll
        for (int i = 0; i < kOrderPerThread; ++i) {
            const uint32_t w = tile + i * 256u + threadIdx.x;
            if (w < rg.n) {
                bk[i] = key[rg.base + w];
                rank[i] = atomicAdd(&cnt[bk[i]], 1u);
            }
        }
        __syncthreads();
        if (threadIdx.x < kOrderBuckets) {
            const unsigned int c = cnt[threadIdx.x];
            cnt[threadIdx.x] = c ? off[threadIdx.x] + atomicAdd(&cursor[threadIdx.x], c) : 0u;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kOrderPerThread; ++i) {
            const uint32_t w = tile + i * 256u + threadIdx.x;
            if (w < rg.n) perm[rg.base + cnt[bk[i]] + rank[i]] = w;
        }
        __syncthreads();  // cnt is reset for the next tile
    }
}

// Scene of a lane's ray.  Single-scene launches read uniform kernel parameters and
// the block's shared grid lines; multi-scene launches keep only a pointer into the
// scene table and re-read fields at their point of use (L1-resident), which keeps the
// kernel at 64 registers (4 blocks of 256 per SM).
template <bool kMulti>
struct SceneAccess;

template <>
struct SceneAccess<false> {
    const TsdfSceneDev* s;
    GridView g;
    float3 b0_, bn_, sc_, of_;
    __device__ __forceinline__ const uint32_t* recs() const { return s->recs; }
    __device__ __forceinline__ const uint64_t* ext() const { return s->ext; }
    __device__ __forceinline__ uint32_t root() const { return s->root; }
    __device__ __forceinline__ uint32_t n_recs() const { return s->n_recs; }
    __device__ __forceinline__ uint32_t n_ext() const { return s->n_ext; }
    __device__ __forceinline__ int depth() const { return s->depth; }
    __device__ __forceinline__ float eps() const { return s->eps; }
    __device__ __forceinline__ GridView grid() const { return g; }
    __device__ __forceinline__ float3 b0() const { return b0_; }
    __device__ __forceinline__ float3 bn() const { return bn_; }
    __device__ __forceinline__ float3 scale() const { return sc_; }
    __device__ __forceinline__ float3 offs() const { return of_; }
};

template <>
struct SceneAccess<true> {
    const TsdfSceneDev* s;
    __device__ __forceinline__ const uint32_t* recs() const
    {
        return reinterpret_cast<const uint32_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&s->recs)));
    }
    __device__ __forceinline__ const uint64_t* ext() const
    {
        return reinterpret_cast<const uint64_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&s->ext)));
    }
    __device__ __forceinline__ uint32_t root() const { return __ldg(&s->root); }
    __device__ __forceinline__ uint32_t n_recs() const { return __ldg(&s->n_recs); }
    __device__ __forceinline__ uint32_t n_ext() const { return __ldg(&s->n_ext); }
    __device__ __forceinline__ int depth() const { return __ldg(&s->depth); }
    __device__ __forceinline__ float eps() const { return __ldg(&s->eps); }
    __device__ __forceinline__ GridView grid() const
    {
        GridView g;
        g.lines = reinterpret_cast<const float*>(__ldg(reinterpret_cast<const unsigned long long*>(&s->lines)));
        g.n = 1 << depth();
        return g;
    }
    __device__ __forceinline__ float3 b0() const { return make_float3(__ldg(&s->bmin[0]), __ldg(&s->bmin[1]), __ldg(&s->bmin[2])); }
    __device__ __forceinline__ float3 bn() const { return make_float3(__ldg(&s->bmax[0]), __ldg(&s->bmax[1]), __ldg(&s->bmax[2])); }
    __device__ __forceinline__ float3 scale() const { return make_float3(__ldg(&s->scale[0]), __ldg(&s->scale[1]), __ldg(&s->scale[2])); }
    __device__ __forceinline__ float3 offs() const { return make_float3(__ldg(&s->offs[0]), __ldg(&s->offs[1]), __ldg(&s->offs[2])); }
};

// Four resident blocks of 256 per SM (up to 64 registers, no spills).  An instance held
// to five blocks (48 registers, 24 bytes of spill slots) won 3 % on long launches before the
// start of a step lost its branches, and lost 3.5 % on config 5 after.
template <bool kFan, bool kMulti, int kLevels>
__global__ void __launch_bounds__(kThreads, 4) trace_grid_kernel(const TraceArgs a)
{
    constexpr bool kShared = !kMulti;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t* s_stack = reinterpret_cast<uint32_t*>(smem_raw);   // [kStackLevels][kThreads]
    float* s_rcp = reinterpret_cast<float*>(s_stack + kStackLevels * kThreads);  // [3][kThreads]
    float* s_lines = s_rcp + 3 * kThreads;                             // [3][line_row(2^D)]

    SceneAccess<kMulti> S;
    S.s = kMulti ? a.table : &a.scene;
    if constexpr (!kMulti) {
        const float3 b0 = make_float3(a.scene.bmin[0], a.scene.bmin[1], a.scene.bmin[2]);
        const float3 bn = make_float3(a.scene.bmax[0], a.scene.bmax[1], a.scene.bmax[2]);
        S.b0_ = b0;
        S.bn_ = bn;
        S.sc_ = make_float3(a.scene.scale[0], a.scene.scale[1], a.scene.scale[2]);
        S.of_ = make_float3(a.scene.offs[0], a.scene.offs[1], a.scene.offs[2]);
        S.g.n = 1 << a.scene.depth;
        S.g.lines = s_lines + 1;
        // grid lines by the midpoint rule, level by level, between the -inf / +inf sentinels
        const int n = S.g.n;
        if (threadIdx.x < 3) {
            const unsigned ax = threadIdx.x;
            float* row = s_lines + ax * line_row(n);
            row[0] = -__int_as_float(0x7f800000);
            row[1] = ax == 0 ? b0.x : (ax == 1 ? b0.y : b0.z);
            row[n + 1] = ax == 0 ? bn.x : (ax == 1 ? bn.y : bn.z);
            row[n + 2] = __int_as_float(0x7f800000);
        }
        __syncthreads();
        for (int lvl = 0; lvl < a.scene.depth; ++lvl) {
            const int stride = n >> lvl;
            const int cells = 1 << lvl;
            for (int w = threadIdx.x; w < 3 * cells; w += blockDim.x) {
                const int axis = w / cells;
                const int c = w - axis * cells;
                float* row = s_lines + axis * line_row(n) + 1;
                row[c * stride + (stride >> 1)] = (row[c * stride] + row[c * stride + stride]) * 0.5f;
            }
            __syncthreads();
        }
    }

    // per-scene launch of a scene table: the scene's actor range, read once
    uint32_t seg_base = 0, n_work = a.n_rays;
    if constexpr (kFan && !kMulti) {
        if (a.seg) {
            seg_base = __ldg(a.seg);
            const uint32_t seg_end = __ldg(a.seg + 1);
            const bool ok = checked(a.err, seg_base <= seg_end && seg_end <= a.n_rays / a.rays_per_actor, kErrActor);
            n_work = ok ? (seg_end - seg_base) * a.rays_per_actor : 0u;
        }
    }
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t* my_stack = s_stack + threadIdx.x;
    float* my_rcp = s_rcp + threadIdx.x;
    uint32_t q_next = 0, q_end = 0;
    bool exhausted = false;

    bool active = false;
    uint32_t ray = 0;
    float3 o = make_float3(0.f, 0.f, 0.f), d = o;
    float t = 0.f, dist = 0.f;
    int32_t sem = 0;
    int step = 0;
    uint32_t flags = 0;
    int jx = 0, jy = 0, jz = 0, jpx = 0, jpy = 0, jpz = 0;
    // cached cells as doubled-coordinate bases and spans: leaf (closed), void (interior),
    // depth-4 prefix (closed; its span follows from the depth)
    int lbx = 0, lby = 0, lbz = 0, lsp = 0, vbx = 0, vby = 0, vbz = 0, vsp = 0, pbx = 0, pby = 0, pbz = 0;
    float leaf_d = 0.f;
    int32_t leaf_s = 0;
    uint32_t pre_rec = 0, node = 0;
    int lvl = 0;  // level of `node` in the descent under way

    for (;;) {
        const uint32_t mine = claim_ray(q_next, q_end, exhausted, active, lane, a.counter, a.chunk, n_work);
        if (mine != 0xFFFFFFFFu) {
            int scene = 0;
            ray = work_ray<kFan, kMulti>(a, mine, seg_base);
            load_ray<kFan>(a, ray, o, d, scene);
            my_rcp[0] = axis_reciprocal(d.x);
            my_rcp[kThreads] = axis_reciprocal(d.y);
            my_rcp[2 * kThreads] = axis_reciprocal(d.z);
            active = true;
            t = 0.f;
            dist = 0.f;
            sem = 0;
            step = 0;
            flags = fmaxf(fmaxf(fabsf(d.x), fabsf(d.y)), fabsf(d.z)) < tsdf::kQuotientMaxDivisor ? 0u : kWideRay;
            if constexpr (kMulti) {
                if (static_cast<uint32_t>(scene) >= a.n_scenes) {
                    // no such scene: the ray is not traced (NaN distance, semantic 0, 0 steps)
                    finish_ray(a, ray, __int_as_float(0x7fc00000), 0, 0);
                    active = false;
                } else {
                    S.s = a.table + scene;
                }
            }
        }
        if (!__any_sync(kFull, active)) break;
        if (!active) continue;

        const int D = S.depth();
        bool step_done = false;
        bool leaf_step = false;  // the step ends in the cached leaf cell
        // the descent's end, recorded where it is reached and completed once below
        bool done = false;
        uint32_t fin = 0;   // the slot it ends in: tsdf::kSlotVoid or a leaf slot
        int fin_level = 0;  // level of that cell
        if (!(flags & kInDesc)) {
            // ---- start of a march step (kernel.cu:260-294) ----
            const GridView g = S.grid();
            const float3 scale = S.scale(), offs = S.offs();
            const float3 p = make_float3(__fmaf_rn(t, d.x, o.x), __fmaf_rn(t, d.y, o.y), __fmaf_rn(t, d.z, o.z));
            int X2, Y2, Z2;
            const int X = grid_coord<kShared>(g, 0, p.x, scale.x, offs.x, X2);
            const int Y = grid_coord<kShared>(g, 1, p.y, scale.y, offs.y, Y2);
            const int Z = grid_coord<kShared>(g, 2, p.z, scale.z, offs.z, Z2);
            // The reference's tests in its order (kernel.cu:265 void cache, :108 domain, :114 leaf
            // cache), all evaluated and combined with selects rather than a chain of branches:
            // lanes of a warp take different outcomes, and the branchy form measured 8 % slower
            // on config 2 and 2.4 % on config 5.  The exit distance of a void-cache hit comes
            // below, with the descents that end in a void cell.
            const bool hit_void = ((flags & kVoidOk) != 0) & in_span(X, vbx, vsp) & in_span(Y, vby, vsp) &
                                  in_span(Z, vbz, vsp);
            // closed box test of the domain: lines 0 to n
            const int dom = 2 * g.n + 1;
            const bool inside = in_span(X, 0, dom) & in_span(Y, 0, dom) & in_span(Z, 0, dom);
            const bool hit_leaf = ((flags & kLeafOk) != 0) & in_span(X, lbx, lsp) & in_span(Y, lby, lsp) &
                                  in_span(Z, lbz, lsp);
            const bool outside = !hit_void & !inside;
            const bool leaf_hit = !hit_void & inside & hit_leaf;
            flags = hit_void ? (flags | kNeedExit) : flags;
            dist = outside ? kOutside : (leaf_hit ? leaf_d : dist);
            sem = outside ? 0 : (leaf_hit ? leaf_s : sem);
            step_done = hit_void | outside | leaf_hit;
            leaf_step = leaf_hit;
            if (!step_done) {
                const int psh = D - kPrefixDepth;  // prefix cells: 2^psh finest cells a side
                const int psp = closed_span(max(psh, 0));
                const bool use_pre = (flags & kPreOk) && in_span(X, pbx, psp) && in_span(Y, pby, psp) &&
                                     in_span(Z, pbz, psp);
                // descent coordinates, doubled (2 x the cell index): on the start box's top face
                // the reference keeps taking the upper half
                if (use_pre) {
                    const int top = (2 << psh) - 2;
                    jx = min(X2, pbx + top);
                    jy = min(Y2, pby + top);
                    jz = min(Z2, pbz + top);
                } else {
                    jx = min(X2, 2 * g.n - 2);
                    jy = min(Y2, 2 * g.n - 2);
                    jz = min(Z2, 2 * g.n - 2);
                }
                const int start = use_pre ? kPrefixDepth : 0;
                const int sd = static_cast<int>((flags >> kSdShift) & 31u);
                const int sv = (flags & kSvHigh) ? kPrefixDepth : 0;
                const int common = D - 31 + __clz((jx ^ jpx) | (jy ^ jpy) | (jz ^ jpz));
                const int reuse = min(common, sd - 1);
                // resume at the deepest valid stack level on the path, else at the start node
                const bool resume = (reuse >= start) & (reuse >= sv);
                const int level = resume ? reuse : start;
                const uint32_t kept =  // level <= D - 1 < kStackLevels
                    checked(a.err, level < kStackLevels, kErrStack) ? my_stack[level * kThreads] : S.root();
                node = resume ? kept : (use_pre ? pre_rec : S.root());
                flags = resume ? flags : (use_pre ? (flags | kSvHigh) : (flags & ~kSvHigh));
                flags = (flags & ~kUsePre) | kInDesc | (use_pre ? kUsePre : 0u);
                lvl = level;
                if (node >= tsdf::kSlotExtBit) {
                    // the root slot of a one-leaf DAG (stack and prefix entries are records)
                    fin = node;
                    fin_level = 0;
                    done = true;
                }
            }
        }
        bool descend = (flags & kInDesc) && !done;
#pragma unroll
        for (int it = 0; it < kLevels && descend; ++it) {
            // ---- one descent level (kernel.cu:136-198) ----
            if (checked(a.err, lvl < kStackLevels, kErrStack)) my_stack[lvl * kThreads] = node;
            const int sh = D - lvl;  // bit of the level in the doubled coordinates
            const uint32_t oct = ((jx >> sh) & 1) | (((jy >> sh) & 1) << 1) | (((jz >> sh) & 1) << 2);
            uint32_t slot = tsdf::kSlotVoid;
            if (checked(a.err, node < S.n_recs(), kErrRecord))
                slot = __ldg(S.recs() + (static_cast<size_t>(node) * 8u + oct));
            // A record graph of height D <= 12 ends every path by level D, so the
            // reference's 32-level cap (kernel.cu:136) is never reached here.
            ++lvl;
            if (slot >= tsdf::kSlotExtBit) {  // an empty octant or a leaf
                fin = slot;
                fin_level = lvl;
                done = true;
                descend = false;
            } else {
                node = slot;
            }
        }
        if (done) {
            // The cell the descent ends in, a cube of 2^sh finest cells a side: an empty octant,
            // cached as its interior, or a leaf, cached as its closed box (kernel.cu:177-190).
            const bool vd = fin == tsdf::kSlotVoid;
            const int sh = D - fin_level;
            const int keep = -2 << sh;
            const int bx = jx & keep, by = jy & keep, bz = jz & keep;
            vbx = vd ? (bx | 1) : vbx;
            vby = vd ? (by | 1) : vby;
            vbz = vd ? (bz | 1) : vbz;
            vsp = vd ? (2 << sh) - 1 : vsp;
            lbx = vd ? lbx : bx;
            lby = vd ? lby : by;
            lbz = vd ? lbz : bz;
            lsp = vd ? lsp : (2 << sh) + 1;
            flags |= vd ? (kVoidOk | kNeedExit) : 0u;
            if (!vd) {
                uint32_t leaf = fin & ~tsdf::kSlotLeafBit;
                if (!(fin & tsdf::kSlotLeafBit)) {
                    // a leaf stored out of line (semantic >= 0x7FFF)
                    leaf = 0;
                    if (checked(a.err, (fin & tsdf::kSlotIndexMask) < S.n_ext(), kErrLeafTable))
                        leaf = static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned long long*>(S.ext()) +
                                                           (fin & tsdf::kSlotIndexMask)));
                }
                leaf_d = leaf_distance(leaf);
                leaf_s = static_cast<int32_t>(leaf >> 16);
                flags |= kLeafOk;
                leaf_step = true;
                dist = leaf_d;
                sem = leaf_s;
            }
            // The reference caches the depth-4 node of a descent that did not start there
            // (kernel.cu:154-163): the record at level 4 of this path, from the stack.
            if (!(flags & kUsePre) && fin_level > kPrefixDepth) {
                pre_rec = my_stack[kPrefixDepth * kThreads];
                const int pmask = -2 << (D - kPrefixDepth);
                pbx = jx & pmask;
                pby = jy & pmask;
                pbz = jz & pmask;
                flags |= kPreOk;
            }
            // records of levels 0..fin_level-1 now lie on the path of (jx, jy, jz)
            jpx = jx;
            jpy = jy;
            jpz = jz;
            flags = (flags & ~(kInDesc | (31u << kSdShift))) | (static_cast<uint32_t>(fin_level) << kSdShift);
            step_done = true;
        }
        if (flags & kNeedExit) {
            // the step ended in the void cell (cached or just found): its exit distance,
            // computed here once for both kinds of lanes (kernel.cu:54-85, :188)
            flags &= ~kNeedExit;
            const float3 p = make_float3(__fmaf_rn(t, d.x, o.x), __fmaf_rn(t, d.y, o.y), __fmaf_rn(t, d.z, o.z));
            const float3 rcp = make_float3(my_rcp[0], my_rcp[kThreads], my_rcp[2 * kThreads]);
            dist = cell_exit_distance<kShared>(S.grid(), p, d, rcp, vbx, vby, vbz, vsp, (flags & kWideRay) != 0);
            sem = 0;
        }
        if (step_done) {
            // ---- end of the march step (kernel.cu:297-304), then, after a step that ended in
            // the cached leaf cell, up to leaf_run more steps in place while the next position
            // stays in that cell.  Such a step is a leaf-cache hit in the reference: a point of
            // the closed leaf box is inside the domain and not strictly inside the void cell
            // (octree cells have disjoint interiors), so the tests before the leaf test
            // (kernel.cu:265, :108) fail.
            const float eps = S.eps();
            // the hit, horizon and leaf-cell tests as selects, like the start of a step
            // (configs 2-5: +2-3 % over the branchy form)
            for (uint32_t run = 0;; ++run) {
                const bool hit = (sem != 0) & (dist < eps);
                const float tn = t + dist;
                t = hit ? t : tn;
                step = hit ? step : step + 1;
                const bool over = !hit & ((t > a.max_distance) | (step >= a.max_steps));
                if (hit | over) {
                    finish_ray(a, ray, t, hit ? sem : 0, hit ? step + 1 : step);
                    active = false;
                    break;
                }
                // multi-scene launches read the lines from global memory, where the run
                // costs more than it saves (config 3: -9%); single-scene launches only
                if (kMulti || run >= a.leaf_run || !leaf_step) break;
                const float3 p = make_float3(__fmaf_rn(t, d.x, o.x), __fmaf_rn(t, d.y, o.y), __fmaf_rn(t, d.z, o.z));
                const GridView g = S.grid();
                // inclusive bounds of the leaf cell: its grid lines (kernel.cu:114)
                const int size = lsp >> 1, lx = lbx >> 1, ly = lby >> 1, lz = lbz >> 1;
                if (!((p.x >= line_at<kShared>(g, 0, lx)) & (p.x <= line_at<kShared>(g, 0, lx + size)) &
                      (p.y >= line_at<kShared>(g, 1, ly)) & (p.y <= line_at<kShared>(g, 1, ly + size)) &
                      (p.z >= line_at<kShared>(g, 2, lz)) & (p.z <= line_at<kShared>(g, 2, lz + size))))
                    break;
                dist = leaf_d;
                sem = leaf_s;
            }
        }
    }
}

}  // namespace

namespace {

using tsdf::cuda_fail;
using tsdf::fail;

bool finite3(const float* v) { return std::isfinite(v[0]) && std::isfinite(v[1]) && std::isfinite(v[2]); }

int common_checks(int64_t n_rays, float* out_d, int32_t* out_s, int max_steps, float max_distance,
                  void* workspace)
{
    if (n_rays < 0 || n_rays > kMaxRays)
        return fail(TSDF_ERR_INVALID, "number of rays must be in [0, 2^31 - 2^24]");
    if (max_steps <= 0) return fail(TSDF_ERR_INVALID, "max_steps must be a positive integer");
    if (!std::isfinite(max_distance) || max_distance <= 0.0f)
        return fail(TSDF_ERR_INVALID, "max_distance must be a finite positive float");
    if (n_rays > 0 && (!out_d || !out_s)) return fail(TSDF_ERR_INVALID, "output pointers must not be null");
    if (n_rays > 0 && !workspace) return fail(TSDF_ERR_INVALID, "workspace must not be null");
    return TSDF_OK;
}

enum class Kind { kFloat, kGrid };

// Workspace layout: the work counter and error word (kLaunchWords words, cleared by every
// launch), then from kScratchOffset either the multi-scene actor order (4 bytes per actor)
// or the single-scene claim order (order_scratch_bytes).
constexpr size_t kLaunchWords = 2;
constexpr size_t kScratchOffset = 256;

uint64_t order_scratch_bytes(int64_t n_rays)
{
    const uint64_t n = static_cast<uint64_t>(n_rays);
    return 2u * kOrderBuckets * sizeof(unsigned int) + n * sizeof(uint32_t) + ((n + 15u) & ~uint64_t(15));
}
constexpr int64_t kSmemReservedPerBlock = 1024;  // shared memory the driver reserves per resident block

// Buckets of the claim order per unit of exit distance: kOrderBuckets over the box diagonal.
float exit_buckets_per_unit(const TsdfSceneDev& s)
{
    double diag2 = 0.0;
    for (int i = 0; i < 3; ++i) {
        const double ext = static_cast<double>(s.bmax[i]) - s.bmin[i];
        diag2 += ext * ext;
    }
    return static_cast<float>(kOrderBuckets / std::sqrt(diag2));
}

// Per-device launch constants, read once per device and kernel instead of on every
// cast: the SM count, shared memory per SM, the resident blocks per SM of a kernel at a
// dynamic shared-memory size, and the largest dynamic shared memory a kernel has been
// allowed (cudaFuncAttributeMaxDynamicSharedMemorySize, per device and kernel).
constexpr int kMaxInfoDevices = 64;
struct DeviceInfo {
    int sms = 0;
    int smem_per_sm = 0;
};
struct OccupancyEntry {
    int device;
    const void* kern;
    size_t smem;
    int blocks;
};
struct SmemAttrEntry {
    int device;
    const void* kern;
    size_t smem;
};
std::mutex g_info_mu;
DeviceInfo g_info[kMaxInfoDevices];
std::vector<OccupancyEntry> g_occupancy;  // under g_info_mu
std::vector<SmemAttrEntry> g_smem_attr;   // under g_info_mu

int device_info(int device, DeviceInfo& out)
{
    if (device < 0 || device >= kMaxInfoDevices) return fail(TSDF_ERR_INVALID, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_info_mu);
    DeviceInfo& d = g_info[device];
    if (d.sms == 0) {
        int sms = 0, smem = 0;
        cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        d.smem_per_sm = smem;
        d.sms = sms;
    }
    out = d;
    return TSDF_OK;
}

// Lets `kern` launch with `smem` bytes of dynamic shared memory on the current device
// (`device`), once per device, kernel and size above what was already allowed.
int allow_smem(int device, const void* kern, size_t smem)
{
    if (smem <= 48u * 1024u) return TSDF_OK;
    std::lock_guard<std::mutex> lock(g_info_mu);
    for (SmemAttrEntry& en : g_smem_attr) {
        if (en.device == device && en.kern == kern) {
            if (en.smem >= smem) return TSDF_OK;
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
            en.smem = smem;
            return TSDF_OK;
        }
    }
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    g_smem_attr.push_back({device, kern, smem});
    return TSDF_OK;
}

// Resident blocks of kThreads threads per SM for `kern` at `smem` bytes (current device `device`).
int resident_blocks(int device, const void* kern, size_t smem, int& blocks)
{
    {
        std::lock_guard<std::mutex> lock(g_info_mu);
        for (const OccupancyEntry& en : g_occupancy)
            if (en.device == device && en.kern == kern && en.smem == smem) {
                blocks = en.blocks;
                return TSDF_OK;
            }
    }
    int rc = allow_smem(device, kern, smem);
    if (rc != TSDF_OK) return rc;
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    std::lock_guard<std::mutex> lock(g_info_mu);
    g_occupancy.push_back({device, kern, smem, n});
    blocks = n;
    return TSDF_OK;
}

template <bool kFan, bool kMulti>
int launch(Kind kind, TraceArgs& a, int device, void* workspace, cudaStream_t stream, bool order = true,
           unsigned int* counter = nullptr)
{
    tsdf::DeviceScope scope(device);
    cudaError_t e = scope.error();
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    DeviceInfo info;
    int rc = device_info(device, info);
    if (rc != TSDF_OK) return rc;
    const int sms = info.sms;
    void (*kern)(TraceArgs);
    size_t base;  // shared memory besides the staged records
    if (kind == Kind::kGrid) {
        // the grid kernel reads records through L1 (staging the top records in shared
        // memory measured slower on every configuration); option smem_records applies to
        // the float kernel only
        a.n_smem = 0;
        kern = trace_grid_kernel<kFan, kMulti, 4>;
        base = static_cast<size_t>(kStackLevels + 3) * kThreads * 4u;  // descent stack, reciprocals
        if (!kMulti) base += 3u * static_cast<size_t>(line_row(1 << a.scene.depth)) * 4u;
    } else {
        kern = trace_float_kernel<kFan, kMulti>;
        base = 0;
    }
    // Stage no more top records than the register-limited occupancy leaves room for:
    // a deep grid (2^11 lines per axis) with 1024 records would drop a block per SM.
    const void* kid = reinterpret_cast<const void*>(kern);
    if (a.n_smem > 0) {
        int reg_blocks = 0;
        rc = resident_blocks(device, kid, base, reg_blocks);
        if (rc != TSDF_OK) return rc;
        if (reg_blocks > 0) {
            const int64_t per_block = static_cast<int64_t>(info.smem_per_sm) / reg_blocks - kSmemReservedPerBlock;
            const int64_t fit = (per_block - static_cast<int64_t>(base)) / 32;
            a.n_smem = static_cast<uint32_t>(std::max<int64_t>(0, std::min<int64_t>(a.n_smem, fit)));
        }
    }
    const size_t smem = base + static_cast<size_t>(a.n_smem) * 32u;
    rc = allow_smem(device, kid, smem);
    if (rc != TSDF_OK) return rc;
    int per_sm = static_cast<int>(g_blocks_per_sm.load());
    if (per_sm <= 0) {
        rc = resident_blocks(device, kid, smem, per_sm);
        if (rc != TSDF_OK) return rc;
        if (per_sm <= 0) return fail(TSDF_ERR_INVALID, "trace kernel does not fit on an SM with this shared-memory stage");
    }
    const int64_t need = (static_cast<int64_t>(a.n_rays) + kThreads - 1) / kThreads;
    const int blocks = static_cast<int>(std::min<int64_t>(static_cast<int64_t>(sms) * per_sm, need));
    if (counter) {
        a.counter = counter;  // cleared by the caller
        a.err = counter + 1;
    } else {
        a.counter = static_cast<unsigned int*>(workspace);
        a.err = a.counter + 1;
        e = cudaMemsetAsync(workspace, 0, kLaunchWords * sizeof(unsigned int), stream);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
    }
    if constexpr (!kMulti) {
        // claim order into the workspace after the counter: bucket counts and cursors,
        // the order itself, the per-ray bucket keys (per-scene launches bring their own)
        if (order) a.ray_perm = nullptr;
        if (order && g_order.load() == 1) {
            const size_t n = a.n_rays;
            auto* hist = reinterpret_cast<unsigned int*>(static_cast<char*>(workspace) + kScratchOffset);
            unsigned int* cursor = hist + kOrderBuckets;
            auto* perm = reinterpret_cast<uint32_t*>(cursor + kOrderBuckets);
            auto* key = reinterpret_cast<uint8_t*>(perm + n);
            const float buckets_per_unit = exit_buckets_per_unit(a.scene);
            const unsigned kb = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(sms) * 8));
            e = cudaMemsetAsync(hist, 0, 2 * kOrderBuckets * sizeof(unsigned int), stream);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(claim order)");
            order_key_kernel<kFan><<<kb, 256, 0, stream>>>(a, buckets_per_unit, key, hist);
            order_scatter_kernel<kFan><<<static_cast<unsigned>(std::min<int64_t>((n + kOrderTile - 1) / kOrderTile,
                                                                                 static_cast<int64_t>(sms) * 8)),
                                         256, 0, stream>>>(a, key, hist, cursor, perm);
            e = cudaGetLastError();
            if (e != cudaSuccess) return cuda_fail(e, "claim-order launch");
            a.ray_perm = perm;
        }
    }
    kern<<<blocks, kThreads, smem, stream>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "trace kernel launch");
    if constexpr (kBoundsCheck) {
        unsigned int bits = 0;
        e = cudaMemcpyAsync(&bits, a.err, sizeof bits, cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return cuda_fail(e, "reading the bounds-check word");
        if (bits) {
            char msg[96];
            std::snprintf(msg, sizeof msg, "bounds check failed in the trace kernel (bits 0x%x)", bits);
            return fail(TSDF_ERR_LAYOUT, msg);
        }
    }
    return TSDF_OK;
}

// Grid descent for this pool and box?  Cached per pool for the last box.
bool pool_grid_ok(tsdf_pool* pool, const float* bmin, const float* bmax)
{
    if (g_descent.load() != 0) return false;
    if (pool->height < 0 || pool->height > tsdf::kMaxGridDepth) return false;
    std::lock_guard<std::mutex> lock(pool->grid_mu);
    if (pool->grid_ok >= 0 && std::memcmp(pool->grid_bmin, bmin, sizeof pool->grid_bmin) == 0 &&
        std::memcmp(pool->grid_bmax, bmax, sizeof pool->grid_bmax) == 0)
        return pool->grid_ok == 1;
    std::vector<float> lines((static_cast<size_t>(1) << pool->height) + 2);
    bool ok = true;
    for (int axis = 0; axis < 3 && ok; ++axis) ok = tsdf::build_grid_lines(bmin[axis], bmax[axis], pool->height, lines.data());
    std::memcpy(pool->grid_bmin, bmin, sizeof pool->grid_bmin);
    std::memcpy(pool->grid_bmax, bmax, sizeof pool->grid_bmax);
    pool->grid_ok = ok ? 1 : 0;
    return ok;
}

// Multi-scene fan launches: actor order by scene (scene_sort_kernel) into perm_mem
// (4 bytes per actor of the caller's workspace), on `stream` before the trace.
constexpr uint32_t kMaxSortedScenes = 8192;  // shared-memory buckets of the sort

int sort_by_scene(TraceArgs& a, const tsdf_scenes* scenes, int64_t n_actors, void* perm_mem, cudaStream_t stream,
                  uint32_t* seg = nullptr)
{
    a.n_scenes = static_cast<uint32_t>(scenes->n);
    a.perm = nullptr;
    if (static_cast<uint32_t>(scenes->n) > kMaxSortedScenes) return TSDF_OK;  // actor order as given
    tsdf::DeviceScope scope(scenes->device);
    cudaError_t e = scope.error();
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    auto* perm = static_cast<uint32_t*>(perm_mem);
    const size_t smem = (static_cast<size_t>(scenes->n) + 1) * sizeof(unsigned int);
    scene_sort_kernel<<<1, 1024, smem, stream>>>(a.poses, static_cast<uint32_t>(n_actors),
                                                 static_cast<uint32_t>(scenes->n), perm, seg);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "scene sort launch");
    a.perm = perm;
    return TSDF_OK;
}

// Multiplier and shift of div_rpa for rays_per_actor (>= 1).
void set_rpa_divisor(TraceArgs& a)
{
    const uint32_t d = a.rays_per_actor ? a.rays_per_actor : 1u;
    uint32_t l = 0;
    while ((uint64_t(1) << l) < d) ++l;
    const uint64_t num = uint64_t(1) << (31 + l);
    a.rpa_magic = static_cast<uint32_t>((num + d - 1) / d);
    a.rpa_shift = 31 + l;
}

// Rays a warp claims with one atomicAdd: option "chunk" when set, else 16 where the
// launch's tail is exposed and 32 where it is not.  Larger chunks mean fewer atomics and
// longer runs of neighbouring rays per warp, but leave more claimed rays waiting in busy
// warps while others sit idle at the end.  Per-scene launches overlap their ends with
// the next launch on the other stream, and launches of 2^21 rays or more spend little of
// their time in the tail (measured with lanes refilled in pairs: config 2, 786k rays: 16
// beats 8, 4 and 64 by 1.7, 2.5 and 12 %; per-scene launches of config 5: 32 beats 16 and
// 64 by 0.1 and 1.4 %; before the paired refill, 4.2 M and 12.6 M rays: 32 won 1.6 % and
// 2.6 % over 8, and on config 2 8 beat 32 by 6 %).
uint32_t pick_chunk(uint32_t n_rays, bool per_scene)
{
    const int64_t c = g_chunk.load();
    if (c > 0) return static_cast<uint32_t>(c > 1024 ? 1024 : c);
    return (per_scene || n_rays >= (1u << 21)) ? 32u : 16u;
}

// Scene tables of up to kMaxPerSceneLaunch scenes trace one single-scene launch per
// scene (option "per_scene", default 1) instead of the multi-scene kernel: each launch
// keeps its scene in uniform parameters and its grid lines in shared memory and takes
// leaf runs, which the multi-scene kernel cannot (on config 3's actors all in one scene
// the multi-scene kernel is 12% slower than the single-scene one).  The actor order by
// scene and each scene's actor range come from scene_sort_kernel on the device, so the
// host needs no counts: every launch reads its range at start and exits at once when it
// is empty.  Workspace after the actor order: the scene bounds, then a work counter and
// error word per launch.
constexpr int kMaxPerSceneLaunch = 64;
constexpr size_t kPerSceneBytes = 1024;  // (kMaxPerSceneLaunch + 2) bounds + 2 words per launch
static_assert((kMaxPerSceneLaunch + 2) * 4 + kMaxPerSceneLaunch * 8 <= kPerSceneBytes, "per-scene workspace");
// claim order of each scene's rays: bucket counts and cursors per scene, then the order
// and the keys of all rays (each scene's at its own rays' offset)
constexpr size_t kPerSceneOrderBytes = static_cast<size_t>(kMaxPerSceneLaunch) * 2 * kOrderBuckets * 4;
std::atomic<int64_t> g_per_scene{1};

size_t actor_order_bytes(int64_t n_actors)
{
    return (static_cast<size_t>(n_actors) * 4u + 15u) & ~size_t(15);
}

bool per_scene_launches(const tsdf_scenes* scenes)
{
    return scenes->n > 1 && scenes->n <= kMaxPerSceneLaunch && g_per_scene.load() != 0;
}

// Library streams that per-scene launches alternate on, so that a launch's blocks fill
// the SMs the previous launch frees as its last rays finish (one pair per device, made
// on first use; the caller's stream forks to them and joins back through events, which
// stream capture follows).
constexpr int kPerSceneStreams = 2;
struct SceneStreams {
    cudaStream_t s[kPerSceneStreams] = {};
    cudaEvent_t fork = nullptr;
    cudaEvent_t join[kPerSceneStreams] = {};
    bool ready = false;
    std::mutex mu;  // one call at a time between fork and join: the events are shared
};
constexpr int kMaxStreamDevices = 64;
std::mutex g_streams_mu;
SceneStreams g_streams[kMaxStreamDevices];

SceneStreams* scene_streams(int device)
{
    if (device < 0 || device >= kMaxStreamDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_streams_mu);
    SceneStreams& st = g_streams[device];
    if (!st.ready) {
        bool ok = cudaEventCreateWithFlags(&st.fork, cudaEventDisableTiming) == cudaSuccess;
        for (int i = 0; i < kPerSceneStreams && ok; ++i)
            ok = cudaStreamCreateWithFlags(&st.s[i], cudaStreamNonBlocking) == cudaSuccess &&
                 cudaEventCreateWithFlags(&st.join[i], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            cudaGetLastError();
            return nullptr;  // the launches stay on the caller's stream
        }
        st.ready = true;
    }
    return &st;
}

int trace_per_scene(TraceArgs& a, const tsdf_scenes* scenes, int64_t n_actors, void* workspace, cudaStream_t stream)
{
    char* ws = static_cast<char*>(workspace);
    auto* seg = reinterpret_cast<uint32_t*>(ws + kScratchOffset + actor_order_bytes(n_actors));
    auto* counters = seg + (kMaxPerSceneLaunch + 2);
    auto* hist = reinterpret_cast<unsigned int*>(ws + kScratchOffset + actor_order_bytes(n_actors) + kPerSceneBytes);
    auto* ray_order = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(hist) + kPerSceneOrderBytes);
    auto* keys = reinterpret_cast<uint8_t*>(ray_order + a.n_rays);
    const bool order = g_order.load() == 1;
    tsdf::DeviceScope scope(scenes->device);
    cudaError_t e = scope.error();
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    DeviceInfo info;
    int rc = device_info(scenes->device, info);
    if (rc != TSDF_OK) return rc;
    const int sms = info.sms;
    rc = sort_by_scene(a, scenes, n_actors, ws + kScratchOffset, stream, seg);
    if (rc != TSDF_OK) return rc;
    e = cudaMemsetAsync(counters, 0, 2 * sizeof(unsigned int) * scenes->n, stream);
    if (e == cudaSuccess && order)
        e = cudaMemsetAsync(hist, 0, 2 * kOrderBuckets * sizeof(unsigned int) * scenes->n, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(per-scene counters)");
    const bool grid_ok = g_descent.load() == 0;
    SceneStreams* st = scene_streams(scenes->device);
    std::unique_lock<std::mutex> hold;
    if (st) hold = std::unique_lock<std::mutex>(st->mu);
    if (st) {
        e = cudaEventRecord(st->fork, stream);
        for (int i = 0; i < kPerSceneStreams && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(st->s[i], st->fork, 0);
        if (e != cudaSuccess) return cuda_fail(e, "forking the per-scene streams");
    }
    // After the fork every exit joins the side streams back to the caller's stream, the
    // failing ones included, so that the caller's stream stays ordered after the work
    // already queued there and a capture in progress sees no unjoined fork.
    auto join = [&]() -> cudaError_t {
        cudaError_t je = cudaSuccess;
        if (!st) return je;
        for (int i = 0; i < kPerSceneStreams; ++i) {
            cudaError_t r = cudaEventRecord(st->join[i], st->s[i]);
            if (r == cudaSuccess) r = cudaStreamWaitEvent(stream, st->join[i], 0);
            if (je == cudaSuccess) je = r;
        }
        return je;
    };
    for (int s = 0; s < scenes->n; ++s) {
        TraceArgs b = a;
        b.table = nullptr;
        b.n_scenes = 0;
        b.scene = scenes->host[s];
        b.seg = seg + s;
        b.chunk = pick_chunk(b.n_rays, true);
        b.n_smem = static_cast<uint32_t>(std::min<int64_t>(std::max<int64_t>(g_smem_records.load(), 0),
                                                           static_cast<int64_t>(b.scene.n_recs)));
        const bool grid = grid_ok && b.scene.depth >= 0;
        if (!grid) b.scene.depth = -1;
        const cudaStream_t ss = st ? st->s[s % kPerSceneStreams] : stream;
        b.ray_perm = nullptr;
        if (order) {  // the scene's rays by box-exit distance, longest first
            unsigned int* h = hist + 2 * kOrderBuckets * s;
            const unsigned grid_n = static_cast<unsigned>(sms) * 8u;
            order_key_kernel<true><<<grid_n, 256, 0, ss>>>(b, exit_buckets_per_unit(b.scene), keys, h);
            order_scatter_kernel<true><<<grid_n, 256, 0, ss>>>(b, keys, h, h + kOrderBuckets, ray_order);
            e = cudaGetLastError();
            if (e != cudaSuccess) {
                join();
                return cuda_fail(e, "per-scene claim-order launch");
            }
            b.ray_perm = ray_order;
        }
        rc = launch<true, false>(grid ? Kind::kGrid : Kind::kFloat, b, scenes->device, workspace, ss,
                                 /*order=*/false, counters + 2 * s);
        if (rc != TSDF_OK) {
            join();  // keeps the launch's error message: a join failure is secondary
            return rc;
        }
    }
    e = join();
    if (e != cudaSuccess) return cuda_fail(e, "joining the per-scene streams");
    unknown_scene_kernel<<<static_cast<unsigned>(sms), 256, 0, stream>>>(
        seg + scenes->n, a.perm, static_cast<uint32_t>(n_actors), a.rays_per_actor, a.out_d, a.out_s, a.out_steps);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "unknown-scene launch");
    return TSDF_OK;
}

}  // namespace

extern "C" {

int tsdf_cast(const tsdf_pool* pool, const float* origins, const float* dirs, int64_t n_rays,
              float* out_dist, int32_t* out_sem, int32_t* out_steps, int max_steps,
              float max_distance, const float bbox_min[3], const float bbox_max[3],
              float hit_epsilon, void* workspace, void* stream)
{
    if (!pool) return fail(TSDF_ERR_INVALID, "pool must not be null");
    int rc = common_checks(n_rays, out_dist, out_sem, max_steps, max_distance, workspace);
    if (rc != TSDF_OK) return rc;
    if (!bbox_min || !bbox_max) return fail(TSDF_ERR_INVALID, "bbox_min and bbox_max must contain exactly 3 floats");
    if (!finite3(bbox_min) || !finite3(bbox_max))
        return fail(TSDF_ERR_INVALID, "bbox_min and bbox_max must contain only finite floats");
    for (int i = 0; i < 3; ++i)
        if (!(bbox_min[i] < bbox_max[i]))
            return fail(TSDF_ERR_INVALID, "bbox_min entries must be strictly less than bbox_max entries");
    if (std::isnan(hit_epsilon)) return fail(TSDF_ERR_INVALID, "hit_epsilon must not be NaN");
    if (n_rays == 0) return TSDF_OK;
    if (!origins || !dirs) return fail(TSDF_ERR_INVALID, "origins and dirs must not be null");

    TraceArgs a;
    std::memset(&a, 0, sizeof a);
    a.scene.recs = pool->d_recs;
    a.scene.ext = pool->d_ext;
    a.scene.root = pool->root;
    a.scene.n_recs = static_cast<uint32_t>(pool->records);
    a.scene.n_ext = static_cast<uint32_t>(pool->ext);
    for (int i = 0; i < 3; ++i) {
        a.scene.bmin[i] = bbox_min[i];
        a.scene.bmax[i] = bbox_max[i];
    }
    a.scene.eps = hit_epsilon;
    a.origins = origins;
    a.dirs = dirs;
    a.n_rays = static_cast<uint32_t>(n_rays);
    a.max_steps = max_steps;
    a.max_distance = max_distance;
    a.n_smem = static_cast<uint32_t>(std::min<int64_t>(std::max<int64_t>(g_smem_records.load(), 0),
                                                       static_cast<int64_t>(pool->records)));
    a.chunk = pick_chunk(a.n_rays, false);
    a.leaf_run = static_cast<uint32_t>(g_leaf_run.load());
    a.out_d = out_dist;
    a.out_s = out_sem;
    a.out_steps = out_steps;
    const bool grid = pool_grid_ok(const_cast<tsdf_pool*>(pool), bbox_min, bbox_max);
    a.scene.depth = grid ? pool->height : -1;
    tsdf::set_grid_scale(a.scene);
    return launch<false, false>(grid ? Kind::kGrid : Kind::kFloat, a, pool->device, workspace,
                                static_cast<cudaStream_t>(stream));
}

int tsdf_cast_fan(const tsdf_scenes* scenes, const tsdf_pose* poses, int64_t n_actors,
                  const float* fan_dirs, int64_t rays_per_actor, int use_pitch, float* out_dist,
                  int32_t* out_sem, int32_t* out_steps, int max_steps, float max_distance,
                  void* workspace, void* stream)
{
    if (!scenes || scenes->n <= 0) return fail(TSDF_ERR_INVALID, "scenes must not be null");
    if (n_actors < 0 || rays_per_actor < 0) return fail(TSDF_ERR_INVALID, "sizes must not be negative");
    if (rays_per_actor > 0 && n_actors > kMaxRays / rays_per_actor)
        return fail(TSDF_ERR_INVALID, "number of rays must be in [0, 2^31 - 2^24]");
    const int64_t n_rays = n_actors * rays_per_actor;
    int rc = common_checks(n_rays, out_dist, out_sem, max_steps, max_distance, workspace);
    if (rc != TSDF_OK) return rc;
    if (n_rays == 0) return TSDF_OK;
    if (!poses || !fan_dirs) return fail(TSDF_ERR_INVALID, "poses and fan_dirs must not be null");
    if (reinterpret_cast<uintptr_t>(poses) % 16u != 0)
        return fail(TSDF_ERR_INVALID, "poses must be 16-byte aligned");

    TraceArgs a;
    std::memset(&a, 0, sizeof a);
    a.poses = reinterpret_cast<const float4*>(poses);
    a.fan = fan_dirs;
    a.rays_per_actor = static_cast<uint32_t>(rays_per_actor);
    set_rpa_divisor(a);
    a.use_pitch = use_pitch ? 1 : 0;
    a.n_rays = static_cast<uint32_t>(n_rays);
    a.max_steps = max_steps;
    a.max_distance = max_distance;
    a.chunk = pick_chunk(a.n_rays, false);
    a.leaf_run = static_cast<uint32_t>(g_leaf_run.load());
    a.out_d = out_dist;
    a.out_s = out_sem;
    a.out_steps = out_steps;
    if (scenes->n == 1) {
        a.scene = scenes->host[0];
        a.n_smem = static_cast<uint32_t>(std::min<int64_t>(std::max<int64_t>(g_smem_records.load(), 0),
                                                           static_cast<int64_t>(a.scene.n_recs)));
        const bool grid = scenes->grid && g_descent.load() == 0;
        if (!grid) a.scene.depth = -1;
        return launch<true, false>(grid ? Kind::kGrid : Kind::kFloat, a, scenes->device, workspace,
                                   static_cast<cudaStream_t>(stream));
    }
    a.table = scenes->d_table;
    a.scene = scenes->host[0];
    if (per_scene_launches(scenes)) return trace_per_scene(a, scenes, n_actors, workspace, static_cast<cudaStream_t>(stream));
    rc = sort_by_scene(a, scenes, n_actors, static_cast<char*>(workspace) + kScratchOffset,
                       static_cast<cudaStream_t>(stream));
    if (rc != TSDF_OK) return rc;
    return launch<true, true>(scenes->grid && g_descent.load() == 0 ? Kind::kGrid : Kind::kFloat, a, scenes->device, workspace,
                              static_cast<cudaStream_t>(stream));
}

uint64_t tsdf_workspace_bytes(int64_t n_rays)
{
    return n_rays <= 0 ? kScratchOffset : kScratchOffset + order_scratch_bytes(n_rays);
}

uint64_t tsdf_fan_workspace_bytes(const tsdf_scenes* scenes, int64_t n_actors, int64_t rays_per_actor)
{
    if (n_actors <= 0 || rays_per_actor <= 0) return kScratchOffset;
    const uint64_t n_rays = static_cast<uint64_t>(n_actors) * static_cast<uint64_t>(rays_per_actor);
    const uint64_t by_scene = actor_order_bytes(n_actors) + kPerSceneBytes +
                              ((!scenes || scenes->n <= kMaxPerSceneLaunch)
                                   ? kPerSceneOrderBytes + 4u * n_rays + ((n_rays + 15u) & ~uint64_t(15)) : 0u);
    const uint64_t order = order_scratch_bytes(n_actors * rays_per_actor);
    if (!scenes) return kScratchOffset + std::max(by_scene, order);
    return kScratchOffset + (scenes->n > 1 ? by_scene : order);
}

uint64_t tsdf_observe_workspace_bytes(const tsdf_scenes* scenes, int64_t n_actors, int64_t rays_per_actor)
{
    return tsdf_fan_workspace_bytes(scenes, n_actors, rays_per_actor);
}

int tsdf_cast_fan_observe(const tsdf_scenes* scenes, const tsdf_pose* poses, int64_t n_actors,
                          const float* fan_dirs, int64_t rays_per_actor, int use_pitch, float* out_dist,
                          int32_t* out_sem, int32_t* out_steps, int max_steps, float max_distance,
                          const tsdf_observe* observe, void* workspace, void* stream)
{
    if (!observe) return fail(TSDF_ERR_INVALID, "observe must not be null");
    if (!scenes || scenes->n <= 0) return fail(TSDF_ERR_INVALID, "scenes must not be null");
    if (observe->azimuth_bins <= 0 || observe->elevation_bins <= 0 ||
        static_cast<int64_t>(observe->azimuth_bins) * observe->elevation_bins != rays_per_actor)
        return fail(TSDF_ERR_INVALID, "azimuth_bins * elevation_bins must equal rays_per_actor");
    if (n_actors < 0 || rays_per_actor < 0) return fail(TSDF_ERR_INVALID, "sizes must not be negative");
    if (rays_per_actor > 0 && n_actors > kMaxRays / rays_per_actor)
        return fail(TSDF_ERR_INVALID, "number of rays must be in [0, 2^31 - 2^24]");
    const int64_t n_rays = n_actors * rays_per_actor;
    int rc = common_checks(n_rays, out_dist, out_sem, max_steps, max_distance, workspace);
    if (rc != TSDF_OK) return rc;
    if (n_rays == 0) return TSDF_OK;
    if (!poses || !fan_dirs) return fail(TSDF_ERR_INVALID, "poses and fan_dirs must not be null");
    if (!observe->observation || !observe->actor_stats)
        return fail(TSDF_ERR_INVALID, "observation and actor_stats must not be null");
    if (reinterpret_cast<uintptr_t>(poses) % 16u != 0)
        return fail(TSDF_ERR_INVALID, "poses must be 16-byte aligned");

    TraceArgs a;
    std::memset(&a, 0, sizeof a);
    a.poses = reinterpret_cast<const float4*>(poses);
    a.fan = fan_dirs;
    a.rays_per_actor = static_cast<uint32_t>(rays_per_actor);
    set_rpa_divisor(a);
    a.use_pitch = use_pitch ? 1 : 0;
    a.n_rays = static_cast<uint32_t>(n_rays);
    a.max_steps = max_steps;
    a.max_distance = max_distance;
    a.chunk = pick_chunk(a.n_rays, false);
    a.leaf_run = static_cast<uint32_t>(g_leaf_run.load());
    a.out_d = out_dist;
    a.out_s = out_sem;
    a.out_steps = out_steps;
    ObserveArgs ob;
    std::memset(&ob, 0, sizeof ob);
    ob.rays_per_actor = a.rays_per_actor;
    ob.az_bins = static_cast<uint32_t>(observe->azimuth_bins);
    ob.el_bins = static_cast<uint32_t>(observe->elevation_bins);
    ob.fwd_half = static_cast<uint32_t>(std::max(1, observe->azimuth_bins / 6));
    ob.max_distance = max_distance;
    // the reference's scalars are Python floats: thresholds are formed in double, then
    // rounded to float32 by the tensor op; torch divides by the scalar log1p(max) by
    // multiplying with its reciprocal formed in double and rounded once to float32
    ob.sat_thr = static_cast<float>(static_cast<double>(max_distance) - 1e-3);
    ob.band_min = observe->structure_band_min;
    ob.band_max = observe->structure_band_max;
    ob.prox = observe->proximity_threshold;
    ob.band_on = observe->structure_band_max > observe->structure_band_min ? 1 : 0;
    ob.prox_on = observe->proximity_threshold > 0.0f ? 1 : 0;
    ob.inv_log_denom = static_cast<float>(1.0 / std::log1p(static_cast<double>(max_distance)));
    const float fa = static_cast<float>(n_actors);
    ob.f_all = fa / static_cast<float>(n_rays);
    ob.f_fwd = fa / static_cast<float>(n_actors * 2 * static_cast<int64_t>(ob.fwd_half) * observe->elevation_bins);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    tsdf::DeviceScope scope(scenes->device);  // the observation pass launches on the scenes' device too
    cudaError_t se = scope.error();
    if (se != cudaSuccess) return cuda_fail(se, "cudaSetDevice");
    if (scenes->n == 1) {
        a.scene = scenes->host[0];
        a.n_smem = static_cast<uint32_t>(std::min<int64_t>(std::max<int64_t>(g_smem_records.load(), 0),
                                                           static_cast<int64_t>(a.scene.n_recs)));
        const bool grid = scenes->grid && g_descent.load() == 0;
        if (!grid) a.scene.depth = -1;
        rc = launch<true, false>(grid ? Kind::kGrid : Kind::kFloat, a, scenes->device, workspace, s);
    } else if (per_scene_launches(scenes)) {
        a.table = scenes->d_table;
        a.scene = scenes->host[0];
        rc = trace_per_scene(a, scenes, n_actors, workspace, s);
    } else {
        a.table = scenes->d_table;
        a.scene = scenes->host[0];
        rc = sort_by_scene(a, scenes, n_actors, static_cast<char*>(workspace) + kScratchOffset, s);
        if (rc == TSDF_OK)
            rc = launch<true, true>(scenes->grid && g_descent.load() == 0 ? Kind::kGrid : Kind::kFloat, a,
                                    scenes->device, workspace, s);
    }
    if (rc != TSDF_OK) return rc;
    // one block per actor, up to 1024 threads: a few rays per thread even for small batches
    const unsigned threads = static_cast<unsigned>(std::min<int64_t>(1024, std::max<int64_t>(32, (rays_per_actor + 31) / 32 * 32)));
    observe_kernel<<<static_cast<unsigned>(n_actors), threads, 0, s>>>(out_dist, out_sem, observe->observation,
                                                                       observe->actor_stats, ob);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "observation pass launch");
    return TSDF_OK;
}

int tsdf_set_option(const char* key, int64_t value, int64_t* old_value)
{
    if (!key) return fail(TSDF_ERR_INVALID, "key must not be null");
    std::atomic<int64_t>* slot = nullptr;
    if (std::strcmp(key, "smem_records") == 0) {
        if (value < 0 || value > 6000) return fail(TSDF_ERR_INVALID, "smem_records must be in [0, 6000]");
        slot = &g_smem_records;
    } else if (std::strcmp(key, "chunk") == 0) {
        if (value < 0 || value > 1024) return fail(TSDF_ERR_INVALID, "chunk must be in [0, 1024] (0: automatic)");
        slot = &g_chunk;
    } else if (std::strcmp(key, "leaf_run") == 0) {
        if (value < 0 || value > 4096) return fail(TSDF_ERR_INVALID, "leaf_run must be in [0, 4096]");
        slot = &g_leaf_run;
    } else if (std::strcmp(key, "per_scene") == 0) {
        if (value < 0 || value > 1) return fail(TSDF_ERR_INVALID, "per_scene must be 0 or 1");
        slot = &g_per_scene;
    } else if (std::strcmp(key, "order") == 0) {
        if (value < 0 || value > 1) return fail(TSDF_ERR_INVALID, "order must be 0 or 1");
        slot = &g_order;
    } else if (std::strcmp(key, "descent") == 0) {
        if (value < 0 || value > 1) return fail(TSDF_ERR_INVALID, "descent must be 0 (grid where possible) or 1 (float)");
        slot = &g_descent;
    } else if (std::strcmp(key, "blocks_per_sm") == 0) {
        if (value < 0 || value > 32) return fail(TSDF_ERR_INVALID, "blocks_per_sm must be in [0, 32]");
        slot = &g_blocks_per_sm;
    } else {
        return fail(TSDF_ERR_INVALID, std::string("unknown option: ") + key);
    }
    const int64_t old = slot->exchange(value);
    if (old_value) *old_value = old;
    return TSDF_OK;
}

}  // extern "C"

// ============================================================================
// Allocation-free cast.
//
// tsdf_cast needs a caller-provided device workspace (the work-queue counter of
// the persistent kernel).  Some callers cannot allocate device memory once they
// are running: a fixed-rate control loop (on the vehicle, say) must not stall in
// cudaMalloc, which may synchronise the whole device, and a host that only
// hands the library buffers it registered up front has nothing to hand over for
// scratch.  tsdf_cast_noalloc takes no workspace: the counter lives in the
// file-scope device array below, which every GPU that loads this library holds
// until the process exits.
//
// Host code may not use the array's name as a device address (on the host it
// names a stand-in object), so the address is fetched once per device with
// cudaGetSymbolAddress, with that device current, by the first call on that
// device.  Make that first call before any stream capture.  All calls on a
// device share the array and it keeps the last call's contents: the counter is
// cleared (cudaMemsetAsync on the caller's stream) before every launch, and two
// calls whose kernels overlap on the GPU (different streams, no ordering between
// them) race on it and produce wrong outputs; order them on one stream.  The
// fetched address belongs to the device's current context: after cudaDeviceReset
// on that device it is stale, so a process that resets a device must not call
// this entry point on it again.
// ============================================================================

constexpr size_t kNoAllocScratchBytes = 256;  // stated maximum scratch of one cast
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};
float g_noalloc_lines[(1 << tsdf::kMaxGridDepth) + 2];  // grid-line check buffer, under g_noalloc_mu

// Same decision as pool_grid_ok, with a static buffer instead of a heap vector.
bool noalloc_grid_ok(tsdf_pool* pool, const float* bmin, const float* bmax)
{
    if (g_descent.load() != 0) return false;
    if (pool->height < 0 || pool->height > tsdf::kMaxGridDepth) return false;
    std::lock_guard<std::mutex> lock(pool->grid_mu);
    if (pool->grid_ok >= 0 && std::memcmp(pool->grid_bmin, bmin, sizeof pool->grid_bmin) == 0 &&
        std::memcmp(pool->grid_bmax, bmax, sizeof pool->grid_bmax) == 0)
        return pool->grid_ok == 1;
    bool ok = true;
    {
        std::lock_guard<std::mutex> buf_lock(g_noalloc_mu);
        for (int axis = 0; axis < 3 && ok; ++axis)
            ok = tsdf::build_grid_lines(bmin[axis], bmax[axis], pool->height, g_noalloc_lines);
    }
    std::memcpy(pool->grid_bmin, bmin, sizeof pool->grid_bmin);
    std::memcpy(pool->grid_bmax, bmax, sizeof pool->grid_bmax);
    pool->grid_ok = ok ? 1 : 0;
    return ok;
}
}  // namespace

extern "C" int tsdf_cast_noalloc(const tsdf_pool* pool, const float* origins, const float* dirs,
                                 int64_t n_rays, float* out_dist, int32_t* out_sem, int32_t* out_steps,
                                 int max_steps, float max_distance, const float bbox_min[3],
                                 const float bbox_max[3], float hit_epsilon, void* stream)
{
    if (!pool) return fail(TSDF_ERR_INVALID, "pool must not be null");
    // the persistent kernel's scratch: its work counter and the error word after it
    const size_t need = kLaunchWords * sizeof(unsigned int);
    if (need > kNoAllocScratchBytes)
        return fail(TSDF_ERR_INVALID, "tsdf_cast_noalloc: the cast needs more scratch than the 256-byte static array");
    if (pool->device < 0 || pool->device >= kNoAllocMaxDevices)
        return fail(TSDF_ERR_INVALID, "tsdf_cast_noalloc supports device ordinals 0..63");
    static int present;  // stands for the workspace argument this entry point does not take
    int rc = common_checks(n_rays, out_dist, out_sem, max_steps, max_distance, &present);
    if (rc != TSDF_OK) return rc;
    if (!bbox_min || !bbox_max) return fail(TSDF_ERR_INVALID, "bbox_min and bbox_max must contain exactly 3 floats");
    if (!finite3(bbox_min) || !finite3(bbox_max))
        return fail(TSDF_ERR_INVALID, "bbox_min and bbox_max must contain only finite floats");
    for (int i = 0; i < 3; ++i)
        if (!(bbox_min[i] < bbox_max[i]))
            return fail(TSDF_ERR_INVALID, "bbox_min entries must be strictly less than bbox_max entries");
    if (std::isnan(hit_epsilon)) return fail(TSDF_ERR_INVALID, "hit_epsilon must not be NaN");
    if (n_rays == 0) return TSDF_OK;
    if (!origins || !dirs) return fail(TSDF_ERR_INVALID, "origins and dirs must not be null");

    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_addr[pool->device]) {
            tsdf::DeviceScope scope(pool->device);  // the address is per device; the caller's device is kept
            cudaError_t e = scope.error();
            if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
            void* addr = nullptr;
            e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
            g_noalloc_addr[pool->device] = addr;
        }
        scratch = g_noalloc_addr[pool->device];
    }

    TraceArgs a;
    std::memset(&a, 0, sizeof a);
    a.scene.recs = pool->d_recs;
    a.scene.ext = pool->d_ext;
    a.scene.root = pool->root;
    a.scene.n_recs = static_cast<uint32_t>(pool->records);
    a.scene.n_ext = static_cast<uint32_t>(pool->ext);
    for (int i = 0; i < 3; ++i) {
        a.scene.bmin[i] = bbox_min[i];
        a.scene.bmax[i] = bbox_max[i];
    }
    a.scene.eps = hit_epsilon;
    a.origins = origins;
    a.dirs = dirs;
    a.n_rays = static_cast<uint32_t>(n_rays);
    a.max_steps = max_steps;
    a.max_distance = max_distance;
    a.n_smem = static_cast<uint32_t>(std::min<int64_t>(std::max<int64_t>(g_smem_records.load(), 0),
                                                       static_cast<int64_t>(pool->records)));
    a.chunk = pick_chunk(a.n_rays, false);
    a.leaf_run = static_cast<uint32_t>(g_leaf_run.load());
    a.out_d = out_dist;
    a.out_s = out_sem;
    a.out_steps = out_steps;
    const bool grid = noalloc_grid_ok(const_cast<tsdf_pool*>(pool), bbox_min, bbox_max);
    a.scene.depth = grid ? pool->height : -1;
    tsdf::set_grid_scale(a.scene);
    return launch<false, false>(grid ? Kind::kGrid : Kind::kFloat, a, pool->device, scratch,
                                static_cast<cudaStream_t>(stream), /*order=*/false);
}
