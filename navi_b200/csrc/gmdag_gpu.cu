// Device scene compiler: triangle mesh -> dense unsigned SDF -> .gmdag DAG words on one GPU.
//
// Same output words as the host compiler (gmdag_compiler.cpp) and therefore as the
// reference voxel-dag compiler (projects/voxel-dag/src/compiler.cpp) for power-of-two
// resolutions; the float arithmetic lives in gmdag_math.h and this file is built with
// -fmad=false and IEEE division / square root so that every value is the host's.
//
// Stages and how each maps to the GPU:
//   seeding  (compiler.cpp:453-490)  one CTA per work item (a triangle's voxel box, cut
//            into pieces of at most kItemVoxels voxels); the grid update is a min, done
//            with atomicMin on the float's bits (all distances are >= +0, and NaN bit
//            patterns compare above FLT_MAX so they never win, as `d < grid` rejects them).
//   sweeps   (compiler.cpp:492-529)  each of the 8 Gauss-Seidel sweeps reads only the
//            three upwind neighbours, all already updated in the same sweep.  The grid is
//            cut into 16^3 tiles; tiles on one anti-diagonal X+Y+Z = k (sweep order) are
//            independent, one launch per diagonal.  Inside a tile the voxels on one plane
//            x+y+z = p are independent, one __syncthreads per plane.  The values are the
//            ones of the sequential z/y/x loop.
//   pyramids min/max of aligned 2^L blocks, L = 1..log2 N (the uniform-block test of
//            compiler.cpp:600-613 and block minima of :563-577 read them).
//   DAG      (compiler.cpp:579-674)  level by level: top-down, the blocks the recursive
//            build visits (root; children of a non-uniform block whose minimum is within
//            the octant extent), with their leaf words; bottom-up, internal nodes are
//            deduplicated structurally in a device hash table (mask + child identities,
//            compared in full, across levels as the reference's single map does).  The
//            host then emits the unique nodes in the reference's post-order (octants
//            0..7, first occurrence wins, root copied to word 0): a depth-first walk of
//            the deduplicated DAG that skips nodes already emitted gives exactly the
//            order of the reference's walk of the full tree, whose repeated subtrees
//            emit nothing.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include <cub/device/device_scan.cuh>

#include "gmdag.h"
#include "gmdag_math.h"

namespace {

thread_local std::string g_err;

constexpr float kBig = std::numeric_limits<float>::max();
constexpr int kTile = 16;                 // sweep tile edge (voxels)
constexpr uint32_t kItemVoxels = 4096;    // seeding work item size
constexpr int kMaxLevels = 13;            // log2(4096) + 1
constexpr unsigned long long kEmpty = ~0ull;

struct CudaError {
    cudaError_t e;
    const char* what;
};

#define CK(call)                                   \
    do {                                           \
        const cudaError_t e_ = (call);             \
        if (e_ != cudaSuccess) throw CudaError{e_, #call}; \
    } while (0)

template <class T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() { reset(); }
    void reset()
    {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    void alloc(size_t count)
    {
        reset();
        if (count == 0) count = 1;
        CK(cudaMalloc(&p, count * sizeof(T)));
        n = count;
    }
};

struct GpuResult {
    std::vector<uint64_t> words;
    float bmin[3] = {0, 0, 0};
    float bmax[3] = {0, 0, 0};
    float voxel = 0;
    gmdag_gpu_timing timing{};
};

using Clock = std::chrono::steady_clock;
double ms_since(Clock::time_point t0)
{
    return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

__host__ __device__ __forceinline__ size_t vidx(int x, int y, int z, int N)
{
    return (static_cast<size_t>(z) * N + y) * N + x;
}

// ------------------------------------------------------------------ seeding

struct SeedItem {
    uint32_t tri;
    uint16_t x0, xn, y0, yn, z0, zn;
};
static_assert(sizeof(SeedItem) == 16, "seed item layout");

__global__ void fill_kernel(float* __restrict__ g, size_t n, float v)
{
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        g[i] = v;
}

__global__ void __launch_bounds__(128) seed_kernel(float* __restrict__ g, int N, const float* __restrict__ verts,
                                                   const uint32_t* __restrict__ idx,
                                                   const SeedItem* __restrict__ items, uint32_t n_items,
                                                   float bx, float by, float bz, float dx, float dy, float dz)
{
    for (uint32_t w = blockIdx.x; w < n_items; w += gridDim.x) {
        const SeedItem it = items[w];
        float v0[3], v1[3], v2[3];
        const uint32_t i0 = idx[3 * static_cast<size_t>(it.tri)];
        const uint32_t i1 = idx[3 * static_cast<size_t>(it.tri) + 1];
        const uint32_t i2 = idx[3 * static_cast<size_t>(it.tri) + 2];
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            v0[a] = verts[3 * static_cast<size_t>(i0) + a];
            v1[a] = verts[3 * static_cast<size_t>(i1) + a];
            v2[a] = verts[3 * static_cast<size_t>(i2) + a];
        }
        const uint32_t xn = it.xn, yn = it.yn;
        const uint32_t total = xn * yn * it.zn;
        for (uint32_t v = threadIdx.x; v < total; v += blockDim.x) {
            const uint32_t r = v / xn;
            const int x = it.x0 + static_cast<int>(v - r * xn);
            const uint32_t q = r / yn;
            const int y = it.y0 + static_cast<int>(r - q * yn);
            const int z = it.z0 + static_cast<int>(q);
            // compiler.cpp:472-486: voxel corner position, exact distance, keep the minimum
            const float pz = bz + z * dz;
            const float py = by + y * dy;
            const float px = bx + x * dx;
            const float d = sqrtf(gmdag::point_triangle_dist_sq(px, py, pz, v0, v1, v2));
            atomicMin(reinterpret_cast<unsigned int*>(g + vidx(x, y, z, N)), __float_as_uint(d));
        }
    }
}

// ------------------------------------------------------------------ sweeps

// Tile (X, Y, Z) of anti-diagonal k in sweep coordinates (xp = x for +x sweeps,
// N-1-x for -x sweeps, likewise y and z).
__global__ void __launch_bounds__(kTile * kTile) sweep_kernel(float* __restrict__ g, int N, int NT, int k, int sx,
                                                              int sy, int sz, float h, int z_first)
{
    const int Z = z_first + static_cast<int>(blockIdx.y);
    const int Y = max(0, k - Z - (NT - 1)) + static_cast<int>(blockIdx.x);
    const int X = k - Y - Z;
    if (Y > min(NT - 1, k - Z) || X < 0 || X >= NT) return;  // whole block: no barrier reached

    __shared__ float t[kTile + 1][kTile + 1][kTile + 1];  // [z][y][x], index 0 = upwind face
    const int xb = X * kTile, yb = Y * kTile, zb = Z * kTile;
    auto mx = [&](int xp) { return sx > 0 ? xp : N - 1 - xp; };
    auto my = [&](int yp) { return sy > 0 ? yp : N - 1 - yp; };
    auto mz = [&](int zp) { return sz > 0 ? zp : N - 1 - zp; };

    for (int i = threadIdx.x; i < kTile * kTile * kTile; i += blockDim.x) {
        const int xx = i % kTile, yy = (i / kTile) % kTile, zz = i / (kTile * kTile);
        const int xp = xb + xx, yp = yb + yy, zp = zb + zz;
        float v = kBig;
        if (xp < N && yp < N && zp < N) v = g[vidx(mx(xp), my(yp), mz(zp), N)];
        t[zz + 1][yy + 1][xx + 1] = v;
    }
    for (int i = threadIdx.x; i < 3 * kTile * kTile; i += blockDim.x) {
        const int f = i / (kTile * kTile);
        const int u = i % kTile, w = (i / kTile) % kTile;
        float v = kBig;
        if (f == 0) {  // x face: (yy, zz) = (u, w) at xp = xb - 1
            const int yp = yb + u, zp = zb + w;
            if (xb > 0 && yp < N && zp < N) v = g[vidx(mx(xb - 1), my(yp), mz(zp), N)];
            t[w + 1][u + 1][0] = v;
        } else if (f == 1) {  // y face: (xx, zz) = (u, w) at yp = yb - 1
            const int xp = xb + u, zp = zb + w;
            if (yb > 0 && xp < N && zp < N) v = g[vidx(mx(xp), my(yb - 1), mz(zp), N)];
            t[w + 1][0][u + 1] = v;
        } else {  // z face: (xx, yy) = (u, w) at zp = zb - 1
            const int xp = xb + u, yp = yb + w;
            if (zb > 0 && xp < N && yp < N) v = g[vidx(mx(xp), my(yp), mz(zb - 1), N)];
            t[0][w + 1][u + 1] = v;
        }
    }
    __syncthreads();

    const int yy = threadIdx.x % kTile, zz = threadIdx.x / kTile;
    const bool line_ok = (yb + yy < N) && (zb + zz < N);
    for (int p = 0; p < 3 * kTile - 2; ++p) {
        const int xx = p - yy - zz;
        if (line_ok && xx >= 0 && xx < kTile && xb + xx < N) {
            // compiler.cpp:515-525: upwind a (x), b (y), c (z); keep the smaller value
            const float a = t[zz + 1][yy + 1][xx];
            const float b = t[zz + 1][yy][xx + 1];
            const float c = t[zz][yy + 1][xx + 1];
            const float u = gmdag::eikonal_update(a, b, c, h);
            if (u < t[zz + 1][yy + 1][xx + 1]) t[zz + 1][yy + 1][xx + 1] = u;
        }
        __syncthreads();
    }

    for (int i = threadIdx.x; i < kTile * kTile * kTile; i += blockDim.x) {
        const int xx = i % kTile, yy2 = (i / kTile) % kTile, zz2 = i / (kTile * kTile);
        const int xp = xb + xx, yp = yb + yy2, zp = zb + zz2;
        if (xp < N && yp < N && zp < N) g[vidx(mx(xp), my(yp), mz(zp), N)] = t[zz2 + 1][yy2 + 1][xx + 1];
    }
}

// ------------------------------------------------------------------ pyramids

__global__ void pyramid_kernel(const float* __restrict__ smn, const float* __restrict__ smx, float* __restrict__ dmn,
                               float* __restrict__ dmx, int M)
{
    const size_t total = static_cast<size_t>(M) * M * M;
    const int P = 2 * M;
    for (size_t d = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; d < total;
         d += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int x = static_cast<int>(d % M);
        const int y = static_cast<int>((d / M) % M);
        const int z = static_cast<int>(d / (static_cast<size_t>(M) * M));
        float lo = __int_as_float(0x7f800000);
        float hi = -__int_as_float(0x7f800000);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const size_t s = vidx(2 * x + (k & 1), 2 * y + ((k >> 1) & 1), 2 * z + ((k >> 2) & 1), P);
            const float a = smn[s], b = smx[s];
            lo = (a < lo) ? a : lo;  // std::min(lo, a)
            hi = (hi < b) ? b : hi;  // std::max(hi, b)
        }
        dmn[d] = lo;
        dmx[d] = hi;
    }
}

// ------------------------------------------------------------------ DAG levels

__host__ __device__ __forceinline__ uint64_t pack_block(uint32_t x, uint32_t y, uint32_t z)
{
    return static_cast<uint64_t>(x) | (static_cast<uint64_t>(y) << 21) | (static_cast<uint64_t>(z) << 42);
}

struct LevelView {
    const uint64_t* canon[kMaxLevels];
    const uint32_t* kid_off[kMaxLevels];
    const uint8_t* mask[kMaxLevels];
};

// Blocks of level L (edge 2^L): leaf word, or (mask, number of children).
__global__ void classify_kernel(const uint64_t* __restrict__ blocks, uint32_t n, int L, int N,
                                const float* __restrict__ grid, const float* __restrict__ mnL,
                                const float* __restrict__ mxL, const float* __restrict__ mnC, float voxel,
                                uint64_t* __restrict__ canon, uint8_t* __restrict__ mask, uint32_t* __restrict__ nk)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t b = blocks[i];
    const int bx = static_cast<int>(b & 0x1FFFFF), by = static_cast<int>((b >> 21) & 0x1FFFFF),
              bz = static_cast<int>(b >> 42);
    const int size = 1 << L;
    const int M = N >> L;
    const float two_vox = voxel * 2.0f;
    const float first = grid[vidx(bx * size, by * size, bz * size, N)];
    const size_t k = vidx(bx, by, bz, M);
    const float lo = mnL[k], hi = mxL[k];
    uint64_t word = 0;
    uint8_t m = 0;
    if (gmdag::uniform_block(lo, hi, first)) {
        word = gmdag::leaf_word(first, first < two_vox ? 1 : 0);  // compiler.cpp:622-629
    } else {
        const int half = size >> 1;
        const float extent = static_cast<float>(half) * voxel * 1.7321f;  // compiler.cpp:633
        const int MC = N >> (L - 1);
#pragma unroll
        for (int o = 0; o < 8; ++o) {
            const float v = mnC[vidx(2 * bx + (o & 1), 2 * by + ((o >> 1) & 1), 2 * bz + ((o >> 2) & 1), MC)];
            if (!(v > extent)) m |= static_cast<uint8_t>(1u << o);  // compiler.cpp:646-649
        }
        if (m == 0)  // compiler.cpp:653-656: far leaf from the block minimum, semantic 0
            word = (1ull << 63) | static_cast<uint64_t>(gmdag::half_from_float_ref(lo));
    }
    canon[i] = word;
    mask[i] = m;
    nk[i] = static_cast<uint32_t>(__popc(m));
}

__global__ void scatter_children_kernel(const uint64_t* __restrict__ blocks, uint32_t n,
                                        const uint8_t* __restrict__ mask, const uint32_t* __restrict__ kid_off,
                                        uint64_t* __restrict__ child_blocks)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint8_t m = mask[i];
    if (!m) return;
    const uint64_t b = blocks[i];
    const uint32_t bx = static_cast<uint32_t>(b & 0x1FFFFF), by = static_cast<uint32_t>((b >> 21) & 0x1FFFFF),
                   bz = static_cast<uint32_t>(b >> 42);
    uint32_t j = kid_off[i];
    for (int o = 0; o < 8; ++o)
        if (m & (1u << o))
            child_blocks[j++] = pack_block(2 * bx + (o & 1), 2 * by + ((o >> 1) & 1), 2 * bz + ((o >> 2) & 1));
}

// Level 0: single voxels (compiler.cpp:585-597).
__global__ void voxel_leaf_kernel(const uint64_t* __restrict__ blocks, uint32_t n, int N,
                                  const float* __restrict__ grid, float voxel, uint64_t* __restrict__ canon,
                                  uint8_t* __restrict__ mask)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t b = blocks[i];
    const float d = grid[vidx(static_cast<int>(b & 0x1FFFFF), static_cast<int>((b >> 21) & 0x1FFFFF),
                              static_cast<int>(b >> 42), N)];
    canon[i] = gmdag::leaf_word(d, d < voxel * 2.0f ? 1 : 0);
    mask[i] = 0;
}

__device__ __forceinline__ uint64_t mix64(uint64_t h)
{
    // splitmix64 finaliser (S. Vigna)
    h ^= h >> 30;
    h *= 0xbf58476d1ce4e5b9ull;
    h ^= h >> 27;
    h *= 0x94d049bb133111ebull;
    h ^= h >> 31;
    return h;
}

__device__ __forceinline__ bool same_node(const LevelView& v, int La, uint32_t ia, int Lb, uint32_t ib, uint8_t m)
{
    if (v.mask[La][ia] != m) return false;
    const uint64_t* ca = v.canon[La - 1] + v.kid_off[La][ia];
    const uint64_t* cb = v.canon[Lb - 1] + v.kid_off[Lb][ib];
    const int n = __popc(m);
    for (int j = 0; j < n; ++j)
        if (ca[j] != cb[j]) return false;
    return true;
}

// Internal nodes of level L: structural identity = slot of the first inserted equal node.
__global__ void dedup_kernel(LevelView v, int L, uint32_t n, unsigned long long* __restrict__ table,
                             uint64_t cap_mask, uint64_t* __restrict__ canon, int* __restrict__ error)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint8_t m = v.mask[L][i];
    if (!m) return;
    const uint64_t* kids = v.canon[L - 1] + v.kid_off[L][i];
    const int nk = __popc(m);
    uint64_t h = mix64(m);
    for (int j = 0; j < nk; ++j) h = mix64(h ^ kids[j]);
    const unsigned long long me = (static_cast<unsigned long long>(L) << 40) | i;
    uint64_t slot = h & cap_mask;
    for (uint64_t probe = 0; probe <= cap_mask; ++probe) {
        unsigned long long owner = atomicCAS(table + slot, kEmpty, me);
        if (owner == kEmpty || owner == me) {
            canon[i] = slot;
            return;
        }
        const int Lo = static_cast<int>(owner >> 40);
        const uint32_t io = static_cast<uint32_t>(owner & 0xFFFFFFFFFFull);
        if (same_node(v, Lo, io, L, i, m)) {
            canon[i] = slot;
            return;
        }
        slot = (slot + 1) & cap_mask;
    }
    atomicExch(error, 1);  // table full: cannot happen with capacity > number of nodes
}

__global__ void used_kernel(const unsigned long long* __restrict__ table, uint64_t cap, uint32_t* __restrict__ used)
{
    for (uint64_t s = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; s < cap;
         s += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        used[s] = table[s] != kEmpty ? 1u : 0u;
}

__global__ void compact_count_kernel(const unsigned long long* __restrict__ table, uint64_t cap,
                                     const uint32_t* __restrict__ cidx, LevelView v, uint8_t* __restrict__ out_mask,
                                     uint32_t* __restrict__ out_n)
{
    for (uint64_t s = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; s < cap;
         s += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const unsigned long long o = table[s];
        if (o == kEmpty) continue;
        const int L = static_cast<int>(o >> 40);
        const uint32_t i = static_cast<uint32_t>(o & 0xFFFFFFFFFFull);
        const uint8_t m = v.mask[L][i];
        out_mask[cidx[s]] = m;
        out_n[cidx[s]] = static_cast<uint32_t>(__popc(m));
    }
}

__device__ __forceinline__ uint64_t remap(uint64_t c, const uint32_t* cidx)
{
    return (c >> 63) ? c : static_cast<uint64_t>(cidx[c]);
}

__global__ void compact_fill_kernel(const unsigned long long* __restrict__ table, uint64_t cap,
                                    const uint32_t* __restrict__ cidx, const uint32_t* __restrict__ out_off,
                                    LevelView v, uint64_t* __restrict__ out_kids)
{
    for (uint64_t s = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; s < cap;
         s += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const unsigned long long o = table[s];
        if (o == kEmpty) continue;
        const int L = static_cast<int>(o >> 40);
        const uint32_t i = static_cast<uint32_t>(o & 0xFFFFFFFFFFull);
        const int n = __popc(v.mask[L][i]);
        const uint64_t* kids = v.canon[L - 1] + v.kid_off[L][i];
        uint64_t* dst = out_kids + out_off[cidx[s]];
        for (int j = 0; j < n; ++j) dst[j] = remap(kids[j], cidx);
    }
}

unsigned blocks_for(size_t n, unsigned threads, unsigned cap = 148u * 64u)
{
    const size_t b = (n + threads - 1) / threads;
    return static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>(b, cap)));
}

template <class T>
void exclusive_scan(const T* in, T* out, size_t n, cudaStream_t st)
{
    size_t bytes = 0;
    CK(cub::DeviceScan::ExclusiveSum(nullptr, bytes, in, out, static_cast<int64_t>(n), st));
    DevBuf<unsigned char> tmp;
    tmp.alloc(bytes);
    CK(cub::DeviceScan::ExclusiveSum(tmp.p, bytes, in, out, static_cast<int64_t>(n), st));
}

template <class T>
T read_back(const T* dev, cudaStream_t st)
{
    T v;
    CK(cudaMemcpyAsync(&v, dev, sizeof(T), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return v;
}

// ------------------------------------------------------------------ host driver

// Puts the caller's current device back when an entry point returns (the compiler
// makes its own device current while it runs); declared before the compiler, so it
// is destroyed after the compiler's buffers are freed.
struct KeepCurrentDevice {
    int prev = -1;
    KeepCurrentDevice()
    {
        if (cudaGetDevice(&prev) != cudaSuccess) {
            cudaGetLastError();
            prev = -1;
        }
    }
    ~KeepCurrentDevice()
    {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

class DeviceCompiler {
public:
    DeviceCompiler(int N, int device) : N_(N), device_(device)
    {
        CK(cudaSetDevice(device));
        CK(cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking));
        levels_ = 0;
        while ((1 << levels_) < N_) ++levels_;
    }
    ~DeviceCompiler()
    {
        if (st_) cudaStreamDestroy(st_);
    }

    DevBuf<float> grid;

    void alloc_grid()
    {
        grid.alloc(static_cast<size_t>(N_) * N_ * N_);
        fill_kernel<<<blocks_for(grid.n, 256, 148u * 32u), 256, 0, st_>>>(grid.p, grid.n, kBig);
        CK(cudaGetLastError());
    }

    void upload_grid(const float* host)
    {
        grid.alloc(static_cast<size_t>(N_) * N_ * N_);
        CK(cudaMemcpyAsync(grid.p, host, grid.n * sizeof(float), cudaMemcpyHostToDevice, st_));
    }

    void seed(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri, const float* bmin,
              const gmdag::GridFrame& f)
    {
        std::vector<SeedItem> items;
        items.reserve(n_tri + 1024);
        for (uint64_t tr = 0; tr < n_tri; ++tr) {
            const float* v0 = &verts[static_cast<size_t>(idx[3 * tr]) * 3];
            const float* v1 = &verts[static_cast<size_t>(idx[3 * tr + 1]) * 3];
            const float* v2 = &verts[static_cast<size_t>(idx[3 * tr + 2]) * 3];
            const gmdag::VoxelBox b = gmdag::triangle_voxels(v0, v1, v2, bmin, f, N_);
            if (b.x1 < b.x0 || b.y1 < b.y0 || b.z1 < b.z0) continue;
            const uint32_t nx = b.x1 - b.x0 + 1, ny = b.y1 - b.y0 + 1, nz = b.z1 - b.z0 + 1;
            SeedItem it;
            it.tri = static_cast<uint32_t>(tr);
            it.x0 = static_cast<uint16_t>(b.x0);
            it.xn = static_cast<uint16_t>(nx);
            if (nx * ny <= kItemVoxels) {
                const uint32_t zstep = std::max<uint32_t>(1, kItemVoxels / (nx * ny));
                it.y0 = static_cast<uint16_t>(b.y0);
                it.yn = static_cast<uint16_t>(ny);
                for (uint32_t z = 0; z < nz; z += zstep) {
                    it.z0 = static_cast<uint16_t>(b.z0 + z);
                    it.zn = static_cast<uint16_t>(std::min(zstep, nz - z));
                    items.push_back(it);
                }
            } else {
                const uint32_t ystep = std::max<uint32_t>(1, kItemVoxels / nx);
                it.zn = 1;
                for (uint32_t z = 0; z < nz; ++z) {
                    it.z0 = static_cast<uint16_t>(b.z0 + z);
                    for (uint32_t y = 0; y < ny; y += ystep) {
                        it.y0 = static_cast<uint16_t>(b.y0 + y);
                        it.yn = static_cast<uint16_t>(std::min(ystep, ny - y));
                        items.push_back(it);
                    }
                }
            }
        }
        if (items.empty()) return;
        DevBuf<float> d_verts;
        DevBuf<uint32_t> d_idx;
        DevBuf<SeedItem> d_items;
        d_verts.alloc(3 * n_verts);
        d_idx.alloc(3 * n_tri);
        d_items.alloc(items.size());
        CK(cudaMemcpyAsync(d_verts.p, verts, 3 * n_verts * sizeof(float), cudaMemcpyHostToDevice, st_));
        CK(cudaMemcpyAsync(d_idx.p, idx, 3 * n_tri * sizeof(uint32_t), cudaMemcpyHostToDevice, st_));
        CK(cudaMemcpyAsync(d_items.p, items.data(), items.size() * sizeof(SeedItem), cudaMemcpyHostToDevice, st_));
        const uint32_t n_items = static_cast<uint32_t>(items.size());
        seed_kernel<<<std::min<uint32_t>(n_items, 1u << 20), 128, 0, st_>>>(
            grid.p, N_, d_verts.p, d_idx.p, d_items.p, n_items, bmin[0], bmin[1], bmin[2], f.dx, f.dy, f.dz);
        CK(cudaGetLastError());
        CK(cudaStreamSynchronize(st_));
    }

    void sweep(float h)
    {
        static const int kDirs[8][3] = {{1, 1, 1},  {-1, 1, 1},  {1, -1, 1},  {-1, -1, 1},
                                        {1, 1, -1}, {-1, 1, -1}, {1, -1, -1}, {-1, -1, -1}};
        const int NT = (N_ + kTile - 1) / kTile;
        for (int sw = 0; sw < 8; ++sw) {
            for (int k = 0; k <= 3 * (NT - 1); ++k) {
                const int z_first = std::max(0, k - 2 * (NT - 1));
                const int z_last = std::min(NT - 1, k);
                const dim3 grid_dim(static_cast<unsigned>(std::min(NT, k + 1)), static_cast<unsigned>(z_last - z_first + 1));
                sweep_kernel<<<grid_dim, kTile * kTile, 0, st_>>>(grid.p, N_, NT, k, kDirs[sw][0], kDirs[sw][1],
                                                                  kDirs[sw][2], h, z_first);
            }
            CK(cudaGetLastError());
        }
        CK(cudaStreamSynchronize(st_));
    }

    void pyramids()
    {
        mn_.resize(levels_ + 1);
        mx_.resize(levels_ + 1);
        for (int L = 1; L <= levels_; ++L) {
            const int M = N_ >> L;
            const size_t cnt = static_cast<size_t>(M) * M * M;
            mn_[L] = std::make_unique<DevBuf<float>>();
            mx_[L] = std::make_unique<DevBuf<float>>();
            mn_[L]->alloc(cnt);
            mx_[L]->alloc(cnt);
            const float* smn = L == 1 ? grid.p : mn_[L - 1]->p;
            const float* smx = L == 1 ? grid.p : mx_[L - 1]->p;
            pyramid_kernel<<<blocks_for(cnt, 256), 256, 0, st_>>>(smn, smx, mn_[L]->p, mx_[L]->p, M);
            CK(cudaGetLastError());
        }
        CK(cudaStreamSynchronize(st_));
    }

    // Visited blocks per level, dedup, compaction; returns the remapped root identity.
    uint64_t levels(float voxel, gmdag_gpu_timing& tm)
    {
        const int T = levels_;
        blocks_.resize(T + 1);
        canon_.resize(T + 1);
        mask_.resize(T + 1);
        kid_off_.resize(T + 1);
        count_.assign(T + 1, 0);
        for (int L = 0; L <= T; ++L) {
            blocks_[L] = std::make_unique<DevBuf<uint64_t>>();
            canon_[L] = std::make_unique<DevBuf<uint64_t>>();
            mask_[L] = std::make_unique<DevBuf<uint8_t>>();
            kid_off_[L] = std::make_unique<DevBuf<uint32_t>>();
        }
        // top-down: the root block, then the children of every internal block
        blocks_[T]->alloc(1);
        const uint64_t root_block = 0;
        CK(cudaMemcpyAsync(blocks_[T]->p, &root_block, sizeof root_block, cudaMemcpyHostToDevice, st_));
        count_[T] = 1;
        for (int L = T; L >= 1; --L) {
            const uint32_t n = count_[L];
            canon_[L]->alloc(n);
            mask_[L]->alloc(n);
            kid_off_[L]->alloc(n);
            DevBuf<uint32_t> nk;
            nk.alloc(n);
            if (n) {
                const float* mnC = (L == 1) ? grid.p : mn_[L - 1]->p;
                classify_kernel<<<(n + 255) / 256, 256, 0, st_>>>(blocks_[L]->p, n, L, N_, grid.p, mn_[L]->p,
                                                                  mx_[L]->p, mnC, voxel, canon_[L]->p, mask_[L]->p,
                                                                  nk.p);
                CK(cudaGetLastError());
                exclusive_scan(nk.p, kid_off_[L]->p, n, st_);
                const uint32_t last_off = read_back(kid_off_[L]->p + (n - 1), st_);
                const uint32_t last_n = read_back(nk.p + (n - 1), st_);
                const uint64_t total = static_cast<uint64_t>(last_off) + last_n;
                if (total > 0xFFFFFFF0ull) throw std::bad_alloc();
                count_[L - 1] = static_cast<uint32_t>(total);
            }
            blocks_[L - 1]->alloc(count_[L - 1]);
            if (count_[L - 1])
                scatter_children_kernel<<<(n + 255) / 256, 256, 0, st_>>>(blocks_[L]->p, n, mask_[L]->p,
                                                                          kid_off_[L]->p, blocks_[L - 1]->p);
            CK(cudaGetLastError());
        }
        // level 0: voxel leaves
        canon_[0]->alloc(count_[0]);
        mask_[0]->alloc(count_[0]);
        kid_off_[0]->alloc(1);
        if (count_[0])
            voxel_leaf_kernel<<<(count_[0] + 255) / 256, 256, 0, st_>>>(blocks_[0]->p, count_[0], N_, grid.p, voxel,
                                                                       canon_[0]->p, mask_[0]->p);
        CK(cudaGetLastError());

        LevelView v{};
        uint64_t internal_bound = 0;
        for (int L = 0; L <= T; ++L) {
            v.canon[L] = canon_[L]->p;
            v.kid_off[L] = kid_off_[L]->p;
            v.mask[L] = mask_[L]->p;
            tm.visited_blocks += count_[L];
            if (L >= 1) internal_bound += count_[L];
        }
        // bottom-up: structural dedup of internal nodes, level by level
        uint64_t cap = 1024;
        while (cap < 2 * internal_bound) cap <<= 1;
        DevBuf<unsigned long long> table;
        table.alloc(cap);
        CK(cudaMemsetAsync(table.p, 0xFF, cap * sizeof(unsigned long long), st_));
        DevBuf<int> err;
        err.alloc(1);
        CK(cudaMemsetAsync(err.p, 0, sizeof(int), st_));
        for (int L = 1; L <= T; ++L) {
            if (!count_[L]) continue;
            dedup_kernel<<<(count_[L] + 255) / 256, 256, 0, st_>>>(v, L, count_[L], table.p, cap - 1, canon_[L]->p,
                                                                   err.p);
            CK(cudaGetLastError());
        }
        if (read_back(err.p, st_) != 0) throw CudaError{cudaErrorUnknown, "node table overflow"};

        // compaction of the used slots: dense ids, child lists with remapped identities
        DevBuf<uint32_t> used, cidx;
        used.alloc(cap);
        cidx.alloc(cap);
        used_kernel<<<blocks_for(cap, 256), 256, 0, st_>>>(table.p, cap, used.p);
        CK(cudaGetLastError());
        exclusive_scan(used.p, cidx.p, cap, st_);
        const uint64_t U = static_cast<uint64_t>(read_back(cidx.p + (cap - 1), st_)) + read_back(used.p + (cap - 1), st_);
        tm.unique_internal = U;
        uint64_t root = read_back(canon_[T]->p, st_);
        if (!(root >> 63) && T >= 1) root = read_back(cidx.p + root, st_);
        tm.levels_ms = 0;  // set by the caller
        u_mask_.assign(U, 0);
        u_off_.assign(U + 1, 0);
        u_kids_.clear();
        if (U) {
            DevBuf<uint8_t> cmask;
            DevBuf<uint32_t> cn, coff;
            cmask.alloc(U);
            cn.alloc(U);
            coff.alloc(U);
            compact_count_kernel<<<blocks_for(cap, 256), 256, 0, st_>>>(table.p, cap, cidx.p, v, cmask.p, cn.p);
            CK(cudaGetLastError());
            exclusive_scan(cn.p, coff.p, U, st_);
            const uint64_t K = static_cast<uint64_t>(read_back(coff.p + (U - 1), st_)) + read_back(cn.p + (U - 1), st_);
            DevBuf<uint64_t> ckids;
            ckids.alloc(K);
            compact_fill_kernel<<<blocks_for(cap, 256), 256, 0, st_>>>(table.p, cap, cidx.p, coff.p, v, ckids.p);
            CK(cudaGetLastError());
            u_kids_.resize(K);
            CK(cudaMemcpyAsync(u_mask_.data(), cmask.p, U, cudaMemcpyDeviceToHost, st_));
            CK(cudaMemcpyAsync(u_off_.data(), coff.p, U * sizeof(uint32_t), cudaMemcpyDeviceToHost, st_));
            CK(cudaMemcpyAsync(u_kids_.data(), ckids.p, K * sizeof(uint64_t), cudaMemcpyDeviceToHost, st_));
            CK(cudaStreamSynchronize(st_));
            u_off_[U] = static_cast<uint32_t>(K);
        }
        return root;
    }

    // Post-order emission (compiler.cpp:579-674 order): leaves and internal nodes at
    // their first occurrence, root copied to word 0.
    std::vector<uint64_t> emit(uint64_t root) const
    {
        std::vector<uint64_t> pool;
        pool.push_back(0);
        std::vector<uint32_t> leaf_at(1u << 17, 0xFFFFFFFFu);
        std::vector<uint64_t> leaf_other_words;
        std::vector<uint32_t> leaf_other_at;
        std::vector<uint32_t> memo(u_mask_.size(), 0xFFFFFFFFu);

        auto leaf = [&](uint64_t w) -> uint32_t {
            const uint64_t low = w & ~(1ull << 63);
            if (low < (1ull << 17)) {
                uint32_t& slot = leaf_at[low];
                if (slot == 0xFFFFFFFFu) {
                    slot = static_cast<uint32_t>(pool.size());
                    pool.push_back(w);
                }
                return slot;
            }
            for (size_t j = 0; j < leaf_other_words.size(); ++j)
                if (leaf_other_words[j] == w) return leaf_other_at[j];
            leaf_other_words.push_back(w);
            leaf_other_at.push_back(static_cast<uint32_t>(pool.size()));
            pool.push_back(w);
            return leaf_other_at.back();
        };

        // explicit stack: (node id, next child)
        struct Frame {
            uint64_t id;
            uint32_t next;
            uint32_t kids[8];
        };
        std::vector<Frame> stack;
        uint32_t result = 0;
        auto push = [&](uint64_t c) -> bool {  // true when the value is resolved into `result`
            if (c >> 63) {
                result = leaf(c);
                return true;
            }
            if (memo[c] != 0xFFFFFFFFu) {
                result = memo[c];
                return true;
            }
            Frame f;
            f.id = c;
            f.next = 0;
            stack.push_back(f);
            return false;
        };
        if (push(root)) {
            pool[0] = pool[result];
            return pool;
        }
        while (!stack.empty()) {
            Frame& f = stack.back();
            const uint32_t n = u_off_[f.id + 1] - u_off_[f.id];
            if (f.next < n) {
                const uint64_t c = u_kids_[u_off_[f.id] + f.next];
                if (push(c)) {
                    Frame& g = stack.back();
                    g.kids[g.next++] = result;
                }
                continue;
            }
            const uint32_t p = static_cast<uint32_t>(pool.size());
            pool.push_back((static_cast<uint64_t>(u_mask_[f.id]) << 55) | (p + 1));
            for (uint32_t j = 0; j < n; ++j) pool.push_back(f.kids[j]);
            memo[f.id] = p;
            result = p;
            stack.pop_back();
            if (!stack.empty()) {
                Frame& g = stack.back();
                g.kids[g.next++] = result;
            }
        }
        pool[0] = pool[result];
        return pool;
    }

    void download_grid(float* host)
    {
        CK(cudaMemcpyAsync(host, grid.p, grid.n * sizeof(float), cudaMemcpyDeviceToHost, st_));
        CK(cudaStreamSynchronize(st_));
    }

    void release_levels()
    {
        blocks_.clear();
        canon_.clear();
        mask_.clear();
        kid_off_.clear();
        mn_.clear();
        mx_.clear();
    }

    int levels_count() const { return levels_; }

private:
    int N_;
    int device_;
    int levels_ = 0;
    cudaStream_t st_ = nullptr;
    std::vector<std::unique_ptr<DevBuf<float>>> mn_, mx_;
    std::vector<std::unique_ptr<DevBuf<uint64_t>>> blocks_, canon_;
    std::vector<std::unique_ptr<DevBuf<uint8_t>>> mask_;
    std::vector<std::unique_ptr<DevBuf<uint32_t>>> kid_off_;
    std::vector<uint32_t> count_;
    std::vector<uint8_t> u_mask_;
    std::vector<uint32_t> u_off_;
    std::vector<uint64_t> u_kids_;
};

int fail(int code, const std::string& msg)
{
    g_err = msg;
    return code;
}

bool pow2(uint32_t n) { return n && !(n & (n - 1)); }

int check_mesh(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri)
{
    if (!verts || n_verts == 0 || !idx || n_tri == 0) return fail(-1, "mesh must contain at least one triangle");
    if (n_tri > 0xFFFFFFFFull) return fail(-1, "at most 2^32 - 1 triangles");
    for (uint64_t i = 0; i < 3 * n_tri; ++i)
        if (idx[i] >= n_verts) return fail(-1, "triangle index out of range");
    return 0;
}

// Runs the DAG stage on a compiler whose grid is filled; fills r->words and timings.
void dag_stage(DeviceCompiler& dc, float voxel, GpuResult* r)
{
    auto t0 = Clock::now();
    if (dc.levels_count() >= 1) dc.pyramids();
    r->timing.pyramid_ms = ms_since(t0);
    t0 = Clock::now();
    const uint64_t root = dc.levels(voxel, r->timing);
    r->timing.levels_ms = ms_since(t0);
    t0 = Clock::now();
    dc.release_levels();
    r->words = dc.emit(root);
    r->timing.emit_ms = ms_since(t0);
}

template <class F>
int guarded(F&& body)
{
    g_err.clear();
    try {
        return body();
    } catch (const CudaError& e) {
        return fail(-4, std::string(e.what) + ": " + cudaGetErrorString(e.e));
    } catch (const std::bad_alloc&) {
        return fail(-3, "out of host memory while compiling");
    }
}

}  // namespace

extern "C" {

const char* gmdag_gpu_last_error(void) { return g_err.c_str(); }

int gmdag_gpu_compile_mesh(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri,
                           uint32_t resolution, int device, void** out)
{
    g_err.clear();
    if (!out) return fail(-1, "out must not be null");
    *out = nullptr;
    if (int rc = check_mesh(verts, n_verts, idx, n_tri)) return rc;
    if (!pow2(resolution) || resolution > 4096) return fail(-1, "resolution must be a power of two in [1, 4096]");
    return guarded([&]() -> int {
        auto r = std::make_unique<GpuResult>();
        const int N = static_cast<int>(resolution);
        gmdag::mesh_bounds(verts, n_verts, resolution, r->bmin, r->bmax, &r->voxel);
        const gmdag::GridFrame f = gmdag::grid_frame(r->bmin, r->bmax, N);
        auto t0 = Clock::now();
        KeepCurrentDevice keep;
        DeviceCompiler dc(N, device);
        dc.alloc_grid();
        r->timing.upload_ms = ms_since(t0);
        t0 = Clock::now();
        dc.seed(verts, n_verts, idx, n_tri, r->bmin, f);
        r->timing.seed_ms = ms_since(t0);
        t0 = Clock::now();
        dc.sweep(f.h);
        r->timing.sweep_ms = ms_since(t0);
        dag_stage(dc, r->voxel, r.get());
        if (r->words.size() > 0xFFFFFFFFull) return fail(-2, "DAG exceeds 2^32 words");
        *out = r.release();
        return 0;
    });
}

int gmdag_gpu_compute_sdf(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri,
                          uint32_t resolution, int device, float* out_grid, float* bmin, float* bmax, float* voxel)
{
    g_err.clear();
    if (!out_grid || !bmin || !bmax || !voxel) return fail(-1, "invalid arguments");
    if (int rc = check_mesh(verts, n_verts, idx, n_tri)) return rc;
    if (resolution == 0 || resolution > 4096) return fail(-1, "resolution must be in [1, 4096]");
    return guarded([&]() -> int {
        const int N = static_cast<int>(resolution);
        gmdag::mesh_bounds(verts, n_verts, resolution, bmin, bmax, voxel);
        const gmdag::GridFrame f = gmdag::grid_frame(bmin, bmax, N);
        KeepCurrentDevice keep;
        DeviceCompiler dc(N, device);
        dc.alloc_grid();
        dc.seed(verts, n_verts, idx, n_tri, bmin, f);
        dc.sweep(f.h);
        dc.download_grid(out_grid);
        return 0;
    });
}

int gmdag_gpu_compile_grid(const float* grid, uint32_t resolution, float voxel, int device, void** out)
{
    g_err.clear();
    if (!grid || !out) return fail(-1, "invalid arguments");
    *out = nullptr;
    if (!pow2(resolution) || resolution > 4096) return fail(-1, "resolution must be a power of two in [1, 4096]");
    return guarded([&]() -> int {
        auto r = std::make_unique<GpuResult>();
        const int N = static_cast<int>(resolution);
        r->voxel = voxel;
        for (int a = 0; a < 3; ++a) r->bmax[a] = voxel * static_cast<float>(N);
        auto t0 = Clock::now();
        KeepCurrentDevice keep;
        DeviceCompiler dc(N, device);
        dc.upload_grid(grid);
        r->timing.upload_ms = ms_since(t0);
        dag_stage(dc, voxel, r.get());
        *out = r.release();
        return 0;
    });
}

uint64_t gmdag_gpu_result_num_words(const void* r) { return r ? static_cast<const GpuResult*>(r)->words.size() : 0; }

void gmdag_gpu_result_header(const void* r, float* bmin, float* bmax, float* voxel)
{
    const auto* c = static_cast<const GpuResult*>(r);
    for (int a = 0; a < 3; ++a) {
        bmin[a] = c->bmin[a];
        bmax[a] = c->bmax[a];
    }
    *voxel = c->voxel;
}

void gmdag_gpu_result_copy_words(const void* r, uint64_t* dst)
{
    const auto* c = static_cast<const GpuResult*>(r);
    std::memcpy(dst, c->words.data(), c->words.size() * sizeof(uint64_t));
}

void gmdag_gpu_result_timing(const void* r, gmdag_gpu_timing* out)
{
    if (r && out) *out = static_cast<const GpuResult*>(r)->timing;
}

void gmdag_gpu_result_free(void* r) { delete static_cast<GpuResult*>(r); }

}  // extern "C"
