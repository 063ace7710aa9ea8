// Scene compiler: triangle mesh -> dense unsigned SDF -> octree DAG words (.gmdag payload).
//
// The output is defined by the reference voxel-dag compiler
// (projects/voxel-dag/src/compiler.cpp); every stage below follows the same
// arithmetic so that the words are identical for the same triangles:
//   bounds and voxel size          compiler.cpp:313-329
//   triangle seeding               compiler.cpp:453-490 (point-triangle distance :342-422,
//                                  the region-based method of D. Eberly, Geometric Tools)
//   8-direction fast sweeping      compiler.cpp:492-529 (Eikonal update :424-442)
//   DAG build, dedup, root copy    compiler.cpp:579-674 (half conversion :542-560)
//
// What is different is how the work is scheduled:
//   - seeding is split into z-slabs, one per thread (the update is a min, so the
//     result does not depend on the order);
//   - each sweep runs as a wavefront over (y, z) lines: a line depends only on its
//     predecessors in y and z, which belong to the previous anti-diagonal, so the
//     values are the ones the sequential z/y/x loop produces;
//   - block minima and the uniform-block test read min/max pyramids instead of
//     rescanning the block.  The uniform test |v - first| <= 1e-6f over a block
//     equals the same test on the block's min and max, because rounded
//     subtraction is monotone;
//   - node dedup compares whole nodes, as the reference does after its hash
//     lookup, so the node order (post-order DFS, octants 0..7) is the same.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "gmdag.h"
#include "gmdag_io.h"
#include "gmdag_math.h"
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

thread_local std::string g_err;

struct CompileResult {
    std::vector<uint64_t> words;
    float bmin[3];
    float bmax[3];
    float voxel;
    uint32_t resolution;
};

using gmdag::eikonal_update;
using gmdag::half_from_float_ref;
using gmdag::leaf_word;
using gmdag::mesh_bounds;
using gmdag::point_triangle_dist_sq;

int threads_or_default(int n_threads)
{
#ifdef _OPENMP
    return n_threads > 0 ? n_threads : omp_get_max_threads();
#else
    (void)n_threads;
    return 1;
#endif
}

// ---------------------------------------------------------------- SDF stage

void seed_triangles(std::vector<float>& grid, int N, const float* bmin, const gmdag::GridFrame& frame,
                    const float* verts, const uint32_t* idx, uint64_t n_tri, int n_threads)
{
    const int T = threads_or_default(n_threads);
#ifdef _OPENMP
#pragma omp parallel num_threads(T)
#endif
    {
#ifdef _OPENMP
        const int tid = omp_get_thread_num();
        const int nth = omp_get_num_threads();
#else
        const int tid = 0, nth = 1;
#endif
        const int z_lo = static_cast<int>(static_cast<int64_t>(N) * tid / nth);
        const int z_hi = static_cast<int>(static_cast<int64_t>(N) * (tid + 1) / nth) - 1;
        for (uint64_t tr = 0; tr < n_tri; ++tr) {
            const float* v0 = &verts[static_cast<size_t>(idx[3 * tr]) * 3];
            const float* v1 = &verts[static_cast<size_t>(idx[3 * tr + 1]) * 3];
            const float* v2 = &verts[static_cast<size_t>(idx[3 * tr + 2]) * 3];
            const gmdag::VoxelBox vb = gmdag::triangle_voxels(v0, v1, v2, bmin, frame, N);
            const int x0 = vb.x0, x1 = vb.x1, y0 = vb.y0, y1 = vb.y1;
            int zs = vb.z0, ze = vb.z1;
            zs = std::max(zs, z_lo);
            ze = std::min(ze, z_hi);
            for (int z = zs; z <= ze; ++z) {
                const float pz = bmin[2] + z * frame.dz;
                for (int y = y0; y <= y1; ++y) {
                    const float py = bmin[1] + y * frame.dy;
                    float* row = &grid[(static_cast<size_t>(z) * N + y) * N];
                    for (int x = x0; x <= x1; ++x) {
                        const float px = bmin[0] + x * frame.dx;
                        const float d = std::sqrt(point_triangle_dist_sq(px, py, pz, v0, v1, v2));
                        if (d < row[x]) row[x] = d;
                    }
                }
            }
        }
    }
}

void fast_sweep(std::vector<float>& grid, int N, float h, int n_threads)
{
    static const int kDirs[8][3] = {{1, 1, 1},  {-1, 1, 1},  {1, -1, 1},  {-1, -1, 1},
                                    {1, 1, -1}, {-1, 1, -1}, {1, -1, -1}, {-1, -1, -1}};
    const float kBig = std::numeric_limits<float>::max();
    const size_t NN = static_cast<size_t>(N) * N;
    const int T = threads_or_default(n_threads);
    for (int sw = 0; sw < 8; ++sw) {
        const int sx = kDirs[sw][0], sy = kDirs[sw][1], sz = kDirs[sw][2];
        // anti-diagonal j = y' + z' in sweep coordinates; lines on one diagonal are independent
        for (int j = 0; j <= 2 * (N - 1); ++j) {
            const int yp_lo = std::max(0, j - (N - 1));
            const int yp_hi = std::min(N - 1, j);
#ifdef _OPENMP
#pragma omp parallel for num_threads(T) schedule(static) if (yp_hi - yp_lo > 8)
#endif
            for (int yp = yp_lo; yp <= yp_hi; ++yp) {
                const int zp = j - yp;
                const int y = sy > 0 ? yp : N - 1 - yp;
                const int z = sz > 0 ? zp : N - 1 - zp;
                float* row = &grid[static_cast<size_t>(z) * NN + static_cast<size_t>(y) * N];
                const bool has_b = (y - sy >= 0 && y - sy < N);
                const bool has_c = (z - sz >= 0 && z - sz < N);
                const float* row_b = has_b ? row - static_cast<ptrdiff_t>(sy) * N : nullptr;
                const float* row_c = has_c ? row - static_cast<ptrdiff_t>(sz) * static_cast<ptrdiff_t>(NN) : nullptr;
                for (int xp = 0; xp < N; ++xp) {
                    const int x = sx > 0 ? xp : N - 1 - xp;
                    const float a = (x - sx >= 0 && x - sx < N) ? row[x - sx] : kBig;
                    const float b = has_b ? row_b[x] : kBig;
                    const float c = has_c ? row_c[x] : kBig;
                    const float u = eikonal_update(a, b, c, h);
                    if (u < row[x]) row[x] = u;
                }
            }
        }
    }
}

// ---------------------------------------------------------------- DAG stage

// min/max of aligned blocks of size 2^L, L = 1..log2(N); level 0 is the grid itself.
struct Pyramid {
    int N = 0;
    int levels = 0;
    std::vector<std::vector<float>> mn, mx;

    static bool is_pow2(int n) { return n > 0 && (n & (n - 1)) == 0; }

    void build(const std::vector<float>& grid, int n, int n_threads)
    {
        N = n;
        levels = 0;
        while ((1 << levels) < N) ++levels;
        mn.assign(levels + 1, {});
        mx.assign(levels + 1, {});
        const int T = threads_or_default(n_threads);
        for (int L = 1; L <= levels; ++L) {
            const int M = N >> L;
            const int P = N >> (L - 1);
            mn[L].resize(static_cast<size_t>(M) * M * M);
            mx[L].resize(static_cast<size_t>(M) * M * M);
            const float* smn = (L == 1) ? grid.data() : mn[L - 1].data();
            const float* smx = (L == 1) ? grid.data() : mx[L - 1].data();
            float* dmn = mn[L].data();
            float* dmx = mx[L].data();
#ifdef _OPENMP
#pragma omp parallel for num_threads(T) schedule(static)
#endif
            for (int z = 0; z < M; ++z) {
                for (int y = 0; y < M; ++y) {
                    for (int x = 0; x < M; ++x) {
                        float lo = std::numeric_limits<float>::infinity();
                        float hi = -std::numeric_limits<float>::infinity();
                        for (int k = 0; k < 8; ++k) {
                            const size_t s = (static_cast<size_t>(2 * z + ((k >> 2) & 1)) * P +
                                              (2 * y + ((k >> 1) & 1))) * P + (2 * x + (k & 1));
                            lo = std::min(lo, smn[s]);
                            hi = std::max(hi, smx[s]);
                        }
                        const size_t d = (static_cast<size_t>(z) * M + y) * M + x;
                        dmn[d] = lo;
                        dmx[d] = hi;
                    }
                }
            }
        }
    }
};

class DagBuilder {
public:
    DagBuilder(const std::vector<float>& grid, int N, float voxel, const Pyramid* pyr)
        : grid_(grid), N_(N), voxel_(voxel), pyr_(pyr)
    {
    }

    std::vector<uint64_t> run()
    {
        pool_.clear();
        pool_.push_back(0);  // compiler.cpp:663 — index 0 reserved for the root copy
        const uint32_t root = build(0, 0, 0, N_);
        pool_[0] = pool_[root];  // compiler.cpp:671
        return std::move(pool_);
    }

private:
    const std::vector<float>& grid_;
    const int N_;
    const float voxel_;
    const Pyramid* pyr_;
    std::vector<uint64_t> pool_;
    std::unordered_map<uint64_t, uint32_t> leaves_;
    // internal nodes: hash of (mask, children) -> candidate node indices
    std::unordered_map<uint64_t, std::vector<uint32_t>> internals_;

    float at(int x, int y, int z) const
    {
        return grid_[(static_cast<size_t>(z) * N_ + y) * N_ + x];
    }

    int level_of(int size) const
    {
        int L = 0;
        while ((1 << L) < size) ++L;
        return L;
    }

    // compiler.cpp:563-577 (min over the block, clipped to the grid)
    float block_min(int x, int y, int z, int size) const
    {
        if (pyr_ && (size & (size - 1)) == 0 && x % size == 0 && y % size == 0 &&
            z % size == 0 && x + size <= N_ && y + size <= N_ && z + size <= N_) {
            if (size == 1) return at(x, y, z);
            const int L = level_of(size);
            const int M = N_ >> L;
            return pyr_->mn[L][(static_cast<size_t>(z / size) * M + y / size) * M + x / size];
        }
        float m = std::numeric_limits<float>::max();
        for (int bz = z; bz < z + size && bz < N_; ++bz)
            for (int by = y; by < y + size && by < N_; ++by)
                for (int bx = x; bx < x + size && bx < N_; ++bx) m = std::min(m, at(bx, by, bz));
        return m;
    }

    // compiler.cpp:600-613: every voxel of the block within 1e-6f of the first one
    bool block_uniform(int x, int y, int z, int size, float first) const
    {
        if (pyr_ && (size & (size - 1)) == 0 && x % size == 0 && y % size == 0 &&
            z % size == 0 && x + size <= N_ && y + size <= N_ && z + size <= N_) {
            const int L = level_of(size);
            const int M = N_ >> L;
            const size_t k = (static_cast<size_t>(z / size) * M + y / size) * M + x / size;
            const float lo = pyr_->mn[L][k], hi = pyr_->mx[L][k];
            return gmdag::uniform_block(lo, hi, first);
        }
        for (int bz = z; bz < z + size && bz < N_; ++bz)
            for (int by = y; by < y + size && by < N_; ++by)
                for (int bx = x; bx < x + size && bx < N_; ++bx)
                    if (std::fabs(at(bx, by, bz) - first) > 1e-6f) return false;
        return true;
    }

    uint32_t add_leaf(uint64_t w)
    {
        auto it = leaves_.find(w);
        if (it != leaves_.end()) return it->second;
        const uint32_t p = static_cast<uint32_t>(pool_.size());
        pool_.push_back(w);
        leaves_.emplace(w, p);
        return p;
    }

    static uint64_t mix(uint64_t h, uint64_t v)
    {
        h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
        return h;
    }

    uint32_t add_internal(uint8_t mask, const uint32_t* kids, int n)
    {
        uint64_t h = mask;
        for (int i = 0; i < n; ++i) h = mix(h, kids[i]);
        auto& bucket = internals_[h];
        for (uint32_t cand : bucket) {
            const uint64_t w = pool_[cand];
            if (static_cast<uint8_t>((w >> 55) & 0xFF) != mask) continue;
            const uint32_t base = static_cast<uint32_t>(w & 0xFFFFFFFFu);
            bool same = true;
            for (int i = 0; i < n && same; ++i) same = (pool_[base + i] == kids[i]);
            if (same) return cand;
        }
        const uint32_t p = static_cast<uint32_t>(pool_.size());
        pool_.push_back(0);
        const uint32_t base = static_cast<uint32_t>(pool_.size());
        for (int i = 0; i < n; ++i) pool_.push_back(kids[i]);
        pool_[p] = (static_cast<uint64_t>(mask) << 55) | base;
        bucket.push_back(p);
        return p;
    }

    // compiler.cpp:579-659
    uint32_t build(int x, int y, int z, int size)
    {
        const float two_vox = voxel_ * 2.0f;
        if (size == 1) {
            const float d = at(x, y, z);
            return add_leaf(leaf_word(d, d < two_vox ? 1 : 0));
        }
        const float first = at(x, y, z);
        if (block_uniform(x, y, z, size, first)) {
            return add_leaf(leaf_word(first, first < two_vox ? 1 : 0));
        }
        const int half = size / 2;
        const float octant_extent = static_cast<float>(half) * voxel_ * 1.7321f;
        uint8_t mask = 0;
        uint32_t kids[8];
        int n = 0;
        for (int i = 0; i < 8; ++i) {
            const int ox = (i & 1) ? half : 0;
            const int oy = (i & 2) ? half : 0;
            const int oz = (i & 4) ? half : 0;
            if (block_min(x + ox, y + oy, z + oz, half) > octant_extent) continue;
            kids[n++] = build(x + ox, y + oy, z + oz, half);
            mask |= static_cast<uint8_t>(1u << i);
        }
        if (mask == 0) {
            const float m = block_min(x, y, z, size);
            return add_leaf((1ull << 63) | static_cast<uint64_t>(half_from_float_ref(m)));
        }
        return add_internal(mask, kids, n);
    }
};

}  // namespace

extern "C" {

const char* gmdag_last_error(void) { return g_err.c_str(); }

// Compile a triangle mesh.  verts: [n_verts][3] f32, idx: [n_tri][3] u32.
// On success *out receives an opaque result; read it with gmdag_result_* and
// release it with gmdag_result_free.  Returns 0 or a negative error code.
int gmdag_compile_mesh(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri,
                       uint32_t resolution, int n_threads, void** out)
{
    g_err.clear();
    if (!out) {
        g_err = "out must not be null";
        return -1;
    }
    *out = nullptr;
    if (!verts || n_verts == 0 || !idx || n_tri == 0) {
        g_err = "mesh must contain at least one triangle";
        return -1;
    }
    if (resolution == 0 || resolution > 4096) {
        g_err = "resolution must be in [1, 4096]";
        return -1;
    }
    for (uint64_t i = 0; i < 3 * n_tri; ++i) {
        if (idx[i] >= n_verts) {
            g_err = "triangle index out of range";
            return -1;
        }
    }
    try {
        auto res = std::make_unique<CompileResult>();
        res->resolution = resolution;
        mesh_bounds(verts, n_verts, resolution, res->bmin, res->bmax, &res->voxel);
        const int N = static_cast<int>(resolution);
        // compiler.cpp:446-451
        std::vector<float> grid(static_cast<size_t>(N) * N * N, std::numeric_limits<float>::max());
        const gmdag::GridFrame frame = gmdag::grid_frame(res->bmin, res->bmax, N);
        seed_triangles(grid, N, res->bmin, frame, verts, idx, n_tri, n_threads);
        fast_sweep(grid, N, frame.h, n_threads);
        Pyramid pyr;
        const bool use_pyr = Pyramid::is_pow2(N) && N > 1;
        if (use_pyr) pyr.build(grid, N, n_threads);
        DagBuilder b(grid, N, res->voxel, use_pyr ? &pyr : nullptr);
        res->words = b.run();
        if (res->words.size() > 0xFFFFFFFFull) {
            g_err = "DAG exceeds 2^32 words";
            return -2;
        }
        *out = res.release();
        return 0;
    } catch (const std::bad_alloc&) {
        g_err = "out of host memory while compiling";
        return -3;
    }
}

// Stage 2 only: dense unsigned SDF of a mesh on the compiler's grid, [res][res][res]
// (z, y, x) into out_grid, with the bounds of stage 1.
int gmdag_compute_sdf(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri,
                      uint32_t resolution, int n_threads, float* out_grid, float* bmin, float* bmax,
                      float* voxel)
{
    g_err.clear();
    if (!verts || !idx || !out_grid || n_verts == 0 || n_tri == 0 || resolution == 0 || resolution > 1024) {
        g_err = "invalid arguments";
        return -1;
    }
    for (uint64_t i = 0; i < 3 * n_tri; ++i)
        if (idx[i] >= n_verts) {
            g_err = "triangle index out of range";
            return -1;
        }
    const int N = static_cast<int>(resolution);
    mesh_bounds(verts, n_verts, resolution, bmin, bmax, voxel);
    std::vector<float> grid(static_cast<size_t>(N) * N * N, std::numeric_limits<float>::max());
    const gmdag::GridFrame frame = gmdag::grid_frame(bmin, bmax, N);
    seed_triangles(grid, N, bmin, frame, verts, idx, n_tri, n_threads);
    fast_sweep(grid, N, frame.h, n_threads);
    std::memcpy(out_grid, grid.data(), grid.size() * sizeof(float));
    return 0;
}

// Stage 3 only: DAG words of a dense grid [res][res][res] (z, y, x) with the given voxel size.
int gmdag_compile_grid(const float* grid_in, uint32_t resolution, float voxel, int n_threads, void** out)
{
    g_err.clear();
    if (!grid_in || !out || resolution == 0 || resolution > 4096) {
        g_err = "invalid arguments";
        return -1;
    }
    *out = nullptr;
    try {
        const int N = static_cast<int>(resolution);
        std::vector<float> grid(grid_in, grid_in + static_cast<size_t>(N) * N * N);
        auto res = std::make_unique<CompileResult>();
        res->resolution = resolution;
        res->voxel = voxel;
        for (int a = 0; a < 3; ++a) {
            res->bmin[a] = 0.0f;
            res->bmax[a] = voxel * static_cast<float>(N);
        }
        Pyramid pyr;
        const bool use_pyr = Pyramid::is_pow2(N) && N > 1;
        if (use_pyr) pyr.build(grid, N, n_threads);
        DagBuilder b(grid, N, voxel, use_pyr ? &pyr : nullptr);
        res->words = b.run();
        *out = res.release();
        return 0;
    } catch (const std::bad_alloc&) {
        g_err = "out of host memory while compiling";
        return -3;
    }
}

uint64_t gmdag_result_num_words(const void* r)
{
    return r ? static_cast<const CompileResult*>(r)->words.size() : 0;
}

void gmdag_result_header(const void* r, float* bmin, float* bmax, float* voxel)
{
    const auto* c = static_cast<const CompileResult*>(r);
    for (int a = 0; a < 3; ++a) {
        bmin[a] = c->bmin[a];
        bmax[a] = c->bmax[a];
    }
    *voxel = c->voxel;
}

void gmdag_result_copy_words(const void* r, uint64_t* dst)
{
    const auto* c = static_cast<const CompileResult*>(r);
    std::memcpy(dst, c->words.data(), c->words.size() * sizeof(uint64_t));
}

void gmdag_result_free(void* r) { delete static_cast<CompileResult*>(r); }

int gmdag_file_read(const char* path, uint64_t* dst, uint64_t dst_words, int validate, gmdag_file_info* info,
                    gmdag_layout_error* layout)
{
    g_err.clear();
    gmdag_file_info local{};
    gmdag_file_info& I = info ? *info : local;
    if (layout) *layout = gmdag_layout_error{};
    const int st = gmdag_io::read_file(path, dst, dst_words, &I);
    if (st != GMDAG_FILE_OK) {
        g_err = gmdag_io::message(path, st, I);
        return st;
    }
    if (dst && validate) {
        gmdag_layout_error e{};
        if (!gmdag_io::validate_layout(dst, I.node_count, &e)) {
            if (layout) *layout = e;
            g_err = gmdag_io::layout_message(e);
            return GMDAG_FILE_BAD_LAYOUT;
        }
    }
    return GMDAG_FILE_OK;
}

int gmdag_validate_layout(const uint64_t* nodes, uint64_t n_nodes, gmdag_layout_error* err)
{
    g_err.clear();
    if (!nodes && n_nodes) {
        g_err = "nodes must not be null";
        return -1;
    }
    gmdag_layout_error e{};
    const bool ok = gmdag_io::validate_layout(nodes, n_nodes, &e);
    if (err) *err = e;
    if (ok) return 0;
    g_err = gmdag_io::layout_message(e);
    return 1;
}

// The reference's float->half conversion, exposed for tests.
uint16_t gmdag_half_from_float(float f) { return half_from_float_ref(f); }

}  // extern "C"
