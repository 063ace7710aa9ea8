// Float arithmetic of the scene compiler, shared by the host compiler
// (gmdag_compiler.cpp, g++ -ffp-contract=off) and the device compiler
// (gmdag_gpu.cu, nvcc -fmad=false, IEEE division and square root).
//
// Every expression keeps the evaluation order of the reference voxel-dag
// compiler (projects/voxel-dag/src/compiler.cpp) so that both builds give the
// reference's values bit for bit: no contraction to FMA, correctly rounded
// division and sqrtf, denormals kept.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>

#ifdef __CUDACC__
#define GMDAG_HD __host__ __device__ __forceinline__
#else
#define GMDAG_HD inline
#endif

namespace gmdag {

GMDAG_HD float min3(float a, float b, float c)
{
    // std::min({a, b, c}): keeps the first of equal values
    float m = a;
    if (b < m) m = b;
    if (c < m) m = c;
    return m;
}

GMDAG_HD float max3(float a, float b, float c)
{
    float m = a;
    if (m < b) m = b;
    if (m < c) m = c;
    return m;
}

// clamp of the edge parameter from b over a: 0 when b >= 0, 1 when -b >= a, else -b / a
GMDAG_HD float edge_param(float b, float a)
{
    if (b >= 0) return 0.0f;
    if (-b >= a) return 1.0f;
    return -b / a;
}

// compiler.cpp:342-422 — squared distance from p to triangle (v0, v1, v2), the
// region-based method of D. Eberly (Geometric Tools, "Distance Between Point and
// Triangle in 3D").
GMDAG_HD float point_triangle_dist_sq(float px, float py, float pz, const float* v0, const float* v1,
                                      const float* v2)
{
    const float dfx = px - v0[0], dfy = py - v0[1], dfz = pz - v0[2];
    const float e0x = v1[0] - v0[0], e0y = v1[1] - v0[1], e0z = v1[2] - v0[2];
    const float e1x = v2[0] - v0[0], e1y = v2[1] - v0[1], e1z = v2[2] - v0[2];
    const float a00 = e0x * e0x + e0y * e0y + e0z * e0z;
    const float a01 = e0x * e1x + e0y * e1y + e0z * e1z;
    const float a11 = e1x * e1x + e1y * e1y + e1z * e1z;
    const float b0 = -(dfx * e0x + dfy * e0y + dfz * e0z);
    const float b1 = -(dfx * e1x + dfy * e1y + dfz * e1z);
    const float det = fabsf(a00 * a11 - a01 * a01);
    float s = a01 * b1 - a11 * b0;
    float t = a01 * b0 - a00 * b1;

    if (s + t <= det) {
        if (s < 0) {
            if (t < 0) {
                if (b0 < 0) {
                    t = 0;
                    s = (-b0 >= a00) ? 1.0f : -b0 / a00;
                } else {
                    s = 0;
                    t = edge_param(b1, a11);
                }
            } else {
                s = 0;
                t = edge_param(b1, a11);
            }
        } else if (t < 0) {
            t = 0;
            s = edge_param(b0, a00);
        } else {
            const float inv = 1.0f / det;
            s *= inv;
            t *= inv;
        }
    } else {
        if (s < 0) {
            const float tmp0 = a01 + b0;
            const float tmp1 = a11 + b1;
            if (tmp1 > tmp0) {
                const float numer = tmp1 - tmp0;
                const float denom = a00 - 2.0f * a01 + a11;
                s = (numer >= denom) ? 1.0f : numer / denom;
                t = 1 - s;
            } else {
                s = 0;
                if (tmp1 >= 0) t = 0;
                else if (-b1 >= a11) t = 1;
                else t = -b1 / a11;
            }
        } else if (t < 0) {
            const float tmp0 = a01 + b1;
            const float tmp1 = a00 + b0;
            if (tmp1 > tmp0) {
                const float numer = tmp1 - tmp0;
                const float denom = a00 - 2.0f * a01 + a11;
                t = (numer >= denom) ? 1.0f : numer / denom;
                s = 1 - t;
            } else {
                t = 0;
                if (tmp1 >= 0) s = 0;
                else if (-b0 >= a00) s = 1;
                else s = -b0 / a00;
            }
        } else {
            const float numer = a11 + b1 - a01 - b0;
            if (numer <= 0) {
                s = 0;
                t = 1;
            } else {
                const float denom = a00 - 2.0f * a01 + a11;
                s = (numer >= denom) ? 1.0f : numer / denom;
                t = 1 - s;
            }
        }
    }
    const float rx = v0[0] + s * e0x + t * e1x - px;
    const float ry = v0[1] + s * e0y + t * e1y - py;
    const float rz = v0[2] + s * e0z + t * e1z - pz;
    return rx * rx + ry * ry + rz * rz;
}

// compiler.cpp:424-442 — Godunov upwind update from the three neighbours, sorted.
GMDAG_HD float eikonal_update(float a, float b, float c, float h)
{
    float tmp;
    if (a > b) { tmp = a; a = b; b = tmp; }
    if (b > c) { tmp = b; b = c; c = tmp; }
    if (a > b) { tmp = a; a = b; b = tmp; }
    float d = a + h;
    if (d <= b) return d;
    d = 0.5f * (a + b + sqrtf(2.0f * h * h - (a - b) * (a - b)));
    if (d <= c) return d;
    const float sum = a + b + c;
    const float sum_sq = a * a + b * b + c * c;
    const float disc = sum * sum - 3.0f * (sum_sq - h * h);
    if (disc >= 0.0f) return (sum + sqrtf(disc)) / 3.0f;
    return d;
}

// compiler.cpp:542-560.  Truncating float->half with an unsigned exponent: a biased
// exponent below 112 (|f| < 2^-15, zero included) wraps and encodes as infinity.
// The reference behaves this way and the DAG words must match it.
GMDAG_HD uint16_t half_from_float_ref(float f)
{
    uint32_t i;
    memcpy(&i, &f, sizeof i);
    const uint32_t s = (i >> 16) & 0x00008000u;
    const uint32_t e = ((i >> 23) & 0x000000ffu) - (127u - 15u);
    uint32_t m = i & 0x007fffffu;
    if (e == 0u) {  // the reference's `e <= 0` on an unsigned value
        m = (m | 0x00800000u) >> 1;
        return static_cast<uint16_t>(s | (m >> 13));
    }
    if (e == 0xffu - (127u - 15u)) {
        if (m == 0) return static_cast<uint16_t>(s | 0x7c00u);
        return static_cast<uint16_t>(s | 0x7c00u | (m >> 13) | 1u);
    }
    if (e > 30u) return static_cast<uint16_t>(s | 0x7c00u);
    return static_cast<uint16_t>(s | (e << 10) | (m >> 13));
}

// leaf word: bit 63, semantic in bits 16..31, half distance in bits 0..15 (docs/GMDAG.md)
GMDAG_HD uint64_t leaf_word(float dist, uint16_t semantic)
{
    return (1ull << 63) | (static_cast<uint64_t>(semantic) << 16) |
           static_cast<uint64_t>(half_from_float_ref(dist));
}

// compiler.cpp:600-613 — every voxel of a block within 1e-6f of its first voxel,
// tested on the block's min and max (rounded subtraction is monotone).
GMDAG_HD bool uniform_block(float lo, float hi, float first)
{
    return !(fabsf(hi - first) > 1e-6f) && !(fabsf(lo - first) > 1e-6f);
}

// compiler.cpp:313-329 — cubic bounds padded by 1 m on every side, voxel = edge / res.
inline void mesh_bounds(const float* verts, uint64_t n_verts, uint32_t res, float* bmin, float* bmax,
                        float* voxel)
{
    float lo[3] = {std::numeric_limits<float>::max(), std::numeric_limits<float>::max(),
                   std::numeric_limits<float>::max()};
    float hi[3] = {std::numeric_limits<float>::lowest(), std::numeric_limits<float>::lowest(),
                   std::numeric_limits<float>::lowest()};
    for (uint64_t v = 0; v < n_verts; ++v) {
        for (int a = 0; a < 3; ++a) {
            const float c = verts[3 * v + a];
            if (c < lo[a]) lo[a] = c;
            if (c > hi[a]) hi[a] = c;
        }
    }
    const float ext = max3(hi[0] - lo[0], hi[1] - lo[1], hi[2] - lo[2]);
    *voxel = (ext + 2.0f) / static_cast<float>(res);
    for (int a = 0; a < 3; ++a) {
        const float c = (hi[a] + lo[a]) / 2.0f;
        bmin[a] = c - (ext + 2.0f) / 2.0f;
        bmax[a] = c + (ext + 2.0f) / 2.0f;
    }
}

// compiler.cpp:446-451 — grid step per axis and the sweep spacing h.
struct GridFrame {
    float dx, dy, dz, h;
};

inline GridFrame grid_frame(const float* bmin, const float* bmax, int N)
{
    GridFrame f;
    f.dx = (bmax[0] - bmin[0]) / N;
    f.dy = (bmax[1] - bmin[1]) / N;
    f.dz = (bmax[2] - bmin[2]) / N;
    f.h = min3(f.dx, f.dy, f.dz);
    return f;
}

// compiler.cpp:458-471 — voxel range a triangle seeds: its bounds grown by h, cut to the grid.
struct VoxelBox {
    int x0, x1, y0, y1, z0, z1;
};

inline VoxelBox triangle_voxels(const float* v0, const float* v1, const float* v2, const float* bmin,
                                const GridFrame& f, int N)
{
    const float lo_x = min3(v0[0], v1[0], v2[0]) - f.h;
    const float hi_x = max3(v0[0], v1[0], v2[0]) + f.h;
    const float lo_y = min3(v0[1], v1[1], v2[1]) - f.h;
    const float hi_y = max3(v0[1], v1[1], v2[1]) + f.h;
    const float lo_z = min3(v0[2], v1[2], v2[2]) - f.h;
    const float hi_z = max3(v0[2], v1[2], v2[2]) + f.h;
    VoxelBox b;
    b.x0 = static_cast<int>((lo_x - bmin[0]) / f.dx);
    b.x1 = static_cast<int>((hi_x - bmin[0]) / f.dx);
    b.y0 = static_cast<int>((lo_y - bmin[1]) / f.dy);
    b.y1 = static_cast<int>((hi_y - bmin[1]) / f.dy);
    b.z0 = static_cast<int>((lo_z - bmin[2]) / f.dz);
    b.z1 = static_cast<int>((hi_z - bmin[2]) / f.dz);
    b.x0 = b.x0 > 0 ? b.x0 : 0;
    b.y0 = b.y0 > 0 ? b.y0 : 0;
    b.z0 = b.z0 > 0 ? b.z0 : 0;
    b.x1 = b.x1 < N - 1 ? b.x1 : N - 1;
    b.y1 = b.y1 < N - 1 ? b.y1 : N - 1;
    b.z1 = b.z1 < N - 1 ? b.z1 : N - 1;
    return b;
}

}  // namespace gmdag
