/*
 * Scene compiler C ABI: triangle mesh -> dense unsigned SDF -> .gmdag DAG words.
 *
 * Two builds of the same algorithm, with the same output words:
 *   libnavi_gmdag.so      host compiler (OpenMP), gmdag_*
 *   libnavi_gmdag_gpu.so  device compiler (one B200), gmdag_gpu_*
 *
 * Reference interfaces replaced (projects/voxel-dag/):
 *   src/compiler.hpp:37-41   voxeldag::Compiler::compile(input_path, output_path)
 *                            (mesh -> .gmdag; here the mesh arrives as arrays: the
 *                            Assimp import of compiler.cpp:260-311 stays with the caller)
 *   src/compiler.cpp:444-536 Compiler::computeSDF      -> gmdag_compute_sdf / gmdag_gpu_compute_sdf
 *   src/compiler.cpp:661-678 Compiler::compressToDAG   -> gmdag_compile_grid / gmdag_gpu_compile_grid
 *   src/compiler.cpp:542-560 Compiler::float_to_half   -> gmdag_half_from_float
 *
 * Results are opaque handles read with *_result_* and released with
 * *_result_free.  Every int-returning call returns 0 on success or a negative
 * code, with the message in *_last_error() (thread-local).
 */
#ifndef NAVI_GMDAG_H
#define NAVI_GMDAG_H

#include <stdint.h>

#if defined(__GNUC__)
#define GMDAG_API __attribute__((visibility("default")))
#else
#define GMDAG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- host compiler */

GMDAG_API const char* gmdag_last_error(void);

/* verts: [n_verts][3] f32; idx: [n_tri][3] u32; resolution in [1, 4096];
 * n_threads <= 0: all OpenMP threads. */
GMDAG_API int gmdag_compile_mesh(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri,
                                 uint32_t resolution, int n_threads, void** out);

/* The SDF stage alone: out_grid [res][res][res] (z, y, x) f32, resolution <= 1024. */
GMDAG_API int gmdag_compute_sdf(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri,
                                uint32_t resolution, int n_threads, float* out_grid, float* bmin, float* bmax,
                                float* voxel);

/* The DAG stage alone, from a dense grid [res][res][res] (z, y, x). */
GMDAG_API int gmdag_compile_grid(const float* grid, uint32_t resolution, float voxel, int n_threads, void** out);

GMDAG_API uint64_t gmdag_result_num_words(const void* result);
GMDAG_API void gmdag_result_header(const void* result, float* bmin, float* bmax, float* voxel);
GMDAG_API void gmdag_result_copy_words(const void* result, uint64_t* dst);
GMDAG_API void gmdag_result_free(void* result);
GMDAG_API uint16_t gmdag_half_from_float(float f);

/* ---------------------------------------------------------------- device compiler */

/* Stage times of a device compile, milliseconds (host wall clock around each stage). */
typedef struct gmdag_gpu_timing {
    double upload_ms;   /* mesh upload, grid fill */
    double seed_ms;     /* exact triangle distances near the surface */
    double sweep_ms;    /* 8 fast-sweeping passes */
    double pyramid_ms;  /* min/max pyramids */
    double levels_ms;   /* visited blocks, level by level, and node dedup */
    double emit_ms;     /* download of the unique nodes and the post-order word emission */
    uint64_t visited_blocks;
    uint64_t unique_internal;
} gmdag_gpu_timing;

GMDAG_API const char* gmdag_gpu_last_error(void);

/* Power-of-two resolution in [1, 4096]; device: CUDA ordinal.  Blocks the calling
 * thread until the words are on the host. */
GMDAG_API int gmdag_gpu_compile_mesh(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri,
                                     uint32_t resolution, int device, void** out);

/* The SDF stage alone on the device, copied to out_grid (host, [res]^3 f32). */
GMDAG_API int gmdag_gpu_compute_sdf(const float* verts, uint64_t n_verts, const uint32_t* idx, uint64_t n_tri,
                                    uint32_t resolution, int device, float* out_grid, float* bmin, float* bmax,
                                    float* voxel);

/* The DAG stage alone, from a host grid [res]^3 (z, y, x), power-of-two resolution. */
GMDAG_API int gmdag_gpu_compile_grid(const float* grid, uint32_t resolution, float voxel, int device, void** out);

GMDAG_API uint64_t gmdag_gpu_result_num_words(const void* result);
GMDAG_API void gmdag_gpu_result_header(const void* result, float* bmin, float* bmax, float* voxel);
GMDAG_API void gmdag_gpu_result_copy_words(const void* result, uint64_t* dst);
GMDAG_API void gmdag_gpu_result_timing(const void* result, gmdag_gpu_timing* out);
GMDAG_API void gmdag_gpu_result_free(void* result);

#ifdef __cplusplus
}
#endif

#endif /* NAVI_GMDAG_H */
