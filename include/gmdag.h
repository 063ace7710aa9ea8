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

/* ---------------------------------------------------------------- files and layout */

/* Replaces integration/voxel_dag.py:193-259 (load_gmdag_asset: header "<4sIIffffI",
 * version 1, payload, no trailing bytes) and :29-78 (_validate_gmdag_dag_layout, a
 * recursive Python walk; here an explicit stack in the same depth-first order, so the
 * first error reported is the reference's).  Messages, in gmdag_last_error(), are the
 * reference's texts. */
typedef enum gmdag_file_status {
    GMDAG_FILE_OK = 0,
    GMDAG_FILE_NOT_FOUND = 1,          /* "gmdag asset does not exist: ..." (FileNotFoundError) */
    GMDAG_FILE_SHORT_HEADER = 2,
    GMDAG_FILE_BAD_MAGIC = 3,
    GMDAG_FILE_BAD_VERSION = 4,
    GMDAG_FILE_BAD_RESOLUTION = 5,
    GMDAG_FILE_BAD_VOXEL = 6,
    GMDAG_FILE_BAD_NODE_COUNT = 7,
    GMDAG_FILE_BAD_BOUNDS = 8,
    GMDAG_FILE_SHORT_PAYLOAD = 9,
    GMDAG_FILE_TRAILING_BYTES = 10,
    GMDAG_FILE_IO_ERROR = 11,
    GMDAG_FILE_BUFFER_TOO_SMALL = 12,
    GMDAG_FILE_BAD_LAYOUT = 13
} gmdag_file_status;

typedef enum gmdag_layout_kind {
    GMDAG_LAYOUT_OK = 0,
    GMDAG_LAYOUT_NODE_OUT_OF_RANGE = 1,
    GMDAG_LAYOUT_CYCLE = 2,
    GMDAG_LAYOUT_EMPTY_MASK = 3,
    GMDAG_LAYOUT_TABLE_BEYOND_PAYLOAD = 4,
    GMDAG_LAYOUT_TABLE_EXCEEDS_PAYLOAD = 5,
    GMDAG_LAYOUT_CHILD_OUT_OF_RANGE = 6
} gmdag_layout_kind;

typedef struct gmdag_file_info {
    char magic[4];
    uint32_t version;
    uint32_t resolution;
    float bbox_min[3];
    float voxel_size;
    uint32_t node_count;
    uint64_t nodes_found;     /* whole payload words present, at most node_count */
    uint64_t trailing_bytes;  /* bytes after node_count words */
} gmdag_file_info;

typedef struct gmdag_layout_error {
    int32_t kind;             /* gmdag_layout_kind */
    uint32_t reserved;
    uint64_t node;            /* node the message names */
    uint64_t value;           /* child table index or child reference, where the message quotes one */
} gmdag_layout_error;

/* dst == NULL: header and size checks only (info filled as far as parsed).  Otherwise
 * dst_words >= node_count and the payload is read into dst; validate != 0 also walks
 * the layout (GMDAG_FILE_BAD_LAYOUT, *layout filled).  Returns a gmdag_file_status. */
GMDAG_API int gmdag_file_read(const char* path, uint64_t* dst, uint64_t dst_words, int validate,
                              gmdag_file_info* info, gmdag_layout_error* layout);

/* 0: valid; 1: invalid (*err filled, message in gmdag_last_error()); -1: bad arguments. */
GMDAG_API int gmdag_validate_layout(const uint64_t* nodes, uint64_t n_nodes, gmdag_layout_error* err);

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
