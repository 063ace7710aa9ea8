/*
 * tsdf.h — C ABI of the B200 sphere tracer over .gmdag signed-distance DAGs.
 *
 * Library: navi_b200/_lib/libnavi_tsdf.so (sm_100a).  Every function returns
 * TSDF_OK (0) or a negative tsdf_status; the text of the last error on the
 * calling thread is returned by tsdf_last_error().  No function frees memory
 * it did not allocate.  Device pointers are plain CUDA device addresses;
 * `stream` is a cudaStream_t (NULL = legacy default stream).  All cast calls
 * are asynchronous on `stream` and never synchronise the host.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   projects/torch-sdf/cpp_src/bindings.cpp:43-110   cast_rays_forward
 *   projects/torch-sdf/cpp_src/kernel.cu:311-326     launch_sphere_trace_kernel
 *   projects/torch-sdf/cpp_src/kernel.cuh:7-11       compile-time constants
 *   projects/environment/src/navi_environment/backends/sdfdag_backend.py:1296-1312
 *                                                     yaw-rotated fan + origin broadcast
 *   projects/environment/src/navi_environment/backends/sdfdag_backend.py:1896-1900
 *                                                     DAG device upload
 */
#ifndef NAVI_B200_TSDF_H
#define NAVI_B200_TSDF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TSDF_ABI_VERSION 1

#if defined(__GNUC__)
#define TSDF_API __attribute__((visibility("default")))
#else
#define TSDF_API
#endif

typedef enum tsdf_status {
    TSDF_OK = 0,
    TSDF_ERR_INVALID = -1,     /* bad argument (null pointer, size, range) */
    TSDF_ERR_LAYOUT = -2,      /* DAG words that cannot be traversed */
    TSDF_ERR_CUDA = -3,        /* a CUDA runtime call failed */
    TSDF_ERR_NO_MEMORY = -4,   /* host or device allocation failed */
    TSDF_ERR_UNSUPPORTED = -5, /* device is not sm_100 */
    TSDF_ERR_NOT_FOUND = -6,   /* a file that does not exist */
    TSDF_ERR_FILE = -7         /* a file that cannot be read or is malformed */
} tsdf_status;

/* Reference constants (kernel.cuh:7-11, kernel.cu:9). */
#define TSDF_DEFAULT_HIT_EPSILON 0.01f
#define TSDF_OUTSIDE_DOMAIN_DISTANCE 1000.0f
#define TSDF_DIRECTION_NORM_EPSILON 1e-4f
#define TSDF_PREFIX_DEPTH 4

/* Opaque device node pool built from .gmdag words (one device). */
typedef struct tsdf_pool tsdf_pool;
/* Opaque device table of scenes (pools + bounds + hit epsilon) for fan casts. */
typedef struct tsdf_scenes tsdf_scenes;

typedef struct tsdf_pool_stats {
    uint64_t source_words;   /* words in the .gmdag payload */
    uint64_t records;        /* internal nodes reachable from word 0 (32-byte records) */
    uint64_t ext_leaves;     /* leaves with semantic >= 0x7FFF, stored out of line */
    uint64_t device_bytes;   /* bytes of device memory held by the pool */
    uint32_t root_slot;      /* encoded root (record 0, or a leaf) */
    uint32_t bfs_levels;     /* BFS levels of the record graph */
    int32_t device;          /* CUDA ordinal */
    int32_t reserved;
} tsdf_pool_stats;

/* Per-actor pose for fan casts: 32 bytes, 16-byte aligned.  cos/sin are
 * supplied by the caller (the reference computes them with torch.cos/sin on
 * the device, sdfdag_backend.py:1301-1302) so the directions match it bit
 * for bit. */
typedef struct tsdf_pose {
    float ox, oy, oz;
    float cos_yaw;
    float sin_yaw;
    float cos_pitch;
    float sin_pitch;
    int32_t scene;           /* index into the tsdf_scenes table */
} tsdf_pose;

TSDF_API int tsdf_version(void);
TSDF_API const char* tsdf_last_error(void);

/* Build a node pool on `device` from .gmdag words in host memory.  Replaces
 * the int64 DAG upload (sdfdag_backend.py:1896-1900); the words are re-packed
 * into 32-byte records (8 child slots, one per octant).  flags: reserved, 0. */
TSDF_API int tsdf_pool_create(const uint64_t* host_words, uint64_t n_words, int device, uint32_t flags,
                     tsdf_pool** out_pool);

/* Same, from words already in device memory (the dag_tensor argument of
 * torch_sdf.cast_rays).  Copies the words to the host on `stream` and waits
 * for that copy. */
TSDF_API int tsdf_pool_create_from_device(const uint64_t* device_words, uint64_t n_words, int device,
                                 uint32_t flags, void* stream, tsdf_pool** out_pool);

/* Same, from a .gmdag file: the file-to-device path of sdfdag_backend.py:1893-1905
 * (load_gmdag_asset, integration/voxel_dag.py:193-259, with its checks and texts;
 * validate != 0 adds the layout walk of :29-78) in one call.  bbox_min / bbox_max
 * (may be null) receive the box the reference derives: bmin from the header and
 * bmin + voxel_size * resolution formed in double, rounded to float. */
TSDF_API int tsdf_pool_create_from_file(const char* path, int validate, int device, uint32_t flags,
                                        tsdf_pool** out_pool, float* bbox_min, float* bbox_max);

/* On-disk cache of a re-packed pool (records, out-of-line leaves), so that a scene
 * loads without re-packing.  The file is this library's own format ("NPOL", version
 * 1); loading checks every slot against the record and leaf counts and recomputes
 * the record-graph height, so a damaged file is rejected, not traced. */
TSDF_API int tsdf_pool_save(const tsdf_pool* pool, const char* path);
TSDF_API int tsdf_pool_load(const char* path, int device, tsdf_pool** out_pool);

TSDF_API int tsdf_pool_destroy(tsdf_pool* pool);
TSDF_API int tsdf_pool_stats_get(const tsdf_pool* pool, tsdf_pool_stats* out);

/* Device bytes of scratch that tsdf_cast needs in `workspace` for n_rays rays; the
 * caller allocates it (16-byte aligned), on the device of the pool.  It holds the work
 * counter and the claim order: 256 + 512 + 5 * n_rays bytes, rounded up to 16. */
TSDF_API uint64_t tsdf_workspace_bytes(int64_t n_rays);

/* Explicit-ray cast: the semantics of sphere_trace_kernel (kernel.cu:203-309)
 * for rays [n_rays][3] origins / dirs (f32, device), writing distance (f32),
 * semantic (i32, 0 on miss) and, if out_steps is not NULL, the number of
 * march iterations (i32).  Replaces launch_sphere_trace_kernel
 * (kernel.cu:311-326) and the launch in cast_rays_forward (bindings.cpp:91-109).
 * hit_epsilon = TSDF_DEFAULT_HIT_EPSILON reproduces the reference exactly. */
TSDF_API int tsdf_cast(const tsdf_pool* pool, const float* origins, const float* dirs, int64_t n_rays,
              float* out_dist, int32_t* out_sem, int32_t* out_steps, int max_steps,
              float max_distance, const float bbox_min[3], const float bbox_max[3],
              float hit_epsilon, void* workspace, void* stream);

/* Scene table for fan casts: n pools with their bounds ([n][3] each, host)
 * and hit epsilons ([n], host). */
TSDF_API int tsdf_scenes_create(const tsdf_pool* const* pools, int n, const float* bbox_min,
                       const float* bbox_max, const float* hit_epsilon, tsdf_scenes** out);
TSDF_API int tsdf_scenes_destroy(tsdf_scenes* scenes);

/* Device bytes of workspace tsdf_cast_fan needs for n_actors x rays_per_actor rays
 * on `scenes`: the work counter and, for a table of one scene, the claim order (as
 * tsdf_workspace_bytes); for more than one scene the actor order by scene (4 bytes
 * per actor, rounded up to 16) and 1 KB of per-scene bounds and counters, and for
 * tables of up to 64 scenes (traced one launch per scene) each scene's claim order:
 * 32 KB of bucket counts plus 5 bytes per ray (rounded up to 16).  scenes = NULL
 * gives the largest of these. */
TSDF_API uint64_t tsdf_fan_workspace_bytes(const tsdf_scenes* scenes, int64_t n_actors,
                                           int64_t rays_per_actor);

/* Fused fan cast: ray (a, r) starts at pose a's origin with the local fan
 * direction fan_dirs[r] (device, [rays_per_actor][3] f32), pitched about the
 * local x axis when use_pitch != 0, then yaw-rotated as
 * sdfdag_backend.py:1303-1310 does, and is traced in scene poses[a].scene.
 * Outputs are [n_actors * rays_per_actor], actor-major.  workspace:
 * tsdf_fan_workspace_bytes(scenes, n_actors, rays_per_actor) bytes on the scenes' device.  Multi-scene
 * tables trace the actors grouped by scene (the outputs do not depend on the
 * order); an actor whose scene index is outside the table is not traced: its
 * rays get a NaN distance, semantic 0 and 0 steps. */
TSDF_API int tsdf_cast_fan(const tsdf_scenes* scenes, const tsdf_pose* poses, int64_t n_actors,
                  const float* fan_dirs, int64_t rays_per_actor, int use_pitch,
                  float* out_dist, int32_t* out_sem, int32_t* out_steps, int max_steps,
                  float max_distance, void* workspace, void* stream);

/* Observation settings of tsdf_cast_fan_observe (the reference's post-processing,
 * sdfdag_backend.py:366-473, and observation stack, :1518-1525). */
typedef struct tsdf_observe {
    int32_t azimuth_bins;        /* fan is azimuth-major: ray = az * elevation_bins + el */
    int32_t elevation_bins;
    float structure_band_min;    /* structure-band ratios are 0 unless max > min */
    float structure_band_max;
    float proximity_threshold;   /* proximity ratio is 0 unless > 0 */
    float* observation;          /* device [actors][3][az][el] f32: depth, semantic, valid */
    float* actor_stats;          /* device [actors][5] f32: min clamped distance, starvation,
                                    proximity, structure band, forward structure band */
} tsdf_observe;

/* Device bytes of workspace tsdf_cast_fan_observe needs (the same as
 * tsdf_fan_workspace_bytes). */
TSDF_API uint64_t tsdf_observe_workspace_bytes(const tsdf_scenes* scenes, int64_t n_actors,
                                               int64_t rays_per_actor);

/* tsdf_cast_fan plus the reference's post-processing, one pass over the cast's
 * outputs on `stream` right after it (one block per actor): distances are clamped to
 * [0, max_distance], depth = clamp(log1p(d) / log1p(max), 0, 1), valid = isfinite(d);
 * the observation tensor and the per-actor reductions
 * (_compute_observation_ratios_tensor, sdfdag_backend.py:366-405; min distance :459).
 * Replaces _postprocess_cast_outputs_tensor (sdfdag_backend.py:408-473) and the stack
 * at :1518-1525. */
TSDF_API int tsdf_cast_fan_observe(const tsdf_scenes* scenes, const tsdf_pose* poses, int64_t n_actors,
                                   const float* fan_dirs, int64_t rays_per_actor, int use_pitch,
                                   float* out_dist, int32_t* out_sem, int32_t* out_steps, int max_steps,
                                   float max_distance, const tsdf_observe* observe, void* workspace,
                                   void* stream);

/* Allocation-free variant of tsdf_cast (no counterpart in the reference): the
 * same cast with no workspace argument, for callers that cannot allocate device
 * memory while they run (a fixed-rate control loop must not stall in cudaMalloc;
 * a host may hand the library only buffers registered up front).  Its scratch is
 * a 256-byte static device array inside the library, held by every GPU that
 * loads it; its address is looked up by the first call on each device, which
 * must come before any stream capture.  All calls share that array: calls whose
 * kernels may overlap on the GPU race and must be ordered on one stream.  The
 * looked-up address is tied to the device's context: after cudaDeviceReset of
 * that device it is stale, and the entry point must not be called on it again.
 * Allocates nothing: no cudaMalloc, no cudaFree.  With no room for a claim order,
 * rays are claimed in index order.  Leaves the caller's current device as it was. */
TSDF_API int tsdf_cast_noalloc(const tsdf_pool* pool, const float* origins, const float* dirs,
                               int64_t n_rays, float* out_dist, int32_t* out_sem, int32_t* out_steps,
                               int max_steps, float max_distance, const float bbox_min[3],
                               const float bbox_max[3], float hit_epsilon, void* stream);

/* Tuning knobs (process-wide): "smem_records" (top records staged in shared
 * memory per block by the float-descent kernel, default 0: on sm_100 the L1 serves
 * them as fast; capped so the block keeps its register-limited occupancy; the grid
 * kernel always reads records through L1), "chunk" (rays a warp claims
 * at once; default 0 = per launch: 32 for the per-scene launches of scene tables
 * and for launches of 2^21 rays or more, else 16), "leaf_run" (leaf-cache steps a single-scene lane takes in
 * place after a step, default 1), "blocks_per_sm" (0 = occupancy maximum),
 * "descent" (0 = integer grid descent wherever the DAG allows it, 1 = float
 * descent only), "order" (single-scene claim order: 1 = rays that can travel
 * farthest inside the scene box are claimed first, the default; 0 = ray index
 * order), "per_scene" (scene tables of 2 to 64 scenes: 1 = one single-scene launch
 * per scene over the actors sorted by scene on the device, the default; 0 = one
 * multi-scene launch).  No knob changes results.  Returns the old value through
 * *old_value when not NULL. */
TSDF_API int tsdf_set_option(const char* key, int64_t value, int64_t* old_value);

#ifdef __cplusplus
}
#endif

#endif /* NAVI_B200_TSDF_H */
