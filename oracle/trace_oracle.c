/*
 * CPU oracle for the batched sphere trace over a .gmdag DAG.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path may call this code:
 * it is the checker used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py.
 *
 * It restates the reference kernel step by step, in plain C:
 *   projects/torch-sdf/cpp_src/kernel.cuh:7-11   constants
 *   projects/torch-sdf/cpp_src/kernel.cu:11-31   point_in_bounds / _strict
 *   projects/torch-sdf/cpp_src/kernel.cu:33-52   load_dag_word, leaf decode
 *   projects/torch-sdf/cpp_src/kernel.cu:54-85   distance_to_bounds_exit
 *   projects/torch-sdf/cpp_src/kernel.cu:88-200  query_dag_stackless
 *   projects/torch-sdf/cpp_src/kernel.cu:203-309 sphere_trace_kernel
 *
 * Differences from the reference, all additive:
 *   - hit_epsilon is a parameter (the reference hard-codes 0.01f);
 *   - the number of loop iterations per ray is reported (steps);
 *   - the number of DAG word loads per ray is reported (the W_ref figure of
 *     the roofline accounting: every load_dag_word call, kernel.cu:137 and
 *     kernel.cu:198, including the ones the reference serves from its
 *     shared-memory prefix);
 *   - the position update o + t*d can be evaluated fused (one rounding) or
 *     unfused (two roundings); which one the reference build uses is pinned
 *     by comparing outputs, never by reading compiled code;
 *   - a node index outside the payload is reported as an error instead of
 *     being read (the reference reads such words unchecked).
 *
 * Build: oracle/build.py (gcc, -ffp-contract=off so that no other expression
 * is contracted; fmaf() is the C99 correctly rounded fused multiply-add).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_OUTSIDE_DOMAIN 1000.0f   /* kernel.cuh:8  kOutsideDomainDistance */
#define OR_DIR_EPS 1e-4f            /* kernel.cuh:9  kDirectionNormEpsilon */
#define OR_PREFIX_DEPTH 4           /* kernel.cuh:11 kTraversalCacheDepth */
#define OR_VOID_ADVANCE 1e-5f       /* kernel.cu:9   kVoidAdvanceEpsilon */
#define OR_MAX_DEPTH 32             /* kernel.cu:136 descent cap */

/* IEEE binary16 -> binary32, exact by definition (the reference uses
 * __half2float, kernel.cu:43-47, which is exact for every input). */
static float half_bits_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* subnormal half: value = man * 2^-24, normalise */
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

float oracle_half_to_float(uint16_t h) { return half_bits_to_float(h); }

static int in_closed(float px, float py, float pz, const float *mn, const float *mx)
{
    return px >= mn[0] && px <= mx[0] && py >= mn[1] && py <= mx[1] &&
           pz >= mn[2] && pz <= mx[2];
}

static int in_open(float px, float py, float pz, const float *mn, const float *mx)
{
    return px > mn[0] && px < mx[0] && py > mn[1] && py < mx[1] &&
           pz > mn[2] && pz < mx[2];
}

/* kernel.cu:54-85 */
static float exit_distance(float px, float py, float pz, float dx, float dy, float dz,
                           const float *mn, const float *mx)
{
    float t = OR_OUTSIDE_DOMAIN;
    if (dx > OR_DIR_EPS) t = fminf(t, (mx[0] - px) / dx);
    else if (dx < -OR_DIR_EPS) t = fminf(t, (mn[0] - px) / dx);
    if (dy > OR_DIR_EPS) t = fminf(t, (mx[1] - py) / dy);
    else if (dy < -OR_DIR_EPS) t = fminf(t, (mn[1] - py) / dy);
    if (dz > OR_DIR_EPS) t = fminf(t, (mx[2] - pz) / dz);
    else if (dz < -OR_DIR_EPS) t = fminf(t, (mn[2] - pz) / dz);
    return fmaxf(t, OR_VOID_ADVANCE);
}

typedef struct {
    /* prefix (depth-4) cache, kernel.cu:120-132, :154-163 */
    uint32_t pre_ptr;
    float pre_mn[3], pre_mx[3];
    int pre_valid;
    /* void cache, kernel.cu:178-190, :265 */
    float void_mn[3], void_mx[3];
    int void_valid;
    /* leaf cache, kernel.cu:114-118, :139-152 */
    float leaf_mn[3], leaf_mx[3];
    float leaf_dist;
    int32_t leaf_sem;
    int leaf_valid;
} ray_caches;

typedef struct {
    const uint64_t *dag;
    uint64_t n;
    float mn[3], mx[3];
} dag_view;

/* kernel.cu:33-39 (the shared-memory copy holds the same words) */
static int load_word(const dag_view *v, uint32_t ptr, uint64_t *out, int64_t *loads)
{
    (*loads)++;
    if ((uint64_t)ptr >= v->n) return -1;
    *out = v->dag[ptr];
    return 0;
}

/* Step mix (optional, oracle_trace_mix): what each march step of the reference did. */
enum { MIX_STEPS, MIX_VOID_CACHE, MIX_OUTSIDE, MIX_LEAF_CACHE, MIX_DESCENTS, MIX_DESC_LEAF, MIX_DESC_VOID,
       MIX_LEVELS, MIX_N };

/* kernel.cu:88-200.  Returns 0, or -1 on an index outside the payload. */
static int query(const dag_view *v, float px, float py, float pz, float dx, float dy, float dz,
                 ray_caches *c, float *out_dist, int32_t *out_sem, int64_t *loads, int64_t *mix)
{
    if (!in_closed(px, py, pz, v->mn, v->mx)) {
        if (mix) mix[MIX_OUTSIDE]++;
        *out_dist = OR_OUTSIDE_DOMAIN;
        *out_sem = 0;
        return 0;
    }
    if (c->leaf_valid && in_closed(px, py, pz, c->leaf_mn, c->leaf_mx)) {
        if (mix) mix[MIX_LEAF_CACHE]++;
        *out_dist = c->leaf_dist;
        *out_sem = c->leaf_sem;
        return 0;
    }
    if (mix) mix[MIX_DESCENTS]++;
    const int use_prefix = c->pre_valid && in_closed(px, py, pz, c->pre_mn, c->pre_mx);
    uint32_t ptr = use_prefix ? c->pre_ptr : 0u;
    float mn[3], mx[3];
    for (int a = 0; a < 3; ++a) {
        mn[a] = use_prefix ? c->pre_mn[a] : v->mn[a];
        mx[a] = use_prefix ? c->pre_mx[a] : v->mx[a];
    }
    int depth = use_prefix ? OR_PREFIX_DEPTH : 0;
    for (; depth < OR_MAX_DEPTH; ++depth) {
        uint64_t node;
        if (mix) mix[MIX_LEVELS]++;
        if (load_word(v, ptr, &node, loads)) return -1;
        if ((node >> 63) == 1) {
            if (mix) mix[MIX_DESC_LEAF]++;
            for (int a = 0; a < 3; ++a) {
                c->leaf_mn[a] = mn[a];
                c->leaf_mx[a] = mx[a];
            }
            c->leaf_dist = half_bits_to_float((uint16_t)(node & 0xFFFFu));
            c->leaf_sem = (int32_t)((node >> 16) & 0xFFFFu);
            c->leaf_valid = 1;
            *out_dist = c->leaf_dist;
            *out_sem = c->leaf_sem;
            return 0;
        }
        if (!use_prefix && depth == OR_PREFIX_DEPTH) {
            c->pre_ptr = ptr;
            for (int a = 0; a < 3; ++a) {
                c->pre_mn[a] = mn[a];
                c->pre_mx[a] = mx[a];
            }
            c->pre_valid = 1;
        }
        const float mxm = (mn[0] + mx[0]) * 0.5f;
        const float mym = (mn[1] + mx[1]) * 0.5f;
        const float mzm = (mn[2] + mx[2]) * 0.5f;
        const int oct = (px >= mxm ? 1 : 0) | (py >= mym ? 2 : 0) | (pz >= mzm ? 4 : 0);
        if (px >= mxm) mn[0] = mxm; else mx[0] = mxm;
        if (py >= mym) mn[1] = mym; else mx[1] = mym;
        if (pz >= mzm) mn[2] = mzm; else mx[2] = mzm;
        const uint32_t mask = (uint32_t)((node >> 55) & 0xFFu);
        if ((mask & (1u << oct)) == 0) {
            for (int a = 0; a < 3; ++a) {
                c->void_mn[a] = mn[a];
                c->void_mx[a] = mx[a];
            }
            c->void_valid = 1;
            if (mix) mix[MIX_DESC_VOID]++;
            *out_dist = exit_distance(px, py, pz, dx, dy, dz, c->void_mn, c->void_mx);
            *out_sem = 0;
            return 0;
        }
        const uint32_t base = (uint32_t)(node & 0xFFFFFFFFu);
        const uint32_t off = (uint32_t)__builtin_popcount(mask & ((1u << oct) - 1u));
        uint64_t child;
        if (load_word(v, base + off, &child, loads)) return -1;
        ptr = (uint32_t)child;
    }
    /* descent cap reached without a leaf or void octant: outputs unchanged */
    return 0;
}

typedef struct {
    float t;
    int32_t sem;
    int32_t steps;
    int64_t loads;
    int err;
} ray_result;

/* kernel.cu:203-309 for one ray */
static ray_result trace_one(const dag_view *v, float ox, float oy, float oz, float dx, float dy,
                            float dz, int max_steps, float max_distance, float hit_eps,
                            int use_fma, int64_t *mix)
{
    ray_result r = {0.0f, 0, 0, 0, 0};
    ray_caches c;
    memset(&c, 0, sizeof c);
    float t = 0.0f;
    float dist = 0.0f;
    int32_t sem = 0;
    int step = 0;
    for (step = 0; step < max_steps; ++step) {
        float px, py, pz;
        if (use_fma) {
            px = fmaf(t, dx, ox);
            py = fmaf(t, dy, oy);
            pz = fmaf(t, dz, oz);
        } else {
            px = ox + t * dx;
            py = oy + t * dy;
            pz = oz + t * dz;
        }
        if (mix) mix[MIX_STEPS]++;
        if (c.void_valid && in_open(px, py, pz, c.void_mn, c.void_mx)) {
            if (mix) mix[MIX_VOID_CACHE]++;
            dist = exit_distance(px, py, pz, dx, dy, dz, c.void_mn, c.void_mx);
            sem = 0;
        } else if (query(v, px, py, pz, dx, dy, dz, &c, &dist, &sem, &r.loads, mix)) {
            r.err = 1;
            return r;
        }
        if (sem != 0 && dist < hit_eps) {
            r.t = t;
            r.sem = sem;
            r.steps = step + 1;
            return r;
        }
        t += dist;
        if (t > max_distance) {
            r.t = t;
            r.sem = 0;
            r.steps = step + 1;
            return r;
        }
    }
    r.t = t;
    r.sem = 0;
    r.steps = max_steps;
    return r;
}

/*
 * Trace n_rays rays given as [n_rays][3] origins and directions.
 * out_steps and out_loads may be NULL.  Returns 0, or the negative
 * (1-based) index of the first ray that met an index outside the payload.
 */
int64_t oracle_trace(const uint64_t *dag, uint64_t n_words, const float *bmin, const float *bmax,
                     const float *origins, const float *dirs, int64_t n_rays, int max_steps,
                     float max_distance, float hit_eps, int use_fma, int n_threads,
                     float *out_dist, int32_t *out_sem, int32_t *out_steps, int64_t *out_loads)
{
    dag_view v;
    v.dag = dag;
    v.n = n_words;
    for (int a = 0; a < 3; ++a) {
        v.mn[a] = bmin[a];
        v.mx[a] = bmax[a];
    }
    int64_t first_err = 0;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel for schedule(dynamic, 64)
#endif
    for (int64_t i = 0; i < n_rays; ++i) {
        const float *o = origins + 3 * i;
        const float *d = dirs + 3 * i;
        ray_result r = trace_one(&v, o[0], o[1], o[2], d[0], d[1], d[2], max_steps, max_distance,
                                 hit_eps, use_fma, NULL);
        out_dist[i] = r.t;
        out_sem[i] = r.sem;
        if (out_steps) out_steps[i] = r.steps;
        if (out_loads) out_loads[i] = r.loads;
        if (r.err) {
#ifdef _OPENMP
#pragma omp critical
#endif
            if (first_err == 0 || -(i + 1) > first_err) first_err = -(i + 1);
        }
    }
    return first_err;
}

/*
 * Step mix of the reference algorithm over n_rays rays: mix[8] receives the number of
 * march steps, void-cache hits (kernel.cu:265), steps outside the box (:108), leaf-cache
 * hits (:114), descents, descents ending in a leaf (:139) and in an empty octant (:178),
 * and descent levels (node words loaded at :137).  Returns 0 or the negative index of
 * the first ray that met an index outside the payload.
 */
int64_t oracle_trace_mix(const uint64_t *dag, uint64_t n_words, const float *bmin, const float *bmax,
                         const float *origins, const float *dirs, int64_t n_rays, int max_steps,
                         float max_distance, float hit_eps, int n_threads, int64_t *mix)
{
    dag_view v;
    v.dag = dag;
    v.n = n_words;
    for (int a = 0; a < 3; ++a) {
        v.mn[a] = bmin[a];
        v.mx[a] = bmax[a];
    }
    for (int k = 0; k < MIX_N; ++k) mix[k] = 0;
    int64_t first_err = 0;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel
#endif
    {
        int64_t local[MIX_N] = {0};
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 64)
#endif
        for (int64_t i = 0; i < n_rays; ++i) {
            const float *o = origins + 3 * i;
            const float *d = dirs + 3 * i;
            ray_result r = trace_one(&v, o[0], o[1], o[2], d[0], d[1], d[2], max_steps, max_distance, hit_eps, 1,
                                     local);
            if (r.err) {
#ifdef _OPENMP
#pragma omp critical
#endif
                if (first_err == 0 || -(i + 1) > first_err) first_err = -(i + 1);
            }
        }
#ifdef _OPENMP
#pragma omp critical
#endif
        for (int k = 0; k < MIX_N; ++k) mix[k] += local[k];
    }
    return first_err;
}

/* Point query with fresh caches (one call of query_dag_stackless). */
int oracle_point_query(const uint64_t *dag, uint64_t n_words, const float *bmin,
                       const float *bmax, float px, float py, float pz, float *out_dist,
                       int32_t *out_sem)
{
    dag_view v;
    v.dag = dag;
    v.n = n_words;
    for (int a = 0; a < 3; ++a) {
        v.mn[a] = bmin[a];
        v.mx[a] = bmax[a];
    }
    ray_caches c;
    memset(&c, 0, sizeof c);
    int64_t loads = 0;
    *out_dist = 0.0f;
    *out_sem = 0;
    return query(&v, px, py, pz, 1.0f, 0.0f, 0.0f, &c, out_dist, out_sem, &loads, NULL);
}

int oracle_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
