// Pool builder: .gmdag words -> 32-byte octant records, plus the pool and
// scene-table entry points of the C ABI.
//
// The reference traverses the raw words: per level it loads the node word and
// then the child-pointer word (kernel.cu:137, :198).  Here every internal node
// reachable from word 0 becomes one record of 8 u32 slots indexed directly by
// octant, so a level costs one 4-byte load from one 32-byte sector, and a leaf
// child is decoded from the slot without another load.  Records are numbered
// in BFS order from the root, so the top levels are contiguous at the start of
// the pool (they are staged in shared memory by the trace kernel).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <deque>
#include <limits>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "gmdag_io.h"
#include "tsdf_internal.h"

namespace tsdf {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg)
{
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what)
{
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return TSDF_ERR_CUDA;
}

const char* last_error_cstr() { return g_last_error.c_str(); }

// Height of the record graph (longest chain of records from the root), iterative DFS;
// a back edge means a cycle (height -1), which only the float descent (32-level cap)
// handles.
void compute_height(HostPool& hp)
{
    const size_t nr = hp.recs.size() / 8;
    hp.height = 0;
    if (nr > 0) {
        std::vector<int32_t> h(nr, 0);
        std::vector<uint8_t> state(nr, 0);  // 0 new, 1 open, 2 done
        std::vector<std::pair<uint32_t, int>> st;
        st.emplace_back(0u, 0);
        state[0] = 1;
        bool cyclic = false;
        while (!st.empty() && !cyclic) {
            auto& top = st.back();
            const uint32_t r = top.first;
            if (top.second == 8) {
                int32_t best = 0;
                for (int o = 0; o < 8; ++o) {
                    const uint32_t sl = hp.recs[8 * static_cast<size_t>(r) + o];
                    if (sl != kSlotVoid && !(sl & (kSlotLeafBit | kSlotExtBit))) best = std::max(best, h[sl]);
                }
                h[r] = best + 1;
                state[r] = 2;
                st.pop_back();
                continue;
            }
            const uint32_t sl = hp.recs[8 * static_cast<size_t>(r) + top.second];
            ++top.second;
            if (sl == kSlotVoid || (sl & (kSlotLeafBit | kSlotExtBit))) continue;
            if (state[sl] == 1) {
                cyclic = true;
            } else if (state[sl] == 0) {
                state[sl] = 1;
                st.emplace_back(sl, 0);
            }
        }
        hp.height = cyclic ? -1 : h[0];
    }
}

// Slot checks and derived figures of a record array read from a pool file: every
// internal slot names a record, every out-of-line slot a leaf, and the height and BFS
// levels are recomputed rather than trusted.
int check_records(HostPool& hp, std::string& err)
{
    const uint64_t nr = hp.recs.size() / 8;
    const uint64_t ne = hp.ext.size();
    auto slot_ok = [&](uint32_t sl) {
        if (sl == kSlotVoid || (sl & kSlotLeafBit)) return true;
        if (sl & kSlotExtBit) return static_cast<uint64_t>(sl & kSlotIndexMask) < ne;
        return static_cast<uint64_t>(sl) < nr;
    };
    if (nr > kMaxRecords || ne > kMaxRecords) {
        err = "pool file: too many records";
        return TSDF_ERR_FILE;
    }
    // the root is record 0 whenever it is internal (records are numbered in BFS order)
    const bool root_leaf = (hp.root & (kSlotLeafBit | kSlotExtBit)) != 0;
    if (hp.root == kSlotVoid || !slot_ok(hp.root) || (!root_leaf && hp.root != 0) || (root_leaf != (nr == 0))) {
        err = "pool file: root slot out of range";
        return TSDF_ERR_FILE;
    }
    for (uint64_t i = 0; i < hp.recs.size(); ++i)
        if (!slot_ok(hp.recs[i])) {
            err = "pool file: slot " + std::to_string(i) + " out of range";
            return TSDF_ERR_FILE;
        }
    for (uint64_t i = 0; i < ne; ++i)
        if ((hp.ext[i] >> 63) != 1) {
            err = "pool file: out-of-line entry " + std::to_string(i) + " is not a leaf word";
            return TSDF_ERR_FILE;
        }
    // BFS levels from record 0
    hp.levels = 0;
    if (nr > 0 && !(hp.root & (kSlotLeafBit | kSlotExtBit))) {
        std::vector<uint32_t> level(nr, 0xFFFFFFFFu);
        std::vector<uint32_t> q;
        q.push_back(hp.root);
        level[hp.root] = 0;
        uint32_t maxl = 0;
        for (size_t h = 0; h < q.size(); ++h) {
            const uint32_t r = q[h];
            maxl = std::max(maxl, level[r]);
            for (int o = 0; o < 8; ++o) {
                const uint32_t sl = hp.recs[8 * static_cast<size_t>(r) + o];
                if (sl == kSlotVoid || (sl & (kSlotLeafBit | kSlotExtBit))) continue;
                if (level[sl] == 0xFFFFFFFFu) {
                    level[sl] = level[r] + 1;
                    q.push_back(sl);
                }
            }
        }
        hp.levels = maxl + 1;
    }
    compute_height(hp);
    return TSDF_OK;
}

int build_host_pool(const uint64_t* w, uint64_t n, HostPool& hp, std::string& err)
{
    if (n == 0) {
        err = "DAG payload is empty";
        return TSDF_ERR_LAYOUT;
    }
    if (n > 0xFFFFFFFFull + 1) {
        err = "DAG payload exceeds 2^32 words";
        return TSDF_ERR_LAYOUT;
    }
    std::vector<int32_t> rec_of(static_cast<size_t>(n), -1);
    std::vector<uint32_t> rec_node;  // record -> source word index
    std::vector<uint32_t> rec_level;
    std::unordered_map<uint64_t, uint32_t> ext_of;
    hp.recs.clear();
    hp.ext.clear();

    auto encode = [&](uint32_t idx, uint32_t level, uint32_t& slot) -> int {
        const uint64_t word = w[idx];
        if ((word >> 63) == 1) {
            const uint32_t sem = static_cast<uint32_t>((word >> 16) & 0xFFFFu);
            if (sem < 0x7FFFu) {
                slot = encode_leaf_inline(word);
                return TSDF_OK;
            }
            const uint64_t key = word & 0x80000000FFFFFFFFull;
            auto it = ext_of.find(key);
            if (it == ext_of.end()) {
                if (hp.ext.size() >= kMaxRecords) {
                    err = "too many out-of-line leaves";
                    return TSDF_ERR_LAYOUT;
                }
                it = ext_of.emplace(key, static_cast<uint32_t>(hp.ext.size())).first;
                hp.ext.push_back(word);
            }
            slot = kSlotExtBit | it->second;
            return TSDF_OK;
        }
        if (rec_of[idx] < 0) {
            if (rec_node.size() >= kMaxRecords) {
                err = "too many internal nodes";
                return TSDF_ERR_LAYOUT;
            }
            rec_of[idx] = static_cast<int32_t>(rec_node.size());
            rec_node.push_back(idx);
            rec_level.push_back(level);
        }
        slot = static_cast<uint32_t>(rec_of[idx]);
        return TSDF_OK;
    };

    int rc = encode(0, 0, hp.root);
    if (rc != TSDF_OK) return rc;
    uint32_t max_level = 0;
    for (size_t r = 0; r < rec_node.size(); ++r) {
        const uint32_t idx = rec_node[r];
        const uint32_t lvl = rec_level[r];
        max_level = std::max(max_level, lvl);
        const uint64_t word = w[idx];
        const uint32_t mask = static_cast<uint32_t>((word >> 55) & 0xFFu);
        const uint64_t base = word & 0xFFFFFFFFull;
        uint32_t slots[8];
        for (int oct = 0; oct < 8; ++oct) {
            if ((mask & (1u << oct)) == 0) {
                slots[oct] = kSlotVoid;
                continue;
            }
            const uint64_t ci = base + static_cast<uint64_t>(__builtin_popcount(mask & ((1u << oct) - 1u)));
            if (ci >= n) {
                err = "Invalid gmdag DAG layout: child pointer table exceeds payload bounds for node " +
                      std::to_string(idx);
                return TSDF_ERR_LAYOUT;
            }
            const uint32_t child = static_cast<uint32_t>(w[ci]);
            if (child >= n) {
                err = "Invalid gmdag DAG layout: child reference out of range (" +
                      std::to_string(child) + ") from node " + std::to_string(idx);
                return TSDF_ERR_LAYOUT;
            }
            rc = encode(child, lvl + 1, slots[oct]);
            if (rc != TSDF_OK) return rc;
        }
        hp.recs.insert(hp.recs.end(), slots, slots + 8);
    }
    hp.levels = rec_node.empty() ? 0 : max_level + 1;

    compute_height(hp);
    return TSDF_OK;
}

bool build_grid_lines(float lo, float hi, int depth, float* out)
{
    const int n = 1 << depth;
    out[0] = lo;
    out[n] = hi;
    out[n + 1] = std::numeric_limits<float>::infinity();  // the +inf sentinel above the top face
    for (int lvl = 0; lvl < depth; ++lvl) {
        const int stride = n >> lvl;
        const int half = stride >> 1;
        for (int a = 0; a < n; a += stride) out[a + half] = (out[a] + out[a + stride]) * 0.5f;
    }
    for (int k = 0; k < n; ++k)
        if (!(out[k] < out[k + 1])) return false;
    // The kernel estimates the cell of p as e = floor(v(p)), v(p) = RN(p * scale + offs) (one
    // fused multiply-add) with scale = RN(n / RN(hi - lo)) and offs = RN(-lo * scale - 1/2),
    // and then picks cell e or e + 1 by the line above e.  v is monotone in p (scale > 0), so
    // k - 1 <= v(out[k]) < k at every line k puts e at the cell of p or the one below it
    // everywhere (below the box e <= -1, at or above its top e >= n - 1).
    const float scale = grid_scale(lo, hi, depth);
    const float offs = grid_offset(lo, scale);
    for (int k = 0; k <= n; ++k) {
        const float v = std::fma(out[k], scale, offs);
        if (!(v >= static_cast<float>(k - 1) && v < static_cast<float>(k))) return false;
    }
    return true;
}

}  // namespace tsdf

using tsdf::cuda_fail;
using tsdf::fail;

extern "C" {

const char* tsdf_last_error(void) { return tsdf::last_error_cstr(); }

int tsdf_version(void) { return TSDF_ABI_VERSION; }


static int check_device(int device)
{
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= count) return fail(TSDF_ERR_INVALID, "device ordinal out of range");
    int major = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    if (major != 10) return fail(TSDF_ERR_UNSUPPORTED, "libnavi_tsdf is built for sm_100a (B200) only");
    return TSDF_OK;
}

// Device copy of a host pool (records + out-of-line leaves).
static int upload_pool(const tsdf::HostPool& hp, uint64_t source_words, int device, tsdf_pool** out_pool)
{
    tsdf::DeviceScope scope(device);
    cudaError_t e = scope.error();
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    auto* pool = new (std::nothrow) tsdf_pool();
    if (!pool) return fail(TSDF_ERR_NO_MEMORY, "out of host memory");
    pool->device = device;
    pool->records = hp.recs.size() / 8;
    pool->ext = hp.ext.size();
    pool->source_words = source_words;
    pool->root = hp.root;
    pool->levels = hp.levels;
    pool->height = hp.height;
    const size_t rec_bytes = std::max<size_t>(hp.recs.size() * sizeof(uint32_t), 32);
    const size_t ext_bytes = std::max<size_t>(hp.ext.size() * sizeof(uint64_t), 8);
    e = cudaMalloc(&pool->d_recs, rec_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&pool->d_ext, ext_bytes);
    if (e != cudaSuccess) {
        cudaFree(pool->d_recs);
        delete pool;
        cudaGetLastError();
        return fail(TSDF_ERR_NO_MEMORY, std::string("cudaMalloc for the node pool failed: ") +
                                            cudaGetErrorString(e));
    }
    pool->bytes = rec_bytes + ext_bytes;
    if (!hp.recs.empty())
        e = cudaMemcpy(pool->d_recs, hp.recs.data(), hp.recs.size() * sizeof(uint32_t),
                       cudaMemcpyHostToDevice);
    if (e == cudaSuccess && !hp.ext.empty())
        e = cudaMemcpy(pool->d_ext, hp.ext.data(), hp.ext.size() * sizeof(uint64_t),
                       cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(pool->d_recs);
        cudaFree(pool->d_ext);
        delete pool;
        return cuda_fail(e, "cudaMemcpy of the node pool");
    }
    *out_pool = pool;
    return TSDF_OK;
}

int tsdf_pool_create(const uint64_t* host_words, uint64_t n_words, int device, uint32_t flags,
                     tsdf_pool** out_pool)
{
    (void)flags;
    if (!out_pool) return fail(TSDF_ERR_INVALID, "out_pool must not be null");
    *out_pool = nullptr;
    if (!host_words && n_words) return fail(TSDF_ERR_INVALID, "words must not be null");
    int rc = check_device(device);
    if (rc != TSDF_OK) return rc;
    tsdf::HostPool hp;
    std::string err;
    try {
        rc = tsdf::build_host_pool(host_words, n_words, hp, err);
    } catch (const std::bad_alloc&) {
        return fail(TSDF_ERR_NO_MEMORY, "out of host memory while re-packing the DAG");
    }
    if (rc != TSDF_OK) return fail(rc, err);

    return upload_pool(hp, n_words, device, out_pool);
}

int tsdf_pool_create_from_device(const uint64_t* device_words, uint64_t n_words, int device,
                                 uint32_t flags, void* stream, tsdf_pool** out_pool)
{
    if (!out_pool) return fail(TSDF_ERR_INVALID, "out_pool must not be null");
    *out_pool = nullptr;
    if (!device_words || n_words == 0) return fail(TSDF_ERR_LAYOUT, "DAG payload is empty");
    int rc = check_device(device);
    if (rc != TSDF_OK) return rc;
    std::vector<uint64_t> host;
    try {
        host.resize(n_words);
    } catch (const std::bad_alloc&) {
        return fail(TSDF_ERR_NO_MEMORY, "out of host memory");
    }
    cudaError_t e;
    {
        tsdf::DeviceScope scope(device);
        e = scope.error();
        if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        e = cudaMemcpyAsync(host.data(), device_words, n_words * sizeof(uint64_t), cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "copying the DAG words to the host");
    return tsdf_pool_create(host.data(), n_words, device, flags, out_pool);
}

int tsdf_pool_create_from_file(const char* path, int validate, int device, uint32_t flags,
                               tsdf_pool** out_pool, float* bbox_min, float* bbox_max)
{
    if (!out_pool) return fail(TSDF_ERR_INVALID, "out_pool must not be null");
    *out_pool = nullptr;
    if (!path) return fail(TSDF_ERR_INVALID, "path must not be null");
    int rc = check_device(device);
    if (rc != TSDF_OK) return rc;
    gmdag_file_info info{};
    int st = gmdag_io::read_file(path, nullptr, 0, &info);
    std::vector<uint64_t> words;
    if (st == GMDAG_FILE_OK) {
        try {
            words.resize(info.node_count);
        } catch (const std::bad_alloc&) {
            return fail(TSDF_ERR_NO_MEMORY, "out of host memory");
        }
        st = gmdag_io::read_file(path, words.data(), words.size(), &info);
    }
    if (st != GMDAG_FILE_OK)
        return fail(st == GMDAG_FILE_NOT_FOUND ? TSDF_ERR_NOT_FOUND : TSDF_ERR_FILE, gmdag_io::message(path, st, info));
    if (validate) {
        gmdag_layout_error le{};
        if (!gmdag_io::validate_layout(words.data(), words.size(), &le))
            return fail(TSDF_ERR_LAYOUT, gmdag_io::layout_message(le));
    }
    // voxel_dag.py:244-250: bbox_max = bmin + voxel * resolution in double
    for (int a = 0; a < 3; ++a) {
        if (bbox_min) bbox_min[a] = info.bbox_min[a];
        if (bbox_max)
            bbox_max[a] = static_cast<float>(static_cast<double>(info.bbox_min[a]) +
                                             static_cast<double>(info.voxel_size) * static_cast<double>(info.resolution));
    }
    return tsdf_pool_create(words.data(), words.size(), device, flags, out_pool);
}

namespace {

struct PoolFileHeader {
    char magic[4];
    uint32_t version;
    uint32_t root;
    uint32_t reserved;
    uint64_t records;
    uint64_t ext;
    uint64_t source_words;
};
static_assert(sizeof(PoolFileHeader) == 40, "pool file header layout");

}  // namespace

int tsdf_pool_save(const tsdf_pool* pool, const char* path)
{
    if (!pool || !path) return fail(TSDF_ERR_INVALID, "pool and path must not be null");
    std::vector<uint32_t> recs;
    std::vector<uint64_t> ext;
    try {
        recs.resize(pool->records * 8);
        ext.resize(pool->ext);
    } catch (const std::bad_alloc&) {
        return fail(TSDF_ERR_NO_MEMORY, "out of host memory");
    }
    cudaError_t e;
    {
        tsdf::DeviceScope scope(pool->device);
        e = scope.error();
        if (e == cudaSuccess && !recs.empty())
            e = cudaMemcpy(recs.data(), pool->d_recs, recs.size() * sizeof(uint32_t), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && !ext.empty())
            e = cudaMemcpy(ext.data(), pool->d_ext, ext.size() * sizeof(uint64_t), cudaMemcpyDeviceToHost);
    }
    if (e != cudaSuccess) return cuda_fail(e, "copying the node pool to the host");
    PoolFileHeader h{};
    std::memcpy(h.magic, "NPOL", 4);
    h.version = 1;
    h.root = pool->root;
    h.records = pool->records;
    h.ext = pool->ext;
    h.source_words = pool->source_words;
    const std::string tmp = std::string(path) + ".tmp";
    FILE* f = std::fopen(tmp.c_str(), "wb");
    if (!f) return fail(TSDF_ERR_FILE, "cannot write " + tmp);
    bool ok = std::fwrite(&h, sizeof h, 1, f) == 1;
    ok = ok && (recs.empty() || std::fwrite(recs.data(), sizeof(uint32_t), recs.size(), f) == recs.size());
    ok = ok && (ext.empty() || std::fwrite(ext.data(), sizeof(uint64_t), ext.size(), f) == ext.size());
    ok = (std::fclose(f) == 0) && ok;
    if (!ok || std::rename(tmp.c_str(), path) != 0) {
        std::remove(tmp.c_str());
        return fail(TSDF_ERR_FILE, std::string("cannot write ") + path);
    }
    return TSDF_OK;
}

int tsdf_pool_load(const char* path, int device, tsdf_pool** out_pool)
{
    if (!out_pool) return fail(TSDF_ERR_INVALID, "out_pool must not be null");
    *out_pool = nullptr;
    if (!path) return fail(TSDF_ERR_INVALID, "path must not be null");
    int rc = check_device(device);
    if (rc != TSDF_OK) return rc;
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(TSDF_ERR_NOT_FOUND, std::string("pool file does not exist: ") + path);
    PoolFileHeader h{};
    tsdf::HostPool hp;
    std::string err;
    bool ok = std::fread(&h, sizeof h, 1, f) == 1 && std::memcmp(h.magic, "NPOL", 4) == 0 && h.version == 1 &&
              h.records <= tsdf::kMaxRecords && h.ext <= tsdf::kMaxRecords;
    if (ok) {
        try {
            hp.recs.resize(h.records * 8);
            hp.ext.resize(h.ext);
        } catch (const std::bad_alloc&) {
            std::fclose(f);
            return fail(TSDF_ERR_NO_MEMORY, "out of host memory");
        }
        ok = (hp.recs.empty() || std::fread(hp.recs.data(), sizeof(uint32_t), hp.recs.size(), f) == hp.recs.size()) &&
             (hp.ext.empty() || std::fread(hp.ext.data(), sizeof(uint64_t), hp.ext.size(), f) == hp.ext.size());
        unsigned char extra;
        ok = ok && std::fread(&extra, 1, 1, f) == 0;  // nothing after the arrays
    }
    std::fclose(f);
    if (!ok) return fail(TSDF_ERR_FILE, std::string("not a navi pool file (or truncated): ") + path);
    hp.root = h.root;
    rc = tsdf::check_records(hp, err);
    if (rc != TSDF_OK) return fail(rc, err);
    return upload_pool(hp, h.source_words, device, out_pool);
}

int tsdf_pool_destroy(tsdf_pool* pool)
{
    if (!pool) return TSDF_OK;
    cudaError_t e1, e2;
    {
        tsdf::DeviceScope scope(pool->device);
        e1 = cudaFree(pool->d_recs);
        e2 = cudaFree(pool->d_ext);
    }
    delete pool;
    if (e1 != cudaSuccess) return cuda_fail(e1, "cudaFree");
    if (e2 != cudaSuccess) return cuda_fail(e2, "cudaFree");
    return TSDF_OK;
}

int tsdf_pool_stats_get(const tsdf_pool* pool, tsdf_pool_stats* out)
{
    if (!pool || !out) return fail(TSDF_ERR_INVALID, "pool and out must not be null");
    std::memset(out, 0, sizeof *out);
    out->source_words = pool->source_words;
    out->records = pool->records;
    out->ext_leaves = pool->ext;
    out->device_bytes = pool->bytes;
    out->root_slot = pool->root;
    out->bfs_levels = pool->levels;
    out->device = pool->device;
    return TSDF_OK;
}

int tsdf_scenes_create(const tsdf_pool* const* pools, int n, const float* bbox_min,
                       const float* bbox_max, const float* hit_epsilon, tsdf_scenes** out)
{
    if (!out) return fail(TSDF_ERR_INVALID, "out must not be null");
    *out = nullptr;
    if (!pools || n <= 0 || !bbox_min || !bbox_max || !hit_epsilon)
        return fail(TSDF_ERR_INVALID, "scene table needs n > 0 pools, bounds and epsilons");
    const int device = pools[0] ? pools[0]->device : -1;
    auto* sc = new (std::nothrow) tsdf_scenes();
    if (!sc) return fail(TSDF_ERR_NO_MEMORY, "out of host memory");
    sc->device = device;
    sc->n = n;
    sc->host.resize(n);
    std::vector<float> lines;
    std::vector<size_t> line_off(n, 0);
    bool grid = true;
    for (int i = 0; i < n; ++i) {
        const tsdf_pool* p = pools[i];
        if (!p || p->device != device) {
            delete sc;
            return fail(TSDF_ERR_INVALID, "every pool of a scene table must live on the same device");
        }
        TsdfSceneDev& d = sc->host[i];
        std::memset(&d, 0, sizeof d);
        d.recs = p->d_recs;
        d.ext = p->d_ext;
        d.root = p->root;
        d.n_recs = static_cast<uint32_t>(p->records);
        d.n_ext = static_cast<uint32_t>(p->ext);
        for (int a = 0; a < 3; ++a) {
            d.bmin[a] = bbox_min[3 * i + a];
            d.bmax[a] = bbox_max[3 * i + a];
            if (!std::isfinite(d.bmin[a]) || !std::isfinite(d.bmax[a]) || !(d.bmin[a] < d.bmax[a])) {
                delete sc;
                return fail(TSDF_ERR_INVALID, "bbox_min entries must be finite and strictly less than bbox_max entries");
            }
        }
        d.eps = hit_epsilon[i];
        d.depth = -1;
        if (p->height >= 0 && p->height <= tsdf::kMaxGridDepth) {
            // rows of -inf, B[0..n], +inf (the kernels' line_row layout); `lines` points at B[0]
            const size_t m = (size_t(1) << p->height) + 3;
            line_off[i] = lines.size() + 1;
            lines.resize(lines.size() + 3 * m);
            bool ok = true;
            for (int a = 0; a < 3; ++a) {
                lines[line_off[i] + a * m - 1] = -std::numeric_limits<float>::infinity();
                ok = ok && tsdf::build_grid_lines(d.bmin[a], d.bmax[a], p->height, &lines[line_off[i] + a * m]);
            }
            if (ok) d.depth = p->height;
        }
        tsdf::set_grid_scale(d);
        grid = grid && d.depth >= 0;
    }
    sc->grid = grid;
    tsdf::DeviceScope scope(device);
    cudaError_t e = scope.error();
    if (e == cudaSuccess && !lines.empty()) e = cudaMalloc(&sc->d_lines, lines.size() * sizeof(float));
    if (e == cudaSuccess && !lines.empty())
        e = cudaMemcpy(sc->d_lines, lines.data(), lines.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        for (int i = 0; i < n; ++i)
            if (sc->host[i].depth >= 0) sc->host[i].lines = sc->d_lines + line_off[i];
        e = cudaMalloc(&sc->d_table, sizeof(TsdfSceneDev) * n);
    }
    if (e == cudaSuccess)
        e = cudaMemcpy(sc->d_table, sc->host.data(), sizeof(TsdfSceneDev) * n, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(sc->d_table);
        cudaFree(sc->d_lines);
        delete sc;
        return cuda_fail(e, "uploading the scene table");
    }
    *out = sc;
    return TSDF_OK;
}

int tsdf_scenes_destroy(tsdf_scenes* scenes)
{
    if (!scenes) return TSDF_OK;
    cudaError_t e;
    {
        tsdf::DeviceScope scope(scenes->device);
        e = cudaFree(scenes->d_table);
        cudaFree(scenes->d_lines);
    }
    delete scenes;
    if (e != cudaSuccess) return cuda_fail(e, "cudaFree");
    return TSDF_OK;
}

}  // extern "C"
