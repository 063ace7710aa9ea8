// Internal types shared by the pool builder and the trace kernels.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "tsdf.h"

namespace tsdf {

// ---- child-slot encoding of the re-packed pool -------------------------------
// A record is one internal DAG node: 8 u32 slots indexed by octant
// (x | y<<1 | z<<2, kernel.cu:171).  A slot holds one of:
//   kSlotVoid                 mask bit clear: empty octant (kernel.cu:177-190)
//   1 | sem:15 | half:16      leaf inline (semantic < 0x7FFF)
//   01 | index:30             leaf stored out of line (semantic >= 0x7FFF)
//   00 | record:30            internal child
constexpr uint32_t kSlotVoid = 0xFFFFFFFFu;
constexpr uint32_t kSlotLeafBit = 0x80000000u;
constexpr uint32_t kSlotExtBit = 0x40000000u;
constexpr uint32_t kSlotIndexMask = 0x3FFFFFFFu;
constexpr uint32_t kMaxRecords = 0x3FFFFFFFu;

inline uint32_t encode_leaf_inline(uint64_t word)
{
    const uint32_t sem = static_cast<uint32_t>((word >> 16) & 0xFFFFu);
    return kSlotLeafBit | (sem << 16) | static_cast<uint32_t>(word & 0xFFFFu);
}

// Deepest grid the integer descent supports: 2^12 cells per axis.
constexpr int kMaxGridDepth = 12;

struct HostPool {
    std::vector<uint32_t> recs;      // 8 per record
    std::vector<uint64_t> ext;       // out-of-line leaf words
    uint32_t root = kSlotVoid;
    uint32_t levels = 0;
    int32_t height = 0;              // records on the longest root path; -1 if the graph has a cycle
};

// Per-axis grid lines of the reference's midpoint rule: B[0] = lo, B[2^D] = hi, and for
// every cell [B[a], B[b]] met by the descent its midpoint B[(a+b)/2] = (B[a] + B[b]) * 0.5f
// (kernel.cu:166-176); out has 2^D + 2 entries, the last one +inf.  Returns false when the
// lines are not strictly increasing or the kernel's cell estimate bound does not hold.
bool build_grid_lines(float lo, float hi, int depth, float* out);

// Record-graph height (hp.height, -1 when cyclic) from record 0.
void compute_height(HostPool& hp);

// Checks of a record array read from a pool file (slot ranges, root, leaf table) and
// the recomputed BFS levels and height.
int check_records(HostPool& hp, std::string& err);

// Re-pack .gmdag words; returns TSDF_OK or an error with `err` set.
int build_host_pool(const uint64_t* words, uint64_t n, HostPool& out, std::string& err);

}  // namespace tsdf

struct tsdf_pool {
    int device = 0;
    int32_t height = 0;              // -1: cyclic record graph
    uint32_t* d_recs = nullptr;      // [records][8]
    uint64_t* d_ext = nullptr;       // [ext leaves]
    uint64_t records = 0;
    uint64_t ext = 0;
    uint64_t source_words = 0;
    uint64_t bytes = 0;
    uint32_t root = tsdf::kSlotVoid;
    uint32_t levels = 0;
    // last bounding box checked for strictly increasing grid lines (tsdf_cast)
    std::mutex grid_mu;
    float grid_bmin[3] = {0.f, 0.f, 0.f};
    float grid_bmax[3] = {0.f, 0.f, 0.f};
    int grid_ok = -1;  // -1 unknown, 0 float descent, 1 grid descent
};

// Device view of one scene (fan casts index a table of these).
struct TsdfSceneDev {
    const uint32_t* recs;
    const uint64_t* ext;
    const float* lines;              // B[0] of 3 rows of -inf, B[0..2^depth], +inf, or null (float descent)
    uint32_t root;
    uint32_t n_recs;
    float bmin[3];
    float bmax[3];
    float eps;
    int32_t depth;                   // grid depth D (cells per axis 2^D); -1: float descent
    float scale[3];                  // 2^D / (bmax - bmin) per axis, float division
    uint32_t n_ext;                  // out-of-line leaves (bounds-checked builds)
    float offs[3];                   // fma(-bmin, scale, -0.5) per axis: cell estimate v = fma(p, scale, offs)
};
static_assert(sizeof(TsdfSceneDev) == 96, "scene record layout");

struct tsdf_scenes {
    int device = 0;
    int n = 0;
    bool grid = false;               // every scene supports the integer descent
    TsdfSceneDev* d_table = nullptr;
    float* d_lines = nullptr;
    std::vector<TsdfSceneDev> host;
};

namespace tsdf {
// Cells per unit length along each axis, 2^D / (bmax - bmin), each an IEEE float
// subtraction and division (the same values the device's __fsub_rn / __fdiv_rn give),
// and the offset of the cell estimate v(p) = fma(p, scale, offs), offs = -bmin * scale - 1/2
// rounded once (half a cell below the cell coordinate); build_grid_lines proves the
// estimate's bound with the same values.
inline float grid_scale(float lo, float hi, int depth) { return static_cast<float>(1 << depth) / (hi - lo); }
inline float grid_offset(float lo, float scale) { return std::fma(-lo, scale, -0.5f); }
inline void set_grid_scale(TsdfSceneDev& d)
{
    for (int a = 0; a < 3; ++a) {
        d.scale[a] = d.depth >= 0 ? grid_scale(d.bmin[a], d.bmax[a], d.depth) : 0.0f;
        d.offs[a] = d.depth >= 0 ? grid_offset(d.bmin[a], d.scale[a]) : 0.0f;
    }
}
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

// Makes `device` the calling thread's current device for the scope and puts the
// caller's current device back when the scope ends, so that a call on a pool of
// another GPU does not move the caller's later allocations and launches (torch keeps
// its current device in the same per-thread runtime state).
class DeviceScope {
public:
    explicit DeviceScope(int device)
    {
        if (cudaGetDevice(&prev_) != cudaSuccess) {
            cudaGetLastError();
            prev_ = -1;
        }
        if (prev_ != device) {
            err_ = cudaSetDevice(device);
            switched_ = err_ == cudaSuccess && prev_ >= 0;
        }
    }
    ~DeviceScope()
    {
        if (switched_) cudaSetDevice(prev_);
    }
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;
    cudaError_t error() const { return err_; }

private:
    int prev_ = -1;
    bool switched_ = false;
    cudaError_t err_ = cudaSuccess;
};
}  // namespace tsdf
