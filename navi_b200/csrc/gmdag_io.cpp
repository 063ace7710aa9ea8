// .gmdag reading and layout validation; see gmdag_io.h.
#include "gmdag_io.h"

#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <vector>

#include <sys/stat.h>

namespace gmdag_io {

namespace {

constexpr size_t kHeaderBytes = 32;  // struct "<4sIIffffI" (voxel_dag.py:26)

// Python's repr of a double: shortest round-trip digits, fixed notation for
// decimal exponents in (-4, 16], otherwise d.ddde+XX.
std::string py_repr(double x)
{
    if (std::isnan(x)) return "nan";
    if (std::isinf(x)) return x > 0 ? "inf" : "-inf";
    if (x == 0.0) return std::signbit(x) ? "-0.0" : "0.0";
    char buf[64];
    for (int p = 1; p <= 17; ++p) {
        std::snprintf(buf, sizeof buf, "%.*e", p - 1, x);
        if (std::strtod(buf, nullptr) == x) break;
    }
    // buf = [-]d[.ddd]e[+-]XX
    std::string s(buf);
    std::string sign;
    if (s[0] == '-') {
        sign = "-";
        s.erase(0, 1);
    }
    const size_t epos = s.find('e');
    const int exp10 = std::atoi(s.c_str() + epos + 1);
    std::string digits;
    for (size_t i = 0; i < epos; ++i)
        if (s[i] != '.') digits.push_back(s[i]);
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    const int n = static_cast<int>(digits.size());
    const int decpt = exp10 + 1;
    std::string out;
    if (decpt <= -4 || decpt > 16) {
        out = digits.substr(0, 1);
        if (n > 1) out += "." + digits.substr(1);
        char e[16];
        std::snprintf(e, sizeof e, "e%+03d", decpt - 1);
        out += e;
    } else if (decpt <= 0) {
        out = "0." + std::string(static_cast<size_t>(-decpt), '0') + digits;
    } else if (decpt >= n) {
        out = digits + std::string(static_cast<size_t>(decpt - n), '0') + ".0";
    } else {
        out = digits.substr(0, static_cast<size_t>(decpt)) + "." + digits.substr(static_cast<size_t>(decpt));
    }
    return sign + out;
}

// Python's repr of bytes (b'...'), for the magic.
std::string py_bytes_repr(const char* b, size_t n)
{
    bool has_sq = false, has_dq = false;
    for (size_t i = 0; i < n; ++i) {
        has_sq |= b[i] == '\'';
        has_dq |= b[i] == '"';
    }
    const char q = (has_sq && !has_dq) ? '"' : '\'';
    std::string out = "b";
    out.push_back(q);
    for (size_t i = 0; i < n; ++i) {
        const unsigned char c = static_cast<unsigned char>(b[i]);
        if (c == static_cast<unsigned char>(q) || c == '\\') {
            out.push_back('\\');
            out.push_back(static_cast<char>(c));
        } else if (c == '\t') {
            out += "\\t";
        } else if (c == '\n') {
            out += "\\n";
        } else if (c == '\r') {
            out += "\\r";
        } else if (c < 0x20 || c >= 0x7f) {
            char e[8];
            std::snprintf(e, sizeof e, "\\x%02x", c);
            out += e;
        } else {
            out.push_back(static_cast<char>(c));
        }
    }
    out.push_back(q);
    return out;
}

uint32_t rd_u32(const unsigned char* p)
{
    uint32_t v;
    std::memcpy(&v, p, 4);
    return v;
}

float rd_f32(const unsigned char* p)
{
    float v;
    std::memcpy(&v, p, 4);
    return v;
}

}  // namespace

bool validate_layout(const uint64_t* nodes, uint64_t n, gmdag_layout_error* err)
{
    gmdag_layout_error e{};
    auto fail = [&](int32_t kind, uint64_t node, uint64_t value) {
        e.kind = kind;
        e.node = node;
        e.value = value;
        if (err) *err = e;
        return false;
    };
    if (err) *err = e;
    if (n == 0) return fail(GMDAG_LAYOUT_NODE_OUT_OF_RANGE, 0, 0);  // visit(0) on an empty payload
    std::vector<uint8_t> state(n, 0);  // 0 new, 1 on the active path, 2 done
    struct Frame {
        uint64_t node;
        uint32_t next;
    };
    std::vector<Frame> stack;
    // entering a node: the checks of visit() before its children (voxel_dag.py:35-62)
    auto enter = [&](uint64_t idx) -> bool {  // false: error recorded
        if (state[idx] == 2) return true;
        if (state[idx] == 1) return fail(GMDAG_LAYOUT_CYCLE, idx, 0);
        const uint64_t w = nodes[idx];
        if ((w >> 63) != 0) {
            state[idx] = 2;  // a leaf has no children
            return true;
        }
        const uint32_t mask = static_cast<uint32_t>((w >> 55) & 0xFF);
        if (mask == 0) return fail(GMDAG_LAYOUT_EMPTY_MASK, idx, 0);
        const uint64_t base = w & 0xFFFFFFFFull;
        const uint64_t count = static_cast<uint64_t>(__builtin_popcount(mask));
        if (base >= n) return fail(GMDAG_LAYOUT_TABLE_BEYOND_PAYLOAD, idx, base);
        if (base + count > n) return fail(GMDAG_LAYOUT_TABLE_EXCEEDS_PAYLOAD, idx, base);
        state[idx] = 1;
        stack.push_back({idx, 0});
        return true;
    };
    if (!enter(0)) return false;
    while (!stack.empty()) {
        Frame& f = stack.back();
        const uint64_t w = nodes[f.node];
        const uint32_t count = static_cast<uint32_t>(__builtin_popcount(static_cast<uint32_t>((w >> 55) & 0xFF)));
        if (f.next >= count) {
            state[f.node] = 2;
            stack.pop_back();
            continue;
        }
        const uint64_t base = w & 0xFFFFFFFFull;
        const uint64_t parent = f.node;
        const uint64_t child = nodes[base + f.next];
        ++f.next;
        if (child >= n) return fail(GMDAG_LAYOUT_CHILD_OUT_OF_RANGE, parent, child);
        if (!enter(child)) return false;
    }
    return true;
}

int read_file(const char* path, uint64_t* dst, uint64_t dst_words, gmdag_file_info* info)
{
    gmdag_file_info z{};
    if (info) *info = z;
    gmdag_file_info& I = info ? *info : z;
    struct stat st;
    if (!path || ::stat(path, &st) != 0) return GMDAG_FILE_NOT_FOUND;
    FILE* fh = std::fopen(path, "rb");
    if (!fh) return GMDAG_FILE_IO_ERROR;
    struct Closer {
        FILE* f;
        ~Closer() { std::fclose(f); }
    } closer{fh};
    unsigned char h[kHeaderBytes];
    const size_t got = std::fread(h, 1, kHeaderBytes, fh);
    if (got != kHeaderBytes) return GMDAG_FILE_SHORT_HEADER;
    std::memcpy(I.magic, h, 4);
    I.version = rd_u32(h + 4);
    I.resolution = rd_u32(h + 8);
    for (int a = 0; a < 3; ++a) I.bbox_min[a] = rd_f32(h + 12 + 4 * a);
    I.voxel_size = rd_f32(h + 24);
    I.node_count = rd_u32(h + 28);
    if (std::memcmp(I.magic, "GDAG", 4) != 0) return GMDAG_FILE_BAD_MAGIC;
    if (I.version != 1) return GMDAG_FILE_BAD_VERSION;
    if (I.resolution == 0) return GMDAG_FILE_BAD_RESOLUTION;
    if (!std::isfinite(I.voxel_size) || I.voxel_size <= 0.0f) return GMDAG_FILE_BAD_VOXEL;
    if (I.node_count == 0) return GMDAG_FILE_BAD_NODE_COUNT;
    for (int a = 0; a < 3; ++a)
        if (!std::isfinite(I.bbox_min[a])) return GMDAG_FILE_BAD_BOUNDS;
    const uint64_t payload = static_cast<uint64_t>(st.st_size) - kHeaderBytes;
    I.nodes_found = std::min<uint64_t>(payload / 8, I.node_count);
    if (I.nodes_found < I.node_count) return GMDAG_FILE_SHORT_PAYLOAD;
    I.trailing_bytes = payload - static_cast<uint64_t>(I.node_count) * 8;
    if (I.trailing_bytes) return GMDAG_FILE_TRAILING_BYTES;
    if (dst) {
        if (dst_words < I.node_count) return GMDAG_FILE_BUFFER_TOO_SMALL;
        if (std::fread(dst, 8, I.node_count, fh) != I.node_count) return GMDAG_FILE_IO_ERROR;
    }
    return GMDAG_FILE_OK;
}

std::string message(const char* path, int status, const gmdag_file_info& I)
{
    char rp[PATH_MAX];
    const std::string p = (path && ::realpath(path, rp)) ? std::string(rp) : std::string(path ? path : "");
    switch (status) {
    case GMDAG_FILE_OK: return "";
    case GMDAG_FILE_NOT_FOUND: return "gmdag asset does not exist: " + p;
    case GMDAG_FILE_SHORT_HEADER: return "Invalid gmdag header in " + p;
    case GMDAG_FILE_BAD_MAGIC: return "Unsupported gmdag magic in " + p + ": " + py_bytes_repr(I.magic, 4);
    case GMDAG_FILE_BAD_VERSION: return "Unsupported gmdag version in " + p + ": " + std::to_string(I.version);
    case GMDAG_FILE_BAD_RESOLUTION: return "Invalid gmdag resolution in " + p + ": " + std::to_string(I.resolution);
    case GMDAG_FILE_BAD_VOXEL:
        return "Invalid gmdag voxel size in " + p + ": " + py_repr(static_cast<double>(I.voxel_size));
    case GMDAG_FILE_BAD_NODE_COUNT: return "Invalid gmdag node count in " + p + ": " + std::to_string(I.node_count);
    case GMDAG_FILE_BAD_BOUNDS: return "Invalid gmdag bounds in " + p + ": non-finite bbox_min values detected";
    case GMDAG_FILE_SHORT_PAYLOAD:
        return "Invalid gmdag node payload in " + p + ": expected " + std::to_string(I.node_count) + " nodes, found " +
               std::to_string(I.nodes_found);
    case GMDAG_FILE_TRAILING_BYTES: return "Invalid gmdag payload in " + p + ": trailing bytes detected";
    case GMDAG_FILE_IO_ERROR: return "could not read " + p;
    case GMDAG_FILE_BUFFER_TOO_SMALL: return "destination holds fewer words than the node count of " + p;
    default: return "gmdag read failed";
    }
}

}  // namespace gmdag_io

namespace gmdag_io {

std::string layout_message(const gmdag_layout_error& e)
{
    const std::string pre = "Invalid gmdag DAG layout: ";
    switch (e.kind) {
    case GMDAG_LAYOUT_NODE_OUT_OF_RANGE: return pre + "node index out of range: " + std::to_string(e.node);
    case GMDAG_LAYOUT_CYCLE: return pre + "cycle detected at node index " + std::to_string(e.node);
    case GMDAG_LAYOUT_EMPTY_MASK: return pre + "internal node " + std::to_string(e.node) + " has empty child mask";
    case GMDAG_LAYOUT_TABLE_BEYOND_PAYLOAD:
        return pre + "child pointer table starts beyond payload at index " + std::to_string(e.value);
    case GMDAG_LAYOUT_TABLE_EXCEEDS_PAYLOAD:
        return pre + "child pointer table exceeds payload bounds for node " + std::to_string(e.node);
    case GMDAG_LAYOUT_CHILD_OUT_OF_RANGE:
        return pre + "child reference out of range (" + std::to_string(e.value) + ") from node " +
               std::to_string(e.node);
    default: return "";
    }
}

}  // namespace gmdag_io
