// .gmdag file reading and DAG layout validation, shared by the scene library
// (libnavi_gmdag.so, C ABI gmdag_file_read / gmdag_validate_layout) and the trace
// library (libnavi_tsdf.so, tsdf_pool_create_from_file).
//
// Follows projects/environment/src/navi_environment/integration/voxel_dag.py:
//   load_gmdag_asset            :193-259  (checks in the same order)
//   _validate_gmdag_dag_layout  :29-78    (same depth-first order, so the first
//                                          error found is the reference's)
// Errors are returned as a status plus the values the reference's messages quote;
// callers format the texts.
#pragma once

#include <cstdint>
#include <string>

#include "gmdag.h"

namespace gmdag_io {

// Walks the DAG from word 0 depth-first, children in table order, with an explicit
// stack.  Returns true when valid; otherwise fills err (kind, node, value).
bool validate_layout(const uint64_t* nodes, uint64_t n, gmdag_layout_error* err);

// Reads header and payload into dst (dst_words >= node_count).  dst may be null:
// header and size checks only.  Returns the GMDAG_FILE_* status; info is filled as
// far as the file was parsed.
int read_file(const char* path, uint64_t* dst, uint64_t dst_words, gmdag_file_info* info);

// The reference's message for a failed read (voxel_dag.py:196-236 texts; the path is
// resolved with realpath, floats printed as Python's repr prints them).
std::string message(const char* path, int status, const gmdag_file_info& info);

// The reference's message for a layout error (voxel_dag.py:39-68 texts).
std::string layout_message(const gmdag_layout_error& e);

}  // namespace gmdag_io
