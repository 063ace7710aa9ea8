// Driver for the reference scene compiler (projects/voxel-dag/src/compiler.cpp),
// built against the Assimp stand-in: ref_voxel_dag <input.obj> <output.gmdag> <resolution>.
// TEST INFRASTRUCTURE ONLY.
#include <cstdio>
#include <cstdlib>
#include <exception>

#include "compiler.hpp"

int main(int argc, char** argv)
{
    if (argc != 4) {
        std::fprintf(stderr, "usage: %s input.obj output.gmdag resolution\n", argv[0]);
        return 2;
    }
    try {
        voxeldag::Compiler c(static_cast<uint32_t>(std::strtoul(argv[3], nullptr, 10)));
        c.compile(argv[1], argv[2]);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "%s\n", e.what());
        return 1;
    }
    return 0;
}
