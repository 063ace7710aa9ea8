// Stand-in post-processing flags (values are irrelevant: the stand-in reader
// only accepts triangles and applies no transform).  TEST INFRASTRUCTURE ONLY.
#pragma once

enum aiPostProcessSteps {
    aiProcess_JoinIdenticalVertices = 0x2,
    aiProcess_Triangulate = 0x8,
    aiProcess_PreTransformVertices = 0x100,
};
