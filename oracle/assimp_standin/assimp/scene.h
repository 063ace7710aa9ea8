// Minimal stand-in for the Assimp scene types that projects/voxel-dag/src/compiler.cpp
// reads (compiler.cpp:260-311): meshes with vertices and triangle faces.
// TEST INFRASTRUCTURE ONLY: lets oracle/build.py compile the reference compiler
// without Assimp, for OBJ files holding `v x y z` and `f a b c` lines.
#pragma once

#include <vector>

struct aiVector3D {
    float x, y, z;
};

struct aiFace {
    unsigned int mNumIndices = 0;
    unsigned int* mIndices = nullptr;
};

struct aiMesh {
    unsigned int mNumVertices = 0;
    aiVector3D* mVertices = nullptr;
    unsigned int mNumFaces = 0;
    aiFace* mFaces = nullptr;
};

struct aiNode {
    int unused = 0;
};

#define AI_SCENE_FLAGS_INCOMPLETE 0x1

struct aiScene {
    unsigned int mFlags = 0;
    aiNode* mRootNode = nullptr;
    unsigned int mNumMeshes = 0;
    aiMesh** mMeshes = nullptr;
};
