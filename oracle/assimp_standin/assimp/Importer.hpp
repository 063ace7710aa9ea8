// Stand-in Assimp::Importer: reads `v` and `f` lines of an OBJ file into one
// triangle mesh (vertex coordinates parsed with strtof, which round-trips the
// %.9g text the tests write).  TEST INFRASTRUCTURE ONLY.
#pragma once

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "scene.h"

namespace Assimp {

class Importer {
public:
    const aiScene* ReadFile(const std::string& path, unsigned int /*flags*/)
    {
        std::ifstream in(path);
        if (!in) {
            err_ = "cannot open " + path;
            return nullptr;
        }
        std::string line;
        while (std::getline(in, line)) {
            if (line.size() > 2 && line[0] == 'v' && line[1] == ' ') {
                const char* p = line.c_str() + 2;
                char* end = nullptr;
                aiVector3D v;
                v.x = std::strtof(p, &end);
                v.y = std::strtof(end, &end);
                v.z = std::strtof(end, &end);
                verts_.push_back(v);
            } else if (line.size() > 2 && line[0] == 'f' && line[1] == ' ') {
                const char* p = line.c_str() + 2;
                char* end = nullptr;
                unsigned int tri[3];
                for (int k = 0; k < 3; ++k) {
                    tri[k] = static_cast<unsigned int>(std::strtoul(p, &end, 10)) - 1u;
                    while (*end && *end != ' ') ++end;
                    p = end;
                }
                for (unsigned int t : tri) idx_.push_back(t);
            }
        }
        if (verts_.empty() || idx_.empty()) {
            err_ = "no triangles in " + path;
            return nullptr;
        }
        faces_.resize(idx_.size() / 3);
        for (size_t f = 0; f < faces_.size(); ++f) {
            faces_[f].mNumIndices = 3;
            faces_[f].mIndices = &idx_[3 * f];
        }
        mesh_.mNumVertices = static_cast<unsigned int>(verts_.size());
        mesh_.mVertices = verts_.data();
        mesh_.mNumFaces = static_cast<unsigned int>(faces_.size());
        mesh_.mFaces = faces_.data();
        mesh_ptr_ = &mesh_;
        scene_.mRootNode = &root_;
        scene_.mNumMeshes = 1;
        scene_.mMeshes = &mesh_ptr_;
        return &scene_;
    }

    const char* GetErrorString() const { return err_.c_str(); }

private:
    std::string err_;
    std::vector<aiVector3D> verts_;
    std::vector<unsigned int> idx_;
    std::vector<aiFace> faces_;
    aiMesh mesh_;
    aiMesh* mesh_ptr_ = nullptr;
    aiNode root_;
    aiScene scene_;
};

}  // namespace Assimp
