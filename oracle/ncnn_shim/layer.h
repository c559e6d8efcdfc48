// Clean-room ncnn::Layer / Option subset for compiling the reference's layer
// sources (adaptive_window_attention.cpp, shared_linear.cpp; NCNN_VULKAN=0)
// into the CPU oracle.  TEST INFRASTRUCTURE ONLY.
//
// create_layer()/create_layer_cpu() return the oracle's CPU restatements of
// ncnn's built-in "SDPA" and "Gemm" layers (ncnn itself is not available in
// this build environment); see ncnn_shim.cpp.
#ifndef S2_ORACLE_NCNN_SHIM_LAYER_H
#define S2_ORACLE_NCNN_SHIM_LAYER_H

#include <vector>

#include "mat.h"
#include "modelbin.h"
#include "paramdict.h"

namespace ncnn {

class Option
{
public:
    Option() : blob_allocator(0), workspace_allocator(0), num_threads(1), use_vulkan_compute(false) {}
    Allocator* blob_allocator;
    Allocator* workspace_allocator;
    int num_threads;
    bool use_vulkan_compute;
};

class Layer
{
public:
    Layer() : one_blob_only(false), support_inplace(false), userdata(0) {}
    virtual ~Layer() {}

    virtual int load_param(const ParamDict&) { return 0; }
    virtual int load_model(const ModelBin&) { return 0; }
    virtual int create_pipeline(const Option&) { return 0; }
    virtual int destroy_pipeline(const Option&) { return 0; }

    virtual int forward(const std::vector<Mat>& bottom_blobs, std::vector<Mat>& top_blobs, const Option& opt) const
    {
        if (bottom_blobs.size() != 1 || top_blobs.size() != 1) return -1;
        return forward(bottom_blobs[0], top_blobs[0], opt);
    }
    virtual int forward(const Mat&, Mat&, const Option&) const { return -1; }

    bool one_blob_only;
    bool support_inplace;
    void* userdata;
};

Layer* create_layer(const char* type);
Layer* create_layer_cpu(const char* type);

} // namespace ncnn

#endif
