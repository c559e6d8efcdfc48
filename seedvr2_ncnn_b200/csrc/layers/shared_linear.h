// ncnn custom-layer surface of SharedLinear, backed by libseedvr2_cuda's
// tcgen05 GEMM.  Same class name, parameter ids (0 num_output, 1 num_input,
// 2 bias_term), weight order ([num_output][num_input] fp32, then bias), blob
// arity (two token streams in, two out) and error codes as the reference
// layer (src/seedvr2/shared_linear.h:14-48, shared_linear.cpp:27-96).  Both
// streams run in ONE launch against one bf16 copy of the weight (uploaded on
// first use, the upload_model analogue).
#pragma once

#include "adaptive_window_attention.h"

namespace seedvr2 {

class SharedLinear : public ncnn::Layer
{
public:
    SharedLinear();
    virtual ~SharedLinear();

    virtual int load_param(const ncnn::ParamDict& pd);
    virtual int load_model(const ncnn::ModelBin& mb);
    // [video, text] fp32 host Mats (dims 2, w = num_input) -> [video_out, text_out].
    virtual int forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                        const ncnn::Option& opt) const;
    // Device blobs: bf16 inputs [rows][num_input]; outputs bf16 or fp32
    // [rows][num_output] allocated by the caller; epilogue S2_EPI_* with
    // `gate` for S2_EPI_GATE_RESIDUAL (outputs are then the fp32 residual).
    int forward_cuda(const std::vector<CudaBlob>& bottom_blobs, std::vector<CudaBlob>& top_blobs,
                     int epilogue = S2_EPI_STORE, const float* gate = nullptr) const;

private:
    int upload() const;

    int num_output;
    int num_input;
    bool bias_term;
    ncnn::Mat weight_data;
    ncnn::Mat bias_data;
    mutable void* d_weight; // bf16 [num_output][num_input]
    mutable float* d_bias;  // fp32 [num_output] or null
};

ncnn::Layer* shared_linear_layer_creator(void* userdata);

} // namespace seedvr2
