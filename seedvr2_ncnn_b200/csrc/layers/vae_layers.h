// ncnn custom-layer surface of the SeedVR2 VAE layers, backed by
// libseedvr2_cuda: DecomposedConv3D (decomposed_conv3d.h:15-88),
// VAEDownsample3D (vae_downsample3d.h:13-44), VAEUpsample3D
// (vae_upsample3d.h:13-46) and VAEChunkedMHA (vae_chunked_mha.h:13-52), all
// under src/seedvr2/ of the reference.  Same class names, parameter ids, the
// same ModelBin load sequence, one blob in / one out, the same thread-local
// temporal-memory state and the same error codes (0 / -1 / -100, plus the
// library's -3 CUDA / -5 no device).
//
// forward(Mat) takes host fp32 blobs (upload, run, download), like the
// reference's CPU path; forward_cuda takes device fp32 planes (the VkMat-path
// analogue).  The weights go to the device on the first forward (the
// upload_model analogue); each convolution's cached frames live on the device
// next to it.
#pragma once

#include <vector>

#include "adaptive_window_attention.h"

namespace seedvr2 {

// The VAE's chunked-decode memory switch (decomposed_conv3d.h:15-23): thread
// local, read by every VAE layer's forward.
enum class MemoryState
{
    DISABLED,
    INITIALIZING,
    ACTIVE
};

MemoryState get_vae_memory_state();
void set_vae_memory_state(MemoryState state);

class DecomposedConv3D : public ncnn::Layer
{
public:
    DecomposedConv3D();
    virtual ~DecomposedConv3D();

    // ids 0-15: num_output, num_input, kernel_w, kernel_h, kernel_t, stride_t,
    // dilation_t, head_frames, stride_w, stride_h, dilation_w, dilation_h,
    // pad_w, pad_h, groups, bias_term (load_model's config blob overrides them)
    virtual int load_param(const ncnn::ParamDict& pd);
    // config (16 values), bias [num_output] when bias_term, then kernel_t
    // spatial kernels [num_output][num_input / groups][kernel_h][kernel_w]
    virtual int load_model(const ncnn::ModelBin& mb);
    // this build's limits: groups 1, stride_w <= 2 (-1 otherwise)
    virtual int create_pipeline(const ncnn::Option& opt);
    virtual int destroy_pipeline(const ncnn::Option& opt);
    // 4-D blob (w, h, d = frames, c = num_input) -> (w', h', d', num_output)
    virtual int forward(const ncnn::Mat& bottom_blob, ncnn::Mat& top_blob, const ncnn::Option& opt) const;

    // The reference frees the Vulkan copy of the previous chunk's frames here,
    // kept alive for command buffers recorded but not yet run; this path runs
    // each forward to completion, so there is nothing to free.
    void release_completed_temporal_memory() const;
    void reset_temporal_memory() const;

    // Device planes: in fp32 [num_input][in_cstep], out fp32
    // [num_output][out_cstep]; shapes as output_shape() gives them.
    int output_shape(int w, int h, int d, int* out_whdc) const;
    int forward_cuda(const float* in, int64_t in_cstep, int w, int h, int d, float* out, int64_t out_cstep) const;

    // The float sequence load_model read (config, bias, kernels).
    void append_model(std::vector<float>& blob) const;

private:
    int upload() const;

    int num_output;
    int num_input;
    int kernel_w;
    int kernel_h;
    int kernel_t;
    int stride_t;
    int dilation_t;
    int head_frames;
    int stride_w;
    int stride_h;
    int dilation_w;
    int dilation_h;
    int pad_w;
    int pad_h;
    int groups;
    bool bias_term;

    ncnn::Mat bias_data;
    std::vector<ncnn::Mat> spatial_weights;
    mutable s2_conv3d* device_layer;
};

class VAEDownsample3D : public ncnn::Layer
{
public:
    VAEDownsample3D();
    virtual ~VAEDownsample3D();

    // channels, pad_right, pad_bottom, then the DecomposedConv3D's model
    virtual int load_model(const ncnn::ModelBin& mb);
    virtual int create_pipeline(const ncnn::Option& opt);
    virtual int destroy_pipeline(const ncnn::Option& opt);
    // zero padding on the right / bottom of every frame, then the convolution
    virtual int forward(const ncnn::Mat& bottom_blob, ncnn::Mat& top_blob, const ncnn::Option& opt) const;

    void release_completed_temporal_memory() const;
    void reset_temporal_memory() const;

    int output_shape(int w, int h, int d, int* out_whdc) const;
    int forward_cuda(const float* in, int64_t in_cstep, int w, int h, int d, float* out, int64_t out_cstep) const;

private:
    int upload() const;

    int channels;
    int pad_right;
    int pad_bottom;
    DecomposedConv3D* convolution;
    mutable s2_vae_resample* device_layer;
};

class VAEUpsample3D : public ncnn::Layer
{
public:
    VAEUpsample3D();
    virtual ~VAEUpsample3D();

    // channels, temporal_ratio, spatial_ratio, remove_temporal_head, then the
    // post conv's model and the upscale conv's model
    virtual int load_model(const ncnn::ModelBin& mb);
    virtual int create_pipeline(const ncnn::Option& opt);
    virtual int destroy_pipeline(const ncnn::Option& opt);
    // upscale conv, pixel / temporal shuffle (frame 1 dropped unless the
    // memory is ACTIVE when the temporal ratio is 2), post conv
    virtual int forward(const ncnn::Mat& bottom_blob, ncnn::Mat& top_blob, const ncnn::Option& opt) const;

    void release_completed_temporal_memory() const;
    void reset_temporal_memory() const;

    int output_shape(int w, int h, int d, int* out_whdc) const;
    int forward_cuda(const float* in, int64_t in_cstep, int w, int h, int d, float* out, int64_t out_cstep) const;

private:
    int upload() const;

    int channels;
    int temporal_ratio;
    int spatial_ratio;
    bool remove_temporal_head;
    DecomposedConv3D* post_conv;
    DecomposedConv3D* upscale_conv;
    mutable s2_vae_resample* device_layer;
};

class VAEChunkedMHA : public ncnn::Layer
{
public:
    VAEChunkedMHA();
    virtual ~VAEChunkedMHA();

    // ids 0 embed_dim, 1 num_heads, 2 weight_data_size, 3 kdim, 4 vdim,
    // 6 scale (default 1/sqrt(embed_dim / num_heads)), 20 chunk_size
    virtual int load_param(const ncnn::ParamDict& pd);
    // q w, q b, k w, k b, v w, v b, out w, out b
    virtual int load_model(const ncnn::ModelBin& mb);
    // this build's limits: one head, kdim = vdim = qdim = embed_dim, a
    // multiple of 8 (-1 otherwise)
    virtual int create_pipeline(const ncnn::Option& opt);
    virtual int destroy_pipeline(const ncnn::Option& opt);
    // x [tokens][qdim] (dims 2) -> [tokens][qdim]
    virtual int forward(const ncnn::Mat& bottom_blob, ncnn::Mat& top_blob, const ncnn::Option& opt) const;

    // Device rows: x, out fp32 [tokens][embed_dim].
    int forward_cuda(const float* x, int tokens, float* out) const;

private:
    bool supported() const;
    int upload() const;

    int embed_dim;
    int num_heads;
    int weight_data_size;
    int kdim;
    int vdim;
    float scale;
    int chunk_size; // the reference's query chunk; this path picks its own (the score chunk stays under 256 MiB)
    ncnn::Mat weights[8];
    mutable s2_vae_mha* device_layer;
};

ncnn::Layer* decomposed_conv3d_layer_creator(void* userdata);
ncnn::Layer* vae_downsample3d_layer_creator(void* userdata);
ncnn::Layer* vae_upsample3d_layer_creator(void* userdata);
ncnn::Layer* vae_chunked_mha_layer_creator(void* userdata);

} // namespace seedvr2
