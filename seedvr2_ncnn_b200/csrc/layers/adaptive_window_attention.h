// ncnn custom-layer surface of AdaptiveWindowAttention, backed by
// libseedvr2_cuda.  Same class name, parameter ids, weight order, blob arity,
// error codes and creator as the reference layer
// (src/seedvr2/adaptive_window_attention.h:16-118), so a block graph that
// registers "AdaptiveWindowAttention" (seedvr2_dit.cpp:614-616) gets this
// implementation unchanged.  forward(Mat) takes host blobs (uploads, runs the
// sm_100a kernels, downloads); forward_cuda takes device blobs and keeps the
// data on the GPU (the analogue of the reference's VkMat forward).
#pragma once

#include <array>
#include <vector>

#include "../../../include/seedvr2_cuda.h"
#include "ncnn_compat.h"

namespace seedvr2 {

struct WindowSlice
{
    int sample_index;
    int t0;
    int t1;
    int h0;
    int h1;
    int w0;
    int w1;
    int partition_offset;
    int token_count;
};

struct AdaptiveWindowPlan
{
    std::vector<WindowSlice> windows;
    std::vector<int> sample_window_count;
    std::vector<int> video_indices;
    std::vector<int> inverse_video_indices;
    std::vector<std::array<int, 3> > local_positions;
};

struct AdaptiveWindowRuntimeState
{
    std::vector<std::array<int, 3> > video_shapes;
    std::vector<int> text_lengths;
};

// build_adaptive_window_plan (adaptive_window_attention.h:46-49): the tuple is
// a target window count per axis; returns 0, -1 or -2 like the reference.
int build_adaptive_window_plan(const std::vector<std::array<int, 3> >& video_shapes,
                               const std::array<int, 3>& target_windows, bool shifted, AdaptiveWindowPlan& plan);

// A device blob for forward_cuda: [h rows][w elements] of `dtype`
// (S2_DTYPE_F32 / S2_DTYPE_BF16), rows `ld` elements apart.
struct CudaBlob
{
    void* data = nullptr;
    int w = 0;
    int h = 0;
    int ld = 0;
    int dtype = S2_DTYPE_F32;
};

class AdaptiveWindowAttention : public ncnn::Layer
{
public:
    AdaptiveWindowAttention();
    explicit AdaptiveWindowAttention(AdaptiveWindowRuntimeState* runtime_state);
    virtual ~AdaptiveWindowAttention();

    // ids 0 heads, 1 head_dim, 2-4 target windows, 5 shifted, 6 epsilon,
    // 7 rope pairs per axis, 8 shared_norm, 9 shape values int32,
    // 10 official bf16 attention (adaptive_window_attention.cpp:700-714);
    // 11 window_mode (0 = target count as the reference, 1 = extent; an
    // extension for explicit window extents).
    virtual int load_param(const ncnn::ParamDict& pd);
    // video_norm_q, video_norm_k, [text_norm_q, text_norm_k], rope_freqs (:716-738)
    virtual int load_model(const ncnn::ModelBin& mb);
    // 4 blobs [video_qkv, text_qkv, video_shape, text_length] or 8 blobs
    // [vq, vk, vv, tq, tk, tv, video_shape, text_length]; fp32 host Mats.
    virtual int forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                        const ncnn::Option& opt) const;
    // Device blobs: 2 or 6 qkv blobs, shapes from the runtime state (as the
    // reference's Vulkan forward, :1059-1114); outputs allocated by the
    // caller (video [Nv][inner], text [Nt][inner]).
    int forward_cuda(const std::vector<CudaBlob>& bottom_blobs, std::vector<CudaBlob>& top_blobs) const;

    // Test/runtime setup helpers (adaptive_window_attention.h:74-85).
    void configure(int heads, int head_dim, const std::array<int, 3>& target_windows, bool shifted, float epsilon,
                   int rope_pairs_per_axis, bool shape_values_are_int32 = false,
                   bool official_bf16_attention = false);
    int set_weights(const std::vector<float>& video_norm_q, const std::vector<float>& video_norm_k,
                    const std::vector<float>& text_norm_q, const std::vector<float>& text_norm_k,
                    const std::vector<float>& rope_freqs);
    void set_runtime_shapes(const std::vector<std::array<int, 3> >& video_shapes,
                            const std::vector<int>& text_lengths);

private:
    int upload_weights() const;
    int run(const std::vector<std::array<int, 3> >& shapes, const std::vector<int>& text_lengths, int in_dtype,
            const void* const* qkv, int64_t video_ld, int64_t text_ld, int out_dtype, void* video_out,
            void* text_out) const;

    int heads;
    int head_dim;
    std::array<int, 3> target_windows;
    bool shifted;
    float epsilon;
    int rope_pairs_per_axis;
    bool shared_norm;
    bool shape_values_are_int32;
    bool official_bf16_attention;
    int window_mode;

    ncnn::Mat video_norm_q;
    ncnn::Mat video_norm_k;
    ncnn::Mat text_norm_q;
    ncnn::Mat text_norm_k;
    ncnn::Mat rope_freqs;

    AdaptiveWindowRuntimeState owned_runtime_state;
    AdaptiveWindowRuntimeState* runtime_state;

    // device copies of the weights: [4][head_dim] norms then the freqs
    mutable float* d_weights;
    mutable bool weights_dirty;
};

ncnn::Layer* adaptive_window_attention_layer_creator(void* userdata);

// The library context used by the layers (one per process, on the CUDA
// device current at first use); the analogue of ncnn's Vulkan device.
s2_context* layer_context();

} // namespace seedvr2
