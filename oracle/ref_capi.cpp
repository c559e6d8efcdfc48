// extern "C" wrapper around the reference's OWN layer code, compiled
// unmodified from the reference tree (src/seedvr2/adaptive_window_attention.cpp
// and src/seedvr2/shared_linear.cpp, NCNN_VULKAN=0) against the clean-room
// ncnn API shim in oracle/ncnn_shim.  Built by oracle/Makefile into
// oracle/_ref/libs2_ref.so.
//
// TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline / reference arm load this library as the checker or as the
// timed CPU baseline; the shipped library never links it.
#include <array>
#include <cstring>
#include <vector>

#include "adaptive_window_attention.h"
#include "shared_linear.h"

using seedvr2::AdaptiveWindowPlan;

extern "C" {

// build_adaptive_window_plan (adaptive_window_attention.cpp:565-655).
// Returns an opaque plan handle in *out (free with s2ref_plan_free).
int s2ref_plan_build(const int* shapes, int batch, const int* target, int shifted, void** out)
{
    *out = 0;
    std::vector<std::array<int, 3> > video_shapes((size_t)batch);
    for (int s = 0; s < batch; s++)
        for (int a = 0; a < 3; a++) video_shapes[s][a] = shapes[s * 3 + a];
    std::array<int, 3> tw = {target[0], target[1], target[2]};
    AdaptiveWindowPlan* plan = new AdaptiveWindowPlan;
    const int ret = seedvr2::build_adaptive_window_plan(video_shapes, tw, shifted != 0, *plan);
    if (ret != 0)
    {
        delete plan;
        return ret;
    }
    *out = plan;
    return 0;
}

void s2ref_plan_sizes(const void* handle, int* num_windows, int* num_tokens, int* num_samples)
{
    const AdaptiveWindowPlan* plan = (const AdaptiveWindowPlan*)handle;
    *num_windows = (int)plan->windows.size();
    *num_tokens = (int)plan->video_indices.size();
    *num_samples = (int)plan->sample_window_count.size();
}

// windows: 9 ints per window in WindowSlice field order.
void s2ref_plan_copy(const void* handle, int* windows, int* sample_window_count, int* video_indices,
                     int* inverse_video_indices, int* local_positions)
{
    const AdaptiveWindowPlan* plan = (const AdaptiveWindowPlan*)handle;
    for (size_t i = 0; i < plan->windows.size(); i++)
    {
        const seedvr2::WindowSlice& w = plan->windows[i];
        int* o = windows + i * 9;
        o[0] = w.sample_index;
        o[1] = w.t0;
        o[2] = w.t1;
        o[3] = w.h0;
        o[4] = w.h1;
        o[5] = w.w0;
        o[6] = w.w1;
        o[7] = w.partition_offset;
        o[8] = w.token_count;
    }
    for (size_t i = 0; i < plan->sample_window_count.size(); i++) sample_window_count[i] = plan->sample_window_count[i];
    for (size_t i = 0; i < plan->video_indices.size(); i++)
    {
        video_indices[i] = plan->video_indices[i];
        inverse_video_indices[i] = plan->inverse_video_indices[i];
        for (int a = 0; a < 3; a++) local_positions[i * 3 + a] = plan->local_positions[i][a];
    }
}

void s2ref_plan_free(void* handle)
{
    delete (AdaptiveWindowPlan*)handle;
}

// AdaptiveWindowAttention::forward(Mat) (adaptive_window_attention.cpp:764-978)
// driven through the layer's ncnn surface: creator, load_param (ids 0-10,
// :700-714), load_model (raw fp32 blobs in the order of :716-738), forward.
//
// params: heads, head_dim, target0..2, shifted, rope_pairs, shared_norm,
//         shape_values_int32, official_bf16_attention (10 ints) + epsilon.
// weights: video_norm_q, video_norm_k, [text_norm_q, text_norm_k], rope_freqs.
// split=0: inputs[0]=video_qkv [Nv x 3*inner], inputs[1]=text_qkv [Nt x 3*inner]
// split=1: inputs[0..5]=vq,vk,vv,tq,tk,tv each [rows x inner]
// shape_blob: batch x 3 values; text_blob: batch x 1 values (floats, or int32
// bit patterns when shape_values_int32).
int s2ref_awa_forward(const int* params, float epsilon, const float* weights, int num_weights, int split,
                      const float* const* inputs, int video_tokens, int text_tokens, const void* shape_blob,
                      const void* text_blob, int batch, float* video_out, float* text_out)
{
    ncnn::ParamDict pd;
    pd.set(0, params[0]);
    pd.set(1, params[1]);
    pd.set(2, params[2]);
    pd.set(3, params[3]);
    pd.set(4, params[4]);
    pd.set(5, params[5]);
    pd.set(6, epsilon);
    pd.set(7, params[6]);
    pd.set(8, params[7]);
    pd.set(9, params[8]);
    pd.set(10, params[9]);

    ncnn::Layer* layer = seedvr2::adaptive_window_attention_layer_creator(0);
    int ret = layer->load_param(pd);
    if (ret == 0)
    {
        ncnn::ModelBinFromFloats mb(weights, (size_t)num_weights);
        ret = layer->load_model(mb);
    }
    if (ret != 0)
    {
        delete layer;
        return ret;
    }

    const int heads = params[0];
    const int head_dim = params[1];
    const int inner = heads * head_dim;
    std::vector<ncnn::Mat> bottom(split ? 8 : 4);
    if (split)
    {
        for (int p = 0; p < 6; p++)
        {
            const int rows = p < 3 ? video_tokens : text_tokens;
            bottom[p].create(inner, rows);
            std::memcpy(bottom[p].data, inputs[p], (size_t)inner * rows * sizeof(float));
        }
    }
    else
    {
        bottom[0].create(inner * 3, video_tokens);
        std::memcpy(bottom[0].data, inputs[0], (size_t)inner * 3 * video_tokens * sizeof(float));
        bottom[1].create(inner * 3, text_tokens);
        std::memcpy(bottom[1].data, inputs[1], (size_t)inner * 3 * text_tokens * sizeof(float));
    }
    ncnn::Mat& shape_mat = bottom[split ? 6 : 2];
    ncnn::Mat& text_mat = bottom[split ? 7 : 3];
    shape_mat.create(3, batch);
    std::memcpy(shape_mat.data, shape_blob, (size_t)3 * batch * 4);
    text_mat.create(1, batch);
    std::memcpy(text_mat.data, text_blob, (size_t)batch * 4);

    std::vector<ncnn::Mat> top(2);
    ncnn::Option opt;
    ret = layer->forward(bottom, top, opt);
    if (ret == 0)
    {
        std::memcpy(video_out, top[0].data, (size_t)inner * video_tokens * sizeof(float));
        std::memcpy(text_out, top[1].data, (size_t)inner * text_tokens * sizeof(float));
    }
    delete layer;
    return ret;
}

// SharedLinear (shared_linear.cpp:27-96) through its ncnn surface.
// weights: [num_output x num_input] row-major, then bias[num_output] if bias_term.
int s2ref_shared_linear_forward(int num_output, int num_input, int bias_term, const float* weights,
                                const float* video, int video_rows, const float* text, int text_rows,
                                float* video_out, float* text_out)
{
    ncnn::Layer* layer = seedvr2::shared_linear_layer_creator(0);
    ncnn::ParamDict pd;
    pd.set(0, num_output);
    pd.set(1, num_input);
    pd.set(2, bias_term);
    int ret = layer->load_param(pd);
    if (ret == 0)
    {
        const size_t count = (size_t)num_output * num_input + (bias_term ? (size_t)num_output : 0);
        ncnn::ModelBinFromFloats mb(weights, count);
        ret = layer->load_model(mb);
    }
    if (ret != 0)
    {
        delete layer;
        return ret;
    }
    std::vector<ncnn::Mat> bottom(2);
    bottom[0].create(num_input, video_rows);
    std::memcpy(bottom[0].data, video, (size_t)num_input * video_rows * sizeof(float));
    bottom[1].create(num_input, text_rows);
    std::memcpy(bottom[1].data, text, (size_t)num_input * text_rows * sizeof(float));
    std::vector<ncnn::Mat> top(2);
    ncnn::Option opt;
    ret = layer->forward(bottom, top, opt);
    if (ret == 0)
    {
        std::memcpy(video_out, top[0].data, (size_t)num_output * video_rows * sizeof(float));
        std::memcpy(text_out, top[1].data, (size_t)num_output * text_rows * sizeof(float));
    }
    delete layer;
    return ret;
}

} // extern "C"
