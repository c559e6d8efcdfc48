// extern "C" driver of the ncnn-surface layers (libseedvr2_ncnn.so): builds a
// layer through its creator, feeds load_param / load_model exactly as ncnn's
// Net would, and runs forward() on host blobs.  It exists so that callers
// without a C++ toolchain (ctypes, tests) can exercise the same layer surface
// the reference's block graph uses.  Argument order matches the oracle's
// reference driver, so parity tests call both the same way.
#include <cstring>
#include <vector>

#include "shared_linear.h"

using seedvr2::AdaptiveWindowAttention;

namespace {

ncnn::Mat vec(const float* p, int n)
{
    ncnn::Mat m(n);
    std::memcpy(m.data, p, (size_t)n * 4);
    return m;
}

} // namespace

extern "C" {

// params: heads, head_dim, window0..2, shifted, rope_pairs, shared_norm,
// shape_values_int32, official_bf16_attention (10 ints) + epsilon; weights
// concatenated in load_model order; split=0: inputs[0..1] = video_qkv,
// text_qkv; split=1: inputs[0..5] = vq, vk, vv, tq, tk, tv.  shape_blob
// [batch][3] and text_blob [batch] as floats (or int32 bits).
int s2layer_awa_forward(const int* params, float epsilon, const float* weights, int num_weights, int split,
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
    ncnn::Layer* layer = seedvr2::adaptive_window_attention_layer_creator(nullptr);
    int ret = layer->load_param(pd);
    const int hd = params[1], pairs = params[6];
    const int n_norm = params[7] ? 2 : 4;
    if (ret == 0 && num_weights != n_norm * hd + pairs) ret = -1;
    if (ret == 0)
    {
        std::vector<ncnn::Mat> w;
        for (int i = 0; i < n_norm; i++) w.push_back(vec(weights + (size_t)i * hd, hd));
        w.push_back(vec(weights + (size_t)n_norm * hd, pairs));
        ret = layer->load_model(ncnn::ModelBinFromMatArray(w.data()));
    }
    if (ret != 0)
    {
        delete layer;
        return ret;
    }
    const int inner = params[0] * hd;
    std::vector<ncnn::Mat> bottom(split ? 8 : 4);
    if (split)
        for (int p = 0; p < 6; p++)
        {
            const int rows = p < 3 ? video_tokens : text_tokens;
            bottom[p].create(inner, rows);
            std::memcpy(bottom[p].data, inputs[p], (size_t)inner * rows * 4);
        }
    else
    {
        bottom[0].create(inner * 3, video_tokens);
        std::memcpy(bottom[0].data, inputs[0], (size_t)inner * 3 * video_tokens * 4);
        bottom[1].create(inner * 3, text_tokens);
        std::memcpy(bottom[1].data, inputs[1], (size_t)inner * 3 * text_tokens * 4);
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
        std::memcpy(video_out, top[0].data, (size_t)inner * video_tokens * 4);
        std::memcpy(text_out, top[1].data, (size_t)inner * text_tokens * 4);
    }
    delete layer;
    return ret;
}

// weights: [num_output][num_input] then bias[num_output] when bias_term.
int s2layer_shared_linear_forward(int num_output, int num_input, int bias_term, const float* weights,
                                  const float* video, int video_rows, const float* text, int text_rows,
                                  float* video_out, float* text_out)
{
    ncnn::Layer* layer = seedvr2::shared_linear_layer_creator(nullptr);
    ncnn::ParamDict pd;
    pd.set(0, num_output);
    pd.set(1, num_input);
    pd.set(2, bias_term);
    int ret = layer->load_param(pd);
    if (ret == 0)
    {
        ncnn::Mat w[2];
        w[0] = vec(weights, num_output * num_input);
        if (bias_term) w[1] = vec(weights + (size_t)num_output * num_input, num_output);
        ret = layer->load_model(ncnn::ModelBinFromMatArray(w));
    }
    if (ret != 0)
    {
        delete layer;
        return ret;
    }
    std::vector<ncnn::Mat> bottom(2), top(2);
    bottom[0].create(num_input, video_rows);
    std::memcpy(bottom[0].data, video, (size_t)num_input * video_rows * 4);
    bottom[1].create(num_input, text_rows);
    std::memcpy(bottom[1].data, text, (size_t)num_input * text_rows * 4);
    ncnn::Option opt;
    ret = layer->forward(bottom, top, opt);
    if (ret == 0)
    {
        std::memcpy(video_out, top[0].data, (size_t)num_output * video_rows * 4);
        std::memcpy(text_out, top[1].data, (size_t)num_output * text_rows * 4);
    }
    delete layer;
    return ret;
}

} // extern "C"
