// extern "C" driver of the ncnn-surface layers (libseedvr2_ncnn.so): builds a
// layer through its creator, feeds load_param / load_model exactly as ncnn's
// Net would, and runs forward() on host blobs.  It exists so that callers
// without a C++ toolchain (ctypes, tests) can exercise the same layer surface
// the reference's block graph uses.  Argument order matches the oracle's
// reference driver, so parity tests call both the same way.
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "net.h"
#include "shared_linear.h"
#include "vae_layers.h"

using seedvr2::AdaptiveWindowAttention;

namespace {

ncnn::Mat vec(const float* p, int n)
{
    ncnn::Mat m(n);
    std::memcpy(m.data, p, (size_t)n * 4);
    return m;
}

// ModelBin over one flat fp32 array, as ncnn's reads a .bin: load(w, type)
// hands out the next w values, or an empty Mat when fewer are left.  Both
// types read raw fp32 (type 0's tag word is not part of these arrays).
class FloatModelBin : public ncnn::ModelBin
{
public:
    FloatModelBin(const float* data, size_t count) : data(data), count(count) {}
    virtual ncnn::Mat load(int w, int type) const
    {
        if ((type != 0 && type != 1) || w <= 0 || cursor + (size_t)w > count) return ncnn::Mat();
        ncnn::Mat m = vec(data + cursor, w);
        cursor += (size_t)w;
        return m;
    }

private:
    const float* data;
    size_t count;
    mutable size_t cursor = 0;
};

// [c][d][h][w] dense floats <-> a 4-D Mat (channel steps padded to 16 bytes)
ncnn::Mat blob_4d(const float* p, int w, int h, int d, int c)
{
    ncnn::Mat m(w, h, d, c);
    const size_t plane = (size_t)w * h * d;
    for (int ch = 0; ch < c; ch++) std::memcpy((float*)m.data + m.cstep * ch, p + plane * ch, plane * 4);
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

// VAE layers, built the way ncnn's Net builds them: kind 0 DecomposedConv3D
// (its 16 config values also go through load_param ids 0-15), 1
// VAEDownsample3D, 2 VAEUpsample3D; blob = the floats the layer's load_model
// reads.  Returns the first nonzero code of load_param / load_model /
// create_pipeline, else 0 with the layer in *out.
int s2layer_vae_create(int kind, const float* blob, size_t count, void** out)
{
    *out = nullptr;
    ncnn::Layer* layer = kind == 0   ? seedvr2::decomposed_conv3d_layer_creator(nullptr)
                         : kind == 1 ? seedvr2::vae_downsample3d_layer_creator(nullptr)
                         : kind == 2 ? seedvr2::vae_upsample3d_layer_creator(nullptr)
                                     : nullptr;
    if (!layer) return -1;
    int ret = 0;
    if (kind == 0 && count >= 16)
    {
        ncnn::ParamDict pd;
        for (int i = 0; i < 16; i++) pd.set(i, (int)blob[i]);
        ret = layer->load_param(pd);
    }
    if (ret == 0) ret = layer->load_model(FloatModelBin(blob, count));
    ncnn::Option opt;
    if (ret == 0) ret = layer->create_pipeline(opt);
    if (ret != 0)
    {
        delete layer;
        return ret;
    }
    *out = layer;
    return 0;
}

// One forward under the given memory state (0 disabled, 1 initializing, 2
// active): in dense [c][d][h][w] fp32, out dense [c][d][h][w] of at most
// out_capacity floats, out_dims = (w, h, d, c).  Returns the layer's code.
int s2layer_vae_forward(void* handle, int memory_state, const float* in, int w, int h, int d, int c, float* out,
                        size_t out_capacity, int* out_dims)
{
    const ncnn::Layer* layer = static_cast<const ncnn::Layer*>(handle);
    seedvr2::set_vae_memory_state(static_cast<seedvr2::MemoryState>(memory_state));
    ncnn::Mat top;
    ncnn::Option opt;
    const int r = layer->forward(blob_4d(in, w, h, d, c), top, opt);
    if (r != 0) return r;
    out_dims[0] = top.w;
    out_dims[1] = top.h;
    out_dims[2] = top.d;
    out_dims[3] = top.c;
    const size_t plane = (size_t)top.w * top.h * top.d;
    if (plane * top.c > out_capacity) return -1;
    for (int ch = 0; ch < top.c; ch++) std::memcpy(out + plane * ch, (const float*)top.data + top.cstep * ch, plane * 4);
    return 0;
}

// Output extents (w, h, d, c) of a forward on a w x h x d input under the
// given memory state (uploads the weights on first use).
int s2layer_vae_output_shape(void* handle, int memory_state, int w, int h, int d, int* out_whdc)
{
    const ncnn::Layer* layer = static_cast<const ncnn::Layer*>(handle);
    seedvr2::set_vae_memory_state(static_cast<seedvr2::MemoryState>(memory_state));
    if (auto* l = dynamic_cast<const seedvr2::DecomposedConv3D*>(layer)) return l->output_shape(w, h, d, out_whdc);
    if (auto* l = dynamic_cast<const seedvr2::VAEDownsample3D*>(layer)) return l->output_shape(w, h, d, out_whdc);
    if (auto* l = dynamic_cast<const seedvr2::VAEUpsample3D*>(layer)) return l->output_shape(w, h, d, out_whdc);
    return -1;
}

// reset_temporal_memory of a layer from s2layer_vae_create.
void s2layer_vae_reset(void* handle)
{
    const ncnn::Layer* layer = static_cast<const ncnn::Layer*>(handle);
    if (auto* l = dynamic_cast<const seedvr2::DecomposedConv3D*>(layer)) l->reset_temporal_memory();
    if (auto* l = dynamic_cast<const seedvr2::VAEDownsample3D*>(layer)) l->reset_temporal_memory();
    if (auto* l = dynamic_cast<const seedvr2::VAEUpsample3D*>(layer)) l->reset_temporal_memory();
}

void s2layer_vae_free(void* handle)
{
    delete static_cast<ncnn::Layer*>(handle);
}

// VAEChunkedMHA: ip = embed_dim, num_heads, weight_data_size, kdim, vdim,
// chunk_size (param ids 0-4 and 20), scale = param 6; weights in load_model
// order (q w, q b, k w, k b, v w, v b, out w, out b).  Same return
// convention as s2layer_vae_create.
int s2layer_mha_create(const int* ip, float scale, const float* weights, size_t count, void** out)
{
    *out = nullptr;
    ncnn::Layer* layer = seedvr2::vae_chunked_mha_layer_creator(nullptr);
    ncnn::ParamDict pd;
    pd.set(0, ip[0]);
    pd.set(1, ip[1]);
    pd.set(2, ip[2]);
    pd.set(3, ip[3]);
    pd.set(4, ip[4]);
    pd.set(6, scale);
    pd.set(20, ip[5]);
    int ret = layer->load_param(pd);
    if (ret == 0) ret = layer->load_model(FloatModelBin(weights, count));
    ncnn::Option opt;
    if (ret == 0) ret = layer->create_pipeline(opt);
    if (ret != 0)
    {
        delete layer;
        return ret;
    }
    *out = layer;
    return 0;
}

// x [tokens][qdim] -> out [tokens][qdim] through forward(Mat).
int s2layer_mha_forward(void* handle, const float* x, int tokens, int qdim, float* out)
{
    const ncnn::Layer* layer = static_cast<const ncnn::Layer*>(handle);
    ncnn::Mat bottom(qdim, tokens);
    std::memcpy(bottom.data, x, (size_t)qdim * tokens * 4);
    ncnn::Mat top;
    ncnn::Option opt;
    const int r = layer->forward(bottom, top, opt);
    if (r != 0) return r;
    std::memcpy(out, top.data, (size_t)top.w * top.h * 4);
    return 0;
}

// ---------------------------------------------------------------- graph
// A block graph read from ncnn .param / .bin files with SeedVR2's two custom
// layers registered the way seedvr2_dit.cpp:614-618 registers them
// (AdaptiveWindowAttention with the caller-mutated runtime state as its
// userdata, SharedLinear), run on device blobs by name.
struct S2Net
{
    seedvr2::Net net;
    seedvr2::AdaptiveWindowRuntimeState state;
};

void* s2net_create(void)
{
    S2Net* h = new S2Net;
    h->net.register_custom_layer("AdaptiveWindowAttention", seedvr2::adaptive_window_attention_layer_creator, 0,
                                 &h->state);
    h->net.register_custom_layer("SharedLinear", seedvr2::shared_linear_layer_creator);
    return h;
}

void s2net_destroy(void* h)
{
    delete static_cast<S2Net*>(h);
}

int s2net_load(void* h, const char* param_path, const char* bin_path)
{
    if (!h) return -1;
    S2Net* n = static_cast<S2Net*>(h);
    const int r = n->net.load_param(param_path);
    return r != 0 ? r : n->net.load_model(bin_path);
}

int s2net_info(void* h, int* layers, int* blobs)
{
    if (!h || !layers || !blobs) return -1;
    S2Net* n = static_cast<S2Net*>(h);
    *layers = n->net.layer_count();
    *blobs = n->net.blob_count();
    return 0;
}

// The runtime state read by the attention layers at the next extract
// (seedvr2_dit.cpp:724-725 sets it before each extract).
int s2net_set_runtime(void* h, const int* shapes, const int* text_lengths, int batch)
{
    if (!h || !shapes || !text_lengths || batch <= 0) return -1;
    S2Net* n = static_cast<S2Net*>(h);
    n->state.video_shapes.assign(batch, {0, 0, 0});
    n->state.text_lengths.assign(text_lengths, text_lengths + batch);
    for (int b = 0; b < batch; b++)
        n->state.video_shapes[b] = {shapes[3 * b], shapes[3 * b + 1], shapes[3 * b + 2]};
    return 0;
}

// Inputs: fp32 device blobs [rows][cols] by name; outputs: each named blob
// is computed and copied into the caller's fp32 device buffer of the given
// shape (-1 on a shape mismatch).  Synchronous.
int s2net_extract_cuda(void* h, int n_in, const char* const* in_names, void* const* in_ptrs, const int* in_rows,
                       const int* in_cols, int n_out, const char* const* out_names, void* const* out_ptrs,
                       const int* out_rows, const int* out_cols)
{
    if (!h || n_in < 0 || n_out <= 0) return -1;
    S2Net* n = static_cast<S2Net*>(h);
    seedvr2::Extractor ex = n->net.create_extractor();
    for (int i = 0; i < n_in; i++)
    {
        seedvr2::CudaBlob b;
        b.data = in_ptrs[i];
        b.w = in_cols[i];
        b.h = in_rows[i];
        b.ld = in_cols[i];
        b.dtype = S2_DTYPE_F32;
        const int r = ex.input_cuda(in_names[i], b);
        if (r != 0) return r;
    }
    for (int i = 0; i < n_out; i++)
    {
        seedvr2::CudaBlob b;
        int r = ex.extract_cuda(out_names[i], b);
        if (r != 0) return r;
        if (b.w != out_cols[i] || b.h != out_rows[i]) return -1;
        if ((r = s2_status(seedvr2::layer_context())) != 0) return r;
        if (cudaMemcpy(out_ptrs[i], b.data, (size_t)b.w * b.h * 4, cudaMemcpyDeviceToDevice) != cudaSuccess)
            return S2_ERR_CUDA;
    }
    return 0;
}

} // extern "C"
