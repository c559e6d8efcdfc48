// extern "C" wrapper around the reference's OWN VAE layers DecomposedConv3D,
// VAEDownsample3D, VAEUpsample3D and VAEChunkedMHA
// (src/seedvr2/decomposed_conv3d.cpp, vae_downsample3d.cpp,
// vae_upsample3d.cpp, vae_chunked_mha.cpp, compiled unmodified with
// NCNN_VULKAN=0 against the clean-room ncnn shim, whose "Convolution"
// restates ncnn's spatial convolution).  Built by oracle/Makefile into
// oracle/_ref/libs2_ref_vae.so.
//
// TEST INFRASTRUCTURE ONLY: the tests and the fixture generator load it as the
// checker; the shipped library never links it.
#include <cstring>
#include <vector>

#include "decomposed_conv3d.h"
#include "modelbin.h"
#include "vae_chunked_mha.h"
#include "vae_downsample3d.h"
#include "vae_upsample3d.h"

using seedvr2::DecomposedConv3D;

extern "C" {

// cfg[16]: the layer's config blob in load_model order (num_output, num_input,
// kernel_w, kernel_h, kernel_t, stride_t, dilation_t, head_frames, stride_w,
// stride_h, dilation_w, dilation_h, pad_w, pad_h, groups, bias_term);
// weights: bias [num_output] when bias_term, then kernel_t spatial kernels
// [num_output][num_input][kernel_h][kernel_w].  Returns a layer handle or 0.
void* s2ref_conv3d_create(const float* cfg, const float* weights, size_t count)
{
    DecomposedConv3D* layer = new DecomposedConv3D;
    ncnn::ParamDict pd;
    for (int i = 0; i < 16; i++) pd.set(i, (int)cfg[i]);
    if (layer->load_param(pd) != 0)
    {
        delete layer;
        return 0;
    }
    std::vector<float> blob(cfg, cfg + 16);
    blob.insert(blob.end(), weights, weights + count);
    ncnn::ModelBinFromFloats mb(blob.data(), blob.size());
    ncnn::Option opt;
    if (layer->load_model(mb) != 0 || layer->create_pipeline(opt) != 0)
    {
        delete layer;
        return 0;
    }
    return layer;
}

// One forward: in dense [c][d][h][w] fp32 under the given memory state
// (0 disabled, 1 initializing, 2 active); out dense [c][d][h][w] of at most
// out_capacity floats, out_dims = (w, h, d, c).  Returns the layer's code.
int s2ref_conv3d_forward(void* handle, int memory_state, const float* in, int w, int h, int d, int c, float* out,
                         size_t out_capacity, int* out_dims)
{
    const DecomposedConv3D* layer = static_cast<const DecomposedConv3D*>(handle);
    seedvr2::set_vae_memory_state(static_cast<seedvr2::MemoryState>(memory_state));
    ncnn::Mat bottom(w, h, d, c, 4u, 1, 1);
    const size_t plane = (size_t)w * h * d;
    for (int ch = 0; ch < c; ch++) std::memcpy(bottom.channel(ch).data, in + plane * ch, plane * sizeof(float));
    ncnn::Mat top;
    ncnn::Option opt;
    const int r = layer->forward(bottom, top, opt);
    if (r != 0) return r;
    out_dims[0] = top.w;
    out_dims[1] = top.h;
    out_dims[2] = top.d;
    out_dims[3] = top.c;
    const size_t oplane = (size_t)top.w * top.h * top.d;
    if (oplane * top.c > out_capacity) return -1;
    for (int ch = 0; ch < top.c; ch++) std::memcpy(out + oplane * ch, top.channel(ch).data, oplane * sizeof(float));
    return 0;
}

void s2ref_conv3d_free(void* handle)
{
    delete static_cast<DecomposedConv3D*>(handle);
}

// VAEDownsample3D (kind 0) or VAEUpsample3D (kind 1) from the weight blob
// sequence its load_model reads (config values, then each DecomposedConv3D's
// config, bias and kernels).  Returns a layer handle or 0.
void* s2ref_resample_create(int kind, const float* blob, size_t count)
{
    ncnn::Layer* layer = kind == 0 ? static_cast<ncnn::Layer*>(new seedvr2::VAEDownsample3D)
                                   : static_cast<ncnn::Layer*>(new seedvr2::VAEUpsample3D);
    ncnn::ModelBinFromFloats mb(blob, count);
    ncnn::Option opt;
    if (layer->load_model(mb) != 0 || layer->create_pipeline(opt) != 0)
    {
        delete layer;
        return 0;
    }
    return layer;
}

int s2ref_resample_forward(void* handle, int memory_state, const float* in, int w, int h, int d, int c, float* out,
                           size_t out_capacity, int* out_dims)
{
    const ncnn::Layer* layer = static_cast<const ncnn::Layer*>(handle);
    seedvr2::set_vae_memory_state(static_cast<seedvr2::MemoryState>(memory_state));
    ncnn::Mat bottom(w, h, d, c, 4u, 1, 1);
    const size_t plane = (size_t)w * h * d;
    for (int ch = 0; ch < c; ch++) std::memcpy(bottom.channel(ch).data, in + plane * ch, plane * sizeof(float));
    ncnn::Mat top;
    ncnn::Option opt;
    const int r = layer->forward(bottom, top, opt);
    if (r != 0) return r;
    out_dims[0] = top.w;
    out_dims[1] = top.h;
    out_dims[2] = top.d;
    out_dims[3] = top.c;
    const size_t oplane = (size_t)top.w * top.h * top.d;
    if (oplane * top.c > out_capacity) return -1;
    for (int ch = 0; ch < top.c; ch++) std::memcpy(out + oplane * ch, top.channel(ch).data, oplane * sizeof(float));
    return 0;
}

void s2ref_resample_free(void* handle)
{
    delete static_cast<ncnn::Layer*>(handle);
}

// The load-time codes of one layer, built the way ncnn's Net builds it: kind 0
// DecomposedConv3D (its 16 config values also go through load_param ids
// 0-15), 1 VAEDownsample3D, 2 VAEUpsample3D; blob = the floats load_model
// reads.  Returns the first nonzero code of load_param / load_model /
// create_pipeline, else 0.
int s2ref_vae_load(int kind, const float* blob, size_t count)
{
    ncnn::Layer* layer = kind == 0   ? static_cast<ncnn::Layer*>(new DecomposedConv3D)
                         : kind == 1 ? static_cast<ncnn::Layer*>(new seedvr2::VAEDownsample3D)
                                     : static_cast<ncnn::Layer*>(new seedvr2::VAEUpsample3D);
    int r = 0;
    if (kind == 0 && count >= 16)
    {
        ncnn::ParamDict pd;
        for (int i = 0; i < 16; i++) pd.set(i, (int)blob[i]);
        r = layer->load_param(pd);
    }
    ncnn::ModelBinFromFloats mb(blob, count);
    ncnn::Option opt;
    if (r == 0) r = layer->load_model(mb);
    if (r == 0) r = layer->create_pipeline(opt);
    delete layer;
    return r;
}

// VAEChunkedMHA: params (embed_dim, num_heads, weight_data_size, kdim, vdim,
// scale, chunk_size), weights in load_model order (q w, q b, k w, k b, v w,
// v b, out w, out b).  x [tokens][qdim] -> out [tokens][qdim].
int s2ref_mha_forward(const int* ip, float scale, const float* weights, size_t count, const float* x, int tokens,
                      float* out)
{
    seedvr2::VAEChunkedMHA layer;
    ncnn::ParamDict pd;
    pd.set(0, ip[0]);
    pd.set(1, ip[1]);
    pd.set(2, ip[2]);
    pd.set(3, ip[3]);
    pd.set(4, ip[4]);
    pd.set(6, scale);
    pd.set(20, ip[5]);
    int r = layer.load_param(pd);
    ncnn::ModelBinFromFloats mb(weights, count);
    ncnn::Option opt;
    if (r == 0) r = layer.load_model(mb);
    if (r == 0) r = layer.create_pipeline(opt);
    if (r != 0) return r;
    const int qdim = ip[2] / ip[0];
    ncnn::Mat bottom(qdim, tokens);
    std::memcpy(bottom.data, x, sizeof(float) * (size_t)qdim * tokens);
    ncnn::Mat top;
    r = layer.forward(bottom, top, opt);
    if (r != 0) return r;
    std::memcpy(out, top.data, sizeof(float) * (size_t)qdim * tokens);
    return 0;
}

} // extern "C"
