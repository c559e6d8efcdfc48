// The VAE layers on libseedvr2_cuda (see the header).  load_param /
// load_model restate the reference's own checks and load sequence
// (decomposed_conv3d.cpp:399-478, vae_downsample3d.cpp:98-112,
// vae_upsample3d.cpp:191-213, vae_chunked_mha.cpp:109-140); forward checks
// the blob as the reference's CPU forward does (decomposed_conv3d.cpp:605-622,
// vae_downsample3d.cpp:145-152, vae_upsample3d.cpp:258-265,
// vae_chunked_mha.cpp:197-203) and runs the device layer.
#include "vae_layers.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>

namespace seedvr2 {

namespace {

thread_local MemoryState current_memory_state = MemoryState::DISABLED;

int abi_state(MemoryState s)
{
    switch (s)
    {
    case MemoryState::ACTIVE:
        return S2_VAE_MEMORY_ACTIVE;
    case MemoryState::INITIALIZING:
        return S2_VAE_MEMORY_INITIALIZING;
    default:
        return S2_VAE_MEMORY_DISABLED;
    }
}

size_t align256(size_t x)
{
    return (x + 255) & ~size_t(255);
}

// Grow-only device staging of the host-blob forwards, one per thread.
struct Staging
{
    void* ptr = nullptr;
    size_t bytes = 0;
    ~Staging()
    {
        if (ptr) cudaFree(ptr);
    }
    uint8_t* get(size_t n)
    {
        if (n > bytes)
        {
            if (ptr) cudaFree(ptr);
            ptr = nullptr;
            bytes = 0;
            if (cudaMalloc(&ptr, n) != cudaSuccess)
            {
                ptr = nullptr;
                return nullptr;
            }
            bytes = n;
        }
        return static_cast<uint8_t*>(ptr);
    }
};

Staging& staging()
{
    static thread_local Staging s;
    return s;
}

// Host fp32 blob -> device, run(in, in_cstep, out, out_cstep), device -> host.
// `top` is already created; both blobs keep their channel steps on the device.
template <class Run>
int run_on_device(const ncnn::Mat& bottom, ncnn::Mat& top, Run run)
{
    const size_t in_bytes = bottom.cstep * bottom.c * 4, out_bytes = top.cstep * top.c * 4;
    uint8_t* buf = staging().get(align256(in_bytes) + out_bytes);
    if (!buf) return -100;
    float* din = reinterpret_cast<float*>(buf);
    float* dout = reinterpret_cast<float*>(buf + align256(in_bytes));
    if (cudaMemcpy(din, bottom.data, in_bytes, cudaMemcpyHostToDevice) != cudaSuccess) return S2_ERR_CUDA;
    int r = run(din, (int64_t)bottom.cstep, dout, (int64_t)top.cstep);
    if (r == S2_OK) r = s2_status(layer_context());
    if (r == S2_OK && cudaMemcpy(top.data, dout, out_bytes, cudaMemcpyDeviceToHost) != cudaSuccess) r = S2_ERR_CUDA;
    return r;
}

const float* floats(const ncnn::Mat& m)
{
    return static_cast<const float*>(m.data);
}

} // namespace

MemoryState get_vae_memory_state()
{
    return current_memory_state;
}

void set_vae_memory_state(MemoryState state)
{
    current_memory_state = state;
}

// ---------------------------------------------------------------- DecomposedConv3D

DecomposedConv3D::DecomposedConv3D()
    : num_output(0), num_input(0), kernel_w(0), kernel_h(0), kernel_t(0), stride_t(1), dilation_t(1),
      head_frames(0), stride_w(1), stride_h(1), dilation_w(1), dilation_h(1), pad_w(0), pad_h(0), groups(1),
      bias_term(false), device_layer(nullptr)
{
    one_blob_only = true;
    support_inplace = false;
}

DecomposedConv3D::~DecomposedConv3D()
{
    s2_conv3d_free(device_layer);
}

int DecomposedConv3D::load_param(const ncnn::ParamDict& pd)
{
    num_output = pd.get(0, 0);
    num_input = pd.get(1, 0);
    kernel_w = pd.get(2, 0);
    kernel_h = pd.get(3, 0);
    kernel_t = pd.get(4, 0);
    stride_t = pd.get(5, 1);
    dilation_t = pd.get(6, 1);
    head_frames = pd.get(7, 0);
    stride_w = pd.get(8, 1);
    stride_h = pd.get(9, 1);
    dilation_w = pd.get(10, 1);
    dilation_h = pd.get(11, 1);
    pad_w = pd.get(12, 0);
    pad_h = pd.get(13, 0);
    groups = pd.get(14, 1);
    bias_term = pd.get(15, 0) != 0;
    return 0;
}

int DecomposedConv3D::load_model(const ncnn::ModelBin& mb)
{
    s2_conv3d_free(device_layer);
    device_layer = nullptr;
    spatial_weights.clear();
    bias_data = ncnn::Mat();
    const ncnn::Mat config = mb.load(16, 1);
    if (config.empty()) return -100;
    const float* v = floats(config);
    num_output = (int)v[0];
    num_input = (int)v[1];
    kernel_w = (int)v[2];
    kernel_h = (int)v[3];
    kernel_t = (int)v[4];
    stride_t = (int)v[5];
    dilation_t = (int)v[6];
    head_frames = (int)v[7];
    stride_w = (int)v[8];
    stride_h = (int)v[9];
    dilation_w = (int)v[10];
    dilation_h = (int)v[11];
    pad_w = (int)v[12];
    pad_h = (int)v[13];
    groups = (int)v[14];
    bias_term = (int)v[15] != 0;
    if (num_output <= 0 || num_input <= 0 || kernel_w <= 0 || kernel_h <= 0 || kernel_t <= 0 || stride_t <= 0 ||
        dilation_t <= 0 || stride_w <= 0 || stride_h <= 0 || dilation_w <= 0 || dilation_h <= 0 || groups <= 0 ||
        num_input % groups != 0 || num_output % groups != 0 || head_frames < 0)
        return -1;
    if (bias_term)
    {
        bias_data = mb.load(num_output, 1);
        if (bias_data.empty()) return -100;
    }
    const int weight_data_size = num_output * (num_input / groups) * kernel_w * kernel_h;
    spatial_weights.reserve(kernel_t);
    for (int t = 0; t < kernel_t; t++)
    {
        ncnn::Mat weight = mb.load(weight_data_size, 1);
        if (weight.empty()) return -100;
        // the reference's per-frame spatial Convolution rejects negative
        // pads (ncnn's "same" modes, which the exporter never writes) in its
        // load_param
        if (pad_w < 0 || pad_h < 0) return -1;
        spatial_weights.push_back(weight);
    }
    return 0;
}

int DecomposedConv3D::create_pipeline(const ncnn::Option&)
{
    if ((int)spatial_weights.size() != kernel_t) return -1;
    if (groups != 1 || stride_w > 2) return -1; // this build's implicit GEMM
    return 0;
}

int DecomposedConv3D::destroy_pipeline(const ncnn::Option&)
{
    s2_conv3d_free(device_layer);
    device_layer = nullptr;
    return 0;
}

void DecomposedConv3D::release_completed_temporal_memory() const {}

void DecomposedConv3D::reset_temporal_memory() const
{
    s2_conv3d_reset_memory(device_layer);
}

void DecomposedConv3D::append_model(std::vector<float>& blob) const
{
    const float cfg[16] = {(float)num_output, (float)num_input,  (float)kernel_w,   (float)kernel_h,
                           (float)kernel_t,   (float)stride_t,   (float)dilation_t, (float)head_frames,
                           (float)stride_w,   (float)stride_h,   (float)dilation_w, (float)dilation_h,
                           (float)pad_w,      (float)pad_h,      (float)groups,     bias_term ? 1.f : 0.f};
    blob.insert(blob.end(), cfg, cfg + 16);
    if (bias_term) blob.insert(blob.end(), floats(bias_data), floats(bias_data) + num_output);
    for (const ncnn::Mat& w : spatial_weights) blob.insert(blob.end(), floats(w), floats(w) + w.w);
}

int DecomposedConv3D::upload() const
{
    if (device_layer) return 0;
    if ((int)spatial_weights.size() != kernel_t || kernel_t <= 0) return -1;
    s2_context* ctx = layer_context();
    if (!ctx) return S2_ERR_DEVICE;
    std::vector<float> blob;
    append_model(blob);
    const int cfg[16] = {num_output, num_input,  kernel_w,   kernel_h,   kernel_t, stride_t, dilation_t, head_frames,
                         stride_w,   stride_h,   dilation_w, dilation_h, pad_w,    pad_h,    groups,     bias_term};
    const size_t weights_at = 16 + (bias_term ? (size_t)num_output : 0);
    return s2_conv3d_create(ctx, cfg, bias_term ? blob.data() + 16 : nullptr, blob.data() + weights_at,
                            &device_layer);
}

int DecomposedConv3D::output_shape(int w, int h, int d, int* out_whdc) const
{
    int r = upload();
    if (r != 0) return r;
    return s2_conv3d_output_shape(device_layer, w, h, d, abi_state(get_vae_memory_state()), out_whdc);
}

int DecomposedConv3D::forward_cuda(const float* in, int64_t in_cstep, int w, int h, int d, float* out,
                                   int64_t out_cstep) const
{
    int r = upload();
    if (r != 0) return r;
    return s2_conv3d_forward(device_layer, in, in_cstep, w, h, d, num_input, abi_state(get_vae_memory_state()),
                             out, out_cstep);
}

int DecomposedConv3D::forward(const ncnn::Mat& bottom_blob, ncnn::Mat& top_blob, const ncnn::Option& opt) const
{
    const MemoryState state = get_vae_memory_state();
    if (state != MemoryState::ACTIVE) s2_conv3d_reset_memory(device_layer);
    if (bottom_blob.dims != 4 || bottom_blob.c * bottom_blob.elempack != num_input || bottom_blob.n != 1 ||
        (int)spatial_weights.size() != kernel_t)
        return -1;
    if (bottom_blob.elempack != 1 || bottom_blob.elemsize != 4) return -1; // host fp32 blobs
    int r = upload();
    if (r != 0) return r;
    const int st = abi_state(state);
    int whdc[4];
    if ((r = s2_conv3d_output_shape(device_layer, bottom_blob.w, bottom_blob.h, bottom_blob.d, st, whdc)) != 0)
        return r;
    top_blob.create(whdc[0], whdc[1], whdc[2], whdc[3], 4u, 1, 1, opt.blob_allocator);
    if (top_blob.empty()) return -100;
    return run_on_device(bottom_blob, top_blob, [&](const float* in, int64_t ic, float* out, int64_t oc) {
        return s2_conv3d_forward(device_layer, in, ic, bottom_blob.w, bottom_blob.h, bottom_blob.d, bottom_blob.c, st,
                                 out, oc);
    });
}

// ---------------------------------------------------------------- resampling layers
//
// A call rejected for its shape under a non-ACTIVE state leaves every
// convolution of the layer without cached frames; the reference's may keep or
// refresh some of them, depending on which convolution's check failed.

namespace {

int resample_forward(s2_vae_resample* layer, const ncnn::Mat& bottom_blob, ncnn::Mat& top_blob,
                     const ncnn::Option& opt)
{
    const int st = abi_state(get_vae_memory_state());
    int whdc[4];
    int r = s2_vae_resample_output_shape(layer, bottom_blob.w, bottom_blob.h, bottom_blob.d, st, whdc);
    if (r != 0)
    {
        if (st != S2_VAE_MEMORY_ACTIVE) s2_vae_resample_reset_memory(layer);
        return r;
    }
    top_blob.create(whdc[0], whdc[1], whdc[2], whdc[3], 4u, 1, 1, opt.blob_allocator);
    if (top_blob.empty()) return -100;
    return run_on_device(bottom_blob, top_blob, [&](const float* in, int64_t ic, float* out, int64_t oc) {
        return s2_vae_resample_forward(layer, in, ic, bottom_blob.w, bottom_blob.h, bottom_blob.d, bottom_blob.c, st,
                                       out, oc);
    });
}

} // namespace

VAEDownsample3D::VAEDownsample3D()
    : channels(0), pad_right(0), pad_bottom(0), convolution(nullptr), device_layer(nullptr)
{
    one_blob_only = true;
    support_inplace = false;
}

VAEDownsample3D::~VAEDownsample3D()
{
    s2_vae_resample_free(device_layer);
    delete convolution;
}

int VAEDownsample3D::load_model(const ncnn::ModelBin& mb)
{
    s2_vae_resample_free(device_layer);
    device_layer = nullptr;
    delete convolution;
    convolution = nullptr;
    const ncnn::Mat config = mb.load(3, 1);
    if (config.empty()) return -100;
    const float* v = floats(config);
    channels = (int)v[0];
    pad_right = (int)v[1];
    pad_bottom = (int)v[2];
    if (channels <= 0 || pad_right < 0 || pad_bottom < 0 || (pad_right == 0 && pad_bottom == 0)) return -1;
    convolution = new DecomposedConv3D;
    return convolution->load_model(mb);
}

int VAEDownsample3D::create_pipeline(const ncnn::Option& opt)
{
    return convolution ? convolution->create_pipeline(opt) : -1;
}

int VAEDownsample3D::destroy_pipeline(const ncnn::Option& opt)
{
    s2_vae_resample_free(device_layer);
    device_layer = nullptr;
    return convolution ? convolution->destroy_pipeline(opt) : 0;
}

void VAEDownsample3D::release_completed_temporal_memory() const {}

void VAEDownsample3D::reset_temporal_memory() const
{
    s2_vae_resample_reset_memory(device_layer);
}

int VAEDownsample3D::upload() const
{
    if (device_layer) return 0;
    if (!convolution) return -1;
    s2_context* ctx = layer_context();
    if (!ctx) return S2_ERR_DEVICE;
    std::vector<float> blob = {(float)channels, (float)pad_right, (float)pad_bottom};
    convolution->append_model(blob);
    return s2_vae_resample_create(ctx, S2_VAE_DOWNSAMPLE, blob.data(), blob.size(), &device_layer);
}

int VAEDownsample3D::output_shape(int w, int h, int d, int* out_whdc) const
{
    int r = upload();
    if (r != 0) return r;
    return s2_vae_resample_output_shape(device_layer, w, h, d, abi_state(get_vae_memory_state()), out_whdc);
}

int VAEDownsample3D::forward_cuda(const float* in, int64_t in_cstep, int w, int h, int d, float* out,
                                  int64_t out_cstep) const
{
    int r = upload();
    if (r != 0) return r;
    return s2_vae_resample_forward(device_layer, in, in_cstep, w, h, d, channels, abi_state(get_vae_memory_state()),
                                   out, out_cstep);
}

int VAEDownsample3D::forward(const ncnn::Mat& bottom_blob, ncnn::Mat& top_blob, const ncnn::Option& opt) const
{
    if (!convolution || bottom_blob.dims != 4 || bottom_blob.n != 1 || bottom_blob.c != channels ||
        bottom_blob.elempack != 1 || bottom_blob.elemsize != sizeof(float))
        return -1;
    const int r = upload();
    if (r != 0) return r;
    return resample_forward(device_layer, bottom_blob, top_blob, opt);
}

VAEUpsample3D::VAEUpsample3D()
    : channels(0), temporal_ratio(0), spatial_ratio(0), remove_temporal_head(false), post_conv(nullptr),
      upscale_conv(nullptr), device_layer(nullptr)
{
    one_blob_only = true;
    support_inplace = false;
}

VAEUpsample3D::~VAEUpsample3D()
{
    s2_vae_resample_free(device_layer);
    delete post_conv;
    delete upscale_conv;
}

int VAEUpsample3D::load_model(const ncnn::ModelBin& mb)
{
    s2_vae_resample_free(device_layer);
    device_layer = nullptr;
    delete post_conv;
    delete upscale_conv;
    post_conv = upscale_conv = nullptr;
    const ncnn::Mat config = mb.load(4, 1);
    if (config.empty()) return -100;
    const float* v = floats(config);
    channels = (int)v[0];
    temporal_ratio = (int)v[1];
    spatial_ratio = (int)v[2];
    remove_temporal_head = (int)v[3] != 0;
    if (channels <= 0 || (temporal_ratio != 1 && temporal_ratio != 2) || (spatial_ratio != 1 && spatial_ratio != 2) ||
        remove_temporal_head != (temporal_ratio == 2))
        return -1;
    // stored lexically: config, post conv, upscale conv
    post_conv = new DecomposedConv3D;
    upscale_conv = new DecomposedConv3D;
    int ret = post_conv->load_model(mb);
    if (ret == 0) ret = upscale_conv->load_model(mb);
    return ret;
}

int VAEUpsample3D::create_pipeline(const ncnn::Option& opt)
{
    int ret = post_conv ? post_conv->create_pipeline(opt) : -1;
    if (ret == 0) ret = upscale_conv ? upscale_conv->create_pipeline(opt) : -1;
    return ret;
}

int VAEUpsample3D::destroy_pipeline(const ncnn::Option& opt)
{
    s2_vae_resample_free(device_layer);
    device_layer = nullptr;
    if (post_conv) post_conv->destroy_pipeline(opt);
    if (upscale_conv) upscale_conv->destroy_pipeline(opt);
    return 0;
}

void VAEUpsample3D::release_completed_temporal_memory() const {}

void VAEUpsample3D::reset_temporal_memory() const
{
    s2_vae_resample_reset_memory(device_layer);
}

int VAEUpsample3D::upload() const
{
    if (device_layer) return 0;
    if (!post_conv || !upscale_conv) return -1;
    s2_context* ctx = layer_context();
    if (!ctx) return S2_ERR_DEVICE;
    std::vector<float> blob = {(float)channels, (float)temporal_ratio, (float)spatial_ratio,
                               remove_temporal_head ? 1.f : 0.f};
    post_conv->append_model(blob);
    upscale_conv->append_model(blob);
    return s2_vae_resample_create(ctx, S2_VAE_UPSAMPLE, blob.data(), blob.size(), &device_layer);
}

int VAEUpsample3D::output_shape(int w, int h, int d, int* out_whdc) const
{
    int r = upload();
    if (r != 0) return r;
    return s2_vae_resample_output_shape(device_layer, w, h, d, abi_state(get_vae_memory_state()), out_whdc);
}

int VAEUpsample3D::forward_cuda(const float* in, int64_t in_cstep, int w, int h, int d, float* out,
                                int64_t out_cstep) const
{
    int r = upload();
    if (r != 0) return r;
    return s2_vae_resample_forward(device_layer, in, in_cstep, w, h, d, channels, abi_state(get_vae_memory_state()),
                                   out, out_cstep);
}

int VAEUpsample3D::forward(const ncnn::Mat& bottom_blob, ncnn::Mat& top_blob, const ncnn::Option& opt) const
{
    if (!post_conv || !upscale_conv || bottom_blob.dims != 4 || bottom_blob.c != channels || bottom_blob.n != 1 ||
        bottom_blob.elempack != 1 || bottom_blob.elemsize != sizeof(float))
        return -1;
    const int r = upload();
    if (r != 0) return r;
    return resample_forward(device_layer, bottom_blob, top_blob, opt);
}

// ---------------------------------------------------------------- VAEChunkedMHA

VAEChunkedMHA::VAEChunkedMHA()
    : embed_dim(0), num_heads(0), weight_data_size(0), kdim(0), vdim(0), scale(0.f), chunk_size(128),
      device_layer(nullptr)
{
    one_blob_only = true;
    support_inplace = false;
}

VAEChunkedMHA::~VAEChunkedMHA()
{
    s2_vae_mha_free(device_layer);
}

int VAEChunkedMHA::load_param(const ncnn::ParamDict& pd)
{
    embed_dim = pd.get(0, 0);
    num_heads = pd.get(1, 1);
    weight_data_size = pd.get(2, 0);
    kdim = pd.get(3, embed_dim);
    vdim = pd.get(4, embed_dim);
    // the default divides by zero heads like the reference's; checked below
    scale = pd.get(6, num_heads > 0 ? 1.f / std::sqrt((float)(embed_dim / num_heads)) : 0.f);
    chunk_size = pd.get(20, 128);
    if (embed_dim <= 0 || num_heads <= 0 || embed_dim % num_heads != 0 || weight_data_size <= 0 ||
        weight_data_size % embed_dim != 0 || kdim <= 0 || vdim <= 0 || chunk_size <= 0)
        return -1;
    return 0;
}

int VAEChunkedMHA::load_model(const ncnn::ModelBin& mb)
{
    s2_vae_mha_free(device_layer);
    device_layer = nullptr;
    const int qdim = weight_data_size / embed_dim;
    weights[0] = mb.load(embed_dim * qdim, 0);
    weights[1] = mb.load(embed_dim, 1);
    weights[2] = mb.load(embed_dim * kdim, 0);
    weights[3] = mb.load(embed_dim, 1);
    weights[4] = mb.load(embed_dim * vdim, 0);
    weights[5] = mb.load(embed_dim, 1);
    weights[6] = mb.load(qdim * embed_dim, 0);
    weights[7] = mb.load(qdim, 1);
    for (const ncnn::Mat& w : weights)
        if (w.empty()) return -100;
    return 0;
}

int VAEChunkedMHA::create_pipeline(const ncnn::Option&)
{
    return supported() ? 0 : -1;
}

// Weights loaded, and this build's shape: the VAE's one head (512 wide) with
// q, k, v and out all embed_dim x embed_dim, as tensor-core GEMMs.
bool VAEChunkedMHA::supported() const
{
    for (const ncnn::Mat& w : weights)
        if (w.empty()) return false;
    return num_heads == 1 && weight_data_size == embed_dim * embed_dim && kdim == embed_dim && vdim == embed_dim &&
           embed_dim % 8 == 0;
}

int VAEChunkedMHA::destroy_pipeline(const ncnn::Option&)
{
    s2_vae_mha_free(device_layer);
    device_layer = nullptr;
    return 0;
}

int VAEChunkedMHA::upload() const
{
    if (device_layer) return 0;
    if (!supported()) return -1;
    s2_context* ctx = layer_context();
    if (!ctx) return S2_ERR_DEVICE;
    std::vector<float> blob;
    for (const ncnn::Mat& w : weights) blob.insert(blob.end(), floats(w), floats(w) + w.w);
    return s2_vae_mha_create(ctx, embed_dim, num_heads, scale, blob.data(), &device_layer);
}

int VAEChunkedMHA::forward_cuda(const float* x, int tokens, float* out) const
{
    int r = upload();
    if (r != 0) return r;
    return s2_vae_mha_forward(device_layer, x, tokens, out);
}

int VAEChunkedMHA::forward(const ncnn::Mat& bottom_blob, ncnn::Mat& top_blob, const ncnn::Option& opt) const
{
    if (bottom_blob.dims != 2 || bottom_blob.w != weight_data_size / embed_dim) return -1;
    if (bottom_blob.elempack != 1 || bottom_blob.elemsize != 4) return -1; // host fp32 rows
    int r = upload();
    if (r != 0) return r;
    top_blob.create(bottom_blob.w, bottom_blob.h, 4u, opt.blob_allocator);
    if (top_blob.empty()) return -100;
    const int tokens = bottom_blob.h;
    return run_on_device(bottom_blob, top_blob, [&](const float* in, int64_t, float* out, int64_t) {
        return s2_vae_mha_forward(device_layer, in, tokens, out);
    });
}

ncnn::Layer* decomposed_conv3d_layer_creator(void*)
{
    return new DecomposedConv3D;
}

ncnn::Layer* vae_downsample3d_layer_creator(void*)
{
    return new VAEDownsample3D;
}

ncnn::Layer* vae_upsample3d_layer_creator(void*)
{
    return new VAEUpsample3D;
}

ncnn::Layer* vae_chunked_mha_layer_creator(void*)
{
    return new VAEChunkedMHA;
}

} // namespace seedvr2
