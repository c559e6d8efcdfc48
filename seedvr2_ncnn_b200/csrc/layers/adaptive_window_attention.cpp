// AdaptiveWindowAttention on libseedvr2_cuda (see the header).  Validation
// and error codes follow AdaptiveWindowAttention::forward of the reference
// (src/seedvr2/adaptive_window_attention.cpp:764-831, Vulkan :1059-1114).
#include "adaptive_window_attention.h"

#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

namespace seedvr2 {

namespace {

std::mutex g_ctx_mutex;
s2_context* g_ctx = nullptr;

int read_shape_value(const ncnn::Mat& values, int row, int column, bool int32_values)
{
    const float* base = values.dims == 1 ? static_cast<const float*>(values.data) : values.row(row);
    if (int32_values)
    {
        int v;
        std::memcpy(&v, base + column, sizeof(int));
        return v;
    }
    return static_cast<int>(base[column]);
}

// Grow-only device buffer.
struct Scratch
{
    void* ptr = nullptr;
    size_t bytes = 0;
    void* get(size_t want)
    {
        if (want <= bytes) return ptr;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
        if (cudaMalloc(&ptr, want) != cudaSuccess) return nullptr;
        bytes = want;
        return ptr;
    }
};

} // namespace

s2_context* layer_context()
{
    std::lock_guard<std::mutex> lock(g_ctx_mutex);
    if (!g_ctx)
    {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
        if (s2_init(dev, nullptr, &g_ctx) != S2_OK) g_ctx = nullptr;
    }
    return g_ctx;
}

int build_adaptive_window_plan(const std::vector<std::array<int, 3> >& video_shapes,
                               const std::array<int, 3>& target_windows, bool shifted, AdaptiveWindowPlan& plan)
{
    plan = AdaptiveWindowPlan();
    std::vector<int> flat;
    for (const auto& s : video_shapes) flat.insert(flat.end(), s.begin(), s.end());
    s2_plan* p = nullptr;
    int r = s2_plan_build(flat.data(), static_cast<int>(video_shapes.size()), target_windows.data(),
                          S2_WINDOW_TARGET, shifted ? 1 : 0, &p);
    if (r != S2_OK) return r;
    int nw = 0, nt = 0, mx = 0;
    s2_plan_info(p, &nw, &nt, &mx);
    std::vector<int> win(9 * (size_t)nw), pos(3 * (size_t)nt);
    plan.sample_window_count.resize(video_shapes.size());
    plan.video_indices.resize(nt);
    plan.inverse_video_indices.resize(nt);
    s2_plan_copy(p, win.data(), plan.sample_window_count.data(), plan.video_indices.data(),
                 plan.inverse_video_indices.data(), pos.data());
    s2_plan_free(p);
    plan.windows.resize(nw);
    for (int i = 0; i < nw; i++)
    {
        const int* w = &win[9 * (size_t)i];
        plan.windows[i] = WindowSlice{w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7], w[8]};
    }
    plan.local_positions.resize(nt);
    for (int i = 0; i < nt; i++) plan.local_positions[i] = {pos[3 * i], pos[3 * i + 1], pos[3 * i + 2]};
    return S2_OK;
}

AdaptiveWindowAttention::AdaptiveWindowAttention() : AdaptiveWindowAttention(nullptr) {}

AdaptiveWindowAttention::AdaptiveWindowAttention(AdaptiveWindowRuntimeState* state)
    : heads(20), head_dim(128), target_windows({4, 3, 3}), shifted(false), epsilon(1e-5f), rope_pairs_per_axis(21),
      shared_norm(false), shape_values_are_int32(false), official_bf16_attention(false), window_mode(S2_WINDOW_TARGET),
      runtime_state(state), d_weights(nullptr), weights_dirty(true)
{
    one_blob_only = false;
    support_inplace = false;
}

AdaptiveWindowAttention::~AdaptiveWindowAttention()
{
    if (d_weights) cudaFree(d_weights);
}

void AdaptiveWindowAttention::configure(int new_heads, int new_head_dim, const std::array<int, 3>& new_target,
                                        bool new_shifted, float new_epsilon, int new_pairs, bool int32_values,
                                        bool bf16_attention)
{
    heads = new_heads;
    head_dim = new_head_dim;
    target_windows = new_target;
    shifted = new_shifted;
    epsilon = new_epsilon;
    rope_pairs_per_axis = new_pairs;
    shape_values_are_int32 = int32_values;
    official_bf16_attention = bf16_attention;
    weights_dirty = true;
}

int AdaptiveWindowAttention::load_param(const ncnn::ParamDict& pd)
{
    heads = pd.get(0, 20);
    head_dim = pd.get(1, 128);
    target_windows[0] = pd.get(2, 4);
    target_windows[1] = pd.get(3, 3);
    target_windows[2] = pd.get(4, 3);
    shifted = pd.get(5, 0) != 0;
    epsilon = pd.get(6, 1e-5f);
    rope_pairs_per_axis = pd.get(7, 21);
    shared_norm = pd.get(8, 0) != 0;
    shape_values_are_int32 = pd.get(9, 0) != 0;
    official_bf16_attention = pd.get(10, 0) != 0;
    window_mode = pd.get(11, 0);
    weights_dirty = true;
    return 0;
}

int AdaptiveWindowAttention::load_model(const ncnn::ModelBin& mb)
{
    video_norm_q = mb.load(head_dim, 1);
    video_norm_k = mb.load(head_dim, 1);
    if (video_norm_q.empty() || video_norm_k.empty()) return -100;
    if (shared_norm)
    {
        text_norm_q = video_norm_q;
        text_norm_k = video_norm_k;
    }
    else
    {
        text_norm_q = mb.load(head_dim, 1);
        text_norm_k = mb.load(head_dim, 1);
        if (text_norm_q.empty() || text_norm_k.empty()) return -100;
    }
    rope_freqs = mb.load(rope_pairs_per_axis, 1);
    weights_dirty = true;
    return rope_freqs.empty() ? -100 : 0;
}

int AdaptiveWindowAttention::set_weights(const std::vector<float>& vq, const std::vector<float>& vk,
                                         const std::vector<float>& tq, const std::vector<float>& tk,
                                         const std::vector<float>& freqs)
{
    auto copy = [](const std::vector<float>& src, int n, ncnn::Mat& dst) {
        if (static_cast<int>(src.size()) != n) return -1;
        dst.create(n);
        if (dst.empty()) return -100;
        std::memcpy(dst.data, src.data(), n * sizeof(float));
        return 0;
    };
    if (copy(vq, head_dim, video_norm_q) || copy(vk, head_dim, video_norm_k) || copy(tq, head_dim, text_norm_q) ||
        copy(tk, head_dim, text_norm_k) || copy(freqs, rope_pairs_per_axis, rope_freqs))
        return -1;
    weights_dirty = true;
    return 0;
}

void AdaptiveWindowAttention::set_runtime_shapes(const std::vector<std::array<int, 3> >& shapes,
                                                 const std::vector<int>& lengths)
{
    owned_runtime_state.video_shapes = shapes;
    owned_runtime_state.text_lengths = lengths;
    runtime_state = &owned_runtime_state;
}

// upload_model analogue (adaptive_window_attention.cpp:1041-1057).
int AdaptiveWindowAttention::upload_weights() const
{
    if (!weights_dirty && d_weights) return 0;
    const size_t n = 4 * (size_t)head_dim + rope_pairs_per_axis;
    std::vector<float> host(n);
    std::memcpy(host.data(), video_norm_q.data, head_dim * 4);
    std::memcpy(host.data() + head_dim, video_norm_k.data, head_dim * 4);
    std::memcpy(host.data() + 2 * head_dim, text_norm_q.data, head_dim * 4);
    std::memcpy(host.data() + 3 * head_dim, text_norm_k.data, head_dim * 4);
    std::memcpy(host.data() + 4 * head_dim, rope_freqs.data, rope_pairs_per_axis * 4);
    if (d_weights) cudaFree(d_weights);
    d_weights = nullptr;
    if (cudaMalloc(&d_weights, n * 4) != cudaSuccess) return -100;
    if (cudaMemcpy(d_weights, host.data(), n * 4, cudaMemcpyHostToDevice) != cudaSuccess) return S2_ERR_CUDA;
    weights_dirty = false;
    return 0;
}

int AdaptiveWindowAttention::run(const std::vector<std::array<int, 3> >& shapes, const std::vector<int>& lengths,
                                 int in_dtype, const void* const* qkv, int64_t video_ld, int64_t text_ld,
                                 int out_dtype, void* video_out, void* text_out) const
{
    s2_context* ctx = layer_context();
    if (!ctx) return S2_ERR_DEVICE;
    int r = upload_weights();
    if (r != 0) return r;
    s2_awa_params p;
    p.heads = heads;
    p.head_dim = head_dim;
    p.window[0] = target_windows[0];
    p.window[1] = target_windows[1];
    p.window[2] = target_windows[2];
    p.window_mode = window_mode;
    p.shifted = shifted ? 1 : 0;
    p.epsilon = epsilon;
    p.rope_pairs = rope_pairs_per_axis;
    p.official_bf16_attention = official_bf16_attention ? 1 : 0;
    p.norm_weights = d_weights;
    p.rope_freqs = d_weights + 4 * head_dim;
    std::vector<int> flat;
    for (const auto& s : shapes) flat.insert(flat.end(), s.begin(), s.end());
    return s2_awa_forward(ctx, &p, nullptr, flat.data(), lengths.data(), static_cast<int>(shapes.size()), in_dtype,
                          qkv[0], qkv[1], qkv[2], video_ld, qkv[3], qkv[4], qkv[5], text_ld, out_dtype, video_out,
                          text_out);
}

int AdaptiveWindowAttention::forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                                     const ncnn::Option& opt) const
{
    (void)opt;
    const bool split_qkv = bottom_blobs.size() == 8;
    if ((!split_qkv && bottom_blobs.size() != 4) || top_blobs.size() != 2 || heads <= 0 || head_dim <= 0 ||
        rope_pairs_per_axis * 6 > head_dim || video_norm_q.empty() || video_norm_k.empty() || text_norm_q.empty() ||
        text_norm_k.empty() || rope_freqs.empty())
        return -1;
    const int inner = heads * head_dim;
    const ncnn::Mat& video_shape_blob = bottom_blobs[split_qkv ? 6 : 2];
    const ncnn::Mat& text_length_blob = bottom_blobs[split_qkv ? 7 : 3];
    if (split_qkv)
    {
        for (int part = 0; part < 6; part++)
            if (bottom_blobs[part].dims != 2 || bottom_blobs[part].w != inner || bottom_blobs[part].elempack != 1 ||
                bottom_blobs[part].elemsize != sizeof(float))
                return -1;
        if (video_shape_blob.w != 3) return -1;
    }
    else if (bottom_blobs[0].dims != 2 || bottom_blobs[1].dims != 2 || bottom_blobs[0].w != inner * 3 ||
             bottom_blobs[1].w != inner * 3 || video_shape_blob.w != 3)
        return -1;

    const int batch = video_shape_blob.dims == 1 ? 1 : video_shape_blob.h;
    const int text_batch = text_length_blob.dims == 1 ? text_length_blob.w : text_length_blob.h;
    if (batch <= 0 || text_batch != batch) return -1;
    std::vector<std::array<int, 3> > shapes(batch);
    std::vector<int> lengths(batch);
    int nv = 0, nt = 0;
    for (int s = 0; s < batch; s++)
    {
        for (int a = 0; a < 3; a++) shapes[s][a] = read_shape_value(video_shape_blob, s, a, shape_values_are_int32);
        lengths[s] = read_shape_value(text_length_blob, s, 0, shape_values_are_int32);
        if (lengths[s] <= 0) return -1;
        nv += shapes[s][0] * shapes[s][1] * shapes[s][2];
        nt += lengths[s];
    }
    if (split_qkv)
    {
        for (int part = 0; part < 3; part++)
            if (bottom_blobs[part].h != nv || bottom_blobs[part + 3].h != nt) return -1;
    }
    else if (bottom_blobs[0].h != nv || bottom_blobs[1].h != nt)
        return -1;
    if (head_dim != 128) return -1; // the tensor-core kernels are built for head_dim 128
    if (!layer_context()) return S2_ERR_DEVICE;

    ncnn::Mat& video_output = top_blobs[0];
    ncnn::Mat& text_output = top_blobs[1];
    video_output.create(inner, nv, 4u, opt.blob_allocator);
    text_output.create(inner, nt, 4u, opt.blob_allocator);
    if (video_output.empty() || text_output.empty()) return -100;

    // host blobs -> device, forward, device -> host
    const size_t in_v = (size_t)nv * inner * (split_qkv ? 1 : 3), in_t = (size_t)nt * inner * (split_qkv ? 1 : 3);
    const size_t bytes = ((split_qkv ? 3 : 1) * (in_v + in_t) + (size_t)(nv + nt) * inner) * 4 + 1024;
    static thread_local Scratch scratch;
    uint8_t* dev = static_cast<uint8_t*>(scratch.get(bytes));
    if (!dev) return -100;
    const void* ptr[6];
    size_t off = 0;
    if (split_qkv)
    {
        for (int part = 0; part < 6; part++)
        {
            const size_t n = (part < 3 ? (size_t)nv : (size_t)nt) * inner * 4;
            if (cudaMemcpy(dev + off, bottom_blobs[part].data, n, cudaMemcpyHostToDevice) != cudaSuccess)
                return S2_ERR_CUDA;
            ptr[part] = dev + off;
            off += (n + 255) & ~size_t(255);
        }
    }
    else
    {
        const size_t nvb = in_v * 4, ntb = in_t * 4;
        if (cudaMemcpy(dev, bottom_blobs[0].data, nvb, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(dev + ((nvb + 255) & ~size_t(255)), bottom_blobs[1].data, ntb, cudaMemcpyHostToDevice) !=
                cudaSuccess)
            return S2_ERR_CUDA;
        const uint8_t* v = dev;
        const uint8_t* t = dev + ((nvb + 255) & ~size_t(255));
        ptr[0] = v;
        ptr[1] = v + inner * 4;
        ptr[2] = v + 2 * inner * 4;
        ptr[3] = t;
        ptr[4] = t + inner * 4;
        ptr[5] = t + 2 * inner * 4;
        off = ((nvb + 255) & ~size_t(255)) + ((ntb + 255) & ~size_t(255));
    }
    uint8_t* vo = dev + off;
    uint8_t* to = vo + (((size_t)nv * inner * 4 + 255) & ~size_t(255));
    const int64_t ld = split_qkv ? inner : 3 * inner;
    int r = run(shapes, lengths, S2_DTYPE_F32, ptr, ld, ld, S2_DTYPE_F32, vo, to);
    if (r != S2_OK) return r;
    if (cudaMemcpy(video_output.data, vo, (size_t)nv * inner * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(text_output.data, to, (size_t)nt * inner * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return S2_ERR_CUDA;
    return s2_status(layer_context());
}

int AdaptiveWindowAttention::forward_cuda(const std::vector<CudaBlob>& bottom, std::vector<CudaBlob>& top) const
{
    const bool split_qkv = bottom.size() == 6;
    if ((!split_qkv && bottom.size() != 2) || top.size() != 2 || !runtime_state ||
        runtime_state->video_shapes.empty() ||
        runtime_state->video_shapes.size() != runtime_state->text_lengths.size())
        return -1;
    const int inner = heads * head_dim;
    const int dtype = bottom[0].dtype;
    for (const CudaBlob& b : bottom)
        if (!b.data || b.dtype != dtype || b.w != (split_qkv ? inner : 3 * inner) || b.ld < b.w) return -1;
    int nv = 0, nt = 0;
    for (size_t s = 0; s < runtime_state->video_shapes.size(); s++)
    {
        const auto& sh = runtime_state->video_shapes[s];
        if (sh[0] <= 0 || sh[1] <= 0 || sh[2] <= 0 || runtime_state->text_lengths[s] <= 0) return -1;
        nv += sh[0] * sh[1] * sh[2];
        nt += runtime_state->text_lengths[s];
    }
    const int nvid = split_qkv ? 3 : 1;
    for (int i = 0; i < (int)bottom.size(); i++)
        if (bottom[i].h != (i < nvid ? nv : nt)) return -1;
    if (!top[0].data || !top[1].data || top[0].w != inner || top[1].w != inner || top[0].h != nv ||
        top[1].h != nt || top[0].dtype != top[1].dtype)
        return -1;
    const size_t es = dtype == S2_DTYPE_BF16 ? 2 : 4;
    const void* ptr[6];
    if (split_qkv)
        for (int i = 0; i < 6; i++) ptr[i] = bottom[i].data;
    else
        for (int i = 0; i < 3; i++)
        {
            ptr[i] = static_cast<const uint8_t*>(bottom[0].data) + i * inner * es;
            ptr[3 + i] = static_cast<const uint8_t*>(bottom[1].data) + i * inner * es;
        }
    return run(runtime_state->video_shapes, runtime_state->text_lengths, dtype, ptr, bottom[0].ld,
               bottom[split_qkv ? 3 : 1].ld, top[0].dtype, top[0].data, top[1].data);
}

ncnn::Layer* adaptive_window_attention_layer_creator(void* userdata)
{
    return new AdaptiveWindowAttention(static_cast<AdaptiveWindowRuntimeState*>(userdata));
}

} // namespace seedvr2
