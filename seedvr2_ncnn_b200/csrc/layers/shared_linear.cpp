// SharedLinear on libseedvr2_cuda (see the header).
#include "shared_linear.h"

#include <cuda_runtime.h>

#include <cstring>

namespace seedvr2 {

namespace {

// Grow-only device staging of the host-blob forward (one per host thread):
// repeated calls of the same or smaller size allocate nothing.
struct Staging
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

SharedLinear::SharedLinear()
    : num_output(0), num_input(0), bias_term(false), d_weight(nullptr), d_bias(nullptr)
{
    one_blob_only = false;
    support_inplace = false;
}

SharedLinear::~SharedLinear()
{
    if (d_weight) cudaFree(d_weight);
    if (d_bias) cudaFree(d_bias);
}

int SharedLinear::load_param(const ncnn::ParamDict& pd)
{
    num_output = pd.get(0, 0);
    num_input = pd.get(1, 0);
    bias_term = pd.get(2, 0) != 0;
    if (num_output <= 0 || num_input <= 0) return -1;
    return 0;
}

int SharedLinear::load_model(const ncnn::ModelBin& mb)
{
    weight_data = mb.load(num_input * num_output, 1);
    if (weight_data.empty()) return -100;
    weight_data = weight_data.reshape(num_input, num_output);
    if (weight_data.empty()) return -100;
    if (bias_term)
    {
        bias_data = mb.load(num_output, 1);
        if (bias_data.empty()) return -100;
    }
    if (d_weight)
    {
        cudaFree(d_weight);
        d_weight = nullptr;
    }
    return 0;
}

// fp32 weight -> bf16 on the device (once), bias kept fp32.
int SharedLinear::upload() const
{
    if (d_weight) return 0;
    s2_context* ctx = layer_context();
    if (!ctx) return S2_ERR_DEVICE;
    const size_t n = (size_t)num_output * num_input;
    float* tmp = nullptr;
    if (cudaMalloc(&tmp, n * 4) != cudaSuccess) return -100;
    if (cudaMalloc(&d_weight, n * 2) != cudaSuccess)
    {
        cudaFree(tmp);
        d_weight = nullptr;
        return -100;
    }
    int r = cudaMemcpy(tmp, weight_data.data, n * 4, cudaMemcpyHostToDevice) == cudaSuccess ? S2_OK : S2_ERR_CUDA;
    if (r == S2_OK) r = s2_convert_f32_bf16(ctx, tmp, d_weight, (int64_t)n);
    if (r == S2_OK) r = s2_status(ctx);
    cudaFree(tmp);
    if (r == S2_OK && bias_term)
    {
        if (cudaMalloc(&d_bias, num_output * 4) != cudaSuccess) return -100;
        if (cudaMemcpy(d_bias, bias_data.data, num_output * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return S2_ERR_CUDA;
    }
    if (r != S2_OK)
    {
        cudaFree(d_weight);
        d_weight = nullptr;
    }
    return r;
}

int SharedLinear::forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                          const ncnn::Option& opt) const
{
    if (weight_data.empty() || bottom_blobs.size() != 2 || top_blobs.size() != 2 || bottom_blobs[0].dims != 2 ||
        bottom_blobs[1].dims != 2 || bottom_blobs[0].w != num_input || bottom_blobs[1].w != num_input)
        return -1;
    if (num_output % 8 || num_input % 8) return -1; // the tensor-core GEMM takes multiples of 8
    int r = upload();
    if (r != 0) return r;
    s2_context* ctx = layer_context();
    const int m0 = bottom_blobs[0].h, m1 = bottom_blobs[1].h;
    top_blobs[0].create(num_output, m0, 4u, opt.blob_allocator);
    top_blobs[1].create(num_output, m1, 4u, opt.blob_allocator);
    if (top_blobs[0].empty() || top_blobs[1].empty()) return -100;
    // staging: fp32 inputs, bf16 inputs, fp32 outputs (grow-only, per host thread)
    const size_t K = num_input, N = num_output, M = (size_t)m0 + m1;
    const size_t b_in32 = (M * K * 4 + 255) & ~size_t(255), b_in16 = (M * K * 2 + 255) & ~size_t(255);
    static thread_local Staging staging;
    uint8_t* buf = static_cast<uint8_t*>(staging.get(b_in32 + b_in16 + M * N * 4 + 256));
    if (!buf) return -100;
    float* in32 = reinterpret_cast<float*>(buf);
    uint8_t* in16 = buf + b_in32;
    float* out = reinterpret_cast<float*>(buf + b_in32 + b_in16);
    r = S2_OK;
    if (cudaMemcpy(in32, bottom_blobs[0].data, (size_t)m0 * K * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(in32 + (size_t)m0 * K, bottom_blobs[1].data, (size_t)m1 * K * 4, cudaMemcpyHostToDevice) !=
            cudaSuccess)
        r = S2_ERR_CUDA;
    if (r == S2_OK) r = s2_convert_f32_bf16(ctx, in32, in16, (int64_t)(M * K));
    // the two streams are adjacent here, but go through the two-stream entry point
    if (r == S2_OK)
        r = s2_shared_linear(ctx, m0, m1, num_output, num_input, in16, in16 + (size_t)m0 * K * 2, d_weight, d_bias,
                             S2_EPI_STORE, nullptr, S2_DTYPE_F32, out, out + (size_t)m0 * N);
    if (r == S2_OK) r = s2_status(ctx);
    if (r == S2_OK &&
        (cudaMemcpy(top_blobs[0].data, out, (size_t)m0 * N * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
         cudaMemcpy(top_blobs[1].data, out + (size_t)m0 * N, (size_t)m1 * N * 4, cudaMemcpyDeviceToHost) !=
             cudaSuccess))
        r = S2_ERR_CUDA;
    return r;
}

int SharedLinear::forward_cuda(const std::vector<CudaBlob>& bottom, std::vector<CudaBlob>& top, int epilogue,
                               const float* gate) const
{
    if (weight_data.empty() || bottom.size() != 2 || top.size() != 2) return -1;
    for (int i = 0; i < 2; i++)
        if (bottom[i].dtype != S2_DTYPE_BF16 || bottom[i].w != num_input || bottom[i].ld != num_input ||
            top[i].w != num_output || top[i].ld != num_output || top[i].h != bottom[i].h ||
            top[i].dtype != top[0].dtype)
            return -1;
    int r = upload();
    if (r != 0) return r;
    return s2_shared_linear(layer_context(), bottom[0].h, bottom[1].h, num_output, num_input, bottom[0].data,
                            bottom[1].data, d_weight, d_bias, epilogue, gate, top[0].dtype, top[0].data,
                            top[1].data);
}

ncnn::Layer* shared_linear_layer_creator(void* /*userdata*/)
{
    return new SharedLinear;
}

} // namespace seedvr2
