// Device forms of the few ncnn built-in layers a DiT block graph places
// between the custom layers (BinaryOp with row broadcast, RMSNorm /
// LayerNorm, GELU), for the graph executor of the ncnn-surface library
// (csrc/layers/net.cpp).  fp32 row-major [rows][cols] blobs, HBM-bound
// passes with 16-byte accesses where the widths allow.
#include "s2_common.cuh"
#include "s2_internal.h"
#include "s2_objects.h"

namespace s2 {

namespace {

template <int OP>
__device__ __forceinline__ float binop(float a, float b)
{
    if (OP == S2_BINARY_ADD) return a + b;
    if (OP == S2_BINARY_SUB) return a - b;
    if (OP == S2_BINARY_MUL) return a * b;
    return a / b;
}

// out[r][c] = a[r][c] op b[r or 0][c]; cols % 4 == 0 (float4 lanes)
template <int OP>
__global__ void binary_kernel(const float4* __restrict__ a, const float4* __restrict__ b, float4* __restrict__ out,
                              int64_t count4, int cols4, int b_broadcast)
{
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count4; i += stride)
    {
        const float4 x = a[i];
        const float4 y = b[b_broadcast ? i % cols4 : i];
        out[i] = make_float4(binop<OP>(x.x, y.x), binop<OP>(x.y, y.y), binop<OP>(x.z, y.z), binop<OP>(x.w, y.w));
    }
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

// One warp per row: LayerNorm (centred) or RMSNorm, then gamma / beta when given.
template <bool LAYER>
__global__ void norm_f32_kernel(int rows, int D, const float* __restrict__ x, float eps,
                                const float* __restrict__ gamma, const float* __restrict__ beta,
                                float* __restrict__ y)
{
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + (int64_t)row * D;
    float* yr = y + (int64_t)row * D;
    float mean = 0.f;
    if (LAYER)
    {
        float s = 0.f;
        for (int c = lane; c < D; c += 32) s += xr[c];
        mean = warp_sum(s) / D;
    }
    float ss = 0.f;
    for (int c = lane; c < D; c += 32)
    {
        const float d = xr[c] - mean;
        ss += d * d;
    }
    const float inv = 1.f / sqrtf(warp_sum(ss) / D + eps);
    for (int c = lane; c < D; c += 32)
    {
        float v = (xr[c] - mean) * inv;
        if (gamma) v *= gamma[c];
        if (beta) v += beta[c];
        yr[c] = v;
    }
}

__global__ void gelu_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t count, int fast)
{
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride)
    {
        const float v = x[i];
        y[i] = fast ? gelu_tanh(v) : 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
    }
}

int grid_for(Context& ctx, int64_t n)
{
    const int64_t blocks = (n + 255) / 256;
    const int64_t cap = (int64_t)ctx.num_sms * 8;
    return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

} // namespace

int launch_binary_op(Context& ctx, int op, int rows, int cols, const float* a, const float* b, int b_rows, float* out)
{
    if (rows < 0 || cols <= 0 || cols % 4 || (b_rows != 1 && b_rows != rows) || op < 0 || op > 3 ||
        (reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(out)) & 15)
        return S2_ERR_INVALID;
    const int64_t count4 = (int64_t)rows * cols / 4;
    if (count4 == 0) return S2_OK;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)rows * cols * 12.0);
    const int g = grid_for(ctx, count4);
    const float4 *A = reinterpret_cast<const float4*>(a), *B = reinterpret_cast<const float4*>(b);
    float4* O = reinterpret_cast<float4*>(out);
    const int bc = b_rows == 1 && rows != 1;
    switch (op)
    {
    case S2_BINARY_ADD: binary_kernel<S2_BINARY_ADD><<<g, 256, 0, ctx.stream>>>(A, B, O, count4, cols / 4, bc); break;
    case S2_BINARY_SUB: binary_kernel<S2_BINARY_SUB><<<g, 256, 0, ctx.stream>>>(A, B, O, count4, cols / 4, bc); break;
    case S2_BINARY_MUL: binary_kernel<S2_BINARY_MUL><<<g, 256, 0, ctx.stream>>>(A, B, O, count4, cols / 4, bc); break;
    default: binary_kernel<S2_BINARY_DIV><<<g, 256, 0, ctx.stream>>>(A, B, O, count4, cols / 4, bc); break;
    }
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

int launch_norm_f32(Context& ctx, int layer, int rows, int D, const float* x, float eps, const float* gamma,
                    const float* beta, float* y)
{
    if (rows < 0 || D <= 0 || (layer != 0 && layer != 1)) return S2_ERR_INVALID;
    if (rows == 0) return S2_OK;
    ProfileScope prof(ctx, K_NORM, 0.0, (double)rows * D * 8.0);
    const int warps = 8;
    const int g = (rows + warps - 1) / warps;
    if (layer)
        norm_f32_kernel<true><<<g, warps * 32, 0, ctx.stream>>>(rows, D, x, eps, gamma, beta, y);
    else
        norm_f32_kernel<false><<<g, warps * 32, 0, ctx.stream>>>(rows, D, x, eps, gamma, beta, y);
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

int launch_gelu_f32(Context& ctx, int fast, int64_t count, const float* x, float* y)
{
    if (count < 0) return S2_ERR_INVALID;
    if (count == 0) return S2_OK;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)count * 8.0);
    gelu_kernel<<<grid_for(ctx, count), 256, 0, ctx.stream>>>(x, y, count, fast);
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

} // namespace s2

extern "C" {

int s2_binary_op(s2_context* ctx, int op, int rows, int cols, const float* a, const float* b, int b_rows, float* out)
{
    if (!ctx || !a || !b || !out) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return s2::launch_binary_op(ctx->c, op, rows, cols, a, b, b_rows, out);
}

int s2_norm_f32(s2_context* ctx, int layer, int rows, int D, const float* x, float eps, const float* gamma,
                const float* beta, float* out)
{
    if (!ctx || !x || !out) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return s2::launch_norm_f32(ctx->c, layer, rows, D, x, eps, gamma, beta, out);
}

int s2_gelu_f32(s2_context* ctx, int fast, int64_t count, const float* x, float* out)
{
    if (!ctx || !x || !out) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return s2::launch_gelu_f32(ctx->c, fast, count, x, out);
}

} // extern "C"
