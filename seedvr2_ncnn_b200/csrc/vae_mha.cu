// VAEChunkedMHA on sm_100a (vae_chunked_mha.cpp:109-217): self-attention of
// one blob x [T][E] with a single head of width E (the VAE mid block's 512).
// A 512-wide head does not fit the window-attention kernel's TMEM plan (the
// O accumulator alone would take all 512 columns), so the layer runs as
// tensor-core GEMMs around an HBM-bound softmax, in query chunks that bound
// the score matrix like the reference's Vulkan path does:
//   q, k, v = bf16(x) W^T + b                  (SharedLinear GEMM, bf16 out)
//   per chunk of Qc queries:
//     S = q_c k^T                              (GEMM, fp32 [Qc][T8])
//     P = bf16(softmax(scale * S))             (row kernel below)
//     o_c = P v                                (GEMM against v^T [E][T8])
//   out = o Wout^T + b                         (GEMM, fp32)
// T8 = T rounded up to 8 (16-byte GEMM rows); k's padding rows and v^T's
// padding columns are zero and the softmax ignores columns >= T.
#include <algorithm>
#include <cmath>
#include <memory>
#include <vector>

#include "s2_common.cuh"
#include "s2_internal.h"
#include "s2_objects.h"

namespace s2 {

namespace {

// P[r][j] = bf16(exp(scale * S[r][j] - m) / sum) over j < T, 0 for T <= j < T8;
// one block per row, fp32 max / sum reductions.
__global__ void __launch_bounds__(256) mha_softmax_kernel(const float* __restrict__ S, int T, int T8, float scale,
                                                          __nv_bfloat16* __restrict__ P)
{
    __shared__ float red[8];
    const int r = blockIdx.x;
    const float* s = S + (int64_t)r * T8;
    __nv_bfloat16* p = P + (int64_t)r * T8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float m = -INFINITY;
    for (int j = threadIdx.x; j < T; j += blockDim.x) m = fmaxf(m, s[j] * scale);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int i = 1; i < 8; i++) m = fmaxf(m, red[i]);
    __syncthreads();
    float sum = 0.f;
    for (int j = threadIdx.x; j < T; j += blockDim.x) sum += expf(s[j] * scale - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    sum = 0.f;
    for (int i = 0; i < 8; i++) sum += red[i];
    const float inv = 1.f / sum;
    for (int j = threadIdx.x; j < T8; j += blockDim.x)
        p[j] = __float2bfloat16_rn(j < T ? expf(s[j] * scale - m) * inv : 0.f);
}

// vt[e][t] = v[t][e] for t < T, 0 for T <= t < T8 (32 x 32 tiles).
__global__ void mha_transpose_kernel(const __nv_bfloat16* __restrict__ v, int T, int T8, int E,
                                     __nv_bfloat16* __restrict__ vt)
{
    __shared__ __nv_bfloat16 tile[32][34];
    const int t0 = blockIdx.x * 32, e0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5; // 32 x 8
    for (int i = ty; i < 32; i += 8)
    {
        const int t = t0 + i, e = e0 + tx;
        tile[i][tx] = (t < T && e < E) ? v[(int64_t)t * E + e] : __float2bfloat16_rn(0.f);
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8)
    {
        const int e = e0 + i, t = t0 + tx;
        if (e < E && t < T8) vt[(int64_t)e * T8 + t] = tile[tx][i];
    }
}

} // namespace

} // namespace s2

struct s2_vae_mha
{
    s2_context* ctx = nullptr;
    int E = 0;
    float scale = 1.f;
    void* w = nullptr;     // bf16 q, k, v, out weights [4][E][E]
    float* b = nullptr;    // fp32 q, k, v, out biases [4][E]
    s2::DeviceBuffer ws;
    ~s2_vae_mha()
    {
        if (w) cudaFree(w);
        if (b) cudaFree(b);
    }
};

namespace {
size_t a256(size_t x)
{
    return (x + 255) & ~size_t(255);
}
} // namespace

extern "C" {

int s2_vae_mha_create(s2_context* ctx, int embed_dim, int num_heads, float scale, const float* weights,
                      s2_vae_mha** out)
{
    // load_param's checks (vae_chunked_mha.cpp:109-123); one head per this build
    if (!ctx || !weights || !out || embed_dim <= 0 || num_heads <= 0 || embed_dim % num_heads) return S2_ERR_INVALID;
    *out = nullptr;
    if (num_heads != 1 || embed_dim % 8) return S2_ERR_INVALID;
    s2::Context& c = ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    std::unique_ptr<s2_vae_mha> l(new s2_vae_mha);
    l->ctx = ctx;
    l->E = embed_dim;
    l->scale = scale;
    const size_t E = embed_dim, EE = E * E;
    // load_model order: q w, q b, k w, k b, v w, v b, out w, out b
    std::vector<__nv_bfloat16> w(4 * EE);
    std::vector<float> b(4 * E);
    for (int i = 0; i < 4; i++)
    {
        const float* src = weights + i * (EE + E);
        for (size_t j = 0; j < EE; j++) w[i * EE + j] = __float2bfloat16(src[j]);
        for (size_t j = 0; j < E; j++) b[i * E + j] = src[EE + j];
    }
    if (cudaMalloc(&l->w, w.size() * 2) != cudaSuccess)
    {
        l->w = nullptr;
        return S2_ERR_ALLOC;
    }
    if (cudaMalloc(&l->b, b.size() * 4) != cudaSuccess)
    {
        l->b = nullptr;
        return S2_ERR_ALLOC;
    }
    if (cudaMemcpy(l->w, w.data(), w.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(l->b, b.data(), b.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return S2_ERR_CUDA;
    *out = l.release();
    return S2_OK;
}

int s2_vae_mha_forward(s2_vae_mha* l, const float* x, int tokens, float* out)
{
    if (!l || !x || !out || tokens <= 0) return S2_ERR_INVALID;
    s2::Context& c = l->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int E = l->E, T = tokens, T8 = (tokens + 7) & ~7;
    // query chunk: the fp32 score chunk stays under 256 MiB
    int64_t qc = ((int64_t)1 << 26) / T8;
    qc = std::max<int64_t>(128, qc / 128 * 128);
    const int Qc = (int)std::min<int64_t>(qc, (T + 127) / 128 * 128);
    const size_t s_x = a256((size_t)T * E * 2), s_k = a256((size_t)T8 * E * 2), s_vt = a256((size_t)E * T8 * 2),
                 s_S = a256((size_t)Qc * T8 * 4), s_P = a256((size_t)Qc * T8 * 2);
    // xb | q | k (T8 rows) | v | vt | S | P | o
    int r = l->ws.ensure(s_x * 4 + s_k + s_vt + s_S + s_P);
    if (r != S2_OK) return r;
    uint8_t* p = static_cast<uint8_t*>(l->ws.ptr);
    __nv_bfloat16* xb = reinterpret_cast<__nv_bfloat16*>(p);
    __nv_bfloat16* q = reinterpret_cast<__nv_bfloat16*>(p + s_x);
    __nv_bfloat16* k = reinterpret_cast<__nv_bfloat16*>(p + 2 * s_x);
    __nv_bfloat16* v = reinterpret_cast<__nv_bfloat16*>(p + 2 * s_x + s_k);
    __nv_bfloat16* vt = reinterpret_cast<__nv_bfloat16*>(p + 3 * s_x + s_k);
    float* S = reinterpret_cast<float*>(p + 3 * s_x + s_k + s_vt);
    __nv_bfloat16* P = reinterpret_cast<__nv_bfloat16*>(p + 3 * s_x + s_k + s_vt + s_S);
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p + 3 * s_x + s_k + s_vt + s_S + s_P);
    const __nv_bfloat16* W = static_cast<const __nv_bfloat16*>(l->w);
    const size_t EE = (size_t)E * E;
    r = s2::launch_convert_f32_bf16(c, x, xb, (int64_t)T * E);
    // k's padding rows must read as zero keys
    if (r == S2_OK && T8 > T &&
        cudaMemsetAsync(k + (size_t)T * E, 0, (size_t)(T8 - T) * E * 2, c.stream) != cudaSuccess)
        r = S2_ERR_CUDA;
    if (r == S2_OK)
        r = s2::launch_shared_linear(c, T, 0, E, E, xb, nullptr, W, l->b, s2::EPI_STORE, nullptr, 0, q, nullptr);
    if (r == S2_OK)
        r = s2::launch_shared_linear(c, T, 0, E, E, xb, nullptr, W + EE, l->b + E, s2::EPI_STORE, nullptr, 0, k,
                                     nullptr);
    if (r == S2_OK)
        r = s2::launch_shared_linear(c, T, 0, E, E, xb, nullptr, W + 2 * EE, l->b + 2 * E, s2::EPI_STORE, nullptr, 0,
                                     v, nullptr);
    if (r == S2_OK)
    {
        s2::ProfileScope prof(c, s2::K_OTHER, 0.0, (double)T8 * E * 4.0);
        s2::mha_transpose_kernel<<<dim3((T8 + 31) / 32, (E + 31) / 32), 256, 0, c.stream>>>(v, T, T8, E, vt);
        c.launches++;
        if (cudaGetLastError() != cudaSuccess) r = S2_ERR_CUDA;
    }
    for (int q0 = 0; q0 < T && r == S2_OK; q0 += Qc)
    {
        const int m = std::min(Qc, T - q0);
        r = s2::launch_shared_linear(c, m, 0, T8, E, q + (size_t)q0 * E, nullptr, k, nullptr, s2::EPI_STORE, nullptr,
                                     1, S, nullptr);
        if (r == S2_OK)
        {
            s2::ProfileScope prof(c, s2::K_OTHER, 0.0, (double)m * T8 * 6.0);
            s2::mha_softmax_kernel<<<m, 256, 0, c.stream>>>(S, T, T8, l->scale, P);
            c.launches++;
            if (cudaGetLastError() != cudaSuccess) r = S2_ERR_CUDA;
        }
        if (r == S2_OK)
            r = s2::launch_shared_linear(c, m, 0, E, T8, P, nullptr, vt, nullptr, s2::EPI_STORE, nullptr, 0,
                                         o + (size_t)q0 * E, nullptr);
    }
    if (r == S2_OK)
        r = s2::launch_shared_linear(c, T, 0, E, E, o, nullptr, W + 3 * EE, l->b + 3 * E, s2::EPI_STORE, nullptr, 1,
                                     out, nullptr);
    return r;
}

void s2_vae_mha_free(s2_vae_mha* l)
{
    if (!l) return;
    cudaSetDevice(l->ctx->c.device);
    cudaStreamSynchronize(l->ctx->c.stream);
    delete l;
}

} // extern "C"
