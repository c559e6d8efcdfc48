// VAE runtime pieces around the encoder / decoder graphs (SeedVR2VAE,
// seedvr2_vae.h:17-43, seedvr2_vae.cpp:408-601): the temporal segment plan of
// extract_temporal_slices, the posterior sampling and scaling of
// moments_to_latent, and decode's unscaling.  The graphs themselves are
// exported .param/.bin files that the reference tree does not hold; each
// segment runs through the VAE layers of this library (DecomposedConv3D,
// VAEDownsample3D / VAEUpsample3D, VAEChunkedMHA), whose temporal-memory
// states are the S2_VAE_MEMORY_* values the plan assigns.
#include <algorithm>
#include <cuda_runtime.h>
#include <random>

#include "s2_internal.h"
#include "s2_objects.h"
#include "seedvr2_cuda.h"

namespace {

// latent[c][i] = (mean[c][i] + exp(0.5 clamp(logvar[c][i], -30, 20)) *
// noise[c][i]) * 0.9152 over 16 channels of `plane` values; moments holds the
// 16 mean channels, then the 16 logvar channels.  Explicit roundings keep the
// reference's separate multiply and add (no contraction into an FMA).
__global__ void moments_to_latent_kernel(const float* __restrict__ moments, const float* __restrict__ noise,
                                         int64_t plane, float* __restrict__ latent)
{
    const int64_t n = 16 * plane;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    {
        const int64_t c = i / plane, j = i - c * plane;
        float v = moments[c * plane + j];
        if (noise)
        {
            const float lv = fminf(20.f, fmaxf(-30.f, moments[(c + 16) * plane + j]));
            v = __fadd_rn(v, __fmul_rn(expf(__fmul_rn(0.5f, lv)), noise[i]));
        }
        latent[i] = __fmul_rn(v, S2_VAE_SCALING_FACTOR);
    }
}

__global__ void unscale_kernel(float* __restrict__ x, int64_t n)
{
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = __fdiv_rn(x[i], S2_VAE_SCALING_FACTOR);
}

int grid_for(const s2::Context& c, int64_t n)
{
    const int64_t blocks = (n + 255) / 256;
    return (int)std::min<int64_t>(blocks, (int64_t)c.num_sms * 8);
}

} // namespace

extern "C" {

int s2_vae_temporal_segments(int frames, int first, int active, int capacity, int* segments)
{
    if (frames <= 0 || first <= 0 || active <= 0 || capacity < 0 || (capacity > 0 && !segments)) return -1;
    // one run without temporal memory when the input fits the first segment
    if (frames <= first)
    {
        if (capacity >= 1)
        {
            segments[0] = 0;
            segments[1] = frames;
            segments[2] = S2_VAE_MEMORY_DISABLED;
        }
        return 1;
    }
    int n = 0;
    for (int start = 0; start < frames; n++)
    {
        const int count = std::min(start == 0 ? first : active, frames - start);
        if (n < capacity)
        {
            segments[3 * n] = start;
            segments[3 * n + 1] = count;
            segments[3 * n + 2] = start == 0 ? S2_VAE_MEMORY_INITIALIZING : S2_VAE_MEMORY_ACTIVE;
        }
        start += count;
    }
    return n;
}

int s2_vae_encode_frames(int frames)
{
    // encode_moments (seedvr2_vae.cpp:551-565): more than five frames must be 4n + 1
    if (frames <= 0 || (frames > 5 && (frames - 1) % 4 != 0)) return -1;
    return (frames - 1) / 4 + 1;
}

int s2_vae_decode_frames(int latent_frames)
{
    // decode (seedvr2_vae.cpp:578-599)
    return latent_frames <= 0 ? -1 : (latent_frames - 1) * 4 + 1;
}

int s2_vae_posterior_noise(uint64_t seed, int64_t count, float* out)
{
    if (count < 0 || (count > 0 && !out)) return S2_ERR_INVALID;
    // the reference's generator and distribution, drawn in its order
    // (channel-major, moments_to_latent seedvr2_vae.cpp:461-475)
    std::mt19937_64 generator(seed);
    std::normal_distribution<float> normal(0.f, 1.f);
    for (int64_t i = 0; i < count; i++) out[i] = normal(generator);
    return S2_OK;
}

int s2_vae_moments_to_latent(s2_context* ctx, const float* moments, int w, int h, int d, const float* noise,
                             float* latent)
{
    if (!ctx || !moments || !latent || w <= 0 || h <= 0 || d <= 0) return S2_ERR_INVALID;
    s2::Context& c = ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int64_t plane = (int64_t)w * h * d;
    moments_to_latent_kernel<<<grid_for(c, 16 * plane), 256, 0, c.stream>>>(moments, noise, plane, latent);
    if (cudaGetLastError() != cudaSuccess) return S2_ERR_CUDA;
    c.launches++;
    return S2_OK;
}

int s2_vae_unscale_latent(s2_context* ctx, float* latent, int64_t count)
{
    if (!ctx || !latent || count <= 0) return S2_ERR_INVALID;
    s2::Context& c = ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    unscale_kernel<<<grid_for(c, count), 256, 0, c.stream>>>(latent, count);
    if (cudaGetLastError() != cudaSuccess) return S2_ERR_CUDA;
    c.launches++;
    return S2_OK;
}

} // extern "C"
