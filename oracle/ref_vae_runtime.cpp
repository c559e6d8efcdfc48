// extern "C" wrapper around the reference's OWN posterior sampling
// moments_to_latent and its shape check is_latent_shape
// (src/seedvr2/seedvr2_vae.cpp:198-203, :454-478).  They sit in an anonymous
// namespace of a file that needs the Vulkan runtime, so oracle/Makefile cuts
// exactly those two functions, unmodified, out of the reference tree into the
// git-ignored oracle/_ref/vae_rt_extract.inc, and this file compiles them
// against the clean-room ncnn Mat shim into oracle/_ref/libs2_ref_vae_rt.so.
// The two declarations they use from seedvr2_vae.h (which pulls in the Vulkan
// net.h) are restated here with the header's values: VAEEncodeOptions
// (seedvr2_vae.h:11-15) and SeedVR2VAE::scaling_factor (:35).
//
// TEST INFRASTRUCTURE ONLY: the tests load it as the checker; the shipped
// library never links it.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>

#include "mat.h"

namespace seedvr2 {

struct VAEEncodeOptions
{
    bool sample_posterior = true;
    uint64_t seed = 666;
};

struct SeedVR2VAE
{
    static constexpr float scaling_factor() { return 0.9152f; }
};

namespace {
#include "vae_rt_extract.inc"
} // namespace
} // namespace seedvr2

extern "C" {

// moments fp32 [32][d][h][w] (host) -> latent fp32 [16][d][h][w]; returns the
// reference's code (0, -1 for a bad shape, -100 for a failed allocation)
int ref_vae_moments_to_latent(const float* moments, int w, int h, int d, int sample_posterior, uint64_t seed,
                              float* latent)
{
    ncnn::Mat m;
    m.create(w, h, d, 32);
    const size_t plane = (size_t)w * h * d;
    for (int c = 0; c < 32; c++) std::memcpy(m.channel(c).data, moments + c * plane, plane * 4);
    seedvr2::VAEEncodeOptions options;
    options.sample_posterior = sample_posterior != 0;
    options.seed = seed;
    ncnn::Mat out;
    const int r = seedvr2::moments_to_latent(m, out, options);
    if (r != 0) return r;
    for (int c = 0; c < 16; c++) std::memcpy(latent + c * plane, out.channel(c).data, plane * 4);
    return 0;
}

} // extern "C"
