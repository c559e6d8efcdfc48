// extern "C" wrapper around the reference's OWN token-format functions
// patchify_video, make_timestep_embedding and unpatchify_prediction
// (src/seedvr2/seedvr2_dit.cpp:167-326) and the classifier-free guidance
// combine apply_cfg (src/seedvr2/seedvr2_pipeline.cpp:171-210).  They sit in
// anonymous namespaces of files that need the Vulkan runtime, so
// oracle/Makefile cuts exactly those ranges, unmodified, out of the reference
// tree into the git-ignored oracle/_ref/{dit_io,cfg}_extract.inc, and this
// file compiles them against the clean-room ncnn Mat shim into
// oracle/_ref/libs2_ref_dit_io.so.
//
// TEST INFRASTRUCTURE ONLY: the tests and the fixture generator load it as the
// checker; the shipped library never links it.
#include <array>
#include <cmath>
#include <cstring>
#include <vector>

#include "mat.h"

namespace seedvr2 {
namespace {
#include "dit_io_extract.inc"
#include "cfg_extract.inc"
} // namespace
} // namespace seedvr2

namespace {

std::vector<std::array<int, 3> > to_shapes(const int* shapes, int batch)
{
    std::vector<std::array<int, 3> > v((size_t)batch);
    for (int s = 0; s < batch; s++)
        for (int a = 0; a < 3; a++) v[s][a] = shapes[3 * s + a];
    return v;
}

} // namespace

extern "C" {

// src [rows][33] -> dst [patches][132]; out_shapes [batch][3].  Returns the
// reference's code (0, -1, -100).
int s2ref_patchify_video(const float* src, int rows, const int* shapes, int batch, float* dst, int* out_shapes)
{
    ncnn::Mat in(33, rows);
    if (rows > 0) std::memcpy(in.data, src, sizeof(float) * 33 * (size_t)rows);
    ncnn::Mat out;
    std::vector<std::array<int, 3> > os;
    const int r = seedvr2::patchify_video(in, to_shapes(shapes, batch), out, os);
    if (r != 0) return r;
    std::memcpy(dst, out.data, sizeof(float) * 132 * (size_t)out.h);
    for (size_t s = 0; s < os.size(); s++)
        for (int a = 0; a < 3; a++) out_shapes[3 * s + a] = os[s][a];
    return 0;
}

// src [patches][64] -> dst [tokens][16]; shapes are the latent shapes.
int s2ref_unpatchify_prediction(const float* src, int rows, const int* shapes, int batch, float* dst)
{
    ncnn::Mat in(64, rows);
    if (rows > 0) std::memcpy(in.data, src, sizeof(float) * 64 * (size_t)rows);
    std::vector<std::array<int, 3> > latent = to_shapes(shapes, batch), patched = latent;
    for (auto& p : patched) p[1] /= 2, p[2] /= 2;
    ncnn::Mat out;
    const int r = seedvr2::unpatchify_prediction(in, latent, patched, out);
    if (r != 0) return r;
    std::memcpy(dst, out.data, sizeof(float) * 16 * (size_t)out.h);
    return 0;
}

// out [batch][256]
int s2ref_timestep_embedding(const float* timesteps, int batch, float* out)
{
    std::vector<float> t(timesteps, timesteps + (batch > 0 ? batch : 0));
    ncnn::Mat e;
    const int r = seedvr2::make_timestep_embedding(t, e);
    if (r != 0) return r;
    std::memcpy(out, e.data, sizeof(float) * 256 * (size_t)batch);
    return 0;
}

// cfg [count] = apply_cfg(pos, neg) on [rows][w] blobs
int s2ref_apply_cfg(const float* pos, const float* neg, int w, int rows, float scale, float rescale, float* cfg)
{
    ncnn::Mat p(w, rows), n(w, rows), out;
    std::memcpy(p.data, pos, sizeof(float) * (size_t)w * rows);
    std::memcpy(n.data, neg, sizeof(float) * (size_t)w * rows);
    seedvr2::apply_cfg(p, n, scale, rescale, out);
    std::memcpy(cfg, out.data, sizeof(float) * (size_t)w * rows);
    return 0;
}

} // extern "C"
