// Token formats and small dense passes on either side of the block stack:
//   patchify / unpatchify of 1x2x2 latent patches (patchify_video and
//   unpatchify_prediction, seedvr2_dit.cpp:167-230, :255-326),
//   the 256-wide sinusoidal timestep embedding (make_timestep_embedding,
//   :232-253), and the batch-row matrix-vector products of the timestep MLP
//   in the frontend net (forward_frontend, :1183-1295).
// All are HBM-bound and tiny next to one block; grids are sized by elements,
// capped at a few waves of the 148 SMs.
#include <cmath>

#include "s2_common.cuh"
#include "s2_internal.h"

namespace s2 {

namespace {

inline int launched(Context& ctx)
{
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

inline int grid_for(const Context& ctx, int64_t items, int threads)
{
    int64_t b = (items + threads - 1) / threads;
    const int64_t cap = (int64_t)ctx.num_sms * 16;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

// dst row p (patch (frame, py, px) of one sample) = the four tokens
// (frame, 2py + y, 2px + x) of src, 33 channels each, in (y, x) order.
// BF16: rows of kPatchPitch bf16 with zeros after the 132 features (the GEMM
// operand of the video input projection); otherwise rows of 132 fp32.
// Token rows of the DiT video input: either [tokens][33] rows (rows != null)
// or, fused with SeedVR2Pipeline::predict's assembly (seedvr2_pipeline.cpp:
// 296-318), channel c < 16 of latent plane c, 16 <= c < 32 of condition plane
// c - 16, and c = 32 the constant 1.
struct PatchSource
{
    const float* rows;
    const float* latent;
    int64_t latent_cstep;
    const float* condition;
    int64_t condition_cstep;
    __device__ __forceinline__ float at(int64_t tok, int c) const
    {
        if (rows) return __ldg(rows + tok * kLatentChannels + c);
        if (c < kPredChannels) return __ldg(latent + c * latent_cstep + tok);
        if (c < 2 * kPredChannels) return __ldg(condition + (c - kPredChannels) * condition_cstep + tok);
        return 1.f;
    }
};

template <bool BF16>
__global__ void patchify_kernel(const PatchSource src, int T, int H, int W, void* __restrict__ dst, int out_w)
{
    const int ph = H >> 1, pw = W >> 1;
    const int64_t per_frame = (int64_t)ph * pw;
    const int64_t total = (int64_t)T * per_frame * out_w;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x)
    {
        const int64_t p = i / out_w;
        const int f = (int)(i - p * out_w);
        float v = 0.f;
        if (f < kPatchFeatures)
        {
            const int q = f / kLatentChannels, c = f - q * kLatentChannels;
            const int64_t fr = p / per_frame;
            const int rem = (int)(p - fr * per_frame);
            const int py = rem / pw, px = rem - py * pw;
            const int64_t tok = (fr * H + 2 * py + (q >> 1)) * (int64_t)W + 2 * px + (q & 1);
            v = src.at(tok, c);
        }
        if (BF16)
            static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
        else
            static_cast<float*>(dst)[i] = v;
    }
}

// dst token (frame, yy, xx), channels 4c4..4c4+3 = features (y*2 + x)*16 + 4c4..
// of patch (frame, yy/2, xx/2), y = yy & 1, x = xx & 1 (one float4 per thread).
__global__ void unpatchify_kernel(const float4* __restrict__ src, int T, int H, int W, float4* __restrict__ dst)
{
    const int ph = H >> 1, pw = W >> 1;
    const int64_t hw = (int64_t)H * W;
    const int64_t total = (int64_t)T * hw * (kPredChannels / 4);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x)
    {
        const int64_t tok = i >> 2;
        const int c4 = (int)(i & 3);
        const int64_t fr = tok / hw;
        const int rem = (int)(tok - fr * hw);
        const int yy = rem / W, xx = rem - yy * W;
        const int64_t p = (fr * ph + (yy >> 1)) * pw + (xx >> 1);
        const int q = (yy & 1) * 2 + (xx & 1);
        dst[i] = __ldg(src + p * (kPredFeatures / 4) + q * (kPredChannels / 4) + c4);
    }
}

// out[s][k] = sin(t_s * f_k), out[s][128 + k] = cos(t_s * f_k).  The 128
// frequencies come from the host, computed with the reference's expression,
// so the phase is the reference's fp32 product.
struct TimestepArgs
{
    float freq[kTimeFeatures / 2];
    float t[kTimestepChunk];
    int batch;
};

__global__ void timestep_kernel(const TimestepArgs a, float* __restrict__ out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int half = kTimeFeatures / 2;
    if (i >= a.batch * half) return;
    const int s = i / half, k = i - s * half;
    const float phase = a.t[s] * a.freq[k];
    out[(size_t)s * kTimeFeatures + k] = sinf(phase);
    out[(size_t)s * kTimeFeatures + half + k] = cosf(phase);
}

// y(b, n) = act(bias[n] + sum_k W[n][k] x[b][k]) for up to kGemvRows batch
// rows; one warp per output n streams W's row once (16-byte loads) and keeps
// one fp32 sum per batch row.  y(b, n) lands at
// y[(n / chunk) * s_chunk + b * s_b + n % chunk].
template <int ACT>
__global__ void __launch_bounds__(256) gemv_kernel(const __nv_bfloat16* __restrict__ W, const float* __restrict__ bias,
                                                   int N, int K, const float* __restrict__ x, int ldx, int B,
                                                   float* __restrict__ y, int chunk, int64_t s_chunk, int64_t s_b)
{
    const int n = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    const __nv_bfloat16* w = W + (size_t)n * K;
    float acc[kGemvRows];
#pragma unroll
    for (int b = 0; b < kGemvRows; b++) acc[b] = 0.f;
#pragma unroll 2
    for (int k = lane * 8; k < K; k += 256)
    {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(w + k));
        float wf[8];
        float2 f;
        f = unpack_bf16x2(u.x), wf[0] = f.x, wf[1] = f.y;
        f = unpack_bf16x2(u.y), wf[2] = f.x, wf[3] = f.y;
        f = unpack_bf16x2(u.z), wf[4] = f.x, wf[5] = f.y;
        f = unpack_bf16x2(u.w), wf[6] = f.x, wf[7] = f.y;
#pragma unroll
        for (int b = 0; b < kGemvRows; b++)
        {
            if (b >= B) break;
            const float4 x0 = __ldg(reinterpret_cast<const float4*>(x + (size_t)b * ldx + k));
            const float4 x1 = __ldg(reinterpret_cast<const float4*>(x + (size_t)b * ldx + k + 4));
            acc[b] += wf[0] * x0.x + wf[1] * x0.y + wf[2] * x0.z + wf[3] * x0.w + wf[4] * x1.x + wf[5] * x1.y +
                      wf[6] * x1.z + wf[7] * x1.w;
        }
    }
    const float bn = bias ? __ldg(bias + n) : 0.f;
    const int64_t col = (int64_t)(n / chunk) * s_chunk + (n % chunk);
#pragma unroll
    for (int b = 0; b < kGemvRows; b++)
    {
        if (b >= B) break;
        float v = acc[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0)
        {
            v += bn;
            if (ACT == 1) v = v / (1.f + expf(-v)); // SiLU
            y[col + (int64_t)b * s_b] = v;
        }
    }
}

// apply_cfg (seedvr2_pipeline.cpp:171-210), deterministic two-level double
// reductions (per-block partials in a fixed grid, summed in block order by one
// block):
//   combine: cfg = neg + scale * (pos - neg) (no contraction, as the reference),
//            partial sums of pos and cfg;
//   PASS 0 finish: means; deviations: partial sums of squared deviations;
//   PASS 1 finish: factor = float(rescale * std(pos) / std(cfg) + (1 - rescale)),
//            1 when std(cfg) == 0.
constexpr int kCfgBlocks = 512;
constexpr int kCfgThreads = 256;

__device__ __forceinline__ double2 block_sum2(double a, double b)
{
    __shared__ double sa[kCfgThreads / 32], sb[kCfgThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) sa[w] = a, sb[w] = b;
    __syncthreads();
    double2 r = make_double2(0.0, 0.0);
    if (threadIdx.x == 0)
        for (int i = 0; i < kCfgThreads / 32; i++) r.x += sa[i], r.y += sb[i];
    return r;
}

__global__ void __launch_bounds__(kCfgThreads) cfg_combine_kernel(const float* __restrict__ pos,
                                                                  const float* __restrict__ neg, int64_t n,
                                                                  float scale, float* __restrict__ out,
                                                                  double2* __restrict__ partial)
{
    double sp = 0.0, sc = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    {
        const float p = pos[i], q = neg[i];
        const float c = __fadd_rn(q, __fmul_rn(scale, __fsub_rn(p, q)));
        out[i] = c;
        sp += (double)p;
        sc += (double)c;
    }
    if (!partial) return;
    const double2 r = block_sum2(sp, sc);
    if (threadIdx.x == 0) partial[blockIdx.x] = r;
}

__global__ void __launch_bounds__(kCfgThreads) cfg_deviation_kernel(const float* __restrict__ pos,
                                                                    const float* __restrict__ cfg, int64_t n,
                                                                    const double* __restrict__ means,
                                                                    double2* __restrict__ partial)
{
    const double pm = means[0], cm = means[1];
    double vp = 0.0, vc = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    {
        const double p = (double)pos[i] - pm, c = (double)cfg[i] - cm;
        vp = __dadd_rn(vp, __dmul_rn(p, p));
        vc = __dadd_rn(vc, __dmul_rn(c, c));
    }
    const double2 r = block_sum2(vp, vc);
    if (threadIdx.x == 0) partial[blockIdx.x] = r;
}

template <int PASS>
__global__ void __launch_bounds__(kCfgThreads) cfg_finish_kernel(const double2* __restrict__ partial, int blocks,
                                                                 int64_t n, float rescale, double* __restrict__ means,
                                                                 float* __restrict__ factor)
{
    double a = 0.0, b = 0.0;
    for (int i = threadIdx.x; i < blocks; i += blockDim.x) a += partial[i].x, b += partial[i].y;
    const double2 r = block_sum2(a, b);
    if (threadIdx.x != 0) return;
    if (PASS == 0)
    {
        means[0] = r.x / (double)n;
        means[1] = r.y / (double)n;
    }
    else
    {
        const double pos_std = sqrt(r.x / (double)(n - 1));
        const double cfg_std = sqrt(r.y / (double)(n - 1));
        *factor = cfg_std == 0.0 ? 1.f : (float)((double)rescale * pos_std / cfg_std + (double)(1.f - rescale));
    }
}

__global__ void scale_kernel(float* __restrict__ x, int64_t n, const float* __restrict__ factor)
{
    const float f = *factor;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = __fmul_rn(x[i], f);
}

// Euler step of SeedVR2Pipeline::denoise (seedvr2_pipeline.cpp:572-586):
// latent[c][t] += delta * (pred[t][c] * factor), factor from apply_cfg's
// rescale (null: none); products and sums rounded separately, as the reference.
__global__ void euler_kernel(float* __restrict__ latent, int64_t cstep, int64_t tokens,
                             const float* __restrict__ pred, const float* __restrict__ factor, float delta)
{
    const float f = factor ? *factor : 1.f;
    const int64_t n = tokens * kPredChannels;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    {
        const int c = (int)(i / tokens);
        const int64_t t = i - (int64_t)c * tokens;
        float v = __ldg(pred + t * kPredChannels + c);
        if (factor) v = __fmul_rn(v, f);
        float* l = latent + c * cstep + t;
        *l = __fadd_rn(*l, __fmul_rn(delta, v));
    }
}

} // namespace

int patchify_rows(const int* shapes, int batch, int rows, int64_t* patches)
{
    // patchify_video's checks (seedvr2_dit.cpp:172-193)
    if (batch < 0 || (batch > 0 && !shapes)) return S2_ERR_INVALID;
    int64_t nt = 0, np = 0;
    for (int s = 0; s < batch; s++)
    {
        const int t = shapes[3 * s], h = shapes[3 * s + 1], w = shapes[3 * s + 2];
        if (t <= 0 || h <= 0 || w <= 0 || (h & 1) || (w & 1)) return S2_ERR_INVALID;
        nt += (int64_t)t * h * w;
        np += (int64_t)t * (h / 2) * (w / 2);
    }
    if (nt != rows) return S2_ERR_INVALID;
    if (np == 0) return S2_ERR_ALLOC; // the reference's Mat::create of zero rows fails
    if (patches) *patches = np;
    return S2_OK;
}

int unpatchify_rows(const int* shapes, int batch, int rows, int64_t* tokens)
{
    // unpatchify_prediction's checks (seedvr2_dit.cpp:261-285): even h/w and
    // matching rows; a zero-extent sample adds no rows; negative extents are
    // invalid
    if (batch < 0 || (batch > 0 && !shapes)) return S2_ERR_INVALID;
    int64_t nt = 0, np = 0;
    for (int s = 0; s < batch; s++)
    {
        const int t = shapes[3 * s], h = shapes[3 * s + 1], w = shapes[3 * s + 2];
        if (t < 0 || h < 0 || w < 0 || (h & 1) || (w & 1)) return S2_ERR_INVALID;
        nt += (int64_t)t * h * w;
        np += (int64_t)t * (h / 2) * (w / 2);
    }
    if (np != rows) return S2_ERR_INVALID;
    if (nt == 0) return S2_ERR_ALLOC;
    if (tokens) *tokens = nt;
    return S2_OK;
}

int launch_patchify(Context& ctx, const float* src, int T, int H, int W, void* dst, int bf16_out)
{
    if (T <= 0 || H <= 0 || W <= 0 || (H & 1) || (W & 1) || !src || !dst) return S2_ERR_INVALID;
    const int out_w = bf16_out ? kPatchPitch : kPatchFeatures;
    const int64_t patches = (int64_t)T * (H / 2) * (W / 2);
    const int64_t total = patches * out_w;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)patches * (kPatchFeatures * 4.0 + out_w * (bf16_out ? 2.0 : 4.0)));
    const int grid = grid_for(ctx, total, 256);
    const PatchSource ps = {src, nullptr, 0, nullptr, 0};
    if (bf16_out)
        patchify_kernel<true><<<grid, 256, 0, ctx.stream>>>(ps, T, H, W, dst, out_w);
    else
        patchify_kernel<false><<<grid, 256, 0, ctx.stream>>>(ps, T, H, W, dst, out_w);
    return launched(ctx);
}

int launch_patchify_planar(Context& ctx, const float* latent, int64_t latent_cstep, const float* condition,
                           int64_t condition_cstep, int T, int H, int W, void* dst)
{
    if (T <= 0 || H <= 0 || W <= 0 || (H & 1) || (W & 1) || !latent || !condition || !dst) return S2_ERR_INVALID;
    const int64_t tokens = (int64_t)T * H * W;
    if (latent_cstep < tokens || condition_cstep < tokens) return S2_ERR_INVALID;
    const int64_t patches = tokens / 4;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)tokens * 32 * 4.0 + (double)patches * kPatchPitch * 2.0);
    const int grid = grid_for(ctx, patches * kPatchPitch, 256);
    const PatchSource ps = {nullptr, latent, latent_cstep, condition, condition_cstep};
    patchify_kernel<true><<<grid, 256, 0, ctx.stream>>>(ps, T, H, W, dst, kPatchPitch);
    return launched(ctx);
}

size_t cfg_scratch_bytes()
{
    return (size_t)kCfgBlocks * sizeof(double2) + 2 * sizeof(double) + 16;
}

int launch_apply_cfg(Context& ctx, const float* pos, const float* neg, int64_t n, float scale, float rescale,
                     float* out, void* scratch, int apply_factor, const float** factor_out)
{
    if (n <= 0 || !pos || !neg || !out || !scratch) return S2_ERR_INVALID;
    double2* partial = static_cast<double2*>(scratch);
    double* means = reinterpret_cast<double*>(partial + kCfgBlocks);
    float* factor = reinterpret_cast<float*>(means + 2);
    const bool rescaled = rescale != 0.f && n >= 2;
    if (factor_out) *factor_out = rescaled ? factor : nullptr;
    int64_t b = (n + kCfgThreads - 1) / kCfgThreads;
    const int blocks = (int)(b < kCfgBlocks ? b : kCfgBlocks);
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)n * (rescaled ? 24.0 : 12.0));
    cfg_combine_kernel<<<blocks, kCfgThreads, 0, ctx.stream>>>(pos, neg, n, scale, out, rescaled ? partial : nullptr);
    int r = launched(ctx);
    if (r != S2_OK || !rescaled) return r;
    cfg_finish_kernel<0><<<1, kCfgThreads, 0, ctx.stream>>>(partial, blocks, n, rescale, means, factor);
    if ((r = launched(ctx)) != S2_OK) return r;
    cfg_deviation_kernel<<<blocks, kCfgThreads, 0, ctx.stream>>>(pos, out, n, means, partial);
    if ((r = launched(ctx)) != S2_OK) return r;
    cfg_finish_kernel<1><<<1, kCfgThreads, 0, ctx.stream>>>(partial, blocks, n, rescale, means, factor);
    if ((r = launched(ctx)) != S2_OK) return r;
    if (apply_factor)
    {
        scale_kernel<<<grid_for(ctx, n, 256), 256, 0, ctx.stream>>>(out, n, factor);
        r = launched(ctx);
    }
    return r;
}

int launch_euler(Context& ctx, float* latent, int64_t cstep, int64_t tokens, const float* pred, const float* factor,
                 float delta)
{
    if (tokens <= 0 || cstep < tokens || !latent || !pred) return S2_ERR_INVALID;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)tokens * kPredChannels * 12.0);
    euler_kernel<<<grid_for(ctx, tokens * kPredChannels, 256), 256, 0, ctx.stream>>>(latent, cstep, tokens, pred,
                                                                                      factor, delta);
    return launched(ctx);
}

int launch_unpatchify(Context& ctx, const float* src, int T, int H, int W, float* dst)
{
    if (T < 0 || H < 0 || W < 0 || (H & 1) || (W & 1) || !src || !dst) return S2_ERR_INVALID;
    if ((int64_t)T * H * W == 0) return S2_OK;
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) return S2_ERR_INVALID;
    const int64_t tokens = (int64_t)T * H * W;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)tokens * kPredChannels * 8.0);
    const int grid = grid_for(ctx, tokens * (kPredChannels / 4), 256);
    unpatchify_kernel<<<grid, 256, 0, ctx.stream>>>(reinterpret_cast<const float4*>(src), T, H, W,
                                                    reinterpret_cast<float4*>(dst));
    return launched(ctx);
}

int launch_timestep_embedding(Context& ctx, const float* timesteps, int batch, float* out)
{
    if (batch <= 0 || !timesteps || !out) return S2_ERR_INVALID;
    TimestepArgs a;
    const int half = kTimeFeatures / 2;
    for (int i = 0; i < half; i++)
    {
        // make_timestep_embedding's expression, evaluated by the host libm
        const float exponent = -std::log(10000.f) * i / half;
        a.freq[i] = std::exp(exponent);
    }
    for (int s0 = 0; s0 < batch; s0 += kTimestepChunk)
    {
        a.batch = batch - s0 < kTimestepChunk ? batch - s0 : kTimestepChunk;
        for (int s = 0; s < a.batch; s++)
        {
            if (!std::isfinite(timesteps[s0 + s])) return S2_ERR_INVALID;
            a.t[s] = timesteps[s0 + s];
        }
        ProfileScope prof(ctx, K_OTHER, 0.0, (double)a.batch * kTimeFeatures * 4.0);
        timestep_kernel<<<(a.batch * half + 127) / 128, 128, 0, ctx.stream>>>(a, out + (size_t)s0 * kTimeFeatures);
        const int r = launched(ctx);
        if (r != S2_OK) return r;
    }
    return S2_OK;
}

int launch_gemv(Context& ctx, const void* W, const float* bias, int N, int K, const float* x, int ldx, int B, int act,
                float* y, int chunk, int64_t s_chunk, int64_t s_b)
{
    if (N <= 0 || K <= 0 || K % 8 || ldx % 4 || B <= 0 || chunk <= 0 || !W || !x || !y) return S2_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(x)) & 15) return S2_ERR_INVALID;
    for (int b0 = 0; b0 < B; b0 += kGemvRows)
    {
        const int nb = B - b0 < kGemvRows ? B - b0 : kGemvRows;
        ProfileScope prof(ctx, K_OTHER, 2.0 * N * K * nb, (double)N * K * 2.0 + (double)nb * (K + N) * 4.0);
        const int grid = (int)(((int64_t)N * 32 + 255) / 256);
        const float* xb = x + (size_t)b0 * ldx;
        float* yb = y + (int64_t)b0 * s_b;
        if (act)
            gemv_kernel<1><<<grid, 256, 0, ctx.stream>>>(static_cast<const __nv_bfloat16*>(W), bias, N, K, xb, ldx,
                                                         nb, yb, chunk, s_chunk, s_b);
        else
            gemv_kernel<0><<<grid, 256, 0, ctx.stream>>>(static_cast<const __nv_bfloat16*>(W), bias, N, K, xb, ldx,
                                                         nb, yb, chunk, s_chunk, s_b);
        const int r = launched(ctx);
        if (r != S2_OK) return r;
    }
    return S2_OK;
}

} // namespace s2
