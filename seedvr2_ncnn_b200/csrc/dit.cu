// DiT block stack: the 32 fused blocks of blocks/seedvr2_blocks.ncnn run as
// a fixed sequence of this library's kernels (replaces the ncnn block graph
// that SeedVR2DiTBlocks::load registers the custom layers into and
// record_blocks walks, seedvr2_dit.cpp:531-634, :636-1094).
//
// Per block (the exported graph is not part of the reference tree; this op
// sequence is the assumption the CPU oracle restates in s2o_block_forward):
//   h   = rmsnorm(x) * (mod[1] + ada[1]) + (mod[0] + ada[0])          bf16
//   qkv = SharedLinear_qkv(h)                                        bf16
//   ctx = AdaptiveWindowAttention(qkv)   (odd blocks: shifted windows) bf16
//   x  += SharedLinear_out(ctx) * (mod[2] + ada[2])                  fp32
//   h   = rmsnorm(x) * (mod[4] + ada[4]) + (mod[3] + ada[3])          bf16
//   u   = gelu_tanh(SharedLinear_up(h))                              bf16
//   x  += SharedLinear_down(u) * (mod[5] + ada[5])                   fp32
// x holds the video rows then the text rows of one sample, so every
// token-wise op is a single launch over both streams.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <vector>

#include "s2_common.cuh"
#include "s2_internal.h"
#include "s2_objects.h"

struct s2_dit
{
    s2_context* ctx = nullptr;
    s2_dit_config cfg;
    struct Block
    {
        __nv_bfloat16 *w_qkv, *w_out, *w_up, *w_down;
        float *b_qkv, *b_out, *b_up, *b_down;
        float* qk_norm;
        float* freqs;
        int norm_layer = 0; // the block's two AdaLN norms: 0 RMSNorm, 1 LayerNorm
    };
    std::vector<Block> blocks;
    float* ada_all = nullptr; // [blocks][6][D]
    void* weights = nullptr;  // one allocation for all weights
    size_t weight_bytes = 0;
    // per-shape plans (unshifted, shifted)
    std::map<std::vector<int>, std::unique_ptr<s2_plan>> plans;
    s2::DeviceBuffer act; // activations of one forward
    s2::DeviceBuffer mods; // [blocks][6][D]
    s2::DeviceBuffer host_x; // staging for s2_dit_forward_host
    // s2_dit_forward_host_async: two staging buffers used in turn, an upload
    // and a download stream beside the context's compute stream, and per
    // buffer the events that order the three
    struct HostPipe
    {
        s2::DeviceBuffer x[2];
        cudaStream_t up = nullptr, down = nullptr;
        cudaEvent_t uploaded[2] = {}, computed[2] = {}, downloaded[2] = {};
        int next = 0;
        bool ready = false;
    } pipe;
    // RoPE rotation tables [blocks][rope_pos][pairs] (cos, sin), rebuilt when
    // the weights change or a shape needs more positions
    s2::DeviceBuffer rope;
    int rope_pos = 0;
    bool rope_stale = true;
    // multi-GPU: ownership plan and schedules per (shape, text, rank, world)
    struct Shard
    {
        s2::ShardPlan sp;
        s2::AttnSchedule sched[2];
        // Peer-visible exchange buffer (same layout on every rank):
        // fused QKV packing (D % 256 == 0): packed Q | K | V [R][D] bf16, written
        //   by every rank's QKV projection for the windows this rank owns;
        // otherwise qkv [E][3D] bf16 rows pushed to window owners;
        // then ctx [E][D] bf16 | text partial [2][T][D] f32 | flags.
        // The text partial is double-buffered by block parity: a block without
        // row pushes has no first barrier, so a rank may write block b+1's
        // partial while a slower rank still sums block b's.
        void* xbuf = nullptr;
        bool fused = false;
        size_t off_q = 0, off_k = 0, off_v = 0; // packed Q/K/V (fused)
        size_t off_ctx = 0, off_text = 0, off_flags = 0;
        std::vector<void*> peer_q, peer_k, peer_v;
        // fused: per plan, own row -> packed row at the window owner (peer field)
        // and its RoPE positions (window-local (t + T, h, w))
        int* d_pack[2] = {nullptr, nullptr}; // [n] dst | [n][3] positions
        int max_pos = 0;                     // 1 + largest RoPE position this rank uses
        std::vector<void*> base;                     // every rank's xbuf (mapped)
        std::vector<void*> peer_qkv, peer_ctx, peer_text[2], peer_flags;
        int4* d_push[2] = {nullptr, nullptr};        // {own row, rank, row there, 0}
        int push_count[2] = {0, 0};
        bool any_push[2] = {false, false};           // some rank pushes rows for this plan
        ~Shard()
        {
            for (int p = 0; p < 2; p++)
            {
                if (d_push[p]) cudaFree(d_push[p]);
                if (d_pack[p]) cudaFree(d_pack[p]);
            }
            if (xbuf) cudaFree(xbuf);
        }
    };
    std::map<std::vector<int>, std::unique_ptr<Shard>> shards;
    // frontend / tail nets (s2_dit_set_io_weights, s2_dit_init_random); one
    // allocation made on first use
    struct Io
    {
        __nv_bfloat16 *w_vid_in, *w_txt_in, *w_emb0, *w_emb1, *w_emb2, *w_out;
        float *b_vid_in, *b_txt_in, *b_emb0, *b_emb1, *b_emb2, *tail_ada, *b_out;
    } io = {};
    void* io_weights = nullptr;
    bool io_loaded = false;
    s2::DeviceBuffer io_ws;   // frontend / tail activations
    s2::DeviceBuffer io_host; // staging of s2_dit_forward_step_host
    // finite checks (s2_dit_set_check_finite): NaN / Inf counters of the
    // video and text rows at the block stack's input and after every block,
    // [blocks + 1][2]; the last checked forward's first non-finite point
    bool check_finite = false;
    s2::DeviceBuffer finite;
    bool finite_checked = false;
    int nonfinite_block = 0;
    int64_t nonfinite_video = 0, nonfinite_text = 0;
    // block checkpoints (s2_dit_set_checkpoints): caller-owned device
    // destinations of chosen blocks' outputs; s2_dit_forward_host sets the
    // row offsets of the sample it runs
    struct Checkpoint
    {
        int block;
        float* video;
        float* text;
    };
    std::vector<Checkpoint> checkpoints;
    size_t cp_video_row = 0, cp_text_row = 0;
};

namespace {

size_t align256(size_t b)
{
    return (b + 255) & ~size_t(255);
}

// NaN / Inf counts of the residual's video rows [Nv][D] and text rows
// [Nt][D] into counters[0] / counters[1].
int count_rows_nonfinite(s2::Context& c, const float* x, int Nv, int Nt, int D, unsigned long long* counters)
{
    const int r = s2::launch_count_nonfinite(c, x, (int64_t)Nv * D, S2_DTYPE_F32, counters);
    if (r != S2_OK) return r;
    return s2::launch_count_nonfinite(c, x + (size_t)Nv * D, (int64_t)Nt * D, S2_DTYPE_F32, counters + 1);
}

int get_plan(s2_dit* d, const int* shape, int shifted, s2_plan** out)
{
    std::vector<int> key(shape, shape + 3);
    key.push_back(shifted);
    std::unique_ptr<s2_plan>& slot = d->plans[key];
    if (!slot)
    {
        std::unique_ptr<s2_plan> p(new s2_plan);
        const int r = s2::build_plan(shape, 1, d->cfg.window, d->cfg.window_mode, shifted, p->plan);
        if (r != S2_OK)
        {
            d->plans.erase(key);
            return r;
        }
        slot = std::move(p);
    }
    *out = slot.get();
    return S2_OK;
}

// ---------------------------------------------------------------- frontend / tail
// Weights of the frontend and tail nets, one allocation: bf16 w_vid_in
// [D][kPatchPitch] (zero columns 132..135) | w_txt_in [D][5120] | w_emb0
// [D][256] | w_emb1 [D][D] | w_emb2 [6D][D] | w_out [64][D], then fp32
// b_vid_in, b_txt_in, b_emb0, b_emb1 [D] | b_emb2 [6D] | tail_ada [2][D] | b_out [64].
int ensure_io_weights(s2_dit* d)
{
    if (d->io_weights) return S2_OK;
    const size_t D = d->cfg.hidden;
    const size_t n_bf16 = D * s2::kPatchPitch + D * s2::kTextChannels + D * s2::kTimeFeatures + D * D + 6 * D * D +
                          (size_t)s2::kPredFeatures * D;
    const size_t n_f32 = 10 * D + 2 * D + s2::kPredFeatures;
    const size_t bytes = align256(n_bf16 * 2) + align256(n_f32 * 4);
    if (cudaMalloc(&d->io_weights, bytes) != cudaSuccess)
    {
        d->io_weights = nullptr;
        return S2_ERR_ALLOC;
    }
    if (cudaMemset(d->io_weights, 0, bytes) != cudaSuccess) return S2_ERR_CUDA;
    s2_dit::Io& io = d->io;
    __nv_bfloat16* w = static_cast<__nv_bfloat16*>(d->io_weights);
    io.w_vid_in = w, w += D * s2::kPatchPitch;
    io.w_txt_in = w, w += D * s2::kTextChannels;
    io.w_emb0 = w, w += D * s2::kTimeFeatures;
    io.w_emb1 = w, w += D * D;
    io.w_emb2 = w, w += 6 * D * D;
    io.w_out = w;
    float* f = reinterpret_cast<float*>(static_cast<uint8_t*>(d->io_weights) + align256(n_bf16 * 2));
    io.b_vid_in = f, f += D;
    io.b_txt_in = f, f += D;
    io.b_emb0 = f, f += D;
    io.b_emb1 = f, f += D;
    io.b_emb2 = f, f += 6 * D;
    io.tail_ada = f, f += 2 * D;
    io.b_out = f;
    return S2_OK;
}

// Seeded synthetic frontend / tail weights (streams disjoint from the blocks').
int init_io_random(s2_dit* d, uint64_t seed)
{
    int r = ensure_io_weights(d);
    if (r != S2_OK) return r;
    s2::Context& c = d->ctx->c;
    const int64_t D = d->cfg.hidden;
    const s2_dit::Io& io = d->io;
    const uint64_t s = seed * 1000003ull + (uint64_t)d->cfg.num_blocks * 64 + 7;
    r = s2::launch_fill_normal_bf16(c, io.w_vid_in, D * s2::kPatchPitch, s + 1, 0.f, 0.02f);
    if (r == S2_OK && cudaMemset2DAsync(io.w_vid_in + s2::kPatchFeatures, s2::kPatchPitch * 2, 0,
                                        (s2::kPatchPitch - s2::kPatchFeatures) * 2, D, c.stream) != cudaSuccess)
        r = S2_ERR_CUDA;
    if (r == S2_OK) r = s2::launch_fill_normal_bf16(c, io.w_txt_in, D * s2::kTextChannels, s + 2, 0.f, 0.02f);
    if (r == S2_OK) r = s2::launch_fill_normal_bf16(c, io.w_emb0, D * s2::kTimeFeatures, s + 3, 0.f, 0.02f);
    if (r == S2_OK) r = s2::launch_fill_normal_bf16(c, io.w_emb1, D * D, s + 4, 0.f, 0.02f);
    if (r == S2_OK) r = s2::launch_fill_normal_bf16(c, io.w_emb2, 6 * D * D, s + 5, 0.f, 0.02f);
    if (r == S2_OK) r = s2::launch_fill_normal_bf16(c, io.w_out, s2::kPredFeatures * D, s + 6, 0.f, 0.02f);
    if (r == S2_OK) r = s2::launch_fill_normal_f32(c, io.b_vid_in, 10 * D, s + 7, 0.f, 0.02f);
    const float sd = 1.f / std::sqrt((float)D);
    if (r == S2_OK) r = s2::launch_fill_normal_f32(c, io.tail_ada, D, s + 8, 0.f, sd);
    if (r == S2_OK) r = s2::launch_fill_normal_f32(c, io.tail_ada + D, D, s + 9, 1.f, sd);
    if (r == S2_OK) r = s2::launch_fill_normal_f32(c, io.b_out, s2::kPredFeatures, s + 10, 0.f, 0.02f);
    if (r == S2_OK) d->io_loaded = true;
    return r;
}

// split_dit_inputs_by_sample's checks (seedvr2_dit.cpp:369-427) plus
// patchify_video's even h/w (:178-184).  Sums the rows per side.
int check_dit_inputs(const int* shapes, const int* text_lengths, const float* timesteps, int batch, int video_rows,
                     int text_rows, int64_t* patches_total)
{
    if (!shapes || !text_lengths || !timesteps || batch <= 0 || video_rows <= 0 || text_rows <= 0)
        return S2_ERR_INVALID;
    int64_t v = 0, t = 0, p = 0;
    for (int s = 0; s < batch; s++)
    {
        const int* shp = shapes + 3 * s;
        if (shp[0] <= 0 || shp[1] <= 0 || shp[2] <= 0 || text_lengths[s] <= 0 || !std::isfinite(timesteps[s]))
            return S2_ERR_INVALID;
        if ((shp[1] & 1) || (shp[2] & 1)) return S2_ERR_INVALID;
        const int64_t tok = (int64_t)shp[0] * shp[1] * shp[2];
        if (tok > 0x7fffffff) return S2_ERR_INVALID;
        v += tok;
        t += text_lengths[s];
        p += tok / 4;
    }
    if (v != video_rows || t != text_rows) return S2_ERR_INVALID;
    if (patches_total) *patches_total = p;
    return S2_OK;
}

// Timestep embedding and the frontend's timestep MLP for `batch` samples:
// temb [B][256] -> e0, e1 [B][D] -> modulation, stored [6][B][D] (ref_layout,
// the frontend's out2..out7) or [B][6][D] (one [6][D] block per sample).
int run_emb(s2_dit* d, const float* timesteps, int batch, float* temb, float* e0, float* e1, float* mod,
            bool ref_layout)
{
    s2::Context& c = d->ctx->c;
    const int D = d->cfg.hidden;
    const s2_dit::Io& io = d->io;
    int r = s2::launch_timestep_embedding(c, timesteps, batch, temb);
    if (r == S2_OK)
        r = s2::launch_gemv(c, io.w_emb0, io.b_emb0, D, s2::kTimeFeatures, temb, s2::kTimeFeatures, batch, 1, e0, D,
                            0, D);
    if (r == S2_OK) r = s2::launch_gemv(c, io.w_emb1, io.b_emb1, D, D, e0, D, batch, 1, e1, D, 0, D);
    if (r == S2_OK)
        r = ref_layout ? s2::launch_gemv(c, io.w_emb2, io.b_emb2, 6 * D, D, e1, D, batch, 0, mod, D, (int64_t)batch * D,
                                         D)
                       : s2::launch_gemv(c, io.w_emb2, io.b_emb2, 6 * D, D, e1, D, batch, 0, mod, 6 * D, 0, 6 * D);
    return r;
}

// Tail net + unpatchify for one sample: x = its [patches][D] block output,
// mod0 / mod1 = its shift / scale modulation rows.  h [patches][D] bf16,
// pp [patches][64] fp32 and tm [2][D] fp32 are workspace.
int run_tail(s2_dit* d, const int* shape, const float* x, const float* mod0, const float* mod1, float* pred,
             __nv_bfloat16* h, float* pp, float* tm)
{
    s2::Context& c = d->ctx->c;
    const int D = d->cfg.hidden;
    const s2_dit::Io& io = d->io;
    const int np = shape[0] * (shape[1] / 2) * (shape[2] / 2);
    int r = s2::launch_add_vectors(c, io.tail_ada, mod0, tm, D, D);
    if (r == S2_OK) r = s2::launch_add_vectors(c, io.tail_ada + D, mod1, tm + D, D, D);
    if (r == S2_OK) r = s2::launch_ada_rmsnorm(c, np, D, x, d->cfg.norm_eps, tm, tm + D, h);
    if (r == S2_OK)
        r = s2::launch_shared_linear(c, np, 0, s2::kPredFeatures, D, h, nullptr, io.w_out, io.b_out, s2::EPI_STORE,
                                     nullptr, 1, pp, nullptr);
    if (r == S2_OK) r = s2::launch_unpatchify(c, pp, shape[0], shape[1], shape[2], pred);
    return r;
}

// Activations of one whole-DiT pass, carved out of io_ws: x [np + T][D] f32 |
// patches bf16 [np][136] | text bf16 [T][5120] | h bf16 [np][D] | pp [np][64] |
// tm [2][D] | temb [B][256] | e0, e1 [B][D] | emb [B][6][D] | `extra` bytes.
struct StepWs
{
    float* x;
    __nv_bfloat16 *patches, *tb, *h;
    float *pp, *tm, *temb, *e0, *e1, *emb;
    void* extra;
};

int step_workspace(s2_dit* d, int64_t np_max, int64_t nt_max, int batch, size_t extra, StepWs& w)
{
    const int D = d->cfg.hidden;
    const size_t sz[11] = {align256((size_t)(np_max + nt_max) * D * 4),
                           align256((size_t)np_max * s2::kPatchPitch * 2),
                           align256((size_t)nt_max * s2::kTextChannels * 2),
                           align256((size_t)np_max * D * 2),
                           align256((size_t)np_max * s2::kPredFeatures * 4),
                           align256((size_t)2 * D * 4),
                           align256((size_t)batch * s2::kTimeFeatures * 4),
                           align256((size_t)batch * D * 4),
                           align256((size_t)batch * D * 4),
                           align256((size_t)batch * 6 * D * 4),
                           align256(extra)};
    size_t total = 0;
    for (size_t b : sz) total += b;
    const int r = d->io_ws.ensure(total);
    if (r != S2_OK) return r;
    uint8_t* p = static_cast<uint8_t*>(d->io_ws.ptr);
    void* at[11];
    for (int i = 0; i < 11; i++) at[i] = p, p += sz[i];
    w.x = static_cast<float*>(at[0]);
    w.patches = static_cast<__nv_bfloat16*>(at[1]);
    w.tb = static_cast<__nv_bfloat16*>(at[2]);
    w.h = static_cast<__nv_bfloat16*>(at[3]);
    w.pp = static_cast<float*>(at[4]);
    w.tm = static_cast<float*>(at[5]);
    w.temb = static_cast<float*>(at[6]);
    w.e0 = static_cast<float*>(at[7]);
    w.e1 = static_cast<float*>(at[8]);
    w.emb = static_cast<float*>(at[9]);
    w.extra = at[10];
    return S2_OK;
}

// Where a sample's DiT video input comes from: [tokens][33] rows, or the
// latent / condition planes SeedVR2Pipeline::predict assembles them from.
struct PatchSrc
{
    const float* rows;
    const float* latent;
    int64_t latent_cstep;
    const float* condition;
    int64_t condition_cstep;
};

// One sample through frontend (token nets), all blocks and tail: shape = its
// latent (t, h, w), mod = its [6][D] modulation; text_out may be null.
int run_sample(s2_dit* d, const int* shp, const PatchSrc& src, const float* text, int nt, const float* mod,
               float* prediction, float* text_out, const StepWs& w)
{
    s2::Context& c = d->ctx->c;
    const int D = d->cfg.hidden;
    const s2_dit::Io& io = d->io;
    const int pshape[3] = {shp[0], shp[1] / 2, shp[2] / 2};
    const int np = pshape[0] * pshape[1] * pshape[2];
    // frontend: x = [video patches W_vid_in^T + b | text W_txt_in^T + b]
    int r = src.rows ? s2::launch_patchify(c, src.rows, shp[0], shp[1], shp[2], w.patches, 1)
                     : s2::launch_patchify_planar(c, src.latent, src.latent_cstep, src.condition, src.condition_cstep,
                                                  shp[0], shp[1], shp[2], w.patches);
    if (r == S2_OK)
        r = s2::launch_shared_linear(c, np, 0, D, s2::kPatchPitch, w.patches, nullptr, io.w_vid_in, io.b_vid_in,
                                     s2::EPI_STORE, nullptr, 1, w.x, nullptr);
    if (r == S2_OK) r = s2::launch_convert_f32_bf16(c, text, w.tb, (int64_t)nt * s2::kTextChannels);
    if (r == S2_OK)
        r = s2::launch_shared_linear(c, nt, 0, D, s2::kTextChannels, w.tb, nullptr, io.w_txt_in, io.b_txt_in,
                                     s2::EPI_STORE, nullptr, 1, w.x + (size_t)np * D, nullptr);
    // all blocks, in place
    if (r == S2_OK) r = s2_dit_forward(d, pshape, nt, w.x, mod);
    // tail -> prediction tokens; text rows out
    if (r == S2_OK) r = run_tail(d, shp, w.x, mod, mod + D, prediction, w.h, w.pp, w.tm);
    if (r == S2_OK && text_out &&
        cudaMemcpyAsync(text_out, w.x + (size_t)np * D, (size_t)nt * D * 4, cudaMemcpyDeviceToDevice, c.stream) !=
            cudaSuccess)
        r = S2_ERR_CUDA;
    return r;
}

} // namespace

extern "C" {

int s2_dit_create(s2_context* ctx, const s2_dit_config* cfg, s2_dit** out)
{
    if (!ctx || !cfg || !out) return S2_ERR_INVALID;
    *out = nullptr;
    const int D = cfg->hidden, F = cfg->mlp_hidden;
    if (cfg->num_blocks <= 0 || cfg->head_dim != 128 || cfg->heads * cfg->head_dim != D || F <= 0 || F % 64 ||
        cfg->rope_pairs <= 0 || cfg->rope_pairs * 6 > cfg->head_dim)
        return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    std::unique_ptr<s2_dit> d(new s2_dit);
    d->ctx = ctx;
    d->cfg = *cfg;
    const size_t w_elems = (size_t)3 * D * D + (size_t)D * D + (size_t)2 * F * D;
    const size_t per_block = align256(w_elems * 2) + align256((size_t)(3 * D + D + F + D) * 4) +
                             align256((size_t)4 * cfg->head_dim * 4) + align256((size_t)cfg->rope_pairs * 4);
    d->weight_bytes = per_block * cfg->num_blocks + align256((size_t)cfg->num_blocks * 6 * D * 4);
    if (cudaMalloc(&d->weights, d->weight_bytes) != cudaSuccess) return S2_ERR_ALLOC;
    if (cudaMemset(d->weights, 0, d->weight_bytes) != cudaSuccess) return S2_ERR_CUDA;
    uint8_t* p = static_cast<uint8_t*>(d->weights);
    d->blocks.resize(cfg->num_blocks);
    for (int b = 0; b < cfg->num_blocks; b++)
    {
        s2_dit::Block& bl = d->blocks[b];
        uint8_t* q = p + per_block * b;
        bl.w_qkv = reinterpret_cast<__nv_bfloat16*>(q);
        bl.w_out = bl.w_qkv + (size_t)3 * D * D;
        bl.w_up = bl.w_out + (size_t)D * D;
        bl.w_down = bl.w_up + (size_t)F * D;
        q += align256(w_elems * 2);
        bl.b_qkv = reinterpret_cast<float*>(q);
        bl.b_out = bl.b_qkv + 3 * D;
        bl.b_up = bl.b_out + D;
        bl.b_down = bl.b_up + F;
        q += align256((size_t)(3 * D + D + F + D) * 4);
        bl.qk_norm = reinterpret_cast<float*>(q);
        q += align256((size_t)4 * cfg->head_dim * 4);
        bl.freqs = reinterpret_cast<float*>(q);
    }
    d->ada_all = reinterpret_cast<float*>(p + per_block * cfg->num_blocks);
    *out = d.release();
    return S2_OK;
}

void s2_dit_free(s2_dit* d)
{
    if (!d) return;
    cudaSetDevice(d->ctx->c.device);
    cudaStreamSynchronize(d->ctx->c.stream);
    s2_dit::HostPipe& hp = d->pipe;
    for (cudaStream_t st : {hp.up, hp.down})
        if (st)
        {
            cudaStreamSynchronize(st);
            cudaStreamDestroy(st);
        }
    for (int b = 0; b < 2; b++)
        for (cudaEvent_t e : {hp.uploaded[b], hp.computed[b], hp.downloaded[b]})
            if (e) cudaEventDestroy(e);
    d->plans.clear();
    d->shards.clear();
    if (d->weights) cudaFree(d->weights);
    if (d->io_weights) cudaFree(d->io_weights);
    delete d;
}

int s2_dit_set_block_weights(s2_dit* d, int block, const s2_block_host_weights* w)
{
    if (d) d->rope_stale = true;
    if (!d || !w || block < 0 || block >= d->cfg.num_blocks || !w->ada || !w->w_qkv || !w->w_out || !w->w_up ||
        !w->w_down || !w->qk_norm || !w->rope_freqs)
        return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int D = d->cfg.hidden, F = d->cfg.mlp_hidden;
    const s2_dit::Block& bl = d->blocks[block];
    // Upload fp32, convert to bf16 on the device (ncnn use_bf16_storage analogue).
    s2::DeviceBuffer tmp;
    const size_t biggest = (size_t)F * D;
    if (tmp.ensure(biggest * 4) != S2_OK) return S2_ERR_ALLOC;
    auto up_bf16 = [&](const float* src, __nv_bfloat16* dst, size_t n) -> int {
        if (cudaMemcpyAsync(tmp.ptr, src, n * 4, cudaMemcpyHostToDevice, c.stream) != cudaSuccess) return S2_ERR_CUDA;
        return s2::launch_convert_f32_bf16(c, static_cast<float*>(tmp.ptr), dst, (int64_t)n);
    };
    auto up_f32 = [&](const float* src, float* dst, size_t n) -> int {
        if (!src) return cudaMemsetAsync(dst, 0, n * 4, c.stream) == cudaSuccess ? S2_OK : S2_ERR_CUDA;
        return cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyHostToDevice, c.stream) == cudaSuccess ? S2_OK
                                                                                                 : S2_ERR_CUDA;
    };
    int r = S2_OK;
    if (r == S2_OK) r = up_bf16(w->w_qkv, bl.w_qkv, (size_t)3 * D * D);
    if (r == S2_OK) r = up_bf16(w->w_out, bl.w_out, (size_t)D * D);
    if (r == S2_OK) r = up_bf16(w->w_up, bl.w_up, (size_t)F * D);
    if (r == S2_OK) r = up_bf16(w->w_down, bl.w_down, (size_t)D * F);
    if (r == S2_OK) r = up_f32(w->b_qkv, bl.b_qkv, 3 * D);
    if (r == S2_OK) r = up_f32(w->b_out, bl.b_out, D);
    if (r == S2_OK) r = up_f32(w->b_up, bl.b_up, F);
    if (r == S2_OK) r = up_f32(w->b_down, bl.b_down, D);
    if (r == S2_OK) r = up_f32(w->qk_norm, bl.qk_norm, 4 * d->cfg.head_dim);
    if (r == S2_OK) r = up_f32(w->rope_freqs, bl.freqs, d->cfg.rope_pairs);
    if (r == S2_OK) r = up_f32(w->ada, d->ada_all + (size_t)block * 6 * D, 6 * D);
    if (r == S2_OK && cudaStreamSynchronize(c.stream) != cudaSuccess) r = S2_ERR_CUDA;
    return r;
}

int s2_dit_set_check_finite(s2_dit* d, int enable)
{
    if (!d) return S2_ERR_INVALID;
    d->check_finite = enable != 0;
    return S2_OK;
}

int s2_dit_set_block_norm(s2_dit* d, int block, int norm_type)
{
    if (!d || block < 0 || block >= d->cfg.num_blocks || (norm_type != S2_NORM_RMS && norm_type != S2_NORM_LAYER))
        return S2_ERR_INVALID;
    d->blocks[block].norm_layer = norm_type == S2_NORM_LAYER;
    return S2_OK;
}

int s2_dit_set_checkpoints(s2_dit* d, const int* blocks, int count, float* const* video, float* const* text)
{
    if (!d || count < 0 || (count > 0 && (!blocks || !video || !text))) return S2_ERR_INVALID;
    std::vector<s2_dit::Checkpoint> cps;
    for (int i = 0; i < count; i++)
    {
        // record_blocks' range check (seedvr2_dit.cpp:820-825)
        if (blocks[i] < 0 || blocks[i] >= d->cfg.num_blocks || !video[i] || !text[i]) return S2_ERR_INVALID;
        cps.push_back({blocks[i], video[i], text[i]});
    }
    d->checkpoints.swap(cps);
    return S2_OK;
}

int s2_dit_nonfinite_report(const s2_dit* d, int* block, int64_t* video_count, int64_t* text_count)
{
    if (!d || !d->finite_checked) return S2_ERR_INVALID;
    if (block) *block = d->nonfinite_block;
    if (video_count) *video_count = d->nonfinite_video;
    if (text_count) *text_count = d->nonfinite_text;
    return S2_OK;
}

int s2_dit_init_random(s2_dit* d, uint64_t seed)
{
    if (d) d->rope_stale = true;
    if (!d) return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int D = d->cfg.hidden, F = d->cfg.mlp_hidden, hd = d->cfg.head_dim, np = d->cfg.rope_pairs;
    std::vector<float> freqs(np);
    for (int i = 0; i < np; i++) freqs[i] = (float)(1.0 / std::pow(10000.0, (2.0 * i) / (2.0 * np)));
    int r = S2_OK;
    for (int b = 0; b < d->cfg.num_blocks && r == S2_OK; b++)
    {
        const s2_dit::Block& bl = d->blocks[b];
        const uint64_t s = seed * 1000003ull + (uint64_t)b * 64;
        r = s2::launch_fill_normal_bf16(c, bl.w_qkv, (int64_t)3 * D * D, s + 1, 0.f, 0.02f);
        if (r == S2_OK) r = s2::launch_fill_normal_bf16(c, bl.w_out, (int64_t)D * D, s + 2, 0.f, 0.02f);
        if (r == S2_OK) r = s2::launch_fill_normal_bf16(c, bl.w_up, (int64_t)F * D, s + 3, 0.f, 0.02f);
        if (r == S2_OK) r = s2::launch_fill_normal_bf16(c, bl.w_down, (int64_t)D * F, s + 4, 0.f, 0.02f);
        if (r == S2_OK) r = s2::launch_fill_normal_f32(c, bl.b_qkv, (int64_t)3 * D + D + F + D, s + 5, 0.f, 0.02f);
        if (r == S2_OK) r = s2::launch_fill_normal_f32(c, bl.qk_norm, (int64_t)4 * hd, s + 6, 1.f, 0.02f);
        if (r == S2_OK)
            r = cudaMemcpyAsync(bl.freqs, freqs.data(), np * 4, cudaMemcpyHostToDevice, c.stream) == cudaSuccess
                    ? S2_OK
                    : S2_ERR_CUDA;
        float* ada = d->ada_all + (size_t)b * 6 * D;
        const float sd = 1.f / std::sqrt((float)D);
        for (int k = 0; k < 6 && r == S2_OK; k++)
            r = s2::launch_fill_normal_f32(c, ada + (size_t)k * D, D, s + 10 + k, (k == 1 || k == 4) ? 1.f : 0.f, sd);
    }
    if (r == S2_OK) r = init_io_random(d, seed);
    if (r == S2_OK && cudaStreamSynchronize(c.stream) != cudaSuccess) r = S2_ERR_CUDA;
    return r;
}

namespace {

// RoPE rotation tables of every block for positions [0, max_pos).
int ensure_rope_tables(s2_dit* d, int max_pos)
{
    if (!d->rope_stale && max_pos <= d->rope_pos) return S2_OK;
    const int np = d->cfg.rope_pairs;
    const int pos = std::max(max_pos, d->rope_pos);
    const size_t per_block = (size_t)pos * np * 8;
    int r = d->rope.ensure(per_block * d->cfg.num_blocks);
    for (int b = 0; b < d->cfg.num_blocks && r == S2_OK; b++)
        r = s2::launch_rope_table(d->ctx->c, d->blocks[b].freqs, np, pos,
                                  static_cast<uint8_t*>(d->rope.ptr) + per_block * b);
    if (r != S2_OK) return r;
    d->rope_pos = pos;
    d->rope_stale = false;
    return S2_OK;
}

} // namespace

int s2_dit_forward(s2_dit* d, const int* video_shape, int text_length, float* x, const float* modulation)
{
    if (!d || !video_shape || text_length <= 0 || !x || !modulation) return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const s2_dit_config& cfg = d->cfg;
    const int D = cfg.hidden, F = cfg.mlp_hidden, H = cfg.heads;
    int r;
    s2_plan* plans[2];
    const s2::AttnSchedule* sched[2];
    for (int s = 0; s < 2; s++)
    {
        if ((r = get_plan(d, video_shape, s, &plans[s])) != S2_OK) return r;
        if ((r = s2::ensure_schedule(plans[s], &text_length, c, &sched[s])) != S2_OK) return r;
    }
    const int Nv = video_shape[0] * video_shape[1] * video_shape[2];
    const int Nt = text_length;
    const int M = Nv + Nt;
    int max_packed = 0, max_partial = 0;
    for (int s = 0; s < 2; s++)
    {
        max_packed = std::max(max_packed, sched[s]->packed_rows);
        max_partial = std::max(max_partial, sched[s]->partial_rows);
    }
    // The QKV projection's epilogue writes the packed windows directly when a
    // 256-column tile holds whole heads (D % 256 == 0); otherwise qkv rows go
    // through a buffer and the prepare kernel.
    const bool fused_qkv = D % 256 == 0;
    if (fused_qkv && (r = ensure_rope_tables(d, std::max(sched[0]->max_pos, sched[1]->max_pos))) != S2_OK) return r;
    const size_t rope_block = (size_t)d->rope_pos * cfg.rope_pairs * 8;
    // activations: h [M][D] bf16 | (qkv [M][3D] bf16) | Q,K,V [R][D] bf16 | ctx [M][D] bf16 |
    //              partial [P][D] f32 | u [M][F] bf16
    const size_t sz_h = align256((size_t)M * D * 2), sz_qkv = fused_qkv ? 0 : align256((size_t)M * 3 * D * 2),
                 sz_pk = align256((size_t)max_packed * D * 2), sz_ctx = sz_h,
                 sz_part = align256((size_t)max_partial * D * 4), sz_u = align256((size_t)M * F * 2);
    if ((r = d->act.ensure(sz_h + sz_qkv + 3 * sz_pk + sz_ctx + sz_part + sz_u)) != S2_OK) return r;
    if ((r = d->mods.ensure((size_t)cfg.num_blocks * 6 * D * 4)) != S2_OK) return r;
    uint8_t* a = static_cast<uint8_t*>(d->act.ptr);
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(a);
    __nv_bfloat16* qkv = reinterpret_cast<__nv_bfloat16*>(a + sz_h);
    uint8_t* pk = a + sz_h + sz_qkv;
    __nv_bfloat16* ctxb = reinterpret_cast<__nv_bfloat16*>(pk + 3 * sz_pk);
    float* partial = reinterpret_cast<float*>(pk + 3 * sz_pk + sz_ctx);
    __nv_bfloat16* u = reinterpret_cast<__nv_bfloat16*>(pk + 3 * sz_pk + sz_ctx + sz_part);
    float* mods = static_cast<float*>(d->mods.ptr);

    // per-block modulation = shared frontend modulation + block offsets
    if ((r = s2::launch_add_vectors(c, d->ada_all, modulation, mods, cfg.num_blocks * 6 * D, 6 * D)) != S2_OK)
        return r;

    // finite checks: the block stack's input (the frontend's output), then
    // every block's output, counted on the device; read once at the end
    unsigned long long* fin = nullptr;
    const size_t nfin = 2 * (size_t)(cfg.num_blocks + 1);
    if (d->check_finite)
    {
        if ((r = d->finite.ensure(nfin * sizeof(unsigned long long))) != S2_OK) return r;
        fin = static_cast<unsigned long long*>(d->finite.ptr);
        if (cudaMemsetAsync(fin, 0, nfin * sizeof(unsigned long long), c.stream) != cudaSuccess) return S2_ERR_CUDA;
        if ((r = count_rows_nonfinite(c, x, Nv, Nt, D, fin)) != S2_OK) return r;
    }

    for (int b = 0; b < cfg.num_blocks; b++)
    {
        const s2_dit::Block& bl = d->blocks[b];
        const float* mb = mods + (size_t)b * 6 * D;
        const int sh = b & 1; // odd blocks use the half-shifted windows
        const s2::AttnSchedule& S = *sched[sh];
        if ((r = s2::launch_ada_norm(c, M, D, x, cfg.norm_eps, mb, mb + D, h, bl.norm_layer)) != S2_OK) return r;
        __nv_bfloat16* Qp = reinterpret_cast<__nv_bfloat16*>(pk);
        __nv_bfloat16* Kp = reinterpret_cast<__nv_bfloat16*>(pk + sz_pk);
        __nv_bfloat16* Vp = reinterpret_cast<__nv_bfloat16*>(pk + 2 * sz_pk);
        if (fused_qkv)
        {
            // QKV projection + qk norm + RoPE + window packing in one kernel
            if ((r = s2::launch_qkv_packed(c, S, Nv, Nt, D, h, h + (size_t)Nv * D, bl.w_qkv,
                                           cfg.qkv_bias ? bl.b_qkv : nullptr, H, cfg.rope_pairs, cfg.qk_eps,
                                           bl.qk_norm, static_cast<uint8_t*>(d->rope.ptr) + rope_block * b,
                                           d->rope_pos, Qp, Kp, Vp)) != S2_OK)
                return r;
        }
        else
        {
            if ((r = s2::launch_shared_linear(c, M, 0, 3 * D, D, h, nullptr, bl.w_qkv,
                                              cfg.qkv_bias ? bl.b_qkv : nullptr, s2::EPI_STORE, nullptr, 0, qkv,
                                              nullptr)) != S2_OK)
                return r;
            const __nv_bfloat16* tq = qkv + (size_t)Nv * 3 * D;
            if ((r = s2::launch_prepare_qkv(c, S, H, cfg.head_dim, cfg.rope_pairs, cfg.qk_eps, bl.qk_norm, bl.freqs,
                                            1, qkv, qkv + D, qkv + 2 * D, 3 * D, tq, tq + D, tq + 2 * D, 3 * D, Qp,
                                            Kp, Vp)) != S2_OK)
                return r;
        }
        if ((r = s2::launch_window_attention(c, S, H, Qp, Kp, Vp, 0, 0, ctxb, partial)) != S2_OK) return r;
        if ((r = s2::launch_text_pool(c, S, D, partial, 0, 0, ctxb + (size_t)Nv * D)) != S2_OK) return r;
        if ((r = s2::launch_shared_linear(c, M, 0, D, D, ctxb, nullptr, bl.w_out, cfg.out_bias ? bl.b_out : nullptr,
                                          s2::EPI_GATE_RESIDUAL, mb + 2 * D, 1, x, nullptr)) != S2_OK)
            return r;
        if ((r = s2::launch_ada_norm(c, M, D, x, cfg.norm_eps, mb + 3 * D, mb + 4 * D, h, bl.norm_layer)) != S2_OK) return r;
        if ((r = s2::launch_shared_linear(c, M, 0, F, D, h, nullptr, bl.w_up, cfg.mlp_bias ? bl.b_up : nullptr,
                                          s2::EPI_GELU_TANH, nullptr, 0, u, nullptr)) != S2_OK)
            return r;
        if ((r = s2::launch_shared_linear(c, M, 0, D, F, u, nullptr, bl.w_down, cfg.mlp_bias ? bl.b_down : nullptr,
                                          s2::EPI_GATE_RESIDUAL, mb + 5 * D, 1, x, nullptr)) != S2_OK)
            return r;
        if (fin && (r = count_rows_nonfinite(c, x, Nv, Nt, D, fin + 2 * (b + 1))) != S2_OK) return r;
        for (const s2_dit::Checkpoint& cp : d->checkpoints)
            if (cp.block == b &&
                (cudaMemcpyAsync(cp.video + d->cp_video_row * D, x, (size_t)Nv * D * 4, cudaMemcpyDeviceToDevice,
                                 c.stream) != cudaSuccess ||
                 cudaMemcpyAsync(cp.text + d->cp_text_row * D, x + (size_t)Nv * D, (size_t)Nt * D * 4,
                                 cudaMemcpyDeviceToDevice, c.stream) != cudaSuccess))
                return S2_ERR_CUDA;
    }
    if (fin)
    {
        // -1 as the reference returns when its frontend or block-graph output
        // is non-finite (seedvr2_dit.cpp:700-716, :1068-1071); counting every
        // block's output as well names the first block that produced one (the
        // blocks after it have run)
        std::vector<unsigned long long> h(nfin);
        if (cudaMemcpyAsync(h.data(), fin, nfin * sizeof(unsigned long long), cudaMemcpyDeviceToHost, c.stream) !=
                cudaSuccess ||
            cudaStreamSynchronize(c.stream) != cudaSuccess)
            return S2_ERR_CUDA;
        d->finite_checked = true;
        d->nonfinite_block = cfg.num_blocks;
        d->nonfinite_video = d->nonfinite_text = 0;
        for (int i = 0; i <= cfg.num_blocks; i++)
            if (h[2 * i] || h[2 * i + 1])
            {
                d->nonfinite_block = i - 1;
                d->nonfinite_video = (int64_t)h[2 * i];
                d->nonfinite_text = (int64_t)h[2 * i + 1];
                return S2_ERR_INVALID;
            }
    }
    return S2_OK;
}

int s2_dit_forward_sharded(s2_dit* d, const int* video_shape, int text_length, float* x, const float* modulation)
{
    if (!d || !video_shape || text_length <= 0 || !x || !modulation) return S2_ERR_INVALID;
    // block checkpoints are a one-GPU feature: a rank holds only its own rows
    if (!d->checkpoints.empty()) return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    s2::Dist* dist = d->ctx->dist.get();
    const int rank = dist ? dist->rank : 0, world = dist ? dist->world : 1;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const s2_dit_config& cfg = d->cfg;
    const int D = cfg.hidden, F = cfg.mlp_hidden, H = cfg.heads, T = text_length;
    int r;
    std::vector<int> key(video_shape, video_shape + 3);
    key.push_back(T);
    key.push_back(rank);
    key.push_back(world);
    std::unique_ptr<s2_dit::Shard>& slot = d->shards[key];
    if (!slot)
    {
        // Collective set-up (every rank builds the same shape): ownership,
        // schedules, the exchange buffer and its IPC mapping on every peer.
        std::unique_ptr<s2_dit::Shard> sh(new s2_dit::Shard);
        r = s2::build_shard(video_shape, T, cfg.window, cfg.window_mode, rank, world, sh->sp);
        const s2::ShardPlan& sp = sh->sp;
        int E = 0;
        for (int q = 0; q < world && r == S2_OK; q++)
            E = std::max(E, sp.n_local[q] + T + std::max(sp.m_foreign_all[0][q], sp.m_foreign_all[1][q]));
        // Fused packing: every window's rows land at its owner, windows in
        // ascending order, each = its tokens (partition order) then T text
        // rows -- the order build_schedule_ex packs the owner's windows in.
        sh->fused = D % 256 == 0;
        std::vector<int> pack_tab[2];
        int R = 1;
        for (int p = 0; p < 2 && r == S2_OK && sh->fused; p++)
        {
            const s2::Plan& pl = sp.plan[p];
            const int nw = static_cast<int>(pl.windows.size() / 9);
            std::vector<int> seq(world, 0), seq_off(nw, 0);
            for (int w = 0; w < nw; w++)
            {
                const int q = sp.owner[p][w];
                seq_off[w] = seq[q];
                seq[q] += pl.windows[9 * w + 8] + T;
            }
            for (int q = 0; q < world; q++) R = std::max(R, seq[q]);
            const int n = sp.n_local[rank];
            pack_tab[p].assign((size_t)n * 4, -1);
            for (int w = 0; w < nw; w++)
            {
                const int q = sp.owner[p][w], part = pl.windows[9 * w + 7], cnt = pl.windows[9 * w + 8];
                for (int i = 0; i < cnt; i++)
                {
                    const int g = pl.video_indices[part + i];
                    if (sp.token_owner[g] != rank) continue;
                    const int row = sp.token_local[g];
                    const int dst = seq_off[w] + i;
                    pack_tab[p][row] = q == rank ? dst : ((q + 1) << s2::kPeerShift) | dst;
                    pack_tab[p][n + 3 * row] = pl.local_positions[3 * (part + i)] + T;
                    pack_tab[p][n + 3 * row + 1] = pl.local_positions[3 * (part + i) + 1];
                    pack_tab[p][n + 3 * row + 2] = pl.local_positions[3 * (part + i) + 2];
                }
            }
            for (size_t i = (size_t)n; i < pack_tab[p].size(); i++) sh->max_pos = std::max(sh->max_pos, pack_tab[p][i] + 1);
            if (cudaMalloc(&sh->d_pack[p], std::max<size_t>(pack_tab[p].size(), 4) * 4) != cudaSuccess)
                r = S2_ERR_ALLOC;
            else if (!pack_tab[p].empty() &&
                     cudaMemcpy(sh->d_pack[p], pack_tab[p].data(), pack_tab[p].size() * 4, cudaMemcpyHostToDevice) !=
                         cudaSuccess)
                r = S2_ERR_CUDA;
        }
        const size_t sz_pk = align256((size_t)R * D * 2);
        sh->off_q = 0;
        sh->off_k = sh->fused ? sz_pk : 0;
        sh->off_v = sh->fused ? 2 * sz_pk : 0;
        sh->off_ctx = sh->fused ? 3 * sz_pk : align256((size_t)E * 3 * D * 2);
        sh->off_text = sh->off_ctx + align256((size_t)E * D * 2);
        sh->off_flags = sh->off_text + 2 * align256((size_t)T * D * 4);
        const size_t xbytes = sh->off_flags + 256;
        if (r == S2_OK && cudaMalloc(&sh->xbuf, xbytes) != cudaSuccess) r = S2_ERR_ALLOC;
        if (r == S2_OK && cudaMemset(sh->xbuf, 0, xbytes) != cudaSuccess) r = S2_ERR_CUDA;
        if (r == S2_OK)
        {
            if (world > 1)
                r = dist->share_buffer(c, sh->xbuf, sh->base);
            else
                sh->base.assign(1, sh->xbuf);
        }
        for (int q = 0; q < world && r == S2_OK; q++)
        {
            uint8_t* b = static_cast<uint8_t*>(sh->base[q]);
            sh->peer_qkv.push_back(b);
            sh->peer_q.push_back(b + sh->off_q);
            sh->peer_k.push_back(b + sh->off_k);
            sh->peer_v.push_back(b + sh->off_v);
            sh->peer_ctx.push_back(b + sh->off_ctx);
            sh->peer_text[0].push_back(b + sh->off_text);
            sh->peer_text[1].push_back(b + sh->off_text + align256((size_t)T * D * 4));
            sh->peer_flags.push_back(b + sh->off_flags);
        }
        for (int p = 0; p < 2 && r == S2_OK; p++)
        {
            // context rows of foreign tokens go straight to their owner's buffer
            std::vector<int> out(sp.Nv, -1);
            for (int g = 0; g < sp.Nv; g++)
            {
                if (sp.row[p][g] < 0) continue;
                const int o = sp.token_owner[g];
                out[g] = o == rank ? sp.token_local[g] : ((o + 1) << s2::kPeerShift) | sp.token_local[g];
            }
            r = s2::build_schedule_ex(sp.plan[p], &T, &sp.win_mine[p], &sp.row[p], sh->sched[p], c.stream, &out);
            std::vector<int4> push;
            for (int q = 0; q < world; q++)
            {
                const int base_row = sp.n_local[q] + T + sp.recv_off_all[p][(size_t)q * world + rank];
                for (size_t k = 0; k < sp.send_tokens[p][q].size(); k++)
                    push.push_back(make_int4(sp.token_local[sp.send_tokens[p][q][k]], q, base_row + (int)k, 0));
            }
            for (int q = 0; q < world; q++) sh->any_push[p] = sh->any_push[p] || sp.m_foreign_all[p][q] > 0;
            sh->push_count[p] = static_cast<int>(push.size());
            if (r == S2_OK && !push.empty())
            {
                if (cudaMalloc(&sh->d_push[p], push.size() * sizeof(int4)) != cudaSuccess)
                    r = S2_ERR_ALLOC;
                else if (cudaMemcpy(sh->d_push[p], push.data(), push.size() * sizeof(int4), cudaMemcpyHostToDevice) !=
                         cudaSuccess)
                    r = S2_ERR_CUDA;
            }
        }
        if (r != S2_OK)
        {
            d->shards.erase(key);
            return r;
        }
        slot = std::move(sh);
    }
    s2_dit::Shard& sh = *slot;
    const s2::ShardPlan& sp = sh.sp;
    const int n = sp.n_local[rank];
    const int M = n + T; // rows of x / h / u (own video rows, then text)
    const int max_packed = std::max(sh.sched[0].packed_rows, sh.sched[1].packed_rows);
    const int max_partial = std::max(sh.sched[0].partial_rows, sh.sched[1].partial_rows);
    if (sh.fused &&
        (r = ensure_rope_tables(d, std::max(sh.max_pos, std::max(sh.sched[0].max_pos, sh.sched[1].max_pos)))) !=
            S2_OK)
        return r;
    const size_t rope_block = (size_t)d->rope_pos * cfg.rope_pairs * 8;
    const size_t sz_h = align256((size_t)M * D * 2),
                 sz_pk = sh.fused ? 0 : align256((size_t)std::max(max_packed, 1) * D * 2),
                 sz_part = align256((size_t)std::max(max_partial, 1) * D * 4), sz_u = align256((size_t)M * F * 2);
    if ((r = d->act.ensure(sz_h + 3 * sz_pk + sz_part + sz_u)) != S2_OK) return r;
    if ((r = d->mods.ensure((size_t)cfg.num_blocks * 6 * D * 4)) != S2_OK) return r;
    uint8_t* a = static_cast<uint8_t*>(d->act.ptr);
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(a);
    uint8_t* pk = a + sz_h;
    float* partial = reinterpret_cast<float*>(pk + 3 * sz_pk);
    __nv_bfloat16* u = reinterpret_cast<__nv_bfloat16*>(pk + 3 * sz_pk + sz_part);
    __nv_bfloat16* qkv = static_cast<__nv_bfloat16*>(sh.xbuf);
    __nv_bfloat16* ctxb = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(sh.xbuf) + sh.off_ctx);
    float* text32_buf[2] = {reinterpret_cast<float*>(static_cast<uint8_t*>(sh.xbuf) + sh.off_text),
                            reinterpret_cast<float*>(static_cast<uint8_t*>(sh.xbuf) + sh.off_text +
                                                     align256((size_t)T * D * 4))};
    uint32_t* my_flags = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(sh.xbuf) + sh.off_flags);
    float* mods = static_cast<float*>(d->mods.ptr);
    if ((r = s2::launch_add_vectors(c, d->ada_all, modulation, mods, cfg.num_blocks * 6 * D, 6 * D)) != S2_OK)
        return r;
    auto barrier = [&]() -> int {
        if (world == 1) return S2_OK;
        return s2::launch_peer_barrier(c, sh.peer_flags.data(), my_flags, rank, world, ++dist->epoch);
    };

    for (int b = 0; b < cfg.num_blocks; b++)
    {
        const s2_dit::Block& bl = d->blocks[b];
        const float* mb = mods + (size_t)b * 6 * D;
        const int shf = b & 1;
        const s2::AttnSchedule& S = sh.sched[shf];
        if ((r = s2::launch_ada_norm(c, M, D, x, cfg.norm_eps, mb, mb + D, h, bl.norm_layer)) != S2_OK) return r;
        __nv_bfloat16 *Qp, *Kp, *Vp;
        if (sh.fused)
        {
            // QKV projection + qk norm + RoPE, each row stored into the packed
            // window of the GPU that owns it (NVLink peer stores)
            Qp = static_cast<__nv_bfloat16*>(sh.peer_q[rank]);
            Kp = static_cast<__nv_bfloat16*>(sh.peer_k[rank]);
            Vp = static_cast<__nv_bfloat16*>(sh.peer_v[rank]);
            s2::QkvPeers peers;
            peers.dst0 = sh.d_pack[shf];
            peers.dst0_rows = n;
            peers.pos0 = sh.d_pack[shf] + n;
            peers.q = sh.peer_q.data();
            peers.k = sh.peer_k.data();
            peers.v = sh.peer_v.data();
            peers.num_peers = world;
            if ((r = s2::launch_qkv_packed(c, S, n, T, D, h, h + (size_t)n * D, bl.w_qkv,
                                           cfg.qkv_bias ? bl.b_qkv : nullptr, H, cfg.rope_pairs, cfg.qk_eps,
                                           bl.qk_norm, static_cast<uint8_t*>(d->rope.ptr) + rope_block * b,
                                           d->rope_pos, Qp, Kp, Vp, &peers)) != S2_OK)
                return r;
            if (world > 1 && sh.any_push[shf] && (r = barrier()) != S2_OK) return r;
        }
        else
        {
            if ((r = s2::launch_shared_linear(c, M, 0, 3 * D, D, h, nullptr, bl.w_qkv,
                                              cfg.qkv_bias ? bl.b_qkv : nullptr, s2::EPI_STORE, nullptr, 0, qkv,
                                              nullptr)) != S2_OK)
                return r;
            if (world > 1 && sh.any_push[shf])
            {
                // own qkv rows of tokens in other ranks' windows -> straight into the owners' buffers
                if ((r = s2::launch_push_rows(c, qkv, 3 * D, sh.d_push[shf], sh.push_count[shf],
                                              sh.peer_qkv.data(), world)) != S2_OK)
                    return r;
                if ((r = barrier()) != S2_OK) return r;
            }
            Qp = reinterpret_cast<__nv_bfloat16*>(pk);
            Kp = reinterpret_cast<__nv_bfloat16*>(pk + sz_pk);
            Vp = reinterpret_cast<__nv_bfloat16*>(pk + 2 * sz_pk);
            const __nv_bfloat16* tq = qkv + (size_t)n * 3 * D;
            if ((r = s2::launch_prepare_qkv(c, S, H, cfg.head_dim, cfg.rope_pairs, cfg.qk_eps, bl.qk_norm, bl.freqs,
                                            1, qkv, qkv + D, qkv + 2 * D, 3 * D, tq, tq + D, tq + 2 * D, 3 * D, Qp,
                                            Kp, Vp)) != S2_OK)
                return r;
        }
        // context rows of foreign tokens are stored into their owners' buffers by the epilogue
        if ((r = s2::launch_window_attention(c, S, H, Qp, Kp, Vp, 0, 0, ctxb, partial, sh.peer_ctx.data(),
                                             world > 1 ? world : 0)) != S2_OK)
            return r;
        if (world == 1)
        {
            if ((r = s2::launch_text_pool(c, S, D, partial, 0, 0, ctxb + (size_t)n * D)) != S2_OK) return r;
        }
        else
        {
            if ((r = s2::launch_text_pool(c, S, D, partial, 1, 0, text32_buf[b & 1])) != S2_OK) return r;
            if ((r = barrier()) != S2_OK) return r;
            // text rows: sum of every rank's partial, read over NVLink in rank order
            if ((r = s2::launch_text_reduce_peers(c, sh.peer_text[b & 1].data(), world, (int64_t)T * D,
                                                  ctxb + (size_t)n * D)) != S2_OK)
                return r;
        }
        if ((r = s2::launch_shared_linear(c, M, 0, D, D, ctxb, nullptr, bl.w_out, cfg.out_bias ? bl.b_out : nullptr,
                                          s2::EPI_GATE_RESIDUAL, mb + 2 * D, 1, x, nullptr)) != S2_OK)
            return r;
        if ((r = s2::launch_ada_norm(c, M, D, x, cfg.norm_eps, mb + 3 * D, mb + 4 * D, h, bl.norm_layer)) != S2_OK) return r;
        if ((r = s2::launch_shared_linear(c, M, 0, F, D, h, nullptr, bl.w_up, cfg.mlp_bias ? bl.b_up : nullptr,
                                          s2::EPI_GELU_TANH, nullptr, 0, u, nullptr)) != S2_OK)
            return r;
        if ((r = s2::launch_shared_linear(c, M, 0, D, F, u, nullptr, bl.w_down, cfg.mlp_bias ? bl.b_down : nullptr,
                                          s2::EPI_GATE_RESIDUAL, mb + 5 * D, 1, x, nullptr)) != S2_OK)
            return r;
    }
    return S2_OK;
}

int s2_dit_forward_host(s2_dit* d, const int* video_shapes, const int* text_lengths, int batch, const float* video,
                        const float* text, const float* modulation, float* video_out, float* text_out)
{
    if (!d || !video_shapes || !text_lengths || batch <= 0 || !video || !text || !modulation || !video_out ||
        !text_out)
        return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int D = d->cfg.hidden;
    size_t v_off = 0, t_off = 0;
    int r = S2_OK;
    for (int s = 0; s < batch && r == S2_OK; s++)
    {
        const int* shp = video_shapes + 3 * s;
        if (shp[0] <= 0 || shp[1] <= 0 || shp[2] <= 0 || text_lengths[s] <= 0) return S2_ERR_INVALID;
        const size_t nv = (size_t)shp[0] * shp[1] * shp[2], nt = text_lengths[s];
        const size_t x_bytes = (nv + nt) * D * 4;
        if ((r = d->host_x.ensure(x_bytes + (size_t)6 * D * 4)) != S2_OK) return r;
        float* x = static_cast<float*>(d->host_x.ptr);
        float* mod = x + (nv + nt) * D;
        if (cudaMemcpyAsync(x, video + v_off * D, nv * D * 4, cudaMemcpyHostToDevice, c.stream) != cudaSuccess ||
            cudaMemcpyAsync(x + nv * D, text + t_off * D, nt * D * 4, cudaMemcpyHostToDevice, c.stream) !=
                cudaSuccess)
            return S2_ERR_CUDA;
        // modulation host layout [6][batch][D] (six frontend outputs, one row per sample)
        for (int k = 0; k < 6; k++)
            if (cudaMemcpyAsync(mod + (size_t)k * D, modulation + ((size_t)k * batch + s) * D, (size_t)D * 4,
                                cudaMemcpyHostToDevice, c.stream) != cudaSuccess)
                return S2_ERR_CUDA;
        // checkpoints land at this sample's rows, like its outputs
        d->cp_video_row = v_off;
        d->cp_text_row = t_off;
        r = s2_dit_forward(d, shp, text_lengths[s], x, mod);
        d->cp_video_row = d->cp_text_row = 0;
        if (r != S2_OK) return r;
        if (cudaMemcpyAsync(video_out + v_off * D, x, nv * D * 4, cudaMemcpyDeviceToHost, c.stream) != cudaSuccess ||
            cudaMemcpyAsync(text_out + t_off * D, x + nv * D, nt * D * 4, cudaMemcpyDeviceToHost, c.stream) !=
                cudaSuccess)
            return S2_ERR_CUDA;
        v_off += nv;
        t_off += nt;
    }
    if (cudaStreamSynchronize(c.stream) != cudaSuccess) return S2_ERR_CUDA;
    return r;
}

namespace {

int host_pipe_init(s2_dit* d)
{
    s2_dit::HostPipe& p = d->pipe;
    if (p.ready) return S2_OK;
    if (!p.up && cudaStreamCreateWithFlags(&p.up, cudaStreamNonBlocking) != cudaSuccess) return S2_ERR_CUDA;
    if (!p.down && cudaStreamCreateWithFlags(&p.down, cudaStreamNonBlocking) != cudaSuccess) return S2_ERR_CUDA;
    for (int b = 0; b < 2; b++)
        for (cudaEvent_t* e : {&p.uploaded[b], &p.computed[b], &p.downloaded[b]})
            if (!*e && cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return S2_ERR_CUDA;
    p.ready = true;
    return S2_OK;
}

} // namespace

int s2_dit_forward_host_async(s2_dit* d, const int* video_shapes, const int* text_lengths, int batch,
                              const float* video, const float* text, const float* modulation, float* video_out,
                              float* text_out)
{
    if (!d || !video_shapes || !text_lengths || batch <= 0 || !video || !text || !modulation || !video_out ||
        !text_out)
        return S2_ERR_INVALID;
    for (int s = 0; s < batch; s++)
        if (video_shapes[3 * s] <= 0 || video_shapes[3 * s + 1] <= 0 || video_shapes[3 * s + 2] <= 0 ||
            text_lengths[s] <= 0)
            return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    int r = host_pipe_init(d);
    if (r != S2_OK) return r;
    s2_dit::HostPipe& p = d->pipe;
    const int D = d->cfg.hidden;
    size_t v_off = 0, t_off = 0;
    for (int s = 0; s < batch; s++)
    {
        const int* shp = video_shapes + 3 * s;
        const size_t nv = (size_t)shp[0] * shp[1] * shp[2], nt = text_lengths[s];
        const size_t x_bytes = (nv + nt) * D * 4 + (size_t)6 * D * 4;
        const int b = p.next;
        p.next ^= 1;
        if (p.x[b].bytes < x_bytes)
        {
            // growing frees the old buffer: every stream finishes with it first
            if (cudaStreamSynchronize(p.up) != cudaSuccess || cudaStreamSynchronize(p.down) != cudaSuccess ||
                cudaStreamSynchronize(c.stream) != cudaSuccess)
                return S2_ERR_CUDA;
            if ((r = p.x[b].ensure(x_bytes)) != S2_OK) return r;
        }
        float* x = static_cast<float*>(p.x[b].ptr);
        float* mod = x + (nv + nt) * D;
        // upload once the buffer's previous download has read it
        if (cudaStreamWaitEvent(p.up, p.downloaded[b], 0) != cudaSuccess ||
            cudaMemcpyAsync(x, video + v_off * D, nv * D * 4, cudaMemcpyHostToDevice, p.up) != cudaSuccess ||
            cudaMemcpyAsync(x + nv * D, text + t_off * D, nt * D * 4, cudaMemcpyHostToDevice, p.up) != cudaSuccess)
            return S2_ERR_CUDA;
        for (int k = 0; k < 6; k++)
            if (cudaMemcpyAsync(mod + (size_t)k * D, modulation + ((size_t)k * batch + s) * D, (size_t)D * 4,
                                cudaMemcpyHostToDevice, p.up) != cudaSuccess)
                return S2_ERR_CUDA;
        if (cudaEventRecord(p.uploaded[b], p.up) != cudaSuccess ||
            cudaStreamWaitEvent(c.stream, p.uploaded[b], 0) != cudaSuccess)
            return S2_ERR_CUDA;
        d->cp_video_row = v_off;
        d->cp_text_row = t_off;
        r = s2_dit_forward(d, shp, text_lengths[s], x, mod);
        d->cp_video_row = d->cp_text_row = 0;
        if (r != S2_OK)
        {
            // whatever the failed forward enqueued still reads and writes
            // buffer b: its next upload waits for that work, through the
            // events a download would have recorded
            if (cudaEventRecord(p.computed[b], c.stream) == cudaSuccess &&
                cudaStreamWaitEvent(p.down, p.computed[b], 0) == cudaSuccess)
                cudaEventRecord(p.downloaded[b], p.down);
            return r;
        }
        // download once the forward is done
        if (cudaEventRecord(p.computed[b], c.stream) != cudaSuccess ||
            cudaStreamWaitEvent(p.down, p.computed[b], 0) != cudaSuccess ||
            cudaMemcpyAsync(video_out + v_off * D, x, nv * D * 4, cudaMemcpyDeviceToHost, p.down) != cudaSuccess ||
            cudaMemcpyAsync(text_out + t_off * D, x + nv * D, nt * D * 4, cudaMemcpyDeviceToHost, p.down) !=
                cudaSuccess ||
            cudaEventRecord(p.downloaded[b], p.down) != cudaSuccess)
            return S2_ERR_CUDA;
        v_off += nv;
        t_off += nt;
    }
    return S2_OK;
}

int s2_dit_host_wait(s2_dit* d)
{
    if (!d) return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const s2_dit::HostPipe& p = d->pipe;
    if ((p.down && cudaStreamSynchronize(p.down) != cudaSuccess) ||
        (p.up && cudaStreamSynchronize(p.up) != cudaSuccess) || cudaStreamSynchronize(c.stream) != cudaSuccess)
        return S2_ERR_CUDA;
    return S2_OK;
}

// ---------------------------------------------------------------- frontend / tail
int s2_dit_set_io_weights(s2_dit* d, const s2_dit_io_host_weights* w)
{
    if (!d || !w || !w->w_vid_in || !w->w_txt_in || !w->w_emb0 || !w->w_emb1 || !w->w_emb2 || !w->tail_ada ||
        !w->w_out)
        return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    int r = ensure_io_weights(d);
    if (r != S2_OK) return r;
    d->io_loaded = false;
    const size_t D = d->cfg.hidden;
    const s2_dit::Io& io = d->io;
    s2::DeviceBuffer tmp;
    if ((r = tmp.ensure(std::max<size_t>(6 * D * D, D * s2::kTextChannels) * 4)) != S2_OK) return r;
    float* t = static_cast<float*>(tmp.ptr);
    auto up_bf16 = [&](const float* src, __nv_bfloat16* dst, size_t n) -> int {
        if (cudaMemcpyAsync(t, src, n * 4, cudaMemcpyHostToDevice, c.stream) != cudaSuccess) return S2_ERR_CUDA;
        return s2::launch_convert_f32_bf16(c, t, dst, (int64_t)n);
    };
    auto up_f32 = [&](const float* src, float* dst, size_t n) -> int {
        if (!src) return cudaMemsetAsync(dst, 0, n * 4, c.stream) == cudaSuccess ? S2_OK : S2_ERR_CUDA;
        return cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyHostToDevice, c.stream) == cudaSuccess ? S2_OK
                                                                                                 : S2_ERR_CUDA;
    };
    // video input projection: rows of 132 placed at a pitch of kPatchPitch, zero padded
    if (cudaMemsetAsync(t, 0, D * s2::kPatchPitch * 4, c.stream) != cudaSuccess ||
        cudaMemcpy2DAsync(t, s2::kPatchPitch * 4, w->w_vid_in, s2::kPatchFeatures * 4, s2::kPatchFeatures * 4, D,
                          cudaMemcpyHostToDevice, c.stream) != cudaSuccess)
        return S2_ERR_CUDA;
    r = s2::launch_convert_f32_bf16(c, t, io.w_vid_in, (int64_t)D * s2::kPatchPitch);
    // the staging buffer is reused below: order the conversion before the next upload
    if (r == S2_OK && cudaStreamSynchronize(c.stream) != cudaSuccess) r = S2_ERR_CUDA;
    const float* srcs[5] = {w->w_txt_in, w->w_emb0, w->w_emb1, w->w_emb2, w->w_out};
    __nv_bfloat16* dsts[5] = {io.w_txt_in, io.w_emb0, io.w_emb1, io.w_emb2, io.w_out};
    const size_t ns[5] = {D * s2::kTextChannels, D * s2::kTimeFeatures, D * D, 6 * D * D, s2::kPredFeatures * D};
    for (int i = 0; i < 5 && r == S2_OK; i++) r = up_bf16(srcs[i], dsts[i], ns[i]);
    if (r == S2_OK) r = up_f32(w->b_vid_in, io.b_vid_in, D);
    if (r == S2_OK) r = up_f32(w->b_txt_in, io.b_txt_in, D);
    if (r == S2_OK) r = up_f32(w->b_emb0, io.b_emb0, D);
    if (r == S2_OK) r = up_f32(w->b_emb1, io.b_emb1, D);
    if (r == S2_OK) r = up_f32(w->b_emb2, io.b_emb2, 6 * D);
    if (r == S2_OK) r = up_f32(w->tail_ada, io.tail_ada, 2 * D);
    if (r == S2_OK) r = up_f32(w->b_out, io.b_out, s2::kPredFeatures);
    if (r == S2_OK && cudaStreamSynchronize(c.stream) != cudaSuccess) r = S2_ERR_CUDA;
    if (r == S2_OK) d->io_loaded = true;
    return r;
}

int s2_dit_forward_frontend(s2_dit* d, const int* video_shapes, const int* text_lengths, const float* timesteps,
                            int batch, const float* video, int video_rows, const float* text, int text_rows,
                            float* video_out, float* text_out, float* modulation)
{
    // forward_frontend returns -1 before the frontend net is loaded (seedvr2_dit.cpp:1186-1187)
    if (!d || !d->io_loaded || !video || !text || !video_out || !text_out || !modulation) return S2_ERR_INVALID;
    int64_t np = 0;
    int r = check_dit_inputs(video_shapes, text_lengths, timesteps, batch, video_rows, text_rows, &np);
    if (r != S2_OK) return r;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int D = d->cfg.hidden;
    const s2_dit::Io& io = d->io;
    // workspace: patches bf16 [np][136] | text bf16 [T][5120] | temb [B][256] | e0, e1 [B][D]
    const size_t sz_p = align256((size_t)np * s2::kPatchPitch * 2),
                 sz_t = align256((size_t)text_rows * s2::kTextChannels * 2),
                 sz_e = align256((size_t)batch * (s2::kTimeFeatures + 2 * D) * 4);
    if ((r = d->io_ws.ensure(sz_p + sz_t + sz_e)) != S2_OK) return r;
    uint8_t* ws = static_cast<uint8_t*>(d->io_ws.ptr);
    __nv_bfloat16* patches = reinterpret_cast<__nv_bfloat16*>(ws);
    __nv_bfloat16* tb = reinterpret_cast<__nv_bfloat16*>(ws + sz_p);
    float* temb = reinterpret_cast<float*>(ws + sz_p + sz_t);
    float* e0 = temb + (size_t)batch * s2::kTimeFeatures;
    float* e1 = e0 + (size_t)batch * D;
    int64_t v_off = 0, p_off = 0;
    for (int s = 0; s < batch && r == S2_OK; s++)
    {
        const int* shp = video_shapes + 3 * s;
        r = s2::launch_patchify(c, video + v_off * s2::kLatentChannels, shp[0], shp[1], shp[2],
                                patches + p_off * s2::kPatchPitch, 1);
        v_off += (int64_t)shp[0] * shp[1] * shp[2];
        p_off += (int64_t)shp[0] * (shp[1] / 2) * (shp[2] / 2);
    }
    // token-wise nets: every sample's rows in one launch each
    if (r == S2_OK)
        r = s2::launch_shared_linear(c, (int)np, 0, D, s2::kPatchPitch, patches, nullptr, io.w_vid_in, io.b_vid_in,
                                     s2::EPI_STORE, nullptr, 1, video_out, nullptr);
    if (r == S2_OK) r = s2::launch_convert_f32_bf16(c, text, tb, (int64_t)text_rows * s2::kTextChannels);
    if (r == S2_OK)
        r = s2::launch_shared_linear(c, text_rows, 0, D, s2::kTextChannels, tb, nullptr, io.w_txt_in, io.b_txt_in,
                                     s2::EPI_STORE, nullptr, 1, text_out, nullptr);
    if (r == S2_OK) r = run_emb(d, timesteps, batch, temb, e0, e1, modulation, true);
    return r;
}

int s2_dit_forward_tail(s2_dit* d, const int* video_shapes, int batch, const float* video, int video_rows,
                        const float* modulation, float* prediction)
{
    if (!d || !d->io_loaded || !video_shapes || batch <= 0 || !video || !modulation || !prediction)
        return S2_ERR_INVALID;
    int64_t np_max = 0, np_total = 0;
    for (int s = 0; s < batch; s++)
    {
        const int* shp = video_shapes + 3 * s;
        if (shp[0] <= 0 || shp[1] <= 0 || shp[2] <= 0 || (shp[1] & 1) || (shp[2] & 1)) return S2_ERR_INVALID;
        const int64_t np = (int64_t)shp[0] * (shp[1] / 2) * (shp[2] / 2);
        np_max = std::max(np_max, np);
        np_total += np;
    }
    if (np_total != video_rows) return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int D = d->cfg.hidden;
    const size_t sz_h = align256((size_t)np_max * D * 2), sz_pp = align256((size_t)np_max * s2::kPredFeatures * 4);
    int r = d->io_ws.ensure(sz_h + sz_pp + align256((size_t)2 * D * 4));
    if (r != S2_OK) return r;
    uint8_t* ws = static_cast<uint8_t*>(d->io_ws.ptr);
    int64_t p_off = 0, t_off = 0;
    for (int s = 0; s < batch && r == S2_OK; s++)
    {
        const int* shp = video_shapes + 3 * s;
        // modulation rows [0][s] (shift) and [1][s] (scale) of the [6][batch][D] frontend output
        r = run_tail(d, shp, video + p_off * D, modulation + (size_t)s * D, modulation + ((size_t)batch + s) * D,
                     prediction + t_off * s2::kPredChannels, reinterpret_cast<__nv_bfloat16*>(ws),
                     reinterpret_cast<float*>(ws + sz_h), reinterpret_cast<float*>(ws + sz_h + sz_pp));
        p_off += (int64_t)shp[0] * (shp[1] / 2) * (shp[2] / 2);
        t_off += (int64_t)shp[0] * shp[1] * shp[2];
    }
    return r;
}

int s2_dit_forward_step(s2_dit* d, const int* video_shapes, const int* text_lengths, const float* timesteps,
                        int batch, const float* video, int video_rows, const float* text, int text_rows,
                        float* prediction, float* text_out)
{
    // SeedVR2DiTBlocks::forward(DiTInputs) returns -1 unless the frontend, the
    // tail and the block graph are loaded (seedvr2_dit.cpp:1301-1302)
    if (!d || !d->io_loaded || !video || !text || !prediction || !text_out) return S2_ERR_INVALID;
    int r = check_dit_inputs(video_shapes, text_lengths, timesteps, batch, video_rows, text_rows, nullptr);
    if (r != S2_OK) return r;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int D = d->cfg.hidden;
    int64_t np_max = 0, nt_max = 0;
    for (int s = 0; s < batch; s++)
    {
        const int* shp = video_shapes + 3 * s;
        np_max = std::max(np_max, (int64_t)shp[0] * (shp[1] / 2) * (shp[2] / 2));
        nt_max = std::max(nt_max, (int64_t)text_lengths[s]);
    }
    StepWs w;
    if ((r = step_workspace(d, np_max, nt_max, batch, 0, w)) != S2_OK) return r;
    // timestep MLP of every sample at once; per sample [6][D]
    if ((r = run_emb(d, timesteps, batch, w.temb, w.e0, w.e1, w.emb, false)) != S2_OK) return r;
    int64_t v_off = 0, t_off = 0, p_off = 0;
    for (int s = 0; s < batch && r == S2_OK; s++)
    {
        const int* shp = video_shapes + 3 * s;
        const PatchSrc src = {video + v_off * s2::kLatentChannels, nullptr, 0, nullptr, 0};
        // block checkpoints land at this sample's block-stack rows (patches,
        // then text rows), samples one after another
        d->cp_video_row = (size_t)p_off;
        d->cp_text_row = (size_t)t_off;
        r = run_sample(d, shp, src, text + t_off * s2::kTextChannels, text_lengths[s], w.emb + (size_t)s * 6 * D,
                       prediction + v_off * s2::kPredChannels, text_out + t_off * D, w);
        v_off += (int64_t)shp[0] * shp[1] * shp[2];
        p_off += (int64_t)shp[0] * (shp[1] / 2) * (shp[2] / 2);
        t_off += text_lengths[s];
    }
    d->cp_video_row = d->cp_text_row = 0;
    return r;
}

int s2_dit_forward_step_host(s2_dit* d, const int* video_shapes, const int* text_lengths, const float* timesteps,
                             int batch, const float* video, int video_rows, const float* text, int text_rows,
                             float* prediction, float* text_out)
{
    if (!d || !d->io_loaded || !video || !text || !prediction || !text_out) return S2_ERR_INVALID;
    int r = check_dit_inputs(video_shapes, text_lengths, timesteps, batch, video_rows, text_rows, nullptr);
    if (r != S2_OK) return r;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int D = d->cfg.hidden;
    const size_t bv = align256((size_t)video_rows * s2::kLatentChannels * 4),
                 bt = align256((size_t)text_rows * s2::kTextChannels * 4),
                 bp = align256((size_t)video_rows * s2::kPredChannels * 4), bo = align256((size_t)text_rows * D * 4);
    if ((r = d->io_host.ensure(bv + bt + bp + bo)) != S2_OK) return r;
    uint8_t* p = static_cast<uint8_t*>(d->io_host.ptr);
    float* dv = reinterpret_cast<float*>(p);
    float* dt = reinterpret_cast<float*>(p + bv);
    float* dp = reinterpret_cast<float*>(p + bv + bt);
    float* dto = reinterpret_cast<float*>(p + bv + bt + bp);
    if (cudaMemcpyAsync(dv, video, (size_t)video_rows * s2::kLatentChannels * 4, cudaMemcpyHostToDevice, c.stream) !=
            cudaSuccess ||
        cudaMemcpyAsync(dt, text, (size_t)text_rows * s2::kTextChannels * 4, cudaMemcpyHostToDevice, c.stream) !=
            cudaSuccess)
        return S2_ERR_CUDA;
    r = s2_dit_forward_step(d, video_shapes, text_lengths, timesteps, batch, dv, video_rows, dt, text_rows, dp, dto);
    if (r != S2_OK) return r;
    if (cudaMemcpyAsync(prediction, dp, (size_t)video_rows * s2::kPredChannels * 4, cudaMemcpyDeviceToHost,
                        c.stream) != cudaSuccess ||
        cudaMemcpyAsync(text_out, dto, (size_t)text_rows * D * 4, cudaMemcpyDeviceToHost, c.stream) != cudaSuccess)
        return S2_ERR_CUDA;
    return cudaStreamSynchronize(c.stream) == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

// ---------------------------------------------------------------- denoise loop
int s2_apply_cfg(s2_context* ctx, const float* pos, const float* neg, int64_t count, float scale, float rescale,
                 float* out)
{
    if (!ctx || !pos || !neg || !out || count <= 0) return S2_ERR_INVALID;
    s2::Context& c = ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    s2::DeviceBuffer& scratch = c.ws[3];
    int r = scratch.ensure(s2::cfg_scratch_bytes());
    if (r != S2_OK) return r;
    return s2::launch_apply_cfg(c, pos, neg, count, scale, rescale, out, scratch.ptr, 1, nullptr);
}

int s2_dit_denoise(s2_dit* d, const int* latent_shape, float* latent, int64_t latent_cstep, const float* condition,
                   int64_t condition_cstep, const float* positive_text, int positive_rows, const float* negative_text,
                   int negative_rows, const s2_denoise_options* opt)
{
    // restore()'s checks (seedvr2_pipeline.cpp:337-340) and predict()'s
    // is_latent / is_text (:14-26, :289-292)
    if (!d || !d->io_loaded || !latent_shape || !latent || !condition || !positive_text || !opt || opt->steps <= 0 ||
        positive_rows <= 0)
        return S2_ERR_INVALID;
    const bool cfg = opt->cfg_scale != 1.f;
    if (cfg && (!negative_text || negative_rows <= 0)) return S2_ERR_INVALID;
    const int T = latent_shape[0], H = latent_shape[1], W = latent_shape[2];
    if (T <= 0 || H <= 0 || W <= 0 || (H & 1) || (W & 1)) return S2_ERR_INVALID;
    const int64_t tokens = (int64_t)T * H * W;
    if (tokens > 0x7fffffff || latent_cstep < tokens || condition_cstep < tokens) return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const int64_t n16 = tokens * s2::kPredChannels;
    const size_t pred_bytes = align256((size_t)n16 * 4);
    StepWs w;
    int r = step_workspace(d, tokens / 4, std::max(positive_rows, cfg ? negative_rows : 0), 1,
                           3 * pred_bytes + s2::cfg_scratch_bytes(), w);
    if (r != S2_OK) return r;
    float* pos = static_cast<float*>(w.extra);
    float* neg = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(pos) + pred_bytes);
    float* guided = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(neg) + pred_bytes);
    void* scratch = reinterpret_cast<uint8_t*>(guided) + pred_bytes;
    const PatchSrc src = {nullptr, latent, latent_cstep, condition, condition_cstep};
    for (int step = 0; step < opt->steps && r == S2_OK; step++)
    {
        // the schedule of SeedVR2Pipeline::denoise (:542-545), same fp32 expressions
        const float timestep = 1000.f * (opt->steps - step) / opt->steps;
        const float next_timestep = 1000.f * (opt->steps - step - 1) / opt->steps;
        const float delta = (next_timestep - timestep) / 1000.f;
        r = run_emb(d, &timestep, 1, w.temb, w.e0, w.e1, w.emb, false);
        if (r == S2_OK) r = run_sample(d, latent_shape, src, positive_text, positive_rows, w.emb, pos, nullptr, w);
        const float* pred = pos;
        const float* factor = nullptr;
        if (r == S2_OK && cfg)
        {
            r = run_sample(d, latent_shape, src, negative_text, negative_rows, w.emb, neg, nullptr, w);
            if (r == S2_OK)
                r = s2::launch_apply_cfg(c, pos, neg, n16, opt->cfg_scale, opt->cfg_rescale, guided, scratch, 0,
                                         &factor);
            pred = guided;
        }
        if (r == S2_OK) r = s2::launch_euler(c, latent, latent_cstep, tokens, pred, factor, delta);
    }
    return r;
}

int s2_dit_denoise_host(s2_dit* d, const int* latent_shape, float* latent, int64_t latent_cstep,
                        const float* condition, int64_t condition_cstep, const float* positive_text,
                        int positive_rows, const float* negative_text, int negative_rows,
                        const s2_denoise_options* opt)
{
    if (!d || !d->io_loaded || !latent_shape || !latent || !condition || !positive_text || !opt || opt->steps <= 0 ||
        positive_rows <= 0)
        return S2_ERR_INVALID;
    const bool cfg = opt->cfg_scale != 1.f;
    if (cfg && (!negative_text || negative_rows <= 0)) return S2_ERR_INVALID;
    const int T = latent_shape[0], H = latent_shape[1], W = latent_shape[2];
    if (T <= 0 || H <= 0 || W <= 0) return S2_ERR_INVALID;
    const int64_t tokens = (int64_t)T * H * W;
    if (latent_cstep < tokens || condition_cstep < tokens) return S2_ERR_INVALID;
    s2::Context& c = d->ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const size_t plane = (size_t)tokens * 4, planes = align256(plane * s2::kPredChannels);
    const size_t bp = align256((size_t)positive_rows * s2::kTextChannels * 4),
                 bn = cfg ? align256((size_t)negative_rows * s2::kTextChannels * 4) : 0;
    int r = d->io_host.ensure(2 * planes + bp + bn);
    if (r != S2_OK) return r;
    uint8_t* p = static_cast<uint8_t*>(d->io_host.ptr);
    float* dl = reinterpret_cast<float*>(p);
    float* dc = reinterpret_cast<float*>(p + planes);
    float* dp = reinterpret_cast<float*>(p + 2 * planes);
    float* dn = cfg ? reinterpret_cast<float*>(p + 2 * planes + bp) : nullptr;
    // 16 planes each, host plane stride cstep -> dense device planes
    if (cudaMemcpy2DAsync(dl, plane, latent, (size_t)latent_cstep * 4, plane, s2::kPredChannels,
                          cudaMemcpyHostToDevice, c.stream) != cudaSuccess ||
        cudaMemcpy2DAsync(dc, plane, condition, (size_t)condition_cstep * 4, plane, s2::kPredChannels,
                          cudaMemcpyHostToDevice, c.stream) != cudaSuccess ||
        cudaMemcpyAsync(dp, positive_text, (size_t)positive_rows * s2::kTextChannels * 4, cudaMemcpyHostToDevice,
                        c.stream) != cudaSuccess ||
        (cfg && cudaMemcpyAsync(dn, negative_text, (size_t)negative_rows * s2::kTextChannels * 4,
                                cudaMemcpyHostToDevice, c.stream) != cudaSuccess))
        return S2_ERR_CUDA;
    r = s2_dit_denoise(d, latent_shape, dl, tokens, dc, tokens, dp, positive_rows, dn, negative_rows, opt);
    if (r != S2_OK) return r;
    if (cudaMemcpy2DAsync(latent, (size_t)latent_cstep * 4, dl, plane, plane, s2::kPredChannels,
                          cudaMemcpyDeviceToHost, c.stream) != cudaSuccess)
        return S2_ERR_CUDA;
    return cudaStreamSynchronize(c.stream) == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

} // extern "C"
