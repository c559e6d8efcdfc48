// extern "C" entry points of libseedvr2_cuda (include/seedvr2_cuda.h).
#include <cuda_bf16.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <tuple>
#include <vector>

#include "s2_common.cuh"
#include "s2_internal.h"

#include "s2_objects.h"

using s2::Context;

int s2::ensure_schedule(s2_plan* p, const int* text_lengths, Context& ctx, const s2::AttnSchedule** out)
{
    const std::vector<int> tl(text_lengths, text_lengths + p->plan.batch);
    if (!p->sched || p->sched_text != tl || p->sched_device != ctx.device)
    {
        for (int v : tl)
            if (v <= 0) return S2_ERR_INVALID;
        std::unique_ptr<s2::AttnSchedule> s(new s2::AttnSchedule);
        const int r = s2::build_schedule(p->plan, text_lengths, *s, ctx.stream);
        if (r != S2_OK) return r;
        p->sched = std::move(s);
        p->sched_text = tl;
        p->sched_device = ctx.device;
    }
    *out = p->sched.get();
    return S2_OK;
}

namespace {

// Workspace slot assignment.
enum
{
    WS_QKV_PACKED = 0, // AWA: packed bf16 Q, K, V
    WS_TEXT_PARTIAL = 1,
    WS_DIT = 2, // DiT forward activations
    WS_CFG = 3,    // apply_cfg reduction scratch (s2_apply_cfg, dit.cu)
    WS_FINITE = 4, // s2_count_nonfinite's counter
};

} // namespace

extern "C" {

int s2_version(void)
{
    return 1;
}

const char* s2_error_string(int code)
{
    switch (code)
    {
    case S2_OK: return "ok";
    case S2_ERR_INVALID: return "invalid argument or shape";
    case S2_ERR_PLAN: return "inconsistent window plan";
    case S2_ERR_CUDA: return "CUDA error";
    case S2_ERR_TIMEOUT: return "bounded device wait expired";
    case S2_ERR_DEVICE: return "unsupported device (needs sm_100)";
    case S2_ERR_TOO_LARGE: return "input exceeds the fixed static workspace";
    case S2_ERR_ALLOC: return "allocation failure";
    default: return "unknown error";
    }
}

int s2_init(int device, void* stream, s2_context** out)
{
    if (!out) return S2_ERR_INVALID;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) return S2_ERR_DEVICE;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return S2_ERR_CUDA;
    if (prop.major != 10) return S2_ERR_DEVICE; // tcgen05 kernels are built for sm_100a
    if (cudaSetDevice(device) != cudaSuccess) return S2_ERR_CUDA;
    s2_context* c = new s2_context;
    c->c.device = device;
    c->c.stream = static_cast<cudaStream_t>(stream);
    c->c.num_sms = prop.multiProcessorCount;
    if (cudaMalloc(&c->c.status, sizeof(int)) != cudaSuccess)
    {
        delete c;
        return S2_ERR_ALLOC;
    }
    if (cudaMemset(c->c.status, 0, sizeof(int)) != cudaSuccess)
    {
        cudaFree(c->c.status);
        delete c;
        return S2_ERR_CUDA;
    }
    constexpr int kSplitFlagSlots = 16384;
    if (cudaMalloc(&c->c.split_flags, kSplitFlagSlots * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(c->c.split_flags, 0, kSplitFlagSlots * sizeof(unsigned)) != cudaSuccess)
    {
        if (c->c.split_flags) cudaFree(c->c.split_flags);
        cudaFree(c->c.status);
        delete c;
        return S2_ERR_ALLOC;
    }
    c->c.split_slots = kSplitFlagSlots;
    *out = c;
    return S2_OK;
}

void s2_destroy(s2_context* ctx)
{
    if (!ctx) return;
    cudaSetDevice(ctx->c.device);
    cudaStreamSynchronize(ctx->c.stream);
    ctx->plan_cache.clear();
    if (ctx->dist) ctx->dist->destroy();
    ctx->dist.reset();
    ctx->c.prof.release();
    for (auto& b : ctx->c.ws) b.release();
    if (ctx->c.split_flags) cudaFree(ctx->c.split_flags);
    if (ctx->c.status) cudaFree(ctx->c.status);
    delete ctx;
}

int s2_set_stream(s2_context* ctx, void* stream)
{
    if (!ctx) return S2_ERR_INVALID;
    ctx->c.stream = static_cast<cudaStream_t>(stream);
    return S2_OK;
}

uint64_t s2_launch_count(const s2_context* ctx)
{
    return ctx ? ctx->c.launches : 0;
}

int s2_status(s2_context* ctx)
{
    if (!ctx) return S2_ERR_INVALID;
    if (cudaStreamSynchronize(ctx->c.stream) != cudaSuccess) return S2_ERR_CUDA;
    int h = 0;
    if (cudaMemcpy(&h, ctx->c.status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return S2_ERR_CUDA;
    if (h != 0 && cudaMemset(ctx->c.status, 0, sizeof(int)) != cudaSuccess) return S2_ERR_CUDA;
    if (h == s2::kStatusTimeout) return S2_ERR_TIMEOUT;
    if (h != 0) return S2_ERR_INVALID;
    return S2_OK;
}

int s2_profile_enable(s2_context* ctx, int enable)
{
    if (!ctx) return S2_ERR_INVALID;
    ctx->c.prof.reset();
    ctx->c.prof.on = enable != 0;
    return S2_OK;
}

int s2_profile_read(s2_context* ctx, int kind, int64_t* launches, double* milliseconds, double* flops, double* bytes)
{
    if (!ctx || kind < 0 || kind >= S2_NUM_KERNEL_KINDS) return S2_ERR_INVALID;
    const int r = ctx->c.prof.collect();
    if (launches) *launches = ctx->c.prof.launches[kind];
    if (milliseconds) *milliseconds = ctx->c.prof.ms[kind];
    if (flops) *flops = ctx->c.prof.flops[kind];
    if (bytes) *bytes = ctx->c.prof.bytes[kind];
    return r;
}

// ------------------------------------------------------------------ plan
int s2_plan_build(const int* video_shapes, int batch, const int* window, int window_mode, int shifted, s2_plan** out)
{
    if (!out) return S2_ERR_INVALID;
    *out = nullptr;
    s2_plan* p = new s2_plan;
    const int r = s2::build_plan(video_shapes, batch, window, window_mode, shifted, p->plan);
    if (r != S2_OK)
    {
        delete p;
        return r;
    }
    *out = p;
    return S2_OK;
}

int s2_plan_info(const s2_plan* p, int* num_windows, int* num_tokens, int* max_window_tokens)
{
    if (!p) return S2_ERR_INVALID;
    if (num_windows) *num_windows = static_cast<int>(p->plan.windows.size() / 9);
    if (num_tokens) *num_tokens = static_cast<int>(p->plan.video_indices.size());
    if (max_window_tokens) *max_window_tokens = p->plan.max_window_tokens;
    return S2_OK;
}

int s2_plan_copy(const s2_plan* p, int* windows, int* sample_window_count, int* video_indices,
                 int* inverse_video_indices, int* local_positions)
{
    if (!p) return S2_ERR_INVALID;
    const s2::Plan& q = p->plan;
    if (windows) std::memcpy(windows, q.windows.data(), q.windows.size() * 4);
    if (sample_window_count) std::memcpy(sample_window_count, q.sample_window_count.data(), q.batch * 4);
    if (video_indices) std::memcpy(video_indices, q.video_indices.data(), q.video_indices.size() * 4);
    if (inverse_video_indices)
        std::memcpy(inverse_video_indices, q.inverse_video_indices.data(), q.inverse_video_indices.size() * 4);
    if (local_positions) std::memcpy(local_positions, q.local_positions.data(), q.local_positions.size() * 4);
    return S2_OK;
}

int s2_plan_schedule_copy(s2_context* ctx, s2_plan* p, const int* text_lengths, int* sizes, int* row_src,
                          int* row_pos, int* win_info, int* video_indices, int* pack_dst)
{
    if (!ctx || !p || !text_lengths || !sizes) return S2_ERR_INVALID;
    s2::Context& c = ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    const s2::AttnSchedule* s = nullptr;
    int r = s2::ensure_schedule(p, text_lengths, c, &s);
    if (r != S2_OK) return r;
    const int tokens = static_cast<int>(p->plan.video_indices.size());
    sizes[0] = s->packed_rows;
    sizes[1] = s->num_windows;
    sizes[2] = tokens;
    sizes[3] = s->pack_dst_rows;
    // the tables as the kernels read them: copied back from the device
    auto get = [&](int* dst, const void* src, size_t bytes) {
        return !dst || !bytes || cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost) == cudaSuccess;
    };
    if (!get(row_src, s->row_src, (size_t)s->packed_rows * 4) || !get(row_pos, s->row_pos, (size_t)s->packed_rows * 12) ||
        !get(win_info, s->win_info, (size_t)s->num_windows * 16) ||
        !get(video_indices, s->video_indices, (size_t)tokens * 4) ||
        !get(pack_dst, s->pack_dst, (size_t)s->pack_dst_rows * 4))
        return S2_ERR_CUDA;
    return S2_OK;
}

int s2_debug_poke_schedule(s2_context* ctx, s2_plan* p, int table, int index, int value)
{
#ifdef S2_DEBUG_BOUNDS
    if (!ctx || !p || !p->sched || (table != 0 && table != 1) || index < 0) return S2_ERR_INVALID;
    const s2::AttnSchedule& s = *p->sched;
    int* base = table == 0 ? s.row_src : s.video_indices;
    const int n = table == 0 ? s.packed_rows : s.num_video_indices;
    if (index >= n) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return cudaMemcpy(base + index, &value, 4, cudaMemcpyHostToDevice) == cudaSuccess ? S2_OK : S2_ERR_CUDA;
#else
    // only a build whose kernels check table indices may run a corrupted table
    (void)ctx, (void)p, (void)table, (void)index, (void)value;
    return S2_ERR_INVALID;
#endif
}

void s2_plan_free(s2_plan* p)
{
    delete p;
}

// ------------------------------------------------------------------ AWA
int s2_awa_forward(s2_context* ctx, const s2_awa_params* prm, const s2_plan* plan_in, const int* video_shapes,
                   const int* text_lengths, int batch, int in_dtype, const void* video_q, const void* video_k,
                   const void* video_v, int64_t video_ld, const void* text_q, const void* text_k, const void* text_v,
                   int64_t text_ld, int out_dtype, void* video_out, void* text_out)
{
    // Validation mirrors AdaptiveWindowAttention::forward (:766-831).
    if (!ctx || !prm || !text_lengths || batch <= 0 || !video_q || !video_k || !video_v || !text_q || !text_k ||
        !text_v || !video_out || !text_out)
        return S2_ERR_INVALID;
    if (prm->heads <= 0 || prm->head_dim != 128 || prm->rope_pairs <= 0 || prm->rope_pairs * 6 > prm->head_dim ||
        !prm->norm_weights || !prm->rope_freqs)
        return S2_ERR_INVALID;
    if ((in_dtype != S2_DTYPE_F32 && in_dtype != S2_DTYPE_BF16) ||
        (out_dtype != S2_DTYPE_F32 && out_dtype != S2_DTYPE_BF16))
        return S2_ERR_INVALID;
    const int inner = prm->heads * prm->head_dim;
    if (video_ld < inner || text_ld < inner) return S2_ERR_INVALID;
    for (int b = 0; b < batch; b++)
        if (text_lengths[b] <= 0) return S2_ERR_INVALID;
    Context& c = ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;

    s2_plan* plan = const_cast<s2_plan*>(plan_in);
    if (!plan)
    {
        if (!video_shapes) return S2_ERR_INVALID;
        std::vector<int> key(video_shapes, video_shapes + 3 * batch);
        key.push_back(prm->window[0]);
        key.push_back(prm->window[1]);
        key.push_back(prm->window[2]);
        key.push_back(prm->window_mode);
        key.push_back(prm->shifted);
        std::unique_ptr<s2_plan>& slot = ctx->plan_cache[key];
        if (!slot)
        {
            std::unique_ptr<s2_plan> fresh(new s2_plan);
            const int r = s2::build_plan(video_shapes, batch, prm->window, prm->window_mode, prm->shifted, fresh->plan);
            if (r != S2_OK)
            {
                ctx->plan_cache.erase(key);
                return r;
            }
            slot = std::move(fresh);
        }
        plan = slot.get();
    }
    else
    {
        if (plan->plan.batch != batch) return S2_ERR_INVALID;
        if (video_shapes && std::memcmp(video_shapes, plan->plan.shapes.data(), 12 * (size_t)batch) != 0)
            return S2_ERR_INVALID;
    }
    const s2::AttnSchedule* sched = nullptr;
    int r = s2::ensure_schedule(plan, text_lengths, c, &sched);
    if (r != S2_OK) return r;

    const size_t packed_bytes = (size_t)sched->packed_rows * inner * 2;
    if ((r = c.ws[WS_QKV_PACKED].ensure(3 * packed_bytes + 256)) != S2_OK) return r;
    if ((r = c.ws[WS_TEXT_PARTIAL].ensure((size_t)sched->partial_rows * inner * 4 + 256)) != S2_OK) return r;
    uint8_t* qkv = static_cast<uint8_t*>(c.ws[WS_QKV_PACKED].ptr);
    float* partial = static_cast<float*>(c.ws[WS_TEXT_PARTIAL].ptr);

    r = s2::launch_prepare_qkv(c, *sched, prm->heads, prm->head_dim, prm->rope_pairs, prm->epsilon,
                               prm->norm_weights, prm->rope_freqs, in_dtype == S2_DTYPE_BF16, video_q, video_k,
                               video_v, video_ld, text_q, text_k, text_v, text_ld, qkv, qkv + packed_bytes,
                               qkv + 2 * packed_bytes);
    if (r != S2_OK) return r;
    const int out_f32 = out_dtype == S2_DTYPE_F32;
    r = s2::launch_window_attention(c, *sched, prm->heads, qkv, qkv + packed_bytes, qkv + 2 * packed_bytes, out_f32,
                                    prm->official_bf16_attention, video_out, partial);
    if (r != S2_OK) return r;
    return s2::launch_text_pool(c, *sched, inner, partial, out_f32, prm->official_bf16_attention, text_out);
}

// ------------------------------------------------------------------ SharedLinear & block ops
int s2_shared_linear(s2_context* ctx, int M0, int M1, int N, int K, const void* A0, const void* A1, const void* W,
                     const float* bias, int epilogue, const float* gate, int out_dtype, void* out0, void* out1)
{
    if (!ctx || (out_dtype != S2_DTYPE_F32 && out_dtype != S2_DTYPE_BF16) || (N % 8) != 0) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return s2::launch_shared_linear(ctx->c, M0, M1, N, K, A0, A1, W, bias, epilogue, gate,
                                    out_dtype == S2_DTYPE_F32, out0, out1);
}

int s2_ada_rmsnorm(s2_context* ctx, int rows, int D, const float* x, float eps, const float* shift,
                   const float* scale, void* out_bf16)
{
    if (!ctx || !x || !shift || !scale || !out_bf16) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return s2::launch_ada_rmsnorm(ctx->c, rows, D, x, eps, shift, scale, out_bf16);
}

int s2_ada_layernorm(s2_context* ctx, int rows, int D, const float* x, float eps, const float* shift,
                     const float* scale, void* out_bf16)
{
    if (!ctx || !x || !shift || !scale || !out_bf16) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return s2::launch_ada_norm(ctx->c, rows, D, x, eps, shift, scale, out_bf16, 1);
}

int s2_convert_f32_bf16(s2_context* ctx, const float* in, void* out, int64_t count)
{
    if (!ctx || !in || !out) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return s2::launch_convert_f32_bf16(ctx->c, in, out, count);
}

int s2_count_nonfinite(s2_context* ctx, const void* data, int64_t count, int dtype, int64_t* nonfinite)
{
    if (!ctx || !nonfinite || count < 0) return S2_ERR_INVALID;
    *nonfinite = 0;
    if (count == 0) return S2_OK;
    s2::Context& c = ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    int r = c.ws[WS_FINITE].ensure(sizeof(unsigned long long));
    if (r != S2_OK) return r;
    unsigned long long* d = static_cast<unsigned long long*>(c.ws[WS_FINITE].ptr);
    if (cudaMemsetAsync(d, 0, sizeof(*d), c.stream) != cudaSuccess) return S2_ERR_CUDA;
    if ((r = s2::launch_count_nonfinite(c, data, count, dtype, d)) != S2_OK) return r;
    unsigned long long h = 0;
    if (cudaMemcpyAsync(&h, d, sizeof(h), cudaMemcpyDeviceToHost, c.stream) != cudaSuccess ||
        cudaStreamSynchronize(c.stream) != cudaSuccess)
        return S2_ERR_CUDA;
    *nonfinite = (int64_t)h;
    return S2_OK;
}

// ------------------------------------------------------- token formats
int s2_patchify_video(s2_context* ctx, const float* video, int rows, const int* shapes, int batch, float* out)
{
    if (!ctx) return S2_ERR_INVALID;
    const int r = s2::patchify_rows(shapes, batch, rows, nullptr);
    if (r != S2_OK) return r;
    if (!video || !out) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    int64_t v_off = 0, p_off = 0;
    for (int s = 0; s < batch; s++)
    {
        const int* shp = shapes + 3 * s;
        const int e = s2::launch_patchify(ctx->c, video + v_off * s2::kLatentChannels, shp[0], shp[1], shp[2],
                                          out + p_off * s2::kPatchFeatures, 0);
        if (e != S2_OK) return e;
        v_off += (int64_t)shp[0] * shp[1] * shp[2];
        p_off += (int64_t)shp[0] * (shp[1] / 2) * (shp[2] / 2);
    }
    return S2_OK;
}

int s2_unpatchify_prediction(s2_context* ctx, const float* pred, int rows, const int* shapes, int batch, float* out)
{
    if (!ctx) return S2_ERR_INVALID;
    const int r = s2::unpatchify_rows(shapes, batch, rows, nullptr);
    if (r != S2_OK) return r;
    if (!pred || !out) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    int64_t p_off = 0, t_off = 0;
    for (int s = 0; s < batch; s++)
    {
        const int* shp = shapes + 3 * s;
        const int e = s2::launch_unpatchify(ctx->c, pred + p_off * s2::kPredFeatures, shp[0], shp[1], shp[2],
                                            out + t_off * s2::kPredChannels);
        if (e != S2_OK) return e;
        p_off += (int64_t)shp[0] * (shp[1] / 2) * (shp[2] / 2);
        t_off += (int64_t)shp[0] * shp[1] * shp[2];
    }
    return S2_OK;
}

int s2_timestep_embedding(s2_context* ctx, const float* timesteps, int batch, float* out)
{
    // make_timestep_embedding returns -1 for an empty batch (seedvr2_dit.cpp:235-236)
    if (!ctx || batch <= 0 || !timesteps || !out) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return s2::launch_timestep_embedding(ctx->c, timesteps, batch, out);
}

// ------------------------------------------------------------------ multi-GPU
int s2_shard_build(const int* video_shape, int text_length, const int* window, int window_mode, int rank, int world,
                   s2_shard** out)
{
    if (!out) return S2_ERR_INVALID;
    *out = nullptr;
    std::unique_ptr<s2_shard> sh(new s2_shard);
    const int r = s2::build_shard(video_shape, text_length, window, window_mode, rank, world, sh->sp);
    if (r != S2_OK) return r;
    *out = sh.release();
    return S2_OK;
}

int s2_shard_counts(const s2_shard* sh, int shifted, int* n_local, int* send_counts, int* recv_counts)
{
    if (!sh || shifted < 0 || shifted > 1) return S2_ERR_INVALID;
    const s2::ShardPlan& sp = sh->sp;
    if (n_local) *n_local = sp.n_local[sp.rank];
    for (int p = 0; p < sp.world; p++)
    {
        if (send_counts) send_counts[p] = static_cast<int>(sp.send_rows[shifted][p].size());
        if (recv_counts) recv_counts[p] = static_cast<int>(sp.recv_tokens[shifted][p].size());
    }
    return S2_OK;
}

int s2_shard_lists(const s2_shard* sh, int shifted, int* local_tokens, int* send_tokens, int* recv_tokens)
{
    if (!sh || shifted < 0 || shifted > 1) return S2_ERR_INVALID;
    const s2::ShardPlan& sp = sh->sp;
    if (local_tokens) std::memcpy(local_tokens, sp.local_tokens.data(), sp.local_tokens.size() * 4);
    for (int p = 0; p < sp.world; p++)
    {
        const std::vector<int>& st = sp.send_tokens[shifted][p];
        const std::vector<int>& rt = sp.recv_tokens[shifted][p];
        if (send_tokens)
        {
            std::memcpy(send_tokens, st.data(), st.size() * 4);
            send_tokens += st.size();
        }
        if (recv_tokens)
        {
            std::memcpy(recv_tokens, rt.data(), rt.size() * 4);
            recv_tokens += rt.size();
        }
    }
    return S2_OK;
}

int s2_shard_windows(const s2_shard* sh, int shifted, int* count, int* windows)
{
    if (!sh || shifted < 0 || shifted > 1 || !count) return S2_ERR_INVALID;
    const std::vector<int>& wm = sh->sp.win_mine[shifted];
    *count = static_cast<int>(wm.size());
    if (windows) std::memcpy(windows, wm.data(), wm.size() * 4);
    return S2_OK;
}

void s2_shard_free(s2_shard* sh)
{
    delete sh;
}

int s2_dist_unique_id(void* id128)
{
    if (!id128) return S2_ERR_INVALID;
    return s2::nccl_unique_id(id128);
}

int s2_dist_init(s2_context* ctx, const void* id128, int rank, int world, int timeout_ms)
{
    if (!ctx || !id128 || world <= 0 || rank < 0 || rank >= world) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    std::unique_ptr<s2::Dist> d(new s2::Dist);
    const int r = d->init(id128, rank, world, timeout_ms);
    if (r != S2_OK) return r;
    if (ctx->dist) ctx->dist->destroy();
    ctx->dist = std::move(d);
    return S2_OK;
}

int s2_dist_sync(s2_context* ctx)
{
    if (!ctx) return S2_ERR_INVALID;
    if (!ctx->dist) return cudaStreamSynchronize(ctx->c.stream) == cudaSuccess ? S2_OK : S2_ERR_CUDA;
    return ctx->dist->sync(ctx->c.stream);
}

int s2_dist_destroy(s2_context* ctx)
{
    if (!ctx) return S2_ERR_INVALID;
    if (ctx->dist) ctx->dist->destroy();
    ctx->dist.reset();
    return S2_OK;
}

int s2_peer_barrier(s2_context* ctx, void* const* peer_flags, uint32_t* my_flags, int rank, int world,
                    uint32_t epoch)
{
    if (!ctx || !peer_flags || !my_flags || world <= 0 || world > s2::kMaxPeers || rank < 0 || rank >= world)
        return S2_ERR_INVALID;
    for (int i = 0; i < world; i++)
        if (!peer_flags[i] || (reinterpret_cast<uintptr_t>(peer_flags[i]) & 3)) return S2_ERR_INVALID;
    if (reinterpret_cast<uintptr_t>(my_flags) & 3) return S2_ERR_INVALID;
    if (cudaSetDevice(ctx->c.device) != cudaSuccess) return S2_ERR_CUDA;
    return s2::launch_peer_barrier(ctx->c, peer_flags, my_flags, rank, world, epoch);
}

} // extern "C"
