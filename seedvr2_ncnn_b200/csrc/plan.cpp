// Host side of the window path: the window plan (bit-exact with the
// reference's build_adaptive_window_plan), the device attention schedule
// derived from it, TMA descriptor encoding and workspace buffers.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>

#include "s2_internal.h"

namespace s2 {

// ---------------------------------------------------------------- plan
namespace {

int ceil_div(int a, int b)
{
    return (a + b - 1) / b;
}

// Extents per axis.  Target mode: adaptive_window_attention.cpp:577-588 --
// scale = sqrt(3600 / (h*w)), resized extents rounded half-to-even
// (nearbyint under the default rounding mode, :439-444), window =
// ceil(min(t,30)/n_t), ceil(round(h*scale)/n_h), ceil(round(w*scale)/n_w).
// Extent mode: the tuple is the window extent itself.
int extents(int t, int h, int w, int mode, const int* win, int& wt, int& wh, int& ww)
{
    if (t <= 0 || h <= 0 || w <= 0 || win[0] <= 0 || win[1] <= 0 || win[2] <= 0) return S2_ERR_INVALID;
    if (mode == S2_WINDOW_TARGET)
    {
        const double scale = std::sqrt(3600.0 / static_cast<double>(h * w));
        const int rh = static_cast<int>(std::nearbyint(h * scale));
        const int rw = static_cast<int>(std::nearbyint(w * scale));
        wt = ceil_div(std::min(t, 30), win[0]);
        wh = ceil_div(rh, win[1]);
        ww = ceil_div(rw, win[2]);
    }
    else if (mode == S2_WINDOW_EXTENT)
    {
        wt = win[0];
        wh = win[1];
        ww = win[2];
    }
    else
        return S2_ERR_INVALID;
    return (wt > 0 && wh > 0 && ww > 0) ? S2_OK : S2_ERR_INVALID;
}

struct Axis
{
    int count;
    double shift;
};

// :592-598: a half-window shift applies only when shifted and window < extent;
// shifted count = ceil((ext - 0.5) / win) + 1, else ceil(ext / win).
Axis axis(int ext, int win, int shifted)
{
    Axis a;
    a.shift = (shifted && win < ext) ? 0.5 : 0.0;
    if (!shifted)
        a.count = ceil_div(ext, win);
    else
        a.count = a.shift > 0.0 ? static_cast<int>(std::ceil((ext - a.shift) / win)) + 1 : 1;
    return a;
}

// :611-629: shifted bounds truncate toward zero (static_cast<int>) before the clamp.
void bounds(int i, int ext, int win, int shifted, double s, int& lo, int& hi)
{
    if (shifted)
    {
        lo = std::max(static_cast<int>((i - s) * win), 0);
        hi = std::min(static_cast<int>((i - s + 1.0) * win), ext);
    }
    else
    {
        lo = i * win;
        hi = std::min((i + 1) * win, ext);
    }
}

} // namespace

int build_plan(const int* shapes, int batch, const int* window, int window_mode, int shifted, Plan& plan)
{
    plan = Plan();
    if (!shapes || !window || batch <= 0) return S2_ERR_INVALID;
    plan.batch = batch;
    plan.shapes.assign(shapes, shapes + 3 * batch);
    int total = 0;
    for (int s = 0; s < batch; s++)
    {
        const int t = shapes[3 * s], h = shapes[3 * s + 1], w = shapes[3 * s + 2];
        int wt, wh, ww;
        const int r = extents(t, h, w, window_mode, window, wt, wh, ww);
        if (r != S2_OK) return r;
        const Axis at = axis(t, wt, shifted), ah = axis(h, wh, shifted), aw = axis(w, ww, shifted);
        const int first = static_cast<int>(plan.windows.size() / 9);
        plan.sample_first_window.push_back(first);
        // Window order w outer, h, t inner (:600-630); tokens t, h, w inside
        // a window (append_slice, :446-473).
        for (int iw = 0; iw < aw.count; iw++)
        {
            int w0, w1;
            bounds(iw, w, ww, shifted, aw.shift, w0, w1);
            if (w1 <= w0) continue;
            for (int ih = 0; ih < ah.count; ih++)
            {
                int h0, h1;
                bounds(ih, h, wh, shifted, ah.shift, h0, h1);
                if (h1 <= h0) continue;
                for (int it = 0; it < at.count; it++)
                {
                    int t0, t1;
                    bounds(it, t, wt, shifted, at.shift, t0, t1);
                    if (t1 <= t0) continue;
                    const int offset = static_cast<int>(plan.video_indices.size());
                    const int count = (t1 - t0) * (h1 - h0) * (w1 - w0);
                    const int rec[9] = {s, t0, t1, h0, h1, w0, w1, offset, count};
                    plan.windows.insert(plan.windows.end(), rec, rec + 9);
                    plan.max_window_tokens = std::max(plan.max_window_tokens, count);
                    for (int ti = t0; ti < t1; ti++)
                        for (int hi = h0; hi < h1; hi++)
                            for (int wi = w0; wi < w1; wi++)
                            {
                                plan.video_indices.push_back(total + (ti * h + hi) * w + wi);
                                plan.local_positions.push_back(ti - t0);
                                plan.local_positions.push_back(hi - h0);
                                plan.local_positions.push_back(wi - w0);
                            }
                }
            }
        }
        plan.sample_window_count.push_back(static_cast<int>(plan.windows.size() / 9) - first);
        total += t * h * w;
    }
    // Coverage: every token exactly once (:642-653).
    if (static_cast<int>(plan.video_indices.size()) != total) return S2_ERR_PLAN;
    plan.inverse_video_indices.assign(total, -1);
    for (int p = 0; p < total; p++)
    {
        const int src = plan.video_indices[p];
        if (src < 0 || src >= total || plan.inverse_video_indices[src] != -1) return S2_ERR_PLAN;
        plan.inverse_video_indices[src] = p;
    }
    return S2_OK;
}

// ---------------------------------------------------------------- schedule
AttnSchedule::~AttnSchedule()
{
    if (block) cudaFree(block);
}

int build_schedule(const Plan& plan, const int* text_lengths, AttnSchedule& s, cudaStream_t stream)
{
    return build_schedule_ex(plan, text_lengths, nullptr, nullptr, s, stream, nullptr);
}

// Schedule over a subset of the plan's windows (nullptr = all), with video
// tokens mapped to the rows of the caller's qkv / output buffers through
// row_of_token (nullptr = identity).  Text rows are pooled with the
// sample's GLOBAL window count, so per-rank partial sums add up to the mean
// (adaptive_window_attention.cpp:963-974).
int build_schedule_ex(const Plan& plan, const int* text_lengths, const std::vector<int>* windows_subset,
                      const std::vector<int>* row_of_token, AttnSchedule& s, cudaStream_t stream,
                      const std::vector<int>* out_of_token)
{
    const int nw_all = static_cast<int>(plan.windows.size() / 9);
    std::vector<int> wsel;
    if (windows_subset)
        wsel = *windows_subset;
    else
    {
        wsel.resize(nw_all);
        std::iota(wsel.begin(), wsel.end(), 0);
    }
    const int nw = static_cast<int>(wsel.size());
    auto row_of = [&](int token) { return row_of_token ? (*row_of_token)[token] : token; };
    // where the attention epilogue stores the token's context row (defaults to its input row)
    auto out_of = [&](int token) { return out_of_token ? (*out_of_token)[token] : row_of(token); };
    std::vector<int> text_offset(plan.batch, 0);
    int total_text = 0, max_text = 0;
    for (int b = 0; b < plan.batch; b++)
    {
        if (text_lengths[b] <= 0) return S2_ERR_INVALID;
        text_offset[b] = total_text;
        total_text += text_lengths[b];
        max_text = std::max(max_text, text_lengths[b]);
    }
    std::vector<int> row_src, row_pos, vidx;
    std::vector<int4> win_info(nw);
    std::vector<int> win_pool(nw);
    std::vector<int2> items;
    std::vector<int> item_cost;
    std::vector<int> sample_first(plan.batch, -1), sample_count(plan.batch, 0);
    int seq = 0, pool = 0;
    s.attn_flops_per_head = 0;
    for (int k = 0; k < nw; k++)
    {
        const int w = wsel[k];
        if (w < 0 || w >= nw_all) return S2_ERR_INVALID;
        const int* rec = &plan.windows[9 * w];
        const int sample = rec[0], part = rec[7], L = rec[8], T = text_lengths[sample];
        if (sample_first[sample] < 0) sample_first[sample] = k;
        sample_count[sample]++;
        win_info[k] = make_int4(seq, L, T, static_cast<int>(vidx.size()));
        win_pool[k] = pool;
        for (int r = 0; r < L; r++)
        {
            const int token = plan.video_indices[part + r];
            const int row = row_of(token);
            if (row < 0 || out_of(token) < 0) return S2_ERR_PLAN;
            row_src.push_back(row);
            vidx.push_back(out_of(token));
            // video RoPE position: window-local (t + text_len, h, w) (:904-905)
            row_pos.push_back(plan.local_positions[3 * (part + r)] + T);
            row_pos.push_back(plan.local_positions[3 * (part + r) + 1]);
            row_pos.push_back(plan.local_positions[3 * (part + r) + 2]);
        }
        for (int j = 0; j < T; j++)
        {
            row_src.push_back(-1 - (text_offset[sample] + j));
            // text RoPE position (i, i, i) (:915)
            row_pos.push_back(j);
            row_pos.push_back(j);
            row_pos.push_back(j);
        }
        const int S = L + T;
        const int ntiles = (S + 127) / 128;
        s.attn_flops_per_head += 4.0 * S * (double)S * 128.0;
        for (int q0 = 0; q0 < S; q0 += 256) // one item = a pair of 128-row query tiles
        {
            items.push_back(make_int2(k, q0));
            item_cost.push_back(ntiles);
        }
        seq += S;
        pool += T;
    }
    // Longest-first: q-tiles of the biggest windows start first.
    std::vector<int> order(items.size());
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return item_cost[a] > item_cost[b]; });
    std::vector<int2> sorted(items.size());
    for (size_t i = 0; i < order.size(); i++) sorted[i] = items[order[i]];

    std::vector<int4> reduce(total_text);
    std::vector<float> scale(total_text);
    for (int b = 0; b < plan.batch; b++)
    {
        const int cnt = sample_count[b], total = plan.sample_window_count[b];
        for (int j = 0; j < text_lengths[b]; j++)
        {
            reduce[text_offset[b] + j] = make_int4(cnt > 0 ? win_pool[sample_first[b]] + j : 0, text_lengths[b], cnt, 0);
            scale[text_offset[b] + j] = total > 0 ? 1.f / total : 0.f;
        }
    }

    // Inverse of row_src: packed row of each video row, and the packed rows
    // (one per window) of each text row.
    int max_row = -1;
    for (int v : row_src) max_row = std::max(max_row, v);
    std::vector<int> pack_dst(max_row + 1, -1);
    std::vector<std::vector<int>> text_rows(total_text);
    for (size_t r = 0; r < row_src.size(); r++)
    {
        if (row_src[r] >= 0)
            pack_dst[row_src[r]] = static_cast<int>(r);
        else
            text_rows[-1 - row_src[r]].push_back(static_cast<int>(r));
    }
    std::vector<int> text_dst_off(total_text + 1, 0), text_dst;
    for (int t = 0; t < total_text; t++)
    {
        text_dst_off[t] = static_cast<int>(text_dst.size());
        text_dst.insert(text_dst.end(), text_rows[t].begin(), text_rows[t].end());
    }
    text_dst_off[total_text] = static_cast<int>(text_dst.size());

    // One device block for every table.
    const size_t n_tok = vidx.size();
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~size_t(255);
        return o;
    };
    const size_t o_src = take(row_src.size() * 4), o_pos = take(row_pos.size() * 4), o_win = take(nw * 16),
                 o_pool = take(nw * 4), o_items = take(sorted.size() * 8), o_vi = take(n_tok * 4),
                 o_red = take(total_text * 16), o_scale = take(total_text * 4), o_pd = take(pack_dst.size() * 4),
                 o_tdo = take(text_dst_off.size() * 4), o_td = take(text_dst.size() * 4);
    if (s.block)
    {
        cudaFree(s.block);
        s.block = nullptr;
    }
    if (cudaMalloc(&s.block, off ? off : 256) != cudaSuccess) return S2_ERR_ALLOC;
    std::vector<uint8_t> host(off ? off : 256, 0);
    auto put = [&](size_t o, const void* src, size_t bytes) {
        if (bytes) std::memcpy(host.data() + o, src, bytes);
    };
    put(o_src, row_src.data(), row_src.size() * 4);
    put(o_pos, row_pos.data(), row_pos.size() * 4);
    put(o_win, win_info.data(), nw * 16);
    put(o_pool, win_pool.data(), nw * 4);
    put(o_items, sorted.data(), sorted.size() * 8);
    put(o_vi, vidx.data(), n_tok * 4);
    put(o_red, reduce.data(), total_text * 16);
    put(o_scale, scale.data(), total_text * 4);
    put(o_pd, pack_dst.data(), pack_dst.size() * 4);
    put(o_tdo, text_dst_off.data(), text_dst_off.size() * 4);
    put(o_td, text_dst.data(), text_dst.size() * 4);
    if (cudaMemcpyAsync(s.block, host.data(), host.size(), cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
        return S2_ERR_CUDA;
    uint8_t* base = static_cast<uint8_t*>(s.block);
    s.row_src = reinterpret_cast<int*>(base + o_src);
    s.row_pos = reinterpret_cast<int*>(base + o_pos);
    s.win_info = reinterpret_cast<int4*>(base + o_win);
    s.win_pool = reinterpret_cast<int*>(base + o_pool);
    s.items = reinterpret_cast<int2*>(base + o_items);
    s.video_indices = reinterpret_cast<int*>(base + o_vi);
    s.text_reduce = reinterpret_cast<int4*>(base + o_red);
    s.text_scale = reinterpret_cast<float*>(base + o_scale);
    s.pack_dst = reinterpret_cast<int*>(base + o_pd);
    s.pack_dst_rows = static_cast<int>(pack_dst.size());
    s.max_pos = 0;
    for (int v : row_pos) s.max_pos = std::max(s.max_pos, v + 1);
    s.text_dst_off = reinterpret_cast<int*>(base + o_tdo);
    s.text_dst = reinterpret_cast<int*>(base + o_td);
    s.num_windows = nw;
    s.packed_rows = seq;
    s.num_items = static_cast<int>(sorted.size());
    s.total_text = total_text;
    s.max_text = max_text;
    s.partial_rows = pool;
    s.num_video_indices = static_cast<int>(n_tok);
    s.src_rows = max_row + 1;
    s.out_rows = 0;
    for (int v : vidx) s.out_rows = std::max(s.out_rows, (v & ((1 << kPeerShift) - 1)) + 1);
    return S2_OK;
}

// ---------------------------------------------------------------- TMA maps
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn)
    {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}
} // namespace

// 2-D bf16 tensor [outer][inner] with 128-byte swizzle; box = box_inner x
// box_outer (box_inner * 2 bytes must be 128); out-of-range elements read 0.
int make_tmap_2d(CUtensorMap* map, const void* base, int f32, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return S2_ERR_DEVICE;
    const uint32_t esz = f32 ? 4 : 2;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15) || box_inner * esz != 128)
        return S2_ERR_INVALID;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                          const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? S2_OK : S2_ERR_INVALID;
}

int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                      uint32_t box_inner, uint32_t box_outer)
{
    return make_tmap_2d(map, base, 0, inner, outer, row_stride_bytes, box_inner, box_outer);
}

int make_tmap_bf16_4d(CUtensorMap* map, const void* base, const uint64_t* dims, const uint64_t* stride_bytes,
                      const uint32_t* box, const uint32_t* element_strides)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return S2_ERR_DEVICE;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || box[0] * 2 != 128) return S2_ERR_INVALID;
    for (int i = 0; i < 3; i++)
        if (stride_bytes[i] & 15) return S2_ERR_INVALID;
    const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
    const cuuint64_t st[3] = {stride_bytes[0], stride_bytes[1], stride_bytes[2]};
    const cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
    const cuuint32_t estr[4] = {element_strides[0], element_strides[1], element_strides[2], element_strides[3]};
    if (estr[0] != 1) return S2_ERR_INVALID;
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), d, st, bx, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? S2_OK : S2_ERR_INVALID;
}

// ---------------------------------------------------------------- buffers
int DeviceBuffer::ensure(size_t want)
{
    if (want <= bytes) return S2_OK;
    release();
    want = (want + 4095) & ~size_t(4095);
    if (cudaMalloc(&ptr, want) != cudaSuccess)
    {
        ptr = nullptr;
        return S2_ERR_ALLOC;
    }
    bytes = want;
    return S2_OK;
}

void DeviceBuffer::release()
{
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
}

} // namespace s2

// ---------------------------------------------------------------- counters
namespace s2 {

void Profiler::reset()
{
    collect();
    for (int k = 0; k < K_NUM; k++)
    {
        launches[k] = 0;
        ms[k] = flops[k] = bytes[k] = 0.0;
    }
}

int Profiler::collect()
{
    int r = S2_OK;
    for (Record& rec : pending)
    {
        float t = 0.f;
        if (cudaEventSynchronize(rec.stop) != cudaSuccess || cudaEventElapsedTime(&t, rec.start, rec.stop) != cudaSuccess)
            r = S2_ERR_CUDA;
        launches[rec.kind] += 1;
        ms[rec.kind] += t;
        flops[rec.kind] += rec.flops;
        bytes[rec.kind] += rec.bytes;
        pool.push_back(rec.start);
        pool.push_back(rec.stop);
    }
    pending.clear();
    return r;
}

void Profiler::release()
{
    collect();
    for (cudaEvent_t e : pool) cudaEventDestroy(e);
    pool.clear();
}

static cudaEvent_t take_event(Profiler& p)
{
    if (!p.pool.empty())
    {
        cudaEvent_t e = p.pool.back();
        p.pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

ProfileScope::ProfileScope(Context& c, int kind, double f, double b) : ctx(c), on(c.prof.on)
{
    if (!on) return;
    rec.kind = kind;
    rec.flops = f;
    rec.bytes = b;
    rec.start = take_event(c.prof);
    rec.stop = take_event(c.prof);
    cudaEventRecord(rec.start, c.stream);
}

ProfileScope::~ProfileScope()
{
    if (!on) return;
    cudaEventRecord(rec.stop, ctx.stream);
    ctx.prof.pending.push_back(rec);
}

} // namespace s2
