// s2_awa_forward_static: the AdaptiveWindowAttention forward for callers that
// cannot allocate device memory.
//
// Who needs it: hosts that own every byte of device memory and hand plugins
// only their inputs and outputs (an ncnn-style allocator, an inference
// server's fixed memory budget, an MPS client with a hard memory cap), and
// latency-critical loops that must not call cudaMalloc/cudaFree, which can
// synchronise the whole device.  s2_awa_forward needs a context (s2_init
// allocates a status word) plus workspace and schedule tables it allocates
// on first use; this entry point needs neither.
//
// Its scratch -- schedule tables, the packed bf16 Q/K/V of every window,
// the per-window text partials and a status word -- lives in one file-scope
// __device__ array of S2_AWA_STATIC_SCRATCH_BYTES, which every GPU that loads
// the library holds until the process exits.  The window plan is built on
// the host into a file-scope static table (no heap either).
//
// Host code cannot use the array's name as a device address (it is a host
// stand-in), so the first call on each device, with that device current,
// resolves it with cudaGetSymbolAddress and caches the result; make that
// first call before any stream capture.  Every call shares the array and
// leaves its contents behind: the status word is cleared on entry and every
// other byte a call reads is written earlier by the same call.  Calls whose
// GPU work overlaps (different streams, or several host threads) race on the
// array; the host-side part is serialised by a mutex.
//
// A bounded device wait that runs out (or a bad table index) is recorded in
// the scratch's status word, not returned by the call, which only enqueues;
// s2_awa_static_status reads it back (after the stream's work) and clears it.
// Each call clears the word on entry, so read it before the next call.
#include <math.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "s2_common.cuh"
#include "s2_internal.h"

namespace {

constexpr size_t kScratchBytes = S2_AWA_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
constexpr size_t kHostTableInts = size_t(4) << 20; // 16 MiB of host table space

__device__ __align__(256) unsigned char g_awa_scratch[kScratchBytes];

int g_host_tables[kHostTableInts];
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices];
int g_num_sms[kMaxDevices];

size_t up256(size_t b)
{
    return (b + 255) & ~size_t(255);
}

int ceil_div(int a, int b)
{
    return (a + b - 1) / b;
}

// Window extents and shifted bounds: the rule of build_adaptive_window_plan
// (adaptive_window_attention.cpp:577-629), as in the allocating planner.
int extents(int t, int h, int w, int mode, const int* win, int& wt, int& wh, int& ww)
{
    if (t <= 0 || h <= 0 || w <= 0 || win[0] <= 0 || win[1] <= 0 || win[2] <= 0) return S2_ERR_INVALID;
    if (mode == S2_WINDOW_TARGET)
    {
        const double scale = sqrt(3600.0 / static_cast<double>(h * w));
        const int rh = static_cast<int>(nearbyint(h * scale));
        const int rw = static_cast<int>(nearbyint(w * scale));
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

void axis_of(int ext, int win, int shifted, int& count, double& shift)
{
    shift = (shifted && win < ext) ? 0.5 : 0.0;
    if (!shifted)
        count = ceil_div(ext, win);
    else
        count = shift > 0.0 ? static_cast<int>(ceil((ext - shift) / win)) + 1 : 1;
}

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

// First video token / text row of sample s in the flattened batch.
int nt_offset_video(const int* shapes, int s)
{
    int o = 0;
    for (int i = 0; i < s; i++) o += shapes[3 * i] * shapes[3 * i + 1] * shapes[3 * i + 2];
    return o;
}

int text_offset(const int* tl, int s)
{
    int o = 0;
    for (int i = 0; i < s; i++) o += tl[i];
    return o;
}

// Host table layout (ints), mirrored 1:1 into the device scratch:
//   row_src[R] row_pos[3R] win_info[4 nw] win_pool[nw] items[2 ni]
//   video_indices[n] text_reduce[4 Nt] text_scale[Nt] (float bits)
struct Layout
{
    int R = 0, nw = 0, ni = 0, n = 0, nt = 0, pool = 0;
    size_t o_src, o_pos, o_win, o_pool, o_items, o_vi, o_red, o_scale, total_ints;
    void place()
    {
        size_t o = 0;
        auto take = [&](size_t ints) {
            const size_t r = o;
            o += (ints + 63) & ~size_t(63); // 256-byte aligned pieces
            return r;
        };
        o_src = take(R);
        o_pos = take(3 * (size_t)R);
        o_win = take(4 * (size_t)nw);
        o_pool = take(nw);
        o_items = take(2 * (size_t)ni);
        o_vi = take(n);
        o_red = take(4 * (size_t)nt);
        o_scale = take(nt);
        total_ints = o;
    }
};

// Walks the plan twice: sizes only (fill=false), then fills the host tables.
// Also checks that every video token is covered exactly once (-2 otherwise,
// as :642-653), using the scratch range after the tables for the inverse map.
int walk(const s2_awa_params* p, const int* shapes, const int* tl, int batch, Layout& L, bool fill)
{
    int* T = g_host_tables;
    int nw = 0, n = 0, seq = 0, pool = 0, ni = 0, nt = 0;
    for (int s = 0; s < batch; s++)
    {
        if (tl[s] <= 0) return S2_ERR_INVALID;
        const int t = shapes[3 * s], h = shapes[3 * s + 1], w = shapes[3 * s + 2];
        int wt, wh, ww;
        const int r = extents(t, h, w, p->window_mode, p->window, wt, wh, ww);
        if (r != S2_OK) return r;
        int ct, ch, cw;
        double st, sh, sw;
        axis_of(t, wt, p->shifted, ct, st);
        axis_of(h, wh, p->shifted, ch, sh);
        axis_of(w, ww, p->shifted, cw, sw);
        const int sample_first_pool = pool, first_window = nw;
        const int vbase = nt_offset_video(shapes, s);
        for (int iw = 0; iw < cw; iw++)
        {
            int w0, w1;
            bounds(iw, w, ww, p->shifted, sw, w0, w1);
            if (w1 <= w0) continue;
            for (int ih = 0; ih < ch; ih++)
            {
                int h0, h1;
                bounds(ih, h, wh, p->shifted, sh, h0, h1);
                if (h1 <= h0) continue;
                for (int it = 0; it < ct; it++)
                {
                    int t0, t1;
                    bounds(it, t, wt, p->shifted, st, t0, t1);
                    if (t1 <= t0) continue;
                    const int Lw = (t1 - t0) * (h1 - h0) * (w1 - w0);
                    if (fill)
                    {
                        int* win = T + L.o_win + 4 * (size_t)nw;
                        win[0] = seq;
                        win[1] = Lw;
                        win[2] = tl[s];
                        win[3] = n;
                        T[L.o_pool + nw] = pool;
                        int row = seq, part = n;
                        for (int ti = t0; ti < t1; ti++)
                            for (int hi = h0; hi < h1; hi++)
                                for (int wi = w0; wi < w1; wi++, row++, part++)
                                {
                                    const int src = vbase + (ti * h + hi) * w + wi;
                                    T[L.o_src + row] = src;
                                    T[L.o_pos + 3 * (size_t)row] = ti - t0 + tl[s];
                                    T[L.o_pos + 3 * (size_t)row + 1] = hi - h0;
                                    T[L.o_pos + 3 * (size_t)row + 2] = wi - w0;
                                    T[L.o_vi + part] = src;
                                }
                        const int text0 = text_offset(tl, s);
                        for (int j = 0; j < tl[s]; j++, row++)
                        {
                            T[L.o_src + row] = -1 - (text0 + j);
                            T[L.o_pos + 3 * (size_t)row] = j;
                            T[L.o_pos + 3 * (size_t)row + 1] = j;
                            T[L.o_pos + 3 * (size_t)row + 2] = j;
                        }
                    }
                    ni += ceil_div(Lw + tl[s], 256);
                    seq += Lw + tl[s];
                    pool += tl[s];
                    n += Lw;
                    nw++;
                }
            }
        }
        const int cnt = nw - first_window;
        if (fill)
            for (int j = 0; j < tl[s]; j++)
            {
                int* red = T + L.o_red + 4 * (size_t)(nt + j);
                red[0] = cnt > 0 ? sample_first_pool + j : 0;
                red[1] = tl[s];
                red[2] = cnt;
                red[3] = 0;
                const float sc = cnt > 0 ? 1.f / cnt : 0.f;
                std::memcpy(T + L.o_scale + nt + j, &sc, 4);
            }
        nt += tl[s];
    }
    if (!fill)
    {
        L.R = seq;
        L.nw = nw;
        L.ni = ni;
        L.n = n;
        L.nt = nt;
        L.pool = pool;
        return S2_OK;
    }
    // q-tiles longest-first, ties in window order (same order as the
    // allocating path's stable sort).
    int max_tiles = 0;
    for (int w = 0; w < L.nw; w++)
        max_tiles = std::max(max_tiles, ceil_div(T[L.o_win + 4 * w + 1] + T[L.o_win + 4 * w + 2], 128));
    int k = 0;
    for (int cost = max_tiles; cost >= 1; cost--)
        for (int w = 0; w < L.nw; w++)
        {
            const int S = T[L.o_win + 4 * w + 1] + T[L.o_win + 4 * w + 2];
            if (ceil_div(S, 128) != cost) continue;
            for (int q0 = 0; q0 < S; q0 += 256, k++)
            {
                T[L.o_items + 2 * (size_t)k] = w;
                T[L.o_items + 2 * (size_t)k + 1] = q0;
            }
        }
    // coverage check on the host table space past the tables: the windows
    // hold exactly the samples' t*h*w tokens, each once (plan.cpp's check)
    long long total = 0;
    for (int s = 0; s < batch; s++) total += (long long)shapes[3 * s] * shapes[3 * s + 1] * shapes[3 * s + 2];
    if (total != L.n) return S2_ERR_PLAN;
    int* inv = T + L.total_ints;
    for (int i = 0; i < L.n; i++) inv[i] = -1;
    for (int i = 0; i < L.n; i++)
    {
        const int src = T[L.o_vi + i];
        if (src < 0 || src >= L.n || inv[src] != -1) return S2_ERR_PLAN;
        inv[src] = i;
    }
    return S2_OK;
}

} // namespace

extern "C" int s2_awa_forward_static(const s2_awa_params* prm, const int* video_shapes, const int* text_lengths,
                                     int batch, int in_dtype, const void* video_q, const void* video_k,
                                     const void* video_v, int64_t video_ld, const void* text_q, const void* text_k,
                                     const void* text_v, int64_t text_ld, int out_dtype, void* video_out,
                                     void* text_out, void* stream)
{
    if (!prm || !video_shapes || !text_lengths || batch <= 0 || !video_q || !video_k || !video_v || !text_q ||
        !text_k || !text_v || !video_out || !text_out)
        return S2_ERR_INVALID;
    if (prm->heads <= 0 || prm->head_dim != 128 || prm->rope_pairs <= 0 || prm->rope_pairs * 6 > prm->head_dim ||
        !prm->norm_weights || !prm->rope_freqs)
        return S2_ERR_INVALID;
    if ((in_dtype != S2_DTYPE_F32 && in_dtype != S2_DTYPE_BF16) ||
        (out_dtype != S2_DTYPE_F32 && out_dtype != S2_DTYPE_BF16))
        return S2_ERR_INVALID;
    const int inner = prm->heads * prm->head_dim;
    if (video_ld < inner || text_ld < inner) return S2_ERR_INVALID;

    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return S2_ERR_CUDA;
    if (device < 0 || device >= kMaxDevices) return S2_ERR_DEVICE;

    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_scratch_ptr[device])
    {
        // Once per device, with that device current.
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_awa_scratch) != cudaSuccess || !ptr) return S2_ERR_CUDA;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return S2_ERR_CUDA;
        g_num_sms[device] = sms;
        g_scratch_ptr[device] = ptr;
    }

    Layout L;
    int r = walk(prm, video_shapes, text_lengths, batch, L, false);
    if (r != S2_OK) return r;
    L.place();
    // Limits: host tables (+ the coverage map) and the device scratch.
    const size_t table_bytes = L.total_ints * 4;
    const size_t packed_bytes = up256((size_t)L.R * inner * 2);
    const size_t partial_bytes = up256((size_t)L.pool * inner * 4);
    const size_t need = 256 + up256(table_bytes) + 3 * packed_bytes + partial_bytes;
    if (L.total_ints + (size_t)L.n > kHostTableInts || need > kScratchBytes) return S2_ERR_TOO_LARGE;
    r = walk(prm, video_shapes, text_lengths, batch, L, true);
    if (r != S2_OK) return r;

    unsigned char* base = static_cast<unsigned char*>(g_scratch_ptr[device]);
    int* status = reinterpret_cast<int*>(base);
    unsigned char* tables = base + 256;
    unsigned char* q = tables + up256(table_bytes);
    unsigned char* k = q + packed_bytes;
    unsigned char* v = k + packed_bytes;
    float* partial = reinterpret_cast<float*>(v + packed_bytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The status word must start at zero; everything else read below is
    // written earlier in this call.
    if (cudaMemsetAsync(status, 0, sizeof(int), st) != cudaSuccess) return S2_ERR_CUDA;
    if (cudaMemcpyAsync(tables, g_host_tables, table_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return S2_ERR_CUDA;

    s2::AttnSchedule s; // views into the scratch; owns nothing (block stays null)
    int* dt = reinterpret_cast<int*>(tables);
    s.num_windows = L.nw;
    s.packed_rows = L.R;
    s.num_items = L.ni;
    s.total_text = L.nt;
    s.partial_rows = L.pool;
    // video rows are the tokens themselves here (gather and scatter by token id)
    s.num_video_indices = s.src_rows = s.out_rows = L.n;
    s.row_src = dt + L.o_src;
    s.row_pos = dt + L.o_pos;
    s.win_info = reinterpret_cast<int4*>(dt + L.o_win);
    s.win_pool = dt + L.o_pool;
    s.items = reinterpret_cast<int2*>(dt + L.o_items);
    s.video_indices = dt + L.o_vi;
    s.text_reduce = reinterpret_cast<int4*>(dt + L.o_red);
    s.text_scale = reinterpret_cast<float*>(dt + L.o_scale);

    s2::Context c; // stack context: no workspace, counters off
    c.device = device;
    c.stream = st;
    c.num_sms = g_num_sms[device];
    c.status = status;
    r = s2::launch_prepare_qkv(c, s, prm->heads, prm->head_dim, prm->rope_pairs, prm->epsilon, prm->norm_weights,
                               prm->rope_freqs, in_dtype == S2_DTYPE_BF16, video_q, video_k, video_v, video_ld,
                               text_q, text_k, text_v, text_ld, q, k, v);
    if (r != S2_OK) return r;
    const int out_f32 = out_dtype == S2_DTYPE_F32;
    r = s2::launch_window_attention(c, s, prm->heads, q, k, v, out_f32, prm->official_bf16_attention, video_out,
                                    partial);
    if (r != S2_OK) return r;
    return s2::launch_text_pool(c, s, inner, partial, out_f32, prm->official_bf16_attention, text_out);
}

extern "C" int s2_awa_static_status(void* stream)
{
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return S2_ERR_CUDA;
    if (device < 0 || device >= kMaxDevices) return S2_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(g_mutex);
    // no call has run on this device yet: nothing can have been recorded
    if (!g_scratch_ptr[device]) return S2_OK;
    int* status = static_cast<int*>(g_scratch_ptr[device]);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int h = 0;
    if (cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return S2_ERR_CUDA;
    if (h != 0 && (cudaMemsetAsync(status, 0, sizeof(int), st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess))
        return S2_ERR_CUDA;
    if (h == s2::kStatusTimeout) return S2_ERR_TIMEOUT;
    return h != 0 ? S2_ERR_INVALID : S2_OK;
}
