// Multi-GPU plumbing: the token-ownership plan of a sharded DiT forward and a
// NCCL binding (one process per GPU).
//
// Ownership.  The reference runs one device (seedvr2_main.cpp:89-100 forces
// --sp-size 1); sharding is this library's addition.  Every token-wise op of
// a block (norms, the four SharedLinear GEMMs) only needs the token's own row,
// and attention only needs the rows of one window, so:
//   * rank r owns an equal contiguous range of the UNSHIFTED plan's token
//     order (window after window), so the GEMMs are balanced to one row;
//   * every window (unshifted in even blocks, shifted in odd blocks) belongs
//     to the rank holding most of its tokens; that rank receives the raw qkv
//     rows of the window's other tokens (one grouped send/recv exchange) and
//     sends their context rows back (a second exchange) -- in even blocks
//     only the few windows cut by a range boundary exchange anything;
//   * text tokens are replicated on every rank; each rank pools the text rows
//     of its own windows with the sample's global window count and the
//     partial sums are all-reduced (sum), which reproduces the reference's
//     mean over all windows (adaptive_window_attention.cpp:963-974).
//
// NCCL is loaded with dlopen (the copy torch already loaded, else the
// system's), communicators are created non-blocking, and every host wait on
// them is bounded: on expiry the communicator is aborted and S2_ERR_TIMEOUT
// returned.
#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <numeric>
#include <thread>

#include "s2_dist.h"

namespace s2 {

// ---------------------------------------------------------------- ownership
int build_shard(const int* shape, int text_length, const int* window, int window_mode, int rank, int world,
                ShardPlan& sp)
{
    sp = ShardPlan();
    if (!shape || text_length <= 0 || world <= 0 || rank < 0 || rank >= world) return S2_ERR_INVALID;
    for (int p = 0; p < 2; p++)
    {
        const int r = build_plan(shape, 1, window, window_mode, p, sp.plan[p]);
        if (r != S2_OK) return r;
    }
    sp.world = world;
    sp.rank = rank;
    sp.T = text_length;
    const int Nv = static_cast<int>(sp.plan[0].video_indices.size());
    sp.Nv = Nv;

    // Tokens: equal contiguous ranges of the unshifted plan's partition order
    // (window after window), so every token-wise op is balanced to one row.
    sp.token_owner.assign(Nv, -1);
    sp.token_local.assign(Nv, -1);
    sp.n_local.assign(world, 0);
    for (int i = 0; i < Nv; i++)
    {
        const int o = static_cast<int>(((long long)i * world) / Nv);
        const int g = sp.plan[0].video_indices[i];
        sp.token_owner[g] = o;
        sp.token_local[g] = sp.n_local[o]++;
    }
    sp.local_tokens.resize(sp.n_local[rank]);
    for (int g = 0; g < Nv; g++)
        if (sp.token_owner[g] == rank) sp.local_tokens[sp.token_local[g]] = g;

    const int n = sp.n_local[rank];
    for (int p = 0; p < 2; p++)
    {
        const Plan& pl = sp.plan[p];
        const int nw = static_cast<int>(pl.windows.size() / 9);
        // Window owners: the rank holding most of the window's tokens, then
        // windows move from the most to the least loaded rank (preferring
        // windows that rank already holds tokens of) while a move lowers the
        // larger of the two loads.  A window's load is the attention kernel's
        // work for it: per head, ceil(S/256) units (pairs of 128-row query
        // tiles), each walking ceil(S/128) key tiles plus about one key
        // tile's worth of unit set-up and epilogue.  (S^2 undercounts the
        // small boundary windows of the shifted plan, whose every head still
        // costs a whole unit: with it the slowest rank's shifted attention ran
        // 3-7 % longer at 2, 4 and 8 GPUs on the 720p and 1080p plans.)
        sp.owner[p].assign(nw, 0);
        std::vector<std::vector<int>> w_votes(nw, std::vector<int>(world, 0));
        std::vector<double> load(world, 0.0);
        auto cost = [&](int w) {
            const int S = pl.windows[9 * w + 8] + text_length;
            return static_cast<double>(((S + 255) / 256) * ((S + 127) / 128 + 1));
        };
        double total = 0.0;
        for (int w = 0; w < nw; w++)
        {
            const int part = pl.windows[9 * w + 7], cnt = pl.windows[9 * w + 8];
            for (int i = 0; i < cnt; i++) w_votes[w][sp.token_owner[pl.video_indices[part + i]]]++;
            sp.owner[p][w] = static_cast<int>(std::max_element(w_votes[w].begin(), w_votes[w].end()) -
                                              w_votes[w].begin());
            load[sp.owner[p][w]] += cost(w);
            total += cost(w);
        }
        const double mean = total / world;
        for (int iter = 0; iter < 4 * nw; iter++)
        {
            const int hi = static_cast<int>(std::max_element(load.begin(), load.end()) - load.begin());
            const int lo = static_cast<int>(std::min_element(load.begin(), load.end()) - load.begin());
            if (load[hi] <= mean) break;
            int pick = -1;
            double pick_key = -1.0;
            for (int w = 0; w < nw; w++)
            {
                if (sp.owner[p][w] != hi || load[lo] + cost(w) >= load[hi]) continue;
                const double key = (double)w_votes[w][lo] / pl.windows[9 * w + 8] + 1e-9 * cost(w);
                if (key > pick_key)
                {
                    pick = w;
                    pick_key = key;
                }
            }
            if (pick < 0) break;
            sp.owner[p][pick] = lo;
            load[hi] -= cost(pick);
            load[lo] += cost(pick);
        }
        // Exchange lists: both sides walk the destination's windows in plan
        // order and their tokens in partition order.
        sp.send_rows[p].assign(world, {});
        sp.send_tokens[p].assign(world, {});
        sp.recv_tokens[p].assign(world, {});
        for (int w = 0; w < nw; w++)
        {
            const int q = sp.owner[p][w], part = pl.windows[9 * w + 7], cnt = pl.windows[9 * w + 8];
            if (q == rank) sp.win_mine[p].push_back(w);
            for (int i = 0; i < cnt; i++)
            {
                const int g = pl.video_indices[part + i];
                const int s = sp.token_owner[g];
                if (s == q) continue;
                if (s == rank)
                {
                    sp.send_rows[p][q].push_back(sp.token_local[g]);
                    sp.send_tokens[p][q].push_back(g);
                }
                if (q == rank) sp.recv_tokens[p][s].push_back(g);
            }
        }
        sp.recv_off[p].assign(world, 0);
        sp.send_off[p].assign(world, 0);
        int acc = 0, sacc = 0;
        for (int s = 0; s < world; s++)
        {
            sp.recv_off[p][s] = acc;
            acc += static_cast<int>(sp.recv_tokens[p][s].size());
            sp.send_off[p][s] = sacc;
            sacc += static_cast<int>(sp.send_rows[p][s].size());
        }
        sp.m_foreign[p] = acc;
        sp.m_send[p] = sacc;
        // Every rank's receive offsets (for direct stores into its buffer).
        sp.recv_off_all[p].assign((size_t)world * world, 0);
        sp.m_foreign_all[p].assign(world, 0);
        {
            std::vector<int> cnt((size_t)world * world, 0);
            for (int w = 0; w < nw; w++)
            {
                const int q = sp.owner[p][w], part = pl.windows[9 * w + 7], c = pl.windows[9 * w + 8];
                for (int i = 0; i < c; i++)
                {
                    const int s_ = sp.token_owner[pl.video_indices[part + i]];
                    if (s_ != q) cnt[(size_t)q * world + s_]++;
                }
            }
            for (int q = 0; q < world; q++)
            {
                int a2 = 0;
                for (int s_ = 0; s_ < world; s_++)
                {
                    sp.recv_off_all[p][(size_t)q * world + s_] = a2;
                    a2 += cnt[(size_t)q * world + s_];
                }
                sp.m_foreign_all[p][q] = a2;
            }
        }
        // Rows of this rank's buffers: [own video | text | foreign video].
        sp.row[p].assign(Nv, -1);
        for (int i = 0; i < n; i++) sp.row[p][sp.local_tokens[i]] = i;
        for (int s = 0; s < world; s++)
            for (size_t k = 0; k < sp.recv_tokens[p][s].size(); k++)
                sp.row[p][sp.recv_tokens[p][s][k]] = n + text_length + sp.recv_off[p][s] + static_cast<int>(k);
    }
    return S2_OK;
}

// ---------------------------------------------------------------- NCCL
namespace {

struct NcclApi
{
    void* handle = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    bool ok = false;
};

NcclApi& api()
{
    static NcclApi a;
    static bool tried = false;
    if (tried) return a;
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
    a.handle = h;
#define S2_SYM(name, field) a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name))
    S2_SYM("ncclGetUniqueId", GetUniqueId);
    S2_SYM("ncclCommInitRankConfig", CommInitRankConfig);
    S2_SYM("ncclCommDestroy", CommDestroy);
    S2_SYM("ncclCommAbort", CommAbort);
    S2_SYM("ncclCommGetAsyncError", CommGetAsyncError);
    S2_SYM("ncclGroupStart", GroupStart);
    S2_SYM("ncclGroupEnd", GroupEnd);
    S2_SYM("ncclSend", Send);
    S2_SYM("ncclRecv", Recv);
    S2_SYM("ncclAllReduce", AllReduce);
    S2_SYM("ncclAllGather", AllGather);
#undef S2_SYM
    a.ok = a.GetUniqueId && a.CommInitRankConfig && a.CommDestroy && a.CommAbort && a.CommGetAsyncError &&
           a.GroupStart && a.GroupEnd && a.Send && a.Recv && a.AllReduce && a.AllGather;
    return a;
}

} // namespace

bool nccl_available()
{
    return api().ok;
}

int nccl_unique_id(void* out128)
{
    NcclApi& a = api();
    if (!a.ok) return S2_ERR_DEVICE;
    ncclUniqueId id;
    if (a.GetUniqueId(&id) != ncclSuccess) return S2_ERR_CUDA;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    std::memcpy(out128, &id, 128);
    return S2_OK;
}

// Bounded wait for a non-blocking communicator to leave ncclInProgress.
int Dist::wait_ready(Context* ctx)
{
    NcclApi& a = api();
    const auto t0 = std::chrono::steady_clock::now();
    while (true)
    {
        ncclResult_t st = ncclSuccess;
        if (a.CommGetAsyncError(comm, &st) != ncclSuccess) return fail(S2_ERR_CUDA);
        if (st == ncclSuccess)
        {
            if (ctx && ctx->prof.on)
            {
                ctx->prof.launches[K_HOST_WAIT] += 1;
                ctx->prof.ms[K_HOST_WAIT] +=
                    std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
            }
            return S2_OK;
        }
        if (st != ncclInProgress) return fail(S2_ERR_CUDA);
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) return fail(S2_ERR_TIMEOUT);
        std::this_thread::yield();
    }
}

int Dist::fail(int code)
{
    if (comm && !aborted)
    {
        api().CommAbort(comm);
        aborted = true;
        comm = nullptr;
    }
    return code;
}

int Dist::init(const void* id128, int r, int w, int tmo)
{
    NcclApi& a = api();
    if (!a.ok) return S2_ERR_DEVICE;
    rank = r;
    world = w;
    timeout_ms = tmo > 0 ? tmo : 60000;
    ncclUniqueId id;
    std::memcpy(&id, id128, 128);
    // Creation is non-blocking so a peer that never joins is a bounded wait;
    // data-path calls then enqueue without host polling (see exchange_bf16).
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t res = a.CommInitRankConfig(&comm, world, id, rank, &cfg);
    if (res != ncclSuccess && res != ncclInProgress)
    {
        comm = nullptr;
        return S2_ERR_CUDA;
    }
    return wait_ready();
}

void Dist::destroy()
{
    for (void* p : opened) cudaIpcCloseMemHandle(p);
    opened.clear();
    if (comm && !aborted) api().CommDestroy(comm);
    comm = nullptr;
}

int Dist::share_buffer(Context& ctx, void* local, std::vector<void*>& peers)
{
    if (!comm) return S2_ERR_INVALID;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "cudaIpcMemHandle_t size");
    cudaIpcMemHandle_t mine;
    if (cudaIpcGetMemHandle(&mine, local) != cudaSuccess) return S2_ERR_CUDA;
    void* dev = nullptr;
    if (cudaMalloc(&dev, (size_t)64 * (world + 1)) != cudaSuccess) return S2_ERR_ALLOC;
    std::vector<uint8_t> all((size_t)64 * world);
    int r = S2_OK;
    if (cudaMemcpyAsync(dev, &mine, 64, cudaMemcpyHostToDevice, ctx.stream) != cudaSuccess) r = S2_ERR_CUDA;
    if (r == S2_OK)
    {
        const ncclResult_t res =
            api().AllGather(dev, static_cast<uint8_t*>(dev) + 64, 64, ncclUint8, comm, ctx.stream);
        if (res != ncclSuccess && res != ncclInProgress) r = fail(S2_ERR_CUDA);
        if (r == S2_OK) r = wait_ready(&ctx);
    }
    if (r == S2_OK) r = sync(ctx.stream);
    if (r == S2_OK &&
        cudaMemcpy(all.data(), static_cast<uint8_t*>(dev) + 64, all.size(), cudaMemcpyDeviceToHost) != cudaSuccess)
        r = S2_ERR_CUDA;
    cudaFree(dev);
    if (r != S2_OK) return r;
    peers.assign(world, nullptr);
    for (int q = 0; q < world; q++)
    {
        if (q == rank)
        {
            peers[q] = local;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, all.data() + (size_t)64 * q, 64);
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return S2_ERR_CUDA;
        opened.push_back(p);
        peers[q] = p;
    }
    return S2_OK;
}

int Dist::all_reduce_sum_f32(Context& ctx, float* buf, size_t count)
{
    if (!comm) return S2_ERR_INVALID;
    NcclApi& a = api();
    ncclResult_t res;
    {
        ProfileScope prof(ctx, K_COMM, 0.0, (double)count * 4.0 * 2.0);
        res = a.AllReduce(buf, buf, count, ncclFloat32, ncclSum, comm, ctx.stream);
    }
    if (res != ncclSuccess && res != ncclInProgress) return fail(S2_ERR_CUDA);
    return wait_ready(&ctx);
}

// Grouped point-to-point exchange of bf16 rows of `row_elems` elements:
// send_counts[p] rows from send + send_off[p] rows, recv_counts[p] rows into
// recv + recv_off[p] rows.
int Dist::exchange_bf16(Context& ctx, const void* send, const std::vector<int>& send_counts,
                        const std::vector<int>& send_off, void* recv, const std::vector<int>& recv_counts,
                        const std::vector<int>& recv_off, size_t row_elems)
{
    if (!comm) return S2_ERR_INVALID;
    NcclApi& a = api();
    cudaStream_t stream = ctx.stream;
    const size_t rb = row_elems * 2;
    double bytes = 0.0;
    for (int p = 0; p < world; p++) bytes += (double)(send_counts[p] + recv_counts[p]) * rb;
    ProfileScope prof(ctx, K_COMM, 0.0, bytes);
    if (a.GroupStart() != ncclSuccess) return fail(S2_ERR_CUDA);
    for (int p = 0; p < world; p++)
    {
        if (p == rank) continue;
        if (send_counts[p] > 0)
            a.Send(static_cast<const uint8_t*>(send) + (size_t)send_off[p] * rb, (size_t)send_counts[p] * rb,
                   ncclUint8, p, comm, stream);
        if (recv_counts[p] > 0)
            a.Recv(static_cast<uint8_t*>(recv) + (size_t)recv_off[p] * rb, (size_t)recv_counts[p] * rb, ncclUint8, p,
                   comm, stream);
    }
    const ncclResult_t res = a.GroupEnd();
    if (res != ncclSuccess && res != ncclInProgress) return fail(S2_ERR_CUDA);
    return wait_ready(&ctx);
}

// Waits (bounded) for the stream; on expiry the communicator is aborted so
// the ranks' NCCL kernels return and the caller sees S2_ERR_TIMEOUT.
int Dist::sync(cudaStream_t stream)
{
    const auto t0 = std::chrono::steady_clock::now();
    while (true)
    {
        const cudaError_t e = cudaStreamQuery(stream);
        if (e == cudaSuccess) return S2_OK;
        if (e != cudaErrorNotReady) return S2_ERR_CUDA;
        if (comm)
        {
            ncclResult_t st = ncclSuccess;
            api().CommGetAsyncError(comm, &st);
            if (st != ncclSuccess && st != ncclInProgress) return fail(S2_ERR_CUDA);
        }
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) return fail(S2_ERR_TIMEOUT);
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

} // namespace s2
