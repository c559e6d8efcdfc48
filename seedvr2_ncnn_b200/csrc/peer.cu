// Cross-GPU data movement of the sharded forward over NVLink peer memory
// (one process per GPU; every rank maps the other ranks' exchange buffers
// through CUDA IPC):
//   * push_rows:   own qkv rows of tokens in another rank's windows are
//                  stored straight into that rank's qkv buffer;
//   * barrier:     each rank stores an epoch into a flag slot of every peer
//                  and waits (bounded) until every peer's epoch has arrived
//                  in its own flags -- this replaces NCCL in the block loop;
//   * text_reduce: the text-pool partial sums of all ranks are read over
//                  NVLink and added in rank order (identical on every rank).
// Writers end with a system-scope fence so their stores are visible to the
// peer once the writer has passed its next barrier.  No TMA and no
// multicast: plain 16-byte loads and stores.
#include "s2_common.cuh"
#include "s2_dist.h"
#include "s2_internal.h"

namespace s2 {

namespace {

struct PeerPtrs
{
    void* p[kMaxPeers];
};

// table entries: {own row, destination rank, destination row, 0}
__global__ void push_rows_kernel(const uint4* __restrict__ src, int row_vecs, const int4* __restrict__ table,
                                 int count, PeerPtrs dst)
{
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row < count)
    {
        const int4 e = __ldg(table + row);
        const uint4* s = src + (int64_t)e.x * row_vecs;
        uint4* d = reinterpret_cast<uint4*>(dst.p[e.y]) + (int64_t)e.z * row_vecs;
        for (int c = lane; c < row_vecs; c += 32) d[c] = __ldg(s + c);
    }
    __threadfence_system();
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One warp: lane i < world signals peer i and waits for peer i.
__global__ void barrier_kernel(PeerPtrs peer_flags, uint32_t* my_flags, int rank, int world, uint32_t epoch,
                               int* status)
{
    const int i = threadIdx.x;
    if (i < world)
    {
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t*>(peer_flags.p[i]) + rank, epoch);
        const uint64_t t0 = global_timer_ns();
        while (ld_acquire_sys(my_flags + i) < epoch)
        {
            if (global_timer_ns() - t0 > kWaitLimitNs)
            {
                record_status(status, kStatusTimeout);
                break;
            }
        }
    }
    __syncwarp();
}

// out[t][c] (bf16) = sum over ranks r = 0..world-1 of part_r[t][c] (fp32).
__global__ void text_reduce_kernel(PeerPtrs parts, int world, int count4, __nv_bfloat16* out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count4) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; r++)
    {
        const float4 v = reinterpret_cast<const float4*>(parts.p[r])[i];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    uint2 u;
    u.x = pack_bf16x2(acc.x, acc.y);
    u.y = pack_bf16x2(acc.z, acc.w);
    reinterpret_cast<uint2*>(out)[i] = u;
}

PeerPtrs peers(void* const* p, int n)
{
    PeerPtrs pp;
    for (int i = 0; i < kMaxPeers; i++) pp.p[i] = i < n ? p[i] : nullptr;
    return pp;
}

} // namespace

int launch_push_rows(Context& ctx, const void* src, int row_elems, const int4* table, int count, void* const* dst,
                     int world)
{
    if (count <= 0) return S2_OK;
    if (row_elems % 8 || world > kMaxPeers) return S2_ERR_INVALID;
    const int warps = 8;
    ProfileScope prof(ctx, K_COMM, 0.0, (double)count * row_elems * 2.0 * 2.0);
    push_rows_kernel<<<(count + warps - 1) / warps, warps * 32, 0, ctx.stream>>>(
        static_cast<const uint4*>(src), row_elems / 8, table, count, peers(dst, world));
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

int launch_peer_barrier(Context& ctx, void* const* peer_flags, uint32_t* my_flags, int rank, int world, uint32_t epoch)
{
    if (world > kMaxPeers) return S2_ERR_INVALID;
    ProfileScope prof(ctx, K_COMM, 0.0, 0.0);
    barrier_kernel<<<1, 32, 0, ctx.stream>>>(peers(peer_flags, world), my_flags, rank, world, epoch, ctx.status);
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

int launch_text_reduce_peers(Context& ctx, void* const* parts, int world, int64_t count, void* out_bf16)
{
    if (count % 4 || world > kMaxPeers) return S2_ERR_INVALID;
    const int count4 = static_cast<int>(count / 4);
    ProfileScope prof(ctx, K_COMM, 0.0, (double)count * 4.0 * world + (double)count * 2.0);
    text_reduce_kernel<<<(count4 + 255) / 256, 256, 0, ctx.stream>>>(peers(parts, world), world, count4,
                                                                      static_cast<__nv_bfloat16*>(out_bf16));
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

} // namespace s2
