// SharedLinear on sm_100a: out_s = A_s W^T + bias (+ epilogue) for two token
// streams s in one persistent launch.
//
// Replaces the two ncnn Gemm calls of SharedLinear::forward
// (shared_linear.cpp:83-96 CPU, :128-143 Vulkan).  Design:
//   * 128x256 output tile per CTA, K staged 64 at a time (one 128-byte
//     swizzle row) by TMA into a 4-stage shared-memory ring;
//   * one thread issues tcgen05.mma (M=128, N=256, K=16, bf16 -> fp32) into
//     one of two TMEM accumulators (2 x 256 columns), so the epilogue of tile
//     i overlaps the MMAs of tile i+1;
//   * four epilogue warps drain TMEM with tcgen05.ld (one accumulator row per
//     thread), apply bias and the fused epilogue (store, GELU-tanh, or
//     gate * acc + fp32 residual), stage each 32-row x 128-byte box in
//     128-byte-swizzled shared memory (two boxes per warp in flight) and
//     write it with one TMA store, so global writes are whole lines;
//   * every mbarrier wait is bounded (s2_common.cuh) and unwinds the CTA.
#include "s2_common.cuh"
#include "s2_internal.h"

namespace s2 {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int A_BYTES = BM * BK * 2;
// warp 0 TMA, warp 1 MMA, then the epilogue warps: 4 (one per TMEM lane
// quarter), or 8 for the QKV packing epilogue (two per quarter, one head of
// the tile each), whose per-row work needs two warps per SMSP to hide latency
__host__ __device__ constexpr int epilogue_warps(int EK)
{
    return EK == 2 ? 8 : 4;
}
__host__ __device__ constexpr int num_threads(int EK)
{
    return 64 + 32 * epilogue_warps(EK);
}

// Tile width BN (256, or 128 when a problem has too few 256-wide tiles to
// fill the SMs evenly).  224 KB of shared memory is split between SKB KB of
// operand stages and the epilogue's 4 KB boxes (R per epilogue warp):
//   * SKB = 192: R = 2 (store double buffering; a gate-residual epilogue
//     loads its residual box one box ahead);
//   * SKB = 144, gate-residual only: R = 5 or 6, so each warp keeps R-1
//     residual boxes in flight from HBM -- for short K, where the epilogue
//     of a tile has little mainloop time to hide behind.
// Epilogue kinds EK: 0 store / GELU (runtime), 1 gate-residual (fp32 in
// place, TMA), 2 QKV packing (norm + RoPE, rows scattered to packed windows).
template <int BN, int SKB, int EK>
struct Tile
{
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (SKB * 1024) / STAGE_BYTES;
    static constexpr int R = (224 * 1024 - STAGES * STAGE_BYTES) / (4 * 4096);
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN, 0, 0);
    static constexpr int EPI_BYTES = 4 * R * 4096; // 4 warps x R boxes of 32 rows x 128 bytes
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 512;
    static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// QKV packing epilogue (EK 2): see launch_qkv_packed.
struct PackArgs
{
    int D;      // heads * 128 (columns of each of q, k, v)
    int pairs;  // RoPE pairs per axis
    float eps;
    const int* dst0; // [dst0_rows] packed row of each stream-0 (video) row, -1: none;
                     // row | (peer + 1) << kPeerShift: the row lives on a peer GPU
    int dst0_rows;
    const int* pos0; // [dst0_rows][3] RoPE positions of stream-0 rows (null: row_pos of the packed row)
    const int* tdst_off; // [M1 + 1] CSR offsets of each stream-1 (text) row's packed rows
    const int* tdst;
    const int* row_pos;  // [packed rows][3] RoPE positions
    const float* norms;  // [4][128]: q video, k video, q text, k text
    const float2* rope;  // [positions][pairs] (cos, sin)
    int rope_entries;    // positions * pairs; staged in shared memory when it fits
    __nv_bfloat16* out[3]; // packed q, k, v [packed rows][D]
    __nv_bfloat16* peer_out[3][kMaxPeers]; // the same buffers on peer GPUs (NVLink peer memory)
};

struct GemmArgs
{
    int M0, M1, N, K;
    int mblk0, mblk1, nblk, num_tiles, num_kb;
    int group_m; // M blocks per raster group (tiles walk M fastest inside a group)
    int ksplit;  // K halves per tile (2: split-K units, gate-residual CTA pairs only; else 1)
    // split-K ordering: one flag per 32-row x 256-column output box (rows of
    // stream 1 start at box row split_row32_1); the first half's unit writes
    // split_epoch into it once its adds have completed
    unsigned* split_flags;
    unsigned split_epoch;
    int split_row32_1;
    // narrow tail (CTA pairs, no split): units from full_units on are the two
    // 128-column halves of the last tiles
    int narrow;
    int full_units;
    int epilogue;
    int out_f32;
    int tma_out; // outputs written through tmap_o0 / tmap_o1
    const float* bias;
    const float* gate;
    void* out0;
    void* out1;
    int* status;
    PackArgs pack;
};

// Tile t -> (stream, first row, first column); M blocks of BMT rows
// (128, or 256 for a CTA pair), raster of group_m M blocks.
template <int BN, int BMT = BM>
__device__ __forceinline__ void decode_tile(const GemmArgs& a, int t, int& stream, int& m0, int& n0)
{
    const int mb_total = a.mblk0 + a.mblk1;
    const int per_group = a.group_m * a.nblk;
    const int g = t / per_group;
    const int first_m = g * a.group_m;
    const int gm = min(a.group_m, mb_total - first_m);
    const int r = t - g * per_group;
    const int mb = first_m + r % gm;
    const int nb = r / gm;
    stream = mb < a.mblk0 ? 0 : 1;
    m0 = (stream ? mb - a.mblk0 : mb) * BMT;
    n0 = nb * BN;
}

// Work unit t -> its tile and K part: with split-K every tile's first half
// comes before any second half (t = khalf * tiles + tile), so a second half
// -- which adds only after its first half's adds have landed -- normally
// runs a round after it and finds its flag set; khalf = -1 without a split.
__device__ __forceinline__ int unit_tile(const GemmArgs& a, int t, int& khalf)
{
    if (a.ksplit > 1)
    {
        const int tiles = a.num_tiles / a.ksplit;
        khalf = t / tiles;
        return t - khalf * tiles;
    }
    khalf = -1;
    return t;
}

// The unit's K blocks [kb0, kb1).
__device__ __forceinline__ void unit_kblocks(const GemmArgs& a, int khalf, int& kb0, int& kb1)
{
    if (khalf < 0)
    {
        kb0 = 0;
        kb1 = a.num_kb;
        return;
    }
    const int per = (a.num_kb + a.ksplit - 1) / a.ksplit;
    kb0 = khalf * per;
    kb1 = min(a.num_kb, kb0 + per);
}

// Split-K ordering flag of the output box whose first row is `row` (a
// multiple of 32) in `stream`, columns [256 nb, 256 nb + 256).
__device__ __forceinline__ unsigned* split_flag(const GemmArgs& a, int stream, int row, int nb)
{
    return a.split_flags + (size_t)((stream ? a.split_row32_1 : 0) + row / 32) * a.nblk + nb;
}

// The wait is bounded: a grid that is not resident all at once (other work
// on the GPU holding SMs) may leave the first half unstarted, and past the
// limit the add goes ahead unordered -- the sum is complete either way, only
// its rounding order is then open.  Within one stream's kernels both halves
// run a round apart (or, with fewer tiles than CTA pairs, side by side) and
// the wait is at most the first half's epilogue.
constexpr uint64_t kSplitWaitNs = 1000000ull;

__device__ __forceinline__ void split_wait_first_half(const unsigned* flag, unsigned epoch)
{
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_gpu(flag) != epoch)
    {
        if (global_timer_ns() - t0 > kSplitWaitNs) break;
        __nanosleep(64);
    }
    fence_proxy_async_global();
}

// First half done: its reduces have completed (all of this thread's bulk
// groups), then the flag is released to the second half.
__device__ __forceinline__ void split_signal_first_half(unsigned* flag, unsigned epoch)
{
    bulk_wait<0>();
    fence_proxy_async_global();
    st_release_gpu(flag, epoch);
}

// Pair-mode unit t -> its tile's stream, first row (of the 256-row pair
// tile) and first column; returns the unit's width.  Split-K units cover
// their tile's full width.  With a narrow tail, a last wave of at most half
// the CTA pairs' worth of tiles runs as one round of 256 x 128 units (both
// halves of each of those tiles) instead of one round of full tiles.
__device__ __forceinline__ int pair_unit(const GemmArgs& a, int t, int& stream, int& m0, int& n0)
{
    int khalf;
    int tile = unit_tile(a, t, khalf);
    int half = -1;
    if (a.narrow && t >= a.full_units)
    {
        const int u = t - a.full_units;
        tile = a.full_units + (u >> 1);
        half = u & 1;
    }
    decode_tile<256, 2 * BM>(a, tile, stream, m0, n0);
    if (half < 0) return 256;
    n0 += half * 128;
    return 128;
}

// Tile walk of one CTA: a single CTA per tile, or a CTA pair (cluster of 2)
// per 256-row tile, each CTA owning 128 of its rows.
struct SingleWalk
{
    __device__ int first() const { return blockIdx.x; }
    __device__ int step() const { return gridDim.x; }
    // unit t -> (stream, first row, first column); returns the unit's width
    template <int BN>
    __device__ int decode(const GemmArgs& a, int t, int& stream, int& m0, int& n0) const
    {
        decode_tile<BN>(a, t, stream, m0, n0);
        return BN;
    }
    __device__ void arrive_tempty(uint64_t* bar) const { mbar_arrive(bar); }
};

struct PairWalk
{
    uint32_t rank; // 0 = leader (issues the MMAs)
    __device__ int first() const { return blockIdx.x >> 1; }
    __device__ int step() const { return gridDim.x >> 1; }
    // unit t -> this CTA's rows (stream, first row, first column); returns
    // the unit's width
    template <int BN>
    __device__ int decode(const GemmArgs& a, int t, int& stream, int& m0, int& n0) const
    {
        const int w = pair_unit(a, t, stream, m0, n0);
        m0 += (int)rank * BM;
        return w;
    }
    // accumulator release goes to the leader's barrier
    __device__ void arrive_tempty(uint64_t* bar) const { mbar_arrive_cluster(mapa_shared(bar, 0)); }
};

// Wait for all in-flight work tracked by `bar` (phase `parity`) with a time
// limit only; used on the unwind path so no async copy or MMA outlives the CTA.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity)
{
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_timer_ns() - t0 > kWaitLimitNs) break;
}

__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, int stream, int row, int n, const uint32_t (&v)[32])
{
    const int M = stream ? a.M1 : a.M0;
    if (row >= M) return;
    const int N = a.N;
    float x[32];
#pragma unroll
    for (int j = 0; j < 32; j++) x[j] = __uint_as_float(v[j]);
    const bool full = n + 32 <= N;
    if (a.bias)
    {
        if (full)
        {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
            {
                const float4 b = __ldg(reinterpret_cast<const float4*>(a.bias + n + j));
                x[j] += b.x;
                x[j + 1] += b.y;
                x[j + 2] += b.z;
                x[j + 3] += b.w;
            }
        }
        else
        {
            for (int j = 0; j < 32; j++)
                if (n + j < N) x[j] += __ldg(a.bias + n + j);
        }
    }
    void* outp = stream ? a.out1 : a.out0;
    const size_t base = (size_t)row * N + n;
    if (a.epilogue == EPI_GATE_RESIDUAL)
    {
        float* o = reinterpret_cast<float*>(outp) + base;
        if (full)
        {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
            {
                const float4 g = __ldg(reinterpret_cast<const float4*>(a.gate + n + j));
                float4 r = *reinterpret_cast<float4*>(o + j);
                r.x += x[j] * g.x;
                r.y += x[j + 1] * g.y;
                r.z += x[j + 2] * g.z;
                r.w += x[j + 3] * g.w;
                *reinterpret_cast<float4*>(o + j) = r;
            }
        }
        else
        {
            for (int j = 0; j < 32; j++)
                if (n + j < N) o[j] += x[j] * __ldg(a.gate + n + j);
        }
        return;
    }
    if (a.epilogue == EPI_GELU_TANH)
    {
#pragma unroll
        for (int j = 0; j < 32; j++) x[j] = gelu_tanh(x[j]);
    }
    if (a.out_f32)
    {
        float* o = reinterpret_cast<float*>(outp) + base;
        if (full)
        {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(o + j) = make_float4(x[j], x[j + 1], x[j + 2], x[j + 3]);
        }
        else
        {
            for (int j = 0; j < 32; j++)
                if (n + j < N) o[j] = x[j];
        }
    }
    else
    {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(outp) + base;
        if (full)
        {
#pragma unroll
            for (int j = 0; j < 32; j += 8)
            {
                uint4 p;
                p.x = pack_bf16x2(x[j], x[j + 1]);
                p.y = pack_bf16x2(x[j + 2], x[j + 3]);
                p.z = pack_bf16x2(x[j + 4], x[j + 5]);
                p.w = pack_bf16x2(x[j + 6], x[j + 7]);
                *reinterpret_cast<uint4*>(o + j) = p;
            }
        }
        else
        {
            for (int j = 0; j < 32; j++)
                if (n + j < N) o[j] = __float2bfloat16_rn(x[j]);
        }
    }
}

// Epilogue of one tile for one warp (accumulator rows quarter*32 .. +31)
// through shared-memory staging and TMA stores: each 128-byte-wide box
// (32 fp32 or 64 bf16 columns x 32 rows) is written by the lanes in the
// 128-byte swizzle (16-byte unit u of row r at unit u ^ (r & 7), which is
// free of bank conflicts) and stored by lane 0.  `stg` holds the warp's two
// 4 KB boxes; `slot` alternates between them.
// khalf >= 0: a split-K unit of a gate-residual tile -- (acc [+ bias on the
// first half]) * gate is reduce-added into the fp32 output in L2, no residual
// is read.  The second half's first add waits for the first half's flag, so
// every element is (r + first) + second on every run.
template <int BN>
__device__ __forceinline__ void epilogue_tile_tma(const GemmArgs& a, const CUtensorMap* tmap_out, uint8_t* stg, int& slot,
                                                  uint32_t t_row, int stream, int m0, int n0, int quarter, int lane,
                                                  int khalf = -1, int width = BN)
{
    const bool split = khalf >= 0;
    const int M = stream ? a.M1 : a.M0;
    const int N = a.N;
    const int row = m0 + quarter * 32 + lane;
    const bool live = row < M;
    const bool box_live = m0 + quarter * 32 < M;
    const int box_cols = a.out_f32 ? 32 : 64;
    const float* res_row = reinterpret_cast<const float*>(stream ? a.out1 : a.out0) + (size_t)row * N;
    const int sw = lane & 7;
#pragma unroll 1
    for (int c0 = 0; c0 < width && n0 + c0 < N; c0 += box_cols)
    {
        if (lane == 0) bulk_wait_read<1>(); // this slot's previous store has read it
        __syncwarp();
        uint8_t* srow = stg + slot * 4096 + lane * 128;
#pragma unroll 1
        for (int k = 0; k < box_cols / 32; k++)
        {
            const int n = n0 + c0 + 32 * k;
            const bool full = n + 32 <= N;
            float4 r[8];
            if (a.epilogue == EPI_GATE_RESIDUAL && !split)
            {
                if (live && full)
                {
#pragma unroll
                    for (int j = 0; j < 8; j++) r[j] = *reinterpret_cast<const float4*>(res_row + n + 4 * j);
                }
                else
                {
#pragma unroll
                    for (int j = 0; j < 8; j++)
                    {
                        float e[4];
#pragma unroll
                        for (int q = 0; q < 4; q++) e[q] = (live && n + 4 * j + q < N) ? res_row[n + 4 * j + q] : 0.f;
                        r[j] = make_float4(e[0], e[1], e[2], e[3]);
                    }
                }
            }
            uint32_t v[32];
            tmem_ld32(t_row + c0 + 32 * k, v);
            tmem_ld_wait();
            float x[32];
#pragma unroll
            for (int j = 0; j < 32; j++) x[j] = __uint_as_float(v[j]);
            if (a.bias && khalf <= 0)
            {
                if (full)
                {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                    {
                        const float4 b = __ldg(reinterpret_cast<const float4*>(a.bias + n + j));
                        x[j] += b.x;
                        x[j + 1] += b.y;
                        x[j + 2] += b.z;
                        x[j + 3] += b.w;
                    }
                }
                else
                {
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (n + j < N) x[j] += __ldg(a.bias + n + j);
                }
            }
            if (a.epilogue == EPI_GATE_RESIDUAL)
            {
#pragma unroll
                for (int j = 0; j < 8; j++)
                {
                    float4 g;
                    if (full)
                        g = __ldg(reinterpret_cast<const float4*>(a.gate + n + 4 * j));
                    else
                    {
                        g.x = n + 4 * j < N ? __ldg(a.gate + n + 4 * j) : 0.f;
                        g.y = n + 4 * j + 1 < N ? __ldg(a.gate + n + 4 * j + 1) : 0.f;
                        g.z = n + 4 * j + 2 < N ? __ldg(a.gate + n + 4 * j + 2) : 0.f;
                        g.w = n + 4 * j + 3 < N ? __ldg(a.gate + n + 4 * j + 3) : 0.f;
                    }
                    if (split)
                    {
                        x[4 * j] *= g.x;
                        x[4 * j + 1] *= g.y;
                        x[4 * j + 2] *= g.z;
                        x[4 * j + 3] *= g.w;
                    }
                    else
                    {
                        x[4 * j] = r[j].x + x[4 * j] * g.x;
                        x[4 * j + 1] = r[j].y + x[4 * j + 1] * g.y;
                        x[4 * j + 2] = r[j].z + x[4 * j + 2] * g.z;
                        x[4 * j + 3] = r[j].w + x[4 * j + 3] * g.w;
                    }
                }
            }
            else if (a.epilogue == EPI_GELU_TANH)
            {
#pragma unroll
                for (int j = 0; j < 32; j++) x[j] = gelu_tanh(x[j]);
            }
            if (a.out_f32)
            {
#pragma unroll
                for (int j = 0; j < 8; j++)
                    *reinterpret_cast<float4*>(srow + ((j ^ sw) << 4)) =
                        make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
            }
            else
            {
#pragma unroll
                for (int j = 0; j < 4; j++)
                {
                    uint4 p;
                    p.x = pack_bf16x2(x[8 * j], x[8 * j + 1]);
                    p.y = pack_bf16x2(x[8 * j + 2], x[8 * j + 3]);
                    p.z = pack_bf16x2(x[8 * j + 4], x[8 * j + 5]);
                    p.w = pack_bf16x2(x[8 * j + 6], x[8 * j + 7]);
                    *reinterpret_cast<uint4*>(srow + (((4 * k + j) ^ sw) << 4)) = p;
                }
            }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0)
        {
            if (box_live)
            {
                if (split && khalf == 1 && c0 == 0)
                    split_wait_first_half(split_flag(a, stream, m0 + quarter * 32, n0 / BN), a.split_epoch);
                if (split)
                    tma_reduce_add_2d(tmap_out, stg + slot * 4096, n0 + c0, m0 + quarter * 32);
                else
                    tma_store_2d(tmap_out, stg + slot * 4096, n0 + c0, m0 + quarter * 32);
            }
            bulk_commit();
        }
        slot ^= 1;
    }
}

__device__ __forceinline__ float bf16_round(float x)
{
    return __bfloat162float(__float2bfloat16_rn(x));
}

// QKV packing epilogue of one tile for one warp (one accumulator row per
// thread).  The tile's 128-column heads lie in one of q, k, v (D is a
// multiple of BN).  Per head: x = bf16(acc + bias); for q and k,
// x * rsqrt(mean(x^2) + eps) * w then 3D RoPE on adjacent pairs (axis a
// covers head dims [2*pairs*a, 2*pairs*(a+1)), rotation (cos, sin) of
// pos[a] * freqs[pair] from the precomputed table);
// the bf16 row segment is stored to every packed row of the token (one for
// a video row, one per window of the sample for a text row).  The same
// arithmetic as prepare_qkv_kernel, which reads the rounded qkv rows back.
template <int BN>
__device__ __forceinline__ void epilogue_tile_pack(const GemmArgs& a, const float2* rope, uint32_t t_row, int stream,
                                                   int m0, int n0, int quarter, int lane, int half)
{
    const PackArgs& p = a.pack;
    const int M = stream ? a.M1 : a.M0;
    const int row = m0 + quarter * 32 + lane;
    const int part = n0 / p.D;
    const int col0 = n0 - part * p.D;
    __nv_bfloat16* base = p.out[part];
    bool remote = false;
    int first = -1, cnt = 0;
    const int* list = nullptr;
    if (row < M)
    {
        if (stream == 0)
        {
            first = row < p.dst0_rows ? __ldg(p.dst0 + row) : -1;
            cnt = first >= 0 ? 1 : 0;
            const int peer = first >= 0 ? first >> kPeerShift : 0;
            if (peer)
            {
                base = p.peer_out[part][peer - 1];
                first &= (1 << kPeerShift) - 1;
                remote = true;
            }
        }
        else
        {
            const int o = __ldg(p.tdst_off + row);
            cnt = __ldg(p.tdst_off + row + 1) - o;
            list = p.tdst + o;
            first = cnt > 0 ? __ldg(list) : -1;
        }
    }
    const bool qk = part < 2;
    const float* w = p.norms + (stream ? 256 : 0) + part * 128;
    // rows of the rotation table for the three axes (text rows share their
    // positions (i, i, i) across windows)
    const float2* rp0 = rope;
    const float2* rp1 = rope;
    const float2* rp2 = rope;
    if (qk && first >= 0)
    {
        const int* pp = (stream == 0 && p.pos0) ? p.pos0 + 3 * row : p.row_pos + 3 * first;
        rp0 = rope + __ldg(pp) * p.pairs;
        rp1 = rope + __ldg(pp + 1) * p.pairs;
        rp2 = rope + __ldg(pp + 2) * p.pairs;
    }
    const int aw = 2 * p.pairs;
    const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
    // head hh of the tile: the two warps of a lane quarter take one head each
#pragma unroll 1
    for (int hh = half; hh < BN / 128; hh += 2)
    {
        const uint32_t th = t_row + hh * 128;
        const int nb = n0 + hh * 128; // GEMM column of the head's first element
        float inv = 1.f;
        if (qk)
        {
            float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
            for (int c = 0; c < 4; c++)
            {
                // operands first: the TMEM load below orders all memory accesses
                float4 b4[8];
#pragma unroll
                for (int j = 0; j < 8; j++)
                    b4[j] = a.bias ? __ldg(reinterpret_cast<const float4*>(a.bias + nb + c * 32) + j) : zero4;
                uint32_t v[32];
                tmem_ld32(th + c * 32, v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 8; j++)
                {
                    const float x0 = bf16_round(__uint_as_float(v[4 * j]) + b4[j].x);
                    const float x1 = bf16_round(__uint_as_float(v[4 * j + 1]) + b4[j].y);
                    const float x2 = bf16_round(__uint_as_float(v[4 * j + 2]) + b4[j].z);
                    const float x3 = bf16_round(__uint_as_float(v[4 * j + 3]) + b4[j].w);
                    ss[0] += x0 * x0;
                    ss[1] += x1 * x1;
                    ss[2] += x2 * x2;
                    ss[3] += x3 * x3;
                }
            }
            inv = 1.f / sqrtf(((ss[0] + ss[1]) + (ss[2] + ss[3])) / 128.f + p.eps);
        }
#pragma unroll 1
        for (int c = 0; c < 4; c++)
        {
            float4 b4[8], w4[8];
            float2 r2[16];
#pragma unroll
            for (int j = 0; j < 8; j++)
            {
                b4[j] = a.bias ? __ldg(reinterpret_cast<const float4*>(a.bias + nb + c * 32) + j) : zero4;
                w4[j] = qk ? __ldg(reinterpret_cast<const float4*>(w + c * 32) + j) : zero4;
            }
#pragma unroll
            for (int j = 0; j < 16; j++)
            {
                const int d = c * 32 + 2 * j;
                const int axis = d >= 2 * aw ? 2 : (d >= aw ? 1 : 0);
                const float2* rp = axis == 0 ? rp0 : (axis == 1 ? rp1 : rp2);
                // generic load: the table is in shared or global memory
                r2[j] = (qk && d < 3 * aw) ? rp[(d - axis * aw) >> 1] : make_float2(1.f, 0.f);
            }
            uint32_t v[32];
            tmem_ld32(th + c * 32, v);
            tmem_ld_wait();
            float x[32];
#pragma unroll
            for (int j = 0; j < 8; j++)
            {
                x[4 * j] = bf16_round(__uint_as_float(v[4 * j]) + b4[j].x);
                x[4 * j + 1] = bf16_round(__uint_as_float(v[4 * j + 1]) + b4[j].y);
                x[4 * j + 2] = bf16_round(__uint_as_float(v[4 * j + 2]) + b4[j].z);
                x[4 * j + 3] = bf16_round(__uint_as_float(v[4 * j + 3]) + b4[j].w);
            }
            if (qk)
            {
#pragma unroll
                for (int j = 0; j < 8; j++)
                {
                    x[4 * j] = x[4 * j] * inv * w4[j].x;
                    x[4 * j + 1] = x[4 * j + 1] * inv * w4[j].y;
                    x[4 * j + 2] = x[4 * j + 2] * inv * w4[j].z;
                    x[4 * j + 3] = x[4 * j + 3] * inv * w4[j].w;
                }
#pragma unroll
                for (int j = 0; j < 16; j++)
                {
                    // (cos, sin) = (1, 0) past the rotated dims
                    const float cs = r2[j].x, sn = r2[j].y;
                    const float x0 = x[2 * j], x1 = x[2 * j + 1];
                    x[2 * j] = x0 * cs - x1 * sn;
                    x[2 * j + 1] = x0 * sn + x1 * cs;
                }
            }
            uint32_t u0[8], u1[8];
#pragma unroll
            for (int q = 0; q < 8; q++)
            {
                u0[q] = pack_bf16x2(x[2 * q], x[2 * q + 1]);
                u1[q] = pack_bf16x2(x[16 + 2 * q], x[16 + 2 * q + 1]);
            }
            const size_t coff = (size_t)col0 + hh * 128 + c * 32;
            for (int i = 0; i < cnt; i++)
            {
                // two full 32-byte sectors of the packed row
                const int r = stream == 0 ? first : __ldg(list + i);
                __nv_bfloat16* dst = base + (size_t)r * p.D + coff;
                st_v8(dst, u0);
                st_v8(dst + 16, u1);
            }
        }
    }
    // rows stored into a peer GPU must be visible there once this rank
    // passes its next cross-GPU barrier
    if (remote) __threadfence_system();
}

// Gate-residual epilogue of one warp over all of the CTA's tiles, fp32
// residual in place: out = out + (acc + bias) * gate.  Boxes (32 rows x 32
// columns) run in a fixed sequence over the CTA's tiles; lane 0 TMA-loads the
// residual box R-1 boxes ahead into one of the warp's R shared-memory boxes
// (barrier rfull[slot]), the lanes combine it with the accumulator row in
// place, and lane 0 TMA-stores it back.  A box is reloaded only after its
// previous store has read it.  Returns false on a failed wait.
template <int BN, int R, class Walk>
__device__ __forceinline__ bool epilogue_gate_residual(const GemmArgs& a, const Walk& wk, const CUtensorMap* tmap_o0,
                                                       const CUtensorMap* tmap_o1, uint8_t* stg, uint64_t* rfull,
                                                       uint64_t* tfull, uint64_t* tempty, uint32_t tmem_base,
                                                       int quarter, int lane, volatile int* abort_flag)
{
    const int N = a.N;
    const int sw = lane & 7;
    // loader cursor (lane 0): next box to load
    int lt = wk.first(), lc = 0, lq = 0;
    auto issue_load = [&]() {
        int s_, m0_, n0_, w_;
        for (;;)
        {
            if (lt >= a.num_tiles) return;
            w_ = wk.template decode<BN>(a, lt, s_, m0_, n0_);
            if (lc < w_ && n0_ + lc < N) break;
            // a unit with no columns inside N (the second half of a narrow
            // tile past N) has no boxes, as in the consumer loop below
            lc = 0;
            lt += wk.step();
        }
        const int slot = lq % R;
        mbar_arrive_expect_tx(&rfull[slot], 4096);
        tma_load_2d(stg + slot * 4096, s_ ? tmap_o1 : tmap_o0, &rfull[slot], n0_ + lc, m0_ + quarter * 32);
        lq++;
        lc += 32;
        if (lc >= w_ || n0_ + lc >= N)
        {
            lc = 0;
            lt += wk.step();
        }
    };
    if (lane == 0)
        for (int i = 0; i < R - 1; i++) issue_load();
    int q = 0; // boxes consumed
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int t = wk.first(); t < a.num_tiles && ok; t += wk.step())
    {
        int w = 0;
        if (lane == 0) w = mbar_wait<true>(&tfull[acc], acc_phase, abort_flag, a.status) ? 1 : 0;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w)
        {
            ok = false;
            break;
        }
        __syncwarp();
        tc_fence_after();
        int stream, m0, n0;
        const int width = wk.template decode<BN>(a, t, stream, m0, n0);
        const int M = stream ? a.M1 : a.M0;
        const bool box_live = m0 + quarter * 32 < M;
        const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
        for (int c0 = 0; c0 < width && n0 + c0 < N; c0 += 32, q++)
        {
            const int slot = q % R;
            int r = 0;
            if (lane == 0) r = mbar_wait<true>(&rfull[slot], (uint32_t)(q / R) & 1u, abort_flag, a.status) ? 1 : 0;
            r = __shfl_sync(0xffffffffu, r, 0);
            if (!r)
            {
                ok = false;
                break;
            }
            uint8_t* srow = stg + slot * 4096 + lane * 128;
            const int n = n0 + c0;
            const bool full = n + 32 <= N;
            uint32_t v[32];
            tmem_ld32(t_row + c0, v);
            float4 res[8];
#pragma unroll
            for (int j = 0; j < 8; j++) res[j] = *reinterpret_cast<const float4*>(srow + ((j ^ sw) << 4));
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 8; j++)
            {
                float4 g, b = make_float4(0.f, 0.f, 0.f, 0.f);
                if (full)
                {
                    g = __ldg(reinterpret_cast<const float4*>(a.gate + n + 4 * j));
                    if (a.bias) b = __ldg(reinterpret_cast<const float4*>(a.bias + n + 4 * j));
                }
                else
                {
                    float ge[4], be[4];
#pragma unroll
                    for (int e = 0; e < 4; e++)
                    {
                        const bool in = n + 4 * j + e < N;
                        ge[e] = in ? __ldg(a.gate + n + 4 * j + e) : 0.f;
                        be[e] = (in && a.bias) ? __ldg(a.bias + n + 4 * j + e) : 0.f;
                    }
                    g = make_float4(ge[0], ge[1], ge[2], ge[3]);
                    b = make_float4(be[0], be[1], be[2], be[3]);
                }
                float4 o;
                o.x = res[j].x + (__uint_as_float(v[4 * j]) + b.x) * g.x;
                o.y = res[j].y + (__uint_as_float(v[4 * j + 1]) + b.y) * g.y;
                o.z = res[j].z + (__uint_as_float(v[4 * j + 2]) + b.z) * g.z;
                o.w = res[j].w + (__uint_as_float(v[4 * j + 3]) + b.w) * g.w;
                *reinterpret_cast<float4*>(srow + ((j ^ sw) << 4)) = o;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0)
            {
                if (box_live) tma_store_2d(stream ? tmap_o1 : tmap_o0, stg + slot * 4096, n, m0 + quarter * 32);
                bulk_commit();
                bulk_wait_read<1>(); // the store of box q-1 has read box (q-1) % R
                issue_load();        // box q+R-1 into it
            }
        }
        if (!ok) break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) wk.arrive_tempty(&tempty[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
    }
    if (lane == 0)
    {
        // no TMA load may land after the CTA exits
        for (int i = q; i < lq; i++) drain_wait(&rfull[i % R], (uint32_t)(i / R) & 1u);
        bulk_wait<0>();
    }
    __syncwarp();
    return ok;
}

template <int BN, int SKB, int EK>
__global__ void __launch_bounds__(num_threads(EK), 1)
    shared_linear_kernel(const __grid_constant__ CUtensorMap tmap_a0, const __grid_constant__ CUtensorMap tmap_a1,
                         const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_o0,
                         const __grid_constant__ CUtensorMap tmap_o1, const GemmArgs args)
{
    using TL = Tile<BN, SKB, EK>;
    constexpr bool GR = EK == 1;
    constexpr int STAGES = TL::STAGES;
    constexpr int STAGE_BYTES = TL::STAGE_BYTES;
    constexpr int TMEM_COLS = TL::TMEM_COLS;
    constexpr uint32_t IDESC = TL::IDESC;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* epi_stage = smem + STAGES * STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + TL::EPI_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint64_t* rfull = drain + 1; // [4 warps][R] residual boxes (GR)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rfull + 4 * TL::R);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0)
    {
        for (int s = 0; s < STAGES; s++)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++)
        {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], epilogue_warps(EK));
        }
        mbar_init(drain, 1);
        if (GR)
            for (int i = 0; i < 4 * TL::R; i++) mbar_init(&rfull[i], 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&tmap_a0);
        tma_prefetch_desc(&tmap_a1);
        tma_prefetch_desc(&tmap_w);
        if (args.tma_out)
        {
            tma_prefetch_desc(&tmap_o0);
            tma_prefetch_desc(&tmap_o1);
        }
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0)
    {
        if (lane == 0)
        {
            // ---------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            int issued[STAGES];
            uint32_t last_phase[STAGES];
            for (int s = 0; s < STAGES; s++) issued[s] = 0, last_phase[s] = 0;
            for (int t = blockIdx.x; t < args.num_tiles && !*abort_flag; t += gridDim.x)
            {
                int stream, m0, n0;
                decode_tile<BN>(args, t, stream, m0, n0);
                const CUtensorMap* ta = stream ? &tmap_a1 : &tmap_a0;
                for (int kb = 0; kb < args.num_kb; kb++)
                {
                    if (!mbar_wait<true>(&empty[stage], phase ^ 1, abort_flag, args.status)) break;
                    uint8_t* sa = smem + stage * STAGE_BYTES;
                    uint8_t* sb = sa + A_BYTES;
                    mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                    tma_load_2d(sa, ta, &full[stage], kb * BK, m0);
                    tma_load_2d(sb, &tmap_w, &full[stage], kb * BK, n0);
                    issued[stage] = 1;
                    last_phase[stage] = phase;
                    if (++stage == STAGES)
                    {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag)
            {
                // No TMA write may land after the CTA exits.
                for (int s = 0; s < STAGES; s++)
                    if (issued[s]) drain_wait(&full[s], last_phase[s]);
            }
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            // ---------------- MMA issuer
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool any = false;
            for (int t = blockIdx.x; t < args.num_tiles && !*abort_flag; t += gridDim.x)
            {
                if (!mbar_wait<true>(&tempty[acc], acc_phase ^ 1, abort_flag, args.status)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                bool ok = true;
                for (int kb = 0; kb < args.num_kb; kb++)
                {
                    if (!mbar_wait<true>(&full[stage], phase, abort_flag, args.status))
                    {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
                    const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                    {
                        const uint64_t ad = umma_desc_sw128(a_addr + k * 32, 16, 1024);
                        const uint64_t bd = umma_desc_sw128(b_addr + k * 32, 16, 1024);
                        umma_bf16(d_tmem, ad, bd, IDESC, (kb | k) != 0);
                    }
                    umma_commit(&empty[stage]);
                    any = true;
                    if (++stage == STAGES)
                    {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            if (any)
            {
                // Every MMA issued by this thread completes before TMEM is freed.
                umma_commit(drain);
                drain_wait(drain, 0);
            }
        }
    }
    else
    {
        // ---------------- epilogue (warps 2..5)
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2; // second warp of the lane quarter (8 epilogue warps)
        // QKV packing: the RoPE table goes into the (otherwise unused) epilogue
        // staging memory when it fits
        const float2* rope = args.pack.rope;
        if constexpr (EK == 2)
        {
            if (args.pack.rope_entries > 0 && args.pack.rope_entries * 8 <= TL::EPI_BYTES)
            {
                float2* tab = reinterpret_cast<float2*>(epi_stage);
                for (int i = threadIdx.x - 64; i < args.pack.rope_entries; i += 32 * epilogue_warps(EK))
                    tab[i] = __ldg(args.pack.rope + i);
                named_barrier_sync(1, 32 * epilogue_warps(EK));
                rope = tab;
            }
        }
        const int row_in_tile = quarter * 32 + lane;
        uint8_t* stg = epi_stage + quarter * (TL::R * 4096);
        if constexpr (GR)
        {
            epilogue_gate_residual<BN, TL::R>(args, SingleWalk{}, &tmap_o0, &tmap_o1, stg, rfull + quarter * TL::R, tfull, tempty,
                                              tmem_base, quarter, lane, abort_flag);
        }
        else
        {
            int slot = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int t = blockIdx.x; t < args.num_tiles; t += gridDim.x)
            {
                int ok = 0;
                if (lane == 0) ok = mbar_wait<true>(&tfull[acc], acc_phase, abort_flag, args.status) ? 1 : 0;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                __syncwarp();
                tc_fence_after();
                int stream, m0, n0;
                decode_tile<BN>(args, t, stream, m0, n0);
                const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
                if constexpr (EK == 2)
                {
                    epilogue_tile_pack<BN>(args, rope, t_row, stream, m0, n0, quarter, lane, half);
                }
                else if (args.tma_out)
                {
                    epilogue_tile_tma<BN>(args, stream ? &tmap_o1 : &tmap_o0, stg, slot, t_row, stream, m0, n0,
                                          quarter, lane);
                }
                else
                {
#pragma unroll 1
                    for (int c = 0; c < BN / 32; c++)
                    {
                        uint32_t v[32];
                        tmem_ld32(t_row + c * 32, v);
                        tmem_ld_wait();
                        if (n0 + c * 32 < args.N) epilogue_chunk(args, stream, m0 + row_in_tile, n0 + c * 32, v);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            // every TMA store of this warp has completed before the CTA exits
            if (lane == 0) bulk_wait<0>();
            __syncwarp();
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ---------------------------------------------------------------- CTA pairs
// 256 x 256 output tile per cluster of two CTAs (tcgen05 .cta_group::2): each
// CTA loads its 128 rows of A and its 128 rows of W (half of N) per K step --
// 32 KB instead of the 48 KB a lone 128 x 256 tile needs -- and receives a
// 128 x 256 fp32 accumulator in its own TMEM.  The leader (rank 0) issues the
// M = 256 MMAs; its `full` barriers count both CTAs' TMA bytes, commits
// arrive in both CTAs, and both CTAs' epilogue warps release an accumulator
// on the leader's `tempty`.  Loads carry no multicast.
template <int SKB, int EK>
struct PairTile
{
    static constexpr int A_STAGE = BM * BK * 2;  // 128 rows of A
    static constexpr int B_STAGE = 128 * BK * 2; // 128 rows of W
    static constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
    static constexpr int STAGES = (SKB * 1024) / STAGE_BYTES;
    static constexpr int R = (224 * 1024 - STAGES * STAGE_BYTES) / (4 * 4096);
    static constexpr int TMEM_COLS = 512; // two 256-column accumulators
    static constexpr uint32_t IDESC = umma_idesc_bf16(256, 256, 0, 0);
    static constexpr uint32_t IDESC_NARROW = umma_idesc_bf16(256, 128, 0, 0); // narrow-tail units
    static constexpr int EPI_BYTES = 4 * R * 4096;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 512;
    static_assert(SMEM_BYTES <= 232448, "shared memory");
};

template <int SKB, int EK>
__global__ void __launch_bounds__(num_threads(EK), 1)
    shared_linear_pair_kernel(const __grid_constant__ CUtensorMap tmap_a0, const __grid_constant__ CUtensorMap tmap_a1,
                              const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_w64,
                              const __grid_constant__ CUtensorMap tmap_o0, const __grid_constant__ CUtensorMap tmap_o1,
                              const GemmArgs args)
{
    constexpr int BN = 256;
    using TL = PairTile<SKB, EK>;
    constexpr bool GR = EK == 1;
    constexpr int STAGES = TL::STAGES;
    constexpr int STAGE_BYTES = TL::STAGE_BYTES;
    constexpr int EW = epilogue_warps(EK);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* epi_stage = smem + STAGES * STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + TL::EPI_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint64_t* rfull = drain + 1; // [4 warps][R] residual boxes (GR)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rfull + 4 * TL::R);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const PairWalk walk{cluster_ctarank()};
    const bool leader = walk.rank == 0;

    if (threadIdx.x == 0)
    {
        for (int s = 0; s < STAGES; s++)
        {
            mbar_init(&full[s], 1);  // leader: its producer's expect_tx for both CTAs' bytes
            mbar_init(&empty[s], 1); // the leader's commit, in both CTAs
        }
        for (int b = 0; b < 2; b++)
        {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * EW); // leader: epilogue warps of both CTAs
        }
        mbar_init(drain, 1);
        if (GR)
            for (int i = 0; i < 4 * TL::R; i++) mbar_init(&rfull[i], 1);
        *abort_flag = 0;
        *tmem_slot = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&tmap_a0);
        tma_prefetch_desc(&tmap_a1);
        tma_prefetch_desc(&tmap_w);
        if (args.narrow) tma_prefetch_desc(&tmap_w64);
        if (args.tma_out)
        {
            tma_prefetch_desc(&tmap_o0);
            tma_prefetch_desc(&tmap_o1);
        }
    }
    __syncthreads();
    if (warp == 1) tmem_alloc_pair(tmem_slot, TL::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    cluster_sync(); // both CTAs' barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0)
    {
        if (lane == 0)
        {
            // ---------------- TMA producer (both CTAs; completion on the leader's barriers)
            int stage = 0;
            uint32_t phase = 0;
            int issued[STAGES];
            uint32_t last_phase[STAGES];
            for (int s = 0; s < STAGES; s++) issued[s] = 0, last_phase[s] = 0;
            for (int t = walk.first(); t < args.num_tiles && !*abort_flag; t += walk.step())
            {
                int khalf, kb0, kb1;
                unit_tile(args, t, khalf);
                unit_kblocks(args, khalf, kb0, kb1);
                int stream, m0, n0p;
                const int width = walk.decode<BN>(args, t, stream, m0, n0p);
                // each CTA loads its half of the unit's W rows (a 64-row box for narrow units)
                const int nb = n0p + (int)walk.rank * (width / 2);
                const CUtensorMap* ta = stream ? &tmap_a1 : &tmap_a0;
                const CUtensorMap* tw = width == BN ? &tmap_w : &tmap_w64;
                const uint32_t stage_tx = width == BN ? 2 * STAGE_BYTES : 2 * (TL::A_STAGE + TL::B_STAGE / 2);
                for (int kb = kb0; kb < kb1; kb++)
                {
                    if (!mbar_wait<true>(&empty[stage], phase ^ 1, abort_flag, args.status)) break;
                    uint8_t* sa = smem + stage * STAGE_BYTES;
                    uint8_t* sb = sa + TL::A_STAGE;
                    if (leader) mbar_arrive_expect_tx(&full[stage], stage_tx);
                    const uint32_t fb = mapa_shared(&full[stage], 0);
                    tma_load_2d_pair(sa, ta, fb, kb * BK, m0);
                    tma_load_2d_pair(sb, tw, fb, kb * BK, nb);
                    issued[stage] = 1;
                    last_phase[stage] = phase;
                    if (++stage == STAGES)
                    {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag && leader)
            {
                // No TMA write may land after the CTAs exit (the peer's loads
                // complete on these barriers too).
                for (int s = 0; s < STAGES; s++)
                    if (issued[s]) drain_wait(&full[s], last_phase[s]);
            }
        }
    }
    else if (warp == 1)
    {
        if (lane == 0 && leader)
        {
            // ---------------- MMA issuer (leader only)
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int t = walk.first(); t < args.num_tiles && !*abort_flag; t += walk.step())
            {
                if (!mbar_wait<true>(&tempty[acc], acc_phase ^ 1, abort_flag, args.status)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                int khalf, kb0, kb1;
                unit_tile(args, t, khalf);
                unit_kblocks(args, khalf, kb0, kb1);
                int us, um, un;
                const uint32_t idesc = walk.decode<BN>(args, t, us, um, un) == BN ? TL::IDESC : TL::IDESC_NARROW;
                bool ok = true;
                for (int kb = kb0; kb < kb1; kb++)
                {
                    if (!mbar_wait<true>(&full[stage], phase, abort_flag, args.status))
                    {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
                    const uint32_t b_addr = a_addr + TL::A_STAGE;
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                    {
                        const uint64_t ad = umma_desc_sw128(a_addr + k * 32, 16, 1024);
                        const uint64_t bd = umma_desc_sw128(b_addr + k * 32, 16, 1024);
                        umma_bf16_pair(d_tmem, ad, bd, idesc, (kb != kb0) || k != 0);
                    }
                    umma_commit_pair(&empty[stage], 0x3);
                    if (++stage == STAGES)
                    {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit_pair(&tfull[acc], 0x3);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            // every MMA completes (in both CTAs) before TMEM is released
            umma_commit_pair(drain, 0x3);
        }
        if (lane == 0) drain_wait(drain, 0);
    }
    else
    {
        // ---------------- epilogue (warps 2..): this CTA's 128 rows of the tile
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row_in_tile = quarter * 32 + lane;
        uint8_t* stg = epi_stage + quarter * (TL::R * 4096);
        const float2* rope = args.pack.rope;
        if constexpr (EK == 2)
        {
            if (args.pack.rope_entries > 0 && args.pack.rope_entries * 8 <= TL::EPI_BYTES)
            {
                float2* tab = reinterpret_cast<float2*>(epi_stage);
                for (int i = threadIdx.x - 64; i < args.pack.rope_entries; i += 32 * EW) tab[i] = __ldg(args.pack.rope + i);
                named_barrier_sync(1, 32 * EW);
                rope = tab;
            }
        }
        bool done = false;
        if constexpr (GR)
        {
            // split-K units take the reduce-add path of the generic loop below
            if (args.ksplit <= 1)
            {
                epilogue_gate_residual<BN, TL::R>(args, walk, &tmap_o0, &tmap_o1, stg, rfull + quarter * TL::R,
                                                  tfull, tempty, tmem_base, quarter, lane, abort_flag);
                done = true;
            }
        }
        if (!done)
        {
            int slot = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int t = walk.first(); t < args.num_tiles; t += walk.step())
            {
                int ok = 0;
                if (lane == 0) ok = mbar_wait<true>(&tfull[acc], acc_phase, abort_flag, args.status) ? 1 : 0;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                __syncwarp();
                tc_fence_after();
                int khalf;
                unit_tile(args, t, khalf);
                int stream, m0, n0;
                const int width = walk.decode<BN>(args, t, stream, m0, n0);
                const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
                if constexpr (EK == 2)
                {
                    epilogue_tile_pack<BN>(args, rope, t_row, stream, m0, n0, quarter, lane, half);
                }
                else if (args.tma_out)
                {
                    epilogue_tile_tma<BN>(args, stream ? &tmap_o1 : &tmap_o0, stg, slot, t_row, stream, m0, n0,
                                          quarter, lane, khalf, width);
                }
                else
                {
#pragma unroll 1
                    for (int c = 0; c < width / 32; c++)
                    {
                        uint32_t v[32];
                        tmem_ld32(t_row + c * 32, v);
                        tmem_ld_wait();
                        if (n0 + c * 32 < args.N) epilogue_chunk(args, stream, m0 + row_in_tile, n0 + c * 32, v);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) walk.arrive_tempty(&tempty[acc]);
                if constexpr (GR)
                {
                    if (khalf == 0 && lane == 0)
                        split_signal_first_half(split_flag(args, stream, m0 + quarter * 32, n0 / BN),
                                                args.split_epoch);
                }
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            if (lane == 0) bulk_wait<0>();
            __syncwarp();
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync(); // no remote arrival or MMA operand read outlives either CTA
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, TL::TMEM_COLS);
}

// Persistent grid of CTA pairs: one pair per tile up to the number of pairs
// that can be resident at once (cudaOccupancyMaxActiveClusters).
template <int SKB, int EK>
cudaError_t launch_pair_variant(cudaStream_t stream, const CUtensorMap& ta0, const CUtensorMap& ta1,
                                const CUtensorMap& tw, const CUtensorMap& tw64, const CUtensorMap& to0,
                                const CUtensorMap& to1, const GemmArgs& a)
{
    static std::atomic<uint64_t> configured{0}; // per instantiation and device
    static std::atomic<int> max_clusters{0};     // the same on every B200
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(num_threads(EK));
    cfg.dynamicSmemBytes = PairTile<SKB, EK>::SMEM_BYTES;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (first_on_device(configured))
    {
        const cudaError_t e = cudaFuncSetAttribute(shared_linear_pair_kernel<SKB, EK>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   PairTile<SKB, EK>::SMEM_BYTES);
        if (e != cudaSuccess) return e;
    }
    if (max_clusters.load() == 0)
    {
        cfg.gridDim = dim3(2);
        int n = 0;
        const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, shared_linear_pair_kernel<SKB, EK>, &cfg);
        if (e != cudaSuccess) return e;
        if (n <= 0) return cudaErrorInvalidConfiguration;
        max_clusters.store(n);
    }
    const int mc = max_clusters.load();
    const int pairs = a.num_tiles < mc ? a.num_tiles : mc;
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(num_threads(EK));
    cfg.dynamicSmemBytes = PairTile<SKB, EK>::SMEM_BYTES;
    return cudaLaunchKernelEx(&cfg, shared_linear_pair_kernel<SKB, EK>, ta0, ta1, tw, tw64, to0, to1, a);
}

// CTA pairs resident at once (every pair kernel holds one CTA per SM, so
// one configuration answers for all), queried once per process; half the
// SMs if the query fails.
int pair_slots(const Context& ctx)
{
    static std::atomic<int> slots{0};
    int n = slots.load();
    if (n > 0) return n;
    using TL = PairTile<192, 1>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(num_threads(1));
    cfg.dynamicSmemBytes = TL::SMEM_BYTES;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    n = 0;
    if (cudaFuncSetAttribute(shared_linear_pair_kernel<192, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TL::SMEM_BYTES) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, shared_linear_pair_kernel<192, 1>, &cfg) != cudaSuccess || n <= 0)
    {
        (void)cudaGetLastError();
        n = ctx.num_sms / 2;
    }
    slots.store(n);
    return n;
}

template <int BN, int SKB, int EK>
cudaError_t launch_variant(int grid, cudaStream_t stream, const CUtensorMap& ta0, const CUtensorMap& ta1,
                           const CUtensorMap& tw, const CUtensorMap& to0, const CUtensorMap& to1, const GemmArgs& a)
{
    static std::atomic<uint64_t> configured{0}; // per instantiation and device
    if (first_on_device(configured))
    {
        const cudaError_t e =
            cudaFuncSetAttribute(shared_linear_kernel<BN, SKB, EK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Tile<BN, SKB, EK>::SMEM_BYTES);
        if (e != cudaSuccess) return e;
    }
    shared_linear_kernel<BN, SKB, EK>
        <<<grid, num_threads(EK), Tile<BN, SKB, EK>::SMEM_BYTES, stream>>>(ta0, ta1, tw, to0, to1, a);
    return cudaGetLastError();
}

} // namespace

namespace {

enum TileMode
{
    TILE_256 = 0,  // one CTA per 128 x 256 tile
    TILE_128 = 1,  // one CTA per 128 x 128 tile
    TILE_PAIR = 2, // one CTA pair per 256 x 256 tile
};

// Operand tensor maps, tile count and tile shape shared by the launchers.
// The pair tile needs fewer operand bytes per MMA; a narrower tile is taken
// only when it fills the SMs markedly more evenly.
int gemm_setup(Context& ctx, int M0, int M1, int N, int K, const void* A0, const void* A1, const void* W,
               CUtensorMap& ta0, CUtensorMap& ta1, CUtensorMap& tw, CUtensorMap& tw64, GemmArgs& a, int& mode,
               bool allow_split, bool allow_narrow)
{
    int r = make_tmap_bf16_2d(&ta0, A0, K, M0 > 0 ? M0 : 1, (uint64_t)K * 2, BK, BM);
    if (r == 0) r = make_tmap_bf16_2d(&ta1, M1 > 0 ? A1 : A0, K, M1 > 0 ? M1 : (M0 > 0 ? M0 : 1), (uint64_t)K * 2, BK, BM);
    if (r != 0) return r;
    a = GemmArgs{};
    a.M0 = M0;
    a.M1 = M1;
    a.N = N;
    a.K = K;
    a.mblk0 = (M0 + BM - 1) / BM;
    a.mblk1 = (M1 + BM - 1) / BM;
    a.num_kb = (K + BK - 1) / BK;
    a.status = ctx.status;
    a.ksplit = 1;
    auto wave_eff = [&](int tiles, int slots) {
        const int waves = (tiles + slots - 1) / slots;
        return (double)tiles / ((double)waves * slots);
    };
    const int t256 = (a.mblk0 + a.mblk1) * ((N + 255) / 256);
    const int t128 = (a.mblk0 + a.mblk1) * ((N + 127) / 128);
    const int pm0 = (M0 + 2 * BM - 1) / (2 * BM), pm1 = (M1 + 2 * BM - 1) / (2 * BM);
    const int tpair = (pm0 + pm1) * ((N + 255) / 256);
    const int pairs = pair_slots(ctx);
    const double e256 = wave_eff(t256, ctx.num_sms), e128 = wave_eff(t128, ctx.num_sms);
    const double esingle = e128 > 1.15 * e256 ? e128 : e256;
    // Split-K by two (gate-residual epilogues, reduce-add into the fp32
    // output) when whole pair tiles leave a part-empty last wave that half-K
    // units fill: one GPU's 2,765 rows x N 2560 make 110 pair tiles for 74
    // pairs (1.49 waves), 220 half-K units make 2.97 -- instead of falling
    // back to 128 x 128 single-CTA tiles, which read shared memory at the full
    // 128 B per clock and re-read A for every 128 columns (MLP down at that
    // size: 110 vs 149 us).  Only long K: half units of K = 2560 are too short
    // for their epilogue (attention out: 62 vs 49 us).  Large M keeps whole
    // tiles.  The halves' adds are ordered through one flag per 32 x 256
    // output box, so results do not depend on the run.
    int ks = 1;
    double epair = wave_eff(tpair, pairs);
    const int split_boxes = (pm0 + pm1) * (2 * BM / 32) * ((N + 255) / 256);
    if (allow_split && ctx.split_flags && split_boxes <= ctx.split_slots && a.num_kb >= 64 &&
        wave_eff(2 * tpair, pairs) > 1.15 * epair)
    {
        ks = 2;
        epair = wave_eff(2 * tpair, pairs);
    }
    // Narrow tail: a last wave of r <= pairs / 2 tiles runs as 2r units of
    // 256 x 128 in one round of about 0.65 of a full one (half the MMAs; the
    // operand traffic per MMA is higher).  Attention-out at 2,765 rows: 110
    // tiles for 74 pairs, 1.49 rounds of whole tiles -> 1 + 0.65.
    constexpr double kNarrowRound = 0.65;
    const int tail = tpair % pairs;
    const bool narrow = allow_narrow && ks == 1 && tpair >= pairs && tail > 0 && 2 * tail <= pairs;
    if (narrow) epair = (double)tpair / (((double)(tpair / pairs) + kNarrowRound) * pairs);
    if (ks * tpair >= pairs && 1.1 * epair >= esingle)
    {
        mode = TILE_PAIR;
        a.mblk0 = pm0;
        a.mblk1 = pm1;
        a.nblk = (N + 255) / 256;
        a.ksplit = ks;
        if (ks > 1)
        {
            // a fresh epoch per split launch; flags left by earlier launches
            // (or by one that stopped early) hold other values
            if (++ctx.split_epoch == 0)
            {
                if (cudaMemsetAsync(ctx.split_flags, 0, (size_t)ctx.split_slots * sizeof(unsigned), ctx.stream) !=
                    cudaSuccess)
                    return S2_ERR_CUDA;
                ctx.split_epoch = 1;
            }
            a.split_flags = ctx.split_flags;
            a.split_epoch = ctx.split_epoch;
            a.split_row32_1 = pm0 * (2 * BM / 32);
        }
    }
    else
    {
        mode = e128 > 1.15 * e256 ? TILE_128 : TILE_256;
        a.nblk = (N + (mode == TILE_128 ? 127 : 255)) / (mode == TILE_128 ? 128 : 256);
    }
    a.num_tiles = (a.mblk0 + a.mblk1) * a.nblk * a.ksplit;
    if (mode == TILE_PAIR && narrow)
    {
        a.narrow = 1;
        a.full_units = tpair - tail;
        a.num_tiles = tpair + tail;
    }
    // Raster group height: long-K operands (MLP down) walk N first (height
    // 1: each A block is read once while the weight stays in L2), narrow-N
    // short-K ones (attention out) a medium group; measured on the 720p
    // shapes (differences of 2-4 %).
    a.group_m = K >= 8192 ? 1 : (N <= 4096 ? 8 : 16);
    r = make_tmap_bf16_2d(&tw, W, K, N, (uint64_t)K * 2, BK, mode == TILE_256 ? 256 : 128);
    if (r != 0) return r;
    // narrow units load 64 of W's rows per CTA
    if (a.narrow) return make_tmap_bf16_2d(&tw64, W, K, N, (uint64_t)K * 2, BK, 64);
    tw64 = tw;
    return 0;
}

int grid_of(const Context& ctx, const GemmArgs& a)
{
    return a.num_tiles < ctx.num_sms ? a.num_tiles : ctx.num_sms;
}

} // namespace

int launch_shared_linear(Context& ctx, int M0, int M1, int N, int K, const void* A0, const void* A1, const void* W,
                         const float* bias, int epilogue, const float* gate, int out_f32, void* out0, void* out1)
{
    if (M0 < 0 || M1 < 0 || M0 + M1 <= 0 || N <= 0 || K <= 0 || (K % 8) != 0 || (N % 4) != 0 || !A0 || !W ||
        !out0 || (M1 > 0 && (!A1 || !out1)))
        return S2_ERR_INVALID;
    if (epilogue == EPI_GATE_RESIDUAL && (!gate || !out_f32)) return S2_ERR_INVALID;
    if (epilogue == EPI_GELU_TANH && out_f32) return S2_ERR_INVALID;
    if (epilogue < 0 || epilogue > EPI_GATE_RESIDUAL) return S2_ERR_INVALID;

    // TMA-store epilogue when both outputs admit a tensor map (16-byte aligned
    // bases and row strides); the per-thread store path otherwise.
    CUtensorMap to0, to1;
    const uint32_t esz = out_f32 ? 4 : 2;
    const uint32_t box_cols = 128 / esz;
    int tma_out = (((uint64_t)N * esz) % 16 == 0) ? 1 : 0;
    if (tma_out)
        tma_out = make_tmap_2d(&to0, out0, out_f32, N, M0 > 0 ? M0 : 1, (uint64_t)N * esz, box_cols, 32) == S2_OK;
    if (tma_out)
        tma_out = make_tmap_2d(&to1, M1 > 0 ? out1 : out0, out_f32, N, M1 > 0 ? M1 : (M0 > 0 ? M0 : 1),
                               (uint64_t)N * esz, box_cols, 32) == S2_OK;
    CUtensorMap ta0, ta1, tw, tw64;
    GemmArgs a;
    int mode = TILE_256;
    int r = gemm_setup(ctx, M0, M1, N, K, A0, A1, W, ta0, ta1, tw, tw64, a, mode,
                       tma_out && epilogue == EPI_GATE_RESIDUAL, true);
    if (r != 0) return r;
    if (!tma_out) to1 = to0 = tw;
    a.epilogue = epilogue;
    a.out_f32 = out_f32;
    a.tma_out = tma_out;
    a.bias = bias;
    a.gate = gate;
    a.out0 = out0;
    a.out1 = out1;

    const bool gr = tma_out && epilogue == EPI_GATE_RESIDUAL;
    const int grid = grid_of(ctx, a);
    const double M = (double)M0 + M1;
    const double out_bytes = epilogue == EPI_GATE_RESIDUAL ? 8.0 : (out_f32 ? 4.0 : 2.0);
    ProfileScope prof(ctx, K_GEMM, 2.0 * M * N * K, (M * K + (double)N * K) * 2.0 + M * N * out_bytes);
    const bool deep = gr && K < 4096; // deep residual prefetch for short K
    cudaError_t e;
    if (mode == TILE_PAIR)
        e = deep ? launch_pair_variant<160, 1>(ctx.stream, ta0, ta1, tw, tw64, to0, to1, a)
            : gr ? launch_pair_variant<192, 1>(ctx.stream, ta0, ta1, tw, tw64, to0, to1, a)
                 : launch_pair_variant<192, 0>(ctx.stream, ta0, ta1, tw, tw64, to0, to1, a);
    else if (mode == TILE_128)
        e = deep ? launch_variant<128, 144, 1>(grid, ctx.stream, ta0, ta1, tw, to0, to1, a)
            : gr ? launch_variant<128, 192, 1>(grid, ctx.stream, ta0, ta1, tw, to0, to1, a)
                 : launch_variant<128, 192, 0>(grid, ctx.stream, ta0, ta1, tw, to0, to1, a);
    else
        e = deep ? launch_variant<256, 144, 1>(grid, ctx.stream, ta0, ta1, tw, to0, to1, a)
            : gr ? launch_variant<256, 192, 1>(grid, ctx.stream, ta0, ta1, tw, to0, to1, a)
                 : launch_variant<256, 192, 0>(grid, ctx.stream, ta0, ta1, tw, to0, to1, a);
    if (e != cudaSuccess) return S2_ERR_CUDA;
    ctx.launches++;
    return S2_OK;
}

int launch_qkv_packed(Context& ctx, const AttnSchedule& s, int M0, int M1, int K, const void* A0, const void* A1,
                      const void* W, const float* bias, int heads, int rope_pairs, float eps, const float* norms,
                      const void* rope_table, int rope_positions, void* q_out, void* k_out, void* v_out,
                      const QkvPeers* peers)
{
    const int D = heads * 128;
    if (heads <= 0 || D % 256 != 0 || M0 < 0 || M1 < 0 || M0 + M1 <= 0 || K <= 0 || K % 8 || !A0 || !W ||
        (M1 > 0 && !A1) || M0 > (peers ? peers->dst0_rows : s.pack_dst_rows) || M1 > s.total_text || rope_pairs < 0 ||
        6 * rope_pairs > 128 || (peers && (!peers->dst0 || !peers->pos0 || peers->num_peers < 0 ||
                                            peers->num_peers > kMaxPeers)) ||
        !norms || (rope_pairs > 0 && (!rope_table || rope_positions < s.max_pos)) || !q_out || !k_out || !v_out ||
        (bias && (reinterpret_cast<uintptr_t>(bias) & 15)) || (reinterpret_cast<uintptr_t>(norms) & 15))
        return S2_ERR_INVALID;
    for (const void* o : {q_out, k_out, v_out})
        if (reinterpret_cast<uintptr_t>(o) & 15) return S2_ERR_INVALID;
    if (s.packed_rows == 0) return S2_OK;
    const int N = 3 * D;
    CUtensorMap ta0, ta1, tw, tw64;
    GemmArgs a;
    int mode = TILE_256;
    int r = gemm_setup(ctx, M0, M1, N, K, A0, A1, W, ta0, ta1, tw, tw64, a, mode, false, false);
    if (r != 0) return r;
    a.epilogue = EPI_STORE;
    a.bias = bias;
    a.pack.D = D;
    a.pack.pairs = rope_pairs;
    a.pack.eps = eps;
    a.pack.dst0 = peers ? peers->dst0 : s.pack_dst;
    a.pack.dst0_rows = peers ? peers->dst0_rows : s.pack_dst_rows;
    a.pack.pos0 = peers ? peers->pos0 : nullptr;
    if (peers)
        for (int i = 0; i < peers->num_peers; i++)
        {
            a.pack.peer_out[0][i] = static_cast<__nv_bfloat16*>(peers->q[i]);
            a.pack.peer_out[1][i] = static_cast<__nv_bfloat16*>(peers->k[i]);
            a.pack.peer_out[2][i] = static_cast<__nv_bfloat16*>(peers->v[i]);
        }
    a.pack.tdst_off = s.text_dst_off;
    a.pack.tdst = s.text_dst;
    a.pack.row_pos = s.row_pos;
    a.pack.norms = norms;
    a.pack.rope = static_cast<const float2*>(rope_table);
    a.pack.rope_entries = s.max_pos * rope_pairs;
    a.pack.out[0] = static_cast<__nv_bfloat16*>(q_out);
    a.pack.out[1] = static_cast<__nv_bfloat16*>(k_out);
    a.pack.out[2] = static_cast<__nv_bfloat16*>(v_out);
    const int grid = grid_of(ctx, a);
    const double M = (double)M0 + M1;
    ProfileScope prof(ctx, K_GEMM, 2.0 * M * N * K,
                      (M * K + (double)N * K) * 2.0 + (double)s.packed_rows * N * 2.0);
    const cudaError_t e = mode == TILE_PAIR ? launch_pair_variant<192, 2>(ctx.stream, ta0, ta1, tw, tw, tw, tw, a)
                          : mode == TILE_128 ? launch_variant<128, 192, 2>(grid, ctx.stream, ta0, ta1, tw, tw, tw, a)
                                             : launch_variant<256, 192, 2>(grid, ctx.stream, ta0, ta1, tw, tw, tw, a);
    if (e != cudaSuccess) return S2_ERR_CUDA;
    ctx.launches++;
    return S2_OK;
}

} // namespace s2
