// Varlen window attention on sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the per-window ncnn SDPA call and the scatter shader of
// AdaptiveWindowAttention::forward (adaptive_window_attention.cpp:873-975 CPU,
// :1172-1268 Vulkan, scatter shader :353-409).  Each window's sequence is its
// L video rows followed by the sample's T text rows, packed contiguously
// (window after window) in bf16 [rows][heads*128] by the prepare kernel.
//
// Work unit = (window, pair of 128-row query tiles A and B, head); a
// persistent grid of one CTA per SM walks the units.  K/V tiles are loaded
// once for both query tiles.  Warp roles:
//   warp 0     TMA: Q_A and Q_B per unit, K tiles into a 3-stage ring and V
//              tiles into a 2-stage ring (a K stage is released after its
//              last S MMA, a V stage after its last PV MMA);
//   warp 1     one thread issues every tcgen05.mma, ping-ponging the tiles:
//                S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) | ...
//              so the tensor core works on one tile while the other tile's
//              softmax runs;
//   warps 2-5  softmax of tile A, warps 6-9 softmax of tile B: one query row
//              per thread (TMEM lane).  S is read from TMEM, P = exp2(S*c - m)
//              is written back over S as packed bf16 and fed to the PV MMA as
//              its TMEM A operand; O accumulates in TMEM across key tiles.
//              The running max is only raised (and O, l rescaled in place)
//              when it grows by more than 2^8, so most tiles skip the
//              rescale.  S_X(j) is committed after PV_X(j-1), so O is stable
//              whenever the softmax may rescale it.
// Epilogue: O / l -- video rows stored straight to their source token (the
// scatter), text rows to a per-window fp32 partial that text_pool averages
// over the sample's windows.  Keys past the window's sequence are masked;
// query rows past it are computed but never stored.
#include "s2_common.cuh"
#include "s2_internal.h"

namespace s2 {

namespace {

constexpr int HD = 128;                      // head_dim
constexpr int TILE = 128;                    // q rows / keys per tile
constexpr int CHUNK_BYTES = TILE * 128;      // 128 rows x 64 bf16 (one swizzle row each)
constexpr int TILE_BYTES = 2 * CHUNK_BYTES;  // 128 x 128 bf16
constexpr int NUM_THREADS = 320;             // TMA, MMA, 2 x 4 softmax warps
constexpr int TMEM_COLS = 512;               // S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512)
constexpr uint32_t IDESC_O = umma_idesc_bf16(128, 128, 0, 1); // A (= P) K-major, B (= V) MN-major
constexpr int K_STAGES = 2;
// Q_A, Q_B | K ring (2) | V (1) | P_A, P_B  = 7 x 32 KB
constexpr int SMEM_BYTES = (2 + K_STAGES + 1 + 2) * TILE_BYTES + 1024 + 256;
constexpr float RESCALE_THRESHOLD = 8.0f;                     // log2 units

struct AttnArgs
{
    const int4* win_info; // {seq_offset, L, T, partition_offset}
    const int* win_pool;  // partial row of the window's first text row
    const int2* items;    // {window, q0 of tile A}
    const int* video_indices;
    int inner;
    float scale_log2;
    int out_f32;
    int round_bf16;
    void* video_out;
    float* text_partial;
    int* status;
    int heads;
    int num_work; // items x heads
    // peer output bases (multi-GPU): a video_indices entry with a non-zero
    // peer field is stored into peer_out[peer - 1] over NVLink
    void* peer_out[kMaxPeers];
};

__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed fp32 pairs (sm_100 f32x2 FMA / ADD) and a 3-input max.
__device__ __forceinline__ uint64_t pk2(uint32_t lo, uint32_t hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}

__device__ __forceinline__ void upk2(uint64_t v, float& lo, float& hi)
{
    uint32_t a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(a), "=r"(b) : "l"(v));
    lo = __uint_as_float(a);
    hi = __uint_as_float(b);
}

__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ float fmax3(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Row max over NV raw scores (FULL: no masked columns; otherwise columns
// >= valid are ignored); four independent 3-input max chains.
template <bool FULL, int NV>
__device__ __forceinline__ float row_max(const uint32_t (&v)[NV], int valid)
{
    float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int i = 0; i < NV; i += 8)
    {
#pragma unroll
        for (int c = 0; c < 4; c++)
        {
            float a = __uint_as_float(v[i + 2 * c]), b = __uint_as_float(v[i + 2 * c + 1]);
            if (!FULL)
            {
                a = i + 2 * c < valid ? a : -INFINITY;
                b = i + 2 * c + 1 < valid ? b : -INFINITY;
            }
            m[c] = fmax3(m[c], a, b);
        }
    }
    return fmax3(m[0], m[1], fmaxf(m[2], m[3]));
}

// P = exp2(S * c - m) for 64 columns of the row (columns >= valid -> 0) as
// 32 packed bf16 pairs.  The exponent t = S * c - m is formed in fp32
// (packed pairs) and exponentiated in fp32 (ex2.approx.ftz.f32); the row sum
// adds those fp32 values (packed partial sums in sum2) and P is rounded to
// bf16 for the PV MMA.  Against exponentiating bf16 pairs in one MUFU
// operation, this issues fewer instructions per pair (no unpacking for the
// sum) for one more MUFU operation: measured 4.5-6.4 % faster per launch.
template <bool FULL>
__device__ __forceinline__ void row_exp64(const uint32_t (&v)[64], int valid, uint64_t c2, uint64_t negm2,
                                          uint32_t (&p)[32], uint64_t (&sum2)[4])
{
#pragma unroll
    for (int q = 0; q < 32; q++)
    {
        const int i = 2 * q;
        const uint64_t t2 = ffma2(pk2(v[i], v[i + 1]), c2, negm2);
        float t0, t1;
        upk2(t2, t0, t1);
        if (!FULL)
        {
            t0 = i < valid ? t0 : -INFINITY;
            t1 = i + 1 < valid ? t1 : -INFINITY;
        }
        const float e0 = ex2(t0), e1 = ex2(t1);
        p[q] = pack_bf16x2(e0, e1);
        sum2[q & 3] = fadd2(sum2[q & 3], pk2(__float_as_uint(e0), __float_as_uint(e1)));
    }
}

// Half H (64 columns = one 128-byte chunk) of row `row` of a 128 x 128 bf16
// tile in the 128-byte-swizzled K-major layout TMA gives Q and K (chunks of
// 128 rows x 128 bytes; 16-byte unit u of row r at unit u ^ (r & 7)), so the
// PV MMA reads P like Q.
template <int H>
__device__ __forceinline__ void store_p_half(uint8_t* tile, int row, const uint32_t (&p)[32])
{
    uint8_t* r0 = tile + H * CHUNK_BYTES + row * 128;
    const int sw = row & 7;
#pragma unroll
    for (int u = 0; u < 8; u++)
        *reinterpret_cast<uint4*>(r0 + ((u ^ sw) << 4)) = make_uint4(p[4 * u], p[4 * u + 1], p[4 * u + 2], p[4 * u + 3]);
}

__device__ __forceinline__ float bf16_round_f32(float x)
{
    return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status)
{
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort, status) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity)
{
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_timer_ns() - t0 > kWaitLimitNs) break;
}

// Stores 32 output columns [col0, col0+32) of query row qi of the window with
// 32-byte (full-sector) stores: video rows to their source token, text rows
// to the window's fp32 partial.
// Returns true when the row went to a peer GPU.
__device__ __forceinline__ bool store_row(const AttnArgs& a, int item_window, int part_off, int L, int qi, int col0,
                                          const float* o, float inv)
{
    const bool video = qi < L;
    int src = 0;
    void* vbase = a.video_out;
    bool remote = false;
    if (video)
    {
        src = a.video_indices[part_off + qi];
        const int peer = src >> kPeerShift;
        if (peer)
        {
            vbase = a.peer_out[peer - 1];
            src &= (1 << kPeerShift) - 1;
            remote = true;
        }
    }
    if (video && !a.out_f32)
    {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(vbase) + (size_t)src * a.inner + col0;
#pragma unroll
        for (int i = 0; i < 32; i += 16)
        {
            uint32_t r[8];
#pragma unroll
            for (int k = 0; k < 8; k++) r[k] = pack_bf16x2(o[i + 2 * k] * inv, o[i + 2 * k + 1] * inv);
            st_v8(dst + i, r);
        }
        return remote;
    }
    float* dst = video ? reinterpret_cast<float*>(vbase) + (size_t)src * a.inner + col0
                       : a.text_partial + (size_t)(a.win_pool[item_window] + (qi - L)) * a.inner + col0;
#pragma unroll
    for (int i = 0; i < 32; i += 8)
    {
        uint32_t r[8];
#pragma unroll
        for (int k = 0; k < 8; k++)
        {
            float w = o[i + k] * inv;
            if (a.round_bf16) w = bf16_round_f32(w);
            r[k] = __float_as_uint(w);
        }
        st_v8(dst + i, r);
    }
    return remote;
}

// One unit of work: (item, head); consecutive units share the item.
struct Work
{
    int window, seq_off, L, part_off, S_len, q0, has_b, nkv, head;
};

__device__ __forceinline__ Work decode_work(const AttnArgs& a, int w)
{
    Work r;
    const int it = w / a.heads;
    r.head = w - it * a.heads;
    const int2 item = a.items[it];
    const int4 wi = a.win_info[item.x];
    r.window = item.x;
    r.seq_off = wi.x;
    r.L = wi.y;
    r.part_off = wi.w;
    r.S_len = wi.y + wi.z;
    r.q0 = item.y;
    r.has_b = r.q0 + TILE < r.S_len;
    r.nkv = (r.S_len + TILE - 1) / TILE;
    return r;
}

// Persistent: CTA b processes units b, b + gridDim.x, ...  Barrier phases run
// on across units, so the next unit's loads and first S MMAs overlap the
// current unit's last tiles and epilogue; Q is reloaded once the unit's last
// S MMA has read it (q_empty).
//
// P lives in shared memory, not over S in TMEM: as soon as a softmax warp
// group has read S_x(j) into registers (s_free) the MMA thread issues
// S_x(j+1) into the same TMEM columns, so the tensor core computes the next
// scores while the exponentials of this tile run; PV_x(j) (shared-memory A =
// P_x, B = V) follows once P_x(j) is stored (p_full).  A softmax group waits
// for PV_x(j-1) (p_empty) before overwriting P_x or rescaling O_x.
__global__ void __launch_bounds__(NUM_THREADS, 1)
    window_attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                            const __grid_constant__ CUtensorMap tv, const AttnArgs args)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                       // Q_A, Q_B
    uint8_t* sK = sQ + 2 * TILE_BYTES;        // K ring
    uint8_t* sV = sK + K_STAGES * TILE_BYTES; // V
    uint8_t* sP = sV + TILE_BYTES;            // P_A, P_B
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * TILE_BYTES);
    uint64_t* q_full = bars + 0;
    uint64_t* q_empty = bars + 1;
    uint64_t* k_full = bars + 2;  // [K_STAGES]
    uint64_t* k_empty = bars + 4; // [K_STAGES]
    uint64_t* v_full = bars + 6;
    uint64_t* v_empty = bars + 7;
    uint64_t* s_full = bars + 8;   // [2] per query tile: S_x computed
    uint64_t* s_free = bars + 10;  // [2] S_x read by the softmax warps (4 arrivals)
    uint64_t* p_full = bars + 12;  // [2] P_x stored (4 arrivals)
    uint64_t* p_empty = bars + 14; // [2] PV_x done (P_x and O_x free)
    uint64_t* o_done = bars + 16;  // [2] last PV_x of the unit done
    uint64_t* drain = bars + 18;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0)
    {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int s = 0; s < K_STAGES; s++)
        {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        mbar_init(v_full, 1);
        mbar_init(v_empty, 1);
        for (int s = 0; s < 2; s++)
        {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_free[s], 4);
            mbar_init(&p_full[s], 4);
            mbar_init(&p_empty[s], 1);
            mbar_init(&o_done[s], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0)
    {
        if (lane == 0)
        {
            // ---------------- TMA producer: Q pair per unit, K tiles into the ring
            int g = 0; // K tiles issued so far
            int it = 0;
            bool q_out = false;
            uint32_t q_par = 0;
            int k_issued[K_STAGES] = {0, 0};
            uint32_t k_par[K_STAGES] = {0, 0};
            for (int w = blockIdx.x; w < args.num_work && !*abort_flag; w += gridDim.x, it++)
            {
                const Work wk = decode_work(args, w);
                const int x0 = wk.head * HD;
                if (it > 0 && !mbar_wait(q_empty, (it - 1) & 1, abort_flag, args.status)) break;
                mbar_arrive_expect_tx(q_full, wk.has_b ? 2 * TILE_BYTES : TILE_BYTES);
                tma_load_2d(sQ, &tq, q_full, x0, wk.seq_off + wk.q0);
                tma_load_2d(sQ + CHUNK_BYTES, &tq, q_full, x0 + 64, wk.seq_off + wk.q0);
                if (wk.has_b)
                {
                    tma_load_2d(sQ + TILE_BYTES, &tq, q_full, x0, wk.seq_off + wk.q0 + TILE);
                    tma_load_2d(sQ + TILE_BYTES + CHUNK_BYTES, &tq, q_full, x0 + 64, wk.seq_off + wk.q0 + TILE);
                }
                q_out = true;
                q_par = it & 1;
                if (w + (int)gridDim.x < args.num_work)
                {
                    const Work nx = decode_work(args, w + gridDim.x);
                    const int ny = nx.seq_off + nx.q0;
                    tma_prefetch_l2_2d(&tq, nx.head * HD, ny);
                    tma_prefetch_l2_2d(&tq, nx.head * HD + 64, ny);
                    if (nx.has_b)
                    {
                        tma_prefetch_l2_2d(&tq, nx.head * HD, ny + TILE);
                        tma_prefetch_l2_2d(&tq, nx.head * HD + 64, ny + TILE);
                    }
                }
                bool ok = true;
                for (int j = 0; j < wk.nkv; j++, g++)
                {
                    const int ks = g % K_STAGES;
                    const uint32_t kp = (uint32_t)(g / K_STAGES) & 1u;
                    if (!mbar_wait(&k_empty[ks], kp ^ 1, abort_flag, args.status))
                    {
                        ok = false;
                        break;
                    }
                    const int y = wk.seq_off + j * TILE;
                    mbar_arrive_expect_tx(&k_full[ks], TILE_BYTES);
                    tma_load_2d(sK + ks * TILE_BYTES, &tk, &k_full[ks], x0, y);
                    tma_load_2d(sK + ks * TILE_BYTES + CHUNK_BYTES, &tk, &k_full[ks], x0 + 64, y);
                    k_issued[ks] = 1;
                    k_par[ks] = kp;
                }
                if (!ok) break;
            }
            if (*abort_flag)
            {
                // no TMA write may land after the CTA exits
                if (q_out) drain_wait(q_full, q_par);
                for (int s = 0; s < K_STAGES; s++)
                    if (k_issued[s]) drain_wait(&k_full[s], k_par[s]);
            }
        }
        else if (lane == 1)
        {
            // ---------------- TMA producer: V tiles (one buffer; V(j) is needed
            // only after the softmax of key tile j, so it reloads behind PV(j-1))
            int g = 0;
            bool issued = false;
            uint32_t last = 0;
            for (int w = blockIdx.x; w < args.num_work && !*abort_flag; w += gridDim.x)
            {
                const Work wk = decode_work(args, w);
                const int x0 = wk.head * HD;
                bool ok = true;
                for (int j = 0; j < wk.nkv; j++, g++)
                {
                    const uint32_t vp = (uint32_t)g & 1u;
                    if (!mbar_wait(v_empty, vp ^ 1, abort_flag, args.status))
                    {
                        ok = false;
                        break;
                    }
                    const int y = wk.seq_off + j * TILE;
                    mbar_arrive_expect_tx(v_full, TILE_BYTES);
                    tma_load_2d(sV, &tv, v_full, x0, y);
                    tma_load_2d(sV + CHUNK_BYTES, &tv, v_full, x0 + 64, y);
                    issued = true;
                    last = vp;
                }
                if (!ok) break;
            }
            if (*abort_flag && issued) drain_wait(v_full, last);
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            // ---------------- MMA issuer
            bool any = false;
            bool ok = true;
            int gk = 0, gv = 0, it = 0;
            uint32_t sfree[2] = {0, 0}, pfull[2] = {0, 0};
            bool s_issued[2] = {false, false};
            // shared-memory matrix descriptors; buffers are one tile (kTileDesc) apart
            const uint64_t q_desc0 = umma_desc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t k_desc0 = umma_desc_sw128(smem_u32(sK), 16, 1024);
            const uint64_t v_desc0 = umma_desc_sw128(smem_u32(sV), CHUNK_BYTES, 1024);
            const uint64_t p_desc0 = umma_desc_sw128(smem_u32(sP), 16, 1024);
            constexpr uint32_t kTileDesc = TILE_BYTES >> 4;
            for (int w = blockIdx.x; w < args.num_work && ok; w += gridDim.x, it++)
            {
                const Work wk = decode_work(args, w);
                const int ntiles = wk.has_b ? 2 : 1;
                // S_x = Q_x K^T for key tile j (ring slot of K tile gkk); a ragged
                // last tile runs with N = its keys rounded up to 16.  Compile-time
                // descriptor offsets keep the issue path MMAs only.
                auto issue_s = [&](int x, int gkk, int j) {
                    const int valid = wk.S_len - j * TILE;
                    const int n = valid >= TILE ? TILE : ((valid + 15) & ~15);
                    const uint32_t idesc = umma_idesc_bf16(128, n, 0, 0);
                    const uint64_t qd = q_desc0 + (x ? kTileDesc : 0u);
                    const uint64_t kd = k_desc0 + (uint32_t)(gkk % K_STAGES) * kTileDesc;
                    const uint32_t d = tmem + x * 128;
                    umma_bf16_i<0>(d, qd, kd, idesc);
#pragma unroll
                    for (int k = 1; k < HD / 16; k++)
                    {
                        const uint32_t off = ((k >> 2) * CHUNK_BYTES + (k & 3) * 32) >> 4;
                        umma_bf16_i<1>(d, qd + off, kd + off, idesc);
                    }
                    umma_commit(&s_full[x]);
                };
                // O_x (+)= P_x V over the tile's keys (16 per MMA; P is zero past
                // the window's sequence)
                auto issue_pv = [&](int x, int j) {
                    const int valid = wk.S_len - j * TILE;
                    const uint64_t pd = p_desc0 + (x ? kTileDesc : 0u);
                    const uint32_t o_tmem = tmem + 256 + x * 128;
                    if (valid >= TILE)
                    {
                        if (j == 0)
                            umma_bf16_i<0>(o_tmem, pd, v_desc0, IDESC_O);
                        else
                            umma_bf16_i<1>(o_tmem, pd, v_desc0, IDESC_O);
#pragma unroll
                        for (int k = 1; k < TILE / 16; k++)
                        {
                            const uint32_t aoff = ((k >> 2) * CHUNK_BYTES + (k & 3) * 32) >> 4;
                            umma_bf16_i<1>(o_tmem, pd + aoff, v_desc0 + ((k * 16 * 128) >> 4), IDESC_O);
                        }
                    }
                    else
                    {
                        const int ksteps = (valid + 15) / 16;
                        for (int k = 0; k < ksteps; k++)
                        {
                            const uint32_t aoff = ((k >> 2) * CHUNK_BYTES + (k & 3) * 32) >> 4;
                            umma_bf16(o_tmem, pd + aoff, v_desc0 + ((k * 16 * 128) >> 4), IDESC_O, (j | k) != 0);
                        }
                    }
                    umma_commit(&p_empty[x]);
                };
                auto wait_k = [&](int g_) {
                    return mbar_wait(&k_full[g_ % K_STAGES], (uint32_t)(g_ / K_STAGES) & 1u, abort_flag, args.status);
                };
                // S_x(j) may overwrite S_x once the softmax has read the previous one
                auto s_ready = [&](int x) {
                    if (!s_issued[x]) return true;
                    const bool r = mbar_wait(&s_free[x], sfree[x] & 1u, abort_flag, args.status);
                    sfree[x]++;
                    return r;
                };
                if (!mbar_wait(q_full, it & 1, abort_flag, args.status) || !wait_k(gk))
                {
                    ok = false;
                    break;
                }
                for (int x = 0; x < ntiles && ok; x++)
                {
                    if (!s_ready(x))
                    {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_s(x, gk, 0);
                    s_issued[x] = true;
                }
                if (!ok) break;
                umma_commit(&k_empty[gk % K_STAGES]);
                gk++;
                any = true;
                if (wk.nkv == 1) umma_commit(q_empty);
                for (int j = 0; j < wk.nkv && ok; j++)
                {
                    // next scores first: they only need the softmax to have read S(j)
                    if (j + 1 < wk.nkv)
                    {
                        if (!wait_k(gk))
                        {
                            ok = false;
                            break;
                        }
                        for (int x = 0; x < ntiles && ok; x++)
                        {
                            if (!s_ready(x))
                            {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            issue_s(x, gk, j + 1);
                        }
                        if (!ok) break;
                        umma_commit(&k_empty[gk % K_STAGES]);
                        gk++;
                        if (j + 2 == wk.nkv) umma_commit(q_empty); // the unit's last S MMA
                    }
                    if (!mbar_wait(v_full, (uint32_t)gv & 1u, abort_flag, args.status))
                    {
                        ok = false;
                        break;
                    }
                    for (int x = 0; x < ntiles; x++)
                    {
                        if (!mbar_wait(&p_full[x], pfull[x] & 1u, abort_flag, args.status))
                        {
                            ok = false;
                            break;
                        }
                        pfull[x]++;
                        tc_fence_after();
                        issue_pv(x, j);
                        if (j + 1 == wk.nkv) umma_commit(&o_done[x]);
                    }
                    if (!ok) break;
                    umma_commit(v_empty);
                    gv++;
                }
            }
            if (any)
            {
                umma_commit(drain);
                drain_wait(drain, 0);
            }
        }
    }
    else
    {
        // ---------------- softmax + epilogue (warps 2-5: tile A, 6-9: tile B)
        const int x = (warp - 2) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const uint32_t s_addr = tmem + lane_base + x * 128;
        const uint32_t o_addr = tmem + lane_base + 256 + x * 128;
        uint8_t* p_tile = sP + x * TILE_BYTES;
        const uint64_t c2 = pk2(__float_as_uint(args.scale_log2), __float_as_uint(args.scale_log2));
        uint32_t scnt = 0, pecnt = 0, ocnt = 0;
        bool pv_before = false; // a PV_x has been issued (P_x / O_x may be in use)
        bool ok = true;
        for (int w = blockIdx.x; w < args.num_work && ok; w += gridDim.x)
        {
            const Work wk = decode_work(args, w);
            if (x == 1 && !wk.has_b) continue;
            const int qbase = wk.q0 + x * TILE;
            float m_used = -INFINITY;
            float l_run = 0.f;
            for (int j = 0; j < wk.nkv; j++)
            {
                if (!warp_wait(&s_full[x], scnt & 1, abort_flag, args.status))
                {
                    ok = false;
                    break;
                }
                scnt++;
                tc_fence_after();
                const int valid = wk.S_len - j * TILE; // >= 1
                const bool full = valid >= TILE;
                // Scores in two 64-column halves so only one half is live: the
                // max reads the second half in 32-column pieces, the first
                // half's exponentials run, then the second half is reloaded and
                // S released (the next S_x is needed only at the next key tile).
                uint32_t v[64];
                tmem_ld64(s_addr, v);
                float mo;
                {
                    uint32_t t[32];
                    tmem_ld32(s_addr + 64, t);
                    tmem_ld_wait();
                    mo = full ? row_max<true, 32>(t, valid - 64) : row_max<false, 32>(t, valid - 64);
                    tmem_ld32(s_addr + 96, t);
                    tmem_ld_wait();
                    mo = fmaxf(mo, full ? row_max<true, 32>(t, valid - 96) : row_max<false, 32>(t, valid - 96));
                }
                const float mx = fmaxf(mo, full ? row_max<true, 64>(v, valid) : row_max<false, 64>(v, valid));
                const float mt = mx * args.scale_log2;
                float alpha = 1.f;
                const bool rescale = j > 0 && mt > m_used + RESCALE_THRESHOLD;
                if (j == 0)
                    m_used = mt;
                else if (rescale)
                {
                    alpha = ex2(m_used - mt);
                    m_used = mt;
                }
                const uint64_t negm2 = pk2(__float_as_uint(-m_used), __float_as_uint(-m_used));
                uint64_t sum2[4] = {0, 0, 0, 0};
                uint32_t pk[32];
                if (full)
                    row_exp64<true>(v, valid, c2, negm2, pk, sum2);
                else
                    row_exp64<false>(v, valid, c2, negm2, pk, sum2);
                // P_x and O_x are free once the previous PV_x has completed
                if (pv_before)
                {
                    if (!warp_wait(&p_empty[x], pecnt & 1, abort_flag, args.status))
                    {
                        ok = false;
                        break;
                    }
                    pecnt++;
                    tc_fence_after();
                }
                store_p_half<0>(p_tile, row, pk);
                tmem_ld64(s_addr + 64, v);
                tmem_ld_wait();
                // S_x is in registers: the next S_x may be computed into TMEM
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[x]);
                if (full)
                    row_exp64<true>(v, valid - 64, c2, negm2, pk, sum2);
                else
                    row_exp64<false>(v, valid - 64, c2, negm2, pk, sum2);
                store_p_half<1>(p_tile, row, pk);
                float rowsum;
                {
                    const uint64_t s2 = fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3]));
                    float lo, hi;
                    upk2(s2, lo, hi);
                    rowsum = lo + hi;
                }
                if (rescale)
                {
#pragma unroll
                    for (int c = 0; c < 4; c++)
                    {
                        uint32_t o[32];
                        tmem_ld32(o_addr + c * 32, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(o_addr + c * 32, o);
                    }
                    tmem_st_wait();
                    l_run *= alpha;
                }
                l_run += rowsum;
                fence_proxy_async_smem(); // P is read by the tensor core (async proxy)
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[x]);
                pv_before = true;
            }
            if (!ok) break;
            if (!warp_wait(&o_done[x], ocnt & 1, abort_flag, args.status))
            {
                ok = false;
                break;
            }
            ocnt++;
            tc_fence_after();
            const int qi = qbase + row;
            const float inv = 1.f / l_run;
            bool remote = false;
#pragma unroll 1
            for (int c = 0; c < 4; c++)
            {
                uint32_t v[32];
                tmem_ld32(o_addr + c * 32, v);
                tmem_ld_wait();
                if (qi < wk.S_len)
                {
                    float o[32];
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __uint_as_float(v[i]);
                    remote |= store_row(args, wk.window, wk.part_off, wk.L, qi, wk.head * HD + c * 32, o, inv);
                }
            }
            // a row stored into a peer GPU must be visible there once this
            // rank passes its next cross-GPU barrier
            if (remote) __threadfence_system();
            // O has been read: the next unit's first PV may overwrite it
            // (ordered by this group's next p_full arrival)
            tc_fence_before();
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

} // namespace

int launch_window_attention(Context& ctx, const AttnSchedule& s, int heads, const void* q, const void* k,
                            const void* v, int out_f32, int round_bf16, void* video_out, float* text_partial,
                            void* const* peer_out, int num_peers)
{
    if (num_peers < 0 || num_peers > kMaxPeers || (num_peers > 0 && !peer_out)) return S2_ERR_INVALID;
    for (int i = 0; i < num_peers; i++)
        if (reinterpret_cast<uintptr_t>(peer_out[i]) & 31) return S2_ERR_INVALID;
    if (s.num_items <= 0) return S2_OK;
    // The epilogue writes 32-byte vectors straight into the output rows.
    if ((reinterpret_cast<uintptr_t>(video_out) & 31) || (reinterpret_cast<uintptr_t>(text_partial) & 31))
        return S2_ERR_INVALID;
    const int inner = heads * HD;
    CUtensorMap mq, mk, mv;
    int r = make_tmap_bf16_2d(&mq, q, inner, s.packed_rows, (uint64_t)inner * 2, 64, TILE);
    if (r == 0) r = make_tmap_bf16_2d(&mk, k, inner, s.packed_rows, (uint64_t)inner * 2, 64, TILE);
    if (r == 0) r = make_tmap_bf16_2d(&mv, v, inner, s.packed_rows, (uint64_t)inner * 2, 64, TILE);
    if (r != 0) return r;
    AttnArgs a;
    a.win_info = s.win_info;
    a.win_pool = s.win_pool;
    a.items = s.items;
    a.video_indices = s.video_indices;
    a.inner = inner;
    a.scale_log2 = 1.4426950408889634f / sqrtf((float)HD);
    a.out_f32 = out_f32;
    a.round_bf16 = round_bf16;
    a.video_out = video_out;
    a.text_partial = text_partial;
    a.status = ctx.status;
    for (int i = 0; i < kMaxPeers; i++) a.peer_out[i] = i < num_peers ? peer_out[i] : nullptr;
    static std::atomic<uint64_t> configured{0};
    if (first_on_device(configured) &&
        cudaFuncSetAttribute(window_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
        return S2_ERR_CUDA;
    a.heads = heads;
    a.num_work = s.num_items * heads;
    const int grid = a.num_work < ctx.num_sms ? a.num_work : ctx.num_sms;
    const double video_rows = (double)s.packed_rows - s.partial_rows;
    ProfileScope prof(ctx, K_ATTN, s.attn_flops_per_head * heads,
                      (double)s.packed_rows * inner * 2.0 * 3.0 + video_rows * inner * (out_f32 ? 4.0 : 2.0) +
                          (double)s.partial_rows * inner * 4.0);
    window_attention_kernel<<<grid, NUM_THREADS, SMEM_BYTES, ctx.stream>>>(mq, mk, mv, a);
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

} // namespace s2
