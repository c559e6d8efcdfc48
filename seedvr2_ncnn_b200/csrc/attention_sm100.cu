// Varlen window attention on sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the per-window ncnn SDPA call and the scatter shader of
// AdaptiveWindowAttention::forward (adaptive_window_attention.cpp:873-975 CPU,
// :1172-1268 Vulkan, scatter shader :353-409).  Each window's sequence is its
// L video rows followed by the sample's T text rows, packed contiguously
// (window after window) in bf16 [rows][heads*128] by the prepare kernel.
//
// One CTA = (window, pair of 128-row query tiles A and B, head).  K/V tiles
// are loaded once for both query tiles.  Warp roles:
//   warp 0     TMA: Q_A and Q_B once, then K/V tiles into a 2-stage ring;
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
constexpr int TMEM_COLS = 512;               // S/P_A [0,128) S/P_B [128,256) O_A [256,384) O_B [384,512)
constexpr uint32_t IDESC_S = umma_idesc_bf16(128, 128, 0, 0);
constexpr uint32_t IDESC_O = umma_idesc_bf16(128, 128, 0, 1); // B (= V) MN-major
constexpr int SMEM_BYTES = 6 * TILE_BYTES + 1024 + 256;       // Q_A, Q_B, K x2, V x2
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

// 2^x on the FMA and integer pipes, for a share of the softmax exponentials
// so the MUFU unit (ex2.approx) is not the only source: x = j + f with
// j = round(x) (the 1.5*2^23 shift trick, f in [-1/2, 1/2]), 2^f from a cubic
// fitted for this kernel (weighted least squares iterated toward minimum
// relative error on [-1/2, 1/2]; max relative error 7.5e-5, far below the
// 2^-9 of the bf16 P it feeds), and 2^j added into the exponent field.
// x is clamped at -125 (2^-125 is 0 for softmax purposes) so the exponent
// add stays in the normal range.
constexpr uint64_t kMagic2 = 0x4B4000004B400000ull;    // 1.5*2^23 (x2)
constexpr uint64_t kNegMagic2 = 0xCB400000CB400000ull; // -1.5*2^23
constexpr uint64_t kNegOne2 = 0xBF800000BF800000ull;   // -1
constexpr uint64_t kC0 = 0x3F7FFB4A3F7FFB4Aull;        // 0.99992812
constexpr uint64_t kC1 = 0x3F31798D3F31798Dull;        // 0.69326097
constexpr uint64_t kC2 = 0x3E786EE63E786EE6ull;        // 0.24261054
constexpr uint64_t kC3 = 0x3D61FB533D61FB53ull;        // 0.05517132

__device__ __forceinline__ void ex2_poly(uint64_t t2, float& p0, float& p1)
{
    float x0, x1;
    upk2(t2, x0, x1);
    const uint64_t x2 = pk2(__float_as_uint(fmaxf(x0, -125.f)), __float_as_uint(fmaxf(x1, -125.f)));
    const uint64_t r2 = fadd2(x2, kMagic2);
    const uint64_t f2 = ffma2(fadd2(r2, kNegMagic2), kNegOne2, x2);
    uint64_t q2 = ffma2(f2, kC3, kC2);
    q2 = ffma2(q2, f2, kC1);
    q2 = ffma2(q2, f2, kC0);
    float q0, q1, r0, r1;
    upk2(q2, q0, q1);
    upk2(r2, r0, r1);
    p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(r0) << 23));
    p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(r1) << 23));
}

// Row max of the 128 raw scores of one key tile (FULL: no masked columns).
template <bool FULL>
__device__ __forceinline__ float row_max(const uint32_t (&v)[128], int valid)
{
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 128; i += 2)
    {
        float a = __uint_as_float(v[i]), b = __uint_as_float(v[i + 1]);
        if (!FULL)
        {
            a = i < valid ? a : -INFINITY;
            b = i + 1 < valid ? b : -INFINITY;
        }
        mx = fmax3(mx, a, b);
    }
    return mx;
}

// P = exp2(S * c - m) for the row (masked columns -> 0), written over the
// first 64 TMEM columns of the S tile as packed bf16 pairs; returns the fp32
// row sum.  In full tiles 3 of every 8 pairs use the polynomial exp2.
template <bool FULL>
__device__ __forceinline__ float row_exp(const uint32_t (&v)[128], int valid, uint64_t c2, uint64_t negm2,
                                         uint32_t s_addr)
{
    uint64_t sum2 = 0;
#pragma unroll
    for (int c = 0; c < 4; c++)
    {
        uint32_t packed[16];
#pragma unroll
        for (int q = 0; q < 16; q++)
        {
            const int i = c * 32 + 2 * q;
            const uint64_t t2 = ffma2(pk2(v[i], v[i + 1]), c2, negm2);
            float p0, p1;
            if (FULL && (q & 7) < 3)
                ex2_poly(t2, p0, p1);
            else
            {
                float t0, t1;
                upk2(t2, t0, t1);
                p0 = ex2(t0);
                p1 = ex2(t1);
                if (!FULL)
                {
                    p0 = i < valid ? p0 : 0.f;
                    p1 = i + 1 < valid ? p1 : 0.f;
                }
            }
            sum2 = fadd2(sum2, pk2(__float_as_uint(p0), __float_as_uint(p1)));
            packed[q] = pack_bf16x2(p0, p1);
        }
        tmem_st16(s_addr + c * 16, packed);
    }
    float lo, hi;
    upk2(sum2, lo, hi);
    return lo + hi;
}

__device__ __forceinline__ void st_v8(void* p, const uint32_t (&r)[8])
{
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(r[0]), "r"(r[1]), "r"(r[2]),
                 "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
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

__global__ void __launch_bounds__(NUM_THREADS, 1)
    window_attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                            const __grid_constant__ CUtensorMap tv, const AttnArgs args)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                // Q_A, Q_B
    uint8_t* sK = sQ + 2 * TILE_BYTES; // 2 stages
    uint8_t* sV = sK + 2 * TILE_BYTES; // 2 stages
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * TILE_BYTES);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;   // [2]
    uint64_t* v_full = bars + 3;   // [2]
    uint64_t* kv_empty = bars + 5; // [2]
    uint64_t* s_full = bars + 7;   // [2] per query tile
    uint64_t* p_full = bars + 9;   // [2] per query tile
    uint64_t* o_done = bars + 11;  // [2] per query tile
    uint64_t* drain = bars + 13;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int head = blockIdx.y;
    const int2 item = args.items[blockIdx.x];
    const int4 wi = args.win_info[item.x];
    const int seq_off = wi.x, L = wi.y, T = wi.z, part_off = wi.w;
    const int S_len = L + T;
    const int q0 = item.y;
    const bool has_b = q0 + TILE < S_len;
    const int nkv = (S_len + TILE - 1) / TILE;

    if (threadIdx.x == 0)
    {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; s++)
        {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 1);
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], 128);
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
            // ---------------- TMA producer
            const int x0 = head * HD;
            int issued_stage[2] = {0, 0};
            uint32_t last_parity[2] = {0, 0};
            mbar_arrive_expect_tx(q_full, has_b ? 2 * TILE_BYTES : TILE_BYTES);
            tma_load_2d(sQ, &tq, q_full, x0, seq_off + q0);
            tma_load_2d(sQ + CHUNK_BYTES, &tq, q_full, x0 + 64, seq_off + q0);
            if (has_b)
            {
                tma_load_2d(sQ + TILE_BYTES, &tq, q_full, x0, seq_off + q0 + TILE);
                tma_load_2d(sQ + TILE_BYTES + CHUNK_BYTES, &tq, q_full, x0 + 64, seq_off + q0 + TILE);
            }
            for (int j = 0; j < nkv; j++)
            {
                const int st = j & 1;
                const uint32_t par = (j >> 1) & 1;
                if (!mbar_wait(&kv_empty[st], par ^ 1, abort_flag, args.status)) break;
                const int y = seq_off + j * TILE;
                mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
                tma_load_2d(sK + st * TILE_BYTES, &tk, &k_full[st], x0, y);
                tma_load_2d(sK + st * TILE_BYTES + CHUNK_BYTES, &tk, &k_full[st], x0 + 64, y);
                mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
                tma_load_2d(sV + st * TILE_BYTES, &tv, &v_full[st], x0, y);
                tma_load_2d(sV + st * TILE_BYTES + CHUNK_BYTES, &tv, &v_full[st], x0 + 64, y);
                issued_stage[st] = 1;
                last_parity[st] = par;
            }
            if (*abort_flag)
            {
                drain_wait(q_full, 0);
                for (int s = 0; s < 2; s++)
                    if (issued_stage[s])
                    {
                        drain_wait(&k_full[s], last_parity[s]);
                        drain_wait(&v_full[s], last_parity[s]);
                    }
            }
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            // ---------------- MMA issuer
            bool any = false;
            const int ntiles = has_b ? 2 : 1;
            auto issue_s = [&](int x, int j) {
                const uint32_t q_addr = smem_u32(sQ + x * TILE_BYTES);
                const uint32_t k_addr = smem_u32(sK + (j & 1) * TILE_BYTES);
                const uint32_t d = tmem + x * 128;
#pragma unroll
                for (int k = 0; k < HD / 16; k++)
                {
                    const uint32_t off = (k >> 2) * CHUNK_BYTES + (k & 3) * 32;
                    umma_bf16(d, umma_desc_sw128(q_addr + off, 16, 1024), umma_desc_sw128(k_addr + off, 16, 1024),
                              IDESC_S, k != 0);
                }
                umma_commit(&s_full[x]);
            };
            auto issue_pv = [&](int x, int j) {
                const uint32_t v_addr = smem_u32(sV + (j & 1) * TILE_BYTES);
                const uint32_t p_tmem = tmem + x * 128; // P packed bf16x2 over S columns [0,64)
                const uint32_t o_tmem = tmem + 256 + x * 128;
#pragma unroll
                for (int k = 0; k < TILE / 16; k++)
                    umma_bf16_tmem_a(o_tmem, p_tmem + k * 8, umma_desc_sw128(v_addr + k * 16 * 128, CHUNK_BYTES, 1024),
                                     IDESC_O, (j | k) != 0);
            };
            do
            {
                if (!mbar_wait(q_full, 0, abort_flag, args.status)) break;
                if (!mbar_wait(&k_full[0], 0, abort_flag, args.status)) break;
                tc_fence_after();
                for (int x = 0; x < ntiles; x++) issue_s(x, 0);
                any = true;
                bool ok = true;
                for (int j = 0; j < nkv && ok; j++)
                {
                    const int st = j & 1;
                    if (!mbar_wait(&v_full[st], (j >> 1) & 1, abort_flag, args.status)) break;
                    const bool more = j + 1 < nkv;
                    if (more && !mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort_flag, args.status)) break;
                    for (int x = 0; x < ntiles; x++)
                    {
                        if (!mbar_wait(&p_full[x], j & 1, abort_flag, args.status))
                        {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        issue_pv(x, j);
                        if (!more) umma_commit(&o_done[x]);
                        if (x == ntiles - 1) umma_commit(&kv_empty[st]);
                        if (more) issue_s(x, j + 1);
                    }
                }
            } while (0);
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
        const int qbase = q0 + x * TILE;
        if (x == 0 || has_b)
        {
            float m_used = -INFINITY;
            float l_run = 0.f;
            bool ok = true;
            for (int j = 0; j < nkv; j++)
            {
                if (!warp_wait(&s_full[x], j & 1, abort_flag, args.status))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int valid = S_len - j * TILE; // >= 1
                const bool full = valid >= TILE;
                uint32_t v[128];
                tmem_ld128(s_addr, v);
                tmem_ld_wait();
                const float mx = full ? row_max<true>(v, valid) : row_max<false>(v, valid);
                const float mt = mx * args.scale_log2;
                if (j == 0)
                    m_used = mt;
                else if (mt > m_used + RESCALE_THRESHOLD)
                {
                    // O is stable here: S_X(j) was committed after PV_X(j-1).
                    const float alpha = ex2(m_used - mt);
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
                    l_run *= alpha;
                    m_used = mt;
                }
                const uint64_t c2 = pk2(__float_as_uint(args.scale_log2), __float_as_uint(args.scale_log2));
                const uint64_t negm2 = pk2(__float_as_uint(-m_used), __float_as_uint(-m_used));
                const float rowsum = full ? row_exp<true>(v, valid, c2, negm2, s_addr)
                                          : row_exp<false>(v, valid, c2, negm2, s_addr);
                l_run += rowsum;
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&p_full[x]);
            }
            if (ok && warp_wait(&o_done[x], 0, abort_flag, args.status))
            {
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
                    if (qi < S_len)
                    {
                        float o[32];
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __uint_as_float(v[i]);
                        remote |= store_row(args, item.x, part_off, L, qi, head * HD + c * 32, o, inv);
                    }
                }
                // a row stored into a peer GPU must be visible there once this
                // rank passes its next cross-GPU barrier
                if (remote) __threadfence_system();
            }
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
    static bool configured = false;
    if (!configured)
    {
        if (cudaFuncSetAttribute(window_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
            return S2_ERR_CUDA;
        configured = true;
    }
    dim3 grid(s.num_items, heads);
    const double video_rows = (double)s.packed_rows - s.partial_rows;
    ProfileScope prof(ctx, K_ATTN, s.attn_flops_per_head * heads,
                      (double)s.packed_rows * inner * 2.0 * 3.0 + video_rows * inner * (out_f32 ? 4.0 : 2.0) +
                          (double)s.partial_rows * inner * 4.0);
    window_attention_kernel<<<grid, NUM_THREADS, SMEM_BYTES, ctx.stream>>>(mq, mk, mv, a);
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

} // namespace s2
