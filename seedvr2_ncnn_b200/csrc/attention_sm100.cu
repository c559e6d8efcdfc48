// Varlen window attention on sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the per-window ncnn SDPA call and the scatter shader of
// AdaptiveWindowAttention::forward (adaptive_window_attention.cpp:873-975 CPU,
// :1172-1268 Vulkan, scatter shader :353-409).  Each window's sequence is its
// L video rows followed by the sample's T text rows, packed contiguously
// (window after window) in bf16 [rows][heads*128]; every row attends to the
// whole sequence (no mask), softmax(Q K^T / sqrt(128)) V.
//
// Work unit = (pair of 128-row query tiles 0 and 1 of one window, head); a
// persistent grid of one CTA per SM walks the units.  K/V tiles are loaded
// once for both query tiles.  384 threads, three warpgroups:
//   warps 0-3   softmax + epilogue of query tile 0   (200 registers each)
//   warps 4-7   softmax + epilogue of query tile 1   (200 registers each)
//   warp 8      TMA: Q pair per unit, K tiles into a 2-slot ring
//   warp 9      MMA: one thread issues every tcgen05.mma
//   warp 10     TMA: V tiles into a 2-slot ring
//   warp 11     idle (the warpgroup gives its registers to the softmax)
// `setmaxnreg` moves registers from the TMA / MMA warpgroup (104 each) to the
// two softmax warpgroups (200 each), so a thread holds its whole 128-column
// score row in registers.
//
// Tensor memory (512 columns): S_0 [0,128) S_1 [128,256) O_0 [256,384)
// O_1 [384,512).  A softmax thread owns one query row (one TMEM lane): it
// loads the row of S_x(j) into registers, forms P = exp2(S*c - m) and stores
// P as packed bf16 back into the first 64 columns of S_x; the PV MMA reads P
// from tensor memory (A operand) and V from shared memory, so the tensor
// core reads only Q, K and V from shared memory.  The MMA thread issues, per
// key tile j,
//     PV_0(j)  S_0(j+1)  PV_1(j)  S_1(j+1)
// so S_x(j+1) overwrites P_x(j) only after PV_x(j) has read it (tcgen05 MMAs
// of one thread run in issue order), and while the softmax of tile 0 runs
// the tensor core works on tile 1 and the other way round.  The s_full_x
// commit after S_x(j+1) also covers PV_x(j), so when the softmax sees S_x(j)
// the accumulator O_x is stable and it may rescale it in place: the running
// max is raised (and O, l rescaled) only when it grows by more than 2^8.
//
// Exponentials: a quarter of each row's column pairs is exponentiated on the
// FMA pipe (2^t = 2^n * 2^f, n = round(t), f in [-1/2, 1/2], a cubic for
// 2^f) and the rest on the MUFU (ex2.approx): with head_dim 128 a 128 x 128
// tile's 16,384 exponentials alone would take the MUFU as long as the tile's
// two MMAs take the tensor core.  (Measured: a quarter beats none, a half
// and three quarters.)
//
// Epilogue: O / l -- video rows stored straight to their source token (the
// scatter; peer GPUs' rows over NVLink), text rows to a per-window fp32
// partial that text_pool averages over the sample's windows.  Each row's
// destination is read when its unit starts and every role decodes the next
// unit's descriptor one unit ahead, so no dependent global load sits between
// two units.  Keys past the
// window's sequence are masked; query rows past it are computed but never
// stored.  The ragged last key tile loads, exponentiates and stores only its
// 32-column chunks that hold keys, and its MMAs run with N (S) or K (PV)
// rounded up to 16.
//
// Every mbarrier wait is bounded: on expiry the kernel records a timeout in
// the status word, drains its own TMA / MMA work (bounded), frees TMEM and
// returns.
#include "s2_common.cuh"
#include "s2_internal.h"

namespace s2 {

namespace {

constexpr int HD = 128;                      // head_dim
constexpr int TILE = 128;                    // q rows / keys per tile
constexpr int CHUNK_BYTES = TILE * 128;      // 128 rows x 64 bf16 (one swizzle row each)
constexpr int TILE_BYTES = 2 * CHUNK_BYTES;  // 128 x 128 bf16
constexpr int NUM_THREADS = 384;
constexpr int TMEM_COLS = 512;               // S_0 S_1 O_0 O_1
constexpr uint32_t IDESC_O = umma_idesc_bf16(128, 128, 0, 1); // A (= P, tensor memory) K-major, B (= V) MN-major
constexpr int K_STAGES = 2;
constexpr int V_STAGES = 2;
// Q_0, Q_1 | K ring | V ring
constexpr int SMEM_BYTES = (2 + K_STAGES + V_STAGES) * TILE_BYTES + 1024 + 256;
constexpr float RESCALE_THRESHOLD = 8.0f; // log2 units
// Register split (setmaxnreg): the kernel is launched with LAUNCH_REGS per
// thread; the TMA / MMA warpgroup drops to SUPPORT_REGS and the two softmax
// warpgroups rise to SOFTMAX_REGS.  The shares must add up to the launch's
// total exactly (an increase that the freed registers cannot cover waits
// forever), and the launcher checks the compiled register count first.
constexpr int LAUNCH_REGS = 168;
constexpr int SUPPORT_REGS = 104;
constexpr int SOFTMAX_REGS = 200;
static_assert(2 * 128 * SOFTMAX_REGS + 128 * SUPPORT_REGS == NUM_THREADS * LAUNCH_REGS, "register split");
// Column pairs of each 32-column chunk (16 pairs) exponentiated on the FMA pipe.
constexpr int POLY_PAIRS = 4;

struct AttnArgs
{
    const int4* win_info; // {seq_offset, L, T, partition_offset}
    const int* win_pool;  // partial row of the window's first text row
    const int2* items;    // {window, q0 of tile 0}
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
    // bounds of the checked (S2_DEBUG_BOUNDS) build: video_indices entries,
    // output rows, text partial rows, peer outputs
    int num_video_indices;
    int out_rows;
    int partial_rows;
    int num_peers;
    // peer output bases (multi-GPU): a video_indices entry with a non-zero
    // peer field is stored into peer_out[peer - 1] over NVLink
    void* peer_out[kMaxPeers];
};

template <int N>
__device__ __forceinline__ void regs_increase()
{
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

template <int N>
__device__ __forceinline__ void regs_decrease()
{
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

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

__device__ __forceinline__ uint64_t f2(float v)
{
    return pk2(__float_as_uint(v), __float_as_uint(v));
}

// 2^t for a pair on the FMA pipe.  Range reduction (Cody-Waite with one
// constant, exact here): n = round(t) by adding and subtracting 1.5 * 2^23
// (the sum's low mantissa bits then hold n in two's complement), f = t - n in
// [-1/2, 1/2]; 2^f by a cubic fitted for this kernel (Remez exchange,
// minimax relative error on [-1/2, 1/2], 7.5e-5 -- far below the 2^-9 of the
// bf16 P it feeds); 2^n by adding n to the result's exponent field.  t is
// clamped to -126 so the exponent never leaves the normal range (2^-126 is
// zero for every practical purpose in a softmax).
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t t2)
{
    constexpr float kRound = 12582912.0f; // 1.5 * 2^23
    constexpr float c0 = 0.99992806f, c1 = 0.69326097f, c2 = 0.24261113f, c3 = 0.05517167f;
    float a, b;
    upk2(t2, a, b);
    t2 = pk2(__float_as_uint(fmaxf(a, -126.f)), __float_as_uint(fmaxf(b, -126.f)));
    const uint64_t y = fadd2(t2, f2(kRound));
    const uint64_t n = fadd2(y, f2(-kRound));
    const uint64_t f = ffma2(n, f2(-1.f), t2);
    uint64_t p = ffma2(f, f2(c3), f2(c2));
    p = ffma2(p, f, f2(c1));
    p = ffma2(p, f, f2(c0));
    uint32_t ylo, yhi, plo, phi;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(ylo), "=r"(yhi) : "l"(y));
    asm("mov.b64 {%0, %1}, %2;" : "=r"(plo), "=r"(phi) : "l"(p));
    return pk2(plo + (ylo << 23), phi + (yhi << 23));
}

// 32 lanes x 32 consecutive 32-bit columns -> r[B, B + 32) of the row's
// register array (compile-time indices keep it in registers).
template <int B, int N>
__device__ __forceinline__ void tmem_ld32_at(uint32_t taddr, uint32_t (&r)[N])
{
    static_assert(B + 32 <= N, "register window");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[B + 0]), "=r"(r[B + 1]), "=r"(r[B + 2]), "=r"(r[B + 3]), "=r"(r[B + 4]), "=r"(r[B + 5]),
                   "=r"(r[B + 6]), "=r"(r[B + 7]), "=r"(r[B + 8]), "=r"(r[B + 9]), "=r"(r[B + 10]), "=r"(r[B + 11]),
                   "=r"(r[B + 12]), "=r"(r[B + 13]), "=r"(r[B + 14]), "=r"(r[B + 15]), "=r"(r[B + 16]),
                   "=r"(r[B + 17]), "=r"(r[B + 18]), "=r"(r[B + 19]), "=r"(r[B + 20]), "=r"(r[B + 21]),
                   "=r"(r[B + 22]), "=r"(r[B + 23]), "=r"(r[B + 24]), "=r"(r[B + 25]), "=r"(r[B + 26]),
                   "=r"(r[B + 27]), "=r"(r[B + 28]), "=r"(r[B + 29]), "=r"(r[B + 30]), "=r"(r[B + 31])
                 : "r"(taddr));
}

// Max over chunk C (32 columns) of the row into four independent chains;
// with MASKED, only the chunk's first `rem` columns count.
template <int C, bool MASKED>
__device__ __forceinline__ void chunk_max(const uint32_t (&v)[128], int rem, float (&m)[4])
{
#pragma unroll
    for (int i = 0; i < 32; i += 8)
    {
#pragma unroll
        for (int c = 0; c < 4; c++)
        {
            const int k = i + 2 * c;
            float a = __uint_as_float(v[C * 32 + k]), b = __uint_as_float(v[C * 32 + k + 1]);
            if (MASKED)
            {
                a = k < rem ? a : -INFINITY;
                b = k + 1 < rem ? b : -INFINITY;
            }
            m[c] = fmax3(m[c], a, b);
        }
    }
}

// P for chunk C of the row: t = S * c - m in packed pairs, the first
// POLY_PAIRS pairs exponentiated on the FMA pipe, the rest on the MUFU; with
// MASKED, columns >= rem of the chunk give 0.  Sums the fp32 values into
// sum2 and stores the chunk's 16 packed bf16 pairs into tensor memory at
// p_addr (over the chunk's half-width slot of S).
template <int C, bool MASKED, int N>
__device__ __forceinline__ void chunk_exp(const uint32_t (&v)[N], int rem, uint64_t c2, uint64_t negm2,
                                          uint64_t (&sum2)[4], uint32_t p_addr)
{
    uint32_t p[16];
#pragma unroll
    for (int q = 0; q < 16; q++)
    {
        const int k = 2 * q;
        const uint64_t t2 = ffma2(pk2(v[C * 32 + k], v[C * 32 + k + 1]), c2, negm2);
        float e0, e1;
        if (q < POLY_PAIRS)
            upk2(exp2_poly2(t2), e0, e1);
        else
        {
            float t0, t1;
            upk2(t2, t0, t1);
            e0 = ex2(t0);
            e1 = ex2(t1);
        }
        if (MASKED)
        {
            e0 = k < rem ? e0 : 0.f;
            e1 = k + 1 < rem ? e1 : 0.f;
        }
        p[q] = pack_bf16x2(e0, e1);
        sum2[q & 3] = fadd2(sum2[q & 3], pk2(__float_as_uint(e0), __float_as_uint(e1)));
    }
    tmem_st16(p_addr + C * 16, p);
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

// Where query row qi of a unit goes, read once at the start of the unit so
// the epilogue issues no dependent global load: a video row's source token
// (with the peer GPU in the high bits), a text row's row of the window's
// fp32 partial.  -1 for a padding row past the window.
__device__ __forceinline__ int row_target(const AttnArgs& a, int window, int part_off, int L, int S_len, int qi)
{
    if (qi >= S_len) return -1;
    if (qi < L)
    {
        if (!index_ok((int64_t)part_off + qi, a.num_video_indices, a.status)) return -1;
        const int v = a.video_indices[part_off + qi];
        // (checked build) the peer field names a peer output, the row lies in the outputs
        if (kCheckedIndices && !(index_ok(v >> kPeerShift, a.num_peers + 1, a.status) &&
                                 index_ok(v & ((1 << kPeerShift) - 1), a.out_rows, a.status)))
            return -1;
        return v;
    }
    const int t = a.win_pool[window] + (qi - L);
    return index_ok(t, a.partial_rows, a.status) ? t : -1;
}

// Stores 32 output columns [col0, col0+32) of one query row with 32-byte
// (full-sector) stores: a video row to its source token, a text row to the
// window's fp32 partial.  `target` comes from row_target.
// Returns true when the row went to a peer GPU.
__device__ __forceinline__ bool store_row(const AttnArgs& a, bool video, int target, int col0, const float* o,
                                          float inv)
{
    int src = target;
    void* vbase = a.video_out;
    bool remote = false;
    if (video)
    {
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
                       : a.text_partial + (size_t)target * a.inner + col0;
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

// Softmax of one key tile for one query row: the running max from S_x(j)
// (pass 1), then S_x(j) re-read in 64-column pairs of chunks, P = exp2(S*c -
// m) stored as packed bf16 over the first 64 columns of S_x and the row sum
// added to l (pass 2); when the max grows past the threshold, O_x is
// rescaled in place after P is stored (O_x is stable: PV_x(j-1) completed
// before S_x(j) was signalled, and PV_x(j) waits for this tile's p_full).
// Re-reading is safe: the P of chunk c lands on columns [16c, 16c + 16),
// which pass 2 has already read.  Pass 2 is a loop, not unrolled: a fully
// unrolled 128-column softmax is big enough to evict the MMA warp's issue
// code from the instruction cache, which measured 4-6x slower MMA issue.
// FULL: all 128 keys valid; otherwise `valid` (1..127) keys: chunks wholly
// past them are skipped and only the partial chunk is masked.
template <bool FULL>
__device__ __forceinline__ void softmax_tile(uint32_t s_addr, uint32_t o_addr, int valid, bool first,
                                             float scale_log2, float& m_used, float& l)
{
    const int nfull = FULL ? 4 : valid >> 5; // chunks with every key valid
    const int rem = FULL ? 0 : valid & 31;   // keys of the partial chunk (0: none)
    const int nchunks = nfull + (rem ? 1 : 0);
    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    {
        // pass 1: the row max (all four chunks are loaded -- a conditional load
        // leaves part of the row maybe-undefined, which costs the register
        // allocator dearly; columns past the keys are skipped or masked)
        uint32_t v[128];
        tmem_ld32_at<0>(s_addr, v);
        tmem_ld32_at<32>(s_addr + 32, v);
        tmem_ld32_at<64>(s_addr + 64, v);
        tmem_ld32_at<96>(s_addr + 96, v);
        tmem_ld_wait();
#define S2_CHUNK_MAX(C)                                                                                        \
    if (FULL || nfull > C)                                                                                     \
        chunk_max<C, false>(v, 32, m4);                                                                        \
    else if (nfull == C && rem)                                                                                \
        chunk_max<C, true>(v, rem, m4);
        S2_CHUNK_MAX(0)
        S2_CHUNK_MAX(1)
        S2_CHUNK_MAX(2)
        S2_CHUNK_MAX(3)
#undef S2_CHUNK_MAX
    }
    const float mt = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * scale_log2;
    float alpha = 1.f;
    bool rescale = false;
    if (first)
        m_used = mt;
    else if (mt > m_used + RESCALE_THRESHOLD)
    {
        alpha = ex2(m_used - mt);
        m_used = mt;
        rescale = true;
    }
    const uint64_t c2 = f2(scale_log2);
    const uint64_t negm2 = f2(-m_used);
    uint64_t sum2[4] = {0, 0, 0, 0};
    // pass 2: two chunks per iteration (both loads in flight before the wait)
#pragma unroll 1
    for (int c = 0; c < nchunks; c += 2)
    {
        uint32_t v[64];
        const bool two = c + 1 < nchunks;
        tmem_ld32_at<0>(s_addr + c * 32, v);
        if (two) tmem_ld32_at<32>(s_addr + c * 32 + 32, v);
        tmem_ld_wait();
        const uint32_t p_addr = s_addr + c * 16;
        if (FULL || c < nfull)
            chunk_exp<0, false>(v, 32, c2, negm2, sum2, p_addr);
        else
            chunk_exp<0, true>(v, rem, c2, negm2, sum2, p_addr);
        if (two)
        {
            if (FULL || c + 1 < nfull)
                chunk_exp<1, false>(v, 32, c2, negm2, sum2, p_addr);
            else
                chunk_exp<1, true>(v, rem, c2, negm2, sum2, p_addr);
        }
    }
    const uint64_t s2 = fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3]));
    float lo, hi;
    upk2(s2, lo, hi);
    if (rescale)
    {
#pragma unroll 1
        for (int c = 0; c < 4; c++)
        {
            uint32_t o[32];
            tmem_ld32(o_addr + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_addr + c * 32, o);
        }
        l *= alpha;
    }
    l += lo + hi;
}

// Persistent: CTA b processes units b, b + gridDim.x, ...  Barrier phases run
// on across units, so the next unit's loads and first S MMAs overlap the
// current unit's last tiles and epilogue; the Q pair is reloaded once the
// unit's last S MMA has read it (q_empty).
__global__ void __launch_bounds__(NUM_THREADS, 1)
    window_attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                            const __grid_constant__ CUtensorMap tv, const AttnArgs args)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                       // Q_0, Q_1
    uint8_t* sK = sQ + 2 * TILE_BYTES;        // K ring
    uint8_t* sV = sK + K_STAGES * TILE_BYTES; // V ring
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + V_STAGES * TILE_BYTES);
    uint64_t* q_full = bars + 0;
    uint64_t* q_empty = bars + 1;
    uint64_t* k_full = bars + 2;                  // [K_STAGES]
    uint64_t* k_empty = k_full + K_STAGES;        // [K_STAGES]
    uint64_t* v_full = k_empty + K_STAGES;        // [V_STAGES]
    uint64_t* v_empty = v_full + V_STAGES;        // [V_STAGES]
    uint64_t* s_full = v_empty + V_STAGES;        // [2] S_x computed (and PV_x before it done)
    uint64_t* p_full = s_full + 2;                // [2] P_x stored (4 warp arrivals)
    uint64_t* o_done = p_full + 2;                // [2] last PV_x of the unit done
    uint64_t* drain = o_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
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
        for (int s = 0; s < V_STAGES; s++)
        {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int s = 0; s < 2; s++)
        {
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], 4);
            mbar_init(&o_done[s], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 9) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 8)
    {
        regs_decrease<SUPPORT_REGS>();
        if (warp == 8 && lane == 0)
        {
            // ---------------- TMA: Q pair per unit, K tiles into the ring
            int g = 0; // K tiles issued so far
            int it = 0;
            bool q_out = false;
            uint32_t q_par = 0;
            int k_issued[K_STAGES] = {};
            uint32_t k_par[K_STAGES] = {};
            Work nwk = decode_work(args, blockIdx.x < args.num_work ? blockIdx.x : 0);
            for (int w = blockIdx.x; w < args.num_work && !*abort_flag; w += gridDim.x, it++)
            {
                const Work wk = nwk;
                const bool has_next = w + (int)gridDim.x < args.num_work;
                if (has_next) nwk = decode_work(args, w + gridDim.x);
                const int x0 = wk.head * HD;
                if (it > 0 && !mbar_wait<true>(q_empty, (it - 1) & 1, abort_flag, args.status)) break;
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
                if (has_next)
                {
                    const int ny = nwk.seq_off + nwk.q0;
                    tma_prefetch_l2_2d(&tq, nwk.head * HD, ny);
                    tma_prefetch_l2_2d(&tq, nwk.head * HD + 64, ny);
                    if (nwk.has_b)
                    {
                        tma_prefetch_l2_2d(&tq, nwk.head * HD, ny + TILE);
                        tma_prefetch_l2_2d(&tq, nwk.head * HD + 64, ny + TILE);
                    }
                }
                bool ok = true;
                for (int j = 0; j < wk.nkv; j++, g++)
                {
                    const int ks = g % K_STAGES;
                    const uint32_t kp = (uint32_t)(g / K_STAGES) & 1u;
                    if (!mbar_wait<true>(&k_empty[ks], kp ^ 1, abort_flag, args.status))
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
        else if (warp == 10 && lane == 0)
        {
            // ---------------- TMA: V tiles into the ring
            int g = 0;
            int v_issued[V_STAGES] = {};
            uint32_t v_par[V_STAGES] = {};
            Work nwk = decode_work(args, blockIdx.x < args.num_work ? blockIdx.x : 0);
            for (int w = blockIdx.x; w < args.num_work && !*abort_flag; w += gridDim.x)
            {
                const Work wk = nwk;
                if (w + (int)gridDim.x < args.num_work) nwk = decode_work(args, w + gridDim.x);
                const int x0 = wk.head * HD;
                bool ok = true;
                for (int j = 0; j < wk.nkv; j++, g++)
                {
                    const int vs = g % V_STAGES;
                    const uint32_t vp = (uint32_t)(g / V_STAGES) & 1u;
                    if (!mbar_wait<true>(&v_empty[vs], vp ^ 1, abort_flag, args.status))
                    {
                        ok = false;
                        break;
                    }
                    const int y = wk.seq_off + j * TILE;
                    mbar_arrive_expect_tx(&v_full[vs], TILE_BYTES);
                    tma_load_2d(sV + vs * TILE_BYTES, &tv, &v_full[vs], x0, y);
                    tma_load_2d(sV + vs * TILE_BYTES + CHUNK_BYTES, &tv, &v_full[vs], x0 + 64, y);
                    v_issued[vs] = 1;
                    v_par[vs] = vp;
                }
                if (!ok) break;
            }
            if (*abort_flag)
                for (int s = 0; s < V_STAGES; s++)
                    if (v_issued[s]) drain_wait(&v_full[s], v_par[s]);
        }
        else if (warp == 9 && lane == 0)
        {
            // ---------------- MMA issuer
            bool any = false;
            bool ok = true;
            int gk = 0, gv = 0, it = 0;
            uint32_t pfull[2] = {0, 0};
            // shared-memory matrix descriptors; ring slots are one tile (kTileDesc) apart
            const uint64_t q_desc0 = umma_desc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t k_desc0 = umma_desc_sw128(smem_u32(sK), 16, 1024);
            const uint64_t v_desc0 = umma_desc_sw128(smem_u32(sV), CHUNK_BYTES, 1024);
            constexpr uint32_t kTileDesc = TILE_BYTES >> 4;
            Work nwk = decode_work(args, blockIdx.x < args.num_work ? blockIdx.x : 0);
            for (int w = blockIdx.x; w < args.num_work && ok; w += gridDim.x, it++)
            {
                const Work wk = nwk;
                if (w + (int)gridDim.x < args.num_work) nwk = decode_work(args, w + gridDim.x);
                const int ntiles = wk.has_b ? 2 : 1;
                // S_x = Q_x K^T for key tile j (ring slot of K tile gkk); a ragged
                // last tile runs with N = its keys rounded up to 16.
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
                };
                // O_x (+)= P_x V(j): P from tensor memory (packed bf16 over the
                // first 64 columns of S_x), 16 keys per MMA
                auto issue_pv = [&](int x, int j, int vslot) {
                    const int valid = wk.S_len - j * TILE;
                    const uint32_t p_tmem = tmem + x * 128;
                    const uint32_t o_tmem = tmem + 256 + x * 128;
                    const uint64_t vd = v_desc0 + (uint32_t)vslot * kTileDesc;
                    if (valid >= TILE)
                    {
                        if (j == 0)
                            umma_bf16_tmem_a_i<0>(o_tmem, p_tmem, vd, IDESC_O);
                        else
                            umma_bf16_tmem_a_i<1>(o_tmem, p_tmem, vd, IDESC_O);
#pragma unroll
                        for (int k = 1; k < TILE / 16; k++)
                            umma_bf16_tmem_a_i<1>(o_tmem, p_tmem + k * 8, vd + ((k * 16 * 128) >> 4), IDESC_O);
                    }
                    else
                    {
                        const int ksteps = (valid + 15) / 16;
                        for (int k = 0; k < ksteps; k++)
                            umma_bf16_tmem_a(o_tmem, p_tmem + k * 8, vd + ((k * 16 * 128) >> 4), IDESC_O,
                                             (j | k) != 0);
                    }
                };
                auto wait_k = [&](int g_) {
                    return mbar_wait(&k_full[g_ % K_STAGES], (uint32_t)(g_ / K_STAGES) & 1u, abort_flag, args.status);
                };
                if (!mbar_wait(q_full, it & 1, abort_flag, args.status) || !wait_k(gk))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int x = 0; x < ntiles; x++)
                {
                    issue_s(x, gk, 0);
                    umma_commit(&s_full[x]);
                }
                any = true;
                umma_commit(&k_empty[gk % K_STAGES]);
                gk++;
                if (wk.nkv == 1) umma_commit(q_empty);
                for (int j = 0; j < wk.nkv && ok; j++)
                {
                    const int vs = gv % V_STAGES;
                    if (!mbar_wait(&v_full[vs], (uint32_t)(gv / V_STAGES) & 1u, abort_flag, args.status))
                    {
                        ok = false;
                        break;
                    }
                    const bool more = j + 1 < wk.nkv;
                    if (more && !wait_k(gk))
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
                        issue_pv(x, j, vs);
                        if (x == ntiles - 1) umma_commit(&v_empty[vs]);
                        if (more)
                        {
                            issue_s(x, gk, j + 1);
                            umma_commit(&s_full[x]);
                        }
                        else
                            umma_commit(&o_done[x]);
                    }
                    if (!ok) break;
                    gv++;
                    if (more)
                    {
                        umma_commit(&k_empty[gk % K_STAGES]);
                        gk++;
                        if (j + 2 == wk.nkv) umma_commit(q_empty); // the unit's last S MMAs
                    }
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
        // ---------------- softmax + epilogue (warps 0-3: tile 0, 4-7: tile 1)
        regs_increase<SOFTMAX_REGS>();
        const int x = warp >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const uint32_t s_addr = tmem + lane_base + x * 128;
        const uint32_t o_addr = tmem + lane_base + 256 + x * 128;
        uint32_t scnt = 0, ocnt = 0;
        bool ok = true;
        // each unit's descriptor is read one unit ahead (its loads are in
        // flight while the current unit runs)
        Work nwk = decode_work(args, blockIdx.x < args.num_work ? blockIdx.x : 0);
        for (int w = blockIdx.x; w < args.num_work && ok; w += gridDim.x)
        {
            const Work wk = nwk;
            if (w + (int)gridDim.x < args.num_work) nwk = decode_work(args, w + gridDim.x);
            if (x == 1 && !wk.has_b) continue;
            const int qbase = wk.q0 + x * TILE;
            const int qi = qbase + row;
            const int target = row_target(args, wk.window, wk.part_off, wk.L, wk.S_len, qi);
            float m_used = -INFINITY;
            float l_run = 0.f;
            // only the last key tile can be ragged; it runs after the loop so
            // the two forms of the softmax never share a register allocation
            const int last_valid = wk.S_len - (wk.nkv - 1) * TILE;
            const int nfull = last_valid == TILE ? wk.nkv : wk.nkv - 1;
            auto wait_s = [&]() {
                if (!warp_wait(&s_full[x], scnt & 1, abort_flag, args.status)) return false;
                scnt++;
                tc_fence_after();
                return true;
            };
            // P_x (and any rescaled O_x) written: the PV MMA may read them
            auto release_p = [&]() {
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[x]);
            };
            for (int j = 0; j < nfull; j++)
            {
                if (!wait_s())
                {
                    ok = false;
                    break;
                }
                softmax_tile<true>(s_addr, o_addr, TILE, j == 0, args.scale_log2, m_used, l_run);
                release_p();
            }
            if (!ok) break;
            if (nfull < wk.nkv)
            {
                if (!wait_s())
                {
                    ok = false;
                    break;
                }
                softmax_tile<false>(s_addr, o_addr, last_valid, nfull == 0, args.scale_log2, m_used, l_run);
                release_p();
            }
            if (!warp_wait(&o_done[x], ocnt & 1, abort_flag, args.status))
            {
                ok = false;
                break;
            }
            ocnt++;
            tc_fence_after();
            const float inv = 1.f / l_run;
            bool remote = false;
            {
                // the whole O row in one batch of tensor-memory loads
                uint32_t v[128];
                tmem_ld32_at<0>(o_addr, v);
                tmem_ld32_at<32>(o_addr + 32, v);
                tmem_ld32_at<64>(o_addr + 64, v);
                tmem_ld32_at<96>(o_addr + 96, v);
                tmem_ld_wait();
                if (target >= 0)
                {
                    const bool video = qi < wk.L;
#pragma unroll
                    for (int c = 0; c < 4; c++)
                        remote |= store_row(args, video, target, wk.head * HD + c * 32,
                                            reinterpret_cast<const float*>(v) + c * 32, inv);
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
    if (warp == 9) tmem_dealloc(tmem, TMEM_COLS);
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
    if (first_on_device(configured))
    {
        // The register split assumes exactly LAUNCH_REGS per thread at launch
        // (a different count would leave the softmax warps' increase waiting).
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, window_attention_kernel) != cudaSuccess || fa.numRegs != LAUNCH_REGS)
            return S2_ERR_CUDA;
        if (cudaFuncSetAttribute(window_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
            return S2_ERR_CUDA;
    }
    a.heads = heads;
    a.num_work = s.num_items * heads;
    a.num_video_indices = s.num_video_indices;
    a.out_rows = s.out_rows;
    a.partial_rows = s.partial_rows;
    a.num_peers = num_peers;
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
