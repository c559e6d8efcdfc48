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
//     thread) and apply bias and the fused epilogue (store, GELU-tanh, or
//     gate * acc + fp32 residual);
//   * every mbarrier wait is bounded (s2_common.cuh) and unwinds the CTA.
#include "s2_common.cuh"
#include "s2_internal.h"

namespace s2 {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int A_BYTES = BM * BK * 2;
constexpr int GROUP_M = 16;
constexpr int NUM_THREADS = 192; // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue

// Tile width BN (256, or 128 when a problem has too few 256-wide tiles to
// fill the SMs evenly): 192 KB of stages either way.
template <int BN>
struct Tile
{
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN, 0, 0);
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
};

struct GemmArgs
{
    int M0, M1, N, K;
    int mblk0, mblk1, nblk, num_tiles, num_kb;
    int epilogue;
    int out_f32;
    const float* bias;
    const float* gate;
    void* out0;
    void* out1;
    int* status;
};

template <int BN>
__device__ __forceinline__ void decode_tile(const GemmArgs& a, int t, int& stream, int& m0, int& n0)
{
    const int mb_total = a.mblk0 + a.mblk1;
    const int per_group = GROUP_M * a.nblk;
    const int g = t / per_group;
    const int first_m = g * GROUP_M;
    const int gm = min(GROUP_M, mb_total - first_m);
    const int r = t - g * per_group;
    const int mb = first_m + r % gm;
    const int nb = r / gm;
    stream = mb < a.mblk0 ? 0 : 1;
    m0 = (stream ? mb - a.mblk0 : mb) * BM;
    n0 = nb * BN;
}

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

template <int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    shared_linear_kernel(const __grid_constant__ CUtensorMap tmap_a0, const __grid_constant__ CUtensorMap tmap_a1,
                         const __grid_constant__ CUtensorMap tmap_w, const GemmArgs args)
{
    constexpr int STAGES = Tile<BN>::STAGES;
    constexpr int STAGE_BYTES = Tile<BN>::STAGE_BYTES;
    constexpr int TMEM_COLS = Tile<BN>::TMEM_COLS;
    constexpr uint32_t IDESC = Tile<BN>::IDESC;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
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
            mbar_init(&tempty[b], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&tmap_a0);
        tma_prefetch_desc(&tmap_a1);
        tma_prefetch_desc(&tmap_w);
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
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, args.status)) break;
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
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, args.status)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                bool ok = true;
                for (int kb = 0; kb < args.num_kb; kb++)
                {
                    if (!mbar_wait(&full[stage], phase, abort_flag, args.status))
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
        const int row_in_tile = quarter * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < args.num_tiles; t += gridDim.x)
        {
            int ok = 0;
            if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, args.status) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            __syncwarp();
            tc_fence_after();
            int stream, m0, n0;
            decode_tile<BN>(args, t, stream, m0, n0);
            const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
            for (int c = 0; c < BN / 32; c++)
            {
                uint32_t v[32];
                tmem_ld32(t_row + c * 32, v);
                tmem_ld_wait();
                if (n0 + c * 32 < args.N) epilogue_chunk(args, stream, m0 + row_in_tile, n0 + c * 32, v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
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

    CUtensorMap ta0, ta1, tw;
    int r = make_tmap_bf16_2d(&ta0, A0, K, M0 > 0 ? M0 : 1, (uint64_t)K * 2, BK, BM);
    if (r == 0) r = make_tmap_bf16_2d(&ta1, M1 > 0 ? A1 : A0, K, M1 > 0 ? M1 : (M0 > 0 ? M0 : 1), (uint64_t)K * 2, BK, BM);
    if (r == 0) r = make_tmap_bf16_2d(&tw, W, K, N, (uint64_t)K * 2, BK, 256);
    if (r != 0) return r;

    GemmArgs a;
    a.M0 = M0;
    a.M1 = M1;
    a.N = N;
    a.K = K;
    a.mblk0 = (M0 + BM - 1) / BM;
    a.mblk1 = (M1 + BM - 1) / BM;
    a.num_kb = (K + BK - 1) / BK;
    a.epilogue = epilogue;
    a.out_f32 = out_f32;
    a.bias = bias;
    a.gate = gate;
    a.out0 = out0;
    a.out1 = out1;
    a.status = ctx.status;

    // Tile width: 128 when it fills the SMs markedly more evenly than 256.
    auto wave_eff = [&](int bn) {
        const int tiles = (a.mblk0 + a.mblk1) * ((N + bn - 1) / bn);
        const int waves = (tiles + ctx.num_sms - 1) / ctx.num_sms;
        return (double)tiles / ((double)waves * ctx.num_sms);
    };
    const bool narrow = wave_eff(128) > 1.15 * wave_eff(256);
    const int BNsel = narrow ? 128 : 256;
    a.nblk = (N + BNsel - 1) / BNsel;
    a.num_tiles = (a.mblk0 + a.mblk1) * a.nblk;
    if (narrow && (r = make_tmap_bf16_2d(&tw, W, K, N, (uint64_t)K * 2, BK, 128)) != 0) return r;
    static bool configured[2] = {false, false};
    if (!configured[narrow])
    {
        const cudaError_t e =
            narrow ? cudaFuncSetAttribute(shared_linear_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          Tile<128>::SMEM_BYTES)
                   : cudaFuncSetAttribute(shared_linear_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          Tile<256>::SMEM_BYTES);
        if (e != cudaSuccess) return S2_ERR_CUDA;
        configured[narrow] = true;
    }
    const int grid = a.num_tiles < ctx.num_sms ? a.num_tiles : ctx.num_sms;
    const double M = (double)M0 + M1;
    const double out_bytes = epilogue == EPI_GATE_RESIDUAL ? 8.0 : (out_f32 ? 4.0 : 2.0);
    ProfileScope prof(ctx, K_GEMM, 2.0 * M * N * K, (M * K + (double)N * K) * 2.0 + M * N * out_bytes);
    if (narrow)
        shared_linear_kernel<128><<<grid, NUM_THREADS, Tile<128>::SMEM_BYTES, ctx.stream>>>(ta0, ta1, tw, a);
    else
        shared_linear_kernel<256><<<grid, NUM_THREADS, Tile<256>::SMEM_BYTES, ctx.stream>>>(ta0, ta1, tw, a);
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

} // namespace s2
