// VAE DecomposedConv3D on sm_100a: the causal 3-D convolution of
// DecomposedConv3D::forward (decomposed_conv3d.cpp:605-765) as ONE implicit
// GEMM per call instead of kernel_t spatial convolutions and a frame
// accumulation.
//
//   out[co][t][y][x] = bias[co] + sum_{kt, ky, kx, ci} W[co][kt][ky][kx][ci] *
//                      X[t*st + kt*dt][y*sh + ky*dh - ph][x*sw + kx*dw - pw][ci]
//
// X is the layer input with its head frames materialised (the cached frames
// of the previous chunk, or copies of frame 0), stored channels-last in bf16
// ([frames][H][W][Cp], Cp = channels rounded up to 8) by conv_pack_kernel.
// A tile is 128 output pixels (a 128 x 1, 64 x 2 or 32 x 4 block of one
// output frame, whichever pads the frame least) times 128 output channels;
// its K loop walks the taps (kt, ky, kx) and 64-channel blocks.  Warp 0 TMA-
// loads the A box straight out of X with a 4-D tensor map at the tap's
// shifted coordinates (zero padding comes from the out-of-range fill; a
// spatial stride sw is the box's traversal stride along x) and the matching
// 128 x 64 weight box; warp 1 issues tcgen05.mma (128 x 128 x 16,
// bf16 -> fp32) into one of two TMEM accumulators; warps 2-5 add the bias and
// store the tile into the planar fp32 output (ncnn's [c][d][h][w] blob: for
// each output channel a warp writes 32 consecutive pixels, 128 bytes).
// Every mbarrier wait is bounded and unwinds the CTA.
#include "s2_common.cuh"
#include "s2_internal.h"

namespace s2 {

namespace {

constexpr int CBM = 128;                          // output pixels per tile: bx x by, bx * by = 128
constexpr int CBN = 128;                          // output channels per tile
constexpr int CBK = 64;                           // input channels per K block (one 128-byte swizzle row)
constexpr int C_A_BYTES = CBM * CBK * 2;
constexpr int C_STAGE_BYTES = C_A_BYTES + CBN * CBK * 2;
constexpr int C_STAGES = 6;
constexpr int C_THREADS = 192;                    // TMA, MMA, 4 epilogue warps
constexpr int C_TMEM_COLS = 2 * CBN;              // two accumulators
constexpr uint32_t C_IDESC = umma_idesc_bf16(CBM, CBN, 0, 0);
constexpr int C_SMEM = C_STAGES * C_STAGE_BYTES + 1024 + 256;
constexpr int kPackTiles = 4; // 32-pixel tiles per conv_pack_kernel block

struct ConvArgs
{
    int Tout, Ho, Wo, Co;
    int bx, by;                    // tile extent in output pixels (x, y), bx * by = CBM
    int xblocks, yblocks, nblocks, num_tiles;
    int kh, kw, st, dt, sh, sw, dh, dw, ph, pw;
    int cblocks, num_kb, cpad64;
    const float* bias;
    float* out;
    int64_t out_cstep;
    int* status;
};

// tile -> (output frame, first row, first pixel, first channel); channel
// blocks run fastest so the tiles of one pixel block reuse its input in L2
__device__ __forceinline__ void conv_decode(const ConvArgs& a, int t, int& to, int& y0, int& x0, int& n0)
{
    const int nb = t % a.nblocks;
    int r = t / a.nblocks;
    const int xb = r % a.xblocks;
    r /= a.xblocks;
    const int yb = r % a.yblocks;
    to = r / a.yblocks;
    x0 = xb * a.bx;
    y0 = yb * a.by;
    n0 = nb * CBN;
}

__device__ __forceinline__ void conv_drain(uint64_t* bar, uint32_t parity)
{
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_timer_ns() - t0 > kWaitLimitNs) break;
}

__global__ void __launch_bounds__(C_THREADS, 1)
    conv3d_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                  const ConvArgs args)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_STAGES * C_STAGE_BYTES);
    uint64_t* empty = full + C_STAGES;
    uint64_t* tfull = empty + C_STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0)
    {
        for (int s = 0; s < C_STAGES; s++)
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
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    if (warp == 1) tmem_alloc(tmem_slot, C_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int taps_hw = args.kh * args.kw;

    if (warp == 0)
    {
        if (lane == 0)
        {
            // ---------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            int issued[C_STAGES];
            uint32_t last_phase[C_STAGES];
            for (int s = 0; s < C_STAGES; s++) issued[s] = 0, last_phase[s] = 0;
            for (int t = blockIdx.x; t < args.num_tiles && !*abort_flag; t += gridDim.x)
            {
                int to, y0, x0, n0;
                conv_decode(args, t, to, y0, x0, n0);
                int tap = 0, cb = 0;
                for (int kb = 0; kb < args.num_kb; kb++)
                {
                    if (!mbar_wait<true>(&empty[stage], phase ^ 1, abort_flag, args.status)) break;
                    const int k_t = tap / taps_hw, rem = tap - k_t * taps_hw;
                    const int k_y = rem / args.kw, k_x = rem - k_y * args.kw;
                    uint8_t* sa = smem + stage * C_STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], C_STAGE_BYTES);
                    tma_load_4d(sa, &tmap_x, &full[stage], cb * CBK, x0 * args.sw + k_x * args.dw - args.pw,
                                y0 * args.sh + k_y * args.dh - args.ph, to * args.st + k_t * args.dt);
                    tma_load_2d(sa + C_A_BYTES, &tmap_w, &full[stage], tap * args.cpad64 + cb * CBK, n0);
                    issued[stage] = 1;
                    last_phase[stage] = phase;
                    if (++cb == args.cblocks)
                    {
                        cb = 0;
                        tap++;
                    }
                    if (++stage == C_STAGES)
                    {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag)
                for (int s = 0; s < C_STAGES; s++)
                    if (issued[s]) conv_drain(&full[s], last_phase[s]);
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
                const uint32_t d_tmem = tmem_base + acc * CBN;
                bool ok = true;
                for (int kb = 0; kb < args.num_kb; kb++)
                {
                    if (!mbar_wait<true>(&full[stage], phase, abort_flag, args.status))
                    {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * C_STAGE_BYTES);
                    const uint32_t b_addr = a_addr + C_A_BYTES;
#pragma unroll
                    for (int k = 0; k < CBK / 16; k++)
                    {
                        const uint64_t ad = umma_desc_sw128(a_addr + k * 32, 16, 1024);
                        const uint64_t bd = umma_desc_sw128(b_addr + k * 32, 16, 1024);
                        umma_bf16(d_tmem, ad, bd, C_IDESC, (kb | k) != 0);
                    }
                    umma_commit(&empty[stage]);
                    any = true;
                    if (++stage == C_STAGES)
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
                umma_commit(drain);
                conv_drain(drain, 0);
            }
        }
    }
    else
    {
        // ---------------- epilogue (warps 2..5): one output pixel per thread
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
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
            int to, y0, x0, n0;
            conv_decode(args, t, to, y0, x0, n0);
            // accumulator row = the box's (y, x) order; a warp's 32 rows are 32
            // consecutive pixels of one output row (bx >= 32)
            const int y = y0 + row / args.bx, x = x0 + row % args.bx;
            const bool live = x < args.Wo && y < args.Ho;
            float* dst = args.out + ((int64_t)to * args.Ho + y) * args.Wo + x;
            const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * CBN;
#pragma unroll 1
            for (int c = 0; c < CBN / 32; c++)
            {
                uint32_t v[32];
                tmem_ld32(t_row + c * 32, v);
                tmem_ld_wait();
                const int cbase = n0 + c * 32;
#pragma unroll
                for (int j = 0; j < 32; j++)
                {
                    const int co = cbase + j;
                    if (co < args.Co && live)
                    {
                        const float b = args.bias ? __ldg(args.bias + co) : 0.f;
                        dst[(int64_t)co * args.out_cstep] = __uint_as_float(v[j]) + b;
                    }
                }
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
    if (warp == 1) tmem_dealloc(tmem_base, C_TMEM_COLS);
}

// Channels-last bf16 frames of the padded input: frame f of X is input frame
// f - prefix (planar fp32 [c][d][h][w], plane stride in_cstep), or input frame
// 0 for f < prefix when there is no cached memory (the reference's head);
// channels [C, Cp) are zero.  A block moves 32 pixels x 64 channels through
// shared memory: it reads 128-byte runs of each channel plane and writes each
// pixel's 64 channels as 16-byte stores (one 128-byte run per pixel).
__global__ void __launch_bounds__(256) conv_pack_kernel(const float* __restrict__ in, int64_t in_cstep, int C,
                                                        int Cp, int HW, int frame0, int prefix,
                                                        __nv_bfloat16* __restrict__ X)
{
    __shared__ float tile[64][33];
    const int c0 = blockIdx.y * 64;
    const int f = frame0 + blockIdx.z; // frame of X
    const int src_frame = f < prefix ? 0 : f - prefix;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5; // 32 x 8
    const int px = threadIdx.x >> 3, grp = threadIdx.x & 7; // 32 pixels x 8 groups of 8 channels
    // kPackTiles consecutive 32-pixel tiles per block
    for (int k = 0; k < kPackTiles; k++)
    {
        const int p0 = (blockIdx.x * kPackTiles + k) * 32;
        if (p0 >= HW) break;
        if (k) __syncthreads(); // the previous tile has been read out
        for (int i = ty; i < 64; i += 8)
        {
            const int c = c0 + i, p = p0 + tx;
            tile[i][tx] = (c < C && p < HW) ? __ldg(in + (int64_t)c * in_cstep + (int64_t)src_frame * HW + p) : 0.f;
        }
        __syncthreads();
        const int p = p0 + px, c = c0 + grp * 8;
        if (p < HW && c < Cp)
        {
            uint4 u;
            u.x = pack_bf16x2(tile[grp * 8 + 0][px], tile[grp * 8 + 1][px]);
            u.y = pack_bf16x2(tile[grp * 8 + 2][px], tile[grp * 8 + 3][px]);
            u.z = pack_bf16x2(tile[grp * 8 + 4][px], tile[grp * 8 + 5][px]);
            u.w = pack_bf16x2(tile[grp * 8 + 6][px], tile[grp * 8 + 7][px]);
            *reinterpret_cast<uint4*>(X + ((int64_t)f * HW + p) * Cp + c) = u;
        }
    }
}

// VAEUpsample3D's shuffle (vae_upsample3d.cpp:274-318): output channel c,
// frame t, pixel (Y, X) of [ch][out_t][ph*sr][pw*sr] takes packed channel
// ((Y % sr * sr + X % sr) * tr + z) * ch + c, frame s / tr, pixel (Y / sr,
// X / sr), where s = t, or t + 1 past frame 0 when frame 1 is dropped
// (remove_head).  One output element per thread, writes coalesced.
__global__ void upsample_shuffle_kernel(const float* __restrict__ packed, int64_t pcstep, int ch, int tr, int sr,
                                        int ph, int pw, int out_t, int remove_head, float* __restrict__ out,
                                        int64_t ocstep)
{
    const int OW = pw * sr, OH = ph * sr;
    const int64_t per_c = (int64_t)out_t * OH * OW;
    const int64_t total = per_c * ch;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    {
        const int c = (int)(i / per_c);
        int64_t r = i - (int64_t)c * per_c;
        const int t = (int)(r / ((int64_t)OH * OW));
        r -= (int64_t)t * OH * OW;
        const int Y = (int)(r / OW), X = (int)(r - (int64_t)Y * OW);
        const int s = (remove_head && t >= 1) ? t + 1 : t;
        const int frame = s / tr, z = s - frame * tr;
        const int pc = (((Y % sr) * sr + X % sr) * tr + z) * ch + c;
        out[(int64_t)c * ocstep + r + (int64_t)t * OH * OW] =
            __ldg(packed + (int64_t)pc * pcstep + ((int64_t)frame * ph + Y / sr) * pw + X / sr);
    }
}

} // namespace

int conv3d_pack(Context& ctx, const float* in, int64_t in_cstep, int C, int Cp, int HW, int frame0, int frames,
                int prefix, void* X)
{
    if (frames <= 0) return S2_OK;
    if (Cp % 8 || (reinterpret_cast<uintptr_t>(X) & 15)) return S2_ERR_INVALID;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)frames * HW * (C * 4.0 + Cp * 2.0));
    const dim3 grid((HW + 32 * kPackTiles - 1) / (32 * kPackTiles), (Cp + 63) / 64, frames);
    conv_pack_kernel<<<grid, 256, 0, ctx.stream>>>(in, in_cstep, C, Cp, HW, frame0, prefix,
                                                   static_cast<__nv_bfloat16*>(X));
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

int conv3d_gemm(Context& ctx, const Conv3dGeometry& g, const void* X, int frames_x, const void* Wt, const float* bias,
                float* out, int64_t out_cstep)
{
    // Output tile of bx x by = 128 pixels, the shape among 128 x 1, 64 x 2 and
    // 32 x 4 that leaves the fewest padding pixels on this frame (a 160-pixel
    // row takes five 32-wide tiles instead of two 128-wide ones).
    int bx = CBM, by = 1;
    {
        double best = 0.0;
        for (int cx = CBM; cx >= 32; cx /= 2)
        {
            const int cy = CBM / cx;
            const double used = (double)g.Wo * g.Ho /
                                ((double)((g.Wo + cx - 1) / cx) * cx * (double)((g.Ho + cy - 1) / cy) * cy);
            if (used > best + 1e-9)
            {
                best = used;
                bx = cx;
                by = cy;
            }
        }
    }
    // A: X [frames][H][W][Cp] bf16, boxes of 64 channels x bx pixels x by rows;
    // spatial strides are the box's traversal strides (sw * bx pixels wide,
    // sh * by rows high, every sw-th / sh-th one read)
    CUtensorMap tx, tw;
    const uint64_t xd[4] = {(uint64_t)g.Cp, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)frames_x};
    const uint64_t xs[3] = {(uint64_t)g.Cp * 2, (uint64_t)g.W * g.Cp * 2, (uint64_t)g.H * g.W * g.Cp * 2};
    if (g.sw < 1 || g.sh < 1 || bx * g.sw > 256 || by * g.sh > 256 || g.sw > 8 || g.sh > 8) return S2_ERR_INVALID;
    const uint32_t xb[4] = {CBK, (uint32_t)(bx * g.sw), (uint32_t)(by * g.sh), 1};
    const uint32_t xe[4] = {1, (uint32_t)g.sw, (uint32_t)g.sh, 1};
    int r = make_tmap_bf16_4d(&tx, X, xd, xs, xb, xe);
    // B: weights [Co][taps * cpad64] bf16, boxes of 64 x 128
    const int taps = g.kt * g.kh * g.kw;
    if (r == S2_OK)
        r = make_tmap_bf16_2d(&tw, Wt, (uint64_t)taps * g.cpad64, (uint64_t)g.Co, (uint64_t)taps * g.cpad64 * 2, CBK,
                              CBN);
    if (r != S2_OK) return r;
    ConvArgs a;
    a.Tout = g.Tout;
    a.Ho = g.Ho;
    a.Wo = g.Wo;
    a.Co = g.Co;
    a.bx = bx;
    a.by = by;
    a.xblocks = (g.Wo + bx - 1) / bx;
    a.yblocks = (g.Ho + by - 1) / by;
    a.nblocks = (g.Co + CBN - 1) / CBN;
    a.num_tiles = g.Tout * a.yblocks * a.xblocks * a.nblocks;
    a.kh = g.kh;
    a.kw = g.kw;
    a.st = g.st;
    a.dt = g.dt;
    a.sh = g.sh;
    a.sw = g.sw;
    a.dh = g.dh;
    a.dw = g.dw;
    a.ph = g.ph;
    a.pw = g.pw;
    a.cpad64 = g.cpad64;
    a.cblocks = g.cpad64 / CBK;
    a.num_kb = taps * a.cblocks;
    a.bias = bias;
    a.out = out;
    a.out_cstep = out_cstep;
    a.status = ctx.status;
    if (a.num_tiles <= 0) return S2_OK;
    static std::atomic<uint64_t> configured{0};
    if (first_on_device(configured) &&
        cudaFuncSetAttribute(conv3d_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C_SMEM) != cudaSuccess)
        return S2_ERR_CUDA;
    const int grid = a.num_tiles < ctx.num_sms ? a.num_tiles : ctx.num_sms;
    const double flops = 2.0 * g.Tout * g.Ho * g.Wo * (double)g.Co * taps * g.Ci;
    ProfileScope prof(ctx, K_GEMM, flops,
                      (double)frames_x * g.H * g.W * g.Cp * 2.0 + (double)g.Co * taps * g.cpad64 * 2.0 +
                          (double)g.Tout * g.Ho * g.Wo * g.Co * 4.0);
    conv3d_kernel<<<grid, C_THREADS, C_SMEM, ctx.stream>>>(tx, tw, a);
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

} // namespace s2

// ---------------------------------------------------------------- C ABI
#include <vector>

#include "s2_objects.h"

struct s2_conv3d
{
    s2_context* ctx = nullptr;
    int cfg[16];
    s2::Conv3dGeometry geo; // static part (channels, kernel, strides, pads)
    void* wt = nullptr;     // bf16 [Co][kt][kh][kw][cpad64]
    float* bias = nullptr;  // [Co] or null
    s2::DeviceBuffer x;     // padded input, channels-last bf16
    s2::DeviceBuffer mem;   // cached frames of the previous chunk, same layout
    int mem_frames = 0, mem_w = 0, mem_h = 0;
    // zero columns / rows appended on the right / bottom of every frame
    // (VAEDownsample3D's padding, vae_downsample3d.cpp:154-168); they are the
    // tensor map's out-of-range fill, never stored
    int pad_right = 0, pad_bottom = 0;
    ~s2_conv3d()
    {
        if (wt) cudaFree(wt);
        if (bias) cudaFree(bias);
    }
};

namespace {

// DecomposedConv3D's output extents (decomposed_conv3d.cpp:632-636 and the
// spatial Convolution's); prefix = cached frames or head_frames.
int conv3d_shape(const s2_conv3d* l, int w, int h, int d, int prefix, int& Tout, int& Ho, int& Wo)
{
    const s2::Conv3dGeometry& g = l->geo;
    const int padded = d + prefix, extent = g.dt * (g.kt - 1) + 1;
    if (w <= 0 || h <= 0 || d <= 0 || padded < extent) return S2_ERR_INVALID;
    Tout = (padded - extent) / g.st + 1;
    const int ew = w + l->pad_right + 2 * g.pw - (g.dw * (g.kw - 1) + 1);
    const int eh = h + l->pad_bottom + 2 * g.ph - (g.dh * (g.kh - 1) + 1);
    if (ew < 0 || eh < 0) return S2_ERR_INVALID;
    Wo = ew / g.sw + 1;
    Ho = eh / g.sh + 1;
    return S2_OK;
}

int conv3d_prefix(const s2_conv3d* l, int w, int h, int memory_state, bool& use_memory)
{
    use_memory = memory_state == S2_VAE_MEMORY_ACTIVE && l->mem_frames > 0;
    if (use_memory && (l->mem_w != w || l->mem_h != h)) return -1;
    return use_memory ? l->mem_frames : l->cfg[7];
}

} // namespace

extern "C" {

int s2_conv3d_create(s2_context* ctx, const int* cfg, const float* bias, const float* weights, s2_conv3d** out)
{
    if (!ctx || !cfg || !weights || !out) return S2_ERR_INVALID;
    *out = nullptr;
    // load_model's checks (decomposed_conv3d.cpp:437-442) and this build's limits
    const int co = cfg[0], ci = cfg[1], kw = cfg[2], kh = cfg[3], kt = cfg[4];
    if (co <= 0 || ci <= 0 || kw <= 0 || kh <= 0 || kt <= 0 || cfg[5] <= 0 || cfg[6] <= 0 || cfg[8] <= 0 ||
        cfg[9] <= 0 || cfg[10] <= 0 || cfg[11] <= 0 || cfg[14] <= 0 || ci % cfg[14] || co % cfg[14] || cfg[7] < 0)
        return S2_ERR_INVALID;
    if (cfg[14] != 1 || cfg[8] > 2 || cfg[12] < 0 || cfg[13] < 0 || (cfg[15] && !bias)) return S2_ERR_INVALID;
    s2::Context& c = ctx->c;
    if (cudaSetDevice(c.device) != cudaSuccess) return S2_ERR_CUDA;
    std::unique_ptr<s2_conv3d> l(new s2_conv3d);
    l->ctx = ctx;
    for (int i = 0; i < 16; i++) l->cfg[i] = cfg[i];
    s2::Conv3dGeometry& g = l->geo;
    g.Ci = ci;
    g.Cp = (ci + 7) & ~7;
    g.cpad64 = (ci + 63) & ~63;
    g.Co = co;
    g.kt = kt;
    g.kh = kh;
    g.kw = kw;
    g.st = cfg[5];
    g.dt = cfg[6];
    g.sh = cfg[9];
    g.sw = cfg[8];
    g.dw = cfg[10];
    g.dh = cfg[11];
    g.pw = cfg[12];
    g.ph = cfg[13];
    // weights kt x [co][ci][kh][kw] -> bf16 [co][kt][kh][kw][cpad64] (zero channel padding)
    const size_t taps = (size_t)kt * kh * kw, row = taps * g.cpad64;
    std::vector<__nv_bfloat16> w((size_t)co * row, __float2bfloat16(0.f));
    for (int t = 0; t < kt; t++)
        for (int o = 0; o < co; o++)
            for (int q = 0; q < ci; q++)
                for (int y = 0; y < kh; y++)
                    for (int x = 0; x < kw; x++)
                        w[(size_t)o * row + (((size_t)t * kh + y) * kw + x) * g.cpad64 + q] = __float2bfloat16(
                            weights[((((size_t)t * co + o) * ci + q) * kh + y) * kw + x]);
    if (cudaMalloc(&l->wt, w.size() * 2) != cudaSuccess)
    {
        l->wt = nullptr;
        return S2_ERR_ALLOC;
    }
    if (cudaMemcpy(l->wt, w.data(), w.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess) return S2_ERR_CUDA;
    if (cfg[15])
    {
        if (cudaMalloc(&l->bias, (size_t)co * 4) != cudaSuccess)
        {
            l->bias = nullptr;
            return S2_ERR_ALLOC;
        }
        if (cudaMemcpy(l->bias, bias, (size_t)co * 4, cudaMemcpyHostToDevice) != cudaSuccess) return S2_ERR_CUDA;
    }
    *out = l.release();
    return S2_OK;
}

int s2_conv3d_output_shape(const s2_conv3d* l, int w, int h, int d, int memory_state, int* out_whdc)
{
    if (!l || !out_whdc) return S2_ERR_INVALID;
    bool use_memory;
    const int prefix = conv3d_prefix(l, w, h, memory_state, use_memory);
    if (prefix < 0) return S2_ERR_INVALID;
    int Tout, Ho, Wo;
    const int r = conv3d_shape(l, w, h, d, prefix, Tout, Ho, Wo);
    if (r != S2_OK) return r;
    out_whdc[0] = Wo;
    out_whdc[1] = Ho;
    out_whdc[2] = Tout;
    out_whdc[3] = l->geo.Co;
    return S2_OK;
}

int s2_conv3d_forward(s2_conv3d* l, const float* in, int64_t in_cstep, int w, int h, int d, int c, int memory_state,
                      float* out, int64_t out_cstep)
{
    if (!l || !in || !out) return S2_ERR_INVALID;
    s2::Context& ctx = l->ctx->c;
    if (cudaSetDevice(ctx.device) != cudaSuccess) return S2_ERR_CUDA;
    // the memory is dropped unless the state is ACTIVE (decomposed_conv3d.cpp:609-611)
    if (memory_state != S2_VAE_MEMORY_ACTIVE) l->mem_frames = 0;
    if (c != l->geo.Ci || in_cstep < (int64_t)w * h * d) return S2_ERR_INVALID;
    bool use_memory;
    const int prefix = conv3d_prefix(l, w, h, memory_state, use_memory);
    if (prefix < 0) return S2_ERR_INVALID;
    s2::Conv3dGeometry g = l->geo;
    g.H = h;
    g.W = w;
    int r = conv3d_shape(l, w, h, d, prefix, g.Tout, g.Ho, g.Wo);
    if (r != S2_OK) return r;
    if (out_cstep < (int64_t)g.Tout * g.Ho * g.Wo) return S2_ERR_INVALID;
    const int padded = d + prefix;
    const size_t frame_bytes = (size_t)h * w * g.Cp * 2;
    if ((r = l->x.ensure(frame_bytes * padded)) != S2_OK) return r;
    if (use_memory)
    {
        if (cudaMemcpyAsync(l->x.ptr, l->mem.ptr, frame_bytes * prefix, cudaMemcpyDeviceToDevice, ctx.stream) !=
            cudaSuccess)
            return S2_ERR_CUDA;
        r = s2::conv3d_pack(ctx, in, in_cstep, g.Ci, g.Cp, h * w, prefix, d, prefix, l->x.ptr);
    }
    else
        r = s2::conv3d_pack(ctx, in, in_cstep, g.Ci, g.Cp, h * w, 0, padded, prefix, l->x.ptr);
    if (r == S2_OK) r = s2::conv3d_gemm(ctx, g, l->x.ptr, padded, l->wt, l->bias, out, out_cstep);
    if (r != S2_OK) return r;
    // cache the last kernel_t - stride_t padded frames (:733-764)
    const int cache = g.kt - g.st;
    if (memory_state != S2_VAE_MEMORY_DISABLED && cache > 0)
    {
        if (cache > padded) return S2_ERR_INVALID;
        if ((r = l->mem.ensure(frame_bytes * cache)) != S2_OK) return r;
        if (cudaMemcpyAsync(l->mem.ptr, static_cast<uint8_t*>(l->x.ptr) + frame_bytes * (padded - cache),
                            frame_bytes * cache, cudaMemcpyDeviceToDevice, ctx.stream) != cudaSuccess)
            return S2_ERR_CUDA;
        l->mem_frames = cache;
        l->mem_w = w;
        l->mem_h = h;
    }
    return S2_OK;
}

void s2_conv3d_reset_memory(s2_conv3d* l)
{
    if (l) l->mem_frames = 0;
}

void s2_conv3d_free(s2_conv3d* l)
{
    if (!l) return;
    cudaSetDevice(l->ctx->c.device);
    cudaStreamSynchronize(l->ctx->c.stream);
    delete l;
}

} // extern "C"

// ---------------------------------------------------------------- VAE resampling layers
struct s2_vae_resample
{
    s2_context* ctx = nullptr;
    int kind = 0;
    int channels = 0;
    int pad_right = 0, pad_bottom = 0;                   // downsample
    int tr = 1, sr = 1, remove_head = 0;                 // upsample
    s2_conv3d* conv = nullptr;                           // downsample conv / upsample post conv
    s2_conv3d* upscale = nullptr;                        // upsample
    s2::DeviceBuffer packed, shuffled;
    ~s2_vae_resample()
    {
        delete conv;
        delete upscale;
    }
};

namespace {

// One DecomposedConv3D out of a load_model blob: config (16), bias, kernels.
int conv_from_blob(s2_context* ctx, const float* blob, size_t count, size_t& off, s2_conv3d** out)
{
    if (off + 16 > count) return S2_ERR_INVALID;
    int cfg[16];
    for (int i = 0; i < 16; i++) cfg[i] = (int)blob[off + i];
    const size_t co = cfg[0] > 0 ? cfg[0] : 0, ci = cfg[1] > 0 ? cfg[1] : 0, kw = cfg[2] > 0 ? cfg[2] : 0,
                 kh = cfg[3] > 0 ? cfg[3] : 0, kt = cfg[4] > 0 ? cfg[4] : 0;
    size_t o = off + 16;
    const float* bias = nullptr;
    if (cfg[15])
    {
        bias = blob + o;
        o += co;
    }
    const size_t nw = kt * co * ci * kh * kw;
    if (o + nw > count) return S2_ERR_INVALID;
    const int r = s2_conv3d_create(ctx, cfg, bias, blob + o, out);
    off = o + nw;
    return r;
}

// upsample: output frames of the shuffle for `pd` packed frames
int shuffled_frames(const s2_vae_resample* l, int pd, int memory_state)
{
    const bool rm = l->remove_head && memory_state != S2_VAE_MEMORY_ACTIVE;
    return pd * l->tr - (rm ? 1 : 0);
}

} // namespace

extern "C" {

int s2_vae_resample_create(s2_context* ctx, int kind, const float* blob, size_t count, s2_vae_resample** out)
{
    if (!ctx || !blob || !out || (kind != S2_VAE_DOWNSAMPLE && kind != S2_VAE_UPSAMPLE)) return S2_ERR_INVALID;
    *out = nullptr;
    std::unique_ptr<s2_vae_resample> l(new s2_vae_resample);
    l->ctx = ctx;
    l->kind = kind;
    size_t off = 0;
    int r;
    if (kind == S2_VAE_DOWNSAMPLE)
    {
        // VAEDownsample3D::load_model (vae_downsample3d.cpp:98-112)
        if (count < 3) return S2_ERR_INVALID;
        l->channels = (int)blob[0];
        l->pad_right = (int)blob[1];
        l->pad_bottom = (int)blob[2];
        if (l->channels <= 0 || l->pad_right < 0 || l->pad_bottom < 0 || (l->pad_right == 0 && l->pad_bottom == 0))
            return S2_ERR_INVALID;
        off = 3;
        if ((r = conv_from_blob(ctx, blob, count, off, &l->conv)) != S2_OK) return r;
        l->conv->pad_right = l->pad_right;
        l->conv->pad_bottom = l->pad_bottom;
    }
    else
    {
        // VAEUpsample3D::load_model (vae_upsample3d.cpp:191-213): config, post conv, upscale conv
        if (count < 4) return S2_ERR_INVALID;
        l->channels = (int)blob[0];
        l->tr = (int)blob[1];
        l->sr = (int)blob[2];
        l->remove_head = (int)blob[3] != 0;
        if (l->channels <= 0 || (l->tr != 1 && l->tr != 2) || (l->sr != 1 && l->sr != 2) ||
            (l->remove_head != 0) != (l->tr == 2))
            return S2_ERR_INVALID;
        off = 4;
        if ((r = conv_from_blob(ctx, blob, count, off, &l->conv)) != S2_OK) return r;
        if ((r = conv_from_blob(ctx, blob, count, off, &l->upscale)) != S2_OK) return r;
    }
    *out = l.release();
    return S2_OK;
}

int s2_vae_resample_output_shape(const s2_vae_resample* l, int w, int h, int d, int memory_state, int* out_whdc)
{
    if (!l || !out_whdc) return S2_ERR_INVALID;
    if (l->kind == S2_VAE_DOWNSAMPLE) return s2_conv3d_output_shape(l->conv, w, h, d, memory_state, out_whdc);
    int p[4];
    int r = s2_conv3d_output_shape(l->upscale, w, h, d, memory_state, p);
    if (r != S2_OK) return r;
    const int t = shuffled_frames(l, p[2], memory_state);
    if (t <= 0) return S2_ERR_INVALID;
    return s2_conv3d_output_shape(l->conv, p[0] * l->sr, p[1] * l->sr, t, memory_state, out_whdc);
}

int s2_vae_resample_forward(s2_vae_resample* l, const float* in, int64_t in_cstep, int w, int h, int d, int c,
                            int memory_state, float* out, int64_t out_cstep)
{
    if (!l || !in || !out) return S2_ERR_INVALID;
    if (c != l->channels) return S2_ERR_INVALID;
    if (l->kind == S2_VAE_DOWNSAMPLE)
        return s2_conv3d_forward(l->conv, in, in_cstep, w, h, d, c, memory_state, out, out_cstep);
    s2::Context& ctx = l->ctx->c;
    if (cudaSetDevice(ctx.device) != cudaSuccess) return S2_ERR_CUDA;
    // the upscale conv drops its cached frames first, whatever fails later
    // (decomposed_conv3d.cpp:609-611)
    if (memory_state != S2_VAE_MEMORY_ACTIVE) s2_conv3d_reset_memory(l->upscale);
    int p[4];
    int r = s2_conv3d_output_shape(l->upscale, w, h, d, memory_state, p);
    if (r != S2_OK) return r;
    const int64_t pplane = (int64_t)p[0] * p[1] * p[2];
    if ((r = l->packed.ensure((size_t)pplane * p[3] * 4)) != S2_OK) return r;
    float* packed = static_cast<float*>(l->packed.ptr);
    if ((r = s2_conv3d_forward(l->upscale, in, in_cstep, w, h, d, c, memory_state, packed, pplane)) != S2_OK)
        return r;
    // checked after the upscale conv ran, as vae_upsample3d.cpp:268-272 does
    const int ratio = l->tr * l->sr * l->sr;
    if (p[3] != l->channels * ratio) return S2_ERR_INVALID;
    const int ot = shuffled_frames(l, p[2], memory_state);
    if (ot <= 0) return S2_ERR_INVALID;
    const int OW = p[0] * l->sr, OH = p[1] * l->sr;
    const int64_t splane = (int64_t)OW * OH * ot;
    if ((r = l->shuffled.ensure((size_t)splane * l->channels * 4)) != S2_OK) return r;
    float* sh = static_cast<float*>(l->shuffled.ptr);
    {
        const int64_t total = splane * l->channels;
        int64_t blocks = (total + 255) / 256;
        if (blocks > (int64_t)ctx.num_sms * 16) blocks = (int64_t)ctx.num_sms * 16;
        s2::ProfileScope prof(ctx, s2::K_OTHER, 0.0, (double)total * 8.0);
        s2::upsample_shuffle_kernel<<<(int)blocks, 256, 0, ctx.stream>>>(packed, pplane, l->channels, l->tr, l->sr,
                                                                        p[1], p[0], ot,
                                                                        l->remove_head && memory_state !=
                                                                                              S2_VAE_MEMORY_ACTIVE,
                                                                        sh, splane);
        ctx.launches++;
        if (cudaGetLastError() != cudaSuccess) return S2_ERR_CUDA;
    }
    return s2_conv3d_forward(l->conv, sh, splane, OW, OH, ot, l->channels, memory_state, out, out_cstep);
}

void s2_vae_resample_reset_memory(s2_vae_resample* l)
{
    if (!l) return;
    s2_conv3d_reset_memory(l->conv);
    s2_conv3d_reset_memory(l->upscale);
}

void s2_vae_resample_free(s2_vae_resample* l)
{
    if (!l) return;
    cudaSetDevice(l->ctx->c.device);
    cudaStreamSynchronize(l->ctx->c.stream);
    delete l;
}

} // extern "C"
