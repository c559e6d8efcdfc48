// HBM-bound passes of the block: QK-RMSNorm + 3-axis RoPE + window gather
// (prepare_qkv), the text-pool average over windows, AdaLN-style RMSNorm
// modulation, and small utilities.  All are 16-byte vectorised, one warp (or
// 16-lane group) per row, grids sized by rows.
#include "s2_common.cuh"
#include "s2_dist.h"
#include "s2_internal.h"

namespace s2 {

namespace {

// ---------------------------------------------------------------- prepare_qkv
// Replaces the prepare_qkv / prepare_qkv_split shaders
// (adaptive_window_attention.cpp:21-172, :178-333) and the CPU gather of
// :886-938: for packed row r (window w's video row or text row) and head h,
//   q = x_q * (1/sqrt(mean(x_q^2) + eps)) * w_q, same for k (video or text
//   weights), RoPE over 3 axes x `pairs` interleaved pairs at the row's
//   position (angle = pos[axis] * freq[pair]), v copied; all stored as bf16.
// One 16-lane group per (row, head): 8 consecutive dims per lane.
template <typename Tin>
__device__ __forceinline__ void load8(const Tin* p, float (&x)[8]);

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&x)[8])
{
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p + 4));
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
}

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&x)[8])
{
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    float2 f;
    f = unpack_bf16x2(u.x), x[0] = f.x, x[1] = f.y;
    f = unpack_bf16x2(u.y), x[2] = f.x, x[3] = f.y;
    f = unpack_bf16x2(u.z), x[4] = f.x, x[5] = f.y;
    f = unpack_bf16x2(u.w), x[6] = f.x, x[7] = f.y;
}

__device__ __forceinline__ void store8_bf16(__nv_bfloat16* p, const float (&x)[8])
{
    uint4 u;
    u.x = pack_bf16x2(x[0], x[1]);
    u.y = pack_bf16x2(x[2], x[3]);
    u.z = pack_bf16x2(x[4], x[5]);
    u.w = pack_bf16x2(x[6], x[7]);
    *reinterpret_cast<uint4*>(p) = u;
}

template <typename Tin>
__global__ void prepare_qkv_kernel(const int* __restrict__ row_src, const int* __restrict__ row_pos, int heads,
                                   int head_dim, int pairs, float eps, const float* __restrict__ norms,
                                   const float* __restrict__ freqs, const Tin* vq, const Tin* vk, const Tin* vv,
                                   int64_t v_ld, const Tin* tq, const Tin* tk, const Tin* tv, int64_t t_ld,
                                   __nv_bfloat16* qo, __nv_bfloat16* ko, __nv_bfloat16* vo, int src_rows,
                                   int text_rows, int* status)
{
    const int r = blockIdx.x;
    // The block is rounded up to whole warps; lanes past the last head work on
    // head 0 (in-bounds reads, full-warp shuffles) and store nothing.
    const bool active = (int)(threadIdx.x >> 4) < heads;
    const int h = active ? (int)(threadIdx.x >> 4) : 0;
    const int sub = threadIdx.x & 15;
    const int d0 = sub * 8;
    const int src = row_src[r];
    // (uniform over the block: every thread works on packed row r)
    if (!(src >= 0 ? index_ok(src, src_rows, status) : index_ok(-1 - (int64_t)src, text_rows, status))) return;
    const Tin *pq, *pk, *pv;
    const float *wq, *wk;
    if (src >= 0)
    {
        pq = vq + (int64_t)src * v_ld;
        pk = vk + (int64_t)src * v_ld;
        pv = vv + (int64_t)src * v_ld;
        wq = norms;
        wk = norms + head_dim;
    }
    else
    {
        const int t = -1 - src;
        pq = tq + (int64_t)t * t_ld;
        pk = tk + (int64_t)t * t_ld;
        pv = tv + (int64_t)t * t_ld;
        wq = norms + 2 * head_dim;
        wk = norms + 3 * head_dim;
    }
    const int off = h * head_dim + d0;
    float q[8], k[8], v[8];
    load8<Tin>(pq + off, q);
    load8<Tin>(pk + off, k);
    load8<Tin>(pv + off, v);
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++)
    {
        sq += q[i] * q[i];
        sk += k[i] * k[i];
    }
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1)
    {
        sq += __shfl_xor_sync(0xffffffffu, sq, m);
        sk += __shfl_xor_sync(0xffffffffu, sk, m);
    }
    const float inv_q = 1.f / sqrtf(sq / head_dim + eps);
    const float inv_k = 1.f / sqrtf(sk / head_dim + eps);
#pragma unroll
    for (int i = 0; i < 8; i++)
    {
        q[i] = q[i] * inv_q * __ldg(wq + d0 + i);
        k[i] = k[i] * inv_k * __ldg(wk + d0 + i);
    }
    const int axis_width = pairs * 2;
    const int p0 = __ldg(row_pos + r * 3), p1 = __ldg(row_pos + r * 3 + 1), p2 = __ldg(row_pos + r * 3 + 2);
#pragma unroll
    for (int i = 0; i < 8; i += 2)
    {
        const int d = d0 + i;
        if (d < axis_width * 3)
        {
            const int axis = d / axis_width;
            const int pair = (d - axis * axis_width) >> 1;
            const int pos = axis == 0 ? p0 : (axis == 1 ? p1 : p2);
            const float ang = (float)pos * __ldg(freqs + pair);
            float s, c;
            sincosf(ang, &s, &c);
            const float q0 = q[i], q1 = q[i + 1], k0 = k[i], k1 = k[i + 1];
            q[i] = q0 * c - q1 * s;
            q[i + 1] = q0 * s + q1 * c;
            k[i] = k0 * c - k1 * s;
            k[i + 1] = k0 * s + k1 * c;
        }
    }
    if (!active) return;
    const int64_t out = (int64_t)r * heads * head_dim + off;
    store8_bf16(qo + out, q);
    store8_bf16(ko + out, k);
    store8_bf16(vo + out, v);
}

// ---------------------------------------------------------------- text pool
// Replaces the text branch of the scatter (CPU :963-974, shader :395-407):
// text_out[t] = sum over the sample's windows of partial[w][t] * (1 / windows
// in sample).  A block covers 128 column quads of one text row with
// kTextPoolParts threads per quad: part g sums the g-th contiguous run of the
// windows in window order, and the parts are added in part order through
// shared memory -- a fixed order, so the result does not depend on the run,
// with four times the loads in flight of one thread per quad (the pass is
// bound by memory latency: 36-80 dependent rows per quad).
constexpr int kTextPoolParts = 4;
constexpr int kTextPoolQuads = 128;

__global__ void __launch_bounds__(kTextPoolQuads * kTextPoolParts)
    text_pool_kernel(const int4* __restrict__ reduce, const float* __restrict__ scale_of, int inner,
                     const float* __restrict__ partial, int out_f32, void* out, int partial_rows, int* status)
{
    __shared__ float4 part_sum[kTextPoolParts - 1][kTextPoolQuads];
    const int t = blockIdx.x;
    const int g = threadIdx.y;
    const int c = (blockIdx.y * kTextPoolQuads + threadIdx.x) * 4;
    const int4 rd = reduce[t];
    // every partial row summed lies in the partial buffer (first and last,
    // stride >= 0); the outcome is the same for the whole block
    if (rd.z > 0 && !(index_ok(rd.x, partial_rows, status) && rd.y >= 0 &&
                      index_ok(rd.x + (int64_t)(rd.z - 1) * rd.y, partial_rows, status)))
        return;
    const bool live = c < inner;
    const float sc = scale_of[t];
    // windows [w0, w1) of this part
    const int w0 = (int)((int64_t)rd.z * g / kTextPoolParts), w1 = (int)((int64_t)rd.z * (g + 1) / kTextPoolParts);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live)
    {
        const float* base = partial + (int64_t)rd.x * inner + c;
        const int64_t step = (int64_t)rd.y * inner;
        auto add = [&](const float4 p) {
            acc.x += p.x * sc;
            acc.y += p.y * sc;
            acc.z += p.z * sc;
            acc.w += p.w * sc;
        };
        // rounds of eight loads; the last round's surplus loads re-read the
        // part's last row and are replaced by zero before the add
        const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int i = w0; i < w1; i += 8)
        {
            float4 p[8];
#pragma unroll
            for (int k = 0; k < 8; k++)
                p[k] = __ldg(reinterpret_cast<const float4*>(base + min(i + k, w1 - 1) * step));
#pragma unroll
            for (int k = 0; k < 8; k++) add(i + k < w1 ? p[k] : zero);
        }
    }
    if (g > 0) part_sum[g - 1][threadIdx.x] = acc;
    __syncthreads();
    if (g > 0 || !live) return;
#pragma unroll
    for (int k = 0; k < kTextPoolParts - 1; k++)
    {
        const float4 q = part_sum[k][threadIdx.x];
        acc.x += q.x;
        acc.y += q.y;
        acc.z += q.z;
        acc.w += q.w;
    }
    if (out_f32)
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (int64_t)t * inner + c) = acc;
    else
    {
        uint2 u;
        u.x = pack_bf16x2(acc.x, acc.y);
        u.y = pack_bf16x2(acc.z, acc.w);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + (int64_t)t * inner + c) = u;
    }
}

// ---------------------------------------------------------------- ada_rmsnorm / ada_layernorm
// RMSNorm:   y = x * (1/sqrt(mean(x^2) + eps)) * scale + shift
// LayerNorm: y = (x - mean(x)) * (1/sqrt(var(x) + eps)) * scale + shift
// (no affine of their own; var the biased variance from the centred values)
// -> bf16; one warp per row.  For D = 256 G the row is held in registers (2G
// float4 per lane, each warp access 512 contiguous bytes) so x is read from
// HBM once -- LayerNorm adds one warp reduction for the mean -- and two
// 8-warp blocks fit per SM (128 registers) to keep 16 rows in flight; G = 0
// is the generic form for other widths (it re-reads the row).  Rows are taken
// last first: x was just written by a GEMM epilogue whose final tiles hold
// the highest rows, so those are still in L2 when this pass starts, and the
// rows it writes last (the lowest) are the ones the next GEMM reads first.
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

template <int G, bool LAYER>
__global__ void __launch_bounds__(256, 2)
    ada_norm_kernel(int rows, int D, const float* __restrict__ x, float eps, const float* __restrict__ shift,
                    const float* __restrict__ scale, __nv_bfloat16* __restrict__ y)
{
    const int row = rows - 1 - (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5));
    const int lane = threadIdx.x & 31;
    if (row < 0) return;
    const float* xr = x + (int64_t)row * D;
    __nv_bfloat16* yr = y + (int64_t)row * D;
    float mean = 0.f;
    if constexpr (G > 0)
    {
        // 2G float4 per lane; each warp access covers 512 contiguous bytes
        constexpr int Q = 2 * G;
        float4 v[Q];
#pragma unroll
        for (int q = 0; q < Q; q++) v[q] = __ldg(reinterpret_cast<const float4*>(xr + q * 128 + lane * 4));
        if (LAYER)
        {
            float s = 0.f;
#pragma unroll
            for (int q = 0; q < Q; q++) s += (v[q].x + v[q].y) + (v[q].z + v[q].w);
            mean = warp_sum(s) / D;
#pragma unroll
            for (int q = 0; q < Q; q++)
            {
                v[q].x -= mean;
                v[q].y -= mean;
                v[q].z -= mean;
                v[q].w -= mean;
            }
        }
        float ss = 0.f;
#pragma unroll
        for (int q = 0; q < Q; q++) ss += v[q].x * v[q].x + v[q].y * v[q].y + v[q].z * v[q].z + v[q].w * v[q].w;
        const float inv = 1.f / sqrtf(warp_sum(ss) / D + eps);
#pragma unroll
        for (int q = 0; q < Q; q++)
        {
            const int c = q * 128 + lane * 4;
            const float4 sc = __ldg(reinterpret_cast<const float4*>(scale + c));
            const float4 sh = __ldg(reinterpret_cast<const float4*>(shift + c));
            uint2 u;
            u.x = pack_bf16x2(v[q].x * inv * sc.x + sh.x, v[q].y * inv * sc.y + sh.y);
            u.y = pack_bf16x2(v[q].z * inv * sc.z + sh.z, v[q].w * inv * sc.w + sh.w);
            *reinterpret_cast<uint2*>(yr + c) = u;
        }
    }
    else
    {
        if (LAYER)
        {
            float s = 0.f;
            for (int c = lane * 8; c < D; c += 256)
            {
                float v[8];
                load8<float>(xr + c, v);
#pragma unroll
                for (int i = 0; i < 8; i++) s += v[i];
            }
            mean = warp_sum(s) / D;
        }
        float ss = 0.f;
        for (int c = lane * 8; c < D; c += 256)
        {
            float v[8];
            load8<float>(xr + c, v);
#pragma unroll
            for (int i = 0; i < 8; i++) ss += (v[i] - mean) * (v[i] - mean);
        }
        const float inv = 1.f / sqrtf(warp_sum(ss) / D + eps);
        for (int c = lane * 8; c < D; c += 256)
        {
            float v[8], sc[8], sh[8];
            load8<float>(xr + c, v);
            load8<float>(scale + c, sc);
            load8<float>(shift + c, sh);
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = (v[i] - mean) * inv * sc[i] + sh[i];
            store8_bf16(yr + c, v);
        }
    }
}

__global__ void convert_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, int64_t count)
{
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride)
        out[i] = __float2bfloat16_rn(in[i]);
}

// out[i] = a[i] + b[i % period] (per-block modulation = shared + offset).
__global__ void add_kernel(const float* a, const float* b, float* out, int count, int period)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) out[i] = a[i] + b[i % period];
}

// Counter-based normal samples (splitmix64 hash -> Box-Muller), deterministic
// for (seed, index).
__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float normal_at(uint64_t seed, int64_t i)
{
    const uint64_t h = mix64(seed * 0x100000001B3ull ^ mix64((uint64_t)i));
    const float u1 = ((uint32_t)(h >> 40) + 1.0f) * (1.0f / 16777217.0f); // (0,1]
    const float u2 = (uint32_t)(h & 0xFFFFFFu) * (1.0f / 16777216.0f);
    return sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
}

__global__ void fill_normal_bf16_kernel(__nv_bfloat16* out, int64_t count, uint64_t seed, float mean, float stddev)
{
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride)
        out[i] = __float2bfloat16_rn(mean + stddev * normal_at(seed, i));
}

__global__ void fill_normal_f32_kernel(float* out, int64_t count, uint64_t seed, float mean, float stddev)
{
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride)
        out[i] = mean + stddev * normal_at(seed, i);
}

// Row gather / scatter (16-byte vectors); one warp per row.
__global__ void gather_rows_kernel(const uint4* __restrict__ src, const int* __restrict__ idx, int count,
                                   int row_vecs, uint4* __restrict__ dst, int scatter)
{
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= count) return;
    const int r = __ldg(idx + row);
    const uint4* s = src + (int64_t)(scatter ? row : r) * row_vecs;
    uint4* d = dst + (int64_t)(scatter ? r : row) * row_vecs;
    for (int c = lane; c < row_vecs; c += 32) d[c] = __ldg(s + c);
}

inline int finish(Context& ctx)
{
    ctx.launches++;
    return cudaGetLastError() == cudaSuccess ? S2_OK : S2_ERR_CUDA;
}

inline bool aligned16(const void* p)
{
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

} // namespace

int launch_prepare_qkv(Context& ctx, const AttnSchedule& s, int heads, int head_dim, int rope_pairs, float eps,
                       const float* norms, const float* freqs, int in_bf16, const void* vq, const void* vk,
                       const void* vv, int64_t v_ld, const void* tq, const void* tk, const void* tv, int64_t t_ld,
                       void* q_out, void* k_out, void* v_out)
{
    if (head_dim != 128 || heads <= 0 || heads * 16 > 1024 || rope_pairs * 6 > head_dim) return S2_ERR_INVALID;
    const int esz = in_bf16 ? 2 : 4;
    // 16-byte vector loads need every row and head offset 16-byte aligned.
    if ((v_ld * esz) % 16 || (t_ld * esz) % 16 || !aligned16(vq) || !aligned16(vk) || !aligned16(vv) ||
        !aligned16(tq) || !aligned16(tk) || !aligned16(tv))
        return S2_ERR_INVALID;
    if (s.packed_rows == 0) return S2_OK;
    const dim3 grid(s.packed_rows), block((heads * 16 + 31) & ~31);
    ProfileScope prof(ctx, K_PREP, 0.0, (double)s.packed_rows * heads * head_dim * 3.0 * (esz + 2.0));
    if (in_bf16)
        prepare_qkv_kernel<__nv_bfloat16><<<grid, block, 0, ctx.stream>>>(
            s.row_src, s.row_pos, heads, head_dim, rope_pairs, eps, norms, freqs, (const __nv_bfloat16*)vq,
            (const __nv_bfloat16*)vk, (const __nv_bfloat16*)vv, v_ld, (const __nv_bfloat16*)tq,
            (const __nv_bfloat16*)tk, (const __nv_bfloat16*)tv, t_ld, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_out,
            (__nv_bfloat16*)v_out, s.src_rows, s.total_text, ctx.status);
    else
        prepare_qkv_kernel<float><<<grid, block, 0, ctx.stream>>>(
            s.row_src, s.row_pos, heads, head_dim, rope_pairs, eps, norms, freqs, (const float*)vq, (const float*)vk,
            (const float*)vv, v_ld, (const float*)tq, (const float*)tk, (const float*)tv, t_ld, (__nv_bfloat16*)q_out,
            (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out, s.src_rows, s.total_text, ctx.status);
    return finish(ctx);
}

int launch_text_pool(Context& ctx, const AttnSchedule& s, int inner, const float* partial, int out_f32,
                     int round_bf16, void* text_out)
{
    (void)round_bf16;
    if (s.total_text == 0) return S2_OK;
    if (inner % 4) return S2_ERR_INVALID;
    // 128 column quads per block: D = 2560 fills five blocks per text row exactly
    const dim3 block(kTextPoolQuads, kTextPoolParts);
    const dim3 grid(s.total_text, (inner / 4 + kTextPoolQuads - 1) / kTextPoolQuads);
    ProfileScope prof(ctx, K_POOL, 0.0,
                      (double)s.partial_rows * inner * 4.0 + (double)s.total_text * inner * (out_f32 ? 4.0 : 2.0));
    text_pool_kernel<<<grid, block, 0, ctx.stream>>>(s.text_reduce, s.text_scale, inner, partial, out_f32,
                                                        text_out, s.partial_rows, ctx.status);
    return finish(ctx);
}

template <bool LAYER>
static void norm_launch(Context& ctx, int rows, int D, const float* x, float eps, const float* shift,
                        const float* scale, __nv_bfloat16* y)
{
    const int warps = 8;
    const dim3 grid((rows + warps - 1) / warps), block(warps * 32);
    switch (D)
    {
    case 2560: ada_norm_kernel<10, LAYER><<<grid, block, 0, ctx.stream>>>(rows, D, x, eps, shift, scale, y); break;
    case 3072: ada_norm_kernel<12, LAYER><<<grid, block, 0, ctx.stream>>>(rows, D, x, eps, shift, scale, y); break;
    case 1536: ada_norm_kernel<6, LAYER><<<grid, block, 0, ctx.stream>>>(rows, D, x, eps, shift, scale, y); break;
    case 1024: ada_norm_kernel<4, LAYER><<<grid, block, 0, ctx.stream>>>(rows, D, x, eps, shift, scale, y); break;
    case 512: ada_norm_kernel<2, LAYER><<<grid, block, 0, ctx.stream>>>(rows, D, x, eps, shift, scale, y); break;
    case 256: ada_norm_kernel<1, LAYER><<<grid, block, 0, ctx.stream>>>(rows, D, x, eps, shift, scale, y); break;
    default: ada_norm_kernel<0, LAYER><<<grid, block, 0, ctx.stream>>>(rows, D, x, eps, shift, scale, y); break;
    }
}

int launch_ada_norm(Context& ctx, int rows, int D, const float* x, float eps, const float* shift, const float* scale,
                    void* out, int layer)
{
    if (rows < 0 || D <= 0 || D % 8 || !aligned16(x) || !aligned16(shift) || !aligned16(scale) || !aligned16(out) ||
        (layer != 0 && layer != 1))
        return S2_ERR_INVALID;
    if (rows == 0) return S2_OK;
    ProfileScope prof(ctx, K_NORM, 0.0, (double)rows * D * 6.0);
    __nv_bfloat16* y = (__nv_bfloat16*)out;
    if (layer)
        norm_launch<true>(ctx, rows, D, x, eps, shift, scale, y);
    else
        norm_launch<false>(ctx, rows, D, x, eps, shift, scale, y);
    return finish(ctx);
}

int launch_ada_rmsnorm(Context& ctx, int rows, int D, const float* x, float eps, const float* shift,
                       const float* scale, void* out)
{
    return launch_ada_norm(ctx, rows, D, x, eps, shift, scale, out, 0);
}

static int launch_rows(Context& ctx, const void* src, const int* idx, int count, int row_elems, void* dst, int scatter)
{
    if (count <= 0) return S2_OK;
    if (row_elems % 8 || !aligned16(src) || !aligned16(dst)) return S2_ERR_INVALID;
    const int warps = 8;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)count * row_elems * 4.0);
    gather_rows_kernel<<<(count + warps - 1) / warps, warps * 32, 0, ctx.stream>>>(
        static_cast<const uint4*>(src), idx, count, row_elems / 8, static_cast<uint4*>(dst), scatter);
    return finish(ctx);
}

int launch_gather_rows_bf16(Context& ctx, const void* src, const int* idx, int count, int row_elems, void* dst)
{
    return launch_rows(ctx, src, idx, count, row_elems, dst, 0);
}

int launch_scatter_rows_bf16(Context& ctx, const void* src, const int* idx, int count, int row_elems, void* dst)
{
    return launch_rows(ctx, src, idx, count, row_elems, dst, 1);
}

int launch_convert_f32_bf16(Context& ctx, const float* in, void* out, int64_t count)
{
    if (count <= 0) return count == 0 ? S2_OK : S2_ERR_INVALID;
    int64_t blocks = (count + 255) / 256;
    if (blocks > ctx.num_sms * 16) blocks = ctx.num_sms * 16;
    convert_kernel<<<(int)blocks, 256, 0, ctx.stream>>>(in, (__nv_bfloat16*)out, count);
    return finish(ctx);
}

namespace {
// table[pos][pair] = (cos, sin)(pos * freqs[pair]), the RoPE rotation of the
// prepare kernel (same expression, so the same values).
__global__ void rope_table_kernel(const float* __restrict__ freqs, int pairs, int max_pos, float2* __restrict__ table)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= max_pos * pairs) return;
    const int pos = i / pairs, pair = i - pos * pairs;
    float s, c;
    sincosf((float)pos * __ldg(freqs + pair), &s, &c);
    table[i] = make_float2(c, s);
}
} // namespace

int launch_rope_table(Context& ctx, const float* freqs, int pairs, int max_pos, void* table)
{
    if (pairs < 0 || max_pos < 0 || (pairs > 0 && (!freqs || !table))) return S2_ERR_INVALID;
    const int n = pairs * max_pos;
    if (n == 0) return S2_OK;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)n * 8.0);
    rope_table_kernel<<<(n + 255) / 256, 256, 0, ctx.stream>>>(freqs, pairs, max_pos, static_cast<float2*>(table));
    return finish(ctx);
}

namespace {
// *count += number of NaN / Inf elements of x[0, n): the reference's finite
// check (seedvr2_dit.cpp:33-54 sets a flag per blob; a count says the same
// and how much).  An element is non-finite when its exponent bits are all
// ones.  16-byte loads (4 fp32 or 8 bf16) over the aligned body, scalar head
// and tail, one atomic per warp.
template <bool BF16>
__global__ void __launch_bounds__(256) count_nonfinite_kernel(const void* __restrict__ x, int64_t n,
                                                              unsigned long long* __restrict__ count)
{
    constexpr int kPer = BF16 ? 8 : 4; // elements per 16 bytes
    const uintptr_t base = reinterpret_cast<uintptr_t>(x);
    const int esz = BF16 ? 2 : 4;
    // elements before the first 16-byte boundary (the pointer is element aligned)
    int64_t head = (int64_t)(((16 - (base & 15)) & 15) / esz);
    if (head > n) head = n;
    const int64_t vecs = (n - head) / kPer;
    const int64_t tail0 = head + vecs * kPer;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, nthreads = (int64_t)gridDim.x * blockDim.x;
    unsigned int bad = 0;
    const uint4* v = reinterpret_cast<const uint4*>(base + head * esz);
    for (int64_t i = tid; i < vecs; i += nthreads)
    {
        const uint4 u = __ldg(v + i);
        const unsigned int w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; j++)
        {
            if (BF16)
                bad += ((w[j] & 0x7f80u) == 0x7f80u) + ((w[j] & 0x7f800000u) == 0x7f800000u);
            else
                bad += (w[j] & 0x7f800000u) == 0x7f800000u;
        }
    }
    // head and tail elements (fewer than 16 bytes each)
    if (tid < head + (n - tail0))
    {
        const int64_t e = tid < head ? tid : tail0 + (tid - head);
        if (BF16)
            bad += (__ldg(reinterpret_cast<const unsigned short*>(x) + e) & 0x7f80u) == 0x7f80u;
        else
            bad += (__ldg(reinterpret_cast<const unsigned int*>(x) + e) & 0x7f800000u) == 0x7f800000u;
    }
    bad = __reduce_add_sync(0xffffffffu, bad);
    if ((threadIdx.x & 31) == 0 && bad) atomicAdd(count, (unsigned long long)bad);
}
} // namespace

int launch_count_nonfinite(Context& ctx, const void* x, int64_t n, int dtype, unsigned long long* count)
{
    if (n < 0 || !count || (dtype != S2_DTYPE_F32 && dtype != S2_DTYPE_BF16)) return S2_ERR_INVALID;
    if (n == 0) return S2_OK;
    const int esz = dtype == S2_DTYPE_BF16 ? 2 : 4;
    if (!x || (reinterpret_cast<uintptr_t>(x) % esz)) return S2_ERR_INVALID;
    ProfileScope prof(ctx, K_OTHER, 0.0, (double)n * esz);
    // one 16-byte load per thread per pass; the head / tail (< 8 + 8 elements) fit in the first block
    int64_t blocks = (n * esz / 16 + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > ctx.num_sms * 8) blocks = ctx.num_sms * 8;
    if (dtype == S2_DTYPE_BF16)
        count_nonfinite_kernel<true><<<(int)blocks, 256, 0, ctx.stream>>>(x, n, count);
    else
        count_nonfinite_kernel<false><<<(int)blocks, 256, 0, ctx.stream>>>(x, n, count);
    return finish(ctx);
}

int launch_add_vectors(Context& ctx, const float* a, const float* b, float* out, int count, int period)
{
    if (count <= 0) return S2_OK;
    if (period <= 0) return S2_ERR_INVALID;
    add_kernel<<<(count + 255) / 256, 256, 0, ctx.stream>>>(a, b, out, count, period);
    return finish(ctx);
}

int launch_fill_normal_bf16(Context& ctx, void* out, int64_t count, uint64_t seed, float mean, float stddev)
{
    if (count <= 0) return S2_OK;
    int64_t blocks = (count + 255) / 256;
    if (blocks > ctx.num_sms * 32) blocks = ctx.num_sms * 32;
    fill_normal_bf16_kernel<<<(int)blocks, 256, 0, ctx.stream>>>((__nv_bfloat16*)out, count, seed, mean, stddev);
    return finish(ctx);
}

int launch_fill_normal_f32(Context& ctx, float* out, int64_t count, uint64_t seed, float mean, float stddev)
{
    if (count <= 0) return S2_OK;
    int64_t blocks = (count + 255) / 256;
    if (blocks > ctx.num_sms * 32) blocks = ctx.num_sms * 32;
    fill_normal_f32_kernel<<<(int)blocks, 256, 0, ctx.stream>>>(out, count, seed, mean, stddev);
    return finish(ctx);
}

} // namespace s2
