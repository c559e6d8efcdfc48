// Internal (non-ABI) declarations shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <memory>
#include <vector>

#include "../../include/seedvr2_cuda.h"

namespace s2 {

enum
{
    EPI_STORE = S2_EPI_STORE,
    EPI_GELU_TANH = S2_EPI_GELU_TANH,
    EPI_GATE_RESIDUAL = S2_EPI_GATE_RESIDUAL,
};

// Grow-only device workspace slot.
struct DeviceBuffer
{
    void* ptr = nullptr;
    size_t bytes = 0;
    int ensure(size_t want);
    void release();
    ~DeviceBuffer() { release(); }
};

// Per-kernel-class counters: CUDA-event time and algorithmic work.
enum KernelKind
{
    K_GEMM = S2_KERNEL_SHARED_LINEAR,
    K_ATTN = S2_KERNEL_WINDOW_ATTENTION,
    K_PREP = S2_KERNEL_PREPARE_QKV,
    K_NORM = S2_KERNEL_ADA_RMSNORM,
    K_POOL = S2_KERNEL_TEXT_POOL,
    K_OTHER = S2_KERNEL_OTHER,
    K_COMM = S2_KERNEL_COMM,
    K_HOST_WAIT = S2_KERNEL_HOST_WAIT,
    K_NUM = S2_NUM_KERNEL_KINDS,
};

struct Profiler
{
    struct Record
    {
        int kind;
        cudaEvent_t start, stop;
        double flops, bytes;
    };
    bool on = false;
    std::vector<cudaEvent_t> pool;
    std::vector<Record> pending;
    int64_t launches[K_NUM] = {};
    double ms[K_NUM] = {};
    double flops[K_NUM] = {};
    double bytes[K_NUM] = {};
    void reset();
    int collect(); // waits for pending records and folds them in
    void release();
};

struct Context
{
    int device = 0;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    int* status = nullptr; // device status word
    // Split-K ordering flags (one per 32-row x 256-column output box of a
    // split GEMM; zero at creation) and the launch epoch written into them.
    // A context without them runs no split-K GEMM.
    unsigned* split_flags = nullptr;
    int split_slots = 0;
    unsigned split_epoch = 0;
    uint64_t launches = 0;
    Profiler prof;
    // workspace slots (see s2_api.cu for their use)
    DeviceBuffer ws[8];
};

// Brackets one launch with events when counters are on.
struct ProfileScope
{
    Context& ctx;
    bool on;
    Profiler::Record rec;
    ProfileScope(Context& c, int kind, double flops, double bytes);
    ~ProfileScope();
};

// Host window plan (AdaptiveWindowPlan) plus its device-side attention
// schedule, built once per (shapes, window tuple, shift) and cached.
struct Plan
{
    int batch = 0;
    std::vector<int> shapes;              // [batch][3]
    std::vector<int> windows;             // [nw][9]
    std::vector<int> sample_window_count; // [batch]
    std::vector<int> sample_first_window; // [batch]
    std::vector<int> video_indices;       // [n]
    std::vector<int> inverse_video_indices;
    std::vector<int> local_positions; // [n][3]
    int max_window_tokens = 0;
};

int build_plan(const int* shapes, int batch, const int* window, int window_mode, int shifted, Plan& plan);

// Device tables for one (plan, text_lengths) pair.
struct AttnSchedule
{
    int num_windows = 0;
    int packed_rows = 0;    // sum over windows of (L_w + T_s)
    int num_items = 0;      // query-tile pairs (window, q0; 256 rows) in longest-first order
    int total_text = 0;
    int max_text = 0;
    // device arrays
    int* row_src = nullptr;    // [packed_rows] video row (>= 0) or -(1 + text row)
    int* row_pos = nullptr;    // [packed_rows][3] rope positions
    int4* win_info = nullptr;  // [nw] {seq_offset, L, T, partition_offset}
    int* win_pool = nullptr;   // [nw] partial-row offset of the window's text rows
    int2* items = nullptr;     // [num_items] {window, q0 of the first of two 128-row tiles}
    int* video_indices = nullptr; // [n]
    int4* text_reduce = nullptr;  // [total_text] {first partial row, stride (T), count (nw_s), 0}
    float* text_scale = nullptr;  // [total_text] 1/nw_s
    // inverse of row_src, for producers that write packed rows directly:
    int* pack_dst = nullptr;      // [pack_dst_rows] packed row of each video row (-1: none)
    int pack_dst_rows = 0;
    int* text_dst_off = nullptr;  // [total_text + 1] CSR offsets into text_dst
    int* text_dst = nullptr;      // packed rows of each text row (one per window of its sample)
    int max_pos = 0;              // 1 + largest RoPE position in row_pos
    int partial_rows = 0;         // sum over windows of T_s
    // bounds the table-driven gathers / scatters are checked against in a
    // S2_DEBUG_BOUNDS build: video_indices entries, 1 + largest video row
    // row_src gathers, 1 + largest output row video_indices scatters to
    int num_video_indices = 0;
    int src_rows = 0;
    int out_rows = 0;
    double attn_flops_per_head = 0; // sum over windows of 4 * S^2 * 128 (QK^T + PV)
    void* block = nullptr;        // single device allocation backing the arrays
    ~AttnSchedule();
};

int build_schedule(const Plan& plan, const int* text_lengths, AttnSchedule& sched, cudaStream_t stream);
int build_schedule_ex(const Plan& plan, const int* text_lengths, const std::vector<int>* windows_subset,
                      const std::vector<int>* row_of_token, AttnSchedule& sched, cudaStream_t stream,
                      const std::vector<int>* out_of_token = nullptr);

// Output rows of the attention epilogue may live on a peer GPU: an entry of
// AttnSchedule::video_indices is row | (peer + 1) << kPeerShift, and the
// launcher is given the peers' output bases (NVLink peer memory).
constexpr int kPeerShift = 26;
constexpr int kMaxPeers = 8;

int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                      uint32_t box_inner, uint32_t box_outer);
// bf16 (f32 = 0) or fp32 (f32 = 1) row-major 2D map, 128-byte swizzle, box
// rows 128 bytes wide
int make_tmap_2d(CUtensorMap* map, const void* base, int f32, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);

// bf16 4-D tensor (dims[0] innermost, 16-byte aligned strides of dims 1..3 in
// bytes), 128-byte swizzle, box[0] * 2 = 128 bytes; out-of-range elements read
// 0.  element_strides[i]: traversal stride (the box holds box[i] /
// element_strides[i] elements along dim i); element_strides[0] must be 1.
int make_tmap_bf16_4d(CUtensorMap* map, const void* base, const uint64_t* dims, const uint64_t* stride_bytes,
                      const uint32_t* box, const uint32_t* element_strides);

// kernels (launchers return S2_* codes)
int launch_shared_linear(Context& ctx, int M0, int M1, int N, int K, const void* A0, const void* A1, const void* W,
                         const float* bias, int epilogue, const float* gate, int out_f32, void* out0, void* out1);

// QKV projection whose epilogue does the work of launch_prepare_qkv: out =
// A W^T + bias rounded to bf16, per-head RMSNorm (q, k; video / text
// weights) and 3D RoPE, stored straight into the packed rows of `s`
// (stream 0 = video rows indexed like row_src, stream 1 = text rows).
// head_dim 128; heads * 128 a multiple of 256.  rope_table: launch_rope_table
// output for at least s.max_pos positions.
// Multi-GPU form: stream-0 rows are stored to the packed row dst0[row] of
// the GPU named by its peer field (row | (peer + 1) << kPeerShift) with RoPE
// positions pos0[row][3]; q/k/v[i] are peer i's packed buffers.
struct QkvPeers
{
    const int* dst0;
    int dst0_rows;
    const int* pos0;
    void* const* q;
    void* const* k;
    void* const* v;
    int num_peers;
};
int launch_qkv_packed(Context& ctx, const AttnSchedule& s, int M0, int M1, int K, const void* A0, const void* A1,
                      const void* W, const float* bias, int heads, int rope_pairs, float eps, const float* norms,
                      const void* rope_table, int rope_positions, void* q_out, void* k_out, void* v_out,
                      const QkvPeers* peers = nullptr);
// [max_pos][pairs] float2 (cos, sin) of pos * freqs[pair]
int launch_rope_table(Context& ctx, const float* freqs, int pairs, int max_pos, void* table);
int launch_prepare_qkv(Context& ctx, const AttnSchedule& s, int heads, int head_dim, int rope_pairs, float eps,
                       const float* norms, const float* freqs, int in_bf16, const void* vq, const void* vk,
                       const void* vv, int64_t v_ld, const void* tq, const void* tk, const void* tv, int64_t t_ld,
                       void* q_out, void* k_out, void* v_out);

int launch_window_attention(Context& ctx, const AttnSchedule& s, int heads, const void* q, const void* k,
                            const void* v, int out_f32, int round_bf16, void* video_out, float* text_partial,
                            void* const* peer_out = nullptr, int num_peers = 0);

int launch_text_pool(Context& ctx, const AttnSchedule& s, int inner, const float* partial, int out_f32,
                     int round_bf16, void* text_out);

int launch_ada_rmsnorm(Context& ctx, int rows, int D, const float* x, float eps, const float* shift,
                       const float* scale, void* out);
// layer = 0: RMSNorm, 1: LayerNorm (both without affine), then * scale + shift -> bf16
int launch_ada_norm(Context& ctx, int rows, int D, const float* x, float eps, const float* shift, const float* scale,
                    void* out, int layer);

// Token formats around the block stack (seedvr2_dit.cpp:167-326) and the
// frontend / tail nets' dense passes.
constexpr int kLatentChannels = S2_LATENT_CHANNELS;  // 33
constexpr int kPatchFeatures = S2_PATCH_FEATURES;    // 132 = 4 x 33
constexpr int kPatchPitch = 136;                     // bf16 GEMM row: 132 features + zeros (16-byte rows)
constexpr int kPredChannels = S2_PRED_CHANNELS;      // 16
constexpr int kPredFeatures = S2_PRED_FEATURES;      // 64 = 4 x 16
constexpr int kTextChannels = S2_TEXT_CHANNELS;      // 5120
constexpr int kTimeFeatures = S2_TIME_FEATURES;      // 256
constexpr int kTimestepChunk = 64;                   // timesteps per embedding launch
constexpr int kGemvRows = 8;                         // batch rows per matrix-vector launch
// Host checks of patchify_video / unpatchify_prediction over a batch of
// latent shapes (S2_OK, S2_ERR_INVALID, or S2_ERR_ALLOC for an empty output,
// as the reference); the other side's row count is returned.
int patchify_rows(const int* shapes, int batch, int rows, int64_t* patches);
int unpatchify_rows(const int* shapes, int batch, int rows, int64_t* tokens);
// [T][H][W][33] fp32 latent tokens of one sample -> patches: fp32 rows of 132
// (bf16_out = 0) or bf16 rows of kPatchPitch with zero padding (bf16_out = 1)
int launch_patchify(Context& ctx, const float* src, int T, int H, int W, void* dst, int bf16_out);
// Fused SeedVR2Pipeline::predict assembly + patchify: 16 latent planes, 16
// condition planes and a constant 1 per token -> bf16 patch rows of kPatchPitch
int launch_patchify_planar(Context& ctx, const float* latent, int64_t latent_cstep, const float* condition,
                           int64_t condition_cstep, int T, int H, int W, void* dst);
// apply_cfg: out = neg + scale (pos - neg), and with rescale != 0 (n >= 2) the
// rescale factor on the device (*factor_out; null when there is none), applied
// to out when apply_factor.  scratch: cfg_scratch_bytes() device bytes.
size_t cfg_scratch_bytes();
int launch_apply_cfg(Context& ctx, const float* pos, const float* neg, int64_t n, float scale, float rescale,
                     float* out, void* scratch, int apply_factor, const float** factor_out);
// latent[c][t] += delta * pred[t][c] * (*factor, if given)
int launch_euler(Context& ctx, float* latent, int64_t cstep, int64_t tokens, const float* pred, const float* factor,
                 float delta);
// [patches][64] fp32 -> [T][H][W][16] fp32 (16-byte aligned buffers)
int launch_unpatchify(Context& ctx, const float* src, int T, int H, int W, float* dst);
// host timesteps -> [batch][256] fp32 device
int launch_timestep_embedding(Context& ctx, const float* timesteps, int batch, float* out);
// y(b, n) = act(bias[n] + W[n] . x[b]) (act 1 = SiLU), W bf16 [N][K], x fp32
// [B][ldx]; y(b, n) stored at y[(n / chunk) * s_chunk + b * s_b + n % chunk]
int launch_gemv(Context& ctx, const void* W, const float* bias, int N, int K, const float* x, int ldx, int B, int act,
                float* y, int chunk, int64_t s_chunk, int64_t s_b);

// VAE DecomposedConv3D as one implicit GEMM (conv_sm100.cu).  X: the padded
// input, channels-last bf16 [frames][H][W][Cp]; weights bf16
// [Co][kt][kh][kw][cpad64]; out planar fp32 [Co][out_cstep], element
// (t, y, x) at (t * Ho + y) * Wo + x.
struct Conv3dGeometry
{
    int Ci, Cp, cpad64, Co;
    int H, W;
    int kt, kh, kw, st, dt, sh, sw, dh, dw, ph, pw;
    int Tout, Ho, Wo;
};
int conv3d_pack(Context& ctx, const float* in, int64_t in_cstep, int C, int Cp, int HW, int frame0, int frames,
                int prefix, void* X);
int conv3d_gemm(Context& ctx, const Conv3dGeometry& g, const void* X, int frames_x, const void* Wt, const float* bias,
                float* out, int64_t out_cstep);

int launch_convert_f32_bf16(Context& ctx, const float* in, void* out, int64_t count);
// ncnn built-ins of a block graph (graph_ops.cu), fp32 [rows][cols]
int launch_binary_op(Context& ctx, int op, int rows, int cols, const float* a, const float* b, int b_rows, float* out);
int launch_norm_f32(Context& ctx, int layer, int rows, int D, const float* x, float eps, const float* gamma,
                    const float* beta, float* y);
int launch_gelu_f32(Context& ctx, int fast, int64_t count, const float* x, float* y);
int launch_add_vectors(Context& ctx, const float* a, const float* b, float* out, int count, int period);
// *count += NaN / Inf elements of x[0, n) (dtype S2_DTYPE_F32 or S2_DTYPE_BF16)
int launch_count_nonfinite(Context& ctx, const void* x, int64_t n, int dtype, unsigned long long* count);
int launch_fill_normal_bf16(Context& ctx, void* out, int64_t count, uint64_t seed, float mean, float stddev);
int launch_fill_normal_f32(Context& ctx, float* out, int64_t count, uint64_t seed, float mean, float stddev);

} // namespace s2
