/* libseedvr2_cuda -- B200 (sm_100a) implementation of the SeedVR2 DiT block
 * hot path: the AdaptiveWindowAttention and SharedLinear custom layers and
 * the block arithmetic around them.
 *
 * C ABI: plain pointers and sizes, no C++ or torch types.  Unless a comment
 * says "host", pointers are CUDA device pointers owned by the caller; the
 * library owns only its context workspace and plan/model objects.  All work
 * is enqueued on the context's stream; nothing synchronises unless stated.
 *
 * Error convention (the reference layers' own codes plus three):
 *    0 ok, -1 invalid argument / shape, -2 inconsistent window plan,
 *   -100 allocation failure      (adaptive_window_attention.cpp:769-845, :642-653)
 *   -3 CUDA error, -4 a bounded device wait expired, -5 unsupported device.
 *
 * Reference paths below are relative to the reference checkout
 * (Chisato623/seedvr2_ncnn).
 */
#ifndef SEEDVR2_CUDA_H
#define SEEDVR2_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define S2_OK 0
#define S2_ERR_INVALID (-1)
#define S2_ERR_PLAN (-2)
#define S2_ERR_CUDA (-3)
#define S2_ERR_TIMEOUT (-4)
#define S2_ERR_DEVICE (-5)
#define S2_ERR_TOO_LARGE (-6) /* exceeds a fixed workspace (s2_awa_forward_static) */
#define S2_ERR_ALLOC (-100)

#define S2_DTYPE_F32 0
#define S2_DTYPE_BF16 1

/* window_mode: how the AdaptiveWindowAttention window tuple is read. */
#define S2_WINDOW_TARGET 0 /* reference: target window COUNT per axis (param ids 2-4) */
#define S2_WINDOW_EXTENT 1 /* extension: window extent (t,h,w) in tokens */

/* SharedLinear epilogues (out = A W^T + bias, then): */
#define S2_EPI_STORE 0         /* out (bf16 or fp32) = acc */
#define S2_EPI_GELU_TANH 1     /* out (bf16) = gelu_tanh(acc) */
#define S2_EPI_GATE_RESIDUAL 2 /* out (fp32, in place) += acc * gate[n] */

typedef struct s2_context s2_context;
typedef struct s2_plan s2_plan;
typedef struct s2_dit s2_dit;
typedef struct s2_shard s2_shard;

/* ---------------------------------------------------------------------------
 * Context.  Replaces the Vulkan device / VkCompute / allocator set-up the
 * layers get from ncnn (create_pipeline / upload_model lifecycle,
 * adaptive_window_attention.cpp:981-1057, shared_linear.cpp:99-126).
 * stream: a cudaStream_t (NULL = legacy default stream). */
int s2_init(int device, void* stream, s2_context** out);
void s2_destroy(s2_context* ctx);
int s2_set_stream(s2_context* ctx, void* stream);
/* Synchronises the stream and returns (then clears) the first error any
 * kernel recorded in the device status word (S2_ERR_TIMEOUT / S2_ERR_INVALID). */
int s2_status(s2_context* ctx);
const char* s2_error_string(int code);
int s2_version(void);
/* Count of this library's kernel launches on ctx since creation. */
uint64_t s2_launch_count(const s2_context* ctx);

/* Per-kernel counters (the layers' "ncnn counters"): while enabled, every
 * launch is bracketed by CUDA events on the context stream and credited with
 * its algorithmic flops and HBM bytes.  Enabling resets the totals.
 * s2_profile_read synchronises the stream and returns the totals of one
 * kernel kind.  The reference has no counters (wall clock only,
 * examples/seedvr2_blocks_main.cpp:135-149). */
#define S2_KERNEL_SHARED_LINEAR 0
#define S2_KERNEL_WINDOW_ATTENTION 1
#define S2_KERNEL_PREPARE_QKV 2
#define S2_KERNEL_ADA_RMSNORM 3
#define S2_KERNEL_TEXT_POOL 4
#define S2_KERNEL_OTHER 5
#define S2_KERNEL_COMM 6      /* NCCL exchanges / all-reduce (device time) */
#define S2_KERNEL_HOST_WAIT 7 /* host time spent waiting on NCCL calls to be issued */
#define S2_NUM_KERNEL_KINDS 8
int s2_profile_enable(s2_context* ctx, int enable);
int s2_profile_read(s2_context* ctx, int kind, int64_t* launches, double* milliseconds, double* flops,
                    double* bytes);

/* ---------------------------------------------------------------------------
 * Window plan.  Replaces build_adaptive_window_plan
 * (adaptive_window_attention.h:46-49, .cpp:565-655), bit-exact for
 * S2_WINDOW_TARGET; S2_WINDOW_EXTENT applies the same shift/truncation rule
 * to explicit extents.  video_shapes: host [batch][3] (t,h,w). */
int s2_plan_build(const int* video_shapes, int batch, const int* window, int window_mode, int shifted,
                  s2_plan** out);
int s2_plan_info(const s2_plan* plan, int* num_windows, int* num_tokens, int* max_window_tokens);
/* Host copies of the plan (AdaptiveWindowPlan fields, adaptive_window_attention.h:16-36).
 * windows: 9 ints per window (sample, t0,t1,h0,h1,w0,w1, partition_offset, token_count);
 * local_positions: 3 ints per token.  Any pointer may be NULL. */
int s2_plan_copy(const s2_plan* plan, int* windows, int* sample_window_count, int* video_indices,
                 int* inverse_video_indices, int* local_positions);
void s2_plan_free(s2_plan* plan);
/* The plan's attention schedule as the kernels read it, copied back from the
 * device (built for these text lengths first if needed), so the device-side
 * window indexing can be checked bit for bit against the plan's
 * video_indices / inverse_video_indices / local_positions
 * (adaptive_window_attention.cpp:446-473, :954-961).  sizes[4] (host, always
 * written): packed rows R, windows nw, tokens n, pack_dst rows.  Then, for
 * any non-NULL host array: row_src [R] (video token of each packed row, or
 * -1 - text row), row_pos [R][3] (RoPE position: window-local (t + T, h, w)
 * for video rows, (j, j, j) for text row j), win_info [nw][4] (packed row of
 * the window's first row, L, T, partition offset), video_indices [n] (source
 * token of each partition slot), pack_dst [rows] (packed row of each video
 * token).  Synchronous. */
int s2_plan_schedule_copy(s2_context* ctx, s2_plan* plan, const int* text_lengths, int* sizes, int* row_src,
                          int* row_pos, int* win_info, int* video_indices, int* pack_dst);

/* Test hook of the checked build (libseedvr2_cuda_checked.so, compiled with
 * S2_DEBUG_BOUNDS): overwrites entry `index` of one table of the plan's
 * device schedule (built by s2_plan_schedule_copy or a forward) with
 * `value` -- table 0 = row_src (the gather), 1 = video_indices (the
 * scatter).  The checked build's kernels test every index they read from
 * these tables, so a forward over a corrupted schedule records a bad index
 * (s2_status then returns -1) and skips the access.  Any other build returns
 * S2_ERR_INVALID and changes nothing.  No counterpart in the reference (its
 * tables live in host vectors). */
int s2_debug_poke_schedule(s2_context* ctx, s2_plan* plan, int table, int index, int value);

/* ---------------------------------------------------------------------------
 * AdaptiveWindowAttention forward.  Replaces
 * AdaptiveWindowAttention::forward (CPU :764-978, Vulkan :1059-1270) with
 * the layer's parameters (param ids 0-10, :700-714) and weights (:716-738).
 *
 * Inputs: the fused layout is q,k,v at column offsets 0, inner, 2*inner of
 * one [tokens][3*inner] row (pass video_k = video_q + inner elements etc. and
 * ld = 3*inner); the split layout (8-blob form) passes three [tokens][inner]
 * arrays with ld = inner.  in_dtype S2_DTYPE_F32 or S2_DTYPE_BF16.
 * Outputs: video_out [Nv][inner], text_out [Nt][inner] in out_dtype, fully
 * overwritten (video rows scattered back to source order; text rows averaged
 * over the sample's windows).  q/k/v enter the tensor cores as bf16 with
 * fp32 softmax and accumulation. */
typedef struct
{
    int heads;                   /* param 0 */
    int head_dim;                /* param 1 (must be 128) */
    int window[3];               /* params 2-4 */
    int window_mode;             /* S2_WINDOW_TARGET (reference) or S2_WINDOW_EXTENT */
    int shifted;                 /* param 5 */
    float epsilon;               /* param 6 */
    int rope_pairs;              /* param 7 */
    int official_bf16_attention; /* param 10: round the context to bf16 */
    const float* norm_weights;   /* device [4][head_dim]: video_q, video_k, text_q, text_k */
    const float* rope_freqs;     /* device [rope_pairs] */
} s2_awa_params;

int s2_awa_forward(s2_context* ctx, const s2_awa_params* params, const s2_plan* plan, const int* video_shapes,
                   const int* text_lengths, int batch, int in_dtype, const void* video_q, const void* video_k,
                   const void* video_v, int64_t video_ld, const void* text_q, const void* text_k,
                   const void* text_v, int64_t text_ld, int out_dtype, void* video_out, void* text_out);

/* AdaptiveWindowAttention forward that allocates no memory, for callers that
 * cannot call cudaMalloc: plugins whose host owns all device memory and only
 * hands them inputs and outputs, processes under a hard device-memory cap,
 * and loops that must not risk the device-wide synchronisation of
 * cudaMalloc/cudaFree.  No counterpart in the reference (its layers allocate
 * through ncnn's allocators).  Same arguments and results as s2_awa_forward
 * minus the context and plan; `stream` is a cudaStream_t of the CURRENT
 * device.  Scratch (schedule tables, packed bf16 q/k/v, text partials, a
 * status word) is one static __device__ array of S2_AWA_STATIC_SCRATCH_BYTES
 * that every GPU loading the library holds until exit; with 20 heads it fits
 * about 4000 packed rows (video tokens + windows x text tokens), e.g. a
 * 1x32x32 or 1x48x48 token video with 58 text tokens.  Larger inputs return
 * S2_ERR_TOO_LARGE.  The first call on a device resolves the array's device
 * address (cudaGetSymbolAddress) -- make it before any stream capture.  All
 * calls share the array: calls whose GPU work overlaps race (serialise
 * them on one stream).  The call only enqueues: a bounded device wait that
 * runs out, or a bad table index, is recorded in the scratch's status word,
 * which s2_awa_static_status reads back. */
#define S2_AWA_STATIC_SCRATCH_BYTES (64u << 20)
int s2_awa_forward_static(const s2_awa_params* params, const int* video_shapes, const int* text_lengths, int batch,
                          int in_dtype, const void* video_q, const void* video_k, const void* video_v,
                          int64_t video_ld, const void* text_q, const void* text_k, const void* text_v,
                          int64_t text_ld, int out_dtype, void* video_out, void* text_out, void* stream);
/* Status of the last s2_awa_forward_static call on the CURRENT device:
 * synchronises `stream` (the call's stream), then returns and clears the
 * scratch's status word -- S2_ERR_TIMEOUT for an expired device wait,
 * S2_ERR_INVALID for a bad index, S2_OK otherwise (also before any call).
 * Every static call clears the word on entry, so read it before the next
 * call.  Allocates nothing.  No counterpart in the reference. */
int s2_awa_static_status(void* stream);

/* ---------------------------------------------------------------------------
 * SharedLinear forward.  Replaces SharedLinear::forward (shared_linear.cpp:83-96,
 * :128-143): one weight W [N][K] (bf16, row-major, i.e. ncnn's
 * [num_output][num_input]) applied to two token streams A0 [M0][K] and
 * A1 [M1][K] (bf16) in ONE launch, out_s = A_s W^T + bias, then the epilogue.
 * bias: fp32 [N] or NULL.  gate: fp32 [N] (S2_EPI_GATE_RESIDUAL only).
 * out_dtype: S2_DTYPE_BF16 / S2_DTYPE_F32 for S2_EPI_STORE, bf16 for GELU,
 * fp32 (read-modify-write) for GATE_RESIDUAL.  M1 may be 0 (A1/out1 unused).
 * K must be a multiple of 8. */
int s2_shared_linear(s2_context* ctx, int M0, int M1, int N, int K, const void* A0, const void* A1, const void* W,
                     const float* bias, int epilogue, const float* gate, int out_dtype, void* out0, void* out1);

/* ---------------------------------------------------------------------------
 * Block arithmetic around the layers (ops of the exported block graph).
 * ada_rmsnorm: out[r] (bf16) = x[r] * rsqrt(mean(x[r]^2) + eps) * scale + shift,
 * x fp32 [rows][D], shift/scale fp32 [D]. */
int s2_ada_rmsnorm(s2_context* ctx, int rows, int D, const float* x, float eps, const float* shift,
                   const float* scale, void* out_bf16);
/* The LayerNorm form of the same pass (BASELINE's block description names
 * "RMS/LayerNorm"; which one the exported graph uses is not in the tree):
 * out[r] (bf16) = (x[r] - mean(x[r])) * rsqrt(var(x[r]) + eps) * scale + shift,
 * var the biased variance, no affine of its own. */
int s2_ada_layernorm(s2_context* ctx, int rows, int D, const float* x, float eps, const float* shift,
                     const float* scale, void* out_bf16);
/* ncnn built-in layers a DiT block graph places between the custom layers
 * (ncnn's BinaryOp, RMSNorm, LayerNorm and GELU; used by the graph executor
 * of the ncnn-surface library), on fp32 row-major device blobs.
 * s2_binary_op: out[r][c] = a[r][c] op b[r][c], or b[0][c] for every row when
 * b_rows == 1 (ncnn's broadcast of a [1][cols] blob); op = ncnn's op_type
 * 0 add, 1 sub, 2 mul, 3 div; cols % 4 == 0, 16-byte aligned pointers.
 * s2_norm_f32: layer = 0 RMSNorm, 1 LayerNorm over each row of D values,
 * then * gamma[c] and + beta[c] when given (NULL = none).
 * s2_gelu_f32: fast = 1 the tanh approximation, 0 the erf form. */
#define S2_BINARY_ADD 0
#define S2_BINARY_SUB 1
#define S2_BINARY_MUL 2
#define S2_BINARY_DIV 3
int s2_binary_op(s2_context* ctx, int op, int rows, int cols, const float* a, const float* b, int b_rows, float* out);
int s2_norm_f32(s2_context* ctx, int layer, int rows, int D, const float* x, float eps, const float* gamma,
                const float* beta, float* out);
int s2_gelu_f32(s2_context* ctx, int fast, int64_t count, const float* x, float* out);

/* fp32 -> bf16 (round to nearest even). */
int s2_convert_f32_bf16(s2_context* ctx, const float* in, void* out, int64_t count);
/* Number of NaN / Inf values among `count` device elements of dtype
 * S2_DTYPE_F32 or S2_DTYPE_BF16 (the reference's finite-check shader,
 * seedvr2_dit.cpp:33-54, as a count); synchronises. */
int s2_count_nonfinite(s2_context* ctx, const void* data, int64_t count, int dtype, int64_t* nonfinite);

/* ---------------------------------------------------------------------------
 * DiT block stack.  Replaces SeedVR2DiTBlocks' block graph
 * (seedvr2_dit.h:48-86; load :531-634 registers the two custom layers and
 * loads blocks/seedvr2_blocks.ncnn; forward(DiTBlockInputs) :1096-1181).
 * Weights are bf16 on the device; see s2_dit_config for the block shape. */
typedef struct
{
    int num_blocks;    /* 32 */
    int hidden;        /* D = 2560 */
    int heads;         /* 20 */
    int head_dim;      /* 128 */
    int mlp_hidden;    /* F = 10240 */
    int rope_pairs;    /* 21 */
    int window[3];     /* AWA window tuple */
    int window_mode;   /* S2_WINDOW_TARGET / S2_WINDOW_EXTENT */
    float norm_eps;    /* block RMSNorm eps (1e-5) */
    float qk_eps;      /* AWA epsilon (1e-5) */
    int qkv_bias;      /* SharedLinear bias_term of each projection */
    int out_bias;
    int mlp_bias;
} s2_dit_config;

/* Host fp32 weights of one block (converted to bf16 on upload):
 * ada [6][D]: per-block modulation offsets (attn shift/scale/gate, mlp shift/scale/gate);
 * w_qkv [3D][D], w_out [D][D], w_up [F][D], w_down [D][F] (SharedLinear layout), biases or NULL;
 * qk_norm [4][head_dim]; rope_freqs [rope_pairs]. */
typedef struct
{
    const float* ada;
    const float* w_qkv;
    const float* b_qkv;
    const float* w_out;
    const float* b_out;
    const float* w_up;
    const float* b_up;
    const float* w_down;
    const float* b_down;
    const float* qk_norm;
    const float* rope_freqs;
} s2_block_host_weights;

int s2_dit_create(s2_context* ctx, const s2_dit_config* cfg, s2_dit** out);
void s2_dit_free(s2_dit* dit);
int s2_dit_set_block_weights(s2_dit* dit, int block, const s2_block_host_weights* w);
/* The norm of a block's two AdaLN passes (both forms without affine, then
 * the modulation's scale and shift): S2_NORM_RMS (the default) or
 * S2_NORM_LAYER, chosen per block. */
#define S2_NORM_RMS 0
#define S2_NORM_LAYER 1
int s2_dit_set_block_norm(s2_dit* dit, int block, int norm_type);
/* Seeded synthetic weights generated on the device (weights ~N(0,0.02),
 * ada offsets ~N(0,1)/sqrt(D) (+1 on the scale rows), qk norms ~N(1,0.02),
 * rope freqs 1/10000^(2i/(2*pairs))). */
int s2_dit_init_random(s2_dit* dit, uint64_t seed);
/* Finite checks (the reference's SEEDVR2_DIT_CHECK_FINITE,
 * seedvr2_dit.cpp:651-716 and :843-1071).  With enable != 0, every
 * s2_dit_forward (and the step / denoise calls built on it; one GPU) counts
 * the NaN / Inf values of the video and text rows at the block stack's input
 * (the frontend's output) and after every block, on the device, reads the
 * counters once at the end and returns -1, as the reference does, when any
 * is non-zero.  s2_dit_nonfinite_report then gives the first non-finite point
 * of the last checked forward: block -1 = the input, b = block b's output,
 * num_blocks = all finite; and the counts there (-1 before any checked
 * forward). */
int s2_dit_set_check_finite(s2_dit* dit, int enable);
/* Block checkpoints (the checkpoint_blocks of SeedVR2DiTBlocks::record_blocks,
 * seedvr2_dit.cpp:644-649, :817-831, :1073-1089, behind the reference's
 * SEEDVR2_DIT_DUMP_BLOCKS dumps): after block blocks[i] of every following
 * forward (one GPU), the block's video rows are copied to video[i] and its
 * text rows to text[i] (device fp32 [Nv][D] and [Nt][D] of the forward's
 * shape; s2_dit_forward_host writes sample s at its rows, as in its outputs;
 * s2_dit_forward_step at its block-stack rows -- patches, then text rows --
 * samples one after another; the denoise loop's buffers hold its last DiT
 * pass).  A block outside [0, num_blocks) is -1, as the reference's range
 * check.  count 0 clears them.  The pointers are kept, not copied.
 * s2_dit_forward_sharded returns -1 while checkpoints are set (a rank holds
 * only its own rows). */
int s2_dit_set_checkpoints(s2_dit* dit, const int* blocks, int count, float* const* video, float* const* text);
int s2_dit_nonfinite_report(const s2_dit* dit, int* block, int64_t* video_count, int64_t* text_count);
/* Device-resident forward of all blocks for ONE sample:
 * x: fp32 [Nv + Nt][D] (video rows then text rows), updated in place;
 * modulation: fp32 [6][D] device (frontend outputs out2..out7). */
int s2_dit_forward(s2_dit* dit, const int* video_shape, int text_length, float* x, const float* modulation);
/* Same, host buffers in and out (the DiTBlockInputs call), batch >= 1,
 * samples run one after another like the reference (seedvr2_dit.cpp:1107-1121):
 * video [Nv_total][D], text [Nt_total][D], modulation [6][batch][D] (host fp32). */
int s2_dit_forward_host(s2_dit* dit, const int* video_shapes, const int* text_lengths, int batch,
                        const float* video, const float* text, const float* modulation, float* video_out,
                        float* text_out);
/* Pipelined form of s2_dit_forward_host (same arguments and results): it
 * enqueues the uploads, the forward and the downloads and returns without
 * waiting.  Uploads and downloads run on two copy streams of the DiT against
 * two device staging buffers used in turn, so consecutive calls overlap: call
 * i+1's upload and call i-1's download run under call i's forward.  For that
 * overlap the host buffers must be pinned (page-locked); any buffer works,
 * but pageable ones make the copies wait.  Host buffers stay untouched (inputs)
 * and unread (outputs) until s2_dit_host_wait returns, which waits for all
 * enqueued calls and reports a CUDA error among them. */
int s2_dit_forward_host_async(s2_dit* dit, const int* video_shapes, const int* text_lengths, int batch,
                              const float* video, const float* text, const float* modulation, float* video_out,
                              float* text_out);
int s2_dit_host_wait(s2_dit* dit);

/* ---------------------------------------------------------------------------
 * Token formats and the frontend / tail nets around the block stack
 * (seedvr2_dit.cpp).  Widths fixed by the reference: 33 latent channels per
 * token, 1x2x2 patches (132 features in, 64 = 4 x 16 prediction features
 * out), 5120 text-embedding channels, a 256-wide sinusoidal timestep
 * embedding.  shapes: latent (t, h, w) per sample, h and w even. */
#define S2_LATENT_CHANNELS 33
#define S2_PATCH_FEATURES 132
#define S2_PRED_CHANNELS 16
#define S2_PRED_FEATURES 64
#define S2_TEXT_CHANNELS 5120
#define S2_TIME_FEATURES 256

/* patchify_video (seedvr2_dit.cpp:167-230): video fp32 [rows][33] (samples
 * concatenated, rows = sum t*h*w) -> out fp32 [sum t*(h/2)*(w/2)][132];
 * feature (y*2 + x)*33 + c of patch (f, py, px) = channel c of token
 * (f, 2py + y, 2px + x).  -1 on an odd h/w, a non-positive extent or a row
 * count that does not match the shapes. */
int s2_patchify_video(s2_context* ctx, const float* video, int rows, const int* shapes, int batch, float* out);
/* unpatchify_prediction (seedvr2_dit.cpp:255-326): pred fp32 [patches][64]
 * -> out fp32 [tokens][16], the inverse ordering (16-byte aligned buffers). */
int s2_unpatchify_prediction(s2_context* ctx, const float* pred, int rows, const int* shapes, int batch,
                             float* out);
/* make_timestep_embedding (seedvr2_dit.cpp:232-253): host timesteps[batch]
 * -> out fp32 [batch][256] = sin(t f_i) | cos(t f_i), f_i = exp(-ln(1e4) i/128). */
int s2_timestep_embedding(s2_context* ctx, const float* timesteps, int batch, float* out);

/* Host fp32 weights of the frontend and tail nets (frontend.ncnn /
 * tail.ncnn of SeedVR2DiTBlocks, seedvr2_dit.cpp:1183-1295, :1424-1494;
 * the exported graphs are not in the reference tree, so this op sequence is
 * the B200 build's assumption, restated by the CPU oracle):
 *   video  = patches W_vid_in^T + b_vid_in                       [Np][D]
 *   text   = text W_txt_in^T + b_txt_in                          [T][D]
 *   e      = silu(temb W_emb0^T + b0); e = silu(e W_emb1^T + b1)
 *   mod    = e W_emb2^T + b2 = six [D] chunks (out2..out7)       [6][D]
 *   tail:  h = rmsnorm(video) * (mod[1] + tail_ada[1]) + (mod[0] + tail_ada[0])
 *          pred = h W_out^T + b_out                              [Np][64]
 * Shapes: w_vid_in [D][132], w_txt_in [D][5120], w_emb0 [D][256],
 * w_emb1 [D][D], w_emb2 [6D][D], tail_ada [2][D], w_out [64][D]; biases
 * [rows of W] or NULL. */
typedef struct
{
    const float* w_vid_in;
    const float* b_vid_in;
    const float* w_txt_in;
    const float* b_txt_in;
    const float* w_emb0;
    const float* b_emb0;
    const float* w_emb1;
    const float* b_emb1;
    const float* w_emb2;
    const float* b_emb2;
    const float* tail_ada;
    const float* w_out;
    const float* b_out;
} s2_dit_io_host_weights;

/* Uploads the frontend / tail weights (bf16 on the device).  s2_dit_init_random
 * also fills them (weights ~N(0,0.02), tail offsets like the blocks'). */
int s2_dit_set_io_weights(s2_dit* dit, const s2_dit_io_host_weights* w);

/* forward_frontend (seedvr2_dit.cpp:1183-1295): DiTInputs -> DiTBlockInputs.
 * video fp32 [video_rows][33], text fp32 [text_rows][5120], host timesteps
 * [batch]; video_out fp32 [patches][D], text_out fp32 [text_rows][D],
 * modulation fp32 [6][batch][D].  Validation of split_dit_inputs_by_sample
 * (:369-427) and patchify_video; -1 before the weights are set. */
int s2_dit_forward_frontend(s2_dit* dit, const int* video_shapes, const int* text_lengths, const float* timesteps,
                            int batch, const float* video, int video_rows, const float* text, int text_rows,
                            float* video_out, float* text_out, float* modulation);
/* The tail net + unpatchify_prediction: video fp32 [patches][D] (block
 * output), modulation fp32 [6][batch][D] -> prediction fp32 [tokens][16]. */
int s2_dit_forward_tail(s2_dit* dit, const int* video_shapes, int batch, const float* video, int video_rows,
                        const float* modulation, float* prediction);
/* The whole DiT (SeedVR2DiTBlocks::forward(DiTInputs), seedvr2_dit.cpp:1297-1536):
 * frontend, all blocks, tail, per sample like the reference; prediction fp32
 * [video_rows][16], text_out fp32 [text_rows][D] (block stack's text rows). */
int s2_dit_forward_step(s2_dit* dit, const int* video_shapes, const int* text_lengths, const float* timesteps,
                        int batch, const float* video, int video_rows, const float* text, int text_rows,
                        float* prediction, float* text_out);
/* Same, host buffers in and out (synchronises). */
int s2_dit_forward_step_host(s2_dit* dit, const int* video_shapes, const int* text_lengths, const float* timesteps,
                             int batch, const float* video, int video_rows, const float* text, int text_rows,
                             float* prediction, float* text_out);

/* ---------------------------------------------------------------------------
 * Denoise loop on the device (SeedVR2Pipeline::denoise + predict,
 * seedvr2_pipeline.cpp:284-329, :536-588): `steps` Euler steps from
 * t = 1000 down to 0, each a whole-DiT pass on [latent | condition | 1] tokens
 * and, when cfg_scale != 1, a second pass on the negative text combined by
 * apply_cfg (:171-210); no host round trip between steps.
 * latent / condition: 16 fp32 channel planes of t*h*w values (plane stride
 * *_cstep elements, >= t*h*w: the ncnn Mat layout); the latent is updated in
 * place.  positive / negative text fp32 [rows][5120].  -1 for steps <= 0, an
 * odd h/w, empty text, a missing negative text with cfg_scale != 1, or
 * frontend / tail weights not loaded. */
typedef struct
{
    int steps;         /* PipelineOptions::steps (>= 1) */
    float cfg_scale;   /* 1 = no guidance */
    float cfg_rescale; /* 0 = no rescale */
} s2_denoise_options;

int s2_dit_denoise(s2_dit* dit, const int* latent_shape, float* latent, int64_t latent_cstep, const float* condition,
                   int64_t condition_cstep, const float* positive_text, int positive_rows, const float* negative_text,
                   int negative_rows, const s2_denoise_options* options);
/* Same, host buffers (synchronises). */
int s2_dit_denoise_host(s2_dit* dit, const int* latent_shape, float* latent, int64_t latent_cstep,
                        const float* condition, int64_t condition_cstep, const float* positive_text,
                        int positive_rows, const float* negative_text, int negative_rows,
                        const s2_denoise_options* options);
/* apply_cfg (seedvr2_pipeline.cpp:171-210) on device arrays of `count` fp32:
 * out = neg + scale (pos - neg), then with rescale != 0 multiplied by
 * float(rescale std(pos) / std(out) + 1 - rescale) (sample standard
 * deviations in double). */
int s2_apply_cfg(s2_context* ctx, const float* pos, const float* neg, int64_t count, float scale, float rescale,
                 float* out);

/* ---------------------------------------------------------------------------
 * VAE DecomposedConv3D (decomposed_conv3d.h:30-90, forward :605-765): a causal
 * 3-D convolution of a [c][d][h][w] blob, computed here as one implicit GEMM
 * on the tensor cores (bf16 operands, fp32 accumulation).
 * cfg: the layer's 16-value config blob in its load_model order (num_output,
 * num_input, kernel_w, kernel_h, kernel_t, stride_t, dilation_t, head_frames,
 * stride_w, stride_h, dilation_w, dilation_h, pad_w, pad_h, groups,
 * bias_term); bias: host fp32 [num_output] (bias_term) or NULL; weights: host
 * fp32 kernel_t x [num_output][num_input][kernel_h][kernel_w].  This build
 * supports groups = 1 and stride_w <= 2 (-1 otherwise).
 * memory_state: the VAE's temporal-memory state (seedvr2::MemoryState): with
 * ACTIVE the head frames are the previous chunk's cached frames, otherwise
 * head_frames copies of frame 0; any state but DISABLED caches the last
 * kernel_t - stride_t padded input frames for the next call. */
#define S2_VAE_MEMORY_DISABLED 0
#define S2_VAE_MEMORY_INITIALIZING 1
#define S2_VAE_MEMORY_ACTIVE 2
typedef struct s2_conv3d s2_conv3d;
int s2_conv3d_create(s2_context* ctx, const int* cfg, const float* bias, const float* weights, s2_conv3d** out);
/* Output extents (w, h, d, c) of a forward on a w x h x d input, or -1. */
int s2_conv3d_output_shape(const s2_conv3d* layer, int w, int h, int d, int memory_state, int* out_whdc);
/* in: device fp32 [c][plane stride in_cstep >= d*h*w]; out: device fp32
 * [num_output][plane stride out_cstep >= output d*h*w].  -1 on a channel
 * count other than num_input, too few padded frames, or cached frames of
 * another size (as the reference). */
int s2_conv3d_forward(s2_conv3d* layer, const float* in, int64_t in_cstep, int w, int h, int d, int c,
                      int memory_state, float* out, int64_t out_cstep);
/* Drops the cached frames (DecomposedConv3D::reset_temporal_memory,
 * decomposed_conv3d.cpp:596-603); host state only, no device work. */
void s2_conv3d_reset_memory(s2_conv3d* layer);
void s2_conv3d_free(s2_conv3d* layer);

/* VAE resampling layers, built from the weight-blob sequence their
 * load_model reads:
 *   S2_VAE_DOWNSAMPLE  VAEDownsample3D (vae_downsample3d.cpp:98-173): blob =
 *     channels, pad_right, pad_bottom, then one DecomposedConv3D (16 config
 *     values, bias when bias_term, kernels); zero padding on the right /
 *     bottom, then the convolution.
 *   S2_VAE_UPSAMPLE    VAEUpsample3D (vae_upsample3d.cpp:191-320): blob =
 *     channels, temporal_ratio, spatial_ratio, remove_temporal_head, then the
 *     post and the upscale DecomposedConv3D; upscale conv, pixel / temporal
 *     shuffle (frame 1 dropped unless the memory is ACTIVE when the temporal
 *     ratio is 2), post conv.
 * Same shapes, memory states and -1 cases as the reference layers. */
#define S2_VAE_DOWNSAMPLE 0
#define S2_VAE_UPSAMPLE 1
typedef struct s2_vae_resample s2_vae_resample;
int s2_vae_resample_create(s2_context* ctx, int kind, const float* blob, size_t count, s2_vae_resample** out);
int s2_vae_resample_output_shape(const s2_vae_resample* layer, int w, int h, int d, int memory_state, int* out_whdc);
int s2_vae_resample_forward(s2_vae_resample* layer, const float* in, int64_t in_cstep, int w, int h, int d, int c,
                            int memory_state, float* out, int64_t out_cstep);
/* reset_temporal_memory of every convolution inside (vae_downsample3d.cpp:139-143,
 * vae_upsample3d.cpp:250-256). */
void s2_vae_resample_reset_memory(s2_vae_resample* layer);
void s2_vae_resample_free(s2_vae_resample* layer);

/* VAEChunkedMHA (vae_chunked_mha.h, load_param / load_model :109-135, CPU
 * forward :197-217): self-attention of x [tokens][embed_dim]; weights host
 * fp32 in load_model order (q w [E][E], q b [E], k w, k b, v w, v b, out w,
 * out b); scale as param 6 (the reference's default 1/sqrt(E / heads)).
 * This build: one head (the VAE's), embed_dim a multiple of 8.  x and out are
 * device fp32 [tokens][embed_dim]. */
typedef struct s2_vae_mha s2_vae_mha;
int s2_vae_mha_create(s2_context* ctx, int embed_dim, int num_heads, float scale, const float* weights,
                      s2_vae_mha** out);
int s2_vae_mha_forward(s2_vae_mha* layer, const float* x, int tokens, float* out);
void s2_vae_mha_free(s2_vae_mha* layer);

/* VAE runtime around the encoder / decoder graphs (SeedVR2VAE, seedvr2_vae.h
 * :17-43).  The graphs are exported .param/.bin files outside the reference
 * tree; these are the runtime's own steps.
 *
 * s2_vae_temporal_segments: extract_temporal_slices (seedvr2_vae.cpp:408-451)
 * -- the graph runs over frames [start, start + count) with temporal-memory
 * state S2_VAE_MEMORY_*: one DISABLED run when frames <= first, else a first
 * run of `first` frames (INITIALIZING) and runs of `active` frames (ACTIVE).
 * The encoder uses first 5, active 4; the decoder first 2 (1 under the
 * reference's SEEDVR2_VAE_DECODER_FIRST_ONE), active 1.  Writes up to
 * `capacity` (start, count, state) triples and returns the number of runs, or
 * -1 for invalid arguments.
 * s2_vae_encode_frames / s2_vae_decode_frames: the latent frames of a video
 * ((frames - 1) / 4 + 1; more than five frames must be 4n + 1, else -1) and
 * the video frames of a latent ((frames - 1) * 4 + 1), as encode_moments and
 * decode check them (:551-565, :578-599). */
#define S2_VAE_SCALING_FACTOR 0.9152f
int s2_vae_temporal_segments(int frames, int first, int active, int capacity, int* segments);
int s2_vae_encode_frames(int frames);
int s2_vae_decode_frames(int latent_frames);
/* moments_to_latent (seedvr2_vae.cpp:454-478): moments fp32 [32][d][h][w] on
 * the device (16 mean channels, then 16 log-variance channels) -> latent fp32
 * [16][d][h][w] = (mean + exp(0.5 clamp(logvar, -30, 20)) * noise) * 0.9152,
 * or mean * 0.9152 when noise is NULL (sample_posterior false).  noise: fp32
 * [16][d][h][w] device standard normals; s2_vae_posterior_noise writes the
 * reference's sequence for a seed into host memory (std::mt19937_64(seed),
 * std::normal_distribution<float>(0, 1), channel-major; the reference's
 * default seed is 666). */
int s2_vae_posterior_noise(uint64_t seed, int64_t count, float* out_host);
int s2_vae_moments_to_latent(s2_context* ctx, const float* moments, int w, int h, int d, const float* noise,
                             float* latent);
/* decode's unscaling (seedvr2_vae.cpp:583-587): latent /= 0.9152 in place
 * (device fp32, correctly rounded division as the reference's). */
int s2_vae_unscale_latent(s2_context* ctx, float* latent, int64_t count);

/* ---------------------------------------------------------------------------
 * Multi-GPU (one process per GPU over NVLink).  The reference has no
 * distributed path (seedvr2_main.cpp:89-100 forces --sp-size 1); this is the
 * window sharding of the B200 build.
 *
 * Ownership of one sample over `world` ranks: rank r owns a token-balanced
 * contiguous range of the UNSHIFTED plan's token order (window after window);
 * text tokens are replicated.  Each window of a block (unshifted in even
 * blocks, shifted in odd blocks) belongs to the rank holding most of its
 * tokens; the QKV projection stores the packed q/k/v rows of foreign tokens
 * straight into the owner's buffer and attention stores their context rows
 * back (NVLink peer memory); every rank sums the text-pool partials of all
 * peers.  NCCL only exchanges the ids and memory handles at setup.
 * s2_shard_* expose the plan (host only, no GPU needed): local_tokens
 * [n_local] global token ids in local row order; for window plan `shifted`
 * (0/1), send_tokens / recv_tokens concatenated over peer ranks in rank order
 * (counts from s2_shard_counts). */
int s2_shard_build(const int* video_shape, int text_length, const int* window, int window_mode, int rank, int world,
                   s2_shard** out);
int s2_shard_counts(const s2_shard* shard, int shifted, int* n_local, int* send_counts, int* recv_counts);
int s2_shard_lists(const s2_shard* shard, int shifted, int* local_tokens, int* send_tokens, int* recv_tokens);
/* The windows of plan `shifted` whose attention this rank computes, as plan
 * window indices in ascending order: *count always, windows[] when non-null.
 * Owners are balanced by the attention kernel's work per window (sharding
 * is this library's addition; the reference runs one device). */
int s2_shard_windows(const s2_shard* shard, int shifted, int* count, int* windows);
void s2_shard_free(s2_shard* shard);

/* NCCL: rank 0 makes a 128-byte id and shares it out of band; every rank then
 * calls s2_dist_init on its context.  The communicator is non-blocking and
 * every host wait on it is bounded by timeout_ms: on expiry it is aborted and
 * the call returns S2_ERR_TIMEOUT.  s2_dist_sync waits (bounded) for the
 * context stream. */
int s2_dist_unique_id(void* id128);
int s2_dist_init(s2_context* ctx, const void* id128, int rank, int world, int timeout_ms);
int s2_dist_sync(s2_context* ctx);
int s2_dist_destroy(s2_context* ctx);

/* The cross-GPU barrier of the sharded forward (no counterpart in the
 * reference, whose layers never span GPUs): one warp stores `epoch` into
 * slot `rank` of every rank's flag array (peer_flags[i], device or peer
 * memory, 4-byte aligned, world <= 8) and waits until every slot of its own
 * flags (my_flags[0..world)) holds at least `epoch`.  The wait is bounded
 * (2 s of device time): on expiry the kernel records a timeout and returns,
 * and s2_status reports S2_ERR_TIMEOUT -- the context stays usable. */
int s2_peer_barrier(s2_context* ctx, void* const* peer_flags, uint32_t* my_flags, int rank, int world,
                    uint32_t epoch);

/* Sharded forward of all blocks for ONE sample on this rank (collective: every
 * rank calls it with the same shape).  x_local: fp32 [n_local + Nt][D] -- the
 * rank's own video rows in s2_shard local order, then all text rows -- updated
 * in place.  modulation: fp32 [6][D] device. */
int s2_dit_forward_sharded(s2_dit* dit, const int* video_shape, int text_length, float* x_local,
                           const float* modulation);

#ifdef __cplusplus
}
#endif

#endif
