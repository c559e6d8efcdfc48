/* CPU oracle: a plain-C restatement of the SeedVR2 DiT block hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg call it as the checker; the shipped library never links
 * or calls it.  Every function cites the reference code it restates
 * (paths relative to the reference checkout).
 *
 * Parity pin: the restatement is checked bit-for-bit (plan) and to fp32
 * rounding (AWA, SharedLinear) against the reference's OWN layer sources
 * compiled into oracle/_ref/libs2_ref.so (see oracle/Makefile), and against
 * the committed golden fixtures in tests/golden/.
 */
#ifndef S2_ORACLE_H
#define S2_ORACLE_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* window_mode for the plan */
#define S2O_WINDOW_TARGET 0 /* reference: tuple = target window COUNT */
#define S2O_WINDOW_EXTENT 1 /* extension: tuple = window extent (t,h,w) */

/* Plan sizes. Returns 0, -1 (bad shape/target). */
int s2o_plan_sizes(const int* shapes, int batch, int window_mode, const int* window, int shifted,
                   int* num_windows, int* num_tokens);

/* Fills the plan arrays (capacities from s2o_plan_sizes).
 * windows: 9 ints per window (sample, t0,t1,h0,h1,w0,w1, partition_offset, token_count).
 * Returns 0, -1 (bad shape), -2 (inconsistent plan). */
int s2o_plan_build(const int* shapes, int batch, int window_mode, const int* window, int shifted,
                   int* windows, int* sample_window_count, int* video_indices, int* inverse_video_indices,
                   int* local_positions);

float s2o_round_bf16(float v);

/* AdaptiveWindowAttention forward in fp32.
 * iparams: heads, head_dim, window0..2, shifted, rope_pairs, window_mode, official_bf16_attention
 * norms: [4][head_dim] video_q, video_k, text_q, text_k;  freqs: [rope_pairs]
 * vq/vk/vv: row pointers' base + row stride (elements) for video, same for text.
 * video_out [Nv][inner], text_out [Nt][inner] (fully overwritten). */
int s2o_awa_forward(const int* iparams, float epsilon, const float* norms, const float* freqs,
                    const int* shapes, const int* text_lengths, int batch,
                    const float* vq, const float* vk, const float* vv, int v_ld,
                    const float* tq, const float* tk, const float* tv, int t_ld,
                    float* video_out, float* text_out);

/* out[m][n] = sum_k a[m][k] * w[n][k] + bias[n] (bias may be NULL). */
void s2o_linear(const float* a, int m, int k, const float* w, const float* bias, int n, float* out);

/* Block restatement; see s2_oracle.c for the op sequence.
 * dims: D (hidden), heads, head_dim, F (mlp), rope_pairs, window_mode, window0..2, shifted
 * x_video [Nv][D] and x_text [Nt][D] are updated in place (fp32 residual). */
typedef struct
{
    const float* ada;     /* [6][D] per-block modulation offsets */
    const float* w_qkv;   /* [3D][D] */
    const float* b_qkv;   /* [3D] or NULL */
    const float* w_out;   /* [D][D] */
    const float* b_out;   /* [D] or NULL */
    const float* w_up;    /* [F][D] */
    const float* b_up;    /* [F] or NULL */
    const float* w_down;  /* [D][F] */
    const float* b_down;  /* [D] or NULL */
    const float* qk_norm; /* [4][head_dim] */
    const float* freqs;   /* [rope_pairs] */
} s2o_block_weights;

int s2o_block_forward(const int* dims, float eps_norm, float eps_qk, const s2o_block_weights* wts,
                      const float* modulation /* [6][D] */, const int* shapes, const int* text_lengths,
                      int batch, float* x_video, float* x_text, int emulate_bf16);

/* Token formats around the block stack (src/seedvr2/seedvr2_dit.cpp).
 * shapes: latent (t, h, w) per sample.  Return 0 or -1 (bad shape / rows). */
int s2o_patch_rows(const int* shapes, int batch, long* tokens, long* patches);
/* [tokens][33] -> [patches][132] (patchify_video, :167-230) */
int s2o_patchify_video(const float* src, int rows, const int* shapes, int batch, float* dst);
/* [patches][64] -> [tokens][16] (unpatchify_prediction, :255-326) */
int s2o_unpatchify_prediction(const float* src, int rows, const int* shapes, int batch, float* dst);
/* [batch][256] sinusoidal embedding (make_timestep_embedding, :232-253) */
int s2o_timestep_embedding(const float* timesteps, int batch, float* out);

/* Denoise loop pieces (src/seedvr2/seedvr2_pipeline.cpp); latents are 16
 * channel planes of `tokens` values with plane stride cstep. */
void s2o_assemble_dit_input(const float* latent, long latent_cstep, const float* condition, long condition_cstep,
                            long tokens, float* out);
void s2o_apply_cfg(const float* pos, const float* neg, long count, float scale, float rescale, float* cfg);
void s2o_euler_update(float* latent, long cstep, long tokens, const float* pred, float delta);
void s2o_denoise_schedule(int steps, int step, float* timestep, float* delta);

/* VAE DecomposedConv3D (src/seedvr2/decomposed_conv3d.cpp:399-765); cfg is
 * the layer's 16-value config blob.  out_dims = (ow, oh, t_out, co). */
int s2o_conv3d_dims(const int* cfg, int w, int h, int d, int prefix, int* out_dims);
int s2o_conv3d_forward(const int* cfg, const float* bias, const float* weights, const float* in, int w, int h, int d,
                       const float* mem, int mem_frames, float* out, float* next_mem);

/* VAEChunkedMHA's CPU path (vae_chunked_mha.cpp:197-217): ncnn
 * MultiHeadAttention, self-attention over x [T][E]; w = q w, q b, k w, k b,
 * v w, v b, out w, out b (weights [E][E], out = in features last). */
int s2o_mha_forward(int E, int heads, float scale, const float* w, const float* x, int T, float* out);

#ifdef __cplusplus
}
#endif

#endif
