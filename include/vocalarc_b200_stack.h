/* Configurable BS-RoFormer stack on sm_100a (additive; no counterpart in the
 * reference, whose only model is the bundled dim-256 / 90-band / hop-512 one).
 *
 * The stack is the bundled model's forward (forward_model,
 * vocalarc_separation.c:1342-1445) with its sizes made parameters: STFT with
 * hop `hop`, band split over `bands` bands into `dim` columns, `depth` layers
 * of a time-axis and a band-axis block (pre-norm RMSNorm, RoPE attention of
 * 8 heads x 64 with per-head sigmoid gates, FFN), final RMSNorm, per-band mask
 * MLPs (tanh, GLU) and the masked iSTFT.  The FFN is either the bundled
 * Linear -> exact GELU -> Linear, or GEGLU: the first Linear emits 2 * ff_inner
 * rows [value; gate] and h = value * gelu(gate) (Shazeer, "GLU Variants
 * Improve Transformer", 2020).  With the bundled sizes (dim 256, 90 bands of
 * the reference's table, hop 512, GELU, ff_inner 1024, mask_hidden 1024) it
 * computes the same forward as vocalarc_b200_separate.
 *
 * Weights are one float32 array of vocalarc_b200_stack_weight_count() floats,
 * every matrix logical row-major W[out][in] (no 32-lane packing), in this order:
 *   for layer in 0..depth-1, for axis in (time, band):
 *     attn_gamma[dim], qkv[1536][dim], gate_w[8][dim], gate_b[8],
 *     out[dim][512], ff_gamma[dim], ff1[F1][dim], ff1_b[F1],
 *     ff2[dim][ff_inner], ff2_b[dim]            (F1 = ff_inner, x2 with GEGLU)
 *   for band: gamma[4 w_b], weight[dim][4 w_b], bias[dim]
 *   final_gamma[dim]
 *   for band: w1[mask_hidden][dim], b1[mask_hidden],
 *             w2[8 w_b][mask_hidden], b2[8 w_b]
 * (w_b = band_bins[band]; the order is the VSCNAT01 pack's, model_parse
 * vocalarc_separation.c:528-589, without the u64 count prefixes.)
 *
 * Functions returning int give 1 on success, 0 on failure (message on stderr).
 */
#ifndef VOCALARC_B200_STACK_H
#define VOCALARC_B200_STACK_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VOCALARC_B200_STACK_MAX_BANDS 128

typedef struct vocalarc_b200_stack_config {
  int dim;          /* residual width: 256 or 512 */
  int depth;        /* layers; each is a time-axis then a band-axis block */
  int heads;        /* 8 */
  int dim_head;     /* 64 */
  int ff_inner;     /* FFN hidden width: multiple of 256 (GELU) or of 128 (GEGLU) */
  int geglu;        /* 1 = GEGLU FFN, 0 = GELU FFN */
  int mask_hidden;  /* mask MLP hidden width, multiple of 256 */
  int bands;        /* 1..VOCALARC_B200_STACK_MAX_BANDS */
  int band_bins[VOCALARC_B200_STACK_MAX_BANDS]; /* bins per band (1..129), frequency order, sum n_fft/2+1 */
  int n_fft;        /* 2048 */
  int hop;          /* 1..2048; frames = length / hop + 1 */
  int bf16;         /* 1 = bf16 tensor-core operands, 0 = fp16 */
} vocalarc_b200_stack_config;

typedef struct vocalarc_b200_stack vocalarc_b200_stack;

/* Floats in the weight array for `cfg`; 0 when the configuration is not supported. */
size_t vocalarc_b200_stack_weight_count(const vocalarc_b200_stack_config *cfg);

/* Converts and uploads the weights to device `device`; the array is not retained.
   NULL when the configuration or count is invalid or the device is not sm_100. */
vocalarc_b200_stack *vocalarc_b200_stack_create(int device, const vocalarc_b200_stack_config *cfg,
                                                const float *weights, size_t count);
void vocalarc_b200_stack_destroy(vocalarc_b200_stack *stack);

/* Whole-clip forward of `clips` planar clips [clips][2][length] on device
   memory; enqueued on the stack's stream (call vocalarc_b200_stack_synchronize). */
int vocalarc_b200_stack_forward_device(vocalarc_b200_stack *stack, const float *d_audio, int clips, int length,
                                       float *d_vocals);
/* The same from and to host memory; returns when the vocals are written. */
int vocalarc_b200_stack_separate(vocalarc_b200_stack *stack, const float *audio, int clips, int length,
                                 float *vocals);

/* Stages on device memory (enqueued), for parity tests and microbenchmarks.
   spec / mask: frame-major [clips][T][1025][2 ch][re, im]; x: fp32
   [clips][bands][T][dim] (band-major tokens). */
int vocalarc_b200_stack_stage_stft(vocalarc_b200_stack *stack, const float *d_audio, int clips, int length,
                                   float *d_spec);
int vocalarc_b200_stack_stage_band_split(vocalarc_b200_stack *stack, const float *d_spec, int clips, int frames,
                                         float *d_x);
/* One axial block (axis 0 = time, 1 = band) of layer `layer` on d_x in place. */
int vocalarc_b200_stack_stage_block(vocalarc_b200_stack *stack, float *d_x, int clips, int frames, int layer,
                                    int axis);
/* Final RMSNorm and the mask MLPs: d_x -> d_mask. */
int vocalarc_b200_stack_stage_mask(vocalarc_b200_stack *stack, const float *d_x, int clips, int frames,
                                   float *d_mask);
/* Complex mask, inverse STFT and overlap-add -> [clips][2][length]. */
int vocalarc_b200_stack_stage_istft(vocalarc_b200_stack *stack, const float *d_spec, const float *d_mask, int clips,
                                    int length, float *d_audio);

int vocalarc_b200_stack_synchronize(vocalarc_b200_stack *stack);
void *vocalarc_b200_stack_stream(vocalarc_b200_stack *stack);
/* Device-side wait-timeout code recorded since the last call (0 = none); clears it. */
int vocalarc_b200_stack_take_device_error(vocalarc_b200_stack *stack);
long long vocalarc_b200_stack_launch_count(const vocalarc_b200_stack *stack);
/* Per-launch trace on the stack's stream: after trace_end, `out` holds one
   "name\tlaunches\tmilliseconds" line per kernel kind. */
int vocalarc_b200_stack_trace_begin(vocalarc_b200_stack *stack);
int vocalarc_b200_stack_trace_end(vocalarc_b200_stack *stack, char *out, int capacity);

#ifdef __cplusplus
}
#endif

#endif /* VOCALARC_B200_STACK_H */
