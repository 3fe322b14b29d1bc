/* Drop-in provider interface of the VocalArc separation host, implemented by
 * libvocalarc_b200.so (hand-written sm_100a kernels).
 *
 * These declarations must stay identical to the reference's
 * native/native_gpu.h so that native/vocalarc_separation.c compiles and links
 * against this library unchanged.  Each entry cites the reference interface
 * it replaces; the behaviour contract (return 1 = handled, 0 = not handled so
 * the host recomputes on the CPU; never write to stdout) is the reference's.
 */
#ifndef VOCALARC_NATIVE_GPU_H
#define VOCALARC_NATIVE_GPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct native_gpu native_gpu;

/* native_gpu.h:14 -- NULL when no sm_100 device is usable or VOCALARC_GPU is
   "off"/"cpu"; the host then stays on its CPU path. */
native_gpu *native_gpu_create(void);
/* native_gpu.h:15 */
void native_gpu_destroy(native_gpu *gpu);

/* native_gpu.h:17-19 -- per-call host matmul.  Like the reference's fused
   provider (native_gpu_cuda.cu:601-610) this returns 0: band-split and mask
   projections run on the device only inside the resident/extension paths. */
int native_gpu_matmul(native_gpu *gpu, int64_t rows, int in, int out,
                      const float *input, const float *packed_weight,
                      const float *bias, float *output);

/* native_gpu.h:21-22 -- static strings, NULL-safe. Backend is
   "native-cuda-sm100a" when enabled, "native-cpu" otherwise. */
const char *native_gpu_backend(const native_gpu *gpu);
const char *native_gpu_device(const native_gpu *gpu);

/* native_gpu.h:27-28 -- full axial batches; the memory guard uses the free
   device memory and honours VOCALARC_GPU_FULL_BATCHES=0/false/off. */
int native_gpu_uses_full_batches(const native_gpu *gpu);
int native_gpu_can_use_full_batches(const native_gpu *gpu, int frames);

/* native_gpu.h:30-41 -- host pointers into the model blob, 32-lane packed. */
typedef struct {
    const float *gamma;
    const float *qkv;
    const float *gate_weight;
    const float *gate_bias;
    const float *out_weight;
    const float *ff_gamma;
    const float *ff1_weight;
    const float *ff1_bias;
    const float *ff2_weight;
    const float *ff2_bias;
} native_gpu_transformer_weights;

/* native_gpu.h:46-49 -- one block on host data [sequences][length][256],
   updated in place; the scratch pointers are not used. */
int native_gpu_transformer(native_gpu *gpu, int sequences, int length,
                           float *data, float *normed, float *qkv,
                           float *attention_output, float *gates,
                           const native_gpu_transformer_weights *weights);

/* native_gpu.h:53-58 -- resident session: begin uploads [sequences][length][256];
   transformer requires sequences*length == resident tokens and a layout the
   session holds; transpose swaps the logical axes (no data movement on the
   device); end downloads the current logical layout and ends the session. */
int native_gpu_resident_begin(native_gpu *gpu, int sequences, int length,
                              const float *data);
int native_gpu_resident_transformer(native_gpu *gpu, int sequences, int length,
                                    const native_gpu_transformer_weights *weights);
int native_gpu_resident_transpose(native_gpu *gpu, int sequences, int length);
int native_gpu_resident_end(native_gpu *gpu, float *data);

/* native_gpu.h:60-67 */
typedef struct {
    const float *first_weight;
    const float *first_bias;
    const float *second_weight;
    const float *second_bias;
    int input_dim;
    int first_frequency;
} native_gpu_mask_band;

/* native_gpu.h:71-73 -- final RMSNorm + 90 mask MLPs on the resident
   features; writes the full host mask [1025][2][frames][2] and ends the
   session on success. */
int native_gpu_resident_mask(native_gpu *gpu, int frames, const float *final_gamma,
                             float *mask, const native_gpu_mask_band *bands,
                             int band_count);

#ifdef __cplusplus
}
#endif

#endif
