/* Additive extension of the provider interface (no counterpart in the
 * reference's native_gpu.h).
 *
 * The reference ABI stops at the transformer stack and the mask: the host
 * still runs the STFT (vocalarc_separation.c:1066), the band split (:917) and
 * the iSTFT (:1132) serially on the CPU.  These entry points run the complete
 * forward_model (vocalarc_separation.c:1342-1445) on the device -- STFT, band
 * split, 16 x 2 axial blocks, mask head, iSTFT -- and the chunked overlap-add
 * of the ONNX sidecar (Separator::demix, onnx/native/onnx_sidecar.cpp:725-782).
 *
 * All functions return 1 on success and 0 on failure (message on stderr),
 * like the reference provider.  Audio is planar float32 [2][length] at 44.1 kHz.
 */
#ifndef VOCALARC_B200_H
#define VOCALARC_B200_H

#include <stddef.h>
#include <stdint.h>

#include "native_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Provider bound to CUDA device `device` (native_gpu_create binds device 0,
   or VOCALARC_GPU_DEVICE when set). NULL when the device is not sm_100. */
native_gpu *vocalarc_b200_create(int device);

/* Parse a VSCNAT01 pack (layout of model_parse, vocalarc_separation.c:528-589)
   and keep every weight resident on the device in its kernel layout. The blob
   is not retained. */
int vocalarc_b200_load_model(native_gpu *gpu, const void *pack, size_t bytes);

/* The same from a pack file, read through mmap (no copy of the file in memory). */
int vocalarc_b200_load_model_file(native_gpu *gpu, const char *path);

/* Load fast path.  load_model lays out every device pointer first, then takes
   the converted weights (16-bit K-major, gammas folded, mask rows interleaved:
   the exact bytes of the device allocation) from an image file keyed by the
   pack's content hash and the precision, or converts them on several threads
   (VOCALARC_B200_LOAD_THREADS) and writes that file.  Images live in
   VOCALARC_B200_IMAGE_CACHE ("off" disables), else $XDG_CACHE_HOME/vocalarc-b200,
   else $HOME/.cache/vocalarc-b200.  model_from_cache: 1 when the last load used
   an image.  model_image builds the image on the host alone (no GPU; out NULL
   queries the size); store_model_image writes it to the cache directory ahead
   of the first load and returns its path. */
int vocalarc_b200_model_from_cache(const native_gpu *gpu);
int vocalarc_b200_model_image(const void *pack, size_t bytes, int bf16, int threads, void *out, size_t capacity,
                              size_t *image_bytes);
int vocalarc_b200_store_model_image(const void *pack, size_t bytes, int bf16, char *path_out, int capacity);

/* Whole-clip forward: frames = length/512 + 1, exactly forward_model. */
int vocalarc_b200_separate(native_gpu *gpu, const float *audio, int length, float *vocals);

/* Chunked forward: reflect border, chunks of chunk_samples (<= 0 selects
   881559) at step chunk/2, native forward per chunk, linear fade over the last
   chunk/10 samples, weights of the first and final predict batch forced to 1
   (model_batch = the ONNX model's batch size, 1 or 2), divide, crop. */
int vocalarc_b200_separate_chunked(native_gpu *gpu, const float *audio, int length,
                                   int chunk_samples, int model_batch, float *vocals);

/* The ONNX sidecar's quality pass (Separator::separate, onnx/native/onnx_sidecar.cpp:556-575;
   bigshift :784-790): the chunked forward of `bigshifts` circularly rotated copies of the
   mix (shift = length / bigshifts), each rotated back and averaged; with tta != 0 also of
   the channel-swapped and the polarity-flipped mix, combined as the reference does,
   ((v + swapped back) - (-(flipped))) / 3.  All copies run as one batch on the device. */
int vocalarc_b200_separate_tta(native_gpu *gpu, const float *audio, int length, int chunk_samples,
                               int model_batch, int bigshifts, int tta, float *vocals);

/* One clip's whole-clip forward split across `count` providers, normally one
   per GPU of one node, for the latency of a single clip (sequence parallelism;
   no counterpart in the reference).  Every provider must have the same pack
   loaded (checked by its content hash) at the same precision.
   Provider r runs the time-axis blocks for bands [90 r/count, 90 (r+1)/count)
   and the band-axis blocks for frames [T r/count, T (r+1)/count); between the
   axes the rows cross by 2-D peer copies ordered with CUDA events (x, its
   16-bit copy and the row RMSNorm factor), so the result equals
   vocalarc_b200_separate on provider 0 bit for bit.  Provider 0 runs the STFT,
   band split, mask head and iSTFT.  Host buffers; returns when vocals is
   written.  sp_plan lists the copies of one exchange (phase 0: scatter from
   provider 0, 1: band to frame ranges, 2: frame to band ranges, 3: gather to
   provider 0) as 8 values each: source, destination, source row, source pitch,
   destination row, destination pitch, width, height (in token rows); it
   returns the count, or -1. */
int vocalarc_b200_separate_sp(native_gpu *const *gpus, int count, const float *audio, int length, float *vocals);
int vocalarc_b200_sp_plan(int count, int frames, int phase, long long *out, int capacity);

/* Batch separation of WAV files with the file I/O off the critical path: a
   reader thread decodes track i+1 and a writer thread writes track i-1 while
   the device separates track i (whole-clip forward, or chunked when chunked
   != 0).  Inputs are read like the reference host reads them (wav_read,
   to_stereo, resample_linear: PCM 16/24/32-bit or float32, mono or stereo,
   any rate, resampled linearly to 44.1 kHz; vocalarc_separation.c:1152-1222);
   outputs are float32 stereo 44.1 kHz WAVs with non-finite samples written as
   0 (wav_write :1224-1237): vocals_paths[i] and, when instrumental_paths and
   its entry are non-NULL and non-empty, instrumental = mix - vocals
   (:1587-1593).  Returns the number of tracks whose outputs were written;
   failures are reported on stderr. */
int vocalarc_b200_separate_files(native_gpu *gpu, int count, const char *const *input_paths,
                                 const char *const *vocals_paths, const char *const *instrumental_paths,
                                 int chunked);
/* The reader stage alone (host only, no GPU): the decoded planar stereo
   44.1 kHz track of `path` into out[2][*length]; out NULL only sets *length;
   0 when unreadable or capacity < 2 * length floats.  write_track is the
   writer stage: float32 stereo 44.1 kHz, non-finite samples as 0. */
int vocalarc_b200_read_track(const char *path, float *out, long long capacity, int *length);
int vocalarc_b200_write_track(const char *path, const float *audio, int length);

/* Device-pointer variants on the provider's stream; they return after
   enqueueing (call vocalarc_b200_synchronize).  `tracks` planar clips of
   `length` samples each are laid out back to back ([tracks][2][length]). */
int vocalarc_b200_separate_device(native_gpu *gpu, const float *d_audio, int tracks, int length,
                                  int chunked, int chunk_samples, int model_batch, float *d_vocals);
int vocalarc_b200_synchronize(native_gpu *gpu);
/* The provider's cudaStream_t, for callers that order their own work after it. */
void *vocalarc_b200_stream(native_gpu *gpu);
/* First device-side error code recorded by a kernel (0 = none) and clears it. */
int vocalarc_b200_take_device_error(native_gpu *gpu);
/* 0 = fp16 operands (default), 1 = bf16 operands; both accumulate in fp32. */
int vocalarc_b200_set_precision(native_gpu *gpu, int bf16);

/* ---- One track's chunks sharded across GPUs (one provider per GPU).
   The chunk plan of vocalarc_b200_separate_chunked is split into contiguous
   ranges of at least two chunks.  A range owns the padded samples
   [chunk_begin * step, chunk_end * step) (the last range: to the padded end);
   only its seam -- the partial overlap-add sums of the `seam` = chunk - step
   samples its last chunk reaches past that -- crosses to the next range, by a
   peer copy over NVLink.  The merged output is bit-identical to
   vocalarc_b200_separate_chunked.  Sequence per range:
     range_forward -> (next range: seam_import or seam_from) -> range_finish. */

/* Chunk plan for a track of `length` samples (chunk_samples <= 0 selects 881559). */
int vocalarc_b200_chunk_plan(int length, int chunk_samples, int *chunks, int *step, int *border,
                             int *seam);
/* Forward of chunks [chunk_begin, chunk_end) of the device track d_audio
   ([2][length]); keeps the chunk outputs and computes this range's seam.
   Returns after the seam is complete on the device. */
int vocalarc_b200_range_forward(native_gpu *gpu, const float *d_audio, int length, int chunk_samples,
                                int model_batch, int chunk_begin, int chunk_end);
/* Output samples [*s0, *s1) this range writes in range_finish. */
int vocalarc_b200_range_owned(const native_gpu *gpu, int *s0, int *s1);
/* CUDA IPC handle (64 bytes) of this range's seam, for the next range's
   process.  The seam stays valid until this provider's next range_forward. */
int vocalarc_b200_range_seam_export(native_gpu *gpu, void *handle);
/* Copies the previous range's seam from its exported handle (another process,
   any GPU of the node) into this GPU's memory.  The handle's mapping is kept
   for later imports of the same handle (the exporter keeps its seam buffer
   while its range geometry does not grow) and released when a different
   handle arrives or this provider is destroyed. */
int vocalarc_b200_range_seam_import(native_gpu *gpu, const void *handle);
/* Same, from a provider of this process (same or another GPU). */
int vocalarc_b200_range_seam_from(native_gpu *gpu, const native_gpu *prev);
/* Writes this range's output samples into the device buffer d_vocals
   ([2][length]); other samples are not touched. */
int vocalarc_b200_range_finish(native_gpu *gpu, float *d_vocals);

/* Number of kernels this provider has launched (all streams it owns). */
long long vocalarc_b200_launch_count(const native_gpu *gpu);
/* Launch trace: after trace_begin every launch records a CUDA event on the
   provider stream; trace_end synchronises and writes one line per kernel,
   "name<TAB>launches<TAB>total_ms", where a launch's time is the gap to the
   previous event (the stream runs launches back to back). trace_mark adds a
   named boundary, e.g. after a copy the caller enqueued on the stream. */
int vocalarc_b200_trace_begin(native_gpu *gpu);
int vocalarc_b200_trace_mark(native_gpu *gpu, const char *what);
int vocalarc_b200_trace_end(native_gpu *gpu, char *out, int capacity);

/* ---- stage entry points (device pointers, provider stream) used by the
   parity tests to check each kernel against the CPU oracle ---- */

/* C[M][N] = A[M][K] * B[N][K]^T (16-bit A, B), epilogue 0 = 16-bit store
   (+bias), 1 = bias+GELU, 6 = fp32 store.  M >= 1, N % 256 == 0, K % 64 == 0. */
int vocalarc_b200_stage_gemm(native_gpu *gpu, int epilogue, const void *a, const void *b, int m, int n,
                             int k, const float *bias, void *out);
/* Gated attention over qkv [rows][1536] (16-bit, RoPE already applied),
   gates [rows][8]; rows = d3*d2*d1 tokens; positions along dim `pos_dim`
   (1 or 2) of the (d1, d2, d3) token grid. Writes out [rows][512]. */
int vocalarc_b200_stage_attention(native_gpu *gpu, const void *qkv, const float *gates, void *out,
                                  int d1, int d2, int d3, int pos_dim);
/* STFT of `segments` whole clips [segments][2][length] -> spec [segments][T][1025][2][2]. */
int vocalarc_b200_stage_stft(native_gpu *gpu, const float *audio, int segments, int length, float *spec);
/* iSTFT of spec*mask (both [segments][T][1025][2][2]) -> [segments][2][length]. */
int vocalarc_b200_stage_istft(native_gpu *gpu, const float *spec, const float *mask, int segments,
                              int length, float *audio);
/* Same result as vocalarc_b200_stage_istft, but allocates no device memory,
   for callers that cannot call cudaMalloc while they process audio (a
   real-time audio thread such as a plugin's process callback, where a call
   that can block or synchronise the device is not allowed, or an application
   whose GPU memory budget is fixed when it loads the library).  No
   counterpart in the reference.  The frame scratch is a fixed 32 MiB device
   array that every GPU which loads this library holds (from its first call on
   that device at the latest) until the process exits; it serves at most segments * (length/512 + 1) <= 2048 frames (one
   881,559-sample chunk), and larger requests are refused (return 0 with a
   message on stderr).  The first call on a device looks up the array's device
   address (cudaGetSymbolAddress) and should come before any stream capture.
   All calls share that array and it keeps the last call's contents: calls
   that can overlap on the GPU (other streams, other host threads) race. */
int vocalarc_b200_stage_istft_noalloc(native_gpu *gpu, const float *spec, const float *mask, int segments,
                                      int length, float *audio);
/* Check of the kernels' bounded waits (no counterpart in the reference): one
   CTA waits, with the tcgen05 kernels' own wait loop limited to limit_us
   microseconds (1 .. 100000), on an mbarrier for a copy that is never issued.
   The wait runs out, the kernel records its error code and returns, and the
   call then fails the way a kernel wait timeout fails inside a forward:
   message on stderr, provider disabled, 0 returned.  Nothing is left in
   flight, so the CUDA context stays usable.  -1 for a limit out of range. */
int vocalarc_b200_stage_wait_check(native_gpu *gpu, int limit_us);
/* Band split of spec (loaded model) -> x [segments][90][T][256] fp32. */
int vocalarc_b200_stage_band_split(native_gpu *gpu, const float *spec, int segments, int frames, float *x);
/* One transformer block (loaded model, layer, axis 0 = time / 1 = band) in
   place on x [segments][90][T][256]. */
int vocalarc_b200_stage_block(native_gpu *gpu, float *x, int segments, int frames, int layer, int axis);
/* Final norm + mask head (loaded model): x -> mask [segments][T][1025][2][2]. */
int vocalarc_b200_stage_mask(native_gpu *gpu, const float *x, int segments, int frames, float *mask);

#ifdef __cplusplus
}
#endif

#endif
