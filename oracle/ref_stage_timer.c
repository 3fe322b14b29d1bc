/* Stage timer for the reference CPU forward (test and baseline infrastructure).
 *
 * Compiles the reference's native/vocalarc_separation.c in place (REF, read
 * only; oracle/Makefile target `timer`) with its JSONL main renamed, and times
 * the reference's own stage functions on one clip through the same calls and
 * groupings as forward_model (vocalarc_separation.c:1342-1445, CPU branch
 * :1407-1426): stft, band_split, the 16 x {time axis, band axis}
 * transformer_forward layer pairs with their transposes, inplace_norm +
 * mask_band, istft.
 *
 * A whole 881,559-sample chunk (T = 1722) takes minutes on a CPU, so the layer
 * pairs are sampled: each timed repetition runs ONE layer pair over the first
 * `--time-bands` bands on the time axis and the first `--band-frames` frames on
 * the band axis (multiples of the reference's own group sizes).  Every band
 * sequence and every frame of a block is independent and costs the same, so
 * the full layer pair is time_axis * 90 / bands + band_axis * T / frames; the
 * forward is front + 16 * layer pair + transposes + back.  The front (STFT, band
 * split) and back (final norm, mask, iSTFT) run in full once.
 *
 *   ref-stage-timer --model PACK --wav IN.wav [--threads N] [--reps R]
 *                   [--time-bands B] [--band-frames F] [--layer L]
 *
 * Output: one JSON object per line on stdout -- "front", one "layer" per
 * repetition, "back".  Nothing from the reference is copied here: the file
 * includes the reference source where it lies.
 */
#define main vocalarc_reference_main
#include "vocalarc_separation.c"
#undef main

int main(int argc, char **argv) {
    const char *model_path = NULL, *wav_path = NULL;
    int threads = 1, reps = 1, time_bands = BANDS, band_frames = -1, layer = 0;
    for (int i = 1; i + 1 < argc; i += 2) {
        if (strcmp(argv[i], "--model") == 0) model_path = argv[i + 1];
        else if (strcmp(argv[i], "--wav") == 0) wav_path = argv[i + 1];
        else if (strcmp(argv[i], "--threads") == 0) threads = atoi(argv[i + 1]);
        else if (strcmp(argv[i], "--reps") == 0) reps = atoi(argv[i + 1]);
        else if (strcmp(argv[i], "--time-bands") == 0) time_bands = atoi(argv[i + 1]);
        else if (strcmp(argv[i], "--band-frames") == 0) band_frames = atoi(argv[i + 1]);
        else if (strcmp(argv[i], "--layer") == 0) layer = atoi(argv[i + 1]);
    }
    if (model_path == NULL || wav_path == NULL || threads < 1 || reps < 0 || layer < 0 || layer >= DEPTH) {
        fprintf(stderr, "usage: ref-stage-timer --model PACK --wav IN.wav [--threads N] [--reps R] "
                        "[--time-bands B] [--band-frames F] [--layer L]\n");
        return 2;
    }
    select_simd();
    thread_pool *pool = pool_create(threads);
    if (pool == NULL) return 1;
    model network; memset(&network, 0, sizeof(network));
    if (!model_load(&network, model_path, argv[0])) return 1;
    wav_audio input = {0};
    if (!wav_read(wav_path, &input)) return 1;
    int length = 0;
    float *stereo = to_stereo(&input, &length);
    if (stereo == NULL || input.sample_rate != 44100) return 1;
    const int frames = length / HOP + 1;
    /* The JSONL host's automatic CPU groups (vocalarc_separation.c:1574-1577). */
    const int time_group = automatic_time_group(pool->count) > BANDS ? BANDS : automatic_time_group(pool->count);
    int frequency_group = automatic_frequency_group(pool->count);
    if (frequency_group < 1) frequency_group = 1;
    if (time_bands < time_group) time_bands = time_group;
    time_bands = (time_bands + time_group - 1) / time_group * time_group;
    if (time_bands > BANDS) time_bands = BANDS;
    if (band_frames <= 0 || band_frames > frames) band_frames = frames;
    band_frames = (band_frames + frequency_group - 1) / frequency_group * frequency_group;
    if (band_frames > frames) band_frames = frames;

    forward_buffers buffers; memset(&buffers, 0, sizeof(buffers));
    if (!prepare_buffers(&buffers, frames, length, time_group, frequency_group)) return 1;
    float frequencies[DIM_HEAD / 2]; fill_frequencies(frequencies);

    double t0 = monotonic_seconds();
    if (!stft(pool, stereo, length, frames, buffers.source, buffers.fft_buffer)) return 1;
    double t1 = monotonic_seconds();
    band_split(pool, &network, buffers.source, frames, buffers.time_sequences, buffers.input_scratch);
    double t2 = monotonic_seconds();
    printf("{\"stage\":\"front\",\"frames\":%d,\"length\":%d,\"threads\":%d,\"time_group\":%d,"
           "\"frequency_group\":%d,\"stft_s\":%.6f,\"band_split_s\":%.6f}\n",
           frames, length, pool->count, time_group, frequency_group, t1 - t0, t2 - t1);
    fflush(stdout);

    /* One layer pair per repetition, the body of forward_model's CPU loop on
       the sampled bands / frames, the transposes at full size. */
    const transformer_weights *w_time = &network.layers[layer][0];
    const transformer_weights *w_band = &network.layers[layer][1];
    for (int r = 0; r < reps; r++) {
        double a = monotonic_seconds();
        for (int first = 0; first < time_bands; first += time_group) {
            int count = first + time_group > time_bands ? time_bands - first : time_group;
            transformer_forward(pool, w_time, buffers.time_sequences + (size_t)first * frames * DIM, count, frames,
                                buffers.normed, buffers.qkv, buffers.attention_output, buffers.gates, frequencies);
        }
        double b = monotonic_seconds();
        transpose_from_time_sequences(pool, frames, buffers.time_sequences, buffers.features);
        double c = monotonic_seconds();
        for (int first = 0; first < band_frames; first += frequency_group) {
            int count = first + frequency_group > band_frames ? band_frames - first : frequency_group;
            transformer_forward(pool, w_band, buffers.features + (size_t)first * BANDS * DIM, count, BANDS,
                                buffers.normed, buffers.qkv, buffers.attention_output, buffers.gates, frequencies);
        }
        double d = monotonic_seconds();
        transpose_to_time_sequences(pool, frames, buffers.features, buffers.time_sequences);
        double e = monotonic_seconds();
        printf("{\"stage\":\"layer\",\"rep\":%d,\"time_bands\":%d,\"band_frames\":%d,\"time_axis_s\":%.6f,"
               "\"band_axis_s\":%.6f,\"transposes_s\":%.6f}\n",
               r, time_bands, band_frames, b - a, d - c, (c - b) + (e - d));
        fflush(stdout);
    }

    transpose_from_time_sequences(pool, frames, buffers.time_sequences, buffers.features);
    double m0 = monotonic_seconds();
    inplace_norm(pool, (int64_t)frames * BANDS, buffers.features, network.final_gamma);
    memset(buffers.mask, 0, (size_t)FREQ_BINS * CHANNELS * frames * 2 * sizeof(float));
    for (int band = 0; band < BANDS; band++)
        mask_band(&network, pool, frames, band, buffers.features, buffers.mask, buffers.normed, buffers.qkv,
                  buffers.attention_output);
    double m1 = monotonic_seconds();
    istft(buffers.source, buffers.mask, length, frames, buffers.audio_output, buffers.normalization,
          buffers.fft_buffer);
    double m2 = monotonic_seconds();
    printf("{\"stage\":\"back\",\"mask_s\":%.6f,\"istft_s\":%.6f}\n", m1 - m0, m2 - m1);
    fflush(stdout);
    free(stereo);
    free_buffers(&buffers);
    model_unload(&network);
    pool_destroy(pool);
    return 0;
}
