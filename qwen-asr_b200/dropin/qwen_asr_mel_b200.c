/*
 * qwen_asr_mel_b200.c - drop-in for the reference's qwen_mel_spectrogram
 * (qwen_asr_audio.c:293-390, declared qwen_asr_audio.h:32), backed by
 * libqwen_asr_b200.so: same signature, same malloc'd [128, n_frames] result
 * that the caller frees, NULL (with the reference's message) when the audio
 * is too short.
 *
 * qwen_asr_audio.c also holds the WAV / PCM readers, so it stays in the
 * build; compile it with -Dqwen_mel_spectrogram=qwen_mel_spectrogram_cpu so
 * that its own definition is renamed and this one is linked in its place.
 * Runs on the current CUDA device (QWEN_B200_DEVICE picks it, default 0).
 */
#include "qwen_asr_audio.h"
#include "qwen_asr_b200.h"

#include <stdio.h>
#include <stdlib.h>

float *qwen_mel_spectrogram(const float *samples, int n_samples, int *out_frames) {
    if (qdb_mel_frames(n_samples) <= 0) {
        fprintf(stderr, "qwen_mel_spectrogram: audio too short (%d samples)\n", n_samples);
        return NULL;
    }
    float *mel = qdb_mel_spectrogram(samples, n_samples, out_frames);
    if (!mel) fprintf(stderr, "qwen_mel_spectrogram: %s\n", qdb_last_error());
    return mel;
}
