/* Flat C ABI of the B200 voice-detect engine (libvoicedetect_b200.so).
 *
 * Drop-in for the reference's frozen ABI, include/voicedetect_capi.h:31-89 of
 * mudler/voice-detect.cpp (implementation src/voicedetect_capi.cpp:61-176): the
 * same ten symbols with the same argument meaning, ownership and error
 * behaviour, so a consumer that dlopens libvoicedetect.so (LocalAI via purego)
 * can load this library instead. Additive entry points follow the reference's
 * rule that new functions need no ABI bump (voicedetect_capi.h:25-30).
 *
 * Conventions (unchanged from the reference):
 *  - status 0 = success, nonzero = error; the message is in
 *    voicedetect_capi_last_error(ctx) until the next call on ctx;
 *  - embed outputs are reset to NULL / 0 before any work; verify leaves its
 *    outputs unchanged on error;
 *  - returned vectors / strings are malloc'd and released with
 *    voicedetect_capi_free_vec / voicedetect_capi_free_string;
 *  - no C++ exception crosses the boundary.
 * Threading: a context owns a CUDA stream, device buffers and a lock; calls on one
 * context are serialised, calls on different contexts may run concurrently.
 * The model is placed on the CUDA device that is current when voicedetect_capi_load
 * is called.
 */
#ifndef VOICEDETECT_CAPI_H
#define VOICEDETECT_CAPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct voicedetect_ctx voicedetect_ctx;

/* ---- frozen v1 surface (reference include/voicedetect_capi.h) --------------- */

/* ref :31 */ int voicedetect_capi_abi_version(void);
/* ref :36 -- NULL on a missing/bad GGUF or when voicedetect.embedding_dim is absent */
voicedetect_ctx* voicedetect_capi_load(const char* gguf_path);
/* ref :39 -- safe on NULL */
void voicedetect_capi_free(voicedetect_ctx* ctx);
/* ref :45 -- "" for NULL ctx or no error */
const char* voicedetect_capi_last_error(voicedetect_ctx* ctx);
/* ref :49 */ void voicedetect_capi_free_string(char* s);
/* ref :53 */ void voicedetect_capi_free_vec(float* v);
/* ref :61 -- L2-normalised embedding of a WAV file */
int voicedetect_capi_embed_path(voicedetect_ctx* ctx, const char* wav_path, float** out_vec,
                                int* out_dim);
/* ref :67 -- mono f32 PCM; linearly resampled to 16 kHz when sample_rate != 16000 */
int voicedetect_capi_embed_pcm(voicedetect_ctx* ctx, const float* pcm, int n_samples,
                               int sample_rate, float** out_vec, int* out_dim);
/* ref :77 -- distance = 1 - cosine; verified = distance <= threshold */
int voicedetect_capi_verify_paths(voicedetect_ctx* ctx, const char* a, const char* b,
                                  float threshold, float* out_distance, int* out_verified);
/* ref :88 -- the wav2vec2 analyze heads are outside this engine: always returns NULL
 * with a last_error, as the reference does for a model without analyze heads
 * (src/model.cpp:81-84). */
char* voicedetect_capi_analyze_path_json(voicedetect_ctx* ctx, const char* wav_path);

/* ---- additive entry points --------------------------------------------------- */

/* Batched embed (the throughput path): n_clips mono f32 clips pcm[i] of
 * n_samples[i] samples at sample_rate; writes n_clips * dim floats to the caller's
 * `out` (row i = clip i, L2-normalised) and *out_dim = dim. Clips in page-locked
 * memory (cudaHostAlloc / cudaHostRegister) are copied to the GPU straight from the
 * caller's buffers; pageable clips are first gathered into the engine's pinned ring,
 * which costs host memory bandwidth. Results are identical either way. */
int voicedetect_capi_embed_pcm_batch(voicedetect_ctx* ctx, const float* const* pcm,
                                     const int* n_samples, int n_clips, int sample_rate,
                                     float* out, int* out_dim);

/* Identify: cosine of each of n_q queries [n_q][dim] against n_reg registry rows
 * [n_reg][dim]; writes the top-k registry indices (descending score, ties to the
 * lower index) to out_idx [n_q][k] and their cosines to out_score [n_q][k].
 * Host arrays. */
int voicedetect_capi_identify(voicedetect_ctx* ctx, const float* queries, int n_q,
                              const float* registry, int n_reg, int dim, int k, int* out_idx,
                              float* out_score);

/* Number of GPUs a context uses (1 <= n_gpus <= visible GPUs). For n_gpus > 1 the
 * model is loaded on the next n_gpus - 1 devices (after the one current at load)
 * and voicedetect_capi_embed_pcm_batch shards its clips over all of them (longest
 * clips first to the least loaded GPU), one host thread per GPU. Other calls use
 * the load device. */
int voicedetect_capi_set_devices(voicedetect_ctx* ctx, int n_gpus);

/* ---- B200-specific additive entry points --------------------------------------- */

/* Device-resident batched embed: clip i is d_pcm + offsets[i] (16 kHz f32,
 * n_samples[i] samples) in device memory; offsets / n_samples are host arrays;
 * embeddings go to device memory d_out [n_clips][dim]. Asynchronous on `stream`
 * (a cudaStream_t; NULL = the context's own stream). */
int voicedetect_b200_embed_device(voicedetect_ctx* ctx, const float* d_pcm,
                                  const long long* offsets, const int* n_samples, int n_clips,
                                  float* d_out, void* stream);

/* Batch embed of int16 mono clips (the samples a WAV file holds; value / 32768 is
 * the f32 the reference's drwav decode produces) at any sample rate: the int16
 * samples cross PCIe (half the bytes of f32) and are converted and, at rates other
 * than 16 kHz, linearly resampled on the GPU with the reference's resample_linear
 * arithmetic (src/audio_io.cpp:9-23; bitwise equal to the host result). Otherwise as
 * voicedetect_capi_embed_pcm_batch: out [n_clips][dim], status 0 / nonzero with
 * last_error. No reference counterpart (the reference decodes WAV to f32 on the host). */
int voicedetect_b200_embed_s16_batch(voicedetect_ctx* ctx, const int16_t* const* pcm,
                                     const int* n_samples, int n_clips, int sample_rate,
                                     float* out, int* out_dim);

/* The audio front door of embed_path / verify_paths on its own (reference
 * vd::load_audio_16k_mono, src/audio_io.cpp:25-38): decodes a WAV file (PCM u8 /
 * s16 / s24 / s32, IEEE float 32 / 64, mono or multi-channel), averages the
 * channels in f64 and linearly resamples to 16 kHz (src/audio_io.cpp:9-23).
 * *out_pcm receives a malloc'd buffer of *out_n samples (free it with
 * voicedetect_capi_free_vec); both are reset before work. Needs no context or GPU.
 * Status 0 / nonzero; a failure's message is returned by
 * voicedetect_b200_audio_error(). */
int voicedetect_b200_load_audio_16k_mono(const char* wav_path, float** out_pcm, int* out_n);

/* The message of this thread's last failed voicedetect_b200_load_audio_16k_mono
 * ("" after a success). */
const char* voicedetect_b200_audio_error(void);

/* Bucketing policy: at most max_clips clips and max_frames padded FBank frames
 * per batched pass (defaults 512 and 262144). */
int voicedetect_b200_set_bucketing(voicedetect_ctx* ctx, int max_clips, long long max_frames);

/* GPU kernels launched by the last embed call on ctx. */
long long voicedetect_b200_last_launches(voicedetect_ctx* ctx);

/* Device bytes held by the ResNet block conv weights: f16 values, or q8_0 int8 values
 * plus their f16 scales (q8_0 GGUF tensors stay q8_0 on the device: the convs with
 * resident weights expand them in shared memory, the others into one f16 scratch the
 * size of the largest conv, ~1.25 MB for ResNet34, not counted here), QPACK copies
 * included; 0 for other models or NULL. No reference counterpart. */
long long voicedetect_b200_conv_weight_bytes(voicedetect_ctx* ctx);

/* Page-lock `bytes` of the caller's host memory at `ptr` in place (for every device of
 * the process), so that the batch calls copy clips stored there straight to the GPU
 * instead of gathering them first; voicedetect_b200_host_unregister(ptr) undoes it
 * before the memory is freed. 0 on success; otherwise 1 with the reason in
 * vdb_last_error() (e.g. a locked-memory limit), and the memory stays usable as
 * pageable. No reference counterpart. */
int voicedetect_b200_host_register(void* ptr, size_t bytes);
int voicedetect_b200_host_unregister(void* ptr);

/* Embedding dimension of the loaded model (0 for NULL). */
int voicedetect_b200_embedding_dim(voicedetect_ctx* ctx);

/* Synchronise the context's stream and report any kernel-side timeout. */
int voicedetect_b200_sync(voicedetect_ctx* ctx);

/* Synchronise, then drop the context's captured CUDA graphs and free its workspace on
 * every device it uses (weights stay resident). The next embed call re-allocates
 * and re-captures; its results are bit-identical to those before the release.
 * No reference counterpart (the reference frees everything only in
 * voicedetect_capi_free). */
int voicedetect_b200_release_cache(voicedetect_ctx* ctx);

/* Conv-kernel profiling: while enabled, every tensor-core conv launch is bracketed
 * by CUDA events on its own stream. profile_read synchronises and returns, since
 * the previous read, the summed launch durations (ms), the algorithmic conv FLOPs
 * over valid frames (2*OC*IC*k*k*F_out*valid frames), and the number of launches. */
int voicedetect_b200_profile(voicedetect_ctx* ctx, int enable);
int voicedetect_b200_profile_read(voicedetect_ctx* ctx, double* conv_ms, double* conv_flops,
                                  long long* conv_launches);
/* The same read's summed launch durations (ms) by stage, written to ms[0 .. n-1] in
 * the order: convs, FBank, CMN + stem, TSTP + FC + L2, element-wise adds (ERes2Net).
 * No reference counterpart. */
int voicedetect_b200_profile_stages(voicedetect_ctx* ctx, double* ms, int n);
/* The conv launches of the same read, in launch order: for launch i, rec[12*i ..
 * 12*i+11] = duration (ms), algorithmic FLOPs, input channels, output channels, kernel
 * size, stride, output frequency bins, output frames, batch, the second input
 * segment's channels (0 for one segment), 1 when an epilogue residual is read, 1 for a QPACK conv. Writes at most n records; returns the
 * number of launches (so n = 0 sizes the buffer), or -1 for a NULL context. No
 * reference counterpart. */
int voicedetect_b200_profile_convs(voicedetect_ctx* ctx, double* rec, int n);

#ifdef __cplusplus
}
#endif
#endif
