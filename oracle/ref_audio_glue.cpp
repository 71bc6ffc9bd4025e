// extern "C" glue around the reference's OWN audio front door, compiled unmodified
// from the reference checkout by oracle/Makefile into oracle/_ref/libvdref.so:
//   vd::resample_linear        src/audio_io.cpp:9-23
//   vd::load_audio_16k_mono    src/audio_io.cpp:25-38 (dr_wav decode, f64 downmix,
//                              resample to 16 kHz)
//   drwav_open_file_and_read_pcm_frames_f32 (third_party/dr_wav.h, the decoder the
//                              reference vendors, compiled by src/audio_io.cpp's
//                              DR_WAV_IMPLEMENTATION)
//
// TEST INFRASTRUCTURE ONLY: tests/ use it to pin the product's WAV reader and
// device resampler bitwise. The product library never links or loads it.
#include "dr_wav.h"
#include "audio_io.hpp"

#include <cstdlib>
#include <cstring>
#include <vector>

extern "C" {

// vd::resample_linear on `n` samples. Writes min(result, cap) samples to `out` and
// returns the full result length.
long vdref_resample_linear(const float* in, long n, int in_sr, int out_sr, float* out, long cap) {
    std::vector<float> v(in, in + n);
    std::vector<float> r = vd::resample_linear(v, in_sr, out_sr);
    const long m = (long)r.size();
    if (out && cap > 0) std::memcpy(out, r.data(), sizeof(float) * (size_t)(m < cap ? m : cap));
    return m;
}

// vd::load_audio_16k_mono: 16 kHz mono samples of a WAV file. Returns the sample
// count (-1 when the file cannot be decoded) and writes up to `cap` samples.
long vdref_load_audio_16k_mono(const char* path, float* out, long cap) {
    vd::Audio a;
    if (!vd::load_audio_16k_mono(path, a)) return -1;
    const long m = (long)a.samples.size();
    if (out && cap > 0)
        std::memcpy(out, a.samples.data(), sizeof(float) * (size_t)(m < cap ? m : cap));
    return m;
}

// dr_wav's own f32 decode of every channel (interleaved), before any downmix or
// resampling. Returns the frame count (-1 on failure), the channel count and the
// sample rate; writes up to `cap` floats.
long vdref_drwav_decode_f32(const char* path, float* out, long cap, int* channels, int* sr) {
    unsigned int ch = 0, rate = 0;
    drwav_uint64 frames = 0;
    float* pcm = drwav_open_file_and_read_pcm_frames_f32(path, &ch, &rate, &frames, nullptr);
    if (!pcm) return -1;
    const long total = (long)(frames * ch);
    if (out && cap > 0) std::memcpy(out, pcm, sizeof(float) * (size_t)(total < cap ? total : cap));
    drwav_free(pcm, nullptr);
    if (channels) *channels = (int)ch;
    if (sr) *sr = (int)rate;
    return (long)frames;
}

}  // extern "C"
