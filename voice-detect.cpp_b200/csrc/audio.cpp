// WAV decoding for embed_path / verify_paths: RIFF/WAVE with PCM u8 / s16 / s24 /
// s32, IEEE float 32/64, and WAVE_FORMAT_EXTENSIBLE wrapping those. Samples become
// f32 exactly as the reference's decoder (its vendored dr_wav, third_party/dr_wav.h)
// converts them: s16 * 2^-15 and s24 * 2^-23 (exact scalings), s32 / 2^31 in f64,
// u8 as u * f32(2/255) - 1 in f32, f64 rounded to f32. Channels are then averaged
// in f64 as the reference does after decoding (src/audio_io.cpp:25-38). Checked
// bitwise against the compiled reference for every encoding (tests/test_audio_cpu.py).
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "engine.hpp"

namespace vdb {

namespace {
uint32_t rd32(const uint8_t* p) { return p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24); }
uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
}  // namespace

bool read_wav_mono(const std::string& path, std::vector<float>& out, int& sample_rate,
                   std::string& err) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) {
        err = "voicedetect: failed to load audio: " + path;
        return false;
    }
    std::vector<uint8_t> buf;
    uint8_t tmp[1 << 16];
    size_t n;
    while ((n = std::fread(tmp, 1, sizeof(tmp), f)) > 0) buf.insert(buf.end(), tmp, tmp + n);
    std::fclose(f);
    if (buf.size() < 12 || std::memcmp(buf.data(), "RIFF", 4) || std::memcmp(buf.data() + 8, "WAVE", 4)) {
        err = "voicedetect: failed to load audio (not RIFF/WAVE): " + path;
        return false;
    }
    uint16_t fmt = 0, ch = 0, bits = 0;
    uint32_t sr = 0;
    const uint8_t* data = nullptr;
    size_t data_len = 0;
    size_t pos = 12;
    while (pos + 8 <= buf.size()) {
        const uint32_t len = rd32(buf.data() + pos + 4);
        const uint8_t* body = buf.data() + pos + 8;
        const size_t avail = buf.size() - pos - 8;
        if (!std::memcmp(buf.data() + pos, "fmt ", 4) && len >= 16 && avail >= 16) {
            fmt = rd16(body);
            ch = rd16(body + 2);
            sr = rd32(body + 4);
            bits = rd16(body + 14);
            if (fmt == 0xFFFE && len >= 26 && avail >= 26) fmt = rd16(body + 24);
        } else if (!std::memcmp(buf.data() + pos, "data", 4)) {
            data = body;
            data_len = len <= avail ? len : avail;
        }
        pos += 8 + (size_t)len + (len & 1);
    }
    if (!data || ch == 0 || sr == 0 || bits == 0) {
        err = "voicedetect: failed to load audio (missing fmt/data): " + path;
        return false;
    }
    const size_t bps = bits / 8;
    if (bps == 0) {
        err = "voicedetect: failed to load audio (bad bit depth): " + path;
        return false;
    }
    const size_t frames = data_len / (bps * ch);
    out.assign(frames, 0.0f);
    for (size_t i = 0; i < frames; ++i) {
        double acc = 0.0;
        for (uint16_t c = 0; c < ch; ++c) {
            const uint8_t* s = data + (i * ch + c) * bps;
            float v;
            if (fmt == 1 && bits == 16) {
                v = (float)(int16_t)rd16(s) / 32768.0f;
            } else if (fmt == 1 && bits == 8) {
                // 0..255 -> 0..2 -> -1..1, two f32 roundings (no fused multiply-add)
                const float scaled = (float)s[0] * (2.0f / 255.0f);
                v = scaled - 1.0f;
            } else if (fmt == 1 && bits == 24) {
                const int32_t x = (int32_t)((uint32_t)s[0] << 8 | (uint32_t)s[1] << 16 |
                                            (uint32_t)s[2] << 24) >> 8;
                v = (float)((double)x / 8388608.0);
            } else if (fmt == 1 && bits == 32) {
                v = (float)((double)(int32_t)rd32(s) / 2147483648.0);
            } else if (fmt == 3 && bits == 32) {
                std::memcpy(&v, s, 4);
            } else if (fmt == 3 && bits == 64) {
                double d;
                std::memcpy(&d, s, 8);
                v = (float)d;
            } else {
                err = "voicedetect: failed to load audio (unsupported WAV encoding): " + path;
                return false;
            }
            acc += v;
        }
        out[i] = (float)(acc / ch);
    }
    sample_rate = (int)sr;
    return true;
}

}  // namespace vdb
