// The flat C ABI (include/voicedetect_capi.h): same contract as the reference's
// src/voicedetect_capi.cpp:61-176 -- int status, per-context last_error, malloc'd
// outputs, outputs reset before work, nothing thrown across the boundary -- on
// top of the B200 Engine.
#include "voicedetect_capi.h"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <memory>
#include <algorithm>
#include <mutex>
#include <thread>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "engine.hpp"
#include "vdb_internal.h"

#define VOICEDETECT_CAPI_ABI_VERSION 1

struct voicedetect_ctx {
    std::unique_ptr<vdb::Engine> engine;  // on the device current at load time
    // voicedetect_capi_set_devices(n > 1): the same model on n - 1 more GPUs; the
    // batch call shards clips over all of them
    std::vector<std::unique_ptr<vdb::Engine>> extra;
    std::string path;
    std::string last_error;
    std::mutex mu;
};

namespace {

// Restores the calling thread's current CUDA device when it leaves scope, so a host
// application that manages its own device sees it unchanged after any ABI call.
class DeviceRestore {
public:
    DeviceRestore() { ok_ = cudaGetDevice(&dev_) == cudaSuccess; }
    ~DeviceRestore() {
        if (ok_) cudaSetDevice(dev_);
    }
    DeviceRestore(const DeviceRestore&) = delete;
    DeviceRestore& operator=(const DeviceRestore&) = delete;

private:
    int dev_ = 0;
    bool ok_ = false;
};

// Hands an embedding to the caller under the ABI's ownership rule: the vector is a
// fresh malloc'd block that voicedetect_capi_free_vec releases; nothing is written
// to the out-parameters unless the whole call succeeds.
int give_embedding(voicedetect_ctx* ctx, const std::vector<float>& emb, float** out_vec,
                   int* out_dim) {
    const size_t bytes = emb.size() * sizeof(float);
    float* block = bytes ? static_cast<float*>(std::malloc(bytes)) : nullptr;
    if (bytes && !block) {
        ctx->last_error = "out of memory";
        return 1;
    }
    if (bytes) std::memcpy(block, emb.data(), bytes);
    if (out_vec) {
        *out_vec = block;
    } else {
        std::free(block);  // caller asked only for the dimension
    }
    if (out_dim) *out_dim = static_cast<int>(emb.size());
    ctx->last_error.clear();
    return 0;
}

// Embeds 16 kHz PCM through the engine; throws std::runtime_error on failure.
std::vector<float> embed_16k(voicedetect_ctx* ctx, const std::vector<float>& pcm16k) {
    DeviceRestore keep_device;  // the engine switches to its own device
    std::string err;
    const int D = ctx->engine->emb_dim();
    std::vector<float> out((size_t)D);
    const float* p = pcm16k.data();
    const int n = (int)pcm16k.size();
    if (ctx->engine->embed_host(&p, &n, 1, out.data(), err)) throw std::runtime_error(err);
    return out;
}

std::vector<float> embed_path(voicedetect_ctx* ctx, const char* path) {
    std::vector<float> mono;
    int sr = 0;
    std::string err;
    if (!vdb::read_wav_mono(path, mono, sr, err)) throw std::runtime_error(err);
    return embed_16k(ctx, vdb::resample_linear(mono, sr, 16000));
}

// The batch call on several GPUs: clips go to engines by LPT on sample count (the
// longest clip to the least loaded GPU), each engine embeds its shard from its own
// host thread, and rows are scattered back in the caller's order.
// ptrs / ns: raw mono clips of element type `type` (0 f32, 1 int16) at sample_rate.
int embed_sharded(voicedetect_ctx* ctx, const std::vector<const void*>& ptrs,
                  const std::vector<int>& ns, int type, int sample_rate, float* out,
                  std::string& err) {
    std::vector<vdb::Engine*> eng{ctx->engine.get()};
    for (auto& e : ctx->extra) eng.push_back(e.get());
    const int G = (int)eng.size(), n = (int)ptrs.size(), D = ctx->engine->emb_dim();
    std::vector<int> order(n);
    for (int i = 0; i < n; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return ns[a] > ns[b]; });
    std::vector<long long> load(G, 0);
    std::vector<std::vector<int>> shard(G);
    for (int i : order) {
        int g = 0;
        for (int k = 1; k < G; ++k)
            if (load[k] < load[g]) g = k;
        shard[g].push_back(i);
        load[g] += ns[i];
    }
    std::vector<std::vector<float>> res(G);
    std::vector<std::string> errs(G);
    std::vector<int> rcs(G, 0);
    std::vector<std::thread> th;
    for (int g = 0; g < G; ++g) {
        if (shard[g].empty()) continue;
        th.emplace_back([&, g]() {
            // an exception escaping a std::thread would terminate the host process:
            // every failure of a shard becomes its status and message instead
            try {
                if (cudaSetDevice(eng[g]->device()) != cudaSuccess)
                    throw std::runtime_error("cudaSetDevice failed");
                std::vector<const void*> p;
                std::vector<int> c;
                for (int i : shard[g]) {
                    p.push_back(ptrs[i]);
                    c.push_back(ns[i]);
                }
                res[g].resize((size_t)shard[g].size() * D);
                rcs[g] = eng[g]->embed_host_raw(p.data(), type, c.data(), (int)p.size(),
                                                sample_rate, res[g].data(), errs[g]);
            } catch (const std::exception& e) {
                errs[g] = e.what();
                rcs[g] = 1;
            } catch (...) {
                errs[g] = "unknown error";
                rcs[g] = 1;
            }
        });
    }
    for (auto& t : th) t.join();
    for (int g = 0; g < G; ++g)
        if (rcs[g]) {
            err = "GPU " + std::to_string(eng[g]->device()) + ": " + errs[g];
            return 1;
        }
    for (int g = 0; g < G; ++g)
        for (size_t j = 0; j < shard[g].size(); ++j)
            std::memcpy(out + (size_t)shard[g][j] * D, res[g].data() + j * D, sizeof(float) * D);
    return 0;
}

}  // namespace

extern "C" int voicedetect_capi_abi_version(void) { return VOICEDETECT_CAPI_ABI_VERSION; }

extern "C" voicedetect_ctx* voicedetect_capi_load(const char* gguf_path) {
    if (!gguf_path) return nullptr;
    try {
        std::string err;
        std::unique_ptr<vdb::Engine> e = vdb::Engine::load(gguf_path, err);
        if (!e) {
            std::fprintf(stderr, "[voicedetect] load failed: %s\n", err.c_str());
            return nullptr;
        }
        auto* ctx = new (std::nothrow) voicedetect_ctx();
        if (!ctx) return nullptr;
        ctx->engine = std::move(e);
        ctx->path = gguf_path;
        return ctx;
    } catch (...) {
        return nullptr;
    }
}

extern "C" void voicedetect_capi_free(voicedetect_ctx* ctx) {
    try {
        delete ctx;
    } catch (...) {
    }
}

extern "C" const char* voicedetect_capi_last_error(voicedetect_ctx* ctx) {
    if (!ctx) return "";
    return ctx->last_error.c_str();
}

extern "C" void voicedetect_capi_free_string(char* s) { std::free(s); }

extern "C" void voicedetect_capi_free_vec(float* v) { std::free(v); }

extern "C" int voicedetect_capi_embed_path(voicedetect_ctx* ctx, const char* wav_path,
                                           float** out_vec, int* out_dim) {
    if (out_vec) *out_vec = nullptr;
    if (out_dim) *out_dim = 0;
    if (!ctx) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->engine) { ctx->last_error = "context has no loaded model"; return 1; }
    if (!wav_path) { ctx->last_error = "wav_path is NULL"; return 1; }
    try {
        return give_embedding(ctx, embed_path(ctx, wav_path), out_vec, out_dim);
    } catch (const std::exception& e) {
        ctx->last_error = e.what();
        return 1;
    } catch (...) {
        ctx->last_error = "unknown error";
        return 1;
    }
}

extern "C" int voicedetect_capi_embed_pcm(voicedetect_ctx* ctx, const float* pcm, int n_samples,
                                          int sample_rate, float** out_vec, int* out_dim) {
    if (out_vec) *out_vec = nullptr;
    if (out_dim) *out_dim = 0;
    if (!ctx) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->engine) { ctx->last_error = "context has no loaded model"; return 1; }
    if (!pcm || n_samples < 0) { ctx->last_error = "invalid pcm buffer"; return 1; }
    try {
        std::vector<float> samples(pcm, pcm + n_samples);
        if (sample_rate != 16000) samples = vdb::resample_linear(samples, sample_rate, 16000);
        return give_embedding(ctx, embed_16k(ctx, samples), out_vec, out_dim);
    } catch (const std::exception& e) {
        ctx->last_error = e.what();
        return 1;
    } catch (...) {
        ctx->last_error = "unknown error";
        return 1;
    }
}

extern "C" int voicedetect_capi_verify_paths(voicedetect_ctx* ctx, const char* a, const char* b,
                                             float threshold, float* out_distance,
                                             int* out_verified) {
    if (!ctx) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->engine) { ctx->last_error = "context has no loaded model"; return 1; }
    if (!a || !b) { ctx->last_error = "clip path is NULL"; return 1; }
    try {
        const std::vector<float> ea = embed_path(ctx, a);
        const std::vector<float> eb = embed_path(ctx, b);
        if (ea.size() != eb.size() || ea.empty())
            throw std::runtime_error("voicedetect: embedding dimension mismatch in verify");
        // src/model.cpp:65-78: f64 dot of the L2-normalised embeddings.
        double dot = 0.0;
        for (size_t i = 0; i < ea.size(); ++i) dot += (double)ea[i] * (double)eb[i];
        const float distance = 1.0f - (float)dot;
        if (out_distance) *out_distance = distance;
        if (out_verified) *out_verified = distance <= threshold ? 1 : 0;
        ctx->last_error.clear();
        return 0;
    } catch (const std::exception& e) {
        ctx->last_error = e.what();
        return 1;
    } catch (...) {
        ctx->last_error = "unknown error";
        return 1;
    }
}

extern "C" char* voicedetect_capi_analyze_path_json(voicedetect_ctx* ctx, const char* wav_path) {
    if (!ctx) return nullptr;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->engine) { ctx->last_error = "context has no loaded model"; return nullptr; }
    if (!wav_path) { ctx->last_error = "wav_path is NULL"; return nullptr; }
    ctx->last_error = "voicedetect: this model has no age/gender/emotion analyze heads";
    return nullptr;
}

// Batch of raw mono clips through the context's engine(s).
static int embed_raw_batch(voicedetect_ctx* ctx, const void* const* pcm, int type,
                           const int* n_samples, int n_clips, int sample_rate, float* out,
                           std::string& err) {
    std::vector<const void*> ptrs((size_t)n_clips);
    std::vector<int> ns((size_t)n_clips);
    for (int i = 0; i < n_clips; ++i) {
        if (!pcm[i] || n_samples[i] < 0) {
            err = "invalid pcm buffer (clip " + std::to_string(i) + ")";
            return 1;
        }
        ptrs[i] = pcm[i];
        ns[i] = n_samples[i];
    }
    DeviceRestore keep_device;
    if (ctx->extra.empty())
        return ctx->engine->embed_host_raw(ptrs.data(), type, ns.data(), n_clips, sample_rate,
                                           out, err);
    return embed_sharded(ctx, ptrs, ns, type, sample_rate, out, err);
}

extern "C" int voicedetect_b200_embed_s16_batch(voicedetect_ctx* ctx, const int16_t* const* pcm,
                                                const int* n_samples, int n_clips,
                                                int sample_rate, float* out, int* out_dim) {
    if (out_dim) *out_dim = 0;
    if (!ctx) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->engine) { ctx->last_error = "context has no loaded model"; return 1; }
    if (!pcm || !n_samples || !out || n_clips <= 0 || sample_rate <= 0) {
        ctx->last_error = "invalid batch arguments";
        return 1;
    }
    try {
        std::string err;
        if (embed_raw_batch(ctx, reinterpret_cast<const void* const*>(pcm), 1, n_samples,
                            n_clips, sample_rate, out, err)) {
            ctx->last_error = err;
            return 1;
        }
        if (out_dim) *out_dim = ctx->engine->emb_dim();
        ctx->last_error.clear();
        return 0;
    } catch (const std::exception& e) {
        ctx->last_error = e.what();
        return 1;
    }
}

extern "C" int voicedetect_capi_embed_pcm_batch(voicedetect_ctx* ctx, const float* const* pcm,
                                                const int* n_samples, int n_clips,
                                                int sample_rate, float* out, int* out_dim) {
    if (out_dim) *out_dim = 0;
    if (!ctx) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->engine) { ctx->last_error = "context has no loaded model"; return 1; }
    if (!pcm || !n_samples || !out || n_clips <= 0) {
        ctx->last_error = "invalid batch arguments";
        return 1;
    }
    if (sample_rate <= 0) {
        ctx->last_error = "invalid sample rate";
        return 1;
    }
    try {
        std::string err;
        // other rates are resampled on the device (vdb_pcm_ingest, the reference's
        // resample_linear arithmetic)
        if (embed_raw_batch(ctx, reinterpret_cast<const void* const*>(pcm), 0, n_samples,
                            n_clips, sample_rate, out, err)) {
            ctx->last_error = err;
            return 1;
        }
        if (out_dim) *out_dim = ctx->engine->emb_dim();
        ctx->last_error.clear();
        return 0;
    } catch (const std::exception& e) {
        ctx->last_error = e.what();
        return 1;
    } catch (...) {
        ctx->last_error = "unknown error";
        return 1;
    }
}

extern "C" int voicedetect_capi_identify(voicedetect_ctx* ctx, const float* queries, int n_q,
                                         const float* registry, int n_reg, int dim, int k,
                                         int* out_idx, float* out_score) {
    if (!ctx) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->engine) { ctx->last_error = "context has no loaded model"; return 1; }
    if (!queries || !registry || !out_idx || !out_score || n_q <= 0 || n_reg <= 0 || dim <= 0 ||
        k <= 0) {
        ctx->last_error = "invalid identify arguments";
        return 1;
    }
    DeviceRestore keep_device;
    cudaSetDevice(ctx->engine->device());
    cudaStream_t st = ctx->engine->stream();
    float *dq = nullptr, *dr = nullptr, *ds = nullptr;
    int* di = nullptr;
    const size_t qb = sizeof(float) * (size_t)n_q * dim, rb = sizeof(float) * (size_t)n_reg * dim;
    const size_t ob = (size_t)n_q * k;
    int rc = 1;
    if (cudaMalloc(&dq, qb) == cudaSuccess && cudaMalloc(&dr, rb) == cudaSuccess &&
        cudaMalloc(&ds, ob * sizeof(float)) == cudaSuccess &&
        cudaMalloc(&di, ob * sizeof(int)) == cudaSuccess &&
        cudaMemcpyAsync(dq, queries, qb, cudaMemcpyHostToDevice, st) == cudaSuccess &&
        cudaMemcpyAsync(dr, registry, rb, cudaMemcpyHostToDevice, st) == cudaSuccess) {
        if (vdb_identify(dq, n_q, dr, n_reg, dim, k, di, ds, st) != 0) {
            ctx->last_error = vdb_last_error();
        } else if (cudaMemcpyAsync(out_idx, di, ob * sizeof(int), cudaMemcpyDeviceToHost, st) ==
                       cudaSuccess &&
                   cudaMemcpyAsync(out_score, ds, ob * sizeof(float), cudaMemcpyDeviceToHost,
                                   st) == cudaSuccess &&
                   cudaStreamSynchronize(st) == cudaSuccess) {
            rc = 0;
            ctx->last_error.clear();
        } else {
            ctx->last_error = std::string("CUDA error: ") + cudaGetErrorString(cudaGetLastError());
        }
    } else {
        ctx->last_error = "device out of memory (identify)";
    }
    cudaStreamSynchronize(st);
    cudaFree(dq);
    cudaFree(dr);
    cudaFree(ds);
    cudaFree(di);
    return rc;
}

extern "C" int voicedetect_capi_set_devices(voicedetect_ctx* ctx, int n_gpus) {
    if (!ctx) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->engine) { ctx->last_error = "context has no loaded model"; return 1; }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) count = 0;
    if (n_gpus < 1 || n_gpus > count) {
        ctx->last_error = "n_gpus must be between 1 and the number of visible GPUs (" +
                          std::to_string(count) + ")";
        return 1;
    }
    DeviceRestore keep_device;
    try {
        // Devices d0, d0 + 1, ... (mod count), d0 = the load device. Engines beyond
        // n_gpus are released; missing ones load the same GGUF on their device.
        const int d0 = ctx->engine->device();
        while ((int)ctx->extra.size() > n_gpus - 1) ctx->extra.pop_back();
        for (int i = (int)ctx->extra.size() + 1; i < n_gpus; ++i) {
            const int dev = (d0 + i) % count;
            if (cudaSetDevice(dev) != cudaSuccess) {
                ctx->last_error = "cudaSetDevice failed";
                return 1;
            }
            std::string err;
            std::unique_ptr<vdb::Engine> e = vdb::Engine::load(ctx->path, err);
            if (!e) {
                ctx->last_error = "load on GPU " + std::to_string(dev) + " failed: " + err;
                return 1;
            }
            e->max_clips = ctx->engine->max_clips;
            e->max_frames = ctx->engine->max_frames;
            ctx->extra.push_back(std::move(e));
        }
        ctx->last_error.clear();
        return 0;
    } catch (const std::exception& ex) {
        ctx->last_error = ex.what();
        return 1;
    }
}

extern "C" int voicedetect_b200_embed_device(voicedetect_ctx* ctx, const float* d_pcm,
                                             const long long* offsets, const int* n_samples,
                                             int n_clips, float* d_out, void* stream) {
    if (!ctx) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->engine) { ctx->last_error = "context has no loaded model"; return 1; }
    if (!d_pcm || !offsets || !n_samples || !d_out || n_clips <= 0) {
        ctx->last_error = "invalid batch arguments";
        return 1;
    }
    try {
        DeviceRestore keep_device;
        std::string err;
        if (ctx->engine->embed_device(d_pcm, offsets, n_samples, n_clips, d_out,
                                      static_cast<cudaStream_t>(stream), err)) {
            ctx->last_error = err;
            return 1;
        }
        ctx->last_error.clear();
        return 0;
    } catch (const std::exception& e) {
        ctx->last_error = e.what();
        return 1;
    } catch (...) {
        ctx->last_error = "unknown error";
        return 1;
    }
}

extern "C" int voicedetect_b200_set_bucketing(voicedetect_ctx* ctx, int max_clips,
                                              long long max_frames) {
    if (!ctx || !ctx->engine) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (max_clips <= 0 || max_frames <= 0) {
        ctx->last_error = "bucketing limits must be positive";
        return 1;
    }
    ctx->engine->max_clips = max_clips;
    ctx->engine->max_frames = max_frames;
    for (auto& e : ctx->extra) {
        e->max_clips = max_clips;
        e->max_frames = max_frames;
    }
    return 0;
}

extern "C" long long voicedetect_b200_last_launches(voicedetect_ctx* ctx) {
    return (ctx && ctx->engine) ? ctx->engine->last_launches : 0;
}

extern "C" long long voicedetect_b200_conv_weight_bytes(voicedetect_ctx* ctx) {
    return (ctx && ctx->engine) ? ctx->engine->conv_weight_bytes : 0;
}

extern "C" int voicedetect_b200_embedding_dim(voicedetect_ctx* ctx) {
    return (ctx && ctx->engine) ? ctx->engine->emb_dim() : 0;
}

extern "C" int voicedetect_b200_profile(voicedetect_ctx* ctx, int enable) {
    if (!ctx || !ctx->engine) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    ctx->engine->set_profiling(enable != 0);
    return 0;
}

extern "C" int voicedetect_b200_profile_read(voicedetect_ctx* ctx, double* conv_ms,
                                             double* conv_flops, long long* conv_launches) {
    if (!ctx || !ctx->engine) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    double ms = 0, fl = 0;
    long long n = 0;
    std::string err;
    DeviceRestore keep_device;
    cudaSetDevice(ctx->engine->device());
    if (ctx->engine->read_profile(ms, fl, n, err)) {
        ctx->last_error = err;
        return 1;
    }
    if (conv_ms) *conv_ms = ms;
    if (conv_flops) *conv_flops = fl;
    if (conv_launches) *conv_launches = n;
    return 0;
}

extern "C" int voicedetect_b200_profile_stages(voicedetect_ctx* ctx, double* ms, int n) {
    if (!ctx || !ctx->engine || !ms || n < 0) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    // order: conv, FBank, CMN + stem, pooling, other
    const double* v = ctx->engine->stage_ms;
    const double out[5] = {v[0], v[1], v[4], v[2], v[3]};
    for (int i = 0; i < n && i < 5; ++i) ms[i] = out[i];
    return 0;
}

extern "C" int voicedetect_b200_sync(voicedetect_ctx* ctx) {
    if (!ctx || !ctx->engine) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    std::string err;
    DeviceRestore keep_device;
    if (cudaSetDevice(ctx->engine->device()) != cudaSuccess ||
        cudaStreamSynchronize(ctx->engine->stream()) != cudaSuccess) {
        ctx->last_error = std::string("CUDA error: ") + cudaGetErrorString(cudaGetLastError());
        return 1;
    }
    if (ctx->engine->check_device_error(err)) {
        ctx->last_error = err;
        return 1;
    }
    return 0;
}

extern "C" int voicedetect_b200_profile_convs(voicedetect_ctx* ctx, double* rec, int n) {
    if (!ctx || !ctx->engine) return -1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    const auto& v = ctx->engine->conv_records;
    const int k = std::min<int>(n, (int)v.size());
    for (int i = 0; i < k && rec; ++i) {
        const auto& r = v[i];
        double* o = rec + 12 * i;
        o[0] = r.ms;
        o[1] = r.flops;
        o[2] = r.ic;
        o[3] = r.oc;
        o[4] = r.k;
        o[5] = r.stride;
        o[6] = r.f_out;
        o[7] = r.t_out;
        o[8] = r.batch;
        o[9] = r.ic1;
        o[10] = r.res;
        o[11] = r.qpack;
    }
    return (int)v.size();
}

extern "C" int voicedetect_b200_release_cache(voicedetect_ctx* ctx) {
    if (!ctx || !ctx->engine) return 1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceRestore keep_device;
    std::string err;
    auto drop = [&](vdb::Engine& e) -> bool {
        if (cudaSetDevice(e.device()) != cudaSuccess) {
            err = std::string("CUDA error: ") + cudaGetErrorString(cudaGetLastError());
            return false;
        }
        return e.release_cache(err) == 0;
    };
    bool ok = drop(*ctx->engine);
    for (auto& e : ctx->extra) ok = drop(*e) && ok;
    if (!ok) ctx->last_error = err;
    return ok ? 0 : 1;
}

namespace {
thread_local std::string g_audio_error;
}

extern "C" int voicedetect_b200_load_audio_16k_mono(const char* wav_path, float** out_pcm,
                                                    int* out_n) {
    if (out_pcm) *out_pcm = nullptr;
    if (out_n) *out_n = 0;
    if (!wav_path || !out_pcm || !out_n) {
        g_audio_error = "wav_path, out_pcm and out_n must not be NULL";
        return 1;
    }
    try {
        std::vector<float> mono;
        int sr = 0;
        std::string err;
        if (!vdb::read_wav_mono(wav_path, mono, sr, err)) {
            g_audio_error = err;
            return 1;
        }
        const std::vector<float> pcm = vdb::resample_linear(mono, sr, 16000);
        if (pcm.size() > (size_t)INT32_MAX) {
            g_audio_error = "audio too long";
            return 1;
        }
        float* block = static_cast<float*>(std::malloc(pcm.empty() ? 1 : pcm.size() * sizeof(float)));
        if (!block) {
            g_audio_error = "out of memory";
            return 1;
        }
        if (!pcm.empty()) std::memcpy(block, pcm.data(), pcm.size() * sizeof(float));
        *out_pcm = block;
        *out_n = (int)pcm.size();
        g_audio_error.clear();
        return 0;
    } catch (const std::exception& e) {
        g_audio_error = e.what();
        return 1;
    } catch (...) {
        g_audio_error = "unknown error";
        return 1;
    }
}

extern "C" const char* voicedetect_b200_audio_error(void) { return g_audio_error.c_str(); }

extern "C" int voicedetect_b200_host_register(void* ptr, size_t bytes) {
    if (!ptr || bytes == 0) {
        vdb::set_error("voicedetect_b200_host_register: NULL pointer or zero bytes");
        return 1;
    }
    const cudaError_t e = cudaHostRegister(ptr, bytes, cudaHostRegisterPortable);
    if (e != cudaSuccess) {
        cudaGetLastError();  // a failed registration must not surface at a later launch check
        vdb::set_error(std::string("voicedetect_b200_host_register: ") + cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

extern "C" int voicedetect_b200_host_unregister(void* ptr) {
    if (!ptr) {
        vdb::set_error("voicedetect_b200_host_unregister: NULL pointer");
        return 1;
    }
    const cudaError_t e = cudaHostUnregister(ptr);
    if (e != cudaSuccess) {
        cudaGetLastError();
        vdb::set_error(std::string("voicedetect_b200_host_unregister: ") + cudaGetErrorString(e));
        return 1;
    }
    return 0;
}
