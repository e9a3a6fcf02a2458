// The seven moss_transcribe_capi_* symbols (include/moss_transcribe_capi.h).
// Loading keeps the reference contract (one owning context, NULL on failure,
// no exception across the boundary); the decoder weights go to the device.
#include "../../include/moss_transcribe_capi.h"
#include "../../include/mtb_decoder.h"

#include <cstdlib>
#include <cstring>
#include <new>
#include <string>

struct moss_transcribe_ctx {
    mtb_model* model = nullptr;
    std::string last_error;
    ~moss_transcribe_ctx() { mtb_model_free(model); }
};

namespace {
const char kNoFrontEnd[] =
    "a transcript needs WAV decoding and the tokenizer (prompt ids, transcript text), which are not part of "
    "libmoss_transcribe_b200: run the audio front end with mtb_audio_encode and decode prompt ids + audio rows "
    "with mtb_spec_generate_ids";
}

extern "C" int moss_transcribe_capi_abi_version(void) { return 1; }

extern "C" moss_transcribe_ctx* moss_transcribe_capi_load(const char* gguf_path) {
    if (!gguf_path) return nullptr;
    try {
        const char* dev = std::getenv("MTB_DEVICE");
        mtb_model* m = nullptr;
        if (mtb_model_load(gguf_path, dev ? std::atoi(dev) : 0, &m) != 0) return nullptr;
        auto* ctx = new (std::nothrow) moss_transcribe_ctx();
        if (!ctx) {
            mtb_model_free(m);
            return nullptr;
        }
        ctx->model = m;
        return ctx;
    } catch (...) {
        return nullptr;
    }
}

extern "C" void moss_transcribe_capi_free(moss_transcribe_ctx* ctx) { delete ctx; }

extern "C" char* moss_transcribe_capi_transcribe_path(moss_transcribe_ctx* ctx, const char* wav_path, int) {
    if (!ctx) return nullptr;
    if (!ctx->model) { ctx->last_error = "context has no loaded model"; return nullptr; }
    if (!wav_path) { ctx->last_error = "wav_path is NULL"; return nullptr; }
    ctx->last_error = kNoFrontEnd;
    return nullptr;
}

extern "C" char* moss_transcribe_capi_transcribe_pcm(moss_transcribe_ctx* ctx, const float* samples, int n_samples,
                                                     int sample_rate, int) {
    if (!ctx) return nullptr;
    if (!ctx->model) { ctx->last_error = "context has no loaded model"; return nullptr; }
    if (!samples || n_samples < 0) { ctx->last_error = "invalid samples buffer"; return nullptr; }
    if (sample_rate <= 0) { ctx->last_error = "invalid sample rate"; return nullptr; }
    ctx->last_error = kNoFrontEnd;
    return nullptr;
}

extern "C" void moss_transcribe_capi_free_string(char* s) { std::free(s); }

extern "C" const char* moss_transcribe_capi_last_error(moss_transcribe_ctx* ctx) {
    if (!ctx) return "";
    return ctx->last_error.c_str();
}
