// The audio front-end branch a maintainer adds to the reference's
// transcribe_pcm16k in place of AudioEncoder::encode (INTEGRATION.md,
// section 1), as a standalone program built with g++ against include/*.h and
// linked to libmoss_transcribe_b200.so (tests/test_audio_cpp.py).
// usage: audio_branch <gguf> <samples.f32> <device> <rows_out.f32>
// samples.f32: float32 16 kHz mono samples.  Writes the audio rows
// [n_tokens][hidden] to rows_out.f32 and prints "n_tokens hidden".
#include "mtb_decoder.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <vector>

static std::vector<float> encode_branch(const char* gguf_path, int device, const std::vector<float>& samples,
                                        int hidden, int& n_tokens) {
    static mtb_audio* audio = nullptr;  // once per process
    if (!audio && mtb_audio_load(gguf_path, device, &audio) != 0)
        std::fprintf(stderr, "mtb_audio_load: %s\n", mtb_audio_error(nullptr));
    n_tokens = 0;
    std::vector<float> audio_embeds;
    if (audio) {
        const int rows = mtb_audio_tokens(audio, (int)samples.size());  // sum of token_len
        audio_embeds.resize((size_t)std::max(rows, 0) * hidden);
        if (rows <= 0 || mtb_audio_encode(audio, samples.data(), (int)samples.size(), audio_embeds.data(), rows,
                                          &n_tokens) != 0) {
            std::fprintf(stderr, "mtb_audio_encode: %s\n", mtb_audio_error(audio));
            audio_embeds.clear();
        }
    }
    return audio_embeds;
}

int main(int argc, char** argv) {
    if (argc != 5) return 2;
    std::FILE* f = std::fopen(argv[2], "rb");
    if (!f) return 2;
    std::vector<float> samples;
    float v;
    while (std::fread(&v, sizeof(float), 1, f) == 1) samples.push_back(v);
    std::fclose(f);
    // The hidden size comes from the model (Config::text_hidden in the reference).
    mtb_audio* probe = nullptr;
    if (mtb_audio_load(argv[1], std::atoi(argv[3]), &probe) != 0) {
        std::fprintf(stderr, "mtb_audio_load: %s\n", mtb_audio_error(nullptr));
        return 1;
    }
    int32_t dims[10] = {};
    mtb_audio_dims(probe, dims);
    mtb_audio_free(probe);
    int n_tokens = 0;
    const std::vector<float> rows = encode_branch(argv[1], std::atoi(argv[3]), samples, dims[0], n_tokens);
    if (rows.empty()) return 1;
    std::FILE* o = std::fopen(argv[4], "wb");
    if (!o) return 2;
    std::fwrite(rows.data(), sizeof(float), rows.size(), o);
    std::fclose(o);
    std::printf("%d %d\n", n_tokens, dims[0]);
    return 0;
}
