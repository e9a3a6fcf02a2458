// The generate-layer branch a maintainer adds to the reference's
// greedy_generate, as a standalone program built
// by tests/test_gpu_integration_cpp.py with g++ against include/*.h and linked
// to libmoss_transcribe_b200.so.
// usage: generate_branch <gguf> <rows.f32> <seq> <max_new> <eos>
// rows.f32: seq x hidden float32 fused prompt rows.  Prints the ids, one line.
#include "mtb_decoder.h"

#include <cstdio>
#include <cstdlib>
#include <vector>

static std::vector<int32_t> greedy_generate_branch(const char* gguf_path, const std::vector<float>& fused, int seq,
                                                   int max_new, int eos, float penalty) {
    if (const char* dev = std::getenv("MTB_DEVICE")) {
        static mtb_model* model = nullptr;  // once per process
        if (!model && mtb_model_load(gguf_path, std::atoi(dev), &model) != 0)
            std::fprintf(stderr, "mtb_model_load: %s\n", mtb_global_error());
        if (model) {
            mtb_decoder* d = nullptr;
            mtb_decoder_create(model, seq + max_new + 16, MTB_KV_F32, max_new, &d);
            mtb_spec_params p{4, 2, 16, penalty};  // the reference policy
            std::vector<int32_t> ids(max_new);
            int n = 0;
            mtb_counters c{};
            if (d && mtb_spec_generate(d, fused.data(), seq, max_new, eos, &p, ids.data(), &n, &c, nullptr, nullptr,
                                       nullptr) == 0) {
                ids.resize(n);
                mtb_decoder_free(d);
                return ids;
            }
            std::fprintf(stderr, "mtb_spec_generate: %s\n", d ? mtb_decoder_error(d) : mtb_global_error());
            mtb_decoder_free(d);
        }
    }
    return {};
}

int main(int argc, char** argv) {
    if (argc != 6) return 2;
    const int seq = std::atoi(argv[3]), max_new = std::atoi(argv[4]), eos = std::atoi(argv[5]);
    std::FILE* f = std::fopen(argv[2], "rb");
    if (!f) return 3;
    std::vector<float> rows;
    float buf[4096];
    size_t got;
    while ((got = std::fread(buf, sizeof(float), 4096, f)) > 0) rows.insert(rows.end(), buf, buf + got);
    std::fclose(f);
    if (seq <= 0 || rows.size() % size_t(seq)) return 4;
    const std::vector<int32_t> ids = greedy_generate_branch(argv[1], rows, seq, max_new, eos, 1.f);
    if (ids.empty()) return 5;
    for (size_t i = 0; i < ids.size(); ++i) std::printf(i ? " %d" : "%d", ids[i]);
    std::printf("\n");
    return 0;
}
