// mtb_lm_head_argmax_noalloc: the tied LM head with its first-max reduction,
// for callers that must not allocate device memory.
//
// Who needs it: serving processes that hand all free device memory to their
// own pool allocator at start-up and then forbid further cudaMalloc (a late
// cudaMalloc can fail for lack of room, and cudaMalloc / cudaFree synchronise
// the device, which stalls every stream the process has in flight).  Such a
// caller owns its input and output buffers already; what the LM head needs
// beyond them (the q8_0-quantised rows, their scales and the per-CTA argmax
// partials) lives here, in one file-scope device array.
#include "../../include/mtb_decoder.h"
#include "kernels.hpp"

#include <mutex>
#include <string>

using namespace mtb;

// Maximum sizes the scratch is laid out for.
constexpr int kNoAllocMaxHidden = 4096;
constexpr int kNoAllocMaxBlocks = kLmHeadMaxBlocks;  // lm_head_blocks() never exceeds this
static_assert(kNoAllocMaxBlocks >= kLmHeadMaxBlocks, "the scratch covers every LM-head grid");
constexpr size_t kActQBytes = size_t(kNoAllocMaxHidden / 32) * 512;
constexpr size_t kActDBytes = size_t(kNoAllocMaxHidden / 32) * 16 * sizeof(float);
constexpr size_t kPartBytes = size_t(kNoAllocMaxBlocks) * 16 * sizeof(float2);
constexpr size_t kStateBytes = (sizeof(StepState) + 255) / 256 * 256;
constexpr size_t kScratchBytes = kStateBytes + kActQBytes + kActDBytes + kPartBytes;  // about 148 KB

// Every device that loads this library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

namespace {
// Makes a device current and puts the caller's current device back when it
// goes out of scope.
struct DeviceGuard {
    int saved = -1;
    bool enter(int device) {
        if (cudaGetDevice(&saved) != cudaSuccess) saved = -1;
        return saved == device || cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        int now = -1;
        if (saved >= 0 && cudaGetDevice(&now) == cudaSuccess && now != saved) cudaSetDevice(saved);
    }
};

std::mutex g_setup_mutex;
void* g_scratch_ptr[64] = {};  // device address of g_noalloc_scratch, per device
thread_local std::string g_noalloc_error;

int scratch_for(int device, unsigned char** out) {
    if (device < 0 || device >= 64) { g_noalloc_error = "device index out of range"; return -1; }
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[device]) {
        // Host code cannot use the array's name as a device address; ask the
        // runtime for it once per device, with that device current.
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            g_noalloc_error = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e);
            return -1;
        }
        g_scratch_ptr[device] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_ptr[device]);
    return 0;
}
}  // namespace

struct mtb_model;  // defined in decoder.cu; reached through mtb_model_device_view
extern "C" __attribute__((visibility("hidden"))) int mtb_model_device_view(const mtb_model* m, const void** view,
                                                                            int* device);

extern "C" const char* mtb_noalloc_error(void) { return g_noalloc_error.c_str(); }

extern "C" int mtb_lm_head_argmax_noalloc(const mtb_model* m, const float* hidden_rows, int T, int32_t* choices,
                                          void* stream) {
    if (!m || !hidden_rows || !choices) { g_noalloc_error = "null argument"; return -1; }
    const void* view = nullptr;
    int device = 0;
    if (mtb_model_device_view(m, &view, &device) != 0) { g_noalloc_error = "invalid model"; return -1; }
    const DeviceModel& dm = *static_cast<const DeviceModel*>(view);
    if (dm.f16) {
        g_noalloc_error = "the no-allocation LM head takes q8_0 models only";
        return -2;
    }
    if (T < 1 || T > kTMax) {
        g_noalloc_error = "T must be in [1, 16] (the scratch holds 16 rows)";
        return -2;
    }
    if (dm.dims.hidden > kNoAllocMaxHidden) {
        g_noalloc_error = "hidden exceeds the no-allocation scratch limit of 4096";
        return -2;
    }
    if (lm_head_blocks(dm.dims.vocab) > kNoAllocMaxBlocks) {
        g_noalloc_error = "vocabulary exceeds the no-allocation scratch limit";
        return -2;
    }
    // The model's device is made current for the call and the caller's
    // current device is restored on every return path.
    DeviceGuard guard;
    if (!guard.enter(device)) { g_noalloc_error = "cudaSetDevice failed"; return -1; }
    unsigned char* base = nullptr;
    if (scratch_for(device, &base) != 0) return -1;
    auto* state = reinterpret_cast<StepState*>(base);
    auto* act_q = reinterpret_cast<uint8_t*>(base + kStateBytes);
    auto* act_d = reinterpret_cast<float*>(base + kStateBytes + kActQBytes);
    auto* part = reinterpret_cast<float2*>(base + kStateBytes + kActQBytes + kActDBytes);
    launch_lm_argmax_rows(dm, state, hidden_rows, T, act_q, act_d, part, choices, static_cast<cudaStream_t>(stream));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_noalloc_error = std::string("launch: ") + cudaGetErrorString(e);
        return -1;
    }
    return 0;
}
