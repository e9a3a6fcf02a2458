// Minimal GGUF reader (see gguf.hpp).  The container format is the one the
// reference's converter writes through the gguf Python package
// (scripts/convert_moss_transcribe_to_gguf.py) and the reference reads with
// ggml's gguf_init_from_file (src/model_loader.cpp:21-114).
#include "gguf.hpp"

#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace mtb {

uint64_t ggml_row_bytes(uint32_t type, int64_t n) {
    switch (type) {
        case GGML_F32: return uint64_t(n) * 4;
        case GGML_F16: return uint64_t(n) * 2;
        case GGML_Q8_0: return uint64_t(n) / 32 * 34;
        default: return 0;
    }
}

namespace {
struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <class T> T get() {
        T v{};
        if (size_t(end - p) < sizeof(T)) { ok = false; return v; }
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || uint64_t(end - p) < n) { ok = false; return {}; }
        std::string s(reinterpret_cast<const char*>(p), size_t(n));
        p += n;
        return s;
    }
    void skip(uint64_t n) {
        if (uint64_t(end - p) < n) { ok = false; return; }
        p += n;
    }
};

int scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return -1;
    }
}
}  // namespace

GgufFile::~GgufFile() {
    if (map_) munmap(map_, map_size_);
}

bool GgufFile::open(const std::string& path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) { error_ = "cannot open " + path; return false; }
    struct stat st {};
    if (fstat(fd, &st) != 0 || st.st_size < 24) { ::close(fd); error_ = "not a GGUF file: " + path; return false; }
    map_size_ = size_t(st.st_size);
    map_ = mmap(nullptr, map_size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map_ == MAP_FAILED) { map_ = nullptr; error_ = "mmap failed for " + path; return false; }
    Cursor c{static_cast<const uint8_t*>(map_), static_cast<const uint8_t*>(map_) + map_size_};
    if (c.get<uint32_t>() != 0x46554747u) { error_ = "bad GGUF magic"; return false; }
    const uint32_t version = c.get<uint32_t>();
    if (version < 2 || version > 3) { error_ = "unsupported GGUF version"; return false; }
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        const std::string key = c.str();
        const uint32_t t = c.get<uint32_t>();
        if (t == 8) { c.str(); continue; }
        if (t == 9) {
            const uint32_t et = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            if (et == 8) { for (uint64_t j = 0; j < n && c.ok; ++j) c.str(); continue; }
            const int es = scalar_size(et);
            if (es < 0) { error_ = "unsupported GGUF array type"; return false; }
            c.skip(n * uint64_t(es));
            continue;
        }
        switch (t) {
            case 0: u_[key] = c.get<uint8_t>(); break;
            case 1: u_[key] = uint64_t(int64_t(c.get<int8_t>())); break;
            case 2: u_[key] = c.get<uint16_t>(); break;
            case 3: u_[key] = uint64_t(int64_t(c.get<int16_t>())); break;
            case 4: u_[key] = c.get<uint32_t>(); break;
            case 5: u_[key] = uint64_t(int64_t(c.get<int32_t>())); break;
            case 6: f_[key] = c.get<float>(); break;
            case 7: u_[key] = c.get<uint8_t>(); break;
            case 10: u_[key] = c.get<uint64_t>(); break;
            case 11: u_[key] = uint64_t(c.get<int64_t>()); break;
            case 12: f_[key] = c.get<double>(); break;
            default: error_ = "unsupported GGUF value type"; return false;
        }
        if (key == "general.alignment" && u_.count(key)) alignment = u_[key];
    }
    std::vector<GgufTensor> infos;
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        GgufTensor t;
        t.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (nd == 0 || nd > 4) { error_ = "bad tensor rank"; return false; }
        int64_t n = 1;
        for (uint32_t d = 0; d < nd; ++d) { t.ne.push_back(int64_t(c.get<uint64_t>())); n *= t.ne.back(); }
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        const uint64_t row = ggml_row_bytes(t.type, t.ne[0]);
        if (row == 0 && t.type != GGML_F32) { t.nbytes = 0; }
        t.nbytes = row * uint64_t(n / t.ne[0]);
        infos.push_back(std::move(t));
    }
    if (!c.ok) { error_ = "truncated GGUF header"; return false; }
    const uint64_t head = uint64_t(c.p - static_cast<const uint8_t*>(map_));
    const uint64_t data_start = (head + alignment - 1) / alignment * alignment;
    for (auto& t : infos) {
        if (t.nbytes && data_start + t.offset + t.nbytes > map_size_) { error_ = "tensor data past end of file: " + t.name; return false; }
        t.data = static_cast<const uint8_t*>(map_) + data_start + t.offset;
        tensors_[t.name] = t;
    }
    return true;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

uint32_t GgufFile::get_u32(const std::string& key, uint32_t def) const {
    auto it = u_.find(key);
    return it == u_.end() ? def : uint32_t(it->second);
}

float GgufFile::get_f32(const std::string& key, float def) const {
    auto it = f_.find(key);
    return it == f_.end() ? def : float(it->second);
}

}  // namespace mtb
