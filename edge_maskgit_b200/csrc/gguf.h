// gguf.h -- read-only GGUF v3 reader shared by the transformer and VQGAN runtimes.
#pragma once
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace mgc {

struct GgufError : std::runtime_error { using std::runtime_error::runtime_error; };

// ----------------------------------------------------------------------- GGUF (v3) reader
// Format of Model::load (mg-model.cpp:139-201): header, metadata KVs, tensor infos, data
// aligned to general.alignment.  Tensors are referenced in the read-only mapping.
struct GgufTensor { uint32_t type = 0; int64_t ne[4] = {1, 1, 1, 1}; const uint8_t* data = nullptr; size_t bytes = 0; };

struct Gguf {
    void* base = MAP_FAILED; size_t size = 0;
    std::unordered_map<std::string, GgufTensor> tensors;
    std::unordered_map<std::string, int64_t> ints;
    std::unordered_map<std::string, float> floats;
    std::unordered_map<std::string, std::vector<int64_t>> int_arrays;

    ~Gguf() { if (base != MAP_FAILED) munmap(base, size); }

    void open(const char* path) {
        int fd = ::open(path, O_RDONLY);
        if (fd < 0) throw GgufError(std::string("cannot open ") + path);
        struct stat st{};
        fstat(fd, &st);
        size = (size_t)st.st_size;
        base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (base == MAP_FAILED) throw GgufError("mmap failed");
        const uint8_t* b = (const uint8_t*)base;
        size_t p = 0;
        auto need = [&](size_t n) { if (p + n > size) throw GgufError("gguf: unexpected EOF"); };
        auto u32 = [&]() { need(4); uint32_t v; std::memcpy(&v, b + p, 4); p += 4; return v; };
        auto u64 = [&]() { need(8); uint64_t v; std::memcpy(&v, b + p, 8); p += 8; return v; };
        auto str = [&]() { uint64_t n = u64(); need(n); std::string s((const char*)b + p, n); p += n; return s; };
        auto scalar_size = [](uint32_t t) -> size_t {
            switch (t) { case 0: case 1: case 7: return 1; case 2: case 3: return 2;
                         case 4: case 5: case 6: return 4; case 10: case 11: case 12: return 8; }
            throw GgufError("gguf: unsupported metadata type");
        };
        if (u32() != 0x46554747u) throw GgufError("not a GGUF file");
        if (u32() != 3) throw GgufError("unsupported GGUF version");
        const uint64_t nt = u64(), nkv = u64();
        for (uint64_t i = 0; i < nkv; i++) {
            const std::string key = str();
            const uint32_t t = u32();
            if (t == 8) { str(); continue; }
            if (t == 9) {   // arrays: integer ones are kept (e.g. maskgit.vqgan.channel_multipliers)
                const uint32_t sub = u32(); const uint64_t n = u64();
                std::vector<int64_t> vals;
                for (uint64_t j = 0; j < n; j++) {
                    if (sub == 8) { str(); continue; }
                    const size_t sz = scalar_size(sub);
                    need(sz);
                    if (sub == 4) { uint32_t x; std::memcpy(&x, b + p, 4); vals.push_back(x); }
                    else if (sub == 5) { int32_t x; std::memcpy(&x, b + p, 4); vals.push_back(x); }
                    p += sz;
                }
                if (sub == 4 || sub == 5) int_arrays[key] = std::move(vals);
                continue;
            }
            const size_t sz = scalar_size(t);
            need(sz);
            if (t == 6) { float f; std::memcpy(&f, b + p, 4); floats[key] = f; }
            else if (t == 12) { double f; std::memcpy(&f, b + p, 8); floats[key] = (float)f; }
            else {
                int64_t v = 0;
                switch (t) {
                    case 0: case 7: v = b[p]; break; case 1: v = (int8_t)b[p]; break;
                    case 2: { uint16_t x; std::memcpy(&x, b + p, 2); v = x; } break;
                    case 3: { int16_t x; std::memcpy(&x, b + p, 2); v = x; } break;
                    case 4: { uint32_t x; std::memcpy(&x, b + p, 4); v = x; } break;
                    case 5: { int32_t x; std::memcpy(&x, b + p, 4); v = x; } break;
                    case 10: { uint64_t x; std::memcpy(&x, b + p, 8); v = (int64_t)x; } break;
                    case 11: { int64_t x; std::memcpy(&x, b + p, 8); v = x; } break;
                }
                ints[key] = v;
            }
            p += sz;
        }
        struct Info { std::string name; GgufTensor t; uint64_t off; };
        std::vector<Info> infos(nt);
        for (auto& in : infos) {
            in.name = str();
            const uint32_t nd = u32();
            if (nd > 4) throw GgufError("gguf: too many dims on " + in.name);
            for (uint32_t d = 0; d < nd; d++) in.t.ne[d] = (int64_t)u64();
            in.t.type = u32();
            in.off = u64();
        }
        const uint64_t align = ints.count("general.alignment") ? (uint64_t)ints["general.alignment"] : 32;
        const size_t data0 = (p + align - 1) / align * align;
        for (auto& in : infos) {
            const int64_t n = in.t.ne[0] * in.t.ne[1] * in.t.ne[2] * in.t.ne[3];
            switch (in.t.type) {
                case 0: in.t.bytes = (size_t)n * 4; break;
                case 8: in.t.bytes = (size_t)n / 32 * 34; break;
                case 12: in.t.bytes = (size_t)n / 256 * 144; break;
                default: in.t.bytes = 0; break;   // other types are not used by the transformer
            }
            in.t.data = b + data0 + in.off;
            if (data0 + in.off + in.t.bytes > size) throw GgufError("gguf: tensor '" + in.name + "' past EOF");
            tensors[in.name] = in.t;
        }
    }
    const GgufTensor& req(const std::string& n) const {
        auto it = tensors.find(n);
        if (it == tensors.end()) throw GgufError("gguf: missing required tensor '" + n + "'");
        return it->second;
    }
    int geti(const std::string& k, int dflt) const { auto it = ints.find(k); return it == ints.end() ? dflt : (int)it->second; }
    float getf(const std::string& k, float dflt) const { auto it = floats.find(k); return it == floats.end() ? dflt : it->second; }
};

}  // namespace mgc
