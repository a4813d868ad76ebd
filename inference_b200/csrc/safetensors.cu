// safetensors.cu -- checkpoint loading (host code): single-file and sharded
// safetensors checkpoints, as Hugging Face publishes Qwen3 (model.safetensors,
// or model-0000k-of-0000n.safetensors + model.safetensors.index.json).
//
// The reference reads one safetensors file whole into host memory
// (src/lib/model/safetensors.hpp:30-54) and moves each tensor into its
// Weights map.  Here each shard is memory-mapped and every BF16 tensor goes
// straight to q3_engine_set_weight (which packs and tensor-parallel-shards
// it); the engine then checks that every tensor the model needs arrived.
//
// File format: 8-byte little-endian header length N, N bytes of JSON
// {"name": {"dtype": "BF16", "shape": [r, c], "data_offsets": [b, e]}, ...,
// "__metadata__": {...}}, then the data; offsets are relative to the data.
#include <cmath>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "host_util.hpp"
#include "json.hpp"
#include "kernels.cuh"

namespace q3 {
namespace {

// ---------------------------------------------------------------- checkpoint files
struct Tensor {
    std::string name, dtype, file;
    std::vector<uint64_t> shape;
    uint64_t offset = 0, bytes = 0;  // absolute file offset of the data, byte count
};

struct Mapped {
    void* base = MAP_FAILED;
    size_t size = 0;
    ~Mapped() {
        if (base != MAP_FAILED) munmap(base, size);
    }
};

bool read_file(const std::string& path, std::string& out, std::string& err) {
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "cannot open " + path;
        return false;
    }
    struct stat st {};
    fstat(fd, &st);
    out.resize(static_cast<size_t>(st.st_size));
    size_t got = 0;
    while (got < out.size()) {
        const ssize_t r = ::read(fd, &out[got], out.size() - got);
        if (r <= 0) break;
        got += static_cast<size_t>(r);
    }
    close(fd);
    if (got != out.size()) {
        err = "short read of " + path;
        return false;
    }
    return true;
}

size_t dtype_size(const std::string& d) {
    if (d == "BF16" || d == "F16" || d == "I16" || d == "U16") return 2;
    if (d == "F32" || d == "I32" || d == "U32") return 4;
    if (d == "F64" || d == "I64" || d == "U64") return 8;
    if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
    return 0;
}

// A JSON number that is an exact non-negative integer below 2^53 (every such
// integer is a double exactly; larger or fractional values, negative numbers,
// NaN and non-numbers are rejected before any conversion to uint64_t).
bool json_index(const Json& j, uint64_t& out) {
    if (j.kind != Json::Num || !(j.num >= 0.0) || !(j.num < 9007199254740992.0) || j.num != std::floor(j.num))
        return false;
    out = static_cast<uint64_t>(j.num);
    return true;
}

// The tensors of one safetensors file, validated against its size.
bool scan_file(const std::string& path, std::vector<Tensor>& out, std::string& err) {
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "cannot open " + path;
        return false;
    }
    struct stat st {};
    fstat(fd, &st);
    const uint64_t fsize = static_cast<uint64_t>(st.st_size);
    uint64_t hlen = 0;
    bool ok = fsize >= 8 && pread(fd, &hlen, 8, 0) == 8;
    if (!ok || hlen > fsize - 8 || hlen > (100ull << 20)) {
        close(fd);
        err = path + ": bad safetensors header length";
        return false;
    }
    std::string hdr(hlen, '\0');
    ok = pread(fd, &hdr[0], hlen, 8) == static_cast<ssize_t>(hlen);
    close(fd);
    if (!ok) {
        err = path + ": short header";
        return false;
    }
    Json j;
    if (!parse_json(hdr.data(), hdr.size(), j, err) || j.kind != Json::Obj) {
        err = path + ": header JSON: " + (err.empty() ? "not an object" : err);
        return false;
    }
    const uint64_t data0 = 8 + hlen, dsize = fsize - data0;
    for (const auto& kv : j.obj) {
        if (kv.first == "__metadata__") continue;
        const Json* dt = kv.second.get("dtype");
        const Json* sh = kv.second.get("shape");
        const Json* of = kv.second.get("data_offsets");
        if (!dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr || !of || of->kind != Json::Arr ||
            of->arr.size() != 2) {
            err = path + ": malformed entry " + kv.first;
            return false;
        }
        Tensor t;
        t.name = kv.first;
        t.dtype = dt->str;
        t.file = path;
        uint64_t elems = 1;
        bool overflow = false;
        for (const Json& d : sh->arr) {
            uint64_t dim = 0;
            if (!json_index(d, dim)) {
                err = path + ": bad shape of " + kv.first;
                return false;
            }
            t.shape.push_back(dim);
            overflow = overflow || __builtin_mul_overflow(elems, dim, &elems);
        }
        uint64_t b = 0, e = 0, nbytes = 0;
        if (!json_index(of->arr[0], b) || !json_index(of->arr[1], e)) {
            err = path + ": data offsets of " + kv.first + " are not non-negative integers below 2^53";
            return false;
        }
        const size_t es = dtype_size(t.dtype);
        overflow = overflow || __builtin_mul_overflow(elems, static_cast<uint64_t>(es ? es : 1), &nbytes);
        if (overflow) {
            err = path + ": shape of " + kv.first + " overflows 64 bits";
            return false;
        }
        if (e < b || e > dsize || (es && e - b != nbytes)) {
            err = path + ": data offsets of " + kv.first + " out of range or inconsistent with its shape";
            return false;
        }
        t.offset = data0 + b;
        t.bytes = e - b;
        out.push_back(std::move(t));
    }
    return true;
}

std::string dir_of(const std::string& p) {
    const size_t s = p.rfind('/');
    return s == std::string::npos ? std::string(".") : p.substr(0, s);
}

bool is_dir(const std::string& p) {
    struct stat st {};
    return stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}
bool exists(const std::string& p) {
    struct stat st {};
    return stat(p.c_str(), &st) == 0;
}

// A .safetensors file, an index .json, or a directory holding either.
bool collect(const std::string& path_in, std::vector<Tensor>& out, std::string& err) {
    std::string path = path_in;
    if (is_dir(path)) {
        if (exists(path + "/model.safetensors.index.json"))
            path += "/model.safetensors.index.json";
        else if (exists(path + "/model.safetensors"))
            path += "/model.safetensors";
        else {
            err = path + ": no model.safetensors or model.safetensors.index.json";
            return false;
        }
    }
    if (path.size() >= 5 && path.compare(path.size() - 5, 5, ".json") == 0) {
        std::string text;
        if (!read_file(path, text, err)) return false;
        Json j;
        if (!parse_json(text.data(), text.size(), j, err)) {
            err = path + ": " + err;
            return false;
        }
        const Json* wm = j.get("weight_map");
        if (!wm || wm->kind != Json::Obj) {
            err = path + ": no weight_map";
            return false;
        }
        std::map<std::string, std::set<std::string>> by_file;  // shard -> tensors the index assigns it
        for (const auto& kv : wm->obj) {
            if (kv.second.kind != Json::Str || kv.second.str.find('/') != std::string::npos) {
                err = path + ": bad shard name for " + kv.first;
                return false;
            }
            by_file[kv.second.str].insert(kv.first);
        }
        for (const auto& f : by_file) {
            std::vector<Tensor> ts;
            if (!scan_file(dir_of(path) + "/" + f.first, ts, err)) return false;
            std::set<std::string> seen;
            for (Tensor& t : ts)
                if (f.second.count(t.name)) {
                    seen.insert(t.name);
                    out.push_back(std::move(t));
                }
            for (const std::string& n : f.second)
                if (!seen.count(n)) {
                    err = path + ": " + n + " is not in " + f.first;
                    return false;
                }
        }
        return true;
    }
    return scan_file(path, out, err);
}

int list_impl(const char* path, char* out, size_t capacity, size_t* needed) {
    std::vector<q3::Tensor> ts;
    std::string err;
    if (!collect(path, ts, err)) return fail(Q3_ERR_INVALID, err);
    std::string text;
    for (const auto& t : ts) {
        text += t.name + '\t' + t.dtype + '\t';
        for (size_t i = 0; i < t.shape.size(); ++i) text += (i ? "x" : "") + std::to_string(t.shape[i]);
        text += '\t' + t.file + '\t' + std::to_string(t.offset) + '\t' + std::to_string(t.bytes) + '\n';
    }
    *needed = text.size() + 1;
    if (out) {
        Q3_CHECK(capacity >= text.size() + 1, "q3_safetensors_list: output buffer too small");
        std::memcpy(out, text.c_str(), text.size() + 1);
    }
    return Q3_OK;
}

int load_impl(q3_engine* e, const char* path, size_t* n_loaded) {
    std::vector<q3::Tensor> ts;
    std::string err;
    if (!collect(path, ts, err)) return fail(Q3_ERR_INVALID, err);
    std::map<std::string, std::unique_ptr<Mapped>> maps;
    std::set<std::string> loaded;
    for (const auto& t : ts) {
        if (t.dtype != "BF16") return fail(Q3_ERR_UNSUPPORTED, t.name + ": dtype " + t.dtype + " (BF16 checkpoints only)");
        Q3_CHECK(t.shape.size() == 1 || t.shape.size() == 2, t.name + ": expected a 1-D or 2-D tensor");
        auto& m = maps[t.file];
        if (!m) {
            m = std::make_unique<Mapped>();
            const int fd = open(t.file.c_str(), O_RDONLY);
            Q3_CHECK(fd >= 0, "cannot open " + t.file);
            struct stat st {};
            if (fstat(fd, &st) == 0 && st.st_size > 0) {
                m->size = static_cast<size_t>(st.st_size);
                m->base = mmap(nullptr, m->size, PROT_READ, MAP_PRIVATE, fd, 0);
            }
            close(fd);
            Q3_CHECK(m->base != MAP_FAILED, "cannot map " + t.file);
        }
        // the file may have changed since its header was read
        Q3_CHECK(t.offset <= m->size && t.bytes <= m->size - t.offset, t.name + ": data past the end of " + t.file);
        // BF16 data must be 2-byte aligned for the row copies
        Q3_CHECK(t.offset % 2 == 0, t.name + ": misaligned data");
        const uint16_t* src = reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(m->base) + t.offset);
        const size_t rows = t.shape.size() == 2 ? t.shape[0] : 1, cols = t.shape.back();
        const int rc = q3_engine_set_weight(e, t.name.c_str(), src, rows, cols);
        if (rc != Q3_OK) return rc;
        loaded.insert(t.name);
    }
    // every tensor the model reads must have arrived
    std::vector<std::string> need = {"model.embed_tokens.weight", "model.norm.weight"};
    if (!engine_tied(e)) need.push_back("lm_head.weight");
    static const char* leaves[] = {"self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                                   "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                                   "mlp.down_proj.weight", "input_layernorm.weight",
                                   "post_attention_layernorm.weight", "self_attn.q_norm.weight",
                                   "self_attn.k_norm.weight"};
    for (size_t l = 0; l < engine_layers(e); ++l)
        for (const char* leaf : leaves) need.push_back("model.layers." + std::to_string(l) + "." + leaf);
    for (const std::string& n : need)
        if (!loaded.count(n)) return fail(Q3_ERR_INVALID, "checkpoint lacks " + n);
    Q3_CUDA(cudaDeviceSynchronize());
    if (n_loaded) *n_loaded = loaded.size();
    return Q3_OK;
}

}  // namespace
}  // namespace q3

using namespace q3;

extern "C" {

int q3_safetensors_list(const char* path, char* out, size_t capacity, size_t* needed) {
    Q3_CHECK(path && needed, "q3_safetensors_list: null argument");
    return guarded("q3_safetensors_list", [&]() -> int { return list_impl(path, out, capacity, needed); });
}

int q3_engine_load_safetensors(q3_engine* e, const char* path, size_t* n_loaded) {
    Q3_CHECK(e && path, "q3_engine_load_safetensors: null argument");
    return guarded("q3_engine_load_safetensors", [&]() -> int { return load_impl(e, path, n_loaded); });
}

}  // extern "C"
