// gguf.cpp — reader of GGUF weight files, feeding hymoe_load_layer without a host copy.
//
// The reference writes one GGUF file per decoder layer (scripts/convert_to_gguf.py:157-209,
// tensor names :70-137) and reads it through ggml's gguf API, dequantising every tensor to F32
// (src/hunyuan_gguf_loader.cpp:125-281).  Here the file is parsed by this code (GGUF versions 2
// and 3: header, key/value section, tensor infos, aligned data section) and memory-mapped
// read-only; tensors are handed on as views of their raw GGUF blocks, which the device loader
// re-tiles (standard Q4_0/Q8_0 blocks: element j in the low nibble of byte j, element j+16 in
// the high one, value (q-8)*d; not the reference loader's interleaved two's-complement decode,
// src/hunyuan_gguf_loader.cpp:41-72).
//
// Every length, count and extent read from the file is checked against the file size before
// use; a malformed file gives HYMOE_ERR_INVALID_ARG and a message, never a read outside the
// mapping.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "hymoe.h"

namespace {

thread_local std::string g_gguf_error;

hymoe_status gfail(hymoe_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_gguf_error = buf;
    return st;
}

// GGUF value types (the published format).
enum : uint32_t {
    V_U8 = 0, V_I8 = 1, V_U16 = 2, V_I16 = 3, V_U32 = 4, V_I32 = 5, V_F32 = 6, V_BOOL = 7,
    V_STRING = 8, V_ARRAY = 9, V_U64 = 10, V_I64 = 11, V_F64 = 12
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case V_U8: case V_I8: case V_BOOL: return 1;
        case V_U16: case V_I16: return 2;
        case V_U32: case V_I32: case V_F32: return 4;
        case V_U64: case V_I64: case V_F64: return 8;
        default: return 0;
    }
}

// Bytes of a tensor of n elements for the block types this library loads; 0 otherwise.
size_t type_bytes(uint32_t type, uint64_t n) {
    switch (type) {
        case HYMOE_TYPE_F32: return n * 4;
        case HYMOE_TYPE_F16: return n * 2;
        case HYMOE_TYPE_Q4_0: return n % 32 ? 0 : n / 32 * 18;
        case HYMOE_TYPE_Q8_0: return n % 32 ? 0 : n / 32 * 34;
        default: return 0;
    }
}

// Bounds-checked little-endian cursor over the mapping.
struct Cursor {
    const uint8_t* p;
    size_t size, pos = 0;
    bool ok = true;
    bool take(void* dst, size_t n) {
        if (!ok || n > size - pos) return ok = false;
        std::memcpy(dst, p + pos, n);
        pos += n;
        return true;
    }
    bool skip(uint64_t n) {
        if (!ok || n > size - pos) return ok = false;
        pos += static_cast<size_t>(n);
        return true;
    }
    template <class T>
    T get() {
        T v{};
        take(&v, sizeof(T));
        return v;
    }
    bool string(std::string* s) {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > size - pos) return ok = false;
        if (s) s->assign(reinterpret_cast<const char*>(p + pos), static_cast<size_t>(n));
        pos += static_cast<size_t>(n);
        return true;
    }
};

}  // namespace

struct hymoe_gguf {
    int fd = -1;
    const uint8_t* base = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint32_t alignment = 32;
    size_t data_start = 0;
    struct Info {
        uint32_t n_dims = 0;
        int64_t ne[4] = {1, 1, 1, 1};
        uint32_t type = 0;
        uint64_t offset = 0;  // from data_start
        size_t nbytes = 0;    // 0: a type this library does not load
    };
    struct KV {
        uint32_t type = 0;
        size_t pos = 0;  // file position of the value
    };
    std::unordered_map<std::string, Info> tensors;
    std::unordered_map<std::string, KV> kv;
    ~hymoe_gguf() {
        if (base) munmap(const_cast<uint8_t*>(base), size);
        if (fd >= 0) close(fd);
    }
};

namespace {

hymoe_status parse(hymoe_gguf* f) {
    Cursor c{f->base, f->size};
    char magic[4];
    if (!c.take(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0)
        return gfail(HYMOE_ERR_INVALID_ARG, "not a GGUF file (magic)");
    f->version = c.get<uint32_t>();
    if (!c.ok || (f->version != 2 && f->version != 3))
        return gfail(HYMOE_ERR_UNSUPPORTED, "GGUF version %u (2 and 3 are read)", f->version);
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    // every entry takes at least 8 bytes of the file: bounds the loops before they start
    if (!c.ok || n_tensors > f->size / 8 || n_kv > f->size / 8)
        return gfail(HYMOE_ERR_INVALID_ARG, "GGUF header counts exceed the file");
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key;
        if (!c.string(&key)) break;
        hymoe_gguf::KV v;
        v.type = c.get<uint32_t>();
        v.pos = c.pos;
        if (!c.ok) break;
        if (v.type == V_STRING) {
            c.string(nullptr);
        } else if (v.type == V_ARRAY) {
            const uint32_t et = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            if (!c.ok) break;
            if (et == V_STRING) {
                for (uint64_t j = 0; j < n && c.ok; ++j) c.string(nullptr);
            } else {
                const size_t es = scalar_size(et);
                if (es == 0 || n > (c.size - c.pos) / es)
                    return gfail(HYMOE_ERR_INVALID_ARG, "GGUF key %s: bad array", key.c_str());
                c.skip(n * es);
            }
        } else {
            const size_t es = scalar_size(v.type);
            if (es == 0) return gfail(HYMOE_ERR_INVALID_ARG, "GGUF key %s: value type %u", key.c_str(), v.type);
            c.skip(es);
        }
        if (!c.ok) break;
        if (key == "general.alignment") {
            if (v.type != V_U32) return gfail(HYMOE_ERR_INVALID_ARG, "general.alignment is not u32");
            uint32_t a;
            std::memcpy(&a, f->base + v.pos, 4);
            if (a == 0 || (a & (a - 1)) != 0) return gfail(HYMOE_ERR_INVALID_ARG, "alignment %u", a);
            f->alignment = a;
        }
        f->kv[key] = v;
    }
    if (!c.ok) return gfail(HYMOE_ERR_INVALID_ARG, "GGUF key/value section runs past the file end");
    std::vector<std::pair<std::string, hymoe_gguf::Info>> infos;
    for (uint64_t i = 0; i < n_tensors; ++i) {
        std::string name;
        hymoe_gguf::Info t;
        if (!c.string(&name)) break;
        t.n_dims = c.get<uint32_t>();
        if (!c.ok || t.n_dims == 0 || t.n_dims > 4)
            return gfail(HYMOE_ERR_INVALID_ARG, "tensor %s: %u dims", name.c_str(), t.n_dims);
        uint64_t n = 1;
        for (uint32_t d = 0; d < t.n_dims; ++d) {
            const uint64_t v = c.get<uint64_t>();
            if (!c.ok) break;
            if (v == 0 || v > (1ull << 40) || n > (1ull << 40) / v)
                return gfail(HYMOE_ERR_INVALID_ARG, "tensor %s: dimension %llu", name.c_str(),
                             static_cast<unsigned long long>(v));
            t.ne[d] = static_cast<int64_t>(v);
            n *= v;
        }
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        if (!c.ok) break;
        t.nbytes = type_bytes(t.type, n);
        infos.emplace_back(std::move(name), t);
    }
    if (!c.ok) return gfail(HYMOE_ERR_INVALID_ARG, "GGUF tensor infos run past the file end");
    const size_t a = f->alignment;
    f->data_start = (c.pos + a - 1) / a * a;
    for (auto& [name, t] : infos) {
        if (t.nbytes != 0 && (f->data_start > f->size || t.offset > f->size - f->data_start ||
                              t.nbytes > f->size - f->data_start - t.offset))
            return gfail(HYMOE_ERR_INVALID_ARG, "tensor %s: data runs past the file end", name.c_str());
        if (!f->tensors.emplace(name, t).second)
            return gfail(HYMOE_ERR_INVALID_ARG, "tensor %s appears twice", name.c_str());
    }
    return HYMOE_OK;
}

}  // namespace

extern "C" {

const char* hymoe_gguf_last_error(void) { return g_gguf_error.c_str(); }

hymoe_status hymoe_gguf_open(const char* path, hymoe_gguf** out) {
    if (!path || !out) return gfail(HYMOE_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    auto* f = new hymoe_gguf();
    f->fd = open(path, O_RDONLY | O_CLOEXEC);
    struct stat sb;
    if (f->fd < 0 || fstat(f->fd, &sb) != 0) {
        delete f;
        return gfail(HYMOE_ERR_INVALID_ARG, "cannot open %s", path);
    }
    f->size = static_cast<size_t>(sb.st_size);
    if (f->size < 24) {
        delete f;
        return gfail(HYMOE_ERR_INVALID_ARG, "%s: too short for a GGUF header", path);
    }
    void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
    if (m == MAP_FAILED) {
        delete f;
        return gfail(HYMOE_ERR_INVALID_ARG, "%s: mmap failed", path);
    }
    f->base = static_cast<const uint8_t*>(m);
    const hymoe_status st = parse(f);
    if (st != HYMOE_OK) {
        delete f;
        return st;
    }
    *out = f;
    return HYMOE_OK;
}

void hymoe_gguf_close(hymoe_gguf* f) { delete f; }

hymoe_status hymoe_gguf_tensor(const hymoe_gguf* f, const char* name, hymoe_tensor* out) {
    if (!f || !name || !out) return gfail(HYMOE_ERR_INVALID_ARG, "null argument");
    const auto it = f->tensors.find(name);
    if (it == f->tensors.end()) return gfail(HYMOE_ERR_INVALID_ARG, "no tensor %s", name);
    const hymoe_gguf::Info& t = it->second;
    if (t.nbytes == 0) return gfail(HYMOE_ERR_UNSUPPORTED, "tensor %s: GGUF type %u", name, t.type);
    if (t.n_dims > 2) return gfail(HYMOE_ERR_UNSUPPORTED, "tensor %s: %u dims", name, t.n_dims);
    out->data = f->base + f->data_start + t.offset;
    out->ggml_type = static_cast<int32_t>(t.type);
    out->ne[0] = t.ne[0];
    out->ne[1] = t.ne[1];
    out->nbytes = t.nbytes;
    return HYMOE_OK;
}

hymoe_status hymoe_gguf_get_u32(const hymoe_gguf* f, const char* key, uint32_t* out) {
    if (!f || !key || !out) return gfail(HYMOE_ERR_INVALID_ARG, "null argument");
    const auto it = f->kv.find(key);
    if (it == f->kv.end()) return gfail(HYMOE_ERR_INVALID_ARG, "no key %s", key);
    if (it->second.type != V_U32) return gfail(HYMOE_ERR_INVALID_ARG, "key %s is not u32", key);
    std::memcpy(out, f->base + it->second.pos, 4);
    return HYMOE_OK;
}

hymoe_status hymoe_gguf_moe_tensors(const hymoe_gguf* f, uint32_t layer_idx, uint32_t n_experts,
                                    hymoe_tensor* router, hymoe_tensor* shared_gate_up,
                                    hymoe_tensor* shared_down, hymoe_tensor* experts_gate_up,
                                    hymoe_tensor* experts_down) {
    if (!f || !router || !shared_gate_up || !shared_down || (n_experts && (!experts_gate_up || !experts_down)))
        return gfail(HYMOE_ERR_INVALID_ARG, "null argument");
    char name[128];
    auto one = [&](const char* what, hymoe_tensor* t) {
        snprintf(name, sizeof(name), "blk.%u.%s.weight", layer_idx, what);
        return hymoe_gguf_tensor(f, name, t);
    };
    hymoe_status st = one("ffn_gate", router);
    if (st == HYMOE_OK) st = one("ffn_shared_gate_up", shared_gate_up);
    if (st == HYMOE_OK) st = one("ffn_shared_down", shared_down);
    for (uint32_t e = 0; e < n_experts && st == HYMOE_OK; ++e) {
        char what[64];
        snprintf(what, sizeof(what), "ffn_expert_%u_gate_up", e);
        st = one(what, &experts_gate_up[e]);
        if (st == HYMOE_OK) {
            snprintf(what, sizeof(what), "ffn_expert_%u_down", e);
            st = one(what, &experts_down[e]);
        }
    }
    return st;
}

}  // extern "C"
