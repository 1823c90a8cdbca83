// kq_gguf.cu -- GGUF v2/v3 tensor directory and device upload (host code).
//
// The engine reads its weights straight from an mmap'ed GGUF file: parse_gguf_file
// (src/v182_r22_breakthrough_engine.c:376-413) walks the header, the key/value pairs (keeping only
// general.alignment) and the tensor records, then places the data section at the next multiple
// of the alignment; find_tensor (ENG:415-420) looks a record up by name; init_sdot_task takes
// base + abs_offset as the weight of a product (ENG:4163-4181).  This file gives the same
// directory to C callers of libkq and copies quantized matrices into the device tile layout
// (kq_weight_upload), so a whole model's matrices can be resident in HBM before the first product.
//
// Same as the reference: magic "GGUF", versions 2 and 3 only, 1-4 dimensions per tensor,
// dims[0] the values per row, alignment 32 unless general.alignment (u32 or u64) says otherwise,
// byte sizes by compute_ggml_bytes (0 for types it does not know).  Stricter: every read and every
// tensor's data range are checked against the file size (the reference trusts the file), names
// are kept whole (the reference truncates them to 127 bytes), nested arrays are rejected as the
// reference does, and there is no 512-tensor cap.
#include "kq_internal.h"
#include "../../include/kq.h"

#include <cstring>
#include <string>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace {

struct GgufTensorRec {
    std::string name;
    uint32_t type = 0, n_dims = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint64_t n_elems = 1, rel_offset = 0, abs_offset = 0, bytes = 0;
};

struct Reader {
    const uint8_t *base;
    size_t size, pos = 0;
    bool bytes(void *dst, size_t n) {
        if (n > size - pos) return false;
        if (dst) memcpy(dst, base + pos, n);
        pos += n;
        return true;
    }
    bool u32(uint32_t &v) { return bytes(&v, 4); }
    bool u64(uint64_t &v) { return bytes(&v, 8); }
    bool str(std::string *out) {
        uint64_t len = 0;
        if (!u64(len) || len > size - pos) return false;
        if (out) out->assign(reinterpret_cast<const char *>(base + pos), (size_t)len);
        pos += (size_t)len;
        return true;
    }
};

// Size of one scalar GGUF value type (uint8/int8/bool 1, (u)int16 2, (u)int32/float32 4,
// (u)int64/float64 8), 0 otherwise (gguf_scalar_size, ENG:316-323).
size_t scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return 0;
    }
}

// Skip one value of type vt; the value of a u32 / u64 scalar goes to *val (ENG:325-362).
bool skip_value(Reader &r, uint32_t vt, uint64_t *val) {
    if (vt == 8) return r.str(nullptr);
    if (vt == 9) {
        uint32_t et = 0;
        uint64_t count = 0;
        if (!r.u32(et) || !r.u64(count)) return false;
        if (et == 8) {
            for (uint64_t i = 0; i < count; ++i)
                if (!r.str(nullptr)) return false;
            return true;
        }
        const size_t es = scalar_size(et);
        if (es == 0 || count > (r.size - r.pos) / es) return false;
        r.pos += (size_t)(count * es);
        return true;
    }
    const size_t s = scalar_size(vt);
    if (s == 0 || s > r.size - r.pos) return false;
    if (val && vt == 4) {
        uint32_t v = 0;
        memcpy(&v, r.base + r.pos, 4);
        *val = v;
    } else if (val && vt == 10) {
        memcpy(val, r.base + r.pos, 8);
    }
    r.pos += s;
    return true;
}

bool quant_type(uint32_t t) {
    return t == KQ_TYPE_Q4_K || t == KQ_TYPE_Q5_K || t == KQ_TYPE_Q6_K || t == KQ_TYPE_Q8_0;
}

}  // namespace

struct kq_gguf {
    const uint8_t *base = nullptr;
    size_t size = 0;
    bool mapped = false;
    uint32_t version = 0;
    uint64_t alignment = 32, data_offset = 0;
    std::vector<GgufTensorRec> tensors;
};

namespace {

int parse(kq_gguf *g) {
    Reader r{g->base, g->size};
    char magic[4];
    uint64_t n_tensors = 0, n_kv = 0;
    if (!r.bytes(magic, 4) || memcmp(magic, "GGUF", 4) != 0) return KQ_ERR_FORMAT;
    if (!r.u32(g->version) || g->version < 2 || g->version > 3) return KQ_ERR_FORMAT;
    if (!r.u64(n_tensors) || !r.u64(n_kv)) return KQ_ERR_FORMAT;
    // every tensor record takes at least 24 bytes: a bound that rejects absurd counts early
    if (n_tensors > g->size / 24) return KQ_ERR_FORMAT;
    g->alignment = 32;
    std::string key;
    for (uint64_t i = 0; i < n_kv; ++i) {
        uint32_t vt = 0;
        uint64_t val = 0;
        if (!r.str(&key) || !r.u32(vt) || !skip_value(r, vt, &val)) return KQ_ERR_FORMAT;
        if (key == "general.alignment" && val > 0) g->alignment = val;
    }
    g->tensors.resize((size_t)n_tensors);
    for (GgufTensorRec &t : g->tensors) {
        if (!r.str(&t.name) || !r.u32(t.n_dims) || t.n_dims < 1 || t.n_dims > 4) return KQ_ERR_FORMAT;
        for (uint32_t d = 0; d < t.n_dims; ++d) {
            if (!r.u64(t.dims[d])) return KQ_ERR_FORMAT;
            t.n_elems *= t.dims[d];
        }
        if (!r.u32(t.type) || !r.u64(t.rel_offset)) return KQ_ERR_FORMAT;
        t.bytes = kq_row_bytes(t.type, t.n_elems);  // compute_ggml_bytes (ENG:364-374)
    }
    g->data_offset = ((uint64_t)r.pos + g->alignment - 1) / g->alignment * g->alignment;
    for (GgufTensorRec &t : g->tensors) {
        t.abs_offset = g->data_offset + t.rel_offset;
        if (t.abs_offset > g->size || t.bytes > g->size - t.abs_offset) return KQ_ERR_FORMAT;
    }
    return KQ_OK;
}

int finish_open(kq_gguf *g, kq_gguf **out) {
    const int st = parse(g);
    if (st != KQ_OK) {
        kq_gguf_close(g);
        return st;
    }
    *out = g;
    return KQ_OK;
}

}  // namespace

extern "C" int kq_gguf_open(const char *path, kq_gguf **out) {
    if (!path || !out) return KQ_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return KQ_ERR_NOT_FOUND;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
        close(fd);
        return KQ_ERR_FORMAT;
    }
    void *p = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return KQ_ERR_OUT_OF_MEMORY;
    kq_gguf *g = new kq_gguf;
    g->base = static_cast<const uint8_t *>(p);
    g->size = (size_t)sb.st_size;
    g->mapped = true;
    return finish_open(g, out);
}

extern "C" int kq_gguf_open_memory(const void *bytes, size_t size, kq_gguf **out) {
    if (!bytes || !out) return KQ_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    kq_gguf *g = new kq_gguf;
    g->base = static_cast<const uint8_t *>(bytes);
    g->size = size;
    return finish_open(g, out);
}

extern "C" int kq_gguf_close(kq_gguf *g) {
    if (!g) return KQ_ERR_INVALID_ARGUMENT;
    if (g->mapped) munmap(const_cast<uint8_t *>(g->base), g->size);
    delete g;
    return KQ_OK;
}

extern "C" int kq_gguf_info(const kq_gguf *g, uint32_t *version, uint64_t *alignment, uint64_t *data_offset) {
    if (!g) return KQ_ERR_INVALID_ARGUMENT;
    if (version) *version = g->version;
    if (alignment) *alignment = g->alignment;
    if (data_offset) *data_offset = g->data_offset;
    return KQ_OK;
}

extern "C" int kq_gguf_tensor_count(const kq_gguf *g) {
    return g ? (int)g->tensors.size() : KQ_ERR_INVALID_ARGUMENT;
}

extern "C" int kq_gguf_get_tensor(const kq_gguf *g, int index, kq_gguf_tensor *out) {
    if (!g || !out) return KQ_ERR_INVALID_ARGUMENT;
    if (index < 0 || index >= (int)g->tensors.size()) return KQ_ERR_NOT_FOUND;
    const GgufTensorRec &t = g->tensors[(size_t)index];
    out->name = t.name.c_str();
    out->type = t.type;
    out->n_dims = t.n_dims;
    for (int d = 0; d < 4; ++d) out->dims[d] = t.dims[d];
    out->n_elems = t.n_elems;
    out->offset = t.abs_offset;
    out->bytes = t.bytes;
    out->data = g->base + t.abs_offset;
    return KQ_OK;
}

extern "C" int kq_gguf_find_tensor(const kq_gguf *g, const char *name) {
    if (!g || !name) return KQ_ERR_INVALID_ARGUMENT;
    for (size_t i = 0; i < g->tensors.size(); ++i)
        if (g->tensors[i].name == name) return (int)i;
    return KQ_ERR_NOT_FOUND;
}

extern "C" int kq_gguf_upload(kq_ctx *ctx, const kq_gguf *g, int index, kq_weight **out) {
    if (!ctx || !g || !out) return KQ_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (index < 0 || index >= (int)g->tensors.size()) return KQ_ERR_NOT_FOUND;
    const GgufTensorRec &t = g->tensors[(size_t)index];
    if (!quant_type(t.type)) return KQ_ERR_UNSUPPORTED_TYPE;
    // a matrix: rows = dims[1], values per row = dims[0]; higher dimensions must be 1
    if (t.dims[2] != 1 || t.dims[3] != 1 || t.dims[0] > (uint64_t)KQ_MAX_K || t.dims[1] > 0x7fffffffull)
        return KQ_ERR_SHAPE;
    return kq_weight_upload(ctx, g->base + t.abs_offset, t.type, (int)t.dims[1], (int)t.dims[0], out);
}

extern "C" int kq_gguf_upload_all(kq_ctx *ctx, const kq_gguf *g, kq_weight **out, int *n_uploaded) {
    if (!ctx || !g || !out) return KQ_ERR_INVALID_ARGUMENT;
    const int n = (int)g->tensors.size();
    for (int i = 0; i < n; ++i) out[i] = nullptr;
    int count = 0;
    for (int i = 0; i < n; ++i) {
        const GgufTensorRec &t = g->tensors[(size_t)i];
        if (!quant_type(t.type) || t.dims[2] != 1 || t.dims[3] != 1 || t.dims[0] % 256 != 0) continue;
        const int st = kq_gguf_upload(ctx, g, i, &out[i]);
        if (st != KQ_OK) {
            for (int j = 0; j < i; ++j)
                if (out[j]) {
                    kq_weight_free(ctx, out[j]);
                    out[j] = nullptr;
                }
            return st;
        }
        ++count;
    }
    if (n_uploaded) *n_uploaded = count;
    return KQ_OK;
}
