// GGUF reader behind the reference's gguf_* C-ABI (reference csrc/gguf.h:62-84, bound by
// sardyne/capi.py:36-51). The file is mapped read-only once; keys and tensor names are copied,
// values and tensor data stay in the mapping. It accepts and rejects the same files as the
// reference parser (csrc/gguf.c:250-320): GGUF v2/v3 little-endian, strict UTF-8 names without
// NUL, no duplicate keys or tensors, known ggml types, ne[0] a multiple of the block, no size
// overflow, power-of-two alignment up to 1 MiB, aligned offsets, data inside the file.
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <vector>

#include "sardyne_b200.h"

namespace {

enum : uint32_t { V_U8, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64 };

struct TypeInfo {
    const char *name;
    uint32_t block, bytes;
};
// ggml type table: name, elements per block, bytes per block (ids as in GGUF).
const TypeInfo *type_info(uint32_t t) {
    static const TypeInfo tab[] = {
        {"F32", 1, 4},       {"F16", 1, 2},       {"Q4_0", 32, 18},    {"Q4_1", 32, 20},    {nullptr, 0, 0},
        {nullptr, 0, 0},     {"Q5_0", 32, 22},    {"Q5_1", 32, 24},    {"Q8_0", 32, 34},    {"Q8_1", 32, 36},
        {"Q2_K", 256, 84},   {"Q3_K", 256, 110},  {"Q4_K", 256, 144},  {"Q5_K", 256, 176},  {"Q6_K", 256, 210},
        {"Q8_K", 256, 292},  {"IQ2_XXS", 256, 66}, {"IQ2_XS", 256, 74}, {"IQ3_XXS", 256, 98}, {"IQ1_S", 256, 50},
        {"IQ4_NL", 32, 18},  {"IQ3_S", 256, 110}, {"IQ2_S", 256, 82},  {"IQ4_XS", 256, 136}, {"I8", 1, 1},
        {"I16", 1, 2},       {"I32", 1, 4},       {"I64", 1, 8},       {"F64", 1, 8},       {"IQ1_M", 256, 56},
        {"BF16", 1, 2},      {nullptr, 0, 0},     {nullptr, 0, 0},     {nullptr, 0, 0},     {"TQ1_0", 256, 54},
        {"TQ2_0", 256, 66},  {nullptr, 0, 0},     {nullptr, 0, 0},     {nullptr, 0, 0},     {"MXFP4", 32, 17},
    };
    return t < sizeof(tab) / sizeof(tab[0]) && tab[t].name ? &tab[t] : nullptr;
}

size_t scalar_size(uint32_t v) {
    switch (v) {
    case V_U8: case V_I8: case V_BOOL: return 1;
    case V_U16: case V_I16: return 2;
    case V_U32: case V_I32: case V_F32: return 4;
    case V_U64: case V_I64: case V_F64: return 8;
    default: return 0;
    }
}

// Strict UTF-8 without NUL: no overlong forms, no surrogates, nothing above U+10FFFF.
bool utf8_ok(const uint8_t *s, uint64_t n) {
    for (uint64_t i = 0; i < n;) {
        uint8_t c = s[i];
        if (c == 0) return false;
        if (c < 0x80) { i++; continue; }
        int len;
        uint32_t cp;
        if ((c & 0xE0) == 0xC0) { len = 2; cp = c & 0x1F; }
        else if ((c & 0xF0) == 0xE0) { len = 3; cp = c & 0x0F; }
        else if ((c & 0xF8) == 0xF0) { len = 4; cp = c & 0x07; }
        else return false;
        if (n - i < (uint64_t)len) return false;
        for (int k = 1; k < len; k++) {
            if ((s[i + k] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (s[i + k] & 0x3F);
        }
        static const uint32_t min_cp[5] = {0, 0, 0x80, 0x800, 0x10000};
        if (cp < min_cp[len] || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
        i += len;
    }
    return true;
}

struct Cursor {
    const uint8_t *base;
    size_t size, pos = 0;
    std::string err;
    bool fail(const char *fmt, ...) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        err = buf;
        return false;
    }
    bool need(uint64_t n) {
        if (n > size - pos) return fail("file troncato all'offset %zu (servono %llu byte)", pos, (unsigned long long)n);
        return true;
    }
    template <class T> bool get(T *v) {
        if (!need(sizeof(T))) return false;
        memcpy(v, base + pos, sizeof(T));
        pos += sizeof(T);
        return true;
    }
    bool name(std::string *out, const char *what) {
        uint64_t n;
        if (!get(&n) || !need(n)) return false;
        if (!utf8_ok(base + pos, n)) return fail("%s all'offset %zu: UTF-8 non valido o byte NUL", what, pos);
        out->assign((const char *)base + pos, n);
        pos += n;
        return true;
    }
};

}  // namespace

struct gguf_file {
    const uint8_t *map = nullptr;
    size_t size = 0;
    uint32_t version = 0, alignment = 32;
    uint64_t data_offset = 0;
    std::vector<std::string> keys, names;
    std::vector<std::vector<uint64_t>> str_pos;
    std::vector<gguf_kv> kv;
    std::vector<gguf_tensor> tensors;
};

static bool parse(gguf_file *f, Cursor &c) {
    char magic[4];
    if (!c.need(4)) return false;
    memcpy(magic, c.base, 4);
    c.pos = 4;
    if (memcmp(magic, "GGUF", 4) != 0) return c.fail("non è un file GGUF (magic errato)");
    if (!c.get(&f->version)) return false;
    if ((f->version & 0xFFFF) == 0 && (f->version >> 24) >= 1 && (f->version >> 24) <= 3)
        return c.fail("file GGUF big-endian non supportato");
    if (f->version != 2 && f->version != 3) return c.fail("versione GGUF %u non supportata", f->version);
    uint64_t n_tensors, n_kv;
    if (!c.get(&n_tensors) || !c.get(&n_kv)) return false;
    if (n_kv > c.size / 12 || n_tensors > c.size / 32) return c.fail("contatori implausibili");

    f->keys.resize(n_kv);
    f->str_pos.resize(n_kv);
    f->kv.assign(n_kv, gguf_kv{});
    for (uint64_t i = 0; i < n_kv; i++) {
        gguf_kv &kv = f->kv[i];
        if (!c.name(&f->keys[i], "chiave") || !c.get(&kv.type)) return false;
        if (kv.type == V_STR) {
            if (!c.get(&kv.n) || !c.need(kv.n)) return false;
            kv.ptr = c.base + c.pos;
            c.pos += kv.n;
        } else if (kv.type == V_ARR) {
            if (!c.get(&kv.arr_type) || !c.get(&kv.n)) return false;
            kv.ptr = c.base + c.pos;
            size_t es = scalar_size(kv.arr_type);
            if (es) {
                if (kv.n > (c.size - c.pos) / es) return c.fail("array oltre la fine del file");
                c.pos += kv.n * es;
            } else if (kv.arr_type == V_STR) {
                if (kv.n > (c.size - c.pos) / 8) return c.fail("array di stringhe oltre la fine del file");
                auto &sp = f->str_pos[i];
                sp.resize(kv.n ? kv.n : 1);
                for (uint64_t j = 0; j < kv.n; j++) {
                    uint64_t len;
                    sp[j] = c.pos;
                    if (!c.get(&len) || !c.need(len)) return false;
                    c.pos += len;
                }
            } else {
                return c.fail("array di tipo %u non supportato", kv.arr_type);
            }
        } else {
            size_t es = scalar_size(kv.type);
            if (!es) return c.fail("tipo di valore sconosciuto %u", kv.type);
            if (!c.need(es)) return false;
            kv.ptr = c.base + c.pos;
            kv.n = 1;
            c.pos += es;
        }
        if (f->keys[i] == "general.alignment") {
            uint64_t a;
            if (gguf_kv_get_u64(f, (int64_t)i, &a) || a == 0 || a > (1u << 20) || (a & (a - 1)))
                return c.fail("general.alignment non valido");
            f->alignment = (uint32_t)a;
        }
    }

    f->names.resize(n_tensors);
    f->tensors.assign(n_tensors, gguf_tensor{});
    for (uint64_t i = 0; i < n_tensors; i++) {
        gguf_tensor &t = f->tensors[i];
        if (!c.name(&f->names[i], "nome di tensore") || !c.get(&t.n_dims)) return false;
        const char *nm = f->names[i].c_str();
        if (t.n_dims < 1 || t.n_dims > 4) return c.fail("%s: n_dims=%u", nm, t.n_dims);
        for (uint32_t d = 0; d < 4; d++) {
            t.ne[d] = 1;
            if (d < t.n_dims && !c.get(&t.ne[d])) return false;
            if (t.ne[d] == 0) return c.fail("%s: dimensione %u nulla", nm, d);
        }
        if (!c.get(&t.type) || !c.get(&t.offset)) return false;
        const TypeInfo *ti = type_info(t.type);
        if (!ti) return c.fail("%s: tipo ggml sconosciuto %u", nm, t.type);
        if (t.ne[0] % ti->block) return c.fail("%s: ne[0] non multiplo del blocco %u", nm, ti->block);
        unsigned __int128 n = 1;
        for (uint32_t d = 0; d < 4; d++) {
            n *= t.ne[d];
            if (n > UINT64_MAX) return c.fail("%s: dimensioni troppo grandi", nm);
        }
        unsigned __int128 nbytes = (n / ti->block) * ti->bytes;
        if (nbytes > UINT64_MAX) return c.fail("%s: dimensioni troppo grandi", nm);
        t.nbytes = (uint64_t)nbytes;
    }

    auto dup = [&](const std::vector<std::string> &v, const char *what) {
        std::vector<const std::string *> p;
        for (auto &s : v) p.push_back(&s);
        std::sort(p.begin(), p.end(), [](const std::string *a, const std::string *b) { return *a < *b; });
        for (size_t i = 1; i < p.size(); i++)
            if (*p[i] == *p[i - 1]) return c.fail("%s duplicato: %s", what, p[i]->c_str());
        return true;
    };
    if (!dup(f->keys, "metadato") || !dup(f->names, "tensore")) return false;

    f->data_offset = (c.pos + f->alignment - 1) / f->alignment * f->alignment;
    if (f->data_offset > c.size) return c.fail("zona dati oltre la fine del file");
    uint64_t data_size = c.size - f->data_offset;
    for (uint64_t i = 0; i < n_tensors; i++) {
        gguf_tensor &t = f->tensors[i];
        if (t.offset % f->alignment) return c.fail("%s: offset non allineato", f->names[i].c_str());
        if (t.offset > data_size || t.nbytes > data_size - t.offset)
            return c.fail("%s: dati oltre la fine del file", f->names[i].c_str());
        t.data = f->map + f->data_offset + t.offset;
    }
    // Pointers into the owned strings are taken last: the vectors no longer reallocate.
    for (uint64_t i = 0; i < n_kv; i++) {
        f->kv[i].key = f->keys[i].c_str();
        f->kv[i].str_pos = f->str_pos[i].empty() ? nullptr : f->str_pos[i].data();
    }
    for (uint64_t i = 0; i < n_tensors; i++) f->tensors[i].name = f->names[i].c_str();
    return true;
}

extern "C" {

const char *gguf_type_name(uint32_t t) {
    const TypeInfo *ti = type_info(t);
    return ti ? ti->name : nullptr;
}

gguf_file *gguf_open(const char *path, char *err, size_t err_len) {
    auto report = [&](const std::string &m) {
        if (err && err_len) snprintf(err, err_len, "%s", m.c_str());
    };
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        report(std::string("impossibile aprire ") + path + ": " + strerror(errno));
        return nullptr;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        report(std::string("impossibile leggere la dimensione di ") + path);
        close(fd);
        return nullptr;
    }
    void *map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    int merr = errno;
    close(fd);
    if (map == MAP_FAILED) {
        report(std::string("mmap fallita su ") + path + ": " + strerror(merr));
        return nullptr;
    }
    gguf_file *f = new gguf_file();
    f->map = (const uint8_t *)map;
    f->size = (size_t)st.st_size;
    Cursor c{f->map, f->size, 0, std::string()};
    if (!parse(f, c)) {
        report(c.err);
        gguf_close(f);
        return nullptr;
    }
    return f;
}

void gguf_close(gguf_file *f) {
    if (!f) return;
    if (f->map) munmap((void *)f->map, f->size);
    delete f;
}

uint32_t gguf_version(const gguf_file *f) { return f ? f->version : 0; }
uint32_t gguf_alignment(const gguf_file *f) { return f ? f->alignment : 0; }
uint64_t gguf_data_offset(const gguf_file *f) { return f ? f->data_offset : 0; }
uint64_t gguf_n_kv(const gguf_file *f) { return f ? f->kv.size() : 0; }
uint64_t gguf_n_tensors(const gguf_file *f) { return f ? f->tensors.size() : 0; }

const gguf_kv *gguf_get_kv(const gguf_file *f, uint64_t i) { return f && i < f->kv.size() ? &f->kv[i] : nullptr; }
const gguf_tensor *gguf_get_tensor(const gguf_file *f, uint64_t i) {
    return f && i < f->tensors.size() ? &f->tensors[i] : nullptr;
}

int64_t gguf_find_kv(const gguf_file *f, const char *key) {
    if (!f || !key) return -1;
    for (size_t i = 0; i < f->keys.size(); i++)
        if (f->keys[i] == key) return (int64_t)i;
    return -1;
}
int64_t gguf_find_tensor(const gguf_file *f, const char *name) {
    if (!f || !name) return -1;
    for (size_t i = 0; i < f->names.size(); i++)
        if (f->names[i] == name) return (int64_t)i;
    return -1;
}

int gguf_kv_get_u64(const gguf_file *f, int64_t i, uint64_t *out) {
    if (!f || !out || i < 0 || (uint64_t)i >= f->kv.size()) return -1;
    const gguf_kv &kv = f->kv[i];
    int64_t s;
    switch (kv.type) {
    case V_U8: *out = kv.ptr[0]; return 0;
    case V_U16: { uint16_t v; memcpy(&v, kv.ptr, 2); *out = v; return 0; }
    case V_U32: { uint32_t v; memcpy(&v, kv.ptr, 4); *out = v; return 0; }
    case V_U64: memcpy(out, kv.ptr, 8); return 0;
    case V_I8: s = (int8_t)kv.ptr[0]; break;
    case V_I16: { int16_t v; memcpy(&v, kv.ptr, 2); s = v; break; }
    case V_I32: { int32_t v; memcpy(&v, kv.ptr, 4); s = v; break; }
    case V_I64: memcpy(&s, kv.ptr, 8); break;
    default: return -1;
    }
    if (s < 0) return -1;
    *out = (uint64_t)s;
    return 0;
}

int gguf_kv_get_f64(const gguf_file *f, int64_t i, double *out) {
    if (!f || !out || i < 0 || (uint64_t)i >= f->kv.size()) return -1;
    const gguf_kv &kv = f->kv[i];
    if (kv.type == V_F32) { float v; memcpy(&v, kv.ptr, 4); *out = v; return 0; }
    if (kv.type == V_F64) { memcpy(out, kv.ptr, 8); return 0; }
    return -1;
}

const char *gguf_kv_get_str(const gguf_file *f, int64_t i, uint64_t *len) {
    if (!f || !len || i < 0 || (uint64_t)i >= f->kv.size() || f->kv[i].type != V_STR) return nullptr;
    *len = f->kv[i].n;
    return (const char *)f->kv[i].ptr;
}

const char *gguf_kv_get_arr_str(const gguf_file *f, int64_t i, uint64_t j, uint64_t *len) {
    if (!f || !len || i < 0 || (uint64_t)i >= f->kv.size()) return nullptr;
    const gguf_kv &kv = f->kv[i];
    if (kv.type != V_ARR || kv.arr_type != V_STR || j >= kv.n) return nullptr;
    uint64_t pos = kv.str_pos[j], n;
    memcpy(&n, f->map + pos, 8);
    *len = n;
    return (const char *)f->map + pos + 8;
}

}  // extern "C"
