// gguf.cu -- host-side GGUF reader: the tensor index of a GGUF v2/v3 file,
// enough to place a model's expert, router and norm tensors in HBM.
//
// Reference interface replaced: gguf_open / gguf_find_tensor /
// ggml_tensor_nbytes (gguf.c:306-411, gguf.h:80-135), which print and exit(1)
// on a malformed file.  Same format rules: little-endian header
// {magic "GGUF", u32 version 2..3, u64 n_tensors, u64 n_kv}; n_kv metadata
// pairs {string key, u32 value type, value} of which only general.alignment
// (u32) is kept (default 32); n_tensors infos {string name, u32 n_dims <= 4,
// u64 dims[n_dims] (dims[0] innermost), u32 ggml type, u64 offset from the
// data section}; the data section starts at the next multiple of the
// alignment after the infos.  A string is {u64 length, bytes}.  Here every
// read is checked against the file size and failures return status codes.
#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

#include "common.cuh"

struct bread_gguf {
    FILE *fp = nullptr;
    uint32_t version = 0, alignment = 32;
    uint64_t file_size = 0, data_off = 0;
    std::vector<std::string> names;
    std::vector<bread_gguf_tensor_t> tensors;
};

namespace bread {

// (elements per block, bytes per block) of the ggml types (gguf.c:60-100)
static bool ggml_block(uint32_t type, uint64_t &be, uint64_t &bb)
{
    struct T {
        uint32_t t, be, bb;
    };
    static const T tab[] = {
        {0, 1, 4},     {1, 1, 2},     {30, 1, 2},    {28, 1, 8},    {24, 1, 1},    {25, 1, 2},
        {26, 1, 4},    {27, 1, 8},    {2, 32, 18},   {3, 32, 20},   {6, 32, 22},   {7, 32, 24},
        {8, 32, 34},   {9, 32, 36},   {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
        {14, 256, 210}, {15, 256, 292}, {16, 256, 66}, {17, 256, 74}, {18, 256, 98}, {19, 256, 50},
        {20, 32, 18},  {21, 256, 110}, {22, 256, 84}, {23, 256, 136}, {29, 256, 56},
    };
    for (const T &e : tab)
        if (e.t == type) {
            be = e.be;
            bb = e.bb;
            return true;
        }
    return false;
}

struct Reader {
    FILE *fp;
    uint64_t size;
    bool ok = true;
    uint64_t pos() const { return (uint64_t)ftello(fp); }
    bool read(void *dst, size_t n)
    {
        if (!ok || pos() + n > size || fread(dst, 1, n, fp) != n) ok = false;
        return ok;
    }
    bool skip(uint64_t n)
    {
        if (!ok || pos() + n > size || fseeko(fp, (off_t)n, SEEK_CUR) != 0) ok = false;
        return ok;
    }
    uint32_t u32()
    {
        uint32_t v = 0;
        read(&v, 4);
        return v;
    }
    uint64_t u64()
    {
        uint64_t v = 0;
        read(&v, 8);
        return v;
    }
    bool str(std::string *out)
    {
        const uint64_t n = u64();
        if (!ok || n > size) return ok = false;
        if (!out) return skip(n);
        out->resize((size_t)n);
        return n ? read(&(*out)[0], (size_t)n) : ok;
    }
    // one metadata value of type vt (gguf.c:182-240), nested arrays included
    bool skip_value(uint32_t vt, int depth = 0)
    {
        static const uint8_t fixed[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (vt > 12 || depth > 8) return ok = false;
        if (vt == 8) return str(nullptr);
        if (vt != 9) return skip(fixed[vt]);
        const uint32_t et = u32();
        const uint64_t count = u64();
        if (!ok || et > 12) return ok = false;
        if (et != 8 && et != 9) {
            if (count > size) return ok = false;
            return skip(count * fixed[et]);
        }
        for (uint64_t i = 0; i < count && ok; ++i) skip_value(et, depth + 1);
        return ok;
    }
};

}  // namespace bread

using namespace bread;

extern "C" int bread_gguf_close(bread_gguf_t *g)
{
    if (!g) return BREAD_OK;
    if (g->fp) fclose(g->fp);
    delete g;
    return BREAD_OK;
}

extern "C" int bread_gguf_open(const char *path, bread_gguf_t **out)
{
    if (!path || !out) return set_error(BREAD_ERR_ARG, "gguf_open: NULL argument");
    *out = nullptr;
    FILE *fp = fopen(path, "rb");
    if (!fp) return set_error(BREAD_ERR_ARG, "gguf_open: cannot open '%s'", path);
    bread_gguf *g = new bread_gguf();
    g->fp = fp;
    setvbuf(fp, nullptr, _IOFBF, 1 << 20);
    fseeko(fp, 0, SEEK_END);
    g->file_size = (uint64_t)ftello(fp);
    fseeko(fp, 0, SEEK_SET);
    Reader r{fp, g->file_size};
    auto fail = [&](const char *what) {
        set_error(BREAD_ERR_ARG, "gguf_open: '%s': %s", path, what);
        bread_gguf_close(g);
        return BREAD_ERR_ARG;
    };
    if (r.u32() != 0x46554747u) return fail(r.ok ? "bad magic (not a GGUF file)" : "truncated header");
    g->version = r.u32();
    if (!r.ok || g->version < 2 || g->version > 3) return fail("unsupported version (2 and 3 are)");
    const uint64_t n_tensors = r.u64(), n_kv = r.u64();
    if (!r.ok || n_tensors > g->file_size || n_kv > g->file_size) return fail("truncated or corrupt header");
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        std::string key;
        r.str(&key);
        const uint32_t vt = r.u32();
        if (r.ok && key == "general.alignment" && vt == 4) {
            g->alignment = r.u32();
            if (!g->alignment || (g->alignment & (g->alignment - 1))) return fail("general.alignment not a power of two");
        } else {
            r.skip_value(vt);
        }
    }
    if (!r.ok) return fail("truncated or corrupt metadata");
    g->names.resize((size_t)n_tensors);
    g->tensors.resize((size_t)n_tensors);
    for (uint64_t i = 0; i < n_tensors; ++i) {
        bread_gguf_tensor_t &t = g->tensors[i];
        memset(&t, 0, sizeof t);
        r.str(&g->names[i]);
        t.n_dims = r.u32();
        if (!r.ok || t.n_dims > 4) return fail("tensor info truncated or with more than 4 dims");
        t.n_elems = 1;
        for (uint32_t d = 0; d < t.n_dims; ++d) {
            t.dims[d] = r.u64();
            t.n_elems *= t.dims[d];
        }
        t.type = r.u32();
        t.offset = r.u64();
        if (!r.ok) return fail("tensor info truncated");
        uint64_t be = 0, bb = 0;
        t.size = ggml_block(t.type, be, bb) ? t.n_elems / be * bb : 0;
    }
    const uint64_t after = r.pos();
    g->data_off = (after + g->alignment - 1) / g->alignment * g->alignment;
    for (uint64_t i = 0; i < n_tensors; ++i) {
        bread_gguf_tensor_t &t = g->tensors[i];
        t.name = g->names[i].c_str();
        if (t.size && g->data_off + t.offset + t.size > g->file_size) return fail("a tensor's data lies beyond the file end");
    }
    *out = g;
    return BREAD_OK;
}

extern "C" int bread_gguf_info(const bread_gguf_t *g, uint32_t *version, uint64_t *n_tensors, uint32_t *alignment,
                               uint64_t *data_offset)
{
    if (!g) return set_error(BREAD_ERR_ARG, "gguf_info: NULL file");
    if (version) *version = g->version;
    if (n_tensors) *n_tensors = g->tensors.size();
    if (alignment) *alignment = g->alignment;
    if (data_offset) *data_offset = g->data_off;
    return BREAD_OK;
}

extern "C" int bread_gguf_tensor(const bread_gguf_t *g, uint64_t index, bread_gguf_tensor_t *out)
{
    if (!g || !out || index >= g->tensors.size()) return set_error(BREAD_ERR_ARG, "gguf_tensor: bad index");
    *out = g->tensors[index];
    return BREAD_OK;
}

extern "C" int bread_gguf_find(const bread_gguf_t *g, const char *name, bread_gguf_tensor_t *out)
{
    if (!g || !name) return set_error(BREAD_ERR_ARG, "gguf_find: NULL argument");
    for (size_t i = 0; i < g->tensors.size(); ++i)
        if (g->names[i] == name) {
            if (out) *out = g->tensors[i];
            return BREAD_OK;
        }
    return set_error(BREAD_ERR_ARG, "gguf_find: no tensor '%s'", name);
}

// Reads `bytes` at `offset` from the tensor data section into host memory.
extern "C" int bread_gguf_read(const bread_gguf_t *g, uint64_t offset, void *dst, uint64_t bytes)
{
    if (!g || (!dst && bytes)) return set_error(BREAD_ERR_ARG, "gguf_read: NULL argument");
    if (g->data_off + offset + bytes > g->file_size) return set_error(BREAD_ERR_ARG, "gguf_read: beyond the file end");
    if (fseeko(g->fp, (off_t)(g->data_off + offset), SEEK_SET) != 0 || fread(dst, 1, bytes, g->fp) != bytes)
        return set_error(BREAD_ERR_ARG, "gguf_read: short read");
    return BREAD_OK;
}
