// gguf.cu — a read-only view of a GGUF v2/v3 model file (host code).
//
// The GGUF container (the format comment of ggml's gguf.h): the magic "GGUF", a u32 version, a
// u64 tensor count and a u64 key/value count, the key/value pairs (a string key, a u32 value
// type, the value), the tensor index (a string name, a u32 rank, that many u64 dimensions
// fastest-varying first, a u32 ggml type, a u64 offset into the data blob), then the data blob
// at the next multiple of general.alignment (default 32). Strings are a u64 length and that
// many bytes; everything is little-endian.
//
// The file is mapped read-only and parsed in place. Every count and length is checked against
// the bytes that are left before it is used (a corrupt header can claim a 2^63-element array),
// and every tensor's data must lie inside the file, as the reference's reader requires
// (crates/moearc-model/src/gguf.rs:166-279). Stacked expert tensors are addressed slice by slice
// along their last dimension with the checks of tensors.rs:237-289.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace {

thread_local std::string g_err;

int fail_arg(const std::string &m) {
    g_err = m;
    return moearc::ERR_ARG;
}

// ggml's block geometry per type id (elements per block, bytes per block): the public
// type-traits table of ggml; ids this reader does not know are refused at open.
struct qtype {
    unsigned id, block, bytes;
};
constexpr unsigned QK_K = 256;
constexpr qtype QTYPES[] = {
    {0, 1, 4},        {1, 1, 2},        {2, 32, 18},      {3, 32, 20},     {6, 32, 22},       {7, 32, 24},
    {8, 32, 34},      {10, QK_K, 84},   {11, QK_K, 110},  {12, QK_K, 144}, {13, QK_K, 176},   {14, QK_K, 210},
    {15, QK_K, 292},  {16, QK_K, 66},   {17, QK_K, 74},   {18, QK_K, 98},  {19, QK_K, 50},    {20, 32, 18},
    {21, QK_K, 110},  {22, QK_K, 82},   {23, QK_K, 136},  {24, 1, 1},      {25, 1, 2},        {26, 1, 4},
    {27, 1, 8},       {28, 1, 8},       {29, QK_K, 56},   {30, 1, 2},      {34, QK_K, 54},    {35, QK_K, 66},
    {39, 32, 17},
};
const qtype *qtype_of(unsigned id) {
    for (const qtype &t : QTYPES)
        if (t.id == id) return &t;
    return nullptr;
}

constexpr uint64_t DEFAULT_ALIGNMENT = 32;
constexpr uint32_t MAX_DIMS = 4;
constexpr uint64_t MAX_STRING = 1ull << 26;           // longest string materialised
constexpr uint64_t MIN_KV_BYTES = 8 + 4 + 1;          // an empty key, a type, a one-byte value
constexpr uint64_t MIN_TENSOR_BYTES = 8 + 4 + 4 + 8;  // an empty name, a rank, a type, an offset

// value types of the key/value block (gguf.h's enum gguf_type)
enum : uint32_t { V_U8 = 0, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STRING, V_ARRAY, V_U64, V_I64, V_F64 };
int fixed_width(uint32_t t) {
    switch (t) {
    case V_U8: case V_I8: case V_BOOL: return 1;
    case V_U16: case V_I16: return 2;
    case V_U32: case V_I32: case V_F32: return 4;
    case V_U64: case V_I64: case V_F64: return 8;
    default: return 0;
    }
}

struct kv_value {
    uint32_t type;      // scalar type, V_STRING, or V_ARRAY
    uint64_t u = 0;     // unsigned integers and bools
    int64_t i = 0;      // signed integers
    double f = 0.0;     // f32 / f64
    std::string s;      // strings
    uint32_t elem = 0;  // arrays: element type and count (elements are not kept)
    uint64_t len = 0;
};

struct tensor_rec {
    std::string name;
    uint32_t n_dims;
    uint64_t dims[MAX_DIMS];
    uint32_t type;
    uint64_t offset;  // into the data blob
    uint64_t nbytes;
};

struct cursor {
    const uint8_t *base;
    uint64_t size, pos = 0;
    bool need(uint64_t n) const { return n <= size - pos; }
    template <typename T>
    bool get(T &v) {
        if (!need(sizeof(T))) return false;
        std::memcpy(&v, base + pos, sizeof(T));
        pos += sizeof(T);
        return true;
    }
    bool str(std::string &s) {
        uint64_t n;
        if (!get(n) || n > MAX_STRING || !need(n)) return false;
        s.assign(reinterpret_cast<const char *>(base + pos), n);
        pos += n;
        return true;
    }
    bool skip(uint64_t n) {
        if (!need(n)) return false;
        pos += n;
        return true;
    }
};

uint64_t pad_to(uint64_t n, uint64_t a) { return (n + a - 1) / a * a; }

}  // namespace

struct moearc_x_gguf {
    int fd = -1;
    void *map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = DEFAULT_ALIGNMENT, data_offset = 0;
    std::unordered_map<std::string, kv_value> kv;
    std::vector<tensor_rec> tensors;
    std::unordered_map<std::string, size_t> by_name;
};

namespace {

void close_file(moearc_x_gguf *g) {
    if (g->map && g->map != MAP_FAILED) munmap(g->map, g->size);
    if (g->fd >= 0) ::close(g->fd);
    delete g;
}

bool read_scalar(cursor &c, kv_value &v) {
    switch (v.type) {
    case V_U8: { uint8_t x; if (!c.get(x)) return false; v.u = x; return true; }
    case V_I8: { int8_t x; if (!c.get(x)) return false; v.i = x; return true; }
    case V_U16: { uint16_t x; if (!c.get(x)) return false; v.u = x; return true; }
    case V_I16: { int16_t x; if (!c.get(x)) return false; v.i = x; return true; }
    case V_U32: { uint32_t x; if (!c.get(x)) return false; v.u = x; return true; }
    case V_I32: { int32_t x; if (!c.get(x)) return false; v.i = x; return true; }
    case V_F32: { float x; if (!c.get(x)) return false; v.f = x; return true; }
    case V_BOOL: { uint8_t x; if (!c.get(x)) return false; v.u = x != 0; return true; }
    case V_U64: { uint64_t x; if (!c.get(x)) return false; v.u = x; return true; }
    case V_I64: { int64_t x; if (!c.get(x)) return false; v.i = x; return true; }
    case V_F64: { double x; if (!c.get(x)) return false; v.f = x; return true; }
    default: return false;
    }
}

// Parse the header in the mapping; "" on success, else the reason.
std::string parse(moearc_x_gguf *g) {
    cursor c{static_cast<const uint8_t *>(g->map), g->size};
    char magic[4];
    if (!c.get(magic)) return "truncated before the magic";
    if (std::memcmp(magic, "GGUF", 4) != 0) return "bad magic (not a GGUF file)";
    if (!c.get(g->version)) return "truncated in the version";
    if (g->version < 2 || g->version > 3) return "unsupported GGUF version " + std::to_string(g->version);
    uint64_t n_tensors, n_kv;
    if (!c.get(n_tensors) || !c.get(n_kv)) return "truncated in the counts";
    // a count whose smallest possible encoding is larger than the file cannot describe it
    if (n_kv > g->size / MIN_KV_BYTES) return "implausible metadata key count " + std::to_string(n_kv);
    if (n_tensors > g->size / MIN_TENSOR_BYTES) return "implausible tensor count " + std::to_string(n_tensors);

    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key;
        uint32_t type;
        if (!c.str(key)) return "truncated or oversized key " + std::to_string(k);
        if (!c.get(type)) return "truncated in the type of key '" + key + "'";
        kv_value v;
        v.type = type;
        if (type == V_STRING) {
            if (!c.str(v.s)) return "truncated or oversized string value of '" + key + "'";
        } else if (type == V_ARRAY) {
            if (!c.get(v.elem) || !c.get(v.len)) return "truncated array header of '" + key + "'";
            if (v.elem == V_ARRAY) return "nested array in '" + key + "'";
            const int w = fixed_width(v.elem);
            if (w) {
                if (v.len > (c.size - c.pos) / (uint64_t)w || !c.skip(v.len * (uint64_t)w))
                    return "array of '" + key + "' overruns the file";
            } else if (v.elem == V_STRING) {
                // each element takes at least its 8-byte length, so the loop ends with the file
                for (uint64_t j = 0; j < v.len; ++j) {
                    uint64_t n;
                    if (!c.get(n) || !c.skip(n)) return "string array of '" + key + "' overruns the file";
                }
            } else {
                return "bad array element type " + std::to_string(v.elem) + " in '" + key + "'";
            }
        } else if (fixed_width(type)) {
            if (!read_scalar(c, v)) return "truncated value of '" + key + "'";
        } else {
            return "bad value type " + std::to_string(type) + " of '" + key + "'";
        }
        g->kv[key] = std::move(v);  // a repeated key: the later one wins
    }

    auto al = g->kv.find("general.alignment");
    if (al != g->kv.end()) {
        const kv_value &v = al->second;
        if (v.type == V_U8 || v.type == V_U16 || v.type == V_U32 || v.type == V_U64) g->alignment = v.u;
        else if ((v.type == V_I8 || v.type == V_I16 || v.type == V_I32 || v.type == V_I64) && v.i > 0)
            g->alignment = (uint64_t)v.i;
        else return "general.alignment is not a positive integer";
    }
    if (g->alignment == 0 || (g->alignment & (g->alignment - 1)) != 0)
        return "general.alignment " + std::to_string(g->alignment) + " is not a power of two";

    g->tensors.reserve((size_t)n_tensors);
    for (uint64_t t = 0; t < n_tensors; ++t) {
        tensor_rec r{};
        if (!c.str(r.name)) return "truncated or oversized name of tensor " + std::to_string(t);
        if (!c.get(r.n_dims)) return "truncated rank of '" + r.name + "'";
        if (r.n_dims == 0 || r.n_dims > MAX_DIMS) return "tensor '" + r.name + "' has rank " + std::to_string(r.n_dims);
        for (uint32_t d = 0; d < r.n_dims; ++d)
            if (!c.get(r.dims[d])) return "truncated dimensions of '" + r.name + "'";
        if (!c.get(r.type) || !c.get(r.offset)) return "truncated type or offset of '" + r.name + "'";
        const qtype *q = qtype_of(r.type);
        if (!q) return "tensor '" + r.name + "' has unknown type id " + std::to_string(r.type);
        uint64_t n = 1;
        for (uint32_t d = 0; d < r.n_dims; ++d) {
            if (r.dims[d] != 0 && n > UINT64_MAX / r.dims[d]) return "element count of '" + r.name + "' overflows";
            n *= r.dims[d];
        }
        if (n % q->block) return "tensor '" + r.name + "' is not whole blocks of its type";
        r.nbytes = n / q->block * q->bytes;
        g->by_name[r.name] = g->tensors.size();
        g->tensors.push_back(std::move(r));
    }
    g->data_offset = pad_to(c.pos, g->alignment);
    for (const tensor_rec &r : g->tensors) {
        // the blob must hold every tensor, padded to the alignment as the writer lays it out
        const uint64_t padded = pad_to(r.nbytes, g->alignment);
        if (r.offset > g->size || padded > g->size || g->data_offset > g->size - r.offset ||
            padded > g->size - g->data_offset - r.offset)
            return "data of '" + r.name + "' runs past the end of the file";
    }
    return "";
}

void fill(const moearc_x_gguf *g, const tensor_rec &r, moearc_x_gguf_tensor *out) {
    out->n_dims = r.n_dims;
    for (uint32_t d = 0; d < MAX_DIMS; ++d) out->dims[d] = d < r.n_dims ? r.dims[d] : 1;
    out->type_id = r.type;
    out->offset = g->data_offset + r.offset;
    out->nbytes = r.nbytes;
    out->data = static_cast<const uint8_t *>(g->map) + out->offset;
}

}  // namespace

extern "C" {

moearc_x_gguf *moearc_x_gguf_open(const char *path) {
    g_err.clear();
    if (!path) {
        g_err = "null path";
        return nullptr;
    }
    auto *g = new moearc_x_gguf();
    g->fd = ::open(path, O_RDONLY);
    if (g->fd < 0) {
        g_err = std::string("cannot open ") + path + ": " + std::strerror(errno);
        close_file(g);
        return nullptr;
    }
    struct stat st;
    if (fstat(g->fd, &st) != 0 || st.st_size <= 0) {
        g_err = std::string("cannot size ") + path + " (or it is empty)";
        close_file(g);
        return nullptr;
    }
    g->size = (uint64_t)st.st_size;
    g->map = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (g->map == MAP_FAILED) {
        g_err = std::string("cannot map ") + path + ": " + std::strerror(errno);
        g->map = nullptr;
        close_file(g);
        return nullptr;
    }
    const std::string why = parse(g);
    if (!why.empty()) {
        g_err = std::string(path) + ": " + why;
        close_file(g);
        return nullptr;
    }
    return g;
}

void moearc_x_gguf_close(moearc_x_gguf *g) {
    if (g) close_file(g);
}

const char *moearc_x_gguf_last_error(void) { return g_err.c_str(); }

unsigned int moearc_x_gguf_version(moearc_x_gguf *g) { return g ? g->version : 0; }
unsigned long long moearc_x_gguf_alignment(moearc_x_gguf *g) { return g ? g->alignment : 0; }
unsigned long long moearc_x_gguf_n_tensors(moearc_x_gguf *g) { return g ? g->tensors.size() : 0; }

int moearc_x_gguf_key_u64(moearc_x_gguf *g, const char *key, unsigned long long *out) {
    if (!g || !key || !out) return moearc::ERR;
    auto it = g->kv.find(key);
    if (it == g->kv.end()) return fail_arg(std::string("no key '") + key + "'");
    const kv_value &v = it->second;
    switch (v.type) {
    case V_U8: case V_U16: case V_U32: case V_U64: case V_BOOL: *out = v.u; return moearc::OK;
    case V_I8: case V_I16: case V_I32: case V_I64:
        if (v.i < 0) return fail_arg(std::string("key '") + key + "' is negative");
        *out = (unsigned long long)v.i;
        return moearc::OK;
    default: return fail_arg(std::string("key '") + key + "' is not an integer");
    }
}

int moearc_x_gguf_key_f64(moearc_x_gguf *g, const char *key, double *out) {
    if (!g || !key || !out) return moearc::ERR;
    auto it = g->kv.find(key);
    if (it == g->kv.end()) return fail_arg(std::string("no key '") + key + "'");
    if (it->second.type != V_F32 && it->second.type != V_F64)
        return fail_arg(std::string("key '") + key + "' is not a float");
    *out = it->second.f;
    return moearc::OK;
}

int moearc_x_gguf_key_str(moearc_x_gguf *g, const char *key, const char **out) {
    if (!g || !key || !out) return moearc::ERR;
    auto it = g->kv.find(key);
    if (it == g->kv.end()) return fail_arg(std::string("no key '") + key + "'");
    if (it->second.type != V_STRING) return fail_arg(std::string("key '") + key + "' is not a string");
    *out = it->second.s.c_str();
    return moearc::OK;
}

int moearc_x_gguf_find(moearc_x_gguf *g, const char *name, moearc_x_gguf_tensor *out) {
    if (!g || !name || !out) return moearc::ERR;
    auto it = g->by_name.find(name);
    if (it == g->by_name.end()) return fail_arg(std::string("no tensor '") + name + "'");
    fill(g, g->tensors[it->second], out);
    return moearc::OK;
}

int moearc_x_gguf_tensor_at(moearc_x_gguf *g, unsigned long long i, moearc_x_gguf_tensor *out, const char **name) {
    if (!g || !out) return moearc::ERR;
    if (i >= g->tensors.size()) return fail_arg("tensor index " + std::to_string(i) + " out of range");
    fill(g, g->tensors[i], out);
    if (name) *name = g->tensors[i].name.c_str();
    return moearc::OK;
}

int moearc_x_gguf_slice_last(moearc_x_gguf *g, const char *name, unsigned long long index,
                             moearc_x_gguf_tensor *out) {
    if (!g || !name || !out) return moearc::ERR;
    auto it = g->by_name.find(name);
    if (it == g->by_name.end()) return fail_arg(std::string("no tensor '") + name + "'");
    const tensor_rec &r = g->tensors[it->second];
    if (r.n_dims < 2) return fail_arg(std::string("tensor '") + name + "' has no dimension to slice");
    const uint64_t count = r.dims[r.n_dims - 1];
    if (index >= count)
        return fail_arg("slice " + std::to_string(index) + " of '" + name + "' (of " + std::to_string(count) + ")");
    const qtype *q = qtype_of(r.type);
    uint64_t inner = 1;
    for (uint32_t d = 0; d + 1 < r.n_dims; ++d) inner *= r.dims[d];
    if (inner % q->block) return fail_arg(std::string("a slice of '") + name + "' is not whole blocks");
    const uint64_t slice = inner / q->block * q->bytes;
    if (slice * count != r.nbytes) return fail_arg(std::string("slices of '") + name + "' do not tile it");
    fill(g, r, out);
    out->n_dims = r.n_dims - 1;
    out->dims[r.n_dims - 1] = 1;
    out->offset += slice * index;
    out->nbytes = slice;
    out->data = static_cast<const uint8_t *>(g->map) + out->offset;
    return moearc::OK;
}

}  // extern "C"
