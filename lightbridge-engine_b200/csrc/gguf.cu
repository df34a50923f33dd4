// gguf.cu -- GGUF reader over a split set, and the HBM-resident MoE layer
// loader.
//
// Replaces the reference's residency path for the expert tables:
//   - the GGUF v2/v3 reader, its limits and its checks
//     (bridge-gguf/src/reader.rs:184-537, errors src/error.rs:8-110);
//   - split-set discovery and the aggregate tensor directory
//     (bridge-gguf-split/src/discovery.rs:7-186, src/directory.rs:7-97);
//   - the GGML type table (bridge-core/src/ggml_type.rs:9-162) and tensor
//     descriptors (bridge-core/src/tensor.rs:21-122);
//   - the Hy3 MoE tensors of one block (bridge-model-hy3/src/schema.rs:200-258)
//     and their per-expert slabs (checked_expert_slab, schema.rs:524-580),
//     with the configuration keys of resolve_config (config.rs:57-109).
// There each routed expert is read from disk when it is routed; here a whole
// block (or an expert-parallel rank's share of it) is read once, repacked to
// the planar device layout and kept in HBM (lbk_moe_layer_load).
//
// Every failure is LBK_FORMAT_ERROR (or LBK_IO_ERROR) with the kind in the
// error detail's `bits` and the reference's message text.

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "lbk_host.h"

struct lbk_gguf {
    struct Value {
        uint32_t type = 0;
        uint32_t element_type = 0;
        uint64_t count = 0;  // arrays: elements; strings: bytes
        uint64_t u = 0;
        double f = 0.0;
        std::string s;
    };
    struct Shard {
        std::string path;
        int fd = -1;
        uint64_t size = 0;
        uint32_t version = 0;
        bool big = false;
        uint64_t alignment = 32, data_offset = 0;
        std::vector<std::pair<std::string, Value>> meta;
    };
    struct Tensor {
        std::string name;
        int32_t type;
        uint32_t n_dims;
        uint64_t dims[4];
        uint32_t shard;
        uint64_t relative, offset, bytes;
    };
    std::vector<Shard> shards;
    std::vector<Tensor> tensors;  // directory order: shard by shard
    std::unordered_map<std::string, size_t> by_name;

    // the primary shard's metadata (resolve_config reads the first shard)
    const Value* meta(const char* key) const {
        for (const auto& kv : shards[0].meta)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

namespace {

// ------------------------------------------------------------ type tables

struct GgmlInfo {
    int32_t id;
    const char* name;
    uint64_t block, size;
};

// ggml_type.rs:9-162: discriminant, name, elements per block, bytes per block
constexpr GgmlInfo kGgml[] = {
    {0, "F32", 1, 4},         {1, "F16", 1, 2},         {2, "Q4_0", 32, 18},      {3, "Q4_1", 32, 20},
    {6, "Q5_0", 32, 22},      {7, "Q5_1", 32, 24},      {8, "Q8_0", 32, 34},      {9, "Q8_1", 32, 36},
    {10, "Q2_K", 256, 84},    {11, "Q3_K", 256, 110},   {12, "Q4_K", 256, 144},   {13, "Q5_K", 256, 176},
    {14, "Q6_K", 256, 210},   {15, "Q8_K", 256, 292},   {16, "IQ2_XXS", 256, 66}, {17, "IQ2_XS", 256, 74},
    {18, "IQ3_XXS", 256, 98}, {19, "IQ1_S", 256, 50},   {20, "IQ4_NL", 32, 18},   {21, "IQ3_S", 256, 110},
    {22, "IQ2_S", 256, 82},   {23, "IQ4_XS", 256, 136}, {24, "I8", 1, 1},         {25, "I16", 1, 2},
    {26, "I32", 1, 4},        {27, "I64", 1, 8},        {28, "F64", 1, 8},        {29, "IQ1_M", 256, 56},
    {30, "BF16", 1, 2},       {34, "TQ1_0", 256, 54},   {35, "TQ2_0", 256, 66},   {39, "MXFP4", 32, 17},
    {40, "NVFP4", 64, 36},    {41, "Q1_0", 128, 18},    {42, "Q2_0", 64, 18},
};

const GgmlInfo* ggml_info(uint32_t id) {
    for (const auto& g : kGgml)
        if ((uint32_t)g.id == id) return &g;
    return nullptr;
}

// GGUF value types (bridge-gguf/src/value.rs), named as the reference prints them
const char* const kValueNames[13] = {"U8", "I8", "U16", "I16", "U32", "I32", "F32",
                                     "Bool", "String", "Array", "U64", "I64", "F64"};

// ------------------------------------------------------------ errors

struct Fail {
    int32_t status;
    int32_t kind;
    std::string msg;
    uint64_t index = 0, expected = 0, actual = 0;
};

[[noreturn]] void fail(int32_t kind, std::string msg, uint64_t expected = 0, uint64_t actual = 0) {
    throw Fail{LBK_FORMAT_ERROR, kind, std::move(msg), 0, expected, actual};
}

std::string quoted(const std::string& s) {
    std::string q = "\"";
    for (char c : s) {
        if (c == '"' || c == '\\') q += '\\';
        q += c;
    }
    return q + "\"";
}

std::string num(uint64_t v) { return std::to_string(v); }

[[noreturn]] void overflow(const char* what) {
    fail(LBK_GGUF_ARITHMETIC_OVERFLOW, std::string("arithmetic overflow while computing ") + what);
}

uint64_t add(uint64_t a, uint64_t b, const char* what) {
    uint64_t r;
    if (__builtin_add_overflow(a, b, &r)) overflow(what);
    return r;
}

uint64_t mul(uint64_t a, uint64_t b, const char* what) {
    uint64_t r;
    if (__builtin_mul_overflow(a, b, &r)) overflow(what);
    return r;
}

// RFC 3629 well-formedness: no overlong forms, surrogates or code points past
// U+10FFFF (what String::from_utf8 accepts)
bool valid_utf8(const std::string& s) {
    const auto* p = reinterpret_cast<const unsigned char*>(s.data());
    const size_t n = s.size();
    for (size_t i = 0; i < n;) {
        const unsigned c = p[i];
        size_t len;
        uint32_t cp;
        if (c < 0x80) {
            i++;
            continue;
        } else if ((c & 0xE0) == 0xC0) {
            len = 2;
            cp = c & 0x1F;
        } else if ((c & 0xF0) == 0xE0) {
            len = 3;
            cp = c & 0x0F;
        } else if ((c & 0xF8) == 0xF0) {
            len = 4;
            cp = c & 0x07;
        } else {
            return false;
        }
        if (i + len > n) return false;
        for (size_t j = 1; j < len; j++) {
            if ((p[i + j] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (p[i + j] & 0x3F);
        }
        if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) ||
            (cp >= 0xD800 && cp <= 0xDFFF) || cp > 0x10FFFF)
            return false;
        i += len;
    }
    return true;
}

// ------------------------------------------------------------ reader

// Sequential reader of one shard's header (bridge-gguf/src/reader.rs):
// metadata accounting, limits and truncation in the reference's order.
struct Reader {
    int fd;
    uint64_t size;
    const lbk_gguf_limits& lim;
    bool big = false;
    uint64_t pos = 0;
    bool account = false;
    uint64_t meta_bytes = 0, array_elems = 0;
    std::vector<uint8_t> buf = std::vector<uint8_t>(1 << 20);
    uint64_t bstart = 0, blen = 0;

    // read_exact (reader.rs:472-491): charge the metadata budget, then read
    // or report truncation
    void need(uint64_t n, const char* ctx) {
        if (account) {
            uint64_t next;
            if (__builtin_add_overflow(meta_bytes, n, &next)) overflow("metadata bytes");
            if (next > lim.max_metadata_bytes)
                fail(LBK_GGUF_LIMIT_EXCEEDED,
                     "metadata bytes count " + num(next) + " exceeds configured limit " + num(lim.max_metadata_bytes),
                     lim.max_metadata_bytes, next);
            meta_bytes = next;
        }
        if (pos > size || n > size - pos) fail(LBK_GGUF_TRUNCATED, std::string("GGUF is truncated while reading ") + ctx);
    }
    void copy(void* dst, uint64_t n) {
        auto* d = static_cast<uint8_t*>(dst);
        while (n > 0) {
            if (pos < bstart || pos >= bstart + blen) {
                const ssize_t r = pread(fd, buf.data(), buf.size(), (off_t)pos);
                if (r <= 0) throw Fail{LBK_IO_ERROR, LBK_GGUF_IO, "I/O error while inspecting GGUF: short read"};
                bstart = pos;
                blen = (uint64_t)r;
            }
            const uint64_t take = std::min(n, bstart + blen - pos);
            std::memcpy(d, buf.data() + (pos - bstart), take);
            d += take;
            pos += take;
            n -= take;
        }
    }
    void read(void* dst, uint64_t n, const char* ctx) {
        need(n, ctx);
        copy(dst, n);
    }
    template <class T>
    T scalar(const char* ctx) {
        T v;
        read(&v, sizeof(T), ctx);
        if constexpr (sizeof(T) > 1) {
            if (big) {
                auto* b = reinterpret_cast<uint8_t*>(&v);
                for (size_t i = 0; i < sizeof(T) / 2; i++) std::swap(b[i], b[sizeof(T) - 1 - i]);
            }
        }
        return v;
    }
    // read_string (reader.rs:426-445)
    std::string str(const char* ctx) {
        const uint64_t n = scalar<uint64_t>("string length");
        if (n > lim.max_string_bytes)
            fail(LBK_GGUF_LIMIT_EXCEEDED,
                 "string bytes count " + num(n) + " exceeds configured limit " + num(lim.max_string_bytes),
                 lim.max_string_bytes, n);
        need(n, ctx);
        std::string s(n, '\0');
        if (n) copy(&s[0], n);
        if (!valid_utf8(s)) fail(LBK_GGUF_INVALID_UTF8, std::string("invalid UTF-8 in ") + ctx);
        return s;
    }
};

uint32_t value_type(uint32_t t) {
    if (t > 12) fail(LBK_GGUF_UNKNOWN_VALUE_TYPE, "unknown GGUF metadata value type " + num(t), 0, t);
    return t;
}

// check_array_budget (reader.rs:376-424): aggregate elements, then the
// minimum encoding against the remaining metadata budget
void array_budget(Reader& r, uint32_t et, uint64_t count) {
    const uint64_t agg = add(r.array_elems, count, "aggregate array elements");
    if (agg > r.lim.max_array_elements)
        fail(LBK_GGUF_LIMIT_EXCEEDED,
             "array elements count " + num(agg) + " exceeds configured limit " + num(r.lim.max_array_elements),
             r.lim.max_array_elements, agg);
    const uint64_t min_bytes = et == 0 || et == 1 || et == 7 ? 1 : et == 2 || et == 3 ? 2 : et <= 6 ? 4 : 8;
    const uint64_t min_payload = mul(count, min_bytes, "minimum encoded array bytes");
    const uint64_t min_meta = add(r.meta_bytes, min_payload, "metadata bytes");
    if (min_meta > r.lim.max_metadata_bytes)
        fail(LBK_GGUF_LIMIT_EXCEEDED,
             "metadata bytes count " + num(min_meta) + " exceeds configured limit " + num(r.lim.max_metadata_bytes),
             r.lim.max_metadata_bytes, min_meta);
    r.array_elems = agg;
}

// read_value (reader.rs:342-374); array elements are checked and skipped
void read_value(Reader& r, uint32_t type, lbk_gguf::Value& v, bool keep) {
    v.type = type;
    switch (type) {
        case 0: v.u = r.scalar<uint8_t>("u8 metadata value"); break;
        case 1: v.u = (uint64_t)(int64_t)(int8_t)r.scalar<uint8_t>("i8 metadata value"); break;
        case 2: v.u = r.scalar<uint16_t>("u16 metadata value"); break;
        case 3: v.u = (uint64_t)(int64_t)(int16_t)r.scalar<uint16_t>("i16 metadata value"); break;
        case 4: v.u = r.scalar<uint32_t>("u32 metadata value"); break;
        case 5: v.u = (uint64_t)(int64_t)(int32_t)r.scalar<uint32_t>("i32 metadata value"); break;
        case 6: {
            const uint32_t b = r.scalar<uint32_t>("f32 metadata value");
            float f;
            std::memcpy(&f, &b, 4);
            v.f = f;
            v.u = b;
            break;
        }
        case 7: {
            const uint8_t b = r.scalar<uint8_t>("boolean metadata value");
            if (b > 1) fail(LBK_GGUF_INVALID_BOOLEAN, "invalid GGUF boolean byte " + num(b), 0, b);
            v.u = b;
            break;
        }
        case 8: {
            std::string s = r.str("string metadata value");
            v.count = s.size();
            if (keep) v.s = std::move(s);
            break;
        }
        case 9: {
            const uint32_t et = value_type(r.scalar<uint32_t>("array element type"));
            if (et == 9) fail(LBK_GGUF_NESTED_ARRAY, "GGUF arrays may not contain arrays");
            const uint64_t count = r.scalar<uint64_t>("array element count");
            array_budget(r, et, count);
            v.element_type = et;
            v.count = count;
            lbk_gguf::Value e;
            for (uint64_t i = 0; i < count; i++) read_value(r, et, e, false);
            break;
        }
        case 10: v.u = r.scalar<uint64_t>("u64 metadata value"); break;
        case 11: v.u = r.scalar<uint64_t>("i64 metadata value"); break;
        case 12: {
            const uint64_t b = r.scalar<uint64_t>("f64 metadata value");
            std::memcpy(&v.f, &b, 8);
            v.u = b;
            break;
        }
    }
}

// GgufReader::read (reader.rs:184-340) for one shard.
void parse_shard(lbk_gguf::Shard& sh, uint32_t shard, const lbk_gguf_limits& lim, std::vector<lbk_gguf::Tensor>& out) {
    if (lim.max_dimensions > 4)
        fail(LBK_GGUF_INVALID_DIMENSION_LIMIT,
             "configured dimension limit " + num(lim.max_dimensions) + " exceeds GGML's maximum of four", 4,
             lim.max_dimensions);
    Reader r{sh.fd, sh.size, lim};
    uint8_t magic[4];
    r.read(magic, 4, "magic");
    if (std::memcmp(magic, "GGUF", 4) == 0) {
        r.big = false;
    } else if (std::memcmp(magic, "FUGG", 4) == 0) {
        r.big = true;
    } else {
        fail(LBK_GGUF_BAD_MAGIC, "bad GGUF magic bytes [" + num(magic[0]) + ", " + num(magic[1]) + ", " + num(magic[2]) +
                                     ", " + num(magic[3]) + "]");
    }
    sh.big = r.big;
    sh.version = r.scalar<uint32_t>("version");
    if (sh.version < 2 || sh.version > 3)
        fail(LBK_GGUF_UNSUPPORTED_VERSION, "unsupported GGUF version " + num(sh.version), 3, sh.version);
    const uint64_t n_tensors = r.scalar<uint64_t>("tensor count");
    const uint64_t n_kv = r.scalar<uint64_t>("metadata count");
    if (n_tensors > lim.max_tensors)
        fail(LBK_GGUF_LIMIT_EXCEEDED, "tensors count " + num(n_tensors) + " exceeds configured limit " + num(lim.max_tensors),
             lim.max_tensors, n_tensors);
    if (n_kv > lim.max_metadata_entries)
        fail(LBK_GGUF_LIMIT_EXCEEDED,
             "metadata entries count " + num(n_kv) + " exceeds configured limit " + num(lim.max_metadata_entries),
             lim.max_metadata_entries, n_kv);
    std::unordered_set<std::string> keys;
    r.account = true;
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key = r.str("metadata key");
        const uint32_t type = value_type(r.scalar<uint32_t>("metadata value type"));
        lbk_gguf::Value v;
        read_value(r, type, v, true);
        if (!keys.insert(key).second) fail(LBK_GGUF_DUPLICATE_METADATA_KEY, "duplicate GGUF metadata key " + quoted(key));
        sh.meta.emplace_back(std::move(key), std::move(v));
    }
    r.account = false;
    sh.alignment = 32;
    for (const auto& kv : sh.meta) {
        if (kv.first != "general.alignment") continue;
        if (kv.second.type != 4)
            fail(LBK_GGUF_ALIGNMENT_WRONG_TYPE,
                 std::string("general.alignment must have type U32, got ") + kValueNames[kv.second.type]);
        const uint64_t a = kv.second.u;
        if (a == 0 || (a & (a - 1)))
            fail(LBK_GGUF_INVALID_ALIGNMENT, "general.alignment must be a positive u32 power of two, got " + num(a), 0, a);
        sh.alignment = a;
    }
    std::vector<lbk_gguf::Tensor> ts;
    for (uint64_t i = 0; i < n_tensors; i++) {
        lbk_gguf::Tensor t{};
        r.account = true;
        t.name = r.str("tensor name");
        r.account = false;
        t.n_dims = r.scalar<uint32_t>("tensor dimension count");
        if (t.n_dims < 1 || t.n_dims > 4)
            fail(LBK_GGUF_INVALID_DIMENSION_COUNT,
                 "tensor dimension count " + num(t.n_dims) + " is outside GGML's supported 1..=4 dimensions", 4, t.n_dims);
        if (t.n_dims > lim.max_dimensions)
            fail(LBK_GGUF_LIMIT_EXCEEDED,
                 "dimensions count " + num(t.n_dims) + " exceeds configured limit " + num(lim.max_dimensions),
                 lim.max_dimensions, t.n_dims);
        for (int d = 0; d < 4; d++) t.dims[d] = 1;
        for (uint32_t d = 0; d < t.n_dims; d++) t.dims[d] = r.scalar<uint64_t>("tensor dimension");
        const uint32_t ty = r.scalar<uint32_t>("GGML type");
        t.relative = r.scalar<uint64_t>("tensor payload offset");
        // TensorDesc::new (tensor.rs:21-42) and compute_strides (:100-122)
        const GgmlInfo* gi = ggml_info(ty);
        if (gi == nullptr) fail(LBK_GGUF_UNKNOWN_GGML_TYPE, "unknown ggml type discriminant " + num(ty), 0, ty);
        t.type = (int32_t)ty;
        for (uint32_t d = 0; d < t.n_dims; d++)
            if (t.dims[d] == 0) fail(LBK_GGUF_ZERO_TENSOR_DIMENSION, "tensor dimension " + num(d) + " is zero", 0, d);
        if (t.dims[0] % gi->block != 0)
            fail(LBK_GGUF_NOT_BLOCK_ALIGNED,
                 std::string(gi->name) + " requires a leading dimension divisible by " + num(gi->block) + ", got " +
                     num(t.dims[0]),
                 gi->block, t.dims[0]);
        const uint64_t row = mul(t.dims[0] / gi->block, gi->size, "GGML row size");
        uint64_t stride = row;
        for (uint32_t d = 2; d < t.n_dims; d++) stride = mul(stride, t.dims[d - 1], "GGML tensor stride");
        t.bytes = t.n_dims == 1 ? row : mul(stride, t.dims[t.n_dims - 1], "tensor encoded byte length");
        t.shard = shard;
        ts.push_back(std::move(t));
    }
    const uint64_t dir_end = r.pos;
    uint64_t data;
    if (__builtin_add_overflow(dir_end, sh.alignment - 1, &data)) overflow("GGUF data offset");
    data &= ~(sh.alignment - 1);
    if (data > sh.size)
        fail(LBK_GGUF_DATA_OFFSET_BEYOND_FILE,
             "GGUF data offset " + num(data) + " exceeds physical file length " + num(sh.size), sh.size, data);
    sh.data_offset = data;
    uint64_t extent = 0;
    for (auto& t : ts) {
        if (t.relative != extent)
            fail(LBK_GGUF_TENSOR_OFFSET_MISMATCH,
                 "tensor " + quoted(t.name) + " has relative payload offset " + num(t.relative) + ", expected " +
                     num(extent) + " for " + num(sh.alignment) + "-byte alignment",
                 extent, t.relative);
        uint64_t padded;
        if (__builtin_add_overflow(t.bytes, sh.alignment - 1, &padded))
            fail(LBK_GGUF_TENSOR_PADDING_OVERFLOW, "tensor " + quoted(t.name) + " encoded byte length " + num(t.bytes) +
                                                       " overflows " + num(sh.alignment) + "-byte padding");
        padded &= ~(sh.alignment - 1);
        if (__builtin_add_overflow(extent, padded, &extent))
            fail(LBK_GGUF_TENSOR_EXTENT_OVERFLOW, "tensor " + quoted(t.name) + " padded extent overflows");
        // checked_absolute_range (tensor.rs:85-96)
        const uint64_t start = add(data, t.relative, "tensor absolute offset");
        const uint64_t end = add(start, t.bytes, "tensor absolute end offset");
        if (end > sh.size)
            fail(LBK_GGUF_TENSOR_OUT_OF_BOUNDS,
                 "tensor byte range " + num(start) + ".." + num(end) + " exceeds file length " + num(sh.size), sh.size, end);
        t.offset = start;
    }
    uint64_t required;
    if (__builtin_add_overflow(data, extent, &required))
        fail(LBK_GGUF_TENSOR_DATA_END_OVERFLOW, "GGUF tensor data end overflows");
    if (required > sh.size)
        fail(LBK_GGUF_TENSOR_DATA_SECTION_TRUNCATED,
             "GGUF tensor data section requires padded range " + num(data) + ".." + num(required) +
                 ", but physical file length is " + num(sh.size),
             required, sh.size);
    for (auto& t : ts) out.push_back(std::move(t));
}

const lbk_gguf::Value* shard_meta(const lbk_gguf::Shard& sh, const char* key) {
    for (const auto& kv : sh.meta)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

// split.no / split.count (discovery.rs:64-131): U16; required on numbered
// shards, checked when present on a single file
void split_metadata(const lbk_gguf::Shard& sh, uint32_t ordinal, uint32_t count, bool required) {
    const char* keys[2] = {"split.no", "split.count"};
    const uint32_t want[2] = {ordinal, count};
    const lbk_gguf::Value* v[2];
    for (int i = 0; i < 2; i++) {
        v[i] = shard_meta(sh, keys[i]);
        if (v[i] == nullptr) {
            if (required)
                fail(LBK_GGUF_MISSING_SPLIT_METADATA,
                     "numbered GGUF shard " + quoted(sh.path) + " is missing required metadata " + quoted(keys[i]));
            continue;
        }
        if (v[i]->type != 2)
            fail(LBK_GGUF_METADATA_WRONG_TYPE, "GGUF metadata key " + quoted(keys[i]) + " has type " +
                                                   kValueNames[v[i]->type] + ", expected U16");
    }
    if (required && count == 1)
        fail(LBK_GGUF_NUMBERED_SINGLE_SHARD, "numbered GGUF shard " + quoted(sh.path) + " declares only one shard");
    for (int i = 0; i < 2; i++)
        if (v[i] != nullptr && v[i]->u != want[i])
            fail(LBK_GGUF_SPLIT_METADATA_DISAGREEMENT,
                 "numbered GGUF shard " + quoted(sh.path) + " metadata " + quoted(keys[i]) + " does not match its filename",
                 want[i], v[i]->u);
}

bool is_file(const std::string& p) {
    struct stat st {};
    return stat(p.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

std::string canonical(const std::string& p) {
    char buf[PATH_MAX];
    if (realpath(p.c_str(), buf) == nullptr)
        throw Fail{LBK_IO_ERROR, LBK_GGUF_IO, "I/O error while inspecting GGUF: cannot resolve " + p};
    return buf;
}

std::string parent_of(const std::string& p) {
    const size_t s = p.rfind('/');
    if (s == std::string::npos) return ".";
    return s == 0 ? "/" : p.substr(0, s);
}

// NumberedName::parse (discovery.rs:139-176): <prefix>-NNNNN-of-MMMMM.gguf
bool numbered_name(const std::string& file, std::string* prefix, uint32_t* total) {
    const std::string ext = ".gguf";
    if (file.size() < ext.size() || file.compare(file.size() - ext.size(), ext.size(), ext) != 0) return false;
    const std::string stem = file.substr(0, file.size() - ext.size());
    const size_t of = stem.rfind("-of-");
    if (of == std::string::npos) return false;
    const std::string before = stem.substr(0, of), total_text = stem.substr(of + 4);
    const size_t dash = before.rfind('-');
    if (dash == std::string::npos) return false;
    const std::string ordinal_text = before.substr(dash + 1);
    auto digits = [](const std::string& s) {
        if (s.size() != 5) return false;
        for (char c : s)
            if (c < '0' || c > '9') return false;
        return true;
    };
    if (!digits(ordinal_text) || !digits(total_text)) return false;
    const uint32_t ordinal = (uint32_t)std::stoul(ordinal_text), t = (uint32_t)std::stoul(total_text);
    if (ordinal == 0 || t == 0 || ordinal > t || t > 65535)
        fail(LBK_GGUF_INVALID_NUMBERED_FILENAME, "invalid numbered GGUF filename " + quoted(file));
    *prefix = before.substr(0, dash);
    *total = t;
    return true;
}

void add_shard(lbk_gguf* g, const std::string& path) {
    lbk_gguf::Shard sh;
    sh.path = path;
    sh.fd = open(path.c_str(), O_RDONLY);
    struct stat st {};
    if (sh.fd < 0 || fstat(sh.fd, &st) != 0) {
        if (sh.fd >= 0) close(sh.fd);
        throw Fail{LBK_IO_ERROR, LBK_GGUF_IO, "I/O error while inspecting GGUF: cannot open " + path};
    }
    sh.size = (uint64_t)st.st_size;
    g->shards.push_back(std::move(sh));
}

// open_set (bridge-gguf-split/src/lib.rs:155-159): discover and parse every
// shard, then build the aggregate directory.
void open_set(lbk_gguf* g, const std::string& entry, const lbk_gguf_limits& lim) {
    if (!is_file(entry)) fail(LBK_GGUF_NOT_A_FILE, "input path is not a regular file: " + quoted(entry));
    const std::string parent = canonical(parent_of(entry));
    const std::string path = canonical(entry);
    if (parent_of(path) != parent)
        fail(LBK_GGUF_SHARD_ESCAPES_PARENT, "canonical GGUF shard escapes its input parent directory: " + quoted(path));
    std::string prefix;
    uint32_t total = 1;
    const std::string file = path.substr(path.rfind('/') + 1);
    std::vector<lbk_gguf::Tensor> all;
    if (numbered_name(file, &prefix, &total)) {
        for (uint32_t i = 1; i <= total; i++) {
            char name[40];
            std::snprintf(name, sizeof(name), "-%05u-of-%05u.gguf", i, total);
            const std::string expected = parent + "/" + prefix + name;
            if (!is_file(expected))
                fail(LBK_GGUF_MISSING_SHARD, "expected GGUF shard is missing or is not a regular file: " + quoted(expected));
            const std::string p = canonical(expected);
            if (parent_of(p) != parent)
                fail(LBK_GGUF_SHARD_ESCAPES_PARENT, "canonical GGUF shard escapes its input parent directory: " + quoted(p));
            add_shard(g, p);
            parse_shard(g->shards.back(), i - 1, lim, all);
            split_metadata(g->shards.back(), i - 1, total, true);
        }
    } else {
        add_shard(g, path);
        parse_shard(g->shards.back(), 0, lim, all);
        split_metadata(g->shards.back(), 0, 1, false);
    }
    // directory::build (directory.rs:7-97)
    const lbk_gguf::Shard& primary = g->shards[0];
    for (size_t i = 1; i < g->shards.size(); i++) {
        const lbk_gguf::Shard& s = g->shards[i];
        if (s.version != primary.version)
            fail(LBK_GGUF_HETEROGENEOUS_VERSION, "GGUF shard " + quoted(s.path) + " has version " + num(s.version) +
                                                     ", expected common version " + num(primary.version),
                 primary.version, s.version);
        if (s.big != primary.big)
            fail(LBK_GGUF_HETEROGENEOUS_ENDIANNESS, "GGUF shard " + quoted(s.path) + " has endianness " +
                                                        (s.big ? "Big" : "Little") + ", expected common endianness " +
                                                        (primary.big ? "Big" : "Little"));
        if (s.alignment != primary.alignment)
            fail(LBK_GGUF_HETEROGENEOUS_ALIGNMENT, "GGUF shard " + quoted(s.path) + " has alignment " + num(s.alignment) +
                                                       ", expected common alignment " + num(primary.alignment),
                 primary.alignment, s.alignment);
    }
    bool declared = false;
    int64_t declared_count = 0;
    size_t t_index = 0;
    for (uint32_t si = 0; si < g->shards.size(); si++) {
        const lbk_gguf::Shard& s = g->shards[si];
        if (const lbk_gguf::Value* v = shard_meta(s, "split.tensors.count")) {
            if (v->type != 5)
                fail(LBK_GGUF_METADATA_WRONG_TYPE, std::string("GGUF metadata key \"split.tensors.count\" has type ") +
                                                       kValueNames[v->type] + ", expected I32");
            const int64_t c = (int64_t)v->u;
            if (c < 0)
                fail(LBK_GGUF_NEGATIVE_AGGREGATE_TENSOR_COUNT,
                     "aggregate split.tensors.count is negative in " + quoted(s.path));
            if (declared && c != declared_count)
                fail(LBK_GGUF_AGGREGATE_TENSOR_COUNT_DISAGREEMENT, "split.tensors.count disagrees between GGUF shards");
            declared = true;
            declared_count = c;
        }
        for (; t_index < all.size() && all[t_index].shard == si; t_index++) {
            lbk_gguf::Tensor& t = all[t_index];
            if (t.relative % s.alignment != 0)
                fail(LBK_GGUF_UNALIGNED_TENSOR_OFFSET, "tensor " + quoted(t.name) + " in " + quoted(s.path) +
                                                           " has offset " + num(t.relative) + " not aligned to " +
                                                           num(s.alignment));
            if (g->by_name.count(t.name))
                fail(LBK_GGUF_DUPLICATE_TENSOR_NAME, "duplicate tensor name " + quoted(t.name) + " across GGUF shards");
            g->by_name.emplace(t.name, g->tensors.size());
            g->tensors.push_back(t);
        }
    }
    if (declared && (uint64_t)declared_count != g->tensors.size())
        fail(LBK_GGUF_AGGREGATE_TENSOR_DIRECTORY_DISAGREEMENT,
             "split.tensors.count does not match the aggregate tensor directory", (uint64_t)declared_count,
             g->tensors.size());
}

int32_t report(const Fail& f) {
    return lbk::host_fail(f.status, f.msg.c_str(), f.index, f.expected, f.actual, (uint32_t)f.kind);
}

int32_t missing_key(const char* key) {
    return report(Fail{LBK_FORMAT_ERROR, LBK_GGUF_METADATA_MISSING, std::string("missing GGUF metadata key ") + quoted(key)});
}

}  // namespace

// ===================================================================== ABI

LBK_API void lbk_gguf_default_limits(lbk_gguf_limits* out) {
    if (out == nullptr) return;
    // ReaderLimits::default (reader.rs:31-42)
    out->max_dimensions = 4;
    out->max_string_bytes = 1024 * 1024;
    out->max_array_elements = 1000000;
    out->max_tensors = 4000000;
    out->max_metadata_entries = 1000000;
    out->max_metadata_bytes = 64ull * 1024 * 1024;
}

LBK_API int32_t lbk_gguf_open(const char* entry, const lbk_gguf_limits* limits, lbk_gguf** out) {
    if (entry == nullptr || out == nullptr) return lbk::host_fail(LBK_INVALID_PARAMETER, "null pointer", 0, 0, 0, 0);
    *out = nullptr;
    lbk_gguf_limits lim;
    if (limits) lim = *limits;
    else lbk_gguf_default_limits(&lim);
    auto* g = new lbk_gguf{};
    try {
        open_set(g, entry, lim);
    } catch (const Fail& f) {
        lbk_gguf_close(g);
        return report(f);
    } catch (const std::exception& e) {
        lbk_gguf_close(g);
        return report(Fail{LBK_IO_ERROR, LBK_GGUF_IO, std::string("I/O error while inspecting GGUF: ") + e.what()});
    }
    *out = g;
    return lbk::host_ok();
}

LBK_API int32_t lbk_gguf_close(lbk_gguf* g) {
    if (g == nullptr) return LBK_OK;
    for (auto& s : g->shards)
        if (s.fd >= 0) close(s.fd);
    delete g;
    return LBK_OK;
}

LBK_API int32_t lbk_gguf_info(const lbk_gguf* g, lbk_gguf_file_info* out) {
    if (g == nullptr || out == nullptr) return lbk::host_fail(LBK_INVALID_PARAMETER, "null pointer", 0, 0, 0, 0);
    const lbk_gguf::Shard& p = g->shards[0];
    out->version = p.version;
    out->big_endian = p.big ? 1 : 0;
    out->alignment = p.alignment;
    out->shard_count = g->shards.size();
    out->tensor_count = g->tensors.size();
    out->metadata_count = p.meta.size();
    out->data_offset = p.data_offset;
    out->file_len = p.size;
    return lbk::host_ok();
}

LBK_API int32_t lbk_gguf_tensor_at(const lbk_gguf* g, uint64_t index, lbk_gguf_tensor* out, char* name,
                                   uint64_t name_cap) {
    if (g == nullptr || out == nullptr) return lbk::host_fail(LBK_INVALID_PARAMETER, "null pointer", 0, 0, 0, 0);
    if (index >= g->tensors.size())
        return lbk::host_fail(LBK_INVALID_PARAMETER, "tensor index", index, g->tensors.size(), index, 0);
    const lbk_gguf::Tensor& t = g->tensors[index];
    out->type = t.type;
    out->n_dims = t.n_dims;
    for (int d = 0; d < 4; d++) out->dims[d] = t.dims[d];
    out->shard = t.shard;
    out->offset = t.offset;
    out->relative_offset = t.relative;
    out->bytes = t.bytes;
    out->name_len = t.name.size();
    if (name != nullptr && name_cap > 0) {
        const size_t n = std::min<size_t>(t.name.size(), name_cap - 1);
        std::memcpy(name, t.name.data(), n);
        name[n] = '\0';
    }
    return lbk::host_ok();
}

LBK_API int32_t lbk_gguf_find_tensor(const lbk_gguf* g, const char* name, uint64_t* index) {
    if (g == nullptr || name == nullptr || index == nullptr)
        return lbk::host_fail(LBK_INVALID_PARAMETER, "null pointer", 0, 0, 0, 0);
    auto it = g->by_name.find(name);
    if (it == g->by_name.end())
        return report(Fail{LBK_FORMAT_ERROR, LBK_GGUF_MISSING_TENSOR, std::string("missing tensor ") + quoted(name)});
    *index = it->second;
    return lbk::host_ok();
}

LBK_API int32_t lbk_gguf_metadata(const lbk_gguf* g, const char* key, lbk_gguf_value* out) {
    if (g == nullptr || key == nullptr || out == nullptr)
        return lbk::host_fail(LBK_INVALID_PARAMETER, "null pointer", 0, 0, 0, 0);
    const lbk_gguf::Value* v = g->meta(key);
    if (v == nullptr) return missing_key(key);
    out->type = v->type;
    out->element_type = v->element_type;
    out->count = v->count;
    out->u = v->u;
    out->f = v->f;
    return lbk::host_ok();
}

LBK_API int32_t lbk_gguf_metadata_string(const lbk_gguf* g, const char* key, char* buf, uint64_t cap, uint64_t* len) {
    if (g == nullptr || key == nullptr) return lbk::host_fail(LBK_INVALID_PARAMETER, "null pointer", 0, 0, 0, 0);
    const lbk_gguf::Value* v = g->meta(key);
    if (v == nullptr) return missing_key(key);
    if (v->type != 8)
        return report(Fail{LBK_FORMAT_ERROR, LBK_GGUF_METADATA_WRONG_TYPE,
                           "GGUF metadata key " + quoted(key) + " has type " + kValueNames[v->type] + ", expected String"});
    if (len) *len = v->s.size();
    if (buf != nullptr && cap > 0) {
        const size_t n = std::min<size_t>(v->s.size(), cap - 1);
        std::memcpy(buf, v->s.data(), n);
        buf[n] = '\0';
    }
    return lbk::host_ok();
}

// ------------------------------------------------------------ layer loader

namespace {

const lbk_gguf::Value& typed(const lbk_gguf* g, const char* key, uint32_t type) {
    const lbk_gguf::Value* v = g->meta(key);
    if (v == nullptr) fail(LBK_GGUF_METADATA_MISSING, std::string("missing GGUF metadata key ") + quoted(key));
    if (v->type != type)
        fail(LBK_GGUF_METADATA_WRONG_TYPE, "GGUF metadata key " + quoted(key) + " has type " + kValueNames[v->type] +
                                               ", expected " + kValueNames[type]);
    return *v;
}

struct Pinned {
    uint8_t* p = nullptr;
    ~Pinned() {
        if (p) cudaFreeHost(p);
    }
};
struct DevMem {
    uint8_t* p = nullptr;
    ~DevMem() {
        if (p) cudaFree(p);
    }
};

struct LbkStatus {
    int32_t s;  // the failing lbk_* call has filled the error detail
};

void cuda_ok(cudaError_t e, const char* where) {
    if (e != cudaSuccess) throw Fail{LBK_CUDA_ERROR, 0, std::string(where) + ": " + cudaGetErrorString(e)};
}

void lbk_ok(int32_t s) {
    if (s != LBK_OK) throw LbkStatus{s};
}

constexpr uint64_t kChunk = 32ull << 20;

// Reads [offset, offset + bytes) of a shard into device memory through one
// pinned buffer of kChunk bytes.
void read_to_device(const lbk_gguf* g, uint32_t shard, uint64_t offset, uint64_t bytes, uint8_t* dev, uint8_t* pinned,
                    cudaStream_t st) {
    while (bytes > 0) {
        const uint64_t n = std::min(bytes, kChunk);
        for (uint64_t done = 0; done < n;) {
            const ssize_t r = pread(g->shards[shard].fd, pinned + done, n - done, (off_t)(offset + done));
            if (r <= 0) throw Fail{LBK_IO_ERROR, LBK_GGUF_IO, "read error in " + g->shards[shard].path};
            done += (uint64_t)r;
        }
        cuda_ok(cudaMemcpyAsync(dev, pinned, n, cudaMemcpyHostToDevice, st), "upload");
        cuda_ok(cudaStreamSynchronize(st), "upload");  // the pinned buffer is reused
        dev += n;
        offset += n;
        bytes -= n;
    }
}

uint64_t up256(uint64_t v) { return (v + 255) & ~(uint64_t)255; }

bool computed_type(int32_t t) {
    return t == LBK_TYPE_IQ2_S || t == LBK_TYPE_IQ3_S || t == LBK_TYPE_Q4_K || t == LBK_TYPE_Q5_K;
}

int32_t load_layer(lbk_context* ctx, const lbk_gguf* g, uint32_t block, uint64_t first, uint64_t count, void* stream,
                   lbk_moe_layer** out) {
    // resolve_config (config.rs:57-109): the keys an MoE block needs, with
    // the reference's types
    const lbk_gguf::Value& arch = typed(g, "general.architecture", 8);
    if (arch.s != "hy_v3")
        fail(LBK_GGUF_METADATA_VALUE, "metadata \"general.architecture\": expected \"hy_v3\", found " + quoted(arch.s));
    const uint64_t blocks = typed(g, "hy_v3.block_count", 4).u;
    const uint64_t H = typed(g, "hy_v3.embedding_length", 4).u;
    const uint64_t F = typed(g, "hy_v3.expert_feed_forward_length", 4).u;
    const uint64_t Fs = typed(g, "hy_v3.expert_shared_feed_forward_length", 4).u;
    const uint64_t E = typed(g, "hy_v3.expert_count", 4).u;
    const uint64_t k = typed(g, "hy_v3.expert_used_count", 4).u;
    const float scale = (float)typed(g, "hy_v3.expert_weights_scale", 6).f;
    if (!std::isfinite(scale)) fail(LBK_GGUF_NON_FINITE_METADATA, "metadata \"hy_v3.expert_weights_scale\" is not finite");
    if (block >= blocks) fail(LBK_GGUF_BLOCK_OUT_OF_RANGE, "block " + num(block) + " of " + num(blocks), blocks, block);
    if (E == 0) fail(LBK_GGUF_EXPERT_RANGE, "hy_v3.expert_count is 0", 1, 0);
    if (count == 0 && first < E) count = E - first;
    if (first >= E || count > E - first)
        fail(LBK_GGUF_EXPERT_RANGE, "experts [" + num(first) + ", " + num(first + count) + ") of " + num(E), E,
             first + count);
    if (g->shards[0].big) fail(LBK_GGUF_BIG_ENDIAN_PAYLOAD, "big-endian tensor payloads are not loaded to the device");
    if (Fs != F)
        fail(LBK_GGUF_SHARED_WIDTH, "shared expert width " + num(Fs) + " differs from the routed width " + num(F), F, Fs);

    // schema.rs:200-258 for one MoE block, in the schema's order
    const std::string p = "blk." + std::to_string(block) + ".";
    struct Want {
        const char* name;
        uint32_t n_dims;
        uint64_t d[3];
    };
    const Want wants[8] = {{"exp_probs_b", 1, {E, 1, 1}},          {"ffn_gate_inp.weight", 2, {H, E, 1}},
                           {"ffn_gate_exps.weight", 3, {H, F, E}}, {"ffn_up_exps.weight", 3, {H, F, E}},
                           {"ffn_down_exps.weight", 3, {F, H, E}}, {"ffn_gate_shexp.weight", 2, {H, Fs, 1}},
                           {"ffn_up_shexp.weight", 2, {H, Fs, 1}}, {"ffn_down_shexp.weight", 2, {Fs, H, 1}}};
    const lbk_gguf::Tensor* ts[8];
    for (int i = 0; i < 8; i++) {
        const std::string name = p + wants[i].name;
        auto it = g->by_name.find(name);
        if (it == g->by_name.end()) fail(LBK_GGUF_MISSING_TENSOR, "missing tensor " + quoted(name));
        ts[i] = &g->tensors[it->second];
        bool shape = ts[i]->n_dims == wants[i].n_dims;
        for (uint32_t d = 0; shape && d < wants[i].n_dims; d++) shape = ts[i]->dims[d] == wants[i].d[d];
        if (!shape) fail(LBK_GGUF_TENSOR_SHAPE, "tensor " + quoted(name) + " shape");
        const bool type_ok = i < 2 ? ts[i]->type == LBK_TYPE_F32 : computed_type(ts[i]->type);
        if (!type_ok)
            fail(LBK_GGUF_TENSOR_TYPE, "tensor " + quoted(name) + " type " + ggml_info(ts[i]->type)->name, 0, ts[i]->type);
    }
    // checked_expert_slab (schema.rs:524-580): expert e is bytes
    // [e * slab, (e + 1) * slab) of the stacked payload
    uint64_t slab[3];
    for (int i = 0; i < 3; i++) {
        const lbk_gguf::Tensor& t = *ts[2 + i];
        if (t.bytes % E != 0)
            fail(LBK_GGUF_EXPERT_PAYLOAD_NOT_DIVISIBLE,
                 "tensor " + quoted(t.name) + " payload " + num(t.bytes) + " is not divisible by " + num(E) + " experts");
        slab[i] = t.bytes / E;
    }
    uint64_t pl[3], ps[3];
    lbk_ok(lbk_planar_bytes(ts[2]->type, H, F, &pl[0]));
    lbk_ok(lbk_planar_bytes(ts[3]->type, H, F, &pl[1]));
    lbk_ok(lbk_planar_bytes(ts[4]->type, F, H, &pl[2]));
    lbk_ok(lbk_planar_bytes(ts[5]->type, H, F, &ps[0]));
    lbk_ok(lbk_planar_bytes(ts[6]->type, H, F, &ps[1]));
    lbk_ok(lbk_planar_bytes(ts[7]->type, F, H, &ps[2]));

    // one device block owned by the layer: router | bias | experts | shared
    const uint64_t per_expert = up256(pl[0]) + up256(pl[1]) + up256(pl[2]);
    const uint64_t o_bias = up256(E * H * 4), o_exp = o_bias + up256(E * 4);
    const uint64_t o_shared = o_exp + count * per_expert;
    const uint64_t total = o_shared + up256(ps[0]) + up256(ps[1]) + up256(ps[2]);
    uint64_t stage_bytes = std::max(std::max(slab[0], slab[1]), slab[2]);
    for (int i = 5; i < 8; i++) stage_bytes = std::max(stage_bytes, ts[i]->bytes);

    // every check above is host-side; the device work needs the context
    if (ctx == nullptr) throw LbkStatus{lbk::host_fail(LBK_INVALID_PARAMETER, "null context", 0, 0, 0, 0)};
    lbk_ok(lbk::host_set_device(ctx));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    DevMem dev, stage;
    Pinned pinned;
    cuda_ok(cudaMalloc(&dev.p, total), "cudaMalloc layer");
    cuda_ok(cudaMalloc(&stage.p, stage_bytes), "cudaMalloc staging");
    cuda_ok(cudaMallocHost(&pinned.p, std::min(kChunk, std::max<uint64_t>(stage_bytes, E * H * 4))), "cudaMallocHost");

    read_to_device(g, ts[1]->shard, ts[1]->offset, E * H * 4, dev.p, pinned.p, st);
    read_to_device(g, ts[0]->shard, ts[0]->offset, E * 4, dev.p + o_bias, pinned.p, st);
    auto repack = [&](const lbk_gguf::Tensor& t, uint64_t in_w, uint64_t out_w, uint64_t rel, uint64_t raw,
                      uint8_t* dst, uint64_t dst_bytes) {
        read_to_device(g, t.shard, t.offset + rel, raw, stage.p, pinned.p, st);
        const lbk_matrix m{t.type, LBK_LAYOUT_GGUF, in_w, out_w, stage.p, raw};
        lbk_ok(lbk_repack(ctx, &m, dst, dst_bytes, stream));
        cuda_ok(cudaStreamSynchronize(st), "repack");  // the staging buffer is reused
        return lbk_matrix{t.type, LBK_LAYOUT_PLANAR, in_w, out_w, dst, dst_bytes};
    };
    std::vector<lbk_expert> experts(count);
    for (uint64_t i = 0; i < count; i++) {
        const uint64_t e = first + i;
        uint8_t* base = dev.p + o_exp + i * per_expert;
        experts[i].gate = repack(*ts[2], H, F, e * slab[0], slab[0], base, pl[0]);
        experts[i].up = repack(*ts[3], H, F, e * slab[1], slab[1], base + up256(pl[0]), pl[1]);
        experts[i].down = repack(*ts[4], F, H, e * slab[2], slab[2], base + up256(pl[0]) + up256(pl[1]), pl[2]);
    }
    uint8_t* sb = dev.p + o_shared;
    lbk_expert shared;
    shared.gate = repack(*ts[5], H, F, 0, ts[5]->bytes, sb, ps[0]);
    shared.up = repack(*ts[6], H, F, 0, ts[6]->bytes, sb + up256(ps[0]), ps[1]);
    shared.down = repack(*ts[7], F, H, 0, ts[7]->bytes, sb + up256(ps[0]) + up256(ps[1]), ps[2]);

    lbk_moe_weights w{};
    w.experts = experts.data();
    w.expert_count = count;
    w.shared = shared;
    w.router = lbk_matrix{LBK_TYPE_F32, LBK_LAYOUT_GGUF, H, E, dev.p, E * H * 4};
    w.selection_bias = reinterpret_cast<const float*>(dev.p + o_bias);
    w.top_k = (uint32_t)k;
    w.weight_scale = scale;
    lbk_ok(lbk::layer_create_owned(ctx, &w, E, first, stream, dev.p, out));
    dev.p = nullptr;  // owned by the layer now
    return lbk::host_ok();
}

}  // namespace

LBK_API int32_t lbk_moe_layer_load(lbk_context* ctx, const lbk_gguf* g, uint32_t block, uint64_t first_expert,
                                   uint64_t expert_count, void* stream, lbk_moe_layer** out) {
    if (g == nullptr || out == nullptr) return lbk::host_fail(LBK_INVALID_PARAMETER, "null pointer", 0, 0, 0, 0);
    *out = nullptr;
    try {
        return load_layer(ctx, g, block, first_expert, expert_count, stream, out);
    } catch (const Fail& f) {
        return report(f);
    } catch (const LbkStatus& s) {
        return s.s;
    } catch (const std::exception& e) {
        return report(Fail{LBK_IO_ERROR, LBK_GGUF_IO, e.what()});
    }
}
