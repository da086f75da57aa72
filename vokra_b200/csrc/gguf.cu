// gguf.cu — GGUF v3 reader for the model loader (host C++).
//
// Follows GgufFile::parse (crates/vokra-core/src/gguf/reader.rs:132-430):
// magic "GGUF", version 3 only, u64 counts, typed metadata (value.rs:33-57),
// tensor infos with dims in PyTorch order, `general.alignment` (default 32,
// gguf/mod.rs:85-89), tensor offsets relative to the aligned data region, each
// a multiple of the alignment and inside the file. Dtype tags accepted are the
// reference's (F32, F16, BF16, Q4_K, Q5_K, Q6_K; tensor.rs:85) plus this
// library's documented Q4_0 (2) and Q8_0 (8) extension. Malformed input is an
// error (VKB_ERROR_MODEL_LOAD), never a crash.
#include "common.cuh"
#include "gguf.cuh"
#include <fstream>

namespace vkb {

static int64_t tag_payload(uint32_t tag, uint64_t n) {
    switch (tag) {
        case 0: return (int64_t)n * 4;
        case 1: case 30: return (int64_t)n * 2;
        case 2: return n % 32 ? -1 : (int64_t)(n / 32) * 18;
        case 8: return n % 32 ? -1 : (int64_t)(n / 32) * 34;
        case 12: return n % 256 ? -1 : (int64_t)(n / 256) * 144;
        case 13: return n % 256 ? -1 : (int64_t)(n / 256) * 176;
        case 14: return n % 256 ? -1 : (int64_t)(n / 256) * 210;
        default: return -2;
    }
}

struct Cursor {
    const uint8_t* p;
    size_t n, i = 0;
    void need(size_t k, const char* what) {
        if (i + k > n || i + k < i) fail(VKB_ERROR_MODEL_LOAD, std::string("gguf: truncated ") + what);
    }
    template <class T> T get(const char* what) {
        need(sizeof(T), what);
        T v;
        memcpy(&v, p + i, sizeof(T));
        i += sizeof(T);
        return v;
    }
    std::string str(const char* what) {
        uint64_t len = get<uint64_t>(what);
        if (len > n - i) fail(VKB_ERROR_MODEL_LOAD, std::string("gguf: truncated ") + what);
        need((size_t)len, what);
        std::string s((const char*)p + i, (size_t)len);
        i += (size_t)len;
        return s;
    }
};

static GgufValue read_value(Cursor& c, uint32_t type, int depth) {
    GgufValue v;
    v.type = type;
    switch (type) {
        case 0: v.u = c.get<uint8_t>("u8"); break;
        case 1: v.i = c.get<int8_t>("i8"); break;
        case 2: v.u = c.get<uint16_t>("u16"); break;
        case 3: v.i = c.get<int16_t>("i16"); break;
        case 4: v.u = c.get<uint32_t>("u32"); break;
        case 5: v.i = c.get<int32_t>("i32"); break;
        case 6: v.f = c.get<float>("f32"); break;
        case 7:
            v.u = c.get<uint8_t>("bool");
            if (v.u > 1) fail(VKB_ERROR_MODEL_LOAD, "gguf: bool value " + std::to_string(v.u) + " (InvalidBool)");
            break;
        case 8: v.s = c.str("string"); break;
        case 9: {
            if (depth >= 64) fail(VKB_ERROR_MODEL_LOAD, "gguf: nested arrays too deep (ArrayTooDeep)");
            uint32_t et = c.get<uint32_t>("array type");
            uint64_t cnt = c.get<uint64_t>("array count");
            if (cnt > c.n - c.i) fail(VKB_ERROR_MODEL_LOAD, "gguf: array length exceeds file size (Truncated)");
            v.arr.reserve((size_t)std::min<uint64_t>(cnt, 1 << 16));
            for (uint64_t k = 0; k < cnt; ++k) v.arr.push_back(read_value(c, et, depth + 1));
            break;
        }
        case 10: v.u = c.get<uint64_t>("u64"); break;
        case 11: v.i = c.get<int64_t>("i64"); break;
        case 12: v.f = c.get<double>("f64"); break;
        default: fail(VKB_ERROR_MODEL_LOAD, "gguf: unsupported metadata value type " + std::to_string(type));
    }
    return v;
}

GgufFile* gguf_open(const std::string& path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) fail(VKB_ERROR_IO, "gguf: cannot open " + path);
    std::streamsize sz = f.tellg();
    f.seekg(0);
    auto* g = new GgufFile();
    try {
        g->bytes.resize((size_t)sz);
        if (sz && !f.read(reinterpret_cast<char*>(g->bytes.data()), sz)) fail(VKB_ERROR_IO, "gguf: read failed");
        gguf_parse(*g);
    } catch (...) {
        delete g;
        throw;
    }
    return g;
}

// Errors carry the reference's GgufError variant name (gguf/mod.rs) in the
// message, in the order parse_all (reader.rs:333-428) checks them.
void gguf_parse(GgufFile& g) {
    Cursor c{g.bytes.data(), g.bytes.size()};
    c.need(4, "magic (Truncated)");
    if (memcmp(c.p, "GGUF", 4) != 0) fail(VKB_ERROR_MODEL_LOAD, "gguf: bad magic (BadMagic)");
    c.i = 4;
    uint32_t ver = c.get<uint32_t>("version (Truncated)");
    if (ver != 3) fail(VKB_ERROR_MODEL_LOAD, "gguf: unsupported version " + std::to_string(ver) + " (UnsupportedVersion)");
    uint64_t n_t = c.get<uint64_t>("tensor count (Truncated)");
    uint64_t n_kv = c.get<uint64_t>("metadata count (Truncated)");
    // every entry takes at least one byte: larger counts are malformed, caught
    // before any loop or allocation
    if (n_t > c.n - c.i || n_kv > c.n - c.i)
        fail(VKB_ERROR_MODEL_LOAD, "gguf: declared count exceeds file size (Truncated)");
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key = c.str("metadata key (Truncated)");
        uint32_t t = c.get<uint32_t>("metadata type (Truncated)");
        g.meta[key] = read_value(c, t, 0);
    }
    uint64_t align = 32;
    auto it = g.meta.find("general.alignment");
    if (it != g.meta.end()) {
        const uint32_t at = it->second.type;
        if (at != 0 && at != 2 && at != 4 && at != 10)
            fail(VKB_ERROR_MODEL_LOAD, "gguf: general.alignment is not an integer (OffsetOutOfBounds)");
        align = it->second.u;
        if (align == 0 || (align & (align - 1)))
            fail(VKB_ERROR_MODEL_LOAD, "gguf: alignment " + std::to_string(align) +
                                           " is not a power of two (InvalidAlignment)");
    }
    for (uint64_t k = 0; k < n_t; ++k) {
        GgufTensor t;
        t.name = c.str("tensor name (Truncated)");
        uint32_t nd = c.get<uint32_t>("tensor n_dims (Truncated)");
        if (nd > 8) fail(VKB_ERROR_MODEL_LOAD, "gguf: " + std::to_string(nd) + " dimensions for " + t.name +
                                                   " (TooManyDimensions)");
        uint64_t elems = 1;
        bool overflow = false;
        for (uint32_t d = 0; d < nd; ++d) {
            uint64_t dim = c.get<uint64_t>("tensor dim (Truncated)");
            if (dim && elems > UINT64_MAX / dim) overflow = true;
            elems *= dim;
            t.dims.push_back((int64_t)dim);
        }
        t.tag = c.get<uint32_t>("tensor dtype (Truncated)");
        if (tag_payload(t.tag, 0) == -2)
            fail(VKB_ERROR_MODEL_LOAD, "gguf: unsupported dtype " + std::to_string(t.tag) + " for " + t.name +
                                           " (UnsupportedDtype)");
        t.offset = c.get<uint64_t>("tensor offset (Truncated)");
        if (g.index.count(t.name)) fail(VKB_ERROR_MODEL_LOAD, "gguf: duplicate tensor " + t.name + " (DuplicateTensor)");
        if (overflow) fail(VKB_ERROR_MODEL_LOAD, "gguf: element count of " + t.name + " overflows (Overflow)");
        t.n_elem = elems;
        g.index[t.name] = g.tensors.size();
        g.tensors.push_back(t);
    }
    uint64_t base = (c.i + align - 1) / align * align;
    g.data_base = base;
    if (!g.tensors.empty() && base > g.bytes.size())
        fail(VKB_ERROR_MODEL_LOAD, "gguf: tensor-data region starts past end of file (OffsetOutOfBounds)");
    for (auto& t : g.tensors) {
        if (t.offset % align)
            fail(VKB_ERROR_MODEL_LOAD, "gguf: tensor " + t.name + " offset " + std::to_string(t.offset) +
                                           " is not a multiple of " + std::to_string(align) + " (UnalignedTensorOffset)");
        int64_t ps = tag_payload(t.tag, t.n_elem);
        if (ps < 0)
            fail(VKB_ERROR_MODEL_LOAD, "gguf: " + t.name + " is not a whole number of blocks (BlockSizeMisaligned)");
        t.nbytes = (uint64_t)ps;
        if (base + t.offset < base || base + t.offset + t.nbytes < base + t.offset)
            fail(VKB_ERROR_MODEL_LOAD, "gguf: offset of " + t.name + " overflows (Overflow)");
        if (base + t.offset + t.nbytes > g.bytes.size())
            fail(VKB_ERROR_MODEL_LOAD, "gguf: tensor " + t.name + " runs past the end of the file (OffsetOutOfBounds)");
    }
}

const GgufTensor& GgufFile::tensor(const std::string& name, const std::vector<int64_t>& dims) const {
    auto it = index.find(name);
    if (it == index.end()) fail(VKB_ERROR_MODEL_LOAD, "gguf: missing tensor " + name + " (MissingTensor)");
    const GgufTensor& t = tensors[it->second];
    if (!dims.empty() && t.dims != dims) {
        std::string s;
        for (auto d : t.dims) s += std::to_string(d) + ",";
        fail(VKB_ERROR_MODEL_LOAD, "gguf: tensor " + name + " has shape [" + s + "], unexpected");
    }
    return t;
}

uint32_t GgufFile::u32(const std::string& key) const {
    auto it = meta.find(key);
    if (it == meta.end()) fail(VKB_ERROR_MODEL_LOAD, "gguf: missing metadata " + key);
    if (it->second.type != 4 && it->second.type != 5 && it->second.type != 10 && it->second.type != 2 &&
        it->second.type != 0)
        fail(VKB_ERROR_MODEL_LOAD, "gguf: metadata " + key + " is not an integer");
    return (uint32_t)(it->second.type == 5 ? (uint64_t)it->second.i : it->second.u);
}

std::vector<float> GgufFile::f32(const std::string& name, const std::vector<int64_t>& dims) const {
    const GgufTensor& t = tensor(name, dims);
    const uint8_t* p = data(t);
    std::vector<float> out(t.n_elem);
    if (t.tag == 0) {
        memcpy(out.data(), p, t.n_elem * 4);
    } else if (t.tag == 1) {
        for (uint64_t i = 0; i < t.n_elem; ++i) {
            uint16_t h;
            memcpy(&h, p + 2 * i, 2);
            uint32_t sign = (h >> 15) & 1, ex = (h >> 10) & 0x1f, mant = h & 0x3ff;
            float v;
            if (ex == 0) v = std::ldexp((float)mant, -24);
            else if (ex == 31) v = mant ? NAN : INFINITY;
            else v = std::ldexp(1.0f + (float)mant / 1024.0f, (int)ex - 15);
            out[i] = sign ? -v : v;
        }
    } else if (t.tag == 30) {
        for (uint64_t i = 0; i < t.n_elem; ++i) {
            uint32_t b = (uint32_t)(p[2 * i] | (p[2 * i + 1] << 8)) << 16;
            memcpy(&out[i], &b, 4);
        }
    } else {
        fail(VKB_ERROR_MODEL_LOAD, "gguf: tensor " + name + " must be F32/F16/BF16 here");
    }
    return out;
}

}  // namespace vkb

extern "C" vkb_status vkb_gguf_inspect(const void* bytes, size_t len, int64_t* n_tensors, int64_t* n_metadata) {
    return vkb::guard([&] {
        if (!bytes && len) vkb::fail(VKB_ERROR_INVALID_ARGUMENT, "gguf_inspect: null bytes");
        vkb::GgufFile g;
        g.bytes.assign((const uint8_t*)bytes, (const uint8_t*)bytes + len);
        vkb::gguf_parse(g);
        if (n_tensors) *n_tensors = (int64_t)g.tensors.size();
        if (n_metadata) *n_metadata = (int64_t)g.meta.size();
    });
}
