// q38_gguf_file.cpp - GGUF reader for the device model loader (host code).
#include "q38_gguf_file.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace q38 {

uint32_t ggml_block_elements(uint32_t type)
{
    switch (type) {
    case 0: case 1: case 30: return 1;             // F32, F16, BF16
    case 2: case 3: case 6: case 7: case 8: case 20: return 32;  // Q4_0 Q4_1 Q5_0 Q5_1 Q8_0 IQ4_NL
    case 10: case 11: case 12: case 13: case 14:   // Q2_K .. Q6_K
    case 16: case 17: case 18: case 19: case 21: case 22: case 23: case 29:
        return 256;
    default: return 0;
    }
}

uint32_t ggml_block_bytes(uint32_t type)
{
    switch (type) {
    case 0: return 4;
    case 1: case 30: return 2;
    case 2: return 18;
    case 3: return 20;
    case 6: return 22;
    case 7: return 24;
    case 8: return 34;
    case 20: return 18;
    case 10: return 84;
    case 11: return 110;
    case 12: return 144;
    case 13: return 176;
    case 14: return 210;
    case 16: return 66;
    case 17: return 74;
    case 18: return 98;
    case 19: return 50;
    case 21: return 110;
    case 22: return 82;
    case 23: return 136;
    case 29: return 56;
    default: return 0;
    }
}

namespace {

// Bounds-checked little-endian cursor over the mapping.
struct Cursor {
    const uint8_t *at, *end;
    bool failed = false;

    bool take(uint64_t n, const uint8_t **p)
    {
        if (failed || n > static_cast<uint64_t>(end - at)) {
            failed = true;
            return false;
        }
        *p = at;
        at += n;
        return true;
    }
    uint64_t uint(int bytes)
    {
        const uint8_t *p = nullptr;
        if (!take(static_cast<uint64_t>(bytes), &p)) return 0;
        uint64_t v = 0;
        for (int i = bytes - 1; i >= 0; --i) v = v << 8 | p[i];
        return v;
    }
    bool string(std::string *out, const uint8_t **raw = nullptr, uint64_t *raw_len = nullptr)
    {
        const uint64_t n = uint(8);
        const uint8_t *p = nullptr;
        if (!take(n, &p)) return false;
        if (out) out->assign(reinterpret_cast<const char *>(p), n);
        if (raw) *raw = p;
        if (raw_len) *raw_len = n;
        return true;
    }
};

uint64_t scalar_size(uint32_t type)
{
    switch (type) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
    }
}

bool skip_values(Cursor &c, uint32_t type, uint64_t count)
{
    if (type == 8) {
        for (uint64_t i = 0; i < count && !c.failed; ++i) c.string(nullptr);
        return !c.failed;
    }
    const uint64_t size = scalar_size(type);
    if (!size || count > UINT64_MAX / size) return false;
    const uint8_t *p = nullptr;
    return c.take(size * count, &p);
}

}  // namespace

GGUFFile::~GGUFFile() { close(); }

void GGUFFile::close()
{
    if (mapping_) munmap(const_cast<uint8_t *>(mapping_), mapping_size_);
    if (fd_ >= 0) ::close(fd_);
    mapping_ = nullptr;
    mapping_size_ = 0;
    fd_ = -1;
    meta_.clear();
    tensors_.clear();
}

bool GGUFFile::open(const char *path)
{
    close();
    auto fail = [&](const std::string &why) {
        error_ = why;
        close();
        return false;
    };
    fd_ = ::open(path, O_RDONLY);
    if (fd_ < 0) return fail(std::string("cannot open ") + path);
    struct stat st;
    if (fstat(fd_, &st) != 0 || st.st_size < 24) return fail("file too small to hold a GGUF header");
    mapping_size_ = static_cast<uint64_t>(st.st_size);
    void *m = mmap(nullptr, mapping_size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) {
        mapping_ = nullptr;
        return fail("mmap failed");
    }
    mapping_ = static_cast<const uint8_t *>(m);

    Cursor c{mapping_, mapping_ + mapping_size_};
    const uint64_t magic = c.uint(4), version = c.uint(4);
    const uint64_t tensor_count = c.uint(8), meta_count = c.uint(8);
    if (magic != 0x46554747u || version < 2 || version > 3 || tensor_count == 0 ||
        tensor_count > mapping_size_ || meta_count > mapping_size_)
        return fail("unsupported or corrupt GGUF header");

    meta_.resize(meta_count);
    for (auto &m : meta_) {
        if (!c.string(&m.key)) return fail("malformed GGUF metadata");
        m.type = static_cast<uint32_t>(c.uint(4));
        if (c.failed || m.type > 12) return fail("malformed GGUF metadata");
        if (m.type == 8) {
            if (!c.string(nullptr, &m.data, &m.data_size)) return fail("malformed GGUF metadata");
            m.count = 1;
        } else if (m.type == 9) {
            m.array_type = static_cast<uint32_t>(c.uint(4));
            m.count = c.uint(8);
            m.data = c.at;
            if (c.failed || m.array_type == 9 || !skip_values(c, m.array_type, m.count))
                return fail("malformed GGUF metadata");
            m.data_size = static_cast<uint64_t>(c.at - m.data);
        } else {
            const uint64_t size = scalar_size(m.type);
            if (!size || !c.take(size, &m.data)) return fail("malformed GGUF metadata");
            m.data_size = size;
            m.count = 1;
        }
    }

    tensors_.resize(tensor_count);
    for (auto &t : tensors_) {
        if (!c.string(&t.name)) return fail("malformed GGUF tensor table");
        t.n_dims = static_cast<uint32_t>(c.uint(4));
        if (c.failed || t.n_dims == 0 || t.n_dims > 8) return fail("malformed GGUF tensor table");
        uint64_t elements = 1;
        for (uint32_t d = 0; d < t.n_dims; ++d) {
            t.shape[d] = c.uint(8);
            if (!t.shape[d] || elements > UINT64_MAX / t.shape[d]) return fail("malformed GGUF tensor shape");
            elements *= t.shape[d];
        }
        t.type = static_cast<uint32_t>(c.uint(4));
        t.offset = c.uint(8);
        const uint32_t be = ggml_block_elements(t.type), bb = ggml_block_bytes(t.type);
        if (c.failed || !be || !bb || t.shape[0] % be || elements % be || elements / be > UINT64_MAX / bb)
            return fail("GGUF tensor " + t.name + " has an unsupported type or shape");
        t.nbytes = elements / be * bb;
    }

    alignment_ = 32;
    uint32_t declared = 0;
    if (meta_u32("general.alignment", &declared)) {
        if (!declared || (declared & (declared - 1))) return fail("invalid GGUF alignment");
        alignment_ = declared;
    }
    const uint64_t descriptor_end = static_cast<uint64_t>(c.at - mapping_);
    const uint64_t data_offset = (descriptor_end + alignment_ - 1) & ~static_cast<uint64_t>(alignment_ - 1);
    if (data_offset > mapping_size_) return fail("GGUF tensor data begins past end of file");
    for (auto &t : tensors_) {
        if (t.offset > mapping_size_ - data_offset || t.nbytes > mapping_size_ - data_offset - t.offset)
            return fail("tensor outside GGUF file: " + t.name);
        t.data = mapping_ + data_offset + t.offset;
    }
    return true;
}

const GGUFMeta *GGUFFile::find_meta(const char *key) const
{
    for (const auto &m : meta_)
        if (m.key == key) return &m;
    return nullptr;
}

const GGUFTensorInfo *GGUFFile::find_tensor(const char *name) const
{
    for (const auto &t : tensors_)
        if (t.name == name) return &t;
    return nullptr;
}

bool GGUFFile::meta_u32(const char *key, uint32_t *value) const
{
    const GGUFMeta *m = find_meta(key);
    if (!m || m->type != 4 || m->data_size != 4) return false;
    *value = static_cast<uint32_t>(m->data[0]) | static_cast<uint32_t>(m->data[1]) << 8 |
             static_cast<uint32_t>(m->data[2]) << 16 | static_cast<uint32_t>(m->data[3]) << 24;
    return true;
}

bool GGUFFile::meta_string_is(const char *key, const char *expected) const
{
    const GGUFMeta *m = find_meta(key);
    const size_t n = std::strlen(expected);
    return m && m->type == 8 && m->data_size == n && std::memcmp(m->data, expected, n) == 0;
}

}  // namespace q38
