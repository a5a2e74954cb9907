// q38_gguf_file.h - read-only GGUF v2/v3 reader for the device model loader.
//
// Accepts the files the upstream reader accepts (src/io/qwen38_gguf.c:263-413):
// magic "GGUF", version 2 or 3, metadata of the 13 GGUF value types (arrays of
// arrays refused), tensors of 1..8 dimensions whose first dimension is a whole
// number of blocks, `general.alignment` a power of two (default 32), and every
// tensor's bytes inside the file.  The file is memory-mapped; tensor data
// pointers point into the mapping.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace q38 {

struct GGUFMeta {
    std::string key;
    uint32_t type = 0;        // GGUF value type (4 = uint32, 8 = string, 9 = array, ...)
    uint32_t array_type = 0;
    uint64_t count = 0;
    const uint8_t *data = nullptr;
    uint64_t data_size = 0;
};

struct GGUFTensorInfo {
    std::string name;
    uint32_t n_dims = 0;
    uint64_t shape[8] = {0};
    uint32_t type = 0;
    uint64_t offset = 0;
    uint64_t nbytes = 0;
    const uint8_t *data = nullptr;
};

class GGUFFile {
public:
    GGUFFile() = default;
    ~GGUFFile();
    GGUFFile(const GGUFFile &) = delete;
    GGUFFile &operator=(const GGUFFile &) = delete;

    // Returns false (with a message in error()) on any malformed input.
    bool open(const char *path);
    void close();

    const GGUFMeta *find_meta(const char *key) const;
    const GGUFTensorInfo *find_tensor(const char *name) const;
    bool meta_u32(const char *key, uint32_t *value) const;
    bool meta_string_is(const char *key, const char *expected) const;
    const std::string &error() const { return error_; }
    bool is_open() const { return mapping_ != nullptr; }
    uint64_t tensor_count() const { return tensors_.size(); }

private:
    int fd_ = -1;
    const uint8_t *mapping_ = nullptr;
    uint64_t mapping_size_ = 0;
    uint32_t alignment_ = 32;
    std::vector<GGUFMeta> meta_;
    std::vector<GGUFTensorInfo> tensors_;
    std::string error_;
};

// Bytes and elements of one block of a ggml type (0 for unknown types).
uint32_t ggml_block_bytes(uint32_t type);
uint32_t ggml_block_elements(uint32_t type);

}  // namespace q38
