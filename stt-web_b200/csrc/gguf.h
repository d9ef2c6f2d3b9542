// GGUF v2/v3 reader over one or more in-memory shards.
//
// Follows GgufReader (crates/stt-wasm/src/gguf.rs:193-311) and ShardedCursor (gguf.rs:321-397):
// magic "GGUF", version 2 or 3, metadata skipped value by value (types 0-12, arrays nested),
// tensor infos (name, dims in GGUF order, dtype, offset), data section at the header end rounded
// up to 32 bytes, tensor byte size from the dtype.  Duplicate names keep the last entry (the
// reference inserts into a HashMap).
#pragma once

#include <string>
#include <unordered_map>
#include <vector>

#include "common.h"

namespace stt {

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> dims;  // GGUF order (innermost first)
    uint32_t dtype = 0;
    uint64_t offset = 0;         // relative to the data section
    uint64_t numel = 0;
    uint64_t nbytes = 0;
    // PyTorch-order shape (gguf.rs:83-85 reverse_gguf_dims).
    std::vector<uint64_t> shape() const { return std::vector<uint64_t>(dims.rbegin(), dims.rend()); }
};

class GgufFile {
public:
    // Parses the header; returns STT_OK or STT_E_FORMAT / STT_E_INVALID_ARG with the last error set.
    int open(const uint8_t* const* shards, const size_t* lens, int n_shards);

    const GgufTensor* find(const std::string& name) const;
    // Pointer to the tensor bytes when they lie inside one shard; otherwise the bytes are copied
    // into `scratch` and its data pointer is returned.  NULL (with the last error set) if the
    // tensor runs past the end of the input.
    const uint8_t* tensor_data(const GgufTensor& t, std::vector<uint8_t>& scratch) const;

    // Copies n bytes of the logical file (the shards back to back) from byte pos; false past the
    // end.  Safe to call from several threads at once.
    bool read_range(uint64_t pos, void* dst, uint64_t n) const { return read(pos, dst, n); }

    uint32_t version() const { return version_; }
    uint64_t tensor_count() const { return tensor_count_; }
    uint64_t data_offset() const { return data_offset_; }
    uint64_t total_bytes() const { return total_; }

private:
    bool read(uint64_t pos, void* dst, uint64_t n) const;
    std::vector<const uint8_t*> ptr_;
    std::vector<uint64_t> end_;  // cumulative end offsets
    uint64_t total_ = 0;
    uint32_t version_ = 0;
    uint64_t tensor_count_ = 0;
    uint64_t data_offset_ = 0;
    std::unordered_map<std::string, GgufTensor> tensors_;
};

// Byte size of `numel` elements of GGML type `dtype` (gguf.rs:146-155; Q4_0 rounds down to whole
// blocks like the reference).  Returns false for unsupported dtypes.
bool ggml_nbytes(uint32_t dtype, uint64_t numel, uint64_t* out);

}  // namespace stt
