// ssm_format.h — the lite-ssm .ssm container (include/lite_ssm/ssm_format.hpp:22-128,
// docs/ssm_format.md), parsed and planned in host C++.
//
// The on-disk format is fixed by the reference, so the structs keep its exact field
// order and sizes (96-byte header, 32-byte index prefix, 8-byte-aligned entries,
// 64-byte-aligned payloads, INT4_B32 = packed nibbles then fp16 scales).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace lssm {

constexpr uint32_t SSM_VERSION = 1;
constexpr size_t SSM_ALIGN = 64;
enum : uint32_t { DT_F16 = 0, DT_BF16 = 1, DT_F32 = 2, DT_I8 = 3, DT_U8 = 4, DT_I32 = 5, DT_INT4_B32 = 6 };

#pragma pack(push, 1)
struct SsmHeader {
    char magic[4];
    uint32_t version, header_size, n_tensors;
    uint64_t index_offset, data_offset;
    uint32_t d_model, n_layer, d_state, d_conv, expand, vocab_size, n_heads, d_head, chunk_size, default_dtype;
    uint32_t n_groups, norm_before_gate;
    uint32_t reserved[4];
};
struct SsmIndexPrefix {
    uint32_t name_len, rank, dtype, pad0;
    uint64_t offset, nbytes;
};
#pragma pack(pop)
static_assert(sizeof(SsmHeader) == 96, "header must be 96 bytes");
static_assert(sizeof(SsmIndexPrefix) == 32, "index prefix must be 32 bytes");

struct TensorRec {
    std::string name;
    uint32_t dtype = 0, rank = 0;
    uint64_t shape[4] = {0, 0, 0, 0};
    uint64_t offset = 0, nbytes = 0;
    uint64_t numel() const {
        uint64_t n = 1;
        for (uint32_t i = 0; i < rank; ++i) n *= shape[i];
        return n;
    }
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) & ~(a - 1); }

inline size_t dtype_itemsize(uint32_t dt) {
    switch (dt) {
        case DT_F16: case DT_BF16: return 2;
        case DT_F32: case DT_I32: return 4;
        case DT_I8: case DT_U8: return 1;
        default: return 0;
    }
}

inline size_t packed_nbytes(uint32_t dt, uint64_t numel) {
    if (dt == DT_INT4_B32) return numel / 2 + (numel / 32) * 2;
    return numel * dtype_itemsize(dt);
}

struct SsmImage {
    SsmHeader hdr{};
    std::vector<TensorRec> order;                      // index order
    std::unordered_map<std::string, size_t> by_name;  // -> position in order
    const TensorRec* find(const std::string& n) const {
        auto it = by_name.find(n);
        return it == by_name.end() ? nullptr : &order[it->second];
    }
};

// Parse header + index of an .ssm image of `size` bytes. Returns "" on success or the
// reference loader's error message (src/core/ssm_loader.cpp:56-137).
std::string ssm_parse(const uint8_t* base, size_t size, SsmImage* out);

// Plan a file for the given header fields and tensor list (name, dtype, shape):
// fills offsets / nbytes and returns header + index bytes (tools/ssm_format.py:316-340).
std::vector<uint8_t> ssm_plan(const SsmHeader& hp, std::vector<TensorRec>& tensors, uint64_t* data_offset);

}  // namespace lssm
