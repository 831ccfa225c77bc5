// Reader of the Cactus .weights tensor file (graph_io.cpp:497-566 parse_header; writer
// python/src/tensor_io.py:163-321): 80-byte header (magic CACT, version, flags,
// alignment, ndim, 4 x u64 dims, u32 precision, u64 data_bytes, u64 scales_bytes,
// u32 group_size, u32 num_groups), fp16 scales [N, num_groups] at the aligned header end,
// data at the next aligned offset. Errors mirror the reference's messages.
#pragma once
#include <stdint.h>

#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace cb {
namespace eng {

enum Prec : int { kInt8 = 0, kFp16 = 1, kFp32 = 2, kInt4 = 3 };

struct HostTensor {
    std::vector<size_t> shape;
    int prec = kFp16;
    size_t group_size = 0, num_groups = 0;
    std::vector<uint8_t> data;     // raw data bytes
    std::vector<uint16_t> scales;  // fp16 bits [rows, num_groups]
    size_t rows() const { return shape.size() >= 2 ? shape[0] : 1; }
    size_t cols() const { return shape.empty() ? 0 : shape.back(); }
};

inline size_t align_to(size_t off, size_t a) { return a ? (off + a - 1) / a * a : off; }

inline HostTensor read_weights_file(const std::string& path) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("Cannot open weights file: " + path);
    std::fseek(f, 0, SEEK_END);
    const long size = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    std::vector<uint8_t> buf(size > 0 ? (size_t)size : 0);
    const size_t got = buf.empty() ? 0 : std::fread(buf.data(), 1, buf.size(), f);
    std::fclose(f);
    if (got != buf.size()) throw std::runtime_error("Short read: " + path);
    if (buf.size() < 80) throw std::runtime_error("File too small: insufficient data for header");
    auto u32 = [&](size_t o) { uint32_t v; std::memcpy(&v, buf.data() + o, 4); return v; };
    auto u64 = [&](size_t o) { uint64_t v; std::memcpy(&v, buf.data() + o, 8); return v; };
    if (u32(0) != 0x54434143u) throw std::runtime_error("Invalid tensor file: missing CACT magic number");
    uint32_t alignment = u32(12);
    if (alignment == 0) alignment = 1;
    const uint32_t ndim = u32(16);
    HostTensor t;
    for (uint32_t i = 0; i < 4; ++i) {
        const uint64_t d = u64(20 + 8 * i);
        if (i < ndim && d > 0) t.shape.push_back((size_t)d);
    }
    t.prec = (int)u32(52);
    const uint64_t data_bytes = u64(56), scales_bytes = u64(64);
    t.group_size = u32(72);
    t.num_groups = u32(76);
    const size_t hdr = align_to(80, alignment);
    size_t data_off = hdr;
    if (scales_bytes) data_off = align_to(hdr + scales_bytes, alignment);
    if (data_off + data_bytes > buf.size())
        throw std::runtime_error("File corrupted: data extends beyond file size (v2)");
    if (scales_bytes) {
        t.scales.resize(scales_bytes / 2);
        std::memcpy(t.scales.data(), buf.data() + hdr, scales_bytes);
    }
    t.data.assign(buf.begin() + data_off, buf.begin() + data_off + data_bytes);
    return t;
}

}  // namespace eng
}  // namespace cb
