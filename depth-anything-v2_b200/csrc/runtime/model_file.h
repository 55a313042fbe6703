// Read-only, memory-mapped .dav2 model container. The layout and the
// validation rules follow the reference reader (src/model.cpp:27-320): a
// 64-byte header, 192-byte tensor records, an optional 128-byte derivation
// metadata block, 64-byte aligned float32 payloads, CRC-32 per tensor.
#pragma once

#include <array>
#include <cstdint>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

#include "depth_anything_v2.h"

namespace dav2 {

struct TensorView {
    const float* data = nullptr;
    std::array<std::uint64_t, 4> dims{};
    std::uint32_t rank = 0;
    std::uint64_t elements = 0;
    std::uint32_t crc32 = 0;
};

class ModelFile {
public:
    ModelFile(const std::string& path, dav2_encoder expected_encoder);
    ModelFile(const ModelFile&) = delete;
    ModelFile& operator=(const ModelFile&) = delete;
    ~ModelFile();

    const TensorView& tensor(std::string_view name) const;
    bool contains(std::string_view name) const { return tensors_.count(name) != 0; }
    const std::vector<std::string_view>& names() const { return names_; }
    float metric_max_depth() const { return metric_max_depth_; }
    // Verifies every tensor's CRC-32; a mismatch throws StatusError
    // (DAV2_STATUS_MODEL_FORMAT), as do all format violations of the
    // constructor; open/stat/mmap failures are DAV2_STATUS_MODEL_IO.
    void verify_crc() const;

private:
    void unmap() noexcept;
    int fd_ = -1;
    const unsigned char* view_ = nullptr;
    std::uint64_t size_ = 0;
    std::unordered_map<std::string_view, TensorView> tensors_;
    std::vector<std::string_view> names_;
    float metric_max_depth_ = 0.0f;
};

std::uint32_t crc32(const void* data, std::size_t bytes);

}  // namespace dav2
